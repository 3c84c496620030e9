"""nb_paged_decode_noalloc: paged decode for callers that cannot allocate.

Some callers of this library cannot hand it a device workspace: a host that
binds the C ABI through a plain FFI and has no device allocator, a serving
loop that must not call cudaMalloc between launches, or a process whose
device memory is fixed at start-up.  nb_paged_decode_noalloc serves them by
keeping the split-K partials in a fixed array inside the library.  These
tests call it through the C ABI (ctypes, no torch wrapper) and check it
against the workspace-taking nb_paged_decode on the same inputs, twice in a
row with different inputs so that the shared array's leftover contents from
the first call cannot leak into the second.  The file is named to be
collected last, and it needs no state from other tests.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL_BF16 = 2e-2  # the bf16 attention tolerance used throughout the GPU tests


def _case(seed, dev, B=16, H=32, KV=8, D=128, N=2000, maxb=100):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(0, maxb * 16 - 1, (B,), generator=g).to(torch.int32)
    ctx[0] = 0
    ctx[1] = maxb * 16 - 1
    bt = torch.randperm(N, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    cache = torch.randn(2, N, KV, 16, D, generator=g).to(torch.bfloat16)
    return q.to(dev), cache.to(dev), bt.to(dev), ctx.to(dev)


def _call_noalloc(q, cache, bt, ctx, scale, pps, out):
    from needle_b200 import _lib as L
    B, H, D = q.shape
    _, N, KV, BS, _ = cache.shape
    return L.lib().nb_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), cache.data_ptr(), N, KV, BS, D, H,
        bt.data_ptr(), bt.stride(0), bt.shape[1], ctx.data_ptr(), B, scale, out.data_ptr(),
        out.stride(0), out.stride(1), pps, L.NB_DTYPE_BF16,
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda):
    from needle_b200 import _lib as L
    from needle_b200 import ops
    pps = 8  # 13 splits per long sequence: the merge reads the fixed scratch
    for seed in (1, 2):
        q, cache, bt, ctx = _case(seed, cuda)
        B, H, D = q.shape
        scale = 1.0 / math.sqrt(D)
        plan = ops.DecodePlan(B, H, cache.shape[2], D, bt.shape[1], 16, cuda, pages_per_split=pps)
        ref = ops.paged_decode(q, cache, bt, ctx, scale, plan=plan)
        out = torch.full_like(q, float("nan"))
        L.check(_call_noalloc(q, cache, bt, ctx, scale, pps, out))
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= ATOL_BF16, (seed, err)
    assert L.device_errors() == 0


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch(cuda):
    from needle_b200 import _lib as L
    q, cache, bt, ctx = _case(3, cuda, B=2, N=64, maxb=8)
    out = torch.empty_like(q)
    lib = L.lib()
    # claim a batch whose partials need far more than the fixed scratch;
    # the check happens on the host before anything is launched
    rc = lib.nb_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), cache.data_ptr(), 64, 8, 16, 128, 32,
        bt.data_ptr(), 100000, 100000, ctx.data_ptr(), 4096, 0.1, out.data_ptr(),
        out.stride(0), out.stride(1), 1, L.NB_DTYPE_BF16, torch.cuda.current_stream().cuda_stream)
    assert rc == L.NB_ERR_INVALID_ARG
    assert "scratch" in lib.nb_last_error().decode()
