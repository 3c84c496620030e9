"""The decode-step projection ``nb_linear`` (tcgen05; 256-row weight tiles by
default, 128-row tiles with or without a cluster split-K when forced).

Every projection of a decode step of the benchmarked models, a few ragged
shapes (N not a multiple of the 128-row tile, K not a multiple of 64, M
from 1 to 256), strided x / y, bias, fp16, and every tile path, against a float32 matmul of the same 16-bit inputs.  Tolerance:
the output is the fp32 sum rounded once to the 16-bit type, so it is within
one unit in the last place of the reference plus the fp32 summation-order
difference: |y - ref| <= 2^-7 |ref| + 2^-9 * max|ref| (bf16; a quarter of
that for fp16).  Results are deterministic (same bits on a second call).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from needle_b200 import ops
    return ops


def _ref(x, w, b):
    r = x.float() @ w.float().t()
    return r + b.float() if b is not None else r


def _check(y, ref, dt):
    rel = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -9
    tol = rel * ref.abs() + rel / 4 * ref.abs().max()
    err = (y.float() - ref).abs()
    bad = err > tol
    assert not bad.any(), (f"{int(bad.sum())} of {bad.numel()} elements off; max err "
                           f"{err.max().item():.4g} (max |ref| {ref.abs().max().item():.4g})")


SHAPES = [
    # (M, N, K): Llama-3-8B decode projections at config 3 (M = 256)
    (256, 6144, 4096),     # qkv
    (256, 4096, 4096),     # o_proj
    (256, 28672, 4096),    # gate_up
    (256, 4096, 14336),    # down
    (256, 128256, 4096),   # lm_head
    # TP=8 shards of the same
    (256, 768, 4096), (256, 4096, 512), (256, 3584, 4096), (256, 4096, 1792),
    # ragged
    (1, 256, 64), (7, 1152, 896), (33, 200, 136), (129, 1000, 520), (255, 384, 8),
    (64, 130, 4104),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_bf16(cuda, M, N, K):
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    y = ops.linear(x, w)
    assert ops.device_errors() == 0
    _check(y, _ref(x, w, None), torch.bfloat16)
    y2 = ops.linear(x, w)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("split", ["1", "2", "3", "4"])
@pytest.mark.parametrize("M,N,K", [(256, 6144, 4096), (100, 1000, 1000), (32, 256, 192),
                                   (200, 28672, 512)])
def test_linear_every_cluster_size(cuda, monkeypatch, split, M, N, K):
    """The 128-row tile paths, forced: no split with double-buffered
    accumulators ("1") and the cluster split-K with S = 2, 3, 4 (the partial
    sums meet in distributed shared memory); the default 256-row tiles are
    what the other tests run."""
    ops = _ops()
    monkeypatch.setenv("NB_LINEAR_SPLIT", split)
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    y = ops.linear(x, w)
    assert ops.device_errors() == 0
    _check(y, _ref(x, w, None), torch.bfloat16)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_linear_bias_strided_views(cuda, dt):
    """x and y as column slices of wider buffers (a fused projection's
    output, a peer-mapped partial buffer), bias added before the rounding."""
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(9)
    M, N, K = 77, 1152, 896
    xb = torch.randn(M, K + 64, device=cuda, generator=g).to(dt)
    x = xb[:, 32:32 + K]
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(dt)
    b = torch.randn(N, device=cuda, generator=g).to(dt)
    yb = torch.full((M, N + 40), 7.0, device=cuda, dtype=dt)
    y = yb[:, 8:8 + N]
    ops.linear(x, w, b, out=y)
    assert ops.device_errors() == 0
    _check(y, _ref(x, w, b), dt)
    assert (yb[:, :8] == 7).all() and (yb[:, 8 + N:] == 7).all()


def test_linear_is_used_by_the_model_layers(cuda):
    """dense() takes the kernel for a decode batch with many output features
    and torch beyond 256 rows or for few features; all agree with the
    reference."""
    from needle_b200 import ops
    from needle_b200.layers.linear import dense
    g = torch.Generator(device=cuda).manual_seed(3)
    for N in (512, 128256):
        w = (torch.randn(N, 256, device=cuda, generator=g) / 16).to(torch.bfloat16)
        for M in (256, 300):
            x = torch.randn(M, 256, device=cuda, generator=g).to(torch.bfloat16)
            assert ops.linear_preferred(x, w) == (M <= 256 and N == 128256)
            _check(dense(x, w), _ref(x, w, None), torch.bfloat16)


def test_linear_rejects_unsupported(cuda):
    ops = _ops()
    from needle_b200._lib import NeedleB200Error
    x = torch.randn(300, 64, device=cuda, dtype=torch.bfloat16)
    w = torch.randn(64, 64, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(NeedleB200Error):
        ops.linear(x, w)
    assert not ops.linear_supported(x, w)
