"""Parity of the CUDA kernels with the CPU oracle (and through it, needle).

Tolerances are the ones the task fixes for attention outputs: 2e-2 max-abs
in bf16, 1e-4 in fp32.  KV-cache writes and RoPE must be bit-identical.
RMSNorm may differ from the reference by one unit in the last place (the
fp32 sum of squares runs in a different order); the test bounds it so.
"""
import math

import numpy as np
import pytest
import torch

from oracle import needle_oracle as no
from tests.golden import cases as C
from tests.golden.fixtures import load

pytestmark = pytest.mark.gpu

ATOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}


def _ops():
    from needle_b200 import ops
    return ops


def _bits_equal(a, b):
    a, b = a.cpu(), b.cpu()
    if a.dtype in (torch.bfloat16, torch.float16):
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    return torch.equal(a.view(torch.int32), b.view(torch.int32))


def _maxdiff(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


# ---------------------------------------------------------------------------
# store_kvcache
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("kv,D", C.KV_WRITE_SHAPES)
def test_store_kvcache_bit_exact(cuda, dt, kv, D):
    ops = _ops()
    x = C.kv_write_inputs(dt, kv, D)
    ref = x["cache"].clone()
    no.write_kv(x["k"], x["v"], ref, x["block_table"], x["cu_seqlens"], x["context_lens"])
    cache = x["cache"].to(cuda)
    ops.store_kvcache(x["k"].to(cuda), x["v"].to(cuda), cache, x["block_table"].to(cuda),
                      x["context_lens"].to(cuda), cu_seqlens=x["cu_seqlens"].to(cuda))
    assert ops.device_errors() == 0
    assert _bits_equal(cache, ref)


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
def test_store_kvcache_clamp_last_token_wins(cuda, dt):
    ops = _ops()
    x = C.kv_write_clamp_inputs(dt)
    ref = x["cache"].clone()
    no.write_kv(x["k"], x["v"], ref, x["block_table"], x["cu_seqlens"], x["context_lens"])
    cache = x["cache"].to(cuda)
    ops.store_kvcache(x["k"].to(cuda), x["v"].to(cuda), cache, x["block_table"].to(cuda),
                      x["context_lens"].to(cuda), cu_seqlens=x["cu_seqlens"].to(cuda))
    assert _bits_equal(cache, ref)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32, torch.float16])
def test_store_kvcache_decode_form(cuda, dt):
    ops = _ops()
    g = torch.Generator().manual_seed(11)
    B, kv, D, N = 37, 8, 128, 300
    cache = torch.randn(2, N, kv, 16, D, generator=g).to(dt)
    ctx = torch.randint(0, 16 * 8 - 1, (B,), generator=g).to(torch.int32)
    bt = torch.randperm(N, generator=g)[: B * 8].view(B, 8).to(torch.int32)
    k = torch.randn(B, kv, D, generator=g).to(dt)
    v = torch.randn(B, kv, D, generator=g).to(dt)
    ref = cache.clone()
    no.decode_write_kv(k, v, ref, bt, ctx)
    c = cache.to(cuda)
    ops.store_kvcache(k.to(cuda), v.to(cuda), c, bt.to(cuda), ctx.to(cuda))
    assert _bits_equal(c, ref)


def test_store_kvcache_strided_rows(cuda):
    """k/v as column slices of a fused [T, (Hq + 2 Hkv) * D] projection."""
    ops = _ops()
    g = torch.Generator().manual_seed(12)
    T, hq, kv, D, N = 50, 8, 2, 64, 20
    qkv = torch.randn(T, (hq + 2 * kv) * D, generator=g).to(torch.bfloat16)
    k = qkv[:, hq * D:(hq + kv) * D].view(T, kv, D)
    v = qkv[:, (hq + kv) * D:].view(T, kv, D)
    cu = torch.tensor([0, 20, 50], dtype=torch.int32)
    ctx = torch.tensor([3, 0], dtype=torch.int32)
    bt = torch.tensor([[5, 6, 7, 8], [9, 10, 11, 12]], dtype=torch.int32)
    ref = torch.zeros(2, N, kv, 16, D, dtype=torch.bfloat16)
    no.write_kv(k, v, ref, bt, cu, ctx)
    c = torch.zeros_like(ref, device=cuda)
    qkv_d = qkv.to(cuda)
    ops.store_kvcache(qkv_d[:, hq * D:(hq + kv) * D].view(T, kv, D),
                      qkv_d[:, (hq + kv) * D:].view(T, kv, D), c, bt.to(cuda), ctx.to(cuda),
                      cu_seqlens=cu.to(cuda))
    assert _bits_equal(c, ref)


def test_store_kvcache_bad_block_id_is_flagged_not_written(cuda):
    ops = _ops()
    kv, D, N = 2, 64, 8
    cache = torch.zeros(2, N, kv, 16, D, dtype=torch.bfloat16, device=cuda)
    k = torch.ones(2, kv, D, dtype=torch.bfloat16, device=cuda)
    bt = torch.tensor([[N + 5], [1]], dtype=torch.int32, device=cuda)   # first entry out of the pool
    ctx = torch.tensor([0, 0], dtype=torch.int32, device=cuda)
    ops.store_kvcache(k, k, cache, bt, ctx)
    assert ops.device_errors() & 1
    assert cache[:, 1].abs().sum().item() > 0            # the valid sequence was written
    assert cache[:, [0, 2, 3, 4, 5, 6, 7]].abs().sum().item() == 0
    assert ops.device_errors() == 0                        # reading cleared the word


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------

GOLD_ROPE = load("rope")


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("H,kv,D,base", C.ROPE_SHAPES)
def test_rope_bit_exact_vs_needle(cuda, dt, H, kv, D, base):
    ops = _ops()
    x = C.rope_inputs(dt, H, kv, D)
    gold = GOLD_ROPE[f"rope_{dt}_d{D}"]
    q, k = x["q"].to(cuda), x["k"].to(cuda)
    ops.rope_(q, k, gold["cos"].to(cuda), gold["sin"].to(cuda))
    assert _bits_equal(q, gold["q_out"])
    assert _bits_equal(k, gold["k_out"])


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [128, 20])  # 20: rows not 16-byte vectorisable (scalar path)
def test_rope_store_fused_matches_separate(cuda, dt, D):
    ops = _ops()
    g = torch.Generator().manual_seed(13)
    lens = [5, 33, 1, 16]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T, hq, kv, N = int(cu[-1]), 8, 2, 40
    ctx = torch.tensor([0, 7, 100, 15], dtype=torch.int32)
    bt = torch.randperm(N, generator=g)[:4 * 9].view(4, 9).to(torch.int32)
    q = torch.randn(T, hq, D, generator=g).to(dt)
    k = torch.randn(T, kv, D, generator=g).to(dt)
    v = torch.randn(T, kv, D, generator=g).to(dt)
    cos_t, sin_t = no.rope_cache(D, 4096, 5e5)
    pos = torch.cat([torch.arange(c, c + n) for c, n in zip(ctx.tolist(), lens)])
    cos, sin = cos_t.to(dt)[pos], sin_t.to(dt)[pos]
    qr, kr = no.apply_rope(q, k, cos, sin)
    ref = torch.zeros(2, N, kv, 16, D, dtype=dt)
    no.write_kv(kr, v, ref, bt, cu, ctx)
    qd, kd, c = q.to(cuda), k.to(cuda), torch.zeros_like(ref, device=cuda)
    ops.rope_store_kvcache(qd, kd, v.to(cuda), cos.to(cuda), sin.to(cuda), c, bt.to(cuda),
                           ctx.to(cuda), cu_seqlens=cu.to(cuda), write_k_back=True)
    assert _bits_equal(qd, qr)
    assert _bits_equal(kd, kr)
    assert _bits_equal(c, ref)


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------

GOLD_NORM = load("norm")


def _ulp_close(out, ref, dt):
    """Every element within one unit in the last place of the reference."""
    o, r = out.float().cpu(), ref.float().cpu()
    if dt == torch.float32:
        tol = r.abs() * 2.0 ** -23 * 2 + 1e-30
    else:
        tol = r.abs() * 2.0 ** -7 + 1e-30   # 1 bf16 ulp
    bad = (o - r).abs() > tol
    return int(bad.sum()), (o - r).abs().max().item()


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("hid,eps", C.NORM_SHAPES)
def test_rmsnorm_vs_needle(cuda, dt, hid, eps):
    ops = _ops()
    x = C.norm_inputs(dt, hid)
    gold = GOLD_NORM[f"norm_{dt}_h{hid}"]
    y = ops.rmsnorm(x["x"].to(cuda), x["weight"].to(cuda), eps)
    bad, md = _ulp_close(y, gold["y"], C.DTYPES[dt])
    assert bad == 0, (bad, md)
    y2, h = ops.fused_add_rmsnorm(x["x"].to(cuda), x["residual"].to(cuda),
                                  x["weight"].to(cuda), eps)
    assert _bits_equal(h, gold["h"])
    bad, md = _ulp_close(y2, gold["y_add"], C.DTYPES[dt])
    assert bad == 0, (bad, md)


def test_fused_add_rmsnorm_in_place(cuda):
    ops = _ops()
    g = torch.Generator().manual_seed(14)
    x = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    r = torch.randn(64, 4096, generator=g).to(torch.bfloat16)
    w = (torch.rand(4096, generator=g) + 0.5).to(torch.bfloat16)
    ref_y, ref_h = no.add_rms_norm(x, r, w, 1e-5)
    xd, rd = x.to(cuda), r.to(cuda)
    ops.fused_add_rmsnorm(xd, rd, w.to(cuda), 1e-5, out=xd, residual_out=rd)
    assert _bits_equal(rd, ref_h)
    assert _ulp_close(xd, ref_y, torch.bfloat16)[0] == 0


# ---------------------------------------------------------------------------
# Paged decode
# ---------------------------------------------------------------------------

GOLD_DEC = load("decode")


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("H,kv,D", C.DECODE_SHAPES)
@pytest.mark.parametrize("pps", [None, 1, 3])
def test_decode_vs_needle_golden(cuda, dt, H, kv, D, pps):
    """KV write + paged decode on needle's golden cases, with the default
    split plan and with forced 1- and 3-page splits (exercising the merge)."""
    ops = _ops()
    x = C.decode_inputs(dt, H, kv, D)
    gold = GOLD_DEC[f"decode_{dt}_h{H}_kv{kv}_d{D}"]
    cache = x["cache"].to(cuda)
    bt, ctx = x["block_table"].to(cuda), x["context_lens"].to(cuda)
    ops.store_kvcache(x["k"].to(cuda), x["v"].to(cuda), cache, bt, ctx)
    plan = None
    if pps is not None:
        plan = ops.DecodePlan(len(C.DECODE_CTX), H, kv, D, bt.shape[1], 16, cuda,
                              pages_per_split=pps)
    out = ops.paged_decode(x["q"].to(cuda), cache, bt, ctx, 1.0 / math.sqrt(D), plan=plan)
    assert ops.device_errors() == 0
    ref = gold["out"]
    assert _maxdiff(out, ref) <= ATOL[C.DTYPES[dt]], _maxdiff(out, ref)
    # the cache after the write is needle's, byte for byte
    cref = x["cache"].clone()
    no.decode_write_kv(x["k"], x["v"], cref, x["block_table"], x["context_lens"])
    assert _bits_equal(cache, cref)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,kv,D", [(32, 8, 128), (14, 2, 64), (64, 8, 128), (16, 1, 128),
                                    (8, 8, 128), (12, 4, 96), (48, 2, 128), (20, 1, 64)])
def test_decode_random_shapes(cuda, dt, H, kv, D):
    """Group sizes 4, 7, 8, 16, 24 and 20 (beyond one MMA tile: the tensor-core
    kernel takes 16 query heads per CTA in two column tiles, the last chunk
    partial), MHA and an odd head_dim."""
    ops = _ops()
    g = torch.Generator().manual_seed(15)
    B, N, maxb = 9, 400, 40
    ctx = torch.tensor([0, 1, 15, 16, 17, 255, 300, 639, 444], dtype=torch.int32)
    bt = torch.randperm(N, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(dt)
    cache = torch.randn(2, N, kv, 16, D, generator=g).to(dt)
    ref = no.decode_attention(q.float(), cache.float(), bt, ctx, 1 / math.sqrt(D), H, kv, D)
    for pps in (None, 2, 5):
        plan = None if pps is None else ops.DecodePlan(B, H, kv, D, maxb, 16, cuda, pps)
        out = ops.paged_decode(q.to(cuda), cache.to(cuda), bt.to(cuda), ctx.to(cuda),
                               1 / math.sqrt(D), plan=plan)
        assert _maxdiff(out, ref) <= ATOL[dt], (pps, _maxdiff(out, ref))


_DECODE_8HEAD_CHECK = r"""
import math, sys, torch
sys.path.insert(0, '.')
from needle_b200 import ops
from oracle import needle_oracle as no
g = torch.Generator().manual_seed(17)
for H, kv, D in ((48, 2, 128), (20, 1, 64), (32, 2, 128)):
    B, N, maxb = 5, 300, 30
    ctx = torch.tensor([0, 16, 17, 300, 470], dtype=torch.int32)
    bt = torch.randperm(N, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    cache = torch.randn(2, N, kv, 16, D, generator=g).to(torch.bfloat16)
    ref = no.decode_attention(q.float(), cache.float(), bt, ctx, 1 / math.sqrt(D), H, kv, D)
    dev = torch.device('cuda:0')
    out = ops.paged_decode(q.to(dev), cache.to(dev), bt.to(dev), ctx.to(dev), 1 / math.sqrt(D))
    err = (out.float().cpu() - ref.float()).abs().max().item()
    assert err <= 2e-2, (H, kv, D, err)
assert ops.device_errors() == 0
print('ok')
"""


def test_decode_large_groups_in_8_head_chunks(cuda):
    """Groups above 8 with the 16-head tiles switched off (NB_DECODE_N16=0, a
    fresh process): 8-head chunks, several CTAs per KV head."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NB_DECODE_N16="0")
    r = subprocess.run([sys.executable, "-c", _DECODE_8HEAD_CHECK], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_decode_table_width_limits_context(cuda):
    """A context longer than the block table reads only max_blocks pages,
    like the reference's block_table[i, :nb] slice."""
    ops = _ops()
    g = torch.Generator().manual_seed(16)
    B, H, kv, D, N, maxb = 3, 8, 2, 128, 64, 4
    ctx = torch.tensor([10, 63, 200], dtype=torch.int32)
    bt = torch.randperm(N, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    cache = torch.randn(2, N, kv, 16, D, generator=g).to(torch.bfloat16)
    ref = no.decode_attention(q.float(), cache.float(), bt, ctx, 1 / math.sqrt(D), H, kv, D)
    out = ops.paged_decode(q.to(cuda), cache.to(cuda), bt.to(cuda), ctx.to(cuda), 1 / math.sqrt(D))
    assert _maxdiff(out, ref) <= 2e-2


def test_decode_config2_full_size(cuda):
    """Config 2 at full size (B=64, 32/8 heads, D=128, ctx U[512,4096], 20000-block
    pool, bf16) against the oracle, which is needle's own _decode_pytorch math."""
    ops = _ops()
    from needle_b200.synth import decode_op_workload
    w = decode_op_workload(device=cuda)
    out = ops.paged_decode(w["q"], w["kv_cache"], w["block_table"], w["context_lens"], w["scale"])
    cache_cpu = w["kv_cache"].cpu()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = no.decode_attention(w["q"].cpu(), cache_cpu, w["block_table"].cpu(),
                              w["context_lens"].cpu(), w["scale"], 32, 8, 128)
    assert _maxdiff(out, ref) <= 2e-2
    # and against an fp32 evaluation of the same maths, much tighter
    sub = torch.arange(0, 64, 8)
    ref32 = no.decode_attention(w["q"].cpu()[sub].float(), cache_cpu.float(),
                                w["block_table"].cpu()[sub], w["context_lens"].cpu()[sub],
                                w["scale"], 32, 8, 128)
    assert _maxdiff(out[sub.to(cuda)], ref32) <= 1e-2


def test_decode_empty_batch(cuda):
    ops = _ops()
    q = torch.empty(0, 8, 128, dtype=torch.bfloat16, device=cuda)
    cache = torch.zeros(2, 4, 2, 16, 128, dtype=torch.bfloat16, device=cuda)
    bt = torch.zeros(0, 4, dtype=torch.int32, device=cuda)
    ctx = torch.zeros(0, dtype=torch.int32, device=cuda)
    out = ops.paged_decode(q, cache, bt, ctx, 0.1)
    assert out.shape == (0, 8, 128)


# ---------------------------------------------------------------------------
# Prefill
# ---------------------------------------------------------------------------

GOLD_PRE = load("prefill")


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("H,kv,D", C.PREFILL_SHAPES)
def test_prefill_vs_needle_golden(cuda, dt, H, kv, D):
    ops = _ops()
    x = C.prefill_inputs(dt, H, kv, D)
    gold = GOLD_PRE[f"prefill_{dt}_h{H}_kv{kv}_d{D}"]
    out = ops.prefill_attention(x["q"].to(cuda), x["k"].to(cuda), x["v"].to(cuda),
                                x["cu_seqlens"].to(cuda), x["max_seqlen"])
    assert _maxdiff(out, gold["out"]) <= ATOL[C.DTYPES[dt]], _maxdiff(out, gold["out"])


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,kv,D", [(32, 8, 128), (14, 2, 64), (8, 1, 128)])
def test_prefill_random_lengths(cuda, dt, H, kv, D):
    ops = _ops()
    g = torch.Generator().manual_seed(17)
    lens = [1, 127, 128, 129, 300, 0, 64]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T = int(cu[-1])
    q = torch.randn(T, H, D, generator=g).to(dt)
    k = torch.randn(T, kv, D, generator=g).to(dt)
    v = torch.randn(T, kv, D, generator=g).to(dt)
    ref = no.prefill_attention(q.float(), k.float(), v.float(), cu, H, kv)
    out = ops.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), cu.to(cuda), max(lens))
    assert _maxdiff(out, ref) <= ATOL[dt]


_CFG_CHECK = r"""
import math, sys, torch
sys.path.insert(0, '.')
from needle_b200 import ops
from oracle import needle_oracle as no
g = torch.Generator().manual_seed(19)
for H, kv, D in ((32, 8, 128), (14, 2, 64), (8, 1, 128)):
    B, N, maxb = 11, 900, 80
    ctx = torch.randint(0, maxb * 16 - 1, (B,), generator=g).to(torch.int32)
    ctx[0] = 0
    ctx[1] = maxb * 16 - 1
    bt = torch.randperm(N, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    cache = torch.randn(2, N, kv, 16, D, generator=g).to(torch.bfloat16)
    ref = no.decode_attention(q.float(), cache.float(), bt, ctx, 1 / math.sqrt(D), H, kv, D)
    dev = torch.device('cuda:0')
    for pps in (None, 4, 9, 32):
        plan = None if pps is None else ops.DecodePlan(B, H, kv, D, maxb, 16, dev, pps)
        out = ops.paged_decode(q.to(dev), cache.to(dev), bt.to(dev), ctx.to(dev),
                               1 / math.sqrt(D), plan=plan)
        err = (out.float().cpu() - ref).abs().max().item()
        assert err <= 2e-2, (H, kv, D, pps, err)
assert ops.device_errors() == 0
print('ok')
"""


@pytest.mark.parametrize("cfg", ["4,2", "4,3", "4,4", "8,2"])
def test_decode_every_kernel_config(cuda, cfg):
    """Each (warps, stages) instantiation of the tensor-core decode kernel,
    selected through NB_DECODE_CFG in a fresh process."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NB_DECODE_CFG=cfg)
    r = subprocess.run([sys.executable, "-c", _CFG_CHECK], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_silu_mul_matches_needle_ops(cuda, dt):
    """Fused SwiGLU vs needle's F.silu(gate) * up (llama.py:37) evaluated by
    torch on the same device: within one unit in the last place."""
    ops = _ops()
    g = torch.Generator().manual_seed(23)
    T, I = 37, 1792
    gu = (torch.randn(T, 2 * I, generator=g) * 3).to(dt).to(cuda)
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    out = ops.silu_mul(gu)
    bad, md = _ulp_close(out, ref, dt)
    assert bad == 0, (bad, md)


_PREFILL_CHECK = r"""
import math, sys, numpy as np, torch
sys.path.insert(0, '.')
from needle_b200 import ops
from oracle import needle_oracle as no
g = torch.Generator().manual_seed(29)
for dt in (torch.bfloat16, torch.float16):
    for H, kv, D in ((32, 8, 128), (14, 2, 64), (4, 4, 128)):
        lens = [1, 127, 128, 129, 255, 256, 257, 600, 0, 64]
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
        T = int(cu[-1])
        q = torch.randn(T, H, D, generator=g).to(dt)
        k = torch.randn(T, kv, D, generator=g).to(dt)
        v = torch.randn(T, kv, D, generator=g).to(dt)
        ref = no.prefill_attention(q.float(), k.float(), v.float(), cu, H, kv)
        dev = torch.device('cuda:0')
        out = ops.prefill_attention(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), max(lens))
        err = (out.float().cpu() - ref).abs().max().item()
        assert err <= 2e-2, (dt, H, kv, D, err)
assert ops.device_errors() == 0
print('ok')
"""


@pytest.mark.parametrize("version", ["1", "2", "3", "3-rows"])
def test_prefill_every_kernel_version(cuda, version):
    """Every tensor-core prefill kernel (single softmax group / two ping-pong
    groups per CTA / persistent warp-specialised, the last with head-pair
    units for even GQA groups and, "3-rows", with the row halves of one head
    for every group), selected through NB_PREFILL_V / NB_PF3_PAIR in a fresh
    process, on lengths around the 128- and 256-row tile edges, bf16 and
    fp16."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NB_PREFILL_V=version[0])
    if version == "3-rows":
        env["NB_PF3_PAIR"] = "0"
    r = subprocess.run([sys.executable, "-c", _PREFILL_CHECK], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def _sdpa_fp32(q, k, v, cu, H, kv):
    """Causal attention per sequence in fp32 with torch on the GPU (GQA by
    repeating KV heads): the plain reference for large prefill cases."""
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for s in range(len(cu) - 1):
        a, b = int(cu[s]), int(cu[s + 1])
        if b == a:
            continue
        qs = q[a:b].float().transpose(0, 1)
        ks = k[a:b].float().transpose(0, 1).repeat_interleave(H // kv, dim=0)
        vs = v[a:b].float().transpose(0, 1).repeat_interleave(H // kv, dim=0)
        out[a:b] = torch.nn.functional.scaled_dot_product_attention(
            qs, ks, vs, is_causal=True).transpose(0, 1)
    return out


@pytest.mark.parametrize("lens", [[1024] * 16, [3000, 17, 700, 1, 2049, 256, 1500, 90]])
def test_prefill_many_units_per_cta(cuda, lens):
    """Batches with many more (query block, head, sequence) units than SMs,
    so every persistent CTA runs several units back to back (its K/V rings,
    barrier phases and tensor memory carry over from unit to unit), against
    fp32 torch attention; bf16, 32/8 heads, D = 128."""
    ops = _ops()
    H, kv, D = 32, 8, 128
    g = torch.Generator(device=cuda).manual_seed(31)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T = int(cu[-1])
    q = torch.randn(T, H, D, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(T, kv, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(T, kv, D, device=cuda, generator=g).to(torch.bfloat16)
    out = ops.prefill_attention(q, k, v, cu.to(cuda), max(lens))
    ref = _sdpa_fp32(q, k, v, cu, H, kv)
    assert ops.device_errors() == 0
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2, err


_STORE_PATH_CHECK = r"""
import sys
import numpy as np
import torch
from needle_b200 import ops
dev = torch.device("cuda:0")
H, kv, D = 32, 8, 128
lens = [1024, 300, 129, 128]
g = torch.Generator(device=dev).manual_seed(41)
cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32).to(dev)
T = sum(lens)
q = torch.randn(T, H, D, device=dev, generator=g).to(torch.bfloat16)
k = torch.randn(T, kv, D, device=dev, generator=g).to(torch.bfloat16)
v = torch.randn(T, kv, D, device=dev, generator=g).to(torch.bfloat16)
dense = ops.prefill_attention(q, k, v, cu, max(lens))
# a wider row pitch (still 16-byte aligned: the tensor-core kernel takes it)
pitch = H * D + 64
buf = torch.full((T * pitch + 64,), 7.0, device=dev, dtype=torch.bfloat16)
rows = buf[:T * pitch].view(T, pitch)
view = rows[:, :H * D].view(T, H, D)
ops.prefill_attention(q, k, v, cu, max(lens), out=view)
assert ops.device_errors() == 0
assert torch.equal(view.view(torch.int16), dense.view(torch.int16))
assert (rows[:, H * D:] == 7).all() and (buf[T * pitch:] == 7).all()
dense.view(torch.int16).cpu().numpy().tofile(sys.argv[1])
print("ok")
"""


def test_prefill_output_store_paths_agree(cuda, tmp_path):
    """Whole 128-row output tiles leave the tcgen05 kernel through shared
    memory and TMA stores; the ragged last tile of a sequence, and every tile
    with NB_PF3_TMA_STORE=0, through plain per-row 16-byte stores.  Both
    runs (fresh processes) must give the same bits, for a dense output and
    for one with a wider row pitch, whose padding stays untouched.  (An
    output that is not 16-byte aligned never reaches this kernel: the
    library takes its SIMT prefill then.)"""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = []
    for flag in ("1", "0"):
        f = tmp_path / f"out{flag}.bin"
        env = dict(os.environ, NB_PF3_TMA_STORE=flag)
        r = subprocess.run([sys.executable, "-c", _STORE_PATH_CHECK, str(f)], cwd=root, env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
        outs.append(f.read_bytes())
    assert outs[0] == outs[1]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_swap_kv_blocks_round_trip(cuda, dt):
    """Swap-out to a pinned host cache and swap-in to other device blocks,
    all layers in one launch each, against needle's per-block copies
    (runner.py:187-192): cpu[:, dst] = gpu[:, src], then gpu[:, dst] = cpu[:, src]."""
    ops = _ops()
    g = torch.Generator().manual_seed(31)
    L_, N, M, kv, D = 3, 20, 10, 2, 64
    gpu = [torch.randn(2, N, kv, 16, D, generator=g).to(dt).to(cuda) for _ in range(L_)]
    cpu = [torch.zeros(2, M, kv, 16, D, dtype=dt).pin_memory() for _ in range(L_)]
    out_map = {3: 0, 7: 5, 19: 9}
    ops.swap_kv_blocks(gpu, cpu, torch.tensor(list(out_map.items()), dtype=torch.int32,
                                               device=cuda))
    torch.cuda.synchronize()
    for l_ in range(L_):
        ref = torch.zeros_like(cpu[l_])
        for s_, d_ in out_map.items():
            ref[:, d_] = gpu[l_][:, s_].cpu()
        assert _bits_equal(cpu[l_], ref)
    before = [t.clone() for t in gpu]
    in_map = {0: 11, 5: 2, 9: 19}
    ops.swap_kv_blocks(cpu, gpu, torch.tensor(list(in_map.items()), dtype=torch.int32,
                                               device=cuda))
    torch.cuda.synchronize()
    for l_ in range(L_):
        ref = before[l_].cpu()
        for s_, d_ in in_map.items():
            ref[:, d_] = cpu[l_][:, s_]
        assert _bits_equal(gpu[l_], ref)
    assert ops.device_errors() == 0
    ops.swap_kv_blocks(gpu, cpu, torch.tensor([[N + 3, 1]], dtype=torch.int32, device=cuda))
    assert ops.device_errors() & 1        # out-of-range source block flagged, nothing copied
