"""The per-forward KV slot table and the KV writers that read it.

``slot_mapping`` resolves every new token's cache position once per forward
(needle recomputes it per layer, ``needle/layers/attention.py:140-154,
204-246``); ``store_kvcache_slots`` / ``rope_store_kvcache_slots`` then write
through it.  The cache, q and k must come out byte-identical to the oracle's
``write_kv`` / ``decode_write_kv`` / ``apply_rope`` (pinned to needle by the
golden vectors), including the clamp case (last token wins), ctx > 0, empty
sequences, strided rows and out-of-pool block ids (flagged, not written).
"""
import numpy as np
import pytest
import torch

from oracle import needle_oracle as no
from tests.golden import cases as C

pytestmark = pytest.mark.gpu


def _ops():
    from needle_b200 import ops
    return ops


def _bits_equal(a, b):
    a, b = a.cpu(), b.cpu()
    if a.dtype in (torch.bfloat16, torch.float16):
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    return torch.equal(a.view(torch.int32), b.view(torch.int32))


def _slots_host(bt, cu, ctx, bs, nblk):
    """Host restatement of the slot rule: position ctx + i, column clamped to
    the last table column, an earlier token on a clamped slot superseded by a
    later one, block ids outside the pool not written."""
    out = []
    maxb = bt.shape[1]
    for s in range(len(ctx)):
        n = int(cu[s + 1] - cu[s])
        for i in range(n):
            pos = int(ctx[s]) + i
            col_u = pos // bs
            col = min(col_u, maxb - 1)
            if col_u >= maxb - 1 and pos + bs < int(ctx[s]) + n:
                out.append(-1)
                continue
            phys = int(bt[s, col])
            out.append(phys * bs + (pos - col_u * bs) if 0 <= phys < nblk else -1)
    return torch.tensor(out, dtype=torch.int32)


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
@pytest.mark.parametrize("kv,D", C.KV_WRITE_SHAPES)
def test_slot_store_bit_exact(cuda, dt, kv, D):
    ops = _ops()
    x = C.kv_write_inputs(dt, kv, D)
    ref = x["cache"].clone()
    no.write_kv(x["k"], x["v"], ref, x["block_table"], x["cu_seqlens"], x["context_lens"])
    T = x["k"].shape[0]
    slots = ops.slot_mapping(x["block_table"].to(cuda), x["context_lens"].to(cuda),
                             ref.shape[1], ref.shape[3], cu_seqlens=x["cu_seqlens"].to(cuda),
                             num_tokens=T)
    assert torch.equal(slots.cpu(), _slots_host(x["block_table"], x["cu_seqlens"],
                                                x["context_lens"], 16, ref.shape[1]))
    cache = x["cache"].to(cuda)
    ops.store_kvcache_slots(x["k"].to(cuda), x["v"].to(cuda), cache, slots)
    assert ops.device_errors() == 0
    assert _bits_equal(cache, ref)


@pytest.mark.parametrize("dt", ["bfloat16", "float32"])
def test_slot_store_clamp_last_token_wins(cuda, dt):
    ops = _ops()
    x = C.kv_write_clamp_inputs(dt)
    ref = x["cache"].clone()
    no.write_kv(x["k"], x["v"], ref, x["block_table"], x["cu_seqlens"], x["context_lens"])
    slots = ops.slot_mapping(x["block_table"].to(cuda), x["context_lens"].to(cuda),
                             ref.shape[1], 16, cu_seqlens=x["cu_seqlens"].to(cuda),
                             num_tokens=x["k"].shape[0])
    assert int((slots.cpu() < 0).sum()) == 40 - 32   # 8 earlier tokens superseded
    cache = x["cache"].to(cuda)
    ops.store_kvcache_slots(x["k"].to(cuda), x["v"].to(cuda), cache, slots)
    assert _bits_equal(cache, ref)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_slot_store_decode_form(cuda, dt):
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
    slots = ops.slot_mapping(bt.to(cuda), ctx.to(cuda), N, 16)
    ops.store_kvcache_slots(k.to(cuda), v.to(cuda), c, slots)
    assert _bits_equal(c, ref)


def test_slot_bad_block_id_is_flagged_not_written(cuda):
    ops = _ops()
    kv, D, N = 2, 64, 8
    cache = torch.zeros(2, N, kv, 16, D, dtype=torch.bfloat16, device=cuda)
    k = torch.ones(2, kv, D, dtype=torch.bfloat16, device=cuda)
    bt = torch.tensor([[N + 5], [1]], dtype=torch.int32, device=cuda)
    ctx = torch.tensor([0, 0], dtype=torch.int32, device=cuda)
    slots = ops.slot_mapping(bt, ctx, N, 16)
    assert ops.device_errors() & 1
    assert slots.tolist() == [-1, 16]
    ops.store_kvcache_slots(k, k, cache, slots)
    assert cache[:, 1].abs().sum().item() > 0
    assert cache[:, [0, 2, 3, 4, 5, 6, 7]].abs().sum().item() == 0
    # a slot beyond the pool handed in directly is skipped and flagged too
    ops.store_kvcache_slots(k, k, cache, torch.tensor([N * 16 + 3, -1], dtype=torch.int32,
                                                      device=cuda))
    assert ops.device_errors() & 1


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("prefill", [True, False])
def test_slot_rope_store_bit_exact(cuda, dt, prefill):
    """RoPE + KV write through the slot table against the oracle, with q/k/v
    as column slices of a fused projection (strided rows)."""
    ops = _ops()
    g = torch.Generator().manual_seed(13)
    D, hq, kv, N = 128, 8, 2, 40
    lens = [5, 33, 1, 16] if prefill else [1, 1, 1, 1]
    ctx = torch.tensor([0, 7, 100, 15], dtype=torch.int32)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T = int(cu[-1])
    bt = torch.randperm(N, generator=g)[:4 * 9].view(4, 9).to(torch.int32)
    qkv = torch.randn(T, (hq + 2 * kv) * D, generator=g).to(dt)
    q = qkv[:, :hq * D].view(T, hq, D)
    k = qkv[:, hq * D:(hq + kv) * D].view(T, kv, D)
    v = qkv[:, (hq + kv) * D:].view(T, kv, D)
    cos_t, sin_t = no.rope_cache(D, 4096, 5e5)
    pos = torch.cat([torch.arange(c, c + n) for c, n in zip(ctx.tolist(), lens)])
    cos, sin = cos_t.to(dt)[pos], sin_t.to(dt)[pos]
    qr, kr = no.apply_rope(q.clone(), k.clone(), cos, sin)
    ref = torch.zeros(2, N, kv, 16, D, dtype=dt)
    no.write_kv(kr, v, ref, bt, cu, ctx)
    qkv_d = qkv.to(cuda)
    qd = qkv_d[:, :hq * D].view(T, hq, D)
    kd = qkv_d[:, hq * D:(hq + kv) * D].view(T, kv, D)
    vd = qkv_d[:, (hq + kv) * D:].view(T, kv, D)
    c = torch.zeros_like(ref, device=cuda)
    slots = ops.slot_mapping(bt.to(cuda), ctx.to(cuda), N, 16,
                             cu_seqlens=cu.to(cuda) if prefill else None, num_tokens=T)
    ops.rope_store_kvcache_slots(qd, kd, vd, cos.to(cuda), sin.to(cuda), c, slots,
                                 write_k_back=True)
    assert ops.device_errors() == 0
    assert _bits_equal(qd, qr)
    assert _bits_equal(kd, kr)
    assert _bits_equal(c, ref)


def test_slot_writers_match_self_resolving_writers_at_scale(cuda):
    """Prefill-size write (8 x 1024 tokens, kv 8, D 128, shuffled 20000-block
    pool): the slot path and nb_rope_store_kvcache leave identical bytes."""
    ops = _ops()
    g = torch.Generator(device=cuda).manual_seed(0)
    B, S, H, KV, D, N = 8, 1024, 32, 8, 128, 20000
    T = B * S
    mk = lambda h: torch.randn(T, h, D, device=cuda, generator=g, dtype=torch.bfloat16)
    q, k, v = mk(H), mk(KV), mk(KV)
    perm = torch.randperm(N, generator=torch.Generator().manual_seed(0))[:B * S // 16]
    bt = perm.view(B, S // 16).to(device=cuda, dtype=torch.int32)
    ctx = torch.zeros(B, dtype=torch.int32, device=cuda)
    cu = torch.arange(0, T + 1, S, dtype=torch.int32, device=cuda)
    cos_t, sin_t = no.rope_cache(D, S, 1e6)
    pos = torch.arange(S).repeat(B)
    cos, sin = cos_t.to(torch.bfloat16)[pos].to(cuda), sin_t.to(torch.bfloat16)[pos].to(cuda)
    c1 = torch.zeros(2, N, KV, 16, D, dtype=torch.bfloat16, device=cuda)
    c2 = torch.zeros_like(c1)
    q1, k1, q2, k2 = q.clone(), k.clone(), q.clone(), k.clone()
    ops.rope_store_kvcache(q1, k1, v, cos, sin, c1, bt, ctx, cu_seqlens=cu, write_k_back=True)
    slots = ops.slot_mapping(bt, ctx, N, 16, cu_seqlens=cu, num_tokens=T)
    ops.rope_store_kvcache_slots(q2, k2, v, cos, sin, c2, slots, write_k_back=True)
    assert ops.device_errors() == 0
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))
    assert torch.equal(q1.view(torch.int16), q2.view(torch.int16))
    assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))
    c3 = torch.zeros_like(c1)
    ops.store_kvcache_slots(k, v, c3, slots)
    c4 = torch.zeros_like(c1)
    ops.store_kvcache(k, v, c4, bt, ctx, cu_seqlens=cu)
    assert torch.equal(c3.view(torch.int16), c4.view(torch.int16))
