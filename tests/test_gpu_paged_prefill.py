"""Paged prefill: the new tokens of each sequence attend over the sequence's
whole context (its ``context_lens`` cached tokens and the new ones), with K
and V read from the paged cache through the block table.

needle's prefill attends over the new tokens only (``attention.py:101-134``),
which its TODO lists as wrong for continuations; its decode attends over the
cached tokens (``attention.py:291-310``).  So the oracle for a chunk of n new
tokens after c cached ones is n decode steps: new token i equals
``decode_attention`` (pinned to needle's ``_decode_pytorch`` by the golden
vectors) at ``context_lens = c + i``.  Cases: cached prefixes 0, 1, 17, 130
and 1000 tokens; chunk lengths 1 to 300 (tile edges at 128); GQA groups 4
(head-pair units), 7 and 1 (row-half units); head_dim 128 and 64; bf16 and
fp16; the ``context_lens = 0`` case against the contiguous prefill.
Tolerance 2e-2 max-abs (bf16/fp16, as every attention test here).
"""
import math

import numpy as np
import pytest
import torch

from oracle import needle_oracle as no

pytestmark = pytest.mark.gpu


def _ops():
    from needle_b200 import ops
    return ops


def _case(H, kv, D, ctx, lens, dt, seed):
    """A cache holding every sequence's prefix and new tokens (random K/V),
    the new tokens' q, block tables over a shuffled pool."""
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    tot = [c + n for c, n in zip(ctx, lens)]
    maxb = max((t + 15) // 16 for t in tot) + 1
    N = B * maxb + 7
    bt = torch.randperm(N, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    cache = torch.zeros(2, N, kv, 16, D, dtype=dt)
    for s in range(B):
        k = torch.randn(tot[s], kv, D, generator=g).to(dt)
        v = torch.randn(tot[s], kv, D, generator=g).to(dt)
        cu1 = torch.tensor([0, tot[s]], dtype=torch.int32)
        no.write_kv(k, v, cache, bt[s:s + 1], cu1, torch.zeros(1, dtype=torch.int32))
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    q = torch.randn(int(cu[-1]), H, D, generator=g).to(dt)
    return q, cache, bt, torch.tensor(ctx, dtype=torch.int32), cu


def _decode_steps_ref(q, cache, bt, ctx, cu, H, kv, D):
    """New token i of sequence s = one decode step at context_lens = ctx + i."""
    rows, tabs, cls = [], [], []
    for s in range(len(ctx)):
        for i in range(int(cu[s + 1] - cu[s])):
            rows.append(int(cu[s]) + i)
            tabs.append(bt[s])
            cls.append(int(ctx[s]) + i)
    ref = no.decode_attention(q[rows].float(), cache.float(), torch.stack(tabs),
                              torch.tensor(cls, dtype=torch.int32), 1 / math.sqrt(D), H, kv, D)
    return ref


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,kv,D", [(32, 8, 128), (14, 2, 64), (4, 4, 128)])
def test_paged_prefill_equals_decode_steps(cuda, dt, H, kv, D):
    ops = _ops()
    ctx = [0, 1, 17, 130, 1000]
    lens = [300, 7, 128, 129, 40]
    q, cache, bt, cl, cu = _case(H, kv, D, ctx, lens, dt, seed=H + D)
    out = ops.prefill_attention_paged(q.to(cuda), cache.to(cuda), bt.to(cuda), cl.to(cuda),
                                      cu.to(cuda), max(lens))
    assert ops.device_errors() == 0
    ref = _decode_steps_ref(q, cache, bt, cl, cu, H, kv, D)
    err = (out.float().cpu() - ref.float()).abs().max().item()
    assert err <= 2e-2, err


def test_paged_prefill_without_context_equals_prefill(cuda):
    """context_lens = 0: the same result as the contiguous prefill of the
    same tokens (keys are the new tokens only)."""
    ops = _ops()
    H, kv, D = 32, 8, 128
    lens = [1, 127, 128, 129, 600]
    ctx = [0] * len(lens)
    q, cache, bt, cl, cu = _case(H, kv, D, ctx, lens, torch.bfloat16, seed=3)
    # the same K/V rows, gathered back to token-major tensors
    ks, vs = [], []
    for s, n in enumerate(lens):
        pages = bt[s, :(n + 15) // 16].long()
        ks.append(cache[0][pages].transpose(0, 1).reshape(kv, -1, D)[:, :n].transpose(0, 1))
        vs.append(cache[1][pages].transpose(0, 1).reshape(kv, -1, D)[:, :n].transpose(0, 1))
    k, v = torch.cat(ks).contiguous(), torch.cat(vs).contiguous()
    a = ops.prefill_attention_paged(q.to(cuda), cache.to(cuda), bt.to(cuda), cl.to(cuda),
                                    cu.to(cuda), max(lens))
    b = ops.prefill_attention(q.to(cuda), k.to(cuda), v.to(cuda), cu.to(cuda), max(lens))
    assert ops.device_errors() == 0
    assert (a.float() - b.float()).abs().max().item() <= 2e-2


def test_paged_prefill_table_narrower_than_context(cuda):
    """A context longer than the block table reads only its pages, as decode
    does (needle's block_table[i, :nb] slice): keys past max_blocks * 16 do
    not exist for either."""
    ops = _ops()
    H, kv, D = 8, 2, 128
    q, cache, bt, cl, cu = _case(H, kv, D, [200, 0], [60, 40], torch.bfloat16, seed=8)
    bt = bt[:, :12].contiguous()  # 192 keys: shorter than 200 + 60
    out = ops.prefill_attention_paged(q.to(cuda), cache.to(cuda), bt.to(cuda), cl.to(cuda),
                                      cu.to(cuda), 60)
    assert ops.device_errors() == 0
    ref = _decode_steps_ref(q, cache, bt, cl, cu, H, kv, D)
    assert (out.float().cpu() - ref.float()).abs().max().item() <= 2e-2


def test_paged_prefill_bad_block_id_is_flagged(cuda):
    """A block id outside the pool is recorded and read as zeros, not
    followed."""
    ops = _ops()
    H, kv, D = 8, 2, 128
    q, cache, bt, cl, cu = _case(H, kv, D, [20], [10], torch.bfloat16, seed=5)
    bt[0, 0] = cache.shape[1] + 3
    ops.prefill_attention_paged(q.to(cuda), cache.to(cuda), bt.to(cuda), cl.to(cuda),
                                cu.to(cuda), 10)
    assert ops.device_errors() & 1


def test_runner_option_sets_every_layer(cuda):
    from needle_b200.model import ModelRunner, preset
    cfg = preset("qwen2-0.5b")
    r = ModelRunner(cfg, dtype="bfloat16", device=str(cuda), prefill_with_context=True)
    assert all(l.self_attn.prefill_with_context for l in r.model.model.layers)
    r2 = ModelRunner(cfg, dtype="bfloat16", device=str(cuda))
    assert not any(l.self_attn.prefill_with_context for l in r2.model.model.layers)
