"""CPU oracle for needle's attention hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, operation for operation, what mitu626/needle computes on
its PyTorch (non-FlashInfer) path for the functions that the B200 kernels
replace.  It exists to check the CUDA path, never to stand in for it: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product path
(``needle_b200.ops`` and everything above it) never calls into this file and
fails loudly when the CUDA library is missing.

Parity of this restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports needle and runs its
own functions on seeded inputs); ``tests/test_oracle_golden.py`` checks every
function here against those vectors bit for bit.

Integer/byte work (slot computation, KV scatter) is done with numpy on the raw
bit patterns, so it is exact by construction.  Floating-point work uses torch
CPU tensors in the cache / model dtype because that is how the reference
rounds: every elementwise op of a bf16 tensor rounds its result to bf16, the
softmax of the decode fallback runs in bf16, and so on.  Reusing the same
torch ops is the only way to reproduce those rounding points exactly.
"""
from __future__ import annotations

import math
from typing import Tuple

import numpy as np
import torch
import torch.nn.functional as F

__all__ = [
    "slot_mapping",
    "write_kv",
    "decode_write_kv",
    "decode_attention",
    "prefill_attention",
    "rope_cache",
    "apply_rope",
    "rms_norm",
    "add_rms_norm",
]


def _int_view(t: torch.Tensor) -> np.ndarray:
    """Raw bit pattern of a CPU tensor as a numpy integer array (no copy)."""
    bits = {1: torch.int8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.view(bits).numpy()


def slot_mapping(
    block_table: np.ndarray,
    cu_seqlens: np.ndarray,
    context_lens: np.ndarray,
    block_size: int,
) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-token (physical block, in-block offset, sequence index).

    Restates ``needle/layers/attention.py:214-240`` (``_write_kv``): the
    absolute position of token i of sequence s is ``context_lens[s] + i``; the
    block-table column is ``abs_pos // block_size`` clamped to the last
    column (``:235``); the offset is ``abs_pos % block_size``.
    """
    block_table = np.asarray(block_table, dtype=np.int64)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    ctx = np.asarray(context_lens, dtype=np.int64)
    seq_len = cu[1:] - cu[:-1]
    seq_idx = np.repeat(np.arange(len(seq_len), dtype=np.int64), seq_len)
    tok = np.arange(int(cu[-1]), dtype=np.int64)
    abs_pos = ctx[seq_idx] + (tok - cu[:-1][seq_idx])
    col = np.minimum(abs_pos // block_size, block_table.shape[1] - 1)
    phys = block_table[seq_idx, col]
    off = abs_pos % block_size
    return phys, off, seq_idx


def write_kv(
    k: torch.Tensor,
    v: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    cu_seqlens: torch.Tensor,
    context_lens: torch.Tensor,
) -> None:
    """Scatter prefill K/V into the paged cache, in place.

    Restates ``needle/layers/attention.py:204-246``.  ``kv_cache`` is
    ``[2, num_blocks, num_kv_heads, block_size, head_dim]``; ``k``/``v`` are
    ``[T, num_kv_heads, head_dim]``.  The copy is done on raw bit patterns, so
    it is byte-exact.  Tokens are applied in order, so when two tokens of the
    same sequence land on one slot (only possible through the column clamp)
    the later token wins -- the sequential-CPU behaviour of the reference's
    ``index_put_``.
    """
    block_size = kv_cache.shape[3]
    phys, off, _ = slot_mapping(block_table.numpy(), cu_seqlens.numpy(),
                                context_lens.numpy(), block_size)
    cache = _int_view(kv_cache)
    kb = _int_view(k.contiguous())
    vb = _int_view(v.contiguous())
    for t in range(len(phys)):
        cache[0, phys[t], :, off[t], :] = kb[t]
        cache[1, phys[t], :, off[t], :] = vb[t]


def decode_write_kv(
    k: torch.Tensor,
    v: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
) -> None:
    """Write the one new decode token per sequence into the cache, in place.

    Restates ``needle/layers/attention.py:140-154``: the slot of sequence s
    is position ``context_lens[s]`` (the tokens already cached), with the same
    column clamp as the prefill write.
    """
    b = k.shape[0]
    cu = torch.arange(b + 1, dtype=torch.int32)
    write_kv(k, v, kv_cache, block_table, cu, context_lens)


def decode_attention(
    q: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    num_heads: int,
    num_kv_heads: int,
    head_dim: int,
) -> torch.Tensor:
    """Paged decode attention over ``context_lens + 1`` cached tokens.

    Restates ``needle/layers/attention.py:291-310`` (``_decode_pytorch``):
    gather the pages of each sequence, expand K/V to the query heads with
    ``repeat_interleave`` (query head j reads KV head ``j // group``), then
    ``einsum`` QK^T * scale, softmax and ``einsum`` PV -- all in the cache
    dtype, exactly as the reference rounds them.
    """
    num_seqs = q.shape[0]
    block_size = kv_cache.shape[3]
    outs = []
    for i in range(num_seqs):
        ctx_len = int(context_lens[i]) + 1
        nb = (ctx_len + block_size - 1) // block_size
        phys = block_table[i, :nb].long()
        k_full = kv_cache[0][phys].transpose(0, 1).reshape(num_kv_heads, -1, head_dim)[:, :ctx_len]
        v_full = kv_cache[1][phys].transpose(0, 1).reshape(num_kv_heads, -1, head_dim)[:, :ctx_len]
        expand = num_heads // num_kv_heads
        k_exp = k_full.repeat_interleave(expand, dim=0)
        v_exp = v_full.repeat_interleave(expand, dim=0)
        w = torch.einsum("hd,hsd->hs", q[i], k_exp) * scale
        outs.append(torch.einsum("hs,hsd->hd", w.softmax(dim=-1), v_exp))
    return torch.stack(outs, dim=0)


def prefill_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
) -> torch.Tensor:
    """Causal attention over each sequence's new tokens.

    Restates ``needle/layers/attention.py:120-134`` (``_prefill_pytorch``):
    per sequence, ``scaled_dot_product_attention(is_causal=True)`` with the
    default 1/sqrt(D) scale and GQA expanded by ``repeat_interleave``.
    """
    outs = []
    cu = [int(x) for x in cu_seqlens.tolist()]
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        qi = q[s:e].unsqueeze(0).transpose(1, 2)
        ki = k[s:e].unsqueeze(0).transpose(1, 2)
        vi = v[s:e].unsqueeze(0).transpose(1, 2)
        if num_kv_heads != num_heads:
            f = num_heads // num_kv_heads
            ki = ki.repeat_interleave(f, dim=1)
            vi = vi.repeat_interleave(f, dim=1)
        o = F.scaled_dot_product_attention(qi, ki, vi, is_causal=True)
        outs.append(o.transpose(1, 2).squeeze(0))
    return torch.cat(outs, dim=0)


def rope_cache(head_dim: int, max_seq_len: int, base: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin tables ``[max_seq_len, head_dim]`` (NeoX half split).

    Restates ``needle/layers/rope.py:13-24``: ``inv_freq = 1 / base **
    (arange(0, D, 2) / D)`` in fp32, ``freqs = outer(t, inv_freq)``,
    ``emb = cat(freqs, freqs)``.  A bf16 model casts both tables to bf16
    (``model.to(dtype)``, ``needle/model/runner.py:34``).
    """
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2).float() / head_dim))
    t = torch.arange(max_seq_len).float()
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def apply_rope(q, k, cos, sin):
    """``q*cos + rotate_half(q)*sin`` (same for k), rounding after every op.

    Restates ``needle/layers/attention.py:277-288``; cos/sin are ``[T, D]``
    and broadcast over heads.
    """
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    return q * c + _rotate_half(q) * s, k * c + _rotate_half(k) * s


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm as needle computes it (``needle/layers/norm.py:14-17``).

    The variance is an fp32 mean of squares; ``x * rsqrt(var + eps)`` is
    promoted to fp32, rounded back to the weight dtype, then multiplied by
    the weight in that dtype.
    """
    variance = x.float().pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(variance + eps)
    return weight * y.to(weight.dtype)


def add_rms_norm(x, residual, weight, eps):
    """Residual add then RMSNorm (``needle/model/llama.py:67-70``).

    Returns ``(rms_norm(residual + x), residual + x)``; the sum is rounded to
    the model dtype before it is normalised, as in the reference.
    """
    h = residual + x
    return rms_norm(h, weight, eps), h


def default_scale(head_dim: int) -> float:
    """Softmax scale used by needle (``needle/layers/attention.py:48``)."""
    return 1.0 / math.sqrt(head_dim)


def sampler_filtered_logits(logit: torch.Tensor, temperature: float, top_k: int,
                            top_p: float) -> torch.Tensor:
    """One row of needle's sampler before the draw (``needle/model/sampler.py:33-46``).

    ``logit / temperature`` with a Python float (fp32 divide, one rounding to
    the row's dtype), top-k masking ``logit < kth`` -> -inf, then top-p on the
    descending sort: a token is removed when the probability mass before it
    exceeds ``top_p`` (compared in the row's dtype), scattered back.
    """
    logit = logit / temperature
    if top_k > 0:
        k = min(top_k, logit.size(-1))
        kth = logit.topk(k).values[-1]
        logit = logit.masked_fill(logit < kth, float("-inf"))
    if top_p < 1.0:
        sl, si = logit.sort(descending=True)
        cum = sl.softmax(dim=-1).cumsum(dim=-1)
        remove = cum - sl.softmax(dim=-1) > top_p
        sl[remove] = float("-inf")
        logit = logit.scatter(0, si, sl)
    return logit
