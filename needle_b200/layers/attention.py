"""Drop-in replacement for needle's ``Attention`` module on the B200 kernels.

Same constructor (``needle/layers/attention.py:36-63``), same parameter names
(``q_proj``/``k_proj``/``v_proj``/``o_proj``, so needle state dicts load
unchanged) and the same ``forward`` signature and contract
(``needle/layers/attention.py:70-96``):

    forward(hidden_states [T, hidden], positions [T], kv_cache [2, N, kv, bs, D],
            block_table [B, maxb] int32, cu_seqlens [B+1] int32,
            context_lens [B] int32, max_seqlen, is_prefill, cos [T, D], sin [T, D])
        -> [T, hidden]

What changes is underneath: RoPE and the KV-cache write are one fused kernel
(``rope_store_kvcache``); prefill attention and paged split-K decode are
hand-written sm_100a kernels; none of needle's per-layer host syncs
(``.cpu()`` at attention.py:111,170,222-223,297) or Python loops over
sequences remain.  The KV cache is mutated in place, as in needle.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from .linear import ColumnParallelLinear, RowParallelLinear, dense


def _aligned16(*ts) -> bool:
    """Every tensor starts on a 16-byte boundary and its rows stay on one (the
    slot writers move 16-byte vectors)."""
    for t in ts:
        if t.data_ptr() % 16 or (t.stride(0) * t.element_size()) % 16:
            return False
    return True


class Attention(nn.Module):
    def __init__(self, config, layer_idx: int, tp_size: int = 1, tp_rank: int = 0,
                 qkv_bias: bool = False):
        super().__init__()
        self.layer_idx = layer_idx
        self.num_heads = config.num_attention_heads // tp_size
        self.num_kv_heads = max(1, config.num_key_value_heads // tp_size)
        self.head_dim = config.head_dim
        self.scale = 1.0 / math.sqrt(self.head_dim)
        H, KV, D = config.num_attention_heads, config.num_key_value_heads, config.head_dim
        self.q_proj = ColumnParallelLinear(config.hidden_size, H * D, bias=qkv_bias,
                                           tp_size=tp_size, tp_rank=tp_rank)
        self.k_proj = ColumnParallelLinear(config.hidden_size, KV * D, bias=qkv_bias,
                                           tp_size=tp_size, tp_rank=tp_rank)
        self.v_proj = ColumnParallelLinear(config.hidden_size, KV * D, bias=qkv_bias,
                                           tp_size=tp_size, tp_rank=tp_rank)
        self.o_proj = RowParallelLinear(H * D, config.hidden_size, tp_size=tp_size,
                                        tp_rank=tp_rank)
        self._qkv_w = None
        self._qkv_b = None
        # False (needle's prefill): the new tokens attend over the new tokens
        # only; True: over the cached prefix too (ModelRunner's
        # prefill_with_context), the continuation case needle does not handle
        self.prefill_with_context = False

    @torch.no_grad()
    def fuse_qkv(self) -> None:
        """Place the q/k/v weights (and biases) in one buffer so the three
        projections run as one GEMM.  The parameters become views into that
        buffer, so loading ``q_proj.weight`` etc. keeps working."""
        projs = (self.q_proj, self.k_proj, self.v_proj)
        self._qkv_w = torch.cat([p.weight for p in projs], dim=0)
        o = 0
        for p in projs:
            n = p.weight.shape[0]
            p.weight.data = self._qkv_w[o:o + n]
            o += n
        if self.q_proj.bias is not None:
            self._qkv_b = torch.cat([p.bias for p in projs], dim=0)
            o = 0
            for p in projs:
                n = p.bias.shape[0]
                p.bias.data = self._qkv_b[o:o + n]
                o += n

    def forward(self, hidden_states, positions, kv_cache, block_table, cu_seqlens,
                context_lens, max_seqlen, is_prefill, cos, sin, slot_mapping=None):
        """needle's ``Attention.forward``; ``slot_mapping`` (optional, not in
        needle's signature) is the forward's KV slot table from
        ``ops.slot_mapping``, built once and shared by all layers."""
        T = hidden_states.shape[0]
        H, KV, D = self.num_heads, self.num_kv_heads, self.head_dim
        # getattr: patch_needle() binds this method to needle's own Attention,
        # which has no fused q/k/v buffer
        qkv_w = getattr(self, "_qkv_w", None)
        if qkv_w is not None:
            # one GEMM; q/k/v are column slices of its [T, (H + 2 KV) * D] output
            qkv = dense(hidden_states, qkv_w, self._qkv_b)
            q = qkv[:, :H * D].view(T, H, D)
            k = qkv[:, H * D:(H + KV) * D].view(T, KV, D)
            v = qkv[:, (H + KV) * D:].view(T, KV, D)
        else:
            q = self.q_proj(hidden_states).view(T, H, D)
            k = self.k_proj(hidden_states).view(T, KV, D)
            v = self.v_proj(hidden_states).view(T, KV, D)
        if slot_mapping is not None and _aligned16(q, k, v, cos, sin):
            ops.rope_store_kvcache_slots(q, k, v, cos, sin, kv_cache, slot_mapping,
                                         write_k_back=is_prefill)
        elif is_prefill:
            ops.rope_store_kvcache(q, k, v, cos, sin, kv_cache, block_table, context_lens,
                                   cu_seqlens=cu_seqlens, write_k_back=True)
        else:
            ops.rope_store_kvcache(q, k, v, cos, sin, kv_cache, block_table, context_lens)
        if is_prefill and getattr(self, "prefill_with_context", False):
            # every new token attends over its whole context, cached prefix
            # included (K/V from the paged cache, just written above)
            attn = ops.prefill_attention_paged(q, kv_cache, block_table, context_lens,
                                               cu_seqlens, max_seqlen, self.scale)
        elif is_prefill:
            attn = ops.prefill_attention(q, k, v, cu_seqlens, max_seqlen, self.scale)
        else:
            plan = ops.decode_plan(T, H, KV, D, block_table.shape[1], kv_cache.shape[3],
                                   q.device)
            attn = ops.paged_decode(q, kv_cache, block_table, context_lens, self.scale,
                                    plan=plan)
        return self.o_proj(attn.view(T, H * D))
