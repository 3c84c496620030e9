"""Llama decoder on the B200 attention path (mirror of ``needle/model/llama.py``).

Module tree and parameter names are needle's, so needle state dicts (and the
synthetic ones from ``needle_b200.synth``) load unchanged.  The layer
arithmetic is the same sequence as ``needle/model/llama.py:61-72`` with the
residual adds fused into the following RMSNorm: the layer carries
``residual`` forward instead of returning ``residual + mlp_out``, and the
next layer's input norm (or the final norm) performs that add.  The rounding
points are unchanged: the sum is rounded to the model dtype before it is
normalised, exactly as needle's separate ``residual + x`` then ``norm(.)``.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..layers.attention import Attention
from ..layers.linear import ColumnParallelLinear, RowParallelLinear, dense
from ..layers.norm import RMSNorm
from ..layers.rope import RotaryEmbedding


class LlamaMLP(nn.Module):
    """SwiGLU: ``down(silu(gate(x)) * up(x))`` (``needle/model/llama.py:18-37``)."""

    def __init__(self, config, tp_size: int = 1, tp_rank: int = 0):
        super().__init__()
        h, i = config.hidden_size, config.intermediate_size
        self.gate_proj = ColumnParallelLinear(h, i, tp_size=tp_size, tp_rank=tp_rank)
        self.up_proj = ColumnParallelLinear(h, i, tp_size=tp_size, tp_rank=tp_rank)
        self.down_proj = RowParallelLinear(i, h, tp_size=tp_size, tp_rank=tp_rank)
        self._gu_w = None

    @torch.no_grad()
    def fuse_gate_up(self) -> None:
        """One buffer for the gate and up weights (the parameters become
        views into it): one GEMM, then the fused SwiGLU kernel."""
        self._gu_w = torch.cat([self.gate_proj.weight, self.up_proj.weight], dim=0)
        n = self.gate_proj.weight.shape[0]
        self.gate_proj.weight.data = self._gu_w[:n]
        self.up_proj.weight.data = self._gu_w[n:]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._gu_w is not None:
            return self.down_proj(ops.silu_mul(dense(x, self._gu_w)))
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class LlamaDecoderLayer(nn.Module):
    attention_cls = Attention
    qkv_bias = False

    def __init__(self, config, layer_idx: int, tp_size: int = 1, tp_rank: int = 0):
        super().__init__()
        self.self_attn = Attention(config, layer_idx, tp_size=tp_size, tp_rank=tp_rank,
                                   qkv_bias=self.qkv_bias)
        self.mlp = LlamaMLP(config, tp_size=tp_size, tp_rank=tp_rank)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, hidden_states, residual, positions, kv_cache, block_table, cu_seqlens,
                context_lens, max_seqlen, is_prefill, cos, sin, slot_mapping=None):
        """``residual`` is None for the first layer; otherwise ``hidden_states``
        is the previous layer's MLP output still to be added to it.
        ``slot_mapping``: the forward's KV slot table (built once for all
        layers), or None."""
        if residual is None:
            residual = hidden_states
            x = self.input_layernorm(hidden_states)
        else:
            x, residual = self.input_layernorm(hidden_states, residual)
        x = self.self_attn(x, positions, kv_cache, block_table, cu_seqlens, context_lens,
                           max_seqlen, is_prefill, cos, sin, slot_mapping=slot_mapping)
        x, residual = self.post_attention_layernorm(x, residual)
        return self.mlp(x), residual


class LlamaModel(nn.Module):
    layer_cls = LlamaDecoderLayer

    def __init__(self, config, tp_size: int = 1, tp_rank: int = 0):
        super().__init__()
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([self.layer_cls(config, i, tp_size=tp_size, tp_rank=tp_rank)
                                     for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.rotary_emb = RotaryEmbedding(config.head_dim, config.max_position_embeddings,
                                          config.rope_theta)

    def forward(self, input_ids, positions, kv_caches, block_table, cu_seqlens, context_lens,
                max_seqlen, is_prefill):
        cos, sin = self.rotary_emb.get_cos_sin(positions)
        h = self.embed_tokens(input_ids)
        # every layer writes its new K/V rows to the same cache slots: resolve
        # them once (needle recomputes them per layer, attention.py:140-154,
        # 204-246)
        c0 = kv_caches[0]
        slots = ops.slot_mapping(block_table, context_lens, c0.shape[1], c0.shape[3],
                                 cu_seqlens=cu_seqlens if is_prefill else None,
                                 num_tokens=input_ids.shape[0])
        residual = None
        for i, layer in enumerate(self.layers):
            h, residual = layer(h, residual, positions, kv_caches[i], block_table, cu_seqlens,
                                context_lens, max_seqlen, is_prefill, cos, sin,
                                slot_mapping=slots)
        h, _ = self.norm(h, residual)
        return h


class LlamaForCausalLM(nn.Module):
    model_cls = LlamaModel

    def __init__(self, config, tp_size: int = 1, tp_rank: int = 0):
        super().__init__()
        self.config = config
        self.model = self.model_cls(config, tp_size=tp_size, tp_rank=tp_rank)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)

    def fuse_projections(self) -> None:
        """q/k/v and gate/up weights into shared buffers (one GEMM each)."""
        for layer in self.model.layers:
            layer.self_attn.fuse_qkv()
            layer.mlp.fuse_gate_up()

    def forward(self, input_ids, positions, kv_caches, block_table, cu_seqlens, context_lens,
                max_seqlen, is_prefill):
        """Logits of the last token of every sequence, ``[num_seqs, vocab]``
        (``needle/model/llama.py:118-140``)."""
        hidden = self.model(input_ids, positions, kv_caches, block_table, cu_seqlens,
                            context_lens, max_seqlen, is_prefill)
        if is_prefill:
            hidden = hidden[(cu_seqlens[1:] - 1).long()]
        return dense(hidden, self.lm_head.weight, self.lm_head.bias)
