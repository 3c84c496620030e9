"""Seeded synthetic weights and workloads (no checkpoints, no datasets).

Weights use the parameter names of needle's ``state_dict`` so that the same
dictionary loads into needle itself (``needle/model/loader.py:100-134``) and
into ``needle_b200.model``.  Every tensor is drawn from its own CPU
``torch.Generator`` seeded from ``(seed, name)``, so a tensor's values do not
depend on which other tensors were generated or in what order, and are the
same on every machine running the same torch build.

Distributions: linear weights ``U(-sqrt(6/fan_in), +sqrt(6/fan_in))`` (the
bound of needle's ``kaiming_uniform_`` init, ``needle/layers/linear.py:51,90``),
embeddings and an untied ``lm_head`` ``N(0, 1)`` (``nn.Embedding`` default),
QKV biases ``U(-0.1, 0.1)`` and norm weights ``U(0.5, 1.5)`` (non-trivial so
that bias adds and weight multiplies are exercised).
"""
from __future__ import annotations

import math
import zlib
from typing import Dict, Iterator, Optional, Tuple

import torch

from .model.config import ModelConfig


def _gen(seed: int, name: str, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF)
    return g


def weight_shapes(cfg: ModelConfig) -> Iterator[Tuple[str, Tuple[int, ...], str]]:
    """(name, full unsharded shape, kind) for every parameter of the model."""
    H, D, kv = cfg.num_attention_heads, cfg.head_dim, cfg.num_key_value_heads
    hid, inter = cfg.hidden_size, cfg.intermediate_size
    yield "model.embed_tokens.weight", (cfg.vocab_size, hid), "embed"
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        yield p + "self_attn.q_proj.weight", (H * D, hid), "linear"
        yield p + "self_attn.k_proj.weight", (kv * D, hid), "linear"
        yield p + "self_attn.v_proj.weight", (kv * D, hid), "linear"
        if cfg.model_type == "qwen2":
            yield p + "self_attn.q_proj.bias", (H * D,), "bias"
            yield p + "self_attn.k_proj.bias", (kv * D,), "bias"
            yield p + "self_attn.v_proj.bias", (kv * D,), "bias"
        yield p + "self_attn.o_proj.weight", (hid, H * D), "linear"
        yield p + "mlp.gate_proj.weight", (inter, hid), "linear"
        yield p + "mlp.up_proj.weight", (inter, hid), "linear"
        yield p + "mlp.down_proj.weight", (hid, inter), "linear"
        yield p + "input_layernorm.weight", (hid,), "norm"
        yield p + "post_attention_layernorm.weight", (hid,), "norm"
    yield "model.norm.weight", (hid,), "norm"
    if not cfg.tie_word_embeddings:
        yield "lm_head.weight", (cfg.vocab_size, hid), "embed"


def synth_tensor(name: str, shape, kind: str, seed: int = 0,
                 device="cpu", dtype=torch.float32) -> torch.Tensor:
    """One synthetic parameter, generated in fp32 then cast to ``dtype``."""
    g = _gen(seed, name, device)
    t = torch.empty(shape, dtype=torch.float32, device=device)
    if kind == "embed":
        t.normal_(0.0, 1.0, generator=g)
    elif kind == "linear":
        b = math.sqrt(6.0 / shape[1])
        t.uniform_(-b, b, generator=g)
    elif kind == "bias":
        t.uniform_(-0.1, 0.1, generator=g)
    elif kind == "norm":
        t.uniform_(0.5, 1.5, generator=g)
    else:
        raise ValueError(kind)
    return t.to(dtype)


def synth_state_dict(cfg: ModelConfig, seed: int = 0, dtype=torch.float32,
                     device="cpu") -> Dict[str, torch.Tensor]:
    """The full (unsharded) synthetic state dict of ``cfg``."""
    return {n: synth_tensor(n, s, k, seed, device, dtype) for n, s, k in weight_shapes(cfg)}


def synth_prompts(num: int, lo: int, hi: int, vocab: int, seed: int = 0):
    """``num`` prompts with lengths uniform in ``[lo, hi]`` and ids uniform in
    ``[0, vocab)`` (``hi == lo`` gives fixed-length prompts)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (num,), generator=g).tolist()
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


def decode_op_workload(batch: int = 64, num_heads: int = 32, num_kv_heads: int = 8,
                       head_dim: int = 128, block_size: int = 16, pool_blocks: int = 20000,
                       ctx_lo: int = 512, ctx_hi: int = 4096, seed: int = 0,
                       dtype=torch.bfloat16, device="cpu", cache: Optional[torch.Tensor] = None):
    """The isolated paged-decode workload (Q/K/V ~ N(0,1)).

    ``seq_len ~ U[ctx_lo, ctx_hi]`` per sequence; ``context_lens = seq_len - 1``
    in needle's convention (tokens already cached; the decode attends over
    ``context_lens + 1``); the block table is a random permutation of the
    ``pool_blocks``-block pool reshaped to ``[batch, max_blocks]``.
    Returns a dict of CPU (or ``device``) tensors.
    """
    g = torch.Generator().manual_seed(seed)
    seq_len = torch.randint(ctx_lo, ctx_hi + 1, (batch,), generator=g)
    maxb = (int(seq_len.max()) + block_size - 1) // block_size
    if batch * maxb > pool_blocks:
        raise ValueError("block pool too small for the requested batch")
    perm = torch.randperm(pool_blocks, generator=g)[: batch * maxb]
    block_table = perm.view(batch, maxb).to(torch.int32)
    q = torch.randn(batch, num_heads, head_dim, generator=g).to(dtype)
    k_new = torch.randn(batch, num_kv_heads, head_dim, generator=g).to(dtype)
    v_new = torch.randn(batch, num_kv_heads, head_dim, generator=g).to(dtype)
    if cache is None:
        # The pool is filled on the target device with that device's own
        # generator (seeded from ``seed``), in chunks to bound the fp32
        # temporary.
        cache = torch.empty(2, pool_blocks, num_kv_heads, block_size, head_dim,
                            dtype=dtype, device=device)
        gd = torch.Generator(device=device).manual_seed(seed + 1)
        flat = cache.view(-1)
        step = 1 << 26
        for s in range(0, flat.numel(), step):
            n = min(step, flat.numel() - s)
            flat[s:s + n] = torch.randn(n, generator=gd, device=device).to(dtype)
    return dict(q=q.to(device), k_new=k_new.to(device), v_new=v_new.to(device),
                kv_cache=cache, block_table=block_table.to(device),
                context_lens=(seq_len - 1).to(torch.int32).to(device),
                seq_len=seq_len, scale=1.0 / math.sqrt(head_dim))
