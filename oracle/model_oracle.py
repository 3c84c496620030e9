"""CPU oracle for needle's model forward and greedy decode -- TEST INFRASTRUCTURE ONLY.

Restates the parts of needle that sit around the attention hot path and that
an end-to-end parity check needs: the decoder-layer composition of Llama and
Qwen2 (``needle/model/llama.py:48-140``, ``needle/model/qwen2.py:22-109``),
the input preparation of ``ModelRunner._prepare_inputs``
(``needle/model/runner.py:194-249``), greedy sampling
(``needle/model/sampler.py:27-28``) and the engine/scheduler loop for a batch
that fits in memory (``needle/backend/engine.py:110-134``,
``needle/backend/scheduler.py:49-134``, admission and decode block growth).

Like ``needle_oracle`` this is a checker: only tests, ``smoke()`` and the CPU
legs of ``bench.py`` may use it.  Its greedy tokens are pinned against tokens
produced by needle itself (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

from typing import Dict, List, Sequence as Seq

import torch
import torch.nn.functional as F

from . import needle_oracle as no


class OracleModel:
    """Functional Llama/Qwen2 forward over a needle-named state dict."""

    def __init__(self, cfg, state_dict: Dict[str, torch.Tensor], dtype=torch.float32):
        self.cfg = cfg
        self.dtype = dtype
        self.sd = {k: v.to(dtype) for k, v in state_dict.items()}
        if "lm_head.weight" not in self.sd:
            # needle/model/loader.py:138-143 ties lm_head to the embedding
            self.sd["lm_head.weight"] = self.sd["model.embed_tokens.weight"]
        cos, sin = no.rope_cache(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta)
        # model.to(dtype) casts the rope buffers (needle/model/runner.py:34)
        self.cos, self.sin = cos.to(dtype), sin.to(dtype)

    def new_kv_caches(self, num_blocks: int, block_size: int = 16) -> List[torch.Tensor]:
        c = self.cfg
        shape = (2, num_blocks, c.num_key_value_heads, block_size, c.head_dim)
        return [torch.zeros(shape, dtype=self.dtype) for _ in range(c.num_hidden_layers)]

    def forward(self, input_ids, positions, kv_caches, block_table, cu_seqlens,
                context_lens, is_prefill: bool) -> torch.Tensor:
        """Logits of the last token of every sequence, ``[num_seqs, vocab]``."""
        c, sd = self.cfg, self.sd
        H, kv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        eps = c.rms_norm_eps
        cos, sin = self.cos[positions], self.sin[positions]        # llama.py:99
        h = sd["model.embed_tokens.weight"][input_ids]              # llama.py:100
        T = h.shape[0]
        scale = no.default_scale(D)
        for i in range(c.num_hidden_layers):                        # llama.py:102-107
            p = f"model.layers.{i}."
            residual = h
            x = no.rms_norm(h, sd[p + "input_layernorm.weight"], eps)
            q = F.linear(x, sd[p + "self_attn.q_proj.weight"], sd.get(p + "self_attn.q_proj.bias"))
            k = F.linear(x, sd[p + "self_attn.k_proj.weight"], sd.get(p + "self_attn.k_proj.bias"))
            v = F.linear(x, sd[p + "self_attn.v_proj.weight"], sd.get(p + "self_attn.v_proj.bias"))
            q, k, v = q.view(T, H, D), k.view(T, kv, D), v.view(T, kv, D)
            q, k = no.apply_rope(q, k, cos, sin)                    # attention.py:88
            if is_prefill:                                          # attention.py:102-107
                no.write_kv(k, v, kv_caches[i], block_table, cu_seqlens, context_lens)
                a = no.prefill_attention(q, k, v, cu_seqlens, H, kv)
            else:                                                   # attention.py:140-159
                no.decode_write_kv(k, v, kv_caches[i], block_table, context_lens)
                a = no.decode_attention(q, kv_caches[i], block_table, context_lens,
                                        scale, H, kv, D)
            h = residual + F.linear(a.reshape(T, H * D), sd[p + "self_attn.o_proj.weight"])
            residual = h
            x = no.rms_norm(h, sd[p + "post_attention_layernorm.weight"], eps)
            m = F.linear(F.silu(F.linear(x, sd[p + "mlp.gate_proj.weight"]))
                         * F.linear(x, sd[p + "mlp.up_proj.weight"]),
                         sd[p + "mlp.down_proj.weight"])
            h = residual + m
        h = no.rms_norm(h, sd["model.norm.weight"], eps)
        last = h[(cu_seqlens[1:] - 1).long()] if is_prefill else h  # llama.py:134-138
        return F.linear(last, sd["lm_head.weight"])


def prepare_inputs(seqs: Seq[dict], block_tables: Dict[int, List[int]], num_gpu_blocks: int):
    """``ModelRunner._prepare_inputs`` (``needle/model/runner.py:194-249``).

    ``seqs`` are dicts with ``id``, ``tokens`` and ``generated``; a sequence
    with nothing generated feeds its whole prompt (context 0), otherwise only
    its last token (context = length - 1).  Block-table rows are padded with
    the last physical block (``:226-235``).
    """
    ids, pos, cu, ctx = [], [], [0], []
    for s in seqs:
        if s["generated"] == 0:
            toks, c = s["tokens"], 0
        else:
            toks, c = [s["tokens"][-1]], len(s["tokens"]) - 1
        ids.extend(toks)
        pos.extend(range(c, c + len(toks)))
        cu.append(cu[-1] + len(toks))
        ctx.append(c)
    maxb = max(len(block_tables[s["id"]]) for s in seqs)
    dummy = num_gpu_blocks - 1
    bt = [block_tables[s["id"]] + [dummy] * (maxb - len(block_tables[s["id"]])) for s in seqs]
    return dict(input_ids=torch.tensor(ids, dtype=torch.long),
                positions=torch.tensor(pos, dtype=torch.long),
                cu_seqlens=torch.tensor(cu, dtype=torch.int32),
                context_lens=torch.tensor(ctx, dtype=torch.int32),
                block_table=torch.tensor(bt, dtype=torch.int32))


def greedy_generate(model: OracleModel, prompts: List[List[int]], max_new_tokens: int,
                    num_gpu_blocks: int = 512, block_size: int = 16):
    """Greedy decode of all prompts as one continuous batch.

    Follows ``LLMEngine.step`` (``needle/backend/engine.py:110-134``) for a
    batch that the scheduler admits at once: step 1 prefills every prompt in
    one forward, every later step decodes one token per sequence; a sequence
    gets a new block when its length crosses a block boundary
    (``needle/backend/scheduler.py:111-118``).  Blocks come from a free list
    in ascending order like ``BlockAllocator`` (``block_allocator.py:10-30``).

    Returns ``(tokens [num_prompts][max_new_tokens], margins)`` where
    ``margins[step][seq]`` is the gap between the top-2 logits.
    """
    free = list(range(num_gpu_blocks))
    caches = model.new_kv_caches(num_gpu_blocks, block_size)
    seqs, tables = [], {}
    for i, p in enumerate(prompts):
        nb = (len(p) + block_size - 1) // block_size
        tables[i] = [free.pop(0) for _ in range(nb)]
        seqs.append(dict(id=i, tokens=list(p), generated=0))
    out = [[] for _ in prompts]
    margins = []
    with torch.no_grad():
        for step in range(max_new_tokens):
            for s in seqs:  # decode block growth before the forward
                need = (len(s["tokens"]) + block_size - 1) // block_size
                if s["generated"] > 0 and need > len(tables[s["id"]]):
                    tables[s["id"]].append(free.pop(0))
            inp = prepare_inputs(seqs, tables, num_gpu_blocks)
            logits = model.forward(inp["input_ids"], inp["positions"], caches,
                                   inp["block_table"], inp["cu_seqlens"],
                                   inp["context_lens"], is_prefill=(step == 0))
            top2 = logits.float().topk(2, dim=-1).values
            margins.append((top2[:, 0] - top2[:, 1]).tolist())
            for r, s in enumerate(seqs):
                t = int(logits[r].argmax())                         # sampler.py:27-28
                s["tokens"].append(t)
                s["generated"] += 1
                out[s["id"]].append(t)
    return out, margins
