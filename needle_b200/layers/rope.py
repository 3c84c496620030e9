"""RoPE tables, interface-compatible with needle's ``RotaryEmbedding``.

Mirrors ``needle/layers/rope.py:10-27``.  The tables are computed on the CPU
in fp32 exactly as needle computes them (needle builds the model on the CPU
and then moves it, ``needle/model/runner.py:33-34``), so after the move and
the cast to the model dtype they are bit-identical to needle's.  The
rotation itself runs in the fused ``rope_store_kvcache`` kernel.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, max_seq_len: int, base: float = 10000.0):
        super().__init__()
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, device="cpu").float() / head_dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        t = torch.arange(max_seq_len, device="cpu").float()
        freqs = torch.outer(t, inv_freq)
        emb = torch.cat([freqs, freqs], dim=-1)
        self.register_buffer("cos_cached", emb.cos(), persistent=False)
        self.register_buffer("sin_cached", emb.sin(), persistent=False)

    def get_cos_sin(self, positions: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.cos_cached[positions], self.sin_cached[positions]
