"""RMSNorm, interface-compatible with needle's, with an optional fused residual.

``RMSNorm.forward(x)`` is needle's ``needle/layers/norm.py:14-17``;
``RMSNorm.forward(x, residual)`` additionally performs the decoder layer's
residual add (``needle/model/llama.py:67,72``) in the same kernel and returns
``(normed, residual + x)``.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import ops


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None):
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps)
        return ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
