"""RMSNorm, interface-compatible with needle's, with an optional fused residual.

``RMSNorm.forward(x)`` is needle's ``needle/layers/norm.py:14-17``;
``RMSNorm.forward(x, residual)`` additionally performs the decoder layer's
residual add (``needle/model/llama.py:67,72``) in the same kernel and returns
``(normed, residual + x)``.  Under tensor parallelism with a ``TPComm``
attached, ``x`` can be a row-parallel partial sum: the norm then also performs
its all-reduce (``needle/layers/linear.py:92-98``) in the same kernel.
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

    comm = None  # TPComm: x may be a row-parallel partial sum still to be all-reduced

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None):
        # getattr: patch_needle() binds this method to needle's own RMSNorm
        comm = getattr(self, "comm", None)
        if comm is not None and comm.is_partial(x):
            if residual is None:
                raise RuntimeError("the fused TP all-reduce needs the residual")
            return comm.allreduce_add_rmsnorm(x.shape[0], residual, self.weight, self.eps)
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps)
        return ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
