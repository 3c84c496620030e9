"""Tensor-parallel linear layers, interface-compatible with needle's.

Mirrors ``needle/layers/linear.py:21-98``: ``ColumnParallelLinear`` holds
``weight[out/tp, in]`` (+ optional bias) and needs no communication;
``RowParallelLinear`` holds ``weight[out, in/tp]`` and all-reduces (SUM) its
output over the tensor-parallel group before adding the bias.  Every GEMM
goes through ``dense``: decode-size batches (at most 256 rows, bf16 / fp16)
of the LM head on this library's tcgen05 kernel, everything else on torch
(cuBLAS), which measures faster for the narrower projections.  The
all-reduce is NCCL through ``torch.distributed``, or, with a ``TPComm``
attached, the fused all-reduce + residual + RMSNorm kernel run by the
following ``RMSNorm``.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .. import ops

# "0": every GEMM stays on torch (diagnostics, A/B runs)
_LINEAR_TC = os.environ.get("NB_LINEAR_TC", "1") != "0"


def dense(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``F.linear(x, weight, bias)`` (into ``out`` when given): ``ops.linear``
    for decode-size batches where it beats the library GEMM
    (``ops.linear_preferred``), torch otherwise."""
    if _LINEAR_TC and ops.linear_preferred(x, weight) and (
            bias is None or (bias.dtype == x.dtype and bias.is_contiguous())):
        return ops.linear(x, weight, bias, out=out)
    if out is None:
        return F.linear(x, weight, bias)
    torch.mm(x, weight.t(), out=out)
    if bias is not None:
        out += bias
    return out


def tp_group():
    """The tensor-parallel process group: the whole world, as in needle
    (``needle/layers/linear.py:14-18``)."""
    if dist.is_available() and dist.is_initialized():
        return dist.group.WORLD
    return None


class ColumnParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 tp_size: int = 1, tp_rank: int = 0, gather_output: bool = False):
        super().__init__()
        assert out_features % tp_size == 0, (
            f"out_features {out_features} must be divisible by tp_size {tp_size}")
        self.in_features, self.out_features = in_features, out_features
        self.tp_size, self.tp_rank = tp_size, tp_rank
        self.gather_output = gather_output
        self.local_out = out_features // tp_size
        self.weight = nn.Parameter(torch.empty(self.local_out, in_features))
        self.bias = nn.Parameter(torch.zeros(self.local_out)) if bias else None
        nn.init.kaiming_uniform_(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out = dense(x, self.weight, self.bias)
        if self.gather_output and self.tp_size > 1:
            parts = [torch.empty_like(out) for _ in range(self.tp_size)]
            dist.all_gather(parts, out, group=tp_group())
            out = torch.cat(parts, dim=-1)
        return out


class RowParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 tp_size: int = 1, tp_rank: int = 0, reduce_output: bool = True):
        super().__init__()
        assert in_features % tp_size == 0
        self.in_features, self.out_features = in_features, out_features
        self.tp_size, self.tp_rank = tp_size, tp_rank
        self.reduce_output = reduce_output
        self.local_in = in_features // tp_size
        self.weight = nn.Parameter(torch.empty(out_features, self.local_in))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.kaiming_uniform_(self.weight)

    comm = None  # TPComm: defer the all-reduce to the next RMSNorm (fused kernel)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.comm is not None and self.comm.can_fuse(x.shape[0]) and x.dim() == 2:
            # partial sums into the peer-mapped buffer; the following RMSNorm
            # all-reduces them together with the residual add and the norm
            return dense(x, self.weight, out=self.comm.partial[:x.shape[0]])
        out = dense(x, self.weight)
        if self.reduce_output and self.tp_size > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=tp_group())
        if self.bias is not None:
            out = out + self.bias
        return out


def shard_for_rank(name: str, tensor: torch.Tensor, tp_size: int, tp_rank: int) -> torch.Tensor:
    """The slice of a full checkpoint tensor that rank ``tp_rank`` holds.

    Same rule as needle's loader (``needle/model/loader.py:37-43,116-127``):
    q/k/v/gate/up weights and q/k/v biases split along dim 0, o/down weights
    along dim 1, everything else replicated.
    """
    if tp_size == 1:
        return tensor
    col = ("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight",
           "up_proj.weight", "q_proj.bias", "k_proj.bias", "v_proj.bias")
    row = ("o_proj.weight", "down_proj.weight")
    dim: Optional[int] = 0 if name.endswith(col) else (1 if name.endswith(row) else None)
    if dim is None:
        return tensor
    n = tensor.shape[dim] // tp_size
    return tensor.narrow(dim, tp_rank * n, n).contiguous()
