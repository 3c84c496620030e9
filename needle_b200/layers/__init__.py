"""Mirrors of needle's ``needle/layers`` modules on the B200 kernels."""
from .linear import ColumnParallelLinear, RowParallelLinear
from .attention import Attention
from .norm import RMSNorm
from .rope import RotaryEmbedding

__all__ = ["ColumnParallelLinear", "RowParallelLinear", "Attention", "RMSNorm",
           "RotaryEmbedding"]
