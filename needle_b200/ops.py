"""Torch-facing wrappers over the C ABI (``include/needle_b200.h``).

Each function takes CUDA tensors in needle's layouts, checks dtypes and
shapes, and launches on torch's current stream.  There is no CPU or
library fallback: a CPU tensor, an unsupported dtype or a missing library
raises.  Nothing here synchronises the device.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib as L

_DT = {torch.float32: L.NB_DTYPE_F32, torch.float16: L.NB_DTYPE_F16,
       torch.bfloat16: L.NB_DTYPE_BF16}


def _dtype(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"needle_b200: unsupported dtype {t.dtype}") from None


def _cuda(*ts):
    """All tensors on one CUDA device, which is the current device (the
    kernels launch there; a pointer into another GPU's memory must never
    reach them)."""
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("needle_b200 ops take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
            if dev.index != torch.cuda.current_device():
                raise ValueError(f"tensors are on {dev} but the current device is "
                                 f"cuda:{torch.cuda.current_device()}")
        elif t.device != dev:
            raise ValueError(f"tensors on different devices ({dev} and {t.device})")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _rows(t: torch.Tensor, name: str) -> int:
    """Row stride of a token-major [T, heads, D] (or [T, heads*D]) tensor whose
    heads are dense within a row."""
    if t.dim() == 3:
        if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
            raise ValueError(f"{name}: heads must be dense within a token row")
    elif t.dim() == 2:
        if t.stride(1) != 1:
            raise ValueError(f"{name}: last dim must be contiguous")
    else:
        raise ValueError(f"{name}: expected a [T, heads, D] tensor")
    return t.stride(0)


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32 (got {t.dtype})")
    return t


def _cache_dims(kv_cache: torch.Tensor):
    if kv_cache.dim() != 5 or kv_cache.shape[0] != 2 or not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [2, num_blocks, kv_heads, block_size, D] tensor")
    _, n, kvh, bs, d = kv_cache.shape
    return n, kvh, bs, d


def _bt(block_table: torch.Tensor):
    _i32(block_table, "block_table")
    if block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be [num_seqs, max_blocks] with unit column stride")
    return block_table.stride(0), block_table.shape[1]


# --------------------------------------------------------------------------
# KV cache writes and RoPE
# --------------------------------------------------------------------------

def store_kvcache(k: torch.Tensor, v: torch.Tensor, kv_cache: torch.Tensor,
                  block_table: torch.Tensor, context_lens: torch.Tensor,
                  cu_seqlens: Optional[torch.Tensor] = None) -> None:
    """Scatter ``k``/``v`` ``[T, kv_heads, D]`` into the paged cache in place.

    ``cu_seqlens=None`` is the decode case (one token per sequence).
    """
    _cuda(k, v, kv_cache, block_table, context_lens, cu_seqlens)
    n, kvh, bs, d = _cache_dims(kv_cache)
    bts, maxb = _bt(block_table)
    _i32(context_lens, "context_lens")
    if cu_seqlens is not None:
        _i32(cu_seqlens, "cu_seqlens")
    dt = _dtype(kv_cache)
    if k.dtype != kv_cache.dtype or v.dtype != kv_cache.dtype:
        raise TypeError("k/v dtype must match the cache")
    L.check(L.lib().nb_store_kvcache(
        k.data_ptr(), _rows(k, "k"), v.data_ptr(), _rows(v, "v"), kv_cache.data_ptr(),
        n, kvh, bs, d, block_table.data_ptr(), bts, maxb,
        cu_seqlens.data_ptr() if cu_seqlens is not None else None,
        context_lens.data_ptr(), context_lens.shape[0], k.shape[0], dt, _stream(k)))


def slot_mapping(block_table: torch.Tensor, context_lens: torch.Tensor, num_blocks: int,
                 block_size: int, cu_seqlens: Optional[torch.Tensor] = None,
                 num_tokens: Optional[int] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The forward's slot table ``[T]`` int32 (``block * block_size + offset``
    of every new token, -1 = not written), built once and read by every
    layer's ``store_kvcache_slots`` / ``rope_store_kvcache_slots``.
    ``cu_seqlens=None`` is the decode case (one token per sequence)."""
    _cuda(block_table, context_lens, cu_seqlens, out)
    bts, maxb = _bt(block_table)
    _i32(context_lens, "context_lens")
    B = context_lens.shape[0]
    if cu_seqlens is not None:
        _i32(cu_seqlens, "cu_seqlens")
        if num_tokens is None:
            raise ValueError("num_tokens is required with cu_seqlens (no device read)")
    T = B if cu_seqlens is None else int(num_tokens)
    if out is None:
        out = torch.empty(T, dtype=torch.int32, device=context_lens.device)
    elif out.dtype != torch.int32 or out.numel() < T or not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 tensor of at least T elements")
    L.check(L.lib().nb_slot_mapping(
        block_table.data_ptr(), bts, maxb,
        cu_seqlens.data_ptr() if cu_seqlens is not None else None, context_lens.data_ptr(), B,
        T, block_size, num_blocks, out.data_ptr(), _stream(context_lens)))
    return out[:T]


def store_kvcache_slots(k: torch.Tensor, v: torch.Tensor, kv_cache: torch.Tensor,
                        slots: torch.Tensor) -> None:
    """``store_kvcache`` with positions from a slot table (``slot_mapping``)."""
    _cuda(k, v, kv_cache, slots)
    n, kvh, bs, d = _cache_dims(kv_cache)
    _i32(slots, "slots")
    if k.dtype != kv_cache.dtype or v.dtype != kv_cache.dtype:
        raise TypeError("k/v dtype must match the cache")
    if slots.shape[0] < k.shape[0]:
        raise ValueError("fewer slots than tokens")
    L.check(L.lib().nb_store_kvcache_slots(
        k.data_ptr(), _rows(k, "k"), v.data_ptr(), _rows(v, "v"), kv_cache.data_ptr(),
        n, kvh, bs, d, slots.data_ptr(), k.shape[0], _dtype(kv_cache), _stream(k)))


def rope_store_kvcache_slots(q, k, v, cos, sin, kv_cache, slots,
                             write_k_back: bool = False) -> None:
    """``rope_store_kvcache`` with positions from a slot table."""
    _cuda(q, k, v, cos, sin, kv_cache, slots)
    n, kvh, bs, d = _cache_dims(kv_cache)
    _i32(slots, "slots")
    for t in (q, k, v, cos, sin):
        if t.dtype != kv_cache.dtype:
            raise TypeError("q/k/v/cos/sin dtype must match the cache")
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
        raise ValueError("cos/sin must share a row stride with unit column stride")
    if slots.shape[0] < q.shape[0]:
        raise ValueError("fewer slots than tokens")
    L.check(L.lib().nb_rope_store_kvcache_slots(
        q.data_ptr(), _rows(q, "q"), q.shape[1], k.data_ptr(), _rows(k, "k"),
        v.data_ptr(), _rows(v, "v"), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
        kv_cache.data_ptr(), n, kvh, bs, d, slots.data_ptr(), q.shape[0],
        int(bool(write_k_back)), _dtype(kv_cache), _stream(q)))


def rope_(q: torch.Tensor, k: Optional[torch.Tensor], cos: torch.Tensor,
          sin: torch.Tensor) -> None:
    """In-place NeoX RoPE of ``q [T, Hq, D]`` and ``k [T, Hkv, D]``."""
    _cuda(q, k, cos, sin)
    dt = _dtype(q)
    if cos.dtype != q.dtype or sin.dtype != q.dtype:
        raise TypeError("cos/sin dtype must match q")
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
        raise ValueError("cos/sin must share a row stride with unit column stride")
    T, hq, d = q.shape
    L.check(L.lib().nb_rope(
        q.data_ptr(), _rows(q, "q"), hq,
        k.data_ptr() if k is not None else None, _rows(k, "k") if k is not None else 0,
        k.shape[1] if k is not None else 0,
        cos.data_ptr(), sin.data_ptr(), cos.stride(0), T, d, dt, _stream(q)))


def rope_store_kvcache(q, k, v, cos, sin, kv_cache, block_table, context_lens,
                       cu_seqlens=None, write_k_back: bool = False) -> None:
    """RoPE on ``q`` (in place) and ``k``, then K/V into the cache, one launch."""
    _cuda(q, k, v, cos, sin, kv_cache, block_table, context_lens, cu_seqlens)
    n, kvh, bs, d = _cache_dims(kv_cache)
    bts, maxb = _bt(block_table)
    _i32(context_lens, "context_lens")
    dt = _dtype(kv_cache)
    for t in (q, k, v, cos, sin):
        if t.dtype != kv_cache.dtype:
            raise TypeError("q/k/v/cos/sin dtype must match the cache")
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
        raise ValueError("cos/sin must share a row stride with unit column stride")
    L.check(L.lib().nb_rope_store_kvcache(
        q.data_ptr(), _rows(q, "q"), q.shape[1], k.data_ptr(), _rows(k, "k"),
        v.data_ptr(), _rows(v, "v"), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
        kv_cache.data_ptr(), n, kvh, bs, d, block_table.data_ptr(), bts, maxb,
        cu_seqlens.data_ptr() if cu_seqlens is not None else None, context_lens.data_ptr(),
        context_lens.shape[0], q.shape[0], int(bool(write_k_back)), dt, _stream(q)))


# --------------------------------------------------------------------------
# Paged decode
# --------------------------------------------------------------------------

class DecodePlan:
    """Split-K plan plus workspace for one decode step.

    Built once per step from host-known shapes (batch, KV heads, block-table
    width) and reused by every layer of the step: the workspace is consumed
    by each layer's merge before the next layer's decode runs on the same
    stream.
    """

    def __init__(self, num_seqs: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 max_blocks: int, block_size: int, device, pages_per_split: Optional[int] = None):
        lib = L.lib()
        if pages_per_split is None:
            import ctypes
            pps, ms = ctypes.c_int(0), ctypes.c_int(0)
            L.check(lib.nb_paged_decode_plan(num_seqs, num_kv_heads, max_blocks, block_size,
                                             ctypes.byref(pps), ctypes.byref(ms)))
            pages_per_split = pps.value
        self.pages_per_split = int(pages_per_split)
        self.max_splits = -(-max_blocks // self.pages_per_split)
        nbytes = lib.nb_paged_decode_workspace_size(num_seqs, num_q_heads, head_dim,
                                                    self.max_splits)
        self.workspace = (torch.empty(nbytes, dtype=torch.uint8, device=device)
                          if nbytes else None)
        self.key = (num_seqs, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size)


_PLANS: "dict" = {}


def decode_plan(num_seqs: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                max_blocks: int, block_size: int, device) -> DecodePlan:
    """A cached ``DecodePlan`` for this shape: every layer of a decode step (and
    every step with the same batch shape) shares one plan and workspace.

    The cache is cleared when it grows past 64 shapes; eager launches are
    unaffected (a freed workspace is only reused by later work on the same
    stream), but a CUDA graph that captured a plan's workspace must keep the
    plan alive itself (``ModelRunner`` does)."""
    key = (num_seqs, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, str(device))
    p = _PLANS.get(key)
    if p is None:
        if len(_PLANS) > 64:
            _PLANS.clear()
        p = _PLANS[key] = DecodePlan(num_seqs, num_q_heads, num_kv_heads, head_dim, max_blocks,
                                     block_size, device)
    return p


def paged_decode(q: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                 context_lens: torch.Tensor, scale: float, out: Optional[torch.Tensor] = None,
                 plan: Optional[DecodePlan] = None) -> torch.Tensor:
    """Decode attention of ``q [B, Hq, D]`` over ``context_lens + 1`` cached
    tokens per sequence.  Returns ``out [B, Hq, D]``."""
    _cuda(q, kv_cache, block_table, context_lens, out)
    n, kvh, bs, d = _cache_dims(kv_cache)
    bts, maxb = _bt(block_table)
    _i32(context_lens, "context_lens")
    if q.dtype != kv_cache.dtype:
        raise TypeError("q dtype must match the cache")
    B, hq, qd = q.shape
    if qd != d or q.stride(2) != 1:
        raise ValueError("q must be [B, Hq, D] with unit last stride")
    if out is None:
        out = torch.empty((B, hq, d), dtype=q.dtype, device=q.device)
    if B == 0:
        return out
    if plan is None or plan.key != (B, hq, kvh, d, maxb, bs):
        plan = DecodePlan(B, hq, kvh, d, maxb, bs, q.device)
    ws = plan.workspace
    L.check(L.lib().nb_paged_decode(
        q.data_ptr(), q.stride(0), q.stride(1), kv_cache.data_ptr(), n, kvh, bs, d, hq,
        block_table.data_ptr(), bts, maxb, context_lens.data_ptr(), B, float(scale),
        out.data_ptr(), out.stride(0), out.stride(1),
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        plan.pages_per_split, _dtype(q), _stream(q)))
    return out


# --------------------------------------------------------------------------
# Prefill
# --------------------------------------------------------------------------

def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      cu_seqlens: torch.Tensor, max_seqlen: int, scale: Optional[float] = None,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal attention of each sequence's new tokens; ``[T, Hq, D]`` out."""
    _cuda(q, k, v, cu_seqlens, out)
    _i32(cu_seqlens, "cu_seqlens")
    T, hq, d = q.shape
    hk = k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((T, hq, d), dtype=q.dtype, device=q.device)
    L.check(L.lib().nb_prefill_attention(
        q.data_ptr(), _rows(q, "q"), k.data_ptr(), _rows(k, "k"), v.data_ptr(), _rows(v, "v"),
        hq, hk, d, cu_seqlens.data_ptr(), cu_seqlens.shape[0] - 1, T, int(max_seqlen),
        float(scale), out.data_ptr(), _rows(out, "out"), _dtype(q), _stream(q)))
    return out


def prefill_attention_paged(q: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                            context_lens: torch.Tensor, cu_seqlens: torch.Tensor,
                            max_seqlen: int, scale: Optional[float] = None,
                            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal attention of each sequence's new tokens over its whole context
    (``context_lens[s]`` cached tokens + the new ones), K/V read from the
    paged cache; the new tokens' K/V must already be in the cache.
    ``[T, Hq, D]`` out; bf16 / fp16, head_dim 64 or 128."""
    _cuda(q, kv_cache, block_table, context_lens, cu_seqlens, out)
    _i32(cu_seqlens, "cu_seqlens")
    _i32(context_lens, "context_lens")
    N, kvh, bs, d = _cache_dims(kv_cache)
    if bs != 16:
        raise ValueError("paged prefill takes 16-token blocks")
    bts, maxb = _bt(block_table)
    T, hq, dq = q.shape
    if dq != d:
        raise ValueError(f"q head_dim {dq} != cache head_dim {d}")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((T, hq, d), dtype=q.dtype, device=q.device)
    L.check(L.lib().nb_prefill_attention_paged(
        q.data_ptr(), _rows(q, "q"), kv_cache.data_ptr(), N, kvh, block_table.data_ptr(), bts, maxb,
        context_lens.data_ptr(), hq, d, cu_seqlens.data_ptr(), cu_seqlens.shape[0] - 1, T,
        int(max_seqlen), float(scale), out.data_ptr(), _rows(out, "out"), _dtype(q),
        _stream(q)))
    return out


# --------------------------------------------------------------------------
# RMSNorm
# --------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _cuda(x, weight, out)
    if x.stride(-1) != 1 or x.dim() != 2:
        raise ValueError("x must be [T, hidden] with unit last stride")
    if weight.dtype != x.dtype or not weight.is_contiguous():
        raise TypeError("weight must be contiguous with x's dtype")
    if out is None:
        out = torch.empty_like(x)
    T, hid = x.shape
    L.check(L.lib().nb_rmsnorm(x.data_ptr(), x.stride(0), weight.data_ptr(), out.data_ptr(),
                               out.stride(0), T, hid, float(eps), _dtype(x), _stream(x)))
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                      out: Optional[torch.Tensor] = None,
                      residual_out: Optional[torch.Tensor] = None
                      ) -> Tuple[torch.Tensor, torch.Tensor]:
    """``h = residual + x``; returns ``(rmsnorm(h), h)``."""
    _cuda(x, residual, weight, out, residual_out)
    for t in (x, residual):
        if t.stride(-1) != 1 or t.dim() != 2:
            raise ValueError("x/residual must be [T, hidden] with unit last stride")
    if residual.dtype != x.dtype or weight.dtype != x.dtype:
        raise TypeError("dtype mismatch")
    if out is None:
        out = torch.empty_like(x)
    if residual_out is None:
        residual_out = torch.empty_like(residual)
    T, hid = x.shape
    L.check(L.lib().nb_fused_add_rmsnorm(
        x.data_ptr(), x.stride(0), residual.data_ptr(), residual.stride(0), weight.data_ptr(),
        out.data_ptr(), out.stride(0), residual_out.data_ptr(), residual_out.stride(0),
        T, hid, float(eps), _dtype(x), _stream(x)))
    return out, residual_out


def silu_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(gate_up[:, :I]) * gate_up[:, I:]`` for a fused ``[T, 2I]`` input."""
    _cuda(gate_up, out)
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.shape[1] % 2:
        raise ValueError("gate_up must be [T, 2I] with unit column stride")
    T, two_i = gate_up.shape
    inter = two_i // 2
    if out is None:
        out = torch.empty((T, inter), dtype=gate_up.dtype, device=gate_up.device)
    L.check(L.lib().nb_silu_mul(gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(),
                                out.stride(0), T, inter, _dtype(gate_up), _stream(gate_up)))
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ weight.T (+ bias)`` for a decode-size batch (at most 256 rows of
    bf16 / fp16; rows of ``x`` and ``weight`` 16-byte aligned), on the
    tcgen05 kernel ``nb_linear``.  ``out`` may be a row-strided view."""
    _cuda(x, weight, bias, out)
    if x.dim() != 2 or weight.dim() != 2 or x.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("linear: x [M, K] and weight [N, K] with unit column stride")
    M, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] != K or weight.dtype != x.dtype:
        raise ValueError(f"linear: weight {tuple(weight.shape)} {weight.dtype} does not match "
                         f"x {tuple(x.shape)} {x.dtype}")
    if bias is not None and (bias.shape != (N,) or bias.dtype != x.dtype or
                             (N > 1 and bias.stride(0) != 1)):
        raise ValueError("linear: bias must be a contiguous [N] tensor of x's dtype")
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    elif out.shape != (M, N) or out.dtype != x.dtype or out.stride(1) != 1:
        raise ValueError(f"linear: out must be [{M}, {N}] {x.dtype} with unit column stride")
    L.check(L.lib().nb_linear(x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0),
                              bias.data_ptr() if bias is not None else None, out.data_ptr(),
                              out.stride(0), M, N, K, _dtype(x), _stream(x)))
    return out


def linear_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether ``linear`` takes this GEMM (the shape checks of nb_linear)."""
    return (x.is_cuda and x.dim() == 2 and 0 < x.shape[0] <= 256
            and x.dtype in (torch.bfloat16, torch.float16) and weight.dtype == x.dtype
            and weight.dim() == 2 and x.stride(1) == 1 and weight.stride(1) == 1
            and x.shape[1] % 8 == 0 and x.stride(0) % 8 == 0 and weight.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0)


_SMS = {}


def linear_preferred(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether ``linear`` is the faster choice for this GEMM on this GPU:
    supported, and at least three 256-row weight tiles per SM (an LM head:
    128256 x 4096 measured 266 us against cuBLAS's 278 us at 256 rows).
    Narrower projections measure faster on cuBLAS (gate/up 28672 x 4096:
    79 vs 66 us; qkv, o_proj, down: 2-4x slower)."""
    if not linear_supported(x, weight):
        return False
    dev = x.device.index
    if dev not in _SMS:
        _SMS[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    return (weight.shape[0] + 255) // 256 >= 3 * _SMS[dev]


def swap_kv_blocks(src_caches, dst_caches, pairs: torch.Tensor) -> None:
    """Copy blocks ``pairs[i, 0]`` of every layer's ``src_caches`` to blocks
    ``pairs[i, 1]`` of ``dst_caches`` (device <-> pinned host), one launch.

    ``pairs`` is an int32 ``[n, 2]`` tensor on the device.
    """
    import ctypes
    if len(src_caches) != len(dst_caches) or not src_caches:
        raise ValueError("src/dst cache lists must be non-empty and of equal length")
    # one block size and one block count per side: the kernel addresses every
    # layer with layer 0's geometry (V half at num_blocks * block_bytes)
    s0, d0 = src_caches[0], dst_caches[0]
    for s_, d_ in zip(src_caches, dst_caches):
        if s_.dtype != d_.dtype or s_.dim() != 5 or s_.shape[0] != 2 or s_.shape[2:] != d_.shape[2:]:
            raise ValueError("caches must share dtype and [2, *, kv, bs, D] geometry")
        if s_.shape != s0.shape or s_.dtype != s0.dtype:
            raise ValueError(f"every source cache must have shape {tuple(s0.shape)} and dtype "
                             f"{s0.dtype} (got {tuple(s_.shape)}, {s_.dtype})")
        if d_.shape != d0.shape or d_.dtype != d0.dtype:
            raise ValueError(f"every destination cache must have shape {tuple(d0.shape)} and "
                             f"dtype {d0.dtype} (got {tuple(d_.shape)}, {d_.dtype})")
    for s_, d_ in zip(src_caches, dst_caches):
        if not (s_.is_cuda or s_.is_pinned()) or not (d_.is_cuda or d_.is_pinned()):
            raise ValueError("caches must be device tensors or pinned host tensors")
        for t in (s_, d_):
            if t.is_cuda and t.device != pairs.device:
                raise ValueError(f"device caches must be on {pairs.device} (got {t.device})")
        if not s_.is_contiguous() or not d_.is_contiguous():
            raise ValueError("caches must be contiguous")
    _cuda(pairs)
    _i32(pairs, "pairs")
    n = len(src_caches)
    block_bytes = src_caches[0][0, 0].numel() * src_caches[0].element_size()
    src = (ctypes.c_void_p * n)(*[t.data_ptr() for t in src_caches])
    dst = (ctypes.c_void_p * n)(*[t.data_ptr() for t in dst_caches])
    L.check(L.lib().nb_swap_kv_blocks(
        ctypes.cast(src, ctypes.c_void_p), ctypes.cast(dst, ctypes.c_void_p), n,
        pairs.data_ptr(), pairs.shape[0], src_caches[0].shape[1], dst_caches[0].shape[1],
        block_bytes, _stream(pairs)))


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
           top_p: torch.Tensor, uniforms: torch.Tensor, out: Optional[torch.Tensor] = None,
           filtered: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One token per row of ``logits [n, V]`` (``nb_sample``): greedy where
    ``temperature == 0``, else temperature / top-k / top-p and one draw at
    ``uniforms`` (all per-row device tensors: fp32, int32, fp32, fp32).
    Returns int64 token ids on the device; ``filtered`` (optional, like
    ``logits``) receives each sampled row's filtered logits."""
    _cuda(logits, temperature, top_k, top_p, uniforms, out, filtered)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be [n, V] with unit column stride")
    n, V = logits.shape
    for t, dt, name in ((temperature, torch.float32, "temperature"), (top_k, torch.int32, "top_k"),
                        (top_p, torch.float32, "top_p"), (uniforms, torch.float32, "uniforms")):
        if t.dtype != dt or t.numel() < n or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} tensor of at least {n} rows")
    if out is None:
        out = torch.empty(n, dtype=torch.int64, device=logits.device)
    if filtered is not None and (filtered.dtype != logits.dtype or filtered.shape != logits.shape
                                 or filtered.stride(1) != 1):
        raise ValueError("filtered must match logits' shape and dtype")
    L.check(L.lib().nb_sample(
        logits.data_ptr(), logits.stride(0), n, V, temperature.data_ptr(), top_k.data_ptr(),
        top_p.data_ptr(), uniforms.data_ptr(),
        filtered.data_ptr() if filtered is not None else None,
        filtered.stride(0) if filtered is not None else 0, out.data_ptr(), _dtype(logits),
        _stream(logits)))
    return out


def device_errors() -> int:
    """Synchronise and return (and clear) the device error word; see
    ``NB_DEVERR_*`` in the header."""
    return L.device_errors()
