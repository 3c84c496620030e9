"""Peer-mapped buffers for the fused tensor-parallel all-reduce + residual + RMSNorm.

needle all-reduces the output of every row-parallel projection with NCCL
(``needle/layers/linear.py:92-98``) and then runs the decoder's residual add
and RMSNorm (``needle/model/llama.py:67-72``).  ``TPComm`` replaces that pair
with one kernel (``nb_tp_allreduce_add_rmsnorm``): every rank pushes each row
of its partial sums to the rank that owns the row over NVLink, the owner sums
them, adds the residual, normalises and pushes the result to every rank.

Each rank allocates one device buffer of receive and gather slots (filled
with the kernel's sentinel, 0xFF bytes) and exports it with CUDA IPC; the
handles are exchanged once through ``torch.distributed`` and every peer's
buffer is mapped into this process.  ``RowParallelLinear`` writes its partial
GEMM output into ``partial`` and ``RMSNorm`` recognises that tensor and
launches the fused kernel, so the sequence of modules (and needle's module
API) is unchanged.  All pointers are fixed for the life of the object, so the
launches can be captured in CUDA graphs.  Calls with more tokens than the
buffers hold fall back to NCCL.

Failure: every wait of the kernel on a peer is bounded (2 s by default,
``set_wait_limit``).  A kernel that gives up marks the communicator poisoned
in device memory (later launches, graph replays included, return without
touching the buffers) and in a pinned host word that ``check()`` reads with
no device sync.  A poisoned ``TPComm`` refuses further calls (``TPCommError``)
until every rank calls ``reset()``, which refills the buffers and counters.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import _lib as L

_MAX_ROWS_PER_RANK = 1024
_MAX_WORLD = 8
_MAX_HIDDEN = 8192
_SEGMENT = 2 << 20                  # whole allocator segments: nothing else shares the mapping
_EPOCH_WORDS = 2080                 # NB_TP_EPOCH_WORDS: 2 x 1024 call counters + status word
_STATUS_WORD = 2048                 # NB_TP_STATUS_WORD


class TPCommError(RuntimeError):
    """A wait on a peer timed out; the communicator is poisoned until reset()."""


def set_wait_limit(seconds: float) -> None:
    """Bound of every wait of the fused kernel on a peer (process-wide; 0
    restores the default of 2 s).  Launches read it, so graphs keep the value
    they were captured with."""
    L.check(L.lib().nb_tp_set_wait_limit_ns(int(seconds * 1e9)))


class TPComm:
    """One rank's view of the shared all-reduce buffers.

    ``max_tokens`` bounds the rows of one call (decode batch size, or a short
    prefill); it is clamped to ``1024 * world``.
    """

    def __init__(self, max_tokens: int, hidden: int, dtype: torch.dtype, device,
                 group=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("TPComm needs an initialised torch.distributed process group")
        if dtype not in (torch.bfloat16, torch.float16):
            raise TypeError("the fused TP all-reduce supports bf16 and fp16")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _MAX_WORLD:
            raise ValueError(f"world size {self.world} exceeds {_MAX_WORLD}")
        if hidden % 8 or hidden > _MAX_HIDDEN:
            raise ValueError(f"hidden {hidden} must be a multiple of 8 up to {_MAX_HIDDEN}")
        self.hidden, self.dtype = hidden, dtype
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_tokens = min(int(max_tokens), _MAX_ROWS_PER_RANK * self.world)
        # local: partial sums (the GEMM writes here), normalised output, residual
        mk = lambda: torch.zeros(self.max_tokens, hidden, dtype=dtype, device=self.device)
        self.partial, self.out, self.residual = mk(), mk(), mk()
        # shared: receive slots [2][world][slot_rows][hidden], then gather
        # slots [2][world][slot_rows][2][hidden]
        esz = self.partial.element_size()
        self.slot_rows = -(-self.max_tokens // self.world)
        n_recv = 2 * self.world * self.slot_rows * hidden * esz
        n_gather = 2 * n_recv
        total = -(-(n_recv + n_gather) // _SEGMENT) * _SEGMENT
        self._buf = torch.full((total,), 0xFF, dtype=torch.uint8, device=self.device)
        # per-row-index call counters of the kernel's two CTA roles, then the
        # status word (non-zero: poisoned by a timed-out wait)
        self.epochs = torch.zeros(_EPOCH_WORDS, dtype=torch.int32, device=self.device)
        # host-visible copy of the status, written by the kernel over PCIe
        self.status_host = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        torch.cuda.synchronize(self.device)  # sentinels in place before any peer can write

        with torch.cuda.device(self.device):  # peer buffers are mapped into this device
            self._map_peers(group)

    def _map_peers(self, group) -> None:
        lib = L.lib()
        n_recv = 2 * self.world * self.slot_rows * self.hidden * self.partial.element_size()
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_uint64(0)
        L.check(lib.nb_ipc_handle(self._buf.data_ptr(), ctypes.addressof(handle),
                                  ctypes.addressof(offset)))
        entries: List[Optional[tuple]] = [None] * self.world
        dist.all_gather_object(entries, (bytes(handle), offset.value), group=group)
        self._opened: List[int] = []
        bases = []
        try:
            for p, (h, off) in enumerate(entries):
                if p == self.rank:
                    bases.append(self._buf.data_ptr())
                    continue
                hb = (ctypes.c_char * 64).from_buffer_copy(h)
                ptr = ctypes.c_void_p(0)
                L.check(lib.nb_ipc_open(ctypes.addressof(hb), ctypes.addressof(ptr)))
                self._opened.append(ptr.value)
                bases.append(ptr.value + off)
        except Exception:
            self.close()  # unmap what was mapped before the failure
            raise
        W = self.world
        self._recv = (ctypes.c_void_p * W)(*bases)
        self._gather = (ctypes.c_void_p * W)(*[b + n_recv for b in bases])
        self._epochs = ctypes.cast(ctypes.c_void_p(self.epochs.data_ptr()),
                                   ctypes.POINTER(ctypes.c_uint))
        self._status_host = ctypes.cast(ctypes.c_void_p(self.status_host.data_ptr()),
                                        ctypes.POINTER(ctypes.c_uint))
        dist.barrier(group=group)  # every rank has mapped every buffer

    def poisoned(self) -> bool:
        """True once a kernel of this communicator timed out (no device sync:
        reads the pinned host word, which completed kernels have written)."""
        return bool(self.status_host[0].item())

    def check(self) -> None:
        """Raise ``TPCommError`` if a kernel launched so far (and completed)
        timed out waiting on a peer."""
        if self.poisoned():
            raise TPCommError(
                f"fused TP all-reduce on rank {self.rank}: a wait on a peer timed out; the "
                "communicator is poisoned until every rank calls TPComm.reset()")

    def reset(self) -> None:
        """Collective: make a poisoned communicator usable again.  Every rank
        waits for its own work, then all refill their buffers with the
        sentinel and zero the counters and the status, then meet again."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            self._buf.fill_(0xFF)
            self.epochs.zero_()
        torch.cuda.synchronize(self.device)
        self.status_host.zero_()
        dist.barrier(group=self.group)

    def can_fuse(self, num_tokens: int) -> bool:
        return 0 < num_tokens <= self.max_tokens

    def is_partial(self, x: torch.Tensor) -> bool:
        """True if ``x`` is the partial-sum view that ``RowParallelLinear``
        returned for the fused path."""
        return x.data_ptr() == self.partial.data_ptr() and x.dim() == 2

    def allreduce_add_rmsnorm(self, num_tokens: int, residual: torch.Tensor,
                              weight: torch.Tensor, eps: float):
        """All-reduce ``partial[:T]`` over the group, add ``residual``, RMSNorm
        with ``weight``.  Returns ``(normed, new_residual)`` as views of this
        object's ``out`` and ``residual`` buffers (identical on every rank)."""
        T = num_tokens
        res = self.residual[:T]
        if residual.data_ptr() != res.data_ptr():
            res.copy_(residual)
        if weight.dtype != self.dtype or not weight.is_contiguous():
            raise TypeError("weight must be contiguous and of the buffers' dtype")
        if torch.cuda.current_device() != self.device.index:
            raise ValueError(f"TPComm lives on {self.device}; make it the current device")
        self.check()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        L.check(L.lib().nb_tp_allreduce_add_rmsnorm(
            self.partial.data_ptr(), ctypes.cast(self._recv, ctypes.c_void_p),
            ctypes.cast(self._gather, ctypes.c_void_p), self.slot_rows, self.out.data_ptr(),
            self.residual.data_ptr(), self._epochs, self._status_host, self.rank, self.world,
            weight.data_ptr(), T, self.hidden, float(eps),
            2 if self.dtype == torch.bfloat16 else 1, stream))
        return self.out[:T], res

    def close(self) -> None:
        """Unmap the peers' buffers (after all work that uses them finished)."""
        if self._opened:
            torch.cuda.synchronize(self.device)
            lib = L.lib()
            with torch.cuda.device(self.device):
                for p in self._opened:
                    lib.nb_ipc_close(p)
            self._opened = []


def attach(model: torch.nn.Module, comm: Optional[TPComm]) -> None:
    """Point every ``RowParallelLinear`` without bias and every ``RMSNorm`` of
    ``model`` at ``comm`` (``None`` detaches).

    Contract: an attached ``RowParallelLinear`` returns its partial sums
    un-reduced, so its output must go straight into an attached ``RMSNorm``
    called with the residual (as in the Llama/Qwen2 decoder layers here:
    ``o_proj`` -> ``post_attention_layernorm``, ``down_proj`` -> the next
    ``input_layernorm`` or the final norm).  Models that use a row-parallel
    output any other way must not be attached."""
    from .linear import RowParallelLinear
    from .norm import RMSNorm
    for m in model.modules():
        if isinstance(m, RowParallelLinear) and m.bias is None and m.reduce_output:
            m.comm = comm
        elif isinstance(m, RMSNorm):
            m.comm = comm
