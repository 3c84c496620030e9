"""ModelRunner with needle's API on the B200 attention path.

Mirrors ``needle/model/runner.py:14-249``: the same constructor arguments,
``profile_memory``, ``init_kv_cache`` (per-layer caches of shape
``[2, num_blocks, num_kv_heads, block_size, head_dim]``), ``execute
(SchedulerOutput) -> ExecuteOutput`` (mixed prefill/decode batches run as two
forwards, ``:121-153``), ``_prepare_inputs`` (the same ``input_ids``,
``positions``, ``cu_seqlens``, ``context_lens`` and dummy-padded
``block_table``, ``:194-249``) and block swapping (``:175-192``).  It works
with needle's own Scheduler / BlockAllocator / SchedulerOutput objects or
with the mirrors in ``needle_b200.model.sequence``.

Differences, all below the API: the model is materialised directly on the
device (no CPU copy of the weights); host-built step inputs are copied from
pinned memory without a blocking sync; sampling is batched over the whole
step with a single device-to-host read of the token ids (needle reads one
``int(...)`` per sequence, ``needle/model/sampler.py:24-48``; see
``needle_b200.model.sampler``).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.nn.functional as F

from ..layers.linear import shard_for_rank
from ..layers.rope import RotaryEmbedding
from .config import ModelConfig
from .llama import LlamaForCausalLM
from .qwen2 import Qwen2ForCausalLM
from . import steppack
from .sampler import Sampler
from .sequence import ExecuteInput, ExecuteOutput, SchedulerOutput


def build_model(config: ModelConfig, tp_size: int = 1, tp_rank: int = 0):
    """``needle/model/__init__.py:8-17``: pick the class from ``model_type``."""
    mt = config.model_type.lower()
    if mt == "llama":
        return LlamaForCausalLM(config, tp_size=tp_size, tp_rank=tp_rank)
    if mt == "qwen2":
        return Qwen2ForCausalLM(config, tp_size=tp_size, tp_rank=tp_rank)
    raise ValueError(f"Unsupported model_type: {mt!r}")


def _part(sched_out, prefill: bool):
    """The prefill (or decode) half of a mixed ``SchedulerOutput``, as needle
    builds it for its two forwards (``needle/model/runner.py:121-142``)."""
    return SchedulerOutput(
        prefill_seqs=list(sched_out.prefill_seqs) if prefill else [],
        decode_seqs=[] if prefill else list(sched_out.decode_seqs),
        block_tables=sched_out.block_tables, swap_in_map={}, swap_out_map={},
        blocks_to_free=[])


class _InputStage:
    """Pinned staging for a step's host-built input arrays.

    The arrays are packed (16-byte aligned) into one pinned host buffer and
    moved with a single asynchronous copy into a persistent device buffer;
    the step's tensors are views of it.  Two slots alternate, so the two
    input sets of a mixed prefill + decode step never share one; before a
    slot is refilled its previous copy is waited for (an event recorded right
    after it).  A later step writes a slot's device buffer only through a
    copy on the same stream, after the work that read it.  This replaces a
    pinned allocation and a copy per array per step.
    """

    _TORCH = {np.dtype(np.int64): torch.int64, np.dtype(np.int32): torch.int32}

    def __init__(self, device, slots: int = 2):
        self.device = device
        self.host: List[Optional[torch.Tensor]] = [None] * slots
        self.dev: List[Optional[torch.Tensor]] = [None] * slots
        self.events = [torch.cuda.Event() for _ in range(slots)]
        self.recorded = [False] * slots
        self.next = 0
        self.bytes_copied = 0  # host-to-device bytes moved so far (one copy per put)

    def put(self, arrays: List[np.ndarray], table=None) -> List[torch.Tensor]:
        """Device views of ``arrays`` and, if ``table = (rows, width, pad)``
        is given, of the padded int32 block table built from ``rows``
        (written straight into the staging buffer by the ``_steppack``
        extension when it is built)."""
        if table is not None and steppack.ext() is None:
            arrays = list(arrays) + [steppack.block_table_np(*table)]
            table = None
        offs, total = [], 0
        for a in arrays:
            offs.append(total)
            total += -(-a.nbytes // 16) * 16
        t_off, t_bytes = total, 0
        if table is not None:
            t_bytes = len(table[0]) * table[1] * 4
            total += t_bytes
        k = self.next
        self.next = (k + 1) % len(self.host)
        if self.recorded[k]:
            self.events[k].synchronize()  # this slot's previous copy has landed
        if self.host[k] is None or self.host[k].numel() < total:
            cap = max(total, 1 << 16)
            cap = 1 << (cap - 1).bit_length()
            self.host[k] = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
            self.dev[k] = torch.empty(cap, dtype=torch.uint8, device=self.device)
        hb = self.host[k].numpy()
        for a, o in zip(arrays, offs):
            hb[o:o + a.nbytes].view(a.dtype)[:] = np.ascontiguousarray(a).reshape(-1)
        if t_bytes:
            steppack.fill_block_table(table[0], self.host[k].data_ptr() + t_off,
                                      self.host[k].numel() - t_off, table[1], table[2])
        db = self.dev[k]
        if total:
            db[:total].copy_(self.host[k][:total], non_blocking=True)
            self.bytes_copied += total
        self.events[k].record(torch.cuda.current_stream(self.device))
        self.recorded[k] = True
        out = [db[o:o + a.nbytes].view(self._TORCH[a.dtype]).view(a.shape)
               for a, o in zip(arrays, offs)]
        if table is not None:
            out.append(db[t_off:t_off + t_bytes].view(torch.int32).view(len(table[0]), table[1]))
        return out


class _DecodeGraph:
    """One captured decode forward for a fixed (batch, block-table width)."""

    def __init__(self, B: int, width: int, dummy: int, device):
        self.ids = torch.zeros(B, dtype=torch.long, device=device)
        self.pos = torch.zeros(B, dtype=torch.long, device=device)
        self.ctx = torch.zeros(B, dtype=torch.int32, device=device)
        self.cu = torch.arange(B + 1, dtype=torch.int32, device=device)
        self.bt = torch.full((B, width), dummy, dtype=torch.int32, device=device)
        self.graph = torch.cuda.CUDAGraph()
        self.logits: Optional[torch.Tensor] = None
        # device memory the captured kernels address but no graph-pool tensor
        # owns (the split-K plan's workspace): held for the graph's lifetime
        self.keepalive: List[object] = []


class ModelRunner:
    # Block-table width granularity of captured decode graphs: the kernels'
    # grids depend on the width, so graphs are keyed by it, rounded up.
    GRAPH_WIDTH_STEP = 64

    def __init__(self, model_config: ModelConfig, block_size: int = 16, dtype: str = "bfloat16",
                 device: str = "cuda", tensor_parallel_size: int = 1, tp_rank: int = 0,
                 cuda_graph: bool = True, fuse: bool = True, tp_fused_tokens: int = 1024,
                 prefill_with_context: bool = False):
        """needle's ModelRunner arguments, plus this library's options:
        ``cuda_graph`` (decode steps as CUDA graphs), ``fuse`` (one QKV and
        one gate/up GEMM), ``tp_fused_tokens`` (rows up to which the TP
        all-reduce runs fused over NVLink), and ``prefill_with_context``: a
        prefill chunk attends over the sequence's cached prefix too (K/V from
        the paged cache), the multi-turn / continuation case needle's own
        prefill does not handle; False keeps needle's behaviour (the new
        tokens only)."""
        self.model_config = model_config
        self.block_size = block_size
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("needle_b200 runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.tp_size = tensor_parallel_size
        self.tp_rank = tp_rank
        self.dtype = getattr(torch, dtype) if isinstance(dtype, str) else dtype
        with torch.device("meta"):
            model = build_model(model_config, tp_size=tensor_parallel_size, tp_rank=tp_rank)
        model = model.to_empty(device=self.device).to(self.dtype)
        cfg = model_config
        # RoPE tables are computed on the CPU exactly as needle computes them,
        # then moved and cast like the rest of the model.
        model.model.rotary_emb = RotaryEmbedding(
            cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta).to(self.device, self.dtype)
        model.eval()
        if fuse:
            model.fuse_projections()
        for layer in model.model.layers:
            layer.self_attn.prefill_with_context = prefill_with_context
        self.model = model
        self.sampler = Sampler()
        self.kv_caches: List[torch.Tensor] = []
        self.cpu_kv_caches: List[torch.Tensor] = []
        # Under TP the graph also holds the NCCL all-reduces; NB_TP_GRAPH=0
        # turns capture off there (diagnostics).
        if tensor_parallel_size > 1 and os.environ.get("NB_TP_GRAPH", "1") == "0":
            cuda_graph = False
        self.cuda_graph = cuda_graph
        # Under TP with bf16/fp16, calls of up to tp_fused_tokens rows run the
        # row-parallel all-reduce fused with the residual add and RMSNorm over
        # NVLink peer memory; larger calls (long prefills) use NCCL.
        # NB_TP_FUSED=0 keeps NCCL everywhere.
        self.tp_comm = None
        if (tensor_parallel_size > 1 and self.dtype in (torch.bfloat16, torch.float16)
                and tp_fused_tokens > 0 and os.environ.get("NB_TP_FUSED", "1") != "0"):
            from ..layers.tp_comm import TPComm, attach
            self.tp_comm = TPComm(tp_fused_tokens, cfg.hidden_size, self.dtype, self.device)
            attach(self.model, self.tp_comm)
        self.padding_block = 0
        self._stage: Optional[_InputStage] = None
        self._graphs: Dict[tuple, _DecodeGraph] = {}
        self._graph_pool = None

    # ------------------------------------------------------------------ weights

    @torch.no_grad()
    def load_state_dict(self, state_dict: Dict[str, torch.Tensor]) -> None:
        """Load a full (unsharded) needle-named state dict, sharding for this
        rank like ``needle/model/loader.py:100-149`` (lm_head tied to the
        embedding when absent)."""
        params = dict(self.model.named_parameters())
        missing = set(params)
        for name, p in params.items():
            src = state_dict.get(name)
            if src is None and name == "lm_head.weight":
                src = state_dict.get("model.embed_tokens.weight")
            if src is None:
                continue
            t = shard_for_rank(name, src, self.tp_size, self.tp_rank)
            if tuple(t.shape) != tuple(p.shape):
                raise ValueError(f"Shape mismatch for {name}: {tuple(t.shape)} vs {tuple(p.shape)}")
            p.copy_(t.to(device=p.device, dtype=p.dtype))
            missing.discard(name)
        if missing:
            raise ValueError(f"missing weights: {sorted(missing)[:8]}")

    @torch.no_grad()
    def init_synthetic(self, seed: int = 0) -> None:
        """Fill every parameter with the synthetic distributions of
        ``needle_b200.synth`` generated on the device (for large benchmark
        models; values differ from the CPU-generated ones)."""
        from ..synth import synth_tensor, weight_shapes
        params = dict(self.model.named_parameters())
        for name, shape, kind in weight_shapes(self.model_config):
            full = synth_tensor(name, shape, kind, seed=seed, device=self.device,
                                dtype=torch.float32)
            params[name].copy_(shard_for_rank(name, full, self.tp_size, self.tp_rank))
            del full
        if self.model_config.tie_word_embeddings:
            params["lm_head.weight"].copy_(params["model.embed_tokens.weight"])

    # ------------------------------------------------------------------ memory

    def kv_bytes_per_block(self) -> int:
        cfg = self.model_config
        kvh = max(1, cfg.num_key_value_heads // self.tp_size)
        elt = torch.tensor([], dtype=self.dtype).element_size()
        return 2 * kvh * self.block_size * cfg.head_dim * elt * cfg.num_hidden_layers

    def profile_memory(self, gpu_memory_utilization: float = 0.90):
        """Blocks that fit in the free device memory (``runner.py:44-63``)."""
        free, _total = torch.cuda.mem_get_info(self.device)
        n = max(1, int(free * gpu_memory_utilization) // self.kv_bytes_per_block())
        return n, n // 2

    def init_kv_cache(self, num_gpu_blocks: int, num_cpu_blocks: int) -> None:
        """Per-layer caches for the allocator's ``num_gpu_blocks`` blocks plus
        one padding block (index ``num_gpu_blocks``) that block-table rows are
        padded with.  needle pads with its last allocatable block
        (``needle/model/runner.py:226-229``), which its allocator can also hand
        to a sequence; a block no allocator owns cannot alias real KV."""
        cfg = self.model_config
        kvh = max(1, cfg.num_key_value_heads // self.tp_size)
        self.padding_block = num_gpu_blocks
        shape = (2, num_gpu_blocks + 1, kvh, self.block_size, cfg.head_dim)
        self.kv_caches = [torch.zeros(shape, dtype=self.dtype, device=self.device)
                          for _ in range(cfg.num_hidden_layers)]
        self.cpu_kv_caches = []
        if num_cpu_blocks > 0:
            cshape = (2, num_cpu_blocks, kvh, self.block_size, cfg.head_dim)
            self.cpu_kv_caches = [torch.zeros(cshape, dtype=self.dtype, pin_memory=True)
                                  for _ in range(cfg.num_hidden_layers)]

    # ------------------------------------------------------------------ step

    def execute(self, sched_out) -> ExecuteOutput:
        with torch.cuda.device(self.device):  # the kernels launch on this runner's GPU
            return self._execute(sched_out)

    def _execute(self, sched_out) -> ExecuteOutput:
        if sched_out.swap_out_map and self.cpu_kv_caches:
            self._swap_kv_blocks(sched_out.swap_out_map, "gpu_to_cpu")
        if sched_out.swap_in_map and self.cpu_kv_caches:
            self._swap_kv_blocks(sched_out.swap_in_map, "cpu_to_gpu")
        all_seqs = list(sched_out.prefill_seqs) + list(sched_out.decode_seqs)
        with torch.no_grad():
            if sched_out.prefill_seqs and sched_out.decode_seqs:
                # mixed batch: two forwards, as needle (runner.py:121-148)
                pre = self._prepare_inputs(_part(sched_out, prefill=True))
                dec = self._prepare_inputs(_part(sched_out, prefill=False))
                logits = torch.cat([self._forward(pre), self._forward(dec)], dim=0)
            else:
                logits = self._forward(self._prepare_inputs(sched_out))
        params = [s.request.sampling_params for s in all_seqs]
        ids = self.sampler.sample(logits, params)   # synchronises with the step's kernels
        if self.tp_comm is not None:
            self.tp_comm.check()  # a timed-out all-reduce poisons the step: raise, not bad tokens
        return ExecuteOutput(seq_ids=[s.seq_id for s in all_seqs], next_token_ids=ids)

    def _forward(self, inp: ExecuteInput) -> torch.Tensor:
        if self.cuda_graph and not inp.is_prefill:
            return self._forward_decode_graph(inp)
        return self.model(inp.input_ids, inp.position_ids, self.kv_caches, inp.block_table,
                          inp.cu_seqlens, inp.context_lens, inp.max_seqlen, inp.is_prefill)

    # ------------------------------------------------------------------ graphs

    def _forward_decode_graph(self, inp: ExecuteInput) -> torch.Tensor:
        """Decode forward through a captured CUDA graph.

        The graph runs the whole model (embedding, every layer's GEMMs, fused
        RoPE + KV write, paged decode + merge, fused residual + RMSNorm, NCCL
        all-reduces under TP, lm_head) on static input buffers; each step
        copies its inputs into them and replays.  Block-table columns beyond
        the step's width point at needle's padding block, which decode never
        reads (a sequence reads only its own ceil((ctx+1)/16) columns).
        """
        B, width = inp.block_table.shape
        w = -(-width // self.GRAPH_WIDTH_STEP) * self.GRAPH_WIDTH_STEP
        g = self._graphs.get((B, w))
        if g is None:
            g = self._capture_decode(B, w)
        g.ids.copy_(inp.input_ids, non_blocking=True)
        g.pos.copy_(inp.position_ids, non_blocking=True)
        g.ctx.copy_(inp.context_lens, non_blocking=True)
        g.bt[:, :width].copy_(inp.block_table, non_blocking=True)
        g.graph.replay()
        return g.logits

    def _capture_decode(self, B: int, width: int) -> _DecodeGraph:
        g = _DecodeGraph(B, width, self.padding_block, self.device)

        def run():
            return self.model(g.ids, g.pos, self.kv_caches, g.bt, g.cu, g.ctx, 1, False)

        # Warm-up outside the graph (creates the split plan and workspace,
        # sets kernel attributes, initialises NCCL); its KV writes land in
        # the padding block (context 0, every table entry = padding block),
        # which no sequence owns.
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                run()
        torch.cuda.current_stream(self.device).wait_stream(side)
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g.graph, pool=self._graph_pool):
            g.logits = run()
        # The decode layers took their split-K plan (and workspace) from the
        # shared plan cache, which may drop entries later; the graph keeps
        # every plan of its shape alive.
        from .. import ops
        g.keepalive = [p for p in ops._PLANS.values() if p.key[0] == B and p.key[4] == width]
        self._graphs[(B, width)] = g
        return g

    def capture_decode_graphs(self, batch_size: int, max_blocks_per_seq: int,
                              min_blocks_per_seq: int = 1) -> None:
        """Capture the decode graphs a batch of ``batch_size`` will use while
        its block tables grow from ``min_blocks_per_seq`` to
        ``max_blocks_per_seq`` columns, so that no capture (two eager
        warm-up forwards plus the capture itself) happens mid-run.  Servers
        call this at start-up for the batch sizes they serve."""
        if not self.cuda_graph:
            return
        with torch.cuda.device(self.device):
            self._capture_widths(batch_size, max_blocks_per_seq, min_blocks_per_seq)

    def _capture_widths(self, batch_size: int, max_blocks_per_seq: int,
                        min_blocks_per_seq: int) -> None:
        step = self.GRAPH_WIDTH_STEP
        lo = -(-max(1, min_blocks_per_seq) // step) * step
        hi = -(-max(1, max_blocks_per_seq) // step) * step
        with torch.no_grad():
            for w in range(lo, hi + 1, step):
                if (batch_size, w) not in self._graphs:
                    self._capture_decode(batch_size, w)

    def release_graphs(self) -> None:
        """Drop captured graphs (required before destroying an NCCL group)."""
        self._graphs.clear()
        self._graph_pool = None

    def close(self) -> None:
        """Release graphs and unmap the peers' all-reduce buffers; call on
        every rank before destroying the process group."""
        self.release_graphs()
        if self.tp_comm is not None:
            from ..layers.tp_comm import attach
            attach(self.model, None)
            self.tp_comm.close()
            self.tp_comm = None

    def _swap_kv_blocks(self, mapping: dict, direction: str) -> None:
        """Copy whole blocks between the device and pinned host caches
        (``needle/model/runner.py:175-192``): every layer and block in one
        ``nb_swap_kv_blocks`` launch.  ``mapping`` is {source block: target
        block} (gpu->cpu for swap-out, cpu->gpu for swap-in, as in needle)."""
        if not mapping:
            return
        from .. import ops
        pairs = torch.tensor(list(mapping.items()), dtype=torch.int32).pin_memory()
        pairs = pairs.to(self.device, non_blocking=True)
        if direction == "gpu_to_cpu":
            ops.swap_kv_blocks(self.kv_caches, self.cpu_kv_caches, pairs)
        else:
            ops.swap_kv_blocks(self.cpu_kv_caches, self.kv_caches, pairs)

    def _h2d(self, data, dtype=None) -> torch.Tensor:
        t = data if isinstance(data, torch.Tensor) else (
            torch.from_numpy(data) if isinstance(data, np.ndarray) else torch.tensor(data, dtype=dtype))
        return t.pin_memory().to(self.device, non_blocking=True)

    def _h2d_many(self, arrays: List[np.ndarray], table=None) -> List[torch.Tensor]:
        """A step's input arrays (and its block table, ``table = (rows,
        width, pad)``) on the device with one pinned-memory copy (see
        ``_InputStage``)."""
        if self._stage is None:
            self._stage = _InputStage(self.device)
        return self._stage.put(arrays, table)

    def _prepare_inputs(self, sched_out) -> ExecuteInput:
        """``needle/model/runner.py:194-249`` with needle's signature: the same
        tensors from a ``SchedulerOutput`` (its ``prefill_seqs``,
        ``decode_seqs`` and ``block_tables``).  A sequence with nothing
        generated feeds its whole prompt at context 0, any other feeds its
        last token at context ``length - 1``; block-table rows are padded
        (here with the reserved padding block).  Built with numpy; pure decode
        batches take a vectorised path."""
        prefill_seqs, decode_seqs = sched_out.prefill_seqs, sched_out.decode_seqs
        block_tables = sched_out.block_tables
        all_seqs = list(prefill_seqs) + list(decode_seqs)
        is_prefill = len(decode_seqs) == 0 or len(prefill_seqs) > 0
        B = len(all_seqs)
        if B and all(s.num_generated_tokens > 0 for s in all_seqs):
            ids = np.fromiter((s.token_ids[-1] for s in all_seqs), np.int64, B)
            ctx = np.fromiter((len(s.token_ids) - 1 for s in all_seqs), np.int32, B)
            pos = ctx.astype(np.int64)
            cu = np.arange(B + 1, dtype=np.int32)
            max_seqlen = 1
        else:
            ids_l: List[int] = []
            pos_l: List[int] = []
            cu = np.zeros(B + 1, dtype=np.int32)
            ctx = np.zeros(B, dtype=np.int32)
            for i, seq in enumerate(all_seqs):
                if seq.num_generated_tokens == 0:
                    toks, c = seq.token_ids, 0
                else:
                    toks, c = [seq.token_ids[-1]], len(seq.token_ids) - 1
                ids_l.extend(toks)
                pos_l.extend(range(c, c + len(toks)))
                cu[i + 1] = cu[i] + len(toks)
                ctx[i] = c
            ids = np.asarray(ids_l, dtype=np.int64)
            pos = np.asarray(pos_l, dtype=np.int64)
            max_seqlen = int((cu[1:] - cu[:-1]).max()) if B else 1
        tables = [block_tables.get(s.seq_id, []) for s in all_seqs]
        maxb = max(1, max(map(len, tables), default=1))
        d_ids, d_pos, d_cu, d_ctx, d_bt = self._h2d_many([ids, pos, cu, ctx],
                                                         table=(tables, maxb, self.padding_block))
        return ExecuteInput(input_ids=d_ids, position_ids=d_pos, cu_seqlens=d_cu,
                            max_seqlen=max_seqlen, block_table=d_bt, context_lens=d_ctx,
                            is_prefill=is_prefill)
