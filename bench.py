"""Benchmark of the needle_b200 attention hot path.

Default workload (``--workload llama8b``): decode
tokens/s of a Llama-3-8B-shape model (random init, bf16) serving 256
requests with prompts U[128, 1024], greedy, block_size 16, through needle's
runner API (``ModelRunner.execute``, needle/model/runner.py:98-161).  At N=1
it runs on one GPU; for N > 1 (torchrun, one process per GPU) the same
model, requests and batch are sharded tensor-parallel over the N GPUs
(heads and MLP columns per rank, the row-parallel all-reduce fused with the
residual add and RMSNorm over NVLink): "scaling": "strong".

One JSON line (rank 0) carries:
  value          decode tokens/s with the step's inputs resident in HBM (the
                 captured decode graph replayed, greedy tokens fed back on the
                 device), CUDA events on the launching stream, max over ranks;
  e2e            the same metric through ModelRunner.execute with host inputs
                 (pinned H2D copy of the step's arrays, token ids read back);
  roofline       the paged-decode kernels (split + merge) on BASELINE config 2
                 (B=64, 32/8 heads, ctx U[512, 4096]) timed in the same run,
                 against the measured HBM copy bandwidth;
  step_roofline  the whole step against its per-rank HBM bound;
  allreduce      (N > 1) microseconds per fused all-reduce call at the step's
                 shape and its share of the step;
  cpu_baseline   (N=1) needle's CPU path on the host cores, extrapolated from
                 one decoder layer.

Other workloads: llama8b-c4 (config 4), qwen72b (config 5), decode-op
(config 2 alone), prefill, allreduce, store-kv.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

``--impl reference`` times needle's own CPU path for the same workload (the
oracle restatement in oracle/, pinned to needle by golden vectors) on the
host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = ("decode tokens/sec at batch 64/256; paged-attn achieved HBM GB/s vs ~8 TB/s peak")
FALLBACK_HBM_GBS = 6650.0
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "paged_decode_config2.md")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--pages-per-split", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline sample budget (rank 0, N=1 only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-ctx", type=int, default=0,
                    help="prefill workload: cached tokens before each chunk (paged prefill)")
    ap.add_argument("--prefill-shape", default="16x1024",
                    help="prefill workload: sequences x new tokens per sequence")
    ap.add_argument("--workload",
                    choices=["llama8b", "llama8b-c4", "qwen72b", "decode-op", "prefill",
                             "allreduce", "store-kv", "kernel-cases", "step-profile"],
                    default="llama8b",
                    help="llama8b (default): config 3, Llama-3-8B decode at batch 256, tp=N; "
                         "llama8b-c4: config 4 (512 requests, tp=N); qwen72b: config 5 (tp=N, "
                         "N>=4); decode-op: config 2, the paged decode op alone; prefill: the "
                         "prefill kernel; allreduce: the TP all-reduce + residual + RMSNorm "
                         "per call, fused kernel vs NCCL; store-kv: the prefill-size paged KV "
                         "write (T=8192)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_init(n):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={ws}; launch N>1 with torchrun")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    return rank, local, ws


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, ws: int, dev) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks (read-only NVML sampling during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, index: int, period=0.02):
        self.samples, self.reasons, self.ok = [], 0, False
        self.period = period
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - no NVML on this host
            self.err = repr(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    try:
        with open(PROFILE_SUMMARY) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_decode_call:"):
                    return int(float(line.split(":", 1)[1].strip().split()[0]))
    except Exception:
        pass
    return None


def decode_alg_bytes(seq_len, kvh, hq, d, elt):
    """Algorithmic bytes of one paged-decode call: every cached K and V row
    of every sequence read once, Q read and O written once."""
    n_tok = int(seq_len.sum())
    B = int(seq_len.numel())
    return n_tok * kvh * d * 2 * elt + B * hq * d * elt * 2


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def measure_decode_op(dev, ws, batch=64, steps=20, warmup=3, pages_per_split=None,
                      clocks=None):
    """Config 2 (isolated paged decode, one layer): ``steps`` back-to-back
    decode steps (new token's KV write + split-K paged decode + merge), each
    launch bracketed by CUDA events on the launching stream.  Returns the
    roofline of the paged-decode kernels (max over ranks) and the tensors,
    so the decode-op workload can also time the host-buffer path."""
    from needle_b200 import ops
    from needle_b200.synth import decode_op_workload

    H, KVH, D, BS = 32, 8, 128, 16
    w = decode_op_workload(batch=batch, num_heads=H, num_kv_heads=KVH, head_dim=D,
                           block_size=BS, device=dev)
    q, k_new, v_new = w["q"], w["k_new"], w["v_new"]
    cache, bt, ctx = w["kv_cache"], w["block_table"], w["context_lens"]
    B, maxb = bt.shape
    plan = ops.DecodePlan(B, H, KVH, D, maxb, BS, dev, pages_per_split=pages_per_split)
    out = torch.empty_like(q)
    st = torch.cuda.current_stream(dev)

    def step():
        ops.store_kvcache(k_new, v_new, cache, bt, ctx)          # decode KV write
        ops.paged_decode(q, cache, bt, ctx, w["scale"], out=out, plan=plan)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize(dev)
    K = steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    torch.cuda.synchronize(dev)
    start.record(st)
    for i in range(K):
        ev[i][0].record(st)
        ops.store_kvcache(k_new, v_new, cache, bt, ctx)
        ev[i][1].record(st)
        ops.paged_decode(q, cache, bt, ctx, w["scale"], out=out, plan=plan)
        ev[i][2].record(st)
    end.record(st)
    torch.cuda.synchronize(dev)
    barrier(ws)
    t_ms = max_over_ranks(start.elapsed_time(end), ws, dev)
    dec_ms = max_over_ranks(sum(ev[i][1].elapsed_time(ev[i][2]) for i in range(K)) / K, ws, dev)
    store_ms = max_over_ranks(sum(ev[i][0].elapsed_time(ev[i][1]) for i in range(K)) / K, ws,
                              dev)
    elt = cache.element_size()
    alg = decode_alg_bytes(w["seq_len"], KVH, H, D, elt)
    peak, peak_src = measured_hbm_peak()
    achieved = alg / (dec_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "paged_decode_tc + decode_merge (config 2: B=64, "
                                          "32/8 heads, D=128, ctx U[512,4096], bf16)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_src,
                "alg_bytes_per_call": alg, "call_ms": round(dec_ms, 5),
                "traffic": profiled_traffic()}
    detail = {"tokens_cached": int(w["seq_len"].sum()), "pool_blocks": 20000,
              "pages_per_split": plan.pages_per_split, "max_splits": plan.max_splits,
              "store_kvcache_ms": round(store_ms, 5), "paged_decode_ms": round(dec_ms, 5),
              "steps": K, "step_ms": round(t_ms / K, 5),
              "launches": K * (2 + (1 if plan.max_splits > 1 else 0))}
    return {"roofline": roofline, "detail": detail, "t_ms": t_ms, "K": K, "B": B, "w": w,
            "plan": plan, "out": out, "step": step}


def run_ours(args):
    """``--workload decode-op``: config 2 alone (one layer's decode step)."""
    rank, local, ws = dist_init(args.gpus)
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    with clocks:
        m = measure_decode_op(dev, ws, batch=args.batch, steps=args.steps,
                              warmup=args.warmup, pages_per_split=args.pages_per_split)
        # keep the GPU loaded briefly so the sampler sees load clocks even for
        # a short timed region (untimed, same work)
        t_hold = time.time()
        while time.time() - t_hold < max(0.0, 0.5 - m["t_ms"] / 1e3):
            for _ in range(50):
                m["step"]()
            torch.cuda.synchronize(dev)
    w, out, step, K, B = m["w"], m["out"], m["step"], m["K"], m["B"]
    q, k_new, v_new = w["q"], w["k_new"], w["v_new"]
    bt, ctx = w["block_table"], w["context_lens"]
    t_ms = m["t_ms"]
    value = ws * B * K / (t_ms / 1e3)
    st = torch.cuda.current_stream(dev)

    # ---- end to end through the C ABI with host buffers --------------------
    q_h = q.cpu().pin_memory()
    k_h, v_h = k_new.cpu().pin_memory(), v_new.cpu().pin_memory()
    bt_h, ctx_h = bt.cpu().pin_memory(), ctx.cpu().pin_memory()
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h, bt_h, ctx_h))
    d2h = out_h.numel() * out_h.element_size()

    def step_e2e():
        q.copy_(q_h, non_blocking=True)
        k_new.copy_(k_h, non_blocking=True)
        v_new.copy_(v_h, non_blocking=True)
        bt.copy_(bt_h, non_blocking=True)
        ctx.copy_(ctx_h, non_blocking=True)
        step()
        out_h.copy_(out, non_blocking=True)

    for _ in range(3):
        step_e2e()
    torch.cuda.synchronize(dev)
    barrier(ws)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(st)
    for _ in range(K):
        step_e2e()
    e2.record(st)
    torch.cuda.synchronize(dev)
    barrier(ws)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2), ws, dev)
    e2e_value = ws * B * K / (e2e_ms / 1e3)

    # ---- CPU baseline: needle's path (oracle restatement) on host cores ----
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args.cpu_seconds)

    if rank == 0:
        d = m["detail"]
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
            "steps": K, "warmup": max(3, args.warmup), "ms_per_step": round(t_ms / K, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, Q/K/V ~ N(0,1))",
            "config": {"workload": "config2: isolated paged decode op (decode KV write + "
                                   "split-K paged decode + merge), one layer",
                       "batch_per_gpu": B, "q_heads": 32, "kv_heads": 8, "head_dim": 128,
                       "block_size": 16, "ctx": "U[512,4096] seed 0",
                       "tokens_cached": d["tokens_cached"], "pool_blocks": 20000,
                       "pages_per_split": d["pages_per_split"], "max_splits": d["max_splits"],
                       "l2": "inputs larger than L2 (KV working set %.0f MB > 126 MB)"
                             % (m["roofline"]["alg_bytes_per_call"] / 1e6),
                       "parallelism": f"replicas x{ws} (independent batches, no collective)"},
            "roofline": m["roofline"],
            "kernel_ms": {"store_kvcache": d["store_kvcache_ms"],
                          "paged_decode": d["paged_decode_ms"]},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "cpu_baseline": cpu,
            "gpu_launches": d["launches"],
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def cpu_baseline(w, budget_s):
    """Needle's _decode (KV write + _decode_pytorch) restated in oracle/, on
    all host threads, over the same 64-sequence batch; bounded by budget_s."""
    from oracle import needle_oracle as no
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cache = w["kv_cache"].cpu()
    q, k, v = w["q"].cpu(), w["k_new"].cpu(), w["v_new"].cpu()
    bt, ctx = w["block_table"].cpu(), w["context_lens"].cpu()
    B, H, D = q.shape
    kvh = k.shape[1]
    times = []
    t_all = time.time()
    while not times or (time.time() - t_all < budget_s and len(times) < 50):
        t0 = time.time()
        no.decode_write_kv(k, v, cache, bt, ctx)
        no.decode_attention(q, cache, bt, ctx, w["scale"], H, kvh, D)
        times.append(time.time() - t0)
    t = statistics.median(times)
    return {"value": round(B / t, 2), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{len(times)} full calls of the 64-sequence decode "
                                     f"(KV write + attention), median {t * 1e3:.1f} ms"}


# ---------------------------------------------------------------------------
# reference arm: needle's CPU PyTorch path on the host cores
# ---------------------------------------------------------------------------

def run_reference(args):
    """needle's own CPU path for the path under test, on the host cores
    (rank 0 only; other ranks exit without work)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload in MODEL_WORKLOADS:
        return run_reference_model(args)
    return run_reference_op(args)


def run_reference_model(args):
    """Model workloads: needle's decode step on the host cores, EXTRAPOLATED.
    A "step" here is one decoder layer of the full model at the workload's
    batch and the context lengths of the first timed GPU step (needle's CPU
    path as restated in oracle/, pinned to needle by golden vectors); the
    tokens/s figure is batch / (layers x median layer time + lm_head time).
    The full model does not fit the host path's time budget (one full step
    takes seconds), so the layer is the bounded sample."""
    from needle_b200.model import preset
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    torch.set_num_threads(os.cpu_count() or 1)
    preset_name, n_req, lo, hi, out_tokens, name = MODEL_WORKLOADS[args.workload]
    cfg = preset(preset_name)
    prompts, prefill = _model_prompts(args.workload, cfg)
    W = max(1, args.warmup)
    # cached tokens at the GPU arm's first timed step: the prompt, the token
    # of the prefill (or config 5's first token) and its warm-up steps, less
    # the step's own input token
    ctx_lens = [len(p) + max(3, args.warmup) for p in prompts]
    layer, head = _cpu_decode_layer(cfg, ctx_lens)
    for _ in range(W):
        layer()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        layer()
        times.append(time.perf_counter() - t0)
    t_layer = statistics.median(times)
    t0 = time.perf_counter()
    head()
    t_head = (time.perf_counter() - t0) * 8
    step = cfg.num_hidden_layers * t_layer + t_head
    B = len(prompts)
    value = B / step
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": W, "ms_per_step": round(step * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random token ids; zero weights on the CPU path)",
        "config": {"workload": f"{name}: {cfg.model_type} {cfg.hidden_size}h/"
                               f"{cfg.num_hidden_layers}L decode, batch {B} (needle CPU path, "
                               "extrapolated from one layer)",
                   "model": args.workload, "batch": B, "tp": 1,
                   "ctx_at_first_timed_step": round(sum(ctx_lens) / B, 1),
                   "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": cores,
                         "kind": "port", "extrapolated": True,
                         "sample": f"{args.steps} decode steps of one decoder layer at B={B} "
                                   f"(median {t_layer * 1e3:.0f} ms) x{cfg.num_hidden_layers} "
                                   f"layers + lm_head ({t_head * 1e3:.0f} ms); needle's path "
                                   "restated in oracle/"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_op(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    from needle_b200.synth import decode_op_workload
    from oracle import needle_oracle as no
    torch.set_num_threads(os.cpu_count() or 1)
    w = decode_op_workload(batch=args.batch, device="cpu")
    q, k, v = w["q"], w["k_new"], w["v_new"]
    cache, bt, ctx = w["kv_cache"], w["block_table"], w["context_lens"]
    B, H, D = q.shape
    kvh = k.shape[1]

    def step():
        no.decode_write_kv(k, v, cache, bt, ctx)
        no.decode_attention(q, cache, bt, ctx, w["scale"], H, kvh, D)

    for _ in range(max(1, args.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    t = time.perf_counter() - t0
    value = B * args.steps / t
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": max(1, args.warmup),
        "ms_per_step": round(t / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, Q/K/V ~ N(0,1))",
        "config": {"workload": "config2: isolated paged decode op (decode KV write + "
                               "paged decode attention), one layer",
                   "batch": B, "q_heads": H, "kv_heads": kvh, "head_dim": D, "block_size": 16,
                   "ctx": "U[512,4096] seed 0", "pool_blocks": 20000,
                   "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores,
                         "kind": "port",
                         "sample": f"{args.steps} full steps of the 64-sequence decode "
                                   "(needle's _decode restated in oracle/, pinned to needle "
                                   "by golden vectors)"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# model workloads (configs 3-5): decode tokens/s through ModelRunner.execute
# ---------------------------------------------------------------------------

def _weights_read_per_step(runner) -> int:
    """Bytes of weights one decode step reads on this rank: every parameter
    except the embedding table (only B rows of it are gathered)."""
    n = 0
    for name, p in runner.model.named_parameters():
        if name != "model.embed_tokens.weight":
            n += p.numel() * p.element_size()
    return n


def _nb_linear_per_step(runner, B) -> int:
    """Projections of one decode step (batch B) that run on this library's
    GEMM (``ops.linear_preferred``, as ``layers.linear.dense`` decides)."""
    from needle_b200 import ops
    from needle_b200.layers import linear as lin
    if not lin._LINEAR_TC:
        return 0

    def pref(w):
        if w is None:
            return False
        return ops.linear_preferred(torch.empty(B, w.shape[1], dtype=w.dtype, device=w.device), w)
    n = 0
    for layer in runner.model.model.layers:
        attn, mlp = layer.self_attn, layer.mlp
        for w in (getattr(attn, "_qkv_w", None), attn.o_proj.weight, getattr(mlp, "_gu_w", None),
                  mlp.down_proj.weight):
            n += pref(w)
    return n + pref(runner.model.lm_head.weight)


MODEL_WORKLOADS = {
    # name: (preset, requests, prompt lo, prompt hi, output tokens, label)
    "llama8b": ("llama3-8b", 256, 128, 1024, 256, "config3"),
    "llama8b-c4": ("llama3-8b", 512, 256, 2048, 512, "config4"),
    "qwen72b": ("qwen2-72b", 128, 4096, 8192, 128, "config5"),
}


def _model_prompts(workload, cfg):
    """The workload's prompts (seeded): configs 3/4 are prompts that are
    prefilled; config 5 starts from decode with contexts U[4096, 8192]."""
    _, n_req, lo, hi, out_tokens, name = MODEL_WORKLOADS[workload]
    if workload == "qwen72b":
        g = torch.Generator().manual_seed(0)
        ctx = torch.randint(lo, hi + 1, (n_req,), generator=g).tolist()
        return [torch.randint(0, cfg.vocab_size, (c,), generator=g).tolist() for c in ctx], False
    from needle_b200.synth import synth_prompts
    return synth_prompts(n_req, lo, hi, cfg.vocab_size, seed=0), True


def _time_fused_allreduce(comm, T, weight, eps, dev, ws, calls=50, reps=4):
    """Device time of one fused all-reduce + residual + RMSNorm call at the
    decode step's shape: a CUDA graph of ``calls`` back-to-back launches,
    replayed ``reps`` times; max over ranks."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            comm.allreduce_add_rmsnorm(T, comm.residual[:T], weight, eps)
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(calls):
            comm.allreduce_add_rmsnorm(T, comm.residual[:T], weight, eps)
    graph.replay()
    torch.cuda.synchronize(dev)
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / (reps * calls), ws, dev)
    del graph
    comm.check()
    return us


def run_model(args):
    """Decode tokens/s of a whole model through needle's runner API.

    Default (``llama8b``): config 3 -- Llama-3-8B shape, bf16, 256 requests,
    prompts U[128, 1024], greedy -- at N=1, and the same model, requests and
    batch sharded TP=N over N GPUs for N > 1 (strong scaling; the row-parallel
    all-reduce runs as the fused NVLink kernel).  ``llama8b-c4`` is config 4
    (512 requests, prompts U[256, 2048]) and ``qwen72b`` config 5.

    Three measurements, each timed with CUDA events on the launching stream
    and taken as the max over ranks:
    * ``value``: decode steps with the step's inputs resident in HBM -- the
      captured decode graph (every layer, lm_head) replayed K times, the
      greedy token of each step fed back on the device (argmax, positions and
      context lengths advanced in place);
    * ``e2e``: K engine steps through ``ModelRunner.execute`` with host
      inputs (needle's SchedulerOutput: step arrays packed and copied from
      pinned memory, sampled token ids read back to the host every step);
    * ``roofline``: the paged-decode kernels (split + merge) on config 2
      (B=64, 32/8 heads, ctx U[512, 4096]) timed in the same process, their
      algorithmic KV + Q + O bytes against the measured HBM copy bandwidth;
      ``step_roofline`` holds the whole step against its per-rank HBM bound
      (weights + every cached K/V row read once per step).
    """
    rank, local, ws = dist_init(args.gpus)
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    from needle_b200.model import ModelRunner, preset
    from needle_b200.model.driver import BatchDriver, blocks_needed
    from needle_b200.model.sequence import SamplingParams, SchedulerOutput

    # ---- kernel evidence: config 2 paged decode in this process ------------
    kern = measure_decode_op(dev, ws, batch=64, steps=max(20, args.steps),
                             warmup=max(3, args.warmup))
    torch.cuda.empty_cache()

    preset_name, n_req, lo, hi, out_tokens, name = MODEL_WORKLOADS[args.workload]
    cfg = preset(preset_name)
    prompts, prefill = _model_prompts(args.workload, cfg)
    runner = ModelRunner(cfg, block_size=16, dtype="bfloat16", device=str(dev),
                         tensor_parallel_size=ws, tp_rank=rank)
    runner.init_synthetic(seed=0)
    nblk = blocks_needed([len(p) for p in prompts], out_tokens + 1, 16)
    runner.init_kv_cache(nblk, 0)
    drv = BatchDriver(runner, nblk)
    params = SamplingParams(temperature=0.0, max_new_tokens=out_tokens)
    seqs = [drv.add(p, params) for p in prompts]
    st = torch.cuda.current_stream(dev)
    t_prefill_ms = None
    if prefill:
        barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        drv.step()                      # one prefill forward over every prompt
        e1.record(st)
        torch.cuda.synchronize(dev)
        t_prefill_ms = max_over_ranks(e0.elapsed_time(e1), ws, dev)
    else:
        # config 5 starts from decode: a synthetic (random) cache holds each
        # sequence's context, and one token has been "generated" already.
        g = torch.Generator().manual_seed(1)
        gd = torch.Generator(device=dev).manual_seed(1 + rank)
        for c in runner.kv_caches:
            c.normal_(generator=gd)
        for s in seqs:
            s.append_token(int(torch.randint(0, cfg.vocab_size, (1,), generator=g)))
    steps_left = out_tokens - (1 if prefill else 0)
    W = min(max(3, args.warmup), max(1, steps_left // 4))
    K = max(1, min(args.steps, (steps_left - W) // 2))
    B = len(seqs)
    # capture every decode graph the warm-up and both timed loops will use, as
    # a server does at start-up (no capture inside a timed region)
    longest = max(len(s.token_ids) for s in seqs)
    runner.capture_decode_graphs(B, (longest + W + 2 * K + 16) // 16, (longest + 15) // 16)
    for _ in range(W):
        drv.step()
    torch.cuda.synchronize(dev)
    ctx_sum = sum(len(s.token_ids) - 1 for s in seqs)  # tokens cached before the first timed step
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    with clocks:
        # ---- e2e: engine steps through ModelRunner.execute ----------------
        barrier(ws)
        torch.cuda.synchronize(dev)
        h2d0 = runner._stage.bytes_copied
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(st)
        for _ in range(K):
            drv.step()
        s1.record(st)
        torch.cuda.synchronize(dev)
        h2d = (runner._stage.bytes_copied - h2d0) // K
        e2e_ms = max_over_ranks(s0.elapsed_time(s1), ws, dev)
        # ---- value: the decode graph with the step's inputs on the device --
        for s in seqs:   # blocks for the K device steps, as the allocator would hand out
            tbl = drv.tables[s.seq_id]
            while len(tbl) * 16 < len(s.token_ids) + K:
                tbl.append(drv.free.popleft())
        inp = runner._prepare_inputs(SchedulerOutput(
            prefill_seqs=[], decode_seqs=seqs, block_tables=drv.tables, swap_in_map={},
            swap_out_map={}, blocks_to_free=[]))
        merges = _splits(runner, seqs) > 1
        from needle_b200 import ops
        greedy = (torch.zeros(B, dtype=torch.float32, device=dev),
                  torch.zeros(B, dtype=torch.int32, device=dev),
                  torch.ones(B, dtype=torch.float32, device=dev),
                  torch.zeros(B, dtype=torch.float32, device=dev))

        def device_step():
            logits = runner._forward(inp)
            # greedy tokens (the sampler kernel) straight into the next step's ids
            ops.sample(logits, *greedy, out=inp.input_ids)
            inp.position_ids.add_(1)
            inp.context_lens.add_(1)
        device_step()                    # untimed: the graph of this width is warm
        torch.cuda.synchronize(dev)
        barrier(ws)
        torch.cuda.synchronize(dev)
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(st)
        for _ in range(K - 1):
            device_step()
        d1.record(st)
        torch.cuda.synchronize(dev)
        barrier(ws)
        t_ms = max_over_ranks(d0.elapsed_time(d1), ws, dev)
        Kd = K - 1
    if runner.tp_comm is not None:
        runner.tp_comm.check()
    value = B * Kd / (t_ms / 1e3)
    e2e_value = B * K / (e2e_ms / 1e3)
    ms_step = t_ms / Kd
    # ---- per-rank HBM bound of the step (weights + every cached K/V row) ---
    kvh = max(1, cfg.num_key_value_heads // ws)
    kv_tok = 2 * kvh * cfg.head_dim * 2 * cfg.num_hidden_layers
    avg_ctx_bytes = (ctx_sum + B * (K + 1) + B * (Kd + 1) / 2.0) * kv_tok
    w_bytes = _weights_read_per_step(runner)
    step_bytes = w_bytes + avg_ctx_bytes
    peak, peak_src = measured_hbm_peak()
    bound = B * peak * 1e9 / step_bytes
    n_lin = _nb_linear_per_step(runner, B)
    # ---- the all-reduce's share of the step (N > 1) -----------------------
    allreduce = None
    if ws > 1:
        calls = 2 * cfg.num_hidden_layers
        if runner.tp_comm is not None:
            wgt = runner.model.model.layers[0].post_attention_layernorm.weight
            us = _time_fused_allreduce(runner.tp_comm, B, wgt, cfg.rms_norm_eps, dev, ws)
            allreduce = {"kind": "fused all-reduce + residual + RMSNorm over NVLink peer memory",
                         "us_per_call": round(us, 2), "calls_per_step": calls,
                         "share_of_step": round(calls * us / 1e3 / ms_step, 4),
                         "shape": [B, cfg.hidden_size]}
        else:
            allreduce = {"kind": "NCCL", "calls_per_step": calls}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": ws,
            "steps": Kd, "warmup": W, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights and token ids; no checkpoint or dataset)",
            "config": {"workload": f"{name}: {cfg.model_type} {cfg.hidden_size}h/"
                                   f"{cfg.num_hidden_layers}L decode, batch {B}, tp={ws}",
                       "model": args.workload, "batch": B, "tp": ws,
                       "prompt_tokens": sum(len(p) for p in prompts) if prefill else None,
                       "ctx_at_first_timed_step": round(ctx_sum / B, 1),
                       "prefill_ms": round(t_prefill_ms, 1) if t_prefill_ms else None,
                       "parallelism": f"tp{ws}" if ws > 1 else "single GPU",
                       "l2": "inputs larger than L2 (%.1f GB of weights read per step)"
                             % (w_bytes / 1e9),
                       "value_loop": "decode graph replays, greedy token (sampler kernel) fed "
                                     "back on the device",
                       "allreduce": (None if ws == 1 else allreduce["kind"])},
            "roofline": kern["roofline"],
            "step_roofline": {"bound": "hbm", "what": "whole decode step per rank: weights + "
                                                      "every cached K/V row, read once",
                              "achieved": round(step_bytes / (ms_step / 1e3) / 1e9, 1),
                              "peak": peak, "unit": "GB/s", "peak_source": peak_src,
                              "frac": round(value / bound, 4),
                              "bytes_per_step": int(step_bytes), "weights_bytes": int(w_bytes),
                              "tokens_per_s_bound": round(bound, 1)},
            "allreduce": allreduce,
            "kernel_config2": kern["detail"],
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms / K, 4), "steps": K,
                    "path": "ModelRunner.execute(SchedulerOutput): host-built step inputs "
                            "copied from pinned memory, token ids read back every step",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": B * 8},
            "cpu_baseline": None,  # filled in below, after the process group is gone
            # our kernels per decode step: the slot table, the first RMSNorm,
            # per layer the RoPE + KV write, paged decode (+ merge when split),
            # SwiGLU and two fused add+RMSNorm (post-attention, and the next
            # layer's input norm or the final norm; the fused all-reduce under
            # TP), the sampler, and the projections on nb_linear
            "gpu_launches": Kd * (cfg.num_hidden_layers * (5 + (1 if merges else 0)) + 3
                                  + n_lin),
            "nb_linear_per_step": n_lin,
            "clocks": clocks.summary(),
        }
    ctx_now = [len(s.token_ids) - 1 for s in seqs]
    runner.close()
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        if ws == 1 and not args.no_cpu_baseline:
            del runner, drv, inp
            torch.cuda.empty_cache()
            line["cpu_baseline"] = cpu_baseline_model(cfg, ctx_now, args.cpu_seconds)
        print(json.dumps(line), flush=True)


def _cpu_decode_layer(cfg, ctx_lens):
    """needle's decode step for ONE decoder layer of the full (unsharded)
    model on the host cores, at the real batch and context lengths, as
    restated in oracle/ (RMSNorm, the q/k/v/o and MLP GEMMs, RoPE, the decode
    KV write and ``_decode_pytorch``; needle/model/llama.py:61-72,
    needle/layers/attention.py:70-96,140-159,291-310), plus the lm_head GEMM
    over 1/8 of the vocabulary.  Weights and cache hold zeros: the CPU
    kernels' time does not depend on the values.  Returns (layer, head)."""
    import torch.nn.functional as F
    from oracle import needle_oracle as no
    dt = torch.bfloat16
    B = len(ctx_lens)
    H, kv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    hid, inter, eps = cfg.hidden_size, cfg.intermediate_size, cfg.rms_norm_eps
    nb = [(c + 1 + 15) // 16 for c in ctx_lens]   # blocks after the new token's write
    N = sum(nb) + 1
    cache = torch.zeros(2, N, kv, 16, D, dtype=dt)
    bt = torch.full((B, max(nb)), N - 1, dtype=torch.int32)
    o = 0
    for i, n in enumerate(nb):
        bt[i, :n] = torch.arange(o, o + n, dtype=torch.int32)
        o += n
    ctx = torch.tensor(ctx_lens, dtype=torch.int32)
    z = lambda *shape: torch.zeros(*shape, dtype=dt)
    bias = cfg.model_type == "qwen2"
    qw, kw, vw, ow = z(H * D, hid), z(kv * D, hid), z(kv * D, hid), z(hid, H * D)
    qb, kb, vb = (z(H * D), z(kv * D), z(kv * D)) if bias else (None, None, None)
    gw, uw, dw = z(inter, hid), z(inter, hid), z(hid, inter)
    nw = torch.ones(hid, dtype=dt)
    cos_t, sin_t = no.rope_cache(D, max(ctx_lens) + 2, cfg.rope_theta)
    cos, sin = cos_t[ctx.long()].to(dt), sin_t[ctx.long()].to(dt)
    h = torch.randn(B, hid).to(dt)
    scale = no.default_scale(D)

    def layer():
        x = no.rms_norm(h, nw, eps)
        q = F.linear(x, qw, qb).view(B, H, D)
        k = F.linear(x, kw, kb).view(B, kv, D)
        v = F.linear(x, vw, vb).view(B, kv, D)
        q, k = no.apply_rope(q, k, cos, sin)
        no.decode_write_kv(k, v, cache, bt, ctx)
        a = no.decode_attention(q, cache, bt, ctx, scale, H, kv, D)
        h2 = h + F.linear(a.reshape(B, H * D), ow)
        x = no.rms_norm(h2, nw, eps)
        return h2 + F.linear(F.silu(F.linear(x, gw)) * F.linear(x, uw), dw)

    hw = z(-(-cfg.vocab_size // 8), hid)

    def head():
        F.linear(h, hw)
    return layer, head


def cpu_baseline_model(cfg, ctx_lens, budget_s):
    """needle's decode step on the host cores, EXTRAPOLATED from one decoder
    layer (``_cpu_decode_layer``) x the layer count, + lm_head x 8; bounded
    by ``budget_s`` of CPU time."""
    torch.set_num_threads(os.cpu_count() or 1)
    B = len(ctx_lens)
    layer, head = _cpu_decode_layer(cfg, ctx_lens)
    times = []
    t_all = time.time()
    while not times or (time.time() - t_all < budget_s and len(times) < 5):
        t0 = time.time()
        layer()
        times.append(time.time() - t0)
    t_layer = statistics.median(times)
    t0 = time.time()
    head()
    t_head = (time.time() - t0) * 8
    step = cfg.num_hidden_layers * t_layer + t_head
    return {"value": round(B / step, 3), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "extrapolated": True,
            "sample": f"one decoder layer of the full model at B={B}, mean ctx "
                      f"{sum(ctx_lens) / B:.0f}: {len(times)} runs, median {t_layer:.2f} s, "
                      f"x{cfg.num_hidden_layers} layers; lm_head over 1/8 of the vocabulary "
                      f"{t_head / 8:.2f} s x8; step {step:.1f} s"}


def _splits(runner, seqs) -> int:
    """Splits per sequence the decode plan uses for this batch shape."""
    import ctypes
    from needle_b200 import _lib as L
    cfg = runner.model_config
    kvh = max(1, cfg.num_key_value_heads // runner.tp_size)
    maxb = max(len(s.token_ids) for s in seqs) // 16 + 1
    pps, ms = ctypes.c_int(0), ctypes.c_int(0)
    L.check(L.lib().nb_paged_decode_plan(len(seqs), kvh, maxb, 16, ctypes.byref(pps),
                                         ctypes.byref(ms)))
    return ms.value


# ---------------------------------------------------------------------------
# prefill workload: the tcgen05 prefill kernel alone (tensor-pipe roofline)
# ---------------------------------------------------------------------------

def run_prefill(args):
    """Causal prefill attention of ``--prefill-shape`` (default 16 sequences x
    1024 new tokens), 32/8 heads, D=128, bf16 (the config 3 head geometry);
    reports TFLOP/s against the measured dense bf16 peak."""
    rank, local, ws = dist_init(args.gpus)
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    from needle_b200 import ops
    B, S = (int(v) for v in args.prefill_shape.lower().split("x"))
    C = args.prefill_ctx  # cached tokens before each chunk (paged prefill)
    H, KV, D = 32, 8, 128
    g = torch.Generator(device=dev).manual_seed(0)
    T = B * S
    q = torch.randn(T, H, D, device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(T, KV, D, device=dev, generator=g, dtype=torch.bfloat16)
    v = torch.randn(T, KV, D, device=dev, generator=g, dtype=torch.bfloat16)
    cu = torch.arange(0, T + 1, S, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    if C > 0:
        # the paged form: K/V of C cached + S new tokens per sequence in a
        # shuffled block pool, read through the block table
        maxb = (C + S + 15) // 16
        nblk = B * maxb
        cache = torch.randn(2, nblk, KV, 16, D, device=dev, generator=g, dtype=torch.bfloat16)
        bt = torch.randperm(nblk, generator=torch.Generator().manual_seed(0)).view(
            B, maxb).to(device=dev, dtype=torch.int32)
        ctx = torch.full((B,), C, dtype=torch.int32, device=dev)
        call = lambda: ops.prefill_attention_paged(q, cache, bt, ctx, cu, S, out=out)
    else:
        call = lambda: ops.prefill_attention(q, k, v, cu, S, out=out)
    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    K = args.steps
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    with clocks:
        barrier(ws)
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(st)
        for _ in range(K):
            call()
        e0.record(st)
        torch.cuda.synchronize(dev)
        barrier(ws)
    t_ms = max_over_ranks(s0.elapsed_time(e0), ws, dev)
    flops = B * 4 * (S * C + S * (S + 1) / 2) * H * D  # causal QK^T + PV over C + i + 1 keys
    tflops = flops * K / (t_ms / 1e3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        peak, src = 1590.0, "fallback"
    if rank == 0:
        print(json.dumps({
            "metric": "causal prefill attention TFLOP/s", "value": round(tflops, 1),
            "unit": "TFLOP/s", "n_gpus": ws, "steps": K, "warmup": max(3, args.warmup),
            "ms_per_step": round(t_ms / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, N(0,1))",
            "config": {"workload": f"prefill: {B} x {S} new tokens"
                                   + (f" after {C} cached (paged K/V)" if C else "")
                                   + ", 32/8 heads, D=128, causal"},
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tflops / peak, 4),
                         "peak_source": src, "flops_per_call": flops, "traffic": None},
            "gpu_launches": K, "clocks": clocks.summary()}), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_allreduce(args):
    """Per-call latency of the TP all-reduce + residual add + RMSNorm at the
    decode shapes of configs 5 (128 rows x 8192) and 4 (512 x 4096), and a
    16-row case: the fused NVLink kernel against NCCL all-reduce + the
    fused add+RMSNorm kernel.  Each is timed as CUDA-graph replays of 50
    back-to-back calls (device events, max over ranks)."""
    rank, local, ws = dist_init(args.gpus)
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    import torch.distributed as dist
    if ws == 1:  # a one-rank group: the kernel exchanges with itself
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29599")
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
    from needle_b200 import ops
    from needle_b200.layers.tp_comm import TPComm
    calls, reps, W = 50, max(1, args.steps // 50), max(3, args.warmup)
    shapes = [("config5", 128, 8192), ("config4", 512, 4096), ("small", 16, 8192)]
    res = {}
    launches = 0
    for name, T, H in shapes:
        comm = TPComm(T, H, torch.bfloat16, dev)
        g = torch.Generator(device=dev).manual_seed(rank)
        comm.partial.normal_(generator=g)
        comm.residual.normal_(generator=g)
        w = torch.ones(H, dtype=torch.bfloat16, device=dev)
        x = torch.randn(T, H, dtype=torch.bfloat16, device=dev, generator=g)
        r = torch.randn_like(x)
        o = torch.empty_like(x)

        def fused():
            for _ in range(calls):
                comm.allreduce_add_rmsnorm(T, comm.residual[:T], w, 1e-6)

        def nccl():
            for _ in range(calls):
                dist.all_reduce(x)
                ops.fused_add_rmsnorm(x, r, w, 1e-6, out=o, residual_out=r)
        for label, fn in (("fused", fused), ("nccl", nccl)):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream(dev).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            for _ in range(W):
                graph.replay()
            torch.cuda.synchronize(dev)
            barrier(ws)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            us = max_over_ranks(e0.elapsed_time(e1) / (reps * calls) * 1e3, ws, dev)
            res[f"{name}_{label}_us"] = round(us, 2)
            if label == "fused":
                launches += reps * calls
            del graph
        # algorithmic NVLink bytes per rank per call: reduce-scatter push of
        # (W-1)/W of the partial, all-gather push of the residual and normalised rows
        nvl = 3 * (ws - 1) / ws * T * H * 2
        res[f"{name}_nvlink_bytes_per_rank"] = int(nvl)
        barrier(ws)
        comm.close()
    errs = ops.device_errors()
    if rank == 0:
        t = res["config5_fused_us"]
        gbs = res["config5_nvlink_bytes_per_rank"] / (t * 1e-6) / 1e9
        print(json.dumps({
            "metric": "TP all-reduce + residual + RMSNorm, us per call (config 5 decode shape)",
            "value": t, "unit": "us", "n_gpus": ws, "steps": reps * calls, "warmup": W,
            "ms_per_step": round(t / 1e3, 5), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, N(0,1))",
            "config": {"workload": "allreduce: 128 x 8192 (config 5), 512 x 4096 (config 4), "
                                   "16 x 8192 rows per call; CUDA graphs of 50 calls",
                       "parallelism": f"tp{ws}"},
            "roofline": {"bound": "nvlink", "achieved": round(gbs, 1), "peak": 770.0,
                         "unit": "GB/s", "frac": round(gbs / 770.0, 4),
                         "peak_source": "measured peer copy per direction (pool figure)",
                         "traffic": None},
            "shapes": res, "device_errors": errs, "gpu_launches": launches}), flush=True)
    dist.destroy_process_group()


def run_store_kv(args):
    """The prefill-size paged KV write: 8 sequences x 1024 new tokens
    (T = 8192), 8 KV heads, D = 128, bf16, into a 20000-block pool with
    shuffled block tables (`_write_kv`, needle/layers/attention.py:204-246).
    Algorithmic bytes = 2·T·kv·D·2 read + the same written = 64 MiB.  The
    launches rotate over 4 input sets (separate k/v/q tensors and disjoint
    block sets: 256 MiB of K/V traffic, 2x the L2) and are timed back to back
    with one event pair, so no launch finds its data in L2.  The fused RoPE +
    KV write of the same step (q in place, k rotated, K/V stored) is timed
    the same way."""
    rank, local, ws = dist_init(args.gpus)
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    from needle_b200 import ops
    B, S, H, KV, D, N, bs, NS = 8, 1024, 32, 8, 128, 20000, 16, 4
    T = B * S
    g = torch.Generator(device=dev).manual_seed(0)
    mk = lambda h: torch.randn(T, h, D, device=dev, generator=g, dtype=torch.bfloat16)
    ks, vs, qs = [mk(KV) for _ in range(NS)], [mk(KV) for _ in range(NS)], [mk(H) for _ in range(NS)]
    cache = torch.zeros(2, N, KV, bs, D, device=dev, dtype=torch.bfloat16)
    maxb = S // bs
    perm = torch.randperm(N, generator=torch.Generator().manual_seed(0))[:NS * B * maxb]
    bts = [perm[i * B * maxb:(i + 1) * B * maxb].view(B, maxb).to(device=dev, dtype=torch.int32)
           for i in range(NS)]
    ctx = torch.zeros(B, dtype=torch.int32, device=dev)
    cu = torch.arange(0, T + 1, S, dtype=torch.int32, device=dev)
    pos = torch.arange(S, device=dev).repeat(B)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32, device=dev) / D))
    fr = pos[:, None].float() * inv[None, :]
    emb = torch.cat([fr, fr], dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    st = torch.cuda.current_stream(dev)
    W, K = max(3, args.warmup), max(NS, min(args.steps, 200))

    def timed(fn):
        for i in range(W * NS):
            fn(i % NS)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(st)
        for i in range(K):
            fn(i % NS)
        e1.record(st)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / K
    # the forward's slot table of each input set (built once per forward in
    # the model, outside the per-layer writes timed here)
    slots = [ops.slot_mapping(bts[i], ctx, N, bs, cu_seqlens=cu, num_tokens=T)
             for i in range(NS)]
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    with clocks:
        barrier(ws)
        t_store = timed(lambda i: ops.store_kvcache_slots(ks[i], vs[i], cache, slots[i]))
        t_rope = timed(lambda i: ops.rope_store_kvcache_slots(qs[i], ks[i], vs[i], cos, sin,
                                                              cache, slots[i]))
        t_store_r = timed(lambda i: ops.store_kvcache(ks[i], vs[i], cache, bts[i], ctx, cu))
        t_rope_r = timed(lambda i: ops.rope_store_kvcache(qs[i], ks[i], vs[i], cos, sin, cache,
                                                          bts[i], ctx, cu))
        # a plain device copy of the same bytes (32 MiB read + 32 MiB written,
        # rotating over the same four sets): what one launch of this size can
        # reach, next to the kernel
        srcs = [torch.cat([ks[i], vs[i]], dim=0) for i in range(NS)]
        dsts = [torch.empty_like(srcs[i]) for i in range(NS)]
        t_copy = timed(lambda i: dsts[i].copy_(srcs[i]))
        del srcs, dsts
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(K):
            ops.slot_mapping(bts[i % NS], ctx, N, bs, cu_seqlens=cu, num_tokens=T,
                             out=slots[i % NS])
        e1.record(st)
        torch.cuda.synchronize(dev)
        t_map = e0.elapsed_time(e1) / K
        barrier(ws)
    t_store = max_over_ranks(t_store, ws, dev)
    t_rope = max_over_ranks(t_rope, ws, dev)
    t_store_r = max_over_ranks(t_store_r, ws, dev)
    t_rope_r = max_over_ranks(t_rope_r, ws, dev)
    t_copy = max_over_ranks(t_copy, ws, dev)
    peak, src = measured_hbm_peak()
    store_bytes = 2 * (2 * T * KV * D * 2)
    rope_bytes = 2 * T * H * D * 2 + 2 * T * KV * D * 2 + 2 * T * KV * D * 2 + 2 * T * D * 2
    gbs = store_bytes / (t_store * 1e-3) / 1e9
    gb = lambda nbytes, ms: round(nbytes / (ms * 1e-3) / 1e9, 1)
    if rank == 0:
        print(json.dumps({
            "metric": "paged KV write GB/s (prefill-size, T=8192)", "value": round(gbs, 1),
            "unit": "GB/s", "n_gpus": ws, "steps": K, "warmup": W * NS,
            "ms_per_step": round(t_store, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, N(0,1))",
            "config": {"workload": "store-kv: 8 x 1024 new tokens, kv=8, D=128, 20000-block pool, "
                                   "shuffled block tables; 4 rotating input sets (256 MiB of "
                                   "K/V traffic > L2), launches back to back; slot table "
                                   "built once per forward (store_kvcache_slots)"},
            "roofline": {"bound": "hbm", "kernel": "store_kvcache_slots_kernel",
                         "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": src,
                         "bytes_per_launch": store_bytes, "traffic": None},
            "rope_store": {"kernel": "rope_store_slots_kernel", "ms": round(t_rope, 5),
                           "bytes_per_launch": rope_bytes, "GB/s": gb(rope_bytes, t_rope),
                           "frac": round(rope_bytes / (t_rope * 1e-3) / 1e9 / peak, 4)},
            "slot_mapping_ms": round(t_map, 5),
            "same_size_copy": {"what": "torch copy_ of the same 32 MiB of K/V rows",
                               "ms": round(t_copy, 5), "GB/s": gb(store_bytes, t_copy),
                               "frac": round(store_bytes / (t_copy * 1e-3) / 1e9 / peak, 4)},
            "self_resolving": {"store_kvcache_ms": round(t_store_r, 5),
                               "store_GB/s": gb(store_bytes, t_store_r),
                               "rope_store_ms": round(t_rope_r, 5),
                               "rope_store_GB/s": gb(rope_bytes, t_rope_r)},
            "gpu_launches": 5 * K, "clocks": clocks.summary()}), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_step_profile(args):
    """Where a config-3 decode step goes: the captured decode graph replayed
    (as in ``value``) under torch.profiler, CUDA kernel time per step grouped
    by kernel name, next to the CUDA-event time of the same replays without
    the profiler.  One JSON line."""
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    from torch.profiler import ProfilerActivity, profile
    from needle_b200 import ops
    from needle_b200.model import ModelRunner, preset
    from needle_b200.model.driver import BatchDriver, blocks_needed
    from needle_b200.model.sequence import SamplingParams, SchedulerOutput
    cfg = preset("llama3-8b")
    prompts, _ = _model_prompts("llama8b", cfg)
    runner = ModelRunner(cfg, block_size=16, dtype="bfloat16", device=str(dev))
    runner.init_synthetic(seed=0)
    nblk = blocks_needed([len(p) for p in prompts], 257, 16)
    runner.init_kv_cache(nblk, 0)
    drv = BatchDriver(runner, nblk)
    seqs = [drv.add(p, SamplingParams(temperature=0.0, max_new_tokens=256)) for p in prompts]
    drv.step()
    longest = max(len(s.token_ids) for s in seqs)
    runner.capture_decode_graphs(len(seqs), (longest + 64) // 16, (longest + 15) // 16)
    for _ in range(max(3, args.warmup)):
        drv.step()
    for s in seqs:
        tbl = drv.tables[s.seq_id]
        while len(tbl) * 16 < len(s.token_ids) + 24:
            tbl.append(drv.free.popleft())
    inp = runner._prepare_inputs(SchedulerOutput(
        prefill_seqs=[], decode_seqs=seqs, block_tables=drv.tables, swap_in_map={},
        swap_out_map={}, blocks_to_free=[]))
    B = len(seqs)
    greedy = (torch.zeros(B, dtype=torch.float32, device=dev),
              torch.zeros(B, dtype=torch.int32, device=dev),
              torch.ones(B, dtype=torch.float32, device=dev),
              torch.zeros(B, dtype=torch.float32, device=dev))

    def step():
        logits = runner._forward(inp)
        ops.sample(logits, *greedy, out=inp.input_ids)
        inp.position_ids.add_(1)
        inp.context_lens.add_(1)
    for _ in range(3):
        step()
    torch.cuda.synchronize(dev)
    n = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    step_ms = e0.elapsed_time(e1) / n
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            step()
        torch.cuda.synchronize(dev)
    agg = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            a = agg.setdefault(ev.name, [0, 0.0])
            a[0] += 1
            a[1] += ev.device_time_total
    tot = sum(v[1] for v in agg.values())
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    print(json.dumps({
        "metric": "config-3 decode step breakdown (us per step by kernel)",
        "value": round(step_ms, 4), "unit": "ms/step", "n_gpus": 1, "steps": n, "warmup": 3,
        "ms_per_step": round(step_ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "step-profile: config 3 decode graph replay"},
        "kernel_us_per_step_total": round(tot / n, 1),
        "kernels": [{"name": k[:160], "us_per_step": round(v[1] / n, 1),
                     "launches_per_step": v[0] / n, "share": round(v[1] / tot, 4)}
                    for k, v in rows[:24]],
        "gpu_launches": None}), flush=True)
    runner.close()


def run_kernel_cases(args):
    """Per-kernel roofline figures for the kernels around the decode and
    prefill paths, each call timed alone with CUDA events on the launching
    stream after an L2 flush (a 256 MB write), averaged over ``--steps``
    calls: achieved = algorithmic bytes (or FLOPs) / time.  One JSON line."""
    rank, local, ws = dist_init(args.gpus)
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    from needle_b200 import ops
    from needle_b200.synth import decode_op_workload
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *shape: torch.randn(*shape, device=dev, generator=g, dtype=bf)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)
    peak, src = measured_hbm_peak()
    iters = max(5, min(args.steps, 100))
    res = {}

    def case(name, kernels, nbytes, fn, bound="hbm", flops=None):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        tot = 0.0
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            torch.cuda.synchronize(dev)
            tot += e0.elapsed_time(e1)
        ms = tot / iters
        r = {"kernels": kernels, "ms": round(ms, 5), "alg_bytes": int(nbytes),
             "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1)}
        if bound == "hbm":
            r["frac"] = round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)
        if flops:
            r["TFLOP/s"] = round(flops / (ms * 1e-3) / 1e12, 1)
        r["bound"] = bound
        res[name] = r

    H = 4096
    for T, tag in ((256, "decode 256"), (8192, "prefill 8192")):
        x, r, w = rnd(T, H), rnd(T, H), rnd(H)
        o, ro = torch.empty_like(x), torch.empty_like(x)
        case(f"fused_add_rmsnorm {tag} x 4096", "rmsnorm_kernel<ADD>", 4 * T * H * 2 + H * 2,
             lambda: ops.fused_add_rmsnorm(x, r, w, 1e-5, out=o, residual_out=ro))
    x, w = rnd(8192, H), rnd(H)
    o = torch.empty_like(x)
    case("rmsnorm prefill 8192 x 4096", "rmsnorm_kernel", 2 * 8192 * H * 2 + H * 2,
         lambda: ops.rmsnorm(x, w, 1e-5, out=o))
    inter = 14336
    for T, tag in ((256, "decode 256"), (8192, "prefill 8192")):
        gu = rnd(T, 2 * inter)
        o = torch.empty(T, inter, dtype=bf, device=dev)
        case(f"silu_mul {tag} x 14336", "silu_mul_kernel", 3 * T * inter * 2,
             lambda: ops.silu_mul(gu, out=o))
    del x, r, w, o, ro, gu
    # paged decode: config 2 (tensor-core split + merge), GQA group 16 (32
    # query / 2 KV heads: the tensor-core kernel with 16-head tiles) and the
    # SIMT kernel (fp32 cache, config-2 shape)
    for kvh, tag, kern, dt in (
            (8, "config 2 (group 4)", "paged_decode_tc_kernel + decode_merge_kernel", bf),
            (2, "group 16 (32/2 heads)", "paged_decode_tc_kernel + decode_merge_kernel", bf),
            (8, "fp32 config-2 shape (SIMT)", "paged_decode_simt_kernel + decode_merge_kernel",
             torch.float32)):
        wl = decode_op_workload(batch=64, num_heads=32, num_kv_heads=kvh, head_dim=128,
                                block_size=16, dtype=dt, device=dev)
        B, maxb = wl["block_table"].shape
        plan = ops.DecodePlan(B, 32, kvh, 128, maxb, 16, dev)
        out = torch.empty_like(wl["q"])
        case(f"paged_decode {tag}", kern,
             decode_alg_bytes(wl["seq_len"], kvh, 32, 128, wl["q"].element_size()),
             lambda: ops.paged_decode(wl["q"], wl["kv_cache"], wl["block_table"],
                                      wl["context_lens"], wl["scale"], out=out, plan=plan))
        del wl, plan, out
        torch.cuda.empty_cache()
    # the prefill-size slot table
    Bp, S, N = 8, 1024, 20000
    perm = torch.randperm(N, generator=torch.Generator().manual_seed(0))[:Bp * S // 16]
    bt = perm.view(Bp, S // 16).to(device=dev, dtype=torch.int32)
    ctx = torch.zeros(Bp, dtype=torch.int32, device=dev)
    cu = torch.arange(0, Bp * S + 1, S, dtype=torch.int32, device=dev)
    slots = torch.empty(Bp * S, dtype=torch.int32, device=dev)
    case("slot_mapping prefill 8 x 1024", "slot_mapping_prefill_kernel",
         Bp * S * 4 + bt.numel() * 4 + 2 * Bp * 4,
         lambda: ops.slot_mapping(bt, ctx, N, 16, cu_seqlens=cu, num_tokens=Bp * S, out=slots))
    # KV block swap: 32 layers x 64 blocks, device -> pinned host and back
    L_, nb, kv, D = 32, 256, 8, 128
    gpu = [rnd(2, nb, kv, 16, D) for _ in range(L_)]
    cpu = [torch.empty(2, nb, kv, 16, D, dtype=bf).pin_memory() for _ in range(L_)]
    pairs = torch.stack([torch.arange(0, 128, 2), torch.arange(64)], 1).to(torch.int32).to(dev)
    nbytes = L_ * 64 * 2 * kv * 16 * D * 2
    case("swap_kv_blocks gpu->pinned 32 layers x 64 blocks", "swap_blocks_kernel", nbytes,
         lambda: ops.swap_kv_blocks(gpu, cpu, pairs), bound="host link")
    del gpu, cpu
    torch.cuda.empty_cache()
    # the dense projections of a config-3 decode step at M = 256 (cuBLAS
    # through torch, as in the model): weight bytes / time
    for name, (N_, K_) in (("qkv 6144x4096", (6144, 4096)), ("o_proj 4096x4096", (4096, 4096)),
                           ("gate_up 28672x4096", (28672, 4096)),
                           ("down 4096x14336", (4096, 14336)),
                           ("lm_head 128256x4096", (128256, 4096))):
        wgt = rnd(N_, K_)
        xin = rnd(256, K_)
        yout = torch.empty(256, N_, dtype=bf, device=dev)
        case(f"cuBLAS linear M=256 {name}", "cuBLAS (torch F.linear)", N_ * K_ * 2,
             lambda: torch.nn.functional.linear(xin, wgt))
        case(f"nb_linear M=256 {name}", "linear_tc_kernel", N_ * K_ * 2,
             lambda: ops.linear(xin, wgt, out=yout))
        del wgt, xin, yout
    torch.cuda.empty_cache()
    # the batched sampler at the config 3 decode shape (256 x 128256 bf16):
    # greedy rows read the row once; sampled rows (top-k 50, top-p 0.9) make
    # several passes, all but the first from L2
    n, V = 256, 128256
    lg = rnd(n, V)
    ids = torch.empty(n, dtype=torch.int64, device=dev)
    z = torch.zeros(n, dtype=torch.float32, device=dev)
    ki = torch.zeros(n, dtype=torch.int32, device=dev)
    one = torch.ones(n, dtype=torch.float32, device=dev)
    case("sample greedy 256 x 128256", "sample_kernel", n * V * 2 + n * 8,
         lambda: ops.sample(lg, z, ki, one, z, out=ids))
    tt, kk50 = torch.full_like(one, 0.8), torch.full_like(ki, 50)
    p9, u = torch.full_like(one, 0.9), torch.rand(n, device=dev, generator=g)
    case("sample top-k 50 / top-p 0.9 256 x 128256", "sample_kernel", n * V * 2 + n * 8,
         lambda: ops.sample(lg, tt, kk50, p9, u, out=ids))
    del lg
    errs = ops.device_errors()
    if rank == 0:
        print(json.dumps({
            "metric": "per-kernel achieved bandwidth (kernel cases)", "value": None,
            "unit": "GB/s", "n_gpus": ws, "steps": iters, "warmup": 3, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, N(0,1))",
            "config": {"workload": "kernel-cases: each call alone after a 256 MB L2 flush"},
            "peak": peak, "peak_source": src, "cases": res, "device_errors": errs,
            "gpu_launches": None}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "allreduce":
        run_allreduce(args)
    elif args.workload == "store-kv":
        run_store_kv(args)
    elif args.workload == "kernel-cases":
        run_kernel_cases(args)
    elif args.workload == "step-profile":
        run_step_profile(args)
    elif args.workload in MODEL_WORKLOADS:
        run_model(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
