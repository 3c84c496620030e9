"""Fused TP all-reduce + residual add + RMSNorm over NVLink peer memory.

Two ranks (one process per GPU) share their buffers through CUDA IPC
(``TPComm``).  Every rank regenerates every rank's partial sums from seeds, so
the expected result is computed on the CPU:

* the new residual is ``rnd(residual + rnd(sum_p partial_p))`` with the fp32
  sum taken in rank order; the kernel does the same adds in the same order,
  so it must be bit-identical;
* the normalised output follows needle's RMSNorm (``needle/layers/norm.py``);
  the fp32 sum of squares runs in another order, so it is compared within one
  bf16 ulp (tolerance 2e-2 absolute on values of order 1-4);
* both ranks must hold identical bits (each owner computes its rows once and
  pushes them to every rank).

Calls of different row counts exercise the per-row call counters and the
double-buffered slots; a partial holding the exchange's sentinel NaN pattern
must come out as a NaN; a CUDA graph replays the launch with new data; 10^4
calls cycle through every launch shape; a rank that skips a call makes the
other's bounded wait run out, which poisons the communicator until a
collective reset.  The model test runs a TP=2 bf16 decode with the fused path
and with NCCL and compares the logits.  NVLS is off for these multi-process
runs.  Skipped with fewer than two GPUs.
"""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

HIDDEN = 1024
# ranks of the op, mixed-shape and stress tests (NB_TP_TEST_WORLD, default 2;
# 4 or 8 on a box with that many GPUs)
WORLD = int(os.environ.get("NB_TP_TEST_WORLD", "2"))
EPS = 1e-6
ROWS = [1, 7, 64, 33, 2, 64]


def _inputs(T, call, world, hidden=HIDDEN):
    g = torch.Generator().manual_seed(1000 * call + T)
    parts = [torch.randn(T, hidden, generator=g).to(torch.bfloat16) for _ in range(world)]
    res = torch.randn(T, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    return parts, res, w


def _expected(parts, res, w):
    from oracle.needle_oracle import rms_norm
    acc = torch.zeros(parts[0].shape, dtype=torch.float32)
    for p in parts:
        acc = acc + p.float()
    h = res + acc.to(torch.bfloat16)
    return rms_norm(h, w, EPS), h


def _op_worker(rank, world, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device(f"cuda:{rank}")
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        from needle_b200 import ops
        from needle_b200.layers.tp_comm import TPComm
        comm = TPComm(64, HIDDEN, torch.bfloat16, dev)
        report = []

        def check(T, call, out, h):
            parts, res, w = _inputs(T, call, world)
            y_ref, h_ref = _expected(parts, res, w)
            out_c, h_c = out.cpu(), h.cpu()
            # rank 0's bits, to compare ranks against each other
            both = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(both, out.contiguous())
            same = all(torch.equal(both[0], b) for b in both)
            report.append((T, call, torch.equal(h_c, h_ref),
                           float((out_c.float() - y_ref.float()).abs().max()), same))

        for call, T in enumerate(ROWS):
            parts, res, w = _inputs(T, call, world)
            comm.partial[:T].copy_(parts[rank])
            wd = w.to(dev)
            out, h = comm.allreduce_add_rmsnorm(T, res.to(dev), wd, EPS)
            check(T, call, out, h)

        # a partial holding the exchange's sentinel bit pattern (a NaN) must
        # arrive as a NaN, not stall the exchange
        T = 5
        parts, res, w = _inputs(T, 50, world)
        p_local = parts[rank].clone()
        if rank == 0:
            p_local.view(torch.int16)[2, 17] = -1  # 0xFFFF
        comm.partial[:T].copy_(p_local)
        out, h = comm.allreduce_add_rmsnorm(T, res.to(dev), w.to(dev), EPS)
        y_ref, h_ref = _expected(parts, res, w)
        h_c, out_c = h.cpu(), out.cpu()
        other = [0, 1, 3, 4]
        report.append((T, 50, bool(torch.isnan(h_c[2, 17]) and torch.isnan(out_c[2]).all()
                                   and torch.equal(h_c[other], h_ref[other])),
                       float((out_c[other].float() - y_ref[other].float()).abs().max()), True))

        # CUDA graph: capture one launch (plus the copies feeding it), replay with new data
        T = 48
        src = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device=dev)
        rsrc = torch.empty_like(src)
        wd = torch.empty(HIDDEN, dtype=torch.bfloat16, device=dev)
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up: one launch outside the graph on every rank
            comm.partial[:T].copy_(src)
            comm.allreduce_add_rmsnorm(T, rsrc, wd, EPS)
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.cuda.graph(graph):
            comm.partial[:T].copy_(src)
            g_out, g_h = comm.allreduce_add_rmsnorm(T, rsrc, wd, EPS)
        for call in range(100, 103):
            parts, res, w = _inputs(T, call, world)
            src.copy_(parts[rank])
            rsrc.copy_(res)
            wd.copy_(w)
            graph.replay()
            check(T, call, g_out, g_h)
        torch.cuda.synchronize(dev)
        errs = ops.device_errors()
        del graph
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, (report, errs)))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def _run(target, world, extra=()):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=target, args=(r, world, port, q) + tuple(extra))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
    return res


def test_fused_allreduce_rmsnorm_matches_cpu(cuda):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    res = _run(_op_worker, WORLD)
    for r, (report, errs) in res.items():
        assert errs == 0, (r, errs)
        assert len(report) == len(ROWS) + 4
        for T, call, h_exact, y_err, same in report:
            assert h_exact, (r, T, call, "residual not bit-identical")
            assert y_err <= 2e-2, (r, T, call, y_err)
            assert same, (r, T, call, "ranks disagree")


# hidden 8192: one 1024-thread CTA per SM, so 148 resident CTAs.  200 rows over
# 2 ranks (100 row indices) run without the second receive role, 300 rows
# (150 indices) also loop over indices in a CTA, 16 and 7 rows split: the
# sequence mixes all three launch shapes.
MIXED_H = 8192
MIXED_ROWS = [200, 16, 300, 16, 7, 200, 16]


def _mixed_worker(rank, world, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device(f"cuda:{rank}")
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        from needle_b200 import ops
        from needle_b200.layers.tp_comm import TPComm
        comm = TPComm(max(MIXED_ROWS), MIXED_H, torch.bfloat16, dev)
        report = []
        for call, T in enumerate(MIXED_ROWS):
            parts, res, w = _inputs(T, call, world, MIXED_H)
            comm.partial[:T].copy_(parts[rank])
            out, h = comm.allreduce_add_rmsnorm(T, res.to(dev), w.to(dev), EPS)
            y_ref, h_ref = _expected(parts, res, w)
            report.append((T, torch.equal(h.cpu(), h_ref),
                           float((out.cpu().float() - y_ref.float()).abs().max())))
        torch.cuda.synchronize(dev)
        errs = ops.device_errors()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, (report, errs)))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_fused_allreduce_mixed_launch_shapes(cuda):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    res = _run(_mixed_worker, WORLD)
    for r, (report, errs) in res.items():
        assert errs == 0, (r, errs)
        for T, h_exact, y_err in report:
            assert h_exact, (r, T, "residual not bit-identical")
            assert y_err <= 2e-2, (r, T, y_err)


STRESS_ROWS = [7, 16, 200, 300]   # split, split, non-split, non-split with index loops
STRESS_CALLS = 10000


def _stress_worker(rank, world, port, q):
    """10^4 calls cycling through launch shapes with and without the second
    receive role; every 997th call is checked against the CPU result."""
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device(f"cuda:{rank}")
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        from needle_b200 import ops
        from needle_b200.layers.tp_comm import TPComm
        comm = TPComm(max(STRESS_ROWS), MIXED_H, torch.bfloat16, dev)
        sets = {}
        for T in STRESS_ROWS:
            parts, res, w = _inputs(T, 7, world, MIXED_H)
            y_ref, h_ref = _expected(parts, res, w)
            sets[T] = (parts[rank].to(dev), res.to(dev), w.to(dev), y_ref, h_ref)
        bad = []
        checked = 0
        for i in range(STRESS_CALLS):
            T = STRESS_ROWS[(i * 7 + i // 3) % len(STRESS_ROWS)]
            part, res, w, y_ref, h_ref = sets[T]
            comm.partial[:T].copy_(part)
            out, h = comm.allreduce_add_rmsnorm(T, res, w, EPS)
            if i % 997 == 0 or i == STRESS_CALLS - 1:
                checked += 1
                if not torch.equal(h.cpu(), h_ref) or \
                        float((out.cpu().float() - y_ref.float()).abs().max()) > 2e-2:
                    bad.append((i, T))
        torch.cuda.synchronize(dev)
        errs = ops.device_errors()
        poisoned = comm.poisoned()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, (bad, checked, errs, poisoned)))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_fused_allreduce_stress_mixed_shapes(cuda):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    res = _run(_stress_worker, WORLD)
    for r, (bad, checked, errs, poisoned) in res.items():
        assert errs == 0 and not poisoned, (r, errs)
        assert checked >= 10 and not bad, (r, bad)


def _poison_worker(rank, world, port, q):
    """Rank 1 skips one call.  Rank 0's wait on it runs out (0.2 s limit):
    the kernel reports NB_DEVERR_TIMEOUT, the communicator is poisoned and
    refuses the next call on the host.  Rank 1's next call then also times
    out.  After TPComm.reset() on both ranks a call is exact again."""
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device(f"cuda:{rank}")
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        from needle_b200 import ops
        from needle_b200.layers.tp_comm import TPComm, TPCommError, set_wait_limit
        set_wait_limit(0.2)
        comm = TPComm(64, HIDDEN, torch.bfloat16, dev)
        log = {}

        def call(T, seed):
            parts, res, w = _inputs(T, seed, world)
            comm.partial[:T].copy_(parts[rank])
            out, h = comm.allreduce_add_rmsnorm(T, res.to(dev), w.to(dev), EPS)
            torch.cuda.synchronize(dev)
            y_ref, h_ref = _expected(parts, res, w)
            return torch.equal(h.cpu(), h_ref) and \
                float((out.cpu().float() - y_ref.float()).abs().max()) <= 2e-2

        log["good_before"] = call(16, 1)
        log["errs_before"] = ops.device_errors()
        dist.barrier()
        if rank == 0:
            call(16, 2)                         # rank 1 never makes this call
            log["poisoned_after_skip"] = comm.poisoned()
            log["errs_after_skip"] = ops.device_errors()
        dist.barrier()
        try:
            call(16, 3)
            log["next_call"] = "ran"
        except TPCommError:
            log["next_call"] = "refused"
        log["poisoned_end"] = comm.poisoned()
        log["errs_end"] = ops.device_errors()
        comm.reset()
        log["poisoned_after_reset"] = comm.poisoned()
        log["good_after_reset"] = call(16, 4) and call(48, 5)
        log["errs_after_reset"] = ops.device_errors()
        set_wait_limit(0)
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, log))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_fused_allreduce_timeout_poisons_until_reset(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    TIMEOUT = 4  # NB_DEVERR_TIMEOUT
    res = _run(_poison_worker, 2)
    r0, r1 = res[0], res[1]
    for log in (r0, r1):
        assert log["good_before"] and log["errs_before"] == 0, log
        assert log["poisoned_end"], log
        assert log["errs_end"] & TIMEOUT or log.get("errs_after_skip", 0) & TIMEOUT, log
        assert not log["poisoned_after_reset"], log
        assert log["good_after_reset"] and log["errs_after_reset"] == 0, log
    assert r0["poisoned_after_skip"] and r0["errs_after_skip"] & TIMEOUT, r0
    assert r0["next_call"] == "refused", r0      # refused on the host, nothing launched
    assert r1["next_call"] == "ran", r1          # launched, timed out on the device


def _model_worker(rank, world, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device(f"cuda:{rank}")
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        from needle_b200.model.config import ModelConfig
        from needle_b200.model.driver import BatchDriver
        from needle_b200.model.runner import ModelRunner
        from needle_b200.model.sequence import SamplingParams
        from needle_b200.synth import synth_state_dict
        cfg = ModelConfig(model_type="qwen2", hidden_size=1024, num_hidden_layers=2,
                          num_attention_heads=16, num_key_value_heads=4, intermediate_size=2048,
                          vocab_size=1000, max_position_embeddings=1024, rms_norm_eps=1e-6,
                          rope_theta=1e6)
        sd = synth_state_dict(cfg, seed=0)
        prompts = [[(5 * i + 3 * j) % 1000 for j in range(n)] for i, n in enumerate([30, 70, 5])]
        out = {}
        for mode, fused_tokens in (("fused", 1024), ("nccl", 0)):
            r = ModelRunner(cfg, block_size=16, dtype="bfloat16", device=str(dev),
                            tensor_parallel_size=world, tp_rank=rank,
                            tp_fused_tokens=fused_tokens)
            assert (r.tp_comm is not None) == (mode == "fused")
            r.load_state_dict(sd)
            r.init_kv_cache(32, 0)
            d = BatchDriver(r, 32)
            logits = []
            orig = r._forward  # eager prefill, CUDA-graph decode

            def fwd(inp, orig=orig, logits=logits):
                y = orig(inp)
                logits.append(y.float().cpu())
                return y
            r._forward = fwd
            p = SamplingParams(temperature=0.0, max_new_tokens=4)
            for x in prompts:
                d.add(x, p)
            for _ in range(4):
                d.step()
            out[mode] = logits
            r.close()
            del r, d
        dist.barrier()
        dist.destroy_process_group()
        rel = [float((a - b).norm() / b.norm()) for a, b in zip(out["fused"], out["nccl"])]
        q.put((rank, rel))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_tp2_fused_allreduce_model_matches_nccl(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run(_model_worker, 2)
    for r, rel in res.items():
        assert len(rel) == 4, (r, rel)
        # bf16 model: the fused kernel sums in fp32 and rounds once, NCCL
        # rounds per step; the logits agree to bf16 noise
        assert max(rel) < 2e-2, (r, rel)
