"""Tensor parallelism on real GPUs: TP=2 against TP=1 on the same weights.

Two ranks (one process per GPU, NCCL) each build ModelRunner(tp=2, rank=r),
load the same full synthetic state dict (sharded by needle's rule), and run
a prefill plus greedy decode steps through the B200 kernels with the
row-parallel all-reduce.  Rank 0's greedy tokens and first-step logits must
match a single-GPU TP=1 run.  fp32 keeps GEMM/all-reduce rounding far below
the logit margins.  NVLS is disabled (NCCL_NVLS_ENABLE=0) as the pool's
rules ask for multi-process GPU tests.  Skipped with fewer than two GPUs.
"""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from needle_b200.model.config import ModelConfig
    return ModelConfig(model_type="qwen2", hidden_size=512, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2, intermediate_size=512,
                       vocab_size=1000, max_position_embeddings=1024, rms_norm_eps=1e-6,
                       rope_theta=1e6)


PROMPTS = [[(3 * i + 7 * j) % 1000 for j in range(n)] for i, n in enumerate([40, 17, 90])]
NEW = 12


def _generate(tp, rank):
    from needle_b200.model.driver import BatchDriver
    from needle_b200.model.runner import ModelRunner
    from needle_b200.synth import synth_state_dict
    cfg = _cfg()
    r = ModelRunner(cfg, block_size=16, dtype="float32", device=f"cuda:{rank}",
                    tensor_parallel_size=tp, tp_rank=rank, cuda_graph=False)
    r.load_state_dict(synth_state_dict(cfg, seed=0))
    r.init_kv_cache(64, 0)
    d = BatchDriver(r, 64)
    from needle_b200.model.sequence import SamplingParams
    p = SamplingParams(temperature=0.0, max_new_tokens=NEW)
    seqs = [d.add(x, p) for x in PROMPTS]
    for _ in range(NEW):
        d.step()
    return [s.token_ids[len(x):] for s, x in zip(seqs, PROMPTS)]


def _worker(rank, port, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device(f"cuda:{rank}"))
        toks = _generate(2, rank)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, toks))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_tp2_matches_tp1(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ref = _generate(1, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert res[r] == ref, (r, res[r], ref)
