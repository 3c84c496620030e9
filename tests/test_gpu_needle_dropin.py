"""The drop-in proof on needle's OWN classes, on the GPU.

needle (the reference, installed unmodified as ``baseline/_ref``) builds its
own ``ModelRunner`` (``needle/model/runner.py:17-42``), ``Scheduler``,
``BlockAllocator`` and ``LLMEngine`` (``needle/backend/engine.py:110``);
``patch_needle()`` swaps only ``Attention.forward`` and ``RMSNorm.forward`` to
this library.  Config 1 (Qwen2-0.5B shape, fp32, seed-0 synthetic weights,
8 x 128 prompt ids, 65 greedy tokens) then runs on ``cuda:0`` through
needle's engine loop, and its tokens must equal the golden tokens that
needle's own CPU path produced (``tests/golden/e2e_config1.npz``); a
divergence is allowed only where needle's top-2 logit margin is a near-tie.

Skipped when ``baseline/_ref`` is absent (the reference is installed next to
the repository, not into it).
"""
import os
import sys

import numpy as np
import pytest
import torch

from tests.golden.fixtures import load_arrays

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
NEAR_TIE = 0.05   # as tests/test_gpu_model.py: fp32 logits of a random-init model


def _import_needle():
    if not os.path.isdir(os.path.join(REF, "needle")):
        pytest.skip("the reference is not installed in baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import needle  # noqa: F401
    import needle.model  # noqa: F401  (needle.layers.attention alone is a circular import)
    return needle


def test_needle_engine_on_b200_kernels_config1(cuda):
    needle = _import_needle()
    assert needle.__file__.startswith(REF), needle.__file__
    from needle.backend.block_allocator import BlockAllocator
    from needle.backend.engine import LLMEngine
    from needle.backend.scheduler import Scheduler
    from needle.backend.sequence import SamplingParams
    from needle.model.config import ModelConfig as NCfg
    from needle.model.loader import _load_weights_into_model
    from needle.model.runner import ModelRunner as NeedleRunner

    from needle_b200 import ops
    from needle_b200.integration import patch_needle, unpatch_needle
    from needle_b200.model.config import preset
    from needle_b200.synth import synth_state_dict

    g = load_arrays("e2e_config1")
    cfg = preset("qwen2-0.5b")
    ncfg = NCfg(model_type=cfg.model_type, hidden_size=cfg.hidden_size,
                num_hidden_layers=cfg.num_hidden_layers,
                num_attention_heads=cfg.num_attention_heads,
                num_key_value_heads=cfg.num_key_value_heads,
                intermediate_size=cfg.intermediate_size, vocab_size=cfg.vocab_size,
                max_position_embeddings=cfg.max_position_embeddings,
                rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta)
    calls = {"attn": 0}
    patch_needle()
    try:
        import needle.layers.attention as A
        patched = A.Attention.forward

        def counting(self, *a, **k):
            calls["attn"] += 1
            return patched(self, *a, **k)
        A.Attention.forward = counting
        runner = NeedleRunner(ncfg, block_size=16, dtype="float32", device="cuda:0")
        _load_weights_into_model(runner.model, synth_state_dict(cfg, seed=0), ncfg)
        nblocks = 256
        runner.init_kv_cache(nblocks, 0)
        # LLMEngine.__init__ loads a checkpoint from disk; assemble its parts
        # around the runner and use the engine's own add_request / step
        eng = LLMEngine.__new__(LLMEngine)
        eng.block_size = 16
        eng.tensor_parallel_size = 1
        eng.model_runner = runner
        eng.allocator = BlockAllocator(nblocks, 0, 16)
        eng.scheduler = Scheduler(eng.allocator, max_num_seqs=256,
                                  max_num_batched_tokens=1 << 20)
        eng._request_outputs = {}
        prompts = g["prompts"].tolist()
        n_new = g["tokens"].shape[1]
        for i, p in enumerate(prompts):
            eng.add_request(f"r{i}", p, SamplingParams(temperature=0.0, max_new_tokens=n_new))
        results = {}
        while eng.has_unfinished_requests():
            results.update(eng.step())
        torch.cuda.synchronize()
        assert ops.device_errors() == 0
    finally:
        unpatch_needle()
    # every layer of every step ran this library's attention
    assert calls["attn"] == cfg.num_hidden_layers * n_new, calls
    toks = np.array([results[f"r{i}"] for i in range(len(prompts))])
    gold, margins = g["tokens"], g["margins"]
    report = []
    for i in range(gold.shape[0]):
        diff = np.nonzero(toks[i] != gold[i])[0]
        if diff.size:
            t = int(diff[0])
            report.append((i, t, float(margins[t, i])))
    for seq, step, margin in report:
        assert margin < NEAR_TIE, (
            f"sequence {seq} diverges at step {step} where needle's top-2 margin is {margin}")
    assert len(report) <= 1, f"divergences (seq, step, margin): {report}"
