"""Generate the golden vectors that pin the oracle to needle itself.

Run once, in a container that has the needle sources (this is the only
script in the repository that imports needle):

    python tests/golden/make_golden.py --needle-src <path to a needle checkout>

It runs needle's OWN code on CPU -- ``Attention._decode`` and
``Attention._prefill`` (KV write + attention), ``_write_kv``,
``_apply_rope`` with ``RotaryEmbedding`` tables, ``RMSNorm`` with the
decoder's residual add, ``Sampler.sample`` (the probabilities it hands to
``torch.multinomial``, captured), and for the end-to-end case ``LLMEngine.step`` over
``Scheduler`` / ``BlockAllocator`` / ``ModelRunner`` -- on the seeded inputs of
``cases.py`` and stores needle's outputs next to this file as ``.npz``.

Stored per case: a CRC of the inputs, needle's outputs, and for KV-cache
writes the list of cache rows that changed (row index into the cache viewed
as ``[2 * num_blocks * num_kv_heads * block_size, head_dim]``) with a CRC of
their new contents.  bf16 tensors are stored as uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from needle_b200.model.config import preset  # noqa: E402
from needle_b200.synth import synth_state_dict, synth_prompts  # noqa: E402
from tests.golden import cases as C  # noqa: E402
from tests.golden.fixtures import pack  # noqa: E402


def _needle(src):
    sys.path.insert(0, src)
    import needle  # noqa: F401  (needle.layers.attention alone is a circular import)
    import needle.model  # noqa: F401
    from needle.layers import attention as A
    from needle.layers.rope import RotaryEmbedding
    from needle.layers.norm import RMSNorm
    from needle.model.config import ModelConfig
    return A, RotaryEmbedding, RMSNorm, ModelConfig


def _attn(A, ModelConfig, H, kv, D):
    cfg = ModelConfig(hidden_size=H * D, num_attention_heads=H, num_key_value_heads=kv,
                      num_hidden_layers=1, intermediate_size=16, vocab_size=16)
    return A.Attention(cfg, 0)


def changed_rows(before: torch.Tensor, after: torch.Tensor):
    D = before.shape[-1]
    b = before.reshape(-1, D)
    a = after.reshape(-1, D)
    bits = torch.int16 if a.dtype == torch.bfloat16 else torch.int32
    diff = (a.view(bits) != b.view(bits)).any(dim=1).nonzero().flatten()
    return dict(changed_idx=diff.to(torch.int64), changed_crc=torch.tensor(C.crc(a[diff])))


def kv_write_cases(A):
    out = {}
    for dt in ("bfloat16", "float32"):
        for (kv, D) in C.KV_WRITE_SHAPES:
            x = C.kv_write_inputs(dt, kv, D)
            crc = C.crc(*x.values())
            before = x["cache"].clone()
            A._write_kv(x["k"], x["v"], x["cache"], x["block_table"], x["cu_seqlens"],
                        x["context_lens"])
            out[f"write_kv_{dt}_kv{kv}_d{D}"] = dict(
                input_crc=torch.tensor(crc), **changed_rows(before, x["cache"]))
        x = C.kv_write_clamp_inputs(dt)
        crc = C.crc(*x.values())
        before = x["cache"].clone()
        A._write_kv(x["k"], x["v"], x["cache"], x["block_table"], x["cu_seqlens"],
                    x["context_lens"])
        out[f"write_kv_clamp_{dt}"] = dict(input_crc=torch.tensor(crc),
                                           **changed_rows(before, x["cache"]))
    return out


def decode_cases(A, ModelConfig):
    out = {}
    for dt in ("bfloat16", "float32"):
        for (H, kv, D) in C.DECODE_SHAPES:
            x = C.decode_inputs(dt, H, kv, D)
            crc = C.crc(*x.values())
            before = x["cache"].clone()
            attn = _attn(A, ModelConfig, H, kv, D)
            o = attn._decode(x["q"], x["k"], x["v"], x["cache"], x["block_table"],
                             x["context_lens"])
            out[f"decode_{dt}_h{H}_kv{kv}_d{D}"] = dict(
                input_crc=torch.tensor(crc), out=o, **changed_rows(before, x["cache"]))
    return out


def prefill_cases(A, ModelConfig):
    out = {}
    for dt in ("bfloat16", "float32"):
        for (H, kv, D) in C.PREFILL_SHAPES:
            x = C.prefill_inputs(dt, H, kv, D)
            crc = C.crc(*[t for t in x.values() if isinstance(t, torch.Tensor)])
            before = x["cache"].clone()
            attn = _attn(A, ModelConfig, H, kv, D)
            o = attn._prefill(x["q"], x["k"], x["v"], x["cache"], x["block_table"],
                              x["cu_seqlens"], x["context_lens"], x["max_seqlen"])
            out[f"prefill_{dt}_h{H}_kv{kv}_d{D}"] = dict(
                input_crc=torch.tensor(crc), out=o, **changed_rows(before, x["cache"]))
    return out


def rope_cases(A, RotaryEmbedding):
    out = {}
    for dt in ("bfloat16", "float32"):
        for (H, kv, D, base) in C.ROPE_SHAPES:
            x = C.rope_inputs(dt, H, kv, D)
            rope = RotaryEmbedding(D, 4096, base).to(C.DTYPES[dt])
            cos, sin = rope.get_cos_sin(x["positions"])
            qo, ko = A._apply_rope(x["q"], x["k"], cos, sin)
            out[f"rope_{dt}_d{D}"] = dict(input_crc=torch.tensor(C.crc(*x.values())),
                                         cos=cos, sin=sin, q_out=qo, k_out=ko)
    return out


def norm_cases(RMSNorm):
    out = {}
    for dt in ("bfloat16", "float32"):
        for (hid, eps) in C.NORM_SHAPES:
            x = C.norm_inputs(dt, hid)
            norm = RMSNorm(hid, eps).to(C.DTYPES[dt])
            with torch.no_grad():
                norm.weight.copy_(x["weight"])
                y = norm(x["x"])
                h = x["residual"] + x["x"]          # llama.py:67
                y2 = norm(h)
            out[f"norm_{dt}_h{hid}"] = dict(input_crc=torch.tensor(C.crc(*x.values())),
                                           y=y, h=h, y_add=y2)
    return out


def sampler_cases(src):
    """needle's ``Sampler.sample`` on seeded logits: the greedy ids and, for
    every sampled row, the probability vector it passes to
    ``torch.multinomial`` (captured by wrapping that function)."""
    sys.path.insert(0, src)
    from needle.model.sampler import Sampler
    from needle.backend.sequence import SamplingParams
    out = {}
    for dt in ("bfloat16", "float32"):
        x = C.sampler_inputs(dt)
        params = [SamplingParams(temperature=t, top_k=k, top_p=p) for t, k, p in C.SAMPLER_PARAMS]
        seen = []
        real = torch.multinomial

        def capture(probs, num_samples, *a, **kw):
            seen.append(probs.clone())
            return real(probs, num_samples, *a, **kw)
        torch.multinomial = capture
        try:
            ids = Sampler().sample(x["logits"], params)
        finally:
            torch.multinomial = real
        greedy = [i for i, (t, _, _) in enumerate(C.SAMPLER_PARAMS) if t == 0.0]
        out[f"sampler_{dt}"] = dict(input_crc=torch.tensor(C.crc(*x.values())),
                                    greedy_rows=torch.tensor(greedy),
                                    greedy_ids=torch.tensor([ids[i] for i in greedy]),
                                    probs=torch.stack(seen))
    return out


def e2e_config1(num_prompts=8, prompt_len=128, new_tokens=65):
    """Config 1: Qwen2-0.5B shape, fp32, synthetic seed-0 weights, 8 x 128
    prompt ids, 65 greedy tokens (one from the prefill, then 64 decode steps),
    driven through needle's own LLMEngine.step / Scheduler / BlockAllocator /
    ModelRunner on CPU."""
    from needle.model.config import ModelConfig as NCfg
    from needle.model.runner import ModelRunner
    from needle.model.loader import _load_weights_into_model
    from needle.backend.engine import LLMEngine
    from needle.backend.block_allocator import BlockAllocator
    from needle.backend.scheduler import Scheduler
    from needle.backend.sequence import SamplingParams

    cfg = preset("qwen2-0.5b")
    ncfg = NCfg(model_type=cfg.model_type, hidden_size=cfg.hidden_size,
                num_hidden_layers=cfg.num_hidden_layers,
                num_attention_heads=cfg.num_attention_heads,
                num_key_value_heads=cfg.num_key_value_heads,
                intermediate_size=cfg.intermediate_size, vocab_size=cfg.vocab_size,
                max_position_embeddings=cfg.max_position_embeddings,
                rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta)
    sd = synth_state_dict(cfg, seed=0)
    runner = ModelRunner(ncfg, block_size=16, dtype="float32", device="cpu")
    _load_weights_into_model(runner.model, sd, ncfg)
    nblocks = 256
    runner.init_kv_cache(nblocks, 0)
    margins = []
    orig = runner.sampler.sample

    def sample(logits, params):
        t2 = logits.float().topk(2, dim=-1).values
        margins.append((t2[:, 0] - t2[:, 1]).tolist())
        return orig(logits, params)
    runner.sampler.sample = sample
    # LLMEngine.__init__ loads a checkpoint from disk; assemble the same parts
    # around the runner instead and use the engine's own add_request/step.
    eng = LLMEngine.__new__(LLMEngine)
    eng.block_size = 16
    eng.tensor_parallel_size = 1
    eng.model_runner = runner
    eng.allocator = BlockAllocator(nblocks, 0, 16)
    eng.scheduler = Scheduler(eng.allocator, max_num_seqs=256, max_num_batched_tokens=1 << 20)
    eng._request_outputs = {}
    prompts = synth_prompts(num_prompts, prompt_len, prompt_len, cfg.vocab_size, seed=0)
    for i, p in enumerate(prompts):
        eng.add_request(f"r{i}", p, SamplingParams(temperature=0.0, max_new_tokens=new_tokens))
    results = {}
    t0 = time.time()
    while eng.has_unfinished_requests():
        results.update(eng.step())
    secs = time.time() - t0
    tokens = np.array([results[f"r{i}"] for i in range(num_prompts)], dtype=np.int64)
    return dict(tokens=tokens, prompts=np.array(prompts, dtype=np.int64),
                margins=np.array(margins, dtype=np.float64)), secs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--needle-src", required=True, help="path of a needle checkout")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--only", default=None, help="regenerate one fixture file (e.g. sampler)")
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    A, RotaryEmbedding, RMSNorm, ModelConfig = _needle(args.needle_src)
    if args.only == "sampler":
        with open(os.path.join(HERE, "MANIFEST.json")) as f:
            meta = json.load(f)
        cases = sampler_cases(args.needle_src)
        np.savez_compressed(os.path.join(HERE, "sampler.npz"), **pack(cases))
        meta["sampler"] = sorted(cases)
        with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
            json.dump(meta, f, indent=1, sort_keys=True)
        return
    meta = {}
    with torch.no_grad():
        for name, cases in (("kv_write", kv_write_cases(A)),
                            ("decode", decode_cases(A, ModelConfig)),
                            ("prefill", prefill_cases(A, ModelConfig)),
                            ("rope", rope_cases(A, RotaryEmbedding)),
                            ("norm", norm_cases(RMSNorm)),
                            ("sampler", sampler_cases(args.needle_src))):
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **pack(cases))
            meta[name] = sorted(cases)
        if not args.skip_e2e:
            e2e, secs = e2e_config1()
            np.savez_compressed(os.path.join(HERE, "e2e_config1.npz"), **e2e)
            meta["e2e_config1"] = {"needle_cpu_seconds": round(secs, 2),
                                   "min_top2_margin": float(e2e["margins"].min())}
    meta["torch"] = torch.__version__
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print(json.dumps(meta, indent=1)[:1500])


if __name__ == "__main__":
    main()
