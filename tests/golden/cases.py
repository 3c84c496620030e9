"""Seeded inputs of the golden cases, shared by ``make_golden.py`` and the tests.

Each ``*_inputs`` function rebuilds, from a fixed seed, exactly the tensors the
golden generator fed to needle.  The fixtures therefore store only needle's
outputs plus a checksum of the inputs (``input_crc``), which the tests compare
first so that a change in torch's CPU generator shows up as a clear failure
rather than as a parity mismatch.
"""
from __future__ import annotations

import zlib

import numpy as np
import torch

DTYPES = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}

# (H, kv, D): G=4 D=64, G=7 (Qwen2-0.5B), G=4 D=128, G=8 (72B at tp=8), MHA
DECODE_SHAPES = [(8, 2, 64), (14, 2, 64), (8, 2, 128), (8, 1, 128), (4, 4, 64)]
DECODE_CTX = [0, 15, 16, 17, 100, 47]
PREFILL_SHAPES = [(8, 2, 64), (14, 2, 64), (4, 2, 128), (4, 4, 128)]
PREFILL_LENS = [1, 7, 40, 70]
KV_WRITE_SHAPES = [(2, 64), (3, 128)]
ROPE_SHAPES = [(14, 2, 64, 1e6), (16, 4, 128, 5e5)]
NORM_SHAPES = [(896, 1e-6), (4096, 1e-5)]
# (temperature, top_k, top_p) per row of the sampler case; temperature 0 = greedy
SAMPLER_PARAMS = [(0.0, -1, 1.0), (0.7, 50, 1.0), (1.0, -1, 0.9), (1.3, 5, 0.5),
                  (0.5, 0, 0.95), (2.0, 2000, 0.3), (0.9, 1, 1.0), (0.0, 10, 0.5),
                  (1.0, -1, 1.0), (0.37, 17, 0.8)]
SAMPLER_VOCAB = 1000


def crc(*tensors) -> int:
    c = 0
    for t in tensors:
        t = t.detach().contiguous().cpu()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        c = zlib.crc32(t.numpy().tobytes(), c)
    return c


def kv_write_inputs(dt: str, kv: int, D: int):
    """Five sequences incl. ctx>0 and an empty one, written into a 32-block pool."""
    g = torch.Generator().manual_seed(1)
    lens = [1, 17, 33, 0, 5]
    ctx = [0, 0, 5, 3, 30]
    nblk, maxb = 32, 4
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T = int(cu[-1])
    bt = torch.randperm(nblk, generator=g)[: len(lens) * maxb].view(len(lens), maxb).to(torch.int32)
    k = torch.randn(T, kv, D, generator=g).to(DTYPES[dt])
    v = torch.randn(T, kv, D, generator=g).to(DTYPES[dt])
    cache = torch.randn(2, nblk, kv, 16, D, generator=g).to(DTYPES[dt])
    return dict(k=k, v=v, cache=cache, block_table=bt, cu_seqlens=cu,
                context_lens=torch.tensor(ctx, dtype=torch.int32))


def kv_write_clamp_inputs(dt: str):
    """40 tokens into a 2-column block table: positions >= 16 share column 1."""
    g = torch.Generator().manual_seed(2)
    kv, D = 2, 64
    k = torch.randn(40, kv, D, generator=g).to(DTYPES[dt])
    v = torch.randn(40, kv, D, generator=g).to(DTYPES[dt])
    return dict(k=k, v=v, cache=torch.zeros(2, 8, kv, 16, D, dtype=DTYPES[dt]),
                block_table=torch.tensor([[7, 3]], dtype=torch.int32),
                cu_seqlens=torch.tensor([0, 40], dtype=torch.int32),
                context_lens=torch.tensor([0], dtype=torch.int32))


def decode_inputs(dt: str, H: int, kv: int, D: int):
    g = torch.Generator().manual_seed(3)
    B = len(DECODE_CTX)
    nblk, maxb = 48, 8
    bt = torch.randperm(nblk, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(B, H, D, generator=g).to(DTYPES[dt])
    k = torch.randn(B, kv, D, generator=g).to(DTYPES[dt])
    v = torch.randn(B, kv, D, generator=g).to(DTYPES[dt])
    cache = torch.randn(2, nblk, kv, 16, D, generator=g).to(DTYPES[dt])
    return dict(q=q, k=k, v=v, cache=cache, block_table=bt,
                context_lens=torch.tensor(DECODE_CTX, dtype=torch.int32))


def prefill_inputs(dt: str, H: int, kv: int, D: int):
    g = torch.Generator().manual_seed(4)
    lens = PREFILL_LENS
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T, B = int(cu[-1]), len(lens)
    nblk, maxb = 48, 9
    bt = torch.randperm(nblk, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = torch.randn(T, H, D, generator=g).to(DTYPES[dt])
    k = torch.randn(T, kv, D, generator=g).to(DTYPES[dt])
    v = torch.randn(T, kv, D, generator=g).to(DTYPES[dt])
    return dict(q=q, k=k, v=v, cache=torch.zeros(2, nblk, kv, 16, D, dtype=DTYPES[dt]),
                block_table=bt, cu_seqlens=cu, context_lens=torch.zeros(B, dtype=torch.int32),
                max_seqlen=max(lens))


def rope_inputs(dt: str, H: int, kv: int, D: int):
    """q/k and the positions; the cos/sin tables come from the rope module."""
    g = torch.Generator().manual_seed(5)
    T = 17
    pos = torch.randint(0, 4096, (T,), generator=g)
    q = torch.randn(T, H, D, generator=g).to(DTYPES[dt])
    k = torch.randn(T, kv, D, generator=g).to(DTYPES[dt])
    return dict(q=q, k=k, positions=pos)


def norm_inputs(dt: str, hid: int):
    g = torch.Generator().manual_seed(6)
    T = 7
    w = (torch.rand(hid, generator=g) + 0.5).to(DTYPES[dt])
    x = (torch.randn(T, hid, generator=g) * 3).to(DTYPES[dt])
    res = (torch.randn(T, hid, generator=g) * 3).to(DTYPES[dt])
    return dict(x=x, residual=res, weight=w)


def sampler_inputs(dt: str):
    """Logits ``[rows, vocab]`` for the sampler case, with a block of ties."""
    g = torch.Generator().manual_seed(606)
    logits = (3 * torch.randn(len(SAMPLER_PARAMS), SAMPLER_VOCAB, generator=g)).to(DTYPES[dt])
    logits[3, 10:20] = logits[3, 10]
    return {"logits": logits}
