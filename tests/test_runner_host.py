"""ModelRunner's host-side input preparation on CPU against the oracle's
restatement of needle's ``_prepare_inputs`` (``needle/model/runner.py:194-249``).

The runner pads block-table rows with its reserved padding block instead of
needle's last pool block (a block no sequence owns, so decode never reads
it); everything else must be identical: ids, positions, cu_seqlens,
context_lens and the table entries each sequence owns.
"""
import random

import numpy as np
import torch

from needle_b200.model import steppack
from needle_b200.model.runner import ModelRunner
from needle_b200.model.sequence import (Request, SamplingParams, SchedulerOutput, Sequence,
                                         SequenceStatus)
from oracle import model_oracle as mo


class _HostRunner:
    """Just the host half of ModelRunner (no device)."""
    block_size = 16
    padding_block = 999
    _prepare_inputs = ModelRunner._prepare_inputs

    def _h2d_many(self, arrays, table=None):
        out = [torch.from_numpy(np.ascontiguousarray(a)) for a in arrays]
        if table is not None:
            out.append(torch.from_numpy(steppack.block_table_np(*table)))
        return out


def _seq(sid, tokens, generated):
    s = Sequence(seq_id=sid, request=Request(str(sid), list(tokens[:len(tokens) - generated]),
                                             SamplingParams(temperature=0.0)),
                 token_ids=list(tokens), logical_blocks=[], block_size=16,
                 status=SequenceStatus.RUNNING)
    s.num_generated_tokens = generated
    return s


def _check(prefill, decode, tables):
    r = _HostRunner()
    got = r._prepare_inputs(SchedulerOutput(prefill_seqs=list(prefill), decode_seqs=list(decode),
                                            block_tables=tables, swap_in_map={},
                                            swap_out_map={}, blocks_to_free=[]))
    seqs = [dict(id=s.seq_id, tokens=s.token_ids, generated=s.num_generated_tokens)
            for s in list(prefill) + list(decode)]
    ref = mo.prepare_inputs(seqs, tables, num_gpu_blocks=1000)
    assert torch.equal(got.input_ids, ref["input_ids"])
    assert torch.equal(got.position_ids, ref["positions"])
    assert torch.equal(got.cu_seqlens, ref["cu_seqlens"])
    assert torch.equal(got.context_lens, ref["context_lens"])
    assert got.block_table.shape == ref["block_table"].shape
    for i, s in enumerate(seqs):
        n = len(tables[s["id"]])
        assert torch.equal(got.block_table[i, :n], ref["block_table"][i, :n])
        assert bool((got.block_table[i, n:] == 999).all())


def test_prepare_inputs_decode_batch_ragged_tables():
    rnd = random.Random(0)
    decode, tables = [], {}
    for sid in range(1, 40):
        L = rnd.randint(1, 700)
        decode.append(_seq(sid, [rnd.randrange(1000) for _ in range(L)], rnd.randint(1, 5)))
        tables[sid] = rnd.sample(range(998), (L + 15) // 16)
    _check([], decode, tables)


def test_prepare_inputs_prefill_and_mixed():
    rnd = random.Random(1)
    pre, tables = [], {}
    for sid in range(1, 6):
        L = rnd.randint(1, 90)
        pre.append(_seq(sid, [rnd.randrange(1000) for _ in range(L)], 0))
        tables[sid] = rnd.sample(range(998), (L + 15) // 16)
    _check(pre, [], tables)
    dec = [_seq(9, list(range(33)), 2)]
    tables[9] = [5, 6, 7]
    _check(pre, dec, tables)


def test_steppack_extension_matches_numpy():
    """The C packing of the block table equals the numpy one, pads, and
    refuses rows wider than the table or buffers too small."""
    import ctypes
    import pytest
    assert steppack.ext() is not None, "build the host extension: python -m needle_b200.build"
    rnd = random.Random(2)
    rows = [[rnd.randrange(1 << 20) for _ in range(rnd.randint(0, 70))] for _ in range(33)]
    width = max(map(len, rows))
    ref = steppack.block_table_np(rows, width, 12345)
    buf = np.full(len(rows) * width + 8, -7, dtype=np.int32)
    steppack.fill_block_table(rows, buf.ctypes.data, buf.nbytes, width, 12345)
    assert np.array_equal(buf[:len(rows) * width].reshape(len(rows), width), ref)
    assert (buf[len(rows) * width:] == -7).all()          # nothing written past the table
    with pytest.raises(ValueError):
        steppack.fill_block_table(rows, buf.ctypes.data, buf.nbytes, width - 1, 0)
    with pytest.raises(ValueError):
        steppack.fill_block_table(rows, buf.ctypes.data, 16, width, 0)
