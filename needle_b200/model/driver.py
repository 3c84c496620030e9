"""A minimal engine loop around ``ModelRunner`` for batches that fit at once.

It issues exactly the ``SchedulerOutput`` sequence that needle's
``LLMEngine.step`` + ``Scheduler.schedule`` produce when every request is
admitted on the first step and no preemption happens
(``needle/backend/engine.py:110-134``, ``needle/backend/scheduler.py:69-134``):
one prefill step for all prompts, then one decode step per token; a
sequence gets a new block when its length crosses a block boundary; blocks
come from an ascending free list like ``BlockAllocator``
(``needle/backend/block_allocator.py:10-30``).  Needle's real scheduler can
drive the runner just as well; this loop exists so that tests and benchmarks
run where needle itself is not installed.
"""
from __future__ import annotations

import itertools
from collections import deque
from typing import List, Optional

import torch

from .sequence import Request, SamplingParams, SchedulerOutput, Sequence, SequenceStatus


class BatchDriver:
    def __init__(self, runner, num_gpu_blocks: int, block_order: Optional[List[int]] = None):
        self.runner = runner
        self.bs = runner.block_size
        # the runner keeps its own padding block beyond num_gpu_blocks
        self.free = deque(block_order if block_order is not None else range(num_gpu_blocks))
        self.tables = {}
        self.seqs: List[Sequence] = []
        self._ids = itertools.count(1)

    def add(self, prompt: List[int], params: SamplingParams) -> Sequence:
        sid = next(self._ids)
        nb = (len(prompt) + self.bs - 1) // self.bs
        seq = Sequence(seq_id=sid, request=Request(str(sid), list(prompt), params),
                       token_ids=list(prompt), logical_blocks=list(range(nb)), block_size=self.bs,
                       status=SequenceStatus.RUNNING)
        if len(self.free) < nb:
            raise MemoryError("KV pool too small for the batch")
        self.tables[sid] = [self.free.popleft() for _ in range(nb)]
        self.seqs.append(seq)
        return seq

    def _grow(self):
        for s in self.seqs:
            if s.num_generated_tokens > 0 and s.num_logical_blocks > len(self.tables[s.seq_id]):
                if not self.free:
                    raise MemoryError("KV pool exhausted")
                self.tables[s.seq_id].append(self.free.popleft())

    def step(self) -> List[int]:
        """One engine step over all live sequences; returns the new tokens."""
        self._grow()
        pre = [s for s in self.seqs if s.num_generated_tokens == 0]
        dec = [s for s in self.seqs if s.num_generated_tokens > 0]
        out = self.runner.execute(SchedulerOutput(prefill_seqs=pre, decode_seqs=dec,
                                                  block_tables=self.tables,
                                                  swap_in_map={}, swap_out_map={},
                                                  blocks_to_free=[]))
        by_id = dict(zip(out.seq_ids, out.next_token_ids))
        for s in self.seqs:
            s.append_token(by_id[s.seq_id])
        return [by_id[s.seq_id] for s in self.seqs]

    def generate(self, prompts: List[List[int]], max_new_tokens: int) -> List[List[int]]:
        params = SamplingParams(temperature=0.0, max_new_tokens=max_new_tokens)
        seqs = [self.add(p, params) for p in prompts]
        for _ in range(max_new_tokens):
            self.step()
        return [s.token_ids[s.prompt_len:] for s in seqs]


def blocks_needed(prompt_lens: List[int], new_tokens: int, block_size: int) -> int:
    """KV blocks a batch needs to generate ``new_tokens`` per prompt."""
    return sum((n + new_tokens + block_size - 1) // block_size for n in prompt_lens)


def top2_margins(logits: torch.Tensor) -> List[float]:
    t = logits.float().topk(2, dim=-1).values
    return (t[:, 0] - t[:, 1]).tolist()
