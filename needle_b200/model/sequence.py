"""The scheduler <-> runner interface types, field-for-field as needle's.

Mirrors ``needle/backend/sequence.py:12-122`` (``SamplingParams``,
``Request``, ``Sequence``, ``SchedulerOutput``, ``ExecuteInput``,
``ExecuteOutput``) so that ``needle_b200.model.runner.ModelRunner`` accepts
the objects needle's ``Scheduler`` produces -- or these -- interchangeably
(the runner only reads their attributes).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, Optional

import torch


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_new_tokens: int = 512
    stop_token_ids: List[int] = field(default_factory=list)
    stream: bool = False

    def __post_init__(self):
        assert self.temperature >= 0.0, "temperature must be >= 0"
        assert 0.0 < self.top_p <= 1.0, "top_p must be in (0, 1]"
        assert self.max_new_tokens > 0, "max_new_tokens must be > 0"


@dataclass
class Request:
    request_id: str
    prompt_token_ids: List[int]
    sampling_params: SamplingParams
    arrival_time: float = field(default_factory=time.time)


class SequenceStatus(Enum):
    WAITING = "waiting"
    RUNNING = "running"
    SWAPPED = "swapped"
    FINISHED = "finished"


@dataclass
class Sequence:
    seq_id: int
    request: Request
    token_ids: List[int]
    logical_blocks: List[int]
    block_size: int
    status: SequenceStatus = SequenceStatus.WAITING
    num_generated_tokens: int = 0

    @property
    def length(self) -> int:
        return len(self.token_ids)

    @property
    def prompt_len(self) -> int:
        return len(self.request.prompt_token_ids)

    @property
    def num_logical_blocks(self) -> int:
        return (self.length + self.block_size - 1) // self.block_size

    @property
    def last_token_id(self) -> int:
        return self.token_ids[-1]

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)
        self.num_generated_tokens += 1
        if self.length % self.block_size == 1:
            self.logical_blocks.append(len(self.logical_blocks))


@dataclass
class SchedulerOutput:
    prefill_seqs: List[Sequence]
    decode_seqs: List[Sequence]
    block_tables: Dict[int, List[int]]
    swap_in_map: Dict[int, int]
    swap_out_map: Dict[int, int]
    blocks_to_free: List[int]

    @property
    def num_seqs(self) -> int:
        return len(self.prefill_seqs) + len(self.decode_seqs)

    @property
    def is_empty(self) -> bool:
        return self.num_seqs == 0


@dataclass
class ExecuteInput:
    input_ids: torch.Tensor
    position_ids: torch.Tensor
    cu_seqlens: torch.Tensor
    max_seqlen: int
    block_table: torch.Tensor
    context_lens: torch.Tensor
    is_prefill: bool


@dataclass
class ExecuteOutput:
    seq_ids: List[int]
    next_token_ids: List[int]
    logprobs: Optional[torch.Tensor] = None
