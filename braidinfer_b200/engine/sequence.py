"""A generation request: private tokens plus the cached chunk segments it reads.

The reference kept a single ``block_table`` into which it concatenated the
pages of every chunk (``braidinfer/engine/llm_engine.py:504-540``) and then
wrote new tokens into chunk pages.  Here a sequence *reads* chunk KV through
``segments`` (shared, refcounted, never written) and *writes* only its own
``pages`` — the private segment that starts at global position ``pos_base``.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum, auto
from itertools import count
from typing import Any, List, Optional

from ..sampling_params import SamplingParams


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


@dataclass
class SegmentRef:
    """A read-only KV segment (a cached chunk) placed in a composition."""

    pages: List[int]
    offset: int      # slot of the first key in pages[0]
    length: int      # number of keys
    pos0: int        # global position of the first key in this composition
    delta: int       # pos0 - position at which the keys were rotated
    chunk: Any = None


class Sequence:
    counter = count()

    def __init__(self, token_ids: List[int], sampling_params: Optional[SamplingParams] = None,
                 segments: Optional[List[SegmentRef]] = None, pos_base: int = 0):
        sp = sampling_params or SamplingParams()
        self.seq_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.token_ids: List[int] = list(token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        self.num_cached_tokens = 0
        self.pages: List[int] = []
        self.segments: List[SegmentRef] = list(segments or [])
        self.pos_base = pos_base
        self.sampling_params = sp
        self.temperature = sp.temperature
        self.top_k = sp.top_k
        self.top_p = sp.top_p
        self.min_p = sp.min_p
        self.max_tokens = sp.max_tokens
        self.ignore_eos = sp.ignore_eos
        self.stop_token_ids = list(sp.stop_token_ids or [])
        self.stop_sequences: List[List[int]] = []
        self.retain_output_cache = sp.retain_output_cache
        self.seed = sp.seed if sp.seed is not None else (self.seq_id * 1000003 + 12345)
        self.first_hidden = None   # logits source when the private prompt is empty
        self.active_chunks = [s.chunk for s in self.segments if s.chunk is not None] or None
        self.finish_reason: Optional[str] = None
        self.arrival_time = 0.0
        self.first_token_time: Optional[float] = None

    # -- parity properties ---------------------------------------------------
    def __len__(self):
        return self.num_tokens

    @property
    def num_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def last_token(self) -> int:
        return self.token_ids[-1]

    @property
    def block_table(self) -> List[int]:
        return self.pages

    @property
    def is_finished(self) -> bool:
        return self.status == SequenceStatus.FINISHED

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> List[int]:
        return self.token_ids[: self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> List[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def total_prompt_len(self) -> int:
        """Prompt tokens including the cached chunks this sequence reads."""
        return self.pos_base + self.num_prompt_tokens

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(int(token_id))
