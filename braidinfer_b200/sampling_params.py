"""Sampling parameters for a generation request.

Field names and defaults follow the reference API
(``braidinfer/sampling_params.py:6-15``) so user code ports unchanged:
``temperature == 0`` selects greedy decoding, ``top_k == 0`` disables top-k,
``top_p == 1`` disables nucleus filtering, ``min_p == 0`` disables min-p.
``stop`` strings may span several tokens here (the reference honoured only
single-token stop strings).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Union


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    max_tokens: int = 64
    ignore_eos: bool = False
    stop_token_ids: Optional[List[int]] = field(default=None)
    stop: Optional[Union[str, List[str]]] = field(default=None)
    retain_output_cache: bool = False
    # Per-request RNG seed for reproducible sampling (None: engine stream).
    seed: Optional[int] = None

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError("top_p must be in (0, 1]")
        if not (0.0 <= self.min_p <= 1.0):
            raise ValueError("min_p must be in [0, 1]")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0

    def stop_strings(self) -> List[str]:
        if self.stop is None:
            return []
        return [self.stop] if isinstance(self.stop, str) else list(self.stop)
