"""Inference metrics (TTFT, TPOT, tok/s, per-phase totals).

The reference's ``MetricsCollector`` (``braidinfer/engine/metrics.py:13-168``)
was never called and ``LLMEngine.get_metrics`` pointed at a missing method;
here the engine records every step.  Step durations are host wall time around
a step that ends with the device→host token read, so they include the device
work of that step.
"""
from __future__ import annotations

import threading
import time
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Dict, List


@dataclass
class InferenceMetrics:
    prefill_tokens: int = 0
    decode_tokens: int = 0
    prefill_time_s: float = 0.0
    decode_time_s: float = 0.0
    steps: int = 0
    ttft_s: List[float] = field(default_factory=list)
    requests_finished: int = 0
    preemptions: int = 0

    def summary(self) -> Dict[str, float]:
        ttft = sorted(self.ttft_s)
        return {
            "steps": self.steps,
            "prefill_tokens": self.prefill_tokens,
            "decode_tokens": self.decode_tokens,
            "prefill_tok_s": self.prefill_tokens / self.prefill_time_s if self.prefill_time_s else 0.0,
            "decode_tok_s": self.decode_tokens / self.decode_time_s if self.decode_time_s else 0.0,
            "tpot_ms": 1e3 * self.decode_time_s / max(1, self.steps_decode) if hasattr(self, "steps_decode") else 0.0,
            "ttft_mean_ms": 1e3 * sum(ttft) / len(ttft) if ttft else 0.0,
            "ttft_p50_ms": 1e3 * ttft[len(ttft) // 2] if ttft else 0.0,
            "requests_finished": self.requests_finished,
            "preemptions": self.preemptions,
        }


class MetricsCollector:
    def __init__(self):
        self._lock = threading.Lock()
        self.m = InferenceMetrics()
        self.m.steps_decode = 0

    def record_step(self, is_prefill: bool, tokens: int, dt: float) -> None:
        with self._lock:
            self.m.steps += 1
            if is_prefill:
                self.m.prefill_tokens += tokens
                self.m.prefill_time_s += dt
            else:
                self.m.decode_tokens += tokens
                self.m.decode_time_s += dt
                self.m.steps_decode += 1

    def record_ttft(self, s: float) -> None:
        with self._lock:
            self.m.ttft_s.append(s)

    def record_finished(self, n: int = 1) -> None:
        with self._lock:
            self.m.requests_finished += n

    def reset(self) -> None:
        with self._lock:
            self.m = InferenceMetrics()
            self.m.steps_decode = 0

    def summary(self) -> Dict[str, float]:
        with self._lock:
            return self.m.summary()


@contextmanager
def timed():
    t = [time.perf_counter(), 0.0]
    yield t
    t[1] = time.perf_counter() - t[0]
