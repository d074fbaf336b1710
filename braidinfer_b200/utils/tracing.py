"""NVTX ranges around the engine's host-side phases.

Off by default (one flag test per range).  With ``BRAID_NVTX=1`` in the
environment, or ``tracing.enable()``, every engine step is bracketed by a
range named for its phase and batch (``decode b=8 t=8``, ``prefill b=1
t=2048``) and the model runner marks its sub-phases (eager forward, CUDA-graph
replay, sampling), so a timeline profiler that records NVTX (Nsight Systems,
``ncu --nvtx --nvtx-include``) shows the device work grouped per engine step,
and a ``torch.profiler`` trace carries the same names as ``record_function``
events.  Ranges are host-side: inside a CUDA-graph replay the individual
kernels are not annotated, the replay as a whole is.

The reference has no tracing layer of its own (it relies on external
profilers and ad-hoc ``time.time()`` prints in its benchmark scripts).
"""
from __future__ import annotations

import contextlib
import os
from typing import Callable, Iterator, Optional

_enabled = os.environ.get("BRAID_NVTX", "0") == "1"
_push: Optional[Callable[[str], object]] = None
_pop: Optional[Callable[[], object]] = None


def enable(on: bool = True, push: Optional[Callable[[str], object]] = None,
           pop: Optional[Callable[[], object]] = None) -> None:
    """Turn the ranges on or off; ``push``/``pop`` replace the NVTX calls
    (tests record the ranges with them)."""
    global _enabled, _push, _pop
    _enabled = on
    _push, _pop = push, pop


def enabled() -> bool:
    return _enabled


def _nvtx_calls():
    if _push is not None and _pop is not None:
        return _push, _pop
    import torch

    return torch.cuda.nvtx.range_push, torch.cuda.nvtx.range_pop


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    """``with nvtx_range("decode b=8"): ...`` — a no-op unless enabled.  When
    enabled the range is also a ``torch.profiler.record_function`` scope, so
    the same names label the host events of a ``torch.profiler`` trace."""
    if not _enabled:
        yield
        return
    import torch

    push, pop = _nvtx_calls()
    push(name)
    try:
        with torch.profiler.record_function(name):
            yield
    finally:
        pop()
