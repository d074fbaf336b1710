"""Typed error hierarchy.

Mirrors the reference's ``NanoVLLMError`` family
(``braidinfer/engine/errors.py:9-88``) but classifies by exception *type*
instead of message substrings, and adds the errors the multi-GPU runtime
needs (``CommTimeoutError`` raised when a device-side bounded wait expires,
``PeerFailureError`` when a rank stops heart-beating).
"""
from __future__ import annotations

import functools
import logging
import traceback

log = logging.getLogger("braidinfer_b200")


class BraidError(Exception):
    """Base class of every error raised by this package."""


class ModelLoadError(BraidError):
    pass


class InferenceError(BraidError):
    pass


class PlanValidationError(InferenceError):
    """A step's kernel metadata indexes outside its buffers (raised only with
    plan validation on: ``Config.validate_plans`` or ``BRAID_VALIDATE_PLAN=1``)."""


class OutOfPagesError(BraidError, MemoryError):
    """The paged KV pool has no free page even after eviction and preemption."""


# Alias kept for API parity with the reference's ``MemoryError`` subclass.
KVMemoryError = OutOfPagesError


class DistributedError(BraidError):
    pass


class CommTimeoutError(DistributedError):
    """A bounded device-side wait on a peer flag expired.

    ``status`` holds the decoded status word: rank, peer, epoch, code.
    """

    def __init__(self, msg: str, status: dict | None = None):
        super().__init__(msg)
        self.status = status or {}


class PeerFailureError(DistributedError):
    """A peer rank stopped answering (missed heartbeat or left the group)."""


class ConfigurationError(BraidError, ValueError):
    pass


class KernelUnavailableError(BraidError, RuntimeError):
    """A CUDA tensor reached an op whose native extension is not built."""


class ErrorContext:
    """Context manager that re-types unexpected exceptions as ``InferenceError``.

    ``BraidError`` subclasses pass through unchanged; torch OOM becomes
    ``OutOfPagesError``-compatible ``KVMemoryError`` only when raised by the
    page pool, otherwise it is an ``InferenceError`` with the original chained.
    """

    def __init__(self, what: str):
        self.what = what

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc is None or isinstance(exc, BraidError):
            return False
        if isinstance(exc, (KeyboardInterrupt, SystemExit, GeneratorExit)):
            return False
        raise InferenceError(f"{self.what} failed: {exc_type.__name__}: {exc}") from exc


def handle_inference_error(what: str):
    """Decorator form of :class:`ErrorContext` that also logs the traceback."""

    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*a, **kw):
            try:
                with ErrorContext(what):
                    return fn(*a, **kw)
            except BraidError:
                log.debug("%s failed:\n%s", what, traceback.format_exc())
                raise

        return wrapper

    return deco
