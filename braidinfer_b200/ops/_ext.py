"""Loader of the in-tree native extension ``braidinfer_b200._C``.

The extension holds every hand-written sm_100a kernel.  CUDA tensors must go
through it: if it is missing on a GPU box the op raises
``KernelUnavailableError`` instead of silently falling back to PyTorch.  CPU
tensors use the PyTorch restatement of each op, which is the numerical oracle
of the tests (and the only way the engine runs without a GPU).
"""
from __future__ import annotations

import os

from ..errors import KernelUnavailableError

_C = None
_err: Exception | None = None

# Number of native kernel launches issued through ``ext()`` (each kernel
# binding launches one kernel; ops that launch more add the difference via
# ``count``).  Bindings that launch nothing are not counted.
launches = 0
_NOT_LAUNCHES = frozenset({
    "span_trace", "span_names", "gemm_set_trace", "attn_set_trace", "gemm_force_bn", "gemm_force_splits",
    "gemm_check_error", "gemm_prefetch_next", "comm_alloc", "comm_open", "comm_close", "comm_free",
    "comm_tensor", "tp_sample_record_bytes", "attn_select_prefill_tc",
    "attn_prefill_tile_rows", "attn_set_exp2_poly", "attn_tc_set_trace",
    "bounds_check_status", "bounds_check_enabled"})


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn) or name in _NOT_LAUNCHES:
            return fn

        def call(*a, **kw):
            global launches
            launches += 1
            return fn(*a, **kw)

        return call


def count(n: int) -> None:
    global launches
    launches += n


def ext():
    global _C, _err
    if _C is None:
        try:
            if os.environ.get("BRAID_BOUNDS_CHECK") == "1":  # the bounds-checked build
                from .. import _C_checked as mod  # type: ignore[attr-defined]
            else:
                from .. import _C as mod  # type: ignore[attr-defined]
        except Exception as e:  # pragma: no cover - depends on build
            _err = e
            raise KernelUnavailableError(
                "braidinfer_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"(import error: {e})") from e
        _C = _Counted(mod)
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except KernelUnavailableError:
        return False
