"""Collectives used by the tensor-parallel model.

``nccl`` backend: plain ``torch.distributed`` calls — the baseline.
``fused`` backend: the all-reduce of row-parallel GEMM outputs is done by the
native one-shot push kernel over peer memory (``csrc/comm.cu``) when the
symmetric workspace is available; otherwise it falls back to NCCL with a log
line, never silently on a GPU box where the workspace was requested.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .state import get_tp

_fused = None  # set by parallel.symm when a symmetric workspace is created


def set_fused_comm(obj) -> None:
    global _fused
    _fused = obj


def get_fused_comm():
    return _fused


def all_reduce(x: torch.Tensor) -> torch.Tensor:
    tp = get_tp()
    if tp.size == 1:
        return x
    if _fused is not None and x.is_cuda and _fused.can_all_reduce(x):
        return _fused.all_reduce(x)
    dist.all_reduce(x, group=tp.group)
    return x


def all_reduce_add(partial: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """``residual += sum_ranks(partial)`` (activation dtype), returns residual."""
    tp = get_tp()
    if tp.size > 1 and _fused is not None and partial.is_cuda and _fused.can_all_reduce(partial):
        return _fused.all_reduce_add(partial, residual)
    s = all_reduce(partial)
    residual.copy_((residual.float() + s.float()).to(residual.dtype))
    return residual


def all_reduce_add_rms_norm(partial: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                            out: Optional[torch.Tensor] = None):
    """``residual += sum_ranks(partial)``; return ``(rms_norm(residual), residual)``."""
    from ..ops.norm import add_rms_norm

    tp = get_tp()
    if tp.size > 1 and _fused is not None and partial.is_cuda and _fused.can_all_reduce(partial):
        return _fused.all_reduce_add_rms_norm(partial, residual, w, eps, out)
    s = all_reduce(partial)
    return add_rms_norm(s, residual, w, eps, out)


def all_gather_last(x: torch.Tensor, full: Optional[int] = None) -> torch.Tensor:
    """Concatenate ``x[..., n]`` of every rank along the last dim (vocab shards)."""
    tp = get_tp()
    if tp.size == 1:
        return x
    x = x.contiguous()
    g = torch.empty((tp.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(g, x, group=tp.group)
    g = g.view((tp.size,) + tuple(x.shape))
    y = g.movedim(0, -2).reshape(*x.shape[:-1], tp.size * x.shape[-1])
    return y[..., :full] if full is not None else y


def broadcast_obj(obj, src: int = 0):
    tp = get_tp()
    if tp.size == 1:
        return obj
    box = [obj]
    dist.broadcast_object_list(box, src=src, group=tp.group)
    return box[0]
