"""Tensor-parallel process state: one process per GPU, ``torch.distributed``
for bootstrap and the NCCL baseline collectives.

The reference is single-GPU; its only collective is a dead
``dist.all_reduce`` (``braidinfer/layers/linear_distributed.py:170-174``).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class TPState:
    rank: int = 0
    size: int = 1
    group: Optional[object] = None
    backend: str = "none"

    @property
    def enabled(self) -> bool:
        return self.size > 1


_TP = TPState()


def get_tp() -> TPState:
    return _TP


def set_tp(state: TPState) -> None:
    global _TP
    _TP = state


def init_tp(size: int, timeout_s: float = 60.0, backend: Optional[str] = None) -> TPState:
    """Join (or create) the default process group and bind this rank's GPU.

    Reads RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR / MASTER_PORT from the
    environment (torchrun).  ``size`` must equal WORLD_SIZE.
    """
    global _TP
    if size == 1:
        _TP = TPState()
        return _TP
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != size:
        raise RuntimeError(f"tensor_parallel_size={size} but WORLD_SIZE={world}; launch one process per GPU")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    _TP = TPState(rank=dist.get_rank(), size=dist.get_world_size(), group=dist.group.WORLD, backend=backend)
    return _TP
