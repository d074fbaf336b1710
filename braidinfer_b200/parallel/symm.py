"""Symmetric-memory workspace for the fused tensor-parallel collectives (stub
until the peer-memory runtime lands: keeps the NCCL baseline active)."""
from __future__ import annotations

from ..utils.logging import get_logger

log = get_logger("symm")


def maybe_enable_fused_comm(config, runner) -> bool:
    log.info("fused comm not available yet; using NCCL")
    return False
