"""Host-side liveness of tensor-parallel ranks.

Before each engine step every rank publishes a heartbeat (its step number and
wall time) in the process group's key-value store and checks its peers'.  A
peer that is missing, or behind by more than ``timeout_s`` of wall time, makes
``check`` raise ``PeerFailureError`` *before* this rank launches the step's
collectives, so survivors fail fast between steps instead of blocking inside
a collective.  The device-side counterpart is the bounded wait of the fused
collectives (``CommTimeoutError``).
"""
from __future__ import annotations

import time
from typing import Optional

import torch.distributed as dist

from ..errors import PeerFailureError


class Heartbeat:
    def __init__(self, timeout_s: float = 10.0, store: Optional[dist.Store] = None, prefix: str = "braid/hb"):
        self.timeout_s = timeout_s
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.store = store or dist.distributed_c10d._get_default_store()
        self.prefix = prefix

    def beat(self, step: int) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", f"{step}:{time.time():.3f}")

    def check(self, step: int) -> None:
        """Publish this rank's heartbeat for ``step`` and wait (bounded) until
        every peer has reached it."""
        self.beat(step)
        deadline = time.time() + self.timeout_s
        for r in range(self.world):
            if r == self.rank:
                continue
            key = f"{self.prefix}/{r}"
            while True:
                try:
                    self.store.wait([key], __import__("datetime").timedelta(seconds=max(0.1, deadline - time.time())))
                    val = self.store.get(key).decode()
                    peer_step = int(val.split(":")[0])
                except Exception as e:  # store timeout or a dead store
                    raise PeerFailureError(f"rank {r} missed its heartbeat for step {step}: {e}") from e
                if peer_step >= step:
                    break
                if time.time() > deadline:
                    raise PeerFailureError(f"rank {r} stuck at step {peer_step}, expected {step}")
                time.sleep(0.01)
