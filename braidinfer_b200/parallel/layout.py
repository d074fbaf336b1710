"""Sharding arithmetic for Megatron-style tensor parallelism.

Column-parallel: QKV (by head) and gate/up (by intermediate row); row-parallel:
o_proj and down_proj (by input column); vocab-parallel embedding and LM head.
When ``num_kv_heads < tp`` each KV head is replicated on ``tp / num_kv_heads``
consecutive ranks (TinyLlama: 4 KV heads at TP8 → 2 ranks per head), matching
the query heads those ranks own.  The reference's dead TP code split only
evenly divisible shapes (``braidinfer/layers/linear_distributed.py:55-174``).
"""
from __future__ import annotations

from dataclasses import dataclass

from ..errors import ConfigurationError


@dataclass(frozen=True)
class TPLayout:
    tp: int
    rank: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    block: int = 64  # SwiGLU interleave block; local intermediate is padded to it

    def __post_init__(self):
        if self.num_heads % self.tp:
            raise ConfigurationError(f"num_heads={self.num_heads} not divisible by tp={self.tp}")
        if self.num_kv_heads >= self.tp and self.num_kv_heads % self.tp:
            raise ConfigurationError(f"num_kv_heads={self.num_kv_heads} not divisible by tp={self.tp}")
        if self.num_kv_heads < self.tp and self.tp % self.num_kv_heads:
            raise ConfigurationError(f"tp={self.tp} not a multiple of num_kv_heads={self.num_kv_heads}")

    @property
    def q_heads(self) -> int:
        return self.num_heads // self.tp

    @property
    def q_head_start(self) -> int:
        return self.rank * self.q_heads

    @property
    def kv_heads(self) -> int:
        return max(1, self.num_kv_heads // self.tp)

    @property
    def kv_head_start(self) -> int:
        if self.num_kv_heads >= self.tp:
            return self.rank * self.kv_heads
        return self.rank * self.num_kv_heads // self.tp

    @property
    def inter(self) -> int:
        """Unpadded local intermediate rows: ceil split, last rank may hold fewer."""
        per = -(-self.intermediate // self.tp)
        return max(0, min(per, self.intermediate - self.rank * per))

    @property
    def inter_start(self) -> int:
        return self.rank * (-(-self.intermediate // self.tp))

    @property
    def inter_pad(self) -> int:
        per = -(-self.intermediate // self.tp)
        return -(-per // self.block) * self.block

    @property
    def vocab_per_rank(self) -> int:
        return -(-self.vocab // self.tp)

    @property
    def vocab_start(self) -> int:
        return self.rank * self.vocab_per_rank

    @property
    def vocab_local(self) -> int:
        return max(0, min(self.vocab_per_rank, self.vocab - self.vocab_start))
