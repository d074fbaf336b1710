"""Token embedding gather (vocab-parallel aware).

Rows of ids outside ``[vocab_start, vocab_start + rows)`` produce zeros so a
tensor-parallel rank contributes only the rows it owns before the reduction
(the Megatron vocab-parallel rule; the reference's ``VocabParallelEmbedding``
was a plain ``F.embedding``, ``braidinfer/layers/embed_head.py:14-29``).
"""
from __future__ import annotations

from typing import Optional

import torch

from ._ext import ext


def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if weight.is_cuda:
        if out is None:
            out = torch.empty(ids.shape[0], weight.shape[1], dtype=weight.dtype, device=weight.device)
        ext().embedding(out, ids, weight, int(vocab_start))
        return out
    local = ids.long() - vocab_start
    ok = (local >= 0) & (local < weight.shape[0])
    rows = weight[local.clamp(0, weight.shape[0] - 1)]
    y = torch.where(ok[:, None], rows, torch.zeros_like(rows))
    if out is not None:
        out.copy_(y)
        return out
    return y
