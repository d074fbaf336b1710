"""Refcounted paged KV pool, HND layout ``[L, P, 2, Hkv, page, D]``.

Same pool layout and page-table vocabulary as the reference
(``braidinfer/engine/page_manager.py:13-353``: ``allocate_for_chunk``,
``free_for_chunk``, ``chunk_page_tables``, ``seq_page_tables``,
``get_sequence_cache_info``), with ownership made explicit:

* every page has a reference count; a page returns to the free list when it
  drops to zero;
* a chunk owns one reference on each of its pages; a sequence that reads a
  chunk holds one more for as long as it runs, so deleting/evicting the chunk
  cannot free pages under a live reader (the reference's double free);
* a sequence owns its private pages; finishing frees them unless the output
  KV is retained, in which case the retained sequence keeps them until
  ``release``.

The last page of the pool is reserved as a scratch page: padded rows of a
CUDA-graph batch write their K/V there.
"""
from __future__ import annotations

from collections import deque
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

from ..errors import OutOfPagesError
from .sequence import Sequence


class PageManager:
    def __init__(self, num_pages: int, page_size: int, num_layers: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device):
        if num_pages < 2:
            raise OutOfPagesError("KV pool needs at least 2 pages")
        self.num_pages = num_pages
        self.page_size = page_size
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.kv_cache = torch.zeros(num_layers, num_pages, 2, num_kv_heads, page_size, head_dim,
                                    dtype=dtype, device=device)
        self.scratch_page = num_pages - 1
        self.refcount = np.zeros(num_pages, dtype=np.int32)
        self.refcount[self.scratch_page] = 1 << 30
        self.free_pages = deque(range(num_pages - 1))
        self.chunk_page_tables: Dict[str, List[int]] = {}
        self.chunk_lengths: Dict[str, int] = {}
        self.seq_page_tables: Dict[int, List[int]] = {}
        self.seq_lengths: Dict[int, int] = {}
        # Called when allocation fails; frees some chunk KV and returns True if it did.
        self.evictor: Optional[Callable[[], bool]] = None

    # ---------------------------------------------------------------- basics
    @property
    def bytes_per_page(self) -> int:
        return 2 * self.num_layers * self.num_kv_heads * self.page_size * self.head_dim * self.kv_cache.element_size()

    @property
    def num_free_pages(self) -> int:
        return len(self.free_pages)

    def pages_for(self, n_tokens: int) -> int:
        return -(-n_tokens // self.page_size)

    def alloc(self, n: int, evict: bool = True) -> List[int]:
        while len(self.free_pages) < n:
            if not (evict and self.evictor is not None and self.evictor()):
                raise OutOfPagesError(f"need {n} KV pages, {len(self.free_pages)} free")
        out = [self.free_pages.popleft() for _ in range(n)]
        for p in out:
            self.refcount[p] = 1
        return out

    def incref(self, pages: List[int]) -> None:
        for p in pages:
            self.refcount[p] += 1

    def decref(self, pages: List[int]) -> None:
        for p in pages:
            self.refcount[p] -= 1
            if self.refcount[p] == 0:
                self.free_pages.append(p)
            elif self.refcount[p] < 0:
                raise RuntimeError(f"page {p} refcount underflow")

    def is_shared(self, pages: List[int]) -> bool:
        return any(self.refcount[p] > 1 for p in pages)

    # ---------------------------------------------------------------- chunks
    def allocate_for_chunk(self, chunk_id: str, n_tokens: int) -> List[int]:
        if chunk_id in self.chunk_page_tables:
            return self.chunk_page_tables[chunk_id]
        pages = self.alloc(self.pages_for(n_tokens)) if n_tokens else []
        self.chunk_page_tables[chunk_id] = pages
        self.chunk_lengths[chunk_id] = n_tokens
        return pages

    def adopt_for_chunk(self, chunk_id: str, pages: List[int], n_tokens: int) -> None:
        """Give a chunk its own reference on existing pages (retained output)."""
        self.incref(pages)
        self.chunk_page_tables[chunk_id] = list(pages)
        self.chunk_lengths[chunk_id] = n_tokens

    def free_for_chunk(self, chunk_id: str) -> None:
        pages = self.chunk_page_tables.pop(chunk_id, None)
        self.chunk_lengths.pop(chunk_id, None)
        if pages:
            self.decref(pages)

    def release_chunk(self, chunk) -> None:
        self.free_for_chunk(chunk.chunk_id)

    # ------------------------------------------------------------- sequences
    def ensure_capacity(self, seq: Sequence, n_tokens: int, evict: bool = True) -> bool:
        need = self.pages_for(n_tokens) - len(seq.pages)
        if need <= 0:
            return True
        try:
            seq.pages.extend(self.alloc(need, evict=evict))
        except OutOfPagesError:
            return False
        self.seq_page_tables[seq.seq_id] = seq.pages
        return True

    def can_allocate(self, seq: Sequence) -> bool:
        return self.pages_for(seq.num_tokens) - len(seq.pages) <= len(self.free_pages)

    def acquire_segments(self, seq: Sequence) -> None:
        for s in seq.segments:
            self.incref(s.pages)

    def release_segments(self, seq: Sequence) -> None:
        for s in seq.segments:
            self.decref(s.pages)
        seq.segments = []

    def free_private(self, seq: Sequence) -> None:
        if seq.pages:
            self.decref(seq.pages)
        seq.pages = []
        seq.num_cached_tokens = 0
        self.seq_page_tables.pop(seq.seq_id, None)
        self.seq_lengths.pop(seq.seq_id, None)

    def deallocate(self, seq: Sequence) -> None:
        self.free_private(seq)
        self.release_segments(seq)

    def update_sequence_lengths(self, seqs: List[Sequence]) -> None:
        for s in seqs:
            self.seq_lengths[s.seq_id] = s.num_cached_tokens

    def get_sequence_cache_info(self, seq: Sequence) -> dict:
        return {
            "seq_id": seq.seq_id,
            "page_table": list(seq.pages),
            "kv_length": seq.num_cached_tokens,
            "position_start": seq.pos_base,
            "page_size": self.page_size,
            "segments": [(s.pos0, s.length) for s in seq.segments],
        }

    def stats(self) -> dict:
        used = self.num_pages - 1 - len(self.free_pages)
        return {"num_pages": self.num_pages - 1, "used_pages": used, "free_pages": len(self.free_pages),
                "page_size": self.page_size, "bytes_per_page": self.bytes_per_page,
                "chunk_pages": sum(len(p) for p in self.chunk_page_tables.values())}
