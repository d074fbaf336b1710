"""Thread-safe LRU registry of chunks with content-hash deduplication.

Behavioural parity with ``braidinfer/chunk_registry.py:14-268`` (register with
dedup hit → MRU, LRU eviction at ``max_chunks``, filtered listing, stats with
hit rate).  Two fixes: ``evict_unused_chunks`` releases KV pages (the reference
leaked them, ``braidinfer/chunk_registry.py:213-236``), and page release goes
through the refcounted pool so chunks read by in-flight requests stay valid.
"""
from __future__ import annotations

import threading
import time
from collections import OrderedDict
from datetime import datetime
from typing import Any, Callable, Dict, List, Optional

from .chunks import Chunk, ChunkNotFoundError, ChunkType


class ChunkRegistry:
    def __init__(self, max_chunks: int = 1000, enable_deduplication: bool = True,
                 page_manager=None, on_release: Optional[Callable[[Chunk], None]] = None):
        self.max_chunks = max_chunks
        self.enable_deduplication = enable_deduplication
        self.page_manager = page_manager
        self._on_release = on_release
        self._lock = threading.RLock()
        self._chunks: "OrderedDict[str, Chunk]" = OrderedDict()
        self.stats = {"total_registered": 0, "cache_hits": 0, "cache_misses": 0, "evictions": 0}

    # -- internal -----------------------------------------------------------
    def _release(self, chunk: Chunk) -> None:
        if chunk.kv_cache_allocated:
            if self._on_release is not None:
                self._on_release(chunk)
            elif self.page_manager is not None:
                self.page_manager.release_chunk(chunk)
        chunk.drop_kv()

    def _evict_lru(self, count: int = 1) -> None:
        for _ in range(min(count, len(self._chunks))):
            _, chunk = self._chunks.popitem(last=False)
            self._release(chunk)
            self.stats["evictions"] += 1

    # -- public -------------------------------------------------------------
    def register(self, chunk: Chunk) -> str:
        with self._lock:
            if self.enable_deduplication and chunk.chunk_id in self._chunks:
                existing = self._chunks.pop(chunk.chunk_id)
                self._chunks[chunk.chunk_id] = existing
                existing.update_access()
                if chunk.metadata:
                    existing.metadata.update(chunk.metadata)
                self.stats["cache_hits"] += 1
                return existing.chunk_id
            self.stats["cache_misses"] += 1
            if chunk.chunk_id in self._chunks:  # dedup disabled: replace
                self._release(self._chunks.pop(chunk.chunk_id))
            if len(self._chunks) >= self.max_chunks:
                self._evict_lru()
            self._chunks[chunk.chunk_id] = chunk
            self.stats["total_registered"] += 1
            return chunk.chunk_id

    def get(self, chunk_id: str) -> Chunk:
        with self._lock:
            if chunk_id not in self._chunks:
                raise ChunkNotFoundError(f"Chunk {chunk_id} not found")
            chunk = self._chunks.pop(chunk_id)
            self._chunks[chunk_id] = chunk
            chunk.update_access()
            self.stats["cache_hits"] += 1
            return chunk

    def peek(self, chunk_id: str) -> Optional[Chunk]:
        """Return a chunk without touching LRU order or statistics."""
        with self._lock:
            return self._chunks.get(chunk_id)

    def __contains__(self, chunk_id: str) -> bool:
        with self._lock:
            return chunk_id in self._chunks

    def __len__(self) -> int:
        with self._lock:
            return len(self._chunks)

    def chunks(self) -> List[Chunk]:
        with self._lock:
            return list(self._chunks.values())

    def list_chunks(self, chunk_type: Optional[ChunkType] = None,
                    metadata_filter: Optional[Dict[str, Any]] = None) -> List[Dict[str, Any]]:
        with self._lock:
            out = []
            for c in self._chunks.values():
                if chunk_type is not None and c.chunk_type != chunk_type:
                    continue
                if metadata_filter and not all(c.metadata.get(k) == v for k, v in metadata_filter.items()):
                    continue
                out.append({
                    "chunk_id": c.chunk_id,
                    "chunk_type": c.chunk_type.value,
                    "content_preview": c.content_preview,
                    "token_count": c.token_count,
                    "metadata": dict(c.metadata),
                    "created_at": datetime.fromtimestamp(c.created_at).isoformat(),
                    "last_accessed": datetime.fromtimestamp(c.last_accessed).isoformat(),
                    "access_count": c.access_count,
                    "kv_cache_allocated": c.kv_cache_allocated,
                })
            return out

    def delete(self, chunk_id: str) -> bool:
        with self._lock:
            chunk = self._chunks.pop(chunk_id, None)
            if chunk is None:
                return False
            self._release(chunk)
            return True

    def clear(self, chunk_type: Optional[ChunkType] = None) -> int:
        with self._lock:
            ids = [cid for cid, c in self._chunks.items()
                   if chunk_type is None or c.chunk_type == chunk_type]
            for cid in ids:
                self._release(self._chunks.pop(cid))
            return len(ids)

    def evict_unused_chunks(self, max_age_seconds: float) -> int:
        now = time.time()
        with self._lock:
            ids = [cid for cid, c in self._chunks.items() if now - c.last_accessed > max_age_seconds]
            for cid in ids:
                self._release(self._chunks.pop(cid))
                self.stats["evictions"] += 1
            return len(ids)

    def evict_lru_with_kv(self, is_busy: Callable[[Chunk], bool]) -> bool:
        """Free the KV of the least recently used chunk no request is reading.

        The chunk stays registered (it is re-prefilled on next use).  Returns
        False when no chunk could give pages back.
        """
        with self._lock:
            for c in self._chunks.values():
                if c.kv_cache_allocated and c.page_table and not is_busy(c):
                    self._release(c)
                    self.stats["evictions"] += 1
                    return True
            return False

    def get_stats(self) -> Dict[str, Any]:
        with self._lock:
            lookups = self.stats["cache_hits"] + self.stats["cache_misses"]
            return {
                "total_chunks": len(self._chunks),
                "max_chunks": self.max_chunks,
                "cache_hits": self.stats["cache_hits"],
                "cache_misses": self.stats["cache_misses"],
                "hit_rate": self.stats["cache_hits"] / lookups if lookups else 0.0,
                "evictions": self.stats["evictions"],
                "total_registered": self.stats["total_registered"],
            }
