"""Chunk abstractions: content-addressed, reusable pieces of a prompt.

API parity with the reference (``braidinfer/chunks.py:13-98``):

* ``ChunkType`` has the same four members and string values;
* ``Chunk.from_content`` derives ``chunk_id = sha256(f"{type.value}:{content}")``
  (``braidinfer/chunks.py:56``) so ids computed by either implementation agree;
* the KV bookkeeping fields (``kv_cache_allocated``, ``page_table``,
  ``kv_length``, ``cached_position_start`` ...) keep their names.

What differs is ownership: a chunk's KV pages are reference counted by the
page pool, so deleting or evicting a chunk that a running request still reads
only drops the registry's reference (the reference freed pages under live
readers, see its scheduler/page-manager double free).
"""
from __future__ import annotations

import hashlib
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional


class ChunkType(Enum):
    SYSTEM_PROMPT = "system_prompt"
    CONTEXT = "context"
    QUERY = "query"
    OUTPUT = "output"


def chunk_id_for(content: str, chunk_type: ChunkType) -> str:
    return hashlib.sha256(f"{chunk_type.value}:{content}".encode()).hexdigest()


@dataclass
class Chunk:
    chunk_id: str
    chunk_type: ChunkType
    content: str
    token_ids: List[int]
    token_count: int
    metadata: Dict[str, Any] = field(default_factory=dict)
    created_at: float = field(default_factory=time.time)
    last_accessed: float = field(default_factory=time.time)
    access_count: int = 0

    # KV cache state (set by the engine)
    kv_cache_allocated: bool = False
    cascade_level: Optional[int] = None
    page_table: Optional[List[int]] = None
    kv_length: int = 0
    # Slot offset of the first cached token inside page_table[0]; non-zero for
    # OUTPUT chunks that share their first page with the prompt that made them.
    kv_offset: int = 0
    position_offset: int = 0
    global_position_start: int = 0
    global_position_end: int = 0
    cached_position_start: int = 0
    # Final-norm hidden state of the chunk's last token from its own prefill
    # (used when a composition ends on a cached chunk, so that the first
    # generated token needs no private prefill token).
    last_hidden: Any = None

    @classmethod
    def from_content(cls, content: str, chunk_type: ChunkType, tokenizer=None,
                     metadata: Optional[Dict[str, Any]] = None,
                     token_ids: Optional[List[int]] = None) -> "Chunk":
        if token_ids is None:
            token_ids = tokenizer.encode(content, add_special_tokens=False) if tokenizer else []
        return cls(chunk_id=chunk_id_for(content, chunk_type), chunk_type=chunk_type,
                   content=content, token_ids=list(token_ids), token_count=len(token_ids),
                   metadata=dict(metadata or {}))

    def update_access(self) -> None:
        self.last_accessed = time.time()
        self.access_count += 1

    @property
    def content_preview(self) -> str:
        p = self.content[:50].replace("\n", " ")
        return p + "..." if len(self.content) > 50 else p

    def drop_kv(self) -> None:
        """Forget KV state (the engine has released the pages)."""
        self.kv_cache_allocated = False
        self.page_table = None
        self.kv_length = 0
        self.kv_offset = 0
        self.last_hidden = None


class ChunkNotFoundError(KeyError):
    pass


class IncompatibleChunksError(ValueError):
    pass


class InvalidCompositionError(ValueError):
    pass
