"""Chunk ids, registry dedup/LRU/stats/threading (parity with braidinfer/chunk_registry.py)."""
import hashlib
import threading
import time

import pytest

from braidinfer_b200.chunk_registry import ChunkRegistry
from braidinfer_b200.chunks import Chunk, ChunkNotFoundError, ChunkType


def mk(content, t=ChunkType.CONTEXT, md=None):
    return Chunk.from_content(content, t, metadata=md, token_ids=[len(content)])


def test_chunk_id_is_sha256_of_type_and_content():
    c = mk("hello", ChunkType.SYSTEM_PROMPT)
    assert c.chunk_id == hashlib.sha256(b"system_prompt:hello").hexdigest()
    assert mk("hello", ChunkType.CONTEXT).chunk_id != c.chunk_id


def test_dedup_and_stats():
    r = ChunkRegistry(max_chunks=10)
    a = r.register(mk("x"))
    b = r.register(mk("x"))
    assert a == b and len(r) == 1
    st = r.get_stats()
    assert st["cache_hits"] == 1 and st["cache_misses"] == 1 and st["total_registered"] == 1
    assert st["hit_rate"] == 0.5


def test_dedup_disabled_replaces():
    r = ChunkRegistry(max_chunks=10, enable_deduplication=False)
    r.register(mk("x"))
    r.register(mk("x"))
    assert len(r) == 1 and r.get_stats()["cache_misses"] == 2


def test_lru_eviction_order_and_release():
    released = []
    r = ChunkRegistry(max_chunks=2, on_release=lambda c: released.append(c.chunk_id))
    ids = [r.register(mk(s)) for s in ("a", "b")]
    r.get(ids[0])  # a becomes MRU
    for cid in ids:
        r.peek(cid).kv_cache_allocated = True
    r.register(mk("c"))
    assert ids[1] not in r and ids[0] in r
    assert released == [ids[1]]
    assert r.get_stats()["evictions"] == 1


def test_get_missing_raises():
    with pytest.raises(ChunkNotFoundError):
        ChunkRegistry().get("nope")


def test_list_filter_delete_clear():
    r = ChunkRegistry()
    r.register(mk("s", ChunkType.SYSTEM_PROMPT))
    r.register(mk("c1", md={"role": "user", "k": 1}))
    r.register(mk("c2", md={"k": 2}))
    assert len(r.list_chunks(ChunkType.CONTEXT)) == 2
    assert [c["metadata"]["k"] for c in r.list_chunks(metadata_filter={"k": 2})] == [2]
    info = r.list_chunks(ChunkType.SYSTEM_PROMPT)[0]
    for key in ("chunk_id", "chunk_type", "content_preview", "token_count", "metadata", "created_at",
                "last_accessed", "access_count", "kv_cache_allocated"):
        assert key in info
    assert r.clear(ChunkType.CONTEXT) == 2 and len(r) == 1
    sid = r.list_chunks()[0]["chunk_id"]
    assert r.delete(sid) and not r.delete(sid)


def test_evict_unused_releases_kv():
    released = []
    r = ChunkRegistry(on_release=lambda c: released.append(c.chunk_id))
    cid = r.register(mk("old"))
    r.peek(cid).kv_cache_allocated = True
    r.peek(cid).last_accessed = time.time() - 100
    assert r.evict_unused_chunks(10) == 1
    assert released == [cid]


def test_concurrent_register():
    r = ChunkRegistry(max_chunks=10000)

    def work(k):
        for i in range(200):
            r.register(mk(f"{i % 50}"))

    ts = [threading.Thread(target=work, args=(k,)) for k in range(8)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert len(r) == 50
    st = r.get_stats()
    assert st["cache_hits"] + st["cache_misses"] == 1600
