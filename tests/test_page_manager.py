"""Refcounted paged KV pool: allocation, sharing, no leaks, eviction hook."""
import pytest
import torch

from braidinfer_b200.engine.page_manager import PageManager
from braidinfer_b200.engine.sequence import SegmentRef, Sequence
from braidinfer_b200.errors import OutOfPagesError


def pm(n=9):
    return PageManager(n, 16, 2, 2, 8, torch.float32, torch.device("cpu"))


def test_layout_and_scratch_page():
    p = pm()
    assert tuple(p.kv_cache.shape) == (2, 9, 2, 2, 16, 8)
    assert p.num_free_pages == 8 and p.scratch_page == 8


def test_chunk_pages_survive_until_last_reader():
    p = pm()
    pages = p.allocate_for_chunk("c", 40)
    assert len(pages) == 3 and p.num_free_pages == 5
    s = Sequence([1, 2, 3], segments=[SegmentRef(pages, 0, 40, 0, 0)])
    p.acquire_segments(s)
    p.free_for_chunk("c")  # registry drops the chunk while the sequence reads it
    assert p.num_free_pages == 5
    p.deallocate(s)
    assert p.num_free_pages == 8


def test_sequence_capacity_and_free():
    p = pm()
    s = Sequence(list(range(20)))
    assert p.ensure_capacity(s, 20) and len(s.pages) == 2
    assert p.ensure_capacity(s, 33) and len(s.pages) == 3
    p.free_private(s)
    assert p.num_free_pages == 8 and s.pages == []


def test_out_of_pages_and_evictor():
    p = pm(4)
    p.allocate_for_chunk("a", 16)
    p.allocate_for_chunk("b", 32)
    with pytest.raises(OutOfPagesError):
        p.alloc(1, evict=False)
    calls = []

    def ev():
        calls.append(1)
        if "a" in p.chunk_page_tables:
            p.free_for_chunk("a")
            return True
        return False

    p.evictor = ev
    assert len(p.alloc(1)) == 1 and calls
    with pytest.raises(OutOfPagesError):
        p.alloc(1)


def test_refcount_underflow_detected():
    p = pm()
    pages = p.alloc(1)
    p.decref(pages)
    with pytest.raises(RuntimeError):
        p.decref(pages)
