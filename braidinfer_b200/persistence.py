"""Chunk persistence: save cached chunk KV to disk and restore it later.

The reference carried a ``chunk_persistence_dir`` config field that nothing
used (``braidinfer/config.py:23``) and listed "no saved KV cache between
sessions" as a gap.  Here a chunk's KV slots are gathered from its pages into
a dense ``[layers, 2, kv_heads, tokens, head_dim]`` tensor and written with
safetensors, one file per tensor-parallel rank, next to a JSON manifest of the
chunk records.  Restoring re-registers each chunk (same SHA256 id), allocates
fresh pages and scatters the KV back, so a restored chunk is reused without any
prefill.  A fingerprint of the model architecture, dtype and TP layout guards
against loading KV computed by a different model or sharding.
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Any, Dict

import torch

from .chunks import Chunk, ChunkType
from .parallel.state import get_tp

MANIFEST = "chunks.json"


def fingerprint(cl) -> str:
    eng = cl.llm
    spec = eng.config.spec
    tp = get_tp()
    desc = json.dumps({"spec": {k: v for k, v in spec.__dict__.items() if k not in ("eos_token_id", "bos_token_id")},
                       "dtype": str(eng.model_runner.dtype), "tp": tp.size, "page": eng.page_manager.page_size},
                      sort_keys=True, default=str)
    return hashlib.sha256(desc.encode()).hexdigest()


def _gather(pm, chunk: Chunk) -> torch.Tensor:
    ps = pm.page_size
    slots = torch.arange(chunk.kv_offset, chunk.kv_offset + chunk.kv_length)
    pages = torch.tensor(chunk.page_table, dtype=torch.long)[slots // ps]
    off = slots % ps
    dev = pm.kv_cache.device
    # advanced indices separated by slices put the token dim first: [n, L, 2, Hkv, D]
    kv = pm.kv_cache[:, pages.to(dev), :, :, off.to(dev), :]
    return kv.permute(1, 2, 3, 0, 4).contiguous().cpu()      # [L, 2, Hkv, n, D]


def save_chunks(cl, path: str) -> int:
    """Write every chunk that holds KV; returns the number of chunks written."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    pm = cl.page_manager
    tp = get_tp()
    tensors: Dict[str, torch.Tensor] = {}
    records = []
    for c in cl.registry.chunks():
        rec: Dict[str, Any] = {"chunk_id": c.chunk_id, "chunk_type": c.chunk_type.value, "content": c.content,
                               "token_ids": c.token_ids, "metadata": c.metadata,
                               "cached_position_start": c.cached_position_start, "kv_length": 0,
                               "cascade_level": c.cascade_level}
        if c.kv_cache_allocated and c.page_table and c.kv_length:
            tensors[c.chunk_id] = _gather(pm, c)
            rec["kv_length"] = c.kv_length
            if c.last_hidden is not None:
                tensors[c.chunk_id + ".last_hidden"] = c.last_hidden.detach().float().cpu().contiguous()
        records.append(rec)
    if tensors:
        save_file(tensors, os.path.join(path, f"kv_rank{tp.rank}.safetensors"))
    if tp.rank == 0:
        with open(os.path.join(path, MANIFEST), "w") as f:
            json.dump({"fingerprint": fingerprint(cl), "tp": tp.size, "chunks": records}, f)
    return len(records)


def load_chunks(cl, path: str) -> int:
    """Register the saved chunks and restore their KV; returns chunks restored."""
    from safetensors import safe_open

    with open(os.path.join(path, MANIFEST)) as f:
        man = json.load(f)
    if man["fingerprint"] != fingerprint(cl):
        raise ValueError("saved chunks were computed by a different model, dtype, page size or TP layout")
    tp = get_tp()
    kvfile = os.path.join(path, f"kv_rank{tp.rank}.safetensors")
    sf = safe_open(kvfile, framework="pt", device="cpu") if os.path.exists(kvfile) else None
    pm = cl.page_manager
    n = 0
    for rec in man["chunks"]:
        cid = cl.register_chunk(rec["content"], ChunkType(rec["chunk_type"]), metadata=rec["metadata"],
                                token_ids=rec["token_ids"])
        c = cl.registry.peek(cid)
        n += 1
        if rec["kv_length"] == 0 or c.kv_cache_allocated or sf is None:
            continue
        kv = sf.get_tensor(cid)  # [L, 2, Hkv, n, D]
        pages = pm.allocate_for_chunk(cid, rec["kv_length"])
        ps = pm.page_size
        slots = torch.arange(rec["kv_length"])
        dev = pm.kv_cache.device
        pg = torch.tensor(pages, dtype=torch.long)[slots // ps].to(dev)
        off = (slots % ps).to(dev)
        pm.kv_cache[:, pg, :, :, off, :] = kv.permute(3, 0, 1, 2, 4).to(dev, pm.kv_cache.dtype)
        c.page_table, c.kv_length, c.kv_offset = pages, rec["kv_length"], 0
        c.cached_position_start = rec["cached_position_start"]
        c.cascade_level = rec["cascade_level"]
        if cid + ".last_hidden" in sf.keys():
            c.last_hidden = sf.get_tensor(cid + ".last_hidden").to(dev)
        c.kv_cache_allocated = True
    return n
