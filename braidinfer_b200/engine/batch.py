"""Host-side planning of one forward pass: token inputs, KV write slots and the
cascade attention plan, packed into ONE int32 buffer so a step costs a single
host→device copy (and so CUDA-graph replays only refresh that buffer).

The reference rebuilt page indices inside every attention layer with Python
loops (``braidinfer/engine/page_manager.py:121-157``,
``braidinfer/layers/attention.py:55-124``); here the plan is built once per
step and shared by all layers.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from ..ops.attention import AttnMeta
from .sequence import SegmentRef

FIELDS = ("input_ids", "positions", "slots", "qo_indptr", "seg_indptr", "seg_page_indptr",
          "seg_offset", "seg_len", "seg_pos0", "seg_delta", "page_ids", "logits_idx")
# shared-prefix decode plans also carry: the group's token range, its shared
# segments (appended after every sequence's own), and a per-sequence member flag
GROUP_FIELDS = ("grp_qo_indptr", "grp_seg_indptr", "seq_nsh")


def _seg_key(s: SegmentRef, page_size: int):
    npg = -(-(s.offset + s.length) // page_size)
    return (tuple(s.pages[:npg]), s.offset, s.length, s.pos0, s.delta)


def find_shared_group(items: List["FwdItem"], page_size: int, min_keys: int = 256):
    """Decode items that attend to the same cached segments (same pages,
    offset, length, position and RoPE delta) can share one pass over them.
    Returns ``(member indices, shared segment keys)`` for the segment set that
    saves the most key reads (members x shared keys), or ``None`` when no
    segment of at least ``min_keys`` keys is used by two or more items."""
    from collections import Counter

    per_item = [{_seg_key(sg, page_size) for sg in it.segments if sg.length > 0} for it in items]
    cnt = Counter(k for keys in per_item for k in keys)
    best, best_gain = None, 0
    for k, c in cnt.items():
        if c < 2 or k[2] < min_keys:
            continue
        members = [i for i, keys in enumerate(per_item) if k in keys]
        common = set.intersection(*(per_item[i] for i in members))
        gain = (len(members) - 1) * sum(x[2] for x in common)
        if gain > best_gain:
            best, best_gain = (members, common), gain
    return best


@dataclass
class FwdItem:
    tokens: List[int]
    pos0: int                 # global position of tokens[0]
    priv_index0: int          # private-token index of tokens[0]
    priv_pages: List[int]
    priv_pos0: int            # global position of private token 0
    segments: List[SegmentRef] = field(default_factory=list)
    logits: bool = True


@dataclass
class Plan:
    arrays: dict
    num_seqs: int
    num_tokens: int
    max_q_len: int
    max_kv_len: int
    decode: bool
    sizes: dict


def build_plan(items: List[FwdItem], page_size: int, pad_seqs: int = 0, scratch_page: int = 0,
               seg_cap: Optional[int] = None, page_cap: Optional[int] = None, pad_tokens: int = -1,
               group: Optional[tuple] = None) -> Plan:
    """Flatten ``items`` into the kernel metadata.  ``pad_seqs`` appends dummy
    one-token sequences (CUDA-graph padding) that write to ``scratch_page``;
    ``pad_tokens >= 0`` appends ONE dummy sequence of that many tokens (padding
    of a prefill graph's token count), also confined to ``scratch_page`` and
    without a logits row.

    ``group = (n_members, shared keys)`` (decode plans, members first): the
    first ``n_members`` items skip the segments whose keys are in ``shared``;
    those segments are appended once after all others and described by
    ``grp_qo_indptr`` / ``grp_seg_indptr``; ``seq_nsh`` flags the members.
    ``group = (0, set())`` emits the same arrays for an empty group."""
    ids, pos, slots = [], [], []
    qo, segi = [0], [0]
    spi, soff, slen, spos0, sdelta, pids = [0], [], [], [], [], []
    lidx = []
    max_q = max_kv = 0
    n_members, shared = group if group is not None else (0, set())
    shared_segs = []
    for idx, it in enumerate(items):
        n = len(it.tokens)
        t0 = len(ids)
        ids.extend(it.tokens)
        pos.extend(range(it.pos0, it.pos0 + n))
        for k in range(it.priv_index0, it.priv_index0 + n):
            slots.append(it.priv_pages[k // page_size] * page_size + k % page_size)
        qo.append(len(ids))
        kv = 0
        for s in it.segments:
            if s.length <= 0:
                continue
            if idx < n_members and _seg_key(s, page_size) in shared:
                if idx == 0:
                    shared_segs.append(s)
                kv += s.length
                continue
            npg = -(-(s.offset + s.length) // page_size)
            pids.extend(s.pages[:npg])
            spi.append(len(pids))
            soff.append(s.offset)
            slen.append(s.length)
            spos0.append(s.pos0)
            sdelta.append(s.delta)
            kv += s.length
        priv_len = it.priv_index0 + n
        if priv_len > 0:
            npg = -(-priv_len // page_size)
            pids.extend(it.priv_pages[:npg])
            spi.append(len(pids))
            soff.append(0)
            slen.append(priv_len)
            spos0.append(it.priv_pos0)
            sdelta.append(0)
            kv += priv_len
        segi.append(len(slen))
        if it.logits and n > 0:
            lidx.append(t0 + n - 1)
        max_q = max(max_q, n)
        max_kv = max(max_kv, kv)
    for _ in range(pad_seqs):
        ids.append(0)
        pos.append(0)
        slots.append(scratch_page * page_size)
        qo.append(len(ids))
        pids.append(scratch_page)
        spi.append(len(pids))
        soff.append(0)
        slen.append(1)
        spos0.append(0)
        sdelta.append(0)
        segi.append(len(slen))
        lidx.append(len(ids) - 1)
        max_q = max(max_q, 1)
        max_kv = max(max_kv, 1)
    if pad_tokens >= 0:
        for j in range(pad_tokens):
            ids.append(0)
            pos.append(j)
            slots.append(scratch_page * page_size + j % page_size)
        qo.append(len(ids))
        if pad_tokens > 0:
            pids.append(scratch_page)
            spi.append(len(pids))
            soff.append(0)
            slen.append(min(pad_tokens, page_size))
            spos0.append(0)
            sdelta.append(0)
        segi.append(len(slen))
        max_q = max(max_q, pad_tokens)
    grp = None
    if group is not None:
        g0 = len(slen)
        for sg in shared_segs:
            npg = -(-(sg.offset + sg.length) // page_size)
            pids.extend(sg.pages[:npg])
            spi.append(len(pids))
            soff.append(sg.offset)
            slen.append(sg.length)
            spos0.append(sg.pos0)
            sdelta.append(sg.delta)
        grp = {"grp_qo_indptr": [0, n_members if shared_segs else 0], "grp_seg_indptr": [g0, len(slen)],
               "seq_nsh": [1 if i < n_members and shared_segs else 0 for i in range(len(qo) - 1)]}
    S = len(slen)
    if seg_cap is not None:
        if S > seg_cap:
            raise OverflowError("segment capacity")
        pad = seg_cap - S
        soff += [0] * pad
        slen += [0] * pad
        spos0 += [0] * pad
        sdelta += [0] * pad
        spi += [spi[-1]] * pad
    if page_cap is not None:
        if len(pids) > page_cap:
            raise OverflowError("page capacity")
        pids += [scratch_page] * (page_cap - len(pids))
    arrays = {
        "input_ids": ids, "positions": pos, "slots": slots, "qo_indptr": qo, "seg_indptr": segi,
        "seg_page_indptr": spi, "seg_offset": soff, "seg_len": slen, "seg_pos0": spos0, "seg_delta": sdelta,
        "page_ids": pids, "logits_idx": lidx,
    }
    if grp is not None:
        arrays.update(grp)
    arrays = {k: np.asarray(v, dtype=np.int32) for k, v in arrays.items()}
    sizes = {k: len(v) for k, v in arrays.items()}
    nseq = len(items) + pad_seqs + (1 if pad_tokens >= 0 else 0)
    return Plan(arrays, nseq, len(ids), max_q, max_kv, decode=(max_q == 1 and len(ids) == nseq), sizes=sizes)


def validate_plan(plan: Plan, page_size: int, num_pages: int, rope_len: Optional[int] = None) -> None:
    """Host-side check of a step's metadata before it is uploaded: every page
    id inside the KV pool, every KV slot inside the cache, every position
    inside the RoPE table, the index arrays non-decreasing, every segment
    given the pages its keys need.  Raises ``PlanValidationError`` naming the
    field; a kernel given such a plan would read or write outside its buffers."""
    from ..errors import PlanValidationError

    a = plan.arrays

    def bad(field: str, what: str):
        raise PlanValidationError(f"step plan: {field} {what}")

    n = len(a["input_ids"])
    pids, slots, pos = a["page_ids"], a["slots"], a["positions"]
    if pids.size and (pids.min() < 0 or pids.max() >= num_pages):
        bad("page_ids", f"outside the pool [0, {num_pages}): {int(pids.min())}..{int(pids.max())}")
    if slots.size and (slots.min() < 0 or slots.max() >= num_pages * page_size):
        bad("slots", f"outside the cache [0, {num_pages * page_size}): {int(slots.min())}..{int(slots.max())}")
    if rope_len is not None and pos.size and (pos.min() < 0 or pos.max() >= rope_len):
        bad("positions", f"outside the RoPE table [0, {rope_len}): {int(pos.min())}..{int(pos.max())}")
    for k in ("qo_indptr", "seg_indptr", "seg_page_indptr"):
        if a[k].size and (a[k][0] != 0 or np.any(np.diff(a[k]) < 0)):
            bad(k, "does not start at 0 or decreases")
    if a["qo_indptr"][-1] > n:
        bad("qo_indptr", f"ends past the {n} tokens")
    spi, off, ln = a["seg_page_indptr"], a["seg_offset"], a["seg_len"]
    if spi[-1] > len(pids):
        bad("seg_page_indptr", f"ends past the {len(pids)} page ids")
    if np.any(ln < 0) or np.any(off < 0):
        bad("seg_len/seg_offset", "negative")
    if a["seg_indptr"][-1] > len(ln):
        bad("seg_indptr", f"ends past the {len(ln)} segments")
    live = ln > 0
    need = -(-(off + ln) // page_size)
    if np.any(np.diff(spi)[:len(ln)][live] < need[live]):
        bad("seg_page_indptr", "gives a segment fewer pages than its keys need")
    li = a["logits_idx"]
    if li.size and (li.min() < 0 or li.max() >= n):
        bad("logits_idx", f"outside the {n} tokens")


def _fields(keys) -> tuple:
    return FIELDS + (GROUP_FIELDS if "seq_nsh" in keys else ())


def pack(plan: Plan) -> np.ndarray:
    return np.concatenate([plan.arrays[k] for k in _fields(plan.arrays)])


def unpack(buf: torch.Tensor, sizes: dict) -> dict:
    out, o = {}, 0
    for k in _fields(sizes):
        n = sizes[k]
        out[k] = buf[o:o + n]
        o += n
    return out


def make_meta(views: dict, plan: Plan, num_splits: int = 1, shared_splits: int = 0) -> AttnMeta:
    host = None
    if not views["qo_indptr"].is_cuda:
        host = {k: torch.from_numpy(v) for k, v in plan.arrays.items()}
    grouped = "seq_nsh" in views and shared_splits > 0
    return AttnMeta(qo_indptr=views["qo_indptr"], positions=views["positions"], seg_indptr=views["seg_indptr"],
                    seg_page_indptr=views["seg_page_indptr"], seg_offset=views["seg_offset"],
                    seg_len=views["seg_len"], seg_pos0=views["seg_pos0"], seg_delta=views["seg_delta"],
                    page_ids=views["page_ids"], num_seqs=plan.num_seqs, max_q_len=plan.max_q_len,
                    max_kv_len=plan.max_kv_len, decode=plan.decode, num_splits=num_splits, host=host,
                    grp_qo_indptr=views["grp_qo_indptr"] if grouped else None,
                    grp_seg_indptr=views["grp_seg_indptr"] if grouped else None,
                    seq_nsh=views["seq_nsh"] if grouped else None,
                    shared_splits=shared_splits if grouped else 0,
                    grp_max_q=plan.num_seqs if grouped else 0)
