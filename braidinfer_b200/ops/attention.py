"""Paged cascade attention over chunk lists, and the fused QKV epilogue.

KV layout (per layer): ``[P, 2, Hkv, page, D]`` — the reference's HND pool
(``braidinfer/engine/page_manager.py:39-42``) with one K and one V slab per
(page, head).  A flat *slot* is ``page * page_size + offset``.

Attention metadata describes, for every sequence of a batch, an ordered list
of KV *segments*: cached chunks (system, contexts, retained outputs) followed
by the sequence's private pages.  Segment ``s`` holds ``seg_len[s]`` keys that
start at slot ``seg_offset[s]`` of its first page (pages listed in
``page_ids[seg_page_indptr[s]:seg_page_indptr[s+1]]``), whose first key sits at
global position ``seg_pos0[s]`` in the current composition and was rotated
when cached at ``seg_pos0[s] - seg_delta[s]``.

Masking rule: key ``j`` of segment ``s`` is visible to a query at position
``p`` iff ``seg_pos0[s] + j <= p``.  This gives causal attention inside the
private segment and inside a chunk's own prefill, and full visibility of every
earlier chunk — the cascade of ``braidinfer/layers/cascade_attention.py:50-231``
without its per-page Python loop.

Queries are stored *unrotated*; the kernel rotates them by ``p - seg_delta[s]``
per segment (differential RoPE on the query side, O(|Q|) per chunk instead of
re-rotating O(|K|) cached keys).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ._ext import ext
from .norm import rms_norm_ref
from .rope import apply_rope_ref


@dataclass
class AttnMeta:
    """Per-forward attention plan (device tensors, int32)."""

    qo_indptr: torch.Tensor       # [B+1]
    positions: torch.Tensor       # [T]
    seg_indptr: torch.Tensor      # [B+1]
    seg_page_indptr: torch.Tensor  # [S+1]
    seg_offset: torch.Tensor      # [S]
    seg_len: torch.Tensor         # [S]
    seg_pos0: torch.Tensor        # [S]
    seg_delta: torch.Tensor       # [S]
    page_ids: torch.Tensor        # [NP]
    num_seqs: int
    max_q_len: int
    max_kv_len: int
    decode: bool = False          # every sequence has exactly one query token
    num_splits: int = 1           # split-KV factor of the decode kernel
    # host copies (CPU reference path and planning)
    host: Optional[dict] = None
    # shared-prefix decode: the group's tokens [grp_qo_indptr[0], grp_qo_indptr[1])
    # attend once to segments [grp_seg_indptr[0], grp_seg_indptr[1]) (split into
    # shared_splits key ranges); seq_nsh flags the member sequences, whose own
    # segment lists leave those segments out
    grp_qo_indptr: Optional[torch.Tensor] = None
    grp_seg_indptr: Optional[torch.Tensor] = None
    seq_nsh: Optional[torch.Tensor] = None
    shared_splits: int = 0
    grp_max_q: int = 0


def qkv_prepare(qkv: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                kv_layer: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
                cos: torch.Tensor, sin: torch.Tensor, q_norm: Optional[torch.Tensor] = None,
                k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6, use_rope: bool = True) -> torch.Tensor:
    """Split ``qkv[T, (Hq+2Hkv)*D]``; per-head q/k RMSNorm (Qwen3); RoPE on k;
    append k/v to the paged cache at ``slot_mapping``; return unrotated q ``[T, Hq, D]``.

    Replaces the reference's per-token ``.item()`` append loop
    (``braidinfer/kernels/kv_cache_utils.py:9-78``) with one kernel.
    """
    T = qkv.shape[0]
    if qkv.is_cuda:
        q = torch.empty(T, num_q_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
        ext().qkv_prepare(q, qkv, positions, slot_mapping, kv_layer, q_norm, k_norm, float(eps), cos, sin,
                          num_q_heads, num_kv_heads, head_dim, bool(use_rope))
        return q
    qs, ks = num_q_heads * head_dim, num_kv_heads * head_dim
    q = qkv[:, :qs].reshape(T, num_q_heads, head_dim)
    k = qkv[:, qs:qs + ks].reshape(T, num_kv_heads, head_dim)
    v = qkv[:, qs + ks:qs + 2 * ks].reshape(T, num_kv_heads, head_dim)
    if q_norm is not None:
        q = rms_norm_ref(q, q_norm, eps)
        k = rms_norm_ref(k, k_norm, eps)
    if use_rope:
        k = apply_rope_ref(k, positions, cos, sin).to(qkv.dtype)
    P, _, Hkv, page, D = kv_layer.shape
    slots = slot_mapping.long()
    pg, off = slots // page, slots % page
    kv_layer[pg, 0, :, off, :] = k.to(kv_layer.dtype)
    kv_layer[pg, 1, :, off, :] = v.to(kv_layer.dtype)
    return q.contiguous()


def qkv_gemm(x: torch.Tensor, w_qkv: torch.Tensor, bias: Optional[torch.Tensor], rms_eps: Optional[float],
             positions: torch.Tensor, slot_mapping: torch.Tensor, kv_layer: torch.Tensor, num_q_heads: int,
             num_kv_heads: int, head_dim: int, cos: torch.Tensor, sin: torch.Tensor,
             q_norm: Optional[torch.Tensor] = None, k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6,
             use_rope: bool = True, rs_vec: Optional[torch.Tensor] = None,
             sp: Optional[torch.Tensor] = None) -> torch.Tensor:
    """QKV projection (fused input RMSNorm when ``rms_eps`` is set, norm weight
    folded into ``w_qkv``) with the q/k-norm, RoPE(k) and paged KV append done
    in the GEMM epilogue on CUDA.  Returns unrotated q ``[T, Hq, D]``.
    ``rs_vec``/``sp``: precomputed ``1/rms`` and sequence-parallel parameters
    (CUDA tensor-parallel prefill)."""
    T = x.shape[0]
    if x.is_cuda:
        q = torch.empty(T, num_q_heads, head_dim, dtype=x.dtype, device=x.device)
        ext().gemm_qkv(q, x, w_qkv, bias, -1.0 if rms_eps is None else float(rms_eps), positions, slot_mapping,
                       kv_layer, q_norm, k_norm, float(eps), cos, sin, num_q_heads, num_kv_heads, head_dim,
                       bool(use_rope), rs_vec, sp)
        return q
    from .linear import linear

    qkv = linear(x, w_qkv, bias, rms_eps=rms_eps)
    return qkv_prepare(qkv, positions, slot_mapping, kv_layer, num_q_heads, num_kv_heads, head_dim, cos, sin,
                       q_norm, k_norm, eps, use_rope)


def attention_ref(q: torch.Tensor, kv_layer: torch.Tensor, meta: AttnMeta, cos: torch.Tensor,
                  sin: torch.Tensor, scale: float, use_rope: bool = True) -> torch.Tensor:
    """fp32 restatement of the cascade kernel (one softmax over all segments)."""
    h = meta.host
    T, Hq, D = q.shape
    P, _, Hkv, page, _ = kv_layer.shape
    G = Hq // Hkv
    out = torch.zeros(T, Hq, D, dtype=torch.float32)
    qo, segp = h["qo_indptr"], h["seg_indptr"]
    for b in range(meta.num_seqs):
        t0, t1 = int(qo[b]), int(qo[b + 1])
        if t1 == t0:
            continue
        pos = h["positions"][t0:t1].long()
        scores, values = [], []
        segs = list(range(int(segp[b]), int(segp[b + 1])))
        if meta.seq_nsh is not None and int(h["seq_nsh"][b]):
            # a shared-prefix group member: its shared segments are listed once for the group
            segs = list(range(int(h["grp_seg_indptr"][0]), int(h["grp_seg_indptr"][1]))) + segs
        for s in segs:
            n = int(h["seg_len"][s])
            if n == 0:
                continue
            p0, p1 = int(h["seg_page_indptr"][s]), int(h["seg_page_indptr"][s + 1])
            pages = h["page_ids"][p0:p1].long()
            slot = int(h["seg_offset"][s]) + torch.arange(n)
            pg = pages[slot // page]
            off = slot % page
            k = kv_layer[pg, 0, :, off, :].float()  # [n, Hkv, D]
            v = kv_layer[pg, 1, :, off, :].float()
            qq = q[t0:t1].float()
            if use_rope:
                qq = apply_rope_ref(qq, pos - int(h["seg_delta"][s]), cos, sin)
            kk = k.repeat_interleave(G, dim=1)  # [n, Hq, D]
            sc = torch.einsum("thd,nhd->htn", qq, kk) * scale
            kpos = int(h["seg_pos0"][s]) + torch.arange(n)
            mask = kpos[None, :] > pos[:, None]  # [t, n]
            sc = sc.masked_fill(mask[None], float("-inf"))
            scores.append(sc)
            values.append(v.repeat_interleave(G, dim=1))
        if not scores:
            continue
        sc = torch.cat(scores, dim=-1)
        vv = torch.cat(values, dim=0)
        p = torch.softmax(sc, dim=-1)
        p = torch.nan_to_num(p, nan=0.0)
        out[t0:t1] = torch.einsum("htn,nhd->thd", p, vv)
    return out.to(q.dtype).reshape(T, Hq * D)


def attention(q: torch.Tensor, kv_layer: torch.Tensor, meta: AttnMeta, cos: torch.Tensor, sin: torch.Tensor,
              scale: float, use_rope: bool = True, workspace: Optional[dict] = None) -> torch.Tensor:
    if q.is_cuda:
        T, Hq, D = q.shape
        out = torch.empty(T, Hq * D, dtype=q.dtype, device=q.device)
        ws = workspace or {}
        ext().attention(out, q, kv_layer, meta.qo_indptr, meta.positions, meta.seg_indptr,
                        meta.seg_page_indptr, meta.seg_offset, meta.seg_len, meta.seg_pos0, meta.seg_delta,
                        meta.page_ids, cos, sin, float(scale), bool(use_rope), int(meta.num_seqs),
                        int(meta.max_q_len), int(meta.max_kv_len), bool(meta.decode), int(meta.num_splits),
                        ws.get("partial_o"), ws.get("partial_lse"), meta.grp_qo_indptr, meta.grp_seg_indptr,
                        meta.seq_nsh, int(meta.shared_splits), int(meta.grp_max_q))
        return out
    return attention_ref(q, kv_layer, meta, cos, sin, scale, use_rope)
