"""Rotary position embedding tables and the PyTorch restatement of RoPE.

Neox half-split convention (``braidinfer/layers/rotary_embedding.py:6-24``):
``x1, x2 = x[:d/2], x[d/2:]``; ``out = (x1 cos - x2 sin, x2 cos + x1 sin)``.
Tables are built in fp32 exactly as HF builds them (fp32 ``inv_freq`` times
fp32 positions), so cached K matches an HF forward.  Llama-3 ``rope_scaling``
(type ``llama3``) is supported; the reference asserted it away
(``braidinfer/layers/rotary_embedding.py:76``).

Differential RoPE: a chunk cached at position ``c`` and composed at global
position ``g`` needs keys at ``g+i`` but holds keys rotated at ``c+i``.  Since
``<R(p) q, R(g+i) k> = <R(p-δ) q, R(c+i) k>`` with ``δ = g - c``, the attention
kernels rotate the *query* by ``p - δ`` per chunk instead of re-rotating the
cached keys (the reference re-rotated every cached key on every step,
``braidinfer/layers/cascade_attention.py:152-174``).
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def inv_freq(head_dim: int, theta: float, scaling: Optional[dict] = None) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    if not scaling:
        return inv
    kind = scaling.get("rope_type", scaling.get("type"))
    if kind in (None, "default"):
        return inv
    if kind == "linear":
        return inv / float(scaling["factor"])
    if kind == "llama3":
        # Frequency-dependent interpolation: long wavelengths are divided by
        # `factor`, short ones kept, the band between blended linearly in
        # 1/wavelength (Llama-3.1 release notes).
        factor = float(scaling["factor"])
        lo = float(scaling.get("low_freq_factor", 1.0))
        hi = float(scaling.get("high_freq_factor", 4.0))
        orig = float(scaling.get("original_max_position_embeddings", 8192))
        wavelen = 2 * math.pi / inv
        lo_wl, hi_wl = orig / lo, orig / hi
        scaled = torch.where(wavelen > lo_wl, inv / factor, inv)
        smooth = (orig / wavelen - lo) / (hi - lo)
        blended = (1 - smooth) * scaled / factor + smooth * scaled
        mid = (wavelen >= hi_wl) & (wavelen <= lo_wl)
        return torch.where(mid, blended, scaled)
    raise NotImplementedError(f"rope_scaling type {kind!r}")


def build_cos_sin(head_dim: int, theta: float, max_pos: int, scaling: Optional[dict] = None,
                  device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(cos, sin)`` fp32 tables of shape ``[max_pos, head_dim // 2]``."""
    inv = inv_freq(head_dim, theta, scaling)
    t = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    return freqs.cos().contiguous().to(device), freqs.sin().contiguous().to(device)


def apply_rope_ref(x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate ``x[..., T, H, D]`` at integer positions ``pos[T]`` (fp32 math)."""
    d2 = x.shape[-1] // 2
    c = cos[pos.long()].unsqueeze(-2)
    s = sin[pos.long()].unsqueeze(-2)
    xf = x.float()
    x1, x2 = xf[..., :d2], xf[..., d2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
