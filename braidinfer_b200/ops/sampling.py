"""Token sampler: greedy / temperature / min-p / top-k / top-p.

Semantics of ``braidinfer/layers/sampler.py:10-91`` (temperature 0 means
greedy argmax of the raw logits; min-p relative to the top probability, then
top-k, then nucleus, then renormalised sampling), computed without the
reference's per-row Python loops.  Sampling is a Gumbel-max race in logit
space, ``argmax(logit/T - log(-log u))``, with ``u`` from a counter-based hash
of ``(seed, step, token)`` (SplitMix64 finaliser, Steele et al. 2014), so a
request's samples are reproducible and identical on the CPU restatement and
the CUDA kernel.  Nucleus filtering keeps the smallest prefix of the sorted
distribution whose mass reaches ``top_p`` (the token that crosses the
threshold is kept).
"""
from __future__ import annotations

import torch

from ._ext import ext

_M64 = (1 << 64) - 1


def _s64(v: int) -> int:
    v &= _M64
    return v - (1 << 64) if v >= (1 << 63) else v


_G = _s64(0x9E3779B97F4A7C15)
_C1 = _s64(0xBF58476D1CE4E5B9)
_C2 = _s64(0x94D049BB133111EB)


def _srl(x: torch.Tensor, k: int) -> torch.Tensor:
    return (x >> k) & ((1 << (64 - k)) - 1)


def _mix(x: torch.Tensor) -> torch.Tensor:
    z = x + _G
    z = (z ^ _srl(z, 30)) * _C1
    z = (z ^ _srl(z, 27)) * _C2
    return z ^ _srl(z, 31)


def uniform_ref(seed: torch.Tensor, step: torch.Tensor, n: int) -> torch.Tensor:
    """u in (0, 1], shape [B, n]; bit-identical to the device ``hash_uniform``."""
    key = _mix(seed.long() ^ _mix(step.long()))
    idx = torch.arange(n, dtype=torch.int64)
    h = _mix(key[:, None] + idx[None, :])
    return (_srl(h, 40).double() + 1.0).float() / 16777216.0


def sample_ref(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
               min_p: torch.Tensor, seed: torch.Tensor, step: torch.Tensor) -> torch.Tensor:
    lf = logits.float()
    B, V = lf.shape
    greedy = lf.argmax(-1)
    t = temperature.float().clamp(min=1e-10)[:, None]
    z = lf / t
    zmax = z.max(-1, keepdim=True).values
    keep = torch.ones_like(z, dtype=torch.bool)
    mp = min_p.float()[:, None]
    keep &= (mp <= 0) | (z >= zmax + torch.log(mp.clamp(min=1e-30)))
    k = top_k.long()
    sorted_z, _ = z.sort(-1, descending=True)
    kth = sorted_z.gather(1, (k.clamp(1, V) - 1)[:, None])
    keep &= (k[:, None] <= 0) | (z >= kth)
    zk = z.masked_fill(~keep, float("-inf"))
    pr = torch.softmax(zk, -1)
    sp, _ = pr.sort(-1, descending=True)
    before = sp.cumsum(-1) - sp
    tp = top_p.float()[:, None]
    # threshold = smallest kept probability of the nucleus
    nuc = before < tp
    thr = torch.where(nuc, sp, torch.full_like(sp, 2.0)).min(-1, keepdim=True).values
    keep &= (tp >= 1.0) | (pr >= thr)
    u = uniform_ref(seed, step, V)
    g = -torch.log(-torch.log(u))
    score = torch.where(keep, z + g, torch.full_like(z, float("-inf")))
    sampled = score.argmax(-1)
    return torch.where(temperature == 0, greedy, sampled)


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           min_p: torch.Tensor, seed: torch.Tensor, step: torch.Tensor, out: torch.Tensor | None = None,
           all_greedy: bool = False) -> torch.Tensor:
    if logits.is_cuda:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device) if out is None else out
        ext().sample(out, logits, temperature, top_k, top_p, min_p, seed, step, bool(all_greedy))
        return out
    r = sample_ref(logits, temperature, top_k, top_p, min_p, seed, step).to(torch.int32)
    if out is not None:
        out.copy_(r)
        return out
    return r
