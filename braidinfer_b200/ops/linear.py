"""GEMM entry points: ``y = x @ w.T`` with fused epilogues.

On CUDA these run the hand-written tcgen05 kernel (``csrc/gemm_tcgen05.cu``):
TMA-fed shared-memory stages, one elected thread issuing ``tcgen05.mma`` into a
TMEM accumulator, and an epilogue warp group that adds bias/residual or
applies SwiGLU before the bf16 store.  Decode-sized ``M`` swaps operands so the
weight rows fill the 128-wide MMA M dimension.

Epilogue rounding mirrors an HF forward: the GEMM result is rounded to bf16
before the residual add, and SwiGLU rounds gate, up and ``silu(gate)`` to
bf16 before the product (``braidinfer/layers/activation.py:6-13``).

SwiGLU weights are stored block-interleaved: rows ``[g0..g63, u0..u63, g64..]``
(blocks of ``SWIGLU_BLOCK``) so one 128-row tile holds matching gate and up
rows.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from ._ext import ext

SWIGLU_BLOCK = 64


def _round(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t.to(dtype).float() if dtype != torch.float32 else t


def _rstd(x: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)


def _acc(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], rms_eps: Optional[float]) -> torch.Tensor:
    y = F.linear(x.float(), w.float())
    if rms_eps is not None:
        y = y * _rstd(x, rms_eps)
    if bias is not None:
        y = y + bias.float()
    return y


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
           residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           rms_eps: Optional[float] = None) -> torch.Tensor:
    """``y = x @ w.T (+bias) (+residual)``.  With ``rms_eps`` the input is
    RMS-normalised on the fly: ``w`` must already carry the norm weight folded
    into its columns, and ``1/rms(x_t)`` scales each token's row."""
    if x.is_cuda:
        M = x.shape[0]
        out = torch.empty(M, w.shape[0], dtype=x.dtype, device=x.device) if out is None else out
        ext().gemm(out, x, w, bias, residual, 0, -1.0 if rms_eps is None else float(rms_eps))
        return out
    y = _acc(x, w, bias, rms_eps)
    if residual is not None:
        y = _round(y, x.dtype) + residual.float()
    y = y.to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def prefetch_next(w: Optional[torch.Tensor], tokens: int, skip: int = 0) -> int:
    """Name the weight of a later decode GEMM: the NEXT native launch pulls
    K-blocks ``[skip, skip + depth)`` of every K-slice of ``w`` into L2 once
    its own loads are issued (``gemm_prefetch_next``), so the weight stream
    continues across kernel boundaries.  Returns ``skip + depth`` (the blocks
    of each slice now requested).  No-op on CPU, for ``None`` and for
    prefill-sized ``tokens`` (> 64)."""
    if w is not None and w.is_cuda and tokens <= 64:
        return skip + int(ext().gemm_prefetch_next(w, int(tokens), int(skip)))
    return skip


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    """``[I, K] x2 -> [2*I_pad, K]`` with zero-padded ``I_pad = ceil(I/block)*block``."""
    I, K = gate.shape
    Ip = (I + block - 1) // block * block
    if Ip != I:
        z = gate.new_zeros(Ip - I, K)
        gate, up = torch.cat([gate, z]), torch.cat([up, z])
    g = gate.view(Ip // block, block, K)
    u = up.view(Ip // block, block, K)
    return torch.stack([g, u], dim=1).reshape(2 * Ip, K).contiguous()


def swiglu_ref_from_interleaved(y: torch.Tensor, dtype: torch.dtype, block: int = SWIGLU_BLOCK) -> torch.Tensor:
    M, N2 = y.shape
    y = y.view(M, N2 // (2 * block), 2, block)
    g = _round(y[:, :, 0], dtype)
    u = _round(y[:, :, 1], dtype)
    s = _round(F.silu(g), dtype)
    return (s * u).reshape(M, N2 // 2).to(dtype)


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, out: Optional[torch.Tensor] = None,
                  rms_eps: Optional[float] = None, rs_vec: Optional[torch.Tensor] = None,
                  sp: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(x @ Wg.T) * (x @ Wu.T)`` from the block-interleaved ``w_gu``.

    ``rs_vec`` (CUDA only) supplies each token's precomputed ``1/rms``; ``sp`` is
    the sequence-parallel parameter block (the GEMM waits for gathered rows)."""
    if x.is_cuda:
        M = x.shape[0]
        out = torch.empty(M, w_gu.shape[0] // 2, dtype=x.dtype, device=x.device) if out is None else out
        ext().gemm(out, x, w_gu, None, None, 1, -1.0 if rms_eps is None else float(rms_eps), rs_vec, sp)
        return out
    y = _acc(x, w_gu, None, rms_eps)
    r = swiglu_ref_from_interleaved(y, x.dtype)
    if out is not None:
        out.copy_(r)
        return out
    return r


def gelu_new(x: torch.Tensor) -> torch.Tensor:
    """GPT-2's tanh GELU (``braidinfer/layers/activation.py:16-25``)."""
    if x.is_cuda:
        out = torch.empty_like(x)
        ext().gelu_tanh(out, x)
        return out
    xf = x.float()
    return (0.5 * xf * (1.0 + torch.tanh(0.7978845608028654 * (xf + 0.044715 * xf.pow(3))))).to(x.dtype)
