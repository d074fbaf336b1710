"""RMSNorm / LayerNorm.

Cast order follows HF and the reference (``braidinfer/layers/layernorm.py:35-44``):
variance in fp32, normalise in fp32, round to the activation dtype, then
multiply by the weight (rounded again).  That order keeps the extreme Qwen3
``k_norm`` weights (|w| up to ~100) finite in bf16.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ._ext import ext


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if x.is_cuda:
        out = torch.empty_like(x) if out is None else out
        ext().rms_norm(out, x, w, float(eps))
        return out
    y = rms_norm_ref(x, w, eps)
    if out is not None:
        out.copy_(y)
        return out
    return y


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                 out: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """``residual += x`` (activation dtype), return ``(rms_norm(residual), residual)``."""
    if x.is_cuda:
        out = torch.empty_like(x) if out is None else out
        ext().add_rms_norm(out, residual, x, w, float(eps))
        return out, residual
    residual.copy_((residual + x).to(residual.dtype))
    return rms_norm(residual, w, eps, out), residual


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    if x.is_cuda:
        out = torch.empty_like(x)
        ext().layer_norm(out, x, w, b, float(eps))
        return out
    return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), eps).to(x.dtype)


def row_rstd(x: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``1/rms`` of each row of ``x`` in fp32 (the scale a fused-norm GEMM applies)."""
    if out is None:
        out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    if x.is_cuda:
        ext().row_rstd(x, float(eps), out)
        return out
    out.copy_(torch.rsqrt(x.float().pow(2).mean(-1) + eps))
    return out
