"""Numerical-risk check of a checkpoint's per-head q/k RMSNorm weights.

Parity with ``braidinfer/utils/kernel_compatibility.py:17-349`` (same
thresholds and verdicts so a model is classified identically): per layer the
max / median / max÷median of ``q_norm`` and ``k_norm`` weights; a layer is
*extreme* when either max exceeds 10; the score is
``0.4·ratio_score + 0.3·extreme_layer_score + 0.3·max_weight_score`` with
COMPATIBLE ≥ 0.8 > WARNING ≥ 0.5 > INCOMPATIBLE; the amplification estimate
compounds ``1 + 1e-3 · mean(max_k, max_q)`` over extreme layers.

Differences: the check reads only the norm tensors straight from the
safetensors files (no model construction, no GPU), and it is also available
on a loaded engine model.  The fused kernels of this package keep HF's
RMSNorm cast order (normalise in fp32, round, then scale), which is what keeps
extreme Qwen3 ``k_norm`` weights finite, so the verdict is advisory.
"""
from __future__ import annotations

import glob
import json
import math
import os
import re
from dataclasses import asdict, dataclass, field
from typing import Iterable, List, Optional, Tuple

import torch

from .logging import get_logger

log = get_logger("compat")

RATIO_LIMIT = 20.0
RATIO_WARN = 15.0
EXTREME_WEIGHT = 10.0
MAX_WEIGHT_LIMIT = 50.0
MAX_WEIGHT_WARN = 20.0
KERNEL_ERROR = 1e-3


@dataclass
class LayerMetrics:
    layer_idx: int
    max_k_weight: float
    max_q_weight: float
    median_k_weight: float
    median_q_weight: float
    k_weight_ratio: float
    q_weight_ratio: float
    has_extreme_weights: bool


@dataclass
class CompatibilityResult:
    status: str
    score: float
    reason: str
    layer_metrics: List[LayerMetrics] = field(default_factory=list)
    estimated_amplification: float = 1.0
    recommendations: List[str] = field(default_factory=list)

    def to_dict(self) -> dict:
        return asdict(self)


def _stats(w: Optional[torch.Tensor]) -> Tuple[float, float, float]:
    if w is None:
        return 1.0, 1.0, 1.0
    w = w.detach().float().cpu()
    mx, med = float(w.max()), float(w.median())
    ratio = (math.inf if mx != 0 else 1.0) if med == 0 else mx / med
    return mx, med, ratio


def layer_metrics(norms: Iterable[Tuple[int, Optional[torch.Tensor], Optional[torch.Tensor]]]) -> List[LayerMetrics]:
    out = []
    for idx, qn, kn in norms:
        if qn is None and kn is None:
            continue
        kmx, kmed, kr = _stats(kn)
        qmx, qmed, qr = _stats(qn)
        out.append(LayerMetrics(idx, kmx, qmx, kmed, qmed, kr, qr, kmx > EXTREME_WEIGHT or qmx > EXTREME_WEIGHT))
    return out


def _ratio_score(ms: List[LayerMetrics]) -> float:
    r = max(m.k_weight_ratio for m in ms)
    if r > RATIO_LIMIT:
        return 0.0
    if r > RATIO_WARN:
        return 0.5 * (RATIO_LIMIT - r) / (RATIO_LIMIT - RATIO_WARN)
    return 1.0


def _extreme_score(ms: List[LayerMetrics]) -> float:
    frac = sum(m.has_extreme_weights for m in ms) / len(ms)
    if frac > 0.5:
        return 0.0
    if frac > 0.3:
        return 1.0 - 2.0 * (frac - 0.3)
    return 1.0


def _max_weight_score(ms: List[LayerMetrics]) -> float:
    mx = max(m.max_k_weight for m in ms)
    if mx > MAX_WEIGHT_LIMIT:
        return 0.0
    if mx > MAX_WEIGHT_WARN:
        return (MAX_WEIGHT_LIMIT - mx) / (MAX_WEIGHT_LIMIT - MAX_WEIGHT_WARN)
    return 1.0


def evaluate(ms: List[LayerMetrics]) -> CompatibilityResult:
    if not ms:
        return CompatibilityResult("COMPATIBLE", 1.0, "Model has no per-head q/k norms.", [], 1.0,
                                   ["Model is compatible with fused kernels"])
    score = 0.4 * _ratio_score(ms) + 0.3 * _extreme_score(ms) + 0.3 * _max_weight_score(ms)
    status = "INCOMPATIBLE" if score < 0.5 else ("WARNING" if score < 0.8 else "COMPATIBLE")
    amp = 1.0
    for m in ms:
        if m.has_extreme_weights:
            amp *= 1.0 + KERNEL_ERROR * (m.max_k_weight + m.max_q_weight) / 2.0
    extreme = [m for m in ms if m.has_extreme_weights]
    if extreme:
        reason = (f"Found {len(extreme)}/{len(ms)} layers with extreme weights; "
                  f"Maximum weight: {max(m.max_k_weight for m in ms):.1f}; "
                  f"Estimated error amplification: {amp:.1f}x")
    else:
        reason = "Model weights are within normal ranges."
    recs = {"INCOMPATIBLE": ["Use standard kernels only",
                             "Consider model quantization or pruning to reduce weight magnitudes"],
            "WARNING": ["Test thoroughly before using fused kernels in production",
                        "Monitor generation quality for anomalies"],
            "COMPATIBLE": ["Model is compatible with fused kernels"]}[status]
    if extreme:
        recs = recs + [f"Layers {[m.layer_idx for m in extreme[:3]]} have particularly extreme weights"]
    return CompatibilityResult(status, score, reason, ms, amp, recs)


_NORM = re.compile(r"(?:^|\.)layers\.(\d+)\.self_attn\.([qk])_norm\.weight$")


def checkpoint_norms(path: str):
    """Yield ``(layer, q_norm, k_norm)`` read from a checkpoint directory."""
    if not os.path.isdir(path):
        raise FileNotFoundError(f"no checkpoint directory at {path}")
    found = {}
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files and not glob.glob(os.path.join(path, "*.bin")):
        raise FileNotFoundError(f"no *.safetensors or *.bin weights under {path}")
    if files:
        from safetensors import safe_open

        for f in files:
            with safe_open(f, framework="pt", device="cpu") as sf:
                for name in sf.keys():
                    m = _NORM.search(name)
                    if m:
                        found.setdefault(int(m.group(1)), {})[m.group(2)] = sf.get_tensor(name)
    else:
        for f in sorted(glob.glob(os.path.join(path, "*.bin"))):
            sd = torch.load(f, map_location="cpu", weights_only=True)
            for name, t in sd.items():
                m = _NORM.search(name)
                if m:
                    found.setdefault(int(m.group(1)), {})[m.group(2)] = t
    for idx in sorted(found):
        yield idx, found[idx].get("q"), found[idx].get("k")


def model_norms(model):
    for idx, w in enumerate(getattr(model, "layers", [])):
        qn, kn = getattr(w, "q_norm", None), getattr(w, "k_norm", None)
        yield idx, qn, kn


class FusedKernelCompatibilityChecker:
    """Object form kept for API parity; caches results by model name."""

    MAX_SAFE_WEIGHT_RATIO = RATIO_LIMIT
    WARNING_WEIGHT_RATIO = RATIO_WARN
    EXTREME_WEIGHT_THRESHOLD = EXTREME_WEIGHT

    def __init__(self):
        self.cache = {}

    def check_model(self, model, model_name: Optional[str] = None) -> CompatibilityResult:
        if model_name and model_name in self.cache:
            return self.cache[model_name]
        src = list(checkpoint_norms(model)) if isinstance(model, str) else model_norms(model)
        res = evaluate(layer_metrics(src))
        if model_name:
            self.cache[model_name] = res
        return res


def check_model_compatibility(model, model_name: Optional[str] = None) -> Tuple[bool, CompatibilityResult]:
    res = FusedKernelCompatibilityChecker().check_model(model, model_name)
    if res.status == "INCOMPATIBLE":
        log.error("model incompatible with fused kernels: %s", res.reason)
        return False, res
    if res.status == "WARNING":
        log.warning("fused kernels may cause issues: %s", res.reason)
    return True, res


def generate_compatibility_report(res: CompatibilityResult, model_name: str = "Unknown", verbose: bool = False) -> str:
    lines = ["Model Compatibility Report", "=" * 50, f"Model: {model_name}", f"Status: {res.status}",
             f"Score: {res.score:.2f}", f"Reason: {res.reason}",
             f"Estimated amplification: {res.estimated_amplification:.2f}x", "", "Recommendations:"]
    lines += [f"  - {r}" for r in res.recommendations]
    if verbose and res.layer_metrics:
        lines += ["", "Per-layer norm weights (max / median / ratio):"]
        for m in res.layer_metrics:
            flag = "  EXTREME" if m.has_extreme_weights else ""
            lines.append(f"  layer {m.layer_idx:3d}: k {m.max_k_weight:8.2f} / {m.median_k_weight:7.3f} / "
                         f"{m.k_weight_ratio:7.2f}   q {m.max_q_weight:8.2f} / {m.median_q_weight:7.3f}{flag}")
    return "\n".join(lines)


def export_json(res: CompatibilityResult, path: str) -> None:
    with open(path, "w") as f:
        json.dump(res.to_dict(), f, indent=1, default=float)
