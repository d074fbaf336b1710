"""Compatibility checker verdicts on synthetic q/k-norm weights (parity of
thresholds with the reference's checker) and the CLI exit codes."""
import json

import torch

from braidinfer_b200.utils import kernel_compatibility as kc
from braidinfer_b200.utils.check_compatibility_cli import main
from braidinfer_b200.utils.synthetic import make_checkpoint


def _norms(kmax, n=4, extreme_layers=None):
    out = []
    for i in range(n):
        k = torch.ones(64)
        if extreme_layers is None or i in extreme_layers:
            k[0] = kmax
        out.append((i, torch.ones(64), k))
    return out


def test_normal_weights_compatible():
    r = kc.evaluate(kc.layer_metrics(_norms(1.0)))
    assert r.status == "COMPATIBLE" and r.score == 1.0 and r.estimated_amplification == 1.0


def test_extreme_weights_incompatible():
    r = kc.evaluate(kc.layer_metrics(_norms(96.5)))
    assert r.status == "INCOMPATIBLE" and r.score == 0.0
    assert "extreme" in r.reason and r.estimated_amplification > 1.0


def test_warning_band():
    # ratio 18 (in the warning band), 1/4 layers extreme, max 18 -> 0.4*0.2 + 0.3 + 0.3 = 0.68
    r = kc.evaluate(kc.layer_metrics(_norms(18.0, extreme_layers={0})))
    assert r.status == "WARNING" and abs(r.score - 0.68) < 1e-6


def test_checkpoint_and_cli(tmp_path):
    good = make_checkpoint(str(tmp_path / "good"), "tiny-qwen3", dtype=torch.float32)
    bad = make_checkpoint(str(tmp_path / "bad"), "tiny-qwen3", k_norm_range=100.0, dtype=torch.float32)
    llama = make_checkpoint(str(tmp_path / "llama"), "tiny-llama", dtype=torch.float32)
    assert main([good]) == 0
    assert main([bad, "-v", "--export", str(tmp_path / "r.json")]) == 2
    assert json.load(open(tmp_path / "r.json"))["status"] == "INCOMPATIBLE"
    assert main([llama]) == 0  # no q/k norms at all
    assert main([str(tmp_path / "missing")]) == 3
