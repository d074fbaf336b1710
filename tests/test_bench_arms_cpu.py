"""The two arms of bench.py measure the same thing: the reference harness
writes checkpoints of exactly the architectures this engine's synthetic
presets describe, and each secondary point of the reference line pairs with
one of ours (same model, batch, prompt length, k_norm init bound)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _harness():
    path = os.path.join(ROOT, "baseline", "ref_tp")
    if path not in sys.path:
        sys.path.insert(0, path)
    import harness

    return harness


def test_reference_checkpoints_have_our_architectures():
    from braidinfer_b200.utils.synthetic import PRESETS

    h = _harness()
    for name in ("llama3-8b", "llama3-70b", "tinyllama-1.1b", "qwen3-0.6b"):
        arch = h.ARCH[name]
        for key, value in arch.items():
            if key == "k_norm_range":
                continue
            assert PRESETS[name].get(key, "llama" if key == "model_type" else None) == value, (name, key)


def test_reference_secondary_points_pair_with_ours():
    import bench

    h = _harness()
    ours = {p[0]: p for p in bench.EXTRA_POINTS}
    for label, model, batch, plen, _warmup, _steps in h.REF_EXTRAS:
        assert label in ours, label
        _, m, b, n, k_norm = ours[label]
        assert (m, b, n) == (model, batch, plen)
        assert k_norm == h.ARCH[model].get("k_norm_range")
