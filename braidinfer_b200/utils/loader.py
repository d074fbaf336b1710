"""HF checkpoint loader: safetensors (or ``.bin``) → this rank's weight shards.

Parity with ``braidinfer/utils/loader.py:14-104`` (local directory glob of
``*.safetensors``, ``.bin`` fallback, q/k/v → fused QKV and gate/up → fused
gate_up through the model's packed mapping, GPT-2 ``transformer.`` names,
unknown names skipped with a warning).  Each tensor is sliced to this rank's
shard and copied straight into the pre-allocated device weight, so a
checkpoint larger than host RAM still loads; tied embeddings need no
``lm_head.weight`` (the reference left it uninitialised).
"""
from __future__ import annotations

import glob
import os

import torch

from ..errors import ModelLoadError
from .logging import get_logger

log = get_logger("loader")


def iter_checkpoint(path: str):
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if files:
        from safetensors import safe_open

        for f in files:
            with safe_open(f, framework="pt", device="cpu") as sf:
                for name in sf.keys():
                    yield name, sf.get_tensor(name)
        return
    bins = sorted(glob.glob(os.path.join(path, "*.bin")))
    if not bins:
        raise ModelLoadError(f"no *.safetensors or *.bin weights under {path}")
    for f in bins:
        sd = torch.load(f, map_location="cpu", weights_only=True)
        for name, t in sd.items():
            yield name, t


def load_model(model, path: str) -> int:
    n = 0
    for name, t in iter_checkpoint(path):
        try:
            ok = model.load_hf_tensor(name, t)
        except Exception as e:
            raise ModelLoadError(f"loading {name} {tuple(t.shape)}: {e}") from e
        if ok:
            n += 1
        else:
            log.warning("skipping unknown checkpoint tensor %s", name)
    if n == 0:
        raise ModelLoadError(f"no tensor of {path} matched the model")
    return n
