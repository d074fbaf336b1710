"""The reference arm's harness (``baseline/ref_tp/harness.py``) on CPU: the
streamed synthetic checkpoint loads through safetensors, the transformers-5.5
config shim gives the reference a ``None`` rope_scaling with θ kept, and the
tensor-parallel build swaps in the reference's own NCCL/gloo all-reduce
``RowParallelLinear`` over a per-rank shard (gloo ranks, world 2)."""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "baseline", "ref_tp")
REF = os.path.join(ROOT, "baseline", "_ref")

TINY = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
            intermediate_size=688, vocab_size=1024, rms_norm_eps=1e-6, rope_theta=10000.0,
            max_position_embeddings=4096)


def _harness():
    if HARNESS not in sys.path:
        sys.path.insert(0, HARNESS)
    import harness

    harness.ARCH.setdefault("tiny-llama", TINY)
    return harness


def test_streamed_checkpoint_and_rope_shim(tmp_path):
    h = _harness()
    d = h.write_checkpoint(str(tmp_path / "ck"), "tiny-llama", tp=2, seed=1)
    from safetensors import safe_open

    with safe_open(os.path.join(d, "model.safetensors"), "pt", "cpu") as f:
        q = f.get_tensor("model.layers.1.self_attn.q_proj.weight")
        o = f.get_tensor("model.layers.0.self_attn.o_proj.weight")
        n = f.get_tensor("model.norm.weight")
    assert q.shape == (2 * 64, 256) and o.shape == (256, 2 * 64) and q.dtype == torch.bfloat16
    assert abs(q.float().std().item() - 0.02) < 2e-3 and torch.all(n == 1)
    h.apply_rope_config_shim()
    from transformers import AutoConfig

    cfg = AutoConfig.from_pretrained(d)
    assert cfg.rope_scaling is None and cfg.rope_theta == 10000.0 and cfg.num_attention_heads == 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, port, d, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        h = _harness()
        sys.path.insert(0, REF)
        h.apply_rope_config_shim()
        h.install_tp_row_parallel()
        from transformers import AutoConfig

        from braidinfer.models.llama import LlamaForCausalLM
        from braidinfer.utils.loader import load_model

        m = LlamaForCausalLM(AutoConfig.from_pretrained(d))
        load_model(m, d)
        o = m.model.layers[0].self_attn.o_proj
        x = torch.randn(3, o.weight.shape[1], generator=torch.Generator().manual_seed(rank))
        y = o(x)
        want = torch.nn.functional.linear(x, o.weight)
        dist.all_reduce(want)
        q.put((rank, type(o).__name__, tuple(o.weight.shape), tuple(m.model.layers[0].mlp.down_proj.weight.shape),
               bool(torch.allclose(y, want, atol=1e-5))))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "braidinfer")), reason="reference not installed")
@pytest.mark.timeout(300)
def test_tp_build_uses_reference_all_reduce(tmp_path):
    h = _harness()
    d = h.write_checkpoint(str(tmp_path / "ck"), "tiny-llama", tp=2)
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_tp_worker, args=(r, port, d, q)) for r in range(2)]
    [p.start() for p in ps]
    res = [q.get(timeout=240) for _ in range(2)]
    [p.join(timeout=60) for p in ps]
    for rank, name, o_shape, down_shape, ok in res:
        assert name == "RowParallelLocalShard"
        assert o_shape == (256, 128) and down_shape == (256, 344)
        assert ok, f"rank {rank}: row-parallel output is not the all-reduced sum"


def test_qwen3_checkpoint_has_head_norms_with_extreme_k_norm(tmp_path):
    """The reference arm's Qwen3 checkpoint: per-head q_norm / k_norm tensors,
    k_norm drawn up to |w| = 100, the reference's own lm_head written out."""
    h = _harness()
    h.ARCH.setdefault("tiny-qwen3", dict(TINY, model_type="qwen3", tie_word_embeddings=True, k_norm_range=100.0))
    d = h.write_checkpoint(str(tmp_path / "q3"), "tiny-qwen3", seed=2)
    import json

    from safetensors import safe_open

    cfg = json.load(open(os.path.join(d, "config.json")))
    assert cfg["model_type"] == "qwen3" and cfg["architectures"] == ["Qwen3ForCausalLM"]
    assert "k_norm_range" not in cfg
    with safe_open(os.path.join(d, "model.safetensors"), "pt", "cpu") as f:
        kn = f.get_tensor("model.layers.1.self_attn.k_norm.weight").float()
        qn = f.get_tensor("model.layers.0.self_attn.q_norm.weight").float()
        assert "lm_head.weight" in f.keys()
    assert kn.shape == (64,) and 50 < kn.abs().max().item() <= 100
    assert torch.equal(qn, torch.ones(64))
