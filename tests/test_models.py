"""Model families beyond Llama (reference ``braidinfer/models/qwen3.py:208-373``,
``gpt2.py:129-204``, ``ernie.py:92-217``) through the engine, against the
independent fp32 oracle on CPU, and the native kernels against the CPU
engine on the GPU.

* Qwen3: per-head q_norm/k_norm (with k_norm weights drawn up to |w| = 100,
  the extreme-weight case of the Qwen3-0.6B benchmark configuration), tied
  LM head, non-unit RMSNorm weights (folded into the following GEMMs).
* GPT-2: learned positions, LayerNorm, tanh-GELU, Conv1D weights, tied head.
* ERNIE-4.5: interleaved ("GLM") rotary pairs, handled by a q/k row
  permutation at load time.
Each is checked on plain generation and on a chunk composition (cascade
with differential RoPE vs the block-causal oracle).
"""
import pytest
import torch
from safetensors.torch import load_file

from braidinfer_b200 import LLM, ChunkedLLM, ChunkType, SamplingParams
from braidinfer_b200.utils import oracle
from braidinfer_b200.utils.synthetic import hf_config, make_checkpoint

KW = dict(num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32")
TYPES = [ChunkType.SYSTEM_PROMPT, ChunkType.CONTEXT, ChunkType.CONTEXT, ChunkType.QUERY]
CASES = {
    "tiny-qwen3": dict(k_norm_range=100.0, norm_jitter=0.3),
    "tiny-gpt2": dict(),
    "tiny-ernie": dict(norm_jitter=0.3),
}


@pytest.fixture(scope="module", params=list(CASES))
def model(request, tmp_path_factory):
    name = request.param
    d = make_checkpoint(str(tmp_path_factory.mktemp(name)), name, seed=1, dtype=torch.float32, **CASES[name])
    return name, d, hf_config(name), load_file(d + "/model.safetensors")


def _max_diff(got, ref):
    return max((a[0] - b).abs().max().item() for a, b in zip(got, ref))


def _scale(ref):
    return max(b.abs().max().item() for b in ref)


def test_generate_matches_oracle(model):
    name, d, cfg, sd = model
    llm = LLM(d, **KW)
    llm.model_runner.capture_logits = []
    prompt = list(range(5, 60))
    out = llm.generate(prompt, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))[0]
    toks, lg = oracle.greedy(cfg, sd, prompt, [1] * len(prompt), 0, 8)
    assert out["token_ids"] == toks
    assert _max_diff(llm.model_runner.capture_logits, lg) < 1e-4 * max(1.0, _scale(lg))


def test_cascade_matches_block_causal_oracle(model):
    name, d, cfg, sd = model
    g = torch.Generator().manual_seed(0)
    chunks = [torch.randint(3, 1024, (n,), generator=g).tolist() for n in (24, 40, 33, 12)]
    cl = ChunkedLLM(d, **KW)
    ids = [cl.register_chunk(f"c{i}", t, token_ids=chunks[i]) for i, t in enumerate(TYPES)]
    cl.llm.model_runner.capture_logits = []
    out = cl.generate_from_chunks(ids[0], ids[3], ids[1:3], dict(temperature=0, max_tokens=6, ignore_eos=True))
    blocks = sum([[i] * len(t) for i, t in enumerate(chunks)], [])
    toks, lg = oracle.greedy(cfg, sd, sum(chunks, []), blocks, 3, 6)
    assert out["token_ids"] == toks
    assert _max_diff(cl.llm.model_runner.capture_logits, lg) < 1e-4 * max(1.0, _scale(lg))


def test_qwen3_extreme_k_norm_reaches_random_init(tmp_path):
    """``init_k_norm_range`` (benchmark random init) draws k_norm weights up to the bound."""
    d = make_checkpoint(str(tmp_path / "q"), "tiny-qwen3", write_weights=False)
    llm = LLM(d, load_weights=False, init_k_norm_range=100.0, **KW)
    kn = torch.stack([w.k_norm for w in llm.model_runner.model.layers])
    assert kn.abs().max().item() > 50 and kn.abs().max().item() <= 100


@pytest.mark.gpu
def test_native_greedy_matches_cpu_engine(model):
    """bf16 native kernels vs the fp32 CPU engine: first logits within a
    relative bound and the same first greedy tokens.  For Qwen3 this bounds
    the error of the folded input RMSNorm and of the epilogue q/k-norm with
    k_norm weights up to |w| = 100 at model level."""
    name, _, _, _ = model
    import tempfile

    d = make_checkpoint(tempfile.mkdtemp(prefix=f"gpu_{name}_"), name, seed=1, dtype=torch.bfloat16,
                        **CASES[name])
    prompt = list(range(3, 150))
    res = []
    for kw in (dict(enforce_eager=True), dict(device="cpu", dtype="float32")):
        llm = LLM(d, num_kvcache_blocks=32, kvcache_block_size=16, **kw)
        llm.model_runner.capture_logits = []
        o = llm.generate(prompt, SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))[0]
        res.append((o["token_ids"], llm.model_runner.capture_logits[0][0]))
    (tg, lg), (tc, lc) = res
    err = (lg - lc).abs().max().item()
    assert err / lc.abs().max().item() < 0.06, err
    # random-init logits are nearly flat: the GPU's first token must be the
    # CPU's argmax up to the measured error (a near-tie may flip either way)
    assert lc[tg[0]].item() >= lc.max().item() - 2 * err
