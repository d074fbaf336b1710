"""Scripted CLI session (reference cli.py command set) and chunk persistence
round trip: restored chunks are reused without prefill and give identical
greedy output."""
import torch

from braidinfer_b200 import ChunkedLLM, ChunkType
from braidinfer_b200.cli import CascadeSession
from braidinfer_b200.persistence import load_chunks, save_chunks
from braidinfer_b200.utils.synthetic import make_checkpoint

KW = dict(num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32")


def _ckpt(tmp_path):
    return make_checkpoint(str(tmp_path / "m"), "tiny-llama", seed=0, dtype=torch.float32, chat_template=True)


def test_scripted_cli_session(tmp_path):
    cl = ChunkedLLM(_ckpt(tmp_path), **KW)
    lines = []
    s = CascadeSession(cl, lines.append, temperature=0.0, max_tokens=5)
    script = ["/help", "/infer", "/system w10 w11 w12", "/context w20 w21 w22 w23", "w30 w31",
              "/infer", "/output", "/use-output 1", "/query w40 w41", "/infer", "/list", "/stats",
              "/clear context", "/delete-output 1", "/bogus", "/exit"]
    alive = [s.handle(x) for x in script]
    assert alive[-1] is False and all(alive[:-1])
    text = "\n".join(lines)
    assert "a system prompt is required" in text
    assert text.count("tokens, TTFT") == 2
    assert "output chunk #1" in text and "added as context" in text and "deleted output chunk" in text
    assert "unknown command" in text
    assert s.last["tokens"] == 5


def test_persistence_round_trip(tmp_path):
    ck = _ckpt(tmp_path)
    g = torch.Generator().manual_seed(0)
    toks = [torch.randint(5, 1024, (n,), generator=g).tolist() for n in (20, 37, 9)]
    a = ChunkedLLM(ck, **KW)
    ids = [a.register_chunk(f"c{i}", t, token_ids=toks[i])
           for i, t in enumerate([ChunkType.SYSTEM_PROMPT, ChunkType.CONTEXT, ChunkType.QUERY])]
    sp = dict(temperature=0, max_tokens=6, ignore_eos=True)
    ref = a.generate_from_chunks(ids[0], ids[2], [ids[1]], sp)["token_ids"]
    assert save_chunks(a, str(tmp_path / "saved")) == 3
    b = ChunkedLLM(ck, **KW)
    assert load_chunks(b, str(tmp_path / "saved")) == 3
    assert b.registry.peek(ids[1]).kv_cache_allocated
    before = b.llm.model_runner.timing["prefill_tokens"]
    out = b.generate_from_chunks(ids[0], ids[2], [ids[1]], sp)["token_ids"]
    assert out == ref
    # only the private query tokens (+ generation prompt) were prefilled
    assert b.llm.model_runner.timing["prefill_tokens"] - before < len(toks[1])
