"""Chat front-ends on CPU (reference ``chat.py`` and ``chat_chunked.py``):
scripted sessions through the session classes, and the real ``main`` loops
fed a script on standard input in a child process."""
import os
import subprocess
import sys

import torch

from braidinfer_b200 import LLM, ChunkedLLM
from braidinfer_b200.chat import ChatSession, strip_think
from braidinfer_b200.chat_chunked import ChunkedChatSession
from braidinfer_b200.utils.synthetic import make_checkpoint

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KW = dict(num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32")


def _ckpt(tmp_path):
    return make_checkpoint(str(tmp_path / "m"), "tiny-llama", seed=0, dtype=torch.float32, chat_template=True)


def test_strip_think():
    assert strip_think("a<think>x</think>b<think>y</think>c") == "abc"
    assert strip_think("a<think>unclosed") == "a<think>unclosed"
    assert strip_think("plain") == "plain"


def test_chat_session_keeps_history_and_stats(tmp_path):
    llm = LLM(_ckpt(tmp_path), **KW)
    lines = []
    s = ChatSession(llm, lines.append, temperature=0.0, max_tokens=4, debug_tokens=True)
    for x in ["w10 w11 w12", "stats", "w20 w21", "clear", "", "w30"]:
        assert s.handle(x)
    assert not s.handle("exit")
    text = "\n".join(lines)
    assert text.count("[Generated 4 tokens") == 3
    assert "=== Performance Statistics ===" in text and "Total generations: 1" in text
    assert "Conversation history cleared." in text and "Goodbye!" in text
    assert "[Prompt token IDs" in text and "Position 0: <s>" in text
    # after "clear" only the last exchange remains
    assert [m["role"] for m in s.messages] == ["user", "assistant"] and s.messages[0]["content"] == "w30"
    # the second turn's prompt carried the first exchange
    assert s.stats.runs and len(s.stats.runs) == 3


def test_chat_greedy_turn_equals_generate(tmp_path):
    llm = LLM(_ckpt(tmp_path), **KW)
    s = ChatSession(llm, lambda _: None, temperature=0.0, max_tokens=6, show_prompt=False)
    prompt_before = None
    s.messages.append({"role": "user", "content": "w5 w6 w7"})
    prompt_before = s.prompt()
    s.messages.clear()
    text = s.turn("w5 w6 w7")
    ref = llm.generate(prompt_before, __import__("braidinfer_b200").SamplingParams(temperature=0, max_tokens=6))[0]
    assert text == ref["text"]


def test_chunked_chat_session_reuses_conversation_chunks(tmp_path):
    cl = ChunkedLLM(_ckpt(tmp_path), **KW)
    lines = []
    s = ChunkedChatSession(cl, lines.append, max_conversation_chunks=4, temperature=0.0, max_tokens=4)
    for x in ["w10 w11", "w12 w13", "/cache", "/system w40 w41", "w10 w11", "/stats", "/clear"]:
        assert s.handle(x)
    assert not s.handle("q")
    text = "\n".join(lines)
    assert text.count("[Generated 4 tokens") == 3
    assert "System prompt updated!" in text and "Cache:" in text and "=== Chunk Statistics ===" in text
    # repeating the first user line deduplicated against its cached chunks
    assert "[Cache hits this generation:" in text
    roles = [cl.registry.peek(cid).metadata["role"] for _, cid in s.history] if s.history else []
    assert roles == []  # /clear emptied the history
    assert any(c.metadata.get("role") == "assistant" for c in cl.registry.chunks())


def _run_main(module, ck, script, extra=()):
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, "-m", module, "--model", ck, "--kv-pages", "64", "--temperature", "0",
                        "--max-tokens", "3", *extra], input=script, capture_output=True, text=True, timeout=300,
                       cwd=ROOT, env=env)
    assert p.returncode == 0, p.stderr[-2000:]
    return p.stdout


def test_chat_main_reads_stdin(tmp_path):
    out = _run_main("braidinfer_b200.chat", _ckpt(tmp_path), "w10 w11\nstats\nw12\nexit\n")
    assert out.count("[Generated 3 tokens") == 2 and "Goodbye!" in out and "Average speed" in out


def test_chunked_chat_main_reads_stdin(tmp_path):
    out = _run_main("braidinfer_b200.chat_chunked", _ckpt(tmp_path), "w10 w11\n/cache\nw12\n", ("--max-chunks", "6"))
    assert out.count("[Generated 3 tokens") == 2 and "Total chunks:" in out
