"""Chat over chunks: ``python -m braidinfer_b200.chat_chunked --model DIR [--max-chunks N]``.

Behaviour of the reference's ``chat_chunked.py`` (``chat_chunked.py:18-406``):
the system prompt is a ``SYSTEM_PROMPT`` chunk; each user line becomes a
``QUERY`` chunk and is answered by ``ChunkedLLM.generate_from_chunks`` over
the last ``max_chunks`` conversation chunks; afterwards the user line and the
reply (``<think>`` spans removed) are registered as ``CONTEXT`` chunks with
``metadata.role`` = ``user`` / ``assistant``, so later turns attend to their
cached KV instead of re-reading the transcript.  Repeated content hits the
registry's deduplication (reported per turn as cache hits).

Commands: ``exit``/``quit``/``q``, ``/stats``, ``/clear`` (history only; the
chunks stay cached), ``/cache``, ``/system <prompt>``.

``ChunkedChatSession.handle(line)`` runs one input line, so the loop can be
driven by scripted input (tests) as well as by the terminal loop in ``main``.
"""
from __future__ import annotations

import argparse
import sys
import time
from typing import Callable, List, Optional, Tuple

from .chat import TurnStats, stream_reply, strip_think
from .chunked_llm import ChunkedLLM
from .chunks import ChunkType

DEFAULT_SYSTEM = "You are a helpful AI assistant. Please respond in English."


class ChunkedChatSession:
    def __init__(self, llm: ChunkedLLM, out: Callable[[str], None] = print, max_conversation_chunks: int = 20,
                 temperature: float = 0.7, max_tokens: int = 512, system_prompt: str = DEFAULT_SYSTEM):
        self.llm = llm
        self.out = out
        self.max_chunks = max_conversation_chunks
        self.temperature = temperature
        self.max_tokens = max_tokens
        self.history: List[Tuple[str, str]] = []  # (role, chunk id), oldest first
        self.system_id: Optional[str] = None
        self.stats = TurnStats()
        self.set_system(system_prompt)

    def set_system(self, prompt: str) -> None:
        self.system_id = self.llm.register_chunk(prompt, ChunkType.SYSTEM_PROMPT,
                                                 metadata={"role": "system", "timestamp": time.time()})
        self.out(f"System prompt registered (chunk: {self.system_id[:8]}...)")

    def context_ids(self) -> List[str]:
        return [cid for _, cid in self.history[-self.max_chunks:]]

    def handle(self, line: str) -> bool:
        """Run one input line; returns False when the session should end."""
        line = line.strip()
        low = line.lower()
        if low in ("exit", "quit", "q"):
            self.out("Goodbye!")
            return False
        if low == "/stats":
            for s in self.stats.lines() + self.chunk_stat_lines():
                self.out(s)
        elif low == "/clear":
            self.history = []
            self.out("Conversation history cleared. (Chunks remain in cache for potential reuse)")
        elif low == "/cache":
            st = self.llm.get_chunk_stats()
            self.out(f"Cache: {st['total_chunks']} chunks, {st['memory_used_mb']:.1f} MB")
            self.out(f"Hit rate: {st['hit_rate']:.1%} ({st['cache_hits']} hits)")
        elif low.startswith("/system"):
            prompt = line[len("/system"):].strip()
            if prompt:
                self.set_system(prompt)
                self.out("System prompt updated!")
            else:
                self.out("Please provide a system prompt.")
        elif line:
            try:
                self.turn(line)
            except Exception as e:  # noqa: BLE001 - an interactive loop reports and continues
                self.out(f"Error: {type(e).__name__}: {e}")
        return True

    def turn(self, user_text: str) -> str:
        hits0 = self.llm.get_chunk_stats()["cache_hits"]
        qid = self.llm.register_chunk(user_text, ChunkType.QUERY, metadata={"role": "user", "timestamp": time.time()})
        sp = dict(temperature=self.temperature, max_tokens=self.max_tokens, ignore_eos=False)
        recs = self.llm.generate_from_chunks(self.system_id, qid, self.context_ids() or None, sp, stream=True)
        text, ids, ttft, dt = stream_reply(recs, self.out)
        reply = strip_think(text).strip()
        uid = self.llm.register_chunk(user_text, ChunkType.CONTEXT, metadata={"role": "user", "timestamp": time.time()})
        self.history.append(("user", uid))
        aid = self.llm.register_chunk(reply, ChunkType.CONTEXT,
                                      metadata={"role": "assistant", "timestamp": time.time()})
        self.history.append(("assistant", aid))
        self.history = self.history[-2 * self.max_chunks:]
        self.stats.add(len(ids), dt)
        if ids:
            self.out(f"[Generated {len(ids)} tokens in {dt:.2f}s = {len(ids) / max(dt, 1e-9):.1f} tok/s]")
        if ttft is not None:
            self.out(f"[Time to first token: {ttft:.3f}s]")
        st = self.llm.get_chunk_stats()
        if st["cache_hits"] > hits0:
            self.out(f"[Cache hits this generation: {st['cache_hits'] - hits0}, Total hit rate: {st['hit_rate']:.1%}]")
        return text

    def chunk_stat_lines(self) -> List[str]:
        st = self.llm.get_chunk_stats()
        return ["=== Chunk Statistics ===", f"Total chunks: {st['total_chunks']}",
                f"Memory used: {st['memory_used_mb']:.1f} MB", f"Cache hits: {st['cache_hits']}",
                f"Hit rate: {st['hit_rate']:.1%}", f"Evictions: {st['evictions']}",
                f"Conversation chunks: {len(self.history)}"]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="chat over ChunkedLLM (cached conversation chunks)")
    ap.add_argument("--model", required=True, help="HF-layout checkpoint directory")
    ap.add_argument("--max-chunks", type=int, default=20, help="conversation chunks kept as context")
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--kv-pages", type=int, default=-1, help="KV pool pages (default: auto)")
    a = ap.parse_args(argv)
    t0 = time.perf_counter()
    llm = ChunkedLLM(a.model, max_chunks=1000, chunk_memory_ratio=0.5, enable_deduplication=True,
                     num_kvcache_blocks=a.kv_pages)
    print(f"Model loaded ({time.perf_counter() - t0:.1f}s). Commands: exit, /stats, /clear, /cache, /system <p>")
    sess = ChunkedChatSession(llm, print, a.max_chunks, a.temperature, a.max_tokens)
    interactive = sys.stdin.isatty()
    try:
        while True:
            try:
                line = input("\nYou: " if interactive else "")
            except EOFError:
                break
            if not sess.handle(line):
                break
    finally:
        for s in sess.stats.lines() + sess.chunk_stat_lines():
            print(s)
        llm.llm.exit()
    return 0


if __name__ == "__main__":
    sys.exit(main())
