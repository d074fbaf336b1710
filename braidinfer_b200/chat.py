"""Streaming chat over ``LLM.generate``: ``python -m braidinfer_b200.chat --model DIR``.

Behaviour of the reference's ``chat.py`` (``chat.py:17-372``): every turn the
whole conversation is rendered with the tokenizer's chat template (a plain
``role: content`` transcript when the tokenizer has none), generated with
streaming, and the reply is printed as it arrives with its token count,
tok/s and time to first token.  ``<think>…</think>`` spans are dropped from
the reply before it enters the history; the history keeps the last 10
exchanges.  Commands: ``exit``/``quit``/``q``, ``stats``, ``clear``.
``--debug-tokens`` prints the prompt's and the reply's token ids and the
special tokens among them.

``ChatSession.handle(line)`` runs one input line, so the loop can be driven by
scripted input (tests) as well as by the terminal loop in ``main``.
"""
from __future__ import annotations

import argparse
import sys
import time
from typing import Callable, Dict, List, Optional, Tuple

from .llm import LLM
from .sampling_params import SamplingParams

MAX_MESSAGES = 20  # last 10 exchanges


def strip_think(text: str) -> str:
    """Drop every closed ``<think>…</think>`` span; an unclosed one is kept."""
    out, pos = [], 0
    while True:
        a = text.find("<think>", pos)
        if a < 0:
            out.append(text[pos:])
            break
        out.append(text[pos:a])
        b = text.find("</think>", a)
        if b < 0:
            out.append(text[a:])
            break
        pos = b + len("</think>")
    return "".join(out)


def special_token_report(tokenizer, ids: List[int], limit: int = 50) -> List[str]:
    """``Position i: <tok> (ID: n)`` for the special tokens among the first ``limit`` ids."""
    special = set(getattr(tokenizer, "all_special_ids", []) or [])
    added = getattr(tokenizer, "added_tokens_decoder", {}) or {}
    special |= {i for i, t in added.items() if getattr(t, "special", False)}
    lines = []
    for i, t in enumerate(ids[:limit]):
        if t in special:
            lines.append(f"  Position {i}: {tokenizer.convert_ids_to_tokens(t)} (ID: {t})")
    return lines


class TurnStats:
    def __init__(self):
        self.runs: List[Tuple[int, float]] = []  # (tokens, seconds)

    def add(self, n: int, dt: float) -> None:
        if n > 0:
            self.runs.append((n, dt))

    def lines(self) -> List[str]:
        if not self.runs:
            return []
        tot_n = sum(n for n, _ in self.runs)
        tot_t = sum(t for _, t in self.runs)
        speeds = [(n / t, n, t) for n, t in self.runs if t > 0]
        out = ["=== Performance Statistics ===", f"Total generations: {len(self.runs)}",
               f"Total tokens generated: {tot_n}", f"Total generation time: {tot_t:.2f}s",
               f"Average speed: {tot_n / tot_t if tot_t > 0 else 0.0:.1f} tok/s"]
        if speeds:
            b, w = max(speeds), min(speeds)
            out += [f"Best run: {b[0]:.1f} tok/s ({b[1]} tokens in {b[2]:.2f}s)",
                    f"Worst run: {w[0]:.1f} tok/s ({w[1]} tokens in {w[2]:.2f}s)"]
        return out


def stream_reply(records, out: Callable[[str], None]) -> Tuple[str, List[int], Optional[float], float]:
    """Consume ``generate(..., stream=True)`` records, printing the text deltas;
    returns (final text, final token ids, seconds to first token, total seconds)."""
    t0 = time.perf_counter()
    first = None
    parts: List[str] = []
    text, ids = "", []
    for rec in records:
        if not rec.get("finished"):
            if first is None and rec["text"].strip():
                first = time.perf_counter() - t0
            parts.append(rec["text"])
        else:
            fin = rec["final_output"]
            text, ids = fin["text"], list(fin["token_ids"])
    if not text and parts:
        text = "".join(parts)
    out("".join(parts))
    return text, ids, first, time.perf_counter() - t0


class ChatSession:
    def __init__(self, llm: LLM, out: Callable[[str], None] = print, temperature: float = 0.7,
                 max_tokens: int = 512, debug_tokens: bool = False, show_prompt: bool = True):
        self.llm = llm
        self.out = out
        self.messages: List[Dict[str, str]] = []
        self.temperature = temperature
        self.max_tokens = max_tokens
        self.debug_tokens = debug_tokens
        self.show_prompt = show_prompt
        self.stats = TurnStats()

    def prompt(self) -> str:
        tok = self.llm.tokenizer
        if getattr(tok, "chat_template", None):
            return tok.apply_chat_template(self.messages, tokenize=False, add_generation_prompt=True)
        return "".join(f"{m['role']}: {m['content']}\n" for m in self.messages) + "assistant: "

    def handle(self, line: str) -> bool:
        """Run one input line; returns False when the session should end."""
        line = line.strip()
        low = line.lower()
        if low in ("exit", "quit", "q"):
            self.out("Goodbye!")
            return False
        if low == "stats":
            for s in self.stats.lines():
                self.out(s)
            return True
        if low == "clear":
            self.messages = []
            self.out("Conversation history cleared.")
            return True
        if not line:
            return True
        try:
            self.turn(line)
        except Exception as e:  # noqa: BLE001 - an interactive loop reports and continues
            self.out(f"Error: {type(e).__name__}: {e}")
        return True

    def turn(self, user_text: str) -> str:
        self.messages.append({"role": "user", "content": user_text})
        prompt = self.prompt()
        if self.show_prompt:
            self.out("[Prompt sent to model:]")
            self.out(repr(prompt))
        if self.debug_tokens:
            ids = self.llm.tokenizer.encode(prompt, add_special_tokens=False)
            self.out(f"[Prompt token IDs ({len(ids)} tokens):] {ids[:50]}{' ...' if len(ids) > 50 else ''}")
            for s in special_token_report(self.llm.tokenizer, ids):
                self.out(s)
        sp = SamplingParams(temperature=self.temperature, max_tokens=self.max_tokens)
        text, ids, ttft, dt = stream_reply(self.llm.generate(prompt, sp, stream=True), self.out)
        self.stats.add(len(ids), dt)
        if ids:
            self.out(f"[Generated {len(ids)} tokens in {dt:.2f}s = {len(ids) / max(dt, 1e-9):.1f} tok/s]")
        if ttft is not None:
            self.out(f"[Time to first token: {ttft:.3f}s]")
        if self.debug_tokens and ids:
            self.out(f"[Generated token IDs ({len(ids)} tokens):] {ids[:50]}{' ...' if len(ids) > 50 else ''}")
            for s in special_token_report(self.llm.tokenizer, ids):
                self.out(s)
        self.messages.append({"role": "assistant", "content": strip_think(text)})
        self.messages = self.messages[-MAX_MESSAGES:]
        return text


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="streaming chat over LLM.generate")
    ap.add_argument("--model", required=True, help="HF-layout checkpoint directory")
    ap.add_argument("--debug-tokens", action="store_true", help="show prompt/reply token ids and special tokens")
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--kv-pages", type=int, default=-1, help="KV pool pages (default: auto)")
    a = ap.parse_args(argv)
    t0 = time.perf_counter()
    llm = LLM(a.model, num_kvcache_blocks=a.kv_pages)
    print(f"Model loaded ({time.perf_counter() - t0:.1f}s). Commands: exit, stats, clear")
    sess = ChatSession(llm, print, a.temperature, a.max_tokens, a.debug_tokens)
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
        for s in sess.stats.lines():
            print(s)
        llm.exit()
    return 0


if __name__ == "__main__":
    sys.exit(main())
