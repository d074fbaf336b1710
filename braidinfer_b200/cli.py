"""Interactive chunk-composition shell: ``python -m braidinfer_b200.cli --model DIR``.

Command set of the reference's ``cli.py`` (``cli.py:242-268``, ``:544-617``):

    /system <text>        set the system prompt chunk
    /context <text>       add a context chunk (several allowed)
    /query <text>         set the query chunk (bare text does the same)
    /infer                stream a generation from the current chunks, retain
                          its output KV as an OUTPUT chunk, report TTFT and tok/s
    /clear [system|context|query]
    /list                 registry contents
    /stats                registry / KV-pool statistics
    /output               list output chunks
    /use-output <n>       add output chunk n as context (its KV is reused)
    /delete-output <n>    delete output chunk n
    /save <dir>, /load <dir>   persist / restore chunk KV
    /help, /exit, /quit

``CascadeSession`` holds the state and executes one command line at a time so
it can be driven by scripted input (tests) or by the terminal loop in
``main``.  Rendering uses ``rich`` when it is importable, plain text otherwise.
"""
from __future__ import annotations

import argparse
import sys
import time
from typing import Callable, List, Optional

from .chunked_llm import ChunkedLLM
from .chunks import ChunkType


class CascadeSession:
    def __init__(self, llm: ChunkedLLM, out: Callable[[str], None] = print, temperature: float = 0.7,
                 max_tokens: int = 512):
        self.llm = llm
        self.out = out
        self.system_id: Optional[str] = None
        self.context_ids: List[str] = []
        self.query_id: Optional[str] = None
        self.outputs: List[str] = []  # output chunk ids in creation order
        self.temperature = temperature
        self.max_tokens = max_tokens
        self.last: dict = {}

    # ------------------------------------------------------------------
    def handle(self, line: str) -> bool:
        """Execute one input line; returns False when the session should end."""
        line = line.strip()
        if not line:
            return True
        if not line.startswith("/"):
            return self.handle("/query " + line)
        cmd, _, arg = line.partition(" ")
        arg = arg.strip()
        h = {
            "/system": self._system, "/context": self._context, "/query": self._query, "/infer": self._infer,
            "/clear": self._clear, "/list": self._list, "/stats": self._stats, "/output": self._output,
            "/use-output": self._use_output, "/delete-output": self._delete_output, "/help": self._help,
            "/save": self._save, "/load": self._load,
        }.get(cmd)
        if cmd in ("/exit", "/quit"):
            return False
        if h is None:
            self.out(f"unknown command {cmd}; /help lists the commands")
            return True
        try:
            h(arg)
        except Exception as e:  # noqa: BLE001 - an interactive shell reports and continues
            self.out(f"error: {type(e).__name__}: {e}")
        return True

    def _system(self, arg):
        if not arg:
            return self.out("usage: /system <text>")
        self.system_id = self.llm.register_chunk(arg, ChunkType.SYSTEM_PROMPT)
        self.out(f"system chunk {self.system_id[:12]}")

    def _context(self, arg):
        if not arg:
            return self.out("usage: /context <text>")
        cid = self.llm.register_chunk(arg, ChunkType.CONTEXT)
        if cid not in self.context_ids:
            self.context_ids.append(cid)
        self.out(f"context chunk {cid[:12]} ({len(self.context_ids)} active)")

    def _query(self, arg):
        if not arg:
            return self.out("usage: /query <text>")
        self.query_id = self.llm.register_chunk(arg, ChunkType.QUERY)
        self.out(f"query chunk {self.query_id[:12]}")

    def _infer(self, _arg):
        if self.system_id is None:
            return self.out("a system prompt is required: /system <text>")
        if self.query_id is None:
            return self.out("a query is required: /query <text>")
        sp = dict(temperature=self.temperature, max_tokens=self.max_tokens, retain_output_cache=True)
        t0 = time.perf_counter()
        first = None
        n = 0
        text = []
        final = None
        for rec in self.llm.generate_from_chunks(self.system_id, self.query_id, self.context_ids or None, sp,
                                                 stream=True):
            if not rec.get("finished"):
                if first is None:
                    first = time.perf_counter()
                n += len(rec["token_ids"])
                text.append(rec["text"])
            else:
                final = rec
        dt = time.perf_counter() - t0
        self.out("".join(text))
        ttft = (first - t0) if first else dt
        tps = n / max(dt - ttft, 1e-9) if n > 1 else 0.0
        self.out(f"[{n} tokens, TTFT {1e3 * ttft:.1f} ms, {tps:.1f} tok/s]")
        if final is not None:
            sid = final.get("seq_id")
            oc = self.llm.register_output_chunk_from_retained(sid, metadata={"query_id": self.query_id})
            self.llm.release_retained_sequence(sid)
            if oc is not None and oc not in self.outputs:
                self.outputs.append(oc)
                self.out(f"output chunk #{len(self.outputs)} {oc[:12]} retained")
        self.last = {"tokens": n, "ttft_s": ttft, "tok_s": tps}

    def _clear(self, arg):
        if arg in ("", "all"):
            self.system_id, self.context_ids, self.query_id = None, [], None
        elif arg == "system":
            self.system_id = None
        elif arg in ("context", "contexts"):
            self.context_ids = []
        elif arg == "query":
            self.query_id = None
        else:
            return self.out("usage: /clear [system|context|query]")
        self.out("cleared " + (arg or "all active chunks"))

    def _list(self, _arg):
        rows = self.llm.list_chunks()
        if not rows:
            return self.out("registry is empty")
        for r in rows:
            flag = "kv" if r["kv_cache_allocated"] else "--"
            self.out(f"{r['chunk_id'][:12]} {r['chunk_type']:13s} {r['token_count']:6d} tok {flag}  "
                     f"{r['content_preview']}")

    def _stats(self, _arg):
        st = self.llm.get_chunk_stats()
        self.out(" ".join(f"{k}={v:.3f}" if isinstance(v, float) else f"{k}={v}" for k, v in st.items()))
        pool = self.llm.llm.page_manager.stats()
        self.out(" ".join(f"{k}={v}" for k, v in pool.items()))
        if self.last:
            self.out(f"last: {self.last}")

    def _output(self, _arg):
        if not self.outputs:
            return self.out("no output chunks yet")
        for i, oc in enumerate(self.outputs, 1):
            c = self.llm.registry.peek(oc)
            prev = c.content_preview if c else "(evicted)"
            self.out(f"#{i} {oc[:12]} {prev}")

    def _pick_output(self, arg) -> Optional[str]:
        try:
            i = int(arg)
        except ValueError:
            self.out("usage: /use-output <n>")
            return None
        if not 1 <= i <= len(self.outputs):
            self.out(f"no output chunk #{i}")
            return None
        return self.outputs[i - 1]

    def _use_output(self, arg):
        oc = self._pick_output(arg)
        if oc is not None and oc not in self.context_ids:
            self.context_ids.append(oc)
            self.out(f"output chunk {oc[:12]} added as context")

    def _delete_output(self, arg):
        oc = self._pick_output(arg)
        if oc is not None:
            self.llm.delete_chunk(oc)
            self.outputs.remove(oc)
            self.context_ids = [c for c in self.context_ids if c != oc]
            self.out(f"deleted output chunk {oc[:12]}")

    def _save(self, arg):
        from .persistence import save_chunks

        n = save_chunks(self.llm, arg or "braid_chunks")
        self.out(f"saved {n} chunks")

    def _load(self, arg):
        from .persistence import load_chunks

        n = load_chunks(self.llm, arg or "braid_chunks")
        self.out(f"loaded {n} chunks")

    def _help(self, _arg):
        self.out(__doc__.split("\n\n")[1])


def _printer():
    try:
        from rich.console import Console

        c = Console()
        return lambda s: c.print(s, markup=False, highlight=False)
    except Exception:  # pragma: no cover - rich is optional
        return print


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="chunk-composition shell")
    ap.add_argument("--model", required=True)
    ap.add_argument("--max-chunks", type=int, default=1000)
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--kv-pages", type=int, default=-1, help="KV pool pages (default: auto)")
    a = ap.parse_args(argv)
    out = _printer()
    llm = ChunkedLLM(a.model, max_chunks=a.max_chunks, num_kvcache_blocks=a.kv_pages)
    sess = CascadeSession(llm, out, a.temperature, a.max_tokens)
    out("braidinfer_b200 chunk shell; /help for commands")
    interactive = sys.stdin.isatty()
    while True:
        try:
            line = input("> " if interactive else "")
        except EOFError:
            break
        if not sess.handle(line):
            break
    return 0


if __name__ == "__main__":
    sys.exit(main())
