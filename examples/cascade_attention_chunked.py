"""Cascade attention through the chunk API (the reference's
``examples/cascade_attention_chunked.py``): a shared system prompt and shared
documents are registered once as chunks, several users' questions are
answered over them, and ``preview_composition`` / ``get_chunk_stats`` report
the composition levels and the KV memory actually held.

    python examples/cascade_attention_chunked.py [--model DIR]

Level 0 is the system chunk, level 1 the context/output chunks, level 2 the
query (``preview_composition``'s ``num_levels``).  Memory figures come
from the KV pages the chunks own, not an estimate.
"""
import argparse
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from braidinfer_b200 import ChunkedLLM, ChunkType  # noqa: E402

DOCS = [
    "Python lists are ordered, mutable sequences; comprehensions build them from any iterable.",
    "Files are opened with open(); a with-block closes them even when an exception is raised.",
    "Decorators are callables that take a function and return a replacement function.",
]
QUESTIONS = ["How do I build a list of squares?", "How should I read a file safely?",
             "What does @functools.wraps do?", "Can a decorator take arguments?"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    ap.add_argument("--max-tokens", type=int, default=16)
    a = ap.parse_args()
    model = a.model
    if model is None:
        from braidinfer_b200.utils.synthetic import make_checkpoint
        model = make_checkpoint(tempfile.mkdtemp(), "tiny-llama", chat_template=True)
    cl = ChunkedLLM(model, num_kvcache_blocks=256, kvcache_block_size=16)
    sys_id = cl.register_chunk("You are a concise Python tutor.", ChunkType.SYSTEM_PROMPT)
    doc_ids = [cl.register_chunk(d, ChunkType.CONTEXT, metadata={"doc": i}) for i, d in enumerate(DOCS)]
    sp = dict(temperature=0.0, max_tokens=a.max_tokens)
    for i, question in enumerate(QUESTIONS):
        q = cl.register_chunk(question, ChunkType.QUERY, metadata={"user": i})
        prev = cl.preview_composition(sys_id, q, doc_ids)
        out = cl.generate_from_chunks(sys_id, q, doc_ids, sp)
        print(f"user {i}: {question!r} -> {out['text'][:80]!r}  "
              f"({prev['total_tokens']} tokens, {prev['num_levels']} levels)")
    st = cl.get_chunk_stats()
    shared_tokens = sum(cl.registry.peek(c).token_count for c in [sys_id] + doc_ids)
    print(f"shared chunks: {1 + len(DOCS)}, {shared_tokens} tokens cached once for {len(QUESTIONS)} users")
    print(f"KV held by chunks: {st['kv_pages_used']} pages = {st['memory_used_mb']:.2f} MB "
          f"(without sharing: {len(QUESTIONS)}x the shared part)")
    print(f"registry: {st['total_chunks']} chunks, hit rate {st['hit_rate']:.1%}")


if __name__ == "__main__":
    main()
