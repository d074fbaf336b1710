"""A shared system prompt cascaded under several requests on the plain
``LLM`` API (the reference's ``examples/cascade_attention.py``).

The system prompt is a cached chunk: its KV pages are computed once and every
request composes over it (``LLM.add_composition``), so N requests hold one
copy of the shared prefix plus their private tokens.  The script decodes the
requests as one batch and prints the KV page accounting against the same
requests without sharing.

    python examples/cascade_attention.py [--model DIR] [--requests N]
"""
import argparse
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from braidinfer_b200 import LLM, SamplingParams  # noqa: E402
from braidinfer_b200.chunks import Chunk, ChunkType  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    ap.add_argument("--requests", type=int, default=3)
    ap.add_argument("--max-tokens", type=int, default=16)
    a = ap.parse_args()
    model = a.model
    if model is None:
        from braidinfer_b200.utils.synthetic import make_checkpoint
        model = make_checkpoint(tempfile.mkdtemp(), "tiny-llama", chat_template=True)
    llm = LLM(model, num_kvcache_blocks=256, kvcache_block_size=16)
    system = "You are a helpful assistant with expertise in Python programming. " * 4
    queries = ["What is a list comprehension?", "How do I read a file?", "Explain decorators.",
               "What is a generator?", "How do dataclasses work?"][:a.requests]
    sysc = Chunk.from_content(system, ChunkType.SYSTEM_PROMPT, token_ids=llm.chat.chunk_tokens(
        ChunkType.SYSTEM_PROMPT, system))
    llm.prefill_chunks([sysc])                      # the shared prefix: computed once
    sp = SamplingParams(temperature=0.0, max_tokens=a.max_tokens)
    seqs = []
    for q in queries:
        qc = Chunk.from_content(q, ChunkType.QUERY, token_ids=llm.chat.chunk_tokens(ChunkType.QUERY, q))
        seqs.append(llm.add_composition({"system_chunk": sysc, "context_chunks": [], "query_chunk": qc}, sp))
    while any(not s.is_finished for s in seqs):
        llm.step()
    for q, s in zip(queries, seqs):
        print(f"{q!r}: {llm.decode(s.completion_token_ids)[:100]}")
    shared = len(sysc.page_table or [])
    n_sys = sysc.token_count
    per_req = [len(s.token_ids) for s in seqs]
    tok_with = n_sys + sum(per_req)
    tok_without = sum(n_sys + t for t in per_req)
    print(f"shared system chunk: {n_sys} tokens in {shared} pages, held once")
    print(f"KV tokens with sharing: {tok_with}; without: {tok_without} "
          f"({100 * (1 - tok_with / tok_without):.1f}% saved)")


if __name__ == "__main__":
    main()
