"""Multi-agent style reuse of shared context chunks (``ChunkedLLM``).

Several queries run over the same system prompt and documents; each document
is prefilled once and reused at whatever position it lands in a composition.

    python examples/chunked_api.py [--model DIR]
"""
import argparse
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from braidinfer_b200 import ChunkedLLM, ChunkType  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    a = ap.parse_args()
    model = a.model
    if model is None:
        from braidinfer_b200.utils.synthetic import make_checkpoint
        model = make_checkpoint(tempfile.mkdtemp(), "tiny-llama", chat_template=True)
    cl = ChunkedLLM(model, num_kvcache_blocks=128, kvcache_block_size=16)
    sys_id = cl.register_chunk("w1 w2 w3 w4 w5", ChunkType.SYSTEM_PROMPT)
    docs = [cl.register_chunk(" ".join(f"w{100 + 10 * d + i}" for i in range(40)), ChunkType.CONTEXT)
            for d in range(3)]
    for i, order in enumerate([[0, 1], [1, 2], [2, 0, 1]]):
        q = cl.register_chunk(f"w{900 + i} w{901 + i}", ChunkType.QUERY)
        print(cl.preview_composition(sys_id, q, [docs[k] for k in order]))
        out = cl.generate_from_chunks(sys_id, q, [docs[k] for k in order], dict(temperature=0, max_tokens=6))
        print(f"query {i} over docs {order}: {out['text']}")
    print("prefilled tokens in total:", cl.llm.model_runner.timing["prefill_tokens"])
    print(cl.get_chunk_stats())


if __name__ == "__main__":
    main()
