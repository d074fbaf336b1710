"""Branching conversations: retain a generated answer's KV as an OUTPUT chunk
and reuse it as context in follow-up turns without recomputing it.

    python examples/conversation_reuse.py [--model DIR]
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
    first = cl.generate_and_retain_output("w1 w2 w3", "w10 w11 w12", context=["w50 w51 w52 w53"],
                                          sampling_params=dict(temperature=0, max_tokens=8))
    print("turn 1:", first["text"], "-> output chunk", first["output_chunk_id"][:12])
    sys_id = first["chunk_ids"]["system"]
    for branch in ("w20 w21", "w30 w31 w32"):
        q = cl.register_chunk(branch, ChunkType.QUERY)
        before = cl.llm.model_runner.timing["prefill_tokens"]
        out = cl.generate_from_chunks(sys_id, q, [first["output_chunk_id"]], dict(temperature=0, max_tokens=6))
        print(f"branch {branch!r}: {out['text']}  (prefilled {cl.llm.model_runner.timing['prefill_tokens'] - before} "
              "tokens; the retained answer was not recomputed)")
    cl.release_retained_sequence(first["retained_seq_id"])


if __name__ == "__main__":
    main()
