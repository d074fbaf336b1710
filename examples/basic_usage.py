"""Batch generation with sampling settings (``LLM.generate``).

    python examples/basic_usage.py [--model DIR]

Without ``--model`` a small random-weight checkpoint is synthesised, so the
example runs anywhere (on CPU when no GPU is present).
"""
import argparse
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from braidinfer_b200 import LLM, SamplingParams  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    a = ap.parse_args()
    model = a.model
    if model is None:
        from braidinfer_b200.utils.synthetic import make_checkpoint
        model = make_checkpoint(tempfile.mkdtemp(), "tiny-llama", chat_template=True)
    llm = LLM(model, num_kvcache_blocks=64, kvcache_block_size=16)
    prompts = ["w5 w6 w7 w8", "w100 w200 w300", [11, 12, 13, 14, 15]]
    greedy = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8))
    sampled = llm.generate(prompts, SamplingParams(temperature=0.8, top_p=0.9, top_k=50, max_tokens=8, seed=1))
    for p, g, s in zip(prompts, greedy, sampled):
        print(f"{p!r}\n  greedy : {g['text']}\n  sampled: {s['text']}")
    print("streaming:", end=" ")
    for rec in llm.generate("w1 w2 w3", SamplingParams(temperature=0.0, max_tokens=6), stream=True):
        if not rec["finished"]:
            print(rec["text"], end=" ", flush=True)
    print("\nmetrics:", {k: v for k, v in llm.get_metrics().items() if k != "kv_pool"})


if __name__ == "__main__":
    main()
