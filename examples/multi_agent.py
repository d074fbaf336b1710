"""Several agents with their own system prompts over the same shared context
(the reference's ``examples/multi_agent.py``), on ``ChunkedLLM``.

* Every agent's system prompt is one SYSTEM_PROMPT chunk; the report sections
  are CONTEXT chunks registered once.  Each section's KV is computed once and
  attended by every agent through the cascade (differential RoPE puts it at
  whatever position it lands in each composition).
* The agents' questions run as ONE batch (``batch_generate_from_chunks``):
  one decode step serves all agents.
* The collaborative round chains agents: each answer is retained as an OUTPUT
  chunk (its KV kept) and becomes context for the next agent.

    python examples/multi_agent.py [--model DIR] [--max-tokens N]

Without ``--model`` a tiny random-init checkpoint is generated, so the text
is noise; the chunk and KV accounting is the point.
"""
import argparse
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from braidinfer_b200 import ChunkedLLM, ChunkType  # noqa: E402

AGENTS = {
    "DataAnalyst": "You are a data analyst. Focus on patterns, trends and quantitative findings.",
    "BusinessStrategist": "You are a business strategy consultant. Focus on market opportunities.",
    "RiskAnalyst": "You are a risk assessment specialist. Identify risks and mitigations.",
    "TechAdvisor": "You are a technical implementation advisor. Focus on feasibility.",
}
REPORT = [
    "Q4 performance: revenue 12.5M (up 23% YoY); active users 2.1M (up 45%); churn 5.2% (down from 6.8%); "
    "server uptime 99.2% against a 99.9% target.",
    "Market context: industry growing 15% a year; the main competitor launched a similar feature last month; "
    "new regulations arrive in Q2; mobile is 73% of traffic.",
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default=None)
    ap.add_argument("--max-tokens", type=int, default=24)
    a = ap.parse_args()
    model = a.model
    if model is None:
        from braidinfer_b200.utils.synthetic import make_checkpoint
        model = make_checkpoint(tempfile.mkdtemp(), "tiny-llama", chat_template=True)
    cl = ChunkedLLM(model, max_chunks=1000, enable_deduplication=True, num_kvcache_blocks=256, kvcache_block_size=16)
    sp = dict(temperature=0.0, max_tokens=a.max_tokens)
    systems = {n: cl.register_chunk(p, ChunkType.SYSTEM_PROMPT, metadata={"agent": n}) for n, p in AGENTS.items()}
    ctx = [cl.register_chunk(t, ChunkType.CONTEXT, metadata={"document": f"report_section_{i + 1}"})
           for i, t in enumerate(REPORT)]
    question = "What are the top 3 priorities for next quarter based on this data?"

    print("=== Multi-agent analysis (one batch) ===")
    reqs = []
    for n, sid in systems.items():
        q = cl.register_chunk(question, ChunkType.QUERY, metadata={"agent": n})
        reqs.append({"system_chunk_id": sid, "query_chunk_id": q, "context_chunk_ids": ctx})
    before = cl.llm.model_runner.timing["prefill_tokens"]
    outs = cl.batch_generate_from_chunks(reqs, sp)
    for n, o in zip(systems, outs):
        print(f"{n}: {o['text'][:160]}")
    st = cl.get_chunk_stats()
    ctx_tokens = sum(cl.registry.peek(c).token_count for c in ctx)
    print(f"prefilled tokens: {cl.llm.model_runner.timing['prefill_tokens'] - before} "
          f"(the {ctx_tokens} context tokens once, not {len(AGENTS)} times)")
    without = len(AGENTS) * (2 + len(ctx))
    print(f"chunks: {st['total_chunks']} registered vs {without} without sharing; "
          f"KV pages held by chunks: {st['kv_pages_used']} ({st['memory_used_mb']:.2f} MB)")

    print("\n=== Collaborative round (each answer becomes the next agent's context) ===")
    chain = list(ctx)
    for n in ("DataAnalyst", "RiskAnalyst", "BusinessStrategist"):
        q = cl.register_chunk(f"{n}: build on the analysis so far. {question}", ChunkType.QUERY)
        out = cl.generate_from_chunks(systems[n], q, chain, dict(sp, retain_output_cache=True))
        oc = cl.register_output_chunk_from_retained(out["seq_id"], metadata={"agent": n})
        cl.release_retained_sequence(out["seq_id"])
        chain.append(oc)
        print(f"{n}: {out['text'][:160]}  [output chunk {oc[:8]}, {cl.registry.peek(oc).kv_length} KV tokens kept]")
    print(cl.get_chunk_stats())


if __name__ == "__main__":
    main()
