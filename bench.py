"""Headline benchmark: batched greedy decode throughput (tokens/s) of a
Llama-3-8B-architecture model (random-init bf16 weights, synthetic prompts),
tensor-parallel over the GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--prompt-len S]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)
    python bench.py --impl reference ...                     (the reference build)

Timing: W untimed decode steps, then K timed decode steps bracketed by a
barrier and ``torch.cuda.synchronize()``.  ``value`` is device time: CUDA
events around each step's graph replay, summed, max over ranks.  ``e2e`` is
the same K steps timed on the host through the public engine API
(``LLM.step``), which includes each step's host->device metadata upload from
pinned memory and the device->host read of the sampled tokens.  Weights
(16 GB) exceed L2 (126 MB) so no flush is needed between steps.

The default 1-GPU run (no --model / --batch) then measures secondary points of
the baseline configurations the same way and adds them under
``other_configs``: Qwen3-0.6B bs1/bs8 (k_norm weights up to |w| = 100),
TinyLlama-1.1B bs8, Llama-3-8B bs1/bs32 (64 timed steps each) and the
TinyLlama cached-chunk TTFT.  ``--no-extras`` skips them.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))

PUBLISHED_BS8 = 237.0  # reference README.md:68, RTX 4090 / TinyLlama (other hardware & model)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--workload", default="decode", choices=["decode", "ttft", "cascade"],
                    help="decode: batched decode throughput (headline); ttft: time to first token with cached "
                         "chunks vs full prefill (TinyLlama cascade/RAG config); cascade: shared-context "
                         "chunk under concurrent queries (Llama-3-70B TP8 config)")
    ap.add_argument("--ctx-len", type=int, default=8192, help="cascade: shared context chunk tokens")
    ap.add_argument("--query-len", type=int, default=256, help="cascade: tokens per query")
    ap.add_argument("--no-extras", action="store_true",
                    help="1-GPU default run: skip the secondary configuration points (other models, batches, TTFT)")
    a = ap.parse_args()
    a.model_given = any(x == "--model" or x.startswith("--model=") for x in sys.argv[1:])
    a.batch_given = any(x == "--batch" or x.startswith("--batch=") for x in sys.argv[1:])
    return a


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,timestamp")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = None
        self.window = None  # (t0, t1) epoch seconds of the timed region; samples outside are dropped

    def mark(self, t0: float, t1: float) -> None:
        self.window = (t0, t1)

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        import datetime

        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[9], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                ts = None
            lines.append((ts, parts))
        where = "whole run"
        if self.window is not None:
            inside = [x for x in lines if x[0] is not None and self.window[0] <= x[0] <= self.window[1]]
            where = "timed region"
            if len(inside) < 2:  # very short timed regions: the samples closest around it
                mid = 0.5 * (self.window[0] + self.window[1])
                inside = sorted((x for x in lines if x[0] is not None), key=lambda x: abs(x[0] - mid))[:3]
                where = "3 samples nearest the timed region"
            lines = inside
        for _, parts in lines:
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "sampled": where}


def make_config_dir(preset: str, with_weights: bool, rank: int = 0) -> str:
    from braidinfer_b200.utils.synthetic import make_checkpoint

    d = os.path.join(tempfile.gettempdir(), f"braid_bench_{preset}_{'w' if with_weights else 'cfg'}")
    if rank == 0 and not os.path.exists(os.path.join(d, "config.json" if not with_weights else "model.safetensors")):
        make_checkpoint(d, preset, write_weights=with_weights)
    return d


def prompts_for(batch: int, plen: int, vocab: int, seed: int = 3):
    import torch

    g = torch.Generator().manual_seed(seed)
    return [torch.randint(3, vocab, (plen,), generator=g).tolist() for _ in range(batch)]


def timed_decode(llm, args, n: int):
    """W untimed then K timed decode steps of every running sequence through
    ``LLM.step``; returns (device ms = sum of graph-replay events, max over
    ranks; wall seconds, max over ranks; our kernel launches per step; clocks)."""
    import torch
    import torch.distributed as dist

    runner = llm.model_runner
    # the clock sampler starts before warm-up (nvidia-smi needs ~1 s to start)
    # and keeps only the samples taken inside the timed region
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for _ in range(args.warmup):
            llm.step()
        # count our kernel launches of one decode step (graph contents)
        launches = runner.launches_per_decode_step(args.batch)
        torch.cuda.synchronize()
        if n > 1:
            dist.barrier()
        torch.cuda.synchronize()
        runner.event_log = []
        e0 = time.time()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            llm.step()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        clocks.mark(e0, time.time())
    if n > 1:
        dist.barrier()
    torch.cuda.synchronize()
    dev_ms = sum(a.elapsed_time(b) for a, b in runner.event_log)
    runner.event_log = None
    if len(llm.scheduler.running) != args.batch:
        raise RuntimeError(f"batch shrank during the timed region: {len(llm.scheduler.running)} running, "
                           f"{len(llm.scheduler.waiting)} waiting, {llm.scheduler.num_preemptions} preemptions "
                           f"(max_model_len {llm.config.max_model_len})")
    t = torch.tensor([dev_ms, wall], device="cuda", dtype=torch.float64)
    if n > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0]), float(t[1]), launches, clocks


def init_dist(n: int):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if n > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank


# --------------------------------------------------------------------- ours
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from braidinfer_b200 import LLM, SamplingParams
    from braidinfer_b200.ops import _ext

    n = args.gpus
    rank = init_dist(n)
    cfg_dir = make_config_dir(args.model, with_weights=False, rank=rank)
    if n > 1:
        dist.barrier()
    max_len = args.prompt_len + args.warmup + args.steps + 64
    page = 256
    pages = args.batch * (-(-max_len // page)) + 8
    llm = LLM(cfg_dir, load_weights=False, tensor_parallel_size=n, max_num_seqs=args.batch,
              max_model_len=max_len, num_kvcache_blocks=pages, kvcache_block_size=page,
              max_graph_batch=max(args.batch, 1), comm_backend=args.comm, max_num_batched_tokens=max(16384, max_len))
    vocab = llm.config.spec.vocab_size
    sp = SamplingParams(temperature=0.0, max_tokens=args.warmup + args.steps + 4, ignore_eos=True)
    for p in prompts_for(args.batch, args.prompt_len, vocab):
        llm.add_request(p, sp)
    # prefill
    while llm.scheduler.waiting:
        llm.step()
    runner = llm.model_runner
    dev_ms, wall, launches, clocks = timed_decode(llm, args, n)
    toks = args.batch * args.steps
    value = toks / (dev_ms / 1e3)
    e2e = toks / wall
    if rank == 0:
        B = args.batch
        plan_bytes = runner.last_h2d_bytes
        line = {
            "metric": f"decode tok/s (bs{B}) {args.model} TP{n}",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": round(value / PUBLISHED_BS8, 3) if B == 8 else None,
            "dtype": "bf16", "data": "synthetic token ids (seed 3), random-init N(0,0.02) weights",
            "config": {"model": args.model, "global_batch": B, "seq_len": args.prompt_len,
                       "parallelism": f"tp{n}", "l2": "weights (16 GB) larger than L2; no flush",
                       "decode": "CUDA-graph step, greedy, paged HND KV (page 256)", "comm": args.comm if n > 1 else None},
            "clocks": clocks.summary(),
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": plan_bytes,
                    "d2h_bytes_per_step": 4 * B, "api": "LLM.add_request + LLM.step"},
            "gpu_launches": launches * args.steps,
            "gpu_launches_per_step": launches,
            "impl": "ours",
        }
    llm.exit()
    if rank == 0 and n == 1 and not (args.no_extras or args.model_given or args.batch_given):
        del llm, runner
        line["other_configs"] = measure_extras(args)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()


# Secondary points of the baseline configurations, measured on one GPU after
# the headline (same timing rules: warm-up steps, CUDA events around each
# graph-replayed step, host wall time through LLM.step for e2e).
EXTRA_POINTS = [  # label, model, batch, prompt tokens, Qwen3 k_norm init bound
    ("qwen3-0.6b bs1 (k_norm |w|<=100)", "qwen3-0.6b", 1, 512, 100.0),
    ("qwen3-0.6b bs8 (k_norm |w|<=100)", "qwen3-0.6b", 8, 512, 100.0),
    ("tinyllama-1.1b bs8", "tinyllama-1.1b", 8, 2048, None),
    ("llama3-8b bs1", "llama3-8b", 1, 2048, None),
    ("llama3-8b bs32", "llama3-8b", 32, 2048, None),
]


def _free_gpu() -> None:
    import gc

    import torch

    gc.collect()
    torch.cuda.empty_cache()


def measure_decode_point(model: str, batch: int, plen: int, steps: int, warmup: int, k_norm=None) -> dict:
    import types

    from braidinfer_b200 import LLM, SamplingParams

    cfg_dir = make_config_dir(model, with_weights=False)
    max_len = plen + warmup + steps + 64
    page = 256
    kw = dict(init_k_norm_range=k_norm) if k_norm is not None else {}
    llm = LLM(cfg_dir, load_weights=False, max_num_seqs=batch, max_model_len=max_len,
              num_kvcache_blocks=batch * (-(-max_len // page)) + 8, kvcache_block_size=page,
              max_graph_batch=batch, max_num_batched_tokens=max(16384, max_len), **kw)
    sp = SamplingParams(temperature=0.0, max_tokens=warmup + steps + 4, ignore_eos=True)
    for p in prompts_for(batch, plen, llm.config.spec.vocab_size):
        llm.add_request(p, sp)
    while llm.scheduler.waiting:
        llm.step()
    a = types.SimpleNamespace(warmup=warmup, steps=steps, batch=batch)
    dev_ms, wall, launches, clocks = timed_decode(llm, a, 1)
    llm.exit()
    toks = batch * steps
    return {"value": round(toks / (dev_ms / 1e3), 2), "unit": "tokens/s", "ms_per_step": round(dev_ms / steps, 4),
            "e2e": round(toks / wall, 2), "steps": steps, "warmup": warmup, "prompt_len": plen,
            "gpu_launches_per_step": launches, "clocks": clocks.summary()}


def measure_extras(args) -> dict:
    out = {}
    for label, model, batch, plen, k_norm in EXTRA_POINTS:
        _free_gpu()
        try:
            out[label] = measure_decode_point(model, batch, plen, 64, 8, k_norm)
        except Exception as e:  # noqa: BLE001 - a secondary point never breaks the headline line
            out[label] = {"error": f"{type(e).__name__}: {e}"[:300]}
    _free_gpu()
    try:
        import types

        out["tinyllama-1.1b TTFT, cached chunks"] = measure_ttft(types.SimpleNamespace(model_given=False, steps=24))
    except Exception as e:  # noqa: BLE001
        out["tinyllama-1.1b TTFT, cached chunks"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return out


# ------------------------------------------------------------------ cascade
def run_cascade(args) -> None:
    """Shared-context cascade (Llama-3-70B TP8 configuration): one 8192-token
    context chunk (plus a 32-token system chunk) prefilled once and cascaded
    under ``batch`` concurrent 256-token queries; reports the decode tok/s of
    the whole batch and the prefill time of all queries over the cached chunk."""
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from braidinfer_b200 import ChunkedLLM, ChunkType, SamplingParams

    n = args.gpus
    rank = init_dist(n)
    # the configuration names Llama-3-70B at TP8; --model picks another architecture
    model = args.model if args.model_given else "llama3-70b"
    cfg_dir = make_config_dir(model, with_weights=False, rank=rank)
    if n > 1:
        dist.barrier()
    B, ctx_len, q_len = args.batch, args.ctx_len, args.query_len
    page = 256
    per_seq = q_len + args.warmup + args.steps + 64
    pages = -(-(32 + ctx_len) // page) + B * -(-per_seq // page) + 16
    cl = ChunkedLLM(cfg_dir, load_weights=False, tensor_parallel_size=n, max_num_seqs=B,
                    max_model_len=32 + ctx_len + per_seq, num_kvcache_blocks=pages, kvcache_block_size=page,
                    max_graph_batch=max(B, 1), comm_backend=args.comm,
                    max_num_batched_tokens=max(16384, ctx_len + 64, B * q_len))
    llm = cl.llm
    vocab = llm.config.spec.vocab_size
    g = torch.Generator().manual_seed(4)
    rnd = lambda k: torch.randint(3, vocab, (k,), generator=g).tolist()  # noqa: E731
    sysc = cl.registry.get(cl.register_chunk("system", ChunkType.SYSTEM_PROMPT, token_ids=rnd(32)))
    ctx = cl.registry.get(cl.register_chunk("shared context", ChunkType.CONTEXT, token_ids=rnd(ctx_len)))
    qs = [cl.registry.get(cl.register_chunk(f"query {i}", ChunkType.QUERY, token_ids=rnd(q_len))) for i in range(B)]
    sp = SamplingParams(temperature=0.0, max_tokens=args.warmup + args.steps + 4, ignore_eos=True)
    # the shared chunks are prefilled once (first placement), then every query composes over them
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    cl._ensure_kv(cl._place(sysc, [ctx], qs[0]))
    torch.cuda.synchronize()
    chunk_ms = (time.perf_counter() - t0) * 1e3
    for q in qs:
        cl._ensure_kv(cl._place(sysc, [ctx], q))
        llm.add_composition({"system_chunk": sysc, "context_chunks": [ctx], "query_chunk": q}, sp)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while llm.scheduler.waiting:
        llm.step()
    torch.cuda.synchronize()
    first_ms = (time.perf_counter() - t0) * 1e3
    dev_ms, wall, launches, clocks = timed_decode(llm, args, n)
    toks = B * args.steps
    if rank == 0:
        print(json.dumps({
            "metric": f"cascade decode tok/s (bs{B}) {model} TP{n}", "value": round(toks / (dev_ms / 1e3), 2),
            "unit": "tokens/s", "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic token ids (seed 4), random-init weights",
            "config": {"model": model, "global_batch": B, "shared_context": ctx_len, "query_len": q_len,
                       "parallelism": f"tp{n}", "comm": args.comm if n > 1 else None},
            "shared_chunk_prefill_ms": round(chunk_ms, 2),
            "ttft_all_queries_ms": round(first_ms, 2),
            "clocks": clocks.summary(),
            "e2e": {"value": round(toks / wall, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": llm.model_runner.last_h2d_bytes, "d2h_bytes_per_step": 4 * B,
                    "api": "ChunkedLLM chunks + LLM.add_composition + LLM.step"},
            "gpu_launches": launches * args.steps, "gpu_launches_per_step": launches, "impl": "ours"}), flush=True)
    llm.exit()
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------- reference
def run_reference(args) -> None:
    """The unmodified reference through its public API (``baseline/ref_tp/harness.py``):
    one GPU, or its NCCL all-reduce tensor-parallel build under torchrun.
    Nothing from ``braidinfer_b200`` is imported on this path."""
    n = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    if not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "braidinfer")):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}), flush=True)
        return
    sys.path.insert(0, os.path.join(ROOT, "baseline", "ref_tp"))
    import harness

    if args.model not in harness.ARCH:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"no reference harness for {args.model}"}),
                  flush=True)
        return
    if n == 1:
        harness.run_tp1(args, ClockSampler, PUBLISHED_BS8)
    else:
        harness.run_tp(args, ClockSampler, PUBLISHED_BS8)


# ------------------------------------------------------------------ TTFT
def run_ttft(args) -> None:
    print(json.dumps(measure_ttft(args)), flush=True)


def measure_ttft(args) -> dict:
    """TTFT of a RAG-style composition: a 128-token system chunk plus 3 of 16
    registered 1024-token contexts plus a 64-token query (the cascade/RAG configuration,
    TinyLlama-1.1B architecture), with the chunks' KV cached, against a full
    prefill of the same 3264 tokens.  Device time (CUDA events) through the
    public API, max of ranks not needed (one GPU)."""
    import random

    import torch

    sys.path.insert(0, ROOT)
    from braidinfer_b200 import LLM, ChunkedLLM, ChunkType, SamplingParams

    model = args.model if args.model_given else "tinyllama-1.1b"
    d = make_config_dir(model, with_weights=False)
    cl = ChunkedLLM(d, load_weights=False, num_kvcache_blocks=400, kvcache_block_size=256, max_model_len=8192,
                    max_num_batched_tokens=32768, max_graph_batch=8)
    vocab = cl.llm.config.spec.vocab_size
    g = torch.Generator().manual_seed(2)
    rnd = lambda n: torch.randint(3, vocab, (n,), generator=g).tolist()
    sys_id = cl.register_chunk("system", ChunkType.SYSTEM_PROMPT, token_ids=rnd(128))
    ctx = [cl.register_chunk(f"ctx{i}", ChunkType.CONTEXT, token_ids=rnd(1024)) for i in range(16)]
    rng = random.Random(2)
    sp = dict(temperature=0.0, max_tokens=1, ignore_eos=True)

    def timed(fn):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    # warm: prefill every context chunk once (cached afterwards)
    for i in range(0, 16, 3):
        q = cl.register_chunk(f"warm{i}", ChunkType.QUERY, token_ids=rnd(64))
        cl.generate_from_chunks(sys_id, q, ctx[i:i + 3], sp)
    cached, full = [], []
    for r in range(max(3, args.steps // 8)):
        picks = rng.sample(ctx, 3)
        qt = rnd(64)
        q = cl.register_chunk(f"q{r}", ChunkType.QUERY, token_ids=qt)
        cached.append(timed(lambda: cl.generate_from_chunks(sys_id, q, picks, sp)))
        prompt = cl.registry.peek(sys_id).token_ids + sum((cl.registry.peek(c).token_ids for c in picks), []) + qt
        full.append(timed(lambda: cl.llm.generate(prompt, SamplingParams(**sp))))
    cached, full = sorted(cached)[1:-1] or cached, sorted(full)[1:-1] or full
    c_ms, f_ms = sum(cached) / len(cached), sum(full) / len(full)
    # device share of the cached-chunk TTFT: the captured query-prefill graph
    # replayed alone (its last plan; the rest of TTFT is host-side engine work)
    dev_ms = None
    graphs = cl.llm.model_runner.prefill_graphs
    if graphs:
        g = graphs[min(graphs)]
        dev_ms = min(timed(g.graph.replay) for _ in range(10))
    cl.llm.exit()
    return ({"metric": f"TTFT ms with cached chunks ({model}, 128+3x1024 cached + 64 query)",
                      "value": round(c_ms, 3), "unit": "ms", "higher_is_better": False, "n_gpus": 1,
                      "device_prefill_graph_ms": round(dev_ms, 3) if dev_ms is not None else None,
                      "full_prefill_ms": round(f_ms, 3), "speedup_vs_full_prefill": round(f_ms / c_ms, 2),
                      "dtype": "bf16", "data": "synthetic token ids (seed 2), random-init weights",
                      "impl": "ours"})


def main():
    args = parse()
    if args.impl == "ours" and args.workload == "ttft":
        run_ttft(args)
        return
    if args.impl == "ours" and args.workload == "cascade":
        run_cascade(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
