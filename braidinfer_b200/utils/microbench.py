"""Kernel micro-benchmarks and profiler entry points (device time, CUDA events).

    python -m braidinfer_b200.utils.microbench gemm M N K [--epi 0|1] [--graph] [--rms] [--splits S | --sweep-splits]
    python -m braidinfer_b200.utils.microbench attn-decode B L HQ HKV [--splits S]
    python -m braidinfer_b200.utils.microbench attn-prefill L HQ HKV [--batch B] [--ctx C] [--head-dim D] [--splits S] [--trace]
    python -m braidinfer_b200.utils.microbench decode-step MODEL B PROMPT_LEN
    [torchrun --nproc-per-node N -m] braidinfer_b200.utils.microbench decode-trace MODEL B PROMPT_LEN [--out F]
    torchrun --nproc-per-node N -m braidinfer_b200.utils.microbench tp-gemm [--tokens-decode 8] ...

``decode-step`` runs one eager decode step of a random-init model between
``cudaProfilerStart``/``Stop`` (for ``ncu --profile-from-start off``).  Timings
are taken after warm-up with CUDA events on the launching stream; ``--graph``
replays 20 back-to-back launches from a CUDA graph (the decode setting).
Consecutive launches rotate through enough copies of the weights / KV pool /
activations to exceed twice the 126 MB L2, so every launch reads from HBM.
"""
from __future__ import annotations

import argparse
import math

import torch


L2_BYTES = 126 << 20


def _copies(nbytes: int) -> int:
    """Input copies whose total exceeds twice the L2, so that consecutive
    launches (which rotate through them) read from HBM, not from L2."""
    return max(2, min(64, -(-2 * L2_BYTES // max(1, nbytes)) + 1))


def _graph_time(fn, n: int = 20) -> float:
    """fn(i) launches with input copy i; n launches replayed from one graph."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n * 1e3


def _eager_time(fn, n: int = 10) -> float:
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n * 1e3


def bench_gemm(M: int, N: int, K: int, epi: int = 0, graph: bool = False, splits: int = -1,
               rms: bool = False, bn: int = 0) -> dict:
    from ..ops._ext import ext

    nc = _copies((N + M) * K * 2)  # weight and activation copies rotate: HBM, not L2
    xs = [torch.randn(M, K, device="cuda").bfloat16() for _ in range(nc)]
    w0 = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    ws = [w0] + [w0.clone() for _ in range(nc - 1)]
    out = torch.empty(M, N // 2 if epi else N, device="cuda", dtype=torch.bfloat16)
    ext().gemm_force_splits(splits)
    ext().gemm_force_bn(bn)
    fn = lambda i: ext().gemm(out, xs[i % nc], ws[i % nc], None, None, epi, 1e-5 if rms else -1.0)  # noqa: E731
    us = (_graph_time if graph else _eager_time)(fn)
    ext().gemm_force_splits(-1)
    ext().gemm_force_bn(0)
    return {"kernel": "gemm_tcgen05", "M": M, "N": N, "K": K, "epi": epi, "rms": rms, "splits": splits, "bn": bn,
            "us": round(us, 2), "weight_TBps": round(N * K * 2 / us / 1e6, 3),
            "TFLOPS": round(2 * M * N * K / us / 1e6, 1), "l2": f"{nc} rotating input copies (> L2)"}


def _decode_meta(B: int, L: int, PS: int = 256):
    from ..ops.attention import AttnMeta

    npg = -(-L // PS)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    return AttnMeta(qo_indptr=i32(list(range(B + 1))), positions=i32([L - 1] * B),
                    seg_indptr=i32(list(range(B + 1))), seg_page_indptr=i32([i * npg for i in range(B + 1)]),
                    seg_offset=i32([0] * B), seg_len=i32([L] * B), seg_pos0=i32([0] * B), seg_delta=i32([0] * B),
                    page_ids=i32(list(range(B * npg))), num_seqs=B, max_q_len=1, max_kv_len=L, decode=True), npg


def bench_attn_decode(B: int, L: int, Hq: int, Hkv: int, splits: int = 0, D: int = 128) -> dict:
    from .. import ops

    meta, npg = _decode_meta(B, L)
    byts = B * L * Hkv * D * 2 * 2
    nc = _copies(byts)
    kvs = [torch.randn(B * npg + 1, 2, Hkv, 256, D, device="cuda").bfloat16() for _ in range(nc)]
    q = torch.randn(B, Hq, D, device="cuda").bfloat16()
    cos, sin = ops.build_cos_sin(D, 500000.0, 2 * L + 16, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    meta.num_splits = splits or max(1, min(16, (2 * sms) // (B * Hkv), -(-L // 64)))
    us = _graph_time(lambda i: ops.attention(q, kvs[i % nc], meta, cos, sin, D ** -0.5))
    return {"kernel": "attn_decode", "B": B, "L": L, "Hq": Hq, "Hkv": Hkv, "splits": meta.num_splits,
            "us": round(us, 2), "kv_TBps": round(byts / us / 1e6, 3), "l2": f"{nc} rotating KV pools (> L2)"}


def bench_attn_prefill(L: int, Hq: int, Hkv: int, B: int = 1, D: int = 128, ctx: int = 0,
                       splits: int = 0, graph: bool = False, trace: bool = False) -> dict:
    """Causal prefill of L query tokens per sequence; with ``ctx`` the queries
    follow a cached segment of ctx keys (a query over cached chunks)."""
    from .. import ops
    from ..ops.attention import AttnMeta

    PS = 256
    npg, ncg = -(-L // PS), -(-ctx // PS)
    per = npg + ncg
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    segs = 2 if ctx else 1
    spi, soff, slen, spos0 = [0], [], [], []
    for b in range(B):
        if ctx:
            spi.append(spi[-1] + ncg), soff.append(0), slen.append(ctx), spos0.append(0)
        spi.append(spi[-1] + npg), soff.append(0), slen.append(L), spos0.append(ctx)
    meta = AttnMeta(qo_indptr=i32([i * L for i in range(B + 1)]), positions=i32(list(range(ctx, ctx + L)) * B),
                    seg_indptr=i32([i * segs for i in range(B + 1)]), seg_page_indptr=i32(spi),
                    seg_offset=i32(soff), seg_len=i32(slen), seg_pos0=i32(spos0), seg_delta=i32([0] * len(slen)),
                    page_ids=i32(list(range(B * per))), num_seqs=B, max_q_len=L, max_kv_len=L + ctx, decode=False,
                    num_splits=splits or 1)
    kv_bytes = (B * per + 1) * 2 * Hkv * PS * D * 2
    nc = _copies(kv_bytes + B * L * Hq * D * 2)
    kvs = [torch.randn(B * per + 1, 2, Hkv, PS, D, device="cuda").bfloat16() for _ in range(nc)]
    qs = [torch.randn(B * L, Hq, D, device="cuda").bfloat16() for _ in range(nc)]
    cos, sin = ops.build_cos_sin(D, 500000.0, 2 * (L + ctx) + 16, device="cuda")
    us = (_graph_time if graph else _eager_time)(
        lambda i: ops.attention(qs[i % nc], kvs[i % nc], meta, cos, sin, D ** -0.5))
    flops = B * 4 * (L * L / 2 + L * ctx) * Hq * D
    res = {"kernel": "attn_prefill", "L": L, "ctx": ctx, "Hq": Hq, "Hkv": Hkv, "D": D, "B": B, "us": round(us, 1),
           "TFLOPS_causal": round(flops / us / 1e6, 1)}
    if trace:
        res["tc_trace"] = _tc_trace(lambda: ops.attention(qs[0], kvs[0], meta, cos, sin, D ** -0.5),
                                    -(-L * (Hq // Hkv) // 256) * B * Hkv * 32)
    return res


def _tc_trace(run, max_ctas: int) -> dict:
    """One launch of the tcgen05 prefill kernel with its per-tile timestamps:
    softmax time per key tile (S ready -> P handed over), MMA turnaround (P
    handed over -> next S ready), first S after the CTA start, CTA length."""
    import numpy as np

    from ..ops._ext import ext

    buf = torch.zeros(max_ctas * 128, dtype=torch.int64, device="cuda")
    ext().attn_tc_set_trace(buf)
    try:
        run()
        torch.cuda.synchronize()
    finally:
        ext().attn_tc_set_trace(torch.empty(0, dtype=torch.int64, device="cuda"))
    t = buf.view(-1, 2, 64).cpu().numpy().astype(np.float64)
    t = t[t[:, 0, 62] > 0]
    soft, turn, first, cta, setup, kfirst, qbuilt, s0 = [], [], [], [], [], [], [], []
    for c in t:
        t0 = c[0, 62]
        cta.append((c[0, 63] - t0) / 1e3)
        setup.append((c[1, 62] - t0) / 1e3)
        if c[1, 63] > 0:
            kfirst.append((c[1, 63] - t0) / 1e3)
        if c[0, 61] > 0:
            s0.append((c[0, 61] - t0) / 1e3)
        for q in range(2):
            if c[q, 60] > 0:
                qbuilt.append((c[q, 60] - t0) / 1e3)
            s, pp = c[q, 0:60:2], c[q, 1:60:2]
            n = int(np.count_nonzero(s))
            if n == 0:
                continue
            first.append((s[0] - c[0, 62]) / 1e3)
            soft += list((pp[:n] - s[:n]) / 1e3)
            turn += list((s[1:n] - pp[:n - 1]) / 1e3)
    q = lambda v: {"median": round(float(np.median(v)), 3), "mean": round(float(np.mean(v)), 3)} if v else None  # noqa: E731
    return {"ctas": int(len(t)), "softmax_us": q(soft), "turnaround_us": q(turn), "first_s_us": q(first),
            "cta_us": q(cta), "setup_us": q(setup), "first_k_issued_us": q(kfirst), "q_built_us": q(qbuilt),
            "s0_issued_us": q(s0)}


def decode_step(model: str, B: int, plen: int) -> None:
    import os
    import tempfile

    from .. import LLM, SamplingParams
    from .synthetic import make_checkpoint

    d = os.path.join(tempfile.gettempdir(), f"braid_mb_{model}")
    if not os.path.exists(os.path.join(d, "config.json")):
        make_checkpoint(d, model, write_weights=False)
    page = 256
    llm = LLM(d, load_weights=False, max_num_seqs=B, max_model_len=plen + 64,
              num_kvcache_blocks=B * math.ceil((plen + 64) / page) + 8, enforce_eager=True,
              max_num_batched_tokens=max(16384, plen + 64))
    g = torch.Generator().manual_seed(3)
    for _ in range(B):
        llm.add_request(torch.randint(3, llm.config.spec.vocab_size, (plen,), generator=g).tolist(),
                        SamplingParams(temperature=0, max_tokens=16, ignore_eos=True))
    while llm.scheduler.waiting:
        llm.step()
    for _ in range(3):
        llm.step()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    llm.step()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()


def bench_sample(B: int, V: int, greedy: bool = True) -> dict:
    """Device sampler over [B, V] bf16 logits (greedy, or temperature 0.8 with
    top-k 50 / top-p 0.9); logits copies rotate so each launch reads HBM."""
    from .. import ops

    nc = _copies(B * V * 2)
    xs = [torch.randn(B, V, device="cuda").bfloat16() for _ in range(nc)]
    t = torch.full((B,), 0.0 if greedy else 0.8, device="cuda")
    k = torch.full((B,), 0 if greedy else 50, device="cuda", dtype=torch.int32)
    p = torch.full((B,), 1.0 if greedy else 0.9, device="cuda")
    m = torch.zeros(B, device="cuda")
    seed = torch.arange(B, device="cuda", dtype=torch.int64)
    step = torch.zeros(B, device="cuda", dtype=torch.int64)
    out = torch.empty(B, dtype=torch.int32, device="cuda")
    us = _graph_time(lambda i: ops.sample(xs[i % nc], t, k, p, m, seed, step, out=out))
    return {"kernel": "sample_kernel", "B": B, "V": V, "greedy": greedy, "us": round(us, 2),
            "logits_TBps": round(B * V * 2 / us / 1e6, 3)}


def gemm_trace(M: int, N: int, K: int, kind: str = "plain", rms: bool = True, splits: int = -1,
               bn: int = 0) -> dict:
    """Per-CTA phases of one decode-shaped GEMM launch that follows another
    GEMM in a CUDA graph (so its prologue overlaps a predecessor, as in a
    decode step).  ``kind``: plain (epi 0), swiglu (epi 1) or qkv (epi 2 with
    q/k-norm, RoPE and the paged KV append; N = (Hq + 2 Hkv) * 128).

    Per CTA (``gemm_set_trace``): t0 start, t1 MMA issuer ready, t2 first
    K-block landed, t3 accumulator complete, t4 epilogue done.  Reports the
    launch span, the medians/maxima of first-data latency, mainloop and
    epilogue, and the tail = last epilogue end - last accumulator complete
    (split-K reduction and epilogue of the tiles' last CTAs)."""
    import numpy as np

    from .. import ops
    from ..ops._ext import ext

    C = ext()
    nc = _copies(N * K * 2)
    ws = [(torch.randn(N, K, device="cuda") * 0.02).bfloat16() for _ in range(nc)]
    x = torch.randn(M, K, device="cuda").bfloat16()
    pre_w = (torch.randn(8192, K, device="cuda") * 0.02).bfloat16()
    pre_out = torch.empty(M, 8192, device="cuda", dtype=torch.bfloat16)
    eps = 1e-5 if rms else -1.0
    if kind == "qkv":
        D, Hkv = 128, 8
        Hq = N // D - 2 * Hkv
        PS = 256
        kv = torch.zeros(M + 1, 2, Hkv, PS, D, device="cuda", dtype=torch.bfloat16)
        pos = torch.arange(M, device="cuda", dtype=torch.int32) + 100
        slots = torch.arange(M, device="cuda", dtype=torch.int32) * PS
        cos, sin = ops.build_cos_sin(D, 500000.0, 4096, None, torch.device("cuda"))
        q = torch.empty(M, Hq, D, device="cuda", dtype=torch.bfloat16)
        out = None
    else:
        out = torch.empty(M, N // 2 if kind == "swiglu" else N, device="cuda", dtype=torch.bfloat16)

    def launch(i, traced):
        C.gemm(pre_out, x, pre_w, None, None, 0, -1.0)
        if traced:
            C.gemm_set_trace(buf)
        w = ws[i % nc]
        if kind == "qkv":
            C.gemm_qkv(q, x, w, None, eps, pos, slots, kv, None, None, 1e-6, cos, sin, Hq, Hkv, D, True)
        else:
            C.gemm(out, x, w, None, None, 1 if kind == "swiglu" else 0, eps)
        if traced:
            C.gemm_set_trace(torch.empty(0, dtype=torch.int64))

    C.gemm_force_splits(splits)
    C.gemm_force_bn(bn)
    buf = torch.zeros(8 * 4096, dtype=torch.int64, device="cuda")
    for i in range(3):
        launch(i, False)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        launch(0, False)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        for i in range(4):
            launch(i, i == 3)
    rows = []
    for _ in range(5):
        buf.zero_()
        g.replay()
        torch.cuda.synchronize()
        t = buf.view(-1, 8)[:, :5].cpu().numpy().astype("int64")
        t = t[t[:, 0] > 0]
        rows.append(t)
    C.gemm_force_splits(-1)
    C.gemm_force_bn(0)
    t = rows[len(rows) // 2]
    t0 = t[:, 0].min()
    first = (t[:, 2] - t[:, 0]) / 1e3
    main = (t[:, 3] - t[:, 2]) / 1e3
    epi = (t[:, 4] - t[:, 3]) / 1e3
    med = lambda a: round(float(np.median(a)), 2)  # noqa: E731
    return {"kind": kind, "M": M, "N": N, "K": K, "ctas": int(len(t)),
            "span_us": round((t[:, 4].max() - t0) / 1e3, 2),
            "last_start_us": round((t[:, 0].max() - t0) / 1e3, 2),
            "first_data_us": {"median": med(first), "max": round(float(first.max()), 2)},
            "mainloop_us": {"median": med(main), "max": round(float(main.max()), 2)},
            "epilogue_us": {"median": med(epi), "max": round(float(epi.max()), 2)},
            "last_acc_us": round((t[:, 3].max() - t0) / 1e3, 2),
            "tail_us": round((t[:, 4].max() - t[:, 3].max()) / 1e3, 2),
            "weight_MB": round(N * K * 2 / 1e6, 1)}


def decode_trace(model: str, B: int, plen: int, replays: int = 5, out_path: str = "", ctx: int = 0) -> dict:
    """Per-launch timeline of one graph-replayed decode step (one GPU, or every
    rank under torchrun with ``tensor_parallel_size`` = world size).

    Every native launch of the captured step records, on the device, its first
    CTA start, the first moment a CTA passed its dependency wait (for the
    collectives: the bounded wait for the peers) and its last CTA end
    (``span_trace``).  Per launch name it reports, per step, the summed
    ``busy`` time (dependency release to last CTA end: the launch's share of
    the critical path), ``lead`` (start to release: prologue overlapped with
    the predecessor, or, for a collective, the wait for the slowest peer) and
    ``release`` gaps (previous launch's end to this launch's release).  Under
    TP each rank reports; rank 0 prints all and the step time of each.
    ``ctx > 0``: every request composes a 32-token system chunk and one shared
    ``ctx``-token context chunk (cached once) before its ``plen``-token query.
    """
    import datetime
    import json
    import os
    import tempfile

    import torch.distributed as dist

    from .. import LLM, SamplingParams
    from ..ops._ext import ext
    from .synthetic import make_checkpoint

    n = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if n > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    rank = dist.get_rank() if n > 1 else 0
    d = os.path.join(tempfile.gettempdir(), f"braid_mb_{model}")
    if rank == 0 and not os.path.exists(os.path.join(d, "config.json")):
        make_checkpoint(d, model, write_weights=False)
    if n > 1:
        dist.barrier()
    page = 256
    per_seq = plen + 64 + replays + 16
    max_len = per_seq + (32 + ctx if ctx else 0)
    pages = B * math.ceil(per_seq / page) + 8 + (math.ceil((32 + ctx) / page) if ctx else 0)
    kw = dict(load_weights=False, tensor_parallel_size=n, max_num_seqs=B, max_model_len=max_len,
              num_kvcache_blocks=pages, kvcache_block_size=page, max_graph_batch=B,
              max_num_batched_tokens=max(16384, max_len, B * plen + 64))
    g = torch.Generator().manual_seed(3)
    sp = SamplingParams(temperature=0, max_tokens=replays + 16, ignore_eos=True)
    if ctx:
        from .. import ChunkedLLM, ChunkType

        cl = ChunkedLLM(d, **kw)
        llm = cl.llm
        V = llm.config.spec.vocab_size
        rnd = lambda k: torch.randint(3, V, (k,), generator=g).tolist()  # noqa: E731
        sysc = cl.registry.get(cl.register_chunk("system", ChunkType.SYSTEM_PROMPT, token_ids=rnd(32)))
        shared = cl.registry.get(cl.register_chunk("shared", ChunkType.CONTEXT, token_ids=rnd(ctx)))
        for i in range(B):
            q = cl.registry.get(cl.register_chunk(f"q{i}", ChunkType.QUERY, token_ids=rnd(plen)))
            cl._ensure_kv(cl._place(sysc, [shared], q))
            llm.add_composition({"system_chunk": sysc, "context_chunks": [shared], "query_chunk": q}, sp)
    else:
        llm = LLM(d, **kw)
        for _ in range(B):
            llm.add_request(torch.randint(3, llm.config.spec.vocab_size, (plen,), generator=g).tolist(), sp)
    while llm.scheduler.waiting:
        llm.step()
    for _ in range(3):
        llm.step()
    runner = llm.model_runner
    C = ext()
    buf = torch.zeros(4 * 4096, dtype=torch.int64, device="cuda")
    # force a re-capture of this bucket (whichever graph table the step uses)
    runner.graphs.pop(B, None)
    runner.graphs_gather.pop(B, None)
    for k in [k for k in runner.graphs_shared if k[0] == B]:
        runner.graphs_shared.pop(k)
    C.span_trace(buf)
    llm.step()  # re-captures the bucket with span slots baked into the launches
    names = C.span_names()
    C.span_trace(torch.empty(0, dtype=torch.int64))
    # the capture runs the step twice eagerly before recording it: three equal
    # runs of traced launches, the graph's are the last third
    if len(names) % 3 or not names:
        raise RuntimeError(f"{len(names)} traced launches is not three equal runs")
    L = len(names) // 3
    base = 2 * L
    names = names[base:]
    MAXU = -1  # all bits set: the initial value for the atomicMin fields
    steps = []
    for _ in range(replays):
        v = buf.view(-1, 4)
        v[base:base + L, 0] = MAXU
        v[base:base + L, 1] = MAXU
        v[base:base + L, 2] = 0
        torch.cuda.synchronize()
        if n > 1:
            dist.barrier()
        llm.step()
        torch.cuda.synchronize()
        a = v[base:base + L, :3].cpu().numpy().astype("uint64")
        steps.append(a)
    per = {}
    step_us = []
    for a in steps:
        t0 = int(a[:, 0].min())
        start = (a[:, 0] - t0).astype("float64") / 1e3
        waited = a[:, 1].copy()
        waited[waited == (2 ** 64 - 1)] = a[waited == (2 ** 64 - 1), 0]
        waited = (waited - t0).astype("float64") / 1e3
        end = (a[:, 2] - t0).astype("float64") / 1e3
        step_us.append(float(end.max()))
        for i, nm in enumerate(names):
            r = per.setdefault(nm, {"count": 0, "busy_us": 0.0, "lead_us": 0.0, "release_us": 0.0})
            r["count"] += 1
            r["busy_us"] += max(0.0, end[i] - waited[i])
            r["lead_us"] += max(0.0, waited[i] - start[i])
            if i:
                r["release_us"] += max(0.0, waited[i] - end[i - 1])
    R = len(steps)
    for r in per.values():
        r["count"] //= R
        for k in ("busy_us", "lead_us", "release_us"):
            r[k] = round(r[k] / R, 1)
    res = {"rank": rank, "tp": n, "model": model, "batch": B, "prompt_len": plen, "shared_ctx": ctx, "launches": L,
           "step_us": round(sorted(step_us)[len(step_us) // 2], 1), "per_name": per}
    if n > 1:
        allr = [None] * n
        dist.all_gather_object(allr, res)
    else:
        allr = [res]
    out = {"kind": "decode_trace", "ranks": allr,
           "step_us_max_over_ranks": max(r["step_us"] for r in allr)}
    if rank == 0:
        print(json.dumps(out), flush=True)
        if out_path:
            with open(out_path, "w") as f:
                json.dump(out, f, indent=1)
    llm.exit()
    if n > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


def bench_tp_gemm(T_dec: int = 8, T_pre: int = 4096, H: int = 4096, I: int = 14336) -> None:
    """Row-parallel GEMM + its collective over the TP group (run under torchrun,
    one process per GPU).  Llama-3-8B down_proj shape: ``x [T, I/tp] @ w[H, I/tp]^T``.

    * decode (T_dec tokens): our GEMM whose epilogue pushes tiles to every peer
      + bounded-wait reduce kernel, vs ``F.linear``-equivalent GEMM + NCCL
      all_reduce; both replayed from CUDA graphs.
    * prefill (T_pre tokens): our GEMM with the reduce-scatter epilogue + owner
      reduce / all-gather of rows and 1/rms (sequence parallel), vs GEMM + NCCL
      all_reduce; eager.
    Times are device time (CUDA events), max over ranks.  Roofline per GPU = the
    slower of the GEMM at the bf16 peak, its weight bytes at HBM bandwidth and
    the bytes it must send over NVLink at the measured 770 GB/s per direction.
    """
    import datetime
    import json
    import os

    import torch.distributed as dist

    from .. import ops
    from ..ops._ext import ext
    from ..parallel.state import init_tp
    from ..parallel.symm import FusedComm

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    tp = init_tp(dist.get_world_size())
    n, rank = tp.size, tp.rank
    K = I // n
    fc = FusedComm(tp, H, torch.device("cuda", local), max_tokens=64, timeout_s=10.0, sp_max_tokens=T_pre)
    PEAK, HBM, LINK = 1.59e15, 6.65e12, 770e9
    nw = _copies(H * K * 2)
    ws = [(torch.randn(H, K, device="cuda") * 0.02).bfloat16() for _ in range(nw)]

    def maxrank(us: float) -> float:
        t = torch.tensor([us], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    out = {"kernel": "tp_gemm_collective", "tp": n, "H": H, "K_per_rank": K}
    # ---- decode: one-shot push all-reduce (graph) vs NCCL all_reduce (graph)
    x = torch.randn(T_dec, K, device="cuda").bfloat16()
    res = torch.zeros(T_dec, H, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(T_dec, H, device="cuda", dtype=torch.bfloat16)
    ours = maxrank(_graph_time(lambda i: fc.linear_all_reduce_add(x, ws[i % nw], res)))
    fc.check()

    def nccl_dec(i):
        ext().gemm(y, x, ws[i % nw], None, None, 0, -1.0)
        dist.all_reduce(y, group=tp.group)

    base = maxrank(_graph_time(nccl_dec))
    roof = max(2 * T_dec * H * K / PEAK, H * K * 2 / HBM, T_dec * H * 2 * (n - 1) / LINK) * 1e6
    out["decode"] = {"T": T_dec, "ours_us": round(ours, 2), "nccl_us": round(base, 2),
                     "roofline_us": round(roof, 2), "of_roofline": round(roof / ours, 3)}
    # ---- prefill: GEMM -> reduce-scatter epilogue, reduce + all-gather (eager) vs NCCL
    xp = torch.randn(T_pre, K, device="cuda").bfloat16()
    G, rstd = fc.sp_begin(T_pre)
    G.zero_()

    def ours_pre(i):
        fc.sp_linear_reduce_scatter(xp, ws[i % nw], G)
        fc.sp_reduce_allgather(1e-5)

    ours_p = _eager_time(ours_pre)
    fc.sp_wait()
    torch.cuda.synchronize()
    fc.check()
    ours_p = maxrank(ours_p)
    yp = torch.empty(T_pre, H, device="cuda", dtype=torch.bfloat16)

    def nccl_pre(i):
        ext().gemm(yp, xp, ws[i % nw], None, None, 0, -1.0)
        dist.all_reduce(yp, group=tp.group)

    base_p = maxrank(_eager_time(nccl_pre))
    rows = -(-T_pre // n)
    link = (T_pre - rows) * H * 2 + rows * H * 2 * (n - 1)  # reduce-scatter out + all-gather out
    roof_p = max(2 * T_pre * H * K / PEAK, link / LINK) * 1e6
    out["prefill"] = {"T": T_pre, "ours_us": round(ours_p, 1), "nccl_us": round(base_p, 1),
                      "roofline_us": round(roof_p, 1), "of_roofline": round(roof_p / ours_p, 3)}
    if rank == 0:
        print(json.dumps(out), flush=True)
    fc.close()
    dist.barrier()
    dist.destroy_process_group()


def main(argv=None) -> None:
    import json

    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("M", type=int), g.add_argument("N", type=int), g.add_argument("K", type=int)
    g.add_argument("--epi", type=int, default=0)
    g.add_argument("--graph", action="store_true")
    g.add_argument("--splits", type=int, default=-1, help="force the split-K factor (-1: heuristic)")
    g.add_argument("--rms", action="store_true", help="fused input RMSNorm")
    g.add_argument("--sweep-splits", action="store_true", help="time every split-K factor 1..16")
    g.add_argument("--bn", type=int, default=0, help="force the decode token-tile width 16/32/64")
    a = sub.add_parser("attn-decode")
    for n in ("B", "L", "Hq", "Hkv"):
        a.add_argument(n, type=int)
    a.add_argument("--splits", type=int, default=0)
    p = sub.add_parser("attn-prefill")
    for n in ("L", "Hq", "Hkv"):
        p.add_argument(n, type=int)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--ctx", type=int, default=0, help="cached keys before the queries")
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--splits", type=int, default=0, help="force key splits (0: automatic)")
    p.add_argument("--graph", action="store_true", help="time 20 launches replayed from a CUDA graph")
    p.add_argument("--trace", action="store_true", help="tcgen05 kernel: per-tile softmax / MMA turnaround times")
    tg = sub.add_parser("tp-gemm", help="row-parallel GEMM + collective, under torchrun (one rank per GPU)")
    tg.add_argument("--tokens-decode", type=int, default=8)
    tg.add_argument("--tokens-prefill", type=int, default=4096)
    tg.add_argument("--hidden", type=int, default=4096)
    tg.add_argument("--inter", type=int, default=14336)
    s = sub.add_parser("decode-step")
    s.add_argument("model"), s.add_argument("B", type=int), s.add_argument("plen", type=int)
    sm = sub.add_parser("sample", help="device sampler over [B, V] logits")
    sm.add_argument("B", type=int), sm.add_argument("V", type=int)
    sm.add_argument("--sampled", action="store_true", help="temperature 0.8, top-k 50, top-p 0.9 (default greedy)")
    gt = sub.add_parser("gemm-trace", help="per-CTA phases of a decode GEMM after a predecessor GEMM")
    gt.add_argument("M", type=int), gt.add_argument("N", type=int), gt.add_argument("K", type=int)
    gt.add_argument("--kind", default="plain", choices=["plain", "swiglu", "qkv"])
    gt.add_argument("--no-rms", action="store_true")
    gt.add_argument("--splits", type=int, default=-1)
    gt.add_argument("--bn", type=int, default=0)
    t = sub.add_parser("decode-trace", help="per-launch timeline of a graph-replayed decode step (torchrun for TP)")
    t.add_argument("model"), t.add_argument("B", type=int), t.add_argument("plen", type=int)
    t.add_argument("--replays", type=int, default=5)
    t.add_argument("--ctx", type=int, default=0, help="shared context chunk tokens (cascade composition)")
    t.add_argument("--out", default="", help="also write the JSON here")
    args = ap.parse_args(argv)
    if args.cmd == "gemm":
        if args.sweep_splits:
            for sp in (0, 1, 2, 3, 4, 6, 8, 12, 16):
                print(json.dumps(bench_gemm(args.M, args.N, args.K, args.epi, args.graph, sp, args.rms, args.bn)))
        else:
            print(json.dumps(bench_gemm(args.M, args.N, args.K, args.epi, args.graph, args.splits, args.rms,
                                        args.bn)))
    elif args.cmd == "tp-gemm":
        bench_tp_gemm(args.tokens_decode, args.tokens_prefill, args.hidden, args.inter)
    elif args.cmd == "sample":
        print(json.dumps(bench_sample(args.B, args.V, not args.sampled)))
    elif args.cmd == "gemm-trace":
        print(json.dumps(gemm_trace(args.M, args.N, args.K, args.kind, not args.no_rms, args.splits, args.bn)))
    elif args.cmd == "decode-trace":
        decode_trace(args.model, args.B, args.plen, args.replays, args.out, args.ctx)
    elif args.cmd == "attn-decode":
        print(json.dumps(bench_attn_decode(args.B, args.L, args.Hq, args.Hkv, args.splits)))
    elif args.cmd == "attn-prefill":
        print(json.dumps(bench_attn_prefill(args.L, args.Hq, args.Hkv, args.batch, args.head_dim, args.ctx,
                                            args.splits, args.graph, args.trace)))
    else:
        decode_step(args.model, args.B, args.plen)
        print("decode step done")


if __name__ == "__main__":
    main()
