"""Tensor parallelism on 2, 4 and 8 GPUs (child processes, one per GPU, NCCL
with NVLS off; our kernels use plain peer stores, never multimem).  Each test
runs at every world size the box has GPUs for.

* the fused peer-memory all-reduce equals NCCL's;
* the sequence-parallel prefill path (GEMM -> reduce-scatter epilogue, owner
  reduce + all-gather of rows and 1/rms, all-gather -> fused-norm GEMM) equals
  NCCL all-reduce + the single-GPU kernels;
* the vocab-parallel sampler (per-shard records over peer memory) picks the
  token the single-GPU sampler picks from the full logits: greedy, plain
  temperature, top-k with top-p / min-p;
* a TP-N engine (fused and NCCL backends) matches TP1 tokens and logits, on
  a layout whose KV heads are replicated across ranks (8 query / 2 KV heads)
  and one with one KV head per rank at TP8 (16 query / 8 KV heads);
* a peer that never signals makes the bounded wait expire: every rank gets
  CommTimeoutError and the CUDA context stays usable.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

WORLDS = [2, 4, 8]


def _visible() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


worlds = pytest.mark.parametrize("world", [pytest.param(w, marks=pytest.mark.skipif(
    _visible() < w, reason=f"needs {w} GPUs")) for w in WORLDS])


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _env(rank, world, port):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")


def _w_allreduce(rank, world, port, q):
    _env(rank, world, port)
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from braidinfer_b200.parallel.state import init_tp
        from braidinfer_b200.parallel.symm import FusedComm
        tp = init_tp(world)
        fc = FusedComm(tp, 1024, torch.device("cuda", rank), max_tokens=64, timeout_s=5.0)
        errs = []
        for it in range(6):
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            x = torch.randn(7 + it, 1024, device="cuda", generator=g).bfloat16()
            res = torch.randn(7 + it, 1024, device="cuda", generator=torch.Generator(device="cuda").manual_seed(it)).bfloat16()
            ref = x.float().clone()
            dist.all_reduce(ref)
            ref = (res.float() + ref.bfloat16().float())
            out = fc.all_reduce_add(x, res.clone())
            torch.cuda.synchronize()
            fc.check()
            errs.append((out.float() - ref).abs().max().item())
        # GEMM with the all-reduce inside the kernel (fused_reduce) and, in
        # between, the two-kernel form (push epilogue + reduce kernel)
        w = (torch.randn(1024, 512, device="cuda", generator=torch.Generator(device="cuda").manual_seed(rank)) * 0.05).bfloat16()
        for it, (T, fused) in enumerate([(5, True), (1, True), (16, False), (8, True), (13, True), (3, False),
                                         (16, True), (40, True), (64, False), (64, True), (37, False)]):
            xw = torch.randn(T, 512, device="cuda", generator=torch.Generator(device="cuda").manual_seed(50 + it + 7 * rank)).bfloat16()
            part = (xw.float() @ w.float().t()).bfloat16()
            ref = part.float().clone()
            dist.all_reduce(ref)
            res0 = torch.randn(T, 1024, device="cuda", generator=torch.Generator(device="cuda").manual_seed(90 + it)).bfloat16()
            ref = res0.float() + ref.bfloat16().float()
            fc.fused_reduce = fused
            out = fc.linear_all_reduce_add(xw, w, res0.clone())
            torch.cuda.synchronize()
            fc.check()
            errs.append((out.float() - ref).abs().max().item())
        q.put((rank, errs))
        fc.close()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _w_seqpar(rank, world, port, q):
    _env(rank, world, port)
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from braidinfer_b200 import ops
        from braidinfer_b200.parallel.state import init_tp
        from braidinfer_b200.parallel.symm import FusedComm
        tp = init_tp(world)
        H, eps = 2048, 1e-5
        fc = FusedComm(tp, H, torch.device("cuda", rank), max_tokens=16, timeout_s=5.0, sp_max_tokens=1280)
        errs = []
        # T=300: partial tiles span two owners, small-grid GEMMs; T=1200: persistent GEMMs
        for it, (T, K) in enumerate([(300, 512), (1200, 1024), (300, 512), (97, 256)]):
            gs = torch.Generator(device="cuda").manual_seed(1000 + it)  # same on every rank
            gr = torch.Generator(device="cuda").manual_seed(2000 + 10 * it + rank)  # rank-local
            res = torch.randn(T, H, device="cuda", generator=gs).bfloat16()
            x = torch.randn(T, K, device="cuda", generator=gr).bfloat16()
            w = (torch.randn(H, K, device="cuda", generator=gr) * 0.05).bfloat16()
            part = (x.float() @ w.float().t()).bfloat16().float()
            dist.all_reduce(part)
            ref = (res.float() + part.bfloat16().float()).bfloat16()
            G, rstd = fc.sp_begin(T)
            G.copy_(res)
            fc.sp_linear_reduce_scatter(x, w, G)
            fc.sp_reduce_allgather(eps)
            # all-gather -> fused-norm GEMM (SwiGLU, N = 8192 columns)
            wgu = (torch.randn(8192, H, device="cuda", generator=gs) * 0.05).bfloat16()
            y = ops.linear_swiglu(G, wgu, rms_eps=eps, rs_vec=rstd, sp=fc.sp_params())
            fc.sp_wait()
            torch.cuda.synchronize()
            fc.check()
            y_ref = ops.linear_swiglu(ref, wgu, rms_eps=eps)
            rs_ref = torch.rsqrt(ref.float().pow(2).mean(-1) + eps)
            # relative errors: G differs from the reference by bf16 rounding of the GEMM partials
            errs.append(max((G.float() - ref.float()).abs().max().item() / ref.float().abs().max().item(),
                            (rstd - rs_ref).abs().max().item() / rs_ref.abs().max().item(),
                            (y.float() - y_ref.float()).abs().max().item() / y_ref.float().abs().max().item()))
        q.put((rank, errs))
        fc.close()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _w_timeout(rank, world, port, q):
    _env(rank, world, port)
    import datetime
    import time
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from braidinfer_b200.errors import CommTimeoutError
        from braidinfer_b200.parallel.state import init_tp
        from braidinfer_b200.parallel.symm import FusedComm
        tp = init_tp(world)
        fc = FusedComm(tp, 256, torch.device("cuda", rank), max_tokens=8, timeout_s=0.5)
        fc.push_fault = rank == 0  # rank 0 never signals its arrival
        x = torch.ones(4, 256, device="cuda", dtype=torch.bfloat16)
        t0 = time.time()
        raised = False
        try:
            fc.all_reduce(x)
            torch.cuda.synchronize()
            fc.check()
        except CommTimeoutError as e:
            raised = e.status.get("peer") == 0
        dt = time.time() - t0
        y = (torch.arange(10, device="cuda") * 2).sum().item()  # context still usable
        q.put((rank, raised, dt, y))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), 0, 0))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _w_engine(rank, world, port, ckpt, backend, q):
    _env(rank, world, port)
    import torch.distributed as dist
    try:
        from braidinfer_b200 import LLM, SamplingParams
        llm = LLM(ckpt, num_kvcache_blocks=32, kvcache_block_size=16, tensor_parallel_size=world,
                  comm_backend=backend, max_graph_batch=4)
        llm.model_runner.capture_logits = []
        out = llm.generate([list(range(3, 60)), list(range(5, 20))],
                           SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
        lg = llm.model_runner.capture_logits[0].numpy()
        q.put((rank, [o["token_ids"] for o in out], lg))
        llm.exit()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _w_sampler(rank, world, port, q):
    _env(rank, world, port)
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from braidinfer_b200 import ops
        from braidinfer_b200.parallel.state import init_tp
        from braidinfer_b200.parallel.symm import FusedComm
        tp = init_tp(world)
        fc = FusedComm(tp, 1024, torch.device("cuda", rank), max_tokens=64, timeout_s=5.0)
        V, B = 5003, 8
        per = -(-V // world)
        dev = torch.device("cuda", rank)
        f = lambda v: torch.tensor(v, device=dev)  # noqa: E731
        temp = f([0.0, 0.8, 1.0, 0.7, 1.2, 0.0, 0.5, 1.0]).float()
        topk = f([0, 0, 10, 32, 5, 0, 1, 0]).int()
        topp = f([1.0, 1.0, 1.0, 0.9, 1.0, 1.0, 1.0, 1.0]).float()
        minp = f([0.0, 0.0, 0.0, 0.0, 0.05, 0.0, 0.0, 0.0]).float()
        mism = []
        for it in range(4):
            full = (torch.randn(B, V, device=dev, generator=torch.Generator(device=dev).manual_seed(it)) * 3).bfloat16()
            seed = f([11 * it + i for i in range(B)]).long()
            step = f([it] * B).long()
            ref = ops.sample(full, temp, topk, topp, minp, seed, step)
            local = torch.zeros(B, per, device=dev, dtype=torch.bfloat16)
            n = max(0, min(per, V - rank * per))
            local[:, :n] = full[:, rank * per:rank * per + n]
            out = torch.empty(B, dtype=torch.int32, device=dev)
            fc.sample(local, rank * per, V, temp, topk, topp, minp, seed, step, out)
            torch.cuda.synchronize()
            fc.check()
            mism += [(it, i, int(a), int(b)) for i, (a, b) in enumerate(zip(out.tolist(), ref.tolist())) if a != b]
        q.put((rank, mism))
        fc.close()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(fn, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=fn, args=(r, world, port) + args + (q,)) for r in range(world)]
    [p.start() for p in ps]
    out = [q.get(timeout=600) for _ in ps]
    [p.join(timeout=120) for p in ps]
    return sorted(out, key=lambda r: r[0])


@worlds
def test_fused_all_reduce_matches_nccl(world):
    for r in _spawn(_w_allreduce, world):
        assert isinstance(r[1], list), r[1]
        assert max(r[1]) < 0.05, r[1]


@worlds
def test_sequence_parallel_prefill_collectives(world):
    for r in _spawn(_w_seqpar, world):
        assert isinstance(r[1], list), r[1]
        assert max(r[1]) < 0.02, r[1]


@worlds
def test_vocab_parallel_sampler_matches_single_gpu(world):
    for r in _spawn(_w_sampler, world):
        assert isinstance(r[1], list), r[1]
        assert r[1] == [], f"rank {r[0]}: (call, row, tp token, single-GPU token) {r[1]}"


@worlds
def test_peer_never_signals_times_out(world):
    res = _spawn(_w_timeout, world)
    for r in res:
        assert r[1] is True or r[1] is False, r[1]
        assert r[1], f"rank {r[0]} did not raise CommTimeoutError"
        assert r[2] < 20
        assert r[3] == 90


LAYOUTS = {
    # 8 query / 2 KV heads: KV heads replicated on tp/2 ranks at TP4 and TP8
    "kv_replicated": dict(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=64),
    # 16 query / 8 KV heads: one KV head per rank at TP8 (the Llama-3-70B TP8 layout)
    "kv_one_per_rank": dict(hidden_size=1024, num_attention_heads=16, num_key_value_heads=8, head_dim=64),
}


@worlds
@pytest.mark.parametrize("layout", list(LAYOUTS))
@pytest.mark.parametrize("backend", ["fused", "nccl"])
def test_tp_engine_matches_tp1(tmp_path, world, layout, backend):
    from braidinfer_b200 import LLM, SamplingParams
    from braidinfer_b200.utils.synthetic import make_checkpoint
    ckpt = make_checkpoint(str(tmp_path / "m"), "tiny-llama", seed=3, dtype=torch.bfloat16, **LAYOUTS[layout])
    llm = LLM(ckpt, num_kvcache_blocks=32, kvcache_block_size=16, max_graph_batch=4)
    llm.model_runner.capture_logits = []
    ref_out = llm.generate([list(range(3, 60)), list(range(5, 20))],
                           SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    ref = llm.model_runner.capture_logits[0].numpy()
    ref_tokens = [o["token_ids"] for o in ref_out]
    llm.exit()
    del llm
    res = _spawn(_w_engine, world, ckpt, backend)
    for r in res:
        assert r[2] is not None, r[1]
        d = abs(r[2] - ref).max()
        assert d < 0.05 * abs(ref).max() + 0.05, d
        # greedy decode (CUDA graphs; the fused backend samples through the
        # record exchange): same first tokens as TP1 (bf16 partial sums may
        # flip a later near-tie)
        assert [t[:2] for t in r[1]] == [t[:2] for t in ref_tokens], (r[1], ref_tokens)
