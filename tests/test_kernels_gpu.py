"""Numerics of the native sm_100a kernels against fp32 PyTorch references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ext():
    from braidinfer_b200.ops._ext import ext
    return ext()


def _check_err():
    assert _ext().gemm_check_error(torch.cuda.current_device()) == 0


@pytest.fixture(params=[1, 0], ids=["tc", "mma"])
def prefill_kernel(request):
    """Runs the test on each prefill attention kernel for head_dim 128, forced
    for every prefill call (and the shared-prefix pass): the tcgen05 kernel
    (attention_tc.cu) and the mma.sync kernel (attention.cu)."""
    _ext().attn_select_prefill_tc(request.param)
    yield request.param
    _ext().attn_select_prefill_tc(-1)


@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (7, 4096, 1024), (16, 1536, 2048), (33, 640, 256),
                                   (64, 2048, 4096), (65, 384, 512), (200, 1024, 1024), (1000, 2560, 2048),
                                   (513, 6144, 4096)])
def test_gemm_plain(M, N, K):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    _ext().gemm(out, x, w, None, None, 0, -1.0)
    torch.cuda.synchronize()
    _check_err()
    ref = x.float() @ w.float().t()
    torch.testing.assert_close(out.float(), ref, atol=2e-2 * math.sqrt(K / 256), rtol=2e-2)


@pytest.mark.parametrize("M,N,K", [(3, 512, 1024), (100, 768, 512)])
def test_gemm_bias_residual(M, N, K):
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    b = torch.randn(N, device=DEV).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    _ext().gemm(out, x, w, b, r, 0, -1.0)
    ref = (x.float() @ w.float().t() + b.float()).bfloat16().float() + r.float()
    torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=2e-2)
    # in place residual update (out aliases the residual)
    r2 = r.clone()
    _ext().gemm(r2, x, w, b, r2, 0, -1.0)
    torch.testing.assert_close(r2.float(), ref, atol=5e-2, rtol=2e-2)


@pytest.mark.parametrize("M,I,K", [(1, 384, 1024), (8, 1792, 4096), (48, 704, 2048), (300, 3072, 1024)])
def test_gemm_swiglu(M, I, K):
    from braidinfer_b200.ops.linear import interleave_gate_up, swiglu_ref_from_interleaved
    x = torch.randn(M, K, device=DEV).bfloat16()
    _check_err()
    wg = (torch.randn(I, K, device=DEV) * 0.05).bfloat16()
    wu = (torch.randn(I, K, device=DEV) * 0.05).bfloat16()
    w = interleave_gate_up(wg, wu)
    out = torch.empty(M, w.shape[0] // 2, device=DEV, dtype=torch.bfloat16)
    _ext().gemm(out, x, w, None, None, 1, -1.0)
    ref = swiglu_ref_from_interleaved(x.float() @ w.float().t(), torch.bfloat16)
    torch.testing.assert_close(out.float(), ref.float(), atol=3e-2, rtol=3e-2)
    direct = torch.nn.functional.silu(x.float() @ wg.float().t()) * (x.float() @ wu.float().t())
    torch.testing.assert_close(out.float()[:, :I], direct, atol=5e-2, rtol=5e-2)


@pytest.mark.parametrize("M,N,K", [(5, 1024, 2048), (64, 512, 4096), (300, 768, 1024)])
def test_gemm_fused_rmsnorm(M, N, K):
    """rms(x) @ (W diag(g))^T == (x / rms(x) * g) @ W^T"""
    from braidinfer_b200 import ops
    x = (torch.randn(M, K, device=DEV) * 3).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    g = (torch.rand(K, device=DEV) + 0.5).bfloat16()
    wf = (w.float() * g.float()).bfloat16()
    out = ops.linear(x, wf, rms_eps=1e-5)
    xn = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5) * g.float()
    torch.testing.assert_close(out.float(), xn @ w.float().t(), atol=5e-2, rtol=3e-2)
    sw = ops.linear_swiglu(x, torch.cat([wf[:128], wf[:128]])[:256].contiguous(), rms_eps=1e-5)
    assert sw.shape == (M, 128) and torch.isfinite(sw.float()).all()


@pytest.mark.parametrize("T,D,Hq,Hkv,qk_norm,bias", [(3, 128, 16, 8, True, False), (40, 64, 32, 4, False, True),
                                                      (200, 128, 8, 2, True, True), (1, 64, 4, 2, False, False)])
def test_gemm_qkv_epilogue(T, D, Hq, Hkv, qk_norm, bias):
    """Fused QKV GEMM epilogue == linear + qkv_prepare (both native), and the CPU path."""
    from braidinfer_b200 import ops
    H, PS, P = 512, 16, 64
    x = torch.randn(T, H, device=DEV).bfloat16()
    w = (torch.randn((Hq + 2 * Hkv) * D, H, device=DEV) * 0.05).bfloat16()
    b = (torch.randn((Hq + 2 * Hkv) * D, device=DEV) * 0.1).bfloat16() if bias else None
    pos = torch.randint(0, 900, (T,), device=DEV, dtype=torch.int32)
    slots = torch.randperm(P * PS, device=DEV)[:T].int()
    cos, sin = ops.build_cos_sin(D, 10000.0, 1024, device=DEV)
    qn = (torch.rand(D, device=DEV) * 2).bfloat16() if qk_norm else None
    kn = (torch.rand(D, device=DEV) * 80 - 40).bfloat16() if qk_norm else None
    kv1 = torch.zeros(P, 2, Hkv, PS, D, device=DEV, dtype=torch.bfloat16)
    kv2 = kv1.clone()
    q1 = ops.qkv_gemm(x, w, b, 1e-6, pos, slots, kv1, Hq, Hkv, D, cos, sin, qn, kn, 1e-6, True)
    qkv = ops.linear(x, w, b, rms_eps=1e-6)
    q2 = ops.qkv_prepare(qkv, pos, slots, kv2, Hq, Hkv, D, cos, sin, qn, kn, 1e-6, True)
    tol = 0.05 * (40 if qk_norm else 1)
    torch.testing.assert_close(q1.float(), q2.float(), atol=tol, rtol=3e-2)
    torch.testing.assert_close(kv1.float(), kv2.float(), atol=tol, rtol=3e-2)
    _check_err()


@pytest.mark.parametrize("M,N,K,mode", [(1000, 6144, 1024, "bias_res"), (700, 8192, 1024, "swiglu"),
                                        (777, 8192, 2048, "rms"), (1000, 2560, 512, "plain"),
                                        (4100, 4096, 1024, "bias_res")])
def test_gemm_persistent(M, N, K, mode):
    """Shapes with >= one tile per SM run the persistent kernel (double-buffered
    TMEM accumulators); compare with the fp32 reference of the same op."""
    from braidinfer_b200 import ops
    from braidinfer_b200.ops.linear import swiglu_ref_from_interleaved
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = (torch.randn(M, K, device=DEV, generator=g) * (3 if mode == "rms" else 1)).bfloat16()
    w = (torch.randn(N, K, device=DEV, generator=g) * 0.05).bfloat16()
    tol = dict(atol=3e-2 * math.sqrt(K / 256), rtol=3e-2)
    if mode == "swiglu":
        out = ops.linear_swiglu(x, w)
        ref = swiglu_ref_from_interleaved(x.float() @ w.float().t(), torch.bfloat16)
        torch.testing.assert_close(out.float(), ref.float(), **tol)
    elif mode == "rms":
        out = ops.linear(x, w, rms_eps=1e-5)
        ref = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5)) @ w.float().t()
        torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=3e-2)
        # precomputed 1/rms gives the same result
        rs = ops.row_rstd(x, 1e-5)
        out2 = torch.empty_like(out)
        _ext().gemm(out2, x, w, None, None, 0, -1.0, rs, None)
        torch.testing.assert_close(out2.float(), out.float(), atol=1e-2, rtol=1e-2)
    elif mode == "bias_res":
        b = torch.randn(N, device=DEV, generator=g).bfloat16()
        r = torch.randn(M, N, device=DEV, generator=g).bfloat16()
        out = ops.linear(x, w, b, residual=r.clone())
        ref = (x.float() @ w.float().t() + b.float()).bfloat16().float() + r.float()
        torch.testing.assert_close(out.float(), ref, atol=6e-2, rtol=2e-2)
    else:
        out = ops.linear(x, w)
        torch.testing.assert_close(out.float(), x.float() @ w.float().t(), **tol)
    torch.cuda.synchronize()
    _check_err()


def test_gemm_qkv_persistent():
    """Prefill-sized fused QKV (persistent kernel) == linear + qkv_prepare."""
    from braidinfer_b200 import ops
    T, D, Hq, Hkv, H, PS, P = 1000, 128, 32, 8, 512, 16, 80
    x = torch.randn(T, H, device=DEV).bfloat16()
    w = (torch.randn((Hq + 2 * Hkv) * D, H, device=DEV) * 0.05).bfloat16()
    pos = torch.arange(T, device=DEV, dtype=torch.int32)
    slots = torch.randperm(P * PS, device=DEV)[:T].int()
    cos, sin = ops.build_cos_sin(D, 10000.0, 1024, device=DEV)
    qn = (torch.rand(D, device=DEV) * 2).bfloat16()
    kn = (torch.rand(D, device=DEV) * 2).bfloat16()
    kv1 = torch.zeros(P, 2, Hkv, PS, D, device=DEV, dtype=torch.bfloat16)
    kv2 = kv1.clone()
    q1 = ops.qkv_gemm(x, w, None, 1e-6, pos, slots, kv1, Hq, Hkv, D, cos, sin, qn, kn, 1e-6, True)
    qkv = ops.linear(x, w, None, rms_eps=1e-6)
    q2 = ops.qkv_prepare(qkv, pos, slots, kv2, Hq, Hkv, D, cos, sin, qn, kn, 1e-6, True)
    torch.testing.assert_close(q1.float(), q2.float(), atol=0.05, rtol=3e-2)
    torch.testing.assert_close(kv1.float(), kv2.float(), atol=0.05, rtol=3e-2)
    _check_err()


def test_rmsnorm_and_add():
    from braidinfer_b200.ops.norm import rms_norm_ref
    for H in (256, 1024, 4096, 8192):
        x = torch.randn(13, H, device=DEV).bfloat16()
        w = (torch.rand(H, device=DEV) * 2).bfloat16()
        out = torch.empty_like(x)
        _ext().rms_norm(out, x, w, 1e-6)
        torch.testing.assert_close(out.float(), rms_norm_ref(x, w, 1e-6).float(), atol=2e-2, rtol=1e-2)
        res = torch.randn(13, H, device=DEV).bfloat16()
        res0 = res.clone()
        _ext().add_rms_norm(out, res, x, w, 1e-6)
        s = (res0.float() + x.float()).bfloat16()
        torch.testing.assert_close(res.float(), s.float())
        torch.testing.assert_close(out.float(), rms_norm_ref(s, w, 1e-6).float(), atol=2e-2, rtol=1e-2)


def test_embedding_vocab_parallel():
    w = torch.randn(100, 256, device=DEV).bfloat16()
    ids = torch.tensor([0, 5, 99, 100, 150, 120], device=DEV, dtype=torch.int32)
    out = torch.empty(6, 256, device=DEV, dtype=torch.bfloat16)
    _ext().embedding(out, ids, w, 50)
    ref = torch.zeros(6, 256, device=DEV, dtype=torch.bfloat16)
    for i, t in enumerate(ids.tolist()):
        if 50 <= t < 150:
            ref[i] = w[t - 50]
    assert torch.equal(out, ref)


@pytest.mark.parametrize("D,qk_norm", [(64, False), (128, True)])
def test_qkv_prepare(D, qk_norm):
    from braidinfer_b200 import ops
    T, Hq, Hkv, PS, P = 37, 8, 2, 16, 8
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV).bfloat16()
    pos = torch.randint(0, 500, (T,), device=DEV, dtype=torch.int32)
    slots = torch.randperm(P * PS, device=DEV)[:T].int()
    cos, sin = ops.build_cos_sin(D, 10000.0, 1024, device=DEV)
    qn = (torch.rand(D, device=DEV) * 3).bfloat16() if qk_norm else None
    kn = (torch.rand(D, device=DEV) * 100 - 50).bfloat16() if qk_norm else None
    kv = torch.zeros(P, 2, Hkv, PS, D, device=DEV, dtype=torch.bfloat16)
    kv_ref = kv.clone().float()
    q = ops.qkv_prepare(qkv, pos, slots, kv, Hq, Hkv, D, cos, sin, qn, kn, 1e-6, True)
    q_ref = ops.qkv_prepare(qkv.float().cpu(), pos.cpu(), slots.cpu(), kv_ref.cpu(), Hq, Hkv, D, cos.cpu(),
                            sin.cpu(), None if qn is None else qn.cpu(), None if kn is None else kn.cpu(), 1e-6, True)
    torch.testing.assert_close(q.float().cpu(), q_ref.float(), atol=3e-2 * (50 if qk_norm else 1), rtol=2e-2)


def _rand_plan(seqs, PS, P, device, decode):
    """seqs: list of (q_len, [(seg_len, offset, delta)]) -> (meta tensors host dict, T)."""
    import numpy as np
    from braidinfer_b200.ops.attention import AttnMeta
    rng = np.random.default_rng(0)
    free = list(rng.permutation(P))
    qo, segi, spi, soff, slen, spos0, sdelta, pids, pos = [0], [0], [0], [], [], [], [], [], []
    for qlen, segs in seqs:
        p = 0
        for (n, off, delta) in segs:
            npg = -(-(off + n) // PS)
            pids += [free.pop() for _ in range(npg)]
            spi.append(len(pids)); soff.append(off); slen.append(n); spos0.append(p); sdelta.append(delta)
            p += n
        pos += list(range(p - qlen, p))
        qo.append(qo[-1] + qlen)
        segi.append(len(slen))
    host = {k: torch.tensor(v, dtype=torch.int32) for k, v in dict(
        qo_indptr=qo, positions=pos, seg_indptr=segi, seg_page_indptr=spi, seg_offset=soff, seg_len=slen,
        seg_pos0=spos0, seg_delta=sdelta, page_ids=pids).items()}
    dev = {k: v.to(device) for k, v in host.items()}
    maxq = max(q for q, _ in seqs)
    maxkv = max(sum(s[0] for s in segs) for _, segs in seqs)
    meta = AttnMeta(num_seqs=len(seqs), max_q_len=maxq, max_kv_len=maxkv, decode=decode, host=host, **dev)
    return meta, qo[-1]


@pytest.mark.parametrize("D,G", [(64, 8), (128, 2), (128, 4), (128, 8)])
@pytest.mark.parametrize("splits", [1, 3])
def test_attention_decode(D, G, splits):
    from braidinfer_b200 import ops
    PS, P, Hkv = 16, 512, 2
    Hq = Hkv * G
    seqs = [(1, [(37, 0, 5), (100, 3, -7), (9, 0, 0)]), (1, [(1, 0, 0)]), (1, [(300, 0, 0)]),
            (1, [(64, 0, 2), (64, 0, 0), (130, 0, 0)])]
    meta, T = _rand_plan(seqs, PS, P, DEV, True)
    meta.num_splits = splits
    kv = torch.randn(P, 2, Hkv, PS, D, device=DEV).bfloat16()
    q = torch.randn(T, Hq, D, device=DEV).bfloat16()
    cos, sin = ops.build_cos_sin(D, 10000.0, 2048, device=DEV)
    out = ops.attention(q, kv, meta, cos, sin, D ** -0.5, True)
    ref = ops.attention_ref(q.cpu().float(), kv.cpu().float(), meta, cos.cpu(), sin.cpu(), D ** -0.5, True)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("D,G", [(64, 8), (128, 2), (128, 4)])
@pytest.mark.parametrize("splits", [1, 3, 7])
def test_attention_prefill(D, G, splits, prefill_kernel):
    """splits > 1: keys divided over CTAs, partials merged by the last CTA."""
    from braidinfer_b200 import ops
    PS, P, Hkv = 16, 1024, 2
    Hq = Hkv * G
    # (q_len, segments): last segment is the private one holding the queries
    seqs = [(50, [(40, 0, 3), (70, 5, -11), (50, 0, 0)]), (1, [(1, 0, 0)]), (200, [(200, 0, 0)]),
            (17, [(128, 0, 0), (33, 0, 0)])]
    meta, T = _rand_plan(seqs, PS, P, DEV, False)
    meta.num_splits = splits
    kv = torch.randn(P, 2, Hkv, PS, D, device=DEV).bfloat16()
    q = torch.randn(T, Hq, D, device=DEV).bfloat16()
    cos, sin = ops.build_cos_sin(D, 10000.0, 2048, device=DEV)
    out = ops.attention(q, kv, meta, cos, sin, D ** -0.5, True)
    ref = ops.attention_ref(q.cpu().float(), kv.cpu().float(), meta, cos.cpu(), sin.cpu(), D ** -0.5, True)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("D,G", [(64, 8), (128, 4)])
def test_attention_prefill_short_query_long_context(D, G, prefill_kernel):
    """A short query over long cached chunks picks key splits automatically."""
    from braidinfer_b200 import ops
    PS, P, Hkv = 16, 1024, 2
    Hq = Hkv * G
    seqs = [(20, [(300, 0, 4), (500, 7, -3), (129, 3, 9), (20, 0, 0)])]
    meta, T = _rand_plan(seqs, PS, P, DEV, False)
    kv = torch.randn(P, 2, Hkv, PS, D, device=DEV).bfloat16()
    q = torch.randn(T, Hq, D, device=DEV).bfloat16()
    cos, sin = ops.build_cos_sin(D, 10000.0, 2048, device=DEV)
    out = ops.attention(q, kv, meta, cos, sin, D ** -0.5, True)
    ref = ops.attention_ref(q.cpu().float(), kv.cpu().float(), meta, cos.cpu(), sin.cpu(), D ** -0.5, True)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)


def test_sampler_greedy_and_filters():
    from braidinfer_b200.ops.sampling import sample_ref
    B, V = 6, 50000
    logits = torch.randn(B, V, device=DEV) * 3
    temp = torch.tensor([0.0, 1.0, 0.7, 1.0, 1.3, 0.5], device=DEV)
    topk = torch.tensor([0, 0, 5, 1, 0, 50], device=DEV, dtype=torch.int32)
    topp = torch.tensor([1.0, 1.0, 1.0, 1.0, 0.5, 0.9], device=DEV)
    minp = torch.tensor([0.0, 0.0, 0.0, 0.0, 0.0, 0.1], device=DEV)
    seed = torch.arange(B, device=DEV, dtype=torch.int64) + 11
    step = torch.full((B,), 3, device=DEV, dtype=torch.int64)
    out = torch.empty(B, dtype=torch.int32, device=DEV)
    _ext().sample(out, logits, temp, topk, topp, minp, seed, step, False)
    ref = sample_ref(logits.cpu(), temp.cpu(), topk.cpu(), topp.cpu(), minp.cpu(), seed.cpu(), step.cpu())
    assert out[0].item() == logits[0].argmax().item()
    assert out[3].item() == logits[3].argmax().item()  # top_k = 1
    top5 = set(logits[2].topk(5).indices.tolist())
    assert out[2].item() in top5
    # same hash on both sides: identical draws
    assert out.cpu().tolist() == ref.tolist()


@pytest.mark.parametrize("D,G", [(128, 4), (128, 8), (64, 8)])
@pytest.mark.parametrize("own_splits,shared_splits", [(1, 5), (2, 9)])
def test_attention_shared_prefix_decode(D, G, own_splits, shared_splits, prefill_kernel):
    """Decode where five of seven sequences compose the same cached chunks at
    the same positions: the shared segments are attended once for the group
    (prefill kernel over the group's tokens, partials only) and merged with
    each sequence's private keys by the decode kernel.  Checked against the
    fp32 restatement of the ungrouped plan."""
    from braidinfer_b200 import ops
    from braidinfer_b200.engine.batch import FwdItem, build_plan, find_shared_group, make_meta, pack, unpack
    from braidinfer_b200.engine.sequence import SegmentRef
    PS, P, Hkv = 16, 512, 2
    Hq = Hkv * G
    sys_seg = SegmentRef(pages=[0], offset=0, length=10, pos0=0, delta=0)
    ctx = SegmentRef(pages=list(range(1, 21)), offset=0, length=300, pos0=10, delta=3)
    ctx_moved = SegmentRef(pages=list(range(1, 21)), offset=0, length=300, pos0=20, delta=13)
    items, nxt = [], 40
    for b, plen in enumerate([5, 17, 1, 33, 9, 12, 40]):
        member = b not in (2, 5)
        segs = [sys_seg, ctx] if member else [ctx_moved]
        base = 310 if member else 320
        pages = list(range(nxt, nxt + 3))
        nxt += 3
        items.append(FwdItem(tokens=[1], pos0=base + plen - 1, priv_index0=plen - 1, priv_pages=pages,
                             priv_pos0=base, segments=segs))
    members, keys = find_shared_group(items, PS)
    assert sorted(members) == [0, 1, 3, 4, 6]
    order = members + [i for i in range(len(items)) if i not in members]
    items = [items[i] for i in order]
    plan_g = build_plan(items, PS, group=(len(members), keys))
    plan_u = build_plan(items, PS)
    views = unpack(torch.from_numpy(pack(plan_g)).to(DEV), plan_g.sizes)
    meta_g = make_meta(views, plan_g, own_splits, shared_splits=shared_splits)
    meta_u = make_meta(unpack(torch.from_numpy(pack(plan_u)), plan_u.sizes), plan_u)
    g = torch.Generator(device=DEV).manual_seed(D + G)
    kv = torch.randn(P, 2, Hkv, PS, D, device=DEV, generator=g).bfloat16()
    q = torch.randn(len(items), Hq, D, device=DEV, generator=g).bfloat16()
    cos, sin = ops.build_cos_sin(D, 10000.0, 2048, device=DEV)
    for _ in range(2):  # the partial slots are reused call after call
        out = ops.attention(q, kv, meta_g, cos, sin, D ** -0.5, True)
        torch.cuda.synchronize()
    ref = ops.attention_ref(q.cpu().float(), kv.cpu().float(), meta_u, cos.cpu(), sin.cpu(), D ** -0.5, True)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("splits", [1, 4])
@pytest.mark.parametrize("G", [1, 4, 8])
@pytest.mark.parametrize("poly", [0, 2, 4])
def test_attention_prefill_pages256(G, splits, prefill_kernel, poly):
    """Prefill with head_dim 128 and 256-token pages (64-row TMA boxes):
    segments with RoPE deltas, offsets into their first page, a long causal
    private segment (several 128-key tiles, several query tiles) and a
    1-token sequence.  ``poly``: share of the tcgen05 softmax exponentials
    computed by polynomial (every 2nd / 4th)."""
    if poly and not prefill_kernel:
        pytest.skip("the polynomial share applies to the tcgen05 kernel")
    _ext().attn_set_exp2_poly(poly)
    try:
        _prefill_pages256(G, splits)
    finally:
        _ext().attn_set_exp2_poly(-1)


@pytest.mark.parametrize("splits", [1, 2])
def test_attention_prefill_growing_scores(splits, prefill_kernel):
    """Scores that grow along the keys (key norms ramp up): the row maximum
    rises by far more than 2^8 per 128-key tile, so the tcgen05 kernel
    rescales O in tensor memory on every tile."""
    from braidinfer_b200 import ops
    PS, P, Hkv, G, D = 16, 128, 2, 4, 128
    seqs = [(600, [(600, 0, 0)]), (130, [(70, 0, 3), (130, 0, 0)])]
    meta, T = _rand_plan(seqs, PS, P, DEV, False)
    meta.num_splits = splits
    g = torch.Generator(device=DEV).manual_seed(5)
    kv = torch.randn(P, 2, Hkv, PS, D, device=DEV, generator=g).abs()
    h = meta.host
    ramp = torch.ones(P, PS)
    for si in range(len(h["seg_len"])):  # key norm grows with the key's position in its sequence
        pg0, off, pos0 = int(h["seg_page_indptr"][si]), int(h["seg_offset"][si]), int(h["seg_pos0"][si])
        for i in range(int(h["seg_len"][si])):
            ramp[int(h["page_ids"][pg0 + (off + i) // PS]), (off + i) % PS] = 0.5 + (pos0 + i) / 60.0
    kv[:, 0] *= ramp.to(DEV)[:, None, :, None]
    kv = kv.bfloat16()
    q = torch.randn(T, Hkv * G, D, device=DEV, generator=g).abs().bfloat16()
    cos, sin = ops.build_cos_sin(D, 10000.0, 2048, device=DEV)
    out = ops.attention(q, kv, meta, cos, sin, D ** -0.5, False)
    ref = ops.attention_ref(q.cpu().float(), kv.cpu().float(), meta, cos.cpu(), sin.cpu(), D ** -0.5, False)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=3e-2, rtol=3e-2)


def _prefill_pages256(G, splits):
    from braidinfer_b200 import ops
    PS, P, Hkv = 256, 64, 2
    Hq = Hkv * G
    seqs = [(300, [(130, 0, 7), (260, 40, -5), (300, 0, 0)]), (1, [(1, 0, 0)]), (77, [(500, 0, 0), (77, 0, 0)])]
    meta, T = _rand_plan(seqs, PS, P, DEV, False)
    meta.num_splits = splits
    g = torch.Generator(device=DEV).manual_seed(G * 10 + splits)
    kv = torch.randn(P, 2, Hkv, PS, 128, device=DEV, generator=g).bfloat16()
    q = torch.randn(T, Hq, 128, device=DEV, generator=g).bfloat16()
    cos, sin = ops.build_cos_sin(128, 500000.0, 4096, device=DEV)
    out = ops.attention(q, kv, meta, cos, sin, 128 ** -0.5, True)
    ref = ops.attention_ref(q.cpu().float(), kv.cpu().float(), meta, cos.cpu(), sin.cpu(), 128 ** -0.5, True)
    torch.testing.assert_close(out.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)
