"""The bounds-checked build (``braidinfer_b200._C_checked``, -DBRAID_BOUNDS_CHECK)
records indices read from data that fall outside their buffer, and skips the
access, instead of faulting the GPU.

compute-sanitizer is not available on the B200 pool, so this build is the
substitute for its memcheck on the paths that index memory with values taken
from the step's metadata: the KV append (slot), RoPE (position) and the paged
K/V reads (page id).  Every test here is safe even if a check were missing:
the KV pool and the RoPE tables are views of larger allocations, and the
out-of-range index points into the guard region just past the view, which
the test then checks is untouched.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture
def checked():
    """Routes the ops through the checked build for the duration of a test."""
    try:
        from braidinfer_b200 import _C_checked as C
    except ImportError:
        pytest.skip("bounds-checked build not present: BRAID_BOUNDS_CHECK=1 python setup.py build_ext --inplace "
                    "--build-temp build/checked")
    assert C.bounds_check_enabled()
    from braidinfer_b200.ops import _ext
    _ext.ext()  # regular build loaded first (restored afterwards)
    saved = _ext._C
    _ext._C = _ext._Counted(C)
    C.bounds_check_status()  # clear
    yield C
    torch.cuda.synchronize()
    _ext._C = saved


def _status(C):
    v = int(C.bounds_check_status())
    return v >> 48, v & 0xFFFFFFFFFFFF


def _qkv_inputs(T, Hq, Hkv, D, P, PS, rope_len):
    g = torch.Generator(device=DEV).manual_seed(1)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV, generator=g).bfloat16()
    big_kv = torch.zeros(P + 1, 2, Hkv, PS, D, device=DEV, dtype=torch.bfloat16)
    from braidinfer_b200 import ops
    cos_big, sin_big = ops.build_cos_sin(D, 10000.0, rope_len + 8, device=DEV)
    return qkv, big_kv, cos_big, sin_big


def test_regular_build_reports_checks_off():
    from braidinfer_b200.ops._ext import ext
    assert not ext().bounds_check_enabled() and ext().bounds_check_status() == 0


@pytest.mark.parametrize("path", ["qkv_prepare", "qkv_gemm"])
def test_kv_slot_and_rope_position_out_of_range(checked, path):
    from braidinfer_b200 import ops
    T, Hq, Hkv, D, P, PS, rope_len = 8, 8, 2, 128, 4, 16, 256
    qkv, big_kv, cos_big, sin_big = _qkv_inputs(T, Hq, Hkv, D, P, PS, rope_len)
    kv = big_kv[:P]
    cos, sin = cos_big[:rope_len], sin_big[:rope_len]
    w = (torch.randn((Hq + 2 * Hkv) * D, 512, device=DEV) * 0.05).bfloat16()
    x = torch.randn(T, 512, device=DEV).bfloat16()

    def run(pos, slots):
        if path == "qkv_prepare":
            return ops.qkv_prepare(qkv, pos, slots, kv, Hq, Hkv, D, cos, sin, None, None, 1e-6, True)
        return ops.qkv_gemm(x, w, None, None, pos, slots, kv, Hq, Hkv, D, cos, sin, None, None, 1e-6, True)

    pos = torch.arange(T, device=DEV, dtype=torch.int32) * 3
    good = torch.arange(T, device=DEV, dtype=torch.int32) * 5
    run(pos, good)
    torch.cuda.synchronize()
    assert _status(checked) == (0, 0)
    ref = kv.clone()

    # one slot just past the cache: skipped (the guard page stays zero), recorded
    bad = good.clone()
    bad[3] = P * PS
    kv.zero_()
    run(pos, bad)
    torch.cuda.synchronize()
    assert _status(checked) == (1, P * PS)
    assert torch.count_nonzero(big_kv[P]) == 0
    keep = torch.ones(P * PS, dtype=torch.bool, device=DEV)
    keep[int(good[3])] = False
    flat = lambda t: t.permute(0, 3, 1, 2, 4).reshape(P * PS, -1)  # noqa: E731
    assert torch.equal(flat(kv)[keep], flat(ref)[keep])

    # a position just past the RoPE table: clamped, recorded
    bad_pos = pos.clone()
    bad_pos[5] = rope_len
    run(bad_pos, good)
    torch.cuda.synchronize()
    assert _status(checked) == (2, rope_len)


def test_page_id_outside_the_pool(checked):
    from braidinfer_b200 import ops
    from test_kernels_gpu import _rand_plan
    PS, P, Hkv, G, D = 16, 64, 2, 4, 128
    seqs = [(1, [(40, 0, 0)]), (1, [(70, 0, 0)])]
    meta, T = _rand_plan(seqs, PS, P, DEV, True)
    meta.num_splits = 1
    big = torch.randn(P + 1, 2, Hkv, PS, D, device=DEV).bfloat16()
    kv = big[:P]
    q = torch.randn(T, Hkv * G, D, device=DEV).bfloat16()
    cos, sin = ops.build_cos_sin(D, 10000.0, 512, device=DEV)
    ops.attention(q, kv, meta, cos, sin, D ** -0.5, True)
    torch.cuda.synchronize()
    assert _status(checked) == (0, 0)
    meta.page_ids[0] = P  # the first page of the first sequence lies past the pool
    out = ops.attention(q, kv, meta, cos, sin, D ** -0.5, True)
    torch.cuda.synchronize()
    assert _status(checked) == (4, P)
    assert torch.isfinite(out.float()).all()
