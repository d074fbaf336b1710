"""The allocation-free GEMM entry point (``braid_gemm_noalloc``, exported with
C linkage from the native extension) must give the same result as the regular
``gemm`` binding and as a plain fp32 PyTorch computation of the same op, call
after call, while allocating nothing itself.

It serves callers that cannot allocate device memory: code running inside a
custom allocator's callbacks (allocating there would re-enter the allocator),
plugin hosts that forbid ``cudaMalloc`` after start-up, and latency-critical
loops that cannot take an allocation's implicit synchronisation.  Its split-K
scratch is a fixed file-scope device array, so these tests also cover the
first call's set-up on a non-default stream, the K-slice clamp that keeps a
large problem inside that array, and the device error word, which must read
0 after correct calls.  This file is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import braidinfer_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.braid_gemm_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_void_p]
    err = lib.braid_gemm_noalloc_last_error
    err.restype = ctypes.c_char_p
    chk = lib.braid_gemm_noalloc_check_error
    chk.restype = ctypes.c_int
    chk.argtypes = [ctypes.c_void_p]
    return fn, err, chk


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _fp32_reference(x, w, b, r, eps):
    """out = bf16(bf16(rms(x) @ w^T + b) + r), computed in fp32."""
    xf = x.float()
    if eps >= 0:
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = xf @ w.float().t()
    if b is not None:
        y = y + b.float()
    y = y.bfloat16().float()
    if r is not None:
        y = y + r.float()
    return y.bfloat16().float()


def _inputs(T, N, K, use_bias, use_res, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16() if use_bias else None
    r = torch.randn(T, N, device="cuda", generator=g).bfloat16() if use_res else None
    return x, w, b, r


def _call(fn, err, x, w, b, r, eps, stream):
    T, K = x.shape
    N = w.shape[0]
    out = torch.full((T, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc = fn(_ptr(out), _ptr(x), _ptr(w), _ptr(b), _ptr(r), T, N, K, N, K, K, N if r is not None else 0, eps,
            ctypes.c_void_p(stream))
    assert rc == 0, err().decode()
    return out


def test_noalloc_first_call_on_a_side_stream():
    """Set-up (address lookup and scratch clear) ordered on a non-blocking
    stream created before the first call; the first GEMM follows on it."""
    fn, err, chk = _lib()
    side = torch.cuda.Stream()
    x, w, b, r = _inputs(8, 4096, 4096, True, True, 7)
    with torch.cuda.stream(side):
        outs = [_call(fn, err, x, w, b, r, -1.0, side.cuda_stream) for _ in range(2)]
    side.synchronize()
    ref = _fp32_reference(x, w, b, r, -1.0)
    for out in outs:
        torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=2e-2)
    assert chk(ctypes.c_void_p(side.cuda_stream)) == 0


@pytest.mark.parametrize("T,N,K,use_bias,use_res,rms", [(1, 4096, 4096, False, False, False),
                                                        (8, 6144, 4096, True, False, False),
                                                        (16, 1024, 14336, False, True, False),
                                                        (40, 2048, 1024, True, True, True),
                                                        # 64 tiles x 4 slices x 32 KB would exceed the
                                                        # 4 MiB partial area: runs with fewer slices
                                                        (64, 8192, 4096, False, True, False)])
def test_noalloc_matches_regular_entry_and_fp32(T, N, K, use_bias, use_res, rms):
    from braidinfer_b200.ops._ext import ext

    fn, err, chk = _lib()
    x, w, b, r = _inputs(T, N, K, use_bias, use_res, T * 131 + N)
    eps = 1e-5 if rms else -1.0
    regular = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm(regular, x, w, b, r, 0, eps)
    ref = _fp32_reference(x, w, b, r, eps)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row reuse the same scratch
        out = _call(fn, err, x, w, b, r, eps, stream)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), regular.float(), atol=3e-2, rtol=2e-2)
        torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=3e-2)
    assert chk(ctypes.c_void_p(stream)) == 0


def test_noalloc_rejects_out_of_range_sizes():
    fn, err, _ = _lib()
    x = torch.zeros(65, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(128, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(65, 128, device="cuda", dtype=torch.bfloat16)
    rc = fn(_ptr(out), _ptr(x), _ptr(w), None, None, 65, 128, 64, 128, 64, 64, 0, -1.0, None)
    assert rc != 0 and b"[1, 64]" in err()
