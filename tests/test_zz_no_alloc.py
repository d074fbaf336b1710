"""The allocation-free GEMM entry point (``braid_gemm_noalloc``, exported with
C linkage from the native extension) must give the same result as the regular
``gemm`` binding, call after call, while allocating nothing itself.

It serves callers that cannot allocate device memory (allocator callbacks,
plugin hosts that forbid cudaMalloc after start-up, latency-critical loops);
its split-K scratch is a fixed file-scope device array.  This file is named to
be collected last.
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
    return fn, err


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("T,N,K,use_bias,use_res,rms", [(1, 4096, 4096, False, False, False),
                                                        (8, 6144, 4096, True, False, False),
                                                        (16, 1024, 14336, False, True, False),
                                                        (40, 2048, 1024, True, True, True)])
def test_noalloc_matches_regular_entry(T, N, K, use_bias, use_res, rms):
    from braidinfer_b200.ops._ext import ext

    fn, err = _lib()
    g = torch.Generator(device="cuda").manual_seed(T * 131 + N)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16() if use_bias else None
    r = torch.randn(T, N, device="cuda", generator=g).bfloat16() if use_res else None
    eps = 1e-5 if rms else -1.0
    ref = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    ext().gemm(ref, x, w, b, r, 0, eps)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row reuse the same scratch
        out = torch.full((T, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc = fn(_ptr(out), _ptr(x), _ptr(w), _ptr(b), _ptr(r), T, N, K, N, K, K, N if use_res else 0, eps,
                ctypes.c_void_p(stream))
        assert rc == 0, err().decode()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=3e-2, rtol=2e-2)


def test_noalloc_rejects_out_of_range_sizes():
    fn, err = _lib()
    x = torch.zeros(65, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(128, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(65, 128, device="cuda", dtype=torch.bfloat16)
    rc = fn(_ptr(out), _ptr(x), _ptr(w), None, None, 65, 128, 64, 128, 64, 64, 0, -1.0, None)
    assert rc != 0 and b"[1, 64]" in err()
