// Allocation-free decode GEMM entry point.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that must not allocate device memory themselves or
// through us: code running inside a custom allocator's callbacks, a plugin
// host that forbids cudaMalloc after start-up, or a latency-critical loop that
// cannot afford an allocation (or its implicit device synchronisation).  It is
// the split-K tcgen05 GEMM of gemm_tcgen05.cu, but its split-K scratch (fp32
// partial tiles, tile counters and the error word) lives in one file-scope
// device array of fixed size instead of a workspace we allocate on demand.
//
//   out[T, N] = x[T, K] @ w[N, K]^T (+ bias[N]) (+ residual[T, N]),  bf16,
//   optionally with the fused input RMSNorm (rs_eps >= 0; w must then carry
//   the norm weight folded into its columns).
//
// Limits: 1 <= T <= 64 tokens (the decode shape), K and the row strides
// multiples of 8 elements, 16-byte aligned operands.  Split-K partials are
// limited to BRAID_NOALLOC_PARTIAL_BYTES; larger problems run with fewer
// K-slices (never with more scratch).
//
// Set-up: the first call on each device looks up the device address of the
// scratch array (with that device current), clears it on the caller's stream
// and waits for that clear; make that first call before any stream capture.
// Every later call reuses the same array and clears the tile counters on the
// caller's stream.  All calls on one device share that device's array, so two
// calls that can execute at the same time on one device (for example on two
// streams with no ordering between them) race on it and must be serialised
// by the caller; calls on different devices use different copies.
//
// Returns 0 once the kernel is launched; otherwise a nonzero code, and
// braid_gemm_noalloc_last_error() describes the problem.  Problems the kernel
// meets on the GPU (a bounded pipeline wait that ran out) are recorded in the
// array's error word, which stays set until braid_gemm_noalloc_check_error()
// reads it: that call waits for `stream`, returns the word (0 = no error,
// -1 = the read itself failed) and clears it.  Nothing here calls cudaMalloc,
// cudaFree, or any allocating library routine.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define BRAID_NOALLOC_MAX_TOKENS 64
#define BRAID_NOALLOC_PARTIAL_BYTES (4u << 20)
#define BRAID_NOALLOC_MAX_TILES 16384

int braid_gemm_noalloc(void* out, const void* x, const void* w, const void* bias, const void* residual, int T,
                       int N, int K, int ldo, int ldx, int ldw, int ldr, float rs_eps, void* stream);
const char* braid_gemm_noalloc_last_error(void);
int braid_gemm_noalloc_check_error(void* stream);

#ifdef __cplusplus
}
#endif
