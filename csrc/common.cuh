// Shared device helpers for the sm_100a kernels: bf16 packing, warp
// reductions, and thin inline-PTX wrappers for mbarriers, TMA
// (cp.async.bulk.tensor, no cluster multicast anywhere in this project) and
// the tcgen05 tensor-core / tensor-memory instructions.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define BRAID_DEVICE __device__ __forceinline__

namespace braid {

// ---- bounds-checked build (-DBRAID_BOUNDS_CHECK; python setup.py with
// BRAID_BOUNDS_CHECK=1 builds it as braidinfer_b200._C_checked).  Indices that
// kernels take from data (KV slots, RoPE positions, page ids) are checked
// before use: a violation records {code << 48 | value} in this translation
// unit's status word (first violation wins) and the access is skipped or
// clamped, never trapped, so the context stays usable.  Codes: 1 KV slot
// outside the cache, 2 position outside the RoPE table, 4 page id outside the
// KV pool.  In the regular build the checks compile to nothing.
#ifdef BRAID_BOUNDS_CHECK
static __device__ unsigned long long g_bounds_status;
BRAID_DEVICE bool bounds_ok(bool ok, unsigned code, long long value) {
  if (!ok)
    atomicCAS(&g_bounds_status, 0ull,
              ((unsigned long long)code << 48) | ((unsigned long long)value & 0xFFFFFFFFFFFFull));
  return ok;
}
#define BRAID_IN_BOUNDS(cond, code, value) ::braid::bounds_ok((cond), (code), (long long)(value))
// Host reader of this translation unit's status word: waits for the device,
// returns the word and clears it.
#define BRAID_BOUNDS_READER(fn)                                                             \
  unsigned long long fn() {                                                                 \
    unsigned long long v = 0, z = 0;                                                        \
    C10_CUDA_CHECK(cudaDeviceSynchronize());                                                \
    C10_CUDA_CHECK(cudaMemcpyFromSymbol(&v, ::braid::g_bounds_status, sizeof(v)));         \
    C10_CUDA_CHECK(cudaMemcpyToSymbol(::braid::g_bounds_status, &z, sizeof(z)));           \
    return v;                                                                               \
  }
#else
#define BRAID_IN_BOUNDS(cond, code, value) true
#define BRAID_BOUNDS_READER(fn) \
  unsigned long long fn() { return 0; }
#endif

BRAID_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
BRAID_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }
// Round-trip through bf16 (emulates an HF op boundary in bf16).
BRAID_DEVICE float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

BRAID_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
BRAID_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

BRAID_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
BRAID_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
BRAID_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
BRAID_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
BRAID_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
BRAID_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
BRAID_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Launch-span trace (profiling): span[0] = earliest CTA start, span[1] =
// earliest time a CTA passed its dependency wait, span[2] = latest CTA end.
BRAID_DEVICE void span_start(unsigned long long* span) {
  if (span != nullptr) atomicMin(span, (unsigned long long)globaltimer_ns());
}
BRAID_DEVICE void span_waited(unsigned long long* span) {
  if (span != nullptr) atomicMin(span + 1, (unsigned long long)globaltimer_ns());
}
BRAID_DEVICE void span_end(unsigned long long* span) {
  if (span != nullptr) atomicMax(span + 2, (unsigned long long)globaltimer_ns());
}

// Acquire load at system scope (flags written by peer GPUs over NVLink).
BRAID_DEVICE uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Release store at system scope (a flag a peer GPU polls).
BRAID_DEVICE void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// Orders this thread's earlier generic-proxy accesses (and what they acquired)
// before its later async-proxy (TMA) accesses of global memory.
BRAID_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// Bounded wait on an mbarrier phase: gives up after `timeout_ns` of wall time
// (checked every 256 polls).  Returns false on timeout so the caller can
// record an error and unwind instead of hanging the GPU.
BRAID_DEVICE bool mbar_wait(uint64_t* bar, uint32_t phase, uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}
// Programmatic dependent launch: wait until the preceding grid in the stream
// has completed and its memory is visible (no-op without the PDL attribute);
// allow the next grid to begin launching.
BRAID_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
BRAID_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Thread-block cluster helpers (distributed shared memory).
BRAID_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
BRAID_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
BRAID_DEVICE uint32_t dsmem_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_addr), "r"(rank));
  return d;
}
// Volatile (kept in program order relative to the cluster barriers) but
// without a memory clobber, so consecutive loads are issued back to back.
BRAID_DEVICE float4 dsmem_ld_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// GPU-scope acquire/release fence.  After a CTA barrier, one thread's fence is
// cumulative over the writes the barrier ordered before it (release side);
// before a CTA barrier it orders the other threads' later reads (acquire side).
BRAID_DEVICE void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// atomicAdd with acquire-release semantics at GPU scope (release is cumulative
// over writes ordered before it by a CTA barrier).
BRAID_DEVICE int atomic_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

BRAID_DEVICE void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// --------------------------------------------------------------------- TMA
BRAID_DEVICE void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}
// 2D tiled load global -> shared (this CTA only), completion on `bar`.
BRAID_DEVICE void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 cache policy for streams read exactly once (decode weights, this step's
// K/V): evicted first, so they do not push out lines other kernels prefetched.
BRAID_DEVICE uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// 2D tiled load with an L2 cache-policy hint.
BRAID_DEVICE void tma_load_2d_hint(void* smem_dst, const void* desc, uint64_t* bar, int x, int y, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y),
        "l"(pol)
      : "memory");
}
// Prefetch one tile of a tensor map into L2 (no shared memory, no completion).
BRAID_DEVICE void tma_prefetch_l2_2d(const void* desc, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
               ::"l"(reinterpret_cast<uint64_t>(desc)), "r"(x), "r"(y)
               : "memory");
}

// Cross-kernel weight prefetch: a decode-step kernel, once its own loads are
// issued, pulls the first K-blocks of the NEXT GEMM's weight into L2, in the
// order that GEMM's CTAs will read them (K-slice `split` of 128-row tile `mt`
// starts at K-block split * kbps).  So the HBM stream does not stall across
// the kernel boundary (this kernel's tail, the next kernel's ramp).  The tile
// is the next GEMM's own TMA box (64 columns x 128 rows, its tensor map).
struct PrefetchArgs {
  int m_tiles;   // 128-row tiles of the next weight
  int splits;    // its K-slices
  int kbps;      // K-blocks per slice
  int kb_total;  // K-blocks of a row
  int skip;      // K-blocks of every slice already prefetched by an earlier launch
  int depth;     // K-blocks of every slice to prefetch after those (0: none)
};
// This CTA's share (CTA `cta` of `ncta`) of the prefetch, issued by one thread.
BRAID_DEVICE void prefetch_next_weight(const void* tmap, const PrefetchArgs& pf, int cta, int ncta) {
  if (pf.depth <= 0) return;
  const int per_depth = pf.m_tiles * pf.splits;
  const int total = per_depth * pf.depth;
  for (int i = cta; i < total; i += ncta) {
    const int j = i / per_depth, r = i % per_depth;
    const int split = r / pf.m_tiles, mt = r % pf.m_tiles;
    const int kb = split * pf.kbps + pf.skip + j;
    if (pf.skip + j < pf.kbps && kb < pf.kb_total) tma_prefetch_l2_2d(tmap, kb * 64, mt * 128);
  }
}

// ----------------------------------------------------------------- tcgen05
BRAID_DEVICE void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
BRAID_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
BRAID_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
BRAID_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
BRAID_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate.
BRAID_DEVICE void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread completes.
BRAID_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
BRAID_DEVICE void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32-bit, 16 consecutive columns -> 16 registers per thread.
BRAID_DEVICE void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// D[tmem] (+)= A[tmem] * B[smem desc]: the A operand (M rows = TMEM lanes,
// two bf16 K-elements per 32-bit column, lower K index in the low half) read
// from tensor memory.
BRAID_DEVICE void tc_mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                 uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
BRAID_DEVICE void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32-bit, 32 consecutive columns <-> 32 registers per thread.
BRAID_DEVICE void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
BRAID_DEVICE void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: 8-row x 128-byte atoms, atoms 1024 bytes apart
// (stride byte offset), leading byte offset unused for swizzled K-major,
// descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
BRAID_DEVICE uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // LBO (16 B units), ignored for SW128 K-major
  d |= (uint64_t)(1024 >> 4) << 32;       // SBO = 1024 B
  d |= (uint64_t)1 << 46;                 // version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A=B=bf16, D=f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace braid

namespace braid {
// ------------------------------------------------------- mma.sync helpers
BRAID_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
BRAID_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D  (fp32)
BRAID_DEVICE void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
BRAID_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// 16-byte async copy global->shared; src_bytes = 0 zero-fills the destination.
BRAID_DEVICE void cp_async16(uint32_t smem_addr, const void* gmem, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gmem), "r"(n) : "memory");
}
BRAID_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
BRAID_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
}  // namespace braid
