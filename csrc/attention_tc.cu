// tcgen05 prefill attention for sm_100a (head_dim 128): the tensor-core path
// of paged cascade attention for prefill-shaped work — chunk self-prefill,
// a request's prompt over cached chunks, and the shared-prefix pass of a
// batched decode step.
//
// One CTA owns 256 query rows, each a (token, head-of-the-KV-group) pair of
// one sequence (or of one shared-prefix group), as two 128-row Q tiles
// against one KV head.  Tensor memory (512 columns):
//   [0, 128)    S(0) = Q(0) K^T, fp32; P(0) as bf16 pairs in its columns [64, 128)
//   [128, 256)  S(1), P(1)
//   [256, 384)  O(0) += P(0) V   (P read from tensor memory, V MN-major from smem)
//   [384, 512)  O(1)
// Warp roles (10 warps):
//   warp 0      TMA producer: 128-key K and V tiles of the paged KV cache
//               (128-byte swizzle), separate 2-stage K and V rings
//   warp 1      MMA issuer (one lane), per key tile j in the order
//                 P(0,j)V, S(0,j+1), P(1,j)V, S(1,j+1)
//               so the tensor core runs one tile's MMAs while the other
//               tile's softmax warps work
//   warps 2..5  softmax of Q tile 0, warps 6..9 of Q tile 1: one row per
//               thread (its TMEM lane); the rotated query row (differential
//               RoPE per segment) is built into shared memory; per key tile
//               one read of the S row, masks only on boundary tiles, ex2,
//               P stored back as bf16; the running maximum moves only when a
//               tile's exceeds it by more than 2^8, and only then is O
//               rescaled in tensor memory
// Same semantics and output modes as attn_prefill_kernel (attention.cu):
// key j of segment s is visible to a row at position p iff seg_pos0[s]+j <= p;
// with num_splits > 1 each CTA covers one range of the visible keys and the
// last CTA of the q tile merges (log-sum-exp); partial_only publishes the
// partials for the decode kernel (shared-prefix decode).
// Replaces the reference's per-page Triton online-softmax calls
// (braidinfer/kernels/online_softmax.py:15-214) on the prefill side.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "attention_types.cuh"
#include "common.cuh"
#include "launch.cuh"

namespace braid {

constexpr int TC_D = 128;          // head dim
constexpr int TC_ROWS = 128;       // query rows per Q tile (MMA M)
constexpr int TC_QT = 2;           // Q tiles per CTA
constexpr int TC_CTA_ROWS = TC_QT * TC_ROWS;
constexpr int TC_KEYS = 128;       // keys per tile (MMA N of S, K of P V)
constexpr int TC_STAGES = 2;       // depth of the K ring and of the V ring
constexpr int TC_P_COL = 64;       // P(t) columns within S(t)
constexpr int TC_THREADS = 64 + 128 * TC_QT;
constexpr int TC_HALF = TC_KEYS * 128;  // bytes of one 64-column half of a 128-row bf16 tile (16 KB)
constexpr int TC_TILE = 2 * TC_HALF;    // one 128 x 128 bf16 tile (32 KB)

struct TcSmem {
  static constexpr int Q = 0;                              // [Q tile][2 halves][128 rows][128 B]
  static constexpr int K = Q + TC_QT * TC_TILE;            // [stage][2 dim halves][128 keys][128 B]
  static constexpr int V = K + TC_STAGES * TC_TILE;        // same layout
  static constexpr int BAR = V + TC_STAGES * TC_TILE;
  static constexpr int TOTAL = BAR + 256 + 1024;           // barriers + TMEM address, 1024 alignment slack
};

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle:
// 64-element (128-byte) rows along MN, 8-row groups along K `sbo` bytes
// apart, 64-element MN blocks `lbo` bytes apart (canonical SW128 MN-major
// layout of the tcgen05 matrix descriptor), descriptor version 1.
BRAID_DEVICE uint64_t smem_desc_sw128_mn(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Generic-proxy shared-memory writes (Q, P) before tcgen05.mma reads them.
BRAID_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of 16-byte chunk c (0..15, 8 bf16 each) of row r in a 128-row,
// 128-column bf16 tile stored as two 64-column halves with 128-byte swizzle.
BRAID_DEVICE uint32_t tc_off(int r, int c) {
  const int h = c >> 3, cc = c & 7;
  return (uint32_t)(h * TC_HALF + r * 128 + ((cc ^ (r & 7)) << 4));
}

// The walk over this CTA's key tiles (identical in every warp role): segment
// s, key range [lo, hi) of it (visible keys within this split), tiles of 128
// cache slots starting at the 128-aligned slot below off + lo.
struct TcWalk {
  int s, s1, segstart, lo, hi, off, sl;
};

struct TcRange {
  int max_pos, r0, r1;
};

BRAID_DEVICE int tc_seg_vis(const AttnParams& p, int s, int max_pos) {
  return max(0, min(p.seg_len[s], max_pos - p.seg_pos0[s] + 1));
}

// Advance w to the next segment with keys in [r0, r1); false when done.
BRAID_DEVICE bool tc_settle(const AttnParams& p, const TcRange& rg, TcWalk& w) {
  while (w.s < w.s1) {
    const int vis = tc_seg_vis(p, w.s, rg.max_pos);
    w.lo = max(0, rg.r0 - w.segstart);
    w.hi = min(vis, rg.r1 - w.segstart);
    if (w.lo < w.hi) {
      w.off = p.seg_offset[w.s];
      w.sl = (w.off + w.lo) & ~(TC_KEYS - 1);
      return true;
    }
    w.segstart += vis;
    ++w.s;
  }
  return false;
}

// Next tile; returns false when the walk is over.  *new_seg is set when the
// next tile belongs to a different segment than the current one.
BRAID_DEVICE bool tc_next(const AttnParams& p, const TcRange& rg, TcWalk& w, bool* new_seg) {
  w.sl += TC_KEYS;
  *new_seg = false;
  if (w.sl < w.off + w.hi) return true;
  w.segstart += tc_seg_vis(p, w.s, rg.max_pos);
  ++w.s;
  *new_seg = true;
  return tc_settle(p, rg, w);
}

// Rotated query row r (token tok, head) for a segment with RoPE delta `delta`,
// written into the K-major swizzled Q tile; rows past the tile are zero.  All
// 16 loads of the row are issued first and the cos/sin rows follow in two
// halves of 16 float4 loads each (about three memory round trips per row).
BRAID_DEVICE void tc_build_q_row(const AttnParams& p, uint8_t* qs, int r, bool live, int tok, int head, int rpos,
                                 int delta) {
  const __nv_bfloat16* qp = p.q + ((size_t)tok * p.Hq + head) * TC_D;
  uint4 qa[8], qb[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    qa[c] = live ? __ldg(reinterpret_cast<const uint4*>(qp + c * 8)) : make_uint4(0, 0, 0, 0);
    qb[c] = live ? __ldg(reinterpret_cast<const uint4*>(qp + 64 + c * 8)) : make_uint4(0, 0, 0, 0);
  }
  if (live && p.use_rope) {
    int pos = rpos - delta;
    pos = pos < 0 ? 0 : (pos >= p.rope_len ? p.rope_len - 1 : pos);
    const float4* cp = reinterpret_cast<const float4*>(p.cos + (size_t)pos * 64);
    const float4* sp = reinterpret_cast<const float4*>(p.sin + (size_t)pos * 64);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float4 cs[8], sn[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        cs[u] = __ldg(cp + hf * 8 + u);
        sn[u] = __ldg(sp + hf * 8 + u);
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c = hf * 4 + cc;
        const float cf[8] = {cs[2 * cc].x, cs[2 * cc].y, cs[2 * cc].z, cs[2 * cc].w,
                             cs[2 * cc + 1].x, cs[2 * cc + 1].y, cs[2 * cc + 1].z, cs[2 * cc + 1].w};
        const float sf[8] = {sn[2 * cc].x, sn[2 * cc].y, sn[2 * cc].z, sn[2 * cc].w,
                             sn[2 * cc + 1].x, sn[2 * cc + 1].y, sn[2 * cc + 1].z, sn[2 * cc + 1].w};
        const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&qa[c]);
        const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&qb[c]);
        uint4 o1, o2;
        __nv_bfloat16* y1 = reinterpret_cast<__nv_bfloat16*>(&o1);
        __nv_bfloat16* y2 = reinterpret_cast<__nv_bfloat16*>(&o2);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x1 = bf2f(a[e]), x2 = bf2f(bb[e]);
          y1[e] = f2bf(x1 * cf[e] - x2 * sf[e]);
          y2[e] = f2bf(x2 * cf[e] + x1 * sf[e]);
        }
        qa[c] = o1;
        qb[c] = o2;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    *reinterpret_cast<uint4*>(qs + tc_off(r, c)) = qa[c];
    *reinterpret_cast<uint4*>(qs + tc_off(r, c + 8)) = qb[c];
  }
}

// Barrier block of the kernel (8-byte mbarriers, then the TMEM address).
struct TcBars {
  uint64_t kfull[TC_STAGES], kempty[TC_STAGES];  // K tile landed / both S MMAs of it completed
  uint64_t vfull[TC_STAGES], vempty[TC_STAGES];  // V tile landed / both P V MMAs of it completed
  uint64_t sfull[TC_QT];                         // S(t, j) in TMEM (and every earlier MMA of the CTA done)
  uint64_t pready[TC_QT];                        // 128 arrivals: completion 0 = Q(t) built, j + 1 = P(t, j) in TMEM
  uint64_t odone[TC_QT];                         // the last P V of tile t completed
  uint32_t tmem;
};

// ex2.approx with flush-to-zero: the MUFU exponential, -inf -> 0.
BRAID_DEVICE float tc_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

static_assert(sizeof(TcBars) <= 256, "barrier block exceeds its shared-memory slot");
static_assert(TcSmem::TOTAL <= 227 * 1024, "shared memory per CTA");

// 2^x on the FMA and integer pipes, for the share of the softmax exponentials
// taken off the MUFU unit (16 per clock per SM, which at head_dim 128 is as
// slow as the tensor core): x = n + f with n = round(x) (the 1.5 * 2^23
// addition leaves n in the low mantissa bits) and f in [-0.5, 0.5];
// 2^f ~ c0 + c1 f + c2 f^2 + c3 f^3, coefficients fitted for this kernel by
// iteratively reweighted least squares on Chebyshev nodes (maximum relative
// error 7.5e-5, a 26th of a bf16 half-ulp); 2^n added to the exponent field.
// x < -126 (masked keys, -inf) gives exactly 0.
BRAID_DEVICE float tc_exp2_poly(float x) {
  const float xc = fmaxf(x, -126.f);
  const float t = xc + 12582912.f;
  const float f = xc - (t - 12582912.f);
  const float q = fmaf(fmaf(fmaf(0.0551716573f, f, 0.2426111400f), f, 0.6932609677f), f, 0.9999280572f);
  const float y = __int_as_float(__float_as_int(q) + ((__float_as_int(t) - 0x4B400000) << 23));
  return x < -126.f ? 0.f : y;
}

// POLY: every POLY-th exponential of a row runs tc_exp2_poly (0: none).
template <int BR, int POLY>
__global__ void __launch_bounds__(TC_THREADS, 1) attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmkv,
                                                                        const AttnParams p) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kst = sm + TcSmem::K;
  uint8_t* vst = sm + TcSmem::V;
  TcBars& bar = *reinterpret_cast<TcBars*>(sm + TcSmem::BAR);
  __shared__ int s_abort, s_last;

  const int S = p.num_splits;
  // Blocks are dispatched in linear order: the q tile is the slowest index
  // and runs backwards, so the CTAs with the most causal keys (late query
  // tiles of every head and sequence) start in the first wave and the short
  // ones fill the tail.
  const int yz = gridDim.y * gridDim.z;
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int qtile = gridDim.x - 1 - lin / yz;
  const int b = (lin % yz) % gridDim.y, z = (lin % yz) / gridDim.y;
  const int kh = z / S, split = z % S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // profiling (p.tc_trace): per CTA 128 timestamps; Q tile t at 64 t:
  // [2j] S(t, j) ready, [2j + 1] P(t, j) handed to the MMA warp (j < 30),
  // [60] Q(t) built; [61] S(0, 0) issued, [62] CTA start, [63] end,
  // [126] barriers and TMEM set up, [127] first K tile issued
  unsigned long long* trc = p.tc_trace ? p.tc_trace + (size_t)lin * 128 : nullptr;
  if (trc != nullptr && threadIdx.x == 0) trc[62] = globaltimer_ns();
  const int G = p.G;
  const int t0 = p.qo_indptr[b], nt = p.qo_indptr[b + 1] - t0;
  const int rows = nt * G;
  const int cta_rows = p.cta_rows == TC_ROWS ? TC_ROWS : TC_CTA_ROWS;
  const int row0 = qtile * cta_rows;
  if (row0 >= rows) return;
  const int nrows = min(cta_rows, rows - row0);
  const int nq = nrows > TC_ROWS ? 2 : 1;  // Q tiles with live rows (CTA-uniform)
  // largest position among the CTA's rows (rows of a shared-prefix group are not ordered)
  TcRange rg;
  {
    int mx = -(1 << 30);
    const int ta = t0 + row0 / G, tb = t0 + (row0 + nrows - 1) / G;
    for (int tk = ta + lane; tk <= tb; tk += 32) mx = max(mx, p.positions[tk]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    rg.max_pos = mx;
  }
  const int s0 = p.seg_indptr[b], s1 = p.seg_indptr[b + 1];
  rg.r0 = 0;
  rg.r1 = 1 << 30;
  if (S > 1) {
    int total = 0;
    for (int s = s0; s < s1; ++s) total += tc_seg_vis(p, s, rg.max_pos);
    const int per = ((total + S - 1) / S + TC_KEYS - 1) / TC_KEYS * TC_KEYS;
    rg.r0 = min(total, split * per);
    rg.r1 = min(total, rg.r0 + per);
  }
  if (threadIdx.x == 0) {
    span_start(p.span);
    tma_prefetch_desc(&tmkv);
    for (int i = 0; i < TC_STAGES; ++i) {
      mbar_init(&bar.kfull[i], 1);
      mbar_init(&bar.kempty[i], 1);
      mbar_init(&bar.vfull[i], 1);
      mbar_init(&bar.vempty[i], 1);
    }
    for (int t = 0; t < TC_QT; ++t) {
      mbar_init(&bar.sfull[t], 1);
      mbar_init(&bar.pready[t], 128);
      mbar_init(&bar.odone[t], 1);
    }
    fence_barrier_init();
    s_abort = 0;
  }
  if (warp == 1) {
    tmem_alloc(&bar.tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem;
  pdl_trigger();
  if (trc != nullptr && threadIdx.x == 0) trc[126] = globaltimer_ns();

  TcWalk w{s0, s1, 0, 0, 0, 0, 0};
  bool more = tc_settle(p, rg, w);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && more) {
      pdl_wait();
      span_waited(p.span);
      int j = 0, kiss = 0, viss = 0;
      while (more) {
        const int st = j % TC_STAGES;
        const uint32_t ph = ((j / TC_STAGES) & 1) ^ 1;
        const int* pages = p.page_ids + p.seg_page_indptr[w.s];
        const int npages = p.seg_page_indptr[w.s + 1] - p.seg_page_indptr[w.s];
        int rk[TC_KEYS / BR];
#pragma unroll
        for (int q = 0; q < TC_KEYS / BR; ++q) {
          const int slot = w.sl + q * BR;
          const int page = pages[min(slot / p.PS, npages - 1)];
          (void)BRAID_IN_BOUNDS(page >= 0 && page < p.num_pages, 4, page);  // TMA zero-fills outside the pool
          rk[q] = ((page * 2 + 0) * p.Hkv + kh) * p.PS + slot % p.PS;
        }
        if (j >= TC_STAGES && !mbar_wait(&bar.kempty[st], ph)) {
          s_abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&bar.kfull[st], TC_TILE);
#pragma unroll
        for (int q = 0; q < TC_KEYS / BR; ++q)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(kst + st * TC_TILE + h * TC_HALF + q * BR * 128, &tmkv, &bar.kfull[st], h * 64, rk[q]);
        if (trc != nullptr && j == 0) trc[127] = globaltimer_ns();
        ++kiss;
        if (j >= TC_STAGES && !mbar_wait(&bar.vempty[st], ph)) {
          s_abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&bar.vfull[st], TC_TILE);
#pragma unroll
        for (int q = 0; q < TC_KEYS / BR; ++q)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_2d(vst + st * TC_TILE + h * TC_HALF + q * BR * 128, &tmkv, &bar.vfull[st], h * 64,
                        rk[q] + p.Hkv * p.PS);
        ++viss;
        bool ns;
        more = tc_next(p, rg, w, &ns);
        ++j;
      }
      // every copy this CTA issued lands before the CTA can finish (a consumer
      // that gave up would otherwise leave copies in flight)
      for (int i = max(0, kiss - TC_STAGES); i < kiss; ++i)
        if (!mbar_wait(&bar.kfull[i % TC_STAGES], (i / TC_STAGES) & 1)) s_abort = 1;
      for (int i = max(0, viss - TC_STAGES); i < viss; ++i)
        if (!mbar_wait(&bar.vfull[i % TC_STAGES], (i / TC_STAGES) & 1)) s_abort = 1;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && more) {
      constexpr uint32_t idS = idesc_bf16_f32(TC_ROWS, TC_KEYS);
      constexpr uint32_t idPV = idesc_bf16_f32(TC_ROWS, TC_D) | (1u << 16);  // B (V) MN-major
      auto issue_s = [&](int t, int st) {
        const uint8_t* qs = sm + TcSmem::Q + t * TC_TILE;
#pragma unroll
        for (int k = 0; k < TC_D / 16; ++k) {
          const uint64_t a = smem_desc_sw128(smem_u32(qs + (k >> 2) * TC_HALF)) + 2 * (k & 3);
          const uint64_t bd = smem_desc_sw128(smem_u32(kst + st * TC_TILE + (k >> 2) * TC_HALF)) + 2 * (k & 3);
          tc_mma_bf16(tmem + t * TC_KEYS, a, bd, idS, k > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int st, bool acc) {
#pragma unroll
        for (int k = 0; k < TC_KEYS / 16; ++k) {
          const uint64_t bv = smem_desc_sw128_mn(smem_u32(vst + st * TC_TILE + k * 2048), TC_HALF, 1024);
          tc_mma_bf16_ta(tmem + 2 * TC_KEYS + t * TC_D, tmem + t * TC_KEYS + TC_P_COL + k * 8, bv, idPV,
                         (acc || k > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      for (int t = 0; t < nq && ok; ++t) ok = mbar_wait(&bar.pready[t], 0);  // Q tiles built
      ok = ok && mbar_wait(&bar.kfull[0], 0);
      if (ok) {
        tc_fence_after();
        if (trc != nullptr) trc[61] = globaltimer_ns();
        for (int t = 0; t < nq; ++t) {
          issue_s(t, 0);
          tc_commit(&bar.sfull[t]);
        }
        tc_commit(&bar.kempty[0]);
      }
      int j = 0;
      while (ok) {
        const int st = j % TC_STAGES, st1 = (j + 1) % TC_STAGES;
        bool ns;
        const bool nxt = tc_next(p, rg, w, &ns);
        if (!mbar_wait(&bar.vfull[st], (j / TC_STAGES) & 1)) {
          ok = false;
          break;
        }
        // tile t: P(t, j) V(j), then S(t, j + 1) into the same columns (the
        // MMAs of one thread execute in issue order)
        for (int t = 0; t < nq && ok; ++t) {
          if (!mbar_wait(&bar.pready[t], (j + 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, st, j > 0);
          if (nxt) {
            if (t == 0 && !mbar_wait(&bar.kfull[st1], ((j + 1) / TC_STAGES) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(t, st1);
            tc_commit(&bar.sfull[t]);
          } else {
            tc_commit(&bar.odone[t]);
          }
        }
        if (!ok) break;
        tc_commit(&bar.vempty[st]);
        if (!nxt) break;
        tc_commit(&bar.kempty[st1]);
        ++j;
      }
      if (!ok) s_abort = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 2) >> 2;  // Q tile of this warpgroup
    if (t < nq) {
      const int q4 = warp & 3;        // TMEM lane quarter this warp may access
      const int r = q4 * 32 + lane;   // row within the Q tile = TMEM lane
      const int rr = row0 + t * TC_ROWS + r;
      const bool live = rr < rows;
      const int tok = t0 + (live ? rr / G : 0), head = kh * G + (live ? rr % G : 0);
      const int rpos = live ? p.positions[tok] : -1;
      const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
      const uint32_t tS = tmem + lane_off + t * TC_KEYS;
      const uint32_t tO = tmem + lane_off + 2 * TC_KEYS + t * TC_D;
      uint8_t* qs = sm + TcSmem::Q + t * TC_TILE;
      const float sl2 = p.scale_log2;
      float m_run = -INFINITY, l_run = 0.f;
      int j = 0;
      if (more) {
        const int delta0 = p.seg_delta[w.s];
        pdl_wait();
        tc_build_q_row(p, qs, r, live, tok, head, rpos, delta0);
        fence_proxy_async_smem();
        mbar_arrive(&bar.pready[t]);
        if (trc != nullptr && r == 0) trc[t * 64 + 60] = globaltimer_ns();
      }
      while (more) {
        const int pos0 = p.seg_pos0[w.s], j0 = w.sl - w.off, lo = w.lo, hi = w.hi;
        if (!mbar_wait(&bar.sfull[t], j & 1)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        if (trc != nullptr && r == 0 && j < 30) trc[t * 64 + 2 * j] = globaltimer_ns();
        uint32_t sr[TC_KEYS];
#pragma unroll
        for (int c = 0; c < TC_KEYS / 32; ++c) tmem_ld32(tS + c * 32, sr + c * 32);
        tc_wait_ld();
        // keys outside [lo, hi) of the segment, or after the row's position,
        // are masked; interior tiles (every key visible to this row) skip it
        if (live && !(j0 >= lo && j0 + TC_KEYS <= hi && pos0 + j0 + TC_KEYS - 1 <= rpos)) {
#pragma unroll
          for (int i = 0; i < TC_KEYS; ++i) {
            const int key = j0 + i;
            if (!(key >= lo && key < hi && pos0 + key <= rpos)) sr[i] = __float_as_uint(-INFINITY);
          }
        }
        // eight independent partial maxima (a 128-long dependent chain otherwise)
        float m8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) m8[u] = __uint_as_float(sr[u]);
#pragma unroll
        for (int i = 8; i < TC_KEYS; ++i) m8[i & 7] = fmaxf(m8[i & 7], __uint_as_float(sr[i]));
        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                               fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        // running maximum (base 2) moves only when the tile's exceeds it by
        // more than 8: P <= 2^8 stays exact enough in bf16 and fp32 sums, and
        // O in TMEM is rescaled rarely
        const float m_new = fmaxf(m_run, mx * sl2);
        const bool resc = m_new > m_run + 8.f;
        const float alpha = resc ? tc_ex2(m_run - m_new) : 1.f;
        if (resc) {
          l_run *= alpha;
          m_run = m_new;
        }
        const float mneg = m_run == -INFINITY ? 0.f : -m_run;
        float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < TC_KEYS / 2; ++i) {
          const float x0 = fmaf(__uint_as_float(sr[2 * i]), sl2, mneg);
          const float x1 = fmaf(__uint_as_float(sr[2 * i + 1]), sl2, mneg);
          const float e0 = (POLY > 0 && (2 * i) % POLY == POLY - 1) ? tc_exp2_poly(x0) : tc_ex2(x0);
          const float e1 = (POLY > 0 && (2 * i + 1) % POLY == POLY - 1) ? tc_exp2_poly(x1) : tc_ex2(x1);
          l8[i & 7] += e0 + e1;
          sr[i] = pack_bf16(e0, e1);
        }
        l_run += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
        // P(t, j) as bf16 pairs into columns [TC_P_COL, TC_P_COL + 64) of S(t)
        tmem_st32(tS + TC_P_COL, sr);
        tmem_st32(tS + TC_P_COL + 32, sr + 32);
        if (__any_sync(0xffffffffu, resc && j > 0)) {
          // O(t) holds P V of tiles < j (complete: S(t, j) was issued after
          // them) and P(t, j) V is not issued before this thread's arrival
#pragma unroll 1
          for (int c = 0; c < TC_D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
        }
        tc_wait_st();
        bool ns;
        more = tc_next(p, rg, w, &ns);
        // S(t, j) is consumed and S(t, j + 1) waits for this arrival: the next
        // segment's rotated queries can replace the Q tile now
        if (more && ns) tc_build_q_row(p, qs, r, live, tok, head, rpos, p.seg_delta[w.s]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bar.pready[t]);
        if (trc != nullptr && r == 0 && j < 30) trc[t * 64 + 2 * j + 1] = globaltimer_ns();
        ++j;
      }
      const bool have = j > 0 && !s_abort;
      if (have && !mbar_wait(&bar.odone[t], 0)) s_abort = 1;
      tc_fence_after();
      // ------------------------------------------------------------ output
      const bool direct = S == 1 && !p.partial_only;
      const int stride = p.split_stride > 0 ? p.split_stride : S;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const size_t idx = ((size_t)tok * p.Hq + head) * stride + p.split_base + split;
#pragma unroll 1
      for (int c = 0; c < TC_D / 32; ++c) {
        uint32_t o[32];
        if (have) {
          tmem_ld32(tO + c * 32, o);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (!live || s_abort) continue;
        if (direct) {
          __nv_bfloat16* out = p.out + ((size_t)tok * p.Hq + head) * TC_D + c * 32;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(out + u * 8) = make_uint4(
                pack_bf16(__uint_as_float(o[8 * u]) * inv, __uint_as_float(o[8 * u + 1]) * inv),
                pack_bf16(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv),
                pack_bf16(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv),
                pack_bf16(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv));
        } else {
          float* po = p.part_o + idx * TC_D + c * 32;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(po + 4 * u) =
                make_float4(__uint_as_float(o[4 * u]) * inv, __uint_as_float(o[4 * u + 1]) * inv,
                            __uint_as_float(o[4 * u + 2]) * inv, __uint_as_float(o[4 * u + 3]) * inv);
        }
      }
      if (live && !s_abort && !direct) p.part_lse[idx] = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
      if (!direct && !p.partial_only) {
        // the last split CTA of this q tile merges every split's partial
        named_bar_sync(1, 128 * nq);
        if (threadIdx.x == 64) {
          int* ctr = p.counters + ((size_t)b * p.Hkv + kh) * gridDim.x + qtile;
          const int old = atomic_add_acq_rel_gpu(ctr, 1);  // releases this CTA's partials, acquires the others'
          s_last = old == S - 1;
          if (s_last) *ctr = 0;
        }
        named_bar_sync(1, 128 * nq);
        if (s_last && live) {
          const size_t base = ((size_t)tok * p.Hq + head) * stride;
          float wq[32];
          float mxl = -INFINITY;
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            wq[q] = q < S ? __ldcg(p.part_lse + base + q) : -INFINITY;
            mxl = fmaxf(mxl, wq[q]);
          }
          float sum = 0.f;
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            wq[q] = (mxl == -INFINITY || wq[q] == -INFINITY) ? 0.f : exp2f(wq[q] - mxl);
            sum += wq[q];
          }
          const float winv = sum > 0.f ? 1.f / sum : 0.f;
          __nv_bfloat16* o = p.out + ((size_t)tok * p.Hq + head) * TC_D;
          for (int d = 0; d < TC_D; d += 8) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int q0 = 0; q0 < S; q0 += 8) {
              // eight splits' partials of these 8 dims in flight before any is summed
              float4 v[8][2];
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const bool use = q0 + u < S;
                const float4* src = reinterpret_cast<const float4*>(p.part_o + (base + q0 + u) * TC_D + d);
                v[u][0] = use ? __ldcg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
                v[u][1] = use ? __ldcg(src + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const float wu = q0 + u < S ? wq[q0 + u] : 0.f;
                acc[0] += wu * v[u][0].x; acc[1] += wu * v[u][0].y; acc[2] += wu * v[u][0].z; acc[3] += wu * v[u][0].w;
                acc[4] += wu * v[u][1].x; acc[5] += wu * v[u][1].y; acc[6] += wu * v[u][1].z; acc[7] += wu * v[u][1].w;
              }
            }
            *reinterpret_cast<uint4*>(o + d) =
                make_uint4(pack_bf16(acc[0] * winv, acc[1] * winv), pack_bf16(acc[2] * winv, acc[3] * winv),
                           pack_bf16(acc[4] * winv, acc[5] * winv), pack_bf16(acc[6] * winv, acc[7] * winv));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (trc != nullptr && threadIdx.x == 0) trc[63] = globaltimer_ns();
  if (threadIdx.x == 0) span_end(p.span);
}

}  // namespace braid

namespace braid {

CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);

// Prefill kernel choice for head_dim 128.  Mode 1 always takes this kernel,
// 0 the mma.sync kernel of attention.cu, -1 (auto) this kernel for prefill
// calls of at least 1024 (token, head) rows: on B200 it runs 2.2-2.9x faster
// there (2048 causal: 59 vs 170 us; 256 queries over 7000 cached keys: 79 vs
// 174 us), while for a short query over a long cached context and for the
// shared-prefix pass of a grouped decode step (256 rows and fewer) the
// mma.sync kernel's 64-row tiles spread the keys over more SMs (64 queries
// over 3200 keys: 35 vs 50 us).  Mode: attn_select_prefill_tc, else
// BRAID_ATTN_TC (1 / 0), else auto.
static int g_attn_tc = -1;

void attn_select_prefill_tc(int64_t mode) { g_attn_tc = mode < 0 ? -1 : (mode ? 1 : 0); }

static int attn_tc_mode() {
  static const int env_mode = [] {
    const char* e = getenv("BRAID_ATTN_TC");
    return e == nullptr ? -1 : (e[0] == '1' ? 1 : 0);
  }();
  return g_attn_tc >= 0 ? g_attn_tc : env_mode;
}

// Prefill call of `rows` (token, head) rows with head dim D.
bool attn_prefill_tc_use(int D, int64_t rows) {
  if (D != TC_D) return false;
  const int m = attn_tc_mode();
  return m == 1 || (m < 0 && rows >= 1024);
}

// Shared-prefix pass of a grouped decode step.
bool attn_shared_tc_use(int D) { return D == TC_D && attn_tc_mode() == 1; }

// Share of the tcgen05 prefill softmax exponentials computed by polynomial
// (every n-th of a row; 0 none; -1 follows BRAID_ATTN_POLY); 256-token pages.
static int g_attn_poly = -1;
void attn_set_exp2_poly(int64_t n) { g_attn_poly = n < 0 ? -1 : (n == 2 || n == 4 ? (int)n : 0); }

int attn_prefill_tc_rows() { return TC_CTA_ROWS; }
int attn_prefill_tc_min_rows() { return TC_ROWS; }

// Query rows per CTA of the kernel that runs the shared-prefix pass of a
// grouped decode step for head_dim D (the tcgen05 kernel holds one CTA per
// SM, the mma.sync kernel two).
int64_t attn_prefill_tile_rows(int64_t D) { return attn_shared_tc_use((int)D) ? TC_CTA_ROWS : 64; }

void launch_attn_prefill_tc(const AttnParams& p, int num_seqs, int max_q_len, int64_t P, cudaStream_t st) {
  const int64_t rows = P * 2 * p.Hkv * p.PS;  // the layer pool as rows of head_dim elements
  const int cr = p.cta_rows == TC_ROWS ? TC_ROWS : TC_CTA_ROWS;
  const int qt = (max_q_len * p.G + cr - 1) / cr;
  const dim3 grid(qt, num_seqs, p.Hkv * p.num_splits);
  static const int env_poly = [] {  // tuning knob: BRAID_ATTN_POLY = 0, 2 or 4
    const char* e = getenv("BRAID_ATTN_POLY");
    return e ? atoi(e) : 0;
  }();
  const int poly = g_attn_poly >= 0 ? g_attn_poly : env_poly;
  auto go = [&](auto k, int br) {
    static bool attr[8] = {};
    const int slot = (br == 64 ? 4 : 0) + (poly == 2 ? 1 : poly == 4 ? 2 : 0);
    if (!attr[slot]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::TOTAL));
      attr[slot] = true;
    }
    launch_pdl(k, grid, dim3(TC_THREADS), TcSmem::TOTAL, st, make_tmap(p.kv, rows, TC_D, TC_D, br), p);
  };
  if (p.PS % 64 == 0) {
    if (poly == 2)
      go(attn_prefill_tc_kernel<64, 2>, 64);
    else if (poly == 4)
      go(attn_prefill_tc_kernel<64, 4>, 64);
    else
      go(attn_prefill_tc_kernel<64, 0>, 64);
  } else {
    go(attn_prefill_tc_kernel<16, 0>, 16);
  }
}

}  // namespace braid

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_attention_tc)
}  // namespace braid
