// tcgen05 prefill attention for sm_100a (head_dim 128): the tensor-core path
// of paged cascade attention for prefill-shaped work — chunk self-prefill,
// a request's prompt over cached chunks, and the shared-prefix pass of a
// batched decode step.
//
// One CTA owns 128 query rows, each a (token, head-of-the-KV-group) pair of
// one sequence (or of one shared-prefix group), against one KV head:
//   warp 0      TMA producer: 128-key K and V tiles of the paged KV cache
//               (128-byte swizzle) into a 2-stage mbarrier ring
//   warp 1      MMA issuer (one elected lane):
//                 S = Q K^T   M=128, N=128 keys, K=128 dims -> TMEM cols [0,128)
//                 O_t = P V   M=128, N=128 dims, K=128 keys -> TMEM cols [128,256)
//               (V is read as an MN-major operand: the cache stores keys as rows)
//   warps 2..5  one query row per thread (TMEM lane): build the rotated query
//               tile (differential RoPE per segment), online softmax in base 2
//               on S read with tcgen05.ld, P written to shared memory as bf16
//               (K-major, 128-byte swizzle), O accumulated in registers from
//               each O_t, then the output or the split partial.
// Per tile j: S(j) -> softmax(j) (waits O_t(j-1), rescales O, writes P(j)) ->
// P V(j) issued together with S(j+1).
//
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

constexpr int TC_D = 128;       // head dim
constexpr int TC_ROWS = 128;    // query rows per CTA (MMA M)
constexpr int TC_KEYS = 128;    // keys per tile (MMA N of S, K of P V)
constexpr int TC_STAGES = 2;    // K/V ring depth
constexpr int TC_HALF = TC_KEYS * 128;  // bytes of one 64-column half of a 128-row bf16 tile (16 KB)
constexpr int TC_TILE = 2 * TC_HALF;    // one 128 x 128 bf16 tile (32 KB)

struct TcSmem {
  static constexpr int Q = 0;                              // [2 halves][128 rows][128 B]
  static constexpr int P = Q + TC_TILE;                    // [2 key halves][128 rows][128 B]
  static constexpr int K = P + TC_TILE;                    // [stage][2 dim halves][128 keys][128 B]
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
// written into the K-major swizzled Q tile; rows past the tile are zero.
BRAID_DEVICE void tc_build_q_row(const AttnParams& p, uint8_t* qs, int r, bool live, int tok, int head, int rpos,
                                 int delta) {
  const __nv_bfloat16* qp = p.q + ((size_t)tok * p.Hq + head) * TC_D;
  int pos = rpos - delta;
  pos = pos < 0 ? 0 : (pos >= p.rope_len ? p.rope_len - 1 : pos);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 o1 = make_uint4(0, 0, 0, 0), o2 = make_uint4(0, 0, 0, 0);
    if (live) {
      const uint4 a4 = *reinterpret_cast<const uint4*>(qp + c * 8);
      const uint4 b4 = *reinterpret_cast<const uint4*>(qp + 64 + c * 8);
      if (p.use_rope) {
        const float* cp = p.cos + (size_t)pos * 64 + c * 8;
        const float* sp = p.sin + (size_t)pos * 64 + c * 8;
        const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&a4);
        const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&b4);
        __nv_bfloat16* y1 = reinterpret_cast<__nv_bfloat16*>(&o1);
        __nv_bfloat16* y2 = reinterpret_cast<__nv_bfloat16*>(&o2);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float x1 = bf2f(a[e]), x2 = bf2f(bb[e]), cs = cp[e], sn = sp[e];
          y1[e] = f2bf(x1 * cs - x2 * sn);
          y2[e] = f2bf(x2 * cs + x1 * sn);
        }
      } else {
        o1 = a4;
        o2 = b4;
      }
    }
    *reinterpret_cast<uint4*>(qs + tc_off(r, c)) = o1;
    *reinterpret_cast<uint4*>(qs + tc_off(r, c + 8)) = o2;
  }
}

template <int BR>
__global__ void __launch_bounds__(192, 1) attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmkv,
                                                                 const AttnParams p) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = sm + TcSmem::Q;
  uint8_t* ps = sm + TcSmem::P;
  uint8_t* kst = sm + TcSmem::K;
  uint8_t* vst = sm + TcSmem::V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + TcSmem::BAR);
  uint64_t* kfull = bars;                 // [TC_STAGES]: K and V of a tile landed
  uint64_t* kempty = bars + TC_STAGES;    // [TC_STAGES]: the P V of that tile completed
  uint64_t* s_full = bars + 2 * TC_STAGES;
  uint64_t* o_full = s_full + 1;
  uint64_t* pq = s_full + 2;              // 128 arrivals: completion 0 = Q tile, j + 1 = P(j)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 3);
  __shared__ int s_abort, s_last;

  const int S = p.num_splits;
  const int b = blockIdx.y, kh = blockIdx.z / S, split = blockIdx.z % S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G;
  const int t0 = p.qo_indptr[b], nt = p.qo_indptr[b + 1] - t0;
  const int rows = nt * G;
  const int row0 = blockIdx.x * TC_ROWS;
  if (row0 >= rows) return;
  const int nrows = min(TC_ROWS, rows - row0);
  // positions of the tile's rows (not ordered by row for shared-prefix groups)
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
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(o_full, 1);
    mbar_init(pq, 128);
    fence_barrier_init();
    s_abort = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_trigger();

  TcWalk w{s0, s1, 0, 0, 0, 0, 0};
  bool more = tc_settle(p, rg, w);
  // softmax warps: one query row per thread, the row's TMEM lane
  const int q4 = warp & 3;
  const int r = q4 * 32 + lane;
  const int rr = row0 + r;
  const bool live = warp >= 2 && r < nrows;
  const int tok = t0 + (live ? rr / G : 0), head = kh * G + (live ? rr % G : 0);
  const int rpos = live ? p.positions[tok] : -1;
  const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
  float O[TC_D];
#pragma unroll
  for (int d = 0; d < TC_D; ++d) O[d] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && more) {
      pdl_wait();
      int j = 0;
      while (more) {
        const int st = j % TC_STAGES;
        if (j >= TC_STAGES && !mbar_wait(&kempty[st], ((j / TC_STAGES) & 1) ^ 1)) {
          s_abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&kfull[st], 2 * TC_TILE);
        const int* pages = p.page_ids + p.seg_page_indptr[w.s];
        const int npages = p.seg_page_indptr[w.s + 1] - p.seg_page_indptr[w.s];
#pragma unroll
        for (int q = 0; q < TC_KEYS / BR; ++q) {
          const int slot = w.sl + q * BR;
          const int page = pages[min(slot / p.PS, npages - 1)];
          const int row_k = ((page * 2 + 0) * p.Hkv + kh) * p.PS + slot % p.PS;
          const int row_v = row_k + p.Hkv * p.PS;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tma_load_2d(kst + st * TC_TILE + h * TC_HALF + q * BR * 128, &tmkv, &kfull[st], h * 64, row_k);
            tma_load_2d(vst + st * TC_TILE + h * TC_HALF + q * BR * 128, &tmkv, &kfull[st], h * 64, row_v);
          }
        }
        bool ns;
        more = tc_next(p, rg, w, &ns);
        ++j;
      }
      // every copy this CTA issued has landed before the CTA can finish (a
      // consumer that gave up would otherwise leave copies in flight)
      for (int i = max(0, j - TC_STAGES); i < j; ++i)
        if (!mbar_wait(&kfull[i % TC_STAGES], (i / TC_STAGES) & 1)) s_abort = 1;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && more) {
      constexpr uint32_t idS = idesc_bf16_f32(TC_ROWS, TC_KEYS);
      constexpr uint32_t idPV = idesc_bf16_f32(TC_ROWS, TC_D) | (1u << 16);  // B (V) MN-major
      int j = 0;
      bool ok = mbar_wait(pq, 0);  // Q tile written
      while (more && ok) {
        const int st = j % TC_STAGES;
        if (!mbar_wait(&kfull[st], (j / TC_STAGES) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < TC_D / 16; ++k) {
          const uint64_t a = smem_desc_sw128(smem_u32(qs + (k >> 2) * TC_HALF)) + 2 * (k & 3);
          const uint64_t bd = smem_desc_sw128(smem_u32(kst + st * TC_TILE + (k >> 2) * TC_HALF)) + 2 * (k & 3);
          tc_mma_bf16(tmem, a, bd, idS, k > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        if (!mbar_wait(pq, (j + 1) & 1)) {  // P(j) written (and Q rebuilt for the next segment)
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < TC_KEYS / 16; ++k) {
          const uint64_t a = smem_desc_sw128(smem_u32(ps + (k >> 2) * TC_HALF)) + 2 * (k & 3);
          const uint64_t bv = smem_desc_sw128_mn(smem_u32(vst + st * TC_TILE + k * 2048), TC_HALF, 1024);
          tc_mma_bf16(tmem + TC_KEYS, a, bv, idPV, k > 0 ? 1u : 0u);
        }
        tc_commit(o_full);
        tc_commit(&kempty[st]);
        bool ns;
        more = tc_next(p, rg, w, &ns);
        ++j;
      }
      if (!ok) s_abort = 1;
    }
  } else if (more) {
    // ------------------------------------------------------------ softmax
    pdl_wait();
    tc_build_q_row(p, qs, r, live, tok, head, rpos, p.seg_delta[w.s]);
    fence_proxy_async_smem();
    mbar_arrive(pq);
    int j = 0;
    while (more) {
      const int pos0 = p.seg_pos0[w.s], j0 = w.sl - w.off, lo = w.lo, hi = w.hi;
      if (!mbar_wait(s_full, j & 1)) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      // pass 1: this tile's row maximum over visible keys (base-2 scaled logits)
      float mx = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < TC_KEYS; c0 += 16) {
        float v[16];
        tmem_ld16(trow + c0, v);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = j0 + c0 + i;
          if (live && key >= lo && key < hi && pos0 + key <= rpos) mx = fmaxf(mx, v[i] * p.scale_log2);
        }
      }
      const float m_new = fmaxf(m_run, mx);
      // O_t(j-1) = P(j-1) V(j-1) is relative to m_run: add it, then rescale to m_new
      if (j > 0) {
        if (!mbar_wait(o_full, (j - 1) & 1)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < TC_D; c0 += 16) {
          float v[16];
          tmem_ld16(trow + TC_KEYS + c0, v);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) O[c0 + i] += v[i];
        }
      }
      const float alpha = (m_run == -INFINITY || m_new == -INFINITY) ? 1.f : exp2f(m_run - m_new);
#pragma unroll
      for (int d = 0; d < TC_D; ++d) O[d] *= alpha;
      l_run *= alpha;
      // pass 2: P(j) = exp2(s - m_new) as bf16 into the swizzled P tile
#pragma unroll
      for (int c0 = 0; c0 < TC_KEYS; c0 += 16) {
        float v[16];
        tmem_ld16(trow + c0, v);
        tc_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float e[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int key = j0 + c0 + i + u;
            const bool vis = live && key >= lo && key < hi && pos0 + key <= rpos && m_new != -INFINITY;
            e[u] = vis ? exp2f(v[i + u] * p.scale_log2 - m_new) : 0.f;
          }
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(e[0], e[1]);
          // the sum uses the rounded values the tensor core multiplies
          l_run += __low2float(h2) + __high2float(h2);
          pk[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
        }
#pragma unroll
        for (int c = 0; c < 2; ++c)
          *reinterpret_cast<uint4*>(ps + tc_off(r, c0 / 8 + c)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      m_run = m_new;
      bool ns;
      more = tc_next(p, rg, w, &ns);
      // S(j) is consumed and S(j+1) is not issued before this arrival: the
      // next segment's rotated queries can replace the Q tile now
      if (more && ns) tc_build_q_row(p, qs, r, live, tok, head, rpos, p.seg_delta[w.s]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pq);
      ++j;
    }
    // the last tile's P V
    if (j > 0 && !s_abort) {
      if (mbar_wait(o_full, (j - 1) & 1)) {
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < TC_D; c0 += 16) {
          float v[16];
          tmem_ld16(trow + TC_KEYS + c0, v);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) O[c0 + i] += v[i];
        }
      } else {
        s_abort = 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
  if (warp >= 2) {
    // ------------------------------------------------------------ output
    const bool direct = S == 1 && !p.partial_only;
    const int stride = p.split_stride > 0 ? p.split_stride : S;
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    if (live && !s_abort) {
      if (direct) {
        __nv_bfloat16* o = p.out + ((size_t)tok * p.Hq + head) * TC_D;
#pragma unroll
        for (int c = 0; c < TC_D / 8; ++c) {
          uint32_t pk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(O[c * 8 + 2 * u] * inv, O[c * 8 + 2 * u + 1] * inv);
            pk[u] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(o + c * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      } else {
        const size_t idx = ((size_t)tok * p.Hq + head) * stride + p.split_base + split;
        float* po = p.part_o + idx * TC_D;
#pragma unroll
        for (int d = 0; d < TC_D; d += 4)
          *reinterpret_cast<float4*>(po + d) = make_float4(O[d] * inv, O[d + 1] * inv, O[d + 2] * inv, O[d + 3] * inv);
        p.part_lse[idx] = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
      }
    }
    if (!direct && !p.partial_only) {
      // the last split CTA of this q tile merges every split's partial
      named_bar_sync(1, 128);
      if (threadIdx.x == 64) {
        int* ctr = p.counters + ((size_t)b * p.Hkv + kh) * gridDim.x + blockIdx.x;
        const int old = atomic_add_acq_rel_gpu(ctr, 1);  // releases this CTA's partials, acquires the others'
        s_last = old == S - 1;
        if (s_last) *ctr = 0;
      }
      named_bar_sync(1, 128);
      if (s_last && live) {
        const size_t base = ((size_t)tok * p.Hq + head) * stride;
        float wq[32];
        float mx = -INFINITY;
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          wq[q] = q < S ? __ldcg(p.part_lse + base + q) : -INFINITY;
          mx = fmaxf(mx, wq[q]);
        }
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          wq[q] = (mx == -INFINITY || wq[q] == -INFINITY) ? 0.f : exp2f(wq[q] - mx);
          sum += wq[q];
        }
        const float winv = sum > 0.f ? 1.f / sum : 0.f;
        __nv_bfloat16* o = p.out + ((size_t)tok * p.Hq + head) * TC_D;
        for (int d = 0; d < TC_D; d += 4) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q = 0; q < S; ++q) {
            if (wq[q] == 0.f) continue;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(p.part_o + (base + q) * TC_D + d));
            acc.x += wq[q] * v.x;
            acc.y += wq[q] * v.y;
            acc.z += wq[q] * v.z;
            acc.w += wq[q] * v.w;
          }
          *reinterpret_cast<__nv_bfloat162*>(o + d) = __floats2bfloat162_rn(acc.x * winv, acc.y * winv);
          *reinterpret_cast<__nv_bfloat162*>(o + d + 2) = __floats2bfloat162_rn(acc.z * winv, acc.w * winv);
        }
      }
    }
  }
  if (threadIdx.x == 0) span_end(p.span);
}

}  // namespace braid

namespace braid {

CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);

// tcgen05 prefill for head_dim 128 (BRAID_ATTN_TC=0 keeps the mma.sync
// kernel).  Measured on B200, L = 2048 causal, 32 q / 8 KV heads: 170 us
// against 356 us for the mma.sync kernel.
bool attn_prefill_tc_enabled(int D) {
  static const bool on = [] {
    const char* e = getenv("BRAID_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  return on && D == TC_D;
}

int attn_prefill_tc_rows() { return TC_ROWS; }

void launch_attn_prefill_tc(const AttnParams& p, int num_seqs, int max_q_len, int64_t P, cudaStream_t st) {
  const int64_t rows = P * 2 * p.Hkv * p.PS;  // the layer pool as rows of head_dim elements
  const int qt = (max_q_len * p.G + TC_ROWS - 1) / TC_ROWS;
  const dim3 grid(qt, num_seqs, p.Hkv * p.num_splits);
  if (p.PS % 64 == 0) {
    auto k = attn_prefill_tc_kernel<64>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::TOTAL));
      attr = true;
    }
    launch_pdl(k, grid, dim3(192), TcSmem::TOTAL, st, make_tmap(p.kv, rows, TC_D, TC_D, 64), p);
  } else {
    auto k = attn_prefill_tc_kernel<16>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::TOTAL));
      attr = true;
    }
    launch_pdl(k, grid, dim3(192), TcSmem::TOTAL, st, make_tmap(p.kv, rows, TC_D, TC_D, 16), p);
  }
}

}  // namespace braid
