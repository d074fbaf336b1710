// Paged cascade attention for sm_100a (decode and prefill), GQA, query-side
// differential RoPE, fp32 online softmax.
//
// A sequence attends to an ordered list of KV segments (cached chunks, then
// its private pages).  Segment s holds seg_len[s] keys starting at slot
// seg_offset[s] of its first page; its first key sits at global position
// seg_pos0[s] and was rotated when cached at seg_pos0[s] - seg_delta[s].  The
// query (stored unrotated) is rotated by (p - seg_delta[s]) for segment s,
// which equals rotating every cached key to its composed position.  Key j of
// segment s is visible to a query at position p iff seg_pos0[s] + j <= p.
//
// Replaces the reference's cascade loop (braidinfer/layers/cascade_attention.py:50-231),
// which launched one Triton online-softmax program per page per chunk per
// layer (braidinfer/kernels/online_softmax.py, a scalar per-token loop), and
// its standard path's torch.cat of every past page (braidinfer/layers/attention.py:55-124).
//
// Tensor-core path: mma.sync m16n8k16 (bf16 in, fp32 accumulate), K/V tiles of
// 64 keys staged with cp.async into XOR-swizzled shared memory, ldmatrix
// fragments.  Rows of the Q tile are (query token, head-in-KV-group) pairs, so
// one K/V tile serves every query head that shares the KV head.
//   decode  : grid (seq, kv_head, split); the 4 warps split each 64-key tile,
//             partial states merged in shared memory; with several splits the
//             last-arriving split CTA of a (token, kv head) merges all splits
//             (log-sum-exp weights) from a fp32 scratch, so no merge launch.
//   prefill : grid (64-row q tile, seq, kv_head); each warp owns 16 rows and
//             walks every tile; key tiles beyond the tile's last query
//             position are skipped.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"
#include "tmap.h"
#include "attention_types.cuh"

#include <mutex>
#include <unordered_map>

namespace braid {


// byte offset of 16-byte chunk c of row r in a swizzled [rows x D] bf16 tile
template <int D>
BRAID_DEVICE uint32_t swz(int r, int c) {
  return (uint32_t)(r * D * 2 + ((c ^ (r & 7)) << 4));
}

BRAID_DEVICE size_t kv_row(const AttnParams& p, int page, int kv, int kh, int slot, int D) {
  return ((((size_t)page * 2 + kv) * p.Hkv + kh) * p.PS + slot) * (size_t)D;
}

// Stage rows [0, nrows) of a 64-key K and V tile of segment s (keys j0..j0+63).
template <int D>
BRAID_DEVICE void load_kv_tile(const AttnParams& p, int s, int kh, int j0, int jend, uint8_t* ks, uint8_t* vs) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  const int off = p.seg_offset[s];
  const int* pages = p.page_ids + p.seg_page_indptr[s];
  for (int i = threadIdx.x; i < KT * CH; i += blockDim.x) {
    const int row = i / CH, c = i % CH;
    const int j = j0 + row;
    bool ok = j < jend;
    const __nv_bfloat16* kp = p.kv;
    const __nv_bfloat16* vp = p.kv;
    if (ok) {
      const int slot = off + j;
      const int page = pages[slot / p.PS];
      if (BRAID_IN_BOUNDS(page >= 0 && page < p.num_pages, 4, page)) {
        kp = p.kv + kv_row(p, page, 0, kh, slot % p.PS, D) + c * 8;
        vp = p.kv + kv_row(p, page, 1, kh, slot % p.PS, D) + c * 8;
      } else {
        ok = false;  // zero-filled
      }
    }
    cp_async16(smem_u32(ks) + swz<D>(row, c), kp, ok);
    cp_async16(smem_u32(vs) + swz<D>(row, c), vp, ok);
  }
}

// Rotate (or copy) query rows into a swizzled bf16 tile.  Row r of the tile is
// (token tok_of(r), head kh*G + g_of(r)); rows beyond nrows are zero.
template <int D, typename RowFn>
BRAID_DEVICE void build_q_tile(const AttnParams& p, int kh, int delta, int nrows, int tile_rows, uint8_t* qs,
                               RowFn row_tok) {
  constexpr int H2 = D / 2;
  for (int i = threadIdx.x; i < tile_rows * H2; i += blockDim.x) {
    const int r = i / H2, d = i % H2;
    float x1 = 0.f, x2 = 0.f;
    if (r < nrows) {
      int tok, g;
      row_tok(r, tok, g);
      const __nv_bfloat16* qp = p.q + ((size_t)tok * p.Hq + kh * p.G + g) * D;
      float a = bf2f(qp[d]), b = bf2f(qp[d + H2]);
      if (p.use_rope) {
        int pos = p.positions[tok] - delta;
        pos = pos < 0 ? 0 : (pos >= p.rope_len ? p.rope_len - 1 : pos);
        const float cs = p.cos[(size_t)pos * H2 + d], sn = p.sin[(size_t)pos * H2 + d];
        x1 = a * cs - b * sn;
        x2 = b * cs + a * sn;
      } else {
        x1 = a;
        x2 = b;
      }
    }
    __nv_bfloat16* t = reinterpret_cast<__nv_bfloat16*>(qs);
    t[(swz<D>(r, d / 8) >> 1) + (d & 7)] = f2bf(x1);
    t[(swz<D>(r, (d + H2) / 8) >> 1) + ((d + H2) & 7)] = f2bf(x2);
  }
}

// Load the A fragments of a 16-row Q slab (rows rbase..rbase+15) for all D/16 k-steps.
template <int D>
BRAID_DEVICE void load_q_frags(const uint8_t* qs, int rbase, uint32_t (*qf)[4]) {
  const int lane = threadIdx.x & 31;
  const int r = rbase + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int c = kk * 2 + (lane >> 4);
    ldsm_x4(smem_u32(qs) + swz<D>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }
}

// S[16 x 8*NB] = Q(16 x D) * K(keys kbase.. kbase+8*NB)^T
template <int D, int NB>
BRAID_DEVICE void qk_tile(const uint32_t (*qf)[4], const uint8_t* ks, int kbase, float (*s)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; kk += 2) {
      uint32_t b0, b1, b2, b3;
      const int row = kbase + nb * 8 + (lane & 7);
      const int c = kk * 2 + (lane >> 3);
      ldsm_x4(smem_u32(ks) + swz<D>(row, c), b0, b1, b2, b3);
      mma16816(s[nb], qf[kk], b0, b1);
      mma16816(s[nb], qf[kk + 1], b2, b3);
    }
  }
}

// acc[16 x D] += P(16 x 16*NK keys) * V(keys kbase.., D)
template <int D, int NK>
BRAID_DEVICE void pv_tile(const float (*s)[4], const uint8_t* vs, int kbase, float (*acc)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NK; ++j) {
    uint32_t a[4];
    a[0] = pack_bf16(s[2 * j][0], s[2 * j][1]);
    a[1] = pack_bf16(s[2 * j][2], s[2 * j][3]);
    a[2] = pack_bf16(s[2 * j + 1][0], s[2 * j + 1][1]);
    a[3] = pack_bf16(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
    for (int nb = 0; nb < D / 8; nb += 2) {
      uint32_t b0, b1, b2, b3;
      const int row = kbase + j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = nb + (lane >> 4);
      ldsm_x4_t(smem_u32(vs) + swz<D>(row, c), b0, b1, b2, b3);
      mma16816(acc[nb], a, b0, b1);
      mma16816(acc[nb + 1], a, b2, b3);
    }
  }
}

// Online-softmax update for one 16-row slab: s holds scores (already scaled
// to log2 units and masked with -inf); m/l are per-thread row states for rows
// g and g+8.
template <int NB, int D>
BRAID_DEVICE void softmax_update(float (*s)[4], float* m, float* l, float (*acc)[4]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) mx = fmaxf(mx, fmaxf(s[nb][2 * h], s[nb][2 * h + 1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(m[h], mx);
    const float base = mnew == -INFINITY ? 0.f : mnew;
    const float corr = exp2f(m[h] - base);
    float sum = 0.f;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const float p0 = exp2f(s[nb][2 * h] - base), p1 = exp2f(s[nb][2 * h + 1] - base);
      s[nb][2 * h] = p0;
      s[nb][2 * h + 1] = p1;
      sum += p0 + p1;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l[h] = l[h] * corr + sum;
    m[h] = mnew;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      acc[nb][2 * h] *= corr;
      acc[nb][2 * h + 1] *= corr;
    }
  }
}

// --------------------------------------------------------------- decode
// Byte offset of 16-byte chunk c (of D/8) in row r of a TMA-written tile
// stored as D/64 column halves of [ROWS x 128 B] with 128-byte swizzle.
template <int ROWS>
BRAID_DEVICE uint32_t tswz(int r, int c) {
  return (uint32_t)((c >> 3) * (ROWS * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Producer cursor over the (segment, 64-key tile) sequence of one split range,
// walked by warp 0; page ids are fetched 32 at a time into registers and
// broadcast with shuffles (no dependent global load per box).
struct ProdCursor {
  int s, s1, segstart, lo, hi, off, sl, npages, win, win_page;
  const int* pages;
};

BRAID_DEVICE bool pc_settle(const AttnParams& p, ProdCursor& c, int r0, int r1) {
  while (c.s < c.s1 && c.segstart < r1) {
    const int len = p.seg_len[c.s];
    c.lo = max(r0 - c.segstart, 0);
    c.hi = min(r1 - c.segstart, len);
    if (c.lo < c.hi) {
      c.off = p.seg_offset[c.s];
      c.pages = p.page_ids + p.seg_page_indptr[c.s];
      c.npages = p.seg_page_indptr[c.s + 1] - p.seg_page_indptr[c.s];
      c.sl = (c.off + c.lo) & ~(KT - 1);
      c.win = -(1 << 30);
      return true;
    }
    c.segstart += len;
    ++c.s;
  }
  c.s = c.s1;
  return false;
}

BRAID_DEVICE void pc_next(const AttnParams& p, ProdCursor& c, int r0, int r1) {
  c.sl += KT;
  if (c.sl < c.off + c.hi) return;
  c.segstart += p.seg_len[c.s];
  ++c.s;
  pc_settle(p, c, r0, r1);
}

// Decode attention.  Four warps; warp 0 also streams 64-key K/V tiles with TMA
// into a STAGES-deep mbarrier ring (boxes of BR rows x 64 columns; BR = 64 when
// the page size is a multiple of 64, else 16 so a box never straddles a page),
// issuing tile i+STAGES-1 just before the CTA computes tile i.  Each warp takes
// 16 keys of every tile (mma.sync, fp32 online softmax).  Tiles are aligned in
// slot space; keys outside the segment or the split range are masked.
template <int D, int STAGES, int BR>
__global__ void __launch_bounds__(128, 2) attn_decode_kernel(const __grid_constant__ CUtensorMap tmkv,
                                                             const AttnParams p,
                                                             const __grid_constant__ CUtensorMap tmP) {
  constexpr int TILE = KT * D * 2;  // bytes of one K (or V) tile
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kbuf = sm;                         // STAGES x TILE
  uint8_t* vbuf = sm + STAGES * TILE;         // STAGES x TILE
  uint8_t* qs = vbuf + STAGES * TILE;         // [16][D] bf16, tswz<16> layout
  uint64_t* full = reinterpret_cast<uint64_t*>(qs + 16 * D * 2);
  uint64_t* empty = full + STAGES;
  const int b = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned long long* tr = p.trace
      ? p.trace + 8 * ((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) : nullptr;
  if (threadIdx.x == 0) {
    if (tr != nullptr) tr[0] = globaltimer_ns();
    span_start(p.span);
    tma_prefetch_desc(&tmkv);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // The step's metadata (plan buffer, page table, RoPE tables) is not written
  // by the preceding kernel: read it and walk to the first K/V tile before
  // waiting for that kernel (which produces q and appends this step's K/V).
  pdl_trigger();
  const int t = p.qo_indptr[b];
  if (p.qo_indptr[b + 1] - t < 1) return;
  const int qpos = p.positions[t];
  const int s0 = p.seg_indptr[b], s1 = p.seg_indptr[b + 1];
  int total = 0;
  for (int s = s0; s < s1; ++s) total += p.seg_len[s];
  int per = (total + p.num_splits - 1) / p.num_splits;
  per = (per + KT - 1) / KT * KT;
  const int r0 = split * per, r1 = min(total, r0 + per);
  const int G = p.G;

  // warp 0: issue one tile into stage st (all lanes take part in the page lookup)
  ProdCursor pc{s0, s1, 0, 0, 0, 0, 0, 0, 0, 0, nullptr};
  auto issue = [&](int st) {
#pragma unroll
    for (int q = 0; q < KT / BR; ++q) {
      const int slot = pc.sl + q * BR;
      const int pidx = min(slot / p.PS, pc.npages - 1);
      if (pidx < pc.win || pidx >= pc.win + 32) {
        pc.win = pidx;
        pc.win_page = pc.win + lane < pc.npages ? pc.pages[pc.win + lane] : 0;
      }
      const int page = __shfl_sync(0xffffffffu, pc.win_page, pidx - pc.win);
      if (lane == 0) (void)BRAID_IN_BOUNDS(page >= 0 && page < p.num_pages, 4, page);  // TMA zero-fills outside the pool
      if (lane == 0) {
        const int row_k = ((page * 2 + 0) * p.Hkv + kh) * p.PS + slot % p.PS;
        const int row_v = row_k + p.Hkv * p.PS;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
          uint8_t* dk = kbuf + st * TILE + h * (KT * 128) + q * BR * 128;
          uint8_t* dv = vbuf + st * TILE + h * (KT * 128) + q * BR * 128;
          if (p.kv_evict_first) {
            const uint64_t pol = l2_evict_first_policy();
            tma_load_2d_hint(dk, &tmkv, &full[st], h * 64, row_k, pol);
            tma_load_2d_hint(dv, &tmkv, &full[st], h * 64, row_v, pol);
          } else {
            tma_load_2d(dk, &tmkv, &full[st], h * 64, row_k);
            tma_load_2d(dv, &tmkv, &full[st], h * 64, row_v);
          }
        }
      }
    }
  };
  int issued = 0;
  bool first_v = false;
  if (warp == 0) first_v = pc_settle(p, pc, r0, r1);
  pdl_wait();
  if (threadIdx.x == 0) span_waited(p.span);
  if (warp == 0) {
    bool v = first_v;
    for (; issued < STAGES - 1 && v; ++issued) {
      if (lane == 0) mbar_arrive_expect_tx(&full[issued], 2 * TILE);
      issue(issued);
      pc_next(p, pc, r0, r1);
      v = pc.s < pc.s1;
    }
    // K/V streaming leaves HBM bandwidth unused: the next GEMM's weight can
    // come into L2 alongside it
    if (p.pf_early && lane == 0)
      prefetch_next_weight(&tmP, p.pf, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                           gridDim.x * gridDim.y * gridDim.z);
  }

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  uint32_t qf[D / 16][4];
  int it = 0, segstart = 0;
  bool ok = true;
  for (int s = s0; s < s1 && segstart < r1 && ok; ++s) {
    const int len = p.seg_len[s];
    const int lo = max(r0 - segstart, 0), hi = min(r1 - segstart, len);
    if (lo < hi) {
      __syncthreads();
      {
        // query rows rotated for this segment: one position for every row,
        // all loads independent (issued together)
        // (one item = 8 dims of each rotary half of one row, 16-byte accesses)
        constexpr int H2 = D / 2, CH = H2 / 8;
        int pos = qpos - p.seg_delta[s];
        pos = pos < 0 ? 0 : (pos >= p.rope_len ? p.rope_len - 1 : pos);
        if (threadIdx.x < 16 * CH) {
          const int r = threadIdx.x / CH, c8 = (threadIdx.x % CH) * 8;
          uint4 o1 = make_uint4(0, 0, 0, 0), o2 = make_uint4(0, 0, 0, 0);
          if (r < G) {
            const __nv_bfloat16* qp = p.q + ((size_t)t * p.Hq + kh * G + r) * D;
            const uint4 a4 = *reinterpret_cast<const uint4*>(qp + c8);
            const uint4 b4 = *reinterpret_cast<const uint4*>(qp + H2 + c8);
            if (p.use_rope) {
              const float* cp = p.cos + (size_t)pos * H2 + c8;
              const float* sp = p.sin + (size_t)pos * H2 + c8;
              float cs[8], sn[8];
              *reinterpret_cast<float4*>(cs) = *reinterpret_cast<const float4*>(cp);
              *reinterpret_cast<float4*>(cs + 4) = *reinterpret_cast<const float4*>(cp + 4);
              *reinterpret_cast<float4*>(sn) = *reinterpret_cast<const float4*>(sp);
              *reinterpret_cast<float4*>(sn + 4) = *reinterpret_cast<const float4*>(sp + 4);
              const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&a4);
              const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&b4);
              __nv_bfloat16* y1 = reinterpret_cast<__nv_bfloat16*>(&o1);
              __nv_bfloat16* y2 = reinterpret_cast<__nv_bfloat16*>(&o2);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float x1 = bf2f(a[j]), x2 = bf2f(bb[j]);
                y1[j] = f2bf(x1 * cs[j] - x2 * sn[j]);
                y2[j] = f2bf(x2 * cs[j] + x1 * sn[j]);
              }
            } else {
              o1 = a4;
              o2 = b4;
            }
          }
          *reinterpret_cast<uint4*>(qs + tswz<16>(r, c8 / 8)) = o1;
          *reinterpret_cast<uint4*>(qs + tswz<16>(r, (H2 + c8) / 8)) = o2;
        }
      }
      __syncthreads();
      {
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          ldsm_x4(smem_u32(qs) + tswz<16>(r, kk * 2 + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
      if (tr != nullptr && threadIdx.x == 0 && tr[1] == 0) tr[1] = globaltimer_ns();
      const int off = p.seg_offset[s], pos0 = p.seg_pos0[s];
      for (int sl = (off + lo) & ~(KT - 1); sl < off + hi; sl += KT, ++it) {
        // refill: tile `issued` goes into the stage released after tile it-1
        if (warp == 0 && pc.s < pc.s1) {
          const int st2 = issued % STAGES;
          int okw = 1;
          if (lane == 0) {
            if (issued >= STAGES) okw = mbar_wait(&empty[st2], ((issued / STAGES) & 1) ^ 1) ? 1 : 0;
            if (okw) mbar_arrive_expect_tx(&full[st2], 2 * TILE);
          }
          if (__shfl_sync(0xffffffffu, okw, 0)) {
            issue(st2);
            pc_next(p, pc, r0, r1);
            ++issued;
          } else {
            pc.s = pc.s1;
          }
        }
        const int st = it % STAGES;
        if (!mbar_wait(&full[st], (it / STAGES) & 1)) {
          ok = false;
          break;
        }
        const uint8_t* ks = kbuf + st * TILE;
        const uint8_t* vs = vbuf + st * TILE;
        float sc[2][4];
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
          const int row = warp * 16 + nb * 8 + (lane & 7);
#pragma unroll
          for (int kk = 0; kk < D / 16; kk += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(smem_u32(ks) + tswz<KT>(row, kk * 2 + (lane >> 3)), b0, b1, b2, b3);
            mma16816(sc[nb], qf[kk], b0, b1);
            mma16816(sc[nb], qf[kk + 1], b2, b3);
          }
        }
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = sl + warp * 16 + nb * 8 + 2 * (lane & 3) + (e & 1) - off;  // segment-local key
            const bool vis = j >= lo && j < hi && pos0 + j <= qpos;
            sc[nb][e] = vis ? sc[nb][e] * p.scale_log2 : -INFINITY;
          }
        softmax_update<2, D>(sc, m, l, acc);
        {
          uint32_t a[4];
          a[0] = pack_bf16(sc[0][0], sc[0][1]);
          a[1] = pack_bf16(sc[0][2], sc[0][3]);
          a[2] = pack_bf16(sc[1][0], sc[1][1]);
          a[3] = pack_bf16(sc[1][2], sc[1][3]);
          const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
          for (int nb = 0; nb < D / 8; nb += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(smem_u32(vs) + tswz<KT>(row, nb + (lane >> 4)), b0, b1, b2, b3);
            mma16816(acc[nb], a, b0, b1);
            mma16816(acc[nb + 1], a, b2, b3);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (tr != nullptr && threadIdx.x == 0 && tr[2] == 0) tr[2] = globaltimer_ns();
      }
    }
    segstart += len;
  }

  // ---- merge the 4 warps' partial states (reuse the K/V buffers)
  // Partials: split_stride slots per (token, head); this launch's splits
  // start at split_base; nsh shared-prefix partials of this sequence (slots
  // [0, nsh)) were published by the shared pass before this kernel.
  const int stride = p.split_stride > 0 ? p.split_stride : p.num_splits;
  const int nsh = (p.seq_nsh != nullptr && p.seq_nsh[b] != 0) ? p.split_base : 0;
  const bool direct = p.num_splits == 1 && nsh == 0;
  __syncthreads();
  if (threadIdx.x == 0 && !p.pf_early)  // every K/V tile has landed: pull this CTA's share of the next GEMM's weight into L2
    prefetch_next_weight(&tmP, p.pf, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                         gridDim.x * gridDim.y * gridDim.z);
  if (tr != nullptr && threadIdx.x == 0) tr[3] = globaltimer_ns();
  constexpr int AW_LD = D + 4;  // padded rows: no bank conflicts
  float* mw = reinterpret_cast<float*>(kbuf);        // [4][16]
  float* lw = mw + 64;                                // [4][16]
  float* aw = lw + 64;                                // [4][16][D]
  const int g = lane >> 2, c = lane & 3;
  if (c == 0) {
    mw[warp * 16 + g] = m[0];
    mw[warp * 16 + g + 8] = m[1];
    lw[warp * 16 + g] = l[0];
    lw[warp * 16 + g + 8] = l[1];
  }
#pragma unroll
  for (int nb = 0; nb < D / 8; ++nb) {
    const int d = nb * 8 + 2 * c;
    aw[(warp * 16 + g) * AW_LD + d] = acc[nb][0];
    aw[(warp * 16 + g) * AW_LD + d + 1] = acc[nb][1];
    aw[(warp * 16 + g + 8) * AW_LD + d] = acc[nb][2];
    aw[(warp * 16 + g + 8) * AW_LD + d + 1] = acc[nb][3];
  }
  __syncthreads();
  // one float4 (4 dims of one head row) per thread and pass
  for (int i = threadIdx.x; i < G * (D / 4); i += 128) {
    const int row = i / (D / 4), d = (i % (D / 4)) * 4;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mw[w * 16 + row]);
    float L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float e = exp2f(mw[w * 16 + row] - M);
        L += lw[w * 16 + row] * e;
        const float* a = aw + (w * 16 + row) * AW_LD + d;
        O.x += a[0] * e;
        O.y += a[1] * e;
        O.z += a[2] * e;
        O.w += a[3] * e;
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    O.x *= inv;
    O.y *= inv;
    O.z *= inv;
    O.w *= inv;
    const int h = kh * G + row;
    if (direct) {
      __nv_bfloat16* o = p.out + (size_t)t * p.Hq * D + h * D + d;
      *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(O.x, O.y);
      *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(O.z, O.w);
    } else {
      const size_t idx = ((size_t)t * p.Hq + h) * stride + p.split_base + split;
      *reinterpret_cast<float4*>(p.part_o + idx * D + d) = O;
      if (d == 0) p.part_lse[idx] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
  if (tr != nullptr && threadIdx.x == 0) tr[4] = globaltimer_ns();
  if (direct) {
    if (threadIdx.x == 0) span_end(p.span);
    return;
  }
  // ---- the last split CTA of (token, kv head) merges every split's partial
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    int* c = p.counters + (size_t)t * p.Hkv + kh;
    // releases this CTA's partials, acquires the other splits'
    const int old = atomic_add_acq_rel_gpu(c, 1);
    s_last = old == p.num_splits - 1;
    if (s_last) *c = 0;
  }
  __syncthreads();
  if (!s_last) {
    if (threadIdx.x == 0) span_end(p.span);
    return;
  }
  // slots [0, nsh) (shared prefix) and [split_base, split_base + num_splits) (this pass)
  const int ns = p.split_base + p.num_splits;
  const int sb = p.split_base;
  for (int i = threadIdx.x; i < G * (D / 4); i += 128) {
    const int row = i / (D / 4), d = (i % (D / 4)) * 4;
    const size_t base = ((size_t)t * p.Hq + kh * G + row) * stride;
    float lse[32];
#pragma unroll
    for (int q = 0; q < 32; ++q)
      lse[q] = (q < ns && (q < nsh || q >= sb)) ? __ldcg(p.part_lse + base + q) : -INFINITY;
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < 32; ++q) M = fmaxf(M, lse[q]);
    float W = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q0 = 0; q0 < 32; q0 += 16) {  // at most two passes of 16 partials in flight
      if (q0 < ns) {
        float4 o[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          o[k] = (q0 + k < ns && (q0 + k < nsh || q0 + k >= sb))
                     ? __ldcg(reinterpret_cast<const float4*>(p.part_o + (base + q0 + k) * D + d))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float w = (M == -INFINITY || q0 + k >= ns || lse[q0 + k] == -INFINITY) ? 0.f
                                                                                         : exp2f(lse[q0 + k] - M);
          W += w;
          O.x += w * o[k].x;
          O.y += w * o[k].y;
          O.z += w * o[k].z;
          O.w += w * o[k].w;
        }
      }
    }
    const float inv = W > 0.f ? 1.f / W : 0.f;
    __nv_bfloat16* o = p.out + (size_t)t * p.Hq * D + (kh * G + row) * D + d;
    *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(O.x * inv, O.y * inv);
    *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(O.z * inv, O.w * inv);
  }
  if (tr != nullptr && threadIdx.x == 0) tr[5] = globaltimer_ns();
  if (threadIdx.x == 0) span_end(p.span);
}

// -------------------------------------------------------------- prefill
// Prefill (or chunk self-prefill) attention: grid (64-row q tile, seq,
// kv head x splits); rows are (token, head-in-group) pairs.  Warp 0 streams
// 64-key K/V tiles with TMA into a STAGES-deep mbarrier ring (as in decode)
// while each warp computes its 16 rows against every tile; keys past the last
// query position of the q tile are never loaded.  With num_splits > 1 (a short
// query over long cached chunks: few q tiles) the visible keys are divided
// into contiguous ranges, one per CTA; each CTA writes its normalised partial
// and log-sum-exp and the last CTA of the q tile merges them.
template <int D, int STAGES, int BR>
__global__ void __launch_bounds__(128, 2) attn_prefill_kernel(const __grid_constant__ CUtensorMap tmkv,
                                                              const AttnParams p) {
  constexpr int TILE = KT * D * 2;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kbuf = sm;
  uint8_t* vbuf = sm + STAGES * TILE;
  uint8_t* qs = vbuf + STAGES * TILE;  // [64][D], tswz<64>
  uint64_t* full = reinterpret_cast<uint64_t*>(qs + 64 * D * 2);
  uint64_t* empty = full + STAGES;
  __shared__ int s_last;
  const int S = p.num_splits;
  const int b = blockIdx.y, kh = blockIdx.z / S, split = blockIdx.z % S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    span_start(p.span);
    tma_prefetch_desc(&tmkv);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // metadata first (not written by the preceding kernel), then wait for q / K/V
  pdl_trigger();
  unsigned long long* tr = p.trace
      ? p.trace + 8 * ((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[0] = globaltimer_ns();
  const int G = p.G;
  const int t0 = p.qo_indptr[b], nt = p.qo_indptr[b + 1] - t0;
  const int rows = nt * G;
  const int row0 = blockIdx.x * 64;
  if (row0 >= rows) return;
  const int nrows = min(64, rows - row0);
  int max_pos = p.positions[t0 + (row0 + nrows - 1) / G];
  int min_pos = p.positions[t0 + row0 / G];
  if (p.partial_only) {
    // the rows of a shared-prefix group are decode tokens of different
    // sequences: positions are not ordered by row
    for (int tk = t0 + row0 / G; tk <= t0 + (row0 + nrows - 1) / G; ++tk) {
      max_pos = max(max_pos, p.positions[tk]);
      min_pos = min(min_pos, p.positions[tk]);
    }
  }
  const int gq = lane >> 2;
  int rpos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = row0 + warp * 16 + gq + 8 * h;
    rpos[h] = rr < rows ? p.positions[t0 + rr / G] : -1;
  }
  const int s0 = p.seg_indptr[b], s1 = p.seg_indptr[b + 1];
  // keys some row of this tile can see: a prefix of each segment
  auto seg_vis = [&](int s) { return max(0, min(p.seg_len[s], max_pos - p.seg_pos0[s] + 1)); };
  // this split's range [r0, r1) of the concatenated visible keys
  int r0 = 0, r1 = 1 << 30;
  if (S > 1) {
    int total = 0;
    for (int s = s0; s < s1; ++s) total += seg_vis(s);
    const int per = ((total + S - 1) / S + KT - 1) / KT * KT;
    r0 = min(total, split * per);
    r1 = min(total, r0 + per);
  }
  // producer cursor (warp 0): segment s, keys [lo, hi) of it, next tile sl
  ProdCursor pc{s0, s1, 0, 0, 0, 0, 0, 0, 0, 0, nullptr};
  int pc_vis = 0;
  auto settle = [&]() {
    while (pc.s < pc.s1) {
      pc_vis = seg_vis(pc.s);
      pc.lo = max(0, r0 - pc.segstart);
      pc.hi = min(pc_vis, r1 - pc.segstart);
      if (pc.lo < pc.hi) {
        pc.off = p.seg_offset[pc.s];
        pc.pages = p.page_ids + p.seg_page_indptr[pc.s];
        pc.npages = p.seg_page_indptr[pc.s + 1] - p.seg_page_indptr[pc.s];
        pc.sl = (pc.off + pc.lo) & ~(KT - 1);
        pc.win = -(1 << 30);
        return;
      }
      pc.segstart += pc_vis;
      ++pc.s;
    }
  };
  auto advance = [&]() {
    pc.sl += KT;
    if (pc.sl < pc.off + pc.hi) return;
    pc.segstart += pc_vis;
    ++pc.s;
    settle();
  };
  auto issue = [&](int st) {
#pragma unroll
    for (int q = 0; q < KT / BR; ++q) {
      const int slot = pc.sl + q * BR;
      const int pidx = min(slot / p.PS, pc.npages - 1);
      if (pidx < pc.win || pidx >= pc.win + 32) {
        pc.win = pidx;
        pc.win_page = pc.win + lane < pc.npages ? pc.pages[pc.win + lane] : 0;
      }
      const int page = __shfl_sync(0xffffffffu, pc.win_page, pidx - pc.win);
      if (lane == 0) (void)BRAID_IN_BOUNDS(page >= 0 && page < p.num_pages, 4, page);  // TMA zero-fills outside the pool
      if (lane == 0) {
        const int row_k = ((page * 2 + 0) * p.Hkv + kh) * p.PS + slot % p.PS;
        const int row_v = row_k + p.Hkv * p.PS;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
          tma_load_2d(kbuf + st * TILE + h * (KT * 128) + q * BR * 128, &tmkv, &full[st], h * 64, row_k);
          tma_load_2d(vbuf + st * TILE + h * (KT * 128) + q * BR * 128, &tmkv, &full[st], h * 64, row_v);
        }
      }
    }
  };
  int issued = 0;
  if (warp == 0) settle();
  pdl_wait();
  if (threadIdx.x == 0) span_waited(p.span);
  if (warp == 0) {
    for (; issued < STAGES - 1 && pc.s < pc.s1; ++issued) {
      if (lane == 0) mbar_arrive_expect_tx(&full[issued], 2 * TILE);
      issue(issued);
      advance();
    }
  }

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  uint32_t qf[D / 16][4];
  int it = 0;
  bool ok = true;
  int segstart = 0;
  // every warp runs the same segment iterations (and so the same barriers),
  // even after a timed-out wait has stopped its tile loop
  for (int s = s0; s < s1; ++s) {
    const int pos0 = p.seg_pos0[s];
    const int vis = seg_vis(s);
    const int lo = max(0, r0 - segstart), hi = min(vis, r1 - segstart);
    segstart += vis;
    if (lo >= hi) continue;
    __syncthreads();
    {
      // Rotated query tile: one item = 8 dims of each rotary half of one row
      // (16-byte q loads, 32-byte cos/sin loads, 16-byte swizzled smem stores).
      constexpr int H2 = D / 2, CH = H2 / 8;
      const int delta = p.seg_delta[s];
#pragma unroll
      for (int k = 0; k < 64 * CH / 128; ++k) {
        const int i = threadIdx.x + 128 * k;
        const int r = i / CH, c8 = (i % CH) * 8;
        uint4 o1 = make_uint4(0, 0, 0, 0), o2 = make_uint4(0, 0, 0, 0);
        if (r < nrows) {
          const int rr = row0 + r;
          const int tok = t0 + rr / G, g = rr % G;
          const __nv_bfloat16* qp = p.q + ((size_t)tok * p.Hq + kh * G + g) * D;
          const uint4 a4 = *reinterpret_cast<const uint4*>(qp + c8);
          const uint4 b4 = *reinterpret_cast<const uint4*>(qp + H2 + c8);
          if (p.use_rope) {
            int pos = p.positions[tok] - delta;
            pos = pos < 0 ? 0 : (pos >= p.rope_len ? p.rope_len - 1 : pos);
            const float* cp = p.cos + (size_t)pos * H2 + c8;
            const float* sp = p.sin + (size_t)pos * H2 + c8;
            float cs[8], sn[8];
            *reinterpret_cast<float4*>(cs) = *reinterpret_cast<const float4*>(cp);
            *reinterpret_cast<float4*>(cs + 4) = *reinterpret_cast<const float4*>(cp + 4);
            *reinterpret_cast<float4*>(sn) = *reinterpret_cast<const float4*>(sp);
            *reinterpret_cast<float4*>(sn + 4) = *reinterpret_cast<const float4*>(sp + 4);
            const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&a4);
            const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&b4);
            __nv_bfloat16* y1 = reinterpret_cast<__nv_bfloat16*>(&o1);
            __nv_bfloat16* y2 = reinterpret_cast<__nv_bfloat16*>(&o2);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float x1 = bf2f(a[j]), x2 = bf2f(bb[j]);
              y1[j] = f2bf(x1 * cs[j] - x2 * sn[j]);
              y2[j] = f2bf(x2 * cs[j] + x1 * sn[j]);
            }
          } else {
            o1 = a4;
            o2 = b4;
          }
        }
        *reinterpret_cast<uint4*>(qs + tswz<64>(r, c8 / 8)) = o1;
        *reinterpret_cast<uint4*>(qs + tswz<64>(r, (H2 + c8) / 8)) = o2;
      }
    }
    __syncthreads();
    {
      const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        ldsm_x4(smem_u32(qs) + tswz<64>(r, kk * 2 + (lane >> 4)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
    if (tr != nullptr && threadIdx.x == 0 && tr[1] == 0) tr[1] = globaltimer_ns();
    const int off = p.seg_offset[s];
    for (int sl = (off + lo) & ~(KT - 1); sl < off + hi && ok; sl += KT, ++it) {
      if (warp == 0 && pc.s < pc.s1) {
        const int st2 = issued % STAGES;
        int okw = 1;
        if (lane == 0) {
          if (issued >= STAGES) okw = mbar_wait(&empty[st2], ((issued / STAGES) & 1) ^ 1) ? 1 : 0;
          if (okw) mbar_arrive_expect_tx(&full[st2], 2 * TILE);
        }
        if (__shfl_sync(0xffffffffu, okw, 0)) {
          issue(st2);
          advance();
          ++issued;
        } else {
          pc.s = pc.s1;
        }
      }
      const int st = it % STAGES;
      if (!mbar_wait(&full[st], (it / STAGES) & 1)) {
        ok = false;
        break;
      }
      const uint8_t* ks = kbuf + st * TILE;
      const uint8_t* vs = vbuf + st * TILE;
      float sc[8][4];
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
        const int row = nb * 8 + (lane & 7);
#pragma unroll
        for (int kk = 0; kk < D / 16; kk += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(smem_u32(ks) + tswz<KT>(row, kk * 2 + (lane >> 3)), b0, b1, b2, b3);
          mma16816(sc[nb], qf[kk], b0, b1);
          mma16816(sc[nb], qf[kk + 1], b2, b3);
        }
      }
      const int j0 = sl - off;
      const bool need_mask = (pos0 + j0 + KT - 1 > min_pos) || j0 < lo || (j0 + KT > hi);
      if (need_mask) {
#pragma unroll
        for (int nb = 0; nb < 8; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j0 + nb * 8 + 2 * (lane & 3) + (e & 1);
            const bool v = j >= lo && j < hi && pos0 + j <= rpos[e >> 1];
            sc[nb][e] = v ? sc[nb][e] * p.scale_log2 : -INFINITY;
          }
      } else {
#pragma unroll
        for (int nb = 0; nb < 8; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[nb][e] *= p.scale_log2;
      }
      softmax_update<8, D>(sc, m, l, acc);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t a[4];
        a[0] = pack_bf16(sc[2 * j][0], sc[2 * j][1]);
        a[1] = pack_bf16(sc[2 * j][2], sc[2 * j][3]);
        a[2] = pack_bf16(sc[2 * j + 1][0], sc[2 * j + 1][1]);
        a[3] = pack_bf16(sc[2 * j + 1][2], sc[2 * j + 1][3]);
        const int row = j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int nb = 0; nb < D / 8; nb += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(vs) + tswz<KT>(row, nb + (lane >> 4)), b0, b1, b2, b3);
          mma16816(acc[nb], a, b0, b1);
          mma16816(acc[nb + 1], a, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }
  const int c = lane & 3;
  if (tr != nullptr && threadIdx.x == 0) tr[2] = globaltimer_ns();
  if (p.partial_only) {
    // shared-prefix pass: publish (normalised partial, log-sum-exp) at slot
    // split_base + split; the decode pass merges them
    const int stride = p.split_stride > 0 ? p.split_stride : S;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rr = row0 + warp * 16 + gq + 8 * h;
      if (rr >= rows) continue;
      const int tok = t0 + rr / G, head = kh * G + rr % G;
      const size_t idx = ((size_t)tok * p.Hq + head) * stride + p.split_base + split;
      const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
      float* po = p.part_o + idx * D;
#pragma unroll
      for (int nb = 0; nb < D / 8; ++nb)
        *reinterpret_cast<float2*>(po + nb * 8 + 2 * c) =
            make_float2(acc[nb][2 * h] * inv, acc[nb][2 * h + 1] * inv);
      if (c == 0) p.part_lse[idx] = l[h] > 0.f ? m[h] + log2f(l[h]) : -INFINITY;
    }
    if (threadIdx.x == 0) span_end(p.span);
    return;
  }
  if (S == 1) {
    // ---- normalise and store
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rr = row0 + warp * 16 + gq + 8 * h;
      if (rr >= rows) continue;
      const int tok = t0 + rr / G, head = kh * G + rr % G;
      const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
      __nv_bfloat16* o = p.out + (size_t)tok * p.Hq * D + head * D;
#pragma unroll
      for (int nb = 0; nb < D / 8; ++nb) {
        const int d = nb * 8 + 2 * c;
        *reinterpret_cast<__nv_bfloat162*>(o + d) =
            __floats2bfloat162_rn(acc[nb][2 * h] * inv, acc[nb][2 * h + 1] * inv);
      }
    }
    if (threadIdx.x == 0) span_end(p.span);
    return;
  }
  // ---- split: publish this CTA's partial, the last CTA of the q tile merges
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = row0 + warp * 16 + gq + 8 * h;
    if (rr >= rows) continue;
    const int tok = t0 + rr / G, head = kh * G + rr % G;
    const size_t idx = ((size_t)tok * p.Hq + head) * S + split;
    const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
    float* po = p.part_o + idx * D;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb)
      *reinterpret_cast<float2*>(po + nb * 8 + 2 * c) = make_float2(acc[nb][2 * h] * inv, acc[nb][2 * h + 1] * inv);
    if (c == 0) p.part_lse[idx] = l[h] > 0.f ? m[h] + log2f(l[h]) : -INFINITY;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = p.counters + ((size_t)b * p.Hkv + kh) * gridDim.x + blockIdx.x;
    // releases this CTA's partial, acquires the other splits' partials
    const int old = atomic_add_acq_rel_gpu(ctr, 1);
    s_last = old == S - 1;
    if (s_last) *ctr = 0;
  }
  __syncthreads();
  if (tr != nullptr && threadIdx.x == 0) tr[3] = globaltimer_ns();
  if (!s_last) {
    if (threadIdx.x == 0) span_end(p.span);
    return;
  }
  // merge weights per row in shared memory (the K ring is idle now); every
  // lse / partial load of a row is issued before any is used
  float* wsm = reinterpret_cast<float*>(kbuf);  // [64][S]
  if (threadIdx.x < nrows) {
    const int rr = row0 + threadIdx.x;
    const size_t base = (((size_t)(t0 + rr / G)) * p.Hq + kh * G + rr % G) * S;
    float lse[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) lse[q] = q < S ? __ldcg(p.part_lse + base + q) : -INFINITY;
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < 32; ++q) mx = fmaxf(mx, lse[q]);
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      lse[q] = (mx == -INFINITY || q >= S) ? 0.f : exp2f(lse[q] - mx);
      sum += lse[q];
    }
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
#pragma unroll
    for (int q = 0; q < 32; ++q)
      if (q < S) wsm[threadIdx.x * S + q] = lse[q] * inv;
  }
  __syncthreads();
  constexpr int C4 = D / 4;
  for (int i0 = threadIdx.x; i0 < nrows * C4; i0 += 256) {
    // two output float4s per thread per pass, 8 splits of each in flight
    float4 o4[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    size_t pb[2];
    int rr_[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = min(i0 + 128 * u, nrows * C4 - 1);
      const int r = i / C4, d = (i % C4) * 4;
      const int rr = row0 + r;
      rr_[u] = r;
      pb[u] = (((size_t)(t0 + rr / G)) * p.Hq + kh * G + rr % G) * S * D + d;
    }
    for (int q0 = 0; q0 < S; q0 += 8) {
      float4 v[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          v[u][k] = q0 + k < S ? __ldcg(reinterpret_cast<const float4*>(p.part_o + pb[u] + (size_t)(q0 + k) * D))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float w = q0 + k < S ? wsm[rr_[u] * S + q0 + k] : 0.f;
          o4[u].x += w * v[u][k].x;
          o4[u].y += w * v[u][k].y;
          o4[u].z += w * v[u][k].z;
          o4[u].w += w * v[u][k].w;
        }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = i0 + 128 * u;
      if (i >= nrows * C4) continue;
      const int r = i / C4, d = (i % C4) * 4;
      const int rr = row0 + r;
      const int tok = t0 + rr / G, head = kh * G + rr % G;
      __nv_bfloat16* o = p.out + (size_t)tok * p.Hq * D + head * D + d;
      *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(o4[u].x, o4[u].y);
      *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(o4[u].z, o4[u].w);
    }
  }
  if (tr != nullptr && threadIdx.x == 0) tr[4] = globaltimer_ns();
  if (threadIdx.x == 0) span_end(p.span);
}

// ------------------------------------------------------------------ host
static unsigned long long* g_attn_trace = nullptr;
// Profiling: per-CTA phase timestamps of subsequent attention launches (int64 [8 * CTAs]).
void attn_set_trace(torch::Tensor buf) {
  g_attn_trace = buf.defined() && buf.numel() ? reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>()) : nullptr;
}
// Profiling: per-tile softmax timestamps of subsequent tcgen05 prefill launches
// (int64 [128 * CTAs]; attention_tc.cu documents the layout).
static unsigned long long* g_attn_tc_trace = nullptr;
void attn_tc_set_trace(torch::Tensor buf) {
  g_attn_tc_trace =
      buf.defined() && buf.numel() ? reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>()) : nullptr;
}

int gemm_num_sms();
unsigned long long* next_span(const char* name);
PrefetchArgs take_prefetch(CUtensorMap* map, const CUtensorMap& fallback);

// Per-device split-merge counters (zeroed once; the merging CTA re-arms its counter).
static int* attn_counters(int dev, size_t n) {
  static std::mutex mu;
  static std::unordered_map<int, std::pair<int*, size_t>> all;
  std::lock_guard<std::mutex> g(mu);
  auto& e = all[dev];
  if (n > e.second) {
    // growth happens only outside graph capture (warm-up runs the same shapes first)
    if (e.first) C10_CUDA_CHECK(cudaFree(e.first));
    const size_t m = std::max(n, (size_t)1 << 16);
    C10_CUDA_CHECK(cudaMalloc(&e.first, m * sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(e.first, 0, m * sizeof(int)));
    e.second = m;
  }
  return e.first;
}

bool attn_prefill_tc_use(int D, int64_t rows);
bool attn_shared_tc_use(int D);
int attn_prefill_tc_rows();
int attn_prefill_tc_min_rows();
void launch_attn_prefill_tc(const AttnParams& p, int num_seqs, int max_q_len, int64_t P, cudaStream_t st);

template <int D>
static void launch_attn(AttnParams& p, int num_seqs, int max_q_len, bool decode, int T, int64_t P,
                        cudaStream_t st) {
  if (!decode && p.use_tc) {  // tcgen05 prefill (attention_tc.cu)
    launch_attn_prefill_tc(p, num_seqs, max_q_len, P, st);
    return;
  }
  if (decode) {
    constexpr int STAGES = D == 128 ? 3 : 4;
    const int smem = 2 * STAGES * KT * D * 2 + 16 * D * 2 + 2 * STAGES * 8 + 1024;
    // the layer pool viewed as rows of D elements: row = ((page*2 + kv)*Hkv + kh)*PS + slot
    const int64_t rows = P * 2 * p.Hkv * p.PS;
    if (p.PS % 64 == 0) {
      auto k = attn_decode_kernel<D, STAGES, 64>;
      static bool attr = false;
      if (!attr) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr = true;
      }
      CUtensorMap tm = make_tmap(p.kv, rows, D, D, 64);
      CUtensorMap tp;
      p.pf = take_prefetch(&tp, tm);
      launch_pdl(k, dim3(num_seqs, p.Hkv, p.num_splits), dim3(128), smem, st, tm, p, tp);
    } else {
      auto k = attn_decode_kernel<D, STAGES, 16>;
      static bool attr = false;
      if (!attr) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr = true;
      }
      CUtensorMap tm = make_tmap(p.kv, rows, D, D, 16);
      CUtensorMap tp;
      p.pf = take_prefetch(&tp, tm);
      launch_pdl(k, dim3(num_seqs, p.Hkv, p.num_splits), dim3(128), smem, st, tm, p, tp);
    }
  } else {
    constexpr int STAGES = D == 128 ? 2 : 3;
    const int smem = 2 * STAGES * KT * D * 2 + 64 * D * 2 + 2 * STAGES * 8 + 1024;
    const int64_t rows = P * 2 * p.Hkv * p.PS;
    const int qt = (max_q_len * p.G + 63) / 64;
    if (p.PS % 64 == 0) {
      auto k = attn_prefill_kernel<D, STAGES, 64>;
      static bool attr = false;
      if (!attr) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr = true;
      }
      CUtensorMap tm = make_tmap(p.kv, rows, D, D, 64);
      launch_pdl(k, dim3(qt, num_seqs, p.Hkv * p.num_splits), dim3(128), smem, st, tm, p);
    } else {
      auto k = attn_prefill_kernel<D, STAGES, 16>;
      static bool attr = false;
      if (!attr) {
        C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr = true;
      }
      CUtensorMap tm = make_tmap(p.kv, rows, D, D, 16);
      launch_pdl(k, dim3(qt, num_seqs, p.Hkv * p.num_splits), dim3(128), smem, st, tm, p);
    }
  }
}

void attention(torch::Tensor out, torch::Tensor q, torch::Tensor kv, torch::Tensor qo_indptr,
               torch::Tensor positions, torch::Tensor seg_indptr, torch::Tensor seg_page_indptr,
               torch::Tensor seg_offset, torch::Tensor seg_len, torch::Tensor seg_pos0, torch::Tensor seg_delta,
               torch::Tensor page_ids, torch::Tensor cos, torch::Tensor sin, double scale, bool use_rope,
               int64_t num_seqs, int64_t max_q_len, int64_t max_kv_len, bool decode, int64_t num_splits,
               c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_lse,
               c10::optional<torch::Tensor> grp_qo_indptr, c10::optional<torch::Tensor> grp_seg_indptr,
               c10::optional<torch::Tensor> seq_nsh, int64_t shared_splits, int64_t grp_max_q) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && kv.scalar_type() == at::kBFloat16);
  TORCH_CHECK(q.is_contiguous() && kv.is_contiguous() && out.is_contiguous());
  const int T = q.size(0), Hq = q.size(1), D = q.size(2);
  const int Hkv = kv.size(2), PS = kv.size(3);
  TORCH_CHECK(kv.size(4) == D && Hq % Hkv == 0, "attention: head layout mismatch");
  const int G = Hq / Hkv;
  TORCH_CHECK(G <= 16 || !decode, "attention: decode supports up to 16 query heads per KV head");
  TORCH_CHECK(PS % 16 == 0, "attention: page size must be a multiple of 16");
  if (T == 0 || num_seqs == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  AttnParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.kv = reinterpret_cast<const __nv_bfloat16*>(kv.data_ptr());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.qo_indptr = qo_indptr.data_ptr<int>();
  p.positions = positions.data_ptr<int>();
  p.seg_indptr = seg_indptr.data_ptr<int>();
  p.seg_page_indptr = seg_page_indptr.data_ptr<int>();
  p.seg_offset = seg_offset.data_ptr<int>();
  p.seg_len = seg_len.data_ptr<int>();
  p.seg_pos0 = seg_pos0.data_ptr<int>();
  p.seg_delta = seg_delta.data_ptr<int>();
  p.page_ids = page_ids.data_ptr<int>();
  p.cos = cos.data_ptr<float>();
  p.sin = sin.data_ptr<float>();
  p.rope_len = cos.size(0);
  p.scale_log2 = (float)scale * LOG2E;
  p.use_rope = use_rope ? 1 : 0;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = G;
  p.PS = PS;
  p.num_pages = (int)kv.size(0);
  size_t n_counters = (size_t)T * Hkv;
  if (decode) {
    p.num_splits = (int)std::max<int64_t>(1, num_splits);
  } else {
    // Prefill: split the keys when the q tiles alone leave SMs idle (a short
    // query over long cached chunks); each split keeps >= 2 key tiles.
    const int sms_ = gemm_num_sms();
    int tile_rows = 64;
    p.use_tc = attn_prefill_tc_use(D, (int64_t)T * G) ? 1 : 0;
    if (p.use_tc) {
      // tcgen05 kernel: 256-row CTAs (two Q tiles), or 128-row CTAs when the
      // 256-row work units would fill less than half of the SMs
      const int64_t w256 = (int64_t)((max_q_len * G + attn_prefill_tc_rows() - 1) / attn_prefill_tc_rows()) *
                           num_seqs * Hkv;
      tile_rows = w256 * 2 <= sms_ ? attn_prefill_tc_min_rows() : attn_prefill_tc_rows();
    }
    p.cta_rows = tile_rows;
    const int qt = (int)((max_q_len * G + tile_rows - 1) / tile_rows);
    const int64_t work = (int64_t)qt * num_seqs * Hkv;
    static const int forced = [] {  // tuning knob: BRAID_PREFILL_SPLITS=n
      const char* e = getenv("BRAID_PREFILL_SPLITS");
      return e ? atoi(e) : 0;
    }();
    int ns = 1;
    const int sms = gemm_num_sms();
    if (work < sms && p.use_tc) {
      // one CTA per SM: pick the split count with the fewest (waves x key
      // tiles per CTA, plus about two tiles of fixed cost per CTA), plus the
      // merge, whose last CTA reads every split's 256-row partial (about one
      // tile's time per split)
      const int64_t kvt = std::max<int64_t>(1, (max_kv_len + 127) / 128);
      int64_t best = INT64_MAX;
      for (int n = 1; n <= 32 && n <= kvt; ++n) {
        const int64_t est = ((work * n + sms - 1) / sms) * ((kvt + n - 1) / n + 2) + (n > 1 ? n : 0);
        if (est < best) {
          best = est;
          ns = n;
        }
      }
    } else if (work < sms) {
      ns = (int)std::min<int64_t>({(2 * sms + work - 1) / work, 32, std::max<int64_t>(1, max_kv_len / 128)});
    }
    if (num_splits > 1) ns = (int)std::min<int64_t>(num_splits, 32);
    if (forced > 0) ns = std::min(forced, 32);
    p.num_splits = std::max(1, ns);
    n_counters = (size_t)qt * num_seqs * Hkv;
  }
  p.trace = g_attn_trace;
  p.tc_trace = g_attn_tc_trace;
  // Decode K/V are read once per step (shared chunk pages by CTAs running at
  // the same time): evict-first keeps them from pushing out other lines.
  // Tuning knob: BRAID_KV_EVICT_FIRST=0 uses the default L2 policy.
  static const int kv_ef = [] {
    const char* e = getenv("BRAID_KV_EVICT_FIRST");
    return e && e[0] == '0' ? 0 : 1;
  }();
  p.kv_evict_first = kv_ef;
  static const int pf_early = [] {  // tuning knob: BRAID_ATTN_PF_EARLY=1
    const char* e = getenv("BRAID_ATTN_PF_EARLY");
    return e && e[0] == '1' ? 1 : 0;
  }();
  p.pf_early = pf_early;
  // Shared-prefix decode: a group of sequences whose common segments are
  // attended once (prefill kernel over the group's decode tokens, partials
  // only), then each sequence's own segments (decode kernel) merged with them.
  const bool grouped = decode && shared_splits > 0 && grp_qo_indptr.has_value() && grp_qo_indptr->defined();
  const int S_sh = grouped ? (int)shared_splits : 0;
  const int S_tot = S_sh + p.num_splits;
  TORCH_CHECK(S_tot <= 32, "attention: at most 32 partial slots per (token, head)");
  torch::Tensor po, pl;
  if (S_tot > 1) {
    if (part_o.has_value() && part_o->defined() && part_o->numel() >= (int64_t)T * Hq * S_tot * D &&
        part_lse.has_value() && part_lse->defined() && part_lse->numel() >= (int64_t)T * Hq * S_tot) {
      po = *part_o;
      pl = *part_lse;
    } else {
      po = torch::empty({(int64_t)T * Hq * S_tot * D}, q.options().dtype(at::kFloat));
      pl = torch::empty({(int64_t)T * Hq * S_tot}, q.options().dtype(at::kFloat));
    }
    p.part_o = po.data_ptr<float>();
    p.part_lse = pl.data_ptr<float>();
    p.counters = attn_counters(q.get_device(), n_counters);
  }
  auto run = [&](AttnParams& a, int64_t nseq, int64_t mq, bool dec) {
    if (D == 128)
      launch_attn<128>(a, (int)nseq, (int)mq, dec, T, kv.size(0), st);
    else if (D == 64)
      launch_attn<64>(a, (int)nseq, (int)mq, dec, T, kv.size(0), st);
    else
      TORCH_CHECK(false, "attention: head_dim must be 64 or 128");
  };
  if (grouped) {
    TORCH_CHECK(grp_seg_indptr.has_value() && seq_nsh.has_value() && seq_nsh->numel() >= num_seqs,
                "attention: shared-prefix group metadata incomplete");
    AttnParams a = p;
    a.qo_indptr = grp_qo_indptr->data_ptr<int>();
    a.seg_indptr = grp_seg_indptr->data_ptr<int>();
    a.num_splits = S_sh;
    a.split_base = 0;
    a.split_stride = S_tot;
    a.partial_only = 1;
    a.use_tc = attn_shared_tc_use(D) ? 1 : 0;
    a.span = next_span("attn_shared_prefix");
    run(a, grp_qo_indptr->numel() - 1, std::max<int64_t>(1, grp_max_q), false);
    p.split_base = S_sh;
    p.split_stride = S_tot;
    p.seq_nsh = seq_nsh->data_ptr<int>();
  }
  p.span = next_span(decode ? "attn_decode" : "attn_prefill");
  run(p, num_seqs, max_q_len, decode);
}

}  // namespace braid

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_attention)
}  // namespace braid
