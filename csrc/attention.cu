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

#include <mutex>
#include <unordered_map>

namespace braid {

struct AttnParams {
  const __nv_bfloat16* q;  // [T, Hq, D] unrotated
  const __nv_bfloat16* kv; // layer pool [P, 2, Hkv, PS, D]
  __nv_bfloat16* out;      // [T, Hq*D]
  const int* qo_indptr;
  const int* positions;
  const int* seg_indptr;
  const int* seg_page_indptr;
  const int* seg_offset;
  const int* seg_len;
  const int* seg_pos0;
  const int* seg_delta;
  const int* page_ids;
  const float* cos;
  const float* sin;
  float scale_log2;
  int use_rope;
  int rope_len;
  int Hq, Hkv, G, PS;
  int num_splits;
  float* part_o;    // [T, Hq, splits, D]
  float* part_lse;  // [T, Hq, splits]
  int* counters;    // [T * Hkv] split arrival counters, kept at zero between launches
};

constexpr float LOG2E = 1.4426950408889634f;
constexpr int KT = 64;  // keys per tile

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
    const bool ok = j < jend;
    const __nv_bfloat16* kp = p.kv;
    const __nv_bfloat16* vp = p.kv;
    if (ok) {
      const int slot = off + j;
      const int page = pages[slot / p.PS];
      kp = p.kv + kv_row(p, page, 0, kh, slot % p.PS, D) + c * 8;
      vp = p.kv + kv_row(p, page, 1, kh, slot % p.PS, D) + c * 8;
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
template <int D>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* qs = sm;                                  // [16][D]
  uint8_t* kbuf = sm + 16 * D * 2;                   // 2 x [64][D]
  uint8_t* vbuf = kbuf + 2 * KT * D * 2;             // 2 x [64][D]
  const int b = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
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

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  uint32_t qf[D / 16][4];
  const int G = p.G;

  int segstart = 0;
  for (int s = s0; s < s1 && segstart < r1; ++s) {
    const int len = p.seg_len[s];
    const int lo = max(r0 - segstart, 0), hi = min(r1 - segstart, len);
    if (lo < hi) {
      __syncthreads();
      build_q_tile<D>(p, kh, p.seg_delta[s], G, 16, qs, [&](int r, int& tok, int& g) { tok = t; g = r; });
      load_kv_tile<D>(p, s, kh, lo, hi, kbuf, vbuf);
      cp_async_commit();
      __syncthreads();
      load_q_frags<D>(qs, 0, qf);
      const int pos0 = p.seg_pos0[s];
      int buf = 0;
      for (int j0 = lo; j0 < hi; j0 += KT) {
        if (j0 + KT < hi) {
          load_kv_tile<D>(p, s, kh, j0 + KT, hi, kbuf + (buf ^ 1) * KT * D * 2, vbuf + (buf ^ 1) * KT * D * 2);
          cp_async_commit();
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
        __syncthreads();
        const uint8_t* ks = kbuf + buf * KT * D * 2;
        const uint8_t* vs = vbuf + buf * KT * D * 2;
        float sc[2][4];
        qk_tile<D, 2>(qf, ks, warp * 16, sc);
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j0 + warp * 16 + nb * 8 + 2 * (lane & 3) + (e & 1);
            const bool vis = j < hi && pos0 + j <= qpos;
            sc[nb][e] = vis ? sc[nb][e] * p.scale_log2 : -INFINITY;
          }
        softmax_update<2, D>(sc, m, l, acc);
        pv_tile<D, 1>(sc, vs, warp * 16, acc);
        __syncthreads();
        buf ^= 1;
      }
    }
    segstart += len;
  }

  // ---- merge the 4 warps' partial states (reuse the K/V buffers)
  __syncthreads();
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
    aw[(warp * 16 + g) * D + d] = acc[nb][0];
    aw[(warp * 16 + g) * D + d + 1] = acc[nb][1];
    aw[(warp * 16 + g + 8) * D + d] = acc[nb][2];
    aw[(warp * 16 + g + 8) * D + d + 1] = acc[nb][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int row = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mw[w * 16 + row]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float e = exp2f(mw[w * 16 + row] - M);
        L += lw[w * 16 + row] * e;
        O += aw[(w * 16 + row) * D + d] * e;
      }
    }
    const int h = kh * G + row;
    if (p.num_splits == 1) {
      p.out[(size_t)t * p.Hq * D + h * D + d] = f2bf(L > 0.f ? O / L : 0.f);
    } else {
      const size_t idx = ((size_t)t * p.Hq + h) * p.num_splits + split;
      p.part_o[idx * D + d] = L > 0.f ? O / L : 0.f;
      if (d == 0) p.part_lse[idx] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
  if (p.num_splits == 1) return;
  // ---- the last split CTA of (token, kv head) merges every split's partial
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* c = p.counters + (size_t)t * p.Hkv + kh;
    const int old = atomicAdd(c, 1);
    s_last = old == p.num_splits - 1;
    if (s_last) *c = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int ns = p.num_splits;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int row = i / D, d = i % D;
    const size_t base = ((size_t)t * p.Hq + kh * G + row) * ns;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, __ldcg(p.part_lse + base + s));
    float W = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < ns; ++s) {
        const float w = exp2f(__ldcg(p.part_lse + base + s) - M);
        W += w;
        O += w * __ldcg(p.part_o + (base + s) * D + d);
      }
    }
    p.out[(size_t)t * p.Hq * D + (kh * G + row) * D + d] = f2bf(W > 0.f ? O / W : 0.f);
  }
}

// -------------------------------------------------------------- prefill
template <int D>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* qs = sm;                                  // [64][D]
  uint8_t* kbuf = sm + 64 * D * 2;                   // 2 x [64][D]
  uint8_t* vbuf = kbuf + 2 * KT * D * 2;
  const int b = blockIdx.y, kh = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  const int G = p.G;
  const int t0 = p.qo_indptr[b], nt = p.qo_indptr[b + 1] - t0;
  const int rows = nt * G;
  const int row0 = blockIdx.x * 64;
  if (row0 >= rows) return;
  const int nrows = min(64, rows - row0);
  const int max_pos = p.positions[t0 + (row0 + nrows - 1) / G];
  const int min_pos = p.positions[t0 + row0 / G];
  auto row_tok = [&](int r, int& tok, int& g) {
    const int rr = row0 + r;
    tok = t0 + rr / G;
    g = rr % G;
  };
  // positions of this thread's two rows (g and g+8 of the warp's slab)
  const int gq = lane >> 2;
  int rpos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = row0 + warp * 16 + gq + 8 * h;
    rpos[h] = rr < rows ? p.positions[t0 + rr / G] : -1;
  }

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  uint32_t qf[D / 16][4];

  const int s0 = p.seg_indptr[b], s1 = p.seg_indptr[b + 1];
  for (int s = s0; s < s1; ++s) {
    const int pos0 = p.seg_pos0[s];
    const int hi = min(p.seg_len[s], max_pos - pos0 + 1);
    if (hi <= 0) continue;
    __syncthreads();
    build_q_tile<D>(p, kh, p.seg_delta[s], nrows, 64, qs, row_tok);
    load_kv_tile<D>(p, s, kh, 0, hi, kbuf, vbuf);
    cp_async_commit();
    __syncthreads();
    load_q_frags<D>(qs, warp * 16, qf);
    int buf = 0;
    for (int j0 = 0; j0 < hi; j0 += KT) {
      if (j0 + KT < hi) {
        load_kv_tile<D>(p, s, kh, j0 + KT, hi, kbuf + (buf ^ 1) * KT * D * 2, vbuf + (buf ^ 1) * KT * D * 2);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const uint8_t* ks = kbuf + buf * KT * D * 2;
      const uint8_t* vs = vbuf + buf * KT * D * 2;
      float sc[8][4];
      qk_tile<D, 8>(qf, ks, 0, sc);
      const bool need_mask = (pos0 + j0 + KT - 1 > min_pos) || (j0 + KT > hi);
      if (need_mask) {
#pragma unroll
        for (int nb = 0; nb < 8; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = j0 + nb * 8 + 2 * (lane & 3) + (e & 1);
            const bool vis = j < hi && pos0 + j <= rpos[e >> 1];
            sc[nb][e] = vis ? sc[nb][e] * p.scale_log2 : -INFINITY;
          }
      } else {
#pragma unroll
        for (int nb = 0; nb < 8; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[nb][e] *= p.scale_log2;
      }
      softmax_update<8, D>(sc, m, l, acc);
      pv_tile<D, 4>(sc, vs, 0, acc);
      __syncthreads();
      buf ^= 1;
    }
  }
  // ---- normalise and store
  const int c = lane & 3;
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
      *reinterpret_cast<__nv_bfloat162*>(o + d) = __floats2bfloat162_rn(acc[nb][2 * h] * inv, acc[nb][2 * h + 1] * inv);
    }
  }
}

// ------------------------------------------------------------------ host
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

template <int D>
static void launch_attn(AttnParams& p, int num_seqs, int max_q_len, bool decode, int T, cudaStream_t st) {
  if (decode) {
    const int smem = 16 * D * 2 + 4 * KT * D * 2;
    auto k = attn_decode_kernel<D>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr = true;
    }
    launch_pdl(k, dim3(num_seqs, p.Hkv, p.num_splits), dim3(128), smem, st, p);
  } else {
    const int smem = 64 * D * 2 + 4 * KT * D * 2;
    auto k = attn_prefill_kernel<D>;
    static bool attr = false;
    if (!attr) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr = true;
    }
    const int qt = (max_q_len * p.G + 63) / 64;
    launch_pdl(k, dim3(qt, num_seqs, p.Hkv), dim3(128), smem, st, p);
  }
}

void attention(torch::Tensor out, torch::Tensor q, torch::Tensor kv, torch::Tensor qo_indptr,
               torch::Tensor positions, torch::Tensor seg_indptr, torch::Tensor seg_page_indptr,
               torch::Tensor seg_offset, torch::Tensor seg_len, torch::Tensor seg_pos0, torch::Tensor seg_delta,
               torch::Tensor page_ids, torch::Tensor cos, torch::Tensor sin, double scale, bool use_rope,
               int64_t num_seqs, int64_t max_q_len, int64_t max_kv_len, bool decode, int64_t num_splits,
               c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_lse) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && kv.scalar_type() == at::kBFloat16);
  TORCH_CHECK(q.is_contiguous() && kv.is_contiguous() && out.is_contiguous());
  const int T = q.size(0), Hq = q.size(1), D = q.size(2);
  const int Hkv = kv.size(2), PS = kv.size(3);
  TORCH_CHECK(kv.size(4) == D && Hq % Hkv == 0, "attention: head layout mismatch");
  const int G = Hq / Hkv;
  TORCH_CHECK(G <= 16 || !decode, "attention: decode supports up to 16 query heads per KV head");
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
  p.num_splits = decode ? (int)std::max<int64_t>(1, num_splits) : 1;
  torch::Tensor po, pl;
  if (p.num_splits > 1) {
    if (part_o.has_value() && part_o->defined() && part_o->numel() >= (int64_t)T * Hq * p.num_splits * D) {
      po = *part_o;
      pl = *part_lse;
    } else {
      po = torch::empty({(int64_t)T * Hq * p.num_splits * D}, q.options().dtype(at::kFloat));
      pl = torch::empty({(int64_t)T * Hq * p.num_splits}, q.options().dtype(at::kFloat));
    }
    p.part_o = po.data_ptr<float>();
    p.part_lse = pl.data_ptr<float>();
    p.counters = attn_counters(q.get_device(), (size_t)T * Hkv);
  }
  if (D == 128)
    launch_attn<128>(p, num_seqs, max_q_len, decode, T, st);
  else if (D == 64)
    launch_attn<64>(p, num_seqs, max_q_len, decode, T, st);
  else
    TORCH_CHECK(false, "attention: head_dim must be 64 or 128");
}

}  // namespace braid
