// tcgen05 GEMM for sm_100a:  D[M, N] = A[M, K] * B[N, K]^T  (bf16 in, fp32 accumulate)
//
// One CTA computes one 128 x BN output tile (optionally one K-slice of it):
//   warp 0      TMA producer: 128B-swizzled A/B K-blocks into a STAGES-deep ring
//   warp 1      MMA issuer: one elected lane issues tcgen05.mma (M=128, N=BN,
//               K=16 per instruction) into a TMEM accumulator, frees ring slots
//               with tcgen05.commit
//   warps 2..5  epilogue: tcgen05.ld from TMEM (each warp owns 32 TMEM lanes),
//               split-K reduction, bias / residual / SwiGLU, bf16 stores
//
// Two operand roles serve the model:
//   normal  (prefill):  A = activations [tokens, K],  B = weight [features, K]
//   swapped (decode):   A = weight [features, K],     B = activations [tokens, K]
//     The weight fills the 128-row MMA M dimension and the small token count
//     is the MMA N (16..128), so a decode step streams the weight once at HBM
//     rate; the epilogue writes the transposed tile to Y[token, feature].
// Split-K (decode shapes with few output tiles): each K-slice CTA writes an
// fp32 partial tile to a workspace; the last CTA to arrive on the tile's
// counter sums the partials, applies the epilogue and re-arms the counter.
//
// Epilogue rounding follows an HF bf16 forward: y = bf16(acc + bias); with a
// residual, out = bf16(y + residual); SwiGLU rounds gate, up and silu(gate).
// SwiGLU weights are block-interleaved in 64-row blocks (gate rows, then the
// matching up rows), so a 128-row (swapped) or 128-column (normal) tile holds
// both halves of 64 output features.
//
// Replaces the reference's Triton GEMMs (fused_rmsnorm_qkv_*.py, tl.dot with
// 16x64x64 tiles) and the cuBLAS F.linear calls of braidinfer/layers/linear.py.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "gemm_types.cuh"
#include "launch.cuh"

namespace braid {


template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int XCH = BM * XCH_LD * 4;
  static constexpr int RSTD = 256 * 4;
  static constexpr int BAR_OFF = RING + XCH + RSTD;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 1) * 8 + 16 + 1024;  // +1024 alignment slack
};

// Per-head q/k norm + RoPE on E = D/32 consecutive dims held by this lane;
// the rotary partner of dim e (< D/2) is e + D/2, held by lane ^ 16.
template <int E>
BRAID_DEVICE void qkv_head_store(const QkvEpi& q, float* v, int head, int t, int lane) {
  const int D = E * 32;
  const bool is_q = head < q.Hq, is_k = !is_q && head < q.Hq + q.Hkv;
  const __nv_bfloat16* nw = is_q ? q.q_norm : (is_k ? q.k_norm : nullptr);
  if (nw != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) ss += v[i] * v[i];
    const float r = rsqrtf(warp_sum(ss) / D + q.eps);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = rbf(rbf(v[i] * r) * bf2f(nw[lane * E + i]));
  }
  if (is_q) {
    __nv_bfloat16* dst = q.q_out + ((size_t)t * q.Hq + head) * D + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = f2bf(v[i]);
    return;
  }
  if (is_k && q.use_rope) {
    int pos = q.positions[t];
    if (!BRAID_IN_BOUNDS(pos >= 0 && pos < q.rope_len, 2, pos)) pos = 0;
    float pr[E];
#pragma unroll
    for (int i = 0; i < E; ++i) pr[i] = __shfl_xor_sync(0xffffffffu, v[i], 16);
    const bool first = lane < 16;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int d = (lane & 15) * E + i;
      const float c = q.cos[(size_t)pos * (D / 2) + d], s = q.sin[(size_t)pos * (D / 2) + d];
      v[i] = first ? v[i] * c - pr[i] * s : v[i] * c + pr[i] * s;
    }
  }
  const int slot = q.slots[t];
  if (!BRAID_IN_BOUNDS(slot >= 0 && slot < q.num_slots, 1, slot)) return;
  const int page = slot / q.PS, off = slot % q.PS;
  const int kh = is_k ? head - q.Hq : head - q.Hq - q.Hkv;
  __nv_bfloat16* dst =
      q.kv + ((((size_t)page * 2 + (is_k ? 0 : 1)) * q.Hkv + kh) * q.PS + off) * D + lane * E;
#pragma unroll
  for (int i = 0; i < E; ++i) dst[i] = f2bf(v[i]);
}

BRAID_DEVICE bool et_is_epi_last(int tid) { return tid == 191; }

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 2) gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                                                               const __grid_constant__ CUtensorMap tmB,
                                                               const GemmArgs args,
                                                               const __grid_constant__ CUtensorMap tmP) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ringA = smem;
  uint8_t* ringB = smem + STAGES * S::A_BYTES;
  float* xch = reinterpret_cast<float*>(smem + S::RING);
  float* rstd_s = reinterpret_cast<float*>(smem + S::RING + S::XCH);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_full + 1);
  int* s_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y, split = blockIdx.z;
  const int m0 = m_tile * BM, n0 = n_tile * BN;
  const int kb_total = (args.K + BK - 1) / BK;
  const int kb0 = split * args.kb_per_split;
  const int nkb = min(args.kb_per_split, kb_total - kb0);
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  unsigned long long* tr = args.trace
      ? args.trace + 8 * ((size_t)(blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[0] = globaltimer_ns();
  if (threadIdx.x == 0) span_start(args.span);

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_trigger();
  // epilogue-thread geometry (used by warps 2..5 only)
  const int wq = warp & 3;             // TMEM lane quarter this warp may access
  const int r = wq * 32 + lane;        // row of the tile owned by this thread
  const int et = threadIdx.x - 64;     // 0..127 epilogue thread id
  const int ew = et >> 5;              // epilogue warp 0..3
  const uint32_t trow = tmem + ((uint32_t)(wq * 32) << 16);
  const int tile = m_tile * gridDim.y + n_tile;
  float rs_row = 1.f;
  bool has_acc = false;

  if (warp == 0) {
    if (lane == 0) {
      // The weight operand does not depend on the preceding kernel: start
      // streaming it before the dependency wait (swapped mode: A is the weight,
      // read once per step, so it is loaded with the evict-first L2 policy).
      const uint64_t pol = l2_evict_first_policy();
      auto load_a = [&](void* dst, uint64_t* bar, int kx) {
        if (args.swap) tma_load_2d_hint(dst, &tmA, bar, kx, m0, pol);
        else tma_load_2d(dst, &tmA, bar, kx, m0);
      };
      if (args.pf.depth > 0) tma_prefetch_desc(&tmP);
      const int pre = args.swap ? min(nkb, STAGES) : 0;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], S::A_BYTES + S::B_BYTES);
        load_a(ringA + i * S::A_BYTES, &full[i], (kb0 + i) * BK);
      }
      pdl_wait();
      span_waited(args.span);
      // sequence-parallel prefill: the A rows must have been gathered from their owners
      if (!args.swap && !sp_wait_rows(args.sp, m0, min(m0 + BM, args.M))) atomicExch(args.err, 4);
      for (int i = 0; i < pre; ++i) tma_load_2d(ringB + i * S::B_BYTES, &tmB, &full[i], (kb0 + i) * BK, n0);
      for (int i = pre; i < nkb; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1)) {
          atomicExch(args.err, 1);
          break;
        }
        mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
        const int kx = (kb0 + i) * BK;
        load_a(ringA + s * S::A_BYTES, &full[s], kx);
        tma_load_2d(ringB + s * S::B_BYTES, &tmB, &full[s], kx, n0);
      }
      // this CTA's loads are all issued: pull its share of the next GEMM's
      // first K-blocks into L2 while the grid drains
      prefetch_next_weight(&tmP, args.pf, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                           gridDim.x * gridDim.y * gridDim.z);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      if (tr != nullptr) tr[1] = globaltimer_ns();
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
          atomicExch(args.err, 2);
          break;
        }
        if (tr != nullptr && i == 0) tr[2] = globaltimer_ns();
        tc_fence_after();
        const uint64_t ad = smem_desc_sw128(smem_u32(ringA + s * S::A_BYTES));
        const uint64_t bd = smem_desc_sw128(smem_u32(ringB + s * S::B_BYTES));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      tc_commit(tmem_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    // Fused input RMSNorm (swapped mode): 1/rms of every token of the tile,
    // overlapping the mainloop.  Two tokens per warp iteration with up to 16
    // 16-byte loads in flight per lane (one memory round trip per 2K columns).
    // Normal mode receives the values precomputed in rs_vec.
    if (args.rs_x != nullptr && args.swap) {
      for (int tt = ew; tt < BN; tt += 8) {
        float ss[2] = {0.f, 0.f};
        const int t0 = n0 + tt;
        for (int k0 = lane * 8; k0 < args.K; k0 += 256 * 8) {
          uint4 u[2][8];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int t = t0 + 4 * h;
            const bool live = tt + 4 * h < BN && t < args.N;
            const __nv_bfloat16* xr = args.rs_x + (size_t)t * args.rs_ld;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              u[h][i] = (live && k0 + 256 * i < args.K) ? *reinterpret_cast<const uint4*>(xr + k0 + 256 * i)
                                                         : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[h][i]);
#pragma unroll
              for (int j = 0; j < 8; ++j) ss[h] += bf2f(e[j]) * bf2f(e[j]);
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float v = warp_sum(ss[h]);
          if (lane == 0 && tt + 4 * h < BN) rstd_s[tt + 4 * h] = rsqrtf(v / args.K + args.rs_eps);
        }
      }
      named_bar_sync(1, 128);
    }
    const bool ready = mbar_wait(tmem_full, 0);
    if (!ready) atomicExch(args.err, 3);
    if (tr != nullptr && et == 0) tr[3] = globaltimer_ns();
    tc_fence_after();
    has_acc = ready && nkb > 0;
    if (args.rs_vec != nullptr && !args.swap && m0 + r < args.M) {
      sp_wait_rows(args.sp, m0 + r, m0 + r + 1);
      rs_row = args.rs_vec[m0 + r];
    }
    if (args.cluster) {
      // Cluster split-K: stage this slice's fp32 partial in the (now idle) A ring.
      float* part = reinterpret_cast<float*>(ringA) + (size_t)r * BN;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        if (has_acc) {
          tmem_ld16(trow + c0, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(part + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    }
  }
  // Every thread of every CTA of the cluster: the partials are now visible.
  if (args.cluster) cluster_sync_all();
  if (warp >= 2) {
    // Split-K (global path): publish this slice's partial, elect the last CTA of the tile.
    bool last = args.cluster ? cluster_rank() == 0 : true;
    if (args.splits > 1 && !args.cluster) {
      // Partial tile layout [BN/4][BM] float4: a warp's 32 rows of one 4-column
      // chunk are 512 contiguous bytes, so publishing and summing coalesce.
      float* mine = args.ws + (size_t)(tile * args.splits + split) * BM * BN;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        if (has_acc) {
          tmem_ld16(trow + c0, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(mine + ((size_t)((c0 + j) >> 2) * BM + r) * 4) =
              make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
      named_bar_sync(1, 128);
      if (et == 0) {
        // releases this CTA's partial, acquires the other slices' partials
        const int old = atomic_add_acq_rel_gpu(&args.counters[tile], 1);
        *s_flag = (old == args.splits - 1);
        if (old == args.splits - 1) args.counters[tile] = 0;
      }
      named_bar_sync(1, 128);
      last = *s_flag != 0;
    }

    if (last) {
      // Columns [c0, c0+16) of this thread's row: split-K sum, times 1/rms of
      // the token, plus bias (bias before any rounding, as in an HF linear).
      auto load_cols = [&](int c0, float* v) {
        if (args.cluster) {
          // all splits' partials of 4 columns are requested before any is summed
          const uint32_t mine = smem_u32(reinterpret_cast<float*>(ringA) + (size_t)r * BN + c0);
          const int ns = args.splits;
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            float4 f[16];
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (q < ns) f[q] = dsmem_ld_f4(dsmem_map(mine, (uint32_t)q) + 4 * j);
            float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (q < ns) {
                acc4.x += f[q].x; acc4.y += f[q].y; acc4.z += f[q].z; acc4.w += f[q].w;
              }
            v[j] = acc4.x; v[j + 1] = acc4.y; v[j + 2] = acc4.z; v[j + 3] = acc4.w;
          }
        } else if (args.splits > 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
          for (int s0 = 0; s0 < args.splits; s0 += 8) {
            float4 f[8][4];
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (s0 + q < args.splits) {
                const float* p = args.ws + (size_t)(tile * args.splits + s0 + q) * BM * BN;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  f[q][j] = __ldcg(reinterpret_cast<const float4*>(p + ((size_t)((c0 >> 2) + j) * BM + r) * 4));
              }
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (s0 + q < args.splits) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  v[4 * j] += f[q][j].x; v[4 * j + 1] += f[q][j].y; v[4 * j + 2] += f[q][j].z; v[4 * j + 3] += f[q][j].w;
                }
              }
          }
        } else if (has_acc) {
          tmem_ld16(trow + c0, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
        if (args.rs_x != nullptr || args.rs_vec != nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= args.swap ? rstd_s[c0 + j] : rs_row;
        }
        if (args.bias != nullptr) {
          if (args.swap) {
            const float b = m0 + r < args.M ? bf2f(args.bias[m0 + r]) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += b;
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += n0 + c0 + j < args.N ? bf2f(args.bias[n0 + c0 + j]) : 0.f;
          }
        }
      };

      if (!args.swap) {
        store_tile_normal<BN>(args, m0, n0, r, load_cols);
      } else if (args.epi == 0) {
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          load_cols(c0, v);
          {
            const int m = m0 + r;  // feature
            if (m < args.M) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;  // token
                if (t < args.N) {
                  float y = rbf(v[j]);
                  if (args.residual) y += bf2f(args.residual[(size_t)t * args.ldr + m]);
                  args.out[(size_t)t * args.ldo + m] = f2bf(y);
                }
              }
            }
          }
        }
      } else if (args.epi == 3) {
        // Push: result tile -> every peer's receive slot, then arrival counters.
        const PushEpi& ps = args.push;
        const int slot = (int)(ps.epoch_state[0] & 1);
        const int m = m0 + r;  // feature (swapped mode)
        // 16 tokens at a time: the tile is staged token-major in shared memory
        // (bf16), then every thread sends 16-byte runs of 8 features to each
        // peer (8x fewer NVLink stores than one element per store).
        constexpr int XS_LD = BM + 8;
        __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xch);  // [16][XS_LD]
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          load_cols(c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) xs[j * XS_LD + r] = f2bf(v[j]);
          named_bar_sync(1, 128);
          for (int q = et; q < 16 * (BM / 8); q += 128) {
            const int j = q / (BM / 8), c8 = (q % (BM / 8)) * 8;
            const int t = n0 + c0 + j, mm = m0 + c8;
            if (t < args.N && mm < args.M) {
              const uint4 val = *reinterpret_cast<const uint4*>(xs + j * XS_LD + c8);
              const size_t off = (((size_t)slot * ps.tp + ps.rank) * ps.maxT + t) * args.M + mm;
              for (int p = 0; p < ps.tp; ++p)
                *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(ps.peers[p]) + off) = val;
            }
          }
          named_bar_sync(1, 128);
        }
        __threadfence_system();
        named_bar_sync(1, 128);
        if (!ps.fused) {
          if (et == 0) {
            for (int p = 0; p < ps.tp; ++p)
              atomicAdd(reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(ps.peers[p]) + ps.flags_off) +
                            ps.rank, 1ull);
          }
        } else {
          // fused all-reduce of this 128-feature tile
          const uint64_t epoch = ps.epoch_state[0];
          if (et == 0) {
            __threadfence_system();
            for (int p = 0; p < ps.tp; ++p)
              st_release_sys_u64(reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(ps.peers[p]) + ps.tile_flags_off) +
                                     (size_t)ps.rank * ps.max_tiles + tile,
                                 epoch + 1);
          }
          int* s_ok = s_flag;
          if (et == 0) *s_ok = 1;
          named_bar_sync(1, 128);
          if (et < ps.tp) {
            const uint64_t* f = reinterpret_cast<const uint64_t*>(reinterpret_cast<const char*>(ps.peers[ps.rank]) +
                                                                  ps.tile_flags_off) + (size_t)et * ps.max_tiles + tile;
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_sys_u64(f) < epoch + 1) {
              if (globaltimer_ns() - t0 > ps.timeout_ns) {
                if (atomicCAS(ps.status, 0, 1) == 0) {
                  ps.status[1] = ps.rank;
                  ps.status[2] = et;
                  ps.status[3] = (int)epoch;
                }
                *s_ok = 0;
                break;
              }
              __nanosleep(32);
            }
          }
          named_bar_sync(1, 128);
          if (*s_ok && m < args.M) {
            // this tile's tokens [n0, t_end): 8 tokens x up to 8 sources per pass, loads in flight
            const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(ps.peers[ps.rank]) +
                                        (size_t)slot * ps.tp * ps.maxT * args.M + m;
            const int t_end = min(args.N, n0 + BN);
            for (int t0 = n0; t0 < t_end; t0 += 8) {
              __nv_bfloat16 pv[8][8];
              float res[8];
#pragma unroll
              for (int src = 0; src < 8; ++src)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  pv[src][j] = (src < ps.tp && t0 + j < t_end)
                                   ? __ldcv(recv + ((size_t)src * ps.maxT + t0 + j) * args.M)
                                   : __float2bfloat16(0.f);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                res[j] = (args.residual && t0 + j < t_end) ? bf2f(args.residual[(size_t)(t0 + j) * args.ldr + m])
                                                            : 0.f;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (t0 + j >= t_end) continue;
                float acc = 0.f;
#pragma unroll
                for (int src = 0; src < 8; ++src) acc += bf2f(pv[src][j]);
                args.out[(size_t)(t0 + j) * args.ldo + m] = f2bf(res[j] + rbf(acc));
              }
            }
          }
          // the last tile to finish advances the epoch
          named_bar_sync(1, 128);
          if (et == 0) {
            __threadfence();
            const unsigned long long done =
                atomicAdd(reinterpret_cast<unsigned long long*>(ps.epoch_state + 2), 1ull);
            if (done == (unsigned long long)(gridDim.x * gridDim.y - 1)) {
              ps.epoch_state[2] = 0;
              ps.epoch_state[0] = epoch + 1;
            }
          }
        }
      } else if (args.epi == 1) {
        // Swapped SwiGLU: tile rows [0,64) gate, [64,128) up of the same 64 features.
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          load_cols(c0, v);
          if (r >= 64) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xch[(r - 64) * XCH_LD + j] = v[j];
          }
          named_bar_sync(1, 128);
          if (r < 64) {
            const int f = m0 / 2 + r;
            if (2 * f < args.M) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;
                if (t < args.N) {
                  const float gg = rbf(v[j]), uu = rbf(xch[r * XCH_LD + j]);
                  const float sg = rbf(gg / (1.f + __expf(-gg)));
                  args.out[(size_t)t * args.ldo + f] = f2bf(sg * uu);
                }
              }
            }
          }
          named_bar_sync(1, 128);
        }
      } else {
        // Swapped QKV: rows = 128 features (one D=128 head or two D=64 heads),
        // columns = tokens.  Stage 16 tokens at a time, then one warp per token.
        const int D = args.qkv.D;
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          load_cols(c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) xch[r * XCH_LD + j] = rbf(v[j]);
          named_bar_sync(1, 128);
#pragma unroll
          for (int j = ew; j < 16; j += 4) {  // unrolled: the tokens' metadata loads overlap
            const int t = n0 + c0 + j;
            if (t >= args.N) continue;
            for (int hl = 0; hl < BM / D; ++hl) {
              const int head = (m0 + hl * D) / D;
              if (m0 + hl * D >= args.M) break;
              if (D == 128) {
                float hv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) hv[i] = xch[(hl * D + lane * 4 + i) * XCH_LD + j];
                qkv_head_store<4>(args.qkv, hv, head, t, lane);
              } else {
                float hv[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) hv[i] = xch[(hl * D + lane * 2 + i) * XCH_LD + j];
                qkv_head_store<2>(args.qkv, hv, head, t, lane);
              }
            }
          }
          named_bar_sync(1, 128);
        }
      }
    }
  }

  // keep this CTA's partial alive until the cluster leader has read it
  if (args.cluster) cluster_sync_all();
  if (tr != nullptr && et_is_epi_last(threadIdx.x)) tr[4] = globaltimer_ns();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0) span_end(args.span);
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled unavailable");
  return fn;
}

// Row-major bf16 matrix [rows, cols] with leading dimension ld (elements);
// box = [64 cols (128 bytes), box_rows], 128-byte swizzle, zero OOB fill.
CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  struct Key {
    const void* p; int64_t r, c, ld; int br;
    bool operator==(const Key& o) const { return p == o.p && r == o.r && c == o.c && ld == o.ld && br == o.br; }
  };
  struct H {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ (size_t)(k.r * 1000003 + k.c * 10007 + k.ld * 31 + k.br);
    }
  };
  static std::unordered_map<Key, CUtensorMap, H> cache;
  static std::mutex mu;
  Key key{ptr, rows, cols, ld, box_rows};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  return m;
}

// Per-device split-K scratch: fp32 partial tiles + tile counters (zeroed once;
// the last CTA of each tile re-arms its counter).
struct SplitKScratch {
  float* ws = nullptr;
  size_t ws_bytes = 0;
  int* counters = nullptr;
  size_t n_counters = 0;
  int* err = nullptr;
};

static SplitKScratch& scratch_for(int dev, size_t ws_bytes, size_t n_counters) {
  static std::mutex mu;
  static std::unordered_map<int, SplitKScratch> all;
  std::lock_guard<std::mutex> g(mu);
  SplitKScratch& s = all[dev];
  if (s.err == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&s.err, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(s.err, 0, sizeof(int)));
  }
  if (ws_bytes > s.ws_bytes) {
    // growth happens only outside graph capture (warm-up runs the same shapes first)
    if (s.ws) C10_CUDA_CHECK(cudaFree(s.ws));
    size_t b = std::max(ws_bytes, (size_t)32 << 20);
    C10_CUDA_CHECK(cudaMalloc(&s.ws, b));
    s.ws_bytes = b;
  }
  if (n_counters > s.n_counters) {
    if (s.counters) C10_CUDA_CHECK(cudaFree(s.counters));
    size_t n = std::max(n_counters, (size_t)65536);
    C10_CUDA_CHECK(cudaMalloc(&s.counters, n * sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(s.counters, 0, n * sizeof(int)));
    s.n_counters = n;
  }
  return s;
}

int* gemm_error_flag(int dev) { return scratch_for(dev, 0, 0).err; }

template <int BN, int STAGES>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid, cudaStream_t st,
                   const CUtensorMap& tp) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    attr = true;
  }
  launch_pdl_cluster(kern, grid, dim3(192), S::TOTAL, st, a.cluster ? dim3(1, 1, a.splits) : dim3(1, 1, 1), ta, tb,
                     a, tp);
}

int gemm_num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

static unsigned long long* g_span_buf = nullptr;
static int64_t g_span_cap = 0, g_span_seq = 0;
static std::vector<std::string> g_span_names;
// Profiling: record the span of every later native launch into consecutive
// 4 x u64 slots of `buf` (an empty tensor switches it off), with the launch's
// name kept on the host.  Returns the number of slots used since the previous call.
int64_t span_trace(torch::Tensor buf) {
  const int64_t used = g_span_seq;
  g_span_buf = buf.defined() && buf.numel() ? reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>()) : nullptr;
  g_span_cap = g_span_buf ? buf.numel() / 4 : 0;
  g_span_seq = 0;
  g_span_names.clear();
  return used;
}
// Names of the launches recorded since span tracing was last switched on.
std::vector<std::string> span_names() { return g_span_names; }
unsigned long long* next_span(const char* name) {
  if (g_span_buf == nullptr || g_span_seq >= g_span_cap) return nullptr;
  g_span_names.emplace_back(name ? name : "");
  return g_span_buf + 4 * (g_span_seq++);
}

static int g_forced_splits = -1;
// Tuning: force the split-K factor of later tile-per-CTA launches (0 = heuristic, -1 = environment).
void gemm_force_splits(int64_t n) { g_forced_splits = (int)n; }
static int g_forced_bn = 0;
// Tuning: force the token-tile width (16/32/64) of later decode-mode launches (0 = heuristic).
void gemm_force_bn(int64_t n) { g_forced_bn = (int)n; }

static unsigned long long* g_trace = nullptr;
// Profiling: record per-CTA phase timestamps of subsequent GEMM launches into
// `buf` (int64 [8 * CTAs]); an empty tensor switches recording off.
void gemm_set_trace(torch::Tensor buf) {
  g_trace = buf.defined() && buf.numel() ? reinterpret_cast<unsigned long long*>(buf.data_ptr<int64_t>()) : nullptr;
}

static inline const __nv_bfloat16* opt_bf(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<const __nv_bfloat16*>(t->data_ptr()) : nullptr;
}

// Common driver: picks operand roles, tile width, split-K and launches.
void launch_row_rstd(const __nv_bfloat16* x, int ld, int T, int K, float eps, float* out, cudaStream_t st);

// Sequence-parallel parameters from a CPU int64 tensor: [peers (device address of
// int64[tp]), recv_off, rs_flags_off, ag_flags_off, ag_expected, status (device
// address), timeout_ns, rank, tp, rows_per_rank, H].
static void fill_sp(GemmArgs& a, const c10::optional<torch::Tensor>& sp) {
  if (!sp.has_value() || !sp->defined()) return;
  TORCH_CHECK(!sp->is_cuda() && sp->scalar_type() == at::kLong && sp->numel() >= 11, "gemm: bad sp params");
  const int64_t* v = sp->data_ptr<int64_t>();
  SpArgs& p = a.sp;
  p.peers = reinterpret_cast<const uint64_t*>(v[0]);
  p.recv_off = v[1];
  p.rs_flags_off = v[2];
  p.ag_flags_off = v[3];
  p.ag_expected = (uint64_t)v[4];
  p.status = reinterpret_cast<int*>(v[5]);
  p.timeout_ns = (uint64_t)v[6];
  p.rank = (int)v[7];
  p.tp = (int)v[8];
  p.rows_per_rank = (int)v[9];
  p.H = (int)v[10];
  TORCH_CHECK(p.rows_per_rank > 0 && p.tp > 0, "gemm: bad sp layout");
}

// Token-tile width of a swapped (decode) GEMM of T tokens: the narrowest
// tile for <= 32 tokens; for 33-64 tokens several narrow tiles beat one
// 64-wide tile unless the weight alone fills the machine (measured on B200,
// HBM-resident weights): the smallest width whose grid fits one wave with at
// most 32 K-blocks per CTA, else the width (of those fitting one wave) with
// the fewest K-blocks per CTA.
static int swapped_bn(int T, int F, int K) {
  int BN = T <= 16 ? 16 : T <= 32 ? 32 : 64;
  const int kb_total = (K + BK - 1) / BK;
  if (T > 32) {
    const int slots2 = gemm_num_sms() * 2, mt = (F + BM - 1) / BM;
    auto kb_per_cta = [&](int bn) {
      const int tiles = mt * ((T + bn - 1) / bn);
      const int sp = std::max(1, std::min({slots2 / tiles, kb_total / 2, 16, 256 / bn}));
      return (kb_total + sp - 1) / sp;
    };
    int pick = 0;
    for (int bn : {16, 32}) {
      if (mt * ((T + bn - 1) / bn) <= slots2 && kb_per_cta(bn) <= 32) {
        pick = bn;
        break;
      }
    }
    if (!pick) {
      int best = 1 << 30;
      for (int bn : {16, 32, 64})
        if (mt * ((T + bn - 1) / bn) <= slots2 && kb_per_cta(bn) < best) {
          best = kb_per_cta(bn);
          pick = bn;
        }
    }
    if (pick) BN = pick;
  }
  if (g_forced_bn == 16 || g_forced_bn == 32 || g_forced_bn == 64) BN = g_forced_bn;
  return BN;
}

// Split-K so that one wave of resident CTAs (2 per SM for decode tiles)
// covers the machine; decode shapes have few output tiles.  The last CTA of a
// tile sums splits x BM x BN fp32 partials alone; past 256 partial columns
// that tail outweighs the shorter K loop (measured on B200 over decode and
// short-prefill shapes: BN 64 is best at 1-4 splits).
static void split_plan(int tiles, int kb_total, int BN, bool swap, int& splits, int& kbps) {
  splits = 1;
  const int slots = gemm_num_sms() * (swap ? 2 : 1);
  if (tiles < slots) splits = std::max(1, std::min({slots / tiles, kb_total / 2, 16}));
  splits = std::max(1, std::min(splits, 256 / BN));
  // With 16+ output tiles, more than 8 slices measured slower on B200 (the last
  // CTA's sum of 9-16 partials outweighs the extra streams); only a handful
  // of tiles needs up to 16 slices to fill the machine.
  if (tiles >= 16) splits = std::min(splits, 8);
  const int forced = g_forced_splits >= 0 ? g_forced_splits : [] {  // BRAID_GEMM_SPLITS=n forces the factor
    static const int env = [] {
      const char* e = getenv("BRAID_GEMM_SPLITS");
      return e ? atoi(e) : 0;
    }();
    return env;
  }();
  if (forced > 0) splits = std::max(1, std::min(forced, kb_total));
  kbps = (kb_total + splits - 1) / splits;
  splits = (kb_total + kbps - 1) / kbps;
}

// ---- cross-kernel weight prefetch (see PrefetchArgs in common.cuh)
// The host names the weight of the GEMM that follows the next launch
// (gemm_prefetch_next); that launch receives its tensor map and split plan and
// pulls the leading K-blocks of every K-slice into L2 (BRAID_PREFETCH_MB caps
// the bytes per boundary, 0 switches it off).
struct PendingPrefetch {
  bool set = false;
  CUtensorMap map;
  PrefetchArgs pf;
};
static PendingPrefetch g_prefetch;

static size_t prefetch_budget() {
  static const size_t b = [] {
    const char* e = getenv("BRAID_PREFETCH_MB");
    return (size_t)(e ? atof(e) : 48.0) << 20;
  }();
  return b;
}

// Returns the K-blocks per slice that the next launch will prefetch after `skip`.
int64_t gemm_prefetch_next(torch::Tensor w, int64_t T, int64_t skip) {
  g_prefetch.set = false;
  if (!w.defined() || !w.is_cuda() || w.dim() != 2 || T < 1 || T > 64 || prefetch_budget() == 0) return 0;
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.stride(1) == 1, "gemm_prefetch_next: bf16 row-major weight");
  const int F = w.size(0), K = w.size(1);
  const int BN = swapped_bn((int)T, F, K);
  const int m_tiles = (F + BM - 1) / BM, kb_total = (K + BK - 1) / BK;
  int splits, kbps;
  split_plan(m_tiles * (((int)T + BN - 1) / BN), kb_total, BN, true, splits, kbps);
  PrefetchArgs pf;
  pf.m_tiles = m_tiles;
  pf.splits = splits;
  pf.kbps = kbps;
  pf.kb_total = kb_total;
  pf.skip = (int)std::max<int64_t>(0, skip);
  const size_t box = (size_t)BM * BK * 2;
  const size_t per_depth = (size_t)m_tiles * splits * box;
  pf.depth = (int)std::min<size_t>(std::max(0, kbps - pf.skip),
                                   std::max<size_t>(1, prefetch_budget() / per_depth));
  if (pf.depth <= 0) return 0;
  g_prefetch.map = make_tmap(w.data_ptr(), F, K, w.stride(0), BM);
  g_prefetch.pf = pf;
  g_prefetch.set = true;
  return pf.depth;
}

// Consumed by the next launch: its prefetch arguments and tensor map
// (`fallback` when nothing is pending; depth 0 then disables the prefetch).
PrefetchArgs take_prefetch(CUtensorMap* map, const CUtensorMap& fallback) {
  PrefetchArgs pf{};
  if (g_prefetch.set) {
    pf = g_prefetch.pf;
    *map = g_prefetch.map;
    g_prefetch.set = false;
  } else {
    *map = fallback;
  }
  return pf;
}

static int64_t run_gemm(GemmArgs& a, const torch::Tensor& x, const torch::Tensor& w, bool fused_rms) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm: bf16 only");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "gemm: inner dim must be contiguous");
  const int T = x.size(0), K = x.size(1), F = w.size(0);
  TORCH_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0, "gemm: K and strides must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0, "gemm: 16-byte aligned operands required");
  if (a.epi == 1) TORCH_CHECK(F % 128 == 0, "gemm: swiglu weight rows must be a multiple of 128");
  if (T == 0) return 0;
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  a.K = K;
  a.rs_x = fused_rms ? reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()) : nullptr;
  a.rs_ld = x.stride(0);
  const int kb_total = (K + BK - 1) / BK;
  const bool swap = T <= 64 && a.epi != 4 && a.rs_vec == nullptr && a.sp.peers == nullptr;
  a.swap = swap;
  int BN, m_tiles, n_tiles;
  if (swap) {
    BN = swapped_bn(T, F, K);
    a.M = F;
    a.N = T;
    m_tiles = (F + BM - 1) / BM;
    n_tiles = (T + BN - 1) / BN;
  } else {
    BN = (F >= 4096 && T >= 512 && a.epi != 2) ? 256 : 128;
    a.M = T;
    a.N = F;
    m_tiles = (T + BM - 1) / BM;
    n_tiles = (F + BN - 1) / BN;
  }
  const int tiles = m_tiles * n_tiles;
  // reduce-scatter epilogue: partial tiles this rank (as row owner) receives from every source;
  // push epilogue (epi 3): every output tile bumps each peer's counter once
  int64_t arrivals = a.epi == 3 ? tiles : 0;
  if (a.epi == 4) {
    TORCH_CHECK(a.sp.peers != nullptr && a.sp.H == F, "gemm: epi 4 needs sequence-parallel params");
    const int r0 = a.sp.rank * a.sp.rows_per_rank, r1 = std::min(T, r0 + a.sp.rows_per_rank);
    if (r1 > r0) arrivals = (int64_t)n_tiles * ((r1 - 1) / BM - r0 / BM + 1);
  }
  static const bool persist_on = [] {  // tuning knob: BRAID_GEMM_PERSISTENT=0 keeps one tile per CTA
    const char* e = getenv("BRAID_GEMM_PERSISTENT");
    return !(e && e[0] == '0');
  }();
  if (!swap && persist_on && tiles >= gemm_num_sms()) {
    torch::Tensor rstd;
    if (fused_rms && a.rs_vec == nullptr) {
      rstd = torch::empty({T}, x.options().dtype(at::kFloat));
      launch_row_rstd(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), T, K, a.rs_eps,
                      rstd.data_ptr<float>(), st);
      a.rs_vec = rstd.data_ptr<float>();
    }
    a.rs_x = nullptr;
    a.splits = 1;
    a.kb_per_split = kb_total;
    a.cluster = 0;
    a.err = scratch_for(x.get_device(), 0, 0).err;
    CUtensorMap ta = make_tmap(x.data_ptr(), T, K, x.stride(0), BM);
    CUtensorMap tb = make_tmap(w.data_ptr(), F, K, w.stride(0), BN);
    a.span = next_span(a.epi == 2 ? "gemm_qkv_persistent" : a.epi == 1 ? "gemm_swiglu_persistent"
                       : a.epi == 4 ? "gemm_rs_persistent" : "gemm_persistent");
    launch_gemm_persistent(ta, tb, a, BN, st);
    return arrivals;
  }
  torch::Tensor rstd_tmp;
  if (!swap && a.rs_x != nullptr && a.rs_vec == nullptr) {
    rstd_tmp = torch::empty({T}, x.options().dtype(at::kFloat));
    launch_row_rstd(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), T, K, a.rs_eps,
                    rstd_tmp.data_ptr<float>(), st);
    a.rs_vec = rstd_tmp.data_ptr<float>();
  }
  if (a.rs_vec != nullptr) a.rs_x = nullptr;
  int splits, kbps;
  split_plan(tiles, kb_total, BN, swap, splits, kbps);
  a.splits = splits;
  a.kb_per_split = kbps;
  // Optional (BRAID_GEMM_CLUSTER=1): up to 16 K-slices reduce through
  // distributed shared memory inside one thread-block cluster.  Measured
  // slower than the global workspace on B200 for decode shapes, so off by default.
  static const bool use_cluster = [] {
    const char* e = getenv("BRAID_GEMM_CLUSTER");
    return e && e[0] == '1';
  }();
  a.cluster = (splits > 1 && splits <= 16 && use_cluster) ? 1 : 0;
  const int dev = x.get_device();
  SplitKScratch& sc = scratch_for(dev, splits > 1 ? (size_t)tiles * splits * BM * BN * 4 : 0, tiles);
  a.ws = sc.ws;
  a.counters = sc.counters;
  a.err = sc.err;
  a.trace = g_trace;
  a.span = next_span(a.epi == 2 ? "gemm_qkv" : a.epi == 1 ? "gemm_swiglu" : a.epi == 3 ? "gemm_push"
                     : a.epi == 4 ? "gemm_rs" : "gemm");
  dim3 grid(m_tiles, n_tiles, splits);
  const void* pa = swap ? w.data_ptr() : x.data_ptr();
  const void* pb = swap ? x.data_ptr() : w.data_ptr();
  const int64_t ra = swap ? F : T, rb = swap ? T : F;
  const int64_t lda = swap ? w.stride(0) : x.stride(0), ldb = swap ? x.stride(0) : w.stride(0);
  CUtensorMap ta = make_tmap(pa, ra, K, lda, BM);
  CUtensorMap tb = make_tmap(pb, rb, K, ldb, BN);
  CUtensorMap tp;
  a.pf = take_prefetch(&tp, ta);
  if (!swap) a.pf.depth = 0;
  switch (BN) {
    case 16: launch<16, 4>(ta, tb, a, grid, st, tp); break;
    case 32: launch<32, 4>(ta, tb, a, grid, st, tp); break;
    case 64: launch<64, 4>(ta, tb, a, grid, st, tp); break;
    case 128: launch<128, 6>(ta, tb, a, grid, st, tp); break;
    default: launch<256, 4>(ta, tb, a, grid, st, tp); break;
  }
  return arrivals;
}

// out = rms?(x) @ w^T (+bias) (+residual); epi: 0 plain, 1 swiglu (w block-interleaved).
// rs_eps >= 0 enables the fused input RMSNorm (w must carry the folded norm weight).
// rs_vec (float [T]) supplies precomputed 1/rms per token instead; sp carries the
// sequence-parallel parameters (epi 4 = reduce-scatter push, and the all-gather
// wait before A rows are read).  Returns, for epi 4, the partial tiles this rank
// receives from each source.
int64_t gemm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
             c10::optional<torch::Tensor> residual, int64_t epi, double rs_eps, c10::optional<torch::Tensor> rs_vec,
             c10::optional<torch::Tensor> sp) {
  TORCH_CHECK(out.is_cuda() && out.stride(1) == 1, "gemm: out must be row-contiguous");
  GemmArgs a{};
  a.epi = (int)epi;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.bias = opt_bf(bias);
  a.residual = opt_bf(residual);
  a.ldr = a.residual ? residual->stride(0) : 0;
  a.rs_eps = (float)rs_eps;
  if (rs_vec.has_value() && rs_vec->defined()) {
    TORCH_CHECK(rs_vec->scalar_type() == at::kFloat && rs_vec->numel() >= x.size(0), "gemm: rs_vec");
    a.rs_vec = rs_vec->data_ptr<float>();
  }
  fill_sp(a, sp);
  return run_gemm(a, x, w, rs_eps >= 0 && a.rs_vec == nullptr);
}

// qkv = rms?(x) @ w^T (+bias), then per-head q/k RMSNorm, RoPE(k) and the
// paged KV append, all in the epilogue; q is written unrotated to q_out.
void gemm_qkv(torch::Tensor q_out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
              double rs_eps, torch::Tensor positions, torch::Tensor slots, torch::Tensor kv,
              c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double head_eps,
              torch::Tensor cos, torch::Tensor sin, int64_t Hq, int64_t Hkv, int64_t D, bool use_rope,
              c10::optional<torch::Tensor> rs_vec, c10::optional<torch::Tensor> sp) {
  TORCH_CHECK(D == 64 || D == 128, "gemm_qkv: head_dim must be 64 or 128");
  TORCH_CHECK(w.size(0) == (Hq + 2 * Hkv) * D, "gemm_qkv: weight rows != (Hq + 2 Hkv) * D");
  TORCH_CHECK(kv.is_contiguous() && kv.size(2) == Hkv && kv.size(4) == D, "gemm_qkv: cache layout");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt, "gemm_qkv: int32 metadata");
  GemmArgs a{};
  a.epi = 2;
  a.bias = opt_bf(bias);
  a.rs_eps = (float)rs_eps;
  QkvEpi& q = a.qkv;
  q.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  q.kv = reinterpret_cast<__nv_bfloat16*>(kv.data_ptr());
  q.slots = slots.data_ptr<int>();
  q.positions = positions.data_ptr<int>();
  q.q_norm = opt_bf(q_norm);
  q.k_norm = opt_bf(k_norm);
  q.cos = cos.data_ptr<float>();
  q.sin = sin.data_ptr<float>();
  q.Hq = Hq;
  q.Hkv = Hkv;
  q.D = D;
  q.PS = kv.size(3);
  q.use_rope = use_rope ? 1 : 0;
  q.eps = (float)head_eps;
  q.num_slots = (int)(kv.size(0) * kv.size(3));
  q.rope_len = (int)cos.size(0);
  if (rs_vec.has_value() && rs_vec->defined()) {
    TORCH_CHECK(rs_vec->scalar_type() == at::kFloat && rs_vec->numel() >= x.size(0), "gemm_qkv: rs_vec");
    a.rs_vec = rs_vec->data_ptr<float>();
  }
  fill_sp(a, sp);
  run_gemm(a, x, w, rs_eps >= 0 && a.rs_vec == nullptr);
}

int64_t gemm_check_error(int64_t device) {
  int* e = gemm_error_flag((int)device);
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, e, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) C10_CUDA_CHECK(cudaMemset(e, 0, sizeof(int)));
  return h;
}

}  // namespace braid

namespace braid {
// Row-parallel GEMM whose epilogue pushes the result to every tensor-parallel
// peer (decode shapes).  Returns the number of tiles pushed, i.e. the arrivals
// each peer must count from this rank for this call.
// residual += sum over the TP group of x @ w^T, reduced inside this GEMM (see PushEpi).
void gemm_allreduce_add(torch::Tensor residual, torch::Tensor x, torch::Tensor w, torch::Tensor peers,
                        int64_t flags_off, int64_t tile_flags_off, int64_t max_tiles, int64_t rank, int64_t tp,
                        int64_t maxT, torch::Tensor epoch_state, torch::Tensor status, double timeout_s) {
  TORCH_CHECK(x.size(0) <= 64 && x.size(0) <= maxT, "gemm_allreduce_add: decode shapes only (<= 64 tokens)");
  TORCH_CHECK((w.size(0) + BM - 1) / BM * ((x.size(0) + 15) / 16) <= max_tiles,
              "gemm_allreduce_add: too many output tiles for the flag area");
  TORCH_CHECK(tp >= 1 && tp <= 8, "gemm_allreduce_add: one NVLink domain of at most 8 ranks");
  TORCH_CHECK(w.size(0) % 8 == 0, "gemm_allreduce_add: output features must be a multiple of 8");
  TORCH_CHECK(residual.is_contiguous() && residual.size(0) == x.size(0) && residual.size(1) == w.size(0));
  GemmArgs a{};
  a.epi = 3;
  a.out = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  a.ldo = residual.stride(0);
  a.residual = a.out;
  a.ldr = a.ldo;
  a.push.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.push.flags_off = flags_off;
  a.push.epoch_state = reinterpret_cast<uint64_t*>(epoch_state.data_ptr<int64_t>());
  a.push.rank = rank;
  a.push.tp = tp;
  a.push.maxT = maxT;
  a.push.fused = 1;
  a.push.tile_flags_off = tile_flags_off;
  a.push.max_tiles = (int)max_tiles;
  a.push.status = status.data_ptr<int>();
  a.push.timeout_ns = (uint64_t)(timeout_s * 1e9);
  run_gemm(a, x, w, false);
}

int64_t gemm_push(torch::Tensor x, torch::Tensor w, torch::Tensor peers, int64_t flags_off, int64_t rank, int64_t tp,
                  int64_t maxT, torch::Tensor epoch_state) {
  TORCH_CHECK(x.size(0) <= 64 && x.size(0) <= maxT, "gemm_push: decode shapes only (<= 64 tokens)");
  TORCH_CHECK(w.size(0) % 8 == 0, "gemm_push: output features must be a multiple of 8 (16-byte peer stores)");
  GemmArgs a{};
  a.epi = 3;
  a.push.peers = reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>());
  a.push.flags_off = flags_off;
  a.push.epoch_state = reinterpret_cast<uint64_t*>(epoch_state.data_ptr<int64_t>());
  a.push.rank = rank;
  a.push.tp = tp;
  a.push.maxT = maxT;
  return run_gemm(a, x, w, false);
}
}  // namespace braid

// ===================================================================
// Allocation-free entry point (declared and documented in gemm_noalloc.h).
// ===================================================================
#include "gemm_noalloc.h"

namespace braid {
namespace noalloc {

struct Scratch {
  float partial[BRAID_NOALLOC_PARTIAL_BYTES / sizeof(float)];
  int counters[BRAID_NOALLOC_MAX_TILES];
  int err;
};
// One fixed scratch per device for the whole process lifetime.
static __device__ __align__(256) Scratch g_scratch;

constexpr int kMaxDevices = 64;
// Device address of g_scratch per device (set once under g_setup_mu).
static std::atomic<Scratch*> g_addr[kMaxDevices];
// Per device: bit i set once the kernel for token-tile width 16 << i has its
// shared-memory attribute (set under g_setup_mu).
static std::atomic<unsigned> g_attr_done[kMaxDevices];
static std::mutex g_setup_mu;
static thread_local char g_msg[256] = "";

static int fail(int code, const char* what) {
  snprintf(g_msg, sizeof(g_msg), "braid_gemm_noalloc: %s", what);
  return code;
}

static CUtensorMap encode(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, bool* ok) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *ok = r == CUDA_SUCCESS;
  return m;
}

// First use on `dev` (current): resolve the array's device address and clear
// it on the caller's stream, then wait for the clear, so no later launch on
// any stream can overtake it.
static Scratch* setup(int dev, cudaStream_t st, int* code) {
  Scratch* sc = g_addr[dev].load(std::memory_order_acquire);
  if (sc != nullptr) return sc;
  std::lock_guard<std::mutex> g(g_setup_mu);
  sc = g_addr[dev].load(std::memory_order_relaxed);
  if (sc != nullptr) return sc;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
  if (e == cudaSuccess && p != nullptr) e = cudaMemsetAsync(p, 0, sizeof(Scratch), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess || p == nullptr) {
    *code = fail(6, cudaGetErrorString(e));
    return nullptr;
  }
  sc = static_cast<Scratch*>(p);
  g_addr[dev].store(sc, std::memory_order_release);
  return sc;
}

template <int BN>
static cudaError_t launch_plain(int dev, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid,
                                cudaStream_t st) {
  using S = GemmSmem<BN, 4>;
  auto kern = gemm_tcgen05_kernel<BN, 4>;
  const unsigned bit = BN == 16 ? 1u : BN == 32 ? 2u : 4u;
  if (!(g_attr_done[dev].load(std::memory_order_acquire) & bit)) {
    std::lock_guard<std::mutex> g(g_setup_mu);
    if (!(g_attr_done[dev].load(std::memory_order_relaxed) & bit)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL);
      if (e != cudaSuccess) return e;
      g_attr_done[dev].fetch_or(bit, std::memory_order_release);
    }
  }
  kern<<<grid, 192, S::TOTAL, st>>>(ta, tb, a, ta);  // a.pf.depth == 0: no prefetch
  return cudaGetLastError();
}

}  // namespace noalloc
}  // namespace braid

extern "C" const char* braid_gemm_noalloc_last_error(void) { return braid::noalloc::g_msg; }

extern "C" int braid_gemm_noalloc_check_error(void* stream) {
  using namespace braid::noalloc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  Scratch* sc = g_addr[dev].load(std::memory_order_acquire);
  if (sc == nullptr) return 0;  // never called on this device
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
  if (cudaMemcpy(&h, &sc->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (h != 0 && cudaMemset(&sc->err, 0, sizeof(int)) != cudaSuccess) return -1;
  return h;
}

extern "C" int braid_gemm_noalloc(void* out, const void* x, const void* w, const void* bias, const void* residual,
                                  int T, int N, int K, int ldo, int ldx, int ldw, int ldr, float rs_eps,
                                  void* stream) {
  using namespace braid;
  using namespace braid::noalloc;
  g_msg[0] = 0;
  if (out == nullptr || x == nullptr || w == nullptr) return fail(1, "null operand");
  if (T < 1 || T > BRAID_NOALLOC_MAX_TOKENS) return fail(2, "T must be in [1, 64] (decode shapes only)");
  if (N < 1 || K < 8 || K % 8 || ldx % 8 || ldw % 8 || ldx < K || ldw < K || ldo < N)
    return fail(3, "K and the row strides must be multiples of 8 and at least the row length");
  if (((uintptr_t)x | (uintptr_t)w) & 15) return fail(4, "x and w must be 16-byte aligned");
  if (residual != nullptr && ldr < N) return fail(3, "residual stride shorter than N");
  const int m_tiles = (N + BM - 1) / BM;
  if (m_tiles > BRAID_NOALLOC_MAX_TILES) return fail(10, "N exceeds the tile-counter capacity (2097152 rows)");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(5, "no current CUDA device");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int code = 0;
  Scratch* sc = setup(dev, st, &code);
  if (sc == nullptr) return code;
  GemmArgs a{};
  a.K = K;
  a.swap = 1;
  a.epi = 0;
  a.M = N;
  a.N = T;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.ldr = ldr;
  a.rs_x = rs_eps >= 0.f ? static_cast<const __nv_bfloat16*>(x) : nullptr;
  a.rs_ld = ldx;
  a.rs_eps = rs_eps;
  const int BN = T <= 16 ? 16 : T <= 32 ? 32 : 64;
  const int tiles = m_tiles;
  const int kb_total = (K + BK - 1) / BK;
  // same split-K rule as the regular entry point (one resident wave, at most
  // 16 slices and 256 / BN partial columns for the last CTA to sum) ...
  int splits = 1;
  const int slots = gemm_num_sms() * 2;
  if (tiles < slots) splits = std::max(1, std::min({slots / tiles, kb_total / 2, 16}));
  splits = std::max(1, std::min(splits, 256 / BN));
  if (tiles >= 16) splits = std::min(splits, 8);
  // ... and never more partial space than the fixed array holds
  while (splits > 1 && (size_t)tiles * splits * BM * BN * 4 > BRAID_NOALLOC_PARTIAL_BYTES) --splits;
  int kbps = (kb_total + splits - 1) / splits;
  splits = (kb_total + kbps - 1) / kbps;
  a.splits = splits;
  a.kb_per_split = kbps;
  a.ws = sc->partial;
  a.counters = sc->counters;
  a.err = &sc->err;
  // the tile counters must start at zero (the last CTA of each tile re-arms
  // its counter; clearing also recovers from a call that timed out)
  if (splits > 1 && cudaMemsetAsync(sc->counters, 0, sizeof(int) * tiles, st) != cudaSuccess)
    return fail(7, "clearing the scratch counters failed");
  bool ok1 = false, ok2 = false;
  CUtensorMap ta = encode(w, N, K, ldw, BM, &ok1);
  CUtensorMap tb = encode(x, T, K, ldx, BN, &ok2);
  if (!ok1 || !ok2) return fail(8, "tensor map encoding failed");
  dim3 grid(m_tiles, 1, splits);
  cudaError_t e;
  switch (BN) {
    case 16: e = launch_plain<16>(dev, ta, tb, a, grid, st); break;
    case 32: e = launch_plain<32>(dev, ta, tb, a, grid, st); break;
    default: e = launch_plain<64>(dev, ta, tb, a, grid, st); break;
  }
  if (e != cudaSuccess) return fail(9, cudaGetErrorString(e));
  return 0;
}

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_gemm)
}  // namespace braid
