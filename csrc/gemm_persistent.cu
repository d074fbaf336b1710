// Persistent tcgen05 GEMM for prefill-sized problems (sm_100a):
//   D[M, N] = A[M, K] * B[N, K]^T, A = activations [tokens, K], B = weight.
//
// One CTA per SM walks the output tiles tile = blockIdx.x + i * gridDim.x
// (M index fastest, so the CTAs resident at one time share a few weight
// column blocks and the weight streams from HBM about once).  Warp roles:
//   warp 0      TMA producer: A/B K-blocks into a STAGES-deep mbarrier ring
//               that runs continuously across the CTA's tiles
//   warp 1      MMA issuer (one lane): tcgen05.mma 128 x BN x 16 into one of
//               two TMEM accumulators (2 x BN columns), commits the ring slot
//               after each K-block and the accumulator after each tile
//   warps 2..5  epilogue: drain accumulator i & 1 with tcgen05.ld while the MMA
//               warp already fills the other one, then release it
// so the epilogue of tile i overlaps the mainloop of tile i + 1.  The per-token
// 1/rms of a fused input RMSNorm comes precomputed (rs_vec; row_rstd_kernel
// below, or the sequence-parallel reduce kernel which pushes it with the rows).
// Every wait is bounded; a timeout sets the GEMM error word and unwinds.
//
// No reference counterpart beyond what the tile-per-CTA kernel replaces (the
// Triton/cuBLAS linears of braidinfer/layers/linear.py).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_types.cuh"
#include "launch.cuh"

namespace braid {

template <int BN, int STAGES>
struct PersistSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int BAR_OFF = RING;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 4) * 8 + 16 + 1024;  // +1024 alignment slack
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1) gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                  const __grid_constant__ CUtensorMap tmB,
                                                                  const GemmArgs args) {
  using S = PersistSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ringA = smem;
  uint8_t* ringB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] accumulator ready (MMA -> epilogue)
  uint64_t* tempty = tfull + 2;      // [2] accumulator drained (epilogue -> MMA)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (args.M + BM - 1) / BM, n_tiles = (args.N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int kb_total = (args.K + BK - 1) / BK;
  constexpr uint32_t TMEM_COLS = 2 * BN;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
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
  if (threadIdx.x == 0) span_start(args.span);

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      span_waited(args.span);
      uint32_t g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
        if (!sp_wait_rows(args.sp, m0, min(m0 + BM, args.M))) atomicExch(args.err, 4);
        for (int kb = 0; kb < kb_total; ++kb, ++g) {
          const int s = g % STAGES;
          if (g >= STAGES && !mbar_wait(&empty[s], ((g / STAGES) & 1) ^ 1)) {
            atomicExch(args.err, 1);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
          tma_load_2d(ringA + s * S::A_BYTES, &tmA, &full[s], kb * BK, m0);
          tma_load_2d(ringB + s * S::B_BYTES, &tmB, &full[s], kb * BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      uint32_t g = 0;
      bool ok = true;
      int i = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++i) {
        const int acc = i & 1;
        if (i >= 2 && !mbar_wait(&tempty[acc], ((i >> 1) & 1) ^ 1)) {
          atomicExch(args.err, 5);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kb_total; ++kb, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait(&full[s], (g / STAGES) & 1)) {
            atomicExch(args.err, 2);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = smem_desc_sw128(smem_u32(ringA + s * S::A_BYTES));
          const uint64_t bd = smem_desc_sw128(smem_u32(ringB + s * S::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) tc_mma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    const int wq = warp & 3;       // TMEM lane quarter this warp may access
    const int r = wq * 32 + lane;  // tile row owned by this thread
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
      const int acc = i & 1;
      const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
      if (!mbar_wait(&tfull[acc], (i >> 1) & 1)) {
        atomicExch(args.err, 3);
        break;
      }
      tc_fence_after();
      float rs_row = 1.f;
      if (args.rs_vec != nullptr && m0 + r < args.M) {
        sp_wait_rows(args.sp, m0 + r, m0 + r + 1);
        rs_row = args.rs_vec[m0 + r];
      }
      __syncwarp();
      const uint32_t trow = tmem + acc * BN + ((uint32_t)(wq * 32) << 16);
      auto load_cols = [&](int c0, float* v) {
        tmem_ld16(trow + c0, v);
        tc_wait_ld();
        if (args.rs_vec != nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= rs_row;
        }
        if (args.bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += n0 + c0 + j < args.N ? bf2f(args.bias[n0 + c0 + j]) : 0.f;
        }
      };
      store_tile_normal<BN>(args, m0, n0, r, load_cols);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0) span_end(args.span);
}

template <int BN, int STAGES>
static void launch_p(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, cudaStream_t st) {
  using S = PersistSmem<BN, STAGES>;
  auto kern = gemm_persistent_kernel<BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr = true;
  }
  const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  launch_pdl(kern, dim3(std::min(tiles, gemm_num_sms())), dim3(192), S::TOTAL, st, ta, tb, a);
}

void launch_gemm_persistent(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int BN,
                            cudaStream_t st) {
  if (BN == 256)
    launch_p<256, 4>(ta, tb, a, st);
  else
    launch_p<128, 6>(ta, tb, a, st);
}

// 1/rms of each row of x [T, K] (bf16) in fp32: one warp per row.
__global__ void row_rstd_kernel(const __nv_bfloat16* __restrict__ x, int ld, int T, int K, float eps,
                                float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const __nv_bfloat16* xr = x + (size_t)row * ld;
  float ss = 0.f;
  for (int k0 = lane * 8; k0 < K; k0 += 256 * 8) {
    uint4 u[8];  // 8 loads in flight per lane
#pragma unroll
    for (int i = 0; i < 8; ++i)
      u[i] = k0 + 256 * i < K ? *reinterpret_cast<const uint4*>(xr + k0 + 256 * i) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += bf2f(e[j]) * bf2f(e[j]);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) out[row] = rsqrtf(ss / K + eps);
}

void launch_row_rstd(const __nv_bfloat16* x, int ld, int T, int K, float eps, float* out, cudaStream_t st) {
  launch_pdl(row_rstd_kernel, dim3((T + 7) / 8), dim3(256), 0, st, x, ld, T, K, eps, out);
}

// out[T] = 1/rms(x[t, :]) (float32), eps as in the model's RMSNorm.
void row_rstd(torch::Tensor x, double eps, torch::Tensor out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1);
  TORCH_CHECK(x.size(1) % 8 == 0 && x.stride(0) % 8 == 0, "row_rstd: rows must be 16-byte aligned");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= x.size(0));
  if (x.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  launch_row_rstd(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), x.size(0), x.size(1),
                  (float)eps, out.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
}

}  // namespace braid

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_gemm_persistent)
}  // namespace braid
