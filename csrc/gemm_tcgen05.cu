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

#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace braid {

struct GemmArgs {
  int M, N, K;        // A rows, B rows, reduction length
  int swap;           // 1: A is the weight, output written transposed
  int epi;            // 0 plain, 1 swiglu
  __nv_bfloat16* out;
  int ldo;
  const __nv_bfloat16* bias;      // indexed by feature
  const __nv_bfloat16* residual;  // same layout as out
  int ldr;
  int splits;
  int kb_per_split;
  float* ws;          // split-K partials
  int* counters;      // one per output tile, kept at zero between launches
  int* err;           // error flag (bounded-wait timeout)
};

constexpr int BM = 128;
constexpr int BK = 64;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int XCH = BN <= 64 ? 64 * (BN + 1) * 4 : 0;  // swapped-SwiGLU exchange
  static constexpr int BAR_OFF = RING + XCH;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 1) * 8 + 16 + 1024;  // +1024 alignment slack
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1) gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                                                               const __grid_constant__ CUtensorMap tmB,
                                                               const GemmArgs args) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ringA = smem;
  uint8_t* ringB = smem + STAGES * S::A_BYTES;
  float* xch = reinterpret_cast<float*>(smem + S::RING);
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

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1)) {
          atomicExch(args.err, 1);
          break;
        }
        mbar_arrive_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
        const int kx = (kb0 + i) * BK;
        tma_load_2d(ringA + s * S::A_BYTES, &tmA, &full[s], kx, m0);
        tma_load_2d(ringB + s * S::B_BYTES, &tmB, &full[s], kx, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
          atomicExch(args.err, 2);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = smem_desc_sw128(smem_u32(ringA + s * S::A_BYTES));
        const uint64_t bd = smem_desc_sw128(smem_u32(ringB + s * S::B_BYTES));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      (void)ok;
      tc_commit(tmem_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;             // TMEM lane quarter this warp may access
    const int r = wq * 32 + lane;        // row of the tile owned by this thread
    const int et = threadIdx.x - 64;     // 0..127 epilogue thread id
    const bool ready = mbar_wait(tmem_full, 0);
    if (!ready) atomicExch(args.err, 3);
    tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)(wq * 32) << 16);
    const int tile = m_tile * gridDim.y + n_tile;
    const bool has_acc = ready && nkb > 0;

    // Split-K: publish this slice's partial, elect the last CTA of the tile.
    bool last = true;
    if (args.splits > 1) {
      float* mine = args.ws + ((size_t)(tile * args.splits + split) * BM + r) * BN;
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
        for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(mine + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (et == 0) {
        const int old = atomicAdd(&args.counters[tile], 1);
        *s_flag = (old == args.splits - 1);
        if (old == args.splits - 1) args.counters[tile] = 0;
      }
      named_bar_sync(1, 128);
      last = *s_flag != 0;
      __threadfence();
    }

    if (last) {
      // Load columns [c0, c0+16) of this thread's row, summed over split-K slices.
      auto load_cols = [&](int c0, float* v) {
        if (args.splits > 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
          for (int s = 0; s < args.splits; ++s) {
            const float* p = args.ws + ((size_t)(tile * args.splits + s) * BM + r) * BN + c0;
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              const float4 q = __ldcg(reinterpret_cast<const float4*>(p + j));
              v[j] += q.x; v[j + 1] += q.y; v[j + 2] += q.z; v[j + 3] += q.w;
            }
          }
        } else if (has_acc) {
          tmem_ld16(trow + c0, v);
          tc_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
      };

      if (args.epi == 0) {
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          load_cols(c0, v);
          if (!args.swap) {
            const int m = m0 + r;
            if (m < args.M) {
              __nv_bfloat16* o = args.out + (size_t)m * args.ldo;
              const __nv_bfloat16* res = args.residual ? args.residual + (size_t)m * args.ldr : nullptr;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int n = n0 + c0 + j;
                if (n < args.N) {
                  float y = v[j];
                  if (args.bias) y += bf2f(args.bias[n]);
                  y = rbf(y);
                  if (res) y += bf2f(res[n]);
                  o[n] = f2bf(y);
                }
              }
            }
          } else {
            const int m = m0 + r;  // feature
            if (m < args.M) {
              const float b = args.bias ? bf2f(args.bias[m]) : 0.f;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;  // token
                if (t < args.N) {
                  float y = rbf(v[j] + b);
                  if (args.residual) y += bf2f(args.residual[(size_t)t * args.ldr + m]);
                  args.out[(size_t)t * args.ldo + m] = f2bf(y);
                }
              }
            }
          }
        }
      } else if (!args.swap) {
        // Normal SwiGLU: per 128-column block, gate = cols [0,64), up = [64,128).
        const int m = m0 + r;
        for (int blk = 0; blk < BN / 128; ++blk) {
          for (int c0 = 0; c0 < 64; c0 += 16) {
            float g[16], u[16];
            load_cols(blk * 128 + c0, g);
            load_cols(blk * 128 + 64 + c0, u);
            if (m < args.M) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int f = (n0 + blk * 128) / 2 + c0 + j;
                if (2 * f < args.N) {
                  const float gg = rbf(g[j]), uu = rbf(u[j]);
                  const float sg = rbf(gg / (1.f + __expf(-gg)));
                  args.out[(size_t)m * args.ldo + f] = f2bf(sg * uu);
                }
              }
            }
          }
        }
      } else {
        // Swapped SwiGLU: tile rows [0,64) gate, [64,128) up of the same 64 features.
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          load_cols(c0, v);
          if (r >= 64) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xch[(r - 64) * (BN + 1) + c0 + j] = v[j];
          }
          named_bar_sync(1, 128);
          if (r < 64) {
            const int f = m0 / 2 + r;
            if (2 * f < args.M) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int t = n0 + c0 + j;
                if (t < args.N) {
                  const float gg = rbf(v[j]), uu = rbf(xch[r * (BN + 1) + c0 + j]);
                  const float sg = rbf(gg / (1.f + __expf(-gg)));
                  args.out[(size_t)t * args.ldo + f] = f2bf(sg * uu);
                }
              }
            }
          }
          named_bar_sync(1, 128);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
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
static CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
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
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, dim3 grid, cudaStream_t st) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES>;
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr = true;
  }
  kern<<<grid, 192, S::TOTAL, st>>>(ta, tb, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// out = x @ w^T (+bias) (+residual) ;  epi: 0 plain, 1 swiglu (w block-interleaved)
void gemm(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
          c10::optional<torch::Tensor> residual, int64_t epi) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm: bf16 only");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm: shape mismatch");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1, "gemm: inner dim must be contiguous");
  const int T = x.size(0), K = x.size(1), F = w.size(0);
  TORCH_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0, "gemm: K and strides must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0, "gemm: 16-byte aligned operands required");
  if (epi == 1) TORCH_CHECK(F % 128 == 0, "gemm: swiglu weight rows must be a multiple of 128");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  GemmArgs a{};
  a.K = K;
  a.epi = (int)epi;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.bias = bias.has_value() && bias->defined() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  a.residual = residual.has_value() && residual->defined() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  a.ldr = a.residual ? residual->stride(0) : 0;
  const int kb_total = (K + BK - 1) / BK;
  const bool swap = T <= 64;
  a.swap = swap;
  int BN;
  int m_tiles, n_tiles;
  if (swap) {
    BN = T <= 16 ? 16 : T <= 32 ? 32 : 64;
    a.M = F;
    a.N = T;
    m_tiles = (F + BM - 1) / BM;
    n_tiles = (T + BN - 1) / BN;
  } else {
    BN = (F >= 4096 && T >= 512) ? 256 : 128;
    a.M = T;
    a.N = F;
    m_tiles = (T + BM - 1) / BM;
    n_tiles = (F + BN - 1) / BN;
  }
  const int tiles = m_tiles * n_tiles;
  // split-K so that the grid covers the machine (decode shapes have few tiles)
  int splits = 1;
  const int sms = num_sms();
  if (tiles < sms) {
    splits = std::max(1, std::min({(sms + tiles - 1) / tiles, kb_total / 4, 16}));
  }
  int kbps = (kb_total + splits - 1) / splits;
  splits = (kb_total + kbps - 1) / kbps;
  a.splits = splits;
  a.kb_per_split = kbps;
  int dev = x.get_device();
  SplitKScratch& s = scratch_for(dev, splits > 1 ? (size_t)tiles * splits * BM * BN * 4 : 0, tiles);
  a.ws = s.ws;
  a.counters = s.counters;
  a.err = s.err;
  dim3 grid(m_tiles, n_tiles, splits);
  const void* pa = swap ? w.data_ptr() : x.data_ptr();
  const void* pb = swap ? x.data_ptr() : w.data_ptr();
  const int64_t ra = swap ? F : T, rb = swap ? T : F;
  const int64_t lda = swap ? w.stride(0) : x.stride(0), ldb = swap ? x.stride(0) : w.stride(0);
  CUtensorMap ta = make_tmap(pa, ra, K, lda, BM);
  CUtensorMap tb = make_tmap(pb, rb, K, ldb, BN);
  switch (BN) {
    case 16: launch<16, 10>(ta, tb, a, grid, st); break;
    case 32: launch<32, 10>(ta, tb, a, grid, st); break;
    case 64: launch<64, 8>(ta, tb, a, grid, st); break;
    case 128: launch<128, 6>(ta, tb, a, grid, st); break;
    default: launch<256, 4>(ta, tb, a, grid, st); break;
  }
}

int64_t gemm_check_error(int64_t device) {
  int* e = gemm_error_flag((int)device);
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, e, sizeof(int), cudaMemcpyDeviceToHost));
  if (h) C10_CUDA_CHECK(cudaMemset(e, 0, sizeof(int)));
  return h;
}

}  // namespace braid
