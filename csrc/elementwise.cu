// Row-wise and element-wise kernels: RMSNorm (+ fused residual add),
// LayerNorm, tanh-GELU, vocab-parallel embedding gather, and the fused QKV
// epilogue (per-head q/k RMSNorm, RoPE on k, paged KV append).
//
// Replaces: braidinfer/kernels/rmsnorm_f32.py (Triton row RMSNorm),
// braidinfer/layers/layernorm.py, braidinfer/layers/activation.py,
// braidinfer/layers/embed_head.py:14-29, the Qwen3 q_norm/k_norm + RoPE
// sequence (braidinfer/models/qwen3.py:258-309) and the per-token paged append
// loop with .item() syncs (braidinfer/kernels/kv_cache_utils.py:9-78).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

namespace braid {

template <int NT>
BRAID_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

// out = w * bf16(x * rsqrt(mean(x^2) + eps)); with `res`: x = bf16(res + x), res <- x.
template <int NT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(__nv_bfloat16* __restrict__ out, __nv_bfloat16* res,
                                                     const __nv_bfloat16* x, const __nv_bfloat16* __restrict__ w,
                                                     int H, float eps) {
  __shared__ float red[NT / 32];
  const size_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  __nv_bfloat16* rr = res ? res + row * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += NT * 8) {
    uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&u);
    if (rr) {
      uint4 ru = *reinterpret_cast<const uint4*>(rr + i);
      __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&ru);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = f2bf(bf2f(e[j]) + bf2f(re[j]));
      *reinterpret_cast<uint4*>(rr + i) = u;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = bf2f(e[j]);
      ss += f * f;
    }
  }
  const float rstd = rsqrtf(block_sum<NT>(ss, red) / H + eps);
  const __nv_bfloat16* src = rr ? rr : xr;
  for (int i = threadIdx.x * 8; i < H; i += NT * 8) {
    uint4 u = *reinterpret_cast<const uint4*>(src + i);
    uint4 wu = *reinterpret_cast<const uint4*>(w + i);
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&u);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wu);
#pragma unroll
    for (int j = 0; j < 8; ++j) e[j] = f2bf(rbf(bf2f(e[j]) * rstd) * bf2f(we[j]));
    *reinterpret_cast<uint4*>(out + row * H + i) = u;
  }
}

template <int NT>
__global__ void __launch_bounds__(NT) layernorm_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* x,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       const __nv_bfloat16* __restrict__ b, int H, float eps) {
  __shared__ float red[NT / 32];
  const size_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += NT) s += bf2f(xr[i]);
  const float mean = block_sum<NT>(s, red) / H;
  float v = 0.f;
  for (int i = threadIdx.x; i < H; i += NT) {
    const float d = bf2f(xr[i]) - mean;
    v += d * d;
  }
  const float rstd = rsqrtf(block_sum<NT>(v, red) / H + eps);
  for (int i = threadIdx.x; i < H; i += NT)
    out[row * H + i] = f2bf((bf2f(xr[i]) - mean) * rstd * bf2f(w[i]) + bf2f(b[i]));
}

__global__ void gelu_tanh_kernel(__nv_bfloat16* out, const __nv_bfloat16* x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = bf2f(x[i]);
    out[i] = f2bf(0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v))));
  }
}

__global__ void embedding_kernel(__nv_bfloat16* __restrict__ out, const int* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ w, int H, int rows, int vocab_start,
                                 unsigned long long* span) {
  if (threadIdx.x == 0) span_start(span);
  const int t = blockIdx.x;
  const int id = ids[t] - vocab_start;
  const bool ok = id >= 0 && id < rows;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    uint4 u = make_uint4(0, 0, 0, 0);
    if (ok) u = *reinterpret_cast<const uint4*>(w + (size_t)id * H + i);
    *reinterpret_cast<uint4*>(out + (size_t)t * H + i) = u;
  }
  if (threadIdx.x == 0) span_end(span);
}

// One warp per (token, head).  Heads [0,Hq) are q, [Hq,Hq+Hkv) k, then v.
// Each lane holds E = D/32 consecutive elements; the rotary partner of element
// i (< D/2) is i + D/2, held by lane ^ 16.
template <int D>
__global__ void __launch_bounds__(128) qkv_prepare_kernel(
    __nv_bfloat16* __restrict__ q_out, const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ positions,
    const int* __restrict__ slots, __nv_bfloat16* __restrict__ kv, const __nv_bfloat16* __restrict__ qn,
    const __nv_bfloat16* __restrict__ kn, float eps, const float* __restrict__ cos, const float* __restrict__ sin,
    int Hq, int Hkv, int PS, int use_rope, int ld_qkv, int num_slots, int rope_len) {
  constexpr int E = D / 32;
  const int t = blockIdx.x;
  const int head = blockIdx.y * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int nh = Hq + 2 * Hkv;
  if (head >= nh) return;
  const __nv_bfloat16* src = qkv + (size_t)t * ld_qkv + (size_t)head * D + lane * E;
  float v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = bf2f(src[j]);
  const bool is_q = head < Hq, is_k = !is_q && head < Hq + Hkv;
  const __nv_bfloat16* nw = is_q ? qn : (is_k ? kn : nullptr);
  if (nw != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss += v[j] * v[j];
    const float rstd = rsqrtf(warp_sum(ss) / D + eps);
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = rbf(rbf(v[j] * rstd) * bf2f(nw[lane * E + j]));
  }
  if (is_q) {
    __nv_bfloat16* dst = q_out + ((size_t)t * Hq + head) * D + lane * E;
#pragma unroll
    for (int j = 0; j < E; ++j) dst[j] = f2bf(v[j]);
    return;
  }
  if (is_k && use_rope) {
    int pos = positions[t];
    if (!BRAID_IN_BOUNDS(pos >= 0 && pos < rope_len, 2, pos)) pos = 0;
    float partner[E];
#pragma unroll
    for (int j = 0; j < E; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, v[j], 16);
    const bool first = lane < 16;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int d = (lane & 15) * E + j;  // index within the half
      const float c = cos[(size_t)pos * (D / 2) + d], s = sin[(size_t)pos * (D / 2) + d];
      v[j] = first ? v[j] * c - partner[j] * s : v[j] * c + partner[j] * s;
    }
  }
  const int slot = slots[t];
  if (!BRAID_IN_BOUNDS(slot >= 0 && slot < num_slots, 1, slot)) return;
  const int page = slot / PS, off = slot % PS;
  const int kh = is_k ? head - Hq : head - Hq - Hkv;
  __nv_bfloat16* dst = kv + ((((size_t)page * 2 + (is_k ? 0 : 1)) * Hkv + kh) * PS + off) * D + lane * E;
#pragma unroll
  for (int j = 0; j < E; ++j) dst[j] = f2bf(v[j]);
}

// ------------------------------------------------------------------ host
static inline const __nv_bfloat16* bp(const torch::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr());
}
static inline __nv_bfloat16* bpm(torch::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

static void check_rows(const torch::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "bf16 contiguous CUDA tensor required");
  TORCH_CHECK(x.size(-1) % 8 == 0, "hidden size must be a multiple of 8");
}

void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps) {
  check_rows(x);
  const int H = x.size(-1), rows = x.numel() / H;
  if (!rows) return;
  const at::cuda::CUDAGuard g(x.device());
  rmsnorm_kernel<256><<<rows, 256, 0, at::cuda::getCurrentCUDAStream()>>>(bpm(out), nullptr, bp(x), bp(w), H, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void add_rms_norm(torch::Tensor out, torch::Tensor residual, torch::Tensor x, torch::Tensor w, double eps) {
  check_rows(x);
  check_rows(residual);
  const int H = x.size(-1), rows = x.numel() / H;
  if (!rows) return;
  const at::cuda::CUDAGuard g(x.device());
  rmsnorm_kernel<256><<<rows, 256, 0, at::cuda::getCurrentCUDAStream()>>>(bpm(out), bpm(residual), bp(x), bp(w), H,
                                                                           (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void layer_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps) {
  check_rows(x);
  const int H = x.size(-1), rows = x.numel() / H;
  if (!rows) return;
  const at::cuda::CUDAGuard g(x.device());
  layernorm_kernel<256><<<rows, 256, 0, at::cuda::getCurrentCUDAStream()>>>(bpm(out), bp(x), bp(w), bp(b), H,
                                                                            (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_tanh(torch::Tensor out, torch::Tensor x) {
  const size_t n = x.numel();
  if (!n) return;
  const at::cuda::CUDAGuard g(x.device());
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 16);
  gelu_tanh_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(bpm(out), bp(x), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

unsigned long long* next_span(const char* name);

void embedding(torch::Tensor out, torch::Tensor ids, torch::Tensor w, int64_t vocab_start) {
  TORCH_CHECK(ids.scalar_type() == at::kInt, "embedding: int32 ids");
  const int T = ids.size(0), H = w.size(1);
  TORCH_CHECK(H % 8 == 0, "embedding: hidden must be a multiple of 8");
  if (!T) return;
  const at::cuda::CUDAGuard g(w.device());
  embedding_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(bpm(out), ids.data_ptr<int>(), bp(w), H,
                                                                   (int)w.size(0), (int)vocab_start,
                                                                   next_span("embedding"));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qkv_prepare(torch::Tensor q_out, torch::Tensor qkv, torch::Tensor positions, torch::Tensor slots,
                 torch::Tensor kv, c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm,
                 double eps, torch::Tensor cos, torch::Tensor sin, int64_t Hq, int64_t Hkv, int64_t D,
                 bool use_rope) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && kv.scalar_type() == at::kBFloat16);
  TORCH_CHECK(qkv.stride(1) == 1 && kv.is_contiguous());
  TORCH_CHECK(kv.size(2) == Hkv && kv.size(4) == D, "qkv_prepare: cache layout mismatch");
  const int T = qkv.size(0);
  if (!T) return;
  const at::cuda::CUDAGuard g(qkv.device());
  const __nv_bfloat16* qn = q_norm.has_value() && q_norm->defined() ? bp(*q_norm) : nullptr;
  const __nv_bfloat16* kn = k_norm.has_value() && k_norm->defined() ? bp(*k_norm) : nullptr;
  dim3 grid(T, (Hq + 2 * Hkv + 3) / 4);
  auto st = at::cuda::getCurrentCUDAStream();
  const int PS = kv.size(3);
  if (D == 128)
    qkv_prepare_kernel<128><<<grid, 128, 0, st>>>(bpm(q_out), bp(qkv), positions.data_ptr<int>(), slots.data_ptr<int>(),
                                                  bpm(kv), qn, kn, (float)eps, cos.data_ptr<float>(),
                                                  sin.data_ptr<float>(), Hq, Hkv, PS, use_rope, qkv.stride(0),
                                                  (int)(kv.size(0) * PS), (int)cos.size(0));
  else if (D == 64)
    qkv_prepare_kernel<64><<<grid, 128, 0, st>>>(bpm(q_out), bp(qkv), positions.data_ptr<int>(), slots.data_ptr<int>(),
                                                 bpm(kv), qn, kn, (float)eps, cos.data_ptr<float>(),
                                                 sin.data_ptr<float>(), Hq, Hkv, PS, use_rope, qkv.stride(0),
                                                  (int)(kv.size(0) * PS), (int)cos.size(0));
  else
    TORCH_CHECK(false, "qkv_prepare: head_dim must be 64 or 128");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace braid

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_elementwise)
}  // namespace braid
