// Device sampler: greedy argmax, or temperature + min-p + top-k + top-p with a
// Gumbel-max race, one CTA per row, no host synchronisation.
//
// Semantics of braidinfer/layers/sampler.py:10-91 without its per-row Python
// loops and sorts: top-k and nucleus thresholds are found by bisection on the
// scaled logit value (each probe is one pass over the row, which stays in L2),
// and the sample is argmax(z + g) over kept tokens with g = -log(-log u),
// u = SplitMix64 finaliser (Steele, Lea, Flood 2014) of (seed, step, token).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

namespace braid {

constexpr int SNT = 1024;

BRAID_DEVICE uint64_t mix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

BRAID_DEVICE float hash_uniform(uint64_t key, uint64_t idx) {
  const uint64_t h = mix64(key + idx);
  return (float)((double)((h >> 40) + 1) / 16777216.0);
}

struct ArgMax {
  float v;
  int i;
};
BRAID_DEVICE ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

BRAID_DEVICE ArgMax block_argmax(ArgMax a, ArgMax* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = a;
  __syncthreads();
  if (w == 0) {
    a = l < SNT / 32 ? red[l] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
      a = better(a, b);
    }
    if (l == 0) red[0] = a;
  }
  __syncthreads();
  ArgMax r = red[0];
  __syncthreads();
  return r;
}

BRAID_DEVICE float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < SNT / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}
BRAID_DEVICE float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < SNT / 32; ++i) t = fmaxf(t, red[i]);
  __syncthreads();
  return t;
}

template <typename T>
BRAID_DEVICE float ld(const T* p, size_t i);
template <>
BRAID_DEVICE float ld<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) { return bf2f(p[i]); }
template <>
BRAID_DEVICE float ld<float>(const float* p, size_t i) { return p[i]; }

template <typename T>
__global__ void __launch_bounds__(SNT) sample_kernel(int* __restrict__ out, const T* __restrict__ logits, int V,
                                                     int ld_row, const float* __restrict__ temperature,
                                                     const int* __restrict__ top_k, const float* __restrict__ top_p,
                                                     const float* __restrict__ min_p,
                                                     const int64_t* __restrict__ seed, const int64_t* __restrict__ step,
                                                     int all_greedy, unsigned long long* span) {
  __shared__ ArgMax ared[SNT / 32];
  if (threadIdx.x == 0) span_start(span);
  __shared__ float fred[SNT / 32];
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld_row;
  const float temp = all_greedy ? 0.f : temperature[row];
  if (temp <= 0.f) {
    ArgMax a{-INFINITY, 0x7fffffff};
    for (int i = threadIdx.x; i < V; i += SNT) a = better(a, ArgMax{ld(x, i), i});
    a = block_argmax(a, ared);
    if (threadIdx.x == 0) {
      out[row] = a.i;
      span_end(span);
    }
    return;
  }
  const float inv_t = 1.f / fmaxf(temp, 1e-10f);
  float zmax = -INFINITY;
  for (int i = threadIdx.x; i < V; i += SNT) zmax = fmaxf(zmax, ld(x, i) * inv_t);
  zmax = block_reduce_max(zmax, fred);
  // lower bound on kept z values
  float lo_keep = -INFINITY;
  const float mp = min_p[row];
  if (mp > 0.f) lo_keep = zmax + logf(mp);
  const int k = top_k[row];
  if (k > 0 && k < V) {
    // largest threshold t with count(z >= t) >= k
    float lo = zmax - 100.f, hi = zmax;
    for (int it = 0; it < 30; ++it) {
      const float mid = 0.5f * (lo + hi);
      float c = 0.f;
      for (int i = threadIdx.x; i < V; i += SNT) c += (ld(x, i) * inv_t >= mid) ? 1.f : 0.f;
      c = block_reduce_sum(c, fred);
      if (c >= (float)k) lo = mid; else hi = mid;
    }
    lo_keep = fmaxf(lo_keep, lo);
  }
  const float tp = top_p[row];
  if (tp < 1.f) {
    float tot = 0.f;
    for (int i = threadIdx.x; i < V; i += SNT) {
      const float z = ld(x, i) * inv_t;
      if (z >= lo_keep) tot += __expf(z - zmax);
    }
    tot = block_reduce_sum(tot, fred);
    float lo = fmaxf(lo_keep, zmax - 100.f), hi = zmax;
    for (int it = 0; it < 30; ++it) {
      const float mid = 0.5f * (lo + hi);
      float s = 0.f;
      for (int i = threadIdx.x; i < V; i += SNT) {
        const float z = ld(x, i) * inv_t;
        if (z >= mid && z >= lo_keep) s += __expf(z - zmax);
      }
      s = block_reduce_sum(s, fred);
      if (s >= tp * tot) lo = mid; else hi = mid;
    }
    lo_keep = fmaxf(lo_keep, lo);
  }
  const uint64_t key = mix64((uint64_t)seed[row] ^ mix64((uint64_t)step[row]));
  ArgMax a{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += SNT) {
    const float z = ld(x, i) * inv_t;
    if (z >= lo_keep) {
      const float u = hash_uniform(key, (uint64_t)i);
      a = better(a, ArgMax{z - logf(-logf(u)), i});
    }
  }
  a = block_argmax(a, ared);
  if (threadIdx.x == 0) {
    out[row] = a.i;
    span_end(span);
  }
}

unsigned long long* next_span(const char* name);

void sample(torch::Tensor out, torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_k,
            torch::Tensor top_p, torch::Tensor min_p, torch::Tensor seed, torch::Tensor step, bool all_greedy) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample: [B, V] logits");
  const int B = logits.size(0), V = logits.size(1);
  if (!B) return;
  const at::cuda::CUDAGuard g(logits.device());
  auto st = at::cuda::getCurrentCUDAStream();
  unsigned long long* span = next_span("sample");
  if (logits.scalar_type() == at::kBFloat16)
    sample_kernel<__nv_bfloat16><<<B, SNT, 0, st>>>(
        out.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), V, logits.stride(0),
        temperature.data_ptr<float>(), top_k.data_ptr<int>(), top_p.data_ptr<float>(), min_p.data_ptr<float>(),
        seed.data_ptr<int64_t>(), step.data_ptr<int64_t>(), all_greedy ? 1 : 0, span);
  else
    sample_kernel<float><<<B, SNT, 0, st>>>(out.data_ptr<int>(), logits.data_ptr<float>(), V, logits.stride(0),
                                            temperature.data_ptr<float>(), top_k.data_ptr<int>(),
                                            top_p.data_ptr<float>(), min_p.data_ptr<float>(),
                                            seed.data_ptr<int64_t>(), step.data_ptr<int64_t>(), all_greedy ? 1 : 0,
                                            span);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace braid
