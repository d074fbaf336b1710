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

// Block-wide argmax of x[0, n) (ids id0 + i): 16-byte loads when the row is
// 16-byte aligned, scalar loads for the tail.
BRAID_DEVICE ArgMax row_argmax(const __nv_bfloat16* x, int n, int id0) {
  ArgMax a{-INFINITY, 0x7fffffff};
  int head = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    head = n & ~7;
    for (int i = threadIdx.x * 8; i < head; i += SNT * 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + i);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) a = better(a, ArgMax{bf2f(e[j]), id0 + i + j});
    }
  }
  for (int i = head + threadIdx.x; i < n; i += SNT) a = better(a, ArgMax{bf2f(x[i]), id0 + i});
  return a;
}
BRAID_DEVICE ArgMax row_argmax(const float* x, int n, int id0) {
  ArgMax a{-INFINITY, 0x7fffffff};
  int head = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    head = n & ~3;
    for (int i = threadIdx.x * 4; i < head; i += SNT * 4) {
      const float4 u = *reinterpret_cast<const float4*>(x + i);
      a = better(a, ArgMax{u.x, id0 + i});
      a = better(a, ArgMax{u.y, id0 + i + 1});
      a = better(a, ArgMax{u.z, id0 + i + 2});
      a = better(a, ArgMax{u.w, id0 + i + 3});
    }
  }
  for (int i = head + threadIdx.x; i < n; i += SNT) a = better(a, ArgMax{x[i], id0 + i});
  return a;
}

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
    ArgMax a = row_argmax(x, V, 0);
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


// ------------------------------------------------------------------------
// Vocab-parallel sampling under tensor parallelism (one kernel, no NCCL).
//
// Each rank holds the logits of its vocabulary shard [B, Vl] (global id =
// vocab_start + i).  One CTA per row reduces the shard to a fixed-size
// record, stores it into every peer's receive slot over NVLink, bumps each
// peer's arrival counter for this rank, waits (bounded) until every source's
// records of this call have arrived, and merges the tp records.  Every rank
// merges the same records the same way, so all ranks pick the same token.
//   greedy rows            record = local (max logit, id); merge = argmax
//   temperature only       record = local argmax of z + g(id) (the Gumbel-max
//                          race restricted to the shard); merge = argmax.
//                          Exact: g depends only on (seed, step, global id).
//   top-k <= TPS_KC        record = local top-TPS_KC candidates of z and the
//                          local z max; the global top-k (and every token that
//                          min-p / top-p keep after it) lies among the tp x
//                          TPS_KC candidates, so the merge applies min-p,
//                          top-k, top-p and the Gumbel race exactly there.
// Other settings (top-p or min-p without top-k, top-k > TPS_KC) need the full
// distribution: the host routes such steps to the logits all-gather.
// Replaces the per-row loops of braidinfer/layers/sampler.py:48-81 and the
// logits all-gather of the tensor-parallel decode step.
constexpr int TPS_KC = 32;
struct TpsRec {  // 4-byte words
  float zmax;    // local max of z (sampled) or of the logit (greedy)
  float gval;    // winner value of the local race
  int gid;       // its global token id
  int ncand;     // candidates stored
  float cz[TPS_KC];
  int cid[TPS_KC];
};
static_assert(sizeof(TpsRec) % 16 == 0, "TpsRec is moved in 16-byte units");

__global__ void __launch_bounds__(SNT) tp_sample_kernel(
    int* __restrict__ out, const __nv_bfloat16* __restrict__ logits, int Vl, int ld_row, int vocab_start,
    int vocab_size, const float* __restrict__ temperature, const int* __restrict__ top_k,
    const float* __restrict__ top_p, const float* __restrict__ min_p, const int64_t* __restrict__ seed,
    const int64_t* __restrict__ step, const uint64_t* __restrict__ peers, int64_t recv_off, int64_t flags_off,
    int rank, int tp, int maxB, uint64_t* epoch_state, int* status, uint64_t timeout_ns, unsigned long long* span) {
  __shared__ ArgMax ared[SNT / 32];
  __shared__ float fred[SNT / 32];
  __shared__ __align__(16) TpsRec rec;
  __shared__ int s_n, s_fail;
  __shared__ float s_cz[8 * TPS_KC];
  __shared__ int s_cid[8 * TPS_KC];
  if (threadIdx.x == 0) span_start(span);
  pdl_wait();
  if (threadIdx.x == 0) span_waited(span);
  const int row = blockIdx.x, B = gridDim.x;
  const uint64_t epoch = epoch_state[0];
  const uint64_t expected = epoch_state[1] + (uint64_t)B;
  const int slot = (int)(epoch & 1);
  const __nv_bfloat16* x = logits + (size_t)row * ld_row;
  const int nvalid = max(0, min(Vl, vocab_size - vocab_start));
  const float temp = temperature[row];
  const int k = top_k[row];
  const bool greedy = temp <= 0.f;
  const float inv_t = greedy ? 1.f : 1.f / fmaxf(temp, 1e-10f);
  if (threadIdx.x == 0) {
    s_n = 0;
    s_fail = 0;
  }
  // ---- local record (the z max only matters for the top-k candidates)
  float zmax = -INFINITY;
  if (!greedy && k > 0) {
    for (int i = threadIdx.x; i < nvalid; i += SNT) zmax = fmaxf(zmax, bf2f(x[i]) * inv_t);
    zmax = block_reduce_max(zmax, fred);
  }
  ArgMax a{-INFINITY, 0x7fffffff};
  if (greedy) {
    a = row_argmax(x, nvalid, vocab_start);
  } else if (k <= 0) {
    const uint64_t key = mix64((uint64_t)seed[row] ^ mix64((uint64_t)step[row]));
    for (int i = threadIdx.x; i < nvalid; i += SNT) {
      const int gid = vocab_start + i;
      const float u = hash_uniform(key, (uint64_t)gid);
      a = better(a, ArgMax{bf2f(x[i]) * inv_t - logf(-logf(u)), gid});
    }
  }
  a = block_argmax(a, ared);
  if (!greedy && k > 0) {
    // largest threshold with at least TPS_KC local values above it (bisection)
    const int want = min(TPS_KC, nvalid);
    float lo = zmax - 100.f, hi = zmax;
    for (int it = 0; it < 30; ++it) {
      const float mid = 0.5f * (lo + hi);
      float c = 0.f;
      for (int i = threadIdx.x; i < nvalid; i += SNT) c += (bf2f(x[i]) * inv_t >= mid) ? 1.f : 0.f;
      c = block_reduce_sum(c, fred);
      if (c >= (float)want) lo = mid; else hi = mid;
    }
    // Values >= hi are fewer than `want`: take all of them first, then fill
    // the remaining slots with values in [lo, hi) (ties at the boundary), so
    // an overflow of ties can never push out a larger value.
    for (int pass = 0; pass < 2; ++pass) {
      for (int i = threadIdx.x; i < nvalid; i += SNT) {
        const float z = bf2f(x[i]) * inv_t;
        if (pass == 0 ? z >= hi : (z >= lo && z < hi)) {
          const int j = atomicAdd(&s_n, 1);
          if (j < TPS_KC) {
            rec.cz[j] = z;
            rec.cid[j] = vocab_start + i;
          }
        }
      }
      __syncthreads();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    rec.zmax = zmax;
    rec.gval = a.v;
    rec.gid = a.i;
    rec.ncand = min(s_n, TPS_KC);
  }
  __syncthreads();
  // ---- push the record to every rank (self included), then count it there
  constexpr int NV = sizeof(TpsRec) / 16;
  if (threadIdx.x < NV) {
    const uint4 v = reinterpret_cast<const uint4*>(&rec)[threadIdx.x];
    const size_t off = (size_t)recv_off + (((size_t)slot * tp + rank) * maxB + row) * sizeof(TpsRec);
    for (int p = 0; p < tp; ++p)
      reinterpret_cast<uint4*>(reinterpret_cast<char*>(peers[p]) + off)[threadIdx.x] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int p = 0; p < tp; ++p)
      atomicAdd(reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(peers[p]) + flags_off) + rank, 1ull);
  // ---- wait for every source's records of this call (bounded)
  if (threadIdx.x < tp) {
    const uint64_t* f = reinterpret_cast<const uint64_t*>(reinterpret_cast<const char*>(peers[rank]) + flags_off) +
                        threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u64(f) < expected) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (atomicCAS(status, 0, 4) == 0) {
          status[1] = rank;
          status[2] = threadIdx.x;
          status[3] = (int)epoch;
        }
        s_fail = 1;
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  int token = 0;
  if (!s_fail) {
    const TpsRec* recs =
        reinterpret_cast<const TpsRec*>(reinterpret_cast<const char*>(peers[rank]) + recv_off) + (size_t)slot * tp * maxB;
    if (greedy || k <= 0) {
      ArgMax b{-INFINITY, 0x7fffffff};
      if (threadIdx.x < tp) {
        const TpsRec* r = recs + (size_t)threadIdx.x * maxB + row;
        b = ArgMax{__ldcv(&r->gval), __ldcv(&r->gid)};
      }
      token = block_argmax(b, ared).i;
    } else {
      // candidates of every source: thread i holds candidate i
      float gz = -INFINITY;
      for (int src = 0; src < tp; ++src) gz = fmaxf(gz, __ldcv(&recs[(size_t)src * maxB + row].zmax));
      const int ncap = tp * TPS_KC;
      if (threadIdx.x < ncap) {
        const int src = threadIdx.x / TPS_KC, j = threadIdx.x % TPS_KC;
        const TpsRec* r = recs + (size_t)src * maxB + row;
        const bool ok = j < __ldcv(&r->ncand);
        s_cz[threadIdx.x] = ok ? __ldcv(&r->cz[j]) : -INFINITY;
        s_cid[threadIdx.x] = ok ? __ldcv(&r->cid[j]) : 0x7fffffff;
      }
      __syncthreads();
      const bool mine = threadIdx.x < ncap && s_cz[threadIdx.x] != -INFINITY;
      const float z = mine ? s_cz[threadIdx.x] : -INFINITY;
      const int id = mine ? s_cid[threadIdx.x] : 0x7fffffff;
      // order: larger z first, then smaller id
      int before = 0;
      if (mine)
        for (int j = 0; j < ncap; ++j)
          before += (s_cz[j] > z || (s_cz[j] == z && s_cid[j] < id)) ? 1 : 0;
      // k-th largest value: the candidate ranked k - 1 publishes it
      __shared__ float s_kth;
      if (threadIdx.x == 0) s_kth = -INFINITY;
      __syncthreads();
      if (mine && before == k - 1) s_kth = z;
      __syncthreads();
      bool keep = mine && z >= s_kth;
      const float mp = min_p[row];
      if (mp > 0.f) keep = keep && z >= gz + logf(mp);
      const float tpp = top_p[row];
      if (tpp < 1.f) {
        const float e = keep ? __expf(z - gz) : 0.f;
        const float tot = block_reduce_sum(e, fred);
        __shared__ float s_pr[8 * TPS_KC];
        if (threadIdx.x < ncap) s_pr[threadIdx.x] = keep ? e / tot : -1.f;
        __syncthreads();
        // mass of the kept candidates ordered before this one
        float mass = 0.f;
        if (keep)
          for (int j = 0; j < ncap; ++j)
            if (s_pr[j] >= 0.f && (s_cz[j] > z || (s_cz[j] == z && s_cid[j] < id))) mass += s_pr[j];
        const bool nuc = keep && mass < tpp;
        const float thr = -block_reduce_max(nuc ? -(e / tot) : -INFINITY, fred);
        keep = keep && e / tot >= thr;
      }
      ArgMax b{-INFINITY, 0x7fffffff};
      if (keep) {
        const uint64_t key = mix64((uint64_t)seed[row] ^ mix64((uint64_t)step[row]));
        const float u = hash_uniform(key, (uint64_t)id);
        b = ArgMax{z - logf(-logf(u)), id};
      }
      token = block_argmax(b, ared).i;
    }
  }
  if (threadIdx.x == 0) {
    out[row] = token;
    // advance the epoch once every row of this call is merged
    __threadfence();
    const unsigned long long done = atomicAdd(reinterpret_cast<unsigned long long*>(epoch_state + 2), 1ull);
    if (done == (unsigned long long)(B - 1)) {
      epoch_state[2] = 0;
      epoch_state[1] = expected;
      epoch_state[0] = epoch + 1;
    }
    span_end(span);
  }
}

int64_t tp_sample_record_bytes() { return sizeof(TpsRec); }

void tp_sample(torch::Tensor out, torch::Tensor logits, int64_t vocab_start, int64_t vocab_size,
               torch::Tensor temperature, torch::Tensor top_k, torch::Tensor top_p, torch::Tensor min_p,
               torch::Tensor seed, torch::Tensor step, torch::Tensor peers, int64_t recv_off, int64_t flags_off,
               int64_t rank, int64_t tp, int64_t maxB, torch::Tensor epoch_state, torch::Tensor status,
               double timeout_s) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16,
              "tp_sample: bf16 [B, V_local] logits");
  TORCH_CHECK(tp >= 1 && tp <= 8, "tp_sample: at most 8 ranks");
  const int B = logits.size(0), Vl = logits.size(1);
  TORCH_CHECK(B <= maxB, "tp_sample: batch exceeds the receive area");
  if (!B) return;
  const at::cuda::CUDAGuard g(logits.device());
  launch_pdl(tp_sample_kernel, dim3(B), dim3(SNT), 0, at::cuda::getCurrentCUDAStream(), out.data_ptr<int>(),
             reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), Vl, (int)logits.stride(0), (int)vocab_start,
             (int)vocab_size, temperature.data_ptr<float>(), top_k.data_ptr<int>(), top_p.data_ptr<float>(),
             min_p.data_ptr<float>(), seed.data_ptr<int64_t>(), step.data_ptr<int64_t>(),
             reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), recv_off, flags_off, (int)rank, (int)tp,
             (int)maxB, reinterpret_cast<uint64_t*>(epoch_state.data_ptr<int64_t>()), status.data_ptr<int>(),
             (uint64_t)(timeout_s * 1e9), next_span("tp_sample"));
}

}  // namespace braid

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_sampling)
}  // namespace braid
