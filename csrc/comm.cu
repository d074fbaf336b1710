// Tensor-parallel collectives over NVLink peer memory.
//
// Runtime: each rank cudaMalloc's one communication buffer, exports a CUDA IPC
// handle, the handles are exchanged over the process group (host side), and
// every rank maps every peer's buffer.  Kernels then write peers' memory with
// plain st.global (P2P over NVLink 5 / NVSwitch); no multicast objects and no
// TMA loads of peer memory are used.
//
// One-shot push all-reduce (decode-sized tensors):
//   producer  the row-parallel GEMM epilogue (gemm_tcgen05.cu, epi 3) or
//             tp_push_kernel writes its bf16 partial [T, H] into slot
//             (epoch & 1), source row `rank`, of every peer's receive area,
//             then bumps that peer's arrival counter for `rank` (system-scope
//             release).
//   consumer  tp_reduce_add_kernel waits (bounded by a wall-clock timeout) until
//             every source's counter reaches the cumulative expected count,
//             sums the tp partials in fp32, adds the residual, and advances the
//             epoch.  Two slots suffice: a rank can only be one call ahead of
//             the slowest peer, because every call waits for all peers.
// On timeout the kernel records {code, rank, source, epoch} in a status word
// and returns; the host raises CommTimeoutError and the context stays usable.
//
// Replaces the reference's only collective, a dead dist.all_reduce in
// braidinfer/layers/linear_distributed.py:170-174.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "launch.cuh"

#include <tuple>

namespace braid {

unsigned long long* next_span(const char* name);
PrefetchArgs take_prefetch(CUtensorMap* map, const CUtensorMap& fallback);

// Layout of one rank's communication buffer (offsets in bytes):
//   [0, data_bytes)                recv[2][tp][maxT][H] bf16
//   [data_bytes, +8*tp)            arrivals[tp] u64 (written by peers)
struct CommLayout {
  int64_t tp, maxT, H;
  int64_t data_bytes() const { return 2 * tp * maxT * H * 2; }
  int64_t flags_off() const { return (data_bytes() + 255) / 256 * 256; }
  int64_t total() const { return flags_off() + 8 * tp + 256; }
};

// Push a bf16 partial [T, H] to every peer (generic producer; the GEMM epilogue
// does the same work in place of its local store).
__global__ void tp_push_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, const uint64_t* __restrict__ peers,
                               int64_t flags_off, int rank, int tp, int maxT, const uint64_t* epoch_state) {
  const int slot = (int)(epoch_state[0] & 1);
  const size_t n = (size_t)T * H;
  for (size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 8; i < n; i += (size_t)gridDim.x * blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + i);
    const size_t t = i / H, h = i % H;
    for (int p = 0; p < tp; ++p) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers[p]) + (((size_t)slot * tp + rank) * maxT + t) * H + h;
      *reinterpret_cast<uint4*>(dst) = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int p = 0; p < tp; ++p) {
      uint64_t* f = reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(peers[p]) + flags_off) + rank;
      atomicAdd(reinterpret_cast<unsigned long long*>(f), 1ull);
    }
  }
}

// epoch_state (local device memory, u64[4]): [0] completed calls (epoch),
// [1] cumulative expected arrivals per source, [2] CTA done counter.
__global__ void tp_reduce_add_kernel(__nv_bfloat16* __restrict__ residual, int T, int H, const char* __restrict__ buf,
                                     int64_t flags_off, int tp, int maxT, int rank, uint64_t arrivals_per_call,
                                     uint64_t* epoch_state, int* status, uint64_t timeout_ns, int add_residual,
                                     __nv_bfloat16* __restrict__ out, unsigned long long* span,
                                     const __grid_constant__ CUtensorMap tmP, PrefetchArgs pf) {
  __shared__ int s_fail;
  if (threadIdx.x == 0) {
    span_start(span);
    // while the peers' partials are in flight, pull the next GEMM's weight into L2
    prefetch_next_weight(&tmP, pf, blockIdx.x, gridDim.x);
  }
  // Programmatic dependent launch: let the next kernel (the consuming GEMM)
  // launch at once so its weight prefetch overlaps this wait; its own
  // dependency wait still covers all of this kernel.  The epoch state was last
  // written by the previous reduce, which the producing GEMM's dependency
  // chain has completed once this kernel's own dependency wait returns.
  pdl_trigger();
  pdl_wait();
  const uint64_t epoch = epoch_state[0];
  const uint64_t expected = epoch_state[1] + arrivals_per_call;
  const int slot = (int)(epoch & 1);
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < tp) {
    const uint64_t* f = reinterpret_cast<const uint64_t*>(buf + flags_off) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u64(f) < expected) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (atomicCAS(status, 0, 1) == 0) {
          status[1] = rank;
          status[2] = threadIdx.x;
          status[3] = (int)epoch;
        }
        s_fail = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) span_waited(span);
  if (!s_fail) {
    const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(buf) + (size_t)slot * tp * maxT * H;
    const size_t n = (size_t)T * H;
    for (size_t i = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) * 8; i < n;
         i += (size_t)gridDim.x * blockDim.x * 8) {
      const size_t t = i / H, h = i % H;
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int src = 0; src < tp; ++src) {
        const uint4 v = __ldcv(reinterpret_cast<const uint4*>(recv + ((size_t)src * maxT + t) * H + h));
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] += bf2f(e[j]);
      }
      uint4 r = make_uint4(0, 0, 0, 0);
      if (add_residual) r = *reinterpret_cast<const uint4*>(residual + i);
      __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&r);
#pragma unroll
      for (int j = 0; j < 8; ++j) re[j] = f2bf((add_residual ? bf2f(re[j]) : 0.f) + rbf(s[j]));
      *reinterpret_cast<uint4*>(out + i) = r;
    }
  }
  // advance the epoch once every CTA is done with this call's slot
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long old = atomicAdd(reinterpret_cast<unsigned long long*>(epoch_state + 2), 1ull);
    if (old == gridDim.x - 1) {
      epoch_state[2] = 0;
      epoch_state[1] = expected;
      epoch_state[0] = epoch + 1;
    }
    span_end(span);
  }
}

// -------------------------------------------- sequence parallel (prefill)
// Reduce + all-gather of row-parallel GEMM partials for prefill-sized batches.
// This rank owns token rows [rank*rpr, rank*rpr + rpr).  The GEMM epilogue
// (epi 4) pushed every source's bf16 partial rows of this block into
// recv[src]; one warp per owned row waits (bounded) for every source's tile
// count, sums the tp partials in fp32, adds the residual row held in the
// gathered buffer G, computes the row's 1/rms, and stores the new row and its
// 1/rms into G / rstd of EVERY rank (peer stores over NVLink), then bumps each
// rank's all-gather counter for this owner once per CTA.  The next GEMM waits
// on that counter tile by tile (sp_wait_rows), so the gather overlaps its math.
__global__ void __launch_bounds__(256) sp_reduce_allgather_kernel(
    const uint64_t* __restrict__ peers, int64_t recv_off, int64_t rs_flags_off, int64_t ag_flags_off, int64_t g_off,
    int64_t rstd_off, int rank, int tp, int rpr, int T, int H, uint64_t rs_expected, float eps, int* status,
    uint64_t timeout_ns) {
  __shared__ int s_fail;
  pdl_wait();
  const char* local = reinterpret_cast<const char*>(peers[rank]);
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < tp) {
    const uint64_t* f = reinterpret_cast<const uint64_t*>(local + rs_flags_off) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u64(f) < rs_expected) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (atomicCAS(status, 0, 3) == 0) {
          status[1] = rank;
          status[2] = threadIdx.x;
          status[3] = (int)rs_expected;
        }
        s_fail = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (s_fail) return;  // no all-gather signal: the consumers time out and report
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lr = blockIdx.x * 8 + warp;
  const int row = rank * rpr + lr;
  if (lr < rpr && row < T) {
    const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(local + recv_off);
    const __nv_bfloat16* g_row = reinterpret_cast<const __nv_bfloat16*>(local + g_off) + (size_t)row * H;
    float ss = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int src = 0; src < tp; ++src) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(recv + ((size_t)src * rpr + lr) * H + c));
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += bf2f(e[j]);
      }
      uint4 rv = *reinterpret_cast<const uint4*>(g_row + c);
      __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&rv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        re[j] = f2bf(bf2f(re[j]) + rbf(acc[j]));
        const float y = bf2f(re[j]);
        ss += y * y;
      }
      for (int p = 0; p < tp; ++p)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(peers[p]) + g_off) +
                                  (size_t)row * H + c) = rv;
    }
    ss = warp_sum(ss);
    if (lane < tp)
      reinterpret_cast<float*>(reinterpret_cast<char*>(peers[lane]) + rstd_off)[row] = rsqrtf(ss / H + eps);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < tp; ++p)
      atomicAdd(reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(peers[p]) + ag_flags_off) + rank, 1ull);
  }
}

// Bounded wait until every owner's all-gather count reaches `expected`; later
// kernels on the stream may then read all of G with plain loads.
__global__ void sp_wait_kernel(const char* __restrict__ local, int64_t ag_flags_off, int tp, int rank,
                               uint64_t expected, int* status, uint64_t timeout_ns) {
  pdl_wait();
  if (threadIdx.x < tp) {
    const uint64_t* f = reinterpret_cast<const uint64_t*>(local + ag_flags_off) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u64(f) < expected) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (atomicCAS(status, 0, 2) == 0) {
          status[1] = rank;
          status[2] = threadIdx.x;
          status[3] = (int)expected;
        }
        break;
      }
      __nanosleep(64);
    }
  }
  __threadfence();
}

// ------------------------------------------------------------------ host
// cudaMalloc'd communication buffer + its IPC handle (64 bytes, CPU uint8 tensor).
std::vector<torch::Tensor> comm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, nbytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, nbytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto ht = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(ht.data_ptr(), &h, sizeof(h));
  auto pt = torch::tensor({(int64_t)reinterpret_cast<uintptr_t>(p)}, torch::kInt64);
  return {pt, ht};
}

int64_t comm_open(torch::Tensor handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t), "comm_open: bad handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}

void comm_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

void comm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaFree(reinterpret_cast<void*>(ptr));
}

void tp_push(torch::Tensor x, torch::Tensor peers, int64_t flags_off, int64_t rank, int64_t tp, int64_t maxT,
             torch::Tensor epoch_state) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && x.size(1) % 8 == 0);
  const int T = x.size(0), H = x.size(1);
  TORCH_CHECK(T <= maxT, "tp_push: too many tokens for the communication buffer");
  const at::cuda::CUDAGuard g(x.device());
  const int blocks = std::max(1, std::min(32, (int)((int64_t)T * H / 8 / 256)));
  tp_push_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), T, H,
      reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), flags_off, rank, tp, maxT,
      reinterpret_cast<const uint64_t*>(epoch_state.data_ptr<int64_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_reduce_add(torch::Tensor out, torch::Tensor residual, bool add_residual, int64_t buf, int64_t flags_off,
                   int64_t tp, int64_t maxT, int64_t rank, int64_t arrivals_per_call, torch::Tensor epoch_state,
                   torch::Tensor status, double timeout_s) {
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.size(1) % 8 == 0);
  const int T = out.size(0), H = out.size(1);
  TORCH_CHECK(T <= maxT, "tp_reduce_add: too many tokens for the communication buffer");
  const at::cuda::CUDAGuard g(out.device());
  const int blocks = std::max(1, std::min(64, (int)(((int64_t)T * H / 8 + 255) / 256)));
  static const bool use_pdl = [] {  // tuning knob: BRAID_REDUCE_PDL=0 launches it as a plain kernel
    const char* e = getenv("BRAID_REDUCE_PDL");
    return !(e && e[0] == '0');
  }();
  unsigned long long* span = next_span("tp_reduce_add");
  CUtensorMap pf_map;
  CUtensorMap none{};
  const PrefetchArgs pf = take_prefetch(&pf_map, none);
  auto args = std::make_tuple(reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), T, H,
                              reinterpret_cast<const char*>(buf), flags_off, (int)tp, (int)maxT, (int)rank,
                              (uint64_t)arrivals_per_call, reinterpret_cast<uint64_t*>(epoch_state.data_ptr<int64_t>()),
                              status.data_ptr<int>(), (uint64_t)(timeout_s * 1e9), add_residual ? 1 : 0,
                              reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), span, pf_map, pf);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (use_pdl) {
    std::apply([&](auto... a) { launch_pdl(tp_reduce_add_kernel, dim3(blocks), dim3(256), 0, st, a...); }, args);
  } else {
    std::apply([&](auto... a) { tp_reduce_add_kernel<<<blocks, 256, 0, st>>>(a...); }, args);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// Returns the all-gather arrivals each rank receives from this owner per call (CTAs).
int64_t sp_reduce_allgather(torch::Tensor peers, int64_t recv_off, int64_t rs_flags_off, int64_t ag_flags_off,
                            int64_t g_off, int64_t rstd_off, int64_t rank, int64_t tp, int64_t rpr, int64_t T,
                            int64_t H, int64_t rs_expected, double eps, torch::Tensor status, double timeout_s) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong && peers.numel() == tp);
  TORCH_CHECK(H % 8 == 0, "sp_reduce_allgather: hidden size must be a multiple of 8");
  const at::cuda::CUDAGuard g(peers.device());
  const int blocks = std::max<int64_t>(1, (rpr + 7) / 8);
  launch_pdl(sp_reduce_allgather_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), recv_off, rs_flags_off, ag_flags_off,
             g_off, rstd_off, (int)rank, (int)tp, (int)rpr, (int)T, (int)H, (uint64_t)rs_expected, (float)eps,
             status.data_ptr<int>(), (uint64_t)(timeout_s * 1e9));
  return blocks;
}

void sp_wait(int64_t local_ptr, int64_t ag_flags_off, int64_t tp, int64_t rank, int64_t expected,
             torch::Tensor status, double timeout_s) {
  const at::cuda::CUDAGuard g(status.device());
  launch_pdl(sp_wait_kernel, dim3(1), dim3(32), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const char*>(local_ptr), ag_flags_off, (int)tp, (int)rank, (uint64_t)expected,
             status.data_ptr<int>(), (uint64_t)(timeout_s * 1e9));
}

// A tensor view of comm-buffer memory (no ownership; the buffer outlives it).
torch::Tensor comm_tensor(int64_t ptr, int64_t offset, std::vector<int64_t> shape, int64_t dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype == 0 ? at::kBFloat16 : at::kFloat).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<char*>(ptr) + offset, shape, opts);
}

}  // namespace braid

// status word of this file's kernels (checked build; 0 otherwise)
namespace braid {
BRAID_BOUNDS_READER(bounds_status_comm)
}  // namespace braid
