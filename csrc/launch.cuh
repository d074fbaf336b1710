// Kernel launch with the programmatic-stream-serialization attribute, so that
// a kernel's prologue (barrier init, TMEM allocation, weight prefetch) overlaps
// the tail of the preceding kernel; kernels call pdl_wait() before touching
// data the preceding kernel produced.  Works under CUDA-graph capture.
#pragma once
#include <cuda_runtime.h>
#include <c10/cuda/CUDAException.h>

namespace braid {

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

}  // namespace braid
