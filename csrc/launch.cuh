// Kernel launch with the programmatic-stream-serialization attribute, so that
// a kernel's prologue (barrier init, TMEM allocation, weight prefetch) overlaps
// the tail of the preceding kernel; kernels call pdl_wait() before touching
// data the preceding kernel produced.  Works under CUDA-graph capture.
#pragma once
#include <cuda_runtime.h>
#include <c10/cuda/CUDAException.h>
#include <cstdlib>

namespace braid {

inline bool pdl_enabled() {
  static const bool on = [] {  // tuning knob: BRAID_NO_PDL=1 launches without the PDL attribute
    const char* e = getenv("BRAID_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

// `cluster` (x*y*z > 1) launches thread-block clusters of that shape.
template <typename... KArgs, typename... Args>
inline void launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  launch_pdl_cluster(kern, grid, block, smem, st, dim3(1, 1, 1), std::forward<Args>(args)...);
}

}  // namespace braid
