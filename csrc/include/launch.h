// Kernel launch helper: every kernel of the decode step is launched with programmatic stream
// serialization so its prologue overlaps the tail of the kernel before it (the kernels call
// griddepcontrol.wait before touching data produced upstream). Can be disabled at runtime
// (MESH_PDL=0) for A/B measurements.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>

namespace mesh {

inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESH_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// cluster_x > 1 launches thread-block clusters of cluster_x CTAs along x
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kc(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  int n = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  return launch_kc(kern, grid, block, smem, st, 1, std::forward<Args>(args)...);
}

}  // namespace mesh
