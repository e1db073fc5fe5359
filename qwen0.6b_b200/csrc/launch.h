// Internal: kernel launch with an optional programmatic-dependent-launch
// attribute, shared by the translation units of libqwen_b200.so.
#pragma once
#include <cuda_runtime.h>

// Launches `kernel` on `st`; with pdl, as a programmatic dependent of the
// stream's previous kernel (it may start before that kernel ends and must call
// griddepcontrol.wait before touching its outputs).
// cluster_z > 1: thread-block clusters of (1, 1, cluster_z).
template <typename... KArgs, typename... Args>
cudaError_t qb200_launch_cl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, bool pdl, int cluster_z, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = static_cast<unsigned>(cluster_z);
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t qb200_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t st, bool pdl, Args... args) {
  return qb200_launch_cl(kernel, grid, block, smem, st, pdl, 1, args...);
}
