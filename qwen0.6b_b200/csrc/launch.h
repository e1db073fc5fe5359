// Internal: kernel launch with an optional programmatic-dependent-launch
// attribute, shared by the translation units of libqwen_b200.so.
#pragma once
#include <cuda_runtime.h>

// Launches `kernel` on `st`; with pdl, as a programmatic dependent of the
// stream's previous kernel (it may start before that kernel ends and must call
// griddepcontrol.wait before touching its outputs).
template <typename... KArgs, typename... Args>
cudaError_t qb200_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
