// launch.h -- kernel launch with optional programmatic dependent launch (PDL).
//
// With `pdl`, the launch carries cudaLaunchAttributeProgrammaticStreamSerialization:
// the kernel may start while the previous kernel of the stream is still running;
// it must execute griddepcontrol.wait (dev::GridWait) before touching anything
// the previous kernel writes.  Captured into a CUDA graph this becomes a
// programmatic dependency edge.
#pragma once

#include <cuda_runtime.h>

#include "common.h"

namespace rpgb {

template <typename... Args>
void LaunchKernelArgs(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  void* argv[] = {static_cast<void*>(&args)...};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1u : 0u;
  RPGB_CUDA(cudaLaunchKernelExC(&cfg, fn, argv));
}

// As LaunchKernelArgs, with thread-block clusters of `cluster_x` blocks along x.
template <typename... Args>
void LaunchKernelClusterArgs(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             unsigned cluster_x, Args... args) {
  void* argv[] = {static_cast<void*>(&args)...};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2u : 1u;
  RPGB_CUDA(cudaLaunchKernelExC(&cfg, fn, argv));
}

}  // namespace rpgb
