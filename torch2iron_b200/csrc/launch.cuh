// Kernel launch with programmatic dependent launch enabled.
#pragma once

#include <cuda_runtime.h>

#include "../../include/t2b.h"

namespace t2b {

template <typename Kern, typename... Args>
static int launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&... args) {
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  return e == cudaSuccess ? T2B_OK : T2B_ERR_LAUNCH;
}

// Same, as a thread-block cluster of `cluster_y` CTAs along grid y.
template <typename Kern, typename... Args>
static int launch_pdl_cluster(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_y,
                              Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = cluster_y;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  return e == cudaSuccess ? T2B_OK : T2B_ERR_LAUNCH;
}

// Raise the dynamic shared-memory limit of a kernel above 48 KB.  Cheap and
// idempotent; called before every launch that needs it.
template <typename Kern>
static int allow_smem(Kern kern, size_t bytes) {
  if (bytes <= 48 * 1024) return T2B_OK;
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess
             ? T2B_OK
             : T2B_ERR_LAUNCH;
}

}  // namespace t2b
