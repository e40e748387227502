// Launch helpers: per-device one-time kernel attributes and cluster launches.
#pragma once

#include "common.cuh"

namespace lfb {

// Raise a kernel's dynamic shared-memory limit on the current device when `bytes`
// exceeds what was configured there before, and ask for the largest shared-memory
// carveout: otherwise the driver may size the SM's split for one CTA of a kernel that
// is meant to run two per SM (a function attribute of this process, not a device
// setting).  `configured` holds one entry per device (devices 0..63) for this kernel.
template <typename Kernel>
inline int ensure_smem(Kernel kernel, int bytes, int* configured) {
  if (bytes <= 48 * 1024) return LF_OK;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return check_launch("cudaGetDevice");
  int& have = configured[device & 63];
  if (have >= bytes) return LF_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return check_launch("cudaFuncSetAttribute");
  have = bytes;
  return LF_OK;
}

// Launch `kernel` with a (1, 1, cluster_z) thread-block cluster.
template <typename... Params, typename... Args>
inline cudaError_t launch_cluster_z(void (*kernel)(Params...), dim3 grid, dim3 block,
                                    size_t smem, cudaStream_t stream, int cluster_z,
                                    Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = cluster_z;
  config.attrs = attr;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

}  // namespace lfb
