// Host-side helpers shared by the C-ABI translation units: thread-local
// error text and CUDA-call checking.  No entry point throws across the ABI.
#pragma once

#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/iconnx_b200.h"

namespace icx {

void set_error(const char* fmt, ...);
void clear_error();

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Launch with programmatic stream serialisation: the kernel may be scheduled
// while its predecessor on the stream finishes; it synchronises on the
// predecessor itself with griddepcontrol.wait (pdl_wait in common.cuh).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Same, launched as clusters of `cluster_x` CTAs along x (gridDim.x must be
// a multiple of it).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t s, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace icx

#define ICX_REQUIRE(cond, ...)          \
  do {                                  \
    if (!(cond)) {                      \
      ::icx::set_error(__VA_ARGS__);    \
      return ICX_ERR_INVALID;           \
    }                                   \
  } while (0)

#define ICX_CUDA(call)                                                    \
  do {                                                                    \
    cudaError_t _e = (call);                                              \
    if (_e != cudaSuccess) {                                              \
      ::icx::set_error("%s failed: %s", #call, cudaGetErrorString(_e));   \
      return ICX_ERR_CUDA;                                                \
    }                                                                     \
  } while (0)

#define ICX_LAUNCH_CHECK()                                                \
  do {                                                                    \
    cudaError_t _e = cudaGetLastError();                                  \
    if (_e != cudaSuccess) {                                              \
      ::icx::set_error("kernel launch failed: %s", cudaGetErrorString(_e)); \
      return ICX_ERR_CUDA;                                                \
    }                                                                     \
  } while (0)
