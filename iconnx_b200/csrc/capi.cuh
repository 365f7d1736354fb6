// Host-side helpers shared by the C-ABI translation units: thread-local
// error text and CUDA-call checking.  No entry point throws across the ABI.
#pragma once

#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/iconnx_b200.h"

namespace icx {

void set_error(const char* fmt, ...);
void clear_error();

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

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
