// Library-wide C-ABI pieces: error reporting, version, device status word.
#include "capi.cuh"
#include "common.cuh"

namespace icx {

__device__ int g_icx_device_status = 0;

static thread_local std::string t_last_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

void clear_error() { t_last_error.clear(); }

// One warp waits on an mbarrier that nothing arrives on: the bounded wait
// gives up after limit_ns, records ICX_DEVICE_TIMEOUT_SELFTEST and the kernel
// returns normally.
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, ICX_DEVICE_TIMEOUT_SELFTEST, limit_ns);
  __syncwarp();
}

}  // namespace icx

extern "C" int icx_selftest_bounded_wait(void* stream, uint64_t limit_ns) {
  ICX_REQUIRE(limit_ns > 0 && limit_ns <= 100000000ull,
              "selftest_bounded_wait: limit %llu ns outside (0, 100 ms]",
              (unsigned long long)limit_ns);
  icx::bounded_wait_selftest_kernel<<<1, 32, 0, icx::as_stream(stream)>>>(limit_ns);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

extern "C" const char* icx_last_error(void) {
  return icx::t_last_error.c_str();
}

extern "C" const char* icx_version(void) { return "iconnx_b200 0.1 sm_100a"; }

extern "C" int icx_device_status(int device, int* status_out) {
  ICX_REQUIRE(status_out != nullptr, "icx_device_status: null status_out");
  int prev = 0;
  ICX_CUDA(cudaGetDevice(&prev));
  ICX_CUDA(cudaSetDevice(device));
  int v = 0, zero = 0;
  cudaError_t e =
      cudaMemcpyFromSymbol(&v, icx::g_icx_device_status, sizeof(int));
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbol(icx::g_icx_device_status, &zero, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    icx::set_error("icx_device_status: %s", cudaGetErrorString(e));
    return ICX_ERR_CUDA;
  }
  *status_out = v;
  return ICX_OK;
}
