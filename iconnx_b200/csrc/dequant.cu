// DequantizeLinear: y = (f32(x) - f32(zp)) * scale, per tensor or per axis.
// Arithmetic follows the reference CPU forward
// (src/operators/dequantize_linear.rs:32-179): both operands are converted to
// f32 first, one f32 subtraction, one f32 multiply (no FMA).  The reference
// GPU kernel (src/cuda/ops/quantize_kernels.rs:52-81) subtracts in 64-bit
// integers instead; the two agree whenever x - zp is exactly representable,
// and this implementation matches the CPU oracle in every case.
#include "capi.cuh"
#include "common.cuh"

namespace icx {

template <typename T>
__global__ void dequantize_kernel(const T* __restrict__ x, size_t total,
                                  size_t axis_len, size_t inner,
                                  const float* __restrict__ scale,
                                  size_t scale_len, const T* __restrict__ zp,
                                  float* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const size_t si = scale_len == 1 ? 0 : (i / inner) % axis_len;
    const float xv = (float)x[i];
    const float zv = zp ? (float)zp[si] : 0.0f;
    y[i] = __fmul_rn(__fsub_rn(xv, zv), scale[si]);
  }
}

}  // namespace icx

using namespace icx;

extern "C" int icx_dequantize_linear(void* stream, const void* d_x, int x_type,
                                     size_t outer, size_t axis_len, size_t inner,
                                     const float* d_scale, size_t scale_len,
                                     const void* d_zp, float* d_y) {
  ICX_REQUIRE(x_type == ICX_U8 || x_type == ICX_S8 || x_type == ICX_S32,
              "DequantizeLinear: input dtype must be Int8, UInt8 or Int32");
  ICX_REQUIRE(scale_len == 1 || scale_len == axis_len,
              "DequantizeLinear: per-axis scale length %zu doesn't match axis dim %zu",
              scale_len, axis_len);
  const size_t total = outer * axis_len * inner;
  if (total == 0) return ICX_OK;
  ICX_REQUIRE(d_x && d_y && d_scale, "DequantizeLinear: null pointer");
  cudaStream_t s = as_stream(stream);
  const int threads = 256;
  size_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  switch (x_type) {
    case ICX_U8:
      launch_pdl(dequantize_kernel<uint8_t>, dim3((unsigned)blocks), dim3(threads), 0, s, 
          static_cast<const uint8_t*>(d_x), total, axis_len, inner, d_scale,
          scale_len, static_cast<const uint8_t*>(d_zp), d_y);
      break;
    case ICX_S8:
      launch_pdl(dequantize_kernel<int8_t>, dim3((unsigned)blocks), dim3(threads), 0, s, 
          static_cast<const int8_t*>(d_x), total, axis_len, inner, d_scale,
          scale_len, static_cast<const int8_t*>(d_zp), d_y);
      break;
    default:
      launch_pdl(dequantize_kernel<int32_t>, dim3((unsigned)blocks), dim3(threads), 0, s, 
          static_cast<const int32_t*>(d_x), total, axis_len, inner, d_scale,
          scale_len, static_cast<const int32_t*>(d_zp), d_y);
  }
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}
