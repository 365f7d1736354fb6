// Fused fp32 attention for the engine's attention fusion: for each
// (batch, head) and 64-query tile,
//     ctx = softmax(Q K^T / c + mask) V
// in one kernel, with online (running max / running sum) softmax over
// 64-key tiles, so the [B, heads, S, S] score tensor never reaches HBM.
// It replaces the MatMul -> Div -> Add -> Softmax -> MatMul sequence the
// reference runs as cuBLAS SGEMMs and NVRTC kernels (src/cuda/matmul.rs,
// src/cuda/reduction.rs).  Arithmetic is fp32 throughout, like the
// reference: Div by c and Add of the mask are each rounded as the separate
// ops round them; the softmax normalisation order differs (online), within
// fp32 rounding.
//
// Layout: q / k / v rows are `ld` floats apart (the merged QKV GEMM output
// has ld = 3H), head h occupies columns [h*dh, (h+1)*dh); ctx is [B, S, H].
// Tiles: 128 threads; thread (ty, tx) = (tid / 16, tid % 16) owns score
// rows ty + 8 i (i < 8) and key columns tx + 16 j (j < 4), and context
// columns 4 tx .. 4 tx + 3 of the same rows: 12 shared 16-byte loads per
// 128 FMAs.  Shared rows are padded to 68 floats so the strided column
// pattern is bank-conflict free.
#include "capi.cuh"
#include "common.cuh"
#include "glue.h"

namespace icx {

constexpr int kAttDh = 64;
constexpr int kAttTile = 64;
constexpr int kAttPad = 68;
constexpr int kAttThreads = 128;
constexpr int kAttRows = 8;  // score / context rows per thread
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kAttThreads)
    attention_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                         const float* __restrict__ v, int ld, float* __restrict__ out,
                         int H, int S, int nh, float c, const float* __restrict__ mask,
                         int mask_per_batch) {
  extern __shared__ float sm[];
  float* sQ = sm;                           // [64][68] query rows
  float* sK = sQ + kAttTile * kAttPad;      // [64][68] key rows
  float* sV = sK + kAttTile * kAttPad;      // [64][68] value rows
  float* sP = sV + kAttTile * kAttPad;      // [64][68] probabilities
  const int bh = blockIdx.x;
  const int b = bh / nh, h = bh % nh;
  const int q0 = blockIdx.y * kAttTile;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const size_t head = (size_t)b * S * ld + (size_t)h * kAttDh;
  const float* mrow = mask ? mask + (mask_per_batch ? (size_t)b * S : 0) : nullptr;
  int cexp;
  const bool c_pow2 = frexpf(c, &cexp) == 0.5f;
  const float inv_c = 1.0f / c;

  // load the query tile (16 threads per 256-byte row)
  for (int r = tid >> 4; r < kAttTile; r += kAttThreads / 16) {
    const int qi = q0 + r;
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qi < S) val = *reinterpret_cast<const float4*>(q + head + (size_t)qi * ld + tx * 4);
    *reinterpret_cast<float4*>(sQ + r * kAttPad + tx * 4) = val;
  }

  float m_run[kAttRows], l_run[kAttRows], acc[kAttRows][4];
#pragma unroll
  for (int i = 0; i < kAttRows; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.0f;
#pragma unroll
    for (int d = 0; d < 4; ++d) acc[i][d] = 0.0f;
  }

  for (int k0 = 0; k0 < S; k0 += kAttTile) {
    __syncthreads();  // previous tile's sK / sV / sP reads are done
    for (int r = tid >> 4; r < kAttTile; r += kAttThreads / 16) {
      const int ki = k0 + r;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (ki < S) {
        kv = *reinterpret_cast<const float4*>(k + head + (size_t)ki * ld + tx * 4);
        vv = *reinterpret_cast<const float4*>(v + head + (size_t)ki * ld + tx * 4);
      }
      *reinterpret_cast<float4*>(sK + r * kAttPad + tx * 4) = kv;
      *reinterpret_cast<float4*>(sV + r * kAttPad + tx * 4) = vv;
    }
    __syncthreads();

    // scores for rows ty + 8 i, keys tx + 16 j
    float s[kAttRows][4];
#pragma unroll
    for (int i = 0; i < kAttRows; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < kAttDh; d += 4) {
      float4 qa[kAttRows], ka[4];
#pragma unroll
      for (int i = 0; i < kAttRows; ++i) qa[i] = *reinterpret_cast<const float4*>(sQ + (ty + 8 * i) * kAttPad + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) ka[j] = *reinterpret_cast<const float4*>(sK + (tx + 16 * j) * kAttPad + d);
#pragma unroll
      for (int i = 0; i < kAttRows; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qa[i].x, ka[j].x, s[i][j]);
          s[i][j] = fmaf(qa[i].y, ka[j].y, s[i][j]);
          s[i][j] = fmaf(qa[i].z, ka[j].z, s[i][j]);
          s[i][j] = fmaf(qa[i].w, ka[j].w, s[i][j]);
        }
    }
    // Div(c), Add(mask), out-of-range keys -> -inf; online softmax update
#pragma unroll
    for (int i = 0; i < kAttRows; ++i) {
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + tx + 16 * j;
        // Div(c): when c is a power of two, x * (1/c) is the same correctly
        // rounded value as x / c, without the division sequence
        float t = c_pow2 ? __fmul_rn(s[i][j], inv_c) : __fdiv_rn(s[i][j], c);
        if (mrow) t = __fadd_rn(t, key < S ? mrow[key] : 0.0f);
        if (key >= S) t = -INFINITY;
        s[i][j] = t;
        rmax = fmaxf(rmax, t);
      }
#pragma unroll
      for (int o = 8; o; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
      const float m_new = fmaxf(m_run[i], rmax);
      // exp(a - m) = 2^(a*log2e - m*log2e): one FMA and the hardware exp2
      const float ml = m_new * kLog2e;
      const float alpha = m_run[i] == -INFINITY ? 0.0f : ex2f(fmaf(m_run[i], kLog2e, -ml));
      float rsum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = s[i][j] == -INFINITY ? 0.0f : ex2f(fmaf(s[i][j], kLog2e, -ml));
        s[i][j] = p;
        rsum += p;
      }
#pragma unroll
      for (int o = 8; o; o >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
      l_run[i] = l_run[i] * alpha + rsum;
      m_run[i] = m_new;
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[i][d] *= alpha;
#pragma unroll
      for (int j = 0; j < 4; ++j) sP[(ty + 8 * i) * kAttPad + tx + 16 * j] = s[i][j];
    }
    __syncthreads();
    // acc[row][4 tx .. 4 tx + 3] += sum_key P[row][key] V[key][.]
#pragma unroll 4
    for (int kk = 0; kk < kAttTile; kk += 4) {
      float4 pa[kAttRows], va[4];
#pragma unroll
      for (int i = 0; i < kAttRows; ++i) pa[i] = *reinterpret_cast<const float4*>(sP + (ty + 8 * i) * kAttPad + kk);
#pragma unroll
      for (int u = 0; u < 4; ++u) va[u] = *reinterpret_cast<const float4*>(sV + (kk + u) * kAttPad + tx * 4);
#pragma unroll
      for (int i = 0; i < kAttRows; ++i) {
        const float pu[4] = {pa[i].x, pa[i].y, pa[i].z, pa[i].w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc[i][0] = fmaf(pu[u], va[u].x, acc[i][0]);
          acc[i][1] = fmaf(pu[u], va[u].y, acc[i][1]);
          acc[i][2] = fmaf(pu[u], va[u].z, acc[i][2]);
          acc[i][3] = fmaf(pu[u], va[u].w, acc[i][3]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kAttRows; ++i) {
    const int qi = q0 + ty + 8 * i;
    if (qi >= S) continue;
    const float inv = 1.0f / l_run[i];
    *reinterpret_cast<float4*>(out + ((size_t)b * S + qi) * H + (size_t)h * kAttDh + tx * 4) =
        make_float4(acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv);
  }
}

bool attention_supported(int64_t dh, int64_t ld, int64_t H) {
  return dh == kAttDh && ld % 4 == 0 && H % 4 == 0;
}

int launch_attention_f32(cudaStream_t s, const float* q, const float* k, const float* v, int64_t ld,
                         float* out, int64_t B, int64_t S, int64_t H, int64_t nh, float c,
                         const float* mask, bool mask_per_batch) {
  ICX_REQUIRE(attention_supported(H / nh, ld, H), "Attention: head size %lld unsupported",
              (long long)(H / nh));
  ICX_REQUIRE((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) == 0,
              "Attention: q/k/v/out must be 16-byte aligned");
  const int smem = 4 * kAttTile * kAttPad * (int)sizeof(float);
  ICX_CUDA(cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid((unsigned)(B * nh), (unsigned)((S + kAttTile - 1) / kAttTile));
  attention_f32_kernel<<<grid, kAttThreads, smem, s>>>(q, k, v, (int)ld, out, (int)H, (int)S, (int)nh,
                                                       c, mask, mask_per_batch ? 1 : 0);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

}  // namespace icx
