// DynamicQuantizeLinear on the GPU, bit-exact with the reference CPU forward
// (src/operators/dynamic_quantize_linear.rs:32-112).
//
// Two HBM-bound passes:
//   1. dql_minmax_kernel: vectorised 16-byte loads, per-thread fminf/fmaxf
//      seeded with 0 (fminf/fmaxf drop NaN exactly like the reference's
//      `continue`), warp-shuffle then block reduction, one (min, max) pair
//      per block written to the caller's workspace.  It also zeroes the
//      optional row-sum output.
//   2. dql_quantize_kernel: every block folds the partials (a few KB, L2
//      resident), derives scale/zero-point in f64 exactly as the reference
//      does, then quantises 512 elements per warp iteration (four coalesced
//      512-byte loads, four coalesced 128-byte stores) and optionally
//      accumulates per-row sums of y.
//
// Exactness of the per-element quantisation.  The reference computes
// rte(f64(x) / scale) with an f64 division.  Here t = x * f32(1/scale) is
// computed in f32; since |x / scale| <= 255, |t - x/scale| < 3.1e-5.  If t is
// farther than 1e-4 from the nearest half-integer, rounding t and rounding
// the exact quotient give the same integer, so rintf(t) is the reference's
// result.  The vector path rounds u = fma(x, f32(1/scale), zp) instead
// (|u - (x/scale + zp)| < 4.6e-5, zp an integer), with the same 1e-4 band.
// Otherwise (about 0.02% of random inputs, and all exact ties) the
// element takes the f64 division path.  Non-finite values and scales whose
// reciprocal is not a normal f32 also take the f64 path.
#include <mutex>

#include "capi.cuh"
#include "common.cuh"

namespace icx {

constexpr int kMinmaxThreads = 512;
constexpr int kQuantThreads = 256;
constexpr int kMaxPartials = ICX_MAX_MINMAX_PARTIALS;

__device__ __forceinline__ void warp_minmax(float& mn, float& mx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
}

// Block-wide (min, max) reduction; result valid in thread 0.
template <int THREADS>
__device__ __forceinline__ void block_minmax(float& mn, float& mx) {
  __shared__ float s_mn[THREADS / 32], s_mx[THREADS / 32];
  warp_minmax(mn, mx);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    s_mn[w] = mn;
    s_mx[w] = mx;
  }
  __syncthreads();
  if (w == 0) {
    mn = l < THREADS / 32 ? s_mn[l] : 0.0f;
    mx = l < THREADS / 32 ? s_mx[l] : 0.0f;
    warp_minmax(mn, mx);
  }
}

__global__ void __launch_bounds__(kMinmaxThreads)
    dql_minmax_kernel(const float* __restrict__ x, size_t n,
                      float2* __restrict__ partials,
                      int32_t* __restrict__ rowsum, size_t nrows) {
  pdl_wait();
  pdl_trigger();
  float mn = 0.0f, mx = 0.0f;  // the reference seeds the scan with 0.0
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t head = n;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const size_t n4 = n / 4;
    size_t i = tid;
    // four independent 16-byte loads in flight per thread
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(x4 + i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        mn = fminf(fminf(mn, v[u].x), fminf(v[u].y, fminf(v[u].z, v[u].w)));
        mx = fmaxf(fmaxf(mx, v[u].x), fmaxf(v[u].y, fmaxf(v[u].z, v[u].w)));
      }
    }
    for (; i < n4; i += stride) {
      float4 v = __ldg(x4 + i);
      mn = fminf(fminf(mn, v.x), fminf(v.y, fminf(v.z, v.w)));
      mx = fmaxf(fmaxf(mx, v.x), fmaxf(v.y, fmaxf(v.z, v.w)));
    }
    head = n4 * 4;
  } else {
    head = 0;
  }
  for (size_t i = head + tid; i < n; i += stride) {
    float v = __ldg(x + i);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  block_minmax<kMinmaxThreads>(mn, mx);
  if (threadIdx.x == 0) partials[blockIdx.x] = make_float2(mn, mx);
  if (rowsum != nullptr)
    for (size_t r = tid; r < nrows; r += stride) rowsum[r] = 0;
}

struct DqlParams {
  double scale;   // f64 scale (0 when min == max)
  float inv32;    // f32(1 / scale) for the fast path
  float zpf;      // zero point as float
  int fast;       // inv32 usable
  int zero;       // min == max: everything quantises to 0
};

// scale / zero point exactly as dynamic_quantize_linear.rs:75-92.
__device__ __forceinline__ DqlParams dql_params(float fmn, float fmx) {
  DqlParams p;
  const double mn = (double)fmn, mx = (double)fmx;
  if (mn == mx) {
    p.scale = 0.0;
    p.inv32 = 0.0f;
    p.zpf = 0.0f;
    p.fast = 0;
    p.zero = 1;
    return p;
  }
  p.zero = 0;
  p.scale = (mx - mn) / 255.0;
  double izp = rint(0.0 - mn / p.scale);
  izp = izp < 0.0 ? 0.0 : (izp > 255.0 ? 255.0 : izp);  // NaN handled below
  if (isnan(izp)) izp = 0.0;
  p.zpf = (float)izp;
  const double inv = 1.0 / p.scale;
  p.inv32 = (float)inv;
  p.fast = (isfinite(p.scale) && inv >= 1.2e-38 && inv <= 3.0e38) ? 1 : 0;
  return p;
}

// f64 division path (ties, near-ties, non-finite inputs, extreme scales);
// kept out of line so the common path stays small.
__device__ __noinline__ uint32_t quant_exact(float xv, double scale, float zpf) {
  const double q = rint((double)xv / scale) + (double)zpf;
  return q > 0.0 ? (q < 255.0 ? (uint32_t)q : 255u) : 0u;  // NaN -> 0
}

__device__ __forceinline__ uint32_t quant1(float xv, const DqlParams& p) {
  if (p.zero) return 0u;
  if (p.fast) {
    const float t = xv * p.inv32;
    const float r = rintf(t);
    const float f = fabsf(t - r);
    if (fabsf(f - 0.5f) > 1e-4f) {
      const float q = r + p.zpf;
      return q > 0.0f ? (q < 255.0f ? (uint32_t)q : 255u) : 0u;
    }
  }
  return quant_exact(xv, p.scale, p.zpf);
}

// Four elements at once.  Common case (finite scale, no element within 1e-4
// of a half-integer): u = x * (1/scale) + zp in one FMA, clamped to [0, 255]
// with fmaxf / fminf (NaN -> 0; clamping first is exact because the bounds
// are integers), then rounded to nearest even by adding 1.5 * 2^23: the sum
// lies in [2^23, 2^24), where the float spacing is 1, so its low byte is the
// quantised value and subtracting the constant again gives it as a float.
// All full-rate FP32 operations; one compare per four elements decides
// whether any of them lies in the near-tie band.  Otherwise every element
// takes quant1 (with its exact f64 path where needed).
template <bool SUM>
__device__ __forceinline__ uint32_t quant4(float4 v, const DqlParams& p, uint32_t& sum) {
  if (p.fast) {
    // u = x * f32(1/scale) + zp in one rounding: |u - (x/scale + zp)| <=
    // 255 * 2^-24 + 2^-15 < 4.6e-5 (|u| < 512), so away from the 1e-4 band
    // around half-integers rint(u) = rte(x/scale) + zp (zp is an integer)
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    const float c0 = fminf(fmaxf(__fmaf_rn(v.x, p.inv32, p.zpf), 0.0f), 255.0f);
    const float c1 = fminf(fmaxf(__fmaf_rn(v.y, p.inv32, p.zpf), 0.0f), 255.0f);
    const float c2 = fminf(fmaxf(__fmaf_rn(v.z, p.inv32, p.zpf), 0.0f), 255.0f);
    const float c3 = fminf(fmaxf(__fmaf_rn(v.w, p.inv32, p.zpf), 0.0f), 255.0f);
    const float t0 = __fadd_rn(c0, kRound), t1 = __fadd_rn(c1, kRound);
    const float t2 = __fadd_rn(c2, kRound), t3 = __fadd_rn(c3, kRound);
    const float q0 = __fsub_rn(t0, kRound), q1 = __fsub_rn(t1, kRound);
    const float q2 = __fsub_rn(t2, kRound), q3 = __fsub_rn(t3, kRound);
    const float d = fmaxf(fmaxf(fabsf(c0 - q0), fabsf(c1 - q1)), fmaxf(fabsf(c2 - q2), fabsf(c3 - q3)));
    if (d < 0.5f - 1e-4f) {
      if (SUM) sum += (uint32_t)((q0 + q1) + (q2 + q3));
      const uint32_t b0 = __float_as_uint(t0), b1 = __float_as_uint(t1);
      const uint32_t b2 = __float_as_uint(t2), b3 = __float_as_uint(t3);
      return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
    }
  }
  const uint32_t a = quant1(v.x, p), b = quant1(v.y, p), c = quant1(v.z, p), d = quant1(v.w, p);
  if (SUM) sum += a + b + c + d;
  return a | (b << 8) | (c << 16) | (d << 24);
}

__global__ void __launch_bounds__(kQuantThreads, 3)
    dql_quantize_kernel(const float* __restrict__ x, size_t n,
                        const float2* __restrict__ partials, int nparts,
                        uint8_t* __restrict__ y, float* __restrict__ scale_out,
                        uint8_t* __restrict__ zp_out,
                        int32_t* __restrict__ rowsum, size_t row_len,
                        int vec16) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const size_t warp_g = ((size_t)blockIdx.x * kQuantThreads + threadIdx.x) >> 5;
  const size_t nwarps = ((size_t)gridDim.x * kQuantThreads) >> 5;
  const size_t nblk = vec16 ? n / 512 : 0;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  // this warp's first 512 elements are requested before the partials are
  // folded, so the fold and the f64 scale overlap the load latency
  float4 nv[4];
  if (warp_g < nblk) {
#pragma unroll
    for (int j = 0; j < 4; ++j) nv[j] = __ldg(x4 + warp_g * 128 + 32 * j + lane);
  }
  // every warp folds the partials itself (no block barrier) and all lanes
  // derive the f64 scale / zero point in parallel
  DqlParams p;
  {
    // eight independent loads in flight per lane (a dependent loop would pay
    // one L2 round trip per 32 partials)
    float mn = 0.0f, mx = 0.0f;
    for (int i0 = 0; i0 < nparts; i0 += 256) {
      float2 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + 32 * u + lane;
        v[u] = i < nparts ? partials[i] : make_float2(0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        mn = fminf(mn, v[u].x);
        mx = fmaxf(mx, v[u].y);
      }
    }
    warp_minmax(mn, mx);
    p = dql_params(mn, mx);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      *scale_out = (float)p.scale;
      *zp_out = (uint8_t)p.zpf;
    }
  }

  size_t done = 0;
  if (vec16) {
    // Each warp quantises 512 consecutive elements per iteration: four fully
    // coalesced 512-byte float4 loads (lane l takes float4 32*j + l) and four
    // coalesced 128-byte stores of the packed u8 words.  A 4-element word
    // never straddles a row because the host selects this path only when
    // row_len % 4 == 0 (or no row sums are requested).
    uint32_t* y4 = reinterpret_cast<uint32_t*>(y);
    // the next iteration's four loads are issued before this one is processed
    for (size_t blk = warp_g; blk < nblk; blk += nwarps) {
      const size_t base4 = blk * 128;
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = nv[j];
      const size_t nxt = blk + nwarps;
      if (nxt < nblk) {
#pragma unroll
        for (int j = 0; j < 4; ++j) nv[j] = __ldg(x4 + nxt * 128 + 32 * j + lane);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t sum = 0;
        if (rowsum == nullptr) {
          y4[base4 + 32 * j + lane] = quant4<false>(v[j], p, sum);
        } else {
          y4[base4 + 32 * j + lane] = quant4<true>(v[j], p, sum);
          const unsigned long long row =
              (unsigned long long)((base4 + 32 * j + lane) * 4 / row_len);
          const unsigned mask = __match_any_sync(0xffffffffu, row);
          const uint32_t tot = __reduce_add_sync(mask, sum);
          if (lane == __ffs(mask) - 1) atomicAdd(rowsum + row, (int32_t)tot);
        }
      }
    }
    done = nblk * 512;
  }
  // scalar path: misaligned buffers, rows not a multiple of 16, and tails
  const size_t tid = (size_t)blockIdx.x * kQuantThreads + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * kQuantThreads;
  for (size_t i = done + tid; i < n; i += stride) {
    const uint32_t q = quant1(__ldg(x + i), p);
    y[i] = (uint8_t)q;
    if (rowsum != nullptr && q != 0) atomicAdd(rowsum + i / row_len, (int32_t)q);
  }
}

// Row-wise quantise pass: each warp owns whole rows of row_len elements
// (row_len % 4 == 0, 16-byte aligned x and y) and issues all of a row's
// 16-byte loads before quantising it (up to 8 per lane in flight), so the
// per-row sum of y for the weight zero-point correction is a warp reduction
// and one plain store: no atomics and no zeroing pass.  Same arithmetic as
// dql_quantize_kernel (quant4 / quant1).
constexpr int kRowThreads = 256;

__global__ void __launch_bounds__(kRowThreads)
    dql_quantize_rows_kernel(const float* __restrict__ x, size_t n, size_t nrows, size_t row_len,
                             const float2* __restrict__ partials, int nparts,
                             uint8_t* __restrict__ y, float* __restrict__ scale_out,
                             uint8_t* __restrict__ zp_out, int32_t* __restrict__ rowsum) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const size_t warp_g = ((size_t)blockIdx.x * kRowThreads + threadIdx.x) >> 5;
  const size_t nwarps = ((size_t)gridDim.x * kRowThreads) >> 5;
  const size_t r4 = row_len / 4;  // float4 per row
  const float4* x4 = reinterpret_cast<const float4*>(x);
  uint32_t* y4 = reinterpret_cast<uint32_t*>(y);
  // this warp's first row is requested before the partials are folded
  constexpr int kU = 8;
  float4 v[kU];
  if (warp_g < nrows) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const size_t j = (size_t)lane + 32 * u;
      if (j < r4) v[u] = __ldg(x4 + warp_g * r4 + j);
    }
  }
  DqlParams p;
  {
    float mn = 0.0f, mx = 0.0f;
    for (int i0 = 0; i0 < nparts; i0 += 256) {
      float2 w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + 32 * u + lane;
        w[u] = i < nparts ? partials[i] : make_float2(0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        mn = fminf(mn, w[u].x);
        mx = fmaxf(mx, w[u].y);
      }
    }
    warp_minmax(mn, mx);
    p = dql_params(mn, mx);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      *scale_out = (float)p.scale;
      *zp_out = (uint8_t)p.zpf;
    }
  }
  for (size_t row = warp_g; row < nrows; row += nwarps) {
    const float4* xr = x4 + row * r4;
    uint32_t* yr = y4 + row * r4;
    uint32_t sum = 0;
    for (size_t j0 = 0; j0 < r4; j0 += 32 * kU) {
      if (j0 > 0) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const size_t j = j0 + lane + 32 * u;
          if (j < r4) v[u] = __ldg(xr + j);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const size_t j = j0 + lane + 32 * u;
        if (j < r4) {
          if (rowsum != nullptr) yr[j] = quant4<true>(v[u], p, sum);
          else yr[j] = quant4<false>(v[u], p, sum);
        }
      }
    }
    // the next row's first loads go out before this row's sum is reduced
    const size_t nxt = row + nwarps;
    if (nxt < nrows) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const size_t j = (size_t)lane + 32 * u;
        if (j < r4) v[u] = __ldg(x4 + nxt * r4 + j);
      }
    }
    if (rowsum != nullptr) {
      sum = __reduce_add_sync(0xffffffffu, sum);
      if (lane == 0) rowsum[row] = (int32_t)sum;
    }
  }
  // elements past the last whole row (none when row_len divides n)
  const size_t done = nrows * row_len;
  const size_t tid = (size_t)blockIdx.x * kRowThreads + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * kRowThreads;
  for (size_t i = done + tid; i < n; i += stride) y[i] = (uint8_t)quant1(__ldg(x + i), p);
}

// Launches the quantise pass over x with its (min, max) partials: the
// row-wise kernel when x and y are 16-byte aligned and rows hold a multiple
// of 4 elements, else the element-wise kernel.
static int launch_quantize(cudaStream_t s, const float* x, size_t n, const float2* partials,
                           int nparts, uint8_t* y, float* scale, uint8_t* zp, int32_t* rowsum,
                           size_t row_len, bool rowsum_zeroed) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  // (measured: the row-wise kernel pays off with row sums, whose atomics it
  // removes; without them the element-wise kernel is faster on small tensors)
  const size_t rl = row_len;
  if (rowsum != nullptr && aligned && rl % 4 == 0 && rl > 0) {
    const size_t nrows = n / rl;
    size_t blocks = (nrows * 32 + kRowThreads - 1) / kRowThreads;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    launch_pdl(dql_quantize_rows_kernel, dim3((unsigned)blocks), dim3(kRowThreads), 0, s, x, n,
               nrows, rl, partials, nparts, y, scale, zp, rowsum);
    ICX_LAUNCH_CHECK();
    return ICX_OK;
  }
  if (rowsum && !rowsum_zeroed) ICX_CUDA(cudaMemsetAsync(rowsum, 0, (n / row_len) * sizeof(int32_t), s));
  const int vec16 = aligned && (rowsum == nullptr || row_len % 4 == 0);
  size_t work = vec16 ? n / 16 : n;
  size_t qb = (work + kQuantThreads - 1) / kQuantThreads;
  if (qb < 1) qb = 1;
  if (qb > 148 * 3) qb = 148 * 3;
  launch_pdl(dql_quantize_kernel, dim3((int)qb), dim3(kQuantThreads), 0, s, x, n, partials, nparts, y,
             scale, zp, rowsum, row_len ? row_len : 1, vec16);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// Global DynamicQuantizeLinear over batch-sharded executors: the local
// partials fold into one pair (-min, max) so that a single MAX all-reduce
// across the executors yields the global (min, max) of the whole batch;
// unfold writes it back as one (min, max) partial for the quantise pass.
__global__ void minmax_fold_kernel(const float2* __restrict__ parts, int n, float* __restrict__ g) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_mn[8], s_mx[8];
  float mn = 0.0f, mx = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float2 v = parts[i];
    mn = fminf(mn, v.x);
    mx = fmaxf(mx, v.y);
  }
  warp_minmax(mn, mx);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_mn[w] = mn;
    s_mx[w] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) {
      mn = fminf(mn, s_mn[i]);
      mx = fmaxf(mx, s_mx[i]);
    }
    g[0] = -mn;
    g[1] = mx;
  }
}

__global__ void minmax_unfold_kernel(const float* __restrict__ g, float2* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) out[0] = make_float2(-g[0], g[1]);
}

int launch_minmax_fold(cudaStream_t s, const float* partials, int n, float* g) {
  launch_pdl(minmax_fold_kernel, dim3(1), dim3(256), 0, s, reinterpret_cast<const float2*>(partials),
             n, g);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

int launch_minmax_unfold(cudaStream_t s, const float* g, float* out) {
  launch_pdl(minmax_unfold_kernel, dim3(1), dim3(32), 0, s, g, reinterpret_cast<float2*>(out));
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

static int minmax_blocks(size_t n) {
  size_t per_block = (size_t)kMinmaxThreads * 16;
  size_t b = (n + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > (size_t)kMaxPartials) b = kMaxPartials;
  return (int)b;
}

int dql_minmax_partials(size_t n) { return minmax_blocks(n); }

int launch_dql_minmax(cudaStream_t s, const float* x, size_t n, float2* partials) {
  launch_pdl(dql_minmax_kernel, dim3(minmax_blocks(n)), dim3(kMinmaxThreads), 0, s, x, n, partials, nullptr, 0);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

}  // namespace icx

using namespace icx;

extern "C" size_t icx_dql_workspace_bytes(size_t n) {
  return (size_t)minmax_blocks(n) * sizeof(float2);
}

extern "C" int icx_dql_f32_u8(void* stream, const float* d_x, size_t n,
                              uint8_t* d_y, float* d_scale, uint8_t* d_zp,
                              int32_t* d_rowsum, size_t row_len,
                              void* d_workspace, size_t workspace_bytes) {
  ICX_REQUIRE(d_scale && d_zp, "DynamicQuantizeLinear: null scale/zp output");
  ICX_REQUIRE(n == 0 || (d_x && d_y), "DynamicQuantizeLinear: null x or y");
  ICX_REQUIRE(d_rowsum == nullptr || (row_len > 0 && n % row_len == 0),
              "DynamicQuantizeLinear: row_len %zu must divide n %zu", row_len,
              n);
  const int blocks = minmax_blocks(n);
  ICX_REQUIRE(d_workspace != nullptr &&
                  workspace_bytes >= (size_t)blocks * sizeof(float2),
              "DynamicQuantizeLinear: workspace %zu bytes < %zu required",
              workspace_bytes, (size_t)blocks * sizeof(float2));
  cudaStream_t s = as_stream(stream);
  const size_t nrows = d_rowsum ? n / row_len : 0;
  launch_pdl(dql_minmax_kernel, dim3(blocks), dim3(kMinmaxThreads), 0, s, 
      d_x, n, static_cast<float2*>(d_workspace), d_rowsum, nrows);
  ICX_LAUNCH_CHECK();
  return launch_quantize(s, d_x, n, static_cast<const float2*>(d_workspace), blocks, d_y, d_scale,
                         d_zp, d_rowsum, row_len, /*rowsum_zeroed=*/true);
}

extern "C" int icx_dql_quantize_f32_u8(void* stream, const float* d_x, size_t n,
                                       const float* d_minmax, int n_minmax,
                                       uint8_t* d_y, float* d_scale, uint8_t* d_zp,
                                       int32_t* d_rowsum, size_t row_len) {
  ICX_REQUIRE(d_scale && d_zp, "DynamicQuantizeLinear: null scale/zp output");
  ICX_REQUIRE(n == 0 || (d_x && d_y), "DynamicQuantizeLinear: null x or y");
  ICX_REQUIRE(d_minmax != nullptr && n_minmax >= 1 && n_minmax <= ICX_MAX_MINMAX_PARTIALS,
              "DynamicQuantizeLinear: need 1..%d (min, max) partials, got %d",
              ICX_MAX_MINMAX_PARTIALS, n_minmax);
  ICX_REQUIRE(d_rowsum == nullptr || (row_len > 0 && n % row_len == 0),
              "DynamicQuantizeLinear: row_len %zu must divide n %zu", row_len, n);
  cudaStream_t s = as_stream(stream);
  return launch_quantize(s, d_x, n, reinterpret_cast<const float2*>(d_minmax), n_minmax, d_y,
                         d_scale, d_zp, d_rowsum, row_len, /*rowsum_zeroed=*/false);
}

// ---------------------------------------------------------------------------
// Allocation-free DynamicQuantizeLinear.
//
// Some callers cannot allocate device memory at the moment they quantise:
// code running inside a fixed memory budget that was reserved up front, a
// host runtime whose allocator may not be re-entered from its execution
// thread, or an embedder that forbids cudaMalloc after start-up because
// cudaMalloc can synchronise the device.  For them this entry point keeps its
// scratch (the per-block (min, max) partials) in a file-scope device array
// instead of a caller-provided workspace.
//
// The array holds ICX_MAX_MINMAX_PARTIALS pairs (9472 bytes) and stays
// resident on every GPU that loads this library until the process exits.
// Each pair summarises at most 2^17 elements of x on this path, so the
// largest input is ICX_DQL_NOALLOC_MAX_N = 1184 * 2^17 elements (592 MiB of
// f32); larger inputs are rejected before any launch.
// Nothing in it needs clearing between calls: every block of the min/max pass
// overwrites its own slot before the quantise pass reads it.  All calls on a
// device share the one array, so two calls whose kernels overlap on the GPU
// (different streams, no ordering between them) race on it.
static __device__ __align__(256) float2 g_dql_noalloc_scratch[ICX_MAX_MINMAX_PARTIALS];
static_assert(ICX_DQL_NOALLOC_MAX_N == (unsigned long long)ICX_MAX_MINMAX_PARTIALS << 17,
              "the no-alloc limit is 2^17 elements per scratch pair");

namespace icx {
namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
float2* g_noalloc_ptr[kNoallocMaxDevices] = {};

// Device address of the scratch array on the current device.  The symbol's
// name in host code is only a host-side handle; the real address comes from
// cudaGetSymbolAddress, looked up once per device with that device current
// and cached for the life of the process.  The cache assumes the primary
// context: after cudaDeviceReset (or with another context current on the
// device) the module is loaded again at a new address, and the cached
// pointer would be stale.
int noalloc_scratch(float2** out) {
  int dev = 0;
  ICX_CUDA(cudaGetDevice(&dev));
  ICX_REQUIRE(dev >= 0 && dev < kNoallocMaxDevices, "DynamicQuantizeLinear: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    ICX_CUDA(cudaGetSymbolAddress(&p, g_dql_noalloc_scratch));
    g_noalloc_ptr[dev] = static_cast<float2*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return ICX_OK;
}
}  // namespace
}  // namespace icx

extern "C" int icx_dql_f32_u8_noalloc(void* stream, const float* d_x, size_t n,
                                      uint8_t* d_y, float* d_scale, uint8_t* d_zp,
                                      int32_t* d_rowsum, size_t row_len) {
  ICX_REQUIRE(n <= ICX_DQL_NOALLOC_MAX_N,
              "DynamicQuantizeLinear (no-alloc): n = %zu exceeds the maximum of %llu elements",
              n, (unsigned long long)ICX_DQL_NOALLOC_MAX_N);
  ICX_REQUIRE(d_scale && d_zp, "DynamicQuantizeLinear: null scale/zp output");
  ICX_REQUIRE(n == 0 || (d_x && d_y), "DynamicQuantizeLinear: null x or y");
  ICX_REQUIRE(d_rowsum == nullptr || (row_len > 0 && n % row_len == 0),
              "DynamicQuantizeLinear: row_len %zu must divide n %zu", row_len, n);
  // at most ICX_MAX_MINMAX_PARTIALS blocks, each writing one scratch pair
  const int blocks = minmax_blocks(n);
  float2* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  const size_t nrows = d_rowsum ? n / row_len : 0;
  launch_pdl(dql_minmax_kernel, dim3(blocks), dim3(kMinmaxThreads), 0, s, d_x, n, scratch, d_rowsum, nrows);
  ICX_LAUNCH_CHECK();
  return launch_quantize(s, d_x, n, scratch, blocks, d_y, d_scale, d_zp, d_rowsum, row_len,
                         /*rowsum_zeroed=*/true);
}
