// fp32 "glue" kernels the engine needs around the int8 chain of a
// transformer graph: Gather, broadcasting binary ops, LayerNormalization
// (optionally emitting (min, max) partials for the DynamicQuantizeLinear
// that follows it), Softmax, Transpose, Cast, Erf.  They stand in for the
// reference's NVRTC elementwise / layout / reduction kernels for the ops of
// the int8 DistilBERT graph (src/cuda/kernels/mod.rs, src/cuda/ops/layout,
// src/cuda/reduction.rs).  All are HBM-bound; grids are capped at a multiple
// of the SM count and accesses are vectorised where the shapes allow.
#include "capi.cuh"
#include "common.cuh"
#include "glue.h"

namespace icx {

constexpr int kEltThreads = 256;

static unsigned elt_blocks(size_t n) {
  size_t b = (n + kEltThreads - 1) / kEltThreads;
  if (b < 1) b = 1;
  if (b > 148 * 16) b = 148 * 16;
  return (unsigned)b;
}

size_t dtype_size(int t) {
  switch (t) {
    case ICX_U8:
    case ICX_S8:
    case ICX_BOOL:
      return 1;
    case ICX_S64:
      return 8;
    default:
      return 4;
  }
}

// ------------------------------------------------------------------ Gather
// out[i, :] = table[idx[i], :] (axis 0, negative indices wrap, rows of D
// elements of type T: f32 embeddings, or the u8 / s8 tables of quantised
// exports).  Out-of-range indices write zeros and raise *err (checked by the
// host).
template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ table, int64_t rows,
                                   const int64_t* __restrict__ idx, size_t n, size_t D,
                                   T* __restrict__ out, int* __restrict__ err) {
  pdl_wait();
  pdl_trigger();
  const size_t total = n * D;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    const size_t i = t / D, d = t - i * D;
    int64_t r = idx[i];
    if (r < 0) r += rows;
    if (r < 0 || r >= rows) {
      if (d == 0 && err) atomicExch(err, 1);
      out[t] = T{};
      continue;
    }
    out[t] = table[(size_t)r * D + d];
  }
}

int launch_gather_rows(cudaStream_t s, const void* table, int elem_bytes, int64_t rows,
                       const int64_t* idx, size_t n, size_t D, void* out, int* err) {
  if (n * D == 0) return ICX_OK;
  // rows that are whole 16-byte vectors move as such (f32 embeddings)
  if ((D * elem_bytes) % 16 == 0 &&
      ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const size_t D16 = D * elem_bytes / 16;
    launch_pdl(gather_rows_kernel<uint4>, dim3(elt_blocks(n * D16)), dim3(kEltThreads), 0, s,
               static_cast<const uint4*>(table), rows, idx, n, D16, static_cast<uint4*>(out), err);
    ICX_LAUNCH_CHECK();
    return ICX_OK;
  }
  const dim3 g(elt_blocks(n * D)), b(kEltThreads);
  switch (elem_bytes) {
    case 1:
      launch_pdl(gather_rows_kernel<uint8_t>, g, b, 0, s, static_cast<const uint8_t*>(table), rows,
                 idx, n, D, static_cast<uint8_t*>(out), err);
      break;
    case 4:
      launch_pdl(gather_rows_kernel<uint32_t>, g, b, 0, s, static_cast<const uint32_t*>(table), rows,
                 idx, n, D, static_cast<uint32_t*>(out), err);
      break;
    case 8:
      launch_pdl(gather_rows_kernel<uint64_t>, g, b, 0, s, static_cast<const uint64_t*>(table), rows,
                 idx, n, D, static_cast<uint64_t*>(out), err);
      break;
    default:
      set_error("Gather: element size %d unsupported", elem_bytes);
      return ICX_ERR_UNSUPPORTED;
  }
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// -------------------------------------------------------- binary broadcast
struct BcastShape {
  int rank;
  int64_t out[kMaxRank];
  int64_t sa[kMaxRank];  // element strides of a (0 where broadcast)
  int64_t sb[kMaxRank];
};

template <int OP>
__device__ __forceinline__ float bin(float a, float b) {
  if (OP == kAdd) return __fadd_rn(a, b);
  if (OP == kSub) return __fsub_rn(a, b);
  if (OP == kMul) return __fmul_rn(a, b);
  return __fdiv_rn(a, b);
}

template <int OP>
__global__ void binary_same_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                   float4* __restrict__ o, size_t n4) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 x = a[i], y = b[i];
    o[i] = make_float4(bin<OP>(x.x, y.x), bin<OP>(x.y, y.y), bin<OP>(x.z, y.z), bin<OP>(x.w, y.w));
  }
}

// [rows, P] (op) [P]: an operand that repeats every P elements of the output
// (a bias row, position embeddings over the batch); P % 4 == 0.
template <int OP>
__global__ void binary_rowvec_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                     float4* __restrict__ o, size_t n4, size_t d4, int swap) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 x = a[i], y = b[i % d4];
    o[i] = swap ? make_float4(bin<OP>(y.x, x.x), bin<OP>(y.y, x.y), bin<OP>(y.z, x.z),
                              bin<OP>(y.w, x.w))
                : make_float4(bin<OP>(x.x, y.x), bin<OP>(x.y, y.y), bin<OP>(x.z, y.z),
                              bin<OP>(x.w, y.w));
  }
}

// one operand is a single element
template <int OP>
__global__ void binary_scalar_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                     float* __restrict__ o, size_t n, int scalar_is_a) {
  pdl_wait();
  pdl_trigger();
  const float sv = scalar_is_a ? a[0] : b[0];
  const float* v = scalar_is_a ? b : a;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    o[i] = scalar_is_a ? bin<OP>(sv, v[i]) : bin<OP>(v[i], sv);
}

// general broadcast with 32-bit index arithmetic (n < 2^31)
template <int OP>
__global__ void binary_bcast32_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                      float* __restrict__ o, unsigned n, BcastShape sh) {
  pdl_wait();
  pdl_trigger();
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    unsigned rem = i, ia = 0, ib = 0;
    for (int d = sh.rank - 1; d >= 0; --d) {
      const unsigned ext = (unsigned)sh.out[d];
      const unsigned c = rem % ext;
      rem /= ext;
      ia += c * (unsigned)sh.sa[d];
      ib += c * (unsigned)sh.sb[d];
    }
    o[i] = bin<OP>(a[ia], b[ib]);
  }
}

template <int OP>
__global__ void binary_bcast_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                    float* __restrict__ o, size_t n, BcastShape sh) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    size_t rem = i;
    int64_t ia = 0, ib = 0;
    for (int d = sh.rank - 1; d >= 0; --d) {
      const int64_t c = (int64_t)(rem % (size_t)sh.out[d]);
      rem /= (size_t)sh.out[d];
      ia += c * sh.sa[d];
      ib += c * sh.sb[d];
    }
    o[i] = bin<OP>(a[ia], b[ib]);
  }
}

static int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

int launch_binary(cudaStream_t s, int op, const float* a, const std::vector<int64_t>& ashape,
                  const float* b, const std::vector<int64_t>& bshape, float* out,
                  const std::vector<int64_t>& oshape) {
  const size_t n = (size_t)numel(oshape);
  if (n == 0) return ICX_OK;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const bool a_full = ashape == oshape, b_full = bshape == oshape;
  // the operand repeats along the leading axes: its shape (leading 1s
  // dropped) equals the output's trailing dimensions, e.g. a bias [D] or
  // position embeddings [S, H] added to [B, S, H]
  auto is_rowvec = [&](const std::vector<int64_t>& sh) {
    size_t k = 0;
    while (k < sh.size() && sh[k] == 1) ++k;
    const size_t r = sh.size() - k;
    if (r == 0 || r > oshape.size()) return false;
    for (size_t d = 0; d < r; ++d)
      if (sh[k + d] != oshape[oshape.size() - r + d]) return false;
    return numel(sh) % 4 == 0;
  };
  if (aligned && n % 4 == 0) {
    if (a_full && b_full) {
#define ICX_SAME(OPC)                                                                      \
  launch_pdl(binary_same_kernel<OPC>, dim3(elt_blocks(n / 4)), dim3(kEltThreads), 0, s,                        \
      reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),              \
      reinterpret_cast<float4*>(out), n / 4)
      switch (op) {
        case kAdd: ICX_SAME(kAdd); break;
        case kSub: ICX_SAME(kSub); break;
        case kMul: ICX_SAME(kMul); break;
        default: ICX_SAME(kDiv); break;
      }
#undef ICX_SAME
      ICX_LAUNCH_CHECK();
      return ICX_OK;
    }
    if ((a_full && is_rowvec(bshape)) || (b_full && is_rowvec(ashape))) {
      const int swap = a_full ? 0 : 1;
      const float* m = a_full ? a : b;
      const float* v = a_full ? b : a;
      const size_t period = (size_t)numel(a_full ? bshape : ashape);
#define ICX_ROW(OPC)                                                                       \
  launch_pdl(binary_rowvec_kernel<OPC>, dim3(elt_blocks(n / 4)), dim3(kEltThreads), 0, s,                      \
      reinterpret_cast<const float4*>(m), reinterpret_cast<const float4*>(v),              \
      reinterpret_cast<float4*>(out), n / 4, period / 4, swap)
      switch (op) {
        case kAdd: ICX_ROW(kAdd); break;
        case kSub: ICX_ROW(kSub); break;
        case kMul: ICX_ROW(kMul); break;
        default: ICX_ROW(kDiv); break;
      }
#undef ICX_ROW
      ICX_LAUNCH_CHECK();
      return ICX_OK;
    }
  }
  if (numel(ashape) == 1 || numel(bshape) == 1) {
    const int sa = numel(ashape) == 1 && numel(bshape) != 1;
#define ICX_SC(OPC) launch_pdl(binary_scalar_kernel<OPC>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, a, b, out, n, sa)
    switch (op) {
      case kAdd: ICX_SC(kAdd); break;
      case kSub: ICX_SC(kSub); break;
      case kMul: ICX_SC(kMul); break;
      default: ICX_SC(kDiv); break;
    }
#undef ICX_SC
    ICX_LAUNCH_CHECK();
    return ICX_OK;
  }
  BcastShape sh{};
  sh.rank = (int)oshape.size();
  ICX_REQUIRE(sh.rank <= kMaxRank, "broadcast: rank %d > %d", sh.rank, kMaxRank);
  auto strides = [&](const std::vector<int64_t>& shp, int64_t* st) {
    const int off = sh.rank - (int)shp.size();
    int64_t acc = 1;
    for (int d = sh.rank - 1; d >= 0; --d) {
      const int sd = d - off;
      if (sd < 0) {
        st[d] = 0;
        continue;
      }
      st[d] = shp[sd] == 1 ? 0 : acc;
      acc *= shp[sd];
    }
  };
  for (int d = 0; d < sh.rank; ++d) sh.out[d] = oshape[d];
  strides(ashape, sh.sa);
  strides(bshape, sh.sb);
#define ICX_BC(OPC)                                                                         \
  if (n < (1u << 31))                                                                       \
    launch_pdl(binary_bcast32_kernel<OPC>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, a, b, out, (unsigned)n, sh); \
  else                                                                                      \
    launch_pdl(binary_bcast_kernel<OPC>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, a, b, out, n, sh)
  switch (op) {
    case kAdd: ICX_BC(kAdd); break;
    case kSub: ICX_BC(kSub); break;
    case kMul: ICX_BC(kMul); break;
    default: ICX_BC(kDiv); break;
  }
#undef ICX_BC
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// ------------------------------------------------------- LayerNormalization
// One warp per row of D (D % 4 == 0, D <= 1024), statistics over registers
// (mean, then the centred sum of squares).  Optionally one (min, max) pair
// of y per block, seeded with 0, for the DynamicQuantizeLinear consuming y.
constexpr int kLnVec = 8;
constexpr int kLnWarps = 8;

// One row of LayerNormalization by one warp (D % 4 == 0, D <= 32*4*kLnVec)
// on values already in registers (lane l holds float4 columns l + 32 j):
// mean, then the mean of squared deviations, y = (x - mean) * rstd * g + b.
// The reference (src/operators/layer_normalization.rs:46-76) divides by
// sqrt(var + eps) and sums in ndarray's lane order; the warp-tree sums and
// the rsqrt product here differ from it by fp32 rounding (a few 1e-7 on
// outputs of order 1; a version bit-exact with the reference's order was
// measured 9.7 us against 5.9 us per config-3 LayerNorm).  Tracks the
// (min, max) of y.
__device__ __forceinline__ void ln_row(const float4 (&v)[kLnVec], const float4* __restrict__ g4,
                                       const float4* __restrict__ b4, float* __restrict__ y, int D,
                                       float eps, int lane, float& mn, float& mx) {
  const int nv = D / 4;
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kLnVec; ++j) sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / (float)D;
  float sq = 0.0f;
#pragma unroll
  for (int j = 0; j < kLnVec; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) {
      const float a = v[j].x - mean, b = v[j].y - mean, cc = v[j].z - mean, d = v[j].w - mean;
      sq += (a * a + b * b) + (cc * cc + d * d);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq / (float)D + eps);
  float4* yr = reinterpret_cast<float4*>(y);
#pragma unroll
  for (int j = 0; j < kLnVec; ++j) {
    const int c = lane + 32 * j;
    if (c < nv) {
      const float4 g = __ldg(g4 + c);
      const float4 bb = b4 ? __ldg(b4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 o;
      o.x = (v[j].x - mean) * rstd * g.x + bb.x;
      o.y = (v[j].y - mean) * rstd * g.y + bb.y;
      o.z = (v[j].z - mean) * rstd * g.z + bb.z;
      o.w = (v[j].w - mean) * rstd * g.w + bb.w;
      yr[c] = o;
      mn = fminf(mn, fminf(fminf(o.x, o.y), fminf(o.z, o.w)));
      mx = fmaxf(mx, fmaxf(fmaxf(o.x, o.y), fmaxf(o.z, o.w)));
    }
  }
}

__device__ __forceinline__ void ln_load(const float* __restrict__ x, int nv, int lane,
                                        float4 (&v)[kLnVec]) {
  const float4* xr = reinterpret_cast<const float4*>(x);
#pragma unroll
  for (int j = 0; j < kLnVec; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < nv ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Warps stride over rows; the next row's loads are issued before the current
// row is normalised, so a warp's second row does not wait for its own load.
__global__ void __launch_bounds__(32 * kLnWarps)
    layernorm_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                     const float* __restrict__ beta, float* __restrict__ y, int rows, int D,
                     float eps, float2* __restrict__ minmax) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float mn = 0.0f, mx = 0.0f;
  const int nv = D / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  const int stride = gridDim.x * kLnWarps;
  int row = blockIdx.x * kLnWarps + w;
  float4 cur[kLnVec];
  if (row < rows) ln_load(x + (size_t)row * D, nv, lane, cur);
  while (row < rows) {
    const int next = row + stride;
    float4 nxt[kLnVec];
    if (next < rows) ln_load(x + (size_t)next * D, nv, lane, nxt);
    ln_row(cur, g4, b4, y + (size_t)row * D, D, eps, lane, mn, mx);
#pragma unroll
    for (int j = 0; j < kLnVec; ++j) cur[j] = nxt[j];
    row = next;
  }
  if (minmax) {
    __shared__ float2 red[kLnWarps];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) red[w] = make_float2(mn, mx);
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int i = 1; i < kLnWarps; ++i) {
        mn = fminf(mn, red[i].x);
        mx = fmaxf(mx, red[i].y);
      }
      minmax[blockIdx.x] = make_float2(mn, mx);
    }
  }
}

int layernorm_partials(size_t rows) {
  // grid-stride over rows with at most 2 blocks per SM: few partials for
  // the DynamicQuantizeLinear that reads them
  size_t b = (rows + kLnWarps - 1) / kLnWarps;
  if (b > 148 * 2) b = 148 * 2;
  return b < 1 ? 1 : (int)b;
}

int launch_layernorm(cudaStream_t s, const float* x, const float* gamma, const float* beta,
                     float* y, size_t rows, size_t D, float eps, float* minmax, int* n_minmax) {
  ICX_REQUIRE(D % 4 == 0 && D <= 32 * 4 * kLnVec,
              "LayerNormalization: last dimension %zu unsupported (multiple of 4, <= %d)", D,
              32 * 4 * kLnVec);
  ICX_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0,
              "LayerNormalization: buffers must be 16-byte aligned");
  const int blocks = layernorm_partials(rows);
  if (n_minmax) *n_minmax = blocks;
  if (rows == 0) return ICX_OK;
  launch_pdl(layernorm_kernel, dim3(blocks), dim3(32 * kLnWarps), 0, s, x, gamma, beta, y, (int)rows, (int)D, eps,
                                                    reinterpret_cast<float2*>(minmax));
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// ------------------------------------------------------------------ Softmax
// Row softmax over the last axis, one warp per row (D <= 1024).
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ y, int rows,
                               int D) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + (size_t)row * D;
  float* yr = y + (size_t)row * D;
  float v[32];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < D ? xr[c] : -INFINITY;
    m = fmaxf(m, v[j]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < D ? expf(v[j] - m) : 0.0f;
    sum += v[j];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = lane + 32 * j;
    if (c < D) yr[c] = v[j] * inv;
  }
}

// Attention-score softmax fused with its two producers: y = softmax(x / c +
// mask[b, :]) over the last axis, with the division and the addition each
// rounded exactly as the separate Div and Add ops round them.  Rows are
// [batch, heads, queries]; the additive mask has one row of D per batch
// (broadcast over heads and queries), or is absent.  In place is allowed.
template <int PER_LANE>
__global__ void scale_mask_softmax_kernel(const float* __restrict__ x, float* __restrict__ y,
                                          int rows, int D, float c,
                                          const float* __restrict__ mask, int rows_per_batch) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + (size_t)row * D;
  float* yr = y + (size_t)row * D;
  const float* mr = mask ? mask + (size_t)(row / rows_per_batch) * D : nullptr;
  float v[PER_LANE];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int col = lane + 32 * j;
    float t = -INFINITY;
    if (col < D) {
      t = __fdiv_rn(xr[col], c);
      if (mr) t = __fadd_rn(t, mr[col]);
    }
    v[j] = t;
    m = fmaxf(m, t);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int col = lane + 32 * j;
    v[j] = col < D ? expf(v[j] - m) : 0.0f;
    sum += v[j];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int col = lane + 32 * j;
    if (col < D) yr[col] = v[j] * inv;
  }
}

int launch_scale_mask_softmax(cudaStream_t s, const float* x, float* y, size_t rows, size_t D,
                              float c, const float* mask, size_t rows_per_batch) {
  ICX_REQUIRE(D >= 1 && D <= 1024, "Softmax: last dimension %zu unsupported (1..1024)", D);
  if (rows == 0) return ICX_OK;
  const int wpb = 8;
  const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
  const int rpb = (int)(rows_per_batch ? rows_per_batch : rows);
  if (D <= 128)
    launch_pdl(scale_mask_softmax_kernel<4>, dim3(grid), dim3(32 * wpb), 0, s, x, y, (int)rows, (int)D, c, mask, rpb);
  else if (D <= 512)
    launch_pdl(scale_mask_softmax_kernel<16>, dim3(grid), dim3(32 * wpb), 0, s, x, y, (int)rows, (int)D, c, mask, rpb);
  else
    launch_pdl(scale_mask_softmax_kernel<32>, dim3(grid), dim3(32 * wpb), 0, s, x, y, (int)rows, (int)D, c, mask, rpb);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

int launch_softmax(cudaStream_t s, const float* x, float* y, size_t rows, size_t D) {
  ICX_REQUIRE(D >= 1 && D <= 1024, "Softmax: last dimension %zu unsupported (1..1024)", D);
  if (rows == 0) return ICX_OK;
  const int wpb = 8;
  launch_pdl(softmax_kernel, dim3((unsigned)((rows + wpb - 1) / wpb)), dim3(32 * wpb), 0, s, x, y, (int)rows, (int)D);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// ---------------------------------------------------------------- Transpose
struct PermShape {
  int rank;
  int64_t out[kMaxRank];
  int64_t in_stride[kMaxRank];  // input element stride of each output axis
};

template <typename T>
__global__ void transpose32_kernel(const T* __restrict__ x, T* __restrict__ y, unsigned n,
                                   PermShape ps) {
  pdl_wait();
  pdl_trigger();
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    unsigned rem = i, src = 0;
    for (int d = ps.rank - 1; d >= 0; --d) {
      const unsigned ext = (unsigned)ps.out[d];
      const unsigned c = rem % ext;
      rem /= ext;
      src += c * (unsigned)ps.in_stride[d];
    }
    y[i] = x[src];
  }
}

template <typename T>
__global__ void transpose_kernel(const T* __restrict__ x, T* __restrict__ y, size_t n,
                                 PermShape ps) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    size_t rem = i;
    int64_t src = 0;
    for (int d = ps.rank - 1; d >= 0; --d) {
      const int64_t c = (int64_t)(rem % (size_t)ps.out[d]);
      rem /= (size_t)ps.out[d];
      src += c * ps.in_stride[d];
    }
    y[i] = x[src];
  }
}

int launch_transpose(cudaStream_t s, const void* x, int elem_bytes,
                     const std::vector<int64_t>& in_shape, const std::vector<int64_t>& perm,
                     void* y) {
  PermShape ps{};
  ps.rank = (int)in_shape.size();
  ICX_REQUIRE(ps.rank <= kMaxRank, "Transpose: rank %d > %d", ps.rank, kMaxRank);
  int64_t st[kMaxRank];
  int64_t acc = 1;
  for (int d = ps.rank - 1; d >= 0; --d) {
    st[d] = acc;
    acc *= in_shape[d];
  }
  size_t n = 1;
  for (int d = 0; d < ps.rank; ++d) {
    ps.out[d] = in_shape[perm[d]];
    ps.in_stride[d] = st[perm[d]];
    n *= (size_t)ps.out[d];
  }
  if (n == 0) return ICX_OK;
  switch (elem_bytes) {
    case 1:
      launch_pdl(transpose_kernel<uint8_t>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, 
          static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), n, ps);
      break;
    case 4:
      if (n < (1u << 31))
        launch_pdl(transpose32_kernel<uint32_t>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, 
            static_cast<const uint32_t*>(x), static_cast<uint32_t*>(y), (unsigned)n, ps);
      else
        launch_pdl(transpose_kernel<uint32_t>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, 
            static_cast<const uint32_t*>(x), static_cast<uint32_t*>(y), n, ps);
      break;
    case 8:
      launch_pdl(transpose_kernel<uint64_t>, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, 
          static_cast<const uint64_t*>(x), static_cast<uint64_t*>(y), n, ps);
      break;
    default:
      set_error("Transpose: element size %d unsupported", elem_bytes);
      return ICX_ERR_UNSUPPORTED;
  }
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// --------------------------------------------------------------------- Cast
template <typename S, typename D>
__global__ void cast_kernel(const S* __restrict__ x, D* __restrict__ y, size_t n) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = (D)x[i];
}

int launch_cast(cudaStream_t s, const void* x, int from, void* y, int to, size_t n) {
  if (n == 0) return ICX_OK;
  if (to == from) {
    ICX_CUDA(cudaMemcpyAsync(y, x, n * dtype_size(from), cudaMemcpyDeviceToDevice, s));
    return ICX_OK;
  }
  const unsigned b = elt_blocks(n);
#define ICX_CAST(ST, DT) \
  launch_pdl((cast_kernel<ST, DT>), dim3(b), dim3(kEltThreads), 0, s, static_cast<const ST*>(x), static_cast<DT*>(y), n)
  if (to == ICX_F32) {
    switch (from) {
      case ICX_S32: ICX_CAST(int32_t, float); break;  // round to nearest: Rust `as f32`
      case ICX_S64: ICX_CAST(int64_t, float); break;
      case ICX_U8: ICX_CAST(uint8_t, float); break;
      case ICX_S8: ICX_CAST(int8_t, float); break;
      default: set_error("Cast: source type %d unsupported", from); return ICX_ERR_UNSUPPORTED;
    }
  } else if (to == ICX_S64 && from == ICX_S32) {
    ICX_CAST(int32_t, int64_t);
  } else if (to == ICX_S32 && from == ICX_S64) {
    ICX_CAST(int64_t, int32_t);
  } else {
    set_error("Cast: %d -> %d unsupported", from, to);
    return ICX_ERR_UNSUPPORTED;
  }
#undef ICX_CAST
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// ---------------------------------------------------------------------- Erf
// The Abramowitz & Stegun 7.1.26 formula of the reference's CPU Erf
// (src/operators/erf.rs:30-40), each operation rounded separately.
__device__ __forceinline__ float erf_as(float v) {
  const float sign = isnan(v) ? v : (signbit(v) ? -1.0f : 1.0f);
  const float a = fabsf(v);
  const float t = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(0.3275911f, a)));
  float p = __fsub_rn(__fmul_rn(1.0614054f, t), 1.4531521f);
  p = __fadd_rn(__fmul_rn(p, t), 1.4214138f);
  p = __fsub_rn(__fmul_rn(p, t), 0.28449672f);
  p = __fadd_rn(__fmul_rn(p, t), 0.2548296f);
  p = __fmul_rn(p, t);
  const float e = expf(__fmul_rn(-a, a));
  return __fmul_rn(sign, __fsub_rn(1.0f, __fmul_rn(p, e)));
}

__global__ void erf_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = erf_as(x[i]);
}

// The exported erf-GELU subgraph op by op: Div(x, sqrt2) -> Erf -> Add(1)
// -> Mul(x, .) -> Mul(., 0.5), for GELUs that follow no fusable GEMM.
__global__ void gelu_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
  pdl_wait();
  pdl_trigger();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    const float e = erf_as(__fdiv_rn(v, 1.41421353816986083984375f));
    y[i] = __fmul_rn(__fmul_rn(v, __fadd_rn(e, 1.0f)), 0.5f);
  }
}

int launch_erf(cudaStream_t s, const float* x, float* y, size_t n) {
  if (n == 0) return ICX_OK;
  launch_pdl(erf_kernel, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, x, y, n);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

int launch_gelu(cudaStream_t s, const float* x, float* y, size_t n) {
  if (n == 0) return ICX_OK;
  launch_pdl(gelu_kernel, dim3(elt_blocks(n)), dim3(kEltThreads), 0, s, x, y, n);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

}  // namespace icx
