// CPU oracle for the int8 dynamic-quantization chain — TEST INFRASTRUCTURE ONLY.
//
// This file restates, in plain C++, the reference engine's CPU operators for
//   DynamicQuantizeLinear -> MatMulInteger -> Cast -> Mul(scale) -> Add(bias)
//   [-> Div(sqrt2) -> Erf -> Add(1) -> Mul(x) -> Mul(0.5)]
// and DequantizeLinear.  Only the test suite, the smoke check and the CPU
// baseline leg of the benchmark load it; the product library never links it
// and has no CPU fallback.
//
// Reference sources restated (paths inside the iconnx crate):
//   src/operators/dynamic_quantize_linear.rs:32-112
//   src/operators/matmul_integer.rs:52-179, 189-223, 239-267
//   src/operators/cast.rs:46-48        (i32 -> f32 with `as f32`)
//   src/operators/mul.rs:26-58         (f32 broadcast multiply)
//   src/operators/add.rs:27-85         (f32 broadcast add)
//   src/operators/erf.rs:30-40         (Abramowitz & Stegun 7.1.26)
//   src/operators/dequantize_linear.rs:32-179
// and the fp32 transformer glue around the chain:
//   src/operators/layer_normalization.rs:25-80
//   src/operators/softmax.rs:21-56
//   src/operators/matmul.rs:27-186
// Those three run on ndarray 0.16 (Cargo.toml:21; no Cargo.lock is vendored,
// so the resolved patch version is unknown), whose arithmetic this file
// restates from its published algorithms:
//   * sum_axis / mean_axis over the contiguous last axis sum each lane with
//     ndarray's eight-accumulator unrolled fold (numeric_util::unrolled_fold:
//     p0..p7 take elements i % 8 of every whole group of eight, then
//     acc = ((((0 + (p0 + p4)) + (p1 + p5)) + (p2 + p6)) + (p3 + p7)), then
//     the remaining < 8 elements one by one); mean = sum / n;
//   * Array2::dot of f32 without the blas feature calls matrixmultiply 0.3
//     sgemm, whose x86-64 FMA kernel accumulates every output over k in
//     blocks of kc = 256 with one fused multiply-add per step, the first
//     block stored and later blocks added (c = c + block).

// Build flags matter: -O2 -ffp-contract=off so that no multiply-add pair is
// fused (Rust never contracts f32 expressions), and no -ffast-math.
//
// Parity is pinned by the reference's own known-answer tests and by the
// vendored ONNX 1.18 node tests (see tests/golden/).  The per-column
// b_zero_point extension follows the ONNX MatMulInteger specification, which
// the reference rejects (matmul_integer.rs:189-213), so that one feature is
// pinned only by the specification.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cfenv>
#include <vector>
#include <thread>

extern "C" {

// ---------------------------------------------------------------------------
// Rust `f64 as u8` semantics: NaN -> 0, saturate to [0, 255], truncate.
static inline uint8_t rust_f64_as_u8(double v) {
  if (std::isnan(v)) return 0;
  if (v <= 0.0) return 0;
  if (v >= 255.0) return 255;
  return (uint8_t)v;
}

// Rust f64::clamp(min, max): NaN stays NaN.
static inline double rust_clamp(double v, double lo, double hi) {
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}

// round_ties_even in f64 (nearbyint under the default FE_TONEAREST mode).
static inline double rte(double v) { return std::nearbyint(v); }

// DynamicQuantizeLinear forward.  dynamic_quantize_linear.rs:32-112.
// min/max are seeded with 0.0 and NaN is skipped (:56-69); min == max gives
// the (0..., 0.0, 0) sentinel (:75-84); scale/zp/quantise in f64 (:89-103).
void oracle_dql(const float* x, size_t n, uint8_t* y, float* scale_out,
                uint8_t* zp_out) {
  double min_x = 0.0, max_x = 0.0;
  for (size_t i = 0; i < n; ++i) {
    float v = x[i];
    if (std::isnan(v)) continue;
    double vd = (double)v;
    if (vd < min_x) min_x = vd;
    if (vd > max_x) max_x = vd;
  }
  const double qmin = 0.0, qmax = 255.0;
  if (min_x == max_x) {
    std::memset(y, 0, n);
    *scale_out = 0.0f;
    *zp_out = 0;
    return;
  }
  double scale = (max_x - min_x) / (qmax - qmin);
  double izp = rte(qmin - min_x / scale);
  uint8_t zp = rust_f64_as_u8(rust_clamp(izp, qmin, qmax));
  *scale_out = (float)scale;
  *zp_out = zp;
  for (size_t i = 0; i < n; ++i) {
    double q = rte((double)x[i] / scale) + (double)zp;
    y[i] = rust_f64_as_u8(rust_clamp(q, qmin, qmax));
  }
}

// Row sums of a u8 matrix [M, K] (helper for checking the kernel's optional
// row-sum side output; not a reference operator).
void oracle_rowsum_u8(const uint8_t* a, size_t M, size_t K, int32_t* out) {
  for (size_t m = 0; m < M; ++m) {
    int32_t s = 0;
    for (size_t k = 0; k < K; ++k) s += a[m * K + k];
    out[m] = s;
  }
}

// MatMulInteger forward.  matmul_integer.rs:239-267 (naive triple loop with
// i32 operands and accumulator).  a is [M, K] row-major, b is [K, N]
// row-major, out is [M, N].  a_signed / b_signed select i8 vs u8 element
// interpretation (the four sign variants of :100-165).  b_zp_per_col == 0 is
// the reference's scalar zero-point; b_zp_per_col != 0 applies b_zp[n] per
// output column as the ONNX specification allows (an extension the reference
// rejects at :189-213).  Overflow wraps (the reference panics; the configs
// never reach it, :24-30).
void oracle_matmul_integer(const void* a, int a_signed, const void* b,
                           int b_signed, size_t M, size_t K, size_t N,
                           int32_t a_zp, const int32_t* b_zp,
                           int b_zp_per_col, int32_t* out, int threads) {
  const uint8_t* au = (const uint8_t*)a;
  const int8_t* as = (const int8_t*)a;
  const uint8_t* bu = (const uint8_t*)b;
  const int8_t* bs = (const int8_t*)b;
  auto rows = [&](size_t r0, size_t r1) {
    for (size_t row = r0; row < r1; ++row) {
      for (size_t col = 0; col < N; ++col) {
        int32_t bz = b_zp ? (b_zp_per_col ? b_zp[col] : b_zp[0]) : 0;
        uint32_t acc = 0;
        for (size_t kk = 0; kk < K; ++kk) {
          int32_t av = (a_signed ? (int32_t)as[row * K + kk]
                                 : (int32_t)au[row * K + kk]) - a_zp;
          int32_t bv = (b_signed ? (int32_t)bs[kk * N + col]
                                 : (int32_t)bu[kk * N + col]) - bz;
          acc += (uint32_t)(av * bv);
        }
        out[row * N + col] = (int32_t)acc;
      }
    }
  };
  // threads > 1 splits rows across host threads (the "parallel upper bound"
  // CPU baseline); threads <= 1 is the reference's single-threaded loop.
  if (threads <= 1 || M < 2) {
    rows(0, M);
    return;
  }
  std::vector<std::thread> pool;
  size_t nt = (size_t)threads < M ? (size_t)threads : M;
  for (size_t t = 0; t < nt; ++t)
    pool.emplace_back(rows, M * t / nt, M * (t + 1) / nt);
  for (auto& th : pool) th.join();
}

// Cast Int32 -> Float32 (`x as f32`, round to nearest even).  cast.rs:46-48.
void oracle_cast_i32_f32(const int32_t* x, size_t n, float* y) {
  for (size_t i = 0; i < n; ++i) y[i] = (float)x[i];
}

// Mul of a scalar by a scalar or per-column vector: s[n] = a * w[n].
// mul.rs:26-58 (ndarray `&a * &b`, one IEEE rounding per element).
void oracle_mul_scalar_vec(float a, const float* w, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = a * w[i];
}

// Mul of [M, N] by a broadcast scalar (s_len == 1) or per-column [N] vector.
void oracle_mul_rows(const float* x, size_t M, size_t N, const float* s,
                     size_t s_len, float* out) {
  for (size_t m = 0; m < M; ++m)
    for (size_t n = 0; n < N; ++n)
      out[m * N + n] = x[m * N + n] * (s_len == 1 ? s[0] : s[n]);
}

// Add of [M, N] and a broadcast [N] bias.  add.rs:27-85.
void oracle_add_bias(const float* x, size_t M, size_t N, const float* bias,
                     float* out) {
  for (size_t m = 0; m < M; ++m)
    for (size_t n = 0; n < N; ++n) out[m * N + n] = x[m * N + n] + bias[n];
}

// Abramowitz & Stegun 7.1.26 exactly as erf.rs:30-40 writes it: f32 literals,
// each operation rounded separately, `exp` from the platform libm.
static inline float erf_as(float x) {
  float sign = std::isnan(x) ? x : (std::signbit(x) ? -1.0f : 1.0f);
  float a = std::fabs(x);
  float t = 1.0f / (1.0f + 0.3275911f * a);
  float p = 1.0614054f * t;
  p = p - 1.4531521f;
  p = p * t;
  p = p + 1.4214138f;
  p = p * t;
  p = p - 0.28449672f;
  p = p * t;
  p = p + 0.2548296f;
  p = p * t;
  float e = std::exp(-a * a);
  float y = 1.0f - p * e;
  return sign * y;
}

void oracle_erf(const float* x, size_t n, float* y) {
  for (size_t i = 0; i < n; ++i) y[i] = erf_as(x[i]);
}

// The exported erf-GELU subgraph, op by op: Div(x, sqrt2) -> Erf -> Add(1)
// -> Mul(x, .) -> Mul(., 0.5).  Each op is one f32 rounding (erf.rs:30-40
// for Erf; div/add/mul kernels elsewhere are plain IEEE ops).
static const float kSqrt2f = 1.41421353816986083984375f;  // f32(sqrt(2))
void oracle_gelu(const float* x, size_t n, float* y) {
  for (size_t i = 0; i < n; ++i) {
    float v = x[i];
    float d = v / kSqrt2f;
    float e = erf_as(d);
    float a = e + 1.0f;
    float m = v * a;
    y[i] = m * 0.5f;
  }
}

// DequantizeLinear forward.  dequantize_linear.rs:32-179:
// y = (f32(x) - f32(zp)) * scale, per-tensor (scale_len == 1) or per-axis.
// x_dtype: 0 = i8, 1 = u8, 2 = i32.  zp has x's dtype and scale's length (or
// is null).  outer/axis_len/inner describe the broadcast of a per-axis scale.
void oracle_dequantize_linear(const void* x, int x_dtype, size_t outer,
                              size_t axis_len, size_t inner,
                              const float* scale, size_t scale_len,
                              const void* zp, float* y) {
  size_t total = outer * axis_len * inner;
  for (size_t i = 0; i < total; ++i) {
    size_t ax = (i / inner) % axis_len;
    size_t si = scale_len == 1 ? 0 : ax;
    float xv, zv = 0.0f;
    switch (x_dtype) {
      case 0: xv = (float)((const int8_t*)x)[i];
              if (zp) zv = (float)((const int8_t*)zp)[si]; break;
      case 1: xv = (float)((const uint8_t*)x)[i];
              if (zp) zv = (float)((const uint8_t*)zp)[si]; break;
      default: xv = (float)((const int32_t*)x)[i];
              if (zp) zv = (float)((const int32_t*)zp)[si]; break;
    }
    y[i] = (xv - zv) * scale[si];
  }
}

// The fused chain as the reference's CPU GraphExecutor runs it
// (graph_executor.rs:203-216 for DQL, :356-432 for the rest):
//   q, s_x, zp_x = DQL(x)                      [M, K] f32 -> u8
//   acc          = MatMulInteger(q, W, zp_x, b_zp)   W i8 [K, N]
//   c            = Cast(acc)
//   s            = Mul(s_x, w_scale)           scalar or [N]
//   o            = Mul(c, s)
//   o            = Add(o, bias)
//   [o           = GELU subgraph(o)]
// Intermediates are returned when the pointers are non-null.
void oracle_quant_linear(const float* x, size_t M, size_t K, const int8_t* W,
                         size_t N, const float* w_scale, int w_scale_per_col,
                         const int32_t* b_zp, int b_zp_per_col,
                         const float* bias, int gelu, float* out,
                         uint8_t* q_out, float* sx_out, uint8_t* zpx_out,
                         int32_t* acc_out, int threads) {
  std::vector<uint8_t> q(M * K);
  float sx;
  uint8_t zpx;
  oracle_dql(x, M * K, q.data(), &sx, &zpx);
  std::vector<int32_t> acc(M * N);
  oracle_matmul_integer(q.data(), 0, W, 1, M, K, N, (int32_t)zpx, b_zp,
                        b_zp_per_col, acc.data(), threads);
  std::vector<float> s(N);
  size_t s_len = w_scale_per_col ? N : 1;
  oracle_mul_scalar_vec(sx, w_scale, s_len, s.data());
  for (size_t m = 0; m < M; ++m) {
    for (size_t n = 0; n < N; ++n) {
      float c = (float)acc[m * N + n];
      float o = c * s[s_len == 1 ? 0 : n];
      o = o + bias[n];
      if (gelu) {
        float d = o / kSqrt2f;
        float e = erf_as(d);
        float a = e + 1.0f;
        float mm = o * a;
        o = mm * 0.5f;
      }
      out[m * N + n] = o;
    }
  }
  if (q_out) std::memcpy(q_out, q.data(), M * K);
  if (sx_out) *sx_out = sx;
  if (zpx_out) *zpx_out = zpx;
  if (acc_out) std::memcpy(acc_out, acc.data(), M * N * sizeof(int32_t));
}

// ------------------------------------------------------------ fp32 glue
// ndarray's unrolled_fold(xs, 0, +) on n contiguous floats (see header).
static float sum_unrolled8(const float* x, size_t n) {
  float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int u = 0; u < 8; ++u) p[u] = p[u] + x[i + u];
  float acc = 0.0f;
  acc = acc + (p[0] + p[4]);
  acc = acc + (p[1] + p[5]);
  acc = acc + (p[2] + p[6]);
  acc = acc + (p[3] + p[7]);
  for (; i < n; ++i) acc = acc + x[i];
  return acc;
}

float oracle_sum_f32(const float* x, size_t n) { return sum_unrolled8(x, n); }

// LayerNormalization over the last axis.  layer_normalization.rs:25-80:
// mean = mean_axis(x); centered = x - mean; variance = mean_axis(centered^2);
// std = sqrt(variance + epsilon); y = (centered / std) * scale + bias, every
// step its own f32 rounding.
void oracle_layernorm(const float* x, size_t rows, size_t D, const float* scale,
                      const float* bias, float eps, float* y) {
  std::vector<float> c(D), c2(D);
  const float n = (float)D;
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * D;
    const float mean = sum_unrolled8(xr, D) / n;
    for (size_t i = 0; i < D; ++i) c[i] = xr[i] - mean;
    for (size_t i = 0; i < D; ++i) c2[i] = c[i] * c[i];
    const float var = sum_unrolled8(c2.data(), D) / n;
    const float sd = std::sqrt(var + eps);
    for (size_t i = 0; i < D; ++i) {
      const float normalized = c[i] / sd;
      const float scaled = normalized * scale[i];
      y[r * D + i] = scaled + (bias ? bias[i] : 0.0f);
    }
  }
}

// Softmax over the last axis.  softmax.rs:43-56: max (fold from -inf),
// shifted = x - max, e = exp(shifted) (the platform libm, as Rust's f32::exp),
// sum = sum_axis(e), y = e / sum.
void oracle_softmax(const float* x, size_t rows, size_t D, float* y) {
  std::vector<float> e(D);
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * D;
    float mx = -INFINITY;
    for (size_t i = 0; i < D; ++i) mx = std::fmax(mx, xr[i]);
    for (size_t i = 0; i < D; ++i) e[i] = std::exp(xr[i] - mx);
    const float sum = sum_unrolled8(e.data(), D);
    for (size_t i = 0; i < D; ++i) y[r * D + i] = e[i] / sum;
  }
}

// One [M, K] x [K, N] product the way matrixmultiply's FMA sgemm kernel
// accumulates it (see header): per output, k in blocks of 256, a fused
// multiply-add per step, block sums added in order.
}  // extern "C"

template <bool HW_FMA>
static void matmul_blocks(const float* a, const float* b, size_t M, size_t K, size_t N,
                          float* c) {
  constexpr size_t kKC = 256;
  for (size_t i = 0; i < M; ++i)
    for (size_t j = 0; j < N; ++j) {
      float out = 0.0f;
      for (size_t k0 = 0; k0 < K || k0 == 0; k0 += kKC) {
        float acc = 0.0f;
        const size_t k1 = k0 + kKC < K ? k0 + kKC : K;
        for (size_t k = k0; k < k1; ++k)
          acc = HW_FMA ? __builtin_fmaf(a[i * K + k], b[k * N + j], acc)
                       : std::fma(a[i * K + k], b[k * N + j], acc);
        out = k0 == 0 ? acc : out + acc;
        if (K == 0) break;
      }
      c[i * N + j] = out;
    }
}

__attribute__((target("fma"))) static void matmul_blocks_fma(const float* a, const float* b,
                                                             size_t M, size_t K, size_t N,
                                                             float* c) {
  matmul_blocks<true>(a, b, M, K, N, c);
}

extern "C" {

// MatMul, batched over `batch` pairs of contiguous matrices (matmul.rs:
// 118-176: each batch's [M, K] and [K, N] slice through Array2::dot; a
// stride of 0 broadcasts that operand).
void oracle_matmul(const float* a, const float* b, size_t batch, size_t M, size_t K, size_t N,
                   size_t a_stride, size_t b_stride, float* c) {
  static const bool hw = __builtin_cpu_supports("fma");
  for (size_t t = 0; t < batch; ++t) {
    if (hw) matmul_blocks_fma(a + t * a_stride, b + t * b_stride, M, K, N, c + t * M * N);
    else matmul_blocks<false>(a + t * a_stride, b + t * b_stride, M, K, N, c + t * M * N);
  }
}

int oracle_max_threads(void) {
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

}  // extern "C"
