// MatMulInteger on the 5th-generation tensor cores (tcgen05.mma kind::i8),
// with the zero-point correction and the Cast -> Mul -> Add [-> GELU]
// epilogue fused, so the s32 accumulator stays in tensor memory.
//
// Replaces the reference's one-thread-per-output SIMT kernel
// matmul_integer_u8s8_kernel (src/cuda/ops/quantize_kernels.rs:116-194) and
// the Cast/Mul/Add/Erf launches that follow it (the executor's per-op dispatch,
// src/cuda/executor/layout.rs:1034-1097 and src/cuda/executor/elementwise.rs).
//
// Kernel structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x128-byte A tiles and BNx128-byte B tiles
//               (both K-major, 128-byte swizzle) into an S-stage ring.
//   warp 1      owns the tensor-memory allocation; one elected thread issues
//               tcgen05.mma (M=128, N=BN, K=32 per instruction) into one of
//               two BN-column accumulators, so the epilogue of tile i
//               overlaps the main loop of tile i+1.
//   warps 2..5  epilogue: tcgen05.ld 32x32b.x32 (each warp owns the 32 TMEM
//               lanes of its quadrant), zero-point correction in s32,
//               f32 dequantisation, bias, optional GELU, global stores.
// All mbarrier waits are bounded (common.cuh).
//
// Zero-point correction (exact modulo 2^32; the reference's checked i32
// arithmetic panics where this wraps, which no in-range K reaches):
//   sum_k (a - za)(b - zb[n]) = sum_k a*b - za*colsum_b[n] - zb[n]*rowsum_a[m]
//                               + K*za*zb[n]
// The tensor cores compute sum_k a*b on the raw u8/s8 values.
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "capi.cuh"
#include "common.cuh"

namespace icx {

// from dql.cu
int dql_minmax_partials(size_t n);
int launch_dql_minmax(cudaStream_t s, const float* x, size_t n, float2* partials);

constexpr int kBM = 128;      // rows per tile (UMMA M)
constexpr int kBK = 128;      // K bytes per stage (one 128-byte swizzle atom)
constexpr int kUmmaK = 32;    // K per tcgen05.mma kind::i8

// kEpiLn: dequantisation, bias, residual Add and the LayerNormalization of
// the whole row, computed by a cluster of CTAs that together hold the row
// (ln_epilogue below).
enum EpiMode { kEpiS32 = 0, kEpiF32 = 1, kEpiGelu = 2, kEpiLn = 3 };

struct GemmArgs {
  int M, N, K;
  const void* a_zp;     // nullable, 1 element of A's type
  int a_zp_signed;
  const void* b_zp;     // nullable, 1 or N elements of B's type
  int b_zp_signed;
  int b_zp_per_col;
  const int32_t* colsum;  // [N], sum_k b[k, n]
  const int32_t* rowsum;  // [M], sum_k a[m, k]; needed when b_zp != null
  const float* a_scale;   // device scalar
  const float* w_scale;   // 1 or N
  int w_scale_per_col;
  const float* bias;      // nullable, N
  void* out;              // s32 or f32 [M, N]
  const float* residual;  // nullable: f32 [M, N] added after the bias (residual Add)
  float2* minmax;         // nullable: per-CTA (min, max) of the f32 output,
                          // seeded with 0 like DynamicQuantizeLinear's scan
  const float* ln_gamma;  // kEpiLn: LayerNormalization scale [N]
  const float* ln_beta;   // kEpiLn: nullable, bias [N]
  float ln_eps;
};

__device__ __forceinline__ int32_t ld_zp(const void* p, int is_signed,
                                         int idx) {
  return is_signed ? (int32_t)(static_cast<const int8_t*>(p)[idx])
                   : (int32_t)(static_cast<const uint8_t*>(p)[idx]);
}

// Erf-GELU 0.5*x*(1+erf(x/sqrt2)) with the Abramowitz & Stegun 7.1.26 erf
// the reference uses (src/operators/erf.rs:30-40):
//   erf(d) = sign(d) * (1 - Q),  Q = t*P(t)*exp(-d^2),  t = 1/(1 + p|d|)
// so  GELU(x) = x - x*Q/2  (x >= 0)  or  x*Q/2  (x < 0).
// With u = x * sqrt(log2 e)/sqrt2, exp(-d^2) = 2^(-u^2) and p|d| = k2|u|;
// the 1/2 is folded into the polynomial coefficients (exact power-of-two
// scaling of the reference's f32 literals).  Hardware rcp/ex2 and fused
// multiply-adds keep this within ~1e-6 absolute of the reference's op-by-op
// f32 evaluation (the tests bound it by 1e-5).
__device__ __forceinline__ float gelu_erf(float x) {
  const float u = x * 0.8493217825889587f;          // x/sqrt2 * sqrt(log2 e)
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.2727374732494354f, fabsf(u), 1.0f)));
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-(u * u)));
  float p = fmaf(0.5307027f, t, -0.72657605f);      // 0.5 * A&S coefficients
  p = fmaf(p, t, 0.7107069f);
  p = fmaf(p, t, -0.14224836f);
  p = fmaf(p, t, 0.1274148f);
  const float hq = (p * t) * e;                      // Q/2
  const float xq = x * hq;
  return u >= 0.0f ? x - xq : xq;
}

constexpr int kStageOutBytes = 32 * 32 * 4;          // one warp's 32x32 output box

// Warps: 0 TMA producer, 1 MMA issuer, 2 .. 2+EW-1 epilogue (EW / 4 per TMEM
// lane quadrant).
template <int EW>
constexpr int gemm_threads() { return 64 + 32 * EW; }

// DEEP (K >= 1536): the main loop dominates, so keep a deep stage ring and
// read per-column operands from global memory (L1-prefetched).  Otherwise
// one stage fewer pays for staging each chunk's column operands in a per-warp
// shared-memory slice, where the epilogue (the bottleneck at small K) reads
// them with broadcast loads, and for double-buffered output staging.
template <int BN, bool DEEP, int EW, int CG = 1>
struct Cfg {
  static constexpr int kABytes = kBM * kBK;
  // CG == 2 (a CTA pair computing a 256 x BN tile with cta_group::2): each
  // CTA holds its 128 rows of A and BN / 2 rows of B
  static constexpr int kBBytes = (BN / CG) * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // per-warp column operands of one 32-column chunk: colsum, scale, bias, b_zp
  // (all but the 256-wide DEEP single-CTA tile, whose 4-stage ring leaves no
  // room: that one reads the operands from global memory through L1)
  static constexpr bool kStageOps = !(DEEP && BN == 256 && CG == 1);
  static constexpr int kOpWarpBytes = kStageOps ? 4 * 32 * 4 : 0;
  static constexpr int kBarBytes = 1024;
  // Single CTA: DEEP GEMMs keep a deeper ring and one output staging box per
  // warp; 16 epilogue warps take one stage fewer for their staging boxes.
  // CTA pairs: as many stages as fit beside one staging box per warp.
  static constexpr int kPairStages =
      (227 * 1024 - EW * kStageOutBytes - EW * kOpWarpBytes - kBarBytes - 1024) / kStageBytes;
  static constexpr int kStages = CG == 2 ? (kPairStages > 8 ? 8 : kPairStages)
                                 : DEEP ? (BN == 256 ? 4 : BN == 192 ? (EW == 16 ? 3 : 4) : 5)
                                 : BN == 256 ? 3
                                 : BN == 192 ? (EW == 16 ? 3 : 4)
                                             : (EW == 16 ? 4 : 5);
  // two accumulators of BN columns; the allocation is a power of two
  static constexpr int kTmemCols = BN == 192 ? 512 : 2 * BN;
  static constexpr int kOutOffset = kStages * kStageBytes;
  static constexpr int kFixed = kOutOffset + EW * kOpWarpBytes + kBarBytes + 1024 /*align slack*/;
  // two output staging boxes per warp when they fit (a warp fills one while
  // the TMA store of the other drains)
  static constexpr int kOutBufs =
      (DEEP || CG == 2) ? 1 : kFixed + 2 * EW * kStageOutBytes <= 227 * 1024 ? 2 : 1;
  static constexpr int kOpOffset = kOutOffset + kOutBufs * EW * kStageOutBytes;
  static constexpr int kBarOffset = kOpOffset + EW * kOpWarpBytes;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  // barrier area: full/empty/tfull/tempty at +0, TMEM slot at +192,
  // per-warp (min, max) slots at +256, per-warp residual barriers at +512
  static_assert((2 * kStages + 4) * 8 <= 192, "barrier area");
  static_assert(EW * 8 <= 256, "per-warp slots");
  static_assert(EW % 4 == 0, "whole warps per TMEM lane quadrant");
  static_assert(kStages >= 2, "at least two stages");
  static_assert(CG == 1 || CG == 2, "one CTA or a CTA pair");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// Named barrier among the epilogue warps only.
template <int EW>
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * EW) : "memory");
}

// 2-D TMA store shared -> global of one 32x32 box (tracked by bulk groups).
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src,
                                             int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          tmap),
      "r"(smem_addr(src)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until at most N bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Packed fp32 pairs (sm_100 f32x2 instructions).  Used only inside the GELU,
// whose contract is a tolerance: ptxas may contract a packed multiply and a
// following packed add into an FMA even with .rn, so the bit-exact
// dequantisation uses scalar __fmul_rn / __fadd_rn instead.
__device__ __forceinline__ uint64_t pk(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// The GELU of gelu_erf on a pair of values with packed arithmetic.
__device__ __forceinline__ uint64_t gelu_erf2(uint64_t x) {
  const uint64_t u = mul2(x, pk(0.8493217825889587f, 0.8493217825889587f));
  float u0, u1;
  upk(u, u0, u1);
  const uint64_t den = fma2(pk(0.2727374732494354f, 0.2727374732494354f), pk(fabsf(u0), fabsf(u1)),
                            pk(1.0f, 1.0f));
  float d0, d1, t0, t1, e0, e1;
  upk(den, d0, d1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(d1));
  const uint64_t uu = mul2(u, u);
  float q0, q1;
  upk(uu, q0, q1);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(-q0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(-q1));
  const uint64_t t = pk(t0, t1);
  uint64_t p = fma2(pk(0.5307027f, 0.5307027f), t, pk(-0.72657605f, -0.72657605f));
  p = fma2(p, t, pk(0.7107069f, 0.7107069f));
  p = fma2(p, t, pk(-0.14224836f, -0.14224836f));
  p = fma2(p, t, pk(0.1274148f, 0.1274148f));
  const uint64_t hq = mul2(mul2(p, t), pk(e0, e1));
  const uint64_t xq = mul2(x, hq);
  const uint64_t xm = sub2(x, xq);
  float a0, a1, b0, b1;
  upk(xm, a0, a1);
  upk(xq, b0, b1);
  return pk(u0 >= 0.0f ? a0 : b0, u1 >= 0.0f ? a1 : b1);
}

// Dequantise (and bias / GELU) two corrected accumulators at once.
template <int EPI, bool HAS_BIAS>
__device__ __forceinline__ void finish2(int32_t v0, int32_t v1, float s0, float s1, float b0,
                                        float b1, uint32_t& o0, uint32_t& o1) {
  if (EPI == kEpiS32) {
    o0 = (uint32_t)v0;
    o1 = (uint32_t)v1;
    return;
  }
  // The dequantisation must stay two separately rounded scalar operations:
  // ptxas contracts a packed mul.rn.f32x2 + add.rn.f32x2 pair into an FMA,
  // which would break bit-exactness with the reference's Mul then Add.
  float f0 = __fmul_rn(__int2float_rn(v0), s0), f1 = __fmul_rn(__int2float_rn(v1), s1);
  if (HAS_BIAS) {
    f0 = __fadd_rn(f0, b0);
    f1 = __fadd_rn(f1, b1);
  }
  uint64_t f = pk(f0, f1);
  if (EPI == kEpiGelu) f = gelu_erf2(f);  // tolerance-bound: packed FMAs are fine here
  float a, b;
  upk(f, a, b);
  o0 = __float_as_uint(a);
  o1 = __float_as_uint(b);
}

template <int EPI, bool HAS_BIAS>
__device__ __forceinline__ uint32_t finish1(int32_t v, float sc, float bi) {
  if (EPI == kEpiS32) return (uint32_t)v;
  float f = __fmul_rn(__int2float_rn(v), sc);
  if (HAS_BIAS) f = __fadd_rn(f, bi);
  if (EPI == kEpiGelu) f = gelu_erf(f);
  return __float_as_uint(f);
}

// Loads 4 consecutive elements starting at column n (n % 4 == 0) with
// zero fill past N; `vec` says 16-byte vector loads are legal.
__device__ __forceinline__ int4 ld4i(const int32_t* p, int n, int N, bool vec) {
  if (vec && n + 4 <= N) return __ldg(reinterpret_cast<const int4*>(p + n));
  return make_int4(n < N ? p[n] : 0, n + 1 < N ? p[n + 1] : 0, n + 2 < N ? p[n + 2] : 0,
                   n + 3 < N ? p[n + 3] : 0);
}
__device__ __forceinline__ float4 ld4f(const float* p, int n, int N, bool vec) {
  if (vec && n + 4 <= N) return __ldg(reinterpret_cast<const float4*>(p + n));
  return make_float4(n < N ? p[n] : 0.f, n + 1 < N ? p[n + 1] : 0.f, n + 2 < N ? p[n + 2] : 0.f,
                     n + 3 < N ? p[n + 3] : 0.f);
}

// Epilogue of the LayerNorm-fused GEMM (kEpiLn): a cluster of N / BN CTAs
// (2 to 4), CTA rank r of the cluster holding column tile r of the same 128
// rows, so the cluster holds whole rows.  Epilogue warp e (EW = 12: three
// warps per TMEM lane quadrant, 16-column chunks part, part + 3, ...) per
// tile:
//   1. turns its chunks' accumulators into z = (acc * scale + bias) +
//      residual exactly as the QuantLinear epilogue does (the residual of
//      the next chunk in flight meanwhile) and writes z back over the
//      accumulator columns in TMEM; it also sums z - k0 and (z - k0)^2 with
//      k0 the thread's first value;
//   2. row statistics in one exchange: each thread's (sum, M2) of its 64
//      values (M2 about their own mean, from the shifted sums) goes to every
//      CTA of the cluster (st.shared::cluster into slot [rank][part][row]; a
//      cluster-scope fence per lane and one release.cluster arrive per warp
//      on each CTA's barrier); after the wait each thread combines the
//      3 * (N / BN) pairs of its row with Chan's parallel formula, M2 = sum
//      M2_i + sum n_i (mean_i - mean)^2, var = M2 / N, rstd = rsqrt(var +
//      eps);
//   3. y = (z - mean) * rstd * gamma + beta, the (min, max) of y for the
//      DynamicQuantizeLinear that reads it; each 32 x 16 block goes through
//      a swizzled shared-memory tile so that four lanes store one row's 64
//      contiguous bytes; then the accumulator goes back to the MMA warp.
// The exchange buffers and barriers alternate by tile parity: a CTA writes a
// buffer again only after every CTA arrived for the tile in between, which
// each does after reading that buffer.
// Semantics: the reference's LayerNormalization (layer_normalization.rs:
// 25-80) of the Add output, two-pass mean / variance there and the stable
// parallel combination here (fp32 rounding, as the LayerNorm kernel).
template <int BN, bool HAS_BZ, bool HAS_BIAS, int EW>
__device__ __forceinline__ void ln_epilogue(const GemmArgs& args, uint32_t tmem_base, uint64_t* tfull,
                                            uint64_t* tempty, uint64_t* lnbar, float* xbuf,
                                            uint8_t* ops, float2* red, int warp, int lane, int tile0,
                                            int tstep, int ntiles, int num_n) {
  constexpr int kParts = EW / 4;
  constexpr int kCW = 16;                           // chunk width (columns)
  static_assert(BN % (kCW * kParts) == 0, "LayerNorm epilogue: whole chunks per warp");
  constexpr int kPerWarp = BN / kCW / kParts;       // chunks per warp
  constexpr float kNLocal = (float)(kPerWarp * kCW);
  const int e = warp - 2, quad = warp & 3, part = e >> 2;
  const int M = args.M, N = args.N, K = args.K;
  const int ncl = num_n;                            // CTAs in the cluster
  const uint32_t my_rank = cluster_ctarank();
  const int row = quad * 32 + lane;
  const uint32_t za = args.a_zp ? (uint32_t)ld_zp(args.a_zp, args.a_zp_signed, 0) : 0u;
  const float a_scale = *args.a_scale;
  const float sc_scalar = __fmul_rn(a_scale, args.w_scale[0]);
  const bool sc_per_col = args.w_scale_per_col != 0;
  const bool bz_per_col = args.b_zp_per_col != 0;
  const int32_t bz_scalar = HAS_BZ ? ld_zp(args.b_zp, args.b_zp_signed, 0) : 0;
  // The CTA's column tile is the same for every tile it runs (its rank in
  // the cluster): its column operands go to shared memory once.
  int32_t* op_cs = reinterpret_cast<int32_t*>(ops);
  float* op_sc = reinterpret_cast<float*>(op_cs + BN);
  float* op_bi = op_sc + BN;
  int32_t* op_bz = reinterpret_cast<int32_t*>(op_bi + BN);
  float* op_g = reinterpret_cast<float*>(op_bz + BN);
  float* op_b = op_g + BN;
  // exchange buffers: two (tile parity) of [kMaxCl][kParts][kBM] float2;
  // then this warp's 32 x 16 transpose tile
  constexpr int kMaxCl = 4;
  float2* xch = reinterpret_cast<float2*>(xbuf);
  float* tile_t = xbuf + 2 * 2 * kMaxCl * kParts * kBM + e * 32 * kCW;
  {
    const int ti = threadIdx.x - 64, n = (int)my_rank * BN + ti;
    if (ti < BN) {
      const bool nv = n < N;
      op_cs[ti] = nv ? args.colsum[n] : 0;
      op_sc[ti] = !nv ? 0.0f : sc_per_col ? __fmul_rn(a_scale, args.w_scale[n]) : sc_scalar;
      op_bi[ti] = HAS_BIAS && nv ? args.bias[n] : 0.0f;
      op_bz[ti] = HAS_BZ && bz_per_col && nv ? ld_zp(args.b_zp, args.b_zp_signed, n) : bz_scalar;
      op_g[ti] = nv ? args.ln_gamma[n] : 0.0f;
      op_b[ti] = args.ln_beta && nv ? args.ln_beta[n] : 0.0f;
    }
    epi_sync<EW>();
  }
  int acc = 0;
  uint32_t acc_phase = 0;
  int xb = 0;              // exchange buffer / barrier of this tile
  uint32_t xphase = 0;     // parity of barrier xb's next phase
  bool ok = true;
  float run_mn = 0.0f, run_mx = 0.0f;
  const int kXch = kMaxCl * kParts * kBM;            // float2 per exchange buffer
  const int slot = ((int)my_rank * kParts + part) * kBM + row;
  for (int t = tile0; t < ntiles; t += tstep) {
    const int m0 = (t / num_n) * kBM, n0 = (t % num_n) * BN;
    const int m = m0 + row;
    const bool mv = m < M;
    const float* res_row = args.residual + (size_t)(mv ? m : 0) * N + n0;
    auto load_res = [&](int j, float (&rv)[kCW]) {
      const float4* rr = reinterpret_cast<const float4*>(res_row + (part + kParts * j) * kCW);
#pragma unroll
      for (int q = 0; q < kCW / 4; ++q) {
        const float4 r4 = mv ? __ldg(rr + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        rv[4 * q] = r4.x;
        rv[4 * q + 1] = r4.y;
        rv[4 * q + 2] = r4.z;
        rv[4 * q + 3] = r4.w;
      }
    };
    // 1. the first chunk's residual values are in flight during the wait
    float res[kCW];
    load_res(0, res);
    uint32_t kza_rs = 0;
    if (HAS_BZ) kza_rs = (uint32_t)K * za - (mv ? (uint32_t)args.rowsum[m] : 0u);
    if (ok) ok = mbar_wait_warp(&tfull[acc], acc_phase, ICX_DEVICE_TIMEOUT_EPILOGUE);
    tc_fence_after();
    const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
    // sums of z - k0 and of its squares, k0 = this thread's first value (a
    // shift that keeps the local variance well conditioned)
    float k0 = 0.0f, s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      const int cl = (part + kParts * j) * kCW;   // first column of the chunk in the tile
      uint32_t r[kCW];
      if (ok) {
        tmem_ld_32x32b_x16(t_row + (uint32_t)cl, r);
        tmem_ld_wait_regs16(r);
      }
      float res_next[kCW];
      if (j + 1 < kPerWarp) load_res(j + 1, res_next);
#pragma unroll
      for (int q = 0; q < kCW / 4; ++q) {
        const int c4 = cl + 4 * q;
        const int4 cs = *reinterpret_cast<const int4*>(op_cs + c4);
        const float4 sc = *reinterpret_cast<const float4*>(op_sc + c4);
        const float4 bi = *reinterpret_cast<const float4*>(op_bi + c4);
        const int4 bz = *reinterpret_cast<const int4*>(op_bz + c4);
        int32_t v0 = (int32_t)(r[4 * q + 0] - za * (uint32_t)cs.x);
        int32_t v1 = (int32_t)(r[4 * q + 1] - za * (uint32_t)cs.y);
        int32_t v2 = (int32_t)(r[4 * q + 2] - za * (uint32_t)cs.z);
        int32_t v3 = (int32_t)(r[4 * q + 3] - za * (uint32_t)cs.w);
        if (HAS_BZ) {
          v0 = (int32_t)((uint32_t)v0 + kza_rs * (uint32_t)bz.x);
          v1 = (int32_t)((uint32_t)v1 + kza_rs * (uint32_t)bz.y);
          v2 = (int32_t)((uint32_t)v2 + kza_rs * (uint32_t)bz.z);
          v3 = (int32_t)((uint32_t)v3 + kza_rs * (uint32_t)bz.w);
        }
        uint32_t o[4];
        finish2<kEpiF32, HAS_BIAS>(v0, v1, sc.x, sc.y, bi.x, bi.y, o[0], o[1]);
        finish2<kEpiF32, HAS_BIAS>(v2, v3, sc.z, sc.w, bi.z, bi.w, o[2], o[3]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float zv = __fadd_rn(__uint_as_float(o[u]), res[4 * q + u]);
          if (j == 0 && q == 0 && u == 0) k0 = zv;
          const float d = zv - k0;
          s1 += d;
          s2 = fmaf(d, d, s2);
          r[4 * q + u] = __float_as_uint(zv);
        }
      }
      // z back over its accumulator columns, read again to normalise
      if (ok) tmem_st_32x32b_x16(t_row + (uint32_t)cl, r);
      if (j + 1 < kPerWarp)
#pragma unroll
        for (int u = 0; u < kCW; ++u) res[u] = res_next[u];
    }
    tmem_st_wait();
    // 2. the exchange: (sum, M2 about the local mean) of this thread's values
    const float sum = fmaf(kNLocal, k0, s1);
    const float m2 = fmaxf(s2 - s1 * (s1 / kNLocal), 0.0f);
    float2* buf = xch + xb * kXch;
    for (int r2 = 0; r2 < ncl; ++r2) st_cluster_f32x2(cluster_addr(buf + slot, (uint32_t)r2), sum, m2);
    // every lane's stores are ordered cluster-wide before the warp's one
    // arrival per CTA (lane r2 signals CTA r2, releasing at cluster scope)
    fence_acq_rel_cluster();
    __syncwarp();
    if (lane < ncl) mbar_arrive_cluster(cluster_addr(&lnbar[xb], (uint32_t)lane));
    if (ok) ok = mbar_wait_cluster(&lnbar[xb], xphase, ICX_DEVICE_TIMEOUT_EPILOGUE);
    float mean, rstd;
    {
      float tot = 0.0f;
      for (int i = 0; i < ncl * kParts; ++i) tot += buf[i * kBM + row].x;
      mean = tot / (float)N;
      float M2 = 0.0f;
      for (int i = 0; i < ncl * kParts; ++i) {
        const float2 p = buf[i * kBM + row];
        const float d = p.x / kNLocal - mean;
        M2 += fmaf(kNLocal * d, d, p.y);
      }
      rstd = rsqrtf(M2 / (float)N + args.ln_eps);
    }
    if (xb == 1) xphase ^= 1;
    xb ^= 1;
    // 3. normalise; each chunk through the transpose tile to row-contiguous
    // stores (float4 p of row r at r * 16 + 4 * (p ^ ((r >> 1) & 3)): both
    // the row-wise writes and the transposed reads are bank-conflict free)
    float* out = static_cast<float*>(args.out);
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      const int cl = (part + kParts * j) * kCW;
      uint32_t r[kCW];
      if (ok) {
        tmem_ld_32x32b_x16(t_row + (uint32_t)cl, r);
        tmem_ld_wait_regs16(r);
      }
#pragma unroll
      for (int q = 0; q < kCW / 4; ++q) {
        const float4 g = *reinterpret_cast<const float4*>(op_g + cl + 4 * q);
        const float4 b = *reinterpret_cast<const float4*>(op_b + cl + 4 * q);
        float4 o;
        o.x = (__uint_as_float(r[4 * q]) - mean) * rstd * g.x + b.x;
        o.y = (__uint_as_float(r[4 * q + 1]) - mean) * rstd * g.y + b.y;
        o.z = (__uint_as_float(r[4 * q + 2]) - mean) * rstd * g.z + b.z;
        o.w = (__uint_as_float(r[4 * q + 3]) - mean) * rstd * g.w + b.w;
        if (mv) {
          run_mn = fminf(run_mn, fminf(fminf(o.x, o.y), fminf(o.z, o.w)));
          run_mx = fmaxf(run_mx, fmaxf(fmaxf(o.x, o.y), fmaxf(o.z, o.w)));
        }
        *reinterpret_cast<float4*>(tile_t + lane * kCW + 4 * (q ^ ((lane >> 1) & 3))) = o;
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = (lane >> 2) + 8 * i, c = lane & 3;
        const float4 v = *reinterpret_cast<const float4*>(tile_t + rr * kCW + 4 * (c ^ ((rr >> 1) & 3)));
        const int mr = m0 + quad * 32 + rr;
        if (mr < M) *reinterpret_cast<float4*>(out + (size_t)mr * N + n0 + cl + 4 * c) = v;
      }
      __syncwarp();
    }
    // every column of the accumulator this warp owns has been read back
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&tempty[acc]);
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1;
  }
  if (args.minmax != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      run_mn = fminf(run_mn, __shfl_xor_sync(0xffffffffu, run_mn, o));
      run_mx = fmaxf(run_mx, __shfl_xor_sync(0xffffffffu, run_mx, o));
    }
    if (lane == 0) red[e] = make_float2(run_mn, run_mx);
    epi_sync<EW>();
    if (e == 0 && lane == 0) {
      float mn = 0.0f, mx = 0.0f;
      for (int i = 0; i < EW; ++i) {
        mn = fminf(mn, red[i].x);
        mx = fmaxf(mx, red[i].y);
      }
      args.minmax[blockIdx.x] = make_float2(mn, mx);
    }
  }
}

template <int BN, int EPI, bool HAS_BZ, bool HAS_BIAS, bool DEEP, int EW, int CG>
__global__ void __launch_bounds__(gemm_threads<EW>(), 1)
    qgemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmOut,
                         const __grid_constant__ CUtensorMap tmRes,
                         const GemmArgs args, uint32_t idesc, int tma_store, int vec_cols,
                         int tma_res) {
  using C = Cfg<BN, DEEP, EW, CG>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kABytes;
  uint8_t* sOut = smem + C::kOutOffset;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* tfull = bars + 2 * C::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOffset + 192);
  float2* red = reinterpret_cast<float2*>(smem + C::kBarOffset + 256);
  // residual tile barriers, one per epilogue warp
  uint64_t* rbar = reinterpret_cast<uint64_t*>(smem + C::kBarOffset + 512);
  // LayerNorm exchange barriers (kEpiLn), one per round
  uint64_t* lnbar = reinterpret_cast<uint64_t*>(smem + C::kBarOffset + 768);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int num_n = (N + BN - 1) / BN;
  const int num_m = (M + kBM * CG - 1) / (kBM * CG);   // tiles are kBM * CG rows
  const int ntiles = num_m * num_n;
  const int nk = (K + kBK - 1) / kBK;
  // CTA pairs: rank within the pair (0 = leader), the pair's index and count
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int tile0 = CG == 2 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int tstep = CG == 2 ? (int)nclusters_x() : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], CG * EW);   // the leader's counts both CTAs' epilogues
    }
    for (int w = 0; w < EW; ++w) mbar_init(&rbar[w], 1);
    // LayerNorm exchange rounds: every epilogue warp of every CTA of the
    // cluster arrives once per round
    if (EPI == kEpiLn)
      for (int r = 0; r < 2; ++r) mbar_init(&lnbar[r], (uint32_t)(num_n * EW));
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (tma_store) tma_prefetch_desc(&tmOut);
    if (tma_res) tma_prefetch_desc(&tmRes);
  }
  if (warp == 1) {
    if (CG == 2) {
      tmem_alloc_pair(tmem_slot, C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  // a pair's barriers are signalled across the pair (and a LayerNorm
  // cluster's across the cluster): every CTA's set-up must be visible before
  // any starts
  if (CG == 2 || EPI == kEpiLn) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // setup above overlaps the previous kernel; its outputs (A, a_scale,
  // residual, ...) are read only from here on
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = tile0; t < ntiles && ok; t += tstep) {
        // this CTA's rows of A and of B within the tile
        const int m0 = (t / num_n) * kBM * CG + (int)rank * kBM;
        const int n0 = (t % num_n) * BN + (int)rank * (BN / CG);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, ICX_DEVICE_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (CG == 2) {
            // both CTAs' bytes complete on the leader's barrier; the leader
            // arrives once, expecting the pair's bytes
            const uint32_t fb = cluster_addr(&full[stage], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::kStageBytes);
            tma_load_2d_pair(sA + stage * C::kABytes, &tmA, fb, kb * kBK, m0);
            tma_load_2d_pair(sB + stage * C::kBBytes, &tmB, fb, kb * kBK, n0);
          } else {
            mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
            tma_load_2d(sA + stage * C::kABytes, &tmA, &full[stage], kb * kBK, m0);
            tma_load_2d(sB + stage * C::kBBytes, &tmB, &full[stage], kb * kBK, n0);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    // (of a pair, only the leader's: its MMAs cover both CTAs)
    if ((CG == 1 || rank == 0) && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = tile0; t < ntiles && ok; t += tstep) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, ICX_DEVICE_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, ICX_DEVICE_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_k128(smem_addr(sA + stage * C::kABytes));
          const uint64_t db = smem_desc_k128(smem_addr(sB + stage * C::kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // advance the start address by 32 bytes (encoded >> 4) per step
            if (CG == 2)
              mma_i8_pair(d_tmem, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), idesc,
                          (kb | k) != 0);
            else
              mma_i8(d_tmem, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), idesc,
                     (kb | k) != 0);
          }
          if (CG == 2) {
            // the stage is free in both CTAs once these MMAs have read it
            mma_commit_pair(cluster_addr(&empty[stage], 0));
            mma_commit_pair(cluster_addr(&empty[stage], 1));
          } else {
            mma_commit(&empty[stage]);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (CG == 2) {
          mma_commit_pair(cluster_addr(&tfull[acc], 0));
          mma_commit_pair(cluster_addr(&tfull[acc], 1));
        } else {
          mma_commit(&tfull[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if constexpr (EPI == kEpiLn) {
    static_assert(CG == 1, "LayerNorm epilogue: single-CTA tiles");
    // the exchange buffers and the transpose tiles take the (unused) output
    // staging area, the column operands the operand slices
    static_assert(2 * 4 * (EW / 4) * kBM * 8 + EW * 32 * 16 * 4 <= C::kOutBufs * EW * kStageOutBytes,
                  "exchange buffers");
    static_assert(C::kStageOps && 6 * BN * 4 <= EW * C::kOpWarpBytes, "column operands");
    ln_epilogue<BN, HAS_BZ, HAS_BIAS, EW>(args, tmem_base, tfull, tempty, lnbar,
                                          reinterpret_cast<float*>(sOut), smem + C::kOpOffset, red,
                                          warp, lane, tile0, tstep, ntiles, num_n);
  } else {
    // ----------------------------------------------------------- epilogue
    // Warp e owns TMEM lane quadrant (warp & 3) and the 32-column chunks
    // part, part + kParts, ... of every tile.  Per chunk: the column
    // operands are staged in this warp's own shared slice (no barrier with
    // other warps), the next chunk's tcgen05.ld is issued before this
    // chunk's math so the TMEM read overlaps it, and the accumulator is
    // handed back to the MMA warp as soon as its last chunk is in registers.
    const int e = warp - 2;                       // 0..EW-1
    const int quad = warp & 3;                    // TMEM lanes [32*quad, 32*quad+32)
    const int part = e >> 2;
    constexpr int kParts = EW / 4;
    constexpr int kChunks = BN / 32;
    // two chunk register buffers when the register budget allows it
    constexpr bool kDoubleBuffer = EW <= 8;
    const uint32_t za = args.a_zp ? (uint32_t)ld_zp(args.a_zp, args.a_zp_signed, 0) : 0u;
    float a_scale = 0.0f, sc_scalar = 0.0f;
    if (EPI != kEpiS32) {
      a_scale = *args.a_scale;
      sc_scalar = __fmul_rn(a_scale, args.w_scale[0]);
    }
    const bool sc_per_col = args.w_scale_per_col != 0;
    const bool bz_per_col = args.b_zp_per_col != 0;
    const int32_t bz_scalar = HAS_BZ ? ld_zp(args.b_zp, args.b_zp_signed, 0) : 0;
    const bool vec = (vec_cols & 1) != 0;
    const bool bz_vec = (vec_cols & 2) != 0;  // per-column b_zp readable as 4-byte words
    // this warp's operand slice: colsum, scale, bias, b_zp of one chunk
    int32_t* op_cs = reinterpret_cast<int32_t*>(smem + C::kOpOffset + e * C::kOpWarpBytes);
    float* op_sc = reinterpret_cast<float*>(op_cs + 32);
    float* op_bi = op_sc + 32;
    int32_t* op_bz = reinterpret_cast<int32_t*>(op_bi + 32);
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;  // false once a bounded wait gave up: skip work
    const bool track = (EPI != kEpiS32) && args.minmax != nullptr;
    float run_mn = 0.0f, run_mx = 0.0f;  // the DynamicQuantizeLinear seed
    uint32_t rphase = 0;                 // parity of this warp's residual barrier
    int obuf = 0;                        // output staging box in use

    // column operands of column n for this lane (zero past N)
    int32_t p_cs = 0, p_bz = 0;
    float p_sc = 0.0f, p_bi = 0.0f;
    auto fetch_ops = [&](int nb) {
      if (!C::kStageOps) return;
      const int n = nb + lane;
      p_cs = 0;
      p_sc = sc_scalar;
      p_bi = 0.0f;
      p_bz = bz_scalar;
      if (n < N) {
        p_cs = __ldg(args.colsum + n);
        if (EPI != kEpiS32 && sc_per_col) p_sc = __ldg(args.w_scale + n);
        if (EPI != kEpiS32 && HAS_BIAS) p_bi = __ldg(args.bias + n);
        if (HAS_BZ && bz_per_col) p_bz = ld_zp(args.b_zp, args.b_zp_signed, n);
      }
    };
    auto stage_ops = [&]() {
      if (!C::kStageOps) return;
      __syncwarp();  // every lane is done with the previous chunk's slice
      op_cs[lane] = p_cs;
      op_sc[lane] = (EPI != kEpiS32 && sc_per_col) ? __fmul_rn(a_scale, p_sc) : p_sc;
      op_bi[lane] = p_bi;
      op_bz[lane] = p_bz;
      __syncwarp();
    };

    for (int t = tile0; t < ntiles; t += tstep) {
      const int m0 = (t / num_n) * kBM * CG + (int)rank * kBM;   // this CTA's 128 rows
      const int n0 = (t % num_n) * BN;
      const int mrow0 = m0 + quad * 32;
      const int m = mrow0 + lane;
      uint32_t kza_rs = 0;
      if (HAS_BZ) kza_rs = (uint32_t)K * za - ((m < M) ? (uint32_t)args.rowsum[m] : 0u);
      // chunks of this tile that hold columns < N
      const int nvalid = min(kChunks, (N - n0 + 31) / 32);
      if (!C::kStageOps) {
        // per-column operands come from global memory: pull them into L1
        const int et = threadIdx.x - 64;
        if (et < BN * 4 / 128) {
          const int n = n0 + et * 32;
          if (n < N) {
            asm volatile("prefetch.global.L1 [%0];" ::"l"(args.colsum + n));
            if (EPI != kEpiS32 && HAS_BIAS) asm volatile("prefetch.global.L1 [%0];" ::"l"(args.bias + n));
            if (EPI != kEpiS32 && sc_per_col) asm volatile("prefetch.global.L1 [%0];" ::"l"(args.w_scale + n));
          }
        }
      }
      int c = part;
      if (c < nvalid) fetch_ops(n0 + c * 32);   // loads in flight during the wait
      if (ok) ok = mbar_wait_warp(&tfull[acc], acc_phase, ICX_DEVICE_TIMEOUT_EPILOGUE);
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      bool released = false;
      auto release = [&]() {
        // the accumulator's columns this warp reads are all in registers
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (CG == 2) mbar_arrive_cluster(cluster_addr(&tempty[acc], 0));   // the leader's
          else mbar_arrive(&tempty[acc]);
        }
        released = true;
      };

      // One chunk: zero-point correction, dequantisation [+ GELU]
      // [+ residual], (min, max), store.  r holds the chunk's accumulators.
      auto process = [&](uint32_t (&r)[32], int cc) {
        const int nb = n0 + cc * 32;
        uint8_t* stage_out = sOut + (obuf * EW + e) * kStageOutBytes;
        const bool res_tma = EPI == kEpiF32 && tma_res && mrow0 < M;
        const bool fast = C::kStageOps || (vec && (nb + 32 <= N) && (!(HAS_BZ && bz_per_col) || bz_vec));
        if (fast) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            int4 cs;
            float4 sc = make_float4(sc_scalar, sc_scalar, sc_scalar, sc_scalar);
            float4 bi = make_float4(0.f, 0.f, 0.f, 0.f);
            int4 bz = make_int4(bz_scalar, bz_scalar, bz_scalar, bz_scalar);
            if (!C::kStageOps) {
              cs = __ldg(reinterpret_cast<const int4*>(args.colsum + nb) + q);
              if (EPI != kEpiS32 && sc_per_col) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(args.w_scale + nb) + q);
                sc = make_float4(__fmul_rn(a_scale, w.x), __fmul_rn(a_scale, w.y),
                                 __fmul_rn(a_scale, w.z), __fmul_rn(a_scale, w.w));
              }
              if (EPI != kEpiS32 && HAS_BIAS) bi = __ldg(reinterpret_cast<const float4*>(args.bias + nb) + q);
              if (HAS_BZ && bz_per_col) {
                // four 8-bit zero points in one 32-bit load
                const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(
                                             static_cast<const uint8_t*>(args.b_zp) + nb) + q);
                if (args.b_zp_signed)
                  bz = make_int4((int8_t)(w & 0xff), (int8_t)((w >> 8) & 0xff), (int8_t)((w >> 16) & 0xff),
                                 (int8_t)(w >> 24));
                else
                  bz = make_int4((int)(w & 0xff), (int)((w >> 8) & 0xff), (int)((w >> 16) & 0xff),
                                 (int)(w >> 24));
              }
            } else {
              cs = reinterpret_cast<const int4*>(op_cs)[q];
              if (EPI != kEpiS32 && sc_per_col) sc = reinterpret_cast<const float4*>(op_sc)[q];
              if (EPI != kEpiS32 && HAS_BIAS) bi = reinterpret_cast<const float4*>(op_bi)[q];
              if (HAS_BZ && bz_per_col) bz = reinterpret_cast<const int4*>(op_bz)[q];
            }
            int32_t v0 = (int32_t)(r[4 * q + 0] - za * (uint32_t)cs.x);
            int32_t v1 = (int32_t)(r[4 * q + 1] - za * (uint32_t)cs.y);
            int32_t v2 = (int32_t)(r[4 * q + 2] - za * (uint32_t)cs.z);
            int32_t v3 = (int32_t)(r[4 * q + 3] - za * (uint32_t)cs.w);
            if (HAS_BZ) {
              v0 = (int32_t)((uint32_t)v0 + kza_rs * (uint32_t)bz.x);
              v1 = (int32_t)((uint32_t)v1 + kza_rs * (uint32_t)bz.y);
              v2 = (int32_t)((uint32_t)v2 + kza_rs * (uint32_t)bz.z);
              v3 = (int32_t)((uint32_t)v3 + kza_rs * (uint32_t)bz.w);
            }
            finish2<EPI, HAS_BIAS>(v0, v1, sc.x, sc.y, bi.x, bi.y, r[4 * q + 0], r[4 * q + 1]);
            finish2<EPI, HAS_BIAS>(v2, v3, sc.z, sc.w, bi.z, bi.w, r[4 * q + 2], r[4 * q + 3]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int n = nb + 4 * q;
            const int4 cs = ld4i(args.colsum, n, N, false);
            int4 bz = make_int4(bz_scalar, bz_scalar, bz_scalar, bz_scalar);
            if (HAS_BZ && bz_per_col) {
              bz.x = n < N ? ld_zp(args.b_zp, args.b_zp_signed, n) : 0;
              bz.y = n + 1 < N ? ld_zp(args.b_zp, args.b_zp_signed, n + 1) : 0;
              bz.z = n + 2 < N ? ld_zp(args.b_zp, args.b_zp_signed, n + 2) : 0;
              bz.w = n + 3 < N ? ld_zp(args.b_zp, args.b_zp_signed, n + 3) : 0;
            }
            float4 sc = make_float4(sc_scalar, sc_scalar, sc_scalar, sc_scalar);
            if (EPI != kEpiS32 && sc_per_col) {
              const float4 w = ld4f(args.w_scale, n, N, false);
              sc = make_float4(__fmul_rn(a_scale, w.x), __fmul_rn(a_scale, w.y),
                               __fmul_rn(a_scale, w.z), __fmul_rn(a_scale, w.w));
            }
            float4 bi = make_float4(0.f, 0.f, 0.f, 0.f);
            if (EPI != kEpiS32 && HAS_BIAS) bi = ld4f(args.bias, n, N, false);
            int32_t v0 = (int32_t)(r[4 * q + 0] - za * (uint32_t)cs.x);
            int32_t v1 = (int32_t)(r[4 * q + 1] - za * (uint32_t)cs.y);
            int32_t v2 = (int32_t)(r[4 * q + 2] - za * (uint32_t)cs.z);
            int32_t v3 = (int32_t)(r[4 * q + 3] - za * (uint32_t)cs.w);
            if (HAS_BZ) {
              v0 = (int32_t)((uint32_t)v0 + kza_rs * (uint32_t)bz.x);
              v1 = (int32_t)((uint32_t)v1 + kza_rs * (uint32_t)bz.y);
              v2 = (int32_t)((uint32_t)v2 + kza_rs * (uint32_t)bz.z);
              v3 = (int32_t)((uint32_t)v3 + kza_rs * (uint32_t)bz.w);
            }
            finish2<EPI, HAS_BIAS>(v0, v1, sc.x, sc.y, bi.x, bi.y, r[4 * q + 0], r[4 * q + 1]);
            finish2<EPI, HAS_BIAS>(v2, v3, sc.z, sc.w, bi.z, bi.w, r[4 * q + 2], r[4 * q + 3]);
          }
        }
        if (res_tma) {
          // residual Add(out, r) from the swizzled staging copy of the box
          // (its TMA load was issued before this chunk's accumulator wait)
          if (!mbar_wait_warp(&rbar[e], rphase, ICX_DEVICE_TIMEOUT_EPILOGUE)) ok = false;
          rphase ^= 1;
          const uint8_t* rrow = stage_out + lane * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 rv = *reinterpret_cast<const float4*>(rrow + ((q ^ (lane & 7)) << 4));
            r[4 * q + 0] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 0]), rv.x));
            r[4 * q + 1] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 1]), rv.y));
            r[4 * q + 2] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 2]), rv.z));
            r[4 * q + 3] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 3]), rv.w));
          }
          __syncwarp();  // every lane has read its row before it is overwritten
        } else if (EPI == kEpiF32 && args.residual != nullptr && m < M) {
          // residual Add(out, r): one more separately rounded f32 addition
          const float* rr = args.residual + (size_t)m * N + nb;
          if (vec && nb + 32 <= N && ((reinterpret_cast<uintptr_t>(args.residual) & 15) == 0)) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 rv = __ldg(reinterpret_cast<const float4*>(rr) + q);
              r[4 * q + 0] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 0]), rv.x));
              r[4 * q + 1] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 1]), rv.y));
              r[4 * q + 2] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 2]), rv.z));
              r[4 * q + 3] = __float_as_uint(__fadd_rn(__uint_as_float(r[4 * q + 3]), rv.w));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < N) r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), rr[j]));
          }
        }
        if (track && m < M) {
          if (nb + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              run_mn = fminf(run_mn, __uint_as_float(r[j]));
              run_mx = fmaxf(run_mx, __uint_as_float(r[j]));
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (nb + j < N) {
                run_mn = fminf(run_mn, __uint_as_float(r[j]));
                run_mx = fmaxf(run_mx, __uint_as_float(r[j]));
              }
          }
        }
        if (tma_store) {
          if (mrow0 < M) {
            // this box's previous store (kOutBufs chunks ago) must have been
            // read out of shared memory (the residual path waited already)
            if (lane == 0 && !res_tma) bulk_wait_read<(C::kOutBufs > 1 ? 1 : 0)>();
            __syncwarp();
            uint8_t* row = stage_out + lane * 128;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<uint4*>(row + ((q ^ (lane & 7)) << 4)) =
                  make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmOut, stage_out, nb, mrow0);
              bulk_commit();
            }
            if (C::kOutBufs == 2) obuf ^= 1;
          }
        } else if (m < M) {
          uint32_t* orow = static_cast<uint32_t*>(args.out) + (size_t)m * N + nb;
          if (vec && nb + 32 <= N && (reinterpret_cast<uintptr_t>(args.out) & 15) == 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              reinterpret_cast<uint4*>(orow)[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < N) orow[j] = r[j];
          }
        }
      };
      // residual box of chunk cc -> the staging box it will be stored from
      auto residual_load = [&](int cc) {
        if (EPI == kEpiF32 && tma_res && mrow0 < M && lane == 0) {
          bulk_wait_read<(C::kOutBufs > 1 ? 1 : 0)>();
          uint8_t* stage_out = sOut + (obuf * EW + e) * kStageOutBytes;
          mbar_arrive_expect_tx(&rbar[e], kStageOutBytes);
          tma_load_2d(stage_out, &tmRes, &rbar[e], n0 + cc * 32, mrow0);
        }
      };

      if (kDoubleBuffer) {
        uint32_t ra[32], rb[32];
        if (ok && c < nvalid) {
          tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), ra);
          // chunk pairs (ra, rb): the load of the next chunk is in flight
          // while the current one is processed
          while (true) {
            stage_ops();
            residual_load(c);
            tmem_ld_wait_regs(ra);
            int cn = c + kParts;
            bool more = ok && cn < nvalid;
            if (more) {
              tmem_ld_32x32b_x32(t_row + (uint32_t)(cn * 32), rb);
              fetch_ops(n0 + cn * 32);
            } else {
              release();
            }
            process(ra, c);
            if (!more) break;
            c = cn;
            stage_ops();
            residual_load(c);
            tmem_ld_wait_regs(rb);
            cn = c + kParts;
            more = ok && cn < nvalid;
            if (more) {
              tmem_ld_32x32b_x32(t_row + (uint32_t)(cn * 32), ra);
              fetch_ops(n0 + cn * 32);
            } else {
              release();
            }
            process(rb, c);
            if (!more) break;
            c = cn;
          }
        }
      } else {
        // one register buffer (16 epilogue warps: the other warps hide the
        // TMEM load latency)
        uint32_t ra[32];
        for (; ok && c < nvalid; c += kParts) {
          stage_ops();
          residual_load(c);
          tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), ra);
          tmem_ld_wait_regs(ra);
          const bool more = c + kParts < nvalid;
          if (more) fetch_ops(n0 + (c + kParts) * 32);
          else release();
          process(ra, c);
        }
      }
      if (!released) release();
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (tma_store && lane == 0) bulk_wait0();
    if (track) {
      // CTA-wide (min, max) of everything this CTA wrote: one partial per CTA
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        run_mn = fminf(run_mn, __shfl_xor_sync(0xffffffffu, run_mn, o));
        run_mx = fmaxf(run_mx, __shfl_xor_sync(0xffffffffu, run_mx, o));
      }
      if (lane == 0) red[e] = make_float2(run_mn, run_mx);
      epi_sync<EW>();
      if (e == 0 && lane == 0) {
        float mn = 0.0f, mx = 0.0f;
        for (int i = 0; i < EW; ++i) {
          mn = fminf(mn, red[i].x);
          mx = fmaxf(mx, red[i].y);
        }
        args.minmax[blockIdx.x] = make_float2(mn, mx);
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  // neither CTA of a pair leaves while the other may still signal its
  // barriers or the leader's MMAs may still read its shared memory (nor a
  // CTA of a LayerNorm cluster while the others may still write into its
  // exchange buffers)
  if (CG == 2 || EPI == kEpiLn) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (CG == 2) tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// SIMT kernel for shapes the TMA path cannot address (K not a multiple of 16
// or misaligned operands).  One thread per output; same arithmetic.
template <int EPI>
__global__ void qgemm_simt_kernel(const void* __restrict__ a, int a_signed,
                                  const void* __restrict__ bt, int b_signed,
                                  const GemmArgs args) {
  pdl_wait();
  pdl_trigger();
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int M = args.M, N = args.N, K = args.K;
  if (idx >= (size_t)M * N) return;
  const int m = (int)(idx / N), n = (int)(idx % N);
  uint32_t acc = 0;
  for (int k = 0; k < K; ++k) {
    const int32_t av = a_signed ? (int32_t)static_cast<const int8_t*>(a)[(size_t)m * K + k]
                                : (int32_t)static_cast<const uint8_t*>(a)[(size_t)m * K + k];
    const int32_t bv = b_signed ? (int32_t)static_cast<const int8_t*>(bt)[(size_t)n * K + k]
                                : (int32_t)static_cast<const uint8_t*>(bt)[(size_t)n * K + k];
    acc += (uint32_t)(av * bv);
  }
  const int32_t za = args.a_zp ? ld_zp(args.a_zp, args.a_zp_signed, 0) : 0;
  const int32_t bz = args.b_zp ? ld_zp(args.b_zp, args.b_zp_signed, args.b_zp_per_col ? n : 0) : 0;
  const int32_t rs = args.b_zp ? args.rowsum[m] : 0;
  const int32_t v = (int32_t)(acc + (uint32_t)K * (uint32_t)za * (uint32_t)bz -
                              (uint32_t)za * (uint32_t)args.colsum[n] -
                              (uint32_t)bz * (uint32_t)rs);
  if (EPI == kEpiS32) {
    static_cast<int32_t*>(args.out)[idx] = v;
  } else {
    const float sc = __fmul_rn(*args.a_scale, args.w_scale[args.w_scale_per_col ? n : 0]);
    float f = __fmul_rn(__int2float_rn(v), sc);
    if (args.bias) f = __fadd_rn(f, args.bias[n]);
    if (EPI == kEpiGelu) f = gelu_erf(f);
    if (EPI == kEpiF32 && args.residual) f = __fadd_rn(f, args.residual[idx]);
    static_cast<float*>(args.out)[idx] = f;
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                  void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// K-major byte matrix [rows, K] -> tensor map with a box of box_rows x 128
// bytes and the 128-byte swizzle.  Out-of-range rows/columns read as zero.
static int make_tmap(CUtensorMap* map, const void* base, size_t rows, size_t K,
                     int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return ICX_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) rows=%zu K=%zu", (int)r, rows, K);
    return ICX_ERR_CUDA;
  }
  return ICX_OK;
}

static int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Row-major 32-bit matrix [M, N] -> tensor map with 32x32 boxes and the
// 128-byte swizzle (the epilogue's shared-memory staging layout).
static int make_out_tmap(CUtensorMap* map, void* base, size_t M, size_t N, bool is_float) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return ICX_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)N * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, is_float ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_INT32,
                  2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (output) failed (%d) M=%zu N=%zu", (int)r, M, N);
    return ICX_ERR_CUDA;
  }
  return ICX_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int BN, int EPI, bool DEEP, int EW, int CG>
static int launch_tc(cudaStream_t s, const void* a, bool a_signed, const void* bt,
                     bool b_signed, const GemmArgs& args, int grid) {
  using C = Cfg<BN, DEEP, EW, CG>;
  CUtensorMap ta, tb, tout;
  int rc = make_tmap(&ta, a, (size_t)args.M, (size_t)args.K, kBM);
  if (rc) return rc;
  rc = make_tmap(&tb, bt, (size_t)args.N, (size_t)args.K, BN / CG);
  if (rc) return rc;
  // TMA stores need a 16-byte aligned base and a row pitch multiple of 16 B
  const int tma_store = EPI != kEpiLn && C::kOutBufs > 0 && (args.N % 4 == 0) && aligned16(args.out);
  if (tma_store) {
    rc = make_out_tmap(&tout, args.out, (size_t)args.M, (size_t)args.N, EPI != kEpiS32);
    if (rc) return rc;
  } else {
    memset(&tout, 0, sizeof(tout));
  }
  CUtensorMap tres;
  memset(&tres, 0, sizeof(tres));
  const int tma_res = tma_store && EPI == kEpiF32 && args.residual != nullptr && aligned16(args.residual);
  if (tma_res) {
    rc = make_out_tmap(&tres, const_cast<float*>(args.residual), (size_t)args.M, (size_t)args.N, true);
    if (rc) return rc;
  }
  // bit 0: 16-byte vector loads of the column operands; bit 1: per-column
  // zero points readable as aligned 4-byte words
  const int vec_cols = ((args.N % 4 == 0) && aligned16(args.colsum) &&
                        (args.w_scale == nullptr || !args.w_scale_per_col || aligned16(args.w_scale)) &&
                        (args.bias == nullptr || aligned16(args.bias)))
                           ? 1 | ((args.b_zp && args.b_zp_per_col &&
                                   (reinterpret_cast<uintptr_t>(args.b_zp) & 3) == 0) ? 2 : 0)
                           : 0;
  auto kern = args.b_zp ? (args.bias ? qgemm_tcgen05_kernel<BN, EPI, true, true, DEEP, EW, CG>
                                      : qgemm_tcgen05_kernel<BN, EPI, true, false, DEEP, EW, CG>)
                        : (args.bias ? qgemm_tcgen05_kernel<BN, EPI, false, true, DEEP, EW, CG>
                                     : qgemm_tcgen05_kernel<BN, EPI, false, false, DEEP, EW, CG>);
  ICX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                C::kSmemBytes));
  const uint32_t idesc = idesc_i8(kBM * CG, BN, a_signed, b_signed);
  if (CG == 2)
    launch_pdl_cluster(kern, dim3(grid), dim3(gemm_threads<EW>()), C::kSmemBytes, s, 2u, ta, tb,
                       tout, tres, args, idesc, tma_store, vec_cols, tma_res);
  else if (EPI == kEpiLn)
    launch_pdl_cluster(kern, dim3(grid), dim3(gemm_threads<EW>()), C::kSmemBytes, s,
                       (unsigned)(args.N / BN), ta, tb, tout, tres, args, idesc, tma_store, vec_cols,
                       tma_res);
  else
    launch_pdl(kern, dim3(grid), dim3(gemm_threads<EW>()), C::kSmemBytes, s, ta, tb, tout, tres,
               args, idesc, tma_store, vec_cols, tma_res);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

// CTA pairs of the cta_group::2 kernels that can be resident at once (every
// pair kernel runs one CTA per SM, so one query covers them all; cached per
// device).
static int max_pair_clusters() {
  static int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  if (cached[dev]) return cached[dev];
  using C = Cfg<256, true, 8, 2>;
  auto kern = qgemm_tcgen05_kernel<256, kEpiF32, false, true, true, 8, 2>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(gemm_threads<8>());
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 0;
  }
  cached[dev] = n;
  return n;
}

// Epilogue warps of the shallow (K < 1536) f32 GEMMs: 16 (the epilogue is
// their bottleneck and more warps in flight hide its TMEM and store
// latencies; measured faster than 8 for the GELU and the QKV GEMMs, equal for
// the residual ones); ICX_GEMM_EPI_WARPS=8 forces 8 (read once per process,
// for measurement).
static int epilogue_warps() {
  static int forced = [] {
    const char* v = getenv("ICX_GEMM_EPI_WARPS");
    const int n = v ? atoi(v) : 0;
    return n == 8 || n == 16 ? n : 0;
  }();
  return forced ? forced : 16;
}

// CTA pairs (cta_group::2, 256-row tiles) for large deep GEMMs: half the B
// bytes per CTA and per MAC, which is what bounds the single-CTA kernel there.
// ICX_GEMM_PAIR=0|1 forces them off / on (read once, for measurement).
static int pair_mode() {
  static int mode = [] {
    const char* v = getenv("ICX_GEMM_PAIR");
    return v ? (atoi(v) ? 1 : 0) : -1;
  }();
  return mode;
}

// Which kernel runs a GEMM and with how many CTAs.
struct GemmPlan {
  int bn;     // 128 / 192 / 256 for the tensor-core kernel, 0 for the SIMT kernel
  int grid;   // CTAs (tensor-core path)
  int cg;     // 1 (one CTA per tile) or 2 (CTA pairs, 256-row tiles)
};

static GemmPlan plan_gemm(const GemmArgs& args, const void* a, const void* bt) {
  GemmPlan p{0, 0, 1};
  const bool tma_ok = (args.K % 16 == 0) && args.K > 0 &&
                      ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(bt)) & 15) == 0;
  if (!tma_ok) return p;
  const long sms = sm_count();
  const int pm = pair_mode();
  // (measured: pairs help where the K loop dominates; the shallow GEMMs are
  // bound by their epilogue and run faster on single CTAs)
  const bool pair = pm == 1 || (pm < 0 && args.M >= 8192 && args.K >= 1536);
  const long pairs = pair ? max_pair_clusters() : 0;
  p.cg = pair && pairs > 0 && args.N > 128 ? 2 : 1;
  // Tile width: the persistent kernel's time is set by its busiest CTA (or
  // pair), ceil(tiles / units) tiles, each costing about BN + 64 (its columns
  // plus the per-tile A fetch and epilogue overhead, in the same units); take
  // the BN that minimises that (ties: the wider tile).  E.g. N = 768 at
  // M = 4096 runs 128 tiles of 192 columns (one per CTA) instead of 192
  // tiles of 128.
  const long units = p.cg == 2 ? pairs : sms;
  const long mt = (args.M + kBM * p.cg - 1) / (kBM * p.cg);
  long best = -1;
  for (int bn : {256, 192, 128}) {
    if (p.cg == 2 && bn == 128) continue;   // pairs run 192- or 256-wide tiles
    const long tiles = mt * ((args.N + bn - 1) / bn);
    const long cost = ((tiles + units - 1) / units) * (bn + 64);
    if (best < 0 || cost < best) {
      best = cost;
      p.bn = bn;
    }
  }
  if (args.N <= 128) p.bn = 128;   // (single CTA: pairs need N > 128)
  const long tiles = mt * ((args.N + p.bn - 1) / p.bn);
  p.grid = (int)(tiles < units ? tiles : units) * p.cg;
  return p;
}

// Number of (min, max) partials a fused GEMM writes for its output.
static int gemm_grid(const GemmArgs& args, const void* a, const void* bt) {
  const GemmPlan p = plan_gemm(args, a, bt);
  if (p.bn) return p.grid;
  return dql_minmax_partials((size_t)args.M * args.N);
}

// One tile width: single CTAs or CTA pairs (pairs only for 192 / 256
// columns), a deep ring for K >= 1536, 8 or 16 epilogue warps.
template <int BN, int EPI>
static int launch_bn(cudaStream_t s, const void* a, bool a_signed, const void* bt, bool b_signed,
                     const GemmArgs& args, const GemmPlan& p, bool deep, bool ew16) {
  constexpr int kEw16 = EPI == kEpiS32 ? 8 : 16;
  if (p.cg == 2 && BN != 128)
    return deep   ? launch_tc<BN, EPI, true, 8, (BN == 128 ? 1 : 2)>(s, a, a_signed, bt, b_signed, args, p.grid)
           : ew16 ? launch_tc<BN, EPI, false, kEw16, (BN == 128 ? 1 : 2)>(s, a, a_signed, bt, b_signed, args, p.grid)
                  : launch_tc<BN, EPI, false, 8, (BN == 128 ? 1 : 2)>(s, a, a_signed, bt, b_signed, args, p.grid);
  return deep   ? launch_tc<BN, EPI, true, 8, 1>(s, a, a_signed, bt, b_signed, args, p.grid)
         : ew16 ? launch_tc<BN, EPI, false, kEw16, 1>(s, a, a_signed, bt, b_signed, args, p.grid)
                : launch_tc<BN, EPI, false, 8, 1>(s, a, a_signed, bt, b_signed, args, p.grid);
}

template <int EPI>
static int launch_gemm(cudaStream_t s, const void* a, bool a_signed,
                       const void* bt, bool b_signed, const GemmArgs& args) {
  if (args.M == 0 || args.N == 0) return ICX_OK;
  const GemmPlan p = plan_gemm(args, a, bt);
  const bool deep = args.K >= 1536;
  const bool ew16 = !deep && EPI != kEpiS32 && epilogue_warps() == 16;
  if (p.bn == 256) return launch_bn<256, EPI>(s, a, a_signed, bt, b_signed, args, p, deep, ew16);
  if (p.bn == 192) return launch_bn<192, EPI>(s, a, a_signed, bt, b_signed, args, p, deep, ew16);
  if (p.bn == 128) return launch_bn<128, EPI>(s, a, a_signed, bt, b_signed, args, p, deep, ew16);
  const size_t total = (size_t)args.M * args.N;
  const int threads = 256;
  const size_t blocks = (total + threads - 1) / threads;
  GemmArgs g = args;
  g.minmax = nullptr;
  launch_pdl(qgemm_simt_kernel<EPI>, dim3((unsigned)blocks), dim3(threads), 0, s, a, a_signed, bt, b_signed, g);
  ICX_LAUNCH_CHECK();
  if (EPI != kEpiS32 && args.minmax)
    return launch_dql_minmax(s, static_cast<const float*>(args.out), total, args.minmax);
  return ICX_OK;
}

// ------------------------------------------------------- weight preparation
// bt[n, k] = b[k, n] through a 32x32 shared tile; colsum via atomics of
// per-tile partial column sums.
__global__ void prepare_b_kernel(const uint8_t* __restrict__ b, int b_signed,
                                 int K, int N, uint8_t* __restrict__ bt,
                                 int32_t* __restrict__ colsum) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint8_t tile[32][33];
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int k = k0 + i, n = n0 + tx;
    tile[i][tx] = (k < K && n < N) ? b[(size_t)k * N + n] : 0;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int n = n0 + i, k = k0 + tx;
    if (n < N && k < K) bt[(size_t)n * K + k] = tile[tx][i];
  }
  if (ty == 0 && n0 + tx < N) {
    int32_t s = 0;
    for (int i = 0; i < 32; ++i)
      s += b_signed ? (int32_t)(int8_t)tile[i][tx] : (int32_t)tile[i][tx];
    atomicAdd(colsum + n0 + tx, s);
  }
}

// rowsum[m] = sum_k a[m, k] (one warp per row)
__global__ void rowsum_kernel(const uint8_t* __restrict__ a, int a_signed,
                              int M, int K, int32_t* __restrict__ rowsum) {
  pdl_wait();
  pdl_trigger();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M) return;
  int32_t s = 0;
  for (int k = lane; k < K; k += 32) {
    const uint8_t v = a[(size_t)w * K + k];
    s += a_signed ? (int32_t)(int8_t)v : (int32_t)v;
  }
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) rowsum[w] = s;
}

static bool is_8bit(int t) { return t == ICX_U8 || t == ICX_S8; }

}  // namespace icx

using namespace icx;

extern "C" int icx_prepare_b(void* stream, const void* d_b, int b_type, size_t K,
                             size_t N, void* d_bt, int32_t* d_colsum) {
  ICX_REQUIRE(is_8bit(b_type), "MatMulInteger: b must be Int8 or UInt8");
  ICX_REQUIRE(K < (1u << 30) && N < (1u << 30), "MatMulInteger: b too large");
  if (K == 0 || N == 0) {
    if (N && d_colsum) ICX_CUDA(cudaMemsetAsync(d_colsum, 0, N * 4, as_stream(stream)));
    return ICX_OK;
  }
  ICX_REQUIRE(d_b && d_bt && d_colsum, "MatMulInteger: null weight buffer");
  cudaStream_t s = as_stream(stream);
  ICX_CUDA(cudaMemsetAsync(d_colsum, 0, N * sizeof(int32_t), s));
  dim3 grid((unsigned)((N + 31) / 32), (unsigned)((K + 31) / 32));
  launch_pdl(prepare_b_kernel, dim3(grid), dim3(dim3(32, 8)), 0, s, 
      static_cast<const uint8_t*>(d_b), b_type == ICX_S8, (int)K, (int)N,
      static_cast<uint8_t*>(d_bt), d_colsum);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

extern "C" size_t icx_matmul_integer_workspace_bytes(size_t M, size_t K, size_t N) {
  return align256(N * K) + align256(N * 4) + align256(M * 4);
}

extern "C" int icx_matmul_integer_prepared(
    void* stream, const void* d_a, int a_type, const void* d_bt, int b_type,
    const int32_t* d_colsum, size_t M, size_t K, size_t N, const void* d_a_zp,
    const void* d_b_zp, int b_zp_per_col, const int32_t* d_rowsum_a,
    int32_t* d_out) {
  ICX_REQUIRE(is_8bit(a_type), "MatMulInteger: input a must be Int8 or UInt8");
  ICX_REQUIRE(is_8bit(b_type), "MatMulInteger: input b must be Int8 or UInt8");
  ICX_REQUIRE(M < (1u << 31) && N < (1u << 30) && K < (1u << 30),
              "MatMulInteger: shape too large");
  if (M == 0 || N == 0) return ICX_OK;
  ICX_REQUIRE(d_out && d_colsum && (K == 0 || (d_a && d_bt)),
              "MatMulInteger: null operand");
  ICX_REQUIRE(d_b_zp == nullptr || d_rowsum_a != nullptr,
              "MatMulInteger: b_zero_point needs the row sums of a");
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.a_zp = d_a_zp; g.a_zp_signed = a_type == ICX_S8;
  g.b_zp = d_b_zp; g.b_zp_signed = b_type == ICX_S8; g.b_zp_per_col = b_zp_per_col;
  g.colsum = d_colsum; g.rowsum = d_rowsum_a;
  g.out = d_out;
  cudaStream_t s = as_stream(stream);
  if (K == 0) {
    // empty reduction: every output is K*za*zb = 0
    ICX_CUDA(cudaMemsetAsync(d_out, 0, M * N * 4, s));
    return ICX_OK;
  }
  return launch_gemm<kEpiS32>(s, d_a, a_type == ICX_S8, d_bt, b_type == ICX_S8, g);
}

extern "C" int icx_matmul_integer(void* stream, const void* d_a, int a_type,
                                  const void* d_b, int b_type, size_t M,
                                  size_t K, size_t N, const void* d_a_zp,
                                  const void* d_b_zp, int b_zp_per_col,
                                  int32_t* d_out, void* d_workspace,
                                  size_t workspace_bytes) {
  ICX_REQUIRE(is_8bit(a_type), "MatMulInteger: input a must be Int8 or UInt8");
  ICX_REQUIRE(is_8bit(b_type), "MatMulInteger: input b must be Int8 or UInt8");
  const size_t need = icx_matmul_integer_workspace_bytes(M, K, N);
  ICX_REQUIRE(d_workspace && workspace_bytes >= need,
              "MatMulInteger: workspace %zu bytes < %zu required", workspace_bytes, need);
  uint8_t* ws = static_cast<uint8_t*>(d_workspace);
  void* bt = ws;
  int32_t* colsum = reinterpret_cast<int32_t*>(ws + align256(N * K));
  int32_t* rowsum = reinterpret_cast<int32_t*>(ws + align256(N * K) + align256(N * 4));
  int rc = icx_prepare_b(stream, d_b, b_type, K, N, bt, colsum);
  if (rc) return rc;
  if (d_b_zp && M && K) {
    const int threads = 256;
    const size_t blocks = (M * 32 + threads - 1) / threads;
    launch_pdl(rowsum_kernel, dim3((unsigned)blocks), dim3(threads), 0, as_stream(stream), 
        static_cast<const uint8_t*>(d_a), a_type == ICX_S8, (int)M, (int)K, rowsum);
    ICX_LAUNCH_CHECK();
  } else if (d_b_zp && M) {
    ICX_CUDA(cudaMemsetAsync(rowsum, 0, M * 4, as_stream(stream)));
  }
  return icx_matmul_integer_prepared(stream, d_a, a_type, bt, b_type, colsum, M, K, N,
                                     d_a_zp, d_b_zp, b_zp_per_col, rowsum, d_out);
}

extern "C" int icx_quant_linear(void* stream, const uint8_t* d_q,
                                const float* d_a_scale, const uint8_t* d_a_zp,
                                const int32_t* d_rowsum_q, const int8_t* d_wt,
                                const int32_t* d_colsum, size_t M, size_t K,
                                size_t N, const float* d_w_scale,
                                int w_scale_per_col, const int8_t* d_b_zp,
                                int b_zp_per_col, const float* d_bias, int gelu,
                                const float* d_residual, float* d_out, float* d_minmax,
                                int* n_minmax) {
  ICX_REQUIRE(M < (1u << 31) && N < (1u << 30) && K < (1u << 30),
              "QuantLinear: shape too large");
  if (M == 0 || N == 0) return ICX_OK;
  ICX_REQUIRE(d_out && d_colsum && d_a_scale && d_w_scale && (K == 0 || (d_q && d_wt)),
              "QuantLinear: null operand");
  ICX_REQUIRE(d_b_zp == nullptr || d_rowsum_q != nullptr,
              "QuantLinear: b_zero_point needs the row sums of q");
  ICX_REQUIRE(K > 0, "QuantLinear: K must be positive");
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.a_zp = d_a_zp; g.a_zp_signed = 0;
  g.b_zp = d_b_zp; g.b_zp_signed = 1; g.b_zp_per_col = b_zp_per_col;
  g.colsum = d_colsum; g.rowsum = d_rowsum_q;
  g.a_scale = d_a_scale; g.w_scale = d_w_scale; g.w_scale_per_col = w_scale_per_col;
  g.bias = d_bias;
  g.residual = d_residual;
  g.out = d_out;
  g.minmax = reinterpret_cast<float2*>(d_minmax);
  if (n_minmax) *n_minmax = gemm_grid(g, d_q, d_wt);
  cudaStream_t s = as_stream(stream);
  return gelu ? launch_gemm<kEpiGelu>(s, d_q, false, d_wt, true, g)
              : launch_gemm<kEpiF32>(s, d_q, false, d_wt, true, g);
}

// ------------------------------------------------ QuantLinear + LayerNorm
// Epilogue warps of the LayerNorm-fused GEMM: three per TMEM lane quadrant,
// four 16-column chunks each (64 values per thread within the 128
// registers that 448 threads leave).
constexpr int kLnWarps = 12;

// Clusters of the LayerNorm-fused GEMM (N / 192 CTAs each) that can be
// resident at once, per device, cluster size and ring depth (cached).
template <bool DEEP>
static int max_ln_clusters(int ncl) {
  static int cached[64][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || ncl < 1 || ncl > 8) return 0;
  if (cached[dev][ncl]) return cached[dev][ncl];
  using C = Cfg<192, DEEP, kLnWarps, 1>;
  auto kern = qgemm_tcgen05_kernel<192, kEpiLn, false, true, DEEP, kLnWarps, 1>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ncl * (148 / ncl));
  cfg.blockDim = dim3(gemm_threads<kLnWarps>());
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ncl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 0;
  }
  cached[dev][ncl] = n;
  return n;
}

namespace icx {
bool quant_linear_ln_supported(size_t K, size_t N);
bool quant_linear_ln_preferred(size_t M, size_t K, size_t N);
}  // namespace icx

// Whether the engine should fuse the LayerNorm into the GEMM: where every
// 128-row block gets a cluster of its own (one tile per CTA), so that the
// longer epilogue only adds latency.  With several tiles per CTA the
// epilogue's throughput sets the pace and the unfused GEMM (CTA pairs at
// deep K) plus a separate LayerNorm was measured faster (BERT-base config 4,
// M = 32768: 3926 against 3853 seq/s).
bool icx::quant_linear_ln_preferred(size_t M, size_t K, size_t N) {
  if (!quant_linear_ln_supported(K, N)) return false;
  const int ncl = (int)(N / 192);
  const size_t num_m = (M + kBM - 1) / kBM;
  const int cl = K >= 1536 ? max_ln_clusters<true>(ncl) : max_ln_clusters<false>(ncl);
  return num_m <= (size_t)cl;
}

bool icx::quant_linear_ln_supported(size_t K, size_t N) {
  if (K == 0 || K % 16 != 0 || K >= (1u << 30) || N % 192 != 0) return false;
  const int ncl = (int)(N / 192);
  if (ncl < 2 || ncl > 4) return false;
  return (K >= 1536 ? max_ln_clusters<true>(ncl) : max_ln_clusters<false>(ncl)) > 0;
}

extern "C" int icx_quant_linear_layernorm(void* stream, const uint8_t* d_q, const float* d_a_scale,
                                          const uint8_t* d_a_zp, const int32_t* d_rowsum_q,
                                          const int8_t* d_wt, const int32_t* d_colsum, size_t M,
                                          size_t K, size_t N, const float* d_w_scale,
                                          int w_scale_per_col, const int8_t* d_b_zp, int b_zp_per_col,
                                          const float* d_bias, const float* d_residual,
                                          const float* d_gamma, const float* d_beta, float epsilon,
                                          float* d_out, float* d_minmax, int* n_minmax) {
  ICX_REQUIRE(M < (1u << 31), "QuantLinear+LayerNorm: shape too large");
  ICX_REQUIRE(icx::quant_linear_ln_supported(K, N),
              "QuantLinear+LayerNorm: K=%zu N=%zu unsupported (K %% 16 == 0, N = 192 x 2..4)", K, N);
  if (n_minmax) *n_minmax = 0;
  if (M == 0) return ICX_OK;
  ICX_REQUIRE(d_q && d_wt && d_out && d_colsum && d_a_scale && d_w_scale && d_residual && d_gamma,
              "QuantLinear+LayerNorm: null operand");
  ICX_REQUIRE(d_b_zp == nullptr || d_rowsum_q != nullptr,
              "QuantLinear+LayerNorm: b_zero_point needs the row sums of q");
  ICX_REQUIRE(aligned16(d_q) && aligned16(d_wt) && aligned16(d_out) && aligned16(d_colsum) &&
                  aligned16(d_residual) && aligned16(d_gamma) && (!d_beta || aligned16(d_beta)) &&
                  (!d_bias || aligned16(d_bias)) && (!w_scale_per_col || aligned16(d_w_scale)) &&
                  (!d_b_zp || !b_zp_per_col || (reinterpret_cast<uintptr_t>(d_b_zp) & 3) == 0),
              "QuantLinear+LayerNorm: operands must be 16-byte aligned");
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.a_zp = d_a_zp; g.a_zp_signed = 0;
  g.b_zp = d_b_zp; g.b_zp_signed = 1; g.b_zp_per_col = b_zp_per_col;
  g.colsum = d_colsum; g.rowsum = d_rowsum_q;
  g.a_scale = d_a_scale; g.w_scale = d_w_scale; g.w_scale_per_col = w_scale_per_col;
  g.bias = d_bias;
  g.residual = d_residual;
  g.out = d_out;
  g.minmax = reinterpret_cast<float2*>(d_minmax);
  g.ln_gamma = d_gamma;
  g.ln_beta = d_beta;
  g.ln_eps = epsilon;
  const int ncl = (int)(N / 192);
  const bool deep = K >= 1536;
  const long num_m = (long)((M + kBM - 1) / kBM);
  const long cl = deep ? max_ln_clusters<true>(ncl) : max_ln_clusters<false>(ncl);
  const int grid = (int)(num_m < cl ? num_m : cl) * ncl;
  if (n_minmax) *n_minmax = grid;
  cudaStream_t s = as_stream(stream);
  return deep ? launch_tc<192, kEpiLn, true, kLnWarps, 1>(s, d_q, false, d_wt, true, g, grid)
              : launch_tc<192, kEpiLn, false, kLnWarps, 1>(s, d_q, false, d_wt, true, g, grid);
}

extern "C" int icx_matmul_integer_rowsum(void* stream, const void* d_a, int a_type, size_t M,
                                         size_t K, int32_t* d_rowsum) {
  ICX_REQUIRE(is_8bit(a_type), "MatMulInteger: input a must be Int8 or UInt8");
  ICX_REQUIRE(M < (1u << 31) && K < (1u << 30), "MatMulInteger: shape too large");
  if (M == 0) return ICX_OK;
  ICX_REQUIRE(d_rowsum && (K == 0 || d_a), "MatMulInteger: null pointer");
  cudaStream_t s = as_stream(stream);
  if (K == 0) {
    ICX_CUDA(cudaMemsetAsync(d_rowsum, 0, M * 4, s));
    return ICX_OK;
  }
  const int threads = 256;
  const size_t blocks = (M * 32 + threads - 1) / threads;
  launch_pdl(rowsum_kernel, dim3((unsigned)blocks), dim3(threads), 0, s, static_cast<const uint8_t*>(d_a),
                                                     a_type == ICX_S8, (int)M, (int)K, d_rowsum);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}
