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

#include <cstdlib>
#include <cstring>

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

// ---------------------------------------------------------------------------
// Tensor-core attention on the 5th-generation tensor cores (tcgen05.mma,
// accumulators in TMEM), one CTA per 128 query rows of one (batch, head).
//
// Scores S = Q K^T are computed with exact integer accumulation (the
// "Ozaki" splitting): every row x of Q and of K is scaled by a power of two
// 2^(25-n) (n from the row's largest magnitude, |x| < 2^(n+6)) and rounded
// to a 31-bit integer T, whose four bytes are the slices:
//     T = d0 2^24 + d1 2^16 + d2 2^8 + d3,  d0 signed, d1..d3 unsigned,
// so x = 2^(n-1) (d0 + d1 / 2^8 + d2 / 2^16 + d3 / 2^24) + r, |r| <= 2^(n-26).
// The products of slices with i + j <= 3 run as kind::i8 MMAs (s8 / u8
// operands as the digit requires, K=32 per instruction) accumulated per
// level L = i + j in s32; |acc_L| < 2^24, so the sums are exact and convert
// exactly to fp32.  The score is then
//     s = (((acc3 / 2^24 + acc2 / 2^16) + acc1 / 2^8) + acc0) 2^(nq-1) 2^(nk-1)
// with three fp32 roundings; the neglected products (i + j >= 4) are below
// 2^-30 of |q|max |k|max per term.  Exactness matters because softmax
// amplifies absolute score errors, and scores can be large.
//
// P V uses TF32 with the split-precision trick instead: p and v are split as
// x = hi + lo (hi = tf32(x), lo = tf32(x - hi)) and each product is formed as
// hi*hi + hi*lo + lo*hi (three kind::tf32 MMAs); errors there are not
// amplified (p <= 1).
//
// 16 warps: query row r is TMEM lane r; warp w reads lanes 32*(w%4) .. +31
// (the quadrant a warp may access) and owns columns 16*(w/4) .. +15 of every
// 64-key tile, so four warps share a row and exchange its running max / sum
// through shared memory.  Per 64-key tile:
//   1. all threads slice the tile's K rows (bytes, [key][slice pair][d]) and
//      split V (tf32 hi / lo, stored transposed as [d][key]), both in the
//      128-byte-swizzled K-major layout the MMA reads; the registers were
//      loaded while the previous tile was processed;
//   2. thread 0 issues the 20 integer MMAs of S (M=128, N=64, K=32) into
//      TMEM columns [64 L, 64 L + 64) for L = 0..3;
//   3. each thread combines its 16 scores, applies Div(c) and Add(mask); the
//      row max over the four warps gives the online-softmax update; the
//      unnormalised probabilities P go, split, to shared memory;
//   4. thread 0 issues O_tile = P V (M=128, N=64, K=64 keys) into columns
//      [256, 320); each thread rescales its 16 accumulator columns and adds
//      its O_tile slice.
constexpr int kTcQ = 128;
constexpr int kTcK = 64;
constexpr int kTcThreads = 512;
constexpr int kTcCols = 16;           // score / context columns per thread
constexpr int kQAtom = kTcQ * 128;    // one 128-byte-wide column block of 128 rows
constexpr int kKAtom = kTcK * 128;    // one 128-byte-wide column block of 64 rows
constexpr int kOffQs = 0;                              // Q slices: 2 blocks (slices 0|1, 2|3)
constexpr int kOffKs = kOffQs + 2 * kQAtom;            // K slices: 2 blocks
constexpr int kOffVh = kOffKs + 2 * kKAtom;            // V^T hi / lo: 2 blocks each
constexpr int kOffVl = kOffVh + 2 * kKAtom;
constexpr int kOffPh = kOffVl + 2 * kKAtom;            // P hi / lo: 2 blocks each
constexpr int kOffPl = kOffPh + 2 * kQAtom;
constexpr int kOffRed = kOffPl + 2 * kQAtom;           // [4][128] partial max, [4][128] partial sum
constexpr int kOffScale = kOffRed + 2 * 4 * kTcQ * 4;  // 2^nq per query row, 2^nk per key
constexpr int kOffMask = kOffScale + (kTcQ + kTcK) * 4;  // additive mask per key of the tile
constexpr int kOffBar = kOffMask + kTcK * 4;
constexpr int kTcSmem = kOffBar + 64 + 1024 /*align slack*/;
constexpr uint32_t kTcTmemCols = 512;
constexpr int kTmemO = 4 * kTcK;  // O_tile columns

// Round to the nearest TF32 value (ties away from zero) by integer
// arithmetic on the bit pattern.
__device__ __forceinline__ float tf32_round(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
}

// 2^n as a float, n clamped to the normal range.
__device__ __forceinline__ float pow2f(int n) {
  n = max(-126, min(127, n));
  return __int_as_float((n + 127) << 23);
}

// Byte offset of byte `col` of row `row` in a K-major operand stored as
// 128-byte-wide column blocks `block` bytes apart, 128-byte rows, 128-byte
// swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ int sw128_byte(int block, int row, int col) {
  return (col >> 7) * block + row * 128 + ((((col & 127) >> 4) ^ (row & 7)) << 4) + (col & 15);
}

// Splits fp32 columns col..col+3 of `row` (col % 4 == 0) into tf32 hi / lo.
__device__ __forceinline__ void split_store(uint8_t* hi, uint8_t* lo, int block, int row, int col,
                                            float4 v) {
  const int off = sw128_byte(block, row, col * 4);
  float4 h, l;
  h.x = tf32_round(v.x);
  h.y = tf32_round(v.y);
  h.z = tf32_round(v.z);
  h.w = tf32_round(v.w);
  l.x = tf32_round(__fsub_rn(v.x, h.x));
  l.y = tf32_round(__fsub_rn(v.y, h.y));
  l.z = tf32_round(__fsub_rn(v.z, h.z));
  l.w = tf32_round(__fsub_rn(v.w, h.w));
  *reinterpret_cast<float4*>(hi + off) = h;
  *reinterpret_cast<float4*>(lo + off) = l;
}

// Slices 4 values of a row whose 64 values are spread over 16 consecutive
// lanes (4 each) and stores them: byte i of T (most significant first) of
// the 4 values is one 32-bit word at byte (i % 2) * 64 + col of column block
// i / 2.  Returns 2^(n-1), the row's factor in the score.
__device__ __forceinline__ float slice_row_store(uint8_t* base, int block, int row, int col, float4 v) {
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int o = 8; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  // m < 2^(E - 126) for a normal m with biased exponent E: n = E - 132
  const int n = max(-101, (int)((__float_as_uint(m) >> 23) & 0xff) - 132);
  const float sc = pow2f(25 - n);
  const int t0 = __float2int_rn(__fmul_rn(v.x, sc)), t1 = __float2int_rn(__fmul_rn(v.y, sc));
  const int t2 = __float2int_rn(__fmul_rn(v.z, sc)), t3 = __float2int_rn(__fmul_rn(v.w, sc));
  const int off = sw128_byte(block, row, col);  // slice 0; slice i: ^ (i%2)*64, + (i/2)*block
  const uint32_t lo01 = __byte_perm(t0, t1, 0x7340), hi01 = __byte_perm(t0, t1, 0x5162);
  const uint32_t lo23 = __byte_perm(t2, t3, 0x7340), hi23 = __byte_perm(t2, t3, 0x5162);
  // lo01 = [t0.b0, t1.b0, t0.b3, t1.b3] ... combine into per-byte words
  *reinterpret_cast<uint32_t*>(base + off) = __byte_perm(lo01, lo23, 0x7632);          // byte 3
  *reinterpret_cast<uint32_t*>(base + (off ^ 64)) = __byte_perm(hi01, hi23, 0x5410);   // byte 2
  *reinterpret_cast<uint32_t*>(base + block + off) = __byte_perm(hi01, hi23, 0x7632);  // byte 1
  *reinterpret_cast<uint32_t*>(base + block + (off ^ 64)) = __byte_perm(lo01, lo23, 0x5410);  // byte 0
  return pow2f(n - 1);
}

__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const float* __restrict__ q, const float* __restrict__ k,
                        const float* __restrict__ v, int ld, float* __restrict__ out, int H, int S,
                        int nh, float c, const float* __restrict__ mask, int mask_per_batch) {
  extern __shared__ __align__(1024) uint8_t att_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(att_raw) + 1023) & ~uintptr_t(1023));
  float* red_max = reinterpret_cast<float*>(sm + kOffRed);
  float* red_sum = red_max + 4 * kTcQ;
  float* q_scale = reinterpret_cast<float*>(sm + kOffScale);
  float* k_scale = q_scale + kTcQ;
  float* m_tile = reinterpret_cast<float*>(sm + kOffMask);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_s + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cg = warp >> 2;
  const int row = quad * 32 + lane;  // query row within the tile = TMEM lane
  const int col0 = cg * kTcCols;     // first score / context column of this thread
  const int bh = blockIdx.y;
  const int b = bh / nh, h = bh % nh;
  const int q0 = blockIdx.x * kTcQ;
  const size_t head = (size_t)b * S * ld + (size_t)h * kAttDh;
  const float* mrow = mask ? mask + (mask_per_batch ? (size_t)b * S : 0) : nullptr;
  int cexp;
  const bool c_pow2 = frexpf(c, &cexp) == 0.5f;
  const float inv_c = 1.0f / c;
  // Q / K rows: 16 threads per 256-byte row; V: thread = column d (tid % 64)
  // of keys 8 (tid / 64) .. +7, stored as row d of V^T
  const int kv_row = tid >> 4, kv_col = (tid & 15) * 4;
  const int v_d = tid & 63, v_key = (tid >> 6) * 8;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, kTcTmemCols);
    tmem_relinquish();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (i * kTcThreads + tid) >> 4, qi = q0 + r;
    const float4 x = qi < S ? __ldg(reinterpret_cast<const float4*>(q + head + (size_t)qi * ld + kv_col))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    const float f = slice_row_store(sm + kOffQs, kQAtom, r, kv_col, x);
    if (kv_col == 0) q_scale[r] = f;
  }
  // the first K / V tile into registers
  float4 nk[2], nv[2];
  float nm = 0.0f;  // the tile's additive mask value for key tid (tid < 64)
  auto load_kv = [&](int k0) {
    if (tid < kTcK) {
      const int key = k0 + tid;
      nm = key >= S ? -INFINITY : (mrow ? __ldg(mrow + key) : 0.0f);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int kr = k0 + kv_row + 32 * i;
      nk[i] = kr < S ? __ldg(reinterpret_cast<const float4*>(k + head + (size_t)kr * ld + kv_col))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
      float x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int vr = k0 + v_key + 4 * i + u;
        x[u] = vr < S ? __ldg(v + head + (size_t)vr * ld + v_d) : 0.0f;
      }
      nv[i] = make_float4(x[0], x[1], x[2], x[3]);
    }
  };
  load_kv(0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tslot;
  const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)col0;
  constexpr uint32_t idesc_o = idesc_tf32(kTcQ, kAttDh, false);
  const uint32_t a_qs = smem_addr(sm + kOffQs), a_ks = smem_addr(sm + kOffKs);
  const uint32_t a_v_h = smem_addr(sm + kOffVh), a_v_l = smem_addr(sm + kOffVl);
  const uint32_t a_p_h = smem_addr(sm + kOffPh), a_p_l = smem_addr(sm + kOffPl);
  const float qsc = q_scale[row];
  const float qf = __fmul_rn(qsc, inv_c);  // a power of two when c is

  float m_run = -INFINITY, l_part = 0.0f, o[kTcCols];
#pragma unroll
  for (int d = 0; d < kTcCols; ++d) o[d] = 0.0f;
  bool ok = true;
  uint32_t phase = 0;
  for (int k0 = 0; k0 < S; k0 += kTcK, phase ^= 1) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float f = slice_row_store(sm + kOffKs, kKAtom, kv_row + 32 * i, kv_col, nk[i]);
      if (kv_col == 0) k_scale[kv_row + 32 * i] = f;
      split_store(sm + kOffVh, sm + kOffVl, kKAtom, v_d, v_key + 4 * i, nv[i]);
    }
    // the tile's additive mask; keys past S get -inf
    if (tid < kTcK) m_tile[tid] = nm;
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int L = 0; L < 4; ++L) {
#pragma unroll
        for (int i = 0; i <= L; ++i) {
          const int j = L - i;
#pragma unroll
          for (int hd = 0; hd < 2; ++hd) {
            // slice i of Q / slice j of K, d half hd (32 bytes each)
            const uint32_t ao = (i >> 1) * kQAtom + (i & 1) * 64 + hd * 32;
            const uint32_t bo = (j >> 1) * kKAtom + (j & 1) * 64 + hd * 32;
            // the most significant slice is signed, the others unsigned
            mma_i8(tmem_base + (uint32_t)(L * kTcK), smem_desc_k128(a_qs + ao),
                   smem_desc_k128(a_ks + bo), idesc_i8(kTcQ, kTcK, i == 0, j == 0), (i | hd) != 0);
          }
        }
      }
      mma_commit(bar_s);
    }
    if (k0 + kTcK < S) load_kv(k0 + kTcK);  // lands while this tile is processed
    ok = mbar_wait_warp(bar_s, phase, ICX_DEVICE_TIMEOUT_EPILOGUE);
    tc_fence_after();
    float p[kTcCols];
#pragma unroll
    for (int j = 0; j < kTcCols; ++j) p[j] = 0.0f;
    if (ok) {
      // (((acc3 / 2^24 + acc2 / 2^16) + acc1 / 2^8) + acc0), one rounding per
      // step; the four loads are in flight together
      uint32_t r0[16], r1[16], r2[16], r3[16];
      tmem_ld_32x32b_x16(t_row + (uint32_t)(3 * kTcK), r3);
      tmem_ld_32x32b_x16(t_row + (uint32_t)(2 * kTcK), r2);
      tmem_ld_32x32b_x16(t_row + (uint32_t)(1 * kTcK), r1);
      tmem_ld_32x32b_x16(t_row, r0);
      tmem_ld_wait_regs16(r3);
      tmem_ld_wait_regs16(r2);
      tmem_ld_wait_regs16(r1);
      tmem_ld_wait_regs16(r0);
#pragma unroll
      for (int j = 0; j < kTcCols; ++j) {
        float f = __fmul_rn((float)(int32_t)r3[j], 5.9604644775390625e-08f);
        f = __fmaf_rn((float)(int32_t)r2[j], 1.52587890625e-05f, f);
        f = __fmaf_rn((float)(int32_t)r1[j], 0.00390625f, f);
        p[j] = __fadd_rn((float)(int32_t)r0[j], f);
      }
    }
    // scale by 2^(nq + nk), Div(c), Add(mask) (-inf past S)
    float pmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < kTcCols; ++j) {
      float t;
      if (c_pow2) {
        t = __fmul_rn(__fmul_rn(p[j], qf), k_scale[col0 + j]);  // exact: powers of two
      } else {
        t = __fdiv_rn(__fmul_rn(__fmul_rn(p[j], qsc), k_scale[col0 + j]), c);
      }
      t = __fadd_rn(t, m_tile[col0 + j]);
      p[j] = t;
      pmax = fmaxf(pmax, t);
    }
    red_max[cg * kTcQ + row] = pmax;
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    const float tmax = fmaxf(fmaxf(red_max[row], red_max[kTcQ + row]),
                             fmaxf(red_max[2 * kTcQ + row], red_max[3 * kTcQ + row]));
    // online softmax: exp(a - m) = 2^(a*log2e - m*log2e)
    const float m_new = fmaxf(m_run, tmax);
    const float ml = m_new == -INFINITY ? 0.0f : m_new * kLog2e;  // a fully masked row stays 0
    const float alpha = m_run == -INFINITY ? 0.0f : ex2f(fmaf(m_run, kLog2e, -ml));
    float rsum = 0.0f;
#pragma unroll
    for (int j = 0; j < kTcCols; ++j) {
      p[j] = ex2f(fmaf(p[j], kLog2e, -ml));  // 2^-inf = 0 for masked keys
      rsum += p[j];
    }
    l_part = l_part * alpha + rsum;
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < kTcCols; j += 4)
      split_store(sm + kOffPh, sm + kOffPl, kQAtom, row, col0 + j,
                  make_float4(p[j], p[j + 1], p[j + 2], p[j + 3]));
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < kTcK / 8; ++j) {
        // k-step j = keys 8j..8j+7: P column block j/4, V^T column block j/4
        const uint32_t ao = (j >> 2) * kQAtom + (j & 3) * 32, bo = (j >> 2) * kKAtom + (j & 3) * 32;
        const uint64_t ph = smem_desc_k128(a_p_h + ao), pl = smem_desc_k128(a_p_l + ao);
        const uint64_t vh = smem_desc_k128(a_v_h + bo), vl = smem_desc_k128(a_v_l + bo);
        mma_tf32(tmem_base + kTmemO, ph, vh, idesc_o, j > 0);
        mma_tf32(tmem_base + kTmemO, ph, vl, idesc_o, true);
        mma_tf32(tmem_base + kTmemO, pl, vh, idesc_o, true);
      }
      mma_commit(bar_o);
    }
    ok = mbar_wait_warp(bar_o, phase, ICX_DEVICE_TIMEOUT_EPILOGUE);
    tc_fence_after();
    if (ok) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_row + kTmemO, r);
      tmem_ld_wait_regs16(r);
#pragma unroll
      for (int d = 0; d < kTcCols; ++d) o[d] = fmaf(o[d], alpha, __uint_as_float(r[d]));
    }
    // TMEM reads of this tile are done before the next tile's MMAs overwrite
    tc_fence_before();
  }
  red_sum[cg * kTcQ + row] = l_part;
  ok = __syncthreads_and(ok) != 0;
  const int qi = q0 + row;
  if (ok && qi < S) {
    const float l = (red_sum[row] + red_sum[kTcQ + row]) + (red_sum[2 * kTcQ + row] + red_sum[3 * kTcQ + row]);
    const float inv = 1.0f / l;
    float4* orow = reinterpret_cast<float4*>(out + ((size_t)b * S + qi) * H + (size_t)h * kAttDh + col0);
#pragma unroll
    for (int d = 0; d < kTcCols; d += 4)
      orow[d / 4] = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
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
  if (B == 0 || S == 0 || nh == 0) return ICX_OK;
  static const bool simt = [] {
    const char* e = getenv("ICONNX_ATTENTION");
    return e != nullptr && strcmp(e, "simt") == 0;
  }();
  if (!simt) {
    ICX_REQUIRE(B * nh <= 65535, "Attention: batch x heads %lld too large", (long long)(B * nh));
    ICX_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kTcSmem));
    dim3 grid((unsigned)((S + kTcQ - 1) / kTcQ), (unsigned)(B * nh));
    attention_tc_kernel<<<grid, kTcThreads, kTcSmem, s>>>(q, k, v, (int)ld, out, (int)H, (int)S,
                                                            (int)nh, c, mask, mask_per_batch ? 1 : 0);
    ICX_LAUNCH_CHECK();
    return ICX_OK;
  }
  const int smem = 4 * kAttTile * kAttPad * (int)sizeof(float);
  ICX_CUDA(cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid((unsigned)(B * nh), (unsigned)((S + kAttTile - 1) / kAttTile));
  attention_f32_kernel<<<grid, kAttThreads, smem, s>>>(q, k, v, (int)ld, out, (int)H, (int)S, (int)nh,
                                                       c, mask, mask_per_batch ? 1 : 0);
  ICX_LAUNCH_CHECK();
  return ICX_OK;
}

}  // namespace icx
