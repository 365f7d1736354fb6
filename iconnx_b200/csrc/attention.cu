// Fused attention for the engine's attention fusion: for each (batch, head)
// and query tile,
//     ctx = softmax(Q K^T / c + mask) V
// in one kernel, with online (running max / running sum) softmax over key
// tiles, so the [B, heads, S, S] score tensor never reaches HBM.  It replaces
// the MatMul -> Div -> Add -> Softmax -> MatMul sequence the reference runs
// as cuBLAS SGEMMs and NVRTC kernels (src/cuda/matmul.rs,
// src/cuda/reduction.rs).  Semantics are the reference's fp32: Div by c and
// Add of the mask are each rounded as the separate ops round them; the
// softmax normalisation order differs (online), within fp32 rounding.
//
// Two kernels:
//   attention_tc_kernel   the one the engine runs: scores on the int8 tensor
//                         cores with exact integer accumulation, P V on the
//                         tf32 tensor cores in split precision (see below);
//   attention_f32_kernel  CUDA-core fp32 (ICONNX_ATTENTION=simt), kept for
//                         comparison.
//
// Layout: q / k / v rows are `ld` floats apart (the merged QKV GEMM output
// has ld = 3H), head h occupies columns [h*dh, (h+1)*dh); ctx is [B, S, H].
//
// attention_f32_kernel tiles: 128 threads; thread (ty, tx) = (tid / 16,
// tid % 16) owns score rows ty + 8 i (i < 8) and key columns tx + 16 j
// (j < 4), and context columns 4 tx .. 4 tx + 3 of the same rows: 12 shared
// 16-byte loads per 128 FMAs.  Shared rows are padded to 68 floats so the
// strided column pattern is bank-conflict free.
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
  pdl_wait();
  pdl_trigger();
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
// Tiling (AttTc below): KT keys per tile, NW warps per CTA; query row r is
// TMEM lane r and warp w reads lanes 32*(w%4) .. +31 (the quadrant a warp
// may access); with NW = 8 two warps share each row (columns split, row max
// and sum exchanged through shared memory).  The default <32, 4> runs three
// CTAs per SM, one warp per row block, so one CTA's MMA waits and load
// latencies overlap the others' work.  Per key tile:
//   1. all threads slice the tile's K rows (bytes, [key][slice pair][d],
//      loaded into registers during the previous tile) into the
//      128-byte-swizzled K-major layout the MMA reads;
//   2. thread 0 issues the 20 integer MMAs of S (M=128, N=KT, K=32) into TMEM
//      columns [KT L, KT L + KT) for L = 0..3; meanwhile all threads load V,
//      split it into tf32 hi / lo and store it transposed ([d][key]);
//   3. each thread combines its scores, applies Div(c) and Add(mask), takes
//      the row max (online softmax) and writes the unnormalised
//      probabilities P, split hi / lo, back into TMEM columns [0,KT) /
//      [KT,2KT) (the consumed score columns);
//   4. thread 0 issues O_tile = P V (M=128, N=64, K=KT keys; A = P read from
//      TMEM, B = V^T from shared memory) into columns [2KT, 2KT+64);
//      meanwhile all threads load the next K tile; each thread rescales its
//      accumulator columns and adds its O_tile slice.
constexpr int kTcQ = 128;
constexpr int kQAtom = kTcQ * 128;  // one 128-byte-wide column block of 128 rows

// Tiling of the tensor-core attention: KT keys per tile, NW warps per CTA
// (NW / 4 warps share each TMEM lane quadrant, i.e. each query row).
//   <64, 8>: 84 KB shared memory, 256 TMEM columns, two CTAs per SM;
//   <32, 4>: 58 KB, 128 TMEM columns, three CTAs per SM (every CTA of a
//            batch-32 DistilBERT layer resident at once), one warp per row
//            block (no cross-warp row max / sum exchange).
template <int KT, int NW>
struct AttTc {
  static constexpr int kThreads = 32 * NW;
  static constexpr int kWPQ = NW / 4;          // warps per lane quadrant
  static constexpr int kSC = KT / kWPQ;        // score columns per thread
  static constexpr int kOC = 64 / kWPQ;        // context columns per thread
  static constexpr int kQLoads = 2048 / kThreads;       // float4 of Q per thread
  static constexpr int kKLoads = KT * 16 / kThreads;    // float4 of K per thread per tile
  static constexpr int kVKeys = KT * 64 / kThreads;     // keys of V per thread per tile (one d)
  static constexpr int kKAtom = KT * 128;      // K slices: KT rows x 128 B per block
  static constexpr int kVAtom = 64 * 128;      // V^T: 64 rows (d) x 32 keys (128 B) per block
  static constexpr int kVBlocks = KT / 32;
  static constexpr int kOffQs = 0;                            // Q slices: 2 blocks (0|1, 2|3)
  static constexpr int kOffKs = kOffQs + 2 * kQAtom;          // K slices: 2 blocks
  static constexpr int kOffVh = kOffKs + 2 * kKAtom;          // V^T hi / lo
  static constexpr int kOffVl = kOffVh + kVBlocks * kVAtom;
  static constexpr int kOffRed = kOffVl + kVBlocks * kVAtom;  // row max / sum exchange
  static constexpr int kRedFloats = 2 * kWPQ * kTcQ > 32 ? 2 * kWPQ * kTcQ : 32;
  static constexpr int kOffScale = kOffRed + kRedFloats * 4;  // 2^(nq-1) per row, 2^(nk-1) per key
  static constexpr int kOffMask = kOffScale + (kTcQ + KT) * 4;  // additive mask of the tile
  static constexpr int kOffBar = kOffMask + KT * 4;
  // fp32 staging of the next tile, filled by cp.async while this tile's
  // softmax runs: V always, K too where three CTAs per SM still fit (<32, 4>;
  // <64, 8> keeps K in registers)
  static constexpr bool kStageK = KT == 32;
  static constexpr int kOffRawK = kOffBar + 64;
  static constexpr int kOffRawV = kOffRawK + (kStageK ? KT * 256 : 0);
  static constexpr int kSmem = kOffRawV + KT * 256 + 1024 /*align slack*/;
  static constexpr uint32_t kTmemCols = 4 * KT;  // the score levels; P and O_tile reuse them
  static constexpr int kTmemPh = 0;              // P hi (after the scores are consumed)
  static constexpr int kTmemPl = KT;             // P lo
  static constexpr int kTmemO = 2 * KT;          // O_tile (64 columns)
  static constexpr int kMinBlocks = KT == 64 ? 2 : 3;
  static_assert(kTmemO + 64 <= (int)kTmemCols, "TMEM layout");
  static_assert(kMinBlocks * kSmem <= 227 * 1024, "CTAs per SM");
  static_assert(kSC % 16 == 0 && kOC % 16 == 0, "16-column TMEM accesses");
  // every staging map covers exactly the tile: K rows (16 threads per row),
  // V^T (64 threads per key group), the mask (one thread per key)
  static_assert(kKLoads * kThreads == KT * 16 && kKLoads >= 1, "K staging covers the tile");
  static_assert(kVKeys * kThreads == KT * 64 && kVKeys % 4 == 0, "V staging covers the tile");
  static_assert(kThreads >= KT && kThreads % 64 == 0, "mask / V thread maps");
};

// The value of x, hidden from the optimiser (no hoisting of what depends on it).
__device__ __forceinline__ uint32_t opaque_u32(uint32_t x) {
  asm volatile("mov.b32 %0, %0;" : "+r"(x));
  return x;
}

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

template <int KT, int NW, bool C_POW2>
__global__ void __launch_bounds__(32 * NW, (KT == 64 ? 2 : 3))
    attention_tc_kernel(const float* __restrict__ q, const float* __restrict__ k,
                        const float* __restrict__ v, int ld, float* __restrict__ out, int H, int S,
                        int nh, float c, const float* __restrict__ mask, int mask_per_batch,
                        float2* __restrict__ minmax) {
  using A = AttTc<KT, NW>;
  extern __shared__ __align__(1024) uint8_t att_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(att_raw) + 1023) & ~uintptr_t(1023));
  float* red_max = reinterpret_cast<float*>(sm + A::kOffRed);
  float* red_sum = red_max + A::kWPQ * kTcQ;
  float* q_scale = reinterpret_cast<float*>(sm + A::kOffScale);
  float* k_scale = q_scale + kTcQ;
  float* m_tile = reinterpret_cast<float*>(sm + A::kOffMask);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + A::kOffBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_s + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cg = warp >> 2;
  const int row = quad * 32 + lane;  // query row within the tile = TMEM lane
  const int scol0 = cg * A::kSC;     // first score column of this thread
  const int ocol0 = cg * A::kOC;     // first context column of this thread
  const int bh = blockIdx.y;
  const int b = bh / nh, h = bh % nh;
  const int q0 = blockIdx.x * kTcQ;
  const size_t head = (size_t)b * S * ld + (size_t)h * kAttDh;
  const float* mrow = mask ? mask + (mask_per_batch ? (size_t)b * S : 0) : nullptr;
  const float inv_c = 1.0f / c;  // exact when c is a power of two (C_POW2)
  // Q / K rows: 16 threads per 256-byte row; V: thread = column d (tid % 64)
  // of kVKeys consecutive keys (key group tid / 64), stored as row d of V^T
  const int kv_row = tid >> 4, kv_col = (tid & 15) * 4;
  constexpr int kRowStep = A::kThreads / 16;  // rows between a thread's Q / K loads
  const int v_d = tid & 63, v_key = (tid >> 6) * A::kVKeys;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, A::kTmemCols);
    tmem_relinquish();
  }
  // barrier init and TMEM allocation overlap the previous kernel; q / k / v
  // (its outputs) are read only from here on
  pdl_wait();
  pdl_trigger();
  float4 nk[A::kStageK ? 1 : A::kKLoads];  // next K tile (when not staged in shared memory)
  float nm = 0.0f;  // the tile's additive mask value for key tid (tid < KT)
  float* raw_k = reinterpret_cast<float*>(sm + A::kOffRawK);
  float* raw_v = reinterpret_cast<float*>(sm + A::kOffRawV);
  auto load_k = [&](int k0) {
#pragma unroll
    for (int i = 0; i < A::kKLoads; ++i) {
      const int kr = k0 + kv_row + kRowStep * i;
      nk[i] = kr < S ? __ldg(reinterpret_cast<const float4*>(k + head + (size_t)kr * ld + kv_col))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  // cp.async of the tile's V (and K when staged) rows into the raw buffers,
  // rows past S zero-filled; the mask value of key tid into nm
  auto stage_tile = [&](int k0) {
#pragma unroll
    for (int i = 0; i < A::kKLoads; ++i) {
      const int r = kv_row + kRowStep * i, kr = k0 + r;
      const size_t src = head + (size_t)(kr < S ? kr : 0) * ld + kv_col;
      if (A::kStageK) cp_async16(raw_k + r * 64 + kv_col, k + src, kr < S);
      cp_async16(raw_v + r * 64 + kv_col, v + src, kr < S);
    }
    cp_async_commit();
    if (tid < KT) {
      const int key = k0 + tid;
      nm = key >= S ? -INFINITY : (mrow ? __ldg(mrow + key) : 0.0f);
    }
  };
  {
    float4 vq[A::kQLoads];
#pragma unroll
    for (int i = 0; i < A::kQLoads; ++i) {
      const int r = kv_row + kRowStep * i, qi = q0 + r;
      vq[i] = qi < S ? __ldg(reinterpret_cast<const float4*>(q + head + (size_t)qi * ld + kv_col))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (!A::kStageK) load_k(0);
    stage_tile(0);
#pragma unroll
    for (int i = 0; i < A::kQLoads; ++i) {
      const int r = kv_row + kRowStep * i;
      const float f = slice_row_store(sm + A::kOffQs, kQAtom, r, kv_col, vq[i]);
      if (kv_col == 0) q_scale[r] = f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tslot;
  const uint32_t t_lane = tmem_base + ((uint32_t)(quad * 32) << 16);  // this warp's lanes
  constexpr uint32_t idesc_o = idesc_tf32(kTcQ, kAttDh, false);
  const uint32_t a_sm = smem_addr(sm);
  const float qsc = q_scale[row];
  const float qf = __fmul_rn(qsc, inv_c);  // a power of two when c is

  float m_run = -INFINITY, l_part = 0.0f, o[A::kOC];
#pragma unroll
  for (int d = 0; d < A::kOC; ++d) o[d] = 0.0f;
  bool ok = true;
  uint32_t phase = 0;
  for (int k0 = 0; k0 < S; k0 += KT, phase ^= 1) {
    // 1. K slices, V^T hi / lo and the mask of this tile (the staged rows
    // of every thread are visible after the wait and the barrier)
    cp_async_wait_all();
    __syncthreads();
#pragma unroll
    for (int i = 0; i < A::kKLoads; ++i) {
      const int r = kv_row + kRowStep * i;
      const float4 kx = A::kStageK ? *reinterpret_cast<const float4*>(raw_k + r * 64 + kv_col) : nk[i];
      const float f = slice_row_store(sm + A::kOffKs, A::kKAtom, r, kv_col, kx);
      if (kv_col == 0) k_scale[r] = f;
    }
#pragma unroll
    for (int g = 0; g < A::kVKeys / 4; ++g) {
      const int key = v_key + 4 * g;
      const float4 vx = make_float4(raw_v[key * 64 + v_d], raw_v[(key + 1) * 64 + v_d],
                                    raw_v[(key + 2) * 64 + v_d], raw_v[(key + 3) * 64 + v_d]);
      split_store(sm + A::kOffVh, sm + A::kOffVl, A::kVAtom, v_d, key, vx);
    }
    if (tid < KT) m_tile[tid] = nm;
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    // 2. S = Q K^T, exact per level; V^T of this tile meanwhile
    if (tid == 0) {
      tc_fence_after();
      // the operand addresses are made opaque here so the compiler does not
      // hoist 40 loop-invariant descriptors into registers for the whole loop
      const uint32_t a_qs = opaque_u32(a_sm + A::kOffQs), a_ks = opaque_u32(a_sm + A::kOffKs);
#pragma unroll
      for (int L = 0; L < 4; ++L) {
#pragma unroll
        for (int i = 0; i <= L; ++i) {
          const int j = L - i;
#pragma unroll
          for (int hd = 0; hd < 2; ++hd) {
            // slice i of Q / slice j of K, d half hd (32 bytes each); the
            // most significant slice is signed, the others unsigned
            const uint32_t ao = (i >> 1) * kQAtom + (i & 1) * 64 + hd * 32;
            const uint32_t bo = (j >> 1) * A::kKAtom + (j & 1) * 64 + hd * 32;
            mma_i8(tmem_base + (uint32_t)(L * KT), smem_desc_k128(a_qs + ao),
                   smem_desc_k128(a_ks + bo), idesc_i8(kTcQ, KT, i == 0, j == 0), (i | hd) != 0);
          }
        }
      }
      mma_commit(bar_s);
    }
    // the raw buffers were consumed before the barrier: the next tile's rows
    // stream in while this tile's scores and softmax run
    if (k0 + KT < S) stage_tile(k0 + KT);
    ok = mbar_wait_warp(bar_s, phase, ICX_DEVICE_TIMEOUT_EPILOGUE);
    tc_fence_after();
    // 3. scores: (((acc3 / 2^24 + acc2 / 2^16) + acc1 / 2^8) + acc0), one
    // rounding per step, then 2^(nq-1) 2^(nk-1), Div(c), Add(mask)
    float pmax = -INFINITY;
#pragma unroll
    for (int hcol = 0; hcol < A::kSC; hcol += 16) {
      const uint32_t t = t_lane + (uint32_t)(scol0 + hcol);
      float f[16];
      uint32_t sc[16];
      // one level at a time (16 registers in flight)
#pragma unroll
      for (int L = 3; L >= 0; --L) {
        uint32_t r[16];
        if (ok) {
          tmem_ld_32x32b_x16(t + (uint32_t)(L * KT), r);
          tmem_ld_wait_regs16(r);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float a = (float)(int32_t)r[j];
          f[j] = L == 3 ? __fmul_rn(a, 5.9604644775390625e-08f)
               : L == 2 ? __fmaf_rn(a, 1.52587890625e-05f, f[j])
               : L == 1 ? __fmaf_rn(a, 0.00390625f, f[j])
                        : __fadd_rn(a, f[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float g = f[j];
        const int jj = scol0 + hcol + j;
        float t2 = C_POW2 ? __fmul_rn(__fmul_rn(g, qf), k_scale[jj])  // exact: powers of two
                          : __fdiv_rn(__fmul_rn(__fmul_rn(g, qsc), k_scale[jj]), c);
        t2 = __fadd_rn(t2, m_tile[jj]);  // -inf past S
        sc[j] = __float_as_uint(t2);
        pmax = fmaxf(pmax, t2);
      }
      // park the scores in their (consumed) level-0 columns until the row max
      // is known
      tmem_st_32x32b_x16(t, sc);
    }
    tmem_st_wait();
    float tmax = pmax;
    if (A::kWPQ > 1) {
      // the row max over the warps sharing the row; also: every score
      // column has been read before any P overwrites it
      red_max[cg * kTcQ + row] = pmax;
      tc_fence_before();
      ok = __syncthreads_and(ok) != 0;
      if (!ok) break;
      tc_fence_after();
      tmax = red_max[row];
#pragma unroll
      for (int w = 1; w < A::kWPQ; ++w) tmax = fmaxf(tmax, red_max[w * kTcQ + row]);
    }
    // online softmax: exp(a - m) = 2^(a*log2e - m*log2e)
    const float m_new = fmaxf(m_run, tmax);
    const float ml = m_new == -INFINITY ? 0.0f : m_new * kLog2e;  // a fully masked row stays 0
    const float alpha = m_run == -INFINITY ? 0.0f : ex2f(fmaf(m_run, kLog2e, -ml));
    float rsum = 0.0f;
#pragma unroll
    for (int hcol = 0; hcol < A::kSC; hcol += 16) {
      uint32_t hi[16], lo[16], sc[16];
      tmem_ld_32x32b_x16(t_lane + (uint32_t)(scol0 + hcol), sc);
      tmem_ld_wait_regs16(sc);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float e = ex2f(fmaf(__uint_as_float(sc[j]), kLog2e, -ml));  // 2^-inf = 0 for masked keys
        rsum += e;
        const float eh = tf32_round(e);
        hi[j] = __float_as_uint(eh);
        lo[j] = __float_as_uint(tf32_round(__fsub_rn(e, eh)));
      }
      tmem_st_32x32b_x16(t_lane + (uint32_t)(A::kTmemPh + scol0 + hcol), hi);
      tmem_st_32x32b_x16(t_lane + (uint32_t)(A::kTmemPl + scol0 + hcol), lo);
    }
    l_part = l_part * alpha + rsum;
    m_run = m_new;
    tmem_st_wait();
    fence_proxy_async_smem();  // V^T stores -> the MMA
    tc_fence_before();
    __syncthreads();
    // 4. O_tile = P V; the next K tile meanwhile
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a_v_h = opaque_u32(a_sm + A::kOffVh), a_v_l = opaque_u32(a_sm + A::kOffVl);
#pragma unroll
      for (int j = 0; j < KT / 8; ++j) {
        // k-step j = keys 8j..8j+7: P columns 8j.., V^T column block j/4
        const uint32_t bo = (j >> 2) * A::kVAtom + (j & 3) * 32;
        const uint64_t vh = smem_desc_k128(a_v_h + bo), vl = smem_desc_k128(a_v_l + bo);
        const uint32_t ph = tmem_base + (uint32_t)(A::kTmemPh + 8 * j);
        const uint32_t pl = tmem_base + (uint32_t)(A::kTmemPl + 8 * j);
        mma_tf32_ts(tmem_base + A::kTmemO, ph, vh, idesc_o, j > 0);
        mma_tf32_ts(tmem_base + A::kTmemO, ph, vl, idesc_o, true);
        mma_tf32_ts(tmem_base + A::kTmemO, pl, vh, idesc_o, true);
      }
      mma_commit(bar_o);
    }
    if (!A::kStageK && k0 + KT < S) load_k(k0 + KT);
    ok = mbar_wait_warp(bar_o, phase, ICX_DEVICE_TIMEOUT_EPILOGUE);
    tc_fence_after();
    if (ok) {
#pragma unroll
      for (int hcol = 0; hcol < A::kOC; hcol += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_lane + (uint32_t)(A::kTmemO + ocol0 + hcol), r);
        tmem_ld_wait_regs16(r);
#pragma unroll
        for (int d = 0; d < 16; ++d) o[hcol + d] = fmaf(o[hcol + d], alpha, __uint_as_float(r[d]));
      }
    }
    // TMEM reads of this tile are done before the next tile's MMAs overwrite
    tc_fence_before();
  }
  cp_async_wait_all();  // nothing in flight into shared memory at exit (early break)
  red_sum[cg * kTcQ + row] = l_part;
  ok = __syncthreads_and(ok) != 0;
  const int qi = q0 + row;
  float mn = 0.0f, mx = 0.0f;  // (min, max) of what this CTA writes, seeded like DynamicQuantizeLinear
  if (ok && qi < S) {
    float l = red_sum[row];
#pragma unroll
    for (int w = 1; w < A::kWPQ; ++w) l += red_sum[w * kTcQ + row];
    const float inv = 1.0f / l;
    float4* orow = reinterpret_cast<float4*>(out + ((size_t)b * S + qi) * H + (size_t)h * kAttDh + ocol0);
#pragma unroll
    for (int d = 0; d < A::kOC; d += 4) {
      const float4 w = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
      orow[d / 4] = w;
      mn = fminf(fminf(mn, fminf(w.x, w.y)), fminf(w.z, w.w));
      mx = fmaxf(fmaxf(mx, fmaxf(w.x, w.y)), fmaxf(w.z, w.w));
    }
  }
  if (minmax != nullptr) {
    // one partial per CTA for the DynamicQuantizeLinear that reads `out`
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    if (lane == 0) {
      red_max[warp] = mn;  // the row max / sum areas are free now
      red_max[16 + warp] = mx;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < A::kThreads / 32; ++w) {
        mn = fminf(mn, red_max[w]);
        mx = fmaxf(mx, red_max[16 + w]);
      }
      minmax[blockIdx.y * gridDim.x + blockIdx.x] = make_float2(mn, mx);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, A::kTmemCols);
  }
}

bool attention_supported(int64_t dh, int64_t ld, int64_t H) {
  return dh == kAttDh && ld % 4 == 0 && H % 4 == 0;
}

int attention_partials(int64_t B, int64_t S, int64_t nh) {
  return (int)(((S + kTcQ - 1) / kTcQ) * B * nh);
}

int launch_attention_f32(cudaStream_t s, const float* q, const float* k, const float* v, int64_t ld,
                         float* out, int64_t B, int64_t S, int64_t H, int64_t nh, float c,
                         const float* mask, bool mask_per_batch, float* minmax, int* n_minmax) {
  ICX_REQUIRE(attention_supported(H / nh, ld, H), "Attention: head size %lld unsupported",
              (long long)(H / nh));
  ICX_REQUIRE((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) == 0,
              "Attention: q/k/v/out must be 16-byte aligned");
  if (B == 0 || S == 0 || nh == 0) {
    if (n_minmax) *n_minmax = 0;
    return ICX_OK;
  }
  static const bool simt = [] {
    const char* e = getenv("ICONNX_ATTENTION");
    return e != nullptr && strcmp(e, "simt") == 0;
  }();
  if (!simt) {
    ICX_REQUIRE(B * nh <= 65535, "Attention: batch x heads %lld too large", (long long)(B * nh));
    const int parts = attention_partials(B, S, nh);
    int cexp;
    const bool c_pow2 = frexpf(c, &cexp) == 0.5f;
    // <32, 4> (three CTAs per SM) wins while the key loop is short; from
    // S > 256 on the <64, 8> tiling halves the per-key-tile overhead and is
    // faster (measured: S = 128 -> <32, 4>, S = 512 -> <64, 8>).
    // ICONNX_ATTENTION_TILE=32 or =64 forces one of them.
    static const int forced = [] {
      const char* e = getenv("ICONNX_ATTENTION_TILE");
      return e == nullptr ? 0 : atoi(e);
    }();
    const bool wide = forced == 64 || (forced != 32 && S > 256);
    dim3 grid((unsigned)((S + kTcQ - 1) / kTcQ), (unsigned)(B * nh));
    auto launch = [&](auto kern, int threads, int smem) -> int {
      ICX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      launch_pdl(kern, grid, dim3(threads), smem, s, q, k, v, (int)ld, out, (int)H, (int)S, (int)nh,
                 c, mask, mask_per_batch ? 1 : 0, reinterpret_cast<float2*>(minmax));
      return ICX_OK;
    };
    int rc;
    if (wide)
      rc = c_pow2 ? launch(attention_tc_kernel<64, 8, true>, 256, AttTc<64, 8>::kSmem)
                  : launch(attention_tc_kernel<64, 8, false>, 256, AttTc<64, 8>::kSmem);
    else
      rc = c_pow2 ? launch(attention_tc_kernel<32, 4, true>, 128, AttTc<32, 4>::kSmem)
                  : launch(attention_tc_kernel<32, 4, false>, 128, AttTc<32, 4>::kSmem);
    if (rc) return rc;
    ICX_LAUNCH_CHECK();
    if (n_minmax) *n_minmax = parts;
    return ICX_OK;
  }
  const int smem = 4 * kAttTile * kAttPad * (int)sizeof(float);
  ICX_CUDA(cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid((unsigned)(B * nh), (unsigned)((S + kAttTile - 1) / kAttTile));
  launch_pdl(attention_f32_kernel, dim3(grid), dim3(kAttThreads), smem, s, q, k, v, (int)ld, out, (int)H, (int)S, (int)nh,
                                                       c, mask, mask_per_batch ? 1 : 0);
  ICX_LAUNCH_CHECK();
  if (minmax != nullptr) {
    // the CUDA-core kernel has no fused (min, max): one separate pass
    const size_t n = (size_t)(B * S * H);
    const int rc = launch_dql_minmax(s, out, n, reinterpret_cast<float2*>(minmax));
    if (rc) return rc;
    if (n_minmax) *n_minmax = dql_minmax_partials(n);
  }
  return ICX_OK;
}

}  // namespace icx
