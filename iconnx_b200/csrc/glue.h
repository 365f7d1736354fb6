// Internal launch helpers shared by the engine (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "../../include/iconnx_b200.h"

namespace icx {

constexpr int kMaxRank = 6;
enum BinaryOp { kAdd = 0, kSub = 1, kMul = 2, kDiv = 3 };

size_t dtype_size(int t);

int launch_gather_rows(cudaStream_t s, const void* table, int elem_bytes, int64_t rows,
                       const int64_t* idx, size_t n, size_t D, void* out, int* err);
int launch_binary(cudaStream_t s, int op, const float* a, const std::vector<int64_t>& ashape,
                  const float* b, const std::vector<int64_t>& bshape, float* out,
                  const std::vector<int64_t>& oshape);
int layernorm_partials(size_t rows);
// Whether icx_quant_linear_layernorm runs for this K and N on the current
// device (qgemm.cu).
bool quant_linear_ln_supported(size_t K, size_t N);
// ... and whether the engine prefers it to the unfused GEMM + LayerNorm
// (where every 128-row block gets a cluster of its own).
bool quant_linear_ln_preferred(size_t M, size_t K, size_t N);

int launch_layernorm(cudaStream_t s, const float* x, const float* gamma, const float* beta,
                     float* y, size_t rows, size_t D, float eps, float* minmax, int* n_minmax);
int launch_scale_mask_softmax(cudaStream_t s, const float* x, float* y, size_t rows, size_t D,
                              float c, const float* mask, size_t rows_per_batch);
int launch_softmax(cudaStream_t s, const float* x, float* y, size_t rows, size_t D);
int launch_transpose(cudaStream_t s, const void* x, int elem_bytes,
                     const std::vector<int64_t>& in_shape, const std::vector<int64_t>& perm,
                     void* y);
int launch_cast(cudaStream_t s, const void* x, int from, void* y, int to, size_t n);
int launch_erf(cudaStream_t s, const float* x, float* y, size_t n);
int launch_gelu(cudaStream_t s, const float* x, float* y, size_t n);

// attention.cu
bool attention_supported(int64_t dh, int64_t ld, int64_t H);
// (min, max) partials of the output for the DynamicQuantizeLinear that
// reads it when `minmax` is given (attention_partials of them; the buffer
// must hold that many pairs, which may exceed ICX_MAX_MINMAX_PARTIALS).
int attention_partials(int64_t B, int64_t S, int64_t nh);
int launch_attention_f32(cudaStream_t s, const float* q, const float* k, const float* v, int64_t ld,
                         float* out, int64_t B, int64_t S, int64_t H, int64_t nh, float c,
                         const float* mask, bool mask_per_batch, float* minmax, int* n_minmax);

// dql.cu
int dql_minmax_partials(size_t n);
int launch_dql_minmax(cudaStream_t s, const float* x, size_t n, float2* partials);
// global DQL: n (min, max) partials -> g = (-min, max); g -> one (min, max) partial
int launch_minmax_fold(cudaStream_t s, const float* partials, int n, float* g);
int launch_minmax_unfold(cudaStream_t s, const float* g, float* out);

}  // namespace icx
