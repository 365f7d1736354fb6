/*
 * iconnx_b200 — C ABI of the B200 (sm_100a) int8 dynamic-quantization path.
 *
 * The path is the ONNX Runtime style chain every int8 Linear layer lowers to:
 *   DynamicQuantizeLinear -> MatMulInteger -> Cast -> Mul(scale) -> Add(bias)
 *   [-> erf-GELU]
 * Each entry point below replaces one interface of the reference engine
 * (iconnx, a Rust crate); the citation names the file:line it replaces.
 *
 * Conventions
 *   - Every function returns an int status: ICX_OK (0) or a negative
 *     ICX_ERR_* code.  icx_last_error() returns a thread-local message for the
 *     most recent failure on the calling thread.  No entry point aborts,
 *     panics or traps; invalid arguments are rejected before any launch
 *     (mirrors CudaError::Kernel in src/cuda/context.rs:295-325).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  All work is enqueued asynchronously on it.
 *   - Pointers named d_* are device pointers owned by the caller.  The
 *     kernel entry points never allocate; scratch space is passed in as a
 *     caller-owned workspace whose size a *_workspace_bytes query returns.
 *   - Matrices are row-major and contiguous.
 *   - Element type codes: ICX_U8, ICX_S8, ICX_S32, ICX_F32.
 */
#ifndef ICONNX_B200_H
#define ICONNX_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ICX_API __attribute__((visibility("default")))
#else
#define ICX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define ICX_OK 0
#define ICX_ERR_INVALID (-1)     /* bad argument: dtype, rank, shape, null */
#define ICX_ERR_CUDA (-2)        /* a CUDA runtime/driver call failed       */
#define ICX_ERR_UNSUPPORTED (-3) /* valid ONNX, not supported by this path  */
#define ICX_ERR_WORKSPACE (-4)   /* workspace too small                     */
#define ICX_ERR_SHAPE_MISMATCH (-5) /* input shape differs from the plan    */
#define ICX_ERR_NOT_FOUND (-6)   /* unknown tensor / output name            */

/* device-side status values (icx_device_status) */
#define ICX_DEVICE_TIMEOUT_PRODUCER 0x101
#define ICX_DEVICE_TIMEOUT_MMA 0x102
#define ICX_DEVICE_TIMEOUT_EPILOGUE 0x103
#define ICX_DEVICE_TIMEOUT_SELFTEST 0x1ff

/* Upper bound on the (min, max) partial pairs a producer writes for a
 * following DynamicQuantizeLinear (icx_quant_linear d_minmax, and the
 * partials icx_dql_quantize_f32_u8 consumes). */
#define ICX_MAX_MINMAX_PARTIALS 1184

/* ---- element types ----------------------------------------------------- */
#define ICX_U8 0
#define ICX_S8 1
#define ICX_S32 2
#define ICX_F32 3
#define ICX_S64 4
#define ICX_BOOL 5

/* Message for the last failing call on this thread ("" if none). */
ICX_API const char* icx_last_error(void);

/* Library version string. */
ICX_API const char* icx_version(void);

/* Reads and clears the device-side status word of `device` (0 = no kernel
 * gave up on a bounded wait since the last call). */
ICX_API int icx_device_status(int device, int* status_out);

/* Self-test of the kernels' failure handling (no reference counterpart; the
 * reference's kernels have no bounded waits): enqueues one tiny kernel whose
 * bounded mbarrier wait can never complete, with a limit of limit_ns
 * (0 < limit_ns <= 100 ms) instead of the kernels' 2 s.  The wait gives up,
 * records ICX_DEVICE_TIMEOUT_SELFTEST for icx_device_status and the kernel
 * returns, leaving the context usable; no fault, trap or hang. */
ICX_API int icx_selftest_bounded_wait(void* stream, uint64_t limit_ns);

/* ======================================================================== *
 * DynamicQuantizeLinear
 * Replaces gpu_dynamic_quantize_linear (src/cuda/ops/quantize.rs:296-377),
 * which the reference runs on the host, and follows the CPU forward
 * (src/operators/dynamic_quantize_linear.rs:32-112) bit for bit:
 *   min/max over x and 0 (NaN skipped), scale = (max-min)/255 in f64,
 *   zp = clamp(rte(0 - min/scale)), y = clamp(rte(x/scale) + zp) in f64,
 *   min == max -> scale 0, zp 0, y 0.
 * Outputs: d_y u8[n], d_scale f32[1], d_zp u8[1].
 * Optional side output: d_rowsum s32[n/row_len] = per-row sum of y, used by
 * the per-column weight zero-point correction of the GEMM (pass NULL to
 * skip; row_len must divide n when it is given).
 * ======================================================================== */
ICX_API size_t icx_dql_workspace_bytes(size_t n);

ICX_API int icx_dql_f32_u8(void* stream, const float* d_x, size_t n, uint8_t* d_y,
                   float* d_scale, uint8_t* d_zp, int32_t* d_rowsum,
                   size_t row_len, void* d_workspace, size_t workspace_bytes);

/* Allocation-free DynamicQuantizeLinear.  No counterpart in the reference
 * engine.  For callers that must not allocate device memory while they run
 * (a fixed memory budget reserved at start-up, an allocator that may not be
 * re-entered from the calling thread, or a host that forbids cudaMalloc
 * because it can synchronise the device): same inputs, outputs and bit-exact
 * results as icx_dql_f32_u8, but the scratch lives in a 9472-byte array
 * compiled into this library (resident on each GPU that loads it until the
 * process exits) instead of a caller workspace.  Calls no allocator.
 * Limit: each of the array's ICX_MAX_MINMAX_PARTIALS (min, max) pairs
 * summarises at most 2^17 elements, so n <= ICX_DQL_NOALLOC_MAX_N
 * (155,189,248 elements); larger n is rejected with ICX_ERR_INVALID before
 * any launch.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and caches it for the process: make that
 * first call before any stream capture, and do not use this entry point
 * after cudaDeviceReset.  All calls on a device share the array: calls whose
 * kernels may overlap on the GPU (e.g. unordered streams) race and must be
 * serialised by the caller. */
#define ICX_DQL_NOALLOC_MAX_N (1184ull << 17)
ICX_API int icx_dql_f32_u8_noalloc(void* stream, const float* d_x, size_t n,
                                   uint8_t* d_y, float* d_scale, uint8_t* d_zp,
                                   int32_t* d_rowsum, size_t row_len);

/* The quantise pass of DynamicQuantizeLinear alone, for an x whose producer
 * already wrote (min, max) partials of x (d_minmax: n_minmax float pairs,
 * each seeded with 0 and NaN-skipping, e.g. icx_quant_linear's d_minmax).
 * Same outputs and bit-exact results as icx_dql_f32_u8; saves one full read
 * of x.  Replaces the same reference function as icx_dql_f32_u8. */
ICX_API int icx_dql_quantize_f32_u8(void* stream, const float* d_x, size_t n,
                                    const float* d_minmax, int n_minmax,
                                    uint8_t* d_y, float* d_scale, uint8_t* d_zp,
                                    int32_t* d_rowsum, size_t row_len);

/* ======================================================================== *
 * Weight preparation for MatMulInteger.
 * Transposes b [K, N] (u8 or s8) into the tensor-core operand layout
 * bt [N, K] and writes colsum[n] = sum_k b[k, n] (as the element type's
 * integer value).  Done once per weight at plan build time; the per-op
 * MatMulInteger entry point calls it on its workspace.
 * ======================================================================== */
ICX_API int icx_prepare_b(void* stream, const void* d_b, int b_type, size_t K,
                  size_t N, void* d_bt, int32_t* d_colsum);

/* ======================================================================== *
 * MatMulInteger, int32 output.
 * Replaces gpu_matmul_integer (src/cuda/ops/quantize.rs:398-615) and its
 * kernels matmul_integer_{u8s8,s8s8,s8u8,u8u8}_kernel
 * (src/cuda/ops/quantize_kernels.rs:116-194):
 *   out[m, n] = sum_k (a[m,k] - a_zp) * (b[k,n] - b_zp[n])   (wrapping s32)
 * a: [M, K] (u8 or s8); b: [K, N] (u8 or s8) row-major as in ONNX.
 * d_a_zp: NULL or one element of a's type; d_b_zp: NULL, one element, or
 * N elements (b_zp_per_col != 0; the ONNX per-column form the reference
 * rejects in src/cuda/ops/quantize.rs:625-658).  Zero points stay on the
 * device (no host round trip, unlike resolve_scalar_zp :625-679).
 * Uses workspace for the transposed b, its column sums and row sums of a.
 * ======================================================================== */
ICX_API size_t icx_matmul_integer_workspace_bytes(size_t M, size_t K, size_t N);

ICX_API int icx_matmul_integer(void* stream, const void* d_a, int a_type,
                       const void* d_b, int b_type, size_t M, size_t K,
                       size_t N, const void* d_a_zp, const void* d_b_zp,
                       int b_zp_per_col, int32_t* d_out, void* d_workspace,
                       size_t workspace_bytes);

/* Same GEMM on an already prepared weight (bt [N, K] + colsum from
 * icx_prepare_b).  d_rowsum_a (s32[M]) is required when d_b_zp != NULL. */
ICX_API int icx_matmul_integer_prepared(void* stream, const void* d_a, int a_type,
                                const void* d_bt, int b_type,
                                const int32_t* d_colsum, size_t M, size_t K,
                                size_t N, const void* d_a_zp,
                                const void* d_b_zp, int b_zp_per_col,
                                const int32_t* d_rowsum_a, int32_t* d_out);

/* ======================================================================== *
 * Fused quantized Linear: MatMulInteger -> Cast -> Mul -> Add [-> GELU].
 * Replaces the per-op chain the reference executes for one int8 Linear
 * (src/cuda/executor/layout.rs:1034-1097 MatMulInteger, layout.rs:144 Cast,
 * src/cuda/executor/elementwise.rs:123 Mul and :54 Add with their
 * gpu_expand broadcasts, src/cuda/kernels/mod.rs:246 erf_kernel for GELU):
 *   acc   = sum_k (q[m,k] - a_zp) * (w[k,n] - b_zp[n])          (s32)
 *   s[n]  = f32(a_scale) * w_scale[n]                             (one f32 mul)
 *   out   = f32(acc) * s[n] + bias[n]                             (no FMA)
 *   gelu: out = (out * (1 + erf(out / sqrt2))) * 0.5
 * q: u8 [M, K] from DynamicQuantizeLinear; a_scale/a_zp: its device
 * outputs; wt/colsum: prepared weight; w_scale: 1 or N floats; b_zp: NULL,
 * 1 or N s8 values; bias: N floats (or NULL); out: f32 [M, N].
 * The s32 accumulator never leaves the SM: it lives in tensor memory.
 * d_residual (nullable, f32 [M, N], not with gelu): a following residual
 * Add(out, residual) is applied in the epilogue, rounded separately.
 * d_minmax (nullable, room for ICX_MAX_MINMAX_PARTIALS float pairs): the
 * kernel also writes (min, max) partials of `out` (seeded with 0, NaN
 * skipped) so a following DynamicQuantizeLinear needs only its quantise
 * pass; *n_minmax receives how many pairs were written.
 * ======================================================================== */
ICX_API int icx_quant_linear(void* stream, const uint8_t* d_q, const float* d_a_scale,
                     const uint8_t* d_a_zp, const int32_t* d_rowsum_q,
                     const int8_t* d_wt, const int32_t* d_colsum, size_t M,
                     size_t K, size_t N, const float* d_w_scale,
                     int w_scale_per_col, const int8_t* d_b_zp,
                     int b_zp_per_col, const float* d_bias, int gelu,
                     const float* d_residual, float* d_out, float* d_minmax,
                     int* n_minmax);

/* ======================================================================== *
 * QuantLinear + residual Add + LayerNormalization in one launch:
 *   z = (Cast(MatMulInteger(q, W, a_zp, b_zp)) * (a_scale * w_scale) + bias)
 *       + residual                                  (as icx_quant_linear)
 *   out = LayerNormalization(z, gamma, beta, epsilon) over the last axis
 * Replaces the reference's MatMulInteger -> Cast -> Mul -> Add -> Add ->
 * LayerNormalization chain of one transformer sub-block
 * (src/operators/layer_normalization.rs:25-80 for the last step; the
 * normalisation sums in a different order, fp32 rounding).  z is never
 * written.  N must be 192 x 2..4 and K a multiple of 16 (else
 * ICX_ERR_INVALID); all operands 16-byte aligned.  d_minmax receives one
 * (min, max) pair of `out` per CTA (*n_minmax of them), like
 * icx_quant_linear.
 * ======================================================================== */
ICX_API int icx_quant_linear_layernorm(void* stream, const uint8_t* d_q, const float* d_a_scale,
                                       const uint8_t* d_a_zp, const int32_t* d_rowsum_q,
                                       const int8_t* d_wt, const int32_t* d_colsum, size_t M,
                                       size_t K, size_t N, const float* d_w_scale,
                                       int w_scale_per_col, const int8_t* d_b_zp, int b_zp_per_col,
                                       const float* d_bias, const float* d_residual,
                                       const float* d_gamma, const float* d_beta, float epsilon,
                                       float* d_out, float* d_minmax, int* n_minmax);

/* ======================================================================== *
 * DequantizeLinear: y = (f32(x) - f32(zp)) * scale, per tensor or per axis.
 * Replaces gpu_dequantize_linear (src/cuda/ops/quantize.rs:24-267) and
 * dequantize_linear_{i8,u8,i32}_kernel (src/cuda/ops/quantize_kernels.rs:
 * 52-81); arithmetic follows the CPU forward
 * (src/operators/dequantize_linear.rs:32-179).
 * The tensor is viewed as [outer, axis_len, inner]; scale/zp have
 * scale_len elements (1 = per tensor, axis_len = per axis).
 * ======================================================================== */
ICX_API int icx_dequantize_linear(void* stream, const void* d_x, int x_type,
                          size_t outer, size_t axis_len, size_t inner,
                          const float* d_scale, size_t scale_len,
                          const void* d_zp, float* d_y);

/* Row sums of an 8-bit matrix a [M, K] (the rowsum_a operand of
 * icx_matmul_integer_prepared when b has a zero point).  Part of the
 * MatMulInteger path replacing src/cuda/ops/quantize.rs:398-615. */
ICX_API int icx_matmul_integer_rowsum(void* stream, const void* d_a, int a_type, size_t M,
                                      size_t K, int32_t* d_rowsum);

/* ======================================================================== *
 * Graph executor.  Replaces GpuGraphExecutor (src/cuda/inference/mod.rs:
 * 222-659): new (:222), add_input (:306), add_initializer (:316),
 * add_node (:330), run (:428, host tensors in and out), with lazy lowering
 * on the first run (:484-536) and the input-shape guard (:441-460, error
 * ICX_ERR_SHAPE_MISMATCH).  Lowering fuses every
 * DynamicQuantizeLinear -> MatMulInteger -> Cast -> Mul -> Add [-> GELU]
 * chain into one tensor-core kernel.  One executor per thread (the
 * reference's is !Sync); each owns a CUDA stream on `device`.
 * Element types of inputs/initializers: ICX_* codes; dims are int64.
 * ======================================================================== */
typedef struct icx_engine icx_engine;

/* Node attribute: kind 1 int (i), 2 float (f), 3 ints (ints[n]),
 * 4 string (s), 5 floats (floats[n]). */
typedef struct icx_attr {
  const char* name;
  int kind;
  int64_t i;
  float f;
  const int64_t* ints;
  const float* floats;
  int n;
  const char* s;
} icx_attr;

ICX_API icx_engine* icx_engine_create(int device);  /* NULL on failure */
ICX_API void icx_engine_destroy(icx_engine* e);
ICX_API int icx_engine_add_input(icx_engine* e, const char* name, int dtype, int rank,
                                 const int64_t* dims);  /* dims <= 0: dynamic */
ICX_API int icx_engine_add_initializer(icx_engine* e, const char* name, int dtype, int rank,
                                       const int64_t* dims, const void* host_data);
ICX_API int icx_engine_add_node(icx_engine* e, const char* name, const char* op_type, int n_in,
                                const char* const* inputs, int n_out,
                                const char* const* outputs, int n_attrs, const icx_attr* attrs);
/* Runs the graph on host inputs (dims concatenated over inputs); the
 * requested outputs stay on the device until icx_engine_output_copy. */
ICX_API int icx_engine_run(icx_engine* e, int n_in, const char* const* names, const int* dtypes,
                           const int* ranks, const int64_t* dims, const void* const* host,
                           int n_out, const char* const* outputs);
ICX_API int icx_engine_output_info(icx_engine* e, const char* name, int* dtype, int* rank,
                                   int64_t* dims /* [6] */);
ICX_API int icx_engine_output_copy(icx_engine* e, const char* name, void* host, size_t bytes);
/* Pipelined run for serving loops (no reference counterpart; the reference's
 * run is synchronous): queues the inputs' upload, the plan and the download
 * of the requested outputs into host_out[k] (host_out_bytes[k] bytes each;
 * pinned memory lets the download overlap the next submission's compute)
 * and returns a ticket without waiting.  The host buffers of a submission
 * must stay valid until icx_engine_wait(ticket) returns.  Up to two
 * submissions are in flight; a third waits on the GPU for the oldest
 * download. */
ICX_API int icx_engine_submit(icx_engine* e, int n_in, const char* const* names, const int* dtypes,
                              const int* ranks, const int64_t* dims, const void* const* host,
                              int n_out, const char* const* outputs, void* const* host_out,
                              const size_t* host_out_bytes, int64_t* ticket);
/* Blocks until submission `ticket` has its outputs in its host buffers. */
ICX_API int icx_engine_wait(icx_engine* e, int64_t ticket);

/* Global DynamicQuantizeLinear for batch-sharded executors (no reference
 * counterpart: the reference runs on one GPU).  By default each executor
 * quantises its shard with the shard's own (min, max); with this mode every
 * DynamicQuantizeLinear takes (min, max) over all executors through one
 * 8-byte NCCL MAX all-reduce on the executor's stream, so the shards give
 * bit-for-bit what one executor over the whole batch gives.
 * icx_nccl_unique_id writes a 128-byte id (bytes >= 128) on one rank; every
 * rank then calls icx_engine_set_global_dql with it concurrently (the set-up
 * is collective).  nranks <= 1 turns the mode off.  NCCL (libnccl.so.2) is
 * loaded on first use. */
ICX_API int icx_nccl_unique_id(void* id_out, size_t bytes);
ICX_API int icx_engine_set_global_dql(icx_engine* e, const void* nccl_id, int nranks, int rank);
/* Aborts the global-DQL communicator of `e` (ncclCommAbort; no reference
 * counterpart).  For a sharded run in which one executor failed or stalled:
 * the other executors' all-reduces would otherwise wait on the GPU for a
 * peer that never joins.  May be called from another host thread while e's
 * own thread is blocked in icx_engine_run.  Afterwards run / submit / replay
 * on e fail with ICX_ERR_INVALID until icx_engine_set_global_dql is called
 * again. */
ICX_API int icx_engine_abort_global_dql(icx_engine* e);
/* The compiled plan, one "op node -> output" line per launch step. */
ICX_API const char* icx_engine_plan(icx_engine* e);
/* Replay the compiled plan as a CUDA graph after the first run (default on). */
ICX_API int icx_engine_set_cuda_graphs(icx_engine* e, int enabled);
/* Re-executes the compiled plan on the inputs already on the device from the
 * last run: enqueued on the engine's stream, no copies, no synchronisation
 * (device-resident throughput measurement). */
ICX_API int icx_engine_replay(icx_engine* e);
/* Per-step GPU times of one more eager execution of the compiled plan on the
 * last run's inputs: lines "<ms>\t<op>\t<node>\t<output>" (NULL on error).
 * Replaces run_with_profiling (src/cuda/executor/variants.rs:415) and its
 * ProfileData (src/cuda/inference/mod.rs:88-164). */
ICX_API const char* icx_engine_profile(icx_engine* e);
/* The engine's CUDA stream (cudaStream_t as void*). */
ICX_API void* icx_engine_stream(icx_engine* e);
/* Kernel launches per run of the compiled plan. */
ICX_API int icx_engine_kernel_launches(icx_engine* e);

/* Per-step debug interface: stage-by-stage inspection of the compiled, fused
 * plan without turning fusion off (requesting an intermediate as an output
 * would keep it materialised and change the plan).  Replaces the reference's
 * intermediate-value access in its debug / validation runs
 * (src/cuda/inference/mod.rs:88-164 ProfileData, src/cuda/executor/
 * variants.rs:415 run_with_profiling), which record per-node results.
 *   step_count: steps of the compiled plan (0 before the first run).
 *   step_info:  "op\tnode\toutput\tkey=value;..." naming the values step i
 *               reads and writes (fused Linears: q, s, z, w, ws, bz, bias,
 *               residual, gelu, out; merged Linears list their parts'
 *               initializers '|'-separated; other steps: in=..., outs=...).
 *               NULL if i is out of range.  Valid until the next call.
 *   run_step:   runs step i alone, eagerly, and waits for it.  After a run,
 *               calling it for i = 0, 1, ... in order re-executes the plan
 *               step by step; the values a step reads are live in the arena
 *               just before it runs and the values it writes just after.
 *   value_info / value_copy: shape and current contents of any value the
 *               plan materialises (ICX_ERR_NOT_FOUND for values that live
 *               inside a fused kernel). */
ICX_API int icx_engine_step_count(icx_engine* e);
ICX_API const char* icx_engine_step_info(icx_engine* e, int i);
ICX_API int icx_engine_run_step(icx_engine* e, int i);
ICX_API int icx_engine_value_info(icx_engine* e, const char* name, int* dtype, int* rank,
                                  int64_t* dims /* [6] */);
ICX_API int icx_engine_value_copy(icx_engine* e, const char* name, void* host, size_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* ICONNX_B200_H */
