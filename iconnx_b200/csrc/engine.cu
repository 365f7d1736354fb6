// Graph executor: the B200 counterpart of the reference's GpuGraphExecutor
// (src/cuda/inference/mod.rs:222-659) and its lowering + runtime
// (src/ir/lowering.rs:31-238, src/cuda/executor/mod.rs:107-441).
//
// Lifecycle (mirrors the reference's lazy lowering, mod.rs:484-536):
//   create -> add_input / add_initializer / add_node -> run(...)
// The first run with a given set of input shapes and requested outputs
// compiles a plan:
//   1. topological sort of the nodes;
//   2. shape / dtype inference for every value;
//   3. QuantLinear fusion: DynamicQuantizeLinear's q feeding
//        MatMulInteger -> Cast(FLOAT) -> Mul(., Mul(scale, w_scale))
//        [-> Add(bias)] [-> Div(sqrt2) -> Erf -> Add(1) -> Mul(x, .) -> Mul(0.5)]
//      becomes one tcgen05 GEMM with a fused epilogue (icx_quant_linear);
//   4. producer-fused min/max: a DynamicQuantizeLinear whose input comes from
//      a fused QuantLinear or a LayerNormalization runs as its quantise pass
//      only, the producer's kernel having written (min, max) partials;
//   5. static arena: every intermediate gets an offset in one device
//      allocation, reused by lifetime (the reference's planner exists but is
//      unwired, src/ir/plan.rs:59-71);
//   6. int8 weights are uploaded once and pre-transposed to the tensor-core
//      layout with their column sums.
// Later runs with the same shapes replay the plan as a CUDA graph: only the
// host->device input copies, one graph launch and the device->host output
// copies remain.  A GpuGraphExecutor is single-threaded (the reference's is
// !Sync); use one per thread / GPU.
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include "capi.cuh"
#include "glue.h"

namespace icx {

// ONNX TensorProto data types -> element codes
static int onnx_to_icx(int64_t t) {
  switch (t) {
    case 1: return ICX_F32;
    case 2: return ICX_U8;
    case 3: return ICX_S8;
    case 6: return ICX_S32;
    case 7: return ICX_S64;
    case 9: return ICX_BOOL;
    default: return -1;
  }
}

static const char* type_name(int t) {
  switch (t) {
    case ICX_F32: return "Float32";
    case ICX_U8: return "UInt8";
    case ICX_S8: return "Int8";
    case ICX_S32: return "Int32";
    case ICX_S64: return "Int64";
    case ICX_BOOL: return "Bool";
    default: return "?";
  }
}

using Shape = std::vector<int64_t>;

static int64_t numel(const Shape& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

static std::string shape_str(const Shape& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

struct Attr {
  int kind = 0;  // 1 int, 2 float, 3 ints, 4 string, 5 floats
  int64_t i = 0;
  float f = 0;
  std::vector<int64_t> ints;
  std::vector<float> floats;
  std::string s;
};

struct NodeDef {
  std::string name, op;
  std::vector<std::string> in, out;
  std::map<std::string, Attr> attrs;
  int64_t geti(const char* k, int64_t d) const {
    auto it = attrs.find(k);
    return it == attrs.end() ? d : it->second.i;
  }
  float getf(const char* k, float d) const {
    auto it = attrs.find(k);
    return it == attrs.end() ? d : it->second.f;
  }
  const std::vector<int64_t>* getints(const char* k) const {
    auto it = attrs.find(k);
    return it == attrs.end() ? nullptr : &it->second.ints;
  }
};

struct Init {
  int dtype;
  Shape shape;
  std::vector<uint8_t> data;
  void* dev = nullptr;
};

struct Prepared {  // int8 weight in the tensor-core operand layout
  void* bt = nullptr;
  int32_t* colsum = nullptr;
  int64_t K = 0, N = 0;
  // merged weights only: per-column scale, bias and zero point of the parts
  float* ws = nullptr;
  float* bias = nullptr;
  int8_t* bz = nullptr;
};

struct Val {
  int dtype = -1;
  Shape shape;
  int producer = -1;
  std::vector<int> consumers;
  std::string alias;          // shares the buffer of this value
  bool is_input = false;
  const Init* init = nullptr;
  bool needed = true;         // materialised (false: lives inside a fused kernel)
  int64_t off = -1;           // arena offset
  void* ptr = nullptr;        // resolved device pointer
  int minmax_slot = -1;       // producer writes (min, max) partials here
};

// One fused QuantLinear (step 3 above).
struct FusedQL {
  std::string q, s, z, w, ws, bz, bias, residual, out;
  bool gelu = false;
  // LayerNormalization of the residual sum, in the same kernel (out is then
  // the LayerNorm's output)
  std::string ln_gamma, ln_beta;
  float ln_eps = 0.0f;
  std::vector<FusedQL> parts;  // non-empty: several Linears merged along N
};

// One fused attention block: Reshape/Transpose of Q, K, V -> MatMul ->
// Div(c) -> Add(mask) -> Softmax -> MatMul -> Transpose -> Reshape.
struct FusedAttn {
  std::string q, k, v, mask, scores, out;
  int64_t ld = 0, off_q = 0, off_k = 0, off_v = 0;  // row stride / column offsets of q, k, v
  float c = 1.0f;
  int64_t B = 0, S = 0, H = 0, nh = 0, dh = 0;
  bool mask_per_batch = true;
};

// QuantLinear + residual + LayerNorm in one kernel (default on);
// ICONNX_LN_FUSE=0 keeps the LayerNorm a step of its own (read once, for
// measurement).
static bool ln_fuse_enabled() {
  static const bool on = [] {
    const char* e = getenv("ICONNX_LN_FUSE");
    return !(e && e[0] == '0');
  }();
  return on;
}

struct Step {
  std::string node, op, out;
  std::function<int(cudaStream_t)> fn;
  // "key=value;..." naming the values the step reads and writes (the
  // per-step debug interface, icx_engine_step_info)
  std::string info;
};

// NCCL, loaded on first use (the library has no link-time dependency on it):
// only the global DynamicQuantizeLinear mode of batch-sharded executors uses
// it, for one 8-byte MAX all-reduce per DynamicQuantizeLinear.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

static const NcclApi* nccl_api() {
  static NcclApi api;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy &&
         api.comm_abort && api.error_string;
  });
  return ok ? &api : nullptr;
}

class Engine {
 public:
  explicit Engine(int device) : device_(device) {}
  ~Engine() { release(); }

  int init() {
    ICX_CUDA(cudaSetDevice(device_));
    ICX_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    if (cublasCreate(&blas_) != CUBLAS_STATUS_SUCCESS) {
      set_error("cublasCreate failed");
      return ICX_ERR_CUDA;
    }
    cublasSetStream(blas_, stream_);
    // fixed cuBLAS workspace so captured CUDA graphs never allocate
    ICX_CUDA(cudaMalloc(&blas_ws_, kBlasWorkspace));
    cublasSetWorkspace(blas_, blas_ws_, kBlasWorkspace);
    return ICX_OK;
  }

  int add_input(const std::string& name, int dtype, const Shape& shape) {
    ICX_REQUIRE(!name.empty(), "add_input: empty name");
    inputs_.push_back(name);
    input_defs_[name] = {dtype, shape};
    invalidate();
    return ICX_OK;
  }

  int add_initializer(const std::string& name, int dtype, const Shape& shape, const void* data) {
    ICX_REQUIRE(dtype >= 0 && dtype <= ICX_BOOL, "add_initializer %s: bad dtype", name.c_str());
    auto in = std::make_unique<Init>();
    in->dtype = dtype;
    in->shape = shape;
    const size_t bytes = (size_t)numel(shape) * dtype_size(dtype);
    in->data.resize(bytes);
    if (bytes) {
      ICX_REQUIRE(data != nullptr, "add_initializer %s: null data", name.c_str());
      memcpy(in->data.data(), data, bytes);
    }
    inits_[name] = std::move(in);
    invalidate();
    return ICX_OK;
  }

  int add_node(NodeDef n) {
    ICX_REQUIRE(!n.op.empty(), "add_node: empty op type");
    nodes_.push_back(std::move(n));
    invalidate();
    return ICX_OK;
  }

  // Validates the inputs, (re)compiles when their shapes or the requested
  // outputs change, and queues the inputs' host->device copies on the stream.
  // Validates the inputs, compiles the plan for their shapes when needed and,
  // with `upload`, copies them into the plan's input slots on the compute
  // stream.
  int stage_inputs(const std::vector<std::string>& names, const std::vector<int>& dtypes,
                   const std::vector<Shape>& shapes, const std::vector<const void*>& host,
                   const std::vector<std::string>& outputs, bool upload = true) {
    ICX_CUDA(cudaSetDevice(device_));
    // input-shape guard (src/cuda/inference/mod.rs:441-460): declared
    // static dimensions must match; dynamic ones (<= 0) may vary.
    std::map<std::string, Shape> in_shapes;
    for (size_t i = 0; i < names.size(); ++i) {
      auto it = input_defs_.find(names[i]);
      if (it == input_defs_.end()) {
        set_error("run: unknown input '%s'", names[i].c_str());
        return ICX_ERR_NOT_FOUND;
      }
      if (dtypes[i] != it->second.first) {
        set_error("run: input '%s' has dtype %s, graph declares %s", names[i].c_str(),
                  type_name(dtypes[i]), type_name(it->second.first));
        return ICX_ERR_INVALID;
      }
      const Shape& decl = it->second.second;
      bool ok = decl.empty() || decl.size() == shapes[i].size();
      for (size_t d = 0; ok && d < decl.size(); ++d)
        if (decl[d] > 0 && decl[d] != shapes[i][d]) ok = false;
      if (!ok) {
        set_error("InputShapeMismatch: input '%s' has shape %s, graph declares %s",
                  names[i].c_str(), shape_str(shapes[i]).c_str(), shape_str(decl).c_str());
        return ICX_ERR_SHAPE_MISMATCH;
      }
      in_shapes[names[i]] = shapes[i];
    }
    for (auto& nm : inputs_)
      if (!in_shapes.count(nm)) {
        set_error("run: missing input '%s'", nm.c_str());
        return ICX_ERR_INVALID;
      }
    if (!compiled_ || in_shapes != compiled_shapes_ || outputs != compiled_outputs_) {
      int rc = compile(in_shapes, outputs);
      if (rc) {
        compiled_ = false;
        return rc;
      }
    }
    for (size_t i = 0; i < names.size() && upload; ++i) {
      Val& v = vals_[names[i]];
      const size_t bytes = (size_t)numel(v.shape) * dtype_size(v.dtype);
      if (bytes) ICX_CUDA(cudaMemcpyAsync(v.ptr, host[i], bytes, cudaMemcpyHostToDevice, stream_));
    }
    return ICX_OK;
  }

  int run(const std::vector<std::string>& names, const std::vector<int>& dtypes,
          const std::vector<Shape>& shapes, const std::vector<const void*>& host,
          const std::vector<std::string>& outputs) {
    ICX_REQUIRE(!collectives_aborted_, "run: this executor's collectives were aborted "
                "(call set_global_dql again, or build a new executor)");
    int rc = stage_inputs(names, dtypes, shapes, host, outputs);
    if (rc) return rc;
    rc = execute();
    if (rc) return rc;
    ICX_CUDA(cudaStreamSynchronize(stream_));
    return check_err_flag();
  }

  int check_err_flag() {
    if (err_flag_) {
      int e = 0;
      ICX_CUDA(cudaMemcpy(&e, err_flag_, sizeof(int), cudaMemcpyDeviceToHost));
      if (e) {
        ICX_CUDA(cudaMemset(err_flag_, 0, sizeof(int)));
        set_error("Gather: index out of range");
        return ICX_ERR_INVALID;
      }
    }
    return ICX_OK;
  }

  int output_info(const std::string& name, int* dtype, int* rank, int64_t* dims) {
    auto it = vals_.find(name);
    if (!compiled_ || it == vals_.end() ||
        std::find(compiled_outputs_.begin(), compiled_outputs_.end(), name) == compiled_outputs_.end()) {
      set_error("output '%s' was not requested by the last run", name.c_str());
      return ICX_ERR_NOT_FOUND;
    }
    *dtype = it->second.dtype;
    *rank = (int)it->second.shape.size();
    for (int d = 0; d < *rank && d < kMaxRank; ++d) dims[d] = it->second.shape[d];
    return ICX_OK;
  }

  int output_copy(const std::string& name, void* host, size_t bytes) {
    int dt, rk;
    int64_t dims[kMaxRank];
    int rc = output_info(name, &dt, &rk, dims);
    if (rc) return rc;
    const Val& v = vals_[name];
    const size_t need = (size_t)numel(v.shape) * dtype_size(v.dtype);
    ICX_REQUIRE(bytes >= need, "output '%s': buffer %zu < %zu bytes", name.c_str(), bytes, need);
    if (need) {
      ICX_CUDA(cudaMemcpyAsync(host, resolve(name), need, cudaMemcpyDeviceToHost, stream_));
      ICX_CUDA(cudaStreamSynchronize(stream_));
    }
    return ICX_OK;
  }

  // Pipelined run (a serving loop): stage the inputs, run the plan, snapshot
  // the requested outputs into one of two device staging sets on the compute
  // stream, and download them into the caller's host buffers on a second
  // stream, so the download of one submission overlaps the next one's
  // compute.  The host buffers (ideally pinned) must stay valid until
  // wait(ticket) returns; a staging set is reused only after its download
  // has completed.
  int submit(const std::vector<std::string>& names, const std::vector<int>& dtypes,
             const std::vector<Shape>& shapes, const std::vector<const void*>& host,
             const std::vector<std::string>& outputs, const std::vector<void*>& host_out,
             const std::vector<size_t>& out_bytes, int64_t* ticket) {
    ICX_REQUIRE(!collectives_aborted_, "submit: this executor's collectives were aborted "
                "(call set_global_dql again, or build a new executor)");
    int rc = stage_inputs(names, dtypes, shapes, host, outputs, /*upload=*/false);
    if (rc) return rc;
    if (!copy_stream_) ICX_CUDA(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
    if (!upload_stream_) ICX_CUDA(cudaStreamCreateWithFlags(&upload_stream_, cudaStreamNonBlocking));
    Pending& p = pend_[next_ticket_ & 1];
    if (!p.ready) {
      ICX_CUDA(cudaEventCreateWithFlags(&p.ready, cudaEventDisableTiming));
      ICX_CUDA(cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming));
      ICX_CUDA(cudaEventCreateWithFlags(&p.in_ready, cudaEventDisableTiming));
      ICX_CUDA(cudaEventCreateWithFlags(&p.in_free, cudaEventDisableTiming));
    }
    // Inputs: host -> this slot's device staging on the upload stream, which
    // overlaps the previous submission's compute (an upload on the compute
    // stream would wait for it and then delay this plan), then one device
    // copy per input into the plan's input slots on the compute stream.
    if (p.in_used) ICX_CUDA(cudaStreamWaitEvent(upload_stream_, p.in_free, 0));
    if (p.in_buf.size() < names.size()) {
      p.in_buf.resize(names.size(), nullptr);
      p.in_cap.resize(names.size(), 0);
    }
    std::vector<size_t> in_bytes(names.size());
    for (size_t i = 0; i < names.size(); ++i) {
      const Val& v = vals_[names[i]];
      in_bytes[i] = (size_t)numel(v.shape) * dtype_size(v.dtype);
      if (p.in_cap[i] < in_bytes[i]) {
        ICX_CUDA(cudaStreamSynchronize(stream_));
        if (p.in_buf[i]) ICX_CUDA(cudaFree(p.in_buf[i]));
        ICX_CUDA(cudaMalloc(&p.in_buf[i], in_bytes[i]));
        p.in_cap[i] = in_bytes[i];
      }
      if (in_bytes[i])
        ICX_CUDA(cudaMemcpyAsync(p.in_buf[i], host[i], in_bytes[i], cudaMemcpyHostToDevice,
                                 upload_stream_));
    }
    ICX_CUDA(cudaEventRecord(p.in_ready, upload_stream_));
    ICX_CUDA(cudaStreamWaitEvent(stream_, p.in_ready, 0));
    for (size_t i = 0; i < names.size(); ++i)
      if (in_bytes[i])
        ICX_CUDA(cudaMemcpyAsync(vals_[names[i]].ptr, p.in_buf[i], in_bytes[i],
                                 cudaMemcpyDeviceToDevice, stream_));
    ICX_CUDA(cudaEventRecord(p.in_free, stream_));
    p.in_used = true;
    rc = execute();
    if (rc) return rc;
    if (p.busy) ICX_CUDA(cudaStreamWaitEvent(stream_, p.done, 0));  // its last download is done
    if (p.buf.size() < outputs.size()) {
      p.buf.resize(outputs.size(), nullptr);
      p.cap.resize(outputs.size(), 0);
    }
    std::vector<size_t> need(outputs.size());
    for (size_t k = 0; k < outputs.size(); ++k) {
      const Val& v = vals_[outputs[k]];
      need[k] = (size_t)numel(v.shape) * dtype_size(v.dtype);
      ICX_REQUIRE(out_bytes[k] >= need[k], "submit: output '%s' buffer %zu < %zu bytes",
                  outputs[k].c_str(), out_bytes[k], need[k]);
      if (p.cap[k] < need[k]) {
        ICX_CUDA(cudaStreamSynchronize(stream_));
        if (p.buf[k]) ICX_CUDA(cudaFree(p.buf[k]));
        ICX_CUDA(cudaMalloc(&p.buf[k], need[k]));
        p.cap[k] = need[k];
      }
      if (need[k])
        ICX_CUDA(cudaMemcpyAsync(p.buf[k], resolve(outputs[k]), need[k], cudaMemcpyDeviceToDevice, stream_));
    }
    ICX_CUDA(cudaEventRecord(p.ready, stream_));
    ICX_CUDA(cudaStreamWaitEvent(copy_stream_, p.ready, 0));
    for (size_t k = 0; k < outputs.size(); ++k)
      if (need[k])
        ICX_CUDA(cudaMemcpyAsync(host_out[k], p.buf[k], need[k], cudaMemcpyDeviceToHost, copy_stream_));
    ICX_CUDA(cudaEventRecord(p.done, copy_stream_));
    p.busy = true;
    p.ticket = next_ticket_;
    *ticket = next_ticket_++;
    return ICX_OK;
  }

  // Blocks until submission `ticket` has its outputs in the host buffers.
  int wait(int64_t ticket) {
    ICX_REQUIRE(ticket >= 0 && ticket < next_ticket_, "wait: unknown ticket %lld", (long long)ticket);
    Pending& p = pend_[ticket & 1];
    if (p.busy && p.ticket == ticket) {
      ICX_CUDA(cudaEventSynchronize(p.done));
      p.busy = false;
    }
    // an older ticket of this slot completed before the slot was reused
    return check_err_flag();
  }

  // Human-readable plan: one line per step ("op node -> out").
  std::string plan_text() const {
    std::string s;
    for (auto& st : steps_) s += st.op + " " + st.node + " -> " + st.out + "\n";
    return s;
  }

  // Runs the compiled plan once more (eagerly, on the inputs of the last run)
  // with a CUDA event pair around every step and returns one line per step:
  // "<gpu_ms>\t<op>\t<node>\t<output>".  The counterpart of the reference's
  // run_with_profiling / GpuEventTimer (src/cuda/executor/variants.rs:415,
  // src/cuda/inference/gpu_event_timer.rs:1-45).
  int profile(std::string* text) {
    ICX_REQUIRE(compiled_, "profile: no compiled plan (call run first)");
    ICX_REQUIRE(!collectives_aborted_, "profile: this executor's collectives were aborted");
    ICX_CUDA(cudaSetDevice(device_));
    // Every step is captured alone, kReps times in a row, into a CUDA graph
    // and timed with an event pair around its replay: device time only,
    // without the host launch gaps an eager per-step measurement includes.
    // Steps are idempotent, so repeating one leaves the state unchanged.
    constexpr int kReps = 10;
    cudaEvent_t e0, e1;
    ICX_CUDA(cudaEventCreate(&e0));
    ICX_CUDA(cudaEventCreate(&e1));
    text->clear();
    int rc = ICX_OK;
    for (size_t i = 0; i < steps_.size() && !rc; ++i) {
      cudaGraph_t g = nullptr;
      cudaGraphExec_t ge = nullptr;
      ICX_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
      for (int r = 0; r < kReps && !rc; ++r) rc = steps_[i].fn(stream_);
      cudaError_t ce = cudaStreamEndCapture(stream_, &g);
      if (rc || ce != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        if (!rc) {
          set_error("profile capture failed: %s", cudaGetErrorString(ce));
          rc = ICX_ERR_CUDA;
        }
        break;
      }
      ce = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      if (ce != cudaSuccess) {
        set_error("profile instantiate failed: %s", cudaGetErrorString(ce));
        rc = ICX_ERR_CUDA;
        break;
      }
      cudaGraphLaunch(ge, stream_);  // warm
      cudaEventRecord(e0, stream_);
      cudaGraphLaunch(ge, stream_);
      cudaEventRecord(e1, stream_);
      cudaStreamSynchronize(stream_);
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      cudaGraphExecDestroy(ge);
      char buf[64];
      snprintf(buf, sizeof(buf), "%.4f\t", ms / kReps);
      *text += buf + steps_[i].op + "\t" + steps_[i].node + "\t" + steps_[i].out + "\n";
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return rc;
  }

  // Re-executes the compiled plan on the device-resident inputs of the last
  // run, asynchronously on the engine's stream (no copies, no sync).
  int replay() {
    ICX_REQUIRE(compiled_, "replay: no compiled plan (call run first)");
    ICX_REQUIRE(!collectives_aborted_, "replay: this executor's collectives were aborted");
    ICX_CUDA(cudaSetDevice(device_));
    return execute();
  }

  void set_graphs(bool on) {
    use_graphs_ = on;
    drop_graph();
  }
  int kernel_launches() const { return launches_per_run_; }
  cudaStream_t stream() const { return stream_; }

  // ---- per-step debug interface (stage-by-stage parity of a fused plan)
  int step_count() const { return compiled_ ? (int)steps_.size() : 0; }
  const Step* step(int i) const {
    return compiled_ && i >= 0 && i < (int)steps_.size() ? &steps_[(size_t)i] : nullptr;
  }
  // Runs plan step i alone, eagerly, and waits for it.  Steps must be run in
  // plan order after a run (a step reads what the earlier steps wrote, and
  // the arena reuses a slot once its last reader has run).
  int run_step(int i) {
    ICX_REQUIRE(step(i) != nullptr, "run_step: no step %d in the compiled plan", i);
    ICX_REQUIRE(!collectives_aborted_, "run_step: this executor's collectives were aborted");
    ICX_CUDA(cudaSetDevice(device_));
    int rc = steps_[(size_t)i].fn(stream_);
    if (rc) return rc;
    ICX_CUDA(cudaStreamSynchronize(stream_));
    return check_err_flag();
  }
  // Any value the plan materialises (not only requested outputs); the data
  // is what its arena slot holds now.
  int value_info(const std::string& name, int* dtype, int* rank, int64_t* dims) {
    auto it = vals_.find(name);
    if (!compiled_ || it == vals_.end() || !resolve(name)) {
      set_error("value '%s' is not materialised by the compiled plan", name.c_str());
      return ICX_ERR_NOT_FOUND;
    }
    *dtype = it->second.dtype;
    *rank = (int)it->second.shape.size();
    for (int d = 0; d < *rank && d < kMaxRank; ++d) dims[d] = it->second.shape[d];
    return ICX_OK;
  }
  int value_copy(const std::string& name, void* host, size_t bytes) {
    int dt, rk;
    int64_t dims[kMaxRank];
    int rc = value_info(name, &dt, &rk, dims);
    if (rc) return rc;
    const Val& v = vals_[name];
    const size_t need = (size_t)numel(v.shape) * dtype_size(v.dtype);
    ICX_REQUIRE(bytes >= need, "value '%s': buffer %zu < %zu bytes", name.c_str(), bytes, need);
    ICX_CUDA(cudaSetDevice(device_));
    ICX_CUDA(cudaStreamSynchronize(stream_));
    if (need) ICX_CUDA(cudaMemcpy(host, resolve(name), need, cudaMemcpyDeviceToHost));
    return ICX_OK;
  }

 private:
  // ------------------------------------------------------------ lifecycle
  void invalidate() {
    compiled_ = false;
    drop_graph();
  }
  void drop_graph() {
    if (gexec_) cudaGraphExecDestroy(gexec_);
    gexec_ = nullptr;
    runs_ = 0;
  }
  void release() {
    // nothing of this engine may still run on the buffers freed below
    for (cudaStream_t st : {stream_, copy_stream_, upload_stream_})
      if (st) cudaStreamSynchronize(st);
    drop_graph();
    if (arena_) cudaFree(arena_);
    for (auto& kv : prepared_) {
      cudaFree(kv.second.bt);
      cudaFree(kv.second.colsum);
      if (kv.second.ws) cudaFree(kv.second.ws);
      if (kv.second.bias) cudaFree(kv.second.bias);
      if (kv.second.bz) cudaFree(kv.second.bz);
    }
    for (auto& kv : inits_)
      if (kv.second->dev) cudaFree(kv.second->dev);
    if (err_flag_) cudaFree(err_flag_);
    for (auto& kv : rowsum_bufs_) cudaFree(kv.second);
    for (void* p : scratch_) cudaFree(p);
    if (blas_) cublasDestroy(blas_);
    if (blas_ws_) cudaFree(blas_ws_);
    for (auto& p : pend_) {
      for (void* b : p.buf) if (b) cudaFree(b);
      for (void* b : p.in_buf) if (b) cudaFree(b);
      if (p.ready) cudaEventDestroy(p.ready);
      if (p.done) cudaEventDestroy(p.done);
      if (p.in_ready) cudaEventDestroy(p.in_ready);
      if (p.in_free) cudaEventDestroy(p.in_free);
    }
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    if (upload_stream_) cudaStreamDestroy(upload_stream_);
    if (ncclComm_t c = comm_.exchange(nullptr)) nccl_api()->comm_destroy(c);
    if (gdql_) cudaFree(gdql_);
    if (stream_) cudaStreamDestroy(stream_);
  }

  // ----------------------------------------------------------- utilities
  void* resolve(const std::string& name) {
    const Val* v = &vals_[name];
    while (!v->alias.empty()) v = &vals_[v->alias];
    if (v->init) return v->init->dev;
    return v->ptr;
  }
  const Init* init_of(const std::string& name) const {
    auto it = inits_.find(name);
    return it == inits_.end() ? nullptr : it->second.get();
  }
  static bool scalar_f32(const Init* in, float* v) {
    if (!in || in->dtype != ICX_F32 || numel(in->shape) != 1) return false;
    memcpy(v, in->data.data(), 4);
    return true;
  }
  int fail(const NodeDef& n, const char* fmt, ...) {
    char buf[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    set_error("op %s (%s): %s", n.name.c_str(), n.op.c_str(), buf);
    return ICX_ERR_INVALID;
  }

  // -------------------------------------------------------------- compile
  int compile(const std::map<std::string, Shape>& in_shapes, const std::vector<std::string>& outputs) {
    drop_graph();
    compiled_ = false;
    vals_.clear();
    steps_.clear();
    fused_.clear();
    attn_.clear();
    skip_.clear();
    dql_mode_.clear();
    minmax_count_.clear();
    // initializers derived at the previous compile are derived again
    for (auto& nm : folded_) {
      auto it = inits_.find(nm);
      if (it != inits_.end()) {
        if (it->second->dev) cudaFree(it->second->dev);
        inits_.erase(it);
      }
    }
    folded_.clear();
    for (auto& nm : inputs_) {
      Val v;
      v.dtype = input_defs_[nm].first;
      v.shape = in_shapes.at(nm);
      v.is_input = true;
      vals_[nm] = v;
    }
    for (auto& kv : inits_) {
      if (vals_.count(kv.first)) continue;
      Val v;
      v.dtype = kv.second->dtype;
      v.shape = kv.second->shape;
      v.init = kv.second.get();
      vals_[kv.first] = v;
    }
    int rc = toposort();
    if (rc) return rc;
    for (int idx : order_) {
      rc = infer(nodes_[idx], idx);
      if (rc) return rc;
    }
    fold_constants();
    for (auto& o : outputs)
      if (!vals_.count(o)) {
        set_error("requested output '%s' is not produced by the graph", o.c_str());
        return ICX_ERR_NOT_FOUND;
      }
    fuse();
    rc = upload_weights();
    if (rc) return rc;
    rc = plan_memory(outputs);
    if (rc) return rc;
    rc = build_steps();
    if (rc) return rc;
    compiled_shapes_ = in_shapes;
    compiled_outputs_ = outputs;
    compiled_ = true;
    return ICX_OK;
  }

  int toposort() {
    order_.clear();
    std::set<std::string> have;
    for (auto& nm : inputs_) have.insert(nm);
    for (auto& kv : inits_) have.insert(kv.first);
    std::vector<bool> done(nodes_.size(), false);
    size_t remaining = nodes_.size();
    while (remaining) {
      bool progress = false;
      for (size_t i = 0; i < nodes_.size(); ++i) {
        if (done[i]) continue;
        bool ready = true;
        for (auto& in : nodes_[i].in)
          if (!in.empty() && !have.count(in)) ready = false;
        if (!ready) continue;
        done[i] = true;
        --remaining;
        progress = true;
        order_.push_back((int)i);
        for (auto& o : nodes_[i].out) have.insert(o);
      }
      if (!progress) {
        for (size_t i = 0; i < nodes_.size(); ++i)
          if (!done[i]) {
            for (auto& in : nodes_[i].in)
              if (!in.empty() && !have.count(in)) {
                set_error("op %s (%s): input '%s' is never produced (cycle or missing tensor)",
                          nodes_[i].name.c_str(), nodes_[i].op.c_str(), in.c_str());
                return ICX_ERR_INVALID;
              }
          }
        set_error("graph has a cycle");
        return ICX_ERR_INVALID;
      }
    }
    return ICX_OK;
  }

  Val& out_val(int idx, int k, int dtype, const Shape& s) {
    Val& v = vals_[nodes_[idx].out[k]];
    v.dtype = dtype;
    v.shape = s;
    v.producer = idx;
    return v;
  }

  static bool broadcast(const Shape& a, const Shape& b, Shape* o) {
    const size_t r = std::max(a.size(), b.size());
    o->assign(r, 1);
    for (size_t i = 0; i < r; ++i) {
      const int64_t da = i < r - a.size() ? 1 : a[i - (r - a.size())];
      const int64_t db = i < r - b.size() ? 1 : b[i - (r - b.size())];
      if (da != db && da != 1 && db != 1) return false;
      (*o)[i] = da == 1 ? db : da;
    }
    return true;
  }

  int infer(const NodeDef& n, int idx) {
    std::vector<Val*> in;
    for (auto& nm : n.in) in.push_back(nm.empty() ? nullptr : &vals_[nm]);
    for (auto& nm : n.in)
      if (!nm.empty()) vals_[nm].consumers.push_back(idx);
    auto need = [&](size_t k) { return k < in.size() && in[k] != nullptr; };
    const std::string& op = n.op;
    if (op == "Add" || op == "Sub" || op == "Mul" || op == "Div") {
      if (!need(0) || !need(1)) return fail(n, "needs 2 inputs");
      if (in[0]->dtype != ICX_F32 || in[1]->dtype != ICX_F32)
        return fail(n, "only Float32 operands are supported (got %s, %s)", type_name(in[0]->dtype),
                    type_name(in[1]->dtype));
      Shape o;
      if (!broadcast(in[0]->shape, in[1]->shape, &o))
        return fail(n, "cannot broadcast %s with %s", shape_str(in[0]->shape).c_str(),
                    shape_str(in[1]->shape).c_str());
      out_val(idx, 0, ICX_F32, o);
    } else if (op == "DynamicQuantizeLinear") {
      if (!need(0)) return fail(n, "needs 1 input");
      if (in[0]->dtype != ICX_F32)
        return fail(n, "input must be Float32, got %s", type_name(in[0]->dtype));
      if (n.out.size() != 3) return fail(n, "needs 3 outputs");
      out_val(idx, 0, ICX_U8, in[0]->shape);
      out_val(idx, 1, ICX_F32, {});
      out_val(idx, 2, ICX_U8, {});
    } else if (op == "MatMulInteger") {
      if (!need(0) || !need(1)) return fail(n, "needs a and b");
      for (int k = 0; k < 2; ++k)
        if (in[k]->dtype != ICX_U8 && in[k]->dtype != ICX_S8)
          return fail(n, "input %c must be Int8 or UInt8, got %s", k ? 'b' : 'a', type_name(in[k]->dtype));
      const Shape& a = in[0]->shape;
      const Shape& b = in[1]->shape;
      if (b.size() != 2 || a.size() < 2 || a.size() > 3)
        return fail(n, "unsupported ranks a=%zu b=%zu", a.size(), b.size());
      if (a.back() != b[0])
        return fail(n, "K mismatch — a is %s, b is %s", shape_str(a).c_str(), shape_str(b).c_str());
      for (int k = 2; k < 4; ++k)
        if (need(k) && in[k]->dtype != in[k - 2]->dtype)
          return fail(n, "%c_zero_point dtype %s must match operand dtype %s", k == 2 ? 'a' : 'b',
                      type_name(in[k]->dtype), type_name(in[k - 2]->dtype));
      if (need(2) && numel(in[2]->shape) != 1) return fail(n, "a_zero_point must be scalar");
      if (need(3) && numel(in[3]->shape) != 1 && numel(in[3]->shape) != b[1])
        return fail(n, "b_zero_point must be scalar or per-column");
      Shape o = a;
      o.back() = b[1];
      out_val(idx, 0, ICX_S32, o);
    } else if (op == "DequantizeLinear") {
      if (!need(0) || !need(1)) return fail(n, "needs x and scale");
      if (in[0]->dtype != ICX_U8 && in[0]->dtype != ICX_S8 && in[0]->dtype != ICX_S32)
        return fail(n, "input dtype %s unsupported (must be Int8, UInt8, or Int32)", type_name(in[0]->dtype));
      if (in[1]->dtype != ICX_F32) return fail(n, "scale must be Float32, got %s", type_name(in[1]->dtype));
      if (need(2) && in[2]->dtype != in[0]->dtype)
        return fail(n, "zero_point dtype %s must match input dtype %s", type_name(in[2]->dtype),
                    type_name(in[0]->dtype));
      out_val(idx, 0, ICX_F32, in[0]->shape);
    } else if (op == "Cast") {
      if (!need(0)) return fail(n, "needs 1 input");
      const int to = onnx_to_icx(n.geti("to", 1));
      if (to < 0) return fail(n, "unsupported target type %lld", (long long)n.geti("to", 0));
      out_val(idx, 0, to, in[0]->shape);
    } else if (op == "Erf" || op == "Identity" || op == "Softmax") {
      if (!need(0)) return fail(n, "needs 1 input");
      if (op != "Identity" && in[0]->dtype != ICX_F32) return fail(n, "input must be Float32");
      if (op == "Softmax") {
        const int64_t ax = n.geti("axis", -1);
        if (ax != -1 && ax != (int64_t)in[0]->shape.size() - 1)
          return fail(n, "only the last axis is supported");
      }
      Val& o = out_val(idx, 0, in[0]->dtype, in[0]->shape);
      if (op == "Identity") o.alias = n.in[0];
    } else if (op == "LayerNormalization") {
      if (!need(0) || !need(1)) return fail(n, "needs X and scale");
      const int64_t ax = n.geti("axis", -1);
      if (ax != -1 && ax != (int64_t)in[0]->shape.size() - 1)
        return fail(n, "only the last axis is supported");
      out_val(idx, 0, ICX_F32, in[0]->shape);
    } else if (op == "Gather") {
      if (!need(0) || !need(1)) return fail(n, "needs data and indices");
      if (n.geti("axis", 0) != 0) return fail(n, "only axis 0 is supported");
      if (in[1]->dtype != ICX_S64) return fail(n, "indices must be Int64");
      if (in[0]->dtype == ICX_BOOL) return fail(n, "Bool data unsupported");
      Shape o = in[1]->shape;
      o.insert(o.end(), in[0]->shape.begin() + 1, in[0]->shape.end());
      out_val(idx, 0, in[0]->dtype, o);
    } else if (op == "Reshape" || op == "Unsqueeze" || op == "Squeeze") {
      if (!need(0)) return fail(n, "needs data");
      Shape o;
      if (op == "Reshape") {
        const Init* sh = need(1) ? init_of(n.in[1]) : nullptr;
        if (!sh || sh->dtype != ICX_S64) return fail(n, "shape must be an Int64 initializer");
        Shape t(numel(sh->shape));
        memcpy(t.data(), sh->data.data(), t.size() * 8);
        int64_t known = 1, infer_at = -1;
        for (size_t d = 0; d < t.size(); ++d) {
          if (t[d] == 0) t[d] = in[0]->shape.at(d);
          if (t[d] == -1) infer_at = (int64_t)d;
          else known *= t[d];
        }
        if (infer_at >= 0) t[infer_at] = known ? numel(in[0]->shape) / known : 0;
        if (numel(t) != numel(in[0]->shape))
          return fail(n, "cannot reshape %s to %s", shape_str(in[0]->shape).c_str(), shape_str(t).c_str());
        o = t;
      } else {
        std::vector<int64_t> axes;
        if (const auto* a = n.getints("axes")) axes = *a;
        else if (need(1) && init_of(n.in[1])) {
          const Init* ai = init_of(n.in[1]);
          axes.resize(numel(ai->shape));
          memcpy(axes.data(), ai->data.data(), axes.size() * 8);
        }
        if (op == "Unsqueeze") {
          const int64_t r = (int64_t)(in[0]->shape.size() + axes.size());
          for (auto& a : axes) if (a < 0) a += r;
          std::sort(axes.begin(), axes.end());
          o = in[0]->shape;
          for (auto a : axes) o.insert(o.begin() + a, 1);
        } else {
          const int64_t r = (int64_t)in[0]->shape.size();
          for (auto& a : axes) if (a < 0) a += r;
          for (int64_t d = 0; d < r; ++d) {
            const bool drop = axes.empty() ? in[0]->shape[d] == 1
                                           : std::find(axes.begin(), axes.end(), d) != axes.end();
            if (!drop) o.push_back(in[0]->shape[d]);
          }
        }
      }
      Val& v = out_val(idx, 0, in[0]->dtype, o);
      v.alias = n.in[0];
    } else if (op == "Transpose") {
      if (!need(0)) return fail(n, "needs data");
      const Shape& s = in[0]->shape;
      std::vector<int64_t> perm;
      if (const auto* p = n.getints("perm")) perm = *p;
      else for (int64_t d = (int64_t)s.size() - 1; d >= 0; --d) perm.push_back(d);
      if (perm.size() != s.size()) return fail(n, "perm has the wrong length");
      Shape o;
      for (auto p : perm) o.push_back(s.at(p));
      out_val(idx, 0, in[0]->dtype, o);
    } else if (op == "MatMul") {
      if (!need(0) || !need(1)) return fail(n, "needs 2 inputs");
      if (in[0]->dtype != ICX_F32 || in[1]->dtype != ICX_F32) return fail(n, "only Float32 is supported");
      const Shape& a = in[0]->shape;
      const Shape& b = in[1]->shape;
      if (a.size() < 2 || b.size() < 2) return fail(n, "rank-1 operands are unsupported");
      if (a.back() != b[b.size() - 2])
        return fail(n, "K mismatch — a is %s, b is %s", shape_str(a).c_str(), shape_str(b).c_str());
      Shape ab(a.begin(), a.end() - 2), bb(b.begin(), b.end() - 2), ob;
      if (!broadcast(ab, bb, &ob)) return fail(n, "batch dimensions do not broadcast");
      if (!(bb.empty() || numel(bb) == numel(ob)) || !(ab.empty() || numel(ab) == numel(ob)))
        return fail(n, "partial batch broadcasting is unsupported");
      ob.push_back(a[a.size() - 2]);
      ob.push_back(b.back());
      out_val(idx, 0, ICX_F32, ob);
    } else {
      return fail(n, "unsupported op type");
    }
    return ICX_OK;
  }

  // ----------------------------------------------------------- fusion
  int producer_op(const std::string& v, const char* op) const {
    auto it = vals_.find(v);
    if (it == vals_.end() || it->second.producer < 0) return -1;
    return nodes_[it->second.producer].op == op ? it->second.producer : -1;
  }
  int sole_consumer(const std::string& v) const {
    auto it = vals_.find(v);
    if (it == vals_.end() || it->second.consumers.size() != 1) return -1;
    return it->second.consumers[0];
  }
  // The operand of binary node `nd` that is not `self`.
  static const std::string* other(const NodeDef& nd, const std::string& self) {
    if (nd.in.size() != 2) return nullptr;
    if (nd.in[0] == self) return &nd.in[1];
    if (nd.in[1] == self) return &nd.in[0];
    return nullptr;
  }
  bool is_requested(const std::string& v) const {
    return std::find(pending_outputs_.begin(), pending_outputs_.end(), v) != pending_outputs_.end();
  }

  int pos_of(int node) const {
    for (size_t i = 0; i < order_.size(); ++i)
      if (order_[i] == node) return (int)i;
    return -1;
  }

  // A derived initializer (constant folding, weight conversion), rebuilt at
  // every compile.
  Init* add_derived(const std::string& name, int dtype, const Shape& shape,
                    std::vector<uint8_t> data) {
    auto in = std::make_unique<Init>();
    in->dtype = dtype;
    in->shape = shape;
    in->data = std::move(data);
    Init* p = in.get();
    inits_[name] = std::move(in);
    folded_.insert(name);
    Val& v = vals_[name];
    v.dtype = dtype;
    v.shape = shape;
    v.init = p;
    v.producer = -1;
    v.alias.clear();
    return p;
  }

  // Nodes whose data input is an initializer and that only move or relabel
  // bytes (Transpose, Reshape, Unsqueeze, Squeeze, Identity) run once here on
  // the host: quantised exports store weights as `W_transposed_quantized`
  // behind a Transpose, and the folded weight is what the QuantLinear
  // fusion needs.
  void fold_constants() {
    for (int idx : order_) {
      const NodeDef& n = nodes_[idx];
      const bool relabel = n.op == "Reshape" || n.op == "Unsqueeze" || n.op == "Squeeze" ||
                           n.op == "Identity";
      if (!relabel && n.op != "Transpose") continue;
      if (n.in.empty() || n.out.size() != 1) continue;
      const Init* x = init_of(n.in[0]);
      if (!x || is_requested(n.out[0])) continue;
      const Val& ov = vals_[n.out[0]];
      const Shape oshape = ov.shape;
      std::vector<uint8_t> data;
      if (relabel) {
        data = x->data;
      } else {
        const size_t es = dtype_size(x->dtype);
        const Shape& s = x->shape;
        const size_t r = s.size();
        std::vector<int64_t> perm;
        if (const auto* p = n.getints("perm")) perm = *p;
        else for (int64_t d = (int64_t)r - 1; d >= 0; --d) perm.push_back(d);
        std::vector<int64_t> istride(r, 1);
        for (int64_t d = (int64_t)r - 2; d >= 0; --d) istride[d] = istride[d + 1] * s[d + 1];
        const int64_t total = numel(s);
        data.resize((size_t)total * es);
        std::vector<int64_t> oi(r, 0);
        for (int64_t t = 0; t < total; ++t) {
          int64_t src = 0;
          for (size_t k = 0; k < r; ++k) src += oi[k] * istride[perm[k]];
          memcpy(data.data() + (size_t)t * es, x->data.data() + (size_t)src * es, es);
          for (int64_t k = (int64_t)r - 1; k >= 0; --k) {
            if (++oi[k] < oshape[k]) break;
            oi[k] = 0;
          }
        }
      }
      add_derived(n.out[0], x->dtype, oshape, std::move(data));
      skip_.insert(idx);
    }
  }

  void fuse() {
    for (int idx : order_) {
      const NodeDef& mm = nodes_[idx];
      if (mm.op != "MatMulInteger" || skip_.count(idx)) continue;
      const int dq = producer_op(mm.in[0], "DynamicQuantizeLinear");
      if (dq < 0) continue;
      const NodeDef& d = nodes_[dq];
      if (mm.in.size() < 3 || mm.in[2] != d.out[2]) continue;  // a_zp must be the DQL's zp
      const Init* w = init_of(mm.in[1]);
      if (!w || (w->dtype != ICX_S8 && w->dtype != ICX_U8) || w->shape.size() != 2 || w->shape[0] % 16)
        continue;
      std::string wname = mm.in[1], bz;
      const Init* z = (mm.in.size() > 3 && !mm.in[3].empty()) ? init_of(mm.in[3]) : nullptr;
      if (mm.in.size() > 3 && !mm.in[3].empty() && (!z || z->dtype != w->dtype)) continue;
      if (w->dtype == ICX_U8) {
        // u8 weights w with zero point z (0 when absent): w - z = (w ^ 0x80) - (z ^ 0x80)
        // exactly, with both sides of the right-hand difference in s8
        wname = mm.in[1] + "#s8";
        if (!init_of(wname)) {
          std::vector<uint8_t> d = w->data;
          for (auto& b : d) b ^= 0x80;
          add_derived(wname, ICX_S8, w->shape, std::move(d));
        }
        bz = (z ? mm.in[3] : mm.in[1]) + "#zp_s8";
        if (!init_of(bz)) {
          std::vector<uint8_t> d = z ? z->data : std::vector<uint8_t>(1, 0);
          for (auto& b : d) b ^= 0x80;
          add_derived(bz, ICX_S8, z ? z->shape : Shape{}, std::move(d));
        }
        w = init_of(wname);
      } else if (z) {
        bz = mm.in[3];
      }
      std::vector<int> chain{idx};
      const int cast = sole_consumer(mm.out[0]);
      if (cast < 0 || nodes_[cast].op != "Cast" || onnx_to_icx(nodes_[cast].geti("to", 0)) != ICX_F32 ||
          is_requested(mm.out[0]))
        continue;
      chain.push_back(cast);
      const int mul = sole_consumer(nodes_[cast].out[0]);
      if (mul < 0 || nodes_[mul].op != "Mul" || is_requested(nodes_[cast].out[0])) continue;
      const std::string* sc = other(nodes_[mul], nodes_[cast].out[0]);
      if (!sc) continue;
      const int smul = producer_op(*sc, "Mul");
      if (smul < 0) continue;
      const std::string* ws = other(nodes_[smul], d.out[1]);
      const Init* wsi = ws ? init_of(*ws) : nullptr;
      const int64_t N = w->shape[1];
      if (!wsi || wsi->dtype != ICX_F32 || (numel(wsi->shape) != 1 && numel(wsi->shape) != N)) continue;
      chain.push_back(mul);
      FusedQL f;
      f.q = d.out[0];
      f.s = d.out[1];
      f.z = d.out[2];
      f.w = wname;
      f.ws = *ws;
      f.bz = bz;
      std::string cur = nodes_[mul].out[0];
      // [Add(bias)]
      const int add = sole_consumer(cur);
      if (add >= 0 && nodes_[add].op == "Add" && !is_requested(cur)) {
        const std::string* b = other(nodes_[add], cur);
        const Init* bi = b ? init_of(*b) : nullptr;
        if (bi && bi->dtype == ICX_F32 && numel(bi->shape) == N && bi->shape.back() == N) {
          f.bias = *b;
          chain.push_back(add);
          cur = nodes_[add].out[0];
        }
      }
      // [erf-GELU]: Div(x, sqrt2) -> Erf -> Add(., 1) -> Mul(x, .) -> Mul(., 0.5)
      {
        const Val& cv = vals_[cur];
        if (cv.consumers.size() == 2 && !is_requested(cur)) {
          int dv = -1, mx = -1;
          for (int c : cv.consumers) {
            if (nodes_[c].op == "Div" && nodes_[c].in[0] == cur) dv = c;
            else if (nodes_[c].op == "Mul") mx = c;
          }
          float k = 0;
          if (dv >= 0 && mx >= 0 && scalar_f32(init_of(nodes_[dv].in[1]), &k) &&
              k == 1.41421353816986083984375f) {
            const int er = sole_consumer(nodes_[dv].out[0]);
            const int a1 = er >= 0 && nodes_[er].op == "Erf" ? sole_consumer(nodes_[er].out[0]) : -1;
            const std::string* one = a1 >= 0 && nodes_[a1].op == "Add" ? other(nodes_[a1], nodes_[er].out[0]) : nullptr;
            float kv = 0;
            if (one && scalar_f32(init_of(*one), &kv) && kv == 1.0f) {
              const int m1 = sole_consumer(nodes_[a1].out[0]);
              // Mul(x, 1+erf) then Mul(., 0.5)
              if (m1 == mx && other(nodes_[mx], nodes_[a1].out[0]) && *other(nodes_[mx], nodes_[a1].out[0]) == cur) {
                const int m2 = sole_consumer(nodes_[mx].out[0]);
                const std::string* h = m2 >= 0 && nodes_[m2].op == "Mul" ? other(nodes_[m2], nodes_[mx].out[0]) : nullptr;
                float hv = 0;
                if (h && scalar_f32(init_of(*h), &hv) && hv == 0.5f) {
                  for (int c : {dv, er, a1, mx, m2}) chain.push_back(c);
                  f.gelu = true;
                  cur = nodes_[m2].out[0];
                }
              }
            }
          }
        }
      }
      // [residual Add(out, r)] with r ready before this kernel runs
      if (!f.gelu && sole_consumer(cur) >= 0 && !is_requested(cur)) {
        const int ra = sole_consumer(cur);
        const std::string* r = nodes_[ra].op == "Add" ? other(nodes_[ra], cur) : nullptr;
        if (r && *r != cur) {
          const Val& rv = vals_[*r];
          const int rp = rv.producer;
          const bool ready = rv.is_input || rv.init || (rp >= 0 && pos_of(rp) < pos_of(idx));
          if (ready && rv.dtype == ICX_F32 && rv.shape == vals_[cur].shape) {
            f.residual = *r;
            chain.push_back(ra);
            cur = nodes_[ra].out[0];
          }
        }
      }
      // [LayerNormalization] of the residual sum over its last axis, done by
      // a cluster of the GEMM's CTAs that together hold whole rows
      if (!f.residual.empty() && ln_fuse_enabled() && sole_consumer(cur) >= 0 && !is_requested(cur)) {
        const int ln = sole_consumer(cur);
        const NodeDef& L = nodes_[ln];
        const Init* g = L.op == "LayerNormalization" && L.in.size() >= 2 ? init_of(L.in[1]) : nullptr;
        const Init* b = L.in.size() > 2 && !L.in[2].empty() ? init_of(L.in[2]) : nullptr;
        const int64_t axis = L.op == "LayerNormalization" ? L.geti("axis", -1) : 0;
        const int64_t rank = (int64_t)vals_[cur].shape.size();
        bool only_y = true;
        for (size_t k = 1; k < L.out.size(); ++k) only_y = only_y && L.out[k].empty();
        if (g && L.in[0] == cur && g->dtype == ICX_F32 && numel(g->shape) == N &&
            (L.in.size() <= 2 || L.in[2].empty() || (b && b->dtype == ICX_F32 && numel(b->shape) == N)) &&
            (axis == -1 || axis == rank - 1) && only_y &&
            quant_linear_ln_preferred((size_t)(numel(vals_[cur].shape) / N), (size_t)w->shape[0], (size_t)N)) {
          f.ln_gamma = L.in[1];
          f.ln_beta = L.in.size() > 2 ? L.in[2] : std::string();
          f.ln_eps = L.getf("epsilon", 1e-5f);
          chain.push_back(ln);
          cur = L.out[0];
        }
      }
      f.out = cur;
      for (int c : chain) skip_.insert(c);
      // the scale product is computed inside the kernel when nothing else reads it
      if (vals_[*sc].consumers.size() == 1 && !is_requested(*sc)) skip_.insert(smul);
      fused_[idx] = f;
      skip_.erase(idx);  // the MatMulInteger position runs the fused kernel
    }
    fuse_attention();
    merge_qkv();
    // intermediates of fused chains are never materialised
    for (int idx : order_) {
      if (!skip_.count(idx)) continue;
      for (auto& o : nodes_[idx].out) vals_[o].needed = false;
    }
    for (auto& kv : fused_) {
      for (auto& o : nodes_[kv.first].out) vals_[o].needed = false;
      vals_[kv.second.out].needed = true;
    }
    for (auto& kv : fused_)
      for (auto& part : kv.second.parts) vals_[part.out].needed = false;
    for (auto& kv : attn_) {
      const FusedAttn& a = kv.second;
      // scratch for scores / probabilities (cuBLAS path only)
      vals_[a.scores].needed = !attention_supported(a.dh, a.ld ? a.ld : a.H, a.H);
      Val& o = vals_[kv.second.out];
      o.needed = true;
      o.alias.clear();
    }
    // producer-fused min/max for DynamicQuantizeLinear
    int slot = 0;
    wide_parts_ = 0;
    for (int idx : order_) {
      const NodeDef& d = nodes_[idx];
      if (d.op != "DynamicQuantizeLinear" || skip_.count(idx)) continue;
      Val& x = vals_[d.in[0]];
      if (x.producer < 0 || x.minmax_slot >= 0) {
        if (x.minmax_slot >= 0) dql_mode_[idx] = x.minmax_slot;
        continue;
      }
      const NodeDef& p = nodes_[x.producer];
      bool ok = p.op == "LayerNormalization";
      for (auto& kv : fused_)
        if (kv.second.out == d.in[0]) ok = true;
      for (auto& kv : attn_) {
        const FusedAttn& a = kv.second;
        if (a.out == d.in[0] && attention_supported(a.dh, a.ld ? a.ld : a.H, a.H)) {
          ok = true;
          // more partials than a slot holds: they go to a wider buffer and
          // are folded into the slot's single pair after the kernel
          const size_t parts = (size_t)attention_partials(a.B, a.S, a.nh);
          if (parts > (size_t)ICX_MAX_MINMAX_PARTIALS) wide_parts_ = std::max(wide_parts_, parts);
        }
      }
      if (!ok) continue;
      x.minmax_slot = slot;
      dql_mode_[idx] = slot;
      ++slot;
    }
    n_slots_ = slot;
  }

  // Reshape(t, [0, 0, nh, dh]) -> Transpose(perm) feeding `use`: returns t.
  bool head_split(const std::string& v, const std::vector<int64_t>& perm, std::string* src,
                  std::vector<int>* chain) {
    const int tr = producer_op(v, "Transpose");
    if (tr < 0 || sole_consumer(v) < 0 || is_requested(v)) return false;
    const auto* p = nodes_[tr].getints("perm");
    if (!p || *p != perm) return false;
    const int rs = producer_op(nodes_[tr].in[0], "Reshape");
    if (rs < 0 || sole_consumer(nodes_[tr].in[0]) != tr || is_requested(nodes_[tr].in[0])) return false;
    const Val& x = vals_[nodes_[rs].in[0]];
    const Val& r = vals_[nodes_[rs].out[0]];
    if (x.dtype != ICX_F32 || x.shape.size() != 3 || r.shape.size() != 4) return false;
    if (r.shape[0] != x.shape[0] || r.shape[1] != x.shape[1] || r.shape[2] * r.shape[3] != x.shape[2])
      return false;
    *src = nodes_[rs].in[0];
    chain->push_back(rs);
    chain->push_back(tr);
    return true;
  }

  void fuse_attention() {
    for (int idx : order_) {
      const NodeDef& sm = nodes_[idx];
      if (sm.op != "Softmax" || skip_.count(idx)) continue;
      std::vector<int> chain{idx};
      FusedAttn a;
      std::string x = sm.in[0];
      const int add = producer_op(x, "Add");
      std::string divout = x;
      if (add >= 0) {
        if (sole_consumer(x) != idx || is_requested(x)) continue;
        const NodeDef& an = nodes_[add];
        const int d0 = producer_op(an.in[0], "Div"), d1 = producer_op(an.in[1], "Div");
        const int which = d0 >= 0 ? 0 : (d1 >= 0 ? 1 : -1);
        if (which < 0) continue;
        divout = an.in[which];
        a.mask = an.in[1 - which];
        chain.push_back(add);
      }
      const int dv = producer_op(divout, "Div");
      if (dv < 0 || sole_consumer(divout) != (add >= 0 ? add : idx) || is_requested(divout)) continue;
      if (!scalar_f32(init_of(nodes_[dv].in[1]), &a.c)) continue;
      chain.push_back(dv);
      a.scores = nodes_[dv].in[0];
      const int mm1 = producer_op(a.scores, "MatMul");
      if (mm1 < 0 || sole_consumer(a.scores) != dv || is_requested(a.scores)) continue;
      chain.push_back(mm1);
      if (!head_split(nodes_[mm1].in[0], {0, 2, 1, 3}, &a.q, &chain)) continue;
      if (!head_split(nodes_[mm1].in[1], {0, 2, 3, 1}, &a.k, &chain)) continue;
      const int mm2 = sole_consumer(sm.out[0]);
      if (mm2 < 0 || nodes_[mm2].op != "MatMul" || nodes_[mm2].in[0] != sm.out[0] || is_requested(sm.out[0]))
        continue;
      chain.push_back(mm2);
      if (!head_split(nodes_[mm2].in[1], {0, 2, 1, 3}, &a.v, &chain)) continue;
      const int tr = sole_consumer(nodes_[mm2].out[0]);
      if (tr < 0 || nodes_[tr].op != "Transpose" || is_requested(nodes_[mm2].out[0])) continue;
      const auto* perm = nodes_[tr].getints("perm");
      if (!perm || *perm != std::vector<int64_t>{0, 2, 1, 3}) continue;
      chain.push_back(tr);
      const int rs = sole_consumer(nodes_[tr].out[0]);
      if (rs < 0 || nodes_[rs].op != "Reshape" || is_requested(nodes_[tr].out[0])) continue;
      const Val& qv = vals_[a.q];
      const Val& sv = vals_[a.scores];
      const Val& ov = vals_[nodes_[rs].out[0]];
      a.B = qv.shape[0];
      a.S = qv.shape[1];
      a.H = qv.shape[2];
      a.nh = sv.shape[1];
      a.dh = a.H / a.nh;
      if (vals_[a.k].shape != qv.shape || vals_[a.v].shape != qv.shape || ov.shape != qv.shape ||
          sv.shape != Shape({a.B, a.nh, a.S, a.S}))
        continue;
      if (!a.mask.empty()) {
        const Shape& ms = vals_[a.mask].shape;
        const bool pb = ms == Shape({a.B, 1, 1, a.S});
        const bool shared = ms == Shape({1, 1, 1, a.S}) || ms == Shape({a.S});
        if (!pb && !shared) continue;
        a.mask_per_batch = pb;
      }
      a.out = nodes_[rs].out[0];
      for (int c : chain) skip_.insert(c);
      attn_[rs] = a;
    }
  }

  // Q, K and V projections of one attention block read the same quantised
  // input: run them as ONE GEMM over the concatenated weights [K, 3N]; the
  // attention then reads q / k / v in place with a row stride of 3N.
  void merge_qkv() {
    for (auto& akv : attn_) {
      FusedAttn& a = akv.second;
      int ids[3] = {-1, -1, -1};
      const std::string* outs[3] = {&a.q, &a.k, &a.v};
      for (auto& kv : fused_)
        for (int t = 0; t < 3; ++t)
          if (kv.second.out == *outs[t]) ids[t] = kv.first;
      if (ids[0] < 0 || ids[1] < 0 || ids[2] < 0) continue;
      const FusedQL& f0 = fused_[ids[0]];
      bool ok = true;
      for (int t = 0; t < 3; ++t) {
        const FusedQL& f = fused_[ids[t]];
        if (f.q != f0.q || f.s != f0.s || f.z != f0.z || f.gelu || !f.residual.empty() ||
            f.bias.empty() != f0.bias.empty() || f.bz.empty() != f0.bz.empty() || !f.parts.empty() ||
            vals_[f.out].consumers.size() != 1 || is_requested(f.out) || vals_[f.out].minmax_slot >= 0)
          ok = false;
      }
      if (!ok) continue;
      int first = ids[0];
      for (int t = 1; t < 3; ++t)
        if (pos_of(ids[t]) < pos_of(first)) first = ids[t];
      FusedQL m;
      m.q = f0.q;
      m.s = f0.s;
      m.z = f0.z;
      m.bias = f0.bias.empty() ? "" : "merged";
      m.bz = f0.bz.empty() ? "" : "merged";
      for (int t = 0; t < 3; ++t) m.parts.push_back(fused_[ids[t]]);
      m.w = "qkv:" + m.parts[0].w + "|" + m.parts[1].w + "|" + m.parts[2].w;
      m.out = a.q + "#qkv";
      Val mv;
      mv.dtype = ICX_F32;
      mv.shape = vals_[a.q].shape;
      const int64_t N = mv.shape.back();
      mv.shape.back() = 3 * N;
      mv.producer = first;
      vals_[m.out] = mv;
      for (int t = 0; t < 3; ++t) {
        fused_.erase(ids[t]);
        if (ids[t] != first) skip_.insert(ids[t]);
      }
      fused_[first] = m;
      a.q = a.k = a.v = m.out;
      a.ld = 3 * N;
      a.off_q = 0;
      a.off_k = N;
      a.off_v = 2 * N;
    }
  }

  // ---------------------------------------------------- weights upload
  int upload_weights() {
    for (auto& kv : inits_) {
      Init& in = *kv.second;
      if (in.dev || in.data.empty()) continue;
      ICX_CUDA(cudaMalloc(&in.dev, in.data.size()));
      ICX_CUDA(cudaMemcpy(in.dev, in.data.data(), in.data.size(), cudaMemcpyHostToDevice));
    }
    auto prep = [&](const std::string& wname) -> int {
      if (prepared_.count(wname)) return ICX_OK;
      const Init* w = init_of(wname);
      Prepared p;
      p.K = w->shape[0];
      p.N = w->shape[1];
      ICX_CUDA(cudaMalloc(&p.bt, (size_t)(p.K * p.N) + 16));
      ICX_CUDA(cudaMalloc(&p.colsum, (size_t)p.N * 4 + 16));
      int rc = icx_prepare_b(stream_, w->dev, w->dtype, p.K, p.N, p.bt, p.colsum);
      if (rc) return rc;
      prepared_[wname] = p;
      return ICX_OK;
    };
    for (auto& kv : fused_) {
      const FusedQL& f = kv.second;
      if (f.parts.empty()) {
        int rc = prep(f.w);
        if (rc) return rc;
        continue;
      }
      if (prepared_.count(f.w)) continue;
      Prepared m;
      m.K = init_of(f.parts[0].w)->shape[0];
      for (auto& part : f.parts) {
        int rc = prep(part.w);
        if (rc) return rc;
        m.N += prepared_[part.w].N;
      }
      ICX_CUDA(cudaMalloc(&m.bt, (size_t)(m.K * m.N) + 16));
      ICX_CUDA(cudaMalloc(&m.colsum, (size_t)m.N * 4 + 16));
      std::vector<float> ws, bias;
      std::vector<int8_t> bz;
      int64_t n0 = 0;
      for (auto& part : f.parts) {
        const Prepared& p = prepared_[part.w];
        ICX_CUDA(cudaMemcpy(static_cast<uint8_t*>(m.bt) + n0 * m.K, p.bt, (size_t)(p.N * p.K),
                            cudaMemcpyDeviceToDevice));
        ICX_CUDA(cudaMemcpy(m.colsum + n0, p.colsum, (size_t)p.N * 4, cudaMemcpyDeviceToDevice));
        const Init* wsi = init_of(part.ws);
        for (int64_t j = 0; j < p.N; ++j)
          ws.push_back(reinterpret_cast<const float*>(wsi->data.data())[numel(wsi->shape) > 1 ? j : 0]);
        if (!part.bias.empty()) {
          const Init* bi = init_of(part.bias);
          const float* bp = reinterpret_cast<const float*>(bi->data.data());
          bias.insert(bias.end(), bp, bp + p.N);
        }
        if (!part.bz.empty()) {
          const Init* zi = init_of(part.bz);
          for (int64_t j = 0; j < p.N; ++j)
            bz.push_back(reinterpret_cast<const int8_t*>(zi->data.data())[numel(zi->shape) > 1 ? j : 0]);
        }
        n0 += p.N;
      }
      ICX_CUDA(cudaMalloc(&m.ws, ws.size() * 4));
      ICX_CUDA(cudaMemcpy(m.ws, ws.data(), ws.size() * 4, cudaMemcpyHostToDevice));
      if (!bias.empty()) {
        ICX_CUDA(cudaMalloc(&m.bias, bias.size() * 4));
        ICX_CUDA(cudaMemcpy(m.bias, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice));
      }
      if (!bz.empty()) {
        ICX_CUDA(cudaMalloc(&m.bz, bz.size() + 16));
        ICX_CUDA(cudaMemcpy(m.bz, bz.data(), bz.size(), cudaMemcpyHostToDevice));
      }
      prepared_[f.w] = m;
    }
    for (int idx : order_) {
      if (skip_.count(idx) || fused_.count(idx)) continue;
      const NodeDef& n = nodes_[idx];
      if (n.op == "MatMulInteger") {
        const Init* w = init_of(n.in[1]);
        if (w && w->shape.size() == 2) {
          int rc = prep(n.in[1]);
          if (rc) return rc;
        }
      }
    }
    if (!err_flag_) {
      ICX_CUDA(cudaMalloc(&err_flag_, sizeof(int)));
      ICX_CUDA(cudaMemset(err_flag_, 0, sizeof(int)));
    }
    ICX_CUDA(cudaStreamSynchronize(stream_));
    return ICX_OK;
  }

  // ------------------------------------------------------ memory plan
  std::string root(const std::string& v) {
    std::string r = v;
    while (!vals_[r].alias.empty()) r = vals_[r].alias;
    return r;
  }

  int plan_memory(const std::vector<std::string>& outputs) {
    // lifetimes in step units (position in order_)
    std::map<std::string, std::pair<int, int>> life;  // root -> [def, last use]
    const int end = (int)order_.size() + 1;
    // graph inputs keep their slot for the whole plan so replay() can
    // re-read the inputs of the last run
    for (auto& nm : inputs_) life[nm] = {-1, end};
    for (int pos = 0; pos < (int)order_.size(); ++pos) {
      const int idx = order_[pos];
      const NodeDef& n = nodes_[idx];
      auto fit = fused_.find(idx);
      if (fit != fused_.end()) {
        // the fused kernel runs here: it writes its final output and reads
        // the quantised input, scale and zero point at this position
        const FusedQL& f = fit->second;
        if (!life.count(f.out)) life[f.out] = {pos, pos};
        for (const std::string* i : {&f.q, &f.s, &f.z, &f.residual}) {
          if (i->empty()) continue;
          const std::string r = root(*i);
          auto it = life.find(r);
          if (it != life.end()) it->second.second = std::max(it->second.second, pos);
        }
      }
      auto ait = attn_.find(idx);
      if (ait != attn_.end()) {
        const FusedAttn& at = ait->second;
        if (vals_[at.scores].needed && !life.count(at.scores)) life[at.scores] = {pos, pos};
        for (const std::string* i : {&at.q, &at.k, &at.v, &at.mask}) {
          if (i->empty()) continue;
          const std::string r = root(*i);
          auto it = life.find(r);
          if (it != life.end()) it->second.second = std::max(it->second.second, pos);
        }
      }
      for (auto& o : n.out) {
        const Val& v = vals_[o];
        if (!v.needed || !v.alias.empty()) continue;
        if (!life.count(o)) life[o] = {pos, pos};
      }
      for (auto& i : n.in) {
        if (i.empty()) continue;
        const std::string r = root(i);
        if (vals_[r].init) continue;
        auto it = life.find(r);
        if (it != life.end()) it->second.second = std::max(it->second.second, pos);
      }
    }
    for (auto& o : outputs) {
      const std::string r = root(o);
      if (life.count(r)) life[r].second = end;
    }
    struct Item { std::string name; int a, b; size_t bytes; int64_t off; };
    std::vector<Item> items;
    for (auto& kv : life) {
      const Val& v = vals_[kv.first];
      if (v.init) continue;
      size_t bytes = (size_t)numel(v.shape) * dtype_size(v.dtype);
      bytes = (bytes + 255) & ~size_t(255);
      if (bytes == 0) bytes = 256;
      items.push_back({kv.first, kv.second.first, std::max(kv.second.second, kv.second.first), bytes, -1});
    }
    std::sort(items.begin(), items.end(), [](const Item& x, const Item& y) {
      return x.bytes != y.bytes ? x.bytes > y.bytes : x.name < y.name;
    });
    size_t total = 0;
    for (size_t i = 0; i < items.size(); ++i) {
      std::vector<std::pair<int64_t, int64_t>> busy;
      for (size_t j = 0; j < i; ++j)
        if (!(items[j].b < items[i].a || items[i].b < items[j].a))
          busy.push_back({items[j].off, items[j].off + (int64_t)items[j].bytes});
      std::sort(busy.begin(), busy.end());
      int64_t off = 0;
      for (auto& b : busy) {
        if (off + (int64_t)items[i].bytes <= b.first) break;
        off = std::max(off, b.second);
      }
      items[i].off = off;
      total = std::max(total, (size_t)off + items[i].bytes);
    }
    // (min, max) partial slots and DQL workspaces live at the end
    const size_t slot_bytes = (size_t)ICX_MAX_MINMAX_PARTIALS * 8;
    slots_off_ = total;
    total += slot_bytes * (size_t)(n_slots_ + 1);
    wide_off_ = total;
    if (wide_parts_ > 0) total += wide_parts_ * 8 + 512;  // partials, then the folded pair
    if (total > arena_bytes_) {
      if (arena_) cudaFree(arena_);
      arena_ = nullptr;
      ICX_CUDA(cudaMalloc(&arena_, total));
      arena_bytes_ = total;
    }
    for (auto& it : items) vals_[it.name].ptr = static_cast<uint8_t*>(arena_) + it.off;
    for (auto& kv : vals_)
      if (!kv.second.alias.empty()) kv.second.ptr = nullptr;
    minmax_count_.assign(n_slots_, 1);
    return ICX_OK;
  }

  float* slot_ptr(int slot) {
    return reinterpret_cast<float*>(static_cast<uint8_t*>(arena_) + slots_off_ +
                                    (size_t)slot * ICX_MAX_MINMAX_PARTIALS * 8);
  }
  float* dql_workspace() { return slot_ptr(n_slots_); }
  float* wide_partials() {
    return reinterpret_cast<float*>(static_cast<uint8_t*>(arena_) + wide_off_);
  }

  // --------------------------------------------------------- step build
  int build_steps() {
    launches_per_run_ = 0;
    for (int idx : order_) {
      if (skip_.count(idx)) continue;
      const NodeDef& n = nodes_[idx];
      auto fit = fused_.find(idx);
      auto ait = attn_.find(idx);
      int rc = fit != fused_.end()   ? step_fused(idx, fit->second)
               : ait != attn_.end() ? step_attention(idx, ait->second)
                                    : step_node(idx);
      if (rc) return rc;
    }
    return ICX_OK;
  }

  void add_step(const NodeDef& n, const std::string& op, const std::string& out,
                std::function<int(cudaStream_t)> fn, int launches) {
    std::string info;
    for (size_t k = 0; k < n.in.size(); ++k) info += (k ? "," : "in=") + n.in[k];
    info += ";outs=";
    for (size_t k = 0; k < n.out.size(); ++k) info += (k ? "," : "") + n.out[k];
    steps_.push_back({n.name, op, out, std::move(fn), info});
    launches_per_run_ += launches;
  }

  int step_fused(int idx, const FusedQL& f) {
    const NodeDef& n = nodes_[idx];
    const Prepared& p = prepared_.at(f.w);
    const Val& q = vals_[f.q];
    const int64_t K = q.shape.back();
    const int64_t M = numel(q.shape) / (K ? K : 1);
    const bool merged = !f.parts.empty();
    const Init* ws = merged ? nullptr : init_of(f.ws);
    const Init* bz = merged || f.bz.empty() ? nullptr : init_of(f.bz);
    const Init* bias = merged || f.bias.empty() ? nullptr : init_of(f.bias);
    uint8_t* qp = static_cast<uint8_t*>(resolve(f.q));
    float* sp = static_cast<float*>(resolve(f.s));
    uint8_t* zp = static_cast<uint8_t*>(resolve(f.z));
    float* out = static_cast<float*>(resolve(f.out));
    const int slot = vals_[f.out].minmax_slot;
    float* mm = slot >= 0 ? slot_ptr(slot) : nullptr;
    int* mmc = slot >= 0 ? &minmax_count_[slot] : nullptr;
    const bool has_bz = !f.bz.empty();
    const int32_t* rows = has_bz ? rowsum_for(f.q, M) : nullptr;
    const bool gelu = f.gelu;
    const float* wsp = merged ? p.ws : static_cast<const float*>(ws->dev);
    const int ws_pc = merged ? 1 : numel(ws->shape) > 1;
    const int8_t* bzp = merged ? p.bz : (bz ? static_cast<const int8_t*>(bz->dev) : nullptr);
    const int bz_pc = merged ? 1 : (bz && numel(bz->shape) > 1);
    const float* bp = merged ? p.bias : (bias ? static_cast<const float*>(bias->dev) : nullptr);
    Prepared pw = p;
    const float* res = f.residual.empty() ? nullptr : static_cast<const float*>(resolve(f.residual));
    const bool ln = !f.ln_gamma.empty();
    const std::string label = gelu ? "QuantLinear+GELU"
                              : ln ? "QuantLinear+Residual+LayerNorm"
                              : res ? "QuantLinear+Residual"
                              : merged ? "QuantLinear(QKV)" : "QuantLinear";
    if (ln) {
      const float* gp = static_cast<const float*>(init_of(f.ln_gamma)->dev);
      const float* bp2 = f.ln_beta.empty() ? nullptr : static_cast<const float*>(init_of(f.ln_beta)->dev);
      const float eps = f.ln_eps;
      add_step(n, label, f.out, [=](cudaStream_t s) {
        return icx_quant_linear_layernorm(s, qp, sp, zp, rows, static_cast<const int8_t*>(pw.bt),
                                          pw.colsum, (size_t)M, (size_t)K, (size_t)pw.N, wsp, ws_pc,
                                          bzp, bz_pc, bp, res, gp, bp2, eps, out, mm, mmc);
      }, 1);
    } else {
      add_step(n, label, f.out, [=](cudaStream_t s) {
        return icx_quant_linear(s, qp, sp, zp, rows, static_cast<const int8_t*>(pw.bt), pw.colsum,
                                (size_t)M, (size_t)K, (size_t)pw.N, wsp, ws_pc, bzp, bz_pc, bp,
                                gelu ? 1 : 0, res, out, mm, mmc);
      }, 1);
    }
    // the weights of the step by their initializer names (merged: one
    // '|'-separated entry per part, in column order)
    std::string w, wsn, bzn, bn;
    const std::vector<FusedQL> single{f};
    const std::vector<FusedQL>& parts = merged ? f.parts : single;
    for (size_t k = 0; k < parts.size(); ++k) {
      const char* sep = k ? "|" : "";
      w += sep + parts[k].w;
      wsn += sep + parts[k].ws;
      bzn += sep + parts[k].bz;
      bn += sep + parts[k].bias;
    }
    steps_.back().info = "q=" + f.q + ";s=" + f.s + ";z=" + f.z + ";w=" + w + ";ws=" + wsn +
                         ";bz=" + bzn + ";bias=" + bn + ";residual=" + f.residual +
                         ";gelu=" + (gelu ? "1" : "0") + ";out=" + f.out;
    if (ln) {
      char eb[32];
      snprintf(eb, sizeof(eb), "%.9g", (double)f.ln_eps);
      steps_.back().info += ";ln_gamma=" + f.ln_gamma + ";ln_beta=" + f.ln_beta + ";ln_eps=" + eb;
    }
    return ICX_OK;
  }

  // Attention without any transpose: two pointer-array batched SGEMMs read
  // Q, K, V in place from [B, S, H] (head h is the column block h*dh) and
  // write the context straight back into [B, S, H]; between them one kernel
  // applies Div(c), Add(mask) and Softmax with the rounding of those ops.
  static std::string attention_info(const FusedAttn& a) {
    char buf[256];
    snprintf(buf, sizeof(buf), ";ld=%lld;off_q=%lld;off_k=%lld;off_v=%lld;c=%.9g;B=%lld;S=%lld;H=%lld;nh=%lld",
             (long long)(a.ld ? a.ld : a.H), (long long)a.off_q, (long long)a.off_k,
             (long long)a.off_v, (double)a.c, (long long)a.B, (long long)a.S, (long long)a.H,
             (long long)a.nh);
    return "q=" + a.q + ";k=" + a.k + ";v=" + a.v + ";mask=" + a.mask +
           ";mask_per_batch=" + (a.mask_per_batch ? "1" : "0") + buf + ";out=" + a.out;
  }

  int step_attention(int idx, const FusedAttn& a) {
    const int rc = step_attention_impl(idx, a);
    if (rc == ICX_OK) steps_.back().info = attention_info(a);
    return rc;
  }

  int step_attention_impl(int idx, const FusedAttn& a) {
    const NodeDef& n = nodes_[idx];
    if (attention_supported(a.dh, a.ld ? a.ld : a.H, a.H)) {
      const float* q = static_cast<const float*>(resolve(a.q)) + a.off_q;
      const float* k = static_cast<const float*>(resolve(a.k)) + a.off_k;
      const float* v = static_cast<const float*>(resolve(a.v)) + a.off_v;
      float* out = static_cast<float*>(resolve(a.out));
      const float* mask = a.mask.empty() ? nullptr : static_cast<const float*>(resolve(a.mask));
      const FusedAttn at = a;
      const int64_t ld = a.ld ? a.ld : a.H;
      const int slot = vals_[a.out].minmax_slot;
      float* mm = slot >= 0 ? slot_ptr(slot) : nullptr;
      int* mmc = slot >= 0 ? &minmax_count_[slot] : nullptr;
      const int parts = attention_partials(a.B, a.S, a.nh);
      if (mm != nullptr && parts > ICX_MAX_MINMAX_PARTIALS) {
        // (min, max) is order-independent, so folding the per-CTA partials
        // into one pair leaves the DynamicQuantizeLinear result unchanged
        float* wide = wide_partials();
        float* g = wide + ((size_t)parts * 2 + 63) / 64 * 64;
        add_step(n, "Attention", a.out, [=](cudaStream_t s) {
          int written = 0;
          int rc = launch_attention_f32(s, q, k, v, ld, out, at.B, at.S, at.H, at.nh, at.c, mask,
                                        at.mask_per_batch, wide, &written);
          if (rc == ICX_OK) rc = launch_minmax_fold(s, wide, written, g);
          if (rc == ICX_OK) rc = launch_minmax_unfold(s, g, mm);
          *mmc = 1;
          return rc;
        }, 3);
        return ICX_OK;
      }
      add_step(n, "Attention", a.out, [=](cudaStream_t s) {
        return launch_attention_f32(s, q, k, v, ld, out, at.B, at.S, at.H, at.nh, at.c, mask,
                                    at.mask_per_batch, mm, mmc);
      }, 1);
      return ICX_OK;
    }
    const int64_t nb = a.B * a.nh;
    std::vector<const float*> hA1(nb), hB1(nb), hA2(nb), hB2(nb);
    std::vector<float*> hC1(nb), hC2(nb);
    const float* q = static_cast<const float*>(resolve(a.q));
    const float* k = static_cast<const float*>(resolve(a.k));
    const float* v = static_cast<const float*>(resolve(a.v));
    float* sc = static_cast<float*>(resolve(a.scores));
    float* out = static_cast<float*>(resolve(a.out));
    for (int64_t b = 0; b < a.B; ++b)
      for (int64_t h = 0; h < a.nh; ++h) {
        const int64_t i = b * a.nh + h;
        const int64_t ld = a.ld ? a.ld : a.H;
        const int64_t in_off = b * a.S * ld + h * a.dh;
        const int64_t out_off = b * a.S * a.H + h * a.dh;
        hA1[i] = k + in_off + a.off_k;
        hB1[i] = q + in_off + a.off_q;
        hC1[i] = sc + i * a.S * a.S;
        hA2[i] = v + in_off + a.off_v;
        hB2[i] = sc + i * a.S * a.S;
        hC2[i] = out + out_off;
      }
    void* dptr = nullptr;
    ICX_CUDA(cudaMalloc(&dptr, (size_t)nb * 6 * sizeof(void*)));
    scratch_.push_back(dptr);
    void** d = static_cast<void**>(dptr);
    const size_t pb = (size_t)nb * sizeof(void*);
    ICX_CUDA(cudaMemcpy(d + 0 * nb, hA1.data(), pb, cudaMemcpyHostToDevice));
    ICX_CUDA(cudaMemcpy(d + 1 * nb, hB1.data(), pb, cudaMemcpyHostToDevice));
    ICX_CUDA(cudaMemcpy(d + 2 * nb, hC1.data(), pb, cudaMemcpyHostToDevice));
    ICX_CUDA(cudaMemcpy(d + 3 * nb, hA2.data(), pb, cudaMemcpyHostToDevice));
    ICX_CUDA(cudaMemcpy(d + 4 * nb, hB2.data(), pb, cudaMemcpyHostToDevice));
    ICX_CUDA(cudaMemcpy(d + 5 * nb, hC2.data(), pb, cudaMemcpyHostToDevice));
    const float* mask = a.mask.empty() ? nullptr : static_cast<const float*>(resolve(a.mask));
    const FusedAttn at = a;
    const int64_t lda = a.ld ? a.ld : a.H;
    cublasHandle_t hdl = blas_;
    add_step(n, "Attention", a.out, [=](cudaStream_t s) {
      const float one = 1.0f, zero = 0.0f;
      // scores[b,h] (row-major S x S) = Q_bh K_bh^T
      cublasStatus_t st = cublasSgemmBatched(
          hdl, CUBLAS_OP_T, CUBLAS_OP_N, (int)at.S, (int)at.S, (int)at.dh, &one,
          reinterpret_cast<const float* const*>(d + 0 * nb), (int)lda,
          reinterpret_cast<const float* const*>(d + 1 * nb), (int)lda, &zero,
          reinterpret_cast<float* const*>(d + 2 * nb), (int)at.S, (int)nb);
      if (st != CUBLAS_STATUS_SUCCESS) {
        set_error("cublasSgemmBatched (scores) failed (%d)", (int)st);
        return ICX_ERR_CUDA;
      }
      int rc = launch_scale_mask_softmax(s, sc, sc, (size_t)(nb * at.S), (size_t)at.S, at.c, mask,
                                         at.mask_per_batch ? (size_t)(at.nh * at.S) : 0);
      if (rc) return rc;
      // ctx[b, :, h*dh:(h+1)*dh] = P_bh V_bh
      st = cublasSgemmBatched(hdl, CUBLAS_OP_N, CUBLAS_OP_N, (int)at.dh, (int)at.S, (int)at.S, &one,
                              reinterpret_cast<const float* const*>(d + 3 * nb), (int)lda,
                              reinterpret_cast<const float* const*>(d + 4 * nb), (int)at.S, &zero,
                              reinterpret_cast<float* const*>(d + 5 * nb), (int)at.H, (int)nb);
      if (st != CUBLAS_STATUS_SUCCESS) {
        set_error("cublasSgemmBatched (context) failed (%d)", (int)st);
        return ICX_ERR_CUDA;
      }
      return ICX_OK;
    }, 3);
    return ICX_OK;
  }

  // row sums of a DQL output (needed by per-column weight zero points)
  std::map<std::string, int32_t*> rowsum_bufs_;
  const int32_t* rowsum_for(const std::string& q, int64_t M) {
    auto it = rowsum_bufs_.find(q + "#" + std::to_string(M));
    if (it != rowsum_bufs_.end()) return it->second;
    int32_t* p = nullptr;
    if (cudaMalloc(&p, (size_t)M * 4 + 16) != cudaSuccess) return nullptr;
    rowsum_bufs_[q + "#" + std::to_string(M)] = p;
    return p;
  }

  int step_node(int idx) {
    const NodeDef& n = nodes_[idx];
    const std::string& op = n.op;
    auto shp = [&](size_t k) -> const Shape& { return vals_[n.in[k]].shape; };
    auto ptr = [&](size_t k) -> void* { return k < n.in.size() && !n.in[k].empty() ? resolve(n.in[k]) : nullptr; };
    const std::string& o0 = n.out[0];
    if (!vals_[o0].alias.empty()) return ICX_OK;  // Reshape / Unsqueeze / Squeeze / Identity
    void* out = resolve(o0);
    const Shape oshape = vals_[o0].shape;
    if (op == "Add" || op == "Sub" || op == "Mul" || op == "Div") {
      const int code = op == "Add" ? kAdd : op == "Sub" ? kSub : op == "Mul" ? kMul : kDiv;
      const float* a = static_cast<const float*>(ptr(0));
      const float* b = static_cast<const float*>(ptr(1));
      const Shape as = shp(0), bs = shp(1);
      add_step(n, op, o0, [=](cudaStream_t s) {
        return launch_binary(s, code, a, as, b, bs, static_cast<float*>(out), oshape);
      }, 1);
    } else if (op == "DynamicQuantizeLinear") {
      const float* x = static_cast<const float*>(ptr(0));
      const size_t cnt = (size_t)numel(shp(0));
      uint8_t* y = static_cast<uint8_t*>(out);
      float* sc = static_cast<float*>(resolve(n.out[1]));
      uint8_t* zp = static_cast<uint8_t*>(resolve(n.out[2]));
      // row sums when a fused consumer has a weight zero point
      int32_t* rows = nullptr;
      size_t row_len = 0;
      for (auto& kv : fused_)
        if (kv.second.q == n.out[0] && !kv.second.bz.empty()) {
          row_len = (size_t)shp(0).back();
          rows = const_cast<int32_t*>(rowsum_for(n.out[0], (int64_t)(cnt / (row_len ? row_len : 1))));
        }
      auto mit = dql_mode_.find(idx);
      if (comm_) {
        // global: local partials -> (-min, max) -> MAX all-reduce over the
        // executors -> one (min, max) partial -> the quantise pass
        const bool producer = mit != dql_mode_.end();
        float* mm = producer ? slot_ptr(mit->second) : dql_workspace();
        const int* mmc = producer ? &minmax_count_[mit->second] : nullptr;
        float* g = gdql_;
        ncclComm_t comm = comm_;
        const NcclApi* api = nccl_api();
        add_step(n, "DynamicQuantizeLinear(global)", o0, [=](cudaStream_t s) {
          int nparts;
          if (producer) {
            nparts = *mmc;
          } else {
            const int rc = launch_dql_minmax(s, x, cnt, reinterpret_cast<float2*>(mm));
            if (rc) return rc;
            nparts = dql_minmax_partials(cnt);
          }
          int rc = launch_minmax_fold(s, mm, nparts, g);
          if (rc) return rc;
          const ncclResult_t r = api->all_reduce(g, g, 2, ncclFloat32, ncclMax, comm, s);
          if (r != ncclSuccess) {
            set_error("ncclAllReduce failed: %s", api->error_string(r));
            return ICX_ERR_CUDA;
          }
          rc = launch_minmax_unfold(s, g, g + 2);
          if (rc) return rc;
          return icx_dql_quantize_f32_u8(s, x, cnt, g + 2, 1, y, sc, zp, rows, row_len);
        }, (producer ? 3 : 4) + (rows ? 1 : 0));
      } else if (mit != dql_mode_.end()) {
        const float* mm = slot_ptr(mit->second);
        const int* mmc = &minmax_count_[mit->second];
        add_step(n, "DynamicQuantizeLinear(quantise)", o0, [=](cudaStream_t s) {
          return icx_dql_quantize_f32_u8(s, x, cnt, mm, *mmc, y, sc, zp, rows, row_len);
        }, rows ? 2 : 1);
      } else {
        float* ws = dql_workspace();
        add_step(n, op, o0, [=](cudaStream_t s) {
          return icx_dql_f32_u8(s, x, cnt, y, sc, zp, rows, row_len, ws,
                                (size_t)ICX_MAX_MINMAX_PARTIALS * 8);
        }, 2);
      }
    } else if (op == "MatMulInteger") {
      const Val& a = vals_[n.in[0]];
      const Val& b = vals_[n.in[1]];
      const int64_t K = a.shape.back(), N = b.shape[1];
      const int64_t M = numel(a.shape) / (K ? K : 1);
      const void* ap = ptr(0);
      const void* azp = n.in.size() > 2 ? ptr(2) : nullptr;
      const void* bzp = n.in.size() > 3 ? ptr(3) : nullptr;
      const int bz_pc = bzp && numel(shp(3)) > 1;
      const int at = a.dtype, bt = b.dtype;
      auto pit = prepared_.find(n.in[1]);
      if (pit != prepared_.end()) {
        const Prepared p = pit->second;
        const int32_t* rows = nullptr;
        if (bzp) rows = rowsum_for(n.in[0] + "#mmi", M);
        int32_t* rws = const_cast<int32_t*>(rows);
        add_step(n, op, o0, [=](cudaStream_t s) {
          if (rws) {
            // rows of a for the weight zero-point correction
            int rc = icx_matmul_integer_rowsum(s, ap, at, (size_t)M, (size_t)K, rws);
            if (rc) return rc;
          }
          return icx_matmul_integer_prepared(s, ap, at, p.bt, bt, p.colsum, (size_t)M, (size_t)K,
                                             (size_t)N, azp, bzp, bz_pc, rws,
                                             static_cast<int32_t*>(out));
        }, bzp ? 2 : 1);
      } else {
        const void* bp = ptr(1);
        const size_t wsb = icx_matmul_integer_workspace_bytes(M, K, N);
        void* ws = nullptr;
        ICX_CUDA(cudaMalloc(&ws, wsb));
        scratch_.push_back(ws);
        add_step(n, op, o0, [=](cudaStream_t s) {
          return icx_matmul_integer(s, ap, at, bp, bt, (size_t)M, (size_t)K, (size_t)N, azp, bzp,
                                    bz_pc, static_cast<int32_t*>(out), ws, wsb);
        }, 3);
      }
    } else if (op == "DequantizeLinear") {
      const Val& x = vals_[n.in[0]];
      const Shape xs = x.shape;
      const int64_t sl = numel(shp(1));
      size_t outer = 1, axis_len = 1, inner = (size_t)numel(xs);
      if (sl > 1) {
        int64_t ax = n.geti("axis", 1);
        if (ax < 0) ax += (int64_t)xs.size();
        if (ax < 0 || ax >= (int64_t)xs.size()) return fail(n, "axis out of range");
        if (xs[ax] != sl) return fail(n, "per-axis scale length %lld doesn't match input shape[%lld] = %lld",
                                      (long long)sl, (long long)ax, (long long)xs[ax]);
        outer = (size_t)numel(Shape(xs.begin(), xs.begin() + ax));
        axis_len = (size_t)xs[ax];
        inner = (size_t)numel(Shape(xs.begin() + ax + 1, xs.end()));
      }
      const void* xp = ptr(0);
      const float* sp = static_cast<const float*>(ptr(1));
      const void* zp = n.in.size() > 2 ? ptr(2) : nullptr;
      const int xt = x.dtype;
      add_step(n, op, o0, [=](cudaStream_t s) {
        return icx_dequantize_linear(s, xp, xt, outer, axis_len, inner, sp, (size_t)sl, zp,
                                     static_cast<float*>(out));
      }, 1);
    } else if (op == "Cast") {
      const void* xp = ptr(0);
      const int from = vals_[n.in[0]].dtype, to = vals_[o0].dtype;
      const size_t cnt = (size_t)numel(oshape);
      add_step(n, op, o0, [=](cudaStream_t s) { return launch_cast(s, xp, from, out, to, cnt); }, 1);
    } else if (op == "Erf") {
      const float* xp = static_cast<const float*>(ptr(0));
      const size_t cnt = (size_t)numel(oshape);
      add_step(n, op, o0, [=](cudaStream_t s) { return launch_erf(s, xp, static_cast<float*>(out), cnt); }, 1);
    } else if (op == "Softmax") {
      const float* xp = static_cast<const float*>(ptr(0));
      const size_t D = (size_t)oshape.back(), rows = (size_t)numel(oshape) / (D ? D : 1);
      add_step(n, op, o0, [=](cudaStream_t s) { return launch_softmax(s, xp, static_cast<float*>(out), rows, D); }, 1);
    } else if (op == "LayerNormalization") {
      const float* xp = static_cast<const float*>(ptr(0));
      const float* g = static_cast<const float*>(ptr(1));
      const float* b = n.in.size() > 2 ? static_cast<const float*>(ptr(2)) : nullptr;
      const size_t D = (size_t)oshape.back(), rows = (size_t)numel(oshape) / (D ? D : 1);
      const float eps = n.getf("epsilon", 1e-5f);
      const int slot = vals_[o0].minmax_slot;
      float* mm = slot >= 0 ? slot_ptr(slot) : nullptr;
      int* mmc = slot >= 0 ? &minmax_count_[slot] : nullptr;
      add_step(n, op, o0, [=](cudaStream_t s) {
        return launch_layernorm(s, xp, g, b, static_cast<float*>(out), rows, D, eps, mm, mmc);
      }, 1);
    } else if (op == "Gather") {
      const void* table = ptr(0);
      const int es = (int)dtype_size(vals_[n.in[0]].dtype);
      const int64_t rows = shp(0)[0];
      const size_t D = (size_t)(numel(shp(0)) / (rows ? rows : 1));
      const int64_t* ids = static_cast<const int64_t*>(ptr(1));
      const size_t cnt = (size_t)numel(shp(1));
      int* err = err_flag_;
      add_step(n, op, o0, [=](cudaStream_t s) {
        return launch_gather_rows(s, table, es, rows, ids, cnt, D, out, err);
      }, 1);
    } else if (op == "Transpose") {
      const void* xp = ptr(0);
      const Shape is = shp(0);
      std::vector<int64_t> perm;
      if (const auto* p = n.getints("perm")) perm = *p;
      else for (int64_t d = (int64_t)is.size() - 1; d >= 0; --d) perm.push_back(d);
      const int eb = (int)dtype_size(vals_[o0].dtype);
      add_step(n, op, o0, [=](cudaStream_t s) { return launch_transpose(s, xp, eb, is, perm, out); }, 1);
    } else if (op == "MatMul") {
      const Shape as = shp(0), bs = shp(1);
      const int64_t M = as[as.size() - 2], K = as.back(), N = bs.back();
      const int64_t batch = numel(Shape(oshape.begin(), oshape.end() - 2));
      const long long sa = numel(Shape(as.begin(), as.end() - 2)) > 1 ? (long long)(M * K) : 0;
      const long long sb = numel(Shape(bs.begin(), bs.end() - 2)) > 1 ? (long long)(K * N) : 0;
      const float* a = static_cast<const float*>(ptr(0));
      const float* b = static_cast<const float*>(ptr(1));
      cublasHandle_t h = blas_;
      add_step(n, op, o0, [=](cudaStream_t s) {
        const float one = 1.0f, zero = 0.0f;
        // row-major C = A B  <=>  column-major C^T = B^T A^T
        cublasStatus_t st = cublasSgemmStridedBatched(
            h, CUBLAS_OP_N, CUBLAS_OP_N, (int)N, (int)M, (int)K, &one, b, (int)N, sb, a, (int)K,
            sa, &zero, static_cast<float*>(out),
            (int)N, (long long)M * N, (int)batch);
        if (st != CUBLAS_STATUS_SUCCESS) {
          set_error("cublasSgemmStridedBatched failed (%d)", (int)st);
          return ICX_ERR_CUDA;
        }
        return ICX_OK;
      }, 1);
    } else {
      return fail(n, "unsupported op type");
    }
    return ICX_OK;
  }

  // ------------------------------------------------------------ execute
  int execute() {
    if (use_graphs_ && gexec_) {
      ICX_CUDA(cudaGraphLaunch(gexec_, stream_));
      return ICX_OK;
    }
    if (use_graphs_ && runs_ >= 1) {
      // capture the (already warmed-up) step sequence once, then replay it
      ICX_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
      int rc = run_steps();
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamEndCapture(stream_, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      if (e != cudaSuccess) {
        set_error("graph capture failed: %s", cudaGetErrorString(e));
        return ICX_ERR_CUDA;
      }
      e = cudaGraphInstantiate(&gexec_, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) {
        gexec_ = nullptr;
        set_error("graph instantiate failed: %s", cudaGetErrorString(e));
        return ICX_ERR_CUDA;
      }
      ICX_CUDA(cudaGraphLaunch(gexec_, stream_));
      return ICX_OK;
    }
    ++runs_;
    return run_steps();
  }

  int run_steps() {
    for (auto& st : steps_) {
      int rc = st.fn(stream_);
      if (rc) {
        std::string msg = icx_last_error();
        set_error("op %s (%s) output %s: %s", st.node.c_str(), st.op.c_str(), st.out.c_str(), msg.c_str());
        return rc;
      }
    }
    return ICX_OK;
  }

  // --------------------------------------------------------------- state
  int device_;
  cudaStream_t stream_ = nullptr;
  cublasHandle_t blas_ = nullptr;
  static constexpr size_t kBlasWorkspace = 32u << 20;
  void* blas_ws_ = nullptr;
  std::vector<std::string> inputs_;
  std::map<std::string, std::pair<int, Shape>> input_defs_;
  std::map<std::string, std::unique_ptr<Init>> inits_;
  std::vector<NodeDef> nodes_;

  bool compiled_ = false;
  std::map<std::string, Shape> compiled_shapes_;
  std::vector<std::string> compiled_outputs_;
  std::vector<std::string> pending_outputs_;
  std::vector<int> order_;
  std::unordered_map<std::string, Val> vals_;
  std::map<int, FusedQL> fused_;
  std::map<int, FusedAttn> attn_;
  std::set<int> skip_;
  std::set<std::string> folded_;  // initializers derived at compile (folded / converted)
  // submit / wait: two staging sets of the requested outputs
  struct Pending {
    std::vector<void*> buf;
    std::vector<size_t> cap;
    cudaEvent_t ready = nullptr, done = nullptr;
    // device staging of the submission's inputs (upload stream)
    std::vector<void*> in_buf;
    std::vector<size_t> in_cap;
    cudaEvent_t in_ready = nullptr, in_free = nullptr;
    bool in_used = false;
    bool busy = false;
    int64_t ticket = -1;
  };
  Pending pend_[2];
  cudaStream_t copy_stream_ = nullptr;
  cudaStream_t upload_stream_ = nullptr;
  int64_t next_ticket_ = 0;
  std::atomic<ncclComm_t> comm_{nullptr};  // global DQL (set_global_dql)
  std::atomic<bool> collectives_aborted_{false};
  float* gdql_ = nullptr;      // (-min, max) pair [0..1] and the (min, max) partial [2..3]
  std::map<int, int> dql_mode_;
  int n_slots_ = 0;
  size_t wide_parts_ = 0;  // largest attention partial count above a slot's room
  size_t wide_off_ = 0;
  std::vector<int> minmax_count_;
  std::map<std::string, Prepared> prepared_;
  std::vector<void*> scratch_;
  std::vector<Step> steps_;
  void* arena_ = nullptr;
  size_t arena_bytes_ = 0;
  size_t slots_off_ = 0;
  int* err_flag_ = nullptr;
  bool use_graphs_ = true;
  cudaGraphExec_t gexec_ = nullptr;
  int runs_ = 0;
  int launches_per_run_ = 0;

 public:
  void set_pending_outputs(const std::vector<std::string>& o) { pending_outputs_ = o; }

  // Global DynamicQuantizeLinear: every DQL takes its (min, max) over all
  // `nranks` executors sharing `id` (one per GPU, each with its shard of the
  // batch), so the shards quantise exactly as one executor over the whole
  // batch would.  Every rank must call this concurrently (communicator
  // set-up is collective) and then run the same graph.  nranks <= 1: off.
  // Aborts the global-DQL communicator (ncclCommAbort): all-reduces of this
  // executor that wait for a peer that will never join return, instead of
  // spinning on the GPU forever.  Safe to call from another host thread while
  // this executor's thread is blocked in run(); touches only the
  // communicator.  Afterwards run / submit / replay fail until
  // set_global_dql is called again.
  int abort_global_dql() {
    ncclComm_t c = comm_.exchange(nullptr);
    if (!c) return ICX_OK;
    collectives_aborted_ = true;
    const ncclResult_t r = nccl_api()->comm_abort(c);
    if (r != ncclSuccess) {
      set_error("ncclCommAbort failed: %s", nccl_api()->error_string(r));
      return ICX_ERR_CUDA;
    }
    return ICX_OK;
  }

  int set_global_dql(const void* id, int nranks, int rank) {
    ICX_CUDA(cudaSetDevice(device_));
    collectives_aborted_ = false;
    if (comm_) {
      ICX_CUDA(cudaStreamSynchronize(stream_));
      nccl_api()->comm_destroy(comm_);
      comm_ = nullptr;
    }
    invalidate();
    if (nranks <= 1) return ICX_OK;
    ICX_REQUIRE(id != nullptr && rank >= 0 && rank < nranks, "set_global_dql: bad rank %d of %d",
                rank, nranks);
    const NcclApi* api = nccl_api();
    if (!api) {
      set_error("set_global_dql: libnccl.so.2 could not be loaded");
      return ICX_ERR_UNSUPPORTED;
    }
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    const ncclResult_t r = api->comm_init_rank(&c, nranks, uid, rank);
    if (r != ncclSuccess) {
      set_error("ncclCommInitRank failed: %s", api->error_string(r));
      return ICX_ERR_CUDA;
    }
    comm_ = c;
    if (!gdql_) ICX_CUDA(cudaMalloc(&gdql_, 64));
    return ICX_OK;
  }


};

}  // namespace icx

using icx::Engine;

// ============================================================== C ABI
struct icx_engine {
  std::unique_ptr<Engine> e;
  std::string plan;
};

extern "C" icx_engine* icx_engine_create(int device) {
  icx::clear_error();
  auto h = new icx_engine;
  h->e = std::make_unique<Engine>(device);
  if (h->e->init() != ICX_OK) {
    delete h;
    return nullptr;
  }
  return h;
}

extern "C" void icx_engine_destroy(icx_engine* h) { delete h; }

extern "C" int icx_engine_add_input(icx_engine* h, const char* name, int dtype, int rank,
                                    const int64_t* dims) {
  ICX_REQUIRE(h && name && rank >= 0 && rank <= icx::kMaxRank, "add_input: bad arguments");
  return h->e->add_input(name, dtype, std::vector<int64_t>(dims, dims + rank));
}

extern "C" int icx_engine_add_initializer(icx_engine* h, const char* name, int dtype, int rank,
                                          const int64_t* dims, const void* data) {
  ICX_REQUIRE(h && name && rank >= 0 && rank <= icx::kMaxRank, "add_initializer: bad arguments");
  return h->e->add_initializer(name, dtype, std::vector<int64_t>(dims, dims + rank), data);
}

extern "C" int icx_engine_add_node(icx_engine* h, const char* name, const char* op_type,
                                   int n_in, const char* const* inputs, int n_out,
                                   const char* const* outputs, int n_attrs,
                                   const icx_attr* attrs) {
  ICX_REQUIRE(h && op_type && n_in >= 0 && n_out >= 1, "add_node: bad arguments");
  icx::NodeDef n;
  n.name = name ? name : "";
  n.op = op_type;
  for (int i = 0; i < n_in; ++i) n.in.push_back(inputs[i] ? inputs[i] : "");
  for (int i = 0; i < n_out; ++i) n.out.push_back(outputs[i] ? outputs[i] : "");
  for (int i = 0; i < n_attrs; ++i) {
    icx::Attr a;
    a.kind = attrs[i].kind;
    a.i = attrs[i].i;
    a.f = attrs[i].f;
    if (attrs[i].ints) a.ints.assign(attrs[i].ints, attrs[i].ints + attrs[i].n);
    if (attrs[i].floats) a.floats.assign(attrs[i].floats, attrs[i].floats + attrs[i].n);
    if (attrs[i].s) a.s = attrs[i].s;
    n.attrs[attrs[i].name] = a;
  }
  return h->e->add_node(std::move(n));
}

extern "C" int icx_engine_run(icx_engine* h, int n_in, const char* const* names,
                              const int* dtypes, const int* ranks, const int64_t* dims,
                              const void* const* host, int n_out, const char* const* outputs) {
  ICX_REQUIRE(h && n_in >= 0 && n_out >= 0, "run: bad arguments");
  std::vector<std::string> nm, outs;
  std::vector<int> dt;
  std::vector<std::vector<int64_t>> sh;
  std::vector<const void*> hp;
  size_t off = 0;
  for (int i = 0; i < n_in; ++i) {
    nm.push_back(names[i]);
    dt.push_back(dtypes[i]);
    sh.emplace_back(dims + off, dims + off + ranks[i]);
    off += (size_t)ranks[i];
    hp.push_back(host[i]);
  }
  for (int i = 0; i < n_out; ++i) outs.push_back(outputs[i]);
  h->e->set_pending_outputs(outs);
  return h->e->run(nm, dt, sh, hp, outs);
}

extern "C" int icx_engine_submit(icx_engine* h, int n_in, const char* const* names,
                                 const int* dtypes, const int* ranks, const int64_t* dims,
                                 const void* const* host, int n_out, const char* const* outputs,
                                 void* const* host_out, const size_t* host_out_bytes,
                                 int64_t* ticket) {
  ICX_REQUIRE(h && n_in >= 0 && n_out >= 0 && ticket && (n_out == 0 || (host_out && host_out_bytes)),
              "submit: bad arguments");
  std::vector<std::string> nm, outs;
  std::vector<int> dt;
  std::vector<std::vector<int64_t>> sh;
  std::vector<const void*> hp;
  size_t off = 0;
  for (int i = 0; i < n_in; ++i) {
    nm.push_back(names[i]);
    dt.push_back(dtypes[i]);
    sh.emplace_back(dims + off, dims + off + ranks[i]);
    off += (size_t)ranks[i];
    hp.push_back(host[i]);
  }
  std::vector<void*> ho;
  std::vector<size_t> hb;
  for (int i = 0; i < n_out; ++i) {
    outs.push_back(outputs[i]);
    ho.push_back(host_out[i]);
    hb.push_back(host_out_bytes[i]);
  }
  h->e->set_pending_outputs(outs);
  return h->e->submit(nm, dt, sh, hp, outs, ho, hb, ticket);
}

extern "C" int icx_nccl_unique_id(void* id_out, size_t bytes) {
  ICX_REQUIRE(id_out && bytes >= sizeof(ncclUniqueId), "nccl_unique_id: need %zu bytes",
              sizeof(ncclUniqueId));
  const icx::NcclApi* api = icx::nccl_api();
  if (!api) {
    icx::set_error("nccl_unique_id: libnccl.so.2 could not be loaded");
    return ICX_ERR_UNSUPPORTED;
  }
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) {
    icx::set_error("ncclGetUniqueId failed: %s", api->error_string(r));
    return ICX_ERR_CUDA;
  }
  memcpy(id_out, &id, sizeof(id));
  return ICX_OK;
}

extern "C" int icx_engine_set_global_dql(icx_engine* h, const void* nccl_id, int nranks, int rank) {
  ICX_REQUIRE(h, "set_global_dql: null engine");
  return h->e->set_global_dql(nccl_id, nranks, rank);
}

extern "C" int icx_engine_abort_global_dql(icx_engine* h) {
  ICX_REQUIRE(h, "abort_global_dql: null engine");
  return h->e->abort_global_dql();
}

extern "C" int icx_engine_wait(icx_engine* h, int64_t ticket) {
  ICX_REQUIRE(h, "wait: null engine");
  return h->e->wait(ticket);
}

extern "C" int icx_engine_output_info(icx_engine* h, const char* name, int* dtype, int* rank,
                                      int64_t* dims) {
  ICX_REQUIRE(h && name && dtype && rank && dims, "output_info: bad arguments");
  return h->e->output_info(name, dtype, rank, dims);
}

extern "C" int icx_engine_output_copy(icx_engine* h, const char* name, void* host, size_t bytes) {
  ICX_REQUIRE(h && name && host, "output_copy: bad arguments");
  return h->e->output_copy(name, host, bytes);
}

extern "C" const char* icx_engine_plan(icx_engine* h) {
  if (!h) return "";
  h->plan = h->e->plan_text();
  return h->plan.c_str();
}

extern "C" int icx_engine_set_cuda_graphs(icx_engine* h, int enabled) {
  ICX_REQUIRE(h, "set_cuda_graphs: null engine");
  h->e->set_graphs(enabled != 0);
  return ICX_OK;
}

extern "C" int icx_engine_kernel_launches(icx_engine* h) { return h ? h->e->kernel_launches() : 0; }

extern "C" int icx_engine_replay(icx_engine* h) {
  ICX_REQUIRE(h, "replay: null engine");
  return h->e->replay();
}

extern "C" void* icx_engine_stream(icx_engine* h) { return h ? (void*)h->e->stream() : nullptr; }

extern "C" int icx_engine_step_count(icx_engine* h) { return h ? h->e->step_count() : 0; }

extern "C" const char* icx_engine_step_info(icx_engine* h, int i) {
  const icx::Step* st = h ? h->e->step(i) : nullptr;
  if (!st) return nullptr;
  h->plan = st->op + "\t" + st->node + "\t" + st->out + "\t" + st->info;
  return h->plan.c_str();
}

extern "C" int icx_engine_run_step(icx_engine* h, int i) {
  ICX_REQUIRE(h, "run_step: null engine");
  return h->e->run_step(i);
}

extern "C" int icx_engine_value_info(icx_engine* h, const char* name, int* dtype, int* rank,
                                     int64_t* dims) {
  ICX_REQUIRE(h && name && dtype && rank && dims, "value_info: bad arguments");
  return h->e->value_info(name, dtype, rank, dims);
}

extern "C" int icx_engine_value_copy(icx_engine* h, const char* name, void* host, size_t bytes) {
  ICX_REQUIRE(h && name && host, "value_copy: bad arguments");
  return h->e->value_copy(name, host, bytes);
}

extern "C" const char* icx_engine_profile(icx_engine* h) {
  if (!h) return nullptr;
  if (h->e->profile(&h->plan) != ICX_OK) return nullptr;
  return h->plan.c_str();
}
