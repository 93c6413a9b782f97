// Device executor: runs an optimized inferc plan (an ONNX model as `inferc
// optimize` writes it) node by node on the GPU, in place of the reference's
// CPU interpreter Executor::Run (src/runtime/executor.cc:98-366). Same op
// names, attributes and defaults, same dispatch order (the graph's node list),
// same error messages; every op runs a CUDA kernel of this library, so there
// is no CPU fallback.
//
// Tensors. Every tensor that depends on a graph input's values lives on the
// device. Shape metadata (Shape, Constant, small int64 initializers and the
// arithmetic the exporters build on them: Gather / Unsqueeze / Concat / Slice
// / Cast / Add ... of a few elements) is evaluated on the host when all of an
// op's inputs are known there and its result is at most kFoldElems elements,
// as constant folding; the reference reads the same values on the host
// (ReadInt64Vec, executor.cc:28-37). A device tensor whose values an op must
// read on the host (a Reshape target computed on the device) is copied back
// with a stream synchronisation.
//
// Memory. Initializers are uploaded once per executor, as the reference
// copies them once per Executor (executor.cc:89-96). Activations come from the
// device's stream-ordered pool (cudaMallocAsync on the run's stream, release
// threshold raised so that repeated runs reuse the pages) and are returned
// after the last node that reads them (liveness computed at load), instead of
// living until the end of the run as the reference's tape does.
//
// Fusion at load. MatMul by an initializer followed by Add of a 1-D
// initializer (the bias) and optionally by Add of a same-shape tensor (the
// residual), each intermediate read by that node only, becomes one GEMM with
// a bias(+residual) epilogue; the values are the same sums in the GEMM's
// accumulation order.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include "glue.cuh"
#include "kernels.cuh"
#include "onnx_model.h"

namespace inferc_dev {
void launch_gemm(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                 float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                 cudaStream_t st);
void launch_gemm_op(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                    cudaStream_t st);
void weight_cache_evict_range(const void* base, size_t bytes);
struct PreparedWeight {
  uint16_t* hi;
  uint16_t* lo;
  float* scale2;
  int64_t kp;
  float* samples;
  int* stale_host;
  int* stale_dev;
};
PreparedWeight prepared_weight(const float* W, int64_t K, int64_t N, int64_t ldw, bool trans,
                               cudaStream_t st);
}  // namespace inferc_dev

namespace {

using namespace inferc_dev;
namespace ox = inferc_dev::onnx;

constexpr int64_t kFoldElems = 4096;  // host-evaluated metadata tensors (elements)
constexpr int kMaxRank = kGlueMaxRank;

[[noreturn]] void fail(const std::string& msg) { throw Error(INFERC_ERR_INVALID, msg); }

int64_t numel_of(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

struct DevBuf {
  void* p = nullptr;
  bool pooled = false;
  cudaStream_t st = nullptr;
  ~DevBuf() {
    if (!p) return;
    if (pooled) cudaFreeAsync(p, st);
    else cudaFree(p);
  }
};

struct T {
  int32_t dt = 0;
  std::vector<int64_t> shape;
  std::shared_ptr<DevBuf> dev;                  // device storage (contiguous)
  size_t off = 0;                               // byte offset into dev
  std::shared_ptr<std::vector<uint8_t>> host;   // host values, when known there
  // fp16 hi / lo planes of an fp32 tensor (row stride = last dim; hi, then
  // lo), written by producers whose readers take them (split-fp16 GEMMs and
  // attention); f32 false = only the planes exist.
  std::shared_ptr<DevBuf> pl;
  bool f32 = true;
  uint16_t* phi() const { return static_cast<uint16_t*>(pl->p); }
  uint16_t* plo() const { return phi() + numel(); }
  int64_t numel() const { return numel_of(shape); }
  size_t nbytes() const { return (size_t)(numel() * ox::dtype_bytes(dt)); }
  int64_t esize() const { return ox::dtype_bytes(dt); }
  template <typename U>
  U* d() const { return reinterpret_cast<U*>(static_cast<uint8_t*>(dev->p) + off); }
  template <typename U>
  const U* h() const { return reinterpret_cast<const U*>(host->data()); }
};

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size(), 1);
  for (int i = (int)s.size() - 2; i >= 0; --i) st[i] = st[i + 1] * s[i + 1];
  return st;
}

// numpy broadcast of two shapes (elementwise.cc:21-34).
std::vector<int64_t> broadcast(const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
  const size_t r = std::max(a.size(), b.size());
  std::vector<int64_t> out(r);
  for (size_t i = 0; i < r; ++i) {
    const int64_t da = i < a.size() ? a[a.size() - 1 - i] : 1;
    const int64_t db = i < b.size() ? b[b.size() - 1 - i] : 1;
    int64_t d;
    if (da == db || db == 1) d = da;
    else if (da == 1) d = db;
    else fail("elementwise: broadcast mismatch");
    out[r - 1 - i] = d;
  }
  return out;
}

// Strides of `in` right-aligned against `out`, 0 on broadcast axes.
void bcast_strides(const std::vector<int64_t>& in, const std::vector<int64_t>& out, int64_t* s) {
  const int r = (int)out.size(), skip = r - (int)in.size();
  int64_t st = 1;
  for (int i = 0; i < r; ++i) s[i] = 0;
  for (int i = (int)in.size() - 1; i >= 0; --i) {
    s[skip + i] = in[i] == 1 ? 0 : st;
    st *= in[i];
  }
}

GlueShape glue_shape(const std::vector<int64_t>& out) {
  if ((int)out.size() > kMaxRank) fail("executor: tensors above rank 8 are not supported");
  GlueShape g;
  g.rank = (int)out.size();
  g.n = numel_of(out);
  for (int i = 0; i < g.rank; ++i) g.shape[i] = out[i];
  if (g.rank == 0) {  // scalar
    g.rank = 1;
    g.shape[0] = 1;
  }
  return g;
}

// Host evaluation of a strided copy (the host half of constant folding).
void host_copy(const uint8_t* in, uint8_t* out, int64_t esz, const GlueShape& g) {
  for (int64_t i = 0; i < g.n; ++i) {
    int64_t r = i, io = g.off0, oo = g.off1;
    for (int d = g.rank - 1; d >= 0; --d) {
      const int64_t c = r % g.shape[d];
      r /= g.shape[d];
      io += c * g.s0[d];
      oo += c * g.s1[d];
    }
    std::memcpy(out + oo * esz, in + io * esz, (size_t)esz);
  }
}

int64_t host_i64(const T& t, int64_t i) {
  switch (t.dt) {
    case ox::kInt64: return t.h<int64_t>()[i];
    case ox::kInt32: return t.h<int32_t>()[i];
    case ox::kFloat: return (int64_t)t.h<float>()[i];
    default: return t.h<uint8_t>()[i] ? 1 : 0;
  }
}

struct Step {
  const ox::Node* node = nullptr;
  // fused MatMul(+bias)(+residual): names of bias / residual inputs and the
  // name the fused result is stored under
  bool fused_gemm = false;
  std::string bias, resid, out;
  // FusedQKV whose three outputs feed only the next node, a FusedAttention:
  // one QKV GEMM over the concatenated weights (wcat / bcat, made at load)
  // writing fp16 planes, then the split-fp16 attention on them.
  bool qkv_attn = false;
  std::string wcat, bcat;
  const ox::Node* attn = nullptr;
  std::vector<std::string> reads;  // every tensor name the step reads
};

}  // namespace

struct InfercGraph {
  ox::Model model;
  int device = 0;
  std::unordered_map<std::string, T> inits;
  std::set<std::string> init_names;
  // folded Transpose(perm = [1, 0]) of a 2-D initializer -> that initializer
  std::map<std::string, std::string> transposed_of;
  std::unordered_map<std::string, T> inputs;
  std::unordered_map<std::string, T> outputs;
  std::vector<Step> steps;
  std::unordered_map<std::string, size_t> last_use;
  std::set<std::string> graph_outputs;
  int* err = nullptr;
  // Split-fp16 planes between fused ops: which tensors get them, and whether
  // only the planes are needed. A run that meets a value fp16 cannot carry
  // (the range flag) is rerun without planes, on the fp32 operands.
  std::set<std::string> want_planes, planes_only;
  bool use_planes = true;
  int* range = nullptr;
  int64_t range_reruns = 0;
  cudaStream_t st = nullptr;  // the stream of the current run

  ~InfercGraph() {
    outputs.clear();
    inputs.clear();
    for (auto& kv : inits)
      if (kv.second.dev) weight_cache_evict_range(kv.second.dev->p, kv.second.nbytes() + 1);
    inits.clear();
    if (err) cudaFree(err);
    if (range) cudaFree(range);
  }

  // ------------------------------------------------------------- tensors
  T alloc(int32_t dt, std::vector<int64_t> shape) {
    T t;
    t.dt = dt;
    t.shape = std::move(shape);
    t.dev = std::make_shared<DevBuf>();
    const size_t bytes = std::max<size_t>(t.nbytes(), 16);
    const cudaError_t e = cudaMallocAsync(&t.dev->p, bytes, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Error(e == cudaErrorMemoryAllocation ? INFERC_ERR_OOM : INFERC_ERR_CUDA,
                  "executor: activation allocation of " + std::to_string(bytes) +
                      " B failed: " + cudaGetErrorString(e));
    }
    t.dev->pooled = true;
    t.dev->st = st;
    return t;
  }
  void alloc_planes(T& t) {
    T p = alloc(ox::kInt32, {t.numel()});  // 2 x numel uint16 = numel words of 4 bytes
    t.pl = p.dev;
  }
  SplitOut planes_out(T& t) {
    alloc_planes(t);
    SplitOut so;
    so.hi = t.phi();
    so.lo = t.plo();
    so.ld = t.shape.empty() ? 1 : t.shape.back();
    so.range = range;
    return so;
  }
  static F16GemmA planes_a(const T& x) {
    F16GemmA a;
    a.hi = x.phi();
    a.lo = x.plo();
    a.ld = x.shape.back();
    return a;
  }
  T host_tensor(int32_t dt, std::vector<int64_t> shape) {
    T t;
    t.dt = dt;
    t.shape = std::move(shape);
    t.host = std::make_shared<std::vector<uint8_t>>(std::max<size_t>(t.nbytes(), 1));
    return t;
  }
  void to_dev(T& t) {
    if (t.dev) return;
    T d = alloc(t.dt, t.shape);
    if (t.nbytes())  // pageable source: the copy is staged before this returns
      IDEV_CUDA(cudaMemcpyAsync(d.dev->p, t.host->data(), t.nbytes(), cudaMemcpyHostToDevice, st));
    t.dev = d.dev;
    t.off = 0;
  }
  void to_host(T& t) {
    if (t.host) return;
    t.host = std::make_shared<std::vector<uint8_t>>(std::max<size_t>(t.nbytes(), 1));
    if (t.nbytes()) {
      IDEV_CUDA(cudaMemcpyAsync(t.host->data(), t.d<uint8_t>(), t.nbytes(),
                                cudaMemcpyDeviceToHost, st));
      IDEV_CUDA(cudaStreamSynchronize(st));
    }
  }
  std::vector<int64_t> read_i64(T t) {  // ReadInt64Vec (executor.cc:28-37)
    if (t.dt != ox::kInt64) fail("Executor: expected int64 tensor");
    to_host(t);
    return std::vector<int64_t>(t.h<int64_t>(), t.h<int64_t>() + t.numel());
  }

  // ---------------------------------------------------------------- load
  // The ops Executor::Run dispatches (src/runtime/executor.cc:123-343).
  static void check_ops(const ox::Model& m) {
    static const std::set<std::string> known = {
        "Split", "FusedQKV", "Sqrt", "Erf", "Relu", "Tanh", "Neg", "Abs", "Add", "Sub", "Mul",
        "Div", "Pow", "Equal", "Where", "Gelu", "GeluTanh", "Softmax", "ReduceMean", "MatMul",
        "FusedMatMulAddGELU", "FusedLayerNorm", "FusedAttention", "Gemm", "Reshape",
        "Transpose", "Concat", "Slice", "Unsqueeze", "Squeeze", "Cast", "Expand", "Shape",
        "ConstantOfShape", "Range", "Gather", "Constant", "Identity"};
    for (const auto& n : m.graph.nodes)
      if (!known.count(n.op_type))
        fail("Executor: unsupported op '" + n.op_type + "' (node: " + n.name + ")");
  }

  void load(const uint8_t* bytes, size_t len) {
    std::string perr;
    if (!ox::parse_model(bytes, len, &model, &perr)) fail("ONNX parse error: " + perr);
    check_ops(model);
    IDEV_CUDA(cudaGetDevice(&device));
    cudaMemPool_t pool;
    IDEV_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    uint64_t keep = UINT64_MAX;  // keep freed pages in the pool between runs
    IDEV_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    IDEV_CUDA(cudaMalloc(&err, sizeof(int)));
    IDEV_CUDA(cudaMemset(err, 0, sizeof(int)));
    const ox::Graph& g = model.graph;
    for (const auto& tp : g.initializers) {
      if (ox::dtype_bytes(tp.data_type) == 0)
        fail("executor: initializer '" + tp.name + "' has an unsupported dtype");
      T t;
      t.dt = tp.data_type;
      t.shape = tp.dims;
      std::vector<uint8_t> b = tp.bytes();
      if (b.size() != t.nbytes())
        fail("executor: initializer '" + tp.name + "' size does not match its dims");
      t.dev = std::make_shared<DevBuf>();
      IDEV_CUDA(cudaMalloc(&t.dev->p, std::max<size_t>(b.size(), 16)));
      if (!b.empty())
        IDEV_CUDA(cudaMemcpy(t.dev->p, b.data(), b.size(), cudaMemcpyHostToDevice));
      if (t.numel() <= kFoldElems) t.host = std::make_shared<std::vector<uint8_t>>(std::move(b));
      inits[tp.name] = std::move(t);
      init_names.insert(tp.name);
    }
    for (const auto& vi : g.outputs) graph_outputs.insert(vi.name);
    IDEV_CUDA(cudaMalloc(&range, sizeof(int)));
    IDEV_CUDA(cudaMemset(range, 0, sizeof(int)));
    fold_constant_transposes();
    plan_steps();
    prepare_weights();
  }

  // The split-fp16 planes of every GEMM weight the steps read, made once here
  // (the op-level weight cache), and the concatenated QKV weights.
  void prepare_weights() {
    IDEV_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    auto prep = [&](const std::string& name) {
      const T& w = inits[name];
      prepared_weight(w.d<float>(), w.shape[0], w.shape[1], w.shape[1], false, st);
    };
    for (const Step& s : steps) {
      const ox::Node& n = *s.node;
      if (s.fused_gemm) prep(n.inputs[1]);
      else if (s.qkv_attn) prep(s.wcat);
      else if (n.op_type == "FusedMatMulAddGELU" && is_2d_f32_init(n.inputs[1])) prep(n.inputs[1]);
      else if (n.op_type == "FusedQKV")
        for (int i = 1; i <= 5; i += 2)
          if (is_2d_f32_init(n.inputs[i])) prep(n.inputs[i]);
    }
    IDEV_CUDA(cudaStreamSynchronize(st));
    cudaStreamDestroy(st);
    st = nullptr;
  }

  // Transpose of an initializer is computed once here and becomes an
  // initializer itself, as `inferc decode` folds the tied LM head's
  // Transpose(wte) before building its executors (FoldConstantTranspose,
  // src/cli/main.cpp:745-752, src/ir/passes/constant_fold.cc:12-57).
  std::set<const ox::Node*> folded;
  void fold_constant_transposes() {
    IDEV_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    for (const auto& n : model.graph.nodes) {
      if (n.op_type != "Transpose" || n.inputs.size() != 1 || !init_names.count(n.inputs[0]) ||
          n.outputs.empty())
        continue;
      T t = transpose(inits[n.inputs[0]], n.attr_ints("perm"));
      to_dev(t);
      T owned;  // into a plain allocation that outlives the stream's pool
      owned.dt = t.dt;
      owned.shape = t.shape;
      owned.dev = std::make_shared<DevBuf>();
      IDEV_CUDA(cudaMalloc(&owned.dev->p, std::max<size_t>(t.nbytes(), 16)));
      IDEV_CUDA(cudaMemcpyAsync(owned.dev->p, t.d<void>(), t.nbytes(), cudaMemcpyDeviceToDevice,
                                st));
      IDEV_CUDA(cudaStreamSynchronize(st));
      if (owned.numel() <= kFoldElems) owned.host = t.host;
      inits[n.outputs[0]] = owned;
      init_names.insert(n.outputs[0]);
      const std::vector<int64_t> perm = n.attr_ints("perm");
      if (t.shape.size() == 2 && perm.size() == 2 && perm[0] == 1 && perm[1] == 0)
        transposed_of[n.outputs[0]] = n.inputs[0];
      folded.insert(&n);
    }
    IDEV_CUDA(cudaStreamSynchronize(st));
    cudaStreamDestroy(st);
    st = nullptr;
  }

  // consumers of each tensor name (graph outputs count as a consumer)
  void plan_steps() {
    const auto& nodes = model.graph.nodes;
    std::unordered_map<std::string, int> uses;
    for (const auto& n : nodes)
      for (const auto& i : n.inputs)
        if (!i.empty()) ++uses[i];
    for (const auto& o : graph_outputs) ++uses[o];
    auto single = [&](const std::string& name) { return uses[name] == 1; };
    for (size_t i = 0; i < nodes.size(); ++i) {
      if (folded.count(&nodes[i])) continue;
      Step s;
      s.node = &nodes[i];
      const ox::Node& n = nodes[i];
      // FusedQKV -> FusedAttention(q, k, v[, mask])
      if (n.op_type == "FusedQKV" && i + 1 < nodes.size() && n.outputs.size() == 3 &&
          n.inputs.size() == 7) {
        const ox::Node& at = nodes[i + 1];
        bool ok = at.op_type == "FusedAttention" && at.inputs.size() >= 3 &&
                  at.attr_int("head_dim", 64) == 64;
        for (int j = 0; ok && j < 3; ++j)
          ok = at.inputs[j] == n.outputs[j] && single(n.outputs[j]) &&
               is_2d_f32_init(n.inputs[1 + 2 * j]) && is_bias_any(n.inputs[2 + 2 * j]);
        if (ok) {
          const T& w0 = inits[n.inputs[1]];
          const int64_t K = w0.shape[0], N = w0.shape[1];
          for (int j = 1; ok && j < 3; ++j)
            ok = inits[n.inputs[1 + 2 * j]].shape == w0.shape &&
                 inits[n.inputs[2 + 2 * j]].numel() == N;
          ok = ok && inits[n.inputs[2]].numel() == N && N % 64 == 0 && K % 8 == 0;
          if (ok) {
            s.qkv_attn = true;
            s.attn = &at;
            s.out = at.outputs[0];
            s.wcat = n.name + "/wqkv";
            s.bcat = n.name + "/bqkv";
            concat_qkv(n, K, N, s.wcat, s.bcat);
            s.reads = {n.inputs[0]};
            if (at.inputs.size() >= 4 && !at.inputs[3].empty()) s.reads.push_back(at.inputs[3]);
            steps.push_back(s);
            ++i;
            continue;
          }
        }
      }
      // MatMul(x, W) -> Add(., b) [-> Add(., r)]
      if (n.op_type == "MatMul" && n.inputs.size() == 2 && is_2d_f32_init(n.inputs[1]) &&
          i + 1 < nodes.size() && single(n.outputs[0])) {
        const ox::Node& a1 = nodes[i + 1];
        const int64_t N = inits[n.inputs[1]].shape[1];
        const int bi = add_operand(a1, n.outputs[0]);
        if (bi >= 0 && is_bias(a1.inputs[bi], N)) {
          s.fused_gemm = true;
          s.bias = a1.inputs[bi];
          s.out = a1.outputs[0];
          size_t used = 2;
          if (i + 2 < nodes.size() && single(a1.outputs[0])) {
            const ox::Node& a2 = nodes[i + 2];
            const int ri = add_operand(a2, a1.outputs[0]);
            if (ri >= 0 && !is_bias(a2.inputs[ri], N)) {
              s.resid = a2.inputs[ri];
              s.out = a2.outputs[0];
              used = 3;
            }
          }
          s.reads = {n.inputs[0], n.inputs[1], s.bias};
          if (!s.resid.empty()) s.reads.push_back(s.resid);
          steps.push_back(s);
          i += used - 1;
          continue;
        }
      }
      for (const auto& in : n.inputs)
        if (!in.empty()) s.reads.push_back(in);
      steps.push_back(s);
    }
    for (size_t k = 0; k < steps.size(); ++k)
      for (const auto& r : steps[k].reads) last_use[r] = k;
    // readers that take split-fp16 planes for their A operand
    std::unordered_map<std::string, int> plane_reads, all_reads;
    for (const Step& st_ : steps) {
      for (const auto& r : st_.reads) ++all_reads[r];
      const ox::Node& n = *st_.node;
      const bool planes_a =
          st_.fused_gemm || st_.qkv_attn ||
          (n.op_type == "FusedMatMulAddGELU" && is_2d_f32_init(n.inputs[1]) &&
           inits[n.inputs[1]].shape[0] % 8 == 0);
      if (planes_a) ++plane_reads[n.inputs[0]];
    }
    for (const auto& kv : plane_reads) {
      want_planes.insert(kv.first);
      if (kv.second == all_reads[kv.first] && !graph_outputs.count(kv.first))
        planes_only.insert(kv.first);
    }
  }
  bool is_bias_any(const std::string& name) {
    auto it = inits.find(name);
    return it != inits.end() && it->second.dt == ox::kFloat && it->second.shape.size() == 1;
  }
  // [K, 3N] = [Wq | Wk | Wv] and [3N] = [bq | bk | bv] as new initializers.
  void concat_qkv(const ox::Node& n, int64_t K, int64_t N, const std::string& wname,
                  const std::string& bname) {
    T w, b;
    w.dt = b.dt = ox::kFloat;
    w.shape = {K, 3 * N};
    b.shape = {3 * N};
    w.dev = std::make_shared<DevBuf>();
    b.dev = std::make_shared<DevBuf>();
    IDEV_CUDA(cudaMalloc(&w.dev->p, w.nbytes()));
    IDEV_CUDA(cudaMalloc(&b.dev->p, b.nbytes()));
    for (int j = 0; j < 3; ++j) {
      const T& wj = inits[n.inputs[1 + 2 * j]];
      const T& bj = inits[n.inputs[2 + 2 * j]];
      IDEV_CUDA(cudaMemcpy2D(w.d<float>() + j * N, 3 * N * sizeof(float), wj.d<float>(),
                             N * sizeof(float), N * sizeof(float), K, cudaMemcpyDeviceToDevice));
      IDEV_CUDA(cudaMemcpy(b.d<float>() + j * N, bj.d<float>(), N * sizeof(float),
                           cudaMemcpyDeviceToDevice));
    }
    inits[wname] = w;
    inits[bname] = b;
    init_names.insert(wname);
    init_names.insert(bname);
  }
  bool is_2d_f32_init(const std::string& name) {
    auto it = inits.find(name);
    return it != inits.end() && it->second.dt == ox::kFloat && it->second.shape.size() == 2;
  }
  bool is_bias(const std::string& name, int64_t N) {
    auto it = inits.find(name);
    return it != inits.end() && it->second.dt == ox::kFloat && it->second.shape.size() == 1 &&
           it->second.shape[0] == N;
  }
  // index of the Add operand that is not `prev`, or -1
  static int add_operand(const ox::Node& n, const std::string& prev) {
    if (n.op_type != "Add" || n.inputs.size() != 2) return -1;
    if (n.inputs[0] == prev && n.inputs[1] != prev) return 1;
    if (n.inputs[1] == prev && n.inputs[0] != prev) return 0;
    return -1;
  }

  // ----------------------------------------------------------------- run
  void run(cudaStream_t stream) {
    use_planes = true;
    IDEV_CUDA(cudaMemsetAsync(range, 0, sizeof(int), stream));
    run_once(stream);
    int hr = 0;
    IDEV_CUDA(cudaMemcpyAsync(&hr, range, sizeof(int), cudaMemcpyDeviceToHost, stream));
    IDEV_CUDA(cudaStreamSynchronize(stream));
    if (hr) {  // a value fp16 cannot carry: the same run on the fp32 operands
      ++range_reruns;
      use_planes = false;
      run_once(stream);
      use_planes = true;
    }
  }

  void run_once(cudaStream_t stream) {
    st = stream;
    outputs.clear();
    static const bool trace = [] {
      const char* e = std::getenv("INFERC_EXEC_TRACE");
      return e && e[0] == '1';
    }();
    std::unordered_map<std::string, T> tape;
    auto get = [&](const std::string& name) -> T& {
      auto it = tape.find(name);
      if (it != tape.end()) return it->second;
      auto ii = inputs.find(name);
      if (ii != inputs.end()) return tape[name] = ii->second;
      auto iz = inits.find(name);
      if (iz != inits.end()) return tape[name] = iz->second;
      fail("Executor: missing tensor '" + name + "'");
    };
    for (size_t k = 0; k < steps.size(); ++k) {
      const Step& s = steps[k];
      const ox::Node& n = *s.node;
      try {
        if (s.fused_gemm) run_fused_gemm(s, get, tape);
        else if (s.qkv_attn) run_qkv_attention(s, get, tape);
        else run_node(n, get, tape);
      } catch (const Error& e) {
        throw Error(e.code, std::string(e.what()) + " (node " + n.name + ", " + n.op_type + ")");
      }
      if (trace) {  // INFERC_EXEC_TRACE=1: one line per step with its output shapes
        std::string line = n.op_type + " " + n.name + (s.fused_gemm ? " (fused)" : "") + " ->";
        for (const auto& o : n.outputs) {
          auto it = tape.find(s.fused_gemm ? s.out : o);
          if (it != tape.end()) line += " " + shape_str(it->second.shape);
          if (s.fused_gemm) break;
        }
        fprintf(stderr, "%s\n", line.c_str());
      }
      for (const auto& r : s.reads) {  // free what no later step reads
        auto it = last_use.find(r);
        if (it != last_use.end() && it->second == k && !graph_outputs.count(r)) tape.erase(r);
      }
    }
    for (const auto& name : graph_outputs) {
      auto it = tape.find(name);
      if (it == tape.end()) {
        auto ii = inits.find(name);
        if (ii == inits.end()) fail("Executor: missing graph output '" + name + "'");
        outputs[name] = ii->second;
        continue;
      }
      to_dev(it->second);
      outputs[name] = it->second;
    }
    int herr = 0;
    IDEV_CUDA(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    IDEV_CUDA(cudaStreamSynchronize(st));
    if (herr) {
      IDEV_CUDA(cudaMemset(err, 0, sizeof(int)));
      throw Error(INFERC_ERR_RANGE, "Gather: index out of range");
    }
  }

  template <typename Get>
  void run_fused_gemm(const Step& s, Get& get, std::unordered_map<std::string, T>& tape) {
    const ox::Node& n = *s.node;
    T x = get(n.inputs[0]);
    const T& w = get(n.inputs[1]);
    const T& b = get(s.bias);
    if (x.dt != ox::kFloat || x.shape.empty()) fail("MatMul: only float32 supported in v1");
    const int64_t K = w.shape[0], N = w.shape[1];
    if (x.shape.back() != K) fail("MatMul: inner dim mismatch (K!=K)");
    const bool planes = use_planes && x.pl;
    if (!planes) to_dev(x);
    std::vector<int64_t> os = x.shape;
    os.back() = N;
    const int64_t M = x.numel() / K;
    Epilogue ep;
    ep.bias = b.d<float>();
    ep.bias_mode = 1;
    auto gemm = [&](const Epilogue& e, float* y) {
      if (planes) {
        const PreparedWeight p = prepared_weight(w.d<float>(), K, N, N, false, st);
        launch_gemm_f16s(planes_a(x), p.hi, p.lo, p.kp, p.scale2, range, y, N, SplitOut(), M, N,
                         K, e, st);
      } else {
        launch_gemm_op(x.d<float>(), K, false, w.d<float>(), N, false, y, N, M, N, K, e, st);
      }
    };
    T r;
    if (!s.resid.empty()) {
      r = get(s.resid);
      if (r.dt != ox::kFloat || r.shape != os) {  // not a plain residual: no fusion of it
        T y = alloc(ox::kFloat, os);
        gemm(ep, y.d<float>());
        tape[s.out] = binary(GLUE_ADD, y, r);
        return;
      }
      to_dev(r);
      ep.resid = r.d<float>();
      ep.ldr = N;
    }
    T y = alloc(ox::kFloat, os);
    gemm(ep, y.d<float>());
    tape[s.out] = y;
  }

  // FusedQKV + FusedAttention: x's planes (its producer's, or split here) ->
  // one QKV GEMM over [Wq | Wk | Wv] writing q, k, v as fp16 planes of one
  // [M, 3N] pair -> split-fp16 attention reading them in place. Without
  // planes (a range rerun, or shapes the fp16 kernels do not take) the two
  // nodes run as they are.
  template <typename Get>
  void run_qkv_attention(const Step& s, Get& get, std::unordered_map<std::string, T>& tape) {
    const ox::Node& n = *s.node;
    const ox::Node& at = *s.attn;
    T x = get(n.inputs[0]);
    const T& w = inits[s.wcat];
    const T& bc = inits[s.bcat];
    const int64_t K = w.shape[0], N3 = w.shape[1], N = N3 / 3;
    T m;
    const bool has_mask = at.inputs.size() >= 4 && !at.inputs[3].empty();
    if (has_mask) m = get(at.inputs[3]);
    bool ok = use_planes && x.dt == ox::kFloat && x.shape.size() == 3 && x.shape[2] == K &&
              (!has_mask || (m.dt == ox::kBool && m.shape.size() <= 4));
    AttnF16Args af{};
    T qkv, o;
    if (ok) {
      const int64_t B = x.shape[0], S = x.shape[1], M = B * S;
      af.ld = N3;
      af.bstride = S * N3;
      af.B = B;
      af.S = S;
      af.nH = N / 64;
      af.scale = 0.125f;
      af.fill = at.attr_float("fill", -3.0e38f);
      af.ldo = N;
      af.bstride_o = S * N;
      if (has_mask) {  // right-aligned broadcast strides over [B, nH, S, S] (attention.cc:17-29)
        const int64_t full[4] = {B, af.nH, S, S};
        const int r = (int)m.shape.size();
        int64_t stride = 1;
        for (int i = r - 1; i >= 0 && ok; --i) {
          const int od = 4 - (r - i);
          ok = m.shape[i] == 1 || m.shape[i] == full[od];
          af.ms[od] = m.shape[i] == 1 ? 0 : stride;
          stride *= m.shape[i];
        }
      }
      qkv.dt = ox::kFloat;
      qkv.shape = {M, N3};
      alloc_planes(qkv);
      af.qh = qkv.phi(); af.ql = qkv.plo();
      af.kh = af.qh + N; af.kl = af.ql + N;
      af.vh = af.qh + 2 * N; af.vl = af.ql + 2 * N;
      o.dt = ox::kFloat;
      o.shape = x.shape;
      o.shape[2] = N;
      if (planes_only.count(s.out)) {
        af.so = planes_out(o);
        o.f32 = false;
      } else {
        o = alloc(ox::kFloat, o.shape);
        af.out = o.d<float>();
      }
      ok = ok && attention_f16_supported(af);
      if (ok) {
        if (!x.pl) {  // split x here
          to_dev(x);
          alloc_planes(x);
          launch_split_rows_f16(x.d<float>(), M, K, K, x.phi(), x.plo(), K, range, st);
        }
        if (has_mask) {
          to_dev(m);
          af.mask = m.d<uint8_t>();
        }
        const PreparedWeight p = prepared_weight(w.d<float>(), K, N3, N3, false, st);
        Epilogue ep;
        ep.bias = bc.d<float>();
        ep.bias_mode = 1;
        SplitOut so;
        so.hi = qkv.phi();
        so.lo = qkv.plo();
        so.ld = N3;
        so.range = range;
        launch_gemm_f16s(planes_a(x), p.hi, p.lo, p.kp, p.scale2, range, nullptr, N3, so, M, N3, K,
                         ep, st);
        launch_attention_f16(af, st);
        tape[s.out] = o;
        return;
      }
    }
    run_node(n, get, tape);
    run_node(at, get, tape);
  }

  // ------------------------------------------------------------ elementwise
  T binary(int op, T a, T b) {
    if (a.dt != b.dt) fail("elementwise: dtype mismatch");
    if (a.dt != ox::kFloat && a.dt != ox::kInt64)
      fail("elementwise: only float32 and int64 supported");
    const std::vector<int64_t> os = broadcast(a.shape, b.shape);
    GlueShape g = glue_shape(os);
    bcast_strides(a.shape, os, g.s0);
    bcast_strides(b.shape, os, g.s1);
    if (a.host && b.host && numel_of(os) <= kFoldElems) {
      T o = host_tensor(a.dt, os);
      for (int64_t i = 0; i < g.n; ++i) {
        int64_t r = i, ia = 0, ib = 0;
        for (int d = g.rank - 1; d >= 0; --d) {
          const int64_t c = r % g.shape[d];
          r /= g.shape[d];
          ia += c * g.s0[d];
          ib += c * g.s1[d];
        }
        if (a.dt == ox::kFloat) {
          const float x = a.h<float>()[ia], y = b.h<float>()[ib];
          float v = op == GLUE_ADD ? x + y : op == GLUE_SUB ? x - y : op == GLUE_MUL ? x * y
                  : op == GLUE_DIV ? x / y : (float)std::pow((double)x, (double)y);
          reinterpret_cast<float*>(o.host->data())[i] = v;
        } else {
          const int64_t x = a.h<int64_t>()[ia], y = b.h<int64_t>()[ib];
          int64_t v = op == GLUE_ADD ? x + y : op == GLUE_SUB ? x - y : op == GLUE_MUL ? x * y
                    : op == GLUE_DIV ? (y ? x / y : 0)
                                     : (int64_t)std::pow((double)x, (double)y);
          reinterpret_cast<int64_t*>(o.host->data())[i] = v;
        }
      }
      return o;
    }
    to_dev(a);
    to_dev(b);
    T o = alloc(a.dt, os);
    launch_glue_binary(op, a.dt, a.d<void>(), b.d<void>(), o.d<void>(), g, st);
    return o;
  }

  T equal(T a, T b) {
    const std::vector<int64_t> os = broadcast(a.shape, b.shape);
    GlueShape g = glue_shape(os);
    bcast_strides(a.shape, os, g.s0);
    bcast_strides(b.shape, os, g.s1);
    for (int dt : {a.dt, b.dt})
      if (dt != ox::kInt64 && dt != ox::kInt32 && dt != ox::kFloat && dt != ox::kBool)
        fail("Equal: unsupported dtype");
    if (a.host && b.host && numel_of(os) <= kFoldElems) {
      T o = host_tensor(ox::kBool, os);
      for (int64_t i = 0; i < g.n; ++i) {
        int64_t r = i, ia = 0, ib = 0;
        for (int d = g.rank - 1; d >= 0; --d) {
          const int64_t c = r % g.shape[d];
          r /= g.shape[d];
          ia += c * g.s0[d];
          ib += c * g.s1[d];
        }
        (*o.host)[i] = host_i64(a, ia) == host_i64(b, ib);
      }
      return o;
    }
    to_dev(a);
    to_dev(b);
    T o = alloc(ox::kBool, os);
    launch_glue_equal(a.d<void>(), a.dt, b.d<void>(), b.dt, o.d<uint8_t>(), g, st);
    return o;
  }

  T where(T c, T x, T y) {
    if (c.dt != ox::kBool) fail("Where: condition must be bool");
    if (x.dt != y.dt) fail("Where: x and y dtype mismatch");
    const std::vector<int64_t> os = broadcast(broadcast(c.shape, x.shape), y.shape);
    GlueShape g = glue_shape(os);
    bcast_strides(c.shape, os, g.s0);
    bcast_strides(x.shape, os, g.s1);
    bcast_strides(y.shape, os, g.s2);
    to_dev(c);
    to_dev(x);
    to_dev(y);
    T o = alloc(x.dt, os);
    launch_glue_where((int)x.esize(), c.d<uint8_t>(), x.d<void>(), y.d<void>(), o.d<void>(), g,
                      st);
    return o;
  }

  T unary(int op, T x) {
    if (x.dt != ox::kFloat) fail("elementwise: float32 only in v1");
    to_dev(x);
    T o = alloc(ox::kFloat, x.shape);
    launch_glue_unary(op, x.d<float>(), o.d<float>(), x.numel(), st);
    return o;
  }

  T act(int a, T x) {
    if (x.dt != ox::kFloat) fail("elementwise: float32 only in v1");
    to_dev(x);
    T o = alloc(ox::kFloat, x.shape);
    launch_act(x.d<float>(), o.d<float>(), x.numel(), a, st);
    return o;
  }

  // ---------------------------------------------------------- movement
  static T view(const T& x, std::vector<int64_t> shape) {
    T v = x;
    v.shape = std::move(shape);
    return v;
  }

  T reshape(const T& x, std::vector<int64_t> s) {  // movement.cc:23-50
    int neg = -1;
    int64_t known = 1;
    for (size_t i = 0; i < s.size(); ++i) {
      if (s[i] == -1) {
        if (neg >= 0) fail("Reshape: more than one -1");
        neg = (int)i;
      } else if (s[i] < 0) {
        fail("Reshape: negative dim other than -1");
      } else {
        known *= s[i];
      }
    }
    const int64_t total = x.numel();
    if (neg >= 0) {
      if (known == 0 || total % known != 0) fail("Reshape: cannot infer -1");
      s[neg] = total / known;
    } else if (known != total) {
      fail("Reshape: element count mismatch");
    }
    return view(x, s);
  }

  // copy `in` (viewed through g's s0 / off0) into a fresh contiguous tensor
  T copy_out(T in, int32_t dt, const std::vector<int64_t>& os, GlueShape g) {
    const std::vector<int64_t> cs = contiguous_strides(os);
    for (int d = 0; d < (int)os.size(); ++d) g.s1[d] = cs[d];
    if (os.empty()) g.s1[0] = 0;
    g.off1 = 0;
    if (in.host && numel_of(os) <= kFoldElems) {
      T o = host_tensor(dt, os);
      host_copy(in.host->data(), o.host->data(), in.esize(), g);
      return o;
    }
    to_dev(in);
    T o = alloc(dt, os);
    launch_glue_copy((int)in.esize(), in.d<void>(), o.d<void>(), g, st);
    return o;
  }

  T transpose(const T& x, std::vector<int64_t> perm) {
    const int r = (int)x.shape.size();
    if (perm.empty())
      for (int i = r - 1; i >= 0; --i) perm.push_back(i);
    if ((int)perm.size() != r) fail("Transpose: perm size != rank");
    const std::vector<int64_t> is = contiguous_strides(x.shape);
    std::vector<int64_t> os(r);
    GlueShape g = glue_shape(std::vector<int64_t>(r, 1));
    for (int i = 0; i < r; ++i) {
      if (perm[i] < 0 || perm[i] >= r) fail("Transpose: bad perm");
      os[i] = x.shape[perm[i]];
    }
    g = glue_shape(os);
    for (int i = 0; i < r; ++i) g.s0[i] = is[perm[i]];
    return copy_out(x, x.dt, os, g);
  }

  T slice(const T& x, const std::vector<int64_t>& starts, const std::vector<int64_t>& ends,
          std::vector<int64_t> axes, std::vector<int64_t> steps_) {  // movement.cc:191-251
    const int64_t r = (int64_t)x.shape.size();
    if (axes.empty())
      for (size_t i = 0; i < starts.size(); ++i) axes.push_back((int64_t)i);
    if (steps_.empty()) steps_.assign(starts.size(), 1);
    if (starts.size() != ends.size() || starts.size() != axes.size() ||
        starts.size() != steps_.size())
      fail("Slice: starts/ends/axes/steps size mismatch");
    std::vector<int64_t> st0(r, 0), len = x.shape, step(r, 1);
    for (size_t i = 0; i < starts.size(); ++i) {
      const int64_t ax = axes[i] < 0 ? axes[i] + r : axes[i];
      if (ax < 0 || ax >= r) fail("Slice: axis out of range");
      const int64_t sp = steps_[i];
      if (sp == 0) fail("Slice: step == 0");
      const int64_t dim = x.shape[ax];
      int64_t s = starts[i], e = ends[i];
      if (s < 0) s += dim;
      if (e < 0) e += dim;
      s = std::max<int64_t>(0, std::min(s, dim));
      e = std::max<int64_t>(0, std::min(e, dim));
      const int64_t l = sp > 0 ? std::max<int64_t>(0, (e - s + sp - 1) / sp)
                               : std::max<int64_t>(0, (s - e - sp - 1) / -sp);
      st0[ax] = s;
      len[ax] = l;
      step[ax] = sp;
    }
    const std::vector<int64_t> is = contiguous_strides(x.shape);
    GlueShape g = glue_shape(len);
    g.off0 = 0;
    for (int64_t i = 0; i < r; ++i) {
      g.s0[i] = is[i] * step[i];
      g.off0 += st0[i] * is[i];
    }
    return copy_out(x, x.dt, len, g);
  }

  T concat(std::vector<T> parts, int64_t axis) {  // movement.cc:142-189
    if (parts.empty()) fail("Concat: no inputs");
    const int64_t r = (int64_t)parts[0].shape.size();
    if (axis < 0) axis += r;
    if (axis < 0 || axis >= r) fail("Concat: axis out of range");
    std::vector<int64_t> os = parts[0].shape;
    os[axis] = 0;
    bool all_host = true;
    for (const auto& p : parts) {
      if (p.dt != parts[0].dt) fail("Concat: dtype mismatch");
      if ((int64_t)p.shape.size() != r) fail("Concat: rank mismatch");
      for (int64_t d = 0; d < r; ++d)
        if (d != axis && p.shape[d] != parts[0].shape[d])
          fail("Concat: dim mismatch outside axis");
      os[axis] += p.shape[axis];
      all_host &= (bool)p.host;
    }
    const std::vector<int64_t> ostr = contiguous_strides(os);
    const bool host = all_host && numel_of(os) <= kFoldElems;
    T o = host ? host_tensor(parts[0].dt, os) : alloc(parts[0].dt, os);
    int64_t at = 0;
    for (auto& p : parts) {
      GlueShape g = glue_shape(p.shape);
      const std::vector<int64_t> is = contiguous_strides(p.shape);
      for (int64_t d = 0; d < r; ++d) {
        g.s0[d] = is[d];
        g.s1[d] = ostr[d];
      }
      g.off1 = at * ostr[axis];
      at += p.shape[axis];
      if (host) {
        host_copy(p.host->data(), o.host->data(), p.esize(), g);
      } else {
        to_dev(p);
        launch_glue_copy((int)p.esize(), p.d<void>(), o.d<void>(), g, st);
      }
    }
    return o;
  }

  T expand(const T& x, const std::vector<int64_t>& target) {  // movement.cc:286-335
    const size_t ri = x.shape.size(), ro = target.size();
    if (ri > ro) fail("Expand: input rank > target rank");
    std::vector<int64_t> padded(ro, 1);
    for (size_t i = 0; i < ri; ++i) padded[ro - ri + i] = x.shape[i];
    for (size_t i = 0; i < ro; ++i)
      if (padded[i] != target[i] && padded[i] != 1) fail("Expand: shape not broadcastable");
    GlueShape g = glue_shape(target);
    bcast_strides(padded, target, g.s0);
    return copy_out(x, x.dt, target, g);
  }

  T gather(T data, T idx, int64_t axis) {  // embedding.cc:9-77
    const int64_t r = (int64_t)data.shape.size();
    if (axis < 0) axis += r;
    if (axis < 0 || axis >= r) fail("Gather: axis out of range");
    if (idx.dt != ox::kInt64 && idx.dt != ox::kInt32)
      fail("Gather: indices must be int32 or int64");
    const int64_t axis_dim = data.shape[axis];
    std::vector<int64_t> os(data.shape.begin(), data.shape.begin() + axis);
    os.insert(os.end(), idx.shape.begin(), idx.shape.end());
    os.insert(os.end(), data.shape.begin() + axis + 1, data.shape.end());
    int64_t outer = 1, slice_ = 1;
    for (int64_t i = 0; i < axis; ++i) outer *= data.shape[i];
    for (int64_t i = axis + 1; i < r; ++i) slice_ *= data.shape[i];
    const int64_t nidx = idx.numel(), es = data.esize();
    if (data.host && idx.host && numel_of(os) <= kFoldElems) {
      T o = host_tensor(data.dt, os);
      for (int64_t ob = 0; ob < outer; ++ob)
        for (int64_t k = 0; k < nidx; ++k) {
          int64_t j = host_i64(idx, k);
          if (j < 0) j += axis_dim;
          if (j < 0 || j >= axis_dim) throw Error(INFERC_ERR_RANGE, "Gather: index out of range");
          std::memcpy(o.host->data() + (ob * nidx + k) * slice_ * es,
                      data.host->data() + (ob * axis_dim + j) * slice_ * es,
                      (size_t)(slice_ * es));
        }
      return o;
    }
    to_dev(data);
    to_dev(idx);
    T o = alloc(data.dt, os);
    launch_glue_gather((int)es, data.d<void>(), idx.d<void>(), idx.dt == ox::kInt64, o.d<void>(),
                       outer, axis_dim, nidx, slice_, err, st);
    return o;
  }

  T cast(T x, int32_t to) {  // movement.cc:345-372
    if (x.dt == to) return x;
    const bool ok = (x.dt == 1 && to == 7) || (x.dt == 7 && to == 1) || (x.dt == 6 && to == 1) ||
                    (x.dt == 1 && to == 6) || (x.dt == 9 && to == 1) || (x.dt == 7 && to == 6) ||
                    (x.dt == 6 && to == 7);
    if (!ok) fail("Cast: unsupported dtype pair");
    if (x.host && x.numel() <= kFoldElems) {
      T o = host_tensor(to, x.shape);
      for (int64_t i = 0; i < x.numel(); ++i) {
        double v = x.dt == 1 ? x.h<float>()[i] : x.dt == 7 ? (double)x.h<int64_t>()[i]
                 : x.dt == 6 ? x.h<int32_t>()[i] : (x.h<uint8_t>()[i] ? 1.0 : 0.0);
        if (to == 1) reinterpret_cast<float*>(o.host->data())[i] =
                         x.dt == 7 ? (float)x.h<int64_t>()[i] : (float)v;
        else if (to == 7) reinterpret_cast<int64_t*>(o.host->data())[i] =
                              x.dt == 1 ? (int64_t)x.h<float>()[i] : (int64_t)v;
        else reinterpret_cast<int32_t*>(o.host->data())[i] =
                 x.dt == 1 ? (int32_t)x.h<float>()[i]
                           : x.dt == 7 ? (int32_t)x.h<int64_t>()[i] : (int32_t)v;
      }
      return o;
    }
    to_dev(x);
    T o = alloc(to, x.shape);
    launch_glue_cast(x.dt, to, x.d<void>(), o.d<void>(), x.numel(), st);
    return o;
  }

  T softmax(T x, int64_t axis) {  // activation.cc:52-101
    if (x.dt != ox::kFloat) fail("Softmax: float32 only");
    const int64_t r = (int64_t)x.shape.size();
    if (axis < 0) axis += r;
    if (axis < 0 || axis >= r) fail("Softmax: axis out of range");
    if (axis != r - 1) {  // move the axis last, softmax, move it back
      std::vector<int64_t> perm, inv(r);
      for (int64_t i = 0; i < r; ++i)
        if (i != axis) perm.push_back(i);
      perm.push_back(axis);
      for (int64_t i = 0; i < r; ++i) inv[perm[i]] = i;
      return transpose(softmax(transpose(x, perm), r - 1), inv);
    }
    to_dev(x);
    T o = alloc(ox::kFloat, x.shape);
    const int64_t cols = x.shape.back();
    launch_softmax(x.d<float>(), o.d<float>(), cols ? x.numel() / cols : 0, cols, st);
    return o;
  }

  T reduce_mean(T x, std::vector<int64_t> axes, bool keep) {  // activation.cc:152-210
    if (x.dt != ox::kFloat) fail("ReduceMean: float32 only");
    const int64_t r = (int64_t)x.shape.size();
    std::set<int64_t> ax;
    if (axes.empty())
      for (int64_t i = 0; i < r; ++i) ax.insert(i);
    for (int64_t a : axes) ax.insert(a < 0 ? a + r : a);
    std::vector<int64_t> perm, os;
    int64_t cols = 1;
    for (int64_t i = 0; i < r; ++i)
      if (!ax.count(i)) perm.push_back(i);
    for (int64_t i : ax) {
      perm.push_back(i);
      cols *= x.shape[i];
    }
    for (int64_t i = 0; i < r; ++i) {
      if (ax.count(i)) {
        if (keep) os.push_back(1);
      } else {
        os.push_back(x.shape[i]);
      }
    }
    T moved = transpose(x, perm);
    to_dev(moved);
    T o = alloc(ox::kFloat, os);
    launch_glue_row_mean(moved.d<float>(), o.d<float>(), cols ? moved.numel() / cols : 0, cols,
                         st);
    return o;
  }

  // ------------------------------------------------------------- linear
  T matmul(T a, T b, const std::string& b_name) {  // matmul.cc:63-159
    if (a.dt != ox::kFloat || b.dt != ox::kFloat) fail("MatMul: only float32 supported in v1");
    if (a.shape.empty() || b.shape.empty()) fail("MatMul: tensors must be at least 1D");
    const bool a1 = a.shape.size() == 1, b1 = b.shape.size() == 1;
    if (a1) a.shape.insert(a.shape.begin(), 1);
    if (b1) b.shape.push_back(1);
    const int64_t M = a.shape[a.shape.size() - 2], K = a.shape.back();
    const int64_t Kb = b.shape[b.shape.size() - 2], N = b.shape.back();
    if (K != Kb) fail("MatMul: inner dim mismatch (K!=K)");
    std::vector<int64_t> ab(a.shape.begin(), a.shape.end() - 2), bb(b.shape.begin(), b.shape.end() - 2);
    const std::vector<int64_t> ob = broadcast(ab, bb);
    std::vector<int64_t> os = ob;
    os.push_back(M);
    os.push_back(N);
    to_dev(a);
    to_dev(b);
    T o = alloc(ox::kFloat, os);
    const int64_t batch = numel_of(ob);
    const bool b_is_init = init_names.count(b_name) && bb.empty();
    Epilogue ep;
    const auto tr = transposed_of.find(b_name);
    if (batch == 1 && M == 1 && K <= 8192 && (N % 4 != 0 || !aligned16(b.d<float>())) &&
        tr != transposed_of.end() && bb.empty()) {
      // a row vector by a folded W^T whose rows the vector GEMV cannot read
      // (the tied LM head: N = vocab): the row GEMV over W itself, [N, K]
      RowGemvArgs r{};
      r.x = a.d<float>(); r.w = inits[tr->second].d<float>(); r.y = o.d<float>();
      r.K = K; r.N = N;
      launch_row_gemv(r, st);
    } else if (batch == 1 && M == 1 && K <= 8192) {  // a row vector: the split-K GEMV
      GemvArgs gv{};
      gv.x = a.d<float>(); gv.w = b.d<float>(); gv.y = o.d<float>(); gv.K = K; gv.N = N;
      gv.alpha = 1.f; gv.beta = 1.f; gv.act = ACT_NONE;
      launch_gemv(gv, st);
    } else if (batch == 1) {
      if (b_is_init)
        launch_gemm_op(a.d<float>(), K, false, b.d<float>(), N, false, o.d<float>(), N, M, N, K,
                       ep, st);
      else
        launch_gemm(a.d<float>(), K, false, b.d<float>(), N, false, o.d<float>(), N, M, N, K, ep,
                    st);
    } else {
      int64_t sa[kMaxRank], sb[kMaxRank];
      bcast_strides(ab, ob, sa);
      bcast_strides(bb, ob, sb);
      const int br = (int)ob.size();
      if (M <= kGlueBmmMaxM && batch <= 65535 && br <= kGlueMaxRank) {
        // a few rows per matrix (decode attention: one query row per head):
        // every matrix of the batch in one launch
        GlueShape g;
        g.rank = br;
        g.n = batch;
        for (int d = 0; d < br; ++d) {
          g.shape[d] = ob[d];
          g.s0[d] = sa[d];
          g.s1[d] = sb[d];
        }
        launch_glue_bmm_small(a.d<float>(), b.d<float>(), o.d<float>(), M, K, N, g, st);
        if (a1 || b1) {
          std::vector<int64_t> s2 = ob;
          if (!a1) s2.push_back(M);
          if (!b1) s2.push_back(N);
          o.shape = s2;
        }
        return o;
      }
      for (int64_t i = 0; i < batch; ++i) {
        int64_t rem = i, ia = 0, ib = 0;
        for (int d = br - 1; d >= 0; --d) {
          const int64_t c = rem % ob[d];
          rem /= ob[d];
          ia += c * sa[d];
          ib += c * sb[d];
        }
        launch_gemm(a.d<float>() + ia * M * K, K, false, b.d<float>() + ib * K * N, N, false,
                    o.d<float>() + i * M * N, N, M, N, K, ep, st);
      }
    }
    if (a1 || b1) {
      std::vector<int64_t> s = ob;
      if (!a1) s.push_back(M);
      if (!b1) s.push_back(N);
      o.shape = s;
    }
    return o;
  }

  T gemm(T a, T b, const T* c, float alpha, float beta, bool ta, bool tb,
         const std::string& b_name) {  // matmul.cc:161-228
    if (a.dt != ox::kFloat || b.dt != ox::kFloat) fail("Gemm: float32 only");
    if (a.shape.size() != 2 || b.shape.size() != 2) fail("Gemm: A and B must be 2-D");
    const int64_t M = ta ? a.shape[1] : a.shape[0], K = ta ? a.shape[0] : a.shape[1];
    const int64_t Kb = tb ? b.shape[1] : b.shape[0], N = tb ? b.shape[0] : b.shape[1];
    if (K != Kb) fail("Gemm: inner dim mismatch");
    to_dev(a);
    to_dev(b);
    T cc;
    const bool use_c = c != nullptr && beta != 0.0f;
    int64_t clen = 0;
    if (use_c) {
      cc = *c;
      if (cc.dt != ox::kFloat) fail("Gemm: C must be float32");
      to_dev(cc);
      clen = cc.numel();
      if (!(clen == M * N || clen == N || clen == 1)) fail("Gemm: unsupported C shape for broadcast");
    }
    T o = alloc(ox::kFloat, {M, N});
    if (M == 1 && !tb && !ta && (!use_c || clen == N)) {
      GemvArgs g{};
      g.x = a.d<float>(); g.w = b.d<float>(); g.y = o.d<float>(); g.K = K; g.N = N;
      g.alpha = alpha; g.beta = beta;
      g.bias = use_c ? cc.d<float>() : nullptr;
      g.act = ACT_NONE;
      launch_gemv(g, st);
      return o;
    }
    Epilogue ep;
    ep.alpha = alpha;
    ep.beta = beta;
    if (use_c) {
      ep.bias = cc.d<float>();
      ep.bias_mode = clen == M * N ? 3 : clen == N ? 1 : 2;
      ep.ldbias = N;
    }
    const int64_t lda = ta ? M : K, ldb = tb ? K : N;
    if (init_names.count(b_name))
      launch_gemm_op(a.d<float>(), lda, ta, b.d<float>(), ldb, tb, o.d<float>(), N, M, N, K, ep, st);
    else
      launch_gemm(a.d<float>(), lda, ta, b.d<float>(), ldb, tb, o.d<float>(), N, M, N, K, ep, st);
    return o;
  }

  // ---------------------------------------------------------------- nodes
  template <typename Get>
  void run_node(const ox::Node& n, Get& get, std::unordered_map<std::string, T>& tape) {
    const std::string& op = n.op_type;
    auto in = [&](size_t i) -> T& {
      if (i >= n.inputs.size() || n.inputs[i].empty()) fail(op + ": missing input " + std::to_string(i));
      T& t = get(n.inputs[i]);
      if (!t.f32 && !(op == "FusedMatMulAddGELU" && i == 0 && use_planes))
        fail("executor: '" + n.inputs[i] + "' exists only as fp16 planes");
      return t;
    };
    auto set = [&](T t) {
      if (!n.outputs.empty()) tape[n.outputs[0]] = std::move(t);
    };
    if (op == "Split") {  // executor.cc:128-149
      T x = in(0);
      int64_t axis = n.attr_int("axis", 0);
      if (axis < 0) axis += (int64_t)x.shape.size();
      std::vector<int64_t> sizes = n.inputs.size() >= 2 && !n.inputs[1].empty()
                                       ? read_i64(in(1)) : n.attr_ints("split");
      if (sizes.empty() && !n.outputs.empty()) {
        const int64_t total = x.shape[axis], k = (int64_t)n.outputs.size();
        if (k > 0 && total % k == 0) sizes.assign(k, total / k);
        else fail("Split: cannot infer split sizes");
      }
      if (axis < 0 || axis >= (int64_t)x.shape.size()) fail("Split: axis out of range");
      int64_t sum = 0;
      for (int64_t s : sizes) sum += s;
      if (sum != x.shape[axis]) fail("Split: sum(split_sizes) != x.shape[axis]");
      int64_t at = 0;
      for (size_t i = 0; i < sizes.size() && i < n.outputs.size(); ++i) {
        std::vector<int64_t> st0(x.shape.size(), 0), en = x.shape;
        tape[n.outputs[i]] = slice(x, {at}, {at + sizes[i]}, {axis}, {1});
        at += sizes[i];
      }
      return;
    }
    if (op == "FusedQKV") {  // attention.cc:102-141
      T x = in(0);
      if (x.dt != ox::kFloat) fail("FusedQKVProjection: float32 only");
      to_dev(x);
      const int64_t K = x.shape.back(), M = x.numel() / K;
      for (int i = 0; i < 3 && i < (int)n.outputs.size(); ++i) {
        T w = in(1 + 2 * i), b = in(2 + 2 * i);
        if (w.shape.size() != 2 || w.shape[0] != K) fail("FusedQKVProjection: weight shape");
        const int64_t N = w.shape[1];
        to_dev(w);
        to_dev(b);
        std::vector<int64_t> os = x.shape;
        os.back() = N;
        T o = alloc(ox::kFloat, os);
        Epilogue ep;
        ep.bias = b.d<float>();
        ep.bias_mode = 1;
        if (init_names.count(n.inputs[1 + 2 * i]))
          launch_gemm_op(x.d<float>(), K, false, w.d<float>(), N, false, o.d<float>(), N, M, N, K, ep, st);
        else
          launch_gemm(x.d<float>(), K, false, w.d<float>(), N, false, o.d<float>(), N, M, N, K, ep, st);
        tape[n.outputs[i]] = o;
      }
      return;
    }
    if (op == "Sqrt") return set(unary(GLUE_SQRT, in(0)));
    if (op == "Erf") return set(unary(GLUE_ERF, in(0)));
    if (op == "Relu") return set(unary(GLUE_RELU, in(0)));
    if (op == "Tanh") return set(unary(GLUE_TANH, in(0)));
    if (op == "Neg") return set(unary(GLUE_NEG, in(0)));
    if (op == "Abs") return set(unary(GLUE_ABS, in(0)));
    if (op == "Add") return set(binary(GLUE_ADD, in(0), in(1)));
    if (op == "Sub") return set(binary(GLUE_SUB, in(0), in(1)));
    if (op == "Mul") return set(binary(GLUE_MUL, in(0), in(1)));
    if (op == "Div") return set(binary(GLUE_DIV, in(0), in(1)));
    if (op == "Pow") return set(binary(GLUE_POW, in(0), in(1)));
    if (op == "Equal") return set(equal(in(0), in(1)));
    if (op == "Where") return set(where(in(0), in(1), in(2)));
    if (op == "Gelu") return set(act(ACT_GELU_ERF, in(0)));
    if (op == "GeluTanh") return set(act(ACT_GELU_TANH, in(0)));
    if (op == "Softmax") return set(softmax(in(0), n.attr_int("axis", -1)));
    if (op == "ReduceMean") {
      std::vector<int64_t> axes = n.attr_ints("axes");
      if (axes.empty() && n.inputs.size() >= 2 && !n.inputs[1].empty()) axes = read_i64(in(1));
      return set(reduce_mean(in(0), axes, n.attr_int("keepdims", 1) != 0));
    }
    if (op == "MatMul") return set(matmul(in(0), in(1), n.inputs[1]));
    if (op == "FusedMatMulAddGELU") {  // fused_matmul_add_gelu.cc:13-80
      T x = in(0), w = in(1), b = in(2);
      if (x.dt != ox::kFloat || w.dt != ox::kFloat || b.dt != ox::kFloat)
        fail("FusedMatMulAddGELU: float32 only");
      if (w.shape.size() != 2) fail("FusedMatMulAddGELU: W must be 2-D");
      const int64_t K = w.shape[0], N = w.shape[1];
      if (x.shape.empty() || x.shape.back() != K) fail("FusedMatMulAddGELU: K mismatch");
      if (b.numel() != N) fail("FusedMatMulAddGELU: bias length mismatch");
      to_dev(w);
      to_dev(b);
      std::vector<int64_t> os = x.shape;
      os.back() = N;
      Epilogue ep;
      ep.bias = b.d<float>();
      ep.bias_mode = 1;
      ep.act = ACT_GELU_ERF;
      const int64_t M = x.numel() / K;
      if (use_planes && x.pl && init_names.count(n.inputs[1]) && K % 8 == 0) {
        const PreparedWeight p = prepared_weight(w.d<float>(), K, N, N, false, st);
        T o;
        o.dt = ox::kFloat;
        o.shape = os;
        SplitOut so;
        if (planes_only.count(n.outputs[0]) && N % 16 == 0) {
          so = planes_out(o);  // the next GEMM's A; no fp32 copy is stored
          o.f32 = false;
        } else {
          o = alloc(ox::kFloat, os);
        }
        launch_gemm_f16s(planes_a(x), p.hi, p.lo, p.kp, p.scale2, range,
                         o.f32 ? o.d<float>() : nullptr, N, so, M, N, K, ep, st);
        return set(o);
      }
      to_dev(x);
      T o = alloc(ox::kFloat, os);
      if (init_names.count(n.inputs[1]))
        launch_gemm_op(x.d<float>(), K, false, w.d<float>(), N, false, o.d<float>(), N, M, N, K, ep, st);
      else
        launch_gemm(x.d<float>(), K, false, w.d<float>(), N, false, o.d<float>(), N, M, N, K, ep, st);
      return set(o);
    }
    if (op == "FusedLayerNorm") {  // activation.cc:103-150, executor.cc:213-217
      T x = in(0), g = in(1), b = in(2);
      if (x.dt != ox::kFloat) fail("LayerNorm: float32 only");
      const int64_t feat = x.shape.empty() ? 1 : x.shape.back();
      if (g.numel() != feat || b.numel() != feat) fail("LayerNorm: scale/bias shape mismatch");
      to_dev(x);
      to_dev(g);
      to_dev(b);
      T o = alloc(ox::kFloat, x.shape);
      SplitOut sp;  // also the fp16 planes when a split-fp16 GEMM reads the result
      if (use_planes && want_planes.count(n.outputs[0]) && feat % 128 == 0 && feat <= 1024)
        sp = planes_out(o);
      launch_layernorm(x.d<float>(), g.d<float>(), b.d<float>(), o.d<float>(),
                       feat ? x.numel() / feat : 0, feat, n.attr_float("epsilon", 1e-5f), st, sp);
      return set(o);
    }
    if (op == "FusedAttention") {  // attention.cc:32-100, executor.cc:218-224
      T q = in(0), k = in(1), v = in(2);
      if (q.shape.size() != 3 || k.shape != q.shape || v.shape != q.shape)
        fail("FusedAttention: expect [B,S,H]");
      to_dev(q);
      to_dev(k);
      to_dev(v);
      T o = alloc(ox::kFloat, q.shape);
      const uint8_t* mp = nullptr;
      std::vector<int64_t> ms;
      T m;
      if (n.inputs.size() >= 4 && !n.inputs[3].empty()) {
        m = in(3);
        if (m.dt != ox::kBool) fail("FusedAttention: mask must be bool");
        to_dev(m);
        mp = m.d<uint8_t>();
        ms = m.shape;
      }
      const int rc = inferc_dev_fused_attention(
          q.d<float>(), k.d<float>(), v.d<float>(), mp, ms.empty() ? nullptr : ms.data(),
          (int)ms.size(), q.shape[0], q.shape[1], q.shape[2], n.attr_int("head_dim", 64),
          n.attr_float("fill", -3.0e38f), o.d<float>(), st);
      if (rc) throw Error(rc, inferc_dev_last_error_string());
      return set(o);
    }
    if (op == "Gemm") {
      const bool has_c = n.inputs.size() >= 3 && !n.inputs[2].empty();
      T c;
      if (has_c) c = in(2);
      return set(gemm(in(0), in(1), has_c ? &c : nullptr, n.attr_float("alpha", 1.0f),
                      n.attr_float("beta", 1.0f), n.attr_int("transA", 0) != 0,
                      n.attr_int("transB", 0) != 0, n.inputs[1]));
    }
    if (op == "Reshape") return set(reshape(in(0), read_i64(in(1))));
    if (op == "Transpose") return set(transpose(in(0), n.attr_ints("perm")));
    if (op == "Concat") {
      std::vector<T> parts;
      for (size_t i = 0; i < n.inputs.size(); ++i) parts.push_back(in(i));
      return set(concat(parts, n.attr_int("axis", 0)));
    }
    if (op == "Slice") {
      std::vector<int64_t> s, e, a, p;
      if (n.inputs.size() >= 2) s = read_i64(in(1));
      if (n.inputs.size() >= 3) e = read_i64(in(2));
      if (n.inputs.size() >= 4 && !n.inputs[3].empty()) a = read_i64(in(3));
      if (n.inputs.size() >= 5 && !n.inputs[4].empty()) p = read_i64(in(4));
      return set(slice(in(0), s, e, a, p));
    }
    if (op == "Unsqueeze") {  // movement.cc:253-271
      std::vector<int64_t> axes = n.inputs.size() >= 2 ? read_i64(in(1)) : n.attr_ints("axes");
      T x = in(0);
      const int64_t orank = (int64_t)(x.shape.size() + axes.size());
      for (auto& a : axes)
        if (a < 0) a += orank;
      std::sort(axes.begin(), axes.end());
      std::vector<int64_t> os;
      size_t ii = 0, ai = 0;
      for (int64_t i = 0; i < orank; ++i) {
        if (ai < axes.size() && axes[ai] == i) {
          os.push_back(1);
          ++ai;
        } else if (ii < x.shape.size()) {
          os.push_back(x.shape[ii++]);
        }
      }
      return set(reshape(x, os));
    }
    if (op == "Squeeze") {  // movement.cc:273-284
      std::vector<int64_t> axes = n.inputs.size() >= 2 ? read_i64(in(1)) : n.attr_ints("axes");
      T x = in(0);
      const int64_t r = (int64_t)x.shape.size();
      std::set<int64_t> drop;
      if (axes.empty()) {
        for (int64_t i = 0; i < r; ++i)
          if (x.shape[i] == 1) drop.insert(i);
      } else {
        for (int64_t a : axes) drop.insert(a < 0 ? a + r : a);
      }
      std::vector<int64_t> os;
      for (int64_t i = 0; i < r; ++i)
        if (!drop.count(i)) os.push_back(x.shape[i]);
      return set(reshape(x, os));
    }
    if (op == "Cast") return set(cast(in(0), (int32_t)n.attr_int("to", ox::kFloat)));
    if (op == "Expand") return set(expand(in(0), read_i64(in(1))));
    if (op == "Shape") {  // movement.cc:337-343
      const T& x = in(0);
      T o = host_tensor(ox::kInt64, {(int64_t)x.shape.size()});
      for (size_t i = 0; i < x.shape.size(); ++i)
        reinterpret_cast<int64_t*>(o.host->data())[i] = x.shape[i];
      return set(o);
    }
    if (op == "ConstantOfShape") {  // executor.cc:270-297, movement.cc:374-389
      const std::vector<int64_t> shape = read_i64(in(0));
      int32_t dt = ox::kFloat;
      std::vector<uint8_t> fill_b;
      const ox::Attribute* val = n.attr("value");
      if (val && val->has_t) {
        dt = val->t.data_type;
        fill_b = val->t.bytes();
      }
      const int64_t es = ox::dtype_bytes(dt);
      if (es == 0) fail("ConstantOfShape: unsupported dtype");
      if (fill_b.empty()) fill_b.assign((size_t)es, 0);
      if ((int64_t)fill_b.size() != es) fail("ConstantOfShape: fill_bytes size != dtype size");
      const int64_t cnt = numel_of(shape);
      if (cnt <= kFoldElems) {
        T o = host_tensor(dt, shape);
        for (int64_t i = 0; i < cnt; ++i)
          std::memcpy(o.host->data() + i * es, fill_b.data(), (size_t)es);
        return set(o);
      }
      T o = alloc(dt, shape);
      launch_glue_fill((int)es, o.d<void>(), fill_b.data(), cnt, st);
      return set(o);
    }
    if (op == "Range") {  // movement.cc:433-460
      T s = in(0), l = in(1), d = in(2);
      to_host(s);
      to_host(l);
      to_host(d);
      if (s.dt == ox::kInt64) {
        const int64_t a = s.h<int64_t>()[0], lim = l.h<int64_t>()[0], dl = d.h<int64_t>()[0];
        if (dl == 0) fail("Range: delta must be non-zero");
        const int64_t cnt = dl > 0 ? (lim > a ? (lim - a + dl - 1) / dl : 0)
                                   : (a > lim ? (a - lim - dl - 1) / -dl : 0);
        T o = host_tensor(ox::kInt64, {cnt});
        for (int64_t i = 0; i < cnt; ++i) reinterpret_cast<int64_t*>(o.host->data())[i] = a + i * dl;
        return set(o);
      }
      if (s.dt == ox::kFloat) {
        const float a = s.h<float>()[0], lim = l.h<float>()[0], dl = d.h<float>()[0];
        if (dl == 0.0f) fail("Range: delta must be non-zero");
        int64_t cnt = dl > 0 ? (lim > a ? (int64_t)((lim - a + dl - 1e-7f) / dl) : 0)
                             : (a > lim ? (int64_t)((a - lim + (-dl) - 1e-7f) / (-dl)) : 0);
        if (cnt < 0) cnt = 0;
        T o = host_tensor(ox::kFloat, {cnt});
        for (int64_t i = 0; i < cnt; ++i)
          reinterpret_cast<float*>(o.host->data())[i] = a + (float)i * dl;
        return set(o);
      }
      fail("Range: unsupported dtype");
    }
    if (op == "Gather") return set(gather(in(0), in(1), n.attr_int("axis", 0)));
    if (op == "Constant") return set(constant(n));
    if (op == "Identity") return set(in(0));
    fail("Executor: unsupported op '" + op + "' (node: " + n.name + ")");
  }

  T constant(const ox::Node& n) {  // executor.cc:39-96 MaterializeConstant
    if (const ox::Attribute* v = n.attr("value")) {
      if (v->has_t) {
        T o = host_tensor(v->t.data_type, v->t.dims);
        std::vector<uint8_t> b = v->t.bytes();
        if (b.size() != o.nbytes()) fail("Constant: value size does not match its dims");
        *o.host = std::move(b);
        if (o.host->empty()) o.host->resize(1);
        return o;
      }
    }
    if (const ox::Attribute* v = n.attr("value_int")) {
      T o = host_tensor(ox::kInt64, {});
      reinterpret_cast<int64_t*>(o.host->data())[0] = v->i;
      return o;
    }
    if (const ox::Attribute* v = n.attr("value_float")) {
      T o = host_tensor(ox::kFloat, {});
      reinterpret_cast<float*>(o.host->data())[0] = v->f;
      return o;
    }
    if (const ox::Attribute* v = n.attr("value_ints")) {
      T o = host_tensor(ox::kInt64, {(int64_t)v->ints.size()});
      std::memcpy(o.host->data(), v->ints.data(), v->ints.size() * 8);
      return o;
    }
    fail("Constant: unsupported value attribute");
  }
};

// ------------------------------------------------------------------ C ABI
namespace {
std::string json_str(const std::string& s) {
  std::string r = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') r += '\\';
    r += c;
  }
  return r + "\"";
}
}  // namespace

extern "C" {

int inferc_dev_graph_describe(const void* model, size_t len, char* buf, size_t cap,
                              size_t* needed) {
  return guard([&] {
    IDEV_CHECK_ARG(model != nullptr, "graph_describe: null model");
    ox::Model m;
    std::string perr;
    if (!ox::parse_model(static_cast<const uint8_t*>(model), len, &m, &perr))
      fail("ONNX parse error: " + perr);
    std::map<std::string, int> ops;
    for (const auto& n : m.graph.nodes) ++ops[(n.domain.empty() ? "" : n.domain + ":") + n.op_type];
    std::string j = "{\"ir_version\":" + std::to_string(m.ir_version) + ",\"graph\":" +
                    json_str(m.graph.name) + ",\"nodes\":" + std::to_string(m.graph.nodes.size()) +
                    ",\"initializers\":" + std::to_string(m.graph.initializers.size());
    int64_t params = 0;
    for (const auto& t : m.graph.initializers) params += t.numel();
    j += ",\"initializer_elements\":" + std::to_string(params) + ",\"ops\":{";
    bool first = true;
    for (const auto& kv : ops) {
      j += (first ? "" : ",") + json_str(kv.first) + ":" + std::to_string(kv.second);
      first = false;
    }
    j += "},\"opsets\":[";
    for (size_t i = 0; i < m.opsets.size(); ++i)
      j += (i ? ",[" : "[") + json_str(m.opsets[i].first) + "," +
           std::to_string(m.opsets[i].second) + "]";
    auto vis = [&](const std::vector<ox::ValueInfo>& v) {
      std::string r = "[";
      for (size_t i = 0; i < v.size(); ++i) {
        r += (i ? ",{" : "{") + std::string("\"name\":") + json_str(v[i].name) +
             ",\"dtype\":" + std::to_string(v[i].elem_type) + ",\"shape\":" +
             shape_str(v[i].dims) + "}";
      }
      return r + "]";
    };
    j += "],\"inputs\":" + vis(m.graph.inputs) + ",\"outputs\":" + vis(m.graph.outputs) + "}";
    if (needed) *needed = j.size() + 1;
    IDEV_CHECK_ARG(buf == nullptr || cap >= j.size() + 1, "graph_describe: buffer too small");
    if (buf) std::memcpy(buf, j.c_str(), j.size() + 1);
  });
}

int inferc_dev_graph_load(const void* model, size_t len, inferc_graph_t* out) {
  return guard([&] {
    IDEV_CHECK_ARG(model != nullptr && out != nullptr, "graph_load: null argument");
    *out = nullptr;
    auto g = std::make_unique<InfercGraph>();
    g->load(static_cast<const uint8_t*>(model), len);
    *out = g.release();
  });
}

int inferc_dev_graph_set_input(inferc_graph_t g, const char* name, int dtype,
                               const int64_t* shape, int rank, const void* data,
                               int data_on_device, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(g && name && (rank == 0 || shape), "graph_set_input: null argument");
    IDEV_CHECK_ARG(rank >= 0 && rank <= kMaxRank, "graph_set_input: rank must be in [0, 8]");
    IDEV_CHECK_ARG(ox::dtype_bytes(dtype) > 0, "graph_set_input: unsupported dtype");
    cudaStream_t st = as_stream(stream);
    T t;
    t.dt = dtype;
    t.shape.assign(shape, shape + rank);
    for (int64_t d : t.shape) IDEV_CHECK_ARG(d >= 0, "graph_set_input: negative dim");
    const size_t bytes = t.nbytes();
    IDEV_CHECK_ARG(bytes == 0 || data != nullptr, "graph_set_input: null data");
    auto it = g->inputs.find(name);
    // reuse the previous buffer of this input when it is large enough
    if (it != g->inputs.end() && it->second.dev && it->second.dt == dtype &&
        it->second.nbytes() >= bytes && it->second.dev.use_count() == 1) {
      t.dev = it->second.dev;
    } else {  // from the stream-ordered pool: a decode loop rebinds growing caches
      t.dev = std::make_shared<DevBuf>();
      IDEV_CUDA(cudaMallocAsync(&t.dev->p, std::max<size_t>(bytes, 16), st));
      t.dev->pooled = true;
      t.dev->st = st;
    }
    if (bytes)
      IDEV_CUDA(cudaMemcpyAsync(t.dev->p, data, bytes,
                                data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                st));
    g->inputs[name] = t;
  });
}

int inferc_dev_graph_run(inferc_graph_t g, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(g != nullptr, "graph_run: null graph");
    g->run(as_stream(stream));
  });
}

int inferc_dev_graph_output(inferc_graph_t g, const char* name, int* dtype, int64_t* shape,
                            int* rank, const void** data) {
  return guard([&] {
    IDEV_CHECK_ARG(g && name, "graph_output: null argument");
    auto it = g->outputs.find(name);
    IDEV_CHECK_ARG(it != g->outputs.end(),
                   std::string("graph_output: no output named '") + name + "' (run first)");
    const T& t = it->second;
    if (dtype) *dtype = t.dt;
    if (rank) *rank = (int)t.shape.size();
    if (shape)
      for (size_t i = 0; i < t.shape.size() && i < (size_t)kMaxRank; ++i) shape[i] = t.shape[i];
    if (data) *data = t.dev ? t.d<void>() : nullptr;
  });
}

void inferc_dev_graph_destroy(inferc_graph_t g) {
  if (!g) return;
  cudaDeviceSynchronize();  // activations still in flight are returned first
  delete g;
}

}  // extern "C"
