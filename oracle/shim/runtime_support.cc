// Linux stand-ins for the pieces of the reference runtime that the oracle's
// kernel build needs but whose reference sources depend on macOS or protobuf:
//   - par::ParallelFor and friends (util/parallel.h), reference implementation
//     util/parallel.cc:49-71 uses GCD dispatch_apply; here std::thread, with
//     the same block split (ceil(n / blocks) chunks, blocks = min(MaxThreads,
//     ceil(n / grain))) and the same INFERC_PARALLEL / INFERC_THREADS switches.
//   - DTypeBytes / DTypeName / ShapeToString (ir/graph.cc:43-99), the only
//     graph.cc functions the kernels and rt::Tensor call.
// Worker threads pin OpenBLAS to one thread each (the reference's sgemm calls
// inside ParallelFor are single-threaded Accelerate calls).
// Test infrastructure only.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <sstream>
#include <thread>
#include <vector>

#include "ir/graph.h"
#include "util/parallel.h"

extern "C" void openblas_set_num_threads_local(int);

namespace inferc {

int64_t DTypeBytes(DType dt) {
  switch (dt) {
    case DType::kFloat32: case DType::kInt32: case DType::kUint32: return 4;
    case DType::kFloat16: case DType::kBFloat16: case DType::kInt16:
    case DType::kUint16: return 2;
    case DType::kFloat64: case DType::kInt64: case DType::kUint64: return 8;
    case DType::kInt8: case DType::kUint8: case DType::kBool: return 1;
    default: return 0;
  }
}

const char* DTypeName(DType dt) {
  switch (dt) {
    case DType::kFloat32: return "float32";
    case DType::kInt64: return "int64";
    case DType::kInt32: return "int32";
    case DType::kBool: return "bool";
    case DType::kUint8: return "uint8";
    default: return "other";
  }
}

std::string ShapeToString(const Shape& s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); ++i) o << (i ? "," : "") << s[i];
  o << "]";
  return o.str();
}

namespace par {
namespace {
bool g_enabled = [] {
  const char* e = std::getenv("INFERC_PARALLEL");
  return !(e != nullptr && std::strcmp(e, "0") == 0);
}();
}  // namespace

void SetParallelEnabled(bool on) { g_enabled = on; }
bool ParallelEnabled() { return g_enabled; }

int MaxThreads() {
  static const int n = [] {
    if (const char* e = std::getenv("INFERC_THREADS")) {
      int v = std::atoi(e);
      if (v > 0) return v;
    }
    unsigned hc = std::thread::hardware_concurrency();
    return hc ? static_cast<int>(hc) : 1;
  }();
  return n;
}

void ParallelFor(int64_t n, int64_t grain,
                 const std::function<void(int64_t, int64_t)>& fn) {
  if (n <= 0) return;
  const int64_t max_blocks = std::max<int64_t>(1, MaxThreads());
  const int64_t by_grain = grain > 0 ? (n + grain - 1) / grain : max_blocks;
  const int64_t blocks = std::min(max_blocks, std::max<int64_t>(1, by_grain));
  if (!g_enabled || blocks <= 1) {
    fn(0, n);
    return;
  }
  const int64_t chunk = (n + blocks - 1) / blocks;
  std::vector<std::thread> workers;
  workers.reserve(static_cast<size_t>(blocks));
  for (int64_t b = 0; b < blocks; ++b) {
    const int64_t begin = b * chunk, end = std::min(n, begin + chunk);
    if (begin >= end) continue;
    workers.emplace_back([&fn, begin, end] {
      openblas_set_num_threads_local(1);
      fn(begin, end);
    });
  }
  for (auto& t : workers) t.join();
}

}  // namespace par
}  // namespace inferc
