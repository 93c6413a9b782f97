// Prepared-weight cache of the op-level GEMM entry points
// (inferc_dev_fused_matmul_add_gelu, _fused_qkv, _gemm, _matmul).
//
// The reference's executor copies every initializer once per Executor
// (src/runtime/executor.cc:89-96) and then calls its kernels with the same
// weight tensors run after run. The device counterpart keeps, per device and
// per weight (device pointer, K, N, row stride, transB), the weight's
// split-fp16 planes: made on the first call that sees the weight, reused by
// every later call, so a call does no per-call weight work and runs the
// split-fp16 tensor-core GEMM (three fp16 MMAs per product, fp32-level
// accuracy).
//
// The cache assumes a cached weight's values do not change while it is
// cached. Two guards cover buffers that are freed and reused:
//  - inferc_dev_free evicts every entry whose weight lies in the freed
//    buffer, and inferc_dev_weight_cache_evict / _clear do so explicitly;
//  - every call first runs a one-CTA check kernel that compares 64 weight
//    elements spread over the matrix with the values seen at preparation. A
//    mismatch (another tensor now lives at that address) makes the same call
//    compute its result on the CUDA cores from the raw weight, and marks the
//    entry stale in host-mapped memory, so the next call prepares it again.
//    A change confined to elements the check does not sample (an in-place
//    partial update) is not seen: such callers evict explicitly.
//
// Each (device, stream) also owns one range flag: the split-fp16 GEMM raises
// it when an activation does not fit fp16, and the CUDA-core GEMM queued
// behind it on the same stream recomputes the result only in that case
// (Epilogue::run_if), so the op stays asynchronous and exact.
#include <map>
#include <mutex>
#include <tuple>

#include "kernels.cuh"

namespace inferc_dev {

constexpr int kCheckSamples = 64;
constexpr int kFlagSlots = 4096;  // per-device pool of per-stream flag words

struct PreparedWeight {
  uint16_t* hi = nullptr;
  uint16_t* lo = nullptr;
  float* scale2 = nullptr;
  int64_t kp = 0;
  float* samples = nullptr;  // device [kCheckSamples]: W at the sampled positions
  int* stale_host = nullptr;  // host-mapped: set by the check kernel on a mismatch
  int* stale_dev = nullptr;   // the same word's device address
};

namespace {

using Key = std::tuple<int, const float*, int64_t, int64_t, int64_t, bool>;

struct Cache {
  std::mutex mu;
  std::map<Key, PreparedWeight> weights;
  std::map<std::pair<int, cudaStream_t>, int*> flags;
  std::map<int, std::pair<int*, int>> pools;  // device -> (flag words, used)
  size_t bytes = 0;
};

Cache& cache() {
  static Cache* c = new Cache();  // never destroyed: freed device memory at exit is moot
  return *c;
}

void free_entry(PreparedWeight& p) {
  cudaFree(p.hi);
  cudaFree(p.lo);
  cudaFree(p.scale2);
  cudaFree(p.samples);
  if (p.stale_host) cudaFreeHost(p.stale_host);
  p = PreparedWeight();
}

// Offset (elements) of sample i of a [K, N] weight (row stride ldw), or of
// its [N, K] transB form: positions spread over the logical matrix.
__device__ __forceinline__ int64_t sample_offset(int i, int64_t K, int64_t N, int64_t ldw,
                                                 bool trans) {
  const int64_t total = K * N;
  const int64_t e = (int64_t)((double)i * (double)(total - 1) / (kCheckSamples - 1));
  const int64_t r = trans ? e / K : e / N, c = trans ? e % K : e % N;
  return r * ldw + c;
}

__global__ void take_samples_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                    int64_t ldw, bool trans, float* __restrict__ samples) {
  const int i = threadIdx.x;
  if (i < kCheckSamples) samples[i] = w[sample_offset(i, K, N, ldw, trans)];
}

// flag = 1 when any sampled element differs bitwise from its recorded value
// (and the entry is marked stale), else 0. One CTA of kCheckSamples threads.
__global__ void check_samples_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                     int64_t ldw, bool trans, const float* __restrict__ samples,
                                     int* __restrict__ flag, int* __restrict__ stale) {
  const int i = threadIdx.x;
  const bool differs =
      __float_as_uint(w[sample_offset(i, K, N, ldw, trans)]) != __float_as_uint(samples[i]);
  const int any = __syncthreads_or(differs);
  if (i == 0) {
    *flag = any;
    if (any) *reinterpret_cast<volatile int*>(stale) = 1;
  }
}

}  // namespace

PreparedWeight prepared_weight(const float* W, int64_t K, int64_t N, int64_t ldw,
                               bool trans, cudaStream_t st) {
  int dev = 0;
  IDEV_CUDA(cudaGetDevice(&dev));
  Cache& c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  const Key key{dev, W, K, N, ldw, trans};
  auto it = c.weights.find(key);
  if (it != c.weights.end()) {
    if (*reinterpret_cast<volatile int*>(it->second.stale_host) == 0) return it->second;
    // Another tensor lives at this address now: prepare it again.
    IDEV_CUDA(cudaDeviceSynchronize());
    c.bytes -= 2 * (size_t)N * it->second.kp * sizeof(uint16_t);
    free_entry(it->second);
    c.weights.erase(it);
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  IDEV_CUDA(cudaStreamIsCapturing(st, &cap));
  IDEV_CHECK_ARG(cap == cudaStreamCaptureStatusNone,
                 "op-level GEMM: the first call with a weight prepares it and cannot be "
                 "captured; run it once before capturing");
  PreparedWeight p;
  p.kp = f16_weight_kp(K);
  const size_t plane = (size_t)N * p.kp * sizeof(uint16_t);
  try {
    IDEV_CUDA(cudaMalloc(&p.hi, plane));
    IDEV_CUDA(cudaMalloc(&p.lo, plane));
    IDEV_CUDA(cudaMalloc(&p.scale2, 2 * sizeof(float)));
    IDEV_CUDA(cudaMalloc(&p.samples, kCheckSamples * sizeof(float)));
    IDEV_CUDA(cudaHostAlloc(&p.stale_host, sizeof(int), cudaHostAllocMapped));
    *p.stale_host = 0;
    IDEV_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&p.stale_dev), p.stale_host, 0));
    prepare_weight_f16(W, K, N, ldw, p.hi, p.lo, p.scale2, st, trans);
    take_samples_kernel<<<1, kCheckSamples, 0, st>>>(W, K, N, ldw, trans, p.samples);
    IDEV_LAUNCHED();
    // Other streams may use the weight next: the planes are complete first.
    IDEV_CUDA(cudaStreamSynchronize(st));
  } catch (...) {
    free_entry(p);
    throw;
  }
  c.bytes += 2 * plane;
  auto& pool = c.pools[dev];
  if (pool.first == nullptr) {
    IDEV_CUDA(cudaMalloc(&pool.first, kFlagSlots * sizeof(int)));
    IDEV_CUDA(cudaMemset(pool.first, 0, kFlagSlots * sizeof(int)));
  }
  return c.weights.emplace(key, p).first->second;
}

// Sets *flag (device) to 1 when the weight at W no longer matches the
// prepared entry (the caller's CUDA-core fallback then computes the result),
// else to 0; the split-fp16 GEMM may raise it afterwards.
void launch_weight_check(const PreparedWeight& p, const float* W, int64_t K, int64_t N,
                         int64_t ldw, bool trans, int* flag, cudaStream_t st) {
  check_samples_kernel<<<1, kCheckSamples, 0, st>>>(W, K, N, ldw, trans, p.samples, flag,
                                                    p.stale_dev);
  IDEV_LAUNCHED();
}

// Evicts every entry whose weight starts in [base, base + bytes).
void weight_cache_evict_range(const void* base, size_t bytes) {
  Cache& c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  const uintptr_t lo = reinterpret_cast<uintptr_t>(base), hi = lo + bytes;
  bool any = false;
  for (auto& kv : c.weights) {
    const uintptr_t w = reinterpret_cast<uintptr_t>(std::get<1>(kv.first));
    any |= w >= lo && w < hi;
  }
  if (!any) return;
  IDEV_CUDA(cudaDeviceSynchronize());  // no queued GEMM still reads the planes
  for (auto it = c.weights.begin(); it != c.weights.end();) {
    const uintptr_t w = reinterpret_cast<uintptr_t>(std::get<1>(it->first));
    if (w >= lo && w < hi) {
      c.bytes -= 2 * (size_t)std::get<3>(it->first) * it->second.kp * sizeof(uint16_t);
      free_entry(it->second);
      it = c.weights.erase(it);
    } else {
      ++it;
    }
  }
}

// One flag word per (device, stream), carved from a per-device pool of
// kFlagSlots words allocated with the device's first prepared weight (so a
// new stream met inside a stream capture needs no allocation).
int* stream_range_flag(cudaStream_t st) {
  int dev = 0;
  IDEV_CUDA(cudaGetDevice(&dev));
  Cache& c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  auto it = c.flags.find({dev, st});
  if (it != c.flags.end()) return it->second;
  auto& pool = c.pools[dev];
  if (pool.first == nullptr) {
    IDEV_CUDA(cudaMalloc(&pool.first, kFlagSlots * sizeof(int)));
    IDEV_CUDA(cudaMemset(pool.first, 0, kFlagSlots * sizeof(int)));
  }
  IDEV_CHECK_ARG(pool.second < kFlagSlots, "op-level GEMM: too many streams on one device");
  int* f = pool.first + pool.second++;
  c.flags[{dev, st}] = f;
  return f;
}

}  // namespace inferc_dev

extern "C" {

int inferc_dev_weight_cache_evict(const float* w) {
  using namespace inferc_dev;
  return guard([&] { weight_cache_evict_range(w, 1); });
}

int inferc_dev_weight_cache_clear(void) {
  using namespace inferc_dev;
  return guard([&] {
    Cache& c = cache();
    std::lock_guard<std::mutex> lock(c.mu);
    IDEV_CUDA(cudaDeviceSynchronize());
    for (auto& kv : c.weights) free_entry(kv.second);
    c.weights.clear();
    c.bytes = 0;
  });
}

int64_t inferc_dev_weight_cache_bytes(void) {
  using namespace inferc_dev;
  Cache& c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  return (int64_t)c.bytes;
}

}  // extern "C"
