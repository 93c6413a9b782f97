// GEMM dispatch for raw fp32 weights: the op-level entry points run the
// split-fp16 tensor-core GEMM on cached weight planes (weight_cache.cu); the
// plans' prefill GEMMs run the 3xTF32 kernel (gemm_tc.cu) with a per-call
// weight split; the CUDA-core kernel (gemm_simt.cu) takes transposed A and
// unaligned views.
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "kernels.cuh"

namespace inferc_dev {

bool gemm_tc_supported(const float* A, int64_t lda, const float* Bb, const float* Bs,
                       int64_t ldb, int64_t M, int64_t N, int64_t K);
void launch_gemm_tc(const float* A, int64_t lda, const float* Bb, const float* Bs, int64_t ldb,
                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                    cudaStream_t st);
void launch_split_tf32(const float* x, float* big, float* small, int64_t n, cudaStream_t st);
void launch_split_small(const float* x, float* small, int64_t n, cudaStream_t st);

struct PreparedWeight {
  uint16_t* hi;
  uint16_t* lo;
  float* scale2;
  int64_t kp;
  float* samples;
  int* stale_host;
  int* stale_dev;
};
PreparedWeight prepared_weight(const float* W, int64_t K, int64_t N, int64_t ldw,
                               bool trans, cudaStream_t st);
void launch_weight_check(const PreparedWeight& p, const float* W, int64_t K, int64_t N,
                         int64_t ldw, bool trans, int* flag, cudaStream_t st);
int* stream_range_flag(cudaStream_t st);

namespace {

constexpr int64_t kTcMinRows = 1;

// Per-(device, stream) buffer for the tf32 split of a raw B operand on the
// 3xTF32 path (INFERC_OP_GEMM=tf32x3, or shapes the split-fp16 kernel does
// not take). Calls on one stream are ordered, so they may share it.
float* split_buffer(size_t floats, cudaStream_t st) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<float*, size_t>> bufs;
  int dev = 0;
  IDEV_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto& b = bufs[{dev, st}];
  if (b.second < floats) {
    if (b.first) {
      IDEV_CUDA(cudaStreamSynchronize(st));  // the stream's last split has been read
      IDEV_CUDA(cudaFree(b.first));
    }
    b = {nullptr, 0};
    IDEV_CUDA(cudaMalloc(&b.first, floats * sizeof(float)));
    b.second = floats;
  }
  return b.first;
}

bool op_gemm_tf32x3_forced() {
  static const bool forced = [] {
    const char* e = std::getenv("INFERC_OP_GEMM");
    return e && std::string(e) == "tf32x3";
  }();
  return forced;
}

}  // namespace

bool gemm_use_tc(int64_t M, int64_t N, int64_t K) { return M >= kTcMinRows && N >= 32 && K >= 8; }

// GEMM on a raw fp32 B (the plans' prefill and transposed-operand calls):
// the 3xTF32 kernel with a per-call tf32 split of B when the operands allow,
// else the CUDA-core kernel.
void launch_gemm(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                 float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                 cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  if (!ta && !tb && gemm_use_tc(M, N, K) && ldb == N &&
      gemm_tc_supported(A, lda, B, B, ldb, M, N, K)) {
    float* small = split_buffer((size_t)K * N, st);
    launch_split_small(B, small, K * N, st);
    launch_gemm_tc(A, lda, B, small, N, C, ldc, M, N, K, ep, st);
    return;
  }
  launch_gemm_simt(A, lda, ta, B, ldb, tb, C, ldc, M, N, K, ep, st);
}

// Op-level GEMM of the reference-named entry points (weights are the
// caller's long-lived initializers):
//  - split-fp16 tensor-core GEMM on the weight's cached planes (the first
//    call with a weight prepares them), A split inside the kernel, followed
//    on the same stream by a CUDA-core GEMM that recomputes the result only
//    if the split-fp16 kernel flagged an activation fp16 cannot carry or the
//    check kernel found that the cached planes no longer match the weight;
//  - otherwise (INFERC_OP_GEMM=tf32x3, transposed A, unaligned or in-place
//    operands) launch_gemm.
void launch_gemm_op(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                    cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  // The fallback rereads A, the residual and a full-matrix bias, so none of
  // them may be the output.
  const bool in_place = ep.resid == C || (ep.bias_mode == 3 && ep.bias == C) || A == C;
  if (!ta && !op_gemm_tf32x3_forced() && !in_place && gemm_use_tc(M, N, K) &&
      gemm_f16s_supported(A, lda, M, N, K) && ldb >= (tb ? K : N)) {
    const PreparedWeight p = prepared_weight(B, K, N, ldb, tb, st);
    int* flag = stream_range_flag(st);
    launch_weight_check(p, B, K, N, ldb, tb, flag, st);  // sets the flag: 0, or 1 if stale
    launch_gemm_f16s(A, lda, p.hi, p.lo, p.kp, p.scale2, flag, C, ldc, M, N, K, ep, st);
    Epilogue fb = ep;
    fb.run_if = flag;
    launch_gemm_simt(A, lda, false, B, ldb, tb, C, ldc, M, N, K, fb, st);
    return;
  }
  launch_gemm(A, lda, ta, B, ldb, tb, C, ldc, M, N, K, ep, st);
}

// Plan weights arrive pre-split (w_big / w_small, [K,N] row-major).
void launch_gemm_presplit(const float* A, int64_t lda, const float* W, const float* Wb,
                          const float* Ws, int64_t ldb, float* C, int64_t ldc, int64_t M,
                          int64_t N, int64_t K, const Epilogue& ep, cudaStream_t st) {
  if (gemm_use_tc(M, N, K) && gemm_tc_supported(A, lda, Wb, Ws, ldb, M, N, K)) {
    launch_gemm_tc(A, lda, Wb, Ws, ldb, C, ldc, M, N, K, ep, st);
    return;
  }
  launch_gemm_simt(A, lda, false, W, ldb, false, C, ldc, M, N, K, ep, st);
}

}  // namespace inferc_dev
