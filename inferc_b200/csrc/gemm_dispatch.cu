// GEMM dispatch: the tensor-core 3xTF32 kernel (gemm_tc.cu) for plain
// row-major operands with enough rows to fill the machine, the CUDA-core
// kernel (gemm_simt.cu) otherwise (small M, transposed operands, unaligned
// views).
#include <mutex>
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

namespace {

constexpr int64_t kTcMinRows = 1;

// Per-device buffer for the tf32 split of a raw B operand (op-level calls;
// prepared plans split their weights once at creation).
struct SplitBuf {
  float* p = nullptr;
  size_t floats = 0;
};

float* split_buffer(size_t floats) {
  static std::mutex mu;
  static std::vector<SplitBuf> per_dev;
  int dev = 0;
  IDEV_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if ((int)per_dev.size() <= dev) per_dev.resize(dev + 1);
  SplitBuf& b = per_dev[dev];
  if (b.floats < floats) {
    if (b.p) IDEV_CUDA(cudaFree(b.p));
    b.p = nullptr;
    b.floats = 0;
    IDEV_CUDA(cudaMalloc(&b.p, floats * sizeof(float)));
    b.floats = floats;
  }
  return b.p;
}

}  // namespace

bool gemm_use_tc(int64_t M, int64_t N, int64_t K) { return M >= kTcMinRows && N >= 32 && K >= 8; }

void launch_gemm(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                 float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                 cudaStream_t st) {
  if (!ta && !tb && gemm_use_tc(M, N, K) && ldb == N &&
      gemm_tc_supported(A, lda, B, B, ldb, M, N, K)) {
    float* small = split_buffer((size_t)K * N);
    launch_split_small(B, small, K * N, st);
    launch_gemm_tc(A, lda, B, small, N, C, ldc, M, N, K, ep, st);
    return;
  }
  launch_gemm_simt(A, lda, ta, B, ldb, tb, C, ldc, M, N, K, ep, st);
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
