// GEMM dispatch: every dense contraction of the plans goes through here.
#include "kernels.cuh"

namespace inferc_dev {

void launch_gemm(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                 float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                 cudaStream_t st) {
  launch_gemm_simt(A, lda, ta, B, ldb, tb, C, ldc, M, N, K, ep, st);
}

}  // namespace inferc_dev
