// Linux stand-in for the subset of Apple Accelerate that inferc's CPU kernels
// call (src/kernels/{matmul,activation,attention,fused_matmul_add_gelu,
// elementwise}.cc). Test infrastructure only: it lets the reference's own
// kernel sources compile unchanged on x86 so they can serve as the parity
// oracle and as the timed CPU baseline.
//
// BLAS: cblas_sgemm / cblas_sgemv forward to the LP64 OpenBLAS that scipy
// bundles (exported as scipy_cblas_*; the enum values are the standard CBLAS
// ones). vDSP / vForce: scalar loops with the semantics of Apple's public
// documentation, including the operand order of vDSP_vsub (C = A - B with B
// passed first) and vDSP_vdiv (C = A / B with B passed first).
#pragma once

#include <cmath>
#include <cstddef>

extern "C" {

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void scipy_cblas_sgemm(int order, int ta, int tb, int M, int N, int K,
                       float alpha, const float* A, int lda, const float* B,
                       int ldb, float beta, float* C, int ldc);
void scipy_cblas_sgemv(int order, int ta, int M, int N, float alpha,
                       const float* A, int lda, const float* X, int incx,
                       float beta, float* Y, int incy);
}

inline void cblas_sgemm(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb,
                        int M, int N, int K, float alpha, const float* A, int lda,
                        const float* B, int ldb, float beta, float* C, int ldc) {
  scipy_cblas_sgemm(order, ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
}

inline void cblas_sgemv(CBLAS_ORDER order, CBLAS_TRANSPOSE ta, int M, int N,
                        float alpha, const float* A, int lda, const float* X,
                        int incx, float beta, float* Y, int incy) {
  scipy_cblas_sgemv(order, ta, M, N, alpha, A, lda, X, incx, beta, Y, incy);
}

typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;

inline void vDSP_meanv(const float* a, vDSP_Stride ia, float* c, vDSP_Length n) {
  float s = 0.0f;
  for (vDSP_Length i = 0; i < n; ++i) s += a[i * ia];
  *c = n ? s / static_cast<float>(n) : 0.0f;
}
inline void vDSP_measqv(const float* a, vDSP_Stride ia, float* c, vDSP_Length n) {
  float s = 0.0f;
  for (vDSP_Length i = 0; i < n; ++i) s += a[i * ia] * a[i * ia];
  *c = n ? s / static_cast<float>(n) : 0.0f;
}
inline void vDSP_vsadd(const float* a, vDSP_Stride ia, const float* b, float* c,
                       vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) c[i * ic] = a[i * ia] + *b;
}
inline void vDSP_vsmul(const float* a, vDSP_Stride ia, const float* b, float* c,
                       vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) c[i * ic] = a[i * ia] * *b;
}
inline void vDSP_vma(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib,
                     const float* c, vDSP_Stride ic, float* d, vDSP_Stride id,
                     vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) d[i * id] = a[i * ia] * b[i * ib] + c[i * ic];
}
inline void vDSP_vadd(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib,
                      float* c, vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) c[i * ic] = a[i * ia] + b[i * ib];
}
// C = A - B; B comes first in the argument list.
inline void vDSP_vsub(const float* b, vDSP_Stride ib, const float* a, vDSP_Stride ia,
                      float* c, vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) c[i * ic] = a[i * ia] - b[i * ib];
}
inline void vDSP_vmul(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib,
                      float* c, vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) c[i * ic] = a[i * ia] * b[i * ib];
}
// C = A / B; B comes first in the argument list.
inline void vDSP_vdiv(const float* b, vDSP_Stride ib, const float* a, vDSP_Stride ia,
                      float* c, vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; ++i) c[i * ic] = a[i * ia] / b[i * ib];
}

inline void vvexpf(float* y, const float* x, const int* n) {
  for (int i = 0; i < *n; ++i) y[i] = std::exp(x[i]);
}
inline void vvsqrtf(float* y, const float* x, const int* n) {
  for (int i = 0; i < *n; ++i) y[i] = std::sqrt(x[i]);
}
inline void vvtanhf(float* y, const float* x, const int* n) {
  for (int i = 0; i < *n; ++i) y[i] = std::tanh(x[i]);
}
