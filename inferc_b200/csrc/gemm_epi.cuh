// Compile-time GEMM epilogues shared by the tensor-core GEMM kernels
// (gemm_tc.cu, gemm_f16s.cu): 16 accumulator columns of one output row.
#pragma once

#include "common.cuh"

namespace inferc_dev {

// Epilogue kinds compiled into the kernel (the generic kind evaluates the
// runtime Epilogue description element by element).
enum EpiKind : int { EPI_GENERIC = 0, EPI_BIAS = 1, EPI_BIAS_GELU = 2, EPI_BIAS_RESID = 3 };

template <int EPI>
__device__ __forceinline__ void epilogue16(const Epilogue& ep, const float (&v)[16], int64_t row,
                                           int64_t col0, int N, float* __restrict__ dst,
                                           bool vec_ok) {
  if (EPI != EPI_GENERIC && vec_ok && col0 + 16 <= N) {
    float b[16], r[16];
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(ep.bias + col0 + i));
      b[i] = t.x; b[i + 1] = t.y; b[i + 2] = t.z; b[i + 3] = t.w;
      if (EPI == EPI_BIAS_RESID) {
        const float4 u = *reinterpret_cast<const float4*>(ep.resid + row * ep.ldr + col0 + i);
        r[i] = u.x; r[i + 1] = u.y; r[i + 2] = u.z; r[i + 3] = u.w;
      }
    }
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float t = ep.alpha * v[i] + ep.beta * b[i];
      if (EPI == EPI_BIAS_RESID) t += r[i];
      if (EPI == EPI_BIAS_GELU) t = gelu_erf(t);
      o[i] = t;
    }
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    return;
  }
  for (int i = 0; i < 16; ++i)
    if (col0 + i < N) dst[i] = epilogue_apply(ep, v[i], row, col0 + i);
}


}  // namespace inferc_dev
