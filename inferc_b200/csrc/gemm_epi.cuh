// Compile-time GEMM epilogues shared by the tensor-core GEMM kernels
// (gemm_tc.cu, gemm_f16s.cu, gemm_f16s_2cta.cu): 16 accumulator columns of
// one output row.
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


// Bias (+ GELU) epilogue of 16 columns whose result is stored as its fp16
// hi / lo split (the dispatcher guarantees N % 16 == 0 and aligned planes).
template <int EPI>
__device__ __forceinline__ void epilogue16_split(const Epilogue& ep, const float (&v)[16],
                                                 int64_t row, int64_t col0, const SplitOut& so,
                                                 bool& bad) {
  float o[16];
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(ep.bias + col0 + i));
    o[i] = ep.alpha * v[i] + ep.beta * t.x;
    o[i + 1] = ep.alpha * v[i + 1] + ep.beta * t.y;
    o[i + 2] = ep.alpha * v[i + 2] + ep.beta * t.z;
    o[i + 3] = ep.alpha * v[i + 3] + ep.beta * t.w;
  }
  if (EPI == EPI_BIAS_GELU) {
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = gelu_erf(o[i]);
  }
  uint32_t h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = split_pair(o[2 * i], o[2 * i + 1], l[i], bad);
  uint4* hp = reinterpret_cast<uint4*>(so.hi + row * so.ld + col0);
  uint4* lp = reinterpret_cast<uint4*>(so.lo + row * so.ld + col0);
  hp[0] = make_uint4(h[0], h[1], h[2], h[3]);
  hp[1] = make_uint4(h[4], h[5], h[6], h[7]);
  lp[0] = make_uint4(l[0], l[1], l[2], l[3]);
  lp[1] = make_uint4(l[4], l[5], l[6], l[7]);
}

}  // namespace inferc_dev
