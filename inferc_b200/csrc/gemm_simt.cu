// fp32 GEMM on CUDA cores with the fused Gemm epilogue (bias / residual /
// GELU / ReLU). Exact fp32 FMA arithmetic; used for shapes the tensor-core
// path does not take (small M, transposed A, unaligned operands) and as the
// reference arithmetic for the tensor-core kernel's tests.
//
// Tiling: BM x BN x 16 per CTA, 8x8 outputs per thread split into two 4x4
// quadrants (rows r and r+BM/2, cols c and c+BN/2) so that 128-bit shared
// loads are conflict free; double-buffered shared memory with register
// prefetch of the next K slice.
#include "kernels.cuh"

namespace inferc_dev {
namespace {

constexpr int BK = 16;

template <int BM, int BN, bool VEC>
__global__ void __launch_bounds__((BM / 8) * (BN / 8))
    gemm_simt_kernel(const float* __restrict__ A, int64_t lda, int trans_a,
                     const float* __restrict__ B, int64_t ldb, int trans_b, float* __restrict__ C,
                     int64_t ldc, int64_t M, int64_t N, int64_t K, Epilogue ep) {
  constexpr int TX = BN / 8, TY = BM / 8, NT = TX * TY;
  constexpr int A_ELEMS = BM * BK / NT, B_ELEMS = BN * BK / NT;  // per thread
  static_assert(A_ELEMS % 4 == 0 && B_ELEMS % 4 == 0, "tile/thread mismatch");
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  if (ep.run_if && *reinterpret_cast<const volatile int*>(ep.run_if) == 0) return;
  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  float ra[A_ELEMS], rb[B_ELEMS];

  // Element e (0..BM*BK) of the A tile in "k-major" order: a = (k, m).
  auto load_a = [&](int64_t k0) {
#pragma unroll
    for (int q = 0; q < A_ELEMS / 4; ++q) {
      const int f = tid + q * NT;  // float4 index within the tile
      if (!trans_a) {
        const int row = f / (BK / 4), kq = (f % (BK / 4)) * 4;
        const int64_t gm = m0 + row, gk = k0 + kq;
        if (VEC) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (gm < M && gk < K) v = *reinterpret_cast<const float4*>(A + gm * lda + gk);
          ra[q * 4 + 0] = v.x; ra[q * 4 + 1] = v.y; ra[q * 4 + 2] = v.z; ra[q * 4 + 3] = v.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ra[q * 4 + j] = (gm < M && gk + j < K) ? A[gm * lda + gk + j] : 0.f;
        }
      } else {
        const int k = f / (BM / 4), mq = (f % (BM / 4)) * 4;
        const int64_t gm = m0 + mq, gk = k0 + k;
        if (VEC) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (gm < M && gk < K) v = *reinterpret_cast<const float4*>(A + gk * lda + gm);
          ra[q * 4 + 0] = v.x; ra[q * 4 + 1] = v.y; ra[q * 4 + 2] = v.z; ra[q * 4 + 3] = v.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            ra[q * 4 + j] = (gm + j < M && gk < K) ? A[gk * lda + gm + j] : 0.f;
        }
      }
    }
  };
  auto store_a = [&](int buf) {
#pragma unroll
    for (int q = 0; q < A_ELEMS / 4; ++q) {
      const int f = tid + q * NT;
      if (!trans_a) {
        const int row = f / (BK / 4), kq = (f % (BK / 4)) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) As[buf][kq + j][row] = ra[q * 4 + j];
      } else {
        const int k = f / (BM / 4), mq = (f % (BM / 4)) * 4;
        *reinterpret_cast<float4*>(&As[buf][k][mq]) =
            make_float4(ra[q * 4], ra[q * 4 + 1], ra[q * 4 + 2], ra[q * 4 + 3]);
      }
    }
  };
  auto load_b = [&](int64_t k0) {
#pragma unroll
    for (int q = 0; q < B_ELEMS / 4; ++q) {
      const int f = tid + q * NT;
      if (!trans_b) {
        const int k = f / (BN / 4), nq = (f % (BN / 4)) * 4;
        const int64_t gn = n0 + nq, gk = k0 + k;
        if (VEC) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (gn < N && gk < K) v = *reinterpret_cast<const float4*>(B + gk * ldb + gn);
          rb[q * 4 + 0] = v.x; rb[q * 4 + 1] = v.y; rb[q * 4 + 2] = v.z; rb[q * 4 + 3] = v.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            rb[q * 4 + j] = (gn + j < N && gk < K) ? B[gk * ldb + gn + j] : 0.f;
        }
      } else {
        const int n = f / (BK / 4), kq = (f % (BK / 4)) * 4;
        const int64_t gn = n0 + n, gk = k0 + kq;
        if (VEC) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (gn < N && gk < K) v = *reinterpret_cast<const float4*>(B + gn * ldb + gk);
          rb[q * 4 + 0] = v.x; rb[q * 4 + 1] = v.y; rb[q * 4 + 2] = v.z; rb[q * 4 + 3] = v.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            rb[q * 4 + j] = (gn < N && gk + j < K) ? B[gn * ldb + gk + j] : 0.f;
        }
      }
    }
  };
  auto store_b = [&](int buf) {
#pragma unroll
    for (int q = 0; q < B_ELEMS / 4; ++q) {
      const int f = tid + q * NT;
      if (!trans_b) {
        const int k = f / (BN / 4), nq = (f % (BN / 4)) * 4;
        *reinterpret_cast<float4*>(&Bs[buf][k][nq]) =
            make_float4(rb[q * 4], rb[q * 4 + 1], rb[q * 4 + 2], rb[q * 4 + 3]);
      } else {
        const int n = f / (BK / 4), kq = (f % (BK / 4)) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) Bs[buf][kq + j][n] = rb[q * 4 + j];
      }
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int64_t ktiles = (K + BK - 1) / BK;
  load_a(0);
  load_b(0);
  store_a(0);
  store_b(0);
  __syncthreads();
  for (int64_t t = 0; t < ktiles; ++t) {
    const int buf = (int)(t & 1);
    if (t + 1 < ktiles) {
      load_a((t + 1) * BK);
      load_b((t + 1) * BK);
    }
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4 + BM / 2]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4 + BN / 2]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (t + 1 < ktiles) {
      store_a(buf ^ 1);
      store_b(buf ^ 1);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = m0 + ty * 4 + (i & 3) + (i >= 4 ? BM / 2 : 0);
    if (row >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t col = n0 + tx * 4 + h * (BN / 2);
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = (col + j < N) ? epilogue_apply(ep, acc[i][h * 4 + j], row, col + j) : 0.f;
      if (VEC && col + 3 < N) {
        *reinterpret_cast<float4*>(C + row * ldc + col) = make_float4(o[0], o[1], o[2], o[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < N) C[row * ldc + col + j] = o[j];
      }
    }
  }
}

template <int BM, int BN>
void launch_tile(bool vec, const float* A, int64_t lda, bool ta, const float* B, int64_t ldb,
                 bool tb, float* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                 const Epilogue& ep, cudaStream_t st) {
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  constexpr int threads = (BM / 8) * (BN / 8);
  if (vec)
    gemm_simt_kernel<BM, BN, true><<<grid, threads, 0, st>>>(A, lda, ta, B, ldb, tb, C, ldc, M, N,
                                                             K, ep);
  else
    gemm_simt_kernel<BM, BN, false><<<grid, threads, 0, st>>>(A, lda, ta, B, ldb, tb, C, ldc, M,
                                                              N, K, ep);
}

}  // namespace

void launch_gemm_simt(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                      float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                      cudaStream_t st) {
  if (M <= 0 || N <= 0) return;
  IDEV_CHECK_ARG(M < (1LL << 31) / 1 && N < (1LL << 31), "GEMM dims too large");
  // 128-bit paths need 16-byte aligned bases, leading dims and contiguous
  // extents that are multiples of 4 floats.
  const bool vec = aligned16(A) && aligned16(B) && aligned16(C) && lda % 4 == 0 &&
                   ldb % 4 == 0 && ldc % 4 == 0 && (ta ? M % 4 == 0 : K % 4 == 0) &&
                   (tb ? K % 4 == 0 : N % 4 == 0) &&
                   (ep.resid == nullptr || (aligned16(ep.resid) && ep.ldr % 4 == 0));
  const int64_t tiles128 = ((M + 127) / 128) * ((N + 127) / 128);
  if (tiles128 >= 148)
    launch_tile<128, 128>(vec, A, lda, ta, B, ldb, tb, C, ldc, M, N, K, ep, st);
  else
    launch_tile<64, 64>(vec, A, lda, ta, B, ldb, tb, C, ldc, M, N, K, ep, st);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
