// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05 + TMEM),
// 3xTF32 error compensation, with the Gemm epilogue fused.
//
//   C[M,N] = epilogue(A[M,K] B[K,N]),  A row-major (K-major), B row-major
//   (N-major, the [K,N] MatMul weight layout of the reference plans).
//
// 3xTF32: every fp32 operand is split as x = big + small, big = x rounded to
// tf32 (low 13 mantissa bits zero) and small = x - big (exact in fp32). The
// product is accumulated in fp32 TMEM as a_s*b_b + a_b*b_s + a_b*b_b, which
// keeps ~22 mantissa bits per product, i.e. fp32-level error, at three
// tf32 MMAs per product. The tensor core reads only the top 19 bits of a
// 32-bit tf32 operand (it truncates), so a raw fp32 array already serves as
// its own "big" half and only small = x - trunc13(x) has to be formed: for B
// (the weight) once, in HBM; for A (the activation) in shared memory by the
// converter warps as each tile arrives. (Verified: errors are identical to
// an explicit round-to-nearest big half.)
//
// Persistent kernel (one CTA per SM striding over 128 x BN output tiles),
// STAGES-deep TMA ring, two TMEM accumulators so the epilogue of one tile
// overlaps the MMAs of the next. Warp roles (320 threads):
//   warp 0      TMA producer (one lane): A tile, B_big tile, B_small tile
//   warp 1      TMEM allocation + MMA issuer (one lane)
//   warps 2..5  converter (A -> A_big in place + A_small)
//   warps 6..9  epilogue
//               (tcgen05.ld of the 128 x BN fp32 accumulator, bias / GELU /
//               residual, stores to global).
// Shared-memory layouts are the canonical SWIZZLE_128B UMMA layouts that TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B: A is K-major (128-byte rows of 32
// fp32, 8-row atoms of 1 KiB), B is MN-major (32-column x 32-row boxes of
// 4 KiB, one per 32 columns of N).
//
// Every wait on an mbarrier is bounded; on a timeout the CTA records an
// error flag, stops issuing work, frees its TMEM and exits.
#include <cuda.h>

#include <cstdlib>

#ifndef INFERC_TC_RAW_A
#define INFERC_TC_RAW_A 1
#endif
#include <mutex>

#include "kernels.cuh"
#include "gemm_epi.cuh"
#include "tc_ptx.cuh"

namespace inferc_dev {
namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int kConvThreads = 128;  // warps 2..5
constexpr int kEpiThreads = 256;   // warps 6..13 (two per TMEM lane quarter)
constexpr int kThreadsTc = 64 + kConvThreads + kEpiThreads;

}  // namespace
}  // namespace inferc_dev

namespace inferc_dev {

__device__ int g_tc_error;  // set to 1 by a CTA whose barrier wait timed out

namespace {

// BK = 32 (128-byte A rows, SWIZZLE_128B) or 16 (64-byte A rows, SWIZZLE_64B).
template <int BN, int BK, int STAGES>
struct TcShape {
  static constexpr uint32_t A_BYTES = BM * BK * 4;
  static constexpr uint32_t B_BYTES = BK * BN * 4;
  static constexpr uint32_t B_GROUP = BK * 128;  // one 32-column group of B
  static constexpr uint32_t A_LAYOUT = BK == 32 ? 2 : 4;  // SWIZZLE_128B / _64B
  static constexpr uint32_t A_SBO = 8 * BK * 4;           // 8-row atom
  static_assert(BK == 32 || BK == 16, "BK must be 16 or 32");
  static constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32,256]");
};

template <int BN, int BK, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreadsTc, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmBb,
                       const __grid_constant__ CUtensorMap tmBs, float* __restrict__ C,
                       int64_t ldc, int M, int N, int K, Epilogue ep) {
  using S = TcShape<BN, BK, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES], conv_bar[STAGES], empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2], tempty_bar[2], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ktiles = (K + BK - 1) / BK;
  const int tiles_n = (N + BN - 1) / BN;
  const int total = ((M + BM - 1) / BM) * tiles_n;
  auto stage_a = [&](int s) { return smem + (size_t)s * S::STAGE_BYTES; };
  auto stage_as = [&](int s) { return stage_a(s) + S::A_BYTES; };
  auto stage_bb = [&](int s) { return stage_a(s) + 2 * S::A_BYTES; };
  auto stage_bs = [&](int s) { return stage_a(s) + 2 * S::A_BYTES + S::B_BYTES; };
  auto fail = [&]() {
    abort_sh = 1;
    atomicExch(&g_tc_error, 1);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&conv_bar[s], kConvThreads);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], kEpiThreads);
    }
    mbar_init(&drain_bar, 1);
    abort_sh = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // two accumulators of BN columns each
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"((uint32_t)(2 * BN)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int g = 0;  // k-iteration counter across tiles (stage ring position)
      for (int tile = blockIdx.x; tile < total && !abort_sh; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
        for (int it = 0; it < ktiles && !abort_sh; ++it, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (g >= STAGES && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
            fail();
            break;
          }
          mbar_expect_tx(&full_bar[s], S::A_BYTES + 2 * S::B_BYTES);
          tma_load_2d(stage_a(s), &tmA, &full_bar[s], it * BK, m0);
#pragma unroll
          for (int gi = 0; gi < BN / 32; ++gi) {
            tma_load_2d(stage_bb(s) + gi * S::B_GROUP, &tmBb, &full_bar[s], n0 + gi * 32, it * BK);
            tma_load_2d(stage_bs(s) + gi * S::B_GROUP, &tmBs, &full_bar[s], n0 + gi * 32, it * BK);
          }
        }
      }
      if (abort_sh) drain_tma_ring(full_bar, STAGES, g);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      int g = 0, tl = 0;  // k-iteration counter, local tile counter
      for (int tile = blockIdx.x; tile < total && !abort_sh; tile += gridDim.x, ++tl) {
        const int acc = tl & 1;
        if (tl >= 2 && !mbar_wait(&tempty_bar[acc], ((tl >> 1) - 1) & 1)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int it = 0; it < ktiles && !abort_sh; ++it, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (!mbar_wait(&conv_bar[s], r & 1)) {
            fail();
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(stage_a(s)), as = smem_u32(stage_as(s));
          const uint32_t bb = smem_u32(stage_bb(s)), bs = smem_u32(stage_bs(s));
#pragma unroll
          for (int j = 0; j < BK / 8; ++j) {
            // A: K-major, k-step of 8 tf32 = 32 bytes inside the row.
            const uint64_t da = smem_desc(a + j * 32, 16, S::A_SBO, S::A_LAYOUT);
            const uint64_t das = smem_desc(as + j * 32, 16, S::A_SBO, S::A_LAYOUT);
            // B: MN-major, 128-byte rows of 32 columns in 4-row (512 B) swizzle
            // atoms; a k-step of 8 rows advances 1 KiB; 32-column groups are
            // B_GROUP bytes apart.
            const uint64_t dbb = smem_desc(bb + j * 1024, S::B_GROUP, 512, 1);
            const uint64_t dbs = smem_desc(bs + j * 1024, S::B_GROUP, 512, 1);
            mma_tf32(d, das, dbb, idesc, (it | j) != 0);
            mma_tf32(d, da, dbs, idesc, 1);
            mma_tf32(d, da, dbb, idesc, 1);
          }
          mma_commit(&empty_bar[s]);  // stage s may be refilled once these MMAs finish
        }
        mma_commit(&tfull_bar[acc]);  // accumulator ready for the epilogue
      }
      if (abort_sh) drain_mma(&drain_bar);
    }
  } else if (warp < 2 + kConvThreads / 32) {  // ---------------- converter (warps 2..5)
    const int t = threadIdx.x - 64;
    int g = 0;
    for (int tile = blockIdx.x; tile < total && !abort_sh; tile += gridDim.x) {
      for (int it = 0; it < ktiles && !abort_sh; ++it, ++g) {
        const int s = g % STAGES, r = g / STAGES;
        if (!mbar_wait(&full_bar[s], r & 1)) {
          fail();
          break;
        }
        float4* a4 = reinterpret_cast<float4*>(stage_a(s));
        float4* as4 = reinterpret_cast<float4*>(stage_as(s));
#pragma unroll 4
        for (int i = t; i < (int)(S::A_BYTES / 16); i += kConvThreads) {
          const float4 v = a4[i];
#if INFERC_TC_RAW_A
          // The tensor core reads only the top 19 bits of a tf32 operand, so
          // raw A is its own "big" half; small = A - trunc13(A) (exact).
          float4 b;
          b.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
          b.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
          b.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
          b.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
#else
          float4 b;
          b.x = tf32_round(v.x); b.y = tf32_round(v.y); b.z = tf32_round(v.z); b.w = tf32_round(v.w);
          a4[i] = b;
#endif
          as4[i] = make_float4(v.x - b.x, v.y - b.y, v.z - b.z, v.w - b.w);
        }
        fence_proxy_async();  // generic-proxy writes -> visible to the tensor core
        mbar_arrive(&conv_bar[s]);
      }
    }
  } else {  // ---------------- epilogue (warps 6..13)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2 - kConvThreads / 32) >> 2;  // which half of the columns
    const bool vec_ok = (ldc & 3) == 0 && aligned16(C) &&
                        (EPI != EPI_BIAS_RESID || ((ep.ldr & 3) == 0 && aligned16(ep.resid))) &&
                        (EPI == EPI_GENERIC || aligned16(ep.bias));
    int tl = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++tl) {
      const int acc = tl & 1;
      const bool ok = !abort_sh && mbar_wait(&tfull_bar[acc], (tl >> 1) & 1);
      if (!ok) {
        fail();
        break;
      }
      tc_fence_after();
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
      const int64_t row = m0 + 32 * q + lane;
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
        float v[16];
        tmem_ld16(base + (uint32_t)c0, v);
        if (row >= M) continue;
        const int64_t col0 = (int64_t)n0 + c0;
        epilogue16<EPI>(ep, v, row, col0, N, C + row * ldc + col0, vec_ok);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);  // accumulator may be overwritten
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)(2 * BN)));
  }
}

// small = x - trunc13(x): with raw x used as the big operand (the tensor core
// reads only its top 19 bits), x itself need not be copied.
__global__ void split_small_kernel(const float* __restrict__ x, float* __restrict__ small,
                                   int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    small[i] = v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  }
}

__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ big,
                                  float* __restrict__ small, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float b = tf32_round(v);
    big[i] = b;
    small[i] = v - b;
  }
}

// ------------------------------------------------------------ host side
// 2-D fp32 map over a row-major [rows, cols] matrix with row stride ld
// (elements); box = box_cols x box_rows, 128-byte swizzle span.
CUtensorMap make_map(const float* base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_cols,
                     uint32_t box_rows, CUtensorMapSwizzle swz) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base),
                                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(INFERC_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

int sm_count_tc() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <int BN, int BK, int STAGES, int EPI>
void launch_tc(const float* A, int64_t lda, const float* Bb, const float* Bs, int64_t ldb,
               float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
               cudaStream_t st) {
  using S = TcShape<BN, BK, STAGES>;
  const CUtensorMap ta = make_map(A, M, K, lda, BK, BM,
                                  BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  const CUtensorMap tbb = make_map(Bb, K, N, ldb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  const CUtensorMap tbs = make_map(Bs, K, N, ldb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  IDEV_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel<BN, BK, STAGES, EPI>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)S::SMEM_BYTES));
  const int64_t tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM);
  dim3 grid((unsigned)std::min<int64_t>(tiles, sm_count_tc()));
  gemm_tf32x3_kernel<BN, BK, STAGES, EPI><<<grid, kThreadsTc, S::SMEM_BYTES, st>>>(
      ta, tbb, tbs, C, ldc, (int)M, (int)N, (int)K, ep);
  IDEV_LAUNCHED();
}

}  // namespace

bool gemm_tc_supported(const float* A, int64_t lda, const float* Bb, const float* Bs,
                       int64_t ldb, int64_t M, int64_t N, int64_t K) {
  return M >= 1 && N >= 1 && K >= 1 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) &&
         aligned16(A) && aligned16(Bb) && aligned16(Bs) && lda % 4 == 0 && ldb % 4 == 0 &&
         lda >= K && ldb >= N;
}

void launch_gemm_tc(const float* A, int64_t lda, const float* Bb, const float* Bs, int64_t ldb,
                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                    cudaStream_t st) {
  IDEV_CHECK_ARG(gemm_tc_supported(A, lda, Bb, Bs, ldb, M, N, K),
                 "tensor-core GEMM: unsupported shape or alignment");
  // Compile-time epilogue for the plan's three shapes; anything else (scalar
  // or full-matrix C, other activations) uses the generic one.
  int epi = EPI_GENERIC;
  if (ep.bias_mode == 1 && ep.act == ACT_NONE && ep.resid == nullptr) epi = EPI_BIAS;
  if (ep.bias_mode == 1 && ep.act == ACT_GELU_ERF && ep.resid == nullptr) epi = EPI_BIAS_GELU;
  if (ep.bias_mode == 1 && ep.act == ACT_NONE && ep.resid != nullptr) epi = EPI_BIAS_RESID;
  // BN = 256 when there are enough output tiles to fill the SMs, else BN =
  // 128 (twice the CTAs; three stages fit in shared memory).
  const int64_t tiles256 = ((N + 255) / 256) * ((M + BM - 1) / BM);
  const bool wide = tiles256 >= sm_count_tc() / 2;
#define IDEV_TC(EPIK)                                                                 \
  do {                                                                                \
    if (wide)                                                                         \
      launch_tc<256, 32, 2, EPIK>(A, lda, Bb, Bs, ldb, C, ldc, M, N, K, ep, st);     \
    else                                                                              \
      launch_tc<128, 32, 3, EPIK>(A, lda, Bb, Bs, ldb, C, ldc, M, N, K, ep, st);     \
  } while (0)
  switch (epi) {
    case EPI_BIAS: IDEV_TC(EPI_BIAS); break;
    case EPI_BIAS_GELU: IDEV_TC(EPI_BIAS_GELU); break;
    case EPI_BIAS_RESID: IDEV_TC(EPI_BIAS_RESID); break;
    default: IDEV_TC(EPI_GENERIC); break;
  }
#undef IDEV_TC
}

void launch_split_small(const float* x, float* small, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8);
  split_small_kernel<<<blocks, 256, 0, st>>>(x, small, n);
  IDEV_LAUNCHED();
}

void launch_split_tf32(const float* x, float* big, float* small, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8);
  split_tf32_kernel<<<blocks, 256, 0, st>>>(x, big, small, n);
  IDEV_LAUNCHED();
}

int read_and_clear_attn_tc_error();
int read_and_clear_f16_error();
int read_and_clear_int4_tc_error();
int read_and_clear_f16_2cta_error();
int read_and_clear_attn_f16_error();
int read_and_clear_selftest_error();

int read_and_clear_tc_error() {
  const int others = read_and_clear_attn_tc_error() | read_and_clear_f16_error() |
                     read_and_clear_int4_tc_error() | read_and_clear_f16_2cta_error() |
                     read_and_clear_attn_f16_error() | read_and_clear_selftest_error();
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int)));
  }
  return v | others;
}

}  // namespace inferc_dev
