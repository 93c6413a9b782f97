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
// tf32 MMAs per product. B (the weight) is split once into two [K,N] arrays
// in HBM (split_tf32_kernel); A (the activation) is split in shared memory by
// the converter warps as each tile arrives.
//
// CTA tile 128 x BN x 32 (K), STAGES-deep TMA ring. Warp roles (192 threads):
//   warp 0      TMA producer (one lane): A tile, B_big tile, B_small tile
//   warp 1      TMEM allocation + MMA issuer (one lane)
//   warps 2..5  converter (A -> A_big in place + A_small) and epilogue
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

#include <mutex>

#include "kernels.cuh"

namespace inferc_dev {
namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // fp32 elements per 128-byte swizzle row
constexpr int kThreadsTc = 192;
constexpr uint32_t kSpinLimit = 1u << 22;

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor (version 1, base offset 0).
// layout: 2 = SWIZZLE_128B (K-major A), 1 = SWIZZLE_128B with 32-byte atoms
// (the only layout the tensor core accepts for MN-major tf32, used for B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)layout << 61;
  return d;
}

// Instruction descriptor: kind::tf32, D fp32, A K-major, B MN-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4)                    // D format f32
         | (2u << 7)                  // A format tf32
         | (2u << 10)                 // B format tf32
         | (0u << 15)                 // A K-major
         | (1u << 16)                 // B MN-major
         | ((uint32_t)(n >> 3) << 17)  // N / 8
         | ((uint32_t)(m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

}  // namespace
}  // namespace inferc_dev

namespace inferc_dev {

__device__ int g_tc_error;  // set to 1 by a CTA whose barrier wait timed out

namespace {

template <int BN, int STAGES>
struct TcShape {
  static constexpr uint32_t A_BYTES = BM * BK * 4;  // 16 KiB
  static constexpr uint32_t B_BYTES = BK * BN * 4;  // BN x 128 B
  static constexpr uint32_t STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32,256]");
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreadsTc, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmBb,
                       const __grid_constant__ CUtensorMap tmBs, float* __restrict__ C,
                       int64_t ldc, int M, int N, int K, Epilogue ep) {
  using S = TcShape<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES], conv_bar[STAGES], empty_bar[STAGES];
  __shared__ __align__(8) uint64_t accum_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int ktiles = (K + BK - 1) / BK;
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
      mbar_init(&conv_bar[s], 128);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&accum_bar, 1);
    abort_sh = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"((uint32_t)BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      for (int it = 0; it < ktiles && !abort_sh; ++it) {
        const int s = it % STAGES, r = it / STAGES;
        if (it >= STAGES && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
          fail();
          break;
        }
        mbar_expect_tx(&full_bar[s], S::A_BYTES + 2 * S::B_BYTES);
        tma_load_2d(stage_a(s), &tmA, &full_bar[s], it * BK, m0);
#pragma unroll
        for (int g = 0; g < BN / 32; ++g) {
          tma_load_2d(stage_bb(s) + g * 4096, &tmBb, &full_bar[s], n0 + g * 32, it * BK);
          tma_load_2d(stage_bs(s) + g * 4096, &tmBs, &full_bar[s], n0 + g * 32, it * BK);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      for (int it = 0; it < ktiles && !abort_sh; ++it) {
        const int s = it % STAGES, r = it / STAGES;
        if (!mbar_wait(&conv_bar[s], r & 1)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(stage_a(s)), as = smem_u32(stage_as(s));
        const uint32_t bb = smem_u32(stage_bb(s)), bs = smem_u32(stage_bs(s));
#pragma unroll
        for (int j = 0; j < BK / 8; ++j) {
          // A: K-major, k-step of 8 tf32 = 32 bytes inside the 128-byte row.
          const uint64_t da = smem_desc(a + j * 32, 16, 1024, 2);
          const uint64_t das = smem_desc(as + j * 32, 16, 1024, 2);
          // B: MN-major, 128-byte rows of 32 columns in 4-row (512 B) swizzle
          // atoms; a k-step of 8 rows advances 1 KiB; 32-column groups are
          // 4 KiB apart.
          const uint64_t dbb = smem_desc(bb + j * 1024, 4096, 512, 1);
          const uint64_t dbs = smem_desc(bs + j * 1024, 4096, 512, 1);
          mma_tf32(tmem, das, dbb, idesc, (it | j) != 0);
          mma_tf32(tmem, da, dbs, idesc, 1);
          mma_tf32(tmem, da, dbb, idesc, 1);
        }
        mma_commit(&empty_bar[s]);  // stage s may be refilled once these MMAs finish
      }
      mma_commit(&accum_bar);
    }
  } else {  // ---------------- converter + epilogue (warps 2..5)
    const int t = threadIdx.x - 64;
    for (int it = 0; it < ktiles && !abort_sh; ++it) {
      const int s = it % STAGES, r = it / STAGES;
      if (!mbar_wait(&full_bar[s], r & 1)) {
        fail();
        break;
      }
      float4* a4 = reinterpret_cast<float4*>(stage_a(s));
      float4* as4 = reinterpret_cast<float4*>(stage_as(s));
#pragma unroll 4
      for (int i = t; i < (int)(S::A_BYTES / 16); i += 128) {
        const float4 v = a4[i];
        float4 b;
        b.x = tf32_round(v.x); b.y = tf32_round(v.y); b.z = tf32_round(v.z); b.w = tf32_round(v.w);
        a4[i] = b;
        as4[i] = make_float4(v.x - b.x, v.y - b.y, v.z - b.z, v.w - b.w);
      }
      fence_proxy_async();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(&conv_bar[s]);
    }
    const bool ok = !abort_sh && mbar_wait(&accum_bar, 0);
    if (!ok) fail();
    tc_fence_after();
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int64_t row = m0 + 32 * q + lane;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
      if (!ok || row >= M) continue;
      const int64_t col0 = (int64_t)n0 + c0;
      float o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        o[i] = (col0 + i < N) ? epilogue_apply(ep, v[i], row, col0 + i) : 0.f;
      float* dst = C + row * ldc + col0;
      if (col0 + 16 <= N && (ldc & 3) == 0) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
      } else {
        for (int i = 0; i < 16; ++i)
          if (col0 + i < N) dst[i] = o[i];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)BN));
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
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  if (!fn) throw Error(INFERC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

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

template <int BN, int STAGES>
void launch_tc(const float* A, int64_t lda, const float* Bb, const float* Bs, int64_t ldb,
               float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
               cudaStream_t st) {
  using S = TcShape<BN, STAGES>;
  const CUtensorMap ta = make_map(A, M, K, lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tbb = make_map(Bb, K, N, ldb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  const CUtensorMap tbs = make_map(Bs, K, N, ldb, 32, BK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  IDEV_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel<BN, STAGES>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)S::SMEM_BYTES));
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  gemm_tf32x3_kernel<BN, STAGES><<<grid, kThreadsTc, S::SMEM_BYTES, st>>>(
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
  launch_tc<256, 2>(A, lda, Bb, Bs, ldb, C, ldc, M, N, K, ep, st);
}

void launch_split_tf32(const float* x, float* big, float* small, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8);
  split_tf32_kernel<<<blocks, 256, 0, st>>>(x, big, small, n);
  IDEV_LAUNCHED();
}

int read_and_clear_tc_error() {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int)));
  }
  return v;
}

}  // namespace inferc_dev
