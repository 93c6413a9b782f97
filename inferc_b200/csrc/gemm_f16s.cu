// fp32-accurate GEMM on the fp16 tensor cores ("split fp16"), with the Gemm
// epilogue fused. Same contract as the 3xTF32 kernel (gemm_tc.cu):
//
//   C[M,N] = epilogue(A[M,K] B[K,N]),  A fp32 row-major.
//
// Every fp32 operand is written as x = hi + lo, hi = fp16_rn(x) and
// lo = fp16_rn(x - hi) (x - hi is exact in fp32), and the product is
// accumulated in fp32 TMEM as lo_a*hi_b + hi_a*lo_b + hi_a*hi_b: three
// kind::f16 MMAs, which run at twice the kind::tf32 rate, so this costs half
// the tensor-core time of 3xTF32 for the same ~22 bits per operand.
//   * B (the weight) is split once, ahead of time, into two fp16 [N, Kp]
//     planes (K-major), after scaling by a power of two 2^s chosen so that
//     max|B| 2^s < 2^14: then lo stays in fp16's normal range for every
//     element within 2^-11 of max|B|'s binade, and the epilogue multiplies
//     the accumulator by 2^-s (exact).
//   * A (the activation) is split in shared memory by the converter warps
//     as each fp32 tile lands, in place (the 32 KiB fp32 tile becomes the
//     16 KiB hi plane and the 16 KiB lo plane). Elements below 2^-14 in
//     magnitude keep an absolute error under 2^-25 (fp16 subnormal lo).
//     An element with |a| >= 65520 (or inf / NaN) has no fp16 hi: the
//     converter sets *range_flag, and the caller must rerun that GEMM on
//     the 3xTF32 kernel (the encoder plan does so for the whole batch).
//
// Persistent kernel, one CTA per SM striding over 128 x BN output tiles,
// STAGES-deep TMA ring, two TMEM accumulators (the epilogue of one tile
// overlaps the MMAs of the next). Warp roles (448 threads):
//   warp 0       TMA producer (one lane): A (fp32, two 32-column boxes),
//                B_hi, B_lo (fp16, 64 x BN)
//   warp 1       TMEM allocation + MMA issuer (one lane)
//   warps 2..5   converter (one thread per A row: fp32 -> hi | lo planes)
//   warps 6..13  epilogue (two warps per TMEM lane quarter)
// Shared-memory operands are canonical K-major SWIZZLE_128B UMMA layouts
// (128-byte rows of 64 fp16, 8-row atoms of 1 KiB).
// Every mbarrier wait is bounded; on a timeout the CTA flags g_f16_error,
// stops issuing work, frees its TMEM and exits.
#include <algorithm>
#include <cuda.h>
#include <cuda_fp16.h>

#include "gemm_epi.cuh"
#include "kernels.cuh"
#include <cstdlib>

#include "tc_ptx.cuh"

namespace inferc_dev {

__device__ int g_f16_error;  // a barrier wait timed out
__device__ int g_f16_range;  // default range flag of op-level calls


namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int kConvThreads = 128;  // warps 2..5
constexpr int kEpiThreads = 256;   // warps 6..13
constexpr int kThreadsF16 = 64 + kConvThreads + kEpiThreads;
constexpr uint32_t A_BOX_BYTES = BM * 32 * 4;  // one [128 x 32] fp32 TMA box, 16 KiB

// BK = 64: fp16 rows of 128 B (SWIZZLE_128B, 16-byte chunk c of row r at
// c ^ (r % 8)); BK = 32: rows of 64 B (SWIZZLE_64B, chunk c at
// c ^ ((r / 2) % 4)). Both have 8-row core-matrix groups (SBO = 8 rows).
template <int BN, int BK, int STAGES>
struct F16Shape {
  static constexpr uint32_t A_F32_BYTES = BM * BK * 4;   // BK / 32 fp32 boxes
  static constexpr uint32_t A_PLANE_BYTES = BM * BK * 2;  // the hi plane, then the lo plane
  static constexpr uint32_t ROW_BYTES = BK * 2;
  static constexpr uint32_t LAYOUT = BK == 64 ? 2 : 4;  // UMMA SWIZZLE_128B / _64B
  static constexpr uint32_t SBO = 8 * ROW_BYTES;
  static constexpr uint32_t B_BYTES = BN * BK * 2;  // one fp16 plane
  static constexpr uint32_t STAGE_BYTES = A_F32_BYTES + 2 * B_BYTES;
  static constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  // two accumulators of BN columns; TMEM is allocated in powers of two
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static_assert(BK == 32 || BK == 64, "BK must be 32 or 64");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32,256]");
  static __device__ __forceinline__ uint32_t chunk_swz(int r) {
    return BK == 64 ? (uint32_t)(r & 7) : (uint32_t)((r >> 1) & 3);
  }
};

// Instruction descriptor: kind::f16 with f16 A and B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4)                       // D format f32
         | (0u << 7) | (0u << 10)        // A, B format f16
         | ((uint32_t)(n >> 3) << 17)    // N / 8
         | ((uint32_t)(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// OR of `v` over the 128 converter threads (named barrier 1).
__device__ __forceinline__ bool conv_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(kConvThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) {
  return *reinterpret_cast<uint32_t*>(&h);
}

// AS: A arrives already split (fp16 hi / lo planes, tmA / tmAl), so the
// converter warps idle and the MMA waits on the TMA barrier directly.
// SOUT: the epilogue writes the fp16 hi / lo split of its result (so.hi,
// so.lo) instead of fp32 C, for a following split-fp16 GEMM.
template <int BN, int BK, int STAGES, int EPI, bool AS, bool SOUT>
__global__ void __launch_bounds__(kThreadsF16, 1)
    gemm_f16s_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmAl,
                     const __grid_constant__ CUtensorMap tmBh,
                     const __grid_constant__ CUtensorMap tmBl, const float* __restrict__ b_inv_scale,
                     int* __restrict__ range_flag, float* __restrict__ C, int64_t ldc, int M, int N,
                     int K, Epilogue ep, SplitOut so, int splits, int kper,
                     float* __restrict__ part, unsigned* __restrict__ cnt) {
  using S = F16Shape<BN, BK, STAGES>;
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
  // work units: (tile, k split); unit u covers k tiles [kb0, kb1) of tile u / splits
  const int units = total * splits;
  auto krange = [&](int u, int& kb0, int& kb1) {
    kb0 = (u % splits) * kper;
    kb1 = min(ktiles, kb0 + kper);
  };
  auto stage_a = [&](int s) { return smem + (size_t)s * S::STAGE_BYTES; };
  auto stage_bh = [&](int s) { return stage_a(s) + S::A_F32_BYTES; };
  auto stage_bl = [&](int s) { return stage_a(s) + S::A_F32_BYTES + S::B_BYTES; };
  auto fail = [&]() {
    abort_sh = 1;
    atomicExch(&g_f16_error, 1);
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
                 "r"(S::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  // A, the residual and the outputs' previous readers belong to earlier
  // kernels. Dependents are released at the end: released at the start,
  // their early CTAs slowed config 0 (0.476 -> 0.511 ms per sequence), at
  // the end it measured 0.463.
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int g = 0;
      for (int u = blockIdx.x; u < units && !abort_sh; u += gridDim.x) {
        const int tile = u / splits;
        const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
        int kb0, kb1;
        krange(u, kb0, kb1);
        for (int it = kb0; it < kb1 && !abort_sh; ++it, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (g >= STAGES && !mbar_wait(&empty_bar[s], (r - 1) & 1)) {
            fail();
            break;
          }
          mbar_expect_tx(&full_bar[s], S::A_F32_BYTES + 2 * S::B_BYTES);
          if (AS) {
            tma_load_2d(stage_a(s), &tmA, &full_bar[s], it * BK, m0);
            tma_load_2d(stage_a(s) + S::A_PLANE_BYTES, &tmAl, &full_bar[s], it * BK, m0);
          } else {
#pragma unroll
            for (int kb = 0; kb < BK / 32; ++kb)
              tma_load_2d(stage_a(s) + kb * A_BOX_BYTES, &tmA, &full_bar[s], it * BK + kb * 32,
                          m0);
          }
          tma_load_2d(stage_bh(s), &tmBh, &full_bar[s], it * BK, n0);
          tma_load_2d(stage_bl(s), &tmBl, &full_bar[s], it * BK, n0);
        }
      }
      if (abort_sh) drain_tma_ring(full_bar, STAGES, g);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16(BM, BN);
      int g = 0, tl = 0;
      for (int u = blockIdx.x; u < units && !abort_sh; u += gridDim.x, ++tl) {
        int kb0, kb1;
        krange(u, kb0, kb1);
        const int acc = tl & 1;
        if (tl >= 2 && !mbar_wait(&tempty_bar[acc], ((tl >> 1) - 1) & 1)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int it = kb0; it < kb1 && !abort_sh; ++it, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (!mbar_wait(AS ? &full_bar[s] : &conv_bar[s], r & 1)) {
            fail();
            break;
          }
          tc_fence_after();
          const uint32_t ah = smem_u32(stage_a(s)), al = ah + S::A_PLANE_BYTES;
          const uint32_t bh = smem_u32(stage_bh(s)), bl = smem_u32(stage_bl(s));
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {  // k-step of 16 fp16 = 32 bytes of a row
            const uint64_t dah = smem_desc(ah + j * 32, 16, S::SBO, S::LAYOUT);
            const uint64_t dal = smem_desc(al + j * 32, 16, S::SBO, S::LAYOUT);
            const uint64_t dbh = smem_desc(bh + j * 32, 16, S::SBO, S::LAYOUT);
            const uint64_t dbl = smem_desc(bl + j * 32, 16, S::SBO, S::LAYOUT);
            mma_f16(d, dal, dbh, idesc, (it != kb0 || j != 0) ? 1u : 0u);
            mma_f16(d, dah, dbl, idesc, 1);
            mma_f16(d, dah, dbh, idesc, 1);
          }
          mma_commit(&empty_bar[s]);
        }
        mma_commit(&tfull_bar[acc]);
      }
      if (abort_sh) drain_mma(&drain_bar);
    }
  } else if (warp < 2 + kConvThreads / 32) {  // ---------------- converter (warps 2..5)
    if (!AS) {
    const int r = threadIdx.x - 64;  // A row of the tile
    const uint32_t sw32 = (uint32_t)(r & 7);  // fp32 landing boxes: 128-byte rows
    const uint32_t sw = S::chunk_swz(r);
    int g = 0;
    bool bad = false, stop = false;
    for (int u = blockIdx.x; u < units && !stop; u += gridDim.x) {
      int kb0, kb1;
      krange(u, kb0, kb1);
      for (int it = kb0; it < kb1; ++it, ++g) {
        const int s = g % STAGES, rr = g / STAGES;
        const bool ok = mbar_wait(&full_bar[s], rr & 1);
        if (!ok) fail();
        uint8_t* a = stage_a(s);
        float x[BK];
        if (ok) {
#pragma unroll
          for (int kb = 0; kb < BK / 32; ++kb)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float4 v = *reinterpret_cast<const float4*>(a + kb * A_BOX_BYTES + r * 128 +
                                                                ((c ^ sw32) << 4));
              x[kb * 32 + c * 4 + 0] = v.x;
              x[kb * 32 + c * 4 + 1] = v.y;
              x[kb * 32 + c * 4 + 2] = v.z;
              x[kb * 32 + c * 4 + 3] = v.w;
            }
        }
        // All reads of the tile before any in-place write; the same barrier
        // makes the converters agree on stopping (it must be reached by all
        // 128 of them every iteration).
        stop = conv_any(!ok || abort_sh != 0);
        if (stop) break;
#pragma unroll
        for (int cc = 0; cc < BK / 8; ++cc) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float u = x[cc * 8 + 2 * p], w = x[cc * 8 + 2 * p + 1];
            bad |= !(fabsf(u) < 65520.f) || !(fabsf(w) < 65520.f);
            const __half2 h = __floats2half2_rn(u, w);
            const float2 hf = __half22float2(h);
            hw[p] = h2_bits(h);
            lw[p] = h2_bits(__floats2half2_rn(u - hf.x, w - hf.y));
          }
          const uint32_t off = r * S::ROW_BYTES + ((cc ^ sw) << 4);
          *reinterpret_cast<uint4*>(a + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(a + S::A_PLANE_BYTES + off) =
              make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async();
        mbar_arrive(&conv_bar[s]);
      }
    }
    if (bad) atomicExch(range_flag, 1);
    }
  } else {  // ---------------- epilogue (warps 6..13)
    const int q = warp & 3;
    const int half = (warp - 2 - kConvThreads / 32) >> 2;
    const bool vec_ok = (ldc & 3) == 0 && aligned16(C) &&
                        (EPI != EPI_BIAS_RESID || ((ep.ldr & 3) == 0 && aligned16(ep.resid))) &&
                        (EPI == EPI_GENERIC || aligned16(ep.bias));
    const float sc = __ldg(b_inv_scale);
    bool bad = false;
    int tl = 0;
    // staging rows of the fp32-residual and split-plane fast paths
    __shared__ __align__(16) float stage[kEpiThreads / 32][32 * 20];
    __shared__ int last_sh;
    const int et = threadIdx.x - 64 - kConvThreads;  // 0 .. kEpiThreads-1
    auto epi_sync = [] { asm volatile("bar.sync 2, %0;" ::"r"(kEpiThreads) : "memory"); };
    // AND over the epilogue threads (barrier 2): with split K they meet at
    // epi_sync, so all must leave the loop together
    auto epi_all = [](bool v) {
      uint32_t r;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\t"
          "setp.ne.u32 p, %1, 0;\n\t"
          "bar.red.and.pred q, 2, %2, p;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(r)
          : "r"((uint32_t)v), "r"(kEpiThreads)
          : "memory");
      return r != 0;
    };
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
      const int tile = u / splits;
      const int acc = tl & 1;
      bool ok = !abort_sh && mbar_wait(&tfull_bar[acc], (tl >> 1) & 1);
      if (splits > 1) ok = epi_all(ok);
      if (!ok) {
        fail();
        break;
      }
      tc_fence_after();
      const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
      const int64_t row = m0 + 32 * q + lane;
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN);
      // whole-tile fast paths below (warp-uniform); split outputs have
      // aligned planes and bias by the dispatcher's checks
      const bool staged = (SOUT || vec_ok) && n0 + BN <= N;
      // the epilogue of 16 accumulator columns c0.. of this thread's row
      auto finish = [&](int c0, float (&v)[16]) {
          if constexpr (EPI == EPI_BIAS_RESID && !SOUT) {
            if (staged) {
              // fp32 + residual, staged through shared memory: the warp's
              // 32 rows x 16 columns are written row per lane (rows padded to
              // 20 floats: conflict-free float4 stores) and read back as
              // float4s that cover 8 rows x 64 contiguous bytes per warp
              // instruction, so the residual loads and C stores use whole
              // 32-byte sectors. Arithmetic as in epilogue16<EPI_BIAS_RESID>.
              float* wb = stage[warp - 2 - kConvThreads / 32];
  #pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<float4*>(wb + lane * 20)[j] =
                    make_float4(v[4 * j] * sc, v[4 * j + 1] * sc, v[4 * j + 2] * sc,
                                v[4 * j + 3] * sc);
              __syncwarp();
              const int c4 = (lane & 3) * 4;
              const int64_t col = (int64_t)n0 + c0 + c4;
              const float4 bb = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
              float4 rr[4];
  #pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int64_t grow = m0 + 32 * q + (lane >> 2) + 8 * k;
                rr[k] = grow < M ? *reinterpret_cast<const float4*>(ep.resid + grow * ep.ldr + col)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
              }
  #pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int rl = (lane >> 2) + 8 * k;
                const int64_t grow = m0 + 32 * q + rl;
                if (grow >= M) continue;
                const float4 x = *reinterpret_cast<const float4*>(wb + rl * 20 + c4);
                float4 o;
                o.x = ep.alpha * x.x + ep.beta * bb.x; o.x += rr[k].x;
                o.y = ep.alpha * x.y + ep.beta * bb.y; o.y += rr[k].y;
                o.z = ep.alpha * x.z + ep.beta * bb.z; o.z += rr[k].z;
                o.w = ep.alpha * x.w + ep.beta * bb.w; o.w += rr[k].w;
                *reinterpret_cast<float4*>(C + grow * ldc + col) = o;
              }
              __syncwarp();
              return;
            }
          }
          if constexpr (SOUT && (EPI == EPI_BIAS || EPI == EPI_BIAS_GELU)) {
            if (staged) {
              // fp16 hi / lo planes, staged the same way: each lane finishes 4
              // columns of a row and writes 8 contiguous bytes to each plane
              // (8 rows x 32 bytes per warp instruction). Arithmetic as in
              // epilogue16_split<EPI>.
              float* wb = stage[warp - 2 - kConvThreads / 32];
  #pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<float4*>(wb + lane * 20)[j] =
                    make_float4(v[4 * j] * sc, v[4 * j + 1] * sc, v[4 * j + 2] * sc,
                                v[4 * j + 3] * sc);
              __syncwarp();
              const int c4 = (lane & 3) * 4;
              const int64_t col = (int64_t)n0 + c0 + c4;
              const float4 bb = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
  #pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int rl = (lane >> 2) + 8 * k;
                const int64_t grow = m0 + 32 * q + rl;
                if (grow >= M) continue;
                const float4 x = *reinterpret_cast<const float4*>(wb + rl * 20 + c4);
                float o[4] = {ep.alpha * x.x + ep.beta * bb.x, ep.alpha * x.y + ep.beta * bb.y,
                              ep.alpha * x.z + ep.beta * bb.z, ep.alpha * x.w + ep.beta * bb.w};
                if (EPI == EPI_BIAS_GELU) {
  #pragma unroll
                  for (int i = 0; i < 4; ++i) o[i] = gelu_erf(o[i]);
                }
                uint32_t l0, l1;
                const uint32_t h0 = split_pair(o[0], o[1], l0, bad);
                const uint32_t h1 = split_pair(o[2], o[3], l1, bad);
                *reinterpret_cast<uint2*>(so.hi + grow * so.ld + col) = make_uint2(h0, h1);
                *reinterpret_cast<uint2*>(so.lo + grow * so.ld + col) = make_uint2(l0, l1);
              }
              __syncwarp();
              return;
            }
          }
          if (row >= M) return;
  #pragma unroll
          for (int i = 0; i < 16; ++i) v[i] *= sc;
          const int64_t col0 = (int64_t)n0 + c0;
          if (SOUT) {
            // N % 16 == 0 for split outputs: a chunk is wholly inside or outside
            if (col0 < N) epilogue16_split<EPI>(ep, v, row, col0, so, bad);
          } else {
            epilogue16<EPI>(ep, v, row, col0, N, C + row * ldc + col0, vec_ok);
          }
      };
      if (splits == 1) {
#pragma unroll 1
        for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
          float v[16];
          tmem_ld16(base + (uint32_t)c0, v);
          finish(c0, v);
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
        continue;
      }
      // Split K: this unit's raw partial tile to the scratch, the accumulator
      // released, then the CTA that completes the tile's count sums the
      // partials in split order and finishes the tile.
      float* pu = part + ((size_t)u * BM + 32 * q + lane) * BN;
#pragma unroll 1
      for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
        float v[16];
        tmem_ld16(base + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<float4*>(pu + c0)[i] =
              make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      __threadfence();
      epi_sync();
      if (et == 0) last_sh = atomicAdd(cnt + tile, 1u) == (unsigned)(splits - 1);
      epi_sync();
      if (!last_sh) continue;
      __threadfence();
      const float* pt = part + ((size_t)tile * splits * BM + 32 * q + lane) * BN;
#pragma unroll 1
      for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        for (int k = 0; k < splits; ++k) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 w =
                __ldcg(reinterpret_cast<const float4*>(pt + (size_t)k * BM * BN + c0) + i);
            v[4 * i] += w.x;
            v[4 * i + 1] += w.y;
            v[4 * i + 2] += w.z;
            v[4 * i + 3] += w.w;
          }
        }
        finish(c0, v);
      }
      if (et == 0) cnt[tile] = 0u;  // zero at rest for the next call on this stream
    }
    if (SOUT && bad) atomicExch(so.range, 1);
  }
  tc_fence_before();
  __syncthreads();
  pdl_launch_dependents();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(S::TMEM_COLS));
  }
}

// ------------------------------------------------------------ weight split
__global__ void absmax_kernel(const float* __restrict__ w, int64_t rows, int64_t cols, int64_t ld,
                              unsigned int* __restrict__ out_bits) {
  float m = 0.f;
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(w[(i / cols) * ld + i % cols]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));  // m >= 0
}

// W [K, N] fp32 (row stride ldw; trans: W is [N, K]) -> hi, lo [N, Kp]
// fp16 of W * 2^s, with columns K..Kp-1 zero; writes 2^-s to *inv_scale.
__global__ void split_weight_f16_kernel(const float* __restrict__ w, int64_t K, int64_t N,
                                        int64_t ldw, bool trans, int64_t kp,
                                        const unsigned int* amax_bits,
                                        __half* __restrict__ hi, __half* __restrict__ lo,
                                        float* __restrict__ inv_scale) {
  __shared__ float tile[32][33];
  const float amax = __uint_as_float(*amax_bits);
  int e = 0;
  if (amax > 0.f && amax <= 3.0e38f) frexpf(amax, &e);  // amax < 2^e
  const int s = 14 - e;
  const float scale = ldexpf(1.0f, s);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && threadIdx.y == 0)
    *inv_scale = ldexpf(1.0f, -s);
  const int64_t k0 = (int64_t)blockIdx.y * 32, n0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t k = k0 + i, n = n0 + threadIdx.x;
    const int64_t kt = k0 + threadIdx.x, nt = n0 + i;  // transposed source: coalesced in k
    if (trans)
      tile[threadIdx.x][i] = (kt < K && nt < N) ? w[nt * ldw + kt] * scale : 0.f;
    else
      tile[i][threadIdx.x] = (k < K && n < N) ? w[k * ldw + n] * scale : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < kp) {
      const float v = tile[threadIdx.x][i];
      const __half h = __float2half_rn(v);
      hi[n * kp + k] = h;
      lo[n * kp + k] = __float2half_rn(v - __half2float(h));
    }
  }
}

// x [rows, cols] fp32 (row stride ldx) -> fp16 hi / lo planes (row stride ld).
__global__ void split_rows_f16_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                      int64_t ldx, uint16_t* __restrict__ hi,
                                      uint16_t* __restrict__ lo, int64_t ld, int* range) {
  bool bad = false;
  const int64_t pairs = cols / 2, n = rows * pairs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / pairs, c = 2 * (i % pairs);
    uint32_t l;
    const uint32_t h = split_pair(x[r * ldx + c], x[r * ldx + c + 1], l, bad);
    *reinterpret_cast<uint32_t*>(hi + r * ld + c) = h;
    *reinterpret_cast<uint32_t*>(lo + r * ld + c) = l;
  }
  if (bad) atomicExch(range, 1);
}

// ------------------------------------------------------------ host side
int sm_count_f16() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <int BN, int BK, int STAGES, int EPI, bool AS, bool SOUT>
void launch_f16s(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                 const float* inv_scale, int* range_flag, float* C, int64_t ldc,
                 const SplitOut& so, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                 cudaStream_t st, const SplitK& sk) {
  using S = F16Shape<BN, BK, STAGES>;
  const CUtensorMapSwizzle hswz = BK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap ta, tal;
  if (AS) {
    ta = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A.hi, M, K, A.ld, BK, BM, hswz);
    tal = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A.lo, M, K, A.ld, BK, BM, hswz);
  } else {
    ta = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, A.a32, M, K, A.ld, 32, BM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    tal = ta;
  }
  const CUtensorMap tbh = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bh, N, kp, kp, BK, BN, hswz);
  const CUtensorMap tbl = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bl, N, kp, kp, BK, BN, hswz);
  auto kern = gemm_f16s_kernel<BN, BK, STAGES, EPI, AS, SOUT>;
  IDEV_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)S::SMEM_BYTES));
  const int64_t tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM);
  const int64_t sms = sm_count_f16();
  const int64_t ktiles = (K + BK - 1) / BK;
  // Split K when the tiles leave most SMs idle: at least 8 k tiles per split
  // (the partial-tile fix-up costs a few microseconds, so at K = 768 a split
  // measured slower: FFN1 at M = 128 14.5 -> 20.6 us with 4 k tiles per
  // split), as many splits as the SMs and the caller's scratch allow.
  int64_t splits = 1;
  if (sk.part && sk.cnt && tiles * 2 <= sms && tiles <= sk.cnt_n)
    splits = std::max<int64_t>(1, std::min({sms / tiles, ktiles / 8,
                                            sk.part_floats / (tiles * BM * BN)}));
  const int64_t kper = (ktiles + splits - 1) / splits;
  splits = (ktiles + kper - 1) / kper;  // no empty split
  dim3 grid((unsigned)std::min<int64_t>(tiles * splits, sms));
  launch_pdl(kern, grid, dim3(kThreadsF16), S::SMEM_BYTES, st, ta, tal, tbh, tbl, inv_scale,
             range_flag, C, ldc, (int)M, (int)N, (int)K, ep, so, (int)splits, (int)kper, sk.part,
             sk.cnt);
  IDEV_LAUNCHED();
}

template <int EPI, bool AS, bool SOUT>
void launch_f16s_width(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                       const float* inv_scale, int* range_flag, float* C, int64_t ldc,
                       const SplitOut& so, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                       cudaStream_t st, const SplitK& sk) {
  // Tile width by wave quantisation: of BN = 256, 192 and 128 the one whose
  // tile count fills the SMs' last wave best (a larger BN on a tie, for
  // operand reuse). N = 768 at M = 4096 (a rank's share of the batch-256
  // encoder on 8 GPUs) gets 128 tiles of 192 columns in one 86 % wave
  // instead of 96 tiles of 256 (65 %). INFERC_GEMM_BN forces a width.
  // Pre-split A with K <= 1024: BK = 64 (128-byte TMA rows, 2 stages) —
  // measured 7-9 % faster than BK = 32 at K = 768, where the 64-byte rows of
  // BK = 32 limit the TMA request rate; longer K keeps BK = 32 (4 stages).
  const int64_t sms = sm_count_f16();
  auto util = [&](int64_t bn) {
    const int64_t t = ((N + bn - 1) / bn) * ((M + BM - 1) / BM);
    return (double)t / (double)(((t + sms - 1) / sms) * sms);
  };
  int bn = 256;
  for (int cand : {192, 128})
    if (util(cand) > util(bn) + 1e-9) bn = cand;
  // Small M (a handful of tiles): narrower tiles spread the weight stream over
  // more SMs (config 0's M = 128 GEMMs).
  const int64_t tiles128 = ((N + 127) / 128) * ((M + BM - 1) / BM);
  if (tiles128 * 4 <= sms) bn = (tiles128 * 8 <= sms && N >= 32) ? 32 : 64;
  static const int forced = [] {
    const char* e = std::getenv("INFERC_GEMM_BN");
    return e ? std::atoi(e) : 0;
  }();
  if (forced == 32 || forced == 64 || forced == 128 || forced == 192 || forced == 256) bn = forced;
  const bool bk64 = AS && K <= 1024;
  if (bn == 256) {
    if (bk64)
      launch_f16s<256, 64, 2, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                             N, K, ep, st, sk);
    else
      launch_f16s<256, 32, 4, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                             N, K, ep, st, sk);
  } else if (bn == 192) {
    if (bk64)
      launch_f16s<192, 64, 2, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                             N, K, ep, st, sk);
    else
      launch_f16s<192, 32, 4, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                             N, K, ep, st, sk);
  } else if (bn == 128) {
    launch_f16s<128, 32, 6, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                           N, K, ep, st, sk);
  } else if (bn == 64) {
    // narrow tiles stream mostly A: 128-byte TMA rows (BK = 64) for the planes
    if (AS)
      launch_f16s<64, 64, 4, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                            N, K, ep, st, sk);
    else
      launch_f16s<64, 32, 8, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                            N, K, ep, st, sk);
  } else {
    if (AS)
      launch_f16s<32, 64, 4, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                            N, K, ep, st, sk);
    else
      launch_f16s<32, 32, 8, EPI, AS, SOUT>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                            N, K, ep, st, sk);
  }
}

int read_and_clear(const void* sym) {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, sym, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(sym, &z, sizeof(int)));
  }
  return v;
}

}  // namespace

int64_t f16_weight_kp(int64_t K) { return (K + 7) / 8 * 8; }

void prepare_weight_f16(const float* W, int64_t K, int64_t N, int64_t ldw, uint16_t* hi_u,
                        uint16_t* lo_u, float* scale2, cudaStream_t st, bool trans) {
  __half* hi = reinterpret_cast<__half*>(hi_u);
  __half* lo = reinterpret_cast<__half*>(lo_u);
  IDEV_CHECK_ARG(K >= 1 && N >= 1 && ldw >= (trans ? K : N), "split fp16 weight: bad shape");
  IDEV_CUDA(cudaMemsetAsync(scale2, 0, sizeof(float), st));
  unsigned int* amax = reinterpret_cast<unsigned int*>(scale2);
  const int64_t n = K * N;
  absmax_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8), 256, 0, st>>>(
      W, trans ? N : K, trans ? K : N, ldw, amax);
  IDEV_LAUNCHED();
  const int64_t kp = f16_weight_kp(K);
  dim3 grid((unsigned)((N + 31) / 32), (unsigned)((kp + 31) / 32));
  split_weight_f16_kernel<<<grid, dim3(32, 8), 0, st>>>(W, K, N, ldw, trans, kp, amax, hi, lo,
                                                        scale2 + 1);
  IDEV_LAUNCHED();
}

bool gemm_f16s_supported(const float* A, int64_t lda, int64_t M, int64_t N, int64_t K) {
  return M >= 1 && N >= 1 && K >= 1 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) &&
         aligned16(A) && lda % 4 == 0 && lda >= K;
}

void launch_gemm_f16s(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                      const float* scale2, int* range_flag, float* C, int64_t ldc,
                      const SplitOut& so, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                      cudaStream_t st, const SplitK& sk) {
  const float* inv_scale = scale2 + 1;
  if (!range_flag)  // the current device's copy of the module-wide flag
    IDEV_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&range_flag), g_f16_range));
  const bool as = A.a32 == nullptr;
  IDEV_CHECK_ARG(M >= 1 && N >= 1 && K >= 1 && M < (1LL << 31) && N < (1LL << 31) &&
                     K < (1LL << 31) && kp == f16_weight_kp(K) && aligned16(Bh) && aligned16(Bl),
                 "split fp16 GEMM: unsupported shape or weight alignment");
  if (as)
    IDEV_CHECK_ARG(A.hi && A.lo && aligned16(A.hi) && aligned16(A.lo) && A.ld % 8 == 0 &&
                       A.ld >= K,
                   "split fp16 GEMM: pre-split A needs aligned planes, ld % 8 == 0");
  else
    IDEV_CHECK_ARG(gemm_f16s_supported(A.a32, A.ld, M, N, K),
                   "split fp16 GEMM: fp32 A needs 16-byte alignment, lda % 4 == 0");
  int epi = EPI_GENERIC;
  if (ep.bias_mode == 1 && ep.act == ACT_NONE && ep.resid == nullptr) epi = EPI_BIAS;
  if (ep.bias_mode == 1 && ep.act == ACT_GELU_ERF && ep.resid == nullptr) epi = EPI_BIAS_GELU;
  if (ep.bias_mode == 1 && ep.act == ACT_NONE && ep.resid != nullptr) epi = EPI_BIAS_RESID;
  if (as && gemm_f16s_2cta_usable(A, M, N, K, so.hi != nullptr) &&
      (!so.hi || ((epi == EPI_BIAS || epi == EPI_BIAS_GELU) && N % 16 == 0 && so.lo &&
                  so.range && aligned16(so.hi) && aligned16(so.lo) && so.ld % 8 == 0 &&
                  so.ld >= N && aligned16(ep.bias)))) {
    launch_gemm_f16s_2cta(A, Bh, Bl, kp, scale2, C, ldc, so, M, N, K, epi, ep, st);
    return;
  }
  if (so.hi) {
    IDEV_CHECK_ARG(as && (epi == EPI_BIAS || epi == EPI_BIAS_GELU) && N % 16 == 0 && so.lo &&
                       so.range && aligned16(so.hi) && aligned16(so.lo) && so.ld % 8 == 0 &&
                       so.ld >= N && aligned16(ep.bias),
                   "split fp16 GEMM: split output needs pre-split A, a bias (+GELU) epilogue, "
                   "N % 16 == 0 and aligned planes");
    if (epi == EPI_BIAS)
      launch_f16s_width<EPI_BIAS, true, true>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,
                                              N, K, ep, st, sk);
    else
      launch_f16s_width<EPI_BIAS_GELU, true, true>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc,
                                                   so, M, N, K, ep, st, sk);
    return;
  }
#define IDEV_F16(EPIK)                                                                          \
  do {                                                                                          \
    if (as)                                                                                     \
      launch_f16s_width<EPIK, true, false>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M,  \
                                           N, K, ep, st, sk);                                       \
    else                                                                                        \
      launch_f16s_width<EPIK, false, false>(A, Bh, Bl, kp, inv_scale, range_flag, C, ldc, so, M, \
                                            N, K, ep, st, sk);                                      \
  } while (0)
  switch (epi) {
    case EPI_BIAS: IDEV_F16(EPI_BIAS); break;
    case EPI_BIAS_GELU: IDEV_F16(EPI_BIAS_GELU); break;
    case EPI_BIAS_RESID: IDEV_F16(EPI_BIAS_RESID); break;
    default: IDEV_F16(EPI_GENERIC); break;
  }
#undef IDEV_F16
}

void launch_gemm_f16s(const float* A, int64_t lda, const uint16_t* Bh, const uint16_t* Bl,
                      int64_t kp, const float* scale2, int* range_flag, float* C, int64_t ldc,
                      int64_t M, int64_t N, int64_t K, const Epilogue& ep, cudaStream_t st) {
  F16GemmA a;
  a.a32 = A;
  a.ld = lda;
  launch_gemm_f16s(a, Bh, Bl, kp, scale2, range_flag, C, ldc, SplitOut(), M, N, K, ep, st);
}

void launch_split_rows_f16(const float* x, int64_t rows, int64_t cols, int64_t ldx, uint16_t* hi,
                           uint16_t* lo, int64_t ld, int* range, cudaStream_t st) {
  IDEV_CHECK_ARG(rows >= 0 && cols > 0 && cols % 2 == 0 && ldx >= cols && ld >= cols &&
                     ldx % 2 == 0 && ld % 2 == 0,
                 "f16 split of rows: cols, ldx and ld must be even");
  if (rows == 0) return;
  if (!range) IDEV_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&range), g_f16_range));
  const int64_t n = rows * (cols / 2);
  split_rows_f16_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(
      x, rows, cols, ldx, hi, lo, ld, range);
  IDEV_LAUNCHED();
}

int* f16_range_flag_ptr() {
  int* p = nullptr;
  IDEV_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_f16_range));
  return p;
}

int read_and_clear_f16_error() { return read_and_clear(&g_f16_error); }
int read_and_clear_f16_range() { return read_and_clear(&g_f16_range); }

}  // namespace inferc_dev
