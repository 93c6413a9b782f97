// Split-fp16 GEMM (gemm_f16s.cu's numerics) with the 256-row tcgen05 MMA
// that two SMs execute together (cta_group::2), for A given as its fp16
// hi / lo planes.
//
// Why: the three-product split makes each 128 x 256 tile read 72 KB of
// operands from shared memory per 32-wide k-slab, next to 48 KB of TMA
// writes, which is close to the shared-memory bandwidth of an SM at full
// tensor rate. In the pair, each SM holds its own 128 rows of A and half of
// B (128 of the 256 output columns); one MMA instruction computes the
// 256 x 256 tile and each SM reads only its halves: 2/3 of the traffic.
// With the shared-memory-staged epilogues it is ahead of the one-SM kernel
// for the GEMMs that write fp16 planes and slightly behind for the fp32
// residual ones; gemm_f16s_2cta_usable picks it accordingly.
//
// A cluster of two CTAs per tile (rank 0 leads):
//   warp 0      TMA producer in both CTAs: its A rows and its B columns, both
//               planes, into its own shared memory; the completion bytes go
//               to the leader's stage barrier (cta_group::2 TMA form, no
//               multicast)
//   warp 1      TMEM allocation in both CTAs (cta_group::2, same columns on
//               both SMs); in the leader, the MMA issuer
//   warps 2..9  epilogue in both CTAs: each reads its SM's 128 accumulator
//               rows, and tells the leader when the accumulator is drained
// The leader's MMA issuer commits each stage and each accumulator twice:
// to its own barrier and to the peer CTA's (by its cluster address), so
// neither CTA waits for a forwarded signal.
// Every wait is bounded; on a timeout the CTA sets g_f16_2cta_error and leaves;
// both CTAs meet at a cluster barrier before freeing TMEM and exiting.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdlib>

#include "gemm_epi.cuh"
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace inferc_dev {

__device__ int g_f16_2cta_error;  // a barrier wait timed out

namespace {

using namespace tc;

#ifndef F16_2CTA_BK
#define F16_2CTA_BK 64
#endif
constexpr int kBK = F16_2CTA_BK;                 // fp16 k per stage
constexpr uint32_t kRowB = kBK * 2;              // bytes of one operand row per stage
constexpr uint32_t kLayout = kBK == 64 ? 2 : 4;  // UMMA SWIZZLE_128B / _64B
constexpr uint32_t kSBO = 8 * kRowB;
constexpr int kEpiThreads = 256;                 // warps 2..9
constexpr int kThreads = 64 + kEpiThreads;
constexpr uint32_t kAPlane = 128 * kBK * 2;      // 8 KB: this CTA's 128 rows

template <int BN, int STAGES>
struct Shape2 {
  static constexpr uint32_t B_PLANE = (BN / 2) * kBK * 2;  // this CTA's half of B
  static constexpr uint32_t STAGE = 2 * kAPlane + 2 * B_PLANE;
  static constexpr uint32_t SMEM = STAGES * STAGE + 1024;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// arrive (+ expected bytes) on a barrier given by its cluster address
__device__ __forceinline__ void mbar_arrive_expect_cluster(uint32_t cl_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
                   cl_addr),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr)
               : "memory");
}
// bounded wait with cluster-scope acquire (for barriers peers arrive on)
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const unsigned long long t0 = gclock_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 255 && gclock_ns() - t0 > kWaitLimitNs) return false;
  }
}
__device__ __forceinline__ void tma_load_2d_2sm(uint32_t dst, const CUtensorMap* map,
                                                uint32_t cl_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cl_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_f16_2sm(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void commit_2sm(uint32_t cl_bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cl_bar)
      : "memory");
}
__host__ __device__ constexpr uint32_t idesc_f16_kk(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

template <int BN, int STAGES, int EPI, bool SOUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_f16s_2cta_kernel(const __grid_constant__ CUtensorMap tmAh,
                          const __grid_constant__ CUtensorMap tmAl,
                          const __grid_constant__ CUtensorMap tmBh,
                          const __grid_constant__ CUtensorMap tmBl,
                          const float* __restrict__ b_inv_scale, float* __restrict__ C,
                          int64_t ldc, int M, int N, int K, Epilogue ep, SplitOut so) {
  using S = Shape2<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2], tempty_bar[2], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int ktiles = (K + kBK - 1) / kBK;
  const int tiles_n = (N + BN - 1) / BN;
  const int total = ((M + 255) / 256) * tiles_n;
  const int cl = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  auto stage_base = [&](int s) { return smem + (size_t)s * S::STAGE; };
  auto fail = [&]() {
    abort_sh = 1;
    atomicExch(&g_f16_2cta_error, 1);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 2);   // leader: one expect_tx arrive per CTA
      mbar_init(&empty_bar[s], 1);  // the leader's MMA commit (to both CTAs)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);  // the leader's MMA commit (to both CTAs)
      mbar_init(&tempty_bar[b], 2 * kEpiThreads);  // leader: both CTAs' epilogues
    }
    mbar_init(&drain_bar, 1);
    abort_sh = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // two accumulators of BN columns on both SMs
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base_sh)),
                 "r"((uint32_t)(2 * BN)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer (both CTAs)
      int g = 0;
      for (int tile = cl; tile < total && !abort_sh; tile += ncl) {
        const int m0 = (tile / tiles_n) * 256 + (int)rank * 128;
        const int n0 = (tile % tiles_n) * BN + (int)rank * (BN / 2);
        for (int it = 0; it < ktiles && !abort_sh; ++it, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (r > 0 && !mbar_wait_cl(&empty_bar[s], (r - 1) & 1)) {
            fail();
            break;
          }
          const uint32_t lead_full = map_to_rank(smem_u32(&full_bar[s]), 0);
          mbar_arrive_expect_cluster(lead_full, 2 * kAPlane + 2 * S::B_PLANE);
          const uint32_t base = smem_u32(stage_base(s));
          tma_load_2d_2sm(base, &tmAh, lead_full, it * kBK, m0);
          tma_load_2d_2sm(base + kAPlane, &tmAl, lead_full, it * kBK, m0);
          tma_load_2d_2sm(base + 2 * kAPlane, &tmBh, lead_full, it * kBK, n0);
          tma_load_2d_2sm(base + 2 * kAPlane + S::B_PLANE, &tmBl, lead_full, it * kBK, n0);
        }
      }
      // On abort the leader waits (bounded) for the ring generations it
      // issued. Both CTAs' copies complete on the leader's barriers, so this
      // also covers the peer's copies of those generations; the cluster
      // barrier below keeps the peer resident until then.
      if (abort_sh && leader) {
        for (int j = g > STAGES ? g - STAGES : 0; j < g; ++j)
          mbar_wait_cl(&full_bar[j % STAGES], (uint32_t)(j / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {  // ---------------- MMA issuer (leader)
      constexpr uint32_t idesc = idesc_f16_kk(256, BN);
      int g = 0, tl = 0;
      for (int tile = cl; tile < total && !abort_sh; tile += ncl, ++tl) {
        const int acc = tl & 1;
        if (tl >= 2 && !mbar_wait_cl(&tempty_bar[acc], ((tl >> 1) - 1) & 1)) {
          fail();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int it = 0; it < ktiles && !abort_sh; ++it, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (!mbar_wait_cl(&full_bar[s], r & 1)) {
            fail();
            break;
          }
          tc_fence_after();
          const uint32_t ah = smem_u32(stage_base(s)), al = ah + kAPlane;
          const uint32_t bh = ah + 2 * kAPlane, bl = bh + S::B_PLANE;
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {  // 16 fp16 = 32 bytes per k-step
            const uint64_t dah = smem_desc(ah + j * 32, 16, kSBO, kLayout);
            const uint64_t dal = smem_desc(al + j * 32, 16, kSBO, kLayout);
            const uint64_t dbh = smem_desc(bh + j * 32, 16, kSBO, kLayout);
            const uint64_t dbl = smem_desc(bl + j * 32, 16, kSBO, kLayout);
            mma_f16_2sm(d, dal, dbh, idesc, (it | j) != 0);
            mma_f16_2sm(d, dah, dbl, idesc, 1);
            mma_f16_2sm(d, dah, dbh, idesc, 1);
          }
          // stage s is free in both CTAs once these MMAs finish
          commit_2sm(smem_u32(&empty_bar[s]));
          commit_2sm(map_to_rank(smem_u32(&empty_bar[s]), 1));
        }
        commit_2sm(smem_u32(&tfull_bar[acc]));
        commit_2sm(map_to_rank(smem_u32(&tfull_bar[acc]), 1));
      }
      if (abort_sh) {  // every pair MMA issued so far finishes before TMEM is freed
        commit_2sm(smem_u32(&drain_bar));
        mbar_wait_cl(&drain_bar, 0);
      }
    }
  } else {  // ---------------- epilogue (warps 2..9, both CTAs)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const bool vec_ok = (ldc & 3) == 0 && aligned16(C) &&
                        (EPI != EPI_BIAS_RESID || ((ep.ldr & 3) == 0 && aligned16(ep.resid))) &&
                        (EPI == EPI_GENERIC || aligned16(ep.bias));
    const float sc = __ldg(b_inv_scale);
    const uint32_t lead_tempty0 = map_to_rank(smem_u32(&tempty_bar[0]), 0);
    const uint32_t lead_tempty1 = map_to_rank(smem_u32(&tempty_bar[1]), 0);
    bool bad = false;
    int tl = 0;
    for (int tile = cl; tile < total; tile += ncl, ++tl) {
      const int acc = tl & 1;
      if (abort_sh || !mbar_wait_cl(&tfull_bar[acc], (tl >> 1) & 1)) {
        fail();
        break;
      }
      tc_fence_after();
      const int m0 = (tile / tiles_n) * 256 + (int)rank * 128, n0 = (tile % tiles_n) * BN;
      const int64_t row = m0 + 32 * q + lane;
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN);
      // whole-tile fast paths (warp-uniform), as in gemm_f16s.cu
      const bool staged = (SOUT || vec_ok) && n0 + BN <= N;
#pragma unroll 1
      for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 16) {
        float v[16];
        tmem_ld16(base + (uint32_t)c0, v);
        if (staged && (SOUT ? (EPI == EPI_BIAS || EPI == EPI_BIAS_GELU) : EPI == EPI_BIAS_RESID)) {
          // The warp's 32 rows x 16 columns go through shared memory (rows
          // padded to 20 floats) and come back as float4s covering 8 rows x
          // 64 contiguous bytes per warp instruction: whole-sector residual
          // loads and stores. Arithmetic as in epilogue16 / epilogue16_split.
          __shared__ __align__(16) float stage[kEpiThreads / 32][32 * 20];
          float* wb = stage[warp - 2];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            reinterpret_cast<float4*>(wb + lane * 20)[j] = make_float4(
                v[4 * j] * sc, v[4 * j + 1] * sc, v[4 * j + 2] * sc, v[4 * j + 3] * sc);
          __syncwarp();
          const int c4 = (lane & 3) * 4;
          const int64_t col = (int64_t)n0 + c0 + c4;
          const float4 bb = __ldg(reinterpret_cast<const float4*>(ep.bias + col));
          float4 rr[4];
          if (!SOUT) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int64_t grow = m0 + 32 * q + (lane >> 2) + 8 * k;
              rr[k] = grow < M ? *reinterpret_cast<const float4*>(ep.resid + grow * ep.ldr + col)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int rl = (lane >> 2) + 8 * k;
            const int64_t grow = m0 + 32 * q + rl;
            if (grow >= M) continue;
            const float4 x = *reinterpret_cast<const float4*>(wb + rl * 20 + c4);
            float o[4] = {ep.alpha * x.x + ep.beta * bb.x, ep.alpha * x.y + ep.beta * bb.y,
                          ep.alpha * x.z + ep.beta * bb.z, ep.alpha * x.w + ep.beta * bb.w};
            if (SOUT) {
              if (EPI == EPI_BIAS_GELU) {
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = gelu_erf(o[i]);
              }
              uint32_t l0, l1;
              const uint32_t h0 = split_pair(o[0], o[1], l0, bad);
              const uint32_t h1 = split_pair(o[2], o[3], l1, bad);
              *reinterpret_cast<uint2*>(so.hi + grow * so.ld + col) = make_uint2(h0, h1);
              *reinterpret_cast<uint2*>(so.lo + grow * so.ld + col) = make_uint2(l0, l1);
            } else {
              o[0] += rr[k].x; o[1] += rr[k].y; o[2] += rr[k].z; o[3] += rr[k].w;
              *reinterpret_cast<float4*>(C + grow * ldc + col) = make_float4(o[0], o[1], o[2], o[3]);
            }
          }
          __syncwarp();
          continue;
        }
        if (row >= M) continue;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] *= sc;
        const int64_t col0 = (int64_t)n0 + c0;
        if (SOUT) {
          // N % 16 == 0 for split outputs: a chunk is wholly inside or outside
          if (col0 < N) epilogue16_split<EPI>(ep, v, row, col0, so, bad);
        } else {
          epilogue16<EPI>(ep, v, row, col0, N, C + row * ldc + col0, vec_ok);
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(acc ? lead_tempty1 : lead_tempty0);
    }
    if (SOUT && bad) atomicExch(so.range, 1);
  }
  tc_fence_before();
  // No MMA, TMA or remote arrive of either CTA is still pending here: on the
  // normal path every stage and accumulator was consumed; on abort the
  // leader's producer and MMA thread drained theirs above.
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)(2 * BN)));
  }
}

int sm_count_2cta() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <int BN, int STAGES, int EPI, bool SOUT>
void launch_2cta(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                 const float* inv_scale, float* C, int64_t ldc, const SplitOut& so, int64_t M,
                 int64_t N, int64_t K, const Epilogue& ep, cudaStream_t st) {
  using S = Shape2<BN, STAGES>;
  const CUtensorMapSwizzle swz = kBK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMap tah =
      make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A.hi, M, K, A.ld, kBK, 128, swz);
  const CUtensorMap tal =
      make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A.lo, M, K, A.ld, kBK, 128, swz);
  const CUtensorMap tbh = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bh, N, kp, kp, kBK,
                                      BN / 2, swz);
  const CUtensorMap tbl = make_map_2d(CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, Bl, N, kp, kp, kBK,
                                      BN / 2, swz);
  auto kern = gemm_f16s_2cta_kernel<BN, STAGES, EPI, SOUT>;
  IDEV_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::SMEM));
  // Persistent grid: as many pairs as can be resident together (clusters
  // cannot straddle GPCs, so this can be below half the SM count).
  static int resident_pairs = [&] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sm_count_2cta());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = S::SMEM;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = sm_count_2cta() / 2;
    }
    return n;
  }();
  const int64_t tiles = ((N + BN - 1) / BN) * ((M + 255) / 256);
  const int64_t pairs = std::min<int64_t>(tiles, resident_pairs);
  kern<<<(unsigned)(2 * pairs), kThreads, S::SMEM, st>>>(tah, tal, tbh, tbl, inv_scale, C, ldc,
                                                         (int)M, (int)N, (int)K, ep, so);
  IDEV_LAUNCHED();
}

}  // namespace

int read_and_clear_f16_2cta_error() {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_f16_2cta_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_f16_2cta_error, &z, sizeof(int)));
  }
  return v;
}

bool gemm_f16s_2cta_usable(const F16GemmA& A, int64_t M, int64_t N, int64_t K,
                           bool split_out) {
  // Measured on the encoder's GEMMs, with the staged epilogues: ahead of the
  // one-SM kernel where the result is written as fp16 planes (FFN1 358 vs
  // 367 us, QKV 254 vs 264 us at M = 32768); for the fp32 residual epilogue
  // ahead only with a long K at large M (FFN2, K = 3072: 356 vs 365 us at
  // M = 32768, level at 16384) and behind at K = 768 (113 vs 108 us) and at
  // small M, where the one-SM kernel's tile width follows the wave count
  // (M = 4096: 64 vs 50 us). So by default it takes the split-output GEMMs
  // and fp32-output GEMMs with K >= 2048 and M >= 32768;
  // INFERC_GEMM_2CTA=1 uses it for every eligible GEMM, =0 for none.
  static const int mode = [] {
    const char* e = std::getenv("INFERC_GEMM_2CTA");
    return e == nullptr ? -1 : (e[0] == '1' ? 1 : 0);
  }();
  if (A.a32 != nullptr || M < 512 || N < 256) return false;
  return mode == 1 || (mode == -1 && (split_out || (K >= 2048 && M >= 32768)));
}

void launch_gemm_f16s_2cta(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                           const float* scale2, float* C, int64_t ldc, const SplitOut& so,
                           int64_t M, int64_t N, int64_t K, int epi, const Epilogue& ep,
                           cudaStream_t st) {
  const float* inv = scale2 + 1;
  constexpr int BN = 256, ST = kBK == 64 ? 3 : 6;
  if (so.hi) {
    if (epi == EPI_BIAS)
      launch_2cta<BN, ST, EPI_BIAS, true>(A, Bh, Bl, kp, inv, C, ldc, so, M, N, K, ep, st);
    else
      launch_2cta<BN, ST, EPI_BIAS_GELU, true>(A, Bh, Bl, kp, inv, C, ldc, so, M, N, K, ep, st);
    return;
  }
  switch (epi) {
    case EPI_BIAS:
      launch_2cta<BN, ST, EPI_BIAS, false>(A, Bh, Bl, kp, inv, C, ldc, so, M, N, K, ep, st);
      break;
    case EPI_BIAS_GELU:
      launch_2cta<BN, ST, EPI_BIAS_GELU, false>(A, Bh, Bl, kp, inv, C, ldc, so, M, N, K, ep, st);
      break;
    case EPI_BIAS_RESID:
      launch_2cta<BN, ST, EPI_BIAS_RESID, false>(A, Bh, Bl, kp, inv, C, ldc, so, M, N, K, ep, st);
      break;
    default:
      launch_2cta<BN, ST, EPI_GENERIC, false>(A, Bh, Bl, kp, inv, C, ldc, so, M, N, K, ep, st);
      break;
  }
}

}  // namespace inferc_dev
