// FusedAttention (head_dim 64, S <= 4096) on the fp16 tensor cores with
// fp32-level accuracy, for q, k and v given as the split-fp16 planes the
// QKV GEMM writes (x = hi + lo, gemm_f16s.cu's representation).
//
// S <= 128: persistent CTAs, two per SM, each walking (batch, head) items:
//   * no split step: TMA loads the six hi / lo head tiles (96 KB) directly;
//   * S = Q K^T and O = P V each take three kind::f16 MMAs per product
//     (lo hi + hi lo + hi hi), at twice the tf32 rate;
//   * P is written as fp16 hi / lo (P in [0, 1]: elements below 2^-14 keep
//     an absolute error under 2^-25) into tensor memory over S, and the PV
//     MMAs read it from there, so the Q / K tiles are free as soon as S is
//     done and the next item's loads run under this item's softmax;
//   * the mask is staged as one row (a mask that broadcasts over query rows,
//     the padding mask of the encoder) or read per row from global memory.
// That is ~98 KB of shared memory and 256 TMEM columns per CTA.
//
// Steps per item: TMA -> S = QK^T (M=128 queries, N=128 keys, K=64) -> masked
// softmax (two threads per row, 64 keys each in registers; masked entries
// are REPLACED by `fill`, keys past S get no weight, as rt::FusedAttention,
// src/kernels/attention.cc:77-91) -> P hi / lo into TMEM -> O = P V (V
// MN-major, SWIZZLE_128B) -> O as fp32 or as fp16 planes.
// Every mbarrier wait is bounded; a timeout sets g_attn_f16_error. Only warp
// 0 polls a barrier; the other warps wait at the CTA barrier that follows,
// which takes no issue slots from the other CTA on the SM.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdlib>

#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace inferc_dev {

__device__ int g_attn_f16_error;

namespace {

using namespace tc;

constexpr int kRows = 128;
constexpr int kHd = 64;
constexpr int kThreads = 256;
constexpr uint32_t kTile = 16384;  // [128 rows][128 B]: one fp16 plane of a head tile
// Q hi, Q lo, K hi, K lo, V hi, V lo (P lives in tensor memory).
constexpr uint32_t OFF_QH = 0, OFF_QL = kTile, OFF_KH = 2 * kTile, OFF_KL = 3 * kTile,
                   OFF_VH = 4 * kTile, OFF_VL = 5 * kTile;
constexpr uint32_t OFF_MASK = 6 * kTile;  // one row of kRows bytes
constexpr uint32_t kSmemBytes = 6 * kTile + kRows + 1024;

struct AttnF16Kern {
  const uint8_t* mask;
  int64_t ms[4];
  int S;
  float scale, fill;
  float* out;
  int64_t ldo, bstride_o;
  SplitOut so;
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// Bulk tensor store shared -> global (coordinates start at 0 or above; the
// map clips rows outside the tensor), tracked by the bulk async-group.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// the committed stores have read their shared-memory source
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// the committed stores are complete
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
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

// kind::f16 descriptors: f32 D, f16 A and B; A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool b_mn) {
  return (1u << 4) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// PV with A = P read from tensor memory: 128 lanes = query rows, each 32-bit
// column two consecutive keys (the lower half the even key).
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// split_pair for values known to lie in [0, 1] (no range check): fp16 hi of
// (a, b) packed, the fp16 of the remainders in lo_bits.
__device__ __forceinline__ uint32_t split_unit_pair(float a, float b, uint32_t& lo_bits) {
  uint32_t h, l;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
  const float ha = __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
  const float hb = __half2float(__ushort_as_half((unsigned short)(h >> 16)));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(l) : "f"(b - hb), "f"(a - ha));
  lo_bits = l;
  return h;
}

// 32 consecutive 32-bit columns of this warp's 32 lanes, no wait: the
// caller issues tcgen05.wait::ld once for a batch of loads.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// Persistent: CTA c takes the (batch, head) items c, c + grid, c + 2 grid, ...
// (item = b * nH + h). Per item:
//   S = QK^T (TMEM cols 0..127) -> the next item's Q / K load is issued at once
//   (their tiles are free) -> masked softmax in registers, P written over S as
//   fp16 hi (cols 0..63) / lo (cols 64..127) -> O = P V with A read from TMEM
//   (cols 128..191) -> the next item's V load and S = QK^T are issued -> the
//   epilogue of this item overlaps both.
// So a CTA's loads run under its own softmax and epilogue, and two CTAs per SM
// overlap each other's compute phases.
__global__ void __launch_bounds__(kThreads, 2)
    attention_f16_kernel(const __grid_constant__ CUtensorMap tQh,
                         const __grid_constant__ CUtensorMap tQl,
                         const __grid_constant__ CUtensorMap tKh,
                         const __grid_constant__ CUtensorMap tKl,
                         const __grid_constant__ CUtensorMap tVh,
                         const __grid_constant__ CUtensorMap tVl,
                         const __grid_constant__ CUtensorMap tOh,
                         const __grid_constant__ CUtensorMap tOl, const AttnF16Kern a,
                         int n_items, int nH) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar_qk, bar_v, bar_s, bar_o, bar_drain;
  __shared__ uint32_t tmem_sh;
  __shared__ int fail0;
  __shared__ float red_max[2][kRows], red_sum[2][kRows];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + (tid & 31), col0 = 64 * half;
  const uint32_t lane_base = (uint32_t)(32 * quad) << 16;

  if (tid == 0) {
    mbar_init(&bar_qk, 1);
    mbar_init(&bar_v, 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    mbar_init(&bar_drain, 1);
    fail0 = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // S / P: columns 0..127, O: 128..191
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
        smem_u32(&tmem_sh)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  // Dependents may launch once every CTA holds its TMEM (none can take TMEM
  // this grid still needs); q/k/v come from the previous kernel.
  pdl_launch_dependents();
  pdl_wait();

  // Copies and MMAs are issued by thread 0 only; it counts what it issued
  // and what it saw complete, so that the abort path can wait for the rest.
  uint32_t qk_issued = 0, qk_seen = 0, v_issued = 0, v_seen = 0;
  auto issue_qk = [&](int it) {
    const int b = it / nH, h = it - (it / nH) * nH;
    mbar_expect_tx(&bar_qk, 4 * kTile);
    tma_load_4d(sm + OFF_QH, &tQh, &bar_qk, 0, h, 0, b);
    tma_load_4d(sm + OFF_QL, &tQl, &bar_qk, 0, h, 0, b);
    tma_load_4d(sm + OFF_KH, &tKh, &bar_qk, 0, h, 0, b);
    tma_load_4d(sm + OFF_KL, &tKl, &bar_qk, 0, h, 0, b);
    ++qk_issued;
  };
  auto issue_v = [&](int it) {
    const int b = it / nH, h = it - (it / nH) * nH;
    mbar_expect_tx(&bar_v, 2 * kTile);
    tma_load_4d(sm + OFF_VH, &tVh, &bar_v, 0, h, 0, b);
    tma_load_4d(sm + OFF_VL, &tVl, &bar_v, 0, h, 0, b);
    ++v_issued;
  };
  auto issue_s = [&]() {  // S = Q K^T into columns 0..127
    tc_fence_after();
    constexpr uint32_t idesc = idesc_f16(kRows, kRows, false);
    const uint32_t qh = smem_u32(sm + OFF_QH), ql = smem_u32(sm + OFF_QL);
    const uint32_t kh = smem_u32(sm + OFF_KH), kl = smem_u32(sm + OFF_KL);
#pragma unroll
    for (int j = 0; j < kHd / 16; ++j) {  // 16 fp16 = 32 bytes per k-step
      const uint64_t dqh = smem_desc(qh + j * 32, 16, 1024, 2), dql = smem_desc(ql + j * 32, 16, 1024, 2);
      const uint64_t dkh = smem_desc(kh + j * 32, 16, 1024, 2), dkl = smem_desc(kl + j * 32, 16, 1024, 2);
      mma_f16(tmem, dql, dkh, idesc, j != 0);
      mma_f16(tmem, dqh, dkl, idesc, 1);
      mma_f16(tmem, dqh, dkh, idesc, 1);
    }
    mma_commit(&bar_s);
  };

  const bool mask_bcast = a.mask && a.ms[2] == 0;
  uint8_t* mrow_s = sm + OFF_MASK;
  bool ok = true;
  if (tid == 0 && (int)blockIdx.x < n_items) {
    issue_qk(blockIdx.x);
    issue_v(blockIdx.x);
  }
  // A mask that broadcasts over query rows is staged once per item (one row
  // of kRows bytes, thread j < kRows holds byte j). The next item's bytes are
  // loaded into a register during this item, so no load latency sits between
  // two items.
  auto mask_byte = [&](int itm) -> uint32_t {
    if (!mask_bcast || tid >= kRows || tid >= a.S || itm >= n_items) return 0u;
    const int bb = itm / nH, hh = itm - (itm / nH) * nH;
    return a.mask[(int64_t)bb * a.ms[0] + (int64_t)hh * a.ms[1] + (int64_t)tid * a.ms[3]];
  };
  uint32_t mval = mask_byte(blockIdx.x);
  uint32_t k = 0;  // this CTA's item count
  for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++k) {
    const int b = it / nH, h = it - (it / nH) * nH;
    const int next = it + (int)gridDim.x;
    const uint32_t par = k & 1u;
    // the previous item's readers of the row are past a CTA barrier
    if (mask_bcast && tid < kRows) mrow_s[tid] = (uint8_t)mval;
    if (k == 0) {
      ok = __syncthreads_and(warp != 0 || (mbar_wait(&bar_qk, 0))) != 0;
      if (!ok) break;
      if (tid == 0) {
        ++qk_seen;
        issue_s();
      }
    }
    // S(it) landed: Q / K tiles are free for the next item
    ok = __syncthreads_and(warp != 0 || (fail0 == 0 && mbar_wait(&bar_s, par))) != 0;
    if (!ok) break;
    if (tid == 0 && next < n_items) issue_qk(next);
    mval = mask_byte(next);
    tc_fence_after();
    float s[64];
    {
      float (&s0)[32] = *reinterpret_cast<float(*)[32]>(&s[0]);
      float (&s1)[32] = *reinterpret_cast<float(*)[32]>(&s[32]);
      tmem_ld32_async(tmem + lane_base + (uint32_t)col0, s0);
      tmem_ld32_async(tmem + lane_base + (uint32_t)(col0 + 32), s1);
      tmem_wait_ld();
    }
    const uint8_t* mrow_g =
        (a.mask && !mask_bcast && row < a.S)
            ? a.mask + (int64_t)b * a.ms[0] + (int64_t)h * a.ms[1] + (int64_t)row * a.ms[2]
            : nullptr;
    // scores in the log2 domain: v = scale * s * log2(e); a masked entry is
    // REPLACED by fill (clamped at -1e30, which gives the same weights: 0
    // next to any visible key, uniform in a fully masked row); keys past S
    // get -inf (no weight at all).
    const int nvalid = a.S - col0;  // keys of this thread's half that exist
    const float sc2 = a.scale * kLog2e;
    const float fill2 = fmaxf(a.fill, -1.0e30f) * kLog2e;
    float mx = -INFINITY;
    if (mask_bcast) {
      uint4 mw[4];  // this half's 64 mask bytes
#pragma unroll
      for (int i = 0; i < 4; ++i) mw[i] = reinterpret_cast<const uint4*>(mrow_s + col0)[i];
#pragma unroll
      for (int q = 0; q < 64; ++q) {
        const uint4 w4 = mw[q >> 4];
        const uint32_t w = (q & 15) < 4 ? w4.x : (q & 15) < 8 ? w4.y : (q & 15) < 12 ? w4.z : w4.w;
        const bool masked = (w & (0xffu << (8 * (q & 3)))) != 0u;
        s[q] = masked ? fill2 : sc2 * s[q];
      }
    } else {
#pragma unroll
      for (int q = 0; q < 64; ++q) {
        const bool masked = mrow_g && q < nvalid && mrow_g[(int64_t)(col0 + q) * a.ms[3]] != 0;
        s[q] = masked ? fill2 : sc2 * s[q];
      }
    }
    if (nvalid >= 64) {
#pragma unroll
      for (int q = 0; q < 64; ++q) mx = fmaxf(mx, s[q]);
    } else {
#pragma unroll
      for (int q = 0; q < 64; ++q) {
        if (q >= nvalid) s[q] = -INFINITY;
        mx = fmaxf(mx, s[q]);
      }
    }
    red_max[half][row] = mx;
    // every thread's S reads are complete (tcgen05.wait::ld) before this
    // barrier, so P may overwrite the S columns after it
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    mx = fmaxf(red_max[0][row], red_max[1][row]);
    // P = exp(v - max) = 2^(v2 - max2) on the SFU (ex2.approx, relative error
    // ~2^-22, below the fp16 hi / lo split's resolution), left unnormalised
    // (in [0, 1]); the epilogue divides O by the row sum.
    // P hi: keys 2c, 2c + 1 -> column c (this thread's keys: columns
    // 32 half .. 32 half + 31); P lo at 64 + the same column.
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t hw[16], lw[16];
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        const float e0 = ex2_approx(s[32 * c + 2 * p] - mx);
        const float e1 = ex2_approx(s[32 * c + 2 * p + 1] - mx);
        sum += e0 + e1;
        hw[p] = split_unit_pair(e0, e1, lw[p]);
      }
      tmem_st16(tmem + lane_base + (uint32_t)(32 * half + 16 * c), hw);
      tmem_st16(tmem + lane_base + (uint32_t)(64 + 32 * half + 16 * c), lw);
    }
    red_sum[half][row] = sum;
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    tc_fence_before();
    ok = __syncthreads_and(warp != 0 || (mbar_wait(&bar_v, par))) != 0;
    if (!ok) break;
    if (tid == 0) {
      ++v_seen;
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16(kRows, kHd, true);
      const uint32_t vh = smem_u32(sm + OFF_VH), vl = smem_u32(sm + OFF_VL);
#pragma unroll
      for (int j = 0; j < kRows / 16; ++j) {  // 16 keys (8 P columns) per k-step
        // V: MN-major SWIZZLE_128B, rows of 64 d (128 B), 8-key groups 1 KiB
        // apart; a 16-key step advances 2 KiB. N = 64 is one atom wide.
        const uint64_t dvh = smem_desc(vh + j * 2048, 8192, 1024, 2);
        const uint64_t dvl = smem_desc(vl + j * 2048, 8192, 1024, 2);
        const uint32_t ph = tmem + (uint32_t)(8 * j), pl = tmem + (uint32_t)(64 + 8 * j);
        mma_f16_ta(tmem + kRows, pl, dvh, idesc, j != 0);
        mma_f16_ta(tmem + kRows, ph, dvl, idesc, 1);
        mma_f16_ta(tmem + kRows, ph, dvh, idesc, 1);
      }
      mma_commit(&bar_o);
    }
    ok = __syncthreads_and(warp != 0 || (mbar_wait(&bar_o, par))) != 0;
    if (!ok) break;
    // P and V consumed: the next item's S = QK^T runs under this item's
    // epilogue (S writes columns 0..127, the epilogue reads 128..191).
    if (tid == 0 && next < n_items) {
      if (mbar_wait(&bar_qk, (k + 1) & 1u)) {
        ++qk_seen;
        issue_s();
      } else {
        fail0 = 1;
      }
    }
    tc_fence_after();
    const float inv = 1.0f / (red_sum[0][row] + red_sum[1][row]);
    bool bad = false;
    float ov[32];
    tmem_ld32_async(tmem + lane_base + kRows + (uint32_t)(32 * half), ov);
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 32; ++q) ov[q] *= inv;
    // O is staged in the spent V tiles in the output map's layout ([128 rows]
    // [128 B], 16-byte chunk c of row r at c ^ (r & 7)) and written by bulk
    // tensor stores: whole 128-byte row segments instead of one 16-byte
    // piece per thread and row. Rows past S are clipped by the map.
    const uint32_t swz = (uint32_t)(row & 7);
    if (a.so.hi) {
      // planes: hi tile at OFF_VH, lo at OFF_VL; this thread's 32 columns are
      // chunks 4 half .. 4 half + 3
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) hw[q] = split_pair(ov[8 * c + 2 * q], ov[8 * c + 2 * q + 1], lw[q], bad);
        const uint32_t off = (uint32_t)row * 128 + (((uint32_t)(4 * half + c) ^ swz) << 4);
        *reinterpret_cast<uint4*>(sm + OFF_VH + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(sm + OFF_VL + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    } else {
      // fp32: columns 32 half .. 32 half + 31 are box `half` (128 B per row)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t off = (uint32_t)half * kTile + (uint32_t)row * 128 + (((uint32_t)c ^ swz) << 4);
        *reinterpret_cast<float4*>(sm + OFF_VH + off) =
            make_float4(ov[4 * c], ov[4 * c + 1], ov[4 * c + 2], ov[4 * c + 3]);
      }
    }
    if (bad) atomicExch(a.so.range, 1);
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      if (a.so.hi) {
        tma_store_4d(&tOh, sm + OFF_VH, 0, h, 0, b);
        tma_store_4d(&tOl, sm + OFF_VL, 0, h, 0, b);
      } else {
        tma_store_3d(&tOh, sm + OFF_VH, 64 * h, 0, b);
        tma_store_3d(&tOh, sm + OFF_VH + kTile, 64 * h + 32, 0, b);
      }
      bulk_commit();
      bulk_wait_read();  // the V tiles may be overwritten once the stores read them
      if (next < n_items) issue_v(next);
    }
    // O reads complete before the next item's PV may write O
    tc_fence_before();
  }
  if (!ok && tid == 0) atomicExch(&g_attn_f16_error, 1);
  if (tid == 0) {
    bulk_wait_all();  // this CTA's output stores are complete
    // Abort path: wait (bounded) for copies still landing in this CTA's
    // shared memory and for every MMA this thread issued. On the normal path
    // every copy was seen and the last MMA's commit was waited on.
    for (; qk_seen < qk_issued; ++qk_seen) mbar_wait(&bar_qk, qk_seen & 1u);
    for (; v_seen < v_issued; ++v_seen) mbar_wait(&bar_v, v_seen & 1u);
    if (!ok) drain_mma(&bar_drain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
  }
}


// ---------------------------------------------------------------- S > 128
// Flash form: CTA (q-block, head, batch) holds its 128 query rows and loops
// over 128-key blocks with an online softmax. Per block: S_blk = Q K_blk^T
// (TMEM columns 0..127), running row max m and sum l are updated (two
// threads per row, 64 keys each, in the log2 domain), P_blk = 2^(s - m) (in
// (0, 1], fp16 hi / lo) is written over S_blk in TMEM, O_blk = P_blk V_blk
// (TMEM columns 128..191, A read from TMEM) is merged into the registers:
// O = O c + O_blk with c = 2^(m_old - m). O / l is stored at the end.
// The next block's K load is issued as soon as S_blk is done (K free), its V
// load and S = QK^T as soon as O_blk is done, so copies and MMAs run under
// the softmax and the merge.
// Shared memory: Q 32 KB, K 32 KB, V 32 KB, one mask row (one CTA per SM).
constexpr uint32_t FL_Q = 0, FL_K = 2 * kTile, FL_V = 4 * kTile;
constexpr uint32_t FL_MASK = 6 * kTile;  // one mask row, up to kFlashMaxS bytes
constexpr int kFlashMaxS = 4096;
constexpr uint32_t kFlashSmem = 6 * kTile + kFlashMaxS + 1024;

__global__ void __launch_bounds__(kThreads, 2)
    attention_f16_flash_kernel(const __grid_constant__ CUtensorMap tQh,
                               const __grid_constant__ CUtensorMap tQl,
                               const __grid_constant__ CUtensorMap tKh,
                               const __grid_constant__ CUtensorMap tKl,
                               const __grid_constant__ CUtensorMap tVh,
                               const __grid_constant__ CUtensorMap tVl,
                               const __grid_constant__ CUtensorMap tOh,
                               const __grid_constant__ CUtensorMap tOl, const AttnF16Kern a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar_q, bar_k, bar_v, bar_s, bar_o, bar_drain;
  __shared__ uint32_t tmem_sh;
  __shared__ int fail0;
  __shared__ float red_max[2][kRows], red_sum[2][kRows];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int quad = warp & 3, half = warp >> 2;
  const int lrow = quad * 32 + (tid & 31), col0 = 64 * half;
  const int row = qb * kRows + lrow;  // query row in the sequence
  const uint32_t lane_base = (uint32_t)(32 * quad) << 16;
  const int nkb = (a.S + kRows - 1) / kRows;

  if (tid == 0) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_k, 1);
    mbar_init(&bar_v, 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    mbar_init(&bar_drain, 1);
    fail0 = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
        smem_u32(&tmem_sh)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  // Copies and MMAs are issued by thread 0 only; it counts what it issued
  // and what it saw complete, so that the abort path can wait for the rest.
  uint32_t q_issued = 0, q_seen = 0, k_issued = 0, k_seen = 0, v_issued = 0, v_seen = 0;
  auto load_k = [&](int kb) {
    mbar_expect_tx(&bar_k, 2 * kTile);
    tma_load_4d(sm + FL_K, &tKh, &bar_k, 0, h, kb * kRows, b);
    tma_load_4d(sm + FL_K + kTile, &tKl, &bar_k, 0, h, kb * kRows, b);
    ++k_issued;
  };
  auto load_v = [&](int kb) {
    mbar_expect_tx(&bar_v, 2 * kTile);
    tma_load_4d(sm + FL_V, &tVh, &bar_v, 0, h, kb * kRows, b);
    tma_load_4d(sm + FL_V + kTile, &tVl, &bar_v, 0, h, kb * kRows, b);
    ++v_issued;
  };
  auto issue_s = [&]() {  // S_blk = Q K_blk^T into columns 0..127
    tc_fence_after();
    constexpr uint32_t idesc = idesc_f16(kRows, kRows, false);
    const uint32_t qh = smem_u32(sm + FL_Q), ql = qh + kTile;
    const uint32_t kh = smem_u32(sm + FL_K), kl = kh + kTile;
#pragma unroll
    for (int j = 0; j < kHd / 16; ++j) {
      const uint64_t dqh = smem_desc(qh + j * 32, 16, 1024, 2), dql = smem_desc(ql + j * 32, 16, 1024, 2);
      const uint64_t dkh = smem_desc(kh + j * 32, 16, 1024, 2), dkl = smem_desc(kl + j * 32, 16, 1024, 2);
      mma_f16(tmem, dql, dkh, idesc, j != 0);
      mma_f16(tmem, dqh, dkl, idesc, 1);
      mma_f16(tmem, dqh, dkh, idesc, 1);
    }
    mma_commit(&bar_s);
  };
  if (tid == 0) {
    mbar_expect_tx(&bar_q, 2 * kTile);
    tma_load_4d(sm + FL_Q, &tQh, &bar_q, 0, h, qb * kRows, b);
    tma_load_4d(sm + FL_Q + kTile, &tQl, &bar_q, 0, h, qb * kRows, b);
    ++q_issued;
  }
  const bool mask_bcast = a.mask && a.ms[2] == 0;
  uint8_t* mrow_s = sm + FL_MASK;
  if (mask_bcast) {
    const uint8_t* mb = a.mask + (int64_t)b * a.ms[0] + (int64_t)h * a.ms[1];
    for (int j = tid; j < a.S; j += kThreads) mrow_s[j] = mb[(int64_t)j * a.ms[3]];
  }
  // Key blocks to visit. With a per-key mask and a fill so negative that
  // exp(fill - m) is exactly 0 in fp32, a block whose keys are all masked
  // adds exact zeros to the row sums and leaves the running maximum of any
  // row with a visible key unchanged, so skipping it gives the same bits. A
  // sequence with no visible key keeps every block (the reference then
  // weighs all keys equally).
  uint32_t live = nkb >= 32 ? 0xffffffffu : (1u << nkb) - 1u;
  if (mask_bcast && a.fill <= -1.0e30f) {
    __syncthreads();
    uint32_t lv = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      bool vis = false;
      for (int j = kb * kRows + tid; j < min(a.S, (kb + 1) * kRows); j += kThreads)
        vis |= mrow_s[j] == 0;
      if (__syncthreads_or(vis)) lv |= 1u << kb;
    }
    if (lv) live = lv;
  }
  auto next_live = [&](int kb) {  // first live block after kb (nkb when none)
    const uint32_t rest = kb + 1 >= 32 ? 0u : live >> (kb + 1);
    return rest ? kb + 1 + __ffs(rest) - 1 : nkb;
  };
  const int kb_first = next_live(-1);
  if (tid == 0) {
    load_k(kb_first);
    load_v(kb_first);
  }
  const uint8_t* mrow_g =
      (a.mask && !mask_bcast && row < a.S)
          ? a.mask + (int64_t)b * a.ms[0] + (int64_t)h * a.ms[1] + (int64_t)row * a.ms[2]
          : nullptr;
  bool ok = __syncthreads_and(warp != 0 || (mbar_wait(&bar_q, 0) && mbar_wait(&bar_k, 0))) != 0;
  if (ok && tid == 0) {
    ++q_seen;
    ++k_seen;
    issue_s();
  }
  const float sc2 = a.scale * kLog2e;
  const float fill2 = fmaxf(a.fill, -1.0e30f) * kLog2e;
  float m_run = -INFINITY, l_run = 0.f;
  float o_acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o_acc[i] = 0.f;
  for (int kb = kb_first, it = 0; kb < nkb && ok; ++it) {
    const int nxt = next_live(kb);
    const uint32_t par = (uint32_t)it & 1u;
    ok = __syncthreads_and(warp != 0 || (fail0 == 0 && mbar_wait(&bar_s, par))) != 0;
    if (!ok) break;
    if (tid == 0 && nxt < nkb) load_k(nxt);  // K_blk consumed
    tc_fence_after();
    float s[64];
    {
      float (&s0)[32] = *reinterpret_cast<float(*)[32]>(&s[0]);
      float (&s1)[32] = *reinterpret_cast<float(*)[32]>(&s[32]);
      tmem_ld32_async(tmem + lane_base + (uint32_t)col0, s0);
      tmem_ld32_async(tmem + lane_base + (uint32_t)(col0 + 32), s1);
      tmem_wait_ld();
    }
    // log2-domain scores, as in the S <= 128 kernel: masked -> fill
    // (clamped at -1e30), keys past S -> -inf
    const int nvalid = a.S - kb * kRows - col0;
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      bool masked = false;
      if (q < nvalid) {
        if (mask_bcast) masked = mrow_s[kb * kRows + col0 + q] != 0;
        else if (mrow_g) masked = mrow_g[(int64_t)(kb * kRows + col0 + q) * a.ms[3]] != 0;
      }
      float v = masked ? fill2 : sc2 * s[q];
      if (q >= nvalid) v = -INFINITY;
      s[q] = v;
      mx = fmaxf(mx, v);
    }
    red_max[half][lrow] = mx;
    // every thread's S reads are complete before this barrier, so P may
    // overwrite the S columns after it
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const float m_new = fmaxf(m_run, fmaxf(red_max[0][lrow], red_max[1][lrow]));
    const float corr = ex2_approx(m_run - m_new);  // 0 on the first block (m_run = -inf)
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t hw[16], lw[16];
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        const float e0 = ex2_approx(s[32 * c + 2 * p] - m_new);
        const float e1 = ex2_approx(s[32 * c + 2 * p + 1] - m_new);
        sum += e0 + e1;
        hw[p] = split_unit_pair(e0, e1, lw[p]);
      }
      tmem_st16(tmem + lane_base + (uint32_t)(32 * half + 16 * c), hw);
      tmem_st16(tmem + lane_base + (uint32_t)(64 + 32 * half + 16 * c), lw);
    }
    red_sum[half][lrow] = sum;
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    tc_fence_before();
    ok = __syncthreads_and(warp != 0 || (mbar_wait(&bar_v, par))) != 0;
    if (!ok) break;
    l_run = l_run * corr + red_sum[0][lrow] + red_sum[1][lrow];
    m_run = m_new;
    if (tid == 0) {  // O_blk = P_blk V_blk
      ++v_seen;
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16(kRows, kHd, true);
      const uint32_t vh = smem_u32(sm + FL_V), vl = vh + kTile;
#pragma unroll
      for (int j = 0; j < kRows / 16; ++j) {
        const uint64_t dvh = smem_desc(vh + j * 2048, 8192, 1024, 2);
        const uint64_t dvl = smem_desc(vl + j * 2048, 8192, 1024, 2);
        const uint32_t ph = tmem + (uint32_t)(8 * j), pl = tmem + (uint32_t)(64 + 8 * j);
        mma_f16_ta(tmem + kRows, pl, dvh, idesc, j != 0);
        mma_f16_ta(tmem + kRows, ph, dvl, idesc, 1);
        mma_f16_ta(tmem + kRows, ph, dvh, idesc, 1);
      }
      mma_commit(&bar_o);
    }
    ok = __syncthreads_and(warp != 0 || (mbar_wait(&bar_o, par))) != 0;
    if (!ok) break;
    // P_blk and V_blk consumed: the next block's V load and S run under the merge
    if (tid == 0 && nxt < nkb) {
      load_v(nxt);
      if (mbar_wait(&bar_k, k_seen & 1u)) {
        ++k_seen;
        issue_s();
      } else {
        fail0 = 1;
      }
    }
    tc_fence_after();
    {
      float ov[32];
      tmem_ld32_async(tmem + lane_base + kRows + (uint32_t)(32 * half), ov);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 32; ++q) o_acc[q] = o_acc[q] * corr + ov[q];
    }
    // O_blk reads complete before the next block's PV may write it
    tc_fence_before();
    kb = nxt;
  }
  if (ok) {
    // O / l staged in the spent V tiles and written by bulk tensor stores, as
    // in the S <= 128 kernel (rows past S are clipped by the map)
    const float inv = 1.0f / l_run;
    const uint32_t swz = (uint32_t)(lrow & 7);
    bool bad = false;
#pragma unroll
    for (int q = 0; q < 32; ++q) o_acc[q] *= inv;
    if (a.so.hi) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          hw[q] = split_pair(o_acc[8 * c + 2 * q], o_acc[8 * c + 2 * q + 1], lw[q], bad);
        const uint32_t off = (uint32_t)lrow * 128 + (((uint32_t)(4 * half + c) ^ swz) << 4);
        *reinterpret_cast<uint4*>(sm + FL_V + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(sm + FL_V + kTile + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t off = (uint32_t)half * kTile + (uint32_t)lrow * 128 + (((uint32_t)c ^ swz) << 4);
        *reinterpret_cast<float4*>(sm + FL_V + off) =
            make_float4(o_acc[4 * c], o_acc[4 * c + 1], o_acc[4 * c + 2], o_acc[4 * c + 3]);
      }
    }
    if (bad) atomicExch(a.so.range, 1);
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      if (a.so.hi) {
        tma_store_4d(&tOh, sm + FL_V, 0, h, qb * kRows, b);
        tma_store_4d(&tOl, sm + FL_V + kTile, 0, h, qb * kRows, b);
      } else {
        tma_store_3d(&tOh, sm + FL_V, 64 * h, qb * kRows, b);
        tma_store_3d(&tOh, sm + FL_V + kTile, 64 * h + 32, qb * kRows, b);
      }
      bulk_commit();
      bulk_wait_all();
    }
  } else if (tid == 0) {
    atomicExch(&g_attn_f16_error, 1);
  }
  if (tid == 0) {
    // Abort path: wait (bounded) for copies still landing in this CTA's
    // shared memory and for every MMA this thread issued.
    for (; q_seen < q_issued; ++q_seen) mbar_wait(&bar_q, 0);
    for (; k_seen < k_issued; ++k_seen) mbar_wait(&bar_k, k_seen & 1u);
    for (; v_seen < v_issued; ++v_seen) mbar_wait(&bar_v, v_seen & 1u);
    if (!ok) drain_mma(&bar_drain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
  }
}

// 4-D map over one fp16 plane of Q, K or V inside a [B, S, ld] tensor:
// dims (d: 64, head: nH, s: S, b: B), box (64, 1, 128, 1), 128-byte swizzle.
CUtensorMap plane_map(const uint16_t* base, int nH, int S, int B, int64_t ld, int64_t bstride) {
  CUtensorMap m;
  const cuuint64_t dims[4] = {(cuuint64_t)kHd, (cuuint64_t)nH, (cuuint64_t)S, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)kHd * 2, (cuuint64_t)ld * 2, (cuuint64_t)bstride * 2};
  const cuuint32_t box[4] = {(cuuint32_t)kHd, 1, (cuuint32_t)kRows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                                 const_cast<uint16_t*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(INFERC_ERR_CUDA, "cuTensorMapEncodeTiled (fp16 attention) failed (" +
                                     std::to_string((int)r) + ")");
  return m;
}

// 3-D map over an fp32 [B, S, ldo] output: dims (column: nH * 64, s: S,
// b: B), box (32, 128, 1) = 128-byte rows, 128-byte swizzle.
CUtensorMap out_f32_map(float* base, int nH, int S, int B, int64_t ldo, int64_t bstride) {
  CUtensorMap m;
  const cuuint64_t dims[3] = {(cuuint64_t)nH * kHd, (cuuint64_t)S, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)ldo * 4, (cuuint64_t)bstride * 4};
  const cuuint32_t box[3] = {32, (cuuint32_t)kRows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_NONE,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(INFERC_ERR_CUDA, "cuTensorMapEncodeTiled (attention output) failed (" +
                                     std::to_string((int)r) + ")");
  return m;
}

}  // namespace

int read_and_clear_attn_f16_error() {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_attn_f16_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_attn_f16_error, &z, sizeof(int)));
  }
  return v;
}

bool attention_f16_supported(const AttnF16Args& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool planes = al(a.qh) && al(a.ql) && al(a.kh) && al(a.kl) && al(a.vh) && al(a.vl);
  const bool out_ok = a.so.hi ? (al(a.so.hi) && al(a.so.lo) && a.so.range != nullptr &&
                                 a.bstride_o % 8 == 0)
                              : (al(a.out) && a.ldo % 4 == 0 && a.bstride_o % 4 == 0);
  return a.S >= 1 && a.S <= kFlashMaxS && planes && out_ok && a.ld % 8 == 0 && a.bstride % 8 == 0 &&
         a.ld >= a.nH * kHd && a.bstride >= a.S * a.ld && a.ldo % 8 == 0 && a.B < 65536 &&
         a.nH < 65536;
}

void launch_attention_f16(const AttnF16Args& a, cudaStream_t st) {
  IDEV_CHECK_ARG(attention_f16_supported(a), "fp16 attention: unsupported shape or alignment");
  const int nH = (int)a.nH, S = (int)a.S, B = (int)a.B;
  const CUtensorMap tqh = plane_map(a.qh, nH, S, B, a.ld, a.bstride);
  const CUtensorMap tql = plane_map(a.ql, nH, S, B, a.ld, a.bstride);
  const CUtensorMap tkh = plane_map(a.kh, nH, S, B, a.ld, a.bstride);
  const CUtensorMap tkl = plane_map(a.kl, nH, S, B, a.ld, a.bstride);
  const CUtensorMap tvh = plane_map(a.vh, nH, S, B, a.ld, a.bstride);
  const CUtensorMap tvl = plane_map(a.vl, nH, S, B, a.ld, a.bstride);
  AttnF16Kern k{};
  k.mask = a.mask;
  for (int i = 0; i < 4; ++i) k.ms[i] = a.ms[i];
  k.S = S;
  k.scale = a.scale;
  k.fill = a.fill;
  k.out = a.out;
  k.ldo = a.ldo;
  k.bstride_o = a.bstride_o;
  k.so = a.so;
  // output maps: the hi / lo planes, or the fp32 tensor
  const CUtensorMap toh = a.so.hi ? plane_map(reinterpret_cast<const uint16_t*>(a.so.hi), nH, S, B,
                                              a.ldo, a.bstride_o)
                                  : out_f32_map(a.out, nH, S, B, a.ldo, a.bstride_o);
  const CUtensorMap tol = a.so.hi ? plane_map(reinterpret_cast<const uint16_t*>(a.so.lo), nH, S, B,
                                              a.ldo, a.bstride_o)
                                  : toh;
  if (S <= kRows) {  // one key block: the persistent kernel
    IDEV_CUDA(cudaFuncSetAttribute(attention_f16_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    // persistent: two CTAs per SM, each walking (batch, head) items
    int dev = 0, sms = 0;
    IDEV_CUDA(cudaGetDevice(&dev));
    IDEV_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int items = B * nH;
    const int grid = items < 2 * sms ? items : 2 * sms;
    launch_pdl(attention_f16_kernel, dim3((unsigned)grid), dim3(kThreads), kSmemBytes, st, tqh,
               tql, tkh, tkl, tvh, tvl, toh, tol, k, items, nH);
  } else {
    IDEV_CUDA(cudaFuncSetAttribute(attention_f16_flash_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlashSmem));
    dim3 grid((unsigned)((S + kRows - 1) / kRows), (unsigned)nH, (unsigned)B);
    attention_f16_flash_kernel<<<grid, kThreads, kFlashSmem, st>>>(tqh, tql, tkh, tkl, tvh, tvl,
                                                                   toh, tol, k);
  }
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
