// FusedAttention on the tensor cores for head_dim 64 and S <= 128: one CTA
// per (batch, head) keeps the whole attention block on chip.
//
//   1. TMA loads Q [S x 64], K [S x 64] (K-major UMMA operands, 128-byte
//      swizzle) and V [S x 64] (MN-major, 128-byte swizzle with 32-byte
//      atoms) straight out of the [B, S, H] (or fused [B, S, 3H]) tensors;
//      rows past S are zero-filled.
//   2. 3xTF32 split: the tensor core reads only the top 19 bits of a tf32
//      operand, so the raw tiles are the "big" halves and four warps form the
//      small halves x - trunc13(x) next to them.
//   3. S = Q K^T: 8 k-steps x 3 tcgen05.mma (M=128, N=128) into TMEM.
//   4. Masked row softmax, two threads per query row (its TMEM lane), each
//      holding 64 keys in registers: scores
//      are scaled by 1/sqrt(64), masked entries are REPLACED by `fill`, keys
//      past S get no weight; max, exp(s - max), * 1/sum as rt::FusedAttention
//      does (src/kernels/attention.cc:77-91). P and its small half are
//      written into shared memory in the K-major UMMA layout, over the Q/K
//      tiles that step 3 has finished reading.
//   5. O = P V: 16 k-steps x 3 tcgen05.mma (M=128, N=64) into TMEM.
//   6. O is loaded from TMEM and stored to the [B, S, H] output (or, for a
//      following split-fp16 GEMM, as its fp16 hi / lo planes).
// Waits are bounded; on a timeout the CTA flags g_attn_tc_error, frees its TMEM
// and exits.
#include <cstdlib>

#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace inferc_dev {

__device__ int g_attn_tc_error;  // set to 1 by a CTA whose barrier wait timed out

namespace {

using namespace tc;

constexpr int kRows = 128;       // query rows / keys per CTA (S <= 128)
constexpr int kHd = 64;
constexpr int kAttnThreads = 256;
constexpr uint32_t kTile = 16384;  // [128 rows][128 B]

// Byte offsets inside the 1 KiB-aligned dynamic shared memory.
constexpr uint32_t OFF_Q = 0, OFF_QS = 2 * kTile, OFF_K = 4 * kTile, OFF_KS = 6 * kTile,
                   OFF_V = 8 * kTile, OFF_VS = 10 * kTile;
constexpr uint32_t OFF_P = 0, OFF_PS = 4 * kTile;  // P reuses Q / K after step 3
// Mask tile: one byte per (query row, key); 144-byte rows keep the 16-byte
// reads of a warp (32 rows) on distinct bank groups.
constexpr uint32_t OFF_MASK = 12 * kTile, kMaskLd = 144;
constexpr uint32_t kSmemBytes = 12 * kTile + kRows * kMaskLd + 1024;

struct AttnTcArgs {
  const uint8_t* mask;
  int64_t ms[4];
  int S, nH;
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

__device__ __forceinline__ float trunc13(float v) {
  return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

// Byte offset of element (row, k) in a K-major SWIZZLE_128B operand made of
// 32-column blocks of [128 rows][128 B] (16-byte chunks XOR row % 8).
__device__ __forceinline__ uint32_t kmajor_off(int row, int k) {
  const int kb = k >> 5, c = (k & 31) >> 2;
  return (uint32_t)kb * kTile + (uint32_t)row * 128 + ((uint32_t)(c ^ (row & 7)) << 4) +
         (uint32_t)(k & 3) * 4;
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar_load, bar_s, bar_o;
  __shared__ uint32_t tmem_sh;
  __shared__ float red_max[2][kRows], red_sum[2][kRows];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.z, h = blockIdx.y;

  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
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
  const int quad = warp & 3, half = warp >> 2;  // TMEM lane quarter, key / column half
  const int row = quad * 32 + (tid & 31), col0 = 64 * half;
  const uint32_t lane_base = (uint32_t)(32 * quad) << 16;

  if (tid == 0) {
    mbar_expect_tx(&bar_load, 6 * kTile);
    for (int kb = 0; kb < 2; ++kb) {
      tma_load_4d(sm + OFF_Q + kb * kTile, &tmQ, &bar_load, kb * 32, h, 0, b);
      tma_load_4d(sm + OFF_K + kb * kTile, &tmK, &bar_load, kb * 32, h, 0, b);
      tma_load_4d(sm + OFF_V + kb * kTile, &tmV, &bar_load, kb * 32, h, 0, b);
    }
  }
  // Stage the mask while the tiles are in flight (one row when the mask
  // broadcasts over query rows).
  const int mask_rows = !a.mask ? 0 : (a.ms[2] == 0 ? 1 : a.S);
  uint8_t* msk = sm + OFF_MASK;
  if (mask_rows) {
    const uint8_t* mb = a.mask + (int64_t)b * a.ms[0] + (int64_t)h * a.ms[1];
    for (int i = tid; i < mask_rows * kRows; i += kAttnThreads) {
      const int r = i / kRows, j = i % kRows;
      msk[r * kMaskLd + j] = j < a.S ? mb[(int64_t)r * a.ms[2] + (int64_t)j * a.ms[3]] : 0;
    }
  }
  bool ok = __syncthreads_and(mbar_wait(&bar_load, 0)) != 0;
  if (ok) {
    // small halves of Q, K, V (element-wise; the swizzled layout is kept)
    for (int i = tid; i < 3 * 2 * (int)kTile / 16; i += kAttnThreads) {
      const int t = i / (2 * (int)kTile / 16), e = i % (2 * (int)kTile / 16);
      float4* src = reinterpret_cast<float4*>(sm + 4 * kTile * t) + e;
      float4* dst = reinterpret_cast<float4*>(sm + 4 * kTile * t + 2 * kTile) + e;
      const float4 v = *src;
      *dst = make_float4(v.x - trunc13(v.x), v.y - trunc13(v.y), v.z - trunc13(v.z),
                         v.w - trunc13(v.w));
    }
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_tf32_kk(kRows, kRows);
      const uint32_t q = smem_u32(sm + OFF_Q), qs = smem_u32(sm + OFF_QS);
      const uint32_t k = smem_u32(sm + OFF_K), ks = smem_u32(sm + OFF_KS);
#pragma unroll
      for (int j = 0; j < kHd / 8; ++j) {
        const uint32_t off = (j >> 2) * kTile + (j & 3) * 32;
        const uint64_t dq = smem_desc(q + off, 16, 1024, 2), dqs = smem_desc(qs + off, 16, 1024, 2);
        const uint64_t dk = smem_desc(k + off, 16, 1024, 2), dks = smem_desc(ks + off, 16, 1024, 2);
        mma_tf32(tmem, dqs, dk, idesc, j != 0);
        mma_tf32(tmem, dq, dks, idesc, 1);
        mma_tf32(tmem, dq, dk, idesc, 1);
      }
      mma_commit(&bar_s);
    }
    ok = __syncthreads_and(mbar_wait(&bar_s, 0)) != 0;
  }
  if (ok) {
    tc_fence_after();
    // ---- masked softmax: row `row` is TMEM lane quad*32 + lane; the two
    // warps of a quad hold keys [0, 64) and [64, 128) in registers.
    float s[64];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v[16];
      tmem_ld16(tmem + lane_base + (uint32_t)(col0 + 16 * c), v);
#pragma unroll
      for (int q = 0; q < 16; ++q) s[16 * c + q] = v[q];
    }
    uint4 mw[4] = {};
    if (mask_rows && row < a.S) {
      const uint4* mr = reinterpret_cast<const uint4*>(
          msk + (mask_rows == 1 ? 0 : row) * kMaskLd + col0);
#pragma unroll
      for (int c = 0; c < 4; ++c) mw[c] = mr[c];
    }
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      const int j = col0 + q;
      const uint4 w4 = mw[q >> 4];
      const uint32_t w = (q & 15) < 4 ? w4.x : (q & 15) < 8 ? w4.y : (q & 15) < 12 ? w4.z : w4.w;
      float v;
      if (j >= a.S) v = -INFINITY;  // beyond the sequence: no weight at all
      else if ((w >> (8 * (q & 3))) & 0xFFu) v = a.fill;
      else v = a.scale * s[q];
      s[q] = v;
      mx = fmaxf(mx, v);
    }
    red_max[half][row] = mx;
    __syncthreads();
    mx = fmaxf(red_max[0][row], red_max[1][row]);
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      s[q] = expf(s[q] - mx);
      sum += s[q];
    }
    red_sum[half][row] = sum;
    __syncthreads();
    const float inv = 1.0f / (red_sum[0][row] + red_sum[1][row]);
    uint8_t* P = sm + OFF_P;
    uint8_t* Ps = sm + OFF_PS;
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      const uint32_t o = kmajor_off(row, col0 + 4 * g);
      const float4 p = make_float4(s[4 * g] * inv, s[4 * g + 1] * inv, s[4 * g + 2] * inv,
                                   s[4 * g + 3] * inv);
      *reinterpret_cast<float4*>(P + o) = p;
      *reinterpret_cast<float4*>(Ps + o) = make_float4(
          p.x - trunc13(p.x), p.y - trunc13(p.y), p.z - trunc13(p.z), p.w - trunc13(p.w));
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_tf32(kRows, kHd);
      const uint32_t p = smem_u32(sm + OFF_P), ps = smem_u32(sm + OFF_PS);
      const uint32_t v = smem_u32(sm + OFF_V), vs = smem_u32(sm + OFF_VS);
#pragma unroll
      for (int j = 0; j < kRows / 8; ++j) {
        const uint32_t aoff = (j >> 2) * kTile + (j & 3) * 32;
        const uint64_t dp = smem_desc(p + aoff, 16, 1024, 2), dps = smem_desc(ps + aoff, 16, 1024, 2);
        // V: MN-major, 32-column groups of [128 rows][128 B] (kTile apart);
        // a k-step of 8 rows advances 1 KiB; 4-row (512 B) swizzle atoms.
        const uint64_t dv = smem_desc(v + j * 1024, kTile, 512, 1);
        const uint64_t dvs = smem_desc(vs + j * 1024, kTile, 512, 1);
        mma_tf32(tmem + kRows, dps, dv, idesc, j != 0);
        mma_tf32(tmem + kRows, dp, dvs, idesc, 1);
        mma_tf32(tmem + kRows, dp, dv, idesc, 1);
      }
      mma_commit(&bar_o);
    }
    ok = __syncthreads_and(mbar_wait(&bar_o, 0)) != 0;
  }
  if (ok) {
    tc_fence_after();
    // O columns [32 * half, 32 * half + 32) of row `row`
    const int64_t col = h * kHd + 32 * half;
    float* dst = a.out + (int64_t)b * a.bstride_o + (int64_t)row * a.ldo + col;
    bool bad = false;
#pragma unroll
    for (int c0 = 0; c0 < 32; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + lane_base + kRows + (uint32_t)(32 * half + c0), v);
      if (row >= a.S) continue;
      if (a.so.hi) {  // fp16 hi / lo planes with the layout of out
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) hw[q] = split_pair(v[2 * q], v[2 * q + 1], lw[q], bad);
        const int64_t o = (int64_t)b * a.bstride_o + (int64_t)row * a.ldo + col + c0;
        uint4* hp = reinterpret_cast<uint4*>(a.so.hi + o);
        uint4* lp = reinterpret_cast<uint4*>(a.so.lo + o);
        hp[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        hp[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        lp[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        lp[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
      } else {
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4*>(dst + c0 + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      }
    }
    if (bad) atomicExch(a.so.range, 1);
  } else if (tid == 0) {
    atomicExch(&g_attn_tc_error, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
  }
}

// 4-D map over one of Q / K / V inside a [B, S, rows of ld floats] tensor:
// dims (d: 64, head: nH, s: S, b: B), box (32, 1, 128, 1).
CUtensorMap head_map(const float* base, int nH, int S, int B, int64_t ld, int64_t bstride,
                     CUtensorMapSwizzle swz) {
  CUtensorMap m;
  const cuuint64_t dims[4] = {(cuuint64_t)kHd, (cuuint64_t)nH, (cuuint64_t)S, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)kHd * 4, (cuuint64_t)ld * 4, (cuuint64_t)bstride * 4};
  const cuuint32_t box[4] = {32, 1, (cuuint32_t)kRows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base),
                                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(INFERC_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (" +
                                     std::to_string((int)r) + ")");
  return m;
}

}  // namespace

int read_and_clear_attn_tc_error() {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_attn_tc_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_attn_tc_error, &z, sizeof(int)));
  }
  return v;
}

// INFERC_ATTN_TC=0 selects the CUDA-core kernel (for A/B measurements).
bool attention_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("INFERC_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool attention_tc_supported(const AttnArgs& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return a.hd == kHd && a.S >= 1 && a.S <= kRows && !a.causal && al(a.q) && al(a.k) &&
         al(a.v) && al(a.out) && a.ldq % 4 == 0 && a.ldk % 4 == 0 && a.ldv % 4 == 0 &&
         a.ldo % 4 == 0 && a.bstride_o % 4 == 0 && a.bstride_q % 4 == 0 && a.bstride_k % 4 == 0 && a.bstride_v % 4 == 0 &&
         a.ldq >= a.nH * kHd && a.ldk >= a.nH * kHd && a.ldv >= a.nH * kHd &&
         a.bstride_q >= a.S * a.ldq && a.bstride_k >= a.S * a.ldk && a.bstride_v >= a.S * a.ldv &&
         a.B < 65536 && a.nH < 65536;
}

void launch_attention_tc(const AttnArgs& a, cudaStream_t st) {
  const CUtensorMap tq = head_map(a.q, (int)a.nH, (int)a.S, (int)a.B, a.ldq, a.bstride_q,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tk = head_map(a.k, (int)a.nH, (int)a.S, (int)a.B, a.ldk, a.bstride_k,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tv = head_map(a.v, (int)a.nH, (int)a.S, (int)a.B, a.ldv, a.bstride_v,
                                  CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  AttnTcArgs t{};
  t.mask = a.mask;
  for (int i = 0; i < 4; ++i) t.ms[i] = a.ms[i];
  t.S = (int)a.S;
  t.nH = (int)a.nH;
  t.scale = a.scale;
  t.fill = a.fill;
  t.out = a.out;
  t.ldo = a.ldo;
  t.bstride_o = a.bstride_o;
  t.so = a.so;
  IDEV_CHECK_ARG(!a.so.hi || (a.so.lo && a.so.range && aligned16(a.so.hi) && aligned16(a.so.lo)),
                 "FusedAttention: fp16 split output needs aligned planes and a range flag");
  IDEV_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemBytes));
  dim3 grid(1, (unsigned)a.nH, (unsigned)a.B);
  attention_tc_kernel<<<grid, kAttnThreads, kSmemBytes, st>>>(tq, tk, tv, t);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
