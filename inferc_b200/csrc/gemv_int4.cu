// int4 per-row-scale GEMV, batched over many matrices in one launch.
//
// Restates scalar_int4_gemv_perRow (bench/amx/int4_gemv_amx.cc:258-271):
//   y[r] = sum_k (s_r * (q[r,k] - 8)) * x[k]
// with W [N, K/2] bytes, byte r*(K/2)+k/2 holding even k in the low nibble
// and odd k in the high nibble. The scale is factored out of the sum
// (y = s_r * sum_k (q-8) x_k) and the sum is fp32; the reference sums in
// double, so results agree to fp32 rounding, not bit for bit.
//
// HBM-bound. The rows of a matrix are contiguous ([N, K/2] bytes), so a
// block of consecutive rows is one contiguous byte range. Persistent kernel,
// one CTA per SM, each CTA owning a contiguous range of row blocks (about
// 32 KB each) across the batch's matrices:
//   * one producer thread streams the blocks into a STAGES-deep shared-memory
//     ring with 1-D bulk copies (cp.async.bulk + mbarrier), keeping ~160 KB
//     per SM in flight, which is what HBM needs to run at full rate;
//   * 16 consumer warps (8 for K > 1024) take one row per warp at a time: each lane
//     takes the 16-byte chunks (32 weights) of its k range from shared
//     memory and the warp reduces the row.
// The arithmetic is integer: each lane holds its activations as 22-bit
// integers (one scale per matrix) split into three byte digits, re-derived
// only when the CTA moves to the next matrix, and accumulates nibble x digit
// products exactly with dp4a (eight weights cost two masks and six dp4a).
// A lane's partial is an exact integer rounded once to fp32; a warp takes 4
// or 8 consecutive rows and reduces them together (one butterfly). The
// quantisation of x adds at most 2^-23 max|x| per element, which leaves the
// row sums within fp32 accumulation error at these K.
// Every mbarrier wait is bounded; a timeout sets g_int4_error, which
// inferc_dev_stream_synchronize reports.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace inferc_dev {
namespace {



// The activations of one 16-byte weight chunk (32 weights, k = 32c ..
// 32c+31), as integers: x_k ~= xs * a_k with a_k = round(x_k / xs), one
// scale xs = max|x| / (2^22 - 1) per matrix, so |a_k| < 2^22. Each a_k is
// stored as three signed byte digits, a_k = d0 2^16 + d1 2^8 + d2, packed
// four per word in the order the weight nibbles arrive: byte b of word m of
// the weights holds k = 8m + 2b (low nibble) and k = 8m + 2b + 1 (high).
struct XChunk {
  int ev[3][4];  // digit i of k = 8m + {0,2,4,6}
  int od[3][4];  // digit i of k = 8m + {1,3,5,7}
  int asum;      // sum of a_k (for the -8 offset of the weights)
};

__device__ __forceinline__ void load_chunk(const float* __restrict__ x, bool valid,
                                           float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 32; q += 4) {
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) t = __ldg(reinterpret_cast<const float4*>(x + q));
    v[q] = t.x; v[q + 1] = t.y; v[q + 2] = t.z; v[q + 3] = t.w;
  }
}

__device__ __forceinline__ void quantise_chunk(const float (&v)[32], float inv, XChunk& c) {
  int asum = 0;
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int i = 0; i < 3; ++i) c.ev[i][w] = c.od[i][w] = 0;
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    int a = __float2int_rn(v[q] * inv);
    a = max(-4194303, min(4194303, a));
    asum += a;
    const int d2 = ((a + 128) & 255) - 128;
    const int a1 = (a - d2) >> 8;
    const int d1 = ((a1 + 128) & 255) - 128;
    const int d0 = (a1 - d1) >> 8;
    const int w = q >> 3, sh = 8 * ((q & 7) >> 1);
    if (q & 1) {
      c.od[0][w] |= (d0 & 255) << sh;
      c.od[1][w] |= (d1 & 255) << sh;
      c.od[2][w] |= (d2 & 255) << sh;
    } else {
      c.ev[0][w] |= (d0 & 255) << sh;
      c.ev[1][w] |= (d1 & 255) << sh;
      c.ev[2][w] |= (d2 & 255) << sh;
    }
  }
  c.asum = asum;
}

// Per-lane digit sums of one chunk: even-k products exactly, odd-k products
// times 16 (the high nibble is masked in place: bytes 16 q), which stays
// exact in int32 (|sum| < 240 * 128 * K / 2 for K <= 4096).
struct DigitSums {
  int e[3], o16[3];
};

// Four (unsigned byte of a) x (signed byte of b) products added to c.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ void chunk_dot(const uint4 v, const XChunk& c, DigitSums& s) {
  const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t lo = ws[m] & 0x0F0F0F0Fu, hi16 = ws[m] & 0xF0F0F0F0u;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      s.e[i] = dp4a_us(lo, c.ev[i][m], s.e[i]);
      s.o16[i] = dp4a_us(hi16, c.od[i][m], s.o16[i]);
    }
  }
}

// sum_k (q_k - 8) a_k of the lane's chunks, as a float (one rounding).
__device__ __forceinline__ float digits_value(const DigitSums& s, int asum) {
  long long t = -8LL * asum;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const long long di = (long long)s.e[i] + (long long)(s.o16[i] >> 4);
    t += di << (16 - 8 * i);
  }
  return (float)t;
}

// Sums each of R per-lane values over the warp with one butterfly: every
// lane returns the total of value row_of_lane<R>(lane) (the first log2 R
// exchange steps halve the values each lane carries, the rest are a plain
// xor reduction).
template <int R>
__device__ __forceinline__ float multi_warp_sum(float (&v)[R], int lane) {
#pragma unroll
  for (int m = 16, c = R / 2; c >= 1; m >>= 1, c >>= 1) {
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < c; ++i) {
      const float send = up ? v[i] : v[i + c];
      const float keep = up ? v[i + c] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
  float t = v[0];
#pragma unroll
  for (int m = 16 / R; m >= 1; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
  return t;
}
template <int R>
__device__ __forceinline__ int row_of_lane(int lane) {
  return (lane >> (5 - (R == 8 ? 3 : R == 4 ? 2 : R == 2 ? 1 : 0))) & (R - 1);
}

constexpr int kStages = 4;
constexpr uint32_t kStageBytes = 48 * 1024;
// Consumer warps: 16 for rows of K <= 1024 (one chunk per lane), 8 for
// longer rows (the activation digits of several chunks stay in registers).
template <int CPL>
constexpr int consumer_warps() { return CPL == 1 ? 16 : 8; }
// Consecutive rows a consumer warp takes at once (one multi-row reduction).
template <int CPL>
constexpr int rows_per_warp() { return CPL == 1 ? 8 : 4; }
template <int CPL>
constexpr int threads_bulk() { return 32 * (consumer_warps<CPL>() + 1); }  // + producer warp
constexpr int kMaxBulkDescs = 64;

struct Int4BulkBatch {
  InfercInt4Gemv d[kMaxBulkDescs];
  int rows_per_blk[kMaxBulkDescs];
  int blk_start[kMaxBulkDescs + 1];  // prefix sums of the blocks per matrix
  int count;
};

__device__ int g_int4_error;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(tc::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
      : "memory");
}

// CPL = 16-byte chunks per lane (K <= 1024 * CPL); K % 32 == 0, 16-byte
// aligned W.
template <int CPL>
__global__ void __launch_bounds__(threads_bulk<CPL>(), 1)
    gemv_int4_bulk_kernel(const __grid_constant__ Int4BulkBatch bt) {
  constexpr int kConsumerWarps = consumer_warps<CPL>();
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages];
  pdl_launch_dependents();  // the next group of this batch may start its CTAs
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int total = bt.blk_start[bt.count];
  const int j0 = (int)((int64_t)total * blockIdx.x / gridDim.x);
  const int j1 = (int)((int64_t)total * (blockIdx.x + 1) / gridDim.x);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full_bar[s], 1);
      tc::mbar_init(&empty_bar[s], kConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (wid == kConsumerWarps) {  // ---------------- producer
    if (lane == 0) {
      int mi = 0;
      for (int j = j0; j < j1; ++j) {
        const int s = (j - j0) % kStages, r = (j - j0) / kStages;
        if (r > 0 && !tc::mbar_wait(&empty_bar[s], (r - 1) & 1)) {
          atomicExch(&g_int4_error, 1);
          break;
        }
        while (j >= bt.blk_start[mi + 1]) ++mi;
        const InfercInt4Gemv& d = bt.d[mi];
        const int64_t rb = d.k / 2;
        const int64_t r0 = (int64_t)(j - bt.blk_start[mi]) * bt.rows_per_blk[mi];
        const int64_t nr = min((int64_t)bt.rows_per_blk[mi], d.n - r0);
        const uint32_t bytes = (uint32_t)(nr * rb);
        tc::mbar_expect_tx(&full_bar[s], bytes);
        bulk_load(ring + (size_t)s * kStageBytes, d.w + r0 * rb, bytes, &full_bar[s]);
      }
    }
    return;
  }
  // ---------------- consumers
  // Warp w takes rows w R .. w R + R - 1 of a block (R = rows_per_warp);
  // the lane that stores row i fetches its scale one block ahead.
  constexpr int R = rows_per_warp<CPL>();
  const int my_row = wid * R + row_of_lane<R>(lane);
  auto block_scale = [&](int jj, int& mj) -> float {
    if (jj >= j1) return 0.f;
    while (jj >= bt.blk_start[mj + 1]) ++mj;
    const InfercInt4Gemv& dd = bt.d[mj];
    const int64_t rr0 = (int64_t)(jj - bt.blk_start[mj]) * bt.rows_per_blk[mj];
    const int64_t rr = rr0 + my_row;
    return (rr < dd.n && my_row < bt.rows_per_blk[mj]) ? __ldg(dd.scales + rr) : 0.f;
  };
  int mi = 0, loaded = -1, mi_next = 0;
  XChunk xc[CPL];  // this lane's chunks lane + 32 c
  float xs = 0.f;  // activation scale of the loaded matrix
  float sc_next = block_scale(j0, mi_next);
  for (int j = j0; j < j1; ++j) {
    const int s = (j - j0) % kStages, r = (j - j0) / kStages;
    while (j >= bt.blk_start[mi + 1]) ++mi;
    const InfercInt4Gemv& d = bt.d[mi];
    const int64_t chunks = d.k / 32, rb = d.k / 2;
    if (mi != loaded) {  // the warp covers every chunk of x: a warp-wide max
      float v[CPL][32];
      float m = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int64_t ch = lane + 32 * c;
        load_chunk(d.x + ch * 32, ch < chunks, v[c]);
#pragma unroll
        for (int q = 0; q < 32; ++q) m = fmaxf(m, fabsf(v[c][q]));
      }
      m = warp_max(m);
      xs = m > 0.f ? m / 4194303.0f : 0.f;
      const float inv = m > 0.f ? 4194303.0f / m : 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) quantise_chunk(v[c], inv, xc[c]);
      loaded = mi;
    }
    const float sc_lane = sc_next;
    sc_next = block_scale(j + 1, mi_next);
    const int64_t r0 = (int64_t)(j - bt.blk_start[mi]) * bt.rows_per_blk[mi];
    const int nr = (int)min((int64_t)bt.rows_per_blk[mi], d.n - r0);
    if (!tc::mbar_wait(&full_bar[s], r & 1)) {
      if (lane == 0) atomicExch(&g_int4_error, 1);
      break;
    }
    const uint8_t* blk = ring + (size_t)s * kStageBytes;
    if (wid * R < nr) {
      float part[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int row = wid * R + i;
        DigitSums ds = {{0, 0, 0}, {0, 0, 0}};
        int asum = 0;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int64_t ch = lane + 32 * c;
          if (ch < chunks && row < nr) {
            chunk_dot(*reinterpret_cast<const uint4*>(blk + row * rb + ch * 16), xc[c], ds);
            asum += xc[c].asum;
          }
        }
        part[i] = digits_value(ds, asum);
      }
      const float tot = multi_warp_sum<R>(part, lane);
      if ((lane & (32 / R - 1)) == 0 && my_row < nr) d.y[r0 + my_row] = sc_lane * xs * tot;
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty_bar[s]);
  }
}

// Any even K, any alignment: one thread per row, byte loads.
__global__ void gemv_int4_scalar_kernel(InfercInt4Gemv d) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= d.n) return;
  const uint8_t* row = d.w + r * (d.k / 2);
  float acc = 0.f;
  for (int64_t k = 0; k < d.k; k += 2) {
    const uint8_t b = row[k / 2];
    acc = fmaf((float)((int)(b & 0xF) - 8), d.x[k], acc);
    acc = fmaf((float)((int)(b >> 4) - 8), d.x[k + 1], acc);
  }
  d.y[r] = d.scales[r] * acc;
}

bool fast_ok(const InfercInt4Gemv& d) {
  return d.k % 32 == 0 && d.k <= 4096 && aligned16(d.w) && aligned16(d.x);
}

template <int CPL>
void launch_group(const InfercInt4Gemv* ds, const int* idx, int n, cudaStream_t st,
                  bool& first) {
  static int sms = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  const size_t smem = (size_t)kStages * kStageBytes;
  IDEV_CUDA(cudaFuncSetAttribute(gemv_int4_bulk_kernel<CPL>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  for (int base = 0; base < n; base += kMaxBulkDescs) {
    Int4BulkBatch bt{};
    bt.count = std::min(kMaxBulkDescs, n - base);
    int blks = 0;
    for (int i = 0; i < bt.count; ++i) {
      const InfercInt4Gemv& d = ds[idx[base + i]];
      bt.d[i] = d;
      const int64_t rb = d.k / 2;
      bt.rows_per_blk[i] = (int)std::max<int64_t>(
          1, std::min<int64_t>(kStageBytes / rb, consumer_warps<CPL>() * rows_per_warp<CPL>()));
      bt.blk_start[i] = blks;
      blks += (int)((d.n + bt.rows_per_blk[i] - 1) / bt.rows_per_blk[i]);
    }
    bt.blk_start[bt.count] = blks;
    if (blks == 0) continue;
    const int grid = std::min(blks, sms);
    if (first) {  // ordered after all earlier work on the stream
      gemv_int4_bulk_kernel<CPL><<<grid, threads_bulk<CPL>(), smem, st>>>(bt);
      IDEV_LAUNCHED();
      first = false;
    } else {
      // Same batch, independent matrices: may overlap the previous group.
      // Its inputs were complete before the first group started.
      launch_pdl(gemv_int4_bulk_kernel<CPL>, dim3(grid), dim3(threads_bulk<CPL>()), smem, st, bt);
    }
  }
}

}  // namespace

int read_and_clear_int4_error() {
  int v = 0;
  IDEV_CUDA(cudaMemcpyFromSymbol(&v, g_int4_error, sizeof(int)));
  if (v) {
    const int z = 0;
    IDEV_CUDA(cudaMemcpyToSymbol(g_int4_error, &z, sizeof(int)));
  }
  return v;
}

void launch_gemv_int4(const InfercInt4Gemv* ds, int count, cudaStream_t st) {
  IDEV_CHECK_ARG(count >= 0 && (count == 0 || ds != nullptr), "int4 GEMV: bad descriptor list");
  int groups[4][256];
  int ng[4] = {0, 0, 0, 0};
  bool first = true;
  auto flush = [&](int g) {
    if (ng[g] == 0) return;
    switch (g) {
      case 0: launch_group<1>(ds, groups[0], ng[0], st, first); break;
      case 1: launch_group<2>(ds, groups[1], ng[1], st, first); break;
      case 2: launch_group<3>(ds, groups[2], ng[2], st, first); break;
      default: launch_group<4>(ds, groups[3], ng[3], st, first); break;
    }
    ng[g] = 0;
  };
  for (int i = 0; i < count; ++i) {
    const InfercInt4Gemv& d = ds[i];
    IDEV_CHECK_ARG(d.k > 0 && d.k % 2 == 0 && d.n >= 0, "int4 GEMV: K must be even and positive");
    IDEV_CHECK_ARG(d.n == 0 || (d.w && d.scales && d.x && d.y), "int4 GEMV: null pointer");
    if (d.n == 0) continue;
    if (!fast_ok(d)) {
      gemv_int4_scalar_kernel<<<(unsigned)((d.n + 255) / 256), 256, 0, st>>>(d);
      IDEV_LAUNCHED();
      continue;
    }
    const int g = (int)((d.k + 1023) / 1024) - 1;
    groups[g][ng[g]++] = i;
    if (ng[g] == 256) flush(g);
  }
  for (int g = 0; g < 4; ++g) flush(g);
}

}  // namespace inferc_dev
