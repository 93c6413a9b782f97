// int4 per-row-scale GEMV, batched over many matrices in one launch.
//
// Restates scalar_int4_gemv_perRow (bench/amx/int4_gemv_amx.cc:258-271):
//   y[r] = sum_k (s_r * (q[r,k] - 8)) * x[k]
// with W [N, K/2] bytes, byte r*(K/2)+k/2 holding even k in the low nibble
// and odd k in the high nibble. The scale is factored out of the sum
// (y = s_r * sum_k (q-8) x_k) and the sum is fp32; the reference sums in
// double, so results agree to fp32 rounding, not bit for bit.
//
// HBM-bound: one warp per row, each lane loads 16 bytes (32 weights) per
// chunk with coalesced 512-byte warp transactions. The lane keeps the 32
// activations of its chunk(s) in registers for every row the warp touches,
// so x is read from L2 once per CTA. Nibble -> float uses the exponent trick
// float(0x4B000000 | n) - (2^23 + 8) = n - 8, exact for n in [0, 15]
// (one byte permute + one add per weight).
#include "kernels.cuh"

namespace inferc_dev {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// Rows per warp: 8 for K <= 1024; 4 for longer rows, so that the few long
// matrices still spread over every SM.
template <int CPL>
constexpr int rows_per_warp() { return CPL == 1 ? 8 : 4; }
template <int CPL>
constexpr int rows_per_cta() { return kWarps * rows_per_warp<CPL>(); }
constexpr int kMaxDescs = 32;

struct Int4Batch {
  InfercInt4Gemv d[kMaxDescs];
  int cta_start[kMaxDescs + 1];
  int count;
};


// Packed fp32x2 arithmetic (sm_100): two lanes of fp32 per instruction.
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return make_float2(a, b);
}

// (2^23 + lo_nibble(byte), 2^23 + hi_nibble(byte)) of byte `sel` of the
// nibble-split words, as a packed pair.
__device__ __forceinline__ uint64_t nib_pair(uint32_t lo, uint32_t hi, uint32_t sel) {
  return pack2(__int_as_float(__byte_perm(lo, 0x4B000000u, sel)),
               __int_as_float(__byte_perm(hi, 0x4B000000u, sel)));
}

// Accumulates one 16-byte chunk (32 weights, k = 32c .. 32c+31) into the
// packed (even k, odd k) accumulator. Byte b of word m holds k = 8m + 2b
// (low nibble) and k = 8m + 2b + 1 (high nibble), so each byte gives one
// (x[k], x[k+1]) pair.
__device__ __forceinline__ uint64_t chunk_dot(const uint4 v, const uint64_t (&x2)[16], uint64_t acc) {
  const uint64_t bias = pack2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
  const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t lo = ws[m] & 0x0F0F0F0Fu, hi = (ws[m] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint64_t q = add2(nib_pair(lo, hi, 0x7540u + b), bias);  // (q_k - 8, q_k+1 - 8)
      acc = fma2(q, x2[4 * m + b], acc);
    }
  }
  return acc;
}

// CPL = 16-byte chunks per lane (K <= 1024 * CPL); requires K % 32 == 0 and
// 16-byte aligned W rows.
template <int CPL>
__global__ void __launch_bounds__(kThreads) gemv_int4_kernel(const __grid_constant__ Int4Batch bt) {
  constexpr int kRowsPerWarp = rows_per_warp<CPL>();
  constexpr int kRowsPerCta = rows_per_cta<CPL>();
  // Lets the next group of this batch start while this one runs (the groups
  // are independent; see launch_gemv_int4).
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int total = bt.cta_start[bt.count];
  int loaded = -1;  // matrix whose x is in registers
  uint64_t xr[CPL][16];  // (x[k], x[k+1]) pairs of this lane's chunks
  // Persistent: each CTA walks row blocks blockIdx.x, + gridDim.x, ...
  for (int cta = blockIdx.x; cta < total; cta += gridDim.x) {
    int mi = 0;
    while (mi + 1 < bt.count && cta >= bt.cta_start[mi + 1]) ++mi;
    const InfercInt4Gemv& d = bt.d[mi];
    const int64_t chunks = d.k / 32;
    if (mi != loaded) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int64_t ch = lane + 32 * c;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (ch < chunks) v = *reinterpret_cast<const float4*>(d.x + ch * 32 + j);
          xr[c][j / 2] = pack2(v.x, v.y);
          xr[c][j / 2 + 1] = pack2(v.z, v.w);
        }
      }
      loaded = mi;
    }
    const int64_t row0 = (int64_t)(cta - bt.cta_start[mi]) * kRowsPerCta + wid * kRowsPerWarp;
    const int64_t row_bytes = d.k / 2;
#pragma unroll 1
    for (int rr = 0; rr < kRowsPerWarp; rr += 4) {
      uint4 v[4][CPL];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t r = row0 + rr + u;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int64_t ch = lane + 32 * c;
          v[u][c] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // q = 0
          if (r < d.n && ch < chunks)
            v[u][c] = __ldg(reinterpret_cast<const uint4*>(d.w + r * row_bytes) + ch);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t r = row0 + rr + u;
        uint64_t acc2 = pack2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc2 = chunk_dot(v[u][c], xr[c], acc2);
        const float2 a2 = unpack2(acc2);
        const float acc = warp_sum(a2.x + a2.y);
        if (lane == 0 && r < d.n) d.y[r] = d.scales[r] * acc;
      }
    }
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
  constexpr int kRowsPerCta = rows_per_cta<CPL>();
  for (int base = 0; base < n; base += kMaxDescs) {
    Int4Batch bt{};
    bt.count = std::min(kMaxDescs, n - base);
    int ctas = 0;
    for (int i = 0; i < bt.count; ++i) {
      bt.d[i] = ds[idx[base + i]];
      bt.cta_start[i] = ctas;
      ctas += (int)((bt.d[i].n + kRowsPerCta - 1) / kRowsPerCta);
    }
    bt.cta_start[bt.count] = ctas;
    if (ctas == 0) continue;
    // Persistent grid: as many CTAs as fit at once, each walking row blocks.
    static int resident = [] {
      int per_sm = 1, dev = 0, sms = 148;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_int4_kernel<CPL>, kThreads, 0);
      if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      return std::max(1, per_sm) * sms;
    }();
    const int grid = std::min(ctas, resident);
    if (first) {  // ordered after all earlier work on the stream
      gemv_int4_kernel<CPL><<<grid, kThreads, 0, st>>>(bt);
      IDEV_LAUNCHED();
      first = false;
    } else {
      // Same batch, independent matrices: may overlap the previous group.
      // Its inputs were complete before the first group started.
      launch_pdl(gemv_int4_kernel<CPL>, dim3(grid), dim3(kThreads), 0, st, bt);
    }
  }
}

}  // namespace

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
