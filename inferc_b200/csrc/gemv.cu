// Batch-1 decode GEMVs (HBM-bound: every weight byte is read exactly once).
//
//  * gemv_kn: y[N] = act(alpha * x[K] W[K,N] + beta*b + resid) for the
//    [K,N] weights of the decode graph's M==1 Gemm nodes
//    (src/kernels/matmul.cc:202-226). A CTA owns 128 columns (one float4 per
//    lane, coalesced 512-byte row segments) and a slice of K; the K slices
//    of one column tile are spread over CTAs (split-K) so that ~2 CTAs per SM
//    stream weights. Partial sums go to a workspace and the last CTA to
//    finish a column tile adds them in split order, so the result does not
//    depend on CTA scheduling. An optional LayerNorm prologue normalises x
//    in shared memory (the decode graph's FusedLayerNorm feeding the Gemm).
//  * row_gemv: y[N] = W[N,K] x for row-major [N,K] weights (the tied LM head
//    MatMul(x, wte^T)), one warp per row, with optional LayerNorm prologue
//    and a fused greedy argmax (first maximum wins, src/cli/main.cpp:870-875).
#include "kernels.cuh"

#include <mutex>
#include <vector>

namespace inferc_dev {

void Workspace::allocate(size_t floats, size_t n) {
  IDEV_CUDA(cudaMalloc(&partials, floats * sizeof(float)));
  IDEV_CUDA(cudaMalloc(&counters, n * sizeof(unsigned int)));
  IDEV_CUDA(cudaMemset(counters, 0, n * sizeof(unsigned int)));
  partial_floats = floats;
  n_counters = n;
  owned = true;
}

void Workspace::release() {
  if (owned) {
    cudaFree(partials);
    cudaFree(counters);
  }
  partials = nullptr;
  counters = nullptr;
  owned = false;
}

Workspace& workspace_for_current_device() {
  static std::mutex mu;
  static std::vector<Workspace> per_dev;
  int dev = 0;
  IDEV_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if ((int)per_dev.size() <= dev) per_dev.resize(dev + 1);
  Workspace& ws = per_dev[dev];
  if (!ws.owned) ws.allocate(size_t(4) << 20, 8192);  // 16 MB of partials
  return ws;
}

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kColsPerCta = 128;  // 32 lanes x float4
constexpr int kMaxK = 8192;       // shared-memory copy of x

// Normalised (or plain) copy of x[k0:k1) into xs[0:k1-k0). With LN, the
// mean and biased variance of the full x[0:K) are computed first (two
// passes, like rt::LayerNorm).
__device__ void stage_x(const float* __restrict__ x, const float* __restrict__ g,
                        const float* __restrict__ b, float eps, int64_t K, int64_t k0, int64_t k1,
                        float* xs, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (g == nullptr) {
    for (int64_t k = k0 + tid; k < k1; k += kThreads) xs[k - k0] = x[k];
    __syncthreads();
    return;
  }
  float s = 0.f;
  for (int64_t k = tid; k < K; k += kThreads) s += x[k];
  s = warp_sum(s);
  if (lane == 0) red[wid] = s;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < kWarps; ++w) tot += red[w];
  const float mean = tot / (float)K;
  __syncthreads();
  float sq = 0.f;
  for (int64_t k = tid; k < K; k += kThreads) {
    const float d = x[k] - mean;
    sq += d * d;
  }
  sq = warp_sum(sq);
  if (lane == 0) red[wid] = sq;
  __syncthreads();
  float tsq = 0.f;
  for (int w = 0; w < kWarps; ++w) tsq += red[w];
  const float inv = 1.0f / sqrtf(tsq / (float)K + eps);
  for (int64_t k = k0 + tid; k < k1; k += kThreads) xs[k - k0] = ((x[k] - mean) * inv) * g[k] + b[k];
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads)
    gemv_kn_kernel(GemvArgs a, int64_t k_per_split, int splits, float* partials,
                   unsigned int* counters) {
  __shared__ float xs[kMaxK];
  __shared__ float red[kWarps];
  __shared__ float4 wsum[kWarps][32];
  __shared__ bool last;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t n0 = (int64_t)blockIdx.x * kColsPerCta;
  const int split = blockIdx.y;
  const int64_t k0 = split * k_per_split;
  const int64_t k1 = min(a.K, k0 + k_per_split);
  // Weights do not depend on the previous kernel: fetch this warp's first
  // kPrefetch rows into registers before waiting on it.
  constexpr int kPrefetch = 8;
  const int64_t col = n0 + lane * 4;
  const bool colok = col < a.N;
  const float* wp = a.w + col;
  float4 wr[kPrefetch];
#pragma unroll
  for (int r = 0; r < kPrefetch; ++r) {
    const int64_t k = k0 + wid + r * kWarps;
    wr[r] = (colok && k < k1) ? __ldg(reinterpret_cast<const float4*>(wp + k * a.N))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_launch_dependents();
  pdl_wait();
  stage_x(a.x, a.ln_gamma, a.ln_beta, a.ln_eps, a.K, k0, k1, xs, red);

  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kPrefetch; ++r) {
    const int64_t k = k0 + wid + r * kWarps;
    const float x0 = k < k1 ? xs[k - k0] : 0.f;
    acc.x = fmaf(x0, wr[r].x, acc.x); acc.y = fmaf(x0, wr[r].y, acc.y);
    acc.z = fmaf(x0, wr[r].z, acc.z); acc.w = fmaf(x0, wr[r].w, acc.w);
  }
  if (colok) {
    for (int64_t k = k0 + wid + kPrefetch * kWarps; k < k1; k += kWarps) {
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(wp + k * a.N));
      const float x0 = xs[k - k0];
      acc.x = fmaf(x0, w0.x, acc.x); acc.y = fmaf(x0, w0.y, acc.y);
      acc.z = fmaf(x0, w0.z, acc.z); acc.w = fmaf(x0, w0.w, acc.w);
    }
  }
  wsum[wid][lane] = acc;
  __syncthreads();
  // Warps 0..3 each finish 32 columns: sum the 8 warp partials in order.
  float part = 0.f;
  int64_t c = -1;
  if (tid < kColsPerCta) {
    const int l = tid >> 2, e = tid & 3;
    for (int w = 0; w < kWarps; ++w) {
      const float4 v = wsum[w][l];
      part += e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w;
    }
    c = n0 + tid;
  }
  auto finish = [&](float total, int64_t cc) {
    float v = a.alpha * total;
    if (a.bias) v += a.beta * a.bias[cc];
    if (a.resid) v += a.resid[cc];
    a.y[cc] = apply_act(v, a.act);
  };
  if (splits == 1) {
    if (c >= 0 && c < a.N) finish(part, c);
    return;
  }
  if (c >= 0 && c < a.N) partials[(int64_t)split * a.N + c] = part;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&counters[blockIdx.x], 1u);
    last = (prev == (unsigned)splits - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (c >= 0 && c < a.N) {
    float total = 0.f;
    for (int s = 0; s < splits; ++s) total += __ldcg(&partials[(int64_t)s * a.N + c]);
    finish(total, c);
  }
  if (tid == 0) counters[blockIdx.x] = 0u;  // ready for the next launch
}

// Scalar fallback for odd N / unaligned pointers: one thread per column.
// One warp per column (lanes take k = lane, lane + 32, ..., then a fixed-order
// warp sum): a few columns, or a layout the vector kernel cannot take.
__global__ void gemv_kn_scalar_kernel(GemvArgs a) {
  __shared__ float xs[kMaxK];
  __shared__ float red[kWarps];
  stage_x(a.x, a.ln_gamma, a.ln_beta, a.ln_eps, a.K, 0, a.K, xs, red);
  const int lane = threadIdx.x & 31;
  const int64_t c = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (c >= a.N) return;
  float acc = 0.f;
  for (int64_t k = lane; k < a.K; k += 32) acc = fmaf(xs[k], a.w[k * a.N + c], acc);
  acc = warp_sum(acc);
  if (lane != 0) return;
  float v = a.alpha * acc;
  if (a.bias) v += a.beta * a.bias[c];
  if (a.resid) v += a.resid[c];
  a.y[c] = apply_act(v, a.act);
}

// ---------------------------------------------------------------- row gemv

struct BestIdx {
  float v;
  int64_t i;
};
// First maximum wins: larger value, or equal value at a smaller index.
__device__ __forceinline__ bool better(float v, int64_t i, float bv, int64_t bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void warp_best(float& v, int64_t& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) { v = ov; i = oi; }
  }
}

__global__ void __launch_bounds__(kThreads)
    row_gemv_kernel(RowGemvArgs a, float* best_v, int64_t* best_i, unsigned int* counter) {
  __shared__ __align__(16) float xs[kMaxK];
  __shared__ float red[kWarps];
  __shared__ float sv[kWarps];
  __shared__ int64_t si[kWarps];
  __shared__ bool last;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  pdl_launch_dependents();
  pdl_wait();
  stage_x(a.x, a.ln_gamma, a.ln_beta, a.ln_eps, a.K, 0, a.K, xs, red);
  const int64_t K4 = a.K / 4;
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  const int64_t stride = (int64_t)gridDim.x * kWarps;
  // Four rows per warp per iteration: 4 x K4/32 independent 128-bit loads in
  // flight per lane.
  for (int64_t r0 = (int64_t)blockIdx.x * kWarps + wid; r0 < a.N; r0 += 4 * stride) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t k = lane; k < K4; k += 32) {
      const float4 xv = x4[k];
      float4 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t r = r0 + u * stride;
        w[u] = r < a.N ? __ldg(reinterpret_cast<const float4*>(a.w + r * a.K) + k)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc[u] = fmaf(xv.x, w[u].x, acc[u]);
        acc[u] = fmaf(xv.y, w[u].y, acc[u]);
        acc[u] = fmaf(xv.z, w[u].z, acc[u]);
        acc[u] = fmaf(xv.w, w[u].w, acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t r = r0 + u * stride;
      const float v = warp_sum(acc[u]);
      if (r < a.N) {
        if (lane == 0) a.y[r] = v;
        if (better(v, r, bv, bi)) { bv = v; bi = r; }
      }
    }
  }
  if (a.argmax_out == nullptr) return;
  // bv/bi are identical across the lanes of a warp (warp_sum broadcasts).
  if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
  __syncthreads();
  if (tid == 0) {
    float v = sv[0];
    int64_t i = si[0];
    for (int w = 1; w < kWarps; ++w)
      if (better(sv[w], si[w], v, i)) { v = sv[w]; i = si[w]; }
    best_v[blockIdx.x] = v;
    best_i[blockIdx.x] = i;
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (wid == 0) {
    float v = -INFINITY;
    int64_t i = INT64_MAX;
    for (int64_t b = lane; b < gridDim.x; b += 32) {
      const float ov = __ldcg(&best_v[b]);
      const int64_t oi = __ldcg(&best_i[b]);
      if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
    warp_best(v, i);
    if (lane == 0) {
      *a.argmax_out = i;
      if (a.pos_counter) {
        const int64_t pos = *a.pos_counter;
        if (a.token_log) a.token_log[pos - a.log_base] = i;
        *a.pos_counter = pos + 1;
      }
      *counter = 0u;
    }
  }
}

__global__ void argmax_kernel(const float* __restrict__ x, int64_t n, int64_t* out, float* best_v,
                              int64_t* best_i, unsigned int* counter) {
  __shared__ float sv[kWarps];
  __shared__ int64_t si[kWarps];
  __shared__ bool last;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + tid; i < n; i += (int64_t)gridDim.x * kThreads)
    if (better(x[i], i, bv, bi)) { bv = x[i]; bi = i; }
  warp_best(bv, bi);
  if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
  __syncthreads();
  if (tid == 0) {
    float v = sv[0];
    int64_t i = si[0];
    for (int w = 1; w < kWarps; ++w)
      if (better(sv[w], si[w], v, i)) { v = sv[w]; i = si[w]; }
    best_v[blockIdx.x] = v;
    best_i[blockIdx.x] = i;
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || wid != 0) return;
  __threadfence();
  float v = -INFINITY;
  int64_t i = INT64_MAX;
  for (int64_t b = lane; b < gridDim.x; b += 32) {
    const float ov = __ldcg(&best_v[b]);
    const int64_t oi = __ldcg(&best_i[b]);
    if (better(ov, oi, v, i)) { v = ov; i = oi; }
  }
  warp_best(v, i);
  if (lane == 0) {
    // All-NaN input: report index 0, as the reference's scan would.
    *out = (i == INT64_MAX) ? 0 : i;
    *counter = 0u;
  }
}

__global__ void decode_embed_kernel(const int64_t* tok, const int64_t* pos, const float* wte,
                                    const float* wpe, float* x, int64_t H, int64_t vocab,
                                    int64_t max_pos, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t t = *tok, p = *pos - 1;
  if (t < 0 || t >= vocab || p < 0 || p >= max_pos) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, 1);
    return;
  }
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < H;
       c += (int64_t)gridDim.x * blockDim.x)
    x[c] = wte[t * H + c] + wpe[p * H + c];
}

__global__ void rows_embed_kernel(const int64_t* ids, int64_t n, int64_t pos0, const float* wte,
                                  const float* wpe, float* x, int64_t H, int64_t vocab, int* err) {
  const int64_t r = blockIdx.x;
  if (r >= n) return;
  const int64_t t = ids[r];
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0) atomicExch(err, 1);
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) x[r * H + c] = 0.f;
    return;
  }
  for (int64_t c = threadIdx.x; c < H; c += blockDim.x)
    x[r * H + c] = wte[t * H + c] + wpe[(pos0 + r) * H + c];
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}


// ------------------------------------------------------------ int4 rows
// y[r] = act(s_r * sum_k (q[r,k] - 8) x_k + b[r] + resid[r]) over int4 weights
// in the layout of bench/amx/int4_gemv_amx.cc:258-271 (row r = K/2 bytes,
// even k in the low nibble, stored nibble = q + 8), with the optional
// LayerNorm prologue and fused greedy argmax of row_gemv. One warp per row,
// four rows in flight per warp; lane l reads 4-byte words l, l+32, ... of the
// row (8 weights each) and the matching 8 staged x values (two float4 reads,
// 32 bytes apart across lanes: at most 2-way bank conflicts). The weight is
// formed as (q - 8) in fp32 exactly; the row sum is scaled once by s_r.
__global__ void __launch_bounds__(kThreads)
    int4_row_gemv_kernel(Int4RowArgs a, float* best_v, int64_t* best_i, unsigned int* counter) {
  __shared__ __align__(16) float xs[kMaxK];
  __shared__ float red[kWarps];
  __shared__ float sv[kWarps];
  __shared__ int64_t si[kWarps];
  __shared__ bool last;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t words = a.K / 8;
  const int64_t stride = (int64_t)gridDim.x * kWarps;
  auto wload = [&](int64_t r, int64_t wi) {
    return (r < a.N && wi < words)
               ? __ldg(reinterpret_cast<const uint32_t*>(a.w + r * (a.K / 2)) + wi)
               : 0x88888888u;
  };
  // The weights do not depend on the previous kernel: the first row group's
  // first kPre words per row are loaded before waiting on it.
  constexpr int kPre = 4;
  uint32_t pre[4][kPre];
  {
    const int64_t r0 = (int64_t)blockIdx.x * kWarps + wid;
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < kPre; ++j) pre[u][j] = wload(r0 + u * stride, lane + 32 * j);
  }
  pdl_launch_dependents();
  pdl_wait();
  stage_x(a.x, a.ln_gamma, a.ln_beta, a.ln_eps, a.K, 0, a.K, xs, red);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  bool first = true;
  for (int64_t r0 = (int64_t)blockIdx.x * kWarps + wid; r0 < a.N; r0 += 4 * stride) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int j = 0;
    for (int64_t wi = lane; wi < words; wi += 32, ++j) {
      uint32_t wv[4];
      if (first && j < kPre) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int q = 0; q < kPre; ++q)
            if (q == j) wv[u] = pre[u][q];
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) wv[u] = wload(r0 + u * stride, wi);
      }
      const float4 xa = x4[2 * wi], xb = x4[2 * wi + 1];
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          acc[u] = fmaf((float)((int)((wv[u] >> (4 * e)) & 15u) - 8), xv[e], acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t r = r0 + u * stride;
      const float dot = warp_sum(acc[u]);
      if (r < a.N) {
        float v = __ldg(a.scales + r) * dot;
        if (a.bias) v += a.bias[r];
        if (a.resid) v += a.resid[r];
        v = apply_act(v, a.act);
        if (lane == 0) a.y[r] = v;
        if (better(v, r, bv, bi)) { bv = v; bi = r; }
      }
    }
    first = false;
  }
  if (a.argmax_out == nullptr) return;
  if (lane == 0) { sv[wid] = bv; si[wid] = bi; }
  __syncthreads();
  if (tid == 0) {
    float v = sv[0];
    int64_t i = si[0];
    for (int w = 1; w < kWarps; ++w)
      if (better(sv[w], si[w], v, i)) { v = sv[w]; i = si[w]; }
    best_v[blockIdx.x] = v;
    best_i[blockIdx.x] = i;
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (wid == 0) {
    float v = -INFINITY;
    int64_t i = INT64_MAX;
    for (int64_t b = lane; b < gridDim.x; b += 32) {
      const float ov = __ldcg(&best_v[b]);
      const int64_t oi = __ldcg(&best_i[b]);
      if (better(ov, oi, v, i)) { v = ov; i = oi; }
    }
    warp_best(v, i);
    if (lane == 0) {
      *a.argmax_out = i;
      if (a.pos_counter) {
        const int64_t pos = *a.pos_counter;
        if (a.token_log) a.token_log[pos - a.log_base] = i;
        *a.pos_counter = pos + 1;
      }
      *counter = 0u;
    }
  }
}

// Per-row symmetric int4 quantisation of a weight matrix: output row r is
// column r of a [K, N] Conv1D weight (trans = false) or row r of an [N, K]
// weight (trans = true). s_r = max_k |w| / 7 (1 for an all-zero row),
// q = clamp(rint(w / s_r), -8, 7), stored as q + 8 two per byte (even k low).
__global__ void int4_pack_kernel(const float* __restrict__ w, int64_t K, int64_t N, int64_t ldw,
                                 bool trans, uint8_t* __restrict__ out,
                                 float* __restrict__ scales) {
  __shared__ float red[kWarps];
  const int64_t r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  auto at = [&](int64_t k) { return trans ? w[r * ldw + k] : w[k * ldw + r]; };
  float m = 0.f;
  for (int64_t k = tid; k < K; k += kThreads) m = fmaxf(m, fabsf(at(k)));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[wid] = m;
  __syncthreads();
  m = red[0];
  for (int i = 1; i < kWarps; ++i) m = fmaxf(m, red[i]);
  const float s = m > 0.f ? m / 7.0f : 1.0f;
  if (tid == 0) scales[r] = s;
  for (int64_t j = tid; j < K / 2; j += kThreads) {
    const float q0 = fminf(fmaxf(rintf(at(2 * j) / s), -8.f), 7.f);
    const float q1 = fminf(fmaxf(rintf(at(2 * j + 1) / s), -8.f), 7.f);
    out[r * (K / 2) + j] = (uint8_t)(((int)q0 + 8) | (((int)q1 + 8) << 4));
  }
}

}  // namespace

// Split-K count of gemv_kn_kernel for a [K, N] weight: enough CTAs to cover
// the SMs, at most 64 rows per CTA (so that each warp's rows fit the register
// prefetch), bounded by the partial-sum floats and reduction counters of the
// scratch the call uses. *kps receives the rows per split. Both the
// workspace GEMV and the allocation-free one use this rule, so they sum in
// the same order and give identical results.
int64_t gemv_splits(int64_t K, int64_t N, size_t partial_floats, size_t counters,
                    int64_t* kps) {
  const int64_t tiles = (N + kColsPerCta - 1) / kColsPerCta;
  const int64_t target = 2 * (int64_t)sm_count();
  int64_t splits = std::max<int64_t>(1, target / tiles);
  splits = std::max<int64_t>(splits, (K + 63) / 64);
  splits = std::min<int64_t>(splits, std::max<int64_t>(1, K / kWarps));
  while (splits > 1 && (size_t)(splits * N) > partial_floats) --splits;
  if ((size_t)tiles > counters) splits = 1;
  *kps = (K + splits - 1) / splits;
  return (K + *kps - 1) / *kps;
}

void launch_gemv(const GemvArgs& g, cudaStream_t st) {
  if (g.N <= 0) return;
  IDEV_CHECK_ARG(g.K > 0 && g.K <= kMaxK, "GEMV: K must be in [1, 8192]");
  Workspace& ws = g.ws ? *g.ws : workspace_for_current_device();
  const bool vec = g.N % 4 == 0 && aligned16(g.w);
  if (!vec) {
    gemv_kn_scalar_kernel<<<(unsigned)((g.N + kWarps - 1) / kWarps), kThreads, 0, st>>>(g);
    IDEV_LAUNCHED();
    return;
  }
  const int64_t tiles = (g.N + kColsPerCta - 1) / kColsPerCta;
  int64_t kps = 0;
  // the last two counter slots belong to the argmax kernels
  const int64_t splits = gemv_splits(g.K, g.N, ws.partial_floats,
                                     ws.n_counters >= 2 ? ws.n_counters - 2 : 0, &kps);
  dim3 grid((unsigned)tiles, (unsigned)splits);
  launch_pdl(gemv_kn_kernel, grid, dim3(kThreads), 0, st, g, kps, (int)splits, ws.partials,
             ws.counters);
}

void launch_row_gemv(const RowGemvArgs& g, cudaStream_t st) {
  if (g.N <= 0) return;
  IDEV_CHECK_ARG(g.K > 0 && g.K <= kMaxK && g.K % 4 == 0 && aligned16(g.w),
                 "row GEMV: K must be a multiple of 4 in [4, 8192], W 16-byte aligned");
  Workspace& ws = g.ws ? *g.ws : workspace_for_current_device();
  const int64_t want = std::min<int64_t>(4 * (int64_t)sm_count(), (g.N + kWarps - 1) / kWarps);
  const int blocks = (int)std::max<int64_t>(1, want);
  IDEV_CHECK_ARG((size_t)blocks * 3 <= ws.partial_floats && ws.n_counters >= 1,
                 "row GEMV: workspace too small");
  // best values / indices live in the partials buffer: [blocks] floats then
  // [blocks] int64 (8-byte aligned offset).
  float* best_v = ws.partials;
  int64_t* best_i = reinterpret_cast<int64_t*>(ws.partials + ((blocks + 1) & ~1));
  launch_pdl(row_gemv_kernel, dim3(blocks), dim3(kThreads), 0, st, g, best_v, best_i,
             ws.counters + ws.n_counters - 1);
}

void launch_int4_row_gemv(const Int4RowArgs& g, cudaStream_t st) {
  if (g.N <= 0) return;
  IDEV_CHECK_ARG(g.K > 0 && g.K <= kMaxK && g.K % 8 == 0 &&
                     (reinterpret_cast<uintptr_t>(g.w) & 3) == 0 && (g.K / 2) % 4 == 0,
                 "int4 row GEMV: K must be a multiple of 8 in [8, 8192], W 4-byte aligned");
  Workspace& ws = g.ws ? *g.ws : workspace_for_current_device();
  const int64_t want = std::min<int64_t>(4 * (int64_t)sm_count(), (g.N + kWarps - 1) / kWarps);
  const int blocks = (int)std::max<int64_t>(1, want);
  IDEV_CHECK_ARG((size_t)blocks * 3 <= ws.partial_floats && ws.n_counters >= 1,
                 "int4 row GEMV: workspace too small");
  float* best_v = ws.partials;
  int64_t* best_i = reinterpret_cast<int64_t*>(ws.partials + ((blocks + 1) & ~1));
  launch_pdl(int4_row_gemv_kernel, dim3(blocks), dim3(kThreads), 0, st, g, best_v, best_i,
             ws.counters + ws.n_counters - 1);
}

void launch_int4_pack(const float* w, int64_t K, int64_t N, int64_t ldw, bool trans,
                      uint8_t* out, float* scales, cudaStream_t st) {
  IDEV_CHECK_ARG(K > 0 && K % 2 == 0 && N >= 0, "int4 pack: K must be even");
  if (N == 0) return;
  int4_pack_kernel<<<(unsigned)N, kThreads, 0, st>>>(w, K, N, ldw, trans, out, scales);
  IDEV_LAUNCHED();
}

void launch_argmax(const float* x, int64_t n, int64_t* out, cudaStream_t st) {
  IDEV_CHECK_ARG(n > 0, "argmax: empty input");
  Workspace& ws = workspace_for_current_device();
  const int blocks = (int)std::min<int64_t>(2 * sm_count(), (n + kThreads - 1) / kThreads);
  float* best_v = ws.partials;
  int64_t* best_i = reinterpret_cast<int64_t*>(ws.partials + ((blocks + 1) & ~1));
  argmax_kernel<<<blocks, kThreads, 0, st>>>(x, n, out, best_v, best_i,
                                             ws.counters + ws.n_counters - 2);
  IDEV_LAUNCHED();
}

void launch_decode_embed(const int64_t* tok, const int64_t* pos, const float* wte,
                         const float* wpe, float* x, int64_t H, int64_t vocab, int64_t max_pos,
                         int* err, cudaStream_t st) {
  launch_pdl(decode_embed_kernel, dim3((unsigned)((H + 255) / 256)), dim3(256), 0, st, tok, pos,
             wte, wpe, x, H, vocab, max_pos, err);
}

void launch_rows_embed(const int64_t* ids, int64_t n, int64_t pos0, const float* wte,
                       const float* wpe, float* x, int64_t H, int64_t vocab, int* err,
                       cudaStream_t st) {
  if (n <= 0) return;
  rows_embed_kernel<<<(unsigned)n, 256, 0, st>>>(ids, n, pos0, wte, wpe, x, H, vocab, err);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev

// ======================================================================
// Allocation-free GEMV entry point.
//
// Some callers cannot allocate device memory at all: code that runs inside a
// host framework which owns the whole device heap and forbids cudaMalloc
// during inference, allocator-less embedded runtimes, and real-time loops
// where an allocation (and the device synchronisation it can imply) is not
// allowed. inferc_dev_gemv needs a split-K scratch buffer that the library
// allocates lazily on first use; this variant instead takes its scratch from a
// fixed array compiled into the library, so a call allocates nothing.
// ======================================================================

namespace inferc_dev {
namespace {

constexpr size_t kNoAllocPartials = size_t(1) << 18;  // 256 Ki floats = 1 MiB
constexpr size_t kNoAllocCounters = 1024;

// Lives on every device that loads this library, until the process exits.
static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartials];
static __device__ __align__(256) unsigned int g_noalloc_counters[kNoAllocCounters];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_partials_ptr[kMaxDevices] = {};
unsigned int* g_noalloc_counters_ptr[kMaxDevices] = {};

// Device addresses of the two arrays for the current device. The array names
// are host-side stand-ins in host code, so the real addresses are looked up
// once per device, with that device current.
void noalloc_scratch(float** partials, unsigned int** counters) {
  int dev = 0;
  IDEV_CUDA(cudaGetDevice(&dev));
  IDEV_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "gemv_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_partials_ptr[dev] == nullptr) {
    void* p = nullptr;
    void* c = nullptr;
    IDEV_CUDA(cudaGetSymbolAddress(&p, g_noalloc_partials));
    IDEV_CUDA(cudaGetSymbolAddress(&c, g_noalloc_counters));
    g_noalloc_partials_ptr[dev] = static_cast<float*>(p);
    g_noalloc_counters_ptr[dev] = static_cast<unsigned int*>(c);
  }
  *partials = g_noalloc_partials_ptr[dev];
  *counters = g_noalloc_counters_ptr[dev];
}

}  // namespace
}  // namespace inferc_dev

extern "C" int inferc_dev_gemv_noalloc(const float* x, const float* w, const float* b,
                                       const float* resid, float* y, int64_t K, int64_t N,
                                       int act, void* stream) {
  using namespace inferc_dev;
  return guard([&] {
    IDEV_CHECK_ARG(K > 0 && K <= kMaxK, "gemv_noalloc: K must be in [1, 8192]");
    IDEV_CHECK_ARG(N >= 0 && (size_t)N <= kNoAllocPartials,
                   "gemv_noalloc: N exceeds the built-in scratch (max 262144 columns)");
    IDEV_CHECK_ARG(act >= 0 && act <= 3, "gemv_noalloc: unknown activation");
    if (N == 0) return;
    cudaStream_t st = as_stream(stream);
    GemvArgs g{};
    g.x = x; g.w = w; g.bias = b; g.resid = resid; g.y = y; g.K = K; g.N = N;
    g.alpha = 1.0f; g.beta = 1.0f; g.act = act;
    if (!(N % 4 == 0 && aligned16(w))) {  // scalar path: needs no scratch
      gemv_kn_scalar_kernel<<<(unsigned)((N + kWarps - 1) / kWarps), kThreads, 0, st>>>(g);
      IDEV_LAUNCHED();
      return;
    }
    float* partials = nullptr;
    unsigned int* counters = nullptr;
    noalloc_scratch(&partials, &counters);
    const int64_t tiles = (N + kColsPerCta - 1) / kColsPerCta;
    int64_t kps = 0;
    const int64_t splits = gemv_splits(K, N, kNoAllocPartials, kNoAllocCounters, &kps);
    // The counters start at zero (static storage) and the kernel's last CTA
    // per column tile puts its counter back to zero, so no clearing is needed.
    dim3 grid((unsigned)tiles, (unsigned)splits);
    gemv_kn_kernel<<<grid, kThreads, 0, st>>>(g, kps, (int)splits, partials, counters);
    IDEV_LAUNCHED();
  });
}
