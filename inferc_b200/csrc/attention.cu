// Fused multi-head attention (FusedAttention) and the decode-step attention
// over the device KV cache.
//
// FusedAttention (src/kernels/attention.cc:32-100) per (b, h):
//   P = softmax(where(mask, fill, scale * Q_h K_h^T)),  O_h = P V_h
// where a masked score is REPLACED by `fill` (not added to), scale =
// 1/sqrt(head_dim), and head h lives in columns [h*hd, (h+1)*hd) of the
// [B, S, H] tensors. The kernel never materialises the S x S scores: each CTA
// owns 128 query rows of one (b, h), streams 64-key tiles of K and V through
// shared memory and keeps a running (max, sum) per row (online softmax), so
// the HBM traffic is one read of Q, K, V and one write of O.
#include <cfloat>

#include "kernels.cuh"

namespace inferc_dev {
namespace {

constexpr int TQ = 128;  // query rows per CTA
constexpr int TKEYS = 64;  // keys per tile
constexpr int HD = 64;   // head dim of the fast kernel
constexpr int PAD = 68;  // padded row length of the Q, K and P tiles

__device__ __forceinline__ bool is_masked(const AttnArgs& a, int64_t b, int64_t h, int64_t i,
                                          int64_t j) {
  if (a.causal && j > i) return true;
  if (a.mask) return a.mask[b * a.ms[0] + h * a.ms[1] + i * a.ms[2] + j * a.ms[3]] != 0;
  return false;
}

// head_dim 64: a CTA owns TQ = 128 query rows of one (b, h) and streams
// 64-key tiles of K and V. 256 threads = 16 x 16 (tx, ty); thread (tx, ty)
// owns score rows i = ty + 16 r (r < 8) and key columns j = tx + 16 c (c < 4)
// of a tile, and output rows i with head dims [4 tx, 4 tx + 4). Q, K, V, P
// live in shared memory in natural row-major layout with rows padded to 68
// floats; the interleaved row ownership makes every 128-bit shared load
// either a broadcast or conflict free.
__global__ void __launch_bounds__(256, 2) attention_hd64_kernel(AttnArgs a) {
  extern __shared__ __align__(16) float smem[];
  float* Qs = smem;               // [TQ][PAD]
  float* Ks = Qs + TQ * PAD;      // [TKEYS][PAD]
  float* Vs = Ks + TKEYS * PAD;   // [TKEYS][HD]
  float* Ps = Vs + TKEYS * HD;    // [TQ][PAD]

  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t b = blockIdx.z, h = blockIdx.y, i0 = (int64_t)blockIdx.x * TQ;
  const float* Q = a.q + b * a.bstride_q + h * HD;
  const float* K = a.k + b * a.bstride_k + h * HD;
  const float* V = a.v + b * a.bstride_v + h * HD;

  for (int f = tid; f < TQ * HD / 4; f += 256) {
    const int r = f >> 4, d = (f & 15) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i0 + r < a.S) v = *reinterpret_cast<const float4*>(Q + (i0 + r) * a.ldq + d);
    *reinterpret_cast<float4*>(Qs + r * PAD + d) = v;
  }

  float m[8], l[8], o[8][4];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[r][c] = 0.f;
  }

  const int64_t ntiles = (a.S + TKEYS - 1) / TKEYS;
  for (int64_t t = 0; t < ntiles; ++t) {
    const int64_t j0 = t * TKEYS;
    __syncthreads();  // previous tile's Ks / Vs / Ps no longer in use
    for (int f = tid; f < TKEYS * HD / 4; f += 256) {
      const int r = f >> 4, d = (f & 15) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (j0 + r < a.S) {
        kv = *reinterpret_cast<const float4*>(K + (j0 + r) * a.ldk + d);
        vv = *reinterpret_cast<const float4*>(V + (j0 + r) * a.ldv + d);
      }
      *reinterpret_cast<float4*>(Ks + r * PAD + d) = kv;
      *reinterpret_cast<float4*>(Vs + r * HD + d) = vv;
    }
    __syncthreads();

    float s[8][4];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[r][c] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
      float4 kv[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * c) * PAD + d);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4 qv = *reinterpret_cast<const float4*>(Qs + (ty + 16 * r) * PAD + d);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s[r][c] = fmaf(qv.x, kv[c].x, s[r][c]);
          s[r][c] = fmaf(qv.y, kv[c].y, s[r][c]);
          s[r][c] = fmaf(qv.z, kv[c].z, s[r][c]);
          s[r][c] = fmaf(qv.w, kv[c].w, s[r][c]);
        }
      }
    }

#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int64_t i = i0 + ty + 16 * r;
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t j = j0 + tx + 16 * c;
        float v;
        if (j >= a.S) v = -INFINITY;  // beyond the sequence: no weight at all
        else if (i < a.S && is_masked(a, b, h, i, j)) v = a.fill;
        else v = a.scale * s[r][c];
        s[r][c] = v;
        tmax = fmaxf(tmax, v);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float mn = fmaxf(m[r], tmax);
      const float corr = expf(m[r] - mn);  // m = -inf on the first tile -> 0
      float ps = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float p = expf(s[r][c] - mn);
        Ps[(ty + 16 * r) * PAD + tx + 16 * c] = p;
        ps += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[r] = l[r] * corr + ps;
      m[r] = mn;
#pragma unroll
      for (int c = 0; c < 4; ++c) o[r][c] *= corr;
    }
    __syncthreads();
    const int jn = (int)((a.S - j0) < TKEYS ? (a.S - j0) : TKEYS);
#pragma unroll 2
    for (int j = 0; j < jn; j += 4) {
      float4 vv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) vv[q] = *reinterpret_cast<const float4*>(Vs + (j + q) * HD + tx * 4);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4 pv = *reinterpret_cast<const float4*>(Ps + (ty + 16 * r) * PAD + j);
        const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          o[r][0] = fmaf(pa[q], vv[q].x, o[r][0]);
          o[r][1] = fmaf(pa[q], vv[q].y, o[r][1]);
          o[r][2] = fmaf(pa[q], vv[q].z, o[r][2]);
          o[r][3] = fmaf(pa[q], vv[q].w, o[r][3]);
        }
      }
    }
  }

  float* O = a.out + b * a.bstride_o + h * HD;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int64_t i = i0 + ty + 16 * r;
    if (i >= a.S) continue;
    const float inv = 1.0f / l[r];
    *reinterpret_cast<float4*>(O + i * a.ldo + tx * 4) =
        make_float4(o[r][0] * inv, o[r][1] * inv, o[r][2] * inv, o[r][3] * inv);
  }
}

// Any head_dim <= 128, any alignment: one warp per query row, keys streamed
// one at a time with an online softmax.
__global__ void attention_generic_kernel(AttnArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t total = a.B * a.nH * a.S;
  if (row >= total) return;
  const int64_t i = row % a.S, h = (row / a.S) % a.nH, b = row / (a.S * a.nH);
  const float* q = a.q + b * a.bstride_q + i * a.ldq + h * a.hd;
  float qr[4], acc[4];
  for (int u = 0; u < 4; ++u) {
    const int64_t d = lane + 32 * u;
    qr[u] = d < a.hd ? q[d] : 0.f;
    acc[u] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int64_t j = 0; j < a.S; ++j) {
    const float* kr = a.k + b * a.bstride_k + j * a.ldk + h * a.hd;
    float dot = 0.f;
    for (int u = 0; u < 4; ++u) {
      const int64_t d = lane + 32 * u;
      if (d < a.hd) dot = fmaf(qr[u], kr[d], dot);
    }
    dot = warp_sum(dot);
    const float s = is_masked(a, b, h, i, j) ? a.fill : a.scale * dot;
    const float mn = fmaxf(m, s);
    const float corr = expf(m - mn), p = expf(s - mn);
    l = l * corr + p;
    m = mn;
    const float* vr = a.v + b * a.bstride_v + j * a.ldv + h * a.hd;
    for (int u = 0; u < 4; ++u) {
      const int64_t d = lane + 32 * u;
      acc[u] = acc[u] * corr + (d < a.hd ? p * vr[d] : 0.f);
    }
  }
  float* o = a.out + b * a.bstride_o + i * a.ldo + h * a.hd;
  for (int u = 0; u < 4; ++u) {
    const int64_t d = lane + 32 * u;
    if (d < a.hd) o[d] = acc[u] / l;
  }
}

// ---------------------------------------------------------------- decode

constexpr int kDecThreads = 128;

// One CTA per head: optional in-place KV append at position L-1, then
// s_j = (q . k_j) / sqrt(hd), p = softmax(s) (max, exp(s - max), * 1/sum as
// rt::Softmax does), out = sum_j p_j v_j.
__global__ void __launch_bounds__(kDecThreads)
    decode_attention_kernel(const float* __restrict__ q, const float* __restrict__ k_new,
                            const float* __restrict__ v_new, float* kc, float* vc,
                            float* __restrict__ out, int64_t hd, int64_t max_len,
                            const int64_t* len_dev, int64_t len_host) {
  extern __shared__ float sc[];  // [max_len] scores, then [kDecThreads] partials
  __shared__ float red[kDecThreads / 32];
  __shared__ float qs[128];
  const int64_t h = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t L = len_dev ? *len_dev : len_host;
  if (L <= 0 || L > max_len) return;
  float* kh = kc + h * max_len * hd;
  float* vh = vc + h * max_len * hd;
  if (tid < hd) {
    qs[tid] = q[h * hd + tid];
    if (k_new) {
      kh[(L - 1) * hd + tid] = k_new[h * hd + tid];
      vh[(L - 1) * hd + tid] = v_new[h * hd + tid];
    }
  }
  __syncthreads();
  const float sq = sqrtf((float)hd);
  for (int64_t j = wid; j < L; j += kDecThreads / 32) {
    const float* kr = kh + j * hd;
    float dot = 0.f;
    for (int64_t d = lane; d < hd; d += 32) dot = fmaf(qs[d], kr[d], dot);
    dot = warp_sum(dot);
    if (lane == 0) sc[j] = dot / sq;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int64_t j = tid; j < L; j += kDecThreads) mx = fmaxf(mx, sc[j]);
  mx = warp_max(mx);
  if (lane == 0) red[wid] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < kDecThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int64_t j = tid; j < L; j += kDecThreads) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[wid] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < kDecThreads / 32; ++w) sum += red[w];
  const float inv = 1.0f / sum;
  // out[d]: threads split the keys in two halves when hd <= 64.
  const int groups = hd <= 64 ? 2 : 1;
  const int64_t d = tid % (kDecThreads / groups);
  const int g = tid / (kDecThreads / groups);
  float acc = 0.f;
  if (d < hd) {
    const int64_t jb = g * ((L + 1) / 2), je = groups == 1 ? L : (g == 0 ? (L + 1) / 2 : L);
    for (int64_t j = (groups == 1 ? 0 : jb); j < je; ++j) acc = fmaf(sc[j] * inv, vh[j * hd + d], acc);
  }
  float* part = sc + max_len;
  part[tid] = acc;
  __syncthreads();
  if (tid < hd) {
    float r = part[tid];
    if (groups == 2) r += part[tid + kDecThreads / 2];
    out[h * hd + tid] = r;
  }
}

// Vectorised decode attention (head_dim % 4 == 0, head_dim <= 128): scores
// with one thread per key (a whole K row of independent 128-bit loads), then
// out = sum_j p_j v_j with threads split into (float4 of head dims) x (key
// groups) and a fixed-order reduction over the groups.
__global__ void __launch_bounds__(kDecThreads)
    decode_attention_vec_kernel(const float* __restrict__ q, const float* __restrict__ k_new,
                                const float* __restrict__ v_new, float* kc, float* vc,
                                float* __restrict__ out, int64_t hd, int64_t max_len,
                                const int64_t* len_dev, int64_t len_host) {
  extern __shared__ __align__(16) float dsm[];  // [max_len] scores | [kDecThreads*4] partials
  __shared__ __align__(16) float qs[128];
  __shared__ float red[kDecThreads / 32];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t h = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t L = len_dev ? *len_dev : len_host;
  if (L <= 0 || L > max_len) return;
  float* kh = kc + h * max_len * hd;
  float* vh = vc + h * max_len * hd;
  float* sc = dsm;
  if (tid < hd) {
    qs[tid] = q[h * hd + tid];
    if (k_new) {
      kh[(L - 1) * hd + tid] = k_new[h * hd + tid];
      vh[(L - 1) * hd + tid] = v_new[h * hd + tid];
    }
  }
  __syncthreads();
  const int hd4 = (int)(hd / 4);
  const float sq = sqrtf((float)hd);
  const float4* q4 = reinterpret_cast<const float4*>(qs);
  for (int64_t j = tid; j < L; j += kDecThreads) {
    const float4* kr = reinterpret_cast<const float4*>(kh + j * hd);
    float dot = 0.f;
#pragma unroll 8
    for (int d = 0; d < hd4; ++d) {
      const float4 kv = kr[d], qv = q4[d];
      dot = fmaf(qv.x, kv.x, dot);
      dot = fmaf(qv.y, kv.y, dot);
      dot = fmaf(qv.z, kv.z, dot);
      dot = fmaf(qv.w, kv.w, dot);
    }
    sc[j] = dot / sq;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int64_t j = tid; j < L; j += kDecThreads) mx = fmaxf(mx, sc[j]);
  mx = warp_max(mx);
  if (lane == 0) red[wid] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < kDecThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int64_t j = tid; j < L; j += kDecThreads) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[wid] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < kDecThreads / 32; ++w) sum += red[w];
  const float inv = 1.0f / sum;
  const int groups = kDecThreads / hd4;  // key groups
  const int d4 = tid % hd4, g = tid / hd4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (g < groups) {
#pragma unroll 4
    for (int64_t j = g; j < L; j += groups) {
      const float p = sc[j] * inv;
      const float4 vv = reinterpret_cast<const float4*>(vh + j * hd)[d4];
      acc.x = fmaf(p, vv.x, acc.x);
      acc.y = fmaf(p, vv.y, acc.y);
      acc.z = fmaf(p, vv.z, acc.z);
      acc.w = fmaf(p, vv.w, acc.w);
    }
  }
  float4* part = reinterpret_cast<float4*>(dsm + max_len + ((max_len & 3) ? 4 - (max_len & 3) : 0));
  part[tid] = acc;
  __syncthreads();
  if (tid < hd4) {
    float4 r = part[tid];
    for (int gg = 1; gg < groups; ++gg) {
      const float4 t = part[gg * hd4 + tid];
      r.x += t.x; r.y += t.y; r.z += t.z; r.w += t.w;
    }
    reinterpret_cast<float4*>(out + h * hd)[tid] = r;
  }
}

__global__ void kv_append_kernel(const float* __restrict__ k_new, const float* __restrict__ v_new,
                                 int64_t ld_new, float* kc, float* vc, int64_t heads, int64_t hd,
                                 int64_t max_len, const int64_t* pos_dev, int64_t pos_host,
                                 int64_t n) {
  const int64_t pos = pos_dev ? *pos_dev : pos_host;
  const int64_t total = n * heads * hd;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = e % hd, h = (e / hd) % heads, r = e / (hd * heads);
    if (pos + r >= max_len || pos + r < 0) continue;
    const int64_t dst = (h * max_len + pos + r) * hd + d;
    kc[dst] = k_new[r * ld_new + h * hd + d];
    vc[dst] = v_new[r * ld_new + h * hd + d];
  }
}

}  // namespace

void launch_attention(const AttnArgs& a, cudaStream_t st) {
  if (a.B <= 0 || a.S <= 0 || a.nH <= 0) return;
  IDEV_CHECK_ARG(a.hd > 0 && a.hd <= 128, "FusedAttention: head_dim must be in [1, 128]");
  if (attention_tc_supported(a) && attention_tc_enabled()) {
    launch_attention_tc(a, st);
    return;
  }
  IDEV_CHECK_ARG(a.so.hi == nullptr, "FusedAttention: fp16 split output needs the tensor-core path");
  const bool fast = a.hd == HD && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
                    aligned16(a.out) && a.ldq % 4 == 0 && a.ldk % 4 == 0 && a.ldv % 4 == 0 &&
                    a.ldo % 4 == 0 && a.bstride_q % 4 == 0 && a.bstride_k % 4 == 0 &&
                    a.bstride_v % 4 == 0 && a.bstride_o % 4 == 0;
  if (fast) {
    const size_t smem = (size_t)(TQ * PAD + TKEYS * PAD + TKEYS * HD + TQ * PAD) * sizeof(float);
    // Per device and cheap; set on every call so that every device in the
    // process is configured.
    IDEV_CUDA(cudaFuncSetAttribute(attention_hd64_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)((a.S + TQ - 1) / TQ), (unsigned)a.nH, (unsigned)a.B);
    attention_hd64_kernel<<<grid, 256, smem, st>>>(a);
  } else {
    const int64_t rows = a.B * a.nH * a.S;
    attention_generic_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a);
  }
  IDEV_LAUNCHED();
}

void launch_kv_append(const float* k_new, const float* v_new, int64_t ld_new, float* kc,
                      float* vc, int64_t heads, int64_t hd, int64_t max_len,
                      const int64_t* pos_dev, int64_t pos_host, int64_t n, cudaStream_t st) {
  const int64_t total = n * heads * hd;
  if (total <= 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 4096);
  kv_append_kernel<<<blocks, 256, 0, st>>>(k_new, v_new, ld_new, kc, vc, heads, hd, max_len,
                                           pos_dev, pos_host, n);
  IDEV_LAUNCHED();
}

void launch_decode_attention(const float* q, const float* k_new, const float* v_new, float* kc,
                             float* vc, float* out, int64_t heads, int64_t hd, int64_t max_len,
                             const int64_t* len_dev, int64_t len_host, cudaStream_t st) {
  IDEV_CHECK_ARG(hd > 0 && hd <= 128, "decode attention: head_dim must be in [1, 128]");
  IDEV_CHECK_ARG(max_len > 0 && max_len <= 8192, "decode attention: max_len must be <= 8192");
  const bool vec = hd % 4 == 0 && aligned16(q) && aligned16(kc) && aligned16(vc) &&
                   aligned16(out) && (k_new == nullptr || (aligned16(k_new) && aligned16(v_new)));
  if (vec) {
    const size_t smem = (size_t)(max_len + 4 + 4 * kDecThreads) * sizeof(float);
    launch_pdl(decode_attention_vec_kernel, dim3((unsigned)heads), dim3(kDecThreads), smem, st, q,
               k_new, v_new, kc, vc, out, hd, max_len, len_dev, len_host);
    return;
  }
  const size_t smem = (size_t)(max_len + kDecThreads) * sizeof(float);
  decode_attention_kernel<<<(unsigned)heads, kDecThreads, smem, st>>>(
      q, k_new, v_new, kc, vc, out, hd, max_len, len_dev, len_host);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
