// FusedLayerNorm on B200: one warp per row, the row held in registers as
// 128-bit vectors, mean and biased variance by warp-shuffle reductions
// (two passes over registers, one read and one write of HBM per element).
// Restates rt::LayerNorm (src/kernels/activation.cc:134-148): centred row,
// var = mean(xc^2), inv = 1/sqrtf(var+eps), y = (xc*inv)*gamma + beta.
#include "kernels.cuh"

namespace inferc_dev {
namespace {

constexpr int kWarpsPerBlock = 8;

// Normalises one row held as VPT float4 per lane; writes y and, when
// sp.hi is set, the row's fp16 hi / lo split for the split-fp16 GEMM.
template <int VPT>
__device__ __forceinline__ void ln_row_regs(float4 (&v)[VPT], const float* __restrict__ gamma,
                                            const float* __restrict__ beta, float* __restrict__ y,
                                            int64_t feat, float eps, int lane,
                                            const SplitOut& sp, int64_t row) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  s = warp_sum(s);
  const float mean = s / (float)feat;
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
    sq += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
  }
  sq = warp_sum(sq);
  const float inv = 1.0f / sqrtf(sq / (float)feat + eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  float4* y4 = reinterpret_cast<float4*>(y);
  bool bad = false;
  uint2* h2 = sp.hi ? reinterpret_cast<uint2*>(sp.hi + row * sp.ld) : nullptr;
  uint2* l2 = sp.hi ? reinterpret_cast<uint2*>(sp.lo + row * sp.ld) : nullptr;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    const float4 g = __ldg(g4 + c), b = __ldg(b4 + c);
    float4 o;
    o.x = (v[i].x * inv) * g.x + b.x;
    o.y = (v[i].y * inv) * g.y + b.y;
    o.z = (v[i].z * inv) * g.z + b.z;
    o.w = (v[i].w * inv) * g.w + b.w;
    y4[c] = o;
    if (h2) {
      uint2 h, l;
      h.x = split_pair(o.x, o.y, l.x, bad);
      h.y = split_pair(o.z, o.w, l.y, bad);
      h2[c] = h;
      l2[c] = l;
    }
  }
  if (bad) atomicExch(sp.range, 1);
}

template <int VPT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    layernorm_warp_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                          const float* __restrict__ beta, float* y, int64_t rows, float eps,
                          SplitOut sp) {
  pdl_launch_dependents();
  pdl_wait();  // x comes from the previous kernel
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t feat = 128 * VPT;
  const float4* x4 = reinterpret_cast<const float4*>(x + row * feat);
  float4 v[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) v[i] = x4[lane + 32 * i];
  ln_row_regs<VPT>(v, gamma, beta, y + row * feat, feat, eps, lane, sp, row);
}

// Generic path (any feat): one block per row, three sweeps through L1/L2.
__global__ void layernorm_block_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                       const float* __restrict__ beta, float* y, int64_t feat,
                                       float eps) {
  __shared__ float red[32];
  __shared__ float bcast;
  const float* xr = x + (int64_t)blockIdx.x * feat;
  float* yr = y + (int64_t)blockIdx.x * feat;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    if (lane == 0) red[wid] = v;
    __syncthreads();
    if (wid == 0) {
      float t = lane < nw ? red[lane] : 0.0f;
      t = warp_sum(t);
      if (lane == 0) bcast = t;
    }
    __syncthreads();
    const float r = bcast;
    __syncthreads();
    return r;
  };
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < feat; i += blockDim.x) s += xr[i];
  const float mean = block_sum(s) / (float)feat;
  float sq = 0.0f;
  for (int64_t i = threadIdx.x; i < feat; i += blockDim.x) {
    const float d = xr[i] - mean;
    sq += d * d;
  }
  const float inv = 1.0f / sqrtf(block_sum(sq) / (float)feat + eps);
  // x and y may alias: every element is read before it is written by the
  // same thread in this loop, and earlier loops only read.
  for (int64_t i = threadIdx.x; i < feat; i += blockDim.x)
    yr[i] = ((xr[i] - mean) * inv) * gamma[i] + beta[i];
}

template <int VPT>
void launch_warp(const float* x, const float* g, const float* b, float* y, int64_t rows,
                 float eps, const SplitOut& sp, cudaStream_t st) {
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  launch_pdl(layernorm_warp_kernel<VPT>, dim3((unsigned)blocks), dim3(kWarpsPerBlock * 32), 0, st,
             x, g, b, y, rows, eps, sp);
}

// Encoder embedding + LayerNorm: one warp per token.
template <int VPT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    embed_ln_kernel(const int64_t* __restrict__ ids, const int64_t* __restrict__ mask,
                    const float* __restrict__ word, const float* __restrict__ pos, int64_t vocab,
                    const float* __restrict__ gamma, const float* __restrict__ beta,
                    float* __restrict__ y, uint8_t* __restrict__ cond, int64_t BS, int64_t S,
                    float eps, int* err_flag, SplitOut sp) {
  pdl_launch_dependents();
  pdl_wait();  // y may still be read by the previous kernel
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (t >= BS) return;
  constexpr int64_t feat = 128 * VPT;
  int64_t id = ids[t];
  if (id < 0) id += vocab;  // Gather wraps negative indices (embedding.cc:61-62)
  if (lane == 0 && cond) cond[t] = mask[t] == 0 ? 1 : 0;
  float4* y4 = reinterpret_cast<float4*>(y + t * feat);
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicExch(err_flag, 1);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      y4[lane + 32 * i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (sp.hi) {
        reinterpret_cast<uint2*>(sp.hi + t * sp.ld)[lane + 32 * i] = make_uint2(0, 0);
        reinterpret_cast<uint2*>(sp.lo + t * sp.ld)[lane + 32 * i] = make_uint2(0, 0);
      }
    }
    return;
  }
  const float4* w4 = reinterpret_cast<const float4*>(word + id * feat);
  const float4* p4 = reinterpret_cast<const float4*>(pos + (t % S) * feat);
  float4 v[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const float4 a = __ldg(w4 + lane + 32 * i), b = __ldg(p4 + lane + 32 * i);
    v[i] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  }
  ln_row_regs<VPT>(v, gamma, beta, y + t * feat, feat, eps, lane, sp, t);
}

}  // namespace

void launch_layernorm(const float* x, const float* g, const float* b, float* y, int64_t rows,
                      int64_t feat, float eps, cudaStream_t st, const SplitOut& sp) {
  if (rows <= 0) return;
  const bool vec = aligned16(x) && aligned16(y) && aligned16(g) && aligned16(b);
  IDEV_CHECK_ARG(!sp.hi || (vec && feat % 128 == 0 && feat <= 1024 && sp.lo && sp.range &&
                            aligned16(sp.hi) && aligned16(sp.lo) && sp.ld % 8 == 0),
                 "LayerNorm: fp16 split output needs feat % 128 == 0, <= 1024, aligned planes");
  if (vec && feat % 128 == 0 && feat <= 1024) {
    switch (feat / 128) {
      case 1: launch_warp<1>(x, g, b, y, rows, eps, sp, st); break;
      case 2: launch_warp<2>(x, g, b, y, rows, eps, sp, st); break;
      case 3: launch_warp<3>(x, g, b, y, rows, eps, sp, st); break;
      case 4: launch_warp<4>(x, g, b, y, rows, eps, sp, st); break;
      case 5: launch_warp<5>(x, g, b, y, rows, eps, sp, st); break;
      case 6: launch_warp<6>(x, g, b, y, rows, eps, sp, st); break;
      case 7: launch_warp<7>(x, g, b, y, rows, eps, sp, st); break;
      default: launch_warp<8>(x, g, b, y, rows, eps, sp, st); break;
    }
  } else {
    layernorm_block_kernel<<<(unsigned)rows, 256, 0, st>>>(x, g, b, y, feat, eps);
  }
  IDEV_LAUNCHED();
}

void launch_embed_layernorm(const int64_t* ids, const int64_t* mask, const float* word,
                            const float* pos, int64_t vocab, const float* g, const float* b,
                            float* y, uint8_t* cond, int64_t B, int64_t S, int64_t H, float eps,
                            int* err_flag, cudaStream_t st, const SplitOut& sp) {
  IDEV_CHECK_ARG(H % 128 == 0 && H <= 1024, "encoder hidden size must be a multiple of 128, <= 1024");
  const int64_t BS = B * S;
  const unsigned blocks = (unsigned)((BS + kWarpsPerBlock - 1) / kWarpsPerBlock);
#define IDEV_EMB(V)                                                                         \
  launch_pdl(embed_ln_kernel<V>, dim3(blocks), dim3(kWarpsPerBlock * 32), 0, st, ids, mask, word, \
             pos, vocab, g, b, y, cond, BS, S, eps, err_flag, sp)
  switch (H / 128) {
    case 1: IDEV_EMB(1); break;
    case 2: IDEV_EMB(2); break;
    case 3: IDEV_EMB(3); break;
    case 4: IDEV_EMB(4); break;
    case 5: IDEV_EMB(5); break;
    case 6: IDEV_EMB(6); break;
    case 7: IDEV_EMB(7); break;
    default: IDEV_EMB(8); break;
  }
#undef IDEV_EMB
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
