// Standalone pointwise ops of the plan (Gelu, GeluTanh, Softmax) and the
// Gemm C-broadcast prefill. On the fused paths these are folded into GEMM /
// GEMV epilogues and attention; the C ABI still exposes them as ops.
#include "kernels.cuh"

namespace inferc_dev {
namespace {

__global__ void act_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, int act) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = apply_act(x[i], act);
}

// rt::Softmax (activation.cc:75-95): max from -inf, exp(x - max), sum, * 1/sum.
// One block per row.
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t cols) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * cols;
  float* yr = y + (int64_t)blockIdx.x * cols;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) m = fmaxf(m, xr[j]);
  m = warp_max(m);
  if (lane == 0) red[wid] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < nw; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
    const float e = expf(xr[j] - m);
    yr[j] = e;
    s += e;
  }
  s = warp_sum(s);
  if (lane == 0) red[wid] = s;
  __syncthreads();
  s = 0.f;
  for (int w = 0; w < nw; ++w) s += red[w];
  const float inv = 1.0f / s;
  for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) yr[j] *= inv;
}

__global__ void fill_rows_kernel(float* y, const float* c, int64_t c_len, int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = c == nullptr ? 0.f : (c_len == total ? c[i] : c_len == N ? c[i % N] : c[0]);
}

unsigned grid_for(int64_t n) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16));
}

}  // namespace

void launch_act(const float* x, float* y, int64_t n, int act, cudaStream_t st) {
  if (n <= 0) return;
  act_kernel<<<grid_for(n), 256, 0, st>>>(x, y, n, act);
  IDEV_LAUNCHED();
}

void launch_softmax(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return;
  softmax_kernel<<<(unsigned)rows, 256, 0, st>>>(x, y, cols);
  IDEV_LAUNCHED();
}

void launch_fill_rows(float* y, const float* c, int64_t c_len, int64_t M, int64_t N,
                      cudaStream_t st) {
  if (M * N <= 0) return;
  fill_rows_kernel<<<grid_for(M * N), 256, 0, st>>>(y, c, c_len, M, N);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
