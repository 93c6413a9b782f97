// int4 per-row-scale GEMV entry point.
//
// Restates scalar_int4_gemv_perRow (bench/amx/int4_gemv_amx.cc:258-271):
//   y[r] = sum_k (s_r * (q[r,k] - 8)) * x[k]
// with W [N, K/2] bytes, byte r*(K/2)+k/2 holding even k in the low nibble
// and odd k in the high nibble. Matrices with K % 32 == 0, K <= 4096 and
// 16-byte aligned W and x run on the tensor cores (gemv_int4_tc.cu), all of
// a call's matrices in one launch pair; any other shape runs a one-thread-
// per-row kernel. Both compute the sum in fp32-accurate arithmetic (the
// reference sums in double), so results agree to fp32 rounding.
#include <vector>

#include "kernels.cuh"

namespace inferc_dev {
namespace {

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

}  // namespace

bool gemv_int4_tc_ok(const InfercInt4Gemv& d);
void launch_gemv_int4_tc(const InfercInt4Gemv* const* ds, int n, cudaStream_t st);

void launch_gemv_int4(const InfercInt4Gemv* ds, int count, cudaStream_t st) {
  IDEV_CHECK_ARG(count >= 0 && (count == 0 || ds != nullptr), "int4 GEMV: bad descriptor list");
  std::vector<const InfercInt4Gemv*> tc;
  for (int i = 0; i < count; ++i) {
    const InfercInt4Gemv& d = ds[i];
    IDEV_CHECK_ARG(d.k > 0 && d.k % 2 == 0 && d.n >= 0, "int4 GEMV: K must be even and positive");
    IDEV_CHECK_ARG(d.n == 0 || (d.w && d.scales && d.x && d.y), "int4 GEMV: null pointer");
    if (d.n == 0) continue;
    if (gemv_int4_tc_ok(d)) {
      tc.push_back(&d);
      continue;
    }
    gemv_int4_scalar_kernel<<<(unsigned)((d.n + 255) / 256), 256, 0, st>>>(d);
    IDEV_LAUNCHED();
  }
  if (!tc.empty()) launch_gemv_int4_tc(tc.data(), (int)tc.size(), st);
}

}  // namespace inferc_dev
