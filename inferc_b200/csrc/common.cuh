// Shared device helpers and host-side error plumbing for libinferc_b200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <stdexcept>
#include <string>
#include <utility>

#include "../../include/inferc_dev.h"

namespace inferc_dev {

// ------------------------------------------------------------------ errors
// Every extern "C" entry point converts exceptions to a status code and keeps
// the message for inferc_dev_last_error_string() (per host thread).
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string& msg);

#define IDEV_CHECK_ARG(cond, msg)                                        \
  do {                                                                   \
    if (!(cond)) throw ::inferc_dev::Error(INFERC_ERR_INVALID, (msg));   \
  } while (0)

#define IDEV_CUDA(call)                                                           \
  do {                                                                            \
    cudaError_t e_ = (call);                                                      \
    if (e_ != cudaSuccess)                                                        \
      throw ::inferc_dev::Error(INFERC_ERR_CUDA, std::string(#call " failed: ") + \
                                                     cudaGetErrorString(e_));     \
  } while (0)

// Launch-error check after a <<<>>> launch.
#define IDEV_LAUNCHED() IDEV_CUDA(cudaGetLastError())

template <typename Fn>
int guard(Fn&& fn) {
  try {
    fn();
    return INFERC_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return INFERC_ERR_OOM;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return INFERC_ERR_INVALID;
  }
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------ device
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch (PDL). A kernel launched with the
// programmatic-serialization attribute may start while its predecessor in the
// stream is still running; everything before pdl_wait() must not read data
// the predecessor writes. pdl_wait() blocks until the predecessor grid has
// completed and its memory is visible; without the attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches `kernel` with the programmatic-serialization attribute.
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess)
    throw Error(INFERC_ERR_CUDA, std::string("cudaLaunchKernelEx failed: ") + cudaGetErrorString(e));
}

// Activation codes shared by the GEMM / GEMV epilogues.
enum Act : int { ACT_NONE = 0, ACT_GELU_ERF = 1, ACT_GELU_TANH = 2, ACT_RELU = 3 };

// Exact erf GELU: v * 0.5 * (1 + erf(v / sqrt(2))).
__device__ __forceinline__ float gelu_erf(float v) {
  return v * 0.5f * (1.0f + erff(v * 0.70710678118654752440f));
}

// GPT-2 tanh GELU: 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))).
__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case ACT_GELU_ERF: return gelu_erf(v);
    case ACT_GELU_TANH: return gelu_tanh(v);
    case ACT_RELU: return v > 0.0f ? v : 0.0f;
    default: return v;
  }
}

// Epilogue description: y = act(alpha*acc + beta*bias_term + resid[row,col]).
// bias_mode: 0 none, 1 per column (bias[col]), 2 scalar (bias[0]),
// 3 full matrix (bias[row*ldb + col]).
struct Epilogue {
  float alpha = 1.0f;
  float beta = 1.0f;
  const float* bias = nullptr;
  int bias_mode = 0;
  int64_t ldbias = 0;
  const float* resid = nullptr;
  int64_t ldr = 0;
  int act = ACT_NONE;
  // CUDA-core GEMM only: when set, the kernel runs only if *run_if != 0 (a
  // device flag raised by an earlier kernel), else it returns at once. The
  // op-level split-fp16 GEMM uses it to queue its own fallback.
  const int* run_if = nullptr;
};

__device__ __forceinline__ float epilogue_apply(const Epilogue& e, float acc, int64_t row,
                                                int64_t col) {
  float v = e.alpha * acc;
  if (e.bias_mode == 1) v += e.beta * e.bias[col];
  else if (e.bias_mode == 2) v += e.beta * e.bias[0];
  else if (e.bias_mode == 3) v += e.beta * e.bias[row * e.ldbias + col];
  if (e.resid) v += e.resid[row * e.ldr + col];
  return apply_act(v, e.act);
}

// fp32 -> fp16 hi / lo planes for the split-fp16 GEMM (gemm_f16s.cu):
// x = hi + lo with hi = fp16_rn(x), lo = fp16_rn(x - hi). A destination
// that is null writes nothing. `range` is set to 1 by any value fp16 cannot
// carry (|x| >= 65520, inf, NaN), which invalidates the split.
struct SplitOut {
  uint16_t* hi = nullptr;
  uint16_t* lo = nullptr;
  int64_t ld = 0;     // row stride of both planes (elements)
  int* range = nullptr;
};

__device__ __forceinline__ uint32_t split_pair(float a, float b, uint32_t& lo_bits, bool& bad) {
  bad |= !(fabsf(a) < 65520.f) || !(fabsf(b) < 65520.f);
  uint32_t h, l;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));
  const float ha = __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
  const float hb = __half2float(__ushort_as_half((unsigned short)(h >> 16)));
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(l) : "f"(b - hb), "f"(a - ha));
  lo_bits = l;
  return h;
}

}  // namespace inferc_dev
