// Device kernels for the graph's glue ops (the reference's elementwise.cc,
// movement.cc, embedding.cc and ReduceMean), used by the device executor so
// that an optimized plan runs with every tensor that depends on the inputs on
// the GPU:
//   - broadcast binary ops (Add, Sub, Mul, Div, Pow on fp32 / int64; Equal on
//     any integer, bool or fp32 pair, compared as int64 as the reference does),
//   - Where, unary fp32 ops, Cast,
//   - one strided copy for Transpose, Expand, Slice, Split and Concat,
//   - Gather along any axis (out-of-range indices raise a device flag),
//   - mean over the trailing elements of each row (ReduceMean after moving the
//     reduced axes last), and a fill for ConstantOfShape.
// Shapes arrive collapsed by the host (adjacent axes merged where every
// operand is contiguous across them), so the common cases - a residual Add
// of equal shapes, a bias Add over the last axis - reach the vectorised
// rank-1 / rank-2 paths.
#include "glue.cuh"

namespace inferc_dev {
namespace {

constexpr int kThreads = 256;

inline unsigned blocks_for(int64_t n, int64_t per_thread = 1) {
  const int64_t b = (n + kThreads * per_thread - 1) / (kThreads * per_thread);
  return (unsigned)std::min<int64_t>(std::max<int64_t>(b, 1), 148 * 64);
}

// Offset of linear output index i in an operand with per-axis strides s.
__device__ __forceinline__ int64_t bcast_offset(int64_t i, const GlueShape& g, const int64_t* s) {
  int64_t off = 0;
  for (int d = g.rank - 1; d >= 0; --d) {
    const int64_t c = i % g.shape[d];
    i /= g.shape[d];
    off += c * s[d];
  }
  return off;
}

template <typename T>
__device__ __forceinline__ T bin_apply(int op, T x, T y) {
  switch (op) {
    case GLUE_ADD: return x + y;
    case GLUE_SUB: return x - y;
    case GLUE_MUL: return x * y;
    case GLUE_DIV: return x / y;
    default: return (T)pow((double)x, (double)y);  // GLUE_POW, as the reference (double pow)
  }
}

template <typename T>
__global__ void binary_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                              T* __restrict__ out, GlueShape g) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < g.n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = bin_apply<T>(op, a[bcast_offset(i, g, g.s0)], b[bcast_offset(i, g, g.s1)]);
}

// fp32 Add / Sub / Mul / Div with rank <= 2 after collapsing and a last axis
// of stride 1 (or 0) in both operands and a multiple of 4 long: 4 elements
// per thread with one index split.
__global__ void binary_f32x4_kernel(int op, const float* __restrict__ a,
                                    const float* __restrict__ b, float* __restrict__ out,
                                    GlueShape g) {
  const int64_t cols = g.shape[g.rank - 1];
  const int64_t n4 = g.n / 4;
  const int64_t sa0 = g.rank == 2 ? g.s0[0] : 0, sb0 = g.rank == 2 ? g.s1[0] : 0;
  const int64_t sa1 = g.s0[g.rank - 1], sb1 = g.s1[g.rank - 1];
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n4;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = 4 * q;
    const int64_t r = i / cols, c = i - r * cols;
    float4 x, y;
    if (sa1) x = *reinterpret_cast<const float4*>(a + r * sa0 + c);
    else x = make_float4(a[r * sa0], a[r * sa0], a[r * sa0], a[r * sa0]);
    if (sb1) y = *reinterpret_cast<const float4*>(b + r * sb0 + c);
    else y = make_float4(b[r * sb0], b[r * sb0], b[r * sb0], b[r * sb0]);
    *reinterpret_cast<float4*>(out + i) =
        make_float4(bin_apply<float>(op, x.x, y.x), bin_apply<float>(op, x.y, y.y),
                    bin_apply<float>(op, x.z, y.z), bin_apply<float>(op, x.w, y.w));
  }
}

__device__ __forceinline__ int64_t read_as_i64(const void* p, int dt, int64_t i) {
  switch (dt) {
    case 7: return reinterpret_cast<const int64_t*>(p)[i];
    case 6: return reinterpret_cast<const int32_t*>(p)[i];
    case 1: return (int64_t)reinterpret_cast<const float*>(p)[i];
    default: return reinterpret_cast<const uint8_t*>(p)[i] ? 1 : 0;  // bool / uint8
  }
}

__global__ void equal_kernel(const void* a, int da, const void* b, int db,
                             uint8_t* __restrict__ out, GlueShape g) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < g.n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = read_as_i64(a, da, bcast_offset(i, g, g.s0)) ==
             read_as_i64(b, db, bcast_offset(i, g, g.s1));
}

template <typename T>
__global__ void where_kernel(const uint8_t* __restrict__ c, const T* __restrict__ x,
                             const T* __restrict__ y, T* __restrict__ out, GlueShape g) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < g.n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = c[bcast_offset(i, g, g.s0)] ? x[bcast_offset(i, g, g.s1)]
                                         : y[bcast_offset(i, g, g.s2)];
}

__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y,
                             int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    float r;
    switch (op) {
      case GLUE_SQRT: r = sqrtf(v); break;
      case GLUE_ERF: r = erff(v); break;
      case GLUE_RELU: r = v > 0.f ? v : 0.f; break;
      case GLUE_TANH: r = tanhf(v); break;
      case GLUE_NEG: r = -v; break;
      default: r = fabsf(v); break;  // GLUE_ABS
    }
    y[i] = r;
  }
}

template <typename From, typename To>
__global__ void cast_kernel(const From* __restrict__ x, To* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = (To)x[i];
}

__global__ void bool_to_f32_kernel(const uint8_t* __restrict__ x, float* __restrict__ y,
                                   int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = x[i] ? 1.0f : 0.0f;
}

// out[out_off + sum c_d os_d] = in[in_off + sum c_d is_d] over the shape.
template <typename T>
__global__ void strided_copy_kernel(const T* __restrict__ in, T* __restrict__ out,
                                    GlueShape g) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < g.n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i, io = g.off0, oo = g.off1;
    for (int d = g.rank - 1; d >= 0; --d) {
      const int64_t c = r % g.shape[d];
      r /= g.shape[d];
      io += c * g.s0[d];
      oo += c * g.s1[d];
    }
    out[oo] = in[io];
  }
}

// out[o, k, :] = data[o, idx[k], :] (slices of `slice` elements of T).
template <typename T>
__global__ void gather_kernel(const T* __restrict__ data, const void* __restrict__ idx,
                              int idx64, T* __restrict__ out, int64_t outer, int64_t axis_dim,
                              int64_t n_idx, int64_t slice, int* __restrict__ err) {
  const int64_t n = outer * n_idx * slice;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i % slice, ok_ = (i / slice);
    const int64_t k = ok_ % n_idx, o = ok_ / n_idx;
    int64_t j = idx64 ? reinterpret_cast<const int64_t*>(idx)[k]
                      : (int64_t)reinterpret_cast<const int32_t*>(idx)[k];
    if (j < 0) j += axis_dim;
    if (j < 0 || j >= axis_dim) {
      atomicExch(err, 1);
      out[i] = T(0);
      continue;
    }
    out[i] = data[(o * axis_dim + j) * slice + s];
  }
}

// One warp per row: y[r] = mean(x[r, :cols]) (fp32, sequential per lane then
// a shuffle tree).
__global__ void row_mean_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                                int64_t cols) {
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  float s = 0.f;
  for (int64_t c = lane; c < cols; c += 32) s += x[w * cols + c];
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) y[w] = s / (float)cols;
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ out, T v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = v;
}

}  // namespace

void collapse_shape(GlueShape& g, int operands) {
  // Merge axis d into d-1 when every operand steps contiguously across them.
  int64_t* s[3] = {g.s0, g.s1, g.s2};
  int r = 0;
  for (int d = 0; d < g.rank; ++d) {
    if (g.shape[d] == 1) continue;  // size-1 axes never move an offset
    if (r > 0) {
      bool merge = true;
      for (int k = 0; k < operands; ++k)
        merge &= s[k][r - 1] == s[k][d] * g.shape[d];
      if (merge) {
        g.shape[r - 1] *= g.shape[d];
        for (int k = 0; k < operands; ++k) s[k][r - 1] = s[k][d];
        continue;
      }
    }
    g.shape[r] = g.shape[d];
    for (int k = 0; k < operands; ++k) s[k][r] = s[k][d];
    ++r;
  }
  if (r == 0) {  // a single element
    g.shape[0] = 1;
    for (int k = 0; k < operands; ++k) s[k][0] = 0;
    r = 1;
  }
  g.rank = r;
}

void launch_glue_binary(int op, int dt, const void* a, const void* b, void* out, GlueShape g,
                        cudaStream_t st) {
  if (g.n == 0) return;
  collapse_shape(g, 2);
  if (dt == 1) {
    const float* fa = static_cast<const float*>(a);
    const float* fb = static_cast<const float*>(b);
    float* fo = static_cast<float*>(out);
    const int64_t cols = g.shape[g.rank - 1];
    const bool vec = op != GLUE_POW && g.rank <= 2 && cols % 4 == 0 &&
                     (g.s0[g.rank - 1] == 1 || g.s0[g.rank - 1] == 0) &&
                     (g.s1[g.rank - 1] == 1 || g.s1[g.rank - 1] == 0) &&
                     (g.rank == 1 || (g.s0[0] % 4 == 0 && g.s1[0] % 4 == 0)) &&
                     aligned16(fa) && aligned16(fb) && aligned16(fo);
    if (vec) {
      binary_f32x4_kernel<<<blocks_for(g.n / 4), kThreads, 0, st>>>(op, fa, fb, fo, g);
    } else {
      binary_kernel<float><<<blocks_for(g.n), kThreads, 0, st>>>(op, fa, fb, fo, g);
    }
  } else {
    binary_kernel<int64_t><<<blocks_for(g.n), kThreads, 0, st>>>(
        op, static_cast<const int64_t*>(a), static_cast<const int64_t*>(b),
        static_cast<int64_t*>(out), g);
  }
  IDEV_LAUNCHED();
}

void launch_glue_equal(const void* a, int da, const void* b, int db, uint8_t* out, GlueShape g,
                       cudaStream_t st) {
  if (g.n == 0) return;
  collapse_shape(g, 2);
  equal_kernel<<<blocks_for(g.n), kThreads, 0, st>>>(a, da, b, db, out, g);
  IDEV_LAUNCHED();
}

void launch_glue_where(int elem_bytes, const uint8_t* c, const void* x, const void* y, void* out,
                       GlueShape g, cudaStream_t st) {
  if (g.n == 0) return;
  collapse_shape(g, 3);
  const unsigned nb = blocks_for(g.n);
  if (elem_bytes == 4)
    where_kernel<uint32_t><<<nb, kThreads, 0, st>>>(c, static_cast<const uint32_t*>(x),
                                                    static_cast<const uint32_t*>(y),
                                                    static_cast<uint32_t*>(out), g);
  else if (elem_bytes == 8)
    where_kernel<uint64_t><<<nb, kThreads, 0, st>>>(c, static_cast<const uint64_t*>(x),
                                                    static_cast<const uint64_t*>(y),
                                                    static_cast<uint64_t*>(out), g);
  else
    where_kernel<uint8_t><<<nb, kThreads, 0, st>>>(c, static_cast<const uint8_t*>(x),
                                                   static_cast<const uint8_t*>(y),
                                                   static_cast<uint8_t*>(out), g);
  IDEV_LAUNCHED();
}

void launch_glue_unary(int op, const float* x, float* y, int64_t n, cudaStream_t st) {
  if (n == 0) return;
  unary_kernel<<<blocks_for(n), kThreads, 0, st>>>(op, x, y, n);
  IDEV_LAUNCHED();
}

bool launch_glue_cast(int from, int to, const void* x, void* y, int64_t n, cudaStream_t st) {
  if (n == 0) return true;
  const unsigned nb = blocks_for(n);
#define IDEV_CAST(F, T, CF, CT)                                                          \
  if (from == F && to == T) {                                                           \
    cast_kernel<CF, CT><<<nb, kThreads, 0, st>>>(static_cast<const CF*>(x),             \
                                                 static_cast<CT*>(y), n);              \
    IDEV_LAUNCHED();                                                                    \
    return true;                                                                        \
  }
  // The pairs the reference's Cast takes (src/kernels/movement.cc:345-372).
  IDEV_CAST(1, 7, float, int64_t)
  IDEV_CAST(7, 1, int64_t, float)
  IDEV_CAST(6, 1, int32_t, float)
  IDEV_CAST(1, 6, float, int32_t)
  IDEV_CAST(7, 6, int64_t, int32_t)
  IDEV_CAST(6, 7, int32_t, int64_t)
#undef IDEV_CAST
  if (from == 9 && to == 1) {
    bool_to_f32_kernel<<<nb, kThreads, 0, st>>>(static_cast<const uint8_t*>(x),
                                                static_cast<float*>(y), n);
    IDEV_LAUNCHED();
    return true;
  }
  return false;
}

void launch_glue_copy(int elem_bytes, const void* in, void* out, GlueShape g, cudaStream_t st) {
  if (g.n == 0) return;
  collapse_shape(g, 2);
  const unsigned nb = blocks_for(g.n);
  switch (elem_bytes) {
    case 8:
      strided_copy_kernel<uint64_t><<<nb, kThreads, 0, st>>>(
          static_cast<const uint64_t*>(in), static_cast<uint64_t*>(out), g);
      break;
    case 4:
      strided_copy_kernel<uint32_t><<<nb, kThreads, 0, st>>>(
          static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out), g);
      break;
    default:
      strided_copy_kernel<uint8_t><<<nb, kThreads, 0, st>>>(
          static_cast<const uint8_t*>(in), static_cast<uint8_t*>(out), g);
  }
  IDEV_LAUNCHED();
}

void launch_glue_gather(int elem_bytes, const void* data, const void* idx, bool idx64, void* out,
                        int64_t outer, int64_t axis_dim, int64_t n_idx, int64_t slice, int* err,
                        cudaStream_t st) {
  const int64_t n = outer * n_idx * slice;
  if (n == 0) return;
  const unsigned nb = blocks_for(n);
  switch (elem_bytes) {
    case 8:
      gather_kernel<uint64_t><<<nb, kThreads, 0, st>>>(
          static_cast<const uint64_t*>(data), idx, idx64, static_cast<uint64_t*>(out), outer,
          axis_dim, n_idx, slice, err);
      break;
    case 4:
      gather_kernel<uint32_t><<<nb, kThreads, 0, st>>>(
          static_cast<const uint32_t*>(data), idx, idx64, static_cast<uint32_t*>(out), outer,
          axis_dim, n_idx, slice, err);
      break;
    default:
      gather_kernel<uint8_t><<<nb, kThreads, 0, st>>>(
          static_cast<const uint8_t*>(data), idx, idx64, static_cast<uint8_t*>(out), outer,
          axis_dim, n_idx, slice, err);
  }
  IDEV_LAUNCHED();
}

void launch_glue_row_mean(const float* x, float* y, int64_t rows, int64_t cols,
                          cudaStream_t st) {
  if (rows == 0) return;
  const int64_t threads = rows * 32;
  row_mean_kernel<<<(unsigned)((threads + kThreads - 1) / kThreads), kThreads, 0, st>>>(
      x, y, rows, cols);
  IDEV_LAUNCHED();
}

void launch_glue_fill(int elem_bytes, void* out, const void* value, int64_t n, cudaStream_t st) {
  if (n == 0) return;
  const unsigned nb = blocks_for(n);
  if (elem_bytes == 8) {
    uint64_t v;
    std::memcpy(&v, value, 8);
    fill_kernel<uint64_t><<<nb, kThreads, 0, st>>>(static_cast<uint64_t*>(out), v, n);
  } else if (elem_bytes == 4) {
    uint32_t v;
    std::memcpy(&v, value, 4);
    fill_kernel<uint32_t><<<nb, kThreads, 0, st>>>(static_cast<uint32_t*>(out), v, n);
  } else {
    uint8_t v;
    std::memcpy(&v, value, 1);
    fill_kernel<uint8_t><<<nb, kThreads, 0, st>>>(static_cast<uint8_t*>(out), v, n);
  }
  IDEV_LAUNCHED();
}


// One CTA per (32 output columns, matrix): lane = column (coalesced rows of
// B), warp = k slice (k = warp, warp + 8, ...); the 8 slices' partial sums
// are added in slice order.
__global__ void __launch_bounds__(256) bmm_small_kernel(const float* __restrict__ a,
                                                        const float* __restrict__ b,
                                                        float* __restrict__ out, int M, int64_t K,
                                                        int64_t N, GlueShape g) {
  __shared__ float red[8][kGlueBmmMaxM][32];
  const int64_t i = blockIdx.y;
  int64_t rem = i, ia = 0, ib = 0;
  for (int d = g.rank - 1; d >= 0; --d) {
    const int64_t c = rem % g.shape[d];
    rem /= g.shape[d];
    ia += c * g.s0[d];
    ib += c * g.s1[d];
  }
  const float* A = a + ia * M * K;
  const float* B = b + ib * K * N;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t n = (int64_t)blockIdx.x * 32 + tx;
  float acc[kGlueBmmMaxM];
#pragma unroll
  for (int m = 0; m < kGlueBmmMaxM; ++m) acc[m] = 0.f;
  if (n < N)
    for (int64_t k = ty; k < K; k += 8) {
      const float bv = B[k * N + n];
#pragma unroll
      for (int m = 0; m < kGlueBmmMaxM; ++m)
        if (m < M) acc[m] = fmaf(A[m * K + k], bv, acc[m]);
    }
#pragma unroll
  for (int m = 0; m < kGlueBmmMaxM; ++m)
    if (m < M) red[ty][m][tx] = acc[m];
  __syncthreads();
  if (ty < M && n < N) {
    float t = 0.f;
#pragma unroll
    for (int sl = 0; sl < 8; ++sl) t += red[sl][ty][tx];
    out[(i * M + ty) * N + n] = t;
  }
}

void launch_glue_bmm_small(const float* a, const float* b, float* out, int64_t M, int64_t K,
                           int64_t N, const GlueShape& g, cudaStream_t st) {
  if (g.n <= 0 || M <= 0 || N <= 0) return;
  IDEV_CHECK_ARG(M <= kGlueBmmMaxM && g.n <= 65535, "batched small MatMul: M or batch too large");
  dim3 grid((unsigned)((N + 31) / 32), (unsigned)g.n);
  bmm_small_kernel<<<grid, 256, 0, st>>>(a, b, out, (int)M, K, N, g);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
