// Launchers of the glue-op kernels (glue.cu) used by the device executor.
#pragma once

#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace inferc_dev {

constexpr int kGlueMaxRank = 8;

enum GlueBinOp { GLUE_ADD = 0, GLUE_SUB, GLUE_MUL, GLUE_DIV, GLUE_POW };
enum GlueUnaryOp { GLUE_SQRT = 0, GLUE_ERF, GLUE_RELU, GLUE_TANH, GLUE_NEG, GLUE_ABS };

// An index space of n = prod(shape) elements and up to three operands'
// element strides per axis (0 on broadcast axes), plus base offsets for the
// strided copy (off0: source, off1: destination).
struct GlueShape {
  int rank = 0;
  int64_t n = 0;
  int64_t shape[kGlueMaxRank] = {};
  int64_t s0[kGlueMaxRank] = {};
  int64_t s1[kGlueMaxRank] = {};
  int64_t s2[kGlueMaxRank] = {};
  int64_t off0 = 0, off1 = 0;
};

// Merges adjacent axes over which all `operands` stride arrays are
// contiguous and drops size-1 axes (host side; the launchers call it).
void collapse_shape(GlueShape& g, int operands);

// dt: 1 = fp32, 7 = int64 (ONNX codes). Operand strides in s0 (a), s1 (b);
// out is contiguous over g.shape.
void launch_glue_binary(int op, int dt, const void* a, const void* b, void* out, GlueShape g,
                        cudaStream_t st);
// out (bool bytes) = (int64)a == (int64)b; da / db: ONNX dtype codes.
void launch_glue_equal(const void* a, int da, const void* b, int db, uint8_t* out, GlueShape g,
                       cudaStream_t st);
// out = c ? x : y; strides: s0 cond, s1 x, s2 y.
void launch_glue_where(int elem_bytes, const uint8_t* c, const void* x, const void* y, void* out,
                       GlueShape g, cudaStream_t st);
void launch_glue_unary(int op, const float* x, float* y, int64_t n, cudaStream_t st);
// false when the dtype pair is not one the reference's Cast takes.
bool launch_glue_cast(int from, int to, const void* x, void* y, int64_t n, cudaStream_t st);
// out[off1 + c.s1] = in[off0 + c.s0] for every coordinate c of g.shape.
void launch_glue_copy(int elem_bytes, const void* in, void* out, GlueShape g, cudaStream_t st);
void launch_glue_gather(int elem_bytes, const void* data, const void* idx, bool idx64, void* out,
                        int64_t outer, int64_t axis_dim, int64_t n_idx, int64_t slice, int* err,
                        cudaStream_t st);
void launch_glue_row_mean(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t st);
void launch_glue_fill(int elem_bytes, void* out, const void* value, int64_t n, cudaStream_t st);

// Batched MatMul with at most kGlueBmmMaxM rows per matrix: for each index i
// of the batch shape g.shape (g.n matrices), out[i] (M x N) = A[i] (M x K)
// B[i] (K x N), A[i] and B[i] found through the per-axis matrix strides g.s0
// and g.s1 (0 on broadcast axes). Fixed summation order.
constexpr int kGlueBmmMaxM = 8;
void launch_glue_bmm_small(const float* a, const float* b, float* out, int64_t M, int64_t K,
                           int64_t N, const GlueShape& g, cudaStream_t st);

}  // namespace inferc_dev
