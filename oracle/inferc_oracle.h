/* CPU restatement ("port") of inferc's fused-op hot path, in plain C.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker or the timed CPU baseline. The product path
 * (inferc_b200/, libinferc_b200.so) never calls into it.
 *
 * Every function cites the reference function it restates (paths are relative
 * to the dbhan08/inferc source tree). All arrays are dense row-major fp32
 * unless stated. Parity pin: tests/test_oracle.py checks these functions
 * against the known-answer vectors of tests/kernels_test.cc and
 * bench/amx/int4_gemv_amx.cc, and against golden outputs that
 * tests/golden/make_golden.py produced by running the reference's own kernel
 * sources (compiled by oracle/Makefile).
 */
#ifndef INFERC_ORACLE_H_
#define INFERC_ORACLE_H_

#include <stdint.h>

#include "../include/inferc_models.h"

#ifdef __cplusplus
extern "C" {
#endif

/* LayerNorm over the last `feat` elements of each row
 * (src/kernels/activation.cc:103-150). */
void orc_layernorm(const float* x, const float* gamma, const float* beta,
                   float* y, int64_t rows, int64_t feat, float eps);

/* Exact erf GELU (src/kernels/activation.cc:15-29). */
void orc_gelu(const float* x, float* y, int64_t n);

/* GPT-2 tanh GELU (src/kernels/activation.cc:31-50). */
void orc_gelu_tanh(const float* x, float* y, int64_t n);

/* Row softmax over the last axis (src/kernels/activation.cc:52-101). */
void orc_softmax(const float* x, float* y, int64_t rows, int64_t cols);

/* Plain row-major GEMM C = alpha*op(A)*op(B) + beta*C (the arithmetic
 * cblas_sgemm performs at src/kernels/matmul.cc:218). */
void orc_sgemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
               float alpha, const float* A, int64_t lda, const float* B,
               int64_t ldb, float beta, float* C, int64_t ldc);

/* ONNX Gemm with bias broadcast (src/kernels/matmul.cc:161-228).
 * c may be NULL; c_len is M*N, N or 1. Returns 0 or -1 on a bad C shape. */
int orc_gemm(const float* a, const float* b, const float* c, int64_t c_len,
             float* y, int64_t M, int64_t K, int64_t N, float alpha,
             float beta, int trans_a, int trans_b);

/* Y = erfGELU(X*W + b); X [M,K], W [K,N], b [N]
 * (src/kernels/fused_matmul_add_gelu.cc:13-80). */
void orc_fused_matmul_add_gelu(const float* x, const float* w, const float* b,
                               float* y, int64_t M, int64_t K, int64_t N);

/* {X*Wq+bq, X*Wk+bk, X*Wv+bv}; X [M,K], Wi [K,N]
 * (src/kernels/attention.cc:102-141). */
void orc_fused_qkv(const float* x, const float* wq, const float* bq,
                   const float* wk, const float* bk, const float* wv,
                   const float* bv, float* q, float* k, float* v, int64_t M,
                   int64_t K, int64_t N);

/* Multi-head attention on [B,S,H] Q/K/V (src/kernels/attention.cc:32-100).
 * mask: bool bytes, true = masked (score replaced by `fill`), broadcast to
 * [B,nH,S,S] from a right-aligned shape mask_shape[0..mask_rank) (MaskStrides,
 * attention.cc:17-29); NULL or mask_rank == 0 means no mask. */
void orc_fused_attention(const float* q, const float* k, const float* v,
                         const uint8_t* mask, const int64_t* mask_shape,
                         int mask_rank, int64_t B, int64_t S, int64_t H,
                         int64_t head_dim, float fill, float* out);

/* y[N] = W[N,K] x, W int4 with per-row fp32 scale: weight = s*float(q-8)
 * formed in fp32, products and sum in double. Byte r*(K/2)+k/2 holds k even in
 * the low nibble, k odd in the high nibble
 * (bench/amx/int4_gemv_amx.cc:258-271). */
void orc_int4_gemv_rowscale(const uint8_t* w, const float* scales,
                            const float* x, float* y, int64_t N, int64_t K);

/* Per-tensor-scale variant (bench/amx/int4_gemv_amx.cc:243-255). */
void orc_int4_gemv(const uint8_t* w, float scale, const float* x, float* y,
                   int64_t N, int64_t K);

/* Greedy argmax, first maximum wins (src/cli/main.cpp:823-829, :870-875). */
int64_t orc_argmax(const float* x, int64_t n);

/* DistilBERT-architecture encoder forward in the order of the optimized plan
 * (FusedQKV, FusedAttention, MatMul+Add+Add, FusedLayerNorm,
 * FusedMatMulAddGELU, MatMul+Add+Add, FusedLayerNorm per layer; Gather CLS,
 * Gemm+Relu, Gemm head). ids / mask int64 [B,S]; logits [B,n_classes].
 * Returns 0, or -1 on an out-of-range token id. */
int orc_encoder_forward(const InfercEncoderWeights* w, const int64_t* ids,
                        const int64_t* mask, int64_t B, int64_t S,
                        float* logits);

/* GPT-2 greedy decode with KV cache (src/cli/main.cpp:700-945): prefill over
 * the prompt, then max_tokens-1 single-token steps. tokens_out receives
 * max_tokens ids; margins_out (may be NULL) the top1-top2 logit gap of each
 * generated token. Returns 0, or -1 on bad arguments. */
int orc_gpt2_decode_lm(const InfercGpt2Weights* w, const float* lm, const int64_t* prompt,
                       int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                       float* margins_out);
int orc_gpt2_decode(const InfercGpt2Weights* w, const int64_t* prompt,
                    int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                    float* margins_out);

#ifdef __cplusplus
}
#endif

#endif /* INFERC_ORACLE_H_ */
