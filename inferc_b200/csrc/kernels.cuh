// Host-side launchers of the device kernels (one .cu per kernel family).
#pragma once

#include "common.cuh"

namespace inferc_dev {

// ---- layernorm.cu
// sp: optional fp16 hi / lo split of y for the split-fp16 GEMM.
void launch_layernorm(const float* x, const float* gamma, const float* beta, float* y,
                      int64_t rows, int64_t feat, float eps, cudaStream_t st,
                      const SplitOut& sp = SplitOut());
// Encoder embedding: y[b,s,:] = LN(word[ids[b,s]] + pos[s]); cond[b,s] =
// (mask[b,s] == 0). Out-of-range ids set *err_flag (device int) to 1 and
// produce a zero row.
void launch_embed_layernorm(const int64_t* ids, const int64_t* mask, const float* word,
                            const float* pos, int64_t vocab, const float* gamma,
                            const float* beta, float* y, uint8_t* cond, int64_t B,
                            int64_t S, int64_t H, float eps, int* err_flag, cudaStream_t st,
                            const SplitOut& sp = SplitOut());

// ---- gemm_simt.cu : C[M,N] = epilogue(op(A) op(B)) on CUDA cores (fp32 FMA).
void launch_gemm_simt(const float* A, int64_t lda, bool trans_a, const float* B, int64_t ldb,
                      bool trans_b, float* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                      const Epilogue& ep, cudaStream_t st);

// ---- elementwise.cu
void launch_act(const float* x, float* y, int64_t n, int act, cudaStream_t st);
void launch_softmax(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t st);
void launch_fill_rows(float* y, const float* c, int64_t c_len, int64_t M, int64_t N,
                      cudaStream_t st);

// ---- attention.cu
struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  int64_t ldq, ldk, ldv, ldo;  // row strides (elements) of the [B*S, *] views
  int64_t bstride_q, bstride_k, bstride_v, bstride_o;  // batch strides (elements)
  const uint8_t* mask;         // bool, true = masked; may be null
  int64_t ms[4];               // mask element strides over [B, nH, S, S]
  int64_t B, S, nH, hd;
  float scale, fill;
  int causal;                  // 1: additionally mask j > i (prefill)
  SplitOut so;                 // tensor-core path only: write out's fp16 split instead
};
void launch_attention(const AttnArgs& a, cudaStream_t st);

// Split-fp16 tensor-core GEMM (gemm_f16s.cu). Weights: fp16 hi / lo planes
// [N, Kp] (Kp = f16_weight_kp(K)) of W * 2^s and scale2 = {scratch, 2^-s}.
// range_flag: set to 1 when A holds a value fp16 cannot carry (the result is
// then invalid; rerun on the 3xTF32 kernel); null = the module-wide flag.
int64_t f16_weight_kp(int64_t K);
// trans: W is stored [N, K] (the transB operand of a Gemm).
void prepare_weight_f16(const float* W, int64_t K, int64_t N, int64_t ldw, uint16_t* hi,
                        uint16_t* lo, float* scale2, cudaStream_t st, bool trans = false);
bool gemm_f16s_supported(const float* A, int64_t lda, int64_t M, int64_t N, int64_t K);
void launch_gemm_f16s(const float* A, int64_t lda, const uint16_t* Bh, const uint16_t* Bl,
                      int64_t kp, const float* scale2, int* range_flag, float* C, int64_t ldc,
                      int64_t M, int64_t N, int64_t K, const Epilogue& ep, cudaStream_t st);
// A operand of the split-fp16 GEMM: fp32 (a32, split by the kernel) or
// already split into fp16 hi / lo planes (a32 null).
struct F16GemmA {
  const float* a32 = nullptr;
  const uint16_t* hi = nullptr;
  const uint16_t* lo = nullptr;
  int64_t ld = 0;
};
// Split-K scratch of the one-SM split-fp16 GEMM, owned by the caller and
// used by one stream at a time: when the output has too few tiles to fill
// the SMs, K is split over CTAs that store raw partial tiles in `part`
// (part_floats floats); the CTA that completes a tile's counter (cnt, cnt_n
// words, zero at rest and left zero) sums the partials in split order and
// runs the epilogue. Null part: no split. A call that reports a timeout can
// leave counters non-zero: the owner must clear them (or be recreated).
struct SplitK {
  float* part = nullptr;
  int64_t part_floats = 0;
  unsigned* cnt = nullptr;
  int cnt_n = 0;
};
// General form: so.hi set = write the result's fp16 split instead of C
// (pre-split A, bias or bias+GELU epilogue only).
void launch_gemm_f16s(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                      const float* scale2, int* range_flag, float* C, int64_t ldc,
                      const SplitOut& so, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                      cudaStream_t st, const SplitK& sk = SplitK());
int read_and_clear_f16_range();
// Two-SM (cta_group::2, 256-row) form of the split-fp16 GEMM for pre-split A
// (gemm_f16s_2cta.cu): used for split-plane outputs unless INFERC_GEMM_2CTA=0
// (=1: for every eligible GEMM).
bool gemm_f16s_2cta_usable(const F16GemmA& A, int64_t M, int64_t N, int64_t K, bool split_out);
void launch_gemm_f16s_2cta(const F16GemmA& A, const uint16_t* Bh, const uint16_t* Bl, int64_t kp,
                           const float* scale2, float* C, int64_t ldc, const SplitOut& so,
                           int64_t M, int64_t N, int64_t K, int epi, const Epilogue& ep,
                           cudaStream_t st);
int* f16_range_flag_ptr();  // the current device's module-wide range flag
// x [rows, cols] -> fp16 hi / lo planes; range null = the module-wide flag.
void launch_split_rows_f16(const float* x, int64_t rows, int64_t cols, int64_t ldx, uint16_t* hi,
                           uint16_t* lo, int64_t ld, int* range, cudaStream_t st);
// Tensor-core path (head_dim 64, S <= 128, 16-byte aligned operands).
bool attention_tc_supported(const AttnArgs& a);
void launch_attention_tc(const AttnArgs& a, cudaStream_t st);
bool attention_tc_enabled();
// Split-fp16 form (attention_f16.cu): q, k, v as fp16 hi / lo planes of a
// [B, S, ld] tensor (head h at columns h*64..h*64+63), output as fp32 or as
// fp16 planes (so.hi). Requires S <= 128, head_dim 64, 16-byte alignment.
struct AttnF16Args {
  const uint16_t *qh, *ql, *kh, *kl, *vh, *vl;
  int64_t ld, bstride;  // elements
  const uint8_t* mask;
  int64_t ms[4];
  int64_t B, S, nH;
  float scale, fill;
  float* out;
  int64_t ldo, bstride_o;
  SplitOut so;
};
bool attention_f16_supported(const AttnF16Args& a);
void launch_attention_f16(const AttnF16Args& a, cudaStream_t st);
inline bool attention_tc_usable(const AttnArgs& a) {
  return attention_tc_supported(a) && attention_tc_enabled();
}

void launch_kv_append(const float* k_new, const float* v_new, int64_t ld_new, float* kc,
                      float* vc, int64_t heads, int64_t hd, int64_t max_len,
                      const int64_t* pos_dev, int64_t pos_host, int64_t n, cudaStream_t st);
// Decode attention; L (number of visible keys) either from *len_dev (device,
// when non-null) or len_host. When k_new/v_new are given, the kernel first
// writes them at position L-1 of the cache (fused KV append).
void launch_decode_attention(const float* q, const float* k_new, const float* v_new,
                             float* kc, float* vc, float* out, int64_t heads, int64_t hd,
                             int64_t max_len, const int64_t* len_dev, int64_t len_host,
                             cudaStream_t st);

// ---- gemv.cu
struct Workspace;

struct GemvArgs {
  Workspace* ws = nullptr;  // split-K scratch; null = the device's shared one
  const float* x;       // [K] input (raw residual stream when ln_gamma is set)
  const float* ln_gamma;  // optional LayerNorm prologue on x
  const float* ln_beta;
  float ln_eps;
  const float* w;       // [K, N] row-major
  const float* bias;    // [N] or null
  const float* resid;   // [N] or null, may alias y
  float* y;             // [N]
  int64_t K, N;
  float alpha, beta;    // y = act(alpha*acc + beta*bias + resid)
  int act;
};
// Split-K over CTAs; partial sums go to the workspace and the last CTA of
// each column tile reduces them in a fixed order (deterministic).
void launch_gemv(const GemvArgs& g, cudaStream_t st);

// Row-dot GEMV y[N] = W[N,K] x (W rows contiguous), optional LN prologue on x,
// optional fused greedy argmax (first max wins) into *argmax_out; when
// pos_counter is non-null the last block also increments it after writing
// the token to tokens[*pos_counter - base] (decode loop bookkeeping).
struct RowGemvArgs {
  Workspace* ws = nullptr;  // scratch for the fused argmax; null = shared
  const float* x;
  const float* ln_gamma;
  const float* ln_beta;
  float ln_eps;
  const float* w;  // [N, K]
  float* y;        // [N]
  int64_t K, N;
  int64_t* argmax_out;  // optional
  int64_t* pos_counter; // optional
  int64_t* token_log;   // optional, token_log[*pos_counter - log_base] = argmax
  int64_t log_base;
};
void launch_row_gemv(const RowGemvArgs& g, cudaStream_t st);

void launch_argmax(const float* x, int64_t n, int64_t* out, cudaStream_t st);

// int4 per-row-scale row GEMV (gemv.cu) for weight-only int4 decode: W in the
// reference's int4 layout [N, K/2] bytes with scales [N]; y[r] =
// act(s_r * sum_k (q-8) x_k + bias[r] + resid[r]), optional LayerNorm
// prologue on x and fused greedy argmax with the decode-loop bookkeeping of
// RowGemvArgs. K % 8 == 0. (Epilogue order as GemvArgs: act(s*dot + b + resid).)
struct Int4RowArgs {
  Workspace* ws = nullptr;
  const float* x;
  const float* ln_gamma;
  const float* ln_beta;
  float ln_eps;
  const uint8_t* w;
  const float* scales;
  const float* bias;
  const float* resid;  // may alias y
  float* y;
  int64_t K, N;
  int act;
  int64_t* argmax_out;
  int64_t* pos_counter;
  int64_t* token_log;
  int64_t log_base;
};
void launch_int4_row_gemv(const Int4RowArgs& g, cudaStream_t st);
// Per-row symmetric int4 quantisation (s = max|w|/7, q = clamp(rint(w/s)))
// of a [K, N] weight (output row = column; trans: an [N, K] weight) into
// out [N, K/2] + scales [N].
void launch_int4_pack(const float* w, int64_t K, int64_t N, int64_t ldw, bool trans,
                      uint8_t* out, float* scales, cudaStream_t st);

// ---- gemv_int4.cu
void launch_gemv_int4(const InfercInt4Gemv* descs_host, int count, cudaStream_t st);

// ---- decode embedding (gemv.cu): x = wte[*tok] + wpe[*pos - 1]
void launch_decode_embed(const int64_t* tok, const int64_t* pos, const float* wte,
                         const float* wpe, float* x, int64_t H, int64_t vocab,
                         int64_t max_pos, int* err_flag, cudaStream_t st);

// Rows embedding for prefill: x[i] = wte[ids[i]] + wpe[pos0 + i].
void launch_rows_embed(const int64_t* ids, int64_t n, int64_t pos0, const float* wte,
                       const float* wpe, float* x, int64_t H, int64_t vocab, int* err_flag,
                       cudaStream_t st);

// Workspace management (per device), used by split-K reductions.
// Scratch for split-K / cross-CTA reductions. Counters must start at zero;
// every kernel that uses them returns them to zero before it exits. Kernels
// that share one Workspace must be ordered on the device (one stream).
struct Workspace {
  float* partials = nullptr;
  size_t partial_floats = 0;
  unsigned int* counters = nullptr;
  size_t n_counters = 0;
  bool owned = false;
  void allocate(size_t floats, size_t counters);
  void release();
};
Workspace& workspace_for_current_device();

}  // namespace inferc_dev
