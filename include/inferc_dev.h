/* libinferc_b200 — C ABI of the B200 (sm_100a) device executor for inferc's
 * fused-op hot path.
 *
 * This is the boundary the reference's runtime would bind in place of its CPU
 * kernels. The reference dispatches on the op_type string inside
 * Executor::Run (src/runtime/executor.cc:123-343) to free functions
 * `rt::Tensor Op(const rt::Tensor&..., attrs)` that throw std::runtime_error;
 * each entry point below replaces one of those functions (cited per entry)
 * and keeps its argument meaning, its attribute defaults and its checks, but
 * takes raw device pointers and sizes and returns a status code instead of
 * throwing.
 *
 * Conventions
 *   - Return value: INFERC_OK (0) or an INFERC_ERR_* code; the message is
 *     available from inferc_dev_last_error_string() on the calling thread.
 *   - Tensor pointers are DEVICE addresses (cudaMalloc / inferc_dev_alloc)
 *     of dense row-major fp32 data unless stated; "host" marks the
 *     exceptions. Leading dims of the reference's [..., M, K] inputs are
 *     flattened into M by the caller (as the reference kernels do).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Every op
 *     is asynchronous with respect to the host.
 *   - No entry point falls back to the CPU: without a usable CUDA device they
 *     return INFERC_ERR_CUDA.
 */
#ifndef INFERC_DEV_H_
#define INFERC_DEV_H_

#include <stddef.h>
#include <stdint.h>

#include "inferc_models.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
  INFERC_OK = 0,
  INFERC_ERR_INVALID = 1, /* bad shape / argument (reference: runtime_error) */
  INFERC_ERR_CUDA = 2,    /* CUDA runtime or launch failure */
  INFERC_ERR_OOM = 3,     /* device or host allocation failed */
  INFERC_ERR_TIMEOUT = 4, /* a bounded device wait gave up */
  INFERC_ERR_RANGE = 5    /* index or value out of range found on the device */
};

/* ---------------------------------------------------------------- runtime */

/* Message of the last failed call on this host thread (never NULL). */
const char* inferc_dev_last_error_string(void);

/* Library version string, e.g. "inferc_b200 0.1 sm_100a". */
const char* inferc_dev_version(void);

/* Device buffers (replace rt::Tensor's host storage, src/runtime/tensor.cc:53-75). */
int inferc_dev_alloc(void** ptr, size_t bytes);
int inferc_dev_free(void* ptr);
int inferc_dev_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int inferc_dev_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
/* Waits for the stream; also reports INFERC_ERR_TIMEOUT when a bounded
 * device wait of an earlier tensor-core kernel gave up, and INFERC_ERR_RANGE
 * when an earlier split-fp16 call met a value fp16 cannot carry (both flags
 * are then cleared). */
int inferc_dev_stream_synchronize(void* stream);

/* Test hook for the failure path, used by no plan and with no counterpart in
 * the reference: runs one of the library's bounded device waits on something
 * that is never signalled (which = 0: an mbarrier phase as in the TMA /
 * tcgen05 pipelines; 1: a grid-barrier arrival counter as in the persistent
 * decode kernel) with a limit of limit_us microseconds. The wait gives up,
 * sets the device error flag and returns; the next
 * inferc_dev_stream_synchronize reports INFERC_ERR_TIMEOUT and clears it.
 * Nothing traps, faults or hangs; the context stays usable. */
int inferc_dev_selftest_wait_timeout(int which, int64_t limit_us, void* stream);

/* ------------------------------------------------------------- fused ops */

/* FusedLayerNorm (rt::LayerNorm, src/kernels/activation.cc:103-150; executor
 * attribute `epsilon`, default 1e-5, executor.cc:213-217). y = (x-mean) *
 * (1/sqrtf(var+eps)) * gamma + beta over each row of `feat` elements, biased
 * variance. x and y may alias. */
int inferc_dev_layernorm(const float* x, const float* gamma, const float* beta,
                         float* y, int64_t rows, int64_t feat, float eps,
                         void* stream);

/* Op-level GEMMs and their weights. inferc_dev_fused_matmul_add_gelu,
 * _fused_qkv, _gemm (M > 1) and _matmul treat B / W as a long-lived
 * initializer, as the reference's executor does (it copies each initializer
 * once per Executor, src/runtime/executor.cc:89-96): the first call that
 * sees a weight (device pointer, K, N, layout) converts it once into
 * split-fp16 planes kept in a per-device cache, and every later call runs
 * the split-fp16 tensor-core GEMM on those planes (fp32-level accuracy; an
 * activation fp16 cannot carry makes the same call recompute its result on
 * the CUDA cores, on the device, with no host round trip). That first call
 * synchronises its stream and cannot be stream-captured; later calls can.
 * The cache assumes the weight's values stay fixed: before rewriting or
 * freeing a cached weight, call inferc_dev_weight_cache_evict(w) (or _clear)
 * with its device current. Calls on different streams may run concurrently;
 * each stream has its own scratch flag. INFERC_OP_GEMM=tf32x3 selects the
 * 3xTF32 kernel with a per-call weight split instead. */
int inferc_dev_weight_cache_evict(const float* w);
int inferc_dev_weight_cache_clear(void);
/* Device bytes held by the cache (all devices). */
int64_t inferc_dev_weight_cache_bytes(void);

/* FusedMatMulAddGELU (src/kernels/fused_matmul_add_gelu.cc:13-80):
 * Y[M,N] = erfGELU(X[M,K] W[K,N] + b[N]). */
int inferc_dev_fused_matmul_add_gelu(const float* x, const float* w,
                                     const float* b, float* y, int64_t M,
                                     int64_t K, int64_t N, void* stream);

/* FusedQKV (rt::FusedQKVProjection, src/kernels/attention.cc:102-141):
 * q = X Wq + bq, k = X Wk + bk, v = X Wv + bv; X [M,K], Wi [K,N], outputs
 * [M,N]. */
int inferc_dev_fused_qkv(const float* x, const float* wq, const float* bq,
                         const float* wk, const float* bk, const float* wv,
                         const float* bv, float* q, float* k, float* v,
                         int64_t M, int64_t K, int64_t N, void* stream);

/* FusedAttention (src/kernels/attention.cc:32-100; attributes head_dim,
 * default 64, and fill, default -3.0e38, executor.cc:218-224).
 * q, k, v, out: [B,S,H], head h at columns [h*head_dim, (h+1)*head_dim).
 * mask: optional bool bytes (DEVICE), true = masked (score REPLACED by fill),
 * of shape mask_shape[0..mask_rank) (HOST array) right-aligned and broadcast
 * to [B, H/head_dim, S, S]; NULL / rank 0 = no mask. head_dim <= 128. */
int inferc_dev_fused_attention(const float* q, const float* k, const float* v,
                               const uint8_t* mask, const int64_t* mask_shape,
                               int mask_rank, int64_t B, int64_t S, int64_t H,
                               int64_t head_dim, float fill, float* out,
                               void* stream);

/* ONNX Gemm (rt::Gemm, src/kernels/matmul.cc:161-228): Y[M,N] =
 * alpha*op(A) op(B) + beta*C. c may be NULL; c_len is M*N (full), N (row
 * broadcast) or 1 (scalar); other lengths are rejected. M == 1 runs the
 * split-K GEMV kernel (the reference's decode shape). */
int inferc_dev_gemm(const float* a, const float* b, const float* c,
                    int64_t c_len, float* y, int64_t M, int64_t K, int64_t N,
                    float alpha, float beta, int trans_a, int trans_b,
                    void* stream);

/* 2-D MatMul (rt::MatMul, src/kernels/matmul.cc:63-159, batch_count == 1):
 * Y[M,N] = A[M,K] B[K,N]. */
int inferc_dev_matmul(const float* a, const float* b, float* y, int64_t M,
                      int64_t K, int64_t N, void* stream);

/* Gelu / GeluTanh (src/kernels/activation.cc:15-50), elementwise over n. */
int inferc_dev_gelu(const float* x, float* y, int64_t n, void* stream);
int inferc_dev_gelu_tanh(const float* x, float* y, int64_t n, void* stream);

/* Softmax over the last axis (src/kernels/activation.cc:52-101). */
int inferc_dev_softmax(const float* x, float* y, int64_t rows, int64_t cols,
                       void* stream);

/* Weight preparation for the tensor-core path: splits fp32 w[n] into
 * big = w rounded to tf32 and small = w - big (both fp32 arrays of n). An
 * executor does this once per initializer, as the reference copies each
 * initializer once per Executor (src/runtime/executor.cc:89-96). */
int inferc_dev_tf32_split(const float* w, float* big, float* small, int64_t n,
                          void* stream);

/* Prepared-weight GEMM with the fused epilogue of FusedMatMulAddGELU / Gemm:
 * Y[M,N] = act(A[M,K] (B_big + B_small)[K,N] + bias[N] + resid[M,N]) with A
 * and Y row strides lda / ldy and resid row stride ldr; bias / resid may be
 * NULL; act as for inferc_dev_gemv. Runs the tcgen05 3xTF32 kernel when
 * operands are 16-byte aligned, else the CUDA-core kernel on B_big + B_small. */
int inferc_dev_gemm_tf32x3(const float* a, int64_t lda, const float* b_big,
                           const float* b_small, int64_t ldb, const float* bias,
                           const float* resid, int64_t ldr, float* y,
                           int64_t ldy, int64_t M, int64_t N, int64_t K,
                           int act, void* stream);

/* Split-fp16 prepared weights: w [K,N] fp32 (row stride ldw) becomes two
 * fp16 planes hi, lo of shape [N, Kp] (K-major, Kp = inferc_dev_f16_kp(K);
 * uint16 storage of IEEE half) holding w * 2^s = hi + lo, with the power of
 * two 2^s chosen on the device so that max|w| 2^s < 2^14; scale2 is a device
 * array of 2 floats (scale2[1] = 2^-s). Done once per initializer. */
int64_t inferc_dev_f16_kp(int64_t K);
int inferc_dev_f16_split(const float* w, int64_t K, int64_t N, int64_t ldw,
                         uint16_t* hi, uint16_t* lo, float* scale2, void* stream);

/* Prepared-weight GEMM on the fp16 tensor cores with fp32-level accuracy
 * (three fp16 MMAs per product: lo_a hi_b + hi_a lo_b + hi_a hi_b, A split
 * on the fly), same epilogue as inferc_dev_gemm_tf32x3. A must be 16-byte
 * aligned with lda % 4 == 0. A value of A that fp16 cannot carry (|a| >=
 * 65520, inf, NaN) makes the next inferc_dev_stream_synchronize return
 * INFERC_ERR_RANGE: the result is invalid and the caller reruns the GEMM
 * with inferc_dev_gemm_tf32x3. */
int inferc_dev_gemm_f16s(const float* a, int64_t lda, const uint16_t* hi,
                         const uint16_t* lo, const float* scale2, const float* bias,
                         const float* resid, int64_t ldr, float* y, int64_t ldy,
                         int64_t M, int64_t N, int64_t K, int act, void* stream);

/* Activation split for chains of split-fp16 GEMMs: x [rows, cols] fp32
 * (row stride ldx) -> hi, lo fp16 planes (row stride ld); cols, ldx, ld
 * even. Out-of-range values are reported like inferc_dev_gemm_f16s's. */
int inferc_dev_f16_split_rows(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                              uint16_t* hi, uint16_t* lo, int64_t ld, void* stream);

/* inferc_dev_gemm_f16s with A given as its fp16 planes (a_hi, a_lo, row
 * stride lda, a multiple of 8, 16-byte aligned) — the form the encoder plan
 * runs, A split by its producer. When y_hi / y_lo are non-NULL the result is
 * stored as its fp16 split (row stride ldy) instead of y, for the next GEMM
 * of a chain; that form takes a bias (act 0 or 1), no resid, N % 16 == 0. */
int inferc_dev_gemm_f16s_planes(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda,
                                const uint16_t* hi, const uint16_t* lo, const float* scale2,
                                const float* bias, const float* resid, int64_t ldr, float* y,
                                uint16_t* y_hi, uint16_t* y_lo, int64_t ldy, int64_t M,
                                int64_t N, int64_t K, int act, void* stream);

/* FusedAttention (head_dim 64, S <= 128) on the fp16 tensor cores for q, k
 * and v given as fp16 hi / lo planes (inferc_dev_f16_split_rows or a
 * split-output GEMM): head h of token (b, s) at columns h*64.. of row
 * b*S + s, row stride ld (a multiple of 8; q, k, v may be column blocks of
 * one [B*S, 3H] plane pair). key_mask: optional bool [B,S], true = key
 * masked. out: fp32 [B, S, nH*64]. Values fp16 cannot carry are reported
 * like inferc_dev_gemm_f16s's. */
int inferc_dev_fused_attention_planes(const uint16_t* q_hi, const uint16_t* q_lo,
                                      const uint16_t* k_hi, const uint16_t* k_lo,
                                      const uint16_t* v_hi, const uint16_t* v_lo, int64_t ld,
                                      const uint8_t* key_mask, int64_t B, int64_t S,
                                      int64_t heads, float fill, float* out, void* stream);

/* FusedQKV + FusedAttention as one call on prepared weights (the encoder
 * plan's attention block): qkv = X Wqkv + bqkv with Wqkv = [Wq | Wk | Wv]
 * ([H, 3H], split by inferc_dev_tf32_split into w_big / w_small) and bqkv
 * [3H]; then attention over the q/k/v column blocks of qkv read in place
 * (row stride 3H). key_mask: optional bool [B,S], true = key masked (the
 * [B,1,1,S] padding mask of the reference graph); scratch_qkv: caller buffer
 * of B*S*3H floats; out: [B,S,H]. */
int inferc_dev_qkv_attention(const float* x, const float* w_big,
                             const float* w_small, const float* bqkv,
                             const uint8_t* key_mask, int64_t B, int64_t S,
                             int64_t H, int64_t head_dim, float fill,
                             float* scratch_qkv, float* out, void* stream);

/* inferc_dev_qkv_attention on split-fp16 prepared weights (w_hi, w_lo,
 * w_scale2 from inferc_dev_f16_split of Wqkv [H, 3H]): x is split into fp16
 * planes, the QKV GEMM writes q, k, v as planes, and the split-fp16
 * tensor-core attention (head_dim 64, S <= 4096) reads them. scratch: caller
 * buffer of 8*B*S*H uint16 (x planes, then the qkv planes). Values fp16
 * cannot carry are reported like inferc_dev_gemm_f16s's. */
int inferc_dev_qkv_attention_f16(const float* x, const uint16_t* w_hi, const uint16_t* w_lo,
                                 const float* w_scale2, const float* bqkv,
                                 const uint8_t* key_mask, int64_t B, int64_t S, int64_t H,
                                 int64_t head_dim, float fill, uint16_t* scratch, float* out,
                                 void* stream);

/* ------------------------------------------------------------ decode ops */

/* Batch-1 fp32 GEMV with the Gemm epilogue, y[N] = act(x[K] W[K,N] + b[N]
 * (+ resid[N])); act 0 none, 1 erf GELU, 2 tanh GELU, 3 ReLU. The M==1
 * Gemm of the decode graphs (src/kernels/matmul.cc:202-226). b / resid may
 * be NULL; resid may alias y. Split-K with a deterministic reduction. */
int inferc_dev_gemv(const float* x, const float* w, const float* b,
                    const float* resid, float* y, int64_t K, int64_t N,
                    int act, void* stream);

/* Allocation-free variant of inferc_dev_gemv, with the same arguments and
 * the same split-K rule (so the same result, bit for bit, whenever the
 * built-in scratch does not cap the split count; otherwise equal within fp32
 * rounding). No counterpart in the reference: it exists for callers that may not
 * allocate device memory (a host framework that owns the device heap, an
 * allocator-less runtime, a real-time loop), whereas inferc_dev_gemv
 * allocates its split-K scratch on first use. Its scratch is a fixed 1 MiB
 * array built into the library (held on every device that loads it until the
 * process exits), so N is limited to 262144 columns and K to 8192; larger
 * sizes return INFERC_ERR_INVALID. The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress) with the device current;
 * make that first call before any stream capture. All calls share the one
 * array, so calls that overlap on the GPU (different streams, or different
 * host threads on one device) race; order them on one stream. */
int inferc_dev_gemv_noalloc(const float* x, const float* w, const float* b,
                            const float* resid, float* y, int64_t K, int64_t N,
                            int act, void* stream);

/* int4 per-row-scale GEMV (bench/amx/int4_gemv_amx.cc:258-271): y[r] =
 * sum_k (scales[r]*(q[r,k]-8)) x[k]; W [N, K/2] bytes, byte r*(K/2)+k/2
 * holds even k in the low nibble, odd k in the high nibble. K must be even.
 * Accumulates in fp32. */
int inferc_dev_gemv_int4_rowscale(const uint8_t* w, const float* scales,
                                  const float* x, float* y, int64_t N,
                                  int64_t K, void* stream);

/* Many int4 GEMVs in one launch (the decode step's 4 matrices x layers +
 * LM head). descs is a HOST array of `count` descriptors with DEVICE
 * pointers. */
typedef struct InfercInt4Gemv {
  const uint8_t* w;
  const float* scales;
  const float* x;
  float* y;
  int64_t n, k;
} InfercInt4Gemv;
int inferc_dev_gemv_int4_batched(const InfercInt4Gemv* descs, int count,
                                 void* stream);

/* Greedy argmax with the first maximum winning (src/cli/main.cpp:823-829):
 * writes the index (int64, DEVICE) of the first largest of x[0..n). */
int inferc_dev_argmax(const float* x, int64_t n, int64_t* out_index,
                      void* stream);

/* KV-cache append in place, replacing the with-past graph's
 * Concat(past, new) (src/kernels/movement.cc:142-189): copies `n` new rows of
 * K and V (each [n, heads*head_dim], row stride ld_new) into the cache
 * k_cache / v_cache [heads, max_len, head_dim] at positions [pos, pos+n). */
int inferc_dev_kv_append(const float* k_new, const float* v_new,
                         int64_t ld_new, float* k_cache, float* v_cache,
                         int64_t heads, int64_t head_dim, int64_t max_len,
                         int64_t pos, int64_t n, void* stream);

/* Single-query attention over the first L cached positions (the decode
 * step's MatMul, Div(sqrt(head_dim)), Softmax, MatMul): q [heads*head_dim],
 * out [heads*head_dim]. */
int inferc_dev_decode_attention(const float* q, const float* k_cache,
                                const float* v_cache, float* out,
                                int64_t heads, int64_t head_dim,
                                int64_t max_len, int64_t L, void* stream);

/* ------------------------------------------------------- graph executor */

/* A device executor for an optimized inferc plan: the ONNX model `inferc
 * optimize` writes (src/cli/main.cpp:200-227), run node by node on the GPU in
 * place of Executor::Run (src/runtime/executor.cc:98-366) with the same op
 * names (the ONNX ops the reference executor takes and the inferc-domain
 * fused ops), attributes, defaults and error messages. Initializers are
 * uploaded once at load (executor.cc:89-96); activations come from the
 * device's stream-ordered pool and are released after their last reader.
 * Shape metadata (Shape / Constant / small int64 arithmetic) is evaluated on
 * the host when all of an op's inputs are known there; every tensor that
 * depends on an input's values is computed on the device. An op the reference
 * executor does not take makes load fail with its "unsupported op" message. */
typedef struct InfercGraph* inferc_graph_t;

/* Parses `model` (serialized ONNX ModelProto, HOST bytes) without touching a
 * device and writes a JSON summary (node count, op histogram, opsets, inputs,
 * outputs) into buf (NUL-terminated; *needed receives the size it takes;
 * buf may be NULL to query it). */
int inferc_dev_graph_describe(const void* model, size_t len, char* buf, size_t cap,
                              size_t* needed);
/* Parses the model and uploads its initializers to the current device. */
int inferc_dev_graph_load(const void* model, size_t len, inferc_graph_t* out);
/* Binds graph input `name`: dtype is an ONNX TensorProto code (1 float, 6
 * int32, 7 int64, 9 bool, 2 uint8), shape a HOST array of rank dims; data is
 * copied (from HOST memory, or DEVICE memory when data_on_device) on stream
 * into a buffer the graph owns, so it may be reused after the call. */
int inferc_dev_graph_set_input(inferc_graph_t g, const char* name, int dtype,
                               const int64_t* shape, int rank, const void* data,
                               int data_on_device, void* stream);
/* Runs every node on stream and waits for it (the reference's Run is
 * synchronous); a Gather index out of range returns INFERC_ERR_RANGE. */
int inferc_dev_graph_run(inferc_graph_t g, void* stream);
/* Graph output `name` of the last run: dtype, shape (HOST array of at least 8),
 * rank and its DEVICE address, valid until the next run or destroy. */
int inferc_dev_graph_output(inferc_graph_t g, const char* name, int* dtype, int64_t* shape,
                            int* rank, const void** data);
void inferc_dev_graph_destroy(inferc_graph_t g);

/* ------------------------------------------------------------------ plans */

/* A prepared DistilBERT-architecture encoder (the `inferc optimize` plan run
 * by `inferc run`, src/cli/main.cpp:324-420). create copies the weights
 * (HOST pointers in `w`) to the current device once; run executes one
 * forward as a replayed CUDA graph per (B,S). */
typedef struct InfercEncoderPlan* inferc_encoder_t;
int inferc_dev_encoder_create(const InfercEncoderWeights* w, int64_t max_batch,
                              int64_t max_seq, inferc_encoder_t* out);
/* ids, mask: int64 [B,S] DEVICE; logits: [B, n_classes] DEVICE. */
int inferc_dev_encoder_run(inferc_encoder_t plan, const int64_t* ids,
                           const int64_t* mask, int64_t B, int64_t S,
                           float* logits, void* stream);
/* Same with HOST ids / mask / logits: copies in, runs, copies out, syncs. */
int inferc_dev_encoder_run_host(inferc_encoder_t plan, const int64_t* ids,
                                const int64_t* mask, int64_t B, int64_t S,
                                float* logits);
/* Number of batches this plan has rerun on its 3xTF32 graph because the
 * split-fp16 graph met a value fp16 cannot carry (-1 for a NULL plan). */
int64_t inferc_dev_encoder_range_fallbacks(inferc_encoder_t plan);
void inferc_dev_encoder_destroy(inferc_encoder_t plan);

/* A prepared GPT-2 greedy decoder (`inferc decode`, src/cli/main.cpp:700-945)
 * with a device-resident KV cache of max_len positions. */
typedef struct InfercDecoderPlan* inferc_decoder_t;
int inferc_dev_decoder_create(const InfercGpt2Weights* w, int64_t max_len,
                              inferc_decoder_t* out);
/* Greedy decode: prompt (HOST int64 [n_prompt]) -> tokens_out (HOST int64
 * [max_tokens]): the prefill token followed by max_tokens-1 single-token
 * steps, as `inferc decode --max-tokens` does. step_ms_out (HOST, may be NULL)
 * receives the mean device time per single-token step in milliseconds. */
int inferc_dev_decode(inferc_decoder_t plan, const int64_t* prompt,
                      int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                      double* step_ms_out);
/* Weight-only int4 variant of inferc_dev_decoder_create (no counterpart in
 * the reference's runtime, which benchmarks its int4 GEMV only,
 * bench/amx/int4_gemv_amx.cc:258-271): the four matrices of every layer and
 * the tied LM head are quantised on the device, per output row, to the int4
 * per-row-scale layout of inferc_dev_gemv_int4_rowscale (scale = max|w|/7,
 * q = clamp(rint(w/scale), -8, 7)); inferc_dev_decode then runs every
 * position (prompt included) as one single-token step of int4 row GEMVs with
 * fused LayerNorm prologues, bias / GELU / residual epilogues and the greedy
 * argmax, replayed as a CUDA graph. The result is greedy decode of the model
 * whose weights are the dequantised scale * (q - 8). */
int inferc_dev_decoder_create_int4(const InfercGpt2Weights* w, int64_t max_len,
                                   inferc_decoder_t* out);
/* The packer itself: w [K, N] fp32 (row stride ldw; trans: w is [N, K]) ->
 * out [N, K/2] int4 bytes (even k in the low nibble, stored q + 8) and
 * scales [N], as above. K even. */
int inferc_dev_int4_pack_rowscale(const float* w, int64_t K, int64_t N, int64_t ldw, int trans,
                                  uint8_t* out, float* scales, void* stream);
/* Device logits [vocab] of the most recent step (valid after decode). */
const float* inferc_dev_decoder_logits(inferc_decoder_t plan);
void inferc_dev_decoder_destroy(inferc_decoder_t plan);

#ifdef __cplusplus
}
#endif

#endif /* INFERC_DEV_H_ */
