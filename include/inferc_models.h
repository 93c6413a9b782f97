/* Weight tables for the two model plans on inferc's hot path, as plain C
 * structs of pointers so that every consumer (the device executor in
 * libinferc_b200.so, the CPU oracle, ctypes callers) shares one layout.
 *
 * Shapes follow the reference's optimized ONNX plans:
 *   - DistilBERT-architecture encoder (the `inferc optimize` + `inferc run`
 *     plan; FusedQKV / FusedAttention / FusedLayerNorm / FusedMatMulAddGELU,
 *     src/kernels/attention.h:24-34, fused_matmul_add_gelu.h:22,
 *     activation.h:26): projection weights are MatMul right operands [K,N];
 *     the classifier head is two ONNX Gemm nodes with transB=1, so those
 *     weights are [N,K].
 *   - GPT-2-small decode (`inferc decode`, src/cli/main.cpp:700-945): Conv1D
 *     weights are ONNX Gemm right operands with transB=0, i.e. [K,N]; the LM
 *     head is the token embedding used as MatMul(x, wte^T) after constant
 *     folding (src/ir/passes/constant_fold.cc:12-57).
 * Per-layer arrays hold one pointer per layer (layers <= INFERC_MAX_LAYERS).
 * Pointers are host or device addresses depending on the entry point that
 * receives the struct; the header of that entry point says which.
 */
#ifndef INFERC_MODELS_H_
#define INFERC_MODELS_H_

#include <stdint.h>

#define INFERC_MAX_LAYERS 48

typedef struct InfercEncoderWeights {
  int32_t layers, hidden, heads, ffn, vocab, max_pos, n_classes;
  float ln_eps;          /* 1e-12 for DistilBERT */
  float attn_fill;       /* FusedAttention `fill` attribute */
  const float* word_emb; /* [vocab, hidden] */
  const float* pos_emb;  /* [max_pos, hidden] */
  const float* emb_ln_g; /* [hidden] */
  const float* emb_ln_b;
  const float* wq[INFERC_MAX_LAYERS]; /* [hidden, hidden] */
  const float* bq[INFERC_MAX_LAYERS];
  const float* wk[INFERC_MAX_LAYERS];
  const float* bk[INFERC_MAX_LAYERS];
  const float* wv[INFERC_MAX_LAYERS];
  const float* bv[INFERC_MAX_LAYERS];
  const float* wo[INFERC_MAX_LAYERS]; /* [hidden, hidden] */
  const float* bo[INFERC_MAX_LAYERS];
  const float* ln1_g[INFERC_MAX_LAYERS]; /* sa_layer_norm */
  const float* ln1_b[INFERC_MAX_LAYERS];
  const float* w1[INFERC_MAX_LAYERS]; /* [hidden, ffn] */
  const float* b1[INFERC_MAX_LAYERS];
  const float* w2[INFERC_MAX_LAYERS]; /* [ffn, hidden] */
  const float* b2[INFERC_MAX_LAYERS];
  const float* ln2_g[INFERC_MAX_LAYERS]; /* output_layer_norm */
  const float* ln2_b[INFERC_MAX_LAYERS];
  const float* pre_w; /* [hidden, hidden] as [N,K] (Gemm transB=1) */
  const float* pre_b; /* [hidden] */
  const float* cls_w; /* [n_classes, hidden] as [N,K] */
  const float* cls_b; /* [n_classes] */
} InfercEncoderWeights;

typedef struct InfercGpt2Weights {
  int32_t layers, hidden, heads, ffn, vocab, max_pos;
  float ln_eps;     /* 1e-5 for GPT-2 */
  const float* wte; /* [vocab, hidden]; also the tied LM head */
  const float* wpe; /* [max_pos, hidden] */
  const float* ln1_g[INFERC_MAX_LAYERS];
  const float* ln1_b[INFERC_MAX_LAYERS];
  const float* attn_w[INFERC_MAX_LAYERS]; /* [hidden, 3*hidden] */
  const float* attn_b[INFERC_MAX_LAYERS];
  const float* proj_w[INFERC_MAX_LAYERS]; /* [hidden, hidden] */
  const float* proj_b[INFERC_MAX_LAYERS];
  const float* ln2_g[INFERC_MAX_LAYERS];
  const float* ln2_b[INFERC_MAX_LAYERS];
  const float* fc_w[INFERC_MAX_LAYERS]; /* [hidden, ffn] */
  const float* fc_b[INFERC_MAX_LAYERS];
  const float* fcproj_w[INFERC_MAX_LAYERS]; /* [ffn, hidden] */
  const float* fcproj_b[INFERC_MAX_LAYERS];
  const float* lnf_g;
  const float* lnf_b;
} InfercGpt2Weights;

#endif /* INFERC_MODELS_H_ */
