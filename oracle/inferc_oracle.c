/* CPU restatement ("port") of inferc's fused-op hot path. TEST
 * INFRASTRUCTURE ONLY; see inferc_oracle.h for the rules on who may call it.
 * Written from the reference's algorithm, not its code: the reference runs
 * these steps through Accelerate (cblas_sgemm / vDSP / vForce); this file
 * spells the same arithmetic out as scalar loops. */
#include "inferc_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- kernels */

/* activation.cc:134-148: mean, x-mean, biased var of the centred row,
 * inv = 1/sqrtf(var+eps), y = (xc*inv)*gamma + beta. */
void orc_layernorm(const float* x, const float* gamma, const float* beta,
                   float* y, int64_t rows, int64_t feat, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * feat;
    float* yr = y + r * feat;
    float s = 0.0f;
    for (int64_t i = 0; i < feat; ++i) s += xr[i];
    const float mean = s / (float)feat;
    for (int64_t i = 0; i < feat; ++i) yr[i] = xr[i] + (-mean);
    float sq = 0.0f;
    for (int64_t i = 0; i < feat; ++i) sq += yr[i] * yr[i];
    const float var = sq / (float)feat;
    const float inv = 1.0f / sqrtf(var + eps);
    for (int64_t i = 0; i < feat; ++i) yr[i] = (yr[i] * inv) * gamma[i] + beta[i];
  }
}

/* activation.cc:25-27 */
void orc_gelu(const float* x, float* y, int64_t n) {
  const float kInvSqrt2 = 0.70710678118654752440f;
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * 0.5f * (1.0f + erff(x[i] * kInvSqrt2));
}

/* activation.cc:42-48 */
void orc_gelu_tanh(const float* x, float* y, int64_t n) {
  const float kSqrt2OverPi = 0.7978845608028654f, kCoef = 0.044715f;
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    const float inner = kSqrt2OverPi * (v + kCoef * v * v * v);
    y[i] = 0.5f * v * (1.0f + tanhf(inner));
  }
}

/* activation.cc:75-95: max from -inf, exp(x - max), sum, multiply by 1/sum. */
void orc_softmax(const float* x, float* y, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * cols;
    float* yr = y + r * cols;
    float m = -INFINITY;
    for (int64_t j = 0; j < cols; ++j) m = xr[j] > m ? xr[j] : m;
    float sum = 0.0f;
    for (int64_t j = 0; j < cols; ++j) {
      yr[j] = expf(xr[j] - m);
      sum += yr[j];
    }
    const float inv = 1.0f / sum;
    for (int64_t j = 0; j < cols; ++j) yr[j] *= inv;
  }
}

void orc_sgemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K,
               float alpha, const float* A, int64_t lda, const float* B,
               int64_t ldb, float beta, float* C, int64_t ldc) {
  float* acc = (float*)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
  for (int64_t i = 0; i < M; ++i) {
    for (int64_t j = 0; j < N; ++j) acc[j] = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      const float a = trans_a ? A[k * lda + i] : A[i * lda + k];
      if (!trans_b) {
        const float* br = B + k * ldb;
        for (int64_t j = 0; j < N; ++j) acc[j] += a * br[j];
      } else {
        for (int64_t j = 0; j < N; ++j) acc[j] += a * B[j * ldb + k];
      }
    }
    float* cr = C + i * ldc;
    for (int64_t j = 0; j < N; ++j)
      cr[j] = beta == 0.0f ? alpha * acc[j] : alpha * acc[j] + beta * cr[j];
  }
  free(acc);
}

/* matmul.cc:161-228: out pre-filled with C (full, [N] row broadcast or
 * scalar) when beta != 0, then out = alpha*op(A)op(B) + beta*out. */
int orc_gemm(const float* a, const float* b, const float* c, int64_t c_len,
             float* y, int64_t M, int64_t K, int64_t N, float alpha,
             float beta, int trans_a, int trans_b) {
  memset(y, 0, (size_t)(M * N) * sizeof(float));
  if (c != NULL && beta != 0.0f) {
    if (c_len == M * N) {
      memcpy(y, c, (size_t)(M * N) * sizeof(float));
    } else if (c_len == N) {
      for (int64_t i = 0; i < M; ++i) memcpy(y + i * N, c, (size_t)N * sizeof(float));
    } else if (c_len == 1) {
      for (int64_t i = 0; i < M * N; ++i) y[i] = c[0];
    } else {
      return -1;
    }
  }
  orc_sgemm(trans_a, trans_b, M, N, K, alpha, a, trans_a ? M : K, b,
            trans_b ? K : N, beta, y, N);
  return 0;
}

/* fused_matmul_add_gelu.cc:67-77: sgemm, then v = acc + b[c],
 * y = v*0.5*(1+erf(v*0.70710678f)). */
void orc_fused_matmul_add_gelu(const float* x, const float* w, const float* b,
                               float* y, int64_t M, int64_t K, int64_t N) {
  const float kInvSqrt2 = 0.70710678118654752440f;
  orc_sgemm(0, 0, M, N, K, 1.0f, x, K, w, N, 0.0f, y, N);
  for (int64_t r = 0; r < M; ++r)
    for (int64_t c = 0; c < N; ++c) {
      const float v = y[r * N + c] + b[c];
      y[r * N + c] = v * 0.5f * (1.0f + erff(v * kInvSqrt2));
    }
}

/* attention.cc:126-139: three sgemms sharing X, then += bias per row. */
void orc_fused_qkv(const float* x, const float* wq, const float* bq,
                   const float* wk, const float* bk, const float* wv,
                   const float* bv, float* q, float* k, float* v, int64_t M,
                   int64_t K, int64_t N) {
  const float* ws[3] = {wq, wk, wv};
  const float* bs[3] = {bq, bk, bv};
  float* os[3] = {q, k, v};
  for (int i = 0; i < 3; ++i) {
    orc_sgemm(0, 0, M, N, K, 1.0f, x, K, ws[i], N, 0.0f, os[i], N);
    for (int64_t r = 0; r < M; ++r)
      for (int64_t c = 0; c < N; ++c) os[i][r * N + c] += bs[i][c];
  }
}

/* attention.cc:17-29: element stride of each axis of a right-aligned mask
 * shape broadcast to [B,nH,S,S]; 0 on broadcast axes. */
static void mask_strides(const int64_t* shape, int rank, int64_t s[4]) {
  int64_t st = 1;
  s[0] = s[1] = s[2] = s[3] = 0;
  for (int i = rank - 1; i >= 0; --i) {
    const int od = 4 - (rank - i);
    if (od >= 0) s[od] = (shape[i] == 1) ? 0 : st;
    st *= shape[i];
  }
}

/* attention.cc:59-98, per (b,h): scores = scale*Q_h K_h^T; masked entries
 * replaced by fill; row max starts at row[0]; row - max; exp; sum;
 * multiply by 1/sum; context = P V_h written at the head's columns. */
void orc_fused_attention(const float* q, const float* k, const float* v,
                         const uint8_t* mask, const int64_t* mask_shape,
                         int mask_rank, int64_t B, int64_t S, int64_t H,
                         int64_t head_dim, float fill, float* out) {
  const int64_t nH = H / head_dim;
  const float scale = 1.0f / sqrtf((float)head_dim);
  const int have_mask = mask != NULL && mask_rank > 0;
  int64_t ms[4] = {0, 0, 0, 0};
  if (have_mask) mask_strides(mask_shape, mask_rank, ms);
  float* row = (float*)malloc((size_t)S * sizeof(float));
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < nH; ++h) {
      const float* Qh = q + b * S * H + h * head_dim;
      const float* Kh = k + b * S * H + h * head_dim;
      const float* Vh = v + b * S * H + h * head_dim;
      float* Oh = out + b * S * H + h * head_dim;
      for (int64_t i = 0; i < S; ++i) {
        for (int64_t j = 0; j < S; ++j) {
          float acc = 0.0f;
          for (int64_t d = 0; d < head_dim; ++d) acc += Qh[i * H + d] * Kh[j * H + d];
          row[j] = scale * acc;
        }
        if (have_mask)
          for (int64_t j = 0; j < S; ++j)
            if (mask[b * ms[0] + h * ms[1] + i * ms[2] + j * ms[3]]) row[j] = fill;
        float m = row[0];
        for (int64_t j = 1; j < S; ++j) m = row[j] > m ? row[j] : m;
        for (int64_t j = 0; j < S; ++j) row[j] += -m;
        float sum = 0.0f;
        for (int64_t j = 0; j < S; ++j) {
          row[j] = expf(row[j]);
          sum += row[j];
        }
        const float inv = 1.0f / sum;
        for (int64_t j = 0; j < S; ++j) row[j] *= inv;
        for (int64_t d = 0; d < head_dim; ++d) {
          float acc = 0.0f;
          for (int64_t j = 0; j < S; ++j) acc += row[j] * Vh[j * H + d];
          Oh[i * H + d] = acc;
        }
      }
    }
  free(row);
}

/* int4_gemv_amx.cc:258-271 */
void orc_int4_gemv_rowscale(const uint8_t* w, const float* scales,
                            const float* x, float* y, int64_t N, int64_t K) {
  for (int64_t r = 0; r < N; ++r) {
    double acc = 0.0;
    const float s = scales[r];
    for (int64_t k = 0; k < K; ++k) {
      const uint8_t byte = w[r * (K / 2) + k / 2];
      const int nib = (k & 1) ? (byte >> 4) : (byte & 0xf);
      acc += (double)(s * (float)(nib - 8)) * (double)x[k];
    }
    y[r] = (float)acc;
  }
}

/* int4_gemv_amx.cc:243-255 */
void orc_int4_gemv(const uint8_t* w, float scale, const float* x, float* y,
                   int64_t N, int64_t K) {
  for (int64_t r = 0; r < N; ++r) {
    double acc = 0.0;
    for (int64_t k = 0; k < K; ++k) {
      const uint8_t byte = w[r * (K / 2) + k / 2];
      const int nib = (k & 1) ? (byte >> 4) : (byte & 0xf);
      acc += (double)(scale * (float)(nib - 8)) * (double)x[k];
    }
    y[r] = (float)acc;
  }
}

/* main.cpp:823-829: best = x[0], strict > keeps the first maximum. */
int64_t orc_argmax(const float* x, int64_t n) {
  int64_t best_i = 0;
  float best = x[0];
  for (int64_t i = 1; i < n; ++i)
    if (x[i] > best) {
      best = x[i];
      best_i = i;
    }
  return best_i;
}

/* ---------------------------------------------------------------- encoder */

static void add_rows_bias(float* y, const float* b, int64_t M, int64_t N) {
  for (int64_t r = 0; r < M; ++r)
    for (int64_t c = 0; c < N; ++c) y[r * N + c] += b[c];
}

int orc_encoder_forward(const InfercEncoderWeights* w, const int64_t* ids,
                        const int64_t* mask, int64_t B, int64_t S,
                        float* logits) {
  const int64_t H = w->hidden, F = w->ffn, M = B * S, C = w->n_classes;
  if (S > w->max_pos) return -1;
  float* x = (float*)malloc((size_t)(M * H) * sizeof(float));
  float* t = (float*)malloc((size_t)(M * H) * sizeof(float));
  float* q = (float*)malloc((size_t)(M * H) * sizeof(float));
  float* k = (float*)malloc((size_t)(M * H) * sizeof(float));
  float* v = (float*)malloc((size_t)(M * H) * sizeof(float));
  float* ctx = (float*)malloc((size_t)(M * H) * sizeof(float));
  float* hf = (float*)malloc((size_t)(M * F) * sizeof(float));
  uint8_t* cond = (uint8_t*)malloc((size_t)M);
  int rc = 0;
  /* Gather(word) + Gather(position), then LayerNorm. */
  for (int64_t b = 0; b < B; ++b)
    for (int64_t s = 0; s < S; ++s) {
      int64_t id = ids[b * S + s];
      if (id < 0) id += w->vocab;
      if (id < 0 || id >= w->vocab) {
        rc = -1;
        goto done;
      }
      for (int64_t c = 0; c < H; ++c)
        t[(b * S + s) * H + c] = w->word_emb[id * H + c] + w->pos_emb[s * H + c];
    }
  orc_layernorm(t, w->emb_ln_g, w->emb_ln_b, x, M, H, w->ln_eps);
  /* mask_cond = (attention_mask == 0), shape [B,1,1,S]. */
  for (int64_t i = 0; i < M; ++i) cond[i] = mask[i] == 0;
  const int64_t mshape[4] = {B, 1, 1, S};
  for (int l = 0; l < w->layers; ++l) {
    orc_fused_qkv(x, w->wq[l], w->bq[l], w->wk[l], w->bk[l], w->wv[l], w->bv[l],
                  q, k, v, M, H, H);
    orc_fused_attention(q, k, v, cond, mshape, 4, B, S, H, H / w->heads,
                        w->attn_fill, ctx);
    orc_sgemm(0, 0, M, H, H, 1.0f, ctx, H, w->wo[l], H, 0.0f, t, H);
    add_rows_bias(t, w->bo[l], M, H);
    for (int64_t i = 0; i < M * H; ++i) t[i] = t[i] + x[i];
    orc_layernorm(t, w->ln1_g[l], w->ln1_b[l], x, M, H, w->ln_eps);
    orc_fused_matmul_add_gelu(x, w->w1[l], w->b1[l], hf, M, H, F);
    orc_sgemm(0, 0, M, H, F, 1.0f, hf, F, w->w2[l], H, 0.0f, t, H);
    add_rows_bias(t, w->b2[l], M, H);
    for (int64_t i = 0; i < M * H; ++i) t[i] = t[i] + x[i];
    orc_layernorm(t, w->ln2_g[l], w->ln2_b[l], x, M, H, w->ln_eps);
  }
  /* Gather CLS (seq index 0) -> Gemm(transB=1)+Relu -> Gemm(transB=1). */
  for (int64_t b = 0; b < B; ++b) memcpy(q + b * H, x + b * S * H, (size_t)H * sizeof(float));
  orc_gemm(q, w->pre_w, w->pre_b, H, k, B, H, H, 1.0f, 1.0f, 0, 1);
  for (int64_t i = 0; i < B * H; ++i) k[i] = k[i] > 0.0f ? k[i] : 0.0f;
  orc_gemm(k, w->cls_w, w->cls_b, C, logits, B, H, C, 1.0f, 1.0f, 0, 1);
done:
  free(x); free(t); free(q); free(k); free(v); free(ctx); free(hf); free(cond);
  return rc;
}

/* ------------------------------------------------------------------ GPT-2 */

typedef struct {
  float* k; /* [layers][heads][max_len][hd] */
  float* v;
  int64_t max_len;
} KvCache;

/* One forward over n new tokens at positions [pos0, pos0+n), appending their
 * K/V to the cache; writes the logits of the last token to `logits`. Causal
 * masking inside the new block; all cached positions visible. */
static void gpt2_forward(const InfercGpt2Weights* w, const float* lm, KvCache* kv,
                         const int64_t* toks, int64_t n, int64_t pos0,
                         float* logits) {
  const int64_t H = w->hidden, F = w->ffn, nH = w->heads, hd = H / nH;
  const int64_t L = pos0 + n;
  float* x = (float*)malloc((size_t)(n * H) * sizeof(float));
  float* h = (float*)malloc((size_t)(n * H) * sizeof(float));
  float* qkv = (float*)malloc((size_t)(n * 3 * H) * sizeof(float));
  float* ctx = (float*)malloc((size_t)(n * H) * sizeof(float));
  float* a = (float*)malloc((size_t)(n * H) * sizeof(float));
  float* f = (float*)malloc((size_t)(n * F) * sizeof(float));
  float* g = (float*)malloc((size_t)(n * F) * sizeof(float));
  float* sc = (float*)malloc((size_t)L * sizeof(float));
  float* p = (float*)malloc((size_t)L * sizeof(float));
  for (int64_t i = 0; i < n; ++i)
    for (int64_t c = 0; c < H; ++c)
      x[i * H + c] = w->wte[toks[i] * H + c] + w->wpe[(pos0 + i) * H + c];
  for (int l = 0; l < w->layers; ++l) {
    orc_layernorm(x, w->ln1_g[l], w->ln1_b[l], h, n, H, w->ln_eps);
    orc_gemm(h, w->attn_w[l], w->attn_b[l], 3 * H, qkv, n, H, 3 * H, 1.0f, 1.0f, 0, 0);
    float* kc = kv->k + (int64_t)l * nH * kv->max_len * hd;
    float* vc = kv->v + (int64_t)l * nH * kv->max_len * hd;
    for (int64_t i = 0; i < n; ++i)
      for (int64_t hh = 0; hh < nH; ++hh)
        for (int64_t d = 0; d < hd; ++d) {
          kc[(hh * kv->max_len + pos0 + i) * hd + d] = qkv[i * 3 * H + H + hh * hd + d];
          vc[(hh * kv->max_len + pos0 + i) * hd + d] = qkv[i * 3 * H + 2 * H + hh * hd + d];
        }
    for (int64_t i = 0; i < n; ++i)
      for (int64_t hh = 0; hh < nH; ++hh) {
        const float* qi = qkv + i * 3 * H + hh * hd;
        const int64_t visible = pos0 + i + 1;
        for (int64_t j = 0; j < L; ++j) {
          if (j < visible) {
            float acc = 0.0f;
            for (int64_t d = 0; d < hd; ++d) acc += qi[d] * kc[(hh * kv->max_len + j) * hd + d];
            sc[j] = acc / sqrtf((float)hd);
          } else {
            sc[j] = -FLT_MAX; /* Where(causal, scores, finfo.min) */
          }
        }
        orc_softmax(sc, p, 1, L);
        for (int64_t d = 0; d < hd; ++d) {
          float acc = 0.0f;
          for (int64_t j = 0; j < L; ++j) acc += p[j] * vc[(hh * kv->max_len + j) * hd + d];
          ctx[i * H + hh * hd + d] = acc;
        }
      }
    orc_gemm(ctx, w->proj_w[l], w->proj_b[l], H, a, n, H, H, 1.0f, 1.0f, 0, 0);
    for (int64_t i = 0; i < n * H; ++i) x[i] = a[i] + x[i];
    orc_layernorm(x, w->ln2_g[l], w->ln2_b[l], h, n, H, w->ln_eps);
    orc_gemm(h, w->fc_w[l], w->fc_b[l], F, f, n, H, F, 1.0f, 1.0f, 0, 0);
    orc_gelu_tanh(f, g, n * F);
    orc_gemm(g, w->fcproj_w[l], w->fcproj_b[l], H, a, n, F, H, 1.0f, 1.0f, 0, 0);
    for (int64_t i = 0; i < n * H; ++i) x[i] = x[i] + a[i];
  }
  orc_layernorm(x + (n - 1) * H, w->lnf_g, w->lnf_b, h, 1, H, w->ln_eps);
  /* LM head: MatMul(x, wte^T) */
  orc_sgemm(0, 1, 1, w->vocab, H, 1.0f, h, H, lm, H, 0.0f, logits, w->vocab);
  free(x); free(h); free(qkv); free(ctx); free(a); free(f); free(g); free(sc); free(p);
}

static float top2_margin(const float* x, int64_t n, int64_t best) {
  float second = -INFINITY;
  for (int64_t i = 0; i < n; ++i)
    if (i != best && x[i] > second) second = x[i];
  return x[best] - second;
}

/* Greedy decode with the LM head `lm` ([vocab, hidden]; the tied wte in
 * GPT-2, its int4 round trip for the weight-only int4 decoder). */
int orc_gpt2_decode_lm(const InfercGpt2Weights* w, const float* lm, const int64_t* prompt,
                       int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                       float* margins_out) {
  if (n_prompt <= 0 || max_tokens <= 0 || n_prompt + max_tokens - 1 > w->max_pos) return -1;
  for (int64_t i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= w->vocab) return -1;
  const int64_t hd = w->hidden / w->heads;
  KvCache kv;
  kv.max_len = n_prompt + max_tokens;
  const size_t cache = (size_t)w->layers * w->heads * kv.max_len * hd;
  kv.k = (float*)calloc(cache, sizeof(float));
  kv.v = (float*)calloc(cache, sizeof(float));
  float* logits = (float*)malloc((size_t)w->vocab * sizeof(float));
  gpt2_forward(w, lm, &kv, prompt, n_prompt, 0, logits);
  int64_t tok = orc_argmax(logits, w->vocab);
  tokens_out[0] = tok;
  if (margins_out) margins_out[0] = top2_margin(logits, w->vocab, tok);
  for (int64_t step = 1; step < max_tokens; ++step) {
    gpt2_forward(w, lm, &kv, &tok, 1, n_prompt + step - 1, logits);
    tok = orc_argmax(logits, w->vocab);
    tokens_out[step] = tok;
    if (margins_out) margins_out[step] = top2_margin(logits, w->vocab, tok);
  }
  free(kv.k); free(kv.v); free(logits);
  return 0;
}

int orc_gpt2_decode(const InfercGpt2Weights* w, const int64_t* prompt,
                    int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                    float* margins_out) {
  return orc_gpt2_decode_lm(w, w->wte, prompt, n_prompt, max_tokens, tokens_out, margins_out);
}
