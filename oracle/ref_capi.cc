// extern "C" wrappers that drive the reference's OWN kernel sources
// (src/kernels/*.cc, src/runtime/tensor.cc, compiled by oracle/Makefile into
// oracle/_ref/libinferc_ref.so) on raw buffers. TEST INFRASTRUCTURE ONLY: it
// is the parity oracle and the timed CPU baseline ("kind": "reference"), never
// part of the product.
//
// The model-level functions replay the node sequence of the reference's plans
// with the reference kernels, in the order Executor::Run would visit them
// (src/runtime/executor.cc:123-343):
//   encoder: Gather+Gather+Add, FusedLayerNorm, then per layer FusedQKV,
//            FusedAttention, MatMul, Add, Add, FusedLayerNorm,
//            FusedMatMulAddGELU, MatMul, Add, Add, FusedLayerNorm; then
//            Gather(CLS), Gemm(transB=1), Relu, Gemm(transB=1).
//   decode:  `inferc decode` (src/cli/main.cpp:700-945): prefill graph, then a
//            with-past graph per token; per layer FusedLayerNorm, Gemm,
//            Split, Reshape/Transpose, Concat(past, new), MatMul, Div,
//            Where(causal), Softmax, MatMul, Transpose/Reshape, Gemm, Add,
//            FusedLayerNorm, Gemm, GeluTanh, Gemm, Add; final FusedLayerNorm
//            and MatMul(x, wte^T); argmax with the first maximum winning.
// The all-ones attention mask of the decode graphs is an additive zero and is
// not replayed.
#include <cfloat>
#include <cmath>
#include <chrono>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "../include/inferc_models.h"
#include "kernels/activation.h"
#include "kernels/attention.h"
#include "kernels/elementwise.h"
#include "kernels/embedding.h"
#include "kernels/fused_matmul_add_gelu.h"
#include "kernels/matmul.h"
#include "kernels/movement.h"
#include "runtime/tensor.h"

using inferc::DType;
using inferc::Shape;
using inferc::rt::Tensor;
namespace rt = inferc::rt;

namespace {
thread_local std::string g_err;

Tensor F32(Shape s, const float* p) {
  return Tensor::FromHostBytes(DType::kFloat32, std::move(s), p);
}
Tensor I64(Shape s, const int64_t* p) {
  return Tensor::FromHostBytes(DType::kInt64, std::move(s), p);
}
void Out(const Tensor& t, float* dst) {
  Tensor c = t.Contiguous();
  std::memcpy(dst, c.bytes(), static_cast<size_t>(c.byte_size()));
}

template <typename Fn>
int Guard(Fn&& fn) {
  try {
    fn();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_layernorm(const float* x, const float* g, const float* b, float* y,
                  int64_t rows, int64_t feat, float eps) {
  return Guard([&] {
    Out(rt::LayerNorm(F32({rows, feat}, x), F32({feat}, g), F32({feat}, b), eps, 1), y);
  });
}

int ref_gelu(const float* x, float* y, int64_t n) {
  return Guard([&] { Out(rt::Gelu(F32({n}, x)), y); });
}

int ref_gelu_tanh(const float* x, float* y, int64_t n) {
  return Guard([&] { Out(rt::GeluTanh(F32({n}, x)), y); });
}

int ref_softmax(const float* x, float* y, int64_t rows, int64_t cols) {
  return Guard([&] { Out(rt::Softmax(F32({rows, cols}, x), -1), y); });
}

int ref_fused_matmul_add_gelu(const float* x, const float* w, const float* b,
                              float* y, int64_t M, int64_t K, int64_t N) {
  return Guard([&] {
    Out(rt::FusedMatMulAddGELU(F32({M, K}, x), F32({K, N}, w), F32({N}, b)), y);
  });
}

int ref_fused_qkv(const float* x, const float* wq, const float* bq,
                  const float* wk, const float* bk, const float* wv,
                  const float* bv, float* q, float* k, float* v, int64_t M,
                  int64_t K, int64_t N) {
  return Guard([&] {
    auto r = rt::FusedQKVProjection(F32({M, K}, x), F32({K, N}, wq), F32({N}, bq),
                                    F32({K, N}, wk), F32({N}, bk), F32({K, N}, wv),
                                    F32({N}, bv));
    Out(r[0], q);
    Out(r[1], k);
    Out(r[2], v);
  });
}

int ref_fused_attention(const float* q, const float* k, const float* v,
                        const uint8_t* mask, const int64_t* mask_shape,
                        int mask_rank, int64_t B, int64_t S, int64_t H,
                        int64_t head_dim, float fill, float* out) {
  return Guard([&] {
    Tensor m;
    if (mask != nullptr && mask_rank > 0) {
      Shape ms(mask_shape, mask_shape + mask_rank);
      m = Tensor::FromHostBytes(DType::kBool, ms, mask);
    }
    Out(rt::FusedAttention(F32({B, S, H}, q), F32({B, S, H}, k), F32({B, S, H}, v), m,
                           head_dim, fill),
        out);
  });
}

int ref_gemm(const float* a, const float* b, const float* c, int64_t c_len,
             float* y, int64_t M, int64_t K, int64_t N, float alpha, float beta,
             int trans_a, int trans_b) {
  return Guard([&] {
    Tensor ta = trans_a ? F32({K, M}, a) : F32({M, K}, a);
    Tensor tb = trans_b ? F32({N, K}, b) : F32({K, N}, b);
    Tensor tc;
    if (c != nullptr) tc = (c_len == M * N) ? F32({M, N}, c) : F32({c_len}, c);
    Out(rt::Gemm(ta, tb, c ? &tc : nullptr, alpha, beta, trans_a != 0, trans_b != 0), y);
  });
}

int ref_matmul(const float* a, const float* b, float* y, int64_t M, int64_t K,
               int64_t N) {
  return Guard([&] { Out(rt::MatMul(F32({M, K}, a), F32({K, N}, b)), y); });
}

int ref_encoder_forward(const InfercEncoderWeights* w, const int64_t* ids,
                        const int64_t* mask, int64_t B, int64_t S, float* logits) {
  return Guard([&] {
    const int64_t H = w->hidden, F = w->ffn, C = w->n_classes;
    Tensor word = F32({w->vocab, H}, w->word_emb);
    Tensor pos = F32({w->max_pos, H}, w->pos_emb);
    Tensor tids = I64({B, S}, ids);
    std::vector<int64_t> ar(static_cast<size_t>(S));
    for (int64_t i = 0; i < S; ++i) ar[static_cast<size_t>(i)] = i;
    Tensor x = rt::Add(rt::Gather(word, tids, 0), rt::Gather(pos, I64({S}, ar.data()), 0));
    x = rt::LayerNorm(x, F32({H}, w->emb_ln_g), F32({H}, w->emb_ln_b), w->ln_eps, 1);
    Tensor cond(DType::kBool, {B, 1, 1, S});
    for (int64_t i = 0; i < B * S; ++i) cond.data<uint8_t>()[i] = mask[i] == 0;
    for (int l = 0; l < w->layers; ++l) {
      auto qkv = rt::FusedQKVProjection(x, F32({H, H}, w->wq[l]), F32({H}, w->bq[l]),
                                        F32({H, H}, w->wk[l]), F32({H}, w->bk[l]),
                                        F32({H, H}, w->wv[l]), F32({H}, w->bv[l]));
      Tensor ctx = rt::FusedAttention(qkv[0], qkv[1], qkv[2], cond, H / w->heads,
                                      w->attn_fill);
      Tensor sa = rt::Add(rt::MatMul(ctx, F32({H, H}, w->wo[l])), F32({H}, w->bo[l]));
      sa = rt::Add(sa, x);
      x = rt::LayerNorm(sa, F32({H}, w->ln1_g[l]), F32({H}, w->ln1_b[l]), w->ln_eps, 1);
      Tensor hf = rt::FusedMatMulAddGELU(x, F32({H, F}, w->w1[l]), F32({F}, w->b1[l]));
      Tensor ff = rt::Add(rt::MatMul(hf, F32({F, H}, w->w2[l])), F32({H}, w->b2[l]));
      ff = rt::Add(ff, x);
      x = rt::LayerNorm(ff, F32({H}, w->ln2_g[l]), F32({H}, w->ln2_b[l]), w->ln_eps, 1);
    }
    const int64_t zero = 0;
    Tensor cls = rt::Gather(x, I64({}, &zero), 1);  // [B, H]
    Tensor pre_b = F32({H}, w->pre_b), cls_b = F32({C}, w->cls_b);
    Tensor p = rt::Relu(rt::Gemm(cls, F32({H, H}, w->pre_w), &pre_b, 1.0f, 1.0f, false, true));
    Out(rt::Gemm(p, F32({C, H}, w->cls_w), &cls_b, 1.0f, 1.0f, false, true), logits);
  });
}

namespace {

struct Gpt2Ref {
  const InfercGpt2Weights* w;
  const float* lm_head;  // [vocab, hidden]: wte (tied) or its int4 round trip
  std::vector<Tensor> past_k, past_v;  // [1, nH, L, hd] per layer

  // One graph run over n tokens at positions [pos0, pos0+n). Returns the
  // logits of the last token.
  Tensor Run(const std::vector<int64_t>& toks, int64_t pos0) {
    const int64_t H = w->hidden, F = w->ffn, nH = w->heads, hd = H / nH;
    const int64_t n = static_cast<int64_t>(toks.size());
    std::vector<int64_t> posv(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) posv[static_cast<size_t>(i)] = pos0 + i;
    Tensor x = rt::Add(rt::Gather(F32({w->vocab, H}, w->wte), I64({1, n}, toks.data()), 0),
                       rt::Gather(F32({w->max_pos, H}, w->wpe), I64({1, n}, posv.data()), 0));
    const float eight = std::sqrt(static_cast<float>(hd));
    Tensor div = F32({}, &eight);
    const float fmin = -FLT_MAX;
    Tensor fill = F32({}, &fmin);
    const bool first = past_k.empty();
    if (first) {
      past_k.resize(static_cast<size_t>(w->layers));
      past_v.resize(static_cast<size_t>(w->layers));
    }
    for (int l = 0; l < w->layers; ++l) {
      Tensor h = rt::LayerNorm(x, F32({H}, w->ln1_g[l]), F32({H}, w->ln1_b[l]), w->ln_eps, 1);
      Tensor ab = F32({3 * H}, w->attn_b[l]);
      Tensor qkv = rt::Gemm(rt::Reshape(h, {n, H}), F32({H, 3 * H}, w->attn_w[l]), &ab,
                            1.0f, 1.0f, false, false);
      auto parts = rt::Split(rt::Reshape(qkv, {1, n, 3 * H}), 2, {H, H, H});
      auto heads = [&](const Tensor& t) {
        return rt::Transpose(rt::Reshape(t, {1, n, nH, hd}), {0, 2, 1, 3});
      };
      Tensor q = heads(parts[0]);
      Tensor k = heads(parts[1]);
      Tensor v = heads(parts[2]);
      if (!first) {
        k = rt::Concat({past_k[static_cast<size_t>(l)], k}, 2);
        v = rt::Concat({past_v[static_cast<size_t>(l)], v}, 2);
      }
      past_k[static_cast<size_t>(l)] = k.Contiguous();
      past_v[static_cast<size_t>(l)] = v.Contiguous();
      const int64_t L = k.shape()[2];
      Tensor s = rt::Div(rt::MatMul(q, rt::Transpose(k, {0, 1, 3, 2})), div);
      if (n > 1) {
        Tensor causal(DType::kBool, {1, 1, n, L});
        for (int64_t i = 0; i < n; ++i)
          for (int64_t j = 0; j < L; ++j) causal.data<uint8_t>()[i * L + j] = j <= pos0 + i;
        s = rt::Where(causal, s, fill);
      }
      Tensor p = rt::Softmax(s, -1);
      Tensor ctx = rt::Reshape(rt::Transpose(rt::MatMul(p, v), {0, 2, 1, 3}), {n, H});
      Tensor pb = F32({H}, w->proj_b[l]);
      Tensor a = rt::Gemm(ctx, F32({H, H}, w->proj_w[l]), &pb, 1.0f, 1.0f, false, false);
      x = rt::Add(rt::Reshape(a, {1, n, H}), x);
      h = rt::LayerNorm(x, F32({H}, w->ln2_g[l]), F32({H}, w->ln2_b[l]), w->ln_eps, 1);
      Tensor fb = F32({F}, w->fc_b[l]), fpb = F32({H}, w->fcproj_b[l]);
      Tensor f = rt::Gemm(rt::Reshape(h, {n, H}), F32({H, F}, w->fc_w[l]), &fb, 1.0f, 1.0f,
                          false, false);
      f = rt::GeluTanh(f);
      Tensor m = rt::Gemm(f, F32({F, H}, w->fcproj_w[l]), &fpb, 1.0f, 1.0f, false, false);
      x = rt::Add(x, rt::Reshape(m, {1, n, H}));
    }
    x = rt::LayerNorm(x, F32({H}, w->lnf_g), F32({H}, w->lnf_b), w->ln_eps, 1);
    Tensor last = rt::Slice(x, {n - 1}, {n}, {1}, {});
    return rt::MatMul(last, Lm());
  }

  // The folded Transpose(wte) initializer, computed once per decode.
  Tensor lm_;
  const Tensor& Lm() {
    if (lm_.shape().empty())
      lm_ = rt::Transpose(F32({w->vocab, w->hidden}, lm_head), {1, 0}).Contiguous();
    return lm_;
  }
};

int64_t ArgmaxFirst(const float* p, int64_t n, float* margin) {
  int64_t best_i = 0;
  float best = p[0];
  for (int64_t i = 1; i < n; ++i)
    if (p[i] > best) { best = p[i]; best_i = i; }
  if (margin) {
    float second = -INFINITY;
    for (int64_t i = 0; i < n; ++i)
      if (i != best_i && p[i] > second) second = p[i];
    *margin = best - second;
  }
  return best_i;
}

}  // namespace

// Greedy decode through the reference kernels. step_ms_out (may be NULL)
// receives the mean wall-clock ms of the max_tokens-1 single-token steps, the
// number `inferc decode` reports (main.cpp:862-868, :903-909).
// lm: the LM head [vocab, hidden] (the tied wte; its int4 round trip for the
// weight-only int4 decoder).
int ref_gpt2_decode_lm(const InfercGpt2Weights* w, const float* lm, const int64_t* prompt,
                       int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                       float* margins_out, double* step_ms_out) {
  return Guard([&] {
    Gpt2Ref g{w, lm, {}, {}, Tensor()};
    g.Lm();
    std::vector<int64_t> p(prompt, prompt + n_prompt);
    Tensor lg = g.Run(p, 0).Contiguous();
    int64_t tok = ArgmaxFirst(lg.data<float>(), w->vocab, margins_out);
    tokens_out[0] = tok;
    double total = 0.0;
    for (int64_t step = 1; step < max_tokens; ++step) {
      auto t0 = std::chrono::steady_clock::now();
      lg = g.Run({tok}, n_prompt + step - 1).Contiguous();
      auto t1 = std::chrono::steady_clock::now();
      total += std::chrono::duration<double, std::milli>(t1 - t0).count();
      tok = ArgmaxFirst(lg.data<float>(), w->vocab, margins_out ? margins_out + step : nullptr);
      tokens_out[step] = tok;
    }
    if (step_ms_out) *step_ms_out = max_tokens > 1 ? total / double(max_tokens - 1) : 0.0;
  });
}

int ref_gpt2_decode(const InfercGpt2Weights* w, const int64_t* prompt,
                    int64_t n_prompt, int64_t max_tokens, int64_t* tokens_out,
                    float* margins_out, double* step_ms_out) {
  return ref_gpt2_decode_lm(w, w->wte, prompt, n_prompt, max_tokens, tokens_out, margins_out,
                            step_ms_out);
}

}  // extern "C"
