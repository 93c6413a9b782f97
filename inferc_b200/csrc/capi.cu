// extern "C" op entry points of libinferc_b200 (declared in
// include/inferc_dev.h). Each keeps the argument checks of the reference
// kernel it replaces and reports them as INFERC_ERR_INVALID instead of
// throwing across the ABI.
#include <cstring>
#include <string>

#include <mutex>
#include <unordered_map>

#include "kernels.cuh"

namespace inferc_dev {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

int read_and_clear_tc_error();
void launch_split_tf32(const float* x, float* big, float* small, int64_t n, cudaStream_t st);
bool gemm_use_tc(int64_t M, int64_t N, int64_t K);
bool gemm_tc_supported(const float* A, int64_t lda, const float* Bb, const float* Bs,
                       int64_t ldb, int64_t M, int64_t N, int64_t K);
void launch_gemm_tc(const float* A, int64_t lda, const float* Bb, const float* Bs, int64_t ldb,
                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                    cudaStream_t st);

// The tensor-core GEMM (gemm_tc.cu) when it accepts the shape, else the
// CUDA-core kernel. Defined in gemm_dispatch.cu.
void launch_gemm(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                 float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                 cudaStream_t st);
// The op-level form: split-fp16 on cached weight planes (gemm_dispatch.cu).
void launch_gemm_op(const float* A, int64_t lda, bool ta, const float* B, int64_t ldb, bool tb,
                    float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, const Epilogue& ep,
                    cudaStream_t st);

}  // namespace inferc_dev

using namespace inferc_dev;

namespace inferc_dev {
void weight_cache_evict_range(const void* base, size_t bytes);
}  // namespace inferc_dev

namespace {
// Sizes of the buffers inferc_dev_alloc handed out, so that inferc_dev_free
// can drop cached weight planes that lived in the freed range.
std::mutex g_alloc_mu;
std::unordered_map<void*, size_t> g_alloc_sizes;
}  // namespace

extern "C" {

const char* inferc_dev_last_error_string(void) { return g_last_error.c_str(); }

const char* inferc_dev_version(void) { return "inferc_b200 0.1 sm_100a"; }

int inferc_dev_alloc(void** ptr, size_t bytes) {
  return guard([&] {
    IDEV_CHECK_ARG(ptr != nullptr, "alloc: null out pointer");
    *ptr = nullptr;
    if (bytes == 0) return;
    const cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaErrorMemoryAllocation) {
      cudaGetLastError();
      throw Error(INFERC_ERR_OOM, "alloc: out of device memory (" + std::to_string(bytes) + " B)");
    }
    IDEV_CUDA(e);
    std::lock_guard<std::mutex> lock(g_alloc_mu);
    g_alloc_sizes[*ptr] = bytes;
  });
}

int inferc_dev_free(void* ptr) {
  return guard([&] {
    if (!ptr) return;
    size_t bytes = 0;
    {
      std::lock_guard<std::mutex> lock(g_alloc_mu);
      auto it = g_alloc_sizes.find(ptr);
      if (it != g_alloc_sizes.end()) {
        bytes = it->second;
        g_alloc_sizes.erase(it);
      }
    }
    // prepared planes of op-level GEMM weights that lived in this buffer
    if (bytes) weight_cache_evict_range(ptr, bytes);
    IDEV_CUDA(cudaFree(ptr));
  });
}

int inferc_dev_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  return guard([&] {
    IDEV_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
  });
}

int inferc_dev_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  return guard([&] {
    IDEV_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
  });
}

int inferc_dev_stream_synchronize(void* stream) {
  return guard([&] {
    IDEV_CUDA(cudaStreamSynchronize(as_stream(stream)));
    if (read_and_clear_tc_error())
      throw Error(INFERC_ERR_TIMEOUT, "a tensor-core GEMM wait timed out (results invalid)");
    if (read_and_clear_f16_range())
      throw Error(INFERC_ERR_RANGE,
                  "split-fp16 GEMM: an activation does not fit fp16 (results invalid)");
  });
}

int inferc_dev_layernorm(const float* x, const float* gamma, const float* beta, float* y,
                         int64_t rows, int64_t feat, float eps, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(rows >= 0 && feat > 0, "LayerNorm: bad shape");
    IDEV_CHECK_ARG(rows == 0 || (x && gamma && beta && y), "LayerNorm: null pointer");
    launch_layernorm(x, gamma, beta, y, rows, feat, eps, as_stream(stream));
  });
}

int inferc_dev_fused_matmul_add_gelu(const float* x, const float* w, const float* b, float* y,
                                     int64_t M, int64_t K, int64_t N, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && K > 0 && N > 0, "FusedMatMulAddGELU: bad shape");
    IDEV_CHECK_ARG(M == 0 || (x && w && b && y), "FusedMatMulAddGELU: null pointer");
    Epilogue ep;
    ep.bias = b;
    ep.bias_mode = 1;
    ep.act = ACT_GELU_ERF;
    launch_gemm_op(x, K, false, w, N, false, y, N, M, N, K, ep, as_stream(stream));
  });
}

int inferc_dev_fused_qkv(const float* x, const float* wq, const float* bq, const float* wk,
                         const float* bk, const float* wv, const float* bv, float* q, float* k,
                         float* v, int64_t M, int64_t K, int64_t N, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && K > 0 && N > 0, "FusedQKV: bad shape");
    const float* ws[3] = {wq, wk, wv};
    const float* bs[3] = {bq, bk, bv};
    float* os[3] = {q, k, v};
    for (int i = 0; i < 3; ++i) {
      IDEV_CHECK_ARG(M == 0 || (x && ws[i] && bs[i] && os[i]), "FusedQKV: null pointer");
      Epilogue ep;
      ep.bias = bs[i];
      ep.bias_mode = 1;
      launch_gemm_op(x, K, false, ws[i], N, false, os[i], N, M, N, K, ep, as_stream(stream));
    }
  });
}

int inferc_dev_fused_attention(const float* q, const float* k, const float* v,
                               const uint8_t* mask, const int64_t* mask_shape, int mask_rank,
                               int64_t B, int64_t S, int64_t H, int64_t head_dim, float fill,
                               float* out, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(B >= 0 && S >= 0 && H > 0, "FusedAttention: expect [B,S,H]");
    IDEV_CHECK_ARG(head_dim > 0 && H % head_dim == 0,
                   "FusedAttention: H not divisible by head_dim");
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.out = out;
    a.ldq = a.ldk = a.ldv = a.ldo = H;
    a.bstride_q = a.bstride_k = a.bstride_v = a.bstride_o = S * H;
    a.B = B; a.S = S; a.nH = H / head_dim; a.hd = head_dim;
    a.scale = 1.0f / std::sqrt((float)head_dim);
    a.fill = fill;
    a.causal = 0;
    if (mask != nullptr && mask_rank > 0) {
      IDEV_CHECK_ARG(mask_shape != nullptr && mask_rank <= 4,
                     "FusedAttention: mask rank must be 1..4 with a shape");
      // Right-aligned broadcast strides over [B, nH, S, S] (MaskStrides,
      // src/kernels/attention.cc:17-29); each mask axis must be 1 or match.
      const int64_t full[4] = {B, a.nH, S, S};
      int64_t st = 1;
      for (int i = mask_rank - 1; i >= 0; --i) {
        const int od = 4 - (mask_rank - i);
        IDEV_CHECK_ARG(mask_shape[i] == 1 || mask_shape[i] == full[od],
                       "FusedAttention: mask shape does not broadcast to [B,nH,S,S]");
        a.ms[od] = mask_shape[i] == 1 ? 0 : st;
        st *= mask_shape[i];
      }
      a.mask = mask;
    }
    launch_attention(a, as_stream(stream));
  });
}

int inferc_dev_gemm(const float* a, const float* b, const float* c, int64_t c_len, float* y,
                    int64_t M, int64_t K, int64_t N, float alpha, float beta, int trans_a,
                    int trans_b, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && K > 0 && N >= 0, "Gemm: bad shape");
    const bool use_c = c != nullptr && beta != 0.0f;
    if (use_c)
      IDEV_CHECK_ARG(c_len == M * N || c_len == N || c_len == 1,
                     "Gemm: unsupported C shape for broadcast");
    cudaStream_t st = as_stream(stream);
    if (M == 1 && !trans_b && (!use_c || c_len == N)) {
      GemvArgs g{};
      g.x = a; g.w = b; g.y = y; g.K = K; g.N = N;
      g.alpha = alpha; g.beta = beta;
      g.bias = use_c ? c : nullptr;
      g.act = ACT_NONE;
      launch_gemv(g, st);
      return;
    }
    Epilogue ep;
    ep.alpha = alpha;
    ep.beta = beta;
    if (use_c) {
      ep.bias = c;
      ep.bias_mode = c_len == M * N ? 3 : c_len == N ? 1 : 2;
      ep.ldbias = N;
    }
    launch_gemm_op(a, trans_a ? M : K, trans_a != 0, b, trans_b ? K : N, trans_b != 0, y, N, M, N,
                K, ep, st);
  });
}

int inferc_dev_matmul(const float* a, const float* b, float* y, int64_t M, int64_t K, int64_t N,
                      void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && K > 0 && N >= 0, "MatMul: bad shape");
    Epilogue ep;
    launch_gemm_op(a, K, false, b, N, false, y, N, M, N, K, ep, as_stream(stream));
  });
}

int inferc_dev_gelu(const float* x, float* y, int64_t n, void* stream) {
  return guard([&] { launch_act(x, y, n, ACT_GELU_ERF, as_stream(stream)); });
}

int inferc_dev_gelu_tanh(const float* x, float* y, int64_t n, void* stream) {
  return guard([&] { launch_act(x, y, n, ACT_GELU_TANH, as_stream(stream)); });
}

int inferc_dev_softmax(const float* x, float* y, int64_t rows, int64_t cols, void* stream) {
  return guard([&] { launch_softmax(x, y, rows, cols, as_stream(stream)); });
}

int inferc_dev_tf32_split(const float* w, float* big, float* small, int64_t n, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(n >= 0 && (n == 0 || (w && big && small)), "tf32_split: bad arguments");
    launch_split_tf32(w, big, small, n, as_stream(stream));
  });
}

int inferc_dev_gemm_tf32x3(const float* a, int64_t lda, const float* b_big, const float* b_small,
                           int64_t ldb, const float* bias, const float* resid, int64_t ldr,
                           float* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                           void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && N >= 0 && K > 0 && lda >= K && ldb >= N && ldy >= N,
                   "gemm_tf32x3: bad shape / leading dimensions");
    IDEV_CHECK_ARG(act >= 0 && act <= 3, "gemm_tf32x3: unknown activation");
    if (M == 0 || N == 0) return;
    Epilogue ep;
    ep.bias = bias;
    ep.bias_mode = bias ? 1 : 0;
    ep.resid = resid;
    ep.ldr = ldr;
    ep.act = act;
    cudaStream_t st = as_stream(stream);
    if (gemm_use_tc(M, N, K) && gemm_tc_supported(a, lda, b_big, b_small, ldb, M, N, K)) {
      launch_gemm_tc(a, lda, b_big, b_small, ldb, y, ldy, M, N, K, ep, st);
      return;
    }
    // CUDA-core path (small M / unaligned): big + small is the original
    // weight exactly, so y = act(A big + resid) then y = act(A small + y + bias).
    Epilogue first;  // y = A big + resid (resid may alias y: same element, same thread)
    first.resid = resid;
    first.ldr = ldr;
    launch_gemm_simt(a, lda, false, b_big, ldb, false, y, ldy, M, N, K, first, st);
    Epilogue second = ep;
    second.resid = y;
    second.ldr = ldy;
    launch_gemm_simt(a, lda, false, b_small, ldb, false, y, ldy, M, N, K, second, st);
  });
}

int64_t inferc_dev_f16_kp(int64_t K) { return f16_weight_kp(K); }

int inferc_dev_f16_split(const float* w, int64_t K, int64_t N, int64_t ldw, uint16_t* hi,
                         uint16_t* lo, float* scale2, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(K > 0 && N > 0 && ldw >= N && w && hi && lo && scale2,
                   "f16_split: bad arguments");
    prepare_weight_f16(w, K, N, ldw, hi, lo, scale2, as_stream(stream));
  });
}

int inferc_dev_gemm_f16s(const float* a, int64_t lda, const uint16_t* hi, const uint16_t* lo,
                         const float* scale2, const float* bias, const float* resid, int64_t ldr,
                         float* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int act,
                         void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && N >= 0 && K > 0 && lda >= K && ldy >= N,
                   "gemm_f16s: bad shape / leading dimensions");
    IDEV_CHECK_ARG(act >= 0 && act <= 3, "gemm_f16s: unknown activation");
    IDEV_CHECK_ARG(hi && lo && scale2, "gemm_f16s: null weight");
    if (M == 0 || N == 0) return;
    Epilogue ep;
    ep.bias = bias;
    ep.bias_mode = bias ? 1 : 0;
    ep.resid = resid;
    ep.ldr = ldr;
    ep.act = act;
    launch_gemm_f16s(a, lda, hi, lo, f16_weight_kp(K), scale2, nullptr, y, ldy, M, N, K, ep,
                     as_stream(stream));
  });
}

int inferc_dev_f16_split_rows(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                              uint16_t* hi, uint16_t* lo, int64_t ld, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(rows == 0 || (x && hi && lo), "f16_split_rows: null pointer");
    launch_split_rows_f16(x, rows, cols, ldx, hi, lo, ld, nullptr, as_stream(stream));
  });
}

int inferc_dev_gemm_f16s_planes(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda,
                                const uint16_t* hi, const uint16_t* lo, const float* scale2,
                                const float* bias, const float* resid, int64_t ldr, float* y,
                                uint16_t* y_hi, uint16_t* y_lo, int64_t ldy, int64_t M,
                                int64_t N, int64_t K, int act, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(M >= 0 && N >= 0 && K > 0 && lda >= K && ldy >= N,
                   "gemm_f16s_planes: bad shape / leading dimensions");
    IDEV_CHECK_ARG(act >= 0 && act <= 3, "gemm_f16s_planes: unknown activation");
    IDEV_CHECK_ARG(hi && lo && scale2 && a_hi && a_lo, "gemm_f16s_planes: null operand");
    IDEV_CHECK_ARG((y_hi == nullptr) == (y_lo == nullptr) && (y_hi || y),
                   "gemm_f16s_planes: give y, or both y_hi and y_lo");
    if (M == 0 || N == 0) return;
    Epilogue ep;
    ep.bias = bias;
    ep.bias_mode = bias ? 1 : 0;
    ep.resid = resid;
    ep.ldr = ldr;
    ep.act = act;
    F16GemmA a;
    a.hi = a_hi;
    a.lo = a_lo;
    a.ld = lda;
    SplitOut so;
    if (y_hi) {
      so.hi = y_hi;
      so.lo = y_lo;
      so.ld = ldy;
      so.range = f16_range_flag_ptr();
    }
    launch_gemm_f16s(a, hi, lo, f16_weight_kp(K), scale2, nullptr, y, ldy, so, M, N, K, ep,
                     as_stream(stream));
  });
}

int inferc_dev_fused_attention_planes(const uint16_t* q_hi, const uint16_t* q_lo,
                                      const uint16_t* k_hi, const uint16_t* k_lo,
                                      const uint16_t* v_hi, const uint16_t* v_lo, int64_t ld,
                                      const uint8_t* key_mask, int64_t B, int64_t S,
                                      int64_t heads, float fill, float* out, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(B >= 0 && S >= 0 && heads > 0, "fused_attention_planes: bad shape");
    if (B == 0 || S == 0) return;
    AttnF16Args a{};
    a.qh = q_hi; a.ql = q_lo; a.kh = k_hi; a.kl = k_lo; a.vh = v_hi; a.vl = v_lo;
    a.ld = ld;
    a.bstride = S * ld;
    a.mask = key_mask;
    a.ms[0] = S; a.ms[1] = 0; a.ms[2] = 0; a.ms[3] = 1;
    a.B = B; a.S = S; a.nH = heads;
    a.scale = 0.125f;  // 1 / sqrt(64)
    a.fill = fill;
    a.out = out;
    a.ldo = heads * 64;
    a.bstride_o = S * heads * 64;
    IDEV_CHECK_ARG(attention_f16_supported(a),
                   "fused_attention_planes: needs S <= 128, 16-byte aligned planes, ld % 8 == 0");
    launch_attention_f16(a, as_stream(stream));
  });
}

int inferc_dev_qkv_attention(const float* x, const float* w_big, const float* w_small,
                             const float* bqkv, const uint8_t* key_mask, int64_t B, int64_t S,
                             int64_t H, int64_t head_dim, float fill, float* scratch_qkv,
                             float* out, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(B >= 0 && S >= 0 && H > 0, "qkv_attention: bad shape");
    IDEV_CHECK_ARG(head_dim > 0 && H % head_dim == 0,
                   "qkv_attention: H not divisible by head_dim");
    if (B == 0 || S == 0) return;
    cudaStream_t st = as_stream(stream);
    const int64_t M = B * S;
    IDEV_CHECK_ARG(inferc_dev_gemm_tf32x3(x, H, w_big, w_small, 3 * H, bqkv, nullptr, 0,
                                          scratch_qkv, 3 * H, M, 3 * H, H, 0, stream) == 0,
                   std::string("qkv_attention: ") + g_last_error);
    AttnArgs a{};
    a.q = scratch_qkv; a.k = scratch_qkv + H; a.v = scratch_qkv + 2 * H; a.out = out;
    a.ldq = a.ldk = a.ldv = 3 * H;
    a.ldo = H;
    a.bstride_q = a.bstride_k = a.bstride_v = S * 3 * H;
    a.bstride_o = S * H;
    a.mask = key_mask;
    a.ms[0] = S; a.ms[1] = 0; a.ms[2] = 0; a.ms[3] = 1;
    a.B = B; a.S = S; a.nH = H / head_dim; a.hd = head_dim;
    a.scale = 1.0f / std::sqrt((float)head_dim);
    a.fill = fill;
    launch_attention(a, st);
  });
}

int inferc_dev_qkv_attention_f16(const float* x, const uint16_t* w_hi, const uint16_t* w_lo,
                                 const float* w_scale2, const float* bqkv,
                                 const uint8_t* key_mask, int64_t B, int64_t S, int64_t H,
                                 int64_t head_dim, float fill, uint16_t* scratch, float* out,
                                 void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(B >= 0 && S >= 0 && H > 0 && head_dim == 64 && H % 64 == 0,
                   "qkv_attention_f16: head_dim must be 64 and divide H");
    IDEV_CHECK_ARG(x && w_hi && w_lo && w_scale2 && bqkv && scratch && out,
                   "qkv_attention_f16: null pointer");
    if (B == 0 || S == 0) return;
    cudaStream_t st = as_stream(stream);
    const int64_t M = B * S;
    uint16_t* xh = scratch;
    uint16_t* xl = xh + M * H;
    uint16_t* qh = xl + M * H;
    uint16_t* ql = qh + M * 3 * H;
    int* range = f16_range_flag_ptr();
    launch_split_rows_f16(x, M, H, H, xh, xl, H, range, st);
    F16GemmA a;
    a.hi = xh;
    a.lo = xl;
    a.ld = H;
    SplitOut so;
    so.hi = qh;
    so.lo = ql;
    so.ld = 3 * H;
    so.range = range;
    Epilogue ep;
    ep.bias = bqkv;
    ep.bias_mode = 1;
    launch_gemm_f16s(a, w_hi, w_lo, f16_weight_kp(H), w_scale2, range, nullptr, 3 * H, so, M,
                     3 * H, H, ep, st);
    AttnF16Args at{};
    at.qh = qh; at.ql = ql; at.kh = qh + H; at.kl = ql + H; at.vh = qh + 2 * H; at.vl = ql + 2 * H;
    at.ld = 3 * H;
    at.bstride = S * 3 * H;
    at.mask = key_mask;
    at.ms[0] = S; at.ms[1] = 0; at.ms[2] = 0; at.ms[3] = 1;
    at.B = B; at.S = S; at.nH = H / 64;
    at.scale = 0.125f;
    at.fill = fill;
    at.out = out;
    at.ldo = H;
    at.bstride_o = S * H;
    IDEV_CHECK_ARG(attention_f16_supported(at),
                   "qkv_attention_f16: needs S <= 4096 and 16-byte aligned buffers");
    launch_attention_f16(at, st);
  });
}

int inferc_dev_gemv(const float* x, const float* w, const float* b, const float* resid, float* y,
                    int64_t K, int64_t N, int act, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(K > 0 && N >= 0, "GEMV: bad shape");
    IDEV_CHECK_ARG(act >= 0 && act <= 3, "GEMV: unknown activation");
    GemvArgs g{};
    g.x = x; g.w = w; g.bias = b; g.resid = resid; g.y = y; g.K = K; g.N = N;
    g.alpha = 1.0f; g.beta = 1.0f; g.act = act;
    launch_gemv(g, as_stream(stream));
  });
}

int inferc_dev_gemv_int4_rowscale(const uint8_t* w, const float* scales, const float* x, float* y,
                                  int64_t N, int64_t K, void* stream) {
  return guard([&] {
    InfercInt4Gemv d{w, scales, x, y, N, K};
    launch_gemv_int4(&d, 1, as_stream(stream));
  });
}

int inferc_dev_gemv_int4_batched(const InfercInt4Gemv* descs, int count, void* stream) {
  return guard([&] { launch_gemv_int4(descs, count, as_stream(stream)); });
}

int inferc_dev_argmax(const float* x, int64_t n, int64_t* out_index, void* stream) {
  return guard([&] { launch_argmax(x, n, out_index, as_stream(stream)); });
}

int inferc_dev_kv_append(const float* k_new, const float* v_new, int64_t ld_new, float* k_cache,
                         float* v_cache, int64_t heads, int64_t head_dim, int64_t max_len,
                         int64_t pos, int64_t n, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(pos >= 0 && n >= 0 && pos + n <= max_len,
                   "kv_append: positions beyond the cache");
    launch_kv_append(k_new, v_new, ld_new, k_cache, v_cache, heads, head_dim, max_len, nullptr,
                     pos, n, as_stream(stream));
  });
}

int inferc_dev_decode_attention(const float* q, const float* k_cache, const float* v_cache,
                                float* out, int64_t heads, int64_t head_dim, int64_t max_len,
                                int64_t L, void* stream) {
  return guard([&] {
    IDEV_CHECK_ARG(L >= 1 && L <= max_len, "decode_attention: L must be in [1, max_len]");
    launch_decode_attention(q, nullptr, nullptr, const_cast<float*>(k_cache),
                            const_cast<float*>(v_cache), out, heads, head_dim, max_len, nullptr,
                            L, as_stream(stream));
  });
}

}  // extern "C"
