// Persistent decode kernel: every single-token step of GPT-2 greedy decode
// (the with-past graph of `inferc decode`, src/cli/main.cpp:854-889) for any
// number of steps in ONE cooperative launch.
//
// One CTA per SM. A step is a sequence of phases separated by grid barriers:
//   per layer:  QKV   y = LN1(x) W_attn + b            (144 column panels)
//               ATTN  per head: KV append at pos, softmax(q.K/8) V   (12 CTAs)
//               PROJ  x += ctx W_proj + b              (192 panels)
//               FC    f = tanhGELU(LN2(x) W_fc + b)    (192 panels)
//               FP    x += f W_fcproj + b              (192 panels)
//   then        LM    logits = LNf(x) wte^T, per-CTA best (first max wins)
// and the next step's embedding is computed by every CTA from the argmax of
// the 148 per-CTA bests, so no extra phase is needed.
//
// Weights are pre-tiled at plan creation into column panels [K][P]
// (contiguous), so a CTA fetches a panel with one bulk copy into shared
// memory. Four 48 KiB slots form two pairs; while a phase computes from one
// pair, the next weight phase is already streaming into the other, so HBM
// keeps streaming across barriers. Each output column is produced by exactly
// one CTA with a fixed summation order (deterministic).
//
// Inside a step the phases are not separated by grid barriers. Activations
// (x, qkv, the projection partials, f) travel as tagged 64-bit words,
// (tag << 32) | fp32 bits, each word written once per phase instance with a
// tag unique to that instance; a reader loads the words it needs and re-reads
// any whose tag is not yet the expected one. The load is the wait, so a phase
// starts as soon as its own inputs have landed, with no release fence and no
// extra L2 round trip for a barrier. Only the end of a step keeps a grid
// barrier: the argmax needs every CTA's best, and it orders the step's
// KV-cache appends before the next step's reads.
//
// Overwrites are safe without double buffers because every CTA takes part
// in the FC and FP phases: a buffer is rewritten only by a phase whose inputs
// depend (through tagged words) on every CTA having finished the phase that
// read it. The layer input alternates between two buffers for the same
// reason. A reader that sees a newer tag than it expects reports an error.
// All data produced inside the kernel is read from L2, never through L1.
// Every wait (tags, mbarriers, the grid barrier) is bounded: on a timeout the
// kernel sets an error flag, every CTA leaves at its next check, and the host
// reports the failure.
#include <cuda.h>

#include <cfloat>
#include <vector>

#include "decode_mega.cuh"
#include "kernels.cuh"

namespace inferc_dev {

namespace {

constexpr int kMegaThreads = 256;
// The thread that issues the bulk copies: lane 0 of the last warp, not thread
// 0, which leads every CTA reduction. An issue can stall for a microsecond or
// more while the whole grid requests its next panels at once; in this warp
// the stall overlaps the next phase's wait for its inputs.
constexpr int kIssuer = kMegaThreads - 32;
// LM head: warps 0..kLmWarps-1 compute rows; the issuer's warp only refills.
constexpr int kLmWarps = kMegaThreads / 32 - 1;
constexpr int kSlotBytes = 48 * 1024;
constexpr int kSlots = 4;
constexpr unsigned long long kMegaWaitNs = 50ull * 1000 * 1000;  // 50 ms per wait

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mb_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mb_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mb_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ unsigned long long gclock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait (at most kMegaWaitNs) for the phase with the given parity.
__device__ __forceinline__ bool mb_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
  const unsigned long long t0 = gclock();
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 255 && gclock() - t0 > kMegaWaitNs) return false;
  }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes and
// addresses multiples of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk copy of streamed weights: read once per token, so marked first to be
// evicted from L2, which keeps the KV cache and the activations resident.
__device__ __forceinline__ void bulk_load_stream(void* dst, const void* src, uint32_t bytes,
                                                 uint64_t* bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}


constexpr int kLnMax = 800;  // LayerNorm width whose gamma / beta (+ a bias) are prefetched

struct Smem {
  uint64_t bar[kSlots];
  uint64_t empty[kSlots];   // LM head: slot consumed by the kLmWarps row warps
  uint32_t empty_uses[kSlots];  // completed waits on empty[] (issuer only)
  uint32_t uses[kSlots];    // completed waits per slot (parity tracking)
  uint32_t issued[kSlots];  // issued fills per slot (thread 0 only)
  uint64_t ln_bar;          // gamma / beta of the next LayerNorm phase
  uint32_t ln_uses, ln_issued;
  unsigned target;          // arrival count that ends the current grid barrier
  __align__(16) float lnp[3 * kLnMax];  // [gamma | beta | extra vector]
  float xs[3072];         // staged GEMV input (normalised when LN applies)
  float red[2 * kMegaThreads];
  float stat[2];
  float bv[kMegaThreads / 32];
  int64_t bi[kMegaThreads / 32];
  int abort_flag;
  unsigned nbar;  // barriers passed (thread 0)
};

// ---- tagged activation words
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p));
  return w;
}

__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ float word_f(uint64_t w) { return __uint_as_float((uint32_t)w); }

// Waits until every word of w[0:N) (first loads already issued by the
// caller; a slot that needs no word is preset to tag << 32) carries `tag`:
// each round re-reads all stale words at once, so a batch that was loaded
// too early costs one L2 round trip per round, not one per word. Bounded: a
// newer tag (an ordering fault), a timeout or an error raised elsewhere sets
// the error flags, zeroes the values and returns false.
template <int N, typename Addr>
__device__ __forceinline__ bool settle(uint64_t (&w)[N], uint32_t tag, Addr addr,
                                       const MegaArgs& a, Smem& sm) {
  unsigned long long t0 = 0;
  for (uint32_t round = 0;; ++round) {
    bool ready = true, newer = false;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const uint32_t wt = (uint32_t)(w[i] >> 32);
      ready = ready && wt == tag;
      newer = newer || (int)(wt - tag) > 0;
    }
    if (ready) return true;
    bool fail = newer;
    if (round == 0) t0 = gclock();
    else if ((round & 15) == 0) fail = fail || gclock() - t0 > kMegaWaitNs || *(volatile int*)a.err;
    if (fail) {
      atomicExch(a.err, 1);
      sm.abort_flag = 1;
#pragma unroll
      for (int i = 0; i < N; ++i) w[i] = (uint64_t)tag << 32;
      return false;
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
      if ((uint32_t)(w[i] >> 32) != tag) w[i] = ld_word(addr(i));
  }
}

#ifdef INFERC_DECODE_PROFILE
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#endif

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier over a monotonic arrival counter (zeroed by the host
// before each launch): barrier number b completes when the counter reaches
// (b + 1) * gridDim.x. Arrival is a fire-and-forget release add, so CTAs do
// not serialise on returning atomics. Returns false when the kernel must
// stop (timeout here or an error flagged elsewhere).
// Split in two so that thread 0 can issue the next copies between its
// arrival and its wait.
__device__ void grid_arrive(const MegaArgs& a, Smem& sm) {
  __syncthreads();  // the CTA's outputs of the phase precede the release below
  if (threadIdx.x == 0) {
    sm.target = (++sm.nbar) * gridDim.x;
    red_release_add(a.bar_count, 1u);
  }
}

__device__ bool grid_wait(const MegaArgs& a, Smem& sm) {
  if (threadIdx.x == 0) {
    const unsigned target = sm.target;
    uint32_t i = 0;
    const unsigned long long t0 = gclock();
    while ((int)(ld_acquire(a.bar_count) - target) < 0) {
      if ((++i & 63) == 0 && (gclock() - t0 > kMegaWaitNs || *(volatile int*)a.err)) {
        atomicExch(a.err, 1);
        break;
      }
    }
    sm.abort_flag = *(volatile int*)a.err;
  }
  __syncthreads();
  return sm.abort_flag == 0;
}

// Development builds (-DINFERC_DECODE_PROFILE): every CTA stamps event e
// of layer 5 of step 1 into prof[64 + 32 * cta + e].
__device__ __forceinline__ void stamp_event(const MegaArgs& a, bool on, int e, int by = 0) {
#ifdef INFERC_DECODE_PROFILE
  if (a.prof && on && threadIdx.x == by) a.prof[64 + 32 * blockIdx.x + e] = gtimer();
#else
  (void)a; (void)on; (void)e; (void)by;
#endif
}

// End of a phase of this CTA: all threads are past their reads of the slots
// and their writes; false when a wait of the phase failed. With
// -DINFERC_DECODE_PROFILE, CTA 0 stamps the global timer at phase q of step 1.
__device__ __forceinline__ bool phase_end(const MegaArgs& a, Smem& sm, int q, int step) {
  __syncthreads();
#ifdef INFERC_DECODE_PROFILE
  if (a.prof && step == 1 && blockIdx.x == 0 && threadIdx.x == 0) a.prof[q + 1] = gtimer();
#else
  (void)a; (void)q; (void)step;
#endif
  return sm.abort_flag == 0;
}

// Thread 0: bulk copy of a LayerNorm's gamma and beta (K floats each), and
// optionally one more K-vector of the phase, into sm.lnp, completing on
// sm.ln_bar; a no-op when K exceeds kLnMax (the phase then reads them from
// global memory).
// Whether a LayerNorm's vectors go through sm.lnp: bulk copies need 16-byte
// aligned sources and sizes.
__device__ __forceinline__ bool ln_prefetchable(const float* g, const float* b,
                                                const float* extra, int K) {
  auto al = [](const float* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return K <= kLnMax && K % 4 == 0 && al(g) && al(b) && (extra == nullptr || al(extra));
}

__device__ void prefetch_ln(const float* g, const float* b, const float* extra, int K,
                            Smem& sm) {
  if (threadIdx.x != kIssuer || !ln_prefetchable(g, b, extra, K)) return;
  const uint32_t bytes = (uint32_t)K * 4;
  sm.ln_issued++;
  mb_expect_tx(&sm.ln_bar, (extra ? 3 : 2) * bytes);
  bulk_load(sm.lnp, g, bytes, &sm.ln_bar);
  bulk_load(sm.lnp + kLnMax, b, bytes, &sm.ln_bar);
  if (extra) bulk_load(sm.lnp + 2 * kLnMax, extra, bytes, &sm.ln_bar);
}

// Gamma / beta (and the extra vector) of a phase with a LayerNorm of width
// K: the prefetched copy (all threads wait for it, bounded) or, past
// kLnMax, the global arrays.
__device__ bool ln_params(const float* g, const float* b, const float* extra, int K, Smem& sm,
                          const MegaArgs& a, const float** gs, const float** bs,
                          const float** es) {
  if (!ln_prefetchable(g, b, extra, K)) {
    *gs = g;
    *bs = b;
    *es = extra;
    return true;
  }
  const bool ok = __syncthreads_and(mb_wait(&sm.ln_bar, sm.ln_uses & 1)) != 0;
  if (threadIdx.x == 0) {
    sm.ln_uses++;
    if (!ok) atomicExch(a.err, 1);
  }
  __syncthreads();
  *gs = sm.lnp;
  *bs = sm.lnp + kLnMax;
  *es = sm.lnp + 2 * kLnMax;
  return ok;
}

// Issue this CTA's panels of a GEMV phase into slot pair `pair`.
__device__ void prefetch_panels(const MegaPanels& m, int pair, uint8_t* slots, Smem& sm,
                                uint32_t piece) {
  if (threadIdx.x != kIssuer) return;
  for (int j = 0; j < 2; ++j) {
    const int p = blockIdx.x + j * gridDim.x;
    if (p >= m.npanels) break;
    const int s = 2 * pair + j;
    const uint32_t bytes = m.bytes;
    sm.issued[s]++;
    mb_expect_tx(&sm.bar[s], bytes);
    const uint8_t* src = m.data + (size_t)p * m.bytes;
    for (uint32_t off = 0; off < bytes; off += piece)
      bulk_load_stream(slots + (size_t)s * kSlotBytes + off, src + off, min(piece, bytes - off),
                       &sm.bar[s]);
  }
}

// Waits for slot s; all threads; false on timeout.
__device__ bool wait_slot(int s, Smem& sm, const MegaArgs& a) {
  const bool ok = __syncthreads_and(mb_wait(&sm.bar[s], sm.uses[s] & 1)) != 0;
  if (threadIdx.x == 0) {
    sm.uses[s]++;
    if (!ok) atomicExch(a.err, 1);
  }
  __syncthreads();
  return ok;
}

// Before leaving early: wait (bounded) for this CTA's bulk copies still in
// flight, so none lands in shared memory after the CTA has exited.
__device__ void drain(Smem& sm) {
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s)
      while (sm.issued[s] > sm.uses[s]) {
        mb_wait(&sm.bar[s], sm.uses[s] & 1);
        sm.uses[s]++;
      }
    while (sm.ln_issued > sm.ln_uses) {
      mb_wait(&sm.ln_bar, sm.ln_uses & 1);
      sm.ln_uses++;
    }
  }
  __syncthreads();
}

// Stages x (tagged words written in this kernel with `tag`) into sm.xs,
// normalised with (g, b) when g != null (two-pass mean / biased variance, as
// rt::LayerNorm).
__device__ void stage_input(const uint64_t* x, uint32_t tag, int K, const float* g,
                            const float* b, float eps, Smem& sm, const MegaArgs& a) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  // K <= 3072: at most 12 elements per thread; x, gamma and beta loads are
  // all issued before any is used.
  uint64_t xw[12];
  float v[12], gv[12], bv[12];
#pragma unroll
  for (int i = 0; i < 12; ++i) {
    const int k = tid + i * kMegaThreads;
    xw[i] = k < K ? ld_word(x + k) : (uint64_t)tag << 32;
    if (g != nullptr) {  // shared (prefetched) or global
      gv[i] = k < K ? g[k] : 0.f;
      bv[i] = k < K ? b[k] : 0.f;
    }
  }
  settle(xw, tag, [&](int i) { return x + tid + i * kMegaThreads; }, a, sm);
#pragma unroll
  for (int i = 0; i < 12; ++i) v[i] = word_f(xw[i]);
  if (g == nullptr) {
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const int k = tid + i * kMegaThreads;
      if (k < K) sm.xs[k] = v[i];
    }
    __syncthreads();
    return;
  }
  constexpr int nw = kMegaThreads / 32;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 12; ++i) s += v[i];
  s = warp_sum(s);
  if (lane == 0) sm.red[wid] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < nw; ++w) tot += sm.red[w];
  const float mean = tot / (float)K;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 12; ++i) {
    const int k = tid + i * kMegaThreads;
    const float d = k < K ? v[i] - mean : 0.f;
    q += d * d;
  }
  q = warp_sum(q);
  if (lane == 0) sm.red[nw + wid] = q;
  __syncthreads();
  float tq = 0.f;
#pragma unroll
  for (int w = 0; w < nw; ++w) tq += sm.red[nw + w];
  const float inv = 1.0f / sqrtf(tq / (float)K + eps);
#pragma unroll
  for (int i = 0; i < 12; ++i) {
    const int k = tid + i * kMegaThreads;
    if (k < K) sm.xs[k] = ((v[i] - mean) * inv) * gv[i] + bv[i];
  }
  __syncthreads();
}

// LayerNorm of sm.xs[0:K) in place (the values are already staged).
__device__ void stage_smem_ln(int K, const float* g, const float* b, float eps, Smem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int nw = kMegaThreads / 32;
  float s = 0.f;
  for (int k = tid; k < K; k += kMegaThreads) s += sm.xs[k];
  s = warp_sum(s);
  if (lane == 0) sm.red[wid] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < nw; ++w) tot += sm.red[w];
  const float mean = tot / (float)K;
  float q = 0.f;
  for (int k = tid; k < K; k += kMegaThreads) {
    const float d = sm.xs[k] - mean;
    q += d * d;
  }
  q = warp_sum(q);
  if (lane == 0) sm.red[nw + wid] = q;
  __syncthreads();
  float tq = 0.f;
#pragma unroll
  for (int w = 0; w < nw; ++w) tq += sm.red[nw + w];
  const float inv = 1.0f / sqrtf(tq / (float)K + eps);
  __syncthreads();
  for (int k = tid; k < K; k += kMegaThreads) sm.xs[k] = ((sm.xs[k] - mean) * inv) * g[k] + b[k];
  __syncthreads();
}

// Epilogue inputs of this thread's output columns (threads tid < P own
// column p*P + tid of each of the CTA's two panels), loaded before the input
// staging so their latency overlaps it.
struct EpiIn {
  float add[2];
  float sc[2];  // int4: the columns' scales
};

__device__ __forceinline__ EpiIn gemv_preload(const MegaPanels& m, const float* bias,
                                              const uint64_t* resid, uint32_t rtag,
                                              const MegaArgs& a, Smem& sm) {
  EpiIn e{{0.f, 0.f}, {1.f, 1.f}};
  const int tid = threadIdx.x;
  if (tid < m.P) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int p = blockIdx.x + j * gridDim.x;
      const int col = p * m.P + tid;
      if (p < m.npanels && col < m.N) {
        if (m.scale) e.sc[j] = __ldg(m.scale + col);
        float v = __ldg(bias + col);
        if (resid) {
          uint64_t rw[1] = {ld_word(resid + col)};
          settle(rw, rtag, [&](int) { return resid + col; }, a, sm);
          v += word_f(rw[0]);
        }
        e.add[j] = v;
      }
    }
  }
  return e;
}

// y[col] = act(xs . panel[:, c] + bias[col] (+ resid[col])) for this CTA's
// panels (slots 2*pair, 2*pair+1), both panels in one pass; y is written as
// tagged words with `ytag`.
template <bool Q4>
__device__ bool gemv_phase(const MegaPanels& m, int pair, const uint8_t* slots, const EpiIn& e,
                           uint64_t* y, uint32_t ytag, int act, Smem& sm, const MegaArgs& a) {
  const int tid = threadIdx.x;
  const int P = m.P, K = m.K;
  const int P4 = P / 4;                  // float4 columns per row
  const int slices = kMegaThreads / P4;  // rows processed in parallel
  const int c4 = tid % P4, sl = tid / P4;
  const int np = (int)(blockIdx.x < (unsigned)m.npanels) + (int)(blockIdx.x + gridDim.x < (unsigned)m.npanels);
  {  // both panels' copies, one CTA barrier
    bool ok = true;
    for (int j = 0; j < np; ++j) ok = mb_wait(&sm.bar[2 * pair + j], sm.uses[2 * pair + j] & 1) && ok;
    ok = __syncthreads_and(ok) != 0;
    if (threadIdx.x == 0) {
      for (int j = 0; j < np; ++j) sm.uses[2 * pair + j]++;
      if (!ok) atomicExch(a.err, 1);
    }
    __syncthreads();
    if (!ok) return false;
  }
  const float* w0 = reinterpret_cast<const float*>(slots + (size_t)(2 * pair) * kSlotBytes);
  const float* w1 = reinterpret_cast<const float*>(slots + (size_t)(2 * pair + 1) * kSlotBytes);
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
  const float4* w04 = reinterpret_cast<const float4*>(w0);
  const float4* w14 = reinterpret_cast<const float4*>(w1);
  if constexpr (Q4) {
    // words (kg, c): 8 consecutive k of column c; a thread takes a column
    // quad (one 16-byte load per panel) over k groups kg = sl, sl + slices, ...
    const uint4* v0 = reinterpret_cast<const uint4*>(w0);
    const uint4* v1 = reinterpret_cast<const uint4*>(w1);
    const float4* x4 = reinterpret_cast<const float4*>(sm.xs);
    auto dot8 = [](uint32_t q, const float (&xv)[8], float acc) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = fmaf((float)((int)((q >> (4 * i)) & 15u) - 8), xv[i], acc);
      return acc;
    };
    for (int kg = sl; kg < K / 8; kg += slices) {
      const float4 xa = x4[2 * kg], xb = x4[2 * kg + 1];
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      const uint4 u = v0[kg * P4 + c4];
      a0.x = dot8(u.x, xv, a0.x); a0.y = dot8(u.y, xv, a0.y);
      a0.z = dot8(u.z, xv, a0.z); a0.w = dot8(u.w, xv, a0.w);
      if (np == 2) {
        const uint4 t = v1[kg * P4 + c4];
        a1.x = dot8(t.x, xv, a1.x); a1.y = dot8(t.y, xv, a1.y);
        a1.z = dot8(t.z, xv, a1.z); a1.w = dot8(t.w, xv, a1.w);
      }
    }
  } else if (np == 2) {
#pragma unroll 4
    for (int k = sl; k < K; k += slices) {
      const float xv = sm.xs[k];
      const float4 u = w04[k * P4 + c4], t = w14[k * P4 + c4];
      a0.x = fmaf(xv, u.x, a0.x); a0.y = fmaf(xv, u.y, a0.y);
      a0.z = fmaf(xv, u.z, a0.z); a0.w = fmaf(xv, u.w, a0.w);
      a1.x = fmaf(xv, t.x, a1.x); a1.y = fmaf(xv, t.y, a1.y);
      a1.z = fmaf(xv, t.z, a1.z); a1.w = fmaf(xv, t.w, a1.w);
    }
  } else if (np == 1) {
#pragma unroll 4
    for (int k = sl; k < K; k += slices) {
      const float xv = sm.xs[k];
      const float4 u = w04[k * P4 + c4];
      a0.x = fmaf(xv, u.x, a0.x); a0.y = fmaf(xv, u.y, a0.y);
      a0.z = fmaf(xv, u.z, a0.z); a0.w = fmaf(xv, u.w, a0.w);
    }
  }
  // lanes with the same float4 column (lane % P4) hold successive row
  // slices: fold them with shuffles, then add the 8 warps' results in order.
  float r[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  for (int o = P4; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] += __shfl_xor_sync(0xffffffffu, r[i], o);
  constexpr int nw = kMegaThreads / 32;
  if ((tid & 31) < P4) {
    const int wq = tid >> 5, cc = (tid & 31) * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sm.red[wq * P + cc + i] = r[i];
      sm.red[(nw + wq) * P + cc + i] = r[4 + i];
    }
  }
  __syncthreads();
  if (tid < P) {
    for (int j = 0; j < np; ++j) {
      float t = 0.f;
      for (int q = 0; q < nw; ++q) t += sm.red[(j * nw + q) * P + tid];
      const int col = (blockIdx.x + j * gridDim.x) * P + tid;
      if (Q4) t *= e.sc[j];
      if (col < m.N) st_word(y + col, apply_act(t + e.add[j], act), ytag);
    }
  }
  __syncthreads();
  return true;
}

// Attention for head h = blockIdx.x (< heads): append k, v of the current
// token at position pos, then out = softmax(q.k_j / sqrt(hd)) v over j <= pos.
// Loads are issued in independent batches (the cache is read from L2).
__device__ void attention_head(const MegaArgs& a, const MegaLayer& L, int64_t pos, float* scr,
                               Smem& sm, int h, bool append, float* ctx_out, uint32_t qtag) {

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, hd = a.hd, H = a.H;
  float* qs = scr;             // [hd]
  float* kn = scr + 128;       // [hd] new key
  float* vn = scr + 256;       // [hd] new value
  float* sc = scr + 384;       // [max_len] scores
  float* part = sc + a.max_len + 4;  // [8 warps][hd], hd <= 128 (reserved 8 x 128)
  float* kh = L.kc + (size_t)h * a.max_len * hd;
  float* vh = L.vc + (size_t)h * a.max_len * hd;
  if (tid < hd) {
    const uint64_t* qp = a.tqkv + h * hd + tid;
    uint64_t w3[3] = {ld_word(qp), ld_word(qp + H), ld_word(qp + 2 * H)};
    settle(w3, qtag, [&](int i) { return qp + i * H; }, a, sm);
    qs[tid] = word_f(w3[0]);
    kn[tid] = word_f(w3[1]);
    vn[tid] = word_f(w3[2]);
    if (append) {
      kh[pos * hd + tid] = kn[tid];
      vh[pos * hd + tid] = vn[tid];
    }
  }
  __syncthreads();
  const int64_t Lk = pos + 1;
  const float sq = sqrtf((float)hd);
  const int hd4 = hd / 4;
  // scores: one thread per key, the key row's hd/4 128-bit loads in flight
  for (int64_t j = tid; j < Lk; j += kMegaThreads) {
    float4 kv[32];
    if (j == pos) {  // the new key, from shared memory
      const float4* kr = reinterpret_cast<const float4*>(kn);
#pragma unroll
      for (int d = 0; d < 32; ++d)
        if (d < hd4) kv[d] = kr[d];
    } else {
      const float4* kr = reinterpret_cast<const float4*>(kh + j * hd);
#pragma unroll
      for (int d = 0; d < 32; ++d)
        if (d < hd4) kv[d] = __ldcg(kr + d);
    }
    float dot = 0.f;
#pragma unroll
    for (int d = 0; d < 32; ++d)
      if (d < hd4) {
        dot = fmaf(qs[4 * d], kv[d].x, dot);
        dot = fmaf(qs[4 * d + 1], kv[d].y, dot);
        dot = fmaf(qs[4 * d + 2], kv[d].z, dot);
        dot = fmaf(qs[4 * d + 3], kv[d].w, dot);
      }
    sc[j] = dot / sq;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int64_t j = tid; j < Lk; j += kMegaThreads) mx = fmaxf(mx, sc[j]);
  mx = warp_max(mx);
  if (lane == 0) sm.red[wid] = mx;
  __syncthreads();
  mx = sm.red[0];
  for (int w = 1; w < kMegaThreads / 32; ++w) mx = fmaxf(mx, sm.red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int64_t j = tid; j < Lk; j += kMegaThreads) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) sm.red[wid] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < kMegaThreads / 32; ++w) sum += sm.red[w];
  const float inv = 1.0f / sum;
  // out: warp w takes keys w, w+8, ...; lane covers dims lane, lane+32, ...
  // (hd <= 128 -> up to 4 dims per lane); 4 keys per batch of loads.
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int nw = kMegaThreads / 32;
  for (int64_t j0 = wid; j0 < Lk; j0 += 4 * nw) {
    float vv[4][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t j = j0 + u * nw;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = lane + 32 * e;
        float t = 0.f;
        if (j < Lk && d < hd) {
          if (j == pos) t = vn[d];
          else t = __ldcg(vh + j * hd + d);
        }
        vv[u][e] = t;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t j = j0 + u * nw;
      const float pj = j < Lk ? sc[j] * inv : 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = fmaf(pj, vv[u][e], acc[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane + 32 * e;
    if (d < hd) part[wid * hd + d] = acc[e];
  }
  __syncthreads();
  if (tid < hd) {
    float r = 0.f;
    for (int w = 0; w < nw; ++w) r += part[w * hd + tid];
    ctx_out[tid] = r;
  }
  __syncthreads();
}

// head_dim == 64: one pass over the keys. Each thread takes keys tid,
// tid + 256, ...; loads the K and V rows together (one L2 round trip per
// key batch), keeps an online-softmax partial (m, l, o[64]); partials are
// merged with a block max and shuffle sums.
__device__ __noinline__ void attention_head64(const MegaArgs& a, const MegaLayer& L, int64_t pos,
                                              float* scr, Smem& sm, int h, bool append,
                                              float* ctx_out, uint32_t qtag, bool pe) {
  stamp_event(a, pe, 7);
#ifdef INFERC_DECODE_PROFILE
  if (a.prof && pe && threadIdx.x == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    a.prof[64 + 32 * blockIdx.x + 15] = smid;
  }
#endif
  constexpr int HD = 64;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, H = a.H;
  constexpr int nw = kMegaThreads / 32;
  float* qs = scr;        // [64]
  float* kn = scr + 128;  // [64]
  float* vn = scr + 256;  // [64]
  float* part = scr + 384 + a.max_len + 4;  // [8][65]
  float* kh = L.kc + (size_t)h * a.max_len * HD;
  float* vh = L.vc + (size_t)h * a.max_len * HD;
  const int half = tid & 1;  // thread pair (2i, 2i+1) shares key i: each lane holds half the dims
  // Cached keys / values (positions < pos) of one pass of 128 keys; the new
  // key at pos comes from shared memory below, the rest are zero.
  auto load_kv = [&](int64_t base, float4 (&kr)[8], float4 (&vr)[8]) {
    const int64_t j = base + (tid >> 1);
    if (j < pos) {
      const float4* kg = reinterpret_cast<const float4*>(kh + j * HD + 32 * half);
      const float4* vg = reinterpret_cast<const float4*>(vh + j * HD + 32 * half);
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        kr[d] = __ldcg(kg + d);
        vr[d] = __ldcg(vg + d);
      }
    } else {
#pragma unroll
      for (int d = 0; d < 8; ++d) kr[d] = vr[d] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  // The first pass's cached rows do not depend on this step's q / k / v:
  // their loads are in flight while this CTA waits for its head's q / k / v.
  float4 kr[8], vr[8];
  load_kv(0, kr, vr);
  if (tid < HD) {
    const uint64_t* qp = a.tqkv + h * HD + tid;
    uint64_t w3[3] = {ld_word(qp), ld_word(qp + H), ld_word(qp + 2 * H)};
    settle(w3, qtag, [&](int i) { return qp + i * H; }, a, sm);
    stamp_event(a, pe, 18);
    qs[tid] = word_f(w3[0]);
    kn[tid] = word_f(w3[1]);
    vn[tid] = word_f(w3[2]);
    if (append) {
      kh[pos * HD + tid] = kn[tid];
      vh[pos * HD + tid] = vn[tid];
    }
  }
  __syncthreads();
  stamp_event(a, pe, 8);
  const int64_t Lk = pos + 1;
  const float sq = sqrtf((float)HD);
  float m = -INFINITY, l = 0.f, o[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d] = 0.f;
  const float4* q4 = reinterpret_cast<const float4*>(qs + 32 * half);
  // The loop bound is warp-uniform (every lane runs every iteration) because
  // the pair shuffle below needs all 32 lanes.
#pragma unroll 1
  for (int64_t base = 0; base < Lk; base += kMegaThreads / 2) {
    const int64_t j = base + (tid >> 1);
    const bool valid = j < Lk;
    if (base > 0) load_kv(base, kr, vr);
    if (j == pos) {
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        kr[d] = reinterpret_cast<const float4*>(kn + 32 * half)[d];
        vr[d] = reinterpret_cast<const float4*>(vn + 32 * half)[d];
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      const float4 qv = q4[d];
      dot = fmaf(qv.x, kr[d].x, dot);
      dot = fmaf(qv.y, kr[d].y, dot);
      dot = fmaf(qv.z, kr[d].z, dot);
      dot = fmaf(qv.w, kr[d].w, dot);
    }
    // dims 0..31 partial + dims 32..63 partial (same sum order in both lanes)
    const float other = __shfl_xor_sync(0xffffffffu, dot, 1);
    if (!valid) continue;
    const float sc = (half == 0 ? dot + other : other + dot) / sq;
    const float mn = fmaxf(m, sc);
    const float c = expf(m - mn);  // 0 on the first key (m = -inf)
    const float p = expf(sc - mn);
    l = l * c + p;
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      o[4 * d] = fmaf(p, vr[d].x, o[4 * d] * c);
      o[4 * d + 1] = fmaf(p, vr[d].y, o[4 * d + 1] * c);
      o[4 * d + 2] = fmaf(p, vr[d].z, o[4 * d + 2] * c);
      o[4 * d + 3] = fmaf(p, vr[d].w, o[4 * d + 3] * c);
    }
    m = mn;
  }
  stamp_event(a, pe, 11);
  // block max of m
  float mx = warp_max(m);
  if (lane == 0) sm.red[wid] = mx;
  __syncthreads();
  stamp_event(a, pe, 12);
  float M = sm.red[0];
#pragma unroll
  for (int w = 1; w < nw; ++w) M = fmaxf(M, sm.red[w]);
  const float scale = (m == -INFINITY) ? 0.f : expf(m - M);
  l = half == 0 ? l * scale : 0.f;  // count each key once
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d] *= scale;
  l = warp_sum(l);
  // Sum o over the 16 lanes of each half (lane bit 0) by reduce-scatter:
  // each round a lane keeps half of its values and adds its partner's copy
  // of them (30 shuffles, not 128). Afterwards lane holds dims
  // 32 half + (lane & 30) + {0, 1} in o[0], o[1].
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int off = 16 >> r;  // also the number of values passed on
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i >= off) break;
      const float send = up ? o[i] : o[i + off];
      const float keep = up ? o[i + off] : o[i];
      o[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  part[wid * 65 + 32 * half + (lane & 30)] = o[0];
  part[wid * 65 + 32 * half + (lane & 30) + 1] = o[1];
  if (lane == 0) part[wid * 65 + 64] = l;
  __syncthreads();
  stamp_event(a, pe, 13);
  if (tid < HD) {
    float r = 0.f, t = 0.f;
#pragma unroll
    for (int w = 0; w < nw; ++w) {
      r += part[w * 65 + tid];
      t += part[w * 65 + 64];
    }
    ctx_out[tid] = r / t;
  }
  __syncthreads();
}

// FC-phase input: xm = xa + b_proj + sum_h part[h] (heads in order); CTA 0
// publishes xm (the FP residual, tagged xm_tag); then LN2 in place.
__device__ void stage_attn_residual(const MegaArgs& a, const float* proj_b, const float* g,
                                    const float* b, const uint64_t* xa, uint32_t xa_tag,
                                    uint32_t part_tag, uint32_t xm_tag, int chunk_w, Smem& sm) {
  const int tid = threadIdx.x, H = a.H;
  // Every CTA waits here for the attention CTAs, most of them from early in
  // the layer. Until then only warp 0 polls, and only the first word of each
  // (head, column chunk) partial (up to 64 words): the full read of all
  // heads' partials (12 x 768 words per CTA in GPT-2-small) starts once
  // every writer has been seen, so the grid's polling does not load L2
  // while the attention CTAs read the KV cache.
  if (tid < 32) {
    const int nsent = a.heads * a.proj_chunks;
    auto sent = [&](int j) {
      return a.tpart + (size_t)(j / a.proj_chunks) * H + (size_t)(j % a.proj_chunks) * chunk_w;
    };
    uint64_t w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int j = tid + 32 * i;
      w[i] = j < nsent ? ld_word(sent(j)) : (uint64_t)part_tag << 32;
    }
    settle(w, part_tag, [&](int i) { return sent(tid + 32 * i); }, a, sm);
  }
  __syncthreads();
  // All loads of the thread (up to 3 k's x 12 heads + x) are issued before
  // any is used: one L2 round trip, not one per k.
  constexpr int kK = 3, kHeads = 16;
  uint64_t p[kK * kHeads], xw[kK];  // p[i * kHeads + h]: head h at k = tid + 256 i
  float bp[kK];
#pragma unroll
  for (int i = 0; i < kK; ++i) {
    const int k = tid + i * kMegaThreads;
    const bool in = k < H;
#pragma unroll
    for (int h = 0; h < kHeads; ++h)
      p[i * kHeads + h] = (in && h < a.heads) ? ld_word(a.tpart + (size_t)h * H + k)
                                              : (uint64_t)part_tag << 32;
    xw[i] = in ? ld_word(xa + k) : (uint64_t)xa_tag << 32;
    bp[i] = in ? proj_b[k] : 0.f;
  }
  settle(p, part_tag, [&](int j) {
    return a.tpart + (size_t)(j % kHeads) * H + tid + (j / kHeads) * kMegaThreads;
  }, a, sm);
  settle(xw, xa_tag, [&](int i) { return xa + tid + i * kMegaThreads; }, a, sm);
#pragma unroll
  for (int i = 0; i < kK; ++i) {
    const int k = tid + i * kMegaThreads;
    if (k >= H) continue;
    float t = 0.f;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) t += word_f(p[i * kHeads + h]);
    const float v = word_f(xw[i]) + (t + bp[i]);
    sm.xs[k] = v;
    if (blockIdx.x == 0) st_word(a.txm + k, v, xm_tag);
  }
  // wider rows than kK * kMegaThreads (not GPT-2-small): the remainder
  for (int k = tid + kK * kMegaThreads; k < H; k += kMegaThreads) {
    float t = 0.f;
    for (int h = 0; h < a.heads; ++h) {
      const uint64_t* pp = a.tpart + (size_t)h * H + k;
      uint64_t pw[1] = {ld_word(pp)};
      settle(pw, part_tag, [&](int) { return pp; }, a, sm);
      t += word_f(pw[0]);
    }
    uint64_t rw[1] = {ld_word(xa + k)};
    settle(rw, xa_tag, [&](int) { return xa + k; }, a, sm);
    const float v = word_f(rw[0]) + (t + proj_b[k]);
    sm.xs[k] = v;
    if (blockIdx.x == 0) st_word(a.txm + k, v, xm_tag);
  }
  __syncthreads();
  stage_smem_ln(H, g, b, a.eps, sm);
}

// Attention + output projection for one (head, column chunk): CTA c < heads
// * chunks computes head h = c / chunks (redundantly with the other chunks
// of that head; chunk 0 also appends the new K/V to the cache), then
// part[h][cols] = ctx_h . W_proj[h*hd:(h+1)*hd, cols] from its prefetched
// [hd][Wc] panel in slot `slot`. The partials are summed (fixed order) by
// the next phase.
template <bool Q4>
__device__ bool attn_proj_phase(const MegaArgs& a, const MegaLayer& L, int64_t pos, float* scr,
                                const uint8_t* slots, int slot, Smem& sm, uint32_t qtag,
                                uint32_t part_tag, bool pe) {
  const int chunks = a.proj_chunks;
  const int c = blockIdx.x;
  if (c >= a.heads * chunks) return true;
  const int h = c / chunks, cc = c % chunks;
  float* ctx = scr + 384 + a.max_len + 4 + (kMegaThreads / 32) * 128;  // [hd]
  const int tid = threadIdx.x;
  const int Wc = L.proj.P, hd = a.hd;
  // int4: the chunk's column scales, loaded while the attention runs
  float csc = 1.f;
  if (Q4 && tid < Wc && cc * Wc + tid < a.H) csc = __ldg(L.proj.scale + cc * Wc + tid);
  if (a.hd == 64)
    attention_head64(a, L, pos, scr, sm, h, cc == 0, ctx, qtag, pe);
  else
    attention_head(a, L, pos, scr, sm, h, cc == 0, ctx, qtag);
  stamp_event(a, pe, 9);
  if (!wait_slot(slot, sm, a)) return false;
  stamp_event(a, pe, 10);
  // L.proj: K = hd, P = chunk width
  const float* w = reinterpret_cast<const float*>(slots + (size_t)slot * kSlotBytes);
  // threads: (column, row-slice); Wc <= 256
  const int slices = kMegaThreads / Wc;
  const int col = tid % Wc, sl = tid / Wc;
  // four independent partial sums (rows k, k + slices, ...) shorten the chain
  float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
  if constexpr (Q4) {
    // [hd/8][Wc] words: word (kg, c) = 8 consecutive k of column c
    const uint32_t* wq = reinterpret_cast<const uint32_t*>(w);
    for (int kg = sl; sl < slices && kg < hd / 8; kg += slices) {
      const uint32_t q = wq[kg * Wc + col];
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        d0 = fmaf((float)((int)((q >> (4 * i)) & 15u) - 8), ctx[8 * kg + i], d0);
        d1 = fmaf((float)((int)((q >> (4 * i + 4)) & 15u) - 8), ctx[8 * kg + i + 1], d1);
      }
      if (kg & 1) c1 += d0 + d1; else c0 += d0 + d1;
    }
  } else if (sl < slices) {
    int k = sl;
    for (; k + 3 * slices < hd; k += 4 * slices) {
      c0 = fmaf(ctx[k], w[k * Wc + col], c0);
      c1 = fmaf(ctx[k + slices], w[(k + slices) * Wc + col], c1);
      c2 = fmaf(ctx[k + 2 * slices], w[(k + 2 * slices) * Wc + col], c2);
      c3 = fmaf(ctx[k + 3 * slices], w[(k + 3 * slices) * Wc + col], c3);
    }
    for (; k < hd; k += slices) c0 = fmaf(ctx[k], w[k * Wc + col], c0);
  }
  sm.red[tid] = (c0 + c1) + (c2 + c3);
  __syncthreads();
  stamp_event(a, pe, 16);
  if (tid < Wc) {
    float t = 0.f;
    for (int q = 0; q < slices; ++q) t += sm.red[q * Wc + tid];
    const int gcol = cc * Wc + tid;
    if (Q4) t *= csc;
    if (gcol < a.H) st_word(a.tpart + (size_t)h * a.H + gcol, t, part_tag);
  }
  stamp_event(a, pe, 17);
  __syncthreads();
  return true;
}

}  // namespace

template <bool Q4>
__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(const __grid_constant__ MegaArgs a) {
  extern __shared__ __align__(128) uint8_t mega_smem[];
  uint8_t* slots = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mega_smem) + 127) &
                                              ~uintptr_t(127));
  __shared__ Smem sm;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mb_init(&sm.bar[s], 1);
      mb_init(&sm.empty[s], kLmWarps);
      sm.empty_uses[s] = 0;
      sm.uses[s] = 0;
      sm.issued[s] = 0;
    }
    mb_init(&sm.ln_bar, 1);
    sm.ln_uses = 0;
    sm.ln_issued = 0;
    sm.abort_flag = 0;
    sm.nbar = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int H = a.H;
  float* scr = reinterpret_cast<float*>(slots + (size_t)kSlots * kSlotBytes);
  // Tags of one step, increasing in the order the words are written (every
  // buffer sees only growing tags): the embedding (layer 0's input) is
  // tag_step + 1; phase ph (0 QKV, 1 projection partials, 2 FC / xm, 3 FP) of
  // layer l is tag_step + 4 l + ph + 2, so layer l's input is tag_step + 4 l + 1.
  const uint32_t tags_per_step = 4u * (uint32_t)a.layers + 1u;

  int64_t tok = *a.tok;
  // Copies are issued one phase ahead, by thread 0 between its arrival at a
  // grid barrier and its wait there: a slot pair is refilled as soon as this
  // CTA has consumed it, off the critical path of the next phase.
  auto issue_proj = [&](const MegaLayer& Lx) {  // W_proj panel -> slot 2
    if (tid == kIssuer && blockIdx.x < (unsigned)(a.heads * a.proj_chunks)) {
      const uint32_t bytes = Lx.proj.bytes;
      sm.issued[2]++;
      mb_expect_tx(&sm.bar[2], bytes);
      bulk_load_stream(slots + 2 * (size_t)kSlotBytes,
                       Lx.proj.data + (size_t)blockIdx.x * bytes, bytes,
                       &sm.bar[2]);
    }
  };
  // LM head chunks: 16 rows of wte (48 KiB) per chunk, this CTA's row range.
  const int lm_rows = (a.V + gridDim.x - 1) / gridDim.x;
  const int lm_r0 = blockIdx.x * lm_rows;
  const int lm_r1 = min(a.V, lm_r0 + lm_rows);
  // LM-head rows: fp32 wte [V][H] or the int4 head [V][H/2]
  const int lm_row_bytes = Q4 ? H / 2 : H * 4;
  const int lm_crow = kSlotBytes / lm_row_bytes;
  const int lm_nchunks = lm_r1 > lm_r0 ? (lm_r1 - lm_r0 + lm_crow - 1) / lm_crow : 0;
  auto issue_lm = [&](int ch) {
    if (tid != kIssuer || ch >= lm_nchunks) return;
    const int s = ch % kSlots;
    const int ra = lm_r0 + ch * lm_crow, rb = min(lm_r1, ra + lm_crow);
    const uint32_t bytes = (uint32_t)(rb - ra) * lm_row_bytes;
    sm.issued[s]++;
    mb_expect_tx(&sm.bar[s], bytes);
    const uint8_t* src = (Q4 ? a.lm_q : reinterpret_cast<const uint8_t*>(a.wte)) +
                         (size_t)ra * lm_row_bytes;
    for (uint32_t off = 0; off < bytes; off += a.piece)
      bulk_load_stream(slots + (size_t)s * kSlotBytes + off, src + off,
                       min(a.piece, bytes - off), &sm.bar[s]);
  };
  prefetch_ln(a.layer[0].ln1_g, a.layer[0].ln1_b, nullptr, H, sm);
  prefetch_panels(a.layer[0].attn, 0, slots, sm, a.piece);
  issue_proj(a.layer[0]);
  for (int step = 0; step < a.nsteps; ++step) {
    const int64_t pos = a.pos0 + step;
    if (tok < 0 || tok >= a.V || pos < 0 || pos >= a.max_pos || pos >= a.max_len) {
      if (tid == 0) atomicExch(a.err, 2);
      drain(sm);
      return;
    }
    const uint32_t tag_step = a.tag_base + (uint32_t)step * tags_per_step;
#ifdef INFERC_DECODE_PROFILE
    if (a.prof && step == 1 && blockIdx.x == 0 && tid == 0) a.prof[0] = gtimer();
#endif
    for (int l = 0; l < a.layers; ++l) {
      const MegaLayer& L = a.layer[l];  // read on use (keeps registers free)
      const bool last = l + 1 == a.layers;
      const uint32_t tag_in = tag_step + 4u * (uint32_t)l + 1u;  // this layer's input
      const uint32_t tag_l = tag_in;  // phase ph writes tag_l + ph + 1
      const uint64_t* xin = a.tx + (size_t)(l & 1) * H;
      // ---- QKV (pair 0; W_proj is in slot 2, LN1's gamma / beta in sm.lnp)
      const EpiIn e_qkv = gemv_preload(L.attn, L.attn_b, nullptr, 0u, a, sm);
      const float *g1, *b1, *unused;
      if (!ln_params(L.ln1_g, L.ln1_b, nullptr, H, sm, a, &g1, &b1, &unused)) { drain(sm); return; }
      if (l == 0) {
        // Embedding of the current token, built by every CTA; CTA 0 also
        // publishes it as the residual stream.
        for (int k = tid; k < H; k += kMegaThreads) {
          const float v = __ldg(a.wte + tok * H + k) + __ldg(a.wpe + pos * H + k);
          sm.xs[k] = v;
          if (blockIdx.x == 0) st_word(a.tx + k, v, tag_in);
        }
        __syncthreads();
        stage_smem_ln(H, g1, b1, a.eps, sm);
      } else {
        stage_input(xin, tag_in, H, g1, b1, a.eps, sm, a);
      }
      stamp_event(a, step == 1 && l == 5, 0);
      if (!gemv_phase<Q4>(L.attn, 0, slots, e_qkv, a.tqkv, tag_l + 1u, ACT_NONE, sm, a) ||
          !phase_end(a, sm, 4 * l + 0, step)) { drain(sm); return; }
      stamp_event(a, step == 1 && l == 5, 1);
      prefetch_ln(L.ln2_g, L.ln2_b, L.proj_b, H, sm);  // LN1's copy consumed
      prefetch_panels(L.fc, 0, slots, sm, a.piece);  // pair 0 consumed
      stamp_event(a, step == 1 && l == 5, 14, kIssuer);
      // ---- attention + output projection partials (slot 2)
      if (!attn_proj_phase<Q4>(a, L, pos, scr, slots, 2, sm, tag_l + 1u, tag_l + 2u,
                           step == 1 && l == 5) ||
          !phase_end(a, sm, 4 * l + 1, step)) { drain(sm); return; }
      stamp_event(a, step == 1 && l == 5, 2);
      prefetch_panels(L.fp, 1, slots, sm, a.piece);  // slot 2 consumed, slot 3 free
      // ---- FC (pair 0): xm = xa + b_proj + sum_h part[h]; f = gelu(LN2(xm) W + b).
      const EpiIn e_fc = gemv_preload(L.fc, L.fc_b, nullptr, 0u, a, sm);
      const float *g2, *b2, *pb;
      if (!ln_params(L.ln2_g, L.ln2_b, L.proj_b, H, sm, a, &g2, &b2, &pb)) { drain(sm); return; }
      stage_attn_residual(a, pb, g2, b2, xin, tag_in, tag_l + 2u, tag_l + 3u, L.proj.P, sm);
      stamp_event(a, step == 1 && l == 5, 3);
      if (!gemv_phase<Q4>(L.fc, 0, slots, e_fc, a.tf, tag_l + 3u, ACT_GELU_TANH, sm, a) ||
          !phase_end(a, sm, 4 * l + 2, step)) { drain(sm); return; }
      stamp_event(a, step == 1 && l == 5, 4);
      // LN2's copy consumed: the next LayerNorm's vectors (small, first)
      if (!last) prefetch_ln(a.layer[l + 1].ln1_g, a.layer[l + 1].ln1_b, nullptr, H, sm);
      else prefetch_ln(a.lnf_g, a.lnf_b, nullptr, H, sm);
      if (!last) prefetch_panels(a.layer[l + 1].attn, 0, slots, sm, a.piece);  // pair 0 consumed
      // ---- FP (pair 1): x_next = xm + f W + b
      const EpiIn e_fp = gemv_preload(L.fp, L.fp_b, a.txm, tag_l + 3u, a, sm);
      stage_input(a.tf, tag_l + 3u, a.F, nullptr, nullptr, 0.f, sm, a);
      stamp_event(a, step == 1 && l == 5, 5);
      if (!gemv_phase<Q4>(L.fp, 1, slots, e_fp, a.tx + (size_t)((l + 1) & 1) * H, tag_l + 4u,
                      ACT_NONE, sm, a) ||
          !phase_end(a, sm, 4 * l + 3, step)) { drain(sm); return; }
      stamp_event(a, step == 1 && l == 5, 6);
      if (!last) {
        issue_proj(a.layer[l + 1]);  // slot 2 consumed
      } else {
        for (int ch = 0; ch < kSlots; ++ch) issue_lm(ch);  // every slot consumed
      }
    }
    // LM head: logits = LNf(x) . wte[r] for this CTA's row range, streamed
    // through all four slots (the first four chunks are already in flight).
    {
      const float *gf, *bf, *unused;
      if (!ln_params(a.lnf_g, a.lnf_b, nullptr, H, sm, a, &gf, &bf, &unused)) { drain(sm); return; }
      // the last layer's FP output, tagged tag_step + 4 layers + 1
      stage_input(a.tx + (size_t)(a.layers & 1) * H, tag_step + tags_per_step, H, gf, bf,
                  a.eps, sm, a);
    }
    {
      // A ring over the four slots without CTA barriers: row warps wait for a
      // chunk's copy on its full barrier and release the slot on its empty
      // barrier; the issuer refills a slot once all row warps released it.
      const int r0 = lm_r0, r1 = lm_r1, crow = lm_crow, nchunks = lm_nchunks;
      float bv = -INFINITY;
      int64_t bi = INT64_MAX;
      bool ok = true;
      if (wid < kLmWarps) {
        for (int ch = 0; ch < nchunks && ok; ++ch) {
          const int s = ch % kSlots;
          ok = mb_wait(&sm.bar[s], (sm.uses[s] + ch / kSlots) & 1);
          if (!ok) break;
          const uint8_t* w = slots + (size_t)s * kSlotBytes;
          const int ra = r0 + ch * crow, rb = min(r1, ra + crow);
          for (int r = ra + wid; r < rb; r += kLmWarps) {
            const float4* x4 = reinterpret_cast<const float4*>(sm.xs);
            float acc = 0.f;
            if constexpr (Q4) {
              // row of H/8 words (8 consecutive k each, low nibble first)
              const float rs = __ldg(a.lm_s + r);
              const uint32_t* wr = reinterpret_cast<const uint32_t*>(w + (size_t)(r - ra) * (H / 2));
              for (int k = lane; k < H / 8; k += 32) {
                const uint32_t q = wr[k];
                const float4 xa = x4[2 * k], xb = x4[2 * k + 1];
                const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  acc = fmaf((float)((int)((q >> (4 * i)) & 15u) - 8), xv[i], acc);
              }
              acc = warp_sum(acc) * rs;
            } else {
              const float4* wr = reinterpret_cast<const float4*>(w + (size_t)(r - ra) * H * 4);
              for (int k = lane; k < H / 4; k += 32) {
                const float4 wv = wr[k], xv = x4[k];
                acc = fmaf(xv.x, wv.x, acc);
                acc = fmaf(xv.y, wv.y, acc);
                acc = fmaf(xv.z, wv.z, acc);
                acc = fmaf(xv.w, wv.w, acc);
              }
              acc = warp_sum(acc);
            }
            if (lane == 0) a.logits[r] = acc;
            if (acc > bv || (acc == bv && r < bi)) { bv = acc; bi = r; }
          }
          __syncwarp();
          if (lane == 0) mb_arrive(&sm.empty[s]);
        }
      } else if (tid == kIssuer) {
        // chunks 0..kSlots-1 were issued at the end of the last layer
        for (int ch = 0; ch + kSlots < nchunks && ok; ++ch) {
          const int s = ch % kSlots;
          ok = mb_wait(&sm.empty[s], sm.empty_uses[s] & 1);
          sm.empty_uses[s]++;
          if (ok) issue_lm(ch + kSlots);
        }
        // the last chunks' releases, so empty[] parity stays in step
        for (int ch = max(0, nchunks - kSlots); ch < nchunks && ok; ++ch) {
          const int s = ch % kSlots;
          ok = mb_wait(&sm.empty[s], sm.empty_uses[s] & 1);
          sm.empty_uses[s]++;
        }
      }
      if (!ok) {
        atomicExch(a.err, 1);
        sm.abort_flag = 1;
      }
      if (lane == 0) { sm.bv[wid] = bv; sm.bi[wid] = bi; }
      __syncthreads();
      if (tid == 0) {
        // completed waits of the row warps, per slot (after an abort the count
        // stays short, so drain() waits, bounded, for every copy issued)
        if (sm.abort_flag == 0)
          for (int s = 0; s < kSlots; ++s) sm.uses[s] += (nchunks - s + kSlots - 1) / kSlots;
        float v = sm.bv[0];
        int64_t i = sm.bi[0];
        for (int w = 1; w < kMegaThreads / 32; ++w)
          if (sm.bv[w] > v || (sm.bv[w] == v && sm.bi[w] < i)) { v = sm.bv[w]; i = sm.bi[w]; }
        a.best_v[blockIdx.x] = v;
        a.best_i[blockIdx.x] = i;
      }
    }
    // Next step's first weights stream while the argmax is finalised.
    if (!phase_end(a, sm, 4 * a.layers, step)) { drain(sm); return; }
    grid_arrive(a, sm);
    if (step + 1 < a.nsteps) {
      prefetch_ln(a.layer[0].ln1_g, a.layer[0].ln1_b, nullptr, H, sm);
      prefetch_panels(a.layer[0].attn, 0, slots, sm, a.piece);
      issue_proj(a.layer[0]);
    }
    if (!grid_wait(a, sm)) { drain(sm); return; }
    // Every CTA reduces the per-CTA bests in the same order (first max wins).
    if (wid == 0) {
      float v = -INFINITY;
      int64_t i = INT64_MAX;
      for (int b = lane; b < (int)gridDim.x; b += 32) {
        const float ov = __ldcg(a.best_v + b);
        const int64_t oi = __ldcg(a.best_i + b);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
      }
      if (lane == 0) sm.bi[0] = (i == INT64_MAX) ? 0 : i;
    }
    __syncthreads();
    tok = sm.bi[0];
    if (blockIdx.x == 0 && tid == 0) {
      a.token_log[a.log_offset + step] = tok;
      *a.tok = tok;
    }
  }
}

// ------------------------------------------------------------ host side
size_t mega_smem_bytes(int max_len) {
  // attention scratch: q, k_new, v_new (3 x 128), scores [max_len] (+4 pad),
  // per-warp partial outputs [8][128], the head's context [128]
  return (size_t)kSlots * kSlotBytes + 128 +
         (size_t)(384 + max_len + 4 + (kMegaThreads / 32) * 128 + 128) * sizeof(float);
}

void launch_decode_mega(const MegaArgs& a, int grid, bool q4, cudaStream_t st) {
  const size_t smem = mega_smem_bytes(a.max_len);
  const void* fn = q4 ? (const void*)decode_mega_kernel<true> : (const void*)decode_mega_kernel<false>;
  IDEV_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* args[] = {const_cast<MegaArgs*>(&a)};
  IDEV_CUDA(cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kMegaThreads), args, smem, st));
}

int mega_max_grid(int max_len, bool q4) {
  const size_t smem = mega_smem_bytes(max_len);
  const void* fn = q4 ? (const void*)decode_mega_kernel<true> : (const void*)decode_mega_kernel<false>;
  IDEV_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0, dev = 0, sms = 0;
  IDEV_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kMegaThreads, smem));
  IDEV_CUDA(cudaGetDevice(&dev));
  IDEV_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return std::min(per_sm, 1) * sms;
}

// Re-tiles W [K,N] (device, row-major) into panels [npanels][K][P] (zero
// padded past N).
__global__ void panelize_kernel(const float* __restrict__ w, float* __restrict__ out, int K, int N,
                                int P, int npanels) {
  const int64_t total = (int64_t)npanels * K * P;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % P);
    const int k = (int)((e / P) % K);
    const int p = (int)(e / ((int64_t)P * K));
    const int col = p * P + c;
    out[e] = col < N ? w[(int64_t)k * N + col] : 0.f;
  }
}

// W_proj [H, H] -> panels [heads][chunks][hd][Wc]: rows of head h, columns
// of chunk cc (zero padded past H).
__global__ void panelize_proj_kernel(const float* __restrict__ w, float* __restrict__ out, int H,
                                     int hd, int heads, int chunks, int Wc) {
  const int64_t total = (int64_t)heads * chunks * hd * Wc;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % Wc);
    const int k = (int)((e / Wc) % hd);
    const int cc = (int)((e / ((int64_t)Wc * hd)) % chunks);
    const int h = (int)(e / ((int64_t)Wc * hd * chunks));
    const int col = cc * Wc + c;
    out[e] = col < H ? w[(int64_t)(h * hd + k) * H + col] : 0.f;
  }
}

void launch_panelize_proj(const float* w, float* out, int H, int hd, int heads, int chunks, int Wc,
                          cudaStream_t st) {
  panelize_proj_kernel<<<148 * 8, 256, 0, st>>>(w, out, H, hd, heads, chunks, Wc);
  IDEV_LAUNCHED();
}

// int4 [N, K/2] (row n: K/8 words, 8 consecutive k each) -> panels
// [npanels][K/8][P] words; columns past N get 8s (q - 8 = 0).
__global__ void panelize_q4_kernel(const uint8_t* __restrict__ q, uint32_t* __restrict__ out,
                                   int K, int N, int P, int npanels) {
  const int KG = K / 8;
  const int64_t total = (int64_t)npanels * KG * P;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % P);
    const int kg = (int)((e / P) % KG);
    const int p = (int)(e / ((int64_t)P * KG));
    const int n = p * P + c;
    out[e] = n < N ? reinterpret_cast<const uint32_t*>(q + (int64_t)n * (K / 2))[kg] : 0x88888888u;
  }
}

// int4 W_proj [H (out), H/2] -> [heads][chunks][hd/8][Wc] words: k groups of
// head h, columns of chunk cc (8s past H).
__global__ void panelize_proj_q4_kernel(const uint8_t* __restrict__ q, uint32_t* __restrict__ out,
                                        int H, int hd, int heads, int chunks, int Wc) {
  const int KG = hd / 8;
  const int64_t total = (int64_t)heads * chunks * KG * Wc;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % Wc);
    const int kg = (int)((e / Wc) % KG);
    const int cc = (int)((e / ((int64_t)Wc * KG)) % chunks);
    const int h = (int)(e / ((int64_t)Wc * KG * chunks));
    const int n = cc * Wc + c;
    out[e] = n < H ? reinterpret_cast<const uint32_t*>(q + (int64_t)n * (H / 2))[h * KG + kg]
                   : 0x88888888u;
  }
}

void launch_panelize_q4(const uint8_t* q, uint32_t* out, int K, int N, int P, int npanels,
                        cudaStream_t st) {
  const int64_t total = (int64_t)npanels * (K / 8) * P;
  panelize_q4_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16), 256, 0, st>>>(
      q, out, K, N, P, npanels);
  IDEV_LAUNCHED();
}

void launch_panelize_proj_q4(const uint8_t* q, uint32_t* out, int H, int hd, int heads,
                             int chunks, int Wc, cudaStream_t st) {
  panelize_proj_q4_kernel<<<148 * 8, 256, 0, st>>>(q, out, H, hd, heads, chunks, Wc);
  IDEV_LAUNCHED();
}

void launch_panelize(const float* w, float* out, int K, int N, int P, int npanels,
                     cudaStream_t st) {
  const int64_t total = (int64_t)npanels * K * P;
  panelize_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16), 256, 0, st>>>(
      w, out, K, N, P, npanels);
  IDEV_LAUNCHED();
}

}  // namespace inferc_dev
