// Parameters of the persistent decode kernel (decode_mega.cu).
#pragma once

#include "common.cuh"

namespace inferc_dev {

// ------------------------------------------------------------ parameters
// Column panels of one weight matrix, contiguous per panel:
//  - fp32: [npanels][K][P] floats;
//  - int4 (per-output-column scale): [npanels][K/8][P] 32-bit words, word
//    (kg, c) holding q[n][8 kg .. 8 kg + 7] of column n = p P + c in the
//    reference's nibble order (low nibble first); columns past N hold 8s.
struct MegaPanels {
  const uint8_t* data;
  int K, N, P, npanels;
  uint32_t bytes;      // one panel
  const float* scale;  // int4: s[n] per output column; fp32: null
};

struct MegaLayer {
  MegaPanels attn, proj, fc, fp;
  const float *attn_b, *proj_b, *fc_b, *fp_b;
  const float *ln1_g, *ln1_b, *ln2_g, *ln2_b;
  float *kc, *vc;  // [heads][max_len][hd]
};

constexpr int kMegaMaxLayers = 48;

struct MegaArgs {
  // The layer records travel in the kernel parameters (constant bank): with
  // the panel ring taking nearly all of shared memory little L1 is left, and
  // from global memory every phase's first look at its record was an L2
  // round trip on the critical path.
  MegaLayer layer[kMegaMaxLayers];
  int layers, H, heads, hd, F, V, max_len, max_pos;
  float eps;
  const float *wte, *wpe, *lnf_g, *lnf_b;
  const uint8_t* lm_q;  // int4 LM head [V][H/2] (rows contiguous) and its scales [V]
  const float* lm_s;
  // Activations passed between CTAs inside a step. Every 64-bit word holds
  // (tag << 32) | fp32 bits and is written once per phase instance with that
  // instance's tag, so a reader's load is also its wait: it re-reads a word
  // until the tag it expects is there (a single-copy-atomic 8-byte access
  // carries the value and its tag together). Tags run tag_base + 1 ...
  // tag_base + nsteps * (4 * layers + 1) over a launch.
  uint64_t* tx;     // [2][H] layer inputs: layer l reads tx[l & 1]
  uint64_t* txm;    // [H] residual stream after the attention block
  uint64_t* tqkv;   // [3H]
  uint64_t* tpart;  // [heads][H] output-projection partials
  uint64_t* tf;     // [F] FC output
  uint32_t tag_base;
  uint32_t piece;  // bytes per bulk copy of a weight panel or LM-head chunk (multiple of 16)
  float* logits;
  int proj_chunks;  // column chunks per head in the attention block
  float* best_v;
  int64_t* best_i;
  unsigned int* bar_count;  // end-of-step grid barrier (zeroed before each launch)
  int* err;
  int64_t* tok;        // in: current token; out: last generated token
  int64_t* token_log;  // token_log[log_offset + s] = token generated at step s
  int64_t log_offset;
  int64_t pos0;        // position of the current token at the first step
  int nsteps;
  unsigned long long* prof;  // optional: phase timestamps of CTA 0, step 1
};


// Dynamic shared memory the kernel needs for a cache of max_len positions.
size_t mega_smem_bytes(int max_len);
// CTAs that can be co-resident (0 when the kernel does not fit); q4 selects
// the int4-weight form of the kernel.
int mega_max_grid(int max_len, bool q4);
void launch_decode_mega(const MegaArgs& a, int grid, bool q4, cudaStream_t st);
void launch_panelize(const float* w, float* out, int K, int N, int P, int npanels,
                     cudaStream_t st);
void launch_panelize_proj(const float* w, float* out, int H, int hd, int heads, int chunks, int Wc,
                          cudaStream_t st);
// int4 [N, K/2] per-row-scale weights (the reference's layout) into panels.
void launch_panelize_q4(const uint8_t* q, uint32_t* out, int K, int N, int P, int npanels,
                        cudaStream_t st);
void launch_panelize_proj_q4(const uint8_t* q, uint32_t* out, int H, int hd, int heads,
                             int chunks, int Wc, cudaStream_t st);

}  // namespace inferc_dev
