// step.cuh — the whole batch-1 decode step of a single-GPU model as one
// persistent kernel.
//
// Replaces the per-layer kernel chain of the decode step (qkv GEMV ->
// attention -> o GEMV -> gate|up GEMV -> down GEMV, or for a mixture of
// experts router GEMV -> top-k -> the selected experts' gate|up and down
// GEMVs; then the lm_head with argmax; the traced step of
// crates/serve/src/compiled.rs:127-201, the MoE block of
// crates/ops/src/moe.rs:103-207).  One CTA per SM stays resident for
// the whole step.  Each CTA's producer warp streams the packed weights (and
// the KV rows its attention split reads) of phase after phase into a
// shared-memory ring without waiting for the phases to start: weights do not
// depend on activations, so HBM keeps streaming while the consumers wait for
// their inputs.
//
// Phases hand their outputs on through flag words: 64-bit words whose low
// half holds 4 bytes of data (two bf16) and whose high half holds the flag of
// the (step, layer) that wrote them.  A word is written by one 64-bit store
// and read by 64-bit loads, so its data and flag travel together: a consumer
// polls the words of its input vector until every flag is the expected one,
// and needs neither a grid barrier nor a separate flag.  Flags grow by one
// per layer; the host clears the words before the 32-bit flag could wrap.
#pragma once
#include "pgemv_dev.cuh"

namespace emx {

struct StepLayer {
  const unsigned char* w[4];  // packed qkv, o, gate|up, down (pgemv layout; MoE: the expert tensors
                              // [experts][rows / 16][tiles])
  const unsigned char* router;  // packed MoE router [experts][hidden] (nullptr: dense)
  const bf16* in_norm;        // [H]
  const bf16* post_norm;      // [H]
  const bf16* q_norm;         // [128] or nullptr
  const bf16* k_norm;         // [128] or nullptr
  bf16* kc;                   // [n_kv, cap, 128]
  bf16* vc;
};

enum StepMat : int { kMatQkv = 0, kMatO = 1, kMatGu = 2, kMatDown = 3, kMatLm = 4, kMatRouter = 5 };
constexpr int kStepMats = 6;
constexpr int kStepMaxTopK = 16;
constexpr int kStepMaxExperts = 256;

struct StepArgs {
  const StepLayer* layers;  // device array [n_layers]
  int n_layers;
  pg::PGeom geo[kStepMats];  // per matrix kind, offsets in this kernel's layout (MoE: gate|up and
                             // down are the gathered expert matrices, top_k slots)
  int bits[kStepMats];
  const unsigned char* lm_w;  // packed lm_head (the embedding when tied)
  const bf16* final_norm;
  const uint32_t* emb_w;  // quantized embedding table
  const bf16* emb_s;
  const bf16* emb_b;
  int emb_bits, emb_gs, vocab;
  int* token;  // in: this step's token; out: the next one
  int H, I;
  float eps;
  // flag-word exchange buffers (two bf16 per word)
  uint64_t* xw;    // residual stream after a layer [H / 2]
  uint64_t* qkvw;  // fused q|k|v projection [(nq + 2 nkv) * 64]
  uint64_t* attw;  // attention output [nq * 64]
  uint64_t* xmw;   // residual after the attention block [H / 2]
  uint64_t* hw;    // SwiGLU output [I / 2] (MoE: [top_k][moe_inter / 2])
  uint64_t* rlw;   // MoE router logits [experts / 2]
  int moe, n_experts, top_k, norm_topk;
  int egu_lps, edown_lps;  // logical blocks per expert slot of the gate|up and down matrices
  unsigned* epoch;  // steps since the words were cleared (the last CTA adds one)
  unsigned* abort_word;  // nonzero: a CTA gave up on a wait; every CTA leaves
  bf16* logits;          // [vocab]
  const float2* rope_cs;  // (cos, sin) [cap][64]
  int cap, nq, nkv;
  float scale;        // 1 / sqrt(head_dim)
  float scale_log2e;  // scale * log2 e: scores in the base-2 domain
  uint64_t* attn_pw;  // split partials in flag words [n_kv][max_splits][hpg][130]: m, l, unnormalised output
  int max_splits;
  int* pos;  // device offset; += 1 at the end of the step
  int* hist;
  int* hist_n;
  int hist_cap;
  float* am_val;  // [grid]
  int* am_idx;
  unsigned* am_ticket;
  int nsm;  // grid = one CTA per SM
  int slot_bytes, nslots;
  int off_aux, aux_stride, off_res, off_u, off_ring;
  int off_args;  // this structure's copy in shared memory
  int* status;
};

struct StepShape {
  int H, I, nq, nkv, hd, vocab, gs, layers, cap;
  int bits[kStepMats];  // qkv, o, gate|up, down, lm_head, router
  int n_experts, top_k, moe_inter, norm_topk;  // n_experts 0: dense (I the MLP width)
};

struct StepPlan {
  int grid, smem, hpg;
  StepArgs tmpl;  // geometry and layout (pointers unset)
};

constexpr int kStepBuffers = 6;
// Flag-word counts of the exchange buffers (xw, qkvw, attw, xmw, hw, rlw in order).
void step_exchange_words(const StepShape& sh, size_t words[kStepBuffers]);
// Plans the step within `budget` bytes of shared memory per CTA; 0 on success.
int step_make_plan(const StepShape& sh, int num_sms, int budget, StepPlan* plan);
// CTAs of the step kernel that fit on one SM (0: the plan cannot launch).
int step_occupancy(const StepPlan& p);
// Launches one decode step (cooperative: all CTAs resident, which the
// flag-word waits require).
cudaError_t step_launch(const StepArgs& a, const StepPlan& p, cudaStream_t st, bool coop);

}  // namespace emx
