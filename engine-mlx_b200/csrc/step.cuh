// step.cuh — the whole batch-1 decode step of a dense model as one
// persistent kernel.
//
// Replaces, for a dense single-GPU model, the per-layer kernel chain of the
// decode step (qkv GEMV -> attention -> o GEMV -> gate|up GEMV -> down GEMV,
// then the lm_head with argmax; the traced step of
// crates/serve/src/compiled.rs:127-201).  Every CTA stays resident for the
// whole step; phases are separated by a grid-wide barrier on a device
// counter instead of a kernel boundary, and each CTA's producer warp streams
// the packed weights (and the KV rows its attention split reads) of phase
// after phase into a shared-memory ring without waiting for the phases to
// start: weights do not depend on activations, so HBM keeps streaming
// across the barriers.  Work is assigned per SM (two CTAs per SM share an SM's
// slice), so no SM holds more than its share.
#pragma once
#include "pgemv_dev.cuh"

namespace emx {

struct StepLayer {
  const unsigned char* w[4];  // packed qkv, o, gate|up, down (pgemv layout)
  const bf16* in_norm;        // [H]
  const bf16* post_norm;      // [H]
  const bf16* q_norm;         // [128] or nullptr
  const bf16* k_norm;         // [128] or nullptr
  bf16* kc;                   // [n_kv, cap, 128]
  bf16* vc;
};

enum StepMat : int { kMatQkv = 0, kMatO = 1, kMatGu = 2, kMatDown = 3, kMatLm = 4 };

struct StepArgs {
  const StepLayer* layers;  // device array [n_layers]
  int n_layers;
  pg::PGeom geo[5];  // per matrix kind, offsets in this kernel's layout
  int bits[5];
  // prologue / epilogue arguments of the GEMV phases: qkv of layer 0
  // (embedding + norm), qkv, o, gate|up, down, lm_head (+ argmax)
  GemvArgs ga[6];
  const unsigned char* lm_w;  // packed lm_head (the embedding when tied)
  const bf16* final_norm;
  const uint32_t* emb_w;  // quantized embedding table
  const bf16* emb_s;
  const bf16* emb_b;
  int emb_bits, emb_gs, vocab;
  int* token;  // in: this step's token; out: the next one
  int H;
  float eps;
  bf16* h;       // residual stream [H]
  bf16* qkvb;    // [(nq + 2 nkv) * 128]
  bf16* attnb;   // [nq * 128]
  bf16* act;     // SwiGLU output [I]
  bf16* logits;  // [vocab]
  const float2* rope_cs;  // (cos, sin) [cap][64]
  int cap, nq, nkv;
  float scale;
  float* attn_part;  // [n_kv][max_splits][hpg][132]: m, l, pad, pad, unnormalised output
  int max_splits;
  int* pos;  // device offset; += 1 at the end of the step
  int* hist;
  int* hist_n;
  int hist_cap;
  float* am_val;  // [grid]
  int* am_idx;
  unsigned* am_ticket;
  // [0] barrier arrivals, [1] placement fallback, [2] abort, [4, 4 + nsm)
  // per-SM arrivals; all zero between steps (the last CTA resets them)
  unsigned* sync;
  int nsm, cps;  // SMs, CTAs per SM (grid = nsm * cps)
  int slot_bytes, nslots;
  int off_aux, aux_stride, off_u, off_ring;
  int* status;
};

struct StepShape {
  int H, I, nq, nkv, hd, vocab, gs, layers, cap;
  int bits[5];  // qkv, o, gate|up, down, lm_head
};

struct StepPlan {
  int grid, cps, smem, hpg;
  StepArgs tmpl;  // geometry and layout (pointers unset)
};

// Words of the `sync` block for `num_sms` SMs.
size_t step_sync_words(int num_sms);
// Plans the step for `cps` CTAs per SM within `budget` bytes of shared
// memory per CTA.  Returns 0, or -1 when the shape is not supported (the
// caller keeps the per-kernel chain).
int step_make_plan(const StepShape& sh, int num_sms, int cps, int budget, StepPlan* plan);
// Fills a.ga from the other fields (after the pointers are set).
void step_finish_args(StepArgs* a);
// CTAs of the step kernel that fit on one SM with the plan's shared memory.
int step_occupancy(const StepPlan& p);
// One decode step.  `coop` asks for a cooperative launch (co-residency
// checked by the driver).
cudaError_t step_launch(const StepArgs& a, const StepPlan& p, cudaStream_t st, bool coop);

}  // namespace emx
