// qgemv.cuh — batch-1 quantized matrix-vector product (MLX affine layout).
//
// Replaces mlx_quantized_matmul(x, w, scales, biases, transpose=true, gs, bits,
// "affine") for M == 1 (crates/mlx-ffi/src/ops/real/transform.rs:77-89) as
// the served decode step calls it for qkv, o, gate_up, down and lm_head
// (crates/serve/src/compiled.rs:133-198), and the per-expert quantized
// matmuls of moe_forward (crates/ops/src/moe.rs:140-163) as one gathered
// launch.
#pragma once
#include "common.cuh"
#include "peer.cuh"

namespace emx {

// Prologue: how the CTA builds the bf16 input vector x in shared memory.
enum GemvPro : int {
  kProX = 0,          // x read as given (x_slots vectors when x_slots > 1)
  kProNorm = 1,       // x = grouped_rms_norm(src, norm_w, eps, groups), src = a.x
  kProEmbedNorm = 2,  // src = dequant(embed row *token) (CTA 0 stores it to x_out), then norm
  kProAddNorm = 3,    // src = bf16(a.x + addend) (CTA 0 stores it to x_out), then norm;
                      //   addend = bf16(add_f32) if add_round else add_f32 (tensor-parallel
                      //   sum), or sum_s moe_w[s]*moe_y[s] in fp32 (MoE combine) when moe_y
  kProMerge = 4,      // x = the decode attention output: merged here from the splits'
                      //   partials when the attention deferred its merge (few splits;
                      //   CTA 0 stores it to x_out), else read from a.x as kProX
};

// Epilogue: what happens to each finished output row (fp32 accumulator).
enum GemvEpi : int {
  kEpiStore = 0,   // y[n] = bf16(acc)
  kEpiResid = 1,   // y[n] = bf16(res[n] + bf16(acc))   (y may alias res)
  kEpiSwiglu = 2,  // rows [0,I) gate, [I,2I) up: y[n] = silu(g)*u with MLX's bf16 steps
  kEpiArgmax = 3,  // bf16 logits (optionally stored); greedy token over all rows
  kEpiF32 = 4,     // yf[n] = acc (fp32 partial, e.g. before a tensor-parallel sum)
};

struct GemvArgs {
  const uint32_t* w;  // [N, K*bits/32] (or [E, rows_per_expert, ...] with slots)
  const bf16* s;      // [N, K/gs]
  const bf16* b;      // [N, K/gs]
  int N, K;           // physical rows (logical rows x 2 for SwiGLU) and reduction length
  int bits, gs;
  int pro, epi;
  // prologue inputs
  const bf16* x;       // kProX: x[x_slots][K]; kProNorm/kProAddNorm: source[K]
  int x_slots;         // >1: logical slot s uses x + s*K (MoE down projection)
  const bf16* norm_w;  // [K]
  float eps;
  int norm_groups;
  const uint32_t* emb_w;  // kProEmbedNorm: quantized embedding table
  const bf16* emb_s;
  const bf16* emb_b;
  int emb_bits, emb_gs, vocab;
  const int* token;  // device token id
  bf16* x_out;       // kProEmbedNorm / kProAddNorm: the new residual (must not alias x)
  const float* add_f32;
  int add_round;
  const bf16* moe_y;  // [moe_n][K]
  const float* moe_w;
  const int* moe_n;   // device count of valid slots
  // expert gather: logical rows are slots of slot_rows rows each
  const int* slot_expert;  // [slots] local expert id per slot (device) or nullptr
  const int* n_slots;      // device slot count (rows = *n_slots * slot_rows)
  int slot_rows;
  // epilogue
  bf16* y;
  const bf16* res;
  float* yf;
  float* am_val;  // argmax per-CTA partials [grid]
  int* am_idx;
  unsigned* am_ticket;
  int* tok_out;   // next token (argmax)
  int* hist;      // optional token history, hist[*hist_n] = token, (*hist_n)++
  int* hist_n;
  int hist_cap;
  int* pos;       // optional: *pos += pos_inc after the argmax
  int pos_inc;
  int* status;
  const PeerX* peer;  // kEpiF32 producer / kProAddNorm consumer of a peer-memory sum (device), or nullptr
  // kProMerge: the attention's partials [nkv][splits][hpg][head_dim + 2] (m, l,
  // unnormalised output), its position word and split grid
  const float* attn_part;
  const int* attn_pos;
  int attn_hpg, attn_grid;
};

// Host-side launch plan (computed once per weight shape).
struct GemvPlan {
  int grid;         // CTAs
  int lrows;        // logical rows (N, or N/2 for SwiGLU) — the maximum with slots
  int rows_round;   // logical rows per round (multiple of 16)
  int spans_round;  // spans per round (k-range)
  int nbuf;         // ring depth
  int smem;         // dynamic shared memory bytes
  int x_slots;
};

// Returns 0 and fills `plan`, or -1 when the shape is unsupported.
// N = physical rows of one launch's logical range (for SwiGLU 2x the logical rows).
int gemv_make_plan(int N, int K, int bits, int gs, int epi, int x_slots, int num_sms, GemvPlan* plan);
// Launches one GEMV; `pdl` adds the programmatic-dependent-launch attribute.
cudaError_t gemv_launch(const GemvArgs& a, const GemvPlan& p, cudaStream_t st, bool pdl);

}  // namespace emx
