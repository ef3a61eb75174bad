// pgemv.cuh — batch-1 quantized GEMV over the engine's packed weight layout.
//
// Same contract as qgemv (GemvArgs: prologues, epilogues, expert gather),
// but the weights are the MLX affine tensors re-laid out once at load time
// into tiles in MMA fragment order, so that the decode hot loop does no
// address arithmetic, no register shuffling and no bank-conflicted reads.
//
// Packed layout of one weight matrix (bits 4 or 8, group size gs):
//   span      = 8 groups = 8*gs columns; S = ceil(K / (8 gs)) spans; each
//               span is two half-spans of 4 groups
//   tile      = 16 rows x 1 span: A-part then a 512-byte scale/bias part
//   A-part    = [half-span][quad q < gs/16][word set < bits/4][lane][4 words]
//               lane (g = lane/4, t = lane%4), slice j = 4q + w of the
//               half-span holds, for rows g and g+8 and group 4*hs + t,
//               the codes at group offsets 4j..4j+3 — exactly the four
//               bf16x2 A registers of one m16n8k16 MMA once a LOP3 turns
//               them into bf16 (k slots 2t, 2t+1, 2t+8, 2t+9 = group t)
//   sb-part   = [half-span][g][t < 2][s(g,G) s(g,G+1) s(g+8,G) s(g+8,G+1)
//               b(same order)], G = 4*hs + 2t
//   tiles     = [row block][span]; a row block is 16 rows of the source
//               chosen by the row map below (SwiGLU interleaves the gate and
//               up blocks of each 16 logical rows; experts are blocked).
// Rows past N and groups past K/gs are zero (their outputs are never stored).
#pragma once
#include "qgemv.cuh"

namespace emx {

// Where packed row block p comes from: `blocks` source blocks (experts) of R
// rows each; a block's rows split into `halves` halves (2 = SwiGLU gate|up);
// packed order inside a block is [16-row logical block][half].
struct PackMap {
  int blocks;  // experts (1 for a dense matrix)
  int R;       // source rows per block (N for a dense matrix)
  int halves;  // 1, or 2 for a fused gate|up matrix
};

// Bytes of one packed tile / of the packed matrix.
size_t pgemv_tile_bytes(int bits, int gs);
size_t pgemv_packed_bytes(int N, int K, int bits, int gs, const PackMap& map);

// Re-lays out an MLX affine tensor (w [N][K*bits/32], s/b [N][K/gs]) into
// the packed layout (N = blocks * R rows).
cudaError_t pgemv_pack(const uint32_t* w, const bf16* s, const bf16* b, int N, int K, int bits, int gs,
                       const PackMap& map, unsigned char* dst, cudaStream_t st);

struct PgemvPlan {
  int grid;        // CTAs
  int lb_total;    // logical 16-row blocks of one launch (maximum, for gathers)
  int halves;
  int stage_tiles; // tiles per pipeline stage
  int nbuf;        // stage buffers in shared memory
  int smem;        // dynamic shared memory bytes
  int x_slots;
  int lbs_max;     // logical blocks of the busiest CTA
  int norm;        // room for the norm weights (the norm prologues need it)
};

// N = physical rows of one launch (2x logical rows for SwiGLU); `budget` is
// the dynamic shared memory the plan may use; `ctas_per_sm` > 1 spreads a
// streamed matrix over more CTAs (more warps hiding the dequant latency).
// Returns 0 or -1 (unsupported).
// `norm` = 0: the launches use no norm prologue, so no room is kept for
// the norm weights (more for the stage ring).
int pgemv_make_plan(int N, int K, int bits, int gs, int epi, int x_slots, int num_sms, int budget, PgemvPlan* plan,
                    int ctas_per_sm = 1, int norm = 1);

// One GEMV; a.w must point at the packed matrix (a.s / a.b unused).
cudaError_t pgemv_launch(const GemvArgs& a, const PgemvPlan& p, cudaStream_t st, bool pdl);

}  // namespace emx
