// attn_decode.cuh — batch-1 decode attention (flash-decode, split KV).
#pragma once
#include "common.cuh"

namespace emx {

struct AttnDecodeArgs {
  const bf16* qkv;        // fused projection output [ (nq + 2*nkv) * head_dim ], q | k | v
  const bf16* q_norm;     // [head_dim] or nullptr
  const bf16* k_norm;     // [head_dim] or nullptr
  float eps;
  const float* inv_freq;  // rope inverse frequencies [head_dim/2]
  const float2* rope_cs;  // optional (cos, sin) table [cap][head_dim/2] of the same angles
  bf16* kc;               // this layer's K cache [nkv, cap, head_dim]
  bf16* vc;               // this layer's V cache
  int cap;
  int nq, nkv, head_dim;
  const int* pos;         // device-held offset: row of the new token (nullptr: pos_host)
  int pos_host;
  const bf16* q_in;       // non-null: final q heads [nq, head_dim] (no norm/rope, no cache write)
  float scale;
  bf16* out;              // attention output [nq * head_dim]
  float* part;            // split partials [nkv][splits][nq/nkv][head_dim + 2]
  unsigned* ticket;       // [nkv], zero between launches
  int splits;
  int* status;
  // nonzero: when at most kAttnDeferSplits splits are active, every split
  // stores its partial and returns; the consumer (the o-projection GEMV's
  // kProMerge prologue) merges them with the same arithmetic
  int defer_merge;
};

// Fewest cache rows a split is given, and the splits that take part for L
// rows on a grid of `grid` splits (the producer and a deferred merge agree).
constexpr int kAttnMinRows = 64;
constexpr int kAttnDeferSplits = 4;
__host__ __device__ __forceinline__ int attn_active_splits(int L, int grid) {
  const int s = (L + kAttnMinRows - 1) / kAttnMinRows;
  return s < grid ? s : grid;
}

// Split grid size for n_kv KV heads with hpg q heads each.
int attn_decode_splits(int nkv, int num_sms, int hpg);
// (cos, sin) of pos * inv_freq[i] for pos < cap, i < head_dim/2, with the
// exact fp32 steps the decode kernel would take.
cudaError_t rope_table_fill(float2* cs, const float* inv_freq, int cap, int half, cudaStream_t st);
cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st, bool pdl);

}  // namespace emx
