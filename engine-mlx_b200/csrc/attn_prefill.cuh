// attn_prefill.cuh — causal GQA prefill attention.
#pragma once
#include "common.cuh"

namespace emx {

struct AttnPrefillArgs {
  const bf16* q;   // [nq, T, head_dim] (normed + roped)
  const bf16* kc;  // K cache [nkv, cap, head_dim]; the T prompt rows start at `offset`
  const bf16* vc;
  int cap, offset, T;
  // cached rows before the chunk that every query attends as well: keys are
  // cache rows [offset - prefix, offset + T), query t sits at key prefix + t
  // (0: the chunk attends only itself, as the reference's prefill does)
  int prefix;
  int nq, nkv, head_dim;
  float scale;
  bf16* out;       // out_tnd: [T, nq * head_dim]; else [nq, T, head_dim]
  int out_tnd;
};

// `status`: device status word for bounded-wait timeouts (may be null).
cudaError_t attn_prefill_launch(const AttnPrefillArgs& a, cudaStream_t st, int* status = nullptr);

}  // namespace emx
