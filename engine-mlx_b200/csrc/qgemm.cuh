// qgemm.cuh — quantized matmul for M > 1 rows (prefill).
#pragma once
#include "common.cuh"

namespace emx {

enum GemmEpi : int {
  kGemmStore = 0,   // y[m, n] = bf16(acc)
  kGemmResid = 1,   // y[m, n] = bf16(res[m, n] + bf16(acc))
  kGemmSwiglu = 2,  // weight rows [0,I) gate, [I,2I) up; y[m, n] (n < I) = silu(g) * u
  kGemmF32 = 3,     // yf[m, n] = acc (fp32, e.g. a tensor-parallel partial)
};

struct GemmArgs {
  const bf16* x;  // [M, K]
  const uint32_t* w;
  const bf16* s;
  const bf16* b;
  int M, N, K, bits, gs;
  int epi;
  bf16* y;         // [M, N] (or [M, N/2] for SwiGLU)
  const bf16* res; // [M, N] for kGemmResid (may alias y)
  float* yf;       // [M, N] for kGemmF32
  // optional: the same weights in the packed decode-GEMV layout (a dense
  // matrix; gate|up interleaved per 16 rows for SwiGLU); read instead of w/s/b
  const unsigned char* wp;
};

struct GemmCtx;  // per-context scratch + library handles
GemmCtx* gemm_ctx_create(size_t scratch_bytes);
void gemm_ctx_destroy(GemmCtx* c);
// Returns 0 on success, a CUDA error code (or a negative shape error) otherwise.
int gemm_run(GemmCtx* c, const GemmArgs& a, cudaStream_t st);

}  // namespace emx
