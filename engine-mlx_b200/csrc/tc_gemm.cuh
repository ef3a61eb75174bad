// tc_gemm.cuh — bf16 x bf16 -> fp32 GEMM on the 5th-generation tensor cores
// (tcgen05.mma with the accumulator in tensor memory), operands fed by TMA.
//
//   y[M, N] = x[M, K] . W[N, K]^T        (both operands K-major, bf16)
//
// Used by the prefill quantized matmul (qgemm.cu) on the dequantised weight.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace emx {

enum TcEpi : int {
  kTcStore = 0,   // y = bf16(acc)
  kTcResid = 1,   // y = bf16(res + bf16(acc))            (y may alias res)
  kTcSwiglu = 2,  // W rows [0,I) gate, [I,2I) up: y[m, n<I] = silu(g) * u, MLX rounding steps
  kTcF32 = 3,     // yf = acc
};

struct TcGemmArgs {
  const bf16* x;    // [M, K]
  const bf16* w;    // [N_w, K] (N_w = 2*N for SwiGLU)
  int M, N, K;      // N: output columns
  int epi;
  bf16* y;          // [M, N]
  const bf16* res;  // [M, N]
  float* yf;        // [M, N]
  int* status;
};

// True when the shape is supported (K % 64 == 0, N % 32 == 0, 16-byte
// aligned operands).
bool tc_gemm_supported(const TcGemmArgs& a);
// Enqueues the GEMM; returns cudaSuccess or the launch / encode error.
cudaError_t tc_gemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st);

}  // namespace emx
