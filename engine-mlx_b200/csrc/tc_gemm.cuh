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
  // tc_qgemm: the weights as MLX affine codes, group size 64
  const uint32_t* wq;  // [N_w, K*bits/32]
  const bf16* ws;      // [N_w, K/64] scales
  const bf16* wb;      // [N_w, K/64] biases
  int bits;            // 4 or 8
  // tc_pgemm: the weights in the packed decode-GEMV layout (group size 64)
  const unsigned char* wp;  // packed tiles [row block][span]
  int S;                    // spans (8 groups each) per row block
  int nrb;                  // packed 16-row blocks (SwiGLU: gate and up blocks alternate)
  // grouped (MoE) mode: CTA x takes tiles[x] = (expert, first row, end row)
  // of x when x < *n_tiles (others exit); the expert's packed block starts
  // expert * expert_stride bytes into wp; nrb counts one expert's row blocks
  const int4* tiles;
  const int* n_tiles;
  size_t expert_stride;
};

// True when the shape is supported (K % 64 == 0, N % 32 == 0, 16-byte
// aligned operands).
bool tc_gemm_supported(const TcGemmArgs& a);
// Enqueues the GEMM; returns cudaSuccess or the launch / encode error.
cudaError_t tc_gemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st);

// The same GEMM with W given as MLX affine codes (group size 64): the kernel
// dequantises each k-block of its weight tile into shared memory, bit-exactly
// as the dequant pass would, so no bf16 copy of W is written.
bool tc_qgemm_supported(const TcGemmArgs& a);
// When the output has fewer tiles than SMs, K is split across the CTAs of a
// thread-block cluster and the partials are summed (in split order) inside
// the cluster; one launch either way.
cudaError_t tc_qgemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st);

// The same GEMM over the packed decode-GEMV layout (wp, S, nrb): the prefill
// reads the bytes the decode step reads.  SwiGLU output column n of logical
// block n / 16 pairs gate row block 2 (n / 16) with up row block 2 (n / 16) + 1.
bool tc_pgemm_supported(const TcGemmArgs& a);
cudaError_t tc_pgemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st);
// Grouped mode (tiles / n_tiles / expert_stride set): one launch over up to
// max_tiles row tiles of 128 rows, each against its own expert's weights.
cudaError_t tc_pgemm_grouped_launch(const TcGemmArgs& a, int max_tiles, cudaStream_t st);

}  // namespace emx
