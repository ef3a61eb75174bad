// qgemm.cu — quantized matmul for M > 1 rows (prefill), MLX qmm semantics:
// y = x . bf16(dequant(W))^T with fp32 accumulation
// (mlx_quantized_matmul, crates/mlx-ffi/src/ops/real/transform.rs:127-138, as
// forward_qwen3.rs:66-162 calls it over the whole prompt).
//
// This version dequantizes W (bit-exactly, in bounded column chunks) into a
// scratch buffer and runs a plain cuBLAS bf16 GEMM with fp32 accumulation; the
// residual and SwiGLU epilogues are separate elementwise kernels with MLX's
// rounding steps.
#include "qgemm.cuh"

#include <cublas_v2.h>

#include <algorithm>

#include "misc.cuh"

namespace emx {

struct GemmCtx {
  cublasHandle_t h = nullptr;
  void* scratch = nullptr;  // dequantized weight chunk
  size_t scratch_bytes = 0;
  bf16* tmp = nullptr;      // [M, N] accumulator output for fused epilogues
  size_t tmp_bytes = 0;
};

namespace {

__global__ void swiglu_rows_kernel(const bf16* gu, bf16* out, int M, int I) {
  const size_t total = (size_t)M * I;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / I), n = (int)(i % I);
    const float gv = bf2f(gu[(size_t)m * 2 * I + n]);
    const float uv = bf2f(gu[(size_t)m * 2 * I + I + n]);
    const float sg = bfround(sigmoid_f(gv));
    const float sv = bfround(__fmul_rn(gv, sg));
    out[i] = f2bf(__fmul_rn(sv, uv));
  }
}

int grow(void** p, size_t* have, size_t need) {
  if (*have >= need) return 0;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  cudaError_t e = cudaMalloc(p, need);
  if (e != cudaSuccess) return (int)e;
  *have = need;
  return 0;
}

}  // namespace

GemmCtx* gemm_ctx_create(size_t scratch_bytes) {
  GemmCtx* c = new GemmCtx();
  if (cublasCreate(&c->h) != CUBLAS_STATUS_SUCCESS) {
    delete c;
    return nullptr;
  }
  cublasSetMathMode(c->h, CUBLAS_DEFAULT_MATH);
  if (scratch_bytes && grow(&c->scratch, &c->scratch_bytes, scratch_bytes)) {
    cublasDestroy(c->h);
    delete c;
    return nullptr;
  }
  return c;
}

void gemm_ctx_destroy(GemmCtx* c) {
  if (!c) return;
  if (c->scratch) cudaFree(c->scratch);
  if (c->tmp) cudaFree(c->tmp);
  if (c->h) cublasDestroy(c->h);
  delete c;
}

int gemm_run(GemmCtx* c, const GemmArgs& a, cudaStream_t st) {
  if (a.M <= 0) return 0;
  if (cublasSetStream(c->h, st) != CUBLAS_STATUS_SUCCESS) return -1;
  const bool epi_tmp = a.epi == kGemmResid || a.epi == kGemmSwiglu;
  const bool f32out = a.epi == kGemmF32;
  bf16* dst = a.y;
  if (epi_tmp) {
    int e = grow(reinterpret_cast<void**>(&c->tmp), &c->tmp_bytes, (size_t)a.M * a.N * 2);
    if (e) return e;
    dst = c->tmp;
  }
  // rows of W per chunk so that the dequantized chunk fits the scratch (the
  // whole matrix up to 1 GiB, so a prefill GEMM is one library call)
  size_t row_bytes = (size_t)a.K * 2;
  const size_t want = std::min((size_t)a.N * row_bytes, (size_t)1 << 30);
  if (c->scratch_bytes < want) {
    int e = grow(&c->scratch, &c->scratch_bytes, want);
    if (e) return e;
  }
  int rows = (int)std::min<size_t>((size_t)a.N, c->scratch_bytes / row_bytes);
  rows = rows / 16 * 16;
  if (rows <= 0) return -1;
  const int per = 32 / a.bits, ng = a.K / a.gs;
  const float alpha = 1.0f, beta = 0.0f;
  for (int n0 = 0; n0 < a.N; n0 += rows) {
    const int nr = std::min(rows, a.N - n0);
    cudaError_t ce = k_dequantize(a.w + (size_t)n0 * (a.K / per), a.s + (size_t)n0 * ng, a.b + (size_t)n0 * ng,
                                  reinterpret_cast<bf16*>(c->scratch), nr, a.K, a.gs, a.bits, st);
    if (ce != cudaSuccess) return (int)ce;
    // column-major view: C^T[N, M] = W[N, K] . X^T[K, M]
    void* cptr = f32out ? static_cast<void*>(a.yf + n0) : static_cast<void*>(dst + n0);
    cublasStatus_t cs = cublasGemmEx(c->h, CUBLAS_OP_T, CUBLAS_OP_N, nr, a.M, a.K, &alpha, c->scratch, CUDA_R_16BF,
                                     a.K, a.x, CUDA_R_16BF, a.K, &beta, cptr, f32out ? CUDA_R_32F : CUDA_R_16BF,
                                     a.N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    if (cs != CUBLAS_STATUS_SUCCESS) return 1000 + (int)cs;
  }
  if (a.epi == kGemmResid) {
    cudaError_t ce = k_add(a.res, dst, a.y, (size_t)a.M * a.N, st);
    if (ce != cudaSuccess) return (int)ce;
  } else if (a.epi == kGemmSwiglu) {
    const int I = a.N / 2;
    const size_t total = (size_t)a.M * I;
    int blocks = (int)std::min<size_t>((total + 255) / 256, 1u << 20);
    swiglu_rows_kernel<<<blocks, 256, 0, st>>>(dst, a.y, a.M, I);
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) return (int)ce;
  }
  return 0;
}

}  // namespace emx
