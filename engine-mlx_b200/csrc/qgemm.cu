// qgemm.cu — quantized matmul for M > 1 rows (prefill), MLX qmm semantics:
// y = x . bf16(dequant(W))^T with fp32 accumulation
// (mlx_quantized_matmul, crates/mlx-ffi/src/ops/real/transform.rs:127-138, as
// forward_qwen3.rs:66-162 calls it over the whole prompt).
//
// W is dequantised bit-exactly into a bf16 scratch buffer (the whole matrix,
// up to 1 GiB), then the tcgen05 tensor-core GEMM (tc_gemm.cu) multiplies,
// with the residual add, SwiGLU or fp32 output fused into its epilogue.
#include "qgemm.cuh"

#include "misc.cuh"
#include "tc_gemm.cuh"

namespace emx {

struct GemmCtx {
  void* scratch = nullptr;  // dequantized weight
  size_t scratch_bytes = 0;
  int num_sms = 148;
};

namespace {

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
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (scratch_bytes && grow(&c->scratch, &c->scratch_bytes, scratch_bytes)) {
    delete c;
    return nullptr;
  }
  return c;
}

void gemm_ctx_destroy(GemmCtx* c) {
  if (!c) return;
  if (c->scratch) cudaFree(c->scratch);
  delete c;
}

int gemm_run(GemmCtx* c, const GemmArgs& a, cudaStream_t st) {
  if (a.M <= 0) return 0;
  const size_t need = (size_t)a.N * a.K * 2;
  if (need > ((size_t)1 << 30)) return -2;  // larger than any weight of the supported configs
  int e = grow(&c->scratch, &c->scratch_bytes, need);
  if (e) return e;
  cudaError_t ce =
      k_dequantize(a.w, a.s, a.b, reinterpret_cast<bf16*>(c->scratch), a.N, a.K, a.gs, a.bits, st);
  if (ce != cudaSuccess) return (int)ce;
  TcGemmArgs t = {};
  t.x = a.x;
  t.w = reinterpret_cast<const bf16*>(c->scratch);
  t.M = a.M;
  t.N = a.epi == kGemmSwiglu ? a.N / 2 : a.N;
  t.K = a.K;
  t.epi = a.epi == kGemmStore ? kTcStore : a.epi == kGemmResid ? kTcResid : a.epi == kGemmSwiglu ? kTcSwiglu : kTcF32;
  t.y = a.y;
  t.res = a.res;
  t.yf = a.yf;
  if (!tc_gemm_supported(t)) return -3;
  ce = tc_gemm_launch(t, c->num_sms, st);
  return ce == cudaSuccess ? 0 : (int)ce;
}

}  // namespace emx
