// qgemm.cu — quantized matmul for M > 1 rows (prefill), MLX qmm semantics:
// y = x . bf16(dequant(W))^T with fp32 accumulation
// (mlx_quantized_matmul, crates/mlx-ffi/src/ops/real/transform.rs:77-89, as
// forward_qwen3.rs:66-162 calls it over the whole prompt).
//
// Short prompts with group size 64 (every BASELINE config): the tcgen05 GEMM
// dequantises each k-block of its weight tile into shared memory, K split
// across the CTAs of a cluster — over the packed decode layout when the
// caller has it (tc_pgemm), else over the MLX layout (tc_qgemm).  Otherwise W is
// dequantised bit-exactly into a bf16 scratch buffer (the whole matrix, up to 1 GiB) and the tcgen05
// GEMM multiplies.  Either way the residual add, SwiGLU or fp32 output is
// fused into the epilogue.
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
  TcGemmArgs t = {};
  t.x = a.x;
  t.M = a.M;
  t.N = a.epi == kGemmSwiglu ? a.N / 2 : a.N;
  t.K = a.K;
  t.epi = a.epi == kGemmStore ? kTcStore : a.epi == kGemmResid ? kTcResid : a.epi == kGemmSwiglu ? kTcSwiglu : kTcF32;
  t.y = a.y;
  t.res = a.res;
  t.yf = a.yf;
  // With the packed copy (group size 64) the GEMM dequantises inside the
  // kernel up to kPackedMaxRows rows (K split across a cluster when the row
  // tiles leave SMs idle): against a dequantisation pass into bf16 scratch +
  // tc_gemm it measured 1.2-2.5x faster per GEMM from 256 to 2048 rows on the
  // C3 shapes (gate|up at 2048 rows 131.6 -> 106.5 us; a whole 512-token
  // prefill 6.31 -> 4.52 ms), while at 4096 / 8192 rows, where every row
  // tile dequantises the same weights again, the prefill was 3% / 7% slower.
  // Without it, up to 256 rows dequantise the MLX layout inside the kernel
  // (against the scratch pass: N=6144 K=2048 at 256 rows 29.3 -> 23.0 us,
  // a tie at 512, the scratch pass ahead from 1024), longer inputs through
  // the scratch pass.
  constexpr int kPackedMaxRows = 2048;
  t.wq = a.w;
  t.ws = a.s;
  t.wb = a.b;
  t.bits = a.bits;
  if (a.wp && a.gs == 64 && a.M <= kPackedMaxRows) {
    t.wp = a.wp;
    t.S = (a.K / 64 + 7) / 8;
    t.nrb = (a.N + 15) / 16;
    if (tc_pgemm_supported(t)) {
      const cudaError_t ce = tc_pgemm_launch(t, c->num_sms, st);
      return ce == cudaSuccess ? 0 : (int)ce;
    }
  }
  if (a.gs == 64 && a.M <= 256 && tc_qgemm_supported(t)) {
    const cudaError_t ce = tc_qgemm_launch(t, c->num_sms, st);
    return ce == cudaSuccess ? 0 : (int)ce;
  }
  const size_t need = (size_t)a.N * a.K * 2;
  if (need > ((size_t)1 << 30)) return -2;  // larger than any weight of the supported configs
  int e = grow(&c->scratch, &c->scratch_bytes, need);
  if (e) return e;
  cudaError_t ce =
      k_dequantize(a.w, a.s, a.b, reinterpret_cast<bf16*>(c->scratch), a.N, a.K, a.gs, a.bits, st);
  if (ce != cudaSuccess) return (int)ce;
  t.w = reinterpret_cast<const bf16*>(c->scratch);
  if (!tc_gemm_supported(t)) return -3;
  ce = tc_gemm_launch(t, c->num_sms, st);
  return ce == cudaSuccess ? 0 : (int)ce;
}

}  // namespace emx
