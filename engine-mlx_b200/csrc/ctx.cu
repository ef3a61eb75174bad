// ctx.cu — C ABI: context, errors, memory and the op-level entry points that
// stand in for the MlxCtx methods the Qwen3 path calls
// (crates/mlx-ffi/src/ops/real/*.rs).  Every op validates its shape, enqueues
// its kernel on the context stream and returns a status; none has a host
// fallback.
#include "ctx.cuh"
#include "pgemv.cuh"

#include <cstdio>
#include <cstring>
#include <vector>

#include "attn_decode.cuh"
#include "attn_prefill.cuh"
#include "misc.cuh"
#include "qgemm.cuh"
#include "tc_gemm.cuh"
#include "qgemv.cuh"

namespace {

thread_local std::string g_last_error;
emx_error_handler g_handler = nullptr;
void* g_handler_data = nullptr;
std::mutex g_handler_mu;

}  // namespace

namespace emx {

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  emx_error_handler h;
  void* d;
  {
    std::lock_guard<std::mutex> lk(g_handler_mu);
    h = g_handler;
    d = g_handler_data;
  }
  if (h) h(buf, d);
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear a sticky launch error so the context stays usable
  return fail(EMX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int ctx_alloc(emx_ctx* c, size_t bytes, void** p) {
  {
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->active + bytes > c->limit) return fail(EMX_ERR_OOM, "allocation of %zu bytes exceeds the memory limit", bytes);
  }
  if (cudaSetDevice(c->device) != cudaSuccess) return fail(EMX_ERR_CUDA, "cudaSetDevice failed");
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes ? bytes : 1);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(EMX_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> lk(c->mu);
  c->allocs[ptr] = bytes;
  c->active += bytes;
  if (c->active > c->peak) c->peak = c->active;
  *p = ptr;
  return EMX_OK;
}

void ctx_free(emx_ctx* c, void* p) {
  if (!p) return;
  {
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->allocs.find(p);
    if (it == c->allocs.end()) return;
    c->active -= it->second;
    c->allocs.erase(it);
  }
  cudaFree(p);
}

int ctx_scratch(emx_ctx* c, size_t bytes, void** p) {
  if (c->scratch_bytes < bytes) {
    if (c->scratch) {
      cudaStreamSynchronize(c->stream);
      ctx_free(c, c->scratch);
      c->scratch = nullptr;
      c->scratch_bytes = 0;
    }
    int rc = ctx_alloc(c, bytes, &c->scratch);
    if (rc) return rc;
    EMX_CHECK_CUDA(cudaMemsetAsync(c->scratch, 0, bytes, c->stream), "scratch memset");
    c->scratch_bytes = bytes;
  }
  *p = c->scratch;
  return EMX_OK;
}

int ctx_sync_check(emx_ctx* c, const char* what) {
  EMX_CHECK_CUDA(cudaStreamSynchronize(c->stream), what);
  int st = 0;
  EMX_CHECK_CUDA(cudaMemcpy(&st, c->status, sizeof(int), cudaMemcpyDeviceToHost), "status read");
  if (st != 0) {
    static const char* names[] = {"ok", "shared-memory barrier wait timed out", "peer flag wait timed out",
                                  "token id out of range", "KV capacity exceeded"};
    const char* nm = (st > 0 && st < 5) ? names[st] : "unknown";
    return fail(EMX_ERR_DEVICE, "%s: device status %d (%s)", what, st, nm);
  }
  return EMX_OK;
}

}  // namespace emx

using namespace emx;

#define EMX_REQUIRE(cond, ...) \
  do {                         \
    if (!(cond)) return fail(EMX_ERR_INVALID, __VA_ARGS__); \
  } while (0)

extern "C" {

void emx_set_error_handler(emx_error_handler handler, void* data) {
  std::lock_guard<std::mutex> lk(g_handler_mu);
  g_handler = handler;
  g_handler_data = data;
}

const char* emx_last_error(void) { return g_last_error.c_str(); }

const char* emx_version(void) { return "emx 0.1 (sm_100a)"; }

int emx_ctx_create(int device, emx_ctx** out) {
  EMX_REQUIRE(out, "emx_ctx_create: out is null");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(EMX_ERR_CUDA, "emx_ctx_create: no CUDA device (%s)", cudaGetErrorString(e));
  }
  EMX_REQUIRE(device >= 0 && device < n, "emx_ctx_create: device %d out of range [0,%d)", device, n);
  cudaDeviceProp prop;
  EMX_CHECK_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10) return fail(EMX_ERR_CUDA, "emx_ctx_create: device %d is sm_%d%d; libemx is built for sm_100a",
                                    device, prop.major, prop.minor);
  EMX_CHECK_CUDA(cudaSetDevice(device), "cudaSetDevice");
  emx_ctx* c = new emx_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  cudaError_t ce = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) {
    delete c;
    return fail_cuda(ce, "cudaStreamCreate");
  }
  void* st = nullptr;
  int rc = ctx_alloc(c, sizeof(int) * 4, &st);
  if (rc) {
    cudaStreamDestroy(c->stream);
    delete c;
    return rc;
  }
  c->status = static_cast<int*>(st);
  cudaMemset(c->status, 0, sizeof(int) * 4);
  c->gemm = gemm_ctx_create(0);
  if (!c->gemm) {
    ctx_free(c, c->status);
    cudaStreamDestroy(c->stream);
    delete c;
    return fail(EMX_ERR_CUDA, "emx_ctx_create: cuBLAS handle creation failed");
  }
  *out = c;
  return EMX_OK;
}

int emx_ctx_destroy(emx_ctx* c) {
  if (!c) return EMX_OK;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  gemm_ctx_destroy(c->gemm);
  std::vector<void*> left;
  for (auto& kv : c->allocs) left.push_back(kv.first);
  for (void* p : left) ctx_free(c, p);
  cudaStreamDestroy(c->stream);
  delete c;
  return EMX_OK;
}

int emx_ctx_stream(emx_ctx* c, void** s) {
  EMX_REQUIRE(c && s, "emx_ctx_stream: null argument");
  *s = c->stream;
  return EMX_OK;
}

int emx_ctx_num_sms(emx_ctx* c, int* n) {
  EMX_REQUIRE(c && n, "emx_ctx_num_sms: null argument");
  *n = c->num_sms;
  return EMX_OK;
}

int emx_synchronize(emx_ctx* c) {
  EMX_REQUIRE(c, "emx_synchronize: null context");
  return ctx_sync_check(c, "emx_synchronize");
}

int emx_device_status(emx_ctx* c, int* status, int clear) {
  EMX_REQUIRE(c && status, "emx_device_status: null argument");
  EMX_CHECK_CUDA(cudaStreamSynchronize(c->stream), "emx_device_status");
  EMX_CHECK_CUDA(cudaMemcpy(status, c->status, sizeof(int), cudaMemcpyDeviceToHost), "status read");
  if (clear) EMX_CHECK_CUDA(cudaMemset(c->status, 0, sizeof(int)), "status clear");
  return EMX_OK;
}

int emx_malloc(emx_ctx* c, size_t bytes, void** p) {
  EMX_REQUIRE(c && p, "emx_malloc: null argument");
  return ctx_alloc(c, bytes, p);
}

int emx_free(emx_ctx* c, void* p) {
  EMX_REQUIRE(c, "emx_free: null context");
  cudaStreamSynchronize(c->stream);
  ctx_free(c, p);
  return EMX_OK;
}

int emx_memcpy_h2d(emx_ctx* c, void* dst, const void* src, size_t bytes) {
  EMX_REQUIRE(c && (bytes == 0 || (dst && src)), "emx_memcpy_h2d: null argument");
  EMX_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream), "emx_memcpy_h2d");
  return EMX_OK;
}

int emx_memcpy_d2h(emx_ctx* c, void* dst, const void* src, size_t bytes) {
  EMX_REQUIRE(c && (bytes == 0 || (dst && src)), "emx_memcpy_d2h: null argument");
  EMX_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream), "emx_memcpy_d2h");
  return ctx_sync_check(c, "emx_memcpy_d2h");
}

int emx_memset(emx_ctx* c, void* dst, int value, size_t bytes) {
  EMX_REQUIRE(c && (bytes == 0 || dst), "emx_memset: null argument");
  EMX_CHECK_CUDA(cudaMemsetAsync(dst, value, bytes, c->stream), "emx_memset");
  return EMX_OK;
}

int emx_get_active_memory(emx_ctx* c, size_t* b) {
  EMX_REQUIRE(c && b, "emx_get_active_memory: null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  *b = c->active;
  return EMX_OK;
}

int emx_get_peak_memory(emx_ctx* c, size_t* b) {
  EMX_REQUIRE(c && b, "emx_get_peak_memory: null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  *b = c->peak;
  return EMX_OK;
}

int emx_set_memory_limit(emx_ctx* c, size_t limit, size_t* prev) {
  EMX_REQUIRE(c, "emx_set_memory_limit: null context");
  std::lock_guard<std::mutex> lk(c->mu);
  if (prev) *prev = c->limit;
  c->limit = limit;
  return EMX_OK;
}

// ------------------------------------------------------------------- ops

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_quant(int N, int K, int gs, int bits, const char* op) {
  if (!(bits == 4 || bits == 8)) return fail(EMX_ERR_INVALID, "%s: bits=%d unsupported (4 or 8)", op, bits);
  if (!(gs == 32 || gs == 64 || gs == 128))
    return fail(EMX_ERR_INVALID, "%s: group_size=%d unsupported (32, 64 or 128)", op, gs);
  if (N <= 0 || K <= 0 || K % gs != 0)
    return fail(EMX_ERR_INVALID, "%s: K=%d must be a positive multiple of group_size=%d", op, K, gs);
  return EMX_OK;
}

int emx_quantized_matmul(emx_ctx* c, const void* x, const void* w, const void* s, const void* b, void* y, int M,
                         int N, int K, int transpose, int gs, int bits) {
  EMX_REQUIRE(c && x && w && s && b && y, "emx_quantized_matmul: null argument");
  EMX_REQUIRE(transpose == 1, "emx_quantized_matmul: only transpose=true (the reference's only use) is supported");
  int rc = check_quant(N, K, gs, bits, "emx_quantized_matmul");
  if (rc) return rc;
  EMX_REQUIRE(M >= 0, "emx_quantized_matmul: M=%d", M);
  if (M == 0) return EMX_OK;
  if (M == 1) {
    EMX_REQUIRE(N % 16 == 0, "emx_quantized_matmul: N=%d must be a multiple of 16", N);
    EMX_REQUIRE(aligned16(w) && aligned16(s) && aligned16(b), "emx_quantized_matmul: w/scales/biases must be 16-byte aligned");
    GemvPlan plan;
    if (gemv_make_plan(N, K, bits, gs, kEpiStore, 1, c->num_sms, &plan))
      return fail(EMX_ERR_INVALID, "emx_quantized_matmul: unsupported GEMV shape N=%d K=%d", N, K);
    GemvArgs a = {};
    a.w = static_cast<const uint32_t*>(w);
    a.s = static_cast<const bf16*>(s);
    a.b = static_cast<const bf16*>(b);
    a.N = N;
    a.K = K;
    a.bits = bits;
    a.gs = gs;
    a.pro = kProX;
    a.epi = kEpiStore;
    a.x = static_cast<const bf16*>(x);
    a.x_slots = 1;
    a.y = static_cast<bf16*>(y);
    a.status = c->status;
    EMX_CHECK_CUDA(gemv_launch(a, plan, c->stream, false), "emx_quantized_matmul (gemv)");
    return EMX_OK;
  }
  GemmArgs g = {};
  g.x = static_cast<const bf16*>(x);
  g.w = static_cast<const uint32_t*>(w);
  g.s = static_cast<const bf16*>(s);
  g.b = static_cast<const bf16*>(b);
  g.M = M;
  g.N = N;
  g.K = K;
  g.bits = bits;
  g.gs = gs;
  g.epi = kGemmStore;
  g.y = static_cast<bf16*>(y);
  rc = gemm_run(c->gemm, g, c->stream);
  if (rc) return fail(EMX_ERR_CUDA, "emx_quantized_matmul (gemm): error %d", rc);
  return EMX_OK;
}

int emx_qpack_bytes(int N, int K, int gs, int bits, size_t* bytes) {
  EMX_REQUIRE(bytes, "emx_qpack_bytes: null argument");
  int rc = check_quant(N, K, gs, bits, "emx_qpack_bytes");
  if (rc) return rc;
  EMX_REQUIRE(N % 16 == 0, "emx_qpack_bytes: N=%d must be a multiple of 16", N);
  *bytes = pgemv_packed_bytes(N, K, bits, gs, PackMap{1, N, 1});
  return EMX_OK;
}

int emx_qpack(emx_ctx* c, const void* w, const void* s, const void* b, void* out, int N, int K, int gs, int bits) {
  EMX_REQUIRE(c && w && s && b && out, "emx_qpack: null argument");
  int rc = check_quant(N, K, gs, bits, "emx_qpack");
  if (rc) return rc;
  EMX_REQUIRE(N % 16 == 0, "emx_qpack: N=%d must be a multiple of 16", N);
  EMX_CHECK_CUDA(pgemv_pack(static_cast<const uint32_t*>(w), static_cast<const bf16*>(s), static_cast<const bf16*>(b),
                            N, K, bits, gs, PackMap{1, N, 1}, static_cast<unsigned char*>(out), c->stream),
                 "emx_qpack");
  return EMX_OK;
}

int emx_quantized_matvec_packed(emx_ctx* c, const void* x, const void* packed, void* y, int N, int K, int gs,
                                int bits) {
  EMX_REQUIRE(c && x && packed && y, "emx_quantized_matvec_packed: null argument");
  int rc = check_quant(N, K, gs, bits, "emx_quantized_matvec_packed");
  if (rc) return rc;
  EMX_REQUIRE(N % 16 == 0, "emx_quantized_matvec_packed: N=%d must be a multiple of 16", N);
  EMX_REQUIRE(aligned16(packed) && aligned16(x), "emx_quantized_matvec_packed: x / packed must be 16-byte aligned");
  PgemvPlan plan;
  if (pgemv_make_plan(N, K, bits, gs, kEpiStore, 1, c->num_sms, 110 * 1024, &plan))
    return fail(EMX_ERR_INVALID, "emx_quantized_matvec_packed: unsupported shape N=%d K=%d", N, K);
  GemvArgs a = {};
  a.w = static_cast<const uint32_t*>(packed);
  a.N = N;
  a.K = K;
  a.bits = bits;
  a.gs = gs;
  a.pro = kProX;
  a.epi = kEpiStore;
  a.x = static_cast<const bf16*>(x);
  a.x_slots = 1;
  a.y = static_cast<bf16*>(y);
  a.status = c->status;
  EMX_CHECK_CUDA(pgemv_launch(a, plan, c->stream, false), "emx_quantized_matvec_packed");
  return EMX_OK;
}

int emx_quantized_matmul_packed(emx_ctx* c, const void* x, const void* packed, void* y, int M, int N, int K, int gs,
                                int bits) {
  EMX_REQUIRE(c && x && packed && y, "emx_quantized_matmul_packed: null argument");
  EMX_REQUIRE(M >= 1, "emx_quantized_matmul_packed: M=%d must be >= 1", M);
  if (M == 1) return emx_quantized_matvec_packed(c, x, packed, y, N, K, gs, bits);
  int rc = check_quant(N, K, gs, bits, "emx_quantized_matmul_packed");
  if (rc) return rc;
  EMX_REQUIRE(gs == 64, "emx_quantized_matmul_packed: M > 1 needs group size 64 (got %d)", gs);
  EMX_REQUIRE(N % 16 == 0, "emx_quantized_matmul_packed: N=%d must be a multiple of 16", N);
  EMX_REQUIRE(aligned16(packed) && aligned16(x), "emx_quantized_matmul_packed: x / packed must be 16-byte aligned");
  TcGemmArgs t = {};
  t.x = static_cast<const bf16*>(x);
  t.M = M;
  t.N = N;
  t.K = K;
  t.epi = kTcStore;
  t.y = static_cast<bf16*>(y);
  t.status = c->status;
  t.bits = bits;
  t.wp = static_cast<const unsigned char*>(packed);
  t.S = (K / 64 + 7) / 8;
  t.nrb = N / 16;
  EMX_REQUIRE(tc_pgemm_supported(t), "emx_quantized_matmul_packed: unsupported shape M=%d N=%d K=%d", M, N, K);
  EMX_CHECK_CUDA(tc_pgemm_launch(t, c->num_sms, c->stream), "emx_quantized_matmul_packed");
  return EMX_OK;
}

int emx_dequantize(emx_ctx* c, const void* w, const void* s, const void* b, void* out, int N, int K, int gs,
                   int bits) {
  EMX_REQUIRE(c && w && s && b && out, "emx_dequantize: null argument");
  int rc = check_quant(N, K, gs, bits, "emx_dequantize");
  if (rc) return rc;
  EMX_CHECK_CUDA(k_dequantize(static_cast<const uint32_t*>(w), static_cast<const bf16*>(s),
                              static_cast<const bf16*>(b), static_cast<bf16*>(out), N, K, gs, bits, c->stream),
                 "emx_dequantize");
  return EMX_OK;
}

int emx_quantize(emx_ctx* c, const void* src, emx_dtype dt, void* w, void* s, void* b, int N, int K, int gs,
                 int bits) {
  EMX_REQUIRE(c && src && w && s && b, "emx_quantize: null argument");
  EMX_REQUIRE(dt == EMX_F32 || dt == EMX_BF16, "emx_quantize: source must be f32 or bf16");
  int rc = check_quant(N, K, gs, bits, "emx_quantize");
  if (rc) return rc;
  EMX_CHECK_CUDA(k_quantize(dt == EMX_F32 ? static_cast<const float*>(src) : nullptr,
                            dt == EMX_BF16 ? static_cast<const bf16*>(src) : nullptr, static_cast<uint32_t*>(w),
                            static_cast<bf16*>(s), static_cast<bf16*>(b), N, K, gs, bits, c->stream),
                 "emx_quantize");
  return EMX_OK;
}

int emx_rms_norm(emx_ctx* c, const void* x, const void* w, void* out, int rows, int dims, float eps) {
  return emx_grouped_rms_norm(c, x, w, out, rows, dims, eps, 1);
}

int emx_grouped_rms_norm(emx_ctx* c, const void* x, const void* w, void* out, int rows, int dims, float eps,
                         int groups) {
  EMX_REQUIRE(c && x && w && out, "emx_grouped_rms_norm: null argument");
  EMX_REQUIRE(groups >= 1, "grouped_rms_norm: groups must be >= 1, got %d", groups);
  EMX_REQUIRE(dims >= 1 && rows >= 0, "grouped_rms_norm: input must have at least 1 dimension");
  EMX_REQUIRE(dims % groups == 0, "grouped_rms_norm: last dimension %d is not divisible by groups %d", dims, groups);
  EMX_CHECK_CUDA(k_rms_norm(static_cast<const bf16*>(x), static_cast<const bf16*>(w), static_cast<bf16*>(out), rows,
                            dims, eps, groups, c->stream),
                 "emx_grouped_rms_norm");
  return EMX_OK;
}

int emx_rope(emx_ctx* c, const void* x, void* out, int heads, int T, int dims, float theta, int offset,
             const int32_t* offset_dev) {
  EMX_REQUIRE(c && x && out, "emx_rope: null argument");
  EMX_REQUIRE(dims > 0 && dims % 2 == 0 && heads >= 0 && T >= 0, "emx_rope: bad shape");
  void* sc = nullptr;
  int rc = ctx_scratch(c, sizeof(float) * (size_t)dims, &sc);
  if (rc) return rc;
  float* inv = static_cast<float*>(sc);
  EMX_CHECK_CUDA(k_rope_inv_freq(inv, dims, theta, c->stream), "emx_rope inv_freq");
  EMX_CHECK_CUDA(k_rope(static_cast<const bf16*>(x), static_cast<bf16*>(out), heads, T, dims, inv, offset,
                        offset_dev, c->stream),
                 "emx_rope");
  return EMX_OK;
}

int emx_sdpa_causal(emx_ctx* c, const void* q, const void* k, const void* v, void* out, int nq, int nkv, int T,
                    int hd, float scale, int out_tnd) {
  EMX_REQUIRE(c && q && k && v && out, "emx_sdpa_causal: null argument");
  EMX_REQUIRE(hd == 128, "emx_sdpa_causal: head_dim must be 128 (got %d)", hd);
  EMX_REQUIRE(nkv > 0 && nq % nkv == 0, "emx_sdpa_causal: n_q %% n_kv != 0");
  AttnPrefillArgs a = {};
  a.q = static_cast<const bf16*>(q);
  a.kc = static_cast<const bf16*>(k);
  a.vc = static_cast<const bf16*>(v);
  a.cap = T;
  a.offset = 0;
  a.T = T;
  a.nq = nq;
  a.nkv = nkv;
  a.head_dim = hd;
  a.scale = scale;
  a.out = static_cast<bf16*>(out);
  a.out_tnd = out_tnd;
  EMX_CHECK_CUDA(attn_prefill_launch(a, c->stream, c->status), "emx_sdpa_causal");
  return EMX_OK;
}

int emx_sdpa_decode(emx_ctx* c, const void* q, const void* kc, const void* vc, void* out, int nq, int nkv, int cap,
                    int hd, int length, float scale) {
  EMX_REQUIRE(c && q && kc && vc && out, "emx_sdpa_decode: null argument");
  EMX_REQUIRE(hd == 128, "emx_sdpa_decode: head_dim must be 128 (got %d)", hd);
  EMX_REQUIRE(nkv > 0 && nq % nkv == 0 && (nq / nkv == 1 || nq / nkv == 2 || nq / nkv == 4 || nq / nkv == 8),
              "emx_sdpa_decode: n_q/n_kv must be 1, 2, 4 or 8");
  EMX_REQUIRE(length >= 1 && length <= cap, "emx_sdpa_decode: length %d outside [1, cap=%d]", length, cap);
  const int splits = attn_decode_splits(nkv, c->num_sms, nq / nkv);
  const size_t part = (size_t)nkv * splits * (nq / nkv) * (hd + 2) * sizeof(float);
  void* sc = nullptr;
  int rc = ctx_scratch(c, part + 256 + sizeof(unsigned) * nkv, &sc);
  if (rc) return rc;
  AttnDecodeArgs a = {};
  a.q_in = static_cast<const bf16*>(q);
  a.kc = static_cast<bf16*>(const_cast<void*>(kc));
  a.vc = static_cast<bf16*>(const_cast<void*>(vc));
  a.cap = cap;
  a.nq = nq;
  a.nkv = nkv;
  a.head_dim = hd;
  a.pos = nullptr;
  a.pos_host = length - 1;
  a.scale = scale;
  a.out = static_cast<bf16*>(out);
  a.part = static_cast<float*>(sc);
  a.ticket = reinterpret_cast<unsigned*>(static_cast<char*>(sc) + ((part + 255) & ~(size_t)255));
  a.splits = splits;
  a.status = c->status;
  EMX_CHECK_CUDA(cudaMemsetAsync(a.ticket, 0, sizeof(unsigned) * nkv, c->stream), "emx_sdpa_decode tickets");
  EMX_CHECK_CUDA(attn_decode_launch(a, c->stream, false), "emx_sdpa_decode");
  return EMX_OK;
}

int emx_silu(emx_ctx* c, const void* x, void* out, size_t n) {
  EMX_REQUIRE(c && x && out, "emx_silu: null argument");
  EMX_CHECK_CUDA(k_silu(static_cast<const bf16*>(x), static_cast<bf16*>(out), n, c->stream), "emx_silu");
  return EMX_OK;
}

int emx_multiply(emx_ctx* c, const void* a, const void* b, void* out, size_t n) {
  EMX_REQUIRE(c && a && b && out, "emx_multiply: null argument");
  EMX_CHECK_CUDA(k_multiply(static_cast<const bf16*>(a), static_cast<const bf16*>(b), static_cast<bf16*>(out), n,
                            c->stream),
                 "emx_multiply");
  return EMX_OK;
}

int emx_add(emx_ctx* c, const void* a, const void* b, void* out, size_t n) {
  EMX_REQUIRE(c && a && b && out, "emx_add: null argument");
  EMX_CHECK_CUDA(k_add(static_cast<const bf16*>(a), static_cast<const bf16*>(b), static_cast<bf16*>(out), n,
                       c->stream),
                 "emx_add");
  return EMX_OK;
}

int emx_argmax(emx_ctx* c, const void* x, int rows, int n, int32_t* out) {
  EMX_REQUIRE(c && x && out, "emx_argmax: null argument");
  EMX_REQUIRE(n >= 1 && rows >= 0, "emx_argmax: bad shape");
  EMX_CHECK_CUDA(k_argmax(static_cast<const bf16*>(x), rows, n, out, c->stream), "emx_argmax");
  return EMX_OK;
}

int emx_softmax(emx_ctx* c, const void* x, void* out, int rows, int n) {
  EMX_REQUIRE(c && x && out, "emx_softmax: null argument");
  EMX_REQUIRE(n >= 1 && rows >= 0, "emx_softmax: bad shape");
  EMX_CHECK_CUDA(k_softmax(static_cast<const bf16*>(x), static_cast<bf16*>(out), rows, n, c->stream), "emx_softmax");
  return EMX_OK;
}

int emx_embed_quantized(emx_ctx* c, const void* w, const void* s, const void* b, const int32_t* ids, int T,
                        int hidden, int vocab, int gs, int bits, void* out) {
  EMX_REQUIRE(c && w && s && b && ids && out, "emx_embed_quantized: null argument");
  int rc = check_quant(vocab, hidden, gs, bits, "emx_embed_quantized");
  if (rc) return rc;
  EMX_CHECK_CUDA(k_embed(static_cast<const uint32_t*>(w), static_cast<const bf16*>(s), static_cast<const bf16*>(b),
                         ids, T, hidden, gs, bits, vocab, static_cast<bf16*>(out), c->status, c->stream),
                 "emx_embed_quantized");
  return EMX_OK;
}

int emx_slice_update(emx_ctx* c, void* cache, const void* upd, int nkv, int cap, int hd, int offset, int T) {
  EMX_REQUIRE(c && cache && upd, "emx_slice_update: null argument");
  EMX_REQUIRE(offset >= 0 && T >= 0 && offset + T <= cap, "emx_slice_update: rows [%d,%d) outside cap %d", offset,
              offset + T, cap);
  EMX_CHECK_CUDA(k_slice_update(static_cast<bf16*>(cache), static_cast<const bf16*>(upd), nkv, cap, hd, offset,
                                nullptr, T, c->stream),
                 "emx_slice_update");
  return EMX_OK;
}

int emx_scatter_single(emx_ctx* c, void* cache, const int32_t* offset, const void* upd, int nkv, int cap, int hd) {
  EMX_REQUIRE(c && cache && offset && upd, "emx_scatter_single: null argument");
  EMX_CHECK_CUDA(k_slice_update(static_cast<bf16*>(cache), static_cast<const bf16*>(upd), nkv, cap, hd, 0, offset, 1,
                                c->stream),
                 "emx_scatter_single");
  return EMX_OK;
}

int emx_moe_route(emx_ctx* c, const void* logits, int E, int k, int normalize, int32_t* idx, float* w) {
  EMX_REQUIRE(c && logits && idx && w, "emx_moe_route: null argument");
  EMX_REQUIRE(E >= 1 && E <= 1024 && k >= 1 && k <= 64 && k <= E, "emx_moe_route: need 1 <= k <= min(E, 64), E <= 1024");
  void* sc = nullptr;
  int rc = ctx_scratch(c, 256, &sc);
  if (rc) return rc;
  EMX_CHECK_CUDA(k_moe_route(static_cast<const bf16*>(logits), E, k, normalize, 0, E, idx, w, static_cast<int*>(sc),
                             c->stream, false),
                 "emx_moe_route");
  return EMX_OK;
}

int emx_gather_qmm(emx_ctx* c, const void* x, int x_per_slot, const void* w, const void* s, const void* b,
                   const int32_t* idx, int n_slots, void* y, int n_experts, int N, int K, int gs, int bits) {
  EMX_REQUIRE(c && x && w && s && b && idx && y, "emx_gather_qmm: null argument");
  int rc = check_quant(N, K, gs, bits, "emx_gather_qmm");
  if (rc) return rc;
  EMX_REQUIRE(N % 16 == 0 && n_slots >= 1 && n_slots <= 64 && n_experts >= 1, "emx_gather_qmm: bad shape");
  GemvPlan plan;
  if (gemv_make_plan(n_slots * N, K, bits, gs, kEpiStore, x_per_slot ? n_slots : 1, c->num_sms, &plan))
    return fail(EMX_ERR_INVALID, "emx_gather_qmm: unsupported shape N=%d K=%d", N, K);
  void* sc = nullptr;
  rc = ctx_scratch(c, 256, &sc);
  if (rc) return rc;
  EMX_CHECK_CUDA(cudaMemcpyAsync(sc, &n_slots, sizeof(int), cudaMemcpyHostToDevice, c->stream), "n_slots");
  GemvArgs a = {};
  a.w = static_cast<const uint32_t*>(w);
  a.s = static_cast<const bf16*>(s);
  a.b = static_cast<const bf16*>(b);
  a.N = n_slots * N;
  a.K = K;
  a.bits = bits;
  a.gs = gs;
  a.pro = kProX;
  a.epi = kEpiStore;
  a.x = static_cast<const bf16*>(x);
  a.x_slots = x_per_slot ? n_slots : 1;
  a.slot_expert = idx;
  a.n_slots = static_cast<const int*>(sc);
  a.slot_rows = N;
  a.y = static_cast<bf16*>(y);
  a.status = c->status;
  EMX_CHECK_CUDA(gemv_launch(a, plan, c->stream, false), "emx_gather_qmm");
  // the count lives in scratch: finish before another op may reuse it
  return ctx_sync_check(c, "emx_gather_qmm");
}

}  // extern "C"
