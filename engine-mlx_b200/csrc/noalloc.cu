// noalloc.cu — emx_sdpa_decode_noalloc: decode attention that allocates
// nothing.
//
// emx_sdpa_decode keeps its cross-CTA softmax partials and merge tickets in
// the context's grow-only scratch.  The first call of a larger shape grows
// that scratch: a stream synchronise, a free and a cudaMalloc through the
// context, counted against its memory limit.  Some callers cannot take that
// path:
//   * a caller whose context already sits at its memory limit
//     (emx_set_memory_limit) still has to run the attention of a step;
//   * a latency-bound decode loop cannot afford the device-wide stall that a
//     cudaMalloc or cudaFree implies in the middle of the loop;
//   * a caller recovering from an out-of-memory error must not enter the
//     allocator again to finish the step it was on.
// This variant takes its partials and tickets from one fixed, file-scope
// device array instead.  The kernel is the same attn_decode_kernel with the
// same split count, so its output is bit-identical to emx_sdpa_decode's.
//
// Limits and rules:
//   * kNoAllocScratchBytes (1 MiB) bounds the scratch: 256 bytes of tickets
//     (n_kv <= 64) and n_q * splits * (head_dim + 2) fp32 partials; a shape
//     that needs more is rejected with EMX_ERR_INVALID before any launch
//     (every BASELINE model shape needs at most 0.6 MiB);
//   * the tickets must be zero when the kernel starts: each call clears the
//     n_kv ticket words with cudaMemsetAsync on the context stream (no
//     allocation) and the kernel's merging CTA leaves them at zero again;
//     the partials need no initial value;
//   * there is one scratch per device, shared by every context and stream in
//     the process: calls that can overlap in time (two streams, two contexts
//     on one device, two host threads) race on it.  Calls on one stream are
//     ordered and safe;
//   * a call outside a stream capture looks the array's address up with
//     cudaGetSymbolAddress (the first may load the module; after a
//     cudaDeviceReset the next uncaptured call finds the reloaded array); a
//     call inside a capture reuses the last address, so make one call before
//     a capture begins and none across a device reset within a capture.
#include <mutex>

#include "attn_decode.cuh"
#include "ctx.cuh"

namespace emx {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
constexpr size_t kTicketBytes = 256;  // 64 ticket words
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device`.  Looked up again on
// every call made outside a stream capture (cheap once the module is loaded,
// and right after a cudaDeviceReset reloaded it); inside a capture the
// cached address is used.
int scratch_address(int device, cudaStream_t st, void** out) {
  std::lock_guard<std::mutex> lk(g_addr_mu);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) {
    cudaGetLastError();
    cap = cudaStreamCaptureStatusActive;  // unknown: do not touch the module
  }
  if (!g_addr[device] || cap == cudaStreamCaptureStatusNone) {
    int prev = 0;
    EMX_CHECK_CUDA(cudaGetDevice(&prev), "emx_sdpa_decode_noalloc setup");
    EMX_CHECK_CUDA(cudaSetDevice(device), "emx_sdpa_decode_noalloc setup");
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    cudaSetDevice(prev);
    if (e != cudaSuccess) return fail_cuda(e, "emx_sdpa_decode_noalloc setup (cudaGetSymbolAddress)");
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return EMX_OK;
}

}  // namespace
}  // namespace emx

using namespace emx;

#define NA_REQUIRE(cond, ...) \
  do {                        \
    if (!(cond)) return fail(EMX_ERR_INVALID, __VA_ARGS__); \
  } while (0)

extern "C" int emx_sdpa_decode_noalloc(emx_ctx* c, const void* q, const void* kc, const void* vc, void* out, int nq,
                                       int nkv, int cap, int hd, int length, float scale) {
  NA_REQUIRE(c && q && kc && vc && out, "emx_sdpa_decode_noalloc: null argument");
  NA_REQUIRE(hd == 128, "emx_sdpa_decode_noalloc: head_dim must be 128 (got %d)", hd);
  NA_REQUIRE(nkv > 0 && nq % nkv == 0 && (nq / nkv == 1 || nq / nkv == 2 || nq / nkv == 4 || nq / nkv == 8),
             "emx_sdpa_decode_noalloc: n_q/n_kv must be 1, 2, 4 or 8");
  NA_REQUIRE(length >= 1 && length <= cap, "emx_sdpa_decode_noalloc: length %d outside [1, cap=%d]", length, cap);
  NA_REQUIRE(c->device >= 0 && c->device < kMaxDevices, "emx_sdpa_decode_noalloc: device %d unsupported",
             c->device);
  NA_REQUIRE((size_t)nkv * sizeof(unsigned) <= kTicketBytes,
             "emx_sdpa_decode_noalloc: n_kv %d exceeds the %zu tickets of the static scratch", nkv,
             kTicketBytes / sizeof(unsigned));
  const int splits = attn_decode_splits(nkv, c->num_sms, nq / nkv);
  const size_t part = (size_t)nkv * splits * (nq / nkv) * (hd + 2) * sizeof(float);
  NA_REQUIRE(part <= kNoAllocScratchBytes - kTicketBytes,
             "emx_sdpa_decode_noalloc: n_q %d x %d splits needs %zu bytes of partials; the static scratch holds %zu",
             nq, splits, part, kNoAllocScratchBytes - kTicketBytes);
  void* base = nullptr;
  int rc = scratch_address(c->device, c->stream, &base);
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
  a.ticket = static_cast<unsigned*>(base);
  a.part = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kTicketBytes);
  a.splits = splits;
  a.status = c->status;
  EMX_CHECK_CUDA(cudaMemsetAsync(a.ticket, 0, sizeof(unsigned) * nkv, c->stream), "emx_sdpa_decode_noalloc tickets");
  EMX_CHECK_CUDA(attn_decode_launch(a, c->stream, false), "emx_sdpa_decode_noalloc");
  return EMX_OK;
}
