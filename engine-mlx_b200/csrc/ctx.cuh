// ctx.cuh — internal definition of emx_ctx and the error helpers shared by
// the C ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/emx.h"
#include "common.cuh"
#include "qgemm.cuh"

struct emx_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 0;
  int* status = nullptr;  // device-side status word
  std::mutex mu;
  std::unordered_map<void*, size_t> allocs;
  size_t active = 0, peak = 0, limit = (size_t)-1;
  emx::GemmCtx* gemm = nullptr;
  // grow-only scratch for op-level kernels that need cross-CTA partials
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
};

namespace emx {

// Records `msg` as the calling thread's last error, forwards it to the
// installed handler and returns `code`.
int fail(int code, const char* fmt, ...);
int fail_cuda(cudaError_t e, const char* what);
// Tracked device allocation through the context (counts toward active/peak
// memory and the limit).
int ctx_alloc(emx_ctx* c, size_t bytes, void** p);
void ctx_free(emx_ctx* c, void* p);
// Grow-only per-context scratch (stream-ordered reuse).
int ctx_scratch(emx_ctx* c, size_t bytes, void** p);
// Synchronises the stream and turns a device-side status into an error.
int ctx_sync_check(emx_ctx* c, const char* what);

}  // namespace emx

#define EMX_CHECK_CUDA(expr, what)                       \
  do {                                                   \
    cudaError_t _e = (expr);                             \
    if (_e != cudaSuccess) return emx::fail_cuda(_e, what); \
  } while (0)
