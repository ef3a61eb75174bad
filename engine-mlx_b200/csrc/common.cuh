// common.cuh — shared device helpers for the sm_100a kernels of libemx.
//
// PTX wrappers for the Blackwell features the kernels lean on:
//   * programmatic dependent launch (griddepcontrol) so that a kernel's
//     weight streaming overlaps the tail of the kernel before it;
//   * the bulk-copy engine (cp.async.bulk global->shared with mbarrier
//     completion, and cp.async.bulk.prefetch.L2) — the untiled TMA path;
//   * mbarrier arrive/expect-tx/try-wait with a bounded spin.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace emx {

typedef __nv_bfloat16 bf16;

// ---------------------------------------------------------------- status
// Device-side error codes written to a per-context status word when a
// bounded wait gives up; the host reads it after synchronising.
enum : int {
  kDevOk = 0,
  kDevTimeoutMbar = 1,  // an mbarrier wait exceeded its spin limit
  kDevTimeoutPeer = 2,  // a peer flag wait exceeded its spin limit
  kDevBadToken = 3,     // a token id outside [0, vocab)
  kDevKvOverflow = 4,   // position >= KV capacity
};

// Upper bound on the polls of any spin-wait before it reports and returns.
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ void report_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------ bf16
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float bfround(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float bits2f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
__device__ __forceinline__ uint16_t f2bits(float v) {
  bf16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}

// MLX affine dequantization of one code: the bf16 nearest to the exact
// s*q + b (one bf16 FMA; q <= 255 is exact in bf16).
__device__ __forceinline__ bf16 dequant1(uint32_t q, bf16 s, bf16 b) {
  return __hfma(__float2bfloat16_rn((float)q), s, b);
}

// ------------------------------------------------------------------- PDL
// Wait until the preceding kernel in the stream has completed and its
// writes are visible.  A no-op when the launch carried no PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to begin launching.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// -------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Plain arrival (no transaction bytes) on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of an mbarrier phase: cheaper than try_wait when the
// phase has usually completed already.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Longest any bounded wait may take before it gives up.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Bounded wait on an mbarrier phase.  Returns false (and records a status)
// after kWaitLimitNs or kSpinLimit polls; the caller then skips the dependent
// work (its outputs are garbage, the status word says so) and the kernel ends.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  report_status(status, kDevTimeoutMbar);
  return false;
}

// ------------------------------------------------------ bulk copy engine
// One untiled TMA transfer global -> shared, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for data read exactly once (weights streamed per token): evict
// it first, so code, activations and the KV cache stay resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 cache-eviction policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Warm L2 with [src, src+bytes) without touching shared memory.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------- tensor cores
// Warp-level m16n8k16 bf16 MMA with fp32 accumulation (used by the batch-1
// GEMV as a dot-product engine and by the prefill kernels' fragments).  Not
// volatile: it is a pure function of its registers, and the compiler must be
// free to hoist the next shared-memory loads above it.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same MMA on fp16 operands (the batch-1 GEMV: magic-number codes
// against x staged in fp16).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x in one instruction (approximate, ~2 ulp; 0 for large negative x).
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// (v & mask) | magic in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t v, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "r"(mask), "r"(magic));
  return r;
}

// bf16x2 subtract of a packed constant (exact for the magic-number dequant).
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ uint2 lds64(const void* p) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (threadIdx.x < (unsigned)nw) ? red[threadIdx.x] : 0.0f;
  if (warp == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// sigmoid as MLX composes it for silu: 1/(1+exp(-|x|)), mirrored for x<0.
__device__ __forceinline__ float sigmoid_f(float v) {
  float e = expf(-fabsf(v));
  float y = __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
  return v < 0.0f ? __fsub_rn(1.0f, y) : y;
}

}  // namespace emx
