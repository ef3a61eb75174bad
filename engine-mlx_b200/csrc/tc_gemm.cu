// tc_gemm.cu — bf16 GEMM on sm_100a tensor cores: TMA -> shared memory ->
// tcgen05.mma -> tensor memory -> tcgen05.ld epilogue.
//
// One CTA per 128 x BN output tile, six warps:
//   warp 0 (one thread)  TMA producer: 128-row x 64-column tiles of x and
//                        BN-row tiles of W into a 4-stage ring (128-byte
//                        swizzle, the layout the MMA descriptors describe);
//   warp 1 (one thread)  MMA issuer: per stage four tcgen05.mma (K = 16 each)
//                        accumulate into BN tensor-memory columns; a
//                        tcgen05.commit per stage frees the stage, one more
//                        signals the epilogue; the warp owns the TMEM
//                        allocation;
//   warps 2-5            epilogue: each reads its 32 accumulator lanes (rows)
//                        with tcgen05.ld, applies the output step (store,
//                        residual add, SwiGLU with MLX's rounding points, or
//                        fp32) and writes the rows.
// SwiGLU tiles load 128 gate rows and the matching 128 up rows as one
// 256-column accumulator, so the activation fuses into the epilogue.
// Every mbarrier wait is bounded; a CTA always lets its issued copies land
// and always frees its tensor memory before it exits.
#include "tc_gemm.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace emx {

namespace {

constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr int kThreads = 192;
constexpr int A_BYTES = BM * BK * 2;

template <int BN>
struct Cfg {
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = 1024 + STAGES * STAGE + 256;
};

// tcgen05 instruction descriptor, kind::f16: D fp32, A and B bf16, both
// K-major, M = 128, N = n.
constexpr uint32_t make_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive fp32 columns: thread = lane, v[j] = column j.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const TcGemmArgs a) {
  using C = Cfg<BN>;
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;  // output columns of one tile
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment of the stage buffers (the swizzle pattern and the
  // descriptors assume it)
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* issued_slot = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int nt = blockIdx.y;
  const int nk = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *issued_slot = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer
    int issued = 0;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (kb >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((kb / STAGES) - 1) & 1), a.status)) break;
      unsigned char* As = smem + s * C::STAGE;
      unsigned char* Bs = As + A_BYTES;
      mbar_arrive_expect_tx(&full[s], (uint32_t)C::STAGE);
      tma_load_2d(As, &tma_a, kb * BK, m0, &full[s]);
      if (EPI == kTcSwiglu) {
        tma_load_2d(Bs, &tma_b, kb * BK, nt * (BN / 2), &full[s]);
        tma_load_2d(Bs + (BN / 2) * BK * 2, &tma_b, kb * BK, a.N + nt * (BN / 2), &full[s]);
      } else {
        tma_load_2d(Bs, &tma_b, kb * BK, nt * BN, &full[s]);
      }
      issued = kb + 1;
    }
    *issued_slot = issued;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    constexpr uint32_t idesc = make_idesc(BN);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait_bounded(&full[s], (uint32_t)((kb / STAGES) & 1), a.status)) break;
      tc_fence_after();
      const unsigned char* As = smem + s * C::STAGE;
      const uint64_t ad = sw128_desc(As), bd = sw128_desc(As + A_BYTES);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)  // +32 bytes along the swizzled row per K step
        tc_mma(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
      tc_commit(&empty[s]);
    }
    tc_commit(done);  // arrives once every MMA issued above has completed
  } else if (warp >= 2) {
    // ---- epilogue: warp w reads accumulator lanes 32*(w % 4) ...
    const bool ok = mbar_wait_bounded(done, 0u, a.status);
    tc_fence_after();
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
    for (int c0 = 0; c0 < NOUT; c0 += 32) {
      uint32_t v[32], u[32];
      tmem_ld32(tl + c0, v);
      if (EPI == kTcSwiglu) tmem_ld32(tl + NOUT + c0, u);
      tmem_wait_ld();
      const int col = nt * NOUT + c0;
      if (!ok || row >= a.M || col >= a.N) continue;  // N is a multiple of 32
      const size_t o = (size_t)row * a.N + col;
      if (EPI == kTcF32) {
        float4* dst = reinterpret_cast<float4*>(a.yf + o);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]), __uint_as_float(v[4 * j + 2]),
                               __uint_as_float(v[4 * j + 3]));
        continue;
      }
      uint32_t w[16];
      if (EPI == kTcStore) {
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = pack_bf2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
      } else if (EPI == kTcResid) {
        const uint4* rs = reinterpret_cast<const uint4*>(a.res + o);
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const uint4 r = rs[j4];
          const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 4 * j4 + e;
            const float r0 = __uint_as_float(rw[e] << 16), r1 = __uint_as_float(rw[e] & 0xffff0000u);
            w[j] = pack_bf2(__fadd_rn(r0, bfround(__uint_as_float(v[2 * j]))),
                            __fadd_rn(r1, bfround(__uint_as_float(v[2 * j + 1]))));
          }
        }
      } else {  // SwiGLU
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float h[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float gv = bfround(__uint_as_float(v[2 * j + e])), uv = bfround(__uint_as_float(u[2 * j + e]));
            const float sg = bfround(sigmoid_f(gv));
            const float sv = bfround(__fmul_rn(gv, sg));
            h[e] = __fmul_rn(sv, uv);
          }
          w[j] = pack_bf2(h[0], h[1]);
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(a.y + o);
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) dst[j4] = make_uint4(w[4 * j4], w[4 * j4 + 1], w[4 * j4 + 2], w[4 * j4 + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // the last copy issued into each stage has landed before the CTA exits
    const int issued = *issued_slot;
    for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; ++kb)
      mbar_wait_bounded(&full[kb % STAGES], (uint32_t)((kb / STAGES) & 1), a.status);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

// ----------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

cudaError_t encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int BN, int EPI>
cudaError_t launch_t(const TcGemmArgs& a, cudaStream_t st) {
  CUtensorMap ta, tb;
  cudaError_t e = encode_2d(&ta, a.x, (uint64_t)a.K, (uint64_t)a.M, BM);
  if (e != cudaSuccess) return e;
  const uint64_t wrows = EPI == kTcSwiglu ? 2ull * a.N : (uint64_t)a.N;
  e = encode_2d(&tb, a.w, (uint64_t)a.K, wrows, EPI == kTcSwiglu ? BN / 2 : BN);
  if (e != cudaSuccess) return e;
  auto kern = tc_gemm_kernel<BN, EPI>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
  if (e != cudaSuccess) return e;
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;
  dim3 grid((a.M + BM - 1) / BM, (a.N + NOUT - 1) / NOUT);
  kern<<<grid, kThreads, Cfg<BN>::SMEM, st>>>(ta, tb, a);
  return cudaGetLastError();
}

}  // namespace

bool tc_gemm_supported(const TcGemmArgs& a) {
  if (a.M <= 0 || a.K <= 0 || a.N <= 0) return false;
  if (a.K % BK != 0 || a.N % 32 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w)) & 15) return false;
  return true;
}

cudaError_t tc_gemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  if (!tc_gemm_supported(a)) return cudaErrorInvalidValue;
  const int mt = (a.M + BM - 1) / BM;
  // 256-column tiles when they still fill the machine, 128 otherwise
  const bool wide = a.N % 256 == 0 && (long long)mt * (a.N / 256) >= num_sms;
  switch (a.epi) {
    case kTcStore: return wide ? launch_t<256, kTcStore>(a, st) : launch_t<128, kTcStore>(a, st);
    case kTcResid: return wide ? launch_t<256, kTcResid>(a, st) : launch_t<128, kTcResid>(a, st);
    case kTcF32: return wide ? launch_t<256, kTcF32>(a, st) : launch_t<128, kTcF32>(a, st);
    case kTcSwiglu: return launch_t<256, kTcSwiglu>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace emx
