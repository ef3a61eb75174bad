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

#include <algorithm>
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

// Epilogue of one 128 x BN tile (warps 2-5): warp w reads accumulator lanes
// 32*(w % 4) with tcgen05.ld once `done` completes and applies the output
// step (store / residual / SwiGLU / fp32).
template <int BN, int EPI>
__device__ __forceinline__ void tc_epilogue(uint32_t tmem, uint64_t* done, int warp, int lane, int m0, int nt,
                                            const TcGemmArgs& a) {
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;  // output columns of one tile
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

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const TcGemmArgs a) {
  using C = Cfg<BN>;
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
    tc_epilogue<BN, EPI>(tmem, done, warp, lane, m0, nt, a);
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

// ---------------------------------------------------------------------------
// Dequantisation inside the GEMM: the weights stay MLX affine codes in HBM.
// Per 64-column k-block, TMA brings x (128 x 64 bf16, swizzled) and the raw
// codes of the tile's BN weight rows (BN x 32 bytes for int4, 64 for int8,
// unswizzled); sixteen dequant warps (2-17) turn them into bf16 — bit-exactly
// MLX's dequantisation, one rounding of s*q + b (fma.rn.bf16x2) — written in
// the 128-byte-swizzled K-major layout the MMA descriptor reads; warp 1
// issues the MMAs once a stage's tile is complete; warps 2-5 then run the
// epilogue.  The bf16 weights never travel through HBM.
constexpr int QSTAGES = 3;
constexpr int kDqWarps = 16;
constexpr int kQThreads = (2 + kDqWarps) * 32;

template <int BITS, int BN>
struct QCfg {
  static constexpr int ROW = BK * BITS / 8;  // raw code bytes per row per k-block
  static constexpr int RAW = BN * ROW;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES + RAW;  // A | B (bf16) | raw codes
  static constexpr int SMEM = 1024 + QSTAGES * STAGE + 256;
};

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Eight int4 codes (code e at bits 4e) -> eight bf16 in code order.
__device__ __forceinline__ uint4 dq_int4(uint32_t w, uint32_t s2, uint32_t b2) {
  uint32_t p[4];  // (code e, code e+4) as exact bf16 pairs: 128 + code via the exponent, minus 128
#pragma unroll
  for (int e = 0; e < 4; ++e)
    p[e] = bf16x2_fma(bf16x2_sub(lop3_and_or(w >> (4 * e), 0x000F000Fu, 0x43004300u), 0x43004300u), s2, b2);
  return make_uint4(prmt(p[0], p[1], 0x5410u), prmt(p[2], p[3], 0x5410u), prmt(p[0], p[1], 0x7632u),
                    prmt(p[2], p[3], 0x7632u));
}

// Four int8 codes (code e at bits 8e) -> four bf16 in code order.
__device__ __forceinline__ uint2 dq_int8(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t q01 = pack_bf2((float)(w & 0xFFu), (float)((w >> 8) & 0xFFu));   // exact: codes <= 255
  const uint32_t q23 = pack_bf2((float)((w >> 16) & 0xFFu), (float)(w >> 24));
  return make_uint2(bf16x2_fma(q01, s2, b2), bf16x2_fma(q23, s2, b2));
}

template <int BITS, int BN, int EPI>
__global__ void __launch_bounds__(kQThreads, 1)
    tc_qgemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_q,
                    const TcGemmArgs a) {
  using C = QCfg<BITS, BN>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + QSTAGES * C::STAGE);  // x + raw codes landed
  uint64_t* bready = full + QSTAGES;                                        // bf16 weight tile written
  uint64_t* empty = bready + QSTAGES;                                       // the MMAs of the stage are done
  uint64_t* done = empty + QSTAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* issued_slot = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int nt = blockIdx.y;
  // k-blocks [kb0, kb0 + nkl) of this CTA (split-K over blockIdx.z)
  const int nk = a.K / BK;
  const int kb0 = (int)((long long)blockIdx.z * nk / gridDim.z);
  const int nkl = (int)((long long)(blockIdx.z + 1) * nk / gridDim.z) - kb0;
  constexpr int WPB = BK * BITS / 32;  // code words per row per k-block

  if (threadIdx.x == 0) {
    for (int s = 0; s < QSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], kDqWarps);
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
    // ---- TMA producer: x tile and the raw codes of the tile's weight rows
    int issued = 0;
    for (int i = 0; i < nkl; ++i) {
      const int s = i % QSTAGES, kb = kb0 + i;
      if (i >= QSTAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((i / QSTAGES) - 1) & 1), a.status)) break;
      unsigned char* As = smem + s * C::STAGE;
      unsigned char* Rs = As + A_BYTES + C::B_BYTES;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(A_BYTES + C::RAW));
      tma_load_2d(As, &tma_a, kb * BK, m0, &full[s]);
      if (EPI == kTcSwiglu) {
        tma_load_2d(Rs, &tma_q, kb * WPB, nt * (BN / 2), &full[s]);
        tma_load_2d(Rs + (BN / 2) * C::ROW, &tma_q, kb * WPB, a.N + nt * (BN / 2), &full[s]);
      } else {
        tma_load_2d(Rs, &tma_q, kb * WPB, nt * BN, &full[s]);
      }
      issued = i + 1;
    }
    *issued_slot = issued;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    constexpr uint32_t idesc = make_idesc(BN);
    for (int i = 0; i < nkl; ++i) {
      const int s = i % QSTAGES;
      const uint32_t par = (uint32_t)((i / QSTAGES) & 1);
      if (!mbar_wait_bounded(&full[s], par, a.status) || !mbar_wait_bounded(&bready[s], par, a.status)) break;
      tc_fence_after();
      const unsigned char* As = smem + s * C::STAGE;
      const uint64_t ad = sw128_desc(As), bd = sw128_desc(As + A_BYTES);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        tc_mma(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
      tc_commit(&empty[s]);
    }
    tc_commit(done);
  } else if (warp >= 2) {
    // ---- dequantisation: thread t handles weight row t % BN of the tile,
    //      16-byte chunks [c0, c0 + NCH) of its 64 codes
    constexpr int TPR = (kDqWarps * 32) / BN;  // threads per row (2 or 4)
    constexpr int NCH = 8 / TPR;               // 16-byte chunks per thread
    static_assert(NCH * BITS / 4 >= 2, "a thread's codes are whole 8-byte runs");
    const int t = threadIdx.x - 64;
    const int r = t % BN;
    const int c0 = (t / BN) * NCH;
    const int nw_rows = EPI == kTcSwiglu ? 2 * a.N : a.N;  // rows of the weight matrix
    const int grow = EPI == kTcSwiglu ? (r < BN / 2 ? nt * (BN / 2) + r : a.N + nt * (BN / 2) + r - BN / 2)
                                      : nt * BN + r;
    const bool valid = grow < nw_rows;
    const int ng = a.K / 64;
    const uint16_t* sp = reinterpret_cast<const uint16_t*>(a.ws) + (size_t)(valid ? grow : 0) * ng;
    const uint16_t* bp = reinterpret_cast<const uint16_t*>(a.wb) + (size_t)(valid ? grow : 0) * ng;
    uint32_t sn = valid ? __ldg(sp + kb0) : 0u, bn = valid ? __ldg(bp + kb0) : 0u;  // group of the next k-block
    bool ok = true;
    for (int i = 0; i < nkl; ++i) {
      const int s = i % QSTAGES, kb = kb0 + i;
      const uint32_t s2 = sn | (sn << 16), b2 = bn | (bn << 16);
      if (i + 1 < nkl && valid) {
        sn = __ldg(sp + kb + 1);
        bn = __ldg(bp + kb + 1);
      }
      ok = ok && mbar_wait_bounded(&full[s], (uint32_t)((i / QSTAGES) & 1), a.status);
      unsigned char* Bs = smem + s * C::STAGE + A_BYTES;
      const unsigned char* raw = Bs + C::B_BYTES + r * C::ROW;
      unsigned char* dst = Bs + (r >> 3) * 1024 + (r & 7) * 128;
      // this thread's code words first (8- or 16-byte loads), then the chunks
      constexpr int NW = NCH * BITS / 4;  // words
      uint32_t wv[NW];
      const unsigned char* rw = raw + c0 * (BITS / 4) * 4;
      if (NW % 4 == 0) {
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) {
          const uint4 q = *reinterpret_cast<const uint4*>(rw + i * 16);
          wv[4 * i] = q.x, wv[4 * i + 1] = q.y, wv[4 * i + 2] = q.z, wv[4 * i + 3] = q.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < NW / 2; ++i) {
          const uint2 q = *reinterpret_cast<const uint2*>(rw + i * 8);
          wv[2 * i] = q.x, wv[2 * i + 1] = q.y;
        }
      }
#pragma unroll
      for (int i = 0; i < NCH; ++i) {  // chunk c0 + i: codes 8(c0+i) .. +7
        uint4 v;
        if (BITS == 4) {
          v = dq_int4(wv[i], s2, b2);
        } else {
          const uint2 lo = dq_int8(wv[2 * i], s2, b2), hi = dq_int8(wv[2 * i + 1], s2, b2);
          v = make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
        *reinterpret_cast<uint4*>(dst + (((c0 + i) ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[s]);
    }
    (void)ok;
    if (warp < 6) {
      if (gridDim.z == 1) {
        tc_epilogue<BN, EPI>(tmem, done, warp, lane, m0, nt, a);
      } else {
        // split-K: this CTA's fp32 partial of all BN accumulator columns,
        // summed (and the output step applied) by splitk_reduce_kernel
        const bool okd = mbar_wait_bounded(done, 0u, a.status);
        tc_fence_after();
        const int q = warp & 3;
        const int row = m0 + q * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
        const int nw = (EPI == kTcSwiglu ? 2 : 1) * a.N;  // accumulator columns of all tiles
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tl + c0, v);
          tmem_wait_ld();
          if (!okd || row >= a.M || nt * BN + c0 >= nw) continue;
          float4* dst = reinterpret_cast<float4*>(a.part + ((size_t)blockIdx.z * a.M + row) * nw + nt * BN + c0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                 __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0) {
    const int issued = *issued_slot;
    for (int i = issued > QSTAGES ? issued - QSTAGES : 0; i < issued; ++i)
      mbar_wait_bounded(&full[i % QSTAGES], (uint32_t)((i / QSTAGES) & 1), a.status);
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

// Sum of the split-K partials (in split order) and the output step, with the
// rounding points of tc_epilogue; one thread per 8 outputs of a row.
template <int EPI>
__global__ void splitk_reduce_kernel(const TcGemmArgs a, int ksplit, int bn) {
  const int nout_tile = EPI == kTcSwiglu ? bn / 2 : bn;
  const int nw = (EPI == kTcSwiglu ? 2 : 1) * a.N;
  const long long total = (long long)a.M * (a.N / 8);
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(idx / (a.N / 8)), n0 = (int)(idx % (a.N / 8)) * 8;
    const int nt = n0 / nout_tile, j = n0 % nout_tile;
    const int cg = nt * bn + j;  // accumulator column (gate part for SwiGLU)
    float g[8], u[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = u[e] = 0.f;
    for (int z = 0; z < ksplit; ++z) {
      const float* src = a.part + ((size_t)z * a.M + m) * nw;
      const float4 g0 = *reinterpret_cast<const float4*>(src + cg), g1 = *reinterpret_cast<const float4*>(src + cg + 4);
      g[0] += g0.x, g[1] += g0.y, g[2] += g0.z, g[3] += g0.w, g[4] += g1.x, g[5] += g1.y, g[6] += g1.z, g[7] += g1.w;
      if (EPI == kTcSwiglu) {
        const float4 u0 = *reinterpret_cast<const float4*>(src + cg + nout_tile);
        const float4 u1 = *reinterpret_cast<const float4*>(src + cg + nout_tile + 4);
        u[0] += u0.x, u[1] += u0.y, u[2] += u0.z, u[3] += u0.w, u[4] += u1.x, u[5] += u1.y, u[6] += u1.z, u[7] += u1.w;
      }
    }
    const size_t o = (size_t)m * a.N + n0;
    if (EPI == kTcF32) {
      reinterpret_cast<float4*>(a.yf + o)[0] = make_float4(g[0], g[1], g[2], g[3]);
      reinterpret_cast<float4*>(a.yf + o)[1] = make_float4(g[4], g[5], g[6], g[7]);
      continue;
    }
    uint32_t w[4];
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      float h[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int e = 2 * e2 + q;
        if (EPI == kTcStore) {
          h[q] = g[e];
        } else if (EPI == kTcResid) {
          h[q] = __fadd_rn(bf2f(a.res[o + e]), bfround(g[e]));
        } else {
          const float gv = bfround(g[e]), uv = bfround(u[e]);
          const float sg = bfround(sigmoid_f(gv));
          const float sv = bfround(__fmul_rn(gv, sg));
          h[q] = __fmul_rn(sv, uv);
        }
      }
      w[e2] = pack_bf2(h[0], h[1]);
    }
    *reinterpret_cast<uint4*>(a.y + o) = make_uint4(w[0], w[1], w[2], w[3]);
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

// Raw codes [rows][K*bits/32] uint32: boxes of one k-block's words x box_rows
// rows, unswizzled (the dequant warps read them row by row).
cudaError_t encode_codes(CUtensorMap* map, const uint32_t* base, uint64_t words, uint64_t rows, uint32_t box_words,
                         uint32_t box_rows) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {words, rows};
  const cuuint64_t strides[1] = {words * 4};
  const cuuint32_t box[2] = {box_words, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int BITS, int BN, int EPI>
cudaError_t launch_q(const TcGemmArgs& a, cudaStream_t st) {
  CUtensorMap ta, tq;
  cudaError_t e = encode_2d(&ta, a.x, (uint64_t)a.K, (uint64_t)a.M, BM);
  if (e != cudaSuccess) return e;
  const uint64_t wrows = EPI == kTcSwiglu ? 2ull * a.N : (uint64_t)a.N;
  constexpr uint32_t WPB = BK * BITS / 32;
  e = encode_codes(&tq, a.wq, (uint64_t)a.K * BITS / 32, wrows, WPB, EPI == kTcSwiglu ? BN / 2 : BN);
  if (e != cudaSuccess) return e;
  auto kern = tc_qgemm_kernel<BITS, BN, EPI>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, QCfg<BITS, BN>::SMEM);
  if (e != cudaSuccess) return e;
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;
  const int ks = a.part ? a.ksplit : 1;
  dim3 grid((a.M + BM - 1) / BM, (a.N + NOUT - 1) / NOUT, ks);
  kern<<<grid, kQThreads, QCfg<BITS, BN>::SMEM, st>>>(ta, tq, a);
  e = cudaGetLastError();
  if (e != cudaSuccess || ks == 1) return e;
  const long long work = (long long)a.M * (a.N / 8);
  splitk_reduce_kernel<EPI><<<(unsigned)std::min<long long>((work + 255) / 256, 4096), 256, 0, st>>>(a, ks, BN);
  return cudaGetLastError();
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

bool tc_qgemm_supported(const TcGemmArgs& a) {
  if (a.M <= 0 || a.K <= 0 || a.N <= 0) return false;
  if (a.K % BK != 0 || a.N % 32 != 0 || !(a.bits == 4 || a.bits == 8)) return false;
  if (!a.wq || !a.ws || !a.wb) return false;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.wq)) & 15) return false;
  return true;
}

int tc_qgemm_splits(const TcGemmArgs& a, int num_sms, size_t* part_bytes) {
  const int mt = (a.M + BM - 1) / BM;
  const bool wide = a.epi == kTcSwiglu || (a.N % 256 == 0 && (long long)mt * (a.N / 256) >= num_sms);
  const int nout = a.epi == kTcSwiglu ? 128 : wide ? 256 : 128;
  const long long tiles = (long long)mt * ((a.N + nout - 1) / nout);
  const int nk = a.K / BK;
  int ks = 1;
  if (tiles < num_sms) ks = (int)std::min<long long>((num_sms + tiles - 1) / tiles, std::max(1, nk / 4));
  if (part_bytes) *part_bytes = ks > 1 ? (size_t)ks * a.M * (a.epi == kTcSwiglu ? 2 : 1) * a.N * 4 : 0;
  return ks;
}

cudaError_t tc_qgemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  if (!tc_qgemm_supported(a)) return cudaErrorInvalidValue;
  const int mt = (a.M + BM - 1) / BM;
  const bool wide = a.N % 256 == 0 && (long long)mt * (a.N / 256) >= num_sms;
#define EMX_Q(B)                                                                                           \
  switch (a.epi) {                                                                                         \
    case kTcStore: return wide ? launch_q<B, 256, kTcStore>(a, st) : launch_q<B, 128, kTcStore>(a, st);   \
    case kTcResid: return wide ? launch_q<B, 256, kTcResid>(a, st) : launch_q<B, 128, kTcResid>(a, st);   \
    case kTcF32: return wide ? launch_q<B, 256, kTcF32>(a, st) : launch_q<B, 128, kTcF32>(a, st);         \
    case kTcSwiglu: return launch_q<B, 256, kTcSwiglu>(a, st);                                            \
    default: return cudaErrorInvalidValue;                                                                 \
  }
  if (a.bits == 4) {
    EMX_Q(4)
  }
  EMX_Q(8)
#undef EMX_Q
}

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
