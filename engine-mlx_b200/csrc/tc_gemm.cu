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
//
// Short prompts give fewer output tiles than SMs, so K is split across the
// CTAs of a thread-block cluster (grid z = cluster z = splits).  After the
// main loop each CTA owns every splits-th 32-column chunk of the tile: the
// other CTAs write their fp32 partials of that chunk into its shared memory
// (distributed shared memory, into the then idle stage ring), and the owner
// sums the partials in split order (its own straight from tensor memory) and
// applies the output step.  Partials never leave the SM cluster.
constexpr int kDqWarps = 16;
constexpr int kQThreads = (2 + kDqWarps) * 32;
constexpr int kMaxSplits = 8;  // portable cluster size

template <int BITS, int BN>
struct QCfg {
  static constexpr int ROW = BK * BITS / 8;  // raw code bytes per row per k-block
  static constexpr int RAW = BN * ROW;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES + RAW;  // A | B (bf16) | raw codes
  static constexpr int NST = BN == 256 ? 3 : 5;           // stages within 227 KB
  static constexpr int RING = NST * STAGE;
  static constexpr int SMEM = 1024 + RING + 256;
};

// Shared-memory bytes a split owner receives: (splits - 1) partials of its
// chunks, 128 rows each, `cw` fp32 per row and chunk (64 for SwiGLU: gate
// and up).
__host__ __device__ constexpr int q_recv_bytes(int nout, int epi, int ks) {
  return (ks - 1) * ((nout / 32 + ks - 1) / ks) * BM * (epi == kTcSwiglu ? 64 : 32) * 4;
}

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

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of `local` (a shared::cta address of this
// CTA's layout) in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t map_rank(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Output step for W (16 or 32) consecutive outputs of one row (g: gate /
// value accumulators, u: up accumulators for SwiGLU), MLX's rounding points.
template <int EPI, int W>
__device__ __forceinline__ void q_store(const TcGemmArgs& a, int row, int col, const float (&g)[W],
                                        const float (&u)[W]) {
  const size_t o = (size_t)row * a.N + col;
  if (EPI == kTcF32) {
    float4* dst = reinterpret_cast<float4*>(a.yf + o);
#pragma unroll
    for (int j = 0; j < W / 4; ++j) dst[j] = make_float4(g[4 * j], g[4 * j + 1], g[4 * j + 2], g[4 * j + 3]);
    return;
  }
  uint32_t w[W / 2];
  if (EPI == kTcStore) {
#pragma unroll
    for (int j = 0; j < W / 2; ++j) w[j] = pack_bf2(g[2 * j], g[2 * j + 1]);
  } else if (EPI == kTcResid) {
    const uint4* rs = reinterpret_cast<const uint4*>(a.res + o);
#pragma unroll
    for (int j4 = 0; j4 < W / 8; ++j4) {
      const uint4 r = rs[j4];
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * j4 + e;
        const float r0 = __uint_as_float(rw[e] << 16), r1 = __uint_as_float(rw[e] & 0xffff0000u);
        w[j] = pack_bf2(__fadd_rn(r0, bfround(g[2 * j])), __fadd_rn(r1, bfround(g[2 * j + 1])));
      }
    }
  } else {  // SwiGLU
#pragma unroll
    for (int j = 0; j < W / 2; ++j) {
      float h[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gv = bfround(g[2 * j + e]), uv = bfround(u[2 * j + e]);
        const float sg = bfround(sigmoid_f(gv));
        const float sv = bfround(__fmul_rn(gv, sg));
        h[e] = __fmul_rn(sv, uv);
      }
      w[j] = pack_bf2(h[0], h[1]);
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(a.y + o);
#pragma unroll
  for (int j4 = 0; j4 < W / 8; ++j4) dst[j4] = make_uint4(w[4 * j4], w[4 * j4 + 1], w[4 * j4 + 2], w[4 * j4 + 3]);
}

// 32 lanes x 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// Split-K reduction across the cluster (warps 2-5, after `done`): phase 0
// sends this CTA's partials of the chunks other ranks own; after a cluster
// barrier, phase 1 sums the owned chunks in rank order and stores them.
// Receive layout in the owner's ring: [src slot][local chunk][16-byte unit of
// the row's chunk][row], so the 32 lanes (rows) of a warp write and read 512
// contiguous bytes per instruction.
template <int BN, int EPI>
__device__ __forceinline__ void q_cluster_send(uint32_t tmem, int warp, int lane, unsigned char* ring) {
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;
  constexpr int NCH = NOUT / 32, NU = EPI == kTcSwiglu ? 16 : 8;
  const int me = (int)blockIdx.z, ks = (int)gridDim.z;
  const int maxlc = (NCH + ks - 1) / ks;
  const int q = warp & 3, row = q * 32 + lane;
  const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
  const uint32_t base = smem_u32(ring);
#pragma unroll 1
  for (int oc = 0; oc < NCH; ++oc) {
    const int owner = oc % ks;
    if (owner == me) continue;
    uint32_t v[32];
    const int slot = me < owner ? me : me - 1;
    const uint32_t dst =
        map_rank(base + (uint32_t)(((slot * maxlc + oc / ks) * NU * BM + row) * 16), (uint32_t)owner);
    tmem_ld32(tl + oc * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int un = 0; un < 8; ++un)
      st_cluster_v4(dst + un * BM * 16, make_uint4(v[4 * un], v[4 * un + 1], v[4 * un + 2], v[4 * un + 3]));
    if (EPI == kTcSwiglu) {
      tmem_ld32(tl + NOUT + oc * 32, v);
      tmem_wait_ld();
#pragma unroll
      for (int un = 0; un < 8; ++un)
        st_cluster_v4(dst + (8 + un) * BM * 16, make_uint4(v[4 * un], v[4 * un + 1], v[4 * un + 2], v[4 * un + 3]));
    }
  }
}

template <int BN, int EPI>
__device__ __forceinline__ void q_cluster_reduce(uint32_t tmem, int warp, int lane, const unsigned char* ring, int m0,
                                                 int nt, const TcGemmArgs& a, bool ok) {
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;
  constexpr int NCH = NOUT / 32, NU = EPI == kTcSwiglu ? 16 : 8;
  const int me = (int)blockIdx.z, ks = (int)gridDim.z;
  const int maxlc = (NCH + ks - 1) / ks;
  const int q = warp & 3, rl = q * 32 + lane, row = m0 + rl;
  const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
  for (int oc = me; oc < NCH; oc += ks) {
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {  // 16-column halves of the chunk
      float g[16], u[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) g[j] = u[j] = 0.f;
#pragma unroll 1
      for (int r = 0; r < ks; ++r) {  // split order
        if (r == me) {
          uint32_t v[16];
          tmem_ld16(tl + oc * 32 + h * 16, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) g[j] += __uint_as_float(v[j]);
          if (EPI == kTcSwiglu) {
            tmem_ld16(tl + NOUT + oc * 32 + h * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) u[j] += __uint_as_float(v[j]);
          }
        } else {
          const int slot = r < me ? r : r - 1;
          const unsigned char* src = ring + ((slot * maxlc + oc / ks) * NU * BM + rl) * 16;
#pragma unroll
          for (int un = 0; un < 4; ++un) {
            const float4 f = *reinterpret_cast<const float4*>(src + (4 * h + un) * BM * 16);
            g[4 * un] += f.x, g[4 * un + 1] += f.y, g[4 * un + 2] += f.z, g[4 * un + 3] += f.w;
          }
          if (EPI == kTcSwiglu) {
#pragma unroll
            for (int un = 0; un < 4; ++un) {
              const float4 f = *reinterpret_cast<const float4*>(src + (8 + 4 * h + un) * BM * 16);
              u[4 * un] += f.x, u[4 * un + 1] += f.y, u[4 * un + 2] += f.z, u[4 * un + 3] += f.w;
            }
          }
        }
      }
      const int col = nt * NOUT + oc * 32 + h * 16;
      if (ok && row < a.M && col < a.N) q_store<EPI, 16>(a, row, col, g, u);
    }
  }
}

template <int BITS, int BN, int EPI>
__global__ void __launch_bounds__(kQThreads, 1)
    tc_qgemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_q,
                    const TcGemmArgs a) {
  using C = QCfg<BITS, BN>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING);  // x + raw codes landed
  uint64_t* bready = full + C::NST;                             // bf16 weight tile written
  uint64_t* empty = bready + C::NST;                            // the MMAs of the stage are done
  uint64_t* done = empty + C::NST;
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
    for (int s = 0; s < C::NST; ++s) {
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
      const int s = i % C::NST, kb = kb0 + i;
      if (i >= C::NST && !mbar_wait_bounded(&empty[s], (uint32_t)(((i / C::NST) - 1) & 1), a.status)) break;
      unsigned char* As = smem + s * C::STAGE;
      unsigned char* Rs = As + A_BYTES + C::B_BYTES;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(A_BYTES + C::RAW));
      if (EPI == kTcSwiglu) {
        tma_load_2d(Rs, &tma_q, kb * WPB, nt * (BN / 2), &full[s]);
        tma_load_2d(Rs + (BN / 2) * C::ROW, &tma_q, kb * WPB, a.N + nt * (BN / 2), &full[s]);
      } else {
        tma_load_2d(Rs, &tma_q, kb * WPB, nt * BN, &full[s]);
      }
      tma_load_2d(As, &tma_a, kb * BK, m0, &full[s]);
      issued = i + 1;
    }
    *issued_slot = issued;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    constexpr uint32_t idesc = make_idesc(BN);
    for (int i = 0; i < nkl; ++i) {
      const int s = i % C::NST;
      const uint32_t par = (uint32_t)((i / C::NST) & 1);
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
    // ---- dequantisation: thread t handles the 16-byte output chunk t % 8
    //      (codes 8c .. 8c+7) of weight rows t / 8 + 64 x, so a warp reads
    //      a contiguous run of raw codes and writes whole swizzled rows
    constexpr int CPT = BN * 8 / (kDqWarps * 32);  // chunks per thread (2 or 4)
    constexpr int D = 8 / CPT;                     // k-blocks of scales / biases in flight
    const int t = threadIdx.x - 64;
    const int c = t & 7, r0 = t >> 3;
    const int nw_rows = EPI == kTcSwiglu ? 2 * a.N : a.N;  // rows of the weight matrix
    const int ng = a.K / 64;
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(a.ws) + kb0;
    const uint16_t* bbase = reinterpret_cast<const uint16_t*>(a.wb) + kb0;
    int soff[CPT];
    bool valid[CPT];
#pragma unroll
    for (int x = 0; x < CPT; ++x) {
      const int r = r0 + 64 * x;
      const int grow = EPI == kTcSwiglu ? (r < BN / 2 ? nt * (BN / 2) + r : a.N + nt * (BN / 2) + r - BN / 2)
                                        : nt * BN + r;
      valid[x] = grow < nw_rows;
      soff[x] = (valid[x] ? grow : 0) * ng;
      if (c == 0 && valid[x]) {  // this CTA's scales and biases of the row into L2
        asm volatile("prefetch.global.L2 [%0];" ::"l"(sbase + soff[x]));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(bbase + soff[x]));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(sbase + soff[x] + nkl - 1));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(bbase + soff[x] + nkl - 1));
      }
    }
    // scales and biases of k-blocks i .. i + D - 1 in flight
    uint32_t sq[CPT][D], bq[CPT][D];
#pragma unroll
    for (int j = 0; j < D; ++j) {
#pragma unroll
      for (int x = 0; x < CPT; ++x) {
        sq[x][j] = valid[x] && j < nkl ? __ldg(sbase + soff[x] + j) : 0u;
        bq[x][j] = valid[x] && j < nkl ? __ldg(bbase + soff[x] + j) : 0u;
      }
    }
    bool ok = true;
#pragma unroll 1
    for (int i0 = 0; i0 < nkl; i0 += D) {
#pragma unroll
      for (int j = 0; j < D; ++j) {
        const int i = i0 + j;
        if (i >= nkl) break;
        const int s = i % C::NST;
        ok = ok && mbar_wait_bounded(&full[s], (uint32_t)((i / C::NST) & 1), a.status);
        unsigned char* Bs = smem + s * C::STAGE + A_BYTES;
        const unsigned char* raw = Bs + C::B_BYTES;
#pragma unroll
        for (int x = 0; x < CPT; ++x) {
          const int r = r0 + 64 * x;
          const uint32_t s2 = sq[x][j] | (sq[x][j] << 16), b2 = bq[x][j] | (bq[x][j] << 16);
          if (valid[x] && i + D < nkl) {
            sq[x][j] = __ldg(sbase + soff[x] + i + D);
            bq[x][j] = __ldg(bbase + soff[x] + i + D);
          }
          uint4 v;
          if (BITS == 4) {
            v = dq_int4(*reinterpret_cast<const uint32_t*>(raw + r * C::ROW + c * 4), s2, b2);
          } else {
            const uint2 wv = *reinterpret_cast<const uint2*>(raw + r * C::ROW + c * 8);
            const uint2 lo = dq_int8(wv.x, s2, b2), hi = dq_int8(wv.y, s2, b2);
            v = make_uint4(lo.x, lo.y, hi.x, hi.y);
          }
          *reinterpret_cast<uint4*>(Bs + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = v;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[s]);
      }
    }
    (void)ok;
    if (warp < 6 && gridDim.z == 1) tc_epilogue<BN, EPI>(tmem, done, warp, lane, m0, nt, a);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // the last copy issued into each stage has landed before the ring is
    // reused or the CTA exits
    const int issued = *issued_slot;
    for (int i = issued > C::NST ? issued - C::NST : 0; i < issued; ++i)
      mbar_wait_bounded(&full[i % C::NST], (uint32_t)((i / C::NST) & 1), a.status);
  }
  if (gridDim.z > 1) {
    // every CTA of the cluster is past its main loop (its ring is free)
    // before partials are written into it; every partial has landed before
    // an owner reads
    bool okd = true;
    if (warp >= 2 && warp < 6) {
      okd = mbar_wait_bounded(done, 0u, a.status);
      tc_fence_after();
    }
    cluster_sync_all();
    if (warp >= 2 && warp < 6) q_cluster_send<BN, EPI>(tmem, warp, lane, smem);
    cluster_sync_all();
    if (warp >= 2 && warp < 6) q_cluster_reduce<BN, EPI>(tmem, warp, lane, smem, m0, nt, a, okd);
    tc_fence_before();
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

// --------------------------------------------- packed-layout prefill GEMM
// The same GEMM over the packed tiles of the decode GEMV (16 rows x 8 groups
// per tile, codes in MMA-fragment order, scales and biases appended), so the
// prefill reads the weight bytes the decode step reads and needs no
// MLX-layout copy.  Orientation: the dequantised weights are MMA operand A
// and live in tensor memory (128 weight rows = the 128 lanes, 32 columns per
// k-block stage), written by the dequant warps with tcgen05.st; x is operand
// B, NT tokens x 64 columns per k-block from shared memory (TMA, 128-byte
// swizzle); the accumulator D is [128 weight rows x NT tokens].  Shared
// memory then carries only x and the raw codes (no bf16 weight tile is
// written to or read from it).  K-blocks move in groups of two: one barrier
// per group says its x tiles landed and its weight stages are written, one
// tcgen05.commit per group frees them (a barrier wait in the MMA issuer
// stalls the tensor pipe, so it is paid once per group), four groups in
// flight.  Measured on a 128-token prompt: ~0.35 us per k-block, the MMA
// issue itself ~70% of the tensor rate; a bulk copy costs the copy engine
// the same few tens of nanoseconds whatever its size, so weights move as
// whole packed tiles.  Prompts above 128 tokens use the dequant-to-scratch
// GEMM (tc_gemm_kernel), which measured faster there.
//
// Warp roles (19 warps):
//   warp 0 lane 0   x tiles by TMA
//   warp 1 lane 0   tcgen05.mma issuer, owns the tensor memory (512 columns)
//   warp 2          code units by bulk copy, one copy per lane (int4: each
//                   row block's whole tile of a span; int8: each row block's
//                   half-span codes and its scale/bias block)
//   warps 3-18      dequantisation, a group at a time: warp w writes lane
//                   quarter w % 4 (rows 32 (w % 4) ..) and 16-code slice quad
//                   (w - 3) / 4 of each k-block; then all sixteen run the
//                   epilogue.
// SwiGLU row blocks alternate gate and up, so lanes 0-15 of a warp hold gate
// rows and lanes 16-31 the matching up rows of one logical block.  K is split
// across the CTAs of a cluster by whole spans, evenly; each CTA's partial of
// the 32-token column chunks other ranks own goes to their shared memory and
// the owner sums in split order.
constexpr int kWWarps = 19;
constexpr int kWThreads = kWWarps * 32;

template <int BITS, int NT>
struct WCfg {
  static constexpr int TA = 16 * 512 * BITS / 8;  // code bytes of a packed tile
  static constexpr int HALF_A = TA / 2;           // one half-span's codes
  static constexpr int TILE = TA + 512;           // packed tile bytes
  static constexpr bool SPAN = BITS == 4;         // unit = span (else half-span)
  static constexpr int UNIT = SPAN ? 8 * TILE : 8 * (HALF_A + 512);
  static constexpr int UKB = SPAN ? 8 : 4;        // k-blocks per unit
  static constexpr int NCB = 2;                   // units in flight (the next loads while one is dequantised)
  static constexpr int X_BYTES = NT * BK * 2;     // x tile of one k-block
  // k-blocks per group: the MMA thread waits once per group (a wait, even
  // on a completed barrier, idles the tensor pipe for a fraction of a
  // microsecond, so it must sit behind a group's worth of queued MMAs)
  static constexpr int G = 2;
  static constexpr int NXMAX = (225 * 1024 - NCB * UNIT) / X_BYTES;
  static constexpr int NWMAX = (512 - NT) / 32;  // weight stages tensor memory holds
  static constexpr int NGB = (NXMAX < NWMAX ? NXMAX : NWMAX) / G;  // groups in flight
  static constexpr int NS = NGB * G;             // k-block stages (x tiles, weight stages)
  static constexpr int RING = NS * X_BYTES;
  static constexpr int SMEM = 1024 + RING + NCB * UNIT + 512;
  static_assert(NGB >= 2, "at least two groups in flight");
  static_assert(UKB % G == 0, "a unit holds whole groups");
};

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void tc_mma_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Two bf16 codes from bytes 0 and 2 of w: low nibbles as 128 + lo, high
// nibbles as 2048 + 16 hi (exact exponent tricks), then lo + 16 hi exactly.
__device__ __forceinline__ uint32_t bytes02_bf16(uint32_t w) {
  const uint32_t lo = bf16x2_sub(lop3_and_or(w, 0x000F000Fu, 0x43004300u), 0x43004300u);
  const uint32_t hi = bf16x2_sub(lop3_and_or(w >> 4, 0x000F000Fu, 0x45004500u), 0x45004500u);
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(lo), "r"(hi));
  return r;
}

// Output step for 16 tokens of one weight row (feature n = lane's row):
// v[t] = acc of token m0t + t; rows from mend on are not stored.  SwiGLU: lanes 0-15 gate, 16-31 up of the
// same 16 features.
template <int EPI>
__device__ __forceinline__ void w_store16(const TcGemmArgs& a, int n, int m0t, int mend, int lane, float (&v)[16],
                                          bool ok) {
  if (EPI == kTcSwiglu) {
    float h[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const float up = __shfl_down_sync(0xffffffffu, v[t], 16);
      const float gv = bfround(v[t]), uv = bfround(up);
      const float sg = bfround(sigmoid_f(gv));
      const float sv = bfround(__fmul_rn(gv, sg));
      h[t] = __fmul_rn(sv, uv);
    }
    if (!ok || lane >= 16 || n >= a.N) return;
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (m0t + t < mend) a.y[(size_t)(m0t + t) * a.N + n] = f2bf(h[t]);
    return;
  }
  if (!ok || n >= a.N) return;
  if (EPI == kTcResid) {
    // every residual value first (independent loads; y may alias res, and
    // each element belongs to this thread alone), then the stores
    float r[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) r[t] = m0t + t < mend ? bf2f(a.res[(size_t)(m0t + t) * a.N + n]) : 0.f;
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (m0t + t < mend) a.y[(size_t)(m0t + t) * a.N + n] = f2bf(__fadd_rn(r[t], bfround(v[t])));
    return;
  }
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const int m = m0t + t;
    if (m >= mend) break;
    const size_t o = (size_t)m * a.N + n;
    if (EPI == kTcF32) a.yf[o] = v[t];
    else a.y[o] = f2bf(v[t]);
  }
}

template <int BITS, int EPI, int NT>
__global__ void __launch_bounds__(kWThreads, 1)
    tc_pgemm_kernel(const __grid_constant__ CUtensorMap tma_x, const TcGemmArgs a) {
  using C = WCfg<BITS, NT>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* units = smem + C::RING;
  uint64_t* gfull = reinterpret_cast<uint64_t*>(units + C::NCB * C::UNIT);  // group's x landed + weights written
  uint64_t* gempty = gfull + C::NGB;                                        // the group's MMAs are done
  uint64_t* cfull = gempty + C::NGB;                                        // code unit landed
  uint64_t* cempty = cfull + C::NCB;                                        // code unit dequantised
  uint64_t* done = cempty + C::NCB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* issued_x = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued_c = issued_x + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.y;  // 8 packed row blocks
  int m0 = blockIdx.x * NT, mend = a.M;  // rows [m0, min(m0 + NT, mend)) of x
  const unsigned char* wp = a.wp;
  if (a.tiles) {  // grouped: this CTA's tile of one expert, or nothing
    if ((int)blockIdx.x >= *a.n_tiles) return;
    const int4 ti = a.tiles[blockIdx.x];
    wp += (size_t)ti.x * a.expert_stride;
    m0 = ti.y;
    mend = ti.z;
  }
  // spans [sp0, sp0 + nsl) of this CTA
  const int sp0 = (int)((long long)blockIdx.z * a.S / gridDim.z);
  const int nsl = (int)((long long)(blockIdx.z + 1) * a.S / gridDim.z) - sp0;
  const int nkl = 8 * nsl, nun = nkl / C::UKB, ngr = nkl / C::G;

  if (threadIdx.x == 0) {
    for (int q = 0; q < C::NGB; ++q) {
      mbar_init(&gfull[q], 1 + 16);
      mbar_init(&gempty[q], 1);
    }
    for (int u = 0; u < C::NCB; ++u) {
      mbar_init(&cfull[u], 1);
      mbar_init(&cempty[u], 16);
    }
    mbar_init(done, 1);
    *issued_x = 0;
    *issued_c = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- x tiles: NT tokens x 64 columns per k-block (128-row boxes), a
    //      group of k-blocks per barrier
    int issued = 0;
    for (int q = 0; q < ngr; ++q) {
      const int gb = q % C::NGB;
      if (q >= C::NGB && !mbar_wait_bounded(&gempty[gb], (uint32_t)(((q / C::NGB) - 1) & 1), a.status)) break;
      mbar_arrive_expect_tx(&gfull[gb], (uint32_t)(C::G * C::X_BYTES));
      for (int gk = 0; gk < C::G; ++gk) {
        const int i = q * C::G + gk, s = i % C::NS;
#pragma unroll
        for (int h = 0; h < NT / BM; ++h)
          tma_load_2d(smem + s * C::X_BYTES + h * A_BYTES, &tma_x, (8 * sp0 + i) * BK, m0 + h * BM, &gfull[gb]);
      }
      issued = q + 1;
    }
    *issued_x = issued;
  } else if (warp == 2) {
    // ---- code units
    const int rb0 = nt * 8;
    const int nrb = min(8, a.nrb - rb0);
    const uint64_t pol = l2_evict_first_policy();
    int issued = 0;
    for (int u = 0; u < nun; ++u) {
      const int c = u % C::NCB;
      bool go = true;
      if (lane == 0 && u >= C::NCB) go = mbar_wait_bounded(&cempty[c], (uint32_t)(((u / C::NCB) - 1) & 1), a.status);
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      unsigned char* dst = units + c * C::UNIT;
      if (C::SPAN) {
        if (lane == 0) mbar_arrive_expect_tx(&cfull[c], (uint32_t)(nrb * C::TILE));
        __syncwarp();
        if (lane < nrb)
          bulk_g2s_hint(dst + lane * C::TILE, wp + ((size_t)(rb0 + lane) * a.S + sp0 + u) * C::TILE,
                        (uint32_t)C::TILE, &cfull[c], pol);
      } else {
        const int hs = u & 1, sp = sp0 + (u >> 1);
        if (lane == 0) mbar_arrive_expect_tx(&cfull[c], (uint32_t)(nrb * (C::HALF_A + 512)));
        __syncwarp();
        const int j = lane & 7;
        if (lane < 16 && j < nrb) {
          const unsigned char* tile = wp + ((size_t)(rb0 + j) * a.S + sp) * C::TILE;
          if (lane < 8)
            bulk_g2s_hint(dst + j * (C::HALF_A + 512), tile + hs * C::HALF_A, (uint32_t)C::HALF_A, &cfull[c], pol);
          else
            bulk_g2s_hint(dst + j * (C::HALF_A + 512) + C::HALF_A, tile + C::TA, 512u, &cfull[c], pol);
        }
      }
      issued = u + 1;
    }
    if (lane == 0) *issued_c = issued;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: D[128 rows x NT tokens] += W(tmem)[128 x 64] . x[NT x 64]^T
    constexpr uint32_t idesc = make_idesc(NT);
    for (int q = 0; q < ngr; ++q) {
      const int gb = q % C::NGB;
      if (!mbar_wait_bounded(&gfull[gb], (uint32_t)((q / C::NGB) & 1), a.status)) break;
      tc_fence_after();
#pragma unroll
      for (int gk = 0; gk < C::G; ++gk) {
        const int i = q * C::G + gk, s = i % C::NS;
        const uint64_t bd = sw128_desc(smem + s * C::X_BYTES);
        const uint32_t aw = tmem + NT + 32 * s;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) tc_mma_ta(tmem, aw + 8 * k, bd + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
      }
      tc_commit(&gempty[gb]);
    }
    tc_commit(done);
  } else if (warp >= 3) {
    // ---- dequantisation into tensor memory, KG k-blocks at a time so the
    //      loads, the stores to tensor memory and the hand-off overlap
    const int lq = warp & 3, qd = (warp - 3) >> 2;  // lane quarter, 16-code slice quad
    const int r = 32 * lq + lane;                    // weight row of the tile
    const int j = r >> 4, g = r & 7, isb = (r >> 3) & 1;
    const uint32_t tbase = tmem + ((uint32_t)(32 * lq) << 16) + NT + 8 * qd;
    constexpr int KG = C::G;
    bool ok = true;
#pragma unroll 1
    for (int u = 0; u < nun; ++u) {
      const int c = u % C::NCB;
      ok = ok && mbar_wait_bounded(&cfull[c], (uint32_t)((u / C::NCB) & 1), a.status);
      const unsigned char* ubase = units + c * C::UNIT;
#pragma unroll 1
      for (int G0 = 0; G0 < C::UKB; G0 += KG) {
        const int i0 = C::UKB * u + G0, q = i0 / KG, gb = q % C::NGB;
        const int hs = C::SPAN ? (G0 >> 2) : 0;
        // the group's weight stages are free once the MMAs of the group NGB
        // groups ago retired
        if (q >= C::NGB) ok = ok && mbar_wait_bounded(&gempty[gb], (uint32_t)(((q / C::NGB) - 1) & 1), a.status);
        tc_fence_after();
        const unsigned char* codes = C::SPAN ? ubase + j * C::TILE + hs * C::HALF_A : ubase + j * (C::HALF_A + 512);
        const unsigned char* sbp = C::SPAN ? ubase + j * C::TILE + C::TA : ubase + j * (C::HALF_A + 512) + C::HALF_A;
        const int hsg = C::SPAN ? hs : (u & 1);  // half-span of the scale/bias block
        // scale/bias pairs of rows g (x, z) and g+8 (y, w) for groups (0,1) and (2,3) of the half-span
        const uint4 sb01 = *reinterpret_cast<const uint4*>(sbp + hsg * 256 + (g * 2) * 16);
        const uint4 sb23 = *reinterpret_cast<const uint4*>(sbp + hsg * 256 + (g * 2 + 1) * 16);
        const uint32_t sp01 = isb ? sb01.y : sb01.x, bp01 = isb ? sb01.w : sb01.z;
        const uint32_t sp23 = isb ? sb23.y : sb23.x, bp23 = isb ? sb23.w : sb23.z;
        uint4 w4[KG], w4b[KG];
#pragma unroll
        for (int gg = 0; gg < KG; ++gg) {
          const int G = (G0 & 3) + gg;  // group of the half-span
          const int lane_f = 4 * g + G;
          if (BITS == 4) {
            w4[gg] = *reinterpret_cast<const uint4*>(codes + qd * 512 + lane_f * 16);
          } else {
            w4[gg] = *reinterpret_cast<const uint4*>(codes + (2 * qd) * 512 + lane_f * 16);
            w4b[gg] = *reinterpret_cast<const uint4*>(codes + (2 * qd + 1) * 512 + lane_f * 16);
          }
        }
        const int sel = isb ? 8 : 0;  // row b: nibbles 2/3/6/7 (int4), bytes 1/3 (int8)
#pragma unroll
        for (int gg = 0; gg < KG; ++gg) {
          const int G = (G0 & 3) + gg;
          const uint32_t spair = G < 2 ? sp01 : sp23, bpair = G < 2 ? bp01 : bp23;
          const uint32_t sc = (G & 1) ? (spair >> 16) : (spair & 0xFFFFu);
          const uint32_t bi = (G & 1) ? (bpair >> 16) : (bpair & 0xFFFFu);
          const uint32_t s2 = sc | (sc << 16), b2 = bi | (bi << 16);
          const uint32_t wv[4] = {w4[gg].x, w4[gg].y, w4[gg].z, w4[gg].w};
          uint32_t v[8];
          if (BITS == 4) {
#pragma unroll
            for (int x = 0; x < 4; ++x) {  // word x: codes k .. k+3, k = 16 qd + 4x
              v[2 * x] = bf16x2_fma(bf16x2_sub(lop3_and_or(wv[x] >> sel, 0x000F000Fu, 0x43004300u), 0x43004300u),
                                    s2, b2);
              v[2 * x + 1] = bf16x2_fma(
                  bf16x2_sub(lop3_and_or(wv[x] >> (sel + 4), 0x000F000Fu, 0x43004300u), 0x43004300u), s2, b2);
            }
          } else {
            const uint32_t wb[4] = {w4b[gg].x, w4b[gg].y, w4b[gg].z, w4b[gg].w};
#pragma unroll
            for (int x = 0; x < 4; ++x) {
              v[2 * x] = bf16x2_fma(bytes02_bf16(wv[x] >> sel), s2, b2);
              v[2 * x + 1] = bf16x2_fma(bytes02_bf16(wb[x] >> sel), s2, b2);
            }
          }
          tmem_st8(tbase + 32 * ((i0 + gg) % C::NS), v);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&gfull[gb]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&cempty[c]);
    }
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // every copy issued has landed before the ring is reused or the CTA exits
    const int ix = *issued_x, ic = *issued_c;
    for (int q = ix > C::NGB ? ix - C::NGB : 0; q < ix; ++q)
      mbar_wait_bounded(&gfull[q % C::NGB], (uint32_t)((q / C::NGB) & 1), a.status);
    for (int u = ic > C::NCB ? ic - C::NCB : 0; u < ic; ++u)
      mbar_wait_bounded(&cfull[u % C::NCB], (uint32_t)((u / C::NCB) & 1), a.status);
  }
  // ---- epilogue (warps 3-18): warp (lane quarter lq, part p) takes the
  //      owned 32-token chunks with local index % 4 == p
  const bool epi = warp >= 3;
  const int lq = warp & 3, part = (warp - 3) >> 2;
  const uint32_t tl = tmem + ((uint32_t)(32 * lq) << 16);
  constexpr int NCH = NT / 32;
  const int me = (int)blockIdx.z, ks = (int)gridDim.z;
  const int maxlc = (NCH + ks - 1) / ks;
  bool okd = true;
  if (epi) {
    okd = mbar_wait_bounded(done, 0u, a.status);
    tc_fence_after();
  }
  if (ks > 1) {
    __syncthreads();
    cluster_sync_all();  // every CTA of the cluster is past its main loop
    if (epi) {
      const uint32_t base = smem_u32(smem);
      const int row = 32 * lq + lane;
#pragma unroll 1
      for (int oc = part; oc < NCH; oc += 4) {
        const int owner = oc % ks;
        if (owner == me) continue;
        const int slot = me < owner ? me : me - 1;
        uint32_t v[32];
        tmem_ld32(tl + oc * 32, v);
        tmem_wait_ld();
        const uint32_t dst = map_rank(base + (uint32_t)(((slot * maxlc + oc / ks) * 8 * BM + row) * 16), (uint32_t)owner);
#pragma unroll
        for (int un = 0; un < 8; ++un)
          st_cluster_v4(dst + un * BM * 16, make_uint4(v[4 * un], v[4 * un + 1], v[4 * un + 2], v[4 * un + 3]));
      }
    }
    cluster_sync_all();  // every partial has landed
  }
  if (epi) {
    const int row = 32 * lq + lane;
    const int n = EPI == kTcSwiglu ? 16 * (4 * nt + lq) + (lane & 15) : 128 * nt + row;
#pragma unroll 1
    for (int lc = part; lc < maxlc; lc += 4) {
      const int oc = me + lc * ks;
      if (oc >= NCH) break;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float v[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = 0.f;
#pragma unroll 1
        for (int r = 0; r < ks; ++r) {  // split order
          if (r == me) {
            uint32_t u[16];
            tmem_ld16(tl + oc * 32 + h * 16, u);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] += __uint_as_float(u[t]);
          } else {
            const int slot = r < me ? r : r - 1;
            const unsigned char* src = smem + ((slot * maxlc + lc) * 8 * BM + row) * 16;
#pragma unroll
            for (int un = 0; un < 4; ++un) {
              const float4 f = *reinterpret_cast<const float4*>(src + (4 * h + un) * BM * 16);
              v[4 * un] += f.x, v[4 * un + 1] += f.y, v[4 * un + 2] += f.z, v[4 * un + 3] += f.w;
            }
          }
        }
        w_store16<EPI>(a, n, m0 + oc * 32 + h * 16, mend, lane, v, okd);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
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

// Most CTA clusters of `ks` CTAs of the kernel that can be resident at once
// (0: none), cached per split count.
template <int BITS, int BN, int EPI>
int q_active_clusters(int ks) {
  static int cache[kMaxSplits + 1] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[ks]) return cache[ks] > 0 ? cache[ks] : 0;
  auto kern = tc_qgemm_kernel<BITS, BN, EPI>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, ks);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = QCfg<BITS, BN>::SMEM;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)ks;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (void*)kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[ks] = n > 0 ? n : -1;
  return n;
}

// Splits of K for `tiles` output tiles: the most (up to the portable cluster
// size, two k-blocks per split at least, the owners' receive buffers within
// the ring) whose clusters all fit on the machine at once.
template <int BITS, int BN, int EPI>
int q_pick_splits(long long tiles, int nk, int num_sms) {
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;
  int ks = (int)std::min<long long>(std::min<long long>(kMaxSplits, std::max<long long>(1, num_sms / tiles)),
                                    std::max(1, nk / 2));
  for (; ks > 1; --ks) {
    if (q_recv_bytes(NOUT, EPI, ks) > QCfg<BITS, BN>::RING) continue;
    if (tiles <= (long long)q_active_clusters<BITS, BN, EPI>(ks)) break;
  }
  return ks;
}

template <int BITS, int BN, int EPI>
cudaError_t launch_q(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  CUtensorMap ta, tq;
  cudaError_t e = encode_2d(&ta, a.x, (uint64_t)a.K, (uint64_t)a.M, BM);
  if (e != cudaSuccess) return e;
  const uint64_t wrows = EPI == kTcSwiglu ? 2ull * a.N : (uint64_t)a.N;
  constexpr uint32_t WPB = BK * BITS / 32;
  e = encode_codes(&tq, a.wq, (uint64_t)a.K * BITS / 32, wrows, WPB, EPI == kTcSwiglu ? BN / 2 : BN);
  if (e != cudaSuccess) return e;
  auto kern = tc_qgemm_kernel<BITS, BN, EPI>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, QCfg<BITS, BN>::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  constexpr int NOUT = EPI == kTcSwiglu ? BN / 2 : BN;
  const long long tiles = (long long)((a.M + BM - 1) / BM) * ((a.N + NOUT - 1) / NOUT);
  const int ks = q_pick_splits<BITS, BN, EPI>(tiles, a.K / BK, num_sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.M + BM - 1) / BM, (a.N + NOUT - 1) / NOUT, ks);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = QCfg<BITS, BN>::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)ks;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ta, tq, a);
}

template <int BITS, int EPI, int NT>
int p_active_clusters(int ks) {
  static int cache[kMaxSplits + 1] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[ks]) return cache[ks] > 0 ? cache[ks] : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, ks);
  cfg.blockDim = dim3(kWThreads);
  cfg.dynamicSmemBytes = WCfg<BITS, NT>::SMEM;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)ks;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (void*)tc_pgemm_kernel<BITS, EPI, NT>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[ks] = n > 0 ? n : -1;
  return n;
}

// Splits of the S spans: the most that divide S evenly (up to the portable
// cluster size) whose clusters all fit on the machine at once with the
// owners' receive buffers inside the x ring.
template <int BITS, int EPI, int NT>
int p_pick_splits(long long tiles, int S, int num_sms) {
  int best = 1;
  for (int ks = 2; ks <= std::min(kMaxSplits, S); ++ks) {
    if (S % ks != 0 || tiles * ks > num_sms) continue;
    if (q_recv_bytes(NT, kTcStore, ks) > WCfg<BITS, NT>::RING) continue;
    if (tiles > (long long)p_active_clusters<BITS, EPI, NT>(ks)) continue;
    best = ks;
  }
  return best;
}

template <int BITS, int EPI, int NT>
cudaError_t launch_p(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  using C = WCfg<BITS, NT>;
  CUtensorMap tx;
  cudaError_t e = encode_2d(&tx, a.x, (uint64_t)a.K, (uint64_t)a.M, BM);
  if (e != cudaSuccess) return e;
  auto kern = tc_pgemm_kernel<BITS, EPI, NT>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int mt = (a.M + NT - 1) / NT, ntl = (a.nrb + 7) / 8;
  const int ks = p_pick_splits<BITS, EPI, NT>((long long)mt * ntl, a.S, num_sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(mt, ntl, ks);
  cfg.blockDim = dim3(kWThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = (unsigned)ks;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tx, a);
}

// Tokens per CTA: 128 for short prompts, 256 once that still fills the SMs.
template <int BITS, int EPI>
cudaError_t launch_pn(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  const long long tiles256 = (long long)((a.M + 255) / 256) * ((a.nrb + 7) / 8);
  if (a.M > 128 && tiles256 >= num_sms) return launch_p<BITS, EPI, 256>(a, num_sms, st);
  return launch_p<BITS, EPI, 128>(a, num_sms, st);
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

cudaError_t tc_qgemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  if (!tc_qgemm_supported(a)) return cudaErrorInvalidValue;
  const int mt = (a.M + BM - 1) / BM;
  const bool wide = a.N % 256 == 0 && (long long)mt * (a.N / 256) >= num_sms;
#define EMX_Q(B)                                                                                                 \
  switch (a.epi) {                                                                                               \
    case kTcStore: return wide ? launch_q<B, 256, kTcStore>(a, num_sms, st) : launch_q<B, 128, kTcStore>(a, num_sms, st); \
    case kTcResid: return wide ? launch_q<B, 256, kTcResid>(a, num_sms, st) : launch_q<B, 128, kTcResid>(a, num_sms, st); \
    case kTcF32: return wide ? launch_q<B, 256, kTcF32>(a, num_sms, st) : launch_q<B, 128, kTcF32>(a, num_sms, st);       \
    case kTcSwiglu: return launch_q<B, 256, kTcSwiglu>(a, num_sms, st);                                          \
    default: return cudaErrorInvalidValue;                                                                       \
  }
  if (a.bits == 4) {
    EMX_Q(4)
  }
  EMX_Q(8)
#undef EMX_Q
}

template <int BITS, int EPI>
cudaError_t launch_pg(const TcGemmArgs& a, int max_tiles, cudaStream_t st) {
  using C = WCfg<BITS, 128>;
  CUtensorMap tx;
  cudaError_t e = encode_2d(&tx, a.x, (uint64_t)a.K, (uint64_t)a.M, BM);
  if (e != cudaSuccess) return e;
  auto kern = tc_pgemm_kernel<BITS, EPI, 128>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(max_tiles, (a.nrb + 7) / 8, 1);
  cfg.blockDim = dim3(kWThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tx, a);
}

bool tc_pgemm_supported(const TcGemmArgs& a) {
  if (a.M <= 0 || a.K <= 0 || a.N <= 0 || a.nrb <= 0 || a.S <= 0) return false;
  if (a.K % BK != 0 || a.N % 16 != 0 || !(a.bits == 4 || a.bits == 8) || !a.wp) return false;
  if (a.S != (a.K / BK + 7) / 8) return false;
  if (a.epi != kTcSwiglu && a.nrb * 16 < a.N) return false;
  if (a.epi == kTcSwiglu && a.nrb * 8 < a.N) return false;
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.wp)) & 15) return false;
  return true;
}

cudaError_t tc_pgemm_launch(const TcGemmArgs& a, int num_sms, cudaStream_t st) {
  if (!tc_pgemm_supported(a)) return cudaErrorInvalidValue;
#define EMX_P(B)                                                      \
  switch (a.epi) {                                                    \
    case kTcStore: return launch_pn<B, kTcStore>(a, num_sms, st);     \
    case kTcResid: return launch_pn<B, kTcResid>(a, num_sms, st);     \
    case kTcF32: return launch_pn<B, kTcF32>(a, num_sms, st);         \
    case kTcSwiglu: return launch_pn<B, kTcSwiglu>(a, num_sms, st);   \
    default: return cudaErrorInvalidValue;                            \
  }
  if (a.bits == 4) {
    EMX_P(4)
  }
  EMX_P(8)
#undef EMX_P
}

cudaError_t tc_pgemm_grouped_launch(const TcGemmArgs& a, int max_tiles, cudaStream_t st) {
  if (!tc_pgemm_supported(a) || !a.tiles || !a.n_tiles || max_tiles <= 0) return cudaErrorInvalidValue;
  if (a.expert_stride % 16 != 0) return cudaErrorInvalidValue;
  if (a.bits == 4) {
    switch (a.epi) {
      case kTcStore: return launch_pg<4, kTcStore>(a, max_tiles, st);
      case kTcSwiglu: return launch_pg<4, kTcSwiglu>(a, max_tiles, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (a.epi) {
    case kTcStore: return launch_pg<8, kTcStore>(a, max_tiles, st);
    case kTcSwiglu: return launch_pg<8, kTcSwiglu>(a, max_tiles, st);
    default: return cudaErrorInvalidValue;
  }
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
