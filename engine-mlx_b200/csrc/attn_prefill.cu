// attn_prefill.cu — causal GQA attention over the prompt rows (prefill).
//
// Replaces sdpa(q, k, v, scale, causal=true) of the prefill chain
// (crates/serve/src/forward_qwen3.rs:150 via crates/mlx-ffi/src/ops/real/blas.rs:82-97):
// queries are the T prompt rows, keys/values the same T rows (the rows this
// prefill just wrote to the static cache at [offset, offset+T)).
//
// Flash-attention structure: one CTA per (64-query tile, q head), four warps
// of 16 query rows; K/V tiles of 64 rows stream through swizzled shared
// memory with cp.async double buffering; S = Q.K^T and O += P.V run on
// m16n8k16 tensor-core fragments with the online softmax kept in registers.
#include "attn_prefill.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace emx {

namespace {

constexpr int kD = 128;
constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kThreads = 128;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// [rows][128] bf16 tile, 16-byte chunk c of row r stored at chunk c ^ (r & 7).
__device__ __forceinline__ int swz(int r, int c) { return r * kD + ((c ^ (r & 7)) << 3); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(kThreads) attn_prefill_kernel(const AttnPrefillArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem);        // [64][128]
  bf16* sK = sQ + kBM * kD;                        // [2][64][128]
  bf16* sV = sK + 2 * kBN * kD;                    // [2][64][128]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qt = blockIdx.x, h = blockIdx.y;
  const int kvh = h / (a.nq / a.nkv);
  const int q0 = qt * kBM;
  const int T = a.T;
  const bf16* Q = a.q + ((size_t)h * T) * kD;
  const int P = a.prefix, L = P + T;  // keys: P cached rows, then the chunk
  const bf16* K = a.kc + ((size_t)kvh * a.cap + a.offset - P) * kD;
  const bf16* V = a.vc + ((size_t)kvh * a.cap + a.offset - P) * kD;

  // load Q tile
  for (int i = tid; i < kBM * 16; i += kThreads) {
    const int r = i >> 4, c = i & 15;
    cp_async16(sQ + swz(r, c), Q + (size_t)min(q0 + r, T - 1) * kD + c * 8, q0 + r < T);
  }
  auto load_kv = [&](int kt, int buf) {
    const int k0 = kt * kBN;
    for (int i = tid; i < kBN * 16; i += kThreads) {
      const int r = i >> 4, c = i & 15;
      const bool ok = k0 + r < L;
      const size_t row = (size_t)min(k0 + r, L - 1) * kD + c * 8;
      cp_async16(sK + buf * kBN * kD + swz(r, c), K + row, ok);
      cp_async16(sV + buf * kBN * kD + swz(r, c), V + row, ok);
    }
  };
  const int last_q = min(q0 + kBM, T) - 1;
  const int n_kt = (last_q + P) / kBN + 1;
  load_kv(0, 0);
  cp_async_commit();

  const float sl2 = a.scale * 1.4426950408889634f;  // scale * log2(e)
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[8][4];
  const int g = lane >> 2, tig = lane & 3;
  const int row_a = q0 + warp * 16 + g, row_b = row_a + 8;

  for (int kt = 0; kt < n_kt; ++kt) {
    if (kt + 1 < n_kt) load_kv(kt + 1, (kt + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kt == 0) {
      // Q fragments for this warp's 16 rows, 8 k-steps of 16
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldmatrix_x4(qf[ks], sQ + swz(r, c));
      }
    }
    const bf16* cK = sK + (kt & 1) * kBN * kD;
    const bf16* cV = sV + (kt & 1) * kBN * kD;
    // S = Q K^T : 16 x 64 per warp
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int nb = 0; nb < 4; ++nb) {  // pairs of n8 tiles
        uint32_t kf[4];
        const int r = nb * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(kf, cK + swz(r, c));
        mma_bf16_16816(s[2 * nb], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], kf[0], kf[1]);
        mma_bf16_16816(s[2 * nb + 1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], kf[2], kf[3]);
      }
    }
    // causal mask + online softmax (rows row_a, row_b)
    const int k0 = kt * kBN;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = k0 + nt * 8 + tig * 2 + (e & 1);
        const int row = (e < 2) ? row_a : row_b;
        float v = s[nt][e] * sl2;
        if (col > row + P || col >= L) v = -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      alpha[i] = (m_r[i] == -INFINITY) ? 0.f : exp2f(m_r[i] - mx[i]);
      m_r[i] = mx[i];
    }
    // P as A fragments (4 k-steps of 16 keys), split into bf16 hi + lo parts
    // so that P.V keeps ~16 significant bits of each probability.
    uint32_t pf[4][4], pl[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float p[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        p[e] = (mm == -INFINITY) ? 0.f : exp2f(s[nt][e] - mm);
        rs[e >> 1] += p[e];
        lo[e] = p[e] - bfround(p[e]);
      }
      const int ks = nt >> 1, hi = nt & 1;
      pf[ks][hi * 2 + 0] = pack_bf16(p[0], p[1]);
      pf[ks][hi * 2 + 1] = pack_bf16(p[2], p[3]);
      pl[ks][hi * 2 + 0] = pack_bf16(lo[0], lo[1]);
      pl[ks][hi * 2 + 1] = pack_bf16(lo[2], lo[3]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
      l_r[i] = l_r[i] * alpha[i] + rs[i];
    }
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }
    // O += P V : P 16 x 64 (A), V 64 x 128 (B via ldmatrix.trans)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t a0 = pf[ks][0], a1 = pf[ks][1], a2 = pf[ks][2], a3 = pf[ks][3];
#pragma unroll
      for (int db = 0; db < 8; ++db) {  // pairs of n8 tiles over head dims
        uint32_t vf[4];
        const int r = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = db * 2 + (lane >> 4);
        ldmatrix_x4_trans(vf, cV + swz(r, c));
        // A regs order: a0 (row g, k 0-7), a1 (row g+8, k 0-7), a2 (row g, k 8-15), a3 (row g+8, k 8-15)
        mma_bf16_16816(o[2 * db], a0, a1, a2, a3, vf[0], vf[1]);
        mma_bf16_16816(o[2 * db + 1], a0, a1, a2, a3, vf[2], vf[3]);
        mma_bf16_16816(o[2 * db], pl[ks][0], pl[ks][1], pl[ks][2], pl[ks][3], vf[0], vf[1]);
        mma_bf16_16816(o[2 * db + 1], pl[ks][0], pl[ks][1], pl[ks][2], pl[ks][3], vf[2], vf[3]);
      }
    }
    __syncthreads();
  }
  // normalise and store O[t, h*128 + d]
  const float inv_a = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv_b = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + tig * 2;
    if (row_a < T) {
      bf16* dst = a.out + (a.out_tnd ? (size_t)row_a * a.nq * kD + (size_t)h * kD : ((size_t)h * T + row_a) * kD) + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16(o[nt][0] * inv_a, o[nt][1] * inv_a);
    }
    if (row_b < T) {
      bf16* dst = a.out + (a.out_tnd ? (size_t)row_b * a.nq * kD + (size_t)h * kD : ((size_t)h * T + row_b) * kD) + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16(o[nt][2] * inv_b, o[nt][3] * inv_b);
    }
  }
}

// ---------------------------------------------------------------------------
// tcgen05 flash attention: one CTA per (128-query tile, q head), ten warps.
//   warp 0 (one thread)  TMA: the Q tile once, then K and V tiles of 128 keys
//                        into a two-stage ring (128-byte swizzle, 3-D tensor
//                        maps whose row extent is T: rows past the prompt
//                        read as zeros);
//   warp 1 (one thread)  MMA: S_j = Q.K_j^T (M = N = 128, eight K = 16
//                        steps) into one of two tensor-memory S buffers,
//                        issued before O += P_{j-1}.V_{j-1} so that the tensor
//                        pipe computes the next scores while the softmax
//                        warps work; P is operand A straight from tensor
//                        memory (it overwrites its own tile's S), V an
//                        MN-major operand; owns the 512-column TMEM
//                        allocation;
//   warps 2-9            softmax: two threads per query row (warps w and w+4
//                        share a TMEM lane quadrant), each with 64 of the 128
//                        columns; it reads its S half-row with tcgen05.ld,
//                        masks (the diagonal tile only), keeps the running max in
//                        the log2 domain and writes P as bf16 hi + lo parts
//                        (P.V keeps ~16 significant bits of each
//                        probability) over the S buffer it just read, so
//                        the two S buffers double-buffer P as well: tile
//                        j's exponentials run while O += P_{j-1}.V_{j-1}
//                        does (the MMAs execute in issue order, so S_{j+2}
//                        lands in that buffer only after P_j was read).
//                        The max used for the
//                        exponentials only moves when the tile max exceeds it
//                        by more than 8 (O and l are then rescaled in place),
//                        so P <= 2^8 and the final O / l is exact whatever
//                        max was used.
constexpr int kTBM = 128, kTBN = 128;
constexpr int kTcThreads = 320;
constexpr int kBlk = kTBM * 64 * 2;  // 128 rows x 64 columns (128 B rows, swizzled): 16 KB
constexpr int kTileB = 2 * kBlk;     // 128 rows x 128 columns
constexpr int kOffK = kTileB;        // Q | (K V) x 2 | barriers
constexpr int kOffBar = kOffK + 4 * kTileB;
constexpr int kOffX = kOffBar + 128;  // softmax exchange: [2 halves][128 rows] floats
constexpr int kTcSmem = 1024 + kOffX + 2 * kTBM * 4;
constexpr float kRescale = 8.0f;     // log2 growth allowed before O is rescaled
constexpr uint32_t kTmemCols = 512;  // S0 [0,128), O [128,256), S1 [256,384); P_j over S_{j&1}: hi [0,64), lo [64,128)

__device__ __forceinline__ uint64_t desc_kmajor(const void* p) {
  const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// MN-major operand with 128-byte swizzle: 64-element MN blocks kBlk bytes
// apart (LBO), 8-row K groups 1024 bytes apart (SBO).
__device__ __forceinline__ uint64_t desc_mnmajor(const void* p) {
  const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
  return a | ((uint64_t)(kBlk >> 4) << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16, D fp32, A/B bf16, M = N = 128; A K-major; B K-major or MN-major.
constexpr uint32_t idesc_128(bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(128 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// The same with operand A in tensor memory (lane = row, two bf16 of K per column).
__device__ __forceinline__ void umma_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tfence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tfence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tst32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tst32u(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 2^x by the hardware's base-2 exponential (softmax weights; their bf16
// hi + lo split keeps ~16 bits, well inside its accuracy).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_wait_ld_() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st_() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kTcThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, const AttnPrefillArgs a, int* status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* sQ = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;   // [2] per K/V stage
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* s_full = bar + 5;    // [2] per S buffer
  uint64_t* s_free = bar + 7;    // [2]
  uint64_t* p_full = bar + 9;
  uint64_t* pv_done = bar + 11;
  uint64_t* o_done = bar + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 13);
  int* issued_slot = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // the longest rows first
  const int h = blockIdx.y;
  const int kvh = h / (a.nq / a.nkv);
  // key tiles at or before the diagonal: the cached prefix (whole tiles)
  // first, then the chunk's own rows
  const int nt = qt + 1 + a.prefix / kTBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 256);
    }
    mbar_init(p_full, 256);
    mbar_init(pv_done, 1);
    mbar_init(o_done, 1);
    *issued_slot = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tfence_before();
  __syncthreads();
  tfence_after();
  const uint32_t tmem = *tmem_slot;
  auto s_col = [](int b) -> uint32_t { return b ? 256u : 0u; };

  if (warp == 0 && lane == 0) {
    // ---- TMA producer
    mbar_arrive_expect_tx(q_full, (uint32_t)kTileB);
    tma_load_3d(sQ, &tq, 0, qt * kTBM, h, q_full);
    tma_load_3d(sQ + kBlk, &tq, 64, qt * kTBM, h, q_full);
    int issued = 0;
    for (int j = 0; j < nt; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait_bounded(&kv_empty[s], (uint32_t)(((j >> 1) - 1) & 1), status)) break;
      unsigned char* K = smem + kOffK + s * 2 * kTileB;
      unsigned char* V = K + kTileB;
      mbar_arrive_expect_tx(&kv_full[s], (uint32_t)(2 * kTileB));
      tma_load_3d(K, &tk, 0, j * kTBN, kvh, &kv_full[s]);
      tma_load_3d(K + kBlk, &tk, 64, j * kTBN, kvh, &kv_full[s]);
      tma_load_3d(V, &tv, 0, j * kTBN, kvh, &kv_full[s]);
      tma_load_3d(V + kBlk, &tv, 64, j * kTBN, kvh, &kv_full[s]);
      issued = j + 1;
    }
    *issued_slot = issued;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: S_0, then per tile j: S_{j+1} (if any), O += P_j.V_j
    constexpr uint32_t id_s = idesc_128(false), id_pv = idesc_128(true);
    auto issue_s = [&](int j) -> bool {
      const int b = j & 1;
      if (!mbar_wait_bounded(&kv_full[b], (uint32_t)((j >> 1) & 1), status)) return false;
      if (j >= 2 && !mbar_wait_bounded(&s_free[b], (uint32_t)(((j >> 1) - 1) & 1), status)) return false;
      tfence_after();
      const unsigned char* K = smem + kOffK + b * 2 * kTileB;
#pragma unroll
      for (int k = 0; k < 8; ++k)  // 16 head dims per step: block k/4, +32 B per step inside it
        umma(tmem + s_col(b), desc_kmajor(sQ + (k >> 2) * kBlk) + 2 * (k & 3),
             desc_kmajor(K + (k >> 2) * kBlk) + 2 * (k & 3), id_s, k > 0 ? 1u : 0u);
      umma_commit(&s_full[b]);
      return true;
    };
    bool ok = mbar_wait_bounded(q_full, 0u, status) && issue_s(0);
    for (int j = 0; ok && j < nt; ++j) {
      if (j + 1 < nt && !issue_s(j + 1)) break;
      const int b = j & 1;
      if (!mbar_wait_bounded(p_full, (uint32_t)(j & 1), status)) break;
      tfence_after();
      const unsigned char* V = smem + kOffK + b * 2 * kTileB + kTileB;
#pragma unroll
      for (int part = 0; part < 2; ++part) {  // P hi, then P lo, in S buffer b
#pragma unroll
        for (int k = 0; k < 8; ++k)  // 16 keys per step: 8 P columns, V rows 16k.. (+2 KB)
          umma_ta(tmem + 128, tmem + s_col(b) + (uint32_t)(part * 64 + k * 8), desc_mnmajor(V + k * 2048), id_pv,
                  (j > 0 || part > 0 || k > 0) ? 1u : 0u);
      }
      umma_commit(&kv_empty[b]);
      umma_commit(pv_done);
    }
    umma_commit(o_done);
  } else if (warp >= 2) {
    // ---- softmax: query row r of the tile, key (and output) columns
    //      [64 hf, 64 hf + 64); the two threads of a row meet at a named
    //      barrier of their two warps to combine the tile max
    const int quad = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int qrow = qt * kTBM + r;
    const bool valid_q = qrow < a.T;
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(hf * 64);
    const uint32_t tO = tl + 128;
    const float sl2 = a.scale * 1.4426950408889634f;
    float* xch = reinterpret_cast<float*>(smem + kOffX);  // [half][row]
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory"); };
    // barrier of the pair that also ANDs a flag over its 64 threads: both
    // threads of a row leave the tile loop together (a lone thread left at a
    // named barrier would wait for ever)
    auto pair_all = [&](bool v) -> bool {
      uint32_t res;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 64, p;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(res)
          : "r"((uint32_t)v), "r"(1 + quad)
          : "memory");
      return res != 0;
    };
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1;
      ok = mbar_wait_bounded(&s_full[b], (uint32_t)((j >> 1) & 1), status) && ok;
      tfence_after();
      float s[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tld32(tl + s_col(b) + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = v[i];
      }
      tmem_wait_ld_();
      tfence_before();
      mbar_arrive(&s_free[b]);
      const int kv0 = j * kTBN + hf * 64;
      float mx = -INFINITY;
      if (j + 1 < nt) {  // below the diagonal every key is visible
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          s[c] = valid_q ? s[c] * sl2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const bool vis = valid_q && kv0 + c <= qrow + a.prefix;
          s[c] = vis ? s[c] * sl2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      }
      xch[hf * kTBM + r] = mx;
      if (!pair_all(ok)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, xch[(hf ^ 1) * kTBM + r]);
      pair_sync();  // both read before either writes the next tile's max (and both S halves are out)
      if (mx != -INFINITY && mx > m_used + kRescale) {
        const float alpha = m_used == -INFINITY ? 0.f : ex2_approx(m_used - mx);
        if (j > 0 && m_used != -INFINITY) {
          // the O update of tile j-1 has written O before it is rescaled
          ok = mbar_wait_bounded(pv_done, (uint32_t)((j - 1) & 1), status) && ok;
          tfence_after();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float v[32];
            tld32(tO + c * 32, v);
            tmem_wait_ld_();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tst32(tO + c * 32, v);
          }
          tmem_wait_st_();
        }
        l *= alpha;
        m_used = mx;
      }
      // P = exp2(s - m_used) as bf16 hi + lo over this tile's S buffer: keys
      // [64 hf, 64 hf + 64) of row r in columns 32 hf.. (hi) and 64 + 32 hf..
      // (lo), two keys per column
      {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = 2 * e;
          const float p0 = s[c] == -INFINITY ? 0.f : ex2_approx(s[c] - m_used);
          const float p1 = s[c + 1] == -INFINITY ? 0.f : ex2_approx(s[c + 1] - m_used);
          l += p0;
          l += p1;
          const float h0 = bfround(p0), h1 = bfround(p1);
          hi[e] = pack_bf16(h0, h1);
          lo[e] = pack_bf16(p0 - h0, p1 - h1);
        }
        const uint32_t tp = tmem + ((uint32_t)(quad * 32) << 16) + s_col(b) + (uint32_t)(hf * 32);
        tst32u(tp, hi);
        tst32u(tp + 64, lo);
        tmem_wait_st_();
      }
      // O += P_{j-1}.V_{j-1} has finished (it is normally done by now): one
      // completion of pv_done per tile keeps its phases in step
      if (j > 0) ok = mbar_wait_bounded(pv_done, (uint32_t)((j - 1) & 1), status) && ok;
      tfence_before();
      mbar_arrive(p_full);
    }
    // ---- O / l (the two halves' sums combined), stored as bf16
    xch[hf * kTBM + r] = l;
    pair_sync();
    const float lt = l + xch[(hf ^ 1) * kTBM + r];
    const bool okd = mbar_wait_bounded(o_done, 0u, status);
    tfence_after();
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float v[32];
      tld32(tO + c * 32, v);
      tmem_wait_ld_();
      if (!ok || !okd || !valid_q) continue;
      bf16* dst = a.out + (a.out_tnd ? (size_t)qrow * a.nq * kD + (size_t)h * kD : ((size_t)h * a.T + qrow) * kD) +
                  hf * 64 + c * 32;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        reinterpret_cast<uint4*>(dst)[q4] = make_uint4(
            pack_bf16(v[8 * q4 + 0] * inv, v[8 * q4 + 1] * inv), pack_bf16(v[8 * q4 + 2] * inv, v[8 * q4 + 3] * inv),
            pack_bf16(v[8 * q4 + 4] * inv, v[8 * q4 + 5] * inv), pack_bf16(v[8 * q4 + 6] * inv, v[8 * q4 + 7] * inv));
    }
  }
  tfence_before();
  __syncthreads();
  if (warp == 0 && lane == 0) {
    // the last copies issued into each stage have landed before the CTA exits
    const int issued = *issued_slot;
    mbar_wait_bounded(q_full, 0u, status);
    for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
      mbar_wait_bounded(&kv_full[j & 1], (uint32_t)((j >> 1) & 1), status);
  }
  if (warp == 1) {
    tfence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode3 = nullptr;
std::once_flag g_encode3_once;

// [heads][rows][128] bf16 with `head_stride` bytes between heads; boxes of
// 64 columns x 128 rows of one head, 128-byte swizzle; rows past `rows` read
// as zeros.
cudaError_t encode_rows(CUtensorMap* map, const void* base, uint64_t rows, uint64_t heads, uint64_t head_stride) {
  std::call_once(g_encode3_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode3 = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode3) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {(cuuint64_t)kD, rows, heads};
  const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, head_stride};
  const cuuint32_t box[3] = {64, (cuuint32_t)kTBM, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode3(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

cudaError_t attn_prefill_launch(const AttnPrefillArgs& a, cudaStream_t st, int* status) {
  if (a.head_dim != kD || a.nkv <= 0 || a.nq % a.nkv) return cudaErrorInvalidValue;
  if (a.T <= 0) return cudaSuccess;
  if (a.prefix < 0 || a.prefix > a.offset) return cudaErrorInvalidValue;
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc)) & 15) == 0;
  // the tcgen05 kernel takes a chunk attending itself, or a cached prefix of
  // whole 128-row tiles (then the diagonal tiles stay aligned); other
  // prefixes go through the mma.sync kernel
  if (a.prefix % kTBN == 0 && aligned) {
    CUtensorMap tq, tk, tv;
    const size_t k0 = (size_t)(a.offset - a.prefix) * kD;
    const uint64_t rows = (uint64_t)a.prefix + (uint64_t)a.T;
    cudaError_t e = encode_rows(&tq, a.q, (uint64_t)a.T, (uint64_t)a.nq, (uint64_t)a.T * kD * 2);
    if (e == cudaSuccess) e = encode_rows(&tk, a.kc + k0, rows, (uint64_t)a.nkv, (uint64_t)a.cap * kD * 2);
    if (e == cudaSuccess) e = encode_rows(&tv, a.vc + k0, rows, (uint64_t)a.nkv, (uint64_t)a.cap * kD * 2);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.T + kTBM - 1) / kTBM, a.nq);
    attn_prefill_tc_kernel<<<grid, kTcThreads, kTcSmem, st>>>(tq, tk, tv, a, status);
    return cudaGetLastError();
  }
  const int smem = (kBM + 4 * kBN) * kD * 2;
  cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.T + kBM - 1) / kBM, a.nq);
  attn_prefill_kernel<<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace emx
