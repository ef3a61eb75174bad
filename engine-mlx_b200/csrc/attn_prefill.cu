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
  const bf16* K = a.kc + ((size_t)kvh * a.cap + a.offset) * kD;
  const bf16* V = a.vc + ((size_t)kvh * a.cap + a.offset) * kD;

  // load Q tile
  for (int i = tid; i < kBM * 16; i += kThreads) {
    const int r = i >> 4, c = i & 15;
    cp_async16(sQ + swz(r, c), Q + (size_t)min(q0 + r, T - 1) * kD + c * 8, q0 + r < T);
  }
  auto load_kv = [&](int kt, int buf) {
    const int k0 = kt * kBN;
    for (int i = tid; i < kBN * 16; i += kThreads) {
      const int r = i >> 4, c = i & 15;
      const bool ok = k0 + r < T;
      const size_t row = (size_t)min(k0 + r, T - 1) * kD + c * 8;
      cp_async16(sK + buf * kBN * kD + swz(r, c), K + row, ok);
      cp_async16(sV + buf * kBN * kD + swz(r, c), V + row, ok);
    }
  };
  const int last_q = min(q0 + kBM, T) - 1;
  const int n_kt = last_q / kBN + 1;
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
        if (col > row || col >= T) v = -INFINITY;
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

}  // namespace

cudaError_t attn_prefill_launch(const AttnPrefillArgs& a, cudaStream_t st) {
  if (a.head_dim != kD || a.nkv <= 0 || a.nq % a.nkv) return cudaErrorInvalidValue;
  if (a.T <= 0) return cudaSuccess;
  const int smem = (kBM + 4 * kBN) * kD * 2;
  cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.T + kBM - 1) / kBM, a.nq);
  attn_prefill_kernel<<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace emx
