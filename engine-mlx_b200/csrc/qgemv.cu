// qgemv.cu — batch-1 quantized GEMV for sm_100a.
//
// One CTA per SM (at most), each owning a contiguous run of 16-row blocks.
// Data path per CTA:
//   1. before griddepcontrol.wait: the bulk-copy engine streams the CTA's
//      packed weight rows and their scale/bias rows into a shared-memory ring
//      (these never depend on the previous kernel, so with PDL they overlap
//      its tail — the batch-1 decode step becomes one continuous HBM stream);
//   2. after the wait: the input vector is built in shared memory (optionally
//      RMS-normalised, gathered from the quantized embedding for layer 0, or
//      summed with a tensor-parallel / MoE partial), stored in the MMA
//      fragment order;
//   3. each warp takes (16-row block x 8-group span) units: packed nibbles /
//      bytes become bf16 through a magic-number LOP3 and an exact bf16x2
//      subtract, and m16n8k16 tensor-core MMAs compute the per-group dot
//      products — column j of the MMA's B operand carries x masked to group j,
//      so one accumulator tile yields eight group sums at once;
//   4. per row: acc = sum_g ( s*dot_g + b*sum(x_g) ) in fp32 — the MLX qmv
//      factorisation — and a fused epilogue (store / residual add / SwiGLU /
//      greedy argmax / fp32 partial).
// Expert gather (MoE): logical rows come in slots of `slot_rows`; slot s reads
// expert slot_expert[s]'s rows, so the top-k experts' matmuls are one launch.
#include "qgemv.cuh"

#include <algorithm>

namespace emx {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSmemBudget = 110 * 1024;  // two CTAs per SM when possible

struct GemvGeom {
  int K, ng, nspans, kbytes, span_bytes, lrows;
  int swiglu, x_slots;
  // plan
  int rows_round, spans_round, nbuf, nkr;
  int stride;        // smem bytes per weight row in a round buffer
  int groups_round;  // max groups per round
  int buf_bytes;     // bytes per ring slot
  int off_x, off_xs, off_red, off_buf;
};

__host__ __device__ inline int span_k(int gs) { return 8 * gs; }

// Shared-memory carve-up for a given round shape.
__host__ __device__ inline void geom_layout(GemvGeom& g) {
  g.stride = g.spans_round * g.span_bytes + 64;
  g.groups_round = (g.spans_round * 8 < g.ng) ? g.spans_round * 8 : g.ng;
  const int phys = g.rows_round * (g.swiglu ? 2 : 1);
  int sb = phys * g.groups_round * 2;
  sb = (sb + 15) & ~15;
  g.buf_bytes = ((phys * g.stride + 2 * sb) + 127) & ~127;
  g.off_x = 256;
  g.off_xs = g.off_x + ((g.x_slots * g.K * 2 + 15) & ~15);
  g.off_red = g.off_xs + ((g.x_slots * g.ng * 4 + 15) & ~15);
  g.off_buf = (g.off_red + phys * g.nspans * 4 + 127) & ~127;
}

__host__ __device__ inline int geom_smem(const GemvGeom& g) { return g.off_buf + g.nbuf * g.buf_bytes; }

__device__ __forceinline__ int perm_pos(int k, int bits) {
  // MMA fragment order of x inside each 8-element (int4) / 4-element (int8)
  // block: element i sits where the dequantised nibble pairs expect it.
  if (bits == 4) {
    const int i = k & 7;
    return (k & ~7) | (((i & 3) << 1) | (i >> 2));
  }
  const int i = k & 3;
  return (k & ~3) | (((i & 1) << 1) | (i >> 1));
}

// The pre-norm source element k (bf16 value as float).
__device__ __forceinline__ float load_src(const GemvArgs& a, int k, int tok) {
  if (a.pro == kProEmbedNorm) {
    const int per = 32 / a.emb_bits;
    const int ngk = a.K / a.emb_gs;
    const uint32_t word = a.emb_w[(size_t)tok * (a.K / per) + k / per];
    const uint32_t q = (word >> (a.emb_bits * (k % per))) & ((1u << a.emb_bits) - 1u);
    return bf2f(dequant1(q, a.emb_s[(size_t)tok * ngk + k / a.emb_gs], a.emb_b[(size_t)tok * ngk + k / a.emb_gs]));
  }
  if (a.pro == kProAddNorm) {
    float add;
    if (a.moe_y) {
      add = 0.f;
      const int n = *a.moe_n;
      for (int s = 0; s < n; ++s) add = __fadd_rn(add, __fmul_rn(bf2f(a.moe_y[(size_t)s * a.K + k]), a.moe_w[s]));
    } else {
      add = a.add_round ? bfround(a.add_f32[k]) : a.add_f32[k];
    }
    return bfround(__fadd_rn(bf2f(a.x[k]), add));
  }
  return bf2f(a.x[k]);
}

// Physical weight row of logical row L (up == true: the SwiGLU "up" half).
__device__ __forceinline__ int phys_row(const GemvArgs& a, int lrows, int L, bool up) {
  if (a.slot_expert) {
    const int s = L / a.slot_rows, r = L % a.slot_rows;
    const int e = a.slot_expert[s];
    const int per_e = a.slot_rows * (a.epi == kEpiSwiglu ? 2 : 1);
    return e * per_e + r + (up ? a.slot_rows : 0);
  }
  return L + (up ? lrows : 0);
}

template <int BITS, int GS>
__global__ void __launch_bounds__(kThreads, 2) qgemv_kernel(const GemvArgs a, const GemvGeom geo) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem);
  float* scratch = reinterpret_cast<float*>(smem + 64);  // 32 floats
  uint16_t* xp = reinterpret_cast<uint16_t*>(smem + geo.off_x);
  float* xs = reinterpret_cast<float*>(smem + geo.off_xs);
  float* red = reinterpret_cast<float*>(smem + geo.off_red);
  unsigned char* bufs = smem + geo.off_buf;

  constexpr int CHUNK_K = BITS == 4 ? 32 : 16;  // k per 16-byte chunk
  constexpr int SPAN_K = 8 * GS;
  constexpr int CH_SPAN = SPAN_K / CHUNK_K;
  constexpr int J_SPAN = CH_SPAN / 4;
  constexpr int BREG = BITS == 4 ? 16 : 8;  // B-fragment registers per chunk
  constexpr int JP = (J_SPAN * BREG > 64) ? (64 / BREG) : J_SPAN;
  constexpr int NPASS = J_SPAN / JP;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const bool gather = a.slot_expert != nullptr;
  const int rlb = geo.rows_round / 16;
  const int Kb = geo.kbytes;
  const int phys_mult = geo.swiglu ? 2 : 1;

  // Row range of this CTA (known before the wait unless rows come from a
  // device-side slot count).
  int lrows = geo.lrows, lb0 = 0, lb1 = 0, nrounds = 0;
  auto partition = [&]() {
    const int nlb = lrows / 16;
    lb0 = (int)((long long)blockIdx.x * nlb / gridDim.x);
    lb1 = (int)((long long)(blockIdx.x + 1) * nlb / gridDim.x);
    nrounds = ((lb1 - lb0 + rlb - 1) / rlb) * geo.nkr;
  };

  if (tid == 0) {
    for (int i = 0; i < geo.nbuf; ++i) mbar_init(&mbar[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  // ---- one round: weight rows + scale/bias rows into ring slot r % nbuf
  auto issue = [&](int r) {
    const int buf = r % geo.nbuf;
    const int rg = r / geo.nkr, kr = r % geo.nkr;
    const int L0 = (lb0 + rg * rlb) * 16;
    const int nl = min(rlb, lb1 - lb0 - rg * rlb) * 16;
    const int sp0 = kr * geo.spans_round;
    const int sp1 = min(geo.nspans, sp0 + geo.spans_round);
    const int kb0 = sp0 * geo.span_bytes;
    const int kbytes = min((sp1 - sp0) * geo.span_bytes, Kb - kb0);
    const int g0 = sp0 * 8;
    const int Gr = min((sp1 - sp0) * 8, geo.ng - g0);
    const int phys = nl * phys_mult;
    const int sb_bytes = phys * Gr * 2;
    unsigned char* bw = bufs + (size_t)buf * geo.buf_bytes;
    unsigned char* bs = bw + (size_t)phys * geo.stride;
    unsigned char* bb = bs + ((sb_bytes + 15) & ~15);
    mbar_arrive_expect_tx(&mbar[buf], (uint32_t)(phys * kbytes + 2 * sb_bytes));
    const unsigned char* wbase = reinterpret_cast<const unsigned char*>(a.w);
    for (int i = 0; i < phys; ++i) {
      const int src = (i >= nl) ? phys_row(a, lrows, L0 + i - nl, true) : phys_row(a, lrows, L0 + i, false);
      bulk_g2s(bw + (size_t)i * geo.stride, wbase + (size_t)src * Kb + kb0, (uint32_t)kbytes, &mbar[buf]);
    }
    if (Gr == geo.ng) {
      // whole scale/bias rows: one copy per 16-row block (contiguous rows)
      for (int i = 0; i < phys; i += 16) {
        const int src = (i >= nl) ? phys_row(a, lrows, L0 + i - nl, true) : phys_row(a, lrows, L0 + i, false);
        const size_t off = (size_t)src * geo.ng;
        bulk_g2s(bs + (size_t)i * Gr * 2, a.s + off, (uint32_t)(16 * Gr * 2), &mbar[buf]);
        bulk_g2s(bb + (size_t)i * Gr * 2, a.b + off, (uint32_t)(16 * Gr * 2), &mbar[buf]);
      }
    } else {
      for (int i = 0; i < phys; ++i) {
        const int src = (i >= nl) ? phys_row(a, lrows, L0 + i - nl, true) : phys_row(a, lrows, L0 + i, false);
        const size_t off = (size_t)src * geo.ng + g0;
        bulk_g2s(bs + (size_t)i * Gr * 2, a.s + off, (uint32_t)(Gr * 2), &mbar[buf]);
        bulk_g2s(bb + (size_t)i * Gr * 2, a.b + off, (uint32_t)(Gr * 2), &mbar[buf]);
      }
    }
  };

  if (!gather) {
    partition();
    if (tid == 0) {
      const int pre = min(geo.nbuf, nrounds);
      for (int r = 0; r < pre; ++r) issue(r);
    }
  }

  // ---- wait for the producer of x (previous kernel) ---------------------
  pdl_wait();

  if (gather) {
    lrows = min(*a.n_slots * a.slot_rows, geo.lrows);
    partition();
    if (tid == 0) {
      const int pre = min(geo.nbuf, nrounds);
      for (int r = 0; r < pre; ++r) issue(r);
    }
  }

  int tok = 0;
  if (a.pro == kProEmbedNorm) {
    tok = *a.token;
    if (tok < 0 || tok >= a.vocab) {
      if (tid == 0) report_status(a.status, kDevBadToken);
      tok = 0;
    }
  }
  // ---- prologue: x (normalised) into shared memory, fragment order ------
  {
    const int K = geo.K;
    if (a.pro == kProX) {
      for (int i = tid; i < geo.x_slots * K; i += kThreads) {
        const int sl = i / K, k = i % K;
        xp[sl * K + perm_pos(k, BITS)] = *reinterpret_cast<const uint16_t*>(a.x + i);
      }
    } else {
      const int groups = a.norm_groups > 0 ? a.norm_groups : 1;
      const int gd = K / groups;
      const bool store = (a.pro == kProEmbedNorm || a.pro == kProAddNorm) && blockIdx.x == 0 && a.x_out;
      for (int gi = 0; gi < groups; ++gi) {
        float ss = 0.0f;
        for (int k = gi * gd + tid; k < (gi + 1) * gd; k += kThreads) {
          const float v = load_src(a, k, tok);
          ss = fmaf(v, v, ss);
          if (store) a.x_out[k] = f2bf(v);
        }
        ss = block_sum(ss, scratch);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)gd), a.eps)));
        for (int k = gi * gd + tid; k < (gi + 1) * gd; k += kThreads) {
          const float v = load_src(a, k, tok);
          float o;
          if (groups == 1) {
            o = bfround(__fmul_rn(bfround(__fmul_rn(v, inv)), bf2f(a.norm_w[k])));
          } else {
            o = bfround(__fmul_rn(__fmul_rn(v, inv), bf2f(a.norm_w[k])));
          }
          xp[perm_pos(k, BITS)] = f2bits(o);
        }
      }
    }
    __syncthreads();
    for (int i = tid; i < geo.x_slots * geo.ng; i += kThreads) {
      float s = 0.0f;
      const uint16_t* src = xp + (size_t)(i / geo.ng) * K + (i % geo.ng) * GS;
      for (int j = 0; j < GS; ++j) s += bits2f(src[j]);
      xs[i] = s;
    }
    __syncthreads();
  }

  // per-thread argmax state
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;

  const uint32_t MASK = 0x000F000Fu;
  const uint32_t MAGIC_LO = 0x43004300u;  // bf16 128.0 | nibble
  const uint32_t MAGIC_HI = 0x45004500u;  // bf16 2048.0 | nibble  (value 2048 + 16*nibble)

  for (int r = 0; r < nrounds; ++r) {
    const int buf = r % geo.nbuf;
    const int rg = r / geo.nkr, kr = r % geo.nkr;
    const int L0 = (lb0 + rg * rlb) * 16;
    const int nl = min(rlb, lb1 - lb0 - rg * rlb) * 16;
    const int sp0 = kr * geo.spans_round;
    const int sp1 = min(geo.nspans, sp0 + geo.spans_round);
    const int g0 = sp0 * 8;
    const int Gr = min((sp1 - sp0) * 8, geo.ng - g0);
    const int phys = nl * phys_mult;
    const int sb_bytes = phys * Gr * 2;
    const unsigned char* bw = bufs + (size_t)buf * geo.buf_bytes;
    const uint16_t* bsc = reinterpret_cast<const uint16_t*>(bw + (size_t)phys * geo.stride);
    const uint16_t* bbi = reinterpret_cast<const uint16_t*>(bw + (size_t)phys * geo.stride + ((sb_bytes + 15) & ~15));

    const bool ok = mbar_wait_bounded(&mbar[buf], (uint32_t)((r / geo.nbuf) & 1), a.status);
    if (ok) {
      const int nrb = phys / 16;
      const int nspr = sp1 - sp0;
      const int units = nrb * nspr;
      for (int u = warp; u < units; u += kWarps) {
        const int spl = u / nrb, rb = u % nrb;
        const int span = sp0 + spl;
        const int rowA = rb * 16 + g;
        // input slot of this row block (MoE down: one x per expert slot)
        int xsl = 0;
        if (geo.x_slots > 1) {
          const int lr = (rb * 16 < nl) ? rb * 16 : rb * 16 - nl;
          xsl = (L0 + lr) / a.slot_rows;
        }
        const uint16_t* xpv = xp + (size_t)xsl * geo.K;
        const float* xsv = xs + (size_t)xsl * geo.ng;
        const unsigned char* pA = bw + (size_t)rowA * geo.stride + (size_t)spl * geo.span_bytes;
        const unsigned char* pB = pA + (size_t)8 * geo.stride;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int pass = 0; pass < NPASS; ++pass) {
          uint32_t breg[JP][BREG];
#pragma unroll
          for (int jj = 0; jj < JP; ++jj) {
            const int j = pass * JP + jj;
            const int cl = 4 * j + tig;
            const int k0 = span * SPAN_K + cl * CHUNK_K;
            const bool on = ((cl * CHUNK_K) / GS == g) && (k0 < geo.K);
            if (on) {
#pragma unroll
              for (int q = 0; q < BREG / 4; ++q) {
                uint4 v = lds128(xpv + k0 + q * 8);
                breg[jj][q * 4 + 0] = v.x;
                breg[jj][q * 4 + 1] = v.y;
                breg[jj][q * 4 + 2] = v.z;
                breg[jj][q * 4 + 3] = v.w;
              }
            } else {
#pragma unroll
              for (int q = 0; q < BREG; ++q) breg[jj][q] = 0u;
            }
          }
#pragma unroll
          for (int jj = 0; jj < JP; ++jj) {
            const int j = pass * JP + jj;
            const int cl = 4 * j + tig;
            const bool inr = (span * SPAN_K + cl * CHUNK_K) < geo.K;
            uint4 wa = make_uint4(0, 0, 0, 0), wb = make_uint4(0, 0, 0, 0);
            if (inr) {
              wa = lds128(pA + cl * 16);
              wb = lds128(pB + cl * 16);
            }
            const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w};
            const uint32_t wB[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              if (BITS == 4) {
                const uint32_t p0a = bf16x2_sub(lop3_and_or(wA[w], MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p1a = bf16x2_sub(lop3_and_or(wA[w] >> 4, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p2a = bf16x2_sub(lop3_and_or(wA[w] >> 8, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p3a = bf16x2_sub(lop3_and_or(wA[w] >> 12, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p0b = bf16x2_sub(lop3_and_or(wB[w], MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p1b = bf16x2_sub(lop3_and_or(wB[w] >> 4, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p2b = bf16x2_sub(lop3_and_or(wB[w] >> 8, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t p3b = bf16x2_sub(lop3_and_or(wB[w] >> 12, MASK, MAGIC_LO), MAGIC_LO);
                mma_bf16_16816(d, p0a, p0b, p1a, p1b, breg[jj][w * 4 + 0], breg[jj][w * 4 + 1]);
                mma_bf16_16816(d, p2a, p2b, p3a, p3b, breg[jj][w * 4 + 2], breg[jj][w * 4 + 3]);
              } else {
                const uint32_t l0a = bf16x2_sub(lop3_and_or(wA[w], MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t l1a = bf16x2_sub(lop3_and_or(wA[w] >> 8, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t h0a = bf16x2_sub(lop3_and_or(wA[w] >> 4, MASK, MAGIC_HI), MAGIC_HI);
                const uint32_t h1a = bf16x2_sub(lop3_and_or(wA[w] >> 12, MASK, MAGIC_HI), MAGIC_HI);
                const uint32_t l0b = bf16x2_sub(lop3_and_or(wB[w], MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t l1b = bf16x2_sub(lop3_and_or(wB[w] >> 8, MASK, MAGIC_LO), MAGIC_LO);
                const uint32_t h0b = bf16x2_sub(lop3_and_or(wB[w] >> 4, MASK, MAGIC_HI), MAGIC_HI);
                const uint32_t h1b = bf16x2_sub(lop3_and_or(wB[w] >> 12, MASK, MAGIC_HI), MAGIC_HI);
                mma_bf16_16816(d, l0a, l0b, l1a, l1b, breg[jj][w * 2 + 0], breg[jj][w * 2 + 1]);
                mma_bf16_16816(d, h0a, h0b, h1a, h1b, breg[jj][w * 2 + 0], breg[jj][w * 2 + 1]);
              }
            }
          }
        }
        // d[0]=D[g][2tig] d[1]=D[g][2tig+1] d[2]=D[g+8][2tig] d[3]=D[g+8][2tig+1]
        const int Gl = spl * 8 + 2 * tig;  // group index within the round
        const int Gg = g0 + Gl;            // global group index
        float pa = 0.f, pb = 0.f;
        if (Gg < geo.ng && Gl < Gr) {
          pa = fmaf(bits2f(bsc[rowA * Gr + Gl]), d[0], pa);
          pa = fmaf(bits2f(bbi[rowA * Gr + Gl]), xsv[Gg], pa);
          pb = fmaf(bits2f(bsc[(rowA + 8) * Gr + Gl]), d[2], pb);
          pb = fmaf(bits2f(bbi[(rowA + 8) * Gr + Gl]), xsv[Gg], pb);
        }
        if (Gg + 1 < geo.ng && Gl + 1 < Gr) {
          pa = fmaf(bits2f(bsc[rowA * Gr + Gl + 1]), d[1], pa);
          pa = fmaf(bits2f(bbi[rowA * Gr + Gl + 1]), xsv[Gg + 1], pa);
          pb = fmaf(bits2f(bsc[(rowA + 8) * Gr + Gl + 1]), d[3], pb);
          pb = fmaf(bits2f(bbi[(rowA + 8) * Gr + Gl + 1]), xsv[Gg + 1], pb);
        }
        pa += __shfl_xor_sync(0xffffffffu, pa, 1);
        pa += __shfl_xor_sync(0xffffffffu, pa, 2);
        pb += __shfl_xor_sync(0xffffffffu, pb, 1);
        pb += __shfl_xor_sync(0xffffffffu, pb, 2);
        if (tig == 0) {
          red[rowA * geo.nspans + span] = pa;
          red[(rowA + 8) * geo.nspans + span] = pb;
        }
      }
    }
    __syncthreads();
    if (tid == 0 && r + geo.nbuf < nrounds) {
      fence_proxy_async();
      issue(r + geo.nbuf);
    }
    // ---- epilogue for the rows of this row group after its last k-round
    if (kr == geo.nkr - 1) {
      for (int i = tid; i < nl; i += kThreads) {
        float acc = 0.f;
        for (int sp = 0; sp < geo.nspans; ++sp) acc += red[i * geo.nspans + sp];
        const int n = L0 + i;
        switch (a.epi) {
          case kEpiStore:
            a.y[n] = f2bf(acc);
            break;
          case kEpiResid:
            a.y[n] = f2bf(__fadd_rn(bf2f(a.res[n]), bfround(acc)));
            break;
          case kEpiSwiglu: {
            float accu = 0.f;
            for (int sp = 0; sp < geo.nspans; ++sp) accu += red[(nl + i) * geo.nspans + sp];
            const float gv = bfround(acc), uv = bfround(accu);
            const float sg = bfround(sigmoid_f(gv));
            const float sv = bfround(__fmul_rn(gv, sg));
            a.y[n] = f2bf(__fmul_rn(sv, uv));
            break;
          }
          case kEpiArgmax: {
            const float v = bfround(acc);
            if (a.y) a.y[n] = f2bf(v);
            if (v == v && (v > best_v || (v == best_v && n < best_i))) {
              best_v = v;
              best_i = n;
            }
            break;
          }
          default:
            a.yf[n] = acc;
            break;
        }
      }
      __syncthreads();
    }
  }

  if (a.epi == kEpiArgmax) {
    // CTA-level (max, first index), then the last CTA to finish reduces all.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best_v || (ov == best_v && oi < best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    __shared__ float wv[kWarps];
    __shared__ int wi[kWarps];
    __shared__ unsigned last;
    if (lane == 0) {
      wv[warp] = best_v;
      wi[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
      float bv = wv[0];
      int bi = wi[0];
      for (int w = 1; w < kWarps; ++w)
        if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) {
          bv = wv[w];
          bi = wi[w];
        }
      a.am_val[blockIdx.x] = bv;
      a.am_idx[blockIdx.x] = bi;
      __threadfence();
      last = (atomicAdd(a.am_ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (last && tid == 0) {
      __threadfence();
      const volatile float* vv = a.am_val;
      const volatile int* vi = a.am_idx;
      float bv = vv[0];
      int bi = vi[0];
      for (int c = 1; c < (int)gridDim.x; ++c) {
        const float v = vv[c];
        const int i = vi[c];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
      if (bi == 0x7fffffff) bi = 0;
      *a.tok_out = bi;
      if (a.hist && a.hist_n) {
        const int hn = *a.hist_n;
        a.hist[hn % a.hist_cap] = bi;
        *a.hist_n = hn + 1;
      }
      if (a.pos) *a.pos += a.pos_inc;
      *a.am_ticket = 0u;
    }
  }
}

template <int BITS, int GS>
cudaError_t launch_t(const GemvArgs& a, const GemvGeom& geo, int grid, int smem, cudaStream_t st, bool pdl) {
  auto kern = qgemv_kernel<BITS, GS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a, geo);
}

void make_geom(int N, int K, int bits, int gs, int epi, int x_slots, const GemvPlan* p, GemvGeom* g) {
  g->K = K;
  g->ng = K / gs;
  g->nspans = (g->ng + 7) / 8;
  g->kbytes = K * bits / 8;
  g->span_bytes = span_k(gs) * bits / 8;
  g->swiglu = epi == kEpiSwiglu;
  g->x_slots = x_slots > 1 ? x_slots : 1;
  g->lrows = g->swiglu ? N / 2 : N;
  g->rows_round = p ? p->rows_round : 16;
  g->spans_round = p ? p->spans_round : g->nspans;
  g->nbuf = p ? p->nbuf : 1;
  g->nkr = (g->nspans + g->spans_round - 1) / g->spans_round;
  geom_layout(*g);
}

}  // namespace

int gemv_make_plan(int N, int K, int bits, int gs, int epi, int x_slots, int num_sms, GemvPlan* plan) {
  if (!(bits == 4 || bits == 8) || !(gs == 32 || gs == 64 || gs == 128)) return -1;
  if (K <= 0 || N <= 0 || K % gs != 0) return -1;
  if ((K * bits / 8) % 16 != 0) return -1;
  const bool sw = epi == kEpiSwiglu;
  if (sw && (N % 2 != 0)) return -1;
  const int lrows = sw ? N / 2 : N;
  if (lrows % 16 != 0) return -1;
  const int nlb = lrows / 16;
  const int grid = std::max(1, std::min(nlb, num_sms));
  const int lb_per_cta = (nlb + grid - 1) / grid;
  GemvGeom g;
  make_geom(N, K, bits, gs, epi, x_slots, nullptr, &g);
  // Largest round (rows x spans) that fits the budget; prefer whole-K rounds.
  int best_rows = 0, best_spans = 0, best_nbuf = 1;
  for (int spans = g.nspans; spans >= 1 && best_rows == 0; --spans) {
    if (spans < g.nspans && (g.ng % 8) != 0) break;  // per-row s/b copies need 16B rows
    for (int rlb = lb_per_cta; rlb >= 1; --rlb) {
      GemvGeom t = g;
      t.rows_round = rlb * 16;
      t.spans_round = spans;
      t.nkr = (g.nspans + spans - 1) / spans;
      const int nrounds = ((lb_per_cta + rlb - 1) / rlb) * t.nkr;
      t.nbuf = nrounds > 1 ? 2 : 1;
      geom_layout(t);
      if (geom_smem(t) <= kSmemBudget) {
        best_rows = t.rows_round;
        best_spans = spans;
        best_nbuf = t.nbuf;
        break;
      }
    }
  }
  if (best_rows == 0) return -1;
  plan->grid = grid;
  plan->lrows = lrows;
  plan->rows_round = best_rows;
  plan->spans_round = best_spans;
  plan->nbuf = best_nbuf;
  plan->x_slots = x_slots > 1 ? x_slots : 1;
  GemvGeom t;
  make_geom(N, K, bits, gs, epi, x_slots, plan, &t);
  plan->smem = geom_smem(t);
  return 0;
}

cudaError_t gemv_launch(const GemvArgs& a, const GemvPlan& p, cudaStream_t st, bool pdl) {
  GemvGeom g;
  make_geom(a.N, a.K, a.bits, a.gs, a.epi, p.x_slots, &p, &g);
  const int smem = geom_smem(g);
#define EMX_GEMV_CASE(B, G) \
  if (a.bits == B && a.gs == G) return launch_t<B, G>(a, g, p.grid, smem, st, pdl);
  EMX_GEMV_CASE(4, 32)
  EMX_GEMV_CASE(4, 64)
  EMX_GEMV_CASE(4, 128)
  EMX_GEMV_CASE(8, 32)
  EMX_GEMV_CASE(8, 64)
  EMX_GEMV_CASE(8, 128)
#undef EMX_GEMV_CASE
  return cudaErrorInvalidValue;
}

}  // namespace emx
