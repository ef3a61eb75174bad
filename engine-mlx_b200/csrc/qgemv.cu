// qgemv.cu — batch-1 quantized GEMV for sm_100a.
//
// One CTA per SM (at most), each owning a contiguous run of 16-row blocks.
// Data path per CTA:
//   1. before griddepcontrol.wait: warp 0 asks the bulk-copy engine (untiled
//      TMA) for the CTA's first rounds of packed weight rows and their
//      scale/bias rows — one copy per contiguous row run, the lanes issuing
//      in parallel — into a shared-memory ring.  Weights never depend on the
//      previous kernel, so with PDL their transfer overlaps that kernel's
//      tail: the batch-1 decode step becomes one continuous HBM stream;
//   2. after the wait: the input vector is built in shared memory in one
//      vectorised pass (16-byte chunks; optionally RMS-normalised, gathered
//      from the quantized embedding for layer 0, or summed with a tensor-
//      parallel / MoE partial first), written in MMA fragment order, with
//      the per-group sums of x reduced by warp shuffles on the way;
//   3. each warp takes (16-row block x 8-group span) units: packed nibbles /
//      bytes become bf16 through a magic-number LOP3 and an exact bf16x2
//      subtract, and m16n8k16 tensor-core MMAs compute the per-group dot
//      products — column j of the MMA's B operand carries x masked to group
//      j, so one accumulator tile yields eight group sums at once.  Rows are
//      dense in shared memory; odd rows load each pair of 16-byte chunks in
//      the opposite order, so a quarter-warp always touches both halves of a
//      128-byte bank line (no conflicts) — the pair is swapped back in
//      registers;
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
constexpr int kSmemBudget = 112 * 1024;  // two CTAs per SM (228 KB - 2 x 1 KB reserved)

struct GemvGeom {
  int K, ng, nspans, kbytes, span_bytes, lrows;
  int swiglu, x_slots;
  // plan
  int rows_round, spans_round, nbuf, nkr;
  int stride;        // smem bytes per weight row in a round buffer (dense)
  int groups_round;  // max groups per round
  int buf_bytes;     // bytes per ring slot
  int off_x, off_xs, off_red, off_buf;
};

__host__ __device__ inline int span_k(int gs) { return 8 * gs; }

// Shared-memory carve-up for a given round shape.
__host__ __device__ inline void geom_layout(GemvGeom& g) {
  const bool whole = g.spans_round >= g.nspans;
  g.stride = whole ? g.kbytes : g.spans_round * g.span_bytes;
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

// x in MMA fragment order: inside each 8-element (int4) / 4-element (int8)
// block, element i sits where the dequantised nibble pairs expect it.
template <int BITS>
__device__ __forceinline__ uint4 permute8(uint4 v) {
  if (BITS == 4) {  // [x0..x7] -> [x0,x4,x1,x5,x2,x6,x3,x7]
    uint4 r;
    r.x = __byte_perm(v.x, v.z, 0x5410);
    r.y = __byte_perm(v.x, v.z, 0x7632);
    r.z = __byte_perm(v.y, v.w, 0x5410);
    r.w = __byte_perm(v.y, v.w, 0x7632);
    return r;
  } else {  // two blocks [x0,x1,x2,x3] -> [x0,x2,x1,x3]
    uint4 r;
    r.x = __byte_perm(v.x, v.y, 0x5410);
    r.y = __byte_perm(v.x, v.y, 0x7632);
    r.z = __byte_perm(v.z, v.w, 0x5410);
    r.w = __byte_perm(v.z, v.w, 0x7632);
    return r;
  }
}

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 r;
  r.x = (uint32_t)f2bits(f[0]) | ((uint32_t)f2bits(f[1]) << 16);
  r.y = (uint32_t)f2bits(f[2]) | ((uint32_t)f2bits(f[3]) << 16);
  r.z = (uint32_t)f2bits(f[4]) | ((uint32_t)f2bits(f[5]) << 16);
  r.w = (uint32_t)f2bits(f[6]) | ((uint32_t)f2bits(f[7]) << 16);
  return r;
}

// The pre-norm source values of elements [8c, 8c+8) (bf16 values as float).
__device__ __forceinline__ void load_src8(const GemvArgs& a, int c, int tok, float (&v)[8]) {
  const int k0 = c * 8;
  if (a.pro == kProEmbedNorm) {
    const int per = 32 / a.emb_bits;
    const int ngk = a.K / a.emb_gs;
    const uint32_t* row = a.emb_w + (size_t)tok * (a.K / per);
    const bf16 sv = a.emb_s[(size_t)tok * ngk + k0 / a.emb_gs];
    const bf16 bv = a.emb_b[(size_t)tok * ngk + k0 / a.emb_gs];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      const uint32_t q = (row[k / per] >> (a.emb_bits * (k % per))) & ((1u << a.emb_bits) - 1u);
      v[e] = bf2f(dequant1(q, sv, bv));
    }
    return;
  }
  unpack8(*reinterpret_cast<const uint4*>(a.x + k0), v);
  if (a.pro == kProAddNorm) {
    float add[8];
    if (a.moe_y) {
#pragma unroll
      for (int e = 0; e < 8; ++e) add[e] = 0.f;
      const int n = *a.moe_n;
      for (int s = 0; s < n; ++s) {
        float y[8];
        unpack8(*reinterpret_cast<const uint4*>(a.moe_y + (size_t)s * a.K + k0), y);
        const float w = a.moe_w[s];
#pragma unroll
        for (int e = 0; e < 8; ++e) add[e] = __fadd_rn(add[e], __fmul_rn(y[e], w));
      }
    } else {
      const float4 p0 = *reinterpret_cast<const float4*>(a.add_f32 + k0);
      const float4 p1 = *reinterpret_cast<const float4*>(a.add_f32 + k0 + 4);
      add[0] = p0.x, add[1] = p0.y, add[2] = p0.z, add[3] = p0.w;
      add[4] = p1.x, add[5] = p1.y, add[6] = p1.z, add[7] = p1.w;
      if (a.add_round) {
#pragma unroll
        for (int e = 0; e < 8; ++e) add[e] = bfround(add[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = bfround(__fadd_rn(v[e], add[e]));
  }
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
  static_assert(J_SPAN % 2 == 0, "chunks are loaded in pairs");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const bool gather = a.slot_expert != nullptr;
  const int rlb = geo.rows_round / 16;
  const int Kb = geo.kbytes;
  const int phys_mult = geo.swiglu ? 2 : 1;
  const bool kwhole = geo.nkr == 1;

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

  // ---- one round: weight rows + scale/bias rows into ring slot r % nbuf.
  // Called by all 32 lanes of warp 0; copies are spread over the lanes.
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
    if (lane == 0) mbar_arrive_expect_tx(&mbar[buf], (uint32_t)(phys * kbytes + 2 * sb_bytes));
    __syncwarp();
    // contiguous runs of physical rows: the gate / up halves (whole-K), a
    // 16-row block (expert gather), or single rows (k-split rounds)
    const int blk_rows = !kwhole ? 1 : (gather ? 16 : nl);
    const int nblk = phys / blk_rows;
    const unsigned char* wbase = reinterpret_cast<const unsigned char*>(a.w);
    const uint64_t pol = l2_evict_first_policy();
    for (int i = lane; i < 3 * nblk; i += 32) {
      const int blk = i / 3, part = i % 3;
      const int prow = blk * blk_rows;  // first buffer row of the run
      const int src = (prow >= nl) ? phys_row(a, lrows, L0 + prow - nl, true) : phys_row(a, lrows, L0 + prow, false);
      if (part == 0) {
        bulk_g2s_hint(bw + (size_t)prow * geo.stride, wbase + (size_t)src * Kb + kb0,
                      (uint32_t)(blk_rows == 1 ? kbytes : blk_rows * Kb), &mbar[buf], pol);
      } else {
        const bf16* sb = part == 1 ? a.s : a.b;
        unsigned char* dst = (part == 1 ? bs : bb) + (size_t)prow * Gr * 2;
        bulk_g2s_hint(dst, sb + (size_t)src * geo.ng + g0, (uint32_t)(blk_rows * Gr * 2), &mbar[buf], pol);
      }
    }
  };

  if (!gather) {
    partition();
    if (warp == 0) {
      const int pre = min(geo.nbuf, nrounds);
      for (int r = 0; r < pre; ++r) issue(r);
    }
  }

  // ---- wait for the producer of x (previous kernel) ---------------------
  pdl_wait();
  // the next kernel may launch once this one's inputs are final: one kernel
  // ahead streams its weights beside this one, while an earlier trigger lets
  // the chain run several kernels ahead and the block scheduler then stacks
  // two CTAs of one launch on an SM while others hold none
  pdl_trigger();

  if (gather) {
    lrows = min(*a.n_slots * a.slot_rows, geo.lrows);
    partition();
    if (warp == 0) {
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
  // ---- prologue: x (normalised) into shared memory, fragment order, and
  //      the per-group sums of x (GS/8 consecutive 16-byte chunks per group)
  {
    const int K = geo.K;
    const int nch = K / 8;
    constexpr int CPG = GS / 8;  // chunks per group: 4, 8 or 16 consecutive lanes
    auto emit = [&](int c, bool valid, const float (&o)[8]) {
      float ps = 0.f;
      if (valid) {
        *reinterpret_cast<uint4*>(xp + (size_t)c * 8) = permute8<BITS>(pack8(o));
#pragma unroll
        for (int e = 0; e < 8; ++e) ps += o[e];
      }
#pragma unroll
      for (int off = 1; off < CPG; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      if (valid && (c % CPG) == 0) xs[c / CPG] = ps;
    };
    if (a.pro == kProX) {
      const int total = geo.x_slots * nch;
#pragma unroll 1
      for (int it = 0; it * kThreads < total; ++it) {
        const int c = it * kThreads + tid;
        const bool valid = c < total;
        float v[8];
        if (valid) unpack8(*reinterpret_cast<const uint4*>(a.x + (size_t)c * 8), v);
        else
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = 0.f;
        emit(c, valid, v);
      }
    } else {
      // pass 1: the pre-norm source (exact bf16 values) staged in the x
      // buffer in natural order, sums of squares per norm group
      const int groups = a.norm_groups > 0 ? a.norm_groups : 1;
      const int gd = K / groups;
      const bool store = (a.pro == kProEmbedNorm || a.pro == kProAddNorm) && blockIdx.x == 0 && a.x_out;
      float ssg[8];
#pragma unroll
      for (int gi = 0; gi < 8; ++gi) ssg[gi] = 0.f;
#pragma unroll 1
      for (int c = tid; c < nch; c += kThreads) {
        float v[8];
        load_src8(a, c, tok, v);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
        const int grp = (c * 8) / gd;
#pragma unroll
        for (int gi = 0; gi < 8; ++gi)
          if (grp == gi) ssg[gi] += ss;
        const uint4 pk = pack8(v);
        *reinterpret_cast<uint4*>(xp + (size_t)c * 8) = pk;
        if (store) *reinterpret_cast<uint4*>(a.x_out + (size_t)c * 8) = pk;
      }
      float* inv = scratch + 16;  // per-group 1/rms, groups <= 8
      for (int gi = 0; gi < groups; ++gi) {
        float sv = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q == gi) sv = ssg[q];
        const float ss = block_sum(sv, scratch);
        if (tid == 0) inv[gi] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)gd), a.eps)));
      }
      __syncthreads();
      // pass 2: scale, weight, fragment order (each thread rewrites its own chunks)
#pragma unroll 1
      for (int it = 0; it * kThreads < nch; ++it) {
        const int c = it * kThreads + tid;
        const bool valid = c < nch;
        float o[8];
        if (valid) {
          float v[8], w[8];
          unpack8(*reinterpret_cast<const uint4*>(xp + (size_t)c * 8), v);
          unpack8(*reinterpret_cast<const uint4*>(a.norm_w + (size_t)c * 8), w);
          const float iv = inv[(c * 8) / gd];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            o[e] = groups == 1 ? bfround(__fmul_rn(bfround(__fmul_rn(v[e], iv)), w[e]))
                               : bfround(__fmul_rn(__fmul_rn(v[e], iv), w[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = 0.f;
        }
        emit(c, valid, o);
      }
    }
    __syncthreads();
  }

  // per-thread argmax state
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;

  const uint32_t MASK = 0x000F000Fu;
  const uint32_t MAGIC_LO = 0x43004300u;  // bf16 128.0 | nibble
  const uint32_t MAGIC_HI = 0x45004500u;  // bf16 2048.0 | nibble  (value 2048 + 16*nibble)
  const bool odd = (g & 1) != 0;

  for (int r = 0; r < nrounds; ++r) {
    const int buf = r % geo.nbuf;
    const int rg = r / geo.nkr, kr = r % geo.nkr;
    const int L0 = (lb0 + rg * rlb) * 16;
    const int nl = min(rlb, lb1 - lb0 - rg * rlb) * 16;
    const int sp0 = kr * geo.spans_round;
    const int sp1 = min(geo.nspans, sp0 + geo.spans_round);
    const int g0 = sp0 * 8;
    const int Gr = min((sp1 - sp0) * 8, geo.ng - g0);
    const int kbytes_r = min((sp1 - sp0) * geo.span_bytes, Kb - sp0 * geo.span_bytes);
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
        const int span_off = spl * geo.span_bytes;  // byte offset of this span inside the round's rows
        float d[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
        // one pair of 16-byte chunks per iteration (rolled: the body is the
        // whole hot loop, so its instructions stay cached across iterations)
#pragma unroll 1
        for (int jp = 0; jp < J_SPAN / 2; ++jp) {
          // B fragments of the pair: x masked to this lane's column (group)
          uint32_t breg[2][BREG];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int cl = 4 * (2 * jp + h) + tig;
            const int k0 = span * SPAN_K + cl * CHUNK_K;
            const bool on = ((cl * CHUNK_K) / GS == g) && (k0 < geo.K);
            if (on) {
#pragma unroll
              for (int q = 0; q < BREG / 4; ++q) {
                const uint4 v = *reinterpret_cast<const uint4*>(xpv + k0 + q * 8);
                breg[h][q * 4 + 0] = v.x;
                breg[h][q * 4 + 1] = v.y;
                breg[h][q * 4 + 2] = v.z;
                breg[h][q * 4 + 3] = v.w;
              }
            } else {
#pragma unroll
              for (int q = 0; q < BREG; ++q) breg[h][q] = 0u;
            }
          }
          {
            const int j0 = 2 * jp;
            const int cl0 = 4 * j0 + tig, cl1 = cl0 + 4;
            const bool in0 = span_off + cl0 * 16 < kbytes_r, in1 = span_off + cl1 * 16 < kbytes_r;
            // even rows read (cl0, cl1), odd rows (cl1, cl0): each quarter-warp
            // covers both halves of a 128-byte line
            const int f = odd ? cl1 : cl0, sc = odd ? cl0 : cl1;
            const bool inf = odd ? in1 : in0, ins = odd ? in0 : in1;
            const uint4 fa = *reinterpret_cast<const uint4*>(pA + (inf ? f * 16 : 0));
            const uint4 sa = *reinterpret_cast<const uint4*>(pA + (ins ? sc * 16 : 0));
            const uint4 fb = *reinterpret_cast<const uint4*>(pB + (inf ? f * 16 : 0));
            const uint4 sbv = *reinterpret_cast<const uint4*>(pB + (ins ? sc * 16 : 0));
            const uint4 a0 = odd ? sa : fa, a1 = odd ? fa : sa;
            const uint4 b0 = odd ? sbv : fb, b1 = odd ? fb : sbv;
            const uint32_t wA[2][4] = {{a0.x, a0.y, a0.z, a0.w}, {a1.x, a1.y, a1.z, a1.w}};
            const uint32_t wB[2][4] = {{b0.x, b0.y, b0.z, b0.w}, {b1.x, b1.y, b1.z, b1.w}};
            // Codes enter the MMA as bf16 (magic + code); the magic offset is
            // removed once per group in the scale/bias step below.  The four
            // accumulators take consecutive MMAs so none waits on the last.
#pragma unroll
            for (int w = 0; w < 4; ++w) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (BITS == 4) {
                  const uint32_t p0a = lop3_and_or(wA[h][w], MASK, MAGIC_LO);
                  const uint32_t p1a = lop3_and_or(wA[h][w] >> 4, MASK, MAGIC_LO);
                  const uint32_t p2a = lop3_and_or(wA[h][w] >> 8, MASK, MAGIC_LO);
                  const uint32_t p3a = lop3_and_or(wA[h][w] >> 12, MASK, MAGIC_LO);
                  const uint32_t p0b = lop3_and_or(wB[h][w], MASK, MAGIC_LO);
                  const uint32_t p1b = lop3_and_or(wB[h][w] >> 4, MASK, MAGIC_LO);
                  const uint32_t p2b = lop3_and_or(wB[h][w] >> 8, MASK, MAGIC_LO);
                  const uint32_t p3b = lop3_and_or(wB[h][w] >> 12, MASK, MAGIC_LO);
                  mma_bf16_16816(d[2 * h], p0a, p0b, p1a, p1b, breg[h][w * 4 + 0], breg[h][w * 4 + 1]);
                  mma_bf16_16816(d[2 * h + 1], p2a, p2b, p3a, p3b, breg[h][w * 4 + 2], breg[h][w * 4 + 3]);
                } else {
                  const uint32_t l0a = lop3_and_or(wA[h][w], MASK, MAGIC_LO);
                  const uint32_t l1a = lop3_and_or(wA[h][w] >> 8, MASK, MAGIC_LO);
                  const uint32_t h0a = lop3_and_or(wA[h][w] >> 4, MASK, MAGIC_HI);
                  const uint32_t h1a = lop3_and_or(wA[h][w] >> 12, MASK, MAGIC_HI);
                  const uint32_t l0b = lop3_and_or(wB[h][w], MASK, MAGIC_LO);
                  const uint32_t l1b = lop3_and_or(wB[h][w] >> 8, MASK, MAGIC_LO);
                  const uint32_t h0b = lop3_and_or(wB[h][w] >> 4, MASK, MAGIC_HI);
                  const uint32_t h1b = lop3_and_or(wB[h][w] >> 12, MASK, MAGIC_HI);
                  mma_bf16_16816(d[2 * h], l0a, l0b, l1a, l1b, breg[h][w * 2 + 0], breg[h][w * 2 + 1]);
                  mma_bf16_16816(d[2 * h + 1], h0a, h0b, h1a, h1b, breg[h][w * 2 + 0], breg[h][w * 2 + 1]);
                }
              }
            }
          }
        }
        // sum the independent accumulators:
        // d[0]=D[g][2tig] d[1]=D[g][2tig+1] d[2]=D[g+8][2tig] d[3]=D[g+8][2tig+1]
        float dv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) dv[e] = (d[0][e] + d[1][e]) + (d[2][e] + d[3][e]);
        const int Gl = spl * 8 + 2 * tig;  // group index within the round
        const int Gg = g0 + Gl;            // global group index
        // dv = dot + C*sum(x_g) with C the magic offset (128 for int4,
        // 128 + 2048 for the two int8 halves): s*dot + b*sum = s*dv + (b - C*s)*sum
        constexpr float C = BITS == 4 ? 128.0f : 2176.0f;
        float pa = 0.f, pb = 0.f;
        if (Gg < geo.ng && Gl < Gr) {
          const float sA = bits2f(bsc[rowA * Gr + Gl]), sB = bits2f(bsc[(rowA + 8) * Gr + Gl]);
          pa = fmaf(sA, dv[0], pa);
          pa = fmaf(fmaf(-C, sA, bits2f(bbi[rowA * Gr + Gl])), xsv[Gg], pa);
          pb = fmaf(sB, dv[2], pb);
          pb = fmaf(fmaf(-C, sB, bits2f(bbi[(rowA + 8) * Gr + Gl])), xsv[Gg], pb);
        }
        if (Gg + 1 < geo.ng && Gl + 1 < Gr) {
          const float sA = bits2f(bsc[rowA * Gr + Gl + 1]), sB = bits2f(bsc[(rowA + 8) * Gr + Gl + 1]);
          pa = fmaf(sA, dv[1], pa);
          pa = fmaf(fmaf(-C, sA, bits2f(bbi[rowA * Gr + Gl + 1])), xsv[Gg + 1], pa);
          pb = fmaf(sB, dv[3], pb);
          pb = fmaf(fmaf(-C, sB, bits2f(bbi[(rowA + 8) * Gr + Gl + 1])), xsv[Gg + 1], pb);
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
    if (warp == 0 && r + geo.nbuf < nrounds) {
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
  // Largest round (rows x spans) that fits the budget with a ring of up to
  // three slots (two at least when there is more than one round); prefer
  // whole-K rounds (dense contiguous copies).
  int best_rows = 0, best_spans = 0, best_nbuf = 1;
  for (int spans = g.nspans; spans >= 1 && best_rows == 0; --spans) {
    if (spans < g.nspans && (g.ng % 8) != 0) break;  // per-row s/b copies need 16B rows
    for (int rlb = lb_per_cta; rlb >= 1 && best_rows == 0; --rlb) {
      GemvGeom t = g;
      t.rows_round = rlb * 16;
      t.spans_round = spans;
      t.nkr = (g.nspans + spans - 1) / spans;
      const int nrounds = ((lb_per_cta + rlb - 1) / rlb) * t.nkr;
      for (int nbuf = std::min(nrounds, 3); nbuf >= std::min(nrounds, 2); --nbuf) {
        t.nbuf = nbuf;
        geom_layout(t);
        if (geom_smem(t) <= kSmemBudget) {
          best_rows = t.rows_round;
          best_spans = spans;
          best_nbuf = nbuf;
          break;
        }
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
  if (a.pro != kProX && a.norm_groups > 8) return cudaErrorInvalidValue;
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
