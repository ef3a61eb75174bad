// pgemv.cu — batch-1 quantized GEMV over the packed tile layout (sm_100a).
//
// One CTA per SM at most, owning a contiguous run of 16-row logical blocks
// (for SwiGLU a logical block carries its gate and its up rows).  Nine warps:
//   * warp 8 is the producer: one thread asks the bulk-copy engine (untiled
//     TMA) for whole pipeline stages — a stage is a contiguous run of packed
//     tiles, so it is one copy (one per expert run under a gather) — into a
//     ring of shared-memory buffers, waiting on each buffer's "empty"
//     mbarrier before reusing it.  Weights do not depend on the previous
//     kernel, so the first stages are requested before griddepcontrol.wait
//     and stream in while that kernel finishes;
//   * warps 0-7 consume: each waits on a stage's "full" mbarrier, takes
//     (tile, half-span) units round-robin, and arrives on the stage's
//     "empty" mbarrier when done — there is no CTA-wide barrier in the loop.
// A unit: per slice quad, one conflict-free 128-bit shared load per word set
// gives four slices' A registers; a LOP3 per register turns codes into bf16
// (magic-number exponent, exact) and an m16n8k16 MMA per slice adds the
// four group dot products of rows g, g+8 at once: column j < 4 of B holds x
// masked to group j, so only the lanes with g == t load x (two adjacent
// registers per slice from one 8-byte run) and the other lanes read a zero
// block; x groups sit 2*gs + 16 bytes apart, so the four loading lanes hit
// four different bank groups.  Each warp runs two units at once, interleaved
// quad by quad, so one unit's accumulator drain overlaps the other's math.
// Then per row s*dot + (b - C*s)*sum(x_g) in fp32 — the MLX qmv
// factorisation, C being the magic offset — reduced over the lane pair and
// stored to a per-(row, span, half-span) slot.  After the last stage one
// barrier, then the epilogue sums each row's slots in order and applies the
// fused output step (store / residual / SwiGLU / argmax / fp32 partial).
#include "pgemv.cuh"

#include <algorithm>

namespace emx {

namespace {

constexpr int kConsumers = 8;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kMaxBuf = 8;

struct PGeom {
  int K, ng, S;
  int tile_bytes, a_bytes;
  int halves;
  int lb_total;
  int stage_tiles, nbuf;
  int stage_bytes;
  int x_slots, xk;  // x elements per slot (whole spans)
  int gstride;      // bytes per x group in shared memory (2*gs + 16: banks rotate per group)
  int xslot_bytes;  // bytes per x slot
  int red_rows;
  int nw_bytes;  // room for the norm weights (fetched before the wait)
  unsigned long long lbt_magic;  // ceil(2^32 / (halves * S)): tile -> logical block
  unsigned long long lps_magic;  // ceil(2^32 / (slot rows / 16)): logical block -> x slot
  int off_x, off_nw, off_zero, off_xs, off_red, off_buf;
};

__host__ __device__ inline int ptile_bytes(int bits, int gs) { return 16 * 8 * gs * bits / 8 + 512; }

// Shared-memory carve-up (the first 384 bytes: mbarriers, reduction scratch,
// per-group 1/rms, the abort flag and the norm-weight mbarrier).
__host__ __device__ inline int pgeom_layout(PGeom& g, int gs) {
  g.off_x = 384;
  g.off_nw = g.off_x + g.x_slots * g.xslot_bytes;
  g.off_zero = g.off_nw + g.nw_bytes;
  g.off_xs = g.off_zero + 2 * gs;
  g.off_red = g.off_xs + ((g.x_slots * g.S * 8 * 4 + 15) & ~15);
  g.off_buf = (g.off_red + g.red_rows * g.S * 2 * 4 + 127) & ~127;
  return g.off_buf + g.nbuf * g.stage_bytes;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also gives up at once when another warp has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
  }
  report_status(status, kDevTimeoutMbar);
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ void unpack8f(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Eight floats that are bf16 values already (no rounding needed).
__device__ __forceinline__ uint4 pack8exact(const float (&f)[8]) {
  uint4 r;
  r.x = (__float_as_uint(f[0]) >> 16) | (__float_as_uint(f[1]) & 0xffff0000u);
  r.y = (__float_as_uint(f[2]) >> 16) | (__float_as_uint(f[3]) & 0xffff0000u);
  r.z = (__float_as_uint(f[4]) >> 16) | (__float_as_uint(f[5]) & 0xffff0000u);
  r.w = (__float_as_uint(f[6]) >> 16) | (__float_as_uint(f[7]) & 0xffff0000u);
  return r;
}


// The pre-norm source values of elements [8c, 8c+8) (bf16 values as float).
__device__ __forceinline__ void src8(const GemvArgs& a, int c, int tok, float (&v)[8]) {
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
  unpack8f(*reinterpret_cast<const uint4*>(a.x + k0), v);
  if (a.pro == kProAddNorm) {
    float add[8];
    if (a.moe_y) {
#pragma unroll
      for (int e = 0; e < 8; ++e) add[e] = 0.f;
      const int n = *a.moe_n;
      for (int s = 0; s < n; ++s) {
        float y[8];
        unpack8f(*reinterpret_cast<const uint4*>(a.moe_y + (size_t)s * a.K + k0), y);
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

template <int BITS, int GS>
__global__ void __launch_bounds__(kThreads, 2) pgemv_kernel(const GemvArgs a, const PGeom geo) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxBuf;
  float* scratch = reinterpret_cast<float*>(smem + 128);  // 32 floats
  float* inv = scratch + 32;                             // 8 floats
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 320);
  uint64_t* nwbar = reinterpret_cast<uint64_t*>(smem + 336);
  unsigned char* xsm = smem + geo.off_x;  // x: [slot][group][gs bf16 + 16 pad bytes]
  const unsigned char* zero = smem + geo.off_zero;  // read as B by the lanes that carry no x
  const bf16* nwsm = reinterpret_cast<const bf16*>(smem + geo.off_nw);
  float* xs = reinterpret_cast<float*>(smem + geo.off_xs);
  float* red = reinterpret_cast<float*>(smem + geo.off_red);
  unsigned char* bufs = smem + geo.off_buf;

  constexpr int SPAN_K = 8 * GS;
  constexpr int QH = GS / 16;   // slice quads per half-span (4 groups)
  constexpr int HW = BITS / 4;  // word sets per quad
  constexpr int A_BYTES = 16 * SPAN_K * BITS / 8;
  constexpr int CPG = GS / 8;   // 8-element chunks per group
  // byte offset of 8-element chunk c of x slot `slot`
  auto xchunk = [&](int slot, int c) -> unsigned char* {
    return xsm + (size_t)slot * geo.xslot_bytes + (c / CPG) * geo.gstride + (c % CPG) * 16;
  };

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool gather = a.slot_expert != nullptr;
  const int halves = geo.halves, S = geo.S, SKP = S * 2;  // partial slots per row: span x half-span
  const int lb_tiles = halves * S;
  const size_t lb_bytes = (size_t)lb_tiles * geo.tile_bytes;
  const int lps = gather ? a.slot_rows / 16 : 1;  // logical blocks per slot
  const bool producer = warp == kConsumers && lane == 0;

  // this CTA: logical blocks [lb0, lb1) = tiles [T0, T1), in stages of
  // stage_tiles tiles
  int lb_total = geo.lb_total, lb0 = 0, lb1 = 0, T0 = 0, T1 = 0, nst = 0;
  auto partition = [&]() {
    lb0 = (int)((long long)blockIdx.x * lb_total / gridDim.x);
    lb1 = (int)((long long)(blockIdx.x + 1) * lb_total / gridDim.x);
    T0 = lb0 * lb_tiles;
    T1 = lb1 * lb_tiles;
    nst = (T1 - T0 + geo.stage_tiles - 1) / geo.stage_tiles;
  };

  if (tid == 0) {
    for (int i = 0; i < geo.nbuf; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumers);
    }
    mbar_init(nwbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  const unsigned char* wsrc = reinterpret_cast<const unsigned char*>(a.w);
  auto src_of = [&](int lb) -> const unsigned char* {
    if (!gather) return wsrc + (size_t)lb * lb_bytes;
    const int e = a.slot_expert[lb / lps];
    return wsrc + ((size_t)e * lps + lb % lps) * lb_bytes;
  };
  // Stage st: tiles [T0 + st*stage_tiles, ...) into buffer st % nbuf, one
  // copy per run of tiles contiguous in global memory.
  auto issue = [&](int st) {
    const int a0 = T0 + st * geo.stage_tiles, a1 = min(T1, a0 + geo.stage_tiles);
    const int buf = st % geo.nbuf;
    unsigned char* dst = bufs + (size_t)buf * geo.stage_bytes;
    const size_t tb = geo.tile_bytes;
    mbar_arrive_expect_tx(&full[buf], (uint32_t)((a1 - a0) * tb));
    const uint64_t pol = l2_evict_first_policy();
    for (int tl = a0; tl < a1;) {
      const int lb = tl / lb_tiles;
      const unsigned char* src = src_of(lb) + (size_t)(tl - lb * lb_tiles) * tb;
      int end = min(a1, (lb + 1) * lb_tiles);
      while (end < a1 && src_of(end / lb_tiles) == src + (size_t)(end - tl) * tb) end = min(a1, end + lb_tiles);
      bulk_g2s_hint(dst + (size_t)(tl - a0) * tb, src, (uint32_t)((end - tl) * tb), &full[buf], pol);
      tl = end;
    }
  };

  // the norm weights do not depend on the previous kernel either
  const bool norm_pre = a.pro != kProX;
  if (norm_pre && producer) {
    mbar_arrive_expect_tx(nwbar, (uint32_t)(geo.K * 2));
    bulk_g2s(smem + geo.off_nw, a.norm_w, (uint32_t)(geo.K * 2), nwbar);
  }
  int issued = 0;  // producer thread only
  if (!gather) {
    partition();
    if (producer) {
      issued = min(geo.nbuf, nst);
      for (int st = 0; st < issued; ++st) issue(st);
    }
  }

  // ---- wait for the producer of x (the previous kernel) -----------------
  pdl_wait();

  if (gather) {
    lb_total = min(*a.n_slots * lps, geo.lb_total);
    partition();
    if (producer) {
      issued = min(geo.nbuf, nst);
      for (int st = 0; st < issued; ++st) issue(st);
    }
  }

  // residual rows of this CTA's epilogue, loaded now so that their latency
  // overlaps the prologue's
  float res_pre[2] = {0.f, 0.f};
  const bool res_early = a.epi == kEpiResid && (lb1 - lb0) * 16 <= 2 * kThreads;
  if (res_early) {
    const int nlog = (lb1 - lb0) * 16;
    if (tid < nlog) res_pre[0] = bf2f(a.res[lb0 * 16 + tid]);
    if (tid + kThreads < nlog) res_pre[1] = bf2f(a.res[lb0 * 16 + tid + kThreads]);
  }

  int tok = 0;
  if (a.pro == kProEmbedNorm) {
    tok = *a.token;
    if (tok < 0 || tok >= a.vocab) {
      if (tid == 0) report_status(a.status, kDevBadToken);
      tok = 0;
    }
  }

  // ---- prologue: x (padded groups, zero past K to whole spans) and the
  //      group sums of x
  {
    const int K = geo.K;
    const int nch = K / 8;
    auto emit_raw = [&](int slot, int c, bool valid, uint4 raw, const float (&o)[8]) {
      float ps = 0.f;
      if (valid) {
        *reinterpret_cast<uint4*>(xchunk(slot, c)) = raw;
#pragma unroll
        for (int e = 0; e < 8; ++e) ps += o[e];
      }
#pragma unroll
      for (int off = 1; off < CPG; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      if (valid && (c % CPG) == 0) xs[slot * S * 8 + c / CPG] = ps;
    };
    // o holds bf16 values (the norm output is rounded per element)
    auto emit = [&](int slot, int c, bool valid, const float (&o)[8]) {
      emit_raw(slot, c, valid, valid ? pack8exact(o) : make_uint4(0u, 0u, 0u, 0u), o);
    };
    if (a.pro == kProX) {
      for (int slot = 0; slot < geo.x_slots; ++slot) {
#pragma unroll 1
        for (int it = 0; it * kThreads < nch; ++it) {
          const int c = it * kThreads + tid;
          const bool valid = c < nch;
          const uint4 raw = valid ? *reinterpret_cast<const uint4*>(a.x + (size_t)slot * K + c * 8)
                                  : make_uint4(0u, 0u, 0u, 0u);
          float v[8];
          unpack8f(raw, v);
          emit_raw(slot, c, valid, raw, v);
        }
      }
    } else {
      // pass 1: pre-norm source staged in the x buffer, sums of squares per
      // norm group
      const int groups = a.norm_groups > 0 ? a.norm_groups : 1;
      const int gd = K / groups;
      const bool store = (a.pro == kProEmbedNorm || a.pro == kProAddNorm) && blockIdx.x == 0 && a.x_out;
      float ssg[8];
#pragma unroll
      for (int gi = 0; gi < 8; ++gi) ssg[gi] = 0.f;
#pragma unroll 1
      for (int c = tid; c < nch; c += kThreads) {
        float v[8];
        src8(a, c, tok, v);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
        const int grp = (c * 8) / gd;
#pragma unroll
        for (int gi = 0; gi < 8; ++gi)
          if (grp == gi) ssg[gi] += ss;
        const uint4 pk = pack8exact(v);
        *reinterpret_cast<uint4*>(xchunk(0, c)) = pk;
        if (store) *reinterpret_cast<uint4*>(a.x_out + c * 8) = pk;
      }
      for (int gi = 0; gi < groups; ++gi) {
        float sv = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q == gi) sv = ssg[q];
        const float ss = block_sum(sv, scratch);
        if (tid == 0) inv[gi] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)gd), a.eps)));
      }
      __syncthreads();
      // pass 2: scale and weight in place (each thread rewrites its own chunks)
      if (!wait_or_abort(nwbar, 0u, abort_flag, a.status)) {
        // no weights: the outputs are garbage and the status word says so
      }
#pragma unroll 1
      for (int it = 0; it * kThreads < nch; ++it) {
        const int c = it * kThreads + tid;
        const bool valid = c < nch;
        float o[8];
        if (valid) {
          float v[8], w[8];
          unpack8f(*reinterpret_cast<const uint4*>(xchunk(0, c)), v);
          unpack8f(*reinterpret_cast<const uint4*>(nwsm + c * 8), w);
          const float iv = inv[(c * 8) / gd];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            o[e] = groups == 1 ? bfround(__fmul_rn(bfround(__fmul_rn(v[e], iv)), w[e]))
                               : bfround(__fmul_rn(__fmul_rn(v[e], iv), w[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = 0.f;
        }
        emit(0, c, valid, o);
      }
    }
    // zero padding: x past K (whole chunks), group sums past ng
    const int pad = (geo.xk - K) / 8;  // chunks
    for (int i = tid; i < geo.x_slots * pad; i += kThreads)
      *reinterpret_cast<uint4*>(xchunk(i / pad, nch + i % pad)) = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < GS / 2; i += kThreads) reinterpret_cast<uint32_t*>(smem + geo.off_zero)[i] = 0u;
    const int gpad = S * 8 - geo.ng;
    for (int i = tid; i < geo.x_slots * gpad; i += kThreads) xs[(i / gpad) * S * 8 + geo.ng + i % gpad] = 0.f;
  }
  __syncthreads();

  float best_v = -INFINITY;
  int best_i = 0x7fffffff;

  if (warp < kConsumers) {
    const int g = lane >> 2, t = lane & 3, t1 = t & 1;
    const bool has_x = g == t;  // the lanes whose B column carries x
    const uint32_t MASK = 0x000F000Fu;
    const uint32_t MAGIC_LO = 0x43004300u;  // bf16 128 + nibble
    const uint32_t MAGIC_HI = 0x45004500u;  // bf16 2048 + 16 * nibble
    constexpr float C = BITS == 4 ? 128.0f : 2176.0f;
    // tile -> (logical block, half, span) by a 64-bit multiply, not a
    // division: floor(n / d) == (n * ceil(2^32 / d)) >> 32 for n < 2^32 / d
    // (the magic is 2^32 itself for d == 1, hence 64 bits; the host computes
    // it, a 64-bit division here would cost the critical path ~0.5 us)
    const unsigned long long lbt_magic = geo.lbt_magic;
    // one unit = (tile, half-span): where its codes, x, scales and output
    // slot are
    struct Unit {
      const unsigned char* aw;   // this lane's code words
      const unsigned char* px;   // x of the unit's group for this lane (or the zero block)
      const unsigned char* sbp;  // this lane's scale/bias record
      const float* xg;           // the group sums
      int slot;                  // red index of row g (row g+8 is 8 rows on)
    };
    auto unit = [&](int u, int a0, const unsigned char* sbase) -> Unit {
      const int ti = u >> 1, hs = u & 1;
      const int gt = a0 + ti;
      const int lb = (int)(((unsigned long long)gt * lbt_magic) >> 32);
      const int rem = gt - lb * lb_tiles;
      const int h = rem >= S ? 1 : 0;
      const int sp = rem - h * S;
      const int xsl = (int)(((unsigned long long)lb * geo.lps_magic) >> 32);  // 0 unless x_slots > 1
      const unsigned char* tile = sbase + (size_t)ti * geo.tile_bytes;
      Unit r;
      r.aw = tile + hs * (A_BYTES / 2) + lane * 16;
      r.px = has_x ? xsm + (size_t)xsl * geo.xslot_bytes + (size_t)(sp * 8 + hs * 4 + t) * geo.gstride : zero;
      r.sbp = tile + A_BYTES + hs * 256 + (g * 2 + t1) * 16;
      r.xg = xs + xsl * S * 8 + sp * 8 + hs * 4 + 2 * t1;
      r.slot = (((lb - lb0) * halves + h) * 16 + g) * SKP + sp * 2 + hs;
      return r;
    };
    // slice quad q of a unit: HW code loads, two x loads, four (int4) or
    // eight (int8) MMAs into four independent accumulators
    auto quad = [&](const Unit& U, int q, float (&d)[4][4]) {
      uint4 wa[HW];
#pragma unroll
      for (int hw = 0; hw < HW; ++hw) wa[hw] = *reinterpret_cast<const uint4*>(U.aw + (q * HW + hw) * 512);
      const uint4 X0 = *reinterpret_cast<const uint4*>(U.px + q * 32);
      const uint4 X1 = *reinterpret_cast<const uint4*>(U.px + q * 32 + 16);
      const uint32_t bx[8] = {X0.x, X0.y, X0.z, X0.w, X1.x, X1.y, X1.z, X1.w};
      const uint32_t w0v[4] = {wa[0].x, wa[0].y, wa[0].z, wa[0].w};
      const uint32_t w1v[4] = {wa[HW - 1].x, wa[HW - 1].y, wa[HW - 1].z, wa[HW - 1].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (BITS == 4) {
          const uint32_t w = w0v[j];
          mma_bf16_16816(d[j], lop3_and_or(w, MASK, MAGIC_LO), lop3_and_or(w >> 4, MASK, MAGIC_LO),
                         lop3_and_or(w >> 8, MASK, MAGIC_LO), lop3_and_or(w >> 12, MASK, MAGIC_LO), bx[2 * j],
                         bx[2 * j + 1]);
        } else {
          const uint32_t u0 = w0v[j], u1 = w1v[j];
          mma_bf16_16816(d[(j & 1) * 2], lop3_and_or(u0, MASK, MAGIC_LO), lop3_and_or(u0 >> 8, MASK, MAGIC_LO),
                         lop3_and_or(u1, MASK, MAGIC_LO), lop3_and_or(u1 >> 8, MASK, MAGIC_LO), bx[2 * j],
                         bx[2 * j + 1]);
          mma_bf16_16816(d[(j & 1) * 2 + 1], lop3_and_or(u0 >> 4, MASK, MAGIC_HI),
                         lop3_and_or(u0 >> 12, MASK, MAGIC_HI), lop3_and_or(u1 >> 4, MASK, MAGIC_HI),
                         lop3_and_or(u1 >> 12, MASK, MAGIC_HI), bx[2 * j], bx[2 * j + 1]);
        }
      }
    };
    // d: [g][2t] [g][2t+1] [g+8][2t] [g+8][2t+1]; columns 0-3 are the
    // half-span's groups, so lanes t < 2 hold all of them
    auto finish = [&](const Unit& U, const float (&d)[4][4]) {
      float dv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) dv[e] = (d[0][e] + d[1][e]) + (d[2][e] + d[3][e]);
      const uint4 sb = *reinterpret_cast<const uint4*>(U.sbp);
      const float2 xg = *reinterpret_cast<const float2*>(U.xg);
      const float s0 = __uint_as_float(sb.x << 16), s1 = __uint_as_float(sb.x & 0xffff0000u);
      const float s2 = __uint_as_float(sb.y << 16), s3 = __uint_as_float(sb.y & 0xffff0000u);
      const float b0 = __uint_as_float(sb.z << 16), b1 = __uint_as_float(sb.z & 0xffff0000u);
      const float b2 = __uint_as_float(sb.w << 16), b3 = __uint_as_float(sb.w & 0xffff0000u);
      float pa = fmaf(s0, dv[0], 0.f), pb = fmaf(s2, dv[2], 0.f);
      pa = fmaf(fmaf(-C, s0, b0), xg.x, pa);
      pa = fmaf(s1, dv[1], pa);
      pa = fmaf(fmaf(-C, s1, b1), xg.y, pa);
      pb = fmaf(fmaf(-C, s2, b2), xg.x, pb);
      pb = fmaf(s3, dv[3], pb);
      pb = fmaf(fmaf(-C, s3, b3), xg.y, pb);
      pa += __shfl_xor_sync(0xffffffffu, pa, 1);
      pb += __shfl_xor_sync(0xffffffffu, pb, 1);
      if (t == 0) {
        red[U.slot] = pa;
        red[U.slot + 8 * SKP] = pb;
      }
    };
    for (int st = 0; st < nst; ++st) {
      const int buf = st % geo.nbuf;
      const int a0 = T0 + st * geo.stage_tiles, a1 = min(T1, a0 + geo.stage_tiles);
      if (wait_or_abort(&full[buf], (uint32_t)((st / geo.nbuf) & 1), abort_flag, a.status)) {
        const int units = (a1 - a0) * 2;  // (tile, half-span)
        const unsigned char* sbase = bufs + (size_t)buf * geo.stage_bytes;
        // two units at a time, interleaved quad by quad: eight independent
        // accumulator chains, and one unit's drain overlaps the other's math
        int u = warp;
        for (; u + kConsumers < units; u += 2 * kConsumers) {
          const Unit A = unit(u, a0, sbase), B = unit(u + kConsumers, a0, sbase);
          float dA[4][4], dB[4][4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dA[i][0] = dA[i][1] = dA[i][2] = dA[i][3] = 0.f;
            dB[i][0] = dB[i][1] = dB[i][2] = dB[i][3] = 0.f;
          }
#pragma unroll
          for (int q = 0; q < QH; ++q) {
            quad(A, q, dA);
            quad(B, q, dB);
          }
          finish(A, dA);
          finish(B, dB);
        }
        if (u < units) {
          const Unit A = unit(u, a0, sbase);
          float dA[4][4];
#pragma unroll
          for (int i = 0; i < 4; ++i) dA[i][0] = dA[i][1] = dA[i][2] = dA[i][3] = 0.f;
#pragma unroll
          for (int q = 0; q < QH; ++q) quad(A, q, dA);
          finish(A, dA);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[buf]);
    }
  } else if (producer) {
    for (int st = issued; st < nst; ++st) {
      const int buf = st % geo.nbuf;
      if (!wait_or_abort(&empty[buf], (uint32_t)(((st / geo.nbuf) - 1) & 1), abort_flag, a.status)) break;
      fence_proxy_async();
      issue(st);
      issued = st + 1;
    }
    // never leave with copies in flight into this CTA's shared memory: the
    // last stage issued into each buffer must have landed
    if (*abort_flag) {
      for (int st = max(0, issued - geo.nbuf); st < issued; ++st)
        mbar_wait_bounded(&full[st % geo.nbuf], (uint32_t)((st / geo.nbuf) & 1), a.status);
      if (norm_pre) mbar_wait_bounded(nwbar, 0u, a.status);
    }
  }
  __syncthreads();

  // ---- epilogue: each logical row sums its slots in order ---------------
  const int nlog = (lb1 - lb0) * 16;
  for (int i = tid; i < nlog; i += kThreads) {
    const int lbl = i >> 4, r = i & 15;
    const int n = lb0 * 16 + i;
    const int prow = lbl * halves * 16 + r;
    float acc = 0.f;
    for (int j = 0; j < SKP; ++j) acc += red[prow * SKP + j];
    switch (a.epi) {
      case kEpiStore:
        a.y[n] = f2bf(acc);
        break;
      case kEpiResid: {
        const float rv = !res_early ? bf2f(a.res[n]) : (i < kThreads ? res_pre[0] : res_pre[1]);
        a.y[n] = f2bf(__fadd_rn(rv, bfround(acc)));
        break;
      }
      case kEpiSwiglu: {
        float accu = 0.f;
        for (int j = 0; j < SKP; ++j) accu += red[(prow + 16) * SKP + j];
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

  if (a.epi == kEpiArgmax) {
    // CTA-level (max, first index), then the last CTA to finish reduces all
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best_v || (ov == best_v && oi < best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    __shared__ float wv[kConsumers + 1];
    __shared__ int wi[kConsumers + 1];
    __shared__ unsigned last;
    if (lane == 0) {
      wv[warp] = best_v;
      wi[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
      float bv = wv[0];
      int bi = wi[0];
      for (int w = 1; w <= kConsumers; ++w)
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
    if (last) {
      __threadfence();
      // all CTAs' partials, one warp, all loads in flight at once
      if (warp == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < (int)gridDim.x; c += 32) {
          const float v = __ldcg(a.am_val + c);
          const int i = __ldcg(a.am_idx + c);
          if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
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
  }
}

// ------------------------------------------------------------------ packing
// One thread per (tile, lane, half-span, slice quad): the lane's words of
// four slices (and, for quad 0 of lanes t < 2, its scale/bias record).
template <int BITS>
__global__ void pack_kernel(const uint32_t* __restrict__ w, const bf16* __restrict__ s, const bf16* __restrict__ b,
                            int N, int K, int gs, PackMap map, int S, int tile_bytes, long long units,
                            unsigned char* __restrict__ dst) {
  const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= units) return;
  const int QH = gs / 16, HW = BITS / 4, per = 32 / BITS;
  const int q = (int)(u % QH);
  const int hs = (int)((u / QH) % 2);
  const int lane = (int)((u / (2 * QH)) % 32);
  const long long tile = u / (64 * QH);
  const long long p = tile / S;
  const int sp = (int)(tile % S);
  const int g = lane >> 2, t = lane & 3;
  const int lbs_block = map.R / 16;  // packed row blocks per source block
  const long long e = p / lbs_block;
  const int pin = (int)(p % lbs_block);
  const int lb_in = pin / map.halves, half = pin % map.halves;
  const long long row0 = e * map.R + (long long)half * (map.R / map.halves) + (long long)lb_in * 16;
  const int ng = K / gs;
  auto code = [&](long long row, int G, int k) -> uint32_t {
    const int grp = sp * 8 + G;
    if (row >= N || grp >= ng) return 0u;
    const int col = grp * gs + k;
    return (w[row * (K / per) + col / per] >> (BITS * (col % per))) & ((1u << BITS) - 1u);
  };
  const long long rA = row0 + g, rB = row0 + g + 8;
  const int G = hs * 4 + t;
  const int a_bytes = 16 * 8 * gs * BITS / 8;
  unsigned char* tbase = dst + tile * tile_bytes;
  for (int wi = 0; wi < 4; ++wi) {
    const int k = 4 * (4 * q + wi);  // first of the slice's four group offsets
    unsigned char* wp = tbase + ((hs * QH + q) * HW) * 512 + lane * 16 + wi * 4;
    if (BITS == 4) {
      const uint32_t word = code(rA, G, k) | (code(rB, G, k) << 4) | (code(rA, G, k + 2) << 8) |
                            (code(rB, G, k + 2) << 12) | (code(rA, G, k + 1) << 16) | (code(rB, G, k + 1) << 20) |
                            (code(rA, G, k + 3) << 24) | (code(rB, G, k + 3) << 28);
      *reinterpret_cast<uint32_t*>(wp) = word;
    } else {
      const uint32_t w0 = code(rA, G, k) | (code(rB, G, k) << 8) | (code(rA, G, k + 1) << 16) | (code(rB, G, k + 1) << 24);
      const uint32_t w1 =
          code(rA, G, k + 2) | (code(rB, G, k + 2) << 8) | (code(rA, G, k + 3) << 16) | (code(rB, G, k + 3) << 24);
      *reinterpret_cast<uint32_t*>(wp) = w0;
      *reinterpret_cast<uint32_t*>(wp + 512) = w1;
    }
  }
  if (q == 0 && t < 2) {
    auto sbv = [&](const bf16* src, long long row, int Gi) -> uint32_t {
      const int grp = sp * 8 + Gi;
      if (row >= N || grp >= ng) return 0u;
      const bf16 v = src[row * ng + grp];
      return (uint32_t)(*reinterpret_cast<const uint16_t*>(&v));
    };
    const int G0 = hs * 4 + 2 * t;
    uint4 r;
    r.x = sbv(s, rA, G0) | (sbv(s, rA, G0 + 1) << 16);
    r.y = sbv(s, rB, G0) | (sbv(s, rB, G0 + 1) << 16);
    r.z = sbv(b, rA, G0) | (sbv(b, rA, G0 + 1) << 16);
    r.w = sbv(b, rB, G0) | (sbv(b, rB, G0 + 1) << 16);
    *reinterpret_cast<uint4*>(tbase + a_bytes + hs * 256 + (g * 2 + t) * 16) = r;
  }
}

void make_pgeom(int N, int K, int bits, int gs, int epi, const PgemvPlan& p, PGeom* g) {
  g->K = K;
  g->ng = K / gs;
  g->S = (g->ng + 7) / 8;
  g->tile_bytes = ptile_bytes(bits, gs);
  g->a_bytes = g->tile_bytes - 512;
  g->halves = epi == kEpiSwiglu ? 2 : 1;
  g->lb_total = p.lb_total;
  g->stage_tiles = p.stage_tiles;
  g->nbuf = p.nbuf;
  g->stage_bytes = p.stage_tiles * g->tile_bytes;
  g->x_slots = p.x_slots;
  g->xk = g->S * 8 * gs;
  g->gstride = 2 * gs + 16;
  g->xslot_bytes = g->S * 8 * g->gstride;
  g->red_rows = p.lbs_max * g->halves * 16;
  g->nw_bytes = (p.x_slots == 1 && K <= 8192) ? ((K * 2 + 15) & ~15) : 0;
  const unsigned long long lbt = (unsigned long long)g->halves * g->S;
  g->lbt_magic = (0x100000000ull + lbt - 1) / lbt;
  g->lps_magic = 0;
  (void)N;
  pgeom_layout(*g, gs);
}

}  // namespace

size_t pgemv_tile_bytes(int bits, int gs) { return (size_t)ptile_bytes(bits, gs); }

size_t pgemv_packed_bytes(int N, int K, int bits, int gs, const PackMap& map) {
  (void)map;
  const int S = (K / gs + 7) / 8;
  const size_t rb = (size_t)(N + 15) / 16;
  return rb * S * pgemv_tile_bytes(bits, gs);
}

cudaError_t pgemv_pack(const uint32_t* w, const bf16* s, const bf16* b, int N, int K, int bits, int gs,
                       const PackMap& map, unsigned char* dst, cudaStream_t st) {
  if (!(bits == 4 || bits == 8) || !(gs == 32 || gs == 64 || gs == 128) || K % gs != 0) return cudaErrorInvalidValue;
  if (map.R % (16 * map.halves) != 0 || (long long)map.blocks * map.R != N) return cudaErrorInvalidValue;
  const int S = (K / gs + 7) / 8;
  const long long tiles = (long long)(N / 16) * S;
  const long long units = tiles * 32 * 2 * (gs / 16);
  const int tb = ptile_bytes(bits, gs);
  const int threads = 256;
  const unsigned blocks = (unsigned)((units + threads - 1) / threads);
  if (bits == 4)
    pack_kernel<4><<<blocks, threads, 0, st>>>(w, s, b, N, K, gs, map, S, tb, units, dst);
  else
    pack_kernel<8><<<blocks, threads, 0, st>>>(w, s, b, N, K, gs, map, S, tb, units, dst);
  return cudaGetLastError();
}

int pgemv_make_plan(int N, int K, int bits, int gs, int epi, int x_slots, int num_sms, int budget, PgemvPlan* plan,
                    int ctas_per_sm) {
  if (!(bits == 4 || bits == 8) || !(gs == 32 || gs == 64 || gs == 128)) return -1;
  if (K <= 0 || N <= 0 || K % gs != 0) return -1;
  const bool sw = epi == kEpiSwiglu;
  if (sw && (N % 2 != 0)) return -1;
  const int halves = sw ? 2 : 1;
  const int lrows = N / halves;
  if (lrows % 16 != 0) return -1;
  const int LB = lrows / 16;
  PgemvPlan p{};
  p.halves = halves;
  p.lb_total = LB;
  p.x_slots = x_slots > 1 ? x_slots : 1;
  p.grid = std::max(1, std::min(LB, num_sms * std::max(1, ctas_per_sm)));
  p.lbs_max = (LB + p.grid - 1) / p.grid;
  const int S = (K / gs + 7) / 8;
  const int tb = ptile_bytes(bits, gs);
  const int tiles_max = p.lbs_max * halves * S;
  // stages of about 40 KB, then as many ring slots as the budget holds (up
  // to every stage: the whole share resident); smaller stages when that
  // leaves fewer than two slots for a streamed share
  const int st_hi = std::max(1, std::min(tiles_max, 40960 / tb));
  PgemvPlan fallback{};
  bool have_fallback = false;
  for (int st_tiles = st_hi; st_tiles >= 1; st_tiles = st_tiles > 1 ? st_tiles / 2 : 0) {
    p.stage_tiles = st_tiles;
    const int nst = (tiles_max + st_tiles - 1) / st_tiles;
    PGeom g;
    p.nbuf = 0;
    make_pgeom(N, K, bits, gs, epi, p, &g);
    const int fit = (budget - g.off_buf) / (st_tiles * tb);
    const int nbuf = std::min(std::min(nst, kMaxBuf), fit);
    if (nbuf < 1) continue;
    p.nbuf = nbuf;
    make_pgeom(N, K, bits, gs, epi, p, &g);
    p.smem = pgeom_layout(g, gs);
    if (nbuf >= std::min(nst, 2)) {
      *plan = p;
      return 0;
    }
    if (!have_fallback) {
      fallback = p;
      have_fallback = true;
    }
  }
  if (have_fallback) {
    *plan = fallback;
    return 0;
  }
  return -1;
}

cudaError_t pgemv_launch(const GemvArgs& a, const PgemvPlan& p, cudaStream_t st, bool pdl) {
  if (a.pro != kProX && a.norm_groups > 8) return cudaErrorInvalidValue;
  if (a.pro != kProX && p.x_slots > 1) return cudaErrorInvalidValue;
  PGeom g;
  make_pgeom(a.N, a.K, a.bits, a.gs, a.epi, p, &g);
  if (p.x_slots > 1) {
    if (a.slot_rows < 16 || a.slot_rows % 16 != 0) return cudaErrorInvalidValue;
    const unsigned long long lps = (unsigned long long)(a.slot_rows / 16);
    g.lps_magic = (0x100000000ull + lps - 1) / lps;
  }
  if (a.pro != kProX && (g.nw_bytes < a.K * 2 || (reinterpret_cast<uintptr_t>(a.norm_w) & 15) != 0))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
#define EMX_PGEMV_CASE(B, G)                                                                          \
  if (a.bits == B && a.gs == G) {                                                                     \
    auto kern = pgemv_kernel<B, G>;                                                                   \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem); \
    if (e != cudaSuccess) return e;                                                                   \
    return cudaLaunchKernelEx(&cfg, kern, a, g);                                                      \
  }
  EMX_PGEMV_CASE(4, 32)
  EMX_PGEMV_CASE(4, 64)
  EMX_PGEMV_CASE(4, 128)
  EMX_PGEMV_CASE(8, 32)
  EMX_PGEMV_CASE(8, 64)
  EMX_PGEMV_CASE(8, 128)
#undef EMX_PGEMV_CASE
  return cudaErrorInvalidValue;
}

}  // namespace emx
