// pgemv_dev.cuh — device pieces of the packed batch-1 GEMV, shared by the
// one-matrix kernel (pgemv.cu) and the persistent decode-step kernel
// (step.cu): the per-launch geometry, the x prologue (plain / RMSNorm /
// embedding + norm / residual add + norm), the consumption of one pipeline
// stage of packed tiles, and the per-row epilogue.
//
// The packed layout these functions read is described in pgemv.cuh.  The
// math per unit (16 rows x one half-span of 4 groups):
//   one conflict-free 128-bit shared load per word set gives four slices' A
//   registers; a LOP3 per register places codes in the mantissa of an fp16
//   1024 (magic-number exponent, exact: 1024 + q, or 1024 + 16 q for the
//   upper nibble of an int4 byte) and an m16n8k16 f16 MMA per slice adds the
//   four group dot products of rows g, g+8 at once: column j < 4 of B holds
//   x masked to group j, so only the lanes with g == t load x and the other
//   lanes read a zero block.  x is staged in fp16 after an exact
//   power-of-two scaling x' = x * 2^-e that keeps the largest |x'| below 2^15
//   (so every bf16 value above 2^-14 of the largest keeps all its bits); the
//   x elements that meet an upper nibble are stored as x' / 16.  Then per row
//   s*(dot - 1024*sum x'') + b*sum x' in fp32 (the MLX qmv factorisation; the
//   1024 offsets cancel against the sum of the staged fp16 values x''),
//   reduced over the lane pair and stored to a per-(row, span, half-span)
//   slot; the epilogue sums a row's slots in a fixed order and multiplies by
//   2^e, so the result does not depend on which CTA or warp computed a unit.
#pragma once
#include "attn_decode.cuh"
#include "qgemv.cuh"

namespace emx {
namespace pg {

constexpr int kMaxBuf = 8;

struct PGeom {
  int K, ng, S;
  int bits;  // code width: int4 rows stage their upper-nibble x elements as x' / 16
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
  int xsl_mod;  // 0: slots of consecutive blocks; else blocks interleave the slots (x slot = block % xsl_mod,
                // read by pg_stage<..., true>)
  int off_x, off_nw, off_zero, off_xs, off_red, off_buf;
};

__host__ __device__ inline int ptile_bytes(int bits, int gs) { return 16 * 8 * gs * bits / 8 + 512; }

// Shared-memory carve-up from byte `base` on: x slots, norm weights, the zero
// block, the per-group sums of x (pairs of groups: 1024 * sum x'' of both,
// then sum x' of both), the row-slot reduction area, then the stage ring.
__host__ __device__ inline int pgeom_layout(PGeom& g, int gs, int base = 384) {
  g.off_x = base;
  g.off_nw = g.off_x + g.x_slots * g.xslot_bytes;
  g.off_zero = g.off_nw + g.nw_bytes;
  g.off_xs = g.off_zero + 2 * gs;
  g.off_red = g.off_xs + ((g.x_slots * g.S * 8 * 8 + 15) & ~15);
  g.off_buf = (g.off_red + g.red_rows * g.S * 2 * 4 + 127) & ~127;
  return g.off_buf + g.nbuf * g.stage_bytes;
}

// Geometry of one matrix for a plan of `lbs_max` logical blocks per CTA.
inline void pgeom_make(PGeom* g, int K, int bits, int gs, int epi, int lb_total, int stage_tiles, int nbuf,
                       int x_slots, int lbs_max, bool norm_room) {
  g->K = K;
  g->bits = bits;
  g->ng = K / gs;
  g->S = (g->ng + 7) / 8;
  g->tile_bytes = ptile_bytes(bits, gs);
  g->a_bytes = g->tile_bytes - 512;
  g->halves = epi == kEpiSwiglu ? 2 : 1;
  g->lb_total = lb_total;
  g->stage_tiles = stage_tiles;
  g->nbuf = nbuf;
  g->stage_bytes = stage_tiles * g->tile_bytes;
  g->x_slots = x_slots;
  g->xk = g->S * 8 * gs;
  g->gstride = 2 * gs + 16;
  g->xslot_bytes = g->S * 8 * g->gstride;
  g->red_rows = lbs_max * g->halves * 16;
  g->nw_bytes = norm_room ? ((K * 2 + 15) & ~15) : 0;
  const unsigned long long lbt = (unsigned long long)g->halves * g->S;
  g->lbt_magic = (0x100000000ull + lbt - 1) / lbt;
  g->lps_magic = 0;
  g->xsl_mod = 0;
}

// Barrier over the threads that take part in a phase: the whole CTA, or the
// consumer warps only (named barrier 1) while a producer warp runs ahead.
struct SyncCta {
  __device__ static void sync() { __syncthreads(); }
};
template <int N>
struct SyncNamed {
  __device__ static void sync() { asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory"); }
};

template <class Sync>
__device__ __forceinline__ float part_sum(float v, float* scratch, int tid, int nthr) {
  const int lane = tid & 31, warp = tid >> 5, nw = (nthr + 31) >> 5;
  v = warp_sum(v);
  Sync::sync();
  if (lane == 0) scratch[warp] = v;
  Sync::sync();
  float t = tid < nw ? scratch[tid] : 0.0f;
  if (warp == 0) t = warp_sum(t);
  if (tid == 0) scratch[0] = t;
  Sync::sync();
  const float r = scratch[0];
  Sync::sync();
  return r;
}

// Bounded wait that also gives up at once when another warp has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_test_wait(bar, parity)) return true;
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
// `psrc` (kProAddNorm with a peer sum): the world ranks' fp32 partials.
__device__ __forceinline__ void src8(const GemvArgs& a, int c, int tok, float (&v)[8],
                                     const float* const* psrc = nullptr, int pworld = 0) {
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
    } else if (psrc) {
      // the ranks' partials summed in rank order (the same bits on every
      // rank); a TP sum is then rounded like the unsharded projection's bf16
      // output (add_round), an EP expert sum is not
#pragma unroll
      for (int e = 0; e < 8; ++e) add[e] = 0.f;
      for (int r = 0; r < pworld; ++r) {
        const float4 p0 = __ldcg(reinterpret_cast<const float4*>(psrc[r] + k0));
        const float4 p1 = __ldcg(reinterpret_cast<const float4*>(psrc[r] + k0 + 4));
        add[0] += p0.x, add[1] += p0.y, add[2] += p0.z, add[3] += p0.w;
        add[4] += p1.x, add[5] += p1.y, add[6] += p1.z, add[7] += p1.w;
      }
      if (a.add_round) {
#pragma unroll
        for (int e = 0; e < 8; ++e) add[e] = bfround(add[e]);
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

// Shared-memory views of one phase (offsets from the geometry).
struct PgSmem {
  unsigned char* xsm;  // x: [slot][group][gs bf16 + 16 pad bytes]
  unsigned char* zero; // read as B by the lanes that carry no x
  float* xs;           // group sums of x
  float* red;          // row slots
};

__device__ __forceinline__ PgSmem pg_smem(unsigned char* smem, const PGeom& geo) {
  PgSmem s;
  s.xsm = smem + geo.off_x;
  s.zero = smem + geo.off_zero;
  s.xs = reinterpret_cast<float*>(smem + geo.off_xs);
  s.red = reinterpret_cast<float*>(smem + geo.off_red);
  return s;
}

// Byte address of 8-element chunk c of x slot `slot` (groups of gs
// elements sit gstride bytes apart).
template <int GS>
__device__ __forceinline__ unsigned char* pg_xchunk(const PGeom& geo, const PgSmem& sm, int slot, int c) {
  constexpr int CPG = GS / 8;  // 8-element chunks per group
  return sm.xsm + (size_t)slot * geo.xslot_bytes + (c / CPG) * geo.gstride + (c % CPG) * 16;
}

// Exponent e of the power-of-two staging scale for values of magnitude at
// most `bound`: |v| * 2^-e < 2^15 (bound < 2^E from the float's own exponent
// field, e = E - 15), clamped to [-111, 113] so that 2^e, 2^-e and
// 2^-(e+4) are normal floats.  bound <= 0 or NaN: 0.
__device__ __forceinline__ int pg_scale_exp(float bound) {
  if (!(bound > 0.f)) return 0;
  const int E = (int)((__float_as_uint(bound) >> 23) & 0xffu) - 126;
  return min(max(E - 15, -111), 113);
}

// 2^e as a float, -126 <= e <= 127.
__device__ __forceinline__ float pg_pow2(int e) { return __int_as_float((127 + e) << 23); }

// Two floats to packed fp16 (round to nearest even).
__device__ __forceinline__ uint32_t h2bits(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Block-wide (sum, max, max) of three per-thread values over the threads
// [0, nthr) that call it; every thread gets the result (warp totals summed
// in warp order).  `scratch` holds >= 3 * warps floats.
template <class Sync>
__device__ __forceinline__ float3 part_reduce3(float s, float m1, float m2, float* scratch, int tid, int nthr) {
  const int lane = tid & 31, warp = tid >> 5, nw = (nthr + 31) >> 5;
  s = warp_sum(s);
  m1 = warp_max(m1);
  m2 = warp_max(m2);
  Sync::sync();
  if (lane == 0) {
    scratch[warp] = s;
    scratch[nw + warp] = m1;
    scratch[2 * nw + warp] = m2;
  }
  Sync::sync();
  float3 r = make_float3(0.f, 0.f, 0.f);
  for (int w = 0; w < nw; ++w) {
    r.x += scratch[w];
    r.y = fmaxf(r.y, scratch[nw + w]);
    r.z = fmaxf(r.z, scratch[2 * nw + w]);
  }
  return r;
}

// Stores chunk c (values `o`, bf16 values held as floats) of x slot `slot`
// in fp16 scaled by sc = 2^-e (the elements k % 4 >= 2 of an int4 matrix by
// sc / 16: they meet the upper nibble, whose magic-number code is 16x) and,
// from the CPG lanes that hold one group (consecutive c in consecutive lanes;
// all 32 lanes call), the group's 1024 * sum x'' and sum x'.
template <int GS>
__device__ __forceinline__ void pg_emit(const PGeom& geo, const PgSmem& sm, int slot, int c, bool valid,
                                        const float (&o)[8], float sc) {
  constexpr int CPG = GS / 8;
  const float sh = geo.bits == 4 ? sc * 0.0625f : sc;
  float sx = 0.f, sxx = 0.f;
  if (valid) {
    float h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xs = __fmul_rn(o[e], sc);
      h[e] = __half2float(__float2half_rn((e & 2) ? __fmul_rn(o[e], sh) : xs));
      sx += xs;
      sxx += h[e];
    }
    uint4 pk;
    pk.x = h2bits(h[0], h[1]);
    pk.y = h2bits(h[2], h[3]);
    pk.z = h2bits(h[4], h[5]);
    pk.w = h2bits(h[6], h[7]);
    *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, slot, c)) = pk;
  }
#pragma unroll
  for (int off = 1; off < CPG; off <<= 1) {
    sx += __shfl_xor_sync(0xffffffffu, sx, off);
    sxx += __shfl_xor_sync(0xffffffffu, sxx, off);
  }
  if (valid && (c % CPG) == 0) {
    const int G = c / CPG;
    float* p = sm.xs + (size_t)slot * geo.S * 16 + (G >> 1) * 4 + (G & 1);
    p[0] = 1024.0f * sxx;
    p[2] = sx;
  }
}

// Zero padding after x: x past K (whole chunks), the zero block, group sums
// past ng.
template <int GS>
__device__ __forceinline__ void pg_pad(const PGeom& geo, const PgSmem& sm, int tid, int nthr) {
  const int nch = geo.K / 8;
  const int pad = (geo.xk - geo.K) / 8;  // chunks
  for (int i = tid; i < geo.x_slots * pad; i += nthr)
    *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, i / pad, nch + i % pad)) = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < GS / 2; i += nthr) reinterpret_cast<uint32_t*>(sm.zero)[i] = 0u;
  const int S = geo.S;
  const int gpad = S * 8 - geo.ng;
  for (int i = tid; i < geo.x_slots * gpad; i += nthr) {
    const int G = geo.ng + i % gpad;
    float* p = sm.xs + (size_t)(i / gpad) * S * 16 + (G >> 1) * 4 + (G & 1);
    p[0] = 0.f;
    p[2] = 0.f;
  }
}

// The staged bf16 source of x slots [0, nslots) (by any of the threads: the
// reduction's barrier orders it), max |x| per thread in `mx`: one reduction
// fixes the scale, then the threads convert the chunks to the fp16 layout.
template <int GS, class Sync>
__device__ __forceinline__ void pg_convert_staged(const PGeom& geo, const PgSmem& sm, int nslots, float mx,
                                                  float* scratch, float* xsc, int tid, int nthr) {
  const float3 r = part_reduce3<Sync>(0.f, mx, 0.f, scratch, tid, nthr);
  const int e = pg_scale_exp(r.y);
  const float sc = pg_pow2(-e);
  if (tid == 0) *xsc = pg_pow2(e);
  // all slots' chunks in one sweep (K is whole groups, so a group's chunks
  // stay in consecutive lanes)
  const int nch = geo.K / 8, tot = nslots * nch;
#pragma unroll 1
  for (int it = 0; it * nthr < tot; ++it) {
    const int i = it * nthr + tid;
    const bool valid = i < tot;
    const int slot = nslots > 1 ? i / nch : 0;
    const int c = i - slot * nch;
    float v[8];
    if (valid) {
      unpack8f(*reinterpret_cast<const uint4*>(pg_xchunk<GS>(geo, sm, slot, c)), v);
    } else {
#pragma unroll
      for (int e2 = 0; e2 < 8; ++e2) v[e2] = 0.f;
    }
    pg_emit<GS>(geo, sm, slot, c, valid, v, sc);
  }
}

// kProMerge: x = the decode attention output, merged from the splits'
// partials when the attention deferred its merge (1 <= splits <=
// kAttnDeferSplits), with the attention's own arithmetic (attn_decode.cu):
// M = max m_s, w_s = exp(m_s - M), den = the butterfly sum of fma(w_s, l_s)
// over the split lanes, out = bf16(sum_s fma(w_s / den, acc_s)) in split
// order -- the bits the attention's merge would store.  The merged bf16
// values are staged in x slot 0 (chunk c by thread c % nthr) and their max
// |x| accumulated in `mx`.  Returns false when the attention merged itself
// (x is then read from a.x).
template <int GS>
__device__ __forceinline__ bool pg_merge_attn(const GemvArgs& a, const PGeom& geo, const PgSmem& sm, int tid,
                                              int nthr, bool lead, float& mx) {
  const int ns = attn_active_splits(*a.attn_pos + 1, a.attn_grid);
  if (ns < 1 || ns > kAttnDeferSplits) return false;
  constexpr int HD = 128, PS = HD + 2;
  const int hpg = a.attn_hpg;
  const size_t sstride = (size_t)hpg * PS;  // between the splits of one head
  const int nch = geo.K / 8;
  for (int c = tid; c < nch; c += nthr) {
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    const int q = c / (HD / 8), d0 = (c % (HD / 8)) * 8;
    const float* pb = a.attn_part + ((size_t)(q / hpg) * ns * hpg + (q % hpg)) * PS;
    float ms[kAttnDeferSplits], ls[kAttnDeferSplits];
    float2 v[kAttnDeferSplits][4];
#pragma unroll
    for (int s2 = 0; s2 < kAttnDeferSplits; ++s2) {
      ms[s2] = -INFINITY;
      ls[s2] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) v[s2][j] = make_float2(0.f, 0.f);
      if (s2 < ns) {
        const float* ps = pb + s2 * sstride;
        ms[s2] = __ldcg(ps);
        ls[s2] = __ldcg(ps + 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[s2][j] = __ldcg(reinterpret_cast<const float2*>(ps + 2 + d0 + 2 * j));
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < kAttnDeferSplits; ++s2) M = fmaxf(M, ms[s2]);
    float w[kAttnDeferSplits], t[kAttnDeferSplits];
#pragma unroll
    for (int s2 = 0; s2 < kAttnDeferSplits; ++s2) {
      w[s2] = ms[s2] == -INFINITY ? 0.f : expf(ms[s2] - M);
      t[s2] = fmaf(w[s2], ls[s2], 0.f);
    }
    static_assert(kAttnDeferSplits == 4, "the butterfly below covers four split lanes");
    const float den = (t[0] + t[2]) + (t[1] + t[3]);
#pragma unroll
    for (int s2 = 0; s2 < kAttnDeferSplits; ++s2) {
      if (s2 < ns) {
        const float sw = __fdiv_rn(w[s2], den);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[2 * j] = fmaf(sw, v[s2][j].x, o[2 * j]);
          o[2 * j + 1] = fmaf(sw, v[s2][j].y, o[2 * j + 1]);
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      o[e] = bfround(o[e]);
      mx = fmaxf(mx, fabsf(o[e]));
    }
    const uint4 pk = pack8exact(o);
    *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, 0, c)) = pk;
    if (lead && a.x_out) *reinterpret_cast<uint4*>(a.x_out + c * 8) = pk;
  }
  return true;
}

// x prologue: x in padded groups (zero past K to whole spans), fp16 after the
// power-of-two scale (2^e to *xsc), and the group sums, built by threads
// [0, nthr).  The `lead` CTA also stores the new residual of embedding / add
// prologues to a.x_out.  Norm prologues take the weights from `nwsm`, which
// becomes valid when `nwbar` completes phase `nw_parity` (nwbar == nullptr:
// already valid); their scale comes from the bound max|v| * inv * max|w| of
// the normalised values.  `scratch` holds >= 32 floats, `inv` 8.
template <int GS, class Sync>
__device__ __forceinline__ void pg_prologue(const GemvArgs& a, const PGeom& geo, const PgSmem& sm,
                                            const bf16* nwsm, uint64_t* nwbar, uint32_t nw_parity, float* scratch,
                                            float* inv, float* xsc, volatile int* abort_flag, int tok, int tid,
                                            int nthr, bool lead) {
  const int K = geo.K;
  const int nch = K / 8;
  const bool norm = a.pro == kProNorm || a.pro == kProEmbedNorm || a.pro == kProAddNorm;
  if (!norm) {
    // the source in bf16 (merged attention output, or x as given in every
    // slot), then one scale for all of it
    float mx = 0.f;
    const bool merged = a.pro == kProMerge && pg_merge_attn<GS>(a, geo, sm, tid, nthr, lead, mx);
    const int nslots = merged ? 1 : geo.x_slots;
    if (!merged) {
      for (int slot = 0; slot < nslots; ++slot) {
#pragma unroll 1
        for (int c = tid; c < nch; c += nthr) {
          const uint4 raw = *reinterpret_cast<const uint4*>(a.x + (size_t)slot * K + c * 8);
          float v[8];
          unpack8f(raw, v);
#pragma unroll
          for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[e]));
          *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, slot, c)) = raw;
        }
      }
    }
    pg_convert_staged<GS, Sync>(geo, sm, nslots, mx, scratch, xsc, tid, nthr);
  } else {
    // pass 1: pre-norm source staged in the x buffer, sums of squares per
    // norm group, max |v|
    const int groups = a.norm_groups > 0 ? a.norm_groups : 1;
    const int gd = K / groups;
    const bool store = (a.pro == kProEmbedNorm || a.pro == kProAddNorm) && lead && a.x_out;
    // a peer sum: wait until every rank has published reduction e (bounded),
    // then read the ranks' slots
    const float* psrc[kPeerMaxRanks];
    int pworld = 0;
    if (a.pro == kProAddNorm && a.peer) {
      const PeerX& P = *a.peer;
      const unsigned e = *P.epoch;
      pworld = P.world;
      for (int r = 0; r < kPeerMaxRanks; ++r) psrc[r] = r < pworld ? peer_slot(P, P.rank, e, r) : nullptr;
      if (tid == 0) {
        for (int r = 0; r < pworld; ++r) {
          if (r == P.rank) continue;
          const unsigned* flag = peer_flag(P, P.rank, r);
          const uint64_t t0 = globaltimer_ns();
          uint32_t i = 0;
          while ((int)(ld_acquire_sys_u32(flag) - e) < 0) {
            if ((++i & 63u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
              report_status(a.status, kDevTimeoutPeer);
              break;
            }
          }
        }
      }
      Sync::sync();
    }
    float ssg[8];
#pragma unroll
    for (int gi = 0; gi < 8; ++gi) ssg[gi] = 0.f;
    float mv = 0.f;
#pragma unroll 1
    for (int c = tid; c < nch; c += nthr) {
      float v[8];
      src8(a, c, tok, v, pworld ? psrc : nullptr, pworld);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss = fmaf(v[e], v[e], ss);
        mv = fmaxf(mv, fabsf(v[e]));
      }
      const int grp = (c * 8) / gd;
#pragma unroll
      for (int gi = 0; gi < 8; ++gi)
        if (grp == gi) ssg[gi] += ss;
      const uint4 pk = pack8exact(v);
      *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, 0, c)) = pk;
      if (store) *reinterpret_cast<uint4*>(a.x_out + c * 8) = pk;
    }
    // the norm weights (requested before the dependency wait) and their max
    if (nwbar && !wait_or_abort(nwbar, nw_parity, abort_flag, a.status)) {
      // no weights: the outputs are garbage and the status word says so
    }
    float mw = 0.f;
#pragma unroll 1
    for (int c = tid; c < nch; c += nthr) {
      float w[8];
      unpack8f(*reinterpret_cast<const uint4*>(nwsm + c * 8), w);
#pragma unroll
      for (int e = 0; e < 8; ++e) mw = fmaxf(mw, fabsf(w[e]));
    }
    float iv1 = 0.f, ivmax = 0.f, vmax = 0.f, wmax = 0.f;
    for (int gi = 0; gi < groups; ++gi) {
      float sv = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q == gi) sv = ssg[q];
      const float3 r = part_reduce3<Sync>(sv, mv, mw, scratch, tid, nthr);
      const float iv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(r.x, (float)gd), a.eps)));
      if (gi == 0) iv1 = iv;
      if (groups > 1 && tid == 0) inv[gi] = iv;
      ivmax = fmaxf(ivmax, iv);
      vmax = r.y;
      wmax = r.z;
    }
    if (groups > 1) Sync::sync();
    // |bf16(bf16(v * inv) * w)| <= max|v| * inv * max|w| * (1 + 2^-8)^2
    const int e = pg_scale_exp(vmax * ivmax * wmax * 1.02f);
    const float sc = pg_pow2(-e);
    if (tid == 0) *xsc = pg_pow2(e);
    // pass 2: scale and weight in place (each thread rewrites its own chunks)
#pragma unroll 1
    for (int it = 0; it * nthr < nch; ++it) {
      const int c = it * nthr + tid;
      const bool valid = c < nch;
      float o[8];
      if (valid) {
        float v[8], w[8];
        unpack8f(*reinterpret_cast<const uint4*>(pg_xchunk<GS>(geo, sm, 0, c)), v);
        unpack8f(*reinterpret_cast<const uint4*>(nwsm + c * 8), w);
        const float iv = groups == 1 ? iv1 : inv[(c * 8) / gd];
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2)
          o[e2] = groups == 1 ? bfround(__fmul_rn(bfround(__fmul_rn(v[e2], iv)), w[e2]))
                              : bfround(__fmul_rn(__fmul_rn(v[e2], iv), w[e2]));
      } else {
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) o[e2] = 0.f;
      }
      pg_emit<GS>(geo, sm, 0, c, valid, o, sc);
    }
  }
  pg_pad<GS>(geo, sm, tid, nthr);
}

// One stage of packed tiles [a0, a1) (global tile indices; the stage's bytes
// at `sbase`) for warp `warp` of `nwarps` consumer warps.  Units (tile,
// half-span) are dealt round-robin starting at warp `rot`, so that stages
// with fewer units than warps still spread over all of them; each warp runs
// two units at once, interleaved quad by quad (eight independent accumulator
// chains; one unit's drain overlaps the other's math).
template <int BITS, int GS, bool XSL_MOD = false>
__device__ __forceinline__ void pg_stage(const PGeom& geo, const PgSmem& sm, const unsigned char* sbase, int a0,
                                         int a1, int lb0, int warp, int lane, int nwarps, int rot) {
  constexpr int SPAN_K = 8 * GS;
  constexpr int QH = GS / 16;   // slice quads per half-span (4 groups)
  constexpr int HW = BITS / 4;  // word sets per quad
  constexpr int A_BYTES = 16 * SPAN_K * BITS / 8;
  const int halves = geo.halves, S = geo.S, SKP = S * 2;
  const int lb_tiles = halves * S;
  const int g = lane >> 2, t = lane & 3, t1 = t & 1;
  const bool has_x = g == t;  // the lanes whose B column carries x
  const uint32_t M16 = 0x64006400u;  // fp16 1024 in both halves: 1024 + code is exact
  // tile -> (logical block, half, span) by a 64-bit multiply, not a
  // division: floor(n / d) == (n * ceil(2^32 / d)) >> 32 for n < 2^32 / d
  // (the magic is 2^32 itself for d == 1, hence 64 bits; the host computes
  // it, a 64-bit division here would cost the critical path ~0.5 us)
  const unsigned long long lbt_magic = geo.lbt_magic;
  struct Unit {
    const unsigned char* aw;   // this lane's code words
    const unsigned char* px;   // x of the unit's group for this lane (or the zero block)
    const unsigned char* sbp;  // this lane's scale/bias record
    const float* xg;           // the group sums {1024 sum x'' (2 groups), sum x' (2 groups)}
    int slot;                  // red index of row g (row g+8 is 8 rows on)
  };
  auto unit = [&](int u) -> Unit {
    const int ti = u >> 1, hs = u & 1;
    const int gt = a0 + ti;
    const int lb = (int)(((unsigned long long)gt * lbt_magic) >> 32);
    const int rem = gt - lb * lb_tiles;
    const int h = rem >= S ? 1 : 0;
    const int sp = rem - h * S;
    // 0 unless x_slots > 1.  Interleaved slots take an integer remainder: the
    // multiply-shift form of the same quotient gave a warp's later units of a
    // stage the wrong slot here (measured against the per-kernel chain; the
    // cause was not found), the remainder is exact
    const int xsl = XSL_MOD ? lb % geo.xsl_mod : (int)(((unsigned long long)lb * geo.lps_magic) >> 32);
    const unsigned char* tile = sbase + (size_t)ti * geo.tile_bytes;
    Unit r;
    r.aw = tile + hs * (A_BYTES / 2) + lane * 16;
    r.px = has_x ? sm.xsm + (size_t)xsl * geo.xslot_bytes + (size_t)(sp * 8 + hs * 4 + t) * geo.gstride : sm.zero;
    r.sbp = tile + A_BYTES + hs * 256 + (g * 2 + t1) * 16;
    r.xg = sm.xs + (size_t)xsl * S * 16 + (sp * 4 + hs * 2 + t1) * 4;
    r.slot = (((lb - lb0) * halves + h) * 16 + g) * SKP + sp * 2 + hs;
    return r;
  };
  // slice quad q of a unit: HW code loads, two x loads, four MMAs into four
  // independent accumulators.  int4 word: nibbles 0 / 4 (bits 0-3, 16-19) row
  // g at k, k+1; nibbles 2 / 6 row g+8 at k, k+1; nibbles 1 / 5 row g at k+2,
  // k+3 (x16: x staged / 16 there); nibbles 3 / 7 row g+8 at k+2, k+3.  int8
  // words u (k, k+1) and v (k+2, k+3): bytes 0 / 2 row g, bytes 1 / 3 row g+8.
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
        const uint32_t w = w0v[j], w8 = w >> 8;
        mma_f16_16816(d[j], lop3_and_or(w, 0x000F000Fu, M16), lop3_and_or(w8, 0x000F000Fu, M16),
                      lop3_and_or(w, 0x00F000F0u, M16), lop3_and_or(w8, 0x00F000F0u, M16), bx[2 * j],
                      bx[2 * j + 1]);
      } else {
        const uint32_t u0 = w0v[j], u1 = w1v[j];
        mma_f16_16816(d[j], lop3_and_or(u0, 0x00FF00FFu, M16), lop3_and_or(u0 >> 8, 0x00FF00FFu, M16),
                      lop3_and_or(u1, 0x00FF00FFu, M16), lop3_and_or(u1 >> 8, 0x00FF00FFu, M16), bx[2 * j],
                      bx[2 * j + 1]);
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
    const float4 xg = *reinterpret_cast<const float4*>(U.xg);
    const float s0 = __uint_as_float(sb.x << 16), s1 = __uint_as_float(sb.x & 0xffff0000u);
    const float s2 = __uint_as_float(sb.y << 16), s3 = __uint_as_float(sb.y & 0xffff0000u);
    const float b0 = __uint_as_float(sb.z << 16), b1 = __uint_as_float(sb.z & 0xffff0000u);
    const float b2 = __uint_as_float(sb.w << 16), b3 = __uint_as_float(sb.w & 0xffff0000u);
    float pa = fmaf(s0, dv[0] - xg.x, b0 * xg.z);
    pa = fmaf(s1, dv[1] - xg.y, fmaf(b1, xg.w, pa));
    float pb = fmaf(s2, dv[2] - xg.x, b2 * xg.z);
    pb = fmaf(s3, dv[3] - xg.y, fmaf(b3, xg.w, pb));
    pa += __shfl_xor_sync(0xffffffffu, pa, 1);
    pb += __shfl_xor_sync(0xffffffffu, pb, 1);
    if (t == 0) {
      sm.red[U.slot] = pa;
      sm.red[U.slot + 8 * SKP] = pb;
    }
  };
  const int units = (a1 - a0) * 2;  // (tile, half-span)
  int u = warp - rot;
  if (u < 0) u += nwarps;
  for (; u + nwarps < units; u += 2 * nwarps) {
    const Unit A = unit(u), B = unit(u + nwarps);
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
    const Unit A = unit(u);
    float dA[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) dA[i][0] = dA[i][1] = dA[i][2] = dA[i][3] = 0.f;
#pragma unroll
    for (int q = 0; q < QH; ++q) quad(A, q, dA);
    finish(A, dA);
  }
}

// Residual values of a CTA's rows, loaded early so that their latency
// overlaps the prologue's (rows [lb0*16, lb0*16 + nlog), nlog <= 2*nthr).
__device__ __forceinline__ bool pg_res_early(const GemvArgs& a, int lb0, int lb1, int tid, int nthr,
                                             float (&res_pre)[2]) {
  res_pre[0] = res_pre[1] = 0.f;
  const int nlog = (lb1 - lb0) * 16;
  const bool early = a.epi == kEpiResid && nlog <= 2 * nthr;
  if (early) {
    if (tid < nlog) res_pre[0] = bf2f(a.res[lb0 * 16 + tid]);
    if (tid + nthr < nlog) res_pre[1] = bf2f(a.res[lb0 * 16 + tid + nthr]);
  }
  return early;
}

// Epilogue: each logical row of [lb0, lb1) sums its slots in order, scales
// the sum by xscale (2^e of the x staging) and the fused output step runs
// (argmax: this thread's best in best_v / best_i).
__device__ __forceinline__ void pg_epilogue(const GemvArgs& a, const PGeom& geo, const float* red, int lb0, int lb1,
                                            int tid, int nthr, bool res_early, const float (&res_pre)[2],
                                            float& best_v, int& best_i, float xscale) {
  const int halves = geo.halves, SKP = geo.S * 2;
  const int nlog = (lb1 - lb0) * 16;
  for (int i = tid; i < nlog; i += nthr) {
    const int lbl = i >> 4, r = i & 15;
    const int n = lb0 * 16 + i;
    const int prow = lbl * halves * 16 + r;
    float acc = 0.f;
    for (int j = 0; j < SKP; ++j) acc += red[prow * SKP + j];
    acc *= xscale;  // x was staged as x * 2^-e
    switch (a.epi) {
      case kEpiStore:
        a.y[n] = f2bf(acc);
        break;
      case kEpiResid: {
        const float rv = !res_early ? bf2f(a.res[n]) : (i < nthr ? res_pre[0] : res_pre[1]);
        a.y[n] = f2bf(__fadd_rn(rv, bfround(acc)));
        break;
      }
      case kEpiSwiglu: {
        float accu = 0.f;
        for (int j = 0; j < SKP; ++j) accu += red[(prow + 16) * SKP + j];
        accu *= xscale;
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
        if (a.peer) {
          // this rank's partial into every rank's region (peer stores)
          const PeerX& P = *a.peer;
          const unsigned e = *P.epoch + 1u;
          for (int d = 0; d < P.world; ++d) peer_slot(P, d, e, P.rank)[n] = acc;
        } else {
          a.yf[n] = acc;
        }
        break;
    }
  }
}

// After a peer-sum producer GEMV's epilogue (every thread of every CTA).
template <class Sync>
__device__ __forceinline__ void pg_peer_publish(const GemvArgs& a, int tid, unsigned* flag_last) {
  peer_publish<Sync>(*a.peer, tid, flag_last);
}

__device__ __forceinline__ void argmax_pair(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}

// Greedy token over all CTAs: the CTA's (max, first index) of threads
// [0, nwarps*32) goes to am_val/am_idx[cta]; the last CTA to finish (ticket)
// reduces all `ctas` partials, writes the token (+ history, position) and
// returns true.  `wv`/`wi` hold >= nwarps entries; `flag` one word.
template <class Sync>
__device__ __forceinline__ bool pg_argmax_merge(const GemvArgs& a, float best_v, int best_i, int cta, int ctas,
                                                int tid, int nwarps, float* wv, int* wi, unsigned* flag) {
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    argmax_pair(best_v, best_i, ov, oi);
  }
  if (lane == 0) {
    wv[warp] = best_v;
    wi[warp] = best_i;
  }
  Sync::sync();
  if (tid == 0) {
    float bv = wv[0];
    int bi = wi[0];
    for (int w = 1; w < nwarps; ++w) argmax_pair(bv, bi, wv[w], wi[w]);
    a.am_val[cta] = bv;
    a.am_idx[cta] = bi;
    __threadfence();
    *flag = (atomicAdd(a.am_ticket, 1u) == (unsigned)ctas - 1) ? 1u : 0u;
  }
  Sync::sync();
  const bool last = *flag != 0;
  if (!last) return false;
  __threadfence();
  // all CTAs' partials, one warp, all loads in flight at once
  if (warp == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < ctas; c += 32) argmax_pair(bv, bi, __ldcg(a.am_val + c), __ldcg(a.am_idx + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_pair(bv, bi, ov, oi);
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
  return true;
}

}  // namespace pg
}  // namespace emx
