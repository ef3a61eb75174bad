// pgemv_dev.cuh — device pieces of the packed batch-1 GEMV, shared by the
// one-matrix kernel (pgemv.cu) and the persistent decode-step kernel
// (step.cu): the per-launch geometry, the x prologue (plain / RMSNorm /
// embedding + norm / residual add + norm), the consumption of one pipeline
// stage of packed tiles, and the per-row epilogue.
//
// The packed layout these functions read is described in pgemv.cuh.  The
// math per unit (16 rows x one half-span of 4 groups):
//   one conflict-free 128-bit shared load per word set gives four slices' A
//   registers; a LOP3 per register turns codes into bf16 (magic-number
//   exponent, exact) and an m16n8k16 MMA per slice adds the four group dot
//   products of rows g, g+8 at once: column j < 4 of B holds x masked to
//   group j, so only the lanes with g == t load x and the other lanes read a
//   zero block.  Then per row s*dot + (b - C*s)*sum(x_g) in fp32 (the MLX qmv
//   factorisation, C being the magic offset), reduced over the lane pair and
//   stored to a per-(row, span, half-span) slot; the epilogue sums a row's
//   slots in a fixed order, so the result does not depend on which CTA or
//   warp computed a unit.
#pragma once
#include "attn_decode.cuh"
#include "qgemv.cuh"

namespace emx {
namespace pg {

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

// Shared-memory carve-up from byte `base` on: x slots, norm weights, the zero
// block, group sums of x, the row-slot reduction area, then the stage ring.
__host__ __device__ inline int pgeom_layout(PGeom& g, int gs, int base = 384) {
  g.off_x = base;
  g.off_nw = g.off_x + g.x_slots * g.xslot_bytes;
  g.off_zero = g.off_nw + g.nw_bytes;
  g.off_xs = g.off_zero + 2 * gs;
  g.off_red = g.off_xs + ((g.x_slots * g.S * 8 * 4 + 15) & ~15);
  g.off_buf = (g.off_red + g.red_rows * g.S * 2 * 4 + 127) & ~127;
  return g.off_buf + g.nbuf * g.stage_bytes;
}

// Geometry of one matrix for a plan of `lbs_max` logical blocks per CTA.
inline void pgeom_make(PGeom* g, int K, int bits, int gs, int epi, int lb_total, int stage_tiles, int nbuf,
                       int x_slots, int lbs_max, bool norm_room) {
  g->K = K;
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

// Stores chunk c (bf16 bits `raw`, values `o`) of x slot `slot` and, from
// the CPG lanes that hold one group (consecutive c in consecutive lanes; all
// 32 lanes call), the group's sum of x.
template <int GS>
__device__ __forceinline__ void pg_emit(const PGeom& geo, const PgSmem& sm, int slot, int c, bool valid, uint4 raw,
                                        const float (&o)[8]) {
  constexpr int CPG = GS / 8;
  float ps = 0.f;
  if (valid) {
    *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, slot, c)) = raw;
#pragma unroll
    for (int e = 0; e < 8; ++e) ps += o[e];
  }
#pragma unroll
  for (int off = 1; off < CPG; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
  if (valid && (c % CPG) == 0) sm.xs[slot * geo.S * 8 + c / CPG] = ps;
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
  for (int i = tid; i < geo.x_slots * gpad; i += nthr) sm.xs[(i / gpad) * S * 8 + geo.ng + i % gpad] = 0.f;
}

// kProMerge: x = the decode attention output, merged from the splits'
// partials when the attention deferred its merge (1 <= splits <=
// kAttnDeferSplits), with the attention's own arithmetic (attn_decode.cu):
// M = max m_s, w_s = exp(m_s - M), den = the butterfly sum of fma(w_s, l_s)
// over the split lanes, out = bf16(sum_s fma(w_s / den, acc_s)) in split
// order -- the bits the attention's merge would store.  Returns false when
// the attention merged itself (x is then read from a.x).
template <int GS>
__device__ __forceinline__ bool pg_merge_attn(const GemvArgs& a, const PGeom& geo, const PgSmem& sm, int tid,
                                              int nthr, bool lead) {
  const int ns = attn_active_splits(*a.attn_pos + 1, a.attn_grid);
  if (ns < 1 || ns > kAttnDeferSplits) return false;
  constexpr int HD = 128, PS = HD + 2;
  const int hpg = a.attn_hpg;
  const size_t sstride = (size_t)hpg * PS;  // between the splits of one head
  const int nch = geo.K / 8;
  for (int it = 0; it * nthr < nch; ++it) {
    const int c = it * nthr + tid;
    const bool valid = c < nch;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    if (valid) {
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
      for (int e = 0; e < 8; ++e) o[e] = bfround(o[e]);
    }
    const uint4 pk = valid ? pack8exact(o) : make_uint4(0u, 0u, 0u, 0u);
    pg_emit<GS>(geo, sm, 0, c, valid, pk, o);
    if (valid && lead && a.x_out) *reinterpret_cast<uint4*>(a.x_out + c * 8) = pk;
  }
  return true;
}

// x prologue: x in padded groups (zero past K to whole spans) and the group
// sums of x, built by threads [0, nthr).  The `lead` CTA also stores the new
// residual of embedding / add prologues to a.x_out.  Norm prologues take the
// weights from `nwsm`, which becomes valid when `nwbar` completes phase
// `nw_parity` (nwbar == nullptr: already valid).  `scratch` holds >= 32
// floats, `inv` 8.
template <int GS, class Sync>
__device__ __forceinline__ void pg_prologue(const GemvArgs& a, const PGeom& geo, const PgSmem& sm,
                                            const bf16* nwsm, uint64_t* nwbar, uint32_t nw_parity, float* scratch,
                                            float* inv, volatile int* abort_flag, int tok, int tid, int nthr,
                                            bool lead) {
  const int K = geo.K;
  const int nch = K / 8;
  // o holds bf16 values (the norm output is rounded per element)
  auto emit = [&](int slot, int c, bool valid, const float (&o)[8]) {
    pg_emit<GS>(geo, sm, slot, c, valid, valid ? pack8exact(o) : make_uint4(0u, 0u, 0u, 0u), o);
  };
  const bool merged = a.pro == kProMerge && pg_merge_attn<GS>(a, geo, sm, tid, nthr, lead);
  if (merged) {
  } else if (a.pro == kProX || a.pro == kProMerge) {
    for (int slot = 0; slot < geo.x_slots; ++slot) {
#pragma unroll 1
      for (int it = 0; it * nthr < nch; ++it) {
        const int c = it * nthr + tid;
        const bool valid = c < nch;
        const uint4 raw =
            valid ? *reinterpret_cast<const uint4*>(a.x + (size_t)slot * K + c * 8) : make_uint4(0u, 0u, 0u, 0u);
        float v[8];
        unpack8f(raw, v);
        pg_emit<GS>(geo, sm, slot, c, valid, raw, v);
      }
    }
  } else {
    // pass 1: pre-norm source staged in the x buffer, sums of squares per
    // norm group
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
#pragma unroll 1
    for (int c = tid; c < nch; c += nthr) {
      float v[8];
      src8(a, c, tok, v, pworld ? psrc : nullptr, pworld);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
      const int grp = (c * 8) / gd;
#pragma unroll
      for (int gi = 0; gi < 8; ++gi)
        if (grp == gi) ssg[gi] += ss;
      const uint4 pk = pack8exact(v);
      *reinterpret_cast<uint4*>(pg_xchunk<GS>(geo, sm, 0, c)) = pk;
      if (store) *reinterpret_cast<uint4*>(a.x_out + c * 8) = pk;
    }
    for (int gi = 0; gi < groups; ++gi) {
      float sv = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q == gi) sv = ssg[q];
      const float ss = part_sum<Sync>(sv, scratch, tid, nthr);
      if (tid == 0) inv[gi] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)gd), a.eps)));
    }
    Sync::sync();
    // pass 2: scale and weight in place (each thread rewrites its own chunks)
    if (nwbar && !wait_or_abort(nwbar, nw_parity, abort_flag, a.status)) {
      // no weights: the outputs are garbage and the status word says so
    }
#pragma unroll 1
    for (int it = 0; it * nthr < nch; ++it) {
      const int c = it * nthr + tid;
      const bool valid = c < nch;
      float o[8];
      if (valid) {
        float v[8], w[8];
        unpack8f(*reinterpret_cast<const uint4*>(pg_xchunk<GS>(geo, sm, 0, c)), v);
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
  pg_pad<GS>(geo, sm, tid, nthr);
}

// One stage of packed tiles [a0, a1) (global tile indices; the stage's bytes
// at `sbase`) for warp `warp` of `nwarps` consumer warps.  Units (tile,
// half-span) are dealt round-robin starting at warp `rot`, so that stages
// with fewer units than warps still spread over all of them; each warp runs
// two units at once, interleaved quad by quad (eight independent accumulator
// chains; one unit's drain overlaps the other's math).
template <int BITS, int GS>
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
  const uint32_t MASK = 0x000F000Fu;
  const uint32_t MAGIC_LO = 0x43004300u;  // bf16 128 + nibble
  const uint32_t MAGIC_HI = 0x45004500u;  // bf16 2048 + 16 * nibble
  constexpr float C = BITS == 4 ? 128.0f : 2176.0f;
  // tile -> (logical block, half, span) by a 64-bit multiply, not a
  // division: floor(n / d) == (n * ceil(2^32 / d)) >> 32 for n < 2^32 / d
  // (the magic is 2^32 itself for d == 1, hence 64 bits; the host computes
  // it, a 64-bit division here would cost the critical path ~0.5 us)
  const unsigned long long lbt_magic = geo.lbt_magic;
  struct Unit {
    const unsigned char* aw;   // this lane's code words
    const unsigned char* px;   // x of the unit's group for this lane (or the zero block)
    const unsigned char* sbp;  // this lane's scale/bias record
    const float* xg;           // the group sums
    int slot;                  // red index of row g (row g+8 is 8 rows on)
  };
  auto unit = [&](int u) -> Unit {
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
    r.px = has_x ? sm.xsm + (size_t)xsl * geo.xslot_bytes + (size_t)(sp * 8 + hs * 4 + t) * geo.gstride : sm.zero;
    r.sbp = tile + A_BYTES + hs * 256 + (g * 2 + t1) * 16;
    r.xg = sm.xs + xsl * S * 8 + sp * 8 + hs * 4 + 2 * t1;
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

// Epilogue: each logical row of [lb0, lb1) sums its slots in order and the
// fused output step runs (argmax: this thread's best in best_v / best_i).
__device__ __forceinline__ void pg_epilogue(const GemvArgs& a, const PGeom& geo, const float* red, int lb0, int lb1,
                                            int tid, int nthr, bool res_early, const float (&res_pre)[2],
                                            float& best_v, int& best_i) {
  const int halves = geo.halves, SKP = geo.S * 2;
  const int nlog = (lb1 - lb0) * 16;
  for (int i = tid; i < nlog; i += nthr) {
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
        const float rv = !res_early ? bf2f(a.res[n]) : (i < nthr ? res_pre[0] : res_pre[1]);
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
