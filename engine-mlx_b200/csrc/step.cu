// step.cu — persistent decode-step kernel for dense single-GPU models.
//
// Grid: cps CTAs on each of the nsm SMs (cooperative launch, all resident).
// Each CTA has nine warps:
//   * warp 8, lane 0 is the producer.  It walks the step's stage sequence —
//     for every layer: its norm vectors (a double-buffered "aux" area), the
//     qkv GEMV tiles of this CTA, the K/V rows of this CTA's attention split,
//     the o, gate|up and down tiles; then the final norm and the lm_head
//     tiles — and bulk-copies each stage into a ring of `nslots` shared-memory
//     slots (full/empty mbarriers), never waiting for a phase to begin.
//   * warps 0-7 consume, phase by phase, and meet the other CTAs at a grid
//     barrier between phases (the phase's outputs are the next phase's
//     inputs).  GEMV phases use the packed-GEMV pieces of pgemv_dev.cuh
//     unchanged, so a row's result is bit-identical to the one-matrix kernel.
//     The attention phase is split-KV flash-decode: CTA v < n_kv * splits
//     owns (KV head, split); q/k RMSNorm + RoPE of the new token, the KV
//     cache write of row `pos`, online softmax over 32-row tiles, and the
//     merge of the splits by the last CTA of each head (ticket).
//
// Placement: at the start every CTA takes a per-SM arrival number k with an
// atomic and is indexed v = k * nsm + smid, so that a matrix's logical row
// blocks are divided among SMs first and then between the CTAs of an SM —
// no SM does two CTAs' shares while another idles.  Should an SM id or
// arrival number fall outside the expected range, every CTA uses its
// blockIdx instead (still a partition, only not SM-aware).
//
// Barriers: a monotonically increasing arrival counter; barrier b waits for
// b * grid arrivals (release add, acquire poll).  Every wait is bounded
// (kWaitLimitNs); a CTA that gives up raises a global abort word that the
// others see within one poll, and all of them leave.  The CTA that merges
// the argmax last resets the counters for the next step.
#include "step.cuh"

#include <algorithm>

namespace emx {

namespace {

using namespace pg;

constexpr int kCons = 8;             // consumer warps
constexpr int kNT = kCons * 32;      // consumer threads
constexpr int kThreads = kNT + 32;   // + the producer warp
constexpr int kHD = 128;
constexpr int kAT = 32;              // attention rows per tile (stage)
constexpr int kMinRows = 64;         // fewest KV rows an attention split is given
constexpr int kMergeRegs = 4;        // splits merged from registers (one round of loads)
constexpr int kVOff = kAT * kHD * 2; // V rows' offset inside a slot
constexpr int kMaxSlots = 8;
constexpr int kPartStride = kHD + 4;  // floats per (split, head) partial: m, l, pad, pad, output[128]
constexpr int kMaxMergeW = 1024;      // q heads x splits whose merge weights fit the header
// ring slot: 8 int4 tiles or 4 int8 tiles (16 or 8 MMA units), or 32 K + 32 V
// rows; half of that when two CTAs share an SM
constexpr int kSlotBytes = 36864;
using CSync = SyncNamed<kNT>;

struct StepHdr {
  StepArgs args;  // copy of the kernel arguments (shared-memory reads in the phase functions)
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  uint64_t auxfull[2];
  uint64_t auxempty[2];
  int abort_flag;
  int v;         // placement index
  int p;         // position of the new token
  unsigned flag;
  float wv[kCons];
  int wi[kCons];
  float scratch[32];
  float inv[8];
  float xsc;  // 2^e of the current phase's x staging
  float2 rcs[kHD / 2];  // (cos, sin) of this step's RoPE angles
  float swt[kMaxMergeW];  // attention merge weights [q head][split]
};

template <int HPG>
struct AttnSm {
  float qs[HPG][kHD];      // q * scale
  float qn[HPG + 1][kHD];  // normed q heads (+ k) before RoPE
  float sc[HPG][kAT];      // scores -> probabilities of one tile
  float stat_m[HPG], stat_l[HPG], stat_a[HPG];
  float4 sacc[kCons][HPG][32];  // per-warp partial outputs, lane l = dims 4l..4l+3
  bf16 knew[kHD];
  bf16 vnew[kHD];
};

__host__ __device__ inline int round128(int v) { return (v + 127) & ~127; }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Rows [b0, b1) of W work items for placement index v: SM (v % nsm) takes
// its contiguous share of W, CTA (v / nsm) of the SM its part of that.
__device__ __forceinline__ void sm_range(int W, int v, int nsm, int cps, int& b0, int& b1) {
  const int s = v % nsm, k = v / nsm;
  const int A0 = (int)((long long)s * W / nsm), A1 = (int)((long long)(s + 1) * W / nsm);
  b0 = A0 + (A1 - A0) * k / cps;
  b1 = A0 + (A1 - A0) * (k + 1) / cps;
}

__device__ __forceinline__ void split_range(int L, int splits, int split, int& p0, int& p1) {
  p0 = (int)((long long)split * L / splits);
  p1 = (int)((long long)(split + 1) * L / splits);
}

__device__ __forceinline__ int attn_splits(const StepArgs& A, int p) {
  if (p < 0 || p >= A.cap) return 0;
  const int s = (p + 1 + kMinRows - 1) / kMinRows;
  return s < A.max_splits ? s : A.max_splits;
}

// Grid barrier: thread 0 of the group arrives (release) and polls (acquire)
// until `target` arrivals; bounded, and it gives up at once when any CTA has
// raised the abort word.  Returns false (all threads) after an abort.
template <class Sync>
__device__ __forceinline__ bool grid_barrier(const StepArgs& A, unsigned target, int tid, StepHdr& H) {
  Sync::sync();
  // a CTA that gave up on one of its own waits tells the others
  if (tid == 0 && H.abort_flag) *reinterpret_cast<volatile unsigned*>(A.sync + 2) = 1u;
  if (tid == 0 && !H.abort_flag) {
    // the release add, after the group barrier, publishes every thread's
    // writes of the phase (release cumulativity)
    red_release_add(A.sync, 1u);
    volatile unsigned* gabort = A.sync + 2;
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
      if (ld_acquire_u32(A.sync) >= target) break;
      if (*gabort) {
        H.abort_flag = 1;
        break;
      }
      if (i == 0) {
        t0 = globaltimer_ns();
      } else if ((i & 31u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
        report_status(A.status, kDevTimeoutPeer);
        *gabort = 1u;
        H.abort_flag = 1;
        break;
      }
    }
  }
  Sync::sync();
  return !*reinterpret_cast<volatile int*>(&H.abort_flag);
}

struct Cons {
  int seq;  // stages consumed so far
  int rot;  // first warp of the next stage's units
};

// The o projection's x: the attention output, merged from the splits'
// partials (m, l, output) of every head — weights exp(m_s - M) / sum_s
// exp(m_s - M) l_s, the splits summed in order — rounded to bf16.  Up to
// kMergeRegs splits every thread loads its head's (m, l) and its 8 output
// dims of all splits in one round; more splits take a second round (the
// weights first, through shared memory).
__device__ __noinline__ void merge_prologue(const StepArgs& A, StepHdr& H, const PGeom& geo, const PgSmem& sm,
                                               int ns, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int hpg = A.nq / A.nkv;
  const size_t sstride = (size_t)hpg * kPartStride;  // between the splits of one head
  const int nch = geo.K / 8;                         // 16 chunks per head
  float mx = 0.f;
  if (ns > kMergeRegs) {
    for (int q = warp; q < A.nq; q += kCons) {
      const float* pb = A.attn_part + ((size_t)(q / hpg) * ns * hpg + (q % hpg)) * kPartStride;
      float ms = -INFINITY, ls = 0.f, ms2 = -INFINITY, ls2 = 0.f;
      if (lane < ns) {
        ms = __ldcg(pb + lane * sstride);
        ls = __ldcg(pb + lane * sstride + 1);
      }
      if (lane + 32 < ns) {
        ms2 = __ldcg(pb + (lane + 32) * sstride);
        ls2 = __ldcg(pb + (lane + 32) * sstride + 1);
      }
      const float M = warp_max(fmaxf(ms, ms2));
      const float w1 = ms == -INFINITY ? 0.f : expf(ms - M), w2 = ms2 == -INFINITY ? 0.f : expf(ms2 - M);
      const float den = warp_sum(fmaf(w1, ls, w2 * ls2));
      if (lane < ns) H.swt[q * ns + lane] = __fdiv_rn(w1, den);
      if (lane + 32 < ns) H.swt[q * ns + lane + 32] = __fdiv_rn(w2, den);
    }
    CSync::sync();
  }
  for (int it = 0; it * kNT < nch; ++it) {
    const int c = it * kNT + tid;
    const bool valid = c < nch;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    if (valid) {
      const int q = c / (kHD / 8), d0 = (c % (kHD / 8)) * 8;
      const float* pb = A.attn_part + ((size_t)(q / hpg) * ns * hpg + (q % hpg)) * kPartStride;
      auto add = [&](float w, const float4& v0, const float4& v1) {
        o[0] = fmaf(w, v0.x, o[0]);
        o[1] = fmaf(w, v0.y, o[1]);
        o[2] = fmaf(w, v0.z, o[2]);
        o[3] = fmaf(w, v0.w, o[3]);
        o[4] = fmaf(w, v1.x, o[4]);
        o[5] = fmaf(w, v1.y, o[5]);
        o[6] = fmaf(w, v1.z, o[6]);
        o[7] = fmaf(w, v1.w, o[7]);
      };
      if (ns <= kMergeRegs) {
        float ms[kMergeRegs], ls[kMergeRegs];
        float4 v0[kMergeRegs], v1[kMergeRegs];
#pragma unroll
        for (int s2 = 0; s2 < kMergeRegs; ++s2) {
          if (s2 < ns) {
            const float* ps = pb + s2 * sstride;
            ms[s2] = __ldcg(ps);
            ls[s2] = __ldcg(ps + 1);
            v0[s2] = __ldcg(reinterpret_cast<const float4*>(ps + 4 + d0));
            v1[s2] = __ldcg(reinterpret_cast<const float4*>(ps + 8 + d0));
          }
        }
        float M = -INFINITY;
#pragma unroll
        for (int s2 = 0; s2 < kMergeRegs; ++s2)
          if (s2 < ns) M = fmaxf(M, ms[s2]);
        float w[kMergeRegs], den = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < kMergeRegs; ++s2) {
          w[s2] = (s2 < ns && ms[s2] != -INFINITY) ? expf(ms[s2] - M) : 0.f;
          if (s2 < ns) den = fmaf(w[s2], ls[s2], den);
        }
#pragma unroll
        for (int s2 = 0; s2 < kMergeRegs; ++s2)
          if (s2 < ns) add(__fdiv_rn(w[s2], den), v0[s2], v1[s2]);
      } else {
        for (int s2 = 0; s2 < ns; ++s2) {
          const float* ps = pb + s2 * sstride;
          add(H.swt[q * ns + s2], __ldcg(reinterpret_cast<const float4*>(ps + 4 + d0)),
              __ldcg(reinterpret_cast<const float4*>(ps + 8 + d0)));
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = bfround(o[e]);
        mx = fmaxf(mx, fabsf(o[e]));
      }
      *reinterpret_cast<uint4*>(pg_xchunk<64>(geo, sm, 0, c)) = pack8exact(o);
    }
  }
  pg_convert_staged<64, CSync>(geo, sm, 1, mx, H.scratch, &H.xsc, tid, kNT);
  pg_pad<64>(geo, sm, tid, kNT);
}

// One GEMV phase on rows [lb0, lb1) of this CTA (consumer threads only).
// merge_ns > 0: x is the attention merge of merge_ns splits.
template <int BITS>
__device__ __noinline__ void gemv_phase(const StepArgs& A, StepHdr& H, unsigned char* smem, const PGeom& geo,
                                        const GemvArgs& ga, int lb0, int lb1, const bf16* nwsm, uint64_t* nwbar,
                                        uint32_t nwpar, int tok, Cons& cs, int tid, float& best_v, int& best_i,
                                        int release_aux, int merge_ns) {
  const int warp = tid >> 5, lane = tid & 31;
  const PgSmem sm = pg_smem(smem, geo);
  const bool active = lb1 > lb0;
  float res_pre[2] = {0.f, 0.f};
  bool res_early = false;
  if (active) {
    res_early = pg_res_early(ga, lb0, lb1, tid, kNT, res_pre);
    if (merge_ns > 0)
      merge_prologue(A, H, geo, sm, merge_ns, tid);
    else
      pg_prologue<64, CSync>(ga, geo, sm, nwsm, nwbar, nwpar, H.scratch, H.inv, &H.xsc, &H.abort_flag, tok, tid, kNT,
                             lb0 == 0);
  }
  CSync::sync();
  if (release_aux >= 0 && tid == 0) mbar_arrive(&H.auxempty[release_aux]);
  if (!active) return;
  const int lbt = geo.halves * geo.S;
  const int T1 = lb1 * lbt;
  unsigned char* ring = smem + A.off_ring;
  for (int a0 = lb0 * lbt; a0 < T1; a0 += geo.stage_tiles) {
    const int a1 = min(T1, a0 + geo.stage_tiles);
    const int s = cs.seq++;
    const int slot = s % A.nslots;
    if (wait_or_abort(&H.full[slot], (uint32_t)((s / A.nslots) & 1), &H.abort_flag, A.status))
      pg_stage<BITS, 64>(geo, sm, ring + (size_t)slot * A.slot_bytes, a0, a1, lb0, warp, lane, kCons, cs.rot);
    cs.rot = (cs.rot + (a1 - a0) * 2) % kCons;
    __syncwarp();
    if (lane == 0) mbar_arrive(&H.empty[slot]);
  }
  CSync::sync();
  pg_epilogue(ga, geo, sm.red, lb0, lb1, tid, kNT, res_early, res_pre, best_v, best_i, H.xsc);
}

template <int BITS>
__device__ __forceinline__ void gemv_phase_any(int bits, const StepArgs& A, StepHdr& H, unsigned char* smem,
                                               const PGeom& geo, const GemvArgs& ga, int lb0, int lb1,
                                               const bf16* nwsm, uint64_t* nwbar, uint32_t nwpar, int tok, Cons& cs,
                                               int tid, float& best_v, int& best_i, int release_aux, int merge_ns,
                                               int v) {
  (void)v;
  if (bits == 8)
    gemv_phase<8>(A, H, smem, geo, ga, lb0, lb1, nwsm, nwbar, nwpar, tok, cs, tid, best_v, best_i, release_aux,
                  merge_ns);
  else
    gemv_phase<4>(A, H, smem, geo, ga, lb0, lb1, nwsm, nwbar, nwpar, tok, cs, tid, best_v, best_i, release_aux,
                  merge_ns);
}

// The attention phase of one layer for this CTA's (KV head, split), if any.
// `aux` holds the layer's q_norm at [2H] and k_norm at [2H + 128] (bf16).
template <int HPG>
__device__ __noinline__ void attn_phase(const StepArgs& A, StepHdr& H, unsigned char* smem, const StepLayer& LW,
                                        const bf16* aux, uint64_t* auxbar, uint32_t auxpar, int item, int ns, int p,
                                        Cons& cs, int tid) {
  if (item < 0) return;
  AttnSm<HPG>& S = *reinterpret_cast<AttnSm<HPG>*>(smem + A.off_u);
  const int warp = tid >> 5, lane = tid & 31;
  const int kvh = item / ns, split = item % ns;
  int p0, p1;
  split_range(p + 1, ns, split, p0, p1);
  const int ntile = (p1 - p0 + kAT - 1) / kAT;
  const bool owns_new = p >= p0 && p < p1;
  bf16* kc = LW.kc + (size_t)kvh * A.cap * kHD;
  bf16* vc = LW.vc + (size_t)kvh * A.cap * kHD;
  const bf16* nwq = aux + 2 * A.H;
  const bf16* nwk = nwq + kHD;
  if (LW.q_norm || LW.k_norm) wait_or_abort(auxbar, auxpar, &H.abort_flag, A.status);

  // ---- q heads (and k/v of the new row when owned): rms_norm + rope -------
  const int nprep = HPG + (owns_new ? 1 : 0);
  for (int hh = warp; hh < nprep; hh += kCons) {
    const bool is_k = hh == HPG;
    const bf16* src = is_k ? A.qkvb + (size_t)A.nq * kHD + (size_t)kvh * kHD : A.qkvb + (size_t)(kvh * HPG + hh) * kHD;
    const bf16* nw = is_k ? nwk : nwq;
    const bool has_norm = is_k ? LW.k_norm != nullptr : LW.q_norm != nullptr;
    float v[4];
    const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
    v[0] = __uint_as_float(raw.x << 16);
    v[1] = __uint_as_float(raw.x & 0xffff0000u);
    v[2] = __uint_as_float(raw.y << 16);
    v[3] = __uint_as_float(raw.y & 0xffff0000u);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = fmaf(v[e], v[e], ss);
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), A.eps)));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      S.qn[hh][d] = has_norm ? bfround(__fmul_rn(bfround(__fmul_rn(v[e], inv)), bf2f(nw[d]))) : v[e];
    }
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      const int i = d & (kHD / 2 - 1);
      const float2 t2 = H.rcs[i];
      const float cs_ = t2.x, sn = t2.y;
      const float x1 = S.qn[hh][i], x2 = S.qn[hh][i + kHD / 2];
      float o;
      if (d < kHD / 2) o = __fsub_rn(__fmul_rn(x1, cs_), __fmul_rn(x2, sn));
      else o = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs_));
      o = bfround(o);
      if (is_k) {
        kc[(size_t)p * kHD + d] = f2bf(o);
        S.knew[d] = f2bf(o);
      } else {
        S.qs[hh][d] = __fmul_rn(o, A.scale);
      }
    }
    if (is_k) {
      const bf16* vsrc = A.qkvb + (size_t)(A.nq + A.nkv) * kHD + (size_t)kvh * kHD;
      const uint2 vr = *reinterpret_cast<const uint2*>(vsrc + lane * 4);
      *reinterpret_cast<uint2*>(vc + (size_t)p * kHD + lane * 4) = vr;
      *reinterpret_cast<uint2*>(S.vnew + lane * 4) = vr;
    }
  }
  if (tid < HPG) {
    S.stat_m[tid] = -INFINITY;
    S.stat_l[tid] = 0.f;
  }
  CSync::sync();

  float qreg[HPG][4], acc[HPG][4];
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      qreg[h][e] = S.qs[h][lane * 4 + e];
      acc[h][e] = 0.f;
    }

  unsigned char* ring = smem + A.off_ring;
  const int r0 = warp * 4;  // this warp's rows of a tile
  for (int t = 0; t < ntile; ++t) {
    const int t0 = p0 + t * kAT;
    const int tn = min(kAT, p1 - t0);
    const int s = cs.seq++;
    const int slot = s % A.nslots;
    bf16* kt = reinterpret_cast<bf16*>(ring + (size_t)slot * A.slot_bytes);
    bf16* vt = reinterpret_cast<bf16*>(ring + (size_t)slot * A.slot_bytes + kVOff);
    const bool ok = wait_or_abort(&H.full[slot], (uint32_t)((s / A.nslots) & 1), &H.abort_flag, A.status);
    // the new row is never copied: the owner puts it in place
    if (owns_new && p >= t0 && p < t0 + tn) {
      const int r = p - t0;
      if (tid < kHD / 8) {
        reinterpret_cast<uint4*>(kt + (size_t)r * kHD)[tid] = reinterpret_cast<const uint4*>(S.knew)[tid];
        reinterpret_cast<uint4*>(vt + (size_t)r * kHD)[tid] = reinterpret_cast<const uint4*>(S.vnew)[tid];
      }
      CSync::sync();
    }
    // QK^T: warp w scores rows [4w, 4w + 4).  Each lane forms its 4-dim
    // partial of the four rows, then a transpose-reduction (xor 16, 8: halve
    // the rows a lane keeps; xor 4, 2, 1: plain sums) leaves row
    // 2*bit4(lane) + bit3(lane) in the lanes of that row's octet.
    if (ok && r0 < tn) {
      float kf[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint2 kv = r0 + r < tn ? *reinterpret_cast<const uint2*>(kt + (size_t)(r0 + r) * kHD + lane * 4)
                                     : make_uint2(0u, 0u);
        kf[r][0] = __uint_as_float(kv.x << 16);
        kf[r][1] = __uint_as_float(kv.x & 0xffff0000u);
        kf[r][2] = __uint_as_float(kv.y << 16);
        kf[r][3] = __uint_as_float(kv.y & 0xffff0000u);
      }
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        float v[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float s2 = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) s2 = fmaf(qreg[h][e], kf[r][e], s2);
          v[r] = s2;
        }
        const bool up16 = (lane & 16) != 0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float send = up16 ? v[r] : v[r + 2];
          const float keep = up16 ? v[r + 2] : v[r];
          v[r] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
        const bool up8 = (lane & 8) != 0;
        {
          const float send = up8 ? v[0] : v[1];
          const float keep = up8 ? v[1] : v[0];
          v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 4);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
        const int k = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
        if ((lane & 7) == 0 && r0 + k < tn) S.sc[h][r0 + k] = v[0];
      }
    }
    CSync::sync();
    // online softmax update at tile granularity (one warp per head)
    for (int h = warp; h < HPG; h += kCons) {
      const float sv = lane < tn ? S.sc[h][lane] : -INFINITY;
      const float m = warp_max(sv);
      const float mo = S.stat_m[h];
      const float mn = fmaxf(mo, m);
      const float e = lane < tn ? expf(sv - mn) : 0.f;
      if (lane < tn) S.sc[h][lane] = e;
      const float l = warp_sum(e);
      if (lane == 0) {
        const float alpha = (mo == -INFINITY) ? 0.f : expf(mo - mn);
        S.stat_a[h] = alpha;
        S.stat_l[h] = S.stat_l[h] * alpha + l;
        S.stat_m[h] = mn;
      }
    }
    CSync::sync();
    // P.V: warp w accumulates rows [4w, 4w + 4) into its 4 dims per lane
#pragma unroll
    for (int h = 0; h < HPG; ++h) {
      const float al = S.stat_a[h];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[h][e] *= al;
    }
    const int rend = min(tn, r0 + 4);
    for (int jj = r0; jj < rend; ++jj) {
      const uint2 vv = *reinterpret_cast<const uint2*>(vt + (size_t)jj * kHD + lane * 4);
      const float vf[4] = {__uint_as_float(vv.x << 16), __uint_as_float(vv.x & 0xffff0000u),
                           __uint_as_float(vv.y << 16), __uint_as_float(vv.y & 0xffff0000u)};
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        const float pr = S.sc[h][jj];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] = fmaf(pr, vf[e], acc[h][e]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&H.empty[slot]);
    CSync::sync();  // sc is rewritten by the next tile
  }

  // ---- the warps' partial outputs, then this split's result --------------
#pragma unroll
  for (int h = 0; h < HPG; ++h) S.sacc[warp][h][lane] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  CSync::sync();
  // this split's partial: (m, l) and the unnormalised output of each head,
  // merged by the next phase's prologue
  float* part = A.attn_part + ((size_t)kvh * ns + split) * HPG * kPartStride;
  for (int i = tid; i < HPG * kHD; i += kNT) {
    const int h = i / kHD, d = i % kHD;
    float num = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; ++w) num += reinterpret_cast<const float*>(&S.sacc[w][h][0])[d];
    part[h * kPartStride + 4 + d] = num;
  }
  if (tid < HPG) {
    part[tid * kPartStride + 0] = S.stat_m[tid];
    part[tid * kPartStride + 1] = S.stat_l[tid];
  }
}

// The producer thread: every stage of the step for this CTA, in the order the
// consumers take them.
__device__ __noinline__ void producer(const StepArgs& A, StepHdr& H, unsigned char* smem, int v, int p) {
  const int NS = A.nslots, SB = A.slot_bytes;
  unsigned char* ring = smem + A.off_ring;
  const uint64_t pol = l2_evict_first_policy();
  int s = 0;      // stages issued
  int naux = 0;   // aux loads issued
  auto acquire = [&]() -> int {
    const int slot = s % NS;
    if (s >= NS && !wait_or_abort(&H.empty[slot], (uint32_t)(((s / NS) - 1) & 1), &H.abort_flag, A.status))
      return -1;
    fence_proxy_async();
    return slot;
  };
  auto gemv = [&](int mat, const unsigned char* w) -> bool {
    const PGeom& geo = A.geo[mat];
    int b0, b1;
    sm_range(geo.lb_total, v, A.nsm, A.cps, b0, b1);
    const int lbt = geo.halves * geo.S;
    for (int a0 = b0 * lbt; a0 < b1 * lbt; a0 += geo.stage_tiles) {
      const int a1 = min(b1 * lbt, a0 + geo.stage_tiles);
      const int slot = acquire();
      if (slot < 0) return false;
      const uint32_t bytes = (uint32_t)((a1 - a0) * geo.tile_bytes);
      mbar_arrive_expect_tx(&H.full[slot], bytes);
      bulk_g2s_hint(ring + (size_t)slot * SB, w + (size_t)a0 * geo.tile_bytes, bytes, &H.full[slot], pol);
      ++s;
    }
    return true;
  };
  auto aux = [&](int l) -> bool {
    const int b = l & 1;
    if (l >= 2 && !wait_or_abort(&H.auxempty[b], (uint32_t)(((l >> 1) - 1) & 1), &H.abort_flag, A.status))
      return false;
    unsigned char* dst = smem + A.off_aux + b * A.aux_stride;
    const uint32_t hb = (uint32_t)A.H * 2;
    if (l < A.n_layers) {
      const StepLayer& LW = A.layers[l];
      const uint32_t bytes = 2 * hb + (LW.q_norm ? 256u : 0u) + (LW.k_norm ? 256u : 0u);
      mbar_arrive_expect_tx(&H.auxfull[b], bytes);
      bulk_g2s(dst, LW.in_norm, hb, &H.auxfull[b]);
      bulk_g2s(dst + hb, LW.post_norm, hb, &H.auxfull[b]);
      if (LW.q_norm) bulk_g2s(dst + 2 * hb, LW.q_norm, 256u, &H.auxfull[b]);
      if (LW.k_norm) bulk_g2s(dst + 2 * hb + 256, LW.k_norm, 256u, &H.auxfull[b]);
    } else {
      mbar_arrive_expect_tx(&H.auxfull[b], hb);
      bulk_g2s(dst, A.final_norm, hb, &H.auxfull[b]);
    }
    ++naux;
    return true;
  };
  const int ns = attn_splits(A, p);
  const int item = v < A.nkv * ns ? v : -1;
  auto attn = [&](const StepLayer& LW) -> bool {
    if (item < 0) return true;
    const int kvh = item / ns, split = item % ns;
    int p0, p1;
    split_range(p + 1, ns, split, p0, p1);
    const bf16* kc = LW.kc + (size_t)kvh * A.cap * kHD;
    const bf16* vc = LW.vc + (size_t)kvh * A.cap * kHD;
    for (int r0 = p0; r0 < p1; r0 += kAT) {
      const int re = min(min(r0 + kAT, p1), p);  // row p is computed, not copied
      const uint32_t bytes = re > r0 ? (uint32_t)(re - r0) * kHD * 2 : 0u;
      const int slot = acquire();
      if (slot < 0) return false;
      mbar_arrive_expect_tx(&H.full[slot], 2 * bytes);
      if (bytes) {
        bulk_g2s(ring + (size_t)slot * SB, kc + (size_t)r0 * kHD, bytes, &H.full[slot]);
        bulk_g2s(ring + (size_t)slot * SB + kVOff, vc + (size_t)r0 * kHD, bytes, &H.full[slot]);
      }
      ++s;
    }
    return true;
  };
  // the next layer's K/V rows of this split, towards L2 while this layer runs
  auto prefetch_kv = [&](const StepLayer& LW) {
    if (item < 0) return;
    const int kvh = item / ns, split = item % ns;
    int p0, p1;
    split_range(p + 1, ns, split, p0, p1);
    const int re = min(p1, p);
    if (re <= p0) return;
    const uint32_t bytes = (uint32_t)(re - p0) * kHD * 2;
    bulk_prefetch_l2(LW.kc + ((size_t)kvh * A.cap + p0) * kHD, bytes);
    bulk_prefetch_l2(LW.vc + ((size_t)kvh * A.cap + p0) * kHD, bytes);
  };
  bool ok = true;
  if (A.n_layers > 0) prefetch_kv(A.layers[0]);
  for (int l = 0; ok && l < A.n_layers; ++l) {
    const StepLayer& LW = A.layers[l];
    if (l + 1 < A.n_layers) prefetch_kv(A.layers[l + 1]);
    ok = aux(l) && gemv(kMatQkv, LW.w[0]) && attn(LW) && gemv(kMatO, LW.w[1]) && gemv(kMatGu, LW.w[2]) &&
         gemv(kMatDown, LW.w[3]);
  }
  if (ok) ok = aux(A.n_layers) && gemv(kMatLm, A.lm_w);
  // never leave with copies in flight into this CTA's shared memory
  if (!ok || H.abort_flag) {
    for (int t = max(0, s - NS); t < s; ++t) mbar_wait_bounded(&H.full[t % NS], (uint32_t)((t / NS) & 1), A.status);
    for (int l = max(0, naux - 2); l < naux; ++l) mbar_wait_bounded(&H.auxfull[l & 1], (uint32_t)((l >> 1) & 1), A.status);
  }
}

template <int HPG>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepArgs P) {
  extern __shared__ __align__(128) unsigned char smem[];
  StepHdr& H = *reinterpret_cast<StepHdr*>(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned G = gridDim.x;
  {
    static_assert(sizeof(StepArgs) % 4 == 0, "argument block copied by words");
    const int* src = reinterpret_cast<const int*>(&P);
    int* dst = reinterpret_cast<int*>(&H.args);
    for (int i = tid; i < (int)(sizeof(StepArgs) / 4); i += kThreads) dst[i] = src[i];
  }
  __syncthreads();
  const StepArgs& A = H.args;

  if (tid == 0) {
    for (int i = 0; i < A.nslots; ++i) {
      mbar_init(&H.full[i], 1);
      mbar_init(&H.empty[i], kCons);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&H.auxfull[b], 1);
      mbar_init(&H.auxempty[b], 1);
    }
    H.abort_flag = 0;
    fence_mbar_init();
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    unsigned k = 0xffffffffu;
    if (smid < (unsigned)A.nsm) k = atomicAdd(&A.sync[4 + smid], 1u);
    if (smid >= (unsigned)A.nsm || k >= (unsigned)A.cps) atomicOr(&A.sync[1], 1u);
    H.v = (int)(k * (unsigned)A.nsm + smid);
  }
  // barrier 1: every CTA has its placement number
  const bool ok0 = grid_barrier<SyncCta>(A, G, tid, H);
  if (tid == 0) {
    if (ld_acquire_u32(A.sync + 1)) H.v = blockIdx.x;
    H.p = *reinterpret_cast<volatile int*>(A.pos);
  }
  __syncthreads();
  const int v = H.v, p = H.p;
  const bool pos_ok = p >= 0 && p < A.cap;
  if (tid < kHD / 2 && pos_ok) H.rcs[tid] = A.rope_cs[(size_t)p * (kHD / 2) + tid];
  __syncthreads();
  if (!ok0) return;
  if (warp == kCons) {
    if (lane == 0) producer(A, H, smem, v, p);
    return;
  }

  // ---- consumers --------------------------------------------------------
  if (!pos_ok && v == 0 && tid == 0) report_status(A.status, kDevKvOverflow);
  int tok = *A.token;
  if (tok < 0 || tok >= A.vocab) {
    if (tid == 0 && v == 0) report_status(A.status, kDevBadToken);
    tok = 0;
  }
  const int ns = attn_splits(A, p);
  const int item = v < A.nkv * ns ? v : -1;
  Cons cs{0, 0};
  unsigned bar_n = 2;
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  auto range = [&](int mat, int& b0, int& b1) { sm_range(A.geo[mat].lb_total, v, A.nsm, A.cps, b0, b1); };
  int b0, b1;
  for (int l = 0; l < A.n_layers; ++l) {
    const StepLayer& LW = A.layers[l];
    const int ab = l & 1;
    const uint32_t apar = (uint32_t)((l >> 1) & 1);
    const bf16* aux = reinterpret_cast<const bf16*>(smem + A.off_aux + ab * A.aux_stride);
    range(kMatQkv, b0, b1);
    gemv_phase_any<4>(A.bits[kMatQkv], A, H, smem, A.geo[kMatQkv], A.ga[l == 0 ? 0 : 1], b0, b1, aux,
                      &H.auxfull[ab], apar, tok, cs, tid, best_v, best_i, -1, 0, v);
    if (!grid_barrier<CSync>(A, bar_n++ * G, tid, H)) return;
    attn_phase<HPG>(A, H, smem, LW, aux, &H.auxfull[ab], apar, item, ns, p, cs, tid);
    if (!grid_barrier<CSync>(A, bar_n++ * G, tid, H)) return;
    range(kMatO, b0, b1);
    gemv_phase_any<4>(A.bits[kMatO], A, H, smem, A.geo[kMatO], A.ga[2], b0, b1, nullptr, nullptr, 0u, tok, cs, tid,
                      best_v, best_i, -1, ns, v);
    if (!grid_barrier<CSync>(A, bar_n++ * G, tid, H)) return;
    // post-attention norm + gate|up + SwiGLU (the aux buffer is free after its prologue)
    range(kMatGu, b0, b1);
    gemv_phase_any<4>(A.bits[kMatGu], A, H, smem, A.geo[kMatGu], A.ga[3], b0, b1, aux + A.H, &H.auxfull[ab], apar,
                      tok, cs, tid, best_v, best_i, ab, 0, v);
    if (!grid_barrier<CSync>(A, bar_n++ * G, tid, H)) return;
    range(kMatDown, b0, b1);
    gemv_phase_any<4>(A.bits[kMatDown], A, H, smem, A.geo[kMatDown], A.ga[4], b0, b1, nullptr, nullptr, 0u, tok, cs,
                      tid, best_v, best_i, -1, 0, v);
    if (!grid_barrier<CSync>(A, bar_n++ * G, tid, H)) return;
  }
  // ---- final norm + lm_head + greedy argmax -----------------------------
  const int lb = A.n_layers & 1;
  range(kMatLm, b0, b1);
  gemv_phase_any<4>(A.bits[kMatLm], A, H, smem, A.geo[kMatLm], A.ga[5], b0, b1,
                    reinterpret_cast<const bf16*>(smem + A.off_aux + lb * A.aux_stride), &H.auxfull[lb],
                    (uint32_t)((A.n_layers >> 1) & 1), tok, cs, tid, best_v, best_i, -1, 0, v);
  if (H.abort_flag) return;
  if (pg_argmax_merge<CSync>(A.ga[5], best_v, best_i, blockIdx.x, G, tid, kCons, H.wv, H.wi, &H.flag)) {
    // every CTA has passed every barrier: reset the step's counters
    for (int i = tid; i < 4 + A.nsm; i += kNT)
      if (i != 2) A.sync[i] = 0u;
  }
}

template <int HPG>
int attn_bytes() {
  return (int)sizeof(AttnSm<HPG>);
}

}  // namespace

size_t step_sync_words(int num_sms) { return (size_t)(4 + num_sms + 28); }

int step_make_plan(const StepShape& sh, int num_sms, int cps, int budget, StepPlan* plan) {
  static_assert(sizeof(StepArgs) <= 4096, "step arguments exceed the kernel parameter space");
  if (sh.gs != 64 || sh.hd != kHD || sh.nkv <= 0 || sh.nq % sh.nkv != 0 || num_sms <= 0 || cps < 1 || cps > 2)
    return -1;
  const int hpg = sh.nq / sh.nkv;
  if (hpg != 1 && hpg != 2 && hpg != 4) return -1;
  if (sh.H % 64 != 0 || sh.I % 64 != 0) return -1;
  StepPlan P{};
  StepArgs& A = P.tmpl;
  memset(&A, 0, sizeof(A));
  P.cps = cps;
  P.grid = num_sms * cps;
  P.hpg = hpg;
  A.nsm = num_sms;
  A.cps = cps;
  const int slot_bytes = cps == 1 ? kSlotBytes : kSlotBytes / 2;
  A.slot_bytes = slot_bytes;
  A.off_aux = round128((int)sizeof(StepHdr));
  A.aux_stride = round128(4 * sh.H + 512);
  A.off_u = A.off_aux + 2 * A.aux_stride;
  const int N[5] = {(sh.nq + 2 * sh.nkv) * kHD, sh.H, 2 * sh.I, sh.H, sh.vocab};
  const int K[5] = {sh.H, sh.nq * kHD, sh.H, sh.I, sh.H};
  const int epi[5] = {kEpiStore, kEpiResid, kEpiSwiglu, kEpiResid, kEpiArgmax};
  int end = A.off_u;
  for (int m = 0; m < 5; ++m) {
    const int bits = sh.bits[m];
    if (bits != 4 && bits != 8) return -1;
    if (K[m] % 64 != 0) return -1;
    const int halves = epi[m] == kEpiSwiglu ? 2 : 1;
    if ((N[m] / halves) % 16 != 0) return -1;
    const int W = N[m] / halves / 16;
    const int per_sm = (W + num_sms - 1) / num_sms;
    const int lbs_max = (per_sm + cps - 1) / cps;
    const int tb = ptile_bytes(bits, 64);
    const int st = slot_bytes / tb;
    if (st < 1) return -1;
    pgeom_make(&A.geo[m], K[m], bits, 64, epi[m], W, st, 0, 1, lbs_max, false);
    end = std::max(end, pgeom_layout(A.geo[m], 64, A.off_u));
    A.bits[m] = bits;
  }
  const int ab = hpg == 1 ? attn_bytes<1>() : hpg == 2 ? attn_bytes<2>() : attn_bytes<4>();
  end = std::max(end, A.off_u + ab);
  A.off_ring = round128(end);
  const int nslots = std::min(kMaxSlots, (budget - A.off_ring) / slot_bytes);
  if (nslots < 2) return -1;
  A.nslots = nslots;
  P.smem = A.off_ring + nslots * slot_bytes;
  A.max_splits = std::min(std::min(64, P.grid / sh.nkv), kMaxMergeW / sh.nq);
  if (A.max_splits < 1) return -1;
  A.n_layers = sh.layers;
  A.H = sh.H;
  A.nq = sh.nq;
  A.nkv = sh.nkv;
  A.cap = sh.cap;
  A.vocab = sh.vocab;
  A.scale = 1.0f / sqrtf((float)kHD);
  *plan = P;
  return 0;
}

void step_finish_args(StepArgs* a) {
  auto base = [&](int K) {
    GemvArgs g;
    memset(&g, 0, sizeof(g));
    g.K = K;
    g.eps = a->eps;
    g.norm_groups = 1;
    g.x_slots = 1;
    g.status = a->status;
    return g;
  };
  GemvArgs q = base(a->H);  // input norm + qkv
  q.pro = kProNorm;
  q.x = a->h;
  q.epi = kEpiStore;
  q.y = a->qkvb;
  a->ga[1] = q;
  q.pro = kProEmbedNorm;  // layer 0: the token's embedding row, stored as the residual
  q.emb_w = a->emb_w;
  q.emb_s = a->emb_s;
  q.emb_b = a->emb_b;
  q.emb_bits = a->emb_bits;
  q.emb_gs = a->emb_gs;
  q.vocab = a->vocab;
  q.x_out = a->h;
  a->ga[0] = q;
  GemvArgs o = base(a->nq * kHD);  // o projection + residual
  o.pro = kProX;
  o.x = a->attnb;
  o.epi = kEpiResid;
  o.res = a->h;
  o.y = a->h;
  a->ga[2] = o;
  GemvArgs gu = base(a->H);  // post-attention norm + gate|up + SwiGLU
  gu.pro = kProNorm;
  gu.x = a->h;
  gu.epi = kEpiSwiglu;
  gu.y = a->act;
  a->ga[3] = gu;
  GemvArgs d = base(a->geo[kMatDown].K);  // down projection + residual
  d.pro = kProX;
  d.x = a->act;
  d.epi = kEpiResid;
  d.res = a->h;
  d.y = a->h;
  a->ga[4] = d;
  GemvArgs lm = base(a->H);  // final norm + lm_head + greedy argmax
  lm.pro = kProNorm;
  lm.x = a->h;
  lm.epi = kEpiArgmax;
  lm.y = a->logits;
  lm.am_val = a->am_val;
  lm.am_idx = a->am_idx;
  lm.am_ticket = a->am_ticket;
  lm.tok_out = a->token;
  lm.hist = a->hist;
  lm.hist_n = a->hist_n;
  lm.hist_cap = a->hist_cap;
  lm.pos = a->pos;
  lm.pos_inc = 1;
  a->ga[5] = lm;
}

static const void* kernel_for(int hpg) {
  switch (hpg) {
    case 1: return reinterpret_cast<const void*>(step_kernel<1>);
    case 2: return reinterpret_cast<const void*>(step_kernel<2>);
    case 4: return reinterpret_cast<const void*>(step_kernel<4>);
    default: return nullptr;
  }
}

int step_occupancy(const StepPlan& p) {
  const void* k = kernel_for(p.hpg);
  if (!k) return 0;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem) != cudaSuccess) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kThreads, p.smem) != cudaSuccess) return 0;
  return n;
}

cudaError_t step_launch(const StepArgs& a, const StepPlan& p, cudaStream_t st, bool coop) {
  const void* k = kernel_for(p.hpg);
  if (!k) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = coop ? 1 : 0;
  void* args[] = {const_cast<StepArgs*>(&a)};
  return cudaLaunchKernelExC(&cfg, k, args);
}

}  // namespace emx
