// step.cu — persistent decode-step kernel for dense single-GPU models.
//
// Grid: one CTA per SM (cooperative launch, all resident).  Each CTA has
// nine warps:
//   * warp 8, lane 0 is the producer.  It walks the step's stage sequence —
//     for every layer: its norm vectors (a double-buffered "aux" area), the
//     qkv GEMV tiles of this CTA, the K/V rows of this CTA's attention split,
//     the o, gate|up and down tiles; then the final norm and the lm_head
//     tiles — and bulk-copies each stage into a ring of `nslots` shared-memory
//     slots (full/empty mbarriers), never waiting for a phase to begin.
//   * warps 0-7 consume, phase by phase.  A phase's input vector arrives in
//     flag words (step.cuh): the consumers poll the words of the whole vector
//     (up to four chunks' loads in flight before any is checked) until each
//     carries the flag of this step and layer, so a phase starts as soon as
//     the last of its inputs has landed, with no grid barrier.  GEMV phases
//     stage x and run the packed-GEMV pieces of pgemv_dev.cuh; their rows go
//     out as flag words.  The residual stream is kept per CTA in shared
//     memory (`res`): the x of the qkv phase, then the x of the gate|up
//     phase, so the o and down epilogues add their residual without another
//     read.
//   * The attention phase is split-KV flash-decode: CTA v < n_kv * splits
//     owns (KV head, split): q/k RMSNorm + RoPE of the new token, the KV cache
//     write of row `pos` (by the split that owns it), and an online softmax
//     kept by each warp over its rows of the 32-row tiles (no barrier per
//     tile), merged across warps once.  One split per head writes its
//     normalised output; with more, each writes its partial in flag words
//     and then merges a slice of the head's output from all of them.
// The last CTA through the lm_head's argmax ticket writes the token, moves
// the position and adds one to the epoch, so the next step's flags differ.
// Every wait is bounded (kWaitLimitNs); a CTA that gives up raises a global
// abort word that the others see within a poll, and all of them leave.
#include "step.cuh"

#include <algorithm>
#include <cstring>

namespace emx {

namespace {

using namespace pg;

constexpr int kCons = 8;              // consumer warps
constexpr int kNT = kCons * 32;       // consumer threads
constexpr int kThreads = kNT + 32;    // + the producer warp
constexpr int kHD = 128;
constexpr int kAT = 64;               // attention rows per tile (stage)
constexpr int kRowsPerSplit = 256;    // up to this many cache rows: one attention split per KV head
constexpr int kRowsPerSplitLong = 64;  // beyond: one split per tile of rows (up to max_splits)
constexpr int kMaxSplitsMerge = 32;   // splits one head's merge takes (one per lane)
constexpr int kVOff = kAT * kHD * 2;  // V rows' offset inside a slot
constexpr int kMaxSlots = 8;
constexpr int kPartWords = kHD + 2;  // flag words per (split, q head) partial: m, l, output[128]
// ring slot: 8 int4 tiles or 4 int8 tiles (16 MMA units), or 64 K + 64 V rows
constexpr int kSlotBytes = 36864;
using CSync = SyncNamed<kNT>;

struct StepHdr {
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  uint64_t auxfull[2];
  uint64_t auxempty[2];
  uint64_t routed;  // MoE: this layer's top-k is in eidx / ew (consumer warp 0 -> producer)
  int abort_flag;
  int p;           // position of the new token
  int tok;         // this step's token
  unsigned ebase;  // the flag of layer l is ebase + l + 1
  unsigned flag;
  float xsc;  // 2^e of the current phase's x staging
  float wv[kCons];
  int wi[kCons];
  float scratch[32];
  float2 rcs[kHD / 2];  // (cos, sin) of this step's RoPE angles
  int en;               // MoE: experts selected (top_k)
  int eidx[kStepMaxTopK];
  float ew[kStepMaxTopK];
};

// Load pairs per thread of a split merge: (m, l) of every (split, q head),
// then at most W / ns + 1 output words from each split (W = 64 HPG).
__host__ __device__ constexpr int merge_loads(int hpg) {
  return (kMaxSplitsMerge * hpg + hpg * kHD / 2 + kMaxSplitsMerge + kNT - 1) / kNT;
}

template <int HPG>
struct AttnSm {
  float qs[HPG][kHD];      // q * scale * log2 e
  float qn[HPG + 1][kHD];  // normed q heads (+ k) before RoPE
  float wm[kCons][HPG], wl[kCons][HPG];  // per-warp running max and sum
  float4 sacc[kCons][HPG][32];           // per-warp partial outputs, lane l = dims 4l..4l+3
  float swt[HPG][kMaxSplitsMerge];  // merge weights of a head's splits
  float2 mraw[merge_loads(HPG) * kNT];  // the merge's inputs: (m, l) pairs, then partial output pairs
  bf16 knew[kHD];
  bf16 vnew[kHD];
};

__host__ __device__ inline int round128(int v) { return (v + 127) & ~127; }

// Logical blocks [b0, b1) of W for CTA v of G.
__device__ __forceinline__ void cta_range(int W, int v, int G, int& b0, int& b1) {
  b0 = (int)((long long)v * W / G);
  b1 = (int)((long long)(v + 1) * W / G);
}

__device__ __forceinline__ void split_range(int L, int splits, int split, int& p0, int& p1) {
  p0 = (int)((long long)split * L / splits);
  p1 = (int)((long long)(split + 1) * L / splits);
}

// Attention splits per KV head for the new row p (rows 0..p attend).
__device__ __forceinline__ int attn_splits(const StepArgs& A, int p) {
  // a split's cost grows with its q heads: with 4 per KV head the splits
  // start at 128 rows, with 8 at 32 rows, and then take 32 rows each (one
  // group of four rows per warp)
  const int hpg = A.nq / A.nkv;
  const int one = hpg <= 2 ? kRowsPerSplit : hpg == 4 ? kRowsPerSplit / 2 : kRowsPerSplitLong / 2;
  const int per = hpg >= 8 ? kRowsPerSplitLong / 2 : kRowsPerSplitLong;
  const int s = p < one ? 1 : (p + per) / per;
  return s < A.max_splits ? s : A.max_splits;
}

// ------------------------------------------------------------ flag words
__device__ __forceinline__ void fw_store(uint64_t* p, uint32_t d, unsigned flag) {
  const uint64_t v = ((uint64_t)flag << 32) | d;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Two words (16-byte aligned) in one 128-bit store, each with the flag.
__device__ __forceinline__ void fw_store2(uint64_t* p, uint32_t d0, uint32_t d1, unsigned flag) {
  const uint64_t v0 = ((uint64_t)flag << 32) | d0, v1 = ((uint64_t)flag << 32) | d1;
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(v0), "l"(v1) : "memory");
}

__device__ __forceinline__ void fw_load2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ bool fw_ok(uint64_t a, uint64_t b, unsigned flag) {
  return (unsigned)(a >> 32) == flag && (unsigned)(b >> 32) == flag;
}

__device__ __forceinline__ bool aborted(StepHdr& H) { return *reinterpret_cast<volatile int*>(&H.abort_flag) != 0; }

// Polls the two words at p (16-byte aligned) until both carry `flag`.  False
// after kWaitLimitNs (status recorded, the global abort word raised) or once
// another CTA or warp has aborted.
__device__ __noinline__ bool fw_wait2(const uint64_t* p, unsigned flag, uint64_t& a, uint64_t& b,
                                      const StepArgs& A, StepHdr& H) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    fw_load2(p, a, b);
    if (fw_ok(a, b, flag)) return true;
    if ((i & 31u) == 31u) {
      if (aborted(H) || *reinterpret_cast<volatile unsigned*>(A.abort_word)) {
        *reinterpret_cast<volatile int*>(&H.abort_flag) = 1;
        return false;
      }
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report_status(A.status, kDevTimeoutPeer);
        atomicExch(A.abort_word, 1u);
        *reinterpret_cast<volatile int*>(&H.abort_flag) = 1;
        return false;
      }
    }
  }
}

// Reads the 8-element chunks [0, nch) of a bf16 vector held in flag words
// (chunk c = words 4c..4c+3) carrying `flag` into shared memory: chunk c goes
// to dst + (c / cpg) * gstride + (c % cpg) * 16 (the x-slot layout of a GEMV,
// or a plain vector with cpg = nch); with SLOTS, chunk c is chunk i = c % cps
// of slot c / cps, which goes to dst + slot * sbytes + (i / cpg) * gstride +
// (i % cpg) * 16 (SLOTS: cps > 0).  Thread tid takes chunks tid, tid + kNT,
// ...; up to four chunks are polled together: each round issues the loads of
// every chunk not yet seen, then checks them.  On abort the thread stops (the
// caller's next barrier and abort check end the phase).
__device__ __noinline__ void fw_read_vec(const uint64_t* src, int nch, unsigned flag, unsigned char* dst, int cpg,
                                         int gstride, const StepArgs& A, StepHdr& H, int tid, int cps = 0,
                                         int sbytes = 0) {
  constexpr int kPass = 4;  // chunks whose loads are in flight together
  for (int c0 = tid; c0 < nch; c0 += kPass * kNT) {
    uint64_t w[kPass][4];
    unsigned pend = 0u;  // chunks of this pass not yet seen with the flag
#pragma unroll
    for (int j = 0; j < kPass; ++j)
      if (c0 + j * kNT < nch) pend |= 1u << j;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0; pend; ++it) {
#pragma unroll
      for (int j = 0; j < kPass; ++j) {
        if (pend & (1u << j)) {
          const uint64_t* q = src + 4 * (size_t)(c0 + j * kNT);
          fw_load2(q, w[j][0], w[j][1]);
          fw_load2(q + 2, w[j][2], w[j][3]);
        }
      }
#pragma unroll
      for (int j = 0; j < kPass; ++j) {
        if ((pend & (1u << j)) && fw_ok(w[j][0], w[j][1], flag) && fw_ok(w[j][2], w[j][3], flag)) {
          pend &= ~(1u << j);
          const int c = c0 + j * kNT;
          const int sl = cps ? c / cps : 0, i = c - sl * cps;
          *reinterpret_cast<uint4*>(dst + (size_t)sl * sbytes + (size_t)(i / cpg) * gstride + (i % cpg) * 16) =
              make_uint4((uint32_t)w[j][0], (uint32_t)w[j][1], (uint32_t)w[j][2], (uint32_t)w[j][3]);
        }
      }
      if (pend && (it & 31u) == 31u) {
        if (aborted(H) || *reinterpret_cast<volatile unsigned*>(A.abort_word)) {
          *reinterpret_cast<volatile int*>(&H.abort_flag) = 1;
          return;
        }
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report_status(A.status, kDevTimeoutPeer);
          atomicExch(A.abort_word, 1u);
          *reinterpret_cast<volatile int*>(&H.abort_flag) = 1;
          return;
        }
      }
    }
  }
}

// ---------------------------------------------------------------- prologues
// The token's embedding row (dequantised, bf16) into res — the layer-0 input.
__device__ void load_res_embed(const StepArgs& A, int tok, bf16* res, int tid) {
  const int per = 32 / A.emb_bits;
  const int ngk = A.H / A.emb_gs;
  const uint32_t* row = A.emb_w + (size_t)tok * (A.H / per);
  for (int c = tid; c < A.H / 8; c += kNT) {
    const int k0 = c * 8;
    const bf16 sv = A.emb_s[(size_t)tok * ngk + k0 / A.emb_gs];
    const bf16 bv = A.emb_b[(size_t)tok * ngk + k0 / A.emb_gs];
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      const uint32_t q = (row[k / per] >> (A.emb_bits * (k % per))) & ((1u << A.emb_bits) - 1u);
      v[e] = bf2f(dequant1(q, sv, bv));
    }
    *reinterpret_cast<uint4*>(res + k0) = pack8exact(v);
  }
}

// x = rms_norm(res, nw) staged for a GEMV phase (fp16, power-of-two scale to
// H.xsc), with MLX's rounding points: bf16(bf16(x * inv) * w).
__device__ void stage_norm(const PGeom& geo, const PgSmem& sm, const bf16* res, const bf16* nw, float eps,
                           StepHdr& H, int tid) {
  const int K = geo.K, nch = K / 8;
  float ss = 0.f, mv = 0.f, mw = 0.f;
  for (int c = tid; c < nch; c += kNT) {
    float v[8], w[8];
    unpack8f(*reinterpret_cast<const uint4*>(res + c * 8), v);
    unpack8f(*reinterpret_cast<const uint4*>(nw + c * 8), w);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ss = fmaf(v[e], v[e], ss);
      mv = fmaxf(mv, fabsf(v[e]));
      mw = fmaxf(mw, fabsf(w[e]));
    }
  }
  const float3 r = part_reduce3<CSync>(ss, mv, mw, H.scratch, tid, kNT);
  const float iv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(r.x, (float)K), eps)));
  const int e = pg_scale_exp(r.y * iv * r.z * 1.02f);
  const float sc = pg_pow2(-e);
  if (tid == 0) H.xsc = pg_pow2(e);
#pragma unroll 1
  for (int it = 0; it * kNT < nch; ++it) {
    const int c = it * kNT + tid;
    const bool valid = c < nch;
    float o[8];
    if (valid) {
      float v[8], w[8];
      unpack8f(*reinterpret_cast<const uint4*>(res + c * 8), v);
      unpack8f(*reinterpret_cast<const uint4*>(nw + c * 8), w);
#pragma unroll
      for (int e2 = 0; e2 < 8; ++e2) o[e2] = bfround(__fmul_rn(bfround(__fmul_rn(v[e2], iv)), w[e2]));
    } else {
#pragma unroll
      for (int e2 = 0; e2 < 8; ++e2) o[e2] = 0.f;
    }
    pg_emit<64>(geo, sm, 0, c, valid, o, sc);
  }
  pg_pad<64>(geo, sm, tid, kNT);
}

// x read from flag words as given (attention output, SwiGLU output) and
// staged for a GEMV phase.
__device__ void stage_raw_fw(const PGeom& geo, const PgSmem& sm, const uint64_t* src, unsigned flag,
                             const StepArgs& A, StepHdr& H, int tid) {
  const int nch = geo.K / 8;
  fw_read_vec(src, nch, flag, sm.xsm, 8, geo.gstride, A, H, tid);
  float mx = 0.f;  // max |x| over the chunks this thread staged
  for (int c = tid; c < nch; c += kNT) {
    float v[8];
    unpack8f(*reinterpret_cast<const uint4*>(pg_xchunk<64>(geo, sm, 0, c)), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[e]));
  }
  pg_convert_staged<64, CSync>(geo, sm, 1, mx, H.scratch, &H.xsc, tid, kNT);
  pg_pad<64>(geo, sm, tid, kNT);
}

// The same for the MoE experts' SwiGLU outputs: one x slot per selected
// expert, one scale for all slots.
__device__ __noinline__ void stage_raw_slots(const PGeom& geo, const PgSmem& sm, const uint64_t* src,
                                             unsigned flag, const StepArgs& A, StepHdr& H, int tid) {
  const int nch = geo.K / 8, ns = geo.x_slots;
  fw_read_vec(src, ns * nch, flag, sm.xsm, 8, geo.gstride, A, H, tid, nch, geo.xslot_bytes);
  float mx = 0.f;
  for (int i = tid; i < ns * nch; i += kNT) {
    const int sl = i / nch;
    float v[8];
    unpack8f(*reinterpret_cast<const uint4*>(pg_xchunk<64>(geo, sm, sl, i - sl * nch)), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[e]));
  }
  pg_convert_staged<64, CSync>(geo, sm, ns, mx, H.scratch, &H.xsc, tid, kNT);
  pg_pad<64>(geo, sm, tid, kNT);
}

// The residual vector from flag words into res.
__device__ void load_res_fw(const uint64_t* src, int H_, unsigned flag, bf16* res, const StepArgs& A, StepHdr& H,
                            int tid) {
  fw_read_vec(src, H_ / 8, flag, reinterpret_cast<unsigned char*>(res), H_ / 8, 0, A, H, tid);
}

// The MoE routing of a layer by the consumer threads, one expert each:
// p_e = bf16(exp(l_e - max) / sum_e exp(l_e - max)), then the top_k by rank
// (the number of experts ahead of e in (value desc, index asc) order; NaN
// never ranks), which selects and orders them as k rounds of a stable
// argmax do (the largest value, the lowest index among equal ones; with
// nothing left to take, index 0 with its value if that is NaN, else -inf),
// then with norm_topk the weights divided by their sum
// (crates/ops/src/moe.rs:112-128).  The softmax sum is a butterfly per 32
// experts, then one over the group sums, as in the per-kernel routing, so
// both give the same bits.  Into eidx / ew / en, published to the producer
// through `routed`; lg: E bf16 of scratch.  Ends with a consumer barrier;
// false on abort.
__device__ __noinline__ bool route_block(const StepArgs& A, StepHdr& H, bf16* lg, unsigned flag, int tid) {
  const int E = A.n_experts, k = A.top_k, lane = tid & 31, warp = tid >> 5;
  if (tid < E / 4) {  // words 2t, 2t + 1: experts 4t..4t+3
    uint64_t a, b;
    if (fw_wait2(A.rlw + 2 * tid, flag, a, b, A, H)) {
      reinterpret_cast<uint32_t*>(lg)[2 * tid] = (uint32_t)a;
      reinterpret_cast<uint32_t*>(lg)[2 * tid + 1] = (uint32_t)b;
    }
  }
  if (tid < k) H.eidx[tid] = -1;
  CSync::sync();
  if (aborted(H)) return false;
  const float x = tid < E ? bf2f(lg[tid]) : -INFINITY;
  float m = warp_max(x);
  if (lane == 0) H.scratch[warp] = m;
  CSync::sync();
  m = H.scratch[0];
#pragma unroll
  for (int w = 1; w < kCons; ++w) m = fmaxf(m, H.scratch[w]);
  const float t = warp_sum(tid < E ? expf(x - m) : 0.f);
  CSync::sync();
  if (lane == 0) H.scratch[warp] = t;
  CSync::sync();
  const float s = warp_sum(lane < kCons ? H.scratch[lane] : 0.f);
  const float pr = tid < E ? bfround(__fdiv_rn(expf(x - m), s)) : 0.f;
  if (tid < E) lg[tid] = f2bf(pr);  // every thread has its logit in x
  CSync::sync();
  if (tid < E && pr == pr) {
    int rank = 0;
    for (int j = 0; j < E; ++j) {
      const float q = bf2f(lg[j]);
      rank += (q > pr || (q == pr && j < tid)) ? 1 : 0;
    }
    if (rank < k) {
      H.eidx[rank] = tid;
      H.ew[rank] = pr;
    }
  }
  CSync::sync();
  if (tid == 0) {
    const float p0 = bf2f(lg[0]);
    float sum = 0.f;
    for (int r = 0; r < k; ++r) {
      if (H.eidx[r] < 0) {  // fewer than k experts with a value
        H.eidx[r] = 0;
        H.ew[r] = p0 != p0 ? p0 : -INFINITY;
      }
      sum = __fadd_rn(sum, H.ew[r]);
    }
    if (A.norm_topk && sum > 1e-20f)
      for (int r = 0; r < k; ++r) H.ew[r] = __fdiv_rn(H.ew[r], sum);
    H.en = k;
    mbar_arrive(&H.routed);
  }
  CSync::sync();
  return true;
}

// ------------------------------------------------------------- GEMV phases
// The stages of logical blocks [lb0, lb1) from the ring (consumer threads);
// ends with a consumer barrier.  The geometry, the ring's slot and phase
// and the counters live in registers for the whole phase: every asm block
// with a memory clobber (the mbarrier ops) would otherwise force them to be
// re-read per stage.
template <int BITS, bool XSL_MOD = false>
__device__ __noinline__ void gemv_run(const StepArgs& A, StepHdr& H, unsigned char* smem, const PGeom& geo_ref,
                                      int lb0, int lb1, int& seq_ref, int& rot_ref, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const PGeom geo = geo_ref;
  const PgSmem sm = pg_smem(smem, geo);
  const int lbt = geo.halves * geo.S;
  const int T1 = lb1 * lbt;
  unsigned char* ring = smem + A.off_ring;
  const int NS = A.nslots, SB = A.slot_bytes;
  int* const status = A.status;
  int seq = seq_ref, rot = rot_ref;
  int slot = seq % NS;
  uint32_t par = (uint32_t)((seq / NS) & 1);
  for (int a0 = lb0 * lbt; a0 < T1; a0 += geo.stage_tiles) {
    const int a1 = min(T1, a0 + geo.stage_tiles);
    if (wait_or_abort(&H.full[slot], par, &H.abort_flag, status))
      pg_stage<BITS, 64, XSL_MOD>(geo, sm, ring + (size_t)slot * SB, a0, a1, lb0, warp, lane, kCons, rot);
    rot = (rot + (a1 - a0) * 2) & (kCons - 1);
    __syncwarp();
    if (lane == 0) mbar_arrive(&H.empty[slot]);
    ++seq;
    if (++slot == NS) {
      slot = 0;
      par ^= 1u;
    }
  }
  seq_ref = seq;
  rot_ref = rot;
  CSync::sync();
}

template <bool XSL_MOD = false>
__device__ __forceinline__ void gemv_any(int bits, const StepArgs& A, StepHdr& H, unsigned char* smem,
                                         const PGeom& geo, int lb0, int lb1, int& seq, int& rot, int tid) {
  if (bits == 8)
    gemv_run<8, XSL_MOD>(A, H, smem, geo, lb0, lb1, seq, rot, tid);
  else
    gemv_run<4, XSL_MOD>(A, H, smem, geo, lb0, lb1, seq, rot, tid);
}

enum OutKind : int { kOutStore = 0, kOutResid = 1, kOutSwiglu = 2 };

// A row's value: xscale * the sum of its SKP slots in order (SKP even; vector
// loads, so the slots arrive together).
__device__ __forceinline__ float row_value(const float* red, int prow, int SKP, float xscale) {
  const float* r = red + (size_t)prow * SKP;
  float acc = 0.f;
  if ((SKP & 3) == 0) {
#pragma unroll 6
    for (int j = 0; j < SKP; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(r + j);
      acc += q.x;
      acc += q.y;
      acc += q.z;
      acc += q.w;
    }
  } else {
#pragma unroll 4
    for (int j = 0; j < SKP; j += 2) {
      const float2 q = *reinterpret_cast<const float2*>(r + j);
      acc += q.x;
      acc += q.y;
    }
  }
  return acc * xscale;
}

// The phase's rows [lb0*16, lb1*16) out as flag words, one row per thread
// (lane pairs join their rows into a word): bf16(acc) (store),
// bf16(res + bf16(acc)) (residual), or MLX's SwiGLU steps.
template <int OUT>
__device__ void epilogue_fw(const PGeom& geo, const PgSmem& sm, int lb0, int lb1, const bf16* res, uint64_t* dst,
                            unsigned flag, float xscale, int tid) {
  const int halves = geo.halves, SKP = geo.S * 2;
  const int nrow = (lb1 - lb0) * 16;
  for (int i0 = 0; i0 < nrow; i0 += kNT) {
    const int li = i0 + tid;
    float y = 0.f;
    if (li < nrow) {
      const int lbl = li >> 4, r = li & 15;
      const int prow = lbl * halves * 16 + r;
      const float acc = row_value(sm.red, prow, SKP, xscale);
      if (OUT == kOutStore) {
        y = bfround(acc);
      } else if (OUT == kOutResid) {
        y = bfround(__fadd_rn(bf2f(res[lb0 * 16 + li]), bfround(acc)));
      } else {
        const float accu = row_value(sm.red, prow + 16, SKP, xscale);
        const float gv = bfround(acc), uv = bfround(accu);
        const float sg = bfround(sigmoid_f(gv));
        const float sv = bfround(__fmul_rn(gv, sg));
        y = bfround(__fmul_rn(sv, uv));
      }
    }
    const uint32_t bits = f2bits(y);
    const uint32_t hi = __shfl_down_sync(0xffffffffu, bits, 1);
    if (li < nrow && (li & 1) == 0) fw_store(dst + (size_t)(lb0 * 16 + li) / 2, bits | (hi << 16), flag);
  }
}

// The merge of a KV head's split partials (flag words at hw: [split][q
// head][m, l, output[128]]), distributed over the splits: split `split` of
// `ns` merges output words [split * W / ns, (split + 1) * W / ns) of the
// head's W.  Every split of the head is resident and writes its partial
// before it waits here, so the waits end once the slowest split's words
// land; no ticket, no fence.  Arithmetic: weights 2^(m_s - M) / sum_s
// 2^(m_s - M) l_s (M the max), then the weighted partials summed in split
// order.  A thread holds at most merge_loads(HPG) load pairs, all issued
// before any is checked.
template <int HPG>
__device__ __noinline__ void attn_merge_slice(const StepArgs& A, StepHdr& H, AttnSm<HPG>& S, const uint64_t* hw,
                                              uint64_t* out, int split, int ns, unsigned flag, int tid) {
  constexpr int W = HPG * kHD / 2;
  constexpr int NL = merge_loads(HPG);
  const int warp = tid >> 5, lane = tid & 31;
  const int w0 = split * W / ns, w1 = (split + 1) * W / ns;
  const int nml = ns * HPG, tot = nml + (w1 - w0) * ns;  // <= NL * kNT
  auto addr = [&](int t) -> const uint64_t* {
    if (t < nml) return hw + (size_t)t * kPartWords;  // t = split * HPG + q head
    const int u = t - nml, i = w0 + u / ns, s2 = u % ns;
    const int h = (2 * i) / kHD, d = (2 * i) % kHD;
    return hw + ((size_t)s2 * HPG + h) * kPartWords + 2 + d;
  };
  uint64_t v0[NL], v1[NL];
#pragma unroll
  for (int q = 0; q < NL; ++q) {
    const int t = tid + q * kNT;
    v0[q] = v1[q] = 0;
    if (t < tot) fw_load2(addr(t), v0[q], v1[q]);
  }
#pragma unroll
  for (int q = 0; q < NL; ++q) {
    const int t = tid + q * kNT;
    if (t < tot) {
      uint64_t u0 = v0[q], u1 = v1[q];  // scalars: the wait takes them by reference
      if (!fw_ok(u0, u1, flag) && !fw_wait2(addr(t), flag, u0, u1, A, H)) u0 = u1 = 0;
      S.mraw[t] = make_float2(__uint_as_float((uint32_t)u0), __uint_as_float((uint32_t)u1));
    }
  }
  CSync::sync();
  for (int h = warp; h < HPG; h += kCons) {
    const float ms = lane < ns ? S.mraw[lane * HPG + h].x : -INFINITY;
    const float ls = lane < ns ? S.mraw[lane * HPG + h].y : 0.f;
    const float M = warp_max(ms);
    const float w = ms == -INFINITY ? 0.f : ex2f(ms - M);
    const float den = warp_sum(fmaf(w, ls, 0.f));
    if (lane < ns) S.swt[h][lane] = __fdiv_rn(w, den);
  }
  CSync::sync();
  if (tid < w1 - w0) {
    const int i = w0 + tid;
    const int h = (2 * i) / kHD;
    const float2* v = &S.mraw[nml + tid * ns];
    float o0 = 0.f, o1 = 0.f;
    for (int s2 = 0; s2 < ns; ++s2) {
      const float sw = S.swt[h][s2];
      o0 = fmaf(sw, v[s2].x, o0);
      o1 = fmaf(sw, v[s2].y, o1);
    }
    fw_store(out + i, (uint32_t)f2bits(bfround(o0)) | ((uint32_t)f2bits(bfround(o1)) << 16), flag);
  }
}

// ----------------------------------------------------------- attention
// The attention phase of one layer for this CTA's (KV head, split), if any.
// `aux` holds the layer's q_norm at [2H] and k_norm at [2H + 128] (bf16).
template <int HPG>
__device__ __noinline__ void attn_phase(const StepArgs& A, StepHdr& H, unsigned char* smem, const StepLayer& LW,
                                        const bf16* aux, uint64_t* auxbar, uint32_t auxpar, int item, int ns, int p,
                                        unsigned flag, int& seq, int tid) {
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
  // (rows of the qkv projection, read from its flag words: lane l takes
  // elements 4l..4l+3 = words 2l, 2l+1)
  const int nprep = HPG + (owns_new ? 1 : 0);
  for (int hh = warp; hh < nprep; hh += kCons) {
    const bool is_k = hh == HPG;
    const int e0 = is_k ? (A.nq + kvh) * kHD : (kvh * HPG + hh) * kHD;
    const bf16* nw = is_k ? nwk : nwq;
    const bool has_norm = is_k ? LW.k_norm != nullptr : LW.q_norm != nullptr;
    uint64_t w0 = 0, w1 = 0;
    fw_load2(A.qkvw + e0 / 2 + lane * 2, w0, w1);
    if (!fw_ok(w0, w1, flag)) fw_wait2(A.qkvw + e0 / 2 + lane * 2, flag, w0, w1, A, H);
    float v[4];
    v[0] = __uint_as_float((uint32_t)w0 << 16);
    v[1] = __uint_as_float((uint32_t)w0 & 0xffff0000u);
    v[2] = __uint_as_float((uint32_t)w1 << 16);
    v[3] = __uint_as_float((uint32_t)w1 & 0xffff0000u);
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
        S.qs[hh][d] = __fmul_rn(o, A.scale_log2e);
      }
    }
    if (is_k) {
      const int ev = (A.nq + A.nkv + kvh) * kHD;
      uint64_t u0 = 0, u1 = 0;
      fw_load2(A.qkvw + ev / 2 + lane * 2, u0, u1);
      if (!fw_ok(u0, u1, flag)) fw_wait2(A.qkvw + ev / 2 + lane * 2, flag, u0, u1, A, H);
      const uint2 vr = make_uint2((uint32_t)u0, (uint32_t)u1);
      *reinterpret_cast<uint2*>(vc + (size_t)p * kHD + lane * 4) = vr;
      *reinterpret_cast<uint2*>(S.vnew + lane * 4) = vr;
    }
  }
  CSync::sync();

  float qreg[HPG][4], acc[HPG][4], wm[HPG], wl[HPG];
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
    wm[h] = -INFINITY;
    wl[h] = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      qreg[h][e] = S.qs[h][lane * 4 + e];
      acc[h][e] = 0.f;
    }
  }

  // Each warp keeps its own online softmax over the rows it takes (rows
  // [4w, 4w + 4) and [32 + 4w, 36 + 4w) of every tile: a tile of up to 32
  // rows gives every warp one group), so the tiles need no CTA barrier; the
  // warps merge once at the end.  Scores are in the base-2 domain (q carries
  // scale * log2 e), so every exponential is one ex2.
  unsigned char* ring = smem + A.off_ring;
  const int r0 = warp * 4;  // this warp's first row of a tile
  for (int t = 0; t < ntile; ++t) {
    const int t0 = p0 + t * kAT;
    const int tn = min(kAT, p1 - t0);
    const int s = seq++;
    const int slot = s % A.nslots;
    const bf16* kt = reinterpret_cast<const bf16*>(ring + (size_t)slot * A.slot_bytes);
    const bf16* vt = reinterpret_cast<const bf16*>(ring + (size_t)slot * A.slot_bytes + kVOff);
    const bool ok = wait_or_abort(&H.full[slot], (uint32_t)((s / A.nslots) & 1), &H.abort_flag, A.status);
    if (ok && r0 < tn) {
#pragma unroll 1
      for (int g2 = 0; g2 < 2; ++g2) {
        const int rb = r0 + 32 * g2;                 // first row of this group of four
        const int nr = min(4, tn - rb);             // rows of the group in the tile
        if (nr <= 0) break;
        // the new row is never copied into the ring: it is read from S.knew / S.vnew
        float kf[4][4], vf[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int rr = rb + r;
          const bool isnew = owns_new && t0 + rr == p;
          const bf16* kr = isnew ? S.knew : kt + (size_t)rr * kHD;
          const bf16* vr = isnew ? S.vnew : vt + (size_t)rr * kHD;
          const uint2 kv = r < nr ? *reinterpret_cast<const uint2*>(kr + lane * 4) : make_uint2(0u, 0u);
          const uint2 vv = r < nr ? *reinterpret_cast<const uint2*>(vr + lane * 4) : make_uint2(0u, 0u);
          kf[r][0] = __uint_as_float(kv.x << 16);
          kf[r][1] = __uint_as_float(kv.x & 0xffff0000u);
          kf[r][2] = __uint_as_float(kv.y << 16);
          kf[r][3] = __uint_as_float(kv.y & 0xffff0000u);
          vf[r][0] = __uint_as_float(vv.x << 16);
          vf[r][1] = __uint_as_float(vv.x & 0xffff0000u);
          vf[r][2] = __uint_as_float(vv.y << 16);
          vf[r][3] = __uint_as_float(vv.y & 0xffff0000u);
        }
#pragma unroll
        for (int h = 0; h < HPG; ++h) {
          // QK^T: each lane's 4-dim partials of the four rows, then a
          // transpose-reduction (xor 16, 8: halve the rows a lane keeps; xor
          // 4, 2, 1: plain sums) leaves row k in lane 8k (and its octet)
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
          float sk[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) sk[k] = __shfl_sync(0xffffffffu, v[0], k * 8);
          // online softmax over the warp's rows so far
          float mt = sk[0];
#pragma unroll
          for (int k = 1; k < 4; ++k)
            if (k < nr) mt = fmaxf(mt, sk[k]);
          const float mn = fmaxf(wm[h], mt);
          const float alpha = wm[h] == -INFINITY ? 0.f : ex2f(wm[h] - mn);
          float pk[4], ls = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            pk[k] = k < nr ? ex2f(sk[k] - mn) : 0.f;
            ls += pk[k];
          }
          wl[h] = fmaf(wl[h], alpha, ls);
          wm[h] = mn;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float a2 = acc[h][e] * alpha;
#pragma unroll
            for (int k = 0; k < 4; ++k) a2 = fmaf(pk[k], vf[k][e], a2);
            acc[h][e] = a2;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&H.empty[slot]);
  }

  // ---- merge the warps: M = max_w m_w, L = sum_w 2^(m_w - M) l_w,
  // num = sum_w 2^(m_w - M) acc_w (warps in order) -------------------------
#pragma unroll
  for (int h = 0; h < HPG; ++h) {
    S.sacc[warp][h][lane] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    if (lane == 0) {
      S.wm[warp][h] = wm[h];
      S.wl[warp][h] = wl[h];
    }
  }
  CSync::sync();
  // (M, L) of head h and num of dims d, d + 1
  auto merged = [&](int h, int d, float& M, float& Lh, float& n0, float& n1) {
    M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCons; ++w) M = fmaxf(M, S.wm[w][h]);
    Lh = 0.f;
    n0 = 0.f;
    n1 = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; ++w) {
      const float mw = S.wm[w][h];
      const float ew = mw == -INFINITY ? 0.f : ex2f(mw - M);
      Lh = fmaf(ew, S.wl[w][h], Lh);
      const float* aw = reinterpret_cast<const float*>(&S.sacc[w][h][0]);
      n0 = fmaf(ew, aw[d], n0);
      n1 = fmaf(ew, aw[d + 1], n1);
    }
  };
  uint64_t* out = A.attw + (size_t)kvh * HPG * kHD / 2;  // this KV head's q heads, two dims per word
  if (ns == 1) {
    // the normalised output, with the merge's arithmetic for one split:
    // bf16(fma(1 / L, num, 0))
    for (int i = tid; i < HPG * kHD / 2; i += kNT) {
      const int h = (2 * i) / kHD, d = (2 * i) % kHD;
      float M, Lh, n0, n1;
      merged(h, d, M, Lh, n0, n1);
      const float sw = __fdiv_rn(1.0f, Lh);
      const float o0 = bfround(fmaf(sw, n0, 0.f));
      const float o1 = bfround(fmaf(sw, n1, 0.f));
      fw_store(out + i, (uint32_t)f2bits(o0) | ((uint32_t)f2bits(o1) << 16), flag);
    }
    return;
  }
  // several splits: each writes its partial (m, l and the unnormalised
  // output of every q head) in flag words, then merges one slice of the
  // head's output words from all the splits' partials
  uint64_t* const hw = A.attn_pw + (size_t)kvh * A.max_splits * HPG * kPartWords;
  {
    uint64_t* pw = hw + (size_t)split * HPG * kPartWords;
    for (int i = tid; i < HPG * kHD / 2; i += kNT) {
      const int h = (2 * i) / kHD, d = (2 * i) % kHD;
      float M, Lh, n0, n1;
      merged(h, d, M, Lh, n0, n1);
      fw_store2(pw + h * kPartWords + 2 + d, __float_as_uint(n0), __float_as_uint(n1), flag);
      if (d == 0) fw_store2(pw + h * kPartWords, __float_as_uint(M), __float_as_uint(Lh), flag);
    }
  }
  attn_merge_slice<HPG>(A, H, S, hw, out, split, ns, flag, tid);
}

// Logical blocks [d0, d1) of the down phase for CTA v of G.  MoE: whole
// row blocks of H, each the top_k slots' blocks in slot order (block
// rb * top_k + j: rows rb of expert slot j), so a CTA sums its rows over the
// experts itself.
template <bool MOE>
__device__ __forceinline__ void down_range(const StepArgs& A, int v, int G, int& d0, int& d1) {
  if (MOE) {
    cta_range(A.H / 16, v, G, d0, d1);
    d0 *= A.top_k;
    d1 *= A.top_k;
  } else {
    cta_range(A.geo[kMatDown].lb_total, v, G, d0, d1);
  }
}

// A MoE layer's post-attention norm, router GEMV, top-k and the selected
// experts' gate|up + SwiGLU (consumer threads; the router reads the x staged
// for gate|up).  A CTA routes when it has expert work (its producer needs
// the experts, its down epilogue the weights); that work is what the next
// layer's router waits for, so the router logits it reads are not rewritten
// under it.  False on abort.
__device__ __noinline__ bool moe_router_gu(const StepArgs& A, StepHdr& H, unsigned char* smem, bf16* res,
                                           const bf16* aux, int ab, uint32_t apar, int l, unsigned flag, int& seq,
                                           int& rot, int tid) {
  const int G = (int)gridDim.x, v = (int)blockIdx.x;
  int g0, g1, d0, d1, r0, r1;
  cta_range(A.geo[kMatGu].lb_total, v, G, g0, g1);
  down_range<true>(A, v, G, d0, d1);
  cta_range(A.geo[kMatRouter].lb_total, v, G, r0, r1);
  const bool routes = g1 > g0 || d1 > d0;
  if (g1 > g0 || r1 > r0) load_res_fw(A.xmw, A.H, flag, res, A, H, tid);
  CSync::sync();
  if (aborted(H)) return false;
  const PGeom& geo = A.geo[kMatGu];
  if (g1 > g0 || r1 > r0) {
    wait_or_abort(&H.auxfull[ab], apar, &H.abort_flag, A.status);
    stage_norm(geo, pg_smem(smem, geo), res, aux + A.H, A.eps, H, tid);
    CSync::sync();
  }
  if (r1 > r0) {
    const PGeom& rg = A.geo[kMatRouter];
    gemv_any(A.bits[kMatRouter], A, H, smem, rg, r0, r1, seq, rot, tid);
    epilogue_fw<kOutStore>(rg, pg_smem(smem, rg), r0, r1, res, A.rlw, flag, H.xsc, tid);
  }
  if (routes && !route_block(A, H, res, flag, tid)) return false;
  if (g1 > g0) {
    gemv_any(A.bits[kMatGu], A, H, smem, geo, g0, g1, seq, rot, tid);
    epilogue_fw<kOutSwiglu>(geo, pg_smem(smem, geo), g0, g1, res, A.hw, flag, H.xsc, tid);
  }
  return true;
}

// A MoE layer's expert down projections over the logical blocks [d0, d1)
// of down_range (x slot j = slot j's SwiGLU output) and the block's output:
// row n = bf16(xm_n + sum_j w_j bf16(y_jn)), the products summed in slot
// order in fp32 (crates/ops/src/moe.rs:196-207; the per-kernel chain's
// add-and-norm prologue does the same sum), out as the layer's residual.
// The CTA's xm rows go into res first.  False on abort.
__device__ __noinline__ bool moe_down(const StepArgs& A, StepHdr& H, unsigned char* smem, bf16* res, int d0,
                                      int d1, unsigned flag, int& seq, int& rot, int tid) {
  const PGeom& geo = A.geo[kMatDown];
  const int k = A.top_k, rb0 = d0 / k, nrow = (d1 - d0) / k * 16;
  fw_read_vec(A.xmw + (size_t)rb0 * 8, nrow / 8, flag, reinterpret_cast<unsigned char*>(res + rb0 * 16), nrow / 8,
              0, A, H, tid);
  stage_raw_slots(geo, pg_smem(smem, geo), A.hw, flag, A, H, tid);
  CSync::sync();
  if (aborted(H)) return false;
  gemv_any<true>(A.bits[kMatDown], A, H, smem, geo, d0, d1, seq, rot, tid);
  const PgSmem sm = pg_smem(smem, geo);
  const int SKP = geo.S * 2;
  const float xs = H.xsc;
  for (int i0 = 0; i0 < nrow; i0 += kNT) {
    const int li = i0 + tid;
    float y = 0.f;
    if (li < nrow) {
      const int rbl = li >> 4, r = li & 15;
      float add = 0.f;
      for (int j = 0; j < k; ++j)
        add = __fadd_rn(add, __fmul_rn(bfround(row_value(sm.red, (rbl * k + j) * 16 + r, SKP, xs)), H.ew[j]));
      y = bfround(__fadd_rn(bf2f(res[rb0 * 16 + li]), add));
    }
    const uint32_t bits = f2bits(y);
    const uint32_t hi = __shfl_down_sync(0xffffffffu, bits, 1);
    if (li < nrow && (li & 1) == 0) fw_store(A.xw + (size_t)(rb0 * 16 + li) / 2, bits | (hi << 16), flag);
  }
  return true;
}

// ------------------------------------------------------------ producer
// Every stage of the step for this CTA, in the order the consumers take them.
template <bool MOE>
__device__ __noinline__ void producer(const StepArgs& A, StepHdr& H, unsigned char* smem, int v, int G, int p,
                                      int ns) {
  const int NS = A.nslots, SB = A.slot_bytes;
  unsigned char* ring = smem + A.off_ring;
  const uint64_t pol = l2_evict_first_policy();
  int s = 0;     // stages issued
  int naux = 0;  // aux loads issued
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
    cta_range(geo.lb_total, v, G, b0, b1);
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
  // the top_k selected experts' stages.  gate|up: logical block lb of the
  // gathered matrix is block lb % lps of expert eidx[lb / lps] (lps blocks per
  // expert, contiguous), so a stage takes one copy per expert it touches;
  // down (down_range): block lb is block lb / top_k of expert
  // eidx[lb % top_k], one copy per block
  auto gemv_experts = [&](int mat, const unsigned char* w, int lps, int l) -> bool {
    const PGeom& geo = A.geo[mat];
    const bool inter = mat == kMatDown;
    const int k = A.top_k;
    int b0, b1;
    if (inter)
      down_range<true>(A, v, G, b0, b1);
    else
      cta_range(geo.lb_total, v, G, b0, b1);
    if (b1 <= b0) return true;
    if (!wait_or_abort(&H.routed, (uint32_t)(l & 1), &H.abort_flag, A.status)) return false;
    const int lbt = geo.halves * geo.S;
    const size_t tb = geo.tile_bytes, lb_bytes = (size_t)lbt * tb;
    for (int a0 = b0 * lbt; a0 < b1 * lbt; a0 += geo.stage_tiles) {
      const int a1 = min(b1 * lbt, a0 + geo.stage_tiles);
      const int slot = acquire();
      if (slot < 0) return false;
      mbar_arrive_expect_tx(&H.full[slot], (uint32_t)((a1 - a0) * tb));
      for (int tl = a0; tl < a1;) {
        const int lb = tl / lbt;
        const int j = inter ? lb % k : lb / lps, blk = inter ? lb / k : lb - j * lps;
        const unsigned char* src = w + ((size_t)H.eidx[j] * lps + blk) * lb_bytes + (size_t)(tl - lb * lbt) * tb;
        const int end = min(a1, inter ? (lb + 1) * lbt : (j + 1) * lps * lbt);
        bulk_g2s_hint(ring + (size_t)slot * SB + (size_t)(tl - a0) * tb, src, (uint32_t)((end - tl) * tb),
                      &H.full[slot], pol);
        tl = end;
      }
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
    ok = aux(l) && gemv(kMatQkv, LW.w[0]) && attn(LW) && gemv(kMatO, LW.w[1]);
    if (!MOE)
      ok = ok && gemv(kMatGu, LW.w[2]) && gemv(kMatDown, LW.w[3]);
    else
      ok = ok && gemv(kMatRouter, LW.router) && gemv_experts(kMatGu, LW.w[2], A.egu_lps, l) &&
           gemv_experts(kMatDown, LW.w[3], A.edown_lps, l);
  }
  if (ok) ok = aux(A.n_layers) && gemv(kMatLm, A.lm_w);
  // never leave with copies in flight into this CTA's shared memory
  if (!ok || aborted(H)) {
    for (int t = max(0, s - NS); t < s; ++t) mbar_wait_bounded(&H.full[t % NS], (uint32_t)((t / NS) & 1), A.status);
    for (int l = max(0, naux - 2); l < naux; ++l)
      mbar_wait_bounded(&H.auxfull[l & 1], (uint32_t)((l >> 1) & 1), A.status);
  }
}

__device__ __forceinline__ void argmax_pair(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}

// ---------------------------------------------------------------- kernel
template <int HPG, bool MOE>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepArgs Ap) {
  extern __shared__ __align__(128) unsigned char smem[];
  StepHdr& H = *reinterpret_cast<StepHdr*>(smem);
  {
    // the arguments into shared memory: the noinline phases read them through
    // a reference, and a reference to the parameter itself is a generic load
    // of the constant space (slow) where a shared one is a few cycles
    uint32_t* dst = reinterpret_cast<uint32_t*>(smem + Ap.off_args);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&Ap);
    for (int i = threadIdx.x; i < (int)(sizeof(StepArgs) / 4); i += blockDim.x) dst[i] = src[i];
    __syncthreads();
  }
  const StepArgs& A = *reinterpret_cast<const StepArgs*>(smem + Ap.off_args);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = (int)gridDim.x, v = (int)blockIdx.x;
  const int L = A.n_layers;

  if (tid == 0) {
    for (int i = 0; i < A.nslots; ++i) {
      mbar_init(&H.full[i], 1);
      mbar_init(&H.empty[i], kCons);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&H.auxfull[b], 1);
      mbar_init(&H.auxempty[b], 1);
    }
    mbar_init(&H.routed, 1);
    H.en = 0;
    H.abort_flag = *reinterpret_cast<volatile unsigned*>(A.abort_word) ? 1 : 0;
    fence_mbar_init();
    H.p = *reinterpret_cast<volatile int*>(A.pos);
    H.ebase = *reinterpret_cast<volatile unsigned*>(A.epoch) * (unsigned)(L + 1);
    int tok = *A.token;
    if (tok < 0 || tok >= A.vocab) {
      if (v == 0) report_status(A.status, kDevBadToken);
      tok = 0;
    }
    H.tok = tok;
  }
  __syncthreads();
  const int p = H.p;
  if (p < 0 || p >= A.cap) {
    if (tid == 0 && v == 0) report_status(A.status, kDevKvOverflow);
    return;
  }
  if (H.abort_flag) return;  // an earlier step gave up: the words are stale until the host clears them
  if (tid < kHD / 2) H.rcs[tid] = A.rope_cs[(size_t)p * (kHD / 2) + tid];
  __syncthreads();
  const int ns = attn_splits(A, p);
  if (warp == kCons) {
    if (lane == 0) producer<MOE>(A, H, smem, v, G, p, ns);
    return;
  }

  // ---- consumers --------------------------------------------------------
  const int item = v < A.nkv * ns ? v : -1;
  bf16* res = reinterpret_cast<bf16*>(smem + A.off_res);
  int seq = 0, rot = 0;
  int q0, q1, o0, o1, g0, g1, d0, d1;
  cta_range(A.geo[kMatQkv].lb_total, v, G, q0, q1);
  cta_range(A.geo[kMatO].lb_total, v, G, o0, o1);
  cta_range(A.geo[kMatGu].lb_total, v, G, g0, g1);
  down_range<MOE>(A, v, G, d0, d1);
  for (int l = 0; l < L; ++l) {
    const StepLayer& LW = A.layers[l];
    const unsigned flag = H.ebase + (unsigned)l + 1u;
    const int ab = l & 1;
    const uint32_t apar = (uint32_t)((l >> 1) & 1);
    const bf16* aux = reinterpret_cast<const bf16*>(smem + A.off_aux + ab * A.aux_stride);
    // ---- input norm + qkv: x of this layer into res (the o residual too)
    if (q1 > q0 || o1 > o0) {
      if (l == 0)
        load_res_embed(A, H.tok, res, tid);
      else
        load_res_fw(A.xw, A.H, flag - 1u, res, A, H, tid);
    }
    CSync::sync();
    if (aborted(H)) return;
    if (q1 > q0) {
      const PGeom& geo = A.geo[kMatQkv];
      wait_or_abort(&H.auxfull[ab], apar, &H.abort_flag, A.status);
      stage_norm(geo, pg_smem(smem, geo), res, aux, A.eps, H, tid);
      CSync::sync();
      gemv_any(A.bits[kMatQkv], A, H, smem, geo, q0, q1, seq, rot, tid);
      epilogue_fw<kOutStore>(geo, pg_smem(smem, geo), q0, q1, res, A.qkvw, flag, H.xsc, tid);
    }
    // ---- attention (its shared memory overlaps the GEMV phases' slots)
    CSync::sync();
    attn_phase<HPG>(A, H, smem, LW, aux, &H.auxfull[ab], apar, item, ns, p, flag, seq, tid);
    CSync::sync();
    if (aborted(H)) return;
    // ---- o projection + residual
    if (o1 > o0) {
      const PGeom& geo = A.geo[kMatO];
      stage_raw_fw(geo, pg_smem(smem, geo), A.attw, flag, A, H, tid);
      CSync::sync();
      if (aborted(H)) return;
      gemv_any(A.bits[kMatO], A, H, smem, geo, o0, o1, seq, rot, tid);
      epilogue_fw<kOutResid>(geo, pg_smem(smem, geo), o0, o1, res, A.xmw, flag, H.xsc, tid);
    }
    CSync::sync();
    if (MOE) {
      if (!moe_router_gu(A, H, smem, res, aux, ab, apar, l, flag, seq, rot, tid)) return;
    } else if (g1 > g0 || d1 > d0) {
      // ---- post-attention norm + gate|up + SwiGLU: x of the MLP into res
      // (the down residual too)
      load_res_fw(A.xmw, A.H, flag, res, A, H, tid);
    }
    CSync::sync();
    if (aborted(H)) return;
    if (!MOE && g1 > g0) {
      const PGeom& geo = A.geo[kMatGu];
      wait_or_abort(&H.auxfull[ab], apar, &H.abort_flag, A.status);
      stage_norm(geo, pg_smem(smem, geo), res, aux + A.H, A.eps, H, tid);
      CSync::sync();
      gemv_any(A.bits[kMatGu], A, H, smem, geo, g0, g1, seq, rot, tid);
      epilogue_fw<kOutSwiglu>(geo, pg_smem(smem, geo), g0, g1, res, A.hw, flag, H.xsc, tid);
    }
    // the aux buffer of this layer is read for the last time above.  It is
    // handed back only once its load has landed, also in a CTA that read none
    // of it: the producer's next load into the buffer must not overtake this
    // one (two loads on one phase of the count-1 barrier would complete it
    // once, and a later wait on it would never end)
    CSync::sync();
    if (tid == 0) {
      wait_or_abort(&H.auxfull[ab], apar, &H.abort_flag, A.status);
      mbar_arrive(&H.auxempty[ab]);
    }
    // ---- down projection + residual (MoE: the selected experts' down
    // projections, combined in the next input)
    if (MOE) {
      if (d1 > d0 && !moe_down(A, H, smem, res, d0, d1, flag, seq, rot, tid)) return;
    } else if (d1 > d0) {
      const PGeom& geo = A.geo[kMatDown];
      stage_raw_fw(geo, pg_smem(smem, geo), A.hw, flag, A, H, tid);
      CSync::sync();
      if (aborted(H)) return;
      gemv_any(A.bits[kMatDown], A, H, smem, geo, d0, d1, seq, rot, tid);
      epilogue_fw<kOutResid>(geo, pg_smem(smem, geo), d0, d1, res, A.xw, flag, H.xsc, tid);
    }
    CSync::sync();  // res and the slots are rewritten by the next layer
  }
  // ---- final norm + lm_head + greedy argmax -----------------------------
  float best_v = -INFINITY;
  int best_i = 0x7fffffff;
  {
    const PGeom& geo = A.geo[kMatLm];
    int m0, m1;
    cta_range(geo.lb_total, v, G, m0, m1);
    if (m1 > m0) {
      load_res_fw(A.xw, A.H, H.ebase + (unsigned)L, res, A, H, tid);
      CSync::sync();
      if (aborted(H)) return;
      const int lb = L & 1;
      const bf16* fnorm = reinterpret_cast<const bf16*>(smem + A.off_aux + lb * A.aux_stride);
      wait_or_abort(&H.auxfull[lb], (uint32_t)((L >> 1) & 1), &H.abort_flag, A.status);
      const PgSmem sm = pg_smem(smem, geo);
      stage_norm(geo, sm, res, fnorm, A.eps, H, tid);
      CSync::sync();
      gemv_any(A.bits[kMatLm], A, H, smem, geo, m0, m1, seq, rot, tid);
      const int SKP = geo.S * 2;
      const float xs = H.xsc;
      for (int i = tid; i < (m1 - m0) * 16; i += kNT) {
        const int n = m0 * 16 + i;
        const float val = bfround(row_value(sm.red, i, SKP, xs));
        if (A.logits) A.logits[n] = f2bf(val);
        if (val == val && (val > best_v || (val == best_v && n < best_i))) {
          best_v = val;
          best_i = n;
        }
      }
    }
  }
  if (aborted(H)) return;
  // ---- greedy token over all CTAs: (max, first index); the last CTA to
  // arrive (ticket) writes the token and moves the step on
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    argmax_pair(best_v, best_i, ov, oi);
  }
  if (lane == 0) {
    H.wv[warp] = best_v;
    H.wi[warp] = best_i;
  }
  CSync::sync();
  if (tid == 0) {
    float bv = H.wv[0];
    int bi = H.wi[0];
    for (int w = 1; w < kCons; ++w) argmax_pair(bv, bi, H.wv[w], H.wi[w]);
    A.am_val[v] = bv;
    A.am_idx[v] = bi;
    __threadfence();
    H.flag = (atomicAdd(A.am_ticket, 1u) == (unsigned)G - 1) ? 1u : 0u;
  }
  CSync::sync();
  if (!H.flag) return;
  __threadfence();
  if (warp == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < G; c += 32) argmax_pair(bv, bi, __ldcg(A.am_val + c), __ldcg(A.am_idx + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_pair(bv, bi, ov, oi);
    }
    if (lane == 0) {
      if (bi == 0x7fffffff) bi = 0;
      *A.token = bi;
      if (A.hist && A.hist_n) {
        const int hn = *A.hist_n;
        A.hist[hn % A.hist_cap] = bi;
        *A.hist_n = hn + 1;
      }
      *A.pos = p + 1;
      *A.am_ticket = 0u;
      *A.epoch = *reinterpret_cast<volatile unsigned*>(A.epoch) + 1u;
    }
  }
}

template <int HPG>
int attn_bytes() {
  return (int)sizeof(AttnSm<HPG>);
}

// The kernel of a plan: q heads per KV head, and dense or MoE (a compile-time
// switch: the dense kernel carries none of the MoE phases).
const void* kernel_for(int hpg, bool moe) {
  switch (hpg * 2 + (moe ? 1 : 0)) {
    case 2: return reinterpret_cast<const void*>(step_kernel<1, false>);
    case 3: return reinterpret_cast<const void*>(step_kernel<1, true>);
    case 4: return reinterpret_cast<const void*>(step_kernel<2, false>);
    case 5: return reinterpret_cast<const void*>(step_kernel<2, true>);
    case 8: return reinterpret_cast<const void*>(step_kernel<4, false>);
    case 9: return reinterpret_cast<const void*>(step_kernel<4, true>);
    case 16: return reinterpret_cast<const void*>(step_kernel<8, false>);
    case 17: return reinterpret_cast<const void*>(step_kernel<8, true>);
    default: return nullptr;
  }
}

}  // namespace

void step_exchange_words(const StepShape& sh, size_t words[kStepBuffers]) {
  const bool moe = sh.n_experts > 0;
  words[0] = (size_t)sh.H / 2;
  words[1] = (size_t)(sh.nq + 2 * sh.nkv) * kHD / 2;
  words[2] = (size_t)sh.nq * kHD / 2;
  words[3] = (size_t)sh.H / 2;
  words[4] = moe ? (size_t)sh.top_k * sh.moe_inter / 2 : (size_t)sh.I / 2;
  words[5] = moe ? (size_t)sh.n_experts / 2 : 0;
  for (int i = 0; i < kStepBuffers; ++i) words[i] = (words[i] + 1) & ~(size_t)1;  // 16-byte aligned starts
}

int step_make_plan(const StepShape& sh, int num_sms, int budget, StepPlan* plan) {
  static_assert(sizeof(StepArgs) <= 4096, "step arguments exceed the kernel parameter space");
  if (sh.gs != 64 || sh.hd != kHD || sh.nkv <= 0 || sh.nq % sh.nkv != 0 || num_sms <= 0) return -1;
  const int hpg = sh.nq / sh.nkv;
  if (hpg != 1 && hpg != 2 && hpg != 4 && hpg != 8) return -1;
  const bool moe = sh.n_experts > 0;
  if (sh.H % 64 != 0 || (!moe && sh.I % 64 != 0)) return -1;
  // MoE: routing with one expert per consumer thread (up to 256, their
  // probabilities in the H-wide residual buffer), the top-k slots' indices
  // in shared memory, expert widths in whole 64-wide groups
  if (moe && (sh.n_experts > kStepMaxExperts || sh.n_experts > sh.H || sh.n_experts % 16 != 0 || sh.top_k < 1 ||
              sh.top_k > kStepMaxTopK || sh.top_k > sh.n_experts || sh.moe_inter % 64 != 0))
    return -1;
  StepPlan P{};
  StepArgs& A = P.tmpl;
  memset(&A, 0, sizeof(A));
  P.grid = num_sms;
  P.hpg = hpg;
  A.nsm = num_sms;
  A.slot_bytes = kSlotBytes;
  A.off_aux = round128((int)sizeof(StepHdr));
  A.aux_stride = round128(4 * sh.H + 512);
  A.off_res = A.off_aux + 2 * A.aux_stride;
  A.off_u = A.off_res + round128(2 * sh.H);
  // MoE: gate|up over top_k slots of 2 moe_inter rows, down over the
  // top_k slots' blocks of each row block (x slot = block % top_k), and the
  // router
  const int Im = sh.moe_inter, k = sh.top_k;
  const int N[kStepMats] = {(sh.nq + 2 * sh.nkv) * kHD, sh.H, moe ? 2 * k * Im : 2 * sh.I, moe ? k * sh.H : sh.H,
                            sh.vocab, moe ? sh.n_experts : 0};
  const int K[kStepMats] = {sh.H, sh.nq * kHD, sh.H, moe ? Im : sh.I, sh.H, sh.H};
  const int epi[kStepMats] = {kEpiStore, kEpiResid, kEpiSwiglu, moe ? kEpiStore : kEpiResid, kEpiArgmax, kEpiStore};
  int end = A.off_u;
  for (int m = 0; m < (moe ? kStepMats : kStepMats - 1); ++m) {
    const int bits = sh.bits[m];
    if (bits != 4 && bits != 8) return -1;
    if (K[m] % 64 != 0) return -1;
    const int halves = epi[m] == kEpiSwiglu ? 2 : 1;
    if ((N[m] / halves) % 16 != 0) return -1;
    const int W = N[m] / halves / 16;
    const int lbs_max =
        moe && m == kMatDown ? (sh.H / 16 + num_sms - 1) / num_sms * k : (W + num_sms - 1) / num_sms;
    const int tb = ptile_bytes(bits, 64);
    const int st = kSlotBytes / tb;
    if (st < 1) return -1;
    const int xs = moe && m == kMatDown ? k : 1;
    pgeom_make(&A.geo[m], K[m], bits, 64, epi[m], W, st, 0, xs, lbs_max, false);
    if (xs > 1) A.geo[m].xsl_mod = k;
    end = std::max(end, pgeom_layout(A.geo[m], 64, A.off_u));
    A.bits[m] = bits;
  }
  if (moe) {
    // the router reads the gate|up phase's staged x: the same place, and the
    // same code width (int4 staging pre-scales a quarter of x for the upper
    // nibble), else the model decodes through the kernel chain
    const PGeom &r = A.geo[kMatRouter], &g = A.geo[kMatGu];
    if (r.off_x != g.off_x || r.off_zero != g.off_zero || r.off_xs != g.off_xs || r.xslot_bytes != g.xslot_bytes ||
        r.bits != g.bits)
      return -1;
    A.moe = 1;
    A.n_experts = sh.n_experts;
    A.top_k = k;
    A.norm_topk = sh.norm_topk;
    A.egu_lps = Im / 16;
    A.edown_lps = sh.H / 16;
  }
  const int ab = hpg == 1 ? attn_bytes<1>() : hpg == 2 ? attn_bytes<2>() : hpg == 4 ? attn_bytes<4>() : attn_bytes<8>();
  end = std::max(end, A.off_u + ab);
  A.off_args = round128(end);
  end = A.off_args + (int)sizeof(StepArgs);
  A.off_ring = round128(end);
  const int nslots = std::min(kMaxSlots, (budget - A.off_ring) / kSlotBytes);
  if (nslots < 2) return -1;
  A.nslots = nslots;
  P.smem = A.off_ring + nslots * kSlotBytes;
  A.max_splits = std::min(kMaxSplitsMerge, num_sms / sh.nkv);
  if (A.max_splits < 1) return -1;
  A.n_layers = sh.layers;
  A.H = sh.H;
  A.I = sh.I;
  A.nq = sh.nq;
  A.nkv = sh.nkv;
  A.cap = sh.cap;
  A.vocab = sh.vocab;
  A.scale = 1.0f / sqrtf((float)kHD);
  A.scale_log2e = A.scale * 1.4426950408889634f;
  *plan = P;
  return 0;
}

int step_occupancy(const StepPlan& p) {
  const void* k = kernel_for(p.hpg, p.tmpl.moe != 0);
  if (!k) return 0;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem) != cudaSuccess) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kThreads, p.smem) != cudaSuccess) return 0;
  return n;
}

cudaError_t step_launch(const StepArgs& a, const StepPlan& p, cudaStream_t st, bool coop) {
  const void* k = kernel_for(p.hpg, p.tmpl.moe != 0);
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
