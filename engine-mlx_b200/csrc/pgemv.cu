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
// gives four slices' A registers; a LOP3 per register turns codes into fp16
// (magic-number exponent, exact) and an m16n8k16 MMA per slice adds the
// four group dot products of rows g, g+8 at once: column j < 4 of B holds x
// masked to group j, so only the lanes with g == t load x (two adjacent
// registers per slice from one 8-byte run) and the other lanes read a zero
// block; x groups sit 2*gs + 16 bytes apart, so the four loading lanes hit
// four different bank groups.  Each warp runs two units at once, interleaved
// quad by quad, so one unit's accumulator drain overlaps the other's math.
// x is staged in fp16 after an exact power-of-two scaling (pgemv_dev.cuh).
// Then per row s*(dot - 1024*sum x'') + b*sum x' in fp32 — the MLX qmv
// factorisation, 1024 being the magic offset — reduced over the lane pair and
// stored to a per-(row, span, half-span) slot.  After the last stage one
// barrier, then the epilogue sums each row's slots in order and applies the
// fused output step (store / residual / SwiGLU / argmax / fp32 partial).
#include "pgemv.cuh"

#include <algorithm>

#include "pgemv_dev.cuh"

namespace emx {

namespace {

using namespace pg;

constexpr int kConsumers = 8;
constexpr int kThreads = (kConsumers + 1) * 32;

template <int BITS, int GS>
__global__ void __launch_bounds__(kThreads, 2) pgemv_kernel(const GemvArgs a, const PGeom geo) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxBuf;
  float* scratch = reinterpret_cast<float*>(smem + 128);  // 32 floats
  float* inv = scratch + 32;                             // 8 floats
  float* xsc = scratch + 40;                             // 2^e of the x staging
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 320);
  uint64_t* nwbar = reinterpret_cast<uint64_t*>(smem + 336);
  const PgSmem sm = pg_smem(smem, geo);
  unsigned char* bufs = smem + geo.off_buf;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool gather = a.slot_expert != nullptr;
  const int lb_tiles = geo.halves * geo.S;
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
  const bool norm_pre = a.pro != kProX && a.pro != kProMerge;
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
  // the next kernel may launch once this one's inputs are final: one kernel
  // ahead streams its weights beside this one, while an earlier trigger lets
  // the chain run several kernels ahead and the block scheduler then stacks
  // two CTAs of one launch on an SM while others hold none
  pdl_trigger();

  if (gather) {
    lb_total = min(*a.n_slots * lps, geo.lb_total);
    partition();
    if (producer) {
      issued = min(geo.nbuf, nst);
      for (int st = 0; st < issued; ++st) issue(st);
    }
  }

  float res_pre[2];
  const bool res_early = pg_res_early(a, lb0, lb1, tid, kThreads, res_pre);

  int tok = 0;
  if (a.pro == kProEmbedNorm) {
    tok = *a.token;
    if (tok < 0 || tok >= a.vocab) {
      if (tid == 0) report_status(a.status, kDevBadToken);
      tok = 0;
    }
  }

  pg_prologue<GS, SyncCta>(a, geo, sm, reinterpret_cast<const bf16*>(smem + geo.off_nw), norm_pre ? nwbar : nullptr,
                           0u, scratch, inv, xsc, abort_flag, tok, tid, kThreads, blockIdx.x == 0);
  __syncthreads();

  float best_v = -INFINITY;
  int best_i = 0x7fffffff;

  if (warp < kConsumers) {
    for (int st = 0; st < nst; ++st) {
      const int buf = st % geo.nbuf;
      const int a0 = T0 + st * geo.stage_tiles, a1 = min(T1, a0 + geo.stage_tiles);
      if (wait_or_abort(&full[buf], (uint32_t)((st / geo.nbuf) & 1), abort_flag, a.status))
        pg_stage<BITS, GS>(geo, sm, bufs + (size_t)buf * geo.stage_bytes, a0, a1, lb0, warp, lane, kConsumers, 0);
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

  pg_epilogue(a, geo, sm.red, lb0, lb1, tid, kThreads, res_early, res_pre, best_v, best_i, *xsc);
  if (a.epi == kEpiF32 && a.peer) {
    __shared__ unsigned published;
    pg_peer_publish<SyncCta>(a, tid, &published);
  }

  if (a.epi == kEpiArgmax) {
    __shared__ float wv[kConsumers + 1];
    __shared__ int wi[kConsumers + 1];
    __shared__ unsigned last;
    pg_argmax_merge<SyncCta>(a, best_v, best_i, blockIdx.x, gridDim.x, tid, kConsumers + 1, wv, wi, &last);
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
      // low nibbles of the two halves: A registers 0 / 1 (rows g, g+8 at k, k+1);
      // high nibbles: registers 2 / 3 (rows g, g+8 at k+2, k+3)
      const uint32_t word = code(rA, G, k) | (code(rA, G, k + 2) << 4) | (code(rB, G, k) << 8) |
                            (code(rB, G, k + 2) << 12) | (code(rA, G, k + 1) << 16) | (code(rA, G, k + 3) << 20) |
                            (code(rB, G, k + 1) << 24) | (code(rB, G, k + 3) << 28);
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
  (void)N;
  pgeom_make(g, K, bits, gs, epi, p.lb_total, p.stage_tiles, p.nbuf, p.x_slots, p.lbs_max,
             p.norm && p.x_slots == 1 && K <= 8192);
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
                    int ctas_per_sm, int norm) {
  if (!(bits == 4 || bits == 8) || !(gs == 32 || gs == 64 || gs == 128)) return -1;
  if (K <= 0 || N <= 0 || K % gs != 0) return -1;
  const bool sw = epi == kEpiSwiglu;
  if (sw && (N % 2 != 0)) return -1;
  const int halves = sw ? 2 : 1;
  const int lrows = N / halves;
  if (lrows % 16 != 0) return -1;
  const int LB = lrows / 16;
  PgemvPlan p{};
  p.norm = norm ? 1 : 0;
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
  const bool norm = a.pro != kProX && a.pro != kProMerge;
  if (norm && a.norm_groups > 8) return cudaErrorInvalidValue;
  if (a.pro != kProX && p.x_slots > 1) return cudaErrorInvalidValue;
  if (a.pro == kProMerge && (a.K != a.attn_hpg * (a.K / a.attn_hpg) || !a.attn_part || !a.attn_pos ||
                             a.attn_hpg < 1 || a.attn_grid < 1 || a.K % 128 != 0))
    return cudaErrorInvalidValue;
  PGeom g;
  make_pgeom(a.N, a.K, a.bits, a.gs, a.epi, p, &g);
  if (p.x_slots > 1) {
    if (a.slot_rows < 16 || a.slot_rows % 16 != 0) return cudaErrorInvalidValue;
    const unsigned long long lps = (unsigned long long)(a.slot_rows / 16);
    g.lps_magic = (0x100000000ull + lps - 1) / lps;
  }
  if (norm && (g.nw_bytes < a.K * 2 || (reinterpret_cast<uintptr_t>(a.norm_w) & 15) != 0))
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
