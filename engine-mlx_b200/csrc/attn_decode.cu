// attn_decode.cu — batch-1 decode attention over the static bf16 KV cache.
//
// Replaces, for one decode step of one layer, the chain of the traced step
// (crates/serve/src/compiled.rs:134-177): slice q/k/v out of the fused qkv
// projection, q_norm/k_norm rms_norm, rope_dynamic at the device-held offset,
// scatter_single of k/v into the static cache at that offset, and
// sdpa_masked over the cache with the 0/-1e9 additive mask
// (crates/mlx-ffi/src/ops/real/transform.rs:8-30, engine_ext.rs:238-260).
//
// The mask only admits rows 0..offset, so this kernel reads exactly those
// rows (the reference reads all `cap` rows and multiplies the rest by
// exp(-1e9 - m) == 0).  Work split: grid (splits, n_kv); each CTA owns one KV
// head (and the q heads that share it) over a contiguous slice of the valid
// rows, keeps the softmax partial (m, l, acc), and the last CTA of a head
// merges the slices.  Only ceil(L / kAttnMinRows) splits (at most the grid's) take
// part, so short contexts do not pay for a wide merge; the others return at
// once.
//
// Every cached row before the new one is final before this kernel starts
// (it was written by an earlier step), so before griddepcontrol.wait each
// CTA asks the bulk-copy engine for its first 64-row K and V tiles (a ring of
// two) and stages the norm weights and RoPE frequencies: after the wait only
// the new row's q/k/v depend on the previous kernel.  The position is read
// again after the wait; should it differ from the one the copies were
// planned with, the CTA lets those copies land and plans again.
#include "attn_decode.cuh"

namespace emx {

namespace {

constexpr int kHD = 128;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 64;     // rows per K / V tile
// tiles in flight (a buffer is refilled with the tile kNBuf ahead): two, so
// that two CTAs of the kernel share an SM
constexpr int kNBuf = 2;
constexpr int kTileBytes = kTile * kHD * 2;
constexpr int kDynSmem = 128 + 2 * kNBuf * kTileBytes;

__device__ __forceinline__ void split_range(int L, int splits, int split, int& p0, int& p1) {
  p0 = (int)((long long)split * L / splits);
  p1 = (int)((long long)(split + 1) * L / splits);
}

template <int HPG>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(const AttnDecodeArgs a) {
  extern __shared__ __align__(128) unsigned char dsm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(dsm);
  bf16* kb = reinterpret_cast<bf16*>(dsm + 128);  // [kNBuf][kTile][kHD]
  bf16* vb = kb + kNBuf * kTile * kHD;
  __shared__ float qs[HPG][kHD];       // q * scale (fp32 of the bf16 rope output)
  __shared__ float qn[HPG + 1][kHD];   // normed q heads (+ k) before rope
  __shared__ float sc[HPG][kTile];     // scores -> probabilities for one tile
  __shared__ float stat_m[HPG], stat_l[HPG], stat_a[HPG];
  __shared__ __align__(16) float sacc[kWarps][HPG][kHD];  // per-warp partial outputs (float4 stores)
  __shared__ float swt[HPG][64];       // merge weights of the splits
  __shared__ float nwq[kHD], nwk[kHD], invf[kHD / 2];
  __shared__ float2 rcs[kHD / 2];  // (cos, sin) of this step's angles
  __shared__ int rcs_pos;          // position rcs was loaded for (-1: none)
  __shared__ __align__(16) bf16 knew[kHD];  // the new row (owner split)
  __shared__ __align__(16) bf16 vnew[kHD];
  __shared__ int base_use[kNBuf];  // completed uses of each buffer before this plan
  __shared__ int plan_p;           // position the issued copies were planned for
  __shared__ unsigned last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const size_t head_stride = (size_t)a.cap * kHD;
  bf16* kc = a.kc + (size_t)kvh * head_stride;
  bf16* vc = a.vc + (size_t)kvh * head_stride;

  if (tid == 0) {
    for (int i = 0; i < kNBuf; ++i) {
      mbar_init(&mbar[i], 1);
      base_use[i] = 0;
    }
    fence_mbar_init();
    rcs_pos = -1;
  }
  // static inputs (weights, RoPE table) before the wait
  if (!a.q_in) {
    for (int i = tid; i < kHD; i += kThreads) {
      nwq[i] = a.q_norm ? bf2f(a.q_norm[i]) : 1.0f;
      nwk[i] = a.k_norm ? bf2f(a.k_norm[i]) : 1.0f;
    }
    for (int i = tid; i < kHD / 2; i += kThreads) invf[i] = a.inv_freq[i];
  }
  __syncthreads();

  // Tile t of the current plan: rows [p0 + 64t, ...) of this split, minus
  // the new row p when this kernel computes it (never copied); buffer
  // t % kNBuf.  With q given (no new row) every row up to p is copied.
  const int row_end_adj = a.q_in ? 1 : 0;
  auto issue = [&](int t, int p, int p0, int p1) {
    const int buf = t % kNBuf;
    const int r0 = p0 + t * kTile;
    const int r1 = min(min(r0 + kTile, p1), p + row_end_adj);
    const uint32_t bytes = r1 > r0 ? (uint32_t)(r1 - r0) * kHD * 2 : 0u;
    mbar_arrive_expect_tx(&mbar[buf], 2 * bytes);
    if (bytes) {
      bulk_g2s(kb + (size_t)buf * kTile * kHD, kc + (size_t)r0 * kHD, bytes, &mbar[buf]);
      bulk_g2s(vb + (size_t)buf * kTile * kHD, vc + (size_t)r0 * kHD, bytes, &mbar[buf]);
    }
  };
  auto parity = [&](int t) -> uint32_t { return (uint32_t)((base_use[t % kNBuf] + t / kNBuf) & 1); };

  // this step's RoPE angles: every row of the table is final before the
  // kernel starts, so fetch the row of the (pre-wait) position now
  {
    const int pg = a.pos ? *reinterpret_cast<const volatile int*>(a.pos) : a.pos_host;
    if (!a.q_in && a.rope_cs && pg >= 0 && pg < a.cap) {
      if (tid < kHD / 2) rcs[tid] = a.rope_cs[(size_t)pg * (kHD / 2) + tid];
      if (tid == 0) rcs_pos = pg;
    }
  }
  int n_issued = 0;  // thread 0: tiles issued under the current plan
  if (tid == 0) {
    plan_p = -1;
    const int pg = a.pos ? *reinterpret_cast<const volatile int*>(a.pos) : a.pos_host;
    if (pg >= 0 && pg < a.cap) {
      const int splits = attn_active_splits(pg + 1, gridDim.x);
      if (split < splits) {
        int p0, p1;
        split_range(pg + 1, splits, split, p0, p1);
        const int ntile = (p1 - p0 + kTile - 1) / kTile;
        for (; n_issued < min(ntile, kNBuf); ++n_issued) issue(n_issued, pg, p0, p1);
        if (p1 - p0 > kNBuf * kTile) {  // later tiles: an L2 hint only
          const uint32_t rest = (uint32_t)(p1 - p0 - kNBuf * kTile) * kHD * 2;
          bulk_prefetch_l2(kc + (size_t)(p0 + kNBuf * kTile) * kHD, rest);
          bulk_prefetch_l2(vc + (size_t)(p0 + kNBuf * kTile) * kHD, rest);
        }
        plan_p = pg;
      }
    }
  }
  pdl_wait();
  // the next kernel may launch once this one's inputs are final: one kernel
  // ahead streams its weights beside this one, while an earlier trigger lets
  // the chain run several kernels ahead and the block scheduler then stacks
  // two CTAs of one launch on an SM while others hold none
  pdl_trigger();

  const int p = a.pos ? *a.pos : a.pos_host;
  const bool bad = p < 0 || p >= a.cap;
  const int L = p + 1;
  const int splits = bad ? 0 : attn_active_splits(L, gridDim.x);
  int p0 = 0, p1 = 0;
  if (!bad) split_range(L, splits, split, p0, p1);
  const int ntile = (p1 - p0 + kTile - 1) / kTile;
  // a plan for another position (or one no longer needed): let its copies land
  if (tid == 0 && plan_p >= 0 && (plan_p != p || bad || split >= splits)) {
    for (int t = 0; t < n_issued; ++t) mbar_wait_bounded(&mbar[t % kNBuf], parity(t), a.status);
    for (int b = 0; b < kNBuf; ++b) base_use[b] += (n_issued + kNBuf - 1 - b) / kNBuf;
    n_issued = 0;
    plan_p = -1;
  }
  if (bad || split >= splits) {
    if (bad && tid == 0 && split == 0 && kvh == 0) report_status(a.status, kDevKvOverflow);
    return;
  }
  if (tid == 0 && plan_p < 0) {
    for (; n_issued < min(ntile, kNBuf); ++n_issued) issue(n_issued, p, p0, p1);
    plan_p = p;
  }
  const bool owns_new = (p >= p0 && p < p1) && a.q_in == nullptr;
  __syncthreads();  // rcs / rcs_pos visible
  const bool have_rcs = rcs_pos == p;

  // ---- q heads (and k/v of the new row when owned): rms_norm + rope -------
  const int nhead_prep = a.q_in ? 0 : HPG + (owns_new ? 1 : 0);
  if (a.q_in) {
    for (int i = tid; i < HPG * kHD; i += kThreads)
      qs[i / kHD][i % kHD] = __fmul_rn(bf2f(a.q_in[(size_t)kvh * HPG * kHD + i]), a.scale);
  }
  for (int hh = warp; hh < nhead_prep; hh += kWarps) {
    const bool is_k = hh == HPG;
    const bf16* src = is_k ? a.qkv + (size_t)a.nq * kHD + (size_t)kvh * kHD
                           : a.qkv + (size_t)(kvh * HPG + hh) * kHD;
    const float* nw = is_k ? nwk : nwq;
    const bool has_norm = is_k ? a.k_norm != nullptr : a.q_norm != nullptr;
    float v[4];
    float ss = 0.f;
    const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
    v[0] = __uint_as_float(raw.x << 16);
    v[1] = __uint_as_float(raw.x & 0xffff0000u);
    v[2] = __uint_as_float(raw.y << 16);
    v[3] = __uint_as_float(raw.y & 0xffff0000u);
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = fmaf(v[e], v[e], ss);
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), a.eps)));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      qn[hh][d] = has_norm ? bfround(__fmul_rn(bfround(__fmul_rn(v[e], inv)), nw[d])) : v[e];
    }
    __syncwarp();
    const float fp = (float)p;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      const int i = d & (kHD / 2 - 1);
      float sn, cs;
      if (have_rcs) {
        const float2 t2 = rcs[i];
        cs = t2.x;
        sn = t2.y;
      } else {
        sincosf(__fmul_rn(fp, invf[i]), &sn, &cs);
      }
      const float x1 = qn[hh][i], x2 = qn[hh][i + kHD / 2];
      float o;
      if (d < kHD / 2) o = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      else o = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
      o = bfround(o);
      if (is_k) {
        kc[(size_t)p * kHD + d] = f2bf(o);
        knew[d] = f2bf(o);
      } else {
        qs[hh][d] = __fmul_rn(o, a.scale);
      }
    }
    if (is_k) {
      const bf16* vsrc = a.qkv + (size_t)(a.nq + a.nkv) * kHD + (size_t)kvh * kHD;
      const uint2 vr = *reinterpret_cast<const uint2*>(vsrc + lane * 4);
      *reinterpret_cast<uint2*>(vc + (size_t)p * kHD + lane * 4) = vr;
      *reinterpret_cast<uint2*>(vnew + lane * 4) = vr;
    }
  }
  if (tid < HPG) {
    stat_m[tid] = -INFINITY;
    stat_l[tid] = 0.f;
  }
  __syncthreads();

  // lane l owns dims [4l, 4l+4) of every head of the group
  float qreg[HPG][4];
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) qreg[h][e] = qs[h][lane * 4 + e];

  float acc[HPG][4];
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[h][e] = 0.f;

  for (int t = 0; t < ntile; ++t) {
    const int buf = t % kNBuf;
    const int t0 = p0 + t * kTile;
    const int tn = min(kTile, p1 - t0);
    bf16* kt = kb + (size_t)buf * kTile * kHD;
    bf16* vt = vb + (size_t)buf * kTile * kHD;
    mbar_wait_bounded(&mbar[buf], parity(t), a.status);
    // the new row is never copied: the owner puts it in place
    if (owns_new && p >= t0 && p < t0 + tn) {
      const int r = p - t0;
      if (tid < kHD / 8) {
        reinterpret_cast<uint4*>(kt + (size_t)r * kHD)[tid] = reinterpret_cast<const uint4*>(knew)[tid];
        reinterpret_cast<uint4*>(vt + (size_t)r * kHD)[tid] = reinterpret_cast<const uint4*>(vnew)[tid];
      }
      __syncthreads();
    }
    // QK^T: warp w scores rows [8w, 8w + 8).  Each lane forms its 4-dim
    // partial of all eight rows, then a transpose-reduction (xor 16, 8, 4:
    // halve the rows a lane keeps; xor 2, 1: plain sums) leaves row k's
    // score in lanes 4k..4k+3 — 9 shuffles per head for eight rows.
    if (warp * 8 < tn) {
      const int r0 = warp * 8;
      float kf[8][4];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint2 kv = r0 + r < tn ? *reinterpret_cast<const uint2*>(kt + (size_t)(r0 + r) * kHD + lane * 4)
                                     : make_uint2(0u, 0u);
        kf[r][0] = __uint_as_float(kv.x << 16);
        kf[r][1] = __uint_as_float(kv.x & 0xffff0000u);
        kf[r][2] = __uint_as_float(kv.y << 16);
        kf[r][3] = __uint_as_float(kv.y & 0xffff0000u);
      }
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float s2 = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) s2 = fmaf(qreg[h][e], kf[r][e], s2);
          v[r] = s2;
        }
        // xor 16: lanes < 16 keep rows 0-3, the others rows 4-7
        const bool up16 = (lane & 16) != 0;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const float send = up16 ? v[r] : v[r + 4];
          const float keep = up16 ? v[r + 4] : v[r];
          v[r] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
        // xor 8: keep 2 of the 4
        const bool up8 = (lane & 8) != 0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float send = up8 ? v[r] : v[r + 2];
          const float keep = up8 ? v[r + 2] : v[r];
          v[r] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        // xor 4: keep 1 of the 2
        const bool up4 = (lane & 4) != 0;
        {
          const float send = up4 ? v[0] : v[1];
          const float keep = up4 ? v[1] : v[0];
          v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
        // lane 4k holds row k' where k' = 4*bit16 + 2*bit8 + bit4 of the lane
        const int k = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        if ((lane & 3) == 0 && r0 + k < tn) sc[h][r0 + k] = v[0];
      }
    }
    __syncthreads();
    // online softmax update at tile granularity (one warp per head)
    for (int h = warp; h < HPG; h += kWarps) {
      float m = -INFINITY;
      for (int j = lane; j < tn; j += 32) m = fmaxf(m, sc[h][j]);
      m = warp_max(m);
      const float mo = stat_m[h];
      const float mn = fmaxf(mo, m);
      float l = 0.f;
      for (int j = lane; j < tn; j += 32) {
        const float e = expf(sc[h][j] - mn);
        sc[h][j] = e;
        l += e;
      }
      l = warp_sum(l);
      __syncwarp();
      if (lane == 0) {
        const float alpha = (mo == -INFINITY) ? 0.f : expf(mo - mn);
        stat_a[h] = alpha;
        stat_l[h] = stat_l[h] * alpha + l;
        stat_m[h] = mn;
      }
    }
    __syncthreads();
    // P.V: warp w accumulates rows [8w, 8w + 8) into its 4 dims per lane
#pragma unroll
    for (int h = 0; h < HPG; ++h) {
      const float al = stat_a[h];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[h][e] *= al;
    }
    const int rend = min(tn, warp * 8 + 8);
    for (int jj = warp * 8; jj < rend; ++jj) {
      const uint2 vv = *reinterpret_cast<const uint2*>(vt + (size_t)jj * kHD + lane * 4);
      const float vf[4] = {__uint_as_float(vv.x << 16), __uint_as_float(vv.x & 0xffff0000u),
                           __uint_as_float(vv.y << 16), __uint_as_float(vv.y & 0xffff0000u)};
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        const float pr = sc[h][jj];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] = fmaf(pr, vf[e], acc[h][e]);
      }
    }
    __syncthreads();
    // refill this buffer with the tile kNBuf ahead
    if (tid == 0 && t + kNBuf < ntile) {
      fence_proxy_async();
      issue(t + kNBuf, p, p0, p1);
    }
  }

  // ---- the warps' row slots, then this split's partial --------------------
#pragma unroll
  for (int h = 0; h < HPG; ++h)
    *reinterpret_cast<float4*>(&sacc[warp][h][lane * 4]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  __syncthreads();
  // the warps' row slots of one output element, in warp order
  auto warp_total = [&](int h, int d) -> float {
    float num = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) num += sacc[w][h][d];
    return num;
  };
  const bool defer = a.defer_merge && splits <= kAttnDeferSplits;
  if (splits == 1 && !defer) {
    // a single split needs no merge: normalise and store
    for (int i = tid; i < HPG * kHD; i += kThreads) {
      const int h = i / kHD, d = i % kHD;
      const float num = warp_total(h, d);
      a.out[(size_t)(kvh * HPG + h) * kHD + d] = f2bf(__fmul_rn(num, __fdiv_rn(1.0f, stat_l[h])));
    }
    return;
  }
  const size_t part_stride = (size_t)HPG * (kHD + 2);
  float* part = a.part + ((size_t)kvh * splits + split) * part_stride;
  for (int i = tid; i < HPG * kHD; i += kThreads) {
    const int h = i / kHD, d = i % kHD;
    part[h * (kHD + 2) + 2 + d] = warp_total(h, d);
  }
  if (tid < HPG) {
    part[tid * (kHD + 2) + 0] = stat_m[tid];
    part[tid * (kHD + 2) + 1] = stat_l[tid];
  }
  if (defer) return;  // the consumer merges
  __threadfence();
  __syncthreads();
  if (tid == 0) last = (atomicAdd(&a.ticket[kvh], 1u) == (unsigned)splits - 1) ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge: the splits' (m, l) into per-split weights exp(m_s - M) / sum, then
  // every output element sums its splits with all loads in flight at once
  // (L2-coherent loads: the partials were written by other CTAs)
  const float* pb = a.part + (size_t)kvh * splits * part_stride;
  for (int h = warp; h < HPG; h += kWarps) {
    float ms = -INFINITY, ls = 0.f;
    if (lane < splits) {
      ms = __ldcg(pb + (size_t)lane * part_stride + h * (kHD + 2));
      ls = __ldcg(pb + (size_t)lane * part_stride + h * (kHD + 2) + 1);
    }
    float ms2 = -INFINITY, ls2 = 0.f;
    if (lane + 32 < splits) {
      ms2 = __ldcg(pb + (size_t)(lane + 32) * part_stride + h * (kHD + 2));
      ls2 = __ldcg(pb + (size_t)(lane + 32) * part_stride + h * (kHD + 2) + 1);
    }
    const float M = warp_max(fmaxf(ms, ms2));
    const float w1 = ms == -INFINITY ? 0.f : expf(ms - M), w2 = ms2 == -INFINITY ? 0.f : expf(ms2 - M);
    const float den = warp_sum(fmaf(w1, ls, w2 * ls2));
    if (lane < splits) swt[h][lane] = __fdiv_rn(w1, den);
    if (lane + 32 < splits) swt[h][lane + 32] = __fdiv_rn(w2, den);
  }
  __syncthreads();
  for (int i = tid; i < HPG * kHD; i += kThreads) {
    const int h = i / kHD, d = i % kHD;
    const float* src = pb + h * (kHD + 2) + 2 + d;
    float num = 0.f;
#pragma unroll 8
    for (int s2 = 0; s2 < splits; ++s2) num = fmaf(swt[h][s2], __ldcg(src + (size_t)s2 * part_stride), num);
    a.out[(size_t)(kvh * HPG + h) * kHD + d] = f2bf(num);
  }
  if (tid == 0) a.ticket[kvh] = 0u;
}

template <int HPG>
cudaError_t launch_t(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  auto kern = attn_decode_kernel<HPG>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, a.nkv);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kDynSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

__global__ void rope_table_kernel(float2* cs, const float* inv_freq, int cap, int half) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)cap * half) return;
  const int p = (int)(i / half), k = (int)(i % half);
  float sn, c;
  sincosf(__fmul_rn((float)p, inv_freq[k]), &sn, &c);
  cs[i] = make_float2(c, sn);
}

}  // namespace

cudaError_t rope_table_fill(float2* cs, const float* inv_freq, int cap, int half, cudaStream_t st) {
  const size_t n = (size_t)cap * half;
  rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(cs, inv_freq, cap, half);
  return cudaGetLastError();
}

int attn_decode_splits(int nkv, int num_sms, int hpg) {
  // two CTAs per SM (twice the warps hiding the per-row latency; +10% decode
  // at an 8192-row context) unless the partials of eight q heads per KV head
  // would no longer fit the static scratch of the allocation-free entry point
  int s = (hpg >= 8 ? 1 : 2) * num_sms / (nkv > 0 ? nkv : 1);
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return s;
}

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  if (a.head_dim != kHD || a.nkv <= 0 || a.nq % a.nkv != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.kc) | reinterpret_cast<uintptr_t>(a.vc)) & 15) return cudaErrorInvalidValue;
  switch (a.nq / a.nkv) {
    case 1: return launch_t<1>(a, st, pdl);
    case 2: return launch_t<2>(a, st, pdl);
    case 4: return launch_t<4>(a, st, pdl);
    case 8: return launch_t<8>(a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace emx
