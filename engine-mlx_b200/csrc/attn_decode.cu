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
// merges the slices.  Only ceil(L / kMinRows) splits (at most the grid's) take
// part, so short contexts do not pay for a wide merge; the others return at
// once.  Before griddepcontrol.wait each CTA asks L2 to prefetch its K/V
// slice (a hint only, so a stale offset is harmless).
#include "attn_decode.cuh"

namespace emx {

namespace {

constexpr int kHD = 128;
constexpr int kThreads = 128;
constexpr int kTile = 128;
constexpr int kMinRows = 64;  // fewest rows a split is given

__device__ __forceinline__ int active_splits(int L, int grid) {
  const int s = (L + kMinRows - 1) / kMinRows;
  return s < grid ? s : grid;
}

template <int HPG>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(const AttnDecodeArgs a) {
  __shared__ float qs[HPG][kHD];       // q * scale (fp32 of the bf16 rope output)
  __shared__ float qn[HPG + 1][kHD];   // normed q heads (+ k) before rope
  __shared__ float sc[HPG][kTile];     // scores -> probabilities for one tile
  __shared__ float stat_m[HPG], stat_l[HPG], stat_a[HPG];
  __shared__ float sacc[4][HPG][kHD];  // per-warp partial outputs
  __shared__ float swt[HPG][64];       // merge weights of the splits
  __shared__ unsigned last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const size_t head_stride = (size_t)a.cap * kHD;
  bf16* kc = a.kc + (size_t)kvh * head_stride;
  bf16* vc = a.vc + (size_t)kvh * head_stride;

  pdl_trigger();
  // ---- L2 warm-up of this CTA's K/V rows (offset may be one step stale) ----
  if (tid == 0) {
    const int pg = a.pos ? *reinterpret_cast<const volatile int*>(a.pos) : a.pos_host;
    const int splits = active_splits(pg + 1, gridDim.x);
    if (pg >= 0 && pg < a.cap && split < splits) {
      const int L = pg + 1;
      const int p0 = (int)((long long)split * L / splits), p1 = (int)((long long)(split + 1) * L / splits);
      if (p1 > p0) {
        const uint32_t bytes = (uint32_t)(p1 - p0) * kHD * 2;
        bulk_prefetch_l2(kc + (size_t)p0 * kHD, bytes);
        bulk_prefetch_l2(vc + (size_t)p0 * kHD, bytes);
      }
    }
  }
  pdl_wait();

  const int p = a.pos ? *a.pos : a.pos_host;
  if (p < 0 || p >= a.cap) {
    if (tid == 0 && split == 0 && kvh == 0) report_status(a.status, kDevKvOverflow);
    return;
  }
  const int L = p + 1;
  const int splits = active_splits(L, gridDim.x);
  if (split >= splits) return;
  const int p0 = (int)((long long)split * L / splits), p1 = (int)((long long)(split + 1) * L / splits);
  const bool owns_new = (p >= p0 && p < p1) && a.q_in == nullptr;

  // ---- q heads (and k/v of the new row when owned): rms_norm + rope -------
  const int nhead_prep = a.q_in ? 0 : HPG + (owns_new ? 1 : 0);
  if (a.q_in) {
    for (int i = tid; i < HPG * kHD; i += kThreads)
      qs[i / kHD][i % kHD] = __fmul_rn(bf2f(a.q_in[(size_t)kvh * HPG * kHD + i]), a.scale);
  }
  for (int hh = warp; hh < nhead_prep; hh += 4) {
    const bool is_k = hh == HPG;
    const bf16* src = is_k ? a.qkv + (size_t)a.nq * kHD + (size_t)kvh * kHD
                           : a.qkv + (size_t)(kvh * HPG + hh) * kHD;
    const bf16* nw = is_k ? a.k_norm : a.q_norm;
    float v[4];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[e] = bf2f(src[lane * 4 + e]);
      ss = fmaf(v[e], v[e], ss);
    }
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), a.eps)));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      qn[hh][d] = nw ? bfround(__fmul_rn(bfround(__fmul_rn(v[e], inv)), bf2f(nw[d]))) : v[e];
    }
    __syncwarp();
    const float fp = (float)p;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      const int i = d & (kHD / 2 - 1);
      const float th = __fmul_rn(fp, a.inv_freq[i]);
      float sn, cs;
      sincosf(th, &sn, &cs);
      const float x1 = qn[hh][i], x2 = qn[hh][i + kHD / 2];
      float o;
      if (d < kHD / 2) o = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      else o = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
      o = bfround(o);
      if (is_k) kc[(size_t)p * kHD + d] = f2bf(o);
      else qs[hh][d] = __fmul_rn(o, a.scale);
    }
    if (is_k) {
      const bf16* vsrc = a.qkv + (size_t)(a.nq + a.nkv) * kHD + (size_t)kvh * kHD;
#pragma unroll
      for (int e = 0; e < 4; ++e) vc[(size_t)p * kHD + lane * 4 + e] = vsrc[lane * 4 + e];
    }
  }
  if (tid < HPG) {
    stat_m[tid] = -INFINITY;
    stat_l[tid] = 0.f;
  }
  __syncthreads();

  // per-lane q slice: 8 dims starting at dl, for every head of the group
  const int half = lane >> 4, dl = (lane & 15) * 8;
  float qreg[HPG][8];
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int e = 0; e < 8; ++e) qreg[h][e] = qs[h][dl + e];

  float acc[HPG][8];
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;

  for (int t0 = p0; t0 < p1; t0 += kTile) {
    const int tn = min(kTile, p1 - t0);
    // QK^T: two rows per warp step, 16 lanes x 8 dims per row
    // (trip count uniform across the warp: both halves run every shuffle)
    for (int jb = warp * 2; jb < tn; jb += 8) {
      const int jj = jb + half;
      const bool valid = jj < tn;
      const uint4 kv = valid ? *reinterpret_cast<const uint4*>(kc + (size_t)(t0 + jj) * kHD + dl)
                             : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        kf[2 * e] = __uint_as_float(kw[e] << 16);
        kf[2 * e + 1] = __uint_as_float(kw[e] & 0xffff0000u);
      }
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(qreg[h][e], kf[e], s);
        s += __shfl_xor_sync(0xffffffffu, s, 8);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (valid && (lane & 15) == 0) sc[h][jj] = s;
      }
    }
    __syncthreads();
    // online softmax update at tile granularity (one warp per head)
    for (int h = warp; h < HPG; h += 4) {
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
    // P.V: 8 row slots (4 warps x 2 halves), 8 dims per lane
#pragma unroll
    for (int h = 0; h < HPG; ++h) {
      const float al = stat_a[h];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] *= al;
    }
    for (int jj = warp * 2 + half; jj < tn; jj += 8) {
      const uint4 vv = *reinterpret_cast<const uint4*>(vc + (size_t)(t0 + jj) * kHD + dl);
      const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
      float vf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        vf[2 * e] = __uint_as_float(vw[e] << 16);
        vf[2 * e + 1] = __uint_as_float(vw[e] & 0xffff0000u);
      }
#pragma unroll
      for (int h = 0; h < HPG; ++h) {
        const float pr = sc[h][jj];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[h][e] = fmaf(pr, vf[e], acc[h][e]);
      }
    }
    __syncthreads();
  }

  // ---- merge the 8 row slots, publish this split's partial ---------------
#pragma unroll
  for (int h = 0; h < HPG; ++h)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[h][e] += __shfl_xor_sync(0xffffffffu, acc[h][e], 16);
  if (half == 0) {
#pragma unroll
    for (int h = 0; h < HPG; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) sacc[warp][h][dl + e] = acc[h][e];
  }
  __syncthreads();
  const size_t part_stride = (size_t)HPG * (kHD + 2);
  float* part = a.part + ((size_t)kvh * splits + split) * part_stride;
  for (int i = tid; i < HPG * kHD; i += kThreads) {
    const int h = i / kHD, d = i % kHD;
    part[h * (kHD + 2) + 2 + d] = sacc[0][h][d] + sacc[1][h][d] + sacc[2][h][d] + sacc[3][h][d];
  }
  if (tid < HPG) {
    part[tid * (kHD + 2) + 0] = stat_m[tid];
    part[tid * (kHD + 2) + 1] = stat_l[tid];
  }
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
  for (int h = warp; h < HPG; h += 4) {
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, a.nkv);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<HPG>, a);
}

}  // namespace

int attn_decode_splits(int nkv, int num_sms) {
  int s = num_sms / (nkv > 0 ? nkv : 1);
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return s;
}

cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  if (a.head_dim != kHD || a.nkv <= 0 || a.nq % a.nkv != 0) return cudaErrorInvalidValue;
  switch (a.nq / a.nkv) {
    case 1: return launch_t<1>(a, st, pdl);
    case 2: return launch_t<2>(a, st, pdl);
    case 4: return launch_t<4>(a, st, pdl);
    case 8: return launch_t<8>(a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace emx
