// misc.cu — standalone kernels: MLX affine (de)quantization, the seeded
// generator, RMSNorm, RoPE, SwiGLU pieces, argmax, softmax, embedding gather,
// the prefill q/k/v post-processing and static-cache writes.
//
// Each restates one mlx-c op the reference calls through MlxCtx
// (crates/mlx-ffi/src/ops/real/*): dequantize_weight (transform.rs:45-60),
// rms_norm (blas.rs:5-9), grouped_rms_norm (grouped_norm.rs:50-135),
// rope_dynamic (blas.rs:75-80), silu (blas.rs:33-37), multiply/add
// (blas.rs:17-31), argmax (array.rs:6-10), softmax_axis (elementwise.rs:68-72),
// take/embed (core.rs:5-14), slice_update / scatter_single (slice.rs:78-115).
#include "misc.cuh"
#include "moe_route.cuh"

#include <algorithm>

namespace emx {

namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Irwin-Hall(12) normal variate from three 64-bit hashes: the integer sum is
// exact, the int->float conversion and the 2^-16 scale are exact, so only
// std*z and mean+y round — identical on any IEEE host.
__device__ __forceinline__ float normal_at(uint64_t key, uint64_t i, float mean, float std) {
  uint32_t s = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = splitmix64(key + 3ull * i + (uint64_t)j);
    s += (uint32_t)(h & 0xffff) + (uint32_t)((h >> 16) & 0xffff) + (uint32_t)((h >> 32) & 0xffff) +
         (uint32_t)(h >> 48);
  }
  const int t = (int)s - 393210;
  const float z = __fmul_rn(__int2float_rn(t), 1.0f / 65536.0f);
  return __fadd_rn(mean, __fmul_rn(std, z));
}

inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  auto sm = [](uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
  };
  return sm(seed ^ sm(stream));
}

inline int blocks_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  if (b > (size_t)(1u << 30)) b = (size_t)(1u << 30);
  return (int)(b ? b : 1);
}

// One thread per packed word: 8 (int4) or 4 (int8) codes -> one vector store.
template <int BITS>
__global__ void dequant_kernel(const uint32_t* w, const bf16* s, const bf16* b, bf16* out, int N, int K, int gs) {
  constexpr int PER = 32 / BITS;
  const int wpr = K / PER, ng = K / gs;
  const long long total = (long long)N * wpr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / wpr), kw = (int)(i - (long long)n * wpr);
    const uint32_t word = w[i];
    const int g = kw * PER / gs;
    const bf16 sv = s[(size_t)n * ng + g], bv = b[(size_t)n * ng + g];
    __align__(16) bf16 v[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) v[e] = dequant1((word >> (BITS * e)) & ((1u << BITS) - 1u), sv, bv);
    bf16* dst = out + (size_t)n * K + (size_t)kw * PER;
    if (PER == 8) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
    else *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(v);
  }
}

// One thread per (row, group): min/max, scale/bias in bf16, then the codes.
// GEN: values are the generator's elements (row0 + n) * K_full + col0 + k of
// a [*, K_full] tensor, i.e. the shard [row0.., col0..col0+K) of the full one.
template <bool GEN>
__global__ void quant_kernel(const float* src_f, const bf16* src_b, uint64_t key, float std, uint32_t* w, bf16* s,
                             bf16* b, int N, int K, int gs, int bits, size_t row0, int col0, int K_full) {
  const int ng = K / gs;
  const size_t total = (size_t)N * ng;
  const int per = 32 / bits;
  const float maxq = (float)((1 << bits) - 1);
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(idx / ng), g = (int)(idx % ng);
    const size_t base = (size_t)n * K + (size_t)g * gs;
    const size_t gbase = (row0 + n) * (size_t)K_full + col0 + (size_t)g * gs;
    auto val = [&](int i) -> float {
      if (GEN) return normal_at(key, gbase + i, 0.0f, std);
      return src_f ? src_f[base + i] : bf2f(src_b[base + i]);
    };
    float mn = val(0), mx = mn;
    for (int i = 1; i < gs; ++i) {
      const float v = val(i);
      mn = v < mn ? v : mn;
      mx = v > mx ? v : mx;
    }
    const float scale = __fdiv_rn(__fsub_rn(mx, mn), maxq);
    const bf16 sb = f2bf(scale), bb = f2bf(mn);
    s[idx] = sb;
    b[idx] = bb;
    const float sf = bf2f(sb), bf = bf2f(bb);
    uint32_t* wr = w + (size_t)n * (K / per) + (size_t)g * gs / per;
    for (int wi = 0; wi < gs / per; ++wi) {
      uint32_t word = 0;
      for (int e = 0; e < per; ++e) {
        float q = 0.0f;
        if (sf > 0.0f) {
          q = rintf(__fdiv_rn(__fsub_rn(val(wi * per + e), bf), sf));
          q = q < 0.0f ? 0.0f : (q > maxq ? maxq : q);
        }
        word |= ((uint32_t)q) << (bits * e);
      }
      wr[wi] = word;
    }
  }
}

template <typename T>
__global__ void fill_normal_kernel(uint64_t key, size_t n, float mean, float std, T* out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = normal_at(key, i, mean, std);
    if constexpr (sizeof(T) == 4) out[i] = v;
    else out[i] = f2bf(v);
  }
}

__global__ void rms_norm_kernel(const bf16* x, const bf16* w, bf16* out, int dims, float eps, int groups) {
  __shared__ float red[32];
  const bf16* xr = x + (size_t)blockIdx.x * dims;
  bf16* orow = out + (size_t)blockIdx.x * dims;
  const int gd = dims / groups;
  for (int gi = 0; gi < groups; ++gi) {
    float ss = 0.f;
    for (int k = gi * gd + threadIdx.x; k < (gi + 1) * gd; k += blockDim.x) {
      const float v = bf2f(xr[k]);
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)gd), eps)));
    for (int k = gi * gd + threadIdx.x; k < (gi + 1) * gd; k += blockDim.x) {
      const float v = bf2f(xr[k]);
      float o;
      if (groups == 1) o = __fmul_rn(bfround(__fmul_rn(v, inv)), bf2f(w[k]));
      else o = __fmul_rn(__fmul_rn(v, inv), bf2f(w[k]));
      orow[k] = f2bf(o);
    }
  }
}

// One row per CTA, 16-byte chunks held in registers between the sum of
// squares and the scaling (one read of x): RMSNorm without groups, the
// rounding points of rms_norm_kernel.
template <int MAXC>
__global__ void rms_norm_vec_kernel(const bf16* x, const bf16* w, bf16* out, int dims, float eps) {
  __shared__ float red[32];
  const int nch = dims / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)blockIdx.x * dims);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)blockIdx.x * dims);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4 v[MAXC];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    v[i] = c < nch ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(e[j] << 16), hi = __uint_as_float(e[j] & 0xffff0000u);
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
    }
  }
  ss = block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dims), eps)));
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c >= nch) break;
    const uint4 wv = wr[c];
    const uint32_t e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    const uint32_t f[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __fmul_rn(bfround(__fmul_rn(__uint_as_float(e[j] << 16), inv)), __uint_as_float(f[j] << 16));
      const float hi =
          __fmul_rn(bfround(__fmul_rn(__uint_as_float(e[j] & 0xffff0000u), inv)), __uint_as_float(f[j] & 0xffff0000u));
      const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
      o[j] = *reinterpret_cast<const uint32_t*>(&b);
    }
    orow[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void rope_kernel(const bf16* x, bf16* out, int heads, int T, int dims, const float* inv_freq, int offset,
                            const int* offset_dev) {
  const int half = dims / 2;
  const size_t total = (size_t)heads * T * half;
  const int off = offset + (offset_dev ? *offset_dev : 0);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % half);
    const size_t row = i / half;
    const int t = (int)(row % T);
    const bf16* xr = x + row * dims;
    const float th = __fmul_rn((float)(off + t), inv_freq[d]);
    float sn, cs;
    sincosf(th, &sn, &cs);
    const float x1 = bf2f(xr[d]), x2 = bf2f(xr[d + half]);
    out[row * dims + d] = f2bf(__fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn)));
    out[row * dims + d + half] = f2bf(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs)));
  }
}

__global__ void inv_freq_kernel(float* inv, int dims, float theta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < dims / 2) inv[i] = (float)pow((double)theta, -2.0 * (double)i / (double)dims);
}

__global__ void silu_kernel(const bf16* x, bf16* out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = bf2f(x[i]);
    out[i] = f2bf(__fmul_rn(v, bfround(sigmoid_f(v))));
  }
}

__global__ void binop_kernel(const bf16* a, const bf16* b, bf16* out, size_t n, int op) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float x = bf2f(a[i]), y = bf2f(b[i]);
    out[i] = f2bf(op == 0 ? __fmul_rn(x, y) : __fadd_rn(x, y));
  }
}

__global__ void argmax_kernel(const bf16* x, int n, int* out) {
  const bf16* xr = x + (size_t)blockIdx.x * n;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf2f(xr[i]);
    if (v == v && (v > bv || (v == bv && i < bi))) {
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
  __shared__ float wv[32];
  __shared__ int wi[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    wv[warp] = bv;
    wi[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (wv[w] > bv || (wv[w] == bv && wi[w] < bi)) {
        bv = wv[w];
        bi = wi[w];
      }
    out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

__global__ void softmax_kernel(const bf16* x, bf16* out, int n) {
  __shared__ float red[32];
  const bf16* xr = x + (size_t)blockIdx.x * n;
  bf16* orow = out + (size_t)blockIdx.x * n;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, bf2f(xr[i]));
  m = warp_max(m);
  __shared__ float wm[32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  m = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, wm[w]);
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += expf(bf2f(xr[i]) - m);
  s = block_sum(s, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = f2bf(__fdiv_rn(expf(bf2f(xr[i]) - m), s));
}

__global__ void embed_kernel(const uint32_t* w, const bf16* s, const bf16* b, const int* ids, int hidden, int gs,
                             int bits, int vocab, bf16* out, int* status) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report_status(status, kDevBadToken);
    id = 0;
  }
  const int per = 32 / bits, ng = hidden / gs;
  for (int k = threadIdx.x; k < hidden; k += blockDim.x) {
    const uint32_t word = w[(size_t)id * (hidden / per) + k / per];
    const uint32_t q = (word >> (bits * (k % per))) & ((1u << bits) - 1u);
    out[(size_t)t * hidden + k] = dequant1(q, s[(size_t)id * ng + k / gs], b[(size_t)id * ng + k / gs]);
  }
}

// One warp per (token, head): heads [0, nq) are q, [nq, nq+nkv) are k (normed,
// roped, written to the cache), [nq+nkv, nq+2nkv) are v (copied to the cache).
// Lane l holds elements 4l..4l+3 (one 8-byte load and store); the RoPE
// angles come from the (cos, sin) table when given (the same sincosf values).
__global__ void prefill_qkv_kernel(const PrefillQkvArgs a) {
  const int lane = threadIdx.x & 31;
  const int items_per_tok = a.nq + 2 * a.nkv;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= a.T * items_per_tok) return;
  const int t = item / items_per_tok, h = item % items_per_tok;
  constexpr int hd = 128;
  const bf16* src = a.qkv + (size_t)t * items_per_tok * hd + (size_t)h * hd;
  const int pos = a.offset + t;
  const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
  if (h >= a.nq + a.nkv) {
    const int kvh = h - a.nq - a.nkv;
    *reinterpret_cast<uint2*>(a.vc + ((size_t)kvh * a.cap + pos) * hd + lane * 4) = raw;
    return;
  }
  const bool is_k = h >= a.nq;
  const bf16* nw = is_k ? a.k_norm : a.q_norm;
  float v[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), __uint_as_float(raw.y << 16),
                __uint_as_float(raw.y & 0xffff0000u)};
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = fmaf(v[e], v[e], ss);
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), a.eps)));
  float nv[4], pv[4];
  if (nw) {
    const uint2 wr = *reinterpret_cast<const uint2*>(nw + lane * 4);
    const float wv[4] = {__uint_as_float(wr.x << 16), __uint_as_float(wr.x & 0xffff0000u),
                         __uint_as_float(wr.y << 16), __uint_as_float(wr.y & 0xffff0000u)};
#pragma unroll
    for (int e = 0; e < 4; ++e) nv[e] = bfround(__fmul_rn(bfround(__fmul_rn(v[e], inv)), wv[e]));
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) nv[e] = v[e];
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) pv[e] = __shfl_xor_sync(0xffffffffu, nv[e], 16);
  const float fp = (float)pos;
  bf16* dst = is_k ? a.kc + ((size_t)(h - a.nq) * a.cap + pos) * hd : a.q_out + ((size_t)h * a.T + t) * hd;
  float o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane * 4 + e;
    const int i = d & (hd / 2 - 1);
    float sn, cs;
    if (a.rope_cs) {
      const float2 c2 = a.rope_cs[(size_t)pos * (hd / 2) + i];
      cs = c2.x;
      sn = c2.y;
    } else {
      sincosf(__fmul_rn(fp, a.inv_freq[i]), &sn, &cs);
    }
    if (d < hd / 2) o[e] = __fsub_rn(__fmul_rn(nv[e], cs), __fmul_rn(pv[e], sn));
    else o[e] = __fadd_rn(__fmul_rn(pv[e], sn), __fmul_rn(nv[e], cs));
  }
  uint2 out;
  out.x = (uint32_t)f2bits(o[0]) | ((uint32_t)f2bits(o[1]) << 16);
  out.y = (uint32_t)f2bits(o[2]) | ((uint32_t)f2bits(o[3]) << 16);
  *reinterpret_cast<uint2*>(dst + lane * 4) = out;
}

__global__ void slice_update_kernel(bf16* cache, const bf16* upd, int nkv, int cap, int D, int offset,
                                    const int* offset_dev, int T) {
  const int off = offset + (offset_dev ? *offset_dev : 0);
  const size_t total = (size_t)nkv * T * D;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int t = (int)((i / D) % T);
    const int h = (int)(i / ((size_t)D * T));
    if (off + t < cap) cache[((size_t)h * cap + off + t) * D + d] = upd[i];
  }
}

__global__ void moe_route_kernel(const bf16* logits, int E, int k, int normalize, int e_base, int e_local, int* idx,
                                 float* w, int* n) {
  __shared__ float pr[1024];
  __shared__ float red[32];
  pdl_trigger();
  pdl_wait();
  // one token per CTA: row blockIdx.x of logits [T][E], idx / w [T][k], n [T]
  logits += (size_t)blockIdx.x * E;
  idx += (size_t)blockIdx.x * k;
  w += (size_t)blockIdx.x * k;
  n += blockIdx.x;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < E; i += blockDim.x) m = fmaxf(m, bf2f(logits[i]));
  m = warp_max(m);
  __shared__ float wm[32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  m = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, wm[i]);
  float s = 0.f;
  for (int i = threadIdx.x; i < E; i += blockDim.x) s += expf(bf2f(logits[i]) - m);
  s = block_sum(s, red);
  for (int i = threadIdx.x; i < E; i += blockDim.x) pr[i] = bfround(__fdiv_rn(expf(bf2f(logits[i]) - m), s));
  __syncthreads();
  int sel[64];
  float sw[64];
  if (threadIdx.x < 32) {
    // k rounds of an argmax over the probabilities by one warp: the largest
    // value, the lowest index among equal ones (a NaN is never taken; with
    // nothing to take, index 0), then that entry is removed -- the order a
    // sequential scan for the first maximum gives
    const int lane = threadIdx.x;
    for (int r = 0; r < k; ++r) {
      float bv = -INFINITY;
      int bi = E;  // none yet
      for (int i = lane; i < E; i += 32) {
        const float v = pr[i];
        if (v > bv || (bi == E && v == bv)) {
          bv = v;
          bi = i;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi >= E) bi = 0;
      sel[r] = bi;
      sw[r] = pr[bi];
      __syncwarp();
      if (lane == 0) pr[bi] = -INFINITY;
      __syncwarp();
    }
  }
  if (threadIdx.x == 0) {
    if (normalize) {
      float sum = 0.f;
      for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, sw[r]);
      if (sum > 1e-20f)
        for (int r = 0; r < k; ++r) sw[r] = __fdiv_rn(sw[r], sum);
    }
    int j = 0;
    for (int r = 0; r < k; ++r) {
      if (sel[r] >= e_base && sel[r] < e_base + e_local) {
        idx[j] = sel[r] - e_base;
        w[j] = sw[r];
        ++j;
      }
    }
    *n = j;
  }
}

// The routing for up to 32 * EPL experts by one warp (route_warp).
template <int EPL>
__global__ void moe_route_warp_kernel(const bf16* logits, int E, int k, int normalize, int e_base, int e_local,
                                      int* idx, float* w, int* n) {
  pdl_trigger();
  pdl_wait();
  route_warp<EPL>(logits + (size_t)blockIdx.x * E, false, E, k, normalize, e_base, e_local,
                  idx + (size_t)blockIdx.x * k, w + (size_t)blockIdx.x * k, n + blockIdx.x);
}

// Batched MoE prefill, grouping: the (token, slot) pairs of each local
// expert get consecutive positions, experts in order and, inside an expert,
// tokens in order (deterministic); perm [T][k] holds each pair's position,
// src [P] its token; tile list entries (expert, first position, end
// position) cover every expert's positions in runs of `tile` rows.  One
// thread per local expert (E_l <= 1024), one CTA.
__global__ void moe_group_kernel(const int* idx, const int* n, int T, int k, int E_l, int tile, int* perm, int* src,
                                 int4* tiles, int* n_tiles, int* n_pairs) {
  __shared__ int cnt[1024];
  __shared__ int off[1024];
  __shared__ int toff[1024];
  const int e = threadIdx.x;
  int c = 0;
  if (e < E_l)
    for (int t = 0; t < T; ++t) {
      const int nt = n[t];
      for (int j = 0; j < nt; ++j) c += idx[t * k + j] == e;
    }
  if (e < 1024) cnt[e] = e < E_l ? c : 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0, to = 0;
    for (int i = 0; i < E_l; ++i) {
      off[i] = o;
      toff[i] = to;
      o += cnt[i];
      to += (cnt[i] + tile - 1) / tile;
    }
    *n_tiles = to;
    *n_pairs = o;
  }
  __syncthreads();
  if (e < E_l) {
    int pos = off[e];
    for (int t = 0; t < T; ++t) {
      const int nt = n[t];
      for (int j = 0; j < nt; ++j)
        if (idx[t * k + j] == e) {
          perm[t * k + j] = pos;
          src[pos] = t;
          ++pos;
        }
    }
    const int end = off[e] + cnt[e];
    for (int i = 0, p0 = off[e]; p0 < end; ++i, p0 += tile) tiles[toff[e] + i] = make_int4(e, p0, end, 0);
  }
}

// xs[p] = x[src[p]] for the *P grouped positions (rows of H bf16; the grid
// covers Pmax positions).
__global__ void moe_gather_kernel(const bf16* x, const int* src, const int* P_dev, int H, bf16* xs) {
  const int per = H / 8;
  const int P = *P_dev;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)P * per; i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i / per), c = (int)(i % per);
    reinterpret_cast<uint4*>(xs + (size_t)p * H)[c] = reinterpret_cast<const uint4*>(x + (size_t)src[p] * H)[c];
  }
}

// Per token: acc = sum over its slots in order of w * ys[perm]; then
// x = bf16(x + acc) (out == nullptr), or out = acc as an fp32 partial (EP).
__global__ void moe_combine_batch_kernel(bf16* x, const bf16* ys, const float* w, const int* n, const int* perm, int T,
                                         int k, int H, float* out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)T * H; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / H), c = (int)(i % H);
    const int nt = n[t];
    float acc = 0.f;
    for (int j = 0; j < nt; ++j)
      acc = __fadd_rn(acc, __fmul_rn(bf2f(ys[(size_t)perm[t * k + j] * H + c]), w[t * k + j]));
    if (out) out[i] = acc;
    else x[i] = f2bf(__fadd_rn(bf2f(x[i]), acc));
  }
}

__global__ void moe_combine_kernel(const bf16* y, const float* w, const int* n, int H, float* out) {
  pdl_trigger();
  pdl_wait();
  const int ns = *n;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < ns; ++s) acc = __fadd_rn(acc, __fmul_rn(bf2f(y[(size_t)s * H + k]), w[s]));
    out[k] = acc;
  }
}

// The expert-parallel combine through NVLink peer memory: this rank's
// weighted sum of its expert slots (moe_combine_kernel's arithmetic) stored
// into slot [rank] of every rank's region and published; the consumer's
// AddNorm prologue sums the ranks' slots in rank order.
struct BarAll {
  static __device__ __forceinline__ void sync() { __syncthreads(); }
};

__global__ void moe_combine_peer_kernel(const bf16* y, const float* w, const int* n, int H, const PeerX* peer) {
  pdl_trigger();
  pdl_wait();
  const PeerX& P = *peer;
  const unsigned e = *P.epoch + 1u;
  const int ns = *n;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < ns; ++s) acc = __fadd_rn(acc, __fmul_rn(bf2f(y[(size_t)s * H + k]), w[s]));
    for (int d = 0; d < P.world; ++d) peer_slot(P, d, e, P.rank)[k] = acc;
  }
  __shared__ unsigned last;
  peer_publish<BarAll>(P, threadIdx.x, &last);
}

__global__ void add_f32_kernel(bf16* x, const float* add, size_t n, int round) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float a = round ? bfround(add[i]) : add[i];
    x[i] = f2bf(__fadd_rn(bf2f(x[i]), a));
  }
}

__global__ void moe_residual_kernel(bf16* x, const bf16* y, const float* w, const int* n, int H) {
  const int ns = *n;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < ns; ++s) acc = __fadd_rn(acc, __fmul_rn(bf2f(y[(size_t)s * H + k]), w[s]));
    x[k] = f2bf(__fadd_rn(bf2f(x[k]), acc));
  }
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t k_moe_route(const bf16* logits, int E, int k, int normalize, int e_base, int e_local, int* idx,
                        float* w, int* n, cudaStream_t st, bool pdl) {
  if (E <= 0 || E > 1024 || k <= 0 || k > 64 || k > E) return cudaErrorInvalidValue;
  void* args[] = {(void*)&logits, (void*)&E, (void*)&k, (void*)&normalize, (void*)&e_base, (void*)&e_local,
                  (void*)&idx, (void*)&w, (void*)&n};
  if (E <= 128) return launch_pdl((const void*)moe_route_warp_kernel<4>, dim3(1), dim3(32), args, st, pdl);
  if (E <= 256) return launch_pdl((const void*)moe_route_warp_kernel<8>, dim3(1), dim3(32), args, st, pdl);
  return launch_pdl((const void*)moe_route_kernel, dim3(1), dim3(256), args, st, pdl);
}

cudaError_t k_moe_route_batch(const bf16* logits, int T, int E, int k, int normalize, int e_base, int e_local,
                              int* idx, float* w, int* n, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (E <= 0 || E > 1024 || k <= 0 || k > 64 || k > E) return cudaErrorInvalidValue;
  if (E <= 128)
    moe_route_warp_kernel<4><<<T, 32, 0, st>>>(logits, E, k, normalize, e_base, e_local, idx, w, n);
  else if (E <= 256)
    moe_route_warp_kernel<8><<<T, 32, 0, st>>>(logits, E, k, normalize, e_base, e_local, idx, w, n);
  else
    moe_route_kernel<<<T, 256, 0, st>>>(logits, E, k, normalize, e_base, e_local, idx, w, n);
  return cudaGetLastError();
}

cudaError_t k_moe_group(const int* idx, const int* n, int T, int k, int E_l, int tile, int* perm, int* src,
                        int4* tiles, int* n_tiles, int* n_pairs, cudaStream_t st) {
  if (E_l <= 0 || E_l > 1024 || T <= 0) return cudaErrorInvalidValue;
  moe_group_kernel<<<1, (E_l + 31) / 32 * 32, 0, st>>>(idx, n, T, k, E_l, tile, perm, src, tiles, n_tiles, n_pairs);
  return cudaGetLastError();
}

cudaError_t k_moe_gather(const bf16* x, const int* src, const int* P, int Pmax, int H, bf16* xs, cudaStream_t st) {
  if (Pmax <= 0) return cudaSuccess;
  if (H % 8 != 0) return cudaErrorInvalidValue;
  moe_gather_kernel<<<blocks_for((size_t)Pmax * (H / 8), 256), 256, 0, st>>>(x, src, P, H, xs);
  return cudaGetLastError();
}

cudaError_t k_moe_combine_batch(bf16* x, const bf16* ys, const float* w, const int* n, const int* perm, int T, int k,
                                int H, float* out, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  moe_combine_batch_kernel<<<blocks_for((size_t)T * H, 256), 256, 0, st>>>(x, ys, w, n, perm, T, k, H, out);
  return cudaGetLastError();
}

cudaError_t k_add_f32(bf16* x, const float* add, size_t n, int round, cudaStream_t st) {
  if (!n) return cudaSuccess;
  add_f32_kernel<<<blocks_for(n, 256), 256, 0, st>>>(x, add, n, round);
  return cudaGetLastError();
}

cudaError_t k_moe_residual(bf16* x, const bf16* y, const float* w, const int* n, int H, cudaStream_t st) {
  moe_residual_kernel<<<(H + 255) / 256, 256, 0, st>>>(x, y, w, n, H);
  return cudaGetLastError();
}

cudaError_t k_moe_combine(const bf16* y, const float* w, const int* n, int H, float* out, cudaStream_t st, bool pdl) {
  void* args[] = {(void*)&y, (void*)&w, (void*)&n, (void*)&H, (void*)&out};
  return launch_pdl((const void*)moe_combine_kernel, dim3((H + 255) / 256), dim3(256), args, st, pdl);
}

cudaError_t k_moe_combine_peer(const bf16* y, const float* w, const int* n, int H, const PeerX* peer, cudaStream_t st,
                               bool pdl) {
  void* args[] = {(void*)&y, (void*)&w, (void*)&n, (void*)&H, (void*)&peer};
  return launch_pdl((const void*)moe_combine_peer_kernel, dim3((H + 255) / 256), dim3(256), args, st, pdl);
}

cudaError_t k_dequantize(const uint32_t* w, const bf16* s, const bf16* b, bf16* out, int N, int K, int gs, int bits,
                         cudaStream_t st) {
  const size_t words = (size_t)N * K / (32 / bits);
  const int blocks = (int)std::min<size_t>((words + 255) / 256, 148 * 64);
  if (bits == 4) dequant_kernel<4><<<blocks, 256, 0, st>>>(w, s, b, out, N, K, gs);
  else dequant_kernel<8><<<blocks, 256, 0, st>>>(w, s, b, out, N, K, gs);
  return cudaGetLastError();
}

cudaError_t k_quantize(const float* src_f32, const bf16* src_bf16, uint32_t* w, bf16* s, bf16* b, int N, int K,
                       int gs, int bits, cudaStream_t st) {
  quant_kernel<false><<<blocks_for((size_t)N * (K / gs), 128), 128, 0, st>>>(src_f32, src_bf16, 0, 0.f, w, s, b, N,
                                                                             K, gs, bits, 0, 0, K);
  return cudaGetLastError();
}

cudaError_t k_fill_normal_f32(uint64_t seed, uint64_t stream, size_t n, float mean, float std, float* out,
                              cudaStream_t st) {
  fill_normal_kernel<float><<<blocks_for(n, 256), 256, 0, st>>>(stream_key(seed, stream), n, mean, std, out);
  return cudaGetLastError();
}

cudaError_t k_fill_normal_bf16(uint64_t seed, uint64_t stream, size_t n, float mean, float std, bf16* out,
                               cudaStream_t st) {
  fill_normal_kernel<bf16><<<blocks_for(n, 256), 256, 0, st>>>(stream_key(seed, stream), n, mean, std, out);
  return cudaGetLastError();
}

cudaError_t k_fill_quantized(uint64_t seed, uint64_t stream, int N, int K, int gs, int bits, float std, uint32_t* w,
                             bf16* s, bf16* b, cudaStream_t st) {
  return k_fill_quantized_shard(seed, stream, N, K, K, 0, 0, gs, bits, std, w, s, b, K, st);
}

cudaError_t k_fill_quantized_shard(uint64_t seed, uint64_t stream, int n_rows, int n_cols, int K_full, size_t row0,
                                   int col0, int gs, int bits, float std, uint32_t* w, bf16* s, bf16* b, int ldK,
                                   cudaStream_t st) {
  if (ldK != n_cols) return cudaErrorInvalidValue;
  if (n_rows <= 0) return cudaSuccess;
  quant_kernel<true><<<blocks_for((size_t)n_rows * (n_cols / gs), 128), 128, 0, st>>>(
      nullptr, nullptr, stream_key(seed, stream), std, w, s, b, n_rows, n_cols, gs, bits, row0, col0, K_full);
  return cudaGetLastError();
}

cudaError_t k_rms_norm(const bf16* x, const bf16* w, bf16* out, int rows, int dims, float eps, int groups,
                       cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                         reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if (groups == 1 && dims % 8 == 0 && dims <= 8192 && aligned) {
    const int nch = dims / 8;
    const int thr = std::min(256, (nch + 31) / 32 * 32);
    if ((nch + thr - 1) / thr <= 1) rms_norm_vec_kernel<1><<<rows, thr, 0, st>>>(x, w, out, dims, eps);
    else if ((nch + thr - 1) / thr <= 2) rms_norm_vec_kernel<2><<<rows, thr, 0, st>>>(x, w, out, dims, eps);
    else rms_norm_vec_kernel<4><<<rows, thr, 0, st>>>(x, w, out, dims, eps);
    return cudaGetLastError();
  }
  rms_norm_kernel<<<rows, 256, 0, st>>>(x, w, out, dims, eps, groups);
  return cudaGetLastError();
}

cudaError_t k_rope(const bf16* x, bf16* out, int heads, int T, int dims, const float* inv_freq, int offset,
                   const int* offset_dev, cudaStream_t st) {
  const size_t n = (size_t)heads * T * (dims / 2);
  if (!n) return cudaSuccess;
  rope_kernel<<<blocks_for(n, 256), 256, 0, st>>>(x, out, heads, T, dims, inv_freq, offset, offset_dev);
  return cudaGetLastError();
}

cudaError_t k_rope_inv_freq(float* inv_freq, int dims, float theta, cudaStream_t st) {
  inv_freq_kernel<<<(dims / 2 + 127) / 128, 128, 0, st>>>(inv_freq, dims, theta);
  return cudaGetLastError();
}

cudaError_t k_silu(const bf16* x, bf16* out, size_t n, cudaStream_t st) {
  if (!n) return cudaSuccess;
  silu_kernel<<<blocks_for(n, 256), 256, 0, st>>>(x, out, n);
  return cudaGetLastError();
}

cudaError_t k_multiply(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t st) {
  if (!n) return cudaSuccess;
  binop_kernel<<<blocks_for(n, 256), 256, 0, st>>>(a, b, out, n, 0);
  return cudaGetLastError();
}

cudaError_t k_add(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t st) {
  if (!n) return cudaSuccess;
  binop_kernel<<<blocks_for(n, 256), 256, 0, st>>>(a, b, out, n, 1);
  return cudaGetLastError();
}

cudaError_t k_argmax(const bf16* x, int rows, int n, int* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  argmax_kernel<<<rows, 1024, 0, st>>>(x, n, out);
  return cudaGetLastError();
}

cudaError_t k_softmax(const bf16* x, bf16* out, int rows, int n, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  softmax_kernel<<<rows, 256, 0, st>>>(x, out, n);
  return cudaGetLastError();
}

cudaError_t k_embed(const uint32_t* w, const bf16* s, const bf16* b, const int* ids, int T, int hidden, int gs,
                    int bits, int vocab, bf16* out, int* status, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  embed_kernel<<<T, 256, 0, st>>>(w, s, b, ids, hidden, gs, bits, vocab, out, status);
  return cudaGetLastError();
}

cudaError_t k_prefill_qkv(const PrefillQkvArgs& a, cudaStream_t st) {
  if (a.hd != 128) return cudaErrorInvalidValue;
  const int items = a.T * (a.nq + 2 * a.nkv);
  if (!items) return cudaSuccess;
  prefill_qkv_kernel<<<(items + 7) / 8, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t k_slice_update(bf16* cache, const bf16* upd, int nkv, int cap, int D, int offset, const int* offset_dev,
                           int T, cudaStream_t st) {
  const size_t n = (size_t)nkv * T * D;
  if (!n) return cudaSuccess;
  slice_update_kernel<<<blocks_for(n, 256), 256, 0, st>>>(cache, upd, nkv, cap, D, offset, offset_dev, T);
  return cudaGetLastError();
}

}  // namespace emx
