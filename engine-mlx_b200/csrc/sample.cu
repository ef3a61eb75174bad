// sample.cu — sample_token (crates/serve/src/sampler.rs:101-202) on the device.
//
// One CTA of 1024 threads per draw; the logits (bf16, in L2 right after the
// lm_head) are read a few times and the probabilities kept in a scratch
// vector.  The steps and their order are the reference's:
//   1. scaled = logit / max(temperature, 1e-6)                (fp32 division)
//   2. top-k: values below the k-th largest become -inf       (radix select
//      on order-preserving 32-bit keys, exact: the same threshold value)
//   3. softmax over the finite values                         (exp(x - max) / sum)
//   4. top-p: the largest probabilities in stable descending order, until
//      their sum reaches top_p                                (radix select on
//      the probability bits with exact 2^-48 fixed-point bin sums; among
//      probabilities equal to the threshold the lowest indices are taken,
//      as the stable sort would)
//   5. renormalise the kept probabilities
//   6. r = SimpleRng::next_f32 (xorshift64*, bit-exact); the token is the
//      first index whose running sum (index order) exceeds r, else the last
//      kept index.
// Where the reference sums sequentially in fp32 (the softmax denominator,
// the top-p running sum, the renormalisation, the running sum of step 6)
// this sums each thread's contiguous slice in order and then the slices in
// order, so a result can differ from the host's only when r, or the top-p
// running sum, falls within a few ulps of a boundary.  With top_p >= 1 every
// finite probability is kept (the host's fp32 running sum can reach 1.0 a
// few elements early and drop a tail of < 1e-6 total mass).
#include "sample.cuh"

#include "ctx.cuh"
#include "emx.h"

namespace emx {

namespace {

constexpr int kT = 1024;
constexpr int kW = kT / 32;

// Order-preserving key of a float (-0 folded onto +0, as float compares).
__device__ __forceinline__ uint32_t fkey(float f) {
  uint32_t b = __float_as_uint(f);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long fix48(float p) {
  return __float2ull_rn(p * 281474976710656.0f);  // p * 2^48 (exact scaling)
}

struct Sm {
  unsigned cnt[256];
  unsigned long long sum[256];
  float f[kW];
  int i[kW];
  unsigned u[kT];
  float s[kT];
  int sel;
  unsigned rem;
  unsigned long long above;
  int tok;
  float mx, tot;
};

__device__ __forceinline__ float block_max(float v, Sm& S) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) S.f[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = S.f[threadIdx.x];
    w = warp_max(w);
    if (threadIdx.x == 0) S.mx = w;
  }
  __syncthreads();
  return S.mx;
}

// The largest index where `on` holds (-1 if none).
__device__ __forceinline__ int block_max_index(int idx, Sm& S) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) idx = max(idx, __shfl_xor_sync(0xffffffffu, idx, o));
  if ((threadIdx.x & 31) == 0) S.i[threadIdx.x >> 5] = idx;
  __syncthreads();
  if (threadIdx.x < 32) {
    int w = S.i[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) S.tok = w;
  }
  __syncthreads();
  return S.tok;
}

// Sum of per-thread values in thread order (one thread adds them up):
// thread t's value is the sum of its contiguous slice taken in index order.
__device__ __forceinline__ float ordered_total(float v, Sm& S) {
  S.s[threadIdx.x] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < kT; ++k) t += S.s[k];
    S.tot = t;
  }
  __syncthreads();
  return S.tot;
}

// One 8-bit radix step over keys: histogram of the keys matching `prefix`
// under `mask` (count, and optionally the fixed-point probability sum).
template <bool SUM, class Key>
__device__ __forceinline__ void radix_hist(Sm& S, int n, uint32_t prefix, uint32_t mask, int shift, Key key) {
  for (int b = threadIdx.x; b < 256; b += kT) {
    S.cnt[b] = 0u;
    S.sum[b] = 0ull;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += kT) {
    float p;
    const uint32_t k = key(i, p);
    if ((k & mask) == prefix) {
      const int b = (int)((k >> shift) & 255u);
      atomicAdd(&S.cnt[b], 1u);
      if (SUM) atomicAdd(&S.sum[b], fix48(p));
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kT, 1) sample_kernel(const SampleArgs a) {
  __shared__ Sm S;
  const int n = a.n, tid = threadIdx.x;
  const float temp = fmaxf(a.temperature, 1e-6f);
  const int chunk = (n + kT - 1) / kT;
  const int c0 = min(n, tid * chunk), c1 = min(n, c0 + chunk);
  auto scaled = [&](int i) { return __fdiv_rn(bf2f(a.logits[i]), temp); };

  // ---- 2. top-k threshold: the k-th largest scaled value
  const bool topk = a.top_k > 0 && a.top_k < n;
  uint32_t kth = 0u;
  if (topk) {
    uint32_t prefix = 0u, mask = 0u;
    unsigned rem = (unsigned)a.top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      radix_hist<false>(S, n, prefix, mask, shift, [&](int i, float& p) {
        p = 0.f;
        return fkey(scaled(i));
      });
      if (tid == 0) {
        unsigned r = rem;
        int sel = 0;
        for (int b = 255; b >= 0; --b) {
          if (S.cnt[b] >= r) {
            sel = b;
            break;
          }
          r -= S.cnt[b];
        }
        S.sel = sel;
        S.rem = r;
      }
      __syncthreads();
      prefix |= (uint32_t)S.sel << shift;
      mask |= 255u << shift;
      rem = S.rem;
      __syncthreads();
    }
    kth = prefix;
  }
  auto filtered = [&](int i) {
    const float v = scaled(i);
    return (topk && fkey(v) < kth) ? -INFINITY : v;
  };

  // ---- 3. softmax
  float lm = -INFINITY;
  for (int i = tid; i < n; i += kT) {
    const float v = filtered(i);
    if (isfinite(v)) lm = fmaxf(lm, v);
  }
  const float mx = block_max(lm, S);
  float ls = 0.f;
  for (int i = c0; i < c1; ++i) {
    const float v = filtered(i);
    const float e = isfinite(v) ? expf(v - mx) : 0.f;
    a.scratch[i] = e;
    ls += e;
  }
  const float sum = ordered_total(ls, S);
  if (!isfinite(sum) || sum == 0.f) {
    // the host falls back to the last index of the maximum logit
    float lv = -INFINITY;
    for (int i = tid; i < n; i += kT) lv = fmaxf(lv, bf2f(a.logits[i]));
    const float m2 = block_max(lv, S);
    int li = -1;
    for (int i = tid; i < n; i += kT)
      if (bf2f(a.logits[i]) == m2) li = max(li, i);
    const int t = block_max_index(li, S);
    if (tid == 0) {
      *a.tok_out = t < 0 ? 0 : t;
      if (a.hist && *a.hist_n < a.hist_cap) a.hist[(*a.hist_n)++] = t < 0 ? 0 : t;
    }
    return;
  }
  for (int i = c0; i < c1; ++i) a.scratch[i] = __fdiv_rn(a.scratch[i], sum);
  __syncthreads();

  // ---- 4. top-p: the threshold probability and how many of its ties to take
  bool all = a.top_p >= 1.0f;
  uint32_t pth = 0u;
  unsigned take = 0u;
  if (!all) {
    const unsigned long long target = (unsigned long long)((double)a.top_p * 281474976710656.0);
    uint32_t prefix = 0u, mask = 0u;
    unsigned long long above = 0ull;
    for (int shift = 24; shift >= 0 && !all; shift -= 8) {
      radix_hist<true>(S, n, prefix, mask, shift, [&](int i, float& p) {
        p = a.scratch[i];
        return __float_as_uint(p);
      });
      if (tid == 0) {
        unsigned long long ab = above;
        int sel = -1;
        for (int b = 255; b >= 0; --b) {
          if (S.cnt[b] && ab + S.sum[b] >= target) {
            sel = b;
            break;
          }
          ab += S.sum[b];
        }
        S.sel = sel;
        S.above = ab;
      }
      __syncthreads();
      if (S.sel < 0) {
        all = true;  // the whole mass stays below top_p: everything is kept
      } else {
        prefix |= (uint32_t)S.sel << shift;
        mask |= 255u << shift;
        above = S.above;
      }
      __syncthreads();
    }
    if (!all) {
      pth = prefix;
      const unsigned long long unit = fix48(__uint_as_float(pth));
      // ties at the threshold: the lowest indices first until the target
      // (at least one: the host adds an entry before it tests the sum)
      take = unit ? max(1u, (unsigned)((target - above + unit - 1) / unit)) : 0xffffffffu;
    }
  }
  auto keep_base = [&](float p) { return all || __float_as_uint(p) > pth; };
  // rank of each tie in index order: per-thread counts, exclusive scan
  unsigned ties = 0u;
  if (!all)
    for (int i = c0; i < c1; ++i) ties += __float_as_uint(a.scratch[i]) == pth ? 1u : 0u;
  S.u[tid] = ties;
  __syncthreads();
  if (tid == 0) {
    unsigned run = 0u;
    for (int k = 0; k < kT; ++k) {
      const unsigned v = S.u[k];
      S.u[k] = run;
      run += v;
    }
  }
  __syncthreads();
  const unsigned tie0 = S.u[tid];
  auto kept = [&](int i, unsigned& tie_rank) {
    const float p = a.scratch[i];
    if (keep_base(p)) return true;
    if (__float_as_uint(p) == pth) return tie_rank++ < take;
    return false;
  };

  // ---- 5. renormalise over the kept entries
  float lk = 0.f;
  int last_kept = -1;
  {
    unsigned tr = tie0;
    for (int i = c0; i < c1; ++i)
      if (kept(i, tr)) {
        lk += a.scratch[i];
        last_kept = i;
      }
  }
  const float fsum = ordered_total(lk, S);
  const int lastk = block_max_index(last_kept, S);
  {
    unsigned tr = tie0;
    for (int i = c0; i < c1; ++i) {
      const float p = a.scratch[i];
      const bool k = kept(i, tr);
      // the host keeps the unfiltered probabilities when the kept sum is 0
      a.scratch[i] = fsum > 0.f ? (k ? __fdiv_rn(p, fsum) : 0.f) : p;
    }
  }
  __syncthreads();

  // ---- 6. the draw
  if (tid == 0) {
    unsigned long long x = *a.rng;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *a.rng = x;
    const unsigned long long o = x * 0x2545F4914F6CDD1Dull;
    S.mx = __double2float_rn((double)(o >> 11) / 9007199254740992.0);
    S.tok = 0x7fffffff;
  }
  float lw = 0.f;
  for (int i = c0; i < c1; ++i) lw += a.scratch[i];
  S.s[tid] = lw;
  __syncthreads();
  const float r = S.mx;
  if (tid == 0) {
    float run = 0.f;
    for (int k = 0; k < kT; ++k) {
      const float v = S.s[k];
      S.s[k] = run;
      run += v;
    }
  }
  __syncthreads();
  {
    float cs = S.s[tid];
    for (int i = c0; i < c1; ++i) {
      cs += a.scratch[i];
      if (r < cs) {
        atomicMin(&S.tok, i);
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int t = S.tok;
    if (t == 0x7fffffff) t = lastk < 0 ? 0 : lastk;
    *a.tok_out = t;
    if (a.hist && *a.hist_n < a.hist_cap) a.hist[(*a.hist_n)++] = t;
  }
}

}  // namespace

cudaError_t sample_launch(const SampleArgs& a, cudaStream_t st) {
  if (!a.logits || !a.rng || !a.scratch || !a.tok_out || a.n <= 0) return cudaErrorInvalidValue;
  sample_kernel<<<1, kT, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace emx

using namespace emx;

extern "C" int emx_sample_token(emx_ctx* c, const void* logits, int n, float temperature, float top_p, int top_k,
                                uint64_t* rng_state, int32_t* token) {
  if (!c || !logits || !rng_state || !token) return fail(EMX_ERR_INVALID, "emx_sample_token: null argument");
  if (n <= 0 || !(temperature >= 1e-6f) || !(top_p >= 0.f && top_p <= 1.f) || top_k < 0)
    return fail(EMX_ERR_INVALID, "emx_sample_token: n %d / temperature %g / top_p %g / top_k %d out of range", n,
                temperature, top_p, top_k);
  void* sc = nullptr;
  int rc = ctx_scratch(c, sizeof(float) * (size_t)n, &sc);
  if (rc) return rc;
  SampleArgs a = {};
  a.logits = static_cast<const bf16*>(logits);
  a.n = n;
  a.temperature = temperature;
  a.top_p = top_p;
  a.top_k = top_k;
  a.rng = reinterpret_cast<unsigned long long*>(rng_state);
  a.scratch = static_cast<float*>(sc);
  a.tok_out = token;
  EMX_CHECK_CUDA(sample_launch(a, c->stream), "emx_sample_token");
  return EMX_OK;
}
