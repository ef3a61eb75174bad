/*
 * emx_oracle.c — CPU restatement of engine-mlx's quantized Qwen3 forward pass.
 *
 * TEST INFRASTRUCTURE ONLY (see emx_oracle.h).  It is the checker for the
 * libemx CUDA kernels and the timed CPU baseline ("port" kind); the product
 * never links or loads it.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).  Floating
 * point contraction is off so that every a*b+c below rounds twice, exactly as
 * the device kernels' explicit __fmul_rn/__fadd_rn sequences do where the two
 * sides must agree bit-for-bit (generator, quantizer, dequantizer).
 */
#include "emx_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar helpers                                                           */
/* ------------------------------------------------------------------------ */

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void orc_f32_to_bf16_n(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(in[i]);
}

void orc_bf16_to_f32_n(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_bf16_to_f32(in[i]);
}

#define BF(x) orc_bf16_to_f32(x)
#define TOBF(x) orc_f32_to_bf16(x)

/* bf16 nearest to a double: round-to-odd to 24 bits, then RNE to 8 bits
 * (exact because 24 >= 8 + 2). */
uint16_t orc_f64_to_bf16(double d) {
    float f = (float)d;
    if ((double)f != d && f == f) {
        if (fabs((double)f) > fabs(d)) f = nextafterf(f, 0.0f);
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= 1u;
        memcpy(&f, &u, 4);
    }
    return orc_f32_to_bf16(f);
}

/* One dequantized code: the bf16 nearest to the exact s*q + b (the product
 * and sum are exact in double for bf16 s, b and q <= 255). */
static inline uint16_t deq1(uint32_t q, uint16_t s, uint16_t b) {
    return orc_f64_to_bf16((double)BF(s) * (double)q + (double)BF(b));
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* seeded generator                                                         */
/* ------------------------------------------------------------------------ */

uint64_t orc_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

uint64_t orc_name_stream(const char* name) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (const unsigned char* p = (const unsigned char*)name; *p; ++p) {
        h ^= *p;
        h *= 0x100000001b3ull;
    }
    return h;
}

/* 12 uniform 16-bit draws (three 64-bit hashes) summed exactly in integers;
 * centred on their mean 12*32767.5 and scaled by 2^-16 — an Irwin-Hall
 * approximation of N(0,1) whose every step is exact or a single IEEE rounding,
 * so CPU and GPU produce identical bits. */
void orc_fill_normal(uint64_t seed, uint64_t stream, size_t n, float mean, float std, float* out) {
    const uint64_t key = orc_splitmix64(seed ^ orc_splitmix64(stream));
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        uint32_t s = 0;
        for (int j = 0; j < 3; ++j) {
            uint64_t h = orc_splitmix64(key + 3ull * (uint64_t)i + (uint64_t)j);
            s += (uint32_t)(h & 0xffff) + (uint32_t)((h >> 16) & 0xffff) + (uint32_t)((h >> 32) & 0xffff) +
                 (uint32_t)(h >> 48);
        }
        int t = (int)s - 393210;
        float z = (float)t * (1.0f / 65536.0f);
        float y = std * z;
        out[i] = mean + y;
    }
}

/* ------------------------------------------------------------------------ */
/* MLX affine quantization                                                  */
/* ------------------------------------------------------------------------ */

static inline uint32_t qget(const uint32_t* row, int k, int bits) {
    const int per = 32 / bits;
    return (row[k / per] >> (bits * (k % per))) & ((1u << bits) - 1u);
}

void orc_quantize(const float* w, int N, int K, int gs, int bits, uint32_t* wq, uint16_t* scales,
                  uint16_t* biases) {
    const int per = 32 / bits;
    const int ng = K / gs;
    const float maxq = (float)((1 << bits) - 1);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const float* wr = w + (size_t)n * K;
        uint32_t* qr = wq + (size_t)n * (K / per);
        memset(qr, 0, sizeof(uint32_t) * (size_t)(K / per));
        for (int g = 0; g < ng; ++g) {
            float mn = wr[g * gs], mx = wr[g * gs];
            for (int i = 1; i < gs; ++i) {
                float v = wr[g * gs + i];
                mn = v < mn ? v : mn;
                mx = v > mx ? v : mx;
            }
            float scale = (mx - mn) / maxq;
            uint16_t sb = TOBF(scale), bb = TOBF(mn);
            scales[(size_t)n * ng + g] = sb;
            biases[(size_t)n * ng + g] = bb;
            float sf = BF(sb), bf = BF(bb);
            for (int i = 0; i < gs; ++i) {
                int k = g * gs + i;
                float q = 0.0f;
                if (sf > 0.0f) {
                    float d = wr[k] - bf;
                    q = rintf(d / sf);
                    q = q < 0.0f ? 0.0f : (q > maxq ? maxq : q);
                }
                qr[k / per] |= ((uint32_t)q) << (bits * (k % per));
            }
        }
    }
}

/* mlx_dequantize affine -> bf16 (crates/mlx-ffi/src/ops/real/transform.rs:45-60):
 * each element is the bf16 nearest to the exact s*q + b.  (An fp32 evaluation
 * followed by a cast gives the same bits whenever fp32 holds the sum exactly,
 * which is every group whose min and range are within 2^16 of each other.) */
void orc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int N, int K,
                    int gs, int bits, uint16_t* out) {
    const int per = 32 / bits;
    const int ng = K / gs;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const uint32_t* qr = wq + (size_t)n * (K / per);
        for (int k = 0; k < K; ++k)
            out[(size_t)n * K + k] = deq1(qget(qr, k, bits), scales[(size_t)n * ng + k / gs],
                                          biases[(size_t)n * ng + k / gs]);
    }
}

/* mlx_quantized_matmul (crates/mlx-ffi/src/ops/real/transform.rs:77-89),
 * called as qmatmul (crates/ops/src/quant.rs:57-76) for every Qwen3 linear. */
/* Summation order of orc_qmatmul's fp32 reductions: 0 ascending k (the
 * reference's order), 1 descending.  Both are valid fp32 evaluations of the
 * same sums; running a model under each measures the bf16 rounding-noise
 * floor that any re-ordered implementation (a GPU kernel) is held against. */
static int g_sum_reverse = 0;
void orc_set_sum_order(int reverse) { g_sum_reverse = reverse ? 1 : 0; }

void orc_qmatmul(const uint16_t* x, const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                 int M, int N, int K, int gs, int bits, uint16_t* y) {
    const int rev = g_sum_reverse;
    const int per = 32 / bits;
    const int ng = K / gs;
    if (M == 1) {
        float* xf = (float*)malloc(sizeof(float) * (size_t)K);
        float* xs = (float*)malloc(sizeof(float) * (size_t)ng);
        for (int k = 0; k < K; ++k) xf[k] = BF(x[k]);
        for (int g = 0; g < ng; ++g) {
            float s = 0.0f;
            for (int i = 0; i < gs; ++i) s += xf[g * gs + i];
            xs[g] = s;
        }
#pragma omp parallel for schedule(static)
        for (int n = 0; n < N; ++n) {
            const uint32_t* qr = wq + (size_t)n * (K / per);
            float acc = 0.0f;
            for (int gi = 0; gi < ng; ++gi) {
                const int g = rev ? ng - 1 - gi : gi;
                float dot = 0.0f;
                const float* xg = xf + g * gs;
                const uint32_t* qw = qr + (g * gs) / per;
                for (int ii = 0; ii < gs; ++ii) {
                    const int i = rev ? gs - 1 - ii : ii;
                    uint32_t q = (qw[i / per] >> (bits * (i % per))) & ((1u << bits) - 1u);
                    dot += xg[i] * (float)q;
                }
                float sf = BF(scales[(size_t)n * ng + g]);
                float bf = BF(biases[(size_t)n * ng + g]);
                acc += sf * dot + bf * xs[g];
            }
            y[n] = TOBF(acc);
        }
        free(xf);
        free(xs);
        return;
    }
    /* qmm: dequantize to bf16 once, then an fp32-accumulated product. */
    float* wf = (float*)malloc(sizeof(float) * (size_t)N * K);
    float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const uint32_t* qr = wq + (size_t)n * (K / per);
        for (int k = 0; k < K; ++k)
            wf[(size_t)n * K + k] = BF(deq1(qget(qr, k, bits), scales[(size_t)n * ng + k / gs],
                                            biases[(size_t)n * ng + k / gs]));
    }
    for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = BF(x[i]);
#pragma omp parallel for collapse(2) schedule(static)
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            const float* xr = xf + (size_t)m * K;
            const float* wr = wf + (size_t)n * K;
            float acc = 0.0f;
            if (rev)
                for (int k = K - 1; k >= 0; --k) acc += xr[k] * wr[k];
            else
                for (int k = 0; k < K; ++k) acc += xr[k] * wr[k];
            y[(size_t)m * N + n] = TOBF(acc);
        }
    }
    free(wf);
    free(xf);
}

/* ------------------------------------------------------------------------ */
/* norms, rotary, elementwise                                               */
/* ------------------------------------------------------------------------ */

/* mlx_fast_rms_norm (crates/mlx-ffi/src/ops/real/blas.rs:5-9): fp32 sum of
 * squares, x * rsqrt(mean + eps) rounded to bf16, then times the bf16 weight. */
void orc_rms_norm(const uint16_t* x, const uint16_t* w, int rows, int dims, float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint16_t* xr = x + (size_t)r * dims;
        float ss = 0.0f;
        for (int i = 0; i < dims; ++i) {
            float v = BF(xr[i]);
            ss += v * v;
        }
        float inv = 1.0f / sqrtf(ss / (float)dims + eps);
        for (int i = 0; i < dims; ++i) {
            float nv = BF(TOBF(BF(xr[i]) * inv));
            out[(size_t)r * dims + i] = TOBF(nv * BF(w[i]));
        }
    }
}

/* grouped_rms_norm (crates/mlx-ffi/src/ops/real/grouped_norm.rs:50-135):
 * groups == 1 is rms_norm; groups > 1 normalises each group in f32 with no
 * weight, multiplies the full-width weight in f32 and casts back once. */
void orc_grouped_rms_norm(const uint16_t* x, const uint16_t* w, int rows, int dims, float eps, int groups,
                          uint16_t* out) {
    if (groups == 1) {
        orc_rms_norm(x, w, rows, dims, eps, out);
        return;
    }
    const int gd = dims / groups;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint16_t* xr = x + (size_t)r * dims;
        for (int g = 0; g < groups; ++g) {
            float ss = 0.0f;
            for (int i = 0; i < gd; ++i) {
                float v = BF(xr[g * gd + i]);
                ss += v * v;
            }
            float inv = 1.0f / sqrtf(ss / (float)gd + eps);
            for (int i = 0; i < gd; ++i) {
                int c = g * gd + i;
                float y = BF(xr[c]) * inv;
                out[(size_t)r * dims + c] = TOBF(y * BF(w[c]));
            }
        }
    }
}

void orc_grouped_rms_norm_f32(const float* x, const float* w, int rows, int dims, float eps, int groups,
                              float* out) {
    const int gd = dims / groups;
    for (int r = 0; r < rows; ++r) {
        for (int g = 0; g < groups; ++g) {
            float ss = 0.0f;
            for (int i = 0; i < gd; ++i) {
                float v = x[(size_t)r * dims + g * gd + i];
                ss += v * v;
            }
            float inv = 1.0f / sqrtf(ss / (float)gd + eps);
            for (int i = 0; i < gd; ++i) {
                int c = g * gd + i;
                out[(size_t)r * dims + c] = (x[(size_t)r * dims + c] * inv) * w[c];
            }
        }
    }
}

void orc_rope_inv_freq(int dims, float theta, float* inv_freq) {
    for (int i = 0; i < dims / 2; ++i) inv_freq[i] = (float)pow((double)theta, -2.0 * (double)i / (double)dims);
}

/* mlx_fast_rope_dynamic(x, dims, traditional=false, base, scale=1, offset)
 * (crates/mlx-ffi/src/ops/real/blas.rs:67-80): rotate pairs (i, i+dims/2). */
void orc_rope(const uint16_t* x, int heads, int T, int dims, float theta, int offset, uint16_t* out) {
    const int half = dims / 2;
    float* inv = (float*)malloc(sizeof(float) * (size_t)half);
    orc_rope_inv_freq(dims, theta, inv);
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < heads; ++h) {
        for (int t = 0; t < T; ++t) {
            const uint16_t* xr = x + ((size_t)h * T + t) * dims;
            uint16_t* orow = out + ((size_t)h * T + t) * dims;
            float pos = (float)(offset + t);
            for (int i = 0; i < half; ++i) {
                float th = pos * inv[i];
                float c = cosf(th), s = sinf(th);
                float x1 = BF(xr[i]), x2 = BF(xr[i + half]);
                float a = x1 * c, b = x2 * s, d = x1 * s, e = x2 * c;
                orow[i] = TOBF(a - b);
                orow[i + half] = TOBF(d + e);
            }
        }
    }
    free(inv);
}

/* silu = multiply(x, sigmoid(x)) (crates/mlx-ffi/src/ops/real/blas.rs:33-37):
 * two bf16-rounded ops. */
static inline float sigmoid_f(float v) {
    float e = expf(-fabsf(v));
    float y = 1.0f / (1.0f + e);
    return v < 0.0f ? 1.0f - y : y;
}

void orc_silu(const uint16_t* x, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) {
        float v = BF(x[i]);
        float sg = BF(TOBF(sigmoid_f(v)));
        out[i] = TOBF(v * sg);
    }
}

void orc_multiply(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = TOBF(BF(a[i]) * BF(b[i]));
}

void orc_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = TOBF(BF(a[i]) + BF(b[i]));
}

/* mlx_argmax (crates/mlx-ffi/src/ops/real/array.rs:6-10): first index of the
 * maximum; NaNs never win. */
int orc_argmax(const uint16_t* x, int n) {
    int best = 0;
    float bv = -INFINITY;
    int found = 0;
    for (int i = 0; i < n; ++i) {
        float v = BF(x[i]);
        if (v != v) continue;
        if (!found || v > bv) {
            bv = v;
            best = i;
            found = 1;
        }
    }
    return best;
}

/* ------------------------------------------------------------------------ */
/* host sampler (crates/serve/src/sampler.rs)                               */
/* ------------------------------------------------------------------------ */

/* SimpleRng (sampler.rs:50-78): xorshift64*, seed 0 replaced by a constant;
 * next_f32 = ((next >> 11) as f64 / 2^53) as f32. */
uint64_t orc_rng_seed(uint64_t seed) { return seed ? seed : 0x9E3779B97F4A7C15ull; }

static uint64_t rng_next_u64(uint64_t* st) {
    uint64_t x = *st;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *st = x;
    return x * 0x2545F4914F6CDD1Dull;
}

float orc_rng_next_f32(uint64_t* st) {
    const double div = (double)(1ull << 53);
    return (float)((double)(rng_next_u64(st) >> 11) / div);
}

typedef struct {
    float v;
    int i;
} vi_t;

/* descending by value, ties by index: what Rust's stable sort_by with
 * b.partial_cmp(a) leaves (NaN compares Equal there; none occur here) */
static int cmp_desc(const void* a, const void* b) {
    const vi_t* x = (const vi_t*)a;
    const vi_t* y = (const vi_t*)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

/* Iterator::max_by(partial_cmp): the LAST index of the maximum. */
static int last_argmax(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (!(x[i] < x[best])) best = i;
    return best;
}

/* sample_token (sampler.rs:101-202), step for step in f32: temperature
 * scaling; top-k keeps values >= the k-th largest; softmax over the finite
 * values with a sequential sum; top-p keeps the largest probabilities (stable
 * descending order) until their running f32 sum reaches top_p; renormalise
 * with a sequential sum over index order; draw r = next_f32 and return the
 * first index whose running sum (index order, all entries) exceeds r, else
 * the last kept index.  Advances *rng by one draw (only when sampling). */
int orc_sample_token(const float* logits, int n, float temperature, float top_p, int top_k, uint64_t* rng) {
    if (n <= 0) return -1;
    if (temperature < 1e-6f) return last_argmax(logits, n);
    const float temp = temperature > 1e-6f ? temperature : 1e-6f;
    float* f = (float*)malloc(sizeof(float) * (size_t)n);
    vi_t* srt = (vi_t*)malloc(sizeof(vi_t) * (size_t)n);
    float* probs = (float*)malloc(sizeof(float) * (size_t)n);
    char* keep = (char*)calloc((size_t)n, 1);
    int tok = 0;
    for (int i = 0; i < n; ++i) f[i] = logits[i] / temp;
    if (top_k > 0 && top_k < n) {
        for (int i = 0; i < n; ++i) {
            srt[i].v = f[i];
            srt[i].i = i;
        }
        qsort(srt, (size_t)n, sizeof(vi_t), cmp_desc);
        const float kth = srt[top_k - 1].v;
        for (int i = 0; i < n; ++i)
            if (f[i] < kth) f[i] = -INFINITY;
    }
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i)
        if (isfinite(f[i])) mx = fmaxf(mx, f[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        probs[i] = isfinite(f[i]) ? expf(f[i] - mx) : 0.0f;
        sum += probs[i];
    }
    if (!isfinite(sum) || sum == 0.0f) {
        tok = last_argmax(logits, n);
        goto done;
    }
    for (int i = 0; i < n; ++i) probs[i] = probs[i] / sum;
    for (int i = 0; i < n; ++i) {
        srt[i].v = probs[i];
        srt[i].i = i;
    }
    qsort(srt, (size_t)n, sizeof(vi_t), cmp_desc);
    {
        float cum = 0.0f;
        for (int j = 0; j < n; ++j) {
            cum += srt[j].v;
            keep[srt[j].i] = 1;
            if (cum >= top_p) break;
        }
    }
    float fsum = 0.0f;
    for (int i = 0; i < n; ++i)
        if (keep[i]) fsum += probs[i];
    if (fsum > 0.0f)
        for (int i = 0; i < n; ++i) probs[i] = keep[i] ? probs[i] / fsum : 0.0f;
    {
        const float r = orc_rng_next_f32(rng);
        float cs = 0.0f;
        tok = -1;
        for (int i = 0; i < n; ++i) {
            cs += probs[i];
            if (r < cs) {
                tok = i;
                break;
            }
        }
        if (tok < 0) {
            tok = 0;
            for (int i = n - 1; i >= 0; --i)
                if (keep[i]) {
                    tok = i;
                    break;
                }
        }
    }
done:
    free(f);
    free(srt);
    free(probs);
    free(keep);
    return tok;
}

/* ------------------------------------------------------------------------ */
/* attention                                                                */
/* ------------------------------------------------------------------------ */

/* mlx_fast_scaled_dot_product_attention, causal prefill
 * (crates/mlx-ffi/src/ops/real/blas.rs:82-97) and array-masked decode over the
 * static cache (crates/mlx-ffi/src/ops/real/transform.rs:8-30).  The 0/-1e9
 * additive mask of engine_ext.rs:238-260 zeroes every position past the
 * offset exactly (exp underflows), so decode attends rows 0..Tk-1. */
void orc_sdpa(const uint16_t* q, const uint16_t* k, const uint16_t* v, int nq, int nkv, int Tq, int Tk,
              int kv_stride, int D, float scale, int causal, uint16_t* out) {
    const int rep = nq / nkv;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int h = 0; h < nq; ++h) {
        for (int t = 0; t < Tq; ++t) {
            const int kh = h / rep;
            const int last = causal ? (Tk - Tq + t) : (Tk - 1);
            const uint16_t* qr = q + ((size_t)h * Tq + t) * D;
            float qs[512];
            for (int d = 0; d < D; ++d) qs[d] = BF(qr[d]) * scale;
            float* sc = (float*)malloc(sizeof(float) * (size_t)(last + 1));
            float m = -INFINITY;
            for (int j = 0; j <= last; ++j) {
                const uint16_t* kr = k + ((size_t)kh * kv_stride + j) * D;
                float s = 0.0f;
                for (int d = 0; d < D; ++d) s += qs[d] * BF(kr[d]);
                sc[j] = s;
                m = s > m ? s : m;
            }
            float l = 0.0f;
            for (int j = 0; j <= last; ++j) {
                sc[j] = expf(sc[j] - m);
                l += sc[j];
            }
            float acc[512];
            for (int d = 0; d < D; ++d) acc[d] = 0.0f;
            for (int j = 0; j <= last; ++j) {
                const uint16_t* vr = v + ((size_t)kh * kv_stride + j) * D;
                for (int d = 0; d < D; ++d) acc[d] += sc[j] * BF(vr[d]);
            }
            uint16_t* orow = out + ((size_t)h * Tq + t) * D;
            for (int d = 0; d < D; ++d) orow[d] = TOBF(acc[d] / l);
            free(sc);
        }
    }
}

/* slice_update (crates/mlx-ffi/src/ops/real/slice.rs:78-91) of the static
 * cache [1,nkv,cap,D] at rows [offset, offset+T); scatter_single at one row is
 * the T == 1 case (crates/serve/tests/profile_decode.rs:224-260). */
void orc_slice_update(uint16_t* cache, const uint16_t* upd, int nkv, int cap, int D, int offset, int T) {
    for (int h = 0; h < nkv; ++h)
        for (int t = 0; t < T; ++t)
            memcpy(cache + ((size_t)h * cap + offset + t) * D, upd + ((size_t)h * T + t) * D,
                   sizeof(uint16_t) * (size_t)D);
}

/* ------------------------------------------------------------------------ */
/* MoE routing                                                              */
/* ------------------------------------------------------------------------ */

/* softmax_axis(-1) on bf16 router logits (crates/ops/src/moe.rs:124), fp32
 * internally, bf16 out. */
void orc_softmax_bf16(const uint16_t* x, int n, uint16_t* out) {
    float m = -INFINITY;
    for (int i = 0; i < n; ++i) m = BF(x[i]) > m ? BF(x[i]) : m;
    float* e = (float*)malloc(sizeof(float) * (size_t)n);
    float s = 0.0f;
    for (int i = 0; i < n; ++i) {
        e[i] = expf(BF(x[i]) - m);
        s += e[i];
    }
    for (int i = 0; i < n; ++i) out[i] = TOBF(e[i] / s);
    free(e);
}

/* topk_cpu (crates/ops/src/moe.rs:256-271): stable descending sort, first k,
 * optional renormalisation by their fp32 sum. */
void orc_topk(const float* scores, int n, int k, int normalize, int* idx, float* weights) {
    int* order = (int*)malloc(sizeof(int) * (size_t)n);
    for (int i = 0; i < n; ++i) order[i] = i;
    /* insertion sort: stable, n is at most a few hundred experts */
    for (int i = 1; i < n; ++i) {
        int cur = order[i];
        int j = i - 1;
        while (j >= 0 && scores[order[j]] < scores[cur]) {
            order[j + 1] = order[j];
            --j;
        }
        order[j + 1] = cur;
    }
    for (int r = 0; r < k; ++r) {
        idx[r] = order[r];
        weights[r] = scores[order[r]];
    }
    if (normalize) {
        float s = 0.0f;
        for (int r = 0; r < k; ++r) s += weights[r];
        if (s > 1e-20f)
            for (int r = 0; r < k; ++r) weights[r] /= s;
    }
    free(order);
}

/* ------------------------------------------------------------------------ */
/* Qwen3 model                                                              */
/* ------------------------------------------------------------------------ */

typedef struct {
    const uint32_t* w;
    const uint16_t* s;
    const uint16_t* b;
} qt;

typedef struct {
    const uint16_t* in_norm;
    const uint16_t* post_norm;
    const uint16_t* q_norm;
    const uint16_t* k_norm;
    qt q, k, v, o, gate, up, down;
    qt router, e_gate, e_up, e_down; /* MoE */
} orc_layer;

struct orc_model {
    orc_qwen3_config c;
    qt embed, lm;
    const uint16_t* final_norm;
    orc_layer* L;
    uint16_t* kcache; /* [layers][n_kv][cap][hd] */
    uint16_t* vcache;
    int offset;
};

orc_model* orc_qwen3_create(const orc_qwen3_config* cfg) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->L = (orc_layer*)calloc((size_t)cfg->layers, sizeof(orc_layer));
    size_t kv = (size_t)cfg->layers * cfg->n_kv * cfg->kv_cap * cfg->head_dim;
    m->kcache = (uint16_t*)calloc(kv, sizeof(uint16_t));
    m->vcache = (uint16_t*)calloc(kv, sizeof(uint16_t));
    return m;
}

void orc_qwen3_destroy(orc_model* m) {
    if (!m) return;
    free(m->L);
    free(m->kcache);
    free(m->vcache);
    free(m);
}

static int set_qt(qt* t, const char* suffix, const void* data) {
    if (!strcmp(suffix, "weight")) t->w = (const uint32_t*)data;
    else if (!strcmp(suffix, "scales")) t->s = (const uint16_t*)data;
    else if (!strcmp(suffix, "biases")) t->b = (const uint16_t*)data;
    else return -1;
    return 0;
}

int orc_qwen3_set_tensor(orc_model* m, const char* name, const void* data) {
    const char* dot = strrchr(name, '.');
    if (!dot) return -1;
    const char* suffix = dot + 1;
    char base[256];
    size_t bl = (size_t)(dot - name);
    if (bl >= sizeof(base)) return -1;
    memcpy(base, name, bl);
    base[bl] = 0;
    if (!strcmp(base, "model.embed_tokens")) return set_qt(&m->embed, suffix, data);
    if (!strcmp(base, "lm_head")) return set_qt(&m->lm, suffix, data);
    if (!strcmp(name, "model.norm.weight")) {
        m->final_norm = (const uint16_t*)data;
        return 0;
    }
    int li = -1, off = 0;
    if (sscanf(base, "model.layers.%d.%n", &li, &off) != 1 || li < 0 || li >= m->c.layers) return -1;
    const char* rest = base + off;
    orc_layer* L = &m->L[li];
    if (!strcmp(rest, "input_layernorm")) { L->in_norm = (const uint16_t*)data; return 0; }
    if (!strcmp(rest, "post_attention_layernorm")) { L->post_norm = (const uint16_t*)data; return 0; }
    if (!strcmp(rest, "self_attn.q_norm")) { L->q_norm = (const uint16_t*)data; return 0; }
    if (!strcmp(rest, "self_attn.k_norm")) { L->k_norm = (const uint16_t*)data; return 0; }
    if (!strcmp(rest, "self_attn.q_proj")) return set_qt(&L->q, suffix, data);
    if (!strcmp(rest, "self_attn.k_proj")) return set_qt(&L->k, suffix, data);
    if (!strcmp(rest, "self_attn.v_proj")) return set_qt(&L->v, suffix, data);
    if (!strcmp(rest, "self_attn.o_proj")) return set_qt(&L->o, suffix, data);
    if (!strcmp(rest, "mlp.gate_proj")) return set_qt(&L->gate, suffix, data);
    if (!strcmp(rest, "mlp.up_proj")) return set_qt(&L->up, suffix, data);
    if (!strcmp(rest, "mlp.down_proj")) return set_qt(&L->down, suffix, data);
    if (!strcmp(rest, "mlp.gate")) return set_qt(&L->router, suffix, data);
    if (!strcmp(rest, "mlp.switch_mlp.gate_proj")) return set_qt(&L->e_gate, suffix, data);
    if (!strcmp(rest, "mlp.switch_mlp.up_proj")) return set_qt(&L->e_up, suffix, data);
    if (!strcmp(rest, "mlp.switch_mlp.down_proj")) return set_qt(&L->e_down, suffix, data);
    return -1;
}

int orc_qwen3_reset(orc_model* m) {
    m->offset = 0;
    return 0;
}

int orc_qwen3_offset(const orc_model* m) { return m->offset; }

const uint16_t* orc_qwen3_kv(const orc_model* m, int layer, int which) {
    size_t per = (size_t)m->c.n_kv * m->c.kv_cap * m->c.head_dim;
    return (which ? m->vcache : m->kcache) + per * (size_t)layer;
}

static void qmm(const uint16_t* x, const qt* t, int M, int N, int K, orc_quant q, uint16_t* y) {
    orc_qmatmul(x, t->w, t->s, t->b, M, N, K, q.group_size, q.bits, y);
}

/* Qwen3-MoE sparse block for one token, after moe_forward
 * (crates/ops/src/moe.rs:103-166): router qmatmul -> softmax -> top-k (+renorm)
 * -> per-expert SwiGLU (swiglu_mlp, crates/ops/src/mlp.rs:23-35) weighted by
 * the fp32 routing weight and summed in fp32 in rank order. */
static void moe_token(const orc_model* m, const orc_layer* L, const uint16_t* xn, float* out) {
    const orc_qwen3_config* c = &m->c;
    const int H = c->hidden, E = c->n_experts, I = c->moe_inter;
    uint16_t* logits = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)E);
    uint16_t* probs = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)E);
    float* pf = (float*)malloc(sizeof(float) * (size_t)E);
    qmm(xn, &L->router, 1, E, H, c->q_router, logits);
    orc_softmax_bf16(logits, E, probs);
    for (int e = 0; e < E; ++e) pf[e] = BF(probs[e]);
    int idx[64];
    float wt[64];
    orc_topk(pf, E, c->top_k, c->norm_topk, idx, wt);
    for (int i = 0; i < H; ++i) out[i] = 0.0f;
    const int per = 32 / c->q_expert.bits;
    const size_t gw = (size_t)I * (H / per), gsb = (size_t)I * (H / c->q_expert.group_size);
    const size_t dw = (size_t)H * (I / per), dsb = (size_t)H * (I / c->q_expert.group_size);
    uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)I);
    uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)I);
    uint16_t* h = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)I);
    uint16_t* d = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)H);
    for (int r = 0; r < c->top_k; ++r) {
        const int e = idx[r];
        qt tg = {L->e_gate.w + gw * e, L->e_gate.s + gsb * e, L->e_gate.b + gsb * e};
        qt tu = {L->e_up.w + gw * e, L->e_up.s + gsb * e, L->e_up.b + gsb * e};
        qt td = {L->e_down.w + dw * e, L->e_down.s + dsb * e, L->e_down.b + dsb * e};
        qmm(xn, &tg, 1, I, H, c->q_expert, g);
        qmm(xn, &tu, 1, I, H, c->q_expert, u);
        orc_silu(g, (size_t)I, g);
        orc_multiply(g, u, (size_t)I, h);
        qmm(h, &td, 1, H, I, c->q_expert, d);
        for (int i = 0; i < H; ++i) out[i] += BF(d[i]) * wt[r];
    }
    free(logits); free(probs); free(pf); free(g); free(u); free(h); free(d);
}

/* One forward over T tokens at the current offset — the per-layer chain of
 * prefill (crates/serve/src/forward_qwen3.rs:52-166) and of the traced decode
 * step (crates/serve/src/compiled.rs:127-201).  decode == 1 takes the decode
 * attention (scatter at offset, masked SDPA over rows 0..offset); otherwise
 * the prefill attention (slice_update of T rows, causal SDPA over the T new
 * rows only, as forward_qwen3.rs:150 does). */
static int forward(orc_model* m, const int32_t* tokens, int T, int decode, uint16_t* logits_out) {
    const orc_qwen3_config* c = &m->c;
    const int H = c->hidden, nq = c->n_q, nkv = c->n_kv, hd = c->head_dim, I = c->inter;
    const int off = m->offset;
    if (off + T > c->kv_cap) return -1;
    const size_t TH = (size_t)T * H;
    uint16_t* x = (uint16_t*)malloc(sizeof(uint16_t) * TH);
    uint16_t* xn = (uint16_t*)malloc(sizeof(uint16_t) * TH);
    uint16_t* q = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nq * hd);
    uint16_t* k = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nkv * hd);
    uint16_t* v = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nkv * hd);
    uint16_t* qt_ = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nq * hd);
    uint16_t* kt = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nkv * hd);
    uint16_t* vt = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nkv * hd);
    uint16_t* at = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nq * hd);
    uint16_t* a = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * nq * hd);
    uint16_t* o = (uint16_t*)malloc(sizeof(uint16_t) * TH);
    const int FF = c->n_experts ? H : I;
    uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * FF);
    uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * FF);
    float* mo = (float*)malloc(sizeof(float) * (size_t)H);

    /* embed: dequantized table row gather (engine.rs:120-163, engine_ext.rs:45-67) */
    {
        const int per = 32 / c->q_embed.bits, ngr = H / c->q_embed.group_size;
        for (int t = 0; t < T; ++t) {
            const int id = tokens[t];
            if (id < 0 || id >= c->vocab) return -2;
            orc_dequantize(m->embed.w + (size_t)id * (H / per), m->embed.s + (size_t)id * ngr,
                           m->embed.b + (size_t)id * ngr, 1, H, c->q_embed.group_size, c->q_embed.bits,
                           x + (size_t)t * H);
        }
    }
    const size_t layer_kv = (size_t)nkv * c->kv_cap * hd;
    for (int li = 0; li < c->layers; ++li) {
        const orc_layer* L = &m->L[li];
        orc_grouped_rms_norm(x, L->in_norm, T, H, c->eps, c->norm_groups, xn);
        qmm(xn, &L->q, T, nq * hd, H, c->q_attn, q);
        qmm(xn, &L->k, T, nkv * hd, H, c->q_attn, k);
        qmm(xn, &L->v, T, nkv * hd, H, c->q_attn, v);
        if (L->q_norm) orc_rms_norm(q, L->q_norm, T * nq, hd, c->eps, q);
        if (L->k_norm) orc_rms_norm(k, L->k_norm, T * nkv, hd, c->eps, k);
        /* [T, h, hd] -> [h, T, hd] */
        for (int t = 0; t < T; ++t) {
            for (int h = 0; h < nq; ++h)
                memcpy(qt_ + ((size_t)h * T + t) * hd, q + ((size_t)t * nq + h) * hd, 2 * (size_t)hd);
            for (int h = 0; h < nkv; ++h) {
                memcpy(kt + ((size_t)h * T + t) * hd, k + ((size_t)t * nkv + h) * hd, 2 * (size_t)hd);
                memcpy(vt + ((size_t)h * T + t) * hd, v + ((size_t)t * nkv + h) * hd, 2 * (size_t)hd);
            }
        }
        orc_rope(qt_, nq, T, hd, c->rope_theta, off, qt_);
        orc_rope(kt, nkv, T, hd, c->rope_theta, off, kt);
        uint16_t* kc = m->kcache + layer_kv * li;
        uint16_t* vc = m->vcache + layer_kv * li;
        orc_slice_update(kc, kt, nkv, c->kv_cap, hd, off, T);
        orc_slice_update(vc, vt, nkv, c->kv_cap, hd, off, T);
        const float scale = 1.0f / sqrtf((float)hd);
        if (decode)
            orc_sdpa(qt_, kc, vc, nq, nkv, T, off + T, c->kv_cap, hd, scale, 0, at);
        else
            orc_sdpa(qt_, kt, vt, nq, nkv, T, T, T, hd, scale, 1, at);
        for (int t = 0; t < T; ++t)
            for (int h = 0; h < nq; ++h)
                memcpy(a + ((size_t)t * nq + h) * hd, at + ((size_t)h * T + t) * hd, 2 * (size_t)hd);
        qmm(a, &L->o, T, H, nq * hd, c->q_attn, o);
        orc_add(x, o, TH, x);
        orc_grouped_rms_norm(x, L->post_norm, T, H, c->eps, c->norm_groups, xn);
        if (c->n_experts) {
            for (int t = 0; t < T; ++t) {
                moe_token(m, L, xn + (size_t)t * H, mo);
                for (int i = 0; i < H; ++i) x[(size_t)t * H + i] = TOBF(BF(x[(size_t)t * H + i]) + mo[i]);
            }
        } else {
            qmm(xn, &L->gate, T, I, H, c->q_mlp, g);
            qmm(xn, &L->up, T, I, H, c->q_mlp, u);
            orc_silu(g, (size_t)T * I, g);
            orc_multiply(g, u, (size_t)T * I, g);
            qmm(g, &L->down, T, H, I, c->q_mlp, o);
            orc_add(x, o, TH, x);
        }
    }
    /* final norm, last row, lm_head (tied -> embed_tokens), argmax */
    uint16_t* last = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)H);
    orc_grouped_rms_norm(x + (size_t)(T - 1) * H, m->final_norm, 1, H, c->eps, c->norm_groups, last);
    uint16_t* logits = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)c->vocab);
    if (c->tied)
        qmm(last, &m->embed, 1, c->vocab, H, c->q_embed, logits);
    else
        qmm(last, &m->lm, 1, c->vocab, H, c->q_lm, logits);
    int tok = orc_argmax(logits, c->vocab);
    if (logits_out) memcpy(logits_out, logits, sizeof(uint16_t) * (size_t)c->vocab);
    m->offset += T;
    free(last); free(logits);
    free(x); free(xn); free(q); free(k); free(v); free(qt_); free(kt); free(vt); free(at); free(a);
    free(o); free(g); free(u); free(mo);
    return tok;
}

int orc_qwen3_prefill(orc_model* m, const int32_t* tokens, int T, uint16_t* logits) {
    return forward(m, tokens, T, 0, logits);
}

int orc_qwen3_decode(orc_model* m, int32_t token, uint16_t* logits) {
    return forward(m, &token, 1, 1, logits);
}
