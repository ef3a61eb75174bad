/*
 * emx_oracle.h — CPU restatement of engine-mlx's quantized Qwen3 forward pass.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the sm_100a
 * kernels in libemx: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs load it.  Nothing in the product
 * (engine-mlx_b200/) links, loads or calls it.
 *
 * What it restates.  The reference (dangranaz/engine-mlx) is Rust over Apple's
 * MLX; every numeric op is one mlx-c call made through
 * crates/mlx-ffi/src/ops/real/ (one file per op family).  MLX itself is not in the reference tree
 * (Homebrew dylib, mlx-c >=0.7,<0.9 per crates/mlx-ffi/src/mlx_c_version.rs:7-10),
 * so each function below restates MLX's *public* semantics for the op at the
 * call site named in its comment, with bf16 rounding at every op output as an
 * MLX bf16 graph does.
 *
 * Pinning.  Pinned against the reference's own known-answer tests where they
 * exist (grouped RMSNorm KATs in crates/mlx-ffi/tests/grouped_rms_norm.rs:82-200
 * and crates/serve/tests/forward_grouped_norm.rs:43-83; fused==separate qkv /
 * gate_up qmatmul in crates/serve/tests/forward_separate.rs:96-162 on the
 * reference's pattern() inputs; scatter_single==slice_update in
 * crates/serve/tests/profile_decode.rs:224-260).  Everything else — qmatmul
 * accumulation order, RoPE frequency formula, SDPA softmax order, argmax
 * tie-break — is PARITY UNPINNED at the MLX boundary: no reference test fixes
 * those bits and MLX cannot be built or run in this container.
 *
 * Conventions: bf16 values are passed as uint16_t bit patterns; all arrays are
 * dense row-major; quantized weights use the MLX affine layout
 * (uint32 words, element k of a row at bits bits*(k % (32/bits)) of word
 * k / (32/bits); scales/biases bf16 [N, K/group_size]).
 */
#ifndef EMX_ORACLE_H
#define EMX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar helpers ---------------------------------------------------- */
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f); /* round-to-nearest-even, NaN preserved */
uint16_t orc_f64_to_bf16(double d); /* correctly rounded (RNE) */
void orc_f32_to_bf16_n(const float* in, uint16_t* out, size_t n);
void orc_bf16_to_f32_n(const uint16_t* in, float* out, size_t n);
int orc_num_threads(void);
void orc_set_num_threads(int n);
/* 0: reductions in ascending index order (default); 1: descending. */
void orc_set_sum_order(int reverse);

/* ---- seeded synthetic generator (same stream as emx_fill_normal) ------- */
uint64_t orc_splitmix64(uint64_t x);
uint64_t orc_name_stream(const char* name); /* FNV-1a 64 of a tensor name */
/* out[i] = mean + std * z_i, z_i a 12-uniform Irwin-Hall variate from
 * (seed, stream, i); bit-identical to the device generator by construction. */
void orc_fill_normal(uint64_t seed, uint64_t stream, size_t n, float mean, float std, float* out);

/* ---- MLX affine quantization (BASELINE formula: scale=(max-min)/(2^bits-1),
 *      bias=min, both stored bf16; q = clamp(rint((w-b)/s), 0, 2^bits-1)) -- */
void orc_quantize(const float* w, int N, int K, int group_size, int bits,
                  uint32_t* wq, uint16_t* scales, uint16_t* biases);
/* mlx_dequantize(..., "affine", dtype=bf16): the bf16 nearest to s*q + b. */
void orc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                    int N, int K, int group_size, int bits, uint16_t* out);
/* mlx_quantized_matmul(x, w, s, b, transpose=true, gs, bits, "affine").
 * M == 1: MLX qmv form  y = sum_g ( s*sum(x*q) + b*sum(x) ) in fp32.
 * M  > 1: MLX qmm form  y = x . bf16(dequant(W))^T with fp32 accumulation. */
void orc_qmatmul(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
                 const uint16_t* biases, int M, int N, int K, int group_size, int bits,
                 uint16_t* y);

/* ---- normalisation / rotary / elementwise ------------------------------ */
void orc_rms_norm(const uint16_t* x, const uint16_t* w, int rows, int dims, float eps, uint16_t* out);
void orc_grouped_rms_norm(const uint16_t* x, const uint16_t* w, int rows, int dims, float eps,
                          int groups, uint16_t* out);
/* f32-in variant used by the reference KATs (mlx arrays made with new_array). */
void orc_grouped_rms_norm_f32(const float* x, const float* w, int rows, int dims, float eps,
                              int groups, float* out);
/* Non-traditional RoPE over all `dims` of x[heads, T, dims], positions offset+t. */
void orc_rope(const uint16_t* x, int heads, int T, int dims, float theta, int offset, uint16_t* out);
void orc_rope_inv_freq(int dims, float theta, float* inv_freq); /* dims/2 entries */
void orc_silu(const uint16_t* x, size_t n, uint16_t* out);
void orc_multiply(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out);
void orc_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out);
int orc_argmax(const uint16_t* x, int n); /* first index of the maximum */
/* host sampler (crates/serve/src/sampler.rs:50-202) */
uint64_t orc_rng_seed(uint64_t seed);
float orc_rng_next_f32(uint64_t* state);
int orc_sample_token(const float* logits, int n, float temperature, float top_p, int top_k, uint64_t* rng);

/* ---- attention --------------------------------------------------------- */
/* q[nq, Tq, D]; k,v[nkv, kv_stride, D] (first Tk rows used).
 * causal: query t attends keys 0..(Tk-Tq+t).  Output out[nq, Tq, D] bf16. */
void orc_sdpa(const uint16_t* q, const uint16_t* k, const uint16_t* v, int nq, int nkv, int Tq,
              int Tk, int kv_stride, int D, float scale, int causal, uint16_t* out);

/* ---- KV cache writes --------------------------------------------------- */
/* cache[nkv, cap, D]; upd[nkv, T, D] written at rows [offset, offset+T). */
void orc_slice_update(uint16_t* cache, const uint16_t* upd, int nkv, int cap, int D, int offset, int T);

/* ---- MoE routing (crates/ops/src/moe.rs:103-166, 256-271) -------------- */
void orc_softmax_bf16(const uint16_t* x, int n, uint16_t* out);
void orc_topk(const float* scores, int n, int k, int normalize, int* idx, float* weights);

/* ---- Qwen3 model ------------------------------------------------------- */
typedef struct {
    int bits, group_size;
} orc_quant;

typedef struct {
    int hidden, layers, n_q, n_kv, head_dim, inter, vocab;
    float eps, rope_theta;
    int tied;        /* lm_head reuses embed_tokens */
    int norm_groups; /* layernorm_num_groups (1 = plain RMSNorm) */
    orc_quant q_attn, q_mlp, q_embed, q_lm;
    /* MoE (n_experts == 0: dense MLP) */
    int n_experts, top_k, moe_inter, norm_topk;
    orc_quant q_router, q_expert;
    int kv_cap;
} orc_qwen3_config;

typedef struct orc_model orc_model;

orc_model* orc_qwen3_create(const orc_qwen3_config* cfg);
void orc_qwen3_destroy(orc_model* m);
/* Registers a host tensor under its MLX checkpoint name (borrowed pointer). */
int orc_qwen3_set_tensor(orc_model* m, const char* name, const void* data);
int orc_qwen3_reset(orc_model* m);
/* Prefill T tokens at the current offset; returns the greedy token.
 * logits (optional, bf16 [vocab]) receives the last row's logits. */
int orc_qwen3_prefill(orc_model* m, const int32_t* tokens, int T, uint16_t* logits);
int orc_qwen3_decode(orc_model* m, int32_t token, uint16_t* logits);
int orc_qwen3_offset(const orc_model* m);
/* The K (which == 0) or V (which == 1) cache of one layer, [n_kv, cap, head_dim]. */
const uint16_t* orc_qwen3_kv(const orc_model* m, int layer, int which);

#ifdef __cplusplus
}
#endif
#endif
