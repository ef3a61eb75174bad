// misc.cuh — standalone kernels behind the op-level C ABI and the prefill path.
#pragma once
#include "common.cuh"
#include "peer.cuh"

namespace emx {

// MLX affine (de)quantization and the seeded synthetic generator.
cudaError_t k_dequantize(const uint32_t* w, const bf16* s, const bf16* b, bf16* out, int N, int K, int gs, int bits,
                         cudaStream_t st);
// src_f32 or src_bf16 (exactly one non-null) [N, K] -> MLX affine layout.
cudaError_t k_quantize(const float* src_f32, const bf16* src_bf16, uint32_t* w, bf16* s, bf16* b, int N, int K,
                       int gs, int bits, cudaStream_t st);
cudaError_t k_fill_normal_f32(uint64_t seed, uint64_t stream, size_t n, float mean, float std, float* out,
                              cudaStream_t st);
cudaError_t k_fill_normal_bf16(uint64_t seed, uint64_t stream, size_t n, float mean, float std, bf16* out,
                               cudaStream_t st);
// Normal(0, std) weights generated and quantized group by group — the same
// bits as k_fill_normal_f32 followed by k_quantize.
cudaError_t k_fill_quantized(uint64_t seed, uint64_t stream, int N, int K, int gs, int bits, float std, uint32_t* w,
                             bf16* s, bf16* b, cudaStream_t st);
// The shard [row0, row0+n_rows) x [col0, col0+n_cols) of a generated
// [*, K_full] tensor, quantized into rows of ldK (== n_cols) columns.
cudaError_t k_fill_quantized_shard(uint64_t seed, uint64_t stream, int n_rows, int n_cols, int K_full, size_t row0,
                                   int col0, int gs, int bits, float std, uint32_t* w, bf16* s, bf16* b, int ldK,
                                   cudaStream_t st);

// rows x dims RMSNorm (groups == 1) or grouped RMSNorm (groups > 1).
cudaError_t k_rms_norm(const bf16* x, const bf16* w, bf16* out, int rows, int dims, float eps, int groups,
                       cudaStream_t st);
// Non-traditional RoPE over x[heads, T, dims]; position = offset (+ *offset_dev
// when given) + t.
cudaError_t k_rope(const bf16* x, bf16* out, int heads, int T, int dims, const float* inv_freq, int offset,
                   const int* offset_dev, cudaStream_t st);
cudaError_t k_rope_inv_freq(float* inv_freq, int dims, float theta, cudaStream_t st);

cudaError_t k_silu(const bf16* x, bf16* out, size_t n, cudaStream_t st);
cudaError_t k_multiply(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t st);
cudaError_t k_add(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t st);
cudaError_t k_argmax(const bf16* x, int rows, int n, int* out, cudaStream_t st);
cudaError_t k_softmax(const bf16* x, bf16* out, int rows, int n, cudaStream_t st);

// Dequantized-row gather from a quantized embedding table (take + dequant).
cudaError_t k_embed(const uint32_t* w, const bf16* s, const bf16* b, const int* ids, int T, int hidden, int gs,
                    int bits, int vocab, bf16* out, int* status, cudaStream_t st);

// Prefill: q/k rms_norm + rope at offset+t, K/V rows written to the cache,
// q re-laid [nq, T, hd] for attention.
struct PrefillQkvArgs {
  const bf16* qkv;  // [T, (nq + 2*nkv)*hd]
  const bf16* q_norm;
  const bf16* k_norm;
  float eps;
  const float* inv_freq;
  const float2* rope_cs;  // optional: (cos, sin) per [position][hd / 2], the same values as sincosf here
  int T, nq, nkv, hd;
  int offset;
  bf16* q_out;  // [nq, T, hd]
  bf16* kc;     // [nkv, cap, hd]
  bf16* vc;
  int cap;
};
cudaError_t k_prefill_qkv(const PrefillQkvArgs& a, cudaStream_t st);

// MoE routing for one token (crates/ops/src/moe.rs:112-128, 256-271):
// softmax of the bf16 router logits (bf16 probabilities), stable top-k,
// optional renormalisation by the fp32 sum, then the slots whose expert lives
// on this rank ([e_base, e_base + e_local)) compacted in rank order:
// idx[j] = local expert id, w[j] = weight, *n = count.  One CTA; E <= 1024.
cudaError_t k_moe_route(const bf16* logits, int E, int k, int normalize, int e_base, int e_local, int* idx,
                        float* w, int* n, cudaStream_t st, bool pdl);
// out[k] = sum_{s < *n} w[s] * y[s, k] in fp32, slot order (expert-parallel partial).
cudaError_t k_moe_combine(const bf16* y, const float* w, const int* n, int H, float* out, cudaStream_t st, bool pdl);
// The same sum stored into every rank's peer-memory slot and published.
cudaError_t k_moe_combine_peer(const bf16* y, const float* w, const int* n, int H, const PeerX* peer, cudaStream_t st,
                               bool pdl);

// x[i] = bf16(x[i] + addend[i]) with addend = bf16(add[i]) when `round`, else
// add[i] (rows x n, fp32 add) — the residual add after a tensor- / expert-
// parallel sum.
cudaError_t k_add_f32(bf16* x, const float* add, size_t n, int round, cudaStream_t st);
// x[k] = bf16(x[k] + sum_{s < *n} w[s] * y[s, k]) — one token's MoE residual.
cudaError_t k_moe_residual(bf16* x, const bf16* y, const float* w, const int* n, int H, cudaStream_t st);
// Batched MoE prefill (crates/ops/src/moe.rs:174-207 routes each token
// independently; here all T tokens at once): routing of T logits rows into
// idx / w [T][k] and n [T]; grouping of the (token, slot) pairs by local
// expert (perm [T][k] -> position, src [P] -> token, tile list of
// (expert, first, end) runs of `tile` positions, counts in *n_tiles and
// *n_pairs = P); the
// gather of x rows into grouped order; and the weighted combine back into
// the residual (or an fp32 partial when out is set).
cudaError_t k_moe_route_batch(const bf16* logits, int T, int E, int k, int normalize, int e_base, int e_local,
                              int* idx, float* w, int* n, cudaStream_t st);
cudaError_t k_moe_group(const int* idx, const int* n, int T, int k, int E_l, int tile, int* perm, int* src,
                        int4* tiles, int* n_tiles, int* n_pairs, cudaStream_t st);
cudaError_t k_moe_gather(const bf16* x, const int* src, const int* P, int Pmax, int H, bf16* xs, cudaStream_t st);
cudaError_t k_moe_combine_batch(bf16* x, const bf16* ys, const float* w, const int* n, const int* perm, int T, int k,
                                int H, float* out, cudaStream_t st);

// cache[nkv, cap, D] rows [offset, offset+T) <- upd[nkv, T, D].
cudaError_t k_slice_update(bf16* cache, const bf16* upd, int nkv, int cap, int D, int offset, const int* offset_dev,
                           int T, cudaStream_t st);

}  // namespace emx
