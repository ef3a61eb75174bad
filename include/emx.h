/*
 * emx.h — C ABI of libemx, the sm_100a replacement for engine-mlx's
 * crates/mlx-ffi on the quantized Qwen3 forward path.
 *
 * Conventions (mirroring MlxCtx, crates/mlx-ffi/src/ops/real/mod.rs:4-41):
 *   - every call returns int: EMX_OK (0) or an EMX_ERR_* code; the message of
 *     the last failure on the calling thread is emx_last_error(), and it is
 *     also passed to the handler installed with emx_set_error_handler (the
 *     reference installs mlx_set_error_handler at mod.rs:8-23 and maps a
 *     non-zero status to an error in MlxCtx::check, mod.rs:35-40);
 *   - tensors are plain device pointers to dense row-major data; bf16 values
 *     are 16-bit patterns; quantized weights use the MLX affine layout
 *     (uint32 words, element k of a row at bits bits*(k % (32/bits)) of word
 *     k/(32/bits); bf16 scales and biases [N, K/group_size]);
 *   - work is enqueued on the context's CUDA stream in call order (MLX's
 *     lazy graph + eval is replaced by eager stream order: emx_synchronize
 *     is mlx_synchronize, reads back through emx_memcpy_d2h are the sync
 *     points, like to_vec_* at crates/mlx-ffi/src/ops/real/array.rs:103-200).
 * No entry point falls back to the CPU: without a usable sm_100 device every
 * call fails with EMX_ERR_CUDA.
 */
#ifndef EMX_H
#define EMX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define EMX_OK 0
#define EMX_ERR_INVALID 1 /* bad argument or unsupported shape */
#define EMX_ERR_CUDA 2    /* CUDA runtime / library failure */
#define EMX_ERR_OOM 3     /* device allocation failed or over the memory limit */
#define EMX_ERR_DEVICE 4  /* a kernel reported a device-side status (see emx_device_status) */
#define EMX_ERR_NCCL 5    /* collective failure */
#define EMX_ERR_STATE 6   /* call out of order (e.g. KV capacity exceeded) */

/* device-side status codes (emx_device_status) */
#define EMX_DEV_OK 0
#define EMX_DEV_TIMEOUT_MBAR 1 /* a bounded shared-memory barrier wait gave up */
#define EMX_DEV_TIMEOUT_PEER 2 /* a bounded peer-flag wait gave up */
#define EMX_DEV_BAD_TOKEN 3    /* token id outside [0, vocab) */
#define EMX_DEV_KV_OVERFLOW 4  /* position >= KV capacity */

typedef enum { EMX_BF16 = 0, EMX_F32 = 1, EMX_U32 = 2, EMX_I32 = 3 } emx_dtype;

/* ------------------------------------------------------------------ errors */
typedef void (*emx_error_handler)(const char* msg, void* data);
/* Replaces mlx_set_error_handler (crates/mlx-ffi/src/ops/real/mod.rs:8-23). */
void emx_set_error_handler(emx_error_handler handler, void* data);
const char* emx_last_error(void);
const char* emx_version(void);

/* ----------------------------------------------------------------- context */
typedef struct emx_ctx emx_ctx;
/* MlxCtx::new / MlxCtx::gpu + mlx_default_gpu_stream_new
 * (crates/mlx-ffi/src/ops/real/mod.rs:19-33, crates/serve/src/engine.rs:69-80). */
int emx_ctx_create(int device, emx_ctx** out);
int emx_ctx_destroy(emx_ctx* ctx);
int emx_ctx_stream(emx_ctx* ctx, void** cuda_stream);
int emx_ctx_num_sms(emx_ctx* ctx, int* n);
/* mlx_synchronize (crates/serve/src/decode_compiled.rs:29,47). */
int emx_synchronize(emx_ctx* ctx);
/* Reads (and optionally clears) the context's device-side status word. */
int emx_device_status(emx_ctx* ctx, int* status, int clear);

/* ------------------------------------------------------------------ memory */
int emx_malloc(emx_ctx* ctx, size_t bytes, void** ptr);
int emx_free(emx_ctx* ctx, void* ptr);
/* Stream-ordered copies; d2h returns after the copy (and all prior work) is done. */
int emx_memcpy_h2d(emx_ctx* ctx, void* dst, const void* src, size_t bytes);
int emx_memcpy_d2h(emx_ctx* ctx, void* dst, const void* src, size_t bytes);
int emx_memset(emx_ctx* ctx, void* dst, int value, size_t bytes);
/* mlx_get_active_memory / mlx_get_peak_memory / mlx_set_memory_limit
 * (crates/serve/src/engine.rs:84-110, crates/serve/tests/leak_probe.rs). */
int emx_get_active_memory(emx_ctx* ctx, size_t* bytes);
int emx_get_peak_memory(emx_ctx* ctx, size_t* bytes);
int emx_set_memory_limit(emx_ctx* ctx, size_t limit, size_t* previous);

/* --------------------------------------------------------------------- ops
 * One entry per MlxCtx method on the Qwen3 path; all pointers are device
 * pointers, all work is enqueued on ctx's stream. */

/* MlxCtx::quantized_matmul (crates/mlx-ffi/src/ops/real/transform.rs:77-89):
 * y[M,N] = x[M,K] . dequant(w)^T; transpose must be 1; bits 4|8; group 32|64|128.
 * M == 1 runs the batch-1 GEMV, M > 1 the prefill GEMM. */
int emx_quantized_matmul(emx_ctx* ctx, const void* x, const void* w, const void* scales, const void* biases, void* y,
                         int M, int N, int K, int transpose, int group_size, int bits);
/* No reference counterpart (MLX reads the affine layout directly): the
 * load-time re-layout of an affine tensor (w [N][K*bits/32], scales/biases
 * [N][K/group]) into the packed tile layout that the engine's batch-1 decode
 * GEMV streams.  emx_qpack_bytes gives the size of `out` (N a multiple of
 * 16). */
int emx_qpack_bytes(int N, int K, int group_size, int bits, size_t* bytes);
int emx_qpack(emx_ctx* ctx, const void* w, const void* scales, const void* biases, void* out, int N, int K,
              int group_size, int bits);
/* MlxCtx::quantized_matmul at M == 1 (transform.rs:77-89) over a packed
 * tensor: y[N] = x[K] . dequant(w)^T, the decode GEMV the engine runs. */
int emx_quantized_matvec_packed(emx_ctx* ctx, const void* x, const void* packed, void* y, int N, int K,
                                int group_size, int bits);
/* MlxCtx::quantized_matmul (transform.rs:77-89) over a packed tensor at any
 * M: y[M,N] = x[M,K] . dequant(w)^T.  M == 1 is the decode GEMV above; M > 1
 * is the prefill GEMM the engine runs over the same packed bytes (group size
 * 64 only). */
int emx_quantized_matmul_packed(emx_ctx* ctx, const void* x, const void* packed, void* y, int M, int N, int K,
                                int group_size, int bits);
/* MlxCtx::dequantize_weight (transform.rs:45-60): out bf16[N,K]. */
int emx_dequantize(emx_ctx* ctx, const void* w, const void* scales, const void* biases, void* out, int N, int K,
                   int group_size, int bits);
/* MlxCtx::quantize_kv_native / mlx_quantize affine (crates/mlx-ffi/src/ops/real/quant.rs:8-38):
 * src f32 or bf16 [N,K]; scale = (max-min)/(2^bits-1), bias = min (bf16). */
int emx_quantize(emx_ctx* ctx, const void* src, emx_dtype src_dtype, void* w, void* scales, void* biases, int N,
                 int K, int group_size, int bits);
/* MlxCtx::rms_norm (crates/mlx-ffi/src/ops/real/blas.rs:5-9): rows x dims, bf16. */
int emx_rms_norm(emx_ctx* ctx, const void* x, const void* weight, void* out, int rows, int dims, float eps);
/* MlxCtx::grouped_rms_norm (crates/mlx-ffi/src/ops/real/grouped_norm.rs:50-135). */
int emx_grouped_rms_norm(emx_ctx* ctx, const void* x, const void* weight, void* out, int rows, int dims, float eps,
                         int groups);
/* MlxCtx::rope / rope_dynamic (blas.rs:67-80), traditional=false, scale 1:
 * x[heads, T, dims]; position = offset + (*offset_dev if non-null) + t. */
int emx_rope(emx_ctx* ctx, const void* x, void* out, int heads, int T, int dims, float theta, int offset,
             const int32_t* offset_dev);
/* MlxCtx::sdpa(causal=true) (blas.rs:82-97): q[nq,T,D], k,v[nkv,T,D];
 * out[nq,T,D] (out_tnd == 0) or [T,nq,D] (out_tnd == 1, the transposed
 * layout the o_proj consumes).  D must be 128. */
int emx_sdpa_causal(emx_ctx* ctx, const void* q, const void* k, const void* v, void* out, int nq, int nkv, int T,
                    int head_dim, float scale, int out_tnd);
/* MlxCtx::sdpa_masked over the static cache (transform.rs:8-30) with the
 * 0 / -1e9 prefix mask of engine_ext.rs:238-260, given as its valid length:
 * q[nq,D] attends rows [0, length) of k,v[nkv,cap,D]; out[nq,D]. */
int emx_sdpa_decode(emx_ctx* ctx, const void* q, const void* k_cache, const void* v_cache, void* out, int nq,
                    int nkv, int cap, int head_dim, int length, float scale);
/* No counterpart in the reference (MLX allocates every op's output and
 * temporaries itself).  emx_sdpa_decode with the same arguments and a
 * bit-identical result, but it allocates nothing: its split partials and
 * merge tickets live in one static 1 MiB device array (n_kv <= 64 and
 * n_q * splits * (head_dim + 2) * 4 bytes <= 1 MiB - 256, else
 * EMX_ERR_INVALID).  The array is shared per device, so calls that overlap
 * in time race; calls on one stream are safe.  A call outside a stream
 * capture looks the array up (cudaGetSymbolAddress; the first may load the
 * module, and after a cudaDeviceReset it finds the reloaded array); a call
 * inside a capture reuses the last address, so one call should precede any
 * capture. */
int emx_sdpa_decode_noalloc(emx_ctx* ctx, const void* q, const void* k_cache, const void* v_cache, void* out, int nq,
                            int nkv, int cap, int head_dim, int length, float scale);
/* MlxCtx::silu / multiply / add (blas.rs:17-37), bf16 elementwise. */
int emx_silu(emx_ctx* ctx, const void* x, void* out, size_t n);
int emx_multiply(emx_ctx* ctx, const void* a, const void* b, void* out, size_t n);
int emx_add(emx_ctx* ctx, const void* a, const void* b, void* out, size_t n);
/* MlxCtx::argmax (crates/mlx-ffi/src/ops/real/array.rs:6-10): first index of
 * the maximum of each row; out int32[rows] (device). */
int emx_argmax(emx_ctx* ctx, const void* x, int rows, int n, int32_t* out);
/* sample_token (crates/serve/src/sampler.rs:101-202) on the device, for
 * temperature >= 1e-6: temperature scaling, top-k (0 = off), softmax, top-p
 * (stable descending order, ties by index), renormalisation, one draw of
 * SimpleRng (xorshift64*; *rng_state is a device uint64 advanced in place)
 * and the first index whose running sum exceeds it.  logits: bf16 [n]
 * (device); token: int32 (device).  Sums the host takes sequentially in fp32
 * are taken per thread slice, then over the slices in order, so a draw
 * within a few ulps of a boundary may pick the neighbouring token; with
 * top_p >= 1 every entry is kept. */
int emx_sample_token(emx_ctx* ctx, const void* logits, int n, float temperature, float top_p, int top_k,
                     uint64_t* rng_state, int32_t* token);
/* MlxCtx::softmax_axis(-1) (crates/mlx-ffi/src/ops/real/elementwise.rs:68-72), bf16. */
int emx_softmax(emx_ctx* ctx, const void* x, void* out, int rows, int n);
/* Qwen3Engine::embed = take(dequantize(embed_tokens), ids)
 * (crates/serve/src/engine_ext.rs:45-67, engine.rs:120-163), one row at a time:
 * out bf16[T, hidden]. */
int emx_embed_quantized(emx_ctx* ctx, const void* w, const void* scales, const void* biases, const int32_t* ids,
                        int T, int hidden, int vocab, int group_size, int bits, void* out);
/* MlxCtx::slice_update of the static cache (crates/mlx-ffi/src/ops/real/slice.rs:78-91):
 * cache[nkv,cap,D] rows [offset, offset+T) <- upd[nkv,T,D]. */
int emx_slice_update(emx_ctx* ctx, void* cache, const void* upd, int nkv, int cap, int head_dim, int offset, int T);
/* MlxCtx::scatter_single at a device-held offset (slice.rs:106-115): one row. */
int emx_scatter_single(emx_ctx* ctx, void* cache, const int32_t* offset, const void* upd, int nkv, int cap,
                       int head_dim);
/* moe_forward routing (crates/ops/src/moe.rs:112-128, 256-271) on device:
 * softmax of bf16 router logits[E], stable top-k, optional renormalisation;
 * idx int32[k], weights f32[k] (device). */
int emx_moe_route(emx_ctx* ctx, const void* router_logits, int n_experts, int top_k, int normalize, int32_t* idx,
                  float* weights);
/* Gather-quantized-matmul (the per-expert take + quantized_matmul loop of
 * crates/ops/src/moe.rs:140-163 as one launch): for slot s < n_slots,
 * y[s, :] = x_s . dequant(w[idx[s]])^T with w packed [E, N, K*bits/32];
 * x_s = x + s*K when x_per_slot != 0, else x for every slot.  y bf16[n_slots, N]. */
int emx_gather_qmm(emx_ctx* ctx, const void* x, int x_per_slot, const void* w, const void* scales,
                   const void* biases, const int32_t* idx, int n_slots, void* y, int n_experts, int N, int K,
                   int group_size, int bits);

/* ------------------------------------------------------------ collectives */
typedef struct emx_comm emx_comm;
#define EMX_UNIQUE_ID_BYTES 128
/* ncclGetUniqueId on rank 0; the bytes are shared with the other ranks by the caller. */
int emx_comm_unique_id(void* id_out);
int emx_comm_init(emx_ctx* ctx, const void* unique_id, int nranks, int rank, emx_comm** out);
int emx_comm_destroy(emx_comm* comm);
/* In-place sum all-reduce on ctx's stream (f32 or bf16). */
int emx_all_reduce_sum(emx_comm* comm, void* buf, size_t count, emx_dtype dtype);

/* ------------------------------------------------------------------ Qwen3 */
typedef struct {
  int hidden, layers, n_q, n_kv, head_dim, inter, vocab;
  float eps, rope_theta;
  int tied;        /* lm_head reuses model.embed_tokens */
  int norm_groups; /* layernorm_num_groups (crates/serve/src/config.rs:24-27) */
  int attn_bits, attn_group; /* q/k/v/o */
  int mlp_bits, mlp_group;   /* gate/up/down (dense) */
  int embed_bits, embed_group;
  int lm_bits, lm_group;     /* untied lm_head */
  int n_experts, top_k, moe_inter, norm_topk; /* n_experts == 0: dense MLP */
  int router_bits, router_group, expert_bits, expert_group;
  int kv_cap;      /* static KV capacity (MAX_CAP, crates/serve/src/engine.rs:202) */
  int max_prefill; /* largest prompt per prefill call */
} emx_qwen3_config;

typedef struct emx_qwen3 emx_qwen3;

/* Host only: Qwen3Config::from_dir (crates/serve/src/config.rs:77-90, fields
 * and serde defaults at config.rs:8-30, head_dim default at config.rs:92-96)
 * from `model_dir`/config.json (or a config.json path), plus the MoE keys
 * (num_experts, num_experts_per_tok, moe_intermediate_size, norm_topk_prob)
 * and tie_word_embeddings (default true).  Quantization: the model-wide
 * {group_size, bits} of "quantization" and MLX's per-module entries keyed by
 * module name, one setting per kind (attention, dense MLP, embedding,
 * lm_head, router, experts); an unquantized module or two settings within a
 * kind fail with EMX_ERR_INVALID.  kv_cap and max_prefill are the engine's
 * own (MAX_CAP, crates/serve/src/engine.rs:202). */
int emx_qwen3_config_from_dir(const char* model_dir, int kv_cap, int max_prefill, emx_qwen3_config* out);

/* Qwen3Engine::from_init (crates/serve/src/engine.rs:62-227): allocates the
 * weights, the static bf16 KV cache [layers][n_kv][kv_cap][head_dim] and the
 * decode state.  comm == NULL: one GPU; otherwise the model is tensor-parallel
 * (dense: heads and intermediate split across ranks) or expert-parallel (MoE). */
int emx_qwen3_create(emx_ctx* ctx, const emx_qwen3_config* cfg, emx_comm* comm, emx_qwen3** out);
int emx_qwen3_destroy(emx_qwen3* m);
/* load_weights_from_manifest (crates/serve/src/loader/weights.rs:17-284):
 * one tensor under its MLX checkpoint name, host bytes in MLX layout (the full
 * unsharded tensor; each rank keeps its shard).  q/k/v and gate/up are fused
 * at load time as loader/fusion.rs:24-59 does. */
int emx_qwen3_load_tensor(emx_qwen3* m, const char* name, const void* host, size_t bytes);
/* Copies a loaded tensor (this rank's shard, fused layout) back to the host. */
int emx_qwen3_read_tensor(emx_qwen3* m, const char* name, void* host, size_t bytes);
/* load_weights_from_manifest's checkpoint files (crates/serve/src/loader/
 * weights.rs:17-60, dtypes of loader/tensor.rs:5-16): `path` is a model
 * directory -- model_fused.safetensors preferred, else model.safetensors,
 * else the shards named by model.safetensors.index.json -- or one
 * .safetensors file.  Every tensor the model takes is loaded through
 * emx_qwen3_load_tensor (this rank's shard); shipped fused
 * self_attn.qkv_proj / mlp.gate_up_proj tensors are split into their parts
 * (weights.rs:103-118, 166-175); tensors off this path are skipped, as the
 * reference never looks them up.  Fails (EMX_ERR_INVALID) on a malformed
 * container, a dtype or shape the model does not take, an lm_head for a
 * model created tied, or -- after all files -- "missing <name>" for a
 * tensor no file held.  *n_loaded (optional): checkpoint tensors used. */
int emx_qwen3_load_safetensors(emx_qwen3* m, const char* path, int* n_loaded);
/* The MLX checkpoint names of every tensor the model takes, one per line;
 * *need = bytes including the terminating NUL (buf may be NULL). */
int emx_qwen3_tensor_names(emx_qwen3* m, char* buf, size_t cap, size_t* need);
/* Full (unsharded) MLX shape and dtype (EMX_U32 codes, EMX_BF16 scales /
 * biases / norms) of one of those tensors; ndim is 1, 2 or 3. */
int emx_qwen3_tensor_shape(emx_qwen3* m, const char* name, int64_t* shape3, int* ndim, int* dtype);

/* Qwen3Engine::set_sampling (crates/serve/src/engine.rs:230-233) with the
 * host sampler moved onto the device: temperature < 1e-6 keeps the in-graph
 * greedy argmax; otherwise every prefill and decode step ends with
 * emx_sample_token's draw (no logits readback, no host sort).  top_p is
 * clamped to [0, 1] (SamplingParams::with_top_p); the generator restarts
 * from `seed` as SimpleRng::new(seed) (0 -> a fixed constant); the engine
 * starts as SimpleRng::new(42), greedy.  While sampling, the persistent step
 * (emx_qwen3_set_fused) is not used. */
int emx_qwen3_set_sampling(emx_qwen3* m, float temperature, float top_p, int top_k, uint64_t seed);

/* One tensor of a .safetensors file (emx_safetensors_index). */
typedef struct {
  char name[256];
  char dtype[12]; /* as in the header: "BF16", "U32", "F32", ... */
  int ndim;
  int64_t shape[8];
  uint64_t offset; /* byte offset of the data from the start of the file */
  uint64_t bytes;
} emx_st_tensor;
/* Host only (no device needed): validates a .safetensors file the way the
 * safetensors crate's deserialize does (header fits the file, each tensor's
 * bytes are prod(shape) * dtype size, the tensors tile the data section)
 * and lists up to `cap` tensors in header order; *n = the file's count. */
int emx_safetensors_index(const char* file, emx_st_tensor* out, int cap, int* n);
/* Copies layer `layer`'s K (which = 0) or V (which = 1) cache of this rank to
 * the host: bf16 [n_kv_local, kv_cap, head_dim], rows >= offset unspecified.
 * The engine's per-layer kv_bufs pair (crates/serve/src/engine_ext.rs:69-90)
 * holds the same K/V arrays. */
int emx_qwen3_read_kv(emx_qwen3* m, int layer, int which, void* host, size_t bytes);
/* Seeded synthetic weights generated on the device (linears N(0, 0.02^2)
 * quantized with the affine formula, norms 1 + N(0, 0.05^2) in bf16). */
int emx_qwen3_init_random(emx_qwen3* m, uint64_t seed);
/* Qwen3Engine::reset (crates/serve/src/engine_ext.rs:10-36): offset = 0. */
int emx_qwen3_reset(emx_qwen3* m);
int emx_qwen3_offset(emx_qwen3* m, int* offset);
/* Qwen3Engine::prefill (crates/serve/src/forward_qwen3.rs:12-200) of T host
 * token ids at the current offset, then the greedy token of the last row.
 * logits (optional) receives bf16[vocab] of that row. */
int emx_qwen3_prefill(emx_qwen3* m, const int32_t* tokens, int T, int32_t* next_token, void* logits);
/* Chunked prefill (crates/prefill/src/pipeline.rs:60-117 with
 * make_chunks, chunked_prefill.rs:18-20): T host tokens in chunks of
 * min(chunk, max_prefill) at the current offset, each chunk attending the
 * cached rows before it as well as itself, so T may exceed max_prefill and
 * the result is that of one causal pass over all T rows (the reference's
 * forward_fn per chunk, emx_qwen3_prefill above, attends the chunk only).
 * next_token / logits: the last row's, as emx_qwen3_prefill. */
int emx_qwen3_prefill_chunked(emx_qwen3* m, const int32_t* tokens, int T, int chunk, int32_t* next_token,
                              void* logits);
/* Qwen3Engine::decode_step (forward_qwen3.rs:206-243 -> decode_step_static,
 * decode_compiled.rs:14-65): one greedy step, replayed from a CUDA graph. */
int emx_qwen3_decode_step(emx_qwen3* m, int32_t token, int32_t* next_token, void* logits);
/* n greedy steps starting from `token`, one host synchronisation in total;
 * tokens_out receives the n generated ids. */
int emx_qwen3_decode(emx_qwen3* m, int32_t token, int n, int32_t* tokens_out);
/* Called by emx_qwen3_decode_stream with each generated token as it is
 * produced (index = 0, 1, ... within the call); return 0 to go on, nonzero to
 * stop after this token. */
typedef int (*emx_token_cb)(int32_t token, int index, void* user);
/* Per-token streaming for the server's SSE path (crates/serve/src/server.rs:
 * 131-181 generates the whole reply, then splits it into words): up to n
 * steps from `token`, each token handed to cb as soon as its step has run,
 * while greedy decoding keeps up to 8 further steps in flight on the device.
 * When cb returns nonzero the steps run past that token are discarded (the
 * offset, device token and history return to just after it), so a stop at
 * an end-of-sequence token leaves the engine as if decoding had stopped
 * there.  With sampling on, steps run one at a time (no discarded draws).
 * n_done (optional) receives the tokens delivered. */
int emx_qwen3_decode_stream(emx_qwen3* m, int32_t token, int n, emx_token_cb cb, void* user, int* n_done);
/* Device-resident variants for throughput measurement: no host copies.
 * prefill reads ids already on the device; decode runs n graph replays from
 * the device-held token. */
int emx_qwen3_prefill_device(emx_qwen3* m, const int32_t* tokens_dev, int T);
int emx_qwen3_decode_device(emx_qwen3* m, int n);
/* Number of kernel launches one decode step enqueues. */
/* Host only (no device needed): the slice of checkpoint tensor `name` that
 * rank `rank` of `world` keeps under the engine's partitioning — tensor
 * parallel for dense models (q/k/v and gate/up rows, o/down columns),
 * expert parallel for MoE (expert blocks) — as out6 = {row0, n_rows, col0,
 * n_cols, block0, blocks}.  What load_weights_from_manifest would hand each
 * rank (crates/serve/src/loader/weights.rs:17-284; no reference counterpart
 * for the partitioning itself, which is new in this build). */
int emx_qwen3_shard(const emx_qwen3_config* cfg, int world, int rank, const char* name, int32_t* out6);
/* Qwen3Engine::is_compiled (crates/serve/src/engine_ext.rs:212-216) and the
 * choice between the compiled decode closure (decode_compiled.rs:113-120)
 * and the eager per-op step: compiled (default) replays one captured CUDA
 * graph per token with programmatically chained kernels; eager launches the
 * same kernels one by one in plain stream order (for profilers and
 * debugging). */
int emx_qwen3_set_compiled(emx_qwen3* m, int compiled);
int emx_qwen3_is_compiled(emx_qwen3* m, int* compiled);
/* No reference counterpart (the reference's decode step is one traced MLX
 * closure, crates/serve/src/compiled.rs:79-287, whatever its kernels):
 * set_fused(m, 1) runs the whole decode step of a model on one GPU as one
 * persistent kernel whose phases hand off through flag words (dense, or MoE
 * with its router, top-k and the selected experts' projections inside the
 * same launch; the default wherever the model has such a plan);
 * set_fused(m, 0) selects one kernel per operation.  Setting 1 fails with
 * EMX_ERR_INVALID when the model has no such plan (sharded, group size != 64,
 * head_dim != 128, more than 8 q heads per KV head, more than 256 experts or
 * top-16, router and experts of different bit widths). */
int emx_qwen3_set_fused(emx_qwen3* m, int fused);
int emx_qwen3_is_fused(emx_qwen3* m, int* fused);
int emx_qwen3_step_launches(emx_qwen3* m, int* n);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* EMX_H */
