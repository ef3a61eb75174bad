// qwen3.cu — the Qwen3 engine behind the C ABI: what crates/serve's
// Qwen3Engine does through MlxCtx, re-designed for one B200 (or a tensor- /
// expert-parallel group of them).
//
//   reference                                   here
//   ------------------------------------------  -------------------------------------------
//   load_weights_from_manifest + load-time      emx_qwen3_load_tensor: MLX checkpoint names,
//   q/k/v and gate/up fusion                    q|k|v and gate|up fused into one device
//   (loader/weights.rs:17-284, fusion.rs:24-59) tensor each; each rank keeps its shard
//   alloc_kv_static (engine_ext.rs:267-306)     one bf16 KV allocation [L][2][n_kv][cap][128]
//   static mask + offset arrays                 device-held offset (no mask: rows <= offset)
//   compile_shapeless(build_step)               one decode step captured as a CUDA graph
//   (compiled.rs:79-287)                        (5 kernels per layer + lm_head, chained by PDL)
//   prefill (forward_qwen3.rs:12-200)           eager stream-ordered prefill
//   argmax in-graph + to_vec_u32                argmax fused into the lm_head GEMV; 4-byte D2H
#include <sys/stat.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "attn_decode.cuh"
#include "attn_prefill.cuh"
#include "comm.cuh"
#include "ctx.cuh"
#include "misc.cuh"
#include "qgemm.cuh"
#include "tc_gemm.cuh"
#include "pgemv.cuh"
#include "step.cuh"
#include "qgemv.cuh"
#include "safetensors.cuh"
#include "sample.cuh"

namespace emx {

struct QW {
  uint32_t* w = nullptr;
  bf16* s = nullptr;
  bf16* b = nullptr;
  int N = 0, K = 0, bits = 4, gs = 64;
  unsigned char* pk = nullptr;  // packed copy for the decode GEMV (pgemv layout)
  PackMap map{1, 0, 1};
  size_t wbytes() const { return (size_t)N * K / (32 / bits) * 4; }
  size_t sbytes() const { return (size_t)N * (K / gs) * 2; }
};

struct LayerW {
  bf16* in_norm = nullptr;
  bf16* post_norm = nullptr;
  bf16* q_norm = nullptr;
  bf16* k_norm = nullptr;
  QW qkv, o, gate_up, down;  // dense
  QW router, e_gu, e_down;   // MoE: e_gu [E_l][2*Im][H], e_down [E_l][H][Im]
  PgemvPlan p_qkv{}, p_o{}, p_gu{}, p_down{}, p_router{}, p_egu{}, p_edown{};
};

// How one checkpoint tensor maps onto this rank's device memory.
struct Spec {
  void* dst = nullptr;       // first destination byte
  size_t dst_pitch = 0;      // bytes between destination rows
  size_t src_pitch = 0;      // bytes of one full source row
  size_t src_total = 0;      // bytes of the whole source tensor
  size_t src_off = 0;        // byte offset of the first copied element
  size_t col_bytes = 0;      // bytes copied per row
  int rows = 0;              // rows per block
  int blocks = 1;            // expert blocks
  size_t dst_block = 0;      // destination stride between blocks
  size_t src_block = 0;      // source stride between blocks
  // generator description (init_random)
  int kind = 0;              // 0 quantized weight part, 1 norm vector
  int part = 0;              // 0 weight, 1 scales, 2 biases
  std::string base;          // generator stream name
  QW* q = nullptr;           // destination tensor
  int row0 = 0;              // first global row of the shard
  int col0 = 0;              // first global column of the shard
  int K_full = 0;            // full reduction length
  int n_rows = 0;            // shard rows (per block)
  int n_cols = 0;            // shard columns
  int dst_row0 = 0;          // first destination row inside q (per block)
  int dst_block_rows = 0;    // destination rows between blocks
  int src_block_rows = 0;    // source rows between blocks
  int gen_block0 = 0;        // first global block (expert)
  int norm_len = 0;
};

}  // namespace emx

using namespace emx;

// Decode steps emx_qwen3_decode_stream keeps in flight ahead of its callback.
constexpr int kStreamDepth = 8;

struct emx_qwen3 {
  emx_ctx* ctx = nullptr;
  emx_qwen3_config c{};
  emx_comm* comm = nullptr;
  int rank = 0, world = 1;
  bool moe = false, tp = false, ep = false;
  int nq = 0, nkv = 0, hd = 128, H = 0, I = 0, E_l = 0, e_base = 0, Im = 0, Nqkv = 0;
  std::vector<LayerW> L;
  QW embed, lm;
  bf16* final_norm = nullptr;
  float* inv_freq = nullptr;
  float2* rope_cs = nullptr;  // (cos, sin) per position and frequency
  PgemvPlan p_lm{};
  bool packed_ok = false;  // packed copies match the loaded weights
  bool compiled = true;    // decode through the captured graph (PDL chain) or eagerly
  bf16* kv = nullptr;
  size_t kv_layer = 0;  // elements of one layer's K (or V)
  std::map<std::string, Spec> specs;
  std::set<std::string> loaded;  // tensors written by load_tensor / init_random
  std::vector<void*> allocs;
  // decode buffers
  bf16 *xa = nullptr, *xb = nullptr, *qkvb = nullptr, *attnb = nullptr, *hb = nullptr, *logits = nullptr;
  bf16 *moe_y = nullptr, *router_logits = nullptr;
  float *part = nullptr, *moe_w = nullptr, *am_val = nullptr, *attn_part = nullptr;
  int *state = nullptr, *token = nullptr, *pos = nullptr, *hist_n = nullptr, *hist = nullptr, *am_idx = nullptr;
  int *moe_idx = nullptr, *moe_n = nullptr;
  unsigned *am_ticket = nullptr, *attn_ticket = nullptr;
  int attn_splits = 0;
  // prefill buffers
  bf16 *px = nullptr, *pxn = nullptr, *pqkv = nullptr, *pq = nullptr, *pattn = nullptr, *ph = nullptr;
  float* ppart = nullptr;
  int* pids = nullptr;
  int max_T = 0;
  // batched MoE prefill: routing [T][E] logits, [T][k] choices, grouped rows
  bf16 *p_rlog = nullptr, *p_xs = nullptr, *p_hs = nullptr, *p_ys = nullptr;
  int *p_idx = nullptr, *p_n = nullptr, *p_perm = nullptr, *p_src = nullptr, *p_cnt = nullptr;
  float* p_w = nullptr;
  int4* p_tiles = nullptr;
  int p_max_tiles = 0;
  // state
  int offset = 0;
  cudaGraphExec_t gexec = nullptr;
  int step_launches = 0;
  int32_t* pinned = nullptr;  // pinned host staging [kv_cap + 8]
  cudaEvent_t stream_ev[kStreamDepth] = {};  // decode_stream: one per step in flight
  int32_t* stream_st = nullptr;               // decode_stream: device status after each step in flight (pinned)
  // persistent decode step (dense model on one GPU)
  bool step_ok = false;    // the shape has a plan and it fits
  bool fused = false;      // decode through the persistent step kernel
  // device sampling (Qwen3Engine::set_sampling, crates/serve/src/engine.rs:230-233)
  bool sampling = false;   // temperature >= 1e-6: sample instead of the in-graph argmax
  float s_temp = 0.f, s_top_p = 1.f;
  int s_top_k = 0;
  unsigned long long* rng = nullptr;  // SimpleRng state
  float* samp = nullptr;              // [vocab] probabilities
  bool step_coop = true;   // launch it cooperatively
  StepPlan sp{};
  StepArgs sa{};
  uint64_t* step_words = nullptr;  // the persistent step's flag-word exchange buffers
  unsigned* step_ctl = nullptr;    // epoch, abort word
  size_t step_nwords = 0, step_nctl = 0;
  unsigned long long step_epochs = 0;  // persistent steps since the words were cleared
};

namespace {

#define Q_REQUIRE(cond, ...) \
  do {                       \
    if (!(cond)) return fail(EMX_ERR_INVALID, __VA_ARGS__); \
  } while (0)

int alloc(emx_qwen3* m, size_t bytes, void** p) {
  int rc = ctx_alloc(m->ctx, bytes, p);
  if (rc) return rc;
  m->allocs.push_back(*p);
  cudaMemsetAsync(*p, 0, bytes, m->ctx->stream);
  return EMX_OK;
}

template <typename T>
int alloc_t(emx_qwen3* m, size_t count, T** p) {
  void* v = nullptr;
  int rc = alloc(m, count * sizeof(T), &v);
  *p = static_cast<T*>(v);
  return rc;
}

int alloc_qw(emx_qwen3* m, QW& q, int N, int K, int bits, int gs) {
  q.N = N;
  q.K = K;
  q.bits = bits;
  q.gs = gs;
  int rc = alloc_t(m, q.wbytes() / 4, &q.w);
  if (!rc) rc = alloc_t(m, q.sbytes() / 2, &q.s);
  if (!rc) rc = alloc_t(m, q.sbytes() / 2, &q.b);
  return rc;
}

// Registers the three parts of a quantized checkpoint tensor `base`:
// full shape [blocks_full * rows_full_per_block, K_full]; this rank keeps rows
// [row0, row0 + n_rows) of every block in [block0, block0 + blocks) and
// columns [col0, col0 + n_cols), stored at destination row dst_row0 of each
// destination block of dst_block_rows rows in q.
void add_quant(emx_qwen3* m, const std::string& base, QW* q, int rows_full_per_block, int blocks_full, int K_full,
               int row0, int n_rows, int col0, int n_cols, int dst_row0, int block0, int blocks, int dst_block_rows) {
  const int per = 32 / q->bits;
  const int ng_full = K_full / q->gs;
  for (int part = 0; part < 3; ++part) {
    Spec s;
    s.kind = 0;
    s.part = part;
    s.base = base;
    s.q = q;
    s.row0 = row0;
    s.col0 = col0;
    s.K_full = K_full;
    s.n_rows = n_rows;
    s.n_cols = n_cols;
    s.dst_row0 = dst_row0;
    s.dst_block_rows = dst_block_rows;
    s.src_block_rows = rows_full_per_block;
    s.gen_block0 = block0;
    s.rows = n_rows;
    s.blocks = blocks;
    size_t src_row, dst_row, col_off, cols;
    if (part == 0) {
      src_row = (size_t)K_full / per * 4;
      dst_row = (size_t)q->K / per * 4;
      col_off = (size_t)col0 / per * 4;
      cols = (size_t)n_cols / per * 4;
    } else {
      src_row = (size_t)ng_full * 2;
      dst_row = (size_t)(q->K / q->gs) * 2;
      col_off = (size_t)(col0 / q->gs) * 2;
      cols = (size_t)(n_cols / q->gs) * 2;
    }
    char* dbase = part == 0 ? reinterpret_cast<char*>(q->w) : part == 1 ? reinterpret_cast<char*>(q->s)
                                                                         : reinterpret_cast<char*>(q->b);
    s.dst = dbase + (size_t)dst_row0 * dst_row;
    s.dst_pitch = dst_row;
    s.src_pitch = src_row;
    s.src_total = src_row * (size_t)rows_full_per_block * blocks_full;
    s.src_off = (size_t)block0 * rows_full_per_block * src_row + (size_t)row0 * src_row + col_off;
    s.col_bytes = cols;
    s.dst_block = (size_t)dst_block_rows * dst_row;
    s.src_block = (size_t)rows_full_per_block * src_row;
    static const char* sfx[3] = {".weight", ".scales", ".biases"};
    m->specs[base + sfx[part]] = s;
  }
}

void add_norm(emx_qwen3* m, const std::string& name, bf16* dst, int len) {
  Spec s;
  s.kind = 1;
  s.base = name;
  s.dst = dst;
  s.dst_pitch = s.src_pitch = s.col_bytes = (size_t)len * 2;
  s.src_total = (size_t)len * 2;
  s.rows = 1;
  s.norm_len = len;
  m->specs[name] = s;
}

GemvArgs gemv_base(const emx_qwen3* m, const QW& q) {
  GemvArgs a = {};
  a.w = reinterpret_cast<const uint32_t*>(q.pk);
  a.N = q.N;
  a.K = q.K;
  a.bits = q.bits;
  a.gs = q.gs;
  a.x_slots = 1;
  a.eps = m->c.eps;
  a.norm_groups = m->c.norm_groups;
  a.status = m->ctx->status;
  return a;
}

// Shared memory of a decode GEMV CTA: at least half an SM (228 KB, 1 KB
// reserved per CTA), so two GEMV CTAs never share an SM.  The block scheduler
// places a pending launch greedily: when a GEMV's CTAs fit two to an SM, the
// SMs that free up first take two of them and the others none, and the
// pattern repeats down the chain of launches (half the SMs doing twice the
// work).  With one GEMV CTA per SM the next GEMV takes each SM as this one
// leaves it, while decode attention (a 64 KB K/V ring plus up to 32 KB of
// partials) is still resident beside a GEMV and streams its tiles during it.
// The lm_head streams far more than it can hold and its dequant is the
// longest compute of the step: it runs two smaller CTAs per SM.
constexpr int kGemvSmem = 114 * 1024;
constexpr int kGemvBudgetPair = 94 * 1024;

// A GEMV between two GEMVs (gate|up, down) shares its SM with neither, so
// when half an SM leaves its stages short of the 8 tiles that keep each of
// the eight consumer warps on two units at a time (a large-K matrix whose x
// and row slots fill the budget), it may take up to kGemvSmemWide.
constexpr int kGemvSmemWide = 200 * 1024;
constexpr int kFullStageTiles = 8;

// norm: the launches use a norm prologue; widen: the GEMV may grow past
// half an SM (see above).
int plan(emx_qwen3* m, const QW& q, int epi, int x_slots, int n_rows_override, PgemvPlan* p, int ctas_per_sm = 1,
         bool norm = true, bool widen = false) {
  const int N = n_rows_override > 0 ? n_rows_override : q.N;
  const int budget = ctas_per_sm > 1 ? kGemvBudgetPair : kGemvSmem;
  if (pgemv_make_plan(N, q.K, q.bits, q.gs, epi, x_slots, m->ctx->num_sms, budget, p, ctas_per_sm, norm ? 1 : 0))
    return fail(EMX_ERR_INVALID, "no GEMV plan for N=%d K=%d bits=%d group=%d", N, q.K, q.bits, q.gs);
  const int spans = (q.K / q.gs + 7) / 8;
  const int cta_tiles = p->lbs_max * p->halves * spans;
  PgemvPlan wide;
  if (widen && ctas_per_sm == 1 && p->stage_tiles < std::min(kFullStageTiles, cta_tiles) &&
      pgemv_make_plan(N, q.K, q.bits, q.gs, epi, x_slots, m->ctx->num_sms, kGemvSmemWide, &wide, 1, norm ? 1 : 0) ==
          0 &&
      wide.stage_tiles > p->stage_tiles)
    *p = wide;
  if (ctas_per_sm == 1) p->smem = std::max(p->smem, kGemvSmem);
  return EMX_OK;
}

// Device memory for the packed copy of a decode matrix.
int alloc_packed(emx_qwen3* m, QW& q, int blocks, int R, int halves) {
  q.map = PackMap{blocks, R, halves};
  void* v = nullptr;
  int rc = alloc(m, pgemv_packed_bytes(q.N, q.K, q.bits, q.gs, q.map), &v);
  q.pk = static_cast<unsigned char*>(v);
  return rc;
}

int pack_one(emx_qwen3* m, QW& q) {
  if (!q.pk) return EMX_OK;
  cudaError_t e = pgemv_pack(q.w, q.s, q.b, q.N, q.K, q.bits, q.gs, q.map, q.pk, m->ctx->stream);
  return e == cudaSuccess ? EMX_OK : fail_cuda(e, "weight packing");
}

// Re-packs every decode matrix after weights changed (load / init_random).
int ensure_packed(emx_qwen3* m) {
  if (m->packed_ok) return EMX_OK;
  int rc;
  if ((rc = pack_one(m, m->c.tied ? m->embed : m->lm))) return rc;
  for (auto& lw : m->L) {
    if ((rc = pack_one(m, lw.qkv)) || (rc = pack_one(m, lw.o)) || (rc = pack_one(m, lw.gate_up)) ||
        (rc = pack_one(m, lw.down)) || (rc = pack_one(m, lw.router)) || (rc = pack_one(m, lw.e_gu)) ||
        (rc = pack_one(m, lw.e_down)))
      return rc;
  }
  m->packed_ok = true;
  return EMX_OK;
}

// The slice of checkpoint tensor `name` that rank `rank` of `world` keeps:
// o = {row0, n_rows, col0, n_cols, block0, blocks} over the tensor's logical
// [blocks x rows, cols] shape (cols = unpacked columns; quantized parts share
// the weight's slice).  Dense models shard by tensor parallelism: q/k/v rows
// by heads, gate/up rows by intermediate, o/down columns likewise; MoE models
// by expert parallelism: expert blocks.  Everything else is replicated.
// Returns 1 when the name is unknown.
int shard_rule(const emx_qwen3_config& c, int world, int rank, const std::string& name, int32_t o[6]) {
  const int hd = c.head_dim, H = c.hidden;
  const bool moe = c.n_experts > 0, tp = world > 1 && !moe, ep = world > 1 && moe;
  const int W = tp ? world : 1, r = tp ? rank : 0;
  auto set = [&](int row0, int nrows, int col0, int ncols, int b0, int nb) {
    o[0] = row0, o[1] = nrows, o[2] = col0, o[3] = ncols, o[4] = b0, o[5] = nb;
    return 0;
  };
  auto ends = [&](const char* suf) {
    const size_t n = strlen(suf);
    if (name.size() < n || name.compare(name.size() - n, n, suf) != 0) return false;
    return true;
  };
  std::string stem = name;
  for (const char* part : {".weight", ".scales", ".biases"})
    if (ends(part)) stem = name.substr(0, name.size() - strlen(part));
  auto is = [&](const char* suf) {
    const size_t n = strlen(suf);
    return stem.size() >= n && stem.compare(stem.size() - n, n, suf) == 0;
  };
  if (stem == "model.embed_tokens" || stem == "lm_head") return set(0, c.vocab, 0, H, 0, 1);
  if (stem == "model.norm" || is("input_layernorm") || is("post_attention_layernorm")) return set(0, 1, 0, H, 0, 1);
  if (is("self_attn.q_norm") || is("self_attn.k_norm")) return set(0, 1, 0, hd, 0, 1);
  if (is("self_attn.q_proj")) return set(r * (c.n_q / W) * hd, (c.n_q / W) * hd, 0, H, 0, 1);
  if (is("self_attn.k_proj") || is("self_attn.v_proj")) return set(r * (c.n_kv / W) * hd, (c.n_kv / W) * hd, 0, H, 0, 1);
  if (is("self_attn.o_proj")) return set(0, H, r * (c.n_q / W) * hd, (c.n_q / W) * hd, 0, 1);
  if (!moe && (is("mlp.gate_proj") || is("mlp.up_proj"))) return set(r * (c.inter / W), c.inter / W, 0, H, 0, 1);
  if (!moe && is("mlp.down_proj")) return set(0, H, r * (c.inter / W), c.inter / W, 0, 1);
  if (moe && is("mlp.gate")) return set(0, c.n_experts, 0, H, 0, 1);
  const int El = ep ? c.n_experts / world : c.n_experts, e0 = ep ? rank * El : 0;
  if (moe && (is("mlp.switch_mlp.gate_proj") || is("mlp.switch_mlp.up_proj"))) return set(0, c.moe_inter, 0, H, e0, El);
  if (moe && is("mlp.switch_mlp.down_proj")) return set(0, H, 0, c.moe_inter, e0, El);
  return 1;
}

// Shared memory of the persistent step's CTA (one per SM).
constexpr int kStepBudget1 = 227 * 1024;

// Zeroes the persistent step's exchange words and control block (epoch 0:
// no stale word can carry a flag of the steps to come).
int clear_step_words(emx_qwen3* m) {
  if (!m->step_words) return EMX_OK;
  EMX_CHECK_CUDA(cudaMemsetAsync(m->step_words, 0, m->step_nwords * sizeof(uint64_t), m->ctx->stream), "step words");
  EMX_CHECK_CUDA(cudaMemsetAsync(m->step_ctl, 0, m->step_nctl * sizeof(unsigned), m->ctx->stream), "step control");
  m->step_epochs = 0;
  return EMX_OK;
}

// Plans the persistent decode step when the model qualifies (one GPU, group
// size 64 everywhere, head_dim 128, 1/2/4/8 q heads per KV head, one norm
// group; dense, or MoE with up to 256 experts and top-16) and sets up its
// argument block and exchange words; it is then the default decode path
// (sampling still runs the per-kernel chain).
int setup_step(emx_qwen3* m) {
  const emx_qwen3_config& c = m->c;
  if (m->world > 1 || c.norm_groups != 1) return EMX_OK;
  const QW& lmw = c.tied ? m->embed : m->lm;
  const LayerW& l0 = m->L[0];
  const QW& gu0 = m->moe ? l0.e_gu : l0.gate_up;
  const QW& dn0 = m->moe ? l0.e_down : l0.down;
  if (l0.qkv.gs != 64 || l0.o.gs != 64 || gu0.gs != 64 || dn0.gs != 64 || lmw.gs != 64) return EMX_OK;
  if (m->moe && l0.router.gs != 64) return EMX_OK;
  StepShape sh{};
  sh.H = m->H;
  sh.I = m->I;
  sh.nq = m->nq;
  sh.nkv = m->nkv;
  sh.hd = m->hd;
  sh.vocab = c.vocab;
  sh.gs = 64;
  sh.layers = c.layers;
  sh.cap = c.kv_cap;
  const int bits[kStepMats] = {l0.qkv.bits, l0.o.bits, gu0.bits, dn0.bits, lmw.bits, m->moe ? l0.router.bits : 0};
  for (int i = 0; i < kStepMats; ++i) sh.bits[i] = bits[i];
  if (m->moe) {
    sh.n_experts = c.n_experts;
    sh.top_k = c.top_k;
    sh.moe_inter = m->Im;
    sh.norm_topk = c.norm_topk ? 1 : 0;
  }
  StepPlan p{};
  const int nsm = m->ctx->num_sms;
  if (step_make_plan(sh, nsm, kStepBudget1, &p) || step_occupancy(p) < 1) {
    cudaGetLastError();
    return EMX_OK;
  }
  int rc;
  StepLayer* d_layers = nullptr;
  size_t words[kStepBuffers];
  step_exchange_words(sh, words);
  size_t nw = 0;
  for (size_t w : words) nw += w;
  nw = (nw + 1) & ~(size_t)1;  // the partials start 16-byte aligned
  // exchange words, then the attention splits' partials (flag words too, so
  // the host's clearing covers them); epoch and abort word apart
  const size_t npart = (size_t)m->nkv * p.tmpl.max_splits * p.hpg * (m->hd + 2);
  const size_t ctl = 2;
  if ((rc = alloc_t(m, (size_t)c.layers, &d_layers)) || (rc = alloc_t(m, nw + npart, &m->step_words)) ||
      (rc = alloc_t(m, ctl, &m->step_ctl)))
    return rc;
  m->step_nwords = nw + npart;
  m->step_nctl = ctl;
  std::vector<StepLayer> hl(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const LayerW& lw = m->L[l];
    StepLayer& s = hl[l];
    s.w[0] = lw.qkv.pk;
    s.w[1] = lw.o.pk;
    s.w[2] = m->moe ? lw.e_gu.pk : lw.gate_up.pk;
    s.w[3] = m->moe ? lw.e_down.pk : lw.down.pk;
    s.router = m->moe ? lw.router.pk : nullptr;
    s.in_norm = lw.in_norm;
    s.post_norm = lw.post_norm;
    s.q_norm = lw.q_norm;
    s.k_norm = lw.k_norm;
    s.kc = m->kv + m->kv_layer * (2 * (size_t)l);
    s.vc = s.kc + m->kv_layer;
  }
  EMX_CHECK_CUDA(cudaMemcpyAsync(d_layers, hl.data(), sizeof(StepLayer) * hl.size(), cudaMemcpyHostToDevice,
                                 m->ctx->stream),
                 "step layer table");
  StepArgs a = p.tmpl;
  a.layers = d_layers;
  a.lm_w = lmw.pk;
  a.final_norm = m->final_norm;
  a.emb_w = m->embed.w;
  a.emb_s = m->embed.s;
  a.emb_b = m->embed.b;
  a.emb_bits = m->embed.bits;
  a.emb_gs = m->embed.gs;
  a.token = m->token;
  a.eps = c.eps;
  uint64_t* w = m->step_words;
  a.xw = w;
  a.qkvw = a.xw + words[0];
  a.attw = a.qkvw + words[1];
  a.xmw = a.attw + words[2];
  a.hw = a.xmw + words[3];
  a.rlw = a.hw + words[4];
  a.epoch = m->step_ctl;
  a.abort_word = m->step_ctl + 1;
  a.logits = m->logits;
  a.rope_cs = m->rope_cs;
  a.attn_pw = w + nw;
  a.pos = m->pos;
  a.hist = m->hist;
  a.hist_n = m->hist_n;
  a.hist_cap = c.kv_cap;
  a.am_val = m->am_val;
  a.am_idx = m->am_idx;
  a.am_ticket = m->am_ticket;
  a.status = m->ctx->status;
  m->sp = p;
  m->sa = a;
  if ((rc = clear_step_words(m))) return rc;
  EMX_CHECK_CUDA(cudaStreamSynchronize(m->ctx->stream), "step setup");
  m->step_ok = true;
  m->fused = true;
  return EMX_OK;
}

int build(emx_qwen3* m) {
  const emx_qwen3_config& c = m->c;
  const int W = m->world, r = m->rank;
  m->hd = c.head_dim;
  m->H = c.hidden;
  if (m->tp) {
    m->nq = c.n_q / W;
    m->nkv = c.n_kv / W;
    m->I = c.inter / W;
  } else {
    m->nq = c.n_q;
    m->nkv = c.n_kv;
    m->I = c.inter;
  }
  m->Nqkv = (m->nq + 2 * m->nkv) * m->hd;
  if (m->moe) {
    m->Im = c.moe_inter;
    m->E_l = m->ep ? c.n_experts / W : c.n_experts;
    m->e_base = m->ep ? r * m->E_l : 0;
  }
  const int H = m->H, hd = m->hd;
  int rc;
  m->L.resize(c.layers);
  // embedding / lm_head / final norm (replicated)
  if ((rc = alloc_qw(m, m->embed, c.vocab, H, c.embed_bits, c.embed_group))) return rc;
  add_quant(m, "model.embed_tokens", &m->embed, c.vocab, 1, H, 0, c.vocab, 0, H, 0, 0, 1, c.vocab);
  if (!c.tied) {
    if ((rc = alloc_qw(m, m->lm, c.vocab, H, c.lm_bits, c.lm_group))) return rc;
    add_quant(m, "lm_head", &m->lm, c.vocab, 1, H, 0, c.vocab, 0, H, 0, 0, 1, c.vocab);
  }
  if ((rc = alloc_packed(m, c.tied ? m->embed : m->lm, 1, c.vocab, 1))) return rc;
  if ((rc = alloc_t(m, H, &m->final_norm))) return rc;
  add_norm(m, "model.norm.weight", m->final_norm, H);
  for (int l = 0; l < c.layers; ++l) {
    LayerW& lw = m->L[l];
    const std::string p = "model.layers." + std::to_string(l) + ".";
    if ((rc = alloc_t(m, H, &lw.in_norm)) || (rc = alloc_t(m, H, &lw.post_norm)) ||
        (rc = alloc_t(m, hd, &lw.q_norm)) || (rc = alloc_t(m, hd, &lw.k_norm)))
      return rc;
    add_norm(m, p + "input_layernorm.weight", lw.in_norm, H);
    add_norm(m, p + "post_attention_layernorm.weight", lw.post_norm, H);
    add_norm(m, p + "self_attn.q_norm.weight", lw.q_norm, hd);
    add_norm(m, p + "self_attn.k_norm.weight", lw.k_norm, hd);
    // attention: q|k|v rows split by heads under TP
    if ((rc = alloc_qw(m, lw.qkv, m->Nqkv, H, c.attn_bits, c.attn_group))) return rc;
    const int qr0 = m->tp ? r * m->nq * hd : 0, kr0 = m->tp ? r * m->nkv * hd : 0;
    add_quant(m, p + "self_attn.q_proj", &lw.qkv, c.n_q * hd, 1, H, qr0, m->nq * hd, 0, H, 0, 0, 1, m->Nqkv);
    add_quant(m, p + "self_attn.k_proj", &lw.qkv, c.n_kv * hd, 1, H, kr0, m->nkv * hd, 0, H, m->nq * hd, 0, 1,
              m->Nqkv);
    add_quant(m, p + "self_attn.v_proj", &lw.qkv, c.n_kv * hd, 1, H, kr0, m->nkv * hd, 0, H,
              (m->nq + m->nkv) * hd, 0, 1, m->Nqkv);
    if ((rc = alloc_packed(m, lw.qkv, 1, m->Nqkv, 1))) return rc;
    if ((rc = alloc_qw(m, lw.o, H, m->nq * hd, c.attn_bits, c.attn_group))) return rc;
    if ((rc = alloc_packed(m, lw.o, 1, H, 1))) return rc;
    add_quant(m, p + "self_attn.o_proj", &lw.o, H, 1, c.n_q * hd, 0, H, qr0, m->nq * hd, 0, 0, 1, H);
    if (!m->moe) {
      if ((rc = alloc_qw(m, lw.gate_up, 2 * m->I, H, c.mlp_bits, c.mlp_group))) return rc;
      const int ir0 = m->tp ? r * m->I : 0;
      add_quant(m, p + "mlp.gate_proj", &lw.gate_up, c.inter, 1, H, ir0, m->I, 0, H, 0, 0, 1, 2 * m->I);
      add_quant(m, p + "mlp.up_proj", &lw.gate_up, c.inter, 1, H, ir0, m->I, 0, H, m->I, 0, 1, 2 * m->I);
      if ((rc = alloc_packed(m, lw.gate_up, 1, 2 * m->I, 2))) return rc;
      if ((rc = alloc_qw(m, lw.down, H, m->I, c.mlp_bits, c.mlp_group))) return rc;
      if ((rc = alloc_packed(m, lw.down, 1, H, 1))) return rc;
      add_quant(m, p + "mlp.down_proj", &lw.down, H, 1, c.inter, 0, H, ir0, m->I, 0, 0, 1, H);
    } else {
      const int E = c.n_experts, Im = m->Im;
      if ((rc = alloc_qw(m, lw.router, E, H, c.router_bits, c.router_group))) return rc;
      add_quant(m, p + "mlp.gate", &lw.router, E, 1, H, 0, E, 0, H, 0, 0, 1, E);
      if ((rc = alloc_packed(m, lw.router, 1, E, 1))) return rc;
      if ((rc = alloc_qw(m, lw.e_gu, m->E_l * 2 * Im, H, c.expert_bits, c.expert_group))) return rc;
      if ((rc = alloc_packed(m, lw.e_gu, m->E_l, 2 * Im, 2))) return rc;
      add_quant(m, p + "mlp.switch_mlp.gate_proj", &lw.e_gu, Im, E, H, 0, Im, 0, H, 0, m->e_base, m->E_l, 2 * Im);
      add_quant(m, p + "mlp.switch_mlp.up_proj", &lw.e_gu, Im, E, H, 0, Im, 0, H, Im, m->e_base, m->E_l, 2 * Im);
      if ((rc = alloc_qw(m, lw.e_down, m->E_l * H, Im, c.expert_bits, c.expert_group))) return rc;
      if ((rc = alloc_packed(m, lw.e_down, m->E_l, H, 1))) return rc;
      add_quant(m, p + "mlp.switch_mlp.down_proj", &lw.e_down, H, E, Im, 0, H, 0, Im, 0, m->e_base, m->E_l, H);
    }
    // launch plans
    if ((rc = plan(m, lw.qkv, kEpiStore, 1, 0, &lw.p_qkv))) return rc;
    if ((rc = plan(m, lw.o, m->tp ? kEpiF32 : kEpiResid, 1, 0, &lw.p_o, 1, false))) return rc;
    if (!m->moe) {
      if ((rc = plan(m, lw.gate_up, kEpiSwiglu, 1, 0, &lw.p_gu, 1, true, true))) return rc;
      if ((rc = plan(m, lw.down, m->tp ? kEpiF32 : kEpiResid, 1, 0, &lw.p_down, 1, false, true))) return rc;
    } else {
      if ((rc = plan(m, lw.router, kEpiStore, 1, 0, &lw.p_router))) return rc;
      if ((rc = plan(m, lw.e_gu, kEpiSwiglu, 1, c.top_k * 2 * m->Im, &lw.p_egu))) return rc;
      if ((rc = plan(m, lw.e_down, kEpiStore, c.top_k, c.top_k * H, &lw.p_edown, 1, false))) return rc;
    }
  }
  if ((rc = plan(m, c.tied ? m->embed : m->lm, kEpiArgmax, 1, 0, &m->p_lm, 2))) return rc;
  // rope table, KV cache, decode state
  if ((rc = alloc_t(m, hd / 2, &m->inv_freq))) return rc;
  if (k_rope_inv_freq(m->inv_freq, hd, c.rope_theta, m->ctx->stream) != cudaSuccess)
    return fail(EMX_ERR_CUDA, "rope table");
  if ((rc = alloc_t(m, (size_t)c.kv_cap * (hd / 2), &m->rope_cs))) return rc;
  if (rope_table_fill(m->rope_cs, m->inv_freq, c.kv_cap, hd / 2, m->ctx->stream) != cudaSuccess)
    return fail(EMX_ERR_CUDA, "rope table");
  m->kv_layer = (size_t)m->nkv * c.kv_cap * hd;
  if ((rc = alloc_t(m, m->kv_layer * 2 * c.layers, &m->kv))) return rc;
  if ((rc = alloc_t(m, H, &m->xa)) || (rc = alloc_t(m, H, &m->xb)) || (rc = alloc_t(m, m->Nqkv, &m->qkvb)) ||
      (rc = alloc_t(m, (size_t)m->nq * hd, &m->attnb)) || (rc = alloc_t(m, c.vocab, &m->logits)) ||
      (rc = alloc_t(m, H, &m->part)))
    return rc;
  const size_t hsz = m->moe ? (size_t)c.top_k * m->Im : (size_t)m->I;
  if ((rc = alloc_t(m, hsz, &m->hb))) return rc;
  if (m->moe) {
    if ((rc = alloc_t(m, (size_t)c.top_k * H, &m->moe_y)) || (rc = alloc_t(m, c.n_experts, &m->router_logits)) ||
        (rc = alloc_t(m, 64, &m->moe_w)) || (rc = alloc_t(m, 64, &m->moe_idx)) || (rc = alloc_t(m, 4, &m->moe_n)))
      return rc;
  }
  if ((rc = alloc_t(m, 64, &m->state))) return rc;
  if ((rc = alloc_t(m, 1, &m->rng)) || (rc = alloc_t(m, (size_t)c.vocab, &m->samp))) return rc;
  {
    const unsigned long long s0 = sample_rng_seed(42);  // SimpleRng::new(42), engine.rs:218
    EMX_CHECK_CUDA(cudaMemcpy(m->rng, &s0, sizeof(s0), cudaMemcpyHostToDevice), "sampler state");
  }
  m->token = m->state + 0;
  m->pos = m->state + 1;
  m->hist_n = m->state + 2;
  if ((rc = alloc_t(m, (size_t)c.kv_cap, &m->hist))) return rc;
  if ((rc = alloc_t(m, 1024, &m->am_val)) || (rc = alloc_t(m, 1024, &m->am_idx)) ||
      (rc = alloc_t(m, 16, &m->am_ticket)))
    return rc;
  m->attn_splits = attn_decode_splits(m->nkv, m->ctx->num_sms, m->nq / m->nkv);
  const int hpg = m->nq / m->nkv;
  if ((rc = alloc_t(m, (size_t)m->nkv * m->attn_splits * hpg * (hd + 2), &m->attn_part)) ||
      (rc = alloc_t(m, (size_t)m->nkv, &m->attn_ticket)))
    return rc;
  // prefill buffers
  m->max_T = c.max_prefill > 0 ? c.max_prefill : 1;
  const size_t T = (size_t)m->max_T;
  if ((rc = alloc_t(m, T * H, &m->px)) || (rc = alloc_t(m, T * H, &m->pxn)) ||
      (rc = alloc_t(m, T * m->Nqkv, &m->pqkv)) || (rc = alloc_t(m, T * m->nq * hd, &m->pq)) ||
      (rc = alloc_t(m, T * m->nq * hd, &m->pattn)) || (rc = alloc_t(m, T, &m->pids)))
    return rc;
  if (!m->moe && (rc = alloc_t(m, T * 2 * m->I, &m->ph))) return rc;
  if (m->moe) {
    const size_t P = T * c.top_k;  // (token, slot) pairs
    m->p_max_tiles = m->E_l + (int)((P + 127) / 128) + 1;
    if ((rc = alloc_t(m, T * c.n_experts, &m->p_rlog)) || (rc = alloc_t(m, P * H, &m->p_xs)) ||
        (rc = alloc_t(m, P * m->Im, &m->p_hs)) || (rc = alloc_t(m, P * H, &m->p_ys)) ||
        (rc = alloc_t(m, P, &m->p_idx)) || (rc = alloc_t(m, T, &m->p_n)) || (rc = alloc_t(m, P, &m->p_perm)) ||
        (rc = alloc_t(m, P, &m->p_src)) || (rc = alloc_t(m, 2, &m->p_cnt)) || (rc = alloc_t(m, P, &m->p_w)) ||
        (rc = alloc_t(m, (size_t)m->p_max_tiles, &m->p_tiles)))
      return rc;
  }
  if ((m->tp || m->ep) && (rc = alloc_t(m, T * H, &m->ppart))) return rc;
  if (cudaMallocHost(reinterpret_cast<void**>(&m->pinned), sizeof(int32_t) * ((size_t)c.kv_cap + 8)) != cudaSuccess)
    return fail(EMX_ERR_OOM, "pinned staging buffer");
  if ((rc = setup_step(m))) return rc;
  // every registered slice is the one the shard rule states
  for (const auto& kv : m->specs) {
    const Spec& sp = kv.second;
    int32_t o[6];
    if (shard_rule(c, m->world, m->rank, kv.first, o)) return fail(EMX_ERR_STATE, "no shard rule for '%s'", kv.first.c_str());
    const bool ok = sp.kind == 1 ? (o[3] == sp.norm_len)
                                 : (o[0] == sp.row0 && o[1] == sp.n_rows && o[2] == sp.col0 && o[3] == sp.n_cols &&
                                    o[4] == sp.gen_block0 && o[5] == sp.blocks);
    if (!ok) return fail(EMX_ERR_STATE, "shard rule disagrees with the layout of '%s'", kv.first.c_str());
  }
  return ctx_sync_check(m->ctx, "emx_qwen3_create");
}

// ------------------------------------------------------------ decode step

int launch_gemv(emx_qwen3* m, const GemvArgs& a, const PgemvPlan& p, bool pdl) {
  cudaError_t e = pgemv_launch(a, p, m->ctx->stream, pdl);
  if (e != cudaSuccess) return fail_cuda(e, "decode gemv launch");
  ++m->step_launches;
  return EMX_OK;
}

// sample_from_logits (crates/serve/src/sampler.rs:84-96) over the lm_head's
// logits, on the device; the token replaces the argmax in m->token.
int launch_sampler(emx_qwen3* m, int* hist, cudaStream_t st) {
  SampleArgs s = {};
  s.logits = m->logits;
  s.n = m->c.vocab;
  s.temperature = m->s_temp;
  s.top_p = m->s_top_p;
  s.top_k = m->s_top_k;
  s.rng = m->rng;
  s.scratch = m->samp;
  s.tok_out = m->token;
  s.hist = hist;
  s.hist_n = m->hist_n;
  s.hist_cap = m->c.kv_cap;
  const cudaError_t e = sample_launch(s, st);
  return e == cudaSuccess ? EMX_OK : fail_cuda(e, "sampler launch");
}

int enqueue_step(emx_qwen3* m) {
  const emx_qwen3_config& c = m->c;
  cudaStream_t st = m->ctx->stream;
  const bool pdl = m->compiled;  // the eager step is plain stream order
  m->step_launches = 0;
  if (m->fused && !m->sampling) {
    cudaError_t e = step_launch(m->sa, m->sp, st, m->step_coop);
    if (e != cudaSuccess) return fail_cuda(e, "decode step launch");
    m->step_launches = 1;
    return EMX_OK;
  }
  bf16* cur = m->xa;
  bf16* nxt = m->xb;
  bool pending_add = false;  // the previous block's output still has to be added to `cur`
  // tensor parallel: the o / down partials are summed through NVLink peer
  // memory inside the GEMVs (producer epilogue, consumer prologue) when the
  // communicator could map every rank's exchange region; else NCCL
  const PeerX* peer = (m->tp || m->ep) && m->H <= kPeerSlotFloats ? comm_peer(m->comm) : nullptr;
  auto set_add = [&](GemvArgs& a) {
    // the residual add of the previous block's sharded / expert output, fused here
    a.pro = kProAddNorm;
    a.x = cur;
    a.x_out = nxt;
    if (m->moe && !m->ep) {
      a.moe_y = m->moe_y;
      a.moe_w = m->moe_w;
      a.moe_n = m->moe_n;
    } else if (peer) {
      a.peer = peer;
      a.add_round = m->tp ? 1 : 0;  // a TP sum is the unsharded projection's bf16 output
    } else {
      a.add_f32 = m->part;
      a.add_round = m->tp ? 1 : 0;
    }
  };
  auto tp_sum = [&](GemvArgs& a) {  // a tensor-parallel partial producer
    a.epi = kEpiF32;
    if (peer) a.peer = peer;
    else a.yf = m->part;
  };
  int rc;
  for (int l = 0; l < c.layers; ++l) {
    LayerW& lw = m->L[l];
    bf16* kc = m->kv + m->kv_layer * (2 * (size_t)l);
    bf16* vc = kc + m->kv_layer;
    // ---- input norm + fused qkv projection
    {
      GemvArgs a = gemv_base(m, lw.qkv);
      if (l == 0) {
        a.pro = kProEmbedNorm;
        a.emb_w = m->embed.w;
        a.emb_s = m->embed.s;
        a.emb_b = m->embed.b;
        a.emb_bits = m->embed.bits;
        a.emb_gs = m->embed.gs;
        a.vocab = c.vocab;
        a.token = m->token;
        a.x_out = cur;
      } else if (pending_add) {
        set_add(a);
      } else {
        a.pro = kProNorm;
        a.x = cur;
      }
      a.norm_w = lw.in_norm;
      a.epi = kEpiStore;
      a.y = m->qkvb;
      if ((rc = launch_gemv(m, a, lw.p_qkv, pdl && m->step_launches > 0))) return rc;
      if (pending_add) {
        std::swap(cur, nxt);
        pending_add = false;
      }
    }
    // ---- attention (q/k norm, rope, KV write, flash-decode)
    {
      AttnDecodeArgs a = {};
      a.qkv = m->qkvb;
      a.q_norm = lw.q_norm;
      a.k_norm = lw.k_norm;
      a.eps = c.eps;
      a.inv_freq = m->inv_freq;
      a.rope_cs = m->rope_cs;
      a.kc = kc;
      a.vc = vc;
      a.cap = c.kv_cap;
      a.nq = m->nq;
      a.nkv = m->nkv;
      a.head_dim = m->hd;
      a.pos = m->pos;
      a.scale = 1.0f / sqrtf((float)m->hd);
      a.out = m->attnb;
      a.part = m->attn_part;
      a.ticket = m->attn_ticket;
      a.splits = m->attn_splits;
      a.status = m->ctx->status;
      a.defer_merge = 1;  // the o projection's prologue merges a few splits
      cudaError_t e = attn_decode_launch(a, st, pdl);
      if (e != cudaSuccess) return fail_cuda(e, "attention launch");
      ++m->step_launches;
    }
    // ---- o projection (+ residual, or fp32 partial + all-reduce under TP)
    {
      GemvArgs a = gemv_base(m, lw.o);
      a.pro = kProMerge;
      a.x = m->attnb;
      a.attn_part = m->attn_part;
      a.attn_pos = m->pos;
      a.attn_hpg = m->nq / m->nkv;
      a.attn_grid = m->attn_splits;
      if (m->tp) {
        tp_sum(a);
      } else {
        a.epi = kEpiResid;
        a.res = cur;
        a.y = cur;
      }
      if ((rc = launch_gemv(m, a, lw.p_o, pdl))) return rc;
      if (m->tp) {
        if (!peer && (rc = comm_all_reduce(m->comm, m->part, (size_t)m->H, EMX_F32, st))) return rc;
        pending_add = true;
      }
    }
    if (!m->moe) {
      GemvArgs a = gemv_base(m, lw.gate_up);
      if (pending_add) set_add(a);
      else {
        a.pro = kProNorm;
        a.x = cur;
      }
      a.norm_w = lw.post_norm;
      a.epi = kEpiSwiglu;
      a.y = m->hb;
      if ((rc = launch_gemv(m, a, lw.p_gu, pdl))) return rc;
      if (pending_add) {
        std::swap(cur, nxt);
        pending_add = false;
      }
      GemvArgs d = gemv_base(m, lw.down);
      d.pro = kProX;
      d.x = m->hb;
      if (m->tp) {
        tp_sum(d);
      } else {
        d.epi = kEpiResid;
        d.res = cur;
        d.y = cur;
      }
      if ((rc = launch_gemv(m, d, lw.p_down, pdl))) return rc;
      if (m->tp) {
        if (!peer && (rc = comm_all_reduce(m->comm, m->part, (size_t)m->H, EMX_F32, st))) return rc;
        pending_add = true;
      }
    } else {
      // router -> top-k -> gathered expert SwiGLU -> gathered expert down
      GemvArgs ra = gemv_base(m, lw.router);
      ra.pro = kProNorm;
      ra.x = cur;
      ra.norm_w = lw.post_norm;
      ra.epi = kEpiStore;
      ra.y = m->router_logits;
      if ((rc = launch_gemv(m, ra, lw.p_router, pdl))) return rc;
      cudaError_t e = k_moe_route(m->router_logits, c.n_experts, c.top_k, c.norm_topk, m->e_base, m->E_l,
                                  m->moe_idx, m->moe_w, m->moe_n, st, pdl);
      if (e != cudaSuccess) return fail_cuda(e, "moe route");
      ++m->step_launches;
      GemvArgs ga = gemv_base(m, lw.e_gu);
      ga.N = c.top_k * 2 * m->Im;
      ga.pro = kProNorm;
      ga.x = cur;
      ga.norm_w = lw.post_norm;
      ga.epi = kEpiSwiglu;
      ga.y = m->hb;
      ga.slot_expert = m->moe_idx;
      ga.n_slots = m->moe_n;
      ga.slot_rows = m->Im;
      if ((rc = launch_gemv(m, ga, lw.p_egu, pdl))) return rc;
      GemvArgs da = gemv_base(m, lw.e_down);
      da.N = c.top_k * m->H;
      da.pro = kProX;
      da.x = m->hb;
      da.x_slots = c.top_k;
      da.epi = kEpiStore;
      da.y = m->moe_y;
      da.slot_expert = m->moe_idx;
      da.n_slots = m->moe_n;
      da.slot_rows = m->H;
      if ((rc = launch_gemv(m, da, lw.p_edown, pdl))) return rc;
      if (m->ep && peer) {
        e = k_moe_combine_peer(m->moe_y, m->moe_w, m->moe_n, m->H, peer, st, pdl);
        if (e != cudaSuccess) return fail_cuda(e, "moe combine");
        ++m->step_launches;
      } else if (m->ep) {
        e = k_moe_combine(m->moe_y, m->moe_w, m->moe_n, m->H, m->part, st, pdl);
        if (e != cudaSuccess) return fail_cuda(e, "moe combine");
        ++m->step_launches;
        if ((rc = comm_all_reduce(m->comm, m->part, (size_t)m->H, EMX_F32, st))) return rc;
      }
      pending_add = true;
    }
  }
  // ---- final norm + lm_head + greedy argmax (token and offset stay on device)
  {
    const QW& lmw = c.tied ? m->embed : m->lm;
    GemvArgs a = gemv_base(m, lmw);
    if (pending_add) set_add(a);
    else {
      a.pro = kProNorm;
      a.x = cur;
    }
    a.norm_w = m->final_norm;
    a.epi = kEpiArgmax;
    a.y = m->logits;
    a.am_val = m->am_val;
    a.am_idx = m->am_idx;
    a.am_ticket = m->am_ticket;
    a.tok_out = m->token;
    a.hist = m->sampling ? nullptr : m->hist;  // the sampler records its own token
    a.hist_n = m->hist_n;
    a.hist_cap = c.kv_cap;
    a.pos = m->pos;
    a.pos_inc = 1;
    if ((rc = launch_gemv(m, a, m->p_lm, pdl))) return rc;
    if (m->sampling) {
      if ((rc = launch_sampler(m, m->hist, st))) return rc;
      ++m->step_launches;
    }
  }
  return EMX_OK;
}

int ensure_graph(emx_qwen3* m) {
  if (m->gexec) return EMX_OK;
  cudaStream_t st = m->ctx->stream;
  cudaGraph_t g = nullptr;
  EMX_CHECK_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed), "begin capture");
  int rc = enqueue_step(m);
  cudaError_t e = cudaStreamEndCapture(st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail_cuda(e, "end capture");
  e = cudaGraphInstantiate(&m->gexec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    m->gexec = nullptr;
    return fail_cuda(e, "graph instantiate");
  }
  return EMX_OK;
}

int run_steps(emx_qwen3* m, int n) {
  int rc = ensure_packed(m);
  if (rc) return rc;
  if (m->fused && !m->sampling) {
    // the step's flags are epoch * (layers + 1) + layer + 1 in 32 bits:
    // clear the words before the epoch could make a flag wrap
    const unsigned long long lim = 0xffffffffull / (unsigned long long)(m->c.layers + 1) - 2;
    if (m->step_epochs + (unsigned long long)n >= lim && (rc = clear_step_words(m))) return rc;
    m->step_epochs += (unsigned long long)n;
  }
  if (!m->compiled) {  // eager: the same kernels, launched one by one
    for (int i = 0; i < n; ++i)
      if ((rc = enqueue_step(m))) return rc;
    m->offset += n;
    return EMX_OK;
  }
  rc = ensure_graph(m);
  if (rc) return rc;
  for (int i = 0; i < n; ++i) EMX_CHECK_CUDA(cudaGraphLaunch(m->gexec, m->ctx->stream), "graph launch");
  m->offset += n;
  return EMX_OK;
}

// --------------------------------------------------------------- prefill

int gemm(emx_qwen3* m, const QW& q, const bf16* x, int T, int epi, bf16* y, const bf16* res, float* yf = nullptr) {
  GemmArgs g = {};
  g.yf = yf;
  g.x = x;
  g.w = q.w;
  g.s = q.s;
  g.b = q.b;
  g.M = T;
  g.N = q.N;
  g.K = q.K;
  g.bits = q.bits;
  g.gs = q.gs;
  g.epi = epi;
  g.y = y;
  g.res = res;
  if (q.map.blocks == 1) g.wp = q.pk;
  int rc = gemm_run(m->ctx->gemm, g, m->ctx->stream);
  if (rc) return fail(EMX_ERR_CUDA, "prefill gemm failed (%d)", rc);
  return EMX_OK;
}

// The MoE block of one layer over T prompt rows (pxn normalised, px the
// residual): routing of every row (crates/ops/src/moe.rs:103-166: softmax
// over the router logits, stable top-k, renormalised weights), the rows
// grouped by local expert, the experts' gate|up (SwiGLU) and down
// projections as two grouped tensor-core GEMMs over the packed expert tiles,
// then each row's weighted sum over its experts in slot order added to the
// residual — the arithmetic moe_forward_batch applies token by token
// (crates/ops/src/moe.rs:174-207).  Under expert parallelism the weighted
// sums are fp32 partials summed across ranks by one all-reduce per layer.
int moe_prefill(emx_qwen3* m, const LayerW& lw, int T) {
  const emx_qwen3_config& c = m->c;
  cudaStream_t st = m->ctx->stream;
  const int H = m->H, k = c.top_k, Im = m->Im, P = T * k;
  int rc;
  if ((rc = gemm(m, lw.router, m->pxn, T, kGemmStore, m->p_rlog, nullptr))) return rc;
  cudaError_t e = k_moe_route_batch(m->p_rlog, T, c.n_experts, k, c.norm_topk, m->e_base, m->E_l, m->p_idx, m->p_w,
                                    m->p_n, st);
  if (e != cudaSuccess) return fail_cuda(e, "prefill moe route");
  if ((e = k_moe_group(m->p_idx, m->p_n, T, k, m->E_l, 128, m->p_perm, m->p_src, m->p_tiles, m->p_cnt, m->p_cnt + 1,
                       st)) != cudaSuccess)
    return fail_cuda(e, "prefill moe grouping");
  if ((e = k_moe_gather(m->pxn, m->p_src, m->p_cnt + 1, P, H, m->p_xs, st)) != cudaSuccess)
    return fail_cuda(e, "prefill moe gather");
  auto grouped = [&](const QW& q, const bf16* x, int K, int N_out, int epi, bf16* y) -> int {
    TcGemmArgs t = {};
    t.x = x;
    t.M = P;
    t.N = N_out;
    t.K = K;
    t.epi = epi;
    t.y = y;
    t.status = m->ctx->status;
    t.bits = q.bits;
    t.wp = q.pk;
    t.S = (K / 64 + 7) / 8;
    t.nrb = q.map.R / 16;
    t.tiles = m->p_tiles;
    t.n_tiles = m->p_cnt;
    t.expert_stride = (size_t)t.nrb * t.S * pgemv_tile_bytes(q.bits, q.gs);
    if (q.gs != 64 || !tc_pgemm_supported(t)) return fail(EMX_ERR_INVALID, "prefill moe: unsupported expert shape");
    const cudaError_t ce = tc_pgemm_grouped_launch(t, m->p_max_tiles, st);
    return ce == cudaSuccess ? EMX_OK : fail_cuda(ce, "prefill moe experts");
  };
  if ((rc = grouped(lw.e_gu, m->p_xs, H, Im, kTcSwiglu, m->p_hs))) return rc;
  if ((rc = grouped(lw.e_down, m->p_hs, Im, H, kTcStore, m->p_ys))) return rc;
  if (m->ep) {
    if ((e = k_moe_combine_batch(m->px, m->p_ys, m->p_w, m->p_n, m->p_perm, T, k, H, m->ppart, st)) != cudaSuccess)
      return fail_cuda(e, "prefill moe combine");
    if ((rc = comm_all_reduce(m->comm, m->ppart, (size_t)T * H, EMX_F32, st))) return rc;
    if ((e = k_add_f32(m->px, m->ppart, (size_t)T * H, 0, st)) != cudaSuccess) return fail_cuda(e, "prefill residual");
  } else if ((e = k_moe_combine_batch(m->px, m->p_ys, m->p_w, m->p_n, m->p_perm, T, k, H, nullptr, st)) !=
             cudaSuccess) {
    return fail_cuda(e, "prefill moe combine");
  }
  return EMX_OK;
}

// One forward pass over T prompt rows at the current offset.  attend_cache:
// the rows also attend the cached rows before them (chunked prefill); else
// the chunk attends only itself, as Qwen3Engine::prefill does
// (crates/serve/src/forward_qwen3.rs:125-150: sdpa over the chunk's k/v).
int prefill_impl(emx_qwen3* m, const int32_t* ids_dev, int T, bool attend_cache = false) {
  const emx_qwen3_config& c = m->c;
  cudaStream_t st = m->ctx->stream;
  const int H = m->H, hd = m->hd;
  const int off = m->offset;
  int rc = ensure_packed(m);
  if (rc) return rc;
  cudaError_t e = k_embed(m->embed.w, m->embed.s, m->embed.b, ids_dev, T, H, m->embed.gs, m->embed.bits, c.vocab,
                          m->px, m->ctx->status, st);
  if (e != cudaSuccess) return fail_cuda(e, "prefill embed");
  for (int l = 0; l < c.layers; ++l) {
    LayerW& lw = m->L[l];
    bf16* kc = m->kv + m->kv_layer * (2 * (size_t)l);
    bf16* vc = kc + m->kv_layer;
    if ((e = k_rms_norm(m->px, lw.in_norm, m->pxn, T, H, c.eps, c.norm_groups, st)) != cudaSuccess)
      return fail_cuda(e, "prefill norm");
    if ((rc = gemm(m, lw.qkv, m->pxn, T, kGemmStore, m->pqkv, nullptr))) return rc;
    PrefillQkvArgs pa = {};
    pa.qkv = m->pqkv;
    pa.q_norm = lw.q_norm;
    pa.k_norm = lw.k_norm;
    pa.eps = c.eps;
    pa.inv_freq = m->inv_freq;
    pa.rope_cs = m->rope_cs;
    pa.T = T;
    pa.nq = m->nq;
    pa.nkv = m->nkv;
    pa.hd = hd;
    pa.offset = off;
    pa.q_out = m->pq;
    pa.kc = kc;
    pa.vc = vc;
    pa.cap = c.kv_cap;
    if ((e = k_prefill_qkv(pa, st)) != cudaSuccess) return fail_cuda(e, "prefill qkv post");
    AttnPrefillArgs aa = {};
    aa.q = m->pq;
    aa.kc = kc;
    aa.vc = vc;
    aa.cap = c.kv_cap;
    aa.offset = off;
    aa.T = T;
    aa.prefix = attend_cache ? off : 0;
    aa.nq = m->nq;
    aa.nkv = m->nkv;
    aa.head_dim = hd;
    aa.scale = 1.0f / sqrtf((float)hd);
    aa.out = m->pattn;
    aa.out_tnd = 1;
    if ((e = attn_prefill_launch(aa, st, m->ctx->status)) != cudaSuccess) return fail_cuda(e, "prefill attention");
    // row-split o_proj under TP: fp32 partials, sum over ranks, then the residual add
    auto row_parallel = [&](const QW& q, const bf16* x) -> int {
      if (!m->tp) return gemm(m, q, x, T, kGemmResid, m->px, m->px);
      int r2 = gemm(m, q, x, T, kGemmF32, nullptr, nullptr, m->ppart);
      if (r2) return r2;
      if ((r2 = comm_all_reduce(m->comm, m->ppart, (size_t)T * H, EMX_F32, st))) return r2;
      cudaError_t e2 = k_add_f32(m->px, m->ppart, (size_t)T * H, 1, st);
      return e2 == cudaSuccess ? EMX_OK : fail_cuda(e2, "prefill residual");
    };
    if ((rc = row_parallel(lw.o, m->pattn))) return rc;
    if ((e = k_rms_norm(m->px, lw.post_norm, m->pxn, T, H, c.eps, c.norm_groups, st)) != cudaSuccess)
      return fail_cuda(e, "prefill norm");
    if (!m->moe) {
      if ((rc = gemm(m, lw.gate_up, m->pxn, T, kGemmSwiglu, m->ph, nullptr))) return rc;
      if ((rc = row_parallel(lw.down, m->ph))) return rc;
    } else if ((rc = moe_prefill(m, lw, T))) {
      return rc;
    }
  }
  // final norm + lm_head on the last row, greedy token, offset += T
  const QW& lmw = c.tied ? m->embed : m->lm;
  GemvArgs a = gemv_base(m, lmw);
  a.pro = kProNorm;
  a.x = m->px + (size_t)(T - 1) * H;
  a.norm_w = m->final_norm;
  a.epi = kEpiArgmax;
  a.y = m->logits;
  a.am_val = m->am_val;
  a.am_idx = m->am_idx;
  a.am_ticket = m->am_ticket;
  a.tok_out = m->token;
  a.pos = m->pos;
  a.pos_inc = T;
  e = pgemv_launch(a, m->p_lm, st, false);
  if (e != cudaSuccess) return fail_cuda(e, "prefill lm_head");
  if (m->sampling) {
    const int rc = launch_sampler(m, nullptr, st);
    if (rc) return rc;
  }
  m->offset += T;
  return EMX_OK;
}

int init_random_impl(emx_qwen3* m, uint64_t seed) {
  cudaStream_t st = m->ctx->stream;
  for (auto& kv : m->specs) {
    const Spec& s = kv.second;
    const uint64_t stream = [&] {
      uint64_t h = 0xcbf29ce484222325ull;
      for (unsigned char ch : s.base) {
        h ^= ch;
        h *= 0x100000001b3ull;
      }
      return h;
    }();
    cudaError_t e = cudaSuccess;
    if (s.kind == 1) {
      e = k_fill_normal_bf16(seed, stream, (size_t)s.norm_len, 1.0f, 0.05f, static_cast<bf16*>(s.dst), st);
    } else {
      if (s.part != 0) continue;  // weight, scales and biases come from one generator pass
      QW* q = s.q;
      const int per = 32 / q->bits, ngl = q->K / q->gs;
      for (int b = 0; b < s.blocks; ++b) {
        const size_t dst_row = (size_t)b * s.dst_block_rows + s.dst_row0;
        const size_t gen_row0 = (size_t)(s.gen_block0 + b) * s.src_block_rows + s.row0;
        e = k_fill_quantized_shard(seed, stream, s.n_rows, s.n_cols, s.K_full, gen_row0, s.col0, q->gs, q->bits,
                                   0.02f, q->w + dst_row * (q->K / per), q->s + dst_row * ngl,
                                   q->b + dst_row * ngl, q->K, st);
        if (e != cudaSuccess) break;
      }
    }
    if (e != cudaSuccess) return fail_cuda(e, "init_random");
  }
  return ctx_sync_check(m->ctx, "emx_qwen3_init_random");
}

}  // namespace

extern "C" {

int emx_qwen3_create(emx_ctx* ctx, const emx_qwen3_config* cfg, emx_comm* comm, emx_qwen3** out) {
  Q_REQUIRE(ctx && cfg && out, "emx_qwen3_create: null argument");
  *out = nullptr;
  const emx_qwen3_config& c = *cfg;
  Q_REQUIRE(c.hidden > 0 && c.layers > 0 && c.n_q > 0 && c.n_kv > 0 && c.vocab > 0 && c.kv_cap > 0,
            "emx_qwen3_create: bad dimensions");
  Q_REQUIRE(c.head_dim == 128, "emx_qwen3_create: head_dim must be 128 (got %d)", c.head_dim);
  Q_REQUIRE(c.n_q % c.n_kv == 0 && (c.n_q / c.n_kv == 1 || c.n_q / c.n_kv == 2 || c.n_q / c.n_kv == 4 ||
                                    c.n_q / c.n_kv == 8),
            "emx_qwen3_create: n_q / n_kv must be 1, 2, 4 or 8");
  Q_REQUIRE(c.norm_groups >= 1 && c.hidden % c.norm_groups == 0, "emx_qwen3_create: norm_groups");
  Q_REQUIRE(c.n_experts == 0 || (c.top_k >= 1 && c.top_k <= 64 && c.top_k <= c.n_experts && c.moe_inter > 0),
            "emx_qwen3_create: MoE parameters");
  emx_qwen3* m = new emx_qwen3();
  m->ctx = ctx;
  m->c = c;
  m->comm = comm;
  m->moe = c.n_experts > 0;
  if (comm && comm->nranks > 1) {
    m->rank = comm->rank;
    m->world = comm->nranks;
    m->tp = !m->moe;
    m->ep = m->moe;
    if (m->tp && (c.n_q % m->world || c.n_kv % m->world || c.inter % m->world || (c.inter / m->world) % 64)) {
      delete m;
      return fail(EMX_ERR_INVALID, "emx_qwen3_create: heads / intermediate not divisible across %d ranks", m->world);
    }
    if (m->ep && c.n_experts % m->world) {
      delete m;
      return fail(EMX_ERR_INVALID, "emx_qwen3_create: %d experts not divisible across %d ranks", c.n_experts,
                  m->world);
    }
  }
  cudaSetDevice(ctx->device);
  int rc = build(m);
  if (rc) {
    emx_qwen3_destroy(m);
    return rc;
  }
  *out = m;
  return EMX_OK;
}

int emx_qwen3_destroy(emx_qwen3* m) {
  if (!m) return EMX_OK;
  cudaStreamSynchronize(m->ctx->stream);
  if (m->gexec) cudaGraphExecDestroy(m->gexec);
  for (void* p : m->allocs) ctx_free(m->ctx, p);
  if (m->pinned) cudaFreeHost(m->pinned);
  for (cudaEvent_t e : m->stream_ev)
    if (e) cudaEventDestroy(e);
  if (m->stream_st) cudaFreeHost(m->stream_st);
  delete m;
  return EMX_OK;
}

int emx_qwen3_load_tensor(emx_qwen3* m, const char* name, const void* host, size_t bytes) {
  Q_REQUIRE(m && name && host, "emx_qwen3_load_tensor: null argument");
  auto it = m->specs.find(name);
  Q_REQUIRE(it != m->specs.end(), "emx_qwen3_load_tensor: unknown tensor '%s'", name);
  const Spec& s = it->second;
  Q_REQUIRE(bytes == s.src_total, "emx_qwen3_load_tensor: '%s' has %zu bytes, expected %zu", name, bytes,
            s.src_total);
  m->packed_ok = false;
  const char* src = static_cast<const char*>(host);
  for (int b = 0; b < s.blocks; ++b) {
    EMX_CHECK_CUDA(cudaMemcpy2DAsync(static_cast<char*>(s.dst) + (size_t)b * s.dst_block, s.dst_pitch,
                                     src + s.src_off + (size_t)b * s.src_block, s.src_pitch, s.col_bytes, s.rows,
                                     cudaMemcpyHostToDevice, m->ctx->stream),
                   "emx_qwen3_load_tensor");
  }
  const int rc = ctx_sync_check(m->ctx, "emx_qwen3_load_tensor");
  if (rc == EMX_OK) m->loaded.insert(name);
  return rc;
}

namespace {

// Full (unsharded) MLX shape and dtype of a model tensor: quantized parts are
// uint32 codes [rows, K*bits/32] or bf16 scales / biases [rows, K/group]
// (expert tensors [experts, rows, cols]); norms bf16 [len].
void spec_shape(const std::string& name, const Spec& s, int64_t shape[3], int* ndim, int* dtype) {
  if (s.kind == 1) {
    *ndim = 1;
    shape[0] = s.norm_len;
    *dtype = EMX_BF16;
    return;
  }
  const int esz = s.part == 0 ? 4 : 2;
  const int64_t cols = (int64_t)(s.src_pitch / esz);
  const int64_t blocks_full = (int64_t)(s.src_total / (s.src_pitch * (size_t)s.src_block_rows));
  *dtype = s.part == 0 ? EMX_U32 : EMX_BF16;
  if (name.find(".switch_mlp.") != std::string::npos) {
    *ndim = 3;
    shape[0] = blocks_full;
    shape[1] = s.src_block_rows;
    shape[2] = cols;
  } else {
    *ndim = 2;
    shape[0] = (int64_t)s.src_block_rows * blocks_full;
    shape[1] = cols;
  }
}

const char* dtype_name(int dtype) { return dtype == EMX_U32 ? "U32" : "BF16"; }

// One checkpoint tensor (or one row range of a shipped fused one) into the
// model: its dtype and trailing dimensions must be the model's.
int load_checked(emx_qwen3* m, const std::string& name, const StTensor& t, const unsigned char* base,
                 uint64_t off, uint64_t bytes, int64_t rows) {
  const Spec& s = m->specs.at(name);
  int64_t shp[3];
  int nd, dt;
  spec_shape(name, s, shp, &nd, &dt);
  Q_REQUIRE(t.dtype == dtype_name(dt), "load_safetensors: '%s' is %s in the checkpoint, the model takes %s",
            t.name.c_str(), t.dtype.c_str(), dtype_name(dt));
  Q_REQUIRE((int)t.shape.size() == nd && t.shape.back() == shp[nd - 1] && (nd < 3 || t.shape[1] == shp[1]) &&
                (nd == 1 || rows == shp[0]),
            "load_safetensors: '%s' has a shape the model does not take (trailing dimension %lld, model %lld)",
            t.name.c_str(), (long long)t.shape.back(), (long long)shp[nd - 1]);
  return emx_qwen3_load_tensor(m, name.c_str(), base + off, (size_t)bytes);
}

// A shipped fused projection (the reference prefers them:
// crates/serve/src/loader/weights.rs:103-118, 166-175): `parts` row counts in
// concatenation order, each loaded under its separate name.
int load_fused(emx_qwen3* m, const StTensor& t, const unsigned char* base, const std::string& prefix,
               const std::string& suffix, const std::vector<std::pair<std::string, int64_t>>& parts) {
  int64_t total = 0;
  for (const auto& p : parts) total += p.second;
  Q_REQUIRE(t.shape.size() == 2 && t.shape[0] == total,
            "load_safetensors: fused '%s' has %lld rows, expected %lld", t.name.c_str(),
            t.shape.empty() ? 0LL : (long long)t.shape[0], (long long)total);
  const uint64_t row_bytes = total ? t.bytes / (uint64_t)total : 0;
  uint64_t off = t.offset;
  for (const auto& p : parts) {
    const std::string name = prefix + p.first + suffix;
    Q_REQUIRE(m->specs.count(name), "load_safetensors: fused '%s' has no part '%s' in this model", t.name.c_str(),
              name.c_str());
    StTensor part = t;
    part.shape[0] = p.second;
    const uint64_t bytes = row_bytes * (uint64_t)p.second;
    const int rc = load_checked(m, name, part, base, off, bytes, p.second);
    if (rc) return rc;
    off += bytes;
  }
  return EMX_OK;
}

bool is_dir(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

bool is_file(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

}  // namespace

int emx_qwen3_load_safetensors(emx_qwen3* m, const char* path, int* n_loaded) {
  Q_REQUIRE(m && path, "emx_qwen3_load_safetensors: null argument");
  // the files: a directory holds model_fused.safetensors (preferred, as
  // crates/serve/src/loader/weights.rs:21-41), model.safetensors, or the
  // shards a model.safetensors.index.json names; else `path` is one file
  std::vector<std::string> files;
  const std::string dir = path;
  if (is_dir(dir)) {
    const std::string fused = dir + "/model_fused.safetensors", plain = dir + "/model.safetensors",
                      index = dir + "/model.safetensors.index.json";
    if (is_file(fused)) {
      files.push_back(fused);
    } else if (is_file(plain)) {
      files.push_back(plain);
    } else if (is_file(index)) {
      std::vector<std::string> shards;
      int rc = st_index_files(index.c_str(), &shards);
      if (rc) return rc;
      for (const auto& f : shards) files.push_back(dir + "/" + f);
    } else {
      return fail(EMX_ERR_INVALID, "model.safetensors not found at %s", path);
    }
  } else {
    files.push_back(dir);
  }
  const emx_qwen3_config& c = m->c;
  const int hd = c.head_dim > 0 ? c.head_dim : 128;
  int count = 0;
  for (const auto& fpath : files) {
    StFile f;
    int rc = st_open(fpath.c_str(), &f);
    if (rc) return rc;
    for (const StTensor& t : f.tensors) {
      if (m->specs.count(t.name)) {
        rc = load_checked(m, t.name, t, f.base, t.offset, t.bytes, t.shape.empty() ? 0 : t.shape[0]);
        if (rc) return rc;
        ++count;
        continue;
      }
      // shipped fused projections: model.layers.i.self_attn.qkv_proj.* and
      // model.layers.i.mlp.gate_up_proj.*
      const size_t dot = t.name.rfind('.');
      const std::string stem = dot == std::string::npos ? t.name : t.name.substr(0, dot);
      const std::string suffix = dot == std::string::npos ? "" : t.name.substr(dot);
      const std::string kQkv = "self_attn.qkv_proj", kGu = "mlp.gate_up_proj";
      if (stem.size() > kQkv.size() && stem.compare(stem.size() - kQkv.size(), kQkv.size(), kQkv) == 0) {
        const std::string pre = stem.substr(0, stem.size() - kQkv.size()) + "self_attn.";
        rc = load_fused(m, t, f.base, pre, suffix,
                        {{"q_proj", (int64_t)c.n_q * hd}, {"k_proj", (int64_t)c.n_kv * hd}, {"v_proj", (int64_t)c.n_kv * hd}});
        if (rc) return rc;
        ++count;
        continue;
      }
      if (stem.size() > kGu.size() && stem.compare(stem.size() - kGu.size(), kGu.size(), kGu) == 0) {
        const std::string pre = stem.substr(0, stem.size() - kGu.size()) + "mlp.";
        rc = load_fused(m, t, f.base, pre, suffix, {{"gate_proj", (int64_t)c.inter}, {"up_proj", (int64_t)c.inter}});
        if (rc) return rc;
        ++count;
        continue;
      }
      // a separate lm_head makes the model untied (weights.rs:113-127); a
      // model created tied cannot take one
      Q_REQUIRE(t.name.rfind("lm_head.", 0) != 0,
                "load_safetensors: the checkpoint has '%s' but the model was created with tied embeddings",
                t.name.c_str());
      // anything else is not on this path (the reference loads it and never
      // looks it up)
    }
  }
  // every tensor the model takes must have come from some file
  for (const auto& kv : m->specs)
    Q_REQUIRE(m->loaded.count(kv.first), "load_safetensors: missing %s", kv.first.c_str());
  if (n_loaded) *n_loaded = count;
  return EMX_OK;
}

int emx_qwen3_tensor_names(emx_qwen3* m, char* buf, size_t cap, size_t* need) {
  Q_REQUIRE(m && need, "emx_qwen3_tensor_names: null argument");
  std::string all;
  for (const auto& kv : m->specs) {
    all += kv.first;
    all += '\n';
  }
  *need = all.size() + 1;
  if (buf && cap > 0) {
    const size_t n = std::min(cap - 1, all.size());
    std::memcpy(buf, all.data(), n);
    buf[n] = 0;
  }
  return EMX_OK;
}

int emx_qwen3_tensor_shape(emx_qwen3* m, const char* name, int64_t* shape3, int* ndim, int* dtype) {
  Q_REQUIRE(m && name && shape3 && ndim && dtype, "emx_qwen3_tensor_shape: null argument");
  auto it = m->specs.find(name);
  Q_REQUIRE(it != m->specs.end(), "emx_qwen3_tensor_shape: unknown tensor '%s'", name);
  spec_shape(it->first, it->second, shape3, ndim, dtype);
  return EMX_OK;
}

int emx_qwen3_read_tensor(emx_qwen3* m, const char* name, void* host, size_t bytes) {
  Q_REQUIRE(m && name && host, "emx_qwen3_read_tensor: null argument");
  auto it = m->specs.find(name);
  Q_REQUIRE(it != m->specs.end(), "emx_qwen3_read_tensor: unknown tensor '%s'", name);
  const Spec& s = it->second;
  const size_t need = s.col_bytes * s.rows * s.blocks;
  Q_REQUIRE(bytes == need, "emx_qwen3_read_tensor: '%s' shard has %zu bytes, got %zu", name, need, bytes);
  char* dst = static_cast<char*>(host);
  for (int b = 0; b < s.blocks; ++b) {
    EMX_CHECK_CUDA(cudaMemcpy2DAsync(dst + (size_t)b * s.col_bytes * s.rows, s.col_bytes,
                                     static_cast<const char*>(s.dst) + (size_t)b * s.dst_block, s.dst_pitch,
                                     s.col_bytes, s.rows, cudaMemcpyDeviceToHost, m->ctx->stream),
                   "emx_qwen3_read_tensor");
  }
  return ctx_sync_check(m->ctx, "emx_qwen3_read_tensor");
}

int emx_qwen3_read_kv(emx_qwen3* m, int layer, int which, void* host, size_t bytes) {
  Q_REQUIRE(m && host, "emx_qwen3_read_kv: null argument");
  Q_REQUIRE(layer >= 0 && layer < m->c.layers && (which == 0 || which == 1),
            "emx_qwen3_read_kv: layer %d / which %d out of range", layer, which);
  const size_t need = m->kv_layer * sizeof(bf16);
  Q_REQUIRE(bytes == need, "emx_qwen3_read_kv: cache slab has %zu bytes, got %zu", need, bytes);
  const bf16* src = m->kv + m->kv_layer * (2 * (size_t)layer + which);
  EMX_CHECK_CUDA(cudaMemcpyAsync(host, src, need, cudaMemcpyDeviceToHost, m->ctx->stream), "emx_qwen3_read_kv");
  return ctx_sync_check(m->ctx, "emx_qwen3_read_kv");
}

int emx_qwen3_init_random(emx_qwen3* m, uint64_t seed) {
  Q_REQUIRE(m, "emx_qwen3_init_random: null model");
  m->packed_ok = false;
  const int rc = init_random_impl(m, seed);
  if (rc == EMX_OK)
    for (const auto& kv : m->specs) m->loaded.insert(kv.first);
  return rc;
}

int emx_qwen3_reset(emx_qwen3* m) {
  Q_REQUIRE(m, "emx_qwen3_reset: null model");
  m->offset = 0;
  EMX_CHECK_CUDA(cudaMemsetAsync(m->state, 0, sizeof(int) * 64, m->ctx->stream), "reset");
  // last-CTA tickets back to zero (a chain that gave up on a wait may have
  // left one part-way)
  EMX_CHECK_CUDA(cudaMemsetAsync(m->am_ticket, 0, sizeof(unsigned) * 16, m->ctx->stream), "reset");
  EMX_CHECK_CUDA(cudaMemsetAsync(m->attn_ticket, 0, sizeof(unsigned) * m->nkv, m->ctx->stream), "reset");
  const int rc = clear_step_words(m);  // also ends a persistent step that gave up on a wait
  if (rc) return rc;
  return ctx_sync_check(m->ctx, "emx_qwen3_reset");
}

int emx_qwen3_offset(emx_qwen3* m, int* offset) {
  Q_REQUIRE(m && offset, "emx_qwen3_offset: null argument");
  *offset = m->offset;
  return EMX_OK;
}

int emx_qwen3_prefill_device(emx_qwen3* m, const int32_t* ids, int T) {
  Q_REQUIRE(m && ids, "emx_qwen3_prefill: null argument");
  Q_REQUIRE(T >= 1 && T <= m->max_T, "emx_qwen3_prefill: T=%d outside [1, max_prefill=%d]", T, m->max_T);
  if (m->offset + T > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d + T=%d > cap=%d", m->offset, T, m->c.kv_cap);
  return prefill_impl(m, ids, T);
}

int emx_qwen3_prefill(emx_qwen3* m, const int32_t* tokens, int T, int32_t* next_token, void* logits) {
  Q_REQUIRE(m && tokens, "emx_qwen3_prefill: null argument");
  Q_REQUIRE(T >= 1 && T <= m->max_T, "emx_qwen3_prefill: T=%d outside [1, max_prefill=%d]", T, m->max_T);
  if (m->offset + T > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d + T=%d > cap=%d", m->offset, T, m->c.kv_cap);
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->pids, tokens, sizeof(int32_t) * T, cudaMemcpyHostToDevice, m->ctx->stream),
                 "prefill ids");
  int rc = prefill_impl(m, m->pids, T);
  if (rc) return rc;
  if (logits)
    EMX_CHECK_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)m->c.vocab * 2, cudaMemcpyDeviceToHost, m->ctx->stream),
                   "prefill logits");
  if (next_token)
    EMX_CHECK_CUDA(cudaMemcpyAsync(m->pinned, m->token, sizeof(int32_t), cudaMemcpyDeviceToHost, m->ctx->stream),
                   "prefill token");
  rc = ctx_sync_check(m->ctx, "emx_qwen3_prefill");
  if (rc) return rc;
  if (next_token) *next_token = m->pinned[0];
  return EMX_OK;
}

int emx_qwen3_prefill_chunked(emx_qwen3* m, const int32_t* tokens, int T, int chunk, int32_t* next_token,
                              void* logits) {
  Q_REQUIRE(m && tokens, "emx_qwen3_prefill_chunked: null argument");
  Q_REQUIRE(T >= 1 && chunk >= 1, "emx_qwen3_prefill_chunked: T=%d / chunk=%d must be positive", T, chunk);
  if (m->offset + T > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d + T=%d > cap=%d", m->offset, T, m->c.kv_cap);
  const int step = std::min(chunk, m->max_T);
  for (int t0 = 0; t0 < T; t0 += step) {  // make_chunks (crates/prefill/src/chunked_prefill.rs:18-20)
    const int n = std::min(step, T - t0);
    EMX_CHECK_CUDA(cudaMemcpyAsync(m->pids, tokens + t0, sizeof(int32_t) * n, cudaMemcpyHostToDevice,
                                   m->ctx->stream),
                   "prefill ids");
    const int rc = prefill_impl(m, m->pids, n, true);
    if (rc) return rc;
  }
  if (logits)
    EMX_CHECK_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)m->c.vocab * 2, cudaMemcpyDeviceToHost, m->ctx->stream),
                   "prefill logits");
  if (next_token)
    EMX_CHECK_CUDA(cudaMemcpyAsync(m->pinned, m->token, sizeof(int32_t), cudaMemcpyDeviceToHost, m->ctx->stream),
                   "prefill token");
  const int rc = ctx_sync_check(m->ctx, "emx_qwen3_prefill_chunked");
  if (rc) return rc;
  if (next_token) *next_token = m->pinned[0];
  return EMX_OK;
}

int emx_qwen3_decode_step(emx_qwen3* m, int32_t token, int32_t* next_token, void* logits) {
  Q_REQUIRE(m, "emx_qwen3_decode_step: null model");
  Q_REQUIRE(token >= 0 && token < m->c.vocab, "emx_qwen3_decode_step: token %d outside [0, %d)", token, m->c.vocab);
  if (m->offset + 1 > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d cap=%d", m->offset, m->c.kv_cap);
  m->pinned[0] = token;
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->token, m->pinned, sizeof(int32_t), cudaMemcpyHostToDevice, m->ctx->stream),
                 "decode token");
  int rc = run_steps(m, 1);
  if (rc) return rc;
  if (logits)
    EMX_CHECK_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)m->c.vocab * 2, cudaMemcpyDeviceToHost, m->ctx->stream),
                   "decode logits");
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->pinned + 1, m->token, sizeof(int32_t), cudaMemcpyDeviceToHost, m->ctx->stream),
                 "decode next token");
  rc = ctx_sync_check(m->ctx, "emx_qwen3_decode_step");
  if (rc) return rc;
  if (next_token) *next_token = m->pinned[1];
  return EMX_OK;
}

int emx_qwen3_decode(emx_qwen3* m, int32_t token, int n, int32_t* tokens_out) {
  Q_REQUIRE(m && tokens_out, "emx_qwen3_decode: null argument");
  Q_REQUIRE(n >= 1, "emx_qwen3_decode: n=%d", n);
  Q_REQUIRE(token >= 0 && token < m->c.vocab, "emx_qwen3_decode: token %d outside [0, %d)", token, m->c.vocab);
  if (m->offset + n > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d + n=%d > cap=%d", m->offset, n, m->c.kv_cap);
  m->pinned[0] = token;
  m->pinned[1] = 0;
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->token, m->pinned, sizeof(int32_t), cudaMemcpyHostToDevice, m->ctx->stream),
                 "decode token");
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->hist_n, m->pinned + 1, sizeof(int32_t), cudaMemcpyHostToDevice, m->ctx->stream),
                 "decode history");
  int rc = run_steps(m, n);
  if (rc) return rc;
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->pinned, m->hist, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, m->ctx->stream),
                 "decode tokens");
  rc = ctx_sync_check(m->ctx, "emx_qwen3_decode");
  if (rc) return rc;
  memcpy(tokens_out, m->pinned, sizeof(int32_t) * n);
  return EMX_OK;
}

int emx_qwen3_decode_stream(emx_qwen3* m, int32_t token, int n, emx_token_cb cb, void* user, int* n_done) {
  Q_REQUIRE(m && cb, "emx_qwen3_decode_stream: null argument");
  Q_REQUIRE(n >= 1, "emx_qwen3_decode_stream: n=%d", n);
  Q_REQUIRE(token >= 0 && token < m->c.vocab, "emx_qwen3_decode_stream: token %d outside [0, %d)", token,
            m->c.vocab);
  if (n_done) *n_done = 0;
  if (m->offset + n > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d + n=%d > cap=%d", m->offset, n, m->c.kv_cap);
  cudaStream_t st = m->ctx->stream;
  // steps in flight ahead of the callback: greedy decoding runs ahead (the
  // steps past a stop are rolled back below); sampling runs one step at a
  // time so the generator state never holds a discarded draw
  const int depth = m->sampling ? 1 : kStreamDepth;
  if (!m->stream_ev[0]) {
    for (int i = 0; i < kStreamDepth; ++i)
      EMX_CHECK_CUDA(cudaEventCreateWithFlags(&m->stream_ev[i], cudaEventDisableTiming), "stream events");
    if (cudaMallocHost(reinterpret_cast<void**>(&m->stream_st), sizeof(int32_t) * kStreamDepth) != cudaSuccess)
      return fail(EMX_ERR_OOM, "stream status buffer");
  }
  const int offset0 = m->offset;
  m->pinned[0] = token;
  m->pinned[1] = 0;
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->token, m->pinned, sizeof(int32_t), cudaMemcpyHostToDevice, st), "stream token");
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->hist_n, m->pinned + 1, sizeof(int32_t), cudaMemcpyHostToDevice, st),
                 "stream history");
  int32_t* out = m->pinned + 4;  // token of step i at out[i] (pinned holds kv_cap + 8 ints)
  int issued = 0, done = 0, rc = EMX_OK;
  bool stop = false;
  while (done < n && !stop) {
    // keep `depth` steps in flight: each one's token and the device status
    // are copied to pinned memory behind an event
    while (issued < n && issued - done < depth) {
      if ((rc = run_steps(m, 1))) break;
      cudaError_t e = cudaMemcpyAsync(out + issued, m->token, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->stream_st + issued % kStreamDepth, m->ctx->status, sizeof(int32_t),
                            cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess) e = cudaEventRecord(m->stream_ev[issued % kStreamDepth], st);
      if (e != cudaSuccess) {
        rc = fail_cuda(e, "stream step");
        break;
      }
      ++issued;
    }
    if (rc) break;
    const cudaError_t e = cudaEventSynchronize(m->stream_ev[done % kStreamDepth]);
    if (e != cudaSuccess) {
      rc = fail_cuda(e, "stream wait");
      break;
    }
    if (m->stream_st[done % kStreamDepth] != 0) {  // a device error: report it with the stream drained
      rc = ctx_sync_check(m->ctx, "emx_qwen3_decode_stream");
      if (!rc) rc = fail(EMX_ERR_DEVICE, "emx_qwen3_decode_stream: device status %d", m->stream_st[done % kStreamDepth]);
      break;
    }
    const int32_t t = out[done];
    ++done;
    if (n_done) *n_done = done;
    if (cb(t, done - 1, user) != 0) stop = true;
  }
  if (rc) return rc;
  if (issued > done) {
    // the callback stopped early: the steps run past it are discarded
    // (their K/V rows lie beyond the offset and are overwritten later)
    EMX_CHECK_CUDA(cudaStreamSynchronize(st), "stream drain");
    m->offset = offset0 + done;
    m->pinned[0] = out[done - 1];
    m->pinned[1] = offset0 + done;
    m->pinned[2] = done;
    EMX_CHECK_CUDA(cudaMemcpyAsync(m->state, m->pinned, 3 * sizeof(int32_t), cudaMemcpyHostToDevice, st),
                   "stream rollback");
    return ctx_sync_check(m->ctx, "emx_qwen3_decode_stream");
  }
  return EMX_OK;
}

int emx_qwen3_decode_device(emx_qwen3* m, int n) {
  Q_REQUIRE(m && n >= 0, "emx_qwen3_decode_device: bad argument");
  if (m->offset + n > m->c.kv_cap)
    return fail(EMX_ERR_STATE, "static KV overflow offset=%d + n=%d > cap=%d", m->offset, n, m->c.kv_cap);
  return run_steps(m, n);
}

int emx_qwen3_shard(const emx_qwen3_config* cfg, int world, int rank, const char* name, int32_t* out6) {
  Q_REQUIRE(cfg && name && out6, "emx_qwen3_shard: null argument");
  Q_REQUIRE(world >= 1 && rank >= 0 && rank < world, "emx_qwen3_shard: rank %d of %d", rank, world);
  if (world > 1) {
    const bool moe = cfg->n_experts > 0;
    Q_REQUIRE(moe ? cfg->n_experts % world == 0
                  : (cfg->n_q % world == 0 && cfg->n_kv % world == 0 && cfg->inter % world == 0),
              "emx_qwen3_shard: not divisible across %d ranks", world);
  }
  Q_REQUIRE(shard_rule(*cfg, world, rank, name, out6) == 0, "emx_qwen3_shard: unknown tensor '%s'", name);
  return EMX_OK;
}

int emx_qwen3_set_compiled(emx_qwen3* m, int compiled) {
  Q_REQUIRE(m, "emx_qwen3_set_compiled: null model");
  m->compiled = compiled != 0;
  return EMX_OK;
}

int emx_qwen3_is_compiled(emx_qwen3* m, int* compiled) {
  Q_REQUIRE(m && compiled, "emx_qwen3_is_compiled: null argument");
  *compiled = m->compiled ? 1 : 0;
  return EMX_OK;
}

int emx_qwen3_set_fused(emx_qwen3* m, int fused) {
  Q_REQUIRE(m, "emx_qwen3_set_fused: null model");
  Q_REQUIRE(!fused || m->step_ok, "emx_qwen3_set_fused: this model has no persistent step (sharded or shape)");
  if (m->fused != (fused != 0) && m->gexec) {
    cudaGraphExecDestroy(m->gexec);
    m->gexec = nullptr;
  }
  m->fused = fused != 0;
  return EMX_OK;
}

int emx_qwen3_set_sampling(emx_qwen3* m, float temperature, float top_p, int top_k, uint64_t seed) {
  Q_REQUIRE(m, "emx_qwen3_set_sampling: null model");
  Q_REQUIRE(std::isfinite(temperature) && temperature >= 0.f && std::isfinite(top_p) && top_k >= 0,
            "emx_qwen3_set_sampling: temperature %g / top_p %g / top_k %d out of range", temperature, top_p, top_k);
  m->sampling = temperature >= 1e-6f;  // below: greedy, the in-graph argmax
  m->s_temp = temperature;
  m->s_top_p = std::min(1.f, std::max(0.f, top_p));  // SamplingParams::with_top_p clamps
  m->s_top_k = top_k;
  const unsigned long long s0 = sample_rng_seed(seed);
  EMX_CHECK_CUDA(cudaMemcpyAsync(m->rng, &s0, sizeof(s0), cudaMemcpyHostToDevice, m->ctx->stream),
                 "emx_qwen3_set_sampling");
  if (m->gexec) {  // the parameters are part of the captured step
    cudaGraphExecDestroy(m->gexec);
    m->gexec = nullptr;
  }
  return ctx_sync_check(m->ctx, "emx_qwen3_set_sampling");
}

int emx_qwen3_is_fused(emx_qwen3* m, int* fused) {
  Q_REQUIRE(m && fused, "emx_qwen3_is_fused: null argument");
  *fused = m->fused ? 1 : 0;
  return EMX_OK;
}

int emx_qwen3_step_launches(emx_qwen3* m, int* n) {
  Q_REQUIRE(m && n, "emx_qwen3_step_launches: null argument");
  int rc = ensure_graph(m);
  if (rc) return rc;
  *n = m->step_launches;
  return EMX_OK;
}

}  // extern "C"
