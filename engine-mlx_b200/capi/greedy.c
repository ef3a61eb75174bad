/* greedy.c — a plain C caller of libemx through include/emx.h alone: the
 * calls a non-Python host (the engine's Rust crate, a C++ server) makes for a
 * Qwen3 greedy completion.  It creates a context and a model of the shape
 * given on the command line, fills it with the seeded synthetic weights,
 * prefills a deterministic prompt, decodes n greedy tokens with
 * emx_qwen3_decode, decodes them again through the per-token streaming entry
 * point after a reset, and prints both sequences as one line each:
 *
 *   greedy hidden layers n_q n_kv inter vocab attn_bits seed prompt_len n
 *
 * prints "decode t0 t1 ..." and "stream t0 t1 ...", exit status 0 on success.
 * The prompt is token i = (i * 37 + 5) mod vocab. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "emx.h"

static int collect(int32_t token, int index, void* user) {
  ((int32_t*)user)[index] = token;
  return 0;
}

#define CHECK(call)                                                   \
  do {                                                                \
    if ((call) != EMX_OK) {                                           \
      fprintf(stderr, "%s failed: %s\n", #call, emx_last_error());  \
      return 1;                                                       \
    }                                                                 \
  } while (0)

int main(int argc, char** argv) {
  if (argc != 11) {
    fprintf(stderr, "usage: %s hidden layers n_q n_kv inter vocab attn_bits seed prompt_len n\n", argv[0]);
    return 2;
  }
  emx_qwen3_config c;
  memset(&c, 0, sizeof(c));
  c.hidden = atoi(argv[1]);
  c.layers = atoi(argv[2]);
  c.n_q = atoi(argv[3]);
  c.n_kv = atoi(argv[4]);
  c.inter = atoi(argv[5]);
  c.vocab = atoi(argv[6]);
  c.head_dim = 128;
  c.eps = 1e-6f;
  c.rope_theta = 1e6f;
  c.tied = 1;
  c.norm_groups = 1;
  c.attn_bits = atoi(argv[7]);
  c.attn_group = 64;
  c.mlp_bits = 4;
  c.mlp_group = 64;
  c.embed_bits = 4;
  c.embed_group = 64;
  c.lm_bits = 4;
  c.lm_group = 64;
  c.router_bits = 4;
  c.router_group = 64;
  c.expert_bits = 4;
  c.expert_group = 64;
  const unsigned long long seed = strtoull(argv[8], NULL, 10);
  const int T = atoi(argv[9]);
  const int n = atoi(argv[10]);
  c.kv_cap = T + n + 8;
  c.max_prefill = T;

  emx_ctx* ctx = NULL;
  emx_qwen3* m = NULL;
  CHECK(emx_ctx_create(0, &ctx));
  CHECK(emx_qwen3_create(ctx, &c, NULL, &m));
  CHECK(emx_qwen3_init_random(m, seed));
  int32_t* prompt = (int32_t*)malloc(sizeof(int32_t) * (size_t)T);
  int32_t* toks = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  int32_t* streamed = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  for (int i = 0; i < T; ++i) prompt[i] = (int32_t)((i * 37 + 5) % c.vocab);

  int32_t first = 0;
  CHECK(emx_qwen3_prefill(m, prompt, T, &first, NULL));
  CHECK(emx_qwen3_decode(m, first, n, toks));
  printf("decode %d", first);
  for (int i = 0; i < n; ++i) printf(" %d", toks[i]);
  printf("\n");

  CHECK(emx_qwen3_reset(m));
  int32_t again = -1;
  int done = 0;
  CHECK(emx_qwen3_prefill(m, prompt, T, &again, NULL));
  CHECK(emx_qwen3_decode_stream(m, again, n, collect, streamed, &done));
  printf("stream %d", again);
  for (int i = 0; i < done; ++i) printf(" %d", streamed[i]);
  printf("\n");

  CHECK(emx_qwen3_destroy(m));
  CHECK(emx_ctx_destroy(ctx));
  free(prompt);
  free(toks);
  free(streamed);
  return 0;
}
