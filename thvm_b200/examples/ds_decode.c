/* Greedy decode of the config-5 MoE model from C alone, over the library's
 * C ABI (include/thvm_sm100.h): sm100_init, sm100_ds_model_open on a
 * .safetensors weight file, sm100_ds_model_step per position.  The prompt
 * ids of every row are fed one position at a time (teacher forcing), then
 * the model's own choices; every step's next ids are printed as one line.
 *
 *   ds_decode WEIGHTS N_LAYERS DIM HEADS KV_LORA D_NOPE D_ROPE D_V N_EXP TOP_K
 *             MOE_INTER DENSE_INTER N_DENSE N_SHARED VOCAB MAX_CTX BATCH
 *             EPS SCALE PROMPT_LEN STEPS PROMPT_IDS...
 *
 * PROMPT_IDS: BATCH x PROMPT_LEN ids, row-major.  Exit status 0 on success. */
#include <stdio.h>
#include <stdlib.h>

#include "../../include/thvm_sm100.h"

int main(int argc, char **argv) {
  if (argc < 23) {
    fprintf(stderr, "usage: see the comment at the top of ds_decode.c\n");
    return 2;
  }
  Sm100DsCfg c;
  c.n_layers = atoi(argv[2]);
  c.dim = atoi(argv[3]);
  c.heads = atoi(argv[4]);
  c.kv_lora = atoi(argv[5]);
  c.d_nope = atoi(argv[6]);
  c.d_rope = atoi(argv[7]);
  c.d_v = atoi(argv[8]);
  c.n_exp = atoi(argv[9]);
  c.top_k = atoi(argv[10]);
  c.moe_inter = atoi(argv[11]);
  c.dense_inter = atoi(argv[12]);
  c.n_dense = atoi(argv[13]);
  c.n_shared = atoi(argv[14]);
  c.vocab = atoi(argv[15]);
  c.max_ctx = atoi(argv[16]);
  c.batch = atoi(argv[17]);
  c.eps = (float)atof(argv[18]);
  c.scale = (float)atof(argv[19]);
  const int np = atoi(argv[20]), steps = atoi(argv[21]), B = c.batch;
  if (argc != 22 + B * np || np < 1 || steps < np) {
    fprintf(stderr, "ds_decode: need %d prompt ids and STEPS >= PROMPT_LEN\n", B * np);
    return 2;
  }
  int32_t *prompt = (int32_t *)malloc(sizeof(int32_t) * (size_t)B * np), *in = malloc(sizeof(int32_t) * B),
          *out = malloc(sizeof(int32_t) * B);
  if (!prompt || !in || !out) return 1;
  for (int i = 0; i < B * np; i++) prompt[i] = atoi(argv[22 + i]);
  if (sm100_init() != SM100_OK) {
    fprintf(stderr, "sm100_init: %s\n", sm100_last_error());
    return 1;
  }
  Sm100DsModel *m = NULL;
  if (sm100_ds_model_open(&c, argv[1], 0, &m) != SM100_OK) {
    fprintf(stderr, "sm100_ds_model_open: %s\n", sm100_last_error());
    return 1;
  }
  for (int t = 0; t < steps; t++) {
    for (int b = 0; b < B; b++) in[b] = t < np ? prompt[b * np + t] : out[b];
    if (sm100_ds_model_step(m, in, out) != SM100_OK) {
      fprintf(stderr, "sm100_ds_model_step: %s\n", sm100_last_error());
      sm100_ds_model_close(m);
      return 1;
    }
    for (int b = 0; b < B; b++) printf(b ? " %d" : "%d", out[b]);
    printf("\n");
  }
  sm100_ds_model_close(m);
  sm100_shutdown();
  free(prompt);
  free(in);
  free(out);
  return 0;
}
