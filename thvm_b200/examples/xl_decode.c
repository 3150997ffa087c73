/* Prompt pass and greedy decode of the config-3 model from C alone, over the
 * library's C ABI (include/thvm_sm100.h): sm100_init, sm100_xl_model_open on
 * a .safetensors weight file, sm100_xl_model_prefill on the prompts (every
 * position at once), then sm100_xl_model_step per token, each step's input
 * the previous step's choice.  Prints the ids the prompt pass picked, then
 * each step's, one line each.
 *
 *   xl_decode WEIGHTS N_LAYERS DIM HEADS VOCAB MAX_CTX BATCH EPS PROMPT_LEN STEPS PROMPT_IDS...
 *
 * PROMPT_IDS: BATCH x PROMPT_LEN ids, row-major.  Exit status 0 on success. */
#include <stdio.h>
#include <stdlib.h>

#include "../../include/thvm_sm100.h"

int main(int argc, char **argv) {
  if (argc < 11) {
    fprintf(stderr, "usage: see the comment at the top of xl_decode.c\n");
    return 2;
  }
  Sm100XlCfg c;
  c.n_layers = atoi(argv[2]);
  c.dim = atoi(argv[3]);
  c.heads = atoi(argv[4]);
  c.vocab = atoi(argv[5]);
  c.max_ctx = atoi(argv[6]);
  c.batch = atoi(argv[7]);
  c.norm_eps = (float)atof(argv[8]);
  const int np = atoi(argv[9]), steps = atoi(argv[10]), B = c.batch;
  if (np < 1 || steps < 0 || B < 1 || argc != 11 + B * np) {
    fprintf(stderr, "xl_decode: need %d prompt ids\n", B * np);
    return 2;
  }
  int32_t *prompt = (int32_t *)malloc(sizeof(int32_t) * (size_t)B * np), *ids = malloc(sizeof(int32_t) * B);
  if (!prompt || !ids) return 1;
  for (int i = 0; i < B * np; i++) prompt[i] = atoi(argv[11 + i]);
  if (sm100_init() != SM100_OK) {
    fprintf(stderr, "sm100_init: %s\n", sm100_last_error());
    return 1;
  }
  Sm100XlModel *m = NULL;
  if (sm100_xl_model_open(&c, argv[1], 0, &m) != SM100_OK) {
    fprintf(stderr, "sm100_xl_model_open: %s\n", sm100_last_error());
    return 1;
  }
  int rc = sm100_xl_model_prefill(m, prompt, np, ids);
  for (int t = 0; rc == SM100_OK; t++) {
    for (int b = 0; b < B; b++) printf(b ? " %d" : "%d", ids[b]);
    printf("\n");
    if (t == steps) break;
    rc = sm100_xl_model_step(m, NULL, ids);
  }
  if (rc != SM100_OK) fprintf(stderr, "xl_decode: %s\n", sm100_last_error());
  sm100_xl_model_close(m);
  sm100_shutdown();
  free(prompt);
  free(ids);
  return rc == SM100_OK ? 0 : 1;
}
