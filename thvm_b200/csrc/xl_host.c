/* The batched GPT-2-XL-shaped model of config 3 with its host in C, on one
 * GPU: the decode step of thvm_b200/gpt2_xl.py (XLModel.step) and its prompt
 * pass (XLModel.prefill_run) over the library's own ABI only — weights from a
 * .safetensors file (sm100_safetensors_load) or named device pointers,
 * activations and KV caches in backend buffers (sm100_buf_*), the decode step
 * captured once into a graph slot (sm100_graph_*) and replayed.  It plays the
 * part of the reference's GPT-2 driver (bench/gpt2/thvm_gpt2.py:98-128: one
 * forward of the prompt, then one token at a time under TinyJit) for a C
 * caller that links no Python or torch.
 *
 * Tensor names and layouts are those of thvm_b200.gpt2_xl.xl_weights (bf16
 * matrices and embeddings as BF16, f32 vectors as F32); every tensor's byte
 * size is checked against the configuration before the first launch. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/thvm_sm100.h"

#define XL_MAX_TENSORS 4096
#define XL_HD 64 /* head dimension */

int sm100_set_error(int code, const char *fmt, ...);

/* a weight: its device address and size; buf_id != 0 when the model owns
   the buffer (loaded from a file) */
typedef struct {
  char name[128];
  void *ptr;
  uint64_t nbytes;
  uint32_t buf_id;
} XlWeight;

struct Sm100XlModel {
  Sm100XlCfg c;
  XlWeight *w;
  int32_t n_w;
  uint32_t slot;
  int captured;
  /* decode activations (backend buffer ids) */
  uint32_t h, xa, qkv, att, g, logits, tok, pos, vals, idxs, ws, counters;
  uint32_t *kv; /* per layer: [2, B, ctx, D] bf16 */
  /* the prompt pass's buffers, for prompts of pf_len ids */
  int32_t pf_len;
  uint32_t pf_tok, pf_h, pf_x, pf_qkv, pf_q, pf_k, pf_v, pf_o, pf_att, pf_g;
  Sm100SkinnyArgs sk;
};

static void *P(uint32_t id) { return sm100_buf_dptr(id); }

/* the weight `name` (layer l >= 0: "h.<l>.name") of exactly nbytes, or NULL
 * with the error recorded */
static void *W(const Sm100XlModel *m, int l, const char *name, uint64_t nbytes) {
  char key[128];
  if (l >= 0) snprintf(key, sizeof key, "h.%d.%s", l, name);
  else snprintf(key, sizeof key, "%s", name);
  for (int32_t i = 0; i < m->n_w; i++) {
    const XlWeight *e = &m->w[i];
    if (strcmp(e->name, key) != 0) continue;
    if (e->nbytes == nbytes && e->ptr) return e->ptr;
    sm100_set_error(SM100_ERR_ARG, "xl_model: weight %s has %llu bytes, want %llu", key,
                    (unsigned long long)e->nbytes, (unsigned long long)nbytes);
    return NULL;
  }
  sm100_set_error(SM100_ERR_ARG, "xl_model: weight %s missing", key);
  return NULL;
}

static int check_weights(const Sm100XlModel *m) {
  const Sm100XlCfg *c = &m->c;
  const int64_t D = c->dim, F = 4 * D, V = c->vocab;
  if (!W(m, -1, "wte", V * D * 2) || !W(m, -1, "wpe", (int64_t)c->max_ctx * D * 2) || !W(m, -1, "ln_f.w", D * 4) ||
      !W(m, -1, "ln_f.b", D * 4) || !W(m, -1, "lm_head", V * D * 2))
    return SM100_ERR_ARG;
  for (int l = 0; l < c->n_layers; l++)
    if (!W(m, l, "ln_1.w", D * 4) || !W(m, l, "ln_1.b", D * 4) || !W(m, l, "attn.w", 3 * D * D * 2) ||
        !W(m, l, "attn.b", 3 * D * 4) || !W(m, l, "proj.w", D * D * 2) || !W(m, l, "proj.b", D * 4) ||
        !W(m, l, "ln_2.w", D * 4) || !W(m, l, "ln_2.b", D * 4) || !W(m, l, "fc.w", F * D * 2) ||
        !W(m, l, "fc.b", F * 4) || !W(m, l, "p2.w", D * F * 2) || !W(m, l, "p2.b", D * 4))
      return SM100_ERR_ARG;
  return SM100_OK;
}

#define CK(x)                        \
  do {                               \
    const int rc_ = (x);             \
    if (rc_ != SM100_OK) return rc_; \
  } while (0)

/* the skinny product y = x W^T (+ bias) with the epilogue flags; kv != 0:
 * the k, v thirds also into that cache at the model's position */
static int skinny(Sm100XlModel *m, uint32_t x, const void *w, uint32_t y, int64_t K, int64_t N, const float *bias,
                  int32_t flags, uint32_t kv) {
  Sm100SkinnyArgs *a = &m->sk;
  memset(a, 0, sizeof *a);
  a->x = P(x);
  a->w = w;
  a->y = P(y);
  a->bias = bias;
  a->residual = (flags & SM100_SK_RESIDUAL) ? (const float *)P(y) : NULL;
  a->ws = (float *)P(m->ws);
  a->counters = (uint32_t *)P(m->counters);
  if (kv) {
    a->kv_cache = P(kv);
    a->pos = (const int32_t *)P(m->pos);
  }
  a->M = m->c.batch;
  a->N = N;
  a->K = K;
  a->flags = flags;
  a->kv_ctx = m->c.max_ctx;
  return sm100_skinny_bf16(a, sm100_stream());
}

/* ln_f, lm_head and the greedy pick of the B rows in h -> tok */
static int issue_head(Sm100XlModel *m) {
  const Sm100XlCfg *c = &m->c;
  void *st = sm100_stream();
  const int32_t B = c->batch, D = c->dim, V = c->vocab;
  CK(sm100_xl_layernorm((float *)P(m->h), (const float *)W(m, -1, "ln_f.w", (int64_t)D * 4),
                        (const float *)W(m, -1, "ln_f.b", (int64_t)D * 4), P(m->xa), B, D, c->norm_eps, 0, NULL, 0,
                        st));
  CK(skinny(m, m->xa, W(m, -1, "lm_head", (int64_t)V * D * 2), m->logits, D, V, NULL, 0, 0));
  CK(sm100_xl_argmax((float *)P(m->logits), V, B, V, (float *)P(m->vals), (int32_t *)P(m->idxs), 0, 0, st));
  return sm100_xl_pick((const float *)P(m->vals), (const int32_t *)P(m->idxs), 1, B, (int32_t *)P(m->tok), st);
}

/* one decode step on the backend stream (the launches of XLModel.step on one
 * rank): ids in tok at row pos -> next ids in tok, pos + 1 */
static int issue_step(Sm100XlModel *m) {
  const Sm100XlCfg *c = &m->c;
  void *st = sm100_stream();
  const int32_t B = c->batch, D = c->dim, F = 4 * D, V = c->vocab, H = c->heads;
  const float scale = 0.125f; /* 1 / sqrt(64) */
  CK(sm100_xl_embed(W(m, -1, "wte", (int64_t)V * D * 2), W(m, -1, "wpe", (int64_t)c->max_ctx * D * 2),
                    (const int32_t *)P(m->tok), (const int32_t *)P(m->pos), (float *)P(m->h), B, V, D, st));
  for (int l = 0; l < c->n_layers; l++) {
    CK(sm100_xl_layernorm((float *)P(m->h), (const float *)W(m, l, "ln_1.w", (int64_t)D * 4),
                          (const float *)W(m, l, "ln_1.b", (int64_t)D * 4), P(m->xa), B, D, c->norm_eps, 0, NULL, 0,
                          st));
    CK(skinny(m, m->xa, W(m, l, "attn.w", 3 * (int64_t)D * D * 2), m->qkv, D, 3 * D,
              (const float *)W(m, l, "attn.b", 3 * (int64_t)D * 4), SM100_SK_KV, m->kv[l]));
    CK(sm100_xl_attention((float *)P(m->qkv), 3 * D, P(m->kv[l]), (const int32_t *)P(m->pos), P(m->att), B, H, XL_HD,
                          c->max_ctx, scale, 0, st));
    CK(skinny(m, m->att, W(m, l, "proj.w", (int64_t)D * D * 2), m->h, D, D,
              (const float *)W(m, l, "proj.b", (int64_t)D * 4), SM100_SK_RESIDUAL, 0));
    CK(sm100_xl_layernorm((float *)P(m->h), (const float *)W(m, l, "ln_2.w", (int64_t)D * 4),
                          (const float *)W(m, l, "ln_2.b", (int64_t)D * 4), P(m->xa), B, D, c->norm_eps, 0, NULL, 0,
                          st));
    CK(skinny(m, m->xa, W(m, l, "fc.w", (int64_t)F * D * 2), m->g, D, F,
              (const float *)W(m, l, "fc.b", (int64_t)F * 4), SM100_SK_GELU | SM100_SK_OUT_BF16, 0));
    CK(skinny(m, m->g, W(m, l, "p2.w", (int64_t)D * F * 2), m->h, F, D,
              (const float *)W(m, l, "p2.b", (int64_t)D * 4), SM100_SK_RESIDUAL, 0));
  }
  CK(issue_head(m));
  return sm100_pos_add((int32_t *)P(m->pos), 1, st);
}

/* the prompt pass over the pf_len ids in pf_tok (the launches of
 * XLModel.prefill_run on one rank): cache rows 0..P-1, the first ids in tok,
 * pos = P */
static int issue_prefill(Sm100XlModel *m) {
  const Sm100XlCfg *c = &m->c;
  void *st = sm100_stream();
  const int32_t B = c->batch, D = c->dim, F = 4 * D, V = c->vocab, H = c->heads, Pn = m->pf_len;
  const int64_t M = (int64_t)B * Pn;
  float *h = (float *)P(m->pf_h);
  CK(sm100_xl_prefill_embed(W(m, -1, "wte", (int64_t)V * D * 2), W(m, -1, "wpe", (int64_t)c->max_ctx * D * 2),
                            (const int32_t *)P(m->pf_tok), h, B, Pn, V, D, st));
  for (int l = 0; l < c->n_layers; l++) {
    CK(sm100_xl_prefill_layernorm(h, (const float *)W(m, l, "ln_1.w", (int64_t)D * 4),
                                  (const float *)W(m, l, "ln_1.b", (int64_t)D * 4), P(m->pf_x), (int32_t)M, D,
                                  c->norm_eps, st));
    CK(sm100_gemm_bf16_ep(P(m->pf_x), W(m, l, "attn.w", 3 * (int64_t)D * D * 2), P(m->pf_qkv), M, 3 * D, D,
                          (const float *)W(m, l, "attn.b", 3 * (int64_t)D * 4), NULL, SM100_GEMM_OUT_BF16, st));
    CK(sm100_xl_prefill_split(P(m->pf_qkv), P(m->pf_q), P(m->pf_k), P(m->pf_v), P(m->kv[l]), B, Pn, H, c->max_ctx,
                              st));
    CK(sm100_attn_prefill_bf16(P(m->pf_q), P(m->pf_k), P(m->pf_v), (float *)P(m->pf_o), B, H, Pn, 128, 0.125f, 1,
                               st));
    CK(sm100_xl_prefill_merge((const float *)P(m->pf_o), P(m->pf_att), B, Pn, H, st));
    CK(sm100_gemm_bf16_ep(P(m->pf_att), W(m, l, "proj.w", (int64_t)D * D * 2), h, M, D, D,
                          (const float *)W(m, l, "proj.b", (int64_t)D * 4), h, 0, st));
    CK(sm100_xl_prefill_layernorm(h, (const float *)W(m, l, "ln_2.w", (int64_t)D * 4),
                                  (const float *)W(m, l, "ln_2.b", (int64_t)D * 4), P(m->pf_x), (int32_t)M, D,
                                  c->norm_eps, st));
    CK(sm100_gemm_bf16_ep(P(m->pf_x), W(m, l, "fc.w", (int64_t)F * D * 2), P(m->pf_g), M, F, D,
                          (const float *)W(m, l, "fc.b", (int64_t)F * 4), NULL, SM100_GEMM_GELU | SM100_GEMM_OUT_BF16,
                          st));
    CK(sm100_gemm_bf16_ep(P(m->pf_g), W(m, l, "p2.w", (int64_t)D * F * 2), h, M, D, F,
                          (const float *)W(m, l, "p2.b", (int64_t)D * 4), h, 0, st));
  }
  CK(sm100_xl_prefill_last(h, (float *)P(m->h), (int32_t *)P(m->pos), B, Pn, D, st));
  return issue_head(m);
}

void sm100_xl_model_close(Sm100XlModel *m) {
  if (!m) return;
  if (m->captured) sm100_graph_drop(m->slot);
  const uint32_t ids[] = {m->h,      m->xa,     m->qkv,    m->att,    m->g,    m->logits, m->tok,  m->pos,
                          m->vals,   m->idxs,   m->ws,     m->counters, m->pf_tok, m->pf_h, m->pf_x, m->pf_qkv,
                          m->pf_q,   m->pf_k,   m->pf_v,   m->pf_o,   m->pf_att, m->pf_g};
  for (size_t i = 0; i < sizeof ids / sizeof ids[0]; i++)
    if (ids[i]) sm100_buf_decref(ids[i]);
  for (int l = 0; l < m->c.n_layers && m->kv; l++)
    if (m->kv[l]) sm100_buf_decref(m->kv[l]);
  for (int32_t i = 0; i < m->n_w && m->w; i++)
    if (m->w[i].buf_id) sm100_buf_decref(m->w[i].buf_id);
  free(m->kv);
  free(m->w);
  free(m);
}

static uint32_t zbuf(uint64_t nbytes, int *ok) {
  const uint32_t id = sm100_buf_alloc(nbytes ? nbytes : 16);
  if (!id) *ok = 0;
  else sm100_buf_zero(id); /* stream-ordered: zero before any launch that reads it */
  return id;
}

static int cfg_ok(const Sm100XlCfg *cfg, uint32_t graph_slot) {
  return cfg && cfg->batch >= 1 && cfg->batch <= 32 && cfg->n_layers >= 1 && cfg->heads >= 1 &&
         cfg->dim == cfg->heads * XL_HD && cfg->vocab >= 1 && cfg->max_ctx >= 2 && cfg->max_ctx <= 4096 &&
         graph_slot <= 63;
}

static Sm100XlModel *model_new(const Sm100XlCfg *cfg, uint32_t graph_slot, int32_t n_w) {
  Sm100XlModel *m = (Sm100XlModel *)calloc(1, sizeof *m);
  if (!m) return NULL;
  m->c = *cfg;
  m->slot = graph_slot;
  m->w = (XlWeight *)calloc((size_t)(n_w > 0 ? n_w : 1), sizeof *m->w);
  m->kv = (uint32_t *)calloc((size_t)cfg->n_layers, sizeof(uint32_t));
  if (!m->w || !m->kv) {
    sm100_xl_model_close(m);
    return NULL;
  }
  return m;
}

/* the weights checked, then the decode buffers and caches */
static int model_finish(Sm100XlModel *m, Sm100XlModel **out) {
  const int rc = check_weights(m);
  if (rc != SM100_OK) {
    sm100_xl_model_close(m);
    return rc;
  }
  const Sm100XlCfg *c = &m->c;
  const uint64_t B = (uint64_t)c->batch, D = (uint64_t)c->dim, V = (uint64_t)c->vocab;
  int ok = 1;
  m->h = zbuf(B * D * 4, &ok);
  m->xa = zbuf(B * D * 2, &ok);
  m->qkv = zbuf(B * 3 * D * 4, &ok);
  m->att = zbuf(B * D * 2, &ok);
  m->g = zbuf(B * 4 * D * 2, &ok);
  m->logits = zbuf(B * V * 4, &ok);
  m->tok = zbuf(B * 4, &ok);
  m->pos = zbuf(4, &ok);
  m->vals = zbuf(B * 4, &ok);
  m->idxs = zbuf(B * 4, &ok);
  m->ws = zbuf(sm100_skinny_ws_bytes(c->batch), &ok);
  {
    uint64_t nmax = V > 4 * D ? V : 4 * D;
    m->counters = zbuf((nmax / 128 + 2) * 4, &ok);
  }
  for (int l = 0; l < c->n_layers && ok; l++) m->kv[l] = zbuf(2 * B * (uint64_t)c->max_ctx * D * 2, &ok);
  if (!ok) {
    sm100_xl_model_close(m);
    return sm100_set_error(SM100_ERR_OOM, "xl_model: device buffers");
  }
  *out = m;
  return SM100_OK;
}

int sm100_xl_model_open(const Sm100XlCfg *cfg, const char *weights_path, uint32_t graph_slot, Sm100XlModel **out) {
  if (!cfg_ok(cfg, graph_slot) || !weights_path || !out)
    return sm100_set_error(SM100_ERR_ARG, "xl_model_open: bad configuration");
  *out = NULL;
  Sm100TensorEntry *ent = (Sm100TensorEntry *)calloc(XL_MAX_TENSORS, sizeof *ent);
  if (!ent) return sm100_set_error(SM100_ERR_OOM, "xl_model_open: host memory");
  int32_t n = 0;
  const int rc = sm100_safetensors_load(weights_path, ent, XL_MAX_TENSORS, &n);
  if (rc != SM100_OK) {
    free(ent);
    return rc;
  }
  Sm100XlModel *m = model_new(cfg, graph_slot, n);
  if (!m) {
    for (int32_t i = 0; i < n; i++) sm100_buf_decref(ent[i].buf_id);
    free(ent);
    return sm100_set_error(SM100_ERR_OOM, "xl_model_open: host memory");
  }
  for (int32_t i = 0; i < n; i++) {
    snprintf(m->w[i].name, sizeof m->w[i].name, "%s", ent[i].name);
    m->w[i].ptr = sm100_buf_dptr(ent[i].buf_id);
    m->w[i].nbytes = ent[i].nbytes;
    m->w[i].buf_id = ent[i].buf_id;
  }
  m->n_w = n;
  free(ent);
  return model_finish(m, out);
}

int sm100_xl_model_open_ptrs(const Sm100XlCfg *cfg, const char *const *names, void *const *ptrs,
                             const uint64_t *nbytes, int32_t n, uint32_t graph_slot, Sm100XlModel **out) {
  if (!cfg_ok(cfg, graph_slot) || !names || !ptrs || !nbytes || n < 1 || !out)
    return sm100_set_error(SM100_ERR_ARG, "xl_model_open_ptrs: bad configuration");
  *out = NULL;
  Sm100XlModel *m = model_new(cfg, graph_slot, n);
  if (!m) return sm100_set_error(SM100_ERR_OOM, "xl_model_open_ptrs: host memory");
  for (int32_t i = 0; i < n; i++) {
    if (!names[i] || strlen(names[i]) >= sizeof m->w[i].name) {
      sm100_xl_model_close(m);
      return sm100_set_error(SM100_ERR_ARG, "xl_model_open_ptrs: weight name %d", i);
    }
    snprintf(m->w[i].name, sizeof m->w[i].name, "%s", names[i]);
    m->w[i].ptr = ptrs[i];
    m->w[i].nbytes = nbytes[i];
  }
  m->n_w = n;
  return model_finish(m, out);
}

/* the prompt pass's buffers for prompts of len ids (kept while len stays) */
static int prefill_bufs(Sm100XlModel *m, int32_t len) {
  if (m->pf_len == len) return SM100_OK;
  uint32_t *ids[] = {&m->pf_tok, &m->pf_h, &m->pf_x, &m->pf_qkv, &m->pf_q,
                     &m->pf_k,   &m->pf_v, &m->pf_o, &m->pf_att, &m->pf_g};
  for (size_t i = 0; i < sizeof ids / sizeof ids[0]; i++) {
    if (*ids[i]) sm100_buf_decref(*ids[i]);
    *ids[i] = 0;
  }
  m->pf_len = 0;
  const uint64_t B = (uint64_t)m->c.batch, D = (uint64_t)m->c.dim, H = (uint64_t)m->c.heads, L = (uint64_t)len,
                 M = B * L;
  int ok = 1;
  m->pf_tok = zbuf(M * 4, &ok);
  m->pf_h = zbuf(M * D * 4, &ok);
  m->pf_x = zbuf(M * D * 2, &ok);
  m->pf_qkv = zbuf(M * 3 * D * 2, &ok);
  m->pf_q = zbuf(B * H * L * 128 * 2, &ok); /* columns 64.. stay zero */
  m->pf_k = zbuf(B * H * L * 128 * 2, &ok);
  m->pf_v = zbuf(B * H * L * 128 * 2, &ok);
  m->pf_o = zbuf(B * H * L * 128 * 4, &ok);
  m->pf_att = zbuf(M * D * 2, &ok);
  m->pf_g = zbuf(M * 4 * D * 2, &ok);
  if (!ok) return sm100_set_error(SM100_ERR_OOM, "xl_model_prefill: device buffers for %d ids", len);
  m->pf_len = len;
  return SM100_OK;
}

int sm100_xl_model_prefill(Sm100XlModel *m, const int32_t *prompts, int32_t len, int32_t *tok_out) {
  if (!m || !prompts || len < 1 || len >= m->c.max_ctx)
    return sm100_set_error(SM100_ERR_ARG, "xl_model_prefill: %d ids (1 <= len < max_ctx %d)", len,
                           m ? m->c.max_ctx : 0);
  CK(prefill_bufs(m, len));
  CK(sm100_buf_write(m->pf_tok, prompts, (uint64_t)m->c.batch * len * 4));
  CK(issue_prefill(m));
  if (tok_out) CK(sm100_buf_read(m->tok, tok_out, (uint64_t)m->c.batch * 4));
  return SM100_OK;
}

int sm100_xl_model_step(Sm100XlModel *m, const int32_t *tok_in, int32_t *tok_out) {
  if (!m) return sm100_set_error(SM100_ERR_ARG, "xl_model_step: no model");
  if (tok_in) CK(sm100_buf_write(m->tok, tok_in, (uint64_t)m->c.batch * 4));
  if (!m->captured) {
    /* the first step runs eagerly (it sets the launches' attributes); the
       step is then captured once (the capture runs nothing) and every later
       call replays it */
    CK(issue_step(m));
    CK(sm100_graph_capture_begin(m->slot));
    const int rc = issue_step(m);
    const int rc2 = sm100_graph_capture_end(m->slot);
    if (rc != SM100_OK) return rc;
    if (rc2 != SM100_OK) return rc2;
    m->captured = 1;
  } else {
    CK(sm100_graph_replay(m->slot));
  }
  if (tok_out) CK(sm100_buf_read(m->tok, tok_out, (uint64_t)m->c.batch * 4));
  return SM100_OK;
}

int32_t sm100_xl_model_pos(const Sm100XlModel *m) {
  int32_t p = -1;
  if (!m || sm100_buf_read(m->pos, &p, 4) != SM100_OK) return -1;
  return p;
}

uint32_t sm100_xl_model_logits(const Sm100XlModel *m) { return m ? m->logits : 0; }
