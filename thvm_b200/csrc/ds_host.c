/* The batched MoE decode step of config 5 with its host in C: the step of
 * thvm_b200/dsv2.py (one rank) over the library's own ABI only — weights from
 * a .safetensors file (sm100_safetensors_load) or named device pointers,
 * activations and caches in backend buffers (sm100_buf_*), the step captured
 * once into a graph slot (sm100_graph_*) and replayed.  It plays the part of
 * the reference's C decode bench host (bench/dsv2_decode_bench.c: weights,
 * emit, the replay loop :2586-2610) for a C caller that links no Python or
 * torch.
 *
 * Tensor names and layouts are those of thvm_b200.dsv2.ds_weights (bf16 as
 * BF16, fp8 codes as F8_E4M3 or U8, f32 as F32), plus the rotary tables "cos"
 * and "sin" [max_ctx][d_rope] f32.  Every tensor's byte size is checked
 * against the configuration before the first launch. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/thvm_sm100.h"

#define DS_MAX_TENSORS 4096

int sm100_set_error(int code, const char *fmt, ...);

/* a weight: its device address and size; buf_id != 0 when the model owns
   the buffer (loaded from a file) */
typedef struct {
  char name[128];
  void *ptr;
  uint64_t nbytes;
  uint32_t buf_id;
} WeightRef;

struct Sm100DsModel {
  Sm100DsCfg c;
  WeightRef *w;
  int32_t n_w;
  uint32_t slot;
  int captured;
  /* activations (backend buffer ids) */
  uint32_t h, xn, qkva, qo, o, gu, rl, logits, tok, pos, sel, wsel, counter, slot_off, slot_tok, slot_w, a, vals,
      idxs, ws, counters;
  uint32_t *cache_c, *cache_pe;
  Sm100SkinnyArgs sk;
};

static void *P(uint32_t id) { return sm100_buf_dptr(id); }

static const WeightRef *find(const Sm100DsModel *m, const char *name) {
  for (int32_t i = 0; i < m->n_w; i++)
    if (strcmp(m->w[i].name, name) == 0) return &m->w[i];
  return NULL;
}

/* the weight `name` (layer l >= 0: "l<l>.name") of exactly nbytes, or NULL
 * with the error recorded */
static void *W(const Sm100DsModel *m, int l, const char *name, uint64_t nbytes) {
  char key[128];
  if (l >= 0) snprintf(key, sizeof key, "l%d.%s", l, name);
  else snprintf(key, sizeof key, "%s", name);
  const WeightRef *e = find(m, key);
  if (!e || e->nbytes != nbytes || !e->ptr) {
    sm100_set_error(SM100_ERR_ARG, "ds_model: weight %s %s (%llu bytes, want %llu)", key,
                    e ? "has the wrong size" : "missing", (unsigned long long)(e ? e->nbytes : 0),
                    (unsigned long long)nbytes);
    return NULL;
  }
  return e->ptr;
}

static int64_t n_q(const Sm100DsCfg *c) { return (int64_t)c->heads * (c->d_nope + c->d_rope); }
static int64_t n_qkva(const Sm100DsCfg *c) { return n_q(c) + c->kv_lora + c->d_rope; }

/* every weight present with its size (before anything launches) */
static int check_weights(const Sm100DsModel *m) {
  const Sm100DsCfg *c = &m->c;
  const int64_t D = c->dim, V = c->vocab, H = c->heads, KV = c->kv_lora, DN = c->d_nope, DV = c->d_v, E = c->n_exp,
                I = c->moe_inter, DI = c->dense_inter, NS = c->n_shared;
  if (!W(m, -1, "embed", V * D * 2) || !W(m, -1, "norm_f", D * 4) || !W(m, -1, "lm_head", V * D * 2) ||
      !W(m, -1, "cos", (int64_t)c->max_ctx * c->d_rope * 4) || !W(m, -1, "sin", (int64_t)c->max_ctx * c->d_rope * 4))
    return SM100_ERR_ARG;
  for (int l = 0; l < c->n_layers; l++) {
    if (!W(m, l, "attn_norm", D * 4) || !W(m, l, "ffn_norm", D * 4) || !W(m, l, "kv_norm", KV * 4) ||
        !W(m, l, "w_qkva", n_qkva(c) * D * 2) || !W(m, l, "w_uk", H * DN * KV * 2) ||
        !W(m, l, "w_uv", H * DV * KV * 2) || !W(m, l, "w_o", D * H * DV * 2))
      return SM100_ERR_ARG;
    if (l < c->n_dense) {
      if (!W(m, l, "d_gu", 2 * DI * D * 2) || !W(m, l, "d_down", D * DI * 2)) return SM100_ERR_ARG;
    } else {
      const int64_t ne = E + NS;
      if (!W(m, l, "router", E * D * 2) || !W(m, l, "e_gu", ne * 2 * I * D) ||
          !W(m, l, "e_gu_s", ne * ((2 * I + 127) / 128) * ((D + 127) / 128) * 4) || !W(m, l, "e_d", ne * D * I) ||
          !W(m, l, "e_d_s", ne * ((D + 127) / 128) * ((I + 127) / 128) * 4))
        return SM100_ERR_ARG;
    }
  }
  return SM100_OK;
}

static int skinny(Sm100DsModel *m, uint32_t x, const void *w, uint32_t y, int64_t K, int64_t N, int residual) {
  Sm100SkinnyArgs *a = &m->sk;
  memset(a, 0, sizeof *a);
  a->x = P(x);
  a->w = w;
  a->y = P(y);
  a->residual = residual ? P(y) : NULL;
  a->ws = (float *)P(m->ws);
  a->counters = (uint32_t *)P(m->counters);
  a->M = m->c.batch;
  a->N = N;
  a->K = K;
  a->flags = residual ? SM100_SK_RESIDUAL : 0;
  return sm100_skinny_bf16(a, sm100_stream());
}

#define CK(x)                        \
  do {                               \
    const int rc_ = (x);             \
    if (rc_ != SM100_OK) return rc_; \
  } while (0)

/* one decode step on the backend stream (the launches dsv2.py's DSModel.step
 * issues on one rank) */
static int issue_step(Sm100DsModel *m) {
  const Sm100DsCfg *c = &m->c;
  void *st = sm100_stream();
  const int32_t B = c->batch, D = c->dim, KV = c->kv_lora, DN = c->d_nope, DR = c->d_rope, DV = c->d_v,
                H = c->heads, E = c->n_exp, K = c->top_k, I = c->moe_inter, DI = c->dense_inter, NS = c->n_shared;
  const int64_t nq = n_q(c), nqkva = n_qkva(c);
  CK(sm100_ds_embed(W(m, -1, "embed", (int64_t)c->vocab * D * 2), (const int32_t *)P(m->tok), (float *)P(m->h), B,
                    c->vocab, D, st));
  const float *cs = (const float *)W(m, -1, "cos", (int64_t)c->max_ctx * DR * 4);
  const float *sn = (const float *)W(m, -1, "sin", (int64_t)c->max_ctx * DR * 4);
  for (int l = 0; l < c->n_layers; l++) {
    CK(sm100_ds_rmsnorm((const float *)P(m->h), (const float *)W(m, l, "attn_norm", (int64_t)D * 4), P(m->xn), B, D,
                        c->eps, st));
    CK(skinny(m, m->xn, W(m, l, "w_qkva", nqkva * D * 2), m->qkva, D, nqkva, 0));
    CK(sm100_ds_mla_post((const float *)P(m->qkva), nqkva, nq, (const float *)W(m, l, "kv_norm", (int64_t)KV * 4), cs,
                         sn, (const int32_t *)P(m->pos), P(m->qo), W(m, l, "w_uk", (int64_t)H * DN * KV * 2),
                         W(m, l, "w_uv", (int64_t)H * DV * KV * 2), P(m->cache_c[l]), P(m->cache_pe[l]), P(m->o), B, H,
                         DN, DR, DV, KV, c->max_ctx, c->eps, c->scale, st));
    CK(skinny(m, m->o, W(m, l, "w_o", (int64_t)D * H * DV * 2), m->h, (int64_t)H * DV, D, 1));
    CK(sm100_ds_rmsnorm((const float *)P(m->h), (const float *)W(m, l, "ffn_norm", (int64_t)D * 4), P(m->xn), B, D,
                        c->eps, st));
    if (l < c->n_dense) {
      CK(skinny(m, m->xn, W(m, l, "d_gu", (int64_t)2 * DI * D * 2), m->gu, D, 2 * DI, 0));
      CK(sm100_ds_silu_mul((const float *)P(m->gu), P(m->xn), B, DI, st));
      CK(skinny(m, m->xn, W(m, l, "d_down", (int64_t)D * DI * 2), m->h, DI, D, 1));
      continue;
    }
    const int64_t ne = E + NS;
    CK(sm100_ds_router_route(P(m->xn), W(m, l, "router", (int64_t)E * D * 2), (float *)P(m->rl),
                             (int32_t *)P(m->counter), D, E, K, B, 0, E, NS, (int32_t *)P(m->sel), (float *)P(m->wsel),
                             (int32_t *)P(m->slot_off), (int32_t *)P(m->slot_tok), (float *)P(m->slot_w), st));
    CK(sm100_ds_experts(P(m->xn), W(m, l, "e_gu", ne * 2 * I * D),
                        (const float *)W(m, l, "e_gu_s", ne * ((2 * I + 127) / 128) * ((D + 127) / 128) * 4),
                        W(m, l, "e_d", ne * D * I),
                        (const float *)W(m, l, "e_d_s", ne * ((D + 127) / 128) * ((I + 127) / 128) * 4),
                        (const int32_t *)P(m->slot_off), (const int32_t *)P(m->slot_tok), (const float *)P(m->slot_w),
                        P(m->a), (float *)P(m->h), (int32_t)ne, D, I, st));
  }
  CK(sm100_ds_rmsnorm((const float *)P(m->h), (const float *)W(m, -1, "norm_f", (int64_t)D * 4), P(m->xn), B, D,
                      c->eps, st));
  CK(skinny(m, m->xn, W(m, -1, "lm_head", (int64_t)c->vocab * D * 2), m->logits, D, c->vocab, 0));
  CK(sm100_xl_argmax((float *)P(m->logits), c->vocab, B, c->vocab, (float *)P(m->vals), (int32_t *)P(m->idxs), 0, 0,
                     st));
  CK(sm100_xl_pick((const float *)P(m->vals), (const int32_t *)P(m->idxs), 1, B, (int32_t *)P(m->tok), st));
  CK(sm100_pos_add((int32_t *)P(m->pos), 1, st));
  return SM100_OK;
}

void sm100_ds_model_close(Sm100DsModel *m) {
  if (!m) return;
  if (m->captured) sm100_graph_drop(m->slot);
  const uint32_t ids[] = {m->h,        m->xn,     m->qkva,     m->qo,     m->o,     m->gu,      m->rl,
                          m->logits,   m->tok,    m->pos,      m->sel,    m->wsel,  m->counter, m->slot_off,
                          m->slot_tok, m->slot_w, m->a,        m->vals,   m->idxs,  m->ws,      m->counters};
  for (size_t i = 0; i < sizeof ids / sizeof ids[0]; i++)
    if (ids[i]) sm100_buf_decref(ids[i]);
  for (int l = 0; l < m->c.n_layers && m->cache_c && m->cache_pe; l++) {
    if (m->cache_c[l]) sm100_buf_decref(m->cache_c[l]);
    if (m->cache_pe[l]) sm100_buf_decref(m->cache_pe[l]);
  }
  for (int32_t i = 0; i < m->n_w && m->w; i++)
    if (m->w[i].buf_id) sm100_buf_decref(m->w[i].buf_id);
  free(m->cache_c);
  free(m->cache_pe);
  free(m->w);
  free(m);
}

static uint32_t zbuf(uint64_t nbytes, int *ok) {
  const uint32_t id = sm100_buf_alloc(nbytes ? nbytes : 16);   /* new storage reads as zeros */
  if (!id) *ok = 0;
  return id;
}

static int cfg_ok(const Sm100DsCfg *cfg, uint32_t graph_slot) {
  return cfg && cfg->batch >= 1 && cfg->batch <= 32 && cfg->n_layers >= 1 && cfg->dim >= 128 && cfg->dim % 128 == 0 &&
         cfg->moe_inter % 128 == 0 && cfg->n_exp >= 1 && cfg->n_exp <= 64 && cfg->top_k >= 1 &&
         cfg->top_k <= cfg->n_exp && cfg->n_dense >= 0 && cfg->n_dense <= cfg->n_layers && cfg->max_ctx >= 2 &&
         graph_slot <= 63;
}

static Sm100DsModel *model_new(const Sm100DsCfg *cfg, uint32_t graph_slot, int32_t n_w) {
  Sm100DsModel *m = (Sm100DsModel *)calloc(1, sizeof *m);
  if (!m) return NULL;
  m->c = *cfg;
  m->slot = graph_slot;
  m->w = (WeightRef *)calloc((size_t)(n_w > 0 ? n_w : 1), sizeof *m->w);
  m->cache_c = (uint32_t *)calloc((size_t)cfg->n_layers, sizeof(uint32_t));
  m->cache_pe = (uint32_t *)calloc((size_t)cfg->n_layers, sizeof(uint32_t));
  if (!m->w || !m->cache_c || !m->cache_pe) {
    sm100_ds_model_close(m);
    return NULL;
  }
  return m;
}

/* the weights checked, then the activation buffers and caches */
static int model_finish(Sm100DsModel *m, Sm100DsModel **out) {
  const int rc = check_weights(m);
  if (rc != SM100_OK) {
    sm100_ds_model_close(m);
    return rc;
  }
  const Sm100DsCfg *c = &m->c;
  const uint64_t B = (uint64_t)c->batch, D = (uint64_t)c->dim, DI = (uint64_t)c->dense_inter,
                 ns = (uint64_t)c->n_shared, K = (uint64_t)c->top_k, E = (uint64_t)c->n_exp;
  const uint64_t xn_cols = D > DI ? D : DI, slots = B * (K + ns);
  int ok = 1;
  m->h = zbuf(B * D * 4, &ok);
  m->xn = zbuf(B * xn_cols * 2, &ok);
  m->qkva = zbuf(B * (uint64_t)n_qkva(c) * 4, &ok);
  m->qo = zbuf(B * (uint64_t)n_q(c) * 2, &ok);
  m->o = zbuf(B * (uint64_t)c->heads * c->d_v * 2, &ok);
  m->gu = zbuf(B * 2 * DI * 4, &ok);
  m->rl = zbuf(B * E * 4, &ok);
  m->logits = zbuf(B * (uint64_t)c->vocab * 4, &ok);
  m->tok = zbuf(B * 4, &ok);
  m->pos = zbuf(4, &ok);
  m->sel = zbuf(B * K * 4, &ok);
  m->wsel = zbuf(B * K * 4, &ok);
  m->counter = zbuf(4, &ok);
  m->slot_off = zbuf((E + ns + 1) * 4, &ok);
  m->slot_tok = zbuf(slots * 4, &ok);
  m->slot_w = zbuf(slots * 4, &ok);
  m->a = zbuf(slots * (uint64_t)c->moe_inter * 2, &ok);
  m->vals = zbuf(B * 4, &ok);
  m->idxs = zbuf(B * 4, &ok);
  m->ws = zbuf(sm100_skinny_ws_bytes(c->batch), &ok);
  {
    uint64_t nmax = (uint64_t)c->vocab;
    const uint64_t cand[3] = {(uint64_t)n_qkva(c), 2 * DI, D};
    for (int i = 0; i < 3; i++)
      if (cand[i] > nmax) nmax = cand[i];
    m->counters = zbuf((nmax / 128 + 2) * 4, &ok);
  }
  for (int l = 0; l < c->n_layers && ok; l++) {
    m->cache_c[l] = zbuf(B * (uint64_t)c->max_ctx * c->kv_lora * 2, &ok);
    m->cache_pe[l] = zbuf(B * (uint64_t)c->max_ctx * c->d_rope * 2, &ok);
  }
  if (!ok) {
    sm100_ds_model_close(m);
    return sm100_set_error(SM100_ERR_OOM, "ds_model: device buffers");
  }
  *out = m;
  return SM100_OK;
}

int sm100_ds_model_open(const Sm100DsCfg *cfg, const char *weights_path, uint32_t graph_slot, Sm100DsModel **out) {
  if (!cfg_ok(cfg, graph_slot) || !weights_path || !out)
    return sm100_set_error(SM100_ERR_ARG, "ds_model_open: bad configuration");
  *out = NULL;
  Sm100TensorEntry *ent = (Sm100TensorEntry *)calloc(DS_MAX_TENSORS, sizeof *ent);
  if (!ent) return sm100_set_error(SM100_ERR_OOM, "ds_model_open: host memory");
  int32_t n = 0;
  const int rc = sm100_safetensors_load(weights_path, ent, DS_MAX_TENSORS, &n);
  if (rc != SM100_OK) {
    free(ent);
    return rc;
  }
  Sm100DsModel *m = model_new(cfg, graph_slot, n);
  if (!m) {
    for (int32_t i = 0; i < n; i++) sm100_buf_decref(ent[i].buf_id);
    free(ent);
    return sm100_set_error(SM100_ERR_OOM, "ds_model_open: host memory");
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

int sm100_ds_model_open_ptrs(const Sm100DsCfg *cfg, const char *const *names, void *const *ptrs,
                             const uint64_t *nbytes, int32_t n, uint32_t graph_slot, Sm100DsModel **out) {
  if (!cfg_ok(cfg, graph_slot) || !names || !ptrs || !nbytes || n < 1 || !out)
    return sm100_set_error(SM100_ERR_ARG, "ds_model_open_ptrs: bad configuration");
  *out = NULL;
  Sm100DsModel *m = model_new(cfg, graph_slot, n);
  if (!m) return sm100_set_error(SM100_ERR_OOM, "ds_model_open_ptrs: host memory");
  for (int32_t i = 0; i < n; i++) {
    if (!names[i] || strlen(names[i]) >= sizeof m->w[i].name) {
      sm100_ds_model_close(m);
      return sm100_set_error(SM100_ERR_ARG, "ds_model_open_ptrs: weight name %d", i);
    }
    snprintf(m->w[i].name, sizeof m->w[i].name, "%s", names[i]);
    m->w[i].ptr = ptrs[i];
    m->w[i].nbytes = nbytes[i];
  }
  m->n_w = n;
  return model_finish(m, out);
}

int sm100_ds_model_step(Sm100DsModel *m, const int32_t *tok_in, int32_t *tok_out) {
  if (!m) return sm100_set_error(SM100_ERR_ARG, "ds_model_step: no model");
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

int32_t sm100_ds_model_pos(const Sm100DsModel *m) {
  int32_t p = -1;
  if (!m || sm100_buf_read(m->pos, &p, 4) != SM100_OK) return -1;
  return p;
}

int sm100_ds_model_reset(Sm100DsModel *m) {
  if (!m) return sm100_set_error(SM100_ERR_ARG, "ds_model_reset: no model");
  sm100_buf_zero(m->pos);
  return SM100_OK;
}

uint32_t sm100_ds_model_logits(const Sm100DsModel *m) { return m ? m->logits : 0; }
