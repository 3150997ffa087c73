/* CPU oracle (test infrastructure only; see oracle.h).  Plain C restatement of
 * the reference's float32 arithmetic for the GPT-2 decode path. */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

#define LOG2E 1.4426950408889634f /* src/nn/elementwise.c:7-9 */

/* Threads for the row-parallel loops: $THVM_ORACLE_THREADS, else every online
 * core.  Splitting rows across threads leaves each output's summation order
 * unchanged, so results do not depend on the thread count. */
int orc_num_threads(void) {
  static int n = 0;
  if (n == 0) {
    const char *e = getenv("THVM_ORACLE_THREADS");
    n = e && atoi(e) > 0 ? atoi(e) : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 256) n = 256;
  }
  return n;
}

typedef struct {
  void (*fn)(void *ctx, int64_t lo, int64_t hi);
  void *ctx;
  int64_t lo, hi;
} ParTask;

static void *par_run(void *p) {
  ParTask *t = (ParTask *)p;
  t->fn(t->ctx, t->lo, t->hi);
  return NULL;
}

/* fn over [0, n) split into contiguous chunks, one per thread. */
static void par_for(int64_t n, int64_t min_chunk, void (*fn)(void *, int64_t, int64_t),
                    void *ctx) {
  int nt = orc_num_threads();
  if ((int64_t)nt * min_chunk > n) nt = (int)(n / (min_chunk > 0 ? min_chunk : 1));
  if (nt <= 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t th[256];
  ParTask task[256];
  const int64_t per = (n + nt - 1) / nt;
  int launched = 0;
  for (int i = 0; i < nt; i++) {
    const int64_t lo = i * per, hi = lo + per < n ? lo + per : n;
    if (lo >= hi) break;
    task[i] = (ParTask){fn, ctx, lo, hi};
    if (i == 0) continue;
    if (pthread_create(&th[i], NULL, par_run, &task[i]) != 0) {
      fn(ctx, lo, hi); /* run inline if a thread cannot start */
      task[i].fn = NULL;
    }
    launched = i + 1;
  }
  fn(ctx, task[0].lo, task[0].hi);
  for (int i = 1; i < launched; i++)
    if (task[i].fn) pthread_join(th[i], NULL);
}

/* The reference's CPU kernels have no exp2 instruction and use tinygrad's
 * xexp2 decomposition (src/codegen/xexp2f.c:12-33, after tinygrad
 * codegen/decomp/transcendental.py): q = x rounded half away from zero,
 * s = x - q, a degree-6 polynomial in s, times 2^q built from two exponent
 * fields; inputs >= 128 give inf, < -150 give 0, NaN stays NaN.  Every
 * product and sum is rounded on its own (no FMA: -ffp-contract=off). */
static float orc_exp2(float d) {
  static const float c[7] = {0.1535920892e-3f, 0.1339262701e-2f, 0.9618384764e-2f,
                             0.5550347269e-1f, 0.2402264476e+0f, 0.6931471825e+0f, 1.0f};
  const float x = (d == d && d != INFINITY && d != -INFINITY) ? d : 0.0f;
  const int q = (int)(x + (x < 0.0f ? -0.5f : 0.5f));
  const float s = x - (float)q;
  float u = c[0];
  for (int i = 1; i < 7; i++) {
    const float t = u * s;
    u = t + c[i];
  }
  const int h = q >> 1;
  const uint32_t b0 = (uint32_t)(h + 127) << 23, b1 = (uint32_t)(q - h + 127) << 23;
  float p0, p1;
  memcpy(&p0, &b0, sizeof p0);
  memcpy(&p1, &b1, sizeof p1);
  u = u * p0;
  u = u * p1;
  u = d < 128.0f ? u : INFINITY;
  u = d < -150.0f ? 0.0f : u;
  return d == d ? u : NAN;
}

/* exp(x) = exp2(x * log2e) (src/nn/elementwise.c:7-9) */
static inline float orc_exp(float x) { return orc_exp2(x * LOG2E); }

typedef struct {
  const float *x, *w, *b;
  float *y;
  int64_t M, K, N;
} LinCtx;

static void linear_rows(void *p, int64_t lo, int64_t hi) {
  const LinCtx *c = (const LinCtx *)p;
  for (int64_t m = 0; m < c->M; m++) {
    const float *xr = c->x + m * c->K;
    for (int64_t n = lo; n < hi; n++) {
      const float *wr = c->w + n * c->K;
      float acc = 0.0f;
      for (int64_t k = 0; k < c->K; k++) acc += xr[k] * wr[k];
      c->y[m * c->N + n] = c->b ? acc + c->b[n] : acc;
    }
  }
}

void orc_linear_f32(const float *x, const float *w, const float *b, float *y,
                    int64_t M, int64_t K, int64_t N) {
  LinCtx c = {x, w, b, y, M, K, N};
  par_for(N, 64, linear_rows, &c);
}

void orc_layernorm_f32(const float *x, const float *g, const float *b, float *y,
                       int64_t M, int64_t D, float eps) {
  const float inv_n = (float)(1.0 / (double)D); /* nn_mean: sum * (1/count) */
  for (int64_t m = 0; m < M; m++) {
    const float *xr = x + m * D;
    float *yr = y + m * D;
    float s = 0.0f;
    for (int64_t i = 0; i < D; i++) s += xr[i];
    const float mean = s * inv_n;
    float v = 0.0f;
    for (int64_t i = 0; i < D; i++) {
      const float c = xr[i] - mean;
      v += c * c;
    }
    const float var = v * inv_n;
    const float r = 1.0f / sqrtf(var + eps); /* NN_RSQRT = RECIP(SQRT) */
    for (int64_t i = 0; i < D; i++) {
      float o = (xr[i] - mean) * r;
      if (g) o = o * g[i];
      if (b) o = o + b[i];
      yr[i] = o;
    }
  }
}

void orc_rmsnorm_f32(const float *x, const float *g, float *y, int64_t M, int64_t D,
                     float eps) {
  const float inv_n = (float)(1.0 / (double)D);
  for (int64_t m = 0; m < M; m++) {
    const float *xr = x + m * D;
    float s = 0.0f;
    for (int64_t i = 0; i < D; i++) s += xr[i] * xr[i];
    const float r = 1.0f / sqrtf(s * inv_n + eps);
    for (int64_t i = 0; i < D; i++) y[m * D + i] = g ? (xr[i] * r) * g[i] : xr[i] * r;
  }
}

static void softmax_row(const float *x, float *y, int64_t N) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < N; i++) mx = x[i] > mx ? x[i] : mx;
  float s = 0.0f;
  for (int64_t i = 0; i < N; i++) {
    y[i] = orc_exp(x[i] - mx);
    s += y[i];
  }
  const float r = 1.0f / s;
  for (int64_t i = 0; i < N; i++) y[i] = y[i] * r;
}

void orc_softmax_f32(const float *x, float *y, int64_t M, int64_t N) {
  for (int64_t m = 0; m < M; m++) softmax_row(x + m * N, y + m * N, N);
}

static inline float gelu1(float x) {
  const float half = x * 0.5f;
  const float cube = (x * x) * x;
  const float in = x + cube * 0.044715f;
  const float z = in * 0.7978845608028654f;
  const float sg = 1.0f / (orc_exp(-(z * 2.0f)) + 1.0f); /* sigmoid(2z) */
  const float th = sg * 2.0f + -1.0f;
  return half * (th + 1.0f);
}

void orc_gelu_f32(const float *x, float *y, int64_t n) {
  for (int64_t i = 0; i < n; i++) y[i] = gelu1(x[i]);
}

/* One query row of attention: scores over Lk keys, masked where
 * allowed(j) is false (-inf), softmax, mix of v. */
static void attn_row(const float *q, const float *k, const float *v, int64_t k_stride,
                     const float *mask_row, int64_t n_allowed, float *scores, float *y,
                     int64_t Lk, int64_t D, float scale) {
  for (int64_t j = 0; j < Lk; j++) {
    const float *kr = k + j * k_stride;
    float acc = 0.0f;
    for (int64_t d = 0; d < D; d++) acc += q[d] * kr[d];
    float s = acc * scale;
    if (mask_row) s = s + mask_row[j];
    if (j >= n_allowed) s = -INFINITY;
    scores[j] = s;
  }
  softmax_row(scores, scores, Lk);
  for (int64_t d = 0; d < D; d++) {
    float acc = 0.0f;
    for (int64_t j = 0; j < Lk; j++) acc += scores[j] * v[j * k_stride + d];
    y[d] = acc;
  }
}

void orc_sdpa_f32(const float *q, const float *k, const float *v, const float *mask,
                  float *y, int64_t BH, int64_t Lq, int64_t Lk, int64_t D, int causal) {
  const float scale = (float)(1.0 / sqrt((double)D));
  float *scores = (float *)malloc(sizeof(float) * (size_t)(Lk > 0 ? Lk : 1));
  for (int64_t bh = 0; bh < BH; bh++) {
    for (int64_t i = 0; i < Lq; i++) {
      const int64_t allowed = causal ? (i + 1 < Lk ? i + 1 : Lk) : Lk;
      attn_row(q + (bh * Lq + i) * D, k + bh * Lk * D, v + bh * Lk * D, D,
               mask ? mask + i * Lk : NULL, allowed, scores, y + (bh * Lq + i) * D, Lk, D,
               scale);
    }
  }
  free(scores);
}

void orc_argmax_f32(const float *x, int32_t *out, int64_t M, int64_t N) {
  for (int64_t m = 0; m < M; m++) {
    const float *r = x + m * N;
    float mx = -INFINITY;
    for (int64_t i = 0; i < N; i++) mx = r[i] > mx ? r[i] : mx;
    /* max over (x == max) * (N - i); N - that is the first index */
    float best = 0.0f;
    for (int64_t i = 0; i < N; i++) {
      const float t = (r[i] == mx ? 1.0f : 0.0f) * (float)(N - i);
      best = t > best ? t : best;
    }
    out[m] = (int32_t)((float)N - best);
  }
}

void orc_embedding_f32(const float *w, const int32_t *idx, float *y, int64_t n_idx,
                       int64_t V, int64_t D) {
  for (int64_t i = 0; i < n_idx; i++) {
    const int64_t t = idx[i];
    if (t < 0 || t >= V)
      memset(y + i * D, 0, sizeof(float) * (size_t)D);
    else
      memcpy(y + i * D, w + t * D, sizeof(float) * (size_t)D);
  }
}

/* ---- GPT-2 -------------------------------------------------------------- */

struct OrcGPT2State {
  OrcGPT2 m;
  float **kv; /* per layer: [2][max_ctx][dim] (heads interleaved as [H][hd]) */
  float *x, *h, *qkv, *att, *tmp, *fc, *scores;
  int32_t cap_tok;
};

static int ensure_cap(OrcGPT2State *s, int32_t n_tok) {
  if (n_tok <= s->cap_tok) return 0;
  const OrcGPT2 *m = &s->m;
  const size_t d = (size_t)m->dim, T = (size_t)n_tok;
  float **bufs[] = {&s->x, &s->h, &s->qkv, &s->att, &s->tmp, &s->fc};
  const size_t sz[] = {T * d, T * d, T * 3 * d, T * d, T * d, T * 4 * d};
  for (int i = 0; i < 6; i++) {
    free(*bufs[i]);
    *bufs[i] = (float *)malloc(sizeof(float) * sz[i]);
    if (!*bufs[i]) return -1;
  }
  s->cap_tok = n_tok;
  return 0;
}

OrcGPT2State *orc_gpt2_state_new(const OrcGPT2 *m) {
  OrcGPT2State *s = (OrcGPT2State *)calloc(1, sizeof(OrcGPT2State));
  if (!s) return NULL;
  s->m = *m;
  s->kv = (float **)calloc((size_t)m->n_layers, sizeof(float *));
  for (int l = 0; l < m->n_layers; l++)
    s->kv[l] = (float *)calloc((size_t)2 * m->max_ctx * m->dim, sizeof(float));
  s->scores = (float *)malloc(sizeof(float) * (size_t)m->max_ctx);
  return s;
}

void orc_gpt2_state_free(OrcGPT2State *s) {
  if (!s) return;
  for (int l = 0; l < s->m.n_layers; l++) free(s->kv[l]);
  free(s->kv);
  free(s->x); free(s->h); free(s->qkv); free(s->att); free(s->tmp); free(s->fc);
  free(s->scores);
  free(s);
}

int32_t orc_gpt2_forward(OrcGPT2State *s, const int32_t *tokens, int32_t n_tok,
                         int32_t start_pos, float *logits) {
  const OrcGPT2 *m = &s->m;
  if (n_tok <= 0 || start_pos < 0 || start_pos + n_tok > m->max_ctx) return -1;
  if (ensure_cap(s, n_tok)) return -1;
  const int64_t d = m->dim, H = m->n_heads, hd = d / H, T = n_tok, F = 4 * d;
  const float scale = (float)(1.0 / sqrt((double)hd));

  /* h = tok_emb + pos_emb (thvm_gpt2.py:93-103) */
  for (int64_t t = 0; t < T; t++) {
    const int32_t id = tokens[t];
    for (int64_t i = 0; i < d; i++) {
      const float te = (id >= 0 && id < m->vocab) ? m->wte[(int64_t)id * d + i] : 0.0f;
      s->x[t * d + i] = te + m->wpe[(start_pos + t) * d + i];
    }
  }
  for (int l = 0; l < m->n_layers; l++) {
    /* attn(ln_1(x)) (thvm_gpt2.py:36-61) */
    orc_layernorm_f32(s->x, m->ln_1_w[l], m->ln_1_b[l], s->h, T, d, m->norm_eps);
    orc_linear_f32(s->h, m->c_attn_w[l], m->c_attn_b[l], s->qkv, T, d, 3 * d);
    float *kc = s->kv[l], *vc = s->kv[l] + (int64_t)m->max_ctx * d;
    for (int64_t t = 0; t < T; t++) {
      memcpy(kc + (start_pos + t) * d, s->qkv + t * 3 * d + d, sizeof(float) * (size_t)d);
      memcpy(vc + (start_pos + t) * d, s->qkv + t * 3 * d + 2 * d, sizeof(float) * (size_t)d);
    }
    const int64_t L = start_pos + T;
    for (int64_t hh = 0; hh < H; hh++) {
      for (int64_t t = 0; t < T; t++) {
        float sc_local[1024];
        float *sc = L <= 1024 ? sc_local : NULL;
        if (!sc) continue;
        /* mask triu(start_pos + 1) of -inf: key j allowed iff j <= start_pos + t */
        attn_row(s->qkv + t * 3 * d + hh * hd, kc + hh * hd, vc + hh * hd, d, NULL,
                 start_pos + t + 1, sc, s->att + t * d + hh * hd, L, hd, scale);
      }
    }
    orc_linear_f32(s->att, m->c_proj_w[l], m->c_proj_b[l], s->tmp, T, d, d);
    for (int64_t i = 0; i < T * d; i++) s->x[i] = s->x[i] + s->tmp[i];
    /* h + mlp(ln_2(h)) (thvm_gpt2.py:63-79) */
    orc_layernorm_f32(s->x, m->ln_2_w[l], m->ln_2_b[l], s->h, T, d, m->norm_eps);
    orc_linear_f32(s->h, m->c_fc_w[l], m->c_fc_b[l], s->fc, T, d, F);
    orc_gelu_f32(s->fc, s->fc, T * F);
    orc_linear_f32(s->fc, m->mlp_proj_w[l], m->mlp_proj_b[l], s->tmp, T, F, d);
    for (int64_t i = 0; i < T * d; i++) s->x[i] = s->x[i] + s->tmp[i];
  }
  /* logits of the last row, argmax (thvm_gpt2.py:106-124) */
  const float *last = s->x + (T - 1) * d;
  orc_layernorm_f32(last, m->ln_f_w, m->ln_f_b, s->h, 1, d, m->norm_eps);
  float *lg = logits ? logits : (float *)malloc(sizeof(float) * (size_t)m->vocab);
  orc_linear_f32(s->h, m->lm_head, NULL, lg, 1, d, m->vocab);
  int32_t id;
  orc_argmax_f32(lg, &id, 1, m->vocab);
  if (!logits) free(lg);
  return id;
}

int orc_gpt2_generate(const OrcGPT2 *m, const int32_t *prompt, int32_t n_prompt,
                      int32_t n_new, int32_t *out) {
  OrcGPT2State *s = orc_gpt2_state_new(m);
  if (!s) return -1;
  int32_t pos = 0;
  int32_t tok = orc_gpt2_forward(s, prompt, n_prompt, 0, NULL);
  pos = n_prompt;
  for (int32_t i = 0; i < n_new; i++) {
    if (tok < 0) break;
    out[i] = tok;
    if (i + 1 == n_new) break;
    tok = orc_gpt2_forward(s, &out[i], 1, pos, NULL);
    pos++;
  }
  orc_gpt2_state_free(s);
  return tok < 0 ? -1 : 0;
}

/* ---- low-precision storage formats ---------------------------------------- */

uint16_t orc_f32_to_bf16(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))   /* NaN: quiet, sign kept */
    return (uint16_t)(((u & 0x80000000u) | 0x7fc00000u) >> 16);
  const uint32_t lsb = (u >> 16) & 1u;                           /* ties to even */
  return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

float orc_bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float v;
  memcpy(&v, &u, 4);
  return v;
}

/* e4m3: bias 7, 3 mantissa bits, no infinities, 0x7f the NaN, max 448.
 * Finite inputs round to nearest even on the exact value (f64 holds every
 * f32 exactly, so the arithmetic below is exact up to the final rounding). */
uint8_t orc_f32_to_fp8e4m3(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  if ((u & 0x7f800000u) == 0x7f800000u) return (u & 0x007fffffu) ? (uint8_t)(sign | 0x7f) : (uint8_t)(sign | 0x7e);
  double a = fabs((double)v);
  if (a == 0.0) return sign;
  /* the e4m3 quantum at a: 2^(e - 3) for a in [2^e, 2^(e+1)), e >= -6; 2^-9 below */
  int e;
  frexp(a, &e);          /* a = f * 2^e, f in [0.5, 1) -> a in [2^(e-1), 2^e) */
  e -= 1;
  if (e < -6) e = -6;
  const double q = ldexp(1.0, e - 3);
  double n = a / q;       /* exact: q is a power of two */
  double r = floor(n);
  const double frac = n - r;
  if (frac > 0.5 || (frac == 0.5 && fmod(r, 2.0) != 0.0)) r += 1.0;
  double out = r * q;
  if (out > 448.0) out = 448.0;  /* finite overflow saturates */
  /* encode out (a multiple of its quantum, <= 448) */
  if (out == 0.0) return sign;
  int oe;
  frexp(out, &oe);
  oe -= 1;
  uint32_t code;
  if (oe < -6) {                         /* subnormal: out = m * 2^-9, m in 1..7 */
    code = (uint32_t)(out / ldexp(1.0, -9));
  } else {
    const uint32_t mant = (uint32_t)(out / ldexp(1.0, oe - 3)) - 8u;   /* 0..7 */
    code = ((uint32_t)(oe + 7) << 3) | mant;
  }
  return (uint8_t)(sign | code);
}

float orc_fp8e4m3_to_f32(uint8_t b) {
  const uint32_t e = (b >> 3) & 0xfu, m = b & 0x7u;
  const float s = (b & 0x80u) ? -1.0f : 1.0f;
  if (e == 0xfu && m == 0x7u) return s * NAN;
  if (e == 0) return s * (float)ldexp((double)m, -9);
  return s * (float)ldexp((double)(8u + m), (int)e - 10);
}

void orc_f32_to_bf16_n(const float *x, uint16_t *y, int64_t n) {
  for (int64_t i = 0; i < n; i++) y[i] = orc_f32_to_bf16(x[i]);
}

void orc_f32_to_fp8e4m3_n(const float *x, uint8_t *y, int64_t n) {
  for (int64_t i = 0; i < n; i++) y[i] = orc_f32_to_fp8e4m3(x[i]);
}

typedef struct {
  const float *x;
  const void *w;
  const float *scale;
  float *y;
  int64_t M, K, N;
  int kind;   /* 0 bf16, 1 fp8 + block scales */
} LowCtx;

static void low_rows(void *p, int64_t lo, int64_t hi) {
  const LowCtx *c = (const LowCtx *)p;
  const int64_t sc = (c->K + 127) / 128;
  for (int64_t m = 0; m < c->M; m++) {
    const float *xr = c->x + m * c->K;
    for (int64_t n = lo; n < hi; n++) {
      float acc = 0.0f;
      if (c->kind == 0) {
        const uint16_t *wr = (const uint16_t *)c->w + n * c->K;
        for (int64_t k = 0; k < c->K; k++) acc += xr[k] * orc_bf16_to_f32(wr[k]);
      } else {
        const uint8_t *wr = (const uint8_t *)c->w + n * c->K;
        const float *srow = c->scale + (n / 128) * sc;
        for (int64_t k = 0; k < c->K; k++) acc += xr[k] * (orc_fp8e4m3_to_f32(wr[k]) * srow[k / 128]);
      }
      c->y[m * c->N + n] = acc;
    }
  }
}

void orc_linear_bf16(const float *x, const uint16_t *w, float *y, int64_t M, int64_t K, int64_t N) {
  LowCtx c = {x, w, NULL, y, M, K, N, 0};
  par_for(N, 64, low_rows, &c);
}

void orc_linear_fp8bs(const float *x, const uint8_t *w, const float *scale, float *y, int64_t M,
                      int64_t K, int64_t N) {
  LowCtx c = {x, w, scale, y, M, K, N, 1};
  par_for(N, 64, low_rows, &c);
}

typedef struct {
  const uint16_t *a, *b;
  float *c;
  int64_t M, N, K;
} GemmCtx;

static void gemm_rows(void *p, int64_t lo, int64_t hi) {
  const GemmCtx *g = (const GemmCtx *)p;
  float *arow = (float *)malloc(sizeof(float) * (size_t)g->K);
  if (!arow) return;
  for (int64_t m = lo; m < hi; m++) {
    for (int64_t k = 0; k < g->K; k++) arow[k] = orc_bf16_to_f32(g->a[m * g->K + k]);
    for (int64_t n = 0; n < g->N; n++) {
      const uint16_t *br = g->b + n * g->K;
      float acc = 0.0f;
      for (int64_t k = 0; k < g->K; k++) acc += arow[k] * orc_bf16_to_f32(br[k]);
      g->c[m * g->N + n] = acc;
    }
  }
  free(arow);
}

void orc_gemm_bf16(const uint16_t *a, const uint16_t *b, float *c, int64_t M, int64_t N, int64_t K) {
  GemmCtx g = {a, b, c, M, N, K};
  par_for(M, 1, gemm_rows, &g);
}

/* ---- batched bf16 decode step (oracle.h) --------------------------------- */

static void round_bf16_inplace(float *x, int64_t n) {
  for (int64_t i = 0; i < n; i++) x[i] = orc_bf16_to_f32(orc_f32_to_bf16(x[i]));
}

static void add_bias_rows(float *y, const float *b, int64_t M, int64_t N) {
  if (!b) return;
  for (int64_t m = 0; m < M; m++)
    for (int64_t n = 0; n < N; n++) y[m * N + n] += b[n];
}

void orc_xl_step(const OrcXL *m, uint16_t *kv, const int32_t *tok, int32_t pos, float *logits, int32_t *next) {
  const int64_t B = m->batch, D = m->dim, H = m->heads, hd = D / H, F = 4 * D, V = m->vocab, ctx = m->max_ctx;
  float *h = (float *)calloc((size_t)(B * D), sizeof(float));
  float *x = (float *)malloc(sizeof(float) * (size_t)(B * F));
  float *y = (float *)malloc(sizeof(float) * (size_t)(B * (F > 3 * D ? F : 3 * D)));
  float *lg = logits ? logits : (float *)malloc(sizeof(float) * (size_t)(B * V));
  float *e = (float *)malloc(sizeof(float) * (size_t)ctx);
  if (!h || !x || !y || !lg || !e) goto out;
  for (int64_t b = 0; b < B; b++)
    for (int64_t d = 0; d < D; d++) {
      const float t = (tok[b] >= 0 && tok[b] < V) ? orc_bf16_to_f32(m->wte[(int64_t)tok[b] * D + d]) : 0.0f;
      h[b * D + d] = t + orc_bf16_to_f32(m->wpe[(int64_t)pos * D + d]);
    }
  for (int32_t l = 0; l < m->n_layers; l++) {
    uint16_t *kc = kv + (int64_t)l * 2 * B * ctx * D, *vc = kc + B * ctx * D;
    /* attention block */
    orc_layernorm_f32(h, m->ln_1_w[l], m->ln_1_b[l], x, B, D, m->norm_eps);
    round_bf16_inplace(x, B * D);
    orc_linear_bf16(x, m->c_attn_w[l], y, B, D, 3 * D);
    add_bias_rows(y, m->c_attn_b[l], B, 3 * D);
    for (int64_t b = 0; b < B; b++)
      for (int64_t d = 0; d < D; d++) {
        kc[(b * ctx + pos) * D + d] = orc_f32_to_bf16(y[b * 3 * D + D + d]);
        vc[(b * ctx + pos) * D + d] = orc_f32_to_bf16(y[b * 3 * D + 2 * D + d]);
      }
    const float scale = (float)(1.0 / sqrt((double)hd));
    for (int64_t b = 0; b < B; b++)
      for (int64_t hh = 0; hh < H; hh++) {
        const float *q = y + b * 3 * D + hh * hd;
        float mx = -INFINITY;
        for (int64_t j = 0; j <= pos; j++) {
          const uint16_t *kr = kc + (b * ctx + j) * D + hh * hd;
          float s = 0.0f;
          for (int64_t d = 0; d < hd; d++) s += (q[d] * scale) * orc_bf16_to_f32(kr[d]);
          e[j] = s;
          if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (int64_t j = 0; j <= pos; j++) {
          e[j] = expf(e[j] - mx);
          sum += e[j];
        }
        const float inv = 1.0f / sum;
        for (int64_t d = 0; d < hd; d++) {
          float acc = 0.0f;
          for (int64_t j = 0; j <= pos; j++) acc += e[j] * orc_bf16_to_f32(vc[(b * ctx + j) * D + hh * hd + d]);
          x[b * D + hh * hd + d] = orc_bf16_to_f32(orc_f32_to_bf16(acc * inv));
        }
      }
    orc_linear_bf16(x, m->c_proj_w[l], y, B, D, D);
    add_bias_rows(y, m->c_proj_b[l], B, D);
    for (int64_t i = 0; i < B * D; i++) h[i] += y[i];
    /* MLP block */
    orc_layernorm_f32(h, m->ln_2_w[l], m->ln_2_b[l], x, B, D, m->norm_eps);
    round_bf16_inplace(x, B * D);
    orc_linear_bf16(x, m->c_fc_w[l], y, B, D, F);
    add_bias_rows(y, m->c_fc_b[l], B, F);
    orc_gelu_f32(y, x, B * F);
    round_bf16_inplace(x, B * F);
    orc_linear_bf16(x, m->mlp_proj_w[l], y, B, F, D);
    add_bias_rows(y, m->mlp_proj_b[l], B, D);
    for (int64_t i = 0; i < B * D; i++) h[i] += y[i];
  }
  orc_layernorm_f32(h, m->ln_f_w, m->ln_f_b, x, B, D, m->norm_eps);
  round_bf16_inplace(x, B * D);
  orc_linear_bf16(x, m->lm_head, lg, B, D, V);
  for (int64_t b = 0; b < B; b++) {
    int64_t bi = 0;
    for (int64_t v = 1; v < V; v++)
      if (lg[b * V + v] > lg[b * V + bi]) bi = v;
    next[b] = (int32_t)bi;
  }
out:
  free(h);
  free(x);
  free(y);
  free(e);
  if (!logits) free(lg);
}

/* ---- batched MoE decode step (oracle.h) ------------------------------------ */

static float bfr_(float v) { return orc_bf16_to_f32(orc_f32_to_bf16(v)); }

static void rms_bf16(const float *x, const float *g, float *y, int64_t M, int64_t D, float eps) {
  for (int64_t m = 0; m < M; m++) {
    float ss = 0.0f;
    for (int64_t i = 0; i < D; i++) ss += x[m * D + i] * x[m * D + i];
    const float inv = 1.0f / sqrtf(ss * (1.0f / (float)D) + eps);
    for (int64_t i = 0; i < D; i++) y[m * D + i] = bfr_((x[m * D + i] * inv) * g[i]);
  }
}

/* y[m][n] = sum_k x[m][k] * (fp8(w[n][k]) * scale[n/128][k/128]) */
static void linear_fp8_rows(const float *x, const uint8_t *w, const float *sc, float *y, int64_t M, int64_t K,
                            int64_t N) {
  orc_linear_fp8bs(x, w, sc, y, M, K, N);
}

static float silu_(float g) { return g / (1.0f + expf(-g)); }

void orc_ds_step(const OrcDS *m, uint16_t *cache_c, uint16_t *cache_pe, const int32_t *tok, int32_t pos,
                 float *logits, int32_t *next) {
  const int64_t B = m->batch, D = m->dim, H = m->heads, KV = m->kv_lora, DN = m->d_nope, DR = m->d_rope,
                DV = m->d_v, QS = DN + DR, ctx = m->max_ctx, V = m->vocab, E = m->n_exp, K = m->top_k,
                I = m->moe_inter, DI = m->dense_inter, NQ = H * QS + KV + DR, half = DR / 2;
  const int64_t big = (2 * DI > NQ ? 2 * DI : NQ) > 2 * I ? (2 * DI > NQ ? 2 * DI : NQ) : 2 * I;
  float *h = (float *)calloc((size_t)(B * D), sizeof(float));
  float *xn = (float *)malloc(sizeof(float) * (size_t)(B * (DI > D ? DI : D)));
  float *y = (float *)malloc(sizeof(float) * (size_t)(B * big));
  float *o = (float *)malloc(sizeof(float) * (size_t)(B * H * DV));
  float *qo = (float *)malloc(sizeof(float) * (size_t)(B * H * QS));
  float *lg = logits ? logits : (float *)malloc(sizeof(float) * (size_t)(B * V));
  float *sc = (float *)malloc(sizeof(float) * (size_t)ctx), *qlat = (float *)malloc(sizeof(float) * (size_t)KV);
  float *olat = (float *)malloc(sizeof(float) * (size_t)KV), *t1 = (float *)malloc(sizeof(float) * (size_t)(2 * I));
  float *av = (float *)malloc(sizeof(float) * (size_t)I), *yv = (float *)malloc(sizeof(float) * (size_t)D);
  float *rl = (float *)malloc(sizeof(float) * (size_t)(B * (E > 0 ? E : 1)));
  if (!h || !xn || !y || !o || !qo || !lg || !sc || !qlat || !olat || !t1 || !av || !yv || !rl) goto out;
  for (int64_t b = 0; b < B; b++)
    for (int64_t d = 0; d < D; d++)
      h[b * D + d] = (tok[b] >= 0 && tok[b] < V) ? orc_bf16_to_f32(m->embed[(int64_t)tok[b] * D + d]) : 0.0f;
  for (int32_t l = 0; l < m->n_layers; l++) {
    uint16_t *cc = cache_c + (int64_t)l * B * ctx * KV, *cp = cache_pe + (int64_t)l * B * ctx * DR;
    rms_bf16(h, m->attn_norm[l], xn, B, D, m->eps);
    orc_linear_bf16(xn, m->w_qkva[l], y, B, D, NQ);
    for (int64_t b = 0; b < B; b++) {
      const float *q = y + b * NQ, *kva = y + b * NQ + H * QS;
      float *qb = qo + b * H * QS;
      for (int64_t hh = 0; hh < H; hh++) {
        for (int64_t d = 0; d < DN; d++) qb[hh * QS + d] = bfr_(q[hh * QS + d]);
        for (int64_t j = 0; j < half; j++) {
          const float xe = bfr_(q[hh * QS + DN + 2 * j]), xo = bfr_(q[hh * QS + DN + 2 * j + 1]);
          const float c = m->cos_t[(int64_t)pos * DR + j], s = m->sin_t[(int64_t)pos * DR + j];
          qb[hh * QS + DN + j] = bfr_(xe * c - xo * s);
          qb[hh * QS + DN + half + j] = bfr_(xo * c + xe * s);
        }
      }
      float ss = 0.0f;
      for (int64_t i = 0; i < KV; i++) ss += bfr_(kva[i]) * bfr_(kva[i]);
      const float inv = 1.0f / sqrtf(ss * (1.0f / (float)KV) + m->eps);
      for (int64_t i = 0; i < KV; i++)
        cc[(b * ctx + pos) * KV + i] = orc_f32_to_bf16((bfr_(kva[i]) * inv) * m->kv_norm[l][i]);
      for (int64_t j = 0; j < half; j++) {
        const float xe = bfr_(kva[KV + 2 * j]), xo = bfr_(kva[KV + 2 * j + 1]);
        const float c = m->cos_t[(int64_t)pos * DR + j], s = m->sin_t[(int64_t)pos * DR + j];
        cp[(b * ctx + pos) * DR + j] = orc_f32_to_bf16(xe * c - xo * s);
        cp[(b * ctx + pos) * DR + half + j] = orc_f32_to_bf16(xo * c + xe * s);
      }
    }
    for (int64_t b = 0; b < B; b++)
      for (int64_t hh = 0; hh < H; hh++) {
        const float *qb = qo + (b * H + hh) * QS;
        const uint16_t *wk = m->w_uk[l] + hh * DN * KV, *wv = m->w_uv[l] + hh * DV * KV;
        for (int64_t k = 0; k < KV; k++) {
          float a = 0.0f;
          for (int64_t d = 0; d < DN; d++) a += qb[d] * orc_bf16_to_f32(wk[d * KV + k]);
          qlat[k] = a;
        }
        float mx = -INFINITY;
        for (int64_t t = 0; t <= pos; t++) {
          float s = 0.0f;
          for (int64_t k = 0; k < KV; k++) s += qlat[k] * orc_bf16_to_f32(cc[(b * ctx + t) * KV + k]);
          for (int64_t r = 0; r < DR; r++) s += qb[DN + r] * orc_bf16_to_f32(cp[(b * ctx + t) * DR + r]);
          sc[t] = s * m->scale;
          if (sc[t] > mx) mx = sc[t];
        }
        float sum = 0.0f;
        for (int64_t t = 0; t <= pos; t++) {
          sc[t] = expf(sc[t] - mx);
          sum += sc[t];
        }
        const float inv = 1.0f / sum;
        for (int64_t k = 0; k < KV; k++) {
          float a = 0.0f;
          for (int64_t t = 0; t <= pos; t++) a += sc[t] * orc_bf16_to_f32(cc[(b * ctx + t) * KV + k]);
          olat[k] = a * inv;
        }
        for (int64_t r = 0; r < DV; r++) {
          float a = 0.0f;
          for (int64_t k = 0; k < KV; k++) a += olat[k] * orc_bf16_to_f32(wv[r * KV + k]);
          o[b * H * DV + hh * DV + r] = bfr_(a);
        }
      }
    orc_linear_bf16(o, m->w_o[l], y, B, H * DV, D);
    for (int64_t i = 0; i < B * D; i++) h[i] += y[i];
    rms_bf16(h, m->ffn_norm[l], xn, B, D, m->eps);
    if (l < m->n_dense) {
      float *gu = y;
      orc_linear_bf16(xn, m->d_gu[l], gu, B, D, 2 * DI);
      float *a = (float *)malloc(sizeof(float) * (size_t)(B * DI));
      float *dn = (float *)malloc(sizeof(float) * (size_t)(B * D));
      if (a && dn) {
        for (int64_t b = 0; b < B; b++)
          for (int64_t j = 0; j < DI; j++) a[b * DI + j] = bfr_(silu_(gu[b * 2 * DI + j]) * gu[b * 2 * DI + DI + j]);
        orc_linear_bf16(a, m->d_down[l], dn, B, DI, D);
        for (int64_t i = 0; i < B * D; i++) h[i] += dn[i];
      }
      free(a);
      free(dn);
    } else {
      orc_linear_bf16(xn, m->router[l], rl, B, D, E);
      for (int64_t b = 0; b < B; b++) {
        float mx = -INFINITY, sum = 0.0f, pr[64];
        for (int64_t e = 0; e < E; e++) mx = rl[b * E + e] > mx ? rl[b * E + e] : mx;
        for (int64_t e = 0; e < E; e++) sum += expf(rl[b * E + e] - mx);
        for (int64_t e = 0; e < E; e++) pr[e] = expf(rl[b * E + e] - mx) / sum;
        int used[64] = {0};
        const int64_t n_all = K + m->n_shared;
        for (int64_t k = 0; k < n_all; k++) {
          int64_t e;
          float w;
          if (k < K) {   /* the largest remaining prob; ties to the lowest id */
            e = -1;
            for (int64_t c = 0; c < E; c++)
              if (!used[c] && (e < 0 || pr[c] > pr[e])) e = c;
            used[e] = 1;
            w = pr[e];
          } else {
            e = E + (k - K);
            w = 1.0f;
          }
          const int64_t sgu = ((2 * I + 127) / 128) * (D / 128), sd = (D / 128) * ((I + 127) / 128);
          linear_fp8_rows(xn + b * D, m->e_gu[l] + e * 2 * I * D, m->e_gu_s[l] + e * sgu, t1, 1, D, 2 * I);
          for (int64_t j = 0; j < I; j++) av[j] = bfr_(silu_(t1[j]) * t1[I + j]);
          linear_fp8_rows(av, m->e_d[l] + e * D * I, m->e_d_s[l] + e * sd, yv, 1, I, D);
          for (int64_t d = 0; d < D; d++) h[b * D + d] += w * yv[d];
        }
      }
    }
  }
  rms_bf16(h, m->norm_f, xn, B, D, m->eps);
  orc_linear_bf16(xn, m->lm_head, lg, B, D, V);
  for (int64_t b = 0; b < B; b++) {
    int64_t bi = 0;
    for (int64_t v = 1; v < V; v++)
      if (lg[b * V + v] > lg[b * V + bi]) bi = v;
    next[b] = (int32_t)bi;
  }
out:
  free(h);
  free(xn);
  free(y);
  free(o);
  free(qo);
  free(sc);
  free(qlat);
  free(olat);
  free(t1);
  free(av);
  free(yv);
  free(rl);
  if (!logits) free(lg);
}
