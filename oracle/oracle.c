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

void orc_xl_step(const OrcXL *m, void *kv, const int32_t *tok, int32_t pos, float *logits, int32_t *next) {
  const int64_t B = m->batch, D = m->dim, H = m->heads, hd = D / H, F = 4 * D, V = m->vocab, ctx = m->max_ctx;
  const int exact = m->exact != 0;
  /* activations stored as bf16 by the device round here; `exact` keeps f32 */
#define XL_ROUND(ptr, n) \
  do {                                 \
    if (!exact) round_bf16_inplace((ptr), (n)); \
  } while (0)
  float *h = (float *)calloc((size_t)(B * D), sizeof(float));
  float *x = (float *)malloc(sizeof(float) * (size_t)(B * F));
  float *y = (float *)malloc(sizeof(float) * (size_t)(B * (F > 3 * D ? F : 3 * D)));
  float *lg = logits ? logits : (float *)malloc(sizeof(float) * (size_t)(B * V));
  float *e = (float *)malloc(sizeof(float) * (size_t)ctx);
  float *kr = (float *)malloc(sizeof(float) * (size_t)(ctx * hd)), *vr = (float *)malloc(sizeof(float) * (size_t)(ctx * hd));
  if (!h || !x || !y || !lg || !e || !kr || !vr) goto out;
  for (int64_t b = 0; b < B; b++)
    for (int64_t d = 0; d < D; d++) {
      const float t = (tok[b] >= 0 && tok[b] < V) ? orc_bf16_to_f32(m->wte[(int64_t)tok[b] * D + d]) : 0.0f;
      h[b * D + d] = t + orc_bf16_to_f32(m->wpe[(int64_t)pos * D + d]);
    }
  const float scale = (float)(1.0 / sqrt((double)hd));
  for (int32_t l = 0; l < m->n_layers; l++) {
    const int64_t lo = (int64_t)l * 2 * B * ctx * D, vo = lo + B * ctx * D;
    uint16_t *kc = (uint16_t *)kv + lo, *vc = (uint16_t *)kv + vo;
    float *kcf = (float *)kv + lo, *vcf = (float *)kv + vo;
    /* attention block */
    orc_layernorm_f32(h, m->ln_1_w[l], m->ln_1_b[l], x, B, D, m->norm_eps);
    XL_ROUND(x, B * D);
    orc_linear_bf16(x, m->c_attn_w[l], y, B, D, 3 * D);
    add_bias_rows(y, m->c_attn_b[l], B, 3 * D);
    for (int64_t b = 0; b < B; b++)
      for (int64_t d = 0; d < D; d++) {
        const int64_t at = (b * ctx + pos) * D + d;
        if (exact) {
          kcf[at] = y[b * 3 * D + D + d];
          vcf[at] = y[b * 3 * D + 2 * D + d];
        } else {
          kc[at] = orc_f32_to_bf16(y[b * 3 * D + D + d]);
          vc[at] = orc_f32_to_bf16(y[b * 3 * D + 2 * D + d]);
        }
      }
    /* the reference's attention row (the GPT-2 forward's attn_row: (q . k) *
     * scale, softmax, mix) over the cached rows 0..pos */
    for (int64_t b = 0; b < B; b++)
      for (int64_t hh = 0; hh < H; hh++) {
        for (int64_t j = 0; j <= pos; j++)
          for (int64_t d = 0; d < hd; d++) {
            const int64_t at = (b * ctx + j) * D + hh * hd + d;
            kr[j * hd + d] = exact ? kcf[at] : orc_bf16_to_f32(kc[at]);
            vr[j * hd + d] = exact ? vcf[at] : orc_bf16_to_f32(vc[at]);
          }
        attn_row(y + b * 3 * D + hh * hd, kr, vr, hd, NULL, (int64_t)pos + 1, e, x + b * D + hh * hd,
                 (int64_t)pos + 1, hd, scale);
      }
    XL_ROUND(x, B * D);
    orc_linear_bf16(x, m->c_proj_w[l], y, B, D, D);
    add_bias_rows(y, m->c_proj_b[l], B, D);
    for (int64_t i = 0; i < B * D; i++) h[i] += y[i];
    /* MLP block */
    orc_layernorm_f32(h, m->ln_2_w[l], m->ln_2_b[l], x, B, D, m->norm_eps);
    XL_ROUND(x, B * D);
    orc_linear_bf16(x, m->c_fc_w[l], y, B, D, F);
    add_bias_rows(y, m->c_fc_b[l], B, F);
    orc_gelu_f32(y, x, B * F);
    XL_ROUND(x, B * F);
    orc_linear_bf16(x, m->mlp_proj_w[l], y, B, F, D);
    add_bias_rows(y, m->mlp_proj_b[l], B, D);
    for (int64_t i = 0; i < B * D; i++) h[i] += y[i];
  }
  orc_layernorm_f32(h, m->ln_f_w, m->ln_f_b, x, B, D, m->norm_eps);
  XL_ROUND(x, B * D);
#undef XL_ROUND
  orc_linear_bf16(x, m->lm_head, lg, B, D, V);
  for (int64_t b = 0; b < B; b++) orc_argmax_f32(lg + b * V, next + b, 1, V);
out:
  free(h);
  free(x);
  free(y);
  free(e);
  free(kr);
  free(vr);
  if (!logits) free(lg);
}

/* ---- DeepSeek-V2 decode stages shared by the two MoE steps below ------------
 * Each restates one CPU twin of the reference's decode step
 * (bench/dsv2_decode_bench.c, the plain-C sources its custom kernels carry for
 * the CPU backend); both orc_ds_ref_step (the reference's batch-1 bf16 step,
 * pinned to its own output) and orc_ds_step (the batched config-5
 * composition) call them, so the attention, rotary, cache and routing
 * arithmetic of the batched step is the pinned one. */

static float bfr_(float v) { return orc_bf16_to_f32(orc_f32_to_bf16(v)); }

/* gred_q (bench/dsv2_decode_bench.c:435-485): the q row [H][DN + DR] as f32
 * projection outputs -> qb: nope columns rounded to bf16; each rope pair
 * (2j, 2j + 1) rounded to bf16, rotated by the YaRN table row p into columns
 * j and DR/2 + j, rounded to bf16. */
static void ds_q_post(const float *q, float *qb, int64_t H, int64_t DN, int64_t DR, const float *cos_t,
                      const float *sin_t, int64_t p) {
  const int64_t QS = DN + DR, half = DR / 2;
  for (int64_t hh = 0; hh < H; hh++) {
    for (int64_t d = 0; d < DN; d++) qb[hh * QS + d] = bfr_(q[hh * QS + d]);
    for (int64_t j = 0; j < half; j++) {
      const float xe = bfr_(q[hh * QS + DN + 2 * j]), xo = bfr_(q[hh * QS + DN + 2 * j + 1]);
      const float c = cos_t[p * DR + j], s = sin_t[p * DR + j];
      qb[hh * QS + DN + j] = bfr_(xe * c - xo * s);
      qb[hh * QS + DN + half + j] = bfr_(xo * c + xe * s);
    }
  }
}

/* kv_prep (bench/dsv2_decode_bench.c:487-556): kva = [latent KV | rope DR] f32
 * projection outputs; v = bf16(latent), inv = 1 / sqrt(sum v^2 / KV + eps) (one
 * f32 sum in index order), cache row = bf16(v * inv * g); the rope pair rotated
 * as in ds_q_post into the key row. */
static void ds_kv_post(const float *kva, const float *g, uint16_t *c_row, uint16_t *pe_row, int64_t KV,
                       int64_t DR, const float *cos_t, const float *sin_t, int64_t p, float eps) {
  const int64_t half = DR / 2;
  float ss = 0.0f;
  for (int64_t t = 0; t < KV; t++) {
    const float v = bfr_(kva[t]);
    ss += v * v;
  }
  const float inv = 1.0f / sqrtf(ss * (1.0f / (float)KV) + eps);
  for (int64_t t = 0; t < KV; t++) c_row[t] = orc_f32_to_bf16((bfr_(kva[t]) * inv) * g[t]);
  for (int64_t j = 0; j < half; j++) {
    const float xe = bfr_(kva[KV + 2 * j]), xo = bfr_(kva[KV + 2 * j + 1]);
    const float c = cos_t[p * DR + j], s = sin_t[p * DR + j];
    pe_row[j] = orc_f32_to_bf16(xe * c - xo * s);
    pe_row[half + j] = orc_f32_to_bf16(xo * c + xe * s);
  }
}

/* One head of the absorbed MLA (mla_qlat / mla_score / mla_mix / mla_o,
 * bench/dsv2_decode_bench.c:638-785), over the L cache rows c [L][KV] and
 * pe [L][DR] (bf16): qlat[k] = sum_d q_nope[d] * W_uk[d][k]; score_j =
 * (sum_k qlat[k] c_j[k] + sum_r q_pe[r] pe_j[r]) * scale (one accumulator);
 * max (strict >), e_j = expf(score_j - max), sum in j order, p_j = e_j / sum;
 * olat[k] = sum_j p_j c_j[k]; o[r] = bf16(sum_k olat[k] W_uv[r][k]).  qb holds
 * the head's bf16-rounded q (DN nope then DR rope values); sm (>= L) gets the
 * p_j; qlat_out / olat_out (KV each) may be scratch. */
static void ds_mla_head(const float *qb, const uint16_t *wuk, const uint16_t *wuv, const uint16_t *c,
                        const uint16_t *pe, int64_t L, int64_t KV, int64_t DN, int64_t DR, int64_t DV, float scale,
                        float *qlat, float *sm, float *olat, float *o) {
  for (int64_t k = 0; k < KV; k++) {
    float acc = 0.0f;
    for (int64_t d = 0; d < DN; d++) acc += qb[d] * orc_bf16_to_f32(wuk[d * KV + k]);
    qlat[k] = acc;
  }
  float gmax = -1e30f;
  for (int64_t j = 0; j < L; j++) {
    float s = 0.0f;
    for (int64_t k = 0; k < KV; k++) s += qlat[k] * orc_bf16_to_f32(c[j * KV + k]);
    for (int64_t r = 0; r < DR; r++) s += qb[DN + r] * orc_bf16_to_f32(pe[j * DR + r]);
    sm[j] = s * scale;
    if (sm[j] > gmax) gmax = sm[j];
  }
  float gsum = 0.0f;
  for (int64_t j = 0; j < L; j++) {
    sm[j] = expf(sm[j] - gmax);
    gsum += sm[j];
  }
  for (int64_t j = 0; j < L; j++) sm[j] = sm[j] / gsum;
  for (int64_t k = 0; k < KV; k++) {
    float a = 0.0f;
    for (int64_t j = 0; j < L; j++) a += sm[j] * orc_bf16_to_f32(c[j * KV + k]);
    olat[k] = a;
  }
  for (int64_t r = 0; r < DV; r++) {
    float acc = 0.0f;
    for (int64_t k = 0; k < KV; k++) acc += olat[k] * orc_bf16_to_f32(wuv[r * KV + k]);
    o[r] = bfr_(acc);
  }
}

/* route (bench/dsv2_decode_bench.c:787-863): over the E router logits g, mx =
 * the max (strict > from g[0]), sum = sum_e expf(g[e] - mx) in e order; K
 * rounds each take the largest remaining LOGIT (strict >, so ties go to the
 * lowest id) with weight expf(g - mx) / sum (no renormalisation). */
static void ds_route(const float *g, int64_t E, int64_t K, int32_t *sel, float *probs) {
  float mx = g[0];
  for (int64_t e = 1; e < E; e++)
    if (g[e] > mx) mx = g[e];
  float sum = 0.0f;
  for (int64_t e = 0; e < E; e++) sum += expf(g[e] - mx);
  for (int64_t kk = 0; kk < K; kk++) {
    int64_t best = -1;
    float bv = -3.4e38f;
    for (int64_t e = 0; e < E; e++) {
      int used = 0;
      for (int64_t j = 0; j < kk; j++) used |= sel[j] == e;
      if (!used && g[e] > bv) {
        bv = g[e];
        best = e;
      }
    }
    sel[kk] = (int32_t)best;
    probs[kk] = best >= 0 ? expf(g[best] - mx) / sum : 0.0f;
  }
}

void orc_ds_route(const float *g, int64_t B, int64_t E, int64_t K, int32_t *sel, float *probs) {
  for (int64_t b = 0; b < B; b++) ds_route(g + b * E, E, K, sel + b * K, probs + b * K);
}

/* ---- batched MoE decode step (oracle.h) ------------------------------------ */

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
                I = m->moe_inter, DI = m->dense_inter, NQ = H * QS + KV + DR;
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
      ds_q_post(y + b * NQ, qo + b * H * QS, H, DN, DR, m->cos_t, m->sin_t, pos);
      ds_kv_post(y + b * NQ + H * QS, m->kv_norm[l], cc + (b * ctx + pos) * KV, cp + (b * ctx + pos) * DR, KV, DR,
                 m->cos_t, m->sin_t, pos, m->eps);
    }
    for (int64_t b = 0; b < B; b++)
      for (int64_t hh = 0; hh < H; hh++)
        ds_mla_head(qo + (b * H + hh) * QS, m->w_uk[l] + hh * DN * KV, m->w_uv[l] + hh * DV * KV,
                    cc + b * ctx * KV, cp + b * ctx * DR, (int64_t)pos + 1, KV, DN, DR, DV, m->scale, qlat, sc,
                    olat, o + b * H * DV + hh * DV);
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
        int32_t sel[64];
        float pr[64];
        ds_route(rl + b * E, E, K, sel, pr);
        const int64_t n_all = K + m->n_shared;
        for (int64_t k = 0; k < n_all; k++) {
          const int64_t e = k < K ? sel[k] : E + (k - K);
          const float w = k < K ? pr[k] : 1.0f;
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

/* ---- the reference's own batch-1 bf16 decode step (oracle.h) ---------------- */

/* gemv_pick_sk (bench/dsv2_decode_bench.c:1043-1048): the K split of a
 * [K] x [K, N] product. */
static int64_t ref_pick_sk(int64_t K, int64_t N) {
  const int64_t gx = (N + 255) / 256;
  int64_t sk = 1;
  while (gx * sk < 232 && sk * 64 < K) sk *= 2;
  return sk;
}

/* gemv phase 1 + the in-order fold of its partials (src_gemv / src_gred,
 * bench/dsv2_decode_bench.c:1054-1110): chunk = ceil(K / sk); part_s[n] = f32
 * sum over k in chunk s of x[k] * w[k][n] (w {in, out}, bf16 or f32); y[n] =
 * sum_s part_s[n] in s order from 0.  Folds that round (gred's bf16 output)
 * round y afterwards. */
static void ref_gemv(const float *x, const void *w, int w_f32, float *y, int64_t K, int64_t N, int64_t sk) {
  const int64_t chunk = (K + sk - 1) / sk;
  const uint16_t *wb = (const uint16_t *)w;
  const float *wf = (const float *)w;
  for (int64_t n = 0; n < N; n++) {
    float s = 0.0f;
    for (int64_t p = 0; p < sk; p++) {
      const int64_t k0 = p * chunk, k1 = k0 + chunk > K ? K : k0 + chunk;
      float acc = 0.0f;
      for (int64_t k = k0; k < k1; k++) acc += x[k] * (w_f32 ? wf[k * N + n] : orc_bf16_to_f32(wb[k * N + n]));
      s += acc;
    }
    y[n] = s;
  }
}

/* rms1 / rms_f CPU twins (bench/dsv2_decode_bench.c:397-429): one f32 sum of
 * squares in index order, inv = 1 / sqrtf(ss * (1/K) + eps), y = x * inv * w
 * (rounded to bf16 when round_bf16). */
static void ref_rms(const float *x, const float *w, float *y, int64_t K, float eps, int round_bf16) {
  float ss = 0.0f;
  for (int64_t i = 0; i < K; i++) ss += x[i] * x[i];
  const float inv = 1.0f / sqrtf(ss * (1.0f / (float)K) + eps);
  for (int64_t i = 0; i < K; i++) {
    const float v = (x[i] * inv) * w[i];
    y[i] = round_bf16 ? bfr_(v) : v;
  }
}

int32_t orc_ds_ref_step(const OrcDSRef *m, uint16_t *ckv, uint16_t *kpe, int32_t tok, int32_t len, float *logits,
                        OrcDSRefTrace *tr) {
  const int64_t D = m->dim, H = m->heads, KV = m->kv_lora, DN = m->d_nope, DR = m->d_rope, DV = m->d_v,
                QS = DN + DR, ML = m->max_seq, V = m->vocab, E = m->n_exp, K = m->top_k, MI = m->moe_inter,
                SI = m->moe_inter * m->n_shared, DI = m->dense_inter, NQ = H * QS, NQKV = NQ + KV + DR;
  const int64_t p = (int64_t)len - 1;
  const int64_t sk_qkv = ref_pick_sk(D, NQ), sk_o = ref_pick_sk(H * DV, D), sk_gate = ref_pick_sk(D, E),
                sk_ffw = ref_pick_sk(D, DI), sk_down = ref_pick_sk(DI, D), sk_lm = ref_pick_sk(D, V);
  int64_t wide = DI > NQKV ? DI : NQKV;
  wide = wide > D ? wide : D;
  wide = wide > E ? wide : E;
  float *x = (float *)malloc(sizeof(float) * (size_t)D), *x1 = (float *)malloc(sizeof(float) * (size_t)D);
  float *xn = (float *)malloc(sizeof(float) * (size_t)D), *xn2f = (float *)malloc(sizeof(float) * (size_t)D);
  float *xn2b = (float *)malloc(sizeof(float) * (size_t)D), *y = (float *)malloc(sizeof(float) * (size_t)wide);
  float *u = (float *)malloc(sizeof(float) * (size_t)wide), *qb = (float *)malloc(sizeof(float) * (size_t)NQ);
  float *ql = (float *)malloc(sizeof(float) * (size_t)(H * KV)), *ol = (float *)malloc(sizeof(float) * (size_t)(H * KV));
  float *sm = (float *)calloc((size_t)(H * ML), sizeof(float)), *ob = (float *)malloc(sizeof(float) * (size_t)(H * DV));
  float *hbuf = (float *)malloc(sizeof(float) * (size_t)(K * MI + SI));
  float *lg = logits ? logits : (float *)malloc(sizeof(float) * (size_t)V);
  int32_t next = -1;
  if (!x || !x1 || !xn || !xn2f || !xn2b || !y || !u || !qb || !ql || !ol || !sm || !ob || !hbuf || !lg) goto out;
  if (tr && tr->sm) memcpy(sm, tr->sm, sizeof(float) * (size_t)(H * ML));
  for (int64_t i = 0; i < D; i++) x[i] = orc_bf16_to_f32(m->embed[(int64_t)tok * D + i]);   /* embed_row */
  for (int32_t l = 0; l < m->n_layers; l++) {
    uint16_t *cl = ckv + (int64_t)l * ML * KV, *pl = kpe + (int64_t)l * ML * DR;
    ref_rms(x, m->win[l], xn, D, m->eps, 1);
    /* q | kv GEMV: the split factor is the q projection's pick (model_init :2228) */
    ref_gemv(xn, m->wqkv[l], 0, y, D, NQKV, sk_qkv);
    ds_q_post(y, qb, H, DN, DR, m->cos_t, m->sin_t, p);
    ds_kv_post(y + NQ, m->wkvn[l], cl + p * KV, pl + p * DR, KV, DR, m->cos_t, m->sin_t, p, m->eps);
    for (int64_t hh = 0; hh < H; hh++)
      ds_mla_head(qb + hh * QS, m->wuk[l] + hh * DN * KV, m->wuv[l] + hh * DV * KV, cl, pl, len, KV, DN, DR, DV,
                  m->scale, ql + hh * KV, sm + hh * ML, ol + hh * KV, ob + hh * DV);
    /* gemv_o + gred_o_rms (:558-611): x1 = bf16(x + bf16(o W_o)); xn2 = rms(x1) as f32 and bf16 */
    ref_gemv(ob, m->wo[l], 0, y, H * DV, D, sk_o);
    for (int64_t i = 0; i < D; i++) x1[i] = bfr_(x[i] + bfr_(y[i]));
    ref_rms(x1, m->wpost[l], xn2f, D, m->eps, 0);
    for (int64_t i = 0; i < D; i++) xn2b[i] = bfr_(xn2f[i]);
    if (l < m->first_dense) {
      /* gemv_run (gate, up) with bf16 outputs, the scheduler's silu(g) * u
       * (:2042-2050: x * recip(1 + exp2(x * -log2e)) with bf16 CONSTs: the
       * constant is -log2e rounded through bf16 storage, -1.4453125
       * (src/uop/const.c:28), and the CPU backend holds a non-f32 CONST as a
       * double, so the chain runs in doubles with libm's exp2
       * (src/backend/cpu/uop_walk.c:354-356, :720-729), rounded once to bf16;
       * then gemv_sk + gred_down (:613-636) */
      ref_gemv(xn2b, m->wg1[l], 0, y, D, DI, sk_ffw);
      ref_gemv(xn2b, m->wu1[l], 0, u, D, DI, sk_ffw);
      const double c = (double)bfr_(-1.4426950408889634f);
      for (int64_t j = 0; j < DI; j++) {
        y[j] = bfr_(y[j]);
        u[j] = bfr_(u[j]);
        if (tr && tr->g1o) tr->g1o[j] = orc_f32_to_bf16(y[j]);
        if (tr && tr->u1o) tr->u1o[j] = orc_f32_to_bf16(u[j]);
        const double g = (double)y[j];
        const double sig = 1.0 / (1.0 + exp2(g * c));
        y[j] = bfr_((float)((g * sig) * (double)u[j]));
      }
      float *dn = u;
      ref_gemv(y, m->wd1[l], 0, dn, DI, D, sk_down);
      for (int64_t i = 0; i < D; i++) x[i] = bfr_(x1[i] + bfr_(dn[i]));
    } else {
      /* gemv_sk(gate) on the f32 xn2 with f32 weights, route, moe_full_h,
       * moe_full_out (:865-965) */
      int32_t sel[64];
      float probs[64];
      ref_gemv(xn2f, m->gate[l], 1, y, D, E, sk_gate);
      ds_route(y, E, K, sel, probs);
      for (int64_t w = 0; w < K * MI + SI; w++) {
        const uint16_t *wgi, *wui;
        if (w < K * MI) {
          const int64_t se = sel[w / MI], i = w % MI;
          wgi = m->wg[l] + (se * MI + i) * D;
          wui = m->wu[l] + (se * MI + i) * D;
        } else {
          wgi = m->swg[l] + (w - K * MI) * D;
          wui = m->swu[l] + (w - K * MI) * D;
        }
        float g = 0.0f, uu = 0.0f;
        for (int64_t k = 0; k < D; k++) {
          g += xn2b[k] * orc_bf16_to_f32(wgi[k]);
          uu += xn2b[k] * orc_bf16_to_f32(wui[k]);
        }
        hbuf[w] = (g / (1.0f + expf(-g))) * uu;
      }
      for (int64_t d = 0; d < D; d++) {
        float acc = 0.0f;
        for (int64_t e = 0; e < K; e++) {
          const uint16_t *wde = m->wd[l] + ((int64_t)sel[e] * D + d) * MI;
          float s = 0.0f;
          for (int64_t i = 0; i < MI; i++) s += hbuf[e * MI + i] * orc_bf16_to_f32(wde[i]);
          acc += probs[e] * s;
        }
        float s = 0.0f;
        for (int64_t i = 0; i < SI; i++) s += hbuf[K * MI + i] * orc_bf16_to_f32(m->swd[l][d * SI + i]);
        acc += s;
        x[d] = bfr_(x1[d] + bfr_(acc));
      }
    }
  }
  ref_rms(x, m->norm, xn, D, m->eps, 0);   /* rms_f, f32 out */
  ref_gemv(xn, m->lm_head, 0, lg, D, V, sk_lm);
  next = 0;
  for (int64_t v = 1; v < V; v++)
    if (lg[v] > lg[next]) next = (int32_t)v;
  if (tr) {
    if (tr->ql) memcpy(tr->ql, ql, sizeof(float) * (size_t)(H * KV));
    if (tr->sm) memcpy(tr->sm, sm, sizeof(float) * (size_t)(H * ML));
    if (tr->ol) memcpy(tr->ol, ol, sizeof(float) * (size_t)(H * KV));
    if (tr->ob) orc_f32_to_bf16_n(ob, tr->ob, H * DV);
  }
out:
  free(x);
  free(x1);
  free(xn);
  free(xn2f);
  free(xn2b);
  free(y);
  free(u);
  free(qb);
  free(ql);
  free(ol);
  free(sm);
  free(ob);
  free(hbuf);
  if (!logits) free(lg);
  return next;
}
