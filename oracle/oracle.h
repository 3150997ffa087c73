/* CPU oracle: a plain-C restatement of the reference's CPU arithmetic for the
 * tensor track's decode path.  TEST INFRASTRUCTURE ONLY: it is linked by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * as the checker, never by the product path (thvm_b200/).
 *
 * Every function states the reference op it restates (file:line inside the
 * reference project).  Each reduction is one float accumulator walked in index
 * order, as the reference's rendered C loops are (src/codegen/render_uop.c
 * emits a serial in-thread loop per REDUCE; the CPU JIT compiles it with
 * -ffp-contract=off, src/backend/cpu/jit.c).  Elementwise constants are the
 * reference's doubles rounded to float, as a CONST of a float32 graph is.
 *
 * Pinned against the fixtures in tests/golden/, which were produced by running the
 * reference itself (tests/golden/make_golden.py).
 */
#ifndef THVM_ORACLE_H
#define THVM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[m,n] = sum_k x[m,k] * w[n,k] (+ b[n]); w stored (out, in) as nn.Linear
 * keeps it and read through .T (py/thvm/nn.py:12-25, src/nn/linear.c:1-6,
 * src/nn/dot.c:1-20).  b may be NULL. */
void orc_linear_f32(const float *x, const float *w, const float *b, float *y,
                    int64_t M, int64_t K, int64_t N);

/* (x - mean) * recip(sqrt(mean((x-mean)^2) + eps)) * g + b over the last axis
 * (src/nn/layernorm.c:1-7, src/nn/reduce.c:28-35, py/thvm/nn.py:160-164).
 * g, b may be NULL (no affine). */
void orc_layernorm_f32(const float *x, const float *g, const float *b, float *y,
                       int64_t M, int64_t D, float eps);

/* x * recip(sqrt(mean(x^2) + eps)) * g (py/thvm/nn.py RMSNorm._norm). */
void orc_rmsnorm_f32(const float *x, const float *g, float *y, int64_t M, int64_t D,
                     float eps);

/* softmax over the last axis: max, x - max, exp2(.*log2e), sum, * recip(sum)
 * (src/nn/softmax.c:1-16, src/nn/elementwise.c:7-9). */
void orc_softmax_f32(const float *x, float *y, int64_t M, int64_t N);

/* tanh-form GELU, tanh as 2*sigmoid(2x)-1, sigmoid as recip(exp(-x)+1)
 * (src/nn/elementwise.c:13-34). */
void orc_gelu_f32(const float *x, float *y, int64_t n);

/* softmax(q k^T * (1/sqrt(D)) + mask) v per (b, h) (src/nn/scaled_dot_product_attention.c:1-34).
 * q [BH, Lq, D], k and v [BH, Lk, D], y [BH, Lq, D].  mask: NULL, or an additive
 * [Lq, Lk] float mask broadcast over BH.  causal: 0, or 1 for the is_causal
 * mask, key j allowed for query i iff j <= i (tril with diagonal 0 on the
 * [Lq, Lk] grid, src/nn/tri.c:1-17). */
void orc_sdpa_f32(const float *q, const float *k, const float *v, const float *mask,
                  float *y, int64_t BH, int64_t Lq, int64_t Lk, int64_t D, int causal);

/* first index of the row max (py/thvm/tensor.py:998-1011): max, compare,
 * times the descending ramp n..1, max, n - that. */
void orc_argmax_f32(const float *x, int32_t *out, int64_t M, int64_t N);

/* rows of w [V, D] at idx; an id outside [0, V) reads a zero row
 * (py/thvm/tensor.py:1706-1714, py/thvm/nn.py Embedding). */
void orc_embedding_f32(const float *w, const int32_t *idx, float *y, int64_t n_idx,
                       int64_t V, int64_t D);

/* ---- low-precision storage formats (src/dtype/fp_convert.c, src/dtype/fp8.c)
 * f32 -> bf16: round to nearest even on the dropped 16 bits; a NaN becomes the
 * quiet NaN with the input's sign (fp_convert.c f32_to_bf16).  bf16 -> f32:
 * the 16 bits on top (bf16_to_f32). */
uint16_t orc_f32_to_bf16(float v);
float orc_bf16_to_f32(uint16_t b);
/* f32 -> fp8 e4m3 as the kernel store narrows (fp8.c f32_to_fp8e4m3_sat):
 * round to nearest even, finite overflow and +-inf saturate to +-448 (0x7e),
 * a NaN keeps its sign with the e4m3 NaN code 0x7f.  e4m3 -> f32 exact; 0x7f /
 * 0xff decode to NaN (fp8e4m3_to_f32). */
uint8_t orc_f32_to_fp8e4m3(float v);
float orc_fp8e4m3_to_f32(uint8_t b);
void orc_f32_to_bf16_n(const float *x, uint16_t *y, int64_t n);
void orc_f32_to_fp8e4m3_n(const float *x, uint8_t *y, int64_t n);

/* y[m,n] = sum_k x[m,k] * bf16(w[n,k]): a bf16 weight widened to f32, f32
 * products and one f32 accumulator in k order (the reference's CAST to f32
 * then the Linear loop, src/nn/linear.c:1-6). */
void orc_linear_bf16(const float *x, const uint16_t *w, float *y, int64_t M, int64_t K, int64_t N);

/* fp8 e4m3 weights with one f32 scale per 128 x 128 block: the composition
 * W_f32 = W.cast(f32) * scale.repeat(128, 128) followed by the Linear loop
 * (no fp8 block scaling exists in the reference; this is the composition of
 * its own ops, py/thvm/dtypes.py fp8e4m3 + src/dtype/fp8.c).  scale is
 * [ceil(N/128), ceil(K/128)] row-major. */
void orc_linear_fp8bs(const float *x, const uint8_t *w, const float *scale, float *y, int64_t M,
                      int64_t K, int64_t N);

/* C[m,n] = sum_k bf16(A[m,k]) * bf16(B[n,k]) in f32, k order (a bf16 matmul
 * with f32 accumulate, src/nn/dot.c:1-20 on bf16 inputs cast to f32). */
void orc_gemm_bf16(const uint16_t *a, const uint16_t *b, float *c, int64_t M, int64_t N, int64_t K);

/* ---- GPT-2 decoder (bench/gpt2/thvm_gpt2.py:27-128) ------------------------
 * Weights are pointers into caller memory, Linear weights (out, in). */
typedef struct {
  int32_t n_layers, n_heads, dim, vocab, max_ctx;
  float norm_eps;
  const float *wte, *wpe, *ln_f_w, *ln_f_b, *lm_head;
  const float **c_attn_w, **c_attn_b, **c_proj_w, **c_proj_b;
  const float **c_fc_w, **c_fc_b, **mlp_proj_w, **mlp_proj_b;
  const float **ln_1_w, **ln_1_b, **ln_2_w, **ln_2_b;
} OrcGPT2;

/* Opaque decode state: the per-layer KV cache [2, max_ctx, H, hd] and scratch. */
typedef struct OrcGPT2State OrcGPT2State;

OrcGPT2State *orc_gpt2_state_new(const OrcGPT2 *m);
void orc_gpt2_state_free(OrcGPT2State *s);

/* One forward over `n_tok` ids at positions start_pos.., updating the cache,
 * as Transformer.forward (thvm_gpt2.py:91-124): embeddings, the blocks (causal
 * -inf mask when n_tok > 1), ln_f, lm_head of the last row.  Writes that row's
 * logits [vocab] when `logits` is non-NULL and returns its argmax. */
int32_t orc_gpt2_forward(OrcGPT2State *s, const int32_t *tokens, int32_t n_tok,
                         int32_t start_pos, float *logits);

/* The greedy loop of GPT2.generate (thvm_gpt2.py:195-220) at temperature 0:
 * the prompt in one forward, then one id per step.  out gets n_new ids. */
int orc_gpt2_generate(const OrcGPT2 *m, const int32_t *prompt, int32_t n_prompt,
                      int32_t n_new, int32_t *out);

/* ---- batched bf16 GPT-2-XL-shaped decode step ----------
 * The model of bench/gpt2/thvm_gpt2.py:27-128 with bf16 weights, computed
 * with the GPT-2 forward's own operations (orc_gpt2_forward: LayerNorm, the
 * Linear loop, the attention row (q . k) * scale -> softmax -> mix, GELU,
 * argmax) on the widened weights, the residual stream h in f32, plus a bf16
 * rounding where the device stores bf16: each Linear's input (LayerNorm
 * output, attention output, GELU output) and the k, v cache rows.  With
 * `exact` set those roundings are skipped and the cache holds f32, so the
 * step is the pinned f32 GPT-2 forward on bf16-valued weights, bit for bit.
 * Embedding tables bf16.  Weight matrices (out, in). */
typedef struct {
  int32_t n_layers, dim, heads, vocab, max_ctx, batch;
  float norm_eps;
  const uint16_t *wte, *wpe, *lm_head;            /* [V, D], [ctx, D], [V, D] */
  const float *ln_f_w, *ln_f_b;
  const float **ln_1_w, **ln_1_b, **ln_2_w, **ln_2_b;
  const uint16_t **c_attn_w, **c_proj_w, **c_fc_w, **mlp_proj_w;   /* [3D,D] [D,D] [4D,D] [D,4D] */
  const float **c_attn_b, **c_proj_b, **c_fc_b, **mlp_proj_b;
  int32_t exact;
} OrcXL;

/* One decode step of `batch` sequences at position pos: kv is the cache
 * [n_layers][2][batch][max_ctx][dim] (row pos written), bf16 bits, or f32
 * when m->exact; logits [batch, vocab] (may be NULL); next [batch] gets each
 * row's first-index argmax. */
void orc_xl_step(const OrcXL *m, void *kv, const int32_t *tok, int32_t pos, float *logits, int32_t *next);

/* ---- batched MoE decode step ---------------------------
 * A DeepSeek-V2-Lite-shaped decoder (bench/dsv2_decode_bench.c cfg :97-124)
 * at batch B: f32 residual h; xn = bf16(rms(h) * g); q = xn W_q^T and
 * kva = xn W_kva^T (f32); q nope -> bf16, q pe and k pe rounded to bf16, then
 * rotated (pair (2j, 2j+1) -> columns j, DR/2 + j, YaRN tables); latent =
 * bf16(rms(bf16(kva[:KV])) * g_kv); absorbed MLA per head: qlat = W_uk^T q_nope,
 * scores (qlat . c_t + q_pe . pe_t) * scale, softmax, olat = sum p_t c_t,
 * o = bf16(W_uv olat); h += o W_o^T; xn2 = bf16(rms(h) * g2); dense layers:
 * h += bf16(silu(g) * u) W_down^T (bf16 weights); MoE layers: the router
 * logits xn2 W_router^T routed by orc_ds_route (top-K logits, softmax weights,
 * no renormalisation), each chosen expert and each shared half (weight 1):
 * h += w * bf16(silu(g) * u) W_d^T with fp8 weights * block scales; logits =
 * bf16(rms(h) * g_f) W_lm^T.  The rotary, cache, attention and routing stages
 * are the functions orc_ds_ref_step (below) runs, which is pinned bit for bit
 * to the reference's own step; this step differs from it only in the f32
 * residual stream, the fp8 block-scaled experts with a bf16 intermediate, the
 * bf16 router and lm_head inputs and single-accumulator projections. */
typedef struct {
  int32_t dim, n_layers, heads, kv_lora, d_nope, d_rope, d_v, n_exp, top_k, moe_inter, dense_inter, n_dense,
      n_shared, vocab, max_ctx, batch;
  float eps, scale;
  const uint16_t *embed, *lm_head;
  const float *norm_f, *cos_t, *sin_t;   /* [D], [ctx][DR], [ctx][DR] */
  const float **attn_norm, **kv_norm, **ffn_norm;
  const uint16_t **w_qkva;                /* [H*(DN+DR) + KV + DR][D] */
  const uint16_t **w_uk, **w_uv, **w_o;   /* [H][DN][KV], [H][DV][KV], [D][H*DV] */
  const uint16_t **d_gu, **d_down;        /* dense: [2*DI][D], [D][DI] */
  const uint16_t **router;                /* [E][D] */
  const uint8_t **e_gu, **e_d;            /* [E(+n_shared)][2I][D], [E(+n_shared)][D][I]: routed, then shared */
  const float **e_gu_s, **e_d_s;          /* block scales as sm100_ds_experts takes them */
} OrcDS;

/* The routing rule of the reference's route kernel (bench/dsv2_decode_bench.c
 * :787-863) per row of g [B][E]: the K largest logits (strict >, so ties go to
 * the lowest id), probs = expf(g - max) / sum_e expf(g_e - max), no
 * renormalisation.  sel, probs [B][K]. */
void orc_ds_route(const float *g, int64_t B, int64_t E, int64_t K, int32_t *sel, float *probs);

/* One step: cache_c [L][B][ctx][KV], cache_pe [L][B][ctx][DR] (bf16 bits, row
 * pos written); logits [B][V] (may be NULL); next [B] = row argmax (first index). */
void orc_ds_step(const OrcDS *m, uint16_t *cache_c, uint16_t *cache_pe, const int32_t *tok, int32_t pos,
                 float *logits, int32_t *next);

/* ---- the reference's own batch-1 bf16 MoE decode step ----------------------
 * bench/dsv2_decode_bench.c step_build (:2328-2417) with the CPU twins of its
 * custom kernels, op for op: bf16 residual stream (x1 = bf16(x + bf16(o W_o)),
 * x = bf16(x1 + bf16(moe))), every M = 1 projection a split-K GEMV whose
 * partial sums fold in chunk order (gemv_pick_sk), the router on the f32 rms
 * output with f32 weights, top-K over the router logits, bf16 routed and
 * shared experts with an f32 intermediate, the dense MLP's silu as the
 * scheduler evaluates it, the lm_head on the f32 rms output.  Weight layouts
 * are the DSV2PK01 pack's (bench/dsv2_decode_bench.c:229-300): projections
 * {in, out}; w_qkv the q | kv row concatenation [D][H*(DN+DR) + KV + DR];
 * w_uk [H][DN][KV], w_uv [H][DV][KV]; experts wg / wu [E*MI][D], wd
 * [E*D][MI], swg / swu [SI][D], swd [D][SI] (SI = n_shared * MI). */
typedef struct {
  int32_t dim, n_layers, heads, kv_lora, d_nope, d_rope, d_v, n_exp, n_shared, top_k, moe_inter, dense_inter,
      first_dense, vocab, max_seq;
  float eps, scale;
  const uint16_t *embed, *lm_head;        /* [V][D], [D][V] */
  const float *norm, *cos_t, *sin_t;      /* [D], [max_seq][DR] x 2 */
  const float **win, **wkvn, **wpost, **gate;   /* [D], [KV], [D], [D][E] */
  const uint16_t **wqkv, **wuk, **wuv, **wo, **wg1, **wu1, **wd1, **wg, **wu, **wd, **swg, **swu, **swd;
} OrcDSRef;

/* Optional views of the step's intermediates as the reference keeps them
 * (its DSV2_DUMP buffers): the last layer's qlat [H*KV] f32, attention
 * weights [H*max_seq] f32 (read and written in place: rows past len keep
 * what they held), olat [H*KV] f32 and o [H*DV] bf16, and the last dense
 * layer's gate / up outputs [DI] bf16.  Any pointer may be NULL. */
typedef struct {
  float *ql, *sm, *ol;
  uint16_t *ob, *g1o, *u1o;
} OrcDSRefTrace;

/* One decode step of token `tok` with `len` positions (row len - 1 written):
 * ckv [L][max_seq][KV], kpe [L][max_seq][DR] bf16; logits [V] (may be NULL);
 * returns the first-index argmax. */
int32_t orc_ds_ref_step(const OrcDSRef *m, uint16_t *ckv, uint16_t *kpe, int32_t tok, int32_t len, float *logits,
                        OrcDSRefTrace *tr);

/* threads the oracle's row-parallel loops use (pthreads), for reporting. */
int orc_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
