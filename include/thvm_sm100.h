/* thvm_sm100.h - the C ABI of the B200 (sm_100a) device for thvm's tensor track.
 *
 * Three layers, all plain C (no torch or CUDA types in any signature; a
 * stream is passed as `void *` and is a cudaStream_t / CUstream):
 *
 *  1. The Backend vtable entries.  Each replaces the CUDA_BACKEND field of
 *     `struct Backend` (src/thvm.h:751-829, filled at src/backend/cuda/_.c:29-53)
 *     with the same meaning: u32 buffer ids (0 = none), refcounts, a best-fit
 *     freelist that hands recycled storage to a FRESH slot id, zero-filled new
 *     allocations, offset writes for the KV-cache append, stream-ordered
 *     launches and a sync at the realize boundary.
 *  2. sm100_dispatch_kernel: the replacement of
 *     `int (*dispatch_kernel)(KernelEntry *, u32 *in_buf_ids, u32 out_buf_id)`.
 *     The schedule-side router turns a recognised lifted DAG into an
 *     Sm100Kernel descriptor (input slots index in_buf_ids) and calls this.
 *  3. One launcher per kernel family over device pointers and a stream
 *     (sm100_linear, sm100_attention, sm100_layernorm, ...), for hosts that
 *     manage their own memory, and for the dispatcher itself.
 *  4. TinyJit replay as CUDA graphs (replaces cuda_jit_graph_*,
 *     src/backend/cuda/jit.c:444-604, and jit_replay's all-CUDA fast path,
 *     src/jit/capture.c:2695-2738): runtime values that change per step
 *     (a symbolic position, a token id) live in device buffers, so one
 *     captured graph serves every step.
 *
 * Every entry point returns an int status (SM100_OK = 0, negative on error)
 * unless it mirrors a void / u32 vtable field; sm100_last_error() gives the
 * message of the last failure (as thvm_cuda_last_error, src/backend/cuda/init.c:96-101).
 */
#ifndef THVM_SM100_H
#define THVM_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status, dtypes ------------------------------------------------------ */
enum {
  SM100_OK = 0,
  SM100_ERR_ARG = -1,         /* bad id, size, shape or pointer */
  SM100_ERR_CUDA = -2,        /* a CUDA runtime call failed */
  SM100_ERR_UNSUPPORTED = -3, /* kernel kind / dtype / shape not handled */
  SM100_ERR_OOM = -4,         /* device allocation failed */
  SM100_ERR_STATE = -5,       /* not initialised, or wrong capture state */
  SM100_ERR_TIMEOUT = -6      /* a bounded device wait gave up (status word set) */
};

/* dtype ids (the reference's DT_* storage types that reach this path) */
enum {
  SM100_DT_F32 = 0,
  SM100_DT_BF16 = 1,
  SM100_DT_FP8E4M3 = 2, /* weights only, with fp32 128x128 block scales */
  SM100_DT_I32 = 3
};

/* ---- 1. Backend vtable (src/thvm.h:751-829) ------------------------------ */

/* Backend.init / shutdown (cuda_init, src/backend/cuda/init.c:110-143).
 * Selects device $THVM_SM100_DEVICE (default: the current device). */
int sm100_init(void);
void sm100_shutdown(void);
const char *sm100_last_error(void);
/* 1 after a successful sm100_init on an sm_100 device. */
int sm100_ready(void);
/* Host-memory mode for CPU-only tests of the buffer table: buffers are host
 * allocations and no kernel runs.  Call before sm100_init. */
void sm100_debug_host_memory(int on);

/* Buffers: u32 ids into a 65536-slot table (CUDA_BUFS, src/backend/cuda/init.c:47-53).
 * buf_alloc returns 0 on failure (OOM, slot table full, above the per-buffer
 * ceiling $THVM_MAX_BUF_BYTES, 0 = unlimited, default unlimited here since
 * 180 GB of HBM holds whole weight sets); new storage reads as zeros
 * (cuda_buf_alloc's cuMemsetD8, src/backend/cuda/buf_alloc.c:122). */
uint32_t sm100_buf_alloc(uint64_t nbytes);
void sm100_buf_free(uint32_t buf_id);
void sm100_buf_incref(uint32_t buf_id);
void sm100_buf_decref(uint32_t buf_id); /* frees at refcount 0 unless jit-pinned */
void sm100_buf_jit_pin(uint32_t buf_id);
void sm100_buf_jit_unpin(uint32_t buf_id);
int sm100_buf_read(uint32_t buf_id, void *dst, uint64_t nbytes);
int sm100_buf_write(uint32_t buf_id, const void *src, uint64_t nbytes);
int sm100_buf_copy(uint32_t dst_buf_id, uint32_t src_buf_id, uint64_t nbytes);
/* KV-cache append: bounds-checked offset write / copy (src/thvm.h:783-795). */
int sm100_buf_write_at(uint32_t buf_id, uint64_t byte_off, const void *src, uint64_t nbytes);
int sm100_buf_copy_at(uint32_t dst_buf_id, uint64_t dst_byte_off, uint32_t src_buf_id,
                      uint64_t nbytes);
uint32_t sm100_buf_refcount(uint32_t buf_id);
/* Freelist hand-off (src/backend/cuda/buf_freelist.c:10-110): push parks the
 * storage; the next alloc that best-fits it gets a NEW id and the donor id
 * goes dead; remove un-parks a buffer not yet re-issued. */
void sm100_buf_freelist_push(uint32_t buf_id);
void sm100_buf_freelist_remove(uint32_t buf_id);
uint32_t sm100_buf_storage_root(uint32_t buf_id);
uint64_t sm100_buf_nbytes(uint32_t buf_id); /* the requested size */
void sm100_buf_zero(uint32_t buf_id);       /* stream-ordered, no host sync */
/* An arena view: bytes [off, off+nbytes) of parent, sharing its storage
 * (parent_buf_id, src/backend/cuda/buf_alloc.c:196-204). 0 on failure. */
uint32_t sm100_buf_view(uint32_t parent_buf_id, uint64_t off, uint64_t nbytes);
/* Device address of a live buffer (NULL if dead), for launcher callers. */
void *sm100_buf_dptr(uint32_t buf_id);
uint64_t sm100_mem_live_bytes(void);
uint64_t sm100_mem_peak_bytes(void);
uint32_t sm100_buf_live_count(void);

/* Launch stream: the backend's own non-blocking stream unless set. */
void *sm100_stream(void);
int sm100_set_stream(void *stream);

/* dispatch_begin / flush / end (src/backend/dispatch/ *.c): end synchronises
 * the stream at the realize boundary unless a capture is open
 * (cuda_dispatch_end, src/backend/cuda/_.c:23-27). */
void sm100_dispatch_begin(void);
void sm100_dispatch_flush(void);
void sm100_dispatch_end(void);

/* ---- 2. dispatch_kernel -------------------------------------------------- */

enum {
  SM100_K_LINEAR = 1,   /* y = x W^T (+b) [+GELU] [+residual]; optional LN prologue */
  SM100_K_LAYERNORM,    /* y = LN(x) (*g + b) over the last axis */
  SM100_K_RMSNORM,      /* y = x rsqrt(mean(x^2) + eps) (*g) */
  SM100_K_SOFTMAX,      /* softmax over the last axis */
  SM100_K_GELU,         /* tanh-form GELU, elementwise */
  SM100_K_ADD,          /* y = a + b, elementwise */
  SM100_K_ATTENTION,    /* softmax(q k^T scale [+causal]) v over a KV cache */
  SM100_K_EMBEDDING,    /* y[i] = table[idx[i]] (zero row outside [0, V)) [+ pos rows] */
  SM100_K_ARGMAX,       /* first index of each row's max (int32) */
  SM100_K_SCATTER,      /* dst[idx[i]] = src[i] rows, idx outside [0, V) skipped */
  SM100_K_KV_APPEND,    /* cache[:, pos:pos+T] = stack(k, v) at a device position */
  SM100_K_POS_ADD,      /* device int32 counter += value (the kvar bump) */
  SM100_K_DECODE_STEP,  /* the fused GPT-2 decode step (sm100_decode_step) */
  SM100_K_ATTN_PREFILL  /* causal softmax(q k^T scale) v, bf16 q/k/v (sm100_attn_prefill_bf16) */
};

/* Linear flags */
enum {
  SM100_LIN_LN = 1u << 0,        /* x -> layernorm(x) * ln_g + ln_b before the product */
  SM100_LIN_GELU = 1u << 1,      /* tanh GELU after the bias */
  SM100_LIN_RESIDUAL = 1u << 2,  /* y = residual + (xW^T + b) */
  SM100_LIN_KV_APPEND = 1u << 3  /* also store output columns [d, 3d) into the KV cache */
};

/* Input slots of a descriptor index the in_buf_ids array; -1 = absent.
 * Unused fields are 0 / -1. */
typedef struct {
  uint32_t kind;
  uint32_t dtype;   /* weight / table dtype (SM100_DT_*); activations are f32 */
  uint32_t flags;
  int32_t in[10];   /* slot meaning per kind, below */
  int64_t m, n, k;  /* rows, cols / outputs, contraction (per kind, below) */
  int64_t ld_in, ld_out; /* row strides (elements) of the first input / the output; 0 = dense */
  int64_t row_off;  /* first input row to read (e.g. the last prompt row) */
  int32_t heads, head_dim, max_ctx, causal;
  int32_t pos;      /* host value of the runtime position when in[7] < 0 */
  float eps, scale;
} Sm100Kernel;
/* Slot meaning:
 *  LINEAR     in[0]=x [m,k]  in[1]=W [n,k]  in[2]=bias  in[3]=ln_g  in[4]=ln_b
 *             in[5]=residual [m,n] (may be the output)  in[6]=block scales (fp8)
 *             in[7]=position (i32)  in[8]=KV cache [2, max_ctx, n/3] (KV_APPEND:
 *             output columns [n/3, n) also go to cache rows pos+row)
 *  LAYERNORM  in[0]=x [m,k] in[1]=g in[2]=b
 *  RMSNORM    in[0]=x [m,k] in[1]=g
 *  SOFTMAX    in[0]=x [m,k]
 *  GELU       in[0]=x (m*k elements)
 *  ADD        in[0]=a in[1]=b (m*k elements)
 *  ATTENTION  in[0]=q rows [m=T, heads*head_dim] (stride ld_in) in[1]=KV cache
 *             [2, max_ctx, heads*head_dim] in[7]=position; keys 0..pos+t for
 *             query row t (causal within the new rows), scale = 1/sqrt(hd)
 *  EMBEDDING  in[0]=table [n=V, k=D] in[1]=idx i32 [m] in[2]=pos table [*, D]
 *             (optional, adds row pos+i) in[7]=position
 *  ARGMAX     in[0]=x [m, n] (stride ld_in, from row_off); out = i32 [m];
 *             in[7]=position to bump by 1 after the write (optional)
 *  SCATTER    in[0]=src [m, k] in[1]=idx i32 [m]; out = dst [n, k]
 *  KV_APPEND  in[0]=k rows in[1]=v rows [m, k] (stride ld_in) in[7]=position;
 *             out = cache [2, max_ctx, k]
 *  POS_ADD    out = i32 counter; pos = value to add
 *  DECODE_STEP in[0]=an Sm100DecodeModel in device memory; m = n_layers,
 *             k = dim, heads, ld_out = vocab (lm_head rows), max_ctx,
 *             n = tokens (0 means 1); out = the model's io buffer
 *  ATTN_PREFILL in[0]=q in[1]=k in[2]=v, bf16 [m=B, heads, n=S, k=head_dim];
 *             out = f32 [B, heads, S, head_dim]; causal must be 1; scale;
 *             flags bit 0 = single bf16 P (fast; default is the hi+lo split)
 */
int sm100_dispatch_kernel(const Sm100Kernel *k, const uint32_t *in_buf_ids, uint32_t n_in,
                          uint32_t out_buf_id);

/* gather_strided (src/thvm.h:822-828): dst[i] = src[offset + sum_d idx_d * strides[d]]
 * over a row-major walk of dims, elements of elem_bytes (1, 2, 4 or 8). */
typedef struct {
  uint32_t ndim;
  uint32_t elem_bytes;
  int64_t offset;
  int64_t dims[8];
  int64_t strides[8];
} Sm100View;
int sm100_gather_strided(uint32_t dst_buf_id, uint32_t src_buf_id, const Sm100View *view);

/* ---- 3. launchers over device pointers ----------------------------------- */

typedef struct {
  const float *x;        /* [M, K] f32, row stride ldx (>= K) */
  const void *w;         /* [N, K], row-major, wdtype */
  const float *w_scale;  /* fp8: [ceil(N/128), ceil(K/128)] fp32 block scales */
  const float *bias;     /* [N] or NULL */
  const float *ln_g;     /* LN prologue gamma / beta (NULL: no affine) */
  const float *ln_b;
  const float *residual; /* [M, N] stride ldy, may equal y */
  float *y;              /* [M, N] f32, row stride ldy (>= N) */
  float *kv_cache;       /* KV_APPEND: [2, max_ctx, N/3] */
  const int32_t *pos;    /* KV_APPEND: device start position (NULL: host_pos) */
  int64_t M, N, K, ldx, ldy;
  int32_t wdtype, flags, max_ctx, host_pos;
  float eps;
} Sm100LinearArgs;
int sm100_linear(const Sm100LinearArgs *a, void *stream);

typedef struct {
  const float *q;        /* [T, H*hd] rows, stride ldq (a qkv buffer: 3*H*hd) */
  const float *k_cache;  /* [max_ctx, H*hd] */
  const float *v_cache;  /* [max_ctx, H*hd] */
  float *out;            /* [T, H*hd] */
  const int32_t *pos;    /* device start position (NULL: host_pos) */
  int64_t ldq;
  int32_t T, H, hd, max_ctx, host_pos;
  float scale;
} Sm100AttnArgs;
int sm100_attention(const Sm100AttnArgs *a, void *stream);

int sm100_layernorm(const float *x, const float *g, const float *b, float *y, int64_t M,
                    int64_t D, float eps, void *stream);
int sm100_rmsnorm(const float *x, const float *g, float *y, int64_t M, int64_t D, float eps,
                  void *stream);
int sm100_softmax(const float *x, float *y, int64_t M, int64_t N, void *stream);
int sm100_gelu(const float *x, float *y, int64_t n, void *stream);
int sm100_add(const float *a, const float *b, float *y, int64_t n, void *stream);
/* y[i] = table[idx[i]] (+ pos_table[pos + i]); rows of D floats. */
int sm100_embedding(const float *table, const int32_t *idx, const float *pos_table,
                    const int32_t *pos, float *y, int64_t n_idx, int64_t V, int64_t D,
                    void *stream);
/* out[m] = first index of the max of row m (rows of N floats, stride ld);
 * bump (optional) is incremented by 1 after the write. */
int sm100_argmax(const float *x, int64_t M, int64_t N, int64_t ld, int32_t *out,
                 int32_t *bump, void *stream);
/* sm100_argmax without any device allocation.  This entry point has no
 * counterpart in the reference: it is for callers that cannot allocate device
 * memory (a plugin whose device memory all belongs to a host framework's
 * allocator, a service that fixes its memory plan at start-up and allocates
 * nothing after it, a process whose device budget is spent).  Its scratch is
 * a fixed array compiled into this library (about 33 KB per GPU that loads
 * the library,
 * held until the process exits): at most SM100_ARGMAX_NOALLOC_MAX_ROWS rows
 * per call, more is rejected with SM100_ERR_ARG.  Same results as
 * sm100_argmax.  It calls no cudaMalloc / cudaFree; it clears the array's
 * counters with cudaMemsetAsync on `stream` before each launch.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress,
 * which may load the module), so make that first call before any stream
 * capture.  The address is kept per device ordinal for the life of the
 * process: after cudaDeviceReset (which unloads this library's module from
 * that device) the kept address is stale, so do not use this entry point on
 * a device that was reset.  Every call shares the one array: calls that can
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. */
#define SM100_ARGMAX_NOALLOC_MAX_ROWS 64
int sm100_argmax_noalloc(const float *x, int64_t M, int64_t N, int64_t ld, int32_t *out,
                         int32_t *bump, void *stream);
/* ---- the config-5 decode step with its host in C --------------------------- */
/* The step of thvm_b200/dsv2.py on one GPU over this ABI only: weights from a
 * .safetensors file in the device layout (bf16 / fp8 codes / f32 tensors
 * named as thvm_b200.dsv2.ds_weights, plus "cos" / "sin" [max_ctx][d_rope]
 * f32 rotary tables), activations and compressed KV caches in backend
 * buffers, the step captured into graph slot graph_slot on its first call and
 * replayed after (bench/dsv2_decode_bench.c's emit + replay loop, :2014 and
 * :2586-2610).  Call sm100_init first.  step: tok_in [batch] (host; null
 * keeps the ids the last step chose) at the model's position, then the next
 * ids into tok_out (host; null: no read-back, nothing waits); position + 1. */
typedef struct Sm100DsCfg {
  int32_t n_layers, dim, heads, kv_lora, d_nope, d_rope, d_v, n_exp, top_k, moe_inter, dense_inter, n_dense,
      n_shared, vocab, max_ctx, batch;
  float eps, scale;
} Sm100DsCfg;
typedef struct Sm100DsModel Sm100DsModel;
int sm100_ds_model_open(const Sm100DsCfg *cfg, const char *weights_path, uint32_t graph_slot, Sm100DsModel **out);
/* the same with the weights already on the device: n named tensors at ptrs
 * (nbytes each), which the caller keeps alive and owns */
int sm100_ds_model_open_ptrs(const Sm100DsCfg *cfg, const char *const *names, void *const *ptrs,
                             const uint64_t *nbytes, int32_t n, uint32_t graph_slot, Sm100DsModel **out);
int sm100_ds_model_step(Sm100DsModel *m, const int32_t *tok_in, int32_t *tok_out);
int32_t sm100_ds_model_pos(const Sm100DsModel *m);     /* the next step's position (-1 on error) */
int sm100_ds_model_reset(Sm100DsModel *m);             /* position 0 (the caches are overwritten as it advances) */
uint32_t sm100_ds_model_logits(const Sm100DsModel *m); /* buffer id of the last step's f32 logits [batch][vocab] */
void sm100_ds_model_close(Sm100DsModel *m);

/* ---- the config-3 model with its host in C -------------------------------- */
/* The batched GPT-2-XL-shaped model of thvm_b200/gpt2_xl.py on one GPU over
 * this ABI only (bench/gpt2/thvm_gpt2.py:98-128 with bf16 weights: the prompt
 * forward, then one token at a time): weights from a .safetensors file in the
 * device layout (named as thvm_b200.gpt2_xl.xl_weights: bf16 "wte", "wpe",
 * "lm_head", "h.<l>.attn.w" ...; f32 biases and LayerNorm affines),
 * activations and bf16 KV caches [2, batch, max_ctx, dim] per layer in
 * backend buffers.  dim = heads * 64.  Call sm100_init first.
 * prefill: prompts [batch][len] (host, 1 <= len < max_ctx) through every
 * layer at once (sm100_gemm_bf16_ep, sm100_attn_prefill_bf16 and the
 * sm100_xl_prefill_* glue, eager launches): cache rows 0..len-1, the first
 * ids into tok_out (host; null: none), position = len.  step: tok_in [batch]
 * (host; null keeps the ids the last call chose) at the model's position,
 * next ids into tok_out; position + 1; captured into graph slot graph_slot
 * on its first call and replayed after. */
typedef struct Sm100XlCfg {
  int32_t n_layers, dim, heads, vocab, max_ctx, batch;
  float norm_eps;
} Sm100XlCfg;
typedef struct Sm100XlModel Sm100XlModel;
int sm100_xl_model_open(const Sm100XlCfg *cfg, const char *weights_path, uint32_t graph_slot, Sm100XlModel **out);
/* the same with the weights already on the device (kept alive and owned by
 * the caller) */
int sm100_xl_model_open_ptrs(const Sm100XlCfg *cfg, const char *const *names, void *const *ptrs,
                             const uint64_t *nbytes, int32_t n, uint32_t graph_slot, Sm100XlModel **out);
int sm100_xl_model_prefill(Sm100XlModel *m, const int32_t *prompts, int32_t len, int32_t *tok_out);
int sm100_xl_model_step(Sm100XlModel *m, const int32_t *tok_in, int32_t *tok_out);
int32_t sm100_xl_model_pos(const Sm100XlModel *m);     /* the next step's position (-1 on error) */
uint32_t sm100_xl_model_logits(const Sm100XlModel *m); /* buffer id of the last f32 logits [batch][vocab] */
void sm100_xl_model_close(Sm100XlModel *m);

/* ---- blind speculative decode of the batched MoE step --------------------- */
/* n_seq sequences of S rows each (row i S + s) verify S tokens per step
 * (bench/dsv2_decode_bench.c:1110-1195 draft_prep / accept_commit).  Device
 * state per sequence i: the token stream ids [n_seq][ctx] and len[i] = P + 1,
 * P the index of the pending token.  draft: cand[i][0] = ids[i][P],
 * cand[i][1..S) the tokens after the most recent earlier occurrence of the
 * bigram (ids[P-1], ids[P]) in ids[0..P-1] (-1 where there are none), or with
 * forced != 0 the ids already stored at P + 1 ..; tok[i S + s] = cand (the
 * pending token for a -1), row_pos = P + s, row_seq = i (Sm100DsRows with
 * shared_slots).  accept (am: the step's argmax per row): k = the longest
 * prefix with cand[s + 1] == am[s]; ids[P + 1 .. P + k] = cand[1 .. k],
 * ids[P + k + 1] = am[k], len += k + 1, *committed += k + 1 (may be null).
 * A sequence with P + S >= ctx is left as it is (its rows sit at P) and
 * sm100_spec_status reports 1.  S <= 16. */
int sm100_spec_draft(const int32_t *ids, const int32_t *len, int32_t n_seq, int32_t ctx, int32_t S, int32_t forced,
                     int32_t *tok, int32_t *cand, int32_t *row_pos, int32_t *row_seq, void *stream);
int sm100_spec_accept(int32_t *ids, int32_t *len, int32_t n_seq, int32_t ctx, int32_t S, const int32_t *cand,
                      const int32_t *am, uint64_t *committed, void *stream);
/* the sticky status of the two (synchronises the device, clears it) */
uint32_t sm100_spec_status(void);
/* The bookkeeping of a continuous-batching serve loop after a step of B rows,
 * row b its own request in cache slot b at position row_pos[b]
 * (bench/dsv2_decode_bench.c:2760-2900 serves one request at a time): for an
 * active row, inside its prompt (prompt [B][ctx], plen) the next input is the
 * prompt's next id; after it the step's argmax am[b] is appended to out
 * [B][ctx] (n_out[b] ids) and is the next input, and the row stops (active
 * 0, position 0) at eos[b], at its max_new[b]-th id or at the end of the
 * cache.  row_pos / tok advance for the next step. */
int sm100_serve_advance(int32_t *row_pos, int32_t *tok, const int32_t *am, const int32_t *prompt,
                        const int32_t *plen, int32_t *out, int32_t *n_out, const int32_t *max_new, const int32_t *eos,
                        int32_t *active, int32_t B, int32_t ctx, void *stream);

/* dst[idx[i]] = src[i], rows of D elements of elem_bytes; idx outside [0, V) skipped. */
int sm100_scatter_rows(void *dst, const int32_t *idx, const void *src, int64_t n_idx,
                       int64_t V, int64_t D, int32_t elem_bytes, void *stream);
/* cache[0][pos+t] = k[t], cache[1][pos+t] = v[t] for t < T (rows of D floats). */
int sm100_kv_append(float *cache, const float *k, const float *v, int64_t ld, const int32_t *pos,
                    int32_t host_pos, int32_t T, int32_t D, int32_t max_ctx, void *stream);
int sm100_pos_add(int32_t *counter, int32_t value, void *stream);

/* ---- fused decode step ---------------------------------------------------- */
/* One GPT-2 decode step (batch 1, fp32 weights and activations) as one
 * persistent kernel: the whole schedule of bench/gpt2/thvm_gpt2.py's
 * Transformer.forward for a single token at the device position
 * (embedding, n_layers x {ln_1 + c_attn + KV append, attention, c_proj +
 * residual, ln_2 + c_fc + GELU, mlp.c_proj + residual}, ln_f + lm_head,
 * argmax), i.e. what jit_replay runs per token (src/jit/capture.c:2687).
 * The model descriptor lives in DEVICE memory (the caller uploads it);
 * io = [position, token] int32 is read at the start and, unless an error
 * was flagged, the next token written to io[1] (and io[0] += 1 when bump). */
#define SM100_DECODE_MAX_LAYERS 48
#define SM100_DECODE_REPLICAS 8   /* copies of the per-CTA argmax partials a launch writes */
enum {
  SM100_DECODE_ERR_STALL = 1u << 0,   /* a ring (mbarrier) wait timed out */
  SM100_DECODE_ERR_BARRIER = 1u << 1, /* a wait for another CTA's output timed out */
  SM100_DECODE_ERR_ARG = 1u << 2,     /* position outside [0, max_ctx) */
  SM100_DECODE_ERR_RANGE = 1u << 3    /* a split partial sum outside +-2048 (or NaN) */
};
typedef struct {
  /* per layer a 2-D TMA tensor map over its KV cache viewed as [2 max_ctx,
   * dim] f32, box [32 rows, head_dim]; filled by sm100_decode_prepare (the
   * descriptor's device copy must be 64-byte aligned) */
  uint8_t kv_map[SM100_DECODE_MAX_LAYERS][128];
  int32_t n_layers, dim, hidden, vocab, max_ctx, heads, head_dim, bump;
  float eps, attn_scale;
  /* c_attn, c_fc and lm_head weights block-transposed for the decode grid
   * (sm100_decode_block_transpose); the other matrices as the reference stores
   * them, or regrouped (w_o_h, w_p2_t) */
  const float *wte, *wpe, *ln_f_g, *ln_f_b, *lm_head_bt;
  const float *ln1_g[SM100_DECODE_MAX_LAYERS], *ln1_b[SM100_DECODE_MAX_LAYERS];
  const float *w_qkv_bt[SM100_DECODE_MAX_LAYERS], *b_qkv[SM100_DECODE_MAX_LAYERS];
  const float *b_o[SM100_DECODE_MAX_LAYERS];
  const float *ln2_g[SM100_DECODE_MAX_LAYERS], *ln2_b[SM100_DECODE_MAX_LAYERS];
  const float *w_fc_bt[SM100_DECODE_MAX_LAYERS], *b_fc[SM100_DECODE_MAX_LAYERS];
  const float *b_p2[SM100_DECODE_MAX_LAYERS];
  /* the two split projections, regrouped once at load (sm100_decode_regroup):
   * c_proj [heads][dim][head_dim] (w_o_h[h][o][d] = W_o[o][h head_dim + d]),
   * mlp.c_proj transposed [hidden][dim] (w_p2_t[k][o] = W_p2[o][k]) */
  const float *w_o_h[SM100_DECODE_MAX_LAYERS], *w_p2_t[SM100_DECODE_MAX_LAYERS];
  float *kv_cache[SM100_DECODE_MAX_LAYERS]; /* [2, max_ctx, dim] each */
  int32_t *io;                              /* [position, token] */
  /* zero-initialised scratch: q, k, v of the new row as tagged words (float
   * bits | tag << 32), [3 dim]; the split sums' reduction words,
   * sm100_decode_red_bytes() */
  uint64_t *qkv_w, *red_w;
  uint64_t *part_w;                         /* per-CTA argmax partials, sm100_decode_part_bytes() */
  float *logits;                            /* [vocab], or NULL: not stored */
  /* optional timeline of the last token of a launch, or NULL: [grid][3
   * n_layers + 1][8] u64 global-timer ns per CTA and step (per layer: c_attn,
   * attention + c_proj, c_fc + mlp.c_proj; then lm_head): 0 step start, 1
   * thread 0's input landed (attention: every input), 2 weights landed
   * (attention: softmax done), 3 every input landed (attention: its output
   * done), 4 step done, 5 the step's weight transfer issued, 6 its issue
   * began waiting for a free stage, 7 LayerNorm done
   * (sm100_decode_trace_bytes) */
  uint64_t *trace;
  /* zero-initialised scratch of sm100_decode_sync_bytes(): sync[2] the sticky
   * status word (SM100_DECODE_ERR_* bits; cleared by the caller), sync[3] the
   * launch epoch the tags derive from, sync[4] the tokens decoded so far (a
   * token uses reduction set sync[4] mod 3 and clears the next one) */
  uint32_t *sync;
} Sm100DecodeModel;
uint64_t sm100_decode_sync_bytes(void);
uint64_t sm100_decode_part_bytes(void);
uint64_t sm100_decode_trace_bytes(int32_t n_layers);
uint64_t sm100_decode_red_bytes(int32_t n_layers, int32_t dim);
/* block-transposed copy of a row-sliced weight for the decode grid on the
 * current device: kind 0 c_attn [3 dim][dim], 1 c_fc [4 dim][dim], 2 lm_head
 * [vocab][dim]; every slice [r, r + nr) a decode CTA streams is stored at
 * offset r dim as [dim / 4][nr][4] (device pointers, f32) */
int sm100_decode_block_transpose(const float *src, float *dst, int32_t kind, int32_t dim, int32_t heads,
                                 int32_t vocab, void *stream);
/* fills desc->kv_map from kv_cache, max_ctx, dim and head_dim (host memory;
 * call before uploading the descriptor) */
int sm100_decode_prepare(Sm100DecodeModel *desc);
/* CTAs of a decode launch on the current device (heads x members per head;
 * 144 for GPT-2 small on 148 SMs), 0 when the shape has no split */
int32_t sm100_decode_grid(int32_t heads, int32_t head_dim);
/* the regrouped weights of one layer from the reference's layouts: w_o_h
 * [heads][dim][head_dim] from c_proj W_o [dim][dim], w_p2_t [hidden][dim]
 * from mlp.c_proj W_p2 [dim][hidden] (device pointers, f32) */
int sm100_decode_regroup(const float *w_o, const float *w_p2, float *w_o_h, float *w_p2_t, int32_t dim,
                         int32_t heads, int32_t hidden, void *stream);
/* n_tokens greedy tokens in one launch (positions io[0] .. io[0]+n-1, each
 * token's argmax feeding the next).  The scalars repeat the descriptor's
 * (the host checks the shape with them): dim in {512, 768}, heads * 64 ==
 * dim or heads * 32 == dim, hidden = 4 dim, n_tokens * (n_layers + 2) <
 * 65536, and one CTA's slice of every projection within one 76 KB stage
 * (GPT-2 small on 148 SMs: 12 heads x 12 members). */
int sm100_decode_steps(const Sm100DecodeModel *dev_model, int32_t n_tokens, int32_t n_layers,
                       int32_t dim, int32_t heads, int32_t vocab, int32_t max_ctx, void *stream);
/* one token: sm100_decode_steps with n_tokens = 1 */
int sm100_decode_step(const Sm100DecodeModel *dev_model, int32_t n_layers, int32_t dim,
                      int32_t heads, int32_t vocab, int32_t max_ctx, void *stream);

/* ---- dense bf16 GEMM on the tensor cores ------------------------------------- */
/* C[M, N] (f32) = A[M, K] (bf16) . B[N, K]^T (bf16), f32 accumulate: the matmul
 * shape the reference renders as rmu_emit_matmul_tc (src/codegen/render_uop.c:
 * 1784-1986, WMMA) for nn_dot / nn_linear with a K-major weight.  tcgen05 MMA
 * from TMA-loaded 128-byte-swizzled tiles into TMEM; M % 128 == 0,
 * N % 256 == 0, K % 64 == 0, 16-byte aligned.  Device pointers. */
int sm100_gemm_bf16(const void *a, const void *b, float *c, int64_t M, int64_t N, int64_t K, void *stream);
/* non-zero when a GEMM launch since the last call gave up a bounded wait;
 * synchronises the device and clears the word */
uint32_t sm100_gemm_status(void);

/* The same product with its epilogue fused, for the prompt (prefill) pass of
 * the batched decoders: C = epilogue(A . B^T) with, in this order, + bias[n]
 * (f32 [N], or NULL), GELU (SM100_GEMM_GELU; the tanh form of src/nn/gelu.c,
 * evaluated as x sigmoid(2 u) on the fast exponential, ~1e-6 relative),
 * + residual (f32 [M, N], or NULL; may be C itself when C is f32), and the
 * store as f32 or, with SM100_GEMM_OUT_BF16, bf16 (round to nearest even):
 * nn_linear's matmul + bias (src/nn/linear.c:1-6) with the elementwise ops
 * that follow it.  Any M >= 1; N and K multiples of 8 (rows past M, N and K
 * read as zeros); 16-byte aligned pointers.  Device pointers. */
enum {
  SM100_GEMM_GELU = 1u << 0,
  SM100_GEMM_OUT_BF16 = 1u << 1
};
int sm100_gemm_bf16_ep(const void *a, const void *b, void *c, int64_t M, int64_t N, int64_t K, const float *bias,
                       const float *residual, int32_t flags, void *stream);

/* ---- skinny bf16 GEMM for batched decode (M <= 32) ------------------------ */
/* Y[M, N] = epilogue(X[M, K] . W[N, K]^T), bf16 X and W, f32 accumulate: nn_linear
 * on a [B, 1, K] activation (src/nn/linear.c:1-6, py/thvm/nn.py:12-25) at the
 * decode batch of BASELINE config 3.  tcgen05 with the weight rows as the MMA's
 * M and the batch as its N; weight units of 128 x 64 spread evenly over up to
 * 148 CTAs, split row tiles finished deterministically by their last part.
 * Epilogue flags: + bias (when non-NULL), tanh GELU, + residual, bf16 output,
 * and the KV-cache append of the k / v thirds of a fused qkv projection. */
enum {
  SM100_SK_GELU = 1u << 0,
  SM100_SK_RESIDUAL = 1u << 1,
  SM100_SK_OUT_BF16 = 1u << 2,
  SM100_SK_KV = 1u << 3,
  SM100_SK_ACCUM = 1u << 4,   /* y (f32) += X W^T (+ bias once), unordered reductions; alone */
  SM100_SK_X_GELU = 1u << 5,  /* x is f32 [M, K]: the product uses bf16(gelu(x)) */
  SM100_SK_X_LN = 1u << 6     /* x is f32 [M, K]: the product uses bf16(LayerNorm(x) * ln_g + ln_b) */
};
typedef struct {
  const void *x;          /* [M, K] bf16, row stride ld_x (0: K) */
  const void *w;          /* [N, K] bf16, row stride ld_w (0: K) */
  const float *bias;      /* [N] or NULL */
  const float *residual;  /* [M, N] f32, row stride ld_res (0: N); may equal y */
  void *y;                /* [M, N] f32, or bf16 with SM100_SK_OUT_BF16; row stride ld_y (0: N) */
  float *ws;              /* sm100_skinny_ws_bytes(M) bytes of scratch */
  uint32_t *counters;     /* ceil(N / 128) words, zero before the first call; left zero */
  void *kv_cache;         /* SM100_SK_KV: [2, M, kv_ctx, N / 3] bf16; columns [N/3, 2N/3) -> k, rest -> v */
  const int32_t *pos;     /* SM100_SK_KV: device row of the cache to write */
  int64_t M, N, K, ld_x, ld_w, ld_res, ld_y;
  int32_t flags, kv_ctx;
  const float *ln_g, *ln_b; /* SM100_SK_X_LN: the LayerNorm affine over K */
  float eps;
} Sm100SkinnyArgs;
/* M in [1, 32]; K % 8 == 0; x and w 16-byte aligned.  Launches on stream. */
int sm100_skinny_bf16(const Sm100SkinnyArgs *a, void *stream);
uint64_t sm100_skinny_ws_bytes(int32_t M);
/* non-zero when a skinny launch since the last call gave up a bounded wait;
 * synchronises the device and clears the word */
uint32_t sm100_skinny_status(void);

/* ---- the batched bf16 decode step around the skinny GEMM (config 3) ------- */
/* GPT-2-XL-shaped decode of B sequences (bench/gpt2/thvm_gpt2.py:27-128 with
 * bf16 weights): h f32 residual stream, bf16 matmul operands, bf16 KV cache
 * [2, B, ctx, C] (C = heads * 64 of this rank).  Device pointers; launch on
 * stream. */
/* h[b] = wte[tok[b]] + wpe[*pos] (bf16 tables; ids outside [0, V) read zeros) */
int sm100_xl_embed(const void *wte, const void *wpe, const int32_t *tok, const int32_t *pos, float *h,
                   int32_t B, int32_t V, int32_t D, void *stream);
/* y (bf16) = LayerNorm(x) * g + b per row (src/nn/layernorm.c:1-7); zero_x clears
 * x after reading it, zero_buf[0..zero_n) is cleared (accumulators of the next
 * products) */
int sm100_xl_layernorm(float *x, const float *g, const float *b, void *y, int32_t M, int32_t D, float eps,
                       int32_t zero_x, float *zero_buf, int64_t zero_n, void *stream);
/* out (bf16 [B, C]) = softmax(q k^T * scale) v over cache rows 0..*pos, q the
 * first C columns of qkv rows (f32, row stride ld_qkv); hd = 64.  append: qkv
 * rows are complete [q | k | v] sums; k, v enter cache row *pos first and the
 * qkv rows are cleared after use */
int sm100_xl_attention(float *qkv, int64_t ld_qkv, void *kv_cache, const int32_t *pos, void *out, int32_t B,
                       int32_t H, int32_t hd, int32_t ctx, float scale, int32_t append, void *stream);
/* per row: largest value and its first index + idx_offset (py/thvm/tensor.py:998-1011);
 * zero_x clears the rows after reading */
int sm100_xl_argmax(float *x, int64_t ld, int32_t M, int32_t N, float *val, int32_t *idx, int32_t idx_offset,
                    int32_t zero_x, void *stream);
/* tok[b] = index of the largest of R candidates val/idx [R][B] (ties: smaller index) */
int sm100_xl_pick(const float *val, const int32_t *idx, int32_t R, int32_t B, int32_t *tok, void *stream);

/* The prompt pass of the same model (thvm_gpt2.py:98-128 on the [B, P] prompt
 * with start_pos 0): rows r = b P + s of all P positions per layer, the
 * projections by sm100_gemm_bf16_ep and the causal attention by
 * sm100_attn_prefill_bf16 over q, k, v [B, H, P, 128] bf16 whose upper 64
 * columns stay zero (head dimension 64).  Device pointers. */
/* h[b P + s] = wte[tok[b P + s]] + wpe[s] (ids outside [0, V) read zeros) */
int sm100_xl_prefill_embed(const void *wte, const void *wpe, const int32_t *tok, float *h, int32_t B, int32_t P,
                           int32_t V, int32_t D, void *stream);
/* qkv bf16 [B P, 3 C] (C = H * 64) -> q, k, v columns 0..63 of [B, H, P, 128]
 * and k, v into kv_cache [2, B, ctx, C] rows 0..P-1 */
int sm100_xl_prefill_split(const void *qkv, void *q, void *k, void *v, void *kv_cache, int32_t B, int32_t P,
                           int32_t H, int32_t ctx, void *stream);
/* y (bf16) = LayerNorm(x) * g + b over M rows of D (D % 4 == 0, D <= 2048):
 * sm100_xl_layernorm's function, one warp per row */
int sm100_xl_prefill_layernorm(const float *x, const float *g, const float *b, void *y, int32_t M, int32_t D,
                               float eps, void *stream);
/* att bf16 [B P, C] = columns 0..63 of o f32 [B, H, P, 128] */
int sm100_xl_prefill_merge(const float *o, void *att, int32_t B, int32_t P, int32_t H, void *stream);
/* h_last [B, D] = h [B P, D] rows b P + P - 1; *pos = P */
int sm100_xl_prefill_last(const float *h, float *h_last, int32_t *pos, int32_t B, int32_t P, int32_t D,
                          void *stream);

/* ---- the batched MoE decode step pieces (config 5) ------------------------ */
/* DeepSeek-V2-Lite-shaped decode of B <= 32 sequences (bench/dsv2_decode_bench.c
 * :341-1110 at batch 1): f32 residual stream, bf16 matmul operands, bf16
 * compressed KV cache (latent [B, ctx, KV] and rotary [B, ctx, DR]), fp8-e4m3
 * experts with 128 x 128 f32 block scales.  Device pointers; launch on stream. */
/* y (bf16) = x * rsqrt(mean(x^2) + eps) * g per row */
int sm100_ds_rmsnorm(const float *x, const float *g, void *y, int32_t M, int32_t D, float eps, void *stream);
/* h[b] = emb[tok[b]] (bf16 table; ids outside [0, V) read zeros) */
int sm100_ds_embed(const void *emb, const int32_t *tok, float *h, int32_t B, int32_t V, int32_t D, void *stream);
/* q rows [H][DN + DR] -> q_out bf16 (pe rotated by the cos / sin tables [ctx][DR]
 * at row *pos); kva rows [KV + DR] -> RMSNorm(latent) * g_kv and rotated pe
 * appended at cache row *pos.  q and kva rows have stride ld (elements). */
int sm100_ds_qkv_post(const float *q, const float *kva, int64_t ld, const float *g_kv, const float *cos_t,
                      const float *sin_t, const int32_t *pos, void *q_out, void *cache_c, void *cache_pe,
                      int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t KV, int32_t ctx, float eps,
                      void *stream);
/* absorbed multi-head latent attention over cache rows 0..*pos; w_uk / w_uv
 * bf16 [H][DN or DV][KV]; o bf16 [B][H * DV] */
int sm100_ds_mla(const void *q_out, const void *w_uk, const void *w_uv, const void *cache_c, const void *cache_pe,
                 const int32_t *pos, void *o, int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t DV, int32_t KV,
                 int32_t ctx, float scale, void *stream);
/* sm100_ds_qkv_post then sm100_ds_mla in one launch for the DeepSeek-V2-Lite
 * shapes (KV 512, DR 64, DN and DV <= 128): qkva holds the projection's f32
 * rows (stride ld): the H heads' q [H][DN + DR] from column 0 and the latent
 * and key rope [KV + DR] from column kva_off.  Each CTA post-processes its
 * sequences' q and current cache row itself (the same operations) and walks
 * that row from shared memory; the CTAs of head 0 store it in the caches.
 * Other shapes run the two launches (q_out then holds the processed q). */
int sm100_ds_mla_post(const float *qkva, int64_t ld, int64_t kva_off, const float *g_kv, const float *cos_t,
                      const float *sin_t, const int32_t *pos, void *q_out, const void *w_uk, const void *w_uv,
                      void *cache_c, void *cache_pe, void *o, int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t DV,
                      int32_t KV, int32_t ctx, float eps, float scale, void *stream);
/* Rows of a step that are not one sequence each at one shared position: row
 * b appends its latent / key row to cache slot seq[b] at position pos[b] and
 * attends over that slot's rows 0..pos[b] (caches [n_seq][ctx][...]).  With
 * shared_slots != 0 several rows may use one slot (the draft rows of a
 * speculative verify, at consecutive positions): every append then completes
 * before any attention starts (two launches), so a row sees the rows the
 * others append in the same step.  A row outside [0, n_seq) x [0, ctx) is
 * skipped, its attention output is zero, and the status word of
 * sm100_ds_status gets SM100_DECODE_ERR_ARG. */
typedef struct Sm100DsRows {
  const int32_t *pos; /* [B] device */
  const int32_t *seq; /* [B] device */
  int32_t n_seq;
  int32_t shared_slots;
} Sm100DsRows;
/* sm100_ds_mla_post with per-row cache slots and positions */
int sm100_ds_mla_post_rows(const float *qkva, int64_t ld, int64_t kva_off, const float *g_kv, const float *cos_t,
                           const float *sin_t, const Sm100DsRows *rows, void *q_out, const void *w_uk,
                           const void *w_uv, void *cache_c, void *cache_pe, void *o, int32_t B, int32_t H, int32_t DN,
                           int32_t DR, int32_t DV, int32_t KV, int32_t ctx, float eps, float scale, void *stream);
/* the K largest of E <= 64 router logits (ties: lowest id) weighted by their
 * softmax probabilities, no renormalisation (the reference's route kernel,
 * bench/dsv2_decode_bench.c:787-863); sel / wsel [B][K]; slot lists of the
 * experts [e0, e1)
 * followed by n_shared experts taking every token with weight 1:
 * slot_off [e1 - e0 + n_shared + 1], slot_tok / slot_w [B * (K + n_shared)]
 * (expert-major) */
int sm100_ds_route(const float *logits, int32_t E, int32_t K, int32_t B, int32_t e0, int32_t e1, int32_t n_shared,
                   int32_t *sel, float *wsel, int32_t *slot_off, int32_t *slot_tok, float *slot_w, void *stream);
/* the router product and the routing in one launch: logits [B][E] = x .
 * router[e] (x, router bf16 [B][D], [E][D]; f32 sums), then the routing of
 * sm100_ds_route; counter is one int32 of device memory that starts at zero
 * and is left at zero (the launch's CTAs count themselves off on it) */
int sm100_ds_router_route(const void *x, const void *router, float *logits, int32_t *counter, int32_t D, int32_t E,
                          int32_t K, int32_t B, int32_t e0, int32_t e1, int32_t n_shared, int32_t *sel, float *wsel,
                          int32_t *slot_off, int32_t *slot_tok, float *slot_w, void *stream);
/* y[tok] += w * down(bf16(silu(gate x) * (up x))) for the slots of n_exp
 * experts on the tensor cores, fp8 x fp8: the weights stream by TMA as the
 * MMA's e4m3 operand; each token's row times the 128 x 128 block scale and
 * a per-token power of two is split into e4m3 hi + lo terms (about 2^-8 of
 * each value), tokens as the MMA's N <= 32.  w_gu fp8 [n_exp][2I][D] +
 * scales [n_exp][2I/128][D/128], w_d fp8 [n_exp][D][I] + scales
 * [n_exp][D/128][I/128]; D, I multiples of 128 up to 4096; x bf16 [B][D];
 * a_scratch bf16 [slots][I]; y f32 [B][D] (float reductions); w_gu, w_d, x
 * and a_scratch 16-byte aligned */
int sm100_ds_experts(const void *x, const void *w_gu, const float *s_gu, const void *w_d, const float *s_d,
                     const int32_t *slot_off, const int32_t *slot_tok, const float *slot_w, void *a_scratch, float *y,
                     int32_t n_exp, int32_t D, int32_t I, void *stream);
/* non-zero when an expert launch since the last call gave up a bounded wait
 * (SM100_DECODE_ERR_STALL) or met an expert with more than 32 slots
 * (SM100_DECODE_ERR_ARG; the MMA's N); synchronises the device and clears
 * the word */
uint32_t sm100_ds_status(void);
/* a (bf16 [M][I]) = silu(gu[:, :I]) * gu[:, I:] of f32 gate|up rows [M][2I] */
int sm100_ds_silu_mul(const float *gu, void *a, int32_t M, int32_t I, void *stream);

/* ---- collectives over peer memory (tensor / expert parallel decode) -------
 * One process per GPU.  Each rank allocates a comm buffer of
 * sm100_comm_bytes(cols) with sm100_peer_alloc (zero-filled; handle_out gets
 * its 64-byte CUDA IPC handle), the ranks exchange handles on the host, each
 * maps the others' with sm100_peer_open and records every rank's address in
 * its own buffer with sm100_comm_set_peers (peer_ptrs[rank] = its own).  The
 * kernels push data into the peers' buffers with plain stores over NVLink and
 * wait on flags with a bounded spin (a timeout sets sm100_comm_status and the
 * kernel finishes without the missing data).  Every rank must issue the same
 * sequence of these calls.  They are the all-reduce after each row-split
 * projection and the gather of the vocabulary-split argmax; rows <= 32,
 * cols % 4 == 0, cols <= 8192, world <= 8. */
uint64_t sm100_comm_bytes(int32_t cols);
int sm100_peer_alloc(uint64_t nbytes, void **dptr, void *handle_out);
int sm100_peer_open(const void *handle, void **peer_dptr);
int sm100_peer_close(void *peer_dptr);
int sm100_peer_free(void *dptr);
int sm100_comm_set_peers(void *own, void *const *peer_ptrs, int32_t world);
/* h [rows, cols] f32 holds this rank's partial sums; afterwards h = the sum of
 * every rank's partials in rank order (the same on every rank) and y (bf16)
 * = h * rsqrt(mean(h^2) + eps) * g per row; with zero_rest != 0 the ranks
 * other than 0 keep zeros in h instead (y is the same) */
int sm100_comm_allreduce_rmsnorm(float *h, const float *g, void *y, void *own, int32_t rank, int32_t world,
                                 int32_t rows, int32_t cols, float eps, int32_t zero_rest, void *stream);
/* the same exchange with LayerNorm: y = bf16((h - mean) * rsqrt(var + eps) * g
 * + b), mean and biased variance in two passes (src/nn/layernorm.c:1-7) */
int sm100_comm_allreduce_layernorm(float *h, const float *g, const float *b, void *y, void *own, int32_t rank,
                                   int32_t world, int32_t rows, int32_t cols, float eps, void *stream);
/* tok[b] = the index of the largest val over the ranks' (val[b], idx[b])
 * (ties: the smaller index) */
int sm100_comm_pick(const float *val, const int32_t *idx, void *own, int32_t rank, int32_t world, int32_t rows,
                    int32_t *tok, void *stream);
/* non-zero when a comm kernel since the last call gave up a bounded wait;
 * synchronises the device and clears the word */
uint32_t sm100_comm_status(void);

/* ---- causal attention prefill on the tensor cores ------------------------ */
/* O[B, H, S, D] (f32) = softmax(Q K^T * scale + causal mask) V for bf16 Q, K, V
 * [B, H, S, D] contiguous, D = 128, any S >= 0: the reference's
 * nn_scaled_dot_product_attention with causal = 1 (src/nn/
 * scaled_dot_product_attention.c:1-34, reached from Tensor.
 * scaled_dot_product_attention(is_causal=True), py/thvm/tensor.py:1726-1749),
 * fused flash style (QK^T and PV on tcgen05 into TMEM, online softmax between).
 * precise_p = 1 feeds P to the PV product as bf16 hi + bf16 lo (two MMAs,
 * ~16-bit P: ~2e-6 relative to an f32 softmax, row argmax stable); 0 feeds a
 * single bf16 P (~2e-3 relative).  Device pointers, 16-byte aligned. */
int sm100_attn_prefill_bf16(const void *q, const void *k, const void *v, float *o, int32_t B, int32_t H,
                            int32_t S, int32_t D, float scale, int32_t precise_p, void *stream);
/* non-zero when a prefill launch since the last call gave up a bounded wait;
 * synchronises the device and clears the word */
uint32_t sm100_attn_prefill_status(void);

/* ---- weight files straight into device buffers ---------------------------
 * .safetensors (the format py/thvm/nn_state.py safe_load / safe_save read
 * and write, :44-85: an 8-byte little-endian header length, a JSON header of
 * name -> {dtype, shape, data_offsets}, the raw tensor bytes) and the
 * DSV2PK01 pack of the reference's DeepSeek-V2 bench (bench/
 * dsv2_decode_bench.c:229-262).  The file is mapped read-only and each
 * tensor's bytes go into a fresh backend buffer by one copy from the mapping;
 * entries[i] describes tensor i (the pack's shape is the flat element count)
 * and the caller owns the buffers.  On an error no buffer is left allocated. */
typedef struct {
  char name[128];
  char dtype[12];     /* the file's tag: "F32", "BF16", "F8_E4M3", "I32", ... */
  int32_t ndim;
  int64_t shape[8];
  uint64_t nbytes;
  uint32_t buf_id;
} Sm100TensorEntry;
int sm100_safetensors_load(const char *path, Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out);
int sm100_dsv2pack_load(const char *path, Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out);
/* A torch.save checkpoint (py/thvm/nn_state.py torch_load, :123-230): the zip
 * format (<archive>/data.pkl and the storages at <archive>/data/<key>, stored
 * uncompressed; zip64 included) or the legacy pickle stream.  Every
 * top-level tensor or parameter of the state dict, elements row-major in
 * the file's type: dtype "F32", "F64", "F16", "BF16", "I64", "I32", "I16",
 * "I8", "U8" or "BOOL" (the reference widens BF16 and F64 to f32 on read);
 * a permuted tensor (strides a permutation of a row-major layout) is made
 * row-major through a host gather, other strides are refused as there. */
int sm100_torch_load(const char *path, Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out);

/* ---- custom-kernel ABI: raw CUDA-C programs -------------------------------
 * Replaces cuda_custom_dispatch (src/backend/cuda/jit.c:802-893) for the
 * programs kernel_emit_custom_program records (src/schedule/kernel_custom.c:
 * 47-136; the ABI of src/thvm.h's custom_* KernelEntry fields):
 * `extern "C" __global__ void name(T *arg0, ...)`, one device address per
 * argument, launched grid[3] x block[3] with shared_bytes of dynamic shared
 * memory (above 48 KiB opted in per kernel).  sm100_custom_program compiles
 * the source once with NVRTC for sm_100a and loads it (registering the same
 * name and source again returns the same id, recompiling nothing; the launch
 * shape is the latest registration's); it returns the program id (> 0) or a
 * negative SM100_ERR_* with the compiler's log in sm100_last_error.
 * Dispatching only launches, on the backend stream (so graph capture records
 * it): args are buffer ids, and a non-zero out_buf_id rebinds argument slot
 * primary_out_slot (the reference's rebinding of the lowest output slot at
 * replay, kernel_custom.c:11-30).  At most 64 arguments. */
int32_t sm100_custom_program(const char *name, const char *src, const uint32_t grid[3], const uint32_t block[3],
                             uint32_t shared_bytes);
int sm100_custom_dispatch(int32_t prog, const uint32_t *arg_buf_ids, uint32_t n_args, uint32_t primary_out_slot,
                          uint32_t out_buf_id);
/* the same launch over raw device addresses on `stream` */
int sm100_custom_launch(int32_t prog, void *const *arg_ptrs, uint32_t n_args, void *stream);

/* ---- generic device interpreter for lifted UOp DAGs ----------------------
 * Stands in for the rendered kernel (src/codegen/render_uop.c:4964-5113
 * cg_render_uop_kernel_cuda_root) of a DAG no hand-written kernel covers.
 * The host compiles the DAG once into a register program (sm100_ref.c); the
 * device runs it with one thread per output element: the thread's output
 * coordinates fill the first n_glob range slots (slot n_glob - 1 fastest),
 * and every REDUCE is a counted loop over its range slots, evaluated in order
 * as the reference's CPU walker does (src/backend/cpu/uop_walk.c).
 * Registers hold an int64 or the bits of an f32.  Float arithmetic is f32
 * rounded per operation; exp2 is the reference's xexp2 decomposition. */
enum {
  SM100_IOP_CONST = 1,  /* dst = imm: i32 sign-extended (dt 0), u32 zero-extended (dt 1), f32 bits (dt 2) */
  SM100_IOP_RANGE,      /* dst = range slot a */
  SM100_IOP_VAR,        /* dst = vars[a] */
  SM100_IOP_LOAD,       /* dst = buf a [reg b], buffer dtype dt (SM100_UDT_*) */
  SM100_IOP_STORE,      /* buf a [reg b] = reg c (float when imm != 0), buffer dtype dt */
  SM100_IOP_FADD, SM100_IOP_FMUL, SM100_IOP_FNEG, SM100_IOP_FRECIP, SM100_IOP_FEXP2, SM100_IOP_FLOG2,
  SM100_IOP_FSQRT, SM100_IOP_FSIN, SM100_IOP_FLT, SM100_IOP_FEQ,
  SM100_IOP_IADD, SM100_IOP_ISUB, SM100_IOP_IMUL, SM100_IOP_INEG,
  SM100_IOP_IDIV, SM100_IOP_IMOD,  /* in dtype dt (signedness, width); divisor 0 gives 0 */
  SM100_IOP_ILT, SM100_IOP_ULT, SM100_IOP_IEQ, SM100_IOP_IAND, SM100_IOP_IOR, SM100_IOP_IXOR,
  SM100_IOP_ISHL, SM100_IOP_ISHR,  /* in dtype dt */
  SM100_IOP_WRAP,       /* dst = reg a wrapped to int dtype dt (SM100_UDT_*; bool: != 0) */
  SM100_IOP_I2F,        /* dst = f32(reg a), a of int dtype dt */
  SM100_IOP_F2I,        /* dst = int dtype dt of f32 reg a, toward zero */
  SM100_IOP_NARROW,     /* dst = f32 reg a rounded through float dtype dt (f16 / bf16) */
  SM100_IOP_SEL,        /* dst = reg a != 0 ? reg b : reg c */
  SM100_IOP_LOOP,       /* slot a = 0; if reg b <= 0 jump past the ENDLOOP at imm */
  SM100_IOP_ENDLOOP,    /* if ++slot a < reg b jump to imm + 1 (the body after its LOOP) */
  SM100_IOP_ACCF,       /* dst = dst (+ | max | *) f32 reg a, kind dt (0 sum, 1 max, 2 prod) */
  SM100_IOP_ACCI,       /* dst = dst (+ | max | *) int reg a, kind imm, wrapped to int dtype dt */
  SM100_IOP_THREEFRY,   /* dst = threefry2x32 (20 rounds) of u64 reg a keyed by u64 reg b */
  SM100_IOP_SETR,       /* range slot a = reg b (a range bound to a computed index: a gather) */
  SM100_IOP_COUNT
};

/* the interpreter's dtype codes: the reference's DT_* numbering (src/thvm.h:254-271) */
enum {
  SM100_UDT_BOOL = 0, SM100_UDT_I8, SM100_UDT_U8, SM100_UDT_I16, SM100_UDT_U16, SM100_UDT_I32, SM100_UDT_U32,
  SM100_UDT_I64, SM100_UDT_U64, SM100_UDT_FP8E4M3, SM100_UDT_FP8E5M2, SM100_UDT_F16, SM100_UDT_BF16,
  SM100_UDT_F32, SM100_UDT_F64
};

typedef struct {
  uint8_t op, dt;
  uint16_t dst, a, b, c;
  int32_t imm;
} Sm100Insn;

#define SM100_INTERP_MAX_CODE 1280
#define SM100_INTERP_MAX_REGS 192
#define SM100_INTERP_MAX_AXES 16
#define SM100_INTERP_MAX_BUFS 64
#define SM100_INTERP_MAX_VARS 16
#define SM100_INTERP_MAX_STEPS (1ll << 26) /* loop iterations per output element */

/* Runs the program once per output element: total = prod(glob_ext[0..n_glob)).
 * bufs are device addresses (slot 0 is conventionally the output) and
 * buf_bytes their sizes: a load outside its buffer reads 0, a store outside
 * is dropped. */
int sm100_interp_run(const Sm100Insn *code, uint32_t n_code, uint32_t n_regs, uint32_t n_axes, uint32_t n_glob,
                     const int64_t *glob_ext, void *const *bufs, const int64_t *buf_bytes, uint32_t n_bufs,
                     const int64_t *vars, uint32_t n_vars, void *stream);
/* Non-zero when an element's program stopped at SM100_INTERP_MAX_STEPS loop
 * iterations since the last call (its output is then incomplete); clears. */
int sm100_interp_status(void);

/* ---- 4. TinyJit replay as CUDA graphs ------------------------------------ */
/* Capture every launch on the backend stream between begin and end into
 * graph slot `slot` (0..63); replay launches it. */
int sm100_graph_capture_begin(uint32_t slot);
int sm100_graph_capture_end(uint32_t slot);
int sm100_graph_replay(uint32_t slot);
void sm100_graph_drop(uint32_t slot);
int sm100_graph_capturing(void);

/* launches issued by this library since load (for reporting) */
uint64_t sm100_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
