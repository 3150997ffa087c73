// GPT-2 decoding (batch 1, fp32) as ONE persistent kernel that runs n
// greedy tokens: per token the whole schedule of thvm_gpt2.py's
// Transformer.forward (embedding, n_layers x {ln_1 + c_attn, attention + KV
// append, c_proj + residual, ln_2 + c_fc + GELU, mlp.c_proj + residual},
// ln_f + lm_head, argmax), the position and token carried on the device, so
// one launch replaces n TinyJit replays.
//
// A token reads 495 MB of weights once (77 us at the HBM roofline) but is a
// chain of ~60 dependent steps, each too small to fill the GPU, so the design
// attacks latency between steps:
//
//  * No grid barriers.  Each step's output vector is written as 8-byte words
//    (float bits | 32-bit tag << 32); a 64-bit store is single-copy atomic, so
//    a reader that sees the step's tag also sees the value.  Each consumer
//    thread spins (bounded) on exactly the words it needs: one cross-SM hop
//    (~0.5 us on B200) per step.  A step's consumers depend on every CTA's
//    previous step, so no word is overwritten while a slower CTA still needs
//    its older value.  The argmax is folded by every CTA from the per-CTA
//    partial words, so the next token starts without another hop.
//  * Weights never wait for activations.  Each CTA owns a fixed slice of rows
//    of every projection (contiguous: W is [out, in]); one thread keeps two
//    TMA bulk copies (cp.async.bulk + mbarrier) of the coming slices in flight
//    in a 2 x 80 KB shared-memory double buffer, plus L2 bulk prefetches a few
//    slices further on, so HBM streams ahead of the dependent chain; lm_head
//    (154 MB) streams through the same buffers in 24-row chunks.
//  * Short steps: 16 warps; reductions with one CTA barrier; attention (one
//    CTA per head) loads the cached keys / values of earlier positions into
//    registers before it waits for the new row, and appends that row to the
//    cache itself (so a later token reads its own CTA's writes).
//
// Math is the reference's op order (LayerNorm two-pass with recip(sqrt), bias
// then GELU / residual, scale -> max -> xexp2 -> sum -> recip, first index of
// the max); reductions are tree-ordered.
//
// Waits are bounded (~1 s): a timeout sets the status word, every later wait
// returns at once, the kernel runs to its end publishing nothing, and every
// CTA waits (bounded) for its in-flight bulk copies before it exits.  One CTA
// per SM, launched cooperatively (the spin-waits need every CTA resident).
#include "common.cuh"

namespace sm100 {

constexpr int kWarps = 15;                   // consumer warps
constexpr int kThreads = kWarps * 32;        // consumer threads
constexpr int kBlockThreads = kThreads + 32; // + one producer warp (TMA issue)
constexpr int kBufBytes = 81920;   // one half of the weight double buffer
constexpr int kXsFloats = 4096;    // staged input vector / attention scratch
constexpr int kMaxRows = 64;       // rows of one transfer
constexpr int kPrefetchAhead = 4;  // L2 prefetch distance in transfers
constexpr int kKeyRegs = 3;        // cached keys per 8-lane group held in registers
constexpr int kValRegs = 24;       // cached values per thread held in registers
constexpr int kMaxLayers = SM100_DECODE_MAX_LAYERS;
constexpr int kMaxLmChunks = 64;   // lm_head chunks per CTA (vocab <= G * 64 * rows per chunk)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  With abort_on_status a status already
// set by any CTA ends it at once; without it (draining copies before exit)
// only the iteration limit does.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *status,
                                          bool abort_on_status = true) {
  for (uint32_t i = 0; i < (1u << 20); i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u) {
      if (abort_on_status && *(volatile uint32_t *)status) return false;
      if (i >= 1024) __nanosleep(128);
    }
  }
  atomicOr(status, SM100_DECODE_ERR_STALL);
  return false;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_word(uint64_t *p, uint32_t bits, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)bits;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// The payload of a tagged word once its tag is `tag` (bounded spin).
__device__ __forceinline__ uint32_t wait_word(const uint64_t *p, uint32_t tag, uint32_t *status) {
  uint64_t w = ld_word(p);
  if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
  for (uint32_t i = 0; i < (1u << 22); i++) {
    w = ld_word(p);
    if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
    if ((i & 31u) == 31u) {
      if (*(volatile uint32_t *)status) return 0u;
      if (i >= 256) __nanosleep(64);
    }
  }
  atomicOr(status, SM100_DECODE_ERR_BARRIER);
  return 0u;
}

// N tagged words at p[0], p[stride], ...: every load is issued before any tag
// is checked (one L2 round trip when the words are ready), then only the
// words not yet tagged are polled (bounded).  n <= N of them are live.
template <int N>
__device__ __forceinline__ void wait_words(const uint64_t *p, int stride, int n, uint32_t tag, uint32_t *status,
                                           float (&out)[N]) {
  uint64_t w[N];
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = i < n ? ld_word(p + (size_t)i * stride) : ((uint64_t)tag << 32);
#pragma unroll
  for (int i = 0; i < N; i++) {
    if ((uint32_t)(w[i] >> 32) != tag) w[i] = ((uint64_t)tag << 32) | wait_word(p + (size_t)i * stride, tag, status);
    out[i] = i < n ? __uint_as_float((uint32_t)w[i]) : 0.0f;
  }
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// barrier of the consumer warps only (the producer warp never joins it)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

enum { PH_QKV = 0, PH_ATT, PH_O, PH_FC, PH_P2, PH_LM };

struct Phase {
  int kind, layer;
  int64_t N, K;
  const float *W, *bias;
  const float *ln_g, *ln_b;   // LayerNorm of the input (QKV, FC, LM), else null
};

__device__ __forceinline__ Phase phase_of(const Sm100DecodeModel &m, int p) {
  Phase ph;
  ph.ln_g = ph.ln_b = ph.bias = nullptr;
  const int nl = m.n_layers;
  if (p >= 5 * nl) {
    ph.kind = PH_LM; ph.layer = nl; ph.N = m.vocab; ph.K = m.dim; ph.W = m.lm_head;
    ph.ln_g = m.ln_f_g; ph.ln_b = m.ln_f_b;
    return ph;
  }
  const int l = ph.layer = p / 5;
  ph.kind = p % 5;
  switch (ph.kind) {
    case PH_QKV:
      ph.N = 3 * m.dim; ph.K = m.dim; ph.W = m.w_qkv[l]; ph.bias = m.b_qkv[l];
      ph.ln_g = m.ln1_g[l]; ph.ln_b = m.ln1_b[l];
      break;
    case PH_ATT: ph.N = 0; ph.K = 0; ph.W = nullptr; break;
    case PH_O: ph.N = m.dim; ph.K = m.dim; ph.W = m.w_o[l]; ph.bias = m.b_o[l]; break;
    case PH_FC:
      ph.N = m.hidden; ph.K = m.dim; ph.W = m.w_fc[l]; ph.bias = m.b_fc[l];
      ph.ln_g = m.ln2_g[l]; ph.ln_b = m.ln2_b[l];
      break;
    default: ph.N = m.dim; ph.K = m.hidden; ph.W = m.w_p2[l]; ph.bias = m.b_p2[l]; break;
  }
  return ph;
}

__device__ __forceinline__ void rows_of(int64_t N, int c, int G, int64_t &r0, int64_t &r1) {
  r0 = (N * c) / G;
  r1 = (N * (c + 1)) / G;
}

// ---- the per-CTA schedule, built once per launch in shared memory --------
// Step records (one per step of a token) and transfer records (the weight
// slices of one token, in order: one per non-lm_head weight step, then
// lm_head's rows in chunks; the first transfer of a LayerNorm step also
// carries its LayerNorm parameters at the buffer front), so the token loop
// does no index arithmetic and no dependent loads of model pointers.
struct StepRec {
  const float *bias;      // bias of this CTA's first row, or null
  const uint64_t *src;    // input words (null: the embedding)
  uint64_t *dst;          // output words of this CTA's first row (null: lm_head)
  int kind, layer, K, r0, nrows;
};

struct XferRec {
  const float *w, *ln_g, *ln_b;
  uint32_t wbytes, lnbytes;
  int r, nr;              // rows [r, r + nr)
};

__device__ __forceinline__ int lm_rows_per_chunk(int64_t K) {
  const int r = (int)((kBufBytes - 2 * K * 4) / (K * 4));
  return r < kMaxRows ? r : kMaxRows;
}

__device__ __forceinline__ int xfers_per_token(const Sm100DecodeModel &m, int c, int G) {
  int64_t r0, r1;
  rows_of(m.vocab, c, G, r0, r1);
  const int64_t R = lm_rows_per_chunk(m.dim);
  const int64_t chunks = (r1 - r0 + R - 1) / R;
  return 4 * m.n_layers + (int)(chunks > 0 ? chunks : 1);
}

__device__ void build_step(const Sm100DecodeModel &m, int p, int c, int G, StepRec &s) {
  const Phase ph = phase_of(m, p);
  s.kind = ph.kind;
  s.layer = ph.layer;
  s.K = (int)ph.K;
  int64_t r0 = 0, r1 = 0;
  if (ph.N) rows_of(ph.N, c, G, r0, r1);
  s.r0 = (int)r0;
  s.nrows = (int)(r1 - r0);
  s.bias = ph.bias ? ph.bias + r0 : nullptr;
  s.src = ph.kind == PH_O ? m.att_w : ph.kind == PH_P2 ? m.fc_w : (ph.kind == PH_QKV && ph.layer == 0) ? nullptr : m.x_w;
  s.dst = ph.kind == PH_QKV ? m.qkv_w + r0 : ph.kind == PH_FC ? m.fc_w + r0
        : (ph.kind == PH_O || ph.kind == PH_P2) ? m.x_w + r0 : nullptr;
}

__device__ void build_xfer(const Sm100DecodeModel &m, int i, int c, int G, XferRec &x) {
  const int nl = m.n_layers;
  int p;
  int64_t r, nr;
  bool with_ln;
  if (i < 4 * nl) {
    const int l = i / 4, k = i % 4;
    p = 5 * l + (k == 0 ? PH_QKV : k == 1 ? PH_O : k == 2 ? PH_FC : PH_P2);
    const Phase ph = phase_of(m, p);
    int64_t r0, r1;
    rows_of(ph.N, c, G, r0, r1);
    r = r0;
    nr = r1 - r0;
    with_ln = ph.ln_g != nullptr;
  } else {
    const int j = i - 4 * nl;
    int64_t r0, r1;
    rows_of(m.vocab, c, G, r0, r1);
    const int64_t R = lm_rows_per_chunk(m.dim);
    p = 5 * nl;
    r = r0 + (int64_t)j * R;
    nr = (r + R <= r1) ? R : (r1 > r ? r1 - r : 0);
    with_ln = j == 0;
  }
  const Phase ph = phase_of(m, p);
  x.w = ph.W + r * ph.K;
  x.ln_g = with_ln ? ph.ln_g : nullptr;
  x.ln_b = with_ln ? ph.ln_b : nullptr;
  x.wbytes = (uint32_t)(nr * ph.K * 4);
  x.lnbytes = with_ln ? (uint32_t)(2 * ph.K * 4) : 0u;
  x.r = (int)r;
  x.nr = (int)nr;
}

__device__ __forceinline__ void issue(const XferRec &x, int half, float *buf0, uint64_t *full) {
  float *dst = buf0 + (size_t)half * (kBufBytes / 4);
  mbar_expect_tx(&full[half], x.wbytes + x.lnbytes);
  if (x.lnbytes) {
    bulk_g2s(dst, x.ln_g, x.lnbytes / 2, &full[half]);
    bulk_g2s(dst + x.lnbytes / 8, x.ln_b, x.lnbytes / 2, &full[half]);
  }
  if (x.wbytes) bulk_g2s(dst + x.lnbytes / 4, x.w, x.wbytes, &full[half]);
}

// CTA-wide sum / max with one barrier; `red` alternates between two 16-float
// halves (sel) so back-to-back reductions need no second barrier.
__device__ __forceinline__ float bsum(float v, float *red, int &sel) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float *r = red + 16 * sel;
  sel ^= 1;
  v = warp_sum(v);
  if (lane == 0) r[w] = v;
  csync();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kWarps; i++) s += r[i];
  return s;
}

__device__ __forceinline__ float bmax(float v, float *red, int &sel) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float *r = red + 16 * sel;
  sel ^= 1;
  v = warp_max(v);
  if (lane == 0) r[w] = v;
  csync();
  float s = -INFINITY;
#pragma unroll
  for (int i = 0; i < kWarps; i++) s = fmaxf(s, r[i]);
  return s;
}

// (value, index): larger value wins, then the lower index (first max).
__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

__device__ __forceinline__ void warp_best(float &v, int &i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(v2, i2, v, i)) { v = v2; i = i2; }
  }
}

// CTA-wide (value, index) best; every thread gets it (two barriers).
__device__ __forceinline__ void block_best(float &v, int &i, float *rv, int *ri) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  warp_best(v, i);
  if (lane == 0) { rv[w] = v; ri[w] = i; }
  csync();
  v = lane < kWarps ? rv[lane] : -INFINITY;
  i = lane < kWarps ? ri[lane] : 0x7fffffff;
  warp_best(v, i);
  csync();
}

// Attention of head h for the new row at `pos` (thvm_gpt2.py:49-61), which
// also appends that row's key / value to the cache (the KV-cache assign).
// Keys / values of earlier positions are requested before the wait for the
// new row (they do not depend on it).
__device__ void attention_head(const Sm100DecodeModel &m, float *kc, int h, int pos, bool pos_ok, uint32_t tag_qkv,
                               uint32_t tag_att, float *xs, float *red, int &sel, uint32_t *status) {
  const int D = m.dim, hd = m.head_dim, L = pos + 1;
  float *sc = xs;                  // [max_ctx] scores
  float *qs = xs + m.max_ctx;      // [hd]
  float *kn = qs + hd;             // [hd] new key
  float *vn = kn + hd;             // [hd] new value
  float *acc = vn + hd;            // [kThreads / hd][hd]
  float *vc = kc + (int64_t)m.max_ctx * D;
  const int t = threadIdx.x;
  const int grp = t >> 3, gl = t & 7, per4 = hd / 32;   // float4s of a key row per lane
  constexpr int NG = kThreads / 8;                       // key groups
  const int nslice = kThreads / hd, slice = t / hd, d = t % hd;
  float4 kr[kKeyRegs][2];
  float vr[kValRegs];
#pragma unroll
  for (int i = 0; i < kKeyRegs; i++) {
    const int j = grp + NG * i;
#pragma unroll
    for (int v = 0; v < 2; v++)
      if (v < per4 && j < pos)
        kr[i][v] = __ldcg(reinterpret_cast<const float4 *>(kc + (int64_t)j * D + (int64_t)h * hd + gl * per4 * 4) + v);
  }
#pragma unroll
  for (int u = 0; u < kValRegs; u++) {
    const int j = slice + nslice * u;
    vr[u] = (j < pos) ? __ldcg(vc + (int64_t)j * D + (int64_t)h * hd + d) : 0.0f;
  }
  for (int i = t; i < 3 * hd; i += kThreads) {
    const int which = i / hd, dd = i % hd;
    const float v = __uint_as_float(wait_word(m.qkv_w + (int64_t)which * D + (int64_t)h * hd + dd, tag_qkv, status));
    (which == 0 ? qs : which == 1 ? kn : vn)[dd] = v;
    if (which > 0 && pos_ok) (which == 1 ? kc : vc)[(int64_t)pos * D + (int64_t)h * hd + dd] = v;
  }
  csync();
  float4 q4[2];
#pragma unroll
  for (int v = 0; v < 2; v++)
    if (v < per4) q4[v] = reinterpret_cast<const float4 *>(qs + gl * per4 * 4)[v];
  for (int j0 = 0; j0 < L; j0 += NG) {
    const int i = j0 / NG;
    const int j = j0 + grp;
    float s = 0.0f;
    if (j < L) {
      float4 k4[2];
      if (j == pos) {
#pragma unroll
        for (int v = 0; v < 2; v++)
          if (v < per4) k4[v] = reinterpret_cast<const float4 *>(kn + gl * per4 * 4)[v];
      } else if (i < kKeyRegs) {
#pragma unroll
        for (int ii = 0; ii < kKeyRegs; ii++)
          if (ii == i) {
            k4[0] = kr[ii][0];
            k4[1] = kr[ii][1];
          }
      } else {
#pragma unroll
        for (int v = 0; v < 2; v++)
          if (v < per4)
            k4[v] = __ldcg(reinterpret_cast<const float4 *>(kc + (int64_t)j * D + (int64_t)h * hd + gl * per4 * 4) + v);
      }
#pragma unroll
      for (int v = 0; v < 2; v++) {
        if (v < per4) {
          s = fmaf(q4[v].x, k4[v].x, s);
          s = fmaf(q4[v].y, k4[v].y, s);
          s = fmaf(q4[v].z, k4[v].z, s);
          s = fmaf(q4[v].w, k4[v].w, s);
        }
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (j < L && gl == 0) sc[j] = __fmul_rn(s, m.attn_scale);
  }
  csync();
  float mx = -INFINITY;
  for (int j = t; j < L; j += kThreads) mx = fmaxf(mx, sc[j]);
  mx = bmax(mx, red, sel);
  float sum = 0.0f;
  for (int j = t; j < L; j += kThreads) sum += xexp(__fsub_rn(sc[j], mx));
  sum = bsum(sum, red, sel);
  const float r = __frcp_rn(sum);
  // mix: p_j = exp(s_j - max) * recip(sum), as the reference orders it
  if (slice < nslice) {
    float a = 0.0f;
#pragma unroll
    for (int u = 0; u < kValRegs; u++) {
      const int j = slice + nslice * u;
      if (j < L) a = fmaf(__fmul_rn(xexp(__fsub_rn(sc[j], mx)), r), j == pos ? vn[d] : vr[u], a);
    }
    for (int j = slice + nslice * kValRegs; j < L; j += nslice)
      a = fmaf(__fmul_rn(xexp(__fsub_rn(sc[j], mx)), r),
               j == pos ? vn[d] : __ldcg(vc + (int64_t)j * D + (int64_t)h * hd + d), a);
    acc[slice * hd + d] = a;
  }
  csync();
  for (int dd = t; dd < hd; dd += kThreads) {
    float a = 0.0f;
    for (int s2 = 0; s2 < nslice; s2++) a += acc[s2 * hd + dd];
    st_word(m.att_w + (int64_t)h * hd + dd, __float_as_uint(a), tag_att);
  }
}

__global__ void __launch_bounds__(kBlockThreads, 1) decode_kernel(const Sm100DecodeModel *__restrict__ mp, int n_tokens) {
  extern __shared__ __align__(1024) unsigned char smem[];
  float *buf0 = reinterpret_cast<float *>(smem);                         // [2][kBufBytes / 4]
  float *xs = reinterpret_cast<float *>(smem + 2 * kBufBytes);          // [kXsFloats]
  float *xown = xs + kXsFloats;                                          // [kMaxRows] own residual rows
  float *part = xown + kMaxRows;                                         // [kWarps][kMaxRows] partials
  float *red = part + kWarps * kMaxRows;                                 // [2][16]
  uint64_t *full = reinterpret_cast<uint64_t *>(red + 32);               // [2] transfer landed
  uint64_t *empty = full + 2;                                            // [2] half released
  StepRec *steps = reinterpret_cast<StepRec *>(empty + 2);               // [n_phases]
  const Sm100DecodeModel &m = *mp;
  const int n_phases = 5 * m.n_layers + 1;
  XferRec *xfers = reinterpret_cast<XferRec *>(steps + n_phases);        // [nx]
  __shared__ float rbv[kWarps];
  __shared__ int rbi[kWarps];

  const int c = blockIdx.x, G = gridDim.x, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  uint32_t *status = m.sync + 2;
  int nx = xfers_per_token(m, c, G);
  if (nx > 4 * m.n_layers + kMaxLmChunks) {   // vocab too large for the schedule table
    if (threadIdx.x == 0) atomicOr(m.sync + 2, SM100_DECODE_ERR_ARG);
    nx = 4 * m.n_layers + kMaxLmChunks;
  }
  const int total_x = nx * n_tokens;
  // tags: (launch epoch mod 65535 + 1) << 16 | token * stride + step: never
  // 0 (the zero-initialised words), distinct from the previous launch's and
  // within a launch one per (token, step)
  const uint32_t tag_base = ((m.sync[3] % 65535u) + 1u) << 16;
  const uint32_t stride = (uint32_t)n_phases + 1u;
  const int pos0 = m.io[0];
  // a position range outside the cache is an argument error: flag it and keep
  // every access in bounds (positions from 0, no cache write, nothing published)
  const bool pos_ok = pos0 >= 0 && pos0 + n_tokens <= m.max_ctx;
  const float *wte = m.wte, *wpe = m.wpe;
  float *logits = m.logits;
  const int vocab = m.vocab, dim = m.dim;
  const float eps = m.eps;
  int sel = 0;

  for (int p = t; p < n_phases; p += kThreads) build_step(m, p, c, G, steps[p]);
  for (int i = t; i < nx; i += kThreads) build_xfer(m, i, c, G, xfers[i]);
  if (t == 0) {
    if (!pos_ok && c == 0) atomicOr(status, SM100_DECODE_ERR_ARG);
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&empty[0], 1);
    mbar_init(&empty[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == kWarps) {
    // ---- producer: every weight transfer of the launch, in order, into the
    // half its consumer released (two in flight), plus L2 prefetches ahead
    if (lane == 0) {
      int issued = 0, ia = 0;
      for (int qq = 0; qq < total_x; qq++) {
        const int h = qq & 1;
        if (qq >= 2 && !mbar_wait(&empty[h], ((qq >> 1) - 1) & 1, status)) break;
        issue(xfers[qq % nx], h, buf0, full);
        issued = qq + 1;
        for (; ia < qq + 2 + kPrefetchAhead && ia < total_x; ia++) {
          if (ia < 2) continue;
          const XferRec &x = xfers[ia % nx];
          if (x.wbytes) bulk_prefetch_l2(x.w, x.wbytes);
        }
      }
      // every issued transfer has landed before the CTA exits (the halves
      // complete their uses in order; bounded, not cut short by the status)
      for (int qq = issued - 2; qq < issued; qq++)
        if (qq >= 0) mbar_wait(&full[qq & 1], (qq >> 1) & 1, status, false);
    }
    return;
  }
  uint64_t *tr = m.trace ? m.trace + (size_t)c * n_phases * 4 : nullptr;

  int q = 0, qi = 0;   // next transfer: global index, index within the token
  int tok = m.io[1];
  for (int tk = 0; tk < n_tokens; tk++) {
    const int pos = pos_ok ? pos0 + tk : 0;
    const uint32_t tag_tok = tag_base + (uint32_t)tk * stride;
    const bool trace = tr && t == 0 && tk == n_tokens - 1;
    float my_best = -INFINITY;
    int my_idx = 0x7fffffff;
    for (int p = 0; p < n_phases; p++) {
      const StepRec st = steps[p];
      const uint32_t tag = tag_tok + (uint32_t)p;
      if (trace) tr[p * 4 + 0] = gtimer();
      if (st.kind == PH_ATT) {
        if (c < m.heads) attention_head(m, m.kv_cache[st.layer], c, pos, pos_ok, tag - 1, tag, xs, red, sel, status);
        csync();   // xs (attention scratch) is free again
        if (trace) tr[p * 4 + 1] = tr[p * 4 + 2] = tr[p * 4 + 3] = gtimer();
        continue;
      }
      const int K = st.K, K4 = K / 4;
      const bool ln = st.kind == PH_QKV || st.kind == PH_FC || st.kind == PH_LM;
      const float bpre = (st.bias && t < st.nrows) ? st.bias[t] : 0.0f;

      // ---- the input vector: embedding, or the previous step's words ------
      constexpr int KPT = (kXsFloats + kThreads - 1) / kThreads;
      float xv[KPT];
      if (st.src == nullptr) {
        // x = wte[tok] + wpe[pos] (thvm_gpt2.py:93-103); own rows kept for the residual
        const bool tok_ok = tok >= 0 && tok < vocab;
#pragma unroll
        for (int i = 0; i < KPT; i++) {
          const int k = t + i * kThreads;
          xv[i] = k < K ? __fadd_rn(tok_ok ? wte[(int64_t)tok * K + k] : 0.0f, wpe[(int64_t)pos * K + k]) : 0.0f;
        }
        int64_t s0, s1;
        rows_of(dim, c, G, s0, s1);
        if (t < s1 - s0)
          xown[t] = __fadd_rn(tok_ok ? wte[(int64_t)tok * K + s0 + t] : 0.0f, wpe[(int64_t)pos * K + s0 + t]);
      } else {
        const int live = t < K ? (K - 1 - t) / kThreads + 1 : 0;
        wait_words<KPT>(st.src + t, kThreads, live, tag - 1, status, xv);
      }
      if (trace) tr[p * 4 + 1] = gtimer();

      // ---- weights of this step; LayerNorm into xs -------------------------
      XferRec xf = xfers[qi];
      bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
      const float *wb = buf0 + (size_t)(q & 1) * (kBufBytes / 4);
      if (ln) {
        const float inv_n = (float)(1.0 / (double)K);
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < KPT; i++) s += xv[i];
        const float mean = __fmul_rn(bsum(s, red, sel), inv_n);
        float v2 = 0.0f;
#pragma unroll
        for (int i = 0; i < KPT; i++)
          if (t + i * kThreads < K) {
            const float dd = __fsub_rn(xv[i], mean);
            v2 = fmaf(dd, dd, v2);
          }
        const float var = __fmul_rn(bsum(v2, red, sel), inv_n);
        const float rr = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int i = 0; i < KPT; i++) {
          const int k = t + i * kThreads;
          if (k < K) xs[k] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[i], mean), rr), wb[k]), wb[K + k]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < KPT; i++) {
          const int k = t + i * kThreads;
          if (k < K) xs[k] = xv[i];
        }
      }
      csync();
      if (trace) tr[p * 4 + 2] = gtimer();

      // ---- rows: this transfer (and for lm_head the following chunks) ------
      const float4 *x4 = reinterpret_cast<const float4 *>(xs);
      const float *w = wb + xf.lnbytes / 4;
      for (;;) {
        const int nr = xf.nr;
        const int wpr = nr >= kWarps ? 1 : (nr > 0 ? kWarps / nr : 1);
        if (have && nr > 0) {
          // (row, k-slice) per warp: wpr warps per row when rows are few
          const int per_pass = kWarps / wpr;
          for (int i0 = 0; i0 < nr; i0 += per_pass) {
            const int i = i0 + warp / wpr, j = warp % wpr;
            if (i < nr) {
              const int k0 = (K4 * j) / wpr, k1 = (K4 * (j + 1)) / wpr;
              const float4 *wr = reinterpret_cast<const float4 *>(w + (size_t)i * K);
              float a0 = 0.0f, a1 = 0.0f;
              int k = k0 + lane;
              for (; k + 32 < k1; k += 64) {
                const float4 w0 = wr[k], w1 = wr[k + 32];
                const float4 x0 = x4[k], x1 = x4[k + 32];
                a0 = fmaf(w0.x, x0.x, a0); a1 = fmaf(w1.x, x1.x, a1);
                a0 = fmaf(w0.y, x0.y, a0); a1 = fmaf(w1.y, x1.y, a1);
                a0 = fmaf(w0.z, x0.z, a0); a1 = fmaf(w1.z, x1.z, a1);
                a0 = fmaf(w0.w, x0.w, a0); a1 = fmaf(w1.w, x1.w, a1);
              }
              if (k < k1) {
                const float4 w0 = wr[k], x0 = x4[k];
                a0 = fmaf(w0.x, x0.x, a0);
                a0 = fmaf(w0.y, x0.y, a0);
                a0 = fmaf(w0.z, x0.z, a0);
                a0 = fmaf(w0.w, x0.w, a0);
              }
              const float a = warp_sum(a0 + a1);
              if (lane == 0) part[j * kMaxRows + i] = a;
            }
          }
        }
        csync();
        if (trace && st.kind != PH_LM) tr[p * 4 + 3] = gtimer();
        // this half is free again: the producer refills it
        if (t == 0) mbar_arrive(&empty[q & 1]);
        // epilogue: one thread per row
        if (have && t < nr) {
          float a = 0.0f;
          for (int j = 0; j < wpr; j++) a += part[j * kMaxRows + t];
          switch (st.kind) {
            case PH_QKV: st_word(st.dst + t, __float_as_uint(__fadd_rn(a, bpre)), tag); break;
            case PH_O:
            case PH_P2: {
              const float v = __fadd_rn(xown[t], __fadd_rn(a, bpre));   // x + (xW^T + b)
              xown[t] = v;
              st_word(st.dst + t, __float_as_uint(v), tag);
              break;
            }
            case PH_FC: st_word(st.dst + t, __float_as_uint(gelu_tanh(__fadd_rn(a, bpre))), tag); break;
            default: {
              const int n = xf.r + t;
              if (logits) logits[n] = a;
              if (better(a, n, my_best, my_idx)) { my_best = a; my_idx = n; }
              break;
            }
          }
        }
        q++;
        if (++qi == nx) qi = 0;
        if (st.kind != PH_LM || qi == 0) break;
        // next lm_head chunk
        xf = xfers[qi];
        have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        w = buf0 + (size_t)(q & 1) * (kBufBytes / 4) + xf.lnbytes / 4;
        csync();   // the epilogue above has read `part`
      }
      csync();
      if (trace && st.kind == PH_LM) tr[p * 4 + 3] = gtimer();
    }

    // ---- argmax: publish this CTA's best, fold every CTA's -----------------
    float bv = my_best;
    int bi = my_idx;
    block_best(bv, bi, rbv, rbi);
    const uint32_t tag_am = tag_tok + (uint32_t)n_phases;
    if (t == 0) {
      st_word(m.part_w + 2 * c, __float_as_uint(bv), tag_am);
      st_word(m.part_w + 2 * c + 1, (uint32_t)bi, tag_am);
    }
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int b = t; b < G; b += kThreads) {
      float pw[2];
      wait_words<2>(m.part_w + 2 * b, 1, 2, tag_am, status, pw);
      const int ib = (int)__float_as_uint(pw[1]);
      if (better(pw[0], ib, bv, bi)) { bv = pw[0]; bi = ib; }
    }
    block_best(bv, bi, rbv, rbi);
    tok = bi == 0x7fffffff ? 0 : bi;
  }

  if (c == 0 && t == 0) {
    if (*(volatile uint32_t *)status == 0) {
      m.io[1] = tok;
      if (m.bump) m.io[0] = pos0 + n_tokens;
    }
    m.sync[3] += 1u;   // next launch: new tags
  }
}

}  // namespace sm100

using namespace sm100;

static int g_num_sms[64];

extern "C" uint64_t sm100_decode_sync_bytes(void) { return (uint64_t)(4 + 2 * 1024) * 4; }

extern "C" uint64_t sm100_decode_part_bytes(void) { return (uint64_t)2 * 1024 * 8; }

extern "C" uint64_t sm100_decode_trace_bytes(int32_t n_layers) {
  return (uint64_t)1024 * (5 * (uint64_t)(n_layers > 0 ? n_layers : 0) + 1) * 4 * 8;
}

extern "C" int sm100_decode_steps(const Sm100DecodeModel *dev_model, int32_t n_tokens, int32_t n_layers, int32_t dim,
                                  int32_t max_ctx, void *stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sm100_set_error(SM100_ERR_ARG, "decode: device %d", dev);
  if (!g_num_sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0 || n > 1024) return sm100_set_error(SM100_ERR_CUDA, "decode: SM count %d", n);
    g_num_sms[dev] = n;
  }
  const int G = g_num_sms[dev];
  // every step's row slice (+ LayerNorm parameters) fits a buffer half, at
  // most kMaxRows rows; c_fc (N = 4 dim) and mlp.c_proj (K = 4 dim) dominate
  const int64_t rows_n = (4LL * dim + G - 1) / G, rows_d = ((int64_t)dim + G - 1) / G;
  const int64_t fc_bytes = rows_n * dim * 4 + 2LL * dim * 4, p2_bytes = rows_d * 4LL * dim * 4;
  if (!dev_model || n_tokens <= 0 || (int64_t)n_tokens * (5 * n_layers + 2) >= 65536 || n_layers <= 0 ||
      n_layers > kMaxLayers || dim <= 0 ||
      dim % 32 || 4 * dim > kXsFloats || max_ctx + 3 * 64 + kThreads > kXsFloats || fc_bytes > kBufBytes ||
      p2_bytes > kBufBytes || rows_n > kMaxRows || 3LL * dim * 4 > kBufBytes)
    return sm100_set_error(SM100_ERR_ARG, "decode: unsupported shape (tokens %d, layers %d, dim %d, ctx %d, %d SMs)",
                           n_tokens, n_layers, dim, max_ctx, G);
  // + the per-CTA schedule: step records, transfer records (lm_head chunks: at
  // most ceil(vocab / G / rows per chunk))
  const int64_t n_x = 4LL * n_layers + kMaxLmChunks;
  const size_t smem = 2 * (size_t)kBufBytes + (kXsFloats + kMaxRows + kWarps * kMaxRows + 32) * 4 + 4 * 8 +
                      (size_t)(5 * n_layers + 1) * sizeof(StepRec) + (size_t)n_x * sizeof(XferRec);
  cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "decode: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kBlockThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, decode_kernel, dev_model, (int)n_tokens);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "decode: launch: %s", cudaGetErrorString(e));
  return launch_status("decode");
}

extern "C" int sm100_decode_step(const Sm100DecodeModel *dev_model, int32_t n_layers, int32_t dim, int32_t max_ctx,
                                 void *stream) {
  return sm100_decode_steps(dev_model, 1, n_layers, dim, max_ctx, stream);
}
