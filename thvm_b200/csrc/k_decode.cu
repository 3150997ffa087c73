// GPT-2 decoding (batch 1, fp32) as ONE persistent kernel that runs n greedy
// tokens: per token the whole schedule of thvm_gpt2.py's Transformer.forward
// (embedding, n_layers x {ln_1 + c_attn, attention + KV append, c_proj +
// residual, ln_2 + c_fc + GELU, mlp.c_proj + residual}, ln_f + lm_head,
// argmax), the position and token carried on the device, so one launch
// replaces n TinyJit replays.
//
// A token reads 495 MB of weights once (77 us at the HBM roofline) but is a
// chain of ~60 dependent steps, each too small to fill the GPU, so the design
// attacks the latency between steps:
//
//  * Two CTA roles.  CTAs 0..heads-1 are attention CTAs (one per head); the
//    other CTAs own fixed row slices of every projection.  An attention CTA
//    keeps its head's cached keys / values of the earlier positions in shared
//    memory, loaded by TMA bulk copies one layer ahead, so the attention step
//    only waits for q, k, v of the new row.
//  * No grid barriers.  Each step's output vector is written as 8-byte words
//    (float bits | 32-bit tag << 32); a 64-bit store is single-copy atomic, so
//    a reader that sees the step's tag also sees the value.  Consumers poll
//    (bounded) exactly the words they need: one cross-SM hop per step.  A
//    step's consumers depend on every producer of the previous step, so no
//    word is overwritten while a slower CTA still needs its older value.
//  * Weights never wait for activations.  One producer warp per projection
//    CTA keeps TMA bulk copies (cp.async.bulk + mbarrier) of the coming slices
//    in a 2 x 88 KB shared-memory ring plus L2 prefetches a few slices ahead;
//    lm_head (154 MB) streams through the same ring in 27-row chunks.
//  * One CTA barrier per step.  After the input vector lands in shared
//    memory every warp works alone: it computes the LayerNorm statistics with
//    warp shuffles (redundantly, 768 floats), keeps its lanes' normalised
//    inputs in registers, and finishes whole rows (dot product, bias, GELU or
//    residual, publish) without waiting for other warps.  mlp.c_proj (K =
//    4 dim) splits each row in four quarters and adds them after one more
//    barrier, in a fixed order.
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
#include "tma.cuh"

namespace sm100 {

constexpr int kWarps = 15;                   // consumer warps (16 warps in all: 128 registers)
constexpr int kThreads = kWarps * 32;        // consumer threads
constexpr int kBlockThreads = kThreads + 32; // + one producer warp (TMA issue)
constexpr int kStages = 2;                   // weight ring stages
constexpr int kStageBytes = 88 * 1024;       // one stage
constexpr int kXsFloats = 4096;              // one staged input vector (hidden <= 4096)
constexpr int kMaxRows = 64;                 // rows of one CTA's slice (non-lm_head steps)
constexpr int kRowsPerWarp = 6;              // >= ceil(kMaxRows / kWarps), even (rows go in pairs)
constexpr int kPrefetchAhead = 4;            // L2 prefetch distance in transfers
constexpr int kMaxLayers = SM100_DECODE_MAX_LAYERS;
constexpr int kMaxLmChunks = 64;             // lm_head chunks per CTA
constexpr int kBiasFloats = 72;              // stage region of a transfer's biases (kMaxRows + 3, 16-byte multiple)
constexpr int kSmemLimit = 227 * 1024;
constexpr int kTraceSlots = 8;               // u64 timestamps per (CTA, step) in the optional trace
constexpr size_t kPartWords = 2 * 1024;      // argmax partials of one copy: (value, index) per CTA

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_word(uint64_t *p, uint32_t bits, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)bits;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// A step's output word goes to kReplicas copies (stride n words); consumer
// CTA c polls copy c % kReplicas.  Every consumer reads every word; with one
// copy the ~136 CTAs re-polling the same L2 lines slowed each hop (GPT-2
// small on B200: 287 us per token with one copy, 261 with eight).
constexpr int kReplicas = SM100_DECODE_REPLICAS;

__device__ __forceinline__ void st_word_rep(uint64_t *p, size_t n, uint32_t bits, uint32_t tag) {
#pragma unroll
  for (int r = 0; r < kReplicas; r++) st_word(p + (size_t)r * n, bits, tag);
}

// The payload of a tagged word once its tag is `tag` (bounded spin, out of
// line like mbar_wait_slow).
__device__ __noinline__ uint32_t wait_word(const uint64_t *p, uint32_t tag, uint32_t *status) {
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
// is checked (one L2 round trip when the words are ready); the words not yet
// tagged are then re-polled together, one round trip per round (bounded).
// n <= N of them are live.
template <int N>
__device__ __forceinline__ void wait_words(const uint64_t *p, int stride, int n, uint32_t tag, uint32_t *status,
                                           float (&out)[N]) {
  uint64_t w[N];
  uint32_t pending = 0;
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = i < n ? ld_word(p + (size_t)i * stride) : ((uint64_t)tag << 32);
#pragma unroll
  for (int i = 0; i < N; i++)
    if ((uint32_t)(w[i] >> 32) != tag) pending |= 1u << i;
  for (uint32_t it = 0; pending; it++) {
    if (it >= (1u << 22) || ((it & 15u) == 15u && *(volatile uint32_t *)status)) {
      if (it >= (1u << 22)) atomicOr(status, SM100_DECODE_ERR_BARRIER);
      break;
    }
#pragma unroll
    for (int i = 0; i < N; i++)
      if ((pending >> i) & 1u) w[i] = ld_word(p + (size_t)i * stride);
#pragma unroll
    for (int i = 0; i < N; i++)
      if (((pending >> i) & 1u) && (uint32_t)(w[i] >> 32) == tag) pending &= ~(1u << i);
  }
#pragma unroll
  for (int i = 0; i < N; i++) out[i] = (i < n && !((pending >> i) & 1u)) ? __uint_as_float((uint32_t)w[i]) : 0.0f;
}

// Pairs of tagged words (2 i, 2 i + 1) at p[0], p[stride], ... with one
// 16-byte load each (half the polling requests of single words); a pair is
// in when both tags are.  Bounded like wait_words.
__device__ __forceinline__ void ld_pair(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

template <int N>
__device__ __forceinline__ void wait_pairs(const uint64_t *p, int stride, int n, uint32_t tag, uint32_t *status,
                                           float2 (&out)[N]) {
  uint64_t w0[N], w1[N];
  uint32_t pending = 0;
#pragma unroll
  for (int i = 0; i < N; i++) {
    if (i < n) ld_pair(p + (size_t)i * stride, w0[i], w1[i]);
    else w0[i] = w1[i] = (uint64_t)tag << 32;
  }
#pragma unroll
  for (int i = 0; i < N; i++)
    if ((uint32_t)(w0[i] >> 32) != tag || (uint32_t)(w1[i] >> 32) != tag) pending |= 1u << i;
  for (uint32_t it = 0; pending; it++) {
    if (it >= (1u << 22) || ((it & 15u) == 15u && *(volatile uint32_t *)status)) {
      if (it >= (1u << 22)) atomicOr(status, SM100_DECODE_ERR_BARRIER);
      break;
    }
#pragma unroll
    for (int i = 0; i < N; i++)
      if ((pending >> i) & 1u) ld_pair(p + (size_t)i * stride, w0[i], w1[i]);
#pragma unroll
    for (int i = 0; i < N; i++)
      if (((pending >> i) & 1u) && (uint32_t)(w0[i] >> 32) == tag && (uint32_t)(w1[i] >> 32) == tag)
        pending &= ~(1u << i);
  }
#pragma unroll
  for (int i = 0; i < N; i++) {
    const bool ok = i < n && !((pending >> i) & 1u);
    out[i] = make_float2(ok ? __uint_as_float((uint32_t)w0[i]) : 0.0f, ok ? __uint_as_float((uint32_t)w1[i]) : 0.0f);
  }
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// barrier of the consumer warps only (the producer warp never joins it)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

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

enum { PH_QKV = 0, PH_ATT, PH_O, PH_FC, PH_P2, PH_LM };

struct Phase {
  int kind, layer;
  int64_t N, K;
  const float *W, *bias;
  const float *ln_g, *ln_b;   // LayerNorm of the input (QKV, FC, LM), else null
};

__device__ __noinline__ Phase phase_of(const Sm100DecodeModel &m, int p) {
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

// rows [r0, r1) of an N-row projection owned by projection CTA c of P
__device__ __forceinline__ void rows_of(int64_t N, int c, int P, int64_t &r0, int64_t &r1) {
  r0 = (N * c) / P;
  r1 = (N * (c + 1)) / P;
}

// ---- the per-CTA schedule, built once per launch in shared memory --------
// Step records (one per step of a token) and transfer records (the weight
// slices of one token, in order: one per projection step, then lm_head's rows
// in chunks; the first transfer of a LayerNorm step also carries its
// LayerNorm parameters at the stage front), so the token loop does no index
// arithmetic and no dependent loads of model pointers.
struct StepRec {
  const float *bias;      // bias of this CTA's first row, or null
  const uint64_t *src;    // input words, this CTA's copy (null: the embedding)
  uint64_t *dst;          // output words of this CTA's first row, copy 0 (null: lm_head)
  int64_t dst_n;          // words between the output copies
  int kind, layer, K, r0, nrows;
};

// Stage layout of a transfer: [ln_g | ln_b] (lnbytes), then the bias rows
// from the 16-byte boundary at or below row r (bbytes, in a kBiasFloats
// region), then the weight rows at float offset wofs.
struct XferRec {
  const float *w, *ln_g, *ln_b, *b;
  uint32_t wbytes, lnbytes, bbytes;
  int r, nr;              // rows [r, r + nr)
  int bofs, wofs;         // float offsets in the stage: row r's bias, the first weight row
};

__host__ __device__ __forceinline__ int lm_rows_per_chunk(int64_t K) {
  return (int)((kStageBytes - 2 * K * 4 - kBiasFloats * 4) / (K * 4));
}

__device__ __forceinline__ int xfers_per_token(const Sm100DecodeModel &m, int c, int P) {
  int64_t r0, r1;
  rows_of(m.vocab, c, P, r0, r1);
  const int64_t R = lm_rows_per_chunk(m.dim);
  const int64_t chunks = (r1 - r0 + R - 1) / R;
  return 4 * m.n_layers + (int)(chunks > 0 ? chunks : 1);
}

__device__ __noinline__ void build_step(const Sm100DecodeModel &m, int p, int c, int P, StepRec &s) {
  const Phase ph = phase_of(m, p);
  s.kind = ph.kind;
  s.layer = ph.layer;
  s.K = (int)ph.K;
  int64_t r0 = 0, r1 = 0;
  if (ph.N) rows_of(ph.N, c, P, r0, r1);
  s.r0 = (int)r0;
  s.nrows = (int)(r1 - r0);
  s.bias = ph.bias ? ph.bias + r0 : nullptr;
  const int rc = c % kReplicas;
  s.src = ph.kind == PH_O ? m.att_w + (size_t)rc * m.dim : ph.kind == PH_P2 ? m.fc_w + (size_t)rc * m.hidden
        : (ph.kind == PH_QKV && ph.layer == 0) ? nullptr : m.x_w + (size_t)rc * m.dim;
  s.dst = ph.kind == PH_QKV ? m.qkv_w + r0 : ph.kind == PH_FC ? m.fc_w + r0
        : (ph.kind == PH_O || ph.kind == PH_P2) ? m.x_w + r0 : nullptr;
  s.dst_n = ph.N;
}

__device__ __noinline__ void build_xfer(const Sm100DecodeModel &m, int i, int c, int P, XferRec &x) {
  const int nl = m.n_layers;
  int p;
  int64_t r, nr;
  bool with_ln;
  if (i < 4 * nl) {
    const int l = i / 4, k = i % 4;
    p = 5 * l + (k == 0 ? PH_QKV : k == 1 ? PH_O : k == 2 ? PH_FC : PH_P2);
    const Phase ph = phase_of(m, p);
    int64_t r0, r1;
    rows_of(ph.N, c, P, r0, r1);
    r = r0;
    nr = r1 - r0;
    with_ln = ph.ln_g != nullptr;
  } else {
    const int j = i - 4 * nl;
    int64_t r0, r1;
    rows_of(m.vocab, c, P, r0, r1);
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
  // the bias rows ride in the same transfer (a global load of them at the
  // step would wait behind the weight streams): from row r rounded down to a
  // 16-byte boundary, a whole number of 16-byte groups
  const int64_t b0 = r & ~(int64_t)3, b1 = (r + nr + 3) & ~(int64_t)3;
  x.b = (ph.bias && nr > 0) ? ph.bias + b0 : nullptr;
  x.bbytes = x.b ? (uint32_t)((b1 - b0) * 4) : 0u;
  x.bofs = (int)(x.lnbytes / 4) + (int)(r - b0);
  x.wofs = (int)(x.lnbytes / 4) + (ph.bias ? kBiasFloats : 0);
  x.r = (int)r;
  x.nr = (int)nr;
}

__device__ __forceinline__ void issue(const XferRec &x, int stage, float *ring, uint64_t *full, uint64_t pol_stream,
                                      uint64_t pol_keep) {
  float *dst = ring + (size_t)stage * (kStageBytes / 4);
  mbar_expect_tx(&full[stage], x.wbytes + x.lnbytes + x.bbytes);
  if (x.lnbytes) {
    bulk_g2s_hint(dst, x.ln_g, x.lnbytes / 2, &full[stage], pol_keep);
    bulk_g2s_hint(dst + x.lnbytes / 8, x.ln_b, x.lnbytes / 2, &full[stage], pol_keep);
  }
  if (x.bbytes) bulk_g2s_hint(dst + x.lnbytes / 4, x.b, x.bbytes, &full[stage], pol_keep);
  if (x.wbytes) bulk_g2s_hint(dst + x.wofs, x.w, x.wbytes, &full[stage], pol_stream);
}

// Shared-memory layout (bytes), the same for both roles.
struct Smem {
  static constexpr size_t ring = 0;
  static constexpr size_t xs = ring + (size_t)kStages * kStageBytes;   // [2][kXsFloats] f32
  static constexpr size_t xown = xs + 2 * kXsFloats * 4;                // [kMaxRows] f32
  static constexpr size_t part = xown + kMaxRows * 4;                   // [4][kMaxRows] f32
  static constexpr size_t rbv = part + 4 * kMaxRows * 4;                // [kWarps] f32
  static constexpr size_t rbi = rbv + kWarps * 4;                       // [kWarps] i32
  static constexpr size_t tok = rbi + kWarps * 4;                       // [4] i32
  static constexpr size_t bars = tok + 16;                              // full[2], empty[2], pfx
  static constexpr size_t steps = bars + 8 * 8;                         // StepRec[5 L + 1]
  static size_t __host__ __device__ xfers(int n_layers) {
    return steps + (size_t)(5 * n_layers + 1) * sizeof(StepRec);
  }
  static size_t __host__ __device__ total(int n_layers) {
    return xfers(n_layers) + (size_t)(4 * n_layers + kMaxLmChunks) * sizeof(XferRec);
  }
};

struct Launch {
  int n_tokens, pos0;
  bool pos_ok;
  uint32_t tag_base, stride;   // tag of (token tk, step p): tag_base + tk * stride + p
  uint32_t *status;
};

// ---------------------------------------------------------------------------
// Attention CTA: head h of every layer (thvm_gpt2.py:49-61), including the
// KV-cache assign of the new row.  The keys / values of the earlier
// positions (up to smax of them) sit in shared memory, brought in by bulk
// copies issued at the end of the previous layer's attention.
template <int NK>
__device__ __noinline__ void attention_role(const Sm100DecodeModel &m, const Launch &ln, unsigned char *smem) {
  const int h = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int D = m.dim, hd = m.head_dim, nl = m.n_layers, max_ctx = m.max_ctx;
  const int smax = (kStages * kStageBytes) / (8 * hd);   // staged positions
  float *Ks = reinterpret_cast<float *>(smem + Smem::ring);
  float *Vs = Ks + (size_t)smax * hd;
  float *sc = reinterpret_cast<float *>(smem + Smem::xs);   // [max_ctx] scores
  float *pr = sc + max_ctx;                                 // [max_ctx] probabilities
  float *qs = pr + max_ctx, *kn = qs + hd, *vn = kn + hd;   // [hd] each
  float *acc = vn + hd;                                     // [kThreads / hd][hd]
  uint64_t *pfx = reinterpret_cast<uint64_t *>(smem + Smem::bars) + 4;
  uint32_t *status = ln.status;
  const int n_phases = 5 * nl + 1;
  uint64_t *tr = m.trace ? m.trace + (size_t)blockIdx.x * n_phases * kTraceSlots : nullptr;

  // prefix copies of (layer l, rows [0, n)); thread 0 armed the barrier
  auto issue_prefix = [&](int l, int n) {
    const float *kc = m.kv_cache[l], *vc = kc + (size_t)max_ctx * D;
    for (int j = t; j < n; j += kThreads) {
      bulk_g2s(Ks + (size_t)j * hd, kc + (size_t)j * D + (size_t)h * hd, (uint32_t)hd * 4, pfx);
      bulk_g2s(Vs + (size_t)j * hd, vc + (size_t)j * D + (size_t)h * hd, (uint32_t)hd * 4, pfx);
    }
  };
  auto staged = [&](int n) { return n < smax ? n : smax; };

  int pf = 0;          // prefix phases consumed
  bool pending = true; // a prefix phase is armed and not yet waited for
  {
    const int n = staged(ln.pos_ok ? ln.pos0 : 0);
    if (t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * n * hd * 4));
    csync();
    issue_prefix(0, n);
  }
  for (int tk = 0; tk < ln.n_tokens; tk++) {
    const int pos = ln.pos_ok ? ln.pos0 + tk : 0, L = pos + 1;
    const uint32_t tag_tok = ln.tag_base + (uint32_t)tk * ln.stride;
    const bool trace = tr && t == 0 && tk == ln.n_tokens - 1;
    for (int l = 0; l < nl; l++) {
      const int p = 5 * l + PH_ATT;
      const uint32_t tag = tag_tok + (uint32_t)p;
      float *kc = m.kv_cache[l], *vc = kc + (size_t)max_ctx * D;
      if (trace) tr[p * kTraceSlots + 0] = gtimer();
      // the prefix copies are ours and always complete: wait for them even
      // after an error, so the staging area is never written by two phases
      mbar_wait(pfx, (uint32_t)(pf & 1), status, false);
      pf++;
      pending = false;
      // q, k, v of the new row; k, v appended to the cache (global and staged)
      for (int i = t; i < 3 * hd; i += kThreads) {
        const int which = i / hd, dd = i % hd;
        const float v = __uint_as_float(wait_word(m.qkv_w + (size_t)(h % kReplicas) * 3 * D + (size_t)which * D +
                                                  (size_t)h * hd + dd,
                                                  tag - 1, status));
        if (which == 0) {
          qs[dd] = v;
        } else {
          (which == 1 ? kn : vn)[dd] = v;
          if (pos < smax) (which == 1 ? Ks : Vs)[(size_t)pos * hd + dd] = v;
          if (ln.pos_ok) (which == 1 ? kc : vc)[(size_t)pos * D + (size_t)h * hd + dd] = v;
          fence_proxy_async();
        }
      }
      csync();
      if (trace) tr[p * kTraceSlots + 1] = gtimer();
      // scores: 8 lanes per key, hd / 8 floats per lane
      {
        const int grp = t >> 3, gl = t & 7, per4 = hd / 32;
        constexpr int NG = kThreads / 8;
        float4 q4[2];
#pragma unroll
        for (int v = 0; v < 2; v++)
          if (v < per4) q4[v] = reinterpret_cast<const float4 *>(qs)[gl * per4 + v];
        for (int j0 = 0; j0 < L; j0 += NG) {
          const int j = j0 + grp;
          float s = 0.0f;
          if (j < L) {
            float4 k4[2];
            if (j < smax) {
#pragma unroll
              for (int v = 0; v < 2; v++)
                if (v < per4) k4[v] = reinterpret_cast<const float4 *>(Ks + (size_t)j * hd)[gl * per4 + v];
            } else if (j == pos) {
#pragma unroll
              for (int v = 0; v < 2; v++)
                if (v < per4) k4[v] = reinterpret_cast<const float4 *>(kn)[gl * per4 + v];
            } else {
#pragma unroll
              for (int v = 0; v < 2; v++)
                if (v < per4)
                  k4[v] = __ldcg(reinterpret_cast<const float4 *>(kc + (size_t)j * D + (size_t)h * hd) + gl * per4 + v);
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
      }
      csync();
      // softmax: every warp folds max and sum itself (no block reduction),
      // then writes p_j = exp(s_j - max) * recip(sum) for its share of j
      {
        float mx = -INFINITY;
        for (int j = lane; j < L; j += 32) mx = fmaxf(mx, sc[j]);
        mx = warp_max(mx);
        float sum = 0.0f;
        for (int j = lane; j < L; j += 32) sum += xexp(__fsub_rn(sc[j], mx));
        sum = warp_sum(sum);
        const float r = __frcp_rn(sum);
        for (int j = t; j < L; j += kThreads) pr[j] = __fmul_rn(xexp(__fsub_rn(sc[j], mx)), r);
      }
      csync();
      if (trace) tr[p * kTraceSlots + 2] = tr[p * kTraceSlots + 3] = gtimer();
      // p @ v: key slices x dims, then the slices in order
      const int nslice = kThreads / hd, slice = t / hd, d = t % hd;
      if (slice < nslice) {
        float a = 0.0f;
        for (int j = slice; j < L; j += nslice) {
          const float v = j < smax ? Vs[(size_t)j * hd + d] : j == pos ? vn[d] : __ldcg(vc + (size_t)j * D + (size_t)h * hd + d);
          a = fmaf(pr[j], v, a);
        }
        acc[slice * hd + d] = a;
      }
      // the next attention's prefix: this token's next layer (rows < pos), or
      // layer 0 of the next token (rows <= pos)
      const bool more = l + 1 < nl || tk + 1 < ln.n_tokens;
      const int nl2 = l + 1 < nl ? l + 1 : 0;
      const int nrows = more ? staged(l + 1 < nl ? pos : (ln.pos_ok ? pos + 1 : 0)) : 0;
      if (more && t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * nrows * hd * 4));
      csync();
      if (t < hd) {
        float a = 0.0f;
        for (int s2 = 0; s2 < nslice; s2++) a += acc[s2 * hd + t];
        st_word_rep(m.att_w + (size_t)h * hd + t, (size_t)D, __float_as_uint(a), tag);
      }
      if (more) {
        issue_prefix(nl2, nrows);
        pending = true;
      }
      if (trace) tr[p * kTraceSlots + 4] = gtimer();
    }
  }
  // every issued copy has landed before the CTA exits
  if (pending) mbar_wait(pfx, (uint32_t)(pf & 1), status, false);
}

// ---------------------------------------------------------------------------
// Projection CTA (consumer warps): every step's row slice, lm_head chunks and
// the argmax.  NK = dim / 128: float4s per lane of a dim-long row.
template <int NK>
__device__ __forceinline__ void load_x(const float *xb, int lane, float (&xr)[4 * NK]) {
#pragma unroll
  for (int j = 0; j < NK; j++) {
    const float4 v = reinterpret_cast<const float4 *>(xb)[lane + 32 * j];
    xr[4 * j] = v.x; xr[4 * j + 1] = v.y; xr[4 * j + 2] = v.z; xr[4 * j + 3] = v.w;
  }
}

// LayerNorm of the staged vector in the lanes' registers (statistics by warp
// shuffles), with gamma / beta from the stage front.
template <int NK>
__device__ __forceinline__ void layernorm_regs(float (&xr)[4 * NK], const float *g, const float *b, int lane, int K,
                                               float eps) {
  const float inv_n = (float)(1.0 / (double)K);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4 * NK; i++) s += xr[i];
  const float mean = __fmul_rn(warp_sum(s), inv_n);
  float v2 = 0.0f;
#pragma unroll
  for (int i = 0; i < 4 * NK; i++) {
    const float dd = __fsub_rn(xr[i], mean);
    v2 = fmaf(dd, dd, v2);
  }
  const float var = __fmul_rn(warp_sum(v2), inv_n);
  const float rr = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
  for (int j = 0; j < NK; j++) {
    const float4 gv = reinterpret_cast<const float4 *>(g)[lane + 32 * j];
    const float4 bv = reinterpret_cast<const float4 *>(b)[lane + 32 * j];
    const float gg[4] = {gv.x, gv.y, gv.z, gv.w}, bb[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int c = 0; c < 4; c++)
      xr[4 * j + c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[4 * j + c], mean), rr), gg[c]), bb[c]);
  }
}

// Dot products of two rows (w0, w1: float4 rows in shared memory) with the
// lanes' registers; every lane gets both sums.
template <int NK>
__device__ __forceinline__ void dot2(const float4 *w0, const float4 *w1, bool two, const float (&xr)[4 * NK], int lane,
                                     float &a, float &b) {
  float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
#pragma unroll
  for (int j = 0; j < NK; j++) {
    const float4 u = w0[lane + 32 * j];
    float &aa = (j & 1) ? a1 : a0;
    aa = fmaf(u.x, xr[4 * j], aa);
    aa = fmaf(u.y, xr[4 * j + 1], aa);
    aa = fmaf(u.z, xr[4 * j + 2], aa);
    aa = fmaf(u.w, xr[4 * j + 3], aa);
    if (two) {
      const float4 v = w1[lane + 32 * j];
      float &bb = (j & 1) ? b1 : b0;
      bb = fmaf(v.x, xr[4 * j], bb);
      bb = fmaf(v.y, xr[4 * j + 1], bb);
      bb = fmaf(v.z, xr[4 * j + 2], bb);
      bb = fmaf(v.w, xr[4 * j + 3], bb);
    }
  }
  a = a0 + a1;
  b = b0 + b1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
}

template <int NK>
__device__ __forceinline__ void projection_role(const Sm100DecodeModel &m, const Launch &ln, unsigned char *smem, int nx) {
  const int A = m.heads, P = gridDim.x - A, pc = blockIdx.x - A;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float *ring = reinterpret_cast<float *>(smem + Smem::ring);
  float *xs = reinterpret_cast<float *>(smem + Smem::xs);
  float *xown = reinterpret_cast<float *>(smem + Smem::xown);
  float *part = reinterpret_cast<float *>(smem + Smem::part);
  float *rbv = reinterpret_cast<float *>(smem + Smem::rbv);
  int *rbi = reinterpret_cast<int *>(smem + Smem::rbi);
  int *tok_s = reinterpret_cast<int *>(smem + Smem::tok);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars), *empty = full + 2;
  const StepRec *steps = reinterpret_cast<const StepRec *>(smem + Smem::steps);
  const XferRec *xfers = reinterpret_cast<const XferRec *>(smem + Smem::xfers(m.n_layers));
  uint32_t *status = ln.status;
  const int n_phases = 5 * m.n_layers + 1;
  const int dim = m.dim, vocab = m.vocab;
  const float eps = m.eps;
  const float *wte = m.wte, *wpe = m.wpe;
  float *logits = m.logits;
  uint64_t *tr = m.trace ? m.trace + (size_t)blockIdx.x * n_phases * kTraceSlots : nullptr;
  constexpr int PPT = (kXsFloats / 2 + kThreads - 1) / kThreads;   // input word pairs per thread

  int q = 0, qi = 0, sidx = 0;   // next transfer (global, within the token), staged-input parity
  int tok = m.io[1];
  for (int tk = 0; tk < ln.n_tokens; tk++) {
    const int pos = ln.pos_ok ? ln.pos0 + tk : 0;
    const uint32_t tag_tok = ln.tag_base + (uint32_t)tk * ln.stride;
    const bool trace = tr && t == 0 && tk == ln.n_tokens - 1;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    for (int p = 0; p < n_phases; p++) {
      const StepRec st = steps[p];
      if (st.kind == PH_ATT) continue;
      const uint32_t tag = tag_tok + (uint32_t)p;
      if (trace) tr[p * kTraceSlots + 0] = gtimer();
      const int K = st.K, nr = st.nrows;
      float *xb = xs + (size_t)(sidx & 1) * kXsFloats;
      sidx++;

      // ---- the input vector: embedding, or the previous step's words ------
      if (st.src == nullptr) {
        // x = wte[tok] + wpe[pos] (thvm_gpt2.py:93-103); own rows kept for the residual
        const bool tok_ok = tok >= 0 && tok < vocab;
        for (int k = t; k < K; k += kThreads)
          xb[k] = __fadd_rn(tok_ok ? wte[(size_t)tok * K + k] : 0.0f, wpe[(size_t)pos * K + k]);
        int64_t s0, s1;
        rows_of(dim, pc, P, s0, s1);
        if (t < s1 - s0)
          xown[t] = __fadd_rn(tok_ok ? wte[(size_t)tok * K + s0 + t] : 0.0f, wpe[(size_t)pos * K + s0 + t]);
      } else {
        // word pairs (2 j, 2 j + 1), j = t, t + kThreads, ...: one 16-byte poll each
        float2 xv[PPT];
        const int KP = K / 2;
        const int live = t < KP ? (KP - 1 - t) / kThreads + 1 : 0;
        wait_pairs<PPT>(st.src + 2 * t, 2 * kThreads, live, tag - 1, status, xv);
#pragma unroll
        for (int i = 0; i < PPT; i++)
          if (i < live) reinterpret_cast<float2 *>(xb)[t + i * kThreads] = xv[i];
      }
      csync();
      if (trace) tr[p * kTraceSlots + 1] = gtimer();

      // ---- weights of this step; the input in registers --------------------
      XferRec xf = xfers[qi];
      bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
      const float *sb = ring + (size_t)(q & 1) * (kStageBytes / 4);
      if (trace) tr[p * kTraceSlots + 2] = gtimer();
      float xr[4 * NK];
      if (st.kind == PH_P2) {
        load_x<NK>(xb + (warp & 3) * dim, lane, xr);   // this warp's quarter of K
      } else {
        load_x<NK>(xb, lane, xr);
        if (st.kind != PH_O) layernorm_regs<NK>(xr, sb, sb + K, lane, K, eps);
      }
      if (trace) tr[p * kTraceSlots + 3] = gtimer();

      // ---- rows ------------------------------------------------------------
      if (st.kind == PH_P2) {
        // (row, quarter) per warp: warps w = qq (mod 4) take quarter qq of rows
        // w / 4, w / 4 + nq, ...; the quarters are added in order afterwards
        const int qq = warp & 3, nq = (kWarps - qq + 3) >> 2;
        if (have) {
          for (int i = warp >> 2; i < nr; i += 2 * nq) {
            const int i2 = i + nq;
            const bool two = i2 < nr;
            float a, b;
            dot2<NK>(reinterpret_cast<const float4 *>(sb + xf.wofs + (size_t)i * K + qq * dim),
                     reinterpret_cast<const float4 *>(sb + xf.wofs + (size_t)(two ? i2 : i) * K + qq * dim), two, xr,
                     lane, a, b);
            if (lane == 0) {
              part[qq * kMaxRows + i] = a;
              if (two) part[qq * kMaxRows + i2] = b;
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        csync();
        if (have && t < nr) {
          const float a = __fadd_rn(__fadd_rn(__fadd_rn(part[t], part[kMaxRows + t]), part[2 * kMaxRows + t]),
                                    part[3 * kMaxRows + t]);
          const float v = __fadd_rn(xown[t], __fadd_rn(a, sb[xf.bofs + t]));   // x + (h W^T + b)
          xown[t] = v;
          st_word_rep(st.dst + t, (size_t)st.dst_n, __float_as_uint(v), tag);
        }
        q++;
        qi++;
      } else if (st.kind != PH_LM) {
        const float *w = sb + xf.wofs;
        if (have) {
#pragma unroll 1
          for (int k = 0; k < kRowsPerWarp; k += 2) {
            const int i = warp + kWarps * k, i2 = i + kWarps;
            if (i < nr) {
              const bool two = i2 < nr;
              float a, b;
              dot2<NK>(reinterpret_cast<const float4 *>(w + (size_t)i * K),
                       reinterpret_cast<const float4 *>(w + (size_t)(two ? i2 : i) * K), two, xr, lane, a, b);
              if (lane == 0) {
#pragma unroll 1
                for (int u = 0; u < 2; u++) {
                  if (u == 1 && !two) break;
                  const int row = u ? i2 : i;
                  const float y = __fadd_rn(u ? b : a, sb[xf.bofs + row]);
                  switch (st.kind) {
                    case PH_QKV: st_word_rep(st.dst + row, (size_t)st.dst_n, __float_as_uint(y), tag); break;
                    case PH_FC: st_word_rep(st.dst + row, (size_t)st.dst_n, __float_as_uint(gelu_tanh(y)), tag); break;
                    default: {   // PH_O: x + (att W^T + b)
                      const float v = __fadd_rn(xown[row], y);
                      xown[row] = v;
                      st_word_rep(st.dst + row, (size_t)st.dst_n, __float_as_uint(v), tag);
                      break;
                    }
                  }
                }
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        qi++;
      } else {
        // lm_head: the chunks of this CTA's vocab rows, each warp on its own
        const float *w = sb + xf.wofs;
        for (;;) {
          const int cn = xf.nr;
          if (have) {
            for (int i = warp; i < cn; i += 2 * kWarps) {
              const int i2 = i + kWarps;
              const bool two = i2 < cn;
              float a, b;
              dot2<NK>(reinterpret_cast<const float4 *>(w + (size_t)i * K),
                       reinterpret_cast<const float4 *>(w + (size_t)(two ? i2 : i) * K), two, xr, lane, a, b);
              if (lane == 0) {
                const int n = xf.r + i;
                if (logits) logits[n] = a;
                if (better(a, n, best, bidx)) { best = a; bidx = n; }
                if (two) {
                  if (logits) logits[n + kWarps] = b;
                  if (better(b, n + kWarps, best, bidx)) { best = b; bidx = n + kWarps; }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[q & 1]);
          q++;
          if (++qi == nx) qi = 0;
          if (qi == 0) break;
          xf = xfers[qi];
          have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
          w = ring + (size_t)(q & 1) * (kStageBytes / 4) + xf.wofs;
        }
      }
      if (trace) tr[p * kTraceSlots + 4] = gtimer();
    }

    // ---- argmax: publish this CTA's best, fold every CTA's -----------------
    if (lane == 0) {
      rbv[warp] = best;
      rbi[warp] = bidx;
    }
    csync();
    if (warp == 0) {
      const uint32_t tag_am = tag_tok + (uint32_t)n_phases;
      float bv = lane < kWarps ? rbv[lane] : -INFINITY;
      int bi = lane < kWarps ? rbi[lane] : 0x7fffffff;
      warp_best(bv, bi);
      if (lane == 0) {
        st_word_rep(m.part_w + 2 * pc, kPartWords, __float_as_uint(bv), tag_am);
        st_word_rep(m.part_w + 2 * pc + 1, kPartWords, (uint32_t)bi, tag_am);
      }
      bv = -INFINITY;
      bi = 0x7fffffff;
      for (int b = lane; b < P; b += 32) {
        float pw[2];
        wait_words<2>(m.part_w + (size_t)(pc % kReplicas) * kPartWords + 2 * b, 1, 2, tag_am, status, pw);
        const int ib = (int)__float_as_uint(pw[1]);
        if (better(pw[0], ib, bv, bi)) { bv = pw[0]; bi = ib; }
      }
      warp_best(bv, bi);
      if (lane == 0) tok_s[0] = bi == 0x7fffffff ? 0 : bi;
    }
    csync();
    tok = tok_s[0];
  }

  if (pc == 0 && t == 0) {
    if (*(volatile uint32_t *)status == 0) {
      m.io[1] = tok;
      if (m.bump) m.io[0] = ln.pos0 + ln.n_tokens;
    }
    m.sync[3] += 1u;   // next launch: new tags
  }
}

// Producer warp of a projection CTA: every weight transfer of the launch, in
// order, into the stage its consumers released, plus L2 prefetches ahead.
__device__ __noinline__ void producer_role(const Sm100DecodeModel &m, const Launch &ln, unsigned char *smem, int nx) {
  if ((threadIdx.x & 31) != 0) return;
  float *ring = reinterpret_cast<float *>(smem + Smem::ring);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars), *empty = full + 2;
  const XferRec *xfers = reinterpret_cast<const XferRec *>(smem + Smem::xfers(m.n_layers));
  const int total = nx * ln.n_tokens;
  const int n_phases = 5 * m.n_layers + 1;
  uint64_t *tr = m.trace ? m.trace + (size_t)blockIdx.x * n_phases * kTraceSlots : nullptr;
  const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
  int issued = 0, ia = 0;
  for (int qq = 0; qq < total; qq++) {
    const int s = qq & 1, qi = qq % nx;
    // the step a transfer feeds (lm_head: its first chunk), traced on the last token
    const int tp = qi < 4 * m.n_layers ? 5 * (qi / 4) + (qi % 4 == 0 ? 0 : qi % 4 + 1) : (qi == 4 * m.n_layers ? 5 * m.n_layers : -1);
    const bool trace = tr && qq >= total - nx && tp >= 0;
    if (trace) tr[tp * kTraceSlots + 6] = gtimer();
    if (qq >= 2 && !mbar_wait(&empty[s], ((qq >> 1) - 1) & 1, ln.status)) break;
    issue(xfers[qi], s, ring, full, pol_stream, pol_keep);
    if (trace) tr[tp * kTraceSlots + 5] = gtimer();
    issued = qq + 1;
    for (; ia < qq + 2 + kPrefetchAhead && ia < total; ia++) {
      if (ia < 2) continue;
      const XferRec &x = xfers[ia % nx];
      if (x.wbytes) bulk_prefetch_l2(x.w, x.wbytes);
    }
  }
  // every issued transfer has landed before the CTA exits (bounded, not cut
  // short by the status)
  for (int qq = issued - 2; qq < issued; qq++)
    if (qq >= 0) mbar_wait(&full[qq & 1], (qq >> 1) & 1, ln.status, false);
}

template <int NK>
__global__ void __launch_bounds__(kBlockThreads, 1) decode_kernel(const Sm100DecodeModel *__restrict__ mp, int n_tokens) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const Sm100DecodeModel &m = *mp;
  const int c = blockIdx.x, t = threadIdx.x;
  const int A = m.heads, P = gridDim.x - A;
  const bool att = c < A;
  Launch ln;
  ln.n_tokens = n_tokens;
  ln.status = m.sync + 2;
  // tags: (launch epoch mod 65535 + 1) << 16 | token * stride + step: never
  // 0 (the zero-initialised words), distinct from the previous launch's and
  // within a launch one per (token, step)
  ln.tag_base = ((m.sync[3] % 65535u) + 1u) << 16;
  ln.stride = (uint32_t)(5 * m.n_layers + 2);
  ln.pos0 = m.io[0];
  // a position range outside the cache is an argument error: flag it and keep
  // every access in bounds (positions from 0, no cache write, nothing published)
  ln.pos_ok = ln.pos0 >= 0 && ln.pos0 + n_tokens <= m.max_ctx;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  int nx = 0;
  if (!att) {
    StepRec *steps = reinterpret_cast<StepRec *>(smem + Smem::steps);
    XferRec *xfers = reinterpret_cast<XferRec *>(smem + Smem::xfers(m.n_layers));
    const int n_phases = 5 * m.n_layers + 1;
    nx = xfers_per_token(m, c - A, P);
    if (nx > 4 * m.n_layers + kMaxLmChunks) {   // vocab too large for the schedule table
      if (t == 0) atomicOr(ln.status, SM100_DECODE_ERR_ARG);
      nx = 4 * m.n_layers + kMaxLmChunks;
    }
    for (int p = t; p < n_phases; p += kBlockThreads) build_step(m, p, c - A, P, steps[p]);
    for (int i = t; i < nx; i += kBlockThreads) build_xfer(m, i, c - A, P, xfers[i]);
  }
  if (t == 0) {
    if (!ln.pos_ok && c == A) atomicOr(ln.status, SM100_DECODE_ERR_ARG);
    mbar_init(&bars[0], 1);        // full[0], full[1]: armed by the producer
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], kWarps);   // empty[0], empty[1]: one arrival per consumer warp
    mbar_init(&bars[3], kWarps);
    mbar_init(&bars[4], 1);        // attention prefix
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (t >= kThreads) {
    if (!att) producer_role(m, ln, smem, nx);
    return;
  }
  if (att)
    attention_role<NK>(m, ln, smem);
  else
    projection_role<NK>(m, ln, smem, nx);
}

}  // namespace sm100

using namespace sm100;

static int g_num_sms[64];

extern "C" uint64_t sm100_decode_sync_bytes(void) { return (uint64_t)(4 + 2 * 1024) * 4; }

extern "C" uint64_t sm100_decode_part_bytes(void) { return (uint64_t)kPartWords * 8 * kReplicas; }

extern "C" uint64_t sm100_decode_trace_bytes(int32_t n_layers) {
  return (uint64_t)1024 * (5 * (uint64_t)(n_layers > 0 ? n_layers : 0) + 1) * kTraceSlots * 8;
}

template <int NK>
static int launch_decode(const Sm100DecodeModel *dev_model, int n_tokens, int G, size_t smem, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(decode_kernel<NK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "decode: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kBlockThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, decode_kernel<NK>, dev_model, n_tokens);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "decode: launch: %s", cudaGetErrorString(e));
  return launch_status("decode");
}

// The host checks the shape from the scalars it is given (the descriptor
// itself lives in device memory and must carry the same values).
extern "C" int sm100_decode_steps(const Sm100DecodeModel *dev_model, int32_t n_tokens, int32_t n_layers, int32_t dim,
                                  int32_t heads, int32_t vocab, int32_t max_ctx, void *stream) {
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
  const int hd = heads > 0 ? dim / heads : 0, P = G - heads;
  const int64_t K = dim;
  bool ok = dev_model && G <= 1024 && n_tokens > 0 && (int64_t)n_tokens * (5 * n_layers + 2) < 65536 && n_layers > 0 &&
            n_layers <= kMaxLayers && dim > 0 && dim % 128 == 0 && heads > 0 && hd * heads == dim &&
            (hd == 32 || hd == 64) && P >= 1 && vocab > 0 && max_ctx > 0 &&
            2LL * max_ctx + 3LL * hd + kThreads <= 2LL * kXsFloats && 4 * K <= kXsFloats;
  if (ok) {
    const int64_t rq = (3 * K + P - 1) / P, rf = (4 * K + P - 1) / P, rd = (K + P - 1) / P;
    const int64_t R = lm_rows_per_chunk(K), rv = ((int64_t)vocab + P - 1) / P;
    const int64_t extra = 2 * K * 4 + kBiasFloats * 4;   // LayerNorm parameters + biases
    ok = rq <= kMaxRows && rf <= kMaxRows && rd <= kMaxRows && rq * K * 4 + extra <= kStageBytes &&
         rf * K * 4 + extra <= kStageBytes && rd * 4 * K * 4 + kBiasFloats * 4 <= kStageBytes && R >= 1 &&
         (rv + R - 1) / R <= kMaxLmChunks && Smem::total(n_layers) <= (size_t)kSmemLimit;
  }
  if (!ok)
    return sm100_set_error(SM100_ERR_ARG,
                           "decode: unsupported shape (tokens %d, layers %d, dim %d, heads %d, vocab %d, ctx %d, %d SMs)",
                           n_tokens, n_layers, dim, heads, vocab, max_ctx, G);
  const size_t smem = Smem::total(n_layers);
  switch (dim / 128) {
    case 4: return launch_decode<4>(dev_model, n_tokens, G, smem, (cudaStream_t)stream);
    case 6: return launch_decode<6>(dev_model, n_tokens, G, smem, (cudaStream_t)stream);
    case 8: return launch_decode<8>(dev_model, n_tokens, G, smem, (cudaStream_t)stream);
    default:
      return sm100_set_error(SM100_ERR_ARG, "decode: dim %d not built (512, 768 or 1024)", dim);
  }
}

extern "C" int sm100_decode_step(const Sm100DecodeModel *dev_model, int32_t n_layers, int32_t dim, int32_t heads,
                                 int32_t vocab, int32_t max_ctx, void *stream) {
  return sm100_decode_steps(dev_model, 1, n_layers, dim, heads, vocab, max_ctx, stream);
}
