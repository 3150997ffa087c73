// GPT-2 decoding (batch 1, fp32) as ONE persistent kernel that runs n greedy
// tokens: per token the whole schedule of thvm_gpt2.py's Transformer.forward
// (embedding, n_layers x {ln_1 + c_attn, attention + KV append, c_proj +
// residual, ln_2 + c_fc + GELU, mlp.c_proj + residual}, ln_f + lm_head,
// argmax), the position and token carried on the device, so one launch
// replaces n TinyJit replays.
//
// A token reads 495 MB of weights once (77 us at the HBM roofline) but is a
// chain of dependent steps, each too small to fill the GPU; every hand-over
// between CTAs costs ~1-2.5 us (L2 round trips), so the design minimises the
// hand-overs per layer to three:
//
//  * Head groups.  The grid is heads x M CTAs (M members per head, 12 x 12 =
//    144 for GPT-2 small).  Member j of head h computes 3 hd / M rows of
//    c_attn (a contiguous slice of q_h, k_h or v_h; k and v owners also write
//    the KV cache) and publishes them to the group as tagged words (hop 1:
//    12 producers, 12 consumers).  Every member then runs head h's attention
//    itself (the head's earlier keys / values staged in shared memory by bulk
//    copies one layer ahead) and multiplies it by its D / M output rows of
//    c_proj's head-h column block: c_proj is split over its K dimension by
//    head, so attention and c_proj need no hand-over between them.
//  * Reduction words.  The K-split partial sums meet in 64-bit words in
//    global memory: each contribution adds (1 << 48) + round(v * 2^28) with
//    red.add.u64, so the top 16 bits count the contributions and the low 48
//    hold an exact fixed-point sum.  A consumer polls a word until its count
//    reaches the expected value, which makes the sum independent of the
//    order of arrival (deterministic) and needs no separate flag.  c_proj's
//    heads meet in one set (hop 2: H contributions per word), mlp.c_proj's in
//    another (hop 3).
//  * Every CTA does c_fc rows + GELU and immediately the matching K slice of
//    mlp.c_proj (its rows of the transposed weight), so the 4 dim hidden
//    vector is never exchanged.  Each CTA keeps the whole residual stream in
//    shared memory and adds the decoded sums itself (bias, then residual, the
//    reference's order), so LayerNorm needs no further exchange.
//  * Weights never wait for activations.  One producer warp per CTA keeps
//    TMA bulk copies (cp.async.bulk + mbarrier) of the coming slices in a
//    2 x 76 KB shared-memory ring plus L2 prefetches a few slices ahead;
//    lm_head (154 MB) streams through the same ring in chunks.
//
// Math is the reference's op order (LayerNorm two-pass with recip(sqrt), bias
// then GELU / residual, scale -> max -> xexp2 -> sum -> recip, first index of
// the max); dot products are tree-ordered and the split sums are rounded to
// 2^-28 per contribution (~1e-9 absolute, far inside the 1e-4 tolerance).
//
// Waits are bounded (~1 s): a timeout sets the status word, every later wait
// returns at once, the kernel runs to its end, and every CTA waits (bounded)
// for its in-flight bulk copies before it exits.  One CTA per SM, launched
// cooperatively (the spin-waits need every CTA resident).
#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kWarps = 15;                   // consumer warps (16 warps in all: 128 registers)
constexpr int kThreads = kWarps * 32;        // consumer threads
constexpr int kBlockThreads = kThreads + 32; // + one producer warp (TMA issue)
constexpr int kStages = 2;                   // weight ring stages
constexpr int kStageBytes = 76 * 1024;       // one stage
constexpr int kMaxDim = 1024;                // residual stream held in shared memory
constexpr int kRowsPerWarp = 4;              // row slots of a warp in c_attn / c_fc steps (even)
constexpr int kMaxRows = kRowsPerWarp * kWarps;
constexpr int kMaxHd = 64;
constexpr int kPrefetchAhead = 4;            // L2 prefetch distance in transfers
constexpr int kMaxLayers = SM100_DECODE_MAX_LAYERS;
constexpr int kBiasFloats = 64;              // stage region of a transfer's bias slice
constexpr int kSmemLimit = 227 * 1024;
constexpr int kTraceSlots = 8;               // u64 timestamps per (CTA, step) in the optional trace
constexpr size_t kPartWords = 2 * 1024;      // argmax partials of one copy: (value, index) per CTA
constexpr int kFixShift = 28;                // reduction words: fixed point with 28 fraction bits
constexpr float kFixLimit = 2048.0f;         // |contribution| bound (sums stay below 2^47 / 2^28)

// Argmax partials go to kReplicas copies; consumer CTA c polls copy c % kReplicas
// (every CTA reads every CTA's partial).
constexpr int kReplicas = SM100_DECODE_REPLICAS;

// ---- tagged words ------------------------------------------------------------
__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_word(uint64_t *p, uint32_t bits, uint32_t tag) {
  const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)bits;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ void st_word_rep(uint64_t *p, size_t n, uint32_t bits, uint32_t tag) {
#pragma unroll
  for (int r = 0; r < kReplicas; r++) st_word(p + (size_t)r * n, bits, tag);
}

__device__ __forceinline__ void ld_pair(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
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

// One pair of tagged words (p[0], p[1]) with a 16-byte load per poll (bounded).
__device__ __forceinline__ float2 wait_pair(const uint64_t *p, uint32_t tag, uint32_t *status) {
  uint64_t a, b;
  ld_pair(p, a, b);
  for (uint32_t it = 0; (uint32_t)(a >> 32) != tag || (uint32_t)(b >> 32) != tag; it++) {
    if (it >= (1u << 22) || ((it & 15u) == 15u && *(volatile uint32_t *)status)) {
      if (it >= (1u << 22)) atomicOr(status, SM100_DECODE_ERR_BARRIER);
      return make_float2(0.0f, 0.0f);
    }
    ld_pair(p, a, b);
  }
  return make_float2(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b));
}

// ---- reduction words -------------------------------------------------------
// A contribution v adds (1 << 48) + round(v * 2^28) (two's complement, mod
// 2^64).  After C contributions (count taken mod 2^16) the word minus C << 48
// is the exact fixed-point sum, |sum| < 2^47; with k < 2^15 contributions
// still missing it lies at least 2^47 away from that range.
__device__ __forceinline__ void red_word(uint64_t *p, float v, uint32_t *status) {
  if (!(fabsf(v) <= kFixLimit)) {   // also NaN: flagged, counted as 0
    atomicOr(status, SM100_DECODE_ERR_RANGE);
    v = 0.0f;
  }
  const long long q = __float2ll_rn(v * (float)(1 << kFixShift));   // exact scaling by 2^28
  const unsigned long long w = (1ull << 48) + (unsigned long long)q;
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ bool red_done(uint64_t w, uint64_t C) {
  const long long d = (long long)(w - (C << 48));
  return d > -(1ll << 47) && d < (1ll << 47);
}

__device__ __forceinline__ float red_value(uint64_t w, uint64_t C) {
  return __ll2float_rn((long long)(w - (C << 48))) * (1.0f / (float)(1 << kFixShift));
}

// The pair of reduction words (p[0], p[1]) once both counts reach C (bounded).
__device__ __forceinline__ float2 wait_red_pair(const uint64_t *p, uint64_t C, uint32_t *status) {
  uint64_t a, b;
  ld_pair(p, a, b);
  for (uint32_t it = 0; !(red_done(a, C) && red_done(b, C)); it++) {
    if (it >= (1u << 22) || ((it & 15u) == 15u && *(volatile uint32_t *)status)) {
      if (it >= (1u << 22)) atomicOr(status, SM100_DECODE_ERR_BARRIER);
      return make_float2(0.0f, 0.0f);
    }
    ld_pair(p, a, b);
  }
  return make_float2(red_value(a, C), red_value(b, C));
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

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

// rows [r0, r1) of an N-row projection owned by CTA c of P
__host__ __device__ __forceinline__ void rows_of(int64_t N, int c, int P, int64_t &r0, int64_t &r1) {
  r0 = (N * c) / P;
  r1 = (N * (c + 1)) / P;
}

// Members per head: the largest M <= SMs / heads with 3 hd / M rows per member
// dividing hd (a member's c_attn rows lie inside one of q_h, k_h, v_h).
__host__ __device__ __forceinline__ int members_per_head(int heads, int hd, int n_sm) {
  int best = 0;
  for (int s = 1; s <= hd; s++)
    if (hd % s == 0) {
      const int M = 3 * hd / s;
      if (M >= 3 && (int64_t)M * heads <= n_sm && M > best) best = M;
    }
  return best;
}

// Stage layout of a transfer with a header (c_attn, c_fc, lm_head chunks):
// [ln_g | ln_b] (2 dim floats), [bx] (dim floats: the full bias of the
// preceding split projection), [bias slice from the 16-byte boundary at or
// below row r] (kBiasFloats), then the weight rows.  Transfers of the split
// weights (c_proj head block, transposed mlp.c_proj) hold rows only.
__host__ __device__ __forceinline__ int hdr_floats(int D) { return 3 * D + kBiasFloats; }

__host__ __device__ __forceinline__ int lm_rows_per_chunk(int D) {
  return (kStageBytes / 4 - hdr_floats(D)) / D;
}

// One CTA's share of every step.
struct Geo {
  int G, M, h, mb;     // grid, members per head, head, member
  int qn, ql0;         // c_attn rows per member; first local row (of the head's 3 hd)
  int qrow0;           // its first global c_attn row
  int kv_which;        // 0: q rows, 1: k rows, 2: v rows
  int qcol0;           // its first column of the head's k / v in a cache row
  int o0, o1;          // c_proj output rows
  int f0, f1;          // c_fc rows = mlp.c_proj K slice
  int v0, v1, R, n_lm; // lm_head rows, rows per chunk, chunks
  int nx;              // transfers per token
};

__host__ __device__ __forceinline__ Geo geo_of(int c, int G, int heads, int D, int hd, int vocab, int n_layers) {
  Geo g;
  g.G = G;
  g.M = G / heads;
  g.h = c / g.M;
  g.mb = c % g.M;
  g.qn = 3 * hd / g.M;
  g.ql0 = g.mb * g.qn;
  g.kv_which = g.ql0 / hd;
  g.qcol0 = g.h * hd + g.ql0 % hd;
  g.qrow0 = g.kv_which * D + g.qcol0;
  int64_t a, b;
  rows_of(D, g.mb, g.M, a, b);
  g.o0 = (int)a; g.o1 = (int)b;
  rows_of(4 * (int64_t)D, c, G, a, b);
  g.f0 = (int)a; g.f1 = (int)b;
  rows_of(vocab, c, G, a, b);
  g.v0 = (int)a; g.v1 = (int)b;
  g.R = lm_rows_per_chunk(D);
  const int n = g.R > 0 ? (g.v1 - g.v0 + g.R - 1) / g.R : 1;
  g.n_lm = n > 0 ? n : 1;
  g.nx = 4 * n_layers + g.n_lm;
  return g;
}

// One weight transfer: [kind of step, layer] or an lm_head chunk.
struct Xfer {
  const float *w, *ln_g, *ln_b, *bx, *b;
  uint32_t wbytes, bbytes;
  int hdr;     // floats before the weight rows
};

__device__ __forceinline__ Xfer xfer_of(const Sm100DecodeModel &m, const Geo &g, int i) {
  const int D = m.dim, hd = m.head_dim, nl = m.n_layers;
  Xfer x;
  x.ln_g = x.ln_b = x.bx = x.b = nullptr;
  x.bbytes = 0;
  int r = 0, nr = 0;
  const float *bias = nullptr;
  if (i < 4 * nl) {
    const int l = i >> 2;
    switch (i & 3) {
      case 0:   // c_attn rows; header: ln_1, mlp.c_proj bias of layer l - 1
        r = g.qrow0; nr = g.qn;
        x.w = m.w_qkv[l] + (size_t)r * D;
        x.ln_g = m.ln1_g[l]; x.ln_b = m.ln1_b[l];
        x.bx = l > 0 ? m.b_p2[l - 1] : nullptr;
        bias = m.b_qkv[l];
        break;
      case 1:   // c_proj head-h block, output rows [o0, o1)
        nr = g.o1 - g.o0;
        x.w = m.w_o_h[l] + ((size_t)g.h * D + g.o0) * hd;
        x.wbytes = (uint32_t)(nr * hd * 4);
        x.hdr = 0;
        return x;
      case 2:   // c_fc rows; header: ln_2, c_proj bias
        r = g.f0; nr = g.f1 - g.f0;
        x.w = m.w_fc[l] + (size_t)r * D;
        x.ln_g = m.ln2_g[l]; x.ln_b = m.ln2_b[l];
        x.bx = m.b_o[l];
        bias = m.b_fc[l];
        break;
      default:  // transposed mlp.c_proj rows [f0, f1)
        nr = g.f1 - g.f0;
        x.w = m.w_p2_t[l] + (size_t)g.f0 * D;
        x.wbytes = (uint32_t)(nr * D * 4);
        x.hdr = 0;
        return x;
    }
  } else {
    const int j = i - 4 * nl;
    r = g.v0 + j * g.R;
    nr = r + g.R <= g.v1 ? g.R : (g.v1 > r ? g.v1 - r : 0);
    x.w = m.lm_head + (size_t)r * D;
    if (j == 0) {   // header: ln_f, mlp.c_proj bias of the last layer
      x.ln_g = m.ln_f_g; x.ln_b = m.ln_f_b;
      x.bx = m.b_p2[nl - 1];
    }
  }
  x.hdr = hdr_floats(D);
  x.wbytes = (uint32_t)((size_t)nr * D * 4);
  if (bias && nr > 0) {
    const int b0 = r & ~3, b1 = (r + nr + 3) & ~3;
    x.b = bias + b0;
    x.bbytes = (uint32_t)((b1 - b0) * 4);
  }
  return x;
}

__device__ __forceinline__ uint32_t xfer_bytes(const Xfer &x, int D) {
  return x.wbytes + x.bbytes + (x.ln_g ? 8u * D : 0u) + (x.bx ? 4u * D : 0u);
}

__device__ __forceinline__ void issue(const Xfer &x, int D, float *dst, uint64_t *full, uint64_t pol_stream,
                                      uint64_t pol_keep) {
  mbar_expect_tx(full, xfer_bytes(x, D));
  if (x.ln_g) {
    bulk_g2s_hint(dst, x.ln_g, 4u * D, full, pol_keep);
    bulk_g2s_hint(dst + D, x.ln_b, 4u * D, full, pol_keep);
  }
  if (x.bx) bulk_g2s_hint(dst + 2 * D, x.bx, 4u * D, full, pol_keep);
  if (x.bbytes) bulk_g2s_hint(dst + 3 * D, x.b, x.bbytes, full, pol_keep);
  if (x.wbytes) bulk_g2s_hint(dst + x.hdr, x.w, x.wbytes, full, pol_stream);
}

// Shared-memory layout (bytes): fixed part, then the scores and the staged
// keys / values of one head (as many positions as fit, smax).
struct Smem {
  static constexpr size_t ring = 0;
  static constexpr size_t xres = ring + (size_t)kStages * kStageBytes;  // [kMaxDim] residual stream
  static constexpr size_t fv = xres + kMaxDim * 4;                        // [kMaxRows] c_fc outputs
  static constexpr size_t qkvs = fv + 64 * 4;                             // [3 kMaxHd] q, k, v of the head
  static constexpr size_t atts = qkvs + 3 * kMaxHd * 4;                   // [kMaxHd] attention output
  static constexpr size_t acc = atts + kMaxHd * 4;                        // [kThreads] p @ v slices
  static constexpr size_t rbv = acc + kThreads * 4;                       // [kWarps] f32 (+1 pad)
  static constexpr size_t rbi = rbv + 16 * 4;                             // [kWarps] i32
  static constexpr size_t tok = rbi + 16 * 4;                             // [4] i32
  static constexpr size_t bars = tok + 16;                                // full[2], empty[2], pfx
  static constexpr size_t kcs = bars + 8 * 8;                             // [kMaxLayers] cache pointers
  static constexpr size_t sc = kcs + kMaxLayers * 8;                      // [2][max_ctx] scores, probabilities
  static __host__ __device__ size_t kv(int max_ctx) { return (sc + 2 * (size_t)max_ctx * 4 + 127) & ~(size_t)127; }
  static __host__ __device__ int smax(int max_ctx, int hd) {
    const int64_t n = ((int64_t)kSmemLimit - (int64_t)kv(max_ctx)) / (8 * hd);
    return (int)(n < max_ctx ? (n > 0 ? n : 0) : max_ctx);
  }
  static __host__ __device__ size_t total(int max_ctx, int hd) { return kv(max_ctx) + (size_t)smax(max_ctx, hd) * 8 * hd; }
};

struct Launch {
  int n_tokens, pos0;
  bool pos_ok;
  uint32_t tag_base, stride;   // tag of (token tk, step p): tag_base + tk * stride + p
  uint32_t *status;
  uint32_t tok0;               // tokens decoded by earlier launches (selects the reduction sets)
};

template <int NK>
__device__ __forceinline__ void load_x(const float *xb, int lane, float (&xr)[4 * NK]) {
#pragma unroll
  for (int j = 0; j < NK; j++) {
    const float4 v = reinterpret_cast<const float4 *>(xb)[lane + 32 * j];
    xr[4 * j] = v.x; xr[4 * j + 1] = v.y; xr[4 * j + 2] = v.z; xr[4 * j + 3] = v.w;
  }
}

// LayerNorm of the vector in the lanes' registers (statistics by warp
// shuffles), gamma / beta from the stage front.
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

// This thread's pairs j = t + i kThreads of a set of D reduction words
// (count C), decoded; pairs past D read as 0.
constexpr int kPairsPerThread = (kMaxDim / 2 + kThreads - 1) / kThreads;

__device__ __forceinline__ void poll_reduced(const uint64_t *words, int D, uint64_t C, uint32_t *status, int t,
                                             float2 (&sv)[kPairsPerThread]) {
#pragma unroll
  for (int i = 0; i < kPairsPerThread; i++) {
    const int j = t + i * kThreads;
    sv[i] = 2 * j < D ? wait_red_pair(words + 2 * j, C, status) : make_float2(0.0f, 0.0f);
  }
}

// x += (decoded sum + bias), the reference's order: the projection's bias
// first, then the residual.
__device__ __forceinline__ void add_reduced(float *xres, const float *bias, int D, int t,
                                            const float2 (&sv)[kPairsPerThread]) {
#pragma unroll
  for (int i = 0; i < kPairsPerThread; i++) {
    const int j = t + i * kThreads;
    if (2 * j < D) {
      const float2 bb = reinterpret_cast<const float2 *>(bias)[j];
      float2 *xp = reinterpret_cast<float2 *>(xres) + j;
      const float2 xv = *xp;
      *xp = make_float2(__fadd_rn(xv.x, __fadd_rn(sv[i].x, bb.x)), __fadd_rn(xv.y, __fadd_rn(sv[i].y, bb.y)));
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer warps of every CTA: the steps of every token.
template <int NK>
__device__ __forceinline__ void consumer_role(const Sm100DecodeModel &m, const Launch &ln, const Geo &g,
                                              unsigned char *smem) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int D = m.dim, hd = m.head_dim, nl = m.n_layers, max_ctx = m.max_ctx, H = m.heads;
  float *ring = reinterpret_cast<float *>(smem + Smem::ring);
  float *xres = reinterpret_cast<float *>(smem + Smem::xres);
  float *fv = reinterpret_cast<float *>(smem + Smem::fv);
  float *qs = reinterpret_cast<float *>(smem + Smem::qkvs), *kn = qs + hd, *vn = kn + hd;
  float *atts = reinterpret_cast<float *>(smem + Smem::atts);
  float *acc = reinterpret_cast<float *>(smem + Smem::acc);
  float *rbv = reinterpret_cast<float *>(smem + Smem::rbv);
  int *rbi = reinterpret_cast<int *>(smem + Smem::rbi);
  int *tok_s = reinterpret_cast<int *>(smem + Smem::tok);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars), *empty = full + 2, *pfx = full + 4;
  float *const *kcs = reinterpret_cast<float *const *>(smem + Smem::kcs);
  float *sc = reinterpret_cast<float *>(smem + Smem::sc), *pr = sc + max_ctx;
  const int smax = Smem::smax(max_ctx, hd);
  float *Ks = reinterpret_cast<float *>(smem + Smem::kv(max_ctx));
  float *Vs = Ks + (size_t)smax * hd;
  uint32_t *status = ln.status;
  const int vocab = m.vocab;
  const float eps = m.eps;
  float *logits = m.logits;
  uint64_t *tr = m.trace ? m.trace + (size_t)blockIdx.x * (3 * nl + 1) * kTraceSlots : nullptr;
  uint64_t *qkv_w = m.qkv_w + (size_t)g.h * 3 * hd;
  const int hdr = hdr_floats(D);

  // prefix copies of (layer l, rows [0, n)) of head h; thread 0 armed pfx
  auto issue_prefix = [&](int l, int n) {
    const float *kc = kcs[l], *vc = kc + (size_t)max_ctx * D;
    for (int j = t; j < n; j += kThreads) {
      bulk_g2s(Ks + (size_t)j * hd, kc + (size_t)j * D + (size_t)g.h * hd, (uint32_t)hd * 4, pfx);
      bulk_g2s(Vs + (size_t)j * hd, vc + (size_t)j * D + (size_t)g.h * hd, (uint32_t)hd * 4, pfx);
    }
  };
  auto staged = [&](int n) { return n < smax ? n : smax; };

  int q = 0;            // next ring transfer (stage q & 1, phase (q >> 1) & 1)
  int pf = 0;           // prefix phases consumed
  bool pending = true;  // a prefix phase is armed and not yet waited for
  {
    const int n = staged(ln.pos_ok ? ln.pos0 : 0);
    if (t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * n * hd * 4));
    csync();
    issue_prefix(0, n);
  }
  int tok = m.io[1];
  for (int tk = 0; tk < ln.n_tokens; tk++) {
    const int pos = ln.pos_ok ? ln.pos0 + tk : 0, L = pos + 1;
    const uint32_t tag_tok = ln.tag_base + (uint32_t)tk * ln.stride;
    const bool trace = tr && t == 0 && tk == ln.n_tokens - 1;
    const uint64_t C_att = (uint64_t)H, C_mlp = (uint64_t)g.G;
    // reduction words of this token: set (tok0 + tk) mod 3.  This token
    // zeroes the next token's set (last read two tokens ago: every CTA has
    // passed that token's argmax; the zeros are released by this token's
    // argmax publish, before which no CTA starts the next token)
    const size_t n_red = (size_t)2 * nl * D;
    uint64_t *red = m.red_w + (size_t)((ln.tok0 + (uint32_t)tk) % 3u) * n_red;
    {
      uint64_t *nxt = m.red_w + (size_t)((ln.tok0 + (uint32_t)tk + 1u) % 3u) * n_red;
      int64_t z0, z1;
      rows_of((int64_t)n_red, blockIdx.x, g.G, z0, z1);
      for (int64_t i = z0 + t; i < z1; i += kThreads) nxt[i] = 0ull;
    }

    // x = wte[tok] + wpe[pos] (thvm_gpt2.py:93-103)
    {
      const bool tok_ok = tok >= 0 && tok < vocab;
      for (int k = t; k < D; k += kThreads)
        xres[k] = __fadd_rn(tok_ok ? m.wte[(size_t)tok * D + k] : 0.0f, m.wpe[(size_t)pos * D + k]);
    }

    for (int l = 0; l < nl; l++) {
      uint64_t *red_att = red + (size_t)(2 * l) * D, *red_mlp = red_att + D;
      // ===== c_attn rows of this member (ln_1 of x; x += mlp output of l - 1)
      {
        const int p = 3 * l;
        if (trace) tr[p * kTraceSlots + 0] = gtimer();
        float2 sv[kPairsPerThread];
        if (l > 0) poll_reduced(red_mlp - 2 * D, D, C_mlp, status, t, sv);
        if (trace) tr[p * kTraceSlots + 1] = gtimer();
        const bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        const float *sb = ring + (size_t)(q & 1) * (kStageBytes / 4);
        if (trace) tr[p * kTraceSlots + 2] = gtimer();
        if (l > 0) add_reduced(xres, sb + 2 * D, D, t, sv);
        csync();
        if (trace) tr[p * kTraceSlots + 3] = gtimer();
        float xr[4 * NK];
        load_x<NK>(xres, lane, xr);
        layernorm_regs<NK>(xr, sb, sb + D, lane, D, eps);
        if (trace) tr[p * kTraceSlots + 7] = gtimer();
        const int nr = g.qn, bofs = 3 * D + (g.qrow0 & 3);
        const uint32_t tag = tag_tok + (uint32_t)l;
        float *cache = ln.pos_ok && g.kv_which > 0 ? kcs[l] + (size_t)(g.kv_which - 1) * max_ctx * D + (size_t)pos * D + g.qcol0
                                                   : nullptr;
        if (have) {
#pragma unroll 1
          for (int k = 0; k < kRowsPerWarp; k += 2) {
            const int i = warp + kWarps * k, i2 = i + kWarps;
            if (i < nr) {
              const bool two = i2 < nr;
              float a, b;
              dot2<NK>(reinterpret_cast<const float4 *>(sb + hdr + (size_t)i * D),
                       reinterpret_cast<const float4 *>(sb + hdr + (size_t)(two ? i2 : i) * D), two, xr, lane, a, b);
              if (lane == 0) {
                const float y = __fadd_rn(a, sb[bofs + i]);
                st_word(qkv_w + g.ql0 + i, __float_as_uint(y), tag);
                if (cache) cache[i] = y;
                if (two) {
                  const float y2 = __fadd_rn(b, sb[bofs + i2]);
                  st_word(qkv_w + g.ql0 + i2, __float_as_uint(y2), tag);
                  if (cache) cache[i2] = y2;
                }
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        if (trace) tr[p * kTraceSlots + 4] = gtimer();
      }

      // ===== attention of head h, then this member's rows of c_proj's head-h block
      {
        const int p = 3 * l + 1;
        const uint32_t tag = tag_tok + (uint32_t)l;
        if (trace) tr[p * kTraceSlots + 0] = gtimer();
        // the prefix copies are ours and always complete: wait for them even
        // after an error, so the staging area is never written by two phases
        mbar_wait(pfx, (uint32_t)(pf & 1), status, false);
        pf++;
        pending = false;
        // q, k, v of the new row from the group (k, v also staged at pos)
        for (int j = t; 2 * j < 3 * hd; j += kThreads) {
          const float2 v = wait_pair(qkv_w + 2 * j, tag, status);
          reinterpret_cast<float2 *>(qs)[j] = v;
          const int i = 2 * j, which = i / hd, dd = i % hd;
          if (which > 0 && pos < smax)
            *reinterpret_cast<float2 *>((which == 1 ? Ks : Vs) + (size_t)pos * hd + dd) = v;
        }
        csync();
        if (trace) tr[p * kTraceSlots + 1] = gtimer();
        const float *kc = kcs[l], *vc = kc + (size_t)max_ctx * D;
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
                    k4[v] = __ldcg(reinterpret_cast<const float4 *>(kc + (size_t)j * D + (size_t)g.h * hd) + gl * per4 + v);
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
        if (trace) tr[p * kTraceSlots + 2] = gtimer();
        // p @ v: key slices x dims, then the slices in order
        const int nslice = kThreads / hd;
        {
          const int slice = t / hd, d = t % hd;
          if (slice < nslice) {
            float a = 0.0f;
            for (int j = slice; j < L; j += nslice) {
              const float v = j < smax ? Vs[(size_t)j * hd + d] : j == pos ? vn[d] : __ldcg(vc + (size_t)j * D + (size_t)g.h * hd + d);
              a = fmaf(pr[j], v, a);
            }
            acc[slice * hd + d] = a;
          }
        }
        // the next layer's prefix (rows < pos, written in earlier tokens); the
        // next token's layer 0 is staged after the argmax (it needs row pos)
        const bool more = l + 1 < nl;
        const int nrows = more ? staged(pos) : 0;
        if (more && t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * nrows * hd * 4));
        csync();
        if (t < hd) {
          float a = 0.0f;
          for (int s2 = 0; s2 < nslice; s2++) a += acc[s2 * hd + t];
          atts[t] = a;
        }
        if (more) {
          issue_prefix(l + 1, nrows);
          pending = true;
        }
        csync();
        if (trace) tr[p * kTraceSlots + 3] = gtimer();
        // c_proj partial: rows [o0, o1) of the head-h column block, four rows
        // per warp at a time (lanes over the head's dims)
        const bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        const float *sb = ring + (size_t)(q & 1) * (kStageBytes / 4);
        if (have) {
          const int nr = g.o1 - g.o0;
          float av[kMaxHd / 32];
#pragma unroll
          for (int u = 0; u < kMaxHd / 32; u++) av[u] = lane + 32 * u < hd ? atts[lane + 32 * u] : 0.0f;
          for (int i0 = warp * 4; i0 < nr; i0 += kWarps * 4) {
            float s[4];
#pragma unroll
            for (int r = 0; r < 4; r++) {
              s[r] = 0.0f;
              const int i = i0 + r < nr ? i0 + r : i0;
#pragma unroll
              for (int u = 0; u < kMaxHd / 32; u++)
                if (lane + 32 * u < hd) s[r] = fmaf(sb[(size_t)i * hd + lane + 32 * u], av[u], s[r]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
              for (int r = 0; r < 4; r++) s[r] += __shfl_xor_sync(0xffffffffu, s[r], o);
            if (lane < 4 && i0 + lane < nr) {
              const float v = lane == 0 ? s[0] : lane == 1 ? s[1] : lane == 2 ? s[2] : s[3];
              red_word(red_att + g.o0 + i0 + lane, v, status);
            }
          }
        } else {
          for (int i = t; i < g.o1 - g.o0; i += kThreads) red_word(red_att + g.o0 + i, 0.0f, status);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        if (trace) tr[p * kTraceSlots + 4] = gtimer();
      }

      // ===== c_fc rows + GELU, then their K slice of mlp.c_proj
      {
        const int p = 3 * l + 2;
        if (trace) tr[p * kTraceSlots + 0] = gtimer();
        float2 sv[kPairsPerThread];
        poll_reduced(red_att, D, C_att, status, t, sv);
        if (trace) tr[p * kTraceSlots + 1] = gtimer();
        bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        const float *sb = ring + (size_t)(q & 1) * (kStageBytes / 4);
        if (trace) tr[p * kTraceSlots + 2] = gtimer();
        add_reduced(xres, sb + 2 * D, D, t, sv);   // x += (att c_proj + b)
        csync();
        if (trace) tr[p * kTraceSlots + 3] = gtimer();
        float xr[4 * NK];
        load_x<NK>(xres, lane, xr);
        layernorm_regs<NK>(xr, sb, sb + D, lane, D, eps);
        if (trace) tr[p * kTraceSlots + 7] = gtimer();
        const int nr = g.f1 - g.f0, bofs = 3 * D + (g.f0 & 3);
        if (have) {
#pragma unroll 1
          for (int k = 0; k < kRowsPerWarp; k += 2) {
            const int i = warp + kWarps * k, i2 = i + kWarps;
            if (i < nr) {
              const bool two = i2 < nr;
              float a, b;
              dot2<NK>(reinterpret_cast<const float4 *>(sb + hdr + (size_t)i * D),
                       reinterpret_cast<const float4 *>(sb + hdr + (size_t)(two ? i2 : i) * D), two, xr, lane, a, b);
              if (lane == 0) {
                fv[i] = gelu_tanh(__fadd_rn(a, sb[bofs + i]));
                if (two) fv[i2] = gelu_tanh(__fadd_rn(b, sb[bofs + i2]));
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        csync();
        // mlp.c_proj partial over this CTA's hidden rows: outputs over threads
        have = mbar_wait(&full[q & 1], (q >> 1) & 1, status) && have;
        const float *wt = ring + (size_t)(q & 1) * (kStageBytes / 4);
        for (int o = t; o < D; o += kThreads) {
          float a = 0.0f;
          if (have) {
#pragma unroll 8
            for (int k = 0; k < nr; k++) a = fmaf(fv[k], wt[(size_t)k * D + o], a);
          }
          red_word(red_mlp + o, a, status);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        if (trace) tr[p * kTraceSlots + 4] = gtimer();
      }
    }

    // ===== ln_f + lm_head rows, argmax
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    {
      const int p = 3 * nl;
      if (trace) tr[p * kTraceSlots + 0] = gtimer();
      float2 sv[kPairsPerThread];
      poll_reduced(red + (size_t)(2 * nl - 1) * D, D, C_mlp, status, t, sv);
      if (trace) tr[p * kTraceSlots + 1] = gtimer();
      bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
      const float *sb = ring + (size_t)(q & 1) * (kStageBytes / 4);
      if (trace) tr[p * kTraceSlots + 2] = gtimer();
      add_reduced(xres, sb + 2 * D, D, t, sv);
      csync();
      if (trace) tr[p * kTraceSlots + 3] = gtimer();
      float xr[4 * NK];
      load_x<NK>(xres, lane, xr);
      layernorm_regs<NK>(xr, sb, sb + D, lane, D, eps);
      if (trace) tr[p * kTraceSlots + 7] = gtimer();
      for (int j = 0; j < g.n_lm; j++) {
        if (j > 0) {
          have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
          sb = ring + (size_t)(q & 1) * (kStageBytes / 4);
        }
        const int r0 = g.v0 + j * g.R;
        const int cn = r0 + g.R <= g.v1 ? g.R : (g.v1 > r0 ? g.v1 - r0 : 0);
        const float *w = sb + hdr;
        if (have) {
          for (int i = warp; i < cn; i += 2 * kWarps) {
            const int i2 = i + kWarps;
            const bool two = i2 < cn;
            float a, b;
            dot2<NK>(reinterpret_cast<const float4 *>(w + (size_t)i * D),
                     reinterpret_cast<const float4 *>(w + (size_t)(two ? i2 : i) * D), two, xr, lane, a, b);
            if (lane == 0) {
              const int n = r0 + i;
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
      }
      if (trace) tr[p * kTraceSlots + 4] = gtimer();
    }

    // ---- argmax: publish this CTA's best, fold every CTA's -----------------
    // The fence before the publish releases this CTA's KV-cache rows of the
    // token (written by other warps before the barrier); the one after the
    // fold acquires every CTA's, which the next token's staging copies read.
    if (lane == 0) {
      rbv[warp] = best;
      rbi[warp] = bidx;
    }
    csync();
    if (warp == 0) {
      const uint32_t tag_am = tag_tok + (uint32_t)nl;
      float bv = lane < kWarps ? rbv[lane] : -INFINITY;
      int bi = lane < kWarps ? rbi[lane] : 0x7fffffff;
      warp_best(bv, bi);
      if (lane == 0) {
        fence_gpu();
        st_word_rep(m.part_w + 2 * blockIdx.x, kPartWords, __float_as_uint(bv), tag_am);
        st_word_rep(m.part_w + 2 * blockIdx.x + 1, kPartWords, (uint32_t)bi, tag_am);
      }
      bv = -INFINITY;
      bi = 0x7fffffff;
      for (int b = lane; b < g.G; b += 32) {
        float pw[2];
        wait_words<2>(m.part_w + (size_t)(blockIdx.x % kReplicas) * kPartWords + 2 * b, 1, 2, tag_am, status, pw);
        const int ib = (int)__float_as_uint(pw[1]);
        if (better(pw[0], ib, bv, bi)) { bv = pw[0]; bi = ib; }
      }
      warp_best(bv, bi);
      fence_gpu();
      if (lane == 0) tok_s[0] = bi == 0x7fffffff ? 0 : bi;
    }
    // the next token's layer-0 prefix: rows [0, pos] (row pos written this token)
    const bool next = tk + 1 < ln.n_tokens;
    const int nrows = next ? staged(ln.pos_ok ? pos + 1 : 0) : 0;
    if (next && t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * nrows * hd * 4));
    csync();
    tok = tok_s[0];
    if (next) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      issue_prefix(0, nrows);
      pending = true;
    }
  }
  // every issued copy has landed before the CTA exits
  if (pending) mbar_wait(pfx, (uint32_t)(pf & 1), status, false);

  if (blockIdx.x == 0 && t == 0) {
    if (*(volatile uint32_t *)status == 0) {
      m.io[1] = tok;
      if (m.bump) m.io[0] = ln.pos0 + ln.n_tokens;
    }
    m.sync[3] += 1u;   // next launch: new tags
    m.sync[4] = ln.tok0 + (uint32_t)ln.n_tokens;
  }
}

// Producer warp: every weight transfer of the launch, in order, into the
// stage its consumers released, plus L2 prefetches ahead.
__device__ __noinline__ void producer_role(const Sm100DecodeModel &m, const Launch &ln, const Geo &g,
                                           unsigned char *smem) {
  if ((threadIdx.x & 31) != 0) return;
  float *ring = reinterpret_cast<float *>(smem + Smem::ring);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars), *empty = full + 2;
  const int nx = g.nx, total = nx * ln.n_tokens, nl = m.n_layers, D = m.dim;
  uint64_t *tr = m.trace ? m.trace + (size_t)blockIdx.x * (3 * nl + 1) * kTraceSlots : nullptr;
  const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
  int issued = 0, ia = 0;
  for (int qq = 0; qq < total; qq++) {
    const int s = qq & 1, qi = qq % nx;
    // the step a transfer feeds (lm_head: its first chunk), traced on the last token
    const int tp = qi < 4 * nl ? 3 * (qi >> 2) + ((qi & 3) == 0 ? 0 : (qi & 3) == 1 ? 1 : 2) : (qi == 4 * nl ? 3 * nl : -1);
    const bool trace = tr && qq >= total - nx && tp >= 0 && (qi >= 4 * nl || (qi & 3) != 3);
    if (trace) tr[tp * kTraceSlots + 6] = gtimer();
    if (qq >= 2 && !mbar_wait(&empty[s], ((qq >> 1) - 1) & 1, ln.status)) break;
    issue(xfer_of(m, g, qi), D, ring + (size_t)s * (kStageBytes / 4), &full[s], pol_stream, pol_keep);
    if (trace) tr[tp * kTraceSlots + 5] = gtimer();
    issued = qq + 1;
    for (; ia < qq + 2 + kPrefetchAhead && ia < total; ia++) {
      if (ia < 2) continue;
      const Xfer x = xfer_of(m, g, ia % nx);
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
  const int nl = m.n_layers, D = m.dim;
  const Geo g = geo_of(c, (int)gridDim.x, m.heads, D, m.head_dim, m.vocab, nl);
  Launch ln;
  ln.n_tokens = n_tokens;
  ln.status = m.sync + 2;
  // tags: (launch epoch mod 65535 + 1) << 16 | token * stride + step: never
  // 0 (the zero-initialised words), distinct from the previous launch's and
  // within a launch one per (token, step)
  const uint32_t epoch = m.sync[3];
  ln.tag_base = ((epoch % 65535u) + 1u) << 16;
  ln.stride = (uint32_t)(nl + 2);
  ln.tok0 = m.sync[4];
  ln.pos0 = m.io[0];
  // a position range outside the cache is an argument error: flag it and keep
  // every access in bounds (positions from 0, no cache write, nothing published)
  ln.pos_ok = ln.pos0 >= 0 && ln.pos0 + n_tokens <= m.max_ctx;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  float **kcs = reinterpret_cast<float **>(smem + Smem::kcs);
  for (int l = t; l < nl; l += kBlockThreads) kcs[l] = m.kv_cache[l];
  if (t == 0) {
    if (!ln.pos_ok && c == 0) atomicOr(ln.status, SM100_DECODE_ERR_ARG);
    mbar_init(&bars[0], 1);        // full[0], full[1]: armed by the producer
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], kWarps);   // empty[0], empty[1]: one arrival per consumer warp
    mbar_init(&bars[3], kWarps);
    mbar_init(&bars[4], 1);        // attention prefix
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (t >= kThreads) {
    producer_role(m, ln, g, smem);
    return;
  }
  consumer_role<NK>(m, ln, g, smem);
}

}  // namespace sm100

using namespace sm100;

static int g_num_sms[64];

extern "C" uint64_t sm100_decode_sync_bytes(void) { return (uint64_t)(4 + 2 * 1024) * 4; }

extern "C" uint64_t sm100_decode_part_bytes(void) { return (uint64_t)kPartWords * 8 * kReplicas; }

extern "C" uint64_t sm100_decode_trace_bytes(int32_t n_layers) {
  return (uint64_t)1024 * (3 * (uint64_t)(n_layers > 0 ? n_layers : 0) + 1) * kTraceSlots * 8;
}

extern "C" uint64_t sm100_decode_red_bytes(int32_t n_layers, int32_t dim) {
  return (uint64_t)3 * 2 * (uint64_t)(n_layers > 0 ? n_layers : 0) * (uint64_t)(dim > 0 ? dim : 0) * 8;
}

// One-time regrouping of the split projections (plain copies; the reads of
// the transpose are strided, it runs once per model load).
__global__ void regroup_kernel(const float *__restrict__ w_o, const float *__restrict__ w_p2, float *__restrict__ w_o_h,
                               float *__restrict__ w_p2_t, int D, int hd, int F) {
  const int64_t n_o = (int64_t)D * D, n_p = (int64_t)F * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_o + n_p; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n_o) {
      const int64_t h = i / ((int64_t)D * hd), o = (i / hd) % D, d = i % hd;
      w_o_h[i] = w_o[o * D + h * hd + d];
    } else {
      const int64_t j = i - n_o, k = j / D, o = j % D;
      w_p2_t[j] = w_p2[o * F + k];
    }
  }
}

extern "C" int sm100_decode_regroup(const float *w_o, const float *w_p2, float *w_o_h, float *w_p2_t, int32_t dim,
                                    int32_t heads, int32_t hidden, void *stream) {
  if (!w_o || !w_p2 || !w_o_h || !w_p2_t || dim <= 0 || heads <= 0 || dim % heads || hidden <= 0)
    return sm100_set_error(SM100_ERR_ARG, "decode_regroup: bad arguments (dim %d, heads %d, hidden %d)", dim, heads,
                           hidden);
  regroup_kernel<<<592, 256, 0, (cudaStream_t)stream>>>(w_o, w_p2, w_o_h, w_p2_t, dim, dim / heads, hidden);
  return launch_status("decode_regroup");
}

extern "C" int32_t sm100_decode_grid(int32_t heads, int32_t head_dim) {
  int dev = 0;
  cudaGetDevice(&dev);
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 0;
  if (heads <= 0 || head_dim <= 0) return 0;
  return members_per_head(heads, head_dim, n) * heads;
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
  const int hd = heads > 0 ? dim / heads : 0;
  const int M = heads > 0 && hd > 0 ? members_per_head(heads, hd, g_num_sms[dev]) : 0, G = M * heads;
  bool ok = dev_model && M >= 3 && n_tokens > 0 && (int64_t)n_tokens * (n_layers + 2) < 65536 && n_layers > 0 &&
            n_layers <= kMaxLayers && dim > 0 && dim % 128 == 0 && dim <= kMaxDim && hd * heads == dim &&
            (hd == 32 || hd == 64) && vocab > 0 && max_ctx > 0 && Smem::smax(max_ctx, hd) >= 1;
  if (ok) {
    // every CTA's transfers within one stage; row slices within the row slots
    const Geo g0 = geo_of(0, G, heads, dim, hd, vocab, n_layers);
    const int64_t D = dim, frow = (4 * D + G - 1) / G, orow = (D + M - 1) / M;
    const int64_t hdr = hdr_floats(dim);
    ok = g0.qn <= kMaxRows && g0.qn + 6 <= kBiasFloats && (hdr + g0.qn * D) * 4 <= kStageBytes &&
         orow * hd * 4 <= kStageBytes && frow <= kMaxRows && frow <= 64 && frow + 6 <= kBiasFloats &&
         (hdr + frow * D) * 4 <= kStageBytes && g0.R >= 1 && Smem::total(max_ctx, hd) <= (size_t)kSmemLimit;
  }
  if (!ok)
    return sm100_set_error(SM100_ERR_ARG,
                           "decode: unsupported shape (tokens %d, layers %d, dim %d, heads %d, vocab %d, ctx %d, %d SMs)",
                           n_tokens, n_layers, dim, heads, vocab, max_ctx, g_num_sms[dev]);
  const size_t smem = Smem::total(max_ctx, hd);
  switch (dim / 128) {
    case 4: return launch_decode<4>(dev_model, n_tokens, G, smem, (cudaStream_t)stream);
    case 6: return launch_decode<6>(dev_model, n_tokens, G, smem, (cudaStream_t)stream);
    default:
      return sm100_set_error(SM100_ERR_ARG, "decode: dim %d not built (512 or 768)", dim);
  }
}

extern "C" int sm100_decode_step(const Sm100DecodeModel *dev_model, int32_t n_layers, int32_t dim, int32_t heads,
                                 int32_t vocab, int32_t max_ctx, void *stream) {
  return sm100_decode_steps(dev_model, 1, n_layers, dim, heads, vocab, max_ctx, stream);
}
