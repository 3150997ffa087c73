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
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kWarps = 15;                   // consumer warps (16 warps in all: 128 registers)
constexpr int kThreads = kWarps * 32;        // consumer threads
constexpr int kBlockThreads = kThreads + 32; // + one producer warp (TMA issue)
constexpr int kStages = 2;                   // weight ring stages
constexpr int kStageBytes = 76 * 1024;       // one stage
constexpr int kMaxDim = 1024;                // residual stream held in shared memory
constexpr int kMaxRows = 32;                 // rows of one c_attn / c_fc slice or lm_head chunk (a lane each)
constexpr int kMaxHd = 64;
constexpr int kPrefetchAhead = 4;            // L2 prefetch distance in transfers
constexpr int kMaxLayers = SM100_DECODE_MAX_LAYERS;
constexpr int kBiasFloats = 64;              // stage region of a transfer's bias slice
constexpr int kSmemLimit = 227 * 1024;
constexpr int kTraceSlots = 8;               // u64 timestamps per (CTA, step) in the optional trace
constexpr size_t kPartWords = 2 * 1024;      // argmax partials of one copy: (value, index) per CTA
constexpr int kFixShift = 28;                // reduction words: fixed point with 28 fraction bits
constexpr float kFixLimit = 2048.0f;         // |contribution| bound (sums stay below 2^47 / 2^28)
constexpr int kBoxRows = 32;                 // KV staging: rows of one tensor-map box
constexpr int kCpRows = 5;                   // c_proj rows per warp (a member has <= kCpRows kWarps)
static_assert(kCpRows == 5, "cproj_step selects among five rows");

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

// One pair of tagged words (p[0], p[1]) with a 16-byte load per poll
// (bounded); the re-poll loop is out of line (the hot path is one load).
__device__ __noinline__ float2 wait_pair_slow(const uint64_t *p, uint32_t tag, uint32_t *status) {
  uint64_t a, b;
  for (uint32_t it = 0; it < (1u << 22); it++) {
    if ((it & 15u) == 15u && *(volatile uint32_t *)status) return make_float2(0.0f, 0.0f);
    ld_pair(p, a, b);
    if ((uint32_t)(a >> 32) == tag && (uint32_t)(b >> 32) == tag)
      return make_float2(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b));
  }
  atomicOr(status, SM100_DECODE_ERR_BARRIER);
  return make_float2(0.0f, 0.0f);
}

__device__ __forceinline__ float2 wait_pair(const uint64_t *p, uint32_t tag, uint32_t *status) {
  uint64_t a, b;
  ld_pair(p, a, b);
  if ((uint32_t)(a >> 32) == tag && (uint32_t)(b >> 32) == tag)
    return make_float2(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b));
  return wait_pair_slow(p, tag, status);
}

// ---- reduction words -------------------------------------------------------
// A contribution v adds (1 << 48) + round(v * 2^28) (two's complement, mod
// 2^64).  After C contributions (count taken mod 2^16) the word minus C << 48
// is the exact fixed-point sum, |sum| < 2^47; with k < 2^15 contributions
// still missing it lies at least 2^47 away from that range.
__device__ __noinline__ void flag_range(uint32_t *status) { atomicOr(status, SM100_DECODE_ERR_RANGE); }

__device__ __forceinline__ void red_word(uint64_t *p, float v, uint32_t *status) {
  if (!(fabsf(v) <= kFixLimit)) {   // also NaN: flagged, counted as 0
    flag_range(status);
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

// The pair of reduction words (p[0], p[1]) once both counts reach C
// (bounded; the re-poll loop out of line).
__device__ __noinline__ float2 wait_red_pair_slow(const uint64_t *p, uint64_t C, uint32_t *status) {
  uint64_t a, b;
  for (uint32_t it = 0; it < (1u << 22); it++) {
    if ((it & 15u) == 15u && *(volatile uint32_t *)status) return make_float2(0.0f, 0.0f);
    ld_pair(p, a, b);
    if (red_done(a, C) && red_done(b, C)) return make_float2(red_value(a, C), red_value(b, C));
  }
  atomicOr(status, SM100_DECODE_ERR_BARRIER);
  return make_float2(0.0f, 0.0f);
}

__device__ __forceinline__ float2 wait_red_pair(const uint64_t *p, uint64_t C, uint32_t *status) {
  uint64_t a, b;
  ld_pair(p, a, b);
  if (red_done(a, C) && red_done(b, C)) return make_float2(red_value(a, C), red_value(b, C));
  return wait_red_pair_slow(p, C, status);
}

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// 2-D tensor copy (no multicast) of the box at (x, y) of a tensor map in
// global memory into shared memory, completing on bar.
__device__ __forceinline__ void tma_2d(void *dst, const void *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
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
  int z0, z1;          // this CTA's share of a reduction set to zero (words)
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
  rows_of((int64_t)2 * n_layers * D, c, G, a, b);
  g.z0 = (int)a; g.z1 = (int)b;
  return g;
}

// One weight transfer: [kind of step, layer] or an lm_head chunk.
struct Xfer {
  const float *w, *ln_g, *ln_b, *bx, *b;
  uint32_t wbytes, bbytes;
  int hdr;     // floats before the weight rows
  int pad;
};

// Transfers per token of any CTA (the table in shared memory holds them).
__host__ __device__ __forceinline__ int max_transfers(int n_layers, int vocab, int G, int D) {
  const int R = lm_rows_per_chunk(D), rows = (vocab + G - 1) / G;
  const int n_lm = R > 0 ? (rows + R - 1) / R : 1;
  return 4 * n_layers + (n_lm > 0 ? n_lm : 1);
}

__device__ __forceinline__ Xfer xfer_of(const Sm100DecodeModel &m, const Geo &g, int i) {
  const int D = m.dim, hd = m.head_dim, nl = m.n_layers;
  Xfer x;
  x.ln_g = x.ln_b = x.bx = x.b = nullptr;
  x.bbytes = 0;
  x.pad = 0;
  int r = 0, nr = 0;
  const float *bias = nullptr;
  if (i < 4 * nl) {
    const int l = i >> 2;
    switch (i & 3) {
      case 0:   // c_attn rows; header: ln_1, mlp.c_proj bias of layer l - 1
        r = g.qrow0; nr = g.qn;
        x.w = m.w_qkv_bt[l] + (size_t)r * D;
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
        x.w = m.w_fc_bt[l] + (size_t)r * D;
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
    x.w = m.lm_head_bt + (size_t)r * D;
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
  static constexpr size_t xs = ring + (size_t)kStages * kStageBytes;    // [kMaxDim] LayerNorm output
  static constexpr size_t lnp = xs + kMaxDim * 4;                         // [2][16] LayerNorm partial sums
  static constexpr size_t fv = lnp + 32 * 4;                              // [kMaxRows] c_fc outputs
  static constexpr size_t rp = fv + kMaxRows * 4;                         // [2][2 kWarps][32] row partial sums
  static constexpr size_t lmb = rp + 2 * 2 * kWarps * 32 * 4;             // [kMaxRows] f32 + [kMaxRows] i32: row bests
  static constexpr size_t qkvs = lmb + 2 * kMaxRows * 4;                  // [3 kMaxHd] q, k, v of the head
  static constexpr size_t atts = qkvs + 3 * kMaxHd * 4;                   // [kMaxHd] attention output
  static constexpr size_t acc = atts + kMaxHd * 4;                        // [kThreads] p @ v slices
  static constexpr size_t tok = acc + kThreads * 4;                       // [4] i32
  static constexpr size_t bars = tok + 16;                                // full[2], empty[2], pfx
  static constexpr size_t kcs = bars + 8 * 8;                             // [kMaxLayers] cache pointers
  static constexpr size_t cps = kcs + kMaxLayers * 8;                     // [kCpRows kWarps] c_proj partials
  static constexpr size_t xt = cps + kCpRows * kWarps * 4 + 4;            // [nxt] transfer table (Xfer)
  static __host__ __device__ size_t sc(int nxt) { return xt + (size_t)nxt * sizeof(Xfer); }   // [2][max_ctx]
  static __host__ __device__ size_t kv(int nxt, int max_ctx) {
    return (sc(nxt) + 2 * (size_t)max_ctx * 4 + 127) & ~(size_t)127;
  }
  // staged positions: whole boxes (a box may run past max_ctx: V rows, or
  // the fill value past 2 max_ctx)
  static __host__ __device__ int smax(int nxt, int max_ctx, int hd) {
    int64_t n = ((int64_t)kSmemLimit - (int64_t)kv(nxt, max_ctx)) / (8 * hd);
    n = n / kBoxRows * kBoxRows;
    return (int)(n > 0 ? n : 0);
  }
  static __host__ __device__ size_t total(int nxt, int max_ctx, int hd) {
    return kv(nxt, max_ctx) + (size_t)smax(nxt, max_ctx, hd) * 8 * hd;
  }
};

struct Launch {
  int n_tokens, pos0;
  bool pos_ok;
  uint32_t tag_base, stride;   // tag of (token tk, step p): tag_base + tk * stride + p
  uint32_t *status;
  uint32_t tok0;               // tokens decoded by earlier launches (selects the reduction sets)
};

// The per-layer path of the consumer warps is a handful of out-of-line
// functions (one rows loop for c_attn, c_fc and lm_head, one LayerNorm, the
// attention, the two split products): the kernel's code is executed once per
// layer, so the path must stay small enough for the SM's instruction caches.
//
// Thread t < D / 2 owns the residual stream's pair (x[2 t], x[2 t + 1]) in
// registers (D <= 2 kThreads): it adds the decoded sums to it and feeds it to
// the LayerNorm, so the residual stream never needs a barrier.

// The step input: x += (decoded sum of the reduction set `words` (count C)
// + bias bx), the reference's order (the projection's bias, then the
// residual; words == nullptr: x unchanged), then LayerNorm (two-pass
// statistics, one partial sum per warp and a fixed-order fold) of x with
// gamma / beta into xs.  The consumer warps meet three times.  Returns x.
__device__ __noinline__ float2 input_ln(unsigned char *smem, const uint64_t *words, uint64_t C, const float *bx,
                                        const float *gam, const float *bet, float2 xv, int D, float eps,
                                        uint32_t *status) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float *xs = reinterpret_cast<float *>(smem + Smem::xs);
  float *lnp = reinterpret_cast<float *>(smem + Smem::lnp);
  const bool live = 2 * t < D;
  if (words && live) {
    const float2 sv = wait_red_pair(words + 2 * t, C, status);
    const float2 bb = reinterpret_cast<const float2 *>(bx)[t];
    xv = make_float2(__fadd_rn(xv.x, __fadd_rn(sv.x, bb.x)), __fadd_rn(xv.y, __fadd_rn(sv.y, bb.y)));
  }
  const float inv_n = (float)(1.0 / (double)D);
  const float s = warp_sum(live ? __fadd_rn(xv.x, xv.y) : 0.0f);
  if (lane == 0) lnp[warp] = s;
  csync();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; w++) tot += lnp[w];
  const float mean = __fmul_rn(tot, inv_n);
  const float d0 = __fsub_rn(xv.x, mean), d1 = __fsub_rn(xv.y, mean);
  const float v = warp_sum(live ? fmaf(d1, d1, __fmul_rn(d0, d0)) : 0.0f);
  if (lane == 0) lnp[16 + warp] = v;
  csync();
  float vt = 0.0f;
#pragma unroll
  for (int w = 0; w < kWarps; w++) vt += lnp[16 + w];
  const float rr = __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(vt, inv_n), eps)));
  if (live) {
    const float2 gg = reinterpret_cast<const float2 *>(gam)[t], bb = reinterpret_cast<const float2 *>(bet)[t];
    reinterpret_cast<float2 *>(xs)[t] = make_float2(__fadd_rn(__fmul_rn(__fmul_rn(d0, rr), gg.x), bb.x),
                                                    __fadd_rn(__fmul_rn(__fmul_rn(d1, rr), gg.y), bb.y));
  }
  csync();
  return xv;
}

enum { ROWS_QKV = 0, ROWS_FC, ROWS_LM };

// Rows [0, nr) (nr <= 32) of a block-transposed slice wt ([D / 4][nr][4]:
// element (i, k) at ((k / 4) nr + i) 4 + k % 4, sm100_decode_block_transpose)
// dotted with the LayerNorm output.  Lane i of a lane group (16 or 32 lanes)
// takes row i over a K slice (the CTA's K range split over warps and groups:
// the weights are read from shared memory once, the input as broadcasts);
// thread i folds the slices' partial sums in a fixed order and finishes row i:
//  ROWS_QKV: y = dot + bias[i] published to dst[i] (tag) and, for k / v
//            rows, written to the KV cache row (cache[i]);
//  ROWS_FC:  fv[i] = GELU(dot + bias[i]);
//  ROWS_LM:  logits[r0 + i] = dot (when logits), the row's running best
//            (value, index) kept in lmb / lmi.
// par alternates between consecutive calls (two partial-sum buffers).
__device__ __noinline__ void rows_step(unsigned char *smem, const float *wt, const float *bias, int nr, int D, int kind,
                                       uint64_t *dst, uint32_t tag, float *cache, float *logits, int r0, int par) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const float4 *x4 = reinterpret_cast<const float4 *>(smem + Smem::xs);
  const float4 *w4 = reinterpret_cast<const float4 *>(wt);
  float *rp = reinterpret_cast<float *>(smem + Smem::rp) + par * (2 * kWarps * 32);
  const int RP = nr > 16 ? 32 : 16, parts = 32 / RP, np = kWarps * parts;
  const int row = lane & (RP - 1), part = warp * parts + lane / RP, NG = D / 4;
  const int g0 = NG * part / np, g1 = NG * (part + 1) / np;
  float a0 = 0.0f, a1 = 0.0f;
  if (row < nr) {
#pragma unroll 4
    for (int gq = g0; gq < g1; gq++) {
      const float4 wv = w4[(size_t)gq * nr + row], xv = x4[gq];
      a0 = fmaf(wv.x, xv.x, a0);
      a1 = fmaf(wv.y, xv.y, a1);
      a0 = fmaf(wv.z, xv.z, a0);
      a1 = fmaf(wv.w, xv.w, a1);
    }
  }
  rp[part * 32 + row] = __fadd_rn(a0, a1);
  csync();
  if (t < nr) {
    // every partial loaded before the fixed-order fold (np <= 2 kWarps)
    float pv[2 * kWarps];
#pragma unroll
    for (int q = 0; q < 2 * kWarps; q++) pv[q] = q < np ? rp[q * 32 + t] : 0.0f;
    float d = 0.0f;
#pragma unroll
    for (int q = 0; q < 2 * kWarps; q++) d += pv[q];
    if (kind == ROWS_QKV) {
      const float y = __fadd_rn(d, bias[t]);
      st_word(dst + t, __float_as_uint(y), tag);
      if (cache) cache[t] = y;
    } else if (kind == ROWS_FC) {
      reinterpret_cast<float *>(smem + Smem::fv)[t] = gelu_tanh(__fadd_rn(d, bias[t]));
    } else {
      float *lmb = reinterpret_cast<float *>(smem + Smem::lmb);
      int *lmi = reinterpret_cast<int *>(lmb + kMaxRows);
      const int n = r0 + t;
      if (logits) logits[n] = d;
      if (better(d, n, lmb[t], lmi[t])) {
        lmb[t] = d;
        lmi[t] = n;
      }
    }
  }
}

// Attention of head h for the new row at pos (thvm_gpt2.py:49-61): q, k, v
// from the group's tagged words (k, v also staged at pos), scores against the
// staged keys Ks (positions < smax; later ones from the cache in L2),
// softmax, p @ v into atts.  Then the next layer's prefix copies (map_next,
// rows [0, next_rows); map_next == nullptr: none).  The loops stay rolled:
// this runs once per layer and must stay small for the instruction caches.
__device__ __noinline__ void attention_step(unsigned char *smem, float *sc, float *Ks, const uint64_t *qkv_src,
                                            uint32_t tag, const float *kc, int pos, int smax, int hd, int D,
                                            int max_ctx, int h, float scale, const void *map_next, int next_rows,
                                            uint32_t *status) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, L = pos + 1;
  float *qs = reinterpret_cast<float *>(smem + Smem::qkvs), *kn = qs + hd, *vn = kn + hd;
  float *atts = reinterpret_cast<float *>(smem + Smem::atts);
  float *acc = reinterpret_cast<float *>(smem + Smem::acc);
  float *pr = sc + max_ctx, *Vs = Ks + (size_t)smax * hd;
  uint64_t *pfx = reinterpret_cast<uint64_t *>(smem + Smem::bars) + 4;
  const float *vc = kc + (size_t)max_ctx * D;
  if (2 * t < 3 * hd) {
    const float2 v = wait_pair(qkv_src + 2 * t, tag, status);
    reinterpret_cast<float2 *>(qs)[t] = v;
    const int i = 2 * t, which = i / hd, dd = i % hd;
    if (which > 0 && pos < smax) *reinterpret_cast<float2 *>((which == 1 ? Ks : Vs) + (size_t)pos * hd + dd) = v;
  }
  csync();
  // scores: 8 lanes per key, hd / 8 floats per lane (two float4 at hd = 64)
  {
    const int grp = t >> 3, gl = t & 7, per4 = hd / 32;
    const float4 qa = reinterpret_cast<const float4 *>(qs)[gl * per4];
    const float4 qb = per4 > 1 ? reinterpret_cast<const float4 *>(qs)[gl * per4 + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int j0 = 0; j0 < L; j0 += kThreads / 8) {
      const int j = j0 + grp;
      float s = 0.0f;
      if (j < L) {
        const float4 *kr = j < smax ? reinterpret_cast<const float4 *>(Ks + (size_t)j * hd) + gl * per4
                         : j == pos ? reinterpret_cast<const float4 *>(kn) + gl * per4
                                    : reinterpret_cast<const float4 *>(kc + (size_t)j * D + (size_t)h * hd) + gl * per4;
        const float4 ka = j < smax || j == pos ? kr[0] : __ldcg(kr);
        s = fmaf(qa.x, ka.x, fmaf(qa.y, ka.y, fmaf(qa.z, ka.z, __fmul_rn(qa.w, ka.w))));
        if (per4 > 1) {
          const float4 kb = j < smax || j == pos ? kr[1] : __ldcg(kr + 1);
          s = fmaf(qb.x, kb.x, fmaf(qb.y, kb.y, fmaf(qb.z, kb.z, fmaf(qb.w, kb.w, s))));
        }
      }
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      if (j < L && gl == 0) sc[j] = __fmul_rn(s, scale);
    }
  }
  csync();
  // softmax by warp 0: p_j = exp(s_j - max) * recip(sum)
  if (warp == 0) {
    float mx = -INFINITY;
#pragma unroll 1
    for (int j = lane; j < L; j += 32) mx = fmaxf(mx, sc[j]);
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll 1
    for (int j = lane; j < L; j += 32) {
      const float e = xexp(__fsub_rn(sc[j], mx));
      pr[j] = e;
      sum += e;
    }
    const float r = __frcp_rn(warp_sum(sum));
#pragma unroll 1
    for (int j = lane; j < L; j += 32) pr[j] = __fmul_rn(pr[j], r);
  }
  csync();
  // p @ v: key slices x dims, then the slices in order
  const int nslice = kThreads / hd;
  {
    const int slice = t / hd, d = t % hd;
    if (slice < nslice) {
      float a = 0.0f;
#pragma unroll 1
      for (int j = slice; j < L; j += nslice) {
        const float v = j < smax ? Vs[(size_t)j * hd + d] : j == pos ? vn[d] : __ldcg(vc + (size_t)j * D + (size_t)h * hd + d);
        a = fmaf(pr[j], v, a);
      }
      acc[slice * hd + d] = a;
    }
  }
  const int nb = map_next ? (next_rows + kBoxRows - 1) / kBoxRows : 0;
  if (nb && t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * nb * kBoxRows * hd * 4));
  csync();
  if (t < hd) {
    float a = 0.0f;
#pragma unroll 1
    for (int s2 = 0; s2 < nslice; s2++) a += acc[s2 * hd + t];
    atts[t] = a;
  }
  if (t < 2 * nb) {   // keys then values, whole boxes of the next layer's map
    const int v = t >= nb, b = v ? t - nb : t;
    tma_2d((v ? Vs : Ks) + (size_t)b * kBoxRows * hd, map_next, h * hd, (v ? max_ctx : 0) + b * kBoxRows, pfx);
  }
  csync();
}

// c_proj partial: rows [0, nr) of the head's column block (w: nr x hd) times
// the attention output, added to the reduction words out[0, nr); warp w takes
// rows w, w + kWarps, ..., lanes over the dims.
__device__ __noinline__ void cproj_step(unsigned char *smem, const float *w, int nr, int hd, uint64_t *out,
                                        uint32_t *status) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const float *atts = reinterpret_cast<const float *>(smem + Smem::atts);
  const float a0 = atts[lane], a1 = hd > 32 ? atts[lane + 32] : 0.0f;
  float s[kCpRows];
#pragma unroll
  for (int r = 0; r < kCpRows; r++) {
    const int i = warp + kWarps * r;
    s[r] = 0.0f;
    if (i < nr) {
      s[r] = __fmul_rn(w[(size_t)i * hd + lane], a0);
      if (hd > 32) s[r] = fmaf(w[(size_t)i * hd + lane + 32], a1, s[r]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < kCpRows; r++) s[r] += __shfl_xor_sync(0xffffffffu, s[r], o);
  // lane r adds row warp + r kWarps
  const float v = lane == 0 ? s[0] : lane == 1 ? s[1] : lane == 2 ? s[2] : lane == 3 ? s[3] : s[4];
  const int i = warp + kWarps * lane;
  if (lane < kCpRows && i < nr) red_word(out + i, v, status);
}

// mlp.c_proj partial over this CTA's hidden rows: out[o] += sum_k fv[k]
// wt[k][o] (wt: nr x D, the transposed weight's rows); thread t takes the
// outputs 2 t, 2 t + 1 (D <= 2 kThreads).
__device__ __noinline__ void mproj_step(unsigned char *smem, const float *wt, int nr, int D, uint64_t *out,
                                        uint32_t *status) {
  const int t = threadIdx.x;
  const float *fv = reinterpret_cast<const float *>(smem + Smem::fv);
  if (2 * t < D) {
    float a = 0.0f, b = 0.0f;
#pragma unroll 4
    for (int k = 0; k < nr; k++) {
      const float2 w2 = reinterpret_cast<const float2 *>(wt + (size_t)k * D)[t];
      const float f = fv[k];
      a = fmaf(f, w2.x, a);
      b = fmaf(f, w2.y, b);
    }
    // lane l adds words 64 w + l and 64 w + 32 + l (warp w = t / 32): each
    // red instruction covers 32 consecutive words, so the L2 atomic units see
    // whole lines (lane l's words belong to lanes l / 2 and 16 + l / 2)
    const int lane = t & 31, w0 = 64 * (t >> 5);
    const float pa = __shfl_sync(0xffffffffu, a, lane >> 1), pb = __shfl_sync(0xffffffffu, b, lane >> 1);
    const float qa = __shfl_sync(0xffffffffu, a, 16 + (lane >> 1)), qb = __shfl_sync(0xffffffffu, b, 16 + (lane >> 1));
    if (w0 + lane < D) red_word(out + w0 + lane, (lane & 1) ? pb : pa, status);
    if (w0 + 32 + lane < D) red_word(out + w0 + 32 + lane, (lane & 1) ? qb : qa, status);
  }
}

// Argmax over the grid: each CTA publishes its best (value, index) as tagged
// words (kReplicas copies) and folds every CTA's (first index of the max).
// The fence before the publish releases this CTA's KV-cache rows of the token
// (written by other warps before the barrier) and its zeroed reduction words;
// the fence after the fold acquires every CTA's.  Returns the token.
__device__ __noinline__ int argmax_step(unsigned char *smem, uint64_t *part_w, uint32_t tag, int G, uint32_t *status) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  int *tok_s = reinterpret_cast<int *>(smem + Smem::tok);
  csync();
  if (warp == 0) {
    const float *lmb = reinterpret_cast<const float *>(smem + Smem::lmb);
    const int *lmi = reinterpret_cast<const int *>(lmb + kMaxRows);
    float bv = lmb[lane];
    int bi = lmi[lane];
    warp_best(bv, bi);
    if (lane < kReplicas) {   // one copy per lane
      fence_gpu();
      st_word(part_w + (size_t)lane * kPartWords + 2 * blockIdx.x, __float_as_uint(bv), tag);
      st_word(part_w + (size_t)lane * kPartWords + 2 * blockIdx.x + 1, (uint32_t)bi, tag);
    }
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int b = lane; b < G; b += 32) {
      float pw[2];
      wait_words<2>(part_w + (size_t)(blockIdx.x % kReplicas) * kPartWords + 2 * b, 1, 2, tag, status, pw);
      const int ib = (int)__float_as_uint(pw[1]);
      if (better(pw[0], ib, bv, bi)) { bv = pw[0]; bi = ib; }
    }
    warp_best(bv, bi);
    fence_gpu();
    if (lane == 0) tok_s[0] = bi == 0x7fffffff ? 0 : bi;
  }
  csync();
  return tok_s[0];
}

// ---------------------------------------------------------------------------
// Consumer warps of every CTA: the steps of every token.
__device__ __forceinline__ void consumer_role(const Sm100DecodeModel &m, const Launch &ln, const Geo &g,
                                              unsigned char *smem) {
  const int t = threadIdx.x, lane = t & 31;
  const int D = m.dim, hd = m.head_dim, nl = m.n_layers, max_ctx = m.max_ctx, H = m.heads;
  float *ring = reinterpret_cast<float *>(smem + Smem::ring);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars), *empty = full + 2, *pfx = full + 4;
  float *const *kcs = reinterpret_cast<float *const *>(smem + Smem::kcs);
  const int nxt = max_transfers(nl, m.vocab, g.G, D);
  const int smax = Smem::smax(nxt, max_ctx, hd);
  float *sc = reinterpret_cast<float *>(smem + Smem::sc(nxt));
  float *Ks = reinterpret_cast<float *>(smem + Smem::kv(nxt, max_ctx));
  uint32_t *status = ln.status;
  const float eps = m.eps;
  uint64_t *tr0 = m.trace ? m.trace + (size_t)blockIdx.x * (3 * nl + 1) * kTraceSlots : nullptr;
  uint64_t *qkv_w = m.qkv_w + (size_t)g.h * 3 * hd;
  const int hdr = hdr_floats(D);
  const size_t n_red = (size_t)2 * nl * D;
  auto staged = [&](int n) { return n < smax ? n : smax; };
  auto stage = [&](int qq) { return ring + (size_t)(qq & 1) * (kStageBytes / 4); };

  int q = 0;            // next ring transfer (stage q & 1, phase (q >> 1) & 1)
  int pf = 0;           // prefix phases consumed
  bool pending = true;  // a prefix phase is armed and not yet waited for
  {
    const int n = staged(ln.pos_ok ? ln.pos0 : 0), nb = (n + kBoxRows - 1) / kBoxRows;
    if (t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * nb * kBoxRows * hd * 4));
    csync();
    if (t < 2 * nb) {
      const int v = t >= nb, b = v ? t - nb : t;
      tma_2d(Ks + (v ? (size_t)smax * hd : 0) + (size_t)b * kBoxRows * hd, m.kv_map[0], g.h * hd,
             (v ? max_ctx : 0) + b * kBoxRows, pfx);
    }
  }
  int tok = m.io[1];
  for (int tk = 0; tk < ln.n_tokens; tk++) {
    const int pos = ln.pos_ok ? ln.pos0 + tk : 0;
    const uint32_t tag_tok = ln.tag_base + (uint32_t)tk * ln.stride;
    uint64_t *tr = tr0 && t == 0 && tk == ln.n_tokens - 1 ? tr0 : nullptr;
    const uint64_t C_att = (uint64_t)H, C_mlp = (uint64_t)g.G;
    // reduction words of this token: set (tok0 + tk) mod 3.  This token
    // zeroes the next token's set (last read two tokens ago: every CTA has
    // passed that token's argmax; the zeros are released by this token's
    // argmax publish, before which no CTA starts the next token)
    uint64_t *red = m.red_w + (size_t)((ln.tok0 + (uint32_t)tk) % 3u) * n_red;
    {
      uint64_t *nz = m.red_w + (size_t)((ln.tok0 + (uint32_t)tk + 1u) % 3u) * n_red;
      for (int i = g.z0 + t; i < g.z1; i += kThreads) nz[i] = 0ull;
    }
    // x = wte[tok] + wpe[pos] (thvm_gpt2.py:93-103), this thread's pair
    float2 xv = make_float2(0.0f, 0.0f);
    if (2 * t < D) {
      const float2 e = tok >= 0 && tok < m.vocab ? reinterpret_cast<const float2 *>(m.wte + (size_t)tok * D)[t]
                                                 : make_float2(0.0f, 0.0f);
      const float2 pp = reinterpret_cast<const float2 *>(m.wpe + (size_t)pos * D)[t];
      xv = make_float2(__fadd_rn(e.x, pp.x), __fadd_rn(e.y, pp.y));
    }

    for (int l = 0; l < nl; l++) {
      uint64_t *red_att = red + (size_t)(2 * l) * D, *red_mlp = red_att + D;
      // ===== c_attn rows of this member (ln_1 of x; x += mlp output of l - 1)
      {
        uint64_t *ts = tr ? tr + (3 * l) * kTraceSlots : nullptr;
        if (ts) ts[0] = gtimer();
        const bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        const float *sb = stage(q);
        if (ts) ts[2] = gtimer();
        xv = input_ln(smem, l > 0 ? red_mlp - 2 * D : nullptr, C_mlp, sb + 2 * D, sb, sb + D, xv, D, eps, status);
        if (ts) ts[3] = ts[7] = gtimer();
        float *cache = ln.pos_ok && g.kv_which > 0
                           ? kcs[l] + (size_t)(g.kv_which - 1) * max_ctx * D + (size_t)pos * D + g.qcol0
                           : nullptr;
        if (have)
          rows_step(smem, sb + hdr, sb + 3 * D + (g.qrow0 & 3), g.qn, D, ROWS_QKV, qkv_w + g.ql0,
                    tag_tok + (uint32_t)l, cache, nullptr, 0, 0);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        if (ts) ts[4] = gtimer();
      }

      // ===== attention of head h, then this member's rows of c_proj's head-h block
      {
        uint64_t *ts = tr ? tr + (3 * l + 1) * kTraceSlots : nullptr;
        if (ts) ts[0] = gtimer();
        // the prefix copies are ours and always complete: wait for them even
        // after an error, so the staging area is never written by two phases
        mbar_wait(pfx, (uint32_t)(pf & 1), status, false);
        pf++;
        pending = false;
        if (ts) ts[7] = gtimer();
        // the next layer's prefix (rows < pos, written in earlier tokens); the
        // next token's layer 0 is staged after the argmax (it needs row pos)
        const bool more = l + 1 < nl;
        attention_step(smem, sc, Ks, qkv_w, tag_tok + (uint32_t)l, kcs[l], pos, smax, hd, D, max_ctx, g.h,
                       m.attn_scale, more ? m.kv_map[l + 1] : nullptr, more ? staged(pos) : 0, status);
        pending = more;
        if (ts) ts[1] = ts[2] = ts[3] = gtimer();
        const bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        if (have)
          cproj_step(smem, stage(q), g.o1 - g.o0, hd, red_att + g.o0, status);
        else
          for (int i = t; i < g.o1 - g.o0; i += kThreads) red_word(red_att + g.o0 + i, 0.0f, status);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        if (ts) ts[4] = gtimer();
      }

      // ===== c_fc rows + GELU, then their K slice of mlp.c_proj
      {
        uint64_t *ts = tr ? tr + (3 * l + 2) * kTraceSlots : nullptr;
        if (ts) ts[0] = gtimer();
        bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
        const float *sb = stage(q);
        if (ts) ts[2] = gtimer();
        xv = input_ln(smem, red_att, C_att, sb + 2 * D, sb, sb + D, xv, D, eps, status);   // x += (att c_proj + b)
        if (ts) ts[3] = ts[7] = gtimer();
        const int nr = g.f1 - g.f0;
        if (have)
          rows_step(smem, sb + hdr, sb + 3 * D + (g.f0 & 3), nr, D, ROWS_FC, nullptr, 0u, nullptr, nullptr, 0, 1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        csync();
        have = mbar_wait(&full[q & 1], (q >> 1) & 1, status) && have;
        mproj_step(smem, stage(q), have ? nr : 0, D, red_mlp, status);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
        if (ts) ts[4] = gtimer();
      }
    }

    // ===== ln_f + lm_head rows, argmax
    {
      uint64_t *ts = tr ? tr + (3 * nl) * kTraceSlots : nullptr;
      if (ts) ts[0] = gtimer();
      bool have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
      const float *sb = stage(q);
      if (ts) ts[2] = gtimer();
      xv = input_ln(smem, red + (size_t)(2 * nl - 1) * D, C_mlp, sb + 2 * D, sb, sb + D, xv, D, eps, status);
      if (ts) ts[3] = ts[7] = gtimer();
      if (t < kMaxRows) {
        float *lmb = reinterpret_cast<float *>(smem + Smem::lmb);
        lmb[t] = -INFINITY;
        reinterpret_cast<int *>(lmb + kMaxRows)[t] = 0x7fffffff;
      }
      for (int j = 0; j < g.n_lm; j++) {
        if (j > 0) {
          have = mbar_wait(&full[q & 1], (q >> 1) & 1, status);
          sb = stage(q);
        }
        const int r0 = g.v0 + j * g.R;
        const int cn = r0 + g.R <= g.v1 ? g.R : (g.v1 > r0 ? g.v1 - r0 : 0);
        if (have) rows_step(smem, sb + hdr, nullptr, cn, D, ROWS_LM, nullptr, 0u, nullptr, m.logits, r0, j & 1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[q & 1]);
        q++;
      }
      if (ts) ts[4] = gtimer();
    }
    tok = argmax_step(smem, m.part_w, tag_tok + (uint32_t)nl, g.G, status);
    // the next token's layer-0 prefix: rows [0, pos] (row pos written this token)
    if (tk + 1 < ln.n_tokens) {
      const int nb = (staged(ln.pos_ok ? pos + 1 : 0) + kBoxRows - 1) / kBoxRows;
      if (t == 0) mbar_expect_tx(pfx, (uint32_t)(2 * nb * kBoxRows * hd * 4));
      csync();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      if (t < 2 * nb) {
        const int v = t >= nb, b = v ? t - nb : t;
          tma_2d(Ks + (v ? (size_t)smax * hd : 0) + (size_t)b * kBoxRows * hd, m.kv_map[0], g.h * hd,
               (v ? max_ctx : 0) + b * kBoxRows, pfx);
      }
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

// Producer warp: every weight transfer of the launch, in order (from the
// table built at launch), into the stage its consumers released, plus L2
// prefetches ahead.
__device__ __noinline__ void producer_role(const Sm100DecodeModel &m, const Launch &ln, const Geo &g,
                                           unsigned char *smem) {
  if ((threadIdx.x & 31) != 0) return;
  float *ring = reinterpret_cast<float *>(smem + Smem::ring);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Smem::bars), *empty = full + 2;
  const Xfer *xt = reinterpret_cast<const Xfer *>(smem + Smem::xt);
  const int nx = g.nx, total = nx * ln.n_tokens, nl = m.n_layers, D = m.dim;
  uint64_t *tr = m.trace ? m.trace + (size_t)blockIdx.x * (3 * nl + 1) * kTraceSlots : nullptr;
  const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
  int issued = 0, qi = 0, pa = 0, pai = 0;   // pa: prefetched transfers (pai: its index in the token)
  for (int qq = 0; qq < total; qq++) {
    const int s = qq & 1;
    const bool trace = tr && qq >= total - nx && (qi < 4 * nl ? (qi & 3) != 3 : qi == 4 * nl);
    const int tp = qi < 4 * nl ? 3 * (qi >> 2) + ((qi & 3) == 0 ? 0 : (qi & 3) == 1 ? 1 : 2) : 3 * nl;
    if (trace) tr[tp * kTraceSlots + 6] = gtimer();
    if (qq >= 2 && !mbar_wait(&empty[s], ((qq >> 1) - 1) & 1, ln.status)) break;
    issue(xt[qi], D, ring + (size_t)s * (kStageBytes / 4), &full[s], pol_stream, pol_keep);
    if (trace) tr[tp * kTraceSlots + 5] = gtimer();
    issued = qq + 1;
#pragma unroll 1
    for (; pa < qq + 2 + kPrefetchAhead && pa < total; pa++) {
      if (pa >= 2 && xt[pai].wbytes) bulk_prefetch_l2(xt[pai].w, xt[pai].wbytes);
      if (++pai == nx) pai = 0;
    }
    if (++qi == nx) qi = 0;
  }
  // every issued transfer has landed before the CTA exits (bounded, not cut
  // short by the status)
  for (int qq = issued - 2; qq < issued; qq++)
    if (qq >= 0) mbar_wait(&full[qq & 1], (qq >> 1) & 1, ln.status, false);
}

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
  Xfer *xt = reinterpret_cast<Xfer *>(smem + Smem::xt);
  for (int i = t; i < g.nx; i += kBlockThreads) xt[i] = xfer_of(m, g, i);
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
  consumer_role(m, ln, g, smem);
}

}  // namespace sm100

using namespace sm100;

static int g_num_sms[64];
extern "C" int32_t sm100_decode_grid(int32_t heads, int32_t head_dim);

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

// Block-transposed copies of the row-sliced weights: every slice [r, r + nr)
// a decode CTA streams (c_attn: a member's rows, c_fc: a CTA's rows,
// lm_head: a CTA's chunks) is stored at the same offset as [D / 4][nr][4]
// (element (i, k) at r D + ((k / 4) nr + i) 4 + k % 4).  One block per CTA
// of the decode grid, which it recomputes; one-time, at load.
__global__ void block_transpose_kernel(const float *__restrict__ src, float *__restrict__ dst, int kind, int D,
                                       int heads, int hd, int vocab) {
  const Geo g = geo_of(blockIdx.x, (int)gridDim.x, heads, D, hd, vocab, 1);
  const int nb = kind == 2 ? g.n_lm : 1;
  for (int j = 0; j < nb; j++) {
    int r, nr;
    if (kind == 0) { r = g.qrow0; nr = g.qn; }
    else if (kind == 1) { r = g.f0; nr = g.f1 - g.f0; }
    else { r = g.v0 + j * g.R; nr = r + g.R <= g.v1 ? g.R : (g.v1 > r ? g.v1 - r : 0); }
    const float *s0 = src + (size_t)r * D;
    float *d0 = dst + (size_t)r * D;
    for (int e = threadIdx.x; e < nr * D; e += blockDim.x) {
      const int i = e / D, k = e - i * D;
      d0[((size_t)(k >> 2) * nr + i) * 4 + (k & 3)] = s0[e];
    }
  }
}

extern "C" int sm100_decode_block_transpose(const float *src, float *dst, int32_t kind, int32_t dim, int32_t heads,
                                            int32_t vocab, void *stream) {
  const int hd = heads > 0 ? dim / heads : 0;
  const int G = heads > 0 && hd > 0 ? sm100_decode_grid(heads, hd) : 0;
  if (!src || !dst || kind < 0 || kind > 2 || G <= 0 || dim % 4 || vocab <= 0)
    return sm100_set_error(SM100_ERR_ARG, "decode_block_transpose: bad arguments (kind %d, dim %d, heads %d)", kind,
                           dim, heads);
  block_transpose_kernel<<<G, 256, 0, (cudaStream_t)stream>>>(src, dst, kind, dim, heads, hd, vocab);
  return launch_status("decode_block_transpose");
}

typedef CUresult (*DecEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

extern "C" int sm100_decode_prepare(Sm100DecodeModel *desc) {
  static DecEncodeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return sm100_set_error(SM100_ERR_CUDA, "decode_prepare: cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<DecEncodeFn>(p);
  }
  if (!desc || desc->n_layers <= 0 || desc->n_layers > kMaxLayers || desc->dim <= 0 || desc->max_ctx <= 0 ||
      (desc->head_dim != 32 && desc->head_dim != 64))
    return sm100_set_error(SM100_ERR_ARG, "decode_prepare: bad descriptor");
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  for (int l = 0; l < desc->n_layers; l++) {
    const cuuint64_t dims[2] = {(cuuint64_t)desc->dim, 2 * (cuuint64_t)desc->max_ctx};
    const cuuint64_t strides[1] = {(cuuint64_t)desc->dim * 4};
    const cuuint32_t box[2] = {(cuuint32_t)desc->head_dim, (cuuint32_t)kBoxRows};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap *mp = reinterpret_cast<CUtensorMap *>(desc->kv_map[l]);
    if (!desc->kv_cache[l] ||
        fn(mp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, desc->kv_cache[l], dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return sm100_set_error(SM100_ERR_CUDA, "decode_prepare: tensor map of layer %d", l);
  }
  return SM100_OK;
}

extern "C" int32_t sm100_decode_grid(int32_t heads, int32_t head_dim) {
  int dev = 0;
  cudaGetDevice(&dev);
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 0;
  if (heads <= 0 || head_dim <= 0) return 0;
  return members_per_head(heads, head_dim, n) * heads;
}

static int launch_decode(const Sm100DecodeModel *dev_model, int n_tokens, int G, size_t smem, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
  e = cudaLaunchKernelEx(&cfg, decode_kernel, dev_model, n_tokens);
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
            n_layers <= kMaxLayers && dim > 0 && dim % 128 == 0 && dim <= 2 * kThreads && hd * heads == dim &&
            (hd == 32 || hd == 64) && vocab > 0 && max_ctx > 0 &&
            Smem::smax(max_transfers(n_layers, vocab, G, dim), max_ctx, hd) >= 1;
  if (ok) {
    // every CTA's transfers within one stage; row slices within the row slots
    const Geo g0 = geo_of(0, G, heads, dim, hd, vocab, n_layers);
    const int64_t D = dim, frow = (4 * D + G - 1) / G, orow = (D + M - 1) / M;
    const int64_t hdr = hdr_floats(dim);
    ok = g0.qn <= kMaxRows && g0.qn + 6 <= kBiasFloats && (hdr + g0.qn * D) * 4 <= kStageBytes &&
         orow * hd * 4 <= kStageBytes && orow <= kCpRows * kWarps && frow <= kMaxRows && frow + 6 <= kBiasFloats &&
         (hdr + frow * D) * 4 <= kStageBytes && g0.R >= 1 && g0.R <= kMaxRows &&
         Smem::total(max_transfers(n_layers, vocab, G, dim), max_ctx, hd) <= (size_t)kSmemLimit;
  }
  if (!ok)
    return sm100_set_error(SM100_ERR_ARG,
                           "decode: unsupported shape (tokens %d, layers %d, dim %d, heads %d, vocab %d, ctx %d, %d SMs)",
                           n_tokens, n_layers, dim, heads, vocab, max_ctx, g_num_sms[dev]);
  const size_t smem = Smem::total(max_transfers(n_layers, vocab, G, dim), max_ctx, hd);
  return launch_decode(dev_model, n_tokens, G, smem, (cudaStream_t)stream);
}

extern "C" int sm100_decode_step(const Sm100DecodeModel *dev_model, int32_t n_layers, int32_t dim, int32_t heads,
                                 int32_t vocab, int32_t max_ctx, void *stream) {
  return sm100_decode_steps(dev_model, 1, n_layers, dim, heads, vocab, max_ctx, stream);
}
