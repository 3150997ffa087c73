// The batched decode step of a DeepSeek-V2-Lite-shaped MoE decoder (BASELINE
// config 5) around the skinny tensor-core GEMM (k_skinny.cu, bf16 dense
// projections at batch <= 32): RMSNorm to a bf16 operand, the q / compressed-kv
// post-processing (bf16 rounding, RMSNorm of the latent, YaRN rotary of the pe
// slices, cache append), absorbed multi-head latent attention over the
// compressed cache, top-k softmax routing, and the fp8-e4m3 experts with
// 128 x 128 f32 block scales (gate / up with SiLU, then down, weighted into
// the residual).  The reference's decode step is bench/dsv2_decode_bench.c
// (cfg :97-124, kernels :341-1110: rms, gred_q rope, kv_prep, mla_qlat /
// score / mix / o, route, moe_full_h / moe_full_out), bf16 at batch 1; the
// fp8 block-scaled experts are composed as W_fp8 * scale (src/dtype/fp8.c).
//
// Every kernel is launched with programmatic dependent launch and reads its
// inputs after griddepcontrol.wait.
#include <cuda.h>

#include <cstddef>
#include <cstring>
#include <cuda_fp8.h>

#include <algorithm>

#include "common.cuh"
#include "ds_route.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kDsMaxTok = 32;     // decode batch
constexpr int kDsMaxK = 8;        // experts per token
constexpr int kDsMaxCtx = 2048;

// Sticky status of the kernels of this file with bounded waits (a timeout sets it).
__device__ uint32_t g_ds_status;

// Where row b of a step reads and appends the compressed KV cache: slot
// seq[b] (b when seq is null) at position pos[b * pos_stride] (one shared
// position: stride 0).  A row outside [0, n_seq) x [0, ctx) is skipped (its
// outputs zero) and sets SM100_DECODE_ERR_ARG.
struct DsRows {
  const int32_t *pos;
  const int32_t *seq;
  int32_t pos_stride, n_seq;
};

__device__ __forceinline__ bool ds_row(const DsRows &r, int b, int ctx, int &seq, int &p) {
  p = r.pos[(int64_t)b * r.pos_stride];
  seq = r.seq ? r.seq[b] : b;
  if (p >= 0 && p < ctx && seq >= 0 && seq < r.n_seq) return true;
  atomicOr(&g_ds_status, SM100_DECODE_ERR_ARG);
  return false;
}

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// y = bf16(x * rsqrt(mean(x^2) + eps) * g) per row (RMSNorm, deepseek_v2.py's
// RMSNorm as the reference folds it, dsv2_decode_bench.c:341-430), one CTA of
// 256 threads per row.  Rows of D % 4 == 0, D <= 4096 go in float4 chunks
// (thread t: chunks t, t + 256, ..), every load of the row issued before the
// first is used, the gains read before the wait on the previous kernel; ys
// (shared, may be null) receives the row as well.
constexpr int kRmsV = 4;
__device__ __forceinline__ bool ds_rms_vec(int D) { return D % 4 == 0 && D <= 1024 * kRmsV; }

__device__ __forceinline__ void ds_rms_gains(const float *g, int D, float4 (&gv)[kRmsV]) {
#pragma unroll
  for (int i = 0; i < kRmsV; i++) {
    const int c = threadIdx.x + 256 * i;
    gv[i] = 4 * c < D ? __ldg(reinterpret_cast<const float4 *>(g) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

__device__ __forceinline__ void ds_rms_row(const float *xr, const float *g, const float4 (&gv)[kRmsV],
                                           __nv_bfloat16 *yr, __nv_bfloat16 *ys, int D, float eps) {
  __shared__ float red[8];
  float s = 0.0f;
  if (ds_rms_vec(D)) {
    float4 xv[kRmsV];
#pragma unroll
    for (int i = 0; i < kRmsV; i++) {
      const int c = threadIdx.x + 256 * i;
      xv[i] = 4 * c < D ? reinterpret_cast<const float4 *>(xr)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kRmsV; i++)
      s = fmaf(xv[i].w, xv[i].w, fmaf(xv[i].z, xv[i].z, fmaf(xv[i].y, xv[i].y, fmaf(xv[i].x, xv[i].x, s))));
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) t += red[w];
    const float inv = 1.0f / sqrtf(t * (1.0f / (float)D) + eps);
#pragma unroll
    for (int i = 0; i < kRmsV; i++) {
      const int c = threadIdx.x + 256 * i;
      if (4 * c >= D) break;
      const __nv_bfloat162 y0 = __floats2bfloat162_rn((xv[i].x * inv) * gv[i].x, (xv[i].y * inv) * gv[i].y);
      const __nv_bfloat162 y1 = __floats2bfloat162_rn((xv[i].z * inv) * gv[i].z, (xv[i].w * inv) * gv[i].w);
      reinterpret_cast<__nv_bfloat162 *>(yr)[2 * c] = y0;
      reinterpret_cast<__nv_bfloat162 *>(yr)[2 * c + 1] = y1;
      if (ys) {
        reinterpret_cast<__nv_bfloat162 *>(ys)[2 * c] = y0;
        reinterpret_cast<__nv_bfloat162 *>(ys)[2 * c + 1] = y1;
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < D; i += 256) s = fmaf(xr[i], xr[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) t += red[w];
  const float inv = 1.0f / sqrtf(t * (1.0f / (float)D) + eps);
  for (int i = threadIdx.x; i < D; i += 256) {
    const __nv_bfloat16 v = __float2bfloat16_rn((xr[i] * inv) * g[i]);
    yr[i] = v;
    if (ys) ys[i] = v;
  }
}

__global__ void __launch_bounds__(256) ds_rms_kernel(const float *x, const float *g, __nv_bfloat16 *y, int D,
                                                      float eps) {
  float4 gv[kRmsV];
  if (ds_rms_vec(D)) ds_rms_gains(g, D, gv);
  pdl_trigger();
  pdl_wait();
  ds_rms_row(x + (int64_t)blockIdx.x * D, g, gv, y + (int64_t)blockIdx.x * D, nullptr, D, eps);
}

// h[b] = embed[tok[b]] (bf16 table; ids outside [0, V) read zeros)
__global__ void ds_embed_kernel(const __nv_bfloat16 *emb, const int32_t *tok, float *h, int V, int D) {
  pdl_trigger();
  pdl_wait();
  const int id = tok[blockIdx.x];
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    h[(int64_t)blockIdx.x * D + d] = (id >= 0 && id < V) ? bf(emb[(int64_t)id * D + d]) : 0.0f;
}

// Per token b (one CTA; q and kva rows of stride ld): q [H][DN + DR] -> bf16 nope, rotary pe (the pe
// slice is rounded to bf16 first; pair (2j, 2j+1) rotates into columns j and
// DR/2 + j); kva [KV + DR] -> the latent rounded to bf16, RMSNormed with
// g_kv, and the rotary k_pe, both appended to the caches at row pos.
__global__ void __launch_bounds__(256) ds_qkv_post_kernel(const float *q, const float *kva, const float *g_kv,
                                                           const float *cs, const float *sn, const DsRows rows,
                                                           __nv_bfloat16 *qo, __nv_bfloat16 *cc, __nv_bfloat16 *cpe,
                                                           int H, int DN, int DR, int KV, int ctx, float eps,
                                                           int64_t ld) {
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, half = DR / 2, QS = DN + DR;
  int seq, p;
  if (!ds_row(rows, b, ctx, seq, p)) return;
  const float *qb = q + (int64_t)b * ld;
  __nv_bfloat16 *qob = qo + (int64_t)b * H * QS;
  for (int i = threadIdx.x; i < H * DN; i += 256) {
    const int h = i / DN, d = i % DN;
    qob[h * QS + d] = __float2bfloat16_rn(qb[h * QS + d]);
  }
  for (int i = threadIdx.x; i < H * half; i += 256) {
    const int h = i / half, j = i % half;
    const float xe = bfr(qb[h * QS + DN + 2 * j]), xo = bfr(qb[h * QS + DN + 2 * j + 1]);
    const float c = cs[(int64_t)p * DR + j], s = sn[(int64_t)p * DR + j];
    qob[h * QS + DN + j] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(xe, c), __fmul_rn(xo, s)));
    qob[h * QS + DN + half + j] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(xo, c), __fmul_rn(xe, s)));
  }
  const float *kb = kva + (int64_t)b * ld;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < KV; i += 256) {
    const float v = bfr(kb[i]);
    ss = __fmaf_rn(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) t += red[w];
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(t, 1.0f / (float)KV), eps)));
  __nv_bfloat16 *crow = cc + ((int64_t)seq * ctx + p) * KV;
  for (int i = threadIdx.x; i < KV; i += 256) crow[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(bfr(kb[i]), inv), g_kv[i]));
  __nv_bfloat16 *prow = cpe + ((int64_t)seq * ctx + p) * DR;
  for (int j = threadIdx.x; j < half; j += 256) {
    const float xe = bfr(kb[KV + 2 * j]), xo = bfr(kb[KV + 2 * j + 1]);
    const float c = cs[(int64_t)p * DR + j], s = sn[(int64_t)p * DR + j];
    prow[j] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(xe, c), __fmul_rn(xo, s)));
    prow[half + j] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(xo, c), __fmul_rn(xe, s)));
  }
}

// Absorbed MLA of one (token b, head h): qlat = W_uk[h]^T q_nope (KV), scores
// over cache rows 0..pos = (qlat . c_t + q_pe . pe_t) * scale, softmax,
// olat = sum_t p_t c_t, o = bf16(W_uv[h] olat) (DV).  W_uk / W_uv [H][DN or
// DV][KV] bf16 (kv_b_proj split, deepseek_v2.py's absorb).

constexpr int kDsKV = 512;
__global__ void __launch_bounds__(256) ds_mla_kernel(const __nv_bfloat16 *qo, const __nv_bfloat16 *wuk,
                                                      const __nv_bfloat16 *wuv, const __nv_bfloat16 *cc,
                                                      const __nv_bfloat16 *cpe, const DsRows rows, __nv_bfloat16 *o,
                                                      int H, int DN, int DR, int DV, int KV, int ctx, float scale) {
  __shared__ float qlat[kDsKV];
  __shared__ float qn[256];
  __shared__ float qpe[128];
  __shared__ float sc[kDsMaxCtx];
  __shared__ float olat[kDsKV];
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x / H, h = blockIdx.x % H, QS = DN + DR;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int seq, p;
  if (!ds_row(rows, b, ctx, seq, p)) {
    for (int r = threadIdx.x; r < DV; r += 256) o[((int64_t)b * H + h) * DV + r] = __float2bfloat16_rn(0.0f);
    return;
  }
  const int T = p + 1;
  const __nv_bfloat16 *qrow = qo + ((int64_t)b * H + h) * QS;
  for (int i = threadIdx.x; i < DN; i += 256) qn[i] = bf(qrow[i]);
  for (int i = threadIdx.x; i < DR; i += 256) qpe[i] = bf(qrow[DN + i]);
  __syncthreads();
  const __nv_bfloat16 *wk = wuk + (int64_t)h * DN * KV;
  for (int k = threadIdx.x; k < KV; k += 256) {
    float a = 0.0f;
    for (int d = 0; d < DN; d++) a += qn[d] * bf(wk[(int64_t)d * KV + k]);
    qlat[k] = a;
  }
  __syncthreads();
  const __nv_bfloat16 *cb = cc + (int64_t)seq * ctx * KV, *pb = cpe + (int64_t)seq * ctx * DR;
  for (int t = warp; t < T; t += 8) {   // a warp per cache row
    float s = 0.0f;
    for (int k = lane; k < KV; k += 32) s += qlat[k] * bf(cb[(int64_t)t * KV + k]);
    for (int k = lane; k < DR; k += 32) s += qpe[k] * bf(pb[(int64_t)t * DR + k]);
    s = warp_sum(s);
    if (lane == 0) sc[t] = s * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int t = threadIdx.x; t < T; t += 256) m = fmaxf(m, sc[t]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; w++) m = fmaxf(m, red[w]);
  __syncthreads();
  float sum = 0.0f;
  for (int t = threadIdx.x; t < T; t += 256) {
    const float e = expf(sc[t] - m);
    sc[t] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) tot += red[w];
  const float inv = 1.0f / tot;
  for (int k = threadIdx.x; k < KV; k += 256) {
    float a = 0.0f;
    for (int t = 0; t < T; t++) a += sc[t] * bf(cb[(int64_t)t * KV + k]);
    olat[k] = a * inv;
  }
  __syncthreads();
  const __nv_bfloat16 *wv = wuv + (int64_t)h * DV * KV;
  for (int r = warp; r < DV; r += 8) {
    float a = 0.0f;
    for (int k = lane; k < KV; k += 32) a += olat[k] * bf(wv[(int64_t)r * KV + k]);
    a = warp_sum(a);
    if (lane == 0) o[((int64_t)b * H + h) * DV + r] = __float2bfloat16_rn(a);
  }
}

// The same attention, one CTA per (head h, group of NB <= kMlaNB sequences), for
// the DeepSeek-V2-Lite shapes (latent 512, rope 64, nope / v <= 128).  The
// head's absorbed weights are read once per group instead of once per
// sequence: W_uk[h] comes into shared memory by one bulk copy (issued before
// the wait for the previous kernel), q_lat of the group's sequences is taken
// from it, and W_uv[h] is copied into the same buffer while the cache rows
// are walked.  Each warp walks a stripe of a sequence's rows once (16-byte
// loads: lane l holds latent columns [8 l, 8 l + 8) and [256 + 8 l, ...),
// lanes 0-7 the rope columns) with an online softmax, and the warps' (max,
// sum, partial o_lat) are folded in a fixed order.  The softmax is exp(s -
// running max) rescaled (expf), the order of the reference's max / exp / sum
// / divide up to rounding.
constexpr int kMlaNB = 4, kMlaWarps = 16, kMlaKV = 512, kMlaDR = 64, kMlaMaxD = 128;
static_assert(kMlaWarps * 32 == kMlaKV, "q_lat: one latent column per thread");

struct MlaSmem {
  static constexpr size_t w = 0;                                              // [128][512] bf16 W_uk[h], then W_uv[h]
  static constexpr size_t qn = w + kMlaMaxD * kMlaKV * 2;                     // [DN][kMlaNB] f32
  static constexpr size_t qpe = qn + kMlaMaxD * kMlaNB * 4;                   // [kMlaNB][64] f32
  static constexpr size_t qlat = qpe + kMlaNB * kMlaDR * 4;                   // [kMlaNB][512] f32 (then o_lat)
  static constexpr size_t po = qlat + kMlaNB * kMlaKV * 4;                    // [warps][512] f32 (one sequence a warp)
  static constexpr size_t pm = po + (size_t)kMlaWarps * kMlaKV * 4;           // [warps] max
  static constexpr size_t pl = pm + kMlaWarps * 4;                            // [warps] sum
  static constexpr size_t cur = pl + kMlaWarps * 4;                        // [kMlaNB][512 + 64] bf16 current rows
  static constexpr size_t bar = cur + kMlaNB * (kMlaKV + kMlaDR) * 2;
  static constexpr size_t total = bar + 16;
};

// MlaPost: the projection outputs (f32 rows of stride ld: the H heads' q
// [H][DN + DR], then the latent [KV] and the key's rope pair [DR]) come in
// instead of the post-processed q; the CTA does ds_qkv_post's work for its
// sequences itself (same operations, same order): q rounded and rotated,
// the current latent row RMSNormed and the key rotated into shared memory,
// which the walk reads for the current position; the head-0 CTAs store that
// row into the caches for the later steps.
struct MlaPost {
  const float *qkva;
  int64_t ld, kva_off;
  const float *g_kv, *cs, *sn;
  float eps;
};

template <int NB, bool kPost>
__global__ void __launch_bounds__(kMlaWarps * 32, 1)
    ds_mla_group_kernel(const __nv_bfloat16 *qo, const __nv_bfloat16 *wuk, const __nv_bfloat16 *wuv,
                        __nv_bfloat16 *cc, __nv_bfloat16 *cpe, const DsRows rows, __nv_bfloat16 *o, int B,
                        int H, int DN, int DV, int ctx, float scale, MlaPost post) {
  extern __shared__ __align__(128) unsigned char sm[];
  __nv_bfloat16 *wb = reinterpret_cast<__nv_bfloat16 *>(sm + MlaSmem::w);
  float *qn = reinterpret_cast<float *>(sm + MlaSmem::qn), *qpe = reinterpret_cast<float *>(sm + MlaSmem::qpe);
  float *qlat = reinterpret_cast<float *>(sm + MlaSmem::qlat), *po = reinterpret_cast<float *>(sm + MlaSmem::po);
  float *pm = reinterpret_cast<float *>(sm + MlaSmem::pm), *pl = reinterpret_cast<float *>(sm + MlaSmem::pl);
  uint64_t *bar = reinterpret_cast<uint64_t *>(sm + MlaSmem::bar);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int h = blockIdx.x % H, b0 = (blockIdx.x / H) * NB, nb = min(NB, B - b0), QS = DN + kMlaDR;
  uint32_t *status = &g_ds_status;
  if (t == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (t == 0) {   // the weights are static: their copy overlaps the previous kernel
    mbar_expect_tx(bar, (uint32_t)(DN * kMlaKV * 2));
    bulk_g2s(wb, wuk + (int64_t)h * DN * kMlaKV, (uint32_t)(DN * kMlaKV * 2), bar);
  }
  pdl_trigger();
  pdl_wait();
  // each sequence's cache slot and position (rows outside the caches: T = 0,
  // o = 0)
  __shared__ int s_seq[kMlaNB], s_pos[kMlaNB], s_T[kMlaNB];
  if (t < nb) {
    int sq, pp;
    const bool ok = ds_row(rows, b0 + t, ctx, sq, pp);
    s_seq[t] = ok ? sq : 0;
    s_pos[t] = ok ? pp : 0;
    s_T[t] = ok ? pp + 1 : 0;
  }
  __syncthreads();
  __nv_bfloat16 *cur = reinterpret_cast<__nv_bfloat16 *>(sm + MlaSmem::cur);   // [NB][512 latent | 64 rope]
  for (int i = t; i < kMlaNB * QS; i += kMlaWarps * 32) {
    const int b = i / QS, d = i % QS;
    float v = 0.0f;
    if (b < nb) {
      if constexpr (kPost) {   // ds_qkv_post's q: nope rounded; rope pairs rounded, rotated, rounded
        const float *qr = post.qkva + (int64_t)(b0 + b) * post.ld + h * QS;
        const int p = s_pos[b];
        constexpr int half = kMlaDR / 2;
        if (d < DN) {
          v = bfr(qr[d]);
        } else {
          const int j = (d - DN) % half;
          const float xe = bfr(qr[DN + 2 * j]), xo = bfr(qr[DN + 2 * j + 1]);
          const float c = post.cs[(int64_t)p * kMlaDR + j], sv = post.sn[(int64_t)p * kMlaDR + j];
          v = bfr(d - DN < half ? __fsub_rn(__fmul_rn(xe, c), __fmul_rn(xo, sv))
                                : __fadd_rn(__fmul_rn(xo, c), __fmul_rn(xe, sv)));
        }
      } else {
        v = bf(qo[((int64_t)(b0 + b) * H + h) * QS + d]);
      }
    }
    if (d < DN) qn[d * kMlaNB + b] = v;
    else qpe[b * kMlaDR + d - DN] = v;
  }
  if constexpr (kPost) {   // the current latent / key rows (ds_qkv_post's arithmetic, in its order)
    // each 256-thread half takes sequences half, half + 2: thread u sums
    // elements u and u + 256 and the 8 warp sums are added in order, as
    // ds_qkv_post_kernel's 256 threads do for one sequence
    __shared__ float red[kMlaNB][8];
    __shared__ float s_inv[kMlaNB];
    const int half = t >> 8, u = t & 255;
    for (int b = half; b < nb; b += 2) {
      const float *kb = post.qkva + (int64_t)(b0 + b) * post.ld + post.kva_off;
      float ss = 0.0f;
      for (int i = u; i < kMlaKV; i += 256) {
        const float v = bfr(kb[i]);
        ss = __fmaf_rn(v, v, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) red[b][(u >> 5)] = ss;
    }
    __syncthreads();
    if (t < nb) {
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; w++) tot += red[t][w];
      s_inv[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / (float)kMlaKV), post.eps)));
    }
    __syncthreads();
    for (int i = t; i < nb * kMlaKV; i += kMlaWarps * 32) {
      const int b = i / kMlaKV, k = i % kMlaKV;
      const float *kb = post.qkva + (int64_t)(b0 + b) * post.ld + post.kva_off;
      cur[b * (kMlaKV + kMlaDR) + k] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(bfr(kb[k]), s_inv[b]), post.g_kv[k]));
    }
    for (int i = t; i < nb * (kMlaDR / 2); i += kMlaWarps * 32) {
      const int b = i / (kMlaDR / 2), j = i % (kMlaDR / 2);
      const float *kb = post.qkva + (int64_t)(b0 + b) * post.ld + post.kva_off;
      __nv_bfloat16 *prow = cur + b * (kMlaKV + kMlaDR) + kMlaKV;
      const float xe = bfr(kb[kMlaKV + 2 * j]), xo = bfr(kb[kMlaKV + 2 * j + 1]);
      const int p = s_pos[b];
      const float c = post.cs[(int64_t)p * kMlaDR + j], sv = post.sn[(int64_t)p * kMlaDR + j];
      prow[j] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(xe, c), __fmul_rn(xo, sv)));
      prow[kMlaDR / 2 + j] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(xo, c), __fmul_rn(xe, sv)));
    }
    __syncthreads();
    if (h == 0)   // one head's CTAs keep the rows for the later steps
      for (int i = t; i < nb * (kMlaKV + kMlaDR); i += kMlaWarps * 32) {
        const int b = i / (kMlaKV + kMlaDR), c = i % (kMlaKV + kMlaDR);
        if (s_T[b] == 0) continue;
        const __nv_bfloat16 v = cur[i];
        const int64_t row = (int64_t)s_seq[b] * ctx + s_pos[b];
        if (c < kMlaKV) cc[row * kMlaKV + c] = v;
        else cpe[row * kMlaDR + c - kMlaKV] = v;
      }
  }
  __syncthreads();
  const bool wk_ok = mbar_wait(bar, 0, status, false);
  // q_lat[b][k] = sum_d q_nope[b][d] W_uk[h][d][k], k = t
  {
    float a[NB] = {};
    if (wk_ok) {
#pragma unroll 8
      for (int d = 0; d < DN; d++) {
        const float4 q4 = reinterpret_cast<const float4 *>(qn)[d];
        const float w0 = bf(wb[d * kMlaKV + t]);
        const float qq[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int b = 0; b < NB; b++) a[b] = fmaf(qq[b], w0, a[b]);
      }
    }
#pragma unroll
    for (int b = 0; b < NB; b++) qlat[b * kMlaKV + t] = a[b];
  }
  __syncthreads();
  if (t == 0) {   // W_uv[h] into the same buffer (every read of W_uk is done)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, (uint32_t)(DV * kMlaKV * 2));
    bulk_g2s(wb, wuv + (int64_t)h * DV * kMlaKV, (uint32_t)(DV * kMlaKV * 2), bar);
  }
  // one pass over each sequence's rows: the warps are split evenly over the
  // NB sequences (kMlaWarps / NB each), and warp j of sequence b takes its
  // rows j, j + kMlaWarps / NB, ...
  constexpr int kWpb = kMlaWarps / NB;
  {
    const int b = warp / kWpb, j0 = warp % kWpb;
    const float *ql = qlat + b * kMlaKV;
    float qk[16], qp[8], oa[16];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      qk[j] = ql[8 * lane + j];
      qk[8 + j] = ql[256 + 8 * lane + j];
      qp[j] = lane < 8 ? qpe[b * kMlaDR + 8 * lane + j] : 0.0f;
      oa[j] = oa[8 + j] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const int sb = b < nb ? b : 0, p = s_pos[sb], T = b < nb ? s_T[sb] : 0;
    const __nv_bfloat16 *cb = cc + (int64_t)s_seq[sb] * ctx * kMlaKV, *pb = cpe + (int64_t)s_seq[sb] * ctx * kMlaDR;
#pragma unroll 4
    for (int r = j0; r < T; r += kWpb) {
      // with kPost the current row is the one in shared memory
      const __nv_bfloat16 *crow = kPost && r == p ? cur + b * (kMlaKV + kMlaDR) : cb + (int64_t)r * kMlaKV;
      const __nv_bfloat16 *prow = kPost && r == p ? cur + b * (kMlaKV + kMlaDR) + kMlaKV : pb + (int64_t)r * kMlaDR;
      const uint4 c0 = *reinterpret_cast<const uint4 *>(crow + 8 * lane);
      const uint4 c1 = *reinterpret_cast<const uint4 *>(crow + 256 + 8 * lane);
      const uint4 pe = lane < 8 ? *reinterpret_cast<const uint4 *>(prow + 8 * lane) : make_uint4(0, 0, 0, 0);
      const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const uint32_t pw[4] = {pe.x, pe.y, pe.z, pe.w};
      float cv[16];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        cv[2 * j] = __uint_as_float(cw[j] << 16);
        cv[2 * j + 1] = __uint_as_float(cw[j] & 0xFFFF0000u);
      }
      float sdot = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; j++) sdot = fmaf(qk[j], cv[j], sdot);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        sdot = fmaf(qp[2 * j], __uint_as_float(pw[j] << 16), sdot);
        sdot = fmaf(qp[2 * j + 1], __uint_as_float(pw[j] & 0xFFFF0000u), sdot);
      }
      const float sv = warp_sum(sdot) * scale;
      const float mn = fmaxf(m, sv), cr = expf(m - mn), p = expf(sv - mn);
      l = l * cr + p;
#pragma unroll
      for (int j = 0; j < 16; j++) oa[j] = fmaf(p, cv[j], oa[j] * cr);
      m = mn;
    }
    float *pob = po + (size_t)warp * kMlaKV;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      pob[8 * lane + j] = oa[j];
      pob[256 + 8 * lane + j] = oa[8 + j];
    }
    if (lane == 0) {
      pm[warp] = m;
      pl[warp] = l;
    }
  }
  __syncthreads();
  // fold a sequence's warps in order: o_lat[b][k] = sum_w f_w o_w[k] / sum_w f_w l_w,
  // f_w = e^(m_w - M); the factors once per warp, then one pass over the columns
  __shared__ float s_f[kMlaWarps], s_L[kMlaNB];
  if (t < nb) {
    float M = -INFINITY;
    for (int w = t * kWpb; w < (t + 1) * kWpb; w++) M = fmaxf(M, pm[w]);
    float L = 0.0f;
    for (int w = t * kWpb; w < (t + 1) * kWpb; w++) {
      const float f = pm[w] == -INFINITY ? 0.0f : expf(pm[w] - M);
      s_f[w] = f;
      L = fmaf(f, pl[w], L);
    }
    s_L[t] = L;
  }
  __syncthreads();
  for (int i = t; i < nb * kMlaKV; i += kMlaWarps * 32) {
    const int b = i / kMlaKV, k = i % kMlaKV;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kWpb; w++) acc = fmaf(s_f[b * kWpb + w], po[(size_t)(b * kWpb + w) * kMlaKV + k], acc);
    qlat[b * kMlaKV + k] = s_L[b] > 0.0f ? acc / s_L[b] : 0.0f;   // a skipped row: o = 0
  }
  __syncthreads();
  const bool wv_ok = mbar_wait(bar, 1, status, false);
  // o[b][h][r] = sum_k o_lat[b][k] W_uv[h][r][k]: warp w takes rows w, w + 8,
  // ..., lane l the columns 2 (l + 32 i) and 2 (l + 32 i) + 1
  float ov[NB][16];
#pragma unroll
  for (int b = 0; b < NB; b++)
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float2 v = b < nb ? reinterpret_cast<const float2 *>(qlat + b * kMlaKV)[lane + 32 * i] : make_float2(0.f, 0.f);
      ov[b][2 * i] = v.x;
      ov[b][2 * i + 1] = v.y;
    }
  for (int r = warp; r < DV; r += kMlaWarps) {
    float acc[NB] = {};
    if (wv_ok) {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint32_t w2 = reinterpret_cast<const uint32_t *>(wb + r * kMlaKV)[lane + 32 * i];
        const float w0 = __uint_as_float(w2 << 16), w1 = __uint_as_float(w2 & 0xFFFF0000u);
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = fmaf(ov[b][2 * i + 1], w1, fmaf(ov[b][2 * i], w0, acc[b]));
      }
    }
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = warp_sum(acc[b]);
    if (lane < nb) {
      float v = acc[0];
#pragma unroll
      for (int b = 1; b < NB; b++) v = lane == b ? acc[b] : v;
      o[((int64_t)(b0 + lane) * H + h) * DV + r] = __float2bfloat16_rn(v);
    }
  }
}

// Routing of every token by one CTA of >= 256 threads (a warp per token; the
// logits are read at L2: they may come from other CTAs), the rule and the
// packing of ds_route.cuh.
__device__ __forceinline__ void ds_route_block(const float *logits, int E, int K, int B, int e0, int e1, int n_shared,
                                               int32_t *sel, float *wsel, int32_t *slot_off, int32_t *slot_tok,
                                               float *slot_w) {
  __shared__ int32_t s_sel[kDsMaxTok * kDsMaxK];
  __shared__ float s_w[kDsMaxTok * kDsMaxK];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int b = warp; b < B; b += nwarps) {
    const float *lg = logits + (int64_t)b * E;
    const float l0 = lane < E ? __ldcg(lg + lane) : 0.0f, l1 = lane + 32 < E ? __ldcg(lg + lane + 32) : 0.0f;
    ds_route_select(l0, l1, E, K, sel + (int64_t)b * K, wsel + (int64_t)b * K, s_sel + b * K, s_w + b * K);
  }
  __syncthreads();
  ds_route_pack(s_sel, s_w, B, K, e0, e1, n_shared, slot_off, slot_tok, slot_w);
}

__global__ void __launch_bounds__(1024) ds_route_kernel(const float *logits, int E, int K, int B, int e0, int e1,
                                                         int n_shared, int32_t *sel, float *wsel, int32_t *slot_off,
                                                         int32_t *slot_tok, float *slot_w) {
  pdl_trigger();
  pdl_wait();
  ds_route_block(logits, E, K, B, e0, e1, n_shared, sel, wsel, slot_off, slot_tok, slot_w);
}

// The router product and the routing in one launch: CTA e (1024 threads)
// computes the logits of expert e for every token (x . router[e], bf16 x
// bf16 with f32 sums, one warp per token), and the last CTA to finish (a
// device counter, no waiting) routes every token as ds_route_kernel does, a
// warp per token, and resets the counter for the next launch.  The router
// row does not depend on the previous kernel: each lane holds its chunks of
// it in registers before the wait (rows of D <= 8 x 256; longer rows load
// the rest after).  Thread 0 counts the CTA off with an acq_rel atomic
// after a barrier, which releases every warp's logit.
constexpr int kRtPre = 8;
__global__ void __launch_bounds__(1024) ds_router_route_kernel(const __nv_bfloat16 *x, const __nv_bfloat16 *router,
                                                               float *logits, int32_t *counter, int D, int E, int K,
                                                               int B, int e0, int e1, int n_shared, int32_t *sel,
                                                               float *wsel, int32_t *slot_off, int32_t *slot_tok,
                                                               float *slot_w) {
  __shared__ int s_last;
  const int e = blockIdx.x, lane = threadIdx.x & 31, b = threadIdx.x >> 5;
  const __nv_bfloat16 *we = router + (int64_t)e * D;
  uint4 wpre[kRtPre];
#pragma unroll
  for (int i = 0; i < kRtPre; i++) {
    const int k = lane * 8 + 256 * i;
    wpre[i] = b < B && k < D ? __ldg(reinterpret_cast<const uint4 *>(we + k)) : make_uint4(0, 0, 0, 0);
  }
  pdl_trigger();
  pdl_wait();
  // warp b: token b; lane l sums its chunks l, l + 32, .. in order, then the
  // lanes by the butterfly
  if (b < B) {
    const uint4 *xs = reinterpret_cast<const uint4 *>(x + (int64_t)b * D);
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kRtPre; i++) {
      const int k = lane * 8 + 256 * i;
      if (k < D) {
        const uint4 xv = xs[k / 8], wv = wpre[i];
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          acc = fmaf(__uint_as_float(xx[q] << 16), __uint_as_float(ww[q] << 16), acc);
          acc = fmaf(__uint_as_float(xx[q] & 0xFFFF0000u), __uint_as_float(ww[q] & 0xFFFF0000u), acc);
        }
      }
    }
    for (int k = lane * 8 + 256 * kRtPre; k < D; k += 256) {
      const uint4 xv = xs[k / 8], wv = __ldg(reinterpret_cast<const uint4 *>(we + k));
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        acc = fmaf(__uint_as_float(xx[q] << 16), __uint_as_float(ww[q] << 16), acc);
        acc = fmaf(__uint_as_float(xx[q] & 0xFFFF0000u), __uint_as_float(ww[q] & 0xFFFF0000u), acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[(int64_t)b * E + e] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
    s_last = prev == E - 1;
  }
  // the last CTA's thread 0 acquired every CTA's release; the barrier carries
  // that to the CTA's other threads, whose loads go to L2
  __syncthreads();
  if (!s_last) return;
  ds_route_block(logits, E, K, B, e0, e1, n_shared, sel, wsel, slot_off, slot_tok, slot_w);
  if (threadIdx.x == 0) *counter = 0;
}

// The experts on the 5th-generation tensor cores, fp8 in both operands.  A
// work item is (expert e, block of 128 weight rows).  The weights are the
// MMA's A operand as stored: fp8-e4m3 tiles of 128 rows x 128 k that TMA
// copies from HBM into a ring (4 stages up, 8 down) in the 128-byte swizzle,
// with no conversion.  The tokens (up to 32, the MMA's N; rows past the
// count zero) become the B operand: for k-block kb of weight row block t,
// v = x * s[t][kb] * 2^p[t][tok] is split into two e4m3 terms, hi = e4m3(v)
// and lo = e4m3(v - hi), whose sum carries v to about 2^-8 of |v| (bf16's
// precision); 2^p[t][tok] is the power of two that puts the token's largest
// |x| times the row block's largest block scale in [128, 256), so neither
// term saturates.  8 warps build those tiles; one thread issues tcgen05.mma
// kind::f8f6f4 (M=128, N=32, K=32) over the hi and lo tiles into one TMEM
// accumulator (two sets, so an item's epilogue overlaps the next item's
// products); 4 epilogue warps multiply by 2^-p[t][tok] and finish it:
//   kUp:  rows j of gate and up (W_gu [2I][D]) -> a[slot][j] = bf16(silu(g) * u)
//   down: rows r of W_d [D][I]               -> y[tok][r] += w_slot * sum
// An expert without tokens costs one read of its slot count.  Every wait is
// bounded; a timeout sets g_ds_status, and the TMA thread drains its copies
// before the CTA exits.

constexpr int kX8Prep = 8;                              // token-tile warps
constexpr int kX8Tma = kX8Prep, kX8Mma = kX8Prep + 1;   // then 4 epilogue warps
constexpr int kX8Threads = (kX8Prep + 2 + 4) * 32;
constexpr int kX8A = 128 * 128;   // fp8 [128 rows][128 k]: one 128-byte swizzle row per weight row
constexpr int kX8B = 32 * 128;    // fp8 [32 tokens][128 k]
constexpr int kX8MaxKb = 32;      // k-blocks per item (K <= 4096): one block scale per lane

template <bool kUp>
__host__ __device__ constexpr int x8_stages() {
  return kUp ? 4 : 8;
}
// stage: A tiles [kA], then B tiles [kA][hi, lo]
template <bool kUp>
__host__ __device__ constexpr int x8_stage() {
  return (kUp ? 2 : 1) * (kX8A + 2 * kX8B);
}
template <bool kUp>
__host__ __device__ constexpr int x8_smem() {
  return x8_stages<kUp>() * x8_stage<kUp>() + 1024 /* alignment */ + 1024 /* barriers, scales */;
}

__device__ __forceinline__ uint64_t x8_desc(const void *p) {
  const uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// 32 consecutive TMEM columns of this warp's 32 lanes (one f32 each)
__device__ __forceinline__ void x8_tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

// a weight tile into L2 only (no shared memory, no barrier)
__device__ __forceinline__ void x8_prefetch_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void x8_tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 2^p with m * 2^p in [128, 256) for a positive finite m (clamped to
// [2^-126, 2^126]); 1 for zero, inf or nan
__device__ __forceinline__ float x8_pow2(float m) {
  const int eb = (int)((__float_as_uint(m) >> 23) & 0xFFu);
  if (!(m > 0.0f) || eb == 0xFF) return 1.0f;
  return __uint_as_float((uint32_t)min(max(261 - eb, 1), 253) << 23);
}

// |x| max of 8 bf16
__device__ __forceinline__ float x8_absmax8(const uint4 v) {
  float r = 0.0f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; q++) r = fmaxf(r, fmaxf(fabsf(bf16_lo(w[q])), fabsf(bf16_hi(w[q]))));
  return r;
}

// 16 bf16 (a, b) times cf -> e4m3 hi and lo terms (16 bytes each, element
// order kept: the lower k in the lower byte)
__device__ __forceinline__ void x8_split16(const uint4 a, const uint4 b, float cf, uint4 &hi, uint4 &lo) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t h[4], l[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t hh = 0, ll = 0;
#pragma unroll
    for (int p = 0; p < 2; p++) {
      const uint32_t ww = w[2 * q + p];
      const float v0 = bf16_lo(ww) * cf, v1 = bf16_hi(ww) * cf;
      const __nv_fp8x2_storage_t h2 = __nv_cvt_float2_to_fp8x2(make_float2(v0, v1), __NV_SATFINITE, __NV_E4M3);
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(h2, __NV_E4M3);
      const float2 hf = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
      const __nv_fp8x2_storage_t l2 =
          __nv_cvt_float2_to_fp8x2(make_float2(v0 - hf.x, v1 - hf.y), __NV_SATFINITE, __NV_E4M3);
      hh |= (uint32_t)h2 << (16 * p);
      ll |= (uint32_t)l2 << (16 * p);
    }
    h[q] = hh;
    l[q] = ll;
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <bool kUp>
__global__ void __launch_bounds__(kX8Threads, 1)
    ds_x8_kernel(const __grid_constant__ CUtensorMap wmap, const __nv_bfloat16 *xin, const float *sc,
                 const int32_t *slot_off, const int32_t *slot_tok, const float *slot_w, void *out, int D, int I,
                 int64_t s_stride, int n_exp) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int kS = x8_stages<kUp>(), kStage = x8_stage<kUp>(), kA = kUp ? 2 : 1;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kS * kStage);
  uint64_t *full_a = bars, *full_b = bars + kS, *empty = bars + 2 * kS, *acc_full = bars + 3 * kS,
           *acc_empty = acc_full + 2, *sc_full = acc_empty + 2, *done = sc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  float *sout = reinterpret_cast<float *>(smem + kS * kStage + 512);   // [2 sets][kA][32 tokens]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // rows of the product and its contraction: up: 128-row blocks of I, K = D; down: blocks of D, K = I
  const int rows = kUp ? I : D, K = kUp ? D : I, nblk = rows / 128, nkb = K / 128;
  const int rows_w = kUp ? 2 * I : D;   // weight rows of one expert in the tensor map
  const int sc_cols = kUp ? D / 128 : (I + 127) / 128;
  const int n_items = n_exp * nblk;
  uint32_t *status = &g_ds_status;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kS; i++) {
      mbar_init(&full_a[i], 1);
      mbar_init(&full_b[i], kX8Prep);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
      mbar_init(&sc_full[i], kX8Prep);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kX8Mma) {   // accumulators: 2 sets x kA x 64 columns (hi | lo)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // The weights are static, the routing is not known yet: while the previous
  // kernel (the routing) finishes, this CTA's first item's leading tiles come
  // into L2, whether or not its expert gets tokens (most do).
  if (warp == kX8Tma && lane == 0 && blockIdx.x < n_items) {
    const int e = blockIdx.x / nblk, blk = blockIdx.x % nblk;
    const int pre_kb = min(nkb, kUp ? 8 : 12);
    for (int kb = 0; kb < pre_kb; kb++)
#pragma unroll
      for (int t = 0; t < kA; t++) x8_prefetch_2d(&wmap, kb * 128, e * rows_w + (t == 0 ? 0 : I) + blk * 128);
  }
  pdl_wait();

  if (warp < kX8Prep) {
    // token tiles: thread (row r, 16-element chunk c) of every k-block
    const int r = threadIdx.x >> 3, c = threadIdx.x & 7;
    int g = 0, it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const int e = item / nblk, blk = item % nblk, off = slot_off[e], n = slot_off[e + 1] - off;
      if (n == 0) continue;
      if (threadIdx.x == 0 && n > 32) atomicOr(status, SM100_DECODE_ERR_ARG);   // tokens past 32 are not served
      const int a = it & 1;
      const float *se = sc + (int64_t)e * s_stride;
      // block scales of the item's row blocks: lane l holds k-block l's
      float sl[kA], mt[kA];
#pragma unroll
      for (int t = 0; t < kA; t++) {
        sl[t] = lane < nkb ? se[(((t == 0 ? 0 : I) + blk * 128) / 128) * sc_cols + lane] : 0.0f;
        mt[t] = warp_max(sl[t]);
      }
      const int64_t src = r < n ? (kUp ? (int64_t)slot_tok[off + r] : (int64_t)(off + r)) : -1;
      const __nv_bfloat16 *xr = xin + (src >= 0 ? src : 0) * K + c * 16;
      // the token's largest |x| (the 8 threads of a row share it)
      float am = 0.0f;
      if (src >= 0) {
#pragma unroll 4
        for (int k = 0; k < K; k += 128) {
          am = fmaxf(am, x8_absmax8(*reinterpret_cast<const uint4 *>(xr + k)));
          am = fmaxf(am, x8_absmax8(*reinterpret_cast<const uint4 *>(xr + k + 8)));
        }
      }
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
      float inv[kA];
#pragma unroll
      for (int t = 0; t < kA; t++) inv[t] = x8_pow2(am * mt[t]);
      // the epilogue has read this accumulator set's previous scales
      if (it >= 2 && !__all_sync(0xffffffffu, mbar_wait(&acc_empty[a], (uint32_t)(((it >> 1) - 1) & 1), status))) {
        ok = false;
        break;
      }
      if (c == 0)
#pragma unroll
        for (int t = 0; t < kA; t++) sout[(a * kA + t) * 32 + r] = 1.0f / inv[t];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_full[a]);
      uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0, n0 = x0, n1 = x0;
      if (src >= 0) {
        x0 = *reinterpret_cast<const uint4 *>(xr);
        x1 = *reinterpret_cast<const uint4 *>(xr + 8);
      }
      for (int kb = 0; kb < nkb; kb++, g++) {
        const int s = g % kS;
        if (src >= 0 && kb + 1 < nkb) {   // the next k-block's chunk is requested before this one is split
          n0 = *reinterpret_cast<const uint4 *>(xr + (kb + 1) * 128);
          n1 = *reinterpret_cast<const uint4 *>(xr + (kb + 1) * 128 + 8);
        }
        if (g >= kS && !__all_sync(0xffffffffu, mbar_wait(&empty[s], (uint32_t)(((g / kS) - 1) & 1), status))) {
          ok = false;
          break;
        }
        unsigned char *bt = smem + s * kStage + kA * kX8A;
        const int o16 = r * 128 + ((c ^ (r & 7)) * 16);
#pragma unroll
        for (int t = 0; t < kA; t++) {
          uint4 hi, lo;
          x8_split16(x0, x1, __shfl_sync(0xffffffffu, sl[t], kb) * inv[t], hi, lo);
          *reinterpret_cast<uint4 *>(bt + (2 * t) * kX8B + o16) = hi;
          *reinterpret_cast<uint4 *>(bt + (2 * t + 1) * kX8B + o16) = lo;
        }
        x0 = n0;
        x1 = n1;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_b[s]);
      }
      it++;
    }
  } else if (warp == kX8Tma) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int e = item / nblk, blk = item % nblk;
        if (slot_off[e + 1] == slot_off[e]) continue;
        for (int kb = 0; kb < nkb; kb++, g++) {
          const int s = g % kS;
          if (g >= kS && !mbar_wait(&empty[s], (uint32_t)(((g / kS) - 1) & 1), status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full_a[s], kA * kX8A);
#pragma unroll
          for (int t = 0; t < kA; t++)
            x8_tma_2d(smem + s * kStage + t * kX8A, &wmap, kb * 128, e * rows_w + (t == 0 ? 0 : I) + blk * 128,
                      &full_a[s]);
        }
      }
      // the copies of the last use of each stage have landed before the CTA exits
      for (int j = max(g - kS, 0); j < g; j++) mbar_wait(&full_a[j % kS], (uint32_t)((j / kS) & 1), status, false);
    }
  } else if (warp == kX8Mma) {
    if (lane == 0) {
      // f32 accumulate, A and B e4m3, K-major, M = 128, N = 64: the hi and lo
      // token tiles are adjacent 32-row K-major tiles, one 64-row operand, so
      // one product gives hi in columns [0, 32) and lo in [32, 64)
      constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
      int g = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int e = item / nblk, n = slot_off[e + 1] - slot_off[e];
        if (n == 0) continue;
        const int a = it & 1;
        if (it >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)(((it >> 1) - 1) & 1), status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int kb = 0; kb < nkb; kb++, g++) {
          const int s = g % kS;
          if (!mbar_wait(&full_a[s], (uint32_t)((g / kS) & 1), status) ||
              !mbar_wait(&full_b[s], (uint32_t)((g / kS) & 1), status)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          // one shared-memory descriptor per stage; a tile's is the stage's
          // plus its byte offset / 16 in the 14-bit address field (the
          // stages lie below 256 KB, so the field cannot carry over)
          const uint64_t da = x8_desc(smem + s * kStage), db = da + (uint64_t)((kA * kX8A) >> 4);
#pragma unroll
          for (int t = 0; t < kA; t++) {
            const uint64_t at = da + (uint64_t)((t * kX8A) >> 4), bt = db + (uint64_t)((2 * t * kX8B) >> 4);
            asm volatile(
                "{\n\t.reg .pred q, pt;\n\t"
                "setp.ne.b32 q, %4, 0;\n\t"
                "setp.eq.b32 pt, 0, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, q;\n\t"
                "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %5, %6, %3, pt;\n\t"
                "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %7, %8, %3, pt;\n\t"
                "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %9, %10, %3, pt;\n\t}" ::"r"(tmem +
                                                                                     (uint32_t)(a * 128 + t * 64)),
                "l"(at), "l"(bt), "r"(idesc), "r"(kb > 0 ? 1u : 0u), "l"(at + 2), "l"(bt + 2), "l"(at + 4), "l"(bt + 4),
                "l"(at + 6), "l"(bt + 6)
                : "memory");
          }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&empty[s]))
                       : "memory");
        }
        if (!ok) break;
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&acc_full[a]))
                     : "memory");
        it++;
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(done))
                   : "memory");
    }
  } else {
    // epilogue: warp % 4 = TMEM lane quarter = row quarter of the block
    const int q = warp & 3, row = q * 32 + lane;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    int it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int e = item / nblk, blk = item % nblk, off = slot_off[e], n = slot_off[e + 1] - off;
      if (n == 0) continue;
      const int a = it & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[a], (uint32_t)((it >> 1) & 1), status))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // the token scales of this set (written before the set's first k-block)
      const bool sok = __all_sync(0xffffffffu, mbar_wait(&sc_full[a], (uint32_t)((it >> 1) & 1), status));
      // tile t's 64 columns: hi in [0, 32), lo in [32, 64); their sum is the product
      float f0[32], f1[32];
#pragma unroll
      for (int t = 0; t < kA; t++) {
        uint32_t vh[32], vl[32];
        x8_tmem_ld32(tq + (uint32_t)(a * 128 + t * 64), vh);
        x8_tmem_ld32(tq + (uint32_t)(a * 128 + t * 64 + 32), vl);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float *f = t == 0 ? f0 : f1;
#pragma unroll
        for (int c = 0; c < 32; c++)
          f[c] = (__uint_as_float(vh[c]) + __uint_as_float(vl[c])) * sout[(a * kA + t) * 32 + c];
      }
      if (!kUp)
#pragma unroll
        for (int c = 0; c < 32; c++) f1[c] = 0.0f;
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      if (!sok) break;
      const int r = blk * 128 + row;
      if (kUp) {
        __nv_bfloat16 *ao = reinterpret_cast<__nv_bfloat16 *>(out);
#pragma unroll
        for (int s = 0; s < 32; s++) {
          if (s >= n) continue;
          ao[(int64_t)(off + s) * I + r] = __float2bfloat16_rn(f0[s] / (1.0f + expf(-f0[s])) * f1[s]);
        }
      } else {
        float *y = reinterpret_cast<float *>(out);
#pragma unroll
        for (int s = 0; s < 32; s++) {
          if (s >= n) continue;
          atomicAdd(y + (int64_t)slot_tok[off + s] * D + r, slot_w[off + s] * f0[s]);
        }
      }
      it++;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kX8Mma) {
    if (lane == 0) mbar_wait(done, 0, status, false);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
  }
}

typedef CUresult (*X8EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                               const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D map of the fp8 weights of all experts, [rows][K] bytes, box 128 x 128, 128-byte swizzle
static bool x8_map(CUtensorMap *m, const void *w, int64_t rows, int64_t K) {
  static X8EncodeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<X8EncodeFn>(p);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// a = bf16(silu(gu[:, :I]) * gu[:, I:]) for the dense MLP (f32 gate|up rows)
__global__ void ds_silu_mul_kernel(const float *gu, __nv_bfloat16 *a, int M, int I) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * I) return;
  const int64_t m = i / I, j = i % I;
  const float g = gu[m * 2 * I + j], u = gu[m * 2 * I + I + j];
  a[i] = __float2bfloat16_rn(g / (1.0f + expf(-g)) * u);
}

}  // namespace sm100

using namespace sm100;

#define DS_LAUNCH(name, ...)                                                                        \
  do {                                                                                              \
    const cudaError_t e_ = launch_pdl(__VA_ARGS__);                                                 \
    if (e_ != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, name ": %s", cudaGetErrorString(e_)); \
    return launch_status(name);                                                                     \
  } while (0)

extern "C" int sm100_ds_rmsnorm(const float *x, const float *g, void *y, int32_t M, int32_t D, float eps,
                                void *stream) {
  if (!x || !g || !y || M < 1 || D < 1) return sm100_set_error(SM100_ERR_ARG, "ds_rmsnorm: bad arguments");
  DS_LAUNCH("ds_rmsnorm", ds_rms_kernel, dim3(M), dim3(256), 0, (cudaStream_t)stream, x, g, (__nv_bfloat16 *)y, D,
            eps);
}

extern "C" int sm100_ds_embed(const void *emb, const int32_t *tok, float *h, int32_t B, int32_t V, int32_t D,
                              void *stream) {
  if (!emb || !tok || !h || B < 1 || V < 1 || D < 1) return sm100_set_error(SM100_ERR_ARG, "ds_embed: bad arguments");
  DS_LAUNCH("ds_embed", ds_embed_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, (const __nv_bfloat16 *)emb,
            tok, h, V, D);
}

static int qkv_post_rows(const float *q, const float *kva, int64_t ld, const float *g_kv, const float *cos_t,
                         const float *sin_t, const DsRows &rows, void *q_out, void *cache_c, void *cache_pe, int32_t B,
                         int32_t H, int32_t DN, int32_t DR, int32_t KV, int32_t ctx, float eps, void *stream) {
  if (!q || !kva || !g_kv || !cos_t || !sin_t || !rows.pos || !q_out || !cache_c || !cache_pe || B < 1 || H < 1 ||
      (DR & 1) || KV < 1 || ctx < 1 || rows.n_seq < 1)
    return sm100_set_error(SM100_ERR_ARG, "ds_qkv_post: bad arguments");
  DS_LAUNCH("ds_qkv_post", ds_qkv_post_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, q, kva, g_kv, cos_t,
            sin_t, rows, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)cache_c, (__nv_bfloat16 *)cache_pe, H, DN, DR, KV,
            ctx, eps, ld);
}

extern "C" int sm100_ds_qkv_post(const float *q, const float *kva, int64_t ld, const float *g_kv, const float *cos_t,
                                 const float *sin_t, const int32_t *pos, void *q_out, void *cache_c, void *cache_pe,
                                 int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t KV, int32_t ctx, float eps,
                                 void *stream) {
  return qkv_post_rows(q, kva, ld, g_kv, cos_t, sin_t, DsRows{pos, nullptr, 0, B}, q_out, cache_c, cache_pe, B, H, DN,
                       DR, KV, ctx, eps, stream);
}

// The group kernel's launch: sequences per CTA the most (fewer re-reads of
// the head's W_uk / W_uv) that still gives the grid at least 96 CTAs, so a
// tensor-parallel rank with few heads still spreads its cache walks over the
// SMs.
template <bool kPost>
static int mla_group_launch(const void *q_out, const void *w_uk, const void *w_uv, void *cache_c, void *cache_pe,
                            const DsRows &rows, void *o, int32_t B, int32_t H, int32_t DN, int32_t DV, int32_t ctx,
                            float scale, const MlaPost &post, void *stream) {
  const int nb = H * ((B + 3) / 4) >= 96 ? 4 : H * ((B + 1) / 2) >= 96 ? 2 : 1;
  static bool attr[3] = {false, false, false};
  const int ai = nb == 4 ? 2 : nb == 2 ? 1 : 0;
  if (!attr[ai]) {
    const void *fn = nb == 4   ? (const void *)ds_mla_group_kernel<4, kPost>
                     : nb == 2 ? (const void *)ds_mla_group_kernel<2, kPost>
                               : (const void *)ds_mla_group_kernel<1, kPost>;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MlaSmem::total);
    if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "ds_mla: smem attribute: %s", cudaGetErrorString(e));
    attr[ai] = true;
  }
#define DS_MLA_GROUP(NBV)                                                                                           \
  DS_LAUNCH("ds_mla", (ds_mla_group_kernel<NBV, kPost>), dim3(H * ((B + NBV - 1) / NBV)), dim3(kMlaWarps * 32),     \
            MlaSmem::total, (cudaStream_t)stream, (const __nv_bfloat16 *)q_out, (const __nv_bfloat16 *)w_uk,        \
            (const __nv_bfloat16 *)w_uv, (__nv_bfloat16 *)cache_c, (__nv_bfloat16 *)cache_pe, rows,                  \
            (__nv_bfloat16 *)o, B, H, DN, DV, ctx, scale, post)
  if (nb == 4) DS_MLA_GROUP(4);
  if (nb == 2) DS_MLA_GROUP(2);
  DS_MLA_GROUP(1);
#undef DS_MLA_GROUP
}

static bool mla_group_shape(int32_t DN, int32_t DR, int32_t DV, int32_t KV) {
  return KV == kMlaKV && DR == kMlaDR && DN <= kMlaMaxD && DV <= kMlaMaxD;
}

static int mla_rows(const void *q_out, const void *w_uk, const void *w_uv, const void *cache_c, const void *cache_pe,
                    const DsRows &rows, void *o, int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t DV, int32_t KV,
                    int32_t ctx, float scale, void *stream) {
  if (!q_out || !w_uk || !w_uv || !cache_c || !cache_pe || !rows.pos || !o || B < 1 || H < 1 || DN > 256 ||
      DR > 128 || KV > kDsKV || ctx > kDsMaxCtx || rows.n_seq < 1)
    return sm100_set_error(SM100_ERR_ARG, "ds_mla: bad arguments (DN <= 256, DR <= 128, KV <= %d, ctx <= %d)",
                           kDsKV, kDsMaxCtx);
  if (mla_group_shape(DN, DR, DV, KV))
    return mla_group_launch<false>(q_out, w_uk, w_uv, (void *)cache_c, (void *)cache_pe, rows, o, B, H, DN, DV, ctx,
                                   scale, MlaPost{}, stream);
  DS_LAUNCH("ds_mla", ds_mla_kernel, dim3(B * H), dim3(256), 0, (cudaStream_t)stream, (const __nv_bfloat16 *)q_out,
            (const __nv_bfloat16 *)w_uk, (const __nv_bfloat16 *)w_uv, (const __nv_bfloat16 *)cache_c,
            (const __nv_bfloat16 *)cache_pe, rows, (__nv_bfloat16 *)o, H, DN, DR, DV, KV, ctx, scale);
}

extern "C" int sm100_ds_mla(const void *q_out, const void *w_uk, const void *w_uv, const void *cache_c,
                            const void *cache_pe, const int32_t *pos, void *o, int32_t B, int32_t H, int32_t DN,
                            int32_t DR, int32_t DV, int32_t KV, int32_t ctx, float scale, void *stream) {
  return mla_rows(q_out, w_uk, w_uv, cache_c, cache_pe, DsRows{pos, nullptr, 0, B}, o, B, H, DN, DR, DV, KV, ctx,
                  scale, stream);
}

// one_launch: the fused group kernel, whose CTAs walk their own rows' new
// cache rows from shared memory; otherwise the two launches (every row's
// cache append completes before any walk starts)
static int mla_post_rows(const float *qkva, int64_t ld, int64_t kva_off, const float *g_kv, const float *cos_t,
                         const float *sin_t, const DsRows &rows, bool one_launch, void *q_out, const void *w_uk,
                         const void *w_uv, void *cache_c, void *cache_pe, void *o, int32_t B, int32_t H, int32_t DN,
                         int32_t DR, int32_t DV, int32_t KV, int32_t ctx, float eps, float scale, void *stream) {
  if (!qkva || !g_kv || !cos_t || !sin_t || !rows.pos || !q_out || !w_uk || !w_uv || !cache_c || !cache_pe || !o ||
      B < 1 || H < 1 || kva_off < (int64_t)H * (DN + DR) || ld < kva_off + KV + DR || rows.n_seq < 1)
    return sm100_set_error(SM100_ERR_ARG, "ds_mla_post: bad arguments");
  if (!one_launch || !mla_group_shape(DN, DR, DV, KV) || ctx > kDsMaxCtx) {   // the two launches it fuses
    int rc = qkv_post_rows(qkva, qkva + kva_off, ld, g_kv, cos_t, sin_t, rows, q_out, cache_c, cache_pe, B, H, DN, DR,
                           KV, ctx, eps, stream);
    if (rc != SM100_OK) return rc;
    return mla_rows(q_out, w_uk, w_uv, cache_c, cache_pe, rows, o, B, H, DN, DR, DV, KV, ctx, scale, stream);
  }
  const MlaPost post{qkva, ld, kva_off, g_kv, cos_t, sin_t, eps};
  return mla_group_launch<true>(q_out, w_uk, w_uv, cache_c, cache_pe, rows, o, B, H, DN, DV, ctx, scale, post, stream);
}

extern "C" int sm100_ds_mla_post(const float *qkva, int64_t ld, int64_t kva_off, const float *g_kv, const float *cos_t,
                                 const float *sin_t, const int32_t *pos, void *q_out, const void *w_uk,
                                 const void *w_uv, void *cache_c, void *cache_pe, void *o, int32_t B, int32_t H,
                                 int32_t DN, int32_t DR, int32_t DV, int32_t KV, int32_t ctx, float eps, float scale,
                                 void *stream) {
  return mla_post_rows(qkva, ld, kva_off, g_kv, cos_t, sin_t, DsRows{pos, nullptr, 0, B}, true, q_out, w_uk, w_uv,
                       cache_c, cache_pe, o, B, H, DN, DR, DV, KV, ctx, eps, scale, stream);
}

extern "C" int sm100_ds_mla_post_rows(const float *qkva, int64_t ld, int64_t kva_off, const float *g_kv,
                                      const float *cos_t, const float *sin_t, const Sm100DsRows *rows, void *q_out,
                                      const void *w_uk, const void *w_uv, void *cache_c, void *cache_pe, void *o,
                                      int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t DV, int32_t KV, int32_t ctx,
                                      float eps, float scale, void *stream) {
  if (!rows || !rows->pos || !rows->seq || rows->n_seq < 1)
    return sm100_set_error(SM100_ERR_ARG, "ds_mla_post_rows: rows need pos, seq and n_seq >= 1");
  return mla_post_rows(qkva, ld, kva_off, g_kv, cos_t, sin_t, DsRows{rows->pos, rows->seq, 1, rows->n_seq},
                       rows->shared_slots == 0, q_out, w_uk, w_uv, cache_c, cache_pe, o, B, H, DN, DR, DV, KV, ctx, eps,
                       scale, stream);
}

extern "C" int sm100_ds_route(const float *logits, int32_t E, int32_t K, int32_t B, int32_t e0, int32_t e1,
                              int32_t n_shared, int32_t *sel, float *wsel, int32_t *slot_off, int32_t *slot_tok,
                              float *slot_w, void *stream) {
  if (!logits || !sel || !wsel || !slot_off || !slot_tok || !slot_w || E < 1 || E > 64 || K < 1 || K > kDsMaxK ||
      K > E || B < 1 || B > kDsMaxTok || e0 < 0 || e1 > E || e0 > e1 || n_shared < 0 || n_shared > 8)
    return sm100_set_error(SM100_ERR_ARG, "ds_route: E %d K %d B %d [%d, %d)", E, K, B, e0, e1);
  DS_LAUNCH("ds_route", ds_route_kernel, dim3(1), dim3(1024), 0, (cudaStream_t)stream, logits, E, K, B, e0, e1,
            n_shared, sel, wsel, slot_off, slot_tok, slot_w);
}

extern "C" int sm100_ds_router_route(const void *x, const void *router, float *logits, int32_t *counter, int32_t D,
                                     int32_t E, int32_t K, int32_t B, int32_t e0, int32_t e1, int32_t n_shared,
                                     int32_t *sel, float *wsel, int32_t *slot_off, int32_t *slot_tok, float *slot_w,
                                     void *stream) {
  if (!x || !router || !logits || !counter || !sel || !wsel || !slot_off || !slot_tok || !slot_w || E < 1 ||
      E > 64 || K < 1 || K > kDsMaxK || K > E || B < 1 || B > kDsMaxTok || e0 < 0 || e1 > E || e0 > e1 ||
      n_shared < 0 || n_shared > 8 || D < 8 || D % 8 || ((uintptr_t)x | (uintptr_t)router) % 16)
    return sm100_set_error(SM100_ERR_ARG, "ds_router_route: D %d E %d K %d B %d [%d, %d)", D, E, K, B, e0, e1);
  DS_LAUNCH("ds_router_route", ds_router_route_kernel, dim3(E), dim3(1024), 0, (cudaStream_t)stream,
            (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)router, logits, counter, D, E, K, B, e0, e1, n_shared,
            sel, wsel, slot_off, slot_tok, slot_w);
}

extern "C" int sm100_ds_experts(const void *x, const void *w_gu, const float *s_gu, const void *w_d, const float *s_d,
                                const int32_t *slot_off, const int32_t *slot_tok, const float *slot_w, void *a_scratch,
                                float *y, int32_t n_exp, int32_t D, int32_t I, void *stream) {
  if (!x || !w_gu || !s_gu || !w_d || !s_d || !slot_off || !slot_tok || !slot_w || !a_scratch || !y || n_exp < 1 ||
      D % 128 || I % 128 || D < 128 || I < 128 || D > 128 * kX8MaxKb || I > 128 * kX8MaxKb ||
      ((uintptr_t)w_gu & 15) || ((uintptr_t)w_d & 15) || ((uintptr_t)x & 15) || ((uintptr_t)a_scratch & 15))
    return sm100_set_error(SM100_ERR_ARG,
                           "ds_experts: n_exp %d D %d I %d (D, I multiples of 128 up to %d; 16-byte aligned operands)",
                           n_exp, D, I, 128 * kX8MaxKb);
  const int64_t sc_gu = (int64_t)(2 * I / 128) * (D / 128), sc_d = (int64_t)(D / 128) * (I / 128);
  CUtensorMap map_gu, map_d;
  if (!x8_map(&map_gu, w_gu, (int64_t)n_exp * 2 * I, D) || !x8_map(&map_d, w_d, (int64_t)n_exp * D, I))
    return sm100_set_error(SM100_ERR_CUDA, "ds_experts: tensor map encoding failed");
  constexpr int smem_up = x8_smem<true>(), smem_dn = x8_smem<false>();
  static bool attr[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sm100_set_error(SM100_ERR_ARG, "ds_experts: device %d", dev);
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(ds_x8_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_up);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ds_x8_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dn);
    if (e != cudaSuccess)
      return sm100_set_error(SM100_ERR_CUDA, "ds_experts: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  const int items_up = n_exp * (I / 128), items_dn = n_exp * (D / 128);
  cudaError_t e = launch_pdl(ds_x8_kernel<true>, dim3(std::min(items_up, 148)), dim3(kX8Threads), smem_up,
                             (cudaStream_t)stream, map_gu, (const __nv_bfloat16 *)x, s_gu, slot_off, slot_tok, slot_w,
                             a_scratch, D, I, sc_gu, n_exp);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "ds_experts: up: %s", cudaGetErrorString(e));
  const int rc = launch_status("ds_expert_up");
  if (rc != SM100_OK) return rc;
  e = launch_pdl(ds_x8_kernel<false>, dim3(std::min(items_dn, 148)), dim3(kX8Threads), smem_dn, (cudaStream_t)stream,
                 map_d, (const __nv_bfloat16 *)a_scratch, s_d, slot_off, slot_tok, slot_w, (void *)y, D, I, sc_d,
                 n_exp);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "ds_experts: down: %s", cudaGetErrorString(e));
  return launch_status("ds_expert_down");
}

extern "C" uint32_t sm100_ds_status(void) {
  uint32_t v = 0, z = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_ds_status, sizeof(v));
  cudaMemcpyToSymbol(g_ds_status, &z, sizeof(z));
  return v;
}

extern "C" int sm100_ds_silu_mul(const float *gu, void *a, int32_t M, int32_t I, void *stream) {
  if (!gu || !a || M < 1 || I < 1) return sm100_set_error(SM100_ERR_ARG, "ds_silu_mul: bad arguments");
  const int64_t n = (int64_t)M * I;
  DS_LAUNCH("ds_silu_mul", ds_silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
            gu, (__nv_bfloat16 *)a, M, I);
}
