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
#include <cuda_fp8.h>

#include <algorithm>

#include "common.cuh"

namespace sm100 {

constexpr int kDsMaxTok = 32;     // decode batch
constexpr int kDsMaxK = 8;        // experts per token
constexpr int kDsMaxCtx = 2048;

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// y = bf16(x * rsqrt(mean(x^2) + eps) * g) per row (RMSNorm, deepseek_v2.py's
// RMSNorm as the reference folds it, dsv2_decode_bench.c:341-430).
__global__ void __launch_bounds__(256) ds_rms_kernel(const float *x, const float *g, __nv_bfloat16 *y, int D,
                                                      float eps) {
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const float *xr = x + (int64_t)blockIdx.x * D;
  float s = 0.0f;
  for (int i = threadIdx.x; i < D; i += 256) s += xr[i] * xr[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) t += red[w];
  const float inv = 1.0f / sqrtf(t * (1.0f / (float)D) + eps);
  for (int i = threadIdx.x; i < D; i += 256)
    y[(int64_t)blockIdx.x * D + i] = __float2bfloat16_rn((xr[i] * inv) * g[i]);
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
                                                           const float *cs, const float *sn, const int32_t *pos,
                                                           __nv_bfloat16 *qo, __nv_bfloat16 *cc, __nv_bfloat16 *cpe,
                                                           int H, int DN, int DR, int KV, int ctx, float eps,
                                                           int64_t ld) {
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, p = *pos, half = DR / 2, QS = DN + DR;
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
    qob[h * QS + DN + j] = __float2bfloat16_rn(xe * c - xo * s);
    qob[h * QS + DN + half + j] = __float2bfloat16_rn(xo * c + xe * s);
  }
  const float *kb = kva + (int64_t)b * ld;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < KV; i += 256) {
    const float v = bfr(kb[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) t += red[w];
  const float inv = 1.0f / sqrtf(t * (1.0f / (float)KV) + eps);
  __nv_bfloat16 *crow = cc + ((int64_t)b * ctx + p) * KV;
  for (int i = threadIdx.x; i < KV; i += 256) crow[i] = __float2bfloat16_rn((bfr(kb[i]) * inv) * g_kv[i]);
  __nv_bfloat16 *prow = cpe + ((int64_t)b * ctx + p) * DR;
  for (int j = threadIdx.x; j < half; j += 256) {
    const float xe = bfr(kb[KV + 2 * j]), xo = bfr(kb[KV + 2 * j + 1]);
    const float c = cs[(int64_t)p * DR + j], s = sn[(int64_t)p * DR + j];
    prow[j] = __float2bfloat16_rn(xe * c - xo * s);
    prow[half + j] = __float2bfloat16_rn(xo * c + xe * s);
  }
}

// Absorbed MLA of one (token b, head h): qlat = W_uk[h]^T q_nope (KV), scores
// over cache rows 0..pos = (qlat . c_t + q_pe . pe_t) * scale, softmax,
// olat = sum_t p_t c_t, o = bf16(W_uv[h] olat) (DV).  W_uk / W_uv [H][DN or
// DV][KV] bf16 (kv_b_proj split, deepseek_v2.py's absorb).
constexpr int kDsKV = 512;
__global__ void __launch_bounds__(256) ds_mla_kernel(const __nv_bfloat16 *qo, const __nv_bfloat16 *wuk,
                                                      const __nv_bfloat16 *wuv, const __nv_bfloat16 *cc,
                                                      const __nv_bfloat16 *cpe, const int32_t *pos, __nv_bfloat16 *o,
                                                      int H, int DN, int DR, int DV, int KV, int ctx, float scale) {
  __shared__ float qlat[kDsKV];
  __shared__ float qn[256];
  __shared__ float qpe[128];
  __shared__ float sc[kDsMaxCtx];
  __shared__ float olat[kDsKV];
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x / H, h = blockIdx.x % H, QS = DN + DR, T = *pos + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
  const __nv_bfloat16 *cb = cc + (int64_t)b * ctx * KV, *pb = cpe + (int64_t)b * ctx * DR;
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

// Routing of every token (one CTA, a warp per token): probs = softmax(logits)
// (max, exp, sum, divide), the K largest probs (ties: lowest expert id), no
// renormalisation (DeepSeek-V2-Lite: norm_topk_prob false, scaling 1);
// then per-expert lists of (token, weight) for the experts [e0, e1) this
// rank holds, packed expert-major: slot_tok / slot_w / slot_off[e] offsets,
// followed by n_shared shared experts that take every token with weight 1.
__global__ void __launch_bounds__(1024) ds_route_kernel(const float *logits, int E, int K, int B, int e0, int e1,
                                                         int n_shared, int32_t *sel, float *wsel, int32_t *slot_off,
                                                         int32_t *slot_tok, float *slot_w) {
  __shared__ int s_sel[kDsMaxTok * kDsMaxK];
  __shared__ float s_w[kDsMaxTok * kDsMaxK];
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int b = warp; b < B; b += 32) {
    const float *lg = logits + (int64_t)b * E;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e]);
    m = warp_max(m);
    float sum = 0.0f;
    for (int e = lane; e < E; e += 32) sum += expf(lg[e] - m);
    sum = warp_sum(sum);
    // greedy top-K over E <= 64 probabilities held two per lane
    float p0 = lane < E ? expf(lg[lane] - m) / sum : -1.0f;
    float p1 = lane + 32 < E ? expf(lg[lane + 32] - m) / sum : -1.0f;
    for (int k = 0; k < K; k++) {
      float bv = p0 >= p1 ? p0 : p1;
      int bi = p0 >= p1 ? lane : lane + 32;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        s_sel[b * K + k] = bi;
        s_w[b * K + k] = bv;
        sel[b * K + k] = bi;
        wsel[b * K + k] = bv;
      }
      if (bi == lane) p0 = -2.0f;
      if (bi == lane + 32) p1 = -2.0f;
    }
  }
  __syncthreads();
  // expert-major packing: thread e counts its slots, a scan gives the offsets,
  // then it lists its tokens in order
  __shared__ int cnt[64];
  const int ne = e1 - e0;
  if (threadIdx.x < 64) {
    int c = 0;
    if ((int)threadIdx.x < ne)
      for (int i = 0; i < B * K; i++) c += (s_sel[i] == e0 + (int)threadIdx.x);
    cnt[threadIdx.x] = c;
  }
  __syncthreads();
  if (threadIdx.x < 64 && (int)threadIdx.x < ne) {
    int o = 0;
    for (int i = 0; i < (int)threadIdx.x; i++) o += cnt[i];
    slot_off[threadIdx.x] = o;
    if ((int)threadIdx.x == ne - 1) slot_off[ne] = o + cnt[threadIdx.x];
    for (int i = 0; i < B * K; i++)
      if (s_sel[i] == e0 + (int)threadIdx.x) {
        slot_tok[o] = i / K;
        slot_w[o] = s_w[i];
        o++;
      }
  }
  if (ne == 0 && threadIdx.x == 0) slot_off[0] = 0;
  // the shared experts (local ids ne ..) take every token with weight 1
  __syncthreads();
  if (n_shared > 0) {
    for (int i = threadIdx.x; i < n_shared * B; i += blockDim.x) {
      const int k = i / B, b = i % B, o = slot_off[ne] + i;
      slot_tok[o] = b;
      slot_w[o] = 1.0f;
      if (b == 0) slot_off[ne + k + 1] = slot_off[ne] + (k + 1) * B;
    }
  }
}

// 16 fp8-e4m3 codes -> f32 times a block scale (hardware e4m3x2 -> f16x2
// conversions; f16 holds every e4m3 value exactly).
__device__ __forceinline__ void fp8x16(const uint4 w, float sc, float (&f)[16]) {
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; q++) {
#pragma unroll
    for (int hlf = 0; hlf < 2; hlf++) {
      const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)((ww[q] >> (16 * hlf)) & 0xFFFFu);
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3);
      const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
      f[4 * q + 2 * hlf] = v.x * sc;
      f[4 * q + 2 * hlf + 1] = v.y * sc;
    }
  }
}

constexpr int kDsRows = 32;      // weight rows per work item
constexpr int kDsTokChunk = 8;   // tokens staged in shared memory at a time

// Experts, phase 1 (persistent, grid-stride over work items (expert e, block
// of 32 rows); an expert without tokens costs one read of its slot count):
// a[slot][j] = bf16(silu(x . gate_j) * (x . up_j)) for the expert's tokens,
// gate / up fp8 rows [2I][D] with f32 scales [ceil(2I/128)][D/128].  Tokens
// are staged 8 at a time in shared memory; a warp per row pair, lanes over
// D in 16-byte fp8 chunks.
__global__ void __launch_bounds__(256) ds_expert_up_kernel(const __nv_bfloat16 *x, const uint8_t *wgu,
                                                            const float *sgu, const int32_t *slot_off,
                                                            const int32_t *slot_tok, __nv_bfloat16 *a, int D, int I,
                                                            int64_t w_stride, int64_t s_stride, int n_exp) {
  extern __shared__ __nv_bfloat16 xs[];   // [kDsTokChunk][D]
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, rb_n = (I + kDsRows - 1) / kDsRows;
  const int sc_cols = D / 128;
  for (int item = blockIdx.x; item < n_exp * rb_n; item += gridDim.x) {
    const int e = item / rb_n, rb = item % rb_n, off = slot_off[e], n = slot_off[e + 1] - off;
    if (n == 0) continue;
    const uint8_t *we = wgu + (int64_t)e * w_stride;
    const float *se = sgu + (int64_t)e * s_stride;
    for (int t0 = 0; t0 < n; t0 += kDsTokChunk) {
      const int nt = min(kDsTokChunk, n - t0);
      __syncthreads();   // the previous chunk's readers are done
      for (int i = threadIdx.x; i < nt * D / 8; i += 256) {
        const int s = i / (D / 8), c = i % (D / 8);
        reinterpret_cast<uint4 *>(xs)[(int64_t)s * (D / 8) + c] =
            reinterpret_cast<const uint4 *>(x + (int64_t)slot_tok[off + t0 + s] * D)[c];
      }
      __syncthreads();
      for (int r = warp; r < kDsRows; r += 8) {
        const int j = rb * kDsRows + r;
        if (j >= I) break;
        float g[kDsTokChunk], u[kDsTokChunk];
#pragma unroll
        for (int s = 0; s < kDsTokChunk; s++) g[s] = u[s] = 0.0f;
        for (int k0 = lane * 16; k0 < D; k0 += 512) {
          float fg[16], fu[16];
          fp8x16(*reinterpret_cast<const uint4 *>(we + (int64_t)j * D + k0), se[(j / 128) * sc_cols + k0 / 128], fg);
          fp8x16(*reinterpret_cast<const uint4 *>(we + (int64_t)(I + j) * D + k0),
                 se[((I + j) / 128) * sc_cols + k0 / 128], fu);
#pragma unroll
          for (int s = 0; s < kDsTokChunk; s++) {
            if (s >= nt) continue;
            const uint4 *xr = reinterpret_cast<const uint4 *>(xs + (int64_t)s * D + k0);
            float ag = 0.0f, au = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const uint4 xv = xr[h];
              const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
              for (int q = 0; q < 4; q++) {
                const float x0 = __uint_as_float(xw[q] << 16), x1 = __uint_as_float(xw[q] & 0xFFFF0000u);
                ag = fmaf(fg[8 * h + 2 * q], x0, fmaf(fg[8 * h + 2 * q + 1], x1, ag));
                au = fmaf(fu[8 * h + 2 * q], x0, fmaf(fu[8 * h + 2 * q + 1], x1, au));
              }
            }
            g[s] += ag;
            u[s] += au;
          }
        }
#pragma unroll
        for (int s = 0; s < kDsTokChunk; s++) {
          if (s >= nt) continue;
          const float gs = warp_sum(g[s]), us = warp_sum(u[s]);
          if (lane == 0) a[(int64_t)(off + t0 + s) * I + j] = __float2bfloat16_rn(gs / (1.0f + expf(-gs)) * us);
        }
      }
    }
  }
}

// Experts, phase 2 (persistent over (expert, block of 32 output rows)):
// y[tok][r] += w_slot * sum_j a[slot][j] W_d[e][r][j] (fp8 [D][I], scales
// [D/128][ceil(I/128)]); the experts of a token meet in y by float reductions.
__global__ void __launch_bounds__(256) ds_expert_down_kernel(const __nv_bfloat16 *a, const uint8_t *wd, const float *sd,
                                                              const int32_t *slot_off, const int32_t *slot_tok,
                                                              const float *slot_w, float *y, int D, int I,
                                                              int64_t w_stride, int64_t s_stride, int n_exp) {
  extern __shared__ __nv_bfloat16 as[];   // [kDsTokChunk][I]
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, rb_n = (D + kDsRows - 1) / kDsRows;
  const int sc_cols = (I + 127) / 128;
  for (int item = blockIdx.x; item < n_exp * rb_n; item += gridDim.x) {
    const int e = item / rb_n, rb = item % rb_n, off = slot_off[e], n = slot_off[e + 1] - off;
    if (n == 0) continue;
    for (int t0 = 0; t0 < n; t0 += kDsTokChunk) {
      const int nt = min(kDsTokChunk, n - t0);
      __syncthreads();
      for (int i = threadIdx.x; i < nt * I / 8; i += 256)
        reinterpret_cast<uint4 *>(as)[i] = reinterpret_cast<const uint4 *>(a + (int64_t)(off + t0) * I)[i];
      __syncthreads();
      for (int rr = warp; rr < kDsRows; rr += 8) {
        const int r = rb * kDsRows + rr;
        if (r >= D) break;
        const uint8_t *we = wd + (int64_t)e * w_stride + (int64_t)r * I;
        const float *se = sd + (int64_t)e * s_stride + (int64_t)(r / 128) * sc_cols;
        float acc[kDsTokChunk];
#pragma unroll
        for (int s = 0; s < kDsTokChunk; s++) acc[s] = 0.0f;
        for (int k0 = lane * 16; k0 < I; k0 += 512) {
          float f[16];
          fp8x16(*reinterpret_cast<const uint4 *>(we + k0), se[k0 / 128], f);
#pragma unroll
          for (int s = 0; s < kDsTokChunk; s++) {
            if (s >= nt) continue;
            const uint4 *ar = reinterpret_cast<const uint4 *>(as + (int64_t)s * I + k0);
            float t = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const uint4 av = ar[h];
              const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
              for (int q = 0; q < 4; q++)
                t = fmaf(f[8 * h + 2 * q], __uint_as_float(aw[q] << 16),
                         fmaf(f[8 * h + 2 * q + 1], __uint_as_float(aw[q] & 0xFFFF0000u), t));
            }
            acc[s] += t;
          }
        }
#pragma unroll
        for (int s = 0; s < kDsTokChunk; s++) {
          if (s >= nt) continue;
          const float v = warp_sum(acc[s]);
          if (lane == 0) atomicAdd(y + (int64_t)slot_tok[off + t0 + s] * D + r, slot_w[off + t0 + s] * v);
        }
      }
    }
  }
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

extern "C" int sm100_ds_qkv_post(const float *q, const float *kva, int64_t ld, const float *g_kv, const float *cos_t,
                                 const float *sin_t, const int32_t *pos, void *q_out, void *cache_c, void *cache_pe,
                                 int32_t B, int32_t H, int32_t DN, int32_t DR, int32_t KV, int32_t ctx, float eps,
                                 void *stream) {
  if (!q || !kva || !g_kv || !cos_t || !sin_t || !pos || !q_out || !cache_c || !cache_pe || B < 1 || H < 1 ||
      (DR & 1) || KV < 1 || ctx < 1)
    return sm100_set_error(SM100_ERR_ARG, "ds_qkv_post: bad arguments");
  DS_LAUNCH("ds_qkv_post", ds_qkv_post_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, q, kva, g_kv, cos_t,
            sin_t, pos, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)cache_c, (__nv_bfloat16 *)cache_pe, H, DN, DR, KV,
            ctx, eps, ld);
}

extern "C" int sm100_ds_mla(const void *q_out, const void *w_uk, const void *w_uv, const void *cache_c,
                            const void *cache_pe, const int32_t *pos, void *o, int32_t B, int32_t H, int32_t DN,
                            int32_t DR, int32_t DV, int32_t KV, int32_t ctx, float scale, void *stream) {
  if (!q_out || !w_uk || !w_uv || !cache_c || !cache_pe || !pos || !o || B < 1 || H < 1 || DN > 256 || DR > 128 ||
      KV > kDsKV || ctx > kDsMaxCtx)
    return sm100_set_error(SM100_ERR_ARG, "ds_mla: bad arguments (DN <= 256, DR <= 128, KV <= %d, ctx <= %d)",
                           kDsKV, kDsMaxCtx);
  DS_LAUNCH("ds_mla", ds_mla_kernel, dim3(B * H), dim3(256), 0, (cudaStream_t)stream, (const __nv_bfloat16 *)q_out,
            (const __nv_bfloat16 *)w_uk, (const __nv_bfloat16 *)w_uv, (const __nv_bfloat16 *)cache_c,
            (const __nv_bfloat16 *)cache_pe, pos, (__nv_bfloat16 *)o, H, DN, DR, DV, KV, ctx, scale);
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

extern "C" int sm100_ds_experts(const void *x, const void *w_gu, const float *s_gu, const void *w_d, const float *s_d,
                                const int32_t *slot_off, const int32_t *slot_tok, const float *slot_w, void *a_scratch,
                                float *y, int32_t n_exp, int32_t D, int32_t I, void *stream) {
  if (!x || !w_gu || !s_gu || !w_d || !s_d || !slot_off || !slot_tok || !slot_w || !a_scratch || !y || n_exp < 1 ||
      D % 512 || I % 16 || D > 16384 || I > 16384)
    return sm100_set_error(SM100_ERR_ARG, "ds_experts: n_exp %d D %d I %d (D %% 512 == 0, I %% 16 == 0)", n_exp, D, I);
  const int64_t sc_gu = (int64_t)((2 * I + 127) / 128) * (D / 128), sc_d = (int64_t)(D / 128) * ((I + 127) / 128);
  const size_t smem_up = (size_t)kDsTokChunk * D * 2, smem_dn = (size_t)kDsTokChunk * I * 2;
  cudaError_t e = cudaFuncSetAttribute(ds_expert_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_up);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(ds_expert_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dn);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "ds_experts: smem attribute: %s", cudaGetErrorString(e));
  const int items_up = n_exp * ((I + kDsRows - 1) / kDsRows), items_dn = n_exp * ((D + kDsRows - 1) / kDsRows);
  e = launch_pdl(ds_expert_up_kernel, dim3(std::min(items_up, 4 * 148)), dim3(256), smem_up, (cudaStream_t)stream,
                 (const __nv_bfloat16 *)x, (const uint8_t *)w_gu, s_gu, slot_off, slot_tok, (__nv_bfloat16 *)a_scratch,
                 D, I, (int64_t)2 * I * D, sc_gu, n_exp);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "ds_experts: up: %s", cudaGetErrorString(e));
  launch_status("ds_expert_up");
  e = launch_pdl(ds_expert_down_kernel, dim3(std::min(items_dn, 4 * 148)), dim3(256), smem_dn, (cudaStream_t)stream,
                 (const __nv_bfloat16 *)a_scratch, (const uint8_t *)w_d, s_d, slot_off, slot_tok, slot_w, y, D, I,
                 (int64_t)D * I, sc_d, n_exp);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "ds_experts: down: %s", cudaGetErrorString(e));
  return launch_status("ds_expert_down");
}

extern "C" int sm100_ds_silu_mul(const float *gu, void *a, int32_t M, int32_t I, void *stream) {
  if (!gu || !a || M < 1 || I < 1) return sm100_set_error(SM100_ERR_ARG, "ds_silu_mul: bad arguments");
  const int64_t n = (int64_t)M * I;
  DS_LAUNCH("ds_silu_mul", ds_silu_mul_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
            gu, (__nv_bfloat16 *)a, M, I);
}
