// The prompt (prefill) pass of the batched GPT-2-XL-shaped decoder (BASELINE
// config 3): all P prompt positions of the B sequences go through each layer
// at once, so the projections are [B*P, K] x [N, K]^T products on the tensor
// cores (sm100_gemm_bf16_ep) and the causal attention is the flash-style
// tensor-core kernel (sm100_attn_prefill_bf16).  The reference runs the
// prompt as one forward of the whole [B, P] id tensor through the same
// Transformer (bench/gpt2/thvm_gpt2.py:98-128, start_pos 0), which writes the
// cache rows 0..P-1 and takes the next ids from the last position's logits.
//
// The kernels here are the glue between those products, all bandwidth-bound
// copies over 16-byte vectors:
//   xl_prefill_embed  h[b P + s] = wte[tok[b P + s]] + wpe[s];
//   xl_prefill_split  the bf16 qkv product rows -> q, k, v in the attention
//                     kernel's [B, H, P, 128] layout (head dimension 64 in
//                     the first half of each 128-wide row; the second half
//                     stays zero, so it adds nothing to q k^T and leaves the
//                     output's upper half zero) and k, v into cache rows
//                     0..P-1 ([2, B, ctx, C], as the decode step keeps it);
//   xl_prefill_merge  the attention output's first 64 columns per head ->
//                     bf16 [B P, C] rows (the next product's operand);
//   xl_prefill_ln     LayerNorm of the B P rows to the bf16 operand, a warp
//                     per row;
//   xl_prefill_last   h of each sequence's last position -> the decode
//                     step's [B, D] rows, and the cache position = P.
#include "common.cuh"

namespace sm100 {

constexpr int kXpHd = 64, kXpDp = 128;   // head dimension; the attention kernel's row width

__global__ void xl_prefill_embed_kernel(const __nv_bfloat16 *wte, const __nv_bfloat16 *wpe, const int32_t *tok,
                                        float *h, int P, int V, int D) {
  const int r = blockIdx.x, s = r % P, id = tok[r];
  const bool in = id >= 0 && id < V;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float e = in ? __bfloat162float(wte[(int64_t)id * D + d]) : 0.0f;
    h[(int64_t)r * D + d] = e + __bfloat162float(wpe[(int64_t)s * D + d]);
  }
}

// One CTA per product row r = b P + s; 8 bf16 (16 bytes) per step.  C is a
// multiple of 64, so no 8-column group crosses a head or a q / k / v third.
__global__ void xl_prefill_split_kernel(const __nv_bfloat16 *qkv, __nv_bfloat16 *q, __nv_bfloat16 *k,
                                        __nv_bfloat16 *v, __nv_bfloat16 *kv, int B, int P, int H, int ctx) {
  const int r = blockIdx.x, b = r / P, s = r % P, C = H * kXpHd;
  const uint4 *src = reinterpret_cast<const uint4 *>(qkv + (int64_t)r * 3 * C);
  for (int i = threadIdx.x; i < 3 * C / 8; i += blockDim.x) {
    const uint4 val = src[i];
    const int col = i * 8, part = col / C, c = col - part * C, hh = c / kXpHd, d = c - hh * kXpHd;
    __nv_bfloat16 *dst = part == 0 ? q : (part == 1 ? k : v);
    *reinterpret_cast<uint4 *>(dst + (((int64_t)b * H + hh) * P + s) * kXpDp + d) = val;
    if (part > 0)
      *reinterpret_cast<uint4 *>(kv + (((int64_t)(part - 1) * B + b) * ctx + s) * C + c) = val;
  }
}

// att[b P + s, h 64 + d] = bf16(o[b, h, s, d]), d < 64.
__global__ void xl_prefill_merge_kernel(const float *o, __nv_bfloat16 *att, int P, int H) {
  const int r = blockIdx.x, b = r / P, s = r % P, C = H * kXpHd;
  for (int i = threadIdx.x; i < C / 4; i += blockDim.x) {
    const int c = i * 4, hh = c / kXpHd, d = c - hh * kXpHd;
    const float4 t = *reinterpret_cast<const float4 *>(o + (((int64_t)b * H + hh) * P + s) * kXpDp + d);
    const __nv_bfloat162 lo = __floats2bfloat162_rn(t.x, t.y), hi = __floats2bfloat162_rn(t.z, t.w);
    uint2 w;
    w.x = *reinterpret_cast<const uint32_t *>(&lo);
    w.y = *reinterpret_cast<const uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(att + (int64_t)r * C + c) = w;
  }
}

// y = bf16(LayerNorm(x) * g + b) over the B P rows, one warp per row with
// the row in registers (one read of x; xl_ln_kernel's one-CTA-per-row form
// reads it three times and leaves the SMs mostly idle at these row counts).
// Mean and biased variance as sum * (1/D), 1/sqrt (src/nn/layernorm.c:1-7).
constexpr int kXpLnVec = 16;   // float4 per lane: D <= 16 * 128 = 2048

__global__ void __launch_bounds__(256) xl_prefill_ln_kernel(const float *x, const float *g, const float *bt,
                                                             __nv_bfloat16 *y, int M, int D, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)row * D);
  const int n4 = D / 4;
  float4 v[kXpLnVec];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < kXpLnVec; j++) {
    const int i = lane + 32 * j;
    v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  s = warp_sum(s);
  const float inv_n = 1.0f / (float)D, mean = s * inv_n;
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < kXpLnVec; j++) {
    if (lane + 32 * j < n4) {
      const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  q = warp_sum(q);
  const float r = 1.0f / sqrtf(q * inv_n + eps);
  const float4 *g4 = reinterpret_cast<const float4 *>(g), *b4 = reinterpret_cast<const float4 *>(bt);
  uint2 *yr = reinterpret_cast<uint2 *>(y + (int64_t)row * D);
#pragma unroll
  for (int j = 0; j < kXpLnVec; j++) {
    const int i = lane + 32 * j;
    if (i < n4) {
      const float4 gg = g4[i], bb = b4[i];
      const __nv_bfloat162 lo = __floats2bfloat162_rn((v[j].x - mean) * r * gg.x + bb.x,
                                                      (v[j].y - mean) * r * gg.y + bb.y);
      const __nv_bfloat162 hi = __floats2bfloat162_rn((v[j].z - mean) * r * gg.z + bb.z,
                                                      (v[j].w - mean) * r * gg.w + bb.w);
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t *>(&lo);
      w.y = *reinterpret_cast<const uint32_t *>(&hi);
      yr[i] = w;
    }
  }
}

__global__ void xl_prefill_last_kernel(const float *h, float *hl, int32_t *pos, int P, int D) {
  const int b = blockIdx.x;
  const float *src = h + ((int64_t)b * P + P - 1) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) hl[(int64_t)b * D + d] = src[d];
  if (b == 0 && threadIdx.x == 0) *pos = P;
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_xl_prefill_embed(const void *wte, const void *wpe, const int32_t *tok, float *h, int32_t B,
                                      int32_t P, int32_t V, int32_t D, void *stream) {
  if (!wte || !wpe || !tok || !h || B < 1 || P < 1 || V < 1 || D < 1 || (int64_t)B * P > (1 << 30))
    return sm100_set_error(SM100_ERR_ARG, "xl_prefill_embed: bad arguments");
  xl_prefill_embed_kernel<<<B * P, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16 *)wte,
                                                                   (const __nv_bfloat16 *)wpe, tok, h, P, V, D);
  return launch_status("xl_prefill_embed");
}

extern "C" int sm100_xl_prefill_split(const void *qkv, void *q, void *k, void *v, void *kv_cache, int32_t B,
                                      int32_t P, int32_t H, int32_t ctx, void *stream) {
  if (!qkv || !q || !k || !v || !kv_cache || B < 1 || P < 1 || H < 1 || ctx < P || (int64_t)B * P > (1 << 30) ||
      (((uintptr_t)qkv | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)kv_cache) & 15))
    return sm100_set_error(SM100_ERR_ARG, "xl_prefill_split: B %d P %d H %d ctx %d (P <= ctx, 16-byte aligned)", B, P,
                           H, ctx);
  xl_prefill_split_kernel<<<B * P, 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16 *)qkv, (__nv_bfloat16 *)q, (__nv_bfloat16 *)k, (__nv_bfloat16 *)v,
      (__nv_bfloat16 *)kv_cache, B, P, H, ctx);
  return launch_status("xl_prefill_split");
}

extern "C" int sm100_xl_prefill_merge(const float *o, void *att, int32_t B, int32_t P, int32_t H, void *stream) {
  if (!o || !att || B < 1 || P < 1 || H < 1 || (int64_t)B * P > (1 << 30) || (((uintptr_t)o | (uintptr_t)att) & 15))
    return sm100_set_error(SM100_ERR_ARG, "xl_prefill_merge: bad arguments");
  xl_prefill_merge_kernel<<<B * P, 256, 0, (cudaStream_t)stream>>>(o, (__nv_bfloat16 *)att, P, H);
  return launch_status("xl_prefill_merge");
}

extern "C" int sm100_xl_prefill_layernorm(const float *x, const float *g, const float *b, void *y, int32_t M,
                                          int32_t D, float eps, void *stream) {
  if (!x || !g || !b || !y || M < 1 || D < 4 || D % 4 || D > kXpLnVec * 128 ||
      (((uintptr_t)x | (uintptr_t)g | (uintptr_t)b | (uintptr_t)y) & 15))
    return sm100_set_error(SM100_ERR_ARG, "xl_prefill_layernorm: %d x %d (D %% 4, D <= %d, 16-byte aligned)", M, D,
                           kXpLnVec * 128);
  xl_prefill_ln_kernel<<<(M + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, g, b, (__nv_bfloat16 *)y, M, D, eps);
  return launch_status("xl_prefill_layernorm");
}

extern "C" int sm100_xl_prefill_last(const float *h, float *h_last, int32_t *pos, int32_t B, int32_t P, int32_t D,
                                     void *stream) {
  if (!h || !h_last || !pos || B < 1 || P < 1 || D < 1)
    return sm100_set_error(SM100_ERR_ARG, "xl_prefill_last: bad arguments");
  xl_prefill_last_kernel<<<B, 256, 0, (cudaStream_t)stream>>>(h, h_last, pos, P, D);
  return launch_status("xl_prefill_last");
}
