// Decode / prompt attention over the KV cache, f32:
//   out[t, h, :] = softmax(q[t, h] . K[0..pos+t, h]^T * scale) . V[0..pos+t, h]
// which is the reference's scaled_dot_product_attention on the cache slice
// (src/nn/scaled_dot_product_attention.c:1-34; the GPT-2 call site
// bench/gpt2/thvm_gpt2.py:36-61 reads keys = cache_kv[0][:, :start_pos+seqlen]
// and, for a prompt, adds the -inf triu(start_pos+1) mask, so query row t sees
// keys 0..start_pos+t).  The position is read from device memory, so one
// captured CUDA graph serves every decode step.
//
// One CTA per (head, query row).  Scores live in shared memory (max_ctx
// floats).  Keys: groups of 8 lanes own one key row (hd / 8 dims each, 16-byte
// loads), so a warp covers 4 keys per step; the softmax follows the reference's
// order (scale, max, exp via xexp2 of (s - max), sum, * recip(sum)); the mix
// walks keys with each thread owning one output dim for a slice of the keys.
// Bound: the K/V bytes of the live prefix (L2-resident for decode sizes).
#include "common.cuh"

namespace sm100 {

struct AttnParams {
  const float *q, *kc, *vc;
  float *out;
  const int32_t *pos;
  int64_t ldq;
  int32_t T, H, hd, max_ctx, host_pos;
  float scale;
};

__global__ void __launch_bounds__(256) attn_kernel(AttnParams p) {
  extern __shared__ float smem[];
  __shared__ float red[32];
  float *sc = smem;                          // [max_ctx] scores
  float *qs = smem + p.max_ctx;              // [hd] query
  float *acc = qs + p.hd;                    // [256 / hd slices][hd]
  const int h = blockIdx.x, t = blockIdx.y;
  const int D = p.H * p.hd;
  const int start = p.pos ? *p.pos : p.host_pos;
  int L = start + t + 1;
  if (L > p.max_ctx) L = p.max_ctx;
  if (L < 1) L = 1;

  const float *qrow = p.q + (int64_t)t * p.ldq + (int64_t)h * p.hd;
  for (int d = threadIdx.x; d < p.hd; d += blockDim.x) qs[d] = qrow[d];
  __syncthreads();

  // scores: 8-lane groups, one key per group
  const int grp = threadIdx.x >> 3, gl = threadIdx.x & 7, ngrp = blockDim.x >> 3;
  const int per = p.hd / 8;  // dims per lane (hd % 8 == 0)
  // j0 is uniform over the CTA, so every lane reaches the shuffles below.
  for (int j0 = 0; j0 < L; j0 += ngrp) {
    const int j = j0 + grp;
    const bool live = j < L;
    const float *kr = p.kc + (int64_t)(live ? j : 0) * D + (int64_t)h * p.hd + gl * per;
    const float *qq = qs + gl * per;
    float s = 0.0f;
    if (!live) {
    } else if ((per & 3) == 0) {
      for (int i = 0; i < per; i += 4) {
        const float4 kv = *reinterpret_cast<const float4 *>(kr + i);
        s = fmaf(qq[i], kv.x, s);
        s = fmaf(qq[i + 1], kv.y, s);
        s = fmaf(qq[i + 2], kv.z, s);
        s = fmaf(qq[i + 3], kv.w, s);
      }
    } else {
      for (int i = 0; i < per; i++) s = fmaf(qq[i], kr[i], s);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (live && gl == 0) sc[j] = __fmul_rn(s, p.scale);
  }
  __syncthreads();

  float mx = -INFINITY;
  for (int j = threadIdx.x; j < L; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  mx = block_max(mx, red);
  float sum = 0.0f;
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    const float e = xexp(__fsub_rn(sc[j], mx));
    sc[j] = e;
    sum += e;
  }
  sum = block_sum(sum, red);
  const float r = __frcp_rn(sum);
  for (int j = threadIdx.x; j < L; j += blockDim.x) sc[j] = __fmul_rn(sc[j], r);
  __syncthreads();

  // mix: thread (slice, d) sums keys j = slice, slice + nslice, ...
  const int nslice = blockDim.x / p.hd;
  const int slice = threadIdx.x / p.hd, d = threadIdx.x % p.hd;
  if (slice < nslice) {
    float a = 0.0f;
    const float *vcol = p.vc + (int64_t)h * p.hd + d;
    for (int j = slice; j < L; j += nslice) a = fmaf(sc[j], vcol[(int64_t)j * D], a);
    acc[slice * p.hd + d] = a;
  }
  __syncthreads();
  for (int dd = threadIdx.x; dd < p.hd; dd += blockDim.x) {
    float a = 0.0f;
    for (int s2 = 0; s2 < nslice; s2++) a += acc[s2 * p.hd + dd];
    p.out[(int64_t)t * D + (int64_t)h * p.hd + dd] = a;
  }
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_attention(const Sm100AttnArgs *a, void *stream) {
  if (!a || !a->q || !a->k_cache || !a->v_cache || !a->out || a->T <= 0 || a->H <= 0 ||
      a->hd <= 0 || a->hd % 8 || a->hd > 256 || a->max_ctx <= 0)
    return sm100_set_error(SM100_ERR_ARG, "attention: bad arguments");
  AttnParams p;
  p.q = a->q; p.kc = a->k_cache; p.vc = a->v_cache; p.out = a->out; p.pos = a->pos;
  p.ldq = a->ldq ? a->ldq : (int64_t)a->H * a->hd;
  p.T = a->T; p.H = a->H; p.hd = a->hd; p.max_ctx = a->max_ctx; p.host_pos = a->host_pos;
  p.scale = a->scale != 0.0f ? a->scale : (float)(1.0 / sqrt((double)a->hd));
  const size_t smem = sizeof(float) * ((size_t)a->max_ctx + (size_t)a->hd + 256);
  if (smem > 227 * 1024) return sm100_set_error(SM100_ERR_UNSUPPORTED, "attention: max_ctx too large");
  if (smem > 40 * 1024)
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)a->H, (unsigned)a->T);
  attn_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(p);
  return launch_status("attention");
}
