// The batched bf16 decode step of a GPT-2-XL-shaped model
// around the skinny tensor-core GEMM (k_skinny.cu): token + position
// embedding from bf16 tables, LayerNorm to a bf16 matmul operand, attention
// of B sequences over a bf16 KV cache, and the greedy token pick (row argmax,
// combined over vocabulary shards).  The reference composes these from
// Tensor ops (bench/gpt2/thvm_gpt2.py:27-128: Embedding, LayerNorm, SDPA over
// cache_kv, lm_head, argmax) and renders them as separate reductions.
//
// Every kernel here is launched with programmatic dependent launch: it lets
// the next kernel start at once and reads its inputs after griddepcontrol.wait.
//
// Numerics (the oracle's orc_xl_step follows the same order): the
// residual stream h is f32; every matmul operand is h's LayerNorm (or the
// attention output, or the GELU output) rounded to bf16; products accumulate
// in f32; k and v are stored in the cache as bf16.
#include "common.cuh"

namespace sm100 {

// h[b, :] = wte[tok[b], :] + wpe[pos, :] (bf16 tables, f32 out); an id outside
// [0, V) reads a zero row (the reference's one-hot embedding).
__global__ void xl_embed_kernel(const __nv_bfloat16 *wte, const __nv_bfloat16 *wpe, const int32_t *tok,
                                const int32_t *pos, float *h, int V, int D) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, id = tok[b], p = *pos;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float e = (id >= 0 && id < V) ? __bfloat162float(wte[(int64_t)id * D + d]) : 0.0f;
    h[(int64_t)b * D + d] = e + __bfloat162float(wpe[(int64_t)p * D + d]);
  }
}

// y = bf16(LayerNorm(x) * g + b), one row per CTA; mean and biased variance
// in f32 as sum * (1/D), rsqrt as 1/sqrt (src/nn/layernorm.c:1-7).
__global__ void __launch_bounds__(256) xl_ln_kernel(float *x, const float *g, const float *bt, __nv_bfloat16 *y,
                                                     int D, float eps, int zero_x, float *zero_buf, int64_t zero_n) {
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const float *xr = x + (int64_t)blockIdx.x * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float s = 0.0f;
  for (int i = threadIdx.x; i < D; i += 256) s += xr[i];
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) tot += red[w];
  const float inv_n = 1.0f / (float)D, mean = tot * inv_n;
  __syncthreads();
  float v = 0.0f;
  for (int i = threadIdx.x; i < D; i += 256) {
    const float c = xr[i] - mean;
    v += c * c;
  }
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float vt = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) vt += red[w];
  const float r = 1.0f / sqrtf(vt * inv_n + eps);
  __nv_bfloat16 *yr = y + (int64_t)blockIdx.x * D;
  float *xw = x + (int64_t)blockIdx.x * D;
  for (int i = threadIdx.x; i < D; i += 256) {
    yr[i] = __float2bfloat16_rn((xr[i] - mean) * r * g[i] + bt[i]);
    if (zero_x) xw[i] = 0.0f;   // this row is consumed: the next product accumulates into zeros
  }
  if (zero_buf) {   // an accumulator the next products add into
    const int64_t per = (zero_n + gridDim.x - 1) / gridDim.x, lo = per * blockIdx.x;
    for (int64_t i = lo + threadIdx.x; i < zero_n && i < lo + per; i += 256) zero_buf[i] = 0.0f;
  }
}

// Attention of one (sequence b, head h) over cache rows 0..pos:
// softmax(q . k_j * scale) v_j with q f32 (the qkv projection's first third)
// and k, v bf16 from cache [2][B][ctx][C], C = H * 64; out bf16 [B][C].
// 128 threads: scores one key per thread (the whole 64-wide key row from
// global memory, q in registers), block max / sum, then P V with each warp
// over a quarter of the keys and each lane over two output columns.  With
// `append`, qkv holds the complete sums of an accumulating product: the CTA
// first writes its head's k and v into cache row pos, and clears its q, k, v
// columns once read (the next layer's product adds into zeros).
constexpr int kXlHd = 64, kXlMaxCtx = 4096;

__global__ void __launch_bounds__(128) xl_attn_kernel(float *qkv, int64_t ld_qkv, __nv_bfloat16 *kv,
                                                       const int32_t *pos, __nv_bfloat16 *out, int B, int H, int ctx,
                                                       float scale, int append) {
  __shared__ float sc[kXlMaxCtx];
  __shared__ float red[4];
  __shared__ float2 part[4][32];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x / H, h = blockIdx.x % H, C = H * kXlHd;
  const int T = *pos + 1, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *q = qkv + (int64_t)b * ld_qkv + h * kXlHd;
  __nv_bfloat16 *kc = kv + (int64_t)b * ctx * C + h * kXlHd;
  __nv_bfloat16 *vc = kv + ((int64_t)B + b) * ctx * C + h * kXlHd;
  if (append && threadIdx.x < 2 * kXlHd) {
    // this step's k and v of the head (complete sums of the qkv product) into
    // cache row pos as bf16; the qkv row is cleared below for the next product
    const int which = threadIdx.x / kXlHd, d = threadIdx.x % kXlHd;
    (which ? vc : kc)[(int64_t)(T - 1) * C + d] = __float2bfloat16_rn(q[(1 + which) * C + d]);
  }
  __syncthreads();
  float qr[kXlHd];
#pragma unroll
  for (int i = 0; i < kXlHd; i += 4) {
    const float4 t = *reinterpret_cast<const float4 *>(q + i);
    qr[i] = t.x * scale;
    qr[i + 1] = t.y * scale;
    qr[i + 2] = t.z * scale;
    qr[i + 3] = t.w * scale;
  }
  __syncthreads();
  if (append && threadIdx.x < 3 * kXlHd / 2) {   // q, k and v of the head, two floats a thread
    const int part = threadIdx.x / (kXlHd / 2), d = 2 * (threadIdx.x % (kXlHd / 2));
    *reinterpret_cast<float2 *>(q + part * C + d) = make_float2(0.0f, 0.0f);
  }
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < T; j += 128) {
    const uint4 *kr = reinterpret_cast<const uint4 *>(kc + (int64_t)j * C);
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; c++) {
      const uint4 w = kr[c];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        s = fmaf(qr[8 * c + 2 * e], __uint_as_float(ww[e] << 16), s);
        s = fmaf(qr[8 * c + 2 * e + 1], __uint_as_float(ww[e] & 0xFFFF0000u), s);
      }
    }
    sc[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float sum = 0.0f;
  for (int j = threadIdx.x; j < T; j += 128) {
    const float e = exp2f((sc[j] - mx) * 1.4426950408889634f);
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  const float inv = 1.0f / ((red[0] + red[1]) + (red[2] + red[3]));
  float2 acc = make_float2(0.0f, 0.0f);
  for (int j = warp; j < T; j += 4) {
    const uint32_t w = reinterpret_cast<const uint32_t *>(vc + (int64_t)j * C)[lane];
    const float p = sc[j];
    acc.x = fmaf(p, __uint_as_float(w << 16), acc.x);
    acc.y = fmaf(p, __uint_as_float(w & 0xFFFF0000u), acc.y);
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0) {
    float2 t = part[0][lane];
#pragma unroll
    for (int w = 1; w < 4; w++) {
      t.x += part[w][lane].x;
      t.y += part[w][lane].y;
    }
    __nv_bfloat162 o = __floats2bfloat162_rn(t.x * inv, t.y * inv);
    reinterpret_cast<__nv_bfloat162 *>(out + (int64_t)b * C + h * kXlHd)[lane] = o;
  }
}

// Per row of x [M, N] (row stride ld): the largest value and its first index
// + idx_offset (a vocabulary shard's place in the whole): the reference's
// argmax picks the first index of the row maximum (py/thvm/tensor.py:998-1011).
// one CTA of 1024 threads per row; kVec: 16-byte loads (ld, N multiples of 4
// and a 16-byte aligned x), each thread's candidates in increasing index
// order, so the strict compare keeps the first index of the maximum
template <bool kVec>
__global__ void __launch_bounds__(1024) xl_argmax_kernel(float *x, int64_t ld, int N, float *val, int32_t *idx,
                                                          int idx_offset, int zero_x) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_trigger();
  pdl_wait();
  const float *xr = x + (int64_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if constexpr (kVec) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
#pragma unroll 4
    for (int c = threadIdx.x; c < N / 4; c += 1024) {
      const float4 f = x4[c];
      const float v[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (v[q] > bv || (v[q] == bv && 4 * c + q < bi)) {   // a thread's indices only grow
          bv = v[q];
          bi = 4 * c + q;
        }
    }
  } else {
    for (int i = threadIdx.x; i < N; i += 1024) {
      const float v = xr[i];
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (zero_x)   // the row is consumed: the next product accumulates into zeros
    for (int i = threadIdx.x; i < N; i += 1024) const_cast<float *>(xr)[i] = 0.0f;
  if (warp == 0) {
    bv = sv[lane];
    bi = si[lane];
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
      val[blockIdx.x] = bv;
      idx[blockIdx.x] = bi + idx_offset;
    }
  }
}

// tok[b] = the index of the largest of R shard candidates (val, idx laid out
// [R][B]); equal values go to the smaller index.
__global__ void xl_pick_kernel(const float *val, const int32_t *idx, int R, int B, int32_t *tok) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float bv = val[b];
  int bi = idx[b];
  for (int r = 1; r < R; r++) {
    const float v = val[r * B + b];
    const int i = idx[r * B + b];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  tok[b] = bi;
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_xl_embed(const void *wte, const void *wpe, const int32_t *tok, const int32_t *pos, float *h,
                              int32_t B, int32_t V, int32_t D, void *stream) {
  if (!wte || !wpe || !tok || !pos || !h || B < 1 || V < 1 || D < 1)
    return sm100_set_error(SM100_ERR_ARG, "xl_embed: bad arguments");
  const cudaError_t e = launch_pdl(xl_embed_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream,
                                   (const __nv_bfloat16 *)wte, (const __nv_bfloat16 *)wpe, tok, pos, h, V, D);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "xl_embed: %s", cudaGetErrorString(e));
  return launch_status("xl_embed");
}

extern "C" int sm100_xl_layernorm(float *x, const float *g, const float *b, void *y, int32_t M, int32_t D,
                                  float eps, int32_t zero_x, float *zero_buf, int64_t zero_n, void *stream) {
  if (!x || !g || !b || !y || M < 1 || D < 1 || zero_n < 0 || (zero_n && !zero_buf))
    return sm100_set_error(SM100_ERR_ARG, "xl_layernorm: bad arguments");
  const cudaError_t e = launch_pdl(xl_ln_kernel, dim3(M), dim3(256), 0, (cudaStream_t)stream, x, g, b,
                                   (__nv_bfloat16 *)y, D, eps, (int)zero_x, zero_n ? zero_buf : (float *)nullptr,
                                   zero_n);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "xl_layernorm: %s", cudaGetErrorString(e));
  return launch_status("xl_layernorm");
}

extern "C" int sm100_xl_attention(float *qkv, int64_t ld_qkv, void *kv_cache, const int32_t *pos, void *out,
                                  int32_t B, int32_t H, int32_t hd, int32_t ctx, float scale, int32_t append,
                                  void *stream) {
  if (!qkv || !kv_cache || !pos || !out || B < 1 || H < 1 || hd != kXlHd || ctx < 1 || ctx > kXlMaxCtx ||
      ((uintptr_t)qkv & 15) || (ld_qkv % 4) || ((uintptr_t)kv_cache & 15))
    return sm100_set_error(SM100_ERR_ARG, "xl_attention: B %d H %d hd %d ctx %d (hd 64, ctx <= %d, aligned)", B, H,
                           hd, ctx, kXlMaxCtx);
  const cudaError_t e = launch_pdl(xl_attn_kernel, dim3(B * H), dim3(128), 0, (cudaStream_t)stream, qkv, ld_qkv,
                                   (__nv_bfloat16 *)kv_cache, pos, (__nv_bfloat16 *)out, B, H, ctx, scale, (int)append);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "xl_attention: %s", cudaGetErrorString(e));
  return launch_status("xl_attention");
}

extern "C" int sm100_xl_argmax(float *x, int64_t ld, int32_t M, int32_t N, float *val, int32_t *idx,
                               int32_t idx_offset, int32_t zero_x, void *stream) {
  if (!x || !val || !idx || M < 1 || N < 1 || ld < N) return sm100_set_error(SM100_ERR_ARG, "xl_argmax: bad arguments");
  const bool vec = ld % 4 == 0 && N % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const cudaError_t e =
      vec ? launch_pdl(xl_argmax_kernel<true>, dim3(M), dim3(1024), 0, (cudaStream_t)stream, x, ld, N, val, idx,
                       idx_offset, (int)zero_x)
          : launch_pdl(xl_argmax_kernel<false>, dim3(M), dim3(1024), 0, (cudaStream_t)stream, x, ld, N, val, idx,
                       idx_offset, (int)zero_x);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "xl_argmax: %s", cudaGetErrorString(e));
  return launch_status("xl_argmax");
}

extern "C" int sm100_xl_pick(const float *val, const int32_t *idx, int32_t R, int32_t B, int32_t *tok, void *stream) {
  if (!val || !idx || !tok || R < 1 || B < 1) return sm100_set_error(SM100_ERR_ARG, "xl_pick: bad arguments");
  const cudaError_t e =
      launch_pdl(xl_pick_kernel, dim3((B + 127) / 128), dim3(128), 0, (cudaStream_t)stream, val, idx, R, B, tok);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "xl_pick: %s", cudaGetErrorString(e));
  return launch_status("xl_pick");
}
