// Skinny linear y[m, n] = sum_k pro(x)[m, k] * W[n, k] (+ b[n]) [GELU] [+ residual]
// for the decode path: M is 1 (a decode step) to a few dozen (a prompt),
// N and K up to tens of thousands.  This is the reference's matvec after
// rangeify (nn_linear / nn_dot as REDUCE(SUM, MUL(EXPAND)), src/nn/linear.c:1-6,
// src/nn/dot.c:1-20) with Linear's W stored (out, in) and read through .T
// (py/thvm/nn.py:12-25), so each output's weights are one contiguous row.
//
// Bound: HBM.  Every weight byte is read exactly once per launch (per M-tile);
// x (and its LayerNorm) is staged once per CTA in shared memory.  Each output
// row is owned by TPR threads that stream 16-byte vectors of the row with
// no-L1-allocate loads, all loads of a thread issued before its FMAs, then a
// warp-shuffle (+ shared) reduction.  Grid = ceil(N / rows_per_CTA) so that
// every SM holds several CTAs and enough bytes are in flight to cover DRAM
// latency.  Prologue: optional LayerNorm of each x row (the reference's
// nn_layernorm order: mean, centred variance, recip(sqrt(var + eps)), then *g
// + b).  Epilogue: bias, tanh GELU, residual add, and the KV-cache append of
// the k / v thirds of a fused qkv projection.
#include <cuda_fp8.h>

#include "common.cuh"

namespace sm100 {

struct LinParams {
  const float *x;
  const void *w;
  const float *w_scale;
  const float *bias, *ln_g, *ln_b, *residual;
  float *y;
  float *kv_cache;
  const int32_t *pos;
  int64_t M, N, K, ldx, ldy;
  int32_t flags, max_ctx, host_pos, scale_cols;
  float eps;
};

// Elements of W per 16-byte vector.
template <typename WT> struct WVec;
template <> struct WVec<float> { static constexpr int n = 4; };
template <> struct WVec<__nv_bfloat16> { static constexpr int n = 8; };
template <> struct WVec<__nv_fp8_e4m3> { static constexpr int n = 16; };

// Dot of one 16-byte weight vector with x values at xs[0..n).
template <typename WT, int MB>
__device__ __forceinline__ void dot_vec(const uint4 &wv, const float *xs, int64_t K, float (&acc)[MB],
                                        float scale) {
  if constexpr (sizeof(WT) == 4) {
    const float w0 = __uint_as_float(wv.x), w1 = __uint_as_float(wv.y);
    const float w2 = __uint_as_float(wv.z), w3 = __uint_as_float(wv.w);
#pragma unroll
    for (int mb = 0; mb < MB; mb++) {
      const float4 xv = *reinterpret_cast<const float4 *>(xs + mb * K);
      acc[mb] = fmaf(w0, xv.x, acc[mb]);
      acc[mb] = fmaf(w1, xv.y, acc[mb]);
      acc[mb] = fmaf(w2, xv.z, acc[mb]);
      acc[mb] = fmaf(w3, xv.w, acc[mb]);
    }
  } else if constexpr (sizeof(WT) == 2) {
    const uint32_t u[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int mb = 0; mb < MB; mb++) {
      const float4 xa = *reinterpret_cast<const float4 *>(xs + mb * K);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + mb * K + 4);
      float a = acc[mb];
      a = fmaf(bf16_lo(u[0]), xa.x, a);
      a = fmaf(bf16_hi(u[0]), xa.y, a);
      a = fmaf(bf16_lo(u[1]), xa.z, a);
      a = fmaf(bf16_hi(u[1]), xa.w, a);
      a = fmaf(bf16_lo(u[2]), xb.x, a);
      a = fmaf(bf16_hi(u[2]), xb.y, a);
      a = fmaf(bf16_lo(u[3]), xb.z, a);
      a = fmaf(bf16_hi(u[3]), xb.w, a);
      acc[mb] = a;
    }
  } else {
    // fp8 e4m3: 16 weights; the block scale multiplies the 16-term partial.
    const uint32_t u[4] = {wv.x, wv.y, wv.z, wv.w};
    float wf[16];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      __half2_raw h0 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(u[i] & 0xffffu), __NV_E4M3);
      __half2_raw h1 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(u[i] >> 16), __NV_E4M3);
      const float2 f0 = __half22float2(*reinterpret_cast<__half2 *>(&h0));
      const float2 f1 = __half22float2(*reinterpret_cast<__half2 *>(&h1));
      wf[4 * i + 0] = f0.x;
      wf[4 * i + 1] = f0.y;
      wf[4 * i + 2] = f1.x;
      wf[4 * i + 3] = f1.y;
    }
#pragma unroll
    for (int mb = 0; mb < MB; mb++) {
      float part = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 xv = *reinterpret_cast<const float4 *>(xs + mb * K + j);
        part = fmaf(wf[j], xv.x, part);
        part = fmaf(wf[j + 1], xv.y, part);
        part = fmaf(wf[j + 2], xv.z, part);
        part = fmaf(wf[j + 3], xv.w, part);
      }
      acc[mb] = fmaf(part, scale, acc[mb]);
    }
  }
}

template <typename WT>
__device__ __forceinline__ float w_scalar(const WT *w, int64_t i) {
  if constexpr (sizeof(WT) == 4) return w[i];
  else if constexpr (sizeof(WT) == 2) return __bfloat162float(w[i]);
  else return float(w[i]);
}

// Stage rows [m0, m0 + mb_n) of x into xs ([MB][K], zero-padded rows past M),
// applying the LayerNorm prologue when asked.
template <int MB>
__device__ void stage_x(const LinParams &p, int64_t m0, float *xs, float *red) {
  const int64_t K = p.K;
  for (int mb = 0; mb < MB; mb++) {
    const int64_t m = m0 + mb;
    float *dst = xs + mb * K;
    if (m >= p.M) {
      for (int64_t k = threadIdx.x; k < K; k += blockDim.x) dst[k] = 0.0f;
      continue;
    }
    const float *src = p.x + m * p.ldx;
    if (!(p.flags & SM100_LIN_LN)) {
      for (int64_t k = threadIdx.x; k < K; k += blockDim.x) dst[k] = src[k];
      continue;
    }
    const float inv_n = (float)(1.0 / (double)K);  // nn_mean: sum * (1/count)
    float s = 0.0f;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      const float v = src[k];
      dst[k] = v;
      s += v;
    }
    const float mean = __fmul_rn(block_sum(s, red), inv_n);
    float v2 = 0.0f;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      const float c = __fsub_rn(dst[k], mean);
      v2 = fmaf(c, c, v2);
    }
    const float var = __fmul_rn(block_sum(v2, red), inv_n);
    const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(var, p.eps)));
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      float o = __fmul_rn(__fsub_rn(dst[k], mean), r);
      if (p.ln_g) o = __fmul_rn(o, p.ln_g[k]);
      if (p.ln_b) o = __fadd_rn(o, p.ln_b[k]);
      dst[k] = o;
    }
  }
}

__device__ __forceinline__ void epilogue_store(const LinParams &p, int64_t m, int64_t n, float acc) {
  float v = acc;
  if (p.bias) v = __fadd_rn(v, p.bias[n]);
  if (p.flags & SM100_LIN_GELU) v = gelu_tanh(v);
  if (p.flags & SM100_LIN_RESIDUAL) v = __fadd_rn(p.residual[m * p.ldy + n], v);
  p.y[m * p.ldy + n] = v;
  if (p.flags & SM100_LIN_KV_APPEND) {
    const int64_t d = p.N / 3;
    if (n >= d) {
      const int64_t which = n / d - 1, col = n - (which + 1) * d;
      const int64_t pos = (p.pos ? (int64_t)*p.pos : (int64_t)p.host_pos) + m;
      if (pos >= 0 && pos < p.max_ctx) p.kv_cache[(which * p.max_ctx + pos) * d + col] = v;
    }
  }
}

// TPR threads own one output row; 256 / TPR rows per CTA; MB x rows per pass.
template <typename WT, int TPR, int MB, bool VEC>
__global__ void __launch_bounds__(256) linear_kernel(LinParams p) {
  extern __shared__ float4 smem4[];
  float *xs = reinterpret_cast<float *>(smem4);
  __shared__ float red[32];
  __shared__ float part[256 / 32][MB];
  constexpr int RPC = 256 / TPR;
  const int sub = threadIdx.x / TPR, t = threadIdx.x % TPR;
  const int64_t n = (int64_t)blockIdx.x * RPC + sub;
  const int64_t K = p.K;
  const WT *w = static_cast<const WT *>(p.w);

  for (int64_t m0 = 0; m0 < p.M; m0 += MB) {
    stage_x<MB>(p, m0, xs, red);
    __syncthreads();
    float acc[MB];
#pragma unroll
    for (int mb = 0; mb < MB; mb++) acc[mb] = 0.0f;
    if (n < p.N) {
      const WT *wr = w + n * K;
      if constexpr (VEC) {
        constexpr int V = WVec<WT>::n;
        const int64_t nvec = K / V;
        // 4 vectors in flight per thread per iteration.
        int64_t i = t;
        for (; i + 3 * TPR < nvec; i += 4 * TPR) {
          uint4 wv[4];
#pragma unroll
          for (int u = 0; u < 4; u++) wv[u] = ld_stream_u4(wr + (i + u * TPR) * V);
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int64_t k0 = (i + u * TPR) * V;
            const float sc = (sizeof(WT) == 1) ? p.w_scale[(n >> 7) * p.scale_cols + (k0 >> 7)] : 1.0f;
            dot_vec<WT, MB>(wv[u], xs + k0, K, acc, sc);
          }
        }
        for (; i < nvec; i += TPR) {
          const uint4 wv = ld_stream_u4(wr + i * V);
          const int64_t k0 = i * V;
          const float sc = (sizeof(WT) == 1) ? p.w_scale[(n >> 7) * p.scale_cols + (k0 >> 7)] : 1.0f;
          dot_vec<WT, MB>(wv, xs + k0, K, acc, sc);
        }
      } else {
        for (int64_t k = t; k < K; k += TPR) {
          float wk = w_scalar<WT>(wr, k);
          if constexpr (sizeof(WT) == 1) wk *= p.w_scale[(n >> 7) * p.scale_cols + (k >> 7)];
#pragma unroll
          for (int mb = 0; mb < MB; mb++) acc[mb] = fmaf(wk, xs[mb * K + k], acc[mb]);
        }
      }
    }
#pragma unroll
    for (int mb = 0; mb < MB; mb++) acc[mb] = warp_sum(acc[mb]);
    if constexpr (TPR > 32) {
      const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
      if (lane == 0) {
#pragma unroll
        for (int mb = 0; mb < MB; mb++) part[wid][mb] = acc[mb];
      }
      __syncthreads();
      if (t < MB && n < p.N && m0 + t < p.M) {
        float s = 0.0f;
        for (int j = 0; j < TPR / 32; j++) s += part[sub * (TPR / 32) + j][t];
        epilogue_store(p, m0 + t, n, s);
      }
    } else {
      if (n < p.N) {
        // lane mb stores row m0 + mb (all lanes hold all sums after warp_sum)
#pragma unroll
        for (int mb = 0; mb < MB; mb++)
          if (t == mb && m0 + mb < p.M) epilogue_store(p, m0 + mb, n, acc[mb]);
      }
    }
    __syncthreads();
  }
}

template <typename WT, int TPR, int MB>
static int launch_tpr(const LinParams &p, bool vec, cudaStream_t st) {
  constexpr int RPC = 256 / TPR;
  const int64_t grid = (p.N + RPC - 1) / RPC;
  const size_t smem = sizeof(float) * (size_t)MB * (size_t)p.K;
  auto kern = vec ? linear_kernel<WT, TPR, MB, true> : linear_kernel<WT, TPR, MB, false>;
  // dynamic + static shared memory above the default 48 KB needs the opt-in
  if (smem > 40 * 1024) {
    if (smem > 220 * 1024) return sm100_set_error(SM100_ERR_UNSUPPORTED, "linear: K=%lld too large", (long long)p.K);
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  kern<<<(unsigned)grid, 256, smem, st>>>(p);
  return launch_status("linear");
}

template <typename WT, int MB>
static int launch_mb(const LinParams &p, bool vec, int tpr, cudaStream_t st) {
  switch (tpr) {
    case 32: return launch_tpr<WT, 32, MB>(p, vec, st);
    case 64: return launch_tpr<WT, 64, MB>(p, vec, st);
    case 128: return launch_tpr<WT, 128, MB>(p, vec, st);
    default: return launch_tpr<WT, 256, MB>(p, vec, st);
  }
}

template <typename WT>
static int launch_w(const LinParams &p, cudaStream_t st) {
  constexpr int V = WVec<WT>::n;
  const bool vec = (p.K % V == 0) && ((reinterpret_cast<uintptr_t>(p.w) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0 || true);
  // Threads per row: the most that still give every thread >= 3 vectors, so
  // that small-N projections spread over many CTAs; at least a warp.
  const int64_t nvec = (p.K + V - 1) / V;
  int tpr = 32;
  while (tpr < 256 && nvec / (tpr * 2) >= 3 && p.N * tpr < 148LL * 8 * 256) tpr *= 2;
  if (p.M <= 1) return launch_mb<WT, 1>(p, vec, tpr, st);
  if (p.M <= 2) return launch_mb<WT, 2>(p, vec, tpr, st);
  return launch_mb<WT, 4>(p, vec, tpr, st);
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_linear(const Sm100LinearArgs *a, void *stream) {
  if (!a || !a->x || !a->w || !a->y || a->M < 0 || a->N <= 0 || a->K <= 0)
    return sm100_set_error(SM100_ERR_ARG, "linear: bad arguments");
  if (a->M == 0) return SM100_OK;
  if ((a->flags & SM100_LIN_RESIDUAL) && !a->residual)
    return sm100_set_error(SM100_ERR_ARG, "linear: RESIDUAL without a residual");
  if ((a->flags & SM100_LIN_KV_APPEND) && (!a->kv_cache || a->N % 3 || a->max_ctx <= 0))
    return sm100_set_error(SM100_ERR_ARG, "linear: KV_APPEND needs a cache and N = 3d");
  LinParams p;
  p.x = a->x; p.w = a->w; p.w_scale = a->w_scale; p.bias = a->bias;
  p.ln_g = a->ln_g; p.ln_b = a->ln_b; p.residual = a->residual; p.y = a->y;
  p.kv_cache = a->kv_cache; p.pos = a->pos;
  p.M = a->M; p.N = a->N; p.K = a->K;
  p.ldx = a->ldx ? a->ldx : a->K;
  p.ldy = a->ldy ? a->ldy : a->N;
  p.flags = a->flags; p.max_ctx = a->max_ctx; p.host_pos = a->host_pos;
  p.scale_cols = (int32_t)((a->K + 127) / 128);
  p.eps = a->eps;
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->wdtype) {
    case SM100_DT_F32: return launch_w<float>(p, st);
    case SM100_DT_BF16: return launch_w<__nv_bfloat16>(p, st);
    case SM100_DT_FP8E4M3:
      if (!a->w_scale) return sm100_set_error(SM100_ERR_ARG, "linear: fp8 needs block scales");
      return launch_w<__nv_fp8_e4m3>(p, st);
    default: return sm100_set_error(SM100_ERR_UNSUPPORTED, "linear: weight dtype %d", a->wdtype);
  }
}
