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
#include "tma.cuh"

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

// Decode matvec (M = 1, no LayerNorm prologue): one warp per output row.
// Every lane issues all of its weight loads for the row (NV 16-byte vectors,
// streaming, not L1-allocated) at CTA start, before x is staged into shared
// memory, so the HBM latency overlaps the staging; then the dot product, a
// warp reduction and the epilogue (bias / GELU / residual / KV append).
// Bound: HBM, every weight byte read once.  128 threads (4 rows) per CTA
// keeps the last wave short.
template <typename WT, int NV>
__global__ void __launch_bounds__(128) gemv_kernel(LinParams p) {
  extern __shared__ float4 smem4[];
  float *xs = reinterpret_cast<float *>(smem4);
  constexpr int V = WVec<WT>::n;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n = (int64_t)blockIdx.x * 4 + warp, K = p.K;
  const bool live = n < p.N;
  const WT *wr = static_cast<const WT *>(p.w) + (live ? n : 0) * K;
  uint4 wv[NV];
#pragma unroll
  for (int v = 0; v < NV; v++) wv[v] = __ldcs(reinterpret_cast<const uint4 *>(wr + (int64_t)(lane + 32 * v) * V));
  const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
  for (int64_t i = threadIdx.x; i < K / 4; i += blockDim.x) reinterpret_cast<float4 *>(xs)[i] = __ldg(x4 + i);
  __syncthreads();
  float acc[1] = {0.0f};
#pragma unroll
  for (int v = 0; v < NV; v++) {
    const int64_t k0 = (int64_t)(lane + 32 * v) * V;
    const float sc = (sizeof(WT) == 1) ? p.w_scale[(n >> 7) * p.scale_cols + (k0 >> 7)] : 1.0f;
    dot_vec<WT, 1>(wv[v], xs + k0, K, acc, sc);
  }
  const float a = warp_sum(acc[0]);
  if (live && lane == 0) epilogue_store(p, 0, n, a);
}

// Decode matvec streamed through shared memory (M = 1): one CTA per SM owns a
// contiguous slice of rows; one producer thread keeps every stage of a ring
// of (16 / KS)-row stages in flight with TMA bulk copies (L2 evict_first:
// the weights are read once); 16 consumer warps take (row, K slice) each per
// stage, KS slices per row.  A lane always reads the same 16-byte columns of
// its slice (vectors lane, lane + 32, ...), so its NJ slices of x are loaded
// into registers once per launch: shared memory only carries the weights
// (lane-contiguous reads, no bank conflicts).  No CTA barrier per stage:
// each warp leaves its slice's partial in shared memory and the last of a
// row's KS warps (a shared-memory counter) adds the slices in order and runs
// the epilogue; every warp releases the stage itself (an mbarrier of 16
// arrivals).
// Streaming with ~190 KB in flight per SM is what reaches HBM read bandwidth
// (loads issued per thread stall between short-lived CTAs).
constexpr int kGvWarps = 16;                      // consumer warps
constexpr int kGvRows = 32;                       // most rows per stage (KS = 1, 2 rows per warp)
constexpr int kGvThreads = (kGvWarps + 1) * 32;   // + producer warp
constexpr int kGvSmem = 200 * 1024;               // ring + scales + partials + barriers
constexpr int kGvMaxStages = 8;
constexpr int kGvPart = 4 * kGvRows;              // partials of a stage: KS (<= 4) slices x R (<= kGvRows) rows

template <typename WT, int NJ, int KS, int RW>
__global__ void __launch_bounds__(kGvThreads, 1) gemv_tma_kernel(LinParams p, int stages, int stage_floats) {
  constexpr int R = kGvWarps / KS * RW;   // rows per stage (RW rows per warp)
  static_assert(R <= kGvRows && KS * R <= kGvPart, "stage rows / partials");
  extern __shared__ __align__(1024) unsigned char smem[];
  constexpr int V = WVec<WT>::n;
  const int64_t K = p.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (p.N * blockIdx.x) / gridDim.x, r1 = (p.N * (blockIdx.x + 1)) / gridDim.x;
  const int nchunks = (int)((r1 - r0 + R - 1) / R);
  float *ring = reinterpret_cast<float *>(smem);
  float *ss = ring + (size_t)stages * stage_floats;                          // [2][scale_cols]: this CTA's scale rows
  float *part = ss + 2 * (size_t)p.scale_cols;                                // [stages][KS][R] partials
  int *cnt = reinterpret_cast<int *>(part + (size_t)kGvMaxStages * kGvPart);  // [stages][R] slices done
  uint64_t *full = reinterpret_cast<uint64_t *>(cnt + (size_t)kGvMaxStages * kGvRows);   // [stages]
  uint64_t *empty = full + kGvMaxStages;                                      // [stages]
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGvWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = threadIdx.x; i < kGvMaxStages * kGvRows; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  // programmatic dependent launch: the weights are static, so the producer
  // streams them at once, overlapping the previous kernel's tail; the
  // consumers read x and write y only after that kernel has completed
  pdl_trigger();
  const size_t row_bytes = (size_t)K * sizeof(WT);
  if (warp == kGvWarps) {
    // producer: chunk c -> stage c % stages, rows [r0 + R c, ...)
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const unsigned char *w = static_cast<const unsigned char *>(p.w);
      for (int c = 0; c < nchunks; c++) {
        const int s = c % stages;
        if (c >= stages && !mbar_wait(&empty[s], (uint32_t)(((c / stages) - 1) & 1), nullptr)) break;
        const int64_t rr = r0 + (int64_t)c * R, nr = (r1 - rr) < R ? (r1 - rr) : R;
        const uint32_t bytes = (uint32_t)(nr * row_bytes);
        mbar_expect_tx(&full[s], bytes);
        bulk_g2s_hint(ring + (size_t)s * stage_floats, w + rr * row_bytes, bytes, &full[s], pol);
      }
      // every issued copy has landed before the CTA exits (bounded)
      for (int c = nchunks - stages > 0 ? nchunks - stages : 0; c < nchunks; c++)
        mbar_wait(&full[c % stages], (uint32_t)((c / stages) & 1), nullptr, false);
    }
    return;
  }
  // consumers: this lane's x columns into registers, the fp8 block scales of
  // this CTA's rows into shared memory
  const int ct = threadIdx.x, nct = kGvWarps * 32;
  constexpr int WPS = kGvWarps / KS;          // warps per K slice; warp (ks, rw) has rows rw * RW + i
  const int ks = warp / WPS, rw = warp % WPS;
  const int vbase = ks * NJ * 32 + lane;   // vector j of this lane: vbase + 32 j
  float xr[NJ * V];
  pdl_wait();
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const float4 *src = reinterpret_cast<const float4 *>(p.x + (int64_t)(vbase + 32 * j) * V);
#pragma unroll
    for (int q = 0; q < V / 4; q++) {
      const float4 f = __ldg(src + q);
      xr[j * V + 4 * q] = f.x;
      xr[j * V + 4 * q + 1] = f.y;
      xr[j * V + 4 * q + 2] = f.z;
      xr[j * V + 4 * q + 3] = f.w;
    }
  }
  if constexpr (sizeof(WT) == 1) {
    const int64_t sr0 = r0 >> 7;
    for (int i = ct; i < 2 * p.scale_cols; i += nct) {
      const int64_t sr = sr0 + i / p.scale_cols;
      ss[i] = (sr * 128 < p.N) ? p.w_scale[sr * p.scale_cols + i % p.scale_cols] : 0.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kGvWarps * 32) : "memory");
  }
  for (int c = 0; c < nchunks; c++) {
    const int s = c % stages;
    mbar_wait(&full[s], (uint32_t)((c / stages) & 1), nullptr);
    const int64_t nb = r0 + (int64_t)c * R + (int64_t)rw * RW;   // this warp's first row
    if (nb < r1) {
      const uint4 *wrow = reinterpret_cast<const uint4 *>(reinterpret_cast<const unsigned char *>(
                              ring + (size_t)s * stage_floats) + (size_t)rw * RW * row_bytes);
      float acc[RW];
#pragma unroll
      for (int i = 0; i < RW; i++) acc[i] = 0.0f;
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const int v = vbase + 32 * j;
#pragma unroll
        for (int i = 0; i < RW; i++) {
          if (nb + i < r1) {
            const float sc = (sizeof(WT) == 1) ? ss[(((nb + i) >> 7) - (r0 >> 7)) * p.scale_cols + ((v * V) >> 7)] : 1.0f;
            float a1[1] = {acc[i]};
            dot_vec<WT, 1>(wrow[(size_t)i * (row_bytes / 16) + v], xr + j * V, K, a1, sc);
            acc[i] = a1[0];
          }
        }
      }
#pragma unroll
      for (int i = 0; i < RW; i++) acc[i] = warp_sum(acc[i]);
      if (lane == 0) {
        float *ps = part + (size_t)s * kGvPart;
#pragma unroll
        for (int i = 0; i < RW; i++) {
          const int64_t n = nb + i;
          const int slot = rw * RW + i;
          if (n >= r1) break;
          if (KS == 1) {
            epilogue_store(p, 0, n, acc[i]);
          } else {
            ps[ks * R + slot] = acc[i];
            __threadfence_block();
            if (atomicAdd(&cnt[s * kGvRows + slot], 1) == KS - 1) {   // the row's last slice: add them in order
              __threadfence_block();
              float t2 = 0.0f;
#pragma unroll
              for (int k2 = 0; k2 < KS; k2++) t2 += *(volatile float *)&ps[k2 * R + slot];
              cnt[s * kGvRows + slot] = 0;
              epilogue_store(p, 0, n, t2);
            }
          }
        }
      }
    }
    // this warp is done with the stage: the producer may refill it after all 16
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// Stages of the streamed matvec for this shape (0: it does not fit), KS
// (K slices per row: the fewest that keep x within 32 registers a lane) and
// Rows per warp per stage: fp8 rows are short, so four (two when a row is
// one slice) per warp per stage.
template <typename WT>
__host__ __device__ constexpr int gemv_rw(int ks) {
  return sizeof(WT) == 1 ? (ks >= 2 ? 4 : 2) : 1;
}

// NJ, the 16-byte vectors per lane of a slice (K = KS * 32 * NJ * V).
template <typename WT>
static int gemv_tma_stages(const LinParams &p, int &stage_floats, int &nj, int &ks) {
  constexpr int V = WVec<WT>::n;
  nj = 0;
  for (ks = 1; ks <= 4; ks *= 2) {
    if (p.K % ((int64_t)ks * 32 * V)) continue;
    const int64_t n = p.K / ((int64_t)ks * 32 * V);
    if (n * V <= 32 && (n == 1 || n == 2 || n == 3 || n == 4 || n == 6 || n == 8)) {
      nj = (int)n;
      break;
    }
  }
  if (!nj) return 0;
  const size_t stage = (size_t)(kGvWarps / ks * gemv_rw<WT>(ks)) * (size_t)p.K * sizeof(WT);
  const size_t fixed = 2 * (size_t)p.scale_cols * 4 + (size_t)kGvMaxStages * (kGvPart + kGvRows) * 4 +
                       2 * kGvMaxStages * 8 + 64;
  if (stage % 16 || fixed + 2 * stage > (size_t)kGvSmem) return 0;
  stage_floats = (int)(stage / 4);
  const size_t s = (kGvSmem - fixed) / stage;
  return (int)(s < (size_t)kGvMaxStages ? s : (size_t)kGvMaxStages);
}

template <typename WT, int NJ, int KS>
static int launch_gemv_tma_nj(const LinParams &p, int stages, int stage_floats, cudaStream_t st) {
  constexpr int RW = gemv_rw<WT>(KS);   // rows per warp per stage
  constexpr int R = kGvWarps / KS * RW;
  static int num_sms[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sm100_set_error(SM100_ERR_ARG, "gemv: device %d", dev);
  if (!num_sms[dev]) cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int64_t rows_per = (p.N + num_sms[dev] - 1) / num_sms[dev];
  const int grid = rows_per < R ? (int)((p.N + R - 1) / R) : num_sms[dev];
  cudaError_t e =
      cudaFuncSetAttribute(gemv_tma_kernel<WT, NJ, KS, RW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGvSmem);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "gemv: smem attribute: %s", cudaGetErrorString(e));
  e = launch_pdl(gemv_tma_kernel<WT, NJ, KS, RW>, dim3(grid), dim3(kGvThreads), kGvSmem, st, p, stages, stage_floats);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "gemv_tma: %s", cudaGetErrorString(e));
  return launch_status("gemv_tma");
}

template <typename WT, int KS>
static int launch_gemv_tma_ks(const LinParams &p, int stages, int stage_floats, int nj, cudaStream_t st) {
  switch (nj) {
    case 1: return launch_gemv_tma_nj<WT, 1, KS>(p, stages, stage_floats, st);
    case 2: return launch_gemv_tma_nj<WT, 2, KS>(p, stages, stage_floats, st);
    case 3: return launch_gemv_tma_nj<WT, 3, KS>(p, stages, stage_floats, st);
    case 4: return launch_gemv_tma_nj<WT, 4, KS>(p, stages, stage_floats, st);
    case 6: return launch_gemv_tma_nj<WT, 6, KS>(p, stages, stage_floats, st);
    default: return launch_gemv_tma_nj<WT, 8, KS>(p, stages, stage_floats, st);
  }
}

template <typename WT>
static int launch_gemv_tma(const LinParams &p, int stages, int stage_floats, int nj, int ks, cudaStream_t st) {
  switch (ks) {
    case 1: return launch_gemv_tma_ks<WT, 1>(p, stages, stage_floats, nj, st);
    case 2: return launch_gemv_tma_ks<WT, 2>(p, stages, stage_floats, nj, st);
    default: return launch_gemv_tma_ks<WT, 4>(p, stages, stage_floats, nj, st);
  }
}

// NV = K / (V * 32) vectors per lane when it is one of the instantiated
// counts, else 0 (the general kernel takes the shape).
template <typename WT>
static int gemv_nv(const LinParams &p) {
  constexpr int V = WVec<WT>::n;
  if (p.K % (V * 32)) return 0;
  const int64_t nv = p.K / (V * 32);
  return (nv == 2 || nv == 4 || nv == 6 || nv == 8 || nv == 12 || nv == 16) ? (int)nv : 0;
}

template <typename WT, int NV>
static int launch_gemv_nv(const LinParams &p, cudaStream_t st) {
  const size_t smem = sizeof(float) * (size_t)p.K;
  if (smem > 48 * 1024) cudaFuncSetAttribute(gemv_kernel<WT, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  gemv_kernel<WT, NV><<<(unsigned)((p.N + 3) / 4), 128, smem, st>>>(p);
  return launch_status("gemv");
}

template <typename WT>
static int launch_gemv(const LinParams &p, int nv, cudaStream_t st) {
  switch (nv) {
    case 2: return launch_gemv_nv<WT, 2>(p, st);
    case 4: return launch_gemv_nv<WT, 4>(p, st);
    case 6: return launch_gemv_nv<WT, 6>(p, st);
    case 8: return launch_gemv_nv<WT, 8>(p, st);
    case 12: return launch_gemv_nv<WT, 12>(p, st);
    default: return launch_gemv_nv<WT, 16>(p, st);
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
  // decode matvec fast path: one row, no LayerNorm, aligned x / W, K a
  // multiple of 32 vectors with an instantiated count
  if (p.M == 1 && vec && !(p.flags & SM100_LIN_LN) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0)) {
    int stage_floats = 0, nj = 0, ks = 1;
    const int stages = gemv_tma_stages<WT>(p, stage_floats, nj, ks);
    if (stages >= 2 && p.N >= 1024) return launch_gemv_tma<WT>(p, stages, stage_floats, nj, ks, st);
    const int nv = p.K * sizeof(float) <= 200 * 1024 ? gemv_nv<WT>(p) : 0;
    if (nv) return launch_gemv<WT>(p, nv, st);
  }
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
