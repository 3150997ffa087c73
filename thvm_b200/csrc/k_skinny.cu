// Skinny bf16 GEMM on the 5th-generation tensor cores for batched decode:
// Y[M, N] = epilogue(X[M, K] . W[N, K]^T) with M <= 32 rows (the decode batch),
// bf16 X and W, f32 accumulate.  This is nn_linear on a [B, 1, K] activation
// (src/nn/linear.c:1-6, py/thvm/nn.py:12-25: W kept (out, in), y = x W^T + b)
// at the batch of BASELINE config 3.  At M = 16 every weight element feeds 16
// products: 50 GFLOP per GPT-2-XL step, beyond the CUDA cores at HBM speed, so
// the products go to tcgen05 with the weight rows as the MMA's M (128) and the
// batch as its N (16 or 32): the tensor pipe idles, HBM streams.
//
// Work: the N x K weight is cut into units of 128 rows x 64 columns (16 KB);
// the U units are split evenly over G (<= 148) persistent CTAs in row-tile-
// major order, so each CTA streams one contiguous run of the weight.  A CTA
// that holds every k-chunk of a row tile finishes it itself; a row tile split
// between CTAs leaves each part's partial sums in a workspace slot, and the
// last part to arrive (per-tile counter) adds the slots in CTA order and
// finishes the tile: deterministic, no floating-point atomics.
//   warp 0    TMA: W chunk [128 x 64] and X chunk [MB x 64] (128-byte swizzle)
//             into a 5-stage ring (two CTAs fit an SM, so with programmatic
//             dependent launch the next GEMM's CTAs prefetch their first
//             weight chunks while this one finishes; activations are read
//             only after griddepcontrol.wait);
//   warp 1    MMA: 4 x tcgen05.mma (M=128, N=MB, K=16) per chunk into one of
//             two TMEM accumulators (a run's epilogue overlaps the next run);
//   warps 2-5 epilogue: tcgen05.ld a 32-row quarter; bias, tanh GELU,
//             residual, f32 or bf16 store, and the KV-cache append of the
//             attention projection's k / v columns.
// SM100_SK_ACCUM skips the split-K finishing: every part adds its sums (and
// the part holding k-chunk 0 the bias) into y with fire-and-forget
// reductions, leaving the remaining epilogue to the consumer kernel.
// SM100_SK_X_GELU takes X as f32 and feeds bf16(gelu(X)) to the MMA, staged in
// shared memory by the epilogue warps before the products start;
// SM100_SK_X_LN likewise feeds bf16(LayerNorm(X)), so the LayerNorm before a
// projection needs no kernel of its own.
// Every wait is bounded; a timeout sets g_skinny_status.
#include <cuda.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kSkBM = 128, kSkBK = 64, kSkStages = 5, kSkThreads = 6 * 32, kSkMaxGrid = 148;
constexpr int kSkWBytes = kSkBM * kSkBK * 2;   // 16 KB

template <int MB>
__host__ __device__ constexpr int sk_stage_bytes() {
  return kSkWBytes + MB * kSkBK * 2;
}
template <int MB>
__host__ __device__ constexpr int sk_smem(int xslots = 0) {
  return kSkStages * sk_stage_bytes<MB>() + xslots * MB * kSkBK * 2 + 1024 + 256;
}

__device__ uint32_t g_skinny_status;

struct SkParams {
  int N, K, M, T, KC, U, G;
  const float *bias;
  const float *residual;
  int64_t ld_res;
  void *y;
  int64_t ld_y;
  int flags;
  float *ws;            // [2 * G][MB][128] partial sums
  uint32_t *counters;   // [T], zero between launches
  // KV append (SM100_SK_KV): columns [C, 2C) are k, [2C, 3C) are v of C = N / 3;
  // cache [2][M][ctx][C] bf16 at row pos
  __nv_bfloat16 *kv;
  const int32_t *pos;
  int kv_ctx;
  // SM100_SK_X_GELU: X is f32 [M, K] (row stride ld_x) and enters the MMA as
  // bf16(gelu(X)), prepared in shared memory by the epilogue warps
  const float *xf;
  int64_t ld_x;
  int xslots;   // X chunks held per CTA (min(KC, most units of a CTA))
  const float *ln_g, *ln_b;   // SM100_SK_X_LN
  float eps;
};

__device__ __forceinline__ void sk_tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t sk_desc(const void *p) {
  const uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Named barrier over `count` threads returning the AND of v over them.
__device__ __forceinline__ bool sk_bar_and(uint32_t id, uint32_t count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %3, 0;\n\tbar.red.and.pred q, %1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(count), "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// first unit of CTA c, and the CTA that holds unit u
__device__ __forceinline__ int sk_u0(int c, int U, int G) { return (int)(((int64_t)c * U) / G); }
__device__ __forceinline__ int sk_cta(int u, int U, int G) { return (int)((((int64_t)u + 1) * G + U - 1) / U) - 1; }

template <int MB>
__device__ __forceinline__ void sk_tmem_ld(uint32_t taddr, float (&v)[MB]) {
  uint32_t r[MB];
  if constexpr (MB == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < MB; i++) v[i] = __uint_as_float(r[i]);
}

// The finished value of output (b, n): bias, GELU, residual, store; and the
// KV-cache copy of k / v columns.
__device__ __forceinline__ void sk_store(const SkParams &p, int b, int n, float v) {
  if (p.bias) v += p.bias[n];
  if (p.flags & SM100_SK_GELU) v = gelu_tanh(v);
  if (p.flags & SM100_SK_RESIDUAL) v += p.residual[(int64_t)b * p.ld_res + n];
  if (p.flags & SM100_SK_OUT_BF16)
    reinterpret_cast<__nv_bfloat16 *>(p.y)[(int64_t)b * p.ld_y + n] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float *>(p.y)[(int64_t)b * p.ld_y + n] = v;
  if (p.flags & SM100_SK_KV) {
    const int C = p.N / 3;
    if (n >= C) {
      const int which = n >= 2 * C ? 1 : 0, c = n - C * (1 + which);
      p.kv[(((int64_t)which * p.M + b) * p.kv_ctx + *p.pos) * C + c] = __float2bfloat16_rn(v);
    }
  }
}

template <int MB>
__global__ void __launch_bounds__(kSkThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                  const SkParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int kStage = sk_stage_bytes<MB>(), kXTile = MB * kSkBK * 2;
  const bool xg = (p.flags & SM100_SK_X_GELU) != 0;
  unsigned char *xs = smem + kSkStages * kStage;   // X_GELU: the CTA's X chunks
  uint64_t *bars = reinterpret_cast<uint64_t *>(xs + (xg ? p.xslots : 0) * kXTile);
  uint64_t *full = bars, *empty = bars + kSkStages, *acc_full = bars + 2 * kSkStages, *acc_empty = acc_full + 2;
  uint64_t *done = acc_empty + 2, *x_ready = done + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(x_ready + 1);
  volatile uint32_t *last_flag = tmem_slot + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, u0 = sk_u0(c, p.U, p.G), u1 = sk_u0(c + 1, p.U, p.G);
  const int kc_first = u0 % p.KC;   // X_GELU: the X chunk of unit u sits in slot (u % KC - kc_first) mod KC
  uint32_t *status = &g_skinny_status;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSkStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 1);
    mbar_init(x_ready, 4);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {   // two accumulators of MB columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * MB)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // the first stages' weights do not depend on earlier kernels: issue them
      // before waiting for the previous grid, their activations after
      const int pre = min(kSkStages, u1 - u0);
      const uint32_t tx = xg ? kSkWBytes : kStage;
      for (int k = 0; k < pre; k++) {
        const int u = u0 + k;
        mbar_expect_tx(&full[k], tx);
        sk_tma_2d(smem + k * kStage, &map_w, (u % p.KC) * kSkBK, (u / p.KC) * kSkBM, &full[k]);
      }
      pdl_wait();
      if (!xg)
        for (int k = 0; k < pre; k++)
          sk_tma_2d(smem + k * kStage + kSkWBytes, &map_x, ((u0 + k) % p.KC) * kSkBK, 0, &full[k]);
      int i = pre;
      for (int u = u0 + pre; u < u1; u++, i++) {
        const int s = i % kSkStages;
        if (i >= kSkStages && !mbar_wait(&empty[s], (uint32_t)(((i / kSkStages) - 1) & 1), status)) break;
        unsigned char *st = smem + s * kStage;
        mbar_expect_tx(&full[s], tx);
        const int t = u / p.KC, kc = u % p.KC;
        sk_tma_2d(st, &map_w, kc * kSkBK, t * kSkBM, &full[s]);
        if (!xg) sk_tma_2d(st + kSkWBytes, &map_x, kc * kSkBK, 0, &full[s]);
      }
      // the copies in flight land before the CTA may exit
      for (int k = i - kSkStages > 0 ? i - kSkStages : 0; k < i; k++)
        mbar_wait(&full[k % kSkStages], (uint32_t)((k / kSkStages) & 1), status, false);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MB >> 3) << 17) |
                                 ((uint32_t)(kSkBM >> 4) << 24);
      int i = 0, run = 0;
      bool ok = !xg || mbar_wait(x_ready, 0, status);
      for (int u = u0; u < u1 && ok; run++) {
        const int t = u / p.KC, uend = min(u1, (t + 1) * p.KC);
        const int a = run & 1;
        if (run >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)(((run >> 1) - 1) & 1), status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int k = u; k < uend; k++, i++) {
          const int s = i % kSkStages;
          if (!mbar_wait(&full[s], (uint32_t)((i / kSkStages) & 1), status)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const unsigned char *st = smem + s * kStage;
          const unsigned char *xt = xg ? xs + ((k % p.KC - kc_first + p.KC) % p.KC) * kXTile : st + kSkWBytes;
#pragma unroll
          for (int kk = 0; kk < kSkBK / 16; kk++) {
            const uint32_t acc = (k > u || kk > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, q;\n\t}" ::"r"(tmem + (uint32_t)(a * MB)),
                "l"(sk_desc(st) + 2 * kk), "l"(sk_desc(xt) + 2 * kk), "r"(idesc), "r"(acc)
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
        u = uend;
      }
      // marks the completion of every product issued
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(done))
                   : "memory");
    }
  } else {
    // epilogue: warp quarter q = warp % 4 reads TMEM lanes 32q .. 32q + 31 = rows of the tile
    pdl_wait();   // residual, outputs and the split-K workspace belong to the previous grid until it is done
    if (xg) {
      // bf16(gelu(X)) of this CTA's chunks in the MMA's K-major 128-byte
      // swizzle: row b, 16-byte chunk c of a 2 KB tile at b * 128 + (c ^ (b & 7)) * 16
      const int et = threadIdx.x - 64, nslots = min(p.KC, u1 - u0);
      for (int sl = 0; sl < nslots; sl++) {
        const int kc = (kc_first + sl) % p.KC;
        for (int e = et; e < MB * 8; e += 128) {
          const int b = e >> 3, ch = e & 7, k0 = kc * kSkBK + ch * 8;
          uint32_t w[4];
#pragma unroll
          for (int j = 0; j < 4; j++) {
            float v0 = 0.0f, v1 = 0.0f;
            if (b < p.M && k0 + 2 * j < p.K) v0 = gelu_tanh(p.xf[(int64_t)b * p.ld_x + k0 + 2 * j]);
            if (b < p.M && k0 + 2 * j + 1 < p.K) v1 = gelu_tanh(p.xf[(int64_t)b * p.ld_x + k0 + 2 * j + 1]);
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
            w[j] = *reinterpret_cast<const uint32_t *>(&h2);
          }
          *reinterpret_cast<uint4 *>(xs + sl * kXTile + b * 128 + ((ch ^ (b & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);
    }
    const int q = warp & 3, row = q * 32 + lane;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    const int Mv = p.M < MB ? p.M : MB;
    int run = 0;
    for (int u = u0; u < u1; run++) {
      const int t = u / p.KC, uend = min(u1, (t + 1) * p.KC);
      const int a = run & 1;
      // the four epilogue warps leave together (they share named barriers below)
      if (!sk_bar_and(2, 128, mbar_wait(&acc_full[a], (uint32_t)((run >> 1) & 1), status))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float v[MB];
      sk_tmem_ld<MB>(tq + (uint32_t)(a * MB), v);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      const int n = t * kSkBM + row;
      if (p.flags & SM100_SK_ACCUM) {
        // y += this run's sums (the run holding k-chunk 0 adds the bias); the
        // reductions are fire-and-forget, the next kernel sees them complete
        if (n < p.N) {
          const float bias = (p.bias && u == t * p.KC) ? p.bias[n] : 0.0f;
          float *yc = reinterpret_cast<float *>(p.y) + n;
#pragma unroll
          for (int b = 0; b < MB; b++)
            if (b < Mv) atomicAdd(yc + (int64_t)b * p.ld_y, v[b] + bias);
        }
      } else if (u == t * p.KC && uend == (t + 1) * p.KC) {   // the whole row tile: finish it here
        if (n < p.N) {
#pragma unroll
          for (int b = 0; b < MB; b++)
            if (b < Mv) sk_store(p, b, n, v[b]);
        }
      } else {
        // a part of the tile: partial sums to this CTA's slot (0: its first
        // tile, 1: its last), then the last part to arrive finishes the tile
        const int slot = 2 * c + (t == u0 / p.KC ? 0 : 1);
        float *w = p.ws + (size_t)slot * MB * kSkBM;
#pragma unroll
        for (int b = 0; b < MB; b++)
          if (b < Mv) w[b * kSkBM + row] = v[b];
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int c_lo = sk_cta(t * p.KC, p.U, p.G), c_hi = sk_cta((t + 1) * p.KC - 1, p.U, p.G);
        if (threadIdx.x == 64) *last_flag = (atomicAdd(&p.counters[t], 1u) == (uint32_t)(c_hi - c_lo)) ? 1u : 0u;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          __threadfence();
          // the parts in CTA order (deterministic); four slots' loads in
          // flight at a time.  A part other than the tile's first starts inside
          // the tile, so the tile is its first (slot 2cc); the first part's
          // slot is 0 only when it starts exactly at the tile.
          float acc[MB];
#pragma unroll
          for (int b = 0; b < MB; b++) acc[b] = 0.0f;
          const int lo_slot = 2 * c_lo + (sk_u0(c_lo, p.U, p.G) < t * p.KC ? 1 : 0);
          auto slot_ptr = [&](int cc) {
            return p.ws + (size_t)(cc == c_lo ? lo_slot : 2 * cc) * MB * kSkBM + row;
          };
          int cc = c_lo;
          for (; cc + 3 <= c_hi; cc += 4) {
            float v4[4][MB];
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const float *ws = slot_ptr(cc + k);
#pragma unroll
              for (int b = 0; b < MB; b++) v4[k][b] = b < Mv ? __ldcg(ws + b * kSkBM) : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
              for (int b = 0; b < MB; b++) acc[b] += v4[k][b];
          }
          for (; cc <= c_hi; cc++) {
            const float *ws = slot_ptr(cc);
#pragma unroll
            for (int b = 0; b < MB; b++)
              if (b < Mv) acc[b] += __ldcg(ws + b * kSkBM);
          }
          if (n < p.N) {
#pragma unroll
            for (int b = 0; b < MB; b++)
              if (b < Mv) sk_store(p, b, n, acc[b]);
          }
          if (threadIdx.x == 64) p.counters[t] = 0u;   // ready for the next launch
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      u = uend;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    // the MMA thread's last commit: every product is done
    if (lane == 0) mbar_wait(done, 0, status, false);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * MB) : "memory");
  }
}


// Cluster split-K (the default path): grid = C clusters x S CTAs.  With S > 1
// each cluster owns one row tile and its S CTAs stream S contiguous parts of
// its k-chunks; each CTA leaves its partial sums in its own shared memory, the
// cluster synchronises, and CTA 0 of the cluster adds the S partials in rank
// order over distributed shared memory (deterministic) and runs the full
// epilogue.  With S = 1 the clusters are single CTAs walking tiles c, c + C...
template <int MB>
__global__ void __launch_bounds__(kSkThreads, 1)
    skinny_cl_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                     const SkParams p, int S) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int kStage = sk_stage_bytes<MB>(), kXTile = MB * kSkBK * 2;
  const bool xln = (p.flags & SM100_SK_X_LN) != 0;
  unsigned char *xs = smem + kSkStages * kStage;   // X_LN: this CTA's k-chunks of bf16(LayerNorm(x))
  uint64_t *bars = reinterpret_cast<uint64_t *>(xs + (xln ? p.xslots : 0) * kXTile);
  uint64_t *full = bars, *empty = bars + kSkStages, *acc_full = bars + 2 * kSkStages, *acc_empty = acc_full + 2;
  uint64_t *done = acc_empty + 2, *x_ready = done + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(x_ready + 1);
  float *pbuf = reinterpret_cast<float *>(smem);   // S > 1: this CTA's partial [MB][128], over ring stage 0
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)(blockIdx.x % S), cl = (int)(blockIdx.x / S), ncl = (int)(gridDim.x / S);
  const int kc0 = (rank * p.KC) / S, kc1 = ((rank + 1) * p.KC) / S, nk = kc1 - kc0;

  uint32_t *status = &g_skinny_status;

  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSkStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 1);
    mbar_init(x_ready, 4);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * MB)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // chunk i of this CTA: tile cl + (i / nk) * ncl, k-chunk kc0 + i % nk
      const int n_tiles = nk > 0 ? (p.T - cl + ncl - 1) / ncl : 0, total = n_tiles * nk;
      const int pre = min(kSkStages, total);
      const uint32_t tx = xln ? kSkWBytes : kStage;
      for (int i = 0; i < pre; i++) {
        mbar_expect_tx(&full[i], tx);
        sk_tma_2d(smem + i * kStage, &map_w, (kc0 + i % nk) * kSkBK, (cl + (i / nk) * ncl) * kSkBM, &full[i]);
      }
      pdl_wait();
      if (!xln)
        for (int i = 0; i < pre; i++)
          sk_tma_2d(smem + i * kStage + kSkWBytes, &map_x, (kc0 + i % nk) * kSkBK, 0, &full[i]);
      int i = pre;
      for (; i < total; i++) {
        const int s = i % kSkStages;
        if (!mbar_wait(&empty[s], (uint32_t)(((i / kSkStages) - 1) & 1), status)) break;
        unsigned char *st = smem + s * kStage;
        mbar_expect_tx(&full[s], tx);
        sk_tma_2d(st, &map_w, (kc0 + i % nk) * kSkBK, (cl + (i / nk) * ncl) * kSkBM, &full[s]);
        if (!xln) sk_tma_2d(st + kSkWBytes, &map_x, (kc0 + i % nk) * kSkBK, 0, &full[s]);
      }
      for (int k = i - kSkStages > 0 ? i - kSkStages : 0; k < i; k++)
        mbar_wait(&full[k % kSkStages], (uint32_t)((k / kSkStages) & 1), status, false);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MB >> 3) << 17) |
                                 ((uint32_t)(kSkBM >> 4) << 24);
      int i = 0, run = 0;
      bool ok = !xln || nk == 0 || mbar_wait(x_ready, 0, status);
      for (int t = cl; t < p.T && nk > 0 && ok; t += ncl, run++) {
        const int a = run & 1;
        if (run >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)(((run >> 1) - 1) & 1), status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int k = 0; k < nk; k++, i++) {
          const int s = i % kSkStages;
          if (!mbar_wait(&full[s], (uint32_t)((i / kSkStages) & 1), status)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const unsigned char *st = smem + s * kStage;
          const unsigned char *xt = xln ? xs + k * kXTile : st + kSkWBytes;
#pragma unroll
          for (int kk = 0; kk < kSkBK / 16; kk++) {
            const uint32_t acc = (k > 0 || kk > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, q;\n\t}" ::"r"(tmem + (uint32_t)(a * MB)),
                "l"(sk_desc(st) + 2 * kk), "l"(sk_desc(xt) + 2 * kk), "r"(idesc), "r"(acc)
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
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(done))
                   : "memory");
    }
  } else {
    pdl_wait();
    if (xln && nk > 0) {
      // bf16(LayerNorm(x) * g + b) of this CTA's k-chunks, in the MMA's K-major
      // 128-byte swizzle (row b, 16-byte chunk c of a tile at b * 128 + (c ^ (b & 7)) * 16).
      // Statistics over the whole row as src/nn/layernorm.c:1-7: mean = sum *
      // (1/K), var = sum((x - mean)^2) * (1/K), 1/sqrt(var + eps); a warp per row.
      const float inv_k = 1.0f / (float)p.K;
      for (int b = warp - 2; b < MB; b += 4) {
        const float *xr = p.xf + (int64_t)b * p.ld_x;
        float mean = 0.0f, r = 0.0f;
        if (b < p.M) {
          float s1 = 0.0f;
          for (int k = lane; k < p.K; k += 32) s1 += xr[k];
          mean = warp_sum(s1) * inv_k;
          float s2 = 0.0f;
          for (int k = lane; k < p.K; k += 32) {
            const float d = xr[k] - mean;
            s2 += d * d;
          }
          r = 1.0f / sqrtf(warp_sum(s2) * inv_k + p.eps);
        }
        for (int e = lane; e < nk * 8; e += 32) {   // 16-byte chunks: 8 per k-chunk
          const int kc = e >> 3, ch = e & 7, k0 = (kc0 + kc) * kSkBK + ch * 8;
          uint32_t w[4];
#pragma unroll
          for (int j = 0; j < 4; j++) {
            float v0 = 0.0f, v1 = 0.0f;
            const int ka = k0 + 2 * j, kb = ka + 1;
            if (b < p.M && ka < p.K) v0 = (xr[ka] - mean) * r * p.ln_g[ka] + p.ln_b[ka];
            if (b < p.M && kb < p.K) v1 = (xr[kb] - mean) * r * p.ln_g[kb] + p.ln_b[kb];
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
            w[j] = *reinterpret_cast<const uint32_t *>(&h2);
          }
          *reinterpret_cast<uint4 *>(xs + kc * kXTile + b * 128 + ((ch ^ (b & 7)) * 16)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);
    }
    const int q = warp & 3, row = q * 32 + lane;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    const int Mv = p.M < MB ? p.M : MB;
    int run = 0;
    for (int t = cl; t < p.T && nk > 0; t += ncl, run++) {
      const int a = run & 1;
      if (!sk_bar_and(2, 128, mbar_wait(&acc_full[a], (uint32_t)((run >> 1) & 1), status))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float v[MB];
      sk_tmem_ld<MB>(tq + (uint32_t)(a * MB), v);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      const int n = t * kSkBM + row;
      if (S == 1) {
        if (n < p.N) {
#pragma unroll
          for (int b = 0; b < MB; b++)
            if (b < Mv) sk_store(p, b, n, v[b]);
        }
      } else {
        // the ring is idle now (all products done): the partial goes over stage 0
#pragma unroll
        for (int b = 0; b < MB; b++) pbuf[b * kSkBM + row] = v[b];
      }
    }
    if (nk == 0 && S > 1)   // an empty part contributes zeros
      for (int b = 0; b < MB; b++) pbuf[b * kSkBM + row] = 0.0f;
  }
  if (S > 1) {
    // every CTA of the cluster has its partial in shared memory (warps
    // reconverge first: the cluster barrier is warp-aligned)
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (warp >= 2) {
      // every CTA of the cluster folds a slice of the tile's rows: partial r
      // of (row, b) from CTA r, added in rank order (deterministic); the S
      // loads of an element are issued before its adds
      const int r0 = (rank * kSkBM) / S, nr = ((rank + 1) * kSkBM) / S - r0;
      const int Mv = p.M < MB ? p.M : MB;
      const uint32_t local = smem_u32(pbuf);
      uint32_t base[8];
#pragma unroll
      for (int r = 0; r < 8; r++)
        if (r < S) asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(base[r]) : "r"(local), "r"(r));
      for (int idx = threadIdx.x - 64; idx < nr * Mv; idx += 128) {
        const int b = idx / nr, row = r0 + idx % nr, n = cl * kSkBM + row;
        const uint32_t off = (uint32_t)((b * kSkBM + row) * 4);
        float x[8];
#pragma unroll
        for (int r = 0; r < 8; r++)
          if (r < S) asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x[r]) : "r"(base[r] + off));
        float acc = 0.0f;
#pragma unroll
        for (int r = 0; r < 8; r++)
          if (r < S) acc += x[r];
        if (n < p.N) sk_store(p, b, n, acc);
      }
    }
    // the partials stay readable until every CTA is done with them
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait(done, 0, status, false);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * MB) : "memory");
  }
}

typedef CUresult (*SkEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                               const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows, cols] bf16 row-major (row stride ld elements), boxes of 64 x box_rows.
static bool sk_map(CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  static SkEncodeFn fn = nullptr;
  if (!fn) {
    void *q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) != cudaSuccess ||
        r != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<SkEncodeFn>(q);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kSkBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MB>
static int sk_launch(const Sm100SkinnyArgs *a, cudaStream_t st) {
  SkParams p;
  p.N = (int)a->N;
  p.K = (int)a->K;
  p.M = (int)a->M;
  p.T = (p.N + kSkBM - 1) / kSkBM;
  p.KC = (p.K + kSkBK - 1) / kSkBK;
  p.U = p.T * p.KC;
  p.G = p.U < kSkMaxGrid ? p.U : kSkMaxGrid;
  p.bias = a->bias;
  p.residual = a->residual;
  p.ld_res = a->ld_res ? a->ld_res : a->N;
  p.y = a->y;
  p.ld_y = a->ld_y ? a->ld_y : a->N;
  p.flags = a->flags;
  p.ws = a->ws;
  p.counters = a->counters;
  p.kv = reinterpret_cast<__nv_bfloat16 *>(a->kv_cache);
  p.pos = a->pos;
  p.kv_ctx = a->kv_ctx;
  p.xf = reinterpret_cast<const float *>(a->x);
  p.ld_x = a->ld_x ? a->ld_x : a->K;
  p.xslots = (a->flags & SM100_SK_X_GELU) ? std::min(p.KC, (p.U + p.G - 1) / p.G) : 0;
  CUtensorMap mw, mx;
  memset(&mx, 0, sizeof mx);
  if (!sk_map(&mw, a->w, a->N, a->K, a->ld_w ? a->ld_w : a->K, kSkBM) ||
      (!(a->flags & (SM100_SK_X_GELU | SM100_SK_X_LN)) &&
       !sk_map(&mx, a->x, a->M, a->K, a->ld_x ? a->ld_x : a->K, MB)))
    return sm100_set_error(SM100_ERR_CUDA, "skinny: tensor map encoding failed");
  if (!(a->flags & (SM100_SK_ACCUM | SM100_SK_X_GELU))) {
    // cluster split-K: S parts per row tile so that T x S fills the SMs (S <= 8)
    const int S = std::max(1, std::min(8, kSkMaxGrid / p.T));
    const int ncl = S > 1 ? p.T : std::min(p.T, kSkMaxGrid);
    p.xslots = (a->flags & SM100_SK_X_LN) ? (p.KC + S - 1) / S : 0;
    p.ln_g = a->ln_g;
    p.ln_b = a->ln_b;
    p.eps = a->eps;
    const int smem = sk_smem<MB>(p.xslots);
    if (smem > 227 * 1024) return sm100_set_error(SM100_ERR_ARG, "skinny: %d LayerNorm chunks do not fit", p.xslots);
    cudaError_t e = cudaFuncSetAttribute(skinny_cl_kernel<MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "skinny: smem attribute: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ncl * S);
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)S;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, skinny_cl_kernel<MB>, mw, mx, p, S);
    if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "skinny: launch: %s", cudaGetErrorString(e));
    return launch_status("skinny");
  }
  const int smem = sk_smem<MB>(p.xslots);
  if (smem > 227 * 1024) return sm100_set_error(SM100_ERR_ARG, "skinny: %d X chunks do not fit", p.xslots);
  cudaError_t e = cudaFuncSetAttribute(skinny_kernel<MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "skinny: smem attribute: %s", cudaGetErrorString(e));
  e = launch_pdl(skinny_kernel<MB>, dim3(p.G), dim3(kSkThreads), smem, st, mw, mx, p);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "skinny: launch: %s", cudaGetErrorString(e));
  return launch_status("skinny");
}

}  // namespace sm100

using namespace sm100;

extern "C" uint64_t sm100_skinny_ws_bytes(int32_t M) { return (uint64_t)2 * kSkMaxGrid * (M <= 16 ? 16 : 32) * kSkBM * 4; }

extern "C" int sm100_skinny_bf16(const Sm100SkinnyArgs *a, void *stream) {
  if (!a || !a->x || !a->w || !a->y || a->M < 1 || a->M > 32 || a->N < 1 || a->K < 1 || a->N > (1 << 30) ||
      a->K > (1 << 30) || (a->K % 8) || ((a->ld_w ? a->ld_w : a->K) % 8) || ((a->ld_x ? a->ld_x : a->K) % 8) ||
      ((uintptr_t)a->x & 15) || ((uintptr_t)a->w & 15) || !a->ws || !a->counters ||
      ((a->flags & SM100_SK_RESIDUAL) && !a->residual) ||
      ((a->flags & SM100_SK_KV) && (!a->kv_cache || !a->pos || a->kv_ctx < 1 || a->N % 3)) ||
      ((a->flags & SM100_SK_ACCUM) && (a->flags & (SM100_SK_GELU | SM100_SK_RESIDUAL | SM100_SK_OUT_BF16 | SM100_SK_KV))) ||
      ((a->flags & SM100_SK_X_GELU) && ((uintptr_t)a->x & 3)) ||
      ((a->flags & SM100_SK_X_LN) && (!a->ln_g || !a->ln_b || (a->flags & (SM100_SK_ACCUM | SM100_SK_X_GELU)))))
    return sm100_set_error(SM100_ERR_ARG, "skinny: M %lld N %lld K %lld (M <= 32, K %% 8 == 0, aligned, workspace)",
                           (long long)(a ? a->M : 0), (long long)(a ? a->N : 0), (long long)(a ? a->K : 0));
  return a->M <= 16 ? sk_launch<16>(a, (cudaStream_t)stream) : sk_launch<32>(a, (cudaStream_t)stream);
}

extern "C" uint32_t sm100_skinny_status(void) {
  uint32_t v = 0, z = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_skinny_status, sizeof(v));
  cudaMemcpyToSymbol(g_skinny_status, &z, sizeof(z));
  return v;
}
