// Routing of the DeepSeek-V2 MoE decode, shared by the router kernels of
// k_moe.cu and the all-reduce + RMSNorm of k_comm.cu that can end in it.
//
// The rule is the reference's route kernel (bench/dsv2_decode_bench.c:787-863):
// the K largest router LOGITS (ties: lowest expert id), each weighted by its
// softmax probability exp(l - max) / sum (no renormalisation;
// DeepSeek-V2-Lite: norm_topk_prob false, scaling 1); then per-expert lists of
// (token, weight) for the experts [e0, e1) this rank holds, packed
// expert-major: slot_tok / slot_w with slot_off[e] offsets, followed by
// n_shared shared experts that take every token with weight 1.
#pragma once

#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kRtMaxTok = 32;   // decode batch
constexpr int kRtMaxK = 8;      // experts per token
constexpr int kRtMaxE = 64;     // routed experts (two logits per lane)
constexpr int kRtMaxD = 4096;   // model width of the fused norm + router (the row staged in shared memory)

// The router product and routing appended to a per-row norm kernel (one CTA
// of 256 threads per token row); the public struct Sm100DsRoute, as passed.
struct DsRouteArgs {
  const __nv_bfloat16 *router;   // [E][D]
  float *logits;                 // [B][E]
  int32_t *counter;              // CTAs done; the last one packs and leaves it 0
  int32_t *sel;                  // [B][K]
  float *wsel;                   // [B][K]
  int32_t *slot_off;             // [e1 - e0 + n_shared + 1]
  int32_t *slot_tok;             // [B (K + n_shared)]
  float *slot_w;
  int32_t E, K, e0, e1, n_shared;
};

// Host: checks the public routing struct for B rows of width D and copies it
// into out (SM100_OK), else records the error (who: the caller's name).
int ds_route_args(const Sm100DsRoute *r, int B, int D, const char *who, DsRouteArgs *out);

// One token's choices by one warp from its logits held two per lane (l0 =
// logit[lane], l1 = logit[lane + 32]): lane 0 writes sel / wsel (global) and
// s_sel / s_w (shared, may be null).
__device__ __forceinline__ void ds_route_select(float l0, float l1, int E, int K, int32_t *sel, float *wsel,
                                                int32_t *s_sel, float *s_w) {
  const int lane = threadIdx.x & 31;
  float m = fmaxf(lane < E ? l0 : -INFINITY, lane + 32 < E ? l1 : -INFINITY);
  m = warp_max(m);
  float sum = (lane < E ? expf(l0 - m) : 0.0f) + (lane + 32 < E ? expf(l1 - m) : 0.0f);
  sum = warp_sum(sum);
  // greedy top-K over E <= 64 logits held two per lane (a taken or absent
  // expert is out of the contest); a lane offers its larger logit, the
  // lower id on a tie, and the warp keeps the larger, the lower id on a tie
  bool live0 = lane < E, live1 = lane + 32 < E;
  for (int k = 0; k < K; k++) {
    const bool take0 = live0 && (!live1 || l0 >= l1);
    float bv = take0 ? l0 : live1 ? l1 : -INFINITY;
    int bi = take0 ? lane : live1 ? lane + 32 : 0x7FFFFFFF;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    const float w = expf(bv - m) / sum;
    if (lane == 0) {
      if (s_sel) {
        s_sel[k] = bi;
        s_w[k] = w;
      }
      sel[k] = bi;
      wsel[k] = w;
    }
    if (bi == lane) live0 = false;
    if (bi == lane + 32) live1 = false;
  }
}

// Expert-major packing of every token's choices (s_sel / s_w: [B][K] in
// shared memory) by one CTA of >= 256 threads, in entry order (token-major):
// entry i = (token i / K, choice i % K); a warp of entries groups equal
// experts (match), its lowest lane records the group's count, the counts'
// prefix sums give each (warp, expert) its base and an entry its slot: base +
// rank in its group.  The shared experts (local ids e1 - e0 ..) follow.
__device__ __forceinline__ void ds_route_pack(const int32_t *s_sel, const float *s_w, int B, int K, int e0, int e1,
                                              int n_shared, int32_t *slot_off, int32_t *slot_tok, float *slot_w) {
  __shared__ int wcnt[kRtMaxTok * kRtMaxK / 32][kRtMaxE];
  __shared__ int eoff[kRtMaxE + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ne = e1 - e0, n_ent = B * K, nw = (n_ent + 31) / 32;
  for (int i = threadIdx.x; i < nw * kRtMaxE; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  int ent_e = -1, rank = 0;
  if (warp < nw) {
    const int i = warp * 32 + lane;
    const int ex = i < n_ent ? s_sel[i] - e0 : -1;
    ent_e = ex >= 0 && ex < ne ? ex : -1;
    const unsigned mask = __match_any_sync(0xffffffffu, ent_e);
    rank = __popc(mask & ((1u << lane) - 1u));
    if (ent_e >= 0 && rank == 0) wcnt[warp][ent_e] = __popc(mask);
  }
  __syncthreads();
  if (warp == 0) {   // exclusive scan of the expert totals (64 experts, two per lane)
    int c0 = 0, c1 = 0;
    for (int w = 0; w < nw; w++) {
      c0 += 2 * lane < ne ? wcnt[w][2 * lane] : 0;
      c1 += 2 * lane + 1 < ne ? wcnt[w][2 * lane + 1] : 0;
    }
    int incl = c0 + c1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - c0 - c1;
    eoff[2 * lane] = excl;
    eoff[2 * lane + 1] = excl + c0;
    if (lane == 31) eoff[kRtMaxE] = incl;
  }
  __syncthreads();
  if (threadIdx.x <= ne) slot_off[threadIdx.x] = eoff[threadIdx.x];
  if (ent_e >= 0) {
    int o = eoff[ent_e] + rank;
    for (int w = 0; w < warp; w++) o += wcnt[w][ent_e];
    const int i = warp * 32 + lane;
    slot_tok[o] = i / K;
    slot_w[o] = s_w[i];
  }
  // the shared experts (local ids ne ..) take every token with weight 1
  __syncthreads();
  if (n_shared > 0) {
    for (int i = threadIdx.x; i < n_shared * B; i += blockDim.x) {
      const int k = i / B, b = i % B, o = eoff[ne] + i;
      slot_tok[o] = b;
      slot_w[o] = 1.0f;
      if (b == 0) slot_off[ne + k + 1] = eoff[ne] + (k + 1) * B;
    }
  }
}

// A warp's router logit: x (bf16 [D], 16-byte chunks) . w (bf16 [D]) with f32
// sums, lane l taking the chunks l, l + 32, ... in order and the lanes summed
// by the butterfly (the ds_router_route kernel's order, so both give the same
// bits).  xs is shared or global memory.
__device__ __forceinline__ float ds_router_dot(const uint4 *xs, const __nv_bfloat16 *w, int D) {
  const int lane = threadIdx.x & 31;
  float acc = 0.0f;
#pragma unroll 4
  for (int k = lane * 8; k < D; k += 256) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(w + k)), xv = xs[k / 8];
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      acc = fmaf(__uint_as_float(xx[q] << 16), __uint_as_float(ww[q] << 16), acc);
      acc = fmaf(__uint_as_float(xx[q] & 0xFFFF0000u), __uint_as_float(ww[q] & 0xFFFF0000u), acc);
    }
  }
  return warp_sum(acc);
}

// The router weights stream through a ring of kRtStages chunks of 8 experts'
// rows (8 D bf16, contiguous in the [E][D] router) in dynamic shared memory,
// by bulk copies on one mbarrier per stage.
constexpr int kRtStages = 3;
__host__ __device__ constexpr int ds_route_chunk_bytes(int D) { return 8 * D * 2; }
__host__ __device__ constexpr int ds_route_ring_bytes(int D) { return kRtStages * ds_route_chunk_bytes(D); }

__device__ __forceinline__ void ds_route_issue(const DsRouteArgs &a, unsigned char *ring, uint64_t *bars, int D,
                                               int c) {
  const int s = c % kRtStages, ne = min(8, a.E - 8 * c);
  const uint32_t bytes = (uint32_t)(ne * D * 2);
  mbar_expect_tx(&bars[s], bytes);
  bulk_g2s(ring + (size_t)s * ds_route_chunk_bytes(D), a.router + (int64_t)8 * c * D, bytes, &bars[s]);
}

// Before the programmatic-launch wait (the weights do not depend on the
// previous kernel): thread 0 sets up the stage barriers and requests the
// first chunks.  The caller synchronises the CTA before ds_route_row.
__device__ __forceinline__ void ds_route_start(const DsRouteArgs &a, unsigned char *ring, uint64_t *bars, int D) {
  if (threadIdx.x != 0) return;
  for (int s = 0; s < kRtStages; s++) mbar_init(&bars[s], 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const int nch = (a.E + 7) / 8;
  for (int c = 0; c < nch && c < kRtStages; c++) ds_route_issue(a, ring, bars, D, c);
}

// The routing tail of a per-row norm kernel (CTA b of B, 256 threads), after
// ds_route_start, the row's bf16 output staged in shared memory (ys) and a
// CTA barrier: warp w takes expert 8 c + w of chunk c (ds_router_dot's order
// over the weights in shared memory, so the logits are the router kernel's
// bits), warp 0 the row's top-K, and the last CTA to finish (a device
// counter, no waiting) packs every token's choices and resets the counter.
// A stage wait that runs out sets status and gives that chunk's logits NaN.
__device__ __forceinline__ void ds_route_row(const DsRouteArgs &a, const uint4 *ys, unsigned char *ring, uint64_t *bars,
                                             int b, int B, int D, uint32_t *status) {
  __shared__ float s_lg[kRtMaxE];
  __shared__ int32_t s_sel[kRtMaxTok * kRtMaxK];
  __shared__ float s_w[kRtMaxTok * kRtMaxK];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (a.E + 7) / 8;
  for (int c = 0; c < nch; c++) {
    const int s = c % kRtStages, e = 8 * c + warp;
    // every copy is waited for (no early exit on another kernel's error)
    const bool ok = mbar_wait(&bars[s], (uint32_t)((c / kRtStages) & 1), status, false);
    if (e < a.E) {
      const uint4 *wr = reinterpret_cast<const uint4 *>(ring + (size_t)s * ds_route_chunk_bytes(D) + (size_t)warp * D * 2);
      float acc = 0.0f;
#pragma unroll 4
      for (int k = lane * 8; k < D; k += 256) {
        const uint4 wv = wr[k / 8], xv = ys[k / 8];
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          acc = fmaf(__uint_as_float(xx[q] << 16), __uint_as_float(ww[q] << 16), acc);
          acc = fmaf(__uint_as_float(xx[q] & 0xFFFF0000u), __uint_as_float(ww[q] & 0xFFFF0000u), acc);
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) {
        const float l = ok ? acc : __int_as_float(0x7fc00000);
        s_lg[e] = l;
        a.logits[(int64_t)b * a.E + e] = l;
      }
    }
    __syncthreads();   // the stage is read: refill it
    if (threadIdx.x == 0 && c + kRtStages < nch) ds_route_issue(a, ring, bars, D, c + kRtStages);
  }
  // warp 0 chooses; its lane 0 (thread 0) writes the choices and counts the
  // CTA off with a release, so they are visible to whoever acquires the count
  if (warp == 0) {
    const float l0 = lane < a.E ? s_lg[lane] : 0.0f, l1 = lane + 32 < a.E ? s_lg[lane + 32] : 0.0f;
    ds_route_select(l0, l1, a.E, a.K, a.sel + (int64_t)b * a.K, a.wsel + (int64_t)b * a.K, nullptr, nullptr);
    if (lane == 0) {
      int32_t prev;
      asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counter) : "memory");
      s_last = prev == B - 1;
    }
  }
  // the last CTA's thread 0 acquired every CTA's release; the barrier carries
  // that to the CTA's other threads, whose loads go to L2
  __syncthreads();
  if (!s_last) return;
  for (int i = threadIdx.x; i < B * a.K; i += blockDim.x) {
    s_sel[i] = __ldcg(a.sel + i);
    s_w[i] = __ldcg(a.wsel + i);
  }
  __syncthreads();
  ds_route_pack(s_sel, s_w, B, a.K, a.e0, a.e1, a.n_shared, a.slot_off, a.slot_tok, a.slot_w);
  if (threadIdx.x == 0) *a.counter = 0;
}

}  // namespace sm100
