// Routing of the DeepSeek-V2 MoE decode: the pieces of the router kernels of
// k_moe.cu.
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

namespace sm100 {

constexpr int kRtMaxTok = 32;   // decode batch
constexpr int kRtMaxK = 8;      // experts per token
constexpr int kRtMaxE = 64;     // routed experts (two logits per lane)
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

}  // namespace sm100
