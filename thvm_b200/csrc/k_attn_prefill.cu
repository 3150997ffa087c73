// Causal attention prefill in one pass on the 5th-generation tensor cores
// (bf16 Q, K, V [B, H, S, D = 128], f32 O): O = softmax(Q K^T / sqrt(D) +
// causal mask) V.  The reference builds this as scaled_dot_product_attention
// (src/nn/scaled_dot_product_attention.c:1-34): q k^T times 1/sqrt(d), the
// tri / where / -inf causal mask (src/nn/tri.c), softmax (src/nn/softmax.c:
// 1-16: max, x - max, exp, sum, times the reciprocal), then p v.  Here they are
// fused flash style, so the S x S scores never leave the SM.
//
// One CTA per (b*h, pair of 128-query blocks 2t and 2t+1), heaviest pairs
// first.  The two query tiles A and B share one stream of K / V blocks and
// take turns on the tensor cores, so the softmax of one tile runs while the
// products of the other do:
//   warp 0    TMA: Q_A and Q_B once, then K_j and V_j (128 keys each) into
//             2-stage K and V rings (3-D tensor maps [BH, S, D]: rows past S
//             read as zeros); a K slot is refilled once its scores are done;
//   warp 1    MMA: S_X = Q_X K_j^T (tcgen05.mma kind::f16, M = N = 128, both
//             operands K-major in 128-byte-swizzled shared memory) into TMEM,
//             and O_X += P_X V_j with P_X read from TMEM where the softmax
//             wrote it over S_X, V MN-major from shared memory; per block:
//             P_A V, Q_A K_next, P_B V, Q_B K_next;
//   warps 2-5 / 6-9  softmax of tile A / B, one query row per thread (TMEM
//             lane): the score row by tcgen05.ld, causal mask on the diagonal
//             block, row max, P = exp2((s - m) * log2(e) * scale) written back
//             as bf16 pairs by tcgen05.st, the row sum; the running max m is
//             only raised (and O, sum rescaled) when a score exceeds it by
//             8 / (log2(e) * scale), so P <= 2^8 and rescales are rare; at the
//             end O / sum.
// kSplit: P is passed to the tensor cores as bf16 hi + bf16 lo (lo = P -
// hi), two MMAs per key step, so P carries ~16 bits instead of 8: the output
// then agrees with an f32 softmax to ~1e-5 relative and its row-wise argmax
// does not flip on near-ties (a single bf16 P flips ~0.2 % of rows at S=2048).
// The bf16 packing is integer byte permutes, not conversions: the exp2 alone
// fills the SFU pipe.
// Every wait is bounded; a timeout sets g_attn_status.
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kApD = 128, kApBM = 128, kApBN = 128;
constexpr int kApTile = kApBM * kApD * 2;   // 32 KB: one [128 x 128] bf16 tile as two 64-column swizzle halves
constexpr int kApHalf = kApTile / 2;        // 16 KB
constexpr int kApThreads = 18 * 32;
// Q_A, Q_B, K ring, V ring; alignment slack; barriers; the row-half maxima
// (2 parities x 2 tiles x 2 halves x 128 rows) and sums (2 tiles x 2 x 128)
constexpr int kApSmem = 6 * kApTile + 1024 + 256 + (1024 + 512) * 4;

__device__ uint32_t g_attn_status;

__device__ __forceinline__ void ap_tma_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// K-major, 128-byte swizzle: rows of 128 bytes, 8-row atoms of 1024 bytes.
__device__ __forceinline__ uint64_t ap_desc_k(const void *p) {
  const uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// MN-major, 128-byte swizzle, of a [128 K rows][128 N] bf16 tile stored as two
// 64-column halves: leading byte offset = the half stride (16 KB, between
// 64-element N groups), stride byte offset = 8 K rows (1024 bytes).
__device__ __forceinline__ uint64_t ap_desc_mn(const void *p) {
  const uint64_t a = smem_u32(p);
  return ((a >> 4) & 0x3FFFull) | ((uint64_t)(kApHalf >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// bf16 x bf16 -> f32, M = 128, N = 128; B K-major (scores) or MN-major (P V).
constexpr uint32_t kApIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kApBN >> 3) << 17) |
                                ((uint32_t)(kApBM >> 4) << 24);
constexpr uint32_t kApIdescPV = kApIdescQK | (1u << 16);

__device__ __forceinline__ void ap_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}

// The same with A read from TMEM (lane = row of A, bf16 pairs along columns).
__device__ __forceinline__ void ap_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void ap_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define AP_R32(r)                                                                                                    \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),     \
      "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),       \
      "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),      \
      "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define AP_LIST32                                                                                                    \
  "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29," \
  "%30,%31}"

// 32 consecutive f32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void ap_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 " AP_LIST32 ", [%32];" : AP_R32(r) : "r"(taddr));
}

__device__ __forceinline__ void ap_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void ap_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void ap_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void ap_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// Maximum of a 128-score row held as f32 bits: eight independent chains (few
// extra registers while the scores stay live, short dependencies).
__device__ __forceinline__ float ap_max128(const uint32_t (&v)[4][32]) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; k++) a[k] = __uint_as_float(v[0][k]);
#pragma unroll
  for (int i = 8; i < 128; i++) a[i & 7] = fmaxf(a[i & 7], __uint_as_float(v[i >> 5][i & 31]));
  return fmaxf(fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3])), fmaxf(fmaxf(a[4], a[5]), fmaxf(a[6], a[7])));
}

// Named barrier over `count` threads (whole warps).
__device__ __forceinline__ void ap_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// The same, returning the AND of v over the participating threads.
__device__ __forceinline__ bool ap_bar_and(uint32_t id, uint32_t count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %3, 0;\n\tbar.red.and.pred q, %1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(count), "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// Two f32 in one 64-bit register pair, and the sm_100 packed f32x2 arithmetic on them.
__device__ __forceinline__ uint64_t ap_pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void ap_unpack2(uint64_t r, float &a, float &b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ap_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t ap_add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float ap_max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void ap_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void ap_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ap_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ float ap_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A bounded wait whose outcome is the same in every lane of the warp (the
// tcgen05.ld / st that follow are warp-collective).
__device__ __forceinline__ bool ap_wait_warp(uint64_t *bar, uint32_t parity, uint32_t *status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status));
}

template <bool kSplit>
__global__ void __launch_bounds__(kApThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, float *o, int BH, int S, float c_log2, float tau) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char *sq = smem;                 // Q_A, Q_B
  unsigned char *sk = smem + 2 * kApTile;   // K ring (2)
  unsigned char *sv = smem + 4 * kApTile;   // V ring (2)
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 6 * kApTile);
  uint64_t *q_full = bars, *k_full = bars + 1, *k_empty = bars + 3, *v_full = bars + 5, *v_empty = bars + 7;
  uint64_t *s_full = bars + 9, *p_full = bars + 11, *mma_done = bars + 13;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 14);
  float *xmax = reinterpret_cast<float *>(smem + 6 * kApTile + 256), *xsum = xmax + 1024;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (S + kApBM - 1) / kApBM, npairs = (nqb + 1) >> 1;
  const int t = npairs - 1 - (int)(blockIdx.x / BH), bh = (int)(blockIdx.x % BH);   // heaviest pairs first
  const int qbA = 2 * t, qbB = 2 * t + 1;
  const int nA = qbA + 1, nB = qbB < nqb ? qbB + 1 : 0;   // causal key blocks of each tile (B may lie past S)
  const int nK = nB > nA ? nB : nA;
  uint32_t *status = &g_attn_status;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
    }
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {   // TMEM columns: S_A / P_A [0, 128), S_B / P_B [128, 256), O_A [256, 384), O_B [384, 512)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  ap_fence_before();
  __syncthreads();
  ap_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, (nB > 0 ? 2 : 1) * kApTile);
      ap_tma_3d(sq, &map_q, 0, qbA * kApBM, bh, q_full);
      ap_tma_3d(sq + kApHalf, &map_q, 64, qbA * kApBM, bh, q_full);
      if (nB > 0) {
        ap_tma_3d(sq + kApTile, &map_q, 0, qbB * kApBM, bh, q_full);
        ap_tma_3d(sq + kApTile + kApHalf, &map_q, 64, qbB * kApBM, bh, q_full);
      }
      // K_j returns to its ring slot when both tiles' scores against it are
      // done, V_j when both P V products are: K runs up to two blocks ahead of
      // the scores, V two blocks ahead of P V
      int nk = 0, nv = 0;
      for (int j = 0; j < nK; j++) {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)(((j >> 1) - 1) & 1);
        const int y = j * kApBN;
        if (j >= 2 && !mbar_wait(&k_empty[s], ph, status)) break;
        mbar_expect_tx(&k_full[s], kApTile);
        ap_tma_3d(sk + s * kApTile, &map_k, 0, y, bh, &k_full[s]);
        ap_tma_3d(sk + s * kApTile + kApHalf, &map_k, 64, y, bh, &k_full[s]);
        nk++;
        if (j >= 2 && !mbar_wait(&v_empty[s], ph, status)) break;
        mbar_expect_tx(&v_full[s], kApTile);
        ap_tma_3d(sv + s * kApTile, &map_v, 0, y, bh, &v_full[s]);
        ap_tma_3d(sv + s * kApTile + kApHalf, &map_v, 64, y, bh, &v_full[s]);
        nv++;
      }
      // every issued copy has landed before the CTA may exit
      mbar_wait(q_full, 0, status, false);
      for (int i = nk - 2 > 0 ? nk - 2 : 0; i < nk; i++)
        mbar_wait(&k_full[i & 1], (uint32_t)((i >> 1) & 1), status, false);
      for (int i = nv - 2 > 0 ? nv - 2 : 0; i < nv; i++)
        mbar_wait(&v_full[i & 1], (uint32_t)((i >> 1) & 1), status, false);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S_X(j) = Q_X K_j^T into TMEM columns 128X; s_full[X] marks it (and,
      // after a tile's last block, marks its final O)
      auto qk = [&](int X, int j) {
        const unsigned char *kt = sk + (j & 1) * kApTile, *qt = sq + X * kApTile;
#pragma unroll
        for (int kk = 0; kk < kApD / 16; kk++) {
          const int h = kk >> 2, o16 = 2 * (kk & 3);   // 16 elements = 32 bytes = 2 descriptor units
          ap_mma(tmem + (uint32_t)(X * 128), ap_desc_k(qt + h * kApHalf) + o16, ap_desc_k(kt + h * kApHalf) + o16,
                 kApIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, status) && mbar_wait(&k_full[0], 0, status);
      if (ok) {
        ap_fence_after();
        qk(0, 0);
        ap_commit(&s_full[0]);
        if (nB > 0) {
          qk(1, 0);
          ap_commit(&s_full[1]);
        }
        ap_commit(&k_empty[0]);
      }
      for (int j = 0; j < nK && ok; j++) {
        bool v_ready = false, k_ready = false;
        for (int X = 0; X < 2; X++) {
          const int nX = X ? nB : nA;
          if (j >= nX) continue;
          if (!mbar_wait(&p_full[X], (uint32_t)(j & 1), status)) { ok = false; break; }
          if (!v_ready && !(v_ready = mbar_wait(&v_full[j & 1], (uint32_t)((j >> 1) & 1), status))) { ok = false; break; }
          ap_fence_after();
          // O_X += P_X V_j: P from TMEM (bf16 pairs over the S_X columns: hi in
          // [0, 64), lo in [64, 128)), V MN-major from shared memory
          const unsigned char *vt = sv + (j & 1) * kApTile;
          const uint32_t tp = tmem + (uint32_t)(X * 128), to = tmem + 256u + (uint32_t)(X * 128);
#pragma unroll
          for (int kk = 0; kk < kApBN / 16; kk++) {
            const uint64_t dv = ap_desc_mn(vt) + (uint64_t)(kk * (16 * 128) / 16);   // 16 key rows of 128 bytes
            ap_mma_ts(to, tp + (uint32_t)(8 * kk), dv, kApIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
            if constexpr (kSplit) ap_mma_ts(to, tp + 64u + (uint32_t)(8 * kk), dv, kApIdescPV, 1u);
          }
          if (j + 1 < nX) {
            if (!k_ready && !(k_ready = mbar_wait(&k_full[(j + 1) & 1], (uint32_t)(((j + 1) >> 1) & 1), status))) {
              ok = false;
              break;
            }
            ap_fence_after();
            qk(X, j + 1);   // after P_X V_j in the pipe: overwrites P_X only once it is read
          }
          ap_commit(&s_full[X]);
        }
        if (!ok) break;
        ap_commit(&v_empty[j & 1]);
        if (k_ready) ap_commit(&k_empty[(j + 1) & 1]);
      }
      ap_commit(mma_done);
      mbar_wait(mma_done, 0, status, false);
    }
  } else {
    // softmax: warps 2-9 own tile A, 10-17 tile B.  Two threads per query row
    // r = TMEM lane r (a warp may only touch its own 32-lane quarter, warp %
    // 4): half hf of the row's keys (and of its O columns) each.  The halves
    // trade their maxima through shared memory behind a 64-thread named barrier.
    const int X = (warp - 2) >> 3, hf = ((warp - 2) >> 2) & 1, qd = warp & 3, r = qd * 32 + lane;
    const int nX = X ? nB : nA, qbX = X ? qbB : qbA;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
    const uint32_t tS = trow + (uint32_t)(X * 128), tO = trow + 256u + (uint32_t)(X * 128 + 64 * hf);
    const uint32_t bar_id = 1u + (uint32_t)(X * 4 + qd);
    float m = -INFINITY, l = 0.0f;
    bool ok = nX > 0;
    for (int j = 0; j < nX && ok; j++) {
      // both halves of a row leave together: the wait's outcome is combined in
      // the named barrier below (a half that left alone would strand the other)
      const bool got = ap_wait_warp(&s_full[X], (uint32_t)(j & 1), status);
      ap_fence_after();
      uint32_t raw[2][32];
      ap_ld32(tS + (uint32_t)(64 * hf), raw[0]);
      ap_ld32(tS + (uint32_t)(64 * hf + 32), raw[1]);
      ap_wait_ld();
      if (j == qbX) {   // diagonal block: key 64hf + 32c + i of the block is masked above query r
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (64 * hf + 32 * c + i > r) raw[c][i] = __float_as_uint(-INFINITY);
      }
      float mx;
      {   // eight chains of three-input maxima
        float a[8];
#pragma unroll
        for (int k = 0; k < 8; k++) a[k] = __uint_as_float(raw[0][k]);
#pragma unroll
        for (int i = 8; i < 64; i += 16)
#pragma unroll
          for (int k = 0; k < 8; k++)
            a[k] = ap_max3(a[k], __uint_as_float(raw[(i + k) >> 5][(i + k) & 31]),
                           __uint_as_float(raw[(i + 8 + k) >> 5][(i + 8 + k) & 31]));
        mx = ap_max3(ap_max3(a[0], a[1], a[2]), ap_max3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
      }
      xmax[((j & 1) * 2 + X) * 256 + hf * 128 + r] = mx;
      if (!ap_bar_and(bar_id, 64, got)) { ok = false; break; }
      mx = fmaxf(mx, xmax[((j & 1) * 2 + X) * 256 + (hf ^ 1) * 128 + r]);
      if (j == 0) {
        m = mx;   // key 0 is never masked: finite
      } else if (__any_sync(0xffffffffu, mx > m + tau)) {
        // the running maximum is kept until a score exceeds it by tau (P <= 2^8
        // meanwhile); then O and the sum are rescaled (O is stable: the P V of
        // the previous block completed before these scores).  Both halves of a
        // row see the same maximum and decide alike.
        float alpha = 1.0f;
        if (mx > m + tau) {
          alpha = ap_exp2((m - mx) * c_log2);
          m = mx;
        }
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < 8; c++) {   // this half's 64 O columns, 8 at a time
          uint32_t ov[8];
          ap_ld8(tO + (uint32_t)(8 * c), ov);
          ap_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; i++) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          ap_st8(tO + (uint32_t)(8 * c), ov);
        }
      }
      // P = exp2(s * c - m * c): the scale and the sums on packed f32x2 lanes
      // (one instruction per two keys), the exponent on the SFU
      const float nmc = -m * c_log2;
      const uint64_t c2 = ap_pack2(c_log2, c_log2), nm2 = ap_pack2(nmc, nmc), neg2 = ap_pack2(-1.0f, -1.0f);
      uint64_t acc2[2] = {0ull, 0ull};
#pragma unroll
      for (int g = 0; g < 4; g++) {   // keys 64hf + 16g ...: bf16 pairs in columns 32hf + 8g .. (hi), 64 + those (lo)
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int k0 = 16 * g + 2 * i;
          float x0, x1;
          ap_unpack2(ap_fma2(ap_pack2(__uint_as_float(raw[k0 >> 5][k0 & 31]), __uint_as_float(raw[k0 >> 5][(k0 & 31) + 1])),
                             c2, nm2),
                     x0, x1);
          const float p0 = ap_exp2(x0), p1 = ap_exp2(x1);
          const uint64_t pp = ap_pack2(p0, p1);
          acc2[i & 1] = ap_add2(acc2[i & 1], pp);
          const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
          if constexpr (kSplit) {
            // hi = P truncated to bf16 (its upper halves), lo = P - hi (exact in
            // f32, >= 0) truncated to bf16: P to ~2^-15 relative
            hi[i] = __byte_perm(b0, b1, 0x7632);
            float l0, l1;
            ap_unpack2(ap_fma2(ap_pack2(__uint_as_float(b0 & 0xFFFF0000u), __uint_as_float(b1 & 0xFFFF0000u)), neg2, pp),
                       l0, l1);
            lo[i] = __byte_perm(__float_as_uint(l0), __float_as_uint(l1), 0x7632);
          } else {
            hi[i] = __byte_perm(b0 + 0x8000u, b1 + 0x8000u, 0x7632);   // P rounded half-up to bf16
          }
        }
        ap_st8(tS + (uint32_t)(32 * hf + 8 * g), hi);
        if constexpr (kSplit) ap_st8(tS + 64u + (uint32_t)(32 * hf + 8 * g), lo);
      }
      {
        float a0, a1, b0, b1;
        ap_unpack2(acc2[0], a0, a1);
        ap_unpack2(acc2[1], b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      ap_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[X]);
    }
    // the row's sum from both halves, then O / l after the tile's last P V;
    // rows past S are not stored
    if (nX > 0) {
      xsum[X * 256 + hf * 128 + r] = l;
      ap_bar_sync(bar_id, 64);
      l += xsum[X * 256 + (hf ^ 1) * 128 + r];
    }
    if (ok && ap_wait_warp(&s_full[X], (uint32_t)(nX & 1), status)) {
      ap_fence_after();
      // O / l, staged through this tile's Q buffer (its products are all done):
      // 4 KB per warp, 16-byte chunks swizzled by row so that both the row-wise
      // writes and the column-wise reads are free of bank conflicts; each
      // global store instruction then writes four full 128-byte row segments
      const float inv = 1.0f / l;
      float *stage = reinterpret_cast<float *>(sq + X * kApTile) + (hf * 4 + qd) * 1024;
      const int row0 = qbX * kApBM + qd * 32;
#pragma unroll 1
      for (int c = 0; c < 2; c++) {
        uint32_t ov[32];
        ap_ld32(tO + (uint32_t)(32 * c), ov);
        ap_wait_ld();
#pragma unroll
        for (int q = 0; q < 8; q++)
          *reinterpret_cast<float4 *>(stage + lane * 32 + ((q ^ (lane & 7)) * 4)) =
              make_float4(__uint_as_float(ov[4 * q]) * inv, __uint_as_float(ov[4 * q + 1]) * inv,
                          __uint_as_float(ov[4 * q + 2]) * inv, __uint_as_float(ov[4 * q + 3]) * inv);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int rr = (lane >> 3) + 4 * i, ch = lane & 7;
          const float4 v = *reinterpret_cast<const float4 *>(stage + rr * 32 + ((ch ^ (rr & 7)) * 4));
          if (row0 + rr < S)
            *reinterpret_cast<float4 *>(o + ((size_t)bh * S + row0 + rr) * kApD + 64 * hf + 32 * c + 4 * ch) = v;
        }
        __syncwarp();
      }
    }
  }
  ap_fence_before();
  __syncthreads();
  if (warp == 1) {
    ap_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

typedef CUresult (*ApEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                               const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [BH, S, 128] bf16 as a 3-D map, boxes of 64 x 128 x 1 (one swizzle half of a
// 128-row tile); rows at or past S read as zeros.
static bool ap_map(CUtensorMap *m, const void *base, int64_t BH, int64_t S) {
  static ApEncodeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    fn = reinterpret_cast<ApEncodeFn>(p);
  }
  const cuuint64_t dims[3] = {(cuuint64_t)kApD, (cuuint64_t)S, (cuuint64_t)BH};
  const cuuint64_t strides[2] = {(cuuint64_t)kApD * 2, (cuuint64_t)S * kApD * 2};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kSplit>
static int ap_launch(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv, float *o, int BH, int S,
                     float c_log2, cudaStream_t st) {
  cudaError_t e =
      cudaFuncSetAttribute(attn_prefill_kernel<kSplit>, cudaFuncAttributeMaxDynamicSharedMemorySize, kApSmem);
  if (e != cudaSuccess)
    return sm100_set_error(SM100_ERR_CUDA, "attn_prefill: shared memory attribute: %s", cudaGetErrorString(e));
  const int nqb = (S + kApBM - 1) / kApBM;
  const unsigned grid = (unsigned)BH * (unsigned)((nqb + 1) / 2);
  attn_prefill_kernel<kSplit><<<grid, kApThreads, kApSmem, st>>>(mq, mk, mv, o, BH, S, c_log2, 8.0f / c_log2);
  return launch_status("attn_prefill");
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_attn_prefill_bf16(const void *q, const void *k, const void *v, float *o, int32_t B, int32_t H,
                                       int32_t S, int32_t D, float scale, int32_t precise_p, void *stream) {
  if (B == 0 || H == 0 || S == 0) return SM100_OK;   // empty batch: nothing to write
  if (!q || !k || !v || !o || B < 0 || H < 0 || S < 0 || D != kApD || (int64_t)B * H > (1 << 24) ||
      (int64_t)S > (1 << 24) || ((uintptr_t)q & 15) || ((uintptr_t)k & 15) || ((uintptr_t)v & 15) ||
      ((uintptr_t)o & 15) || !(scale > 0.0f && scale < 1e30f))
    return sm100_set_error(SM100_ERR_ARG,
                           "attn_prefill: B %d H %d S %d D %d scale %g (D must be 128, scale > 0; 16-byte aligned)", B,
                           H, S, D, (double)scale);
  const int BH = B * H;
  if ((int64_t)BH * ((S + kApBM - 1) / kApBM) > 0x7FFFFFFF)
    return sm100_set_error(SM100_ERR_ARG, "attn_prefill: grid too large");
  CUtensorMap mq, mk, mv;
  if (!ap_map(&mq, q, BH, S) || !ap_map(&mk, k, BH, S) || !ap_map(&mv, v, BH, S))
    return sm100_set_error(SM100_ERR_CUDA, "attn_prefill: tensor map encoding failed");
  const float c_log2 = scale * 1.4426950408889634f;
  return precise_p ? ap_launch<true>(mq, mk, mv, o, BH, S, c_log2, (cudaStream_t)stream)
                   : ap_launch<false>(mq, mk, mv, o, BH, S, c_log2, (cudaStream_t)stream);
}

extern "C" uint32_t sm100_attn_prefill_status(void) {
  uint32_t v = 0, z = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(v));
  cudaMemcpyToSymbol(g_attn_status, &z, sizeof(z));
  return v;
}
