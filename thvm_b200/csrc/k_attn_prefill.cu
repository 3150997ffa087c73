// Causal attention prefill in one pass on the 5th-generation tensor cores
// (bf16 Q, K, V [B, H, S, D = 128], f32 O): O = softmax(Q K^T / sqrt(D) +
// causal mask) V.  The reference builds this as scaled_dot_product_attention
// (src/nn/scaled_dot_product_attention.c:1-34): q k^T times 1/sqrt(d), the
// tri / where / -inf causal mask (src/nn/tri.c), softmax (src/nn/softmax.c:
// 1-16: max, x - max, exp, sum, times the reciprocal), then p v.  Here they are
// fused flash style, so the S x S scores never leave the SM.
//
// One CTA per (b*h, 128-query block), heaviest query blocks first:
//   warp 0    TMA: Q once, then K_j and V_j (128 keys each) into a 2-stage
//             ring (3-D tensor maps [BH, S, D]: rows past S read as zeros);
//   warp 1    MMA: S_j = Q K_j^T (tcgen05.mma kind::f16, M = N = 128, both
//             operands K-major, 128-byte swizzle) into one of two TMEM score
//             buffers, and O += P_j V_j (P K-major from shared memory, V
//             MN-major) into a TMEM accumulator; QK of block j+1 is issued
//             before PV of block j, so the scores of the next block are ready
//             when the softmax of this one ends;
//   warps 2-5 softmax, one query row per thread (TMEM lane): the score row by
//             tcgen05.ld, causal mask on the diagonal block, online max and
//             sum, P = exp2((s - max) * log2(e) / sqrt(D)), the O rescale in
//             TMEM when a row maximum grew, P into shared memory in the MMA's
//             swizzled layout; at the end O / sum.
// kSplit: P is passed to the tensor cores as bf16 hi + bf16 lo (lo = P -
// hi), two MMAs per key step, so P carries ~16 bits instead of 8: the output
// then agrees with an f32 softmax to ~2e-6 relative and its row-wise argmax
// does not flip on near-ties (a single bf16 P flips ~0.2 % of rows at S=2048).
// Every wait is bounded; a timeout sets g_attn_status.
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kApD = 128, kApBM = 128, kApBN = 128;
constexpr int kApTile = kApBM * kApD * 2;   // 32 KB: one [128 x 128] bf16 tile as two 64-column swizzle halves
constexpr int kApHalf = kApTile / 2;        // 16 KB
constexpr int kApThreads = 6 * 32;

template <bool kSplit>
constexpr int ap_smem() {
  return (kSplit ? 7 : 6) * kApTile + 1024 + 256;
}

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

__device__ __forceinline__ void ap_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void ap_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ap_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ float ap_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// A bounded wait whose outcome is the same in every lane of the warp (the
// tcgen05.ld / st that follow are warp-collective).
__device__ __forceinline__ bool ap_wait_warp(uint64_t *bar, uint32_t parity, uint32_t *status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status));
}

template <bool kSplit>
__global__ void __launch_bounds__(kApThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, float *o, int BH, int S, float c_log2) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int kTiles = kSplit ? 7 : 6;
  unsigned char *sq = smem;                 // Q
  unsigned char *skv = smem + kApTile;      // K0, V0, K1, V1
  unsigned char *sp = smem + 5 * kApTile;   // P (hi), then P lo when split
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kTiles * kApTile);
  uint64_t *q_full = bars, *kv_full = bars + 1, *kv_empty = bars + 3, *s_full = bars + 5, *s_empty = bars + 7;
  uint64_t *p_full = bars + 9, *pv_done = bars + 10, *mma_done = bars + 11;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (S + kApBM - 1) / kApBM;
  const int qb = nqb - 1 - (int)(blockIdx.x / BH), bh = (int)(blockIdx.x % BH);   // heaviest first
  const int nb = qb + 1;                                                           // causal key blocks
  uint32_t *status = &g_attn_status;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {   // TMEM: S0 columns [0, 128), S1 [128, 256), O [256, 384)
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
      mbar_expect_tx(q_full, kApTile);
      ap_tma_3d(sq, &map_q, 0, qb * kApBM, bh, q_full);
      ap_tma_3d(sq + kApHalf, &map_q, 64, qb * kApBM, bh, q_full);
      int j = 0;
      for (; j < nb; j++) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], (uint32_t)(((j >> 1) - 1) & 1), status)) break;
        unsigned char *sk = skv + (size_t)s * 2 * kApTile, *sv = sk + kApTile;
        mbar_expect_tx(&kv_full[s], 2 * kApTile);
        const int y = j * kApBN;
        ap_tma_3d(sk, &map_k, 0, y, bh, &kv_full[s]);
        ap_tma_3d(sk + kApHalf, &map_k, 64, y, bh, &kv_full[s]);
        ap_tma_3d(sv, &map_v, 0, y, bh, &kv_full[s]);
        ap_tma_3d(sv + kApHalf, &map_v, 64, y, bh, &kv_full[s]);
      }
      // every issued copy has landed before the CTA may exit
      mbar_wait(q_full, 0, status, false);
      for (int i = j - 2 > 0 ? j - 2 : 0; i < j; i++)
        mbar_wait(&kv_full[i & 1], (uint32_t)((i >> 1) & 1), status, false);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, status);
      ap_fence_after();
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&kv_full[s], (uint32_t)((j >> 1) & 1), status)) return false;
        if (j >= 2 && !mbar_wait(&s_empty[s], (uint32_t)(((j >> 1) - 1) & 1), status)) return false;
        ap_fence_after();
        const unsigned char *sk = skv + (size_t)s * 2 * kApTile;
#pragma unroll
        for (int kk = 0; kk < kApD / 16; kk++) {
          const int h = kk >> 2, o16 = 2 * (kk & 3);   // 16 elements = 32 bytes = 2 descriptor units
          ap_mma(tmem + (uint32_t)(s * kApBN), ap_desc_k(sq + h * kApHalf) + o16, ap_desc_k(sk + h * kApHalf) + o16,
                 kApIdescQK, kk > 0 ? 1u : 0u);
        }
        ap_commit(&s_full[s]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; j < nb && ok; j++) {
        if (j + 1 < nb && !issue_qk(j + 1)) break;
        if (!mbar_wait(p_full, (uint32_t)(j & 1), status)) break;   // P_j written, O rescaled
        ap_fence_after();
        const unsigned char *sv = skv + (size_t)(j & 1) * 2 * kApTile + kApTile;
#pragma unroll
        for (int kk = 0; kk < kApBN / 16; kk++) {
          const int h = kk >> 2, o16 = 2 * (kk & 3);
          const uint64_t dv = ap_desc_mn(sv) + (uint64_t)(kk * (16 * 128) / 16);   // 16 key rows of 128 bytes
          ap_mma(tmem + 256u, ap_desc_k(sp + h * kApHalf) + o16, dv, kApIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
          if (kSplit) ap_mma(tmem + 256u, ap_desc_k(sp + kApTile + h * kApHalf) + o16, dv, kApIdescPV, 1u);
        }
        ap_commit(pv_done);
        ap_commit(&kv_empty[j & 1]);
      }
      ap_commit(mma_done);
      mbar_wait(mma_done, 0, status, false);
    }
  } else {
    // softmax: thread = query row r = TMEM lane r; a warp may only touch its
    // own 32-lane quarter of TMEM (warp % 4)
    const int qd = warp & 3, r = qd * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nb; j++) {
      const int s = j & 1;
      if (!ap_wait_warp(&s_full[s], (uint32_t)((j >> 1) & 1), status)) { ok = false; break; }
      ap_fence_after();
      uint32_t raw[4][32];
#pragma unroll
      for (int c = 0; c < 4; c++) ap_ld32(trow + (uint32_t)(s * kApBN + 32 * c), raw[c]);
      ap_wait_ld();
      ap_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[s]);
      float sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; c++)
#pragma unroll
        for (int i = 0; i < 32; i++) sv[c][i] = __uint_as_float(raw[c][i]);
      if (j == qb) {   // diagonal block: key 32c + i of this block is masked above query r
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int i = 0; i < 32; i++)
            if (32 * c + i > r) sv[c][i] = -INFINITY;
      }
      float mx = m;
#pragma unroll
      for (int c = 0; c < 4; c++)
#pragma unroll
        for (int i = 0; i < 32; i++) mx = fmaxf(mx, sv[c][i]);
      const float nmc = -mx * c_log2;
      const float alpha = ap_exp2(fmaf(m, c_log2, nmc));   // 0 on the first block (m = -inf)
      float sum = 0.0f;
      uint32_t phi[64], plo[kSplit ? 64 : 1];
#pragma unroll
      for (int c = 0; c < 4; c++)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = ap_exp2(fmaf(sv[c][i], c_log2, nmc)), p1 = ap_exp2(fmaf(sv[c][i + 1], c_log2, nmc));
          sum += p0 + p1;
          const uint32_t h = pack_bf16(p0, p1);
          phi[(32 * c + i) >> 1] = h;
          if (kSplit)
            plo[(32 * c + i) >> 1] = pack_bf16(p0 - __uint_as_float(h << 16), p1 - __uint_as_float(h & 0xFFFF0000u));
        }
      l = fmaf(l, alpha, sum);
      // PV of the previous block done: O is stable and the P buffer free
      if (j > 0) {
        if (!ap_wait_warp(pv_done, (uint32_t)((j - 1) & 1), status)) { ok = false; break; }
        ap_fence_after();
        if (__any_sync(0xffffffffu, mx > m)) {   // rescale the O row by alpha (1 where the max held)
#pragma unroll 1
          for (int c = 0; c < 4; c++) {
            uint32_t ov[32];
            ap_ld32(trow + 256u + (uint32_t)(32 * c), ov);
            ap_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            ap_st32(trow + 256u + (uint32_t)(32 * c), ov);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
      }
      m = mx;
      // P row r in the K-major 128-byte swizzle: 16-byte chunk c of half h at
      // r * 128 + ((c ^ (r & 7)) * 16)
#pragma unroll
      for (int h = 0; h < 2; h++)
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const int w = h * 32 + c * 4;   // packed pairs of keys 64h + 8c ...
          const int off = h * kApHalf + r * 128 + ((c ^ (r & 7)) * 16);
          *reinterpret_cast<uint4 *>(sp + off) = make_uint4(phi[w], phi[w + 1], phi[w + 2], phi[w + 3]);
          if (kSplit)
            *reinterpret_cast<uint4 *>(sp + kApTile + off) = make_uint4(plo[w], plo[w + 1], plo[w + 2], plo[w + 3]);
        }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      ap_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // O / l once the last PV is done; rows past S are not stored
    if (ok && ap_wait_warp(pv_done, (uint32_t)((nb - 1) & 1), status)) {
      ap_fence_after();
      const float inv = 1.0f / l;
      const int qrow = qb * kApBM + r;
      float *orow = o + ((size_t)bh * S + qrow) * kApD;
#pragma unroll 1
      for (int c = 0; c < 4; c++) {
        uint32_t ov[32];
        ap_ld32(trow + 256u + (uint32_t)(32 * c), ov);
        ap_wait_ld();
        if (qrow < S) {
          float4 *dst = reinterpret_cast<float4 *>(orow + 32 * c);
#pragma unroll
          for (int i = 0; i < 8; i++)
            dst[i] = make_float4(__uint_as_float(ov[4 * i]) * inv, __uint_as_float(ov[4 * i + 1]) * inv,
                                 __uint_as_float(ov[4 * i + 2]) * inv, __uint_as_float(ov[4 * i + 3]) * inv);
        }
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
  constexpr int smem = ap_smem<kSplit>();
  cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel<kSplit>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess)
    return sm100_set_error(SM100_ERR_CUDA, "attn_prefill: shared memory attribute: %s", cudaGetErrorString(e));
  const unsigned grid = (unsigned)BH * (unsigned)((S + kApBM - 1) / kApBM);
  attn_prefill_kernel<kSplit><<<grid, kApThreads, smem, st>>>(mq, mk, mv, o, BH, S, c_log2);
  return launch_status("attn_prefill");
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_attn_prefill_bf16(const void *q, const void *k, const void *v, float *o, int32_t B, int32_t H,
                                       int32_t S, int32_t D, float scale, int32_t precise_p, void *stream) {
  if (B == 0 || H == 0 || S == 0) return SM100_OK;   // empty batch: nothing to write
  if (!q || !k || !v || !o || B < 0 || H < 0 || S < 0 || D != kApD || (int64_t)B * H > (1 << 24) ||
      (int64_t)S > (1 << 24) || ((uintptr_t)q & 15) || ((uintptr_t)k & 15) || ((uintptr_t)v & 15) ||
      ((uintptr_t)o & 15))
    return sm100_set_error(SM100_ERR_ARG, "attn_prefill: B %d H %d S %d D %d (D must be 128; 16-byte aligned)", B, H,
                           S, D);
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
