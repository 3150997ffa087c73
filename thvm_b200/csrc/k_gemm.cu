// Dense bf16 GEMM on the 5th-generation tensor cores: C[M, N] (f32) =
// A[M, K] (bf16) . B[N, K]^T (bf16), f32 accumulate.  Both operands K-major,
// as nn.Linear keeps its weight (out, in) and nn_dot contracts the last axis
// (src/nn/dot.c:1-20, src/nn/linear.c:1-6); the reference renders this shape
// as a WMMA 16x16x16 kernel (src/codegen/render_uop.c:1784-1986).
//
// One persistent CTA per SM, warp-specialised, tiles of 256 x 256:
//   warp 0  TMA producer: 2-D tensor copies (cp.async.bulk.tensor, 128-byte
//           swizzle, no multicast) of A [256 x 64] and B [256 x 64] k-blocks
//           into a 3-stage shared-memory ring (64 KB per stage);
//   warp 1  MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16,
//           kind::f16, bf16 in / f32 accumulate) for each 128-row half of
//           the A block against the same B block, four K steps per k-block,
//           into the two halves of TMEM (columns [0, 256) and [256, 512)),
//           then tcgen05.commit frees the stage; the tile's last commit
//           signals the epilogue;
//   warps 2-9 epilogue: tcgen05.ld both accumulators (a warp its 32-lane
//           quarter = 32 rows of each half, and half of the columns), each
//           32 x 32 block through the warp's 4 KB of shared memory (a lane
//           writes its row, then reads four columns of eight rows), so the
//           global stores are whole 128-byte rows (f32; 64 bytes bf16).
// A 256 x 256 tile reads 64 KB of operands per k-block for 8.4 MFLOP, a
// third less per FLOP than a 128 x 256 tile, which is what bounds the
// product at these sizes (L2 -> shared-memory traffic).  The two halves fill
// TMEM, so the next tile's products wait for the epilogue to drain it (eight
// epilogue warps keep that short).  Tiles are walked round-robin over the
// CTAs; when the last round would leave at least half the CTAs idle, its
// tiles are cut into 128 x 256 halves (one product chain each), so up to
// twice as many CTAs share it.
//
// Every wait is bounded: a timeout sets a status word (sm100_gemm_status)
// and the kernel runs to its end.  Shapes: M % 128 == 0, N % 256 == 0,
// K % 64 == 0, 16-byte aligned rows (a last tile row of 128 reads zeros past
// M and stores only its rows).
#include <cuda.h>

#include "common.cuh"
#include "tma.cuh"

namespace sm100 {

constexpr int kGmBM = 128, kGmBN = 256, kGmBK = 64;   // one MMA's M and N; BK = one 128-byte swizzle row of bf16
constexpr int kGmTM = 2 * kGmBM;                        // tile rows: two MMA halves
constexpr int kGmStages = 3;
constexpr int kGmABytes = kGmTM * kGmBK * 2;          // 32 KB
constexpr int kGmBBytes = kGmBN * kGmBK * 2;          // 32 KB
constexpr int kGmStageBytes = kGmABytes + kGmBBytes;
constexpr int kGmEpiWarps = 8;
constexpr int kGmThreads = (2 + kGmEpiWarps) * 32;
constexpr int kGmTmemCols = 2 * kGmBN;                 // the two halves' accumulators
constexpr int kGmStageF = 32 * 32;                     // one epilogue warp's staging block: 32 rows x 32 f32
constexpr int kGmSmem = kGmStages * kGmStageBytes + 1024 /* alignment */ + 256 /* barriers */ +
                        kGmEpiWarps * kGmStageF * 4 /* epilogue staging */;

__device__ uint32_t g_gemm_status;   // set when a bounded wait gave up

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor of a K-major tile with the 128-byte swizzle:
// rows of 128 bytes, 8-row atoms of 1024 bytes stacked contiguously (stride
// byte offset 1024), version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;          // start address (16-byte units)
  d |= (uint64_t)1 << 16;                // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;      // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 A and B, f32 D, K-major both, M = 128, N = 256.
constexpr uint32_t kGmIdesc = (1u << 4)              // D format f32
                              | (1u << 7)            // A bf16
                              | (1u << 10)           // B bf16
                              | ((uint32_t)(kGmBN >> 3) << 17) | ((uint32_t)(kGmBM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kGmIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Work item i: below n_full a whole 256 x 256 tile (row-major tile order);
// past it the remaining tiles in 128-row halves (item n_full + 2 j + h: half
// h of tile n_full + j).  First row r0 and rows (256 or 128).
struct GmItem {
  int r0, tn, rows;
};
__device__ __forceinline__ GmItem gm_item(int item, int tiles_n, int n_full) {
  int tile = item, h = -1;
  if (item >= n_full) {
    tile = n_full + (item - n_full) / 2;
    h = (item - n_full) % 2;
  }
  GmItem r;
  r.r0 = (tile / tiles_n) * kGmTM + (h > 0 ? kGmBM : 0);
  r.tn = tile % tiles_n;
  r.rows = h < 0 ? kGmTM : kGmBM;
  return r;
}

// GELU, tanh form, as x sigmoid(2 u) = x / (1 + e^(-2 u)) with u = sqrt(2/pi)
// (x + 0.044715 x^3) (the same function: 0.5 (1 + tanh u) = sigmoid(2 u)),
// on the fast exponential: ~1e-6 relative, far below the bf16 rounding of
// the products it feeds, and a few instructions where the bit-exact form of
// the fp32 decode path (common.cuh gelu_tanh) takes dozens, which would leave
// the tensor cores idle behind the epilogue.
__device__ __forceinline__ float gm_gelu(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return __fdividef(x, 1.0f + __expf(-2.0f * fmaxf(u, -40.0f)));
}

// The fused epilogue of sm100_gemm_bf16_ep on columns col .. col + 3 of rows
// row0 + 4 i, i < 8 (N % 4 == 0, so the four columns are all below N or
// none): bias, GELU, residual, then an f32 or bf16 store; the order of the
// skinny GEMM's epilogue (k_skinny.cu).  Every load is issued before the
// first store (the residual may be the output itself, so the compiler could
// not move them across the stores).
__device__ __forceinline__ void gm_epilogue4x8(float4 (&v)[8], void *c, const float *bias, const float *res,
                                               int flags, int row0, int col, int M, int N) {
  if (col >= N) return;
  if (bias) {
    const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + col));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      v[i].x += b.x;
      v[i].y += b.y;
      v[i].z += b.z;
      v[i].w += b.w;
    }
  }
  if (flags & SM100_GEMM_GELU) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      v[i].x = gm_gelu(v[i].x);
      v[i].y = gm_gelu(v[i].y);
      v[i].z = gm_gelu(v[i].z);
      v[i].w = gm_gelu(v[i].w);
    }
  }
  if (res) {
    float4 t[8];
#pragma unroll
    for (int i = 0; i < 8; i++)
      t[i] = row0 + 4 * i < M ? *reinterpret_cast<const float4 *>(res + (int64_t)(row0 + 4 * i) * N + col)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      v[i].x += t[i].x;
      v[i].y += t[i].y;
      v[i].z += t[i].z;
      v[i].w += t[i].w;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int row = row0 + 4 * i;
    if (row >= M) continue;
    const int64_t o = (int64_t)row * N + col;
    if (flags & SM100_GEMM_OUT_BF16) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(v[i].x, v[i].y), hi = __floats2bfloat162_rn(v[i].z, v[i].w);
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t *>(&lo);
      w.y = *reinterpret_cast<const uint32_t *>(&hi);
      *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(c) + o) = w;
    } else {
      *reinterpret_cast<float4 *>(reinterpret_cast<float *>(c) + o) = v[i];
    }
  }
}

// kEp = false: the plain product (f32 C, N % 256 == 0, K % 64 == 0);
// kEp = true: any N and K that are multiples of 8 (the tensor maps read zeros
// past them) and the fused epilogue gm_epilogue4x8.
template <bool kEp>
__global__ void __launch_bounds__(kGmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a_half,
                     const __grid_constant__ CUtensorMap map_b, void *c_out, int M, int N, int K, int n_full,
                     const float *bias, const float *res, int flags) {
  float *c = reinterpret_cast<float *>(c_out);
  extern __shared__ unsigned char smem_raw[];
  // the 128-byte swizzle atoms want 1024-byte aligned tiles
  unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kGmStages * kGmStageBytes);   // [stages]
  uint64_t *empty = full + kGmStages;                                                 // [stages]
  uint64_t *acc_full = empty + kGmStages;                                             // [2]
  uint64_t *acc_empty = acc_full + 2;                                                 // [2]
  uint64_t *mma_done = acc_empty + 2;                                                 // all MMAs retired
  uint32_t *tmem_base_s = reinterpret_cast<uint32_t *>(mma_done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (M + kGmTM - 1) / kGmTM, tiles_n = (N + kGmBN - 1) / kGmBN, kb_n = (K + kGmBK - 1) / kGmBK;
  const int n_tiles = n_full + 2 * (tiles_m * tiles_n - n_full);   // work items: whole tiles, then halves
  uint32_t *status = &g_gemm_status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGmStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_empty[0], kGmEpiWarps);
    mbar_init(mma_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {   // TMEM: 512 columns (both accumulators), address into shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base_s)),
                 "r"(kGmTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = *tmem_base_s;

  if (warp == 0) {
    // ---- TMA producer -------------------------------------------------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        const GmItem w = gm_item(tile, tiles_n, n_full);
        if (w.r0 >= M) continue;   // a half wholly past M: no work (every role skips it)
        for (int kb = 0; kb < kb_n; kb++, it++) {
          const int s = it % kGmStages;
          if (it >= kGmStages && !mbar_wait(&empty[s], (uint32_t)(((it / kGmStages) - 1) & 1), status)) {
            ok = false;
            break;
          }
          unsigned char *st = smem + (size_t)s * kGmStageBytes;
          mbar_expect_tx(&full[s], (uint32_t)(w.rows * kGmBK * 2 + kGmBBytes));
          tma_load_2d(st, w.rows == kGmTM ? &map_a : &map_a_half, kb * kGmBK, w.r0, &full[s]);
          tma_load_2d(st + kGmABytes, &map_b, kb * kGmBK, w.tn * kGmBN, &full[s]);
        }
      }
      // the last copies have landed before the CTA may exit
      for (int j = it - kGmStages > 0 ? it - kGmStages : 0; j < it; j++)
        mbar_wait(&full[j % kGmStages], (uint32_t)((j / kGmStages) & 1), status, false);
    }
  } else if (warp == 1) {
    // ---- MMA issuer -----------------------------------------------------------
    if (lane == 0) {
      int it = 0, t_local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        if (gm_item(tile, tiles_n, n_full).r0 >= M) continue;
        // the epilogue has drained TMEM (the previous tile)
        if (t_local >= 1 && !mbar_wait(&acc_empty[0], (uint32_t)((t_local - 1) & 1), status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const bool both = gm_item(tile, tiles_n, n_full).rows == kGmTM;
        for (int kb = 0; kb < kb_n; kb++, it++) {
          const int s = it % kGmStages;
          if (!mbar_wait(&full[s], (uint32_t)((it / kGmStages) & 1), status)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          unsigned char *st = smem + (size_t)s * kGmStageBytes;
          // the second half's rows start 128 rows (16 KB) into the A block
          const uint64_t da0 = smem_desc_sw128(st), da1 = smem_desc_sw128(st + kGmBM * kGmBK * 2),
                         db = smem_desc_sw128(st + kGmABytes);
#pragma unroll
          for (int k = 0; k < kGmBK / 16; k++) {   // K = 16 per MMA: 32 bytes along the swizzled row
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            umma_bf16(tmem_base, da0 + (uint64_t)(2 * k), db + (uint64_t)(2 * k), acc);
            if (both) umma_bf16(tmem_base + (uint32_t)kGmBN, da1 + (uint64_t)(2 * k), db + (uint64_t)(2 * k), acc);
          }
          umma_commit(&empty[s]);   // the stage is free once these MMAs have read it
        }
        umma_commit(&acc_full[0]);  // the accumulators are complete
        t_local++;
      }
      // every MMA issued has retired before TMEM is released (also after a timeout)
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, status, false);
    }
  } else {
    // ---- epilogue: warps 2..9, TMEM lane quarter = warp % 4, column half
    // (warp - 2) / 4 ----------------------------------------------------------
    const int q = warp & 3, c0 = ((warp - 2) >> 2) * (kGmBN / 2);
    float *stg = reinterpret_cast<float *>(smem + kGmStages * kGmStageBytes + 256) + (warp - 2) * kGmStageF;
    int t_local = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
      const GmItem w = gm_item(tile, tiles_n, n_full);
      if (w.r0 >= M) continue;
      if (!mbar_wait(&acc_full[0], (uint32_t)(t_local & 1), status)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
      for (int h = 0; h < w.rows / kGmBM; h++) {
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * kGmBN);
        const int row_w = w.r0 + h * kGmBM + q * 32;   // the warp's first row
#pragma unroll 1
        for (int cc = c0; cc < c0 + kGmBN / 2; cc += 32) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)cc, r);   // every lane of the warp takes part (rows past M included)
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          // through the warp's staging block, so that the global stores are
          // whole 128-byte rows: lane l writes its row l (float4 j at slot
          // j ^ (l & 7): no bank conflicts either way), then lane l takes
          // float4 l & 7 of rows l / 8 + 4 i
          float4 *mine = reinterpret_cast<float4 *>(stg + lane * 32);
#pragma unroll
          for (int j = 0; j < 8; j++)
            mine[j ^ (lane & 7)] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          __syncwarp();
          const int j = lane & 7, col = w.tn * kGmBN + cc + 4 * j;
          float4 v[8];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const int rr = (lane >> 3) + 4 * i;
            v[i] = reinterpret_cast<const float4 *>(stg + rr * 32)[j ^ (rr & 7)];
          }
          __syncwarp();   // the block is read before the next chunk overwrites it
          if constexpr (kEp) {
            gm_epilogue4x8(v, c_out, bias, res, flags, row_w + (lane >> 3), col, M, N);
          } else {
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const int row = row_w + (lane >> 3) + 4 * i;
              if (row < M) *reinterpret_cast<float4 *>(c + (size_t)row * N + col) = v[i];
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[0]);
      t_local++;
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kGmTmemCols) : "memory");
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D map of a row-major bf16 [rows, cols] matrix, box [box_rows, 64 cols], 128-byte swizzle.
static bool make_map(CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGmBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace sm100

using namespace sm100;

// Grid and tile split of one launch (tiles of 256 x 256, whole or halved).
static int gemm_launch(bool ep, const CUtensorMap &ma, const CUtensorMap &mah, const CUtensorMap &mb, void *c,
                       int64_t M, int64_t N, int64_t K, const float *bias, const float *res, int flags,
                       void *stream, const char *name) {
  static int num_sms[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sm100_set_error(SM100_ERR_ARG, "%s: device %d", name, dev);
  if (!num_sms[dev]) cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = ((M + kGmTM - 1) / kGmTM) * ((N + kGmBN - 1) / kGmBN);
  const int grid = (int)(tiles < num_sms[dev] ? tiles : num_sms[dev]);
  // the last round in 128-row halves when its halves fit one round (every
  // tile, when all the halves fit one round of the SMs)
  const int64_t full_rounds = tiles / grid, tail = tiles - full_rounds * grid;
  int n_full = (int)(tail > 0 && 2 * tail <= grid ? full_rounds * grid : tiles);
  if (2 * tiles <= num_sms[dev]) n_full = 0;
  const int grid_items = n_full == 0 ? (int)(2 * tiles) : grid;
  const void *fn = ep ? (const void *)gemm_bf16_kernel<true> : (const void *)gemm_bf16_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kGmSmem);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "%s: smem attribute: %s", name, cudaGetErrorString(e));
  if (ep)
    gemm_bf16_kernel<true><<<grid_items, kGmThreads, kGmSmem, (cudaStream_t)stream>>>(ma, mah, mb, c, (int)M, (int)N, (int)K,
                                                                              n_full, bias, res, flags);
  else
    gemm_bf16_kernel<false><<<grid_items, kGmThreads, kGmSmem, (cudaStream_t)stream>>>(ma, mah, mb, c, (int)M, (int)N,
                                                                               (int)K, n_full, nullptr, nullptr, 0);
  return launch_status(name);
}

extern "C" int sm100_gemm_bf16(const void *a, const void *b, float *c, int64_t M, int64_t N, int64_t K,
                               void *stream) {
  if (!a || !b || !c || M <= 0 || N <= 0 || K <= 0 || M % kGmBM || N % kGmBN || K % kGmBK || M > (1 << 30) ||
      N > (1 << 30) || K > (1 << 30) || ((uintptr_t)a & 15) || ((uintptr_t)b & 15) || ((uintptr_t)c & 15))
    return sm100_set_error(SM100_ERR_ARG,
                           "gemm_bf16: shape %lld x %lld x %lld (M %% 128, N %% 256, K %% 64 must be 0; 16-byte aligned)",
                           (long long)M, (long long)N, (long long)K);
  CUtensorMap ma, mah, mb;
  if (!make_map(&ma, a, M, K, kGmTM) || !make_map(&mah, a, M, K, kGmBM) || !make_map(&mb, b, N, K, kGmBN))
    return sm100_set_error(SM100_ERR_CUDA, "gemm_bf16: tensor map encoding failed");
  return gemm_launch(false, ma, mah, mb, c, M, N, K, nullptr, nullptr, 0, stream, "gemm_bf16");
}

extern "C" int sm100_gemm_bf16_ep(const void *a, const void *b, void *c, int64_t M, int64_t N, int64_t K,
                                  const float *bias, const float *residual, int32_t flags, void *stream) {
  const bool bad_ptr = ((uintptr_t)a & 15) || ((uintptr_t)b & 15) || ((uintptr_t)c & 15) ||
                       ((uintptr_t)bias & 15) || ((uintptr_t)residual & 15);
  if (!a || !b || !c || M <= 0 || N <= 0 || K <= 0 || N % 8 || K % 8 || M > (1 << 30) || N > (1 << 30) ||
      K > (1 << 30) || bad_ptr || (flags & ~(SM100_GEMM_GELU | SM100_GEMM_OUT_BF16)) ||
      (residual && residual == c && (flags & SM100_GEMM_OUT_BF16)))
    return sm100_set_error(SM100_ERR_ARG,
                           "gemm_bf16_ep: shape %lld x %lld x %lld flags %d (N %% 8, K %% 8 must be 0; 16-byte aligned; "
                           "an in-place residual needs f32 output)",
                           (long long)M, (long long)N, (long long)K, (int)flags);
  CUtensorMap ma, mah, mb;
  if (!make_map(&ma, a, M, K, kGmTM) || !make_map(&mah, a, M, K, kGmBM) || !make_map(&mb, b, N, K, kGmBN))
    return sm100_set_error(SM100_ERR_CUDA, "gemm_bf16_ep: tensor map encoding failed");
  return gemm_launch(true, ma, mah, mb, c, M, N, K, bias, residual, flags, stream, "gemm_bf16_ep");
}

// Status of the GEMM launches since the last call (non-zero: a bounded wait
// gave up); reading clears it.  Synchronises the device.
extern "C" uint32_t sm100_gemm_status(void) {
  uint32_t v = 0, z = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v));
  cudaMemcpyToSymbol(g_gemm_status, &z, sizeof(z));
  return v;
}
