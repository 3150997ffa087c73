// Collectives of the tensor / expert-parallel decode over peer memory: each
// GPU of the box holds one comm buffer, mapped into every other rank's
// process with CUDA IPC, and the kernels below move data with plain stores
// into the peers' buffers over NVLink (no multicast, no library).
//
//   sm100_comm_allreduce_rmsnorm  the all-reduce of the residual stream h
//       [rows, cols] fused with the RMSNorm that consumes it: one CTA per row
//       pushes this rank's partial row into slot [parity][rank][row] of every
//       rank's buffer, raises its flag there, waits for every rank's flag in
//       its own buffer, sums the slots in rank order (so every rank computes
//       the same h, bit for bit, independent of arrival order), stores h and
//       y = bf16(h * rsqrt(mean(h^2) + eps) * g); with zero_rest the ranks
//       other than 0 store zeros into h instead (their next partial sums
//       accumulate from zero, rank 0's from the residual).
//   sm100_comm_allreduce_layernorm  the same exchange fused with a LayerNorm
//       (y = bf16((h - mean) * rsqrt(var + eps) * g + b), two passes).
//   sm100_comm_pick  the vocabulary-split argmax: every rank's (max, index)
//       per row gathered the same way, the largest value with the smallest
//       index wins (the reference's first-index rule).
//
// Flags carry use counts (epochs): use e of a row writes slots of parity
// e & 1 and waits for flag value e.  A rank can only start use e + 2 of a
// row after it saw every rank's flag e + 1, so every rank has finished
// reading the parity-e slots by then (its use e kernel completed before its
// use e + 1 began): two slot sets suffice.  Every wait is bounded (about 2 s
// of clock64 cycles); a timeout sets the status word and the kernel goes on
// with whatever it has, so no rank hangs.
#include <cstring>

#include "common.cuh"

using namespace sm100;

namespace {

constexpr int kMaxRanks = 8, kMaxRows = 32, kMaxCols = 8192;
constexpr uint32_t kCommStall = 1u;
constexpr long long kSpinCycles = 4000000000ll;   // ~2 s at 1.965 GHz

// comm buffer layout (bytes)
constexpr size_t kOffPeers = 0;                                      // void *[kMaxRanks]
constexpr size_t kOffEpochRows = 64;                                 // u32 [kMaxRows]: uses per row
constexpr size_t kOffEpochPick = 192;                                // u32: uses of the pick
constexpr size_t kOffFlagRows = 256;                                 // u32 [kMaxRanks][kMaxRows]
constexpr size_t kOffFlagPick = kOffFlagRows + 4 * kMaxRanks * kMaxRows;   // u32 [kMaxRanks]
constexpr size_t kOffPick = 2048;                                    // {f32, i32} [2][kMaxRanks][kMaxRows]
constexpr size_t kOffSlots = 8192;                                   // f32 [2][kMaxRanks][kMaxRows][cols]

__device__ uint32_t g_comm_status;

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// wait until *flag >= e (wrap-safe), bounded; false on timeout
__device__ bool wait_flag(const uint32_t *flag, uint32_t e) {
  const long long t0 = clock64();
  while ((int32_t)(ld_acquire_sys(flag) - e) < 0) {
    if (clock64() - t0 > kSpinCycles) {
      atomicOr(&g_comm_status, kCommStall);
      return false;
    }
    __nanosleep(20);
  }
  return true;
}

template <bool kLN>
__global__ void __launch_bounds__(256) allreduce_norm_kernel(float *h, const float *g, const float *bt,
                                                             __nv_bfloat16 *y, char *own, int rank, int R, int cols,
                                                             float eps, int zero_rest) {
  __shared__ uint32_t s_e;
  __shared__ float red[8];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, t = threadIdx.x;
  char *const *peers = reinterpret_cast<char *const *>(own + kOffPeers);
  uint32_t *epoch = reinterpret_cast<uint32_t *>(own + kOffEpochRows) + b;
  if (t == 0) s_e = *epoch + 1;
  __syncthreads();
  const uint32_t e = s_e, par = e & 1;
  const size_t slot_stride = (size_t)cols * 4;
  const float4 *src = reinterpret_cast<const float4 *>(h + (int64_t)b * cols);
  const int n4 = cols / 4;
  // 1. push this rank's partial row into slot [par][rank][b] of every rank
  for (int p = 0; p < R; p++) {
    float4 *dst = reinterpret_cast<float4 *>(peers[p] + kOffSlots +
                                             (((size_t)par * kMaxRanks + rank) * kMaxRows + b) * slot_stride);
    for (int i = t; i < n4; i += 256) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  if (t < R) st_release_sys(reinterpret_cast<uint32_t *>(peers[t] + kOffFlagRows) + rank * kMaxRows + b, e);
  // 2. every rank's row has arrived in this buffer
  if (t < R) wait_flag(reinterpret_cast<const uint32_t *>(own + kOffFlagRows) + t * kMaxRows + b, e);
  __syncthreads();
  __threadfence();
  // 3. h = the slots summed in rank order (loads at L2: this SM's L1 may still
  // hold the same slot lines from two uses ago); 4. RMSNorm
  const float *slot0 = reinterpret_cast<const float *>(own + kOffSlots) + ((size_t)par * kMaxRanks * kMaxRows + b) * cols;
  float ss = 0.0f;
  for (int i = t; i < n4; i += 256) {
    float4 a = __ldcg(reinterpret_cast<const float4 *>(slot0) + i);
    for (int p = 1; p < R; p++) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(slot0 + (size_t)p * kMaxRows * cols) + i);
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    reinterpret_cast<float4 *>(h + (int64_t)b * cols)[i] = a;
    ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  __syncthreads();
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; w++) tot += red[w];
  const float inv_n = 1.0f / (float)cols;
  float mean = 0.0f, inv;
  if constexpr (kLN) {
    // LayerNorm: ss above summed squares; the reference's two passes instead:
    // mean = sum * (1/D), then the biased variance of (h - mean)
    // (src/nn/layernorm.c:1-7), over the row this thread just wrote
    float sum = 0.0f;
    for (int i = t; i < n4; i += 256) {
      const float4 a = reinterpret_cast<const float4 *>(h + (int64_t)b * cols)[i];
      sum += (a.x + a.y) + (a.z + a.w);
    }
    sum = warp_sum(sum);
    __syncthreads();
    if ((t & 31) == 0) red[t >> 5] = sum;
    __syncthreads();
    float st = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) st += red[w];
    mean = st * inv_n;
    float v = 0.0f;
    for (int i = t; i < n4; i += 256) {
      const float4 a = reinterpret_cast<const float4 *>(h + (int64_t)b * cols)[i];
      const float c0 = a.x - mean, c1 = a.y - mean, c2 = a.z - mean, c3 = a.w - mean;
      v += (c0 * c0 + c1 * c1) + (c2 * c2 + c3 * c3);
    }
    v = warp_sum(v);
    __syncthreads();
    if ((t & 31) == 0) red[t >> 5] = v;
    __syncthreads();
    float vt = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) vt += red[w];
    inv = 1.0f / sqrtf(vt * inv_n + eps);
  } else {
    inv = 1.0f / sqrtf(tot * inv_n + eps);
  }
  const bool zero = zero_rest && rank != 0;
  for (int i = t; i < n4; i += 256) {
    float4 *hp = reinterpret_cast<float4 *>(h + (int64_t)b * cols) + i;
    const float4 a = *hp;
    const float4 gg = reinterpret_cast<const float4 *>(g)[i];
    __nv_bfloat162 *yo = reinterpret_cast<__nv_bfloat162 *>(y + (int64_t)b * cols + 4 * i);
    if constexpr (kLN) {
      const float4 bb = reinterpret_cast<const float4 *>(bt)[i];
      yo[0] = __floats2bfloat162_rn((a.x - mean) * inv * gg.x + bb.x, (a.y - mean) * inv * gg.y + bb.y);
      yo[1] = __floats2bfloat162_rn((a.z - mean) * inv * gg.z + bb.z, (a.w - mean) * inv * gg.w + bb.w);
    } else {
      yo[0] = __floats2bfloat162_rn((a.x * inv) * gg.x, (a.y * inv) * gg.y);
      yo[1] = __floats2bfloat162_rn((a.z * inv) * gg.z, (a.w * inv) * gg.w);
    }
    if (zero) *hp = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (t == 0) *epoch = e;
}

__global__ void pick_kernel(const float *val, const int32_t *idx, char *own, int rank, int R, int rows, int32_t *tok) {
  __shared__ uint32_t s_e;
  pdl_trigger();
  pdl_wait();
  const int t = threadIdx.x;
  char *const *peers = reinterpret_cast<char *const *>(own + kOffPeers);
  uint32_t *epoch = reinterpret_cast<uint32_t *>(own + kOffEpochPick);
  if (t == 0) s_e = *epoch + 1;
  __syncthreads();
  const uint32_t e = s_e, par = e & 1;
  if (t < rows) {
    const float v = val[t];
    const int32_t i = idx[t];
    for (int p = 0; p < R; p++) {
      float2 *dst = reinterpret_cast<float2 *>(peers[p] + kOffPick) + ((size_t)par * kMaxRanks + rank) * kMaxRows + t;
      *dst = make_float2(v, __int_as_float(i));
    }
  }
  __threadfence_system();
  __syncthreads();
  if (t < R) st_release_sys(reinterpret_cast<uint32_t *>(peers[t] + kOffFlagPick) + rank, e);
  if (t < R) wait_flag(reinterpret_cast<const uint32_t *>(own + kOffFlagPick) + t, e);
  __syncthreads();
  __threadfence();
  if (t < rows) {
    const float2 *s = reinterpret_cast<const float2 *>(own + kOffPick) + (size_t)par * kMaxRanks * kMaxRows + t;
    const float2 s0 = __ldcg(s);
    float bv = s0.x;
    int32_t bi = __float_as_int(s0.y);
    for (int p = 1; p < R; p++) {
      const float2 sp = __ldcg(s + (size_t)p * kMaxRows);
      const float v = sp.x;
      const int32_t i = __float_as_int(sp.y);
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
    tok[t] = bi;
  }
  if (t == 0) *epoch = e;
}

}  // namespace

extern "C" uint64_t sm100_comm_bytes(int32_t cols) {
  if (cols < 4 || cols > kMaxCols || cols % 4) return 0;
  return kOffSlots + (uint64_t)2 * kMaxRanks * kMaxRows * cols * 4;
}

extern "C" int sm100_peer_alloc(uint64_t nbytes, void **dptr, void *handle_out) {
  if (!dptr || !handle_out || nbytes == 0) return sm100_set_error(SM100_ERR_ARG, "peer_alloc: bad arguments");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, nbytes);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_OOM, "peer_alloc(%llu): %s", (unsigned long long)nbytes,
                                               cudaGetErrorString(e));
  e = cudaMemset(p, 0, nbytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(handle_out), p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return sm100_set_error(SM100_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  }
  *dptr = p;
  return SM100_OK;
}

extern "C" int sm100_peer_open(const void *handle, void **peer_dptr) {
  if (!handle || !peer_dptr) return sm100_set_error(SM100_ERR_ARG, "peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(peer_dptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "peer_open: %s", cudaGetErrorString(e));
  return SM100_OK;
}

extern "C" int sm100_peer_close(void *peer_dptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_dptr);
  return e == cudaSuccess ? SM100_OK : sm100_set_error(SM100_ERR_CUDA, "peer_close: %s", cudaGetErrorString(e));
}

extern "C" int sm100_peer_free(void *dptr) {
  const cudaError_t e = cudaFree(dptr);
  return e == cudaSuccess ? SM100_OK : sm100_set_error(SM100_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
}

extern "C" int sm100_comm_set_peers(void *own, void *const *peer_ptrs, int32_t world) {
  if (!own || !peer_ptrs || world < 1 || world > kMaxRanks)
    return sm100_set_error(SM100_ERR_ARG, "comm_set_peers: world %d (1..%d)", world, kMaxRanks);
  void *table[kMaxRanks] = {};
  for (int i = 0; i < world; i++) table[i] = peer_ptrs[i];
  const cudaError_t e = cudaMemcpy(static_cast<char *>(own) + kOffPeers, table, sizeof table, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? SM100_OK : sm100_set_error(SM100_ERR_CUDA, "comm_set_peers: %s", cudaGetErrorString(e));
}

extern "C" int sm100_comm_allreduce_rmsnorm(float *h, const float *g, void *y, void *own, int32_t rank, int32_t world,
                                            int32_t rows, int32_t cols, float eps, int32_t zero_rest, void *stream) {
  if (!h || !g || !y || !own || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || rows < 1 ||
      rows > kMaxRows || cols < 4 || cols > kMaxCols || cols % 4 || ((uintptr_t)h | (uintptr_t)g | (uintptr_t)y) % 16)
    return sm100_set_error(SM100_ERR_ARG, "comm_allreduce_rmsnorm: rank %d of %d, %d x %d (rows <= %d, cols %% 4, "
                                          "16-byte aligned)", rank, world, rows, cols, kMaxRows);
  const cudaError_t e = launch_pdl(allreduce_norm_kernel<false>, dim3(rows), dim3(256), 0, (cudaStream_t)stream, h, g,
                                   (const float *)nullptr, (__nv_bfloat16 *)y, (char *)own, rank, world, cols, eps,
                                   zero_rest);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "comm_allreduce_rmsnorm: %s", cudaGetErrorString(e));
  return launch_status("comm_allreduce_rmsnorm");
}

extern "C" int sm100_comm_allreduce_layernorm(float *h, const float *g, const float *b, void *y, void *own,
                                              int32_t rank, int32_t world, int32_t rows, int32_t cols, float eps,
                                              void *stream) {
  if (!h || !g || !b || !y || !own || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || rows < 1 ||
      rows > kMaxRows || cols < 4 || cols > kMaxCols || cols % 4 ||
      ((uintptr_t)h | (uintptr_t)g | (uintptr_t)b | (uintptr_t)y) % 16)
    return sm100_set_error(SM100_ERR_ARG, "comm_allreduce_layernorm: rank %d of %d, %d x %d (rows <= %d, cols %% 4, "
                                          "16-byte aligned)", rank, world, rows, cols, kMaxRows);
  const cudaError_t e = launch_pdl(allreduce_norm_kernel<true>, dim3(rows), dim3(256), 0, (cudaStream_t)stream, h, g,
                                   b, (__nv_bfloat16 *)y, (char *)own, rank, world, cols, eps, 0);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "comm_allreduce_layernorm: %s", cudaGetErrorString(e));
  return launch_status("comm_allreduce_layernorm");
}

extern "C" int sm100_comm_pick(const float *val, const int32_t *idx, void *own, int32_t rank, int32_t world,
                               int32_t rows, int32_t *tok, void *stream) {
  if (!val || !idx || !own || !tok || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || rows < 1 ||
      rows > kMaxRows)
    return sm100_set_error(SM100_ERR_ARG, "comm_pick: rank %d of %d, %d rows", rank, world, rows);
  const cudaError_t e = launch_pdl(pick_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, val, idx, (char *)own,
                                   rank, world, rows, tok);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "comm_pick: %s", cudaGetErrorString(e));
  return launch_status("comm_pick");
}

extern "C" uint32_t sm100_comm_status(void) {
  uint32_t v = 0, z = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_comm_status, sizeof(v));
  cudaMemcpyToSymbol(g_comm_status, &z, sizeof(z));
  return v;
}
