// Shared device helpers for the sm_100a kernels of the thvm tensor-track device.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/thvm_sm100.h"

// Host-side hooks implemented in backend.c.
extern "C" int sm100_set_error(int code, const char *fmt, ...);
extern "C" void sm100_note_launch(void);
// Per-device scratch owned by the backend (bytes >= need), or NULL.
extern "C" void *sm100_workspace(uint64_t need);

namespace sm100 {

// Checks the launch that was just issued; records the error text.
static inline int launch_status(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  sm100_note_launch();
  return SM100_OK;
}

// exp2 as the reference's CPU kernels compute it: tinygrad's xexp2
// decomposition (src/codegen/xexp2f.c:12-33): q = x rounded half away from
// zero, s = x - q, a degree-6 polynomial in s, then times 2^q assembled from
// two exponent fields; >= 128 -> inf, < -150 -> 0, NaN -> NaN.  Each step is
// rounded on its own (the _rn intrinsics keep nvcc from fusing a multiply-add),
// so the device result is the same float as the reference CPU path's.
__device__ __forceinline__ float xexp2(float d) {
  const bool finite = (d == d) && (d != INFINITY) && (d != -INFINITY);
  const float x = finite ? d : 0.0f;
  const int q = (int)__fadd_rn(x, x < 0.0f ? -0.5f : 0.5f);
  const float s = __fsub_rn(x, (float)q);
  float u = 0.1535920892e-3f;
  u = __fadd_rn(__fmul_rn(u, s), 0.1339262701e-2f);
  u = __fadd_rn(__fmul_rn(u, s), 0.9618384764e-2f);
  u = __fadd_rn(__fmul_rn(u, s), 0.5550347269e-1f);
  u = __fadd_rn(__fmul_rn(u, s), 0.2402264476e+0f);
  u = __fadd_rn(__fmul_rn(u, s), 0.6931471825e+0f);
  u = __fadd_rn(__fmul_rn(u, s), 1.0f);
  const int h = q >> 1;
  const float p0 = __uint_as_float((uint32_t)(h + 127) << 23);
  const float p1 = __uint_as_float((uint32_t)(q - h + 127) << 23);
  u = __fmul_rn(__fmul_rn(u, p0), p1);
  u = d < 128.0f ? u : INFINITY;
  u = d < -150.0f ? 0.0f : u;
  return (d == d) ? u : __int_as_float(0x7fc00000);
}

// exp(x) = exp2(x * log2(e)) (src/nn/elementwise.c:7-9)
__device__ __forceinline__ float xexp(float x) { return xexp2(__fmul_rn(x, 1.4426950408889634f)); }

// tanh-form GELU in the reference's construction order (src/nn/elementwise.c:13-34):
// half = x*0.5; in = x + (x*x*x)*0.044715; tanh(z) = 2*sigmoid(2z) - 1 with
// sigmoid(v) = recip(exp(-v) + 1); out = half * (tanh + 1).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float half = __fmul_rn(x, 0.5f);
  const float cube = __fmul_rn(__fmul_rn(x, x), x);
  const float in = __fadd_rn(x, __fmul_rn(cube, 0.044715f));
  const float z = __fmul_rn(in, 0.7978845608028654f);
  const float sg = __frcp_rn(__fadd_rn(xexp(-__fmul_rn(z, 2.0f)), 1.0f));
  const float th = __fadd_rn(__fmul_rn(sg, 2.0f), -1.0f);
  return __fmul_rn(half, __fadd_rn(th, 1.0f));
}

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while the previous kernel on its stream is finishing; it runs its
// independent prologue (barriers, TMEM, weight prefetch), then pdl_wait()
// blocks until the previous grid has completed and its memory is visible.
// pdl_trigger() lets the next kernel start launching.  Both are no-ops in a
// kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum / max over blockDim.x threads (a multiple of 32, <= 1024).
// `red` is >= 32 floats of shared memory; every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}

// Streaming 16-byte global load that is read once (weights): no L1 allocation.
__device__ __forceinline__ float4 ld_stream_f4(const void *p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// e4m3 (fn: no infinities, S.1111.111 = NaN) to float: exact, by the bit layout.
__device__ __forceinline__ float fp8e4m3_to_f32(uint32_t b) {
  const uint32_t s = (b & 0x80u) << 24, e = (b >> 3) & 0xfu, m = b & 0x7u;
  if (e == 0xfu && m == 0x7u) return __int_as_float(0x7fc00000 | s);
  if (e == 0) return __uint_as_float(s) + (s ? -1.0f : 1.0f) * (float)m * 0.001953125f; // m * 2^-9
  return __uint_as_float(s | ((e + 120u) << 23) | (m << 20));
}

}  // namespace sm100
