// Row-wise norms and softmax, elementwise GELU / add, and the index kernels
// (embedding gather, argmax, row scatter, KV-cache append, the device
// position counter, strided gather) of the thvm tensor-track device.
//
// Float results follow the reference's construction order op by op (the
// rounding of each elementwise step is the same IEEE operation); reductions
// are tree-ordered, so sums differ from the reference's serial loops by
// reassociation only.  Index results (gather, argmax, scatter) are exact.
#include "common.cuh"

namespace sm100 {

// LayerNorm of one row per CTA (src/nn/layernorm.c:1-7 + py/thvm/nn.py:160-164).
__global__ void __launch_bounds__(256) layernorm_kernel(const float *x, const float *g, const float *b,
                                                        float *y, int64_t D, float eps) {
  __shared__ float red[32];
  const float *xr = x + blockIdx.x * D;
  float *yr = y + blockIdx.x * D;
  const float inv_n = (float)(1.0 / (double)D);
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) s += xr[i];
  const float mean = __fmul_rn(block_sum(s, red), inv_n);
  float v = 0.0f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    const float c = __fsub_rn(xr[i], mean);
    v = fmaf(c, c, v);
  }
  const float var = __fmul_rn(block_sum(v, red), inv_n);
  const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    float o = __fmul_rn(__fsub_rn(xr[i], mean), r);
    if (g) o = __fmul_rn(o, g[i]);
    if (b) o = __fadd_rn(o, b[i]);
    yr[i] = o;
  }
}

// RMSNorm (py/thvm/nn.py RMSNorm._norm): x * rsqrt(mean(x^2) + eps) (* g).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, const float *g, float *y, int64_t D,
                                                      float eps) {
  __shared__ float red[32];
  const float *xr = x + blockIdx.x * D;
  float *yr = y + blockIdx.x * D;
  const float inv_n = (float)(1.0 / (double)D);
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
  const float ms = __fmul_rn(block_sum(s, red), inv_n);
  const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(ms, eps)));
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    const float o = __fmul_rn(xr[i], r);
    yr[i] = g ? __fmul_rn(o, g[i]) : o;
  }
}

// softmax over the last axis (src/nn/softmax.c:1-16).
__global__ void __launch_bounds__(256) softmax_kernel(const float *x, float *y, int64_t N) {
  __shared__ float red[32];
  const float *xr = x + blockIdx.x * N;
  float *yr = y + blockIdx.x * N;
  float mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) mx = fmaxf(mx, xr[i]);
  mx = block_max(mx, red);
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
    const float e = xexp(__fsub_rn(xr[i], mx));
    yr[i] = e;
    s += e;
  }
  const float r = __frcp_rn(block_sum(s, red));
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) yr[i] = __fmul_rn(yr[i], r);
}

__global__ void gelu_kernel(const float *x, float *y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = gelu_tanh(x[i]);
}

__global__ void add_kernel(const float *a, const float *b, float *y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __fadd_rn(a[i], b[i]);
}

// y[i] = table[idx[i]] (zero row outside [0, V)) + pos_table[pos + i]
// (bench/gpt2/thvm_gpt2.py:93-103: tok_emb + pos_emb; py/thvm/tensor.py:1706-1714).
__global__ void embedding_kernel(const float *table, const int32_t *idx, const float *pos_table,
                                 const int32_t *pos, float *y, int64_t V, int64_t D) {
  const int64_t i = blockIdx.x;
  const int64_t id = idx[i];
  const bool ok = id >= 0 && id < V;
  const int64_t prow = pos_table ? (int64_t)(pos ? *pos : 0) + i : 0;
  for (int64_t k = threadIdx.x; k < D; k += blockDim.x) {
    float v = ok ? table[id * D + k] : 0.0f;
    if (pos_table) v = __fadd_rn(v, pos_table[prow * D + k]);
    y[i * D + k] = v;
  }
}

// (value, index) order for argmax: larger value wins, then the lower index
// (py/thvm/tensor.py:998-1011 returns the first index of the max).  NaN
// entries never win.
__device__ __forceinline__ bool am_better(float v1, int i1, float v2, int i2) {
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

constexpr int kArgmaxMaxBlocks = 64;

// Per row: CTAs scan strided slices, one partial each; the last CTA of the
// row (a completion counter, reset after use) folds the partials.
__global__ void __launch_bounds__(256) argmax_kernel(const float *x, int64_t N, int64_t ld, int32_t *out,
                                                     int32_t *bump, float *pv, int32_t *pi,
                                                     uint32_t *counter) {
  __shared__ float sv[256];
  __shared__ int si[256];
  __shared__ bool last;
  const int64_t m = blockIdx.y;
  const float *xr = x + m * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = xr[i];
    if (am_better(v, (int)i, bv, bi)) { bv = v; bi = (int)i; }
  }
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s && am_better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
      sv[threadIdx.x] = sv[threadIdx.x + s];
      si[threadIdx.x] = si[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    pv[m * kArgmaxMaxBlocks + blockIdx.x] = sv[0];
    pi[m * kArgmaxMaxBlocks + blockIdx.x] = si[0];
    __threadfence();
    last = atomicAdd(&counter[m], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    int id = 0x7fffffff;
    for (unsigned b = 0; b < gridDim.x; b++) {
      const float vb = ((volatile float *)pv)[m * kArgmaxMaxBlocks + b];
      const int ib = ((volatile int *)pi)[m * kArgmaxMaxBlocks + b];
      if (am_better(vb, ib, v, id)) { v = vb; id = ib; }
    }
    out[m] = id == 0x7fffffff ? 0 : id;
    counter[m] = 0;
    if (bump && m == 0) atomicAdd(bump, 1);
  }
}

__global__ void scatter_rows_kernel(char *dst, const int32_t *idx, const char *src, int64_t V, int64_t row_bytes) {
  const int64_t i = blockIdx.x;
  const int64_t id = idx[i];
  if (id < 0 || id >= V) return;
  for (int64_t b = threadIdx.x; b < row_bytes; b += blockDim.x) dst[id * row_bytes + b] = src[i * row_bytes + b];
}

// cache[0][pos + t] = k[t], cache[1][pos + t] = v[t] (the in-place row copy a
// KV-cache assign through a view becomes; src/thvm.h:783-795 buf_copy_at).
__global__ void kv_append_kernel(float *cache, const float *k, const float *v, int64_t ld, const int32_t *pos,
                                 int32_t host_pos, int32_t D, int32_t max_ctx) {
  const int64_t t = blockIdx.x;
  const int64_t row = (int64_t)(pos ? *pos : host_pos) + t;
  if (row < 0 || row >= max_ctx) return;
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
    cache[row * D + d] = k[t * ld + d];
    cache[((int64_t)max_ctx + row) * D + d] = v[t * ld + d];
  }
}

__global__ void pos_add_kernel(int32_t *c, int32_t v) { *c += v; }

struct GatherView {
  int32_t ndim, eb;
  int64_t offset, total;
  int64_t dims[8], strides[8];
};

__global__ void gather_strided_kernel(char *dst, const char *src, GatherView v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < v.total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, off = v.offset;
    for (int d = v.ndim - 1; d >= 0; d--) {
      const int64_t c = rem % v.dims[d];
      rem /= v.dims[d];
      off += c * v.strides[d];
    }
    switch (v.eb) {
      case 1: dst[i] = src[off]; break;
      case 2: reinterpret_cast<uint16_t *>(dst)[i] = reinterpret_cast<const uint16_t *>(src)[off]; break;
      case 4: reinterpret_cast<uint32_t *>(dst)[i] = reinterpret_cast<const uint32_t *>(src)[off]; break;
      default: reinterpret_cast<uint64_t *>(dst)[i] = reinterpret_cast<const uint64_t *>(src)[off]; break;
    }
  }
}

static unsigned ew_grid(int64_t n) {
  int64_t g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace sm100

using namespace sm100;

extern "C" int sm100_layernorm(const float *x, const float *g, const float *b, float *y, int64_t M, int64_t D,
                               float eps, void *stream) {
  if (!x || !y || M < 0 || D <= 0 || M > 0x7fffffff) return sm100_set_error(SM100_ERR_ARG, "layernorm: bad arguments");
  if (M == 0) return SM100_OK;
  layernorm_kernel<<<(unsigned)M, 256, 0, (cudaStream_t)stream>>>(x, g, b, y, D, eps);
  return launch_status("layernorm");
}

extern "C" int sm100_rmsnorm(const float *x, const float *g, float *y, int64_t M, int64_t D, float eps,
                             void *stream) {
  if (!x || !y || M < 0 || D <= 0 || M > 0x7fffffff) return sm100_set_error(SM100_ERR_ARG, "rmsnorm: bad arguments");
  if (M == 0) return SM100_OK;
  rmsnorm_kernel<<<(unsigned)M, 256, 0, (cudaStream_t)stream>>>(x, g, y, D, eps);
  return launch_status("rmsnorm");
}

extern "C" int sm100_softmax(const float *x, float *y, int64_t M, int64_t N, void *stream) {
  if (!x || !y || M < 0 || N <= 0 || M > 0x7fffffff) return sm100_set_error(SM100_ERR_ARG, "softmax: bad arguments");
  if (M == 0) return SM100_OK;
  softmax_kernel<<<(unsigned)M, 256, 0, (cudaStream_t)stream>>>(x, y, N);
  return launch_status("softmax");
}

extern "C" int sm100_gelu(const float *x, float *y, int64_t n, void *stream) {
  if (!x || !y || n < 0) return sm100_set_error(SM100_ERR_ARG, "gelu: bad arguments");
  if (n == 0) return SM100_OK;
  gelu_kernel<<<ew_grid(n), 256, 0, (cudaStream_t)stream>>>(x, y, n);
  return launch_status("gelu");
}

extern "C" int sm100_add(const float *a, const float *b, float *y, int64_t n, void *stream) {
  if (!a || !b || !y || n < 0) return sm100_set_error(SM100_ERR_ARG, "add: bad arguments");
  if (n == 0) return SM100_OK;
  add_kernel<<<ew_grid(n), 256, 0, (cudaStream_t)stream>>>(a, b, y, n);
  return launch_status("add");
}

extern "C" int sm100_embedding(const float *table, const int32_t *idx, const float *pos_table, const int32_t *pos,
                               float *y, int64_t n_idx, int64_t V, int64_t D, void *stream) {
  if (!table || !idx || !y || n_idx < 0 || V <= 0 || D <= 0 || n_idx > 0x7fffffff)
    return sm100_set_error(SM100_ERR_ARG, "embedding: bad arguments");
  if (n_idx == 0) return SM100_OK;
  embedding_kernel<<<(unsigned)n_idx, 256, 0, (cudaStream_t)stream>>>(table, idx, pos_table, pos, y, V, D);
  return launch_status("embedding");
}

extern "C" int sm100_argmax(const float *x, int64_t M, int64_t N, int64_t ld, int32_t *out, int32_t *bump,
                            void *stream) {
  if (!x || !out || M < 0 || N <= 0 || N > 0x7ffffffe || M > 65535)
    return sm100_set_error(SM100_ERR_ARG, "argmax: bad arguments");
  if (M == 0) return SM100_OK;
  // Workspace: per-row completion counters at a fixed offset (each reset to
  // 0 by the CTA that consumes it, so they start at 0 for every launch
  // whatever the previous launch's row count), then the per-CTA partials.
  const uint64_t counters = 65536 * 4;
  const uint64_t need = counters + (uint64_t)M * kArgmaxMaxBlocks * 8;
  char *ws = (char *)sm100_workspace(need);
  if (!ws) return sm100_set_error(SM100_ERR_OOM, "argmax: no workspace");
  uint32_t *counter = (uint32_t *)ws;
  float *pv = (float *)(ws + counters);
  int32_t *pi = (int32_t *)(ws + counters + (uint64_t)M * kArgmaxMaxBlocks * 4);
  int64_t nb = (N + 256 * 8 - 1) / (256 * 8);
  if (nb > kArgmaxMaxBlocks) nb = kArgmaxMaxBlocks;
  dim3 grid((unsigned)nb, (unsigned)M);
  argmax_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, N, ld ? ld : N, out, bump, pv, pi, counter);
  return launch_status("argmax");
}

extern "C" int sm100_scatter_rows(void *dst, const int32_t *idx, const void *src, int64_t n_idx, int64_t V,
                                  int64_t D, int32_t elem_bytes, void *stream) {
  if (!dst || !idx || !src || n_idx < 0 || V <= 0 || D <= 0 || elem_bytes <= 0 || n_idx > 0x7fffffff)
    return sm100_set_error(SM100_ERR_ARG, "scatter: bad arguments");
  if (n_idx == 0) return SM100_OK;
  scatter_rows_kernel<<<(unsigned)n_idx, 256, 0, (cudaStream_t)stream>>>((char *)dst, idx, (const char *)src, V,
                                                                         D * elem_bytes);
  return launch_status("scatter_rows");
}

extern "C" int sm100_kv_append(float *cache, const float *k, const float *v, int64_t ld, const int32_t *pos,
                               int32_t host_pos, int32_t T, int32_t D, int32_t max_ctx, void *stream) {
  if (!cache || !k || !v || T < 0 || D <= 0 || max_ctx <= 0) return sm100_set_error(SM100_ERR_ARG, "kv_append: bad arguments");
  if (T == 0) return SM100_OK;
  kv_append_kernel<<<(unsigned)T, 256, 0, (cudaStream_t)stream>>>(cache, k, v, ld ? ld : D, pos, host_pos, D, max_ctx);
  return launch_status("kv_append");
}

extern "C" int sm100_pos_add(int32_t *counter, int32_t value, void *stream) {
  if (!counter) return sm100_set_error(SM100_ERR_ARG, "pos_add: bad arguments");
  pos_add_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(counter, value);
  return launch_status("pos_add");
}

extern "C" int sm100_gather_strided_dev(void *dst, const void *src, const Sm100View *view, void *stream) {
  if (!dst || !src || !view || view->ndim == 0 || view->ndim > 8) return sm100_set_error(SM100_ERR_ARG, "gather_strided: bad view");
  GatherView v;
  v.ndim = (int32_t)view->ndim;
  v.eb = (int32_t)view->elem_bytes;
  if (v.eb != 1 && v.eb != 2 && v.eb != 4 && v.eb != 8) return sm100_set_error(SM100_ERR_ARG, "gather_strided: elem_bytes");
  v.offset = view->offset;
  v.total = 1;
  for (uint32_t d = 0; d < view->ndim; d++) {
    if (view->dims[d] < 0) return sm100_set_error(SM100_ERR_ARG, "gather_strided: dims");
    v.dims[d] = view->dims[d];
    v.strides[d] = view->strides[d];
    v.total *= view->dims[d];
  }
  if (v.total == 0) return SM100_OK;
  gather_strided_kernel<<<ew_grid(v.total), 256, 0, (cudaStream_t)stream>>>((char *)dst, (const char *)src, v);
  return launch_status("gather_strided");
}

// ---- argmax without device allocation ------------------------------------
// For callers that cannot allocate device memory: a plugin whose device
// memory all belongs to a host framework's allocator, a service that fixes
// its memory plan at start-up and allocates nothing after it, or a process
// whose device-memory budget is already spent.  The scratch that argmax needs
// (per-row completion counters and per-CTA partials) lives in this fixed
// array instead, which every GPU that loads this library holds until the
// process exits.
#define ARGMAX_NOALLOC_COUNTER_BYTES 256
#define ARGMAX_NOALLOC_BYTES \
  (ARGMAX_NOALLOC_COUNTER_BYTES + 2 * SM100_ARGMAX_NOALLOC_MAX_ROWS * 64 * 4)

static __device__ __align__(256) unsigned char g_argmax_noalloc_scratch[ARGMAX_NOALLOC_BYTES];

// Device address of the array per device ordinal (host code may not use the
// array's name as an address: that is only a host-side stand-in).
static void *g_argmax_noalloc_dev[64];

extern "C" int sm100_argmax_noalloc(const float *x, int64_t M, int64_t N, int64_t ld, int32_t *out,
                                    int32_t *bump, void *stream) {
  if (!x || !out || M < 0 || N <= 0 || N > 0x7ffffffe)
    return sm100_set_error(SM100_ERR_ARG, "argmax_noalloc: bad arguments");
  if (M > SM100_ARGMAX_NOALLOC_MAX_ROWS)
    return sm100_set_error(SM100_ERR_ARG, "argmax_noalloc: %lld rows exceed the static scratch limit of %d rows",
                           (long long)M, SM100_ARGMAX_NOALLOC_MAX_ROWS);
  if (M == 0) return SM100_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "argmax_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return sm100_set_error(SM100_ERR_UNSUPPORTED, "argmax_noalloc: device %d", dev);
  char *ws = (char *)__atomic_load_n(&g_argmax_noalloc_dev[dev], __ATOMIC_ACQUIRE);
  if (!ws) {
    // once per device, with that device current (two host threads that race
    // here look up the same address; the first store wins)
    void *p = NULL;
    e = cudaGetSymbolAddress(&p, g_argmax_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return sm100_set_error(SM100_ERR_CUDA, "argmax_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    void *expected = NULL;
    __atomic_compare_exchange_n(&g_argmax_noalloc_dev[dev], &expected, p, false, __ATOMIC_ACQ_REL, __ATOMIC_ACQUIRE);
    ws = (char *)__atomic_load_n(&g_argmax_noalloc_dev[dev], __ATOMIC_ACQUIRE);
  }
  uint32_t *counter = (uint32_t *)ws;
  float *pv = (float *)(ws + ARGMAX_NOALLOC_COUNTER_BYTES);
  int32_t *pi = (int32_t *)(ws + ARGMAX_NOALLOC_COUNTER_BYTES + (size_t)M * kArgmaxMaxBlocks * 4);
  // the array keeps the previous call's contents: the counters must start at 0
  e = cudaMemsetAsync(counter, 0, ARGMAX_NOALLOC_COUNTER_BYTES, (cudaStream_t)stream);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "argmax_noalloc: cudaMemsetAsync: %s", cudaGetErrorString(e));
  int64_t nb = (N + 256 * 8 - 1) / (256 * 8);
  if (nb > kArgmaxMaxBlocks) nb = kArgmaxMaxBlocks;
  dim3 grid((unsigned)nb, (unsigned)M);
  argmax_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, N, ld ? ld : N, out, bump, pv, pi, counter);
  return launch_status("argmax_noalloc");
}
