/* backend.c - the host side of the sm_100a device: the Backend vtable
 * (src/thvm.h:751-829) over the CUDA runtime, the dispatch_kernel router from
 * Sm100Kernel descriptors to the kernel launchers, and TinyJit replay as CUDA
 * graphs.  Plain C11; one host thread drives it (src/thvm.h Backend contract:
 * no locking in backend tables, as the reference's CUDA backend has none).
 *
 * Buffer semantics follow src/backend/cuda/buf_*.c: ids index a 65536-slot
 * table, slot 0 is "none", a fresh allocation is zero-filled, the freelist is
 * best-fit and a recycled block is handed to a FRESH slot id while the donor
 * slot goes dead (buf_freelist.c:42-110), arena views borrow their parent's
 * storage and are never recycled, jit-pinned buffers survive decref.
 * Device memory comes from the stream-ordered pool (cudaMallocAsync), so
 * frees are ordered after the launches that read them (buf_free.c:5-55).
 */
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "../../include/thvm_sm100.h"

#define BUFS_CAP 65536u
#define FREELIST_CAP 65536u
#define GRAPH_SLOTS 64u
#define WORKSPACE_BYTES (8u << 20)

typedef struct {
  char *ptr;          /* device (or host-mode) address; NULL = dead */
  uint64_t nbytes;    /* capacity of the storage block */
  uint64_t req;       /* requested bytes (buf_nbytes) */
  uint32_t refcount;
  uint32_t parent;    /* arena parent (views), 0 for owners */
  uint8_t owns;       /* 1: owns ptr; 0: a view */
  uint8_t jit_pinned;
  uint8_t parked;     /* on the freelist */
} Buf;

static Buf BUFS[BUFS_CAP];
static uint32_t BUFS_NEXT = 1;
static uint32_t FREELIST[FREELIST_CAP];
static uint32_t FREELIST_LEN = 0;
static uint64_t MEM_LIVE = 0, MEM_PEAK = 0;

static int READY = 0;
static int HOST_MODE = 0;
static int DEVICE = 0;
static cudaStream_t STREAM = NULL;
static int OWN_STREAM = 0;
static void *WORKSPACE = NULL;
static uint64_t WORKSPACE_SIZE = 0;
static uint64_t LAUNCHES = 0;

typedef struct {
  cudaGraph_t graph;
  cudaGraphExec_t exec;
  uint64_t kernels;
} GraphSlot;
static GraphSlot GRAPHS[GRAPH_SLOTS];
static int CAPTURING = 0;
static uint32_t CAPTURE_SLOT = 0;

static char LAST_ERROR[512] = "";

int sm100_set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(LAST_ERROR, sizeof LAST_ERROR, fmt, ap);
  va_end(ap);
  if (getenv("THVM_SM100_VERBOSE")) fprintf(stderr, "[sm100] %s\n", LAST_ERROR);
  return code;
}

const char *sm100_last_error(void) { return LAST_ERROR; }
void sm100_note_launch(void) { LAUNCHES++; }
uint64_t sm100_launch_count(void) { return LAUNCHES; }
int sm100_ready(void) { return READY; }

static int cuda_fail(const char *what, cudaError_t e) {
  return sm100_set_error(SM100_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void sm100_debug_host_memory(int on) {
  if (!READY) HOST_MODE = on ? 1 : 0;
}

void *sm100_workspace(uint64_t need) {
  if (!READY || HOST_MODE || need > WORKSPACE_SIZE) return NULL;
  return WORKSPACE;
}

/* ---- init / shutdown (src/backend/cuda/init.c:110-143) ------------------ */

int sm100_init(void) {
  if (READY) return SM100_OK;
  memset(BUFS, 0, sizeof BUFS);
  BUFS_NEXT = 1;
  FREELIST_LEN = 0;
  MEM_LIVE = MEM_PEAK = 0;
  if (HOST_MODE) {
    READY = 1;
    return SM100_OK;
  }
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    return sm100_set_error(SM100_ERR_STATE, "no CUDA device (%s)", cudaGetErrorString(e));
  }
  const char *dev = getenv("THVM_SM100_DEVICE");
  if (dev && dev[0]) {
    DEVICE = atoi(dev);
    if ((e = cudaSetDevice(DEVICE)) != cudaSuccess) return cuda_fail("cudaSetDevice", e);
  } else if ((e = cudaGetDevice(&DEVICE)) != cudaSuccess) {
    return cuda_fail("cudaGetDevice", e);
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, DEVICE);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, DEVICE);
  if (major != 10 || minor != 0)
    return sm100_set_error(SM100_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build is sm_100a only", DEVICE,
                           major, minor);
  if ((e = cudaStreamCreateWithFlags(&STREAM, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail("cudaStreamCreate", e);
  OWN_STREAM = 1;
  if ((e = cudaMalloc(&WORKSPACE, WORKSPACE_BYTES)) != cudaSuccess) return cuda_fail("cudaMalloc(workspace)", e);
  if ((e = cudaMemset(WORKSPACE, 0, WORKSPACE_BYTES)) != cudaSuccess) return cuda_fail("cudaMemset(workspace)", e);
  WORKSPACE_SIZE = WORKSPACE_BYTES;
  /* keep freed pool memory for reuse instead of returning it at each sync */
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, DEVICE) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  READY = 1;
  return SM100_OK;
}

void sm100_shutdown(void) {
  if (!READY) return;
  for (uint32_t s = 0; s < GRAPH_SLOTS; s++) sm100_graph_drop(s);
  for (uint32_t i = 1; i < BUFS_NEXT; i++) {
    if (BUFS[i].ptr && BUFS[i].owns) {
      if (HOST_MODE) free(BUFS[i].ptr);
      else cudaFreeAsync(BUFS[i].ptr, STREAM);
    }
  }
  memset(BUFS, 0, sizeof BUFS);
  BUFS_NEXT = 1;
  FREELIST_LEN = 0;
  MEM_LIVE = 0;
  if (!HOST_MODE) {
    cudaStreamSynchronize(STREAM);
    if (WORKSPACE) cudaFree(WORKSPACE);
    WORKSPACE = NULL;
    WORKSPACE_SIZE = 0;
    if (OWN_STREAM) cudaStreamDestroy(STREAM);
    STREAM = NULL;
    OWN_STREAM = 0;
  }
  READY = 0;
}

void *sm100_stream(void) { return (void *)STREAM; }

int sm100_set_stream(void *stream) {
  if (!READY) return sm100_set_error(SM100_ERR_STATE, "set_stream: not initialised");
  if (CAPTURING) return sm100_set_error(SM100_ERR_STATE, "set_stream: capture open");
  STREAM = (cudaStream_t)stream;
  return SM100_OK;
}

/* ---- buffers ------------------------------------------------------------ */

static int live_id(uint32_t id) { return READY && id != 0 && id < BUFS_NEXT && BUFS[id].ptr != NULL; }

static uint64_t byte_ceiling(void) {
  const char *e = getenv("THVM_MAX_BUF_BYTES");
  return (e && e[0]) ? strtoull(e, NULL, 10) : 0;
}

static int dev_zero(void *p, uint64_t n) {
  if (HOST_MODE) {
    memset(p, 0, (size_t)n);
    return SM100_OK;
  }
  cudaError_t e = cudaMemsetAsync(p, 0, (size_t)n, STREAM);
  return e == cudaSuccess ? SM100_OK : cuda_fail("cudaMemsetAsync", e);
}

/* best-fit pop onto a fresh slot id (src/backend/cuda/buf_freelist.c:42-103) */
static uint32_t freelist_try_pop(uint64_t nbytes) {
  if (BUFS_NEXT >= BUFS_CAP) return 0;
  uint32_t best_i = 0;
  uint64_t best_nb = UINT64_MAX;
  for (uint32_t i = 0; i < FREELIST_LEN; i++) {
    const Buf *b = &BUFS[FREELIST[i]];
    if (!b->ptr || !b->owns || b->nbytes < nbytes) continue;
    if (b->nbytes < best_nb) {
      best_nb = b->nbytes;
      best_i = i;
    }
  }
  if (best_nb == UINT64_MAX) return 0;
  const uint32_t donor = FREELIST[best_i];
  FREELIST[best_i] = FREELIST[--FREELIST_LEN];
  Buf *d = &BUFS[donor];
  const uint32_t id = BUFS_NEXT++;
  Buf *nb = &BUFS[id];
  memset(nb, 0, sizeof *nb);
  nb->ptr = d->ptr;
  nb->nbytes = d->nbytes;
  nb->req = nbytes;
  nb->refcount = 1;
  nb->owns = 1;
  memset(d, 0, sizeof *d); /* the donor id is dead from now on */
  dev_zero(nb->ptr, nbytes);
  return id;
}

uint32_t sm100_buf_alloc(uint64_t nbytes) {
  if (!READY) {
    sm100_set_error(SM100_ERR_STATE, "buf_alloc: not initialised");
    return 0;
  }
  const uint64_t ceil = byte_ceiling();
  if (ceil && nbytes > ceil) {
    sm100_set_error(SM100_ERR_ARG, "buf_alloc: %llu bytes above THVM_MAX_BUF_BYTES %llu",
                    (unsigned long long)nbytes, (unsigned long long)ceil);
    return 0;
  }
  if (nbytes == 0) nbytes = 1;
  const uint32_t rec = freelist_try_pop(nbytes);
  if (rec) return rec;
  if (BUFS_NEXT >= BUFS_CAP) {
    sm100_set_error(SM100_ERR_OOM, "buf_alloc: out of slots (cap=%u)", BUFS_CAP);
    return 0;
  }
  /* round the block to 256 bytes so vector / TMA loads stay in bounds */
  const uint64_t cap = (nbytes + 255u) & ~(uint64_t)255u;
  void *p = NULL;
  if (HOST_MODE) {
    p = aligned_alloc(256, (size_t)cap);
    if (!p) {
      sm100_set_error(SM100_ERR_OOM, "buf_alloc: host allocation of %llu bytes failed", (unsigned long long)cap);
      return 0;
    }
  } else {
    cudaError_t e = cudaMallocAsync(&p, (size_t)cap, STREAM);
    if (e != cudaSuccess) {
      cudaGetLastError();
      sm100_set_error(SM100_ERR_OOM, "buf_alloc: cudaMallocAsync(%llu): %s", (unsigned long long)cap,
                      cudaGetErrorString(e));
      return 0;
    }
  }
  if (dev_zero(p, cap) != SM100_OK) {
    if (HOST_MODE) free(p);
    else cudaFreeAsync(p, STREAM);
    return 0;
  }
  const uint32_t id = BUFS_NEXT++;
  Buf *b = &BUFS[id];
  memset(b, 0, sizeof *b);
  b->ptr = (char *)p;
  b->nbytes = cap;
  b->req = nbytes;
  b->refcount = 1;
  b->owns = 1;
  MEM_LIVE += cap;
  if (MEM_LIVE > MEM_PEAK) MEM_PEAK = MEM_LIVE;
  return id;
}

static void freelist_drop(uint32_t id) {
  for (uint32_t i = 0; i < FREELIST_LEN; i++) {
    if (FREELIST[i] == id) {
      FREELIST[i] = FREELIST[--FREELIST_LEN];
      return;
    }
  }
}

void sm100_buf_free(uint32_t id) {
  if (!live_id(id)) return;
  Buf *b = &BUFS[id];
  if (b->parked) freelist_drop(id);
  if (b->owns) {
    if (HOST_MODE) free(b->ptr);
    else cudaFreeAsync(b->ptr, STREAM);
    MEM_LIVE -= b->nbytes;
  }
  memset(b, 0, sizeof *b);
}

void sm100_buf_incref(uint32_t id) {
  if (live_id(id)) BUFS[id].refcount++;
}

void sm100_buf_decref(uint32_t id) {
  if (!live_id(id)) return;
  Buf *b = &BUFS[id];
  if (b->refcount > 0) b->refcount--;
  if (b->refcount == 0 && !b->jit_pinned && !b->parked) sm100_buf_free(id);
}

void sm100_buf_jit_pin(uint32_t id) {
  if (live_id(id)) BUFS[id].jit_pinned = 1;
}

void sm100_buf_jit_unpin(uint32_t id) {
  if (live_id(id)) BUFS[id].jit_pinned = 0;
}

uint32_t sm100_buf_refcount(uint32_t id) { return live_id(id) ? BUFS[id].refcount : 0; }

uint64_t sm100_buf_nbytes(uint32_t id) { return live_id(id) ? BUFS[id].req : 0; }

void *sm100_buf_dptr(uint32_t id) { return live_id(id) ? BUFS[id].ptr : NULL; }

uint64_t sm100_mem_live_bytes(void) { return MEM_LIVE; }
uint64_t sm100_mem_peak_bytes(void) { return MEM_PEAK; }

uint32_t sm100_buf_live_count(void) {
  uint32_t n = 0;
  for (uint32_t i = 1; i < BUFS_NEXT; i++) n += BUFS[i].ptr != NULL;
  return n;
}

uint32_t sm100_buf_storage_root(uint32_t id) {
  uint32_t guard = 0;
  while (live_id(id) && BUFS[id].parent && guard++ < BUFS_CAP) id = BUFS[id].parent;
  return id;
}

/* (src/backend/cuda/buf_freelist.c:10-41): pinned, views and dead ids are
 * never parked; a parked buffer has refcount 0 */
void sm100_buf_freelist_push(uint32_t id) {
  if (!live_id(id)) return;
  Buf *b = &BUFS[id];
  if (b->jit_pinned || !b->owns || b->parked || FREELIST_LEN >= FREELIST_CAP) return;
  FREELIST[FREELIST_LEN++] = id;
  b->parked = 1;
  b->refcount = 0;
}

void sm100_buf_freelist_remove(uint32_t id) {
  if (!live_id(id) || !BUFS[id].parked) return;
  freelist_drop(id);
  BUFS[id].parked = 0;
  BUFS[id].refcount = 1;
}

uint32_t sm100_buf_view(uint32_t parent, uint64_t off, uint64_t nbytes) {
  if (!live_id(parent)) {
    sm100_set_error(SM100_ERR_ARG, "buf_view: dead parent %u", parent);
    return 0;
  }
  if (off > BUFS[parent].req || nbytes > BUFS[parent].req - off) {
    sm100_set_error(SM100_ERR_ARG, "buf_view: [%llu, +%llu) outside %llu bytes", (unsigned long long)off,
                    (unsigned long long)nbytes, (unsigned long long)BUFS[parent].req);
    return 0;
  }
  if (BUFS_NEXT >= BUFS_CAP) {
    sm100_set_error(SM100_ERR_OOM, "buf_view: out of slots");
    return 0;
  }
  const uint32_t id = BUFS_NEXT++;
  Buf *b = &BUFS[id];
  memset(b, 0, sizeof *b);
  b->ptr = BUFS[parent].ptr + off;
  b->nbytes = b->req = nbytes;
  b->refcount = 1;
  b->parent = parent;
  b->owns = 0;
  return id;
}

static int copy_bytes(void *dst, const void *src, uint64_t n, enum cudaMemcpyKind kind) {
  if (n == 0) return SM100_OK;
  if (HOST_MODE) {
    memmove(dst, src, (size_t)n);
    return SM100_OK;
  }
  cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)n, kind, STREAM);
  if (e != cudaSuccess) return cuda_fail("cudaMemcpyAsync", e);
  if (kind == cudaMemcpyDeviceToHost || kind == cudaMemcpyHostToDevice) {
    /* host memory is the caller's: finish before returning */
    e = cudaStreamSynchronize(STREAM);
    if (e != cudaSuccess) return cuda_fail("cudaStreamSynchronize", e);
  }
  return SM100_OK;
}

int sm100_buf_read(uint32_t id, void *dst, uint64_t nbytes) {
  if (!live_id(id) || (!dst && nbytes)) return sm100_set_error(SM100_ERR_ARG, "buf_read: bad buffer %u", id);
  if (nbytes > BUFS[id].req) return sm100_set_error(SM100_ERR_ARG, "buf_read: %llu bytes > %llu",
                                                      (unsigned long long)nbytes, (unsigned long long)BUFS[id].req);
  if (CAPTURING) return sm100_set_error(SM100_ERR_STATE, "buf_read: capture open");
  return copy_bytes(dst, BUFS[id].ptr, nbytes, cudaMemcpyDeviceToHost);
}

int sm100_buf_write(uint32_t id, const void *src, uint64_t nbytes) { return sm100_buf_write_at(id, 0, src, nbytes); }

int sm100_buf_write_at(uint32_t id, uint64_t off, const void *src, uint64_t nbytes) {
  if (!live_id(id) || (!src && nbytes)) return sm100_set_error(SM100_ERR_ARG, "buf_write: bad buffer %u", id);
  if (off > BUFS[id].req || nbytes > BUFS[id].req - off)
    return sm100_set_error(SM100_ERR_ARG, "buf_write_at: [%llu, +%llu) outside %llu bytes", (unsigned long long)off,
                           (unsigned long long)nbytes, (unsigned long long)BUFS[id].req);
  if (CAPTURING) return sm100_set_error(SM100_ERR_STATE, "buf_write: capture open");
  return copy_bytes(BUFS[id].ptr + off, src, nbytes, cudaMemcpyHostToDevice);
}

int sm100_buf_copy(uint32_t dst, uint32_t src, uint64_t nbytes) { return sm100_buf_copy_at(dst, 0, src, nbytes); }

int sm100_buf_copy_at(uint32_t dst, uint64_t off, uint32_t src, uint64_t nbytes) {
  if (!live_id(dst) || !live_id(src)) return sm100_set_error(SM100_ERR_ARG, "buf_copy: bad buffer");
  if (nbytes > BUFS[src].req || off > BUFS[dst].req || nbytes > BUFS[dst].req - off)
    return sm100_set_error(SM100_ERR_ARG, "buf_copy_at: out of bounds");
  return copy_bytes(BUFS[dst].ptr + off, BUFS[src].ptr, nbytes, cudaMemcpyDeviceToDevice);
}

void sm100_buf_zero(uint32_t id) {
  if (live_id(id)) dev_zero(BUFS[id].ptr, BUFS[id].req);
}

/* ---- realize boundary (src/backend/cuda/_.c:23-27) ---------------------- */

void sm100_dispatch_begin(void) {}
void sm100_dispatch_flush(void) {}

void sm100_dispatch_end(void) {
  if (!READY || HOST_MODE || CAPTURING) return;
  cudaError_t e = cudaStreamSynchronize(STREAM);
  if (e != cudaSuccess) cuda_fail("dispatch_end", e);
}

/* ---- dispatch_kernel ---------------------------------------------------- */

int sm100_gather_strided_dev(void *dst, const void *src, const Sm100View *view, void *stream);

/* device pointer of slot s of the descriptor, NULL when absent */
static char *slot_ptr(const Sm100Kernel *k, const uint32_t *ids, uint32_t n_in, int s, int *bad) {
  if (s < 0 || s >= 10) return NULL;
  const int32_t i = k->in[s];
  if (i < 0) return NULL;
  if ((uint32_t)i >= n_in || !live_id(ids[i])) {
    *bad = 1;
    return NULL;
  }
  return BUFS[ids[i]].ptr;
}

int sm100_dispatch_kernel(const Sm100Kernel *k, const uint32_t *ids, uint32_t n_in, uint32_t out_id) {
  if (!READY) return sm100_set_error(SM100_ERR_STATE, "dispatch_kernel: not initialised");
  if (!k) return sm100_set_error(SM100_ERR_ARG, "dispatch_kernel: no descriptor");
  if (HOST_MODE) return sm100_set_error(SM100_ERR_UNSUPPORTED, "dispatch_kernel: host-memory mode runs no kernels");
  int bad = 0;
  char *p[10];
  for (int s = 0; s < 10; s++) p[s] = slot_ptr(k, ids, n_in, s, &bad);
  char *out = live_id(out_id) ? BUFS[out_id].ptr : NULL;
  if (bad) return sm100_set_error(SM100_ERR_ARG, "dispatch_kernel: dead or out-of-range input slot");
  if (!out && k->kind != SM100_K_POS_ADD)
    return sm100_set_error(SM100_ERR_ARG, "dispatch_kernel: dead output buffer %u", out_id);
  void *st = (void *)STREAM;
  switch (k->kind) {
    case SM100_K_LINEAR: {
      Sm100LinearArgs a;
      memset(&a, 0, sizeof a);
      a.x = (const float *)p[0] + k->row_off * (k->ld_in ? k->ld_in : k->k);
      a.w = p[1];
      a.bias = (const float *)p[2];
      a.ln_g = (const float *)p[3];
      a.ln_b = (const float *)p[4];
      a.residual = (const float *)p[5];
      a.w_scale = (const float *)p[6];
      a.pos = (const int32_t *)p[7];
      a.kv_cache = (float *)p[8];
      a.y = (float *)out;
      a.M = k->m;
      a.N = k->n;
      a.K = k->k;
      a.ldx = k->ld_in;
      a.ldy = k->ld_out;
      a.wdtype = (int32_t)k->dtype;
      a.flags = (int32_t)k->flags;
      a.max_ctx = k->max_ctx;
      a.host_pos = k->pos;
      a.eps = k->eps;
      return sm100_linear(&a, st);
    }
    case SM100_K_LAYERNORM:
      return sm100_layernorm((const float *)p[0], (const float *)p[1], (const float *)p[2], (float *)out, k->m, k->k,
                             k->eps, st);
    case SM100_K_RMSNORM:
      return sm100_rmsnorm((const float *)p[0], (const float *)p[1], (float *)out, k->m, k->k, k->eps, st);
    case SM100_K_SOFTMAX:
      return sm100_softmax((const float *)p[0], (float *)out, k->m, k->k, st);
    case SM100_K_GELU:
      return sm100_gelu((const float *)p[0], (float *)out, k->m * k->k, st);
    case SM100_K_ADD:
      return sm100_add((const float *)p[0], (const float *)p[1], (float *)out, k->m * k->k, st);
    case SM100_K_ATTENTION: {
      Sm100AttnArgs a;
      memset(&a, 0, sizeof a);
      const int64_t d = (int64_t)k->heads * k->head_dim;
      a.q = (const float *)p[0];
      a.k_cache = (const float *)p[1];
      a.v_cache = (const float *)p[1] + (int64_t)k->max_ctx * d;
      a.out = (float *)out;
      a.pos = (const int32_t *)p[7];
      a.ldq = k->ld_in;
      a.T = (int32_t)k->m;
      a.H = k->heads;
      a.hd = k->head_dim;
      a.max_ctx = k->max_ctx;
      a.host_pos = k->pos;
      a.scale = k->scale;
      if (!a.q || !p[1]) return sm100_set_error(SM100_ERR_ARG, "attention: missing q or cache");
      return sm100_attention(&a, st);
    }
    case SM100_K_EMBEDDING:
      if (k->dtype != SM100_DT_F32) return sm100_set_error(SM100_ERR_UNSUPPORTED, "embedding: f32 tables only");
      return sm100_embedding((const float *)p[0], (const int32_t *)p[1], (const float *)p[2], (const int32_t *)p[7],
                             (float *)out, k->m, k->n, k->k, st);
    case SM100_K_ARGMAX:
      return sm100_argmax((const float *)p[0] + k->row_off * (k->ld_in ? k->ld_in : k->n), k->m, k->n, k->ld_in,
                          (int32_t *)out, (int32_t *)p[7], st);
    case SM100_K_SCATTER:
      return sm100_scatter_rows(out, (const int32_t *)p[1], p[0], k->m, k->n, k->k, 4, st);
    case SM100_K_KV_APPEND: {
      const int64_t ld = k->ld_in ? k->ld_in : k->k;
      return sm100_kv_append((float *)out, (const float *)p[0], (const float *)p[1], ld, (const int32_t *)p[7],
                             k->pos, (int32_t)k->m, (int32_t)k->k, k->max_ctx, st);
    }
    case SM100_K_POS_ADD:
      if (!out) return sm100_set_error(SM100_ERR_ARG, "pos_add: dead counter buffer");
      return sm100_pos_add((int32_t *)out, k->pos, st);
    case SM100_K_DECODE_STEP:
      if (!p[0]) return sm100_set_error(SM100_ERR_ARG, "decode_step: no model descriptor");
      return sm100_decode_steps((const Sm100DecodeModel *)p[0], k->n > 0 ? (int32_t)k->n : 1, (int32_t)k->m,
                                (int32_t)k->k, k->heads, (int32_t)k->ld_out, k->max_ctx, st);
    case SM100_K_ATTN_PREFILL:
      if (k->causal != 1) return sm100_set_error(SM100_ERR_UNSUPPORTED, "attn_prefill: causal only");
      if (k->dtype != SM100_DT_BF16) return sm100_set_error(SM100_ERR_UNSUPPORTED, "attn_prefill: bf16 q/k/v only");
      if (k->m > INT32_MAX || k->n > INT32_MAX || k->k > INT32_MAX)
        return sm100_set_error(SM100_ERR_ARG, "attn_prefill: shape out of range");
      return sm100_attn_prefill_bf16(p[0], p[1], p[2], (float *)out, (int32_t)k->m, k->heads, (int32_t)k->n,
                                     (int32_t)k->k, k->scale, (k->flags & 1u) ? 0 : 1, st);
    default:
      return sm100_set_error(SM100_ERR_UNSUPPORTED, "dispatch_kernel: kind %u", k->kind);
  }
}

int sm100_gather_strided(uint32_t dst, uint32_t src, const Sm100View *view) {
  if (!READY || HOST_MODE) return sm100_set_error(SM100_ERR_STATE, "gather_strided: no device");
  if (!live_id(dst) || !live_id(src) || !view) return sm100_set_error(SM100_ERR_ARG, "gather_strided: bad buffers");
  int64_t total = 1, hi = view->offset;
  for (uint32_t d = 0; d < view->ndim && d < 8; d++) {
    total *= view->dims[d];
    if (view->dims[d] > 0) hi += (view->dims[d] - 1) * (view->strides[d] > 0 ? view->strides[d] : 0);
  }
  if ((uint64_t)total * view->elem_bytes > BUFS[dst].req ||
      (total > 0 && (uint64_t)(hi + 1) * view->elem_bytes > BUFS[src].req) || view->offset < 0)
    return sm100_set_error(SM100_ERR_ARG, "gather_strided: view outside the buffers");
  return sm100_gather_strided_dev(BUFS[dst].ptr, BUFS[src].ptr, view, (void *)STREAM);
}

/* ---- CUDA graphs (src/backend/cuda/jit.c:444-604) ----------------------- */

int sm100_graph_capturing(void) { return CAPTURING; }

int sm100_graph_capture_begin(uint32_t slot) {
  if (!READY || HOST_MODE) return sm100_set_error(SM100_ERR_STATE, "graph: no device");
  if (slot >= GRAPH_SLOTS) return sm100_set_error(SM100_ERR_ARG, "graph: slot %u", slot);
  if (CAPTURING) return sm100_set_error(SM100_ERR_STATE, "graph: capture already open");
  sm100_graph_drop(slot);
  cudaError_t e = cudaStreamBeginCapture(STREAM, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_fail("cudaStreamBeginCapture", e);
  CAPTURING = 1;
  CAPTURE_SLOT = slot;
  return SM100_OK;
}

int sm100_graph_capture_end(uint32_t slot) {
  if (!CAPTURING || slot != CAPTURE_SLOT) return sm100_set_error(SM100_ERR_STATE, "graph: no capture open on slot %u", slot);
  CAPTURING = 0;
  cudaGraph_t g = NULL;
  cudaError_t e = cudaStreamEndCapture(STREAM, &g);
  if (e != cudaSuccess) return cuda_fail("cudaStreamEndCapture", e);
  cudaGraphExec_t x = NULL;
  e = cudaGraphInstantiate(&x, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return cuda_fail("cudaGraphInstantiate", e);
  }
  size_t n = 0;
  cudaGraphGetNodes(g, NULL, &n);
  uint64_t kernels = 0;
  if (n) {
    cudaGraphNode_t *nodes = (cudaGraphNode_t *)malloc(sizeof(cudaGraphNode_t) * n);
    if (nodes && cudaGraphGetNodes(g, nodes, &n) == cudaSuccess) {
      for (size_t i = 0; i < n; i++) {
        enum cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
      }
    }
    free(nodes);
  }
  GRAPHS[slot].graph = g;
  GRAPHS[slot].exec = x;
  GRAPHS[slot].kernels = kernels;
  /* launches recorded during capture did not run */
  LAUNCHES -= kernels <= LAUNCHES ? kernels : LAUNCHES;
  return SM100_OK;
}

int sm100_graph_replay(uint32_t slot) {
  if (slot >= GRAPH_SLOTS || !GRAPHS[slot].exec) return sm100_set_error(SM100_ERR_STATE, "graph: slot %u empty", slot);
  cudaError_t e = cudaGraphLaunch(GRAPHS[slot].exec, STREAM);
  if (e != cudaSuccess) return cuda_fail("cudaGraphLaunch", e);
  LAUNCHES += GRAPHS[slot].kernels;
  return SM100_OK;
}

void sm100_graph_drop(uint32_t slot) {
  if (slot >= GRAPH_SLOTS) return;
  if (GRAPHS[slot].exec) cudaGraphExecDestroy(GRAPHS[slot].exec);
  if (GRAPHS[slot].graph) cudaGraphDestroy(GRAPHS[slot].graph);
  memset(&GRAPHS[slot], 0, sizeof GRAPHS[slot]);
}
