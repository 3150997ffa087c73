/* custom.c - the custom-kernel ABI on the sm_100a device: raw CUDA-C
 * programs handed in by the host (the reference's kernel_emit_custom_program,
 * src/schedule/kernel_custom.c:47-136, fired by cuda_custom_dispatch,
 * src/backend/cuda/jit.c:802-893).
 *
 * A program is `extern "C" __global__ void name(T *arg0, ...)` source text
 * with a fixed grid / block and dynamic shared size.  Registration compiles
 * it once with NVRTC for sm_100a (a real-architecture cubin, no PTX JIT at
 * launch) and loads it through the runtime's library API; compiled modules
 * are kept in a table keyed by an FNV-1a hash of (name, source), so
 * registering the same program again compiles nothing.  Dispatch only
 * launches: args[i] = the device address of argument i's buffer, with
 * out_buf_id rebinding the primary output slot (the reference's replay-time
 * rebinding, jit.c:826-833), on the backend stream, so a graph capture of
 * the backend stream records custom launches like any other kernel.
 *
 * NVRTC is loaded with dlopen when the first program is registered: the
 * library itself does not depend on it, and a host without it gets an error
 * from sm100_custom_program, never a fallback.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "../../include/thvm_sm100.h"

/* backend.c: the error string and the launch counter */
int sm100_set_error(int code, const char *fmt, ...);
void sm100_note_launch(void);

#define CUSTOM_CAP 256
#define CUSTOM_MAX_ARGS 64 /* the reference's custom ABI limit (kernel_custom.c) */

/* ---- NVRTC through dlopen (names and signatures of nvrtc.h) --------------- */
typedef int nvrtcResult_;
typedef struct _nvrtcProgram *nvrtcProgram_;
static struct {
  int tried, ok;
  nvrtcResult_ (*create)(nvrtcProgram_ *, const char *, const char *, int, const char *const *, const char *const *);
  nvrtcResult_ (*compile)(nvrtcProgram_, int, const char *const *);
  nvrtcResult_ (*log_size)(nvrtcProgram_, size_t *);
  nvrtcResult_ (*log)(nvrtcProgram_, char *);
  nvrtcResult_ (*cubin_size)(nvrtcProgram_, size_t *);
  nvrtcResult_ (*cubin)(nvrtcProgram_, char *);
  nvrtcResult_ (*destroy)(nvrtcProgram_ *);
  const char *(*err)(nvrtcResult_);
} NV;

static int nvrtc_load(void) {
  if (NV.tried) return NV.ok;
  NV.tried = 1;
  static const char *const names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12",
                                      "/usr/local/cuda/lib64/libnvrtc.so"};
  void *h = NULL;
  for (size_t i = 0; i < sizeof names / sizeof names[0] && !h; i++) h = dlopen(names[i], RTLD_NOW | RTLD_LOCAL);
  if (!h) return 0;
#define NV_SYM(field, sym) *(void **)(&NV.field) = dlsym(h, sym)
  NV_SYM(create, "nvrtcCreateProgram");
  NV_SYM(compile, "nvrtcCompileProgram");
  NV_SYM(log_size, "nvrtcGetProgramLogSize");
  NV_SYM(log, "nvrtcGetProgramLog");
  NV_SYM(cubin_size, "nvrtcGetCUBINSize");
  NV_SYM(cubin, "nvrtcGetCUBIN");
  NV_SYM(destroy, "nvrtcDestroyProgram");
  NV_SYM(err, "nvrtcGetErrorString");
#undef NV_SYM
  NV.ok = NV.create && NV.compile && NV.log_size && NV.log && NV.cubin_size && NV.cubin && NV.destroy && NV.err;
  return NV.ok;
}

/* ---- the tables ------------------------------------------------------------
 * A module is one compiled (name, source); a program is a module with a launch
 * shape.  Registering an identical (name, source, shape) returns its id; the
 * same source with another shape shares the module (no second compile). */
typedef struct {
  uint64_t key;
  char name[128];
  cudaLibrary_t lib;
  cudaKernel_t kernel;
  uint32_t shared_optin; /* the dynamic shared size the kernel is opted in to */
} Module;

typedef struct {
  int32_t module;
  uint32_t grid[3], block[3], shared;
} Program;

static Module MODS[CUSTOM_CAP + 1];   /* index 0 unused */
static Program PROGS[CUSTOM_CAP + 1]; /* id 0 = none */
static int32_t N_MODS = 0, N_PROGS = 0;

static dim3 dims(const uint32_t v[3]) {
  dim3 d;
  d.x = v[0];
  d.y = v[1];
  d.z = v[2];
  return d;
}

static uint64_t fnv1a(uint64_t h, const char *s) {
  for (; *s; s++) h = (h ^ (uint8_t)*s) * 0x100000001b3ull;
  return (h ^ 0xff) * 0x100000001b3ull; /* a separator between the fields */
}

/* compile `src` to an sm_100a cubin; returns a malloc'd image or NULL with the error set */
static char *compile_cubin(const char *name, const char *src, size_t *size) {
  nvrtcProgram_ prog = NULL;
  nvrtcResult_ r = NV.create(&prog, src, name, 0, NULL, NULL);
  if (r != 0) {
    sm100_set_error(SM100_ERR_UNSUPPORTED, "custom %s: nvrtcCreateProgram: %s", name, NV.err(r));
    return NULL;
  }
  static const char *const opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-lineinfo"};
  r = NV.compile(prog, (int)(sizeof opts / sizeof opts[0]), opts);
  if (r != 0) {
    size_t n = 0;
    NV.log_size(prog, &n);
    char *log = (char *)malloc(n + 1);
    if (log) {
      log[0] = 0;
      NV.log(prog, log);
      log[n] = 0;
    }
    sm100_set_error(SM100_ERR_UNSUPPORTED, "custom %s: compile failed: %s", name, log ? log : NV.err(r));
    free(log);
    NV.destroy(&prog);
    return NULL;
  }
  char *img = NULL;
  if (NV.cubin_size(prog, size) == 0 && *size > 0 && (img = (char *)malloc(*size)) != NULL &&
      NV.cubin(prog, img) != 0) {
    free(img);
    img = NULL;
  }
  NV.destroy(&prog);
  if (!img) sm100_set_error(SM100_ERR_UNSUPPORTED, "custom %s: no cubin", name);
  return img;
}

int32_t sm100_custom_program(const char *name, const char *src, const uint32_t grid[3], const uint32_t block[3],
                             uint32_t shared_bytes) {
  if (!name || !src || !grid || !block || !name[0] || strlen(name) >= sizeof MODS[0].name)
    return sm100_set_error(SM100_ERR_ARG, "custom: name, source, grid and block are required");
  uint64_t threads = (uint64_t)block[0] * block[1] * block[2];
  if (!grid[0] || !grid[1] || !grid[2] || !block[0] || !block[1] || !block[2] || threads > 1024 ||
      grid[1] > 65535 || grid[2] > 65535 || block[2] > 64 || shared_bytes > 227u * 1024u)
    return sm100_set_error(SM100_ERR_ARG, "custom %s: launch shape out of range (block <= 1024 threads, "
                                          "shared <= 227 KiB)", name);
  const uint64_t key = fnv1a(fnv1a(0xcbf29ce484222325ull, name), src);
  int32_t m = 0;
  for (int32_t i = 1; i <= N_MODS && !m; i++)
    if (MODS[i].key == key && strcmp(MODS[i].name, name) == 0) m = i;
  if (m)
    for (int32_t i = 1; i <= N_PROGS; i++)
      if (PROGS[i].module == m && !memcmp(PROGS[i].grid, grid, 12) && !memcmp(PROGS[i].block, block, 12) &&
          PROGS[i].shared == shared_bytes)
        return i;
  if (N_PROGS >= CUSTOM_CAP || (!m && N_MODS >= CUSTOM_CAP))
    return sm100_set_error(SM100_ERR_OOM, "custom %s: program table full", name);
  if (!m) {
    if (!nvrtc_load()) return sm100_set_error(SM100_ERR_UNSUPPORTED, "custom %s: libnvrtc not found", name);
    size_t size = 0;
    char *img = compile_cubin(name, src, &size);
    if (!img) return SM100_ERR_UNSUPPORTED;
    if (!sm100_ready()) {
      free(img);
      return sm100_set_error(SM100_ERR_STATE, "custom %s: compiled, but the device is not initialised", name);
    }
    Module md;
    memset(&md, 0, sizeof md);
    cudaError_t e = cudaLibraryLoadData(&md.lib, img, NULL, NULL, 0, NULL, NULL, 0);
    free(img);
    if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "custom %s: load: %s", name, cudaGetErrorString(e));
    e = cudaLibraryGetKernel(&md.kernel, md.lib, name);
    if (e != cudaSuccess) {
      cudaLibraryUnload(md.lib);
      return sm100_set_error(SM100_ERR_ARG, "custom %s: no extern \"C\" __global__ of that name: %s", name,
                             cudaGetErrorString(e));
    }
    md.key = key;
    snprintf(md.name, sizeof md.name, "%s", name);
    MODS[m = ++N_MODS] = md;
  }
  if (shared_bytes > 48u * 1024u && shared_bytes > MODS[m].shared_optin) {   /* the opt-in above 48 KiB */
    const cudaError_t e = cudaFuncSetAttribute((const void *)MODS[m].kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shared_bytes);
    if (e != cudaSuccess)
      return sm100_set_error(SM100_ERR_CUDA, "custom %s: shared %u: %s", name, shared_bytes, cudaGetErrorString(e));
    MODS[m].shared_optin = shared_bytes;
  }
  Program p;
  p.module = m;
  memcpy(p.grid, grid, sizeof p.grid);
  memcpy(p.block, block, sizeof p.block);
  p.shared = shared_bytes;
  PROGS[++N_PROGS] = p;
  return N_PROGS;
}

int sm100_custom_launch(int32_t prog, void *const *arg_ptrs, uint32_t n_args, void *stream) {
  if (prog < 1 || prog > N_PROGS) return sm100_set_error(SM100_ERR_ARG, "custom: no program %d", prog);
  if (n_args > CUSTOM_MAX_ARGS || (n_args && !arg_ptrs))
    return sm100_set_error(SM100_ERR_ARG, "custom: %u arguments (at most %d)", n_args, CUSTOM_MAX_ARGS);
  const Program *p = &PROGS[prog];
  const Module *md = &MODS[p->module];
  void *vals[CUSTOM_MAX_ARGS];
  void *args[CUSTOM_MAX_ARGS];
  for (uint32_t i = 0; i < n_args; i++) {
    vals[i] = arg_ptrs[i];
    args[i] = &vals[i];
  }
  const cudaError_t e = cudaLaunchKernel((const void *)md->kernel, dims(p->grid), dims(p->block), args, p->shared,
                                         (cudaStream_t)stream);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "custom %s: launch: %s", md->name, cudaGetErrorString(e));
  sm100_note_launch();
  return SM100_OK;
}

int sm100_custom_dispatch(int32_t prog, const uint32_t *arg_buf_ids, uint32_t n_args, uint32_t primary_out_slot,
                          uint32_t out_buf_id) {
  if (!sm100_ready()) return sm100_set_error(SM100_ERR_STATE, "custom: not initialised");
  if (n_args > CUSTOM_MAX_ARGS || (n_args && !arg_buf_ids))
    return sm100_set_error(SM100_ERR_ARG, "custom: %u arguments (at most %d)", n_args, CUSTOM_MAX_ARGS);
  void *ptrs[CUSTOM_MAX_ARGS];
  for (uint32_t i = 0; i < n_args; i++) {
    ptrs[i] = sm100_buf_dptr(arg_buf_ids[i]);
    if (!ptrs[i]) return sm100_set_error(SM100_ERR_ARG, "custom: argument %u: dead buffer %u", i, arg_buf_ids[i]);
  }
  if (out_buf_id != 0 && primary_out_slot < n_args) {
    ptrs[primary_out_slot] = sm100_buf_dptr(out_buf_id);
    if (!ptrs[primary_out_slot]) return sm100_set_error(SM100_ERR_ARG, "custom: dead output buffer %u", out_buf_id);
  }
  return sm100_custom_launch(prog, ptrs, n_args, sm100_stream());
}
