// k_interp.cu - the generic device interpreter for lifted UOp DAGs that no
// hand-written kernel covers (include/thvm_sm100.h, "generic device
// interpreter").  The program, the buffer addresses and the runtime values
// travel by value in the kernel parameters (a __grid_constant__ block of
// ~16 KB), so a launch needs no device allocation and a stream capture
// records it whole.  One thread per output element, grid-stride over them;
// registers and range slots are thread-local.
#include "common.cuh"
#include "interp_core.h"

__device__ int g_interp_status;

namespace {

// C instructions of capacity: small programs travel in small parameter blocks
template <int C>
struct InterpParams {
  Sm100Insn code[C];
  void *bufs[SM100_INTERP_MAX_BUFS];
  int64_t buf_bytes[SM100_INTERP_MAX_BUFS];
  int64_t vars[SM100_INTERP_MAX_VARS];
  int64_t glob_ext[SM100_INTERP_MAX_AXES];
  int64_t total;
  uint32_t n_code, n_glob;
};

// The program is copied into shared memory once per CTA: every thread fetches
// the same instruction each step (a broadcast read), far cheaper than an
// indexed read of the parameter block.
template <int C>
__global__ void __launch_bounds__(128) interp_kernel(const __grid_constant__ InterpParams<C> p) {
  __shared__ Sm100Insn code[C];
  for (uint32_t i = threadIdx.x; i < p.n_code; i += blockDim.x) code[i] = p.code[i];
  __syncthreads();
  int64_t r[SM100_INTERP_MAX_REGS];
  int64_t idx[SM100_INTERP_MAX_AXES];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < p.total; t += stride) {
    int64_t rest = t;
    for (int d = (int)p.n_glob - 1; d >= 0; d--) {
      idx[d] = rest % p.glob_ext[d];
      rest /= p.glob_ext[d];
    }
    if (sm100_interp_exec(code, p.n_code, r, idx, p.bufs, p.buf_bytes, p.vars)) atomicOr(&g_interp_status, 1);
  }
}

template <int C>
int interp_launch(const Sm100Insn *code, uint32_t n_code, uint32_t n_glob, const int64_t *glob_ext,
                  void *const *bufs, const int64_t *buf_bytes, uint32_t n_bufs, const int64_t *vars, uint32_t n_vars,
                  int64_t total, cudaStream_t stream) {
  InterpParams<C> p;  // host staging; copied into the launch's parameters
  memset(&p, 0, sizeof p);
  memcpy(p.code, code, n_code * sizeof(Sm100Insn));
  for (uint32_t d = 0; d < n_glob; d++) p.glob_ext[d] = glob_ext[d];
  for (uint32_t i = 0; i < n_bufs; i++) p.bufs[i] = bufs[i], p.buf_bytes[i] = bufs[i] ? buf_bytes[i] : 0;
  for (uint32_t i = 0; i < n_vars; i++) p.vars[i] = vars[i];
  p.total = total;
  p.n_code = n_code;
  p.n_glob = n_glob;
  const int threads = 128;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  interp_kernel<C><<<(unsigned)blocks, threads, 0, stream>>>(p);
  return sm100::launch_status("interp_kernel");
}

}  // namespace

extern "C" int sm100_interp_run(const Sm100Insn *code, uint32_t n_code, uint32_t n_regs, uint32_t n_axes,
                                uint32_t n_glob, const int64_t *glob_ext, void *const *bufs,
                                const int64_t *buf_bytes, uint32_t n_bufs, const int64_t *vars, uint32_t n_vars,
                                void *stream) {
  if (!code || n_code == 0 || n_code > SM100_INTERP_MAX_CODE || n_regs > SM100_INTERP_MAX_REGS ||
      n_axes > SM100_INTERP_MAX_AXES || n_glob > n_axes || n_bufs > SM100_INTERP_MAX_BUFS ||
      n_vars > SM100_INTERP_MAX_VARS || (n_glob && !glob_ext) || (n_bufs && (!bufs || !buf_bytes)) || (n_vars && !vars))
    return sm100_set_error(SM100_ERR_ARG, "interp_run: bad program (%u insns, %u regs, %u axes)", n_code, n_regs,
                           n_axes);
  const Sm100Insn *pc = code;
  // every operand index must name a register / slot of the program
  for (uint32_t i = 0; i < n_code; i++) {
    const Sm100Insn &in = pc[i];
    if (in.op == 0 || in.op >= SM100_IOP_COUNT || in.dst >= SM100_INTERP_MAX_REGS ||
        in.a >= SM100_INTERP_MAX_REGS || in.b >= SM100_INTERP_MAX_REGS || in.c >= SM100_INTERP_MAX_REGS)
      return sm100_set_error(SM100_ERR_ARG, "interp_run: bad instruction %u", i);
    if ((in.op == SM100_IOP_LOAD || in.op == SM100_IOP_STORE) && in.a >= n_bufs)
      return sm100_set_error(SM100_ERR_ARG, "interp_run: instruction %u names buffer %u of %u", i, in.a, n_bufs);
    if ((in.op == SM100_IOP_RANGE || in.op == SM100_IOP_LOOP || in.op == SM100_IOP_ENDLOOP ||
         in.op == SM100_IOP_SETR) && in.a >= n_axes)
      return sm100_set_error(SM100_ERR_ARG, "interp_run: instruction %u names range slot %u", i, in.a);
    if (in.op == SM100_IOP_VAR && in.a >= n_vars)
      return sm100_set_error(SM100_ERR_ARG, "interp_run: instruction %u names var %u", i, in.a);
    if ((in.op == SM100_IOP_LOOP || in.op == SM100_IOP_ENDLOOP) && (in.imm < 0 || (uint32_t)in.imm >= n_code))
      return sm100_set_error(SM100_ERR_ARG, "interp_run: instruction %u jumps outside the program", i);
  }
  if (sm100_interp_check_loops(pc, n_code))
    return sm100_set_error(SM100_ERR_ARG, "interp_run: loops are not well nested");
  int64_t total = 1;
  for (uint32_t d = 0; d < n_glob; d++) {
    if (glob_ext[d] < 0) return sm100_set_error(SM100_ERR_ARG, "interp_run: negative extent");
    total *= glob_ext[d];
  }
  if (total == 0) return SM100_OK;
  const cudaStream_t st = (cudaStream_t)stream;
  if (n_code <= 64) return interp_launch<64>(code, n_code, n_glob, glob_ext, bufs, buf_bytes, n_bufs, vars, n_vars, total, st);
  if (n_code <= 256)
    return interp_launch<256>(code, n_code, n_glob, glob_ext, bufs, buf_bytes, n_bufs, vars, n_vars, total, st);
  return interp_launch<SM100_INTERP_MAX_CODE>(code, n_code, n_glob, glob_ext, bufs, buf_bytes, n_bufs, vars, n_vars,
                                              total, st);
}

extern "C" int sm100_interp_status(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_interp_status, sizeof v) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_interp_status, &z, sizeof z);
  }
  return v;
}
