/* sm100_ref.c - the reference-side half of the sm_100a device: the router
 * that hands the reference scheduler's realized kernels to this device.
 *
 * Compiled as ONE translation unit together with the reference's runtime: it
 * #includes py/csource/thvm_py.c (which #includes src/thvm.c and with it
 * every runtime .c) from the reference checkout, unmodified.  The reference's
 * UOp accessors (term_tag, heap_read, uop_buffer_*, term_dtype_in,
 * uop_dag_classify_matmul_shape, kvar_extent_runtime ...) are static inline
 * in that unit, which is why the router lives here and not in
 * libthvm_sm100.so.
 *
 * Every KernelEntry the backend is asked to run (Backend.dispatch_kernel,
 * src/thvm.h:818; the CUDA one is src/backend/cuda/jit.c:895-1170) goes
 * through sm100_ref_plan():
 *   1. LINEAR: y[M,N] = P[M,K] . W[N,K]^T where the A side P is a plain input
 *      row block or any expression the interpreter can evaluate (a fused
 *      LayerNorm, residual sum, bias + GELU ...) and W a row-major weight
 *      input: the A side runs on the interpreter into a scratch block (none
 *      when it is a plain input), the product on the library's hand-written
 *      matvec / linear kernel (sm100_linear).
 *   2. INTERP: any other single-STORE DAG over f32 / int / bool / f16 / bf16
 *      data compiles to a register program for the generic device
 *      interpreter (sm100_interp_run).
 *   3. Otherwise the reference's own path runs it unchanged (declined, with
 *      the reason).
 * Programs are cached per DAG root.
 *
 * THVM_HAS_CUDA build (the device): at load time CUDA_BACKEND.dispatch_kernel
 * is pointed at the router; routed kernels run on the backend's own device
 * buffers (cuda_buf_dptr) on its current stream (CUDA_CUR_STREAM), so the
 * reference's TinyJit stream capture records them like rendered kernels.
 * THVM_SM100=0 turns routing off.
 *
 * CPU build (the checker, no THVM_HAS_CUDA): with THVM_SM100_CHECK=1 the
 * router runs beside the CPU backend: each dispatched kernel is planned, and
 * each planned one is executed by the same interpreter core on the host
 * (thvm_b200/csrc/interp_core.h) over copies of the buffers the CPU backend
 * read, and compared with the output it wrote.
 *
 * Both builds: THVM_SM100_LOG=<path> writes one line per dispatch (kernel id,
 * route or the reason it was declined), THVM_SM100_DUMP=1 adds the DAG;
 * py_sm100_ref_stats() returns the counters.
 */
#include "py/csource/thvm_py.c"

#include <math.h>
#include <stdarg.h>

#include "thvm_sm100.h"
#include "../csrc/interp_core.h"

/* ---- logging -------------------------------------------------------------- */

static FILE *sm100_log_fp(void) {
  static int init = 0;
  static FILE *fp = NULL;
  if (!init) {
    init = 1;
    const char *p = getenv("THVM_SM100_LOG");
    if (p && *p) fp = fopen(p, "w");
  }
  return fp;
}

static int sm100_env_on(const char *name, int dflt) {
  const char *e = getenv(name);
  return e ? e[0] == '1' : dflt;
}

static const char *sm100_op_name(u32 op) {
  switch (op) {
    case UOP_CONST: return "CONST";
    case UOP_ADD: return "ADD";
    case UOP_MUL: return "MUL";
    case UOP_NEG: return "NEG";
    case UOP_RECIP: return "RECIP";
    case UOP_EXP2: return "EXP2";
    case UOP_LOG2: return "LOG2";
    case UOP_SQRT: return "SQRT";
    case UOP_CMPLT: return "CMPLT";
    case UOP_REDUCE: return "REDUCE";
    case UOP_DEFINE_VAR: return "DEFINE_VAR";
    case UOP_CMPEQ: return "CMPEQ";
    case UOP_CAST: return "CAST";
    case UOP_BITCAST: return "BITCAST";
    case UOP_RANGE: return "RANGE";
    case UOP_INDEX_E: return "INDEX";
    case UOP_IADD: return "IADD";
    case UOP_ISUB: return "ISUB";
    case UOP_IMUL: return "IMUL";
    case UOP_IDIV: return "IDIV";
    case UOP_IMOD: return "IMOD";
    case UOP_ILT: return "ILT";
    case UOP_IAND: return "IAND";
    case UOP_IOR: return "IOR";
    case UOP_IXOR: return "IXOR";
    case UOP_ISHR: return "ISHR";
    case UOP_ISHL: return "ISHL";
    case UOP_IWHERE: return "IWHERE";
    case UOP_INVALID: return "INVALID";
    case UOP_BUFFER: return "BUFFER";
    case UOP_STORE: return "STORE";
    case UOP_AFTER: return "AFTER";
    case UOP_OPT: return "OPT";
    case UOP_POW: return "POW";
    case UOP_THREEFRY: return "THREEFRY";
    case UOP_GATHER: return "GATHER";
    case UOP_SCATTER: return "SCATTER";
    case UOP_SIN: return "SIN";
    default: return "?";
  }
}

static int sm100_is(Term t, u32 op) { return term_tag(t) == TAG_UOP && term_ext(t) == op; }

static int sm100_arity(u32 op) {
  switch (op) {
    case UOP_NEG: case UOP_RECIP: case UOP_EXP2: case UOP_LOG2: case UOP_SQRT: case UOP_SIN: return 1;
    case UOP_IWHERE: case UOP_STORE: return 3;
    case UOP_ADD: case UOP_MUL: case UOP_CMPLT: case UOP_CMPEQ: case UOP_IADD: case UOP_ISUB: case UOP_IMUL:
    case UOP_IDIV: case UOP_IMOD: case UOP_ILT: case UOP_IAND: case UOP_IOR: case UOP_IXOR: case UOP_ISHR:
    case UOP_ISHL: case UOP_INDEX_E: case UOP_AFTER: case UOP_POW: case UOP_THREEFRY: return 2;
    default: return 0;
  }
}

static void sm100_dump(FILE *f, Term t, int depth) {
  if (depth > 28) {
    fputs("...", f);
    return;
  }
  if (term_tag(t) == TAG_NUM) {
    fprintf(f, "#%u", (u32)term_val(t));
    return;
  }
  if (term_tag(t) != TAG_UOP) {
    fprintf(f, "<tag%u>", (u32)term_tag(t));
    return;
  }
  u32 op = term_ext(t);
  u64 loc = term_val(t);
  switch (op) {
    case UOP_CONST: {
      Term n = heap_read(loc);
      u32 bits = (u32)term_val(n);
      float fv;
      memcpy(&fv, &bits, 4);
      if (term_ext(n) == DT_FP32) fprintf(f, "%.9g", (double)fv);
      else fprintf(f, "%d", (int)bits);
      return;
    }
    case UOP_RANGE: fprintf(f, "r%u<%u>", uop_range_axis_id(t), uop_range_extent(t)); return;
    case UOP_BUFFER:
      fprintf(f, "B%u[", uop_buffer_inst_get(t));
      for (u32 d = 0; d < uop_buffer_ndim(t); d++) fprintf(f, d ? ",%u" : "%u", uop_buffer_dim(t, d));
      fputc(']', f);
      return;
    case UOP_DEFINE_VAR: fprintf(f, "var(%u)", (u32)term_val(heap_read(loc))); return;
    case UOP_REDUCE:
      fprintf(f, "REDUCE%u(", uop_reduce_kind(t));
      sm100_dump(f, heap_read(loc), depth + 1);
      for (u32 i = 0; i < uop_reduce_n_axes(t); i++) fprintf(f, ",r%u", uop_reduce_axis(t, i));
      fputc(')', f);
      return;
    case UOP_CAST: case UOP_BITCAST: case UOP_OPT:
      fprintf(f, "%s<%u>(", sm100_op_name(op), (u32)term_val(heap_read(loc + 1)));
      sm100_dump(f, heap_read(loc), depth + 1);
      fputc(')', f);
      return;
    case UOP_INVALID: fputs("INVALID", f); return;
    default: break;
  }
  fprintf(f, "%s(", sm100_op_name(op));
  for (int i = 0; i < sm100_arity(op); i++) {
    if (i) fputc(',', f);
    sm100_dump(f, heap_read(loc + (u64)i), depth + 1);
  }
  fputc(')', f);
}

/* ---- the DAG -> register program compiler ---------------------------------- */

#define SM100_MEMO_CAP 1024
#define SM100_MAX_PRE 16   /* pre-pass programs of a family */
#define SM100_MAX_SCR 16   /* scratch buffers of a family */
#define SM100_AX_CHUNK 62  /* axis ids of the pre-pass programs' own ranges */
#define SM100_AX_STEP 63

typedef struct Sm100Prog Sm100Prog;
struct Sm100Prog {
  /* the program */
  Sm100Insn code[SM100_INTERP_MAX_CODE];
  u32 n_code, n_regs;
  u32 axis_id[SM100_INTERP_MAX_AXES], n_axes, n_glob;
  u32 glob_packed[SM100_INTERP_MAX_AXES]; /* RANGE extent fields of the output axes */
  u32 var_packed[SM100_INTERP_MAX_VARS], n_vars;
  /* compile state */
  u64 bound; /* axis-id mask of the range slots open now */
  Term memo_t[SM100_MEMO_CAP];
  u16 memo_r[SM100_MEMO_CAP];
  u32 n_memo;
  Term dep_t[SM100_MEMO_CAP];
  u64 dep_m[SM100_MEMO_CAP];
  u32 n_dep;
  int bad;
  char why[160];
  /* Reduces that every output element would recompute (they read no range
   * of this program's fastest output axis, or run long) move to pre-pass
   * programs of the family: P1 folds chunks of about sqrt(E) iterations into
   * partials, P2 folds each output row's partials in chunk order, and the
   * readers load the result from scratch.  The family lives on its root
   * program: pre-passes run in list order before it, each with buffer slot
   * 0 bound to its scratch output, slots 1..n_in to the kernel's inputs and
   * slots n_in + 1 + j to scratch j. */
  Sm100Prog *root;
  u32 n_in;
  int allow_pre;
  Sm100Prog *pre[SM100_MAX_PRE];
  int pre_out[SM100_MAX_PRE];
  u32 n_pre;
  u64 scr_bytes[SM100_MAX_SCR];
  void *scr_ptr[SM100_MAX_SCR];
  u32 n_scr;
  Term ur_t[SM100_MAX_PRE];    /* hoisted reduces and their result scratch / row axes */
  u32 ur_scr[SM100_MAX_PRE], ur_dt[SM100_MAX_PRE];
  u64 ur_dmask[SM100_MAX_PRE];
  u32 n_ur;
};

static void sp_fail(Sm100Prog *p, const char *fmt, ...) {
  if (p->bad) return;
  p->bad = 1;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(p->why, sizeof p->why, fmt, ap);
  va_end(ap);
}

static u16 sp_reg(Sm100Prog *p) {
  if (p->n_regs >= SM100_INTERP_MAX_REGS) {
    sp_fail(p, "more than %d registers", SM100_INTERP_MAX_REGS);
    return 0;
  }
  return (u16)p->n_regs++;
}

static u32 sp_emit(Sm100Prog *p, u8 op, u8 dt, u16 dst, u16 a, u16 b, u16 c, i32 imm) {
  if (p->n_code >= SM100_INTERP_MAX_CODE) {
    sp_fail(p, "more than %d instructions", SM100_INTERP_MAX_CODE);
    return 0;
  }
  Sm100Insn *in = &p->code[p->n_code];
  in->op = op, in->dt = dt, in->dst = dst, in->a = a, in->b = b, in->c = c, in->imm = imm;
  return p->n_code++;
}

static u16 sp_op(Sm100Prog *p, u8 op, u8 dt, u16 a, u16 b, u16 c, i32 imm) {
  u16 d = sp_reg(p);
  sp_emit(p, op, dt, d, a, b, c, imm);
  return d;
}

static u16 sp_const_i(Sm100Prog *p, i64 v) {
  if (v < INT32_MIN || v > (i64)UINT32_MAX) sp_fail(p, "int constant %lld", (long long)v);
  return sp_op(p, SM100_IOP_CONST, v < 0 ? 0 : 1, 0, 0, 0, (i32)(u32)v);
}

static u16 sp_const_f(Sm100Prog *p, float f) {
  u32 b;
  memcpy(&b, &f, 4);
  return sp_op(p, SM100_IOP_CONST, 2, 0, 0, 0, (i32)b);
}

static int sp_isfloat(u32 dt) {
  return dt == DT_FP32 || dt == DT_FP64 || dt == DT_FP16 || dt == DT_BF16 || dt == DT_FP8E4M3 || dt == DT_FP8E5M2;
}

/* The C type the reference's walker gives a node (uwalk_term_dtype_of,
 * src/backend/cpu/uop_walk.c:357-412): halves and bf16 compute as f32. */
static u32 sp_ty(Sm100Prog *p, Term t) {
  if (term_tag(t) == TAG_NUM) return DT_INT64;
  if (term_tag(t) != TAG_UOP) return DT_INT64;
  u64 loc = term_val(t);
  u32 dt = DT_FP32;
  switch (term_ext(t)) {
    case UOP_CONST: {
      dt = term_ext(heap_read(loc));
      if (sp_isfloat(dt) && dt != DT_FP32) sp_fail(p, "float constant of dtype %u", dt);
      return dt;
    }
    case UOP_DEFINE_VAR: return DT_INT32;
    case UOP_CAST: case UOP_BITCAST:
      dt = (u32)term_val(heap_read(loc + 1));
      return sp_isfloat(dt) ? (dt == DT_FP64 ? DT_FP64 : DT_FP32) : dt;
    case UOP_INDEX_E: {
      Term b = heap_read(loc);
      dt = sm100_is(b, UOP_BUFFER) ? uop_buffer_dtype(b) : DT_FP32;
      return sp_isfloat(dt) ? (dt == DT_FP64 ? DT_FP64 : DT_FP32) : dt;
    }
    case UOP_REDUCE:
      (void)term_dtype_in(t, 0, &dt);
      if (dtype_is_bool(dt) || dtype_is_int(dt)) return dt;
      return dt == DT_FP64 ? DT_FP64 : DT_FP32;
    case UOP_CMPLT: case UOP_CMPEQ: case UOP_ILT: return DT_BOOL;
    case UOP_RECIP: return sp_ty(p, heap_read(loc)) == DT_FP64 ? DT_FP64 : DT_FP32;
    case UOP_EXP2: case UOP_LOG2: case UOP_SQRT: case UOP_SIN:
      (void)term_dtype_in(t, 0, &dt);
      return dt == DT_FP32 ? DT_FP32 : DT_FP64;
    case UOP_NEG: case UOP_OPT: return sp_ty(p, heap_read(loc));
    case UOP_ADD: case UOP_MUL: case UOP_IWHERE: {
      const u32 a = sp_ty(p, heap_read(loc + (term_ext(t) == UOP_IWHERE ? 1 : 0)));
      const u32 b = sp_ty(p, heap_read(loc + (term_ext(t) == UOP_IWHERE ? 2 : 1)));
      if (a == DT_FP64 || b == DT_FP64) return DT_FP64;
      if (sp_isfloat(a) || sp_isfloat(b)) return DT_FP32;
      return b == DT_UINT64 ? b : a;
    }
    case UOP_POW: case UOP_THREEFRY:
      (void)term_dtype_in(t, 0, &dt);
      return dt;
    default: return DT_INT64;
  }
}

/* axis ids a node reads and does not reduce (memoised) */
static u64 sp_deps(Sm100Prog *p, Term t) {
  if (term_tag(t) != TAG_UOP) return 0;
  for (u32 i = 0; i < p->n_dep; i++)
    if (p->dep_t[i] == t) return p->dep_m[i];
  u32 op = term_ext(t);
  u64 loc = term_val(t), m = 0;
  if (op == UOP_RANGE) {
    u32 id = uop_range_axis_id(t);
    if (id >= 64) sp_fail(p, "axis id %u", id);
    m = 1ull << (id & 63);
  } else if (op == UOP_REDUCE) {
    m = sp_deps(p, heap_read(loc));
    for (u32 i = 0; i < uop_reduce_n_axes(t); i++) m &= ~(1ull << (uop_reduce_axis(t, i) & 63));
  } else if (op == UOP_CAST || op == UOP_BITCAST || op == UOP_OPT) {
    m = sp_deps(p, heap_read(loc));
  } else {
    for (int i = 0; i < sm100_arity(op); i++) m |= sp_deps(p, heap_read(loc + (u64)i));
  }
  if (p->n_dep < SM100_MEMO_CAP) p->dep_t[p->n_dep] = t, p->dep_m[p->n_dep++] = m;
  return m;
}

static int sp_slot(Sm100Prog *p, u32 axis) {
  for (u32 i = 0; i < p->n_axes; i++)
    if (p->axis_id[i] == axis) return (int)i;
  return -1;
}

static int sp_new_slot(Sm100Prog *p, u32 axis) {
  if (p->n_axes >= SM100_INTERP_MAX_AXES) {
    sp_fail(p, "more than %d ranges", SM100_INTERP_MAX_AXES);
    return 0;
  }
  p->axis_id[p->n_axes] = axis;
  return (int)p->n_axes++;
}

/* a register holding a (possibly kvar) packed extent */
static u16 sp_extent(Sm100Prog *p, u32 packed) {
  if (!(packed & KVAR_FLAG)) return sp_const_i(p, packed);
  if (p->n_vars >= SM100_INTERP_MAX_VARS) {
    sp_fail(p, "more than %d runtime values", SM100_INTERP_MAX_VARS);
    return 0;
  }
  p->var_packed[p->n_vars] = packed;
  return sp_op(p, SM100_IOP_VAR, 0, (u16)p->n_vars++, 0, 0, 0);
}

static Term sp_find_range(Term t, u32 axis, int depth) {
  if (term_tag(t) != TAG_UOP || depth > 64) return 0;
  u32 op = term_ext(t);
  if (op == UOP_RANGE) return uop_range_axis_id(t) == axis ? t : 0;
  u64 loc = term_val(t);
  int n = (op == UOP_REDUCE || op == UOP_CAST || op == UOP_BITCAST || op == UOP_OPT) ? 1 : sm100_arity(op);
  for (int i = 0; i < n; i++) {
    Term r = sp_find_range(heap_read(loc + (u64)i), axis, depth + 1);
    if (r) return r;
  }
  return 0;
}

static u16 sp_val(Sm100Prog *p, Term t);

/* t as an f32 register (uwalk_cast_float to f32) */
static u16 sp_float(Sm100Prog *p, Term t) {
  u32 dt = sp_ty(p, t);
  u16 r = sp_val(p, t);
  if (sp_isfloat(dt)) return r;
  return sp_op(p, SM100_IOP_I2F, (u8)dt, r, 0, 0, 0);
}

/* t as an int register (uwalk_eval_int) */
static u16 sp_int(Sm100Prog *p, Term t) {
  u32 dt = sp_ty(p, t);
  u16 r = sp_val(p, t);
  if (!sp_isfloat(dt)) return r;
  return sp_op(p, SM100_IOP_F2I, DT_INT64, r, 0, 0, 0);
}

static u16 sp_memo_get(Sm100Prog *p, Term t, int *hit) {
  for (u32 i = p->n_memo; i-- > 0;)
    if (p->memo_t[i] == t) {
      *hit = 1;
      return p->memo_r[i];
    }
  *hit = 0;
  return 0;
}

static void sp_hoist(Sm100Prog *p, Term t, int depth);

/* f at range `axis` = x, for an int expression of that range and constants
 * only (no load); *ok cleared for anything else */
static i64 sp_eval_pure(Term t, u32 axis, i64 x, int *ok, int depth) {
  if (!*ok || depth > 48 || term_tag(t) != TAG_UOP) {
    *ok = 0;
    return 0;
  }
  const u64 loc = term_val(t);
  switch (term_ext(t)) {
    case UOP_CONST: {
      const u32 dt = term_ext(heap_read(loc)), bits = (u32)term_val(heap_read(loc));
      if (sp_isfloat(dt)) break;
      return dtype_kind(dt) == DK_UINT ? (i64)bits : (i64)(i32)bits;
    }
    case UOP_RANGE:
      if (uop_range_axis_id(t) == axis) return x;
      break;
    case UOP_OPT: return sp_eval_pure(heap_read(loc), axis, x, ok, depth + 1);
    case UOP_NEG: return -sp_eval_pure(heap_read(loc), axis, x, ok, depth + 1);
    case UOP_ADD: case UOP_IADD: case UOP_ISUB: case UOP_MUL: case UOP_IMUL: case UOP_IDIV: case UOP_IMOD: {
      const i64 a = sp_eval_pure(heap_read(loc), axis, x, ok, depth + 1);
      const i64 b = sp_eval_pure(heap_read(loc + 1), axis, x, ok, depth + 1);
      switch (term_ext(t)) {
        case UOP_ADD: case UOP_IADD: return a + b;
        case UOP_ISUB: return a - b;
        case UOP_MUL: case UOP_IMUL: return a * b;
        case UOP_IDIV: return b ? a / b : 0;
        default: return b ? a % b : 0;
      }
    }
    default: break;
  }
  *ok = 0;
  return 0;
}

/* A one-hot reduce: SUM over v of IWHERE(f(v) == key, a(v), 0) with f the
 * identity over v's range (checked at every v) and key not reading v is the
 * gather a(key) for 0 <= key < extent, else 0: exactly the sum's one
 * non-zero term (the tinygrad embedding, py/thvm/tensor.py's one-hot
 * product).  Returns the register, or -1 when t is not of that form. */
static int sp_onehot(Sm100Prog *p, Term t, int is_int) {
  if (uop_reduce_kind(t) != REDUCE_SUM || uop_reduce_n_axes(t) != 1) return -1;
  const u32 ax = uop_reduce_axis(t, 0);
  Term body = uop_reduce_src(t);
  if (!sm100_is(body, UOP_IWHERE)) return -1;
  Term c = heap_read(term_val(body)), a = heap_read(term_val(body) + 1), z = heap_read(term_val(body) + 2);
  u32 zbits = 1;
  if (!(sm100_is(z, UOP_INVALID) || (sm100_is(z, UOP_CONST) && (zbits = (u32)term_val(heap_read(term_val(z)))) == 0)))
    return -1;
  while (sm100_is(c, UOP_CAST)) c = heap_read(term_val(c));
  if (!sm100_is(c, UOP_CMPEQ)) return -1;
  Term f = heap_read(term_val(c)), key = heap_read(term_val(c) + 1);
  const u64 bit = 1ull << (ax & 63);
  if (sp_deps(p, f) != bit) {
    Term tmp = f;
    f = key, key = tmp;
  }
  if (sp_deps(p, f) != bit || (sp_deps(p, key) & bit) || sp_isfloat(sp_ty(p, f)) || sp_isfloat(sp_ty(p, key)))
    return -1;
  Term rg = sp_find_range(a, ax, 0);
  if (!rg) rg = sp_find_range(f, ax, 0);
  if (!rg) return -1;
  const u32 ext = uop_range_extent(rg);
  if ((ext & KVAR_FLAG) || ext == 0 || ext > (1u << 24) || sp_slot(p, ax) >= 0) return -1;
  int ok = 1;
  for (u32 v = 0; v < ext && ok; v++) {
    const i64 fv = sp_eval_pure(f, ax, v, &ok, 0);
    ok = ok && fv == (i64)v;
  }
  if (!ok) return -1;
  const u16 k = sp_int(p, key);
  const u16 inb = sp_op(p, SM100_IOP_IAND, 0, sp_op(p, SM100_IOP_ILT, 0, sp_const_i(p, -1), k, 0, 0),
                        sp_op(p, SM100_IOP_ILT, 0, k, sp_const_i(p, ext), 0, 0), 0, 0);
  const u16 zero_i = sp_const_i(p, 0);
  const int slot = sp_new_slot(p, ax);
  sp_emit(p, SM100_IOP_SETR, 0, 0, (u16)slot, sp_op(p, SM100_IOP_SEL, 0, inb, k, zero_i, 0), 0, 0);
  const u32 memo0 = p->n_memo;
  const u64 bound0 = p->bound;
  p->bound |= bit;
  u16 r;
  if (!is_int) {
    const u16 zf = sp_const_f(p, 0.0f);
    /* 0 + a(key), as the sum's first non-zero step rounds it (a -0 becomes +0) */
    r = sp_op(p, SM100_IOP_FADD, 0, zf, sp_op(p, SM100_IOP_SEL, 0, inb, sp_float(p, a), zf, 0), 0, 0);
  } else {
    r = sp_op(p, SM100_IOP_SEL, 0, inb, sp_int(p, a), zero_i, 0);
  }
  p->n_memo = memo0;
  p->bound = bound0;
  return p->bad ? -1 : r;
}

static void sp_compile_family(Sm100Prog *p, Sm100Prog *root, u32 n_in);
static u16 sp_reduce(Sm100Prog *p, Term t);

/* the chain of same-kind REDUCEs at t: its axes, extents (static) and body */
static int sp_chain(Term t, u32 *axes, u32 *ext, u32 *n, Term *body) {
  const u32 kind = uop_reduce_kind(t);
  Term cur = t;
  *n = 0;
  while (sm100_is(cur, UOP_REDUCE) && uop_reduce_kind(cur) == kind) {
    Term src = uop_reduce_src(cur);
    for (u32 i = 0; i < uop_reduce_n_axes(cur); i++) {
      const u32 ax = uop_reduce_axis(cur, i);
      Term rg = sp_find_range(src, ax, 0);
      if (!rg || *n >= 4) return 0;
      const u32 e = uop_range_extent(rg);
      if (e & KVAR_FLAG) return 0;
      axes[*n] = ax, ext[(*n)++] = e;
    }
    *body = src;
    cur = src;
  }
  return *n > 0;
}

static int sp_new_scratch(Sm100Prog *root, u64 bytes) {
  if (root->n_scr >= SM100_MAX_SCR || root->n_in + 1 + root->n_scr >= SM100_INTERP_MAX_BUFS) return -1;
  root->scr_bytes[root->n_scr] = bytes ? bytes : 8;
  return (int)root->n_scr++;
}

/* linear index of this program's output coordinates on the axes in dmask
 * (in slot order), and the number of rows it spans (static upper bound) */
static u16 sp_row_index(Sm100Prog *p, u64 dmask, u64 *rows) {
  u16 lin = sp_const_i(p, 0);
  *rows = 1;
  for (u32 s2 = 0; s2 < p->n_glob; s2++) {
    if (!(dmask & (1ull << (p->axis_id[s2] & 63)))) continue;
    lin = sp_op(p, SM100_IOP_IMUL, 0, lin, sp_extent(p, p->glob_packed[s2]), 0, 0);
    lin = sp_op(p, SM100_IOP_IADD, 0, lin, sp_op(p, SM100_IOP_RANGE, 0, (u16)s2, 0, 0, 0), 0, 0);
    *rows *= kvar_extent_static(p->glob_packed[s2]);
  }
  return lin;
}

/* a new program of the family over the root program's output axes in dmask
 * (same axis ids, slot order, packed extents), plus the chunk axis when
 * nchunk > 0 */
static Sm100Prog *sp_child(Sm100Prog *p, u64 dmask, u32 nchunk) {
  Sm100Prog *c = (Sm100Prog *)malloc(sizeof(Sm100Prog));
  if (!c) return NULL;
  sp_compile_family(c, p->root, p->root->n_in);
  for (u32 s2 = 0; s2 < p->n_glob; s2++) {
    if (!(dmask & (1ull << (p->axis_id[s2] & 63)))) continue;
    const int k = sp_new_slot(c, p->axis_id[s2]);
    c->glob_packed[k] = p->glob_packed[s2];
    c->bound |= 1ull << (p->axis_id[s2] & 63);
  }
  if (nchunk) {
    const int k = sp_new_slot(c, SM100_AX_CHUNK);
    c->glob_packed[k] = nchunk;
    c->bound |= 1ull << SM100_AX_CHUNK;
  }
  c->n_glob = c->n_axes;
  return c;
}

static int sp_add_pre(Sm100Prog *root, Sm100Prog *c, int out_scr) {
  if (root->n_pre >= SM100_MAX_PRE || c->bad) return 0;
  root->pre[root->n_pre] = c;
  root->pre_out[root->n_pre++] = out_scr;
  return 1;
}

/* The reduce t as a load of its pre-pass result, or -1 when it stays inline. */
static int sp_prepass(Sm100Prog *p, Term t, int is_int, u32 dt) {
  Sm100Prog *root = p->root;
  if (!root || !root->allow_pre || p->bad) return -1;
  const u64 d = sp_deps(p, t);
  u64 gmask = 0;
  for (u32 s2 = 0; s2 < p->n_glob; s2++) gmask |= 1ull << (p->axis_id[s2] & 63);
  if (d & ~gmask) return -1;   /* reads a range of an enclosing loop: stays inline */
  u32 axes[4], ext[4], n;
  Term body;
  if (!sp_chain(t, axes, ext, &n, &body)) return -1;
  u64 E = 1;
  for (u32 i = 0; i < n; i++) E *= ext[i];
  /* worth it: the reduce is the same for every element of some output axis, or long */
  if (E < 64 || (d == gmask && E < 4096)) return -1;
  for (u32 i = 0; i < n; i++)
    if (axes[i] >= SM100_AX_CHUNK) return -1;
  const u32 kind = uop_reduce_kind(t);
  const u8 sdt = is_int ? (u8)DT_INT64 : (u8)DT_FP32;
  for (u32 i = 0; i < root->n_ur; i++)
    if (root->ur_t[i] == t) {
      u64 rows;
      const u16 lin = sp_row_index(p, root->ur_dmask[i], &rows);
      return sp_op(p, SM100_IOP_LOAD, sdt, (u16)(root->n_in + 1 + root->ur_scr[i]), lin, 0, 0);
    }
  if (root->n_ur >= SM100_MAX_PRE || root->n_pre + 2 > SM100_MAX_PRE) return -1;
  u32 L = 1;
  while ((u64)L * L < E) L++;
  const u32 NC = (u32)((E + L - 1) / L);
  u64 rows = 1;
  for (u32 s2 = 0; s2 < p->n_glob; s2++)
    if (d & (1ull << (p->axis_id[s2] & 63))) rows *= kvar_extent_static(p->glob_packed[s2]);
  const int s_part = sp_new_scratch(root, rows * NC * 8), s_res = sp_new_scratch(root, rows * 8);
  if (s_part < 0 || s_res < 0) return -1;
  /* P1: partial[row][c] = fold over the chunk's iterations */
  Sm100Prog *p1 = sp_child(p, d, NC);
  if (!p1) return -1;
  {
    const int cs = p1->n_glob - 1;
    u64 r1;
    const u16 lin = sp_row_index(p1, d, &r1);
    const u16 cidx = sp_op(p1, SM100_IOP_RANGE, 0, (u16)cs, 0, 0, 0);
    const u16 Lr = sp_const_i(p1, L), Er = sp_const_i(p1, (i64)E);
    sp_hoist(p1, body, 0);
    /* the accumulator and the identity the padded iterations add: two registers */
    u16 acc, ident;
    if (!is_int) {
      const float id = kind == REDUCE_MAX ? -INFINITY : kind == REDUCE_PROD ? 1.0f : 0.0f;
      acc = sp_const_f(p1, id), ident = sp_const_f(p1, id);
    } else {
      const i64 id = kind == REDUCE_PROD ? 1 : (kind == REDUCE_MAX && dtype_is_signed(dt))
                                                 ? sm100_i_wrap((int)dt, (i64)((u64)1 << (dtype_info(dt)->bits - 1)))
                                                 : 0;
      acc = sp_const_i(p1, id), ident = sp_const_i(p1, id);
    }
    const u16 base = sp_op(p1, SM100_IOP_IMUL, 0, cidx, Lr, 0, 0);
    const int js = sp_new_slot(p1, SM100_AX_STEP);
    const u32 loop_pc = sp_emit(p1, SM100_IOP_LOOP, 0, 0, (u16)js, Lr, 0, 0);
    const u32 memo0 = p1->n_memo;
    p1->bound |= 1ull << SM100_AX_STEP;
    u16 vf = sp_op(p1, SM100_IOP_IADD, 0, base, sp_op(p1, SM100_IOP_RANGE, 0, (u16)js, 0, 0, 0), 0, 0);
    const u16 valid = sp_op(p1, SM100_IOP_ILT, 0, vf, Er, 0, 0);
    for (int i = (int)n - 1; i >= 0; i--) {   /* the flat index into the chain's axes, last fastest */
      const int as = sp_new_slot(p1, axes[i]);
      const u16 er = sp_const_i(p1, ext[i]);
      sp_emit(p1, SM100_IOP_SETR, 0, 0, (u16)as, sp_op(p1, SM100_IOP_IMOD, DT_INT64, vf, er, 0, 0), 0, 0);
      vf = sp_op(p1, SM100_IOP_IDIV, DT_INT64, vf, er, 0, 0);
      p1->bound |= 1ull << (axes[i] & 63);
    }
    if (!is_int) {
      const u16 v = sp_float(p1, body);
      sp_emit(p1, SM100_IOP_ACCF, (u8)(kind == REDUCE_MAX ? 1 : kind == REDUCE_PROD ? 2 : 0), acc,
              sp_op(p1, SM100_IOP_SEL, 0, valid, v, ident, 0), 0, 0, 0);
    } else {
      const u16 v = sp_int(p1, body);
      sp_emit(p1, SM100_IOP_ACCI, (u8)dt, acc, sp_op(p1, SM100_IOP_SEL, 0, valid, v, ident, 0), 0, 0, (i32)kind);
    }
    const u32 end = sp_emit(p1, SM100_IOP_ENDLOOP, 0, 0, (u16)js, Lr, 0, (i32)loop_pc);
    if (!p1->bad) p1->code[loop_pc].imm = (i32)end;
    p1->n_memo = memo0;
    const u16 off = sp_op(p1, SM100_IOP_IADD, 0, sp_op(p1, SM100_IOP_IMUL, 0, lin, sp_const_i(p1, NC), 0, 0), cidx, 0, 0);
    sp_emit(p1, SM100_IOP_STORE, sdt, 0, 0, off, acc, !is_int);
  }
  if (p1->bad || !sp_add_pre(root, p1, s_part)) {
    free(p1);
    return -1;
  }
  /* P2: result[row] = fold over the row's partials in chunk order */
  Sm100Prog *p2 = sp_child(p, d, 0);
  if (!p2) return -1;
  {
    u64 r2;
    const u16 lin = sp_row_index(p2, d, &r2);
    const u16 base = sp_op(p2, SM100_IOP_IMUL, 0, lin, sp_const_i(p2, NC), 0, 0), NCr = sp_const_i(p2, NC);
    u16 acc;
    if (!is_int) acc = sp_const_f(p2, kind == REDUCE_MAX ? -INFINITY : kind == REDUCE_PROD ? 1.0f : 0.0f);
    else acc = sp_const_i(p2, kind == REDUCE_PROD ? 1 : (kind == REDUCE_MAX && dtype_is_signed(dt))
                                                            ? sm100_i_wrap((int)dt, (i64)((u64)1 << (dtype_info(dt)->bits - 1)))
                                                            : 0);
    const int cs = sp_new_slot(p2, SM100_AX_CHUNK);
    const u32 loop_pc = sp_emit(p2, SM100_IOP_LOOP, 0, 0, (u16)cs, NCr, 0, 0);
    const u16 v = sp_op(p2, SM100_IOP_LOAD, sdt, (u16)(root->n_in + 1 + s_part),
                        sp_op(p2, SM100_IOP_IADD, 0, base, sp_op(p2, SM100_IOP_RANGE, 0, (u16)cs, 0, 0, 0), 0, 0), 0, 0);
    if (!is_int) sp_emit(p2, SM100_IOP_ACCF, (u8)(kind == REDUCE_MAX ? 1 : kind == REDUCE_PROD ? 2 : 0), acc, v, 0, 0, 0);
    else sp_emit(p2, SM100_IOP_ACCI, (u8)dt, acc, v, 0, 0, (i32)kind);
    const u32 end = sp_emit(p2, SM100_IOP_ENDLOOP, 0, 0, (u16)cs, NCr, 0, (i32)loop_pc);
    if (!p2->bad) p2->code[loop_pc].imm = (i32)end;
    sp_emit(p2, SM100_IOP_STORE, sdt, 0, 0, lin, acc, !is_int);
  }
  if (p2->bad || !sp_add_pre(root, p2, s_res)) {
    free(p2);
    root->n_pre--;   /* P1 without its P2 is useless; it is freed with the family */
    free(p1);
    return -1;
  }
  root->ur_t[root->n_ur] = t, root->ur_scr[root->n_ur] = (u32)s_res, root->ur_dt[root->n_ur] = sdt;
  root->ur_dmask[root->n_ur++] = d;
  u64 rows3;
  const u16 lin = sp_row_index(p, d, &rows3);
  return sp_op(p, SM100_IOP_LOAD, sdt, (u16)(root->n_in + 1 + (u32)s_res), lin, 0, 0);
}

static u16 sp_reduce(Sm100Prog *p, Term t) {
  const u32 kind = uop_reduce_kind(t);
  u32 dt = DT_FP32;
  (void)term_dtype_in(t, 0, &dt);
  const int is_int = dtype_is_bool(dt) || dtype_is_int(dt);
  if (!is_int && dt == DT_FP64) sp_fail(p, "f64 reduce");
  if (!is_int || !dtype_is_bool(dt)) {
    const int g = sp_onehot(p, t, is_int);
    if (g >= 0) return (u16)g;
  }
  {
    const int h = sp_prepass(p, t, is_int, dt);
    if (h >= 0) return (u16)h;
  }
  /* a chain of same-kind REDUCEs is one loop nest with one accumulator, as
   * the walker folds it (uop_walk.c uwalk_run_reduce) */
  u32 axes[SM100_INTERP_MAX_AXES], n = 0;
  u16 ext[SM100_INTERP_MAX_AXES];
  Term cur = t, body = t;
  while (sm100_is(cur, UOP_REDUCE) && uop_reduce_kind(cur) == kind && !p->bad) {
    Term src = uop_reduce_src(cur);
    for (u32 i = 0; i < uop_reduce_n_axes(cur); i++) {
      u32 ax = uop_reduce_axis(cur, i);
      Term rg = sp_find_range(src, ax, 0);
      if (!rg) {
        sp_fail(p, "reduce axis %u has no range", ax);
        break;
      }
      if (n >= SM100_INTERP_MAX_AXES || sp_slot(p, ax) >= 0) {
        sp_fail(p, "reduce axis %u reused", ax);
        break;
      }
      axes[n] = ax;
      ext[n++] = sp_extent(p, (u32)term_val(heap_read(term_val(rg) + 2)));
    }
    body = src;
    cur = src;
  }
  if (p->bad) return 0;
  /* loop-invariant parts of the body first */
  sp_hoist(p, body, 0);
  u16 acc;
  if (!is_int) {
    acc = sp_const_f(p, kind == REDUCE_MAX ? -INFINITY : kind == REDUCE_PROD ? 1.0f : 0.0f);
  } else {
    i64 id = kind == REDUCE_PROD ? 1 : 0;
    if (kind == REDUCE_MAX && dtype_is_signed(dt))
      id = sm100_i_wrap((int)dt, (i64)((u64)1 << (dtype_info(dt)->bits - 1)));
    acc = sp_const_i(p, id);
  }
  const u32 memo0 = p->n_memo;
  const u64 bound0 = p->bound;
  u32 loop_pc[SM100_INTERP_MAX_AXES];
  int slot[SM100_INTERP_MAX_AXES];
  for (u32 i = 0; i < n; i++) {
    slot[i] = sp_new_slot(p, axes[i]);
    p->bound |= 1ull << (axes[i] & 63);
    loop_pc[i] = sp_emit(p, SM100_IOP_LOOP, 0, 0, (u16)slot[i], ext[i], 0, 0);
  }
  if (!is_int) {
    u16 v = sp_float(p, body);
    sp_emit(p, SM100_IOP_ACCF, (u8)(kind == REDUCE_MAX ? 1 : kind == REDUCE_PROD ? 2 : 0), acc, v, 0, 0, 0);
  } else {
    if (sp_isfloat(sp_ty(p, body))) sp_fail(p, "int reduce of a float body");
    u16 v = sp_int(p, body);
    sp_emit(p, SM100_IOP_ACCI, (u8)dt, acc, v, 0, 0, (i32)kind);
  }
  for (u32 i = n; i-- > 0;) {
    u32 end = sp_emit(p, SM100_IOP_ENDLOOP, 0, 0, (u16)slot[i], ext[i], 0, (i32)loop_pc[i]);
    if (!p->bad) p->code[loop_pc[i]].imm = (i32)end;
  }
  /* values computed inside the loops are dead after them; the slots stay
   * allocated (a later reduce over the same axis id is refused above) */
  p->n_memo = memo0;
  p->bound = bound0;
  return acc;
}

/* emit the maximal subtrees of t that only read ranges open now */
static void sp_hoist(Sm100Prog *p, Term t, int depth) {
  if (p->bad || term_tag(t) != TAG_UOP || depth > 64) return;
  u32 op = term_ext(t);
  if (op == UOP_CONST || op == UOP_RANGE || op == UOP_DEFINE_VAR || op == UOP_INVALID || op == UOP_BUFFER) return;
  u64 d = sp_deps(p, t);
  if ((d & ~p->bound) == 0) {
    (void)sp_val(p, t);
    return;
  }
  u64 loc = term_val(t);
  int n = (op == UOP_REDUCE || op == UOP_CAST || op == UOP_BITCAST || op == UOP_OPT) ? 1 : sm100_arity(op);
  for (int i = 0; i < n; i++) {
    if (op == UOP_INDEX_E && i == 0) continue;
    sp_hoist(p, heap_read(loc + (u64)i), depth + 1);
  }
}

/* the value of t in its C type (float -> f32 register, int -> int64) */
static u16 sp_val(Sm100Prog *p, Term t) {
  if (p->bad) return 0;
  if (term_tag(t) == TAG_NUM) return sp_const_i(p, (i64)(u32)term_val(t));
  if (term_tag(t) != TAG_UOP) {
    sp_fail(p, "term tag %u", (u32)term_tag(t));
    return 0;
  }
  int hit;
  u16 r = sp_memo_get(p, t, &hit);
  if (hit) return r;
  const u32 op = term_ext(t);
  const u64 loc = term_val(t);
  const u32 ty = sp_ty(p, t);
  switch (op) {
    case UOP_CONST: {
      const u32 dt = term_ext(heap_read(loc)), bits = (u32)term_val(heap_read(loc));
      if (sp_isfloat(dt)) {
        r = sp_op(p, SM100_IOP_CONST, 2, 0, 0, 0, (i32)bits);
      } else {
        i64 v = dtype_kind(dt) == DK_UINT ? sm100_i_wrap((int)dt, (i64)bits) : (i64)(i32)bits;
        r = sp_const_i(p, v);
      }
      break;
    }
    case UOP_RANGE: {
      int s = sp_slot(p, uop_range_axis_id(t));
      if (s < 0 || !(p->bound & (1ull << (uop_range_axis_id(t) & 63)))) {
        sp_fail(p, "range r%u read outside its loop", uop_range_axis_id(t));
        return 0;
      }
      r = sp_op(p, SM100_IOP_RANGE, 0, (u16)s, 0, 0, 0);
      break;
    }
    case UOP_DEFINE_VAR: {
      if (p->n_vars >= SM100_INTERP_MAX_VARS) {
        sp_fail(p, "too many runtime values");
        return 0;
      }
      p->var_packed[p->n_vars] = uop_define_var_extent(t);
      r = sp_op(p, SM100_IOP_VAR, 0, (u16)p->n_vars++, 0, 0, 0);
      break;
    }
    case UOP_INVALID: r = sp_const_i(p, 0); break;
    case UOP_OPT: return sp_val(p, heap_read(loc));
    case UOP_INDEX_E: {
      Term buf = heap_read(loc);
      if (!sm100_is(buf, UOP_BUFFER) || uop_buffer_scope(buf) != UOP_SCOPE_GLOBAL) {
        sp_fail(p, "INDEX of a non-global buffer");
        return 0;
      }
      u32 bdt = uop_buffer_dtype(buf);
      if (bdt == DT_FP8E4M3 || bdt == DT_FP8E5M2 || bdt == DT_INT4 || bdt == DT_UINT4) {
        sp_fail(p, "load of dtype %u", bdt);
        return 0;
      }
      u16 off = sp_int(p, heap_read(loc + 1));
      r = sp_op(p, SM100_IOP_LOAD, (u8)bdt, (u16)uop_buffer_inst_get(buf), off, 0, 0);
      break;
    }
    case UOP_ADD: case UOP_MUL: {
      Term a = heap_read(loc), b = heap_read(loc + 1);
      if (sp_isfloat(ty)) r = sp_op(p, op == UOP_ADD ? SM100_IOP_FADD : SM100_IOP_FMUL, 0, sp_float(p, a), sp_float(p, b), 0, 0);
      else r = sp_op(p, op == UOP_ADD ? SM100_IOP_IADD : SM100_IOP_IMUL, 0, sp_int(p, a), sp_int(p, b), 0, 0);
      break;
    }
    case UOP_NEG:
      if (sp_isfloat(ty)) r = sp_op(p, SM100_IOP_FNEG, 0, sp_float(p, heap_read(loc)), 0, 0, 0);
      else r = sp_op(p, SM100_IOP_INEG, 0, sp_int(p, heap_read(loc)), 0, 0, 0);
      break;
    case UOP_RECIP: case UOP_EXP2: case UOP_LOG2: case UOP_SQRT: case UOP_SIN: {
      if (ty == DT_FP64) {
        sp_fail(p, "f64 %s", sm100_op_name(op));
        return 0;
      }
      u8 o = op == UOP_RECIP ? SM100_IOP_FRECIP : op == UOP_EXP2 ? SM100_IOP_FEXP2 : op == UOP_LOG2 ? SM100_IOP_FLOG2
             : op == UOP_SQRT ? SM100_IOP_FSQRT : SM100_IOP_FSIN;
      r = sp_op(p, o, 0, sp_float(p, heap_read(loc)), 0, 0, 0);
      break;
    }
    case UOP_CMPLT: case UOP_CMPEQ: {
      Term a = heap_read(loc), b = heap_read(loc + 1);
      const u32 da = sp_ty(p, a), db = sp_ty(p, b);
      if (sp_isfloat(da) || sp_isfloat(db))
        r = sp_op(p, op == UOP_CMPLT ? SM100_IOP_FLT : SM100_IOP_FEQ, 0, sp_float(p, a), sp_float(p, b), 0, 0);
      else if (op == UOP_CMPEQ)
        r = sp_op(p, SM100_IOP_IEQ, 0, sp_int(p, a), sp_int(p, b), 0, 0);
      else
        r = sp_op(p, (da == DT_UINT64 || db == DT_UINT64) ? SM100_IOP_ULT : SM100_IOP_ILT, 0, sp_int(p, a), sp_int(p, b), 0, 0);
      break;
    }
    case UOP_IADD: case UOP_ISUB: case UOP_IMUL: case UOP_ILT: case UOP_IAND: case UOP_IOR: case UOP_IXOR: {
      u8 o = op == UOP_IADD ? SM100_IOP_IADD : op == UOP_ISUB ? SM100_IOP_ISUB : op == UOP_IMUL ? SM100_IOP_IMUL
             : op == UOP_ILT ? SM100_IOP_ILT : op == UOP_IAND ? SM100_IOP_IAND : op == UOP_IOR ? SM100_IOP_IOR : SM100_IOP_IXOR;
      r = sp_op(p, o, 0, sp_int(p, heap_read(loc)), sp_int(p, heap_read(loc + 1)), 0, 0);
      break;
    }
    case UOP_IDIV: case UOP_IMOD: case UOP_ISHL: case UOP_ISHR: {
      u32 dt = DT_FP32;
      (void)term_dtype_in(t, 0, &dt);
      if (op == UOP_IDIV || op == UOP_IMOD) {
        if (!dtype_is_int(dt) || dtype_is_bool(dt)) dt = DT_INT64;
      } else if (!dtype_is_int(dt) || dt == DT_INT32 || dtype_is_bool(dt)) {
        dt = DT_INT32;
      }
      u8 o = op == UOP_IDIV ? SM100_IOP_IDIV : op == UOP_IMOD ? SM100_IOP_IMOD : op == UOP_ISHL ? SM100_IOP_ISHL : SM100_IOP_ISHR;
      r = sp_op(p, o, (u8)dt, sp_int(p, heap_read(loc)), sp_int(p, heap_read(loc + 1)), 0, 0);
      break;
    }
    case UOP_IWHERE: {
      Term c = heap_read(loc), a = heap_read(loc + 1), b = heap_read(loc + 2);
      u16 cond;
      int swap = 0;
      if (sp_isfloat(sp_ty(p, c))) {
        cond = sp_op(p, SM100_IOP_FEQ, 0, sp_float(p, c), sp_const_f(p, 0.0f), 0, 0);
        swap = 1; /* (c == 0) selects the else branch */
      } else {
        cond = sp_int(p, c);
      }
      u16 ra, rb;
      if (sp_isfloat(ty)) ra = sp_float(p, a), rb = sp_float(p, b);
      else ra = sp_int(p, a), rb = sp_int(p, b);
      r = sp_op(p, SM100_IOP_SEL, 0, cond, swap ? rb : ra, swap ? ra : rb, 0);
      break;
    }
    case UOP_CAST: {
      Term src = heap_read(loc);
      const u32 dst = (u32)term_val(heap_read(loc + 1));
      if (sp_isfloat(dst)) {
        if (dst == DT_FP64 || dst == DT_FP8E4M3 || dst == DT_FP8E5M2) {
          sp_fail(p, "cast to dtype %u", dst);
          return 0;
        }
        r = sp_float(p, src);
        if (dst == DT_FP16 || dst == DT_BF16) r = sp_op(p, SM100_IOP_NARROW, (u8)dst, r, 0, 0, 0);
      } else {
        const u32 sdt = sp_ty(p, src);
        if (sp_isfloat(sdt)) {
          r = sp_op(p, SM100_IOP_F2I, (u8)dst, sp_val(p, src), 0, 0, 0);
        } else {
          r = sp_op(p, SM100_IOP_WRAP, (u8)sdt, sp_val(p, src), 0, 0, 0);
          r = sp_op(p, SM100_IOP_WRAP, (u8)dst, r, 0, 0, 0);
        }
      }
      break;
    }
    case UOP_BITCAST: {
      Term src = heap_read(loc);
      const u32 dst = (u32)term_val(heap_read(loc + 1)), sdt = sp_ty(p, src);
      if (dst == DT_FP32 && !sp_isfloat(sdt)) {
        r = sp_op(p, SM100_IOP_WRAP, DT_UINT32, sp_val(p, src), 0, 0, 0);
      } else if ((dst == DT_INT32 || dst == DT_UINT32) && sdt == DT_FP32) {
        r = sp_op(p, SM100_IOP_WRAP, (u8)dst, sp_val(p, src), 0, 0, 0);
      } else if ((dst == DT_INT32 || dst == DT_UINT32) && !sp_isfloat(sdt)) {
        r = sp_val(p, src);
      } else {
        sp_fail(p, "bitcast %u -> %u", sdt, dst);
        return 0;
      }
      break;
    }
    case UOP_THREEFRY:
      r = sp_op(p, SM100_IOP_THREEFRY, 0, sp_int(p, heap_read(loc)), sp_int(p, heap_read(loc + 1)), 0, 0);
      break;
    case UOP_REDUCE: r = sp_reduce(p, t); break;
    default:
      sp_fail(p, "op %s", sm100_op_name(op));
      return 0;
  }
  if (p->bad) return 0;
  if (p->n_memo < SM100_MEMO_CAP) p->memo_t[p->n_memo] = t, p->memo_r[p->n_memo++] = r;
  return r;
}

static int sp_collect_glob(Sm100Prog *p, Term t, int depth) {
  if (term_tag(t) != TAG_UOP || depth > 64) return 0;
  u32 op = term_ext(t);
  if (op == UOP_RANGE) {
    u32 ax = uop_range_axis_id(t);
    if (ax >= 64) {
      sp_fail(p, "axis id %u", ax);
      return 0;
    }
    if (sp_slot(p, ax) < 0) {
      /* keep the slots sorted by axis id: the highest id is the fastest */
      int s = sp_new_slot(p, ax);
      while (s > 0 && p->axis_id[s - 1] > ax) {
        p->axis_id[s] = p->axis_id[s - 1];
        p->glob_packed[s] = p->glob_packed[s - 1];
        s--;
      }
      p->axis_id[s] = ax;
      p->glob_packed[s] = (u32)term_val(heap_read(term_val(t) + 2));
      p->bound |= 1ull << ax;
    }
    return 1;
  }
  if (op == UOP_REDUCE) {
    sp_fail(p, "reduce in an address");
    return 0;
  }
  u64 loc = term_val(t);
  int n = (op == UOP_CAST || op == UOP_OPT) ? 1 : sm100_arity(op);
  for (int i = 0; i < n; i++) sp_collect_glob(p, heap_read(loc + (u64)i), depth + 1);
  return 1;
}

/* Program for STORE(out, addr, value) over the ranges of addr; out is
 * buffer slot out_slot (dtype out_dt).  With `lin_glob` the address is not
 * taken from the DAG: the output is the dense row-major block over the given
 * axes (used for a linear's A-side scratch). */
/* an empty program of root's family (root == p: a family of its own) */
static void sp_compile_family(Sm100Prog *p, Sm100Prog *root, u32 n_in) {
  memset(p, 0, sizeof *p);
  p->root = root ? root : p;
  p->n_in = n_in;
}

static void sp_free_family(Sm100Prog *p) {
  if (!p) return;
  for (u32 i = 0; i < p->n_pre; i++) free(p->pre[i]);
  free(p);
}

static void sp_compile(Sm100Prog *p, Term addr, Term value, u32 out_slot, u32 out_dt, const Term *lin_glob,
                       u32 n_lin, u32 n_in, int allow_pre) {
  sp_compile_family(p, NULL, n_in);
  p->allow_pre = allow_pre;
  if (lin_glob) {
    for (u32 i = 0; i < n_lin; i++) {
      int s = sp_new_slot(p, uop_range_axis_id(lin_glob[i]));
      p->glob_packed[s] = (u32)term_val(heap_read(term_val(lin_glob[i]) + 2));
      p->bound |= 1ull << (uop_range_axis_id(lin_glob[i]) & 63);
    }
  } else {
    sp_collect_glob(p, addr, 0);
  }
  p->n_glob = p->n_axes;
  if (p->bad) return;
  u16 off;
  if (lin_glob) {
    off = sp_const_i(p, 0);
    for (u32 i = 0; i < n_lin; i++) {
      u16 e = sp_extent(p, p->glob_packed[i]);
      off = sp_op(p, SM100_IOP_IMUL, 0, off, e, 0, 0);
      off = sp_op(p, SM100_IOP_IADD, 0, off, sp_op(p, SM100_IOP_RANGE, 0, (u16)i, 0, 0, 0), 0, 0);
    }
  } else {
    off = sp_int(p, addr);
  }
  u16 v;
  if (sp_isfloat(out_dt)) {
    v = sp_float(p, value);
  } else if (sp_isfloat(sp_ty(p, value))) {
    v = sp_op(p, SM100_IOP_F2I, (u8)out_dt, sp_val(p, value), 0, 0, 0);
  } else {
    v = sp_int(p, value);
  }
  sp_emit(p, SM100_IOP_STORE, (u8)out_dt, 0, (u16)out_slot, off, v, sp_isfloat(out_dt));
}

/* ---- plans --------------------------------------------------------------- */

enum { SM100_R_NONE = 0, SM100_R_LINEAR = 1, SM100_R_INTERP = 2 };
static const char *const SM100_ROUTE_NAMES[] = {"none", "linear", "interp"};

typedef struct {
  Term root; /* cache key */
  int kind;
  /* LINEAR */
  u32 M, N, K, w_in;
  int x_in;         /* A side is this input read as a dense [M, K] block, or -1: the prologue */
  Sm100Prog *pro;   /* the A-side program (writes the [M, K] scratch, slot 0) */
  /* INTERP */
  Sm100Prog *prog;
  char why[160];
} Sm100Plan;

#define SM100_PLAN_CAP 4096
static Sm100Plan SM100_PLANS[SM100_PLAN_CAP];
static u32 SM100_N_PLANS;

static void sm100_plan_free(Sm100Plan *pl) {
  sp_free_family(pl->pro);
  sp_free_family(pl->prog);
  pl->pro = pl->prog = NULL;
}

/* IADD(IMUL(r_n, K), r_k) in either order, or r_k alone when N == 1 */
static int sm100_match_nk(Term addr, u32 K, Term *rn, Term *rk) {
  if (!sm100_is(addr, UOP_IADD)) return 0;
  for (int o = 0; o < 2; o++) {
    Term mul = heap_read(term_val(addr) + (u64)o), k = heap_read(term_val(addr) + (u64)(1 - o));
    if (!sm100_is(k, UOP_RANGE) || !sm100_is(mul, UOP_IMUL)) continue;
    for (int q = 0; q < 2; q++) {
      Term r = heap_read(term_val(mul) + (u64)q), c = heap_read(term_val(mul) + (u64)(1 - q));
      if (!sm100_is(r, UOP_RANGE) || !sm100_is(c, UOP_CONST)) continue;
      if ((u32)term_val(heap_read(term_val(c))) != K) continue;
      *rn = r, *rk = k;
      return 1;
    }
  }
  return 0;
}

static int sm100_const_u32(Term t, u32 *v) {
  if (!sm100_is(t, UOP_CONST)) return 0;
  *v = (u32)term_val(heap_read(term_val(t)));
  return 1;
}

/* A linear with any A side: STORE(out, m*N + n | n, REDUCE_SUM(MUL(P, W[n*K + k]), k)) */
static int sm100_plan_linear(struct KernelEntry *ke, Term root, Sm100Plan *pl) {
  Term addr = heap_read(term_val(root) + 1), value = heap_read(term_val(root) + 2);
  if (!sm100_is(value, UOP_REDUCE) || uop_reduce_kind(value) != REDUCE_SUM || uop_reduce_n_axes(value) != 1)
    return 0;
  Term mul = uop_reduce_src(value);
  if (!sm100_is(mul, UOP_MUL)) return 0;
  const u32 kax = uop_reduce_axis(value, 0);
  for (int o = 0; o < 2; o++) {
    Term w = heap_read(term_val(mul) + (u64)o), pa = heap_read(term_val(mul) + (u64)(1 - o));
    if (!sm100_is(w, UOP_INDEX_E)) continue;
    Term wb = heap_read(term_val(w));
    if (!sm100_is(wb, UOP_BUFFER) || uop_buffer_dtype(wb) != DT_FP32 || uop_buffer_inst_get(wb) == 0) continue;
    Term kr = sp_find_range(pa, kax, 0);
    if (!kr) continue;
    const u32 K = uop_range_extent(kr);
    if (K & KVAR_FLAG) continue;
    Term rn, rk;
    if (!sm100_match_nk(heap_read(term_val(w) + 1), K, &rn, &rk) || uop_range_axis_id(rk) != kax) continue;
    const u32 N = uop_range_extent(rn);
    if (N & KVAR_FLAG) continue;
    /* output address: n, or m*N + n (m another range) */
    Term rm = 0;
    if (sm100_is(addr, UOP_RANGE)) {
      if (addr != rn) continue;
    } else {
      Term r2, r1;
      if (!sm100_match_nk(addr, N, &r2, &r1) || r1 != rn) continue;
      rm = r2;
    }
    const u32 M = rm ? uop_range_extent(rm) : 1;
    if (M & KVAR_FLAG) continue;
    Sm100Prog scratch;
    (void)scratch;
    /* the A side must not read n */
    Sm100Prog *dp = (Sm100Prog *)calloc(1, sizeof *dp);
    if (!dp) return 0;
    if (sp_deps(dp, pa) & (1ull << (uop_range_axis_id(rn) & 63))) {
      free(dp);
      continue;
    }
    free(dp);
    pl->M = M, pl->N = N, pl->K = K, pl->w_in = uop_buffer_inst_get(wb) - 1;
    /* plain input A: INDEX(B, m*K + k | k) */
    pl->x_in = -1;
    if (sm100_is(pa, UOP_INDEX_E)) {
      Term ab = heap_read(term_val(pa)), aa = heap_read(term_val(pa) + 1);
      Term x1, x2;
      if (sm100_is(ab, UOP_BUFFER) && uop_buffer_dtype(ab) == DT_FP32 && uop_buffer_inst_get(ab) > 0 &&
          ((M == 1 && aa == rk) || (rm && sm100_match_nk(aa, K, &x1, &x2) && x1 == rm && x2 == rk)))
        pl->x_in = (int)uop_buffer_inst_get(ab) - 1;
    }
    if (pl->x_in < 0) {
      Term glob[2];
      u32 ng = 0;
      if (rm) glob[ng++] = rm;
      glob[ng++] = rk;
      pl->pro = (Sm100Prog *)malloc(sizeof(Sm100Prog));
      if (!pl->pro) return 0;
      sp_compile(pl->pro, 0, pa, 0, DT_FP32, glob, ng, ke->n_inputs, sm100_env_on("THVM_SM100_PREPASS", 1));
      if (pl->pro->bad) {
        snprintf(pl->why, sizeof pl->why, "linear A side: %s", pl->pro->why);
        sp_free_family(pl->pro);
        pl->pro = NULL;
        return 0;
      }
    }
    (void)ke;
    return 1;
  }
  return 0;
}

static Sm100Plan *sm100_ref_plan(struct KernelEntry *ke) {
  Term root = ke->cached_lift_init_root ? ke->cached_lift_init_root : ke->cached_lift.store_root;
  for (u32 i = 0; i < SM100_N_PLANS; i++)
    if (SM100_PLANS[i].root == root && root) return &SM100_PLANS[i];
  Sm100Plan *pl;
  if (SM100_N_PLANS < SM100_PLAN_CAP) {
    pl = &SM100_PLANS[SM100_N_PLANS++];
  } else {
    static u32 evict;
    pl = &SM100_PLANS[evict++ % SM100_PLAN_CAP];
    sm100_plan_free(pl);
  }
  memset(pl, 0, sizeof *pl);
  pl->root = root;
  if (root == 0) {
    snprintf(pl->why, sizeof pl->why, "no lifted DAG");
    return pl;
  }
  if (!sm100_is(root, UOP_STORE)) {
    snprintf(pl->why, sizeof pl->why, "root is %s", sm100_op_name(term_ext(root)));
    return pl;
  }
  Term out = heap_read(term_val(root));
  if (!sm100_is(out, UOP_BUFFER) || uop_buffer_inst_get(out) != 0) {
    snprintf(pl->why, sizeof pl->why, "store into a non-output buffer");
    return pl;
  }
  if (ke->n_inputs + 1 > SM100_INTERP_MAX_BUFS) {
    snprintf(pl->why, sizeof pl->why, "%u inputs", ke->n_inputs);
    return pl;
  }
  if (uop_buffer_dtype(out) == DT_FP32 && sm100_plan_linear(ke, root, pl)) {
    pl->kind = SM100_R_LINEAR;
    return pl;
  }
  Sm100Prog *pg = (Sm100Prog *)malloc(sizeof(Sm100Prog));
  if (!pg) {
    snprintf(pl->why, sizeof pl->why, "out of memory");
    return pl;
  }
  const u32 odt = uop_buffer_dtype(out);
  if (odt == DT_FP8E4M3 || odt == DT_FP8E5M2 || odt == DT_INT4 || odt == DT_UINT4) {
    snprintf(pl->why, sizeof pl->why, "store of dtype %u", odt);
    free(pg);
    return pl;
  }
  sp_compile(pg, heap_read(term_val(root) + 1), heap_read(term_val(root) + 2), 0, odt, NULL, 0, ke->n_inputs,
             sm100_env_on("THVM_SM100_PREPASS", 1));
  if (pg->bad) {
    snprintf(pl->why, sizeof pl->why, "%s", pg->why);
    sp_free_family(pg);
    return pl;
  }
  pl->prog = pg;
  pl->kind = SM100_R_INTERP;
  return pl;
}

/* runtime extents / values of a program */
static void sm100_prog_runtime(const Sm100Prog *pg, int64_t *glob_ext, int64_t *vars) {
  for (u32 i = 0; i < pg->n_glob; i++) glob_ext[i] = kvar_extent_runtime(pg->glob_packed[i]);
  for (u32 i = 0; i < pg->n_vars; i++) vars[i] = kvar_extent_runtime(pg->var_packed[i]);
}

/* ---- counters and the dispatch log ------------------------------------------ */

static u64 SM100_N_DISPATCH, SM100_N_LINEAR, SM100_N_INTERP, SM100_N_DECLINED, SM100_N_CHECKED, SM100_N_MISMATCH,
    SM100_N_EXACT;

static void sm100_log(struct KernelEntry *ke, const Sm100Plan *pl) {
  FILE *fp = sm100_log_fp();
  if (!fp) return;
  fprintf(fp, "kid=%u n_in=%u out=%u ", (u32)(ke - KERNELS), ke->n_inputs, ke->output_numel);
  if (pl->kind == SM100_R_LINEAR)
    fprintf(fp, "ROUTE linear M=%u N=%u K=%u w=%u %s", pl->M, pl->N, pl->K, pl->w_in,
            pl->x_in >= 0 ? "plain A" : "A on the interpreter");
  else if (pl->kind == SM100_R_INTERP)
    fprintf(fp, "ROUTE interp %u insns %u regs", pl->prog->n_code, pl->prog->n_regs);
  else
    fprintf(fp, "decline: %s", pl->why);
  if (sm100_env_on("THVM_SM100_DUMP", 0) && pl->root) {
    fputs("\n    ", fp);
    sm100_dump(fp, pl->root, 0);
  }
  if (sm100_env_on("THVM_SM100_DUMP_PROG", 0)) {   /* the register programs, one instruction a line */
    const Sm100Prog *root = pl->kind == SM100_R_INTERP ? pl->prog : pl->pro;
    for (u32 k = 0; root && k <= root->n_pre; k++) {
      const Sm100Prog *pg = k < root->n_pre ? root->pre[k] : root;
      fprintf(fp, "\n   program %u%s: out scratch %d, %u glob axes", k, k < root->n_pre ? " (pre-pass)" : "",
              k < root->n_pre ? root->pre_out[k] : -1, pg->n_glob);
      for (u32 i = 0; i < pg->n_code; i++) {
        const Sm100Insn *in = &pg->code[i];
        fprintf(fp, "\n    %3u: op %2u dt %2u r%-3u a %-3u b %-3u c %-3u imm %d", i, in->op, in->dt, in->dst, in->a,
                in->b, in->c, in->imm);
      }
    }
  }
  fputc('\n', fp);
  fflush(fp);
}

/* dispatches, linear routes, interpreter routes, declined, checked, mismatched, exact */
EXPORT void py_sm100_ref_stats(uint64_t *out7) {
  out7[0] = SM100_N_DISPATCH, out7[1] = SM100_N_LINEAR, out7[2] = SM100_N_INTERP, out7[3] = SM100_N_DECLINED;
  out7[4] = SM100_N_CHECKED, out7[5] = SM100_N_MISMATCH, out7[6] = SM100_N_EXACT;
}

#ifndef THVM_HAS_CUDA
/* ---- the CPU checker ---------------------------------------------------------- */

static int (*SM100_CPU_DISPATCH)(struct KernelEntry *, u32 *, u32);

static void *sm100_cpu_copy(u32 id, u64 *nbytes) {
  u64 n = CPU_BACKEND.buf_nbytes ? CPU_BACKEND.buf_nbytes(id) : 0;
  void *p = calloc(1, n + 16);
  if (p && n && CPU_BACKEND.buf_read(id, p, n) != 0) {
    free(p);
    return NULL;
  }
  *nbytes = n;
  return p;
}

/* runs a program over host buffers, every output element */
static void sm100_cpu_run(const Sm100Prog *pg, void **bufs, const int64_t *bytes) {
  int64_t ge[SM100_INTERP_MAX_AXES], vars[SM100_INTERP_MAX_VARS], r[SM100_INTERP_MAX_REGS], idx[SM100_INTERP_MAX_AXES];
  sm100_prog_runtime(pg, ge, vars);
  int64_t total = 1;
  for (u32 i = 0; i < pg->n_glob; i++) total *= ge[i];
  for (int64_t t = 0; t < total; t++) {
    int64_t rest = t;
    for (int d = (int)pg->n_glob - 1; d >= 0; d--) idx[d] = rest % ge[d], rest /= ge[d];
    (void)sm100_interp_exec(pg->code, pg->n_code, r, idx, bufs, bytes, vars);
  }
}

/* a program and its pre-passes over host buffers (slots 0..n_in given; the
 * family's scratch in fresh host blocks for this run) */
static int sm100_cpu_run_family(const Sm100Prog *pg, void **bufs, int64_t *bytes, u32 n_in) {
  void *scr[SM100_MAX_SCR] = {0};
  int ok = 1;
  for (u32 j = 0; j < pg->n_scr && ok; j++) {
    scr[j] = calloc(1, pg->scr_bytes[j] + 16);
    ok = scr[j] != NULL;
    bufs[n_in + 1 + j] = scr[j];
    bytes[n_in + 1 + j] = (int64_t)pg->scr_bytes[j];
  }
  if (ok) {
    void *out0 = bufs[0];
    const int64_t ob0 = bytes[0];
    for (u32 i = 0; i < pg->n_pre; i++) {
      bufs[0] = scr[pg->pre_out[i]];
      bytes[0] = (int64_t)pg->scr_bytes[pg->pre_out[i]];
      sm100_cpu_run(pg->pre[i], bufs, bytes);
    }
    bufs[0] = out0;
    bytes[0] = ob0;
    sm100_cpu_run(pg, bufs, bytes);
  }
  for (u32 j = 0; j < pg->n_scr; j++) free(scr[j]);
  return ok;
}

static int sm100_cpu_check(struct KernelEntry *ke, const Sm100Plan *pl, u32 *in, u32 out, int *exact) {
  const u32 n_in = ke->n_inputs;
  void *bufs[SM100_INTERP_MAX_BUFS] = {0};
  u64 nb[SM100_INTERP_MAX_BUFS] = {0};
  int64_t bytes[SM100_INTERP_MAX_BUFS] = {0};
  int ok = 1;
  *exact = 0;
  for (u32 i = 0; i < n_in && ok; i++) ok = (bufs[1 + i] = sm100_cpu_copy(in[i], &nb[1 + i])) != NULL;
  void *ref = ok ? sm100_cpu_copy(out, &nb[0]) : NULL;
  if (!ref) ok = 0;
  if (ok) {
    bufs[0] = calloc(1, nb[0] + 16);
    /* the output may also be read (an in-place assign): start from its old
     * contents, which the CPU backend's run has already overwritten, so only
     * write-only outputs are comparable; read-modify-write kernels compare
     * the elements they store. */
    memcpy(bufs[0], ref, nb[0]);
    for (u32 i = 0; i <= n_in; i++) bytes[i] = (int64_t)nb[i];
    if (pl->kind == SM100_R_INTERP) {
      sm100_cpu_run_family(pl->prog, bufs, bytes, n_in);
    } else {
      float *x = pl->x_in >= 0 ? (float *)bufs[1 + pl->x_in] : (float *)calloc((size_t)pl->M * pl->K + 4, 4);
      if (pl->x_in < 0) {
        void *sb[SM100_INTERP_MAX_BUFS];
        int64_t sbytes[SM100_INTERP_MAX_BUFS];
        memcpy(sb, bufs, sizeof sb);
        memcpy(sbytes, bytes, sizeof sbytes);
        sb[0] = x;
        sbytes[0] = (int64_t)pl->M * pl->K * 4;
        sm100_cpu_run_family(pl->pro, sb, sbytes, n_in);
      }
      const float *w = (const float *)bufs[1 + pl->w_in];
      float *y = (float *)bufs[0];
      for (u32 m = 0; m < pl->M; m++)
        for (u32 n = 0; n < pl->N; n++) {
          double acc = 0;
          for (u32 k = 0; k < pl->K; k++) acc += (double)x[(u64)m * pl->K + k] * w[(u64)n * pl->K + k];
          y[(u64)m * pl->N + n] = (float)acc;
        }
      if (pl->x_in < 0) free(x);
    }
    const u64 n_el = nb[0] / 4;
    const int is_f32 = ke->output_dtype == DT_FP32;
    u64 bad = 0, diff = 0;
    for (u64 i = 0; i < n_el; i++) {
      u32 a, b;
      memcpy(&a, (char *)bufs[0] + 4 * i, 4);
      memcpy(&b, (char *)ref + 4 * i, 4);
      if (a == b) continue;
      diff++;
      if (is_f32) {
        float fa, fb;
        memcpy(&fa, &a, 4), memcpy(&fb, &b, 4);
        if (fa != fa && fb != fb) continue;
        if (fabs((double)fa - fb) <= 1e-4 * (fabs((double)fb) + 1e-2)) continue;
      }
      if (bad++ == 0) {
        FILE *fp = sm100_log_fp();
        if (fp) fprintf(fp, "MISMATCH kid=%u elem=%llu ours=%08x ref=%08x\n", (u32)(ke - KERNELS), (unsigned long long)i, a, b);
      }
    }
    ok = bad == 0;
    *exact = diff == 0;
    free(bufs[0]);
  }
  free(ref);
  for (u32 i = 0; i < n_in; i++) free(bufs[1 + i]);
  return ok;
}

static int sm100_ref_dispatch(struct KernelEntry *ke, u32 *in_buf_ids, u32 out_buf_id) {
  SM100_N_DISPATCH++;
  Sm100Plan *pl = sm100_ref_plan(ke);
  sm100_log(ke, pl);
  int rc = SM100_CPU_DISPATCH(ke, in_buf_ids, out_buf_id);
  if (pl->kind == SM100_R_LINEAR) SM100_N_LINEAR++;
  else if (pl->kind == SM100_R_INTERP) SM100_N_INTERP++;
  else SM100_N_DECLINED++;
  if (rc == 0 && pl->kind) {
    int exact;
    SM100_N_CHECKED++;
    if (!sm100_cpu_check(ke, pl, in_buf_ids, out_buf_id, &exact)) SM100_N_MISMATCH++;
    SM100_N_EXACT += exact;
  }
  return rc;
}

__attribute__((constructor)) static void sm100_ref_install(void) {
  if (!sm100_env_on("THVM_SM100_CHECK", 0)) return;
  SM100_CPU_DISPATCH = CPU_BACKEND.dispatch_kernel;
  CPU_BACKEND.dispatch_kernel = sm100_ref_dispatch;
}
#endif

#ifdef THVM_HAS_CUDA
/* ---- the device hook ---------------------------------------------------------- */

static int (*SM100_RENDERED)(struct KernelEntry *, u32 *, u32);
static CUdeviceptr SM100_SCRATCH;
static u64 SM100_SCRATCH_BYTES;

/* A scratch block of >= need bytes for a linear's A side.  Blocks are never
 * freed: a captured graph keeps the address it recorded.  None is allocated
 * while the stream captures. */
static int sm100_scratch(u64 need) {
  if (need <= SM100_SCRATCH_BYTES) return 1;
  CUstreamCaptureStatus cs = CU_STREAM_CAPTURE_STATUS_NONE;
  if (CUDA_CUR_STREAM && cuStreamIsCapturing(CUDA_CUR_STREAM, &cs) == CUDA_SUCCESS &&
      cs != CU_STREAM_CAPTURE_STATUS_NONE)
    return 0;
  u64 n = need < (16u << 20) ? (16u << 20) : need;
  CUdeviceptr p = 0;
  if (cuMemAlloc(&p, n) != CUDA_SUCCESS) return 0;
  SM100_SCRATCH = p;
  SM100_SCRATCH_BYTES = n;
  return 1;
}

static int sm100_buf_ok(u32 id) { return id != 0 && id < CUDA_BUFS_NEXT && cuda_buf_dptr(id) != 0; }

/* Scratch of the pre-pass families: bump allocations from 64 MiB device
 * blocks, never freed (a captured graph keeps the addresses it recorded), and
 * none made while the stream captures. */
static void *sm100_arena(u64 bytes) {
  static CUdeviceptr blk;
  static u64 used, cap;
  bytes = (bytes + 255) & ~(u64)255;
  if (!blk || used + bytes > cap) {
    CUstreamCaptureStatus cs = CU_STREAM_CAPTURE_STATUS_NONE;
    if (CUDA_CUR_STREAM && cuStreamIsCapturing(CUDA_CUR_STREAM, &cs) == CUDA_SUCCESS &&
        cs != CU_STREAM_CAPTURE_STATUS_NONE)
      return NULL;
    const u64 n = bytes > (64ull << 20) ? bytes : (64ull << 20);
    CUdeviceptr p = 0;
    if (cuMemAlloc(&p, n) != CUDA_SUCCESS) return NULL;
    blk = p, used = 0, cap = n;
  }
  void *r = (void *)(uintptr_t)(blk + used);
  used += bytes;
  return r;
}

/* a program and its pre-passes on the device (slots 0..n_in given) */
static int sm100_run_family(Sm100Prog *pg, void **bufs, int64_t *bytes, u32 n_in, void *stream) {
  for (u32 j = 0; j < pg->n_scr; j++) {
    if (!pg->scr_ptr[j] && !(pg->scr_ptr[j] = sm100_arena(pg->scr_bytes[j])))
      return sm100_set_error(SM100_ERR_STATE, "router: no scratch for a pre-pass (%llu B)",
                             (unsigned long long)pg->scr_bytes[j]);
    bufs[n_in + 1 + j] = pg->scr_ptr[j];
    bytes[n_in + 1 + j] = (int64_t)pg->scr_bytes[j];
  }
  const u32 nb = n_in + 1 + pg->n_scr;
  int64_t ge[SM100_INTERP_MAX_AXES], vars[SM100_INTERP_MAX_VARS];
  void *out0 = bufs[0];
  const int64_t ob0 = bytes[0];
  for (u32 i = 0; i < pg->n_pre; i++) {
    const Sm100Prog *q = pg->pre[i];
    bufs[0] = pg->scr_ptr[pg->pre_out[i]];
    bytes[0] = (int64_t)pg->scr_bytes[pg->pre_out[i]];
    sm100_prog_runtime(q, ge, vars);
    const int rc = sm100_interp_run(q->code, q->n_code, q->n_regs, q->n_axes, q->n_glob, ge, bufs, bytes, nb, vars,
                                    q->n_vars, stream);
    if (rc != SM100_OK) return rc;
  }
  bufs[0] = out0;
  bytes[0] = ob0;
  sm100_prog_runtime(pg, ge, vars);
  return sm100_interp_run(pg->code, pg->n_code, pg->n_regs, pg->n_axes, pg->n_glob, ge, bufs, bytes, nb, vars,
                          pg->n_vars, stream);
}

static int sm100_ref_dispatch(struct KernelEntry *ke, u32 *in_buf_ids, u32 out_buf_id) {
  SM100_N_DISPATCH++;
  if (!CUDA_READY || kernel_is_custom(ke) || !sm100_env_on("THVM_SM100", 1)) {
    SM100_N_DECLINED++;
    return SM100_RENDERED(ke, in_buf_ids, out_buf_id);
  }
  Sm100Plan *pl = sm100_ref_plan(ke);
  sm100_log(ke, pl);
  const u32 n_in = ke->n_inputs;
  int ok = pl->kind != SM100_R_NONE && sm100_buf_ok(out_buf_id) && n_in + 1 <= SM100_INTERP_MAX_BUFS;
  for (u32 i = 0; ok && i < n_in; i++) ok = sm100_buf_ok(in_buf_ids[i]);
  if (!ok) {
    SM100_N_DECLINED++;
    return SM100_RENDERED(ke, in_buf_ids, out_buf_id);
  }
  void *bufs[SM100_INTERP_MAX_BUFS] = {0};
  int64_t bytes[SM100_INTERP_MAX_BUFS] = {0};
  bufs[0] = (void *)(uintptr_t)cuda_buf_dptr(out_buf_id);
  bytes[0] = (int64_t)CUDA_BUFS[out_buf_id].nbytes;
  for (u32 i = 0; i < n_in; i++) {
    bufs[1 + i] = (void *)(uintptr_t)cuda_buf_dptr(in_buf_ids[i]);
    bytes[1 + i] = (int64_t)CUDA_BUFS[in_buf_ids[i]].nbytes;
  }
  void *stream = (void *)CUDA_CUR_STREAM;
  int64_t ge[SM100_INTERP_MAX_AXES], vars[SM100_INTERP_MAX_VARS];
  int rc = SM100_OK;
  if (pl->kind == SM100_R_INTERP) {
    rc = sm100_run_family(pl->prog, bufs, bytes, n_in, stream);
    if (rc == SM100_OK) SM100_N_INTERP++;
  } else {
    const u64 xb = (u64)pl->M * pl->K * 4, wb = (u64)pl->N * pl->K * 4, yb = (u64)pl->M * pl->N * 4;
    const float *x = NULL;
    if (pl->x_in >= 0) {
      x = (const float *)bufs[1 + pl->x_in];
      if ((u64)bytes[1 + pl->x_in] < xb) rc = SM100_ERR_ARG;
    } else if (!sm100_scratch(xb)) {
      rc = SM100_ERR_STATE;
    } else {
      void *sb[SM100_INTERP_MAX_BUFS];
      int64_t sbytes[SM100_INTERP_MAX_BUFS];
      memcpy(sb, bufs, sizeof sb);
      memcpy(sbytes, bytes, sizeof sbytes);
      sb[0] = (void *)(uintptr_t)SM100_SCRATCH;
      sbytes[0] = (int64_t)xb;
      rc = sm100_run_family(pl->pro, sb, sbytes, n_in, stream);
      x = (const float *)(uintptr_t)SM100_SCRATCH;
    }
    if (rc == SM100_OK && ((u64)bytes[1 + pl->w_in] < wb || (u64)bytes[0] < yb)) rc = SM100_ERR_ARG;
    if (rc == SM100_OK) {
      Sm100LinearArgs a;
      memset(&a, 0, sizeof a);
      a.x = x;
      a.w = bufs[1 + pl->w_in];
      a.y = (float *)bufs[0];
      a.M = pl->M, a.N = pl->N, a.K = pl->K, a.ldx = pl->K, a.ldy = pl->N;
      a.wdtype = SM100_DT_F32;
      rc = sm100_linear(&a, stream);
    }
    if (rc == SM100_OK) SM100_N_LINEAR++;
  }
  if (rc != SM100_OK) {
    /* nothing of this kernel was left half-done on the stream except a
     * prologue into scratch: the rendered path writes the whole output */
    FILE *fp = sm100_log_fp();
    if (fp) fprintf(fp, "FALLBACK kid=%u: %s\n", (u32)(ke - KERNELS), sm100_last_error());
    SM100_N_DECLINED++;
    return SM100_RENDERED(ke, in_buf_ids, out_buf_id);
  }
  return 0;
}

__attribute__((constructor)) static void sm100_ref_install(void) {
  SM100_RENDERED = CUDA_BACKEND.dispatch_kernel;
  CUDA_BACKEND.dispatch_kernel = sm100_ref_dispatch;
}

/* the interpreter's step-budget word (sm100_interp_status), for tests */
EXPORT int py_sm100_interp_status(void) { return sm100_interp_status(); }
#endif
