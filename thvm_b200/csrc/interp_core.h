/* interp_core.h - the register-program evaluator of the generic device
 * interpreter (include/thvm_sm100.h SM100_IOP_*).  Plain C that nvcc compiles
 * for the device (k_interp.cu) and a C compiler for the host (the CPU check of
 * the reference-side router, thvm_b200/refside/sm100_ref.c), so both run the
 * same steps.  Semantics follow the reference's CPU walker
 * (src/backend/cpu/uop_walk.c): f32 arithmetic rounded per operation, int
 * arithmetic in int64 wrapped where the walker wraps (IDIV / IMOD / shifts,
 * reduce combines, stores), a divisor of 0 giving 0, exp2 as the xexp2
 * decomposition (src/codegen/xexp2f.c:12-33).  Host builds must not contract
 * multiply-adds (-ffp-contract=off). */
#ifndef THVM_SM100_INTERP_CORE_H
#define THVM_SM100_INTERP_CORE_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/thvm_sm100.h"

#ifdef __CUDACC__
#define SM100_HD static __device__ __forceinline__
#define SM100_FADD(a, b) __fadd_rn(a, b)
#define SM100_FSUB(a, b) __fsub_rn(a, b)
#define SM100_FMUL(a, b) __fmul_rn(a, b)
#define SM100_FRCP(a) __frcp_rn(a)
#define SM100_FSQRT(a) __fsqrt_rn(a)
#define SM100_FLOG2(a) log2f(a)
#define SM100_FSIN(a) sinf(a)
#else
#define SM100_HD static inline
#define SM100_FADD(a, b) ((a) + (b))
#define SM100_FSUB(a, b) ((a) - (b))
#define SM100_FMUL(a, b) ((a) * (b))
#define SM100_FRCP(a) (1.0f / (a))
#define SM100_FSQRT(a) sqrtf(a)
#define SM100_FLOG2(a) ((float)log2((double)(a)))
#define SM100_FSIN(a) ((float)sin((double)(a)))
#endif

SM100_HD float sm100_i_f(int64_t r) {
  uint32_t b = (uint32_t)r;
  float f;
  memcpy(&f, &b, 4);
  return f;
}

SM100_HD int64_t sm100_i_r(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return (int64_t)b;
}

SM100_HD float sm100_i_xexp2(float d) {
  const int finite = (d == d) && (d != INFINITY) && (d != -INFINITY);
  const float x = finite ? d : 0.0f;
  const int q = (int)SM100_FADD(x, x < 0.0f ? -0.5f : 0.5f);
  const float s = SM100_FSUB(x, (float)q);
  float u = 0.1535920892e-3f;
  u = SM100_FADD(SM100_FMUL(u, s), 0.1339262701e-2f);
  u = SM100_FADD(SM100_FMUL(u, s), 0.9618384764e-2f);
  u = SM100_FADD(SM100_FMUL(u, s), 0.5550347269e-1f);
  u = SM100_FADD(SM100_FMUL(u, s), 0.2402264476e+0f);
  u = SM100_FADD(SM100_FMUL(u, s), 0.6931471825e+0f);
  u = SM100_FADD(SM100_FMUL(u, s), 1.0f);
  const int h = q >> 1;
  u = SM100_FMUL(SM100_FMUL(u, sm100_i_f((int64_t)((uint32_t)(h + 127) << 23))),
                 sm100_i_f((int64_t)((uint32_t)(q - h + 127) << 23)));
  u = d < 128.0f ? u : INFINITY;
  u = d < -150.0f ? 0.0f : u;
  return (d == d) ? u : sm100_i_f(0x7fc00000);
}

/* int v wrapped to dtype dt (bool: v != 0) */
SM100_HD int64_t sm100_i_wrap(int dt, int64_t v) {
  switch (dt) {
    case SM100_UDT_BOOL: return v != 0;
    case SM100_UDT_I8: return (int8_t)v;
    case SM100_UDT_U8: return (uint8_t)v;
    case SM100_UDT_I16: return (int16_t)v;
    case SM100_UDT_U16: return (uint16_t)v;
    case SM100_UDT_I32: return (int32_t)v;
    case SM100_UDT_U32: return (uint32_t)v;
    default: return v;
  }
}

SM100_HD int sm100_i_signed(int dt) {
  return dt == SM100_UDT_I8 || dt == SM100_UDT_I16 || dt == SM100_UDT_I32 || dt == SM100_UDT_I64;
}

/* f16 / bf16 bits <-> f32 (round to nearest even; NaN kept quiet) */
SM100_HD float sm100_i_h2f(uint32_t h) {
  uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  if (e == 0x1f) return sm100_i_f((int64_t)(s | 0x7f800000u | (m << 13)));
  if (e == 0) {
    float f = (float)m * (1.0f / 16777216.0f);
    return s ? -f : f;
  }
  return sm100_i_f((int64_t)(s | ((e + 112) << 23) | (m << 13)));
}

SM100_HD uint32_t sm100_i_f2h(float f) {
  uint32_t x = (uint32_t)sm100_i_r(f), s = (x >> 16) & 0x8000u;
  uint32_t a = x & 0x7fffffffu;
  if (a > 0x7f800000u) return s | 0x7e00u;
  if (a >= 0x477ff000u) return s | 0x7c00u; /* rounds past the largest half */
  if (a < 0x38800000u) {                    /* subnormal half */
    if (a < 0x33000000u) return s;
    uint32_t m = (a & 0x7fffffu) | 0x800000u, sh = 126 - (a >> 23);
    uint32_t q = m >> sh, rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return s | q;
  }
  uint32_t q = ((a >> 13) - (112u << 10)), rem = a & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return s | q;
}

SM100_HD uint32_t sm100_i_f2bf(float f) {
  uint32_t x = (uint32_t)sm100_i_r(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (x >> 16) | 0x40u;
  return (x + 0x7fffu + ((x >> 16) & 1)) >> 16;
}

SM100_HD int sm100_i_isfloat(int dt) {
  return dt == SM100_UDT_F16 || dt == SM100_UDT_BF16 || dt == SM100_UDT_F32 || dt == SM100_UDT_F64;
}

/* log2 of the element size of dtype dt */
SM100_HD int sm100_i_shift(int dt) {
  switch (dt) {
    case SM100_UDT_BOOL: case SM100_UDT_I8: case SM100_UDT_U8: return 0;
    case SM100_UDT_I16: case SM100_UDT_U16: case SM100_UDT_F16: case SM100_UDT_BF16: return 1;
    case SM100_UDT_I64: case SM100_UDT_U64: case SM100_UDT_F64: return 3;
    default: return 2;
  }
}

SM100_HD int64_t sm100_i_load(const void *p, int64_t off, int dt) {
  switch (dt) {
    case SM100_UDT_F32: return (int64_t)((const uint32_t *)p)[off];
    case SM100_UDT_F16: return sm100_i_r(sm100_i_h2f(((const uint16_t *)p)[off]));
    case SM100_UDT_BF16: return (int64_t)((uint32_t)((const uint16_t *)p)[off] << 16);
    case SM100_UDT_F64: return sm100_i_r((float)((const double *)p)[off]);
    case SM100_UDT_BOOL: return ((const uint8_t *)p)[off] != 0;
    case SM100_UDT_I8: return ((const int8_t *)p)[off];
    case SM100_UDT_U8: return ((const uint8_t *)p)[off];
    case SM100_UDT_I16: return ((const int16_t *)p)[off];
    case SM100_UDT_U16: return ((const uint16_t *)p)[off];
    case SM100_UDT_I32: return ((const int32_t *)p)[off];
    case SM100_UDT_U32: return ((const uint32_t *)p)[off];
    default: return ((const int64_t *)p)[off];
  }
}

SM100_HD void sm100_i_store(void *p, int64_t off, int dt, int64_t v) {
  switch (dt) {
    case SM100_UDT_F32: ((uint32_t *)p)[off] = (uint32_t)v; break;
    case SM100_UDT_F16: ((uint16_t *)p)[off] = (uint16_t)sm100_i_f2h(sm100_i_f(v)); break;
    case SM100_UDT_BF16: ((uint16_t *)p)[off] = (uint16_t)sm100_i_f2bf(sm100_i_f(v)); break;
    case SM100_UDT_F64: ((double *)p)[off] = (double)sm100_i_f(v); break;
    case SM100_UDT_BOOL: ((uint8_t *)p)[off] = v != 0; break;
    case SM100_UDT_I8: case SM100_UDT_U8: ((uint8_t *)p)[off] = (uint8_t)v; break;
    case SM100_UDT_I16: case SM100_UDT_U16: ((uint16_t *)p)[off] = (uint16_t)v; break;
    case SM100_UDT_I32: case SM100_UDT_U32: ((uint32_t *)p)[off] = (uint32_t)v; break;
    default: ((int64_t *)p)[off] = v; break;
  }
}

/* f32 -> int dtype as a C cast: toward zero, NaN 0, saturating past int64 */
SM100_HD int64_t sm100_i_f2i(int dt, float f) {
  if (dt == SM100_UDT_BOOL) return f != 0.0f;
  if (f != f) return 0;
  if (f >= 9223372036854775808.0f) return sm100_i_wrap(dt, dt == SM100_UDT_U64 ? (int64_t)-1 : INT64_MAX);
  if (f < -9223372036854775808.0f) return sm100_i_wrap(dt, INT64_MIN);
  return sm100_i_wrap(dt, (int64_t)f);
}

/* Threefry-2x32, 20 rounds (Salmon et al., "Parallel random numbers: as easy
 * as 1, 2, 3", SC 2011) in the arrangement tinygrad's THREEFRY decomposition
 * uses (src/codegen/threefry.c:10-25): x and key split into 32-bit halves,
 * key words (k1, k0 ^ k1 ^ 0x1BD11BDA, k0), injection every four rounds with
 * the round-group counter added to the second word, halves packed back as
 * (x1 << 32) | x0. */
SM100_HD uint64_t sm100_i_threefry(uint64_t x, uint64_t key) {
  const uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
  const uint32_t ks[3] = {k1, k0 ^ k1 ^ 0x1BD11BDAu, k0};
  const uint32_t rot[8] = {13, 15, 26, 6, 17, 29, 16, 24};
  uint32_t a = (uint32_t)x + k0, b = (uint32_t)(x >> 32) + k1;
  for (uint32_t g = 0; g < 5; g++) {
    for (uint32_t j = 0; j < 4; j++) {
      const uint32_t s = rot[(g & 1) * 4 + j];
      a += b;
      b = a ^ ((b << s) | (b >> (32 - s)));
    }
    a += ks[g % 3];
    b += ks[(g + 1) % 3] + g + 1;
  }
  return ((uint64_t)b << 32) | a;
}

/* Runs the program once: r = registers, idx = range slots (the first n_glob
 * already hold this element's output coordinates).  Every load and store is
 * checked against its buffer's byte size: both arms of a select are
 * evaluated, and the untaken one may address outside its buffer (a padded
 * read), so an out-of-range load reads 0 and an out-of-range store is
 * dropped. */
SM100_HD int sm100_interp_exec(const Sm100Insn *code, uint32_t n_code, int64_t *r, int64_t *idx,
                               void *const *bufs, const int64_t *buf_bytes, const int64_t *vars) {
  int64_t steps = 0; /* loop back-edges taken: a program past the budget stops (returns 1) */
  for (uint32_t pc = 0; pc < n_code; pc++) {
    const Sm100Insn in = code[pc];
    /* operand registers are read by the ops that use them */
#define A r[in.a]
#define B r[in.b]
    switch (in.op) {
      case SM100_IOP_CONST:
        r[in.dst] = in.dt == 0 ? (int64_t)in.imm : (int64_t)(uint32_t)in.imm;
        break;
      case SM100_IOP_RANGE: r[in.dst] = idx[in.a]; break;
      case SM100_IOP_VAR: r[in.dst] = vars[in.a]; break;
      case SM100_IOP_LOAD: {
        const int64_t off = B;
        r[in.dst] = (off >= 0 && off < (buf_bytes[in.a] >> sm100_i_shift(in.dt))) ? sm100_i_load(bufs[in.a], off, in.dt) : 0;
        break;
      }
      case SM100_IOP_STORE: {
        const int64_t off = B;
        if (off >= 0 && off < (buf_bytes[in.a] >> sm100_i_shift(in.dt))) sm100_i_store(bufs[in.a], off, in.dt, r[in.c]);
        break;
      }
      case SM100_IOP_FADD: r[in.dst] = sm100_i_r(SM100_FADD(sm100_i_f(A), sm100_i_f(B))); break;
      case SM100_IOP_FMUL: r[in.dst] = sm100_i_r(SM100_FMUL(sm100_i_f(A), sm100_i_f(B))); break;
      case SM100_IOP_FNEG: r[in.dst] = sm100_i_r(-sm100_i_f(A)); break;
      case SM100_IOP_FRECIP: r[in.dst] = sm100_i_r(SM100_FRCP(sm100_i_f(A))); break;
      case SM100_IOP_FEXP2: r[in.dst] = sm100_i_r(sm100_i_xexp2(sm100_i_f(A))); break;
      case SM100_IOP_FLOG2: r[in.dst] = sm100_i_r(SM100_FLOG2(sm100_i_f(A))); break;
      case SM100_IOP_FSQRT: r[in.dst] = sm100_i_r(SM100_FSQRT(sm100_i_f(A))); break;
      case SM100_IOP_FSIN: r[in.dst] = sm100_i_r(SM100_FSIN(sm100_i_f(A))); break;
      case SM100_IOP_FLT: r[in.dst] = sm100_i_f(A) < sm100_i_f(B); break;
      case SM100_IOP_FEQ: r[in.dst] = sm100_i_f(A) == sm100_i_f(B); break;
      case SM100_IOP_IADD: r[in.dst] = (int64_t)((uint64_t)A + (uint64_t)B); break;
      case SM100_IOP_ISUB: r[in.dst] = (int64_t)((uint64_t)A - (uint64_t)B); break;
      case SM100_IOP_IMUL: r[in.dst] = (int64_t)((uint64_t)A * (uint64_t)B); break;
      case SM100_IOP_INEG: r[in.dst] = (int64_t)(0 - (uint64_t)A); break;
      case SM100_IOP_IDIV: case SM100_IOP_IMOD: {
        const int64_t a = sm100_i_wrap(in.dt, A), b = sm100_i_wrap(in.dt, B);
        int64_t q = 0;
        if (b != 0) {
          if (!sm100_i_signed(in.dt))
            q = (int64_t)(in.op == SM100_IOP_IDIV ? (uint64_t)a / (uint64_t)b : (uint64_t)a % (uint64_t)b);
          else if (b == -1)
            q = in.op == SM100_IOP_IDIV ? (int64_t)(0 - (uint64_t)a) : 0;
          else
            q = in.op == SM100_IOP_IDIV ? a / b : a % b;
        }
        r[in.dst] = sm100_i_wrap(in.dt, q);
        break;
      }
      case SM100_IOP_ILT: r[in.dst] = A < B; break;
      case SM100_IOP_ULT: r[in.dst] = (uint64_t)A < (uint64_t)B; break;
      case SM100_IOP_IEQ: r[in.dst] = A == B; break;
      case SM100_IOP_IAND: r[in.dst] = A & B; break;
      case SM100_IOP_IOR: r[in.dst] = A | B; break;
      case SM100_IOP_IXOR: r[in.dst] = A ^ B; break;
      case SM100_IOP_ISHL: r[in.dst] = sm100_i_wrap(in.dt, (int64_t)((uint64_t)sm100_i_wrap(in.dt, A) << (B & 63))); break;
      case SM100_IOP_ISHR: {
        const int64_t a = sm100_i_wrap(in.dt, A);
        r[in.dst] = sm100_i_signed(in.dt) ? (a >> (B & 63)) : (int64_t)((uint64_t)a >> (B & 63));
        break;
      }
      case SM100_IOP_WRAP: r[in.dst] = sm100_i_wrap(in.dt, A); break;
      case SM100_IOP_I2F:
        r[in.dst] = sm100_i_r(in.dt == SM100_UDT_U64 ? (float)(uint64_t)A : (float)A);
        break;
      case SM100_IOP_F2I: r[in.dst] = sm100_i_f2i(in.dt, sm100_i_f(A)); break;
      case SM100_IOP_NARROW: {
        const float f = sm100_i_f(A);
        if (f != f) r[in.dst] = A;
        else if (in.dt == SM100_UDT_F16) r[in.dst] = sm100_i_r(sm100_i_h2f(sm100_i_f2h(f)));
        else if (in.dt == SM100_UDT_BF16) r[in.dst] = (int64_t)(sm100_i_f2bf(f) << 16);
        else r[in.dst] = A;
        break;
      }
      case SM100_IOP_SEL: r[in.dst] = A != 0 ? B : r[in.c]; break;
      case SM100_IOP_LOOP:
        idx[in.a] = 0;
        if (B <= 0) pc = (uint32_t)in.imm;
        break;
      case SM100_IOP_ENDLOOP:
        if (++idx[in.a] < B) {
          if (++steps > SM100_INTERP_MAX_STEPS) return 1;
          pc = (uint32_t)in.imm;
        }
        break;
      case SM100_IOP_ACCF: {
        const float acc = sm100_i_f(r[in.dst]), v = sm100_i_f(A);
        const float o = in.dt == 0 ? SM100_FADD(acc, v) : in.dt == 1 ? (v > acc ? v : acc) : SM100_FMUL(acc, v);
        r[in.dst] = sm100_i_r(o);
        break;
      }
      case SM100_IOP_ACCI: {
        const int64_t acc = r[in.dst], v = sm100_i_wrap(in.dt, A);
        int64_t o;
        if (in.dt == SM100_UDT_BOOL) o = in.imm == 2 ? (acc & v) : (acc | v);
        else if (in.imm == 0) o = sm100_i_wrap(in.dt, (int64_t)((uint64_t)acc + (uint64_t)v));
        else if (in.imm == 2) o = sm100_i_wrap(in.dt, (int64_t)((uint64_t)acc * (uint64_t)v));
        else if (in.dt == SM100_UDT_U64) o = (uint64_t)acc < (uint64_t)v ? v : acc;
        else o = acc < v ? v : acc;
        r[in.dst] = o;
        break;
      }
      case SM100_IOP_THREEFRY: r[in.dst] = (int64_t)sm100_i_threefry((uint64_t)A, (uint64_t)B); break;
      case SM100_IOP_SETR: idx[in.a] = B; break;
      default: break;
    }
#undef A
#undef B
  }
  return 0;
}

/* 0 when the program's loops are well formed: each LOOP at i names an
 * ENDLOOP at j > i that names it back with the same slot, loops nest, and
 * no open loop's slot is reused inside it (so every loop terminates). */
static inline int sm100_interp_check_loops(const Sm100Insn *code, uint32_t n_code) {
  uint32_t open[SM100_INTERP_MAX_AXES + 1], n_open = 0;
  for (uint32_t i = 0; i < n_code; i++) {
    if (code[i].op == SM100_IOP_LOOP) {
      const int32_t j = code[i].imm;
      if (j <= (int32_t)i || (uint32_t)j >= n_code || code[j].op != SM100_IOP_ENDLOOP || code[j].imm != (int32_t)i ||
          code[j].a != code[i].a || code[j].b != code[i].b || n_open > SM100_INTERP_MAX_AXES)
        return 1;
      for (uint32_t k = 0; k < n_open; k++)
        if (code[open[k]].a == code[i].a) return 1;
      open[n_open++] = i;
    } else if (code[i].op == SM100_IOP_ENDLOOP) {
      if (n_open == 0 || open[n_open - 1] != (uint32_t)code[i].imm) return 1;
      n_open--;
    }
  }
  return n_open != 0;
}

#endif
