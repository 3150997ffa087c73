/* weights.c - weight files straight into device buffers: the .safetensors
 * format the reference reads and writes (py/thvm/nn_state.py safe_load /
 * safe_save :44-85, after tinygrad nn/state.py) and the DSV2PK01 pack its
 * DeepSeek-V2 bench loads (bench/dsv2_decode_bench.c:229-262).
 *
 * The file is mapped read-only and every tensor's bytes are written into a
 * fresh backend buffer with one copy from the mapping (sm100_buf_write: a
 * host-to-device copy, no intermediate host buffer); the caller gets one
 * entry per tensor (name, dtype tag, shape, byte count, buffer id) and owns
 * the buffers (sm100_buf_decref / free).  Errors leave no buffer behind.
 */
#define _GNU_SOURCE
#include <ctype.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/thvm_sm100.h"

int sm100_set_error(int code, const char *fmt, ...);

typedef struct {
  const unsigned char *p;
  size_t n;
  int fd;
} Map;

static int map_open(const char *path, Map *m) {
  struct stat st;
  m->fd = open(path, O_RDONLY);
  if (m->fd < 0 || fstat(m->fd, &st) != 0) {
    if (m->fd >= 0) close(m->fd);
    return sm100_set_error(SM100_ERR_ARG, "weights: cannot open %s", path);
  }
  m->n = (size_t)st.st_size;
  m->p = m->n ? (const unsigned char *)mmap(NULL, m->n, PROT_READ, MAP_PRIVATE, m->fd, 0) : NULL;
  if (m->n && m->p == MAP_FAILED) {
    close(m->fd);
    return sm100_set_error(SM100_ERR_ARG, "weights: cannot map %s", path);
  }
  return SM100_OK;
}

static void map_close(Map *m) {
  if (m->p && m->n) munmap((void *)m->p, m->n);
  close(m->fd);
}

static void drop_all(Sm100TensorEntry *e, int32_t n) {
  for (int32_t i = 0; i < n; i++)
    if (e[i].buf_id) sm100_buf_free(e[i].buf_id);
}

/* one tensor's bytes into a fresh buffer */
static int upload(Sm100TensorEntry *e, const unsigned char *src) {
  e->buf_id = sm100_buf_alloc(e->nbytes ? e->nbytes : 1);
  if (!e->buf_id) return sm100_set_error(SM100_ERR_OOM, "weights: buffer for %s (%llu B)", e->name,
                                         (unsigned long long)e->nbytes);
  return e->nbytes ? sm100_buf_write(e->buf_id, src, e->nbytes) : SM100_OK;
}

/* ---- a JSON reader for the safetensors header ------------------------------
 * The header is one object: name -> {"dtype": str, "shape": [int...],
 * "data_offsets": [int, int]}, plus an optional "__metadata__" object of
 * strings, which is skipped. */
typedef struct {
  const char *s, *end;
} Js;

static void js_ws(Js *j) {
  while (j->s < j->end && isspace((unsigned char)*j->s)) j->s++;
}

static int js_eat(Js *j, char c) {
  js_ws(j);
  if (j->s < j->end && *j->s == c) {
    j->s++;
    return 1;
  }
  return 0;
}

/* a string into out (escapes kept verbatim but for \" and \\) */
static int js_str(Js *j, char *out, size_t cap) {
  js_ws(j);
  if (j->s >= j->end || *j->s != '"') return 0;
  j->s++;
  size_t k = 0;
  while (j->s < j->end && *j->s != '"') {
    char c = *j->s++;
    if (c == '\\' && j->s < j->end) c = *j->s++;
    if (k + 1 < cap) out[k++] = c;
  }
  if (j->s >= j->end) return 0;
  j->s++;
  if (cap) out[k < cap ? k : cap - 1] = 0;
  return 1;
}

static int js_int(Js *j, int64_t *v) {
  js_ws(j);
  char *e = NULL;
  long long x = strtoll(j->s, &e, 10);
  if (e == j->s) return 0;
  j->s = e;
  *v = x;
  return 1;
}

/* skip any value (for __metadata__) */
static int js_skip(Js *j) {
  js_ws(j);
  if (j->s >= j->end) return 0;
  char c = *j->s;
  if (c == '"') {
    char tmp[4];
    return js_str(j, tmp, sizeof tmp);
  }
  if (c == '{' || c == '[') {
    const char close = c == '{' ? '}' : ']';
    j->s++;
    if (js_eat(j, close)) return 1;
    do {
      if (c == '{') {
        char tmp[4];
        if (!js_str(j, tmp, sizeof tmp) || !js_eat(j, ':')) return 0;
      }
      if (!js_skip(j)) return 0;
    } while (js_eat(j, ','));
    return js_eat(j, close);
  }
  while (j->s < j->end && *j->s != ',' && *j->s != '}' && *j->s != ']') j->s++;
  return 1;
}

int sm100_safetensors_load(const char *path, Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out) {
  if (!path || !entries || max_entries < 1 || !n_out) return sm100_set_error(SM100_ERR_ARG, "safetensors: bad arguments");
  *n_out = 0;
  Map m;
  int rc = map_open(path, &m);
  if (rc != SM100_OK) return rc;
  uint64_t hlen = 0;
  if (m.n < 8 || (memcpy(&hlen, m.p, 8), hlen > m.n - 8)) {
    map_close(&m);
    return sm100_set_error(SM100_ERR_ARG, "safetensors: %s: bad header length", path);
  }
  const unsigned char *data = m.p + 8 + hlen;
  const uint64_t data_n = m.n - 8 - hlen;
  Js j = {(const char *)m.p + 8, (const char *)m.p + 8 + hlen};
  int32_t n = 0;
  rc = SM100_OK;
  if (!js_eat(&j, '{')) rc = sm100_set_error(SM100_ERR_ARG, "safetensors: %s: header is not an object", path);
  if (rc == SM100_OK && !js_eat(&j, '}')) {
    do {
      char key[sizeof entries[0].name];
      if (!js_str(&j, key, sizeof key) || !js_eat(&j, ':')) {
        rc = sm100_set_error(SM100_ERR_ARG, "safetensors: %s: malformed header", path);
        break;
      }
      if (strcmp(key, "__metadata__") == 0) {
        if (!js_skip(&j)) {
          rc = sm100_set_error(SM100_ERR_ARG, "safetensors: %s: malformed __metadata__", path);
          break;
        }
        continue;
      }
      if (n >= max_entries) {
        rc = sm100_set_error(SM100_ERR_ARG, "safetensors: %s: more than %d tensors", path, max_entries);
        break;
      }
      Sm100TensorEntry *e = &entries[n];
      memset(e, 0, sizeof *e);
      snprintf(e->name, sizeof e->name, "%s", key);
      int64_t off0 = -1, off1 = -1;
      int ok = js_eat(&j, '{');
      while (ok && !js_eat(&j, '}')) {
        char field[32];
        ok = js_str(&j, field, sizeof field) && js_eat(&j, ':');
        if (!ok) break;
        if (strcmp(field, "dtype") == 0) {
          ok = js_str(&j, e->dtype, sizeof e->dtype);
        } else if (strcmp(field, "shape") == 0) {
          ok = js_eat(&j, '[');
          if (ok && !js_eat(&j, ']')) {
            do {
              int64_t d;
              ok = js_int(&j, &d) && e->ndim < 8 && d >= 0;
              if (ok) e->shape[e->ndim++] = d;
            } while (ok && js_eat(&j, ','));
            ok = ok && js_eat(&j, ']');
          }
        } else if (strcmp(field, "data_offsets") == 0) {
          ok = js_eat(&j, '[') && js_int(&j, &off0) && js_eat(&j, ',') && js_int(&j, &off1) && js_eat(&j, ']');
        } else {
          ok = js_skip(&j);
        }
        if (ok) js_eat(&j, ',');
      }
      if (!ok || off0 < 0 || off1 < off0 || (uint64_t)off1 > data_n || !e->dtype[0]) {
        rc = sm100_set_error(SM100_ERR_ARG, "safetensors: %s: bad entry %s", path, key);
        break;
      }
      e->nbytes = (uint64_t)(off1 - off0);
      rc = upload(e, data + off0);
      if (rc != SM100_OK) break;
      n++;
    } while (js_eat(&j, ','));
    if (rc == SM100_OK && !js_eat(&j, '}'))
      rc = sm100_set_error(SM100_ERR_ARG, "safetensors: %s: unterminated header", path);
  }
  map_close(&m);
  if (rc != SM100_OK) {
    drop_all(entries, n);
    return rc;
  }
  *n_out = n;
  return SM100_OK;
}

int sm100_dsv2pack_load(const char *path, Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out) {
  if (!path || !entries || max_entries < 1 || !n_out) return sm100_set_error(SM100_ERR_ARG, "dsv2pack: bad arguments");
  *n_out = 0;
  Map m;
  int rc = map_open(path, &m);
  if (rc != SM100_OK) return rc;
  uint64_t count = 0;
  if (m.n < 16 || memcmp(m.p, "DSV2PK01", 8) != 0 || (memcpy(&count, m.p + 8, 8), count > (m.n - 16) / 72)) {
    map_close(&m);
    return sm100_set_error(SM100_ERR_ARG, "dsv2pack: %s: not a DSV2PK01 pack", path);
  }
  if (count > (uint64_t)max_entries) {
    map_close(&m);
    return sm100_set_error(SM100_ERR_ARG, "dsv2pack: %s: %llu tensors (room for %d)", path,
                           (unsigned long long)count, max_entries);
  }
  int32_t n = 0;
  for (uint64_t i = 0; i < count && rc == SM100_OK; i++) {
    /* { char name[48]; u32 dtype (0 bf16, 1 f32); u32 pad; u64 offset; u64 nbytes } */
    const unsigned char *t = m.p + 16 + 72 * i;
    uint32_t dt;
    uint64_t off, nb;
    memcpy(&dt, t + 48, 4);
    memcpy(&off, t + 56, 8);
    memcpy(&nb, t + 64, 8);
    Sm100TensorEntry *e = &entries[n];
    memset(e, 0, sizeof *e);
    memcpy(e->name, t, 48);
    e->name[48] = 0;
    if (dt > 1 || off > m.n || nb > m.n - off) {
      rc = sm100_set_error(SM100_ERR_ARG, "dsv2pack: %s: bad entry %s", path, e->name);
      break;
    }
    snprintf(e->dtype, sizeof e->dtype, "%s", dt == 0 ? "BF16" : "F32");
    e->ndim = 1;
    e->shape[0] = (int64_t)(nb / (dt == 0 ? 2 : 4));
    e->nbytes = nb;
    rc = upload(e, m.p + off);
    if (rc == SM100_OK) n++;
  }
  map_close(&m);
  if (rc != SM100_OK) {
    drop_all(entries, n);
    return rc;
  }
  *n_out = n;
  return SM100_OK;
}

/* ---- PyTorch checkpoints (torch.save) ----------------------------------------
 * The state dict of a .pt / .pth / .bin file as py/thvm/nn_state.py torch_load
 * reads it (:123-230, after tinygrad nn/state.py): the zip format
 * (<archive>/data.pkl, each storage at <archive>/data/<key>, stored
 * uncompressed; zip64 records for large files) or the legacy format (a
 * pickle stream: magic, protocol, sys_info, the state pickle, the list of
 * storage keys, then each storage as an 8-byte element count and its bytes).
 * The state pickle runs on a small pickle machine that knows what torch
 * writes: storages arrive as persistent ids ('storage', <type>Storage, key,
 * location, numel), tensors as torch._utils._rebuild_tensor_v2(storage,
 * offset, size, stride, ...), parameters as _rebuild_parameter(tensor, ...),
 * the dict as collections.OrderedDict.  Every top-level entry that is a
 * tensor (or a parameter) becomes one buffer holding its elements in
 * row-major order: a contiguous tensor by one copy from the mapping, a
 * permuted one (strides that are a permutation of a contiguous layout, the
 * only other kind the reference accepts) through a host gather.  Unlike the
 * reference, whose tensors are numpy arrays, elements keep their file type:
 * the entry's dtype tag is the storage's ("F32", "BF16", "F16", "F64",
 * "I64", "I32", "I16", "I8", "U8", "BOOL"; an unknown storage type reads as
 * F32, as there). */

typedef enum { PV_NONE, PV_BOOL, PV_INT, PV_FLOAT, PV_STR, PV_TUPLE, PV_LIST, PV_DICT, PV_GLOBAL, PV_STORAGE,
               PV_TENSOR, PV_OTHER } PvKind;

typedef struct Pv {
  PvKind k;
  int64_t i;                /* INT, STORAGE: numel */
  double f;
  const char *s;            /* STR (bytes of the pickle), GLOBAL: name, STORAGE: type name */
  size_t slen;
  const char *s2;           /* GLOBAL: module, STORAGE: key */
  size_t s2len;
  struct Pv **items;        /* TUPLE / LIST; DICT: key, value pairs */
  int32_t n, cap;
  struct Pv *storage;       /* TENSOR */
  int64_t offset, size[8], stride[8];
  int32_t ndim;
  struct Pv *next_alloc;
} Pv;

typedef struct {
  const unsigned char *p, *end;
  Pv *allocs;               /* every value, for the final free */
  Pv **stack;
  int32_t sp, scap;
  int32_t *marks;
  int32_t mp, mcap;
  Pv **memo;
  int64_t memo_n;
  const char *err;
} Pk;

static Pv *pv_new(Pk *k, PvKind kind) {
  Pv *v = (Pv *)calloc(1, sizeof *v);
  if (!v) {
    k->err = "out of host memory";
    return NULL;
  }
  v->k = kind;
  v->next_alloc = k->allocs;
  k->allocs = v;
  return v;
}

static int pv_add(Pk *k, Pv *c, Pv *item) {
  if (c->n == c->cap) {
    const int32_t cap = c->cap ? 2 * c->cap : 8;
    Pv **it = (Pv **)realloc(c->items, (size_t)cap * sizeof *it);
    if (!it) {
      k->err = "out of host memory";
      return 0;
    }
    c->items = it;
    c->cap = cap;
  }
  c->items[c->n++] = item;
  return 1;
}

static void pk_free(Pk *k) {
  for (Pv *v = k->allocs; v;) {
    Pv *n = v->next_alloc;
    free(v->items);
    free(v);
    v = n;
  }
  k->allocs = NULL;
  free(k->stack);
  free(k->marks);
  free(k->memo);
  k->stack = NULL;
  k->marks = NULL;
  k->memo = NULL;
  k->sp = k->scap = k->mp = k->mcap = 0;
  k->memo_n = 0;
}

static int pk_push(Pk *k, Pv *v) {
  if (!v) return 0;
  if (k->sp == k->scap) {
    const int32_t cap = k->scap ? 2 * k->scap : 64;
    Pv **s = (Pv **)realloc(k->stack, (size_t)cap * sizeof *s);
    if (!s) {
      k->err = "out of host memory";
      return 0;
    }
    k->stack = s;
    k->scap = cap;
  }
  k->stack[k->sp++] = v;
  return 1;
}

static Pv *pk_pop(Pk *k) {
  if (k->sp <= (k->mp ? k->marks[k->mp - 1] : 0)) {
    k->err = "stack underflow";
    return NULL;
  }
  return k->stack[--k->sp];
}

static int pk_need(Pk *k, size_t n) {
  if ((size_t)(k->end - k->p) < n) {
    k->err = "truncated pickle";
    return 0;
  }
  return 1;
}

static uint64_t rd_le(const unsigned char *p, int n) {
  uint64_t v = 0;
  for (int i = n - 1; i >= 0; i--) v = (v << 8) | p[i];
  return v;
}

static int pk_memo_put(Pk *k, int64_t idx, Pv *v) {
  if (idx < 0 || idx > (1 << 26)) {
    k->err = "memo index out of range";
    return 0;
  }
  if (idx >= k->memo_n) {
    int64_t n = k->memo_n ? k->memo_n : 64;
    while (n <= idx) n *= 2;
    Pv **m = (Pv **)realloc(k->memo, (size_t)n * sizeof *m);
    if (!m) {
      k->err = "out of host memory";
      return 0;
    }
    memset(m + k->memo_n, 0, (size_t)(n - k->memo_n) * sizeof *m);
    k->memo = m;
    k->memo_n = n;
  }
  k->memo[idx] = v;
  return 1;
}

static int pv_is(const Pv *v, const char *name) {
  return v && (v->k == PV_GLOBAL || v->k == PV_STR) && v->slen == strlen(name) && memcmp(v->s, name, v->slen) == 0;
}

/* callable(args) for the callables torch's pickles use */
static Pv *pk_call(Pk *k, Pv *fn, Pv *args) {
  if (fn->k == PV_GLOBAL && args->k == PV_TUPLE) {
    if (pv_is(fn, "_rebuild_tensor_v2") || pv_is(fn, "_rebuild_tensor")) {
      if (args->n < 4 || args->items[0]->k != PV_STORAGE || args->items[1]->k != PV_INT ||
          args->items[2]->k != PV_TUPLE || args->items[3]->k != PV_TUPLE ||
          args->items[2]->n != args->items[3]->n || args->items[2]->n > 8) {
        k->err = "unexpected _rebuild_tensor arguments";
        return NULL;
      }
      Pv *t = pv_new(k, PV_TENSOR);
      if (!t) return NULL;
      t->storage = args->items[0];
      t->offset = args->items[1]->i;
      t->ndim = args->items[2]->n;
      for (int32_t d = 0; d < t->ndim; d++) {
        if (args->items[2]->items[d]->k != PV_INT || args->items[3]->items[d]->k != PV_INT) {
          k->err = "non-integer tensor size or stride";
          return NULL;
        }
        t->size[d] = args->items[2]->items[d]->i;
        t->stride[d] = args->items[3]->items[d]->i;
      }
      return t;
    }
    if (pv_is(fn, "_rebuild_parameter") || pv_is(fn, "_rebuild_parameter_with_state"))
      return args->n >= 1 ? args->items[0] : pv_new(k, PV_NONE);
    if (pv_is(fn, "OrderedDict") || pv_is(fn, "dict")) return pv_new(k, PV_DICT);
  }
  return pv_new(k, PV_OTHER);
}

static Pv *pk_str(Pk *k, size_t n) {
  if (!pk_need(k, n)) return NULL;
  Pv *v = pv_new(k, PV_STR);
  if (!v) return NULL;
  v->s = (const char *)k->p;
  v->slen = n;
  k->p += n;
  return v;
}

static Pv *pk_tuple_from(Pk *k, int32_t from) {
  Pv *t = pv_new(k, PV_TUPLE);
  if (!t) return NULL;
  for (int32_t i = from; i < k->sp; i++)
    if (!pv_add(k, t, k->stack[i])) return NULL;
  k->sp = from;
  return t;
}

static int32_t pk_pop_mark(Pk *k) {
  if (k->mp == 0) {
    k->err = "no mark";
    return -1;
  }
  return k->marks[--k->mp];
}

/* one pickle (to its STOP) -> *out; 1 on success */
static int pk_run(Pk *k, Pv **out) {
  while (k->p < k->end) {
    const unsigned char op = *k->p++;
    Pv *v = NULL, *a = NULL, *b = NULL;
    int32_t m;
    switch (op) {
      case 0x80: /* PROTO */
        if (!pk_need(k, 1)) return 0;
        k->p += 1;
        break;
      case 0x95: /* FRAME */
        if (!pk_need(k, 8)) return 0;
        k->p += 8;
        break;
      case '(': /* MARK */
        if (k->mp == k->mcap) {
          const int32_t cap = k->mcap ? 2 * k->mcap : 16;
          int32_t *mk = (int32_t *)realloc(k->marks, (size_t)cap * sizeof *mk);
          if (!mk) {
            k->err = "out of host memory";
            return 0;
          }
          k->marks = mk;
          k->mcap = cap;
        }
        k->marks[k->mp++] = k->sp;
        break;
      case '}': if (!pk_push(k, pv_new(k, PV_DICT))) return 0; break;
      case ']': if (!pk_push(k, pv_new(k, PV_LIST))) return 0; break;
      case ')': if (!pk_push(k, pv_new(k, PV_TUPLE))) return 0; break;
      case 'N': if (!pk_push(k, pv_new(k, PV_NONE))) return 0; break;
      case 0x88:
      case 0x89: /* NEWTRUE / NEWFALSE */
        if (!(v = pv_new(k, PV_BOOL))) return 0;
        v->i = op == 0x88;
        if (!pk_push(k, v)) return 0;
        break;
      case 'J': case 'K': case 'M': { /* BININT, BININT1, BININT2 */
        const int n = op == 'J' ? 4 : op == 'K' ? 1 : 2;
        if (!pk_need(k, (size_t)n) || !(v = pv_new(k, PV_INT))) return 0;
        v->i = op == 'J' ? (int64_t)(int32_t)rd_le(k->p, 4) : (int64_t)rd_le(k->p, n);
        k->p += n;
        if (!pk_push(k, v)) return 0;
        break;
      }
      case 0x8a: { /* LONG1: n little-endian two's-complement bytes */
        if (!pk_need(k, 1)) return 0;
        const int n = *k->p++;
        if (!pk_need(k, (size_t)n)) return 0;
        if (n > 8) {   /* wider than 64 bits (the legacy format's magic number): kept as an opaque value */
          k->p += n;
          if (!pk_push(k, pv_new(k, PV_OTHER))) return 0;
          break;
        }
        if (!(v = pv_new(k, PV_INT))) return 0;
        uint64_t u = n ? rd_le(k->p, n) : 0;
        if (n && n < 8 && (k->p[n - 1] & 0x80)) u |= ~0ull << (8 * n);
        v->i = (int64_t)u;
        k->p += n;
        if (!pk_push(k, v)) return 0;
        break;
      }
      case 'G': { /* BINFLOAT: big-endian double */
        if (!pk_need(k, 8) || !(v = pv_new(k, PV_FLOAT))) return 0;
        uint64_t u = 0;
        for (int i = 0; i < 8; i++) u = (u << 8) | k->p[i];
        memcpy(&v->f, &u, 8);
        k->p += 8;
        if (!pk_push(k, v)) return 0;
        break;
      }
      case 'X': case 'T': case 'B': /* BINUNICODE, BINSTRING, BINBYTES: 4-byte length */
        if (!pk_need(k, 4)) return 0;
        k->p += 4;
        if (!pk_push(k, pk_str(k, (size_t)rd_le(k->p - 4, 4)))) return 0;
        break;
      case 0x8c: case 'U': case 'C': /* SHORT_BINUNICODE, SHORT_BINSTRING, SHORT_BINBYTES */
        if (!pk_need(k, 1)) return 0;
        k->p += 1;
        if (!pk_push(k, pk_str(k, k->p[-1]))) return 0;
        break;
      case 0x8d: case 0x8e: /* BINUNICODE8, BINBYTES8 */
        if (!pk_need(k, 8)) return 0;
        k->p += 8;
        if (!pk_push(k, pk_str(k, (size_t)rd_le(k->p - 8, 8)))) return 0;
        break;
      case 'c': { /* GLOBAL: module \n name \n */
        const unsigned char *nl1 = memchr(k->p, '\n', (size_t)(k->end - k->p));
        const unsigned char *nl2 = nl1 ? memchr(nl1 + 1, '\n', (size_t)(k->end - nl1 - 1)) : NULL;
        if (!nl2 || !(v = pv_new(k, PV_GLOBAL))) {
          if (!k->err) k->err = "malformed GLOBAL";
          return 0;
        }
        v->s2 = (const char *)k->p;
        v->s2len = (size_t)(nl1 - k->p);
        v->s = (const char *)nl1 + 1;
        v->slen = (size_t)(nl2 - nl1 - 1);
        k->p = nl2 + 1;
        if (!pk_push(k, v)) return 0;
        break;
      }
      case 0x93: /* STACK_GLOBAL */
        if (!(b = pk_pop(k)) || !(a = pk_pop(k)) || !(v = pv_new(k, PV_GLOBAL))) return 0;
        v->s2 = a->s;
        v->s2len = a->slen;
        v->s = b->s;
        v->slen = b->slen;
        if (!pk_push(k, v)) return 0;
        break;
      case 'q': /* BINPUT */
        if (!pk_need(k, 1) || k->sp == 0 || !pk_memo_put(k, *k->p, k->stack[k->sp - 1])) {
          if (!k->err) k->err = "BINPUT on an empty stack";
          return 0;
        }
        k->p += 1;
        break;
      case 'r': /* LONG_BINPUT */
        if (!pk_need(k, 4) || k->sp == 0 || !pk_memo_put(k, (int64_t)rd_le(k->p, 4), k->stack[k->sp - 1])) {
          if (!k->err) k->err = "LONG_BINPUT on an empty stack";
          return 0;
        }
        k->p += 4;
        break;
      case 0x94: { /* MEMOIZE */
        int64_t n = 0;
        while (n < k->memo_n && k->memo[n]) n++;
        if (k->sp == 0 || !pk_memo_put(k, n, k->stack[k->sp - 1])) {
          if (!k->err) k->err = "MEMOIZE on an empty stack";
          return 0;
        }
        break;
      }
      case 'h': case 'j': { /* BINGET, LONG_BINGET */
        const int n = op == 'h' ? 1 : 4;
        if (!pk_need(k, (size_t)n)) return 0;
        const int64_t idx = (int64_t)rd_le(k->p, n);
        k->p += n;
        if (idx >= k->memo_n || !k->memo[idx]) {
          k->err = "memo entry missing";
          return 0;
        }
        if (!pk_push(k, k->memo[idx])) return 0;
        break;
      }
      case 't': /* TUPLE */
        if ((m = pk_pop_mark(k)) < 0 || !pk_push(k, pk_tuple_from(k, m))) return 0;
        break;
      case 0x85: case 0x86: case 0x87: { /* TUPLE1..3 */
        const int32_t n = op - 0x84;
        if (k->sp - (k->mp ? k->marks[k->mp - 1] : 0) < n) {
          k->err = "stack underflow";
          return 0;
        }
        if (!pk_push(k, pk_tuple_from(k, k->sp - n))) return 0;
        break;
      }
      case 'a': /* APPEND */
        if (!(v = pk_pop(k)) || k->sp == 0 || !pv_add(k, k->stack[k->sp - 1], v)) return 0;
        break;
      case 'e': /* APPENDS */
        if ((m = pk_pop_mark(k)) < 1) {
          if (!k->err) k->err = "APPENDS without a list";
          return 0;
        }
        for (int32_t i = m; i < k->sp; i++)
          if (!pv_add(k, k->stack[m - 1], k->stack[i])) return 0;
        k->sp = m;
        break;
      case 's': /* SETITEM */
        if (!(b = pk_pop(k)) || !(a = pk_pop(k)) || k->sp == 0 || !pv_add(k, k->stack[k->sp - 1], a) ||
            !pv_add(k, k->stack[k->sp - 1], b))
          return 0;
        break;
      case 'u': /* SETITEMS */
        if ((m = pk_pop_mark(k)) < 1 || ((k->sp - m) & 1)) {
          if (!k->err) k->err = "SETITEMS without a dict";
          return 0;
        }
        for (int32_t i = m; i < k->sp; i++)
          if (!pv_add(k, k->stack[m - 1], k->stack[i])) return 0;
        k->sp = m;
        break;
      case 'R': case 0x81: /* REDUCE, NEWOBJ */
        if (!(b = pk_pop(k)) || !(a = pk_pop(k)) || !pk_push(k, pk_call(k, a, b))) return 0;
        break;
      case 'b': /* BUILD: the state of an object torch restores this way is not needed */
        if (!pk_pop(k)) return 0;
        break;
      case 'Q': { /* BINPERSID: ('storage', <type>, key, location, numel, ...) */
        if (!(a = pk_pop(k))) return 0;
        if (a->k != PV_TUPLE || a->n < 5 || a->items[1]->k != PV_GLOBAL || a->items[2]->k != PV_STR ||
            a->items[4]->k != PV_INT || !(v = pv_new(k, PV_STORAGE))) {
          if (!k->err) k->err = "unexpected persistent id";
          return 0;
        }
        v->s = a->items[1]->s;
        v->slen = a->items[1]->slen;
        v->s2 = a->items[2]->s;
        v->s2len = a->items[2]->slen;
        v->i = a->items[4]->i;
        if (!pk_push(k, v)) return 0;
        break;
      }
      case '0': /* POP */
        if (!pk_pop(k)) return 0;
        break;
      case '.': /* STOP */
        if (!(v = pk_pop(k))) return 0;
        *out = v;
        k->sp = 0;
        k->mp = 0;
        return 1;
      default:
        k->err = "unsupported pickle opcode";
        return 0;
    }
  }
  k->err = "pickle without STOP";
  return 0;
}

/* a new pickle in the same stream: memo and stack start empty, values stay */
static void pk_next(Pk *k) {
  if (k->memo) memset(k->memo, 0, (size_t)k->memo_n * sizeof *k->memo);
  k->sp = 0;
  k->mp = 0;
}

static const struct {
  const char *type, *tag;
  int size;
} kTorchTypes[] = {{"FloatStorage", "F32", 4}, {"DoubleStorage", "F64", 8}, {"HalfStorage", "F16", 2},
                   {"BFloat16Storage", "BF16", 2}, {"LongStorage", "I64", 8}, {"IntStorage", "I32", 4},
                   {"ShortStorage", "I16", 2}, {"CharStorage", "I8", 1}, {"ByteStorage", "U8", 1},
                   {"BoolStorage", "BOOL", 1}};

static int torch_type(const Pv *st, const char **tag) {
  for (size_t i = 0; i < sizeof kTorchTypes / sizeof kTorchTypes[0]; i++)
    if (st->slen == strlen(kTorchTypes[i].type) && memcmp(st->s, kTorchTypes[i].type, st->slen) == 0) {
      *tag = kTorchTypes[i].tag;
      return kTorchTypes[i].size;
    }
  *tag = "F32";
  return 4;
}

/* the stored (uncompressed) members of a zip archive, zip64 included */
typedef struct {
  const char *name;
  size_t nlen;
  const unsigned char *data;
  uint64_t size;
} ZipEnt;

static const char *zip_list(const unsigned char *p, size_t n, ZipEnt **out, int32_t *n_out) {
  *out = NULL;
  *n_out = 0;
  if (n < 22) return "not a zip archive";
  size_t eocd = 0;
  int found = 0;
  for (size_t i = n - 22 + 1; i-- > 0 && n - i <= 22 + 65535;)
    if (rd_le(p + i, 4) == 0x06054b50u) {
      eocd = i;
      found = 1;
      break;
    }
  if (!found) return "no end-of-central-directory record";
  uint64_t count = rd_le(p + eocd + 10, 2), cd_off = rd_le(p + eocd + 16, 4);
  if (count == 0xFFFF || cd_off == 0xFFFFFFFFu) {   /* zip64: the locator sits right before the record */
    if (eocd < 20 || rd_le(p + eocd - 20, 4) != 0x07064b50u) return "zip64 locator missing";
    const uint64_t z = rd_le(p + eocd - 20 + 8, 8);
    if (z + 56 > n || rd_le(p + z, 4) != 0x06064b50u) return "zip64 record missing";
    count = rd_le(p + z + 32, 8);
    cd_off = rd_le(p + z + 48, 8);
  }
  if (count > (1u << 24)) return "too many zip members";
  ZipEnt *e = (ZipEnt *)calloc((size_t)(count ? count : 1), sizeof *e);
  if (!e) return "out of host memory";
  uint64_t q = cd_off;
  for (uint64_t i = 0; i < count; i++) {
    if (q + 46 > n || rd_le(p + q, 4) != 0x02014b50u) {
      free(e);
      return "bad central directory";
    }
    const uint64_t method = rd_le(p + q + 10, 2), nl = rd_le(p + q + 28, 2), xl = rd_le(p + q + 30, 2),
                   cl = rd_le(p + q + 32, 2);
    uint64_t csize = rd_le(p + q + 20, 4), usize = rd_le(p + q + 24, 4), loff = rd_le(p + q + 42, 4);
    if (q + 46 + nl + xl > n) {
      free(e);
      return "bad central directory";
    }
    for (uint64_t x = q + 46 + nl; x + 4 <= q + 46 + nl + xl;) {   /* the zip64 extra field */
      const uint64_t id = rd_le(p + x, 2), len = rd_le(p + x + 2, 2);
      if (id == 1) {
        uint64_t y = x + 4;
        if (usize == 0xFFFFFFFFu && y + 8 <= x + 4 + len) usize = rd_le(p + y, 8), y += 8;
        if (csize == 0xFFFFFFFFu && y + 8 <= x + 4 + len) csize = rd_le(p + y, 8), y += 8;
        if (loff == 0xFFFFFFFFu && y + 8 <= x + 4 + len) loff = rd_le(p + y, 8);
      }
      x += 4 + len;
    }
    if (loff + 30 > n || rd_le(p + loff, 4) != 0x04034b50u) {
      free(e);
      return "bad local header";
    }
    const uint64_t data = loff + 30 + rd_le(p + loff + 26, 2) + rd_le(p + loff + 28, 2);
    if (method != 0 || csize != usize) {
      free(e);
      return "compressed zip member (torch.save stores them uncompressed)";
    }
    if (data + csize > n) {
      free(e);
      return "zip member past the end of the file";
    }
    e[i].name = (const char *)p + q + 46;
    e[i].nlen = (size_t)nl;
    e[i].data = p + data;
    e[i].size = csize;
    q += 46 + nl + xl + cl;
  }
  *out = e;
  *n_out = (int32_t)count;
  return NULL;
}

/* one tensor's elements, row-major, into a fresh buffer (entry e) */
static int torch_tensor(const Pv *t, const unsigned char *sdata, uint64_t slen, Sm100TensorEntry *e) {
  const char *tag;
  const int isz = torch_type(t->storage, &tag);
  snprintf(e->dtype, sizeof e->dtype, "%s", tag);
  e->ndim = t->ndim;
  /* sizes, strides and the offset bounded so that no product below overflows;
     a contiguous or permuted tensor has no more elements than its storage */
  const int64_t kLim = (int64_t)1 << 40;
  int64_t numel = 1, maxoff = t->offset;
  for (int32_t d = 0; d < t->ndim; d++) {
    if (t->size[d] < 0 || t->size[d] > kLim || t->stride[d] < 0 || t->stride[d] > kLim)
      return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: size or stride out of range", e->name);
    e->shape[d] = t->size[d];
    if (t->size[d] == 0) numel = 0;
    else if (numel > kLim / t->size[d]) numel = kLim + 1;   /* saturated: refused below */
    else numel *= t->size[d];
  }
  const int64_t cap = (int64_t)(slen / (uint64_t)isz);   /* the storage's elements */
  if (t->offset < 0 || t->offset > kLim || numel > cap)
    return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: elements past its storage", e->name);
  for (int32_t d = 0; d < t->ndim && numel; d++) {
    if (t->size[d] > 1 && t->stride[d] > (cap - maxoff) / (t->size[d] - 1))
      return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: elements past its storage", e->name);
    maxoff += (t->size[d] - 1) * t->stride[d];
  }
  e->nbytes = (uint64_t)numel * (uint64_t)isz;
  if (numel == 0) return upload(e, NULL);
  if (maxoff >= cap)
    return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: elements past its storage", e->name);
  /* contiguous: the strides of a row-major layout (dimensions of size 1 aside) */
  int contiguous = 1;
  int64_t acc = 1;
  for (int32_t d = t->ndim - 1; d >= 0; d--) {
    if (t->size[d] != 1 && t->stride[d] != acc) contiguous = 0;
    acc *= t->size[d];
  }
  if (contiguous) return upload(e, sdata + (uint64_t)t->offset * (uint64_t)isz);
  /* otherwise a permutation of a row-major layout, as the reference accepts:
     the strides of the dimensions of size > 1, sorted descending, are the
     row-major strides of their sizes in that order */
  int32_t idx[8], n = 0;
  for (int32_t d = 0; d < t->ndim; d++)
    if (t->size[d] != 1) idx[n++] = d;
  for (int32_t a = 1; a < n; a++)
    for (int32_t b = a; b > 0 && t->stride[idx[b]] > t->stride[idx[b - 1]]; b--) {
      const int32_t s = idx[b];
      idx[b] = idx[b - 1];
      idx[b - 1] = s;
    }
  acc = 1;
  for (int32_t a = n - 1; a >= 0; a--) {
    if (t->stride[idx[a]] != acc)
      return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: nonpermutable strides", e->name);
    acc *= t->size[idx[a]];
  }
  unsigned char *tmp = (unsigned char *)malloc((size_t)e->nbytes);
  if (!tmp) return sm100_set_error(SM100_ERR_OOM, "torch_load: %s: host memory", e->name);
  int64_t pos[8] = {0};
  for (int64_t i = 0; i < numel; i++) {
    int64_t off = t->offset;
    for (int32_t d = 0; d < t->ndim; d++) off += pos[d] * t->stride[d];
    memcpy(tmp + (size_t)i * (size_t)isz, sdata + (size_t)off * (size_t)isz, (size_t)isz);
    for (int32_t d = t->ndim - 1; d >= 0; d--) {
      if (++pos[d] < t->size[d]) break;
      pos[d] = 0;
    }
  }
  const int rc = upload(e, tmp);
  free(tmp);
  return rc;
}

typedef struct {
  const char *key;
  size_t klen;
  const unsigned char *data;
  uint64_t size;
} TorchStorage;

/* the top-level tensors of the state dict `root` into entries */
static int torch_entries(const char *path, const Pv *root, const TorchStorage *st, int32_t n_st,
                         Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out) {
  if (!root || root->k != PV_DICT) return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: no state dict", path);
  int32_t n = 0;
  for (int32_t i = 0; i + 1 < root->n; i += 2) {
    const Pv *key = root->items[i], *val = root->items[i + 1];
    if (key->k != PV_STR || val->k != PV_TENSOR) continue;   /* as the reference: tensors only */
    if (n == max_entries) {
      drop_all(entries, n);
      return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: more than %d tensors", path, max_entries);
    }
    Sm100TensorEntry *e = &entries[n];
    memset(e, 0, sizeof *e);
    if (key->slen >= sizeof e->name || val->ndim > 8) {
      drop_all(entries, n);
      return sm100_set_error(SM100_ERR_ARG, "torch_load: %s: tensor name or rank too large", path);
    }
    memcpy(e->name, key->s, key->slen);
    const TorchStorage *s = NULL;
    for (int32_t j = 0; j < n_st && !s; j++)
      if (st[j].klen == val->storage->s2len && memcmp(st[j].key, val->storage->s2, st[j].klen) == 0) s = &st[j];
    const int rc = s ? torch_tensor(val, s->data, s->size, e)
                     : sm100_set_error(SM100_ERR_ARG, "torch_load: %s: storage of %s missing", path, e->name);
    if (rc != SM100_OK) {
      if (e->buf_id) sm100_buf_free(e->buf_id);
      drop_all(entries, n);
      return rc;
    }
    n++;
  }
  *n_out = n;
  return SM100_OK;
}

int sm100_torch_load(const char *path, Sm100TensorEntry *entries, int32_t max_entries, int32_t *n_out) {
  if (!path || !entries || max_entries < 1 || !n_out) return sm100_set_error(SM100_ERR_ARG, "torch_load: bad arguments");
  *n_out = 0;
  Map mp;
  int rc = map_open(path, &mp);
  if (rc != SM100_OK) return rc;
  Pk k;
  memset(&k, 0, sizeof k);
  Pv *root = NULL;
  TorchStorage *st = NULL;
  int32_t n_st = 0;
  ZipEnt *ze = NULL;
  int32_t nz = 0;
  const char *err = NULL;
  if (mp.n >= 4 && rd_le(mp.p, 4) == 0x04034b50u) {
    /* zip: <archive>/data.pkl and <archive>/data/<key> */
    err = zip_list(mp.p, mp.n, &ze, &nz);
    const ZipEnt *pkl = NULL;
    for (int32_t i = 0; !err && i < nz && !pkl; i++)
      if (ze[i].nlen >= 8 && memcmp(ze[i].name + ze[i].nlen - 8, "data.pkl", 8) == 0) pkl = &ze[i];
    if (!err && !pkl) err = "no data.pkl member";
    if (!err) {
      const char *slash = memchr(pkl->name, '/', pkl->nlen);
      const size_t blen = slash ? (size_t)(slash - pkl->name) : 0;
      st = (TorchStorage *)calloc((size_t)(nz ? nz : 1), sizeof *st);
      if (!st) err = "out of host memory";
      for (int32_t i = 0; !err && i < nz; i++) {
        const ZipEnt *z = &ze[i];
        /* <base>/data/<key> */
        if (z->nlen > blen + 6 && memcmp(z->name, pkl->name, blen) == 0 && memcmp(z->name + blen, "/data/", 6) == 0 &&
            !memchr(z->name + blen + 6, '/', z->nlen - blen - 6)) {
          st[n_st].key = z->name + blen + 6;
          st[n_st].klen = z->nlen - blen - 6;
          st[n_st].data = z->data;
          st[n_st].size = z->size;
          n_st++;
        }
      }
      if (!err) {
        k.p = pkl->data;
        k.end = pkl->data + pkl->size;
        if (!pk_run(&k, &root)) err = k.err ? k.err : "bad pickle";
      }
    }
  } else {
    /* legacy: magic, protocol, sys_info, the state, the storage keys, then
       each storage as an 8-byte element count and its elements */
    Pv *skip = NULL, *keys = NULL;
    k.p = mp.p;
    k.end = mp.p + mp.n;
    for (int i = 0; i < 3 && !err; i++) {
      if (!pk_run(&k, &skip)) err = k.err ? k.err : "bad pickle";
      pk_next(&k);
    }
    if (!err && !pk_run(&k, &root)) err = k.err ? k.err : "bad pickle";
    pk_next(&k);
    if (!err && !pk_run(&k, &keys)) err = k.err ? k.err : "bad pickle";
    if (!err && keys->k != PV_LIST) err = "no storage key list";
    if (!err) {
      st = (TorchStorage *)calloc((size_t)(keys->n ? keys->n : 1), sizeof *st);
      if (!st) err = "out of host memory";
    }
    for (int32_t i = 0; !err && i < keys->n; i++) {
      const Pv *key = keys->items[i];
      const Pv *sv = NULL;   /* the storage of that key, for its element size */
      for (const Pv *v = k.allocs; v && !sv; v = v->next_alloc)
        if (v->k == PV_STORAGE && key->k == PV_STR && v->s2len == key->slen && memcmp(v->s2, key->s, key->slen) == 0)
          sv = v;
      if (!sv) {
        err = "a stored storage that no tensor uses";
        break;
      }
      const char *tag;
      const uint64_t isz = (uint64_t)torch_type(sv, &tag);
      if (!pk_need(&k, 8)) {
        err = "truncated storage";
        break;
      }
      const uint64_t count = rd_le(k.p, 8);
      k.p += 8;
      if (count > (uint64_t)(k.end - k.p) / isz) {
        err = "truncated storage";
        break;
      }
      st[n_st].key = key->s;
      st[n_st].klen = key->slen;
      st[n_st].data = k.p;
      st[n_st].size = count * isz;
      n_st++;
      k.p += count * isz;
    }
  }
  if (err) rc = sm100_set_error(SM100_ERR_ARG, "torch_load: %s: %s", path, err);
  else rc = torch_entries(path, root, st, n_st, entries, max_entries, n_out);
  pk_free(&k);
  free(st);
  free(ze);
  map_close(&mp);
  return rc;
}
