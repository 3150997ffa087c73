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
