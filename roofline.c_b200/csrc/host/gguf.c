/* gguf.c -- zero-copy GGUF v2/v3 reader; contract of roofline.c
 * src/gguf.h:146-178 and the validation behaviour of src/gguf.c:295-424
 * (bounds-checked reads, absurd-count rejection, power-of-two alignment,
 * per-tensor payload bounds, big-endian magic named), re-implemented here.
 *
 * The type table (block elements / bytes) is ggml's on-disk geometry; it has
 * to agree with the reference's (src/gguf.c:72-96) entry for entry, because
 * it decides every tensor's byte size. The IQ and TQ families stay
 * unsupported, as there.
 */
#define _DEFAULT_SOURCE
#include "gguf.h"

#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------ type table */

typedef struct { const char *name; uint32_t blck; uint32_t bytes; } tinfo_t;

static const tinfo_t *tinfo(ggml_type_t t)
{
    static const tinfo_t table[GGML_TYPE_MAX] = {
        [GGML_TYPE_F32] = { "F32", 1, 4 },      [GGML_TYPE_F16] = { "F16", 1, 2 },
        [GGML_TYPE_Q4_0] = { "Q4_0", 32, 18 },  [GGML_TYPE_Q4_1] = { "Q4_1", 32, 20 },
        [GGML_TYPE_Q5_0] = { "Q5_0", 32, 22 },  [GGML_TYPE_Q5_1] = { "Q5_1", 32, 24 },
        [GGML_TYPE_Q8_0] = { "Q8_0", 32, 34 },  [GGML_TYPE_Q8_1] = { "Q8_1", 32, 36 },
        [GGML_TYPE_Q2_K] = { "Q2_K", 256, 84 }, [GGML_TYPE_Q3_K] = { "Q3_K", 256, 110 },
        [GGML_TYPE_Q4_K] = { "Q4_K", 256, 144 },[GGML_TYPE_Q5_K] = { "Q5_K", 256, 176 },
        [GGML_TYPE_Q6_K] = { "Q6_K", 256, 210 },[GGML_TYPE_Q8_K] = { "Q8_K", 256, 292 },
        [GGML_TYPE_I8] = { "I8", 1, 1 },        [GGML_TYPE_I16] = { "I16", 1, 2 },
        [GGML_TYPE_I32] = { "I32", 1, 4 },      [GGML_TYPE_I64] = { "I64", 1, 8 },
        [GGML_TYPE_F64] = { "F64", 1, 8 },      [GGML_TYPE_BF16] = { "BF16", 1, 2 },
    };
    if ((unsigned)t >= GGML_TYPE_MAX || table[t].name == NULL) return NULL;
    return &table[t];
}

const char *ggml_type_name(ggml_type_t t) { const tinfo_t *i = tinfo(t); return i ? i->name : "UNSUPPORTED"; }
uint32_t ggml_blck_size(ggml_type_t t)    { const tinfo_t *i = tinfo(t); return i ? i->blck : 0; }
size_t ggml_type_size(ggml_type_t t)      { const tinfo_t *i = tinfo(t); return i ? i->bytes : 0; }
bool ggml_type_supported(ggml_type_t t)   { return tinfo(t) != NULL; }

const char *gguf_type_name(gguf_type_t t)
{
    static const char *const names[GGUF_T_COUNT] = {
        "uint8", "int8", "uint16", "int16", "uint32", "int32", "float32",
        "bool", "string", "array", "uint64", "int64", "float64" };
    return (unsigned)t < GGUF_T_COUNT ? names[t] : "?";
}

/* width in bytes of a fixed-size metadata value, 0 for string / array */
static size_t scalar_width(uint32_t t)
{
    switch (t) {
    case GGUF_T_UINT8: case GGUF_T_INT8: case GGUF_T_BOOL: return 1;
    case GGUF_T_UINT16: case GGUF_T_INT16: return 2;
    case GGUF_T_UINT32: case GGUF_T_INT32: case GGUF_T_FLOAT32: return 4;
    case GGUF_T_UINT64: case GGUF_T_INT64: case GGUF_T_FLOAT64: return 8;
    default: return 0;
    }
}

/* --------------------------------------------------------------- strings */

char *gguf_str_cstr(char *buf, size_t buflen, gguf_str_t s)
{
    if (buflen == 0) return buf;
    size_t n = (s.ptr && s.len) ? (s.len < buflen - 1 ? (size_t)s.len : buflen - 1) : 0;
    if (n) memcpy(buf, s.ptr, n);
    buf[n] = '\0';
    return buf;
}

bool gguf_str_eq(gguf_str_t s, const char *cstr)
{
    const size_t n = strlen(cstr);
    return s.ptr && s.len == (uint64_t)n && memcmp(s.ptr, cstr, n) == 0;
}

/* ---------------------------------------------------------------- reader */

typedef struct {
    const unsigned char *at, *end;
    bool bad;                      /* sticky: any short read poisons the rest */
} span_t;

static size_t left(const span_t *s) { return (size_t)(s->end - s->at); }

static const unsigned char *take(span_t *s, size_t n)
{
    if (s->bad || n > left(s)) { s->bad = true; return NULL; }
    const unsigned char *p = s->at;
    s->at += n;
    return p;
}

static uint32_t take_u32(span_t *s) { uint32_t v = 0; const void *p = take(s, 4); if (p) memcpy(&v, p, 4); return v; }
static uint64_t take_u64(span_t *s) { uint64_t v = 0; const void *p = take(s, 8); if (p) memcpy(&v, p, 8); return v; }

static gguf_str_t take_str(span_t *s)
{
    gguf_str_t r = { NULL, 0 };
    const uint64_t n = take_u64(s);
    if (s->bad) return r;
    if (n > left(s)) { s->bad = true; return r; }   /* corrupt length */
    r.ptr = (const char *)take(s, (size_t)n);
    r.len = n;
    return r;
}

__attribute__((format(printf, 2, 3)))
static bool fail(gguf_t *g, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g->err, sizeof g->err, fmt, ap);
    va_end(ap);
    return false;
}

/* Unmap and fail, keeping the message already written into g->err. */
static bool close_keep_err(gguf_t *g)
{
    char keep[sizeof g->err];
    memcpy(keep, g->err, sizeof keep);
    gguf_close(g);
    memcpy(g->err, keep, sizeof keep);
    return false;
}

static bool read_kv(gguf_t *g, span_t *s, gguf_kv_t *kv, arena_t *a)
{
    kv->key = take_str(s);
    if (s->bad) return fail(g, "truncated while reading a metadata key");
    const uint32_t ty = take_u32(s);
    if (s->bad) return fail(g, "truncated while reading a metadata type");
    if (ty >= GGUF_T_COUNT) return fail(g, "unknown metadata value type %u", ty);
    kv->type = (gguf_type_t)ty;

    if (ty == GGUF_T_STRING) {
        kv->v.str = take_str(s);
        return s->bad ? fail(g, "truncated string value") : true;
    }
    if (ty != GGUF_T_ARRAY) {
        const unsigned char *p = take(s, scalar_width(ty));
        if (!p) return fail(g, "truncated scalar value");
        memcpy(&kv->v, p, scalar_width(ty));
        return true;
    }

    const uint32_t et = take_u32(s);
    const uint64_t n = take_u64(s);
    if (s->bad) return fail(g, "truncated array header");
    if (et >= GGUF_T_COUNT) return fail(g, "unknown array element type %u", et);
    if (et == GGUF_T_ARRAY) return fail(g, "nested arrays are not supported");
    kv->v.arr.type = (gguf_type_t)et;
    kv->v.arr.len = n;
    kv->v.arr.data = NULL;
    kv->v.arr.strs = NULL;

    if (et == GGUF_T_STRING) {
        /* each element needs at least its 8-byte length */
        if (n > left(s) / 8u)
            return fail(g, "array of %llu strings cannot fit in the file", (unsigned long long)n);
        gguf_str_t *idx = NULL;
        if (n) {
            idx = (gguf_str_t *)arena_alloc(a, (size_t)n * sizeof *idx, _Alignof(gguf_str_t));
            if (!idx) return fail(g, "arena exhausted indexing %llu strings", (unsigned long long)n);
        }
        for (uint64_t i = 0; i < n; i++) {
            idx[i] = take_str(s);
            if (s->bad) return fail(g, "truncated at string %llu of %llu",
                                    (unsigned long long)i, (unsigned long long)n);
        }
        kv->v.arr.strs = idx;
        return true;
    }
    const size_t w = scalar_width(et);
    if (w == 0) return fail(g, "array of unsized type %u", et);
    if (n > left(s) / w)
        return fail(g, "array of %llu x %zuB overruns the file", (unsigned long long)n, w);
    kv->v.arr.data = take(s, (size_t)n * w);
    return true;
}

static bool read_tensor(gguf_t *g, span_t *s, gguf_tensor_t *t)
{
    t->name = take_str(s);
    if (s->bad) return fail(g, "truncated tensor name");
    t->n_dims = take_u32(s);
    if (s->bad) return fail(g, "truncated tensor rank");
    if (t->n_dims < 1 || t->n_dims > GGUF_MAX_DIMS)
        return fail(g, "tensor rank %u out of range 1..%d", t->n_dims, GGUF_MAX_DIMS);
    t->n_elem = 1;
    for (int i = 0; i < GGUF_MAX_DIMS; i++) t->dims[i] = 1;
    for (uint32_t i = 0; i < t->n_dims; i++) {
        const uint64_t d = take_u64(s);
        if (s->bad) return fail(g, "truncated tensor dimensions");
        if (d && t->n_elem > UINT64_MAX / d) return fail(g, "tensor element count overflows");
        t->dims[i] = d;
        t->n_elem *= d;
    }
    t->type = (ggml_type_t)take_u32(s);
    if (s->bad) return fail(g, "truncated tensor type");
    t->offset = take_u64(s);
    if (s->bad) return fail(g, "truncated tensor offset");
    t->data = NULL;
    t->nbytes = 0;

    const tinfo_t *ti = tinfo(t->type);
    if (!ti) return true;   /* listed, but unreadable: nbytes stays 0 */
    if (t->n_elem % ti->blck)
        return fail(g, "%.*s: %llu elements is not a multiple of the %s block size %u",
                    (int)t->name.len, t->name.ptr, (unsigned long long)t->n_elem, ti->name, ti->blck);
    t->nbytes = t->n_elem / ti->blck * ti->bytes;
    return true;
}

bool gguf_open(gguf_t *out, const char *path, arena_t *a)
{
    memset(out, 0, sizeof *out);
    out->fd = -1;

    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(out, "cannot open %s: %s", path, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        const int e = errno;
        close(fd);
        return fail(out, "cannot stat %s: %s", path, strerror(e));
    }
    if (st.st_size < 24) {
        close(fd);
        return fail(out, "%s is too small to be a GGUF file (%lld bytes)", path, (long long)st.st_size);
    }
    const size_t size = (size_t)st.st_size;
    void *map = mmap(NULL, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
        const int e = errno;
        close(fd);
        return fail(out, "cannot mmap %s: %s", path, strerror(e));
    }
    out->map = (const unsigned char *)map;
    out->map_size = size;
    out->fd = fd;

    span_t s = { out->map, out->map + size, false };
    const uint32_t magic = take_u32(&s);
    if (magic != GGUF_MAGIC) {
        fail(out, magic == 0x47475546u ? "%s is a big-endian GGUF; this reader is little-endian only"
                                       : "%s is not a GGUF file (magic 0x%08x)", path, magic);
        return close_keep_err(out);
    }
    out->version = take_u32(&s);
    if (out->version != 2 && out->version != 3) {
        fail(out, "unsupported GGUF version %u (expected 2 or 3)", out->version);
        return close_keep_err(out);
    }
    out->n_tensors = take_u64(&s);
    out->n_kv = take_u64(&s);
    if (s.bad) { fail(out, "truncated GGUF header"); return close_keep_err(out); }

    /* a KV takes >= 12 bytes on disk and a tensor info >= 24 */
    if (out->n_kv > size / 12u || out->n_tensors > size / 24u) {
        fail(out, "header claims %llu KVs and %llu tensors, impossible in %zu bytes",
             (unsigned long long)out->n_kv, (unsigned long long)out->n_tensors, size);
        return close_keep_err(out);
    }

    if (out->n_kv) {
        out->kv = (gguf_kv_t *)arena_alloc(a, (size_t)out->n_kv * sizeof *out->kv, _Alignof(gguf_kv_t));
        if (!out->kv) { fail(out, "arena exhausted (kv)"); return close_keep_err(out); }
    }
    for (uint64_t i = 0; i < out->n_kv; i++)
        if (!read_kv(out, &s, &out->kv[i], a)) return close_keep_err(out);

    uint32_t align = GGUF_DEFAULT_ALIGNMENT;
    const gguf_kv_t *ka = gguf_find(out, "general.alignment");
    if (ka && ka->type == GGUF_T_UINT32) align = ka->v.u32;
    if (align == 0 || (align & (align - 1))) {
        fail(out, "general.alignment %u is not a power of two", align);
        return close_keep_err(out);
    }
    out->alignment = align;

    if (out->n_tensors) {
        out->tensors = (gguf_tensor_t *)arena_alloc(a, (size_t)out->n_tensors * sizeof *out->tensors,
                                                    _Alignof(gguf_tensor_t));
        if (!out->tensors) { fail(out, "arena exhausted (tensors)"); return close_keep_err(out); }
    }
    for (uint64_t i = 0; i < out->n_tensors; i++)
        if (!read_tensor(out, &s, &out->tensors[i])) return close_keep_err(out);

    const size_t header = (size_t)(s.at - out->map);
    const size_t data_at = (header + align - 1) & ~((size_t)align - 1);
    if (data_at > size) { fail(out, "tensor data section starts past end of file"); return close_keep_err(out); }
    out->data = out->map + data_at;
    out->data_size = size - data_at;

    for (uint64_t i = 0; i < out->n_tensors; i++) {
        gguf_tensor_t *t = &out->tensors[i];
        if (t->nbytes == 0) continue;
        if (t->offset > out->data_size || t->nbytes > out->data_size - t->offset) {
            char nm[128];
            gguf_str_cstr(nm, sizeof nm, t->name);
            fail(out, "tensor '%s' at +%llu (%llu bytes) overruns the %zu-byte data section",
                 nm, (unsigned long long)t->offset, (unsigned long long)t->nbytes, out->data_size);
            return close_keep_err(out);
        }
        t->data = out->data + t->offset;
    }
    return true;
}

void gguf_close(gguf_t *g)
{
    if (!g) return;
    if (g->map) munmap((void *)g->map, g->map_size);
    if (g->fd >= 0) close(g->fd);
    g->map = NULL;
    g->data = NULL;
    g->fd = -1;
    g->map_size = 0;
    g->data_size = 0;
}

/* ---------------------------------------------------------------- lookup */

const gguf_kv_t *gguf_find(const gguf_t *g, const char *key)
{
    for (uint64_t i = 0; i < g->n_kv; i++)
        if (gguf_str_eq(g->kv[i].key, key)) return &g->kv[i];
    return NULL;
}

bool gguf_get_u64(const gguf_t *g, const char *key, uint64_t *out)
{
    const gguf_kv_t *kv = gguf_find(g, key);
    if (!kv) return false;
    int64_t sv;
    switch (kv->type) {
    case GGUF_T_UINT8:  *out = kv->v.u8;  return true;
    case GGUF_T_UINT16: *out = kv->v.u16; return true;
    case GGUF_T_UINT32: *out = kv->v.u32; return true;
    case GGUF_T_UINT64: *out = kv->v.u64; return true;
    case GGUF_T_BOOL:   *out = kv->v.b;   return true;
    case GGUF_T_INT8:   sv = kv->v.i8;  break;
    case GGUF_T_INT16:  sv = kv->v.i16; break;
    case GGUF_T_INT32:  sv = kv->v.i32; break;
    case GGUF_T_INT64:  sv = kv->v.i64; break;
    default: return false;
    }
    if (sv < 0) return false;      /* a negative count is not a u64 */
    *out = (uint64_t)sv;
    return true;
}

bool gguf_get_i64(const gguf_t *g, const char *key, int64_t *out)
{
    const gguf_kv_t *kv = gguf_find(g, key);
    if (!kv) return false;
    switch (kv->type) {
    case GGUF_T_UINT8:  *out = kv->v.u8;  return true;
    case GGUF_T_UINT16: *out = kv->v.u16; return true;
    case GGUF_T_UINT32: *out = kv->v.u32; return true;
    case GGUF_T_UINT64:
        if (kv->v.u64 > (uint64_t)INT64_MAX) return false;
        *out = (int64_t)kv->v.u64; return true;
    case GGUF_T_INT8:   *out = kv->v.i8;  return true;
    case GGUF_T_INT16:  *out = kv->v.i16; return true;
    case GGUF_T_INT32:  *out = kv->v.i32; return true;
    case GGUF_T_INT64:  *out = kv->v.i64; return true;
    case GGUF_T_BOOL:   *out = kv->v.b;   return true;
    default: return false;
    }
}

bool gguf_get_f32(const gguf_t *g, const char *key, float *out)
{
    const gguf_kv_t *kv = gguf_find(g, key);
    if (!kv) return false;
    if (kv->type == GGUF_T_FLOAT32) { *out = kv->v.f32; return true; }
    if (kv->type == GGUF_T_FLOAT64) { *out = (float)kv->v.f64; return true; }
    return false;
}

bool gguf_get_str(const gguf_t *g, const char *key, gguf_str_t *out)
{
    const gguf_kv_t *kv = gguf_find(g, key);
    if (!kv || kv->type != GGUF_T_STRING) return false;
    *out = kv->v.str;
    return true;
}

uint64_t gguf_u64_or(const gguf_t *g, const char *key, uint64_t fallback)
{
    uint64_t v;
    return gguf_get_u64(g, key, &v) ? v : fallback;
}

float gguf_f32_or(const gguf_t *g, const char *key, float fallback)
{
    float v;
    return gguf_get_f32(g, key, &v) ? v : fallback;
}

const gguf_tensor_t *gguf_tensor(const gguf_t *g, const char *name)
{
    for (uint64_t i = 0; i < g->n_tensors; i++)
        if (gguf_str_eq(g->tensors[i].name, name)) return &g->tensors[i];
    return NULL;
}
