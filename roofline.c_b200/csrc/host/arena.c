/* arena.c -- host bump allocator; contract of roofline.c src/arena.h:37-69
 * (behaviour restated from src/arena.c:23-135: page-rounded anonymous
 * NORESERVE mapping, overflow-safe bump, LIFO release, peak tracking). */
#define _DEFAULT_SOURCE
#include "arena.h"

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <unistd.h>

static size_t round_up(size_t x, size_t a) { return (x + a - 1) & ~(a - 1); }
static bool pow2(size_t x) { return x && !(x & (x - 1)); }

static size_t os_page(void)
{
    static size_t cached;
    if (!cached) {
        long p = sysconf(_SC_PAGESIZE);
        cached = p > 0 ? (size_t)p : 4096u;
    }
    return cached;
}

arena_t arena_create(size_t cap, const char *name)
{
    arena_t a = { NULL, 0, 0, 0, name ? name : "arena" };
    if (cap == 0) return a;
    const size_t bytes = round_up(cap, os_page());
    if (bytes < cap) return a;                       /* wrapped */
    int flags = MAP_PRIVATE | MAP_ANONYMOUS;
#ifdef MAP_NORESERVE
    flags |= MAP_NORESERVE;
#endif
    void *p = mmap(NULL, bytes, PROT_READ | PROT_WRITE, flags, -1, 0);
    if (p == MAP_FAILED) return a;
    a.base = (unsigned char *)p;
    a.cap = bytes;
    return a;
}

void arena_destroy(arena_t *a)
{
    if (!a || !a->base) return;
    munmap(a->base, a->cap);
    a->base = NULL;
    a->cap = a->used = a->peak = 0;
}

bool arena_ok(const arena_t *a) { return a && a->base; }

void *arena_alloc(arena_t *a, size_t size, size_t align)
{
    if (!arena_ok(a)) return NULL;
    if (align == 0) align = ARENA_DEFAULT_ALIGN;
    if (!pow2(align)) return NULL;
    const size_t start = round_up(a->used, align);
    if (start < a->used || start > a->cap || size > a->cap - start) return NULL;
    a->used = start + size;
    if (a->used > a->peak) a->peak = a->used;
    return a->base + start;
}

void *arena_alloc_or_die(arena_t *a, size_t size, size_t align)
{
    void *p = arena_alloc(a, size, align);
    if (p) return p;
    char w[32], f[32], c[32];
    fprintf(stderr, "tc: arena '%s' exhausted: wanted %s, %s free of %s\n",
            (a && a->name) ? a->name : "?", arena_fmt_bytes(w, sizeof w, size),
            arena_fmt_bytes(f, sizeof f, arena_avail(a)),
            arena_fmt_bytes(c, sizeof c, a ? a->cap : 0));
    abort();
}

void *arena_calloc(arena_t *a, size_t count, size_t size, size_t align)
{
    if (count && size > SIZE_MAX / count) return NULL;
    const size_t total = count * size;
    void *p = arena_alloc(a, total, align);
    if (p && total != 0) memset(p, 0, total);
    return p;
}

void *arena_memdup(arena_t *a, const void *src, size_t n, size_t align)
{
    void *p = arena_alloc(a, n, align);
    if (p && n) memcpy(p, src, n);
    return p;
}

size_t arena_mark(const arena_t *a) { return a ? a->used : 0; }

void arena_release(arena_t *a, size_t mark)
{
    if (a && mark <= a->used) a->used = mark;
}

void arena_reset(arena_t *a)
{
    if (a) a->used = 0;
}

size_t arena_used(const arena_t *a) { return a ? a->used : 0; }
size_t arena_peak(const arena_t *a) { return a ? a->peak : 0; }
size_t arena_avail(const arena_t *a) { return a ? a->cap - a->used : 0; }

char *arena_fmt_bytes(char *buf, size_t buflen, size_t bytes)
{
    static const char *const units[] = { "B", "KiB", "MiB", "GiB", "TiB" };
    double v = (double)bytes;
    unsigned u = 0;
    for (; v >= 1024.0 && u < 4; u++) v /= 1024.0;
    if (u == 0) snprintf(buf, buflen, "%zu B", bytes);
    else snprintf(buf, buflen, "%.2f %s", v, units[u]);
    return buf;
}
