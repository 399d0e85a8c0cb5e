/* arena.h -- host bump allocator (drop-in for roofline.c src/arena.h:37-69).
 *
 * Same type, names, arguments and failure behaviour as the reference:
 * a reservation made once (anonymous mmap, committed lazily by the kernel),
 * a bump offset, LIFO mark/release, no per-object free. The library uses it
 * for GGUF descriptors and the model's host-side tables; device memory has
 * its own arena with the same discipline (tcg_arena_* in tcg.h).
 */
#ifndef TC_ARENA_H
#define TC_ARENA_H

#include <stdbool.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ARENA_DEFAULT_ALIGN 64u

typedef struct {
    unsigned char *base;   /* start of the reservation, NULL if none        */
    size_t cap;            /* reserved bytes (page-rounded)                 */
    size_t used;           /* current bump offset                          */
    size_t peak;           /* largest `used` ever reached                   */
    const char *name;      /* for diagnostics                               */
} arena_t;

/* src/arena.h:35-39. base == NULL on failure (and for cap == 0). */
arena_t arena_create(size_t cap, const char *name);
void    arena_destroy(arena_t *a);
bool    arena_ok(const arena_t *a);

/* src/arena.h:41-53. NULL when exhausted or align is not a power of two
 * (align 0 means ARENA_DEFAULT_ALIGN). The _or_die form aborts with a
 * message naming the arena instead of returning NULL. */
void   *arena_alloc(arena_t *a, size_t size, size_t align);
void   *arena_alloc_or_die(arena_t *a, size_t size, size_t align);
void   *arena_calloc(arena_t *a, size_t count, size_t size, size_t align);
void   *arena_memdup(arena_t *a, const void *src, size_t n, size_t align);

/* src/arena.h:55-63 */
size_t  arena_mark(const arena_t *a);
void    arena_release(arena_t *a, size_t mark);
void    arena_reset(arena_t *a);
size_t  arena_used(const arena_t *a);
size_t  arena_peak(const arena_t *a);
size_t  arena_avail(const arena_t *a);

/* src/arena.h:65-66: "1.94 GiB" into buf; returns buf. */
char   *arena_fmt_bytes(char *buf, size_t buflen, size_t bytes);

#define ARENA_NEW(a, T)      ((T *)arena_alloc_or_die((a), sizeof(T), _Alignof(T)))
#define ARENA_ARRAY(a, T, n) ((T *)arena_alloc_or_die((a), sizeof(T) * (size_t)(n), _Alignof(T)))

#ifdef __cplusplus
}
#endif
#endif /* TC_ARENA_H */
