/*
 * B200 replacement for the reference's engine memory pool
 * board/kv260gemv/udmabuf.h:15-36 (u-dma-buf CMA pool, cached CPU mapping).
 *
 * The reference hands the engine physical addresses of CPU-written memory
 * and makes the caller own coherence: clean after the CPU writes, invalidate
 * before the CPU reads (udmabuf.h:1-10). The B200 pool keeps exactly that
 * contract with two copies of the bytes:
 *   base  a pinned host mirror the CPU reads and writes,
 *   phys  the device address of the same offset in HBM (what the engine gets).
 * udmabuf_clean(p, len) copies that range host -> device, udmabuf_invalidate
 * copies it device -> host; both are synchronous, like the reference's
 * cache-maintenance loops. Allocation is the same bump allocator with no free.
 * Return values: 0 or a negative errno value; udmabuf_alloc returns NULL when
 * the pool is full.
 */
#ifndef B200_UDMABUF_H
#define B200_UDMABUF_H

#include <stddef.h>
#include <stdint.h>

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int fd;          /* CUDA device ordinal of the device half */
    uint8_t *base;   /* CPU virtual address: the pinned host mirror */
    uint64_t phys;   /* device address of byte 0 of the pool */
    size_t size;
    size_t used;     /* bump allocator watermark */
} udmabuf_t;

/* Replaces udmabuf.h:23. The reference reads the size from sysfs; here it is
 * $UDMABUF_SIZE_<NAME> bytes (e.g. UDMABUF_SIZE_UDMABUF0), else 256 MiB, on the
 * current CUDA device. */
B200_API int udmabuf_open(udmabuf_t *b, const char *name);
/* Replaces udmabuf.h:24 (void there). */
B200_API int udmabuf_close(udmabuf_t *b);

/* Replaces udmabuf.h:28: bump-allocate, align a power of two; NULL when full. */
B200_API void *udmabuf_alloc(udmabuf_t *b, size_t size, size_t align);

/* Replaces udmabuf.h:30-32 (same formula). */
static inline uint64_t udmabuf_phys(const udmabuf_t *b, const void *p) {
    return b->phys + (uint64_t)((const uint8_t *)p - b->base);
}

/* Replaces udmabuf.h:35-36 (void there): host mirror -> device, device -> host
 * mirror, over [p, p+len) of whichever open pool holds p. */
B200_API int udmabuf_clean(const void *p, size_t len);
B200_API int udmabuf_invalidate(const void *p, size_t len);

/* B200 extension: open a pool of an explicit size on an explicit device. */
B200_API int udmabuf_open_size(udmabuf_t *b, const char *name, size_t size, int device);

#ifdef __cplusplus
}
#endif
#endif
