/*
 * B200 replacement for the reference's two-kernel engine interface
 * board/kv260gemv/gemv2_dev.h:1-80 (fetch kernel + FIFOs + MAC kernel).
 *
 * A call is still two starts. gemv2_fetch_start(W) names the matrix as soon
 * as it is known; on a B200 it issues an L2 bulk prefetch of W's bytes on a
 * side stream (the FIFOs become the 126 MB L2), so the bytes move while the
 * caller does other work. gemv2_mac_start(x, y) then runs the GEMV over the
 * matrix of the pending fetch, bit-exact to src/llm_kv260/q4_0.py:151-182.
 * As in the reference, fetch(W) then mac(W), in order, and the next fetch
 * goes after this mac; a mac without a pending fetch of the same shape
 * returns -EINVAL instead of computing garbage.
 *
 * Layout (unchanged, gemv2_dev.h:46-49): four port regions of rows/4 rows at
 * any 16-byte-aligned addresses; inside a region row i pairs with row
 * i + rows/8 and their 144-byte chunks alternate (gemv2_chunk_offset).
 * rows % 8 == 0 here (the reference needs % 32), k % 256 == 0, k <= 8192.
 * Return values follow gemv_dev.h: 0 or a negative errno value.
 */
#ifndef B200_GEMV2_DEV_H
#define B200_GEMV2_DEV_H

#include <stddef.h>
#include <stdint.h>

#include "gemv_dev.h"

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    gemv_dev_t fetch, mac;   /* fetch: the prefetch side stream; mac: the GEMV stream */
    uint64_t w[4];           /* matrix of the pending fetch */
    int k, rows;
    int fetched;             /* a fetch is pending for the next mac */
} gemv2_dev_t;

#define GEMV2_CHUNK_BYTES 144

/* Replaces gemv2_dev.h:63: -1 (quietly) when there is no CUDA device. */
B200_API int gemv2_dev_open(gemv2_dev_t *d);
/* Replaces gemv2_dev.h:64 (void there). */
B200_API int gemv2_dev_close(gemv2_dev_t *d);

/* Replaces gemv2_dev.h:66-72 (same formula): offset of 144-byte chunk c of
 * row r inside its port region; *port = r / (rows/4). */
static inline size_t gemv2_chunk_offset(int r, int c, int rows, int k, int *port) {
    const int quarter = rows / 4, half = quarter / 2, chunks = k / 256;
    const int pair = (r % quarter) % half, member = (r % quarter) / half;
    *port = r / quarter;
    return (((size_t)pair * chunks + c) * 2 + member) * GEMV2_CHUNK_BYTES;
}

/* Replaces gemv2_dev.h:74-75. fetch_start waits for a previous fetch first. */
B200_API int gemv2_fetch_start(gemv2_dev_t *d, const uint64_t w[4], int k, int rows);
B200_API int gemv2_fetch_wait(gemv2_dev_t *d);
/* Replaces gemv2_dev.h:76-78. mac_idle returns 1 idle, 0 busy, <0 error. */
B200_API int gemv2_mac_start(gemv2_dev_t *d, uint64_t x, uint64_t y, int k, int rows);
B200_API int gemv2_mac_wait(gemv2_dev_t *d);
B200_API int gemv2_mac_idle(gemv2_dev_t *d);
/* Replaces gemv2_dev.h:80: forget a pending fetch and let in-flight work finish. */
B200_API int gemv2_drain(gemv2_dev_t *d);

#ifdef __cplusplus
}
#endif
#endif
