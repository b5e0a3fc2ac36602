/*
 * Engine-level C ABI: the B200 counterpart of the runtime's engine wrapper
 * engine_t (board/tp/tp_llama.cpp:289-375), i.e. the call the decode loop
 * makes per matrix: quantise float32 x to Q8_0, run the Q4_0 GEMV, and name
 * the matrix that comes next so its bytes can start moving early.
 *
 * Weights stay in the GGUF Q4_0 row layout (18-byte blocks, row-major), one
 * contiguous 16-byte-aligned allocation per matrix; no repack. Results are
 * bit-exact to src/llm_kv260/q4_0.py:185-188 (gemv_q4_0_f32).
 *
 * All addresses are CUDA device addresses; all functions return 0 or a
 * negative errno value (see gemv_dev.h), and b200_last_error() says why.
 * An engine belongs to one device and one caller thread.
 */
#ifndef B200_ENGINE_H
#define B200_ENGINE_H

#include <stdint.h>

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_engine b200_engine_t;

/* A Q4_0 matrix in device memory: replaces qmat (tp_llama.cpp:105-119), one
 * region instead of four staggered port quarters (HBM has no DDR-bank
 * collisions to dodge). */
typedef struct {
    uint64_t w;  /* first byte of row 0; rows are k/32*18 bytes apart */
    int rows;
    int k;
} b200_qmat_t;

typedef struct {
    int stage_bytes;     /* target bytes per shared-memory pipeline stage (default 16384) */
    int stages;          /* stages in flight per CTA, 1..8 (default 4) */
    int ctas_per_sm;     /* grid = SMs x this (default 2) */
    int l2_policy;       /* weight bytes: 0 evict-first (default), 1 normal, 2 evict-last */
    int pdl;             /* 1: launch with programmatic dependent launch (default 1) */
    int round_mode;      /* Q8_0 rounding: 0 floor(|s|+0.5f) as q4_0.py:96 (default), 1 roundf as tp_llama.cpp:343 */
    int fuse_quantize;   /* b200_gemv_f32: 1 quantise inside each GEMV CTA, 0 a separate quantise kernel (default 0) */
    int prefetch_next;   /* 1: a `next` hint issues an L2 prefetch of that matrix on a side stream (default 0) */
} b200_engine_config_t;

/* Replaces engine_t::probe + engine_t::open (tp_llama.cpp:303-317). */
B200_API int b200_engine_open(b200_engine_t **e, int device);
B200_API int b200_engine_close(b200_engine_t *e);
B200_API int b200_engine_get_config(b200_engine_t *e, b200_engine_config_t *cfg);
B200_API int b200_engine_set_config(b200_engine_t *e, const b200_engine_config_t *cfg);
/* Queue work on the caller's cudaStream_t (NULL: the legacy default stream).
 * Until this is called the engine uses a non-blocking stream of its own. */
B200_API int b200_engine_set_stream(b200_engine_t *e, void *stream);
B200_API void *b200_engine_stream(b200_engine_t *e);

/* Replaces engine_t::gemv (tp_llama.cpp:355-374): y[rows] = W x for float32
 * x[k]; `next` (may be NULL) is the matrix the caller passes next. */
B200_API int b200_gemv_f32(b200_engine_t *e, const b200_qmat_t *W, uint64_t x, uint64_t y, const b200_qmat_t *next);
/* The same over an already-quantised x in the engine layout, int8[k] then
 * float32[k/32] (q4_0.py:193-200); this is gemv_dev_start's computation. */
B200_API int b200_gemv_q8(b200_engine_t *e, const b200_qmat_t *W, uint64_t xpacked, uint64_t y, const b200_qmat_t *next);
/* Replaces engine_t::quantize_x (tp_llama.cpp:330-352) with the contract's
 * rounding by default: x float32[k] -> xpacked int8[k] + float32[k/32]. */
B200_API int b200_quantize_q8_0(b200_engine_t *e, uint64_t x, uint64_t xpacked, int k);
/* Replaces engine_t::prefetch (tp_llama.cpp:318-323): L2 prefetch of W. */
B200_API int b200_prefetch(b200_engine_t *e, const b200_qmat_t *W);

/* Block until the engine's queued work is done (bounded; -ETIMEDOUT). */
B200_API int b200_engine_sync(b200_engine_t *e, int timeout_ms);
/* Device status word (see gemv_dev_status); reading clears it. */
B200_API int b200_engine_status(b200_engine_t *e, unsigned *status);
/* Launch shape the GEMV would use for W (for roofline accounting). */
B200_API int b200_gemv_plan(b200_engine_t *e, int rows, int k, int fused_f32, int *grid, int *smem_bytes);

B200_API int b200_device_count(void);
/* Message for the last error on this thread (never NULL). */
B200_API const char *b200_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
