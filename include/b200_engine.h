/*
 * Engine-level C ABI: the B200 counterpart of the runtime's engine wrapper
 * engine_t (board/tp/tp_llama.cpp:289-375), i.e. the call the decode loop
 * makes per matrix: quantise float32 x to Q8_0, run the Q4_0 GEMV, and name
 * the matrix that comes next so its bytes can start moving early.
 *
 * Weights are one contiguous 16-byte-aligned allocation per matrix, either
 * in the GGUF Q4_0 row layout (18-byte blocks, row-major) or re-laid once at
 * load into the engine's tiles (b200_repack_q4_0), which the fast kernel
 * reads. Results are bit-exact to src/llm_kv260/q4_0.py:185-188
 * (gemv_q4_0_f32).
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
 * collisions to dodge). Two layouts:
 *   B200_LAYOUT_ROWS   the GGUF bytes as they are: rows of k/32 18-byte blocks;
 *   B200_LAYOUT_TILES  the engine's re-laid form (b200_repack_q4_0), which the
 *                      fast kernel reads; the same 18 bytes per 32 weights, rows
 *                      padded to a multiple of 16 (b200_tiled_bytes).
 * The reference re-lays its weights at load in the same way for its own
 * engine (tp_llama.cpp:102-118, the gemv2 chunk interleave). */
#define B200_LAYOUT_ROWS 0
#define B200_LAYOUT_TILES 1

typedef struct {
    uint64_t w;  /* first byte of the matrix, 16-byte aligned */
    int rows;
    int k;
    int layout;  /* B200_LAYOUT_ROWS or B200_LAYOUT_TILES */
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
    int xreg_chunks;     /* GGUF-row kernel: unused; kept for the layout of this struct (default 8) */
    int kslices;         /* tile kernel: split each row's block dots over at least this many thread slices: 1, 2 or 4 (default 1) */
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

/* Bytes of the tile layout of a rows x k matrix (0 for an unusable shape). */
B200_API uint64_t b200_tiled_bytes(int rows, int k);
/* Re-lay GGUF Q4_0 rows at `src` (2-byte aligned) into tiles at `dst`
 * (16-byte aligned, b200_tiled_bytes(rows, k) bytes) on the engine's stream. */
B200_API int b200_repack_q4_0(b200_engine_t *e, uint64_t src, int rows, int k, uint64_t dst);

/* b200_gemv_f32 plus the greedy pick over its output, fused into the GEMV
 * (the lm_head call of a decode token): y as b200_gemv_f32, and the 8 bytes at
 * `out` as b200_argmax_f32 over y[0..rows). W must be in the tile layout. */
B200_API int b200_gemv_argmax_f32(b200_engine_t *e, const b200_qmat_t *W, uint64_t x, uint64_t y, int index_base,
                                  uint64_t out);

/* Greedy pick over y[0..n) on the device, as the runtime's scan does
 * (tp_llama.cpp:879-882: first index of the largest value): writes the
 * int32 index + index_base, then the float32 value, to the 8 bytes at `out`. */
B200_API int b200_argmax_f32(b200_engine_t *e, uint64_t y, int n, int index_base, uint64_t out);

/* Graphs: record a sequence of engine calls once and replay it with one
 * launch (a decode token is ~70 dependent kernels; replaying them as a CUDA
 * graph with programmatic dependent launch removes the per-kernel CPU cost).
 * Between capture_begin and capture_end the engine's calls are recorded, not
 * run; run every call once before capturing it (first calls set up caches).
 * The engine must be on a stream of its own (not the legacy default). */
typedef struct b200_graph b200_graph_t;
B200_API int b200_capture_begin(b200_engine_t *e);
B200_API int b200_capture_end(b200_engine_t *e, b200_graph_t **g);
B200_API int b200_graph_launch(b200_engine_t *e, b200_graph_t *g);
B200_API int b200_graph_destroy(b200_graph_t *g);
/* Asynchronous copy of `bytes` bytes on the engine's stream, any direction
 * (unified addressing); host memory should be pinned. */
B200_API int b200_copy_async(b200_engine_t *e, uint64_t dst, uint64_t src, uint64_t bytes);

/* The greedy pick of b200_argmax_f32 for callers that cannot allocate device
 * memory. No counterpart in the reference: its engine had no allocator of
 * its own. Opening an engine calls cudaMalloc; this entry point needs no
 * engine and allocates nothing, so it serves code that runs during stream
 * capture, callers whose device memory all comes from their own allocator,
 * and processes where allocating after start-up is not allowed. Its scratch
 * is a fixed 8 KB array inside the library (1024 per-CTA candidates) that
 * every GPU loading the library holds until exit. Runs on the current
 * device, on `stream` (NULL: the legacy default stream); y holds n floats,
 * n <= 33554432 (larger n is refused with -EINVAL); out gets the int32 index
 * + index_base, then the float32 value. The first call on a device looks up
 * the array's device address, so make it before any stream capture. All
 * calls share the array: calls that overlap on the GPU race. */
B200_API int b200_argmax_f32_noalloc(uint64_t y, int n, int index_base, uint64_t out, void *stream);

/* Block until the engine's queued work is done (bounded; -ETIMEDOUT). */
B200_API int b200_engine_sync(b200_engine_t *e, int timeout_ms);
/* Device status word (see gemv_dev_status); reading clears it. */
B200_API int b200_engine_status(b200_engine_t *e, unsigned *status);
/* Launch shape the GEMV would use for W (for roofline accounting). */
B200_API int b200_gemv_plan(b200_engine_t *e, int rows, int k, int layout, int fused_f32, int *grid, int *smem_bytes);

B200_API int b200_device_count(void);
/* Message for the last error on this thread (never NULL). */
B200_API const char *b200_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
