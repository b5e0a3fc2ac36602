/*
 * B200 replacement for the reference engine's control interface
 * board/kv260gemv/gemv_dev.h:10-35 (the gemv_q4_0 FPGA engine).
 *
 * Same function names, same arguments, same meaning: y[rows] = W[rows, k] x
 * with W in Q4_0 rows exactly as a GGUF file stores them and x in the
 * engine's activation layout, int8[k] then float32[k/32]
 * (src/llm_kv260/q4_0.py:193-200). The result is bit-exact to the contract
 * src/llm_kv260/q4_0.py:151-182.
 *
 * What changes on a B200:
 *   - Addresses are CUDA device addresses (uint64_t), not physical ones.
 *     Memory comes from udmabuf.h (this library's device pool with a host
 *     mirror), from cudaMalloc, or from any allocator the caller trusts.
 *   - Every function returns int: 0 on success, a negative errno value on
 *     error (-EINVAL bad shape/alignment, -ENODEV no CUDA device, -ETIMEDOUT
 *     a bounded wait ran out, -EBUSY a start while one is pending, -EIO a
 *     CUDA call failed). The reference returns void from run/start/wait and
 *     spins forever; callers that ignore the result still compile.
 *   - Work runs on a CUDA stream; start enqueues and returns, wait blocks on
 *     an event for at most timeout_ms (default 10000).
 *   - Constraints are relaxed: k % 256 == 0 and 256 <= k <= 8192 as before,
 *     but any rows >= 1 (rows % 4 == 0 for gemv_dev_start4 only); weight
 *     regions and x must be 16-byte aligned, y 4-byte aligned.
 * Threading: one caller thread per gemv_dev_t, one call in flight, as in the
 * reference.
 */
#ifndef B200_GEMV_DEV_H
#define B200_GEMV_DEV_H

#include <stdint.h>

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int fd;            /* CUDA device ordinal (the reference kept the UIO file descriptor here) */
    void *stream;      /* cudaStream_t the engine's work is queued on */
    void *done;        /* cudaEvent_t recorded after each start */
    int pending;       /* a start that has not been waited for */
    int owns_stream;   /* the stream was created by open and is destroyed by close */
    int timeout_ms;    /* bound on gemv_dev_wait; <= 0 means the 10 s default */
    uint64_t started_ns;
} gemv_dev_t;

/* Replaces gemv_dev.h:15. Opens the engine on the current CUDA device. */
B200_API int gemv_dev_open(gemv_dev_t *d);

/* Replaces gemv_dev.h:16. Names: "gemv_q4_0", "gemv_fetch", "gemv_mac"
 * (the reference's UIO names; each is the GEMV engine of a CUDA device),
 * optionally followed by ":<device ordinal>". quiet suppresses the message. */
B200_API int gemv_dev_open_named(gemv_dev_t *d, const char *name, int quiet);

/* Replaces gemv_dev.h:17 (void there). */
B200_API int gemv_dev_close(gemv_dev_t *d);

/* Replaces gemv_dev.h:23: start then wait. */
B200_API int gemv_dev_run(gemv_dev_t *d, uint64_t w, uint64_t x, uint64_t y, int k, int rows);

/* Replaces gemv_dev.h:26-27, the split form. */
B200_API int gemv_dev_start(gemv_dev_t *d, uint64_t w, uint64_t x, uint64_t y, int k, int rows);
B200_API int gemv_dev_wait(gemv_dev_t *d);

/* Replaces gemv_dev.h:35: quarter m of the rows (rows/4 rows) lives at w[m],
 * its outputs at y + m * rows/4 floats. */
B200_API int gemv_dev_start4(gemv_dev_t *d, const uint64_t w[4], uint64_t x, uint64_t y, int k, int rows);

/* B200 extensions (no counterpart in the reference). */
/* Queue the engine's work on the caller's cudaStream_t instead of its own
 * (NULL: the legacy default stream). */
B200_API int gemv_dev_set_stream(gemv_dev_t *d, void *stream);
/* Device status word: bit 0 = a weight stage never landed (kernel gave up
 * after a bounded wait; that call's output is incomplete). Reading clears it. */
B200_API int gemv_dev_status(gemv_dev_t *d, unsigned *status);
/* Message for the last error on this thread (never NULL). */
B200_API const char *gemv_dev_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
