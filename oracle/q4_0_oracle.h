/*
 * CPU oracle for the Q4_0 x Q8_0 GEMV contract and the rank-ordered
 * all-reduce sum. TEST INFRASTRUCTURE ONLY: the parity tests, the smoke
 * check and the bench's CPU-baseline leg link this library as the checker.
 * The product (the CUDA library) never calls it and has no CPU fallback.
 *
 * Each function restates one function of the reference contract
 * `src/llm_kv260/q4_0.py` (CONTRACT_VERSION "llm-kv260/w4a8-q4_0-v2") or of
 * the reference runtime `board/tp/tp_llama.cpp`, and cites the lines it
 * follows. Everything is fixed-width float32 / int32 arithmetic compiled with
 * -ffp-contract=off, so no multiply-add is fused behind the contract's back.
 *
 * Return codes: 0 ok, -1 bad shape (the contract's ValueError), -2 bad
 * argument (null pointer / negative size).
 */
#ifndef Q4_0_ORACLE_H
#define Q4_0_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_QK 32          /* q4_0.py:59 */
#define ORACLE_Q4_0_BYTES 18  /* q4_0.py:60 */
#define ORACLE_LANES 8        /* q4_0.py:62 */

/* Q8_0 rounding of the scaled activation s = x * (1/d).
 * CONTRACT: sign(s) * floor(|s| + 0.5f), the add rounded in float32
 *           (q4_0.py:94-96). This is the default and what the GEMV contract pins.
 * ROUNDF:   roundf(s), ties away from zero, as the runtime's NEON vcvtaq does
 *           (tp_llama.cpp:343). Differs from CONTRACT only at |s| = 0.5 - 2^-25. */
enum { ORACLE_Q8_ROUND_CONTRACT = 0, ORACLE_Q8_ROUND_ROUNDF = 1 };

/* IEEE binary16 <-> binary32, round to nearest even, subnormals kept. */
uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);

/* tree_sum over 8 lanes: ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)) (q4_0.py:67-78). */
float oracle_tree_sum8(const float lanes[8]);

/* quantize_q8_0 (q4_0.py:83-97): x float32[k] -> q int8[k], d float16 bits[k/32]. */
int oracle_quantize_q8_0(const float *x, int64_t k, int8_t *q, uint16_t *d, int round_mode);

/* quantize_q4_0 (q4_0.py:100-121): w float32[n,k] -> blocks uint8[n, k/32*18]. */
int oracle_quantize_q4_0(const float *w, int64_t n, int64_t k, uint8_t *blocks, int threads);

/* unpack_q4_0 (q4_0.py:126-140): ints int8[n,k] in [-8,7], d float16 bits[n,k/32]. */
int oracle_unpack_q4_0(const uint8_t *blocks, int64_t n, int64_t k, int8_t *ints, uint16_t *d);

/* dequantize_q4_0 (q4_0.py:143-146): float32[n,k] = (nibble-8) * f32(d). */
int oracle_dequantize_q4_0(const uint8_t *blocks, int64_t n, int64_t k, float *out);

/* gemv_q4_0 (q4_0.py:151-182): y[n] = W x in the engine's order. The row
 * stride of `blocks` is k/32*18 bytes (the GGUF layout). nb = k/32 must be a
 * multiple of 8 (q4_0.py:166-167) unless allow_ragged_lanes is set, which
 * applies the same lane rule (block b into lane b mod 8) to any nb. */
int oracle_gemv_q4_0(const uint8_t *blocks, int64_t n, int64_t k, const int8_t *xq, const uint16_t *xd,
                     float *y, int threads, int allow_ragged_lanes);

/* gemv_q4_0_f32 (q4_0.py:185-188): quantize_q8_0 then gemv_q4_0. */
int oracle_gemv_q4_0_f32(const uint8_t *blocks, int64_t n, int64_t k, const float *x, float *y, int threads,
                         int round_mode);

/* pack_x_for_engine (q4_0.py:193-200): int8[k] then float32[k/32] (widened d). */
int oracle_pack_x_for_engine(const int8_t *xq, const uint16_t *xd, int64_t k, uint8_t *out);

/* gemv over the engine's packed activation buffer (what gemv_dev_run reads,
 * board/kv260gemv/gemv_dev.h:19-23): x = int8[k] then float32[k/32]. The
 * float32 scales are used as they are (they are widened float16 values). */
int oracle_gemv_q4_0_packed(const uint8_t *blocks, int64_t n, int64_t k, const uint8_t *xpacked, float *y,
                            int threads);

/* The gemv2 chunk interleave (board/kv260gemv/gemv2_dev.h:46-49,66-72): byte
 * offset of 144-byte chunk c of row r inside its port region; *port = r/(rows/4). */
int64_t oracle_gemv2_chunk_offset(int r, int c, int rows, int k, int *port);

/* Rank-ordered sum of n partial vectors (comm_t::allreduce_sum,
 * tp_llama.cpp:515-521): s = p0; s = s + p_r for r = 1..n-1, per element. */
int oracle_allreduce_ordered(const float *const *partials, int n, int64_t len, float *out);

/* Run fn(ctx, lo, hi) over [0, n) split across `threads` threads (the
 * oracle's worker pool); for independent items only. */
void oracle_parallel_for(int64_t n, int threads, void (*fn)(void *ctx, int64_t lo, int64_t hi), void *ctx);

#ifdef __cplusplus
}
#endif
#endif
