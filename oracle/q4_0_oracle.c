/*
 * CPU oracle (test infrastructure only, see q4_0_oracle.h). A C restatement
 * of the reference contract `src/llm_kv260/q4_0.py` and of the rank-ordered
 * sum in `board/tp/tp_llama.cpp`. Built with -O2 -ffp-contract=off.
 *
 * Parity pin: tests/test_oracle_golden.py checks every function here against
 * fixtures that tests/golden/gen_golden.py produced by running the reference
 * q4_0.py itself, including the reference's own golden SHA-256
 * (tests/test_q4_0_contract.py:181-191 in the reference).
 */
#include "q4_0_oracle.h"

#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK ORACLE_QK
#define BLK ORACLE_Q4_0_BYTES
#define LANES ORACLE_LANES

/* ------------------------------------------------------------ threads */

/* Rows are independent, so a static split over threads gives the same bits
 * as one thread. (No OpenMP: the oracle shares a process with torch, which
 * brings its own OpenMP runtime.) The workers persist between calls: a
 * tensor-parallel decode simulates up to 8 ranks, so one token makes several
 * hundred small GEMV calls, and a thread start per call would cost more than
 * the rows themselves. Workers spin briefly on the job counter, then sleep on
 * a condition variable. One caller at a time uses the pool; a second,
 * concurrent caller starts its own threads for that call. */
typedef struct {
    void (*fn)(void *ctx, int64_t lo, int64_t hi);
    void *ctx;
    int64_t lo, hi;
} span_t;

static void *span_run(void *arg) {
    span_t *s = (span_t *)arg;
    s->fn(s->ctx, s->lo, s->hi);
    return NULL;
}

static void spawn_rows(int64_t n, int threads, void (*fn)(void *, int64_t, int64_t), void *ctx) {
    pthread_t tid[256];
    span_t span[256];
    for (int t = 0; t < threads; ++t) {
        span[t].fn = fn;
        span[t].ctx = ctx;
        span[t].lo = n * t / threads;
        span[t].hi = n * (t + 1) / threads;
        if (t == 0) continue;
        /* a thread that cannot start runs its span here instead */
        if (pthread_create(&tid[t], NULL, span_run, &span[t])) {
            fn(ctx, span[t].lo, span[t].hi);
            span[t].fn = NULL;
        }
    }
    fn(ctx, span[0].lo, span[0].hi);
    for (int t = 1; t < threads; ++t) if (span[t].fn) pthread_join(tid[t], NULL);
}

enum { POOL_MAX = 256 };
static pthread_mutex_t pool_busy = PTHREAD_MUTEX_INITIALIZER;   /* held by the pool's one caller */
static pthread_mutex_t pool_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t pool_cv = PTHREAD_COND_INITIALIZER;
static int pool_workers;                  /* started so far (never stopped) */
/* The current job as one word: job number << 32 | span count << 16 | next
 * unclaimed span. A thread claims span i by moving the word from i to i + 1
 * (compare-and-swap), so a claim always names a span of the job that word
 * describes, and every span is run exactly once. The span table is written
 * only between jobs: the caller rewrites it after every span of the previous
 * job has finished (pool_left == 0), and a claim of the new job succeeds
 * only after the word announces it. */
static _Atomic uint64_t pool_claim;
static _Atomic int pool_left;             /* claimed-or-not spans of the current job not yet finished */
static span_t pool_span[POOL_MAX];

/* Run spans of the current job until none is left to claim. */
static void pool_drain(void) {
    for (;;) {
        uint64_t w = atomic_load_explicit(&pool_claim, memory_order_acquire);
        const uint32_t next = (uint32_t)(w & 0xffffu), ns = (uint32_t)((w >> 16) & 0xffffu);
        if (next >= ns) return;
        if (!atomic_compare_exchange_weak_explicit(&pool_claim, &w, w + 1, memory_order_acq_rel, memory_order_acquire))
            continue;
        const span_t *sp = &pool_span[next];
        sp->fn(sp->ctx, sp->lo, sp->hi);
        atomic_fetch_sub_explicit(&pool_left, 1, memory_order_acq_rel);
    }
}

static void *pool_worker(void *arg) {
    (void)arg;
    uint32_t seen = (uint32_t)(atomic_load_explicit(&pool_claim, memory_order_acquire) >> 32);
    for (;;) {
        uint32_t g;
        int spins = 0;
        while ((g = (uint32_t)(atomic_load_explicit(&pool_claim, memory_order_acquire) >> 32)) == seen) {
            if (++spins < 20000) {
                sched_yield();
                continue;
            }
            pthread_mutex_lock(&pool_mu);
            while ((g = (uint32_t)(atomic_load_explicit(&pool_claim, memory_order_acquire) >> 32)) == seen)
                pthread_cond_wait(&pool_cv, &pool_mu);
            pthread_mutex_unlock(&pool_mu);
            break;
        }
        seen = g;
        pool_drain();
    }
    return NULL;
}

static void parallel_rows(int64_t n, int threads, void (*fn)(void *, int64_t, int64_t), void *ctx) {
    if (threads > POOL_MAX) threads = POOL_MAX;
    if (threads < 2 || n < 2) { fn(ctx, 0, n); return; }
    if (threads > n) threads = (int)n;
    if (pthread_mutex_trylock(&pool_busy) != 0) {
        spawn_rows(n, threads, fn, ctx);
        return;
    }
    while (pool_workers < threads - 1) {
        pthread_t tid;
        if (pthread_create(&tid, NULL, pool_worker, NULL)) break;
        pthread_detach(tid);
        ++pool_workers;
    }
    for (int t = 0; t < threads; ++t) {
        pool_span[t].fn = fn;
        pool_span[t].ctx = ctx;
        pool_span[t].lo = n * t / threads;
        pool_span[t].hi = n * (t + 1) / threads;
    }
    atomic_store_explicit(&pool_left, threads, memory_order_relaxed);
    const uint64_t g = (atomic_load_explicit(&pool_claim, memory_order_relaxed) >> 32) + 1;
    pthread_mutex_lock(&pool_mu);
    atomic_store_explicit(&pool_claim, (g << 32) | ((uint64_t)threads << 16), memory_order_release);
    pthread_cond_broadcast(&pool_cv);
    pthread_mutex_unlock(&pool_mu);
    pool_drain();  /* the caller takes spans too */
    while (atomic_load_explicit(&pool_left, memory_order_acquire) > 0) sched_yield();
    pthread_mutex_unlock(&pool_busy);
}

void oracle_parallel_for(int64_t n, int threads, void (*fn)(void *, int64_t, int64_t), void *ctx) {
    parallel_rows(n, threads, fn, ctx);
}

/* ------------------------------------------------------------ float16 */

uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u | (mant >> 13) : 0u));
    const int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++; /* a carry may reach inf, as it should */
    return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        float v = ldexpf((float)mant, -24); /* exact: mant < 2^10 */
        memcpy(&x, &v, 4);
        x |= sign;
    } else if (exp == 31) {
        x = sign | 0x7F800000u | (mant << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------ tree */

/* q4_0.py:67-78, and the engine's tree8 (hls/int4_core/gemv_core.h:85-89). */
float oracle_tree_sum8(const float l[8]) {
    const float a = l[0] + l[1], b = l[2] + l[3], c = l[4] + l[5], d = l[6] + l[7];
    return (a + b) + (c + d);
}

/* ------------------------------------------------------------ quantizers */

/* q4_0.py:83-97. amax / 127 in float32, inv = d == 0 ? 0 : 1/d, then the
 * rounding the contract spells out by hand (line 96), scale stored as float16. */
int oracle_quantize_q8_0(const float *x, int64_t k, int8_t *q, uint16_t *d, int round_mode) {
    if (!x || !q || !d || k < 0) return -2;
    if (k % QK) return -1;
    for (int64_t b = 0; b < k / QK; ++b) {
        const float *xb = x + b * QK;
        float amax = 0.0f;
        for (int j = 0; j < QK; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float db = amax / 127.0f;
        const float inv = db == 0.0f ? 0.0f : 1.0f / db;
        for (int j = 0; j < QK; ++j) {
            const float s = xb[j] * inv;
            float r;
            if (round_mode == ORACLE_Q8_ROUND_ROUNDF) {
                r = roundf(s);
            } else {
                const float m = floorf(fabsf(s) + 0.5f);
                r = s < 0.0f ? -m : (s > 0.0f ? m : 0.0f);
            }
            q[b * QK + j] = (int8_t)(int)r;
        }
        d[b] = oracle_f32_to_f16(db);
    }
    return 0;
}

/* q4_0.py:100-121. d = (signed extreme) / -8, q = trunc(w * inv + 8.5) as
 * uint8 then clipped to 15, byte j = q[j] | q[j+16] << 4, after the float16 d. */
typedef struct { const float *w; int64_t k; uint8_t *blocks; } q4_ctx_t;

static void quantize_q4_0_rows(void *p, int64_t lo, int64_t hi) {
    const q4_ctx_t *c = (const q4_ctx_t *)p;
    const int64_t k = c->k, nb = k / QK;
    for (int64_t r = lo; r < hi; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            const float *wb = c->w + r * k + b * QK;
            uint8_t *out = c->blocks + (r * nb + b) * BLK;
            int imax = 0;
            float best = -1.0f;
            for (int j = 0; j < QK; ++j) {
                const float a = fabsf(wb[j]);
                if (a > best) { best = a; imax = j; } /* first index of the max, as np.argmax */
            }
            const float db = wb[imax] / -8.0f;
            const float inv = db == 0.0f ? 0.0f : 1.0f / db;
            uint8_t qv[QK];
            for (int j = 0; j < QK; ++j) {
                const float v = truncf(wb[j] * inv + 8.5f);
                const unsigned u = (unsigned)(int)v;
                qv[j] = (uint8_t)(u > 15u ? 15u : u);
            }
            const uint16_t h = oracle_f32_to_f16(db);
            out[0] = (uint8_t)(h & 0xFFu);
            out[1] = (uint8_t)(h >> 8);
            for (int j = 0; j < QK / 2; ++j) out[2 + j] = (uint8_t)(qv[j] | (qv[j + QK / 2] << 4));
        }
    }
}

/* q4_0.py:100-121. d = (signed extreme) / -8, q = trunc(w * inv + 8.5) as
 * uint8 then clipped to 15, byte j = q[j] | q[j+16] << 4, after the float16 d. */
int oracle_quantize_q4_0(const float *w, int64_t n, int64_t k, uint8_t *blocks, int threads) {
    if (!w || !blocks || n < 0 || k < 0) return -2;
    if (k % QK) return -1;
    q4_ctx_t c = {w, k, blocks};
    parallel_rows(n, threads, quantize_q4_0_rows, &c);
    return 0;
}

/* ------------------------------------------------------------ codec */

/* q4_0.py:126-140: low nibble of byte j is weight j, high nibble weight j+16, value n-8. */
int oracle_unpack_q4_0(const uint8_t *blocks, int64_t n, int64_t k, int8_t *ints, uint16_t *d) {
    if (!blocks || !ints || !d || n < 0 || k < 0) return -2;
    if (k % QK) return -1;
    const int64_t nb = k / QK;
    for (int64_t r = 0; r < n; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = blocks + (r * nb + b) * BLK;
            d[r * nb + b] = (uint16_t)(blk[0] | (blk[1] << 8));
            int8_t *o = ints + r * k + b * QK;
            for (int j = 0; j < QK / 2; ++j) {
                o[j] = (int8_t)((blk[2 + j] & 0x0F) - 8);
                o[j + QK / 2] = (int8_t)((blk[2 + j] >> 4) - 8);
            }
        }
    return 0;
}

/* q4_0.py:143-146. */
int oracle_dequantize_q4_0(const uint8_t *blocks, int64_t n, int64_t k, float *out) {
    if (!blocks || !out || n < 0 || k < 0) return -2;
    if (k % QK) return -1;
    const int64_t nb = k / QK;
    for (int64_t r = 0; r < n; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = blocks + (r * nb + b) * BLK;
            const float df = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            float *o = out + r * k + b * QK;
            for (int j = 0; j < QK / 2; ++j) {
                o[j] = (float)((blk[2 + j] & 0x0F) - 8) * df;
                o[j + QK / 2] = (float)((blk[2 + j] >> 4) - 8) * df;
            }
        }
    return 0;
}

/* ------------------------------------------------------------ gemv */

/* One row in the contract's order (q4_0.py:169-182):
 *   sumi[b] = sum_j int(w) * int(x)                  int32, order-free
 *   t[b]    = (f32(sumi) * f32(dw)) * f32(dx)        two float32 multiplies
 *   lane[b % 8] = lane[b % 8] + t[b]                 sequential in b, from +0.0f
 *   y = tree_sum(lane)
 * dx[] holds the activation scales already widened to float32. */
static float gemv_row(const uint8_t *row, int64_t nb, const int8_t *xq, const float *dx) {
    float lanes[LANES] = {0};
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *blk = row + b * BLK;
        const int8_t *xb = xq + b * QK;
        int32_t sumi = 0;
        for (int j = 0; j < QK / 2; ++j) {
            sumi += (int32_t)((blk[2 + j] & 0x0F) - 8) * (int32_t)xb[j];
            sumi += (int32_t)((blk[2 + j] >> 4) - 8) * (int32_t)xb[j + QK / 2];
        }
        const float dw = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const float t = ((float)sumi * dw) * dx[b];
        lanes[b % LANES] = lanes[b % LANES] + t;
    }
    return oracle_tree_sum8(lanes);
}

typedef struct { const uint8_t *blocks; int64_t nb; const int8_t *xq; const float *dx; float *y; } gemv_ctx_t;

static void gemv_span(void *p, int64_t lo, int64_t hi) {
    const gemv_ctx_t *c = (const gemv_ctx_t *)p;
    for (int64_t r = lo; r < hi; ++r) c->y[r] = gemv_row(c->blocks + r * c->nb * BLK, c->nb, c->xq, c->dx);
}

static int gemv_rows(const uint8_t *blocks, int64_t n, int64_t k, const int8_t *xq, const float *dx, float *y,
                     int threads, int allow_ragged_lanes) {
    if (k % QK) return -1;
    const int64_t nb = k / QK;
    if (!allow_ragged_lanes && nb % LANES) return -1; /* q4_0.py:166-167 */
    gemv_ctx_t c = {blocks, nb, xq, dx, y};
    parallel_rows(n, threads, gemv_span, &c);
    return 0;
}

int oracle_gemv_q4_0(const uint8_t *blocks, int64_t n, int64_t k, const int8_t *xq, const uint16_t *xd, float *y,
                     int threads, int allow_ragged_lanes) {
    if (!blocks || !xq || !xd || !y || n < 0 || k < 0) return -2;
    if (k % QK) return -1;
    const int64_t nb = k / QK;
    float *dxs = (float *)malloc((size_t)(nb > 0 ? nb : 1) * sizeof(float));
    if (!dxs) return -2;
    for (int64_t b = 0; b < nb; ++b) dxs[b] = oracle_f16_to_f32(xd[b]);
    const int rc = gemv_rows(blocks, n, k, xq, dxs, y, threads, allow_ragged_lanes);
    free(dxs);
    return rc;
}

int oracle_gemv_q4_0_f32(const uint8_t *blocks, int64_t n, int64_t k, const float *x, float *y, int threads,
                         int round_mode) {
    if (!blocks || !x || !y || n < 0 || k < 0) return -2;
    if (k % QK) return -1;
    int8_t *xq = (int8_t *)malloc((size_t)(k > 0 ? k : 1));
    uint16_t *xd = (uint16_t *)malloc((size_t)(k / QK > 0 ? k / QK : 1) * 2);
    int rc = (xq && xd) ? oracle_quantize_q8_0(x, k, xq, xd, round_mode) : -2;
    if (!rc) rc = oracle_gemv_q4_0(blocks, n, k, xq, xd, y, threads, 0);
    free(xq);
    free(xd);
    return rc;
}

/* q4_0.py:193-200. */
int oracle_pack_x_for_engine(const int8_t *xq, const uint16_t *xd, int64_t k, uint8_t *out) {
    if (!xq || !xd || !out || k < 0) return -2;
    if (k % QK) return -1;
    memcpy(out, xq, (size_t)k);
    for (int64_t b = 0; b < k / QK; ++b) {
        const float f = oracle_f16_to_f32(xd[b]);
        memcpy(out + k + 4 * b, &f, 4);
    }
    return 0;
}

int oracle_gemv_q4_0_packed(const uint8_t *blocks, int64_t n, int64_t k, const uint8_t *xpacked, float *y,
                            int threads) {
    if (!blocks || !xpacked || !y || n < 0 || k < 0) return -2;
    if (k % QK) return -1;
    const int64_t nb = k / QK;
    float *dxs = (float *)malloc((size_t)(nb > 0 ? nb : 1) * sizeof(float));
    if (!dxs) return -2;
    memcpy(dxs, xpacked + k, (size_t)nb * 4);
    const int rc = gemv_rows(blocks, n, k, (const int8_t *)xpacked, dxs, y, threads, 0);
    free(dxs);
    return rc;
}

/* board/kv260gemv/gemv2_dev.h:66-72: rows pair up (i, i + rows/8) inside each
 * of four port regions and their 144-byte chunks alternate. */
int64_t oracle_gemv2_chunk_offset(int r, int c, int rows, int k, int *port) {
    const int R = rows / 4, H = R / 2, nch = k / 256;
    const int i = (r % R) % H, which = (r % R) / H;
    *port = r / R;
    return (((int64_t)i * nch + c) * 2 + which) * 144;
}

/* ------------------------------------------------------------ all-reduce */

/* tp_llama.cpp:515-521: every element is p0 + p1 + ... + p{n-1}, left to right. */
int oracle_allreduce_ordered(const float *const *partials, int n, int64_t len, float *out) {
    if (!partials || !out || n < 1 || len < 0) return -2;
    for (int64_t i = 0; i < len; ++i) {
        float s = partials[0][i];
        for (int r = 1; r < n; ++r) s = s + partials[r][i];
        out[i] = s;
    }
    return 0;
}
