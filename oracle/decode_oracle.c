/*
 * CPU oracle for the reference runtime's decode step. TEST INFRASTRUCTURE
 * ONLY (see decode_oracle.h for the rounding rules and what is unpinned).
 * Built with -ffp-contract=off: every fused multiply-add below is an explicit
 * fmaf, everything else rounds per operation.
 */
#include "decode_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "q4_0_oracle.h"

static uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static float u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* v_expf, tp_llama.cpp:530-553: ggml's vector exp, after Arm's optimized
 * routines (exp2 split with a degree-5 polynomial, 1.45358 + 0.5 ulp). One
 * lane of it; the lanes do not interact (the special-case branch picks the
 * same value per lane as the fast path wherever |n| <= 126). */
float odec_v_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, r);
    const float n = z - r;
    float b = fmaf(-n, 0x1.62e4p-1f, x);
    b = fmaf(-n, 0x1.7f7d1cp-20f, b);
    const uint32_t e = f2u(z) << 23;
    const float k = u2f(e + f2u(1.0f));
    const int c = fabsf(n) > 126.0f;
    const float u = b * b;
    const float p1 = fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f);
    const float p2 = fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f);
    const float p3 = fmaf(p2, u, p1);
    const float j = fmaf(p3, u, 0x1.ffffecp-1f * b);
    if (!c) return fmaf(j, k, k);
    const uint32_t dd = n <= 0.0f ? 0x82000000u : 0u;
    const float s1 = u2f(dd + 0x7f000000u);
    const float s2 = u2f(e - dd);
    if (fabsf(n) > 192.0f) return s1 * s1;
    return fmaf(s2, j, s2) * s1;
}

/* rmsnorm, tp_llama.cpp:557-569: sum of squares in double over four lanes
 * (i mod 4; lanes 0,1 in s0 and 2,3 in s1), combined as
 * (s0[0] + s1[0]) + (s0[1] + s1[1]); scale = 1 / sqrtf((float)(ss / n) + eps);
 * out = (x * scale) * w. n % 4 == 0. The square of a float is exact in
 * double, so the fused multiply-add there rounds only the add. */
void odec_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    double a[4] = {0.0, 0.0, 0.0, 0.0};
    for (int i = 0; i < n; i += 4)
        for (int j = 0; j < 4; ++j) a[j] = fma((double)x[i + j], (double)x[i + j], a[j]);
    const double ss = (a[0] + a[2]) + (a[1] + a[3]);
    const float scale = 1.0f / sqrtf((float)(ss / n) + eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * scale) * w[i];
}

/* rope_table, tp_llama.cpp:574-580: theta_i = pos * base^(-2i/d), divided
 * by the model's frequency factor freqs[i] when it has rope_freqs (Llama 3
 * GGUFs do; random-init models do not), all in float. */
void odec_rope_table_freqs(float *cs, int d, int pos, float base, const float *freqs) {
    for (int i = 0; i < d / 2; ++i) {
        float theta = (float)pos * powf(base, -2.0f * (float)i / (float)d);
        if (freqs) theta = theta / freqs[i];
        cs[2 * i] = cosf(theta);
        cs[2 * i + 1] = sinf(theta);
    }
}

void odec_rope_table(float *cs, int d, int pos, float base) { odec_rope_table_freqs(cs, d, pos, base, NULL); }

/* rope, tp_llama.cpp:581-591: adjacent pairs of every head. */
void odec_rope(float *x, int n_heads, int d, const float *cs) {
    for (int i = 0; i < d / 2; ++i) {
        const float c = cs[2 * i], s = cs[2 * i + 1];
        for (int h = 0; h < n_heads; ++h) {
            float *p = x + (int64_t)h * d + 2 * i;
            const float x0 = p[0], x1 = p[1];
            p[0] = x0 * c - x1 * s;
            p[1] = x0 * s + x1 * c;
        }
    }
}

/* embed, tp_llama.cpp:593-604: one Q4_0 row of token_embd, (n - 8) * d. */
void odec_embed(float *out, const uint8_t *token_embd, int token, int n_embd) {
    const uint8_t *row = token_embd + (int64_t)token * (n_embd / 32) * 18;
    for (int b = 0; b < n_embd / 32; ++b) {
        const uint8_t *blk = row + b * 18;
        const float d = oracle_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 16; ++j) {
            out[32 * b + j] = (float)((int)(blk[2 + j] & 0xF) - 8) * d;
            out[32 * b + j + 16] = (float)((int)(blk[2 + j] >> 4) - 8) * d;
        }
    }
}

/* silu_mul, tp_llama.cpp:615-622: act = (g / (1 + v_expf(-g))) * up. */
void odec_silu_mul(float *act, const float *gate, const float *up, int n) {
    for (int i = 0; i < n; ++i) {
        const float g = gate[i];
        const float sg = g / (1.0f + odec_v_expf(-g));
        act[i] = sg * up[i];
    }
}

/* softmax_exp, tp_llama.cpp:626-637: s[i] = v_expf(s[i] - mx); the first
 * n - n%4 values sum in four lanes (i mod 4), then (l0 + l1) + (l2 + l3),
 * then the tail one by one. */
static float softmax_exp(float *s, int n, float mx) {
    float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int i = 0;
    for (; i + 4 <= n; i += 4)
        for (int j = 0; j < 4; ++j) {
            const float e = odec_v_expf(s[i + j] - mx);
            s[i + j] = e;
            lane[j] = lane[j] + e;
        }
    float sum = (lane[0] + lane[1]) + (lane[2] + lane[3]);
    for (; i < n; ++i) {
        s[i] = odec_v_expf(s[i] - mx);
        sum = sum + s[i];
    }
    return sum;
}

static float kv_at(const void *base, int f16, int64_t idx) {
    if (f16) return oracle_f16_to_f32(((const uint16_t *)base)[idx]);
    return ((const float *)base)[idx];
}

/* attention_group, tp_llama.cpp:644-690. Scores: per position t, four
 * fused-multiply-add lanes over d (lane j takes i = j, j+4, ...), combined
 * as vaddvq_f32, times scale; running max from -1e30f. Output column c:
 * acc = fmaf(v[t][c], sc[t] * inv, acc) for t = 0..pos in order. */
void odec_attention(int B, const float *q, const void *kc, const void *vc, int f16, int64_t stride, int pos, int d,
                    float scale, float *sc, int sc_stride, float *out) {
    float mx[4], inv[4];
    for (int b = 0; b < B; ++b) mx[b] = -1e30f;
    for (int t = 0; t <= pos; ++t) {
        for (int b = 0; b < B; ++b) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int i = 0; i < d; i += 4)
                for (int j = 0; j < 4; ++j)
                    acc[j] = fmaf(kv_at(kc, f16, (int64_t)t * stride + i + j), q[b * d + i + j], acc[j]);
            const float sv = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * scale;
            sc[b * sc_stride + t] = sv;
            if (sv > mx[b]) mx[b] = sv;
        }
    }
    for (int b = 0; b < B; ++b) inv[b] = 1.0f / softmax_exp(sc + b * sc_stride, pos + 1, mx[b]);
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < d; ++c) {
            float acc = 0.0f;
            for (int t = 0; t <= pos; ++t) {
                const float p = sc[b * sc_stride + t] * inv[b];
                acc = fmaf(kv_at(vc, f16, (int64_t)t * stride + c), p, acc);
            }
            out[b * d + c] = acc;
        }
}

/* ------------------------------------------------------------------ model */

typedef struct {
    uint8_t *qkv, *o, *gateup, *down;
} shard_layer_t;

typedef struct {
    shard_layer_t *layers;
    uint8_t *lm_head;
    void *kcache, *vcache;  /* [layer][kv head][pos][head_dim] */
    float *qkv_y, *attn, *partial, *gu_y, *act, *logits, *scores;
} rank_t;

struct odec {
    odec_config_t c;
    int q_rows, kv_rows, ff_rows, vocab_rows, o_k, down_k;
    float **attn_norm, **ffn_norm, *output_norm, *rope_freqs;
    uint8_t *token_embd;
    rank_t *rank;
    float *x, *h, *cs, *sum;
};

/* copy_rows, tp_llama.cpp:191-197: rows [r0, r0+rows) of a [N, K] matrix. */
static void copy_rows(uint8_t *dst, int dst_row, const uint8_t *src, int k, int r0, int rows) {
    const int64_t rb = (int64_t)k / 32 * 18;
    memcpy(dst + (int64_t)dst_row * rb, src + (int64_t)r0 * rb, (size_t)(rb * rows));
}

/* copy_cols, tp_llama.cpp:201-207: columns [c0, c0+kk) of every row. */
static uint8_t *copy_cols(const uint8_t *src, int k, int n, int c0, int kk) {
    const int64_t rb = (int64_t)k / 32 * 18, ob = (int64_t)kk / 32 * 18, off = (int64_t)c0 / 32 * 18;
    uint8_t *m = malloc((size_t)(ob * n));
    if (!m) return NULL;
    for (int r = 0; r < n; ++r) memcpy(m + (int64_t)r * ob, src + (int64_t)r * rb + off, (size_t)ob);
    return m;
}

static float *copy_f32(const float *src, int n) {
    float *p = malloc(sizeof(float) * (size_t)n);
    if (p) memcpy(p, src, sizeof(float) * (size_t)n);
    return p;
}

void odec_destroy(odec_t *d) {
    if (!d) return;
    for (int r = 0; d->rank && r < d->c.nranks; ++r) {
        rank_t *R = &d->rank[r];
        for (int l = 0; R->layers && l < d->c.n_layer; ++l) {
            free(R->layers[l].qkv);
            free(R->layers[l].o);
            free(R->layers[l].gateup);
            free(R->layers[l].down);
        }
        free(R->layers);
        free(R->lm_head);
        free(R->kcache);
        free(R->vcache);
        free(R->qkv_y);
        free(R->attn);
        free(R->partial);
        free(R->gu_y);
        free(R->act);
        free(R->logits);
        free(R->scores);
    }
    for (int l = 0; d->attn_norm && l < d->c.n_layer; ++l) {
        free(d->attn_norm[l]);
        free(d->ffn_norm[l]);
    }
    free(d->attn_norm);
    free(d->ffn_norm);
    free(d->output_norm);
    free(d->rope_freqs);
    free(d->token_embd);
    free(d->rank);
    free(d->x);
    free(d->h);
    free(d->cs);
    free(d->sum);
    free(d);
}

int odec_create(odec_t **out, const odec_config_t *cfg, const odec_layer_t *layers, const uint8_t *token_embd,
                const float *output_norm) {
    if (!out || !cfg || !layers || !token_embd || !output_norm) return -2;
    *out = NULL;
    const odec_config_t c = *cfg;
    const int n = c.nranks;
    if (n < 1 || n > 8 || c.n_layer < 1 || c.head_dim % 16 || c.n_embd % 256 || c.n_ff % 256 || c.n_head % c.n_head_kv ||
        c.n_head % n || c.n_head_kv % n || c.n_vocab % n || c.ctx_max < 1 || c.n_embd != c.n_head * c.head_dim)
        return -1;
    odec_t *d = calloc(1, sizeof(odec_t));
    if (!d) return -2;
    d->c = c;
    d->q_rows = c.n_embd / n;
    d->kv_rows = c.n_head_kv * c.head_dim / n;
    d->ff_rows = c.n_ff / n;
    d->vocab_rows = c.n_vocab / n;
    d->o_k = c.n_embd / n;
    d->down_k = c.n_ff / n;
    if (d->o_k % 32 || d->down_k % 256) {  /* o_k % 256: the lane-rule extension (gemv above) */
        free(d);
        return -1;
    }
    const int e = c.n_embd;
    const int64_t erb = (int64_t)e / 32 * 18;
    d->attn_norm = calloc((size_t)c.n_layer, sizeof(float *));
    d->ffn_norm = calloc((size_t)c.n_layer, sizeof(float *));
    d->rank = calloc((size_t)n, sizeof(rank_t));
    d->token_embd = malloc((size_t)(erb * c.n_vocab));
    d->output_norm = copy_f32(output_norm, e);
    d->x = calloc((size_t)e, 4);
    d->h = calloc((size_t)e, 4);
    d->cs = calloc((size_t)c.head_dim, 4);
    d->sum = calloc((size_t)(c.n_embd > c.n_ff ? c.n_embd : c.n_ff), 4);
    if (!d->attn_norm || !d->ffn_norm || !d->rank || !d->token_embd || !d->output_norm || !d->x || !d->h || !d->cs ||
        !d->sum) {
        odec_destroy(d);
        return -2;
    }
    memcpy(d->token_embd, token_embd, (size_t)(erb * c.n_vocab));
    for (int l = 0; l < c.n_layer; ++l) {
        d->attn_norm[l] = copy_f32(layers[l].attn_norm, e);
        d->ffn_norm[l] = copy_f32(layers[l].ffn_norm, e);
        if (!d->attn_norm[l] || !d->ffn_norm[l]) {
            odec_destroy(d);
            return -2;
        }
    }
    const int kvh_local = c.n_head_kv / n;
    const size_t kv_elems = (size_t)c.n_layer * kvh_local * c.ctx_max * c.head_dim;
    const size_t kv_bytes = kv_elems * (c.kv_f16 ? 2 : 4);
    for (int r = 0; r < n; ++r) {
        rank_t *R = &d->rank[r];
        R->layers = calloc((size_t)c.n_layer, sizeof(shard_layer_t));
        R->lm_head = malloc((size_t)(erb * d->vocab_rows));
        R->kcache = calloc(kv_bytes, 1);
        R->vcache = calloc(kv_bytes, 1);
        R->qkv_y = calloc((size_t)(d->q_rows + 2 * d->kv_rows), 4);
        R->attn = calloc((size_t)e, 4);
        R->partial = calloc((size_t)e, 4);
        R->gu_y = calloc((size_t)(2 * d->ff_rows), 4);
        R->act = calloc((size_t)d->ff_rows, 4);
        R->logits = calloc((size_t)d->vocab_rows, 4);
        R->scores = calloc((size_t)4 * c.ctx_max * (c.n_head_kv / n), 4);   /* one score block per KV head */
        if (!R->layers || !R->lm_head || !R->kcache || !R->vcache || !R->qkv_y || !R->attn || !R->partial ||
            !R->gu_y || !R->act || !R->logits || !R->scores) {
            odec_destroy(d);
            return -2;
        }
        /* load_model, tp_llama.cpp:255-279 */
        copy_rows(R->lm_head, 0, token_embd, e, r * d->vocab_rows, d->vocab_rows);
        for (int l = 0; l < c.n_layer; ++l) {
            shard_layer_t *L = &R->layers[l];
            const odec_layer_t *W = &layers[l];
            L->qkv = malloc((size_t)(erb * (d->q_rows + 2 * d->kv_rows)));
            L->gateup = malloc((size_t)(erb * 2 * d->ff_rows));
            if (!L->qkv || !L->gateup) {
                odec_destroy(d);
                return -2;
            }
            copy_rows(L->qkv, 0, W->attn_q, e, r * d->q_rows, d->q_rows);
            copy_rows(L->qkv, d->q_rows, W->attn_k, e, r * d->kv_rows, d->kv_rows);
            copy_rows(L->qkv, d->q_rows + d->kv_rows, W->attn_v, e, r * d->kv_rows, d->kv_rows);
            L->o = copy_cols(W->attn_output, e, e, r * d->o_k, d->o_k);
            copy_rows(L->gateup, 0, W->ffn_gate, e, r * d->ff_rows, d->ff_rows);
            copy_rows(L->gateup, d->ff_rows, W->ffn_up, e, r * d->ff_rows, d->ff_rows);
            L->down = copy_cols(W->ffn_down, c.n_ff, e, r * d->down_k, d->down_k);
            if (!L->o || !L->down) {
                odec_destroy(d);
                return -2;
            }
        }
    }
    *out = d;
    return 0;
}

/* engine_t::gemv (tp_llama.cpp:355-374): quantize_x, then the contract's
 * GEMV. A K-split shard whose block count is not a multiple of 8 (the 3B
 * model's attn_output at 8 ranks: 12 blocks) uses the lane rule b mod 8 as
 * it stands for any count -- a contract extension: q4_0.py:166-167 and
 * load_model (tp_llama.cpp:247) refuse such shards. */
static void gemv(const odec_t *d, const uint8_t *W, int rows, int k, const float *x, float *y) {
    if (k % 256 == 0) {
        oracle_gemv_q4_0_f32(W, rows, k, x, y, d->c.threads, d->c.round_mode);
        return;
    }
    int8_t *xq = (int8_t *)malloc((size_t)k);
    uint16_t *xd = (uint16_t *)malloc((size_t)(k / 32) * 2);
    if (xq && xd && !oracle_quantize_q8_0(x, k, xq, xd, d->c.round_mode))
        oracle_gemv_q4_0(W, rows, k, xq, xd, y, d->c.threads, 1);
    free(xq);
    free(xd);
}

/* rank-ordered all-reduce of every rank's `partial` (tp_llama.cpp:515-521),
 * then add_into(x, sum) (tp_llama.cpp:609-612). */
static void allreduce_add(odec_t *d) {
    const int e = d->c.n_embd;
    for (int i = 0; i < e; ++i) {
        float s = d->rank[0].partial[i];
        for (int r = 1; r < d->c.nranks; ++r) s = s + d->rank[r].partial[i];
        d->x[i] = d->x[i] + s;
    }
}

/* sample_token with temperature 0 (tp_llama.cpp:894-925): every rank keeps
 * the top_k (40) of its shard by insertion (strict >, so the lower index
 * stays first on a tie), the candidates of all ranks are sorted by value
 * descending then index ascending, and the first one wins. */
static void pick(const odec_t *d, int *tok, float *val) {
    enum { K = 40 };
    const int n = d->c.nranks;
    float av[8 * K] = {0.0f};
    int ai[8 * K] = {0};
    int na = 0;
    for (int r = 0; r < n; ++r) {
        float mv[K];
        int mi[K];
        for (int j = 0; j < K; ++j) {
            mv[j] = -1e30f;
            mi[j] = 0;
        }
        const float *y = d->rank[r].logits;
        for (int i = 0; i < d->vocab_rows; ++i) {
            const float v = y[i];
            if (v <= mv[K - 1]) continue;
            int p = K - 1;
            while (p > 0 && mv[p - 1] < v) {
                mv[p] = mv[p - 1];
                mi[p] = mi[p - 1];
                --p;
            }
            mv[p] = v;
            mi[p] = i + r * d->vocab_rows;
        }
        for (int j = 0; j < K; ++j) {
            av[na] = mv[j];
            ai[na] = mi[j];
            ++na;
        }
    }
    int best = 0;
    for (int j = 1; j < na; ++j)
        if (av[j] > av[best] || (av[j] == av[best] && ai[j] < ai[best])) best = j;
    *tok = ai[best];
    *val = av[best];
}

/* attention of (rank, KV head) items [lo, hi) of one layer at one position:
 * the query heads of each KV head in groups of up to 4 (tp_llama.cpp:849-856) */
typedef struct {
    odec_t *d;
    int l, pos;
    float scale;
} attn_job_t;

static void attention_span(void *ctx, int64_t lo, int64_t hi) {
    const attn_job_t *J = (const attn_job_t *)ctx;
    const odec_t *d = J->d;
    const odec_config_t *c = &d->c;
    const int hd = c->head_dim, kvh_local = c->n_head_kv / c->nranks, group = c->n_head / c->n_head_kv;
    const int esz = c->kv_f16 ? 2 : 4;
    for (int64_t it = lo; it < hi; ++it) {
        const int r = (int)(it / kvh_local), kvh = (int)(it % kvh_local);
        const rank_t *R = &d->rank[r];
        const float *q = R->qkv_y;
        const int64_t base = ((int64_t)J->l * kvh_local + kvh) * c->ctx_max * hd;
        const void *kc0 = (const uint8_t *)R->kcache + base * esz;
        const void *vc0 = (const uint8_t *)R->vcache + base * esz;
        float *sc = R->scores + (int64_t)kvh * 4 * c->ctx_max;
        for (int g0 = 0; g0 < group; g0 += 4) {
            const int hq = kvh * group + g0;
            const int B = group - g0 < 4 ? group - g0 : 4;
            odec_attention(B, q + hq * hd, kc0, vc0, c->kv_f16, hd, J->pos, hd, J->scale, sc, c->ctx_max,
                           R->attn + hq * hd);
        }
    }
}

int odec_set_rope_freqs(odec_t *d, const float *freqs) {
    if (!d) return -2;
    free(d->rope_freqs);
    d->rope_freqs = freqs ? copy_f32(freqs, d->c.head_dim / 2) : NULL;
    return freqs && !d->rope_freqs ? -2 : 0;
}

int odec_forward(odec_t *d, int token, int pos, int *tok, float *val) {
    if (!d || !tok || !val) return -2;
    const odec_config_t *c = &d->c;
    if (token < 0 || token >= c->n_vocab || pos < 0 || pos >= c->ctx_max) return -2;
    const int n = c->nranks, e = c->n_embd, hd = c->head_dim;
    const int heads_local = c->n_head / n, kvh_local = c->n_head_kv / n;
    const float scale = 1.0f / sqrtf((float)hd);
    odec_embed(d->x, d->token_embd, token, e);
    odec_rope_table_freqs(d->cs, hd, pos, c->rope_base, d->rope_freqs);
    for (int l = 0; l < c->n_layer; ++l) {
        odec_rmsnorm(d->h, d->x, d->attn_norm[l], e, c->rms_eps);
        for (int r = 0; r < n; ++r) {
            rank_t *R = &d->rank[r];
            shard_layer_t *L = &R->layers[l];
            gemv(d, L->qkv, d->q_rows + 2 * d->kv_rows, e, d->h, R->qkv_y);
            float *q = R->qkv_y, *k = R->qkv_y + d->q_rows, *v = R->qkv_y + d->q_rows + d->kv_rows;
            odec_rope(q, heads_local, hd, d->cs);
            odec_rope(k, kvh_local, hd, d->cs);
            for (int kvh = 0; kvh < kvh_local; ++kvh) {
                const int64_t at = (((int64_t)l * kvh_local + kvh) * c->ctx_max + pos) * hd;
                for (int i = 0; i < hd; ++i) {
                    if (c->kv_f16) {
                        ((uint16_t *)R->kcache)[at + i] = oracle_f32_to_f16(k[kvh * hd + i]);
                        ((uint16_t *)R->vcache)[at + i] = oracle_f32_to_f16(v[kvh * hd + i]);
                    } else {
                        ((float *)R->kcache)[at + i] = k[kvh * hd + i];
                        ((float *)R->vcache)[at + i] = v[kvh * hd + i];
                    }
                }
            }
        }
        /* the KV heads are independent (each has its own score rows): run
         * them side by side, each in the reference's order */
        attn_job_t job = {d, l, pos, scale};
        oracle_parallel_for((int64_t)n * kvh_local, c->threads, attention_span, &job);
        for (int r = 0; r < n; ++r) gemv(d, d->rank[r].layers[l].o, e, d->o_k, d->rank[r].attn, d->rank[r].partial);
        allreduce_add(d);
        odec_rmsnorm(d->h, d->x, d->ffn_norm[l], e, c->rms_eps);
        for (int r = 0; r < n; ++r) {
            rank_t *R = &d->rank[r];
            shard_layer_t *L = &R->layers[l];
            gemv(d, L->gateup, 2 * d->ff_rows, e, d->h, R->gu_y);
            odec_silu_mul(R->act, R->gu_y, R->gu_y + d->ff_rows, d->ff_rows);
            gemv(d, L->down, e, d->down_k, R->act, R->partial);
        }
        allreduce_add(d);
    }
    odec_rmsnorm(d->h, d->x, d->output_norm, e, c->rms_eps);
    for (int r = 0; r < n; ++r) gemv(d, d->rank[r].lm_head, d->vocab_rows, e, d->h, d->rank[r].logits);
    pick(d, tok, val);
    return 0;
}

int odec_generate(odec_t *d, const int *prompt, int n_prompt, int n_gen, int *out) {
    if (!d || !prompt || !out || n_prompt < 1 || n_gen < 1 || n_prompt + n_gen - 1 > d->c.ctx_max) return -2;
    int tok = 0;
    float val = 0.0f;
    for (int i = 0; i < n_prompt; ++i) {
        const int rc = odec_forward(d, prompt[i], i, &tok, &val);
        if (rc) return rc;
    }
    for (int i = 0; i < n_gen; ++i) {
        out[i] = tok;
        if (i + 1 == n_gen) break;
        const int rc = odec_forward(d, tok, n_prompt + i, &tok, &val);
        if (rc) return rc;
    }
    return 0;
}

int odec_read(odec_t *d, int what, int rank, float *out, int64_t n) {
    if (!d || !out) return -2;
    if (what == 0 && n == d->c.n_embd) {
        memcpy(out, d->x, sizeof(float) * (size_t)n);
        return 0;
    }
    if (what == 1 && rank >= 0 && rank < d->c.nranks && n == d->vocab_rows) {
        memcpy(out, d->rank[rank].logits, sizeof(float) * (size_t)n);
        return 0;
    }
    if (what == 2 && n == d->c.n_embd) {
        memcpy(out, d->h, sizeof(float) * (size_t)n);
        return 0;
    }
    return -2;
}
