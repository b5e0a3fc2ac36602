/*
 * CPU oracle for the decode step of the reference runtime, board/tp/tp_llama.cpp
 * (runtime::forward 822-883, its ops 528-705, the greedy branch of
 * sample_token 894-925). TEST INFRASTRUCTURE ONLY: the parity tests, the
 * smoke check and the bench's CPU arms link it as the checker; the product
 * never calls it.
 *
 * The reference's ops are NEON code; this file restates them per lane in
 * plain C compiled with -ffp-contract=off, so every rounding the NEON code
 * does happens here exactly once and no other:
 *   vfmaq_f32(a, b, c)  = fmaf(b, c, a)      (fused, one rounding)
 *   vaddvq_f32(v)       = (v0 + v1) + (v2 + v3)   (GCC's faddp lowering on
 *                          AArch64 -- an assumption, the only one here)
 *   vaddvq_f64(v)       = v0 + v1
 * The GEMVs are the contract's (q4_0.py:185-188) through q4_0_oracle.c.
 *
 * Tensor parallelism is simulated: nranks shards of every matrix cut exactly
 * as load_model does (tp_llama.cpp:238-283: copy_rows for q, k, v, gate, up
 * and lm_head; copy_cols for attn_output and ffn_down), each rank's partial
 * sums combined with the rank-ordered all-reduce (tp_llama.cpp:515-521).
 *
 * Parity of this restatement with the reference itself is UNPINNED: the
 * runtime needs <arm_neon.h>, libllama and a real model, none of which exist
 * here, so it has never been run against it.
 *
 * Deviation BASELINE imposes: kv_f16 = 1 stores the KV cache as float16
 * (round to nearest even) instead of the reference's float32
 * (tp_llama.cpp:792,814-815); kv_f16 = 0 is the reference's cache.
 *
 * Return codes: 0 ok, -1 bad configuration, -2 bad argument.
 */
#ifndef DECODE_ORACLE_H
#define DECODE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab;
    float rope_base, rms_eps;
    int ctx_max;
    int kv_f16;      /* 1: float16 KV cache (RNE on store), 0: float32 */
    int nranks;      /* tensor-parallel ranks simulated here */
    int round_mode;  /* Q8 rounding of the engine calls (q4_0_oracle.h) */
    int threads;     /* GEMV threads */
} odec_config_t;

/* One layer's tensors, full (unsharded), GGUF Q4_0 rows, and its norms. */
typedef struct {
    const uint8_t *attn_q, *attn_k, *attn_v, *attn_output, *ffn_gate, *ffn_up, *ffn_down;
    const float *attn_norm, *ffn_norm;
} odec_layer_t;

typedef struct odec odec_t;

/* Shards every tensor for cfg->nranks ranks (copies; the caller's arrays may
 * go away after). token_embd [n_vocab, n_embd] is also the tied lm_head. */
int odec_create(odec_t **out, const odec_config_t *cfg, const odec_layer_t *layers, const uint8_t *token_embd,
                const float *output_norm);
void odec_destroy(odec_t *d);

/* runtime::forward(token, pos) on every rank, then sample_token's greedy
 * pick over all ranks: *pick = the token, *value = its logit. */
int odec_forward(odec_t *d, int token, int pos, int *pick, float *value);

/* The model's rope_freqs factors (head_dim/2 floats, tp_llama.cpp:577-578,
 * 282), or NULL for none (the default). */
int odec_set_rope_freqs(odec_t *d, const float *freqs);

/* runtime::generate (tp_llama.cpp:942-968) with temperature 0 and no EOG:
 * the prompt at positions 0..n_prompt-1, then n_gen tokens into out
 * (n_prompt + n_gen - 1 forward calls). */
int odec_generate(odec_t *d, const int *prompt, int n_prompt, int n_gen, int *out);

/* Buffers after the last forward: what = 0 the residual x [n_embd],
 * 1 rank `rank`'s logits [n_vocab / nranks], 2 the final normed h [n_embd]. */
int odec_read(odec_t *d, int what, int rank, float *out, int64_t n);

/* The ops on their own, for tests. */
float odec_v_expf(float x);                                              /* tp_llama.cpp:530-553 */
void odec_rmsnorm(float *out, const float *x, const float *w, int n, float eps);   /* 557-569 */
void odec_rope_table(float *cs, int d, int pos, float base);            /* 574-580, no freq factors */
void odec_rope_table_freqs(float *cs, int d, int pos, float base, const float *freqs);   /* 574-580 */
void odec_rope(float *x, int n_heads, int d, const float *cs);          /* 581-591 */
void odec_silu_mul(float *act, const float *gate, const float *up, int n);   /* 615-622 */
void odec_embed(float *out, const uint8_t *token_embd, int token, int n_embd);   /* 593-604 */
/* attention_group (tp_llama.cpp:644-690) for B query heads sharing one KV
 * head; k/v rows `stride` elements apart, float32 (f16 = 0) or float16 bits. */
void odec_attention(int B, const float *q, const void *kc, const void *vc, int f16, int64_t stride, int pos, int d,
                    float scale, float *sc, int sc_stride, float *out);

#ifdef __cplusplus
}
#endif
#endif
