/*
 * Greedy batch-1 decoder: the B200 counterpart of the reference runtime's
 * decode loop, struct runtime (board/tp/tp_llama.cpp:783-968): forward()
 * (822-883), the greedy branch of sample_token() (895-925) and generate()
 * (942-968), with the weights sharded over nranks exactly as load_model
 * shards them (tp_llama.cpp:238-283).
 *
 * Every op keeps the reference's arithmetic order, so a rank's logits and
 * tokens are bit-identical to the reference's CPU path at the same nranks:
 * the Q4_0 x Q8_0 GEMVs are the contract's (src/llm_kv260/q4_0.py:185-188),
 * RMSNorm sums squares in double in four lanes (557-569), RoPE uses a host
 * table from powf/cosf/sinf (574-591), attention runs its fused-multiply-add
 * chains in the reference's order (644-690), SiLU uses ggml's v_expf
 * (530-553, 615-622), and the K-split partials are summed in rank order
 * (515-521). The one deviation BASELINE asks for is optional: kv_f16 = 1
 * keeps the KV cache in float16 (round to nearest even) where the reference
 * keeps float32.
 *
 * On the device (persistent = 0) a token is one CUDA graph of 5 kernels per
 * layer + lm_head (RMSNorm, embedding, RoPE + KV store, SiLU, the residual
 * adds and the cross-rank exchange are fused into the GEMVs; the greedy pick
 * into lm_head); with persistent = 1 one cooperative kernel runs a whole run
 * of tokens as phases between grid barriers. Either way the position, step
 * and token ids live in device memory, so the loop needs no host work
 * between tokens. A decoder whose bounded wait ran out (status non-zero) is
 * not usable afterwards; destroy it.
 *
 * All functions return 0 or a negative errno value; b200_last_error() says
 * why. Pointers to weights are HOST pointers to the full (unsharded) GGUF
 * tensors, Q4_0 rows of 18-byte blocks, as a GGUF file holds them.
 */
#ifndef B200_DECODER_H
#define B200_DECODER_H

#include <stdint.h>

#include "b200_comm.h"

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_decoder b200_decoder_t;

/* hparams (tp_llama.cpp:123-126) plus the decoder's own choices. */
typedef struct {
    int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab;
    float rope_base, rms_eps;
    int ctx_max;     /* positions the KV cache holds (runtime::init, tp_llama.cpp:809-815) */
    int kv_f16;      /* 1: float16 KV cache (BASELINE's), 0: float32 (the reference's) */
    int round_mode;  /* Q8_0 rounding of the GEMV input: 0 floor(|s|+0.5f) (q4_0.py:96), 1 roundf (tp_llama.cpp:343) */
    int exact_norm;  /* 1: RMSNorm always sums squares sequentially (same bits, slower); 0: only when it matters */
    int persistent;  /* 1: one persistent kernel runs whole runs of tokens (one CTA per SM, weights streamed
                        across phase barriers); 0: a CUDA graph of per-op kernels per token. Same bits. */
} b200_decoder_config_t;

/* One rank's decoder on `device`. nranks > 1 needs `comm`: a communicator of
 * this rank created for at least n_embd + 2 floats, with its peers' handles
 * imported, used by this decoder only. The shard constraints of load_model
 * apply (tp_llama.cpp:246-247): n_embd, n_embd/nranks and n_ff/nranks
 * multiples of 256 and <= 8192; head_dim 64 or 128; n_head/n_head_kv <= 4. */
B200_API int b200_decoder_create(b200_decoder_t **d, const b200_decoder_config_t *cfg, int device, int rank,
                                 int nranks, b200_comm_t *comm);

/* Layer `layer`'s tensors (load_model, tp_llama.cpp:255-272): attn_q
 * [n_embd][n_embd], attn_k and attn_v [n_head_kv*head_dim][n_embd],
 * attn_output [n_embd][n_embd], ffn_gate and ffn_up [n_ff][n_embd],
 * ffn_down [n_embd][n_ff] as Q4_0 rows; attn_norm and ffn_norm float32
 * [n_embd]. This rank's shard is cut, copied to the device and re-laid. */
B200_API int b200_decoder_set_layer(b200_decoder_t *d, int layer, const void *attn_q, const void *attn_k,
                                    const void *attn_v, const void *attn_output, const void *ffn_gate,
                                    const void *ffn_up, const void *ffn_down, const float *attn_norm,
                                    const float *ffn_norm);

/* token_embd [n_vocab][n_embd] Q4_0 rows (the embedding table and, tied, the
 * lm_head, tp_llama.cpp:279) and output_norm float32 [n_embd]. */
B200_API int b200_decoder_set_output(b200_decoder_t *d, const void *token_embd, const float *output_norm);

/* runtime::forward(token, pos) then the greedy pick over all ranks: *pick is
 * the token, *value its logit. Every rank must make the same calls. Waits
 * for work queued earlier, then (graph mode) launches one CUDA graph -- the
 * inputs in, the token, the pick and status words out -- and waits for it;
 * the first call captures that graph. */
B200_API int b200_decoder_forward(b200_decoder_t *d, int token, int pos, int32_t *pick, float *value);

/* The same loop, queued without waiting (for callers that time or overlap
 * it): prefill sets the prompt and queues its n_prompt forwards; step queues
 * n more forwards, each taking the previous pick as its token. Neither waits
 * for the device; read buffer 2 (the token ids) afterwards. */
B200_API int b200_decoder_prefill(b200_decoder_t *d, const int32_t *prompt, int n_prompt);
B200_API int b200_decoder_step(b200_decoder_t *d, int n);

/* runtime::generate with temperature 0 and no end-of-generation token:
 * prompt positions 0..n_prompt-1, then n_gen tokens into out (n_prompt +
 * n_gen - 1 forwards; n_prompt + n_gen - 1 <= ctx_max). Each token is copied
 * to the host as it is made. prompt_ms and gen_ms (either may be NULL) receive
 * the device time of the prompt's forwards and of the generation phase: the
 * remaining n_gen - 1 forwards and the n_gen token copies. */
B200_API int b200_decoder_generate(b200_decoder_t *d, const int32_t *prompt, int n_prompt, int n_gen, int32_t *out,
                                   double *prompt_ms, double *gen_ms);

/* Copy a device buffer of the last forward to the host (bytes must match):
 * 0 residual x float32[n_embd], 1 this rank's logits float32[n_vocab/nranks],
 * 2 token ids int32[ctx_max+1], 3 the pick (int32 token, float32 value),
 * 4 the q|k|v rows float32[q+k+v shard rows], 5 the attention output
 * float32[n_embd/nranks], 6 SiLU(gate)*up float32[n_ff/nranks], 7 the phase
 * trace (b200_decoder_trace). */
B200_API int b200_decoder_read(b200_decoder_t *d, int what, void *host, uint64_t bytes);

/* Persistent mode: record a phase trace of the first `tokens` (<= 64) tokens
 * of each later launch -- per (token, phase, CTA) eight values from the
 * device global timer in ns: 0 phase start (its barrier passed), 1 x staged,
 * 2 warpgroup 0's rows done, 3 phase end, 4 and 5 the time warpgroups 0 and 1
 * waited for weight stages, 6 warpgroup 1's rows done, 7 unused -- read back
 * as buffer 7 (uint64[tokens][phases][SMs][8]).
 * Graph mode (tokens 0 or 1): every token run records its 5 * n_layer + 1
 * kernel launches (per layer q|k|v, attention, o, gate|up, down; then
 * lm_head), overwriting the previous token's -- per (launch, CTA < 1024)
 * sixteen stamps: 0 CTA set up, 1 the previous kernel's results visible, 2
 * input staged (attention: p computed), 3 CTA end, and for attention 4 q
 * staged, 5 scores and maxima, 6 exponentials, 7 sums, 8 + 2c / 9 + 2c V
 * chunk c (< 4) landed / consumed; read back as buffer 7
 * (uint64[launches][1024][16], zero where a launch has no such CTA or stamp).
 * 0 turns tracing off. A B200 extension with no reference counterpart. */
B200_API int b200_decoder_trace(b200_decoder_t *d, int tokens);

/* Device status: bit 1 a weight copy wait ran out, bit 2 a peer wait ran
 * out (the outputs since are not valid). Reading clears it. */
B200_API int b200_decoder_status(b200_decoder_t *d, unsigned *status);

/* The model's RoPE frequency factors (rope_freqs.weight, head_dim/2 positive
 * floats; tp_llama.cpp:282 loads them, 577-578 divides each angle by its
 * factor), or NULL for none (the default). Recomputes the decoder's table. */
B200_API int b200_decoder_set_rope_freqs(b200_decoder_t *d, const float *freqs);

/* The RoPE table the decoder uploads (rope_table, tp_llama.cpp:574-580):
 * cs[2i] = cosf(theta_i), cs[2i+1] = sinf(theta_i), theta_i = pos *
 * powf(base, -2i/d), divided by freqs[i] when freqs is not NULL, computed on
 * the host. b200_rope_table is the same without factors. No reference
 * counterpart as a function; exported so a caller can check the table. */
B200_API int b200_rope_table(float *cs, int d, int pos, float base);
B200_API int b200_rope_table_freqs(float *cs, int d, int pos, float base, const float *freqs);

/* The cost of the decoder's launch chain alone: `launches` empty kernels of
 * `ctas` CTAs x `threads` threads, each asking for `smem` bytes of dynamic
 * shared memory, captured into one CUDA graph on device `device` -- with
 * programmatic dependent launch when `pdl` is nonzero (each kernel lets its
 * dependents launch at once, then waits for its predecessor, as the
 * decoder's kernels do), else plain stream order -- replayed `reps` times
 * after three untimed replays and timed with CUDA events. *us_per_launch =
 * the mean time per launch in microseconds. A B200 diagnostic with no
 * reference counterpart. */
B200_API int b200_launch_floor(int device, int launches, int ctas, int threads, int smem, int pdl, int reps,
                               float *us_per_launch);

/* The decoder's CUDA stream (cudaStream_t). */
B200_API void *b200_decoder_stream(b200_decoder_t *d);

B200_API int b200_decoder_destroy(b200_decoder_t *d);

#ifdef __cplusplus
}
#endif
#endif
