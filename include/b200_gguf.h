/*
 * GGUF model loading for the decoder: the B200 counterpart of the reference
 * runtime's gguf_file and load_model (board/tp/tp_llama.cpp:149-188 and
 * 226-283). A GGUF v2/v3 file is mapped read-only; its llama.* keys give the
 * decoder's hyperparameters, and its Q4_0 / float32 tensors go to
 * b200_decoder_set_layer / _set_output / _set_rope_freqs, which cut this
 * rank's shard exactly as load_model does. Host code only.
 *
 * All functions return 0 or a negative errno value; b200_last_error() says
 * why.
 */
#ifndef B200_GGUF_H
#define B200_GGUF_H

#include <stdint.h>

#include "b200_decoder.h"

#ifndef B200_API
#define B200_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_gguf b200_gguf_t;

/* ggml tensor types the loader knows the size of */
enum { B200_GGML_F32 = 0, B200_GGML_F16 = 1, B200_GGML_Q4_0 = 2, B200_GGML_Q8_0 = 8 };

/* gguf_file::open (tp_llama.cpp:154-166): map `path` and read the header,
 * the key/value pairs and the tensor infos (the data section starts at the
 * next multiple of general.alignment, 32 when absent). -EINVAL for a file
 * that is not GGUF v2/v3 or whose tensors lie outside it. */
B200_API int b200_gguf_open(b200_gguf_t **g, const char *path);
B200_API void b200_gguf_close(b200_gguf_t *g);

/* load_model's hyperparameters (tp_llama.cpp:228-236): llama.block_count,
 * .embedding_length, .feed_forward_length, .attention.head_count,
 * .attention.head_count_kv, .vocab_size (when absent: token_embd's rows),
 * head_dim = n_embd / n_head, .rope.freq_base (10000 when absent),
 * .attention.layer_norm_rms_epsilon (1e-5 when absent). Writes those fields
 * of *cfg and leaves the others (ctx_max, kv_f16, ...) as they are. */
B200_API int b200_gguf_config(const b200_gguf_t *g, b200_decoder_config_t *cfg);

/* A tensor by name (gguf_file::data, tp_llama.cpp:175-179): its host
 * address inside the mapping, its byte count (0 for a type listed above as
 * unknown), its ggml type and its dimensions ne[0..3] (ne[0] innermost,
 * unused ones 1). -ENOENT when the file has no such tensor. Any output
 * pointer may be NULL. */
B200_API int b200_gguf_tensor(const b200_gguf_t *g, const char *name, const void **data, uint64_t *bytes, int *type,
                              int64_t ne[4]);

/* load_model (tp_llama.cpp:238-283) into a decoder created from
 * b200_gguf_config's hyperparameters: blk.N.{attn_q, attn_k, attn_v,
 * attn_output, ffn_gate, ffn_up, ffn_down} (Q4_0) and {attn_norm, ffn_norm}
 * (float32) for every layer, token_embd (Q4_0, also the tied lm_head) and
 * output_norm, and rope_freqs when the file holds it. Every tensor's type
 * and shape is checked against the hyperparameters first. The file may be
 * closed afterwards: the decoder keeps device copies. */
B200_API int b200_decoder_load_gguf(b200_decoder_t *d, const b200_gguf_t *g);

#ifdef __cplusplus
}
#endif
#endif
