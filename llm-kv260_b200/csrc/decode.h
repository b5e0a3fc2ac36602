// Internal host-side interface of the decoder's own kernels (attn.cu) and of
// the communicator internals the decoder uses (comm.cu). Not part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/b200_comm.h"
#include "../../include/b200_decoder.h"
#include "q4gemv.h"

namespace b200 {

struct AttnLaunch {
    const float *q = nullptr;       // this rank's roped q rows: [heads_local][head_dim]
    const void *kcache = nullptr;   // this layer's K cache [kv head][kv_stride][head_dim]
    const void *vcache = nullptr;   // and V^T cache [kv head][head_dim][kv_stride] (attn_core.cuh)
    float *out = nullptr;           // [heads_local][head_dim]
    const int *pos = nullptr;       // current position (device)
    int head_dim = 0;               // 64 or 128
    int group = 0;                  // query heads per KV head, 1..4
    int kvh_local = 0;              // KV heads on this rank (one CTA each)
    int ctx_max = 0;
    int kv_stride = 0;              // attn_kv_stride(ctx_max): positions per head in the caches
    int kv_f16 = 1;
    float scale = 0.0f;             // 1 / sqrtf(head_dim)
    bool pdl = true;
    uint64_t *trace = nullptr;      // optional launch trace (q4gemv.h, kTraceCtas)
};

int attn_kv_stride(int ctx_max);  // ctx_max rounded up to a multiple of 8

// The configuration a decoder was created with (decoder.cu; for the GGUF loader).
int decoder_config(const b200_decoder_t *d, b200_decoder_config_t *out);
int attn_smem_bytes(int head_dim, int kv_f16, int ctx_max);       // the cluster kernel (short contexts)
int attn_smem_bytes_long(int head_dim, int kv_f16, int ctx_max);  // the streaming kernel it falls to
int attn_launch(const AttnLaunch &L, cudaStream_t stream);

// ------------------------------------------------------- persistent token kernel
// token.cu: one cooperative launch runs `ntokens` decode tokens, each a list
// of phases (a GEMV over row groups, or attention) separated by grid-wide
// barriers, with every CTA's weight bytes streamed ahead through a
// shared-memory ring independent of the barriers.
enum PhaseKind : int { kPhGemv = 0, kPhAttn = 1 };

struct TokenPhase {
    int kind = kPhGemv;
    const uint8_t *w = nullptr;  // GEMV: tiles
    int rows = 0, k = 0;
    int pro = kProPlain, epi = kEpiStore;
    const float *x = nullptr;       // kProPlain input [k]
    const float *norm_w = nullptr;  // RMSNorm weight [k]
    float *y = nullptr;             // kEpiStore / kEpiRopeKv output
    float *act = nullptr;           // kEpiSiluPairs output
    void *kcache = nullptr;         // this layer's caches (kEpiRopeKv, attention)
    void *vcache = nullptr;
    int ar_index = 0;               // kEpiResidual: exchange index within the token
    int pick = 0;                   // 1: the greedy pick over y (lm_head)
    const float *q = nullptr;       // attention: roped q rows
    float *out = nullptr;           // attention output
};

constexpr int kMaxTokenPhases = 5 * 32 + 1;

struct TokenArgs {
    const TokenPhase *phases = nullptr;  // device array
    int nphases = 0;
    int ntokens = 0;
    float *res = nullptr;                // residual stream [n_embd]
    const uint8_t *embd = nullptr;       // token_embd GGUF rows
    int *tokens = nullptr;               // token id by position [ctx_max + 1]
    int *pos = nullptr;                  // loop state (read at start, written by CTA 0)
    unsigned *step = nullptr;
    const int *n_prompt = nullptr;
    int *pick_out = nullptr;             // the last pick: int32 token, float32 value
    float2 *cand = nullptr;              // per-CTA pick candidates [grid]
    const float *logits = nullptr;       // lm_head output (for the NaN-at-0 rule)
    const float *rope_cs = nullptr;
    int n_embd = 0, head_dim = 0, q_rows = 0, kv_rows = 0, ctx_max = 0, kv_f16 = 1, group = 0, kvh_local = 0;
    int kv_stride = 0;                   // positions per head in the caches (attn_kv_stride)
    int vocab_base = 0;
    float scale = 0.0f, eps = 0.0f;
    int exact_norm = 0, round_mode = 0;
    int nranks = 1, rank = 0;
    uint64_t *win_words[kMaxDecodeRanks] = {};
    uint64_t slot_words = 0;
    int ar_per_token = 0;
    unsigned *peer_status = nullptr;
    unsigned long long *bar_count = nullptr;  // grid barrier arrivals, only ever incremented
    int *abort_flag = nullptr;
    unsigned *status = nullptr;
    int *host_tokens = nullptr;          // mapped host memory: token ids by position, written as made (or null)
    uint64_t *trace = nullptr;           // optional: [token < trace_tokens][phase][CTA][4] global-timer stamps
    int trace_tokens = 0;
};

// Shared memory and consumer warpgroups the kernel needs for these args;
// 0 or kErrInval.
int token_kernel_plan(const TokenArgs &a, int *smem_bytes, int *ring_stages, int *wgs, int *grid);
int token_kernel_launch(const TokenArgs &a, cudaStream_t stream);

// The all-reduce word area of a communicator's windows (comm.cu): every
// rank's mapping in this process, words per (slot, source rank), and the
// status word a timed-out wait marks.
int comm_word_area(b200_comm_t *c, uint64_t *win_words[kMaxDecodeRanks], uint64_t *slot_words, unsigned **status,
                   int *rank, int *nranks);

}  // namespace b200
