// Internal host-side interface of the decoder's own kernels (attn.cu) and of
// the communicator internals the decoder uses (comm.cu). Not part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/b200_comm.h"
#include "q4gemv.h"

namespace b200 {

struct AttnLaunch {
    const float *q = nullptr;       // this rank's roped q rows: [heads_local][head_dim]
    const void *kcache = nullptr;   // this layer's caches: [kv head][ctx_max][head_dim]
    const void *vcache = nullptr;
    float *out = nullptr;           // [heads_local][head_dim]
    const int *pos = nullptr;       // current position (device)
    int head_dim = 0;               // 64 or 128
    int group = 0;                  // query heads per KV head, 1..4
    int kvh_local = 0;              // KV heads on this rank (one CTA each)
    int ctx_max = 0;
    int kv_f16 = 1;
    float scale = 0.0f;             // 1 / sqrtf(head_dim)
    bool pdl = true;
};

int attn_smem_bytes(int head_dim, int group, int ctx_max);
int attn_launch(const AttnLaunch &L, cudaStream_t stream);

// The all-reduce word area of a communicator's windows (comm.cu): every
// rank's mapping in this process, words per (slot, source rank), and the
// status word a timed-out wait marks.
int comm_word_area(b200_comm_t *c, uint64_t *win_words[kMaxDecodeRanks], uint64_t *slot_words, unsigned **status,
                   int *rank, int *nranks);

}  // namespace b200
