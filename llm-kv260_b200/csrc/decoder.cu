// The greedy batch-1 decoder (include/b200_decoder.h): the reference
// runtime's struct runtime (board/tp/tp_llama.cpp:783-968) on one B200 per
// rank.
//
// A token is the launch sequence of enqueue_token(), captured once into a
// CUDA graph:
//   per layer l
//     q|k|v GEMV   prologue: RMSNorm(x, attn_norm) -- at l = 0 of the token's
//                  embedding, which CTA 0 writes to x; epilogue: RoPE of q and
//                  k, k and v into the KV cache at pos           (822-846)
//     attention    this rank's heads                              (847-856)
//     o GEMV       epilogue: x += the rank-ordered sum of the partials (857-862)
//     gate|up GEMV prologue: RMSNorm(x, ffn_norm); epilogue: SiLU(gate) * up
//                  (the rows are stored gate/up interleaved)      (863-868)
//     down GEMV    epilogue: x += the rank-ordered sum            (869-874)
//   lm_head GEMV   prologue: RMSNorm(x, output_norm); the greedy pick fused
//                  (876-882); one rank: then the loop's advance
//   several ranks: the pick exchange, then the advance (895-925)
// Position, step and token ids stay on the device, so every token replays
// the same graph. All ranks' graphs run the same sequence; a rank's K-split
// partials reach its peers through the communicator's windows inside the o
// and down GEMVs (q4tile.cu, kEpiResidual).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstddef>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/b200_decoder.h"
#include "../../include/b200_engine.h"
#include "common.cuh"
#include "decode.h"

using namespace b200;

namespace {

struct DecLayer {
    uint8_t *qkv = nullptr, *o = nullptr, *gateup = nullptr, *down = nullptr;  // tiles
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    uint8_t *kcache = nullptr;  // K   [kv head][kv_stride][head_dim]
    uint8_t *vcache = nullptr;  // V^T [kv head][head_dim][kv_stride] (attn_core.cuh)
    bool set = false;
};

// small device state, one allocation
struct DevState {
    int pos;
    int n_prompt;        // pos, n_prompt and in_token: set together by one copy from the host
    int in_token;        // >= 0: the token at pos (forward's input), which the embedding prologue takes
                         // instead of tokens[pos] and records there; the token's advance resets it to -1
    unsigned step;
    int pick[2];         // the token (int32) and its logit (float32 bits)
    unsigned status[2];  // next to pick: the device and peer status words as the token's advance saw them
    int pick_local[2];   // several ranks: this rank's pick over its vocab shard
};

__global__ void advance_kernel(DevState *st, int *tokens, int ctx_max, const unsigned *status,
                               const unsigned *peer_status) {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    // runtime::generate's step (tp_llama.cpp:951-959) on the device
    const int nx = st->pos + 1;
    if (nx >= st->n_prompt && nx <= ctx_max) tokens[nx] = st->pick[0];
    st->pos = nx;
    st->step += 1u;
    st->in_token = -1;
    st->status[0] = *reinterpret_cast<const volatile unsigned *>(status);
    st->status[1] = peer_status ? *reinterpret_cast<const volatile unsigned *>(peer_status) : 0u;
}

int dfail(int code, const char *fmt, ...) {
    char msg[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    return report_error(code, msg);
}

}  // namespace

namespace {
constexpr int kIoSlots = 8;  // forward(): position, n_prompt, token; then pick, value, status, peer status
}  // namespace

struct b200_decoder {
    b200_decoder_config_t c;
    int device, rank, nranks;
    b200_comm_t *comm;
    int q_rows, kv_rows, ff_rows, vocab_rows, o_k, down_k, heads_local, kvh_local, group;
    int o_kp;  // o_k rounded up to whole 256-column chunks: the o tiles' K, zero blocks past o_k
    cudaStream_t stream;
    std::vector<DecLayer> layers;
    std::vector<void *> allocs;
    uint8_t *token_embd, *lm_head;
    float *output_norm;
    float *res, *qkv_y, *attn, *act, *logits, *rope_cs;
    uint8_t *act_q8;    // act as the down GEMV's packed x: int8[down_k] then float32 scale per 32
    int *tokens;
    DevState *st;
    void *sel_scratch;
    uint8_t *kv;
    bool output_set;
    cudaGraphExec_t graph;   // one token
    cudaGraphExec_t graphk;  // kGraphTokens tokens in a row: dependent launches overlap across token boundaries too
    cudaGraphExec_t fwd;     // forward(): the input copy, one token, the output copy
    int host_pos;       // where the device loop stands after the work queued so far
    int32_t *host_io;   // pinned, mapped: [0, 2) the pick, [2, 2 + ctx_max + 1) token ids by position, then
                        // kIoSlots words for forward(): position, n_prompt, token in; pick, value, status
                        // words out
    Tuning tu;
    // persistent mode
    bool persistent;
    TokenPhase *phases;           // device copy of the token's phase list
    int nphases;
    unsigned long long *bar_count;
    int *abort_flag;
    float2 *cand;
    int *host_tokens_dev;         // host_io + 2 as a device address
    uint64_t *trace;              // optional trace (b200_decoder_trace): persistent phases, or graph launches
    int trace_tokens;
    int trace_launches;           // graph mode: launches with a trace record (5 per layer + lm_head)
    // exchange
    uint64_t *win_words[kMaxDecodeRanks];
    uint64_t slot_words;
    unsigned *peer_status;
};

namespace {

int use_dev(b200_decoder_t *d) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return dfail(kErrNoDev, "decoder: no CUDA device");
    if (cur != d->device && cudaSetDevice(d->device) != cudaSuccess) return dfail(kErrCuda, "decoder: cudaSetDevice failed");
    return 0;
}

template <typename T>
int dalloc(b200_decoder_t *d, T **p, size_t bytes) {
    void *v = nullptr;
    const cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
    if (e != cudaSuccess) return dfail(kErrNoMem, "decoder: cudaMalloc of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    d->allocs.push_back(v);
    *p = static_cast<T *>(v);
    return 0;
}

int h2d(void *dst, const void *src, size_t bytes, cudaStream_t s) {
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
    return e == cudaSuccess ? 0 : dfail(kErrCuda, "decoder: copy to the device failed: %s", cudaGetErrorString(e));
}

// GGUF Q4_0 rows (host) -> a new tiled matrix on the device.
int upload_tiles(b200_decoder_t *d, const std::vector<uint8_t> &rows_host, int rows, int k, uint8_t **out) {
    const size_t tb = tiled_bytes(rows, k);
    if (!tb) return dfail(kErrInval, "decoder: cannot tile a %dx%d matrix", rows, k);
    uint8_t *tiles = nullptr;
    if (int rc = dalloc(d, &tiles, tb)) return rc;
    void *tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, rows_host.size());
    if (e != cudaSuccess) return dfail(kErrNoMem, "decoder: staging allocation failed");
    e = cudaMemcpyAsync(tmp, rows_host.data(), rows_host.size(), cudaMemcpyHostToDevice, d->stream);
    int rc = e == cudaSuccess ? repack_launch(static_cast<const uint8_t *>(tmp), rows, k, tiles, d->stream) : kErrCuda;
    if (rc == 0 && cudaStreamSynchronize(d->stream) != cudaSuccess) rc = kErrCuda;
    cudaFree(tmp);
    if (rc) return dfail(kErrCuda, "decoder: weight upload failed");
    *out = tiles;
    return 0;
}

size_t row_bytes(int k) { return static_cast<size_t>(k) / kQK * kBlockBytes; }

// copy_rows (tp_llama.cpp:191-197): rows [r0, r0+rows) of a [N, k] matrix
void append_rows(std::vector<uint8_t> &dst, const uint8_t *src, int k, int r0, int rows) {
    const size_t rb = row_bytes(k);
    dst.insert(dst.end(), src + r0 * rb, src + (static_cast<size_t>(r0) + rows) * rb);
}

// copy_cols (tp_llama.cpp:201-207): columns [c0, c0+kk) of every row of an [n, k] matrix
std::vector<uint8_t> cut_cols(const uint8_t *src, int k, int n, int c0, int kk) {
    const size_t rb = row_bytes(k), ob = row_bytes(kk), off = row_bytes(c0);
    std::vector<uint8_t> m(ob * n);
    for (int r = 0; r < n; ++r) memcpy(m.data() + r * ob, src + r * rb + off, ob);
    return m;
}

TileLaunch gemv_base(const b200_decoder_t *d, const uint8_t *w, int rows, int k, const void *x, float *y) {
    TileLaunch L;
    L.w = w;
    L.rows = rows;
    L.k = k;
    L.xmode = kXF32;
    L.x = x;
    L.y = y;
    L.round_mode = d->c.round_mode;
    L.l2_policy = kL2EvictFirst;
    L.pdl = true;
    L.ring_to_groups = true;  // the next launch's CTAs start beside this one's
    return L;
}

void norm_prologue(const b200_decoder_t *d, TileLaunch &L, int pro, const float *w) {
    L.dec.pro = pro;
    L.dec.res = d->res;
    L.dec.norm_w = w;
    L.dec.eps = d->c.rms_eps;
    L.dec.exact_norm = d->c.exact_norm;
    L.dec.embd = d->token_embd;
    L.dec.tokens = d->tokens;
    L.dec.in_token = pro == kProEmbedNorm ? &d->st->in_token : nullptr;
    L.dec.pos = &d->st->pos;
}

void residual_epilogue(const b200_decoder_t *d, TileLaunch &L, int ar_index) {
    L.dec.epi = kEpiResidual;
    L.dec.res = d->res;
    L.dec.nranks = d->nranks;
    L.dec.rank = d->rank;
    for (int r = 0; r < kMaxDecodeRanks; ++r) L.dec.win_words[r] = d->win_words[r];
    L.dec.slot_words = d->slot_words;
    L.dec.step = &d->st->step;
    L.dec.ar_per_token = 2 * d->c.n_layer;
    L.dec.ar_index = ar_index;
    L.dec.peer_status = d->peer_status;
}

// Graph mode's launch trace: record `i` of the token's launches, or none.
uint64_t *launch_trace(const b200_decoder_t *d, int i) {
    return (d->trace && !d->persistent) ? d->trace + static_cast<size_t>(i) * kTraceCtas * kTraceStamps : nullptr;
}

int launch(const b200_decoder_t *d, const TileLaunch &L, const char *what) {
    const char *why = nullptr;
    if (tile_validate(L, &why)) return dfail(kErrInval, "decoder: %s GEMV: %s", what, why);
    if (int rc = tile_launch(L, d->tu, d->stream))
        return dfail(rc, "decoder: %s GEMV launch failed: %s", what, cudaGetErrorString(cudaGetLastError()));
    return 0;
}

// One token's launches (see the top of this file).
int enqueue_token(b200_decoder_t *d) {
    const b200_decoder_config_t &c = d->c;
    const int e = c.n_embd;
    for (int l = 0; l < c.n_layer; ++l) {
        const DecLayer &W = d->layers[l];
        TileLaunch A = gemv_base(d, W.qkv, d->q_rows + 2 * d->kv_rows, e, d->res, d->qkv_y);
        norm_prologue(d, A, l == 0 ? kProEmbedNorm : kProRmsnorm, W.attn_norm);
        A.dec.epi = kEpiRopeKv;
        A.dec.rope_cs = d->rope_cs;
        A.dec.head_dim = c.head_dim;
        A.dec.q_rows = d->q_rows;
        A.dec.kv_rows = d->kv_rows;
        A.dec.ctx_max = c.ctx_max;
        A.dec.kv_stride = attn_kv_stride(c.ctx_max);
        A.dec.kv_f16 = c.kv_f16;
        A.dec.kcache = W.kcache;
        A.dec.vcache = W.vcache;
        A.trace = launch_trace(d, 5 * l);
        if (int rc = launch(d, A, "q|k|v")) return rc;

        AttnLaunch T;
        T.q = d->qkv_y;
        T.kcache = W.kcache;
        T.vcache = W.vcache;
        T.out = d->attn;
        T.pos = &d->st->pos;
        T.head_dim = c.head_dim;
        T.group = d->group;
        T.kvh_local = d->kvh_local;
        T.ctx_max = c.ctx_max;
        T.kv_stride = attn_kv_stride(c.ctx_max);
        T.kv_f16 = c.kv_f16;
        T.scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
        T.trace = launch_trace(d, 5 * l + 1);
        if (int rc = attn_launch(T, d->stream))
            return dfail(rc, "decoder: attention launch failed: %s", cudaGetErrorString(cudaGetLastError()));

        TileLaunch O = gemv_base(d, W.o, e, d->o_kp, d->attn, nullptr);
        residual_epilogue(d, O, 2 * l);
        O.trace = launch_trace(d, 5 * l + 2);
        if (int rc = launch(d, O, "o")) return rc;

        TileLaunch G = gemv_base(d, W.gateup, 2 * d->ff_rows, e, d->res, nullptr);
        norm_prologue(d, G, kProRmsnorm, W.ffn_norm);
        G.dec.epi = kEpiSiluPairs;
        G.dec.act = d->act;
        // gate|up also writes act as the down GEMV's packed x, when its row
        // groups still fill the GPU in the whole 4-group units that needs
        const bool act_q8 = 2 * d->ff_rows / kTileRows / 4 >= sm_count() / 2;
        if (act_q8) G.dec.act_q8 = d->act_q8;
        G.trace = launch_trace(d, 5 * l + 3);
        G.max_stages = 4;  // a ring small enough for a down GEMV CTA to start beside it
        if (int rc = launch(d, G, "gate|up")) return rc;

        TileLaunch D = gemv_base(d, W.down, e, d->down_k, act_q8 ? static_cast<const void *>(d->act_q8) : d->act, nullptr);
        if (act_q8) D.xmode = kXPacked;  // quantised by the gate|up CTAs (the same Q8_0 arithmetic)
        residual_epilogue(d, D, 2 * l + 1);
        D.trace = launch_trace(d, 5 * l + 4);
        if (int rc = launch(d, D, "down")) return rc;
    }
    TileLaunch H = gemv_base(d, d->lm_head, d->vocab_rows, e, d->res, d->logits);
    norm_prologue(d, H, kProRmsnorm, d->output_norm);
    H.sel_out = d->nranks == 1 ? d->st->pick : d->st->pick_local;
    H.sel_base = d->rank * d->vocab_rows;
    H.sel_scratch = d->sel_scratch;
    if (d->nranks == 1) {
        H.dec.adv_pos = &d->st->pos;
        H.dec.adv_step = &d->st->step;
        H.dec.adv_tokens = d->tokens;
        H.dec.n_prompt = &d->st->n_prompt;
        H.dec.ctx_max = c.ctx_max;
        H.dec.adv_in_token = &d->st->in_token;
        H.dec.adv_status = d->st->status;
    }
    H.trace = launch_trace(d, 5 * c.n_layer);
    if (int rc = launch(d, H, "lm_head")) return rc;
    if (d->nranks > 1) {
        if (int rc = b200_allgather_pick(d->comm, reinterpret_cast<uint64_t>(d->st->pick_local),
                                         reinterpret_cast<uint64_t>(d->st->pick), d->stream))
            return rc;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(32);
        cfg.stream = d->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, advance_kernel, d->st, d->tokens, c.ctx_max, static_cast<const unsigned *>(status_word()),
                               static_cast<const unsigned *>(d->peer_status)) != cudaSuccess)
            return dfail(kErrCuda, "decoder: advance launch failed");
    }
    return 0;
}

TokenArgs token_args(const b200_decoder_t *d, int ntokens) {
    const b200_decoder_config_t &c = d->c;
    TokenArgs a;
    a.phases = d->phases;
    a.nphases = d->nphases;
    a.ntokens = ntokens;
    a.res = d->res;
    a.embd = d->token_embd;
    a.tokens = d->tokens;
    a.pos = &d->st->pos;
    a.step = &d->st->step;
    a.n_prompt = &d->st->n_prompt;
    a.pick_out = d->st->pick;
    a.cand = d->cand;
    a.logits = d->logits;
    a.rope_cs = d->rope_cs;
    a.n_embd = c.n_embd;
    a.head_dim = c.head_dim;
    a.q_rows = d->q_rows;
    a.kv_rows = d->kv_rows;
    a.ctx_max = c.ctx_max;
    a.kv_stride = attn_kv_stride(c.ctx_max);
    a.kv_f16 = c.kv_f16;
    a.group = d->group;
    a.kvh_local = d->kvh_local;
    a.vocab_base = d->rank * d->vocab_rows;
    a.scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
    a.eps = c.rms_eps;
    a.exact_norm = c.exact_norm;
    a.round_mode = c.round_mode;
    a.nranks = d->nranks;
    a.rank = d->rank;
    for (int r = 0; r < kMaxDecodeRanks; ++r) a.win_words[r] = d->win_words[r];
    a.slot_words = d->slot_words;
    a.ar_per_token = 2 * c.n_layer;
    a.peer_status = d->peer_status;
    a.bar_count = d->bar_count;
    a.abort_flag = d->abort_flag;
    a.status = status_word();
    a.host_tokens = d->host_tokens_dev;
    a.trace = d->trace;
    a.trace_tokens = d->trace_tokens;
    return a;
}

// The persistent kernel's phase list for one token (the same ops, in the
// same order, as enqueue_token).
int build_phases(b200_decoder_t *d) {
    const b200_decoder_config_t &c = d->c;
    const int e = c.n_embd;
    std::vector<TokenPhase> ph;
    for (int l = 0; l < c.n_layer; ++l) {
        const DecLayer &W = d->layers[l];
        TokenPhase A;
        A.w = W.qkv;
        A.rows = d->q_rows + 2 * d->kv_rows;
        A.k = e;
        A.pro = l == 0 ? kProEmbedNorm : kProRmsnorm;
        A.norm_w = W.attn_norm;
        A.epi = kEpiRopeKv;
        A.y = d->qkv_y;
        A.kcache = W.kcache;
        A.vcache = W.vcache;
        ph.push_back(A);
        TokenPhase T;
        T.kind = kPhAttn;
        T.kcache = W.kcache;
        T.vcache = W.vcache;
        T.q = d->qkv_y;
        T.out = d->attn;
        ph.push_back(T);
        TokenPhase O;
        O.w = W.o;
        O.rows = e;
        O.k = d->o_kp;
        O.x = d->attn;
        O.epi = kEpiResidual;
        O.ar_index = 2 * l;
        ph.push_back(O);
        TokenPhase U;
        U.w = W.gateup;
        U.rows = 2 * d->ff_rows;
        U.k = e;
        U.pro = kProRmsnorm;
        U.norm_w = W.ffn_norm;
        U.epi = kEpiSiluPairs;
        U.act = d->act;
        ph.push_back(U);
        TokenPhase D;
        D.w = W.down;
        D.rows = e;
        D.k = d->down_k;
        D.x = d->act;
        D.epi = kEpiResidual;
        D.ar_index = 2 * l + 1;
        ph.push_back(D);
    }
    TokenPhase H;
    H.w = d->lm_head;
    H.rows = d->vocab_rows;
    H.k = e;
    H.pro = kProRmsnorm;
    H.norm_w = d->output_norm;
    H.epi = kEpiStore;
    H.y = d->logits;
    H.pick = 1;
    ph.push_back(H);
    if (static_cast<int>(ph.size()) > kMaxTokenPhases) return dfail(kErrInval, "decoder: too many layers for one token program");
    if (int rc = dalloc(d, &d->phases, sizeof(TokenPhase) * ph.size())) return rc;
    if (int rc = h2d(d->phases, ph.data(), sizeof(TokenPhase) * ph.size(), d->stream)) return rc;
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return dfail(kErrCuda, "decoder: phase upload failed");
    d->nphases = static_cast<int>(ph.size());
    TokenArgs a = token_args(d, 1);
    int smem = 0, ring = 0, wgs = 0, grid = 0;
    if (int rc = token_kernel_plan(a, &smem, &ring, &wgs, &grid))
        return dfail(rc, "decoder: the persistent kernel does not fit this model (context %d too long?)", c.ctx_max);
    return 0;
}

constexpr int kGraphTokens = 8;

// Capture `tokens` tokens' launches into an executable graph.
int capture_tokens(b200_decoder_t *d, int tokens, cudaGraphExec_t *out) {
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) return dfail(kErrCuda, "decoder: capture begin failed: %s", cudaGetErrorString(e));
    int rc = 0;
    for (int t = 0; t < tokens && !rc; ++t) rc = enqueue_token(d);
    e = cudaStreamEndCapture(d->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return dfail(kErrCuda, "decoder: capture failed: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        *out = nullptr;
        return dfail(kErrCuda, "decoder: graph instantiation failed: %s", cudaGetErrorString(e));
    }
    return 0;
}

void drop_graphs(b200_decoder_t *d) {
    if (d->graph) cudaGraphExecDestroy(d->graph);
    if (d->graphk) cudaGraphExecDestroy(d->graphk);
    if (d->fwd) cudaGraphExecDestroy(d->fwd);
    d->graph = d->graphk = d->fwd = nullptr;
}

int ready(b200_decoder_t *d) {
    if (!d) return dfail(kErrInval, "decoder: null handle");
    for (const DecLayer &L : d->layers)
        if (!L.set) return dfail(kErrInval, "decoder: a layer's weights are not set");
    if (!d->output_set) return dfail(kErrInval, "decoder: token_embd / output_norm not set");
    if (int rc = use_dev(d)) return rc;
    if (d->persistent) return d->nphases ? 0 : build_phases(d);
    if (d->graph && d->graphk) return 0;
    drop_graphs(d);
    if (int rc = capture_tokens(d, 1, &d->graph)) return rc;
    if (int rc = capture_tokens(d, kGraphTokens, &d->graphk)) {
        drop_graphs(d);
        return rc;
    }
    return 0;
}

// The loop's position and prompt length, written on the decoder's stream
// (the step counter stays as the device left it: the ranks' epochs follow it).
int set_state(b200_decoder_t *d, int pos, int n_prompt) {
    const int v[3] = {pos, n_prompt, -1};  // pos, n_prompt, in_token
    if (int rc = h2d(&d->st->pos, v, sizeof v, d->stream)) return rc;
    d->host_pos = pos;
    return 0;
}

int launch_steps(b200_decoder_t *d, int n) {
    if (n < 0 || d->host_pos + n > d->c.ctx_max)
        return dfail(kErrInval, "decoder: %d more positions from %d pass ctx_max %d", n, d->host_pos, d->c.ctx_max);
    if (d->persistent) {
        if (n == 0) return 0;
        if (int rc = token_kernel_launch(token_args(d, n), d->stream))
            return dfail(rc, "decoder: persistent kernel launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        d->host_pos += n;
        return 0;
    }
    for (int i = 0; i < n;) {
        const bool k = n - i >= kGraphTokens;
        if (cudaGraphLaunch(k ? d->graphk : d->graph, d->stream) != cudaSuccess)
            return dfail(kErrCuda, "decoder: graph launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        i += k ? kGraphTokens : 1;
    }
    d->host_pos += n;
    return 0;
}

int queue_prefill(b200_decoder_t *d, const int32_t *prompt, int n_prompt) {
    if (!prompt || n_prompt < 1 || n_prompt > d->c.ctx_max) return dfail(kErrInval, "decoder: need 1 <= n_prompt <= ctx_max");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= d->c.n_vocab) return dfail(kErrInval, "decoder: prompt token out of range");
    if (int rc = h2d(d->tokens, prompt, 4 * static_cast<size_t>(n_prompt), d->stream)) return rc;
    if (int rc = set_state(d, 0, n_prompt)) return rc;
    return launch_steps(d, n_prompt);
}

int check_status(b200_decoder_t *d) {
    unsigned s = 0;
    read_status(&s);
    if (d->abort_flag) {
        int ab = 0;
        cudaMemcpy(&ab, d->abort_flag, 4, cudaMemcpyDeviceToHost);
        if (ab) s |= kStatusStageTimeout;
    }
    unsigned ps = 0;
    if (d->peer_status) cudaMemcpy(&ps, d->peer_status, 4, cudaMemcpyDeviceToHost);
    if (s || ps) return dfail(kErrTimeout, "decoder: a bounded wait ran out (status %u, peer status %u)", s, ps);
    return 0;
}

}  // namespace

extern "C" int b200_decoder_create(b200_decoder_t **out, const b200_decoder_config_t *cfg, int device, int rank,
                                   int nranks, b200_comm_t *comm) {
    if (!out || !cfg) return dfail(kErrInval, "decoder: null argument");
    *out = nullptr;
    const b200_decoder_config_t c = *cfg;
    if (nranks < 1 || nranks > kMaxDecodeRanks || rank < 0 || rank >= nranks)
        return dfail(kErrInval, "decoder: need 0 <= rank < nranks <= 8");
    if (nranks > 1 && !comm) return dfail(kErrInval, "decoder: several ranks need a communicator");
    if (c.n_layer < 1 || c.n_embd <= 0 || c.n_ff <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.n_vocab <= 0 ||
        c.ctx_max < 1 || (c.head_dim != 64 && c.head_dim != 128) || c.n_embd != c.n_head * c.head_dim ||
        c.n_head % c.n_head_kv || c.n_head / c.n_head_kv > 4 || c.n_head_kv % nranks || c.n_vocab % nranks ||
        c.n_ff % nranks || (c.round_mode != kRoundContract && c.round_mode != kRoundRoundf) || !(c.rms_eps >= 0.0f))
        return dfail(kErrInval, "decoder: unusable hyperparameters");
    const int o_k = c.n_embd / nranks, down_k = c.n_ff / nranks;
    for (int v : {c.n_embd, down_k})
        if (v % 256 || v > kMaxK) return dfail(kErrInval, "decoder: shard width %d not a multiple of 256 up to 8192", v);
    // attn_output's K shard may end inside a 256-column chunk (the 3B model
    // at 8 ranks: 384 columns, 12 blocks); see set_layer
    if (o_k % kQK || o_k > kMaxK) return dfail(kErrInval, "decoder: attn_output shard width %d unusable", o_k);
    if ((c.n_embd / nranks) % c.head_dim || (c.n_head_kv * c.head_dim / nranks) % kTileRows)
        return dfail(kErrInval, "decoder: heads do not split evenly over the ranks");
    b200_decoder_t *d = new (std::nothrow) b200_decoder_t();
    if (!d) return dfail(kErrNoMem, "decoder: out of host memory");
    d->c = c;
    d->device = device;
    d->rank = rank;
    d->nranks = nranks;
    d->comm = comm;
    d->q_rows = c.n_embd / nranks;
    d->kv_rows = c.n_head_kv * c.head_dim / nranks;
    d->ff_rows = c.n_ff / nranks;
    d->vocab_rows = c.n_vocab / nranks;
    d->o_k = o_k;
    d->o_kp = (o_k + 255) / 256 * 256;
    d->down_k = down_k;
    d->heads_local = c.n_head / nranks;
    d->kvh_local = c.n_head_kv / nranks;
    d->group = c.n_head / c.n_head_kv;
    d->tu.stages = 8;
    d->tu.ctas_per_sm = 4;
    d->tu.kslices = 1;
    d->layers.resize(c.n_layer);
    auto bail = [&](int rc) {
        b200_decoder_destroy(d);
        return rc;
    };
    if (int rc = use_dev(d)) return bail(rc);
    if (!c.persistent && attn_smem_bytes(c.head_dim, c.kv_f16, c.ctx_max) > max_smem_optin() &&
        attn_smem_bytes_long(c.head_dim, c.kv_f16, c.ctx_max) > max_smem_optin())
        return bail(dfail(kErrInval, "decoder: attention over ctx_max %d positions does not fit shared memory", c.ctx_max));
    if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(dfail(kErrCuda, "decoder: stream creation failed"));
    if (nranks > 1) {
        int cr = -1, cn = -1;
        if (comm_word_area(comm, d->win_words, &d->slot_words, &d->peer_status, &cr, &cn) || cr != rank || cn != nranks)
            return bail(dfail(kErrInval, "decoder: the communicator is not this rank's, or its peers are not imported"));
        if (d->slot_words < static_cast<uint64_t>(c.n_embd))
            return bail(dfail(kErrInval, "decoder: the communicator was created for fewer than n_embd floats"));
    }
    const int e = c.n_embd;
    const size_t kv_elems = static_cast<size_t>(c.n_layer) * d->kvh_local * attn_kv_stride(c.ctx_max) * c.head_dim;
    const size_t kv_bytes = kv_elems * (c.kv_f16 ? 2 : 4);
    int rc = 0;
    if (!rc) rc = dalloc(d, &d->res, 4 * static_cast<size_t>(e));
    if (!rc) rc = dalloc(d, &d->qkv_y, 4 * static_cast<size_t>(d->q_rows + 2 * d->kv_rows));
    if (!rc) rc = dalloc(d, &d->attn, 4 * static_cast<size_t>(d->o_kp));
    if (!rc) rc = dalloc(d, &d->act, 4 * static_cast<size_t>(down_k));
    if (!rc) rc = dalloc(d, &d->act_q8, static_cast<size_t>(down_k) + 4 * static_cast<size_t>(down_k / kQK));
    if (!rc) rc = dalloc(d, &d->logits, 4 * static_cast<size_t>(d->vocab_rows));
    if (!rc) rc = dalloc(d, &d->rope_cs, 4 * static_cast<size_t>(c.ctx_max) * c.head_dim);
    if (!rc) rc = dalloc(d, &d->tokens, 4 * (static_cast<size_t>(c.ctx_max) + 1));
    if (!rc) rc = dalloc(d, &d->st, sizeof(DevState));
    if (!rc) rc = dalloc(d, &d->sel_scratch, static_cast<size_t>(tile_select_scratch_bytes()));
    if (!rc) rc = dalloc(d, &d->kv, 2 * kv_bytes);
    if (!rc) rc = dalloc(d, &d->output_norm, 4 * static_cast<size_t>(e));
    if (rc) return bail(rc);
    if (cudaHostAlloc(reinterpret_cast<void **>(&d->host_io), 4 * (static_cast<size_t>(c.ctx_max) + 3 + kIoSlots),
                      cudaHostAllocMapped) != cudaSuccess)
        return bail(dfail(kErrNoMem, "decoder: pinned host buffer allocation failed"));
    d->persistent = c.persistent != 0;
    if (d->persistent) {
        void *hd = nullptr;
        if (cudaHostGetDevicePointer(&hd, d->host_io, 0) != cudaSuccess)
            return bail(dfail(kErrCuda, "decoder: mapped host buffer has no device address"));
        d->host_tokens_dev = static_cast<int *>(hd) + 2;
        const int sms = sm_count();
        if (sms <= 0) return bail(dfail(kErrNoDev, "decoder: no SM count"));
        rc = dalloc(d, &d->bar_count, 8);
        if (!rc) rc = dalloc(d, &d->abort_flag, 4);
        if (!rc) rc = dalloc(d, &d->cand, sizeof(float2) * static_cast<size_t>(sms));
        if (rc) return bail(rc);
        cudaMemsetAsync(d->bar_count, 0, 8, d->stream);
        cudaMemsetAsync(d->abort_flag, 0, 4, d->stream);
        if (nranks > 1 && d->slot_words < static_cast<uint64_t>(c.n_embd) + 2)
            return bail(dfail(kErrInval, "decoder: the communicator needs room for n_embd + 2 floats"));
    }
    cudaMemsetAsync(d->sel_scratch, 0, static_cast<size_t>(tile_select_scratch_bytes()), d->stream);
    cudaMemsetAsync(d->st, 0, sizeof(DevState), d->stream);
    cudaMemsetAsync(d->tokens, 0, 4 * (static_cast<size_t>(c.ctx_max) + 1), d->stream);
    cudaMemsetAsync(d->kv, 0, 2 * kv_bytes, d->stream);
    cudaMemsetAsync(d->res, 0, 4 * static_cast<size_t>(e), d->stream);
    cudaMemsetAsync(d->attn, 0, 4 * static_cast<size_t>(d->o_kp), d->stream);  // the o GEMV's zero x past o_k
    // rope_table (tp_llama.cpp:574-580) for every position, on the host as the
    // reference computes it, shared with the device
    std::vector<float> cs(static_cast<size_t>(c.ctx_max) * c.head_dim);
    for (int p = 0; p < c.ctx_max; ++p) b200_rope_table(cs.data() + static_cast<size_t>(p) * c.head_dim, c.head_dim, p, c.rope_base);
    if (int r2 = h2d(d->rope_cs, cs.data(), cs.size() * 4, d->stream)) return bail(r2);
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return bail(dfail(kErrCuda, "decoder: initialisation failed"));
    const size_t per_layer = static_cast<size_t>(d->kvh_local) * attn_kv_stride(c.ctx_max) * c.head_dim * (c.kv_f16 ? 2 : 4);
    for (int l = 0; l < c.n_layer; ++l) {
        d->layers[l].kcache = d->kv + l * per_layer;
        d->layers[l].vcache = d->kv + kv_bytes + l * per_layer;
    }
    *out = d;
    return 0;
}

extern "C" int b200_decoder_set_layer(b200_decoder_t *d, int layer, const void *attn_q, const void *attn_k,
                                      const void *attn_v, const void *attn_output, const void *ffn_gate,
                                      const void *ffn_up, const void *ffn_down, const float *attn_norm,
                                      const float *ffn_norm) {
    if (!d || layer < 0 || layer >= d->c.n_layer) return dfail(kErrInval, "decoder: bad layer");
    if (!attn_q || !attn_k || !attn_v || !attn_output || !ffn_gate || !ffn_up || !ffn_down || !attn_norm || !ffn_norm)
        return dfail(kErrInval, "decoder: null tensor");
    if (d->layers[layer].set) return dfail(kErrInval, "decoder: layer %d already set", layer);
    if (int rc = use_dev(d)) return rc;
    const int e = d->c.n_embd, r = d->rank;
    const auto *q = static_cast<const uint8_t *>(attn_q);
    const auto *k = static_cast<const uint8_t *>(attn_k);
    const auto *v = static_cast<const uint8_t *>(attn_v);
    DecLayer &L = d->layers[layer];
    // q | k | v shard rows (tp_llama.cpp:258-261)
    std::vector<uint8_t> qkv;
    qkv.reserve(row_bytes(e) * (d->q_rows + 2 * d->kv_rows));
    append_rows(qkv, q, e, r * d->q_rows, d->q_rows);
    append_rows(qkv, k, e, r * d->kv_rows, d->kv_rows);
    append_rows(qkv, v, e, r * d->kv_rows, d->kv_rows);
    if (int rc = upload_tiles(d, qkv, d->q_rows + 2 * d->kv_rows, e, &L.qkv)) return rc;
    // attn_output columns (tp_llama.cpp:263-264). When the shard's width is
    // not whole 256-column chunks, each row is padded with zero blocks (float16
    // scale +0, nibbles 0) to o_kp, and the GEMV's x past o_k is zero: every
    // padded block term is +-0, which leaves every lane sum's bits as they are
    // (a lane starts at +0 and never holds -0), so the result is the lane rule
    // b mod 8 applied to the shard's own blocks -- the contract extension
    // q4_0.py:166-167 and load_model (tp_llama.cpp:247) do not allow.
    {
        std::vector<uint8_t> oc = cut_cols(static_cast<const uint8_t *>(attn_output), e, e, r * d->o_k, d->o_k);
        if (d->o_kp != d->o_k) {
            const size_t rb = row_bytes(d->o_k), pb = row_bytes(d->o_kp);
            std::vector<uint8_t> padded(pb * e, 0);
            for (int i = 0; i < e; ++i) memcpy(padded.data() + i * pb, oc.data() + i * rb, rb);
            oc.swap(padded);
        }
        if (int rc = upload_tiles(d, oc, e, d->o_kp, &L.o)) return rc;
    }
    // gate | up shard rows (tp_llama.cpp:266-268), stored interleaved: row 2i
    // is gate row i, row 2i+1 up row i, so each SiLU pair is a thread pair
    std::vector<uint8_t> gu;
    const size_t rb = row_bytes(e);
    gu.resize(rb * 2 * d->ff_rows);
    const auto *g = static_cast<const uint8_t *>(ffn_gate);
    const auto *u = static_cast<const uint8_t *>(ffn_up);
    for (int i = 0; i < d->ff_rows; ++i) {
        memcpy(gu.data() + (2 * static_cast<size_t>(i)) * rb, g + (static_cast<size_t>(r) * d->ff_rows + i) * rb, rb);
        memcpy(gu.data() + (2 * static_cast<size_t>(i) + 1) * rb, u + (static_cast<size_t>(r) * d->ff_rows + i) * rb, rb);
    }
    if (int rc = upload_tiles(d, gu, 2 * d->ff_rows, e, &L.gateup)) return rc;
    // ffn_down columns (tp_llama.cpp:270-271)
    if (int rc = upload_tiles(d, cut_cols(static_cast<const uint8_t *>(ffn_down), d->c.n_ff, e, r * d->down_k, d->down_k),
                              e, d->down_k, &L.down))
        return rc;
    if (int rc = dalloc(d, &L.attn_norm, 4 * static_cast<size_t>(e))) return rc;
    if (int rc = dalloc(d, &L.ffn_norm, 4 * static_cast<size_t>(e))) return rc;
    if (int rc = h2d(L.attn_norm, attn_norm, 4 * static_cast<size_t>(e), d->stream)) return rc;
    if (int rc = h2d(L.ffn_norm, ffn_norm, 4 * static_cast<size_t>(e), d->stream)) return rc;
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return dfail(kErrCuda, "decoder: norm upload failed");
    L.set = true;
    return 0;
}

extern "C" int b200_decoder_set_output(b200_decoder_t *d, const void *token_embd, const float *output_norm) {
    if (!d || !token_embd || !output_norm) return dfail(kErrInval, "decoder: null argument");
    if (d->output_set) return dfail(kErrInval, "decoder: output already set");
    if (int rc = use_dev(d)) return rc;
    const int e = d->c.n_embd;
    const size_t rb = row_bytes(e), all = rb * d->c.n_vocab;
    if (int rc = dalloc(d, &d->token_embd, all)) return rc;
    if (int rc = h2d(d->token_embd, token_embd, all, d->stream)) return rc;
    // lm_head: this rank's vocabulary rows of the tied table (tp_llama.cpp:279)
    std::vector<uint8_t> lm;
    lm.reserve(rb * d->vocab_rows);
    append_rows(lm, static_cast<const uint8_t *>(token_embd), e, d->rank * d->vocab_rows, d->vocab_rows);
    if (int rc = upload_tiles(d, lm, d->vocab_rows, e, &d->lm_head)) return rc;
    if (int rc = h2d(d->output_norm, output_norm, 4 * static_cast<size_t>(e), d->stream)) return rc;
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return dfail(kErrCuda, "decoder: output upload failed");
    d->output_set = true;
    return 0;
}

namespace {
// forward()'s graph (graph mode): the inputs {pos, n_prompt, in_token} from
// pinned host memory into the device state in one copy, the token's kernels
// (the embedding prologue takes in_token), and {pick, value, status, peer
// status} back in one copy -- one launch and one wait per call.
int forward_graph(b200_decoder_t *d) {
    if (d->fwd) return 0;
    static_assert(offsetof(DevState, n_prompt) == offsetof(DevState, pos) + 4 &&
                      offsetof(DevState, in_token) == offsetof(DevState, pos) + 8,
                  "pos, n_prompt and in_token adjacent");
    static_assert(offsetof(DevState, status) == offsetof(DevState, pick) + 8, "pick and the status words adjacent");
    int32_t *in = d->host_io + 3 + d->c.ctx_max, *out = in + 4;
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeRelaxed) != cudaSuccess)
        return dfail(kErrCuda, "decoder: capture failed: %s", cudaGetErrorString(cudaGetLastError()));
    cudaError_t e = cudaMemcpyAsync(&d->st->pos, in, 12, cudaMemcpyHostToDevice, d->stream);
    const int rc = e == cudaSuccess ? enqueue_token(d) : kErrCuda;
    if (!rc) e = cudaMemcpyAsync(out, d->st->pick, 16, cudaMemcpyDeviceToHost, d->stream);
    const cudaError_t ee = cudaStreamEndCapture(d->stream, &g);
    if (rc || e != cudaSuccess || ee != cudaSuccess || cudaGraphInstantiate(&d->fwd, g, 0) != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        d->fwd = nullptr;
        return dfail(rc ? rc : kErrCuda, "decoder: forward graph failed: %s", cudaGetErrorString(cudaGetLastError()));
    }
    cudaGraphDestroy(g);
    return 0;
}
}  // namespace

extern "C" int b200_decoder_forward(b200_decoder_t *d, int token, int pos, int32_t *pick, float *value) {
    if (int rc = ready(d)) return rc;
    if (token < 0 || token >= d->c.n_vocab || pos < 0 || pos >= d->c.ctx_max)
        return dfail(kErrInval, "decoder: token or position out of range");
    // The step's inputs go from pinned host memory, its result and the status
    // words come back into it, and the call waits once. Earlier queued work
    // (prefill / step) finishes first, so the pinned words are free.
    if (cudaStreamSynchronize(d->stream) != cudaSuccess)
        return dfail(kErrCuda, "decoder: stream failed: %s", cudaGetErrorString(cudaGetLastError()));
    int32_t *in = d->host_io + 3 + d->c.ctx_max, *out = in + 4;  // kIoSlots words
    in[0] = pos;
    in[1] = INT_MAX;  // n_prompt: the loop's advance writes no token
    cudaError_t e = cudaSuccess;
    if (!d->persistent) {
        if (int rc = forward_graph(d)) return rc;
        in[2] = token;  // in_token: the embedding prologue takes it and records it at tokens[pos]
        out[2] = out[3] = 0;
        e = cudaGraphLaunch(d->fwd, d->stream);
        d->host_pos = pos + 1;
    } else {
        // the persistent kernel reads the token from tokens[pos]
        in[2] = -1;
        in[3] = token;
        e = cudaMemcpyAsync(d->tokens + pos, in + 3, 4, cudaMemcpyHostToDevice, d->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&d->st->pos, in, 12, cudaMemcpyHostToDevice, d->stream);
        if (e != cudaSuccess) return dfail(kErrCuda, "decoder: copy to the device failed: %s", cudaGetErrorString(e));
        d->host_pos = pos;
        if (int rc = launch_steps(d, 1)) return rc;
        e = cudaMemcpyAsync(out, d->st->pick, 8, cudaMemcpyDeviceToHost, d->stream);
        out[2] = out[3] = 1;  // the full status check below (and the persistent kernel's abort flag)
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return dfail(kErrCuda, "decoder: forward failed: %s", cudaGetErrorString(e));
    if (out[2] || out[3]) {
        if (int rc = check_status(d)) return rc;  // the full check
    }
    if (pick) *pick = out[0];
    if (value) memcpy(value, &out[1], 4);
    return 0;
}

extern "C" int b200_decoder_prefill(b200_decoder_t *d, const int32_t *prompt, int n_prompt) {
    if (int rc = ready(d)) return rc;
    return queue_prefill(d, prompt, n_prompt);
}

extern "C" int b200_decoder_step(b200_decoder_t *d, int n) {
    if (int rc = ready(d)) return rc;
    return launch_steps(d, n);
}

extern "C" int b200_decoder_generate(b200_decoder_t *d, const int32_t *prompt, int n_prompt, int n_gen, int32_t *out,
                                     double *prompt_ms, double *gen_ms) {
    if (int rc = ready(d)) return rc;
    if (!prompt || !out || n_prompt < 1 || n_gen < 1 || n_prompt + n_gen - 1 > d->c.ctx_max)
        return dfail(kErrInval, "decoder: need n_prompt >= 1, n_gen >= 1, n_prompt + n_gen - 1 <= ctx_max");
    cudaEvent_t ev[3];
    for (auto &x : ev) cudaEventCreate(&x);
    cudaEventRecord(ev[0], d->stream);
    int rc = queue_prefill(d, prompt, n_prompt);
    cudaEventRecord(ev[1], d->stream);
    // each token goes to the host as it is made (4 bytes a step), as the
    // reference streams it to its caller (tp_llama.cpp:955)
    cudaError_t err = cudaSuccess;
    if (d->persistent) {
        // the kernel writes each token to the mapped host buffer as it makes it
        if (rc == 0) rc = launch_steps(d, n_gen - 1);
    } else {
        for (int i = 0; i < n_gen && rc == 0 && err == cudaSuccess; ++i) {
            if (i > 0) rc = launch_steps(d, 1);
            if (rc == 0)
                err = cudaMemcpyAsync(d->host_io + 2 + n_prompt + i, d->tokens + n_prompt + i, 4,
                                      cudaMemcpyDeviceToHost, d->stream);
        }
    }
    cudaEventRecord(ev[2], d->stream);
    if (rc == 0 && err == cudaSuccess) err = cudaStreamSynchronize(d->stream);
    float a = 0.0f, b = 0.0f;
    if (rc == 0 && err == cudaSuccess) {
        cudaEventElapsedTime(&a, ev[0], ev[1]);
        cudaEventElapsedTime(&b, ev[1], ev[2]);
    }
    for (auto &x : ev) cudaEventDestroy(x);
    if (rc) return rc;
    if (err != cudaSuccess) return dfail(kErrCuda, "decoder: generate failed: %s", cudaGetErrorString(err));
    if (int r2 = check_status(d)) return r2;
    memcpy(out, d->host_io + 2 + n_prompt, 4 * static_cast<size_t>(n_gen));
    if (prompt_ms) *prompt_ms = a;
    if (gen_ms) *gen_ms = b;
    return 0;
}

extern "C" int b200_decoder_trace(b200_decoder_t *d, int tokens) {
    if (!d || tokens < 0 || tokens > 64) return dfail(kErrInval, "decoder: trace 0..64 tokens");
    if (!d->persistent) {
        // graph mode: the launches of the last token run, recorded by every replay
        if (tokens > 1) return dfail(kErrInval, "decoder: graph mode traces one token (the last one run)");
        if (int rc = use_dev(d)) return rc;
        if (cudaStreamSynchronize(d->stream) != cudaSuccess)
            return dfail(kErrCuda, "decoder: stream failed: %s", cudaGetErrorString(cudaGetLastError()));
        const int nl = 5 * d->c.n_layer + 1;
        if (tokens && !d->trace_launches) {
            const size_t bytes = static_cast<size_t>(nl) * kTraceCtas * kTraceStamps * 8;
            if (int rc = dalloc(d, &d->trace, bytes)) return rc;
            if (cudaMemset(d->trace, 0, bytes) != cudaSuccess) return dfail(kErrCuda, "decoder: trace reset failed");
            d->trace_launches = nl;
        }
        if (tokens != d->trace_tokens) drop_graphs(d);  // recapture with (or without) the trace pointers
        d->trace_tokens = tokens;
        if (!tokens) {
            d->trace = nullptr;
            d->trace_launches = 0;
        }
        return 0;
    }
    if (int rc = ready(d)) return rc;
    if (tokens > d->trace_tokens) {
        const int sms = sm_count();
        if (int rc = dalloc(d, &d->trace, static_cast<size_t>(tokens) * d->nphases * sms * 8 * 8)) return rc;
    }
    d->trace_tokens = tokens;
    if (!tokens) d->trace = nullptr;
    return 0;
}

extern "C" int b200_decoder_read(b200_decoder_t *d, int what, void *host, uint64_t bytes) {
    if (!d || !host) return dfail(kErrInval, "decoder: null argument");
    if (int rc = use_dev(d)) return rc;
    const void *src = nullptr;
    uint64_t n = 0;
    switch (what) {
        case 0: src = d->res; n = 4ull * d->c.n_embd; break;
        case 1: src = d->logits; n = 4ull * d->vocab_rows; break;
        case 2: src = d->tokens; n = 4ull * (d->c.ctx_max + 1); break;
        case 3: src = d->st->pick; n = 8; break;
        case 4: src = d->qkv_y; n = 4ull * (d->q_rows + 2 * d->kv_rows); break;
        case 5: src = d->attn; n = 4ull * d->o_k; break;
        case 6: src = d->act; n = 4ull * d->down_k; break;
        case 7:
            src = d->trace;
            n = d->persistent ? 8ull * d->trace_tokens * d->nphases * sm_count() * 8
                              : 8ull * d->trace_launches * kTraceCtas * kTraceStamps;
            break;
        default: return dfail(kErrInval, "decoder: unknown buffer %d", what);
    }
    if (bytes != n) return dfail(kErrInval, "decoder: buffer %d holds %llu bytes", what, static_cast<unsigned long long>(n));
    if (cudaStreamSynchronize(d->stream) != cudaSuccess || cudaMemcpy(host, src, n, cudaMemcpyDeviceToHost) != cudaSuccess)
        return dfail(kErrCuda, "decoder: read failed");
    return 0;
}

extern "C" int b200_decoder_status(b200_decoder_t *d, unsigned *status) {
    if (!d || !status) return dfail(kErrInval, "decoder: null argument");
    if (int rc = use_dev(d)) return rc;
    unsigned s = 0, ps = 0;
    if (read_status(&s) || clear_status()) return dfail(kErrCuda, "decoder: status read failed");
    if (d->peer_status) {
        if (cudaMemcpy(&ps, d->peer_status, 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemset(d->peer_status, 0, 4) != cudaSuccess)
            return dfail(kErrCuda, "decoder: peer status read failed");
    }
    *status = s | ps;
    return 0;
}

extern "C" int b200_rope_table_freqs(float *cs, int d, int pos, float base, const float *freqs) {
    if (!cs || d <= 0 || d % 2 || pos < 0) return dfail(kErrInval, "rope table: bad arguments");
    for (int i = 0; i < d / 2; ++i) {
        float theta = static_cast<float>(pos) * powf(base, -2.0f * static_cast<float>(i) / static_cast<float>(d));
        if (freqs) theta = theta / freqs[i];
        cs[2 * i] = cosf(theta);
        cs[2 * i + 1] = sinf(theta);
    }
    return 0;
}

extern "C" int b200_rope_table(float *cs, int d, int pos, float base) {
    return b200_rope_table_freqs(cs, d, pos, base, nullptr);
}

extern "C" int b200_decoder_set_rope_freqs(b200_decoder_t *d, const float *freqs) {
    if (!d) return dfail(kErrInval, "decoder: null handle");
    if (freqs)
        for (int i = 0; i < d->c.head_dim / 2; ++i)
            if (!(freqs[i] > 0.0f)) return dfail(kErrInval, "decoder: rope_freqs[%d] is not a positive factor", i);
    if (int rc = use_dev(d)) return rc;
    const b200_decoder_config_t &c = d->c;
    std::vector<float> cs(static_cast<size_t>(c.ctx_max) * c.head_dim);
    for (int p = 0; p < c.ctx_max; ++p)
        b200_rope_table_freqs(cs.data() + static_cast<size_t>(p) * c.head_dim, c.head_dim, p, c.rope_base, freqs);
    if (cudaStreamSynchronize(d->stream) != cudaSuccess) return dfail(kErrCuda, "decoder: stream failed");
    if (cudaMemcpy(d->rope_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return dfail(kErrCuda, "decoder: rope table upload failed");
    return 0;
}

namespace b200 {
int decoder_config(const b200_decoder_t *d, b200_decoder_config_t *out) {
    if (!d || !out) return dfail(kErrInval, "decoder: null argument");
    *out = d->c;
    return 0;
}
}  // namespace b200

namespace {
// An empty kernel shaped like the decoder's: it lets its dependents launch,
// then waits for its predecessor (both no-ops without the PDL attribute).
__global__ void launch_floor_kernel() {
    pdl_launch_dependents();
    pdl_wait_prior_grid();
}
}  // namespace

extern "C" int b200_launch_floor(int device, int launches, int ctas, int threads, int smem, int pdl, int reps,
                                 float *us_per_launch) {
    if (!us_per_launch || launches < 1 || launches > 4096 || ctas < 1 || ctas > 65535 || threads < 32 ||
        threads > 1024 || smem < 0 || reps < 1 || reps > 100000)
        return dfail(kErrInval, "launch floor: bad arguments");
    if (cudaSetDevice(device) != cudaSuccess) return dfail(kErrNoDev, "launch floor: no device %d", device);
    if (smem > max_smem_optin()) return dfail(kErrInval, "launch floor: %d bytes of shared memory is above the limit", smem);
    if (!ensure_smem(reinterpret_cast<const void *>(launch_floor_kernel), smem > 0 ? smem : 1))
        return dfail(kErrCuda, "launch floor: kernel attributes");
    cudaStream_t st = nullptr;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    auto fail = [&](const char *what) {
        rc = dfail(kErrCuda, "launch floor: %s: %s", what, cudaGetErrorString(cudaGetLastError()));
    };
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
        fail("stream");
    } else if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        fail("capture");
    } else {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(static_cast<unsigned>(ctas));
        cfg.blockDim = dim3(static_cast<unsigned>(threads));
        cfg.dynamicSmemBytes = static_cast<size_t>(smem);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        bool ok = true;
        for (int i = 0; i < launches && ok; ++i) ok = cudaLaunchKernelEx(&cfg, launch_floor_kernel) == cudaSuccess;
        const bool ended = cudaStreamEndCapture(st, &g) == cudaSuccess;
        if (!ok || !ended) fail("launch");
        else if (cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) fail("instantiate");
    }
    if (!rc) {
        bool ok = cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
        for (int i = 0; i < 3 && ok; ++i) ok = cudaGraphLaunch(ge, st) == cudaSuccess;
        ok = ok && cudaEventRecord(e0, st) == cudaSuccess;
        for (int i = 0; i < reps && ok; ++i) ok = cudaGraphLaunch(ge, st) == cudaSuccess;
        ok = ok && cudaEventRecord(e1, st) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess;
        float ms = 0.0f;
        ok = ok && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess;
        if (!ok) fail("replay");
        else *us_per_launch = 1e3f * ms / (static_cast<float>(reps) * static_cast<float>(launches));
    }
    if (st) cudaStreamSynchronize(st);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (st) cudaStreamDestroy(st);
    return rc;
}

extern "C" void *b200_decoder_stream(b200_decoder_t *d) { return d ? d->stream : nullptr; }

extern "C" int b200_decoder_destroy(b200_decoder_t *d) {
    if (!d) return 0;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != d->device) cudaSetDevice(d->device);
    if (d->stream) cudaStreamSynchronize(d->stream);
    drop_graphs(d);
    for (void *p : d->allocs) cudaFree(p);
    if (d->host_io) cudaFreeHost(d->host_io);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
    return 0;
}
