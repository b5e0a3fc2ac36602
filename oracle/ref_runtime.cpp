// The reference runtime's own decode code, compiled on this host: TEST
// INFRASTRUCTURE ONLY (the checker of oracle/decode_oracle.c; nothing in the
// product links it, and it is built only where the reference checkout is
// present).
//
// oracle/Makefile cuts these sections out of board/tp/tp_llama.cpp with sed,
// as the reference's own board/tp/bench/Makefile cuts its ops section, and
// this file #includes them unchanged:
//   memory.inc    pools_t, qmat                           (tp_llama.cpp:76-120)
//   model.inc     hparams, model_t, gguf_file, copy_rows, copy_cols,
//                 new_mat, load_model                     (121-288)
//   engine.inc    engine_t: quantize_x and gemv           (289-376)
//   ops.inc       v_expf, rmsnorm, rope, embed, silu_mul,
//                 softmax_exp, attention_group            (528-706)
//   init.inc      runtime::init                           (809-820)
//   forward.inc   runtime::forward                        (822-883)
//   sample.inc    runtime::sample_token                   (885-925)
// What the host lacks is stood in for, in this file and in oracle/refshim/:
//   * NEON: refshim/arm_neon.h (lane-by-lane ACLE semantics; vaddvq_f32 as
//     (a0 + a1) + (a2 + a3), the one assumption);
//   * ggml/gguf: refshim/ggml.h (float16 conversion) and refshim/gguf.h (a
//     GGUF reader with the calls the model section makes);
//   * the FPGA engine behind board/kv260gemv/gemv_dev.h and gemv2_dev.h (the
//     reference's own headers, included from its checkout): the GEMV is the
//     pinned C restatement of q4_0.py (oracle/q4_0_oracle.c, checked against
//     the reference contract's golden digest), reading the engine's buffers
//     exactly where the reference's driver would point the fabric: the four
//     port quarters of gemv_dev_start4, or gemv2's interleaved chunks;
//   * u-dma-buf: host memory, physical address = virtual address;
//   * the TCP mesh (comm_t): ranks are threads of this process; the
//     all-reduce sums in rank order (tp_llama.cpp:515-521) and the all-gather
//     copies every rank's bytes;
//   * the stats sampler: empty samples.
#include <arm_neon.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "ggml.h"
#include "gguf.h"

extern "C" {
#include "gemv_dev.h"
#include "gemv2_dev.h"
#include "q4_0_oracle.h"
#include "udmabuf.h"
}

namespace {
struct ref_die {};
int g_gemv_threads = 1;   // oracle threads per engine call (ranks run side by side)
bool g_use_gemv2 = false; // which engine the stand-in overlay "provides"
}  // namespace

#define DIE(...)                                       \
    do {                                               \
        fprintf(stderr, "ref runtime: " __VA_ARGS__);  \
        fprintf(stderr, "\n");                         \
        throw ref_die();                               \
    } while (0)

static double now() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

// ---------------------------------------------------------------- u-dma-buf
// Host memory; the "physical" address of a byte is its virtual address. Every
// allocation of a pool is remembered so the harness can free it.
namespace {
std::mutex g_pool_mu;
std::map<int, std::vector<void *>> g_pool_blocks;
int g_pool_next = 1;
}  // namespace

extern "C" int udmabuf_open(udmabuf_t *b, const char *name) {
    (void)name;
    std::lock_guard<std::mutex> lock(g_pool_mu);
    memset(b, 0, sizeof *b);
    b->fd = g_pool_next++;
    b->size = SIZE_MAX;
    g_pool_blocks[b->fd];
    return 0;
}

extern "C" void udmabuf_close(udmabuf_t *b) {
    std::lock_guard<std::mutex> lock(g_pool_mu);
    for (void *p : g_pool_blocks[b->fd]) free(p);
    g_pool_blocks.erase(b->fd);
}

extern "C" void *udmabuf_alloc(udmabuf_t *b, size_t size, size_t align) {
    void *p = nullptr;
    if (posix_memalign(&p, align < sizeof(void *) ? sizeof(void *) : align, size ? size : 1)) return nullptr;
    memset(p, 0, size);
    std::lock_guard<std::mutex> lock(g_pool_mu);
    g_pool_blocks[b->fd].push_back(p);
    b->used += size;
    return p;
}

extern "C" void udmabuf_clean(const void *, size_t) {}
extern "C" void udmabuf_invalidate(const void *, size_t) {}

// ---------------------------------------------------------------- engines
namespace {

// y = W x for rows stored GGUF-style at `w` (k/32*18 bytes a row); x in the
// engine's layout, int8[k] then float32[k/32].
void engine_rows(const uint8_t *w, int rows, int k, uint64_t x, float *y) {
    if (oracle_gemv_q4_0_packed(w, rows, k, reinterpret_cast<const uint8_t *>(x), y, g_gemv_threads))
        DIE("stand-in engine: the oracle refused a %dx%d GEMV", rows, k);
}

struct fetch_state {
    uint64_t w[4];
    int k, rows;
    bool pending;
};
std::mutex g_fetch_mu;
std::map<const void *, fetch_state> g_fetch;

}  // namespace

extern "C" int gemv_dev_open(gemv_dev_t *d) {
    memset(d, 0, sizeof *d);
    return 0;
}
extern "C" int gemv_dev_open_named(gemv_dev_t *d, const char *, int) { return gemv_dev_open(d); }
extern "C" void gemv_dev_close(gemv_dev_t *) {}
extern "C" void gemv_dev_wait(gemv_dev_t *) {}

// Each engine m streams rows [m*R, (m+1)*R) from its own quarter (gemv_dev.h).
extern "C" void gemv_dev_start4(gemv_dev_t *, const uint64_t w[4], uint64_t x, uint64_t y, int k, int rows) {
    const int R = rows / 4;
    float *out = reinterpret_cast<float *>(y);
    for (int m = 0; m < 4; ++m) engine_rows(reinterpret_cast<const uint8_t *>(w[m]), R, k, x, out + m * R);
}

extern "C" void gemv_dev_start(gemv_dev_t *d, uint64_t w, uint64_t x, uint64_t y, int k, int rows) {
    const uint64_t q = static_cast<uint64_t>(rows / 4) * (k / 32) * 18;
    const uint64_t ws[4] = {w, w + q, w + 2 * q, w + 3 * q};
    gemv_dev_start4(d, ws, x, y, k, rows);
}

extern "C" void gemv_dev_run(gemv_dev_t *d, uint64_t w, uint64_t x, uint64_t y, int k, int rows) {
    gemv_dev_start(d, w, x, y, k, rows);
}

extern "C" int gemv2_dev_open(gemv2_dev_t *d) {
    memset(d, 0, sizeof *d);
    return g_use_gemv2 ? 0 : -1;
}
extern "C" void gemv2_dev_close(gemv2_dev_t *) {}
extern "C" int gemv2_mac_idle(gemv2_dev_t *) { return 1; }
extern "C" void gemv2_drain(gemv2_dev_t *d) {
    std::lock_guard<std::mutex> lock(g_fetch_mu);
    g_fetch[d].pending = false;
}
extern "C" void gemv2_fetch_wait(gemv2_dev_t *) {}
extern "C" void gemv2_mac_wait(gemv2_dev_t *) {}

extern "C" void gemv2_fetch_start(gemv2_dev_t *d, const uint64_t w[4], int k, int rows) {
    std::lock_guard<std::mutex> lock(g_fetch_mu);
    fetch_state &f = g_fetch[d];
    memcpy(f.w, w, sizeof f.w);
    f.k = k;
    f.rows = rows;
    f.pending = true;
}

// The MAC consumes the matrix the last fetch streamed: row r's chunk c sits
// at gemv2_chunk_offset(r, c, ...) inside port region p.
extern "C" void gemv2_mac_start(gemv2_dev_t *d, uint64_t x, uint64_t y, int k, int rows) {
    fetch_state f;
    {
        std::lock_guard<std::mutex> lock(g_fetch_mu);
        f = g_fetch[d];
        g_fetch[d].pending = false;
    }
    if (!f.pending || f.k != k || f.rows != rows) DIE("stand-in gemv2: MAC without the matching fetch");
    const int nch = k / 256;
    const size_t rb = static_cast<size_t>(k) / 32 * 18;
    std::vector<uint8_t> flat(rb * rows);
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < nch; ++c) {
            int p = 0;
            const size_t o = gemv2_chunk_offset(r, c, rows, k, &p);
            memcpy(flat.data() + r * rb + static_cast<size_t>(c) * GEMV2_CHUNK_BYTES,
                   reinterpret_cast<const uint8_t *>(f.w[p]) + o, GEMV2_CHUNK_BYTES);
        }
    engine_rows(flat.data(), rows, k, x, reinterpret_cast<float *>(y));
}

// ---------------------------------------------------------------- the reference's sections
#include "memory.inc"
#include "model.inc"
#include "engine.inc"
#include "ops.inc"

// ---------------------------------------------------------------- mesh stand-in
namespace {

// The ranks of one simulated run: a generation barrier and a pointer slot
// per rank.
struct mesh {
    int n = 1;
    std::mutex mu;
    std::condition_variable cv;
    int arrived = 0;
    unsigned gen = 0;
    std::vector<const void *> ptr;
    void wait() {
        std::unique_lock<std::mutex> lock(mu);
        const unsigned g = gen;
        if (++arrived == n) {
            arrived = 0;
            ++gen;
            cv.notify_all();
        } else {
            cv.wait(lock, [&] { return gen != g; });
        }
    }
};

}  // namespace

// comm_t as runtime::forward and sample_token use it.
struct comm_t {
    mesh *m = nullptr;
    int rank = 0, n = 1;
    // Every rank ends with s = p0 + p1 + ... + p{n-1} per element, summed
    // left to right (tp_llama.cpp:515-521).
    void allreduce_sum(float *v, int len, std::vector<float> &scratch) {
        if (n == 1) return;
        m->ptr[rank] = v;
        m->wait();
        scratch.resize(len);
        for (int i = 0; i < len; ++i) {
            float s = 0;
            for (int r = 0; r < n; ++r) {
                const float p = static_cast<const float *>(m->ptr[r])[i];
                s = r == 0 ? p : s + p;
            }
            scratch[i] = s;
        }
        m->wait();
        memcpy(v, scratch.data(), sizeof(float) * len);
    }
    void allgather(const uint8_t *mine, uint8_t *all, int len) {
        m->ptr[rank] = mine;
        m->wait();
        for (int r = 0; r < n; ++r) memcpy(all + static_cast<size_t>(r) * len, m->ptr[r], len);
        m->wait();
    }
};

struct rank_stats {
    float engine_ms = 0, comm_ms = 0, cpu_ms = 0;
};

struct stats_stub {
    void discover() {}
    rank_stats sample(double, double, double, int) { return rank_stats{}; }
};

// The members of struct runtime (tp_llama.cpp:783-808) that init, forward
// and sample_token touch, around their own text.
struct ref_runtime {
    model_t M;
    engine_t E;
    comm_t C;
    int ctx_max = 0;
    std::vector<float> kcache, vcache;
    std::vector<float> x, h, qkv, attn_out, partial, act, scratch, scores, rope_cs;
    double t_engine = 0, t_comm = 0, t_cpu = 0;
    stats_stub sampler;
    std::vector<rank_stats> latest;
    double latest_t = 0;
    int tokens_total = 0;

#include "init.inc"
#include "forward.inc"
#include "sample.inc"
};

namespace {

struct ref_rank {
    ref_runtime R;
    pools_t pools;
    gguf_file f;
    std::pair<int, float> last{0, 0.0f};
    int token = 0;
    bool failed = false;
};

struct ref_handle {
    mesh net;
    std::vector<ref_rank *> ranks;
};

}  // namespace

extern "C" {

// Load a GGUF Q4_0 model as `nranks` ranks of the reference runtime would
// (main, tp_llama.cpp:1271-1279): probe the engine, load_model, open the
// engine, init. Returns 0, or -1 when the reference code DIEs.
int ref_open(const char *gguf_path, int nranks, int ctx_max, int use_gemv2, int threads, void **out) {
    if (!gguf_path || nranks < 1 || nranks > 8 || ctx_max < 1 || !out) return -2;
    g_use_gemv2 = use_gemv2 != 0;
    g_gemv_threads = threads > 0 ? threads : 1;
    ref_handle *H = new ref_handle();
    H->net.n = nranks;
    H->net.ptr.assign(nranks, nullptr);
    try {
        for (int r = 0; r < nranks; ++r) {
            ref_rank *K = new ref_rank();
            H->ranks.push_back(K);
            K->R.M.rank = r;
            K->R.M.nranks = nranks;
            K->pools.open();
            K->f.open(gguf_path);
            K->R.E.probe();
            load_model(K->R.M, K->f, K->pools, K->R.E.v2);
            K->R.E.open(K->pools, std::max(K->R.M.vocab_rows, 2 * K->R.M.ff_rows));
            K->R.C.m = &H->net;
            K->R.C.rank = r;
            K->R.C.n = nranks;
            K->R.init(ctx_max);
        }
    } catch (const ref_die &) {
        for (ref_rank *K : H->ranks) {
            for (auto &b : K->pools.p) udmabuf_close(&b);
            delete K;
        }
        delete H;
        return -1;
    }
    *out = H;
    return 0;
}

// runtime::forward on every rank (one thread each), then sample_token with
// temperature 0 (the greedy pick every rank agrees on). *val is the winning
// logit, read from the rank that owns it.
int ref_forward(void *h, int token, int pos, int *tok, float *val) {
    ref_handle *H = static_cast<ref_handle *>(h);
    if (!H || !tok || !val) return -2;
    std::vector<std::thread> th;
    for (ref_rank *K : H->ranks) {
        K->failed = false;
        th.emplace_back([K, token, pos] {
            try {
                K->last = K->R.forward(token, pos);
                ref_runtime::sampling sp;
                sp.temperature = 0.0f;
                K->token = K->R.sample_token(sp);
            } catch (const ref_die &) {
                K->failed = true;
            }
        });
    }
    for (std::thread &t : th) t.join();
    for (ref_rank *K : H->ranks)
        if (K->failed) return -1;
    const int t = H->ranks[0]->token;
    for (ref_rank *K : H->ranks)
        if (K->token != t) return -3;
    const ref_runtime &owner = H->ranks[t / H->ranks[0]->R.M.vocab_rows]->R;
    *tok = t;
    *val = owner.E.y[t - owner.M.rank * owner.M.vocab_rows];
    return 0;
}

// 0: the residual stream x; 1: rank `rank`'s logits (the engine's y after
// lm_head); 2: the last RMSNorm output h.
int ref_read(void *h, int what, int rank, float *out, int64_t n) {
    ref_handle *H = static_cast<ref_handle *>(h);
    if (!H || !out || rank < 0 || rank >= static_cast<int>(H->ranks.size())) return -2;
    const ref_runtime &R = H->ranks[rank]->R;
    if (what == 0 && n == static_cast<int64_t>(R.x.size())) memcpy(out, R.x.data(), 4 * n);
    else if (what == 1 && n == R.M.vocab_rows) memcpy(out, R.E.y, 4 * n);
    else if (what == 2 && n == static_cast<int64_t>(R.h.size())) memcpy(out, R.h.data(), 4 * n);
    else return -2;
    return 0;
}

void ref_close(void *h) {
    ref_handle *H = static_cast<ref_handle *>(h);
    if (!H) return;
    for (ref_rank *K : H->ranks) {
        for (auto &b : K->pools.p) udmabuf_close(&b);
        delete K;
    }
    delete H;
}

// ---- the ops section's functions, one call each
void ref_v_expf4(const float *in, float *out) { vst1q_f32(out, v_expf(vld1q_f32(in))); }
void ref_rmsnorm(float *out, const float *x, const float *w, int n, float eps) { rmsnorm(out, x, w, n, eps); }
void ref_rope_table(float *cs, int d, int pos, float base) { rope_table(cs, d, pos, base, nullptr); }
void ref_rope(float *x, int n_heads, int d, const float *cs) { rope(x, n_heads, d, cs); }
void ref_embed(float *out, const uint8_t *token_embd, int token, int n_embd) { embed(out, token_embd, token, n_embd); }
void ref_silu_mul(float *act, const float *gate, const float *up, int n) { silu_mul(act, gate, up, n); }
float ref_softmax_exp(float *s, int n, float mx) { return softmax_exp(s, n, mx); }
void ref_attention_heads(int n, const float *q, const float *kc, const float *vc, int64_t stride, int pos, int d,
                         float scale, float *sc, int sc_stride, float *out) {
    attention_heads(n, q, kc, vc, static_cast<size_t>(stride), pos, d, scale, sc, sc_stride, out);
}
// engine_t::quantize_x: int8[k] then float32[k/32], the runtime's roundf rule
void ref_quantize_x(const float *x, int8_t *qs, float *xd, int k) { engine_t::quantize_x(x, qs, xd, k); }

}  // extern "C"
