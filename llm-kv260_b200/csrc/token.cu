// Persistent decode kernel: `ntokens` greedy decode tokens of the reference
// runtime's forward() (board/tp/tp_llama.cpp:822-883) in ONE cooperative
// launch, one CTA per SM.
//
// A token is a list of phases (TokenPhase, built by decoder.cu): per layer
// q|k|v GEMV, attention, o GEMV, gate|up GEMV, down GEMV; then lm_head.
// Consecutive phases are separated by a grid-wide barrier on one 64-bit
// arrival counter that only ever grows (barrier m of the decoder's life is
// passed when the counter reaches (m + 1) * grid), so nothing is reset
// between tokens or launches.
//
// Warp roles. The last warp is the producer: one thread walks the CTA's
// share of every GEMV phase of every token (contiguous 16-row groups, as the
// tile kernel splits them) and streams each group's tiles, 8 chunks = 18,432
// bytes per stage, into a ring of shared-memory stages with 1-D bulk copies
// (no multicast), limited only by free stages -- never by the phase barriers,
// so while the CTAs wait at a barrier the next phases' weights keep arriving.
// The other NWG warpgroups are consumers: at each phase they stage x (with
// the decoder's prologue: plain, RMSNorm, or the token's embedding + RMSNorm),
// then each warpgroup takes every NWG-th row group, runs its lane chains over
// the group's stages in order and applies the epilogue (store, RoPE + KV
// cache, SiLU pairs, residual add -- with several ranks the rank-ordered sum
// of the peers' partial rows, pushed and read through the communicator's
// windows). Attention runs on the first kvh_local CTAs. After lm_head every
// CTA reduces the per-CTA pick candidates itself (no extra barrier) and CTA 0
// advances the loop state for the host.
//
// All arithmetic is the tile kernel's and the attention kernel's, in the
// same order, so results are bit-identical to the per-kernel decoder and to
// the C oracle of forward(). Data written by other CTAs inside the launch is
// read with L2-coherent loads (ld.global.cg); only constants (weights, norm
// weights, the embedding and RoPE tables) go through the read-only path.
//
// Every wait is bounded (2 s; peers 1 s); a wait that runs out sets a status
// bit and the abort flag, every CTA then leaves at its next wait, and the
// producer first lets its own copies in flight land.
#include <cuda_fp16.h>

#include <cmath>

#include "attn_core.cuh"
#include "common.cuh"
#include "decode.cuh"
#include "decode.h"

namespace b200 {

namespace {

constexpr int kStage = 8 * kTileBytes;  // 18432: 8 chunks of one 16-row group
constexpr int kMaxRing = 16;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint64_t kPeerWaitNs = 1000000000ull;
constexpr int kMaxBatch = 4;       // row groups a warpgroup runs side by side

struct MkParams {
    TokenArgs a;
    int ring;  // stages in the ring
    int off_xs, off_xf, off_dred, off_red, off_best, off_attn;
};

// ------------------------------------------------------------------ waits

__device__ __forceinline__ bool aborted(const MkParams &p) {
    return *reinterpret_cast<volatile int *>(p.a.abort_flag) != 0;
}

__device__ __forceinline__ void set_abort(const MkParams &p, unsigned bit) {
    atomicOr(p.a.status, bit);
    atomicExch(p.a.abort_flag, 1);
}

__device__ __noinline__ bool mk_wait_slow(const MkParams &p, uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    for (unsigned spin = 0;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 255u) == 255u) {
            if (aborted(p)) return false;
            if (globaltimer_ns() - t0 > kWaitNs) {
                set_abort(p, kStatusStageTimeout);
                return false;
            }
        }
    }
}

// Bounded mbarrier wait; the first try inline, the rest out of line.
__device__ __forceinline__ bool mk_wait(const MkParams &p, uint64_t *bar, uint32_t parity) {
    return mbar_try_wait(bar, parity) || mk_wait_slow(p, bar, parity);
}

// Consumer thread 0: wait until `target` arrivals (bounded).
__device__ bool mk_grid_wait(const MkParams &p, uint64_t target) {
    const uint64_t t0 = globaltimer_ns();
    for (unsigned spin = 0;; ++spin) {
        if (*reinterpret_cast<volatile unsigned long long *>(p.a.bar_count) >= target) {
            __threadfence();  // acquire: the arrivals' writes before anything this CTA reads next
            return true;
        }
        if ((spin & 63u) == 63u) {
            if (aborted(p)) return false;
            if (globaltimer_ns() - t0 > kWaitNs) {
                set_abort(p, kStatusStageTimeout);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void st_word(uint64_t *p, uint64_t w) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// (value desc, index asc); NaN never beats a number (tp_llama.cpp:879-882 for
// every index but 0, which the final step handles).
__device__ __forceinline__ bool pick_better(float av, int ai, float bv, int bi) {
    if (isnan(bv)) return !isnan(av) || ai < bi;
    if (isnan(av)) return false;
    return av > bv || (av == bv && ai < bi);
}

// Optional phase trace, 8 values per (token t, phase i, CTA): stamps 0 phase
// start, 1 x staged, 2 warpgroup 0's rows done, 3 phase end; 4 and 5 the ns
// warpgroups 0 and 1 spent waiting for weight stages, 6 warpgroup 1's rows
// done.
__device__ __forceinline__ uint64_t *trace_rec(const TokenArgs &a, int t, int i) {
    return (a.trace && t < a.trace_tokens) ? a.trace + ((static_cast<size_t>(t) * a.nphases + i) * gridDim.x + blockIdx.x) * 8
                                           : nullptr;
}

// stamp j of (token t, phase i) for this CTA
__device__ __forceinline__ void stamp(const TokenArgs &a, int t, int i, int j) {
    if (a.trace && t < a.trace_tokens && threadIdx.x == 0)
        a.trace[((static_cast<size_t>(t) * a.nphases + i) * gridDim.x + blockIdx.x) * 8 + j] = globaltimer_ns();
}

// ------------------------------------------------------------------ producer

__device__ void mk_producer(const MkParams &p, uint8_t *ring, uint64_t *full, uint64_t *empty) {
    const TokenArgs &a = p.a;
    const int S = p.ring, G = gridDim.x, cta = blockIdx.x;
    const uint64_t pol = l2_policy_evict_first();
    uint32_t s = 0;
    bool ok = true;
    for (int t = 0; t < a.ntokens && ok; ++t) {
        for (int i = 0; i < a.nphases && ok; ++i) {
            const TokenPhase &ph = a.phases[i];
            if (ph.kind != kPhGemv) continue;
            const int groups = (ph.rows + kTileRows - 1) / kTileRows, nch = ph.k / 256;
            const int g0 = static_cast<int>(static_cast<long long>(groups) * cta / G);
            const int g1 = static_cast<int>(static_cast<long long>(groups) * (cta + 1) / G);
            for (int g = g0; g < g1 && ok; ++g)
                for (int c0 = 0; c0 < nch; c0 += 8) {
                    const int slot = static_cast<int>(s % S);
                    const uint32_t use = s / S;
                    if (use > 0 && !mk_wait(p, &empty[slot], (use & 1u) ^ 1u)) {
                        ok = false;
                        break;
                    }
                    const int nc = min(8, nch - c0);
                    const uint32_t bytes = static_cast<uint32_t>(nc * kTileBytes);
                    mbar_arrive_expect_tx(&full[slot], bytes);
                    bulk_g2s(ring + static_cast<size_t>(slot) * kStage,
                             ph.w + (static_cast<size_t>(g) * nch + c0) * kTileBytes, bytes, &full[slot], pol);
                    ++s;
                }
            if (aborted(p)) ok = false;
        }
    }
    // Leave only after the copies this CTA issued have landed (at once when
    // the consumers took them all; after an abort, each wait bounded).
    const uint32_t first = s > static_cast<uint32_t>(S) ? s - S : 0;
    for (uint32_t r = first; r < s; ++r) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[r % S], (r / S) & 1u))
            if (globaltimer_ns() - t0 > kWaitNs) break;
    }
}

// ------------------------------------------------------------------ x staging

// Q8_0 of one 32-block by a group of TPB threads (thread j of the group holds
// values [j*V, (j+1)*V), V = 32/TPB) into xs, the tile kernel's layout. The
// same values as q8_quant_block (q4_0.py:83-97): the block's largest |x|
// and the sum of its ints do not depend on the order they are combined in.
// All 32 lanes of a warp take part in the shuffles; inactive groups hold 0.
template <int TPB>
__device__ __forceinline__ void quant_group(const float *v, bool active, int b, int j, uint8_t *xs, int k,
                                            int round_mode) {
    constexpr int V = 32 / TPB;
    float m = fabsf(v[0]);
#pragma unroll
    for (int i = 1; i < V; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
    for (int off = 1; off < TPB; off <<= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
    const float db = __fdiv_rn(m, 127.0f);
    const float inv = db == 0.0f ? 0.0f : __fdiv_rn(1.0f, db);
    int sum = 0;
    uint32_t w[V / 4];
#pragma unroll
    for (int i = 0; i < V; i += 4) {
        const int q0 = q8_round(__fmul_rn(v[i], inv), round_mode);
        const int q1 = q8_round(__fmul_rn(v[i + 1], inv), round_mode);
        const int q2 = q8_round(__fmul_rn(v[i + 2], inv), round_mode);
        const int q3 = q8_round(__fmul_rn(v[i + 3], inv), round_mode);
        sum += q0 + q1 + q2 + q3;
        w[i / 4] = (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
                   ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
    }
#pragma unroll
    for (int off = 1; off < TPB; off <<= 1) sum += __shfl_xor_sync(kFullMask, sum, off);
    if (!active) return;
    uint32_t *dst = reinterpret_cast<uint32_t *>(xs_block(xs, b) + j * V);
#pragma unroll
    for (int i = 0; i < V / 4; ++i) dst[i] = w[i];
    if (j == 0) xs_scales(xs, k)[b] = make_int2(__float_as_int(__half2float(__float2half_rn(db))), sum);
}

template <int NWG, int TPB>
__device__ void stage_plain(const TokenPhase &ph, int round_mode, uint8_t *xs) {
    constexpr int V = 32 / TPB;
    const int nb = ph.k / kQK, b = threadIdx.x / TPB, j = threadIdx.x % TPB;
    const bool active = b < nb;
    float v[V];
    if (active) {
        const float4 *src = reinterpret_cast<const float4 *>(ph.x + 32 * b + j * V);
#pragma unroll
        for (int q = 0; q < V / 4; ++q) {
            const float4 f = __ldcg(src + q);
            v[4 * q] = f.x;
            v[4 * q + 1] = f.y;
            v[4 * q + 2] = f.z;
            v[4 * q + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = 0.0f;
    }
    quant_group<TPB>(v, active, b, j, xs, ph.k, round_mode);
}

// RMSNorm prologue (see stage_x_norm in q4tile.cu for the reasoning): x is
// the residual, or the token's embedding row (write_embedding puts that row
// into res). Groups of TPB threads per 32-block, as stage_plain; the norm
// weights are loaded together with x.
template <int NWG, int TPB>
__device__ void stage_norm(const MkParams &p, const TokenPhase &ph, int tok, uint8_t *xs, float *xf, double *dred,
                           volatile float *s_f, volatile int *s_exact) {
    constexpr int kThreads = NWG * 128;
    constexpr int V = 32 / TPB;
    const TokenArgs &a = p.a;
    const int k = ph.k, nb = k / kQK, b = threadIdx.x / TPB, j = threadIdx.x % TPB;
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    const bool active = b < nb;
    float v[V], w[V];
    double ss = 0.0;
    if (active) {
        const float4 *wv = reinterpret_cast<const float4 *>(ph.norm_w + 32 * b + j * V);
#pragma unroll
        for (int q = 0; q < V / 4; ++q) {
            const float4 f = __ldg(wv + q);
            w[4 * q] = f.x;
            w[4 * q + 1] = f.y;
            w[4 * q + 2] = f.z;
            w[4 * q + 3] = f.w;
        }
        if (ph.pro == kProEmbedNorm) {
            const uint8_t *blk = a.embd + (static_cast<size_t>(tok) * nb + b) * kBlockBytes;
            const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(blk))));
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const int e = j * V + i;  // value e: byte e & 15, low nibble below 16
                const int byte = __ldg(blk + 2 + (e & 15));
                v[i] = __fmul_rn(__int2float_rn((e < 16 ? (byte & 0xF) : (byte >> 4)) - 8), d);
            }
        } else {
            const float4 *src = reinterpret_cast<const float4 *>(a.res + 32 * b + j * V);
#pragma unroll
            for (int q = 0; q < V / 4; ++q) {
                const float4 f = __ldcg(src + q);
                v[4 * q] = f.x;
                v[4 * q + 1] = f.y;
                v[4 * q + 2] = f.z;
                v[4 * q + 3] = f.w;
            }
        }
#pragma unroll
        for (int i = 0; i < V; ++i) ss = __dadd_rn(ss, __dmul_rn(static_cast<double>(v[i]), static_cast<double>(v[i])));
        float4 *xd = reinterpret_cast<float4 *>(xf + 32 * b + j * V);
#pragma unroll
        for (int q = 0; q < V / 4; ++q) xd[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = w[i] = 0.0f;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(kFullMask, ss, off));
    if (lane == 0) dred[warp] = ss;
    named_sync(1, kThreads);
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int q = 0; q < kThreads / 32; ++q) tot = __dadd_rn(tot, dred[q]);
        const double qv = __ddiv_rn(tot, static_cast<double>(k));
        const float f = __double2float_rn(qv);
        *s_exact = a.exact_norm || !rms_float_is_safe(qv, f, k);
        *s_f = f;
    }
    named_sync(1, kThreads);
    if (*s_exact) {
        if (threadIdx.x < 4) {
            double acc = 0.0;
            for (int i = threadIdx.x; i < k; i += 4)
                acc = __dadd_rn(acc, __dmul_rn(static_cast<double>(xf[i]), static_cast<double>(xf[i])));
            dred[threadIdx.x] = acc;
        }
        named_sync(1, kThreads);
        if (threadIdx.x == 0) {
            const double ss2 = __dadd_rn(__dadd_rn(dred[0], dred[2]), __dadd_rn(dred[1], dred[3]));
            *s_f = __double2float_rn(__ddiv_rn(ss2, static_cast<double>(k)));
        }
        named_sync(1, kThreads);
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(*s_f, a.eps)));
    float h[V];
#pragma unroll
    for (int i = 0; i < V; ++i) h[i] = __fmul_rn(__fmul_rn(v[i], scale), w[i]);
    quant_group<TPB>(h, active, b, j, xs, k, a.round_mode);
}

// Threads per x block for a phase: as many as fit, up to 8.
__device__ __forceinline__ int group_size(int k, int threads) {
    int tpb = 8;
    while (tpb > 1 && (k / kQK) * tpb > threads) tpb >>= 1;
    return tpb;
}

// embed (tp_llama.cpp:593-604): the token's row of token_embd into res, one
// thread per 32-block; CTA 0 does it whether or not it has rows in the phase.
__device__ void write_embedding(const TokenArgs &a, int k, int tok) {
    const int nb = k / kQK, b = threadIdx.x;
    if (b >= nb) return;
    const uint16_t *blk = reinterpret_cast<const uint16_t *>(a.embd + (static_cast<size_t>(tok) * nb + b) * kBlockBytes);
    uint16_t h[9];
#pragma unroll
    for (int j = 0; j < 9; ++j) h[j] = __ldg(blk + j);
    const float d = __half2float(__ushort_as_half(h[0]));
    float v[32];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int byte = (h[1 + j / 2] >> (8 * (j & 1))) & 0xff;
        v[j] = __fmul_rn(__int2float_rn((byte & 0xF) - 8), d);
        v[j + 16] = __fmul_rn(__int2float_rn((byte >> 4) - 8), d);
    }
    float4 *dst = reinterpret_cast<float4 *>(a.res) + 8 * b;
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// ------------------------------------------------------------------ GEMV phase

// Block term of chunk-tile `tile` for thread u = lane * 16 + row; the tile
// holds row i, lane l at (i * 8 + l) (q4tile.cu).
__device__ __forceinline__ float mk_term(const uint8_t *tile, int u, const XBlock &xb) {
    const int v = (u % kTileRows) * kLanes + u / kTileRows;
    const uint4 nv = *reinterpret_cast<const uint4 *>(tile + v * 16);
    const uint32_t db = *reinterpret_cast<const uint16_t *>(tile + kTileRows * kLanes * 16 + v * 2);
    const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
    return block_term_words(n, db, xb);
}

struct PhaseCtx {
    int P;          // position of this token
    uint32_t step;  // tokens done before this one (exchange epochs)
    int tok;        // this token's id
};

template <int NWG>
__device__ void gemv_phase(const MkParams &p, const TokenPhase &ph, const PhaseCtx &cx, uint8_t *smem, uint8_t *ring,
                           uint64_t *full, uint64_t *empty, uint32_t &s, volatile float *s_f, volatile int *s_exact,
                           volatile int *s_fail, int t, int i) {
    constexpr int kThreads = NWG * 128;
    const TokenArgs &a = p.a;
    const int tid = threadIdx.x, wg = tid / 128, u = tid % 128, L = u / kTileRows;
    const int S = p.ring, G = gridDim.x, cta = blockIdx.x;
    const int groups = (ph.rows + kTileRows - 1) / kTileRows, nch = ph.k / 256, spi = (nch + 7) / 8;
    const int g0 = static_cast<int>(static_cast<long long>(groups) * cta / G);
    const int g1 = static_cast<int>(static_cast<long long>(groups) * (cta + 1) / G);
    const int nitems = g1 - g0;
    uint8_t *xs = smem + p.off_xs;
    float *red = reinterpret_cast<float *>(smem + p.off_red);  // [NWG][2][kMaxBatch][128]
    float2 *best = reinterpret_cast<float2 *>(smem + p.off_best);
    float best_v = __int_as_float(0x7fc00000);
    int best_i = 0x7fffffff;
    if (ph.pro == kProEmbedNorm && cta == 0) write_embedding(a, ph.k, cx.tok);
    if (nitems > 0) {
        float *xf = reinterpret_cast<float *>(smem + p.off_xf);
        double *dred = reinterpret_cast<double *>(smem + p.off_dred);
        const int tpb = group_size(ph.k, kThreads);
        if (ph.pro == kProPlain) {
            if (tpb == 8) stage_plain<NWG, 8>(ph, a.round_mode, xs);
            else if (tpb == 4) stage_plain<NWG, 4>(ph, a.round_mode, xs);
            else if (tpb == 2) stage_plain<NWG, 2>(ph, a.round_mode, xs);
            else stage_plain<NWG, 1>(ph, a.round_mode, xs);
        } else {
            // a normalised x is n_embd <= 2 x 32 x threads long (make_params), so 2+ threads a block
            if (tpb == 8) stage_norm<NWG, 8>(p, ph, cx.tok, xs, xf, dred, s_f, s_exact);
            else if (tpb == 4) stage_norm<NWG, 4>(p, ph, cx.tok, xs, xf, dred, s_f, s_exact);
            else stage_norm<NWG, 2>(p, ph, cx.tok, xs, xf, dred, s_f, s_exact);
        }
        named_sync(1, kThreads);
    }
    stamp(a, t, i, 1);
    const bool xchg = ph.epi == kEpiResidual && a.nranks > 1;
    uint32_t epoch = 0;
    uint64_t slot_off = 0;
    if (xchg) {
        epoch = cx.step * static_cast<uint32_t>(a.ar_per_token) + static_cast<uint32_t>(ph.ar_index) + 1u;
        slot_off = static_cast<uint64_t>(epoch & 1u) * kMaxDecodeRanks * a.slot_words;
    }
    // Row groups go to the warpgroups in blocks of R consecutive ones (block
    // b to warpgroup b % NWG). A warpgroup runs its R groups' lane chains side
    // by side, sharing each x block; R * NWG * spi stages fit in the ring, so
    // every warpgroup's current groups can sit in shared memory at once and
    // the ring's in-order reuse cannot stall a warpgroup on another's stages.
    // s_fail[wg]: a wait of this warpgroup gave up; every decision to leave a
    // loop is read from it after a barrier, so the warpgroup leaves together.
    // as many groups side by side as spread this CTA's share evenly
    const int R = max(1, min(min(kMaxBatch, (nitems + NWG - 1) / NWG), S / (NWG * spi)));
    uint64_t *trec = u == 0 ? trace_rec(a, t, i) : nullptr;
    uint64_t waited = 0;
    int rb = 0;
    for (int blk = wg; blk * R < nitems; blk += NWG) {
        const int j0 = blk * R, nr = min(R, nitems - j0);
        float acc[kMaxBatch];
#pragma unroll
        for (int r = 0; r < kMaxBatch; ++r) acc[r] = 0.0f;
        bool fail = false;
        for (int cs = 0; cs < spi; ++cs) {
            const uint8_t *tl[kMaxBatch];
            bool ok = true;
            const uint64_t w0 = trec ? globaltimer_ns() : 0;
#pragma unroll
            for (int r = 0; r < kMaxBatch; ++r) {
                tl[r] = ring;
                if (r < nr) {
                    const uint32_t idx = s + static_cast<uint32_t>((j0 + r) * spi + cs);
                    const int slot = static_cast<int>(idx % S);
                    if (!mk_wait(p, &full[slot], (idx / S) & 1u)) ok = false;
                    tl[r] = ring + static_cast<size_t>(slot) * kStage;
                }
            }
            if (trec) waited += globaltimer_ns() - w0;
            if (!ok) s_fail[wg] = 1;
            if (ok) {
                const int nc = min(8, nch - 8 * cs);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (c < nc) {
                        XBlock xb;
                        load_xblock_smem(xs, ph.k, 8 * (8 * cs + c) + L, xb);
#pragma unroll
                        for (int r = 0; r < kMaxBatch; ++r)
                            if (r < nr) acc[r] = __fadd_rn(acc[r], mk_term(tl[r] + c * kTileBytes, u, xb));
                    }
                }
            }
            named_sync(2 + wg, 128);
            fail = s_fail[wg] != 0;
            if (u < nr && !fail) {  // thread r frees group r's stage
                const uint32_t idx = s + static_cast<uint32_t>((j0 + u) * spi + cs);
                mbar_arrive(&empty[idx % S]);
            }
            if (fail) break;
        }
        if (fail) break;
        float *rbuf = red + (wg * 2 + rb) * (kMaxBatch * 128);
#pragma unroll
        for (int r = 0; r < kMaxBatch; ++r)
            if (r < nr) rbuf[r * 128 + u] = acc[r];
        named_sync(2 + wg, 128);
        rb ^= 1;
        if (u < kMaxBatch * kTileRows) {
            // 64 threads (two whole warps): group r = u / 16, row u % 16
            const int r = u / kTileRows, ri = u % kTileRows;
            const bool have = r < nr;
            const float *rr = rbuf + r * 128;
            const float yv = have ? tree8(rr[0 * 16 + ri], rr[1 * 16 + ri], rr[2 * 16 + ri], rr[3 * 16 + ri],
                                          rr[4 * 16 + ri], rr[5 * 16 + ri], rr[6 * 16 + ri], rr[7 * 16 + ri])
                                  : 0.0f;
            const int row = (g0 + j0 + r) * kTileRows + ri;
            const bool live = have && row < ph.rows;
            if (ph.epi == kEpiStore) {
                if (live) {
                    ph.y[row] = yv;
                    if (ph.pick && pick_better(yv, row, best_v, best_i)) {
                        best_v = yv;
                        best_i = row;
                    }
                }
            } else if (ph.epi == kEpiRopeKv) {
                // q and k rows start at multiples of head_dim (even), a group at
                // a multiple of 16: rope's pair (2i, 2i+1) is this thread and u ^ 1
                const float other = __shfl_xor_sync(kFullMask, yv, 1);
                if (live) {
                    const int hd = a.head_dim, k0 = a.q_rows, v0 = k0 + a.kv_rows;
                    float out = yv;
                    if (row < v0) {
                        const int i2 = (row % hd) >> 1;
                        const float *cs = a.rope_cs + static_cast<size_t>(cx.P) * hd;
                        const bool even = !(row & 1);
                        out = rope_pair(even ? yv : other, even ? other : yv, __ldg(cs + 2 * i2), __ldg(cs + 2 * i2 + 1),
                                        even);
                    }
                    ph.y[row] = out;
                    if (row >= k0) {
                        // K rows [kv head][stride][hd], lane-major and swizzled by
                        // position (k_slot); V transposed, [kv head][hd][stride]
                        const bool isk = row < v0;
                        const int q = row - (isk ? k0 : v0);
                        const size_t at = isk ? (static_cast<size_t>(q / hd) * a.kv_stride + cx.P) * hd +
                                                    k_slot(q % hd, cx.P, a.kv_f16 ? 2 : 4, hd)
                                              : static_cast<size_t>(q) * a.kv_stride + cx.P;
                        void *cache = isk ? ph.kcache : ph.vcache;
                        if (a.kv_f16)
                            static_cast<__half *>(cache)[at] = __float2half_rn(out);
                        else
                            static_cast<float *>(cache)[at] = out;
                    }
                }
            } else if (ph.epi == kEpiSiluPairs) {
                const float other = __shfl_xor_sync(kFullMask, yv, 1);
                if (live && !(row & 1)) ph.act[row >> 1] = silu_mul(yv, other);
            } else if (live) {  // kEpiResidual
                if (!xchg) {
                    a.res[row] = __fadd_rn(__ldcg(a.res + row), yv);
                } else {
                    const uint64_t word = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(yv);
                    const uint64_t at = slot_off + static_cast<uint64_t>(a.rank) * a.slot_words + row;
                    for (int q = 0; q < a.nranks; ++q) st_word(a.win_words[q] + at, word);
                }
            }
        }
    }
    s += static_cast<uint32_t>(nitems * spi);
    if (trec && wg < 2) {
        trec[wg == 0 ? 2 : 6] = globaltimer_ns();
        trec[4 + wg] = waited;
    }
    if (xchg && u < kMaxBatch * kTileRows && !s_fail[wg]) {
        // the peers' partials of this warpgroup's rows, summed in rank order
        const uint64_t *own = a.win_words[a.rank] + slot_off;
        const int r = u / kTileRows, ri = u % kTileRows;
        for (int blk = wg; blk * R < nitems; blk += NWG) {
            const int j0 = blk * R, nr = min(R, nitems - j0);
            if (r >= nr) continue;
            const int row = (g0 + j0 + r) * kTileRows + ri;
            if (row >= ph.rows) continue;
            float val[kMaxDecodeRanks];
            unsigned pending = (1u << a.nranks) - 1u;
            const uint64_t t0 = globaltimer_ns();
            for (unsigned spin = 0; pending; ++spin) {
                for (int q = 0; q < a.nranks; ++q) {
                    if (!(pending & (1u << q))) continue;
                    const uint64_t w = ld_word(own + static_cast<uint64_t>(q) * a.slot_words + row);
                    if (static_cast<uint32_t>(w >> 32) == epoch) {
                        val[q] = __uint_as_float(static_cast<uint32_t>(w));
                        pending &= ~(1u << q);
                    }
                }
                if (pending && (spin & 63u) == 63u &&
                    (aborted(p) || globaltimer_ns() - t0 > kPeerWaitNs)) {
                    atomicOr(a.peer_status, kStatusPeerTimeout);
                    set_abort(p, kStatusPeerTimeout);
                    break;
                }
            }
            if (pending) break;
            float sum = val[0];
            for (int q = 1; q < a.nranks; ++q) sum = __fadd_rn(sum, val[q]);
            a.res[row] = __fadd_rn(__ldcg(a.res + row), sum);
        }
    }
    if (ph.pick) {
        // this CTA's candidate: the best of its warpgroups' 64 row threads
        if (u < kMaxBatch * kTileRows) best[wg * kMaxBatch * kTileRows + u] = make_float2(best_v, __int_as_float(best_i));
        named_sync(1, kThreads);
        if (tid == 0) {
            float bv = __int_as_float(0x7fc00000);
            int bi = 0x7fffffff;
            for (int q = 0; q < NWG * kMaxBatch * kTileRows; ++q) {
                const float2 c = best[q];
                if (pick_better(c.x, __float_as_int(c.y), bv, bi)) {
                    bv = c.x;
                    bi = __float_as_int(c.y);
                }
            }
            a.cand[cta] = make_float2(bv, __int_as_float(bi));
        }
    }
}

// ------------------------------------------------------------------ attention

constexpr int kAttnColBytes = 256;  // V^T bytes per column per chunk (attn_core.cuh)
__host__ __device__ constexpr int mk_attn_kc(int d, int esz) { return 8192 / (d * esz); }  // K rows per stage: 8 KB

// attention_group (tp_llama.cpp:644-690) for KV head `kvh` = this CTA's
// index, over positions 0..P: attn_core, which states the order of every
// operation (the same code as the per-op kernel, attn.cu).
template <int NWG, int D, int ESZ>
__device__ void attn_phase(const MkParams &p, const TokenPhase &ph, const PhaseCtx &cx, uint8_t *smem, uint64_t *bars,
                           uint32_t &par) {
    const TokenArgs &a = p.a;
    const int kvh = blockIdx.x, G = a.group;
    const size_t head_bytes = static_cast<size_t>(a.kv_stride) * D * ESZ;
    if (!attn_core<D, ESZ, kAttnColBytes, mk_attn_kc(D, ESZ), NWG * 128>(
            ph.q + static_cast<size_t>(kvh) * G * D, static_cast<const uint8_t *>(ph.kcache) + kvh * head_bytes,
            static_cast<const uint8_t *>(ph.vcache) + kvh * head_bytes, a.kv_stride, cx.P + 1, G, a.scale,
            ph.out + static_cast<size_t>(kvh) * G * D, smem + p.off_attn, 1, bars, par, a.status, nullptr) &&
        threadIdx.x == 0)
        set_abort(p, kStatusStageTimeout);
}

template <int NWG>
__device__ void attn_dispatch(const MkParams &p, const TokenPhase &ph, const PhaseCtx &cx, uint8_t *smem, uint64_t *bars,
                              uint32_t &par) {
    if (p.a.head_dim == 64) {
        if (p.a.kv_f16)
            attn_phase<NWG, 64, 2>(p, ph, cx, smem, bars, par);
        else
            attn_phase<NWG, 64, 4>(p, ph, cx, smem, bars, par);
    } else {
        if (p.a.kv_f16)
            attn_phase<NWG, 128, 2>(p, ph, cx, smem, bars, par);
        else
            attn_phase<NWG, 128, 4>(p, ph, cx, smem, bars, par);
    }
}

// ------------------------------------------------------------------ kernel

template <int NWG>
__global__ void __launch_bounds__(NWG * 128 + 32, 1) token_kernel(const __grid_constant__ MkParams p) {
    constexpr int kThreads = NWG * 128;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[kMaxRing], empty[kMaxRing];
    __shared__ uint64_t abar[kAttnBars];  // attention's V^T and K stages
    __shared__ float s_f;
    __shared__ int s_exact, s_stop, s_tok;
    __shared__ int s_fail[4];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint8_t *ring = smem;
    const TokenArgs &a = p.a;
    const int tid = threadIdx.x, G = gridDim.x;
    if (tid == 0) {
        for (int i = 0; i < p.ring; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kAttnBars; ++i) mbar_init(&abar[i], 1);
        fence_mbar_init();
        s_stop = 0;
        s_fail[0] = s_fail[1] = s_fail[2] = s_fail[3] = 0;
    }
    __syncthreads();
    if (tid >= kThreads) {
        if (tid == kThreads) mk_producer(p, ring, full, empty);
        return;
    }
    const int pos0 = *reinterpret_cast<volatile int *>(a.pos);
    const uint32_t step0 = *reinterpret_cast<volatile unsigned *>(a.step);
    const int n_prompt = *a.n_prompt;
    uint32_t s = 0;
    uint32_t apar = 0;  // attention stage parities (attn_core)
    int cur_tok = 0;
    for (int t = 0; t < a.ntokens; ++t) {
        PhaseCtx cx;
        cx.P = pos0 + t;
        cx.step = step0 + static_cast<uint32_t>(t);
        cx.tok = (t == 0 || cx.P < n_prompt) ? __ldcg(a.tokens + cx.P) : cur_tok;
        const uint64_t base = static_cast<uint64_t>(cx.step) * a.nphases;  // barriers before this token
        for (int i = 0; i < a.nphases; ++i) {
            if (i > 0) {
                if (tid == 0 && !mk_grid_wait(p, (base + i) * G)) s_stop = 1;
                named_sync(1, kThreads);
                if (s_stop) return;
            }
            // by value: a reference into global memory would be re-read after
            // every global store the phase makes (the compiler cannot rule out
            // aliasing), inside the innermost loops
            const TokenPhase ph = a.phases[i];
            stamp(a, t, i, 0);
            if (ph.kind == kPhGemv)
                gemv_phase<NWG>(p, ph, cx, smem, ring, full, empty, s, &s_f, &s_exact, s_fail, t, i);
            else if (static_cast<int>(blockIdx.x) < a.kvh_local)
                attn_dispatch<NWG>(p, ph, cx, smem, abar, apar);
            named_sync(1, kThreads);
            stamp(a, t, i, 3);
            if (tid == 0) {
                __threadfence();
                red_release_gpu_add_u64(a.bar_count, 1ull);
                if (aborted(p) || s_fail[0] || s_fail[1] || s_fail[2] || s_fail[3]) s_stop = 1;
            }
            named_sync(1, kThreads);
            if (s_stop) return;
        }
        // every CTA: the pick over all CTAs' candidates, after the last barrier
        if (tid == 0 && !mk_grid_wait(p, (base + a.nphases) * G)) s_stop = 1;
        named_sync(1, kThreads);
        if (s_stop) return;
        if (tid < 32) {
            float bv = __int_as_float(0x7fc00000);
            int bi = 0x7fffffff;
            for (int c = tid; c < G; c += 32) {
                const float2 cd = __ldcg(a.cand + c);
                if (pick_better(cd.x, __float_as_int(cd.y), bv, bi)) {
                    bv = cd.x;
                    bi = __float_as_int(cd.y);
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_down_sync(kFullMask, bv, off);
                const int oi = __shfl_down_sync(kFullMask, bi, off);
                if (pick_better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (tid == 0) {
                const float y0 = __ldcg(a.logits);
                if (isnan(y0) || bi == 0x7fffffff) {  // the scan never leaves index 0 if y[0] is NaN
                    bv = y0;
                    bi = 0;
                }
                bi += a.vocab_base;
                if (a.nranks > 1) {
                    // every rank's pick through the windows' words n_embd and
                    // n_embd + 1; order (value desc, index asc), tp_llama.cpp:924
                    const uint32_t e = cx.step + 1u;
                    const uint64_t off = static_cast<uint64_t>(e & 1u) * kMaxDecodeRanks * a.slot_words;
                    if (blockIdx.x == 0)
                        for (int r = 0; r < a.nranks; ++r) {
                            uint64_t *w = a.win_words[r] + off + static_cast<uint64_t>(a.rank) * a.slot_words + a.n_embd;
                            st_word(w, (static_cast<uint64_t>(e) << 32) | static_cast<uint32_t>(bi));
                            st_word(w + 1, (static_cast<uint64_t>(e) << 32) | __float_as_uint(bv));
                        }
                    float gv = 0.0f;
                    int gi = 0;
                    for (int r = 0; r < a.nranks; ++r) {
                        const uint64_t *w = a.win_words[a.rank] + off + static_cast<uint64_t>(r) * a.slot_words + a.n_embd;
                        const uint64_t t0 = globaltimer_ns();
                        uint64_t wi = 0, wv = 0;
                        for (;;) {
                            wi = ld_word(w);
                            wv = ld_word(w + 1);
                            if (static_cast<uint32_t>(wi >> 32) == e && static_cast<uint32_t>(wv >> 32) == e) break;
                            if (globaltimer_ns() - t0 > kPeerWaitNs || aborted(p)) {
                                atomicOr(a.peer_status, kStatusPeerTimeout);
                                set_abort(p, kStatusPeerTimeout);
                                break;
                            }
                        }
                        const int ci = static_cast<int>(static_cast<uint32_t>(wi));
                        const float cv = __uint_as_float(static_cast<uint32_t>(wv));
                        if (r == 0 || cv > gv || (cv == gv && ci < gi)) {
                            gv = cv;
                            gi = ci;
                        }
                    }
                    bv = gv;
                    bi = gi;
                }
                s_tok = bi;
                if (aborted(p)) s_stop = 1;
                if (blockIdx.x == 0) {
                    // the loop's advance (tp_llama.cpp:951-959), for the host
                    const int nx = cx.P + 1;
                    if (nx >= n_prompt && nx <= a.ctx_max) {
                        a.tokens[nx] = bi;
                        if (a.host_tokens) a.host_tokens[nx] = bi;  // to the host as it is made
                    }
                    *a.pos = nx;
                    *a.step = cx.step + 1u;
                    a.pick_out[0] = bi;
                    a.pick_out[1] = __float_as_int(bv);
                }
            }
        }
        named_sync(1, kThreads);
        if (s_stop) return;
        cur_tok = s_tok;
    }
}

using TokenFn = void (*)(MkParams);

TokenFn pick_fn(int wgs) { return wgs == 2 ? token_kernel<2> : wgs == 3 ? token_kernel<3> : nullptr; }

int make_params(const TokenArgs &a, MkParams *out, int *smem_bytes, int *wgs_out) {
    if (!a.phases || a.nphases <= 0 || a.nphases > kMaxTokenPhases || a.ntokens <= 0) return kErrInval;
    if (a.head_dim != 64 && a.head_dim != 128) return kErrInval;
    const int wgs = a.group * a.head_dim > 256 ? 3 : 2;
    if (a.group * a.head_dim > wgs * 128) return kErrInval;
    if (a.n_embd / kQK > 2 * wgs * 128 / 4 * 2) return kErrInval;  // the RMSNorm staging: 2+ threads per block
    MkParams p{};
    p.a = a;
    int off = 0;
    auto carve = [&](int bytes) {
        const int at = off;
        off += (bytes + 127) / 128 * 128;
        return at;
    };
    const int kmax = 8192;
    // after the ring (placed first): x staging, the RMSNorm copy, reductions,
    // the pick, attention buffers and scores
    MkParams q = p;
    off = 0;
    q.off_xs = carve(xs_bytes(kmax));
    q.off_xf = carve(4 * a.n_embd);
    q.off_dred = carve(32 * 8);
    q.off_red = carve(wgs * 2 * kMaxBatch * 128 * 4);
    q.off_best = carve(wgs * kMaxBatch * kTileRows * 8);
    if (a.kv_stride < a.ctx_max || a.kv_stride % 8) return kErrInval;
    const int esz = a.kv_f16 ? 2 : 4;
    q.off_attn = carve(attn_core_smem_bytes(a.head_dim, esz, kAttnColBytes, mk_attn_kc(a.head_dim, esz), wgs * 128,
                                            a.kv_stride));
    const int fixed = off;
    const int limit = max_smem_optin() - 128 - 1024;  // alignment slack and static shared memory
    int ring = (limit - fixed) / kStage;
    if (ring > kMaxRing) ring = kMaxRing;
    if (ring < 4) return kErrInval;  // a K = 8192 row group needs 4 stages
    const int ring_bytes = ring * kStage;
    q.ring = ring;
    q.off_xs += ring_bytes;
    q.off_xf += ring_bytes;
    q.off_dred += ring_bytes;
    q.off_red += ring_bytes;
    q.off_best += ring_bytes;
    q.off_attn += ring_bytes;
    *out = q;
    *smem_bytes = 128 + ring_bytes + fixed;
    *wgs_out = wgs;
    return 0;
}

}  // namespace

int token_kernel_plan(const TokenArgs &a, int *smem_bytes, int *ring_stages, int *wgs, int *grid) {
    MkParams p;
    int smem = 0, w = 0;
    if (int rc = make_params(a, &p, &smem, &w)) return rc;
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    if (smem_bytes) *smem_bytes = smem;
    if (ring_stages) *ring_stages = p.ring;
    if (wgs) *wgs = w;
    if (grid) *grid = sms;
    return 0;
}

int token_kernel_launch(const TokenArgs &a, cudaStream_t stream) {
    MkParams p;
    int smem = 0, wgs = 0;
    if (int rc = make_params(a, &p, &smem, &wgs)) return rc;
    TokenFn fn = pick_fn(wgs);
    if (!fn) return kErrInval;
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    if (!ensure_smem(reinterpret_cast<const void *>(fn), smem)) return kErrCuda;
    const int threads = wgs * 128 + 32;
    if (resident_ctas(reinterpret_cast<const void *>(fn), threads, smem) < 1) return kErrInval;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(sms);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, p) == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
