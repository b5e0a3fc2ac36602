// Q4_0 x Q8_0 GEMV over the B200 tile layout: the engine path's kernel.
// Bit-exact to src/llm_kv260/q4_0.py:151-182, like the GGUF-layout kernel in
// q4gemv.cu; only where the bytes sit differs.
//
// Tile layout. The reference re-lays every matrix at load for its engine
// (board/tp/tp_llama.cpp:102-118, the gemv2 chunk interleave); this engine
// does the same for HBM. Rows are padded to a multiple of 16. For row group
// g (rows 16g..16g+15) and chunk c (blocks 8c..8c+7) a 2304-byte tile sits at
// byte ((g * nch) + c) * 2304:
//     [0, 2048)     nibbles: 16 bytes for row i, lane l at (i * 8 + l) * 16
//     [2048, 2304)  scales:  float16 bits for row i, lane l at 2048 + (i * 8 + l) * 2
// The 16 nibble bytes of a block are copied unchanged (byte j: weight j in
// the low nibble, weight j+16 in the high one), so the bytes per weight stay
// 18/32 and the algorithmic traffic is the GGUF file's.
//
// Kernel. One producer warp streams whole row groups (one group's tile run =
// one 1-D bulk copy, TMA engine, no multicast) into a ring of shared-memory
// stages, issued before the kernel waits on its predecessor (programmatic
// dependent launch). Two consumer warp-quads take every other group; in a
// quad, warp w owns rows 4w..4w+3 and thread (row i, lane l) runs lane l's
// chain of row i over all chunks in order (q4_0.py:177-179) -- its x blocks
// in registers when K <= 2048. A warp reads its 4 rows' 512 contiguous bytes
// per chunk (conflict-free), meets the 8 lane sums with xor shuffles 1, 2, 4
// -- tree_sum's pairing (q4_0.py:67-78), IEEE addition being commutative --
// and frees its stage with one mbarrier arrival: no CTA-wide barrier per
// stage, so the quads and the producer run independently.
#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"

namespace b200 {

namespace {

constexpr int kQuadThreads = kTileRows * kLanes;  // one 16-row group: 4 warps, 128 threads
constexpr int kQuads = 2;                          // groups in flight per CTA
constexpr int kConsumers = kQuads * kQuadThreads;  // 256
constexpr int kTileThreads = kConsumers + 32;      // + the producer warp
constexpr int kTileNibBytes = kQuadThreads * 16;   // 2048
constexpr int kMaxStages = 8;
constexpr int kSmemAlign = 128;
constexpr int kXregChunks = 8;                     // K <= 2048: x blocks in registers
constexpr int kSelMaxCtas = 4096;                  // fused greedy pick: candidate slots

struct TileParams {
    const uint8_t *w;
    float *y;
    const void *x;
    unsigned *status;
    int rows, k, nb, nch;
    int groups;
    int unit;        // row groups are split over CTAs in whole units of this many groups
    int act_off;     // kEpiSiluPairs with act_q8: byte offset of the CTA's act values after xs
    int slot_bytes;  // nch * 2304: one row group
    int stages;
    int round_mode;
    int l2_policy;
    // Optional greedy pick over y, fused (tp_llama.cpp:879-882): when sel_out
    // is set, every CTA posts its best (value, row) to sel_cand[blockIdx.x],
    // and the last CTA to finish reduces them into sel_out (int32 index +
    // sel_base, then float32 value) and resets the ticket to 0.
    int *sel_out;
    int sel_base;
    float2 *sel_cand;    // gridDim.x entries: (value, row as float bits)
    unsigned *sel_ticket;
    DecodeOps dec;       // decoder prologue / epilogue (q4gemv.h)
    uint64_t *trace;     // optional launch trace (q4gemv.h, kTraceCtas)
};

__device__ __forceinline__ void trace_stamp(uint64_t *trace, int j) {
    if (trace && threadIdx.x == 0 && blockIdx.x < kTraceCtas) trace[blockIdx.x * kTraceStamps + j] = globaltimer_ns();
}

constexpr uint64_t kPeerTimeoutNs = 1000000000ull;  // a peer's row words: 1 s

__device__ __forceinline__ void st_word(uint64_t *p, uint64_t w) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// RMSNorm's sequential fallback (tp_llama.cpp:560-564): lane j sums x[i]^2
// for i = j, j+4, ... in order, threads 0-3, then (l0 + l2) + (l1 + l3);
// returns (float)(ss / k). Out of line: rarely taken, and the hot code stays
// small (each launch fetches its instructions anew).
__device__ __noinline__ float rms_sequential(const float *xf, double *dred, int k) {
    const int t = threadIdx.x;
    if (t < 4) {
        double a = 0.0;
        for (int i = t; i < k; i += 4) a = __dadd_rn(a, __dmul_rn(static_cast<double>(xf[i]), static_cast<double>(xf[i])));
        dred[8 + t] = a;
    }
    named_sync(1, kConsumers);
    const double ss2 = __dadd_rn(__dadd_rn(dred[8], dred[10]), __dadd_rn(dred[9], dred[11]));
    return __double2float_rn(__ddiv_rn(ss2, static_cast<double>(k)));
}

// Consumer side of staging a float32 x into xs (int8[k], then (float32 d,
// int32 sum) per block -- stage_x's layout), TPB threads per 32-block with
// E = 32 / TPB consecutive values each. The prologue's x is the plain input,
// or rmsnorm(res) * norm_w (tp_llama.cpp:557-569), or that of the token's
// embedding row (593-604), which CTA 0 also writes to res. The norm weights
// do not depend on the previous kernel, so they load before this waits for
// it. The sum of squares runs in parallel in double (each square is exact)
// and every thread combines the warp sums in the same order, so all take
// the same decision: rms_float_is_safe, else threads 0-3 redo the
// reference's four sequential lane sums from the copy of x in xf. The
// block's Q8_0 quantisation (q4_0.py:83-97) meets its maximum and its int
// sum across the block's TPB adjacent lanes by xor shuffles: the maximum
// (fmaxf) and an integer sum do not depend on the order.
template <int TPB, int PRO, typename AfterWait>
__device__ __forceinline__ void stage_x_f32(const TileParams &p, uint8_t *xs, float *xf, double *dred,
                                            AfterWait &&after_wait) {
    constexpr int E = 32 / TPB;
    const int k = p.k, nb = k / kQK, t = threadIdx.x, b = t / TPB, r = t % TPB, lane = t % 32, warp = t / 32;
    const bool live = b < nb;
    const int i0 = 32 * b + E * r;
    constexpr int pro = PRO;
    float w[E];
    if (pro != kProPlain && live) {
        const float4 *wv = reinterpret_cast<const float4 *>(p.dec.norm_w + i0);
#pragma unroll
        for (int j = 0; j < E / 4; ++j) {
            const float4 f = __ldg(wv + j);
            w[4 * j] = f.x;
            w[4 * j + 1] = f.y;
            w[4 * j + 2] = f.z;
            w[4 * j + 3] = f.w;
        }
    }
    pdl_wait_prior_grid();
    trace_stamp(p.trace, 1);
    after_wait();
    float v[E];
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = 0.0f;
    if (live) {
        if (pro == kProEmbedNorm) {
            const int at = *p.dec.pos, given = p.dec.in_token ? *p.dec.in_token : -1;
            const int tok = given >= 0 ? given : p.dec.tokens[at];
            if (given >= 0 && blockIdx.x == 0 && threadIdx.x == 0) const_cast<int *>(p.dec.tokens)[at] = given;
            const uint8_t *blk = p.dec.embd + (static_cast<size_t>(tok) * nb + b) * kBlockBytes;
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(blk)));
#pragma unroll
            for (int j = 0; j < E; ++j) {
                const int i = E * r + j;  // weight i of the block: low nibble of byte i, or high of byte i - 16
                const int byte = blk[2 + (i & 15)];
                const int nib = i < 16 ? (byte & 0xF) : (byte >> 4);
                v[j] = __fmul_rn(__int2float_rn(nib - 8), d);
            }
            if (blockIdx.x == 0) {
                float4 *dst = reinterpret_cast<float4 *>(p.dec.res + i0);
#pragma unroll
                for (int j = 0; j < E / 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        } else {
            const float4 *src = reinterpret_cast<const float4 *>((pro == kProPlain ? static_cast<const float *>(p.x) : p.dec.res) + i0);
#pragma unroll
            for (int j = 0; j < E / 4; ++j) {
                const float4 f = __ldcg(src + j);
                v[4 * j] = f.x;
                v[4 * j + 1] = f.y;
                v[4 * j + 2] = f.z;
                v[4 * j + 3] = f.w;
            }
        }
    }
    if (pro != kProPlain) {
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < E; ++j) ss = __dadd_rn(ss, __dmul_rn(static_cast<double>(v[j]), static_cast<double>(v[j])));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(kFullMask, ss, off));
        if (lane == 0) dred[warp] = ss;
        trace_stamp(p.trace, 6);
        if (live) {
            float4 *xd = reinterpret_cast<float4 *>(xf + i0);
#pragma unroll
            for (int j = 0; j < E / 4; ++j) xd[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        named_sync(1, kConsumers);
        double tot = 0.0;
#pragma unroll
        for (int w8 = 0; w8 < kConsumers / 32; ++w8) tot = __dadd_rn(tot, dred[w8]);
        const double q = __ddiv_rn(tot, static_cast<double>(k));
        float f = __double2float_rn(q);
        if (p.dec.exact_norm || !rms_float_is_safe(q, f, k)) f = rms_sequential(xf, dred, k);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, p.dec.eps)));
        trace_stamp(p.trace, 7);
#pragma unroll
        for (int j = 0; j < E; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), w[j]);
    }
    // Q8_0 of the block (q8_quant_block's arithmetic, split over TPB lanes)
    float am = fabsf(v[0]);
#pragma unroll
    for (int j = 1; j < E; ++j) am = fmaxf(am, fabsf(v[j]));
#pragma unroll
    for (int off = 1; off < TPB; off <<= 1) am = fmaxf(am, __shfl_xor_sync(kFullMask, am, off));
    const float db = __fdiv_rn(am, 127.0f);
    const float inv = db == 0.0f ? 0.0f : __fdiv_rn(1.0f, db);
    uint32_t qw[E / 4];
    int sum = 0;
#pragma unroll
    for (int j = 0; j < E / 4; ++j) {
        const int q0 = q8_round(__fmul_rn(v[4 * j], inv), p.round_mode);
        const int q1 = q8_round(__fmul_rn(v[4 * j + 1], inv), p.round_mode);
        const int q2 = q8_round(__fmul_rn(v[4 * j + 2], inv), p.round_mode);
        const int q3 = q8_round(__fmul_rn(v[4 * j + 3], inv), p.round_mode);
        sum += q0 + q1 + q2 + q3;
        qw[j] = (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
                ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
    }
#pragma unroll
    for (int off = 1; off < TPB; off <<= 1) sum += __shfl_xor_sync(kFullMask, sum, off);
    if (live) {
        if constexpr (E == 8) {
            *reinterpret_cast<uint2 *>(xs_block(xs, b) + E * r) = make_uint2(qw[0], qw[1]);
        } else {
#pragma unroll
            for (int j = 0; j < E / 16; ++j)
                reinterpret_cast<uint4 *>(xs_block(xs, b) + E * r)[j] =
                    make_uint4(qw[4 * j], qw[4 * j + 1], qw[4 * j + 2], qw[4 * j + 3]);
        }
        if (r == 0) xs_scales(xs, k)[b] = make_int2(__float_as_int(__half2float(__float2half_rn(db))), sum);
    }
}

// Byte offset of the decoder's x copy (xf) after the staged x, and its size.
__host__ __device__ constexpr int xarea_bytes(int k) { return (xs_bytes(k) + 15) / 16 * 16; }
constexpr int norm_extra_bytes(int k) { return 4 * k + 32 * 8; }  // xf [k] floats + 32 doubles

// (value desc, index asc); NaN never beats a number (the scan's rule for any
// index but 0, which the final step handles).
__device__ __forceinline__ bool sel_better(float av, int ai, float bv, int bi) {
    if (isnan(bv)) return !isnan(av) || ai < bi;
    if (isnan(av)) return false;
    return av > bv || (av == bv && ai < bi);
}

// Q8_0 of a CTA's act values (its row groups [g0, g1) give act values
// [8 g0, 8 g1): whole 32-value blocks) into the packed x at p.dec.act_q8:
// int8 at byte 32 b, then the float16-rounded scale as float32 at K + 4 b
// (K = rows / 2) -- the engine's buffer (q4_0.py:193-200), which the next
// GEMV stages with the packed path. One warp per block, one value per lane;
// the block maximum meets by xor shuffles (fmaxf does not depend on the
// order); the rest is q8_quant_block's arithmetic (q4_0.py:83-97). Called
// by every consumer warp; `ok` must be uniform within each warp.
__device__ __forceinline__ void quantize_act_blocks(const TileParams &p, const float *vals, int g0, int g1, bool ok) {
    const int K = p.rows / 2, lane = threadIdx.x & 31;
    const int b0 = g0 * (kTileRows / 2) / kQK, nblk = (g1 - g0) * (kTileRows / 2) / kQK;
    if (!ok) return;
    for (int bl = threadIdx.x >> 5; bl < nblk; bl += kConsumers / 32) {
        const float v = vals[bl * kQK + lane];
        float am = fabsf(v);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(kFullMask, am, off));
        const float db = __fdiv_rn(am, 127.0f);
        const float inv = db == 0.0f ? 0.0f : __fdiv_rn(1.0f, db);
        p.dec.act_q8[kQK * (b0 + bl) + lane] = static_cast<uint8_t>(q8_round(__fmul_rn(v, inv), p.round_mode) & 0xff);
        if (lane == 0) reinterpret_cast<float *>(p.dec.act_q8 + K)[b0 + bl] = __half2float(__float2half_rn(db));
    }
}

// Block term of one chunk-tile for row i, lane l.
__device__ __forceinline__ float tile_term(const uint8_t *tile, int i, int l, const XBlock &xb) {
    const int u = i * kLanes + l;
    const uint4 nv = *reinterpret_cast<const uint4 *>(tile + u * 16);
    const uint32_t db = *reinterpret_cast<const uint16_t *>(tile + kTileNibBytes + u * 2);
    const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
    return block_term_words(n, db, xb);
}

// Bounded ring wait: gives up when another thread of the CTA gave up, or
// after kStageTimeoutNs (then marks the status and the CTA's abort flag).
__device__ __forceinline__ bool ring_wait(uint64_t *bar, uint32_t parity, unsigned *status, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (unsigned spin = 0;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 255u) == 255u) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > kStageTimeoutNs) {
                atomicOr(status, kStatusStageTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// XREG: K <= 2048, each thread's 8 x blocks stay in registers.
// One instantiation per (x mode, x in registers, prologue, epilogue, fused
// pick) that a caller uses (pick_tile): each launch runs a compact,
// contiguous code path -- a kernel holding every variant is several times
// larger than an SM's instruction cache keeps across the token's launches.
// Registers per thread. The o GEMV (float32 x, plain prologue, residual
// epilogue) stays within what an attention CTA leaves free on its SM (the SM
// has 65536 registers), so its CTAs start beside the attention's; the down
// GEMV (packed x, residual epilogue) runs at 96, which measured faster than
// its uncapped 106.
template <int XMODE, int PRO, int EPI>
struct TileRegs {
    static constexpr int value = (XMODE == kXF32 && PRO == kProPlain && EPI == kEpiResidual)     ? 136
                                 : (XMODE == kXPacked && PRO == kProPlain && EPI == kEpiResidual) ? 96
                                                                                                  : 224;
};

template <int XMODE, bool XREG, int PRO, int EPI, bool PICK>
__global__ void __maxnreg__((TileRegs<XMODE, PRO, EPI>::value)) q4_tile_kernel(const __grid_constant__ TileParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ int s_abort;
    __shared__ unsigned s_last;
    __shared__ float2 s_best[kConsumers / kLanes];
    uint8_t *ring = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + kSmemAlign - 1) & ~static_cast<uintptr_t>(kSmemAlign - 1));
    uint8_t *xs = ring + p.stages * p.slot_bytes;

    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const int units = (p.groups + p.unit - 1) / p.unit;
    const int g0 = min(p.groups, p.unit * static_cast<int>(static_cast<long long>(units) * blockIdx.x / gridDim.x));
    const int g1 = min(p.groups, p.unit * static_cast<int>(static_cast<long long>(units) * (blockIdx.x + 1) / gridDim.x));
    const int S = p.stages, nst = g1 - g0;

    if (t == 0) {
        s_abort = 0;
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kQuadThreads / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    trace_stamp(p.trace, 0);

    if (warp == kConsumers / 32) {
        // producer: the weights do not depend on the previous kernel
        if (lane == 0) {
            const uint64_t policy = make_policy(p.l2_policy);
            int s = 0;
            for (; s < nst; ++s) {
                const int slot = s % S;
                const uint32_t use = static_cast<uint32_t>(s / S);
                if (use > 0 && !ring_wait(&empty[slot], (use & 1u) ^ 1u, p.status, &s_abort)) break;
                mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(p.slot_bytes));
                bulk_g2s(ring + static_cast<size_t>(slot) * p.slot_bytes,
                         p.w + static_cast<size_t>(g0 + s) * p.slot_bytes, static_cast<uint32_t>(p.slot_bytes),
                         &full[slot], policy);
            }
            // leave only after this CTA's copies have landed (at once when the
            // consumers took them all; after an abort, each wait bounded)
            for (int r = s > S ? s - S : 0; r < s; ++r) {
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&full[r % S], static_cast<uint32_t>((r / S) & 1)))
                    if (globaltimer_ns() - t0 > kStageTimeoutNs) break;
            }
        }
        return;
    }

    const int quad = warp / 4, i = (warp % 4) * 4 + (lane >> 3), l = lane & 7;
    constexpr int epi = EPI;
    const bool xchg = epi == kEpiResidual && p.dec.nranks > 1;
    const int row0 = (g0 + quad) * kTileRows + i;
    int dpos = 0;
    uint32_t epoch = 0;
    uint64_t slot_off = 0;
    float pre_res = 0.0f, pre_c = 0.0f, pre_s = 0.0f;
    // The epilogue's global inputs -- the position, the exchange epoch, this
    // thread's first residual value or RoPE pair -- are fetched as soon as
    // the previous kernel's results are visible, so their latency (a
    // dependent pair of loads for RoPE) hides behind the x staging.
    auto after_wait = [&]() {
        if constexpr (EPI == kEpiRopeKv) {
            dpos = *p.dec.pos;
            if (l == 0 && quad < nst && row0 < p.dec.q_rows + p.dec.kv_rows) {
                const int hd = p.dec.head_dim, j = (row0 % hd) >> 1;
                const float *cs = p.dec.rope_cs + static_cast<size_t>(dpos) * hd;
                pre_c = __ldg(cs + 2 * j);
                pre_s = __ldg(cs + 2 * j + 1);
            }
        }
        if constexpr (EPI == kEpiResidual) {
            if (xchg) {
                epoch = *p.dec.step * static_cast<uint32_t>(p.dec.ar_per_token) + static_cast<uint32_t>(p.dec.ar_index) + 1u;
                slot_off = static_cast<uint64_t>(epoch & 1u) * kMaxDecodeRanks * p.dec.slot_words;
            } else if (l == 0 && quad < nst && row0 < p.rows) {
                pre_res = __ldcg(p.dec.res + row0);
            }
        }
    };
    if constexpr (XMODE == kXF32) {
        float *xf = reinterpret_cast<float *>(xs + xarea_bytes(p.k));    // with a norm prologue only
        double *dred = reinterpret_cast<double *>(xs + xarea_bytes(p.k) + 4 * p.k);
        // K <= 2048 (XREG) always stages with 4 threads per block; only the
        // variants a kernel can reach are compiled into it
        if constexpr (XREG) {
            stage_x_f32<4, PRO>(p, xs, xf, dred, after_wait);
        } else {
            if (p.nb * 2 <= kConsumers)
                stage_x_f32<2, PRO>(p, xs, xf, dred, after_wait);
            else
                stage_x_f32<1, PRO>(p, xs, xf, dred, after_wait);
        }
    } else {
        pdl_wait_prior_grid();
        trace_stamp(p.trace, 1);
        after_wait();
        stage_x<XMODE>(p.x, p.k, p.round_mode, xs);
    }
    named_sync(1, kConsumers);
    trace_stamp(p.trace, 2);
    XBlock xr[XREG ? kXregChunks : 1];
    if constexpr (XREG) {
#pragma unroll
        for (int c = 0; c < kXregChunks; ++c)
            if (c < p.nch) load_xblock_smem(xs, p.k, 8 * c + l, xr[c]);
    }
    float best_v = __int_as_float(0x7fc00000);  // NaN: loses to any number
    int best_i = 0x7fffffff;
    bool ok = true;
    for (int s = quad; s < nst; s += kQuads) {
        const int slot = s % S;
        if (!ring_wait(&full[slot], static_cast<uint32_t>((s / S) & 1), p.status, &s_abort)) {
            ok = false;
            break;
        }
        if (s == quad) trace_stamp(p.trace, 4);
        const uint8_t *tiles = ring + static_cast<size_t>(slot) * p.slot_bytes;
        float acc = 0.0f;
        if constexpr (XREG) {
            // four chunks' tile words loaded together, then their terms in
            // chunk order (the lane chain's order)
            const int u = i * kLanes + l;
#pragma unroll
            for (int c0 = 0; c0 < kXregChunks; c0 += 4) {
                uint4 nv[4];
                uint32_t dv[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c0 + c < p.nch) {
                        const uint8_t *tile = tiles + (c0 + c) * kTileBytes;
                        nv[c] = *reinterpret_cast<const uint4 *>(tile + u * 16);
                        dv[c] = *reinterpret_cast<const uint16_t *>(tile + kTileNibBytes + u * 2);
                    }
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c0 + c < p.nch) {
                        const uint32_t n[4] = {nv[c].x, nv[c].y, nv[c].z, nv[c].w};
                        acc = __fadd_rn(acc, block_term_words(n, dv[c], xr[c0 + c]));
                    }
                }
            }
        } else {
#pragma unroll 4
            for (int c = 0; c < p.nch; ++c) {
                XBlock xb;
                load_xblock_smem(xs, p.k, 8 * c + l, xb);
                acc = __fadd_rn(acc, tile_term(tiles + c * kTileBytes, i, l, xb));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        // tree_sum (q4_0.py:67-78): ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7))
        acc = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, 1));
        acc = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, 2));
        const float yv = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, 4));
        const int row = (g0 + s) * kTileRows + i;
        const bool live = row < p.rows && l == 0;
        if (epi == kEpiStore) {
            if (live) {
                p.y[row] = yv;
                if (PICK && sel_better(yv, row, best_v, best_i)) {
                    best_v = yv;
                    best_i = row;
                }
            }
        } else if (epi == kEpiRopeKv) {
            // q and k rows start at multiples of head_dim (even): rope's pair
            // (2j, 2j+1) is rows i and i ^ 1, lanes 8 apart
            const float other = __shfl_xor_sync(kFullMask, yv, 8);
            if (live) {
                const int hd = p.dec.head_dim, k0 = p.dec.q_rows, v0 = k0 + p.dec.kv_rows;
                float out = yv;
                if (row < v0) {
                    const int j = (row % hd) >> 1;
                    const float *cs = p.dec.rope_cs + static_cast<size_t>(dpos) * hd;
                    const bool even = !(row & 1);
                    const float c = s == quad ? pre_c : cs[2 * j], sn = s == quad ? pre_s : cs[2 * j + 1];
                    out = rope_pair(even ? yv : other, even ? other : yv, c, sn, even);
                }
                p.y[row] = out;
                if (row >= k0) {
                    // K rows [kv head][stride][hd], lane-major and swizzled by
                    // position (k_slot); V transposed, [kv head][hd][stride]
                    const bool isk = row < v0;
                    const int rr = row - (isk ? k0 : v0), st = p.dec.kv_stride;
                    const size_t at =
                        isk ? (static_cast<size_t>(rr / hd) * st + dpos) * hd + k_slot(rr % hd, dpos, p.dec.kv_f16 ? 2 : 4, hd)
                            : static_cast<size_t>(rr) * st + dpos;
                    void *cache = isk ? p.dec.kcache : p.dec.vcache;
                    if (p.dec.kv_f16)
                        static_cast<__half *>(cache)[at] = __float2half_rn(out);
                    else
                        static_cast<float *>(cache)[at] = out;
                }
            }
        } else if (epi == kEpiSiluPairs) {
            const float other = __shfl_xor_sync(kFullMask, yv, 8);
            if (live) {
                if (p.y) p.y[row] = yv;
                if (!(row & 1)) {
                    const float a = silu_mul(yv, other);
                    p.dec.act[row >> 1] = a;
                    if (p.dec.act_q8) reinterpret_cast<float *>(xs + p.act_off)[(row >> 1) - g0 * (kTileRows / 2)] = a;
                }
            }
        } else if (live) {  // kEpiResidual
            if (p.y) p.y[row] = yv;
            if (!xchg) {
                p.dec.res[row] = __fadd_rn(s == quad ? pre_res : p.dec.res[row], yv);
            } else {
                const uint64_t word = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(yv);
                const uint64_t at = slot_off + static_cast<uint64_t>(p.dec.rank) * p.dec.slot_words + row;
                for (int r = 0; r < p.dec.nranks; ++r) st_word(p.dec.win_words[r] + at, word);
            }
        }
    }
    trace_stamp(p.trace, 5);
    if constexpr (EPI == kEpiSiluPairs) {
        if (p.dec.act_q8) {
            // this CTA's act values as whole Q8_0 blocks of the next GEMV's
            // packed x (q4_0.py:83-97, 193-200)
            named_sync(1, kConsumers);
            quantize_act_blocks(p, reinterpret_cast<const float *>(xs + p.act_off), g0, g1, __all_sync(kFullMask, ok));
        }
    }
    if (xchg && ok && l == 0) {
        // Every rank computed these rows' partials for its K slice; collect
        // them from this rank's window and sum in rank order
        // (tp_llama.cpp:515-521), then add into the residual (add_into).
        const uint64_t *own = p.dec.win_words[p.dec.rank] + slot_off;
        for (int s = quad; s < nst; s += kQuads) {
            const int row = (g0 + s) * kTileRows + i;
            if (row >= p.rows) continue;
            float val[kMaxDecodeRanks];
            unsigned pending = (1u << p.dec.nranks) - 1u;
            const uint64_t t0 = globaltimer_ns();
            for (unsigned spins = 0; pending; ++spins) {
                for (int r = 0; r < p.dec.nranks; ++r) {
                    if (!(pending & (1u << r))) continue;
                    const uint64_t w = ld_word(own + static_cast<uint64_t>(r) * p.dec.slot_words + row);
                    if (static_cast<uint32_t>(w >> 32) == epoch) {
                        val[r] = __uint_as_float(static_cast<uint32_t>(w));
                        pending &= ~(1u << r);
                    }
                }
                if (pending && (spins & 63u) == 63u && globaltimer_ns() - t0 > kPeerTimeoutNs) {
                    atomicOr(p.dec.peer_status, kStatusPeerTimeout);
                    break;
                }
            }
            if (pending) break;
            float sum = val[0];
            for (int r = 1; r < p.dec.nranks; ++r) sum = __fadd_rn(sum, val[r]);
            p.dec.res[row] = __fadd_rn(p.dec.res[row], sum);
        }
    }
    if constexpr (PICK) {
        // CTA best over the row threads (l == 0), then the last CTA to finish
        // reduces all CTAs' bests
        if (l == 0) s_best[t / kLanes] = make_float2(best_v, __int_as_float(best_i));
        named_sync(1, kConsumers);
        if (t < 32) {
            float bv = __int_as_float(0x7fc00000);
            int bi = 0x7fffffff;
            for (int c = t; c < kConsumers / kLanes; c += 32) {
                const float2 cd = s_best[c];
                if (sel_better(cd.x, __float_as_int(cd.y), bv, bi)) {
                    bv = cd.x;
                    bi = __float_as_int(cd.y);
                }
            }
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_down_sync(kFullMask, bv, off);
                const int oi = __shfl_down_sync(kFullMask, bi, off);
                if (sel_better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (t == 0) {
                p.sel_cand[blockIdx.x] = make_float2(bv, __int_as_float(bi));
                __threadfence();
                s_last = atomicAdd(p.sel_ticket, 1u) == gridDim.x - 1;
            }
        }
        named_sync(1, kConsumers);
        if (s_last && t < 32) {
            __threadfence();
            // the status words for the advance's record, loaded here so their
            // latency passes under the candidates' reduction
            unsigned st0 = 0u, st1 = 0u;
            if (t == 0 && p.dec.adv_status) {
                st0 = *reinterpret_cast<volatile unsigned *>(p.status);
                if (p.dec.peer_status) st1 = *reinterpret_cast<volatile unsigned *>(p.dec.peer_status);
            }
            float bv = __int_as_float(0x7fc00000);
            int bi = 0x7fffffff;
            for (int c = t; c < static_cast<int>(gridDim.x); c += 32) {
                const float2 cd = __ldcg(&p.sel_cand[c]);
                if (sel_better(cd.x, __float_as_int(cd.y), bv, bi)) {
                    bv = cd.x;
                    bi = __float_as_int(cd.y);
                }
            }
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_down_sync(kFullMask, bv, off);
                const int oi = __shfl_down_sync(kFullMask, bi, off);
                if (sel_better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (t == 0) {
                const float y0 = __ldcg(p.y);
                if (isnan(y0) || bi == 0x7fffffff) {  // the scan never leaves index 0 if y[0] is NaN
                    bv = y0;
                    bi = 0;
                }
                p.sel_out[0] = bi + p.sel_base;
                p.sel_out[1] = __float_as_int(bv);
                *p.sel_ticket = 0;
                if (p.dec.adv_pos) {
                    // the decode loop's step (tp_llama.cpp:951-959): the pick is
                    // the next position's token unless the prompt supplies it
                    const int nx = *p.dec.adv_pos + 1;
                    if (nx >= *p.dec.n_prompt && nx <= p.dec.ctx_max) p.dec.adv_tokens[nx] = bi + p.sel_base;
                    *p.dec.adv_pos = nx;
                    *p.dec.adv_step += 1u;
                    if (p.dec.adv_in_token) *p.dec.adv_in_token = -1;
                    if (p.dec.adv_status) {
                        p.dec.adv_status[0] = st0;
                        p.dec.adv_status[1] = st1;
                    }
                }
            }
        }
    }
    if (p.trace) {
        named_sync(1, kConsumers);
        trace_stamp(p.trace, 3);
    }
}

// GGUF rows -> tiles; one thread per (row, block), padded rows become zeros.
__global__ void repack_tiles_kernel(const uint8_t *__restrict__ src, int rows, int k, uint8_t *__restrict__ dst) {
    const int nb = k / kQK, nch = nb / kLanes;
    const long long total = static_cast<long long>((rows + kTileRows - 1) / kTileRows) * kTileRows * nb;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(idx / nb), b = static_cast<int>(idx % nb);
        uint16_t h[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
        if (r < rows) {
            const uint16_t *blk = reinterpret_cast<const uint16_t *>(src + (static_cast<size_t>(r) * nb + b) * kBlockBytes);
#pragma unroll
            for (int j = 0; j < 9; ++j) h[j] = blk[j];
        }
        const int g = r / kTileRows, i = r % kTileRows, c = b / kLanes, l = b % kLanes;
        uint8_t *tile = dst + (static_cast<size_t>(g) * nch + c) * kTileBytes;
        uint4 nv;
        nv.x = h[1] | (static_cast<uint32_t>(h[2]) << 16);
        nv.y = h[3] | (static_cast<uint32_t>(h[4]) << 16);
        nv.z = h[5] | (static_cast<uint32_t>(h[6]) << 16);
        nv.w = h[7] | (static_cast<uint32_t>(h[8]) << 16);
        *reinterpret_cast<uint4 *>(tile + (i * kLanes + l) * 16) = nv;
        *reinterpret_cast<uint16_t *>(tile + kTileNibBytes + (i * kLanes + l) * 2) = h[0];
    }
}

using TileKernelFn = void (*)(TileParams);

template <int XMODE, int PRO, int EPI, bool PICK>
TileKernelFn tile_fn(bool xreg) {
    return xreg ? q4_tile_kernel<XMODE, true, PRO, EPI, PICK> : q4_tile_kernel<XMODE, false, PRO, EPI, PICK>;
}

// The instantiations callers use: the engine's plain GEMV (with or without
// the fused pick) for both x modes, and the decoder's five launch kinds.
// Any other combination is refused.
TileKernelFn pick_tile(int xmode, bool xreg, int pro, int epi, bool pick) {
    if (pro == kProPlain && epi == kEpiStore) {
        if (xmode == kXPacked) return pick ? tile_fn<kXPacked, kProPlain, kEpiStore, true>(xreg)
                                           : tile_fn<kXPacked, kProPlain, kEpiStore, false>(xreg);
        return pick ? tile_fn<kXF32, kProPlain, kEpiStore, true>(xreg) : tile_fn<kXF32, kProPlain, kEpiStore, false>(xreg);
    }
    if (xmode == kXPacked && pro == kProPlain && epi == kEpiResidual && !pick)
        return tile_fn<kXPacked, kProPlain, kEpiResidual, false>(xreg);
    if (xmode != kXF32) return nullptr;
    if (pro == kProEmbedNorm && epi == kEpiRopeKv && !pick) return tile_fn<kXF32, kProEmbedNorm, kEpiRopeKv, false>(xreg);
    if (pro == kProRmsnorm && epi == kEpiRopeKv && !pick) return tile_fn<kXF32, kProRmsnorm, kEpiRopeKv, false>(xreg);
    if (pro == kProPlain && epi == kEpiResidual && !pick) return tile_fn<kXF32, kProPlain, kEpiResidual, false>(xreg);
    if (pro == kProRmsnorm && epi == kEpiSiluPairs && !pick) return tile_fn<kXF32, kProRmsnorm, kEpiSiluPairs, false>(xreg);
    if (pro == kProRmsnorm && epi == kEpiStore && pick) return tile_fn<kXF32, kProRmsnorm, kEpiStore, true>(xreg);
    return nullptr;
}

struct TilePlan {
    TileParams p;
    TileKernelFn fn;
    int grid;
    int smem;
    int threads;
};

int make_tile_plan(const TileLaunch &L, const Tuning &tu, TilePlan *out) {
    const char *why = nullptr;
    if (int rc = tile_validate(L, &why)) return rc;
    const int nb = L.k / kQK, nch = nb / kLanes;
    if (nb > kConsumers) return kErrInval;  // x staging: one consumer thread per block
    TileKernelFn fn = pick_tile(L.xmode, nch <= kXregChunks, L.dec.pro, L.dec.epi, L.sel_out != nullptr);
    if (!fn) return kErrInval;  // a prologue / epilogue / pick combination no caller uses
    TileParams p{};
    p.w = L.w;
    p.y = L.y;
    p.x = L.x;
    p.status = status_word();
    if (!p.status) return kErrNoDev;
    p.rows = L.rows;
    p.k = L.k;
    p.nb = nb;
    p.nch = nch;
    p.groups = (L.rows + kTileRows - 1) / kTileRows;
    p.unit = L.dec.act_q8 ? 4 : 1;
    const int units = (p.groups + p.unit - 1) / p.unit;
    p.slot_bytes = nch * kTileBytes;
    p.round_mode = L.round_mode;
    p.l2_policy = L.l2_policy;
    if (L.sel_out) {
        if (!L.sel_scratch) return kErrInval;
        p.sel_out = L.sel_out;
        p.sel_base = L.sel_base;
        p.sel_cand = static_cast<float2 *>(L.sel_scratch);
        p.sel_ticket = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(L.sel_scratch) + kSelMaxCtas * sizeof(float2));
    }
    p.dec = L.dec;
    p.trace = L.trace;
    int xarea = xarea_bytes(L.k) + (L.dec.pro != kProPlain ? norm_extra_bytes(L.k) : 0);
    if (L.dec.act_q8) {
        // the CTA's act values: at most ceil(units / min(SMs, units)) units
        // (the grid is at least that large)
        const int sms0 = sm_count();
        if (sms0 <= 0) return kErrNoDev;
        const int gmin = units < sms0 ? units : sms0;
        p.act_off = xarea;
        xarea += (units + gmin - 1) / gmin * p.unit * (kTileRows / 2) * 4;
    }
    const int fixed = kSmemAlign + xarea;
    const int limit = max_smem_optin() - 1024;  // static shared memory
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    int cap = tu.stages < 1 ? 1 : (tu.stages > kMaxStages ? kMaxStages : tu.stages);
    if (L.max_stages > 0 && L.max_stages < cap) cap = L.max_stages;
    // The grid decides how many row groups the busiest CTA takes (`need`),
    // and with ring_to_groups how many stages are worth their shared memory
    // (a small ring leaves room on the SM for the next launch's CTA); that
    // memory in turn decides how many CTAs fit on an SM. Start from the
    // asked CTAs per SM and step down until they fit.
    int per_sm = tu.ctas_per_sm < 1 ? 1 : tu.ctas_per_sm;
    int grid = 0, stages = 0, smem = 0;
    for (;;) {
        grid = sms * per_sm;
        if (grid > units) grid = units;
        if (grid > kSelMaxCtas) grid = kSelMaxCtas;
        const int need = (units + grid - 1) / grid * p.unit;
        if (L.ring_to_groups && need <= cap && fixed + need * p.slot_bytes <= limit) {
            stages = need;  // every group its own stage: no stage is filled twice
        } else {
            // A quad waits for a stage by its mbarrier's phase parity, which
            // names the right fill only while the stage's previous group was
            // the same quad's: the quads take groups round-robin, so a stage
            // count that refills stages is a multiple of kQuads (with 1 or 3
            // stages and 2 quads, a quad could pass the wait for its next
            // group on the previous fill and read stale tiles).
            stages = cap < kQuads ? kQuads : cap - cap % kQuads;
            while (stages > kQuads && fixed + stages * p.slot_bytes > limit) stages -= kQuads;
        }
        smem = fixed + stages * p.slot_bytes;
        if (smem > limit) return kErrInval;
        const int fit = resident_ctas(reinterpret_cast<const void *>(fn), kTileThreads, smem);
        if (fit < 1) return kErrInval;
        if (per_sm <= fit) break;  // one wave: every CTA resident at once
        per_sm = fit;
    }
    p.stages = stages;
    out->p = p;
    out->fn = fn;
    out->grid = grid;
    out->smem = smem;
    out->threads = kTileThreads;
    return 0;
}

}  // namespace

int tile_select_scratch_bytes() { return static_cast<int>(kSelMaxCtas * sizeof(float2) + 16); }

size_t tiled_bytes(int rows, int k) {
    if (rows <= 0 || k <= 0 || k % 256) return 0;
    return static_cast<size_t>((rows + kTileRows - 1) / kTileRows) * (k / 256) * kTileBytes;
}

int tile_validate(const TileLaunch &L, const char **why) {
    auto bad = [&](const char *w) { if (why) *why = w; return kErrInval; };
    if (L.xmode != kXPacked && L.xmode != kXF32) return bad("unknown x mode");
    if (L.round_mode != kRoundContract && L.round_mode != kRoundRoundf) return bad("unknown rounding mode");
    if (L.k <= 0 || L.k % 256) return bad("k must be a positive multiple of 256 (nb % 8 == 0, q4_0.py:166)");
    if (L.k > kMaxK) return bad("k above 8192");
    if (L.rows <= 0) return bad("rows must be positive");
    if (!L.w || reinterpret_cast<uintptr_t>(L.w) % 16) return bad("tiles must be 16-byte aligned");
    if (!L.x || reinterpret_cast<uintptr_t>(L.x) % 16) return bad("x must be 16-byte aligned");
    const DecodeOps &D = L.dec;
    const bool y_needed = D.epi == kEpiStore || D.epi == kEpiRopeKv;
    if (y_needed ? (!L.y || reinterpret_cast<uintptr_t>(L.y) % 4) : (L.y && reinterpret_cast<uintptr_t>(L.y) % 4))
        return bad("y must be 4-byte aligned");
    if (D.pro < kProPlain || D.pro > kProEmbedNorm || D.epi < kEpiStore || D.epi > kEpiResidual)
        return bad("unknown decoder prologue or epilogue");
    if (D.pro != kProPlain) {
        if (L.xmode != kXF32) return bad("a normalising prologue needs float32 x");
        if (!D.res || !D.norm_w || reinterpret_cast<uintptr_t>(D.res) % 16 || reinterpret_cast<uintptr_t>(D.norm_w) % 16)
            return bad("rmsnorm prologue: res and norm_w must be 16-byte aligned");
        if (D.pro == kProEmbedNorm && (!D.embd || !D.tokens || !D.pos || reinterpret_cast<uintptr_t>(D.embd) % 2))
            return bad("embedding prologue: token_embd, tokens and pos needed");
    }
    if (D.epi == kEpiRopeKv) {
        if (!D.rope_cs || !D.kcache || !D.vcache || !D.pos || D.head_dim <= 0 || D.head_dim % 2 || D.q_rows % D.head_dim ||
            D.kv_rows % D.head_dim || D.q_rows % kTileRows || D.kv_rows % kTileRows || D.ctx_max <= 0 ||
            D.kv_stride < D.ctx_max || D.kv_stride % 8 || L.rows != D.q_rows + 2 * D.kv_rows)
            return bad("rope/KV epilogue: inconsistent q/k/v rows, head_dim or caches");
    }
    if (D.epi == kEpiSiluPairs && (!D.act || L.rows % 2)) return bad("silu epilogue: act needed, rows even");
    if (D.act_q8 && (D.epi != kEpiSiluPairs || L.rows % 64 || reinterpret_cast<uintptr_t>(D.act_q8) % 16))
        return bad("act_q8: a SiLU epilogue over whole 32-value blocks, 16-byte aligned");
    if (D.epi == kEpiResidual) {
        if (!D.res) return bad("residual epilogue: res needed");
        if (D.nranks < 1 || D.nranks > kMaxDecodeRanks || D.rank < 0 || D.rank >= D.nranks)
            return bad("residual epilogue: bad rank count");
        if (D.nranks > 1) {
            if (!D.step || !D.peer_status || D.slot_words < static_cast<uint64_t>(L.rows)) return bad("residual exchange: window too small");
            for (int r = 0; r < D.nranks; ++r)
                if (!D.win_words[r]) return bad("residual exchange: a peer window is not mapped");
        }
    }
    if (D.adv_pos && (!L.sel_out || !D.adv_step || !D.adv_tokens || !D.n_prompt))
        return bad("advance needs the fused pick, step, tokens and n_prompt");
    return 0;
}

int tile_grid(const TileLaunch &L, const Tuning &tu, int *grid, int *smem_bytes) {
    TilePlan pl;
    if (int rc = make_tile_plan(L, tu, &pl)) return rc;
    if (grid) *grid = pl.grid;
    if (smem_bytes) *smem_bytes = pl.smem;
    return 0;
}

int tile_launch(const TileLaunch &L, const Tuning &tu, cudaStream_t stream) {
    TilePlan pl;
    if (int rc = make_tile_plan(L, tu, &pl)) return rc;
    if (!ensure_smem(reinterpret_cast<const void *>(pl.fn), pl.smem)) return kErrCuda;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(pl.threads);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, pl.fn, pl.p) == cudaSuccess ? 0 : kErrCuda;
}

int repack_launch(const uint8_t *src_rows, int rows, int k, uint8_t *dst_tiles, cudaStream_t stream) {
    if (!src_rows || !dst_tiles || rows <= 0 || k <= 0 || k % 256) return kErrInval;
    if (reinterpret_cast<uintptr_t>(src_rows) % 2 || reinterpret_cast<uintptr_t>(dst_tiles) % 16) return kErrInval;
    const long long total = static_cast<long long>((rows + kTileRows - 1) / kTileRows) * kTileRows * (k / kQK);
    long long blocks = (total + 255) / 256;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    repack_tiles_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src_rows, rows, k, dst_tiles);
    return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
