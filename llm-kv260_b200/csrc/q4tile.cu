// Q4_0 x Q8_0 GEMV over the B200 tile layout: the engine path's kernel.
// Bit-exact to src/llm_kv260/q4_0.py:151-182, like the GGUF-layout kernel in
// q4gemv.cu; only where the bytes sit differs.
//
// Tile layout. The reference re-lays every matrix at load for its engine
// (board/tp/tp_llama.cpp:102-118, the gemv2 chunk interleave); this engine
// does the same for HBM. Rows are padded to a multiple of 16. For row group
// g (rows 16g..16g+15) and chunk c (blocks 8c..8c+7) a 2304-byte tile sits at
// byte ((g * nch) + c) * 2304:
//     [0, 2048)     nibbles: 16 bytes for lane l, row i at (l * 16 + i) * 16
//     [2048, 2304)  scales:  float16 bits for lane l, row i at 2048 + (l * 16 + i) * 2
// The 16 nibble bytes of a block are copied unchanged (byte j: weight j in
// the low nibble, weight j+16 in the high one), so the bytes per weight stay
// 18/32 and the algorithmic traffic is the GGUF file's.
//
// Kernel. A CTA owns whole 16-row groups. Thread (s, l, i) -- K-slice s,
// lane l, row i -- computes the block terms of lane l of row i for the chunks
// of slice s (at most 8, so its x blocks stay in registers). With one slice
// (K <= 2048) the thread adds its terms straight into the lane chain; with
// several, the terms go to shared memory and slice 0 then runs each lane's
// chain over all chunks in order -- the float adds stay sequential exactly as
// q4_0.py:177-179 orders them, only the block dots run in parallel. A stage is
// one row group's whole tile run, moved by ONE 1-D bulk copy (TMA engine, no
// multicast) into an mbarrier ring, issued before the kernel waits on its
// predecessor (programmatic dependent launch). Every block is one conflict-
// free 128-bit shared load (a warp reads 512 contiguous bytes) plus a 16-bit
// scale load and 8 __dp4a; all warps run identical code. Per row group the 8
// lane sums meet in tree_sum's order.
#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"

namespace b200 {

namespace {

constexpr int kTileThreads = kTileRows * kLanes;   // threads per K-slice: 128
constexpr int kTileNibBytes = kTileThreads * 16;   // 2048
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 64;
constexpr int kRedBytes = 2 * kTileThreads * 4;    // double-buffered lane sums
constexpr int kSmemAlign = 128;
constexpr int kMaxCps = 8;                         // chunks per K-slice (x blocks in registers)
constexpr int kSelMaxCtas = 4096;                  // fused greedy pick: candidate slots

struct TileParams {
    const uint8_t *w;
    float *y;
    const void *x;
    unsigned *status;
    int rows, k, nb, nch;
    int groups;
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
};

constexpr uint64_t kPeerTimeoutNs = 1000000000ull;  // a peer's row words: 1 s

__device__ __forceinline__ void st_word(uint64_t *p, uint64_t w) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Decoder prologue: x = rmsnorm(res) * norm_w, quantised into xs (the same
// layout as stage_x). One thread per 32-block. res is the residual stream,
// or (kProEmbedNorm) the token's embedding row, which CTA 0 also writes to
// res. The sum of squares runs in parallel in double; rms_float_is_safe
// decides whether its float is the reference's, else threads 0-3 redo the
// four lane sums in the reference's order from the copy of x in xf.
__device__ __noinline__ void stage_x_norm(const TileParams &p, uint8_t *xs, float *xf, double *dred) {
    __shared__ float s_f;
    __shared__ int s_exact;
    const int k = p.k, nb = k / kQK, b = threadIdx.x, lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    float v[32];
    double ss = 0.0;
    if (b < nb) {
        if (p.dec.pro == kProEmbedNorm) {
            const int tok = p.dec.tokens[*p.dec.pos];
            const uint16_t *blk =
                reinterpret_cast<const uint16_t *>(p.dec.embd + (static_cast<size_t>(tok) * nb + b) * kBlockBytes);
            uint16_t h[9];
#pragma unroll
            for (int j = 0; j < 9; ++j) h[j] = blk[j];
            const float d = __half2float(__ushort_as_half(h[0]));
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int byte = (h[1 + j / 2] >> (8 * (j & 1))) & 0xff;
                v[j] = __fmul_rn(__int2float_rn((byte & 0xF) - 8), d);
                v[j + 16] = __fmul_rn(__int2float_rn((byte >> 4) - 8), d);
            }
            if (blockIdx.x == 0) {
                float4 *dst = reinterpret_cast<float4 *>(p.dec.res) + 8 * b;
#pragma unroll
                for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        } else {
            const float4 *src = reinterpret_cast<const float4 *>(p.dec.res) + 8 * b;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 f = src[j];
                v[4 * j] = f.x;
                v[4 * j + 1] = f.y;
                v[4 * j + 2] = f.z;
                v[4 * j + 3] = f.w;
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) ss = __dadd_rn(ss, __dmul_rn(static_cast<double>(v[j]), static_cast<double>(v[j])));
        float4 *xd = reinterpret_cast<float4 *>(xf) + 8 * b;
#pragma unroll
        for (int j = 0; j < 8; ++j) xd[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(kFullMask, ss, off));
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) tot = __dadd_rn(tot, dred[w]);
        const double q = __ddiv_rn(tot, static_cast<double>(k));
        const float f = __double2float_rn(q);
        s_exact = p.dec.exact_norm || !rms_float_is_safe(q, f, k);
        s_f = f;
    }
    __syncthreads();
    if (s_exact) {
        // tp_llama.cpp:560-564: lane j sums x[i]^2 for i = j, j+4, ... in order
        if (threadIdx.x < 4) {
            double a = 0.0;
            for (int i = threadIdx.x; i < k; i += 4)
                a = __dadd_rn(a, __dmul_rn(static_cast<double>(xf[i]), static_cast<double>(xf[i])));
            dred[threadIdx.x] = a;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            const double ss2 = __dadd_rn(__dadd_rn(dred[0], dred[2]), __dadd_rn(dred[1], dred[3]));
            s_f = __double2float_rn(__ddiv_rn(ss2, static_cast<double>(k)));
        }
        __syncthreads();
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s_f, p.dec.eps)));
    if (b < nb) {
        const float4 *wv = reinterpret_cast<const float4 *>(p.dec.norm_w) + 8 * b;
        float4 hv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 w4 = __ldg(wv + j);
            hv[j].x = __fmul_rn(__fmul_rn(v[4 * j], scale), w4.x);
            hv[j].y = __fmul_rn(__fmul_rn(v[4 * j + 1], scale), w4.y);
            hv[j].z = __fmul_rn(__fmul_rn(v[4 * j + 2], scale), w4.z);
            hv[j].w = __fmul_rn(__fmul_rn(v[4 * j + 3], scale), w4.w);
        }
        uint32_t q[8];
        float d;
        const int sum = q8_quant_block(hv, p.round_mode, q, &d);
        uint4 *qdst = reinterpret_cast<uint4 *>(xs + 32 * b);
        qdst[0] = make_uint4(q[0], q[1], q[2], q[3]);
        qdst[1] = make_uint4(q[4], q[5], q[6], q[7]);
        reinterpret_cast<int2 *>(xs + k)[b] = make_int2(__float_as_int(__half2float(__float2half_rn(d))), sum);
    }
}

// Byte offset of the decoder's x copy (xf) after the staged x, and its size.
__host__ __device__ constexpr int xarea_bytes(int k) { return (k + 8 * (k / kQK) + 15) / 16 * 16; }
constexpr int norm_extra_bytes(int k) { return 4 * k + 32 * 8; }  // xf [k] floats + 32 doubles

// (value desc, index asc); NaN never beats a number (the scan's rule for any
// index but 0, which the final step handles).
__device__ __forceinline__ bool sel_better(float av, int ai, float bv, int bi) {
    if (isnan(bv)) return !isnan(av) || ai < bi;
    if (isnan(av)) return false;
    return av > bv || (av == bv && ai < bi);
}

__device__ __forceinline__ void issue_group(const TileParams &p, uint64_t *bars, uint8_t *ring, int g, int s,
                                            uint64_t policy) {
    const int slot = s % p.stages;
    mbar_arrive_expect_tx(&bars[slot], static_cast<uint32_t>(p.slot_bytes));
    bulk_g2s(ring + slot * p.slot_bytes, p.w + static_cast<size_t>(g) * p.slot_bytes,
             static_cast<uint32_t>(p.slot_bytes), &bars[slot], policy);
}

// Block term of tile `tile` (one chunk of the row group) for this thread's
// (lane, row) slot u = lane * 16 + row.
__device__ __forceinline__ float tile_term(const uint8_t *tile, int u, const XBlock &xb) {
    const uint4 nv = *reinterpret_cast<const uint4 *>(tile + u * 16);
    const uint32_t db = *reinterpret_cast<const uint16_t *>(tile + kTileNibBytes + u * 2);
    const uint32_t n[4] = {nv.x, nv.y, nv.z, nv.w};
    return block_term_words(n, db, xb);
}

// CPS: chunks per K-slice; KS: K-slices (threads = 128 * KS); KS * CPS >= nch.
template <int XMODE, int CPS, int KS>
__global__ void __launch_bounds__(kTileThreads * KS) q4_tile_kernel(const __grid_constant__ TileParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    uint8_t *ring = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + kSmemAlign - 1) & ~static_cast<uintptr_t>(kSmemAlign - 1));
    uint8_t *after = ring + p.stages * p.slot_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(after);
    float *red = reinterpret_cast<float *>(after + kBarBytes);
    float *tv = reinterpret_cast<float *>(after + kBarBytes + kRedBytes);  // [nch][128], KS > 1 only
    uint8_t *xs = after + kBarBytes + kRedBytes + (KS > 1 ? p.nch * kTileThreads * 4 : 0);

    const int t = threadIdx.x, slice = t / kTileThreads, u = t % kTileThreads, L = u / kTileRows;
    const int g0 = static_cast<int>(static_cast<long long>(p.groups) * blockIdx.x / gridDim.x);
    const int g1 = static_cast<int>(static_cast<long long>(p.groups) * (blockIdx.x + 1) / gridDim.x);
    const int S = p.stages;
    const int nst = g1 - g0;

    if (t == 0) {
        s_abort = 0;
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const uint64_t policy = make_policy(p.l2_policy);
    // The weights do not depend on the previous kernel: start them moving,
    // let the next kernel launch, then wait for x.
    if (t == 0)
        for (int s = 0; s < nst && s < S; ++s) issue_group(p, bars, ring, g0 + s, s, policy);
    pdl_launch_dependents();
    pdl_wait_prior_grid();

    // One thread per x block: 128*KS threads >= 8*nch blocks, as KS >= nch/8.
    if (XMODE == kXF32 && p.dec.pro != kProPlain)
        stage_x_norm(p, xs, reinterpret_cast<float *>(xs + xarea_bytes(p.k)),
                     reinterpret_cast<double *>(xs + xarea_bytes(p.k) + 4 * p.k));
    else
        stage_x<XMODE>(p.x, p.k, p.round_mode, xs);
    __syncthreads();
    const int epi = p.dec.epi;
    const int dpos = (epi == kEpiRopeKv) ? *p.dec.pos : 0;
    const bool xchg = epi == kEpiResidual && p.dec.nranks > 1;
    uint32_t epoch = 0;
    uint64_t slot_off = 0;
    if (xchg) {
        epoch = *p.dec.step * static_cast<uint32_t>(p.dec.ar_per_token) + static_cast<uint32_t>(p.dec.ar_index) + 1u;
        slot_off = static_cast<uint64_t>(epoch & 1u) * kMaxDecodeRanks * p.dec.slot_words;
    }
    const int c_first = slice * CPS;
    XBlock xr[CPS];
#pragma unroll
    for (int j = 0; j < CPS; ++j)
        if (c_first + j < p.nch) load_xblock_smem(xs, p.k, 8 * (c_first + j) + L, xr[j]);

    float best_v = __int_as_float(0x7fc00000);  // NaN: loses to any number
    int best_i = 0x7fffffff;
    int s = 0;
    for (; s < nst; ++s) {
        const int slot = s % S;
        if (!wait_stage(&bars[slot], static_cast<uint32_t>((s / S) & 1), p.status)) s_abort = 1;
        const uint8_t *tiles = ring + slot * p.slot_bytes;
        float *rbuf = red + (s & 1) * kTileThreads;
        if constexpr (KS == 1) {
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < CPS; ++j)
                if (j < p.nch) acc = __fadd_rn(acc, tile_term(tiles + j * kTileBytes, u, xr[j]));
            rbuf[u] = acc;
        } else {
#pragma unroll
            for (int j = 0; j < CPS; ++j) {
                const int c = c_first + j;
                if (c < p.nch) tv[c * kTileThreads + u] = tile_term(tiles + c * kTileBytes, u, xr[j]);
            }
            __syncthreads();
            if (slice == 0) {
                // lane chain over all chunks, in order (q4_0.py:177-179)
                float acc = 0.0f;
                for (int c = 0; c < p.nch; ++c) acc = __fadd_rn(acc, tv[c * kTileThreads + u]);
                rbuf[u] = acc;
            }
        }
        __syncthreads();
        if (s_abort) break;
        if (t == 0 && s + S < nst) issue_group(p, bars, ring, g0 + s + S, s + S, policy);
        if (t < kTileRows) {
            const float *r = rbuf + t;
            const float yv = tree8(r[0 * kTileRows], r[1 * kTileRows], r[2 * kTileRows], r[3 * kTileRows],
                                   r[4 * kTileRows], r[5 * kTileRows], r[6 * kTileRows], r[7 * kTileRows]);
            const int row = (g0 + s) * kTileRows + t;
            const bool live = row < p.rows;
            if (epi == kEpiStore) {
                if (live) {
                    p.y[row] = yv;
                    if (sel_better(yv, row, best_v, best_i)) {
                        best_v = yv;
                        best_i = row;
                    }
                }
            } else if (epi == kEpiRopeKv) {
                // q and k rows start at multiples of head_dim (even), and a row
                // group at a multiple of 16, so rope's pair (2i, 2i+1) is this
                // thread and its neighbour t ^ 1
                const float other = __shfl_xor_sync(0x0000ffffu, yv, 1);
                if (live) {
                    const int hd = p.dec.head_dim, k0 = p.dec.q_rows, v0 = k0 + p.dec.kv_rows;
                    float out = yv;
                    if (row < v0) {
                        const int i = (row % hd) >> 1;
                        const float *cs = p.dec.rope_cs + static_cast<size_t>(dpos) * hd;
                        const bool even = !(row & 1);
                        out = rope_pair(even ? yv : other, even ? other : yv, cs[2 * i], cs[2 * i + 1], even);
                    }
                    p.y[row] = out;
                    if (row >= k0) {
                        const bool isk = row < v0;
                        const int rr = row - (isk ? k0 : v0);
                        const size_t at = (static_cast<size_t>(rr / hd) * p.dec.ctx_max + dpos) * hd + rr % hd;
                        void *cache = isk ? p.dec.kcache : p.dec.vcache;
                        if (p.dec.kv_f16)
                            static_cast<__half *>(cache)[at] = __float2half_rn(out);
                        else
                            static_cast<float *>(cache)[at] = out;
                    }
                }
            } else if (epi == kEpiSiluPairs) {
                const float other = __shfl_xor_sync(0x0000ffffu, yv, 1);
                if (live) {
                    if (p.y) p.y[row] = yv;
                    if (!(row & 1)) p.dec.act[row >> 1] = silu_mul(yv, other);
                }
            } else if (live) {  // kEpiResidual
                if (p.y) p.y[row] = yv;
                if (!xchg) {
                    p.dec.res[row] = __fadd_rn(p.dec.res[row], yv);
                } else {
                    const uint64_t word = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(yv);
                    const uint64_t at = slot_off + static_cast<uint64_t>(p.dec.rank) * p.dec.slot_words + row;
                    for (int r = 0; r < p.dec.nranks; ++r) st_word(p.dec.win_words[r] + at, word);
                }
            }
        }
    }
    if (xchg && t < kTileRows && !s_abort) {
        // Every rank computed these rows' partials for its K slice; collect
        // them from this rank's window and sum in rank order
        // (tp_llama.cpp:515-521), then add into the residual (add_into).
        const uint64_t *own = p.dec.win_words[p.dec.rank] + slot_off;
        for (int s2 = 0; s2 < nst; ++s2) {
            const int row = (g0 + s2) * kTileRows + t;
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
    if (p.sel_out) {
        // CTA best over the 16 tree threads (lanes 0..15 of warp 0), then the
        // last CTA to finish reduces all CTAs' bests.
        if (t < 32) {
            for (int off = 8; off > 0; off >>= 1) {
                const float ov = __shfl_down_sync(kFullMask, best_v, off, 16);
                const int oi = __shfl_down_sync(kFullMask, best_i, off, 16);
                if (sel_better(ov, oi, best_v, best_i)) {
                    best_v = ov;
                    best_i = oi;
                }
            }
        }
        __shared__ unsigned s_last;
        if (t == 0) {
            p.sel_cand[blockIdx.x] = make_float2(best_v, __int_as_float(best_i));
            __threadfence();
            s_last = atomicAdd(p.sel_ticket, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (s_last && t < 32) {
            __threadfence();
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
                }
            }
        }
    }
    if (s < nst && t == 0) {
        // Aborted on a stage timeout: let copies already in flight land (each
        // wait bounded) before the CTA's shared memory goes away.
        for (int r = s; r < nst && r < s + S; ++r)
            (void)wait_stage(&bars[r % S], static_cast<uint32_t>((r / S) & 1), p.status);
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
        *reinterpret_cast<uint4 *>(tile + (l * kTileRows + i) * 16) = nv;
        *reinterpret_cast<uint16_t *>(tile + kTileNibBytes + (l * kTileRows + i) * 2) = h[0];
    }
}

using TileKernelFn = void (*)(TileParams);

template <int XMODE, int KS>
TileKernelFn pick_cps(int cps) {
    switch (cps) {
        case 1: return q4_tile_kernel<XMODE, 1, KS>;
        case 2: return q4_tile_kernel<XMODE, 2, KS>;
        case 3: return q4_tile_kernel<XMODE, 3, KS>;
        case 4: return q4_tile_kernel<XMODE, 4, KS>;
        case 5: return q4_tile_kernel<XMODE, 5, KS>;
        case 6: return q4_tile_kernel<XMODE, 6, KS>;
        case 7: return q4_tile_kernel<XMODE, 7, KS>;
        case 8: return q4_tile_kernel<XMODE, 8, KS>;
        default: return nullptr;
    }
}

template <int XMODE>
TileKernelFn pick_tile(int cps, int ks) {
    if (ks == 1) return pick_cps<XMODE, 1>(cps);
    if (ks == 2) return pick_cps<XMODE, 2>(cps);
    if (ks == 4) return pick_cps<XMODE, 4>(cps);
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
    // K-slices: enough that a slice has at most 8 chunks, more if asked.
    int ks = 1;
    while (ks < 4 && (ks * kMaxCps < nch || ks < tu.kslices)) ks *= 2;
    while (ks > 1 && ks > nch) ks /= 2;  // every slice gets at least one chunk
    const int cps = (nch + ks - 1) / ks;
    if (cps > kMaxCps) return kErrInval;
    TileKernelFn fn = L.xmode == kXF32 ? pick_tile<kXF32>(cps, ks) : pick_tile<kXPacked>(cps, ks);
    if (!fn) return kErrInval;
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
    p.slot_bytes = nch * kTileBytes;
    p.stages = tu.stages < 1 ? 1 : (tu.stages > kMaxStages ? kMaxStages : tu.stages);
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
    const int threads = kTileThreads * ks;
    if (L.dec.pro != kProPlain && nb > threads) return kErrInval;  // one thread per x block
    const int xarea = xarea_bytes(L.k) + (L.dec.pro != kProPlain ? norm_extra_bytes(L.k) : 0);
    const int fixed = kSmemAlign + kBarBytes + kRedBytes + (ks > 1 ? nch * kTileThreads * 4 : 0) + xarea;
    const int limit = max_smem_optin();
    while (p.stages > 1 && fixed + p.stages * p.slot_bytes > limit) p.stages -= 1;
    const int smem = fixed + p.stages * p.slot_bytes;
    if (smem > limit) return kErrInval;
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    int per_sm = tu.ctas_per_sm < 1 ? 1 : tu.ctas_per_sm;
    const int fit = resident_ctas(reinterpret_cast<const void *>(fn), threads, smem);
    if (per_sm > fit) per_sm = fit;  // one wave: every CTA resident at once
    int grid = sms * per_sm;
    if (grid > p.groups) grid = p.groups;
    if (grid > kSelMaxCtas) grid = kSelMaxCtas;
    out->p = p;
    out->fn = fn;
    out->grid = grid;
    out->smem = smem;
    out->threads = threads;
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
            L.rows != D.q_rows + 2 * D.kv_rows)
            return bad("rope/KV epilogue: inconsistent q/k/v rows, head_dim or caches");
    }
    if (D.epi == kEpiSiluPairs && (!D.act || L.rows % 2)) return bad("silu epilogue: act needed, rows even");
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
