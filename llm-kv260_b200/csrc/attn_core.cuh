// Decode attention for one KV head and the G <= 4 query heads that share it,
// bit-exact to the reference runtime's attention_group
// (board/tp/tp_llama.cpp:644-690) with softmax_exp (624-634): the shared core
// of the per-op attention kernel (attn.cu) and of the persistent kernel's
// attention phase (token.cu).
//
// Cache layouts, per layer and KV head, `stride` positions per head:
//   K   [kv head][stride][D]   a position's row contiguous, lane-major
//                              (k_slot, decode.cuh): the elements that
//                              fused-multiply-add lane j takes (j, j+4, ...)
//                              stored together, so the thread running lane j
//                              reads only its quarter of the row; 16-byte
//                              segments swizzled by the position, so the
//                              lanes of consecutive positions read distinct
//                              bank groups
//   V^T [kv head][D][stride]   a column's positions contiguous: one 16-byte
//                              shared load feeds 16 / esz steps of a chain
// The reference keeps V position-major and K rows in order; the values and
// the order of every operation on them are unchanged, only where they sit.
// Both are staged into shared memory by 1-D bulk copies (TMA engine, no
// multicast): K in chunks of KC rows (one copy each), V^T in chunks of COLB
// bytes per column (one copy per column).
//
// Phases, NT threads, each in the reference's arithmetic order:
//   scores  four threads per position t, thread j running FMA lane j
//           (element i feeds lane i & 3, i increasing) of every head from
//           its quarter of the K row, then (a0 + a1) + (a2 + a3) by xor
//           shuffles, times scale (652-664);
//   max     per head, the running `>` max from -1e30f: max is exact, so a
//           tree over threads gives the same value (no NaN ever wins, and
//           +-0 ties give the same exponentials);
//   exp     s = v_expf(s - max) per position and head;
//   sums    four threads per head: lane j adds positions j, j+4, ... below
//           n - n % 4 in order, then (l0 + l1) + (l2 + l3) by two xor
//           shuffles, then the tail one position at a time; inv = 1 / sum;
//   p       p_t = s_t * inv;
//   output  thread (column c, head pair): acc = fma(v[t][c], p_t, acc) for
//           t = 0..n-1 in order, from two V^T stages whose first copies are
//           issued before the scores, so they land meanwhile.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"

namespace b200 {

// V^T chunk: COLB bytes of each column per stage, stored COLB + 16 bytes
// apart (an odd number of 16-byte units, so the 32 columns a warp reads in
// one 16-byte load fall on distinct bank groups).
constexpr int kAttnVtStages = 2;
constexpr int kAttnKStages = 2;  // K chunks double-buffered: chunk c + 2 lands while chunk c + 1 is scored
constexpr int kAttnBars = kAttnVtStages + kAttnKStages;  // mbarriers: V^T stages, then the K stages

__host__ __device__ constexpr int attn_core_smem_bytes(int d, int esz, int colb, int kc, int nt, int stride) {
    return kAttnVtStages * d * (colb + 16)  // V^T stages
           + kAttnKStages * kc * d * esz    // K stages: kc rows each
           + 4 * d * 4                      // q, up to 4 heads
           + (nt / 32) * 16                 // per-warp maxima, 4 heads
           + 32                             // 1 / sum per head
           + 16 * stride                    // scores -> exponentials, [position][4 heads]
           + 16 * stride;                   // p, [head pair][position][2]
}

// the reference's running max (`if (s > mx) mx = s`), as a combine
__device__ __forceinline__ float attn_max_gt(float a, float b) { return b > a ? b : a; }

// 16 bytes of a K row or V^T column as floats (ESZ 2: 8 halves, ESZ 4: 4 floats).
template <int ESZ>
__device__ __forceinline__ void attn_seg_floats(const uint4 &v, float *f) {
    if constexpr (ESZ == 2) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 t = __half22float2(h[j]);
            f[2 * j] = t.x;
            f[2 * j + 1] = t.y;
        }
    } else {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
}

template <int ESZ>
__device__ __forceinline__ float attn_elem(const uint8_t *p, int i) {
    if constexpr (ESZ == 2)
        return __half2float(reinterpret_cast<const __half *>(p)[i]);
    else
        return reinterpret_cast<const float *>(p)[i];
}

// 4 floats of shared memory, re-read at every use: q stays in shared memory
// instead of being hoisted into registers across the position loop.
__device__ __forceinline__ float4 lds_f4(const float *p) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(smem_addr(p)));
    return v;
}

__device__ __forceinline__ void attn_stamp_at(uint64_t *rec, int j) {
    if (rec && threadIdx.x == 0) rec[j] = globaltimer_ns();
}

// One warp of the caller may bring this head's K rows and V^T columns for
// positions [0, n_hint) into L2 ahead of time (a hint: any n_hint is safe).
template <int D, int ESZ>
__device__ __forceinline__ void attn_prefetch_l2(const uint8_t *kb, const uint8_t *vtb, int stride, int n_hint) {
    const int lane = threadIdx.x & 31;
    if (n_hint < 1) return;
    if (lane == 0) bulk_prefetch_l2(kb, static_cast<uint32_t>(n_hint) * D * ESZ);
    const uint32_t colb = static_cast<uint32_t>((n_hint * ESZ + 15) / 16 * 16);
    for (int c = lane; c < D; c += 32) bulk_prefetch_l2(vtb + static_cast<size_t>(c) * stride * ESZ, colb);
}

// One KV head's attention over positions [0, n). Every one of the NT
// threads (threadIdx.x < NT) must call it; `bar` is a named barrier for
// exactly those threads. q: the G heads' roped rows (G * D floats, read
// through L2); kb / vtb: this head's K rows and V^T columns (`stride`
// positions); out: G * D floats. smem: attn_core_smem_bytes(D, ESZ, COLB,
// KC, NT, stride) bytes, 16-byte aligned. bars: kAttnBars mbarriers (count
// 1), whose phase parities every thread tracks in `par` (bit b for barrier
// b) across calls. A stage wait that runs out after kStageTimeoutNs sets
// kStatusStageTimeout in *status; the copies in flight are then waited for
// (bounded) and the function returns false with `out` not written.
// rec (optional, thread 0 writes): stamps 4 q staged, 5 scores and maxima,
// 6 exponentials, 7 sums, 2 p; 8 + 2c / 9 + 2c V^T chunk c (< 4) landed /
// consumed.
template <int D, int ESZ, int COLB, int KC, int NT>
__device__ bool attn_core(const float *q, const uint8_t *kb, const uint8_t *vtb, int stride, int n, int G, float scale,
                          float *out, uint8_t *smem, int bar, uint64_t *bars, uint32_t &par, unsigned *status,
                          uint64_t *rec) {
    constexpr int kRowBytes = D * ESZ;
    constexpr int kSegs = kRowBytes / 16;
    constexpr int kPer = 16 / ESZ;         // elements per 16 bytes
    constexpr int kChunkPos = COLB / ESZ;  // positions per V^T chunk
    constexpr int kColStride = COLB + 16;
    constexpr int kStageBytes = D * kColStride;
    constexpr int kKBar = kAttnVtStages;   // K stage s: barrier kKBar + s
    static_assert(kPer % 4 == 0 && kSegs % 8 == 0, "attention shape");
    static_assert(NT % 32 == 0 && NT >= 2 * D && KC % 8 == 0, "one thread per (column, head pair)");

    uint8_t *vt = smem;
    uint8_t *kbuf = smem + kAttnVtStages * kStageBytes;
    float *qs = reinterpret_cast<float *>(kbuf + kAttnKStages * KC * kRowBytes);
    float *part = qs + 4 * D;             // [NT/32][4]
    float *hinv = part + (NT / 32) * 4;   // [4] 1 / sum per head, then a failure flag
    int *fail = reinterpret_cast<int *>(hinv + 4);
    float4 *e = reinterpret_cast<float4 *>(hinv + 8);  // [stride]
    float2 *pp = reinterpret_cast<float2 *>(e + stride);  // [2][stride]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nch = (n + kChunkPos - 1) / kChunkPos, nkc = (n + KC - 1) / KC;
    const uint64_t pol = l2_policy_evict_last();  // the KV cache stays in L2 while the weights stream past
    uint32_t pend = 0;  // barriers with copies issued and not yet waited for (the same in every thread)

    // V^T chunk c into stage c % 2: thread `col` < D copies its column's
    // bytes (rounded up to 16, which stays below stride: stride % 8 == 0);
    // thread 0 posts the stage's byte count with its arrival (a copy that
    // completes first only takes the count below zero for a moment)
    auto stage_vt = [&](int c) {
        if (c >= nch) return;
        const int rows = min(kChunkPos, n - c * kChunkPos);
        const uint32_t colb = static_cast<uint32_t>((rows * ESZ + 15) / 16 * 16);
        const int slot = c % kAttnVtStages;
        if (tid == 0) mbar_arrive_expect_tx(&bars[slot], colb * D);
        if (tid < D)
            bulk_g2s(vt + slot * kStageBytes + tid * kColStride,
                     vtb + static_cast<size_t>(tid) * stride * ESZ + static_cast<size_t>(c) * COLB, colb, &bars[slot], pol);
        pend |= 1u << slot;
    };
    // K rows [kc * KC, ...) into K stage kc % 2: one copy
    auto stage_k = [&](int kc) {
        if (kc >= nkc) return;
        const int r0 = kc * KC, rows = min(KC, n - r0), sb = kKBar + kc % kAttnKStages;
        if (tid == 0) {
            mbar_arrive_expect_tx(&bars[sb], static_cast<uint32_t>(rows * kRowBytes));
            bulk_g2s(kbuf + (kc % kAttnKStages) * KC * kRowBytes, kb + static_cast<size_t>(r0) * kRowBytes,
                     static_cast<uint32_t>(rows * kRowBytes), &bars[sb], pol);
        }
        pend |= 1u << sb;
    };
    auto wait_bar = [&](int b) {
        if (wait_stage(&bars[b], (par >> b) & 1u, status)) {
            par ^= 1u << b;
            pend &= ~(1u << b);
        } else {
            atomicExch(fail, 1);
        }
    };
    // after a barrier that saw *fail: the copies in flight land (each wait
    // bounded) before this shared memory is used for anything else
    auto drain = [&]() {
        if (tid == 0)
            for (int b = 0; b < kAttnBars; ++b)
                if (pend & (1u << b)) (void)wait_stage(&bars[b], (par >> b) & 1u, status);
        named_sync(bar, NT);
        return false;
    };

    // q first: its load is on the critical path, the copies land meanwhile
    float qv[(4 * D + NT - 1) / NT];
#pragma unroll
    for (int u = 0; u < (4 * D + NT - 1) / NT; ++u) {
        const int i = tid + u * NT;
        if (i < G * D) qv[u] = __ldcg(q + i);
    }
    stage_k(0);
    stage_k(1);
#pragma unroll
    for (int u = 0; u < (4 * D + NT - 1) / NT; ++u) {
        const int i = tid + u * NT;
        if (i < G * D) qs[i] = qv[u];
    }
    if (tid == 0) *fail = 0;
    named_sync(bar, NT);
    attn_stamp_at(rec, 4);
    // V^T is needed only by the output chains: its copies start after q
    // has arrived (a load queued behind them would wait for their bytes)
    stage_vt(0);
    stage_vt(1);

    // scores (tp_llama.cpp:652-664) and this thread's maxima: four threads
    // per position, thread j running fused-multiply-add lane j (elements
    // i = j, j+4, ... in order) of every head; the lanes meet as
    // (l0 + l1) + (l2 + l3) by xor shuffles 1 then 2 -- vaddvq_f32's pairing,
    // so all four threads hold the reference's score
    float mx[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
    const int jl = tid & 3;
    for (int kc = 0; kc < nkc; ++kc) {
        const int r0 = kc * KC, r1 = min(n, r0 + KC);
        wait_bar(kKBar + kc % kAttnKStages);
        const uint8_t *kst = kbuf + (kc % kAttnKStages) * KC * kRowBytes;
        for (int t0 = r0; t0 < r1; t0 += NT / 4) {  // the same trip count in every thread
            const int t = t0 + (tid >> 2);
            const bool live = t < r1;
            const uint8_t *row = kst + (live ? t - r0 : 0) * kRowBytes;
            // lane jl's segments jl * L .. jl * L + L - 1: steps m in order
            constexpr int L = kSegs / 4;
            float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            uint4 kr[L];
#pragma unroll
            for (int i = 0; i < L; ++i) kr[i] = *reinterpret_cast<const uint4 *>(row + k_phys_seg(jl * L + i, t) * 16);
#pragma unroll
            for (int i = 0; i < L; ++i) {
                float f[kPer];
                attn_seg_floats<ESZ>(kr[i], f);
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    if (b < G) {
#pragma unroll
                        for (int u = 0; u < kPer; ++u) a[b] = __fmaf_rn(f[u], qs[b * D + 4 * (i * kPer + u) + jl], a[b]);
                    }
                }
            }
            float sv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                if (b < G) {
                    const float x = __fadd_rn(a[b], __shfl_xor_sync(kFullMask, a[b], 1));
                    sv[b] = __fmul_rn(__fadd_rn(x, __shfl_xor_sync(kFullMask, x, 2)), scale);
                    if (live) mx[b] = attn_max_gt(mx[b], sv[b]);
                }
            }
            if (live && jl == 0) e[t] = make_float4(sv[0], sv[1], sv[2], sv[3]);
        }
        if (kc + 1 < nkc) {
            named_sync(bar, NT);  // K stage kc % 2 consumed
            if (*reinterpret_cast<volatile int *>(fail)) return drain();
            stage_k(kc + 2);
        }
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        if (b < G) {
            float m = mx[b];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m = attn_max_gt(m, __shfl_xor_sync(kFullMask, m, off));
            if (lane == 0) part[warp * 4 + b] = m;
        }
    }
    named_sync(bar, NT);
    if (*reinterpret_cast<volatile int *>(fail)) return drain();
    attn_stamp_at(rec, 5);

    // every thread reduces the warp maxima itself, then its exponentials
    float m[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
    for (int w = 0; w < NT / 32; ++w) {
        const float4 pw = *reinterpret_cast<const float4 *>(part + w * 4);
        m[0] = attn_max_gt(m[0], pw.x);
        m[1] = attn_max_gt(m[1], pw.y);
        m[2] = attn_max_gt(m[2], pw.z);
        m[3] = attn_max_gt(m[3], pw.w);
    }
    for (int t = tid; t < n; t += NT) {
        float4 s = e[t];
        s.x = v_expf(__fsub_rn(s.x, m[0]));
        if (G > 1) s.y = v_expf(__fsub_rn(s.y, m[1]));
        if (G > 2) s.z = v_expf(__fsub_rn(s.z, m[2]));
        if (G > 3) s.w = v_expf(__fsub_rn(s.w, m[3]));
        e[t] = s;
    }
    named_sync(bar, NT);
    attn_stamp_at(rec, 6);

    // sums (softmax_exp, tp_llama.cpp:626-633): warp 0, lane = 4 * head + j
    if (warp == 0) {
        const int b = lane >> 2, j = lane & 3, n4 = n & ~3;
        const float *col = reinterpret_cast<const float *>(e) + b;
        float acc = 0.0f;
        if (b < G) {
            // batches of 8 positions, the next batch's loads issued before
            // this batch's adds (the adds are one dependent chain)
            int t = j;
            float cur[8];
            const bool any = t + 28 < n4;
            if (any) {
#pragma unroll
                for (int u = 0; u < 8; ++u) cur[u] = col[4 * (t + 4 * u)];
            }
            while (t + 28 < n4) {
                float nxt[8];
                const bool more = t + 60 < n4;
                if (more) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) nxt[u] = col[4 * (t + 32 + 4 * u)];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, cur[u]);
                t += 32;
                if (!more) break;
#pragma unroll
                for (int u = 0; u < 8; ++u) cur[u] = nxt[u];
            }
            for (; t < n4; t += 4) acc = __fadd_rn(acc, col[4 * t]);
        }
        const float x = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, 1));
        const float y = __fadd_rn(x, __shfl_xor_sync(kFullMask, x, 2));
        if (b < G && j == 0) {
            float sum = y;
            for (int t = n4; t < n; ++t) sum = __fadd_rn(sum, col[4 * t]);
            hinv[b] = __fdiv_rn(1.0f, sum);
        }
    }
    named_sync(bar, NT);
    attn_stamp_at(rec, 7);

    // p_t = s_t * inv (tp_llama.cpp:680), stored per head pair: the output
    // chains of a pair read 2 positions' p in 16 bytes
    {
        const float4 iv = *reinterpret_cast<const float4 *>(hinv);
        for (int t = tid; t < n; t += NT) {
            const float4 s = e[t];
            pp[t] = make_float2(__fmul_rn(s.x, iv.x), G > 1 ? __fmul_rn(s.y, iv.y) : 0.0f);
            if (G > 2) pp[stride + t] = make_float2(__fmul_rn(s.z, iv.z), G > 3 ? __fmul_rn(s.w, iv.w) : 0.0f);
        }
    }
    attn_stamp_at(rec, 2);

    // output chains (tp_llama.cpp:667-687): thread (column, head pair)
    const int nsub = (G + 1) / 2;
    const bool chain = tid < D * nsub;
    const int col = tid % D, h0 = 2 * (tid / D);
    const bool two = h0 + 1 < G;
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int c = 0; c < nch; ++c) {
        const int slot = c % kAttnVtStages;
        wait_bar(slot);
        named_sync(bar, NT);  // chunk c landed everywhere (and, at c = 0, every p written)
        if (c < 4) attn_stamp_at(rec, 8 + 2 * c);
        if (*reinterpret_cast<volatile int *>(fail)) return drain();
        if (chain) {
            // groups of kPer positions: one 16-byte V load and kPer / 2
            // 16-byte p loads (2 positions of the head pair each) feed one
            // fused multiply-add per position and head, in order
            const uint8_t *vc = vt + slot * kStageBytes + col * kColStride;
            const float4 *pc = reinterpret_cast<const float4 *>(pp + (h0 / 2) * stride + c * kChunkPos);
            const int rows = min(kChunkPos, n - c * kChunkPos), full = rows / kPer * kPer;
            int t = 0;
#pragma unroll 4
            for (; t < full; t += kPer) {
                const uint4 vr = *reinterpret_cast<const uint4 *>(vc + t * ESZ);
                float4 pr[kPer / 2];
#pragma unroll
                for (int k = 0; k < kPer / 2; ++k) pr[k] = pc[t / 2 + k];
                float v[8];
                attn_seg_floats<ESZ>(vr, v);
#pragma unroll
                for (int k = 0; k < kPer / 2; ++k) {
                    acc0 = __fmaf_rn(v[2 * k], pr[k].x, acc0);
                    acc1 = __fmaf_rn(v[2 * k], pr[k].y, acc1);
                    acc0 = __fmaf_rn(v[2 * k + 1], pr[k].z, acc0);
                    acc1 = __fmaf_rn(v[2 * k + 1], pr[k].w, acc1);
                }
            }
            const float2 *pc2 = reinterpret_cast<const float2 *>(pc);
            for (; t < rows; ++t) {
                const float v = attn_elem<ESZ>(vc, t);
                const float2 p2 = pc2[t];
                acc0 = __fmaf_rn(v, p2.x, acc0);
                acc1 = __fmaf_rn(v, p2.y, acc1);
            }
        }
        named_sync(bar, NT);  // chunk c consumed
        if (c < 4) attn_stamp_at(rec, 9 + 2 * c);
        stage_vt(c + kAttnVtStages);
    }
    if (chain) {
        out[h0 * D + col] = acc0;
        if (two) out[(h0 + 1) * D + col] = acc1;
    }
    return true;
}

}  // namespace b200
