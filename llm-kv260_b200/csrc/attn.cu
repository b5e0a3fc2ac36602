// Decode attention for one layer, bit-exact to the reference runtime's
// attention_group (board/tp/tp_llama.cpp:644-690) over this rank's heads:
// the per-op decoder's kernel. (The persistent kernel runs the single-CTA
// attn_core of attn_core.cuh; the arithmetic and its order are the same.)
//
// One thread-block cluster of kSplit CTAs per local KV head. CTA r of the
// cluster:
//   scores  the positions [r * per, (r + 1) * per) (per = ceil(n / kSplit)):
//           its K rows land in shared memory by one bulk copy (lane-major
//           rows, k_slot), one thread per position runs the four FMA lanes
//           of every head (q lane-major in shared memory too), and every
//           score row (4 heads) goes to every CTA of the cluster through
//           distributed shared memory; one cluster barrier;
//   softmax every CTA then holds all n scores and runs the reference's max,
//           v_expf, four-lane sums and 1 / sum itself -- the same operations
//           in the same order on the same values, so the same bits;
//   output  the columns [r * D / kSplit, (r + 1) * D / kSplit): their V^T
//           bytes land by one bulk copy per column, and one thread per
//           (column, head) runs the output's fused multiply-add chain over
//           t = 0..n-1 in order.
// Each CTA moves a kSplit-th of the head's K and V bytes and computes a
// kSplit-th of its scores: the single-CTA kernel was bound by one SM's
// ingest and shared-memory broadcasts. No TMA multicast: every copy is a
// plain 1-D bulk copy of this GPU's memory into this CTA's shared memory.
//
// Before the dependency wait, the last warp asks L2 for this CTA's K rows
// and V^T columns of the positions before the current one (a hint sized
// from a position read that may be one token stale; what is read after the
// wait is current either way). Every CTA reaches both cluster barriers on
// every path, failure included, and every mbarrier wait is bounded.
#include <cuda_fp16.h>

#include "attn_core.cuh"
#include "common.cuh"
#include "decode.h"

namespace b200 {

namespace {

constexpr int kAttnThreads = 256;
constexpr int kSplit = 4;  // CTAs per KV head: the cluster size

struct AttnParams {
    const float *q;
    const uint8_t *kcache, *vcache;  // this layer: K [kv head][stride][D] (swizzled), V^T [kv head][D][stride]
    float *out;
    const int *pos;
    unsigned *status;
    int group, stride, ctx_max;
    float scale;
    uint64_t *trace;  // optional launch trace (q4gemv.h, kTraceCtas)
};

// Shared-memory layout of one CTA (byte offsets, 16-byte aligned pieces).
struct AttnSmem {
    int kbuf, vt, qs, part, hinv, e, pv, total;
    int slice_rows;  // K rows a CTA stages at most
    int col_stride;  // bytes between two V^T columns: an odd number of 16-byte units
};

__host__ __device__ inline AttnSmem attn_smem_layout(int d, int esz, int stride) {
    AttnSmem L{};
    const int cw = d / kSplit;
    L.slice_rows = (stride + kSplit - 1) / kSplit;
    L.col_stride = ((stride * esz / 16) | 1) * 16;
    int off = 0;
    auto carve = [&](int bytes) {
        const int at = off;
        off += (bytes + 15) / 16 * 16;
        return at;
    };
    L.kbuf = carve(L.slice_rows * d * esz);
    L.vt = carve(cw * L.col_stride);
    L.qs = carve(4 * d * 4);
    L.part = carve((kAttnThreads / 32) * 16);
    L.hinv = carve(32);
    L.e = carve(16 * stride);
    L.pv = carve(16 * stride);
    L.total = off;
    return L;
}

__device__ __forceinline__ uint64_t *attn_rec(uint64_t *trace) {
    return (trace && blockIdx.x < kTraceCtas) ? trace + blockIdx.x * kTraceStamps : nullptr;
}

template <int D, int ESZ>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_kernel(const __grid_constant__ AttnParams p) {
    constexpr int kRowBytes = D * ESZ;
    constexpr int kSegs = kRowBytes / 16;
    constexpr int kPer = 16 / ESZ;  // elements per 16 bytes
    constexpr int CW = D / kSplit;  // output columns per CTA
    constexpr int L = kSegs / 4, M = D / 4;  // per FMA lane: K segments, steps
    constexpr int kQv = (4 * D + kAttnThreads - 1) / kAttnThreads;
    static_assert(kSegs % 8 == 0 && kPer % 4 == 0 && 4 * CW <= kAttnThreads, "attention shape");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[2];  // 0: this CTA's V^T columns, 1: its K rows
    __shared__ int s_fail;
    const AttnSmem S = attn_smem_layout(D, ESZ, p.stride);
    uint8_t *kbuf = smem + S.kbuf, *vt = smem + S.vt;
    float *qs = reinterpret_cast<float *>(smem + S.qs);  // [head][lane j][step m]: element 4m + j
    float *part = reinterpret_cast<float *>(smem + S.part);
    float *hinv = reinterpret_cast<float *>(smem + S.hinv);
    float4 *e = reinterpret_cast<float4 *>(smem + S.e);  // [position]: the 4 heads' scores, then exponentials
    float *pv = reinterpret_cast<float *>(smem + S.pv);   // [head][position]: p
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = p.group;
    const int kvh = blockIdx.x / kSplit;
    const int r = static_cast<int>(cluster_ctarank());
    const int c0 = r * CW;
    const size_t head_bytes = static_cast<size_t>(p.stride) * D * ESZ;
    const uint8_t *kb = p.kcache + kvh * head_bytes;
    const uint8_t *vtb = p.vcache + kvh * head_bytes;  // column c at c * stride * ESZ
    uint64_t *rec = attn_rec(p.trace);
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
        s_fail = 0;
    }
    __syncthreads();
    pdl_launch_dependents();
    attn_stamp_at(rec, 0);
    if (tid >= kAttnThreads - 32) {  // L2 hint: this CTA's K rows and V^T columns, earlier positions
        int hint = *reinterpret_cast<const volatile int *>(p.pos) + 2;  // may be a token behind
        hint = hint < 1 ? 1 : (hint > p.ctx_max ? p.ctx_max : hint);
        const int hp = (hint + kSplit - 1) / kSplit, h0 = min(hint, r * hp), h1 = min(hint, h0 + hp);
        if (lane == 0 && h1 > h0)
            bulk_prefetch_l2(kb + static_cast<size_t>(h0) * kRowBytes, static_cast<uint32_t>((h1 - h0) * kRowBytes));
        const uint32_t hb = static_cast<uint32_t>((hint * ESZ + 15) / 16 * 16);
        for (int j = lane; j < CW; j += 32) bulk_prefetch_l2(vtb + static_cast<size_t>(c0 + j) * p.stride * ESZ, hb);
    }
    cluster_sync_all();  // every CTA of the cluster runs before any store into its shared memory
    pdl_wait_prior_grid();
    attn_stamp_at(rec, 1);

    const int n = *p.pos + 1;
    const int per = (n + kSplit - 1) / kSplit;
    const int r0 = min(n, r * per), r1 = min(n, r0 + per);
    const bool krows = r1 > r0;
    const uint64_t pol = l2_policy_evict_last();  // the KV cache stays in L2 while the weights stream past
    // q first (on the critical path), then this CTA's K rows in one copy
    float qv[kQv];
#pragma unroll
    for (int u = 0; u < kQv; ++u) {
        const int i = tid + u * kAttnThreads;
        if (i < G * D) qv[u] = __ldcg(p.q + static_cast<size_t>(kvh) * G * D + i);
    }
    if (tid == 0 && krows) {
        const uint32_t kbytes = static_cast<uint32_t>((r1 - r0) * kRowBytes);
        mbar_arrive_expect_tx(&bars[1], kbytes);
        bulk_g2s(kbuf, kb + static_cast<size_t>(r0) * kRowBytes, kbytes, &bars[1], pol);
    }
#pragma unroll
    for (int u = 0; u < kQv; ++u) {
        const int i = tid + u * kAttnThreads;
        if (i < G * D) qs[(i / D) * D + (i & 3) * M + (i % D) / 4] = qv[u];
    }
    __syncthreads();
    attn_stamp_at(rec, 4);
    // this CTA's V^T columns, positions [0, n): one copy per column (rounded
    // up to 16 bytes, which stays below stride: stride % 8 == 0)
    const uint32_t colb = static_cast<uint32_t>((n * ESZ + 15) / 16 * 16);
    if (tid == 0) mbar_arrive_expect_tx(&bars[0], colb * CW);
    if (tid < CW)
        bulk_g2s(vt + tid * S.col_stride, vtb + static_cast<size_t>(c0 + tid) * p.stride * ESZ, colb, &bars[0], pol);

    // scores of positions [r0, r1) (tp_llama.cpp:652-664), to every CTA
    if (krows && !wait_stage(&bars[1], 0u, p.status)) atomicExch(&s_fail, 1);
    for (int t = r0 + tid; t < r1; t += kAttnThreads) {
        const uint8_t *row = kbuf + (t - r0) * kRowBytes;
        const int sw = t & 7;
        float a[4][4];
#pragma unroll
        for (int b = 0; b < 4; ++b) a[b][0] = a[b][1] = a[b][2] = a[b][3] = 0.0f;
#pragma unroll
        for (int s8 = 0; s8 < kSegs; s8 += 8) {
            // logical segments s8 .. s8 + 7, loaded in an order that puts the
            // lanes (8 consecutive positions) on distinct bank groups
            const int g = 2 * ((s8 >> 3) & 3);
            uint4 kr[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) kr[j] = *reinterpret_cast<const uint4 *>(row + (s8 + (j ^ sw ^ g)) * 16);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                // logical segment s: FMA lane s / L, steps (s % L) * kPer ..
                const int sg = s8 + j, ln = sg / L, m0 = (sg % L) * kPer;
                float f[8];
                attn_seg_floats<ESZ>(kr[j], f);
                // the segment's q of all four heads loaded together, then the
                // FMAs (qs holds 4 heads; a head past G is computed, never used)
                float4 qv4[4][kPer / 4];
#pragma unroll
                for (int b = 0; b < 4; ++b)
#pragma unroll
                    for (int m4 = 0; m4 < kPer; m4 += 4)
                        qv4[b][m4 / 4] = *reinterpret_cast<const float4 *>(qs + b * D + ln * M + m0 + m4);
#pragma unroll
                for (int b = 0; b < 4; ++b) {
#pragma unroll
                    for (int u = 0; u < kPer; ++u) {
                        const float4 q4 = qv4[b][u / 4];
                        const float qu = (u & 3) == 0 ? q4.x : (u & 3) == 1 ? q4.y : (u & 3) == 2 ? q4.z : q4.w;
                        a[b][ln] = __fmaf_rn(f[u], qu, a[b][ln]);
                    }
                }
            }
        }
        float sv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int b = 0; b < 4; ++b)
            if (b < G) sv[b] = __fmul_rn(__fadd_rn(__fadd_rn(a[b][0], a[b][1]), __fadd_rn(a[b][2], a[b][3])), p.scale);
        const float4 s4 = make_float4(sv[0], sv[1], sv[2], sv[3]);
#pragma unroll
        for (int q = 0; q < kSplit; ++q) st_cluster_f4(cluster_map(&e[t], static_cast<uint32_t>(q)), s4);
    }
    cluster_sync_all();  // every CTA now holds all n scores
    attn_stamp_at(rec, 5);

    // running max per head over all positions (exact, so any tree of `>`
    // gives the reference's value), then the exponentials
    float mx[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
    for (int t = tid; t < n; t += kAttnThreads) {
        const float4 s = e[t];
        mx[0] = attn_max_gt(mx[0], s.x);
        mx[1] = attn_max_gt(mx[1], s.y);
        mx[2] = attn_max_gt(mx[2], s.z);
        mx[3] = attn_max_gt(mx[3], s.w);
    }
    // the four heads' reductions interleaved (a head past G is never read)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int b = 0; b < 4; ++b) mx[b] = attn_max_gt(mx[b], __shfl_xor_sync(kFullMask, mx[b], off));
    }
    if (lane == 0) *reinterpret_cast<float4 *>(part + warp * 4) = make_float4(mx[0], mx[1], mx[2], mx[3]);
    __syncthreads();
    float m[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
    for (int w = 0; w < kAttnThreads / 32; ++w) {
        const float4 pw = *reinterpret_cast<const float4 *>(part + w * 4);
        m[0] = attn_max_gt(m[0], pw.x);
        m[1] = attn_max_gt(m[1], pw.y);
        m[2] = attn_max_gt(m[2], pw.z);
        m[3] = attn_max_gt(m[3], pw.w);
    }
    for (int t = tid; t < n; t += kAttnThreads) {
        float4 s = e[t];
        s.x = v_expf(__fsub_rn(s.x, m[0]));
        if (G > 1) s.y = v_expf(__fsub_rn(s.y, m[1]));
        if (G > 2) s.z = v_expf(__fsub_rn(s.z, m[2]));
        if (G > 3) s.w = v_expf(__fsub_rn(s.w, m[3]));
        e[t] = s;
    }
    __syncthreads();
    attn_stamp_at(rec, 6);

    // sums (softmax_exp, tp_llama.cpp:626-633): warp 0, lane 4 * head + j
    // adds positions j, j+4, ... below n - n % 4 in order; (l0 + l1) + (l2 + l3)
    // by two xor shuffles; then the tail one by one; inv = 1 / sum
    if (warp == 0) {
        const int b = lane >> 2, j4 = lane & 3, n4 = n & ~3;
        const float *col = reinterpret_cast<const float *>(e) + b;
        float acc = 0.0f;
        if (b < G) {
#pragma unroll 16
            for (int t = j4; t < n4; t += 4) acc = __fadd_rn(acc, col[4 * t]);
        }
        const float x = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, 1));
        const float y = __fadd_rn(x, __shfl_xor_sync(kFullMask, x, 2));
        if (b < G && j4 == 0) {
            float sum = y;
            for (int t = n4; t < n; ++t) sum = __fadd_rn(sum, col[4 * t]);
            hinv[b] = __frcp_rn(sum);  // IEEE 1 / sum, round to nearest: the reference's 1.0f / sum
        }
    }
    __syncthreads();
    attn_stamp_at(rec, 7);

    // p_t = s_t * inv (tp_llama.cpp:680), per head contiguous
    {
        const float4 iv = *reinterpret_cast<const float4 *>(hinv);
        for (int t = tid; t < n; t += kAttnThreads) {
            const float4 s = e[t];
            pv[t] = __fmul_rn(s.x, iv.x);
            if (G > 1) pv[p.stride + t] = __fmul_rn(s.y, iv.y);
            if (G > 2) pv[2 * p.stride + t] = __fmul_rn(s.z, iv.z);
            if (G > 3) pv[3 * p.stride + t] = __fmul_rn(s.w, iv.w);
        }
    }
    if (!wait_stage(&bars[0], 0u, p.status)) atomicExch(&s_fail, 1);
    __syncthreads();  // every p written, this CTA's V^T columns landed
    attn_stamp_at(rec, 2);

    // output chains (tp_llama.cpp:667-687): thread (column c0 + j, head h),
    // acc = fma(v[t][c], p_t, acc) for t = 0..n-1 in order
    const int j = tid % CW, h = tid / CW;
    if (h < G && !s_fail) {
        const uint8_t *vc = vt + j * S.col_stride;
        const float *ph = pv + h * p.stride;
        const int full = n / kPer * kPer;
        float acc = 0.0f;
        int t = 0;
#pragma unroll 8
        for (; t < full; t += kPer) {
            const uint4 vr = *reinterpret_cast<const uint4 *>(vc + t * ESZ);
            float v[8];
            attn_seg_floats<ESZ>(vr, v);
#pragma unroll
            for (int k4 = 0; k4 < kPer; k4 += 4) {
                const float4 p4 = *reinterpret_cast<const float4 *>(ph + t + k4);
                acc = __fmaf_rn(v[k4], p4.x, acc);
                acc = __fmaf_rn(v[k4 + 1], p4.y, acc);
                acc = __fmaf_rn(v[k4 + 2], p4.z, acc);
                acc = __fmaf_rn(v[k4 + 3], p4.w, acc);
            }
        }
        for (; t < n; ++t) acc = __fmaf_rn(attn_elem<ESZ>(vc, t), ph[t], acc);
        p.out[(static_cast<size_t>(kvh) * G + h) * D + c0 + j] = acc;
    }
    if (s_fail) {
        // a copy wait ran out: let this CTA's copies in flight land (each
        // wait bounded) before its shared memory goes away
        if (tid == 0) {
            if (krows) (void)wait_stage(&bars[1], 0u, p.status);
            (void)wait_stage(&bars[0], 0u, p.status);
        }
        __syncthreads();
    }
    if (rec) {
        __syncthreads();
        attn_stamp_at(rec, 3);
    }
}

// Long contexts, cluster form: the cluster kernel's split over kStreamSplit
// CTAs per KV head (CTA r scores an eighth of the positions and chains an
// eighth of the columns) with K and V^T streamed through rings of
// shared-memory stages instead of held whole.
//   scores  4 threads per position (fused-multiply-add lane j each: q's
//           elements j, j+4, ... of every head in registers, the lane's
//           quarter of the lane-major K row from the ring; met by xor
//           shuffles 1 then 2: vaddvq_f32's pairing); every score row to all
//           the cluster's CTAs (distributed shared memory); one cluster
//           barrier;
//   softmax each CTA: maxima, v_expf, the four sequential lane sums per head
//           read from a lane-major copy of the exponentials, 1 / sum, p;
//   output  one thread per (column, head): the fused-multiply-add chain over
//           t = 0..n-1 in order, chunk by chunk.
// The V^T ring reuses the K ring's shared memory and starts filling as soon
// as the scores are done, behind the softmax.
constexpr int kStreamThreads = 256;
constexpr int kStreamSplit = 8;  // CTAs per KV head at long contexts: the cluster size (the portable maximum)
constexpr int kStreamKStages = 4;
constexpr int kStreamVStages = 3;
constexpr int kStreamColBytes = 512;  // V^T bytes of a column per stage

struct StreamSmem {
    int e, pt, ring, qs, part, hinv, total;
    int krows;     // K rows per stage
    int vcol;      // bytes between two V^T columns of a stage (odd number of 16-byte units)
    int vstage;    // bytes of a V^T stage
    int ptq;       // floats between two lane rows of the lane-major exponentials (= 8 mod 32)
};

__host__ __device__ inline StreamSmem stream_smem_layout(int d, int esz, int stride) {
    StreamSmem L{};
    L.krows = 16384 / (d * esz);  // 16 KB per K stage
    L.vcol = kStreamColBytes + 16;
    L.vstage = (d / kStreamSplit) * L.vcol;
    const int kring = kStreamKStages * L.krows * d * esz, vring = kStreamVStages * L.vstage;
    int off = 0;
    auto carve = [&](int bytes) {
        const int at = off;
        off += (bytes + 15) / 16 * 16;
        return at;
    };
    // lane rows of the exponentials ptq = 8 (mod 32) floats apart: the four
    // lanes' stores of 8 consecutive row entries fall on 32 distinct banks
    // (rows stay 16-byte aligned for the sums' loads)
    const int q4 = stride / 4;
    L.ptq = q4 + ((8 - q4 % 32) + 32) % 32;
    const int lanes_bytes = 16 * L.ptq * 4;
    L.e = carve(16 * stride);
    L.pt = carve(lanes_bytes > 16 * stride ? lanes_bytes : 16 * stride);
    L.ring = carve(kring > vring ? kring : vring);
    L.qs = carve(4 * d * 4);
    L.part = carve((kStreamThreads / 32) * 16);
    L.hinv = carve(32);
    L.total = off;
    return L;
}

template <int D, int ESZ>
__global__ void __launch_bounds__(kStreamThreads, 1) attn_stream_kernel(const __grid_constant__ AttnParams p) {
    constexpr int kRowBytes = D * ESZ;
    constexpr int kSegs = kRowBytes / 16;
    constexpr int kPer = 16 / ESZ;
    constexpr int CW = D / kStreamSplit;
    constexpr int kChunkPos = kStreamColBytes / ESZ;  // positions per V^T stage
    constexpr int NT = kStreamThreads;
    constexpr int kQv = (4 * D + NT - 1) / NT;
    static_assert(kSegs % 8 == 0 && kPer % 4 == 0 && 4 * CW <= NT, "attention shape");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t kbar[kStreamKStages], vbar[kStreamVStages];
    __shared__ int s_fail;
    const StreamSmem S = stream_smem_layout(D, ESZ, p.stride);
    float4 *e = reinterpret_cast<float4 *>(smem + S.e);   // [position]: 4 heads' scores, then exponentials
    float *pt = reinterpret_cast<float *>(smem + S.pt);    // exponentials lane-major, then p [head][position]
    uint8_t *ring = smem + S.ring;
    float *qs = reinterpret_cast<float *>(smem + S.qs);
    float *part = reinterpret_cast<float *>(smem + S.part);
    float *hinv = reinterpret_cast<float *>(smem + S.hinv);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = p.group, KC = S.krows;
    const int kvh = blockIdx.x / kStreamSplit;
    const int r = static_cast<int>(cluster_ctarank());
    const int c0 = r * CW;
    const size_t head_bytes = static_cast<size_t>(p.stride) * D * ESZ;
    const uint8_t *kb = p.kcache + kvh * head_bytes;
    const uint8_t *vtb = p.vcache + kvh * head_bytes;
    uint64_t *rec = attn_rec(p.trace);
    if (tid == 0) {
        for (int i = 0; i < kStreamKStages; ++i) mbar_init(&kbar[i], 1);
        for (int i = 0; i < kStreamVStages; ++i) mbar_init(&vbar[i], 1);
        fence_mbar_init();
        s_fail = 0;
    }
    __syncthreads();
    pdl_launch_dependents();
    attn_stamp_at(rec, 0);
    cluster_sync_all();  // every CTA of the cluster runs before any store into its shared memory
    pdl_wait_prior_grid();
    attn_stamp_at(rec, 1);

    const int n = *p.pos + 1;
    const int per = (n + kStreamSplit - 1) / kStreamSplit;
    const int r0 = min(n, r * per), r1 = min(n, r0 + per);
    const int nk = (r1 - r0 + KC - 1) / KC;
    const int nv = (n + kChunkPos - 1) / kChunkPos;
    const uint64_t pol = l2_policy_evict_last();
    auto stage_k = [&](int kc) {  // K rows [r0 + kc * KC, ...) into stage kc % KS (thread 0)
        if (kc >= nk) return;
        const int a = r0 + kc * KC, rows = min(KC, r1 - a), st = kc % kStreamKStages;
        const uint32_t bytes = static_cast<uint32_t>(rows * kRowBytes);
        mbar_arrive_expect_tx(&kbar[st], bytes);
        bulk_g2s(ring + st * KC * kRowBytes, kb + static_cast<size_t>(a) * kRowBytes, bytes, &kbar[st], pol);
    };
    auto stage_v = [&](int c) {  // V^T positions [c * CP, ...) of this CTA's columns into stage c % VS (threads < CW)
        if (c >= nv) return;
        const int rows = min(kChunkPos, n - c * kChunkPos), st = c % kStreamVStages;
        const uint32_t colb = static_cast<uint32_t>((rows * ESZ + 15) / 16 * 16);  // stays below stride: stride % 8 == 0
        if (tid == 0) mbar_arrive_expect_tx(&vbar[st], colb * CW);
        __syncwarp();
        if (tid < CW)
            bulk_g2s(ring + st * S.vstage + tid * S.vcol,
                     vtb + static_cast<size_t>(c0 + tid) * p.stride * ESZ + static_cast<size_t>(c) * kStreamColBytes, colb,
                     &vbar[st], pol);
    };
    // q first (the critical path), then the first K stages
    float qv[kQv];
#pragma unroll
    for (int u = 0; u < kQv; ++u) {
        const int i = tid + u * NT;
        if (i < G * D) qv[u] = __ldcg(p.q + static_cast<size_t>(kvh) * G * D + i);
    }
    if (tid == 0)
        for (int kc = 0; kc < kStreamKStages; ++kc) stage_k(kc);
#pragma unroll
    for (int u = 0; u < kQv; ++u) {
        const int i = tid + u * NT;
        if (i < G * D) qs[i] = qv[u];
    }
    __syncthreads();
    attn_stamp_at(rec, 4);

    // scores of positions [r0, r1) (tp_llama.cpp:652-664), to every CTA:
    // four threads per position, thread jl running FMA lane jl of every
    // head -- its q elements jl, jl+4, ... held in registers, its quarter of
    // the lane-major K row (k_slot) read as L 16-byte segments
    const int jl = tid & 3;
    constexpr int L = kSegs / 4, M = D / 4;
    float qr[4][M];
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int m = 0; m < M; ++m) qr[b][m] = b < G ? qs[b * D + 4 * m + jl] : 0.0f;
    for (int kc = 0; kc < nk; ++kc) {
        const int a0 = r0 + kc * KC, a1 = min(r1, a0 + KC), st = kc % kStreamKStages;
        if (!s_fail && !wait_stage(&kbar[st], static_cast<uint32_t>((kc / kStreamKStages) & 1), p.status))
            atomicExch(&s_fail, 1);
        const uint8_t *kst = ring + st * KC * kRowBytes;
        for (int t0 = a0; t0 < a1; t0 += NT / 4) {  // the same trip count in every thread
            const int t = t0 + (tid >> 2);
            const bool live = t < a1;
            const uint8_t *row = kst + (live ? t - a0 : 0) * kRowBytes;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
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
                        for (int u = 0; u < kPer; ++u) acc[b] = __fmaf_rn(f[u], qr[b][i * kPer + u], acc[b]);
                    }
                }
            }
            float sv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float x = __fadd_rn(acc[b], __shfl_xor_sync(kFullMask, acc[b], 1));
                if (b < G) sv[b] = __fmul_rn(__fadd_rn(x, __shfl_xor_sync(kFullMask, x, 2)), p.scale);
            }
            if (live)  // the four lanes hold the same row: lane j writes the copies of CTAs j, j + 4, ...
                for (int q = jl; q < kStreamSplit; q += 4)
                    st_cluster_f4(cluster_map(&e[t], static_cast<uint32_t>(q)), make_float4(sv[0], sv[1], sv[2], sv[3]));
        }
        __syncthreads();  // stage consumed
        if (tid == 0) stage_k(kc + kStreamKStages);
    }
    // the K ring is done: the V^T stages fill it behind the softmax
    if (!s_fail)
        for (int c = 0; c < kStreamVStages; ++c) stage_v(c);
    cluster_sync_all();  // every CTA now holds all n scores
    attn_stamp_at(rec, 5);

    // running max per head over all positions (exact: any tree of `>` gives
    // the reference's value), then the exponentials -- into e, and lane-major
    // into pt for the sums: exponential of position 4u + j, head b at
    // pt[(4 b + j) * (stride / 4) + u]
    float mx[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
    for (int t = tid; t < n; t += NT) {
        const float4 sc = e[t];
        mx[0] = attn_max_gt(mx[0], sc.x);
        mx[1] = attn_max_gt(mx[1], sc.y);
        mx[2] = attn_max_gt(mx[2], sc.z);
        mx[3] = attn_max_gt(mx[3], sc.w);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
        for (int b = 0; b < 4; ++b) mx[b] = attn_max_gt(mx[b], __shfl_xor_sync(kFullMask, mx[b], off));
    }
    if (lane == 0) *reinterpret_cast<float4 *>(part + warp * 4) = make_float4(mx[0], mx[1], mx[2], mx[3]);
    __syncthreads();
    float m[4] = {-1e30f, -1e30f, -1e30f, -1e30f};
    for (int w = 0; w < NT / 32; ++w) {
        const float4 pw = *reinterpret_cast<const float4 *>(part + w * 4);
        m[0] = attn_max_gt(m[0], pw.x);
        m[1] = attn_max_gt(m[1], pw.y);
        m[2] = attn_max_gt(m[2], pw.z);
        m[3] = attn_max_gt(m[3], pw.w);
    }
    const int q4 = S.ptq;
    for (int t = tid; t < n; t += NT) {
        float4 sc = e[t];
        sc.x = v_expf(__fsub_rn(sc.x, m[0]));
        if (G > 1) sc.y = v_expf(__fsub_rn(sc.y, m[1]));
        if (G > 2) sc.z = v_expf(__fsub_rn(sc.z, m[2]));
        if (G > 3) sc.w = v_expf(__fsub_rn(sc.w, m[3]));
        e[t] = sc;
        const int j = t & 3, u = t >> 2;
        pt[(0 + j) * q4 + u] = sc.x;
        pt[(4 + j) * q4 + u] = sc.y;
        pt[(8 + j) * q4 + u] = sc.z;
        pt[(12 + j) * q4 + u] = sc.w;
    }
    __syncthreads();
    attn_stamp_at(rec, 6);

    // sums (softmax_exp, tp_llama.cpp:626-633): warp 0, lane 4 * head + j
    // adds positions j, j+4, ... below n - n % 4 in order, reading its lane's
    // row of pt 16 bytes at a time; (l0 + l1) + (l2 + l3) by two xor
    // shuffles; then the tail one by one; inv = 1 / sum
    if (warp == 0) {
        const int b = lane >> 2, j4 = lane & 3, n4 = n & ~3, nu = n4 / 4;
        const float *row = pt + (4 * b + j4) * q4;
        float acc = 0.0f;
        if (b < G) {
            // rows are 16-byte aligned (ptq % 4 == 0); each group's four
            // values are loaded while the previous group's adds run
            int u = 0;
            if (nu >= 4) {
                float4 cur = *reinterpret_cast<const float4 *>(row);
#pragma unroll 4
                for (; u + 8 <= nu; u += 4) {
                    const float4 nxt = *reinterpret_cast<const float4 *>(row + u + 4);
                    acc = __fadd_rn(acc, cur.x);
                    acc = __fadd_rn(acc, cur.y);
                    acc = __fadd_rn(acc, cur.z);
                    acc = __fadd_rn(acc, cur.w);
                    cur = nxt;
                }
                acc = __fadd_rn(acc, cur.x);
                acc = __fadd_rn(acc, cur.y);
                acc = __fadd_rn(acc, cur.z);
                acc = __fadd_rn(acc, cur.w);
                u += 4;
            }
            for (; u < nu; ++u) acc = __fadd_rn(acc, row[u]);
        }
        const float x = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, 1));
        const float y = __fadd_rn(x, __shfl_xor_sync(kFullMask, x, 2));
        if (b < G && j4 == 0) {
            float sum = y;
            const float *col = reinterpret_cast<const float *>(e) + b;
            for (int t = n4; t < n; ++t) sum = __fadd_rn(sum, col[4 * t]);
            hinv[b] = __frcp_rn(sum);  // IEEE 1 / sum, round to nearest: the reference's 1.0f / sum
        }
    }
    __syncthreads();
    attn_stamp_at(rec, 7);
    // p_t = s_t * inv (tp_llama.cpp:680), per head contiguous (over pt: the sums are done)
    {
        const float4 iv = *reinterpret_cast<const float4 *>(hinv);
        for (int t = tid; t < n; t += NT) {
            const float4 sc = e[t];
            pt[t] = __fmul_rn(sc.x, iv.x);
            if (G > 1) pt[p.stride + t] = __fmul_rn(sc.y, iv.y);
            if (G > 2) pt[2 * p.stride + t] = __fmul_rn(sc.z, iv.z);
            if (G > 3) pt[3 * p.stride + t] = __fmul_rn(sc.w, iv.w);
        }
    }
    __syncthreads();
    attn_stamp_at(rec, 2);

    // output chains (tp_llama.cpp:667-687): thread (column c0 + j, head h),
    // acc = fma(v[t][c], p_t, acc) for t = 0..n-1 in order, stage by stage
    const int j = tid % CW, h = tid / CW;
    const bool chain = h < G;
    float acc = 0.0f;
    for (int c = 0; c < nv; ++c) {
        const int st = c % kStreamVStages;
        if (!s_fail && !wait_stage(&vbar[st], static_cast<uint32_t>((c / kStreamVStages) & 1), p.status))
            atomicExch(&s_fail, 1);
        if (chain && !s_fail) {
            const uint8_t *vc = ring + st * S.vstage + j * S.vcol;
            const float *ph = pt + h * p.stride + c * kChunkPos;
            const int rows = min(kChunkPos, n - c * kChunkPos), full = rows / kPer * kPer;
            int t = 0;
#pragma unroll 8
            for (; t < full; t += kPer) {
                const uint4 vr = *reinterpret_cast<const uint4 *>(vc + t * ESZ);
                float v[8];
                attn_seg_floats<ESZ>(vr, v);
#pragma unroll
                for (int k4 = 0; k4 < kPer; k4 += 4) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(ph + t + k4);
                    acc = __fmaf_rn(v[k4], p4.x, acc);
                    acc = __fmaf_rn(v[k4 + 1], p4.y, acc);
                    acc = __fmaf_rn(v[k4 + 2], p4.z, acc);
                    acc = __fmaf_rn(v[k4 + 3], p4.w, acc);
                }
            }
            for (; t < rows; ++t) acc = __fmaf_rn(attn_elem<ESZ>(vc, t), ph[t], acc);
        }
        __syncthreads();  // stage consumed
        if (!s_fail) stage_v(c + kStreamVStages);
    }
    if (chain && !s_fail) p.out[(static_cast<size_t>(kvh) * G + h) * D + c0 + j] = acc;
    if (s_fail && tid == 0) {
        // a wait ran out: let this CTA's copies in flight land (each wait
        // bounded) before its shared memory goes away
        for (int i = 0; i < kStreamKStages; ++i) (void)wait_stage(&kbar[i], 0u, p.status), (void)wait_stage(&kbar[i], 1u, p.status);
        for (int i = 0; i < kStreamVStages; ++i) (void)wait_stage(&vbar[i], 0u, p.status), (void)wait_stage(&vbar[i], 1u, p.status);
    }
    __syncthreads();
    attn_stamp_at(rec, 3);
}

using AttnFn = void (*)(AttnParams);

AttnFn pick_attn_stream(int d, int kv_f16) {
    if (d == 64) return kv_f16 ? attn_stream_kernel<64, 2> : attn_stream_kernel<64, 4>;
    if (d == 128) return kv_f16 ? attn_stream_kernel<128, 2> : attn_stream_kernel<128, 4>;
    return nullptr;
}

AttnFn pick_attn(int d, int kv_f16) {
    if (d == 64) return kv_f16 ? attn_kernel<64, 2> : attn_kernel<64, 4>;
    if (d == 128) return kv_f16 ? attn_kernel<128, 2> : attn_kernel<128, 4>;
    return nullptr;
}

}  // namespace

int attn_kv_stride(int ctx_max) { return (ctx_max + 7) / 8 * 8; }

int attn_smem_bytes(int head_dim, int kv_f16, int ctx_max) {
    return attn_smem_layout(head_dim, kv_f16 ? 2 : 4, attn_kv_stride(ctx_max)).total;
}

int attn_smem_bytes_long(int head_dim, int kv_f16, int ctx_max) {
    return stream_smem_layout(head_dim, kv_f16 ? 2 : 4, attn_kv_stride(ctx_max)).total;
}

int attn_launch(const AttnLaunch &L, cudaStream_t stream) {
    AttnFn fn = pick_attn(L.head_dim, L.kv_f16);
    if (!fn) return kErrInval;
    if (L.group < 1 || L.group > 4 || L.kvh_local < 1 || L.ctx_max < 1 || L.kv_stride != attn_kv_stride(L.ctx_max))
        return kErrInval;
    if (!L.q || !L.kcache || !L.vcache || !L.out || !L.pos) return kErrInval;
    if (reinterpret_cast<uintptr_t>(L.kcache) % 16 || reinterpret_cast<uintptr_t>(L.vcache) % 16) return kErrInval;
    int smem = attn_smem_bytes(L.head_dim, L.kv_f16, L.ctx_max);
    const bool long_ctx = smem > max_smem_optin();  // the cluster's slices do not fit: the streaming kernel
    if (long_ctx) {
        fn = pick_attn_stream(L.head_dim, L.kv_f16);
        smem = attn_smem_bytes_long(L.head_dim, L.kv_f16, L.ctx_max);
        if (smem > max_smem_optin()) return kErrInval;
    }
    if (!ensure_smem(reinterpret_cast<const void *>(fn), smem)) return kErrCuda;
    AttnParams p{};
    p.q = L.q;
    p.kcache = static_cast<const uint8_t *>(L.kcache);
    p.vcache = static_cast<const uint8_t *>(L.vcache);
    p.out = L.out;
    p.pos = L.pos;
    p.status = status_word();
    if (!p.status) return kErrNoDev;
    p.group = L.group;
    p.stride = L.kv_stride;
    p.ctx_max = L.ctx_max;
    p.scale = L.scale;
    p.trace = L.trace;
    cudaLaunchConfig_t cfg{};
    const int split = long_ctx ? kStreamSplit : kSplit;
    cfg.gridDim = dim3(L.kvh_local * split);
    cfg.blockDim = dim3(long_ctx ? kStreamThreads : kAttnThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;  // the CTAs of one KV head, scheduled together
    attr[0].val.clusterDim.x = split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, fn, p) == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
