// Decode attention for one layer, bit-exact to the reference runtime's
// attention_group (board/tp/tp_llama.cpp:644-690) over this rank's heads.
//
// One CTA per local KV head, group * head_dim threads (the query heads that
// share the KV head, tp_llama.cpp:866-873). Phases, each in the reference's
// arithmetic order:
//   scores  one thread per position t: its K row (head_dim values, float16 or
//           float32) straight from global memory into registers, then per
//           query head four fused-multiply-add lanes (lane j takes i = j, j+4,
//           ...), combined as (a0 + a1) + (a2 + a3), times scale;
//   max     from -1e30f with `>`, as the reference's running max;
//   exp     s = v_expf(s - max), every position;
//   sum     lane j of each head adds positions j, j+4, ... < n - n%4 in
//           order, then (l0 + l1) + (l2 + l3), then the tail one by one
//           (softmax_exp, tp_llama.cpp:626-637); inv = 1 / sum;
//   p       p_t = s_t * inv;
//   output  thread (head, column c): acc = fmaf(v[t][c], p_t, acc) for
//           t = 0..pos in order -- a chain of pos + 1 fused multiply-adds, the
//           latency term of this kernel.
// V is streamed through a ring of 16 KB shared-memory chunks by 1-D bulk
// copies (no multicast) issued at the start, so it arrives while the scores
// are computed; threads of one head read consecutive columns of a V row.
#include <cuda_fp16.h>

#include "common.cuh"
#include "decode.cuh"
#include "decode.h"

namespace b200 {

namespace {

constexpr int kAttnChunkBytes = 16384;
constexpr int kAttnStages = 6;
constexpr int kAttnMaxThreads = 512;

struct AttnParams {
    const float *q;
    const uint8_t *kcache, *vcache;  // this layer: [kv head][ctx_max][head_dim]
    float *out;
    const int *pos;
    unsigned *status;
    int group, ctx_max;
    float scale;
};

template <int ESZ>
__device__ __forceinline__ float kv_elem(const uint8_t *row, int i) {
    if constexpr (ESZ == 2)
        return __half2float(reinterpret_cast<const __half *>(row)[i]);
    else
        return reinterpret_cast<const float *>(row)[i];
}

// x as 8 floats from a 16-byte segment (ESZ 2: 8 halves; ESZ 4: 4 floats in [0, 4)).
template <int ESZ>
__device__ __forceinline__ void seg_floats(const uint4 &v, float *f) {
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

// the reference's running max (`if (s > mx) mx = s`), as a combine
__device__ __forceinline__ float max_gt(float a, float b) { return b > a ? b : a; }

template <int D, int ESZ>
__global__ void __launch_bounds__(kAttnMaxThreads) attn_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    constexpr int kRowBytes = D * ESZ;
    constexpr int kSegs = kRowBytes / 16;
    constexpr int kTC = kAttnChunkBytes / kRowBytes;  // positions per V chunk
    constexpr int kPer = 16 / ESZ;                    // elements per segment
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + kAttnStages * kAttnChunkBytes);
    float *qs = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + 64);
    float *misc = qs + 4 * D;          // [0,128): warp maxima; [128,144): lane sums; [144,148): max; [148,152): inv
    float *sc = misc + 160;            // [group][ctx_max]
    const int tid = threadIdx.x, nt = blockDim.x, kvh = blockIdx.x, G = p.group;
    const int lane = tid % 32, warp = tid / 32, nwarps = nt / 32;

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kAttnStages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait_prior_grid();

    const int pos = *p.pos, n = pos + 1, nc = (n + kTC - 1) / kTC;
    const uint8_t *kb = p.kcache + static_cast<size_t>(kvh) * p.ctx_max * kRowBytes;
    const uint8_t *vb = p.vcache + static_cast<size_t>(kvh) * p.ctx_max * kRowBytes;
    const uint64_t policy = l2_policy_evict_normal();
    auto issue = [&](int c) {
        const int slot = c % kAttnStages;
        const int rows = min(kTC, n - c * kTC);
        const uint32_t bytes = static_cast<uint32_t>(rows * kRowBytes);
        mbar_arrive_expect_tx(&bars[slot], bytes);
        bulk_g2s(ring + slot * kAttnChunkBytes, vb + static_cast<size_t>(c) * kAttnChunkBytes, bytes, &bars[slot],
                 policy);
    };
    if (tid == 0)
        for (int c = 0; c < nc && c < kAttnStages; ++c) issue(c);
    for (int i = tid; i < G * D; i += nt) qs[i] = p.q[static_cast<size_t>(kvh) * G * D + i];
    __syncthreads();

    // scores (tp_llama.cpp:652-664)
    for (int t = tid; t < n; t += nt) {
        const uint4 *row = reinterpret_cast<const uint4 *>(kb + static_cast<size_t>(t) * kRowBytes);
        // element i of the row feeds lane i & 3 of every head, in increasing i
        float a[4][4];
#pragma unroll
        for (int b = 0; b < 4; ++b) a[b][0] = a[b][1] = a[b][2] = a[b][3] = 0.0f;
#pragma unroll
        for (int s = 0; s < kSegs; ++s) {
            float f[8];
            seg_floats<ESZ>(__ldcg(row + s), f);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                if (b < G) {
                    const float *qb = qs + b * D + s * kPer;
#pragma unroll
                    for (int e = 0; e < kPer; ++e) a[b][e & 3] = __fmaf_rn(f[e], qb[e], a[b][e & 3]);
                }
            }
        }
#pragma unroll
        for (int b = 0; b < 4; ++b)
            if (b < G)
                sc[b * p.ctx_max + t] =
                    __fmul_rn(__fadd_rn(__fadd_rn(a[b][0], a[b][1]), __fadd_rn(a[b][2], a[b][3])), p.scale);
    }
    __syncthreads();
    // running max per head, from -1e30f
    for (int b = 0; b < G; ++b) {
        float m = -1e30f;
        for (int t = tid; t < n; t += nt) m = max_gt(m, sc[b * p.ctx_max + t]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = max_gt(m, __shfl_xor_sync(kFullMask, m, off));
        if (lane == 0) misc[b * 32 + warp] = m;
    }
    __syncthreads();
    if (tid < G) {
        float m = -1e30f;
        for (int w = 0; w < nwarps; ++w) m = max_gt(m, misc[tid * 32 + w]);
        misc[144 + tid] = m;
    }
    __syncthreads();
    // exp (softmax_exp's values)
    for (int b = 0; b < G; ++b) {
        const float mx = misc[144 + b];
        for (int t = tid; t < n; t += nt) sc[b * p.ctx_max + t] = v_expf(__fsub_rn(sc[b * p.ctx_max + t], mx));
    }
    __syncthreads();
    // sums: four lanes per head over the first n - n%4 positions, in order
    const int n4 = n & ~3;
    if (tid < 4 * G) {
        const int b = tid / 4, j = tid % 4;
        const float *s = sc + b * p.ctx_max;
        float a = 0.0f;
#pragma unroll 8
        for (int t = j; t < n4; t += 4) a = __fadd_rn(a, s[t]);
        misc[128 + tid] = a;
    }
    __syncthreads();
    if (tid < G) {
        const float *l = misc + 128 + 4 * tid;
        float sum = __fadd_rn(__fadd_rn(l[0], l[1]), __fadd_rn(l[2], l[3]));
        for (int t = n4; t < n; ++t) sum = __fadd_rn(sum, sc[tid * p.ctx_max + t]);
        misc[148 + tid] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    // p_t = s_t * inv (tp_llama.cpp:680)
    for (int b = 0; b < G; ++b) {
        const float inv = misc[148 + b];
        for (int t = tid; t < n; t += nt) sc[b * p.ctx_max + t] = __fmul_rn(sc[b * p.ctx_max + t], inv);
    }
    __syncthreads();
    // output chains (tp_llama.cpp:676-687)
    const int b = tid / D, col = tid % D;
    const float *pb = sc + b * p.ctx_max;
    float acc = 0.0f;
    int c = 0;
    for (; c < nc; ++c) {
        const int slot = c % kAttnStages;
        if (!wait_stage(&bars[slot], static_cast<uint32_t>((c / kAttnStages) & 1), p.status)) s_abort = 1;
        __syncthreads();
        if (s_abort) break;
        const uint8_t *ch = ring + slot * kAttnChunkBytes;
        const int rows = min(kTC, n - c * kTC);
        const float *pc = pb + c * kTC;
#pragma unroll 8
        for (int t = 0; t < rows; ++t) acc = __fmaf_rn(kv_elem<ESZ>(ch + t * kRowBytes, col), pc[t], acc);
        __syncthreads();
        if (tid == 0 && c + kAttnStages < nc) issue(c + kAttnStages);
    }
    if (!s_abort) {
        p.out[(static_cast<size_t>(kvh) * G + b) * D + col] = acc;
    } else if (tid == 0) {
        // let copies in flight land (each wait bounded) before shared memory goes away
        for (int r = c; r < nc && r < c + kAttnStages; ++r)
            (void)wait_stage(&bars[r % kAttnStages], static_cast<uint32_t>((r / kAttnStages) & 1), p.status);
    }
}

using AttnFn = void (*)(AttnParams);

AttnFn pick_attn(int d, int kv_f16) {
    if (d == 64) return kv_f16 ? attn_kernel<64, 2> : attn_kernel<64, 4>;
    if (d == 128) return kv_f16 ? attn_kernel<128, 2> : attn_kernel<128, 4>;
    return nullptr;
}

}  // namespace

int attn_smem_bytes(int head_dim, int group, int ctx_max) {
    return 128 + kAttnStages * kAttnChunkBytes + 64 + 4 * (4 * head_dim + 160 + group * ctx_max);
}

int attn_launch(const AttnLaunch &L, cudaStream_t stream) {
    AttnFn fn = pick_attn(L.head_dim, L.kv_f16);
    if (!fn) return kErrInval;
    const int threads = L.group * L.head_dim;
    if (L.group < 1 || L.group > 4 || threads % 32 || threads > kAttnMaxThreads || L.kvh_local < 1 || L.ctx_max < 1)
        return kErrInval;
    if (!L.q || !L.kcache || !L.vcache || !L.out || !L.pos) return kErrInval;
    if (reinterpret_cast<uintptr_t>(L.kcache) % 16 || reinterpret_cast<uintptr_t>(L.vcache) % 16) return kErrInval;
    const int smem = attn_smem_bytes(L.head_dim, L.group, L.ctx_max);
    if (smem > max_smem_optin()) return kErrInval;
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
    p.ctx_max = L.ctx_max;
    p.scale = L.scale;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(L.kvh_local);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, p) == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
