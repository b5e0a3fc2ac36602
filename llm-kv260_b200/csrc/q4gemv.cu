// Q4_0 x Q8_0 GEMV for sm_100a, bit-exact to the reference contract
// src/llm_kv260/q4_0.py (gemv_q4_0, lines 151-182).
//
// Data path (one CTA, 256 threads):
//   * The CTA owns a contiguous range of weight units (a row, or a gemv2 row
//     pair) inside one region. One elected thread streams that byte range into
//     a ring of shared-memory stages with 1-D bulk copies (cp.async.bulk, the
//     TMA engine) that complete on mbarriers, so each CTA keeps up to
//     `stages` x ~16 KB in flight with no registers tied up in loads.
//   * x is read once per CTA into registers: every thread always handles the
//     same blocks b = t, t+T, t+2T, ... of every row, so its 8 int8x4 words,
//     float32 scale and int sum per block stay in registers for all rows.
//   * Each row is handled by a team of T = 8/16/32 threads. Thread t reads
//     block b's 18 bytes from shared memory as five aligned 32-bit words and
//     funnel-shifts the nibbles into place (the 2-byte misalignment of odd
//     blocks is a per-thread constant), then computes the block dot with
//     __dp4a: sumi = sum(nibble * x) - 8 * sum(x), exact in int32.
//   * Float work follows the contract to the bit: t = (f32(sumi) * f32(dw)) *
//     f32(dx) as two rounded multiplies; lane b mod 8 accumulates sequentially
//     in b, which the team does by shuffling the (up to) four values a lane
//     receives per T-block step to its owner thread and adding them in order;
//     the final eight lanes go through xor-shuffles 1, 2, 4, which is exactly
//     tree_sum's adjacent-pair tree (float addition is commutative).
// Blocks past nb contribute +0.0f, an exact no-op on a lane that started at
// +0.0f (a lane sum can never be -0.0f).
#include <cuda_fp16.h>

#include <cstdio>

#include "ptx.cuh"
#include "q4gemv.h"

namespace b200 {

__device__ unsigned g_status;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 64;  // kMaxStages mbarriers
constexpr uint64_t kStageTimeoutNs = 2000000000ull;  // 2 s: a healthy stage lands in microseconds
constexpr unsigned kFull = 0xffffffffu;

struct GemvParams {
    const uint8_t *region[4];
    float *y;
    const void *x;
    int units_per_region;  // rows (ROWS) or row pairs (PAIRS) per region
    int rows_per_region;
    int unit_bytes;
    int k, nb;
    int ctas_per_region;
    int su;            // units per stage
    int stages;        // ring depth
    int stage_stride;  // bytes per ring slot
    int xarea_bytes;   // shared bytes for the F32-mode quantised x
    int round_mode;
    int l2_policy;
};

__device__ __forceinline__ int q8_round(float s, int mode) {
    if (mode == kRoundRoundf) return static_cast<int>(roundf(s));
    // q4_0.py:96: sign(s) * floor(|s| + 0.5f), the add rounded in float32.
    const int m = static_cast<int>(floorf(__fadd_rn(fabsf(s), 0.5f)));
    return s < 0.0f ? -m : m;
}

// One Q8_0 block held by 8 consecutive threads (4 values each). Returns this
// thread's 4 int8 packed in a word; *d gets the float32 scale before rounding
// to float16, *sum the block's int sum (all 8 threads get both).
// q4_0.py:89-97: amax / 127, inv = d == 0 ? 0 : 1/d, both IEEE-rounded.
__device__ __forceinline__ uint32_t q8_quant_group(float4 v, int mode, float *d, int *sum) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1, 8));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2, 8));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 4, 8));
    const float db = __fdiv_rn(amax, 127.0f);
    const float inv = db == 0.0f ? 0.0f : __fdiv_rn(1.0f, db);
    const int q0 = q8_round(__fmul_rn(v.x, inv), mode);
    const int q1 = q8_round(__fmul_rn(v.y, inv), mode);
    const int q2 = q8_round(__fmul_rn(v.z, inv), mode);
    const int q3 = q8_round(__fmul_rn(v.w, inv), mode);
    int s = q0 + q1 + q2 + q3;
    s += __shfl_xor_sync(kFull, s, 1, 8);
    s += __shfl_xor_sync(kFull, s, 2, 8);
    s += __shfl_xor_sync(kFull, s, 4, 8);
    *d = db;
    *sum = s;
    return (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
           ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
}

__device__ __forceinline__ uint64_t make_policy(int kind) {
    if (kind == kL2EvictLast) return l2_policy_evict_last();
    if (kind == kL2EvictNormal) return l2_policy_evict_normal();
    return l2_policy_evict_first();
}

// Bounded mbarrier wait. Returns false (and flags the device status) after
// kStageTimeoutNs without the phase completing.
__device__ __forceinline__ bool wait_stage(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kStageTimeoutNs) {
            atomicOr(&g_status, kStatusStageTimeout);
            return false;
        }
    }
    return true;
}

template <int LAYOUT, int XMODE, int T, int NI>
__global__ void __launch_bounds__(kThreads, 2) q4_gemv_kernel(const __grid_constant__ GemvParams p) {
    constexpr int P = 32 / T;  // rows a warp works on at once
    constexpr int M = LAYOUT == kLayoutPairs ? 2 : 1;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint8_t *xarea = smem + kBarBytes;
    uint8_t *ring = smem + kBarBytes + p.xarea_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = lane % T;  // thread within its row team
    const int region = blockIdx.x / p.ctas_per_region;
    const int cr = blockIdx.x - region * p.ctas_per_region;
    const int u0 = static_cast<int>(static_cast<long long>(p.units_per_region) * cr / p.ctas_per_region);
    const int u1 = static_cast<int>(static_cast<long long>(p.units_per_region) * (cr + 1) / p.ctas_per_region);
    const int nunits = u1 - u0;
    const int nst = (nunits + p.su - 1) / p.su;
    const uint8_t *src = p.region[region] + static_cast<size_t>(u0) * p.unit_bytes;
    const int S = p.stages;

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Weights do not depend on the previous kernel: start streaming them
    // before waiting on it (programmatic dependent launch).
    uint64_t policy = 0;
    if (tid == 0) {
        policy = make_policy(p.l2_policy);
        const int first = nst < S ? nst : S;
        for (int s = 0; s < first; ++s) {
            const int cnt = min(p.su, nunits - s * p.su);
            const uint32_t bytes = static_cast<uint32_t>(cnt * p.unit_bytes);
            mbar_arrive_expect_tx(&bars[s], bytes);
            bulk_g2s(ring + s * p.stage_stride, src + static_cast<size_t>(s) * p.su * p.unit_bytes, bytes, &bars[s],
                     policy);
        }
    }
    // Every CTA of this grid is resident once it gets here, so the next
    // kernel in the stream may start its own weight streaming now.
    pdl_launch_dependents();
    pdl_wait_prior_grid();

    // ---- x into registers
    uint32_t xw[NI][8];
    float xdv[NI];
    int xs[NI];
    if constexpr (XMODE == kXF32) {
        const float *xf = static_cast<const float *>(p.x);
        uint32_t *sq = reinterpret_cast<uint32_t *>(xarea);
        float *sd = reinterpret_cast<float *>(xarea + p.k);
        int *ss = reinterpret_cast<int *>(xarea + p.k + 4 * p.nb);
        for (int b0 = 0; b0 < p.nb; b0 += kThreads / 8) {
            const int b = b0 + tid / 8, sub = tid % 8;
            const bool ok = b < p.nb;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) v = __ldg(reinterpret_cast<const float4 *>(xf + 32 * b) + sub);
            float d;
            int sum;
            const uint32_t packed = q8_quant_group(v, p.round_mode, &d, &sum);
            if (ok) {
                sq[8 * b + sub] = packed;
                if (sub == 0) {
                    sd[b] = __half2float(__float2half_rn(d));
                    ss[b] = sum;
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < NI; ++i) {
            const int b = t + T * i;
            if (b < p.nb) {
                const uint4 a = reinterpret_cast<const uint4 *>(sq + 8 * b)[0];
                const uint4 c = reinterpret_cast<const uint4 *>(sq + 8 * b)[1];
                xw[i][0] = a.x; xw[i][1] = a.y; xw[i][2] = a.z; xw[i][3] = a.w;
                xw[i][4] = c.x; xw[i][5] = c.y; xw[i][6] = c.z; xw[i][7] = c.w;
                xdv[i] = sd[b];
                xs[i] = ss[b];
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) xw[i][j] = 0;
                xdv[i] = 0.0f;
                xs[i] = 0;
            }
        }
    } else {
        const uint8_t *xq = static_cast<const uint8_t *>(p.x);
        const float *xd = reinterpret_cast<const float *>(xq + p.k);
#pragma unroll
        for (int i = 0; i < NI; ++i) {
            const int b = t + T * i;
            if (b < p.nb) {
                const uint4 a = __ldg(reinterpret_cast<const uint4 *>(xq + 32 * b));
                const uint4 c = __ldg(reinterpret_cast<const uint4 *>(xq + 32 * b) + 1);
                xw[i][0] = a.x; xw[i][1] = a.y; xw[i][2] = a.z; xw[i][3] = a.w;
                xw[i][4] = c.x; xw[i][5] = c.y; xw[i][6] = c.z; xw[i][7] = c.w;
                xdv[i] = __ldg(xd + b);
                int s = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) s = __dp4a(static_cast<int>(xw[i][j]), 0x01010101, s);
                xs[i] = s;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) xw[i][j] = 0;
                xdv[i] = 0.0f;
                xs[i] = 0;
            }
        }
    }

    // ---- stream the stages
    const int odd = t & 1;  // block b = t + T*i has b & 1 == t & 1 (T even)
    const uint32_t nib_shift = odd ? 32u : 16u;
    const uint32_t d_shift = odd ? 16u : 0u;
    int s = 0;
    for (; s < nst; ++s) {
        const int slot = s % S;
        const bool landed = wait_stage(&bars[slot], static_cast<uint32_t>((s / S) & 1));
        if (!landed) s_abort = 1;
        const uint8_t *sbuf = ring + slot * p.stage_stride;
        const int cnt = min(p.su, nunits - s * p.su);
        const int rows_here = cnt * M;
        for (int base = warp * P; base < rows_here; base += kWarps * P) {
            const int rl = base + lane / T;
            const bool vrow = landed && rl < rows_here;
            const int ul = M == 2 ? (rl >> 1) : rl;
            const int mem = M == 2 ? (rl & 1) : 0;
            const uint8_t *ub = sbuf + ul * p.unit_bytes;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < NI; ++i) {
                const int b = t + T * i;
                float v = 0.0f;
                if (vrow && b < p.nb) {
                    const int off = LAYOUT == kLayoutPairs ? (2 * (b >> 3) + mem) * kChunkBytes + kBlockBytes * (b & 7)
                                                           : kBlockBytes * b;
                    const uint32_t *wp = reinterpret_cast<const uint32_t *>(ub + off - 2 * odd);
                    const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2], w3 = wp[3], w4 = wp[4];
                    const uint32_t n0 = __funnelshift_rc(w0, w1, nib_shift);
                    const uint32_t n1 = __funnelshift_rc(w1, w2, nib_shift);
                    const uint32_t n2 = __funnelshift_rc(w2, w3, nib_shift);
                    const uint32_t n3 = __funnelshift_rc(w3, w4, nib_shift);
                    const uint32_t dbits = __funnelshift_rc(w0, w1, d_shift) & 0xffffu;
                    int sumi = -8 * xs[i];
                    sumi = __dp4a(static_cast<int>(n0 & 0x0f0f0f0fu), static_cast<int>(xw[i][0]), sumi);
                    sumi = __dp4a(static_cast<int>(n1 & 0x0f0f0f0fu), static_cast<int>(xw[i][1]), sumi);
                    sumi = __dp4a(static_cast<int>(n2 & 0x0f0f0f0fu), static_cast<int>(xw[i][2]), sumi);
                    sumi = __dp4a(static_cast<int>(n3 & 0x0f0f0f0fu), static_cast<int>(xw[i][3]), sumi);
                    sumi = __dp4a(static_cast<int>((n0 >> 4) & 0x0f0f0f0fu), static_cast<int>(xw[i][4]), sumi);
                    sumi = __dp4a(static_cast<int>((n1 >> 4) & 0x0f0f0f0fu), static_cast<int>(xw[i][5]), sumi);
                    sumi = __dp4a(static_cast<int>((n2 >> 4) & 0x0f0f0f0fu), static_cast<int>(xw[i][6]), sumi);
                    sumi = __dp4a(static_cast<int>((n3 >> 4) & 0x0f0f0f0fu), static_cast<int>(xw[i][7]), sumi);
                    const float dw = __half2float(__ushort_as_half(static_cast<unsigned short>(dbits)));
                    v = __fmul_rn(__fmul_rn(__int2float_rn(sumi), dw), xdv[i]);
                }
                // Lane (t mod 8) receives blocks t, t+8, t+16, t+24 of this
                // step, in that order: add them sequentially.
                if constexpr (T == 32) {
                    const float v1 = __shfl_down_sync(kFull, v, 8);
                    const float v2 = __shfl_down_sync(kFull, v, 16);
                    const float v3 = __shfl_down_sync(kFull, v, 24);
                    acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v), v1), v2), v3);
                } else if constexpr (T == 16) {
                    const float v1 = __shfl_down_sync(kFull, v, 8, 16);
                    acc = __fadd_rn(__fadd_rn(acc, v), v1);
                } else {
                    acc = __fadd_rn(acc, v);
                }
            }
            // tree_sum over the 8 lanes held by threads t = 0..7.
            acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, 1, 8));
            acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, 2, 8));
            acc = __fadd_rn(acc, __shfl_xor_sync(kFull, acc, 4, 8));
            if (vrow && t == 0) {
                const int u = u0 + s * p.su + ul;
                const int row = region * p.rows_per_region + (M == 2 ? u + mem * p.units_per_region : u);
                p.y[row] = acc;
            }
        }
        __syncthreads();
        if (s_abort) break;
        if (tid == 0 && s + S < nst) {
            const int cnt2 = min(p.su, nunits - (s + S) * p.su);
            const uint32_t bytes = static_cast<uint32_t>(cnt2 * p.unit_bytes);
            mbar_arrive_expect_tx(&bars[slot], bytes);
            bulk_g2s(ring + slot * p.stage_stride, src + static_cast<size_t>(s + S) * p.su * p.unit_bytes, bytes,
                     &bars[slot], policy);
        }
    }
    if (s < nst && tid == 0) {
        // Aborted on a stage timeout: let copies already in flight land
        // (each wait bounded) before the CTA's shared memory goes away.
        const int issued = min(nst, s + S);
        for (int r = s; r < issued; ++r) (void)wait_stage(&bars[r % S], static_cast<uint32_t>((r / S) & 1));
    }
}

// x float32[k] -> int8[k] then float32[k/32]; 8 threads per block.
__global__ void __launch_bounds__(256) q8_quantize_kernel(const float *__restrict__ x, uint8_t *__restrict__ out,
                                                          int k, int round_mode) {
    pdl_wait_prior_grid();
    const int nb = k / kQK;
    const int g = blockIdx.x * (blockDim.x / 8) + threadIdx.x / 8, sub = threadIdx.x % 8;
    const bool ok = g < nb;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) v = __ldg(reinterpret_cast<const float4 *>(x + 32 * g) + sub);
    float d;
    int sum;
    const uint32_t packed = q8_quant_group(v, round_mode, &d, &sum);
    if (ok) {
        reinterpret_cast<uint32_t *>(out)[8 * g + sub] = packed;
        if (sub == 0) reinterpret_cast<float *>(out + k)[g] = __half2float(__float2half_rn(d));
    }
    pdl_launch_dependents();
}

constexpr uint32_t kPrefetchChunk = 32768;

__global__ void l2_prefetch_kernel(const uint8_t *r0, const uint8_t *r1, const uint8_t *r2, const uint8_t *r3,
                                   int nregions, size_t bytes) {
    const uint8_t *regs[4] = {r0, r1, r2, r3};
    const size_t chunks = (bytes + kPrefetchChunk - 1) / kPrefetchChunk;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < chunks * nregions;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / chunks);
        const size_t off = (i % chunks) * kPrefetchChunk;
        const size_t len = (bytes - off < kPrefetchChunk ? bytes - off : kPrefetchChunk) & ~static_cast<size_t>(15);
        if (len) bulk_prefetch_l2(regs[r] + off, static_cast<uint32_t>(len));
    }
}

// ------------------------------------------------------------ dispatch

using KernelFn = void (*)(GemvParams);

template <int LAYOUT, int XMODE>
KernelFn pick(int T, int NI) {
    if (T == 32) {
        switch (NI) {
            case 1: return q4_gemv_kernel<LAYOUT, XMODE, 32, 1>;
            case 2: return q4_gemv_kernel<LAYOUT, XMODE, 32, 2>;
            case 3: return q4_gemv_kernel<LAYOUT, XMODE, 32, 3>;
            case 4: return q4_gemv_kernel<LAYOUT, XMODE, 32, 4>;
            case 5: return q4_gemv_kernel<LAYOUT, XMODE, 32, 5>;
            case 6: return q4_gemv_kernel<LAYOUT, XMODE, 32, 6>;
            case 7: return q4_gemv_kernel<LAYOUT, XMODE, 32, 7>;
            case 8: return q4_gemv_kernel<LAYOUT, XMODE, 32, 8>;
        }
    } else if (T == 16) {
        if (NI == 1) return q4_gemv_kernel<LAYOUT, XMODE, 16, 1>;
        if (NI == 2) return q4_gemv_kernel<LAYOUT, XMODE, 16, 2>;
    } else if (T == 8) {
        if (NI == 1) return q4_gemv_kernel<LAYOUT, XMODE, 8, 1>;
        if (NI == 2) return q4_gemv_kernel<LAYOUT, XMODE, 8, 2>;
    }
    return nullptr;
}

KernelFn pick_kernel(int layout, int xmode, int T, int NI) {
    if (layout == kLayoutRows) return xmode == kXF32 ? pick<kLayoutRows, kXF32>(T, NI) : pick<kLayoutRows, kXPacked>(T, NI);
    return xmode == kXF32 ? pick<kLayoutPairs, kXF32>(T, NI) : pick<kLayoutPairs, kXPacked>(T, NI);
}

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    int sms = 0;
    int smem_optin = 0;
};

// Per-device attributes, read once (launch paths are latency-critical).
const DeviceInfo *device_info() {
    static DeviceInfo info[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    DeviceInfo &d = info[dev];
    if (d.sms == 0) {
        int sms = 0, smem = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return nullptr;
        if (cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return nullptr;
        d.smem_optin = smem;
        d.sms = sms;
    }
    return &d;
}

int sm_count() {
    const DeviceInfo *d = device_info();
    return d ? d->sms : 0;
}

int max_smem_optin() {
    const DeviceInfo *d = device_info();
    return d ? d->smem_optin : 0;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device).
bool ensure_smem(KernelFn fn, int bytes) {
    struct Entry { KernelFn fn; int dev; int bytes; };
    static Entry cache[256];
    static int used = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    for (int i = 0; i < used; ++i)
        if (cache[i].fn == fn && cache[i].dev == dev && cache[i].bytes >= bytes) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    if (used < 256) cache[used++] = Entry{fn, dev, bytes};
    return true;
}

inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

struct Plan {
    GemvParams p;
    KernelFn fn;
    int grid;
    int smem;
};

int make_plan(const GemvLaunch &L, const Tuning &tu, Plan *out) {
    const char *why = nullptr;
    if (int rc = gemv_validate(L, &why)) return rc;
    const int nb = L.k / kQK, row_bytes = nb * kBlockBytes;
    const int M = L.layout == kLayoutPairs ? 2 : 1;
    const int T = nb >= 32 ? 32 : (nb >= 16 ? 16 : 8);
    const int NI = (nb + T - 1) / T;
    KernelFn fn = pick_kernel(L.layout, L.xmode, T, NI);
    if (!fn) return kErrInval;
    GemvParams p{};
    for (int r = 0; r < 4; ++r) p.region[r] = L.region[r < L.nregions ? r : 0];
    p.y = L.y;
    p.x = L.x;
    p.rows_per_region = L.rows / L.nregions;
    p.units_per_region = p.rows_per_region / M;
    p.unit_bytes = M * row_bytes;
    p.k = L.k;
    p.nb = nb;
    p.round_mode = L.round_mode;
    p.l2_policy = L.l2_policy;
    p.stages = tu.stages < 1 ? 1 : (tu.stages > kMaxStages ? kMaxStages : tu.stages);
    int su = tu.stage_bytes / p.unit_bytes;
    if (su < 1) su = 1;
    if (su > p.units_per_region) su = p.units_per_region;
    p.xarea_bytes = L.xmode == kXF32 ? round_up(L.k + 8 * nb, 128) : 0;
    const int limit = max_smem_optin();
    for (;;) {
        p.su = su;
        p.stage_stride = round_up(su * p.unit_bytes + 16, 128);
        const int smem = kBarBytes + p.xarea_bytes + p.stages * p.stage_stride;
        if (smem <= limit || (su == 1 && p.stages == 1)) break;
        if (su > 1) su = (su + 1) / 2;
        else p.stages -= 1;
    }
    const int smem = kBarBytes + p.xarea_bytes + p.stages * p.stage_stride;
    if (smem > limit) return kErrInval;
    const int sms = sm_count();
    if (sms <= 0) return kErrNoDev;
    const int target = sms * (tu.ctas_per_sm < 1 ? 1 : tu.ctas_per_sm);
    const int stages_per_region = (p.units_per_region + su - 1) / su;
    int cpr = target / L.nregions;
    if (cpr < 1) cpr = 1;
    if (cpr > stages_per_region) cpr = stages_per_region;
    p.ctas_per_region = cpr;
    out->p = p;
    out->fn = fn;
    out->grid = cpr * L.nregions;
    out->smem = smem;
    return 0;
}

}  // namespace

int gemv_validate(const GemvLaunch &L, const char **why) {
    auto bad = [&](const char *w) { if (why) *why = w; return kErrInval; };
    if (L.nregions != 1 && L.nregions != 4) return bad("nregions must be 1 or 4");
    if (L.layout != kLayoutRows && L.layout != kLayoutPairs) return bad("unknown layout");
    if (L.xmode != kXPacked && L.xmode != kXF32) return bad("unknown x mode");
    if (L.round_mode != kRoundContract && L.round_mode != kRoundRoundf) return bad("unknown rounding mode");
    if (L.k <= 0 || L.k % 256) return bad("k must be a positive multiple of 256 (nb % 8 == 0, q4_0.py:166)");
    if (L.k > kMaxK) return bad("k above 8192");
    if (L.rows <= 0) return bad("rows must be positive");
    if (L.rows % L.nregions) return bad("rows must divide into the regions");
    if (L.layout == kLayoutPairs && (L.nregions != 4 || L.rows % 8)) return bad("gemv2 layout needs 4 regions and rows % 8 == 0");
    for (int r = 0; r < L.nregions; ++r) {
        if (!L.region[r]) return bad("null weight pointer");
        if (reinterpret_cast<uintptr_t>(L.region[r]) % 16) return bad("weight regions must be 16-byte aligned");
    }
    if (!L.x || reinterpret_cast<uintptr_t>(L.x) % 16) return bad("x must be 16-byte aligned");
    if (!L.y || reinterpret_cast<uintptr_t>(L.y) % 4) return bad("y must be 4-byte aligned");
    return 0;
}

int gemv_grid(const GemvLaunch &L, const Tuning &tu, int *grid, int *smem_bytes) {
    Plan pl;
    if (int rc = make_plan(L, tu, &pl)) return rc;
    if (grid) *grid = pl.grid;
    if (smem_bytes) *smem_bytes = pl.smem;
    return 0;
}

int gemv_launch(const GemvLaunch &L, const Tuning &tu, cudaStream_t stream) {
    Plan pl;
    if (int rc = make_plan(L, tu, &pl)) return rc;
    if (!ensure_smem(pl.fn, pl.smem)) return kErrCuda;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = L.pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, pl.fn, pl.p) != cudaSuccess) return kErrCuda;
    return 0;
}

int quantize_launch(const float *x, uint8_t *xpacked, int k, int round_mode, cudaStream_t stream, bool pdl) {
    if (!x || !xpacked || k <= 0 || k % kQK) return kErrInval;
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(xpacked) % 16) return kErrInval;
    if (round_mode != kRoundContract && round_mode != kRoundRoundf) return kErrInval;
    const int nb = k / kQK;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((nb + 31) / 32);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, q8_quantize_kernel, x, xpacked, k, round_mode) != cudaSuccess) return kErrCuda;
    return 0;
}

int prefetch_l2_launch(const uint8_t *const *region, int nregions, size_t bytes_per_region, cudaStream_t stream) {
    if (nregions < 1 || nregions > 4 || !region) return kErrInval;
    for (int r = 0; r < nregions; ++r)
        if (!region[r] || reinterpret_cast<uintptr_t>(region[r]) % 16) return kErrInval;
    const size_t chunks = (bytes_per_region + kPrefetchChunk - 1) / kPrefetchChunk * nregions;
    int grid = static_cast<int>((chunks + 127) / 128);
    if (grid < 1) grid = 1;
    l2_prefetch_kernel<<<grid, 128, 0, stream>>>(region[0], nregions > 1 ? region[1] : region[0],
                                                  nregions > 2 ? region[2] : region[0],
                                                  nregions > 3 ? region[3] : region[0], nregions, bytes_per_region);
    return cudaGetLastError() == cudaSuccess ? 0 : kErrCuda;
}

int read_status(unsigned *status) {
    if (cudaMemcpyFromSymbol(status, g_status, sizeof(unsigned)) != cudaSuccess) return kErrCuda;
    return 0;
}

int clear_status() {
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_status, &zero, sizeof(unsigned)) == cudaSuccess ? 0 : kErrCuda;
}

}  // namespace b200
