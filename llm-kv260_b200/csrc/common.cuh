// Device helpers shared by the GEMV kernels (q4gemv.cu, q4tile.cu) and the
// host helpers both launchers use.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"
#include "q4gemv.h"

namespace b200 {

constexpr unsigned kFullMask = 0xffffffffu;
constexpr uint64_t kStageTimeoutNs = 2000000000ull;  // 2 s: a healthy stage lands in microseconds

// ------------------------------------------------------------- Q8_0 quantiser

__device__ __forceinline__ int q8_round(float s, int mode) {
    if (mode == kRoundRoundf) return static_cast<int>(roundf(s));
    // q4_0.py:96: sign(s) * floor(|s| + 0.5f), the add rounded in float32.
    const int m = static_cast<int>(floorf(__fadd_rn(fabsf(s), 0.5f)));
    return s < 0.0f ? -m : m;
}

// One Q8_0 block quantised by one thread (q4_0.py:83-97): amax / 127,
// inv = d == 0 ? 0 : 1/d (both IEEE-rounded), the contract's rounding per
// value. Writes 8 int8x4 words to q; returns the int sum, *d the float32 scale.
__device__ __forceinline__ int q8_quant_block(const float4 v[8], int mode, uint32_t q[8], float *d) {
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
    const float amax = fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
    const float db = __fdiv_rn(amax, 127.0f);
    const float inv = db == 0.0f ? 0.0f : __fdiv_rn(1.0f, db);
    int sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int q0 = q8_round(__fmul_rn(v[j].x, inv), mode);
        const int q1 = q8_round(__fmul_rn(v[j].y, inv), mode);
        const int q2 = q8_round(__fmul_rn(v[j].z, inv), mode);
        const int q3 = q8_round(__fmul_rn(v[j].w, inv), mode);
        sum += q0 + q1 + q2 + q3;
        q[j] = (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
               ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
    }
    *d = db;
    return sum;
}

// Staged x in shared memory: block b's 32 int8 at xs + 48 * b (16 bytes of
// padding each, so the blocks of 8 consecutive lanes -- what a quarter warp
// reads in one 16-byte load -- fall in 8 different bank groups), then
// (float32 d, int32 sum of the 32 int8) per block at xs_scales.
constexpr int kXsBlockStride = 48;
__host__ __device__ constexpr int xs_qbytes(int k) { return k / 32 * kXsBlockStride; }
__host__ __device__ constexpr int xs_bytes(int k) { return xs_qbytes(k) + 8 * (k / 32); }
__device__ __forceinline__ uint8_t *xs_block(uint8_t *xs, int b) { return xs + kXsBlockStride * b; }
__device__ __forceinline__ const uint8_t *xs_block(const uint8_t *xs, int b) { return xs + kXsBlockStride * b; }
__device__ __forceinline__ int2 *xs_scales(uint8_t *xs, int k) { return reinterpret_cast<int2 *>(xs + xs_qbytes(k)); }
__device__ __forceinline__ const int2 *xs_scales(const uint8_t *xs, int k) {
    return reinterpret_cast<const int2 *>(xs + xs_qbytes(k));
}

// x into shared memory for the whole CTA in that layout. `x` is float32[k] (quantised
// here, q4_0.py:83-97) or the engine buffer int8[k] + float32[k/32].
// One thread per block, all loads issued before any use and no shuffles, so
// the staging costs one memory round trip plus one block's arithmetic; the
// CTA must have at least k/32 threads.
template <int XMODE>
__device__ __forceinline__ void stage_x(const void *x, int k, int round_mode, uint8_t *xs) {
    const int nb = k / kQK, b = threadIdx.x;
    if (b >= nb) return;
    uint4 *qdst = reinterpret_cast<uint4 *>(xs_block(xs, b));
    if constexpr (XMODE == kXF32) {
        const float4 *src = reinterpret_cast<const float4 *>(x) + 8 * b;
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldg(src + j);
        uint32_t q[8];
        float d;
        const int sum = q8_quant_block(v, round_mode, q, &d);
        qdst[0] = make_uint4(q[0], q[1], q[2], q[3]);
        qdst[1] = make_uint4(q[4], q[5], q[6], q[7]);
        xs_scales(xs, k)[b] = make_int2(__float_as_int(__half2float(__float2half_rn(d))), sum);
    } else {
        const uint8_t *xq = static_cast<const uint8_t *>(x);
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(xq + 32 * b));
        const uint4 c = __ldg(reinterpret_cast<const uint4 *>(xq + 32 * b) + 1);
        const float d = __ldg(reinterpret_cast<const float *>(xq + k) + b);
        int sum = 0;
        sum = __dp4a(static_cast<int>(a.x), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(a.y), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(a.z), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(a.w), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(c.x), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(c.y), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(c.z), 0x01010101, sum);
        sum = __dp4a(static_cast<int>(c.w), 0x01010101, sum);
        qdst[0] = a;
        qdst[1] = c;
        xs_scales(xs, k)[b] = make_int2(__float_as_int(d), sum);
    }
}

// x for one block: 8 int8x4 words, the float32 scale, and -8 times the int
// sum of the 32 values (the nibble offset folded into the dot's start value).
struct XBlock {
    uint32_t q[8];
    float d;
    int s8;
};

__device__ __forceinline__ void load_xblock_smem(const uint8_t *xs, int k, int b, XBlock &xb) {
    const uint4 a = reinterpret_cast<const uint4 *>(xs_block(xs, b))[0];
    const uint4 c = reinterpret_cast<const uint4 *>(xs_block(xs, b))[1];
    const int2 ds = xs_scales(xs, k)[b];
    xb.q[0] = a.x; xb.q[1] = a.y; xb.q[2] = a.z; xb.q[3] = a.w;
    xb.q[4] = c.x; xb.q[5] = c.y; xb.q[6] = c.z; xb.q[7] = c.w;
    xb.d = __int_as_float(ds.x);
    xb.s8 = -8 * ds.y;
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// The contract's block term from 4 nibble words (byte j: weight j low, weight
// j+16 high, value n-8), the float16 scale bits and x:
//   sumi = sum(n * x) - 8 * sum(x)        exact int32 (q4_0.py:170-171)
//   t    = (f32(sumi) * f32(dw)) * f32(dx)  two rounded multiplies (q4_0.py:174)
// The high nibbles enter unshifted, as 16 * n (unsigned bytes): their dot is
// 16 times the wanted one, and the exact >> 4 recovers it (|16 * dot| < 2^19).
__device__ __forceinline__ float block_term_words(const uint32_t n[4], uint32_t dbits, const XBlock &xb) {
    int lo = xb.s8, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        lo = __dp4a(static_cast<int>(n[j] & 0x0f0f0f0fu), static_cast<int>(xb.q[j]), lo);
        hi = dp4a_us(n[j] & 0xf0f0f0f0u, xb.q[4 + j], hi);
    }
    const int sumi = lo + (hi >> 4);
    const float dw = __half2float(__ushort_as_half(static_cast<unsigned short>(dbits)));
    return __fmul_rn(__fmul_rn(__int2float_rn(sumi), dw), xb.d);
}

// tree_sum over 8 lanes (q4_0.py:67-78): ((0+1)+(2+3))+((4+5)+(6+7)).
__device__ __forceinline__ float tree8(float l0, float l1, float l2, float l3, float l4, float l5, float l6,
                                       float l7) {
    return __fadd_rn(__fadd_rn(__fadd_rn(l0, l1), __fadd_rn(l2, l3)), __fadd_rn(__fadd_rn(l4, l5), __fadd_rn(l6, l7)));
}

__device__ __forceinline__ uint64_t make_policy(int kind) {
    if (kind == kL2EvictLast) return l2_policy_evict_last();
    if (kind == kL2EvictNormal) return l2_policy_evict_normal();
    return l2_policy_evict_first();
}

// Bounded mbarrier wait. Returns false (and sets *status) after
// kStageTimeoutNs without the phase completing.
__device__ __forceinline__ bool wait_stage(uint64_t *bar, uint32_t parity, unsigned *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kStageTimeoutNs) {
            atomicOr(status, kStatusStageTimeout);
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------------- host helpers

int sm_count();
int max_smem_optin();
// Raise a kernel's dynamic shared-memory limit once per (kernel, device).
bool ensure_smem(const void *fn, int bytes);
// Resident CTAs per SM for (kernel, threads, dynamic smem), cached per device.
int resident_ctas(const void *fn, int threads, int smem);
// Device address of this device's status word.
unsigned *status_word();

inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

}  // namespace b200
