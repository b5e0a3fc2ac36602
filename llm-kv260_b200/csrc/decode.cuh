// Device restatements of the reference runtime's decode ops
// (board/tp/tp_llama.cpp:528-622), each with the roundings of its NEON code:
// every vfmaq_f32 a single fused multiply-add, every other operation rounded
// on its own (explicit _rn intrinsics, so nvcc cannot contract them).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace b200 {

// v_expf, tp_llama.cpp:530-553: ggml's vector exp after Arm's optimized
// routines (2^(x / ln 2) split into 2^n * 2^(r), a degree-5 polynomial in r,
// max error 1.45358 + 0.5 ulp), one lane. The special-case branch of the
// vector code picks, lane by lane, the same value as the fast path wherever
// |n| <= 126, so per element it is the function below.
__device__ __forceinline__ float v_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, r);
    const float n = __fsub_rn(z, r);
    float b = __fmaf_rn(-n, 0x1.62e4p-1f, x);
    b = __fmaf_rn(-n, 0x1.7f7d1cp-20f, b);
    const uint32_t e = __float_as_uint(z) << 23;
    const float k = __uint_as_float(e + 0x3f800000u);
    const float u = __fmul_rn(b, b);
    const float p1 = __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f);
    const float p2 = __fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f);
    const float p3 = __fmaf_rn(p2, u, p1);
    const float j = __fmaf_rn(p3, u, __fmul_rn(0x1.ffffecp-1f, b));
    if (!(fabsf(n) > 126.0f)) return __fmaf_rn(j, k, k);
    const uint32_t d = n <= 0.0f ? 0x82000000u : 0u;
    const float s1 = __uint_as_float(d + 0x7f000000u);
    const float s2 = __uint_as_float(e - d);
    if (fabsf(n) > 192.0f) return __fmul_rn(s1, s1);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
}

// silu_mul, tp_llama.cpp:615-622: (g / (1 + v_expf(-g))) * up, IEEE divide.
__device__ __forceinline__ float silu_mul(float g, float up) {
    const float sg = __fdiv_rn(g, __fadd_rn(1.0f, v_expf(-g)));
    return __fmul_rn(sg, up);
}

// rope, tp_llama.cpp:581-591, for the pair (x0, x1) = (p[2i], p[2i+1]);
// `even` selects which of the two outputs this thread keeps.
__device__ __forceinline__ float rope_pair(float x0, float x1, float c, float s, bool even) {
    return even ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)) : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

// Where element e (0 <= e < hd) of the K row of position `pos` sits inside
// that row in the K cache (element index; esz 2: float16, 4: float32).
// Lane-major: the reference's scores run four fused-multiply-add lanes, lane
// j taking elements j, j+4, j+8, ... in order (tp_llama.cpp:652-660), so
// element e = 4m + j is step m of lane j, and lane j's steps are stored
// together: logical 16-byte segment s = j * L + m / (16 / esz) (L = hd * esz
// / 64 segments per lane). Logical segment s sits at physical segment
// (s & ~7) | ((s & 7) ^ (pos & 7) ^ 2 ((s >> 3) & 3)): the four lanes of one
// position, the eight lanes of two consecutive positions, and one segment of
// eight consecutive positions each fall on distinct shared-memory bank
// groups (rows are multiples of 128 bytes).
__host__ __device__ __forceinline__ int k_phys_seg(int s, int pos) {
    return (s & ~7) | ((s & 7) ^ (pos & 7) ^ (2 * ((s >> 3) & 3)));
}
__host__ __device__ __forceinline__ int k_slot(int e, int pos, int esz, int hd) {
    const int per = 16 / esz, lanes_segs = hd * esz / 64, j = e & 3, m = e >> 2;
    return k_phys_seg(j * lanes_segs + m / per, pos) * per + m % per;
}

// RMSNorm's sum of squares, tp_llama.cpp:557-564: the reference sums
// x[i]^2 in double in four lanes (i mod 4), sequentially, then
// (l0 + l2) + (l1 + l3), and uses (float)(ss / n). A parallel sum in another
// order differs from that by at most (n/4 + 44) double ulps of the total (all
// terms are >= 0; each square is exact in double), so when the float that
// ss / n rounds to is more than twice that bound away from both of its
// rounding boundaries, any order gives the reference's float. Returns true
// when `q` (a parallel ss / n) is that safe; the caller otherwise redoes the
// sum in the reference's order.
__device__ __forceinline__ bool rms_float_is_safe(double q, float f, int n) {
    const double tol = ldexp(static_cast<double>(n / 4 + 64), -52);
    const double delta = q * tol;
    const float up = nextafterf(f, INFINITY), dn = nextafterf(f, -INFINITY);
    const double mid_hi = 0.5 * (static_cast<double>(f) + static_cast<double>(up));
    const double mid_lo = 0.5 * (static_cast<double>(f) + static_cast<double>(dn));
    return __dsub_rn(q, delta) > mid_lo && __dadd_rn(q, delta) < mid_hi;
}

}  // namespace b200
