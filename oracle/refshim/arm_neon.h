// Portable stand-in for <arm_neon.h>: TEST INFRASTRUCTURE ONLY.
//
// Lets the reference runtime's own NEON sections (board/tp/tp_llama.cpp:
// engine_t::quantize_x, the ops section, forward) compile on this x86 host,
// so the decode oracle can be checked against the reference's source text.
// Each intrinsic below is written from the Arm C Language Extensions' stated
// semantics, lane by lane, with the IEEE-754 rounding of the AArch64
// instruction it names (FPCR as Linux leaves it: round to nearest even,
// denormals kept, NaNs propagated):
//   * vfmaq / vfmsq are single-rounded fused multiply-adds (fmaf / fma);
//   * vaddvq_f32 is lowered by GCC for AArch64 to two FADDP, i.e.
//     (a0 + a1) + (a2 + a3). This is the one assumption here: the ACLE leaves
//     the order of the across-vector add open;
//   * vmaxq / vmaxvq follow FMAX (a NaN operand gives a NaN; +0 beats -0);
//   * vcvtaq_s32_f32 is FCVTAS: nearest, ties away from zero, saturating,
//     NaN -> 0;
//   * vmovn narrows by truncation (XTN).
// Only the intrinsics those sections use are defined.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

struct float32x4_t { float v[4]; };
struct float32x2_t { float v[2]; };
struct float64x2_t { double v[2]; };
struct uint32x4_t { uint32_t v[4]; };
struct uint64x2_t { uint64_t v[2]; };
struct int32x4_t { int32_t v[4]; };
struct int16x4_t { int16_t v[4]; };
struct int16x8_t { int16_t v[8]; };
struct int8x8_t { int8_t v[8]; };
struct int8x16_t { int8_t v[16]; };

namespace neon_shim {
inline uint32_t bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
inline float from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
inline float fmax_arm(float a, float b) {
    if (isnan(a) || isnan(b)) return from_bits(0x7fc00000u);
    if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
    return a > b ? a : b;
}
}  // namespace neon_shim

// ---- loads, stores, lanes
static inline float32x4_t vld1q_f32(const float *p) { float32x4_t r; memcpy(r.v, p, 16); return r; }
static inline void vst1q_f32(float *p, float32x4_t a) { memcpy(p, a.v, 16); }
static inline void vst1q_s8(int8_t *p, int8x16_t a) { memcpy(p, a.v, 16); }
static inline float32x4_t vdupq_n_f32(float x) { return {{x, x, x, x}}; }
static inline uint32x4_t vdupq_n_u32(uint32_t x) { return {{x, x, x, x}}; }
static inline float64x2_t vdupq_n_f64(double x) { return {{x, x}}; }
static inline float32x2_t vget_low_f32(float32x4_t a) { return {{a.v[0], a.v[1]}}; }
#define vgetq_lane_f32(a, lane) ((a).v[(lane)])

// ---- reinterpretation
static inline uint32x4_t vreinterpretq_u32_f32(float32x4_t a) { uint32x4_t r; memcpy(r.v, a.v, 16); return r; }
static inline float32x4_t vreinterpretq_f32_u32(uint32x4_t a) { float32x4_t r; memcpy(r.v, a.v, 16); return r; }
static inline uint64x2_t vreinterpretq_u64_u32(uint32x4_t a) { uint64x2_t r; memcpy(r.v, a.v, 16); return r; }

// ---- float32 arithmetic (each lane rounded once)
static inline float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] + b.v[i]; return r;
}
static inline float32x4_t vsubq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] - b.v[i]; return r;
}
static inline float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] * b.v[i]; return r;
}
static inline float32x4_t vdivq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] / b.v[i]; return r;
}
static inline float32x4_t vnegq_f32(float32x4_t a) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = neon_shim::from_bits(neon_shim::bits(a.v[i]) ^ 0x80000000u); return r;
}
static inline float32x4_t vabsq_f32(float32x4_t a) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = neon_shim::from_bits(neon_shim::bits(a.v[i]) & 0x7fffffffu); return r;
}
// a + b * c, one rounding (FMLA)
static inline float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = fmaf(b.v[i], c.v[i], a.v[i]); return r;
}
// a - b * c, one rounding (FMLS)
static inline float32x4_t vfmsq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = fmaf(-b.v[i], c.v[i], a.v[i]); return r;
}
static inline float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = neon_shim::fmax_arm(a.v[i], b.v[i]); return r;
}
static inline float vmaxvq_f32(float32x4_t a) {
    return neon_shim::fmax_arm(neon_shim::fmax_arm(a.v[0], a.v[1]), neon_shim::fmax_arm(a.v[2], a.v[3]));
}
// FADDP, FADDP: (a0 + a1) + (a2 + a3)
static inline float vaddvq_f32(float32x4_t a) { return (a.v[0] + a.v[1]) + (a.v[2] + a.v[3]); }

// ---- comparisons and bit selects
static inline uint32x4_t vcagtq_f32(float32x4_t a, float32x4_t b) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = fabsf(a.v[i]) > fabsf(b.v[i]) ? 0xffffffffu : 0u; return r;
}
static inline uint32x4_t vclezq_f32(float32x4_t a) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] <= 0.0f ? 0xffffffffu : 0u; return r;
}
static inline float32x4_t vbslq_f32(uint32x4_t m, float32x4_t a, float32x4_t b) {
    float32x4_t r;
    for (int i = 0; i < 4; ++i)
        r.v[i] = neon_shim::from_bits((m.v[i] & neon_shim::bits(a.v[i])) | (~m.v[i] & neon_shim::bits(b.v[i])));
    return r;
}

// ---- integer lanes
static inline uint32x4_t vaddq_u32(uint32x4_t a, uint32x4_t b) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] + b.v[i]; return r;
}
static inline uint32x4_t vsubq_u32(uint32x4_t a, uint32x4_t b) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] - b.v[i]; return r;
}
static inline uint32x4_t vandq_u32(uint32x4_t a, uint32x4_t b) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] & b.v[i]; return r;
}
#define vshlq_n_u32(a, n) neon_shim_shl_u32((a), (n))
static inline uint32x4_t neon_shim_shl_u32(uint32x4_t a, int n) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = a.v[i] << n; return r;
}
static inline uint64_t vpaddd_u64(uint64x2_t a) { return a.v[0] + a.v[1]; }

// FCVTAS: round to nearest with ties away from zero, saturate, NaN -> 0
static inline int32x4_t vcvtaq_s32_f32(float32x4_t a) {
    int32x4_t r;
    for (int i = 0; i < 4; ++i) {
        const float x = a.v[i];
        if (isnan(x)) r.v[i] = 0;
        else if (x >= 2147483648.0f) r.v[i] = INT32_MAX;
        else if (x < -2147483648.0f) r.v[i] = INT32_MIN;
        else r.v[i] = (int32_t)roundf(x);
    }
    return r;
}
static inline int16x4_t vmovn_s32(int32x4_t a) {
    int16x4_t r; for (int i = 0; i < 4; ++i) r.v[i] = (int16_t)(uint16_t)(uint32_t)a.v[i]; return r;
}
static inline int8x8_t vmovn_s16(int16x8_t a) {
    int8x8_t r; for (int i = 0; i < 8; ++i) r.v[i] = (int8_t)(uint8_t)(uint16_t)a.v[i]; return r;
}
static inline int16x8_t vcombine_s16(int16x4_t lo, int16x4_t hi) {
    int16x8_t r; memcpy(r.v, lo.v, 8); memcpy(r.v + 4, hi.v, 8); return r;
}
static inline int8x16_t vcombine_s8(int8x8_t lo, int8x8_t hi) {
    int8x16_t r; memcpy(r.v, lo.v, 8); memcpy(r.v + 8, hi.v, 8); return r;
}

// ---- float64
static inline float64x2_t vcvt_f64_f32(float32x2_t a) { return {{(double)a.v[0], (double)a.v[1]}}; }
static inline float64x2_t vcvt_high_f64_f32(float32x4_t a) { return {{(double)a.v[2], (double)a.v[3]}}; }
static inline float64x2_t vfmaq_f64(float64x2_t a, float64x2_t b, float64x2_t c) {
    return {{fma(b.v[0], c.v[0], a.v[0]), fma(b.v[1], c.v[1], a.v[1])}};
}
static inline float64x2_t vaddq_f64(float64x2_t a, float64x2_t b) { return {{a.v[0] + b.v[0], a.v[1] + b.v[1]}}; }
static inline double vaddvq_f64(float64x2_t a) { return a.v[0] + a.v[1]; }
