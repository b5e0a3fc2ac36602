// Minimal stand-in for ggml.h: TEST INFRASTRUCTURE ONLY (oracle/_ref).
//
// The reference runtime's model and engine sections (board/tp/tp_llama.cpp)
// use ggml for three things: float16 <-> float32 conversion, and the opaque
// context/tensor types of its GGUF reader (gguf.h beside this file). The
// conversions here are IEEE-754 binary16 with round to nearest even, as the
// AArch64 FCVT instruction that ggml uses on the boards performs them.
#pragma once

#include <stddef.h>
#include <stdint.h>
#include <string.h>

typedef uint16_t ggml_fp16_t;

struct ggml_init_params {
    size_t mem_size;
    void *mem_buffer;
    bool no_alloc;
};

struct ggml_tensor;    // only ever handled by pointer
struct ggml_context;   // (both defined in gguf.h)

static inline float ggml_fp16_to_fp32(ggml_fp16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu, u;
    if (exp == 0x1Fu) {
        u = sign | 0x7F800000u | (mant << 13);
    } else if (exp) {
        u = sign | ((exp + 112u) << 23) | (mant << 13);
    } else if (!mant) {
        u = sign;
    } else {  // subnormal: normalise
        int e = -1;
        do { mant <<= 1; ++e; } while (!(mant & 0x400u));
        u = sign | ((uint32_t)(112 - e) << 23) | ((mant & 0x3FFu) << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline ggml_fp16_t ggml_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (ggml_fp16_t)(sign | 0x7E00u | ((a >> 13) & 0x1FFu));  // NaN stays NaN (quiet)
    if (a >= 0x477FF000u) return (ggml_fp16_t)(sign | 0x7C00u);                      // >= 65520 rounds to inf
    if (a >= 0x38800000u) {                                                          // a normal half
        uint32_t h = ((a >> 23) - 112u) << 10 | ((a & 0x7FFFFFu) >> 13);
        const uint32_t rem = a & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;   // a carry moves into the exponent
        return (ggml_fp16_t)(sign | h);
    }
    if (a < 0x33000000u) return (ggml_fp16_t)sign;                // below 2^-25: zero
    // a subnormal half: the value in units of 2^-24, nearest, ties to even
    const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    const int shift = 126 - (int)(a >> 23);                       // 14 .. 24
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;             // 0x400 is the smallest normal's encoding
    return (ggml_fp16_t)(sign | q);
}
