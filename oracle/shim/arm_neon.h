/*
 * TEST INFRASTRUCTURE ONLY -- never linked into the product library.
 *
 * Scalar emulation of the subset of the Arm C Language Extensions (ACLE)
 * Advanced SIMD intrinsics that the reference CPU engine uses
 * (Int8-gemm/gemm_kernels.cpp, Int8-gemm/vec_simd.h), so that the
 * reference's own, unmodified sources compile on x86-64 and serve as the
 * parity oracle and CPU baseline.  Semantics follow the public ACLE
 * specification for each intrinsic:
 *   - vdotq_laneq_s32: 4-way signed 8-bit dot product per 32-bit lane.
 *   - vcvtnq_s32_f32:  round to nearest, ties to even, saturating.
 *   - vqmovn_*:        signed saturating narrow.
 *   - vfmaq/vfmsq:     fused multiply-add / multiply-subtract.
 *   - vmlaq_laneq_f32: multiply then add.
 * Vector types are GCC vector extensions of the matching width.
 */
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#define __fp16 _Float16

typedef float     float32x4_t __attribute__((vector_size(16)));
typedef _Float16  float16x8_t __attribute__((vector_size(16)));
typedef _Float16  float16x4_t __attribute__((vector_size(8)));
typedef int32_t   int32x4_t   __attribute__((vector_size(16)));
typedef uint32_t  uint32x4_t  __attribute__((vector_size(16)));
typedef uint64_t  uint64x2_t  __attribute__((vector_size(16)));
typedef int16_t   int16x8_t   __attribute__((vector_size(16)));
typedef int16_t   int16x4_t   __attribute__((vector_size(8)));
typedef uint16_t  uint16x8_t  __attribute__((vector_size(16)));
typedef uint16_t  uint16x4_t  __attribute__((vector_size(8)));
typedef int8_t    int8x16_t   __attribute__((vector_size(16)));
typedef int8_t    int8x8_t    __attribute__((vector_size(8)));
typedef uint8_t   uint8x16_t  __attribute__((vector_size(16)));

#define SHIM static inline __attribute__((always_inline))

/* ---- loads / stores ---- */
SHIM float32x4_t vld1q_f32(const float* p) { float32x4_t r; memcpy(&r, p, 16); return r; }
SHIM void vst1q_f32(float* p, float32x4_t v) { memcpy(p, &v, 16); }
SHIM int8x16_t vld1q_s8(const int8_t* p) { int8x16_t r; memcpy(&r, p, 16); return r; }
SHIM uint8x16_t vld1q_u8(const uint8_t* p) { uint8x16_t r; memcpy(&r, p, 16); return r; }
SHIM uint16x8_t vld1q_u16(const uint16_t* p) { uint16x8_t r; memcpy(&r, p, 16); return r; }
SHIM uint32x4_t vld1q_u32(const uint32_t* p) { uint32x4_t r; memcpy(&r, p, 16); return r; }
SHIM void vst1q_u32(uint32_t* p, uint32x4_t v) { memcpy(p, &v, 16); }
SHIM float16x8_t vld1q_f16(const _Float16* p) { float16x8_t r; memcpy(&r, p, 16); return r; }
SHIM void vst1_s8(int8_t* p, int8x8_t v) { memcpy(p, &v, 8); }

/* ---- duplicates ---- */
SHIM float32x4_t vdupq_n_f32(float x) { float32x4_t r = {x, x, x, x}; return r; }
SHIM int32x4_t vdupq_n_s32(int32_t x) { int32x4_t r = {x, x, x, x}; return r; }
SHIM uint32x4_t vdupq_n_u32(uint32_t x) { uint32x4_t r = {x, x, x, x}; return r; }
SHIM uint8x16_t vdupq_n_u8(uint8_t x) { uint8x16_t r; for (int i = 0; i < 16; ++i) r[i] = x; return r; }
SHIM int8x16_t vdupq_n_s8(int8_t x) { int8x16_t r; for (int i = 0; i < 16; ++i) r[i] = x; return r; }

/* ---- float arithmetic ---- */
SHIM float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) { return a + b; }
SHIM float32x4_t vsubq_f32(float32x4_t a, float32x4_t b) { return a - b; }
SHIM float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) { return a * b; }
SHIM float32x4_t vdivq_f32(float32x4_t a, float32x4_t b) { return a / b; }
SHIM float32x4_t vnegq_f32(float32x4_t a) { return -a; }
SHIM float32x4_t vmulq_n_f32(float32x4_t a, float s) { return a * s; }
SHIM float32x4_t vabsq_f32(float32x4_t a) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r[i] = fabsf(a[i]); return r;
}
SHIM float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r[i] = a[i] > b[i] ? a[i] : b[i]; return r;
}
SHIM float vmaxvq_f32(float32x4_t a) {
    float m = a[0]; for (int i = 1; i < 4; ++i) m = a[i] > m ? a[i] : m; return m;
}
SHIM float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r[i] = fmaf(b[i], c[i], a[i]); return r;
}
SHIM float32x4_t vfmsq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r[i] = fmaf(-b[i], c[i], a[i]); return r;
}
#define vmlaq_laneq_f32(a, b, v, lane) ((a) + (b) * (v)[(lane)])

/* ---- conversions ---- */
SHIM float32x4_t vcvtq_f32_s32(int32x4_t a) {
    float32x4_t r; for (int i = 0; i < 4; ++i) r[i] = (float)a[i]; return r;
}
SHIM int32x4_t vcvtnq_s32_f32(float32x4_t a) {
    int32x4_t r;
    for (int i = 0; i < 4; ++i) {
        float x = a[i];
        if (x != x) { r[i] = 0; continue; }
        if (x >= 2147483648.0f) { r[i] = INT32_MAX; continue; }
        if (x < -2147483648.0f) { r[i] = INT32_MIN; continue; }
        r[i] = (int32_t)nearbyintf(x);  /* default rounding mode: ties to even */
    }
    return r;
}
SHIM int16x4_t vqmovn_s32(int32x4_t a) {
    int16x4_t r;
    for (int i = 0; i < 4; ++i) r[i] = (int16_t)(a[i] > 32767 ? 32767 : (a[i] < -32768 ? -32768 : a[i]));
    return r;
}
SHIM int16x8_t vcombine_s16(int16x4_t lo, int16x4_t hi) {
    int16x8_t r; for (int i = 0; i < 4; ++i) { r[i] = lo[i]; r[i + 4] = hi[i]; } return r;
}
SHIM int8x8_t vqmovn_s16(int16x8_t a) {
    int8x8_t r;
    for (int i = 0; i < 8; ++i) r[i] = (int8_t)(a[i] > 127 ? 127 : (a[i] < -128 ? -128 : a[i]));
    return r;
}
SHIM float16x4_t vget_low_f16(float16x8_t a) { float16x4_t r; for (int i = 0; i < 4; ++i) r[i] = a[i]; return r; }
SHIM float16x4_t vget_high_f16(float16x8_t a) { float16x4_t r; for (int i = 0; i < 4; ++i) r[i] = a[i + 4]; return r; }
SHIM float32x4_t vcvt_f32_f16(float16x4_t a) { float32x4_t r; for (int i = 0; i < 4; ++i) r[i] = (float)a[i]; return r; }
SHIM uint16x4_t vget_low_u16(uint16x8_t a) { uint16x4_t r; for (int i = 0; i < 4; ++i) r[i] = a[i]; return r; }
SHIM uint16x4_t vget_high_u16(uint16x8_t a) { uint16x4_t r; for (int i = 0; i < 4; ++i) r[i] = a[i + 4]; return r; }
#define vshll_n_u16(a, n) __extension__({ uint16x4_t _a = (a); uint32x4_t _r; \
    for (int _i = 0; _i < 4; ++_i) _r[_i] = ((uint32_t)_a[_i]) << (n); _r; })

/* ---- reinterpret casts ---- */
SHIM float32x4_t vreinterpretq_f32_u32(uint32x4_t a) { float32x4_t r; memcpy(&r, &a, 16); return r; }
SHIM uint32x4_t vreinterpretq_u32_f32(float32x4_t a) { uint32x4_t r; memcpy(&r, &a, 16); return r; }
SHIM int8x16_t vreinterpretq_s8_u8(uint8x16_t a) { int8x16_t r; memcpy(&r, &a, 16); return r; }
SHIM uint64x2_t vreinterpretq_u64_u32(uint32x4_t a) { uint64x2_t r; memcpy(&r, &a, 16); return r; }

/* ---- integer ops ---- */
SHIM uint32x4_t vandq_u32(uint32x4_t a, uint32x4_t b) { return a & b; }
SHIM uint32x4_t vorrq_u32(uint32x4_t a, uint32x4_t b) { return a | b; }
SHIM uint32x4_t vaddq_u32(uint32x4_t a, uint32x4_t b) { return a + b; }
SHIM uint32x4_t vsubq_u32(uint32x4_t a, uint32x4_t b) { return a - b; }
SHIM uint8x16_t vandq_u8(uint8x16_t a, uint8x16_t b) { return a & b; }
SHIM int8x16_t vsubq_s8(int8x16_t a, int8x16_t b) { return a - b; }
#define vshlq_n_u32(a, n) ((uint32x4_t)((a) << (n)))
#define vshrq_n_u32(a, n) ((uint32x4_t)((a) >> (n)))
#define vshrq_n_u8(a, n)  ((uint8x16_t)((a) >> (n)))
#define vgetq_lane_u32(a, lane) ((uint32_t)(a)[(lane)])

/* ---- comparisons / select ---- */
SHIM uint32x4_t vcagtq_f32(float32x4_t a, float32x4_t b) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r[i] = fabsf(a[i]) > fabsf(b[i]) ? 0xFFFFFFFFu : 0u; return r;
}
SHIM uint32x4_t vclezq_f32(float32x4_t a) {
    uint32x4_t r; for (int i = 0; i < 4; ++i) r[i] = a[i] <= 0.0f ? 0xFFFFFFFFu : 0u; return r;
}
SHIM float32x4_t vbslq_f32(uint32x4_t m, float32x4_t a, float32x4_t b) {
    uint32x4_t ua, ub; memcpy(&ua, &a, 16); memcpy(&ub, &b, 16);
    uint32x4_t ur = (m & ua) | (~m & ub);
    float32x4_t r; memcpy(&r, &ur, 16); return r;
}

/* ---- dot product: acc[i] += sum_j b[4i+j] * a[4*lane+j] (signed 8-bit) ---- */
#define vdotq_laneq_s32(acc, b, a, lane) __extension__({                        \
    int32x4_t _acc = (acc); int8x16_t _b = (b); int8x16_t _a = (a);           \
    for (int _i = 0; _i < 4; ++_i) {                                          \
        int32_t _s = 0;                                                       \
        for (int _j = 0; _j < 4; ++_j)                                        \
            _s += (int32_t)_b[4 * _i + _j] * (int32_t)_a[4 * (lane) + _j];    \
        _acc[_i] += _s;                                                       \
    }                                                                         \
    _acc; })
