/*
 * arm_neon.h — portable C stand-in for the subset of ARM NEON intrinsics that
 * the reference kernel library (csrc/libtinygiant.c) and its C test
 * (csrc/test_libtinygiant.c) use, so that those two files compile unmodified
 * on x86-64 for use as a CPU CHECKER.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped tinygiant_b200 library
 * includes this header; it exists so oracle/Makefile can build
 * oracle/_ref/libtinygiant_ref.so from the reference's own sources.
 *
 * Each intrinsic is written from the lane semantics in ARM's public
 * "Arm C Language Extensions / Neon Intrinsics Reference":
 *   - integer ops wrap (vsubq_s8, vaddq_s32) or truncate (vmovn_*);
 *   - vcvtnq_s32_f32 rounds to nearest, ties to even, and saturates;
 *   - vfmaq_f32 is a fused multiply-add (one rounding), vmlsq_f32 is an
 *     unfused multiply then subtract (two roundings);
 *   - vaddvq_f32 reduces pairwise, (a0 + a1) + (a2 + a3), as the FADDP
 *     instruction pair does;
 *   - vdotq_s32 adds, per 32-bit lane i, the four int8 products of bytes
 *     4i..4i+3 (exact in int32);
 *   - vqtbl1q_s8 returns 0 for an index >= 16.
 * Only the intrinsics those two files call are provided.
 */
#ifndef TG_NEON_SHIM_H
#define TG_NEON_SHIM_H

#include <stdint.h>
#include <string.h>
#include <math.h>

typedef struct { float v[4]; } float32x4_t;
typedef struct { int32_t v[4]; } int32x4_t;
typedef struct { int16_t v[4]; } int16x4_t;
typedef struct { int16_t v[8]; } int16x8_t;
typedef struct { int8_t v[16]; } int8x16_t;
typedef struct { uint8_t v[16]; } uint8x16_t;
typedef struct { int8_t v[8]; } int8x8_t;
typedef struct { int32_t v[2]; } int32x2_t;
typedef struct { uint16_t v[4]; } uint16x4_t;
typedef struct { uint16_t v[4]; } float16x4_t;   /* IEEE half bit patterns */

#define TGN_INLINE static inline __attribute__((always_inline))

/* ---- float32x4 ---- */
TGN_INLINE float32x4_t vdupq_n_f32(float a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a; return r; }
TGN_INLINE float32x4_t vld1q_f32(const float *p) { float32x4_t r; memcpy(r.v, p, 16); return r; }
TGN_INLINE void vst1q_f32(float *p, float32x4_t a) { memcpy(p, a.v, 16); }
TGN_INLINE float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i] + b.v[i]; return r; }
TGN_INLINE float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a.v[i] * b.v[i]; return r; }
TGN_INLINE float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = fmaf(b.v[i], c.v[i], a.v[i]); return r;
}
TGN_INLINE float32x4_t vmlsq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
    float32x4_t r;
    for (int i = 0; i < 4; i++) { float p = b.v[i] * c.v[i]; r.v[i] = a.v[i] - p; }
    return r;
}
TGN_INLINE float32x4_t vabsq_f32(float32x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = fabsf(a.v[i]); return r; }
/* FMAX: if either lane is NaN the result is NaN; otherwise the larger value. */
TGN_INLINE float tgn_fmax_nan(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    return a > b ? a : b;
}
TGN_INLINE float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b) {
    float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = tgn_fmax_nan(a.v[i], b.v[i]); return r;
}
TGN_INLINE float vmaxvq_f32(float32x4_t a) {
    return tgn_fmax_nan(tgn_fmax_nan(a.v[0], a.v[1]), tgn_fmax_nan(a.v[2], a.v[3]));
}
TGN_INLINE float vaddvq_f32(float32x4_t a) { float lo = a.v[0] + a.v[1]; float hi = a.v[2] + a.v[3]; return lo + hi; }

/* Round to nearest, ties to even, saturating to int32 (FCVTNS). */
TGN_INLINE int32_t tgn_cvtn(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    float t = truncf(x);
    float diff = x - t;                 /* exact for |x| < 2^24; 0 above that */
    int32_t i = (int32_t)t;
    if (diff > 0.5f || (diff == 0.5f && (i & 1))) i += 1;
    else if (diff < -0.5f || (diff == -0.5f && (i & 1))) i -= 1;
    return i;
}
TGN_INLINE int32x4_t vcvtnq_s32_f32(float32x4_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = tgn_cvtn(a.v[i]); return r; }

/* ---- int32x4 ---- */
TGN_INLINE int32x4_t vdupq_n_s32(int32_t a) { int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = a; return r; }
TGN_INLINE int32x4_t vaddq_s32(int32x4_t a, int32x4_t b) {
    int32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = (int32_t)((uint32_t)a.v[i] + (uint32_t)b.v[i]); return r;
}
TGN_INLINE int32_t vaddvq_s32(int32x4_t a) {
    uint32_t s = (uint32_t)a.v[0] + (uint32_t)a.v[1] + (uint32_t)a.v[2] + (uint32_t)a.v[3];
    return (int32_t)s;
}
TGN_INLINE int32x4_t vdotq_s32(int32x4_t acc, int8x16_t a, int8x16_t b) {
    int32x4_t r;
    for (int i = 0; i < 4; i++) {
        int32_t s = 0;
        for (int j = 0; j < 4; j++) s += (int32_t)a.v[4 * i + j] * (int32_t)b.v[4 * i + j];
        r.v[i] = (int32_t)((uint32_t)acc.v[i] + (uint32_t)s);
    }
    return r;
}
TGN_INLINE int16x4_t vmovn_s32(int32x4_t a) { int16x4_t r; for (int i = 0; i < 4; i++) r.v[i] = (int16_t)(uint16_t)(uint32_t)a.v[i]; return r; }
TGN_INLINE int16x8_t vcombine_s16(int16x4_t lo, int16x4_t hi) {
    int16x8_t r; for (int i = 0; i < 4; i++) { r.v[i] = lo.v[i]; r.v[4 + i] = hi.v[i]; } return r;
}
TGN_INLINE int8x8_t vmovn_s16(int16x8_t a) { int8x8_t r; for (int i = 0; i < 8; i++) r.v[i] = (int8_t)(uint8_t)(uint16_t)a.v[i]; return r; }
TGN_INLINE int32x2_t vreinterpret_s32_s8(int8x8_t a) { int32x2_t r; memcpy(r.v, a.v, 8); return r; }
#define vst1_lane_s32(p, a, lane) do { int32x2_t tgn_t_ = (a); memcpy((p), &tgn_t_.v[(lane)], 4); } while (0)

/* ---- int8x16 / uint8x16 ---- */
TGN_INLINE int8x16_t vld1q_s8(const int8_t *p) { int8x16_t r; memcpy(r.v, p, 16); return r; }
TGN_INLINE uint8x16_t vld1q_u8(const uint8_t *p) { uint8x16_t r; memcpy(r.v, p, 16); return r; }
TGN_INLINE int8x16_t vdupq_n_s8(int8_t a) { int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a; return r; }
TGN_INLINE uint8x16_t vdupq_n_u8(uint8_t a) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a; return r; }
TGN_INLINE uint8x16_t vandq_u8(uint8x16_t a, uint8x16_t b) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a.v[i] & b.v[i]; return r; }
TGN_INLINE uint8x16_t vorrq_u8(uint8x16_t a, uint8x16_t b) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = a.v[i] | b.v[i]; return r; }
#define vshrq_n_u8(a, n) tgn_shr_u8((a), (n))
#define vshlq_n_u8(a, n) tgn_shl_u8((a), (n))
TGN_INLINE uint8x16_t tgn_shr_u8(uint8x16_t a, int n) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (uint8_t)(a.v[i] >> n); return r; }
TGN_INLINE uint8x16_t tgn_shl_u8(uint8x16_t a, int n) { uint8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (uint8_t)(a.v[i] << n); return r; }
TGN_INLINE int8x16_t vsubq_s8(int8x16_t a, int8x16_t b) {
    int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = (int8_t)(uint8_t)((uint8_t)a.v[i] - (uint8_t)b.v[i]); return r;
}
TGN_INLINE int8x16_t vreinterpretq_s8_u8(uint8x16_t a) { int8x16_t r; memcpy(r.v, a.v, 16); return r; }
TGN_INLINE int8x16_t vqtbl1q_s8(int8x16_t t, uint8x16_t idx) {
    int8x16_t r; for (int i = 0; i < 16; i++) r.v[i] = idx.v[i] < 16 ? t.v[idx.v[i]] : 0; return r;
}

/* ---- half precision ---- */
TGN_INLINE uint16x4_t vld1_u16(const uint16_t *p) { uint16x4_t r; memcpy(r.v, p, 8); return r; }
TGN_INLINE float16x4_t vreinterpret_f16_u16(uint16x4_t a) { float16x4_t r; memcpy(r.v, a.v, 8); return r; }
/* Exact IEEE binary16 -> binary32 widening (every half value is representable). */
TGN_INLINE float tgn_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f; memcpy(&f, &bits, 4); return f;
}
TGN_INLINE float32x4_t vcvt_f32_f16(float16x4_t a) { float32x4_t r; for (int i = 0; i < 4; i++) r.v[i] = tgn_half_to_float(a.v[i]); return r; }

#endif /* TG_NEON_SHIM_H */
