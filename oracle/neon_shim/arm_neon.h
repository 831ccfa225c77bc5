/* Portable restatement of the ARM NEON intrinsics that the reference's kernels use, so that
 * the reference's own kernel sources (cactus/kernel/*.cpp) compile on an x86-64 host for use
 * as a CPU oracle. TEST INFRASTRUCTURE ONLY: nothing on the product path includes this.
 *
 * Every intrinsic is written lane by lane from its architectural definition (the ARM
 * Architecture Reference Manual's pseudocode for the instruction it maps to), with IEEE
 * round-to-nearest-even and no flush-to-zero (the Linux / Apple default FPCR):
 *   - fp16 add / sub / mul / div: computed in float and rounded once to fp16 — float has
 *     24 >= 2*11 + 2 significand bits, so this equals the correctly rounded fp16 result;
 *   - fp16 fused multiply-add: exact product in double, TwoSum for the addition, and a
 *     midpoint correction when the double sum sits exactly halfway between two fp16 values;
 *   - fp32 FMLA / FMLS: fmaf; FADDP-based across-lane adds in pairwise order;
 *   - FCVTNS / FCVTZS: round to nearest even / toward zero, saturating, NaN -> 0.
 * The reference's __fp16 scalar type is compiled as GCC's _Float16 without native fp16
 * instructions, whose excess-precision rule (evaluate in float, round on assignment and
 * cast) is the ACLE rule for __fp16 arithmetic.
 */
#ifndef CACTUS_ORACLE_NEON_SHIM_H
#define CACTUS_ORACLE_NEON_SHIM_H

#include <stdint.h>
#include <string.h>
#include <math.h>

#ifdef __cplusplus
#define NS_INLINE static inline __attribute__((always_inline))
#else
#define NS_INLINE static inline
/* kernel_utils.h declares accum_matmul (SMMLA) only for Android and Apple aarch64 but calls
 * it behind cactus_has_i8mm(), which is false elsewhere; this declaration lets the file
 * compile and is never reached on this host (the integer results are the same either way). */
#ifdef __cplusplus
NS_INLINE int32x4_t accum_matmul(int32x4_t acc, int8x16_t a, int8x16_t b) { return vmmlaq_s32(acc, a, b); }
#endif

#endif

typedef _Float16 float16_t;
typedef float float32_t;

typedef _Float16 float16x4_t __attribute__((vector_size(8)));
typedef _Float16 float16x8_t __attribute__((vector_size(16)));
typedef float float32x2_t __attribute__((vector_size(8)));
typedef float float32x4_t __attribute__((vector_size(16)));
typedef int8_t int8x8_t __attribute__((vector_size(8)));
typedef int8_t int8x16_t __attribute__((vector_size(16)));
typedef uint8_t uint8x8_t __attribute__((vector_size(8)));
typedef uint8_t uint8x16_t __attribute__((vector_size(16)));
typedef int16_t int16x4_t __attribute__((vector_size(8)));
typedef int16_t int16x8_t __attribute__((vector_size(16)));
typedef uint16_t uint16x8_t __attribute__((vector_size(16)));
typedef int32_t int32x2_t __attribute__((vector_size(8)));
typedef int32_t int32x4_t __attribute__((vector_size(16)));
typedef uint32_t uint32x4_t __attribute__((vector_size(16)));
typedef int64_t int64x2_t __attribute__((vector_size(16)));

typedef struct { float16x8_t val[2]; } float16x8x2_t;
typedef struct { float16x4_t val[2]; } float16x4x2_t;
typedef struct { float32x4_t val[2]; } float32x4x2_t;
typedef struct { int8x16_t val[2]; } int8x16x2_t;

/* ---- scalar helpers ---- */
NS_INLINE _Float16 ns_h(float x) { return (_Float16)x; } /* float -> fp16, RNE */
NS_INLINE float ns_f(_Float16 h) { return (float)h; }

/* fp16 RNE rounding of an exact value x = s + e, where s = fl64(x) and e is the exact error
 * (TwoSum). Rounding s directly is correct unless s lies exactly halfway between two fp16
 * values (both halfway points and fp16 values are doubles); then the sign of e decides. */
NS_INLINE uint16_t ns_hbits(_Float16 h) { uint16_t u; memcpy(&u, &h, 2); return u; }
NS_INLINE _Float16 ns_bitsh(uint16_t u) { _Float16 h; memcpy(&h, &u, 2); return h; }
NS_INLINE _Float16 ns_round_h_exact(double s, double e) {
    const _Float16 r = (_Float16)s;
    if (e == 0.0 || !isfinite(s)) return r;
    double rd = (double)r;
    if (rd == s) return r;
    if (isinf(rd)) rd = copysign(65536.0, s); /* the value one step past the largest finite */
    const uint16_t u = ns_hbits(r);
    uint16_t v; /* the fp16 neighbour of r on the side of s */
    if (s > rd) v = (u == 0x8000u) ? 0x0001u : ((u & 0x8000u) ? (uint16_t)(u - 1) : (uint16_t)(u + 1));
    else v = (u == 0x0000u) ? 0x8001u : ((u & 0x8000u) ? (uint16_t)(u + 1) : (uint16_t)(u - 1));
    if (isinf((double)r)) v = (s > 0) ? 0x7BFFu : 0xFBFFu;
    const _Float16 other = ns_bitsh(v);
    const double od = (double)other;
    if (s != (rd + od) * 0.5) return r;
    const int want_larger = e > 0.0;
    const int other_larger = od > rd;
    return (want_larger == other_larger) ? other : r;
}

/* fused fp16 a + b*c with a single rounding */
NS_INLINE _Float16 ns_fma_h(_Float16 a, _Float16 b, _Float16 c) {
    const double p = (double)b * (double)c; /* exact: 11 x 11 bits */
    const double x = (double)a;
    const double s = p + x;
    const double bb = s - p;
    const double e = (p - (s - bb)) + (x - bb); /* TwoSum error */
    return ns_round_h_exact(s, e);
}

NS_INLINE int32_t ns_cvtn_s32(float x) { /* FCVTNS */
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)nearbyintf(x);
}
NS_INLINE int32_t ns_cvtz_s32(float x) { /* FCVTZS */
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}
NS_INLINE float ns_fmax(float a, float b) { return (a != a || b != b) ? NAN : (a > b ? a : (b > a ? b : (signbit(a) ? b : a))); }
NS_INLINE float ns_fmin(float a, float b) { return (a != a || b != b) ? NAN : (a < b ? a : (b < a ? b : (signbit(a) ? a : b))); }

#define NS_MAP1(T, N, expr) { T r_; for (int i = 0; i < N; ++i) r_[i] = (expr); return r_; }

/* ---- loads / stores / construction ---- */
NS_INLINE float16x8_t vld1q_f16(const _Float16* p) { float16x8_t r; memcpy(&r, p, 16); return r; }
NS_INLINE float16x4_t vld1_f16(const _Float16* p) { float16x4_t r; memcpy(&r, p, 8); return r; }
NS_INLINE float32x4_t vld1q_f32(const float* p) { float32x4_t r; memcpy(&r, p, 16); return r; }
NS_INLINE int8x16_t vld1q_s8(const int8_t* p) { int8x16_t r; memcpy(&r, p, 16); return r; }
NS_INLINE int8x8_t vld1_s8(const int8_t* p) { int8x8_t r; memcpy(&r, p, 8); return r; }
NS_INLINE uint8x16_t vld1q_u8(const uint8_t* p) { uint8x16_t r; memcpy(&r, p, 16); return r; }
NS_INLINE void vst1q_f16(_Float16* p, float16x8_t v) { memcpy(p, &v, 16); }
NS_INLINE void vst1_f16(_Float16* p, float16x4_t v) { memcpy(p, &v, 8); }
NS_INLINE void vst1q_f32(float* p, float32x4_t v) { memcpy(p, &v, 16); }
NS_INLINE void vst1q_s8(int8_t* p, int8x16_t v) { memcpy(p, &v, 16); }
NS_INLINE void vst1_s8(int8_t* p, int8x8_t v) { memcpy(p, &v, 8); }

NS_INLINE float16x8_t vdupq_n_f16(_Float16 x) NS_MAP1(float16x8_t, 8, x)
NS_INLINE float16x4_t vdup_n_f16(_Float16 x) NS_MAP1(float16x4_t, 4, x)
NS_INLINE float32x4_t vdupq_n_f32(float x) NS_MAP1(float32x4_t, 4, x)
NS_INLINE int32x4_t vdupq_n_s32(int32_t x) NS_MAP1(int32x4_t, 4, x)
NS_INLINE uint8x16_t vdupq_n_u8(uint8_t x) NS_MAP1(uint8x16_t, 16, x)
NS_INLINE int8x16_t vdupq_n_s8(int8_t x) NS_MAP1(int8x16_t, 16, x)

NS_INLINE float16x4_t vget_low_f16(float16x8_t v) NS_MAP1(float16x4_t, 4, v[i])
NS_INLINE float16x4_t vget_high_f16(float16x8_t v) NS_MAP1(float16x4_t, 4, v[i + 4])
NS_INLINE float32x2_t vget_low_f32(float32x4_t v) NS_MAP1(float32x2_t, 2, v[i])
NS_INLINE float32x2_t vget_high_f32(float32x4_t v) NS_MAP1(float32x2_t, 2, v[i + 2])
NS_INLINE int8x8_t vget_low_s8(int8x16_t v) NS_MAP1(int8x8_t, 8, v[i])
NS_INLINE int8x8_t vget_high_s8(int8x16_t v) NS_MAP1(int8x8_t, 8, v[i + 8])
NS_INLINE int16x4_t vget_low_s16(int16x8_t v) NS_MAP1(int16x4_t, 4, v[i])
NS_INLINE int16x4_t vget_high_s16(int16x8_t v) NS_MAP1(int16x4_t, 4, v[i + 4])
NS_INLINE float16x8_t vcombine_f16(float16x4_t a, float16x4_t b) NS_MAP1(float16x8_t, 8, i < 4 ? a[i] : b[i - 4])
NS_INLINE float32x4_t vcombine_f32(float32x2_t a, float32x2_t b) NS_MAP1(float32x4_t, 4, i < 2 ? a[i] : b[i - 2])
NS_INLINE int8x16_t vcombine_s8(int8x8_t a, int8x8_t b) NS_MAP1(int8x16_t, 16, i < 8 ? a[i] : b[i - 8])
NS_INLINE int16x8_t vcombine_s16(int16x4_t a, int16x4_t b) NS_MAP1(int16x8_t, 8, i < 4 ? a[i] : b[i - 4])

#define vgetq_lane_f16(v, n) ((_Float16)((v)[(n)]))
#define vget_lane_f16(v, n) ((_Float16)((v)[(n)]))
#define vgetq_lane_s32(v, n) ((int32_t)((v)[(n)]))
#define vgetq_lane_f32(v, n) ((float)((v)[(n)]))
#define vget_lane_f32(v, n) ((float)((v)[(n)]))
NS_INLINE float16x8_t ns_setq_lane_f16(_Float16 x, float16x8_t v, int n) { v[n] = x; return v; }
#define vsetq_lane_f16(x, v, n) ns_setq_lane_f16((x), (v), (n))

/* ---- bit casts ---- */
#define NS_REINTERPRET(name, TO, FROM) NS_INLINE TO name(FROM v) { TO r; memcpy(&r, &v, sizeof(r)); return r; }
NS_REINTERPRET(vreinterpretq_f16_f32, float16x8_t, float32x4_t)
NS_REINTERPRET(vreinterpretq_f32_f16, float32x4_t, float16x8_t)
NS_REINTERPRET(vreinterpretq_f32_s32, float32x4_t, int32x4_t)
NS_REINTERPRET(vreinterpretq_f32_u32, float32x4_t, uint32x4_t)
NS_REINTERPRET(vreinterpretq_s32_u32, int32x4_t, uint32x4_t)
NS_REINTERPRET(vreinterpretq_u32_f32, uint32x4_t, float32x4_t)
NS_REINTERPRET(vreinterpretq_s8_u8, int8x16_t, uint8x16_t)
NS_REINTERPRET(vreinterpretq_u8_s8, uint8x16_t, int8x16_t)
NS_REINTERPRET(vreinterpretq_s32_f32, int32x4_t, float32x4_t)

/* ---- fp16 arithmetic (one rounding per lane) ---- */
NS_INLINE float16x8_t vaddq_f16(float16x8_t a, float16x8_t b) NS_MAP1(float16x8_t, 8, ns_h(ns_f(a[i]) + ns_f(b[i])))
NS_INLINE float16x8_t vsubq_f16(float16x8_t a, float16x8_t b) NS_MAP1(float16x8_t, 8, ns_h(ns_f(a[i]) - ns_f(b[i])))
NS_INLINE float16x8_t vmulq_f16(float16x8_t a, float16x8_t b) NS_MAP1(float16x8_t, 8, ns_h(ns_f(a[i]) * ns_f(b[i])))
NS_INLINE float16x8_t vdivq_f16(float16x8_t a, float16x8_t b) NS_MAP1(float16x8_t, 8, ns_h(ns_f(a[i]) / ns_f(b[i])))
NS_INLINE float16x4_t vadd_f16(float16x4_t a, float16x4_t b) NS_MAP1(float16x4_t, 4, ns_h(ns_f(a[i]) + ns_f(b[i])))
NS_INLINE float16x8_t vmaxq_f16(float16x8_t a, float16x8_t b) NS_MAP1(float16x8_t, 8, ns_h(ns_fmax(ns_f(a[i]), ns_f(b[i]))))
NS_INLINE float16x8_t vminq_f16(float16x8_t a, float16x8_t b) NS_MAP1(float16x8_t, 8, ns_h(ns_fmin(ns_f(a[i]), ns_f(b[i]))))
NS_INLINE float16x8_t vfmaq_f16(float16x8_t a, float16x8_t b, float16x8_t c) NS_MAP1(float16x8_t, 8, ns_fma_h(a[i], b[i], c[i]))
NS_INLINE float16x8_t vfmsq_f16(float16x8_t a, float16x8_t b, float16x8_t c) NS_MAP1(float16x8_t, 8, ns_fma_h(a[i], (_Float16)(-ns_f(b[i])), c[i]))
NS_INLINE float16x4_t vext_f16(float16x4_t a, float16x4_t b, int n) NS_MAP1(float16x4_t, 4, (i + n < 4) ? a[i + n] : b[i + n - 4])
NS_INLINE float16x8x2_t vtrnq_f16(float16x8_t a, float16x8_t b) {
    float16x8x2_t r;
    for (int i = 0; i < 4; ++i) {
        r.val[0][2 * i] = a[2 * i]; r.val[0][2 * i + 1] = b[2 * i];
        r.val[1][2 * i] = a[2 * i + 1]; r.val[1][2 * i + 1] = b[2 * i + 1];
    }
    return r;
}

/* ---- conversions ---- */
NS_INLINE float32x4_t vcvt_f32_f16(float16x4_t v) NS_MAP1(float32x4_t, 4, ns_f(v[i]))
NS_INLINE float16x4_t vcvt_f16_f32(float32x4_t v) NS_MAP1(float16x4_t, 4, ns_h(v[i]))
NS_INLINE int32x4_t vcvtnq_s32_f32(float32x4_t v) NS_MAP1(int32x4_t, 4, ns_cvtn_s32(v[i]))
NS_INLINE int32x4_t vcvtq_s32_f32(float32x4_t v) NS_MAP1(int32x4_t, 4, ns_cvtz_s32(v[i]))
NS_INLINE float32x4_t vcvtq_f32_s32(int32x4_t v) NS_MAP1(float32x4_t, 4, (float)v[i])

/* ---- fp32 arithmetic ---- */
NS_INLINE float32x4_t vaddq_f32(float32x4_t a, float32x4_t b) NS_MAP1(float32x4_t, 4, a[i] + b[i])
NS_INLINE float32x2_t vadd_f32(float32x2_t a, float32x2_t b) NS_MAP1(float32x2_t, 2, a[i] + b[i])
NS_INLINE float32x4_t vsubq_f32(float32x4_t a, float32x4_t b) NS_MAP1(float32x4_t, 4, a[i] - b[i])
NS_INLINE float32x4_t vmulq_f32(float32x4_t a, float32x4_t b) NS_MAP1(float32x4_t, 4, a[i] * b[i])
NS_INLINE float32x4_t vmulq_n_f32(float32x4_t a, float b) NS_MAP1(float32x4_t, 4, a[i] * b)
NS_INLINE float32x4_t vdivq_f32(float32x4_t a, float32x4_t b) NS_MAP1(float32x4_t, 4, a[i] / b[i])
NS_INLINE float32x4_t vsqrtq_f32(float32x4_t a) NS_MAP1(float32x4_t, 4, sqrtf(a[i]))
NS_INLINE float32x4_t vabsq_f32(float32x4_t a) NS_MAP1(float32x4_t, 4, fabsf(a[i]))
NS_INLINE float32x4_t vnegq_f32(float32x4_t a) NS_MAP1(float32x4_t, 4, -a[i])
NS_INLINE float32x4_t vmaxq_f32(float32x4_t a, float32x4_t b) NS_MAP1(float32x4_t, 4, ns_fmax(a[i], b[i]))
NS_INLINE float32x4_t vminq_f32(float32x4_t a, float32x4_t b) NS_MAP1(float32x4_t, 4, ns_fmin(a[i], b[i]))
NS_INLINE float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) NS_MAP1(float32x4_t, 4, fmaf(b[i], c[i], a[i]))
NS_INLINE float32x4_t vfmaq_n_f32(float32x4_t a, float32x4_t b, float c) NS_MAP1(float32x4_t, 4, fmaf(b[i], c, a[i]))
NS_INLINE float vaddvq_f32(float32x4_t v) { return (v[0] + v[1]) + (v[2] + v[3]); }
NS_INLINE float vmaxvq_f32(float32x4_t v) { return ns_fmax(ns_fmax(v[0], v[1]), ns_fmax(v[2], v[3])); }
NS_INLINE float32x4x2_t vtrnq_f32(float32x4_t a, float32x4_t b) {
    float32x4x2_t r;
    r.val[0][0] = a[0]; r.val[0][1] = b[0]; r.val[0][2] = a[2]; r.val[0][3] = b[2];
    r.val[1][0] = a[1]; r.val[1][1] = b[1]; r.val[1][2] = a[3]; r.val[1][3] = b[3];
    return r;
}
NS_INLINE uint32x4_t vceqq_f32(float32x4_t a, float32x4_t b) NS_MAP1(uint32x4_t, 4, a[i] == b[i] ? 0xFFFFFFFFu : 0u)
NS_INLINE uint32x4_t vcgtq_f32(float32x4_t a, float32x4_t b) NS_MAP1(uint32x4_t, 4, a[i] > b[i] ? 0xFFFFFFFFu : 0u)
NS_INLINE uint32x4_t vcltq_f32(float32x4_t a, float32x4_t b) NS_MAP1(uint32x4_t, 4, a[i] < b[i] ? 0xFFFFFFFFu : 0u)
NS_INLINE float32x4_t vbslq_f32(uint32x4_t m, float32x4_t a, float32x4_t b) {
    uint32x4_t ua, ub, r;
    memcpy(&ua, &a, 16); memcpy(&ub, &b, 16);
    for (int i = 0; i < 4; ++i) r[i] = (m[i] & ua[i]) | (~m[i] & ub[i]);
    float32x4_t f; memcpy(&f, &r, 16); return f;
}

/* ---- integer ---- */
NS_INLINE int32x4_t vaddq_s32(int32x4_t a, int32x4_t b) NS_MAP1(int32x4_t, 4, (int32_t)((uint32_t)a[i] + (uint32_t)b[i]))
NS_INLINE int32x4_t vsubq_s32(int32x4_t a, int32x4_t b) NS_MAP1(int32x4_t, 4, (int32_t)((uint32_t)a[i] - (uint32_t)b[i]))
NS_INLINE int32x4_t vandq_s32(int32x4_t a, int32x4_t b) NS_MAP1(int32x4_t, 4, a[i] & b[i])
NS_INLINE uint32x4_t vandq_u32(uint32x4_t a, uint32x4_t b) NS_MAP1(uint32x4_t, 4, a[i] & b[i])
NS_INLINE uint8x16_t vandq_u8(uint8x16_t a, uint8x16_t b) NS_MAP1(uint8x16_t, 16, (uint8_t)(a[i] & b[i]))
NS_INLINE uint8x16_t vsubq_u8(uint8x16_t a, uint8x16_t b) NS_MAP1(uint8x16_t, 16, (uint8_t)(a[i] - b[i]))
NS_INLINE uint8x16_t vcgtq_u8(uint8x16_t a, uint8x16_t b) NS_MAP1(uint8x16_t, 16, (uint8_t)(a[i] > b[i] ? 0xFF : 0))
NS_INLINE uint8x16_t ns_shrq_n_u8(uint8x16_t a, int n) NS_MAP1(uint8x16_t, 16, (uint8_t)(a[i] >> n))
#define vshrq_n_u8(a, n) ns_shrq_n_u8((a), (n))
NS_INLINE int32x4_t ns_shlq_n_s32(int32x4_t a, int n) NS_MAP1(int32x4_t, 4, (int32_t)((uint32_t)a[i] << n))
#define vshlq_n_s32(a, n) ns_shlq_n_s32((a), (n))
NS_INLINE int32_t vaddvq_s32(int32x4_t v) { return (int32_t)((uint32_t)v[0] + (uint32_t)v[1] + (uint32_t)v[2] + (uint32_t)v[3]); }
NS_INLINE int16x8_t vmovl_s8(int8x8_t v) NS_MAP1(int16x8_t, 8, (int16_t)v[i])
NS_INLINE int32x4_t vmovl_s16(int16x4_t v) NS_MAP1(int32x4_t, 4, (int32_t)v[i])
NS_INLINE int16x8_t vmull_s8(int8x8_t a, int8x8_t b) NS_MAP1(int16x8_t, 8, (int16_t)((int)a[i] * (int)b[i]))
NS_INLINE int32x4_t vpaddlq_s16(int16x8_t v) NS_MAP1(int32x4_t, 4, (int32_t)v[2 * i] + (int32_t)v[2 * i + 1])
NS_INLINE int16x4_t vqmovn_s32(int32x4_t v) NS_MAP1(int16x4_t, 4, (int16_t)(v[i] > 32767 ? 32767 : (v[i] < -32768 ? -32768 : v[i])))
NS_INLINE int8x8_t vqmovn_s16(int16x8_t v) NS_MAP1(int8x8_t, 8, (int8_t)(v[i] > 127 ? 127 : (v[i] < -128 ? -128 : v[i])))
NS_INLINE int32x4_t vdotq_s32(int32x4_t acc, int8x16_t a, int8x16_t b) {
    for (int i = 0; i < 4; ++i) {
        int32_t s = 0;
        for (int j = 0; j < 4; ++j) s += (int32_t)a[4 * i + j] * (int32_t)b[4 * i + j];
        acc[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)s);
    }
    return acc;
}
/* SMMLA: a = 2x8 (row-major), b = 2x8 (row j = column j of the 8x2 operand), acc 2x2 */
NS_INLINE int32x4_t vmmlaq_s32(int32x4_t acc, int8x16_t a, int8x16_t b) {
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            int32_t s = 0;
            for (int k = 0; k < 8; ++k) s += (int32_t)a[8 * i + k] * (int32_t)b[8 * j + k];
            acc[2 * i + j] = (int32_t)((uint32_t)acc[2 * i + j] + (uint32_t)s);
        }
    return acc;
}
NS_INLINE int8x16x2_t vzipq_s8(int8x16_t a, int8x16_t b) {
    int8x16x2_t r;
    for (int i = 0; i < 8; ++i) {
        r.val[0][2 * i] = a[i]; r.val[0][2 * i + 1] = b[i];
        r.val[1][2 * i] = a[i + 8]; r.val[1][2 * i + 1] = b[i + 8];
    }
    return r;
}

/* kernel_utils.h declares accum_matmul (SMMLA) only for Android and Apple aarch64 but calls
 * it behind cactus_has_i8mm(), which is false elsewhere; this declaration lets the file
 * compile and is never reached on this host (the integer results are the same either way). */
#ifdef __cplusplus
NS_INLINE int32x4_t accum_matmul(int32x4_t acc, int8x16_t a, int8x16_t b) { return vmmlaq_s32(acc, a, b); }
#endif

#endif
