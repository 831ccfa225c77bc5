/*
 * refcpu.c — CPU restatement of the Cactus reference kernels (TEST INFRASTRUCTURE).
 *
 * Used only as the parity checker (tests/, smoke()) and as the timed CPU
 * baseline (bench.py cpu_baseline / --impl reference). The product library
 * never links or calls it. Build: oracle/Makefile (gcc -O3 -ffp-contract=off
 * -fopenmp); all fused multiply-adds below are explicit fmaf() calls placed
 * where the reference's NEON code (or its compiler-contracted `acc += a * b`)
 * fuses. See refcpu.h for the per-function reference citations.
 */
#include "refcpu.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

static int g_threads = 0;

void ref_set_threads(int n) { g_threads = n; }
int ref_get_threads(void) { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

/* ---------------------------------------------------------------- fp16 helpers */
float ref_f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}
uint16_t ref_f32_to_f16(float f) {
    _Float16 v = (_Float16)f; /* round to nearest even */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}
static inline float h2f(uint16_t h) { return ref_f16_to_f32(h); }
static inline uint16_t f2h(float f) { return ref_f32_to_f16(f); }
static inline uint16_t d2h(double d) {
    _Float16 v = (_Float16)d; /* direct double -> binary16 rounding (libgcc __truncdfhf2) */
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}
/* one-rounding fp16 arithmetic, as NEON vaddq_f16 / vmulq_f16 / vfmaq_f16 */
static inline uint16_t hadd(uint16_t a, uint16_t b) { return d2h((double)h2f(a) + (double)h2f(b)); }
static inline uint16_t hmul(uint16_t a, uint16_t b) { return d2h((double)h2f(a) * (double)h2f(b)); }
static inline uint16_t hfma(uint16_t a, uint16_t b, uint16_t c) { /* a*b + c, fused */
    return d2h(fma((double)h2f(a), (double)h2f(b), (double)h2f(c)));
}
/* exp / tanh rounded once from double precision (the CUDA path computes the same expression;
 * both equal a correctly rounded expf/tanhf except in vanishingly rare cases) */
static inline float expf_cr(float x) { return (float)exp((double)x); }
static inline float tanhf_cr(float x) { return (float)tanh((double)x); }
static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* vcvtq_s32_f32: truncate toward zero, saturating, NaN -> 0 */
static inline int32_t cvt_trunc_sat(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return 2147483647;
    if (x <= -2147483648.0f) return (int32_t)0x80000000u;
    return (int32_t)x;
}
/* vcvtnq_s32_f32: round half to even, saturating */
static inline int32_t cvt_rne_sat(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return 2147483647;
    if (x <= -2147483648.0f) return (int32_t)0x80000000u;
    return (int32_t)nearbyintf(x); /* default rounding mode: to nearest even */
}
static inline int8_t sat8(int32_t v) { return (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v)); }

/* ---------------------------------------------------------------- activation quantization */
float ref_fp16_max_abs(const uint16_t* src, size_t count) {
    float m = 0.0f;
    for (size_t i = 0; i < count; ++i) {
        float a = fabsf(h2f(src[i]));
        m = a > m ? a : m;
    }
    return m;
}

void ref_fp16_to_int8(const uint16_t* src, int8_t* dst, size_t count, float scale) {
    const float inv = 1.0f / scale;
    const size_t vec_end = (count / 8) * 8;
    for (size_t i = 0; i < vec_end; ++i) {
        float v = h2f(src[i]) * inv;
        v = fmaxf(fminf(v, 127.0f), -128.0f);
        dst[i] = sat8(cvt_rne_sat(v));
    }
    for (size_t i = vec_end; i < count; ++i) {
        float v = h2f(src[i]) * inv;
        dst[i] = (int8_t)roundf(fmaxf(-128.0f, fminf(127.0f, v))); /* std::round: half away from zero */
    }
}

void ref_quantize_activations(const uint16_t* x, int8_t* q, float* scales, size_t M, size_t K) {
    for (size_t m = 0; m < M; ++m) {
        float max_abs = ref_fp16_max_abs(x + m * K, K);
        float scale = max_abs / 127.0f;
        if (scale < 1e-10f) scale = 1e-10f;
        scales[m] = scale;
        ref_fp16_to_int8(x + m * K, q + m * K, K, scale);
    }
}

/* ---------------------------------------------------------------- quantized matmul */
void ref_matmul_int8(const int8_t* A, const float* As, const int8_t* B, const uint16_t* Bs,
                     uint16_t* C, size_t M, size_t K, size_t N, size_t G) {
    const size_t ng = K / G;
#pragma omp parallel for schedule(static) num_threads(ref_get_threads())
    for (size_t n = 0; n < N; ++n) {
        const int8_t* b = B + n * K;
        const uint16_t* bs = Bs + n * ng;
        for (size_t m = 0; m < M; ++m) {
            const int8_t* a = A + m * K;
            float run = 0.0f;
            for (size_t g = 0; g < ng; ++g) {
                int32_t s = 0;
                const int8_t* ag = a + g * G;
                const int8_t* bg = b + g * G;
                for (size_t k = 0; k < G; ++k) s += (int32_t)ag[k] * (int32_t)bg[k];
                run = fmaf((float)s, h2f(bs[g]), run); /* running_sum += group_acc * b_scale (contracted) */
            }
            C[m * N + n] = f2h(run * As[m]);
        }
    }
}

static inline int8_t nib_lo(uint8_t b) { int8_t v = (int8_t)(b & 0x0F); return (v & 0x08) ? (int8_t)(v | 0xF0) : v; }
static inline int8_t nib_hi(uint8_t b) { int8_t v = (int8_t)((b >> 4) & 0x0F); return (v & 0x08) ? (int8_t)(v | 0xF0) : v; }

void ref_unpack_int4(const uint8_t* packed, int8_t* out, size_t count) {
    for (size_t i = 0; i < count; ++i) {
        uint8_t b = packed[i / 2];
        out[i] = (i & 1) ? nib_hi(b) : nib_lo(b);
    }
}

void ref_matmul_int4(const int8_t* A, const float* As, const uint8_t* Bp, const uint16_t* Bs,
                     uint16_t* C, size_t M, size_t K, size_t N, size_t G) {
    const size_t ng = K / G;
#pragma omp parallel num_threads(ref_get_threads())
    {
        int8_t* row = (int8_t*)malloc(K);
#pragma omp for schedule(static)
        for (size_t n = 0; n < N; ++n) {
            ref_unpack_int4(Bp + n * (K / 2), row, K);
            const uint16_t* bs = Bs + n * ng;
            for (size_t m = 0; m < M; ++m) {
                const int8_t* a = A + m * K;
                float run = 0.0f;
                for (size_t g = 0; g < ng; ++g) {
                    int32_t s = 0;
                    for (size_t k = 0; k < G; ++k) s += (int32_t)a[g * G + k] * (int32_t)row[g * G + k];
                    run = fmaf((float)s, h2f(bs[g]), run);
                }
                C[m * N + n] = f2h(run * As[m]);
            }
        }
        free(row);
    }
}

void ref_matmul_f16(const uint16_t* A, const uint16_t* Bt, uint16_t* C, size_t M, size_t K, size_t N) {
    const size_t K16 = (K / 16) * 16, K8 = (K / 8) * 8;
#pragma omp parallel for schedule(static) num_threads(ref_get_threads())
    for (size_t n = 0; n < N; ++n) {
        const uint16_t* b = Bt + n * K;
        for (size_t m = 0; m < M; ++m) {
            const uint16_t* a = A + m * K;
            uint16_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (size_t k = 0; k < K16; k += 16) {
                for (int j = 0; j < 8; ++j) acc[j] = hfma(a[k + j], b[k + j], acc[j]);
                for (int j = 0; j < 8; ++j) acc[j] = hfma(a[k + 8 + j], b[k + 8 + j], acc[j]);
            }
            for (size_t k = K16; k < K8; k += 8)
                for (int j = 0; j < 8; ++j) acc[j] = hfma(a[k + j], b[k + j], acc[j]);
            for (size_t k = K8; k < K; ++k) acc[0] = f2h(fmaf(h2f(a[k]), h2f(b[k]), h2f(acc[0])));
            uint16_t s4[4];
            for (int j = 0; j < 4; ++j) s4[j] = hadd(acc[j], acc[j + 4]);
            uint16_t s20 = hadd(s4[0], s4[2]), s21 = hadd(s4[1], s4[3]);
            C[m * N + n] = hadd(s20, s21);
        }
    }
}

/* ---------------------------------------------------------------- RMSNorm */
void ref_rms_norm_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t rows, size_t dims, float eps) {
    for (size_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * dims;
        uint16_t* yr = y + r * dims;
        float acc[16];
        for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
        size_t i = 0;
        const size_t tile_end = dims >= 16 ? dims - 16 + 1 : 0;
        for (; i < tile_end; i += 16)
            for (int e = 0; e < 16; ++e) { float v = h2f(xr[i + e]); acc[e] = fmaf(v, v, acc[e]); }
        const size_t simd_end = dims >= 8 ? dims - 8 + 1 : 0;
        for (; i < simd_end; i += 8)
            for (int e = 0; e < 8; ++e) { float v = h2f(xr[i + e]); acc[e] = fmaf(v, v, acc[e]); }
        float t[4];
        for (int l = 0; l < 4; ++l) t[l] = ((acc[l] + acc[4 + l]) + acc[8 + l]) + acc[12 + l];
        float ss = (t[0] + t[1]) + (t[2] + t[3]);
        for (; i < dims; ++i) { float v = h2f(xr[i]); ss = fmaf(v, v, ss); }
        float rms = sqrtf(ss / (float)dims + eps);
        float inv = 1.0f / rms;
        uint16_t inv16 = f2h(inv);
        size_t j = 0;
        const size_t vec_end = simd_end > 0 ? ((dims / 8) * 8) : 0;
        for (; j < vec_end; ++j) yr[j] = hmul(hmul(xr[j], inv16), w[j]);
        for (; j < dims; ++j) yr[j] = f2h((h2f(xr[j]) * inv) * h2f(w[j]));
    }
}

/* ---------------------------------------------------------------- RoPE */
void ref_rope_tables(uint16_t* cos_t, uint16_t* sin_t, size_t n_pos, size_t head_dim, float theta) {
    const size_t half = head_dim / 2;
    for (size_t pos = 0; pos < n_pos; ++pos) {
        const float pf = (float)pos;
        for (size_t i = 0; i < half; ++i) {
            const float freq = 1.0f / powf(theta, (2.0f * (float)i) / (float)head_dim);
            const float angle = pf * freq;
            cos_t[pos * half + i] = f2h(cosf(angle));
            sin_t[pos * half + i] = f2h(sinf(angle));
        }
    }
}

void ref_rope_f16(const uint16_t* in, uint16_t* out, size_t batch, size_t seq_len, size_t num_heads,
                  size_t head_dim, size_t start_pos, float theta) {
    const size_t half = head_dim / 2;
    const size_t npos = seq_len + start_pos;
    uint16_t* ct = (uint16_t*)malloc(npos * half * 2);
    uint16_t* st = (uint16_t*)malloc(npos * half * 2);
    ref_rope_tables(ct, st, npos, head_dim, theta);
    const size_t vec_half = (half / 8) * 8;
    for (size_t b = 0; b < batch; ++b)
        for (size_t s = 0; s < seq_len; ++s)
            for (size_t h = 0; h < num_heads; ++h) {
                const size_t off = ((b * seq_len + s) * num_heads + h) * head_dim;
                const uint16_t* c = ct + (start_pos + s) * half;
                const uint16_t* sn = st + (start_pos + s) * half;
                const uint16_t* x = in + off;
                uint16_t* y = out + off;
                for (size_t i = 0; i < vec_half; ++i) {
                    uint16_t x1 = x[i], x2 = x[i + half];
                    /* vfmsq_f16(vmulq_f16(x1, cos), x2, sin) = x1*cos - x2*sin (fused) */
                    uint16_t neg_x2 = (uint16_t)(x2 ^ 0x8000u);
                    uint16_t r1 = hfma(neg_x2, sn[i], hmul(x1, c[i]));
                    uint16_t r2 = hfma(x1, sn[i], hmul(x2, c[i]));
                    y[i] = r1;
                    y[i + half] = r2;
                }
                for (size_t i = vec_half; i < half; ++i) {
                    float x1 = h2f(x[i]), x2 = h2f(x[i + half]);
                    float cv = h2f(c[i]), sv = h2f(sn[i]);
                    y[i] = f2h(x1 * cv - x2 * sv);
                    y[i + half] = f2h(x2 * cv + x1 * sv);
                }
            }
    free(ct);
    free(st);
}

/* ---------------------------------------------------------------- fast approximations */
float ref_fast_exp(float x) {
    x = fmaxf(x, -87.0f);
    x = fminf(x, 87.0f);
    float z = x * 1.4426950408889634f;
    int32_t zi = cvt_trunc_sat(z);
    float zf = z - (float)zi;
    if (zf < 0.0f) { zi -= 1; zf = zf + 1.0f; }
    float t = zf * 0.6931471805599453f;
    float p = 0.009618129842071803f;
    p = fmaf(p, t, 0.05550410866482158f);
    p = fmaf(p, t, 0.2402265069591007f);
    p = fmaf(p, t, 0.6931471805599453f);
    p = fmaf(p, t, 1.0f);
    float scale = bitsf((uint32_t)(zi + 127) << 23);
    return p * scale;
}

float ref_fast_tanh(float x) {
    float x2 = x * x;
    float num = 27.0f + x2;
    float den = fmaf(9.0f, x2, 27.0f);
    float r = x * (num / den);
    if (x > 4.5f) r = 1.0f;
    if (x < -4.5f) r = -1.0f;
    return r;
}

/* quadratic 2^x approximation of the no-cache attention (kernel_attention.cpp:174-195) */
static inline float attn_quad_exp(float s, float block_max) {
    float x = (s - block_max) * 1.442695f;
    int32_t xi = cvt_trunc_sat(x);
    float xf = x - (float)xi;
    float y = fmaf(xf, 0.6931472f, 1.0f);
    y = fmaf(xf * xf, 0.2402265f, y);
    float sc = bitsf((uint32_t)(xi + 127) << 23);
    return y * sc;
}

/* ---------------------------------------------------------------- attention */
static inline float dot8(const float* q, const float* k, size_t hda) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t d = 0; d < hda; d += 8)
        for (int j = 0; j < 8; ++j) a[j] = fmaf(q[d + j], k[d + j], a[j]);
    return ((a[0] + a[4]) + (a[1] + a[5])) + ((a[2] + a[6]) + (a[3] + a[7]));
}

void ref_attention_f16(const uint16_t* Q, const uint16_t* Kc, const uint16_t* V, uint16_t* O,
                       size_t batch, size_t seq_len, size_t kv_seq_len, size_t Hq, size_t Hkv,
                       size_t D, float scale, size_t pos_off, size_t window, int is_causal) {
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)D);
    const size_t hda = (D / 8) * 8;
    const size_t gsz = Hq / Hkv;
    const float NINF = -INFINITY;
#pragma omp parallel for collapse(3) schedule(dynamic, 4) num_threads(ref_get_threads())
    for (size_t b = 0; b < batch; ++b)
        for (size_t h = 0; h < Hq; ++h)
            for (size_t qp = 0; qp < seq_len; ++qp) {
                const size_t kvh = h / gsz;
                const uint16_t* q16 = Q + ((b * seq_len + qp) * Hq + h) * D;
                uint16_t* o = O + ((b * seq_len + qp) * Hq + h) * D;
                float q[1024], kf[1024];
                float acc[1024];
                float sc[32];
                for (size_t d = 0; d < D; ++d) { q[d] = h2f(q16[d]); acc[d] = 0.0f; }
                float run_max = NINF, run_sum = 0.0f;
                const int is_decode = (qp == seq_len - 1) && seq_len > 1;
                const size_t aq = pos_off + qp;
                size_t kv_start = 0, kv_end = kv_seq_len;
                if (window > 0 && window < kv_seq_len) {
                    if (aq > window) kv_start = aq - window;
                    if (is_causal && aq + 1 < kv_end) kv_end = aq + 1;
                } else if (is_causal && aq + 1 < kv_end) {
                    kv_end = aq + 1;
                }
                for (size_t b0 = kv_start; b0 < kv_end; b0 += 32) {
                    const size_t be = (b0 + 32 < kv_seq_len) ? b0 + 32 : kv_seq_len;
                    const size_t bs = be - b0;
                    float bmax = NINF;
                    if (!is_decode && is_causal && b0 > aq) continue;
                    for (size_t i = 0; i < bs; ++i) {
                        const size_t kp = b0 + i;
                        if (!is_decode && is_causal && kp > aq) { sc[i] = NINF; continue; }
                        const uint16_t* k16 = Kc + ((b * kv_seq_len + kp) * Hkv + kvh) * D;
                        for (size_t d = 0; d < D; ++d) kf[d] = h2f(k16[d]);
                        float s = dot8(q, kf, hda);
                        for (size_t d = hda; d < D; ++d) s = fmaf(q[d], kf[d], s);
                        s *= scale;
                        if (is_causal && kp > aq) s = NINF;
                        else if (window > 0 && kp < aq && (aq - kp) > window) s = NINF;
                        sc[i] = s;
                        if (s > bmax) bmax = s;
                    }
                    if (bmax > NINF) {
                        float corr = expf_cr(run_max - bmax);
                        run_sum *= corr;
                        for (size_t d = 0; d < hda; ++d) acc[d] *= corr;
                        run_max = bmax;
                    }
                    float bsum = 0.0f;
                    const size_t vec = (bs / 4) * 4;
                    for (size_t i = 0; i < vec; i += 4) {
                        float y[4];
                        for (int l = 0; l < 4; ++l) y[l] = (sc[i + l] == NINF) ? 0.0f : attn_quad_exp(sc[i + l], bmax);
                        for (int l = 0; l < 4; ++l) sc[i + l] = y[l];
                        bsum += (y[0] + y[1]) + (y[2] + y[3]);
                    }
                    for (size_t i = vec; i < bs; ++i) {
                        if (sc[i] != NINF) { sc[i] = expf_cr(sc[i] - bmax); bsum += sc[i]; }
                        else sc[i] = 0.0f;
                    }
                    for (size_t i = 0; i < bs; ++i) {
                        const float wgt = sc[i];
                        if (wgt == 0.0f) continue;
                        const uint16_t* v16 = V + ((b * kv_seq_len + b0 + i) * Hkv + kvh) * D;
                        for (size_t d = 0; d < hda; ++d) acc[d] = fmaf(h2f(v16[d]), wgt, acc[d]);
                    }
                    run_sum += bsum;
                }
                if (run_sum > 0.0f) {
                    const float inv = 1.0f / run_sum;
                    for (size_t d = 0; d < hda; ++d) o[d] = f2h(acc[d] * inv);
                    for (size_t d = hda; d < D; ++d) o[d] = 0;
                } else {
                    for (size_t d = 0; d < D; ++d) o[d] = 0;
                }
            }
}

void ref_attention_hybrid_int8_fp16(const uint16_t* Q, const int8_t* Kc, const int8_t* Vc,
                                    const float* ks, const float* vs, const uint16_t* Kn,
                                    const uint16_t* Vn, uint16_t* O, size_t batch, size_t seq_len,
                                    size_t cache_len, size_t new_len, size_t Hq, size_t Hkv, size_t D,
                                    float scale, size_t pos_off, int is_causal, size_t qgs) {
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)D);
    const size_t kv_seq_len = cache_len + new_len;
    const size_t hda = (D / 8) * 8;
    const size_t gsz = Hq / Hkv;
    const size_t nqg = (D + qgs - 1) / qgs;
    const float NINF = -INFINITY;
#pragma omp parallel for collapse(3) schedule(dynamic, 4) num_threads(ref_get_threads())
    for (size_t b = 0; b < batch; ++b)
        for (size_t h = 0; h < Hq; ++h)
            for (size_t qp = 0; qp < seq_len; ++qp) {
                const size_t kvh = h / gsz;
                const uint16_t* q16 = Q + ((b * seq_len + qp) * Hq + h) * D;
                uint16_t* o = O + ((b * seq_len + qp) * Hq + h) * D;
                const int8_t* Kcb = Kc + b * cache_len * Hkv * D;
                const int8_t* Vcb = Vc + b * cache_len * Hkv * D;
                const uint16_t* Knb = Kn + b * new_len * Hkv * D;
                const uint16_t* Vnb = Vn + b * new_len * Hkv * D;
                float q[1024], kf[1024], acc[1024], sc[32];
                for (size_t d = 0; d < D; ++d) { q[d] = h2f(q16[d]); acc[d] = 0.0f; }
                float run_max = NINF, run_sum = 0.0f;
                const size_t aq = pos_off + qp;
                const size_t kv_end = is_causal ? (kv_seq_len < aq + 1 ? kv_seq_len : aq + 1) : kv_seq_len;
                for (size_t b0 = 0; b0 < kv_end; b0 += 32) {
                    const size_t be = (b0 + 32 < kv_end) ? b0 + 32 : kv_end;
                    const size_t bs = be - b0;
                    float bmax = NINF;
                    for (size_t i = 0; i < bs; ++i) {
                        const size_t kp = b0 + i;
                        if (is_causal && kp > aq) { sc[i] = NINF; continue; }
                        if (kp < cache_len) {
                            const int8_t* k8 = Kcb + (kp * Hkv + kvh) * D;
                            const float* ksb = ks + (kp * Hkv + kvh) * nqg; /* no batch offset, as the reference */
                            for (size_t d = 0; d < hda; ++d) kf[d] = (float)k8[d] * ksb[d / qgs];
                        } else {
                            const uint16_t* k16 = Knb + ((kp - cache_len) * Hkv + kvh) * D;
                            for (size_t d = 0; d < hda; ++d) kf[d] = h2f(k16[d]);
                        }
                        float s = dot8(q, kf, hda) * scale;
                        sc[i] = s;
                        if (s > bmax) bmax = s;
                    }
                    if (bmax > NINF) {
                        float corr = expf_cr(run_max - bmax);
                        run_sum *= corr;
                        for (size_t d = 0; d < hda; ++d) acc[d] *= corr;
                        run_max = bmax;
                    }
                    float bsum = 0.0f;
                    for (size_t i = 0; i < bs; ++i) {
                        if (sc[i] != NINF) { sc[i] = expf_cr(sc[i] - bmax); bsum += sc[i]; }
                        else sc[i] = 0.0f;
                    }
                    for (size_t i = 0; i < bs; ++i) {
                        const float wgt = sc[i];
                        if (wgt == 0.0f) continue;
                        const size_t kp = b0 + i;
                        if (kp < cache_len) {
                            const int8_t* v8 = Vcb + (kp * Hkv + kvh) * D;
                            const float* vsb = vs + (kp * Hkv + kvh) * nqg;
                            for (size_t d = 0; d < hda; ++d) acc[d] = fmaf((float)v8[d] * vsb[d / qgs], wgt, acc[d]);
                        } else {
                            const uint16_t* v16 = Vnb + ((kp - cache_len) * Hkv + kvh) * D;
                            for (size_t d = 0; d < hda; ++d) acc[d] = fmaf(h2f(v16[d]), wgt, acc[d]);
                        }
                    }
                    run_sum += bsum;
                }
                if (run_sum > 0.0f) {
                    const float inv = 1.0f / run_sum;
                    for (size_t d = 0; d < hda; ++d) o[d] = f2h(acc[d] * inv);
                } else {
                    for (size_t d = 0; d < D; ++d) o[d] = 0;
                }
            }
}

/* ---------------------------------------------------------------- KV quantization */
void ref_quantize_kv(const uint16_t* src, int8_t* dst, float* scales, size_t seq_len, size_t kv_heads,
                     size_t head_dim, size_t G) {
    const size_t ng = (head_dim + G - 1) / G;
    for (size_t idx = 0; idx < seq_len * kv_heads; ++idx) {
        const uint16_t* hs = src + idx * head_dim;
        int8_t* hd = dst + idx * head_dim;
        for (size_t g = 0; g < ng; ++g) {
            const size_t g0 = g * G;
            const size_t cnt = (G < head_dim - g0) ? G : head_dim - g0;
            float m = 0.0f;
            for (size_t k = 0; k < cnt; ++k) { float a = fabsf(h2f(hs[g0 + k])); m = a > m ? a : m; }
            float scale = m / 127.0f;
            if (scale < 1e-10f) scale = 1e-10f;
            const float inv = 1.0f / scale;
            const size_t vec = (cnt / 8) * 8;
            for (size_t k = 0; k < vec; ++k) hd[g0 + k] = sat8(cvt_rne_sat(h2f(hs[g0 + k]) * inv));
            for (size_t k = vec; k < cnt; ++k) {
                int32_t qv = (int32_t)roundf(h2f(hs[g0 + k]) * inv);
                hd[g0 + k] = sat8(qv);
            }
            scales[idx * ng + g] = scale;
        }
    }
}

/* ---------------------------------------------------------------- activations / elementwise */
/* cactus_silu_f16 / cactus_gelu_f16 run under parallel_for with SCALAR_EXPENSIVE {2500, 1250}
 * (kernel_nn.cpp:13,50; kernel_utils.h:410-437, 516-548): from 2500 elements the work is cut
 * into min(workers, ceil(n / 1250)) equal chunks (the last takes the rest), and every chunk
 * ends with its own scalar tail of (length % 8) elements on the libm formula. The worker
 * count is the host's (min(hardware threads, 16)), so those positions follow the host.
 * g_chunk_pool = 0 (the default) restates one chunk: the vector formula everywhere but the
 * tensor's own tail, which is also what the GPU computes; g_chunk_pool = P restates the
 * reference on a host with P pool workers. */
static int g_chunk_pool = 0;
void ref_set_chunk_pool(int workers) { g_chunk_pool = workers < 0 ? 0 : workers; }

static int scalar_tail(size_t i, size_t n) {
    size_t t = 1;
    if (g_chunk_pool > 0 && n >= 2500) {
        t = (n + 1249) / 1250;
        if (t > (size_t)g_chunk_pool) t = (size_t)g_chunk_pool;
    }
    const size_t per = n / t;
    size_t w = i / per;
    if (w > t - 1) w = t - 1;
    const size_t start = w * per, end = (w == t - 1) ? n : start + per;
    return i >= start + ((end - start) / 8) * 8;
}

void ref_silu_f16(const uint16_t* x, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float v = h2f(x[i]);
        if (!scalar_tail(i, n)) {
            float e = ref_fast_exp(-v);
            float sg = 1.0f / (1.0f + e);
            y[i] = f2h(v * sg);
        } else {
            float sg = 1.0f / (1.0f + expf_cr(-v));
            y[i] = f2h(v * sg);
        }
    }
}

void ref_gelu_f16(const uint16_t* x, uint16_t* y, size_t n) {
    const float s2p = 0.7978845608028654f, c = 0.044715f;
    for (size_t i = 0; i < n; ++i) {
        float v = h2f(x[i]);
        if (!scalar_tail(i, n)) {
            float v3 = (v * v) * v;
            float inner = fmaf(c, v3, v);
            inner = s2p * inner;
            float t = ref_fast_tanh(inner);
            y[i] = f2h((0.5f * v) * (1.0f + t));
        } else {
            float inner = s2p * fmaf((c * v) * v, v, v);
            y[i] = f2h((0.5f * v) * (1.0f + tanhf_cr(inner)));
        }
    }
}

void ref_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = hadd(a[i], b[i]);
}
void ref_add_f16_clipped(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float r = h2f(a[i]) + h2f(b[i]);
        r = fminf(fmaxf(r, -65500.0f), 65500.0f);
        y[i] = f2h(r);
    }
}
void ref_multiply_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = hmul(a[i], b[i]);
}
void ref_scalar_multiply_f16(const uint16_t* x, uint16_t* y, size_t n, float s) {
    const uint16_t s16 = f2h(s);
    for (size_t i = 0; i < n; ++i) y[i] = hmul(x[i], s16);
}

void ref_softmax_f16(const uint16_t* x, uint16_t* y, size_t rows, size_t V) {
    for (size_t r = 0; r < rows; ++r) {
        const uint16_t* in = x + r * V;
        uint16_t* out = y + r * V;
        const size_t vv = (V / 32) * 32;
        float mx = -INFINITY;
        for (size_t i = 0; i < V; ++i) { float v = h2f(in[i]); mx = v > mx ? v : mx; }
        float acc[32];
        for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
        for (size_t i = 0; i < vv; i += 32)
            for (int e = 0; e < 32; ++e) {
                float ev = ref_fast_exp(h2f(in[i + e]) - mx);
                out[i + e] = f2h(ev);
                acc[e] += ev;
            }
        float lane[4];
        for (int l = 0; l < 4; ++l) {
            float s = acc[l];
            for (int u = 1; u < 8; ++u) s = s + acc[4 * u + l];
            lane[l] = s;
        }
        float sum = (lane[0] + lane[1]) + (lane[2] + lane[3]);
        for (size_t i = vv; i < V; ++i) {
            float ev = expf_cr(h2f(in[i]) - mx);
            out[i] = f2h(ev);
            sum += ev;
        }
        const float inv = 1.0f / sum;
        const uint16_t inv16 = f2h(inv);
        for (size_t i = 0; i < vv; ++i) out[i] = hmul(out[i], inv16);
        for (size_t i = vv; i < V; ++i) out[i] = f2h(h2f(out[i]) * inv);
    }
}

/* ---------------------------------------------------------------- embedding / argmax */
void ref_embedding_int8(const int8_t* table, const uint16_t* scales, size_t G, size_t ng,
                        const uint32_t* ids, size_t n_ids, size_t hidden, uint16_t* out) {
    for (size_t i = 0; i < n_ids; ++i) {
        const size_t idx = ids[i];
        for (size_t g = 0; g < ng; ++g) {
            const float s = h2f(scales[idx * ng + g]);
            const size_t k1 = (g + 1) * G < hidden ? (g + 1) * G : hidden;
            for (size_t k = g * G; k < k1; ++k) out[i * hidden + k] = f2h((float)table[idx * hidden + k] * s);
        }
    }
}
void ref_embedding_f16(const uint16_t* table, const uint32_t* ids, size_t n_ids, size_t hidden, uint16_t* out) {
    for (size_t i = 0; i < n_ids; ++i) memcpy(out + i * hidden, table + (size_t)ids[i] * hidden, hidden * 2);
}

uint32_t ref_argmax_f16(const uint16_t* logits, size_t V) {
    if (V == 0) return 0;
    size_t best = 0;
    float bv = h2f(logits[0]);
    for (size_t i = 1; i < V; ++i) {
        float v = h2f(logits[i]);
        if (v > bv) { bv = v; best = i; }
    }
    return (uint32_t)best;
}

/* ---------------------------------------------------------------- weight quantizer (tensor_io.py) */
void ref_quantize_weights_int8(const float* w, int8_t* q, uint16_t* scales, size_t N, size_t K, size_t G) {
    const size_t ng = K / G;
    const float floor_s = 1e-10f;
#pragma omp parallel for schedule(static) num_threads(ref_get_threads())
    for (size_t n = 0; n < N; ++n)
        for (size_t g = 0; g < ng; ++g) {
            const float* wg = w + n * K + g * G;
            float m = 0.0f;
            for (size_t k = 0; k < G; ++k) { float a = fabsf(wg[k]); m = a > m ? a : m; }
            float s = m / 127.0f;
            if (s < floor_s) s = floor_s;
            for (size_t k = 0; k < G; ++k) {
                float r = nearbyintf(wg[k] / s);
                r = r < -128.0f ? -128.0f : (r > 127.0f ? 127.0f : r);
                q[n * K + g * G + k] = (int8_t)r;
            }
            scales[n * ng + g] = f2h(s);
        }
}

void ref_quantize_weights_int4(const float* w, uint8_t* packed, uint16_t* scales, size_t N, size_t K, size_t G) {
    const size_t ng = K / G;
    const float floor_s = 1e-10f;
#pragma omp parallel for schedule(static) num_threads(ref_get_threads())
    for (size_t n = 0; n < N; ++n) {
        for (size_t g = 0; g < ng; ++g) {
            const float* wg = w + n * K + g * G;
            float m = 0.0f;
            for (size_t k = 0; k < G; ++k) { float a = fabsf(wg[k]); m = a > m ? a : m; }
            float s = m / 7.0f;
            if (s < floor_s) s = floor_s;
            for (size_t k = 0; k < G; k += 2) {
                float r0 = nearbyintf(wg[k] / s), r1 = nearbyintf(wg[k + 1] / s);
                r0 = r0 < -8.0f ? -8.0f : (r0 > 7.0f ? 7.0f : r0);
                r1 = r1 < -8.0f ? -8.0f : (r1 > 7.0f ? 7.0f : r1);
                int8_t i0 = (int8_t)r0, i1 = (int8_t)r1;
                packed[(n * K + g * G + k) / 2] = (uint8_t)(((uint8_t)i0 & 0x0F) | (((uint8_t)i1 & 0x0F) << 4));
            }
            scales[n * ng + g] = f2h(s);
        }
    }
}

/* ---------------------------------------------------------------- other families' kernels */
/* cactus_conv1d_causal_depthwise_f16 (kernel_conv.cpp:15-110): input / output [N, L, C],
 * weight [C, K] applied reversed (tap k reads x[t - k*dilation], zero before t = 0). Four
 * fp32 lane accumulators take the taps of each 8-block (lane j: taps k+j, then k+4+j), the
 * lanes fold as vaddvq_f32 ((l0 + l1) + (l2 + l3)), and the taps past the last 8-block are
 * added one by one (contracted), skipping positions before the sequence start. */
void ref_conv1d_causal_depthwise_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t N, size_t L, size_t C,
                                     size_t K, size_t dil) {
    for (size_t n = 0; n < N; ++n)
        for (size_t c = 0; c < C; ++c)
            for (size_t t = 0; t < L; ++t) {
                const uint16_t* xb = x + n * L * C;
                float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                size_t k = 0;
                for (; k + 8 <= K; k += 8)
                    for (int half = 0; half < 2; ++half)
                        for (int j = 0; j < 4; ++j) {
                            const size_t kk = k + 4 * half + j;
                            const long long a = (long long)t - (long long)(kk * dil);
                            const float xv = a >= 0 ? h2f(xb[(size_t)a * C + c]) : 0.0f;
                            lane[j] = fmaf(xv, h2f(w[c * K + (K - 1 - kk)]), lane[j]);
                        }
                float acc = (lane[0] + lane[1]) + (lane[2] + lane[3]);
                for (; k < K; ++k) {
                    const long long a = (long long)t - (long long)(k * dil);
                    if (a >= 0) acc = fmaf(h2f(w[c * K + (K - 1 - k)]), h2f(xb[(size_t)a * C + c]), acc);
                }
                y[n * L * C + t * C + c] = f2h(acc);
            }
}

/* cactus_conv1d_f16_k3 (kernel_conv.cpp:112-227): input [N, C_in, L], weight [C_out, C_in, 3],
 * output [N, C_out, (L - 1) / stride + 1], zero padding of one on both sides. Three fp32 lane
 * chains (taps t-1, t, t+1) run over the input channels in order; the fold is
 * (l0 + l2) + (l1 + l3) with lane 3 zero. */
void ref_conv1d_f16_k3(const uint16_t* x, const uint16_t* w, uint16_t* y, size_t N, size_t L, size_t Cin, size_t Cout,
                       size_t stride) {
    const size_t out_len = (L - 1) / stride + 1;
    for (size_t n = 0; n < N; ++n)
        for (size_t oc = 0; oc < Cout; ++oc)
            for (size_t o = 0; o < out_len; ++o) {
                const long long t = (long long)(o * stride);
                float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (size_t ic = 0; ic < Cin; ++ic) {
                    const uint16_t* xc = x + (n * Cin + ic) * L;
                    const uint16_t* wc = w + (oc * Cin + ic) * 3;
                    const float xm = t - 1 >= 0 ? h2f(xc[t - 1]) : 0.0f;
                    const float x0 = h2f(xc[t]);
                    const float xp = t + 1 < (long long)L ? h2f(xc[t + 1]) : 0.0f;
                    lane[0] = fmaf(xm, h2f(wc[0]), lane[0]);
                    lane[1] = fmaf(x0, h2f(wc[1]), lane[1]);
                    lane[2] = fmaf(xp, h2f(wc[2]), lane[2]);
                    lane[3] = fmaf(0.0f, 0.0f, lane[3]);
                }
                y[(n * Cout + oc) * out_len + o] = f2h((lane[0] + lane[2]) + (lane[1] + lane[3]));
            }
}

/* compute_layernorm_node (graph_ops_nn.cpp:373-457), fp16 input / weight / bias / output:
 * in-order fp32 sums for the mean and the variance (diff*diff contracted), divided by the
 * feature count, inv = 1 / sqrtf(var + eps), y = fp16(fma((x - mean) * inv, w, b)). */
void ref_layernorm_f16(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* y, size_t rows, size_t F,
                       float eps) {
    for (size_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * F;
        float mean = 0.0f;
        for (size_t i = 0; i < F; ++i) mean += h2f(xr[i]);
        mean /= (float)F;
        float var = 0.0f;
        for (size_t i = 0; i < F; ++i) {
            const float d = h2f(xr[i]) - mean;
            var = fmaf(d, d, var);
        }
        var /= (float)F;
        const float inv = 1.0f / sqrtf(var + eps);
        for (size_t i = 0; i < F; ++i) y[r * F + i] = f2h(fmaf((h2f(xr[i]) - mean) * inv, h2f(w[i]), h2f(b[i])));
    }
}
