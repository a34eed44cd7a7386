/*
 * s2_oracle.c -- CPU restatement of s2.cpp's dual-AR decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker).  The product library in
 * s2.cpp_b200/ never links or calls this file; see s2_oracle.h for the list
 * of reference functions restated here and the RNG substitution.
 *
 * Compiled with -ffp-contract=off so every float expression rounds exactly
 * as written (the CUDA kernels spell the same operations with __fmul_rn and
 * friends where it matters).
 */
#include "s2_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#include <float.h>
#include <time.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK8_0 32
#define QK_K 256
/* keys per attention split (the CUDA kernels split the same way) */
#define SO_ATTN_SPLIT 64

/* ------------------------------------------------------------------------ */
/* fp16                                                                      */
/* ------------------------------------------------------------------------ */

float so_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { e++; man <<= 1; } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE round-to-nearest-even, as F16C's _cvtss_sh(x, 0) used by ggml on x86 */
uint16_t so_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00 | (absx > 0x7f800000u ? 0x200 : 0));
    }
    if (absx >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00);
    }
    if (absx < 0x38800000u) { /* result is subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to 0 */
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7fffff) | 0x800000;
        uint32_t shift = 126 - e; /* 14 + (113 - e) */
        uint32_t r = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((absx >> 13) - (112u << 10));
    uint32_t rem = absx & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) r++;
    return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------------ */
/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as   */
/* easy as 1, 2, 3", SC'11).  Same rounds and constants as the paper.        */
/* ------------------------------------------------------------------------ */

void so_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0;
        uint32_t n1 = lo1;
        uint32_t n2 = hi0 ^ c3 ^ k1;
        uint32_t n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

double so_philox_uniform(uint64_t seed, uint32_t frame, uint32_t purpose, uint32_t seq) {
    const uint32_t ctr[4] = {frame, purpose, seq, 0x53324b30u /* "S2K0" */};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t o[4];
    so_philox4x32_10(ctr, key, o);
    /* 53-bit double in [0,1) */
    uint64_t a = o[0] >> 5, b = o[1] >> 6;
    return (double)(a * 67108864ull + b) * (1.0 / 9007199254740992.0);
}

/* ------------------------------------------------------------------------ */
/* exp with a fixed sequence of IEEE float operations: the CUDA kernels run  */
/* the same steps (s2k_common.cuh det_expf), so both return identical bits.  */
/* Cody-Waite reduction x = k ln2 + r, Taylor series of exp(r) to degree 7,  */
/* scaling by 2^k.  Accuracy ~1-2 ulp, like libm expf.                       */
/* The scaling is two products by powers of two: p * 2^(k-h) is exact and   */
/* normal for every k in [-150, 128], the product by 2^h rounds once (into   */
/* the subnormals when k < -126), so the result is ldexpf(p, k).             */
/* ------------------------------------------------------------------------ */

static inline float pow2f_bits(int e) {
    const uint32_t u = (uint32_t)(e + 127) << 23;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

float so_pow2_scale(float p, int k) {
    const int h = k < -100 ? -64 : (k > 100 ? 64 : 0);
    return (p * pow2f_bits(k - h)) * pow2f_bits(h);
}

float so_det_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float k = rintf(x * 1.44269502162933349609f);
    const float r = (x - k * 0.693145751953125f) - k * 1.42860682030941723212e-6f;
    float p = 1.98412698412698412526e-4f;
    p = p * r + 1.38888888888888894189e-3f;
    p = p * r + 8.33333333333333321769e-3f;
    p = p * r + 4.16666666666666643537e-2f;
    p = p * r + 1.66666666666666657415e-1f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    return so_pow2_scale(p, (int)k);
}

void so_det_expf_array(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = so_det_expf(x[i]);
}

/* Checker of the scaling step: so_pow2_scale(p, k) against the C library's
 * ldexpf(p, k) for every k in [-150, 128] and n values of p (the reachable
 * [0.70, 1.42], then random bit patterns in [0.5, 2)); returns the number of
 * differing results. */
int64_t so_check_pow2_scale(int64_t n, uint32_t seed) {
    int64_t bad = 0;
    uint32_t st = seed ? seed : 1u;
    for (int k = -150; k <= 128; ++k) {
        for (int64_t j = 0; j < n; ++j) {
            float p;
            if (j < n / 2) {
                p = 0.70f + 0.72f * (float)j / (float)(n / 2);
            } else {
                st = st * 1664525u + 1013904223u;
                const uint32_t u = 0x3f000000u + (st >> 8) % 0x01000000u;  /* [0.5, 2) */
                memcpy(&p, &u, sizeof p);
            }
            const float a = so_pow2_scale(p, k), b = ldexpf(p, k);
            uint32_t ua, ub;
            memcpy(&ua, &a, 4);
            memcpy(&ub, &b, 4);
            bad += ua != ub;
        }
    }
    return bad;
}

/* sin with the same float steps as the CUDA det_sinf (s2k_common.cuh):
 * Cody-Waite reduction by pi in three parts, the Taylor series of sin to
 * degree 13 on |r| <= pi/2, negated for odd multiples; the library sinf
 * beyond |x| = 6400.  (The reference's ggml_sin calls sinf; the two agree to
 * an ulp or two.) */
float so_det_sinf(float x) {
    if (!(fabsf(x) <= 6400.0f)) return sinf(x);
    const float k = rintf(x * 0.318309873342514038f);
    float r = x - k * 3.140625f;
    r = r - k * 9.6750259399414062e-4f;
    r = r - k * 1.5099580252808664e-7f;
    const float r2 = r * r;
    float p = 1.60590443720742825917e-10f;
    p = p * r2 + -2.50521079436794025241e-8f;
    p = p * r2 + 2.75573188446287531406e-6f;
    p = p * r2 + -1.98412701138295233250e-4f;
    p = p * r2 + 8.33333376795053482056e-3f;
    p = p * r2 + -1.66666671633720397949e-1f;
    const float v = r + (r * r2) * p;
    return ((int)k & 1) ? -v : v;
}

/* ------------------------------------------------------------------------ */
/* block formats                                                             */
/* ------------------------------------------------------------------------ */

int64_t so_row_bytes(int type, int64_t n) {
    switch (type) {
    case SO_TYPE_F32: return n * 4;
    case SO_TYPE_F16: return n * 2;
    case SO_TYPE_Q8_0: return n / QK8_0 * 34;
    case SO_TYPE_Q4_K: return n / QK_K * 144;
    case SO_TYPE_Q6_K: return n / QK_K * 210;
    case SO_TYPE_Q8_K: return n / QK_K * 292;
    default: return -1;
    }
}

static inline uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }

/* ggml get_scale_min_k4: 12 bytes hold 8 six-bit scales and 8 six-bit mins */
static inline void q4k_scale_min(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

int so_dequant_row(int type, const void *src, float *y, int64_t n) {
    const uint8_t *p = (const uint8_t *)src;
    switch (type) {
    case SO_TYPE_F32: memcpy(y, p, (size_t)n * 4); return 0;
    case SO_TYPE_F16:
        for (int64_t i = 0; i < n; ++i) y[i] = so_fp16_to_fp32(rd16(p + 2 * i));
        return 0;
    case SO_TYPE_Q8_0: /* dequantize_row_q8_0: y = q * d */
        for (int64_t b = 0; b < n / QK8_0; ++b, p += 34) {
            const float d = so_fp16_to_fp32(rd16(p));
            const int8_t *q = (const int8_t *)(p + 2);
            for (int j = 0; j < QK8_0; ++j) y[b * QK8_0 + j] = (float)q[j] * d;
        }
        return 0;
    case SO_TYPE_Q4_K: /* d(2) dmin(2) scales(12) qs(128) */
        for (int64_t b = 0; b < n / QK_K; ++b, p += 144) {
            const float d = so_fp16_to_fp32(rd16(p));
            const float dmin = so_fp16_to_fp32(rd16(p + 2));
            const uint8_t *sc = p + 4, *q = p + 16;
            float *yb = y + b * QK_K;
            for (int c = 0; c < 4; ++c) {
                int s0, m0, s1, m1;
                q4k_scale_min(2 * c, sc, &s0, &m0);
                q4k_scale_min(2 * c + 1, sc, &s1, &m1);
                const float d1 = d * (float)s0, mm1 = dmin * (float)m0;
                const float d2 = d * (float)s1, mm2 = dmin * (float)m1;
                for (int l = 0; l < 32; ++l) yb[64 * c + l] = d1 * (float)(q[32 * c + l] & 0xF) - mm1;
                for (int l = 0; l < 32; ++l) yb[64 * c + 32 + l] = d2 * (float)(q[32 * c + l] >> 4) - mm2;
            }
        }
        return 0;
    case SO_TYPE_Q6_K: /* ql(128) qh(64) scales(16 x i8) d(2) */
        for (int64_t b = 0; b < n / QK_K; ++b, p += 210) {
            const uint8_t *ql = p, *qh = p + 128;
            const int8_t *sc = (const int8_t *)(p + 192);
            const float d = so_fp16_to_fp32(rd16(p + 208));
            float *yb = y + b * QK_K;
            for (int h = 0; h < 2; ++h) {
                for (int l = 0; l < 32; ++l) {
                    const int is = l / 16;
                    const int q1 = ((ql[64 * h + l] & 0xF) | (((qh[32 * h + l] >> 0) & 3) << 4)) - 32;
                    const int q2 = ((ql[64 * h + l + 32] & 0xF) | (((qh[32 * h + l] >> 2) & 3) << 4)) - 32;
                    const int q3 = ((ql[64 * h + l] >> 4) | (((qh[32 * h + l] >> 4) & 3) << 4)) - 32;
                    const int q4 = ((ql[64 * h + l + 32] >> 4) | (((qh[32 * h + l] >> 6) & 3) << 4)) - 32;
                    yb[128 * h + l + 0] = d * (float)sc[8 * h + is + 0] * (float)q1;
                    yb[128 * h + l + 32] = d * (float)sc[8 * h + is + 2] * (float)q2;
                    yb[128 * h + l + 64] = d * (float)sc[8 * h + is + 4] * (float)q3;
                    yb[128 * h + l + 96] = d * (float)sc[8 * h + is + 6] * (float)q4;
                }
            }
        }
        return 0;
    default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* activation quantizers of the ggml CPU mat-vec                            */
/* ------------------------------------------------------------------------ */

void so_quantize_act_q8_0(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / QK8_0; ++b, out += 34) {
        const float *xb = x + b * QK8_0;
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.f;
        const float id = amax != 0.0f ? 127.f / amax : 0.0f;
        const uint16_t dh = so_fp32_to_fp16(d);
        memcpy(out, &dh, 2);
        int8_t *q = (int8_t *)(out + 2);
        for (int j = 0; j < QK8_0; ++j) q[j] = (int8_t)(int)nearbyintf(xb[j] * id);
    }
}

/* ggml nearest_int: magic-number round-half-even */
static inline int nearest_int(float fval) {
    float val = fval + 12582912.f;
    int i;
    memcpy(&i, &val, sizeof(int));
    return (i & 0x007fffff) - 0x00400000;
}

void so_quantize_act_q8_K(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / QK_K; ++b, out += 292) {
        const float *xb = x + b * QK_K;
        float mx = 0, amax = 0;
        for (int j = 0; j < QK_K; ++j) {
            const float ax = fabsf(xb[j]);
            if (ax > amax) { amax = ax; mx = xb[j]; }
        }
        int8_t *q = (int8_t *)(out + 4);
        int16_t bs[16];
        if (amax == 0.0f) {
            const float z = 0.0f;
            memcpy(out, &z, 4);
            memset(q, 0, QK_K);
            memset(bs, 0, sizeof(bs));
            memcpy(out + 260, bs, 32);
            continue;
        }
        const float iscale = -127.f / mx;
        for (int j = 0; j < QK_K; ++j) {
            int v = nearest_int(iscale * xb[j]);
            q[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int j = 0; j < 16; ++j) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += q[j * 16 + i];
            bs[j] = (int16_t)s;
        }
        const float d = 1.0f / iscale;
        memcpy(out, &d, 4);
        memcpy(out + 260, bs, 32);
    }
}

/* ------------------------------------------------------------------------ */
/* dot products (one weight row . one quantized activation row)             */
/* ------------------------------------------------------------------------ */

static inline int32_t dot_i8(const int8_t *a, const int8_t *b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; ++i) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

/* Every dot below follows the arithmetic convention the CUDA kernels share:
 * each block term is formed exactly (or as ggml rounds its float scale), the
 * terms are summed in double and the row result is rounded to float once.
 * This is the limit every ggml backend's float accumulation approximates, and
 * it makes the result independent of summation order. */

/* vec_dot_q8_0_q8_0: sum_b (int sum_b) * (d_w * d_x); d_w*d_x is exact in float */
static float dot_q8_0(const uint8_t *w, const uint8_t *a, int64_t n) {
    double acc = 0.0;
    for (int64_t b = 0; b < n / QK8_0; ++b, w += 34, a += 34) {
        const int32_t s = dot_i8((const int8_t *)(w + 2), (const int8_t *)(a + 2), QK8_0);
        acc += (double)s * (double)(so_fp16_to_fp32(rd16(w)) * so_fp16_to_fp32(rd16(a)));
    }
    return (float)acc;
}

/* vec_dot_q4_K_q8_K: per super-block
 *   (d_w*d_x) * sum_j sc_j*(q4 . q8)_j  -  (dmin_w*d_x) * sum_j m_j*bsum_j */
static float dot_q4_K(const uint8_t *w, const uint8_t *a, int64_t n) {
    double sumf = 0.0;
    for (int64_t b = 0; b < n / QK_K; ++b, w += 144, a += 292) {
        float dx;
        memcpy(&dx, a, 4);
        const int8_t *q8 = (const int8_t *)(a + 4);
        int16_t bs[16];
        memcpy(bs, a + 260, 32);
        const uint8_t *sc = w + 4, *q = w + 16;
        int32_t isum = 0, msum = 0;
        for (int c = 0; c < 4; ++c) {
            int s0, m0, s1, m1;
            q4k_scale_min(2 * c, sc, &s0, &m0);
            q4k_scale_min(2 * c + 1, sc, &s1, &m1);
            int32_t lo = 0, hi = 0;
            for (int l = 0; l < 32; ++l) {
                lo += (int32_t)(q[32 * c + l] & 0xF) * q8[64 * c + l];
                hi += (int32_t)(q[32 * c + l] >> 4) * q8[64 * c + 32 + l];
            }
            isum += s0 * lo + s1 * hi;
            msum += m0 * (bs[4 * c + 0] + bs[4 * c + 1]) + m1 * (bs[4 * c + 2] + bs[4 * c + 3]);
        }
        const float d = so_fp16_to_fp32(rd16(w)) * dx;
        const float dmin = so_fp16_to_fp32(rd16(w + 2)) * dx;
        sumf += (double)d * (double)isum - (double)dmin * (double)msum;
    }
    return (float)sumf;
}

/* vec_dot_q6_K_q8_K: per super-block (d_w*d_x) * sum_j sc_j*((q6-32) . q8)_j */
static float dot_q6_K(const uint8_t *w, const uint8_t *a, int64_t n) {
    double sumf = 0.0;
    int8_t q6[QK_K];
    for (int64_t b = 0; b < n / QK_K; ++b, w += 210, a += 292) {
        const uint8_t *ql = w, *qh = w + 128;
        const int8_t *sc = (const int8_t *)(w + 192);
        for (int h = 0; h < 2; ++h)
            for (int l = 0; l < 32; ++l) {
                q6[128 * h + l + 0] = (int8_t)(((ql[64 * h + l] & 0xF) | (((qh[32 * h + l] >> 0) & 3) << 4)) - 32);
                q6[128 * h + l + 32] = (int8_t)(((ql[64 * h + l + 32] & 0xF) | (((qh[32 * h + l] >> 2) & 3) << 4)) - 32);
                q6[128 * h + l + 64] = (int8_t)(((ql[64 * h + l] >> 4) | (((qh[32 * h + l] >> 4) & 3) << 4)) - 32);
                q6[128 * h + l + 96] = (int8_t)(((ql[64 * h + l + 32] >> 4) | (((qh[32 * h + l] >> 6) & 3) << 4)) - 32);
            }
        float dx;
        memcpy(&dx, a, 4);
        const int8_t *q8 = (const int8_t *)(a + 4);
        int32_t isum = 0;
        for (int j = 0; j < 16; ++j) isum += (int32_t)sc[j] * dot_i8(q6 + 16 * j, q8 + 16 * j, 16);
        const float d = so_fp16_to_fp32(rd16(w + 208)) * dx;
        sumf += (double)d * (double)isum;
    }
    return (float)sumf;
}

/* ggml_vec_dot_f16 with the activation converted to f16 (vec_dot_type F16) */
static float dot_f16(const uint8_t *w, const uint8_t *a, int64_t n) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i)
        s += (double)(so_fp16_to_fp32(rd16(w + 2 * i)) * so_fp16_to_fp32(rd16(a + 2 * i)));
    return (float)s;
}

static float dot_f32(const uint8_t *w, const uint8_t *a, int64_t n) {
    const float *x = (const float *)w, *y = (const float *)a;
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += (double)(x[i] * y[i]);
    return (float)s;
}

float so_vec_dot(int type, const void *wrow, const void *act, int64_t n) {
    switch (type) {
    case SO_TYPE_Q8_0: return dot_q8_0((const uint8_t *)wrow, (const uint8_t *)act, n);
    case SO_TYPE_Q4_K: return dot_q4_K((const uint8_t *)wrow, (const uint8_t *)act, n);
    case SO_TYPE_Q6_K: return dot_q6_K((const uint8_t *)wrow, (const uint8_t *)act, n);
    case SO_TYPE_F16: return dot_f16((const uint8_t *)wrow, (const uint8_t *)act, n);
    case SO_TYPE_F32: return dot_f32((const uint8_t *)wrow, (const uint8_t *)act, n);
    default: return NAN;
    }
}

static int act_type_for(int wtype) {
    switch (wtype) {
    case SO_TYPE_Q8_0: return SO_TYPE_Q8_0;
    case SO_TYPE_Q4_K:
    case SO_TYPE_Q6_K: return SO_TYPE_Q8_K;
    case SO_TYPE_F16: return SO_TYPE_F16;
    default: return SO_TYPE_F32;
    }
}

static void quantize_act(int wtype, const float *x, int64_t n, uint8_t *out) {
    switch (act_type_for(wtype)) {
    case SO_TYPE_Q8_0: so_quantize_act_q8_0(x, n, out); break;
    case SO_TYPE_Q8_K: so_quantize_act_q8_K(x, n, out); break;
    case SO_TYPE_F16:
        for (int64_t i = 0; i < n; ++i) {
            uint16_t h = so_fp32_to_fp16(x[i]);
            memcpy(out + 2 * i, &h, 2);
        }
        break;
    default: memcpy(out, x, (size_t)n * 4); break;
    }
}

/* Y[t][r] = W[r,:] . X[t,:] for T tokens; each token's activation row is
 * quantized on its own, as ggml does per src1 row. */
static void matmat(int type, const void *w, int64_t rows, int64_t n, int T, const float *X,
                   float *Y, int64_t ldy) {
    const int at = act_type_for(type);
    const int64_t abytes = so_row_bytes(at, n);
    const int64_t wbytes = so_row_bytes(type, n);
    uint8_t *aq = (uint8_t *)malloc((size_t)(abytes * T));
    for (int t = 0; t < T; ++t) quantize_act(type, X + (int64_t)t * n, n, aq + t * abytes);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint8_t *wr = (const uint8_t *)w + r * wbytes;
        for (int t = 0; t < T; ++t) Y[(int64_t)t * ldy + r] = so_vec_dot(type, wr, aq + t * abytes, n);
    }
    free(aq);
}

void so_matvec(int type, const void *w, int64_t rows, int64_t n, const float *x, float *y) {
    matmat(type, w, rows, n, 1, x, y, rows);
}

void so_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* model                                                                     */
/* ------------------------------------------------------------------------ */

typedef struct so_tensor {
    int type;
    int64_t ne0, ne1; /* [in, out] */
    const uint8_t *data;
} so_tensor;

typedef struct so_layer {
    so_tensor attention_norm, ffn_norm, q_norm, k_norm, wqkv, wo, w1, w2, w3;
} so_layer;

struct so_model {
    so_hparams hp;
    so_tensor embeddings, codebook_embeddings, norm, fast_embeddings, fast_norm, fast_output,
        fast_project_in;
    so_layer *layers, *fast_layers;
    uint16_t *kv_k, *kv_v; /* f16 [layer][pos][kv_head][head_dim] (src/s2_model.cpp:746-747) */
    int32_t max_seq_len, n_past;
};

so_model *so_model_create(const so_hparams *hp) {
    so_model *m = (so_model *)calloc(1, sizeof(so_model));
    m->hp = *hp;
    m->layers = (so_layer *)calloc((size_t)(hp->block_count > 0 ? hp->block_count : 1), sizeof(so_layer));
    m->fast_layers =
        (so_layer *)calloc((size_t)(hp->fast_block_count > 0 ? hp->fast_block_count : 1), sizeof(so_layer));
    return m;
}

void so_model_free(so_model *m) {
    if (!m) return;
    free(m->layers);
    free(m->fast_layers);
    free(m->kv_k);
    free(m->kv_v);
    free(m);
}

static so_tensor *find_slot(so_model *m, const char *name) {
    if (!strcmp(name, "embeddings.weight")) return &m->embeddings;
    if (!strcmp(name, "codebook_embeddings.weight")) return &m->codebook_embeddings;
    if (!strcmp(name, "norm.weight")) return &m->norm;
    if (!strcmp(name, "fast_embeddings.weight")) return &m->fast_embeddings;
    if (!strcmp(name, "fast_norm.weight")) return &m->fast_norm;
    if (!strcmp(name, "fast_output.weight")) return &m->fast_output;
    if (!strcmp(name, "fast_project_in.weight")) return &m->fast_project_in;
    int il = -1, fast = 0, off = 0;
    if (sscanf(name, "layers.%d.%n", &il, &off) == 1 && off > 0) {
        fast = 0;
    } else if (sscanf(name, "fast_layers.%d.%n", &il, &off) == 1 && off > 0) {
        fast = 1;
    } else {
        return NULL;
    }
    const int nl = fast ? m->hp.fast_block_count : m->hp.block_count;
    if (il < 0 || il >= nl) return NULL;
    so_layer *L = fast ? &m->fast_layers[il] : &m->layers[il];
    const char *s = name + off;
    if (!strcmp(s, "attention_norm.weight")) return &L->attention_norm;
    if (!strcmp(s, "ffn_norm.weight")) return &L->ffn_norm;
    if (!strcmp(s, "attention.q_norm.weight")) return &L->q_norm;
    if (!strcmp(s, "attention.k_norm.weight")) return &L->k_norm;
    if (!strcmp(s, "attention.wqkv.weight")) return &L->wqkv;
    if (!strcmp(s, "attention.wo.weight")) return &L->wo;
    if (!strcmp(s, "feed_forward.w1.weight")) return &L->w1;
    if (!strcmp(s, "feed_forward.w2.weight")) return &L->w2;
    if (!strcmp(s, "feed_forward.w3.weight")) return &L->w3;
    return NULL;
}

int so_model_set_tensor(so_model *m, const char *name, int type, const int64_t ne[4],
                        const void *data, size_t nbytes) {
    so_tensor *t = find_slot(m, name);
    if (!t) return -1;
    const int64_t ne1 = ne[1] > 0 ? ne[1] : 1;
    if (so_row_bytes(type, ne[0]) < 0 || (size_t)(so_row_bytes(type, ne[0]) * ne1) != nbytes) return -2;
    t->type = type;
    t->ne0 = ne[0];
    t->ne1 = ne1;
    t->data = (const uint8_t *)data;
    return 0;
}

int so_model_check(so_model *m) {
    const so_hparams *hp = &m->hp;
    if (!m->embeddings.data || !m->codebook_embeddings.data || !m->norm.data) return -1;
    for (int i = 0; i < hp->block_count; ++i) {
        so_layer *L = &m->layers[i];
        if (!L->attention_norm.data || !L->ffn_norm.data || !L->wqkv.data || !L->wo.data ||
            !L->w1.data || !L->w2.data || !L->w3.data)
            return -2;
        if (hp->attention_qk_norm && (!L->q_norm.data || !L->k_norm.data)) return -3;
    }
    if (hp->has_fast_decoder) {
        if (!m->fast_embeddings.data || !m->fast_norm.data || !m->fast_output.data) return -4;
        for (int i = 0; i < hp->fast_block_count; ++i) {
            so_layer *L = &m->fast_layers[i];
            if (!L->attention_norm.data || !L->ffn_norm.data || !L->wqkv.data || !L->wo.data ||
                !L->w1.data || !L->w2.data || !L->w3.data)
                return -5;
            if (hp->fast_attention_qk_norm && (!L->q_norm.data || !L->k_norm.data)) return -6;
        }
    }
    return 0;
}

int so_kv_init(so_model *m, int32_t max_seq_len) {
    free(m->kv_k);
    free(m->kv_v);
    const size_t n = (size_t)m->hp.block_count * max_seq_len * m->hp.head_count_kv * m->hp.head_dim;
    m->kv_k = (uint16_t *)calloc(n ? n : 1, 2);
    m->kv_v = (uint16_t *)calloc(n ? n : 1, 2);
    m->max_seq_len = max_seq_len;
    m->n_past = 0;
    return (m->kv_k && m->kv_v) ? 0 : -1;
}

/* Positions 0..n_pos-1 of every layer's cache from k / v laid out
 * [layer][pos][kv_head][head_dim] (the cache layout of src/s2_model.cpp:746-747
 * with max_seq_len = n_pos); n_past = n_pos. */
int so_kv_load(so_model *m, const uint16_t *k, const uint16_t *v, int32_t n_pos) {
    if (!m->kv_k || n_pos < 0 || n_pos > m->max_seq_len) return -1;
    const size_t kvs = (size_t)m->hp.head_count_kv * m->hp.head_dim;
    for (int l = 0; l < m->hp.block_count; ++l) {
        memcpy(m->kv_k + (size_t)l * m->max_seq_len * kvs, k + (size_t)l * n_pos * kvs, (size_t)n_pos * kvs * 2);
        memcpy(m->kv_v + (size_t)l * m->max_seq_len * kvs, v + (size_t)l * n_pos * kvs, (size_t)n_pos * kvs * 2);
    }
    m->n_past = n_pos;
    return 0;
}

void so_kv_clear(so_model *m) {
    free(m->kv_k);
    free(m->kv_v);
    m->kv_k = m->kv_v = NULL;
    m->max_seq_len = 0;
    m->n_past = 0;
}

int32_t so_n_past(const so_model *m) { return m->n_past; }

/* ggml rms_norm (double accumulation of float squares) followed by ggml_mul
 * with the weight: y = (x * scale) * w   (src/s2_model.cpp:46-55) */
static void rms_norm_w(const float *x, const float *w, float eps, int64_t n, float *y) {
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i] * scale;
        y[i] = v * w[i];
    }
}

/* ggml_rope_ext mode 0 on one head: theta starts at pos and is multiplied by
 * theta_scale = base^(-2/n_dims) once per pair (ggml_rope_cache_init). */
static void rope_head(float *v, int hd, int32_t pos, float theta_scale) {
    float theta = (float)pos;
    for (int i0 = 0; i0 < hd; i0 += 2) {
        const float c = cosf(theta), s = sinf(theta);
        const float x0 = v[i0], x1 = v[i0 + 1];
        v[i0] = x0 * c - x1 * s;
        v[i0 + 1] = x0 * s + x1 * c;
        theta *= theta_scale;
    }
}

static inline float silu_f(float x) { return x / (1.0f + so_det_expf(-x)); }

/* One transformer stack over T tokens (shared by the Slow-AR and the Fast-AR).
 * x: [T][dim] residual stream, updated in place.
 * Past keys/values: kv_k/kv_v f16 for positions < n_past (NULL for the
 * Fast-AR), the current T tokens' K/V stay f32 (src/s2_model.cpp:1009-1020). */
static void run_layers(so_model *m, int fast, float *x, int T, int32_t n_past) {
    const so_hparams *hp = &m->hp;
    const int dim = fast ? hp->fast_embedding_length : hp->embedding_length;
    const int H = fast ? hp->fast_head_count : hp->head_count;
    const int Hkv = fast ? hp->fast_head_count_kv : hp->head_count_kv;
    const int hd = fast ? hp->fast_head_dim : hp->head_dim;
    const int ff = fast ? hp->fast_feed_forward_length : hp->feed_forward_length;
    const int nl = fast ? hp->fast_block_count : hp->block_count;
    const float eps = fast ? hp->fast_rms_norm_eps : hp->rms_norm_eps;
    const float base = fast ? hp->fast_rope_freq_base : hp->rope_freq_base;
    const int qkn = fast ? hp->fast_attention_qk_norm : hp->attention_qk_norm;
    const int qs = H * hd, kvs = Hkv * hd, qkvs = qs + 2 * kvs;
    const float theta_scale = powf(base, -2.0f / (float)hd);
    const float attn_scale = 1.0f / sqrtf((float)hd);
    const int rep = H / Hkv;
    const int n_kv = n_past + T;

    float *tmp = (float *)malloc(sizeof(float) * (size_t)T * dim);
    float *qkv = (float *)malloc(sizeof(float) * (size_t)T * qkvs);
    float *attn = (float *)malloc(sizeof(float) * (size_t)T * qs);
    float *h = (float *)malloc(sizeof(float) * (size_t)T * dim);
    float *g = (float *)malloc(sizeof(float) * (size_t)T * ff);
    float *u = (float *)malloc(sizeof(float) * (size_t)T * ff);
    float *kf = (float *)malloc(sizeof(float) * (size_t)n_kv * kvs);
    float *vf = (float *)malloc(sizeof(float) * (size_t)n_kv * kvs);

    for (int il = 0; il < nl; ++il) {
        so_layer *L = fast ? &m->fast_layers[il] : &m->layers[il];
        for (int t = 0; t < T; ++t)
            rms_norm_w(x + (int64_t)t * dim, (const float *)L->attention_norm.data, eps, dim, tmp + (int64_t)t * dim);
        matmat(L->wqkv.type, L->wqkv.data, qkvs, dim, T, tmp, qkv, qkvs);
        for (int t = 0; t < T; ++t) {
            float *q = qkv + (int64_t)t * qkvs, *k = q + qs;
            if (qkn) {
                for (int hh = 0; hh < H; ++hh) rms_norm_w(q + hh * hd, (const float *)L->q_norm.data, eps, hd, q + hh * hd);
                for (int hh = 0; hh < Hkv; ++hh) rms_norm_w(k + hh * hd, (const float *)L->k_norm.data, eps, hd, k + hh * hd);
            }
            for (int hh = 0; hh < H; ++hh) rope_head(q + hh * hd, hd, n_past + t, theta_scale);
            for (int hh = 0; hh < Hkv; ++hh) rope_head(k + hh * hd, hd, n_past + t, theta_scale);
        }
        /* keys / values visible to this call */
        if (!fast && n_past > 0) {
            const size_t lo = (size_t)il * m->max_seq_len * kvs;
            for (int64_t i = 0; i < (int64_t)n_past * kvs; ++i) {
                kf[i] = so_fp16_to_fp32(m->kv_k[lo + i]);
                vf[i] = so_fp16_to_fp32(m->kv_v[lo + i]);
            }
        }
        for (int t = 0; t < T; ++t) {
            memcpy(kf + (int64_t)(n_past + t) * kvs, qkv + (int64_t)t * qkvs + qs, sizeof(float) * kvs);
            memcpy(vf + (int64_t)(n_past + t) * kvs, qkv + (int64_t)t * qkvs + qs + kvs, sizeof(float) * kvs);
        }
        if (!fast) { /* store the call's K/V as f16 at n_past (ggml_cpy f32 -> f16) */
            const size_t lo = (size_t)il * m->max_seq_len * kvs + (size_t)n_past * kvs;
            for (int64_t i = 0; i < (int64_t)T * kvs; ++i) {
                m->kv_k[lo + i] = so_fp32_to_fp16(kf[(int64_t)n_past * kvs + i]);
                m->kv_v[lo + i] = so_fp32_to_fp16(vf[(int64_t)n_past * kvs + i]);
            }
        }
        /* attention: KQ = K.Q, scale, diag_mask_inf(n_past), soft_max, V.KQ
         * (src/s2_model.cpp:1023-1039), in fixed splits of SO_ATTN_SPLIT keys
         * (the convention the CUDA kernels share, so both agree bit for bit):
         *   s_j = float(sum_d double(k_j[d]) * double(q[d])) * scale
         *   split i: m_i = max s_j, e_j = det_expf(s_j - m_i),
         *            S_i = sum double(e_j), O_i[d] = sum double(v_j[d]) * double(e_j)
         *   M = max m_i, w_i = det_expf(m_i - M),
         *   out[d] = float((sum_i O_i[d] * double(w_i)) / (sum_i S_i * double(w_i)))
         * i.e. softmax(s) . V with the exponentials factored per split;
         * keys j >= len (the causal mask) are never visited. */
#pragma omp parallel for collapse(2) schedule(static)
        for (int t = 0; t < T; ++t) {
            for (int hh = 0; hh < H; ++hh) {
                const float *q = qkv + (int64_t)t * qkvs + hh * hd;
                const int kvh = hh / rep;
                const int len = n_past + t + 1;
                const int nsp = (len + SO_ATTN_SPLIT - 1) / SO_ATTN_SPLIT;
                float *sc = (float *)malloc(sizeof(float) * SO_ATTN_SPLIT);
                float *ms = (float *)malloc(sizeof(float) * (size_t)nsp);
                double *ss = (double *)malloc(sizeof(double) * (size_t)nsp);
                double *os = (double *)malloc(sizeof(double) * (size_t)nsp * hd);
                float M = -INFINITY;
                for (int i = 0; i < nsp; ++i) {
                    const int j0 = i * SO_ATTN_SPLIT, j1 = j0 + SO_ATTN_SPLIT < len ? j0 + SO_ATTN_SPLIT : len;
                    float mx = -INFINITY;
                    for (int j = j0; j < j1; ++j) {
                        const float *kk = kf + (int64_t)j * kvs + kvh * hd;
                        double s = 0.0;
                        for (int d = 0; d < hd; ++d) s += (double)kk[d] * (double)q[d];
                        sc[j - j0] = (float)s * attn_scale;
                        if (sc[j - j0] > mx) mx = sc[j - j0];
                    }
                    double sum = 0.0;
                    for (int j = j0; j < j1; ++j) {
                        sc[j - j0] = so_det_expf(sc[j - j0] - mx);
                        sum += (double)sc[j - j0];
                    }
                    for (int d = 0; d < hd; ++d) {
                        double o = 0.0;
                        for (int j = j0; j < j1; ++j) o += (double)vf[(int64_t)j * kvs + kvh * hd + d] * (double)sc[j - j0];
                        os[(size_t)i * hd + d] = o;
                    }
                    ms[i] = mx;
                    ss[i] = sum;
                    if (mx > M) M = mx;
                }
                double S = 0.0;
                for (int i = 0; i < nsp; ++i) {
                    const float w = so_det_expf(ms[i] - M);
                    ms[i] = w;
                    S += ss[i] * (double)w;
                }
                float *o = attn + (int64_t)t * qs + hh * hd;
                for (int d = 0; d < hd; ++d) {
                    double acc = 0.0;
                    for (int i = 0; i < nsp; ++i) acc += os[(size_t)i * hd + d] * (double)ms[i];
                    o[d] = (float)(acc / S);
                }
                free(sc); free(ms); free(ss); free(os);
            }
        }
        matmat(L->wo.type, L->wo.data, dim, qs, T, attn, tmp, dim);
        for (int64_t i = 0; i < (int64_t)T * dim; ++i) h[i] = x[i] + tmp[i];
        for (int t = 0; t < T; ++t)
            rms_norm_w(h + (int64_t)t * dim, (const float *)L->ffn_norm.data, eps, dim, tmp + (int64_t)t * dim);
        matmat(L->w1.type, L->w1.data, ff, dim, T, tmp, g, ff);
        matmat(L->w3.type, L->w3.data, ff, dim, T, tmp, u, ff);
        for (int64_t i = 0; i < (int64_t)T * ff; ++i) g[i] = silu_f(g[i]) * u[i];
        matmat(L->w2.type, L->w2.data, dim, ff, T, g, tmp, dim);
        for (int64_t i = 0; i < (int64_t)T * dim; ++i) x[i] = h[i] + tmp[i];
    }
    free(tmp); free(qkv); free(attn); free(h); free(g); free(u); free(kf); free(vf);
}

static void get_row(const so_tensor *t, int64_t row, float *dst) {
    const int64_t rb = so_row_bytes(t->type, t->ne0);
    so_dequant_row(t->type, t->data + row * rb, dst, t->ne0);
}

/* eval_cached (src/s2_model.cpp:860-1097) */
int so_eval(so_model *m, const int32_t *flat, int32_t T, float *hidden_out, float *logits_out) {
    const so_hparams *hp = &m->hp;
    if (T <= 0) return -1;
    if (m->n_past + T > m->max_seq_len) return -2;
    const int cbd = hp->num_codebooks + 1;
    const int dim = hp->embedding_length;
    const float sem_scale = 1.0f / sqrtf((float)cbd);
    float *x = (float *)malloc(sizeof(float) * (size_t)T * dim);
    float *row = (float *)malloc(sizeof(float) * (size_t)dim);
    float *cbs = (float *)malloc(sizeof(float) * (size_t)dim);
    for (int t = 0; t < T; ++t) {
        const int32_t tok = flat[t * cbd];
        const int is_sem = tok >= hp->semantic_begin_id && tok <= hp->semantic_end_id;
        if (tok < 0 || tok >= m->embeddings.ne1) { free(x); free(row); free(cbs); return -3; }
        float *xt = x + (int64_t)t * dim;
        get_row(&m->embeddings, tok, xt);
        if (hp->num_codebooks > 0) {
            /* codebook_sum = e_0 + e_1 + ... in order, ids offset by cb*codebook_size;
             * text tokens gather row 0 and are multiplied by a 0 mask. */
            for (int cb = 0; cb < hp->num_codebooks; ++cb) {
                int32_t id = is_sem ? flat[t * cbd + cb + 1] + cb * hp->codebook_size : 0;
                if (id < 0 || id >= m->codebook_embeddings.ne1) { free(x); free(row); free(cbs); return -3; }
                get_row(&m->codebook_embeddings, id, row);
                if (cb == 0) memcpy(cbs, row, sizeof(float) * dim);
                else for (int i = 0; i < dim; ++i) cbs[i] = cbs[i] + row[i];
            }
            const float mask = is_sem ? 1.0f : 0.0f;
            for (int i = 0; i < dim; ++i) xt[i] = xt[i] + cbs[i] * mask;
        }
        if (hp->scale_codebook_embeddings) {
            const float s = is_sem ? sem_scale : 1.0f;
            for (int i = 0; i < dim; ++i) xt[i] = xt[i] * s;
        }
    }
    run_layers(m, 0, x, T, m->n_past);
    float *hid = (float *)malloc(sizeof(float) * (size_t)dim);
    rms_norm_w(x + (int64_t)(T - 1) * dim, (const float *)m->norm.data, hp->rms_norm_eps, dim, hid);
    if (hidden_out) memcpy(hidden_out, hid, sizeof(float) * dim);
    if (logits_out) so_matvec(m->embeddings.type, m->embeddings.data, hp->vocab_size, dim, hid, logits_out);
    m->n_past += T;
    free(hid); free(x); free(row); free(cbs);
    return 0;
}

/* fast_decode (src/s2_model.cpp:1099-1255): recomputes the whole prefix */
int so_fast_decode(so_model *m, const float *hidden, const int32_t *prefix, int32_t n_prefix,
                   float *logits_out) {
    const so_hparams *hp = &m->hp;
    if (!hp->has_fast_decoder) return -1;
    if (n_prefix >= hp->num_codebooks || n_prefix < 0) return -2;
    const int dim = hp->fast_embedding_length;
    const int T = n_prefix + 1;
    float *x = (float *)malloc(sizeof(float) * (size_t)T * dim);
    if (m->fast_project_in.data) {
        so_matvec(m->fast_project_in.type, m->fast_project_in.data, dim, hp->embedding_length, hidden, x);
    } else {
        memcpy(x, hidden, sizeof(float) * dim);
    }
    for (int i = 0; i < n_prefix; ++i) {
        if (prefix[i] < 0 || prefix[i] >= m->fast_embeddings.ne1) { free(x); return -3; }
        get_row(&m->fast_embeddings, prefix[i], x + (int64_t)(i + 1) * dim);
    }
    run_layers(m, 1, x, T, 0);
    float *last = (float *)malloc(sizeof(float) * (size_t)dim);
    rms_norm_w(x + (int64_t)(T - 1) * dim, (const float *)m->fast_norm.data, hp->fast_rms_norm_eps, dim, last);
    so_matvec(m->fast_output.type, m->fast_output.data, hp->codebook_size, dim, last, logits_out);
    free(last); free(x);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* sampler (src/s2_sampler.cpp:42-99), ties broken by lowest index           */
/* ------------------------------------------------------------------------ */

typedef struct { float v; int32_t i; } so_item;

static int item_cmp(const void *a, const void *b) {
    const so_item *x = (const so_item *)a, *y = (const so_item *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

int32_t so_sample_token(const float *logits, int32_t n, float temperature, float top_p,
                        int32_t top_k, double u) {
    if (n <= 0) return 0;
    so_item *it = (so_item *)malloc(sizeof(so_item) * (size_t)n);
    for (int32_t i = 0; i < n; ++i) { it[i].v = logits[i]; it[i].i = i; }
    qsort(it, (size_t)n, sizeof(so_item), item_cmp);
    const int32_t k = top_k > 0 ? (top_k < n ? top_k : n) : n;
    const float tp = top_p < 0.0f ? 0.0f : (top_p > 1.0f ? 1.0f : top_p);
    /* softmax at T = 1 over all sorted logits */
    /* softmax_from_sorted_logits with the shared exp and a double-summed,
     * once-rounded normaliser */
    float *p = (float *)malloc(sizeof(float) * (size_t)n);
    const float mx = it[0].v;
    double sumd = 0.0;
    for (int32_t i = 0; i < n; ++i) { p[i] = so_det_expf(it[i].v - mx); sumd += (double)p[i]; }
    const float sum = (float)sumd;
    if (sum > 0.0f) for (int32_t i = 0; i < n; ++i) p[i] /= sum;
    so_item *f = (so_item *)malloc(sizeof(so_item) * (size_t)n);
    int32_t nf = 0;
    float cum = 0.0f;
    for (int32_t i = 0; i < n; ++i) {
        cum += p[i];
        if (i >= k || (i > 0 && cum > tp)) continue;
        f[nf++] = it[i];
    }
    if (nf == 0) f[nf++] = it[0];
    int32_t result = f[0].i;
    if (temperature > 0.0f) {
        float *q = (float *)malloc(sizeof(float) * (size_t)nf);
        float m2 = f[0].v;
        for (int32_t i = 1; i < nf; ++i) if (f[i].v > m2) m2 = f[i].v;
        float s = 0.0f;
        for (int32_t i = 0; i < nf; ++i) { q[i] = so_det_expf((f[i].v - m2) / temperature); s += q[i]; }
        if (s > 0.0f) for (int32_t i = 0; i < nf; ++i) q[i] /= s;
        float sp = 0.0f;
        for (int32_t i = 0; i < nf; ++i) sp += q[i];
        if (sp > 0.0f) {
            for (int32_t i = 0; i < nf; ++i) q[i] /= sp;
            /* std::discrete_distribution: normalised double cdf, lower_bound(u) */
            double tot = 0.0;
            for (int32_t i = 0; i < nf; ++i) tot += (double)q[i];
            double c = 0.0;
            int32_t pick = nf - 1;
            for (int32_t i = 0; i < nf - 1; ++i) {
                c += (double)q[i] / tot;
                if (c >= u) { pick = i; break; }
            }
            result = f[pick].i;
        }
        free(q);
    }
    free(it); free(p); free(f);
    return result;
}

/* ------------------------------------------------------------------------ */
/* generate (src/s2_generate.cpp:11-216)                                     */
/* ------------------------------------------------------------------------ */

static int32_t sample_masked(const so_model *m, const float *logits, int block_end,
                             int32_t im_end, float temp, float top_p, int32_t top_k, double u,
                             float *buf) {
    const so_hparams *hp = &m->hp;
    const int32_t V = hp->vocab_size;
    for (int32_t i = 0; i < V; ++i) buf[i] = -INFINITY;
    for (int32_t i = hp->semantic_begin_id; i <= hp->semantic_end_id && i < V; ++i) buf[i] = logits[i] + 0.0f;
    if (im_end >= 0 && im_end < V) buf[im_end] = logits[im_end] + 0.0f;
    if (block_end && im_end >= 0 && im_end < V) buf[im_end] = -INFINITY;
    return so_sample_token(buf, V, temp, top_p, top_k, u);
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

int so_generate(so_model *m, const int32_t *prompt, int32_t cols, const so_gen_params *gp,
                int32_t *codes_out, int32_t *n_frames_out) {
    double a, b;
    return so_generate_timed(m, prompt, cols, gp, codes_out, n_frames_out, &a, &b);
}

int so_generate_timed(so_model *m, const int32_t *prompt, int32_t cols, const so_gen_params *gp,
                      int32_t *codes_out, int32_t *n_frames_out, double *prefill_ms, double *loop_ms) {
    const so_hparams *hp = &m->hp;
    const int ncb = hp->num_codebooks > 0 ? hp->num_codebooks : 1;
    const int rows = hp->num_codebooks + 1;
    const int32_t V = hp->vocab_size;
    const int32_t maxn = gp->max_new_tokens;
    *n_frames_out = 0;
    int32_t *tm = (int32_t *)malloc(sizeof(int32_t) * (size_t)rows * cols);
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) tm[(size_t)c * rows + r] = prompt[(size_t)r * cols + c];
    float *hidden = (float *)malloc(sizeof(float) * (size_t)hp->embedding_length);
    float *logits = (float *)malloc(sizeof(float) * (size_t)V);
    float *buf = (float *)malloc(sizeof(float) * (size_t)V);
    float *flog = (float *)malloc(sizeof(float) * (size_t)(hp->codebook_size > 0 ? hp->codebook_size : 1));
    int32_t *codes = (int32_t *)calloc((size_t)ncb * (maxn > 0 ? maxn : 1), sizeof(int32_t));
    int rc = 0;
    const double t0 = now_ms();
    *prefill_ms = 0.0;
    *loop_ms = 0.0;
    if (so_eval(m, tm, cols, hidden, logits) != 0) { rc = -1; goto done; }
    *prefill_ms = now_ms() - t0;
    {
        int32_t main_tok = sample_masked(m, logits, gp->min_tokens_before_end > 0, gp->im_end_id,
                                         gp->temperature, gp->top_p, gp->top_k,
                                         so_philox_uniform(gp->seed, 0, SO_RNG_MAIN, gp->seq_id), buf);
        int32_t ras[10];
        int nras = 0;
        int32_t step = 0;
        int32_t cbv[64];
        while (main_tok != gp->im_end_id && step < maxn) {
            int in_win = 0;
            for (int i = 0; i < nras; ++i) if (ras[i] == main_tok) in_win = 1;
            if (nras > 0 && in_win && main_tok >= hp->semantic_begin_id && main_tok <= hp->semantic_end_id) {
                main_tok = sample_masked(m, logits, step < gp->min_tokens_before_end, gp->im_end_id,
                                         1.0f, 0.9f, gp->top_k,
                                         so_philox_uniform(gp->seed, (uint32_t)step, SO_RNG_RAS, gp->seq_id), buf);
            }
            if (nras == 10) { memmove(ras, ras + 1, sizeof(int32_t) * 9); nras = 9; }
            ras[nras++] = main_tok;
            int32_t sem = main_tok - hp->semantic_begin_id;
            if (sem < 0) sem = 0;
            if (sem >= hp->codebook_size) sem = hp->codebook_size - 1;
            cbv[0] = sem;
            for (int cb = 1; cb < ncb; ++cb) {
                if (so_fast_decode(m, hidden, cbv, cb, flog) != 0) {
                    for (int r = cb; r < ncb; ++r) cbv[r] = 0;
                    break;
                }
                cbv[cb] = so_sample_token(flog, hp->codebook_size, gp->temperature, gp->top_p, gp->top_k,
                                          so_philox_uniform(gp->seed, (uint32_t)step, SO_RNG_FAST0 + cb, gp->seq_id));
            }
            for (int cb = 0; cb < ncb; ++cb) codes[(size_t)cb * maxn + step] = cbv[cb];
            (*n_frames_out)++;
            int32_t in[65];
            in[0] = main_tok;
            for (int cb = 0; cb < ncb; ++cb) in[cb + 1] = cbv[cb];
            if (so_eval(m, in, 1, hidden, logits) != 0) { rc = -2; break; }
            step++;
            main_tok = sample_masked(m, logits, step < gp->min_tokens_before_end, gp->im_end_id,
                                     gp->temperature, gp->top_p, gp->top_k,
                                     so_philox_uniform(gp->seed, (uint32_t)step, SO_RNG_MAIN, gp->seq_id), buf);
        }
        *loop_ms = now_ms() - t0 - *prefill_ms;
    }
    {
        const int32_t nf = *n_frames_out;
        for (int cb = 0; cb < ncb; ++cb)
            for (int32_t t = 0; t < nf; ++t) codes_out[(size_t)cb * nf + t] = codes[(size_t)cb * maxn + t];
    }
done:
    free(tm); free(hidden); free(logits); free(buf); free(flog); free(codes);
    return rc;
}
