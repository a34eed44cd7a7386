/*
 * s2synth.c -- seeded synthetic GGUF-native weights for the s2.cpp model family.
 *
 * This is input generation for tests and benchmarks (there are no real
 * checkpoints offline).  It writes tensors in exactly the on-disk block
 * formats s2.cpp reads from GGUF (ggml ne order [in, out], rows of blocks):
 *   F32 / F16                      plain values
 *   Q8_0  (34 B / 32 weights)      ggml's reference quantizer: d = amax/127,
 *                                  q = roundf(x / d)  (identical to gguf-py
 *                                  Q8_0.quantize_blocks, checked in tests)
 *   Q4_K  (144 B / 256 weights)    a simple min/scale fit per 32-sub-block
 *   Q6_K  (210 B / 256 weights)    a simple absmax fit per 16-sub-block
 * The K-quant fits are valid blocks but not ggml's iterative search: the
 * model's weights are by definition the dequantized values.
 *
 * Values are N(mean, std) drawn by Box-Muller from Philox4x32-10 keyed by
 * (seed) and countered by (element pair index, tensor id), so any tensor can
 * be regenerated independently and in parallel.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

static void philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1,
                   uint32_t out[4]) {
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* 4 normals for element group g (elements 4g..4g+3) */
static void normals4(uint64_t seed, uint32_t tensor_id, uint64_t g, float mean, float std, float o[4]) {
    uint32_t r[4];
    philox((uint32_t)g, (uint32_t)(g >> 32), tensor_id, 0x53594e54u, (uint32_t)seed, (uint32_t)(seed >> 32), r);
    for (int k = 0; k < 2; ++k) {
        const float u1 = ((float)(r[2 * k] >> 8) + 1.0f) * (1.0f / 16777216.0f); /* (0,1] */
        const float u2 = (float)(r[2 * k + 1] >> 8) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1));
        const float a = 6.28318530717958647692f * u2;
        o[2 * k] = mean + std * rad * cosf(a);
        o[2 * k + 1] = mean + std * rad * sinf(a);
    }
}

static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000, sh = 126 - e;
        uint32_t r = m >> sh, rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (r & 1))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = (ax >> 13) - (112u << 10), rem = ax & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) r++;
    return (uint16_t)(sign | r);
}

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {
            int e = -1;
            do { e++; man <<= 1; } while ((man & 0x400) == 0);
            bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 0x1f) bits = sign | 0x7f800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static void quant_q8_0(const float *x, uint8_t *o) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) { float a = fabsf(x[j]); if (a > amax) amax = a; }
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t dh = f32_to_f16(d);
    memcpy(o, &dh, 2);
    for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)(int8_t)(int)roundf(x[j] * id);
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q4_K: w = d*sc_j*q - dmin*m_j, q in [0,15], sc/m 6-bit */
static void quant_q4_K(const float *x, uint8_t *o) {
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int l = 1; l < 32; ++l) { float v = x[32 * j + l]; if (v < mn) mn = v; if (v > mx) mx = v; }
        if (mn > 0) mn = 0;
        scale[j] = (mx - mn) / 15.0f;
        minv[j] = -mn;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (minv[j] > max_min) max_min = minv[j];
    }
    const float d = max_scale / 63.0f, dmin = max_min / 63.0f;
    const uint16_t dh = f32_to_f16(d), mh = f32_to_f16(dmin);
    memcpy(o, &dh, 2);
    memcpy(o + 2, &mh, 2);
    const float dd = f16_to_f32(dh), dm = f16_to_f32(mh);
    int sc[8], mi[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = dd > 0 ? clampi((int)lrintf(scale[j] / dd), 0, 63) : 0;
        mi[j] = dm > 0 ? clampi((int)lrintf(minv[j] / dm), 0, 63) : 0;
    }
    uint8_t *s = o + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mi[j] & 63) | ((mi[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mi[j + 4] & 0xF) << 4));
    }
    uint8_t *q = o + 16;
    for (int c = 0; c < 4; ++c) {
        for (int l = 0; l < 32; ++l) {
            int qv[2];
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * c + h;
                const float ds = dd * (float)sc[j], ms = dm * (float)mi[j];
                qv[h] = ds > 0 ? clampi((int)lrintf((x[32 * j + l] + ms) / ds), 0, 15) : 0;
            }
            q[32 * c + l] = (uint8_t)(qv[0] | (qv[1] << 4));
        }
    }
}

/* Q6_K: w = d*sc_j*(q-32), q in [0,63], sc int8 per 16 weights */
static void quant_q6_K(const float *x, uint8_t *o) {
    float sub[16], amax_all = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float a = 0.0f;
        for (int l = 0; l < 16; ++l) { float v = fabsf(x[16 * j + l]); if (v > a) a = v; }
        sub[j] = a / 31.0f;
        if (sub[j] > amax_all) amax_all = sub[j];
    }
    const float d = amax_all / 127.0f;
    const uint16_t dh = f32_to_f16(d);
    const float dd = f16_to_f32(dh);
    int8_t sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = (int8_t)(dd > 0 ? clampi((int)lrintf(sub[j] / dd), -127, 127) : 0);
    uint8_t *ql = o, *qh = o + 128;
    memset(ql, 0, 128);
    memset(qh, 0, 64);
    for (int i = 0; i < 256; ++i) {
        const int j = i / 16;
        const float ds = dd * (float)sc[j];
        const int q = ds > 0 ? clampi((int)lrintf(x[i] / ds), -32, 31) + 32 : 32;
        const int h = i / 128, k = (i % 128) / 32, l = i % 32;
        const int lo = q & 0xF, hi = q >> 4;
        ql[64 * h + (k % 2) * 32 + l] |= (uint8_t)(lo << (4 * (k / 2)));
        qh[32 * h + l] |= (uint8_t)(hi << (2 * k));
    }
    memcpy(o + 192, sc, 16);
    memcpy(o + 208, &dh, 2);
}

int64_t s2synth_row_bytes(int type, int64_t n) {
    switch (type) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q8_0: return n % 32 ? -1 : n / 32 * 34;
    case T_Q4_K: return n % 256 ? -1 : n / 256 * 144;
    case T_Q6_K: return n % 256 ? -1 : n / 256 * 210;
    default: return -1;
    }
}

/* Fill `rows` rows of `n` values of N(mean, std) in GGUF-native `type` blocks. */
int s2synth_fill(int type, int64_t n, int64_t rows, uint64_t seed, uint32_t tensor_id, float mean,
                 float std, void *out) {
    const int64_t rb = s2synth_row_bytes(type, n);
    if (rb < 0 || n % 4) return -1;
    const int64_t blk = (type == T_Q8_0) ? 32 : ((type == T_Q4_K || type == T_Q6_K) ? 256 : 256);
    const int64_t total = n * rows;
    const int64_t nblk = (total + blk - 1) / blk;
    uint8_t *o = (uint8_t *)out;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) {
        float x[256];
        const int64_t e0 = b * blk;
        const int64_t cnt = (e0 + blk <= total) ? blk : total - e0;
        for (int64_t g = 0; g < cnt / 4; ++g) normals4(seed, tensor_id, (uint64_t)(e0 / 4 + g), mean, std, x + 4 * g);
        switch (type) {
        case T_F32: memcpy(o + e0 * 4, x, (size_t)cnt * 4); break;
        case T_F16:
            for (int64_t i = 0; i < cnt; ++i) {
                uint16_t h = f32_to_f16(x[i]);
                memcpy(o + (e0 + i) * 2, &h, 2);
            }
            break;
        case T_Q8_0: quant_q8_0(x, o + b * 34); break;
        case T_Q4_K: quant_q4_K(x, o + b * 144); break;
        case T_Q6_K: quant_q6_K(x, o + b * 210); break;
        }
    }
    return 0;
}

/* Fill int32 token ids uniform in [lo, hi] (inclusive) */
void s2synth_ids(uint64_t seed, uint32_t stream, int32_t lo, int32_t hi, int64_t n, int32_t *out) {
    const uint32_t span = (uint32_t)(hi - lo + 1);
    for (int64_t i = 0; i < n; ++i) {
        uint32_t r[4];
        philox((uint32_t)i, (uint32_t)((uint64_t)i >> 32), stream, 0x49445321u, (uint32_t)seed, (uint32_t)(seed >> 32), r);
        out[i] = lo + (int32_t)(((uint64_t)r[0] * span) >> 32);
    }
}

void s2synth_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* Quantize n floats (n % 32 == 0) to Q8_0 with the same rule s2synth_fill uses. */
void s2synth_quantize_q8_0(const float *x, int64_t n, uint8_t *out) {
    for (int64_t b = 0; b < n / 32; ++b) quant_q8_0(x + 32 * b, out + 34 * b);
}
