/*
 * s2_codec_oracle.c -- CPU restatement of s2.cpp's codec decode
 * (AudioCodec::decode, src/s2_codec.cpp:1297-1447): codes -> audio.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker of the CUDA codec decode
 * (s2.cpp_b200/csrc/s2k_codec.cu).  Only tests/ and bench.py's CPU legs load
 * it.
 *
 * The graph it follows (file:line inside the s2.cpp project):
 *   code clamp                  sanitize_decode_codes     src/s2_codec.cpp:1160-1188
 *   VQ decode, summed in order  build_vq_decode_stage / build_decode_codes_stage_backend  :620-678
 *   post-module transformer     build_transformer          :288-377 (windowed causal mask :264-286)
 *   upsample stages (reversed)  build_quantizer_decode_stage / build_quantizer_stage_up  :449-478
 *   ConvNeXt block              build_convnext_block       :393-418
 *   decoder                     build_decoder / build_decoder_block / build_residual_unit :379-391, 480-522
 *   snake, causal conv, causal transposed conv, layer norm   :183-248
 * The ggml ops it reaches (ggml is an absent submodule) are restated from
 * their published definitions: conv_1d (cross-correlation over a
 * zero-padded input, through an fp16 im2col: both operands rounded to fp16),
 * conv_1d_dw (the same), conv_transpose_1d (output length (L - 1) * s + K,
 * f32 operands after the reference's casts), mul_mat with F16 weights (the
 * activation rounded to fp16, ggml's vec_dot_type), norm / rms_norm,
 * gelu_erf, rope mode 0 with the theta *= base^(-2/n_dims) recurrence,
 * soft_max.  exp and sin are so_det_expf / so_det_sinf, as in the CUDA kernels.  Arithmetic is float
 * with every dot product and reduction accumulated in double; parity with the
 * CUDA path is to a tolerance (audio samples), not bit for bit.
 *
 * Layouts: activations are [time][channel] (ggml's channels-first ne order);
 * weights arrive in GGUF / ggml ne order: linear [in, out] (row o of memory
 * holds output o), conv1d [K, Cin, Cout], dwconv [K, 1, C], conv transpose
 * [K, Cout, Cin], codebook [dim, size].
 */
#include "s2_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    char name[128];
    float *data;  /* f32 copy */
    int64_t ne[4];
    int type;     /* the GGUF type it arrived in */
} sc_tensor;

struct so_codec {
    so_codec_hparams hp;
    sc_tensor *t;
    int n, cap;
};

so_codec *so_codec_create(const so_codec_hparams *hp) {
    so_codec *c = (so_codec *)calloc(1, sizeof(so_codec));
    if (!c) return NULL;
    c->hp = *hp;
    return c;
}

void so_codec_free(so_codec *c) {
    if (!c) return;
    for (int i = 0; i < c->n; ++i) free(c->t[i].data);
    free(c->t);
    free(c);
}

int so_codec_set_tensor(so_codec *c, const char *name, int type, const int64_t ne[4], const void *data) {
    if (type != SO_TYPE_F32 && type != SO_TYPE_F16) return -1;
    if (!strncmp(name, "c.", 2)) name += 2; /* the combined GGUF's codec prefix (src/s2_codec.cpp:812-818) */
    if (c->n == c->cap) {
        c->cap = c->cap ? 2 * c->cap : 64;
        c->t = (sc_tensor *)realloc(c->t, sizeof(sc_tensor) * (size_t)c->cap);
    }
    sc_tensor *t = &c->t[c->n++];
    memset(t, 0, sizeof(*t));
    strncpy(t->name, name, sizeof(t->name) - 1);
    t->type = type;
    int64_t n = 1;
    for (int d = 0; d < 4; ++d) {
        t->ne[d] = ne[d] > 0 ? ne[d] : 1;
        n *= t->ne[d];
    }
    t->data = (float *)malloc(sizeof(float) * (size_t)n);
    if (type == SO_TYPE_F32) {
        memcpy(t->data, data, sizeof(float) * (size_t)n);
    } else {
        const uint16_t *h = (const uint16_t *)data;
        for (int64_t i = 0; i < n; ++i) t->data[i] = so_fp16_to_fp32(h[i]);
    }
    return 0;
}

static const sc_tensor *get(const so_codec *c, const char *name) {
    for (int i = 0; i < c->n; ++i)
        if (!strcmp(c->t[i].name, name)) return &c->t[i];
    return NULL;
}

static int64_t numel(const sc_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

/* ---- ops on [L][C] activations ---- */

/* Accumulation order of the dot products: double (default), or float in
 * sequence when set -- a second valid order, so tests can measure how far
 * two correct evaluations of the fp16-rounded graph drift apart. */
static int g_f32_accum = 0;
void so_codec_set_f32_accum(int on) { g_f32_accum = on; }
static inline void acc(double *s, double v) {
    if (g_f32_accum) *s = (double)((float)*s + (float)v);
    else *s += v;
}

/* fp32 -> fp16 -> fp32, round to nearest even (ggml's fp16 conversions) */
static float r16(float x) { return so_fp16_to_fp32(so_fp32_to_fp16(x)); }

static float *rounded_copy(const float *x, int64_t n) {
    float *r = (float *)malloc(sizeof(float) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) r[i] = r16(x[i]);
    return r;
}

/* y[t][o] = b[o] + sum_i W[o][i] x[t][i].  ggml's mul_mat converts the
 * activation to the weight's vec_dot type: fp16 for F16 weights, so the
 * products are of fp16-rounded activations; F32 weights keep it in f32. */
static void linear(const float *x, int L, int in, const sc_tensor *w, const sc_tensor *b, float *y, int out) {
    float *xr = w->type == SO_TYPE_F16 ? rounded_copy(x, (int64_t)L * in) : NULL;
    const float *xs = xr ? xr : x;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < L; ++t)
        for (int o = 0; o < out; ++o) {
            double s = 0.0;
            const float *wr = w->data + (size_t)o * in;
            for (int i = 0; i < in; ++i) acc(&s, (double)wr[i] * (double)xs[(size_t)t * in + i]);
            y[(size_t)t * out + o] = b ? (float)s + b->data[o] : (float)s;
        }
    free(xr);
}

/* snake: x + sin(a x)^2 / a, per channel (src/s2_codec.cpp:197-204); sin is
 * so_det_sinf, as in the CUDA kernels */
static void snake(float *x, int L, int C, const sc_tensor *alpha) {
    for (int t = 0; t < L; ++t)
        for (int c = 0; c < C; ++c) {
            const float a = alpha->data[c], v = x[(size_t)t * C + c];
            const float s = so_det_sinf(a * v);
            x[(size_t)t * C + c] = v + (s * s) / a;
        }
}

/* causal conv1d, stride 1 (src/s2_codec.cpp:223-234 with stride 1: left pad
 * (K - 1) * dilation, no right pad): weight [Cout][Cin][K].  ggml_conv_1d
 * goes through an fp16 im2col, so both the input and the weight enter the
 * products rounded to fp16, whatever the weight's type. */
static void conv1d(const float *x, int L, int Cin, const sc_tensor *w, const sc_tensor *b, int dilation, float *y,
                   int Cout) {
    const int K = (int)w->ne[0];
    const int pad = (K - 1) * dilation;
    float *xr = rounded_copy(x, (int64_t)L * Cin);
    float *wr16 = rounded_copy(w->data, numel(w));
#pragma omp parallel for schedule(static)
    for (int t = 0; t < L; ++t)
        for (int o = 0; o < Cout; ++o) {
            double s = 0.0;
            for (int k = 0; k < K; ++k) {
                const int src = t - pad + k * dilation;
                if (src < 0) continue;
                const float *wr = wr16 + ((size_t)o * Cin) * K + k;
                for (int i = 0; i < Cin; ++i) acc(&s, (double)wr[(size_t)i * K] * (double)xr[(size_t)src * Cin + i]);
            }
            y[(size_t)t * Cout + o] = (float)s + b->data[o];
        }
    free(xr);
    free(wr16);
}

/* causal transposed conv (src/s2_codec.cpp:236-248): weight [Cin][Cout][K],
 * output length (L - 1) * s + K, then crop_right samples cut off the end.
 * The reference casts weight and input to F32 first: f32 products. */
static int conv_t1d(const float *x, int L, int Cin, const sc_tensor *w, const sc_tensor *b, int s, int crop,
                    float *y, int Cout) {
    const int K = (int)w->ne[0];
    const int Lo = (L - 1) * s + K - crop;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < Lo; ++t)
        for (int o = 0; o < Cout; ++o) {
            double a = 0.0;
            for (int k = t % s; k < K; k += s) {
                const int j = (t - k) / s;
                if (j < 0 || j >= L) continue;
                for (int i = 0; i < Cin; ++i)
                    acc(&a, (double)x[(size_t)j * Cin + i] * (double)w->data[((size_t)i * Cout + o) * K + k]);
            }
            y[(size_t)t * Cout + o] = (float)a + b->data[o];
        }
    return Lo;
}

static void rms_norm_rows(const float *x, int L, int C, const sc_tensor *w, float eps, float *y) {
    for (int t = 0; t < L; ++t) {
        double s = 0.0;
        for (int c = 0; c < C; ++c) s += (double)(x[(size_t)t * C + c] * x[(size_t)t * C + c]);
        const float sc = 1.0f / sqrtf((float)(s / C) + eps);
        for (int c = 0; c < C; ++c) y[(size_t)t * C + c] = (x[(size_t)t * C + c] * sc) * w->data[c];
    }
}

/* ggml_norm then affine (src/s2_codec.cpp:189-195) */
static void layer_norm_rows(float *x, int L, int C, const sc_tensor *w, const sc_tensor *b, float eps) {
    for (int t = 0; t < L; ++t) {
        float *row = x + (size_t)t * C;
        double s = 0.0, v = 0.0;
        for (int c = 0; c < C; ++c) s += row[c];
        const float mean = (float)(s / C);
        for (int c = 0; c < C; ++c) {
            row[c] = row[c] - mean;
            v += (double)row[c] * (double)row[c];
        }
        const float sc = 1.0f / sqrtf((float)(v / C) + eps);
        for (int c = 0; c < C; ++c) row[c] = row[c] * sc * w->data[c] + b->data[c];
    }
}

static float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }
static float silu(float x) { return x / (1.0f + so_det_expf(-x)); }

/* rope mode 0 on one head vector (adjacent pairs, theta recurrence) */
static void rope(float *v, int hd, int pos, float base) {
    const float ts = powf(base, -2.0f / (float)hd);
    float theta = (float)pos;
    for (int i = 0; i < hd; i += 2) {
        const float c = cosf(theta), s = sinf(theta), x0 = v[i], x1 = v[i + 1];
        v[i] = x0 * c - x1 * s;
        v[i + 1] = x0 * s + x1 * c;
        theta *= ts;
    }
}

static char nm[512];
static const char *fmt1(const char *a, int i, const char *b) {
    snprintf(nm, sizeof(nm), "%s%d%s", a, i, b);
    return nm;
}

/* post-module transformer over the code frames (src/s2_codec.cpp:288-377) */
static int transformer(const so_codec *c, float *x, int L) {
    const so_codec_hparams *hp = &c->hp;
    const int dim = hp->rvq_dim, hd = hp->rvq_head_dim, H = dim / hd;
    const int Hk = hp->rvq_n_local_heads > 0 ? hp->rvq_n_local_heads : H, rep = H / Hk;
    const int qs = H * hd, ks = Hk * hd;
    const int W = hp->rvq_window_size;
    float *h = (float *)malloc(sizeof(float) * (size_t)L * dim);
    float *qkv = NULL, *att = (float *)malloc(sizeof(float) * (size_t)L * qs), *tmp = (float *)malloc(sizeof(float) * (size_t)L * dim);
    /* as many layers as the file holds (src/s2_codec.cpp:300-303) */
    for (int l = 0;; ++l) {
        char p[128];
        snprintf(p, sizeof(p), "quantizer.post_module.layers.%d.", l);
#define T(sfx) get(c, (snprintf(nm, sizeof(nm), "%s%s", p, sfx), nm))
        const sc_tensor *wqkv = T("attention.wqkv.weight");
        if (!wqkv) break;
        const sc_tensor *wo = T("attention.wo.weight");
        const sc_tensor *w1 = T("feed_forward.w1.weight"), *w2 = T("feed_forward.w2.weight"), *w3 = T("feed_forward.w3.weight");
        const sc_tensor *an = T("attention_norm.weight"), *fn = T("ffn_norm.weight");
        const sc_tensor *ag = T("attention_layer_scale.gamma"), *fg = T("ffn_layer_scale.gamma");
#undef T
        if (!wqkv || !wo || !w1 || !w2 || !w3 || !an || !fn || !ag || !fg) return -10 - l;
        const int qkvs = (int)wqkv->ne[1], ff = (int)w1->ne[1];
        qkv = (float *)realloc(qkv, sizeof(float) * (size_t)L * qkvs);
        rms_norm_rows(x, L, dim, an, hp->rvq_norm_eps, h);
        linear(h, L, dim, wqkv, NULL, qkv, qkvs);
        for (int t = 0; t < L; ++t) {
            for (int hh = 0; hh < H; ++hh) rope(qkv + (size_t)t * qkvs + hh * hd, hd, t, hp->rvq_rope_base);
            for (int hh = 0; hh < Hk; ++hh) rope(qkv + (size_t)t * qkvs + qs + hh * hd, hd, t, hp->rvq_rope_base);
        }
        const float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel for collapse(2) schedule(static)
        for (int t = 0; t < L; ++t)
            for (int hh = 0; hh < H; ++hh) {
                const float *q = qkv + (size_t)t * qkvs + hh * hd;
                const int kh = hh / rep;
                const int k0 = W > 0 ? (t - W + 1 > 0 ? t - W + 1 : 0) : 0;
                float *sc = (float *)malloc(sizeof(float) * (size_t)(t - k0 + 1));
                float mx = -INFINITY;
                for (int k = k0; k <= t; ++k) {
                    const float *kk = qkv + (size_t)k * qkvs + qs + kh * hd;
                    double s = 0.0;
                    for (int d = 0; d < hd; ++d) acc(&s, (double)q[d] * (double)kk[d]);
                    sc[k - k0] = (float)s * scale;
                    if (sc[k - k0] > mx) mx = sc[k - k0];
                }
                double sum = 0.0;
                for (int k = k0; k <= t; ++k) {
                    sc[k - k0] = so_det_expf(sc[k - k0] - mx);
                    sum += sc[k - k0];
                }
                const float inv = (float)(1.0 / sum);
                for (int k = k0; k <= t; ++k) sc[k - k0] *= inv;
                for (int d = 0; d < hd; ++d) {
                    double o = 0.0;
                    for (int k = k0; k <= t; ++k) acc(&o, (double)sc[k - k0] * (double)qkv[(size_t)k * qkvs + qs + ks + kh * hd + d]);
                    att[(size_t)t * qs + hh * hd + d] = (float)o;
                }
                free(sc);
            }
        linear(att, L, qs, wo, NULL, tmp, dim);
        for (int t = 0; t < L; ++t)
            for (int i = 0; i < dim; ++i) x[(size_t)t * dim + i] += tmp[(size_t)t * dim + i] * ag->data[i];
        rms_norm_rows(x, L, dim, fn, hp->rvq_norm_eps, h);
        float *g = (float *)malloc(sizeof(float) * (size_t)L * ff), *u = (float *)malloc(sizeof(float) * (size_t)L * ff);
        linear(h, L, dim, w1, NULL, g, ff);
        linear(h, L, dim, w3, NULL, u, ff);
        for (int64_t i = 0; i < (int64_t)L * ff; ++i) g[i] = silu(g[i]) * u[i];
        linear(g, L, ff, w2, NULL, tmp, dim);
        for (int t = 0; t < L; ++t)
            for (int i = 0; i < dim; ++i) x[(size_t)t * dim + i] += tmp[(size_t)t * dim + i] * fg->data[i];
        free(g);
        free(u);
    }
    const sc_tensor *nw = get(c, "quantizer.post_module.norm.weight");
    if (!nw) return -9;
    memcpy(h, x, sizeof(float) * (size_t)L * dim);
    rms_norm_rows(h, L, dim, nw, hp->rvq_norm_eps, x);
    free(h);
    free(qkv);
    free(att);
    free(tmp);
    return 0;
}

int64_t so_codec_samples(const so_codec *c, int32_t n_frames) {
    int64_t n = n_frames;
    for (int i = 0; i < c->hp.n_downsample; ++i) n *= c->hp.quantizer_downsample_factor[i];
    for (int i = 0; i < c->hp.n_decoder_rates; ++i) n *= c->hp.decoder_rates[i];
    return n;
}

/* codes [ncb][n_frames] cb-major -> audio [n_samples] */
int so_codec_decode(const so_codec *c, const int32_t *codes, int32_t n_frames, float *audio, int64_t cap,
                    int64_t *n_samples) {
    const so_codec_hparams *hp = &c->hp;
    if (n_frames <= 0) return -1;
    const int nq = hp->quantizer_residual_codebooks + 1;
    /* the largest [time][channel] buffer of the decode, walking its shapes */
    int64_t L = n_frames, Cw = hp->quantizer_input_dim, maxe = L * Cw;
    for (int i = 0; i < hp->n_downsample; ++i) {
        const sc_tensor *tw = get(c, fmt1("quantizer.upsample.", i, ".0.conv.weight"));
        if (!tw) return -5;
        L = (L - 1) * hp->quantizer_downsample_factor[hp->n_downsample - 1 - i] + tw->ne[0];
        Cw = tw->ne[1];
        if (L * Cw > maxe) maxe = L * Cw;
    }
    {
        const sc_tensor *w0 = get(c, "decoder.model.0.conv.weight");
        if (!w0) return -6;
        Cw = w0->ne[2];
        if (L * Cw > maxe) maxe = L * Cw;
    }
    for (int i = 0; i < hp->n_decoder_rates; ++i) {
        const sc_tensor *tw = get(c, fmt1("decoder.model.", i + 1, ".block.1.conv.weight"));
        if (!tw) return -7;
        const int s = hp->decoder_rates[i];
        L = (L - 1) * s + tw->ne[0] - s;
        Cw = tw->ne[1];
        if (L * Cw > maxe) maxe = L * Cw;
    }
    if (cap < L) return -2;
    float *a = (float *)calloc((size_t)maxe, sizeof(float)), *b = (float *)calloc((size_t)maxe, sizeof(float));
    float *r = (float *)calloc((size_t)maxe, sizeof(float));
    if (!a || !b || !r) return -3;
    /* VQ decode: semantic quantizer, then residual ones, added in order */
    const int C0 = hp->quantizer_input_dim;
    for (int q = 0; q < nq; ++q) {
        char p[128];
        if (q == 0) snprintf(p, sizeof(p), "quantizer.semantic_quantizer.quantizers.0.");
        else snprintf(p, sizeof(p), "quantizer.quantizer.quantizers.%d.", q - 1);
        const sc_tensor *cb = get(c, (snprintf(nm, sizeof(nm), "%scodebook.weight", p), nm));
        const sc_tensor *ow = get(c, (snprintf(nm, sizeof(nm), "%sout_proj.weight", p), nm));
        const sc_tensor *ob = get(c, (snprintf(nm, sizeof(nm), "%sout_proj.bias", p), nm));
        if (!cb || !ow || !ob) return -4;
        const int cd = (int)cb->ne[0], cs = (int)cb->ne[1];
        /* out_proj is a kernel-1 conv, [1, cd, out], or a plain [cd, out] matrix (src/s2_codec.cpp:634-638) */
        const int64_t ocd = ow->ne[0] == 1 ? ow->ne[1] : ow->ne[0];
        if (ocd != cd) return -4;
        const int size = q == 0 ? hp->quantizer_semantic_codebook_size : hp->quantizer_residual_codebook_size;
        for (int t = 0; t < n_frames; ++t) {
            int code = codes[(size_t)q * n_frames + t];
            code = code < 0 ? 0 : (code >= size ? size - 1 : code); /* src/s2_codec.cpp:1160-1168 */
            if (code >= cs) code = cs - 1;
            for (int o = 0; o < C0; ++o) {
                double s = 0.0;
                for (int d = 0; d < cd; ++d) acc(&s, (double)ow->data[(size_t)o * cd + d] * (double)cb->data[(size_t)code * cd + d]);
                const float v = (float)s + ob->data[o];
                if (q == 0) a[(size_t)t * C0 + o] = v;
                else a[(size_t)t * C0 + o] += v;
            }
        }
    }
    int rc = transformer(c, a, n_frames);
    if (rc) return rc;
    /* upsample stages, factors in reverse order (src/s2_codec.cpp:472-477) */
    L = n_frames;
    int C = C0;
    for (int i = 0; i < hp->n_downsample; ++i) {
        const int f = hp->quantizer_downsample_factor[hp->n_downsample - 1 - i];
        char p[128];
        snprintf(p, sizeof(p), "quantizer.upsample.%d.", i);
#define T(sfx) get(c, (snprintf(nm, sizeof(nm), "%s%s", p, sfx), nm))
        const sc_tensor *tw = T("0.conv.weight"), *tb = T("0.conv.bias");
        const sc_tensor *dw = T("1.dwconv.conv.weight"), *db = T("1.dwconv.conv.bias");
        const sc_tensor *lw = T("1.norm.weight"), *lb = T("1.norm.bias");
        const sc_tensor *p1w = T("1.pwconv1.weight"), *p1b = T("1.pwconv1.bias");
        const sc_tensor *p2w = T("1.pwconv2.weight"), *p2b = T("1.pwconv2.bias"), *gm = T("1.gamma");
#undef T
        if (!tw || !tb || !dw || !db || !lw || !lb || !p1w || !p1b || !p2w || !p2b || !gm) return -5;
        const int Co = (int)tw->ne[1];
        const int Lo = conv_t1d(a, (int)L, C, tw, tb, f, 0, b, Co);
        L = Lo;
        C = Co;
        /* ConvNeXt: causal depthwise conv (ggml_conv_1d_dw: fp16 im2col, so
         * fp16-rounded input and weight), layer norm, MLP with GELU, gamma,
         * residual */
        const int K = (int)dw->ne[0];
        float *br = rounded_copy(b, L * C), *dwr = rounded_copy(dw->data, numel(dw));
#pragma omp parallel for schedule(static)
        for (int t = 0; t < L; ++t)
            for (int ch2 = 0; ch2 < C; ++ch2) {
                double s = 0.0;
                for (int k = 0; k < K; ++k) {
                    const int src = t - (K - 1) + k;
                    if (src >= 0) acc(&s, (double)dwr[(size_t)ch2 * K + k] * (double)br[(size_t)src * C + ch2]);
                }
                r[(size_t)t * C + ch2] = (float)s + db->data[ch2];
            }
        free(br);
        free(dwr);
        layer_norm_rows(r, (int)L, C, lw, lb, 1e-6f);
        const int hid = (int)p1w->ne[1];
        float *m = (float *)malloc(sizeof(float) * (size_t)L * hid);
        linear(r, (int)L, C, p1w, p1b, m, hid);
        for (int64_t e = 0; e < L * hid; ++e) m[e] = gelu_erf(m[e]);
        linear(m, (int)L, hid, p2w, p2b, r, C);
        free(m);
        for (int64_t e = 0; e < L * C; ++e) a[e] = b[e] + r[e] * gm->data[e % C];
    }
    /* decoder (src/s2_codec.cpp:497-522) */
    {
        const sc_tensor *w0 = get(c, "decoder.model.0.conv.weight"), *b0 = get(c, "decoder.model.0.conv.bias");
        if (!w0 || !b0) return -6;
        const int Co = (int)w0->ne[2];
        conv1d(a, (int)L, C, w0, b0, 1, b, Co);
        C = Co;
        memcpy(a, b, sizeof(float) * (size_t)L * C);
    }
    for (int i = 0; i < hp->n_decoder_rates; ++i) {
        const int s = hp->decoder_rates[i];
        char p[128];
        snprintf(p, sizeof(p), "decoder.model.%d.block.", i + 1);
#define T(sfx) get(c, (snprintf(nm, sizeof(nm), "%s%s", p, sfx), nm))
        const sc_tensor *al = T("0.alpha"), *tw = T("1.conv.weight"), *tb = T("1.conv.bias");
        if (!al || !tw || !tb) return -7;
        snake(a, (int)L, C, al);
        const int Co = (int)tw->ne[1];
        L = conv_t1d(a, (int)L, C, tw, tb, s, s, b, Co);
        C = Co;
        for (int u = 0; u < 3; ++u) {
            const int dil = u == 0 ? 1 : (u == 1 ? 3 : 9);
            char q[32];
            snprintf(q, sizeof(q), "%d.block.", 2 + u);
            const sc_tensor *a0 = get(c, (snprintf(nm, sizeof(nm), "%s%s0.alpha", p, q), nm));
            const sc_tensor *c1w = get(c, (snprintf(nm, sizeof(nm), "%s%s1.conv.weight", p, q), nm));
            const sc_tensor *c1b = get(c, (snprintf(nm, sizeof(nm), "%s%s1.conv.bias", p, q), nm));
            const sc_tensor *a2 = get(c, (snprintf(nm, sizeof(nm), "%s%s2.alpha", p, q), nm));
            const sc_tensor *c3w = get(c, (snprintf(nm, sizeof(nm), "%s%s3.conv.weight", p, q), nm));
            const sc_tensor *c3b = get(c, (snprintf(nm, sizeof(nm), "%s%s3.conv.bias", p, q), nm));
            if (!a0 || !c1w || !c1b || !a2 || !c3w || !c3b) return -8;
            memcpy(r, b, sizeof(float) * (size_t)L * C);
            snake(r, (int)L, C, a0);
            conv1d(r, (int)L, C, c1w, c1b, dil, a, C);
            snake(a, (int)L, C, a2);
            conv1d(a, (int)L, C, c3w, c3b, 1, r, C);
            for (int64_t e = 0; e < L * C; ++e) b[e] += r[e];
        }
#undef T
        memcpy(a, b, sizeof(float) * (size_t)L * C);
    }
    {
        const int last = hp->n_decoder_rates + 1;
        const sc_tensor *al = get(c, fmt1("decoder.model.", last, ".alpha"));
        char w[96], bb[96];
        snprintf(w, sizeof(w), "decoder.model.%d.conv.weight", last + 1);
        snprintf(bb, sizeof(bb), "decoder.model.%d.conv.bias", last + 1);
        const sc_tensor *fw = get(c, w), *fb = get(c, bb);
        if (!al || !fw || !fb) return -9;
        snake(a, (int)L, C, al);
        conv1d(a, (int)L, C, fw, fb, 1, b, (int)fw->ne[2]);
        for (int64_t t = 0; t < L; ++t) audio[t] = tanhf(b[t * (int)fw->ne[2]]);
    }
    *n_samples = L;
    free(a);
    free(b);
    free(r);
    return 0;
}
