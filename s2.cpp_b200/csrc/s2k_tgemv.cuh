// s2k_tgemv.cuh -- Q8_0 dequant-GEMV on tiled weights, shared by the
// persistent decode kernel (s2k_mega.cu) and the standalone GEMV kernel
// (s2k_gemv.cu).
//
// Weight layout (written once at upload from GGUF's 34-byte Q8_0 blocks):
//   the matrix [R][K] is cut into tiles of kTR = 32 rows x kTK = 512 columns;
//   tile (rt, kt) lives at byte ((rt * K/kTK) + kt) * kTileBytes and holds
//     int8 quants [32][512] row-major, then fp16 scales [32][16] row-major.
//   Tiles of one row tile are contiguous, so a CTA's share of the matrix (a
//   contiguous range of tiles) streams with one 17 KB bulk copy per stage.
//
// Work split: CTA c of G owns the whole row tiles [RT*c/G, RT*(c+1)/G) (RT =
// R/32), so no row is ever split across CTAs and no cross-CTA combine is
// needed.  When RT is not a multiple of G some CTAs stream one row tile more
// (or, for RT < G, some stream none); a CTA can pull about twice its even
// share of HBM bandwidth through its ring, so the busier CTAs catch up while
// the others idle and the op stays close to its HBM time.
//
// Consumer mapping: 8 consumer warps, warp w owns rows 4w..4w+3 of every
// tile; lane l owns 16-byte column chunk l of the tile, i.e. half of Q8_0
// block l/2.  A lane keeps its 4 x MT partial row sums in registers across
// all K-tiles of a row tile; the warp reduces them once per row tile with a
// transposing butterfly and lanes 0, 8, 16, 24 store one row each.  Rows (2i, 2i+1) of a SwiGLU matrix (gate/up interleaved at upload)
// sit in the same warp, so the epilogue needs no cross-warp exchange.
//
// Arithmetic (identical to ggml's vec_dot_q8_0_q8_0 terms, summed order-free):
// the term of one 16-value half block, s_half * (d_w * d_x) with |s_half| <
// 2^18 and d_w * d_x exact in float, is exact in double; terms are summed in
// double and each row is rounded to float once.
#pragma once

#include "s2k_common.cuh"

namespace s2k {

constexpr int kTR = 32;                          // rows per tile
constexpr int kTK = 512;                         // columns per tile
constexpr int kTileQ = kTR * kTK;                // int8 quants per tile
constexpr int kTileBytes = kTileQ + kTR * (kTK / 32) * 2;  // + fp16 scales = 17408
constexpr int kTW = 8;                           // consumer warps of a tiled-GEMV CTA
constexpr int kTNC = kTW * 32;                   // consumer threads
constexpr int kTRW = kTR / kTW;                  // rows per warp
constexpr int kNormMax = 4096;                   // longest RMSNorm'd activation row

// K-quant tiles (32 rows x 512 columns = 2 super-blocks of 256 per row):
//   Q4_K: qs [32][2][128] (nibbles as stored by ggml), then per (row, super-
//         block) the 16-byte header d, dmin (fp16), 12 packed 6-bit scale/min
//         bytes: 9216 bytes (144 per super-block, as GGUF).
//   Q6_K: ql [32][2][128], qh [32][2][64], scales [32][2][16] (int8),
//         d [32][2] (fp16): 13440 bytes (210 per super-block).
constexpr int kTileBytesQ4K = kTR * 2 * 144;
constexpr int kTileBytesQ6K = kTR * 2 * 210;
constexpr int kQ4kHdr = kTR * 2 * 128;                  // offset of the Q4_K headers
constexpr int kQ6kQh = kTR * 2 * 128, kQ6kSc = kQ6kQh + kTR * 2 * 64, kQ6kD = kQ6kSc + kTR * 2 * 16;
static_assert(kTileBytesQ4K <= kTileBytes && kTileBytesQ6K <= kTileBytes, "ring slots hold one tile of any type");
static_assert(kTileBytesQ4K % 16 == 0 && kTileBytesQ6K % 16 == 0, "bulk copies need 16-byte multiples");

// F16 tiles: 32 rows x 256 columns of fp16, row-major (16384 bytes), so a
// row tile of K columns holds K / 256 of them.
constexpr int kTKH = 256;
constexpr int kTileBytesF16 = kTR * kTKH * 2;
static_assert(kTileBytesF16 <= kTileBytes && kTileBytesF16 % 16 == 0, "F16 tiles fit a ring slot");

// weight types of the tile engine (TGemv::wtype)
enum TWType : int { TW_Q8_0 = 0, TW_Q4_K = 1, TW_Q6_K = 2, TW_F16 = 3 };

__host__ __device__ constexpr int tile_bytes(int wtype) {
    return wtype == TW_Q4_K ? kTileBytesQ4K
                            : (wtype == TW_Q6_K ? kTileBytesQ6K : (wtype == TW_F16 ? kTileBytesF16 : kTileBytes));
}
// columns of one tile
__host__ __device__ constexpr int tile_cols(int wtype) { return wtype == TW_F16 ? kTKH : kTK; }

static_assert(kTileBytes % 16 == 0, "bulk copies need 16-byte multiples");
static_assert(kTRW == 4, "the row-tile reduction is written for 4 rows per warp");

enum GemvIn : int {
    IN_PLAIN = 0,    // activation = x
    IN_RMSNORM = 1,  // activation = (x * rsqrt(mean(x^2)+eps)) * norm_w
};
enum GemvEpi : int {
    EPI_STORE = 0,   // y[r] = W[r].x  (+ res[r] when res is given)
    EPI_SWIGLU = 1,  // rows interleaved (gate, up): y[i] = silu(W[2i].x) * W[2i+1].x
};

// One GEMV on a tiled Q8_0 matrix (plain data: lives in device op lists).
struct TGemv {
    const uint8_t *w;  // tiles
    int wtype;         // TWType
    int R, K;          // R % 32 == 0, K % 512 == 0
    const float *x;    // [M][ldx]
    int ldx, M, in_mode;
    const float *norm_w;
    float eps;
    int epi;
    float *y;  // [M][ldy]
    int ldy;
    const float *res;  // optional residual [M][ldres]
    int ldres;
    float *act_out;  // optional: CTA 0 stores the (normed) activation [M][K]
    // Tagged activations (persistent kernel): with LL_X / LL_RES / LL_Y set,
    // x / res / y are arrays of 8-byte (float value, uint32 tag) words, and a
    // value counts as written only when its tag equals x_tag / res_tag / y_tag
    // (see ll_pack); readers poll instead of waiting at a grid barrier.
    int ll;
    uint32_t x_tag, res_tag, y_tag;
};

enum : int { LL_X = 1, LL_RES = 2, LL_Y = 4 };

// ggml get_scale_min_k4: 12 bytes hold 8 six-bit scales and 8 six-bit mins
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// The 8 six-bit scales and mins of a Q4_K super-block header, one per byte,
// from its 12 packed bytes in words w0 = bytes 0..3, w1 = 4..7, w2 = 8..11
// (get_scale_min_k4 for all sub-blocks at once, in registers): scales of
// sub-blocks 0..3 / 4..7, mins of 0..3 / 4..7.
__device__ __forceinline__ void q4k_scales4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t &sc_lo, uint32_t &sc_hi,
                                            uint32_t &mn_lo, uint32_t &mn_hi) {
    sc_lo = w0 & 0x3f3f3f3fu;
    mn_lo = w1 & 0x3f3f3f3fu;
    sc_hi = (w2 & 0x0f0f0f0fu) | ((w0 >> 2) & 0x30303030u);
    mn_hi = ((w2 >> 4) & 0x0f0f0f0fu) | ((w1 >> 2) & 0x30303030u);
}

// Shared-memory layout of a Q8_K activation row: byte o of the row is stored
// at q8k_swz(o) (an XOR of 16-byte chunk bits inside each 512-byte block), so
// that the eight lanes of a quarter-warp, which read 16-byte chunks 128 or 256
// bytes apart in the K-quant consumers, hit all 32 banks.  Q4_K readers vary
// chunk bits 2..4 of (o >> 4) at fixed bits 0..1, Q6_K readers bits 0, 3, 4 at
// fixed bits 1..2; the swizzle maps either set onto bank-group bits 0..2.
__device__ __forceinline__ int q8k_swz(int o, int wtype) {
    return wtype == TW_Q6_K ? o ^ (((o >> 6) & 6) << 4) : o ^ (((o >> 7) & 3) << 4);
}

// Element (r, c) of a tiled matrix with K columns, dequantized as ggml's
// dequantize_row_q8_0 / _q4_K / _q6_K do (float products in the same order).
__device__ __forceinline__ float tq_elem(const uint8_t *w, int wtype, int K, long long r, int c) {
    if (wtype == TW_F16) {
        const uint8_t *t = w + ((size_t)(r / kTR) * (K / kTKH) + (size_t)(c / kTKH)) * kTileBytesF16;
        return __half2float(__ldg(reinterpret_cast<const __half *>(t) + (r % kTR) * kTKH + c % kTKH));
    }
    const uint8_t *t = w + ((size_t)(r / kTR) * (K / kTK) + (size_t)(c / kTK)) * tile_bytes(wtype);
    const int rl = (int)(r % kTR), cl = c % kTK;
    if (wtype == TW_Q4_K) {
        const int sb = cl >> 8, cc = cl & 255, j = cc >> 5;
        const uint8_t *hd = t + kQ4kHdr + (rl * 2 + sb) * 16;
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(hd)));
        const float dmin = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(hd + 2)));
        int sc, mn;
        q4k_scale_min(j, hd + 4, &sc, &mn);
        const uint8_t qb = t[(rl * 2 + sb) * 128 + ((cc >> 6) << 5) + (cc & 31)];
        const int q = (cc & 32) ? (qb >> 4) : (qb & 0xF);
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
    }
    if (wtype == TW_Q6_K) {
        const int sb = cl >> 8, cc = cl & 255, h = cc >> 7, k = (cc >> 5) & 3, l = cc & 31;
        const int rb = rl * 2 + sb;
        const uint8_t ql = t[rb * 128 + 64 * h + l + ((k & 1) << 5)];
        const uint8_t qh = t[kQ6kQh + rb * 64 + 32 * h + l];
        const int q = (((k & 2) ? (ql >> 4) : (ql & 0xF)) | (((qh >> (2 * k)) & 3) << 4)) - 32;
        const int8_t sc = (int8_t)t[kQ6kSc + rb * 16 + 8 * h + (l >> 4) + 2 * k];
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(t + kQ6kD + rb * 2)));
        return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
    const float q = (float)(int8_t)__ldg(t + rl * kTK + cl);
    const __half d = __ldg(reinterpret_cast<const __half *>(t + kTileQ) + rl * (kTK / 32) + cl / 32);
    return q * __half2float(d);
}

// Tile range [u0, u1) of CTA `cta` of G: whole row tiles.
__device__ __forceinline__ void tg_range(int R, int K, int wtype, int cta, int G, long long *u0, long long *u1) {
    const long long RT = R / kTR, NKT = K / tile_cols(wtype);
    *u0 = (RT * cta / G) * NKT;
    *u1 = (RT * (cta + 1) / G) * NKT;
}

// ---------------------------------------------------------------------------
// Prologue of the persistent kernel: one 8-value chunk per lane and pass.
// Chunk v of the [M][K] activation (elements 8v..8v+7 of row m, counting
// within the row) is owned by thread v % NT in pass v / (PC * NT); a warp
// loads 1 KB of contiguous activation with one 32-byte load per lane, and
// lanes 4k..4k+3 hold one 32-value Q8_0 block.  RMSNorm weights of a thread's
// chunks are loaded into registers by tg_norm_preload before the grid barrier
// (they do not depend on the previous op); an RMSNorm'd activation must fit
// one pass (M * K <= 8 * PC * NT, checked on the host).  Rounding to the
// nearest integer (ties to even) is done by adding 1.5 * 2^23, which leaves
// round(x) in the low mantissa bits for |x| < 2^22 -- the same rounding as
// ggml's nearest_int and _mm256_round_ps -- so no float-to-int conversion is
// issued per value.
// ---------------------------------------------------------------------------
struct F8 {
    float v[8];
};

__device__ __forceinline__ F8 ld_cg_f8(const float *p) {
    F8 r;
    asm volatile("ld.global.cg.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]), "=f"(r.v[4]), "=f"(r.v[5]), "=f"(r.v[6]),
                   "=f"(r.v[7])
                 : "l"(p));
    return r;
}

__device__ __forceinline__ F8 ld_nc_f8(const float *p) {
    F8 r;
    asm("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]), "=f"(r.v[4]), "=f"(r.v[5]), "=f"(r.v[6]),
          "=f"(r.v[7])
        : "l"(p));
    return r;
}

// Tagged activation words: low 32 bits the float value, high 32 bits the tag
// of the op that wrote it.  An aligned 8-byte store is single-copy atomic, so
// a reader that sees the expected tag sees the value written with it.
__device__ __forceinline__ uint64_t ll_pack(float v, uint32_t tag) {
    return ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
}

__device__ __forceinline__ void ll_store(void *base, size_t i, float v, uint32_t tag) {
    asm volatile("st.global.u64 [%0], %1;" ::"l"(reinterpret_cast<uint64_t *>(base) + i), "l"(ll_pack(v, tag))
                 : "memory");
}

// 8 tagged values at p (32-byte aligned); true when every tag equals `tag`.
__device__ __forceinline__ bool ll_load8(const void *p, uint32_t tag, F8 &out) {
    uint64_t w[8];
    const uint64_t *q = reinterpret_cast<const uint64_t *>(p);
    asm volatile("ld.global.cg.v4.u64 {%0,%1,%2,%3}, [%4];" : "=l"(w[0]), "=l"(w[1]), "=l"(w[2]), "=l"(w[3]) : "l"(q));
    asm volatile("ld.global.cg.v4.u64 {%0,%1,%2,%3}, [%4];" : "=l"(w[4]), "=l"(w[5]), "=l"(w[6]), "=l"(w[7]) : "l"(q + 4));
    bool ok = true;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        out.v[e] = __uint_as_float((uint32_t)w[e]);
        ok &= (uint32_t)(w[e] >> 32) == tag;
    }
    return ok;
}

// Polls 8 tagged values until their tags are current (bounded: sets
// ERR_GRID in *err and returns what it has when the producer never comes).
__device__ __forceinline__ F8 ll_wait8(const void *p, uint32_t tag, int *err) {
    F8 out;
    if (ll_load8(p, tag, out)) return out;
    const long long t0 = clock64(), lim = wait_limit(err);
    for (unsigned it = 1; !ll_load8(p, tag, out); ++it) {
        if (clock64() - t0 > lim ||
            (err && it % kErrPollEvery == 0 && (*reinterpret_cast<volatile int *>(err) & ERR_GRID))) {
            if (err) atomicOr(err, ERR_GRID);
            break;
        }
    }
    return out;
}

__device__ __forceinline__ float ll_wait1(const void *p, size_t i, uint32_t tag, int *err) {
    const uint64_t *q = reinterpret_cast<const uint64_t *>(p) + i;
    uint64_t w = __ldcg(reinterpret_cast<const unsigned long long *>(q));
    if ((uint32_t)(w >> 32) != tag) {
        const long long t0 = clock64(), lim = wait_limit(err);
        unsigned it = 0;
        do {
            if (clock64() - t0 > lim ||
                (err && ++it % kErrPollEvery == 0 && (*reinterpret_cast<volatile int *>(err) & ERR_GRID))) {
                if (err) atomicOr(err, ERR_GRID);
                break;
            }
            w = __ldcg(reinterpret_cast<const unsigned long long *>(q));
        } while ((uint32_t)(w >> 32) != tag);
    }
    return __uint_as_float((uint32_t)w);
}

__device__ __forceinline__ int tg_row_of(int v, int KC, int M) {
    int m = 0;
    while (m + 1 < M && v >= (m + 1) * KC) ++m;
    return m;
}

template <int PC, int NT>
__device__ __forceinline__ void tg_norm_preload(const TGemv &g, F8 (&nw)[PC]) {
    if (g.in_mode != IN_RMSNORM) return;
    const int KC = g.K >> 3, nv = g.M * KC, tid = threadIdx.x;
#pragma unroll
    for (int j = 0; j < PC; ++j) {
        const int v = tid + j * NT;
        if (v < nv) nw[j] = ld_nc_f8(g.norm_w + 8 * (v - tg_row_of(v, KC, g.M) * KC));
    }
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// round-half-even(x) for |x| < 2^22, low byte only
__device__ __forceinline__ uint32_t rne_byte(float x) {
    return (uint32_t)__float_as_int(__fadd_rn(x, 12582912.f));
}

__device__ __forceinline__ uint32_t pack4_rne(float a, float b, float c, float d, float id) {
    const uint32_t qa = rne_byte(__fmul_rn(a, id)), qb = rne_byte(__fmul_rn(b, id));
    const uint32_t qc = rne_byte(__fmul_rn(c, id)), qd = rne_byte(__fmul_rn(d, id));
    return __byte_perm(__byte_perm(qa, qb, 0x0040), __byte_perm(qc, qd, 0x0040), 0x5410);
}

// Q8_K quantization of the 256 values held by the 32 lanes of a warp (8 per
// lane, lane order = value order), ggml quantize_row_q8_K_ref: the value of
// largest magnitude (first one on ties) sets iscale = -127 / max,
// q = min(127, nearest_int(iscale * x)), d = 1 / iscale, bsums of 16 values.
__device__ __forceinline__ void quant_q8k_warp(const float (&y)[8], int lane, bool store, int8_t *xq8, float *d_out,
                                               int16_t *bs_out) {
    float ax = -1.f, mv = 0.f;
    int mi = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float a = fabsf(y[e]);
        if (a > ax) {
            ax = a;
            mv = y[e];
            mi = e;
        }
    }
    int gi = lane * 8 + mi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oax = __shfl_xor_sync(0xffffffffu, ax, o);
        const float omv = __shfl_xor_sync(0xffffffffu, mv, o);
        const int ogi = __shfl_xor_sync(0xffffffffu, gi, o);
        if (oax > ax || (oax == ax && ogi < gi)) {
            ax = oax;
            mv = omv;
            gi = ogi;
        }
    }
    uint32_t w0 = 0, w1 = 0;
    int qsum = 0;
    float d = 0.f;
    if (ax > 0.f) {
        const float iscale = __fdiv_rn(-127.f, mv);
        int q[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            q[e] = min(127, __float_as_int(__fadd_rn(__fmul_rn(iscale, y[e]), 12582912.f)) - 0x4B400000);
            qsum += q[e];
        }
        w0 = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
        w1 = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
        d = __fdiv_rn(1.0f, iscale);
    }
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
    if (!store) return;
    *reinterpret_cast<uint2 *>(xq8) = make_uint2(w0, w1);
    if ((lane & 1) == 0) bs_out[lane >> 1] = (int16_t)qsum;
    if (lane == 0) *d_out = d;
}

// Prologue of the tile engine.  Quantizes the [M][K] activation (after the
// RMSNorm of rms_norm_weighted, src/s2_model.cpp:46-55, when in_mode says so)
// into shared memory: Q8_0 for Q8_0 weights (xq int8 [M][K], xd [M][K/32]
// fp16-rounded scales), Q8_K for K-quant weights (xq, xd [M][K/256] float
// scales, xbs [M][K/16] block sums).  nw holds the norm weights of the
// thread's pass-0 chunks when the activation fits one pass (tg_norm_preload);
// otherwise they are loaded here.  tok [NT/32][tok_ld] is shared scratch.
// Q8ONLY: every weight of the caller is Q8_0, so only that quantizer is
// compiled in (a smaller prologue for the persistent kernel's Q8_0 build).
template <int MT, int NT, int PC, bool Q8ONLY = false>
__device__ __forceinline__ void tg_prologue8(const TGemv &g, const F8 (&nw)[PC], int8_t *xq, float *xd, int16_t *xbs,
                                             double *tok, int tok_ld, bool write_act, int bar_id,
                                             unsigned long long *ts = nullptr, int *err = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = g.K, KC = K >> 3, M = g.M, nv = M * KC;
    const bool rms = g.in_mode == IN_RMSNORM;
    const bool f16 = !Q8ONLY && g.wtype == TW_F16;
    const bool q8k = !Q8ONLY && g.wtype != TW_Q8_0 && !f16;
    const bool one_pass = nv <= PC * NT;
    float sc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sc[m] = 1.f;
    F8 xv[PC];
    int mrow[PC];
    const bool llx = (g.ll & LL_X) != 0;
    auto load_pass = [&](int base) {
        bool ready[PC];
#pragma unroll
        for (int j = 0; j < PC; ++j) {
            const int v = base + tid + j * NT;
            mrow[j] = 0;
            ready[j] = true;
            if (v < nv) {
                const int m = tg_row_of(v, KC, M);
                mrow[j] = m;
                const size_t off = (size_t)m * g.ldx + 8 * (v - m * KC);
                if (llx)
                    ready[j] = ll_load8(reinterpret_cast<const uint64_t *>(g.x) + off, g.x_tag, xv[j]);
                else
                    xv[j] = ld_cg_f8(g.x + off);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) xv[j].v[e] = 0.f;
            }
        }
        if (llx) {  // every load of the pass is in flight before the first retry
#pragma unroll
            for (int j = 0; j < PC; ++j)
                if (!ready[j]) {
                    const int v = base + tid + j * NT;
                    xv[j] = ll_wait8(reinterpret_cast<const uint64_t *>(g.x) + (size_t)mrow[j] * g.ldx +
                                         8 * (v - mrow[j] * KC),
                                     g.x_tag, err);
                }
        }
    };
    load_pass(0);
    if (rms) {
        double tk[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tk[m] = 0.0;
        if (one_pass) {
#pragma unroll
            for (int j = 0; j < PC; ++j)
                if (tid + j * NT < nv) {
                    double s = 0.0;
#pragma unroll
                    for (int e = 0; e < 8; ++e) s += (double)__fmul_rn(xv[j].v[e], xv[j].v[e]);
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        if (m == mrow[j]) tk[m] += s;
                }
        } else {
            for (int v = tid; v < nv; v += NT) {
                const int m = tg_row_of(v, KC, M);
                const size_t off = (size_t)m * g.ldx + 8 * (v - m * KC);
                const F8 x = llx ? ll_wait8(reinterpret_cast<const uint64_t *>(g.x) + off, g.x_tag, err)
                                 : ld_cg_f8(g.x + off);
                double s = 0.0;
#pragma unroll
                for (int e = 0; e < 8; ++e) s += (double)__fmul_rn(x.v[e], x.v[e]);
#pragma unroll
                for (int mm = 0; mm < MT; ++mm)
                    if (mm == m) tk[mm] += s;
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const double t = warp_sum_d(tk[m]);
            if (lane == 0) tok[warp * tok_ld + m] = t;
        }
        if (ts != nullptr && tid == 0) ts[0] = globaltimer_ns();
        named_sync(bar_id, NT);
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (m < M) {
                double tot = 0.0;
                for (int w = 0; w < NT / 32; ++w) tot += tok[w * tok_ld + m];
                const float mean = (float)(tot / (double)K);
                sc[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, g.eps)));
            }
        if (ts != nullptr && tid == 0) ts[1] = globaltimer_ns();
    }
    for (int base = 0; base < nv; base += PC * NT) {
        if (base > 0) load_pass(base);
#pragma unroll
        for (int j = 0; j < PC; ++j) {
            const int v = base + tid + j * NT;
            // 32-chunk warp groups are wholly in or out (nv % 32 == 0 for K % 256 == 0)
            if (base + warp * 32 + j * NT >= nv) continue;
            const bool valid = v < nv;
            F8 y = xv[j];
            if (rms && valid) {
                float s = sc[0];
#pragma unroll
                for (int m = 1; m < MT; ++m)
                    if (m == mrow[j]) s = sc[m];
                const F8 w = one_pass ? nw[j] : ld_nc_f8(g.norm_w + 8 * (v - mrow[j] * KC));
#pragma unroll
                for (int e = 0; e < 8; ++e) y.v[e] = __fmul_rn(__fmul_rn(y.v[e], s), w.v[e]);
            }
            if (valid && write_act && g.act_out != nullptr) {  // act_out is [M][K] contiguous
                float4 *dst = reinterpret_cast<float4 *>(g.act_out + 8 * (size_t)v);
                dst[0] = make_float4(y.v[0], y.v[1], y.v[2], y.v[3]);
                dst[1] = make_float4(y.v[4], y.v[5], y.v[6], y.v[7]);
            }
            if (f16) {  // the activation rounded to fp16 (ggml's vec_dot_type for F16 weights)
                if (valid) {
                    uint4 hv;
                    hv.x = pack_half2(y.v[0], y.v[1]);
                    hv.y = pack_half2(y.v[2], y.v[3]);
                    hv.z = pack_half2(y.v[4], y.v[5]);
                    hv.w = pack_half2(y.v[6], y.v[7]);
                    *reinterpret_cast<uint4 *>(xq + 16 * (size_t)v) = hv;
                }
                continue;
            }
            if (q8k) {
                quant_q8k_warp(y.v, lane, valid, xq + (size_t)mrow[j] * K + q8k_swz(8 * (v - mrow[j] * KC), g.wtype),
                               xd + (v >> 5), xbs + ((v >> 5) << 4));
                continue;
            }
            float amax = fabsf(y.v[0]);
#pragma unroll
            for (int e = 1; e < 8; ++e) amax = fmaxf(amax, fabsf(y.v[e]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            if (!valid) continue;
            const float id = amax != 0.0f ? __fdiv_rn(127.f, amax) : 0.0f;
            *reinterpret_cast<uint2 *>(xq + 8 * (size_t)v) =
                make_uint2(pack4_rne(y.v[0], y.v[1], y.v[2], y.v[3], id), pack4_rne(y.v[4], y.v[5], y.v[6], y.v[7], id));
            if ((lane & 3) == 0) xd[v >> 2] = __half2float(__float2half_rn(__fdiv_rn(amax, 127.f)));
        }
    }
    if (ts != nullptr && tid == 0) ts[3] = globaltimer_ns();
}

// Reduce a warp's 4 row partials (per token) across the 32 lanes with a
// transposing butterfly: after it, lane L holds the sum of row
// r = 2 * (L >> 4) + ((L >> 3) & 1), so lane 8r owns row r.  6 double
// shuffles per token instead of 20 for four separate butterflies.
__device__ __forceinline__ double reduce4_transpose(double a0, double a1, double a2, double a3, int lane) {
    const bool hi16 = lane & 16;
    // level xor 16: keep rows {0,1} (low half) or {2,3} (high half)
    const double s0 = hi16 ? a0 : a2, s1 = hi16 ? a1 : a3;  // the pair this lane gives away
    const double k0 = hi16 ? a2 : a0, k1 = hi16 ? a3 : a1;  // the pair it keeps
    const double b0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 16);
    const double b1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 16);
    // level xor 8: keep the first (bit 3 clear) or second row of the pair
    const bool hi8 = lane & 8;
    double v = (hi8 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, hi8 ? b0 : b1, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v;
}

// Epilogue of row tile rt for warp `warp`: tot[m] is this lane's reduced sum
// of row r(lane) (see reduce4_transpose).  EPI_STORE: lane 8r stores row r
// (+ the residual resv[m] it prefetched); EPI_SWIGLU: lane 16p stores output
// pair p = silu(gate row 2p) * (up row 2p+1, fetched from lane 16p + 8).
template <int MT>
__device__ __forceinline__ void tg_emit(const TGemv &g, int rt, int warp, int lane, const double (&tot)[MT],
                                        const float (&resv)[MT]) {
    const int row0 = rt * kTR + warp * kTRW;
    if (g.epi == EPI_SWIGLU) {
        double up[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) up[m] = __shfl_down_sync(0xffffffffu, tot[m], 8);
        if ((lane & 15) == 0) {
            const int p = lane >> 4;
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < g.M)
                {
                    const float val = __fmul_rn(silu((float)tot[m]), (float)up[m]);
                    const size_t yi = (size_t)m * g.ldy + row0 / 2 + p;
                    if (g.ll & LL_Y)
                        ll_store(g.y, yi, val, g.y_tag);
                    else
                        g.y[yi] = val;
                }
        }
    } else if ((lane & 7) == 0) {
        const int r = 2 * (lane >> 4) + ((lane >> 3) & 1);
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (m < g.M) {
                const float val = (float)tot[m];
                const float outv = g.res ? __fadd_rn(resv[m], val) : val;
                const size_t yi = (size_t)m * g.ldy + row0 + r;
                if (g.ll & LL_Y)
                    ll_store(g.y, yi, outv, g.y_tag);
                else
                    g.y[yi] = outv;
            }
    }
}

// Consumer (the kTNC consumer threads): this CTA's row tiles of one GEMV,
// after the prologue filled xq / xd.  The ring position (slot, phase) is
// carried across ops by the caller.
template <int MT>
__device__ __forceinline__ void tg_consume(const TGemv &g, const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                           int nst, int &slot, uint32_t &phase, const int8_t *xq, const float *xd,
                                           int cta, int G, int *err, unsigned long long *t_first = nullptr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = g.K, NKT = K / kTK, NB = K >> 5, M = g.M;
    const int RT = g.R / kTR;
    const int rt0 = (int)((long long)RT * cta / G), rt1 = (int)((long long)RT * (cta + 1) / G);
    const int rbase = warp * kTRW;
    // lane 8r reads / writes row r of the warp's four (see reduce4_transpose)
    const int my_row = 2 * (lane >> 4) + ((lane >> 3) & 1);
    for (int rt = rt0; rt < rt1; ++rt) {
        double acc[kTRW][MT];
#pragma unroll
        for (int i = 0; i < kTRW; ++i)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[i][m] = 0.0;
        float resv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) resv[m] = 0.f;
        if (g.res != nullptr && (lane & 7) == 0) {
            // residual of this lane's output row, needed at the row tile's end
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) {
                    const size_t ri = (size_t)m * g.ldres + (size_t)rt * kTR + rbase + my_row;
                    resv[m] = (g.ll & LL_RES) ? ll_wait1(g.res, ri, g.res_tag, err) : __ldcg(g.res + ri);
                }
        }
        const int8_t *xql = xq + lane * 16;
        const float *xdl = xd + (lane >> 1);
        for (int kt = 0; kt < NKT; ++kt) {
            // this lane's activation chunk of K-tile kt, per token
            int4 xa[MT];
            float xs[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int mm = m < M ? m : 0;
                xa[m] = *reinterpret_cast<const int4 *>(xql + (size_t)mm * K + kt * kTK);
                xs[m] = xdl[mm * NB + kt * (kTK / 32)];
            }
            mbar_wait(&full[slot], phase, err, ERR_WAIT_FULL);
            if (t_first != nullptr && tid == 0 && rt == rt0 && kt == 0) *t_first = globaltimer_ns();
            const uint8_t *t = ring + (size_t)slot * kTileBytes;
            int4 wv[kTRW];
            float dw[kTRW];
#pragma unroll
            for (int i = 0; i < kTRW; ++i) {
                wv[i] = *reinterpret_cast<const int4 *>(t + (rbase + i) * kTK + lane * 16);
                dw[i] = __half2float(
                    reinterpret_cast<const __half *>(t + kTileQ)[(rbase + i) * (kTK / 32) + (lane >> 1)]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // data is in registers: the slot may refill
            if (++slot == nst) {
                slot = 0;
                phase ^= 1u;
            }
#pragma unroll
            for (int i = 0; i < kTRW; ++i)
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < M) {
                        int sh = dp4a(wv[i].x, xa[m].x, 0);
                        sh = dp4a(wv[i].y, xa[m].y, sh);
                        sh = dp4a(wv[i].z, xa[m].z, sh);
                        sh = dp4a(wv[i].w, xa[m].w, sh);
                        acc[i][m] += (double)sh * (double)__fmul_rn(dw[i], xs[m]);
                    }
        }
        double tot[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tot[m] = reduce4_transpose(acc[0][m], acc[1][m], acc[2][m], acc[3][m], lane);
        tg_emit<MT>(g, rt, warp, lane, tot, resv);
    }
}

// ---------------------------------------------------------------------------
// K-quant consumers (Q8_K activation: xq int8 [M][K] in the q8k_swz layout,
// xd [M][K/256] scales, xbs [M][K/16] block sums).  Lane mapping per warp:
// row r = lane / 8 of the warp's four rows (lane 8r holds row r after the
// reduction, as tg_emit expects), s = lane % 8 picks super-block sb = s / 4 of
// the K-tile and a quarter of its values.  Per super-block the integer sums
// are exact and the block term is formed as ggml's vec_dot_q4_K_q8_K /
// vec_dot_q6_K_q8_K scale it (d_w * d_x in float), then the terms are summed
// in double.  Shared-memory reads are bank-conflict free: the activation by
// its swizzle, the weight tile's two 16-byte halves of a lane by reading them
// in an order that depends on sb.
// ---------------------------------------------------------------------------
template <int MT>
__device__ __forceinline__ void tg_consume_q4k(const TGemv &g, const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                               int nst, int &slot, uint32_t &phase, const int8_t *xq,
                                               const float *xd, const int16_t *xbs, int cta, int G, int *err,
                                               unsigned long long *t_first = nullptr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = g.K, NKT = K / kTK, M = g.M, NSB = K >> 8;
    const int RT = g.R / kTR;
    const int rt0 = (int)((long long)RT * cta / G), rt1 = (int)((long long)RT * (cta + 1) / G);
    const int r = lane >> 3, s = lane & 7, sb = s >> 2, c = s & 3;
    const int row_in_tile = warp * kTRW + r;
    const int sh16 = (c & 1) * 16;  // sub-blocks 2c, 2c+1: bytes 2(c&1), 2(c&1)+1 of the lo (c < 2) / hi scale words
    const int wo0 = sb * 16, wo1 = wo0 ^ 16;  // the two 16-byte quant halves, read in sb order (bank spread)
    for (int rt = rt0; rt < rt1; ++rt) {
        double acc[MT];
        float resv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            acc[m] = 0.0;
            resv[m] = 0.f;
        }
        if (g.res != nullptr && s == 0) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) {
                    const size_t ri = (size_t)m * g.ldres + (size_t)rt * kTR + row_in_tile;
                    resv[m] = (g.ll & LL_RES) ? ll_wait1(g.res, ri, g.res_tag, err) : __ldcg(g.res + ri);
                }
        }
        for (int kt = 0; kt < NKT; ++kt) {
            const int sbg = kt * 2 + sb;  // super-block of the row
            int4 xa[MT][4];
            uint2 bsv[MT];
            float dx[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int mm = m < M ? m : 0;
                const int8_t *xr = xq + (size_t)mm * K;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    xa[m][i] = *reinterpret_cast<const int4 *>(xr + q8k_swz(sbg * 256 + 64 * c + 16 * i, TW_Q4_K));
                bsv[m] = *reinterpret_cast<const uint2 *>(xbs + (size_t)mm * (K >> 4) + sbg * 16 + 4 * c);
                dx[m] = xd[mm * NSB + sbg];
            }
            mbar_wait(&full[slot], phase, err, ERR_WAIT_FULL);
            if (t_first != nullptr && tid == 0 && rt == rt0 && kt == 0) *t_first = globaltimer_ns();
            const uint8_t *t = ring + (size_t)slot * kTileBytes;
            const uint8_t *qb = t + (row_in_tile * 2 + sb) * 128 + 32 * c;
            const int4 qa = *reinterpret_cast<const int4 *>(qb + wo0);
            const int4 qc = *reinterpret_cast<const int4 *>(qb + wo1);
            const int4 hd = *reinterpret_cast<const int4 *>(t + kQ4kHdr + (row_in_tile * 2 + sb) * 16);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == nst) {
                slot = 0;
                phase ^= 1u;
            }
            const int4 q0 = sb ? qc : qa, q1 = sb ? qa : qc;
            uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
            q4k_scales4((uint32_t)hd.y, (uint32_t)hd.z, (uint32_t)hd.w, sc_lo, sc_hi, mn_lo, mn_hi);
            const uint32_t scw = ((c & 2) ? sc_hi : sc_lo) >> sh16, mnw = ((c & 2) ? mn_hi : mn_lo) >> sh16;
            const int sc0 = scw & 0xff, sc1 = (scw >> 8) & 0xff, mn0 = mnw & 0xff, mn1 = (mnw >> 8) & 0xff;
            const float dw = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffff)));
            const float dmw = __half2float(__ushort_as_half((unsigned short)((unsigned)hd.x >> 16)));
            const int qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) {
                    const int xw[16] = {xa[m][0].x, xa[m][0].y, xa[m][0].z, xa[m][0].w, xa[m][1].x, xa[m][1].y,
                                        xa[m][1].z, xa[m][1].w, xa[m][2].x, xa[m][2].y, xa[m][2].z, xa[m][2].w,
                                        xa[m][3].x, xa[m][3].y, xa[m][3].z, xa[m][3].w};
                    int slo = 0, shi = 0;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        slo = dp4a(qw[i] & 0x0F0F0F0F, xw[i], slo);
                        shi = dp4a((qw[i] >> 4) & 0x0F0F0F0F, xw[8 + i], shi);
                    }
                    const int b0 = (int)(short)(bsv[m].x & 0xffff), b1 = (int)(short)(bsv[m].x >> 16);
                    const int b2 = (int)(short)(bsv[m].y & 0xffff), b3 = (int)(short)(bsv[m].y >> 16);
                    int isum = sc0 * slo + sc1 * shi;
                    int msum = mn0 * (b0 + b1) + mn1 * (b2 + b3);
                    isum += __shfl_xor_sync(0xffffffffu, isum, 1);
                    isum += __shfl_xor_sync(0xffffffffu, isum, 2);
                    msum += __shfl_xor_sync(0xffffffffu, msum, 1);
                    msum += __shfl_xor_sync(0xffffffffu, msum, 2);
                    if (c == 0) {
                        const double d = (double)__fmul_rn(dw, dx[m]), dmn = (double)__fmul_rn(dmw, dx[m]);
                        acc[m] += fma(d, (double)isum, -(dmn * (double)msum));
                    }
                }
        }
        double tot[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tot[m] = acc[m] + __shfl_xor_sync(0xffffffffu, acc[m], 4);
        tg_emit<MT>(g, rt, warp, lane, tot, resv);
    }
}

template <int MT>
__device__ __forceinline__ void tg_consume_q6k(const TGemv &g, const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                               int nst, int &slot, uint32_t &phase, const int8_t *xq,
                                               const float *xd, int cta, int G, int *err,
                                               unsigned long long *t_first = nullptr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = g.K, NKT = K / kTK, M = g.M, NSB = K >> 8;
    const int RT = g.R / kTR;
    const int rt0 = (int)((long long)RT * cta / G), rt1 = (int)((long long)RT * (cta + 1) / G);
    const int r = lane >> 3, s = lane & 7, sb = s >> 2, h = (s >> 1) & 1, is = s & 1;
    const int row_in_tile = warp * kTRW + r;
    const int rb = row_in_tile * 2 + sb;
    const int ao0 = sb * 32, ao1 = ao0 ^ 32;  // ql halves A (+0) and B (+32), read in sb order (bank spread)
    for (int rt = rt0; rt < rt1; ++rt) {
        double acc[MT];
        float resv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            acc[m] = 0.0;
            resv[m] = 0.f;
        }
        if (g.res != nullptr && s == 0) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) {
                    const size_t ri = (size_t)m * g.ldres + (size_t)rt * kTR + row_in_tile;
                    resv[m] = (g.ll & LL_RES) ? ll_wait1(g.res, ri, g.res_tag, err) : __ldcg(g.res + ri);
                }
        }
        for (int kt = 0; kt < NKT; ++kt) {
            const int sbg = kt * 2 + sb;
            int4 xa[MT][4];  // values 128h + 32k + 16is .. +16, k = 0..3
            float dx[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int mm = m < M ? m : 0;
                const int8_t *xr = xq + (size_t)mm * K;
                const int o = sbg * 256 + 128 * h + 16 * is;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    xa[m][k] = *reinterpret_cast<const int4 *>(xr + q8k_swz(o + 32 * k, TW_Q6_K));
                dx[m] = xd[mm * NSB + sbg];
            }
            mbar_wait(&full[slot], phase, err, ERR_WAIT_FULL);
            if (t_first != nullptr && tid == 0 && rt == rt0 && kt == 0) *t_first = globaltimer_ns();
            const uint8_t *t = ring + (size_t)slot * kTileBytes;
            const uint8_t *qlb = t + rb * 128 + 64 * h + 16 * is;
            const int4 P0 = *reinterpret_cast<const int4 *>(qlb + ao0);
            const int4 P1 = *reinterpret_cast<const int4 *>(qlb + ao1);
            const int4 Q = *reinterpret_cast<const int4 *>(t + kQ6kQh + rb * 64 + 32 * h + 16 * is);
            const int8_t *scp = reinterpret_cast<const int8_t *>(t + kQ6kSc + rb * 16 + 8 * h + is);
            const int sc0 = scp[0], sc1 = scp[2], sc2 = scp[4], sc3 = scp[6];
            const float dw = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(t + kQ6kD + rb * 2)));
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == nst) {
                slot = 0;
                phase ^= 1u;
            }
            const int4 A = sb ? P1 : P0, B = sb ? P0 : P1;
            const int aw[4] = {A.x, A.y, A.z, A.w}, bw[4] = {B.x, B.y, B.z, B.w}, qw[4] = {Q.x, Q.y, Q.z, Q.w};
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) {
                    const int x0[4] = {xa[m][0].x, xa[m][0].y, xa[m][0].z, xa[m][0].w};
                    const int x1[4] = {xa[m][1].x, xa[m][1].y, xa[m][1].z, xa[m][1].w};
                    const int x2[4] = {xa[m][2].x, xa[m][2].y, xa[m][2].z, xa[m][2].w};
                    const int x3[4] = {xa[m][3].x, xa[m][3].y, xa[m][3].z, xa[m][3].w};
                    int s1 = 0, s2 = 0, s3 = 0, s4 = 0;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const unsigned a = (unsigned)aw[i], b = (unsigned)bw[i], q = (unsigned)qw[i];
                        const unsigned v1 = __vsub4((a & 0x0F0F0F0Fu) | ((q & 0x03030303u) << 4), 0x20202020u);
                        const unsigned v2 = __vsub4((b & 0x0F0F0F0Fu) | (((q >> 2) & 0x03030303u) << 4), 0x20202020u);
                        const unsigned v3 = __vsub4(((a >> 4) & 0x0F0F0F0Fu) | (((q >> 4) & 0x03030303u) << 4), 0x20202020u);
                        const unsigned v4 = __vsub4(((b >> 4) & 0x0F0F0F0Fu) | (((q >> 6) & 0x03030303u) << 4), 0x20202020u);
                        s1 = dp4a((int)v1, x0[i], s1);
                        s2 = dp4a((int)v2, x1[i], s2);
                        s3 = dp4a((int)v3, x2[i], s3);
                        s4 = dp4a((int)v4, x3[i], s4);
                    }
                    int isum = sc0 * s1 + sc1 * s2 + sc2 * s3 + sc3 * s4;
                    isum += __shfl_xor_sync(0xffffffffu, isum, 1);
                    isum += __shfl_xor_sync(0xffffffffu, isum, 2);
                    if ((s & 3) == 0) acc[m] += (double)__fmul_rn(dw, dx[m]) * (double)isum;
                }
        }
        double tot[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tot[m] = acc[m] + __shfl_xor_sync(0xffffffffu, acc[m], 4);
        tg_emit<MT>(g, rt, warp, lane, tot, resv);
    }
}

// ---------------------------------------------------------------------------
// F16 consumer (xq holds the fp16-rounded activation, [M][K] halves).  Lane l
// owns columns 8l..8l+7 of each 256-column tile.  fp16 values become doubles
// exactly with integer moves: the sign and the 15 magnitude bits shifted into
// the double's sign / exponent / mantissa fields give the value times 2^-1008
// (normals and subnormals alike), and one multiply by 2^1008 restores it.  A
// product of two fp16 values is exact in double, so fma(w, x, acc) adds the
// exact product (ggml_vec_dot_f16's terms) and rows are rounded to float once.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void h2_to_d(uint32_t u, double &lo, double &hi) {
    // magnitude bits 0..14 of a half -> bits 10..24 of the double's high word
    const uint32_t l = ((u << 16) & 0x80000000u) | ((u << 10) & 0x01FFFC00u);
    const uint32_t h = (u & 0x80000000u) | ((u >> 6) & 0x01FFFC00u);
    constexpr double k2p1008 = 0x1p1008;
    lo = __hiloint2double((int)l, 0) * k2p1008;
    hi = __hiloint2double((int)h, 0) * k2p1008;
}

template <int MT>
__device__ __forceinline__ void tg_consume_f16(const TGemv &g, const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                               int nst, int &slot, uint32_t &phase, const int8_t *xq, int cta, int G,
                                               int *err, unsigned long long *t_first = nullptr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = g.K, NKT = K / kTKH, M = g.M;
    const int RT = g.R / kTR;
    const int rt0 = (int)((long long)RT * cta / G), rt1 = (int)((long long)RT * (cta + 1) / G);
    const int rbase = warp * kTRW;
    const int my_row = 2 * (lane >> 4) + ((lane >> 3) & 1);
    const __half *xh = reinterpret_cast<const __half *>(xq);
    for (int rt = rt0; rt < rt1; ++rt) {
        double acc[kTRW][MT];
#pragma unroll
        for (int i = 0; i < kTRW; ++i)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[i][m] = 0.0;
        float resv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) resv[m] = 0.f;
        if (g.res != nullptr && (lane & 7) == 0) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) {
                    const size_t ri = (size_t)m * g.ldres + (size_t)rt * kTR + rbase + my_row;
                    resv[m] = (g.ll & LL_RES) ? ll_wait1(g.res, ri, g.res_tag, err) : __ldcg(g.res + ri);
                }
        }
        for (int kt = 0; kt < NKT; ++kt) {
            double xv[MT][8];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int mm = m < M ? m : 0;
                const uint4 a = *reinterpret_cast<const uint4 *>(xh + (size_t)mm * K + kt * kTKH + lane * 8);
                h2_to_d(a.x, xv[m][0], xv[m][1]);
                h2_to_d(a.y, xv[m][2], xv[m][3]);
                h2_to_d(a.z, xv[m][4], xv[m][5]);
                h2_to_d(a.w, xv[m][6], xv[m][7]);
            }
            mbar_wait(&full[slot], phase, err, ERR_WAIT_FULL);
            if (t_first != nullptr && tid == 0 && rt == rt0 && kt == 0) *t_first = globaltimer_ns();
            const uint8_t *t = ring + (size_t)slot * kTileBytes;
            uint4 wv[kTRW];
#pragma unroll
            for (int i = 0; i < kTRW; ++i)
                wv[i] = *reinterpret_cast<const uint4 *>(t + ((rbase + i) * kTKH + lane * 8) * 2);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == nst) {
                slot = 0;
                phase ^= 1u;
            }
#pragma unroll
            for (int i = 0; i < kTRW; ++i) {
                double w[8];
                h2_to_d(wv[i].x, w[0], w[1]);
                h2_to_d(wv[i].y, w[2], w[3]);
                h2_to_d(wv[i].z, w[4], w[5]);
                h2_to_d(wv[i].w, w[6], w[7]);
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < M)
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[i][m] = fma(w[e], xv[m][e], acc[i][m]);
            }
        }
        double tot[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tot[m] = reduce4_transpose(acc[0][m], acc[1][m], acc[2][m], acc[3][m], lane);
        tg_emit<MT>(g, rt, warp, lane, tot, resv);
    }
}

// The consumer of the op's weight type.
template <int MT>
__device__ __forceinline__ void tg_consume_any(const TGemv &g, const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                               int nst, int &slot, uint32_t &phase, const int8_t *xq,
                                               const float *xd, const int16_t *xbs, int cta, int G, int *err,
                                               unsigned long long *t_first = nullptr) {
    if constexpr (MT <= 4) {  // (F16 calls carry at most 4 tokens)
        if (g.wtype == TW_F16) {
            tg_consume_f16<MT>(g, ring, full, empty, nst, slot, phase, xq, cta, G, err, t_first);
            return;
        }
    }
    if (g.wtype == TW_Q4_K)
        tg_consume_q4k<MT>(g, ring, full, empty, nst, slot, phase, xq, xd, xbs, cta, G, err, t_first);
    else if (g.wtype == TW_Q6_K)
        tg_consume_q6k<MT>(g, ring, full, empty, nst, slot, phase, xq, xd, cta, G, err, t_first);
    else
        tg_consume<MT>(g, ring, full, empty, nst, slot, phase, xq, xd, cta, G, err, t_first);
}

// Host-side check of a GEMV for the tiled kernels.
inline bool tg_shape_ok(int R, int K, int M, int in_mode, int epi, bool has_res, int max_k, int max_m) {
    if (R <= 0 || R % kTR != 0 || K <= 0 || K % kTK != 0 || K > max_k || M < 1 || M > max_m) return false;
    if (in_mode == IN_RMSNORM && K > kNormMax) return false;
    if (epi == EPI_SWIGLU && has_res) return false;
    return true;
}

}  // namespace s2k
