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
};

// Element (r, c) of a tiled Q8_0 matrix with K columns, dequantized as ggml
// does (q * d in float).
__device__ __forceinline__ float tq_elem(const uint8_t *w, int K, long long r, int c) {
    const uint8_t *t = w + ((size_t)(r / kTR) * (K / kTK) + (size_t)(c / kTK)) * kTileBytes;
    const int rl = (int)(r % kTR), cl = c % kTK;
    const float q = (float)(int8_t)__ldg(t + rl * kTK + cl);
    const __half d = __ldg(reinterpret_cast<const __half *>(t + kTileQ) + rl * (kTK / 32) + cl / 32);
    return q * __half2float(d);
}

// Tile range [u0, u1) of CTA `cta` of G: whole row tiles.
__device__ __forceinline__ void tg_range(int R, int K, int cta, int G, long long *u0, long long *u1) {
    const long long RT = R / kTR, NKT = K / kTK;
    *u0 = (RT * cta / G) * NKT;
    *u1 = (RT * (cta + 1) / G) * NKT;
}

// One 8-value chunk of an activation row: chunk c of token m covers columns
// 8*c' .. 8*c'+7 with c' = c % (K/8).  Four consecutive lanes hold the four
// chunks of one 32-value Q8_0 block.
struct Chunk8 {
    float4 a, b;
};

__device__ __forceinline__ double sumsq8(const Chunk8 &c) {
    return (double)__fmul_rn(c.a.x, c.a.x) + (double)__fmul_rn(c.a.y, c.a.y) + (double)__fmul_rn(c.a.z, c.a.z) +
           (double)__fmul_rn(c.a.w, c.a.w) + (double)__fmul_rn(c.b.x, c.b.x) + (double)__fmul_rn(c.b.y, c.b.y) +
           (double)__fmul_rn(c.b.z, c.b.z) + (double)__fmul_rn(c.b.w, c.b.w);
}

__device__ __forceinline__ float4 mul4(float4 v, float sc, float4 w) {
    return make_float4(__fmul_rn(__fmul_rn(v.x, sc), w.x), __fmul_rn(__fmul_rn(v.y, sc), w.y),
                       __fmul_rn(__fmul_rn(v.z, sc), w.z), __fmul_rn(__fmul_rn(v.w, sc), w.w));
}

__device__ __forceinline__ int pack4(float4 v, float id) {
    const int q0 = __float2int_rn(__fmul_rn(v.x, id)), q1 = __float2int_rn(__fmul_rn(v.y, id));
    const int q2 = __float2int_rn(__fmul_rn(v.z, id)), q3 = __float2int_rn(__fmul_rn(v.w, id));
    return (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
}

// Quantize the chunk this lane holds (ggml x86 quantize_row_q8_0 on its
// 32-value block: d = amax/127 stored fp16, q = round-half-even(x * 127/amax));
// all 32 lanes must call it, valid = this lane holds a chunk.
__device__ __forceinline__ void quant_chunk(const Chunk8 &c, bool valid, int8_t *xq_chunk, float *xd_blk,
                                            bool first_of_block) {
    float amax = fmaxf(fmaxf(fmaxf(fabsf(c.a.x), fabsf(c.a.y)), fmaxf(fabsf(c.a.z), fabsf(c.a.w))),
                       fmaxf(fmaxf(fabsf(c.b.x), fabsf(c.b.y)), fmaxf(fabsf(c.b.z), fabsf(c.b.w))));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    if (!valid) return;
    const float d = __fdiv_rn(amax, 127.f);
    const float id = amax != 0.0f ? __fdiv_rn(127.f, amax) : 0.0f;
    *reinterpret_cast<int2 *>(xq_chunk) = make_int2(pack4(c.a, id), pack4(c.b, id));
    if (first_of_block) *xd_blk = __half2float(__float2half_rn(d));
}

// Prologue (all NT consumer threads): activation rows -> Q8_0 blocks in shared
// memory (xq [M][K] int8, xd [M][K/32] fp16-rounded scales as float), with the
// RMSNorm of rms_norm_weighted (src/s2_model.cpp:46-55) when in_mode says so.
// nws [kNormMax] receives the norm weights; tok [NT/32][tok_ld] (tok_ld >= MT)
// is small shared scratch.  write_act: this CTA stores act_out (exactly one
// CTA of the grid should).  The caller synchronizes the consumer threads after
// it returns.
// Thread t owns 8-value chunks t, t + NT, ... (CPT of them per pass, all loads
// of a pass issued before any is used), so the whole CTA quantizes in
// parallel and a pass costs one L2 round trip.  Every thread derives the
// RMSNorm scale itself from the per-warp partial sums.
template <int MT, int NT>
__device__ __forceinline__ void tg_prologue(const TGemv &g, int8_t *xq, float *xd, float *nws, double *tok,
                                            int tok_ld, float * /*unused*/, bool write_act, int bar_id,
                                            unsigned long long *ts = nullptr) {
    constexpr int CPT = 5;  // chunks per thread per pass
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = g.K, KC = K >> 3, M = g.M;
    const int nchunks = M * KC;
    const bool rms = g.in_mode == IN_RMSNORM;
    const bool resident = nchunks <= CPT * NT;  // all chunks of the op in registers in one pass
    Chunk8 c[CPT];
    float sc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sc[m] = 1.f;
    if (resident) {
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ci = tid + j * NT;
            if (ci < nchunks) {
                const int m = ci / KC, off = (ci - m * KC) * 8;
                const float4 *src = reinterpret_cast<const float4 *>(g.x + (size_t)m * g.ldx + off);
                c[j].a = __ldcg(src);
                c[j].b = __ldcg(src + 1);
            }
        }
    }
    if (rms) {
        for (int i = tid; i < K / 4; i += NT)
            reinterpret_cast<float4 *>(nws)[i] = __ldg(reinterpret_cast<const float4 *>(g.norm_w) + i);
        double tk[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tk[m] = 0.0;
        if (resident) {
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int ci = tid + j * NT;
                if (ci < nchunks) {
                    const double s = sumsq8(c[j]);
                    const int m = ci / KC;
#pragma unroll
                    for (int mm = 0; mm < MT; ++mm)
                        if (mm == m) tk[mm] += s;
                }
            }
        } else {
            for (int ci = tid; ci < nchunks; ci += NT) {
                const int m = ci / KC, off = (ci - m * KC) * 8;
                const float4 *src = reinterpret_cast<const float4 *>(g.x + (size_t)m * g.ldx + off);
                Chunk8 t;
                t.a = __ldcg(src);
                t.b = __ldcg(src + 1);
                const double s = sumsq8(t);
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
        named_sync(bar_id, NT);  // per-warp sums and norm weights complete
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
    auto finish = [&](Chunk8 &ch, int ci, bool valid) {
        const int m = valid ? ci / KC : 0, off = valid ? (ci - m * KC) * 8 : 0;
        if (valid && rms) {
            float s = sc[0];
#pragma unroll
            for (int mm = 1; mm < MT; ++mm)
                if (mm == m) s = sc[mm];
            const float4 *nw = reinterpret_cast<const float4 *>(nws + off);
            ch.a = mul4(ch.a, s, nw[0]);
            ch.b = mul4(ch.b, s, nw[1]);
        }
        if (valid && g.act_out != nullptr && write_act) {
            float4 *dst = reinterpret_cast<float4 *>(g.act_out + (size_t)m * K + off);
            dst[0] = ch.a;
            dst[1] = ch.b;
        }
        quant_chunk(ch, valid, xq + (size_t)m * K + off, xd + m * (K >> 5) + (off >> 5), (off & 31) == 0);
    };
    if (resident) {
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int ci = tid + j * NT;
            if (j * NT < nchunks) finish(c[j], ci, ci < nchunks);  // warp-uniform guard: all lanes shuffle
        }
    } else {
        for (int base = 0; base < nchunks; base += NT) {
            const int ci = base + tid;
            Chunk8 t;
            t.a = t.b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ci < nchunks) {
                const int m = ci / KC, off = (ci - m * KC) * 8;
                const float4 *src = reinterpret_cast<const float4 *>(g.x + (size_t)m * g.ldx + off);
                t.a = __ldcg(src);
                t.b = __ldcg(src + 1);
            }
            finish(t, ci, ci < nchunks);
        }
    }
    if (ts != nullptr && tid == 0) ts[3] = globaltimer_ns();
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

// round-half-even(x) for |x| < 2^22, low byte only
__device__ __forceinline__ uint32_t rne_byte(float x) {
    return (uint32_t)__float_as_int(__fadd_rn(x, 12582912.f));
}

__device__ __forceinline__ uint32_t pack4_rne(float a, float b, float c, float d, float id) {
    const uint32_t qa = rne_byte(__fmul_rn(a, id)), qb = rne_byte(__fmul_rn(b, id));
    const uint32_t qc = rne_byte(__fmul_rn(c, id)), qd = rne_byte(__fmul_rn(d, id));
    return __byte_perm(__byte_perm(qa, qb, 0x0040), __byte_perm(qc, qd, 0x0040), 0x5410);
}

template <int MT, int NT, int PC>
__device__ __forceinline__ void tg_prologue8(const TGemv &g, const F8 (&nw)[PC], int8_t *xq, float *xd, double *tok,
                                             int tok_ld, bool write_act, int bar_id,
                                             unsigned long long *ts = nullptr) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = g.K, KC = K >> 3, M = g.M, nv = M * KC;
    const bool rms = g.in_mode == IN_RMSNORM;
    float sc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sc[m] = 1.f;
    for (int base = 0; base < nv; base += PC * NT) {
        F8 xv[PC];
        int mrow[PC];
#pragma unroll
        for (int j = 0; j < PC; ++j) {
            const int v = base + tid + j * NT;
            mrow[j] = 0;
            if (v < nv) {
                const int m = tg_row_of(v, KC, M);
                mrow[j] = m;
                xv[j] = ld_cg_f8(g.x + (size_t)m * g.ldx + 8 * (v - m * KC));
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) xv[j].v[e] = 0.f;
            }
        }
        if (rms) {  // single pass (host check): every element of every row is in xv
            double tk[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) tk[m] = 0.0;
#pragma unroll
            for (int j = 0; j < PC; ++j)
                if (base + tid + j * NT < nv) {
                    double s = 0.0;
#pragma unroll
                    for (int e = 0; e < 8; ++e) s += (double)__fmul_rn(xv[j].v[e], xv[j].v[e]);
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        if (m == mrow[j]) tk[m] += s;
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
#pragma unroll
        for (int j = 0; j < PC; ++j) {
            const int v = base + tid + j * NT;
            // 4-lane groups are wholly in or out (nv % 4 == 0): all lanes of a live warp shuffle
            if (base + warp * 32 + j * NT >= nv) continue;
            const bool valid = v < nv;
            F8 y = xv[j];
            if (rms && valid) {
                float s = sc[0];
#pragma unroll
                for (int m = 1; m < MT; ++m)
                    if (m == mrow[j]) s = sc[m];
#pragma unroll
                for (int e = 0; e < 8; ++e) y.v[e] = __fmul_rn(__fmul_rn(y.v[e], s), nw[j].v[e]);
            }
            if (valid && write_act && g.act_out != nullptr) {  // act_out is [M][K] contiguous
                float4 *dst = reinterpret_cast<float4 *>(g.act_out + 8 * (size_t)v);
                dst[0] = make_float4(y.v[0], y.v[1], y.v[2], y.v[3]);
                dst[1] = make_float4(y.v[4], y.v[5], y.v[6], y.v[7]);
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
                    g.y[(size_t)m * g.ldy + row0 / 2 + p] = __fmul_rn(silu((float)tot[m]), (float)up[m]);
        }
    } else if ((lane & 7) == 0) {
        const int r = 2 * (lane >> 4) + ((lane >> 3) & 1);
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (m < g.M) {
                const float val = (float)tot[m];
                g.y[(size_t)m * g.ldy + row0 + r] = g.res ? __fadd_rn(resv[m], val) : val;
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
                if (m < M) resv[m] = __ldcg(g.res + (size_t)m * g.ldres + (size_t)rt * kTR + rbase + my_row);
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

// Host-side check of a GEMV for the tiled kernels.
inline bool tg_shape_ok(int R, int K, int M, int in_mode, int epi, bool has_res, int max_k, int max_m) {
    if (R <= 0 || R % kTR != 0 || K <= 0 || K % kTK != 0 || K > max_k || M < 1 || M > max_m) return false;
    if (in_mode == IN_RMSNORM && K > kNormMax) return false;
    if (epi == EPI_SWIGLU && has_res) return false;
    return true;
}

}  // namespace s2k
