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
// all K-tiles of a row tile; the warp reduces them once per row tile (the
// butterfly leaves every lane with the sums) and lanes 0..3 store one row
// each.  Rows (2i, 2i+1) of a SwiGLU matrix (gate/up interleaved at upload)
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

// Quantize one 32-value block held in registers (ggml x86 quantize_row_q8_0:
// d = amax/127 stored fp16, q = round-half-even(x * 127/amax)).
__device__ __forceinline__ void tg_quant_block(const float4 (&v)[8], int8_t *xq_blk, float *xd_blk) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        amax = fmaxf(fmaxf(fmaxf(amax, fabsf(v[j].x)), fmaxf(fabsf(v[j].y), fabsf(v[j].z))), fabsf(v[j].w));
    const float d = __fdiv_rn(amax, 127.f);
    const float id = amax != 0.0f ? __fdiv_rn(127.f, amax) : 0.0f;
    int pk[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int q0 = __float2int_rn(__fmul_rn(v[j].x, id)), q1 = __float2int_rn(__fmul_rn(v[j].y, id));
        const int q2 = __float2int_rn(__fmul_rn(v[j].z, id)), q3 = __float2int_rn(__fmul_rn(v[j].w, id));
        pk[j] = (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
    }
    int4 *dq = reinterpret_cast<int4 *>(xq_blk);
    dq[0] = make_int4(pk[0], pk[1], pk[2], pk[3]);
    dq[1] = make_int4(pk[4], pk[5], pk[6], pk[7]);
    *xd_blk = __half2float(__float2half_rn(d));
}

__device__ __forceinline__ double sumsq_block(const float4 (&v)[8]) {
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        s += (double)__fmul_rn(v[j].x, v[j].x) + (double)__fmul_rn(v[j].y, v[j].y) +
             (double)__fmul_rn(v[j].z, v[j].z) + (double)__fmul_rn(v[j].w, v[j].w);
    return s;
}

__device__ __forceinline__ void load_block(const float *src, float4 (&v)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(reinterpret_cast<const float4 *>(src) + j);
}

// Prologue (all NT consumer threads): activation rows -> Q8_0 blocks in shared
// memory (xq [M][K] int8, xd [M][K/32] fp16-rounded scales as float), with the
// RMSNorm of rms_norm_weighted (src/s2_model.cpp:46-55) when in_mode says so.
// nws [kNormMax] receives the norm weights; tok [NT/32][tok_ld] (tok_ld >= MT)
// and scale [MT] are small shared scratch arrays.  write_act: this CTA stores
// act_out (exactly one CTA of the grid should).  The caller synchronizes the
// consumer threads after it returns.
// A thread owns whole 32-value blocks (item = token * NB + block).  The norm
// weights are copied to shared memory by loads issued together with the
// activation loads, so at decode widths (one block per thread) the prologue
// costs one L2 round trip, and the activation block stays in registers
// between the sum of squares and the quantizer.
template <int MT, int NT>
__device__ __forceinline__ void tg_prologue(const TGemv &g, int8_t *xq, float *xd, float *nws, double *tok,
                                            int tok_ld, float *scale, bool write_act, int bar_id) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = g.K, NB = K >> 5, M = g.M;
    const int items = M * NB;
    const bool rms = g.in_mode == IN_RMSNORM;
    const bool one = items <= NT;
    float4 v[8];
    if (one && tid < items) load_block(g.x + (size_t)(tid / NB) * g.ldx + (tid % NB) * 32, v);
    if (rms) {
        for (int i = tid; i < K / 4; i += NT)
            reinterpret_cast<float4 *>(nws)[i] = __ldg(reinterpret_cast<const float4 *>(g.norm_w) + i);
        double tk[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tk[m] = 0.0;
        for (int it = tid; it < items; it += NT) {
            const int m = it / NB, b = it - m * NB;
            if (!one) load_block(g.x + (size_t)m * g.ldx + b * 32, v);
            const double s = sumsq_block(v);
#pragma unroll
            for (int mm = 0; mm < MT; ++mm)
                if (mm == m) tk[mm] += s;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const double t = warp_sum_d(tk[m]);
            if (lane == 0) tok[warp * tok_ld + m] = t;
        }
        named_sync(bar_id, NT);  // tok and nws complete
        if (tid < M) {
            double tot = 0.0;
            for (int w = 0; w < NT / 32; ++w) tot += tok[w * tok_ld + tid];
            const float mean = (float)(tot / (double)K);
            scale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, g.eps)));
        }
        named_sync(bar_id, NT);
    }
    for (int it = tid; it < items; it += NT) {
        const int m = it / NB, b = it - m * NB;
        if (!one) load_block(g.x + (size_t)m * g.ldx + b * 32, v);
        if (rms) {
            const float sc = scale[m];
            const float4 *nw = reinterpret_cast<const float4 *>(nws + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 w4 = nw[j];
                v[j].x = __fmul_rn(__fmul_rn(v[j].x, sc), w4.x);
                v[j].y = __fmul_rn(__fmul_rn(v[j].y, sc), w4.y);
                v[j].z = __fmul_rn(__fmul_rn(v[j].z, sc), w4.z);
                v[j].w = __fmul_rn(__fmul_rn(v[j].w, sc), w4.w);
            }
        }
        if (g.act_out != nullptr && write_act) {
            float4 *dst = reinterpret_cast<float4 *>(g.act_out + (size_t)m * K + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = v[j];
        }
        tg_quant_block(v, xq + (size_t)m * K + b * 32, xd + m * NB + b);
    }
}

// Epilogue of row tile rt: lane i < 4 stores row 4w + i (EPI_STORE, with the
// residual resv[m] it prefetched) or, for SwiGLU, lane p < 2 stores output
// pair p of the warp.  tot[i][m] are the warp-reduced row sums (all lanes).
template <int MT>
__device__ __forceinline__ void tg_emit(const TGemv &g, int rt, int warp, int lane, const double (&tot)[kTRW][MT],
                                        const float (&resv)[MT]) {
    const int row0 = rt * kTR + warp * kTRW;
    if (g.epi == EPI_SWIGLU) {
        if (lane < kTRW / 2) {
#pragma unroll
            for (int p = 0; p < kTRW / 2; ++p)
                if (p == lane)
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        if (m < g.M)
                            g.y[(size_t)m * g.ldy + row0 / 2 + p] =
                                __fmul_rn(silu((float)tot[2 * p][m]), (float)tot[2 * p + 1][m]);
        }
    } else if (lane < kTRW) {
#pragma unroll
        for (int i = 0; i < kTRW; ++i)
            if (i == lane)
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < g.M) {
                        const float val = (float)tot[i][m];
                        g.y[(size_t)m * g.ldy + row0 + i] = g.res ? __fadd_rn(resv[m], val) : val;
                    }
    }
}

// Consumer (the kTNC consumer threads): this CTA's row tiles of one GEMV,
// after the prologue filled xq / xd.  cs counts stages consumed over the
// ring's lifetime.
template <int MT>
__device__ __forceinline__ void tg_consume(const TGemv &g, const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                           int nst, int &cs, const int8_t *xq, const float *xd, int cta, int G,
                                           int *err) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = g.K, NKT = K / kTK, NB = K >> 5, M = g.M;
    long long u0, u1;
    tg_range(g.R, K, cta, G, &u0, &u1);
    double acc[kTRW][MT];
#pragma unroll
    for (int i = 0; i < kTRW; ++i)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[i][m] = 0.0;
    float resv[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) resv[m] = 0.f;
    const int rbase = warp * kTRW;
    for (long long u = u0; u < u1; ++u, ++cs) {
        const int rt = (int)(u / NKT), kt = (int)(u - (long long)rt * NKT);
        const int slot = cs % nst;
        if (kt == 0 && g.res != nullptr && lane < kTRW) {
            // residual of this lane's output row, needed at the row tile's end
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < M) resv[m] = __ldcg(g.res + (size_t)m * g.ldres + (size_t)rt * kTR + rbase + lane);
        }
        // this lane's activation chunk of K-tile kt, per token
        int4 xa[MT];
        float xs[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const int mm = m < M ? m : 0;
            xa[m] = *reinterpret_cast<const int4 *>(xq + (size_t)mm * K + kt * kTK + lane * 16);
            xs[m] = xd[mm * NB + kt * (kTK / 32) + (lane >> 1)];
        }
        mbar_wait(&full[slot], (cs / nst) & 1, err, ERR_WAIT_FULL);
        const uint8_t *t = ring + (size_t)slot * kTileBytes;
        int4 wv[kTRW];
        float dw[kTRW];
#pragma unroll
        for (int i = 0; i < kTRW; ++i) {
            wv[i] = *reinterpret_cast<const int4 *>(t + (rbase + i) * kTK + lane * 16);
            dw[i] = __half2float(reinterpret_cast<const __half *>(t + kTileQ)[(rbase + i) * (kTK / 32) + (lane >> 1)]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // data is in registers: the slot may refill
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
        if (kt != NKT - 1) continue;
#pragma unroll
        for (int i = 0; i < kTRW; ++i)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[i][m] = warp_sum_d(acc[i][m]);
        tg_emit<MT>(g, rt, warp, lane, acc, resv);
#pragma unroll
        for (int i = 0; i < kTRW; ++i)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[i][m] = 0.0;
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
