// s2k_prefill.cu -- prompt prefill GEMMs on the 5th-generation tensor cores
// (tcgen05, sm_100a): Y[T][R] = X[T][K] . W[R][K]^T for Q8_0, Q4_K and Q6_K
// weights.
//
// Arithmetic.  The reference's CPU mat-mul quantizes each activation row to
// Q8_0 and sums, per output, the block terms (int32 sum of 32 int8 products)
// * (d_w * d_x) (ggml vec_dot_q8_0_q8_0).  An int8 tensor-core MMA with K = 32
// (tcgen05.mma kind::i8) computes exactly one such block sum for a 128 x 64
// tile of (weight row, token) pairs into TMEM (int32, exact).  The epilogue
// warps read every block's sums from TMEM and add (double)s * ((double)d_w *
// (double)d_x) into double accumulators -- the same exact terms, summed in
// double and rounded to float once, as the GEMV kernels and the CPU oracle.
// So prefill through the tensor cores is bit-compatible with the decode path.
//
// Structure (one CTA per SM, each taking an equal run of (128 weight rows x
// 64 tokens x 512 columns) units, stream-K; see prefill_q8_kernel):
//   warp 0      TMA producer: weight tile slabs (4-D tensor map over the tile
//               layout of s2k_tgemv.cuh, 128 rows x 128 columns, 128-byte
//               swizzle), activation slabs (2-D map, 64 tokens x 128 columns),
//               and per 512-column K-tile the weight scales (bulk copies) and
//               activation scales (2-D map) into an 8-stage ring; the first
//               stages' weights are requested before the previous kernel has
//               finished (programmatic dependent launch).  No multicast loads
//               anywhere.
//   warp 1      MMA issuer (one elected lane): per stage four MMAs (one per
//               32-column block) into TMEM columns of a double-buffered 4 x 64
//               accumulator area, then tcgen05.commit to the stage's empty
//               barrier and the TMEM buffer's full barrier.
//   warps 2..17 epilogue: warp w reads TMEM lane quarter w % 4 (32 weight
//               rows) with tcgen05.ld.32x32b.x16 and forms the block terms in
//               double for its share of (16-token group, block phase).
// Partials of (row block, token tile) pairs split over CTAs go to global
// scratch; the CTA that completes a pair adds them in K order and runs the
// epilogue (residual or SwiGLU), like the GEMV kernels'.
//
// K-quant weights (Q4_K, Q6_K) take the same MMAs on an int8 prefill copy of
// the matrix (built once at finalize, kq_build_kernel), with the exact
// arithmetic of ggml's vec_dot_q4_K_q8_K / vec_dot_q6_K_q8_K kept in the
// epilogue: the activation rows are quantized to Q8_K (quant_rows_q8k_kernel),
// an MMA block of 32 columns gives one exact int32 sub-block sum s_j per
// (row, token), the epilogue forms isum = sum_j sc_j * s_j (and for Q4_K
// msum = sum_j m_j * bsum_j) in integers per 256-value super-block and adds
// the super-block term (d_w*d_x) * isum - (dmin_w*d_x) * msum in double.
// Q6_K's 16-value sub-blocks each get a 32-column MMA block of their own (16
// quants and 16 zeros; the activation rows carry the same zero padding), so
// the copy and the activation rows are twice as wide as the matrix.
#include "s2k_common.cuh"
#include "s2k_kernels.h"
#include "s2k_tc.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

namespace s2k {

constexpr int kPM = 128;                 // weight rows per CTA tile (MMA M)
constexpr int kPN = 64;                  // tokens per CTA tile (MMA N)
constexpr int kPKC = 128;                // K columns per stage (4 Q8_0 blocks, one 128-byte swizzle row)
constexpr int kPStages = 8;
constexpr int kPEpiWarps = 16;
constexpr int kPThreads = (2 + kPEpiWarps) * 32;  // warp 0 TMA, warp 1 MMA, warps 2..17 epilogue
constexpr int kPTmemCols = 512;          // 2 buffers x 4 blocks x 64 columns
constexpr uint32_t kPStageA = kPM * kPKC;  // 16 KB
// Token tile N (the MMA's N) follows the call: 16 or 32 tokens leave room for
// 8 or 4 TMEM accumulator buffers (4 blocks x N columns each), so the MMAs
// run that many chunks ahead of the epilogue; 64 for larger calls (2 buffers).
template <int N>
struct PSmemT {
    static constexpr int kNB = kPTmemCols / (4 * N);  // TMEM buffers
    // block-phase partials of the epilogue warps with phase > 0 (N = 16, 32)
    static constexpr int kRed = N < 64 ? (kPEpiWarps - 4) * 16 * 32 : 1;
    alignas(1024) uint8_t a[kPStages][kPStageA];
    alignas(1024) uint8_t b[kPStages][N * kPKC];
    alignas(128) __half dw[2][kPM][16];   // weight block scales of a 512-column K-tile
    alignas(128) double dx[2][N][16];     // activation block scales of the K-tile
    // K-quant: (d, dmin) of the K-tile's super-blocks per row (N = 64 only)
    alignas(16) __half2 ds[N == 64 ? 2 : 1][N == 64 ? kPM : 1][2];
    alignas(16) double red[kRed];
    uint64_t full[kPStages], empty[kPStages];
    uint64_t sfull[2], sempty[2];
    uint64_t tfull[kNB], tempty[kNB];
    uint32_t tmem_base;
    int last;
};
static_assert(sizeof(PSmemT<16>) + 1024 <= 227 * 1024, "prefill GEMM shared memory");
static_assert(sizeof(PSmemT<32>) + 1024 <= 227 * 1024, "prefill GEMM shared memory");
static_assert(sizeof(PSmemT<64>) + 1024 <= 227 * 1024, "prefill GEMM shared memory");

struct PrefillParams {
    int R, K, T;          // weight rows, columns; tokens
    int epi;              // EPI_STORE / EPI_SWIGLU
    float *y;             // [T][ldy]
    int ldy;
    const float *res;     // optional residual [T][ldres]
    int ldres;
    double *part;         // stream-K partials [gridDim.x][2][kPN][kPM]
    int *counters;        // K-tiles done per (row block, token tile) [R/128][token tiles], zero between launches
    const __half *wtiles; // weight tiles (scales read by bulk copies)
    const __half2 *side;  // K-quant: (d, dmin) per (row block, K-tile, row, super-block)
    int *err;
};

// K-quant modes of the GEMM (template argument KQ)
enum : int { KQ_NONE = 0, KQ_Q4K = 1, KQ_Q6K = 2 };

// Instruction descriptor: kind::i8, D s32, A and B signed int8, both K-major,
// N tokens, M = kPM.
template <int N>
constexpr uint32_t idesc_i8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kPM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0)
        : "memory");
}

// int32 -> double exactly with integer ops and one double add:
// bits(2^52 + 2^31 + s) - (2^52 + 2^31).
__device__ __forceinline__ double i2d_exact(int s) {
    return __hiloint2double(0x43300000, (int)((unsigned)s ^ 0x80000000u)) - 4503601774854144.0;
}

// Work split (stream-K): the (row block, token tile, K-tile) units, K-tile
// fastest, are dealt out in equal contiguous runs to one CTA per SM, so no
// partial wave of CTAs is left when the tile count is not a multiple of the
// SM count.  A CTA's run crosses (row block, token tile) pairs; a pair whose
// K-tiles are split over several CTAs is finished by the CTA that completes
// its count: it adds the CTAs' partials in K order and runs the epilogue.
__device__ __forceinline__ void unit_of(long long u, int NKT, int TT, int &rb, int &tt, int &kt) {
    kt = (int)(u % NKT);
    const long long r = u / NKT;
    tt = (int)(r % TT);
    rb = (int)(r / TT);
}
// first unit of CTA c of G over U units, and the CTA holding unit u
__device__ __forceinline__ long long ulo_of(int c, long long U, int G) { return (long long)c * U / G; }
__device__ __forceinline__ int cta_of(long long u, long long U, int G) { return (int)(((u + 1) * G - 1) / U); }

// Outputs of one weight row (this lane's) for tokens t .. t + n - 1 (n <= 8,
// warp-uniform) from their double sums: residual add or SwiGLU of the
// interleaved (gate, up) row pair.  Residuals are loaded before any store.
__device__ __forceinline__ void store_rows8(const PrefillParams &p, const double (&v)[8], int t, int n, int row,
                                            int lane) {
    if (p.epi == EPI_SWIGLU) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const double up = __shfl_down_sync(0xffffffffu, v[j], 1);
            if ((lane & 1) == 0 && j < n) p.y[(size_t)(t + j) * p.ldy + row / 2] = __fmul_rn(silu((float)v[j]), (float)up);
        }
        return;
    }
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = (p.res && j < n) ? __ldcg(p.res + (size_t)(t + j) * p.ldres + row) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (j < n) {
            const float x = (float)v[j];
            p.y[(size_t)(t + j) * p.ldy + row] = p.res ? __fadd_rn(r[j], x) : x;
        }
}

// 18 warps: 5 of them share a sub-partition's 16K registers, so at most 96
// registers per thread.
template <int N, int KQ>
__global__ void __launch_bounds__(kPThreads, 1)
    prefill_q8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap dxmap, PrefillParams p) {
    static_assert(KQ == KQ_NONE || N == 64, "K-quant epilogue: 64-token tiles (4 token groups, no block phases)");
    using Sm = PSmemT<N>;
    constexpr int NB = Sm::kNB;
    extern __shared__ uint8_t praw[];
    Sm &sm = *reinterpret_cast<Sm *>((reinterpret_cast<uintptr_t>(praw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int NKT = p.K / kTK, TT = (p.T + N - 1) / N, RB = p.R / kPM;
    const long long U = (long long)RB * TT * NKT;
    const long long u_lo = ulo_of(c, U, G), u_hi = ulo_of(c + 1, U, G);
    const int nchunk = (int)(u_hi - u_lo) * (kTK / kPKC);
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < kPStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.sfull[i], 1);
            mbar_init(&sm.sempty[i], kPEpiWarps);
        }
        for (int i = 0; i < NB; ++i) {
            mbar_init(&sm.tfull[i], 1);
            mbar_init(&sm.tempty[i], kPEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 1) {  // TMEM: 512 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                     "r"(kPTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    bool ok = true;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            // Weight tiles and weight scales do not depend on the previous
            // kernel: the first stages' are issued before waiting for it
            // (programmatic dependent launch), activations and their scales
            // after.
            const int pre = min(nchunk, kPStages);
            for (int i = 0; i < pre; ++i) {
                int rb, tt, kt;
                unit_of(u_lo + (i >> 2), NKT, TT, rb, tt, kt);
                const int kc = kt * 4 + (i & 3), st = i;
                if ((i & 3) == 0) {
                    const int sb = (i >> 2) & 1;
                    mbar_arrive_expect_tx(&sm.sfull[sb], 4 * 1024 + N * 16 * 8 + (KQ != KQ_NONE ? kPM * 8 : 0));
                    for (int q = 0; q < 4; ++q) {
                        const uint8_t *tile = reinterpret_cast<const uint8_t *>(p.wtiles) +
                                              ((size_t)(rb * 4 + q) * NKT + kt) * kTileBytes + kTileQ;
                        bulk_g2s_plain(&sm.dw[sb][q * 32][0], tile, 1024, &sm.sfull[sb]);
                    }
                    if constexpr (KQ != KQ_NONE)
                        bulk_g2s_plain(&sm.ds[sb][0][0], p.side + ((size_t)rb * NKT + kt) * kPM * 2, kPM * 8,
                                       &sm.sfull[sb]);
                }
                mbar_arrive_expect_tx(&sm.full[st], kPStageA + N * kPKC);
                tma_load_4d(sm.a[st], &wmap, (kc * kPKC) % kTK, 0, (kc * kPKC) / kTK, rb * 4, &sm.full[st]);
            }
            pdl_wait();
            for (int i = 0; i < pre; ++i) {
                int rb, tt, kt;
                unit_of(u_lo + (i >> 2), NKT, TT, rb, tt, kt);
                const int kc = kt * 4 + (i & 3);
                if ((i & 3) == 0) tma_load_2d(&sm.dx[(i >> 2) & 1][0][0], &dxmap, kt * 16, tt * N, &sm.sfull[(i >> 2) & 1]);
                tma_load_2d(sm.b[i], &xmap, kc * kPKC, tt * N, &sm.full[i]);
            }
            for (int i = pre; i < nchunk && ok; ++i) {
                int rb, tt, kt;
                unit_of(u_lo + (i >> 2), NKT, TT, rb, tt, kt);
                const int kc = kt * 4 + (i & 3), st = i % kPStages;
                if ((i & 3) == 0) {  // scales of a new K-tile
                    const int ti = i >> 2, sb = ti & 1;
                    if (ti >= 2) ok = mbar_wait(&sm.sempty[sb], ((ti >> 1) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                    if (!ok) break;
                    mbar_arrive_expect_tx(&sm.sfull[sb], 4 * 1024 + N * 16 * 8 + (KQ != KQ_NONE ? kPM * 8 : 0));
                    for (int q = 0; q < 4; ++q) {
                        const uint8_t *tile = reinterpret_cast<const uint8_t *>(p.wtiles) +
                                              ((size_t)(rb * 4 + q) * NKT + kt) * kTileBytes + kTileQ;
                        bulk_g2s_plain(&sm.dw[sb][q * 32][0], tile, 1024, &sm.sfull[sb]);
                    }
                    if constexpr (KQ != KQ_NONE)
                        bulk_g2s_plain(&sm.ds[sb][0][0], p.side + ((size_t)rb * NKT + kt) * kPM * 2, kPM * 8,
                                       &sm.sfull[sb]);
                    tma_load_2d(&sm.dx[sb][0][0], &dxmap, kt * 16, tt * N, &sm.sfull[sb]);
                }
                ok = mbar_wait(&sm.empty[st], ((i / kPStages) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                mbar_arrive_expect_tx(&sm.full[st], kPStageA + N * kPKC);
                tma_load_4d(sm.a[st], &wmap, (kc * kPKC) % kTK, 0, (kc * kPKC) / kTK, rb * 4, &sm.full[st]);
                tma_load_2d(sm.b[st], &xmap, kc * kPKC, tt * N, &sm.full[st]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            for (int i = 0; i < nchunk && ok; ++i) {
                const int st = i % kPStages, buf = i % NB;
                ok = mbar_wait(&sm.full[st], (i / kPStages) & 1, p.err, ERR_WAIT_FULL);
                if (ok && i >= NB) ok = mbar_wait(&sm.tempty[buf], ((i / NB) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int blk = 0; blk < 4; ++blk)
                    mma_i8(tmem + buf * 4 * N + blk * N, sw128_desc(sm.a[st] + 32 * blk), sw128_desc(sm.b[st] + 32 * blk),
                           idesc_i8<N>());
                mma_commit(&sm.empty[st]);
                mma_commit(&sm.tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        // Epilogue warp e = warp - 2 reads TMEM lane quarter q = warp % 4
        // (weight rows 32q .. 32q+31 of the row block, one per lane).  Per
        // (row block, token tile) segment the tile's existing tokens are cut
        // into TQ groups of 16 and the 4 blocks of a chunk into BS = 4 / TQ
        // phases, so all 16 warps work whatever the token count: warp e takes
        // token group e/4 % TQ and the blocks b with b % BS == e/4 / TQ.
        // Phase partials are added in phase order at the segment's end (block
        // terms are exact, their double sums order-free).  Every epilogue
        // warp runs the same sequence of named barriers: a failed wait only
        // skips work.
        pdl_wait();
        const int e = warp - 2, q = warp & 3, h4 = e >> 2;
        const int row_local = q * 32 + lane;
        double acc[16];
        int isum[KQ != KQ_NONE ? 16 : 1];  // K-quant: sum_j sc_j * s_j of the current super-block
#pragma unroll
        for (int j = 0; j < (KQ != KQ_NONE ? 16 : 1); ++j) isum[j] = 0;
        int rb, tt, kt, seg_kt0 = 0, TQ = 1, BS = 4, tg = 0, bp = 0, nvalid = 0, nv_tile = 0;
        unit_of(u_lo, NKT, TT, rb, tt, kt);
        bool first_seg = true;
        for (int i = 0; i < nchunk; ++i) {
            const int buf = i % NB, ti = i >> 2, sb = ti & 1;
            if ((i & 3) == 0) {
                if (i > 0 && ++kt == NKT) {  // next unit (K-tile fastest)
                    kt = 0;
                    if (++tt == TT) {
                        tt = 0;
                        ++rb;
                    }
                }
                if (i == 0 || kt == 0) {  // a new segment
                    seg_kt0 = kt;
                    nv_tile = min(N, p.T - tt * N);
                    // (64-token tiles keep 4 groups: no phase partials)
                    TQ = N == 64 ? 4 : (nv_tile <= 16 ? 1 : 2);
                    BS = 4 / TQ;
                    tg = h4 % TQ;
                    bp = h4 / TQ;
                    nvalid = min(16, max(0, nv_tile - 16 * tg));
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[j] = 0.0;
                }
                if (ok) ok = mbar_wait(&sm.sfull[sb], (ti >> 1) & 1, p.err, ERR_WAIT_FULL);
            }
            if (ok) ok = mbar_wait(&sm.tfull[buf], (i / NB) & 1, p.err, ERR_WAIT_FULL);
            if (ok) {
                tc_fence_after();
                if constexpr (KQ != KQ_NONE) {
                    // every block of the chunk (BS = 1): integer super-block sums
                    if (nvalid > 0) {
#pragma unroll
                        for (int blk = 0; blk < 4; ++blk) {
                            const int b = (i & 3) * 4 + blk;
                            int s[16];
                            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + buf * 4 * N + blk * N + 16 * tg, s);
                            const uint32_t scm = __half_as_ushort(sm.dw[sb][row_local][b]);
                            const int sc = KQ == KQ_Q4K ? (int)(scm & 0xff) : (int)(int8_t)(scm & 0xff);
#pragma unroll
                            for (int j = 0; j < 16; ++j) isum[j] += sc * s[j];
                        }
                        const bool sb_end = KQ == KQ_Q4K ? (i & 1) == 1 : (i & 3) == 3;
                        if (sb_end) {
                            const int sbl = KQ == KQ_Q4K ? (i & 3) >> 1 : 0;  // super-block of the K-tile
                            const float2 dd = __half22float2(sm.ds[sb][row_local][sbl]);
                            int mn[8];
                            if constexpr (KQ == KQ_Q4K) {
                                const uint4 pr = *reinterpret_cast<const uint4 *>(&sm.dw[sb][row_local][8 * sbl]);
                                const uint32_t pw[4] = {pr.x, pr.y, pr.z, pr.w};
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    mn[2 * k] = (int)((pw[k] >> 8) & 0xff);
                                    mn[2 * k + 1] = (int)(pw[k] >> 24);
                                }
                            }
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int2 *slot = reinterpret_cast<const int2 *>(&sm.dx[sb][16 * tg + j][8 * sbl]);
                                const float dxf = __int_as_float(slot[0].y);
                                if constexpr (KQ == KQ_Q4K) {
                                    int ms = 0;
#pragma unroll
                                    for (int k = 0; k < 8; ++k) ms += mn[k] * slot[k].x;
                                    const double d = (double)__fmul_rn(dd.x, dxf), dmn = (double)__fmul_rn(dd.y, dxf);
                                    acc[j] += fma(d, (double)isum[j], -(dmn * (double)ms));
                                } else {
                                    acc[j] += (double)__fmul_rn(dd.x, dxf) * (double)isum[j];
                                }
                                isum[j] = 0;
                            }
                        }
                    }
                } else if (nvalid > 0) {
                    for (int blk = bp; blk < 4; blk += BS) {
                        const int b = (i & 3) * 4 + blk;
                        int s[16];
                        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + buf * 4 * N + blk * N + 16 * tg, s);
                        const double dwr = (double)__half2float(sm.dw[sb][row_local][b]);
                        const double *dxc = &sm.dx[sb][16 * tg][b];
#pragma unroll
                        for (int g8 = 0; g8 < 2; ++g8)
                            if (8 * g8 < nvalid) {
#pragma unroll
                                for (int j = 8 * g8; j < 8 * g8 + 8; ++j)
                                    acc[j] = fma(i2d_exact(s[j]), dwr * dxc[j * 16], acc[j]);
                            }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sm.tempty[buf]);
                    if ((i & 3) == 3) mbar_arrive(&sm.sempty[sb]);
                }
            }
            if ((i & 3) != 3 || (kt != NKT - 1 && i != nchunk - 1)) continue;
            // ---- end of a segment: (rb, tt), K-tiles seg_kt0 .. kt ----
            if (N < 64 && BS > 1) {
                // phase partials through shared memory: warps with phase > 0
                // (epilogue warps 4..15) write, phase 0 adds in phase order
                if (bp > 0 && ok)
#pragma unroll
                    for (int j = 0; j < 16; ++j) sm.red[((e - 4) * 16 + j) * 32 + lane] = acc[j];
                named_sync(1, kPEpiWarps * 32);
                if (bp == 0 && ok)
                    for (int ph = 1; ph < BS; ++ph) {
                        const int we = (ph * TQ + tg) * 4 + (e & 3);  // epilogue warp of (q, tg, phase ph)
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[j] += sm.red[((we - 4) * 16 + j) * 32 + lane];
                    }
                named_sync(1, kPEpiWarps * 32);
            }
            const int t0 = tt * N;
            const int row = rb * kPM + row_local;
            if (seg_kt0 == 0 && kt == NKT - 1) {
                // the whole K range: this CTA writes the outputs
                if (bp == 0 && nvalid > 0 && ok)
#pragma unroll
                    for (int h8 = 0; h8 < 2; ++h8)
                        if (8 * h8 < nvalid) {
                            double v8[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) v8[j] = acc[8 * h8 + j];
                            store_rows8(p, v8, t0 + 16 * tg + 8 * h8, nvalid - 8 * h8, row, lane);
                        }
            } else {
                // part of the K range: partials to this CTA's slot (0: its
                // first segment, 1: its last), K-tiles counted per pair
                const int slot = first_seg ? 0 : 1;
                double *mine = p.part + ((size_t)c * 2 + slot) * kPN * kPM;
                if (bp == 0 && nvalid > 0 && ok)
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (j < nvalid) mine[(size_t)(16 * tg + j) * kPM + row_local] = acc[j];
                __threadfence();
                named_sync(1, kPEpiWarps * 32);
                if (e == 0 && lane == 0) {
                    int *ctr = p.counters + rb * TT + tt;
                    const int done = kt - seg_kt0 + 1;
                    const int prev = atomicAdd(ctr, done);
                    sm.last = prev + done == NKT;
                    if (prev + done == NKT) *ctr = 0;
                }
                named_sync(1, kPEpiWarps * 32);
                if (sm.last && ok) {
                    __threadfence();
                    // the CTAs holding this pair's K-tiles, in K order
                    const long long u0 = ((long long)rb * TT + tt) * NKT;
                    const int ca = cta_of(u0, U, G), cb = cta_of(u0 + NKT - 1, U, G);
                    // warp (q, g): rows 32q + lane, tokens 16g .. 16g + 15 of the tile
                    const int g = h4;
                    const int ntok = min(16, nv_tile - 16 * g);
                    if (ntok > 0) {
                        const bool first_is_last = ulo_of(ca, U, G) < u0;
                        for (int h8 = 0; h8 < 2; ++h8) {  // 8 tokens at a time
                            if (8 * h8 >= ntok) break;
                            double sum[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) sum[j] = 0.0;
                            for (int cc = ca; cc <= cb; ++cc) {  // K order
                                const int sl = (cc == ca && first_is_last) ? 1 : 0;
                                const double *src =
                                    p.part + (((size_t)cc * 2 + sl) * kPN + 16 * g + 8 * h8) * kPM + row_local;
                                double v[8];
#pragma unroll
                                for (int j = 0; j < 8; ++j) v[j] = 8 * h8 + j < ntok ? __ldcg(src + (size_t)j * kPM) : 0.0;
#pragma unroll
                                for (int j = 0; j < 8; ++j) sum[j] += v[j];
                            }
                            store_rows8(p, sum, t0 + 16 * g + 8 * h8, ntok - 8 * h8, row, lane);
                        }
                    }
                }
                named_sync(1, kPEpiWarps * 32);
            }
            first_seg = false;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// activation rows -> Q8_0 (int8 [T][K] + double block scales [T][K/32])
// ---------------------------------------------------------------------------
// Grid (token row, chunk of kQBlocks blocks); the arithmetic of the GEMV
// prologue (RMSNorm of rms_norm_weighted when norm_w is given, ggml x86
// quantize_row_q8_0).  Every CTA of a row forms the row's sum of squares
// itself (an L2 re-read of the row) so the chunks need no second launch.
constexpr int kQBlocks = 32;

__global__ void __launch_bounds__(256) quant_rows_q8_kernel(const float *x, int ldx, int K, const float *norm_w,
                                                           float eps, int8_t *xq, double *dx, float *act_out) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *row = x + (size_t)t * ldx;
    __shared__ double red[8];
    float sc = 1.f;
    if (norm_w != nullptr) {
        double s = 0.0;
        for (int i = tid * 4; i < K; i += 256 * 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(row + i));
            s += (double)__fmul_rn(v.x, v.x) + (double)__fmul_rn(v.y, v.y);
            s += (double)__fmul_rn(v.z, v.z) + (double)__fmul_rn(v.w, v.w);
        }
        s = warp_sum_d(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < 8; ++w) tot += red[w];
        const float mean = (float)(tot / (double)K);
        sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    // lane owns one value of a 32-value block; warp w handles blocks w, w + 8, ... of the chunk
    const int b0 = blockIdx.y * kQBlocks, b1 = min(K / 32, b0 + kQBlocks);
    for (int b = b0 + warp; b < b1; b += 8) {
        float v = __ldcg(row + b * 32 + lane);
        if (norm_w != nullptr) v = __fmul_rn(__fmul_rn(v, sc), __ldg(norm_w + b * 32 + lane));
        if (act_out != nullptr) act_out[(size_t)t * K + b * 32 + lane] = v;
        float amax = warp_max(fabsf(v));
        const float id = amax != 0.0f ? __fdiv_rn(127.f, amax) : 0.0f;
        xq[(size_t)t * K + b * 32 + lane] = (int8_t)(__float_as_int(__fadd_rn(__fmul_rn(v, id), 12582912.f)) & 0xff);
        if (lane == 0) dx[(size_t)t * (K / 32) + b] = (double)__half2float(__float2half_rn(__fdiv_rn(amax, 127.f)));
    }
}

// ---------------------------------------------------------------------------
// K-quant prefill copy: int8 tiles in the Q8_0 tile geometry (32 x 512 int8,
// then 2 bytes per (row, 32-column block)) + side (d, dmin) per super-block
// ---------------------------------------------------------------------------
// One thread per (row, 32-column block of the copy).  Q4_K: block j of a
// super-block holds sub-block j's 32 quants (0..15, the nibbles of ggml's qs
// bytes 32*(j/2) .. +31, low nibble for even j) and the bytes (sc_j, m_j) of
// get_scale_min_k4.  Q6_K: copy block j holds sub-block j's 16 quants
// (q - 32, as dequantize_row_q6_K forms them) then 16 zeros, and the bytes
// (sc_j, 0).  side[rb][kt][row % 128][slot] = (d, dmin) of the super-block
// the K-tile's slot covers (Q4_K: two per K-tile; Q6_K: one, dmin 0).
__global__ void kq_build_kernel(const uint8_t *__restrict__ src, int wtype, int R, int K, uint8_t *__restrict__ dst,
                                __half2 *__restrict__ side) {
    const int Ke = wtype == TW_Q6_K ? 2 * K : K;  // copy columns
    const int NBe = Ke / 32, NKTs = K / kTK, NKTe = Ke / kTK;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)R * NBe) return;
    const int row = (int)(idx / NBe), be = (int)(idx % NBe);
    const int kte = be / 16, bl = be % 16;
    const int rl = row % kTR;
    uint8_t *tile = dst + ((size_t)(row / kTR) * NKTe + kte) * kTileBytes;
    // the sub-block's 32 (Q6_K: 16, then 16 zeros) int8 values, four per word,
    // from 16-byte loads of the source planes
    uint32_t w[8];
    uint16_t scm;
    __half2 dd = __floats2half2_rn(0.f, 0.f);
    bool first = false;
    int slot = 0;
    if (wtype == TW_Q4_K) {
        const int sbg = be / 8, j = be % 8;  // super-block of the row, sub-block
        const uint8_t *t = src + ((size_t)(row / kTR) * NKTs + sbg / 2) * kTileBytesQ4K;
        const int rb2 = rl * 2 + (sbg & 1);
        const uint4 *qs = reinterpret_cast<const uint4 *>(t + rb2 * 128 + 32 * (j >> 1));
        const uint4 a0 = qs[0], a1 = qs[1];
        const uint32_t src_w[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const int sh = (j & 1) ? 4 : 0;  // odd sub-blocks: the high nibbles
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = (src_w[k] >> sh) & 0x0F0F0F0Fu;
        const uint8_t *hd = t + kQ4kHdr + rb2 * 16;
        int sc, mn;
        q4k_scale_min(j, hd + 4, &sc, &mn);
        scm = (uint16_t)(sc | (mn << 8));
        first = j == 0;
        slot = sbg & 1;
        dd = __halves2half2(__ushort_as_half(*reinterpret_cast<const unsigned short *>(hd)),
                            __ushort_as_half(*reinterpret_cast<const unsigned short *>(hd + 2)));
    } else {
        const int sbg = kte, j = bl;  // one super-block per copy K-tile, 16-value sub-block j
        const uint8_t *t = src + ((size_t)(row / kTR) * NKTs + sbg / 2) * kTileBytesQ6K;
        const int rb2 = rl * 2 + (sbg & 1);
        // values 16j .. 16j+15 of the super-block: half h, quarter k, lanes l0 .. l0+15
        const int h = j >> 3, k = (j >> 1) & 3, l0 = 16 * (j & 1);
        const uint4 ql = *reinterpret_cast<const uint4 *>(t + rb2 * 128 + 64 * h + l0 + ((k & 1) << 5));
        const uint4 qh = *reinterpret_cast<const uint4 *>(t + kQ6kQh + rb2 * 64 + 32 * h + l0);
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w}, hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const uint32_t lo = ((k & 2) ? (lw[x] >> 4) : lw[x]) & 0x0F0F0F0Fu;
            const uint32_t hi = ((hw[x] >> (2 * k)) & 0x03030303u) << 4;
            w[x] = __vsub4(lo | hi, 0x20202020u);  // q - 32 per byte
        }
#pragma unroll
        for (int x = 4; x < 8; ++x) w[x] = 0;
        scm = (uint16_t)t[kQ6kSc + rb2 * 16 + j];
        first = j == 0;
        slot = 0;
        dd = __halves2half2(__ushort_as_half(*reinterpret_cast<const unsigned short *>(t + kQ6kD + rb2 * 2)),
                            __float2half_rn(0.f));
    }
    uint4 *qd = reinterpret_cast<uint4 *>(tile + rl * kTK + bl * 32);
    qd[0] = make_uint4(w[0], w[1], w[2], w[3]);
    qd[1] = make_uint4(w[4], w[5], w[6], w[7]);
    reinterpret_cast<uint16_t *>(tile + kTileQ)[rl * 16 + bl] = scm;
    if (first) {
        side[(((size_t)(row / kPM) * NKTe + kte) * kPM + row % kPM) * 2 + slot] = dd;
        if (wtype == TW_Q6_K) side[(((size_t)(row / kPM) * NKTe + kte) * kPM + row % kPM) * 2 + 1] = dd;
    }
}

// Activation rows -> Q8_K for the K-quant GEMM: int8 rows [T][Ke] (Q6_K:
// every 16 values followed by 16 zeros) and per 32-column copy block a slot
// (low word: the block's value sum, high word: the super-block's d as float
// bits).  The arithmetic of the GEMV prologue (RMSNorm, quant_q8k_warp).
// Grid (token row, 8 super-blocks per CTA), one warp per super-block.
__global__ void __launch_bounds__(256) quant_rows_q8k_kernel(const float *x, int ldx, int K, const float *norm_w,
                                                            float eps, int wtype, int8_t *xq, double *slots,
                                                            float *act_out) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *row = x + (size_t)t * ldx;
    __shared__ double red[8];
    __shared__ int16_t bs[8][16];
    __shared__ float dsh[8];
    float sc = 1.f;
    if (norm_w != nullptr) {
        double s = 0.0;
        for (int i = tid * 4; i < K; i += 256 * 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(row + i));
            s += (double)__fmul_rn(v.x, v.x) + (double)__fmul_rn(v.y, v.y);
            s += (double)__fmul_rn(v.z, v.z) + (double)__fmul_rn(v.w, v.w);
        }
        s = warp_sum_d(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < 8; ++w) tot += red[w];
        const float mean = (float)(tot / (double)K);
        sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    const int sbi = blockIdx.y * 8 + warp;
    if (sbi >= K / 256) return;
    const int c0 = sbi * 256 + 8 * lane;
    const float4 a = __ldcg(reinterpret_cast<const float4 *>(row + c0));
    const float4 b = __ldcg(reinterpret_cast<const float4 *>(row + c0 + 4));
    float y[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (norm_w != nullptr) {
        const float4 wa = __ldg(reinterpret_cast<const float4 *>(norm_w + c0));
        const float4 wb = __ldg(reinterpret_cast<const float4 *>(norm_w + c0 + 4));
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = __fmul_rn(__fmul_rn(y[e], sc), wv[e]);
    }
    if (act_out != nullptr) {
        float4 *dst = reinterpret_cast<float4 *>(act_out + (size_t)t * K + c0);
        dst[0] = make_float4(y[0], y[1], y[2], y[3]);
        dst[1] = make_float4(y[4], y[5], y[6], y[7]);
    }
    const bool q6 = wtype == TW_Q6_K;
    const int Ke = q6 ? 2 * K : K;
    int8_t *xr = xq + (size_t)t * Ke;
    // Q4_K: values in place; Q6_K: 16-value group g = lane / 2 at copy column 32 g (+ 8 for odd lanes)
    int8_t *dstq = q6 ? xr + (size_t)sbi * 512 + (lane >> 1) * 32 + (lane & 1) * 8 : xr + c0;
    quant_q8k_warp(y, lane, true, dstq, &dsh[warp], &bs[warp][0]);
    if (q6) *reinterpret_cast<uint2 *>(dstq + 16) = make_uint2(0u, 0u);
    __syncwarp();
    const float d = dsh[warp];
    double *sl = slots + (size_t)t * (Ke / 32);
    if (q6) {
        if (lane < 16) sl[sbi * 16 + lane] = __hiloint2double(__float_as_int(d), 0);
    } else if (lane < 8) {
        sl[sbi * 8 + lane] = __hiloint2double(__float_as_int(d), (int)bs[warp][2 * lane] + (int)bs[warp][2 * lane + 1]);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
cudaError_t prefill_setup() {
    if (!encode_fn()) return cudaErrorNotSupported;
    cudaError_t e = cudaFuncSetAttribute(prefill_q8_kernel<16, KQ_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(sizeof(PSmemT<16>) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_q8_kernel<32, KQ_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(sizeof(PSmemT<32>) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_q8_kernel<64, KQ_NONE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(sizeof(PSmemT<64>) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_q8_kernel<64, KQ_Q4K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(sizeof(PSmemT<64>) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_q8_kernel<64, KQ_Q6K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(sizeof(PSmemT<64>) + 1024));
    return e;
}

static bool is_kq(int type) { return type == 12 || type == 14; }

bool prefill_ok(const DevMat &w, int T) {
    if (w.rows % kPM != 0 || w.cols % kTK != 0 || T < 1) return false;
    if (w.type == 8) return true;
    // K-quant: the int8 copy exists and the call fills 64-token tiles
    return is_kq(w.type) && w.pf != nullptr && w.pf_side != nullptr && T >= kPN;
}

size_t kq_prefill_bytes(const DevMat &w, size_t *side_bytes) {
    if (!is_kq(w.type) || w.rows % kPM != 0 || w.cols % kTK != 0) {
        if (side_bytes) *side_bytes = 0;
        return 0;
    }
    const size_t ke = (size_t)w.cols * (w.type == 14 ? 2 : 1);
    if (side_bytes) *side_bytes = (size_t)w.rows * (ke / kTK) * 2 * sizeof(__half2);
    return (size_t)(w.rows / kTR) * (ke / kTK) * kTileBytes;
}

cudaError_t launch_build_kq_prefill(const DevMat &w, cudaStream_t st) {
    size_t sb = 0;
    if (!w.w || !w.pf || !w.pf_side || kq_prefill_bytes(w, &sb) == 0) return cudaErrorInvalidValue;
    const int wt = w.type == 12 ? TW_Q4_K : TW_Q6_K;
    const long long n = (long long)w.rows * (w.cols * (wt == TW_Q6_K ? 2 : 1) / 32);
    count_launch();
    kq_build_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w.w, wt, w.rows, w.cols, w.pf,
                                                                 reinterpret_cast<__half2 *>(w.pf_side));
    return cudaGetLastError();
}

cudaError_t launch_quant_rows_q8k(const float *x, int ldx, int T, int K, const float *norm_w, float eps, int ggml_type,
                                  int8_t *xq, double *slots, float *act_out, cudaStream_t st) {
    if (!is_kq(ggml_type) || K % 256 != 0 || T < 1 || ldx % 4 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0)
        return cudaErrorInvalidValue;
    count_launch();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T, (K / 256 + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quant_rows_q8k_kernel, x, ldx, K, norm_w, eps,
                              ggml_type == 12 ? (int)TW_Q4_K : (int)TW_Q6_K, xq, slots, act_out);
}

cudaError_t launch_prefill_gemm(const PrefillArgs &a, cudaStream_t st) {
    const DevMat &w = *a.w;
    EncodeTiledFn enc = encode_fn();
    if (!enc || !prefill_ok(w, a.T) || !a.xq || !a.dx || !a.counters) return cudaErrorInvalidValue;
    const int kq = w.type == 12 ? KQ_Q4K : (w.type == 14 ? KQ_Q6K : KQ_NONE);
    // K: columns of the operand tiles (the K-quant copy is twice as wide for Q6_K)
    const int R = w.rows, K = w.cols * (kq == KQ_Q6K ? 2 : 1), NKT = K / kTK, RT = R / kTR;
    const int N = a.T <= 16 ? 16 : (a.T <= 32 ? 32 : 64);  // token tile
    uint8_t *wt = kq != KQ_NONE ? w.pf : w.w;
    CUtensorMap wmap, xmap, dxmap;
    {
        const cuuint64_t dims[4] = {(cuuint64_t)kTK, (cuuint64_t)kTR, (cuuint64_t)NKT, (cuuint64_t)RT};
        const cuuint64_t strides[3] = {(cuuint64_t)kTK, (cuuint64_t)kTileBytes, (cuuint64_t)kTileBytes * NKT};
        const cuuint32_t box[4] = {(cuuint32_t)kPKC, (cuuint32_t)kTR, 1, 4};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, wt, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)a.T};
        const cuuint64_t strides[1] = {(cuuint64_t)K};
        const cuuint32_t box[2] = {(cuuint32_t)kPKC, (cuuint32_t)N};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(a.xq), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(K / 32), (cuuint64_t)a.T};
        const cuuint64_t strides[1] = {(cuuint64_t)(K / 32) * 8};
        const cuuint32_t box[2] = {16, (cuuint32_t)N};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&dxmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(a.dx), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    const int RB = R / kPM, TT = (a.T + N - 1) / N;
    const long long U = (long long)RB * TT * NKT;
    const int G = (int)std::min<long long>(a.num_sms, U);
    if (!a.part || prefill_part_doubles(G) > a.part_doubles || (size_t)RB * TT > a.n_counters)
        return cudaErrorInvalidValue;
    PrefillParams p;
    p.R = R;
    p.K = K;
    p.T = a.T;
    p.epi = a.epi;
    p.y = a.y;
    p.ldy = a.ldy;
    p.res = a.res;
    p.ldres = a.ldres;
    p.part = a.part;
    p.counters = a.counters;
    p.wtiles = reinterpret_cast<const __half *>(wt);
    p.side = reinterpret_cast<const __half2 *>(w.pf_side);
    p.err = a.err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = (N == 16 ? sizeof(PSmemT<16>) : N == 32 ? sizeof(PSmemT<32>) : sizeof(PSmemT<64>)) + 1024;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    if (kq == KQ_Q4K) return cudaLaunchKernelEx(&cfg, prefill_q8_kernel<64, KQ_Q4K>, wmap, xmap, dxmap, p);
    if (kq == KQ_Q6K) return cudaLaunchKernelEx(&cfg, prefill_q8_kernel<64, KQ_Q6K>, wmap, xmap, dxmap, p);
    if (N == 16) return cudaLaunchKernelEx(&cfg, prefill_q8_kernel<16, KQ_NONE>, wmap, xmap, dxmap, p);
    if (N == 32) return cudaLaunchKernelEx(&cfg, prefill_q8_kernel<32, KQ_NONE>, wmap, xmap, dxmap, p);
    return cudaLaunchKernelEx(&cfg, prefill_q8_kernel<64, KQ_NONE>, wmap, xmap, dxmap, p);
}

size_t prefill_part_doubles(int ctas) { return (size_t)ctas * 2 * kPN * kPM; }

cudaError_t launch_quant_rows_q8(const float *x, int ldx, int T, int K, const float *norm_w, float eps, int8_t *xq,
                                 double *dx, float *act_out, cudaStream_t st) {
    if (K % 32 != 0 || T < 1 || ldx % 4 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0) return cudaErrorInvalidValue;
    count_launch();
    const int nch = (K / 32 + kQBlocks - 1) / kQBlocks;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T, nch);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, quant_rows_q8_kernel, x, ldx, K, norm_w, eps, xq, dx, act_out);
}

}  // namespace s2k
