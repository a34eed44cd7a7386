// s2k_prefill.cu -- prompt prefill GEMMs on the 5th-generation tensor cores
// (tcgen05, sm_100a): Y[T][R] = X[T][K] . W[R][K]^T for Q8_0 weights.
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
// Structure (one CTA per SM; 128 weight rows x 64 tokens per CTA tile, split
// over K when the tile grid is small):
//   warp 0      TMA producer: weight tile slabs (4-D tensor map over the tile
//               layout of s2k_tgemv.cuh, 128 rows x 128 columns, 128-byte
//               swizzle), activation slabs (2-D map, 64 tokens x 128 columns),
//               and per 512-column K-tile the weight scales (bulk copies) and
//               activation scales (2-D map) into a 4-stage ring.  No
//               multicast loads anywhere.
//   warp 1      MMA issuer (one elected lane): per stage four MMAs (one per
//               32-column block) into TMEM columns of a double-buffered 4 x 64
//               accumulator area, then tcgen05.commit to the stage's empty
//               barrier and the TMEM buffer's full barrier.
//   warps 2..9  epilogue: warp w reads TMEM lane quarter w % 4 (32 weight
//               rows) and token half (w - 2) / 4 (32 tokens) with
//               tcgen05.ld.32x32b.x32, forms the block terms in double.
// Split-K partials go to global scratch; the last CTA of a (row block, token
// tile) to arrive adds them in split order and runs the epilogue (residual or
// SwiGLU), like the GEMV kernels'.
#include "s2k_common.cuh"
#include "s2k_kernels.h"

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
constexpr uint32_t kPStageB = kPN * kPKC;  // 8 KB

struct PSmem {
    alignas(1024) uint8_t a[kPStages][kPStageA];
    alignas(1024) uint8_t b[kPStages][kPStageB];
    alignas(128) __half dw[2][kPM][16];   // weight block scales of a 512-column K-tile
    alignas(128) double dx[2][kPN][16];   // activation block scales of the K-tile
    uint64_t full[kPStages], empty[kPStages];
    uint64_t sfull[2], sempty[2];
    uint64_t tfull[2], tempty[2];
    uint32_t tmem_base;
    int last;
};
static_assert(sizeof(PSmem) + 1024 <= 227 * 1024, "prefill GEMM shared memory");

struct PrefillParams {
    int R, K, T;          // weight rows, columns; tokens
    int nsplit;           // K splits (whole 512-column K-tiles each)
    int epi;              // EPI_STORE / EPI_SWIGLU
    float *y;             // [T][ldy]
    int ldy;
    const float *res;     // optional residual [T][ldres]
    int ldres;
    double *part;         // split partials [nsplit][T][R] (nsplit > 1)
    int *counters;        // [R/128][token tiles], zero between launches
    const __half *wtiles; // weight tiles (scales read by bulk copies)
    int *err;
};

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int x, int y, int z, int w,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzle layout TMA writes: rows of 128 bytes, 8-row atoms of 1024 bytes
// (stride byte offset 1024), leading byte offset 16, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(const void *p) {
    const uint64_t addr = smem_u32(p);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: kind::i8, D s32, A and B signed int8, both K-major,
// N = kPN, M = kPM.
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPN >> 3) << 17) |
                              ((uint32_t)(kPM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdescI8), "r"(0)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// int32 -> double exactly with integer ops and one double add:
// bits(2^52 + 2^31 + s) - (2^52 + 2^31).
__device__ __forceinline__ double i2d_exact(int s) {
    return __hiloint2double(0x43300000, (int)((unsigned)s ^ 0x80000000u)) - 4503601774854144.0;
}

__global__ void __launch_bounds__(kPThreads, 1)
    prefill_q8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap dxmap, PrefillParams p) {
    extern __shared__ uint8_t praw[];
    PSmem &sm = *reinterpret_cast<PSmem *>((reinterpret_cast<uintptr_t>(praw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = blockIdx.x, tt = blockIdx.y, split = blockIdx.z;
    const int NKT = p.K / kTK;
    const int kt0 = NKT * split / p.nsplit, kt1 = NKT * (split + 1) / p.nsplit;
    const int nchunk = (kt1 - kt0) * (kTK / kPKC);
    const int t0 = tt * kPN;
    if (tid == 0) {
        for (int i = 0; i < kPStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.sfull[i], 1);
            mbar_init(&sm.sempty[i], kPEpiWarps);
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
            for (int i = 0; i < nchunk && ok; ++i) {
                const int kc = kt0 * 4 + i, st = i % kPStages;
                if ((i & 3) == 0) {  // scales of a new K-tile
                    const int ti = i >> 2, sb = ti & 1;
                    if (ti >= 2) ok = mbar_wait(&sm.sempty[sb], ((ti >> 1) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                    if (!ok) break;
                    const int kt = kc >> 2;
                    mbar_arrive_expect_tx(&sm.sfull[sb], 4 * 1024 + kPN * 16 * 8);
                    for (int q = 0; q < 4; ++q) {
                        const uint8_t *tile = reinterpret_cast<const uint8_t *>(p.wtiles) +
                                              ((size_t)(rb * 4 + q) * NKT + kt) * kTileBytes + kTileQ;
                        bulk_g2s_plain(&sm.dw[sb][q * 32][0], tile, 1024, &sm.sfull[sb]);
                    }
                    tma_load_2d(&sm.dx[sb][0][0], &dxmap, kt * 16, t0, &sm.sfull[sb]);
                }
                if (i >= kPStages) ok = mbar_wait(&sm.empty[st], ((i / kPStages) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                mbar_arrive_expect_tx(&sm.full[st], kPStageA + kPStageB);
                tma_load_4d(sm.a[st], &wmap, (kc * kPKC) % kTK, 0, (kc * kPKC) / kTK, rb * 4, &sm.full[st]);
                tma_load_2d(sm.b[st], &xmap, kc * kPKC, t0, &sm.full[st]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            for (int i = 0; i < nchunk && ok; ++i) {
                const int st = i % kPStages, buf = i & 1;
                ok = mbar_wait(&sm.full[st], (i / kPStages) & 1, p.err, ERR_WAIT_FULL);
                if (ok && i >= 2) ok = mbar_wait(&sm.tempty[buf], ((i >> 1) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int blk = 0; blk < 4; ++blk)
                    mma_i8(tmem + buf * 256 + blk * kPN, sw128_desc(sm.a[st] + 32 * blk), sw128_desc(sm.b[st] + 32 * blk));
                mma_commit(&sm.empty[st]);
                mma_commit(&sm.tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        // Epilogue warp e = warp - 2 reads TMEM lane quarter q = warp % 4
        // (weight rows 32q .. 32q+31, one per lane).  The tile's existing
        // tokens are cut into TQ groups of 16 and the 4 blocks of a chunk
        // into BS = 4 / TQ phases, so all 16 warps work whatever the token
        // count: warp e takes token group e/4 % TQ and the blocks b with
        // b % BS == e/4 / TQ.  Phase partials are added in phase order at the
        // end (block terms are exact, their double sums order-free).
        const int q = warp & 3, h4 = (warp - 2) >> 2;
        const int row_local = q * 32 + lane;
        const int nv_tile = min(kPN, p.T - t0);
        const int TQ = nv_tile <= 16 ? 1 : (nv_tile <= 32 ? 2 : 4);
        const int BS = 4 / TQ;
        const int tg = h4 % TQ, bp = h4 / TQ;
        const int nvalid = min(16, max(0, nv_tile - 16 * tg));  // warp-uniform
        double acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.0;
        for (int i = 0; i < nchunk && ok; ++i) {
            const int buf = i & 1, ti = i >> 2, sb = ti & 1;
            if ((i & 3) == 0) ok = mbar_wait(&sm.sfull[sb], (ti >> 1) & 1, p.err, ERR_WAIT_FULL);
            if (ok) ok = mbar_wait(&sm.tfull[buf], (i >> 1) & 1, p.err, ERR_WAIT_FULL);
            if (!ok) break;
            tc_fence_after();
            if (nvalid > 0) {
                for (int blk = bp; blk < 4; blk += BS) {
                    const int b = (i & 3) * 4 + blk;
                    int s[16];
                    tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + buf * 256 + blk * kPN + 16 * tg, s);
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
                if ((i & 3) == 3 || i == nchunk - 1) mbar_arrive(&sm.sempty[sb]);
            }
        }
        // ---------------- phase partials ----------------
        // (the stage buffers are idle: every copy was consumed by an MMA whose
        // completion every epilogue warp has waited for)
        double *red = reinterpret_cast<double *>(&sm.a[0][0]);  // [16 warps][16 tokens][32 lanes]
        if (BS > 1) {
            if (bp > 0)
#pragma unroll
                for (int j = 0; j < 16; ++j) red[((warp - 2) * 16 + j) * 32 + lane] = acc[j];
            named_sync(1, kPEpiWarps * 32);
            if (bp == 0)
                for (int ph = 1; ph < BS; ++ph) {
                    const int we = (ph * TQ + tg) * 4 + ((warp - 2) & 3);  // epilogue warp of (q, tg, ph)
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[j] += red[(we * 16 + j) * 32 + lane];
                }
        }
        // ---------------- output ----------------
        const int row = rb * kPM + row_local;
        if (bp == 0 && nvalid > 0) {
            if (p.nsplit == 1) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + 16 * tg + j;
                    if (p.epi == EPI_SWIGLU) {
                        const double up = __shfl_down_sync(0xffffffffu, acc[j], 1);
                        if ((lane & 1) == 0 && j < nvalid)
                            p.y[(size_t)t * p.ldy + row / 2] = __fmul_rn(silu((float)acc[j]), (float)up);
                    } else if (j < nvalid) {
                        const float v = (float)acc[j];
                        p.y[(size_t)t * p.ldy + row] = p.res ? __fadd_rn(p.res[(size_t)t * p.ldres + row], v) : v;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + 16 * tg + j;
                    if (j < nvalid) p.part[((size_t)split * p.T + t) * p.R + row] = acc[j];
                }
            }
        }
    }
    if (p.nsplit > 1) {
        // last CTA of the (row block, token tile) adds the splits in order
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            int *c = p.counters + rb * gridDim.y + tt;
            sm.last = atomicAdd(c, 1) == p.nsplit - 1;
            if (sm.last) *c = 0;
        }
        __syncthreads();
        if (sm.last && warp >= 2) {
            __threadfence();
            // epilogue warp (q, g): rows 32q + lane, tokens 16g .. 16g + 15 of the tile
            const int q = warp & 3, g = (warp - 2) >> 2;
            const int row = rb * kPM + q * 32 + lane;
            for (int j = 0; j < 16; ++j) {
                const int t = t0 + 16 * g + j;
                double sum = 0.0;
                if (t < p.T)
                    for (int k = 0; k < p.nsplit; ++k) sum += __ldcg(p.part + ((size_t)k * p.T + t) * p.R + row);
                if (p.epi == EPI_SWIGLU) {
                    const double up = __shfl_down_sync(0xffffffffu, sum, 1);
                    if ((lane & 1) == 0 && t < p.T)
                        p.y[(size_t)t * p.ldy + row / 2] = __fmul_rn(silu((float)sum), (float)up);
                } else if (t < p.T) {
                    const float v = (float)sum;
                    p.y[(size_t)t * p.ldy + row] = p.res ? __fadd_rn(p.res[(size_t)t * p.ldres + row], v) : v;
                }
            }
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
// host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

cudaError_t prefill_setup() {
    if (!encode_fn()) return cudaErrorNotSupported;
    return cudaFuncSetAttribute(prefill_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(sizeof(PSmem) + 1024));
}

bool prefill_ok(const DevMat &w, int T) {
    return w.type == 8 && w.rows % kPM == 0 && w.cols % kTK == 0 && T >= 1;
}

cudaError_t launch_prefill_gemm(const PrefillArgs &a, cudaStream_t st) {
    const DevMat &w = *a.w;
    EncodeTiledFn enc = encode_fn();
    if (!enc || !prefill_ok(w, a.T) || !a.xq || !a.dx || !a.counters) return cudaErrorInvalidValue;
    const int R = w.rows, K = w.cols, NKT = K / kTK, RT = R / kTR;
    CUtensorMap wmap, xmap, dxmap;
    {
        const cuuint64_t dims[4] = {(cuuint64_t)kTK, (cuuint64_t)kTR, (cuuint64_t)NKT, (cuuint64_t)RT};
        const cuuint64_t strides[3] = {(cuuint64_t)kTK, (cuuint64_t)kTileBytes, (cuuint64_t)kTileBytes * NKT};
        const cuuint32_t box[4] = {(cuuint32_t)kPKC, (cuuint32_t)kTR, 1, 4};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w.w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)a.T};
        const cuuint64_t strides[1] = {(cuuint64_t)K};
        const cuuint32_t box[2] = {(cuuint32_t)kPKC, (cuuint32_t)kPN};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(a.xq), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(K / 32), (cuuint64_t)a.T};
        const cuuint64_t strides[1] = {(cuuint64_t)(K / 32) * 8};
        const cuuint32_t box[2] = {16, (cuuint32_t)kPN};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&dxmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(a.dx), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    const int RB = R / kPM, TT = (a.T + kPN - 1) / kPN;
    int nsplit = std::max(1, std::min(NKT, a.num_sms / std::max(1, RB * TT)));
    nsplit = std::min(nsplit, 8);
    if (nsplit > 1 && (!a.part || (size_t)nsplit * a.T * R > a.part_doubles)) nsplit = 1;
    PrefillParams p;
    p.R = R;
    p.K = K;
    p.T = a.T;
    p.nsplit = nsplit;
    p.epi = a.epi;
    p.y = a.y;
    p.ldy = a.ldy;
    p.res = a.res;
    p.ldres = a.ldres;
    p.part = a.part;
    p.counters = a.counters;
    p.wtiles = reinterpret_cast<const __half *>(w.w);
    p.err = a.err;
    count_launch();
    prefill_q8_kernel<<<dim3(RB, TT, nsplit), kPThreads, sizeof(PSmem) + 1024, st>>>(wmap, xmap, dxmap, p);
    return cudaGetLastError();
}

cudaError_t launch_quant_rows_q8(const float *x, int ldx, int T, int K, const float *norm_w, float eps, int8_t *xq,
                                 double *dx, float *act_out, cudaStream_t st) {
    if (K % 32 != 0 || T < 1 || ldx % 4 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0) return cudaErrorInvalidValue;
    count_launch();
    const int nch = (K / 32 + kQBlocks - 1) / kQBlocks;
    quant_rows_q8_kernel<<<dim3(T, nch), 256, 0, st>>>(x, ldx, K, norm_w, eps, xq, dx, act_out);
    return cudaGetLastError();
}

}  // namespace s2k
