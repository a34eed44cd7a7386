// s2k_gemv.cu -- fused (RMSNorm | SwiGLU) + Q8_0 activation quantization +
// dequant-GEMV for batch-1..8 decode on sm_100a.
//
// Reference semantics (s2.cpp reaches these through ggml's CPU mat-vec):
//   mul_mat(W, x) with W Q8_0 quantizes each activation row to Q8_0 blocks
//   (ggml-cpu quantize_row_q8_0, x86 form) and computes, per output row,
//   sum_b (int sum_b) * (d_w * d_x)      (vec_dot_q8_0_q8_0)
//   The RMSNorm prologue restates rms_norm_weighted (src/s2_model.cpp:46-55);
//   the SwiGLU epilogue (rows interleaved gate/up) restates ggml_swiglu_split
//   (src/s2_model.cpp:1047), so W2 reads silu(gate)*up directly.
//
// Design (memory-bound: every weight byte is read once per pass):
//   * grid = one CTA per SM, each CTA owns a contiguous row range, so its
//     quants and scales are two contiguous runs in HBM;
//   * warp 8 streams S-row stages of that range into a 4-deep shared-memory
//     ring with cp.async.bulk (TMA bulk copy) completing on mbarriers, with
//     an L2 evict-first hint;
//   * the producer starts BEFORE griddepcontrol.wait: with programmatic
//     dependent launch the weights of this kernel stream while the previous
//     kernel is still finishing;
//   * warps 0-7 wait for the previous kernel, build the quantized activation
//     in shared memory, then compute with dp4a from shared memory; lane pairs
//     hold the two 16-byte halves of one 32-weight block so each block's
//     integer sum is exact before it is scaled, as in ggml.
//
// Arithmetic: each block term s_b * (d_w * d_x) is exact in double (s_b < 2^19,
// d_w * d_x is a product of two fp16 values, exact in float), the terms are
// summed in double and the row result is rounded to float once.  The result
// is therefore independent of the summation order, which is what lets the CPU
// oracle reproduce it bit for bit (a sum of the same exact terms in another
// order differs only below float resolution).
#include "s2k_common.cuh"
#include "s2k_kernels.h"

#include <algorithm>

namespace s2k {

constexpr int kNcw = 8;                    // consumer warps
constexpr int kThreads = (kNcw + 1) * 32;  // + producer warp
constexpr int kStages = 4;
constexpr int kStageBudget = 24 * 1024;
constexpr int kMaxMT = 8;
constexpr int kMaxK = 10240;  // input length limit (two 32-blocks per consumer thread at M = 1)
constexpr int kMaxRows = 64;  // residual rows a CTA prefetches (R / grid, rounded up)

struct GemvLayout {
    int S, WPR, BPL, stage_bytes;
    int off_xd, off_bar, off_red, off_res, off_nw, off_tok, off_ring, total;
};

// S rows per stage, WPR warps per row, BPL 32-weight blocks per lane per row slice.
__host__ __device__ inline GemvLayout gemv_layout(int K, int MT) {
    GemvLayout L;
    const int row_bytes = K + K / 16;  // int8 quants + fp16 scales
    int S = 8;
    while (S > 2 && S * row_bytes > kStageBudget) S >>= 1;
    L.S = S;
    L.WPR = kNcw / S;
    L.BPL = (K / 32 / L.WPR + 31) / 32;
    L.stage_bytes = (S * row_bytes + 127) & ~127;
    int off = MT * K;
    L.off_xd = (off + 15) & ~15;
    off = L.off_xd + MT * (K / 32) * 4;
    L.off_bar = (off + 15) & ~15;
    off = L.off_bar + 2 * kStages * 8 + 16;
    L.off_red = (off + 15) & ~15;
    off = L.off_red + 2 * kNcw * MT * 8;
    L.off_res = (off + 15) & ~15;
    off = L.off_res + MT * kMaxRows * 4;
    L.off_nw = (off + 15) & ~15;
    off = L.off_nw + K * 4;
    L.off_tok = (off + 15) & ~15;
    off = L.off_tok + kNcw * MT * 8 + MT * 4;
    L.off_ring = (off + 127) & ~127;
    L.total = L.off_ring + kStages * L.stage_bytes;
    return L;
}

// Dot of one 32-weight block (two 16-byte halves in shared memory) with a
// quantized activation block held in registers: exact int32.
__device__ __forceinline__ int dot_block(const int4 &w0, const int4 &w1, const int (&xb)[8]) {
    int s0 = dp4a(w0.x, xb[0], 0);
    int s1 = dp4a(w1.x, xb[4], 0);
    s0 = dp4a(w0.y, xb[1], s0);
    s1 = dp4a(w1.y, xb[5], s1);
    s0 = dp4a(w0.z, xb[2], s0);
    s1 = dp4a(w1.z, xb[6], s1);
    s0 = dp4a(w0.w, xb[3], s0);
    s1 = dp4a(w1.w, xb[7], s1);
    return s0 + s1;
}

template <int MT, int BPL>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_q8_0_kernel(const int8_t *__restrict__ wq, const __half *__restrict__ wd, int R, int K,
                     const float *x, int ldx, int M, int in_mode, const float *__restrict__ norm_w, float eps,
                     int epi, float *y, int ldy, const float *res, int ldres, float *act_out, const int *done,
                     int *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout L = gemv_layout(K, MT);
    int8_t *xq = reinterpret_cast<int8_t *>(smem);
    float *xd = reinterpret_cast<float *>(smem + L.off_xd);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kStages;
    volatile int *s_flags = reinterpret_cast<volatile int *>(empty + kStages);  // [0] abort, [1] cap
    double *rowpart = reinterpret_cast<double *>(smem + L.off_red);              // [2][kNcw][MT]
    float *s_res = reinterpret_cast<float *>(smem + L.off_res);                  // [MT][kMaxRows]
    float *s_nw = reinterpret_cast<float *>(smem + L.off_nw);                    // [K] RMSNorm weight
    double *s_tok = reinterpret_cast<double *>(smem + L.off_tok);                // [kNcw][MT]
    float *s_scale = reinterpret_cast<float *>(s_tok + kNcw * MT);               // [MT]
    uint8_t *ring = smem + L.off_ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NB = K >> 5;
    const int G = gridDim.x;
    // Row range of this CTA; whole (gate, up) pairs for the SwiGLU epilogue.
    const int unit = (epi == EPI_SWIGLU) ? 2 : 1;
    const int NU = R / unit;
    const int r0 = unit * (int)(((long long)NU * blockIdx.x) / G);
    const int r1 = unit * (int)(((long long)NU * (blockIdx.x + 1)) / G);
    const int S = L.S;
    const int ntiles = (r1 - r0 + S - 1) / S;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kNcw);
        }
        fence_mbar_init();
        s_flags[0] = 0;
        // A finished frame (done already visible) issues no weight traffic.
        const bool early = done != nullptr && *reinterpret_cast<const volatile int *>(done) != 0;
        s_flags[1] = early ? 0 : min(ntiles, kStages);
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kNcw) {  // ---------------- producer ----------------
        if (lane == 0 && s_flags[1] > 0) {
            const uint64_t pol = policy_evict_first();
            for (int t = 0; t < ntiles; ++t) {
                const int slot = t % kStages;
                if (t >= kStages) {
                    if (!mbar_wait(&empty[slot], ((t / kStages) - 1) & 1, err, ERR_WAIT_EMPTY)) break;
                    if (s_flags[0]) break;
                }
                const int rb = r0 + t * S;
                const int rows = min(S, r1 - rb);
                const uint32_t qb = (uint32_t)rows * (uint32_t)K;
                const uint32_t db = (uint32_t)rows * (uint32_t)(K / 16);
                uint8_t *st = ring + (size_t)slot * L.stage_bytes;
                mbar_arrive_expect_tx(&full[slot], qb + db);
                bulk_g2s(st, wq + (size_t)rb * K, qb, &full[slot], pol);
                bulk_g2s(st + (size_t)S * K, reinterpret_cast<const uint8_t *>(wd) + (size_t)rb * (K / 16), db,
                         &full[slot], pol);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int nct = kNcw * 32;
    // The norm weight is a model constant: stage it before waiting on the
    // previous kernel.
    if (in_mode == IN_RMSNORM)
        for (int i = tid; i < K / 4; i += nct)
            reinterpret_cast<float4 *>(s_nw)[i] = reinterpret_cast<const float4 *>(norm_w)[i];
    pdl_wait();
    const int cap = s_flags[1];
    const bool aborted = cap == 0 || (done != nullptr && *reinterpret_cast<const volatile int *>(done) != 0);
    if (aborted) {
        if (tid == 0) s_flags[0] = 1;
        named_sync(1, nct);
        for (int t = 0; t < cap; ++t) {
            const int slot = t % kStages;
            mbar_wait(&full[slot], (t / kStages) & 1, err, ERR_WAIT_FULL);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        return;
    }

    // residual rows of this CTA -> shared memory (their load overlaps the prologue)
    const int nrows = r1 - r0;
    if (res != nullptr)
        for (int i = tid; i < M * nrows; i += nct) {
            const int m = i / nrows, r = i - m * nrows;
            s_res[m * kMaxRows + r] = __ldcg(res + (size_t)m * ldres + r0 + r);
        }

    // prologue: activation -> Q8_0 in shared memory.  Each thread owns whole
    // 32-value blocks (item = token * NB + block), so a block's max, scale and
    // rounding need no cross-lane traffic and all blocks proceed in parallel.
    // When every thread holds at most one block (M = 1 at the model widths) the
    // values stay in registers between the norm's sum of squares and the
    // quantizer; otherwise (prefill) they are read again from L2.
    const int items = M * NB;
    const bool single = items <= nct;
    float4 v[8];
    if (in_mode == IN_RMSNORM) {
        double tok[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tok[m] = 0.0;
        for (int it = tid; it < items; it += nct) {
            const int m = it / NB, b = it - m * NB;
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)m * ldx + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + j);
            double s = 0.0;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                s += (double)__fmul_rn(v[j].x, v[j].x) + (double)__fmul_rn(v[j].y, v[j].y) +
                     (double)__fmul_rn(v[j].z, v[j].z) + (double)__fmul_rn(v[j].w, v[j].w);
#pragma unroll
            for (int mm = 0; mm < MT; ++mm)
                if (mm == m) tok[mm] += s;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < M) {
                const double t = warp_sum_d(tok[m]);
                if (lane == 0) s_tok[warp * MT + m] = t;
            }
        }
        named_sync(1, nct);
        if (tid < M) {
            double tot = 0.0;
            for (int w = 0; w < kNcw; ++w) tot += s_tok[w * MT + tid];
            const float mean = (float)(tot / (double)K);
            s_scale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
        named_sync(1, nct);
    }
    for (int it = tid; it < items; it += nct) {
        const int m = it / NB, b = it - m * NB;
        if (!(single && in_mode == IN_RMSNORM)) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)m * ldx + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + j);
        }
        if (in_mode == IN_RMSNORM) {
            const float sc = s_scale[m];
            const float4 *nw = reinterpret_cast<const float4 *>(s_nw + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 w4 = nw[j];
                v[j].x = __fmul_rn(__fmul_rn(v[j].x, sc), w4.x);
                v[j].y = __fmul_rn(__fmul_rn(v[j].y, sc), w4.y);
                v[j].z = __fmul_rn(__fmul_rn(v[j].z, sc), w4.z);
                v[j].w = __fmul_rn(__fmul_rn(v[j].w, sc), w4.w);
            }
        }
        if (act_out != nullptr && blockIdx.x == 0) {
            float4 *dst = reinterpret_cast<float4 *>(act_out + (size_t)m * K + b * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = v[j];
        }
        // ggml-cpu x86 quantize_row_q8_0: d = amax/127 (fp16), q = rint(x * 127/amax)
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
        int4 *dq = reinterpret_cast<int4 *>(xq + m * K + b * 32);
        dq[0] = make_int4(pk[0], pk[1], pk[2], pk[3]);
        dq[1] = make_int4(pk[4], pk[5], pk[6], pk[7]);
        xd[m * NB + b] = __half2float(__float2half_rn(d));
    }
    named_sync(1, nct);

    // Lane mapping: warp -> (row in stage, K slice); lane -> the blocks
    // slice*BPS + lane + 32*k (k < BPL) of that row.  The lane's activation
    // blocks are the same for every row, so they are loaded once.
    const int WPR = L.WPR;
    const int row_local = warp / WPR, slice = warp - row_local * WPR;
    const int BPS = NB / WPR;  // blocks per slice
    int blk[BPL];
    bool bv[BPL];
#pragma unroll
    for (int k = 0; k < BPL; ++k) {
        const int bi = lane + 32 * k;
        bv[k] = bi < BPS;
        blk[k] = slice * BPS + (bv[k] ? bi : 0);
    }
    constexpr bool kRegX = MT <= 2;
    int xr[kRegX ? MT : 1][BPL][8];
    float xs[kRegX ? MT : 1][BPL];
    if constexpr (kRegX) {
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int k = 0; k < BPL; ++k) {
                const int4 *xp = reinterpret_cast<const int4 *>(xq + m * K + blk[k] * 32);
                const int4 a = xp[0], b = xp[1];
                xr[m][k][0] = a.x; xr[m][k][1] = a.y; xr[m][k][2] = a.z; xr[m][k][3] = a.w;
                xr[m][k][4] = b.x; xr[m][k][5] = b.y; xr[m][k][6] = b.z; xr[m][k][7] = b.w;
                xs[m][k] = xd[m * NB + blk[k]];
            }
    }

    bool broken = false;
    for (int t = 0; t < ntiles; ++t) {
        const int slot = t % kStages;
        const int rb = r0 + t * S;
        const int rows = min(S, r1 - rb);
        if (!broken && !mbar_wait(&full[slot], (t / kStages) & 1, err, ERR_WAIT_FULL)) broken = true;
        const int8_t *sq = reinterpret_cast<const int8_t *>(ring + (size_t)slot * L.stage_bytes);
        const __half *sd = reinterpret_cast<const __half *>(sq + (size_t)S * K);
        double acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.0;
        if (!broken && row_local < rows) {
            const int8_t *wrow = sq + (size_t)row_local * K;
            const __half *drow = sd + (size_t)row_local * NB;
            int4 w0[BPL], w1[BPL];
            float dw[BPL];
#pragma unroll
            for (int k = 0; k < BPL; ++k) {
                const int4 *wp = reinterpret_cast<const int4 *>(wrow + blk[k] * 32);
                w0[k] = wp[0];
                w1[k] = wp[1];
                dw[k] = __half2float(drow[blk[k]]);
            }
#pragma unroll
            for (int k = 0; k < BPL; ++k) {
                if (bv[k]) {
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < M) {
                            if constexpr (kRegX) {
                                const int s = dot_block(w0[k], w1[k], xr[m][k]);
                                acc[m] += (double)s * (double)(dw[k] * xs[m][k]);
                            } else {
                                const int4 *xp = reinterpret_cast<const int4 *>(xq + m * K + blk[k] * 32);
                                const int4 a = xp[0], b = xp[1];
                                const int xb[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                                const int s = dot_block(w0[k], w1[k], xb);
                                acc[m] += (double)s * (double)(dw[k] * xd[m * NB + blk[k]]);
                            }
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = warp_sum_d(acc[m]);
        // stage epilogue through shared memory (double-buffered by stage parity)
        double *rp = rowpart + (t & 1) * kNcw * MT;
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < MT; ++m) rp[warp * MT + m] = acc[m];
        }
        named_sync(2, nct);
        if (!broken) {
            const int items = (rows / unit) * M;
            for (int it = tid; it < items; it += nct) {
                const int u = it / M, m = it - u * M;
                if (epi == EPI_SWIGLU) {
                    double g = rp[(2 * u) * WPR * MT + m], up = rp[(2 * u + 1) * WPR * MT + m];
                    for (int s2 = 1; s2 < WPR; ++s2) {
                        g += rp[((2 * u) * WPR + s2) * MT + m];
                        up += rp[((2 * u + 1) * WPR + s2) * MT + m];
                    }
                    y[(size_t)m * ldy + rb / 2 + u] = __fmul_rn(silu((float)g), (float)up);
                } else {
                    double a = rp[(u * WPR) * MT + m];
                    for (int s2 = 1; s2 < WPR; ++s2) a += rp[(u * WPR + s2) * MT + m];
                    const float v = (float)a;
                    const int r = rb + u;
                    y[(size_t)m * ldy + r] = res ? s_res[m * kMaxRows + (r - r0)] + v : v;
                }
            }
        }
    }
}

size_t DevMat::bytes() const {
    if (type == 8) return (size_t)rows * cols + (size_t)rows * (cols / 32) * 2;
    return 0;
}

static int g_gemv_smem_max = 0;

template <int MT, int BPL>
static cudaError_t set_attr() {
    return cudaFuncSetAttribute(gemv_q8_0_kernel<MT, BPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t gemv_setup() {
    cudaError_t e;
#define S2K_SET(MT)                                                         \
    if ((e = set_attr<MT, 1>()) || (e = set_attr<MT, 2>()) || (e = set_attr<MT, 3>()) || \
        (e = set_attr<MT, 4>()))                                            \
        return e;
    S2K_SET(1)
    S2K_SET(2)
    S2K_SET(4)
    S2K_SET(8)
#undef S2K_SET
    g_gemv_smem_max = 227 * 1024;
    return cudaSuccess;
}

template <int MT, int BPL>
static cudaError_t launch_one(const GemvArgs &a, int m0, int M, int grid, cudaStream_t st) {
    const DevMat &w = *a.w;
    const GemvLayout L = gemv_layout(w.cols, MT);
    if (L.total > g_gemv_smem_max) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    const float *x = a.x + (size_t)m0 * a.ldx;
    float *y = a.y + (size_t)m0 * a.ldy;
    const float *res = a.res ? a.res + (size_t)m0 * a.ldres : nullptr;
    float *act = a.act_out ? a.act_out + (size_t)m0 * w.cols : nullptr;
    return cudaLaunchKernelEx(&cfg, gemv_q8_0_kernel<MT, BPL>, (const int8_t *)w.q, (const __half *)w.d, w.rows,
                              w.cols, x, a.ldx, M, a.in_mode, a.norm_w, a.eps, a.epi, y, a.ldy, res, a.ldres, act,
                              a.done, a.err);
}

template <int MT>
static cudaError_t launch_bpl(const GemvArgs &a, int m0, int M, int grid, cudaStream_t st) {
    switch (gemv_layout(a.w->cols, MT).BPL) {
    case 1: return launch_one<MT, 1>(a, m0, M, grid, st);
    case 2: return launch_one<MT, 2>(a, m0, M, grid, st);
    case 3: return launch_one<MT, 3>(a, m0, M, grid, st);
    case 4: return launch_one<MT, 4>(a, m0, M, grid, st);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(const GemvArgs &a, int num_sms, cudaStream_t st) {
    const DevMat &w = *a.w;
    if (w.type != 8 || w.cols % 256 != 0 || w.cols > kMaxK || w.rows <= 0) return cudaErrorInvalidValue;
    if (a.epi == EPI_SWIGLU && (w.rows % 2 != 0 || a.res != nullptr)) return cudaErrorInvalidValue;
    const int grid = std::min(num_sms, a.epi == EPI_SWIGLU ? w.rows / 2 : w.rows);
    if (a.res != nullptr && (w.rows + grid - 1) / grid > kMaxRows) return cudaErrorInvalidValue;
    for (int m0 = 0; m0 < a.M; m0 += kMaxMT) {
        const int M = std::min(kMaxMT, a.M - m0);
        cudaError_t e;
        if (M == 1) e = launch_bpl<1>(a, m0, M, grid, st);
        else if (M == 2) e = launch_bpl<2>(a, m0, M, grid, st);
        else if (M <= 4) e = launch_bpl<4>(a, m0, M, grid, st);
        else e = launch_bpl<8>(a, m0, M, grid, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------------------
// GGUF Q8_0 blocks -> split planes
// ---------------------------------------------------------------------------
__global__ void relayout_q8_0_kernel(const uint8_t *__restrict__ src, int rows, int cols, int8_t *__restrict__ q,
                                     __half *__restrict__ d, int row_stride, int row_offset) {
    const int nb = cols / 32;
    const long long total = (long long)rows * nb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
        const uint8_t *blk = src + i * 34;
        const long long dr = (long long)r * row_stride + row_offset;
        const unsigned short dbits = (unsigned short)(blk[0] | (blk[1] << 8));
        d[dr * nb + b] = __ushort_as_half(dbits);
        int8_t *qd = q + dr * cols + b * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) qd[j] = (int8_t)blk[2 + j];
    }
}

cudaError_t launch_relayout_q8_0(const uint8_t *src, int rows, int cols, DevMat *dst, int row_stride,
                                 int row_offset, cudaStream_t st) {
    const long long total = (long long)rows * (cols / 32);
    const int block = 256;
    const int grid = (int)std::min<long long>((total + block - 1) / block, 148 * 16);
    count_launch();
    relayout_q8_0_kernel<<<grid, block, 0, st>>>(src, rows, cols, dst->q, dst->d, row_stride, row_offset);
    return cudaGetLastError();
}

}  // namespace s2k
