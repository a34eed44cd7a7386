// s2k_gemv.cu -- fused (RMSNorm | SwiGLU) + Q8_0 activation quantization +
// dequant-GEMV for batch-1..8 decode on sm_100a.
//
// Reference semantics (s2.cpp reaches these through ggml's CPU mat-vec):
//   mul_mat(W, x) with W Q8_0 quantizes each activation row to Q8_0 blocks
//   (ggml-cpu quantize_row_q8_0, x86 form) and computes, per output row,
//   sum_b (int sum_b) * (d_w * d_x)      (vec_dot_q8_0_q8_0)
//   The prologue modes restate rms_norm_weighted (src/s2_model.cpp:46-55)
//   and ggml_swiglu_split (src/s2_model.cpp:1047).
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

struct GemvLayout {
    int S, WPR, stage_bytes;
    int off_xd, off_bar, off_red, off_ring, total;
};

__host__ __device__ inline GemvLayout gemv_layout(int K, int MT) {
    GemvLayout L;
    const int row_bytes = K + K / 16;  // int8 quants + fp16 scales
    int S = 8;
    while (S > 1 && S * row_bytes > kStageBudget) S >>= 1;
    L.S = S;
    L.WPR = kNcw / S;
    L.stage_bytes = (S * row_bytes + 127) & ~127;
    int off = MT * K;
    L.off_xd = (off + 15) & ~15;
    off = L.off_xd + MT * (K / 32) * 4;
    L.off_bar = (off + 15) & ~15;
    off = L.off_bar + 2 * kStages * 8 + 16;
    L.off_red = (off + 15) & ~15;
    off = L.off_red + 2 * kNcw * MT * 8 + kNcw * MT * 8 + MT * 4;
    L.off_ring = (off + 127) & ~127;
    L.total = L.off_ring + kStages * L.stage_bytes;
    return L;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_q8_0_kernel(const int8_t *__restrict__ wq, const __half *__restrict__ wd, int R, int K,
                     const float *x, int ldx, int M, int in_mode,
                     const float *__restrict__ norm_w, float eps, float *y, int ldy,
                     const float *res, int ldres, float *act_out,
                     const int *done, int *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout L = gemv_layout(K, MT);
    int8_t *xq = reinterpret_cast<int8_t *>(smem);
    float *xd = reinterpret_cast<float *>(smem + L.off_xd);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kStages;
    volatile int *s_flags = reinterpret_cast<volatile int *>(empty + kStages);  // [0] abort, [1] cap
    double *red = reinterpret_cast<double *>(smem + L.off_red);                  // [2][kNcw][MT]
    double *nred = red + 2 * kNcw * MT;                                          // [kNcw][MT]
    float *s_scale = reinterpret_cast<float *>(nred + kNcw * MT);                // [MT]
    uint8_t *ring = smem + L.off_ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NB = K >> 5;
    const int G = gridDim.x;
    const int r0 = (int)(((long long)R * blockIdx.x) / G);
    const int r1 = (int)(((long long)R * (blockIdx.x + 1)) / G);
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

    // prologue: activation -> Q8_0 in shared memory
    if (in_mode == IN_RMSNORM) {
        for (int m = 0; m < M; ++m) {
            double s = 0.0;
            for (int i = tid; i < K; i += nct) {
                const float v = __ldcg(x + (size_t)m * ldx + i);
                s += (double)__fmul_rn(v, v);
            }
            s = warp_sum_d(s);
            if (lane == 0) nred[warp * MT + m] = s;
        }
        named_sync(1, nct);
        if (tid < M) {
            double tot = 0.0;
            for (int w = 0; w < kNcw; ++w) tot += nred[w * MT + tid];
            const float mean = (float)(tot / (double)K);
            s_scale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
        named_sync(1, nct);
    }
    for (int item = warp; item < M * NB; item += kNcw) {
        const int m = item / NB, b = item - m * NB;
        const int i = b * 32 + lane;
        float v;
        if (in_mode == IN_SWIGLU) {
            const float g = __ldcg(x + (size_t)m * ldx + 2 * i), u = __ldcg(x + (size_t)m * ldx + 2 * i + 1);
            v = __fmul_rn(silu(g), u);
        } else {
            v = __ldcg(x + (size_t)m * ldx + i);
            if (in_mode == IN_RMSNORM) v = __fmul_rn(__fmul_rn(v, s_scale[m]), norm_w[i]);
        }
        if (act_out != nullptr && blockIdx.x == 0) act_out[(size_t)m * K + i] = v;
        float d;
        const int q = quant_q8_0_lane(v, &d);
        xq[m * K + i] = (int8_t)q;
        if (lane == 0) xd[m * NB + b] = d;
    }
    named_sync(1, nct);

    // main loop over this CTA's stages
    const int WPR = L.WPR;
    const int row_local = warp / WPR, slice = warp - row_local * WPR;
    const int NC = K >> 4;  // 16-byte chunks per row
    const int cps = NC / WPR;
    const int c0 = slice * cps;
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
            for (int base = 0; base < cps; base += 32) {
                const int c = c0 + base + lane;
                const bool valid = base + lane < cps;
                int4 wv = make_int4(0, 0, 0, 0);
                float dw = 0.f;
                if (valid) {
                    wv = *reinterpret_cast<const int4 *>(wrow + c * 16);
                    dw = __half2float(drow[c >> 1]);
                }
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < M) {
                        int s = 0;
                        if (valid) {
                            const int4 xv = *reinterpret_cast<const int4 *>(xq + m * K + c * 16);
                            s = dp4a(wv.x, xv.x, 0);
                            s = dp4a(wv.y, xv.y, s);
                            s = dp4a(wv.z, xv.z, s);
                            s = dp4a(wv.w, xv.w, s);
                        }
                        s += __shfl_xor_sync(0xffffffffu, s, 1);
                        if (valid && !(lane & 1)) acc[m] += (double)s * (double)(dw * xd[m * NB + (c >> 1)]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = warp_sum_d(acc[m]);
        if (WPR == 1) {
            if (lane == 0 && row_local < rows && !broken) {
                const int r = rb + row_local;
                for (int m = 0; m < M; ++m) {
                    const float v = (float)acc[m];
                    y[(size_t)m * ldy + r] = res ? __ldcg(res + (size_t)m * ldres + r) + v : v;
                }
            }
        } else {
            double *rr = red + (t & 1) * kNcw * MT;
            if (lane == 0) {
#pragma unroll
                for (int m = 0; m < MT; ++m) rr[warp * MT + m] = acc[m];
            }
            named_sync(2, nct);
            if (slice == 0 && lane == 0 && row_local < rows && !broken) {
                const int r = rb + row_local;
                for (int m = 0; m < M; ++m) {
                    double a = rr[(row_local * WPR) * MT + m];
                    for (int s2 = 1; s2 < WPR; ++s2) a += rr[(row_local * WPR + s2) * MT + m];
                    const float v = (float)a;
                    y[(size_t)m * ldy + r] = res ? __ldcg(res + (size_t)m * ldres + r) + v : v;
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

cudaError_t gemv_setup() {
    // Largest layout: K = 16384, MT = 8 (well above this model family).
    const int mx = 227 * 1024;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_q8_0_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx))) return e;
    if ((e = cudaFuncSetAttribute(gemv_q8_0_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx))) return e;
    if ((e = cudaFuncSetAttribute(gemv_q8_0_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx))) return e;
    if ((e = cudaFuncSetAttribute(gemv_q8_0_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx))) return e;
    g_gemv_smem_max = mx;
    return cudaSuccess;
}

template <int MT>
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
    return cudaLaunchKernelEx(&cfg, gemv_q8_0_kernel<MT>, (const int8_t *)w.q, (const __half *)w.d, w.rows, w.cols,
                              x, a.ldx, M, a.in_mode, a.norm_w, a.eps, y, a.ldy, res, a.ldres, act, a.done, a.err);
}

cudaError_t launch_gemv(const GemvArgs &a, int num_sms, cudaStream_t st) {
    const DevMat &w = *a.w;
    if (w.type != 8 || w.cols % 256 != 0 || w.rows <= 0) return cudaErrorInvalidValue;
    const int grid = std::min(num_sms, w.rows);
    for (int m0 = 0; m0 < a.M; m0 += kMaxMT) {
        const int M = std::min(kMaxMT, a.M - m0);
        cudaError_t e;
        if (M == 1) e = launch_one<1>(a, m0, M, grid, st);
        else if (M == 2) e = launch_one<2>(a, m0, M, grid, st);
        else if (M <= 4) e = launch_one<4>(a, m0, M, grid, st);
        else e = launch_one<8>(a, m0, M, grid, st);
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
