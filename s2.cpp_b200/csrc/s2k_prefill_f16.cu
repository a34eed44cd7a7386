// s2k_prefill_f16.cu -- prompt prefill GEMMs on the tensor cores for F16
// models (tcgen05.mma kind::f16, fp32 accumulation in TMEM):
// Y[T][R] = X[T][K] . W[R][K]^T, the prompt / voice-clone prefill of
// eval_cached (src/s2_model.cpp:788-853) for fp16 weight tiles.
//
// Arithmetic.  The reference rounds the activation to fp16 for F16 weights
// (ggml's vec_dot_type), as this GEMM does; the tensor cores then add the
// exact fp16 x fp16 products in fp32 over the whole K range instead of the
// exact double sums of the GEMV kernels, so prefill logits agree with the CPU
// oracle to the floating-point tolerance (1e-2 * std), not bit for bit.
// Decode steps after the prefill run on the exact GEMV path.  (K-quant
// weights are not sent here: their reference arithmetic quantizes the
// activation to 8-bit Q8_K, and a 16-bit activation path moves the logits by
// ~8 % of their std -- outside the tolerance.)
//
// Structure (one CTA per SM, persistent over (128-row block, N-token tile)
// pairs, N = 64 or 256; the token tiles of one row block are consecutive, so
// the CTAs working at one time share few weight slabs and weights cross HBM
// about once):
//   warp 0     TMA producer: weight slabs (4-D tensor map over the 32 x 256
//              fp16 tile layout, 128 rows x 64 columns, 128-byte swizzle) and
//              activation slabs (N tokens x 64 columns) into a 4-stage ring;
//              the first stages' weights are requested before the previous
//              kernel has finished (programmatic dependent launch).  No
//              multicast loads.
//   warp 1     MMA issuer (one lane): four 128xNx16 MMAs per stage into one of
//              two TMEM accumulators (N columns each), commit per stage and per
//              tile.
//   warps 2..9 epilogue: warp w reads lane quarter w % 4 (32 weight rows) and
//              column half (w - 2) / 4 of the accumulator with
//              tcgen05.ld.32x32b.x32, then stores the rows (+ residual, or
//              SwiGLU of interleaved gate / up rows).
#include "s2k_common.cuh"
#include "s2k_kernels.h"
#include "s2k_tc.cuh"

#include <algorithm>
#include <cstdint>

namespace s2k {

constexpr int kFM = 128;            // weight rows per tile (MMA M)
constexpr int kFKC = 64;            // fp16 columns per stage (one 128-byte swizzle row)
constexpr int kFStages = 4;
constexpr int kFEpiWarps = 8;
constexpr int kFThreads = (2 + kFEpiWarps) * 32;
constexpr uint32_t kFStageA = kFM * kFKC * 2;  // 16 KB

template <int N>
struct FSmem {
    alignas(1024) uint8_t a[kFStages][kFStageA];
    alignas(1024) uint8_t b[kFStages][N * kFKC * 2];
    uint64_t full[kFStages], empty[kFStages];
    uint64_t tfull[2], tempty[2];
    uint32_t tmem_base;
};
static_assert(sizeof(FSmem<256>) + 1024 <= 227 * 1024, "f16 prefill shared memory");

// kind::f16: D f32, A and B fp16, both K-major, N columns, M = kFM
template <int N>
constexpr uint32_t idesc_f16() {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kFM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

struct F16Params {
    int R, K, T;
    int epi;
    float *y;
    int ldy;
    const float *res;
    int ldres;
    int *err;
};

template <int N>
__global__ void __launch_bounds__(kFThreads, 1)
    prefill_f16_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                       F16Params p) {
    extern __shared__ uint8_t fraw[];
    FSmem<N> &sm = *reinterpret_cast<FSmem<N> *>((reinterpret_cast<uintptr_t>(fraw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int RB = p.R / kFM, TT = (p.T + N - 1) / N, nk = p.K / kFKC;
    const int n_tiles = RB * TT;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < kFStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.tfull[i], 1);
            mbar_init(&sm.tempty[i], kFEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 1) {  // TMEM: two N-column accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                     "r"(2 * N)
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
            const int my_tiles = c < n_tiles ? (n_tiles - 1 - c) / G + 1 : 0;
            const int total = my_tiles * nk;
            const int pre = min(total, kFStages);
            // weights of the first stages before the previous kernel ends
            for (int it = 0; it < pre; ++it) {
                const int t = c + (it / nk) * G, kc = it % nk, rb = t / TT;
                mbar_arrive_expect_tx(&sm.full[it], kFStageA + N * kFKC * 2);
                tma_load_4d(sm.a[it], &wmap, (kc * kFKC) % kTKH, 0, (kc * kFKC) / kTKH, rb * 4, &sm.full[it]);
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it) {
                const int t = c + (it / nk) * G, kc = it % nk, tt = t % TT;
                tma_load_2d(sm.b[it], &xmap, kc * kFKC, tt * N, &sm.full[it]);
            }
            for (int it = pre; it < total && ok; ++it) {
                const int t = c + (it / nk) * G, kc = it % nk, rb = t / TT, tt = t % TT;
                const int st = it % kFStages;
                ok = mbar_wait(&sm.empty[st], ((it / kFStages) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                mbar_arrive_expect_tx(&sm.full[st], kFStageA + N * kFKC * 2);
                tma_load_4d(sm.a[st], &wmap, (kc * kFKC) % kTKH, 0, (kc * kFKC) / kTKH, rb * 4, &sm.full[st]);
                tma_load_2d(sm.b[st], &xmap, kc * kFKC, tt * N, &sm.full[st]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0, ti = 0;
            for (int t = c; t < n_tiles && ok; t += G, ++ti) {
                const int buf = ti & 1;
                if (ti >= 2) ok = mbar_wait(&sm.tempty[buf], ((ti >> 1) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                tc_fence_after();
                for (int kc = 0; kc < nk && ok; ++kc, ++it) {
                    const int st = it % kFStages;
                    ok = mbar_wait(&sm.full[st], (it / kFStages) & 1, p.err, ERR_WAIT_FULL);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int k4 = 0; k4 < 4; ++k4)
                        mma_f16(tmem + buf * N, sw128_desc(sm.a[st] + 32 * k4), sw128_desc(sm.b[st] + 32 * k4),
                                idesc_f16<N>(), (kc | k4) != 0);
                    mma_commit(&sm.empty[st]);
                }
                if (ok) mma_commit(&sm.tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        pdl_wait();
        const int e = warp - 2, q = warp & 3, half = e >> 2;
        int ti = 0;
        for (int t = c; t < n_tiles && ok; t += G, ++ti) {
            const int buf = ti & 1, rb = t / TT, tt = t % TT;
            ok = mbar_wait(&sm.tfull[buf], (ti >> 1) & 1, p.err, ERR_WAIT_FULL);
            if (!ok) break;
            tc_fence_after();
            const int row = rb * kFM + q * 32 + lane;
            for (int cc = 0; cc < N / 64; ++cc) {  // 32 columns (tokens) at a time
                const int col0 = half * (N / 2) + 32 * cc;
                const int t0 = tt * N + col0;
                if (t0 >= p.T) break;  // warp-uniform
                int v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * N + col0, v);
                const int n = min(32, p.T - t0);
                if (p.epi == EPI_SWIGLU) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float g = __int_as_float(v[j]);
                        const float up = __shfl_down_sync(0xffffffffu, g, 1);
                        if ((lane & 1) == 0 && j < n) p.y[(size_t)(t0 + j) * p.ldy + row / 2] = __fmul_rn(silu(g), up);
                    }
                } else {
#pragma unroll
                    for (int h8 = 0; h8 < 32; h8 += 8) {
                        float r[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            r[j] = (p.res && h8 + j < n) ? __ldcg(p.res + (size_t)(t0 + h8 + j) * p.ldres + row) : 0.f;
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (h8 + j < n) {
                                const float x = __int_as_float(v[h8 + j]);
                                p.y[(size_t)(t0 + h8 + j) * p.ldy + row] = p.res ? __fadd_rn(r[j], x) : x;
                            }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.tempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * N) : "memory");
    }
}

// ---------------------------------------------------------------------------
// activation rows -> fp16 [T][K] (after rms_norm_weighted when norm_w is
// given: the sum of squares in double, the scale in float, as the other
// prologues), grid (row, 32-block chunk)
// ---------------------------------------------------------------------------
constexpr int kHBlocks = 32;

__global__ void __launch_bounds__(256) rows_f16_kernel(const float *x, int ldx, int K, const float *norm_w, float eps,
                                                       __half *xh, float *act_out) {
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
    const int b0 = blockIdx.y * kHBlocks, b1 = min(K / 32, b0 + kHBlocks);
    for (int b = b0 + warp; b < b1; b += 8) {
        float v = __ldcg(row + b * 32 + lane);
        if (norm_w != nullptr) v = __fmul_rn(__fmul_rn(v, sc), __ldg(norm_w + b * 32 + lane));
        if (act_out != nullptr) act_out[(size_t)t * K + b * 32 + lane] = v;
        xh[(size_t)t * K + b * 32 + lane] = __float2half_rn(v);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
cudaError_t prefill_f16_setup() {
    if (!encode_fn()) return cudaErrorNotSupported;
    cudaError_t e = cudaFuncSetAttribute(prefill_f16_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(sizeof(FSmem<64>) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(prefill_f16_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(sizeof(FSmem<256>) + 1024));
    return e;
}

bool prefill_f16_ok(const DevMat &w, int T) {
    return tw_of(w.type) == TW_F16 && w.rows % kFM == 0 && w.cols % kTK == 0 && T >= 1;
}

cudaError_t launch_rows_f16(const float *x, int ldx, int T, int K, const float *norm_w, float eps, __half *xh,
                            float *act_out, cudaStream_t st) {
    if (K % 32 != 0 || T < 1 || ldx % 4 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T, (K / 32 + kHBlocks - 1) / kHBlocks);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, rows_f16_kernel, x, ldx, K, norm_w, eps, xh, act_out);
}

cudaError_t launch_prefill_f16_gemm(const uint8_t *wtiles, int R, int K, int T, const __half *xh, int epi, float *y,
                                    int ldy, const float *res, int ldres, int num_sms, int *err, cudaStream_t st) {
    EncodeTiledFn enc = encode_fn();
    if (!enc || R % kFM != 0 || K % kTK != 0 || T < 1 || !xh || !wtiles) return cudaErrorInvalidValue;
    const int N = T <= 64 ? 64 : 256;
    const int NKT = K / kTKH, RT = R / kTR;
    CUtensorMap wmap, xmap;
    {
        const cuuint64_t dims[4] = {(cuuint64_t)kTKH, (cuuint64_t)kTR, (cuuint64_t)NKT, (cuuint64_t)RT};
        const cuuint64_t strides[3] = {(cuuint64_t)kTKH * 2, (cuuint64_t)kTileBytesF16,
                                       (cuuint64_t)kTileBytesF16 * NKT};
        const cuuint32_t box[4] = {(cuuint32_t)kFKC, (cuuint32_t)kTR, 1, 4};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<uint8_t *>(wtiles), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
        const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kFKC, (cuuint32_t)N};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(xh), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    F16Params p;
    p.R = R;
    p.K = K;
    p.T = T;
    p.epi = epi;
    p.y = y;
    p.ldy = ldy;
    p.res = res;
    p.ldres = ldres;
    p.err = err;
    const int n_tiles = (R / kFM) * ((T + N - 1) / N);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(num_sms, n_tiles));
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = (N == 64 ? sizeof(FSmem<64>) : sizeof(FSmem<256>)) + 1024;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    if (N == 64) return cudaLaunchKernelEx(&cfg, prefill_f16_kernel<64>, wmap, xmap, p);
    return cudaLaunchKernelEx(&cfg, prefill_f16_kernel<256>, wmap, xmap, p);
}

}  // namespace s2k
