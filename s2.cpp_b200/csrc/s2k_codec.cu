// s2k_codec.cu -- codec decode on the GPU: RVQ codes -> PCM.
//
// Reference: AudioCodec::decode (src/s2_codec.cpp:1297-1447) and the graph it
// builds: build_decode_codes_stage_backend / build_vq_decode_stage (:620-678),
// build_transformer (:288-377, window mask :264-286), build_quantizer_decode_stage
// / build_quantizer_stage_up / build_convnext_block (:393-478), build_decoder /
// build_decoder_block / build_residual_unit (:379-391, :480-522), and the
// snake / causal conv / causal transposed conv helpers (:183-248).  The
// windowed callers are decode_codes_windowed (src/s2_pipeline.cpp:198-289) and
// Pipeline::synthesize_stream's decode_window_and_emit (:1011-1115).
//
// Arithmetic follows the reference's ggml graph: matrix products with F16
// weights take fp16-rounded activations (ggml's vec_dot_type), ggml_conv_1d /
// ggml_conv_1d_dw run through an fp16 im2col (input and weight rounded to
// fp16), the transposed convolutions cast weight and input to F32.  Here every
// convolution and matrix product is a tcgen05 kind::f16 GEMM with f32
// accumulation in TMEM; the transposed convolutions feed the tensor cores the
// f32 input as an exact fp16 pair (hi = fp16(x), lo = fp16(x - hi)) against the
// (fp16-exact) weight twice, which keeps ~22 bits of the input.  Reductions of
// the small kernels (norms, attention, VQ projection) sum in double.  Audio
// agrees with the CPU oracle to a floating-point tolerance.
//
// Data layout: activations are [time][channel] row-major (ggml's ne order:
// channels contiguous).  A convolution with K taps and dilation d is a GEMM
// over K x C columns whose A tile for tap k is the activation tile shifted by
// k*d - (K-1)*d rows (TMA zero-fills the rows before the window start: the
// causal left padding).  A transposed convolution with stride s and K = m*s
// taps is a GEMM with N = s x Cout columns whose row j holds output rows
// j*s .. j*s+s-1 (so the [L][s*Cout] result is the [L*s][Cout] output), tap q
// reading input row j - q.
//
// Kernels (per decode): vq_decode, per transformer layer rmsnorm -> GEMM(wqkv)
// -> rope -> attention -> GEMM(wo, +gamma*residual) -> rmsnorm -> GEMM(w1|w3,
// SwiGLU) -> GEMM(w2, +gamma*residual); final rmsnorm; per upsample stage
// GEMM(convT) -> dwconv+layernorm -> GEMM(pwconv1, GELU) -> GEMM(pwconv2,
// +gamma*residual); decoder conv; per decoder block GEMM(convT) and per
// residual unit GEMM(conv K=7) -> GEMM(conv K=1, +residual), snake fused into
// the epilogue that produces each convolution's input; output conv + tanh.
#include "../../include/s2k.h"
#include "s2k_model.h"
#include "s2k_tc.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace s2k {
namespace codec {

// ---------------------------------------------------------------------------
// tensor-core GEMM: Y[M][N] = sum over taps t, columns c of
//   A[m + shift0 + t*dshift][c] * B[n][t*kp + c],  fused epilogue
// ---------------------------------------------------------------------------
constexpr int kCM = 128;  // A rows (time) per tile = MMA M
constexpr int kCK = 64;   // fp16 columns per stage (one 128-byte swizzle row)
constexpr int kCEpiWarps = 16;  // 4 per TMEM lane quarter: enough warps in flight to hide L2 latency
constexpr int kCThreads = (2 + kCEpiWarps) * 32;
constexpr uint32_t kCStageA = kCM * kCK * 2;  // 16 KB
constexpr int kScr = 17;  // floats per scratch row (odd: conflict-free row-per-lane reads)

template <int BN>
struct CCfg {
    static constexpr uint32_t kStageB = BN * kCK * 2;
    static constexpr int kFit = (int)((184u * 1024u) / (kCStageA + kStageB));
    static constexpr int kStages = kFit < 8 ? kFit : 8;
    static constexpr uint32_t kAlloc = 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
};

template <int BN>
struct CSmem {
    alignas(1024) uint8_t a[CCfg<BN>::kStages][kCStageA];
    alignas(1024) uint8_t b[CCfg<BN>::kStages][CCfg<BN>::kStageB];
    uint64_t full[CCfg<BN>::kStages], empty[CCfg<BN>::kStages];
    float scratch[kCEpiWarps][32 * kScr];  // per epilogue warp: row <-> coalesced transposes
    uint64_t tfull[2], tempty[2], mdone;
    uint32_t tmem_base;
};

enum : int { ACT_NONE = 0, ACT_GELU = 1, ACT_SWIGLU = 2 };
// 16-bit output of the epilogue: none, fp16(y), fp16(snake(y)), the exact
// pair (hi, lo) of y, or of snake(y)
enum : int { O16_NONE = 0, O16_PLAIN = 1, O16_SNAKE = 2, O16_HILO = 3, O16_SNAKE_HILO = 4 };

// The epilogue of a launch as compile-time features (one kernel per
// combination the decode uses: a small, branch-free epilogue per launch)
enum : int { F_BIAS = 1, F_GAMMA = 2, F_RES = 4, F_Y32 = 8, F_GELU = 16, F_SWIGLU = 32 };
constexpr int f_o16(int o16) { return o16 << 6; }
template <int F>
struct EpiF {
    static constexpr bool bias = (F & F_BIAS) != 0, gamma = (F & F_GAMMA) != 0, res = (F & F_RES) != 0,
                          y32 = (F & F_Y32) != 0, gelu = (F & F_GELU) != 0, swiglu = (F & F_SWIGLU) != 0;
    static constexpr int o16 = (F >> 6) & 7;
    static constexpr bool snake = o16 == O16_SNAKE || o16 == O16_SNAKE_HILO;
    static constexpr bool hilo = o16 == O16_HILO || o16 == O16_SNAKE_HILO;
};

struct CGemm {
    int M, N;            // output rows (time), columns
    int kchunks, kp;     // 64-column chunks of A per tap; B columns per tap
    int ksteps_last;     // 16-column MMA steps with data in a tap's last chunk
    int taps, shift0, dshift;
    int cout;            // period of the per-channel vectors (bias, gamma, alpha)
    const float *bias, *gamma, *alpha;
    int act;
    const float *res;    // [M][ldres] f32 residual (may alias y32)
    int ldres;
    float *y32;
    int ldy32;
    __half *y16;
    int ldy16, o16, lo_off;  // lo half of a pair at y16 + lo_off
    int *err;
};

template <int BN>
constexpr uint32_t idesc_f16() {
    return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kCM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// Bounded wait that ignores the error word: used on the way out of a kernel
// that gave up, for copies / MMAs it issued that may still land.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity, const int *err) {
    const long long t0 = clock64(), lim = wait_limit(err);
    while (!mbar_test(bar, parity))
        if (clock64() - t0 > lim) return;
}

// snake (src/s2_codec.cpp:197-204): x + sin(alpha x)^2 / alpha
__device__ __forceinline__ float snake_f(float x, float a) {
    const float s = det_sinf(__fmul_rn(a, x));
    return __fadd_rn(x, __fdiv_rn(__fmul_rn(s, s), a));
}

// ggml_gelu_erf: 0.5 x (1 + erf(x / sqrt(2)))
__device__ __forceinline__ float gelu_erf_f(float x) {
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752440f))));
}

__device__ __forceinline__ void store_h16(__half *dst, const float (&z)[16]) {
    __half2 h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __floats2half2_rn(z[2 * i], z[2 * i + 1]);
    const uint4 *s = reinterpret_cast<const uint4 *>(h);
    reinterpret_cast<uint4 *>(dst)[0] = s[0];
    reinterpret_cast<uint4 *>(dst)[1] = s[1];
}

// The epilogue works on chunks of 32 rows (one per lane: the TMEM lane
// quarter of the warp) x 16 columns.  Global loads and stores of a chunk go
// through the warp's scratch so that they are coalesced: lane l moves row
// l/4 + 8i, 16-byte piece l%4 (fp32), or row l/2 + 16i, piece l%2 (fp16).

// residual of a chunk, coalesced layout (issued one chunk ahead)
__device__ __forceinline__ void load_res_chunk(const CGemm &p, int row0, int n0, float4 (&r)[4]) {
    if (!p.res || n0 >= p.N) return;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rr = row0 + lane / 4 + 8 * i;
        if (rr < p.M) r[i] = __ldcg(reinterpret_cast<const float4 *>(p.res + (size_t)rr * p.ldres + n0) + (lane & 3));
    }
}

// coalesced layout -> this lane's row
__device__ __forceinline__ void rows_from_coal(const float4 (&r)[4], float *scr, float (&out)[16]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float *d = scr + (lane / 4 + 8 * i) * kScr + 4 * (lane & 3);
        d[0] = r[i].x;
        d[1] = r[i].y;
        d[2] = r[i].z;
        d[3] = r[i].w;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 16; ++j) out[j] = scr[lane * kScr + j];
    __syncwarp();
}

// this lane's row of fp32 -> coalesced stores
__device__ __forceinline__ void store_chunk32(const float (&y)[16], float *scr, float *dst, int ld, int row0, int M,
                                              int n0) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 16; ++j) scr[lane * kScr + j] = y[j];
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rr = lane / 4 + 8 * i;
        const float *sr = scr + rr * kScr + 4 * (lane & 3);
        if (row0 + rr < M)
            reinterpret_cast<float4 *>(dst + (size_t)(row0 + rr) * ld + n0)[lane & 3] = make_float4(sr[0], sr[1], sr[2], sr[3]);
    }
    __syncwarp();
}

// this lane's row rounded to fp16 -> coalesced stores (two lanes per row)
__device__ __forceinline__ void store_chunk16(const float (&z)[16], float *scr, __half *dst, int ld, int row0, int M,
                                              int n0) {
    const int lane = threadIdx.x & 31;
    uint32_t *s32 = reinterpret_cast<uint32_t *>(scr);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __half2 h = __floats2half2_rn(z[2 * i], z[2 * i + 1]);
        s32[lane * kScr + i] = *reinterpret_cast<const uint32_t *>(&h);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int rr = lane / 2 + 16 * i, part = lane & 1;
        const uint32_t *sr = s32 + rr * kScr + 4 * part;
        if (row0 + rr < M)
            reinterpret_cast<uint4 *>(dst + (size_t)(row0 + rr) * ld + n0)[part] = make_uint4(sr[0], sr[1], sr[2], sr[3]);
    }
    __syncwarp();
}

// per-channel vectors of a chunk (loaded before the accumulator is read)
template <int F>
struct ChunkVecs {
    float bias[EpiF<F>::bias ? 16 : 1], gamma[EpiF<F>::gamma ? 16 : 1], alpha[EpiF<F>::snake ? 16 : 1];
};

template <int F>
__device__ __forceinline__ void load_vecs(const CGemm &p, int ch, ChunkVecs<F> &cv) {
    using E = EpiF<F>;
    if constexpr (E::bias) {
#pragma unroll
        for (int j = 0; j < 16; ++j) cv.bias[j] = __ldg(p.bias + ch + j);
    }
    if constexpr (E::gamma) {
#pragma unroll
        for (int j = 0; j < 16; ++j) cv.gamma[j] = __ldg(p.gamma + ch + j);
    }
    if constexpr (E::snake) {
#pragma unroll
        for (int j = 0; j < 16; ++j) cv.alpha[j] = __ldg(p.alpha + ch + j);
    }
}

// 16 accumulator columns n0..n0+15 of the warp's 32 rows from row0 (this
// lane: row0 + lane); r: the chunk's residual in the coalesced layout
template <int F>
__device__ __forceinline__ void epilogue16(const CGemm &p, int row0, int n0, const int (&v)[16], const float4 (&r)[4],
                                           const ChunkVecs<F> &cv, float *scr) {
    using E = EpiF<F>;
    const int lane = threadIdx.x & 31, t = row0 + lane;
    if constexpr (E::swiglu) {  // columns: 8 gates then the 8 matching ups
        if (t >= p.M) return;
        __half2 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float o0 = __fmul_rn(silu(__int_as_float(v[2 * i])), __int_as_float(v[8 + 2 * i]));
            const float o1 = __fmul_rn(silu(__int_as_float(v[2 * i + 1])), __int_as_float(v[8 + 2 * i + 1]));
            h[i] = __floats2half2_rn(o0, o1);
        }
        *reinterpret_cast<uint4 *>(p.y16 + (size_t)t * p.ldy16 + n0 / 2) = *reinterpret_cast<const uint4 *>(h);
    } else {
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] = __int_as_float(v[j]);
        if constexpr (E::bias) {
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = __fadd_rn(y[j], cv.bias[j]);
        }
        if constexpr (E::gelu) {
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = gelu_erf_f(y[j]);
        }
        if constexpr (E::gamma) {
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = __fmul_rn(y[j], cv.gamma[j]);
        }
        if constexpr (E::res) {
            float rr[16];
            rows_from_coal(r, scr, rr);
#pragma unroll
            for (int j = 0; j < 16; ++j) y[j] = __fadd_rn(rr[j], y[j]);
        }
        if constexpr (E::y32) store_chunk32(y, scr, p.y32, p.ldy32, row0, p.M, n0);
        if constexpr (E::o16 != O16_NONE) {
            if constexpr (E::snake) {
#pragma unroll
                for (int j = 0; j < 16; ++j) y[j] = snake_f(y[j], cv.alpha[j]);
            }
            store_chunk16(y, scr, p.y16, p.ldy16, row0, p.M, n0);
            if constexpr (E::hilo) {
#pragma unroll
                for (int j = 0; j < 16; ++j) y[j] = __fsub_rn(y[j], __half2float(__float2half_rn(y[j])));
                store_chunk16(y, scr, p.y16 + p.lo_off, p.ldy16, row0, p.M, n0);
            }
        }
    }
}

template <int BN, int F>
__global__ void __launch_bounds__(kCThreads, 1)
    codec_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, CGemm p) {
    constexpr int S = CCfg<BN>::kStages;
    constexpr uint32_t kTx = kCStageA + CCfg<BN>::kStageB;
    extern __shared__ uint8_t craw[];
    CSmem<BN> &sm = *reinterpret_cast<CSmem<BN> *>((reinterpret_cast<uintptr_t>(craw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int MT = (p.M + kCM - 1) / kCM, NT = (p.N + BN - 1) / BN;
    const int n_tiles = MT * NT, nk = p.taps * p.kchunks;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.tfull[i], 1);
            mbar_init(&sm.tempty[i], kCEpiWarps);
        }
        mbar_init(&sm.mdone, 1);
        fence_mbar_init();
    }
    if (warp == 1) {  // TMEM: two BN-column accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                     "r"(CCfg<BN>::kAlloc)
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
            const int pre = min(total, S);
            auto coords = [&](int it, int &ax, int &ay, int &bx, int &by) {
                const int t = c + (it / nk) * G, kk = it % nk, tap = kk / p.kchunks, kc = kk - tap * p.kchunks;
                const int mb = t / NT, nb = t - mb * NT;
                ax = kc * kCK;
                ay = mb * kCM + p.shift0 + tap * p.dshift;
                bx = tap * p.kp + kc * kCK;
                by = nb * BN;
            };
            int ax, ay, bx, by;
            // weights of the first stages before the previous kernel ends
            for (int it = 0; it < pre; ++it) {
                coords(it, ax, ay, bx, by);
                mbar_arrive_expect_tx(&sm.full[it], kTx);
                tma_load_2d(sm.b[it], &bmap, bx, by, &sm.full[it]);
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it) {
                coords(it, ax, ay, bx, by);
                tma_load_2d(sm.a[it], &amap, ax, ay, &sm.full[it]);
            }
            int issued = pre;
            for (int it = pre; it < total && ok; ++it) {
                const int st = it % S;
                ok = mbar_wait(&sm.empty[st], ((it / S) - 1) & 1, p.err, ERR_WAIT_EMPTY);
                if (!ok) break;
                coords(it, ax, ay, bx, by);
                mbar_arrive_expect_tx(&sm.full[st], kTx);
                tma_load_2d(sm.b[st], &bmap, bx, by, &sm.full[st]);
                tma_load_2d(sm.a[st], &amap, ax, ay, &sm.full[st]);
                issued = it + 1;
            }
            if (!ok)  // copies still in flight land before the CTA leaves
                for (int it = max(0, issued - S); it < issued; ++it) mbar_drain(&sm.full[it % S], (it / S) & 1, p.err);
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
                for (int kk = 0; kk < nk && ok; ++kk, ++it) {
                    const int st = it % S;
                    ok = mbar_wait(&sm.full[st], (it / S) & 1, p.err, ERR_WAIT_FULL);
                    if (!ok) break;
                    tc_fence_after();
                    // a tap's last chunk may be part-filled (zero columns past the input width)
                    const int nsteps = (kk % p.kchunks) == p.kchunks - 1 ? p.ksteps_last : 4;
#pragma unroll
                    for (int k4 = 0; k4 < 4; ++k4)
                        if (k4 < nsteps)
                            mma_f16(tmem + buf * BN, sw128_desc(sm.a[st] + 32 * k4), sw128_desc(sm.b[st] + 32 * k4),
                                    idesc_f16<BN>(), (kk | k4) != 0);
                    mma_commit(&sm.empty[st]);
                }
                if (ok) mma_commit(&sm.tfull[buf]);
            }
            if (!ok) {  // MMAs issued so far finish before TMEM is released
                mma_commit(&sm.mdone);
                mbar_drain(&sm.mdone, 0, p.err);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        // warp quarter q = warp % 4 reads TMEM lanes 32q..32q+31 (rows);
        // the 4 warps of a quarter take the 16-column chunks round-robin.
        // Each chunk's residual is loaded before the accumulator is waited
        // for / read, one chunk ahead.
        pdl_wait();
        const int e = warp - 2, q = warp & 3, grp = e >> 2;
        constexpr int kChunks = BN / 16;
        int ti = 0;
        float4 rnext[4];
        float *scr = sm.scratch[e];
        auto first_chunk = [&](int t, int &row0, int &n0) {
            const int mb = t / NT, nb = t - mb * NT;
            row0 = mb * kCM + q * 32;
            n0 = nb * BN + grp * 16;
        };
        if (c < n_tiles && grp < kChunks) {
            int r0, n0;
            first_chunk(c, r0, n0);
            load_res_chunk(p, r0, n0, rnext);
        }
        for (int t = c; t < n_tiles && ok; t += G, ++ti) {
            const int buf = ti & 1, mb = t / NT, nb = t - mb * NT;
            ok = mbar_wait(&sm.tfull[buf], (ti >> 1) & 1, p.err, ERR_WAIT_FULL);
            if (!ok) break;
            tc_fence_after();
            const int row0 = mb * kCM + q * 32;
            for (int cc = grp; cc < kChunks; cc += 4) {
                const int n0 = nb * BN + cc * 16;
                float4 rcur[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) rcur[j] = rnext[j];
                // next chunk: this tile's, or the first of this CTA's next tile
                if (cc + 4 < kChunks) {
                    load_res_chunk(p, row0, n0 + 64, rnext);
                } else if (t + G < n_tiles) {
                    int r2, n2;
                    first_chunk(t + G, r2, n2);
                    load_res_chunk(p, r2, n2, rnext);
                }
                if (n0 >= p.N) continue;  // warp-uniform; the chain of loads ahead goes on
                ChunkVecs<F> cv;
                load_vecs<F>(p, n0 % p.cout, cv);  // cout % 16 == 0: no wrap inside the chunk
                int v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + cc * 16), v);
                if (row0 < p.M) epilogue16<F>(p, row0, n0, v, rcur, cv, scr);  // warp-uniform
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(CCfg<BN>::kAlloc)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// small kernels
// ---------------------------------------------------------------------------
constexpr int kMaxQ = 16;

struct VqParams {
    int nq, L, C, cd;
    const int *codes;  // [nq][L]
    int size[kMaxQ];   // codes are clamped into [0, size)
    const float *cb[kMaxQ], *ow[kMaxQ], *ob[kMaxQ];  // [size][cd], [C][cd], [C]
};

// x[t][o] = sum over quantizers q (in order) of out_proj_q(codebook_q[code]) + b_q
// (build_vq_decode_stage and the adds of build_decode_codes_stage_backend)
__global__ void __launch_bounds__(128) vq_decode_kernel(VqParams p, float *x) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    {
        const int o = blockIdx.y * blockDim.x + threadIdx.x;
        if (o >= p.C) return;
        float acc = 0.f;
        for (int q = 0; q < p.nq; ++q) {
            int code = p.codes[(size_t)q * p.L + t];
            code = code < 0 ? 0 : (code >= p.size[q] ? p.size[q] - 1 : code);
            const float *cbr = p.cb[q] + (size_t)code * p.cd;
            const float *w = p.ow[q] + (size_t)o * p.cd;
            double s = 0.0;
            for (int d = 0; d < p.cd; ++d) s += (double)__ldg(w + d) * (double)__ldg(cbr + d);
            const float v = __fadd_rn((float)s, __ldg(p.ob[q] + o));
            acc = q == 0 ? v : __fadd_rn(acc, v);
        }
        x[(size_t)t * p.C + o] = acc;
    }
}

__device__ __forceinline__ double block_sum_d(double v, double *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < nw; ++w) s += red[w];
    return s;
}

__device__ __forceinline__ float block_max_f(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = -INFINITY;
    for (int w = 0; w < nw; ++w) m = fmaxf(m, red[w]);
    return m;
}

// rms_norm_weighted_cl (src/s2_codec.cpp:183-187) of rows row0.. of x, into
// fp16 (the next product's rounding) or an exact fp16 pair [hi | lo]
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float *x, int C, const float *w, float eps, int row0,
                                                           __half *out, int ldo, int hilo) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double red[8];
    const int t = blockIdx.x;
    const float *row = x + (size_t)(row0 + t) * C;
    double s = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float v = row[c];
        s += (double)__fmul_rn(v, v);
    }
    s = block_sum_d(s, red);
    const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s / (double)C), eps)));
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float y = __fmul_rn(__fmul_rn(row[c], sc), __ldg(w + c));
        const __half h = __float2half_rn(y);
        out[(size_t)t * ldo + c] = h;
        if (hilo) out[(size_t)t * ldo + C + c] = __float2half_rn(__fsub_rn(y, __half2float(h)));
    }
}

// Attention of the post-module transformer for a tile of kAQ query rows of
// one head: RoPE (ggml_rope_ext mode 0: adjacent pairs, angle pos * ts^i with
// the angles and their cos / sin taken from a table built on the host by the
// same float recurrence) on q and k as they are staged in shared memory, then
// softmax(q.k / sqrt(hd)) over keys [max(0, t-W+1), t] (the window mask, or
// the causal mask when W <= 0) in the reference's order (all scores, their
// max, exp, the sum, the normalised weights), times V; fp16 out (the wo
// product's rounding).  GQA: head h reads kv head h / (H / Hk)
// (repeat_interleave_heads).  Dot products accumulate in f32.
constexpr int kAQ = 8;        // query rows per block
constexpr int kAKC = 64;      // key rows per staged chunk
constexpr int kAThreads = 256;
constexpr int kAMaxHd = 128;

// rows [r0, r0 + n) of one head of the fused qkv rows (column offset col),
// rotated pair by pair, into dst rows of stride hp; threads over (row, pair)
__device__ __forceinline__ void stage_rope(const float *qkv, int ld, int col, int r0, int n, const float2 *rope,
                                           int hd, float *dst, int hp) {
    const int half = hd / 2;
    for (int e = threadIdx.x; e < n * half; e += blockDim.x) {
        const int r = e / half, i = e - r * half;
        const float2 x = *reinterpret_cast<const float2 *>(qkv + (size_t)(r0 + r) * ld + col + 2 * i);
        const float2 cs = rope[(size_t)(r0 + r) * half + i];
        dst[r * hp + 2 * i] = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
        dst[r * hp + 2 * i + 1] = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    }
}

__global__ void __launch_bounds__(kAThreads) codec_attn_kernel(const float *qkv, int ld, int L, int H, int Hk, int hd,
                                                               int qs, int W, float scale, const float2 *rope,
                                                               __half *out, int ldo, int span) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float sh[];
    const int hp = hd + 1;               // padded rows: conflict-free column reads
    float *q = sh;                       // [kAQ][hp]
    float *kv = q + kAQ * hp;            // [kAKC][hp] (K, then V)
    float *sc = kv + kAKC * hp;          // [kAQ][span] scores / weights
    const int q0 = blockIdx.x * kAQ, h = blockIdx.y, kh = h / (H / Hk), tid = threadIdx.x;
    const int nq = min(kAQ, L - q0);
    const int kbeg = W > 0 ? max(0, q0 - W + 1) : 0, kend = q0 + nq;  // keys [kbeg, kend)
    const int ks = Hk * hd;
    stage_rope(qkv, ld, h * hd, q0, nq, rope, hd, q, hp);
    // scores
    for (int c0 = kbeg; c0 < kend; c0 += kAKC) {
        const int nk = min(kAKC, kend - c0);
        __syncthreads();
        stage_rope(qkv, ld, qs + kh * hd, c0, nk, rope, hd, kv, hp);
        __syncthreads();
        for (int e = tid; e < kAQ * kAKC; e += kAThreads) {
            const int qi = e / kAKC, kj = e % kAKC;
            if (qi >= nq || kj >= nk) continue;
            const int t = q0 + qi, key = c0 + kj;
            const int lo = W > 0 ? max(0, t - W + 1) : 0;
            float v = -INFINITY;
            if (key >= lo && key <= t) {
                float s = 0.f;
                for (int d = 0; d < hd; ++d) s = fmaf(q[qi * hp + d], kv[kj * hp + d], s);
                v = __fmul_rn(s, scale);
            }
            sc[qi * span + (key - kbeg)] = v;
        }
    }
    __syncthreads();
    // softmax per query row: one warp per row
    const int warp = tid >> 5, lane = tid & 31, nkeys = kend - kbeg;
    for (int qi = warp; qi < nq; qi += kAThreads / 32) {
        float *row = sc + qi * span;
        float mx = -INFINITY;
        for (int j = lane; j < nkeys; j += 32) mx = fmaxf(mx, row[j]);
        mx = warp_max(mx);
        double sum = 0.0;
        for (int j = lane; j < nkeys; j += 32) {
            const float e = row[j] == -INFINITY ? 0.f : det_expf(__fsub_rn(row[j], mx));
            row[j] = e;
            sum += (double)e;
        }
        sum = warp_sum_d(sum);
        const float inv = (float)(1.0 / sum);
        for (int j = lane; j < nkeys; j += 32) row[j] = __fmul_rn(row[j], inv);
    }
    // weights x V
    float acc[kAQ * kAMaxHd / kAThreads];
    const int per = (kAQ * hd + kAThreads - 1) / kAThreads;
#pragma unroll
    for (int i = 0; i < kAQ * kAMaxHd / kAThreads; ++i) acc[i] = 0.f;
    for (int c0 = kbeg; c0 < kend; c0 += kAKC) {
        const int nk = min(kAKC, kend - c0);
        __syncthreads();
        for (int e = tid; e < nk * hd; e += kAThreads) {
            const int r = e / hd, d = e % hd;
            kv[r * hp + d] = qkv[(size_t)(c0 + r) * ld + qs + ks + kh * hd + d];
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kAQ * kAMaxHd / kAThreads; ++i) {
            if (i >= per) break;
            const int e = tid + i * kAThreads, qi = e / hd, d = e % hd;
            if (qi >= nq) continue;
            const float *w = sc + qi * span + (c0 - kbeg);
            float a = acc[i];
            for (int j = 0; j < nk; ++j) a = fmaf(w[j], kv[j * hp + d], a);
            acc[i] = a;
        }
    }
#pragma unroll
    for (int i = 0; i < kAQ * kAMaxHd / kAThreads; ++i) {
        if (i >= per) break;
        const int e = tid + i * kAThreads, qi = e / hd, d = e % hd;
        if (qi < nq) out[(size_t)(q0 + qi) * ldo + h * hd + d] = __float2half_rn(acc[i]);
    }
}

// ConvNeXt front (src/s2_codec.cpp:393-411): causal depthwise conv (fp16
// im2col: fp16-rounded input and weight) + bias, then layer norm with affine,
// into fp16 (pwconv1's rounding)
__global__ void __launch_bounds__(256) dwconv_ln_kernel(const float *x, int C, const float *dw, int K,
                                                        const float *db, const float *lw, const float *lb, float eps,
                                                        __half *out) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float yrow[];
    __shared__ double red[8];
    const int t = blockIdx.x;
    double s1 = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        double s = 0.0;
        for (int k = 0; k < K; ++k) {
            const int src = t - (K - 1) + k;
            if (src >= 0)
                s += (double)__ldg(dw + (size_t)c * K + k) *
                     (double)__half2float(__float2half_rn(x[(size_t)src * C + c]));
        }
        const float y = __fadd_rn((float)s, __ldg(db + c));
        yrow[c] = y;
        s1 += (double)y;
    }
    s1 = block_sum_d(s1, red);
    const float mean = (float)(s1 / (double)C);
    double s2 = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float d = __fsub_rn(yrow[c], mean);
        yrow[c] = d;
        s2 += (double)d * (double)d;
    }
    s2 = block_sum_d(s2, red);
    const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(s2 / (double)C), eps)));
    for (int c = threadIdx.x; c < C; c += blockDim.x)
        out[(size_t)t * C + c] =
            __float2half_rn(__fadd_rn(__fmul_rn(__fmul_rn(yrow[c], sc), __ldg(lw + c)), __ldg(lb + c)));
}

// output conv (one channel out, K taps, input already snake'd and fp16) + tanh:
// the input rows of a block's samples staged in shared memory with an odd
// word stride (conflict-free half2 reads), the weights alongside
constexpr int kOutRows = 256;

__global__ void __launch_bounds__(kOutRows) codec_out_kernel(const __half *x, int L, int C, const float *w, int K,
                                                             float bias, float *audio) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float osm[];
    const int cs = C + 2;                           // halves per staged row (C % 2 == 0: odd word count)
    float *ws = osm;                                // [K][C]
    __half *tile = reinterpret_cast<__half *>(osm + K * C);  // (kOutRows + K - 1) x cs
    const int t0 = blockIdx.x * kOutRows, rows = kOutRows + K - 1;
    for (int e = threadIdx.x; e < K * C; e += blockDim.x) {
        const int k = e / C, i = e % C;
        ws[e] = w[(size_t)i * K + k];
    }
    for (int e = threadIdx.x; e < rows * (C / 2); e += blockDim.x) {
        const int r = e / (C / 2), i2 = e % (C / 2), src = t0 - (K - 1) + r;
        const __half2 v = (src >= 0 && src < L) ? reinterpret_cast<const __half2 *>(x + (size_t)src * C)[i2]
                                                : __floats2half2_rn(0.f, 0.f);
        reinterpret_cast<__half2 *>(tile + (size_t)r * cs)[i2] = v;
    }
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t >= L) return;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) {
        const __half2 *xr = reinterpret_cast<const __half2 *>(tile + (size_t)(threadIdx.x + k) * cs);
        const float *wk = ws + k * C;
        for (int i2 = 0; i2 < C / 2; ++i2) {
            const float2 v = __half22float2(xr[i2]);
            acc = fmaf(wk[2 * i2], v.x, acc);
            acc = fmaf(wk[2 * i2 + 1], v.y, acc);
        }
    }
    audio[t] = tanhf(__fadd_rn(acc, bias));
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct HostTensor {
    int type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    std::vector<uint8_t> bytes;
    int64_t numel() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
    float at(int64_t i) const {
        if (type == S2K_TYPE_F32) {
            float v;
            std::memcpy(&v, bytes.data() + 4 * i, 4);
            return v;
        }
        uint16_t h;
        std::memcpy(&h, bytes.data() + 2 * i, 2);
        return __half2float(*reinterpret_cast<const __half *>(&h));
    }
};

// a GEMM's B operand and per-column vectors
struct GW {
    __half *w = nullptr;  // [N][taps * kp]
    int N = 0, taps = 1, kp = 0, kin = 0;
    int shift0 = 0, dshift = 0;  // A row of tap k: m + shift0 + k * dshift
    int cout = 0;
    float *bias = nullptr;
};

struct CLayer {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *attn_gamma = nullptr, *ffn_gamma = nullptr;
    GW wqkv, wo, w13, w2;
};

struct UpStage {
    int factor = 1, C = 0, hid = 0, dwK = 0;
    GW convt;
    float *dw = nullptr, *dwb = nullptr, *lnw = nullptr, *lnb = nullptr, *gamma = nullptr;
    GW pw1, pw2;
};

struct ResUnit {
    float *a0 = nullptr, *a2 = nullptr;
    GW c1, c3;
};

struct DecBlock {
    int stride = 1, Cin = 0, Cout = 0;
    float *alpha = nullptr;
    GW convt;
    ResUnit ru[3];
};

float fp16_round(float x) { return __half2float(__float2half_rn(x)); }

}  // namespace codec
}  // namespace s2k

using namespace s2k::codec;

struct s2k_codec {
    int device = 0;
    s2k_codec_hparams hp{};
    cudaStream_t st = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    int num_sms = 148;
    int *d_err = nullptr;
    std::map<std::string, HostTensor> host;
    std::vector<void *> allocs;
    bool ready = false;
    // VQ
    int nq = 0, cd = 0, C0 = 0;
    int vq_size[kMaxQ] = {};
    float *vq_cb[kMaxQ] = {}, *vq_ow[kMaxQ] = {}, *vq_ob[kMaxQ] = {};
    // post-module transformer
    int dim = 0, H = 0, Hk = 0, hd = 0, ff = 0, qs = 0, kvs = 0, W = 0;
    float eps = 1e-5f, rope_ts = 1.f;
    std::vector<CLayer> layers;
    float *final_norm = nullptr;
    // upsample + decoder
    std::vector<UpStage> ups;
    GW dec0;
    std::vector<DecBlock> blocks;
    float *out_alpha = nullptr, *out_w = nullptr;
    int out_K = 0, out_C = 0;
    float out_b = 0.f;
    int spf = 0, history = 0, receptive = 0;
    // workspace (grown on demand)
    size_t ws_tr = 0, ws_dec = 0;
    int *d_codes = nullptr;
    float *X = nullptr, *QKV = nullptr, *P = nullptr, *audio = nullptr;
    float *rope = nullptr;  // [position][head_dim / 2] (cos, sin)
    __half *N16 = nullptr, *G16 = nullptr, *S16 = nullptr, *T16 = nullptr, *HLa = nullptr, *HLb = nullptr;
    std::vector<void *> ws_allocs;
};

namespace s2k {
namespace codec {

template <class T>
s2k_status dev_alloc(s2k_codec *c, T **p, size_t n, std::vector<void *> &list) {
    void *q = nullptr;
    if (n == 0) n = 1;
    if (cudaMalloc(&q, n * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(S2K_ERR_OOM, "codec: device allocation of %zu bytes failed", n * sizeof(T));
    }
    list.push_back(q);
    *p = static_cast<T *>(q);
    return S2K_OK;
}

const HostTensor *find(const s2k_codec *c, const std::string &name) {
    auto it = c->host.find(name);
    return it == c->host.end() ? nullptr : &it->second;
}

s2k_status need(const s2k_codec *c, const std::string &name, const HostTensor **out) {
    *out = find(c, name);
    if (!*out) return fail(S2K_ERR_STATE, "codec: missing tensor %s", name.c_str());
    return S2K_OK;
}

// an f32 device copy of a vector tensor of n values
s2k_status vec(s2k_codec *c, const std::string &name, int64_t n, float **out) {
    const HostTensor *t;
    s2k_status rc = need(c, name, &t);
    if (rc) return rc;
    if (t->numel() != n) return fail(S2K_ERR_ARG, "codec: %s has %lld values, expected %lld", name.c_str(),
                                     (long long)t->numel(), (long long)n);
    std::vector<float> h((size_t)n);
    for (int64_t i = 0; i < n; ++i) h[(size_t)i] = t->at(i);
    rc = dev_alloc(c, out, (size_t)n, c->allocs);
    if (rc) return rc;
    CU(cudaMemcpy(*out, h.data(), (size_t)n * sizeof(float), cudaMemcpyHostToDevice));
    return S2K_OK;
}

// B columns per tap: whole 64-column chunks (128-byte aligned TMA rows)
int round64(int x) { return (x + 63) / 64 * 64; }

s2k_status upload_b(s2k_codec *c, GW &g, const std::vector<__half> &h) {
    s2k_status rc = dev_alloc(c, &g.w, h.size(), c->allocs);
    if (rc) return rc;
    CU(cudaMemcpy(g.w, h.data(), h.size() * sizeof(__half), cudaMemcpyHostToDevice));
    return S2K_OK;
}

// the matrices of F16-weight products must be F16 (the reference rounds the
// activation to fp16 only for those); convolution weights may be F32 (their
// fp16 im2col rounds both operands either way)
s2k_status check_f16(const HostTensor *t, const std::string &name) {
    if (t->type != S2K_TYPE_F16)
        return fail(S2K_ERR_UNSUPPORTED, "codec: %s must be F16 (type %d): an F32 matrix product keeps f32 "
                                         "activations, which this decoder does not", name.c_str(), t->type);
    return S2K_OK;
}

// linear [in, out] (mul_mat weight), optional bias
s2k_status make_linear(s2k_codec *c, const std::string &wname, const std::string &bname, int in, int out, GW &g) {
    const HostTensor *t;
    s2k_status rc = need(c, wname, &t);
    if (rc) return rc;
    if ((rc = check_f16(t, wname))) return rc;
    if (t->ne[0] != in || t->ne[1] * t->ne[2] * t->ne[3] != out)
        return fail(S2K_ERR_ARG, "codec: %s has ne [%lld, %lld], expected [%d, %d]", wname.c_str(), (long long)t->ne[0],
                    (long long)t->ne[1], in, out);
    if (out % 16 != 0 || in % 8 != 0 || in < 64 || out < 64)
        return fail(S2K_ERR_UNSUPPORTED, "codec: %s: widths %d -> %d (multiples of 8 -> 16, at least 64)", wname.c_str(), in, out);
    g.N = out;
    g.taps = 1;
    g.kin = in;
    g.kp = round64(in);
    g.cout = out;
    std::vector<__half> h((size_t)g.N * g.kp, __float2half_rn(0.f));
    for (int o = 0; o < out; ++o)
        for (int i = 0; i < in; ++i) h[(size_t)o * g.kp + i] = __float2half_rn(t->at((int64_t)o * in + i));
    if ((rc = upload_b(c, g, h))) return rc;
    if (!bname.empty()) return vec(c, bname, out, &g.bias);
    return S2K_OK;
}

// causal conv1d weight [K, Cin, Cout], dilation d (ggml_conv_1d: fp16 im2col)
s2k_status make_conv(s2k_codec *c, const std::string &p, int dil, int *Cin_out, int *Cout_out, int *K_out, GW &g) {
    const HostTensor *t;
    s2k_status rc = need(c, p + ".weight", &t);
    if (rc) return rc;
    const int K = (int)t->ne[0], Cin = (int)t->ne[1], Cout = (int)t->ne[2];
    if (K < 1 || Cin < 1 || Cout < 1 || t->ne[3] != 1) return fail(S2K_ERR_ARG, "codec: %s.weight: bad shape", p.c_str());
    if (Cout % 16 != 0 || Cin % 8 != 0 || Cin < 64 || Cout < 64)
        return fail(S2K_ERR_UNSUPPORTED, "codec: %s: channels %d -> %d (multiples of 8 -> 16, at least 64)", p.c_str(), Cin, Cout);
    g.N = Cout;
    g.taps = K;
    g.kin = Cin;
    g.kp = round64(Cin);
    g.cout = Cout;
    g.shift0 = -(K - 1) * dil;
    g.dshift = dil;
    std::vector<__half> h((size_t)g.N * g.taps * g.kp, __float2half_rn(0.f));
    for (int o = 0; o < Cout; ++o)
        for (int i = 0; i < Cin; ++i)
            for (int k = 0; k < K; ++k)
                h[(size_t)o * g.taps * g.kp + (size_t)k * g.kp + i] =
                    __float2half_rn(t->at(((int64_t)o * Cin + i) * K + k));
    if ((rc = upload_b(c, g, h))) return rc;
    if ((rc = vec(c, p + ".bias", Cout, &g.bias))) return rc;
    if (Cin_out) *Cin_out = Cin;
    if (Cout_out) *Cout_out = Cout;
    if (K_out) *K_out = K;
    return S2K_OK;
}

// causal transposed conv weight [K, Cout, Cin], stride s, crop_right:
// N = s * Cout phase-packed columns, m = K / s taps over the exact pair
// [hi | lo] of the f32 input (both halves against the same weight)
s2k_status make_convt(s2k_codec *c, const std::string &p, int s, int crop, int *Cin_out, int *Cout_out, GW &g) {
    const HostTensor *t;
    s2k_status rc = need(c, p + ".weight", &t);
    if (rc) return rc;
    const int K = (int)t->ne[0], Cout = (int)t->ne[1], Cin = (int)t->ne[2];
    if (K < 1 || Cout < 1 || Cin < 1 || t->ne[3] != 1) return fail(S2K_ERR_ARG, "codec: %s.weight: bad shape", p.c_str());
    if (K % s != 0 || crop % s != 0 || crop / s != K / s - 1)
        return fail(S2K_ERR_UNSUPPORTED, "codec: %s: kernel %d, stride %d, crop %d: only K = m*s with crop (m-1)*s",
                    p.c_str(), K, s, crop);
    if (Cout % 16 != 0 || Cin % 8 != 0 || Cin < 32 || Cout < 64)
        return fail(S2K_ERR_UNSUPPORTED, "codec: %s: channels %d -> %d (multiples of 8 -> 16, at least 32 -> 64)", p.c_str(), Cin, Cout);
    const int m = K / s;
    g.N = s * Cout;
    g.taps = m;
    g.kin = 2 * Cin;
    g.kp = round64(2 * Cin);
    g.cout = Cout;
    g.shift0 = 0;
    g.dshift = -1;
    std::vector<__half> h((size_t)g.N * g.taps * g.kp, __float2half_rn(0.f));
    for (int r = 0; r < s; ++r)
        for (int o = 0; o < Cout; ++o)
            for (int q = 0; q < m; ++q)
                for (int i = 0; i < Cin; ++i) {
                    const float v = t->at(((int64_t)i * Cout + o) * K + r + q * s);
                    if (fp16_round(v) != v)
                        return fail(S2K_ERR_UNSUPPORTED, "codec: %s holds values outside fp16 (F32 export)", p.c_str());
                    const size_t base = (size_t)(r * Cout + o) * g.taps * g.kp + (size_t)q * g.kp;
                    h[base + i] = h[base + Cin + i] = __float2half_rn(v);
                }
    if ((rc = upload_b(c, g, h))) return rc;
    if ((rc = vec(c, p + ".bias", Cout, &g.bias))) return rc;
    if (Cin_out) *Cin_out = Cin;
    if (Cout_out) *Cout_out = Cout;
    return S2K_OK;
}

int floor_div(long long a, int b) { return (int)(a >= 0 ? a / b : -((-a + b - 1) / b)); }

// Frames before an emitted frame E the decoder stages read: walk the stages
// backwards from sample E * spf to the latent frame the first emitted sample
// depends on (every stage is causal; left context = (K - 1) * dilation per
// convolution, floor(a / s) - (m - 1) through a transposed one).
int receptive_frames(const s2k_codec *c) {
    int worst = 0;
    for (int E = 1000; E < 1000 + 64; ++E) {
        long long a = (long long)E * c->spf;
        a -= c->out_K - 1;
        for (int b = (int)c->blocks.size() - 1; b >= 0; --b) {
            const DecBlock &B = c->blocks[(size_t)b];
            for (int u = 2; u >= 0; --u) {
                a -= (long long)(B.ru[u].c3.taps - 1) * B.ru[u].c3.dshift;
                a -= (long long)(B.ru[u].c1.taps - 1) * B.ru[u].c1.dshift;
            }
            a = floor_div(a, B.stride) - (B.convt.taps - 1);
        }
        a -= (long long)(c->dec0.taps - 1) * c->dec0.dshift;
        for (int i = (int)c->ups.size() - 1; i >= 0; --i) {
            const UpStage &U = c->ups[(size_t)i];
            a -= U.dwK - 1;
            a = floor_div(a, U.factor) - (U.convt.taps - 1);
        }
        worst = std::max(worst, (int)(E - a));
    }
    return worst + 1;
}

// ---- launches ----
cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

bool g_setup_done = false;
constexpr int kSmallSmemMax = 200 * 1024;  // dynamic shared memory of the non-GEMM kernels

cudaError_t setup() {
    if (g_setup_done) return cudaSuccess;
    if (!encode_fn()) return cudaErrorNotSupported;
    cudaError_t e = cudaFuncSetAttribute(codec_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmallSmemMax);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(codec_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmallSmemMax);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dwconv_ln_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmallSmemMax);
    if (e == cudaSuccess) g_setup_done = true;
    return e;
}

// Tile width from a per-SM cost model: a tile takes the longest of its MMA
// time (128 x BN x K MACs at ~4096 per cycle), its operand traffic
// ((128 + BN) x K fp16 from L2 at ~64 bytes per cycle) and its epilogue
// (~0.3 cycle per output), and the tiles run in waves over the SMs.
int pick_bn(int M, int N, int K, int sms, bool narrow_set) {
    static const int all[] = {256, 192, 128, 96, 64}, narrow[] = {256, 128, 64};
    const int *cands = narrow_set ? narrow : all;
    const int nc = narrow_set ? 3 : 5;
    const long long MT = (M + kCM - 1) / kCM;
    int best = cands[nc - 1];
    double best_cost = -1;
    for (int i = 0; i < nc; ++i) {
        const int bn = cands[i];
        if (bn > N && bn != cands[nc - 1]) continue;
        const long long tiles = MT * ((N + bn - 1) / bn);
        const double mma = 128.0 * bn * K / 4096.0, load = (128.0 + bn) * K * 2.0 / 64.0, epi = 128.0 * bn * 0.3;
        const double cost = (double)((tiles + sms - 1) / sms) * std::max(mma, std::max(load, epi));
        if (best_cost < 0 || cost < best_cost * 0.999) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

struct ARef {  // A operand: fp16 [rows][width], row stride ld (elements)
    const __half *p;
    int rows, width, ld;
};

struct Epi {
    const float *gamma = nullptr, *alpha = nullptr, *res = nullptr;
    int act = ACT_NONE;
    bool no_bias = false;
    float *y32 = nullptr;
    int ldy32 = 0;
    __half *y16 = nullptr;
    int ldy16 = 0, o16 = O16_NONE, lo_off = 0;
};

template <int BN, int F>
cudaError_t launch_gemm_t(const CUtensorMap &amap, const CUtensorMap &bmap, const CGemm &p, int grid, cudaStream_t st) {
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e = cudaFuncSetAttribute(codec_gemm_kernel<BN, F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)(sizeof(CSmem<BN>) + 1024));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(grid), dim3(kCThreads), sizeof(CSmem<BN>) + 1024, st, attr);
    return cudaLaunchKernelEx(&cfg, codec_gemm_kernel<BN, F>, amap, bmap, p);
}

// tile widths compiled for an epilogue: {64, 128, 256} for the transformer's
// products, {64, 96, 128, 192, 256} for the convolutions
template <int F, bool Narrow>
cudaError_t launch_gemm_f(int BN, const CUtensorMap &amap, const CUtensorMap &bmap, const CGemm &p, int grid,
                          cudaStream_t st) {
    switch (BN) {
    case 64: return launch_gemm_t<64, F>(amap, bmap, p, grid, st);
    case 128: return launch_gemm_t<128, F>(amap, bmap, p, grid, st);
    case 256: return launch_gemm_t<256, F>(amap, bmap, p, grid, st);
    default: break;
    }
    if constexpr (!Narrow) {
        if (BN == 96) return launch_gemm_t<96, F>(amap, bmap, p, grid, st);
        if (BN == 192) return launch_gemm_t<192, F>(amap, bmap, p, grid, st);
    }
    return cudaErrorInvalidValue;
}

// the feature set of an epilogue
int epi_features(const CGemm &p) {
    return (p.bias ? F_BIAS : 0) | (p.gamma ? F_GAMMA : 0) | (p.res ? F_RES : 0) | (p.y32 ? F_Y32 : 0) |
           (p.act == ACT_GELU ? F_GELU : 0) | (p.act == ACT_SWIGLU ? F_SWIGLU : 0) | f_o16(p.o16);
}

constexpr int kEpiQKV = F_Y32;                                          // wqkv
constexpr int kEpiResGamma = F_GAMMA | F_RES | F_Y32;                   // wo, w2
constexpr int kEpiSwiglu = F_SWIGLU;                                    // w1 | w3
constexpr int kEpiBias32 = F_BIAS | F_Y32;                              // upsample transposed conv
constexpr int kEpiGelu = F_BIAS | F_GELU | (O16_PLAIN << 6);            // pwconv1
constexpr int kEpiCnxHilo = F_BIAS | F_GAMMA | F_RES | (O16_HILO << 6);  // pwconv2 -> next transposed conv
constexpr int kEpiCnxPlain = F_BIAS | F_GAMMA | F_RES | (O16_PLAIN << 6);  // pwconv2 -> decoder conv
constexpr int kEpiSnakeHilo = F_BIAS | (O16_SNAKE_HILO << 6);           // decoder conv
constexpr int kEpiConvT = F_BIAS | F_Y32 | (O16_SNAKE << 6);             // block transposed conv
constexpr int kEpiSnake = F_BIAS | (O16_SNAKE << 6);                     // residual unit conv 1
constexpr int kEpiResSnake = F_BIAS | F_RES | F_Y32 | (O16_SNAKE << 6);  // residual unit conv 2
constexpr int kEpiResSnakeHilo = F_BIAS | F_RES | (O16_SNAKE_HILO << 6);  // last unit -> next block
constexpr int kEpiResSnakeOut = F_BIAS | F_RES | (O16_SNAKE << 6);       // last unit -> output conv

bool narrow_epilogue(int F) { return F == kEpiQKV || F == kEpiResGamma || F == kEpiSwiglu; }

cudaError_t launch_gemm(int F, int BN, const CUtensorMap &amap, const CUtensorMap &bmap, const CGemm &p, int grid,
                        cudaStream_t st) {
    switch (F) {
    case kEpiQKV: return launch_gemm_f<kEpiQKV, true>(BN, amap, bmap, p, grid, st);
    case kEpiResGamma: return launch_gemm_f<kEpiResGamma, true>(BN, amap, bmap, p, grid, st);
    case kEpiSwiglu: return launch_gemm_f<kEpiSwiglu, true>(BN, amap, bmap, p, grid, st);
    case kEpiBias32: return launch_gemm_f<kEpiBias32, false>(BN, amap, bmap, p, grid, st);
    case kEpiGelu: return launch_gemm_f<kEpiGelu, false>(BN, amap, bmap, p, grid, st);
    case kEpiCnxHilo: return launch_gemm_f<kEpiCnxHilo, false>(BN, amap, bmap, p, grid, st);
    case kEpiCnxPlain: return launch_gemm_f<kEpiCnxPlain, false>(BN, amap, bmap, p, grid, st);
    case kEpiSnakeHilo: return launch_gemm_f<kEpiSnakeHilo, false>(BN, amap, bmap, p, grid, st);
    case kEpiConvT: return launch_gemm_f<kEpiConvT, false>(BN, amap, bmap, p, grid, st);
    case kEpiSnake: return launch_gemm_f<kEpiSnake, false>(BN, amap, bmap, p, grid, st);
    case kEpiResSnake: return launch_gemm_f<kEpiResSnake, false>(BN, amap, bmap, p, grid, st);
    case kEpiResSnakeHilo: return launch_gemm_f<kEpiResSnakeHilo, false>(BN, amap, bmap, p, grid, st);
    case kEpiResSnakeOut: return launch_gemm_f<kEpiResSnakeOut, false>(BN, amap, bmap, p, grid, st);
    default: return cudaErrorNotSupported;
    }
}

s2k_status gemm(s2k_codec *c, const ARef &a, const GW &g, int M, const Epi &e) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(S2K_ERR_UNSUPPORTED, "codec: cuTensorMapEncodeTiled unavailable");
    if (a.width > g.kp || a.width != g.kin) return fail(S2K_ERR_ARG, "codec: GEMM input width %d, weights expect %d", a.width, g.kin);
    CUtensorMap amap, bmap;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)a.width, (cuuint64_t)a.rows};
        const cuuint64_t strides[1] = {(cuuint64_t)a.ld * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kCK, (cuuint32_t)kCM};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(a.p), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(S2K_ERR_CUDA, "codec: activation tensor map (%d x %d, ld %d)", a.rows, a.width, a.ld);
    }
    CGemm p;
    p.M = M;
    p.N = g.N;
    p.kchunks = (a.width + kCK - 1) / kCK;
    p.kp = g.kp;
    p.ksteps_last = (a.width - kCK * (p.kchunks - 1) + 15) / 16;
    p.taps = g.taps;
    p.shift0 = g.shift0;
    p.dshift = g.dshift;
    p.cout = g.cout;
    p.bias = e.no_bias ? nullptr : g.bias;
    p.gamma = e.gamma;
    p.alpha = e.alpha;
    p.act = e.act;
    p.res = e.res;
    p.ldres = e.ldy32 > 0 ? e.ldy32 : g.N;
    p.y32 = e.y32;
    p.ldy32 = e.ldy32 > 0 ? e.ldy32 : g.N;
    p.y16 = e.y16;
    p.ldy16 = e.ldy16;
    p.o16 = e.o16;
    p.lo_off = e.lo_off;
    p.err = c->d_err;
    const int F = epi_features(p);
    const int BN = pick_bn(M, g.N, g.taps * g.kp, c->num_sms, narrow_epilogue(F));
    {
        const cuuint64_t dims[2] = {(cuuint64_t)g.taps * g.kp, (cuuint64_t)g.N};
        const cuuint64_t strides[1] = {(cuuint64_t)g.taps * g.kp * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kCK, (cuuint32_t)BN};
        const cuuint32_t es[2] = {1, 1};
        if (enc(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, g.w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(S2K_ERR_CUDA, "codec: weight tensor map (%d x %d)", g.N, g.taps * g.kp);
    }
    const int MT = (M + kCM - 1) / kCM, NT = (g.N + BN - 1) / BN;
    const int grid = std::min(MT * NT, c->num_sms);
    count_launch();
    const cudaError_t err = launch_gemm(F, BN, amap, bmap, p, grid, c->st);
    if (err == cudaErrorNotSupported) return fail(S2K_ERR_UNSUPPORTED, "codec: no GEMM epilogue for features 0x%x", F);
    CU(err);
    return S2K_OK;
}

template <class... KArgs, class... Args>
s2k_status launch(s2k_codec *c, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(grid, block, smem, c->st, attr);
    count_launch();
    CU(cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...));
    return S2K_OK;
}

// ---- workspace: every buffer sized for n_tr transformer frames and n_dec decoder frames ----
s2k_status ensure_ws(s2k_codec *c, int n_tr, int n_dec) {
    if ((size_t)n_tr <= c->ws_tr && (size_t)n_dec <= c->ws_dec) return S2K_OK;
    cudaStreamSynchronize(c->st);
    for (void *p : c->ws_allocs) cudaFree(p);
    c->ws_allocs.clear();
    const size_t tr = std::max((size_t)n_tr, c->ws_tr), dec = std::max((size_t)n_dec, c->ws_dec);
    c->ws_tr = c->ws_dec = 0;
    size_t p32 = 0, s16 = 0, t16 = 0, hl = 2 * dec * (size_t)c->dim;
    size_t L = dec;
    for (const UpStage &U : c->ups) {
        L *= (size_t)U.factor;
        p32 = std::max(p32, L * U.C);
        s16 = std::max(s16, L * U.C);
        t16 = std::max(t16, L * (size_t)U.hid);
        hl = std::max(hl, 2 * L * U.C);
    }
    hl = std::max(hl, 2 * L * (size_t)c->dec0.N);
    for (const DecBlock &B : c->blocks) {
        L *= (size_t)B.stride;
        p32 = std::max(p32, L * B.Cout);
        s16 = std::max(s16, L * B.Cout);
        t16 = std::max(t16, L * B.Cout);
        hl = std::max(hl, 2 * L * B.Cout);
    }
    const size_t n16 = tr * (size_t)std::max(c->dim, c->qs);
    s2k_status rc;
    if ((rc = dev_alloc(c, &c->d_codes, tr * (size_t)c->nq, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->X, tr * (size_t)c->dim, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->QKV, tr * (size_t)(c->qs + 2 * c->kvs), c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->N16, n16, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->G16, tr * (size_t)c->ff, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->P, p32, c->ws_allocs)) || (rc = dev_alloc(c, &c->S16, s16, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->T16, t16, c->ws_allocs)) || (rc = dev_alloc(c, &c->HLa, hl, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->HLb, hl, c->ws_allocs)) || (rc = dev_alloc(c, &c->audio, L, c->ws_allocs)) ||
        (rc = dev_alloc(c, &c->rope, tr * (size_t)c->hd, c->ws_allocs))) {
        for (void *p : c->ws_allocs) cudaFree(p);
        c->ws_allocs.clear();
        return rc;
    }
    // RoPE angles of every position by ggml's float recurrence theta_{i+1} =
    // theta_i * base^(-2/hd) from theta_0 = pos, and their cos / sin
    {
        const int half = c->hd / 2;
        std::vector<float> tab(tr * (size_t)c->hd);
        for (size_t pos = 0; pos < tr; ++pos) {
            float theta = (float)pos;
            for (int i = 0; i < half; ++i) {
                tab[(pos * half + i) * 2] = ::cosf(theta);
                tab[(pos * half + i) * 2 + 1] = ::sinf(theta);
                theta *= c->rope_ts;
            }
        }
        CU(cudaMemcpy(c->rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    c->ws_tr = tr;
    c->ws_dec = dec;
    return S2K_OK;
}

// The decode of frames [0, n_tr) of the (uploaded) window through the
// transformer and of frames [f0, n_tr) through the decoder stages; the
// audio of those decoder frames lands in c->audio (n_dec * spf samples).
s2k_status run_window(s2k_codec *c, int n_tr, int f0) {
    const int n_dec = n_tr - f0;
    s2k_status rc;
    // VQ decode
    VqParams vp;
    std::memset(&vp, 0, sizeof(vp));
    vp.nq = c->nq;
    vp.L = n_tr;
    vp.C = c->C0;
    vp.cd = c->cd;
    vp.codes = c->d_codes;
    for (int q = 0; q < c->nq; ++q) {
        vp.size[q] = c->vq_size[q];
        vp.cb[q] = c->vq_cb[q];
        vp.ow[q] = c->vq_ow[q];
        vp.ob[q] = c->vq_ob[q];
    }
    if ((rc = launch(c, vq_decode_kernel, dim3(n_tr, (c->C0 + 127) / 128), dim3(128), 0, vp, c->X))) return rc;
    // post-module transformer
    const int qkvs = c->qs + 2 * c->kvs;
    const float scale = 1.0f / std::sqrt((float)c->hd);
    for (const CLayer &ly : c->layers) {
        if ((rc = launch(c, rmsnorm_rows_kernel, dim3(n_tr), dim3(256), 0, (const float *)c->X, c->dim,
                         (const float *)ly.attn_norm, c->eps, 0, c->N16, c->dim, 0)))
            return rc;
        Epi e;
        e.y32 = c->QKV;
        e.ldy32 = qkvs;
        if ((rc = gemm(c, {c->N16, n_tr, c->dim, c->dim}, ly.wqkv, n_tr, e))) return rc;
        const int span = (c->W > 0 ? std::min(c->W, n_tr) : n_tr) + kAQ - 1;
        const size_t asmem = ((size_t)(kAQ + kAKC) * (c->hd + 1) + (size_t)kAQ * span) * sizeof(float);
        if (asmem > (size_t)kSmallSmemMax) return fail(S2K_ERR_UNSUPPORTED, "codec: attention over %d keys", span);
        if ((rc = launch(c, codec_attn_kernel, dim3((n_tr + kAQ - 1) / kAQ, c->H), dim3(kAThreads), asmem,
                         (const float *)c->QKV, qkvs, n_tr, c->H, c->Hk, c->hd, c->qs, c->W, scale,
                         (const float2 *)c->rope, c->N16, c->qs, span)))
            return rc;
        Epi eo;
        eo.gamma = ly.attn_gamma;
        eo.res = c->X;
        eo.y32 = c->X;
        eo.ldy32 = c->dim;
        if ((rc = gemm(c, {c->N16, n_tr, c->qs, c->qs}, ly.wo, n_tr, eo))) return rc;
        if ((rc = launch(c, rmsnorm_rows_kernel, dim3(n_tr), dim3(256), 0, (const float *)c->X, c->dim,
                         (const float *)ly.ffn_norm, c->eps, 0, c->N16, c->dim, 0)))
            return rc;
        Epi es;
        es.act = ACT_SWIGLU;
        es.y16 = c->G16;
        es.ldy16 = c->ff;
        if ((rc = gemm(c, {c->N16, n_tr, c->dim, c->dim}, ly.w13, n_tr, es))) return rc;
        Epi e2;
        e2.gamma = ly.ffn_gamma;
        e2.res = c->X;
        e2.y32 = c->X;
        e2.ldy32 = c->dim;
        if ((rc = gemm(c, {c->G16, n_tr, c->ff, c->ff}, ly.w2, n_tr, e2))) return rc;
    }
    // final norm of the decoder frames -> exact pair for the first transposed conv
    if ((rc = launch(c, rmsnorm_rows_kernel, dim3(n_dec), dim3(256), 0, (const float *)c->X, c->dim,
                     (const float *)c->final_norm, c->eps, f0, c->HLa, 2 * c->dim, 1)))
        return rc;
    // upsample stages
    __half *hl_in = c->HLa, *hl_out = c->HLb;
    int L = n_dec, C = c->dim;
    for (size_t i = 0; i < c->ups.size(); ++i) {
        const UpStage &U = c->ups[i];
        Epi et;
        et.y32 = c->P;
        et.ldy32 = U.convt.N;
        if ((rc = gemm(c, {hl_in, L, 2 * C, 2 * C}, U.convt, L, et))) return rc;
        L *= U.factor;
        C = U.C;
        if ((rc = launch(c, dwconv_ln_kernel, dim3(L), dim3(256), (size_t)C * sizeof(float), (const float *)c->P, C,
                         (const float *)U.dw, U.dwK, (const float *)U.dwb, (const float *)U.lnw, (const float *)U.lnb,
                         1e-6f, c->S16)))
            return rc;
        Epi e1;
        e1.act = ACT_GELU;
        e1.y16 = c->T16;
        e1.ldy16 = U.hid;
        e1.o16 = O16_PLAIN;
        if ((rc = gemm(c, {c->S16, L, C, C}, U.pw1, L, e1))) return rc;
        Epi e2;
        e2.gamma = U.gamma;
        e2.res = c->P;
        e2.ldy32 = C;
        const bool last = i + 1 == c->ups.size();
        if (last) {  // the decoder's first conv rounds its input to fp16
            e2.y16 = c->S16;
            e2.ldy16 = C;
            e2.o16 = O16_PLAIN;
        } else {
            e2.y16 = hl_out;
            e2.ldy16 = 2 * C;
            e2.o16 = O16_HILO;
            e2.lo_off = C;
        }
        if ((rc = gemm(c, {c->T16, L, U.hid, U.hid}, U.pw2, L, e2))) return rc;
        if (!last) std::swap(hl_in, hl_out);
    }
    // decoder conv -> snake of the first block -> exact pair
    {
        Epi e;
        e.y16 = hl_in;
        e.ldy16 = 2 * c->dec0.N;
        e.o16 = O16_SNAKE_HILO;
        e.lo_off = c->dec0.N;
        e.alpha = c->blocks[0].alpha;
        if ((rc = gemm(c, {c->S16, L, C, C}, c->dec0, L, e))) return rc;
        C = c->dec0.N;
    }
    for (size_t b = 0; b < c->blocks.size(); ++b) {
        const DecBlock &B = c->blocks[b];
        Epi et;
        et.y32 = c->P;
        et.ldy32 = B.convt.N;
        et.y16 = c->S16;
        et.ldy16 = B.convt.N;
        et.o16 = O16_SNAKE;
        et.alpha = B.ru[0].a0;
        if ((rc = gemm(c, {hl_in, L, 2 * C, 2 * C}, B.convt, L, et))) return rc;
        L *= B.stride;
        C = B.Cout;
        for (int u = 0; u < 3; ++u) {
            const ResUnit &R = B.ru[u];
            Epi e1;
            e1.y16 = c->T16;
            e1.ldy16 = C;
            e1.o16 = O16_SNAKE;
            e1.alpha = R.a2;
            if ((rc = gemm(c, {c->S16, L, C, C}, R.c1, L, e1))) return rc;
            Epi e3;
            e3.res = c->P;
            e3.ldy32 = C;
            if (u < 2) {
                e3.y32 = c->P;
                e3.y16 = c->S16;
                e3.ldy16 = C;
                e3.o16 = O16_SNAKE;
                e3.alpha = B.ru[u + 1].a0;
            } else if (b + 1 < c->blocks.size()) {
                e3.y16 = hl_out;
                e3.ldy16 = 2 * C;
                e3.o16 = O16_SNAKE_HILO;
                e3.lo_off = C;
                e3.alpha = c->blocks[b + 1].alpha;
            } else {
                e3.y16 = c->S16;
                e3.ldy16 = C;
                e3.o16 = O16_SNAKE;
                e3.alpha = c->out_alpha;
            }
            if ((rc = gemm(c, {c->T16, L, C, C}, R.c3, L, e3))) return rc;
        }
        std::swap(hl_in, hl_out);
    }
    const size_t osmem = (size_t)c->out_K * c->out_C * sizeof(float) +
                         (size_t)(kOutRows + c->out_K - 1) * (c->out_C + 2) * sizeof(__half);
    if (osmem > (size_t)kSmallSmemMax)
        return fail(S2K_ERR_UNSUPPORTED, "codec: output conv of %d taps over %d channels", c->out_K, c->out_C);
    return launch(c, codec_out_kernel, dim3((L + kOutRows - 1) / kOutRows), dim3(kOutRows), osmem, (const __half *)c->S16, L, c->out_C,
                  (const float *)c->out_w, c->out_K, c->out_b, c->audio);
}

s2k_status check_err(s2k_codec *c) {
    int h[kErrBlockInts] = {};
    CU(cudaMemcpy(h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h[0] != 0) {
        cudaMemset(c->d_err, 0, sizeof(int));
        return fail(S2K_ERR_TIMEOUT, "codec: device wait timed out (flags 0x%x)", h[0]);
    }
    return S2K_OK;
}

// decode frames [0, emit_end) of an n_frames window (codes cb-major with row
// length ld), copy the samples of frames [emit_begin, emit_end) to audio
s2k_status decode_range(s2k_codec *c, const int32_t *codes, int ld, int emit_begin, int emit_end, float *audio,
                        size_t cap, int64_t *n_samples, float *ms) {
    if (emit_end <= emit_begin) {
        *n_samples = 0;
        return S2K_OK;
    }
    const int f0 = std::max(0, emit_begin - c->receptive);
    const int n_tr = emit_end, n_dec = n_tr - f0;
    const int64_t n_out = (int64_t)(emit_end - emit_begin) * c->spf;
    if ((int64_t)cap < n_out) return fail(S2K_ERR_ARG, "codec: %lld samples, capacity %zu", (long long)n_out, cap);
    s2k_status rc = ensure_ws(c, n_tr, n_dec);
    if (rc) return rc;
    for (int q = 0; q < c->nq; ++q)
        CU(cudaMemcpyAsync(c->d_codes + (size_t)q * n_tr, codes + (size_t)q * ld, (size_t)n_tr * sizeof(int32_t),
                           cudaMemcpyHostToDevice, c->st));
    CU(cudaEventRecord(c->ev0, c->st));
    if ((rc = run_window(c, n_tr, f0))) return rc;
    CU(cudaEventRecord(c->ev1, c->st));
    CU(cudaMemcpyAsync(audio, c->audio + (size_t)(emit_begin - f0) * c->spf, (size_t)n_out * sizeof(float),
                       cudaMemcpyDeviceToHost, c->st));
    CU(cudaStreamSynchronize(c->st));
    if ((rc = check_err(c))) return rc;
    if (ms) CU(cudaEventElapsedTime(ms, c->ev0, c->ev1));
    *n_samples = n_out;
    return S2K_OK;
}

s2k_status finalize(s2k_codec *c) {
    const s2k_codec_hparams &hp = c->hp;
    s2k_status rc;
    // VQ
    c->nq = hp.quantizer_residual_codebooks + 1;
    if (c->nq < 1 || c->nq > kMaxQ) return fail(S2K_ERR_UNSUPPORTED, "codec: %d codebooks (1..%d)", c->nq, kMaxQ);
    c->C0 = hp.quantizer_input_dim;
    for (int q = 0; q < c->nq; ++q) {
        const std::string p = q == 0 ? std::string("quantizer.semantic_quantizer.quantizers.0.")
                                     : "quantizer.quantizer.quantizers." + std::to_string(q - 1) + ".";
        const HostTensor *cb, *ow;
        if ((rc = need(c, p + "codebook.weight", &cb)) || (rc = need(c, p + "out_proj.weight", &ow))) return rc;
        const int cd = (int)cb->ne[0], rows = (int)cb->ne[1];
        const int ocd = (int)(ow->ne[0] == 1 ? ow->ne[1] : ow->ne[0]);
        const int oc = (int)(ow->ne[0] == 1 ? ow->ne[2] : ow->ne[1]);
        if (ocd != cd || oc != c->C0) return fail(S2K_ERR_ARG, "codec: %sout_proj.weight shape", p.c_str());
        c->cd = cd;
        const int size = q == 0 ? hp.quantizer_semantic_codebook_size : hp.quantizer_residual_codebook_size;
        c->vq_size[q] = std::min(size, rows);
        std::vector<float> h(cb->numel());
        for (int64_t i = 0; i < cb->numel(); ++i) h[(size_t)i] = cb->at(i);
        if ((rc = dev_alloc(c, &c->vq_cb[q], h.size(), c->allocs))) return rc;
        CU(cudaMemcpy(c->vq_cb[q], h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
        h.resize(ow->numel());
        for (int64_t i = 0; i < ow->numel(); ++i) h[(size_t)i] = ow->at(i);
        if ((rc = dev_alloc(c, &c->vq_ow[q], h.size(), c->allocs))) return rc;
        CU(cudaMemcpy(c->vq_ow[q], h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
        if ((rc = vec(c, p + "out_proj.bias", c->C0, &c->vq_ob[q]))) return rc;
    }
    // transformer (as many layers as the file holds, src/s2_codec.cpp:300-303)
    c->dim = hp.rvq_dim;
    c->hd = hp.rvq_head_dim;
    if (c->dim != c->C0 || c->hd < 2 || c->hd % 2 || c->hd > kAMaxHd || c->dim % c->hd)
        return fail(S2K_ERR_UNSUPPORTED, "codec: transformer dim %d / head_dim %d", c->dim, c->hd);
    c->H = c->dim / c->hd;
    c->Hk = hp.rvq_n_local_heads > 0 ? hp.rvq_n_local_heads : c->H;
    if (c->H % c->Hk) return fail(S2K_ERR_UNSUPPORTED, "codec: %d heads over %d kv heads", c->H, c->Hk);
    c->qs = c->H * c->hd;
    c->kvs = c->Hk * c->hd;
    c->W = hp.rvq_window_size;
    c->eps = hp.rvq_norm_eps;
    c->rope_ts = ::powf(hp.rvq_rope_base, -2.0f / (float)c->hd);
    for (int l = 0;; ++l) {
        const std::string p = "quantizer.post_module.layers." + std::to_string(l) + ".";
        if (!find(c, p + "attention.wqkv.weight")) break;
        CLayer ly;
        const HostTensor *w1;
        if ((rc = need(c, p + "feed_forward.w1.weight", &w1))) return rc;
        c->ff = (int)w1->ne[1];
        if (c->ff % 8) return fail(S2K_ERR_UNSUPPORTED, "codec: feed-forward width %d", c->ff);
        if ((rc = make_linear(c, p + "attention.wqkv.weight", "", c->dim, c->qs + 2 * c->kvs, ly.wqkv)) ||
            (rc = make_linear(c, p + "attention.wo.weight", "", c->qs, c->dim, ly.wo)) ||
            (rc = make_linear(c, p + "feed_forward.w2.weight", "", c->ff, c->dim, ly.w2)) ||
            (rc = vec(c, p + "attention_norm.weight", c->dim, &ly.attn_norm)) ||
            (rc = vec(c, p + "ffn_norm.weight", c->dim, &ly.ffn_norm)) ||
            (rc = vec(c, p + "attention_layer_scale.gamma", c->dim, &ly.attn_gamma)) ||
            (rc = vec(c, p + "ffn_layer_scale.gamma", c->dim, &ly.ffn_gamma)))
            return rc;
        // w1 | w3 interleaved by 8 columns: the SwiGLU epilogue sees gate and up together
        const HostTensor *w3;
        if ((rc = need(c, p + "feed_forward.w3.weight", &w3))) return rc;
        if ((rc = check_f16(w1, p + "feed_forward.w1.weight")) || (rc = check_f16(w3, p + "feed_forward.w3.weight")))
            return rc;
        if (w1->ne[0] != c->dim || w3->ne[0] != c->dim || w3->ne[1] != c->ff)
            return fail(S2K_ERR_ARG, "codec: %sfeed_forward shapes", p.c_str());
        GW &g = ly.w13;
        g.N = 2 * c->ff;
        g.taps = 1;
        g.kin = c->dim;
        g.kp = round64(c->dim);
        g.cout = g.N;
        std::vector<__half> h((size_t)g.N * g.kp, __float2half_rn(0.f));
        for (int j = 0; j < c->ff; ++j) {
            const int row = (j / 8) * 16 + j % 8;
            for (int i = 0; i < c->dim; ++i) {
                h[(size_t)row * g.kp + i] = __float2half_rn(w1->at((int64_t)j * c->dim + i));
                h[(size_t)(row + 8) * g.kp + i] = __float2half_rn(w3->at((int64_t)j * c->dim + i));
            }
        }
        if ((rc = upload_b(c, g, h))) return rc;
        c->layers.push_back(ly);
    }
    if (c->layers.empty()) return fail(S2K_ERR_STATE, "codec: no post-module transformer layer");
    if ((rc = vec(c, "quantizer.post_module.norm.weight", c->dim, &c->final_norm))) return rc;
    // upsample stages, factors in reverse order (src/s2_codec.cpp:472-477)
    if (hp.n_downsample < 1 || hp.n_downsample > 8) return fail(S2K_ERR_ARG, "codec: n_downsample %d", hp.n_downsample);
    int C = c->dim;
    for (int i = 0; i < hp.n_downsample; ++i) {
        UpStage U;
        U.factor = hp.quantizer_downsample_factor[hp.n_downsample - 1 - i];
        const std::string p = "quantizer.upsample." + std::to_string(i) + ".";
        int cin = 0;
        if ((rc = make_convt(c, p + "0.conv", U.factor, 0, &cin, &U.C, U.convt))) return rc;
        if (cin != C) return fail(S2K_ERR_ARG, "codec: %s0.conv takes %d channels, stage has %d", p.c_str(), cin, C);
        C = U.C;
        const HostTensor *dw;
        if ((rc = need(c, p + "1.dwconv.conv.weight", &dw))) return rc;
        U.dwK = (int)dw->ne[0];
        if (dw->numel() != (int64_t)U.dwK * C) return fail(S2K_ERR_ARG, "codec: %s1.dwconv.conv.weight shape", p.c_str());
        std::vector<float> h((size_t)dw->numel());
        for (int64_t e = 0; e < dw->numel(); ++e) h[(size_t)e] = fp16_round(dw->at(e));
        if ((rc = dev_alloc(c, &U.dw, h.size(), c->allocs))) return rc;
        CU(cudaMemcpy(U.dw, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
        const HostTensor *p1;
        if ((rc = need(c, p + "1.pwconv1.weight", &p1))) return rc;
        U.hid = (int)p1->ne[1];
        if ((rc = vec(c, p + "1.dwconv.conv.bias", C, &U.dwb)) || (rc = vec(c, p + "1.norm.weight", C, &U.lnw)) ||
            (rc = vec(c, p + "1.norm.bias", C, &U.lnb)) || (rc = vec(c, p + "1.gamma", C, &U.gamma)) ||
            (rc = make_linear(c, p + "1.pwconv1.weight", p + "1.pwconv1.bias", C, U.hid, U.pw1)) ||
            (rc = make_linear(c, p + "1.pwconv2.weight", p + "1.pwconv2.bias", U.hid, C, U.pw2)))
            return rc;
        c->ups.push_back(U);
    }
    // decoder (src/s2_codec.cpp:497-522)
    if (hp.n_decoder_rates < 1 || hp.n_decoder_rates > 8) return fail(S2K_ERR_ARG, "codec: %d decoder rates", hp.n_decoder_rates);
    int cin = 0, K = 0;
    if ((rc = make_conv(c, "decoder.model.0.conv", 1, &cin, &C, &K, c->dec0))) return rc;
    if (cin != c->ups.back().C) return fail(S2K_ERR_ARG, "codec: decoder.model.0.conv input width %d", cin);
    for (int i = 0; i < hp.n_decoder_rates; ++i) {
        DecBlock B;
        B.stride = hp.decoder_rates[i];
        const std::string p = "decoder.model." + std::to_string(i + 1) + ".block.";
        if ((rc = vec(c, p + "0.alpha", C, &B.alpha))) return rc;
        if ((rc = make_convt(c, p + "1.conv", B.stride, B.stride, &B.Cin, &B.Cout, B.convt))) return rc;
        if (B.Cin != C) return fail(S2K_ERR_ARG, "codec: %s1.conv input width %d, block has %d", p.c_str(), B.Cin, C);
        C = B.Cout;
        static const int dil[3] = {1, 3, 9};
        for (int u = 0; u < 3; ++u) {
            const std::string q = p + std::to_string(2 + u) + ".block.";
            int ci = 0, co = 0, co3 = 0;
            if ((rc = vec(c, q + "0.alpha", C, &B.ru[u].a0)) || (rc = vec(c, q + "2.alpha", C, &B.ru[u].a2)) ||
                (rc = make_conv(c, q + "1.conv", dil[u], &ci, &co, nullptr, B.ru[u].c1)) ||
                (rc = make_conv(c, q + "3.conv", 1, nullptr, &co3, nullptr, B.ru[u].c3)))
                return rc;
            if (ci != C || co != C || co3 != C) return fail(S2K_ERR_ARG, "codec: %s convolutions keep %d channels", q.c_str(), C);
        }
        c->blocks.push_back(B);
    }
    {
        const int last = hp.n_decoder_rates + 1;
        if ((rc = vec(c, "decoder.model." + std::to_string(last) + ".alpha", C, &c->out_alpha))) return rc;
        const std::string p = "decoder.model." + std::to_string(last + 1) + ".conv";
        const HostTensor *w, *b;
        if ((rc = need(c, p + ".weight", &w)) || (rc = need(c, p + ".bias", &b))) return rc;
        if (w->ne[1] != C || w->ne[2] != 1 || b->numel() != 1)
            return fail(S2K_ERR_UNSUPPORTED, "codec: %s: a %d-channel input, one output channel expected", p.c_str(), C);
        c->out_K = (int)w->ne[0];
        c->out_C = C;
        std::vector<float> h((size_t)w->numel());
        for (int64_t e = 0; e < w->numel(); ++e) h[(size_t)e] = fp16_round(w->at(e));
        if ((rc = dev_alloc(c, &c->out_w, h.size(), c->allocs))) return rc;
        CU(cudaMemcpy(c->out_w, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
        c->out_b = b->at(0);
    }
    // samples per code frame (src/s2_codec.cpp:858-868) and the streaming history (:870-874)
    int factor = 1;
    for (int i = 0; i < hp.n_downsample; ++i) factor *= std::max(1, hp.quantizer_downsample_factor[i]);
    int rate = 1;
    for (int i = 0; i < hp.n_decoder_rates; ++i) rate *= hp.decoder_rates[i];
    c->spf = rate * factor;
    if (hp.hop_length != rate)
        return fail(S2K_ERR_UNSUPPORTED, "codec: hop_length %d differs from the decoder rates' product %d", hp.hop_length, rate);
    const int rvq_history = std::max(0, hp.rvq_window_size - 1);
    c->history = ((rvq_history + 16 + 7) / 8) * 8;
    if (c->history <= 0) c->history = 160;
    c->receptive = receptive_frames(c);
    c->host.clear();
    c->ready = true;
    return S2K_OK;
}

}  // namespace codec
}  // namespace s2k

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
S2K_API s2k_status s2k_codec_create(int32_t device, const s2k_codec_hparams *hp, s2k_codec **out) {
    if (!hp || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(S2K_ERR_NO_DEVICE, "no CUDA device");
    }
    if (device < 0 || device >= n) return fail(S2K_ERR_ARG, "device %d out of range (%d devices)", device, n);
    if (cudaSetDevice(device) != cudaSuccess) return fail(S2K_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    if (s2k::codec::setup() != cudaSuccess) return fail(S2K_ERR_UNSUPPORTED, "codec: tensor-core GEMM set-up failed");
    std::unique_ptr<s2k_codec> c(new s2k_codec());
    c->device = device;
    c->hp = *hp;
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreate(&c->ev0) != cudaSuccess || cudaEventCreate(&c->ev1) != cudaSuccess)
        return fail(S2K_ERR_CUDA, "codec: stream / event create failed");
    if (cudaMalloc(&c->d_err, kErrBlockInts * sizeof(int)) != cudaSuccess) return fail(S2K_ERR_OOM, "codec: error block");
    cudaMemset(c->d_err, 0, kErrBlockInts * sizeof(int));
    *out = c.release();
    return S2K_OK;
}

S2K_API s2k_status s2k_codec_upload_tensor(s2k_codec *c, const char *name, int32_t ggml_type, const int64_t ne[4],
                                           const void *data, size_t nbytes) {
    if (!c || !name || !ne || !data) return fail(S2K_ERR_ARG, "NULL argument");
    if (c->ready) return fail(S2K_ERR_STATE, "codec already finalized");
    if (ggml_type != S2K_TYPE_F32 && ggml_type != S2K_TYPE_F16)
        return fail(S2K_ERR_UNSUPPORTED, "codec tensor %s: type %d (F32 / F16)", name, ggml_type);
    if (!std::strncmp(name, "c.", 2)) name += 2;  // the combined GGUF's codec prefix
    HostTensor t;
    t.type = ggml_type;
    int64_t n = 1;
    for (int d = 0; d < 4; ++d) {
        t.ne[d] = ne[d] > 0 ? ne[d] : 1;
        n *= t.ne[d];
    }
    const size_t want = (size_t)n * (ggml_type == S2K_TYPE_F32 ? 4 : 2);
    if (nbytes != want) return fail(S2K_ERR_ARG, "codec tensor %s: %zu bytes, expected %zu", name, nbytes, want);
    t.bytes.assign(static_cast<const uint8_t *>(data), static_cast<const uint8_t *>(data) + nbytes);
    c->host[name] = std::move(t);
    return S2K_OK;
}

S2K_API s2k_status s2k_codec_finalize(s2k_codec *c) {
    if (!c) return fail(S2K_ERR_ARG, "NULL codec");
    if (c->ready) return S2K_OK;
    if (cudaSetDevice(c->device) != cudaSuccess) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_status rc = s2k::codec::finalize(c);
    if (rc) {  // back to the uploaded state
        for (void *p : c->allocs) cudaFree(p);
        c->allocs.clear();
        c->layers.clear();
        c->ups.clear();
        c->blocks.clear();
    }
    return rc;
}

S2K_API void s2k_codec_free(s2k_codec *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->st) cudaStreamSynchronize(c->st);
    for (void *p : c->ws_allocs) cudaFree(p);
    for (void *p : c->allocs) cudaFree(p);
    if (c->d_err) cudaFree(c->d_err);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

S2K_API s2k_status s2k_codec_get_hparams(const s2k_codec *c, s2k_codec_hparams *out) {
    if (!c || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = c->hp;
    return S2K_OK;
}

S2K_API int32_t s2k_codec_samples_per_frame(const s2k_codec *c) { return c && c->ready ? c->spf : 0; }
S2K_API int32_t s2k_codec_history_frames(const s2k_codec *c) { return c && c->ready ? c->history : 0; }
S2K_API int32_t s2k_codec_num_codebooks(const s2k_codec *c) {
    return c ? c->hp.quantizer_residual_codebooks + 1 : 0;
}
S2K_API int32_t s2k_codec_receptive_frames(const s2k_codec *c) { return c && c->ready ? c->receptive : 0; }

S2K_API s2k_status s2k_codec_decode_range(s2k_codec *c, const int32_t *codes, int32_t n_frames, int32_t emit_begin,
                                          int32_t emit_end, float *audio, size_t cap, int64_t *n_samples) {
    if (!c || !codes || !n_samples || (!audio && cap > 0)) return fail(S2K_ERR_ARG, "NULL argument");
    if (!c->ready) return fail(S2K_ERR_STATE, "codec not finalized");
    if (n_frames <= 0 || emit_begin < 0 || emit_end > n_frames || emit_begin > emit_end)
        return fail(S2K_ERR_ARG, "codec: frames [%d, %d) of a %d-frame window", emit_begin, emit_end, n_frames);
    if (cudaSetDevice(c->device) != cudaSuccess) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    return s2k::codec::decode_range(c, codes, n_frames, emit_begin, emit_end, audio, cap, n_samples, nullptr);
}

S2K_API s2k_status s2k_codec_decode(s2k_codec *c, const int32_t *codes, int32_t n_frames, float *audio, size_t cap,
                                    int64_t *n_samples) {
    if (n_frames <= 0) return fail(S2K_ERR_ARG, "codec: no frames");  // AudioCodec::decode returns false
    return s2k_codec_decode_range(c, codes, n_frames, 0, n_frames, audio, cap, n_samples);
}

S2K_API s2k_status s2k_codec_decode_windowed(s2k_codec *c, const int32_t *codes, int32_t total_frames,
                                             int32_t num_codebooks, int32_t stride_frames,
                                             int32_t context_frames_override, float *audio, size_t cap,
                                             int64_t *n_samples, double *decode_ms, int32_t *decode_batches) {
    if (!c || !codes || !audio || !n_samples) return fail(S2K_ERR_ARG, "NULL argument");
    if (!c->ready) return fail(S2K_ERR_STATE, "codec not finalized");
    if (total_frames <= 0 || num_codebooks <= 0) return fail(S2K_ERR_ARG, "codec: no frames");
    if (num_codebooks != c->nq) return fail(S2K_ERR_ARG, "codec: %d codebooks, the codec has %d", num_codebooks, c->nq);
    if (cudaSetDevice(c->device) != cudaSuccess) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const int stride = std::max(1, stride_frames > 0 ? stride_frames : 16);
    const int history = context_frames_override >= 0 ? context_frames_override : std::max(0, c->history);
    int committed = 0, batches = 0;
    int64_t written = 0;
    double ms_total = 0.0;
    auto window = [&](int avail, bool finalize) -> s2k_status {
        if (avail <= 0 || avail <= committed) return S2K_OK;
        const int stable = finalize ? avail : std::max(0, avail - history);
        if (stable <= committed && !finalize) return S2K_OK;
        const int start = std::max(0, committed - history);
        const int wframes = avail - start;
        if (wframes <= 0) return S2K_OK;
        const int eb = std::max(0, committed - start);
        const int ee = finalize ? wframes : std::min(wframes, std::max(0, stable - start));
        int64_t n = 0;
        float ms = 0.f;
        if (ee > eb) {
            s2k_status rc = s2k::codec::decode_range(c, codes + start, total_frames, eb, ee, audio + written,
                                                     cap - (size_t)written, &n, &ms);
            if (rc) return rc;
        }
        ms_total += ms;
        ++batches;
        written += n;
        committed = finalize ? avail : stable;
        return S2K_OK;
    };
    for (int avail = std::min(total_frames, stride); avail < total_frames; avail += stride) {
        s2k_status rc = window(avail, false);
        if (rc) return rc;
    }
    s2k_status rc = window(total_frames, true);
    if (rc) return rc;
    *n_samples = written;
    if (decode_ms) *decode_ms = ms_total;
    if (decode_batches) *decode_batches = batches;
    return S2K_OK;
}

struct s2k_codec_stream {
    s2k_codec *c = nullptr;
    int stride = 4, context = 0, holdback = 0;
    int committed = 0, last_decoded = 0, total = 0;
    std::vector<std::vector<int32_t>> codes;  // per codebook
    std::vector<int32_t> window;               // [nq][wframes] staging
};

S2K_API s2k_status s2k_codec_stream_create(s2k_codec *c, int32_t stride_frames, int32_t context_frames,
                                           int32_t holdback_frames, s2k_codec_stream **out) {
    if (!c || !out) return fail(S2K_ERR_ARG, "NULL argument");
    if (!c->ready) return fail(S2K_ERR_STATE, "codec not finalized");
    std::unique_ptr<s2k_codec_stream> s(new s2k_codec_stream());
    s->c = c;
    s->stride = stride_frames > 0 ? stride_frames : 4;
    s->context = context_frames >= 0 ? context_frames : std::max(0, c->history);
    s->holdback = holdback_frames >= 0 ? holdback_frames : s->context;
    s->codes.assign((size_t)c->nq, {});
    *out = s.release();
    return S2K_OK;
}

S2K_API void s2k_codec_stream_free(s2k_codec_stream *s) { delete s; }

static s2k_status stream_window(s2k_codec_stream *s, bool finalize, float *pcm, size_t cap, int64_t *n_pcm) {
    *n_pcm = 0;
    const int total = s->total;
    if (total <= 0 || total <= s->committed) return S2K_OK;
    const int stable = finalize ? total : std::max(0, total - s->holdback);
    if (stable <= s->committed && !finalize) return S2K_OK;
    const int start = std::max(0, s->committed - s->context);
    const int wframes = total - start;
    if (wframes <= 0) return S2K_OK;
    const int nq = s->c->nq;
    s->window.resize((size_t)nq * wframes);
    for (int q = 0; q < nq; ++q)
        std::copy(s->codes[(size_t)q].begin() + start, s->codes[(size_t)q].begin() + total,
                  s->window.begin() + (size_t)q * wframes);
    const int eb = std::max(0, s->committed - start);
    const int ee = finalize ? wframes : std::min(wframes, std::max(0, stable - start));
    if (ee > eb) {
        if (cudaSetDevice(s->c->device) != cudaSuccess) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
        s2k_status rc = s2k::codec::decode_range(s->c, s->window.data(), wframes, eb, ee, pcm, cap, n_pcm, nullptr);
        if (rc) return rc;
    }
    s->committed = finalize ? total : stable;
    s->last_decoded = total;
    return S2K_OK;
}

S2K_API s2k_status s2k_codec_stream_push(s2k_codec_stream *s, const int32_t *frame_codes, float *pcm, size_t cap,
                                         int64_t *n_pcm) {
    if (!s || !frame_codes || !n_pcm) return fail(S2K_ERR_ARG, "NULL argument");
    *n_pcm = 0;
    for (int q = 0; q < s->c->nq; ++q) s->codes[(size_t)q].push_back(frame_codes[q]);
    ++s->total;
    if (s->total - s->last_decoded < s->stride) return S2K_OK;
    return stream_window(s, false, pcm, cap, n_pcm);
}

S2K_API s2k_status s2k_codec_stream_finish(s2k_codec_stream *s, float *pcm, size_t cap, int64_t *n_pcm) {
    if (!s || !n_pcm) return fail(S2K_ERR_ARG, "NULL argument");
    *n_pcm = 0;
    if (s->total > s->last_decoded || s->committed < s->total) return stream_window(s, true, pcm, cap, n_pcm);
    return S2K_OK;
}

S2K_API int64_t s2k_codec_stream_max_release(const s2k_codec_stream *s) {
    if (!s) return 0;
    return (int64_t)(s->total + 1 - s->committed) * s->c->spf;
}
