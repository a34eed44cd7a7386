// s2k_common.cuh -- shared device helpers for the sm_100a decode kernels:
// mbarrier / bulk-async-copy wrappers, programmatic dependent launch,
// bounded waits and the error-flag convention.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace s2k {

// Error bits a kernel ORs into the model's device error word.
enum : int {
    ERR_WAIT_FULL = 1,    // consumer gave up waiting for a weight stage
    ERR_WAIT_EMPTY = 2,   // producer gave up waiting for a free stage
    ERR_BAD_TOKEN = 4,    // token / code id out of range
    ERR_BAD_POS = 8,      // position beyond the sequence's pages
    ERR_SAMPLER = 16,     // sampler found no finite candidate
    ERR_GRID = 32,        // a grid barrier of the persistent kernel timed out
};

// ~2 s at 1.9 GHz: long enough never to fire on a healthy GPU, short enough
// that a lost copy turns into an error status instead of a hang.
constexpr long long kWaitLimitCycles = 4000000000LL;

// The model's error block: int word 0 holds the error bits, the 8-byte word
// at int offset 2 the wait limit in SM cycles (0 = kWaitLimitCycles).  Every
// kernel gets a pointer to word 0; s2k_model_set_wait_limit writes the limit.
constexpr int kErrBlockInts = 4;

__device__ __forceinline__ long long wait_limit(const int *err) {
    if (err == nullptr) return kWaitLimitCycles;
    const long long v = *reinterpret_cast<const volatile long long *>(err + 2);
    return v > 0 ? v : kWaitLimitCycles;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Polls of a bounded wait between looks at the error word: that look is a
// global-memory round trip, so it stays off the fast path of a wait.
constexpr unsigned kErrPollEvery = 64;

// Bounded wait on an mbarrier phase.  Returns false (and sets `code` in *err)
// when the limit is reached.  Once some wait has timed out (an error flag is
// set), the copies the others wait for will not come either: they give up at
// their next look at the error word instead of each spending the full limit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_test(bar, parity)) return true;
    const long long t0 = clock64(), lim = wait_limit(err);
    for (unsigned it = 1; !mbar_test(bar, parity); ++it) {
        if (clock64() - t0 > lim) {
            if (err) atomicOr(err, code);
            return false;
        }
        if (err && it % kErrPollEvery == 0 &&
            (*reinterpret_cast<volatile int *>(err) & (ERR_WAIT_FULL | ERR_WAIT_EMPTY | ERR_GRID)))
            return false;
    }
    return true;
}

// 1-D bulk async copy global -> shared (TMA engine, no tensor map), completing
// `bytes` of transaction count on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
// Weights are read once per pass: hint L2 to evict them first.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 1-D bulk async copy global -> shared with the default L2 policy.
__device__ __forceinline__ void bulk_g2s_plain(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk L2 prefetch of [src, src + bytes) (no completion tracking): the TMA
// engine pulls the range from HBM into L2 so a later bulk copy hits L2.
// src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Programmatic dependent launch (PDL): let the next kernel in the stream start
// its weight prefetch now; wait for the previous kernel's results later.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier among the first `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// ggml-cpu x86 quantize_row_q8_0 on one 32-value block held one value per
// lane: d = amax/127 (stored fp16), q = round-half-even(x * 127/amax).
// Returns q for this lane; *d_out (all lanes) gets the fp16-rounded scale.
__device__ __forceinline__ int quant_q8_0_lane(float v, float *d_out) {
    const float amax = warp_max(fabsf(v));
    const float d = __fdiv_rn(amax, 127.f);
    const float id = amax != 0.0f ? __fdiv_rn(127.f, amax) : 0.0f;
    *d_out = __half2float(__float2half_rn(d));
    return __float2int_rn(__fmul_rn(v, id));
}

// exp(x) for float x with a fixed sequence of IEEE float operations, so the
// CUDA kernels and the CPU oracle (oracle/s2_oracle.c, det_expf) return the
// same bits: Cody-Waite reduction x = k*ln2 + r (ln2 split so k*LN2_HI is
// exact), exp(r) by its Taylor series to degree 7 (|r| <= ln2/2, truncation
// < 1e-8 relative), then scaling by 2^k as two products by powers of two
// (p * 2^(k-h) is exact and normal for every k in [-150, 128], the product
// by 2^h rounds once, into the subnormals when k < -126): the correctly
// rounded p * 2^k, i.e. ldexpf's result, at a fraction of its cost.
__device__ __forceinline__ float pow2_scale(float p, int k) {
    const int h = k < -100 ? -64 : (k > 100 ? 64 : 0);
    return __fmul_rn(__fmul_rn(p, __int_as_float((k - h + 127) << 23)), __int_as_float((h + 127) << 23));
}

__device__ __forceinline__ float det_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float k = rintf(__fmul_rn(x, 1.44269502162933349609f));
    const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(k, 0.693145751953125f)), __fmul_rn(k, 1.42860682030941723212e-6f));
    float p = 1.98412698412698412526e-4f;  // 1/5040
    p = __fadd_rn(__fmul_rn(p, r), 1.38888888888888894189e-3f);  // 1/720
    p = __fadd_rn(__fmul_rn(p, r), 8.33333333333333321769e-3f);  // 1/120
    p = __fadd_rn(__fmul_rn(p, r), 4.16666666666666643537e-2f);  // 1/24
    p = __fadd_rn(__fmul_rn(p, r), 1.66666666666666657415e-1f);  // 1/6
    p = __fadd_rn(__fmul_rn(p, r), 0.5f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    return pow2_scale(p, (int)k);
}

// sin(x) for float x with a fixed sequence of IEEE float operations, so the
// CUDA kernels and the CPU oracle (oracle/s2_oracle.c, so_det_sinf) return the
// same bits: Cody-Waite reduction x = k*pi + r (pi split in three parts, k*P1
// and k*P2 exact for |k| <= 2048), sin(r) by its Taylor series to degree 13
// (|r| <= pi/2: truncation < 7e-10), negated for odd k.  Beyond |x| = 6400
// (outside the reduction's exact range) it is the library sinf.
__device__ __forceinline__ float det_sinf(float x) {
    if (!(fabsf(x) <= 6400.0f)) return sinf(x);
    const float k = rintf(__fmul_rn(x, 0.318309873342514038f));
    float r = __fsub_rn(x, __fmul_rn(k, 3.140625f));
    r = __fsub_rn(r, __fmul_rn(k, 9.6750259399414062e-4f));
    r = __fsub_rn(r, __fmul_rn(k, 1.5099580252808664e-7f));
    const float r2 = __fmul_rn(r, r);
    float p = 1.60590443720742825917e-10f;                    // 1/13!
    p = __fadd_rn(__fmul_rn(p, r2), -2.50521079436794025241e-8f);  // -1/11!
    p = __fadd_rn(__fmul_rn(p, r2), 2.75573188446287531406e-6f);   // 1/9!
    p = __fadd_rn(__fmul_rn(p, r2), -1.98412701138295233250e-4f);  // -1/7!
    p = __fadd_rn(__fmul_rn(p, r2), 8.33333376795053482056e-3f);   // 1/5!
    p = __fadd_rn(__fmul_rn(p, r2), -1.66666671633720397949e-1f);  // -1/3!
    const float v = __fadd_rn(r, __fmul_rn(__fmul_rn(r, r2), p));
    return ((int)k & 1) ? -v : v;
}

// x / (1 + exp(-x)), ggml_silu_f32
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, det_expf(-x))); }

}  // namespace s2k
