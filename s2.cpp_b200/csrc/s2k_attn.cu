// s2k_attn.cu -- per-head QK-norm + RoPE + KV store, and GQA flash-decode
// attention over a paged f16 KV cache plus the current call's f32 K/V.
//
// Reference semantics (src/s2_model.cpp:970-1039 Slow, 1163-1212 Fast):
//   q/k per-head rms_norm_weighted (eps, q_norm / k_norm)      :979-982
//   ggml_rope_ext mode 0, n_dims = head_dim, freq_scale 1,
//     theta = pos * theta_scale^i by repeated multiplication  :984-989
//   K/V of this call stored as f16 at n_past                   :991-1005
//   keys/values: past from the f16 cache (f16 -> f32), this
//     call's tokens from the un-rounded f32 projections        :1007-1020
//   GQA: query head h reads kv head h / (H/Hkv)                :57-68
//   softmax((K.Q) * 1/sqrt(hd), causal from n_past) . V        :1023-1039
#include "s2k_common.cuh"
#include "s2k_kernels.h"

namespace s2k {

// grid (T, H + 2*Hkv), block hd/2: thread i owns the pair (2i, 2i+1).
__global__ void qk_prep_kernel(QkPrepArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && *a.done) return;
    const int t = blockIdx.x, y = blockIdx.y, i = threadIdx.x, hd = a.hd;
    float *row = a.qkv + (size_t)t * a.ldqkv;
    const int pos = (a.pos_base ? *a.pos_base : 0) + a.pos_add + t;
    const bool isq = y < a.H;
    const bool isk = !isq && y < a.H + a.Hkv;
    const int head = isq ? y : (isk ? y - a.H : y - a.H - a.Hkv);
    float *v = row + (isq ? head * hd : (isk ? (a.H + head) * hd : (a.H + a.Hkv + head) * hd));
    float x0 = v[2 * i], x1 = v[2 * i + 1];
    if (isq || isk) {
        const float *nw = isq ? a.q_norm : a.k_norm;
        if (nw) {
            __shared__ double red[8];
            double s = (double)__fmul_rn(x0, x0) + (double)__fmul_rn(x1, x1);
            s = warp_sum_d(s);
            if ((i & 31) == 0) red[i >> 5] = s;
            __syncthreads();
            double tot = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
            const float mean = (float)(tot / (double)hd);
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            x0 = __fmul_rn(__fmul_rn(x0, sc), nw[2 * i]);
            x1 = __fmul_rn(__fmul_rn(x1, sc), nw[2 * i + 1]);
        }
        float theta = (float)pos;
        for (int k = 0; k < i; ++k) theta = __fmul_rn(theta, a.theta_scale);
        const float c = cosf(theta), s = sinf(theta);
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        x0 = y0;
        x1 = y1;
    }
    if (isq) {
        v[2 * i] = x0;
        v[2 * i + 1] = x1;
        return;
    }
    float *cur = (isk ? a.kcur : a.vcur) + ((size_t)(a.cur_base + t) * a.Hkv + head) * hd;
    cur[2 * i] = x0;
    cur[2 * i + 1] = x1;
    if (a.kv.k) {
        const int pg = pos / kPage, slot = pos % kPage;
        if (pos < 0 || pg >= a.kv.n_pages) {
            if (i == 0 && a.err) atomicOr(a.err, ERR_BAD_POS);
            return;
        }
        const int page = a.kv.block_table[pg];
        __half *dst = (isk ? a.kv.k : a.kv.v) +
                      ((((size_t)page * a.kv.n_layers + a.layer) * a.kv.n_kv_heads + head) * kPage + slot) * hd;
        dst[2 * i] = __float2half_rn(x0);
        dst[2 * i + 1] = __float2half_rn(x1);
    }
}

cudaError_t launch_qk_prep(const QkPrepArgs &a, cudaStream_t st) {
    if (a.hd % 64 != 0 || a.hd > 256) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.T, a.H + 2 * a.Hkv);
    cfg.blockDim = dim3(a.hd / 2);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, qk_prep_kernel, a);
}

// grid (Hkv, T, n_splits), block 128 (4 warps).  Each CTA covers the G query
// heads of one kv head over one slice of keys, keeping an online softmax per
// head; the last CTA of a (token, kv head) merges the slices in split order.
constexpr int kAttnWarps = 4;
constexpr int kMaxGroup = 8;

template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(AttnArgs a) {
    constexpr int DPL = HD / 32;  // dims per lane
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && *a.done) return;
    const int g = blockIdx.x, t = blockIdx.y, sp = blockIdx.z;
    const int G = a.H / a.Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = a.n_cached ? *a.n_cached : 0;
    const int Lk = nc + a.cur_base + t + 1;
    const int j0 = (int)(((long long)Lk * sp) / a.n_splits);
    const int j1 = (int)(((long long)Lk * (sp + 1)) / a.n_splits);

    float q[kMaxGroup][DPL], acc[kMaxGroup][DPL], m[kMaxGroup], l[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int d = 0; d < DPL; ++d) {
            acc[h][d] = 0.f;
            q[h][d] = (h < G) ? a.q[(size_t)t * a.ldq + (size_t)(g * G + h) * HD + lane * DPL + d] : 0.f;
        }
    }
    for (int j = j0 + warp; j < j1; j += kAttnWarps) {
        float kv_k[DPL], kv_v[DPL];
        if (j < nc) {
            const int page = a.kv.block_table[j / kPage], slot = j % kPage;
            const size_t off = ((((size_t)page * a.kv.n_layers + a.layer) * a.kv.n_kv_heads + g) * kPage + slot) * HD +
                               lane * DPL;
#pragma unroll
            for (int d = 0; d < DPL; ++d) {
                kv_k[d] = __half2float(a.kv.k[off + d]);
                kv_v[d] = __half2float(a.kv.v[off + d]);
            }
        } else {
            const size_t off = ((size_t)(j - nc) * a.Hkv + g) * HD + lane * DPL;
#pragma unroll
            for (int d = 0; d < DPL; ++d) {
                kv_k[d] = a.kcur[off + d];
                kv_v[d] = a.vcur[off + d];
            }
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h < G) {
                float s = 0.f;
#pragma unroll
                for (int d = 0; d < DPL; ++d) s += kv_k[d] * q[h][d];
                s = warp_sum(s) * a.scale;
                const float mn = fmaxf(m[h], s);
                const float corr = expf(m[h] - mn);
                const float p = expf(s - mn);
                l[h] = l[h] * corr + p;
#pragma unroll
                for (int d = 0; d < DPL; ++d) acc[h][d] = acc[h][d] * corr + p * kv_v[d];
                m[h] = mn;
            }
        }
    }

    // merge the 4 warps
    __shared__ float s_m[kAttnWarps][kMaxGroup], s_l[kAttnWarps][kMaxGroup];
    __shared__ float s_acc[kAttnWarps][kMaxGroup][HD];
    __shared__ int s_last;
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            s_m[warp][h] = m[h];
            s_l[warp][h] = l[h];
        }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
#pragma unroll
        for (int d = 0; d < DPL; ++d) s_acc[warp][h][lane * DPL + d] = acc[h][d];
    __syncthreads();
    const int NS = a.n_splits;
    for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w][h]);
        const size_t base = (((size_t)t * a.H + g * G + h) * NS + sp) * (HD + 2);
        for (int d = threadIdx.x; d < HD; d += blockDim.x) {
            float A = 0.f;
            if (M != -INFINITY)
                for (int w = 0; w < kAttnWarps; ++w) A += s_acc[w][h][d] * expf(s_m[w][h] - M);
            a.part[base + d] = A;
        }
        if (threadIdx.x == 0) {
            float Ls = 0.f;
            if (M != -INFINITY)
                for (int w = 0; w < kAttnWarps; ++w) Ls += s_l[w][h] * expf(s_m[w][h] - M);
            a.part[base + HD] = M;
            a.part[base + HD + 1] = Ls;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int old = atomicAdd(&a.counters[t * a.Hkv + g], 1);
        s_last = (old == NS - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int h = 0; h < G; ++h) {
        const size_t hb = ((size_t)t * a.H + g * G + h) * NS * (HD + 2);
        float M = -INFINITY;
        for (int s = 0; s < NS; ++s) M = fmaxf(M, __ldcg(&a.part[hb + s * (HD + 2) + HD]));
        float Ls = 0.f;
        for (int s = 0; s < NS; ++s) {
            const float ms = __ldcg(&a.part[hb + s * (HD + 2) + HD]);
            if (ms != -INFINITY) Ls += __ldcg(&a.part[hb + s * (HD + 2) + HD + 1]) * expf(ms - M);
        }
        for (int d = threadIdx.x; d < HD; d += blockDim.x) {
            float A = 0.f;
            for (int s = 0; s < NS; ++s) {
                const float ms = __ldcg(&a.part[hb + s * (HD + 2) + HD]);
                if (ms != -INFINITY) A += __ldcg(&a.part[hb + s * (HD + 2) + d]) * expf(ms - M);
            }
            a.out[(size_t)t * a.H * HD + (size_t)(g * G + h) * HD + d] = A / Ls;
        }
    }
    if (threadIdx.x == 0) a.counters[t * a.Hkv + g] = 0;
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) {
    if (a.hd != 128 || a.H % a.Hkv != 0 || a.H / a.Hkv > kMaxGroup || a.n_splits < 1) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.Hkv, a.T, a.n_splits);
    cfg.blockDim = dim3(kAttnWarps * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, attn_kernel<128>, a);
}

}  // namespace s2k
