// s2k_attn.cu -- per-head QK-norm + RoPE + KV store, and GQA decode/prefill
// attention over a paged f16 KV cache plus the current call's f32 K/V.
//
// Reference semantics (src/s2_model.cpp:970-1039 Slow, 1163-1212 Fast):
//   q/k per-head rms_norm_weighted (eps, q_norm / k_norm)      :979-982
//   ggml_rope_ext mode 0, n_dims = head_dim, freq_scale 1       :984-989
//     (cos/sin come from a table the host builds with ggml's recurrence
//      theta_i = theta_{i-1} * base^(-2/n_dims), theta_0 = pos)
//   K/V of this call stored as f16 at n_past                   :991-1005
//   keys/values: past from the f16 cache (f16 -> f32), this
//     call's tokens from the un-rounded f32 projections        :1007-1020
//   GQA: query head h reads kv head h / (H/Hkv)                :57-68
//   softmax((K.Q) * 1/sqrt(hd), causal from n_past) . V        :1023-1039
//
// Arithmetic (shared with the CPU oracle so the two agree bit for bit):
//   s_j  = float(sum_d double(k_j[d]) * double(q[d])) * scale
//   p_j  = det_expf(s_j - max_j s_j),  inv = float(1 / sum_j double(p_j))
//   out  = float(sum_j double(v_j[d]) * double(p_j * inv))
// Products of two floats are exact in double and the double sums are rounded
// to float once, so the split over CTAs does not change the result.
//
// Two kernels per layer: attn_scores (scores + last-CTA softmax statistics)
// and attn_values (weighted values + last-CTA merge of the splits).
#include "s2k_common.cuh"
#include "s2k_kernels.h"

namespace s2k {

// grid (T, H + 2*Hkv), block hd/2: thread i owns the pair (2i, 2i+1).
__global__ void qk_prep_kernel(QkPrepArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    const int t = blockIdx.x, y = blockIdx.y, i = threadIdx.x, hd = a.hd;
    float *row = a.qkv + (size_t)t * a.ldqkv;
    const int pos = (a.pos_base ? __ldcg(a.pos_base) : 0) + a.pos_add + t;
    const bool isq = y < a.H;
    const bool isk = !isq && y < a.H + a.Hkv;
    const int head = isq ? y : (isk ? y - a.H : y - a.H - a.Hkv);
    float *v = row + (isq ? head * hd : (isk ? (a.H + head) * hd : (a.H + a.Hkv + head) * hd));
    float x0 = __ldcg(v + 2 * i), x1 = __ldcg(v + 2 * i + 1);
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
        if (pos < 0 || pos >= a.rope_positions) {
            if (i == 0 && a.err) atomicOr(a.err, ERR_BAD_POS);
            return;
        }
        const float2 cs = a.rope[(size_t)pos * (hd / 2) + i];  // (cos, sin)
        const float y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
        const float y1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
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
        const int page = __ldcg(a.kv.block_table + pg);
        __half *dst = (isk ? a.kv.k : a.kv.v) +
                      ((((size_t)page * a.kv.n_layers + a.layer) * a.kv.n_kv_heads + head) * kPage + slot) * hd;
        dst[2 * i] = __float2half_rn(x0);
        dst[2 * i + 1] = __float2half_rn(x1);
    }
}

static cudaLaunchConfig_t pdl_cfg(dim3 g, dim3 b, size_t smem, cudaStream_t st, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = g;
    cfg.blockDim = b;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

cudaError_t launch_qk_prep(const QkPrepArgs &a, cudaStream_t st) {
    if (a.hd % 64 != 0 || a.hd > 256 || !a.rope) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.T, a.H + 2 * a.Hkv), dim3(a.hd / 2), 0, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, qk_prep_kernel, a);
}

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kMaxGroup = 8;

__device__ __forceinline__ void key_range(const AttnArgs &a, int t, int sp, int nc, int *Lk, int *j0, int *j1) {
    *Lk = nc + a.cur_base + t + 1;
    *j0 = (int)(((long long)*Lk * sp) / a.n_splits);
    *j1 = (int)(((long long)*Lk * (sp + 1)) / a.n_splits);
}

template <int HD>
__device__ __forceinline__ void load_kv_row(const AttnArgs &a, const __half *cache, const float *cur, int j, int nc,
                                            int g, int lane, float out[HD / 32]) {
    constexpr int DPL = HD / 32;
    if (j < nc) {
        const int page = __ldcg(a.kv.block_table + j / kPage), slot = j % kPage;
        const size_t off =
            ((((size_t)page * a.kv.n_layers + a.layer) * a.kv.n_kv_heads + g) * kPage + slot) * HD + lane * DPL;
#pragma unroll
        for (int d = 0; d < DPL; ++d) out[d] = __half2float(__ldcg(cache + off + d));
    } else {
        const size_t off = ((size_t)(j - nc) * a.Hkv + g) * HD + lane * DPL;
#pragma unroll
        for (int d = 0; d < DPL; ++d) out[d] = __ldcg(cur + off + d);
    }
}

// grid (Hkv, T, n_splits).  Writes s_j for the split's keys; the last CTA of a
// (token, kv head) computes max_j s_j and inv = 1/sum_j exp(s_j - max) per head.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_scores_kernel(AttnArgs a) {
    constexpr int DPL = HD / 32;
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    const int g = blockIdx.x, t = blockIdx.y, sp = blockIdx.z;
    const int G = a.H / a.Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = a.n_cached ? __ldcg(a.n_cached) : 0;
    int Lk, j0, j1;
    key_range(a, t, sp, nc, &Lk, &j0, &j1);
    float q[kMaxGroup][DPL];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
#pragma unroll
        for (int d = 0; d < DPL; ++d)
            q[h][d] = (h < G) ? __ldcg(a.q + (size_t)t * a.ldq + (size_t)(g * G + h) * HD + lane * DPL + d) : 0.f;
    float *scores = a.scores + ((size_t)t * a.H + (size_t)g * G) * a.ld_scores;
    for (int j = j0 + warp; j < j1; j += kAttnWarps) {
        float k[DPL];
        load_kv_row<HD>(a, a.kv.k, a.kcur, j, nc, g, lane, k);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h < G) {
                double s = 0.0;
#pragma unroll
                for (int d = 0; d < DPL; ++d) s += (double)k[d] * (double)q[h][d];
                s = warp_sum_d(s);
                if (lane == 0) scores[(size_t)h * a.ld_scores + j] = __fmul_rn((float)s, a.scale);
            }
        }
    }
    __shared__ int s_last;
    __shared__ float s_red[kAttnWarps];
    __shared__ double s_dred[kAttnWarps];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[t * a.Hkv + g], 1) == a.n_splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int h = 0; h < G; ++h) {
        const float *sh = scores + (size_t)h * a.ld_scores;
        float mx = -INFINITY;
        for (int j = threadIdx.x; j < Lk; j += kAttnThreads) mx = fmaxf(mx, __ldcg(sh + j));
        mx = warp_max(mx);
        if (lane == 0) s_red[warp] = mx;
        __syncthreads();
        mx = s_red[0];
        for (int w = 1; w < kAttnWarps; ++w) mx = fmaxf(mx, s_red[w]);
        double sum = 0.0;
        for (int j = threadIdx.x; j < Lk; j += kAttnThreads) sum += (double)det_expf(__fsub_rn(__ldcg(sh + j), mx));
        sum = warp_sum_d(sum);
        if (lane == 0) s_dred[warp] = sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            double tot = 0.0;
            for (int w = 0; w < kAttnWarps; ++w) tot += s_dred[w];
            float *st = a.stats + ((size_t)t * a.H + g * G + h) * 2;
            st[0] = mx;
            st[1] = (float)(1.0 / tot);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) a.counters[t * a.Hkv + g] = 0;
}

// grid (Hkv, T, n_splits).  Accumulates double(v_j) * double(p_j * inv) over the
// split's keys; the last CTA of a (token, kv head) sums the splits in order.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_values_kernel(AttnArgs a) {
    constexpr int DPL = HD / 32;
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    const int g = blockIdx.x, t = blockIdx.y, sp = blockIdx.z;
    const int G = a.H / a.Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = a.n_cached ? __ldcg(a.n_cached) : 0;
    int Lk, j0, j1;
    key_range(a, t, sp, nc, &Lk, &j0, &j1);
    float mx[kMaxGroup], inv[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
        mx[h] = h < G ? __ldcg(a.stats + ((size_t)t * a.H + g * G + h) * 2) : 0.f;
        inv[h] = h < G ? __ldcg(a.stats + ((size_t)t * a.H + g * G + h) * 2 + 1) : 0.f;
    }
    const float *scores = a.scores + ((size_t)t * a.H + (size_t)g * G) * a.ld_scores;
    double acc[kMaxGroup][DPL];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[h][d] = 0.0;
    for (int j = j0 + warp; j < j1; j += kAttnWarps) {
        float v[DPL];
        load_kv_row<HD>(a, a.kv.v, a.vcur, j, nc, g, lane, v);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h < G) {
                const float p = __fmul_rn(det_expf(__fsub_rn(__ldcg(scores + (size_t)h * a.ld_scores + j), mx[h])), inv[h]);
#pragma unroll
                for (int d = 0; d < DPL; ++d) acc[h][d] += (double)v[d] * (double)p;
            }
        }
    }
    __shared__ double s_acc[kAttnWarps][HD];
    __shared__ int s_last;
    double *part = a.part + ((size_t)t * a.H + (size_t)g * G) * a.n_splits * HD;
    for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int d = 0; d < DPL; ++d) s_acc[warp][lane * DPL + d] = acc[h][d];
        __syncthreads();
        for (int d = threadIdx.x; d < HD; d += kAttnThreads) {
            double s = s_acc[0][d];
            for (int w = 1; w < kAttnWarps; ++w) s += s_acc[w][d];
            part[((size_t)h * a.n_splits + sp) * HD + d] = s;
        }
        __syncthreads();
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.counters2[t * a.Hkv + g], 1) == a.n_splits - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int h = 0; h < G; ++h)
        for (int d = threadIdx.x; d < HD; d += kAttnThreads) {
            double s = 0.0;
            for (int k = 0; k < a.n_splits; ++k) s += __ldcg(part + ((size_t)h * a.n_splits + k) * HD + d);
            a.out[(size_t)t * a.H * HD + (size_t)(g * G + h) * HD + d] = (float)s;
        }
    if (threadIdx.x == 0) a.counters2[t * a.Hkv + g] = 0;
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) {
    if (a.hd != 128 || a.H % a.Hkv != 0 || a.H / a.Hkv > kMaxGroup || a.n_splits < 1 || !a.scores || !a.stats ||
        !a.part || !a.counters || !a.counters2)
        return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.Hkv, a.T, a.n_splits), dim3(kAttnThreads), 0, st, attr);
    count_launch();
    cudaError_t e = cudaLaunchKernelEx(&cfg, attn_scores_kernel<128>, a);
    if (e != cudaSuccess) return e;
    count_launch();
    return cudaLaunchKernelEx(&cfg, attn_values_kernel<128>, a);
}

}  // namespace s2k
