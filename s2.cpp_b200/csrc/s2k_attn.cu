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
// Arithmetic (shared with the CPU oracle so the two agree bit for bit): keys
// are taken in fixed splits of kAttnSplit (64) positions,
//   s_j  = float(sum_d double(k_j[d]) * double(q[d])) * scale
//   split i: m_i = max s_j,  e_j = det_expf(s_j - m_i),
//            S_i = sum double(e_j),  O_i[d] = sum double(v_j[d]) * double(e_j)
//   M = max_i m_i,  w_i = det_expf(m_i - M)
//   out  = float((sum_i O_i[d] * double(w_i)) / (sum_i S_i * double(w_i)))
// i.e. softmax . V with the exponentials factored per split.  Products of two
// floats are exact in double and every double sum is rounded to float once,
// so the order of the sums inside a split does not change the result.
//
// One kernel per layer: attn_split_kernel, one CTA per (kv head, token) that
// walks the splits in order (scores, split maxima, then per split the
// exponentials, S_i and O_i folded into the running sums with w_i).
#include "s2k_common.cuh"
#include "s2k_device.h"
#include "s2k_kernels.h"

namespace s2k {

// KV pages of a batched call's sequence (constant while the sequence lives).
__device__ __forceinline__ KvPaged seq_kv(const SeqDev *sd) {
    KvPaged kv;
    kv.k = sd->kv.k;
    kv.v = sd->kv.v;
    kv.block_table = sd->kv.block_table;
    kv.n_layers = sd->kv.n_layers;
    kv.n_kv_heads = sd->kv.n_kv_heads;
    kv.head_dim = sd->kv.head_dim;
    kv.n_pages = sd->kv.n_pages;
    return kv;
}

// grid (T, H + 2*Hkv), block hd/2: thread i owns the pair (2i, 2i+1).
__global__ void qk_prep_kernel(QkPrepArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    const int t = blockIdx.x, y = blockIdx.y, i = threadIdx.x, hd = a.hd;
    float *row = a.qkv + (size_t)t * a.ldqkv;
    int pos, cur_row;
    KvPaged kv = a.kv;
    if (a.rows) {
        const BatchRow r = a.rows[t];
        const SeqDev *sd = a.seqs ? a.seqs[r.slot] : nullptr;
        pos = (sd ? __ldcg(&sd->state.n_past) : 0) + r.off;
        cur_row = r.cur_hi;
        if (sd) kv = seq_kv(sd);
    } else {
        pos = (a.pos_base ? __ldcg(a.pos_base) : 0) + a.pos_add + t;
        cur_row = a.cur_base + t;
    }
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
    float *cur = (isk ? a.kcur : a.vcur) + ((size_t)cur_row * a.Hkv + head) * hd;
    cur[2 * i] = x0;
    cur[2 * i + 1] = x1;
    if (kv.k) {
        const int pg = pos / kPage, slot = pos % kPage;
        if (pos < 0 || pg >= kv.n_pages) {
            if (i == 0 && a.err) atomicOr(a.err, ERR_BAD_POS);
            return;
        }
        const int page = __ldcg(kv.block_table + pg);
        __half *dst = (isk ? kv.k : kv.v) +
                      ((((size_t)page * kv.n_layers + a.layer) * kv.n_kv_heads + head) * kPage + slot) * hd;
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

// Key / value row j of a CTA's key range: positions j < nc from the paged
// cache, later ones from this call's f32 rows (cur holds the range's first).
__device__ __forceinline__ void load_kv_row(const AttnArgs &a, const KvPaged &kv, const __half *cache,
                                            const float *cur, int j, int nc, int g, int lane, float out[4]) {
    if (j < nc) {
        const int page = __ldcg(kv.block_table + j / kPage), slot = j % kPage;
        const size_t off =
            ((((size_t)page * kv.n_layers + a.layer) * kv.n_kv_heads + g) * kPage + slot) * 128 + lane * 4;
        const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(cache + off));
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        out[0] = f0.x;
        out[1] = f0.y;
        out[2] = f1.x;
        out[3] = f1.y;
    } else {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(cur + ((size_t)(j - nc) * a.Hkv + g) * 128) + lane);
        out[0] = v.x;
        out[1] = v.y;
        out[2] = v.z;
        out[3] = v.w;
    }
}

// Dynamic shared memory of attn_split_kernel for G query heads per kv head
// and at most nsp splits.
size_t attn_split_smem(int G, int nsp) {
    return (size_t)kAttnWarps * G * 128 * sizeof(double)  // per-warp O_i partials
           + (size_t)G * kAttnSplit * sizeof(float)        // e_j of the split
           + (size_t)G * nsp * sizeof(float);              // split maxima m_i
}

// grid (Hkv, T), block kAttnThreads; hd = 128 (lane owns dims 4*lane..4*lane+3).
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(AttnArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    extern __shared__ __align__(16) uint8_t smem[];
    const int g = blockIdx.x, t = blockIdx.y;
    const int G = a.H / a.Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int nc, Lk;
    KvPaged kv = a.kv;
    const float *kc = a.kcur, *vc = a.vcur;
    if (a.rows) {
        const BatchRow r = a.rows[t];
        const SeqDev *sd = a.seqs ? a.seqs[r.slot] : nullptr;
        nc = sd ? __ldcg(&sd->state.n_past) : 0;
        if (sd) kv = seq_kv(sd);
        kc += (size_t)r.cur_lo * a.Hkv * 128;
        vc += (size_t)r.cur_lo * a.Hkv * 128;
        Lk = nc + r.cur_hi - r.cur_lo + 1;
    } else {
        nc = a.n_cached ? __ldcg(a.n_cached) : 0;
        Lk = nc + a.cur_base + t + 1;
    }
    if (Lk < 1 || Lk > a.ld_scores || Lk > a.max_keys || (nc > 0 && (nc - 1) / kPage >= kv.n_pages)) {
        if (tid == 0 && a.err) atomicOr(a.err, ERR_BAD_POS);
        return;
    }
    const int nsp = (Lk + kAttnSplit - 1) / kAttnSplit;
    double *red = reinterpret_cast<double *>(smem);                    // [kAttnWarps][G][128]
    float *ebuf = reinterpret_cast<float *>(red + kAttnWarps * G * 128);  // [G][kAttnSplit]
    float *msp = ebuf + G * kAttnSplit;                                 // [G][nsp]
    float q[kMaxGroup][4];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
#pragma unroll
        for (int d = 0; d < 4; ++d)
            q[h][d] = (h < G) ? __ldcg(a.q + (size_t)t * a.ldq + (size_t)(g * G + h) * 128 + lane * 4 + d) : 0.f;
    float *scores = a.scores + ((size_t)t * a.H + (size_t)g * G) * a.ld_scores;
    // pass A: every score of the key range
    for (int j = warp; j < Lk; j += kAttnWarps) {
        float k[4];
        load_kv_row(a, kv, kv.k, kc, j, nc, g, lane, k);
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
            if (h < G) {
                double s = 0.0;
#pragma unroll
                for (int d = 0; d < 4; ++d) s += (double)k[d] * (double)q[h][d];
                s = warp_sum_d(s);
                if (lane == 0) scores[(size_t)h * a.ld_scores + j] = __fmul_rn((float)s, a.scale);
            }
    }
    __syncthreads();
    // split maxima
    for (int p = tid; p < G * nsp; p += kAttnThreads) {
        const int h = p / nsp, i = p - h * nsp;
        const int j0 = i * kAttnSplit, j1 = min(j0 + kAttnSplit, Lk);
        float mx = -INFINITY;
        for (int j = j0; j < j1; ++j) mx = fmaxf(mx, scores[(size_t)h * a.ld_scores + j]);
        msp[h * nsp + i] = mx;
    }
    __syncthreads();
    // pass B: thread tid owns output dim d = tid of every head
    double acc[kMaxGroup], ssum[kMaxGroup];
    float M[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
        acc[h] = 0.0;
        ssum[h] = 0.0;
        M[h] = -INFINITY;
        if (h < G)
            for (int i = 0; i < nsp; ++i) M[h] = fmaxf(M[h], msp[h * nsp + i]);
    }
    for (int i = 0; i < nsp; ++i) {
        const int j0 = i * kAttnSplit, cnt = min(kAttnSplit, Lk - j0);
        for (int p = tid; p < G * kAttnSplit; p += kAttnThreads) {
            const int h = p / kAttnSplit, jj = p - h * kAttnSplit;
            ebuf[p] = jj < cnt ? det_expf(__fsub_rn(scores[(size_t)h * a.ld_scores + j0 + jj], msp[h * nsp + i])) : 0.f;
        }
        __syncthreads();
        double o[kMaxGroup][4];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
#pragma unroll
            for (int d = 0; d < 4; ++d) o[h][d] = 0.0;
        for (int jj = warp; jj < cnt; jj += kAttnWarps) {
            float v[4];
            load_kv_row(a, kv, kv.v, vc, j0 + jj, nc, g, lane, v);
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h)
                if (h < G) {
                    const double e = (double)ebuf[h * kAttnSplit + jj];
#pragma unroll
                    for (int d = 0; d < 4; ++d) o[h][d] += (double)v[d] * e;
                }
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
            if (h < G)
#pragma unroll
                for (int d = 0; d < 4; ++d) red[((size_t)warp * G + h) * 128 + lane * 4 + d] = o[h][d];
        __syncthreads();
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
            if (h < G) {
                double oi = red[(size_t)h * 128 + tid];
                for (int w = 1; w < kAttnWarps; ++w) oi += red[((size_t)w * G + h) * 128 + tid];
                double si = 0.0;
                for (int jj = 0; jj < cnt; ++jj) si += (double)ebuf[h * kAttnSplit + jj];
                const float wi = det_expf(__fsub_rn(msp[h * nsp + i], M[h]));
                acc[h] += oi * (double)wi;
                ssum[h] += si * (double)wi;
            }
        __syncthreads();
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
        if (h < G) a.out[(size_t)t * a.H * 128 + (size_t)(g * G + h) * 128 + tid] = (float)(acc[h] / ssum[h]);
}

constexpr size_t kAttnSmemMax = 200 * 1024;

cudaError_t attn_setup() {
    return cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmemMax);
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) {
    const int G = a.Hkv > 0 ? a.H / a.Hkv : 0;
    if (a.hd != 128 || G < 1 || a.H % a.Hkv != 0 || G > kMaxGroup || !a.scores || a.max_keys < 1)
        return cudaErrorInvalidValue;
    const int nsp = (a.max_keys + kAttnSplit - 1) / kAttnSplit;
    const size_t smem = attn_split_smem(G, nsp);
    if (smem > kAttnSmemMax) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.Hkv, a.T), dim3(kAttnThreads), smem, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, attn_split_kernel, a);
}

}  // namespace s2k
