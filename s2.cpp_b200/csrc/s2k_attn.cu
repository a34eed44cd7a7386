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

#include <algorithm>

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

// ---------------------------------------------------------------------------
// Split-parallel attention for calls with few rows (decode steps, batched
// frames): one CTA per (split i, kv head g, row t).  The CTA copies the
// split's cached K / V rows (4 pages of 16 positions, 4 KB each per layer and
// kv head) into shared memory with 16-byte cp.async, forms the split's
// scores, m_i, e_j, S_i and O_i for the G query heads of kv head g, and
// writes them to the partials; the CTA that arrives last for (t, g) combines
// the splits in split order exactly as attn_split_kernel does.  Keys of this
// call (positions >= the cached count) are read as f32 from kcur / vcur.
// ---------------------------------------------------------------------------
constexpr int kFlThreads = 128;

// 16-byte chunk c of cached key row jj sits at chunk c ^ (jj & 15) of the
// row in shared memory, so the score loop's 8-byte reads of 16 different
// rows hit different banks.
__device__ __forceinline__ int fl_swz(int jj, int c) { return c ^ (jj & 15); }

// Most splits a flash-attention row may have (32768 positions).
constexpr int kFlMaxSplits = 512;

// e_j of the split, reused by the combine for the split weights w_i
__host__ __device__ __forceinline__ int fl_ew(int nsp_cap) { return nsp_cap > kAttnSplit ? nsp_cap : kAttnSplit; }

size_t attn_flash_smem(int G, int nsp_cap) {
    return (size_t)2 * kAttnSplit * 128 * sizeof(__half)  // K, V tiles
           + (size_t)G * 128 * sizeof(double)              // queries
           + (size_t)G * fl_ew(nsp_cap) * sizeof(double)   // e_j / w_i
           + (size_t)G * kAttnSplit * sizeof(float)        // scores
           + 64;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__global__ void __launch_bounds__(kFlThreads) attn_flash_kernel(AttnArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    extern __shared__ __align__(16) uint8_t smem[];
    const int g = blockIdx.y, t = blockIdx.z;
    const int G = a.H / a.Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __half *ks = reinterpret_cast<__half *>(smem);                  // [64][128]
    __half *vs = ks + kAttnSplit * 128;                              // [64][128]
    const int EW = fl_ew(a.fl_nsp);
    double *qs = reinterpret_cast<double *>(vs + kAttnSplit * 128);  // [G][128]
    double *es = qs + G * 128;                                       // [G][EW]
    float *ss = reinterpret_cast<float *>(es + G * EW);              // [G][64]
    int *flag = reinterpret_cast<int *>(ss + G * kAttnSplit);
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
    const int nsp = (Lk + kAttnSplit - 1) / kAttnSplit;
    if (Lk < 1 || nsp > a.fl_nsp || Lk > a.max_keys || (nc > 0 && (nc - 1) / kPage >= kv.n_pages)) {
        if (tid == 0 && blockIdx.x == 0 && a.err) atomicOr(a.err, ERR_BAD_POS);
        return;
    }
    // splits blockIdx.x, blockIdx.x + gridDim.x, ... of this row
    int done_splits = 0;
    for (int i = blockIdx.x; i < nsp; i += gridDim.x, ++done_splits) {
        const int j0 = i * kAttnSplit, cnt = min(kAttnSplit, Lk - j0);
        const int ncache = max(0, min(cnt, nc - j0));  // cached keys of the split: [0, ncache)
        // cached K / V rows: 16 chunks of 16 bytes per row
        for (int c = tid; c < ncache * 16; c += kFlThreads) {
            const int jj = c >> 4, ch = c & 15, j = j0 + jj;
            const int page = __ldcg(kv.block_table + j / kPage);
            const size_t off = ((((size_t)page * kv.n_layers + a.layer) * kv.n_kv_heads + g) * kPage + j % kPage) * 128 + ch * 8;
            cp_async16(ks + jj * 128 + fl_swz(jj, ch) * 8, kv.k + off);
            cp_async16(vs + jj * 128 + fl_swz(jj, ch) * 8, kv.v + off);
        }
        if (done_splits == 0)
            for (int p = tid; p < G * 128; p += kFlThreads)
                qs[p] = (double)__ldcg(a.q + (size_t)t * a.ldq + (size_t)g * G * 128 + p);
        cp_async_wait_all();
        __syncthreads();
        // scores: thread -> key jj = tid % 64, heads h = tid / 64, tid / 64 + 2, ...
        {
            const int jj = tid & (kAttnSplit - 1);
            if (jj < cnt) {
                for (int h = tid >> 6; h < G; h += kFlThreads / kAttnSplit) {
                    double acc = 0.0;
                    if (jj < ncache) {
#pragma unroll 4
                        for (int c = 0; c < 16; ++c) {
                            const uint4 raw = *reinterpret_cast<const uint4 *>(ks + jj * 128 + fl_swz(jj, c) * 8);
                            const __half2 *hv = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const float2 f = __half22float2(hv[u]);
                                acc += (double)f.x * qs[h * 128 + c * 8 + 2 * u];
                                acc += (double)f.y * qs[h * 128 + c * 8 + 2 * u + 1];
                            }
                        }
                    } else {
                        const float *kr = kc + ((size_t)(j0 + jj - nc) * a.Hkv + g) * 128;
                        for (int d = 0; d < 128; d += 4) {
                            const float4 f = __ldcg(reinterpret_cast<const float4 *>(kr + d));
                            acc += (double)f.x * qs[h * 128 + d];
                            acc += (double)f.y * qs[h * 128 + d + 1];
                            acc += (double)f.z * qs[h * 128 + d + 2];
                            acc += (double)f.w * qs[h * 128 + d + 3];
                        }
                    }
                    ss[h * kAttnSplit + jj] = __fmul_rn((float)acc, a.scale);
                }
            }
        }
        __syncthreads();
        // split maximum, exponentials and their sum: warp w handles heads w, w + 4, ...
        double *ms_out = a.fl_ms + ((((size_t)t * a.Hkv + g) * a.fl_nsp + i) * G) * 2;
        for (int h = warp; h < G; h += kFlThreads / 32) {
            float mx = -INFINITY;
            for (int jj = lane; jj < cnt; jj += 32) mx = fmaxf(mx, ss[h * kAttnSplit + jj]);
            mx = warp_max(mx);
            double se = 0.0;
            for (int jj = lane; jj < kAttnSplit; jj += 32) {
                const float e = jj < cnt ? det_expf(__fsub_rn(ss[h * kAttnSplit + jj], mx)) : 0.f;
                es[h * EW + jj] = (double)e;
                se += (double)e;
            }
            se = warp_sum_d(se);
            if (lane == 0) {
                ms_out[h * 2] = (double)mx;
                ms_out[h * 2 + 1] = se;
            }
        }
        __syncthreads();
        // O_i: thread owns dimension d = tid of every head
        double *po = a.fl_part + (((size_t)t * a.Hkv + g) * a.fl_nsp + i) * G * 128;
        {
            double o[kMaxGroup];
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h) o[h] = 0.0;
            const int d = tid;
            for (int jj = 0; jj < cnt; ++jj) {
                float v;
                if (jj < ncache) v = __half2float(vs[jj * 128 + fl_swz(jj, d >> 3) * 8 + (d & 7)]);
                else v = __ldcg(vc + ((size_t)(j0 + jj - nc) * a.Hkv + g) * 128 + d);
                const double vd = (double)v;
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h)
                    if (h < G) o[h] += vd * es[h * EW + jj];
            }
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h)
                if (h < G) po[h * 128 + d] = o[h];
        }
        __syncthreads();  // shared tiles are refilled by the next split
    }
    if (done_splits == 0) return;
    // the last split of (t, g) to arrive combines
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int *ctr = a.fl_counters + (size_t)t * a.Hkv + g;
        const int prev = atomicAdd(ctr, done_splits);
        *flag = prev + done_splits == nsp;
        if (prev + done_splits == nsp) *ctr = 0;
    }
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    const double *pall = a.fl_part + (((size_t)t * a.Hkv + g) * a.fl_nsp) * G * 128;
    const double *msall = a.fl_ms + (((size_t)t * a.Hkv + g) * a.fl_nsp) * G * 2;
    // split weights w_i = det_expf(m_i - M) per head, into es ([G][nsp] <= [G][EW])
    for (int h = warp; h < G; h += kFlThreads / 32) {
        float M = -INFINITY;
        for (int k = lane; k < nsp; k += 32) M = fmaxf(M, (float)__ldcg(msall + ((size_t)k * G + h) * 2));
        M = warp_max(M);
        for (int k = lane; k < nsp; k += 32)
            es[h * EW + k] = (double)det_expf(__fsub_rn((float)__ldcg(msall + ((size_t)k * G + h) * 2), M));
    }
    __syncthreads();
    const int d = tid;
    for (int h = 0; h < G; ++h) {
        double acc = 0.0, ssum = 0.0;
        for (int k = 0; k < nsp; ++k) {
            const double wi = es[h * EW + k];
            acc += __ldcg(pall + ((size_t)k * G + h) * 128 + d) * wi;
            ssum += __ldcg(msall + ((size_t)k * G + h) * 2 + 1) * wi;
        }
        a.out[(size_t)t * a.H * 128 + (size_t)(g * G + h) * 128 + d] = (float)(acc / ssum);
    }
}

// ---------------------------------------------------------------------------
// Prompt prefill attention (one sequence, many query rows): one CTA per (kv
// head g, block of 64 / G query rows), i.e. 64 query vectors (row x group
// head) sharing each key split's K and V tile in shared memory.  Same split
// convention and sums as attn_split_kernel, in two passes over the splits:
//   1. K tile (doubles) -> scores of 64 query vectors x 64 keys with 4 x 4
//      register blocks (written to the score scratch) and the split maxima
//      (kept in shared memory);
//   2. V tile + the split's exponentials (from the stored scores) -> S_i and
//      O_i per query vector, folded with w_i = det_expf(m_i - M) in split
//      order.
// ---------------------------------------------------------------------------
constexpr int kBlkThreads = 256;
constexpr int kBlkQV = 64;         // query vectors per CTA
constexpr int kBlkPad = 129;       // row stride (doubles) of the shared tiles: conflict-free columns
constexpr int kBlkMaxSplits = 128; // longest key range: 8192 positions

size_t attn_block_smem(int nsp) {
    return (size_t)2 * kBlkQV * kBlkPad * sizeof(double)  // q (then e) tile, K / V tile
           + (size_t)kBlkQV * nsp * sizeof(float)           // split maxima
           + (size_t)kBlkQV * (sizeof(float) + sizeof(double) + sizeof(int)) + 64;
}

// K or V rows j0 .. j0+63 of the CTA's kv head as doubles (0 past `lim`).
__device__ __forceinline__ void blk_load_tile(const AttnArgs &a, const __half *cache, const float *cur, int g,
                                              int nc, int j0, int lim, double *dst) {
    for (int idx = threadIdx.x; idx < kAttnSplit * 32; idx += kBlkThreads) {
        const int jj = idx >> 5, d4 = (idx & 31) * 4, j = j0 + jj;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (j < lim) {
            if (j < nc) {
                const int page = __ldcg(a.kv.block_table + j / kPage);
                const size_t off =
                    ((((size_t)page * a.kv.n_layers + a.layer) * a.kv.n_kv_heads + g) * kPage + j % kPage) * 128 + d4;
                const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(cache + off));
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                v[0] = f0.x;
                v[1] = f0.y;
                v[2] = f1.x;
                v[3] = f1.y;
            } else {
                const float4 f = __ldcg(reinterpret_cast<const float4 *>(cur + ((size_t)(j - nc) * a.Hkv + g) * 128 + d4));
                v[0] = f.x;
                v[1] = f.y;
                v[2] = f.z;
                v[3] = f.w;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) dst[jj * kBlkPad + d4 + u] = (double)v[u];
    }
}

__global__ void __launch_bounds__(kBlkThreads, 1) attn_block_kernel(AttnArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    extern __shared__ __align__(16) uint8_t smem[];
    const int g = blockIdx.x;
    const int G = a.H / a.Hkv, BQ = kBlkQV / G;  // query rows per CTA
    const int t0 = blockIdx.y * BQ;
    const int tid = threadIdx.x, qb = tid >> 4, kb = tid & 15;
    const int nc = a.n_cached ? __ldcg(a.n_cached) : 0;
    const int nsp_cap = (a.max_keys + kAttnSplit - 1) / kAttnSplit;
    double *qd = reinterpret_cast<double *>(smem);  // [64][kBlkPad] queries, then the split's e_j
    double *kd = qd + kBlkQV * kBlkPad;               // [64][kBlkPad] K or V tile
    float *mi = reinterpret_cast<float *>(kd + kBlkQV * kBlkPad);  // [64][nsp_cap]
    float *Mx = mi + kBlkQV * nsp_cap;                               // [64]
    double *ss = reinterpret_cast<double *>(((uintptr_t)(Mx + kBlkQV) + 7) & ~(uintptr_t)7);  // [64]
    int *lk = reinterpret_cast<int *>(ss + kBlkQV);                  // [64] key range of each query vector
    // query vector qv: row t0 + qv / G, head g * G + qv % G
    int lim = 0;  // the block's longest key range
    for (int qv = tid; qv < kBlkQV; qv += kBlkThreads) {
        const int t = t0 + qv / G;
        lk[qv] = t < a.T ? nc + a.cur_base + t + 1 : 0;
    }
    {
        const int tl = min(a.T, t0 + BQ) - 1;
        lim = nc + a.cur_base + tl + 1;
    }
    if (lim > a.ld_scores || lim > a.max_keys || (nc > 0 && (nc - 1) / kPage >= a.kv.n_pages)) {
        if (tid == 0 && a.err) atomicOr(a.err, ERR_BAD_POS);
        return;
    }
    const int nsp = (lim + kAttnSplit - 1) / kAttnSplit;
    for (int idx = tid; idx < kBlkQV * 32; idx += kBlkThreads) {
        const int qv = idx >> 5, d4 = (idx & 31) * 4, t = t0 + qv / G;
        float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < a.T)
            f = __ldcg(reinterpret_cast<const float4 *>(a.q + (size_t)t * a.ldq + (size_t)(g * G + qv % G) * 128 + d4));
        qd[qv * kBlkPad + d4] = (double)f.x;
        qd[qv * kBlkPad + d4 + 1] = (double)f.y;
        qd[qv * kBlkPad + d4 + 2] = (double)f.z;
        qd[qv * kBlkPad + d4 + 3] = (double)f.w;
    }
    // ---- pass 1: scores and split maxima ----
    for (int i = 0; i < nsp; ++i) {
        const int j0 = i * kAttnSplit;
        __syncthreads();  // previous tile consumed
        blk_load_tile(a, a.kv.k, a.kcur, g, nc, j0, lim, kd);
        __syncthreads();
        double acc[4][4];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) acc[x][y] = 0.0;
        // thread (qb, kb): query vectors qb + 16x, keys kb + 16y of the split
#pragma unroll 4
        for (int d = 0; d < 128; ++d) {
            double qv4[4], kv4[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) qv4[x] = qd[(qb + 16 * x) * kBlkPad + d];
#pragma unroll
            for (int y = 0; y < 4; ++y) kv4[y] = kd[(kb + 16 * y) * kBlkPad + d];
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y) acc[x][y] = fma(kv4[y], qv4[x], acc[x][y]);
        }
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const int qv = qb + 16 * x, t = t0 + qv / G, gh = g * G + qv % G;
            float mx = -INFINITY;
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int j = j0 + kb + 16 * y;
                if (j < lk[qv]) {
                    const float sc = __fmul_rn((float)acc[x][y], a.scale);
                    a.scores[((size_t)t * a.H + gh) * a.ld_scores + j] = sc;
                    mx = fmaxf(mx, sc);
                }
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (kb == 0) mi[qv * nsp_cap + i] = mx;
        }
    }
    __syncthreads();
    // M per query vector over its own splits
    for (int qv = tid; qv < kBlkQV; qv += kBlkThreads) {
        float M = -INFINITY;
        const int ns = (lk[qv] + kAttnSplit - 1) / kAttnSplit;
        for (int i = 0; i < ns; ++i) M = fmaxf(M, mi[qv * nsp_cap + i]);
        Mx[qv] = M;
    }
    // ---- pass 2: e_j, S_i, O_i, folded in split order ----
    // thread (qb, db): query vectors qb + 16x, dims db + 16y
    double acc[4][8], ssum[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) {
        ssum[x] = 0.0;
#pragma unroll
        for (int y = 0; y < 8; ++y) acc[x][y] = 0.0;
    }
    double *ed = qd;  // [64][kBlkPad]: e_j of the split (queries are no longer needed)
    for (int i = 0; i < nsp; ++i) {
        const int j0 = i * kAttnSplit;
        __syncthreads();
        blk_load_tile(a, a.kv.v, a.vcur, g, nc, j0, lim, kd);
        for (int idx = tid; idx < kBlkQV * kAttnSplit; idx += kBlkThreads) {
            const int qv = idx >> 6, jj = idx & 63, j = j0 + jj;
            float e = 0.f;
            if (j < lk[qv]) {
                const int t = t0 + qv / G, gh = g * G + qv % G;
                e = det_expf(__fsub_rn(__ldcg(a.scores + ((size_t)t * a.H + gh) * a.ld_scores + j), mi[qv * nsp_cap + i]));
            }
            ed[qv * kBlkPad + jj] = (double)e;
        }
        __syncthreads();
        double o[4][8];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 8; ++y) o[x][y] = 0.0;
        for (int jj = 0; jj < kAttnSplit; ++jj) {
            double e4[4], v8[8];
#pragma unroll
            for (int x = 0; x < 4; ++x) e4[x] = ed[(qb + 16 * x) * kBlkPad + jj];
#pragma unroll
            for (int y = 0; y < 8; ++y) v8[y] = kd[jj * kBlkPad + kb + 16 * y];
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 8; ++y) o[x][y] = fma(v8[y], e4[x], o[x][y]);
        }
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const int qv = qb + 16 * x;
            if (j0 >= lk[qv]) continue;  // beyond this query's keys
            const double wi = (double)det_expf(__fsub_rn(mi[qv * nsp_cap + i], Mx[qv]));
#pragma unroll
            for (int y = 0; y < 8; ++y) acc[x][y] += o[x][y] * wi;
            if (kb == 0) {
                double si = 0.0;
                for (int jj = 0; jj < kAttnSplit; ++jj) si += ed[qv * kBlkPad + jj];
                ssum[x] += si * wi;
            }
        }
    }
    if (kb == 0)
#pragma unroll
        for (int x = 0; x < 4; ++x) ss[qb + 16 * x] = ssum[x];
    __syncthreads();
#pragma unroll
    for (int x = 0; x < 4; ++x) {
        const int qv = qb + 16 * x, t = t0 + qv / G;
        if (t >= a.T) continue;
        const double S = ss[qv];
#pragma unroll
        for (int y = 0; y < 8; ++y)
            a.out[(size_t)t * a.H * 128 + (size_t)(g * G + qv % G) * 128 + kb + 16 * y] = (float)(acc[x][y] / S);
    }
}

cudaError_t attn_setup() {
    cudaError_t e = cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kAttnSmemMax);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attn_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_block_smem(kBlkMaxSplits));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_flash_smem(kMaxGroup, kFlMaxSplits));
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) {
    const int G = a.Hkv > 0 ? a.H / a.Hkv : 0;
    if (a.hd != 128 || G < 1 || a.H % a.Hkv != 0 || G > kMaxGroup || !a.scores || a.max_keys < 1)
        return cudaErrorInvalidValue;
    const int nsp = (a.max_keys + kAttnSplit - 1) / kAttnSplit;
    if (a.fl_part && a.fl_ms && a.fl_counters && nsp <= a.fl_nsp && a.fl_nsp <= kFlMaxSplits) {
        cudaLaunchAttribute attr[1];
        // CTAs per (kv head, row): enough for ~8 CTAs per SM, each taking
        // every gx-th split of its row
        const int want = (8 * a.num_sms + a.Hkv * a.T - 1) / (a.Hkv * a.T);
        const int gx = std::max(1, std::min(nsp, want));
        cudaLaunchConfig_t cfg =
            pdl_cfg(dim3(gx, a.Hkv, a.T), dim3(kFlThreads), attn_flash_smem(G, a.fl_nsp), st, attr);
        count_launch();
        return cudaLaunchKernelEx(&cfg, attn_flash_kernel, a);
    }
    if (!a.rows && a.T >= 16 && kBlkQV % G == 0 && nsp <= kBlkMaxSplits) {
        // prompt prefill: 64 query vectors per CTA share the key tiles
        cudaLaunchAttribute attr[1];
        const int bq = kBlkQV / G;
        cudaLaunchConfig_t cfg =
            pdl_cfg(dim3(a.Hkv, (a.T + bq - 1) / bq), dim3(kBlkThreads), attn_block_smem(nsp), st, attr);
        count_launch();
        return cudaLaunchKernelEx(&cfg, attn_block_kernel, a);
    }
    const size_t smem = attn_split_smem(G, nsp);
    if (smem > kAttnSmemMax) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.Hkv, a.T), dim3(kAttnThreads), smem, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, attn_split_kernel, a);
}

}  // namespace s2k
