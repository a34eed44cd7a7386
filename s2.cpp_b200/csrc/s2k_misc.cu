// s2k_misc.cu -- device embedding gathers, the on-device sampler and the
// frame-loop bookkeeping kernels.
//
// Reference semantics:
//   Slow input embedding   src/s2_model.cpp:893-962  (get_rows of the token,
//       sum of 10 codebook rows offset by cb*codebook_size in order cb0..cb9,
//       semantic mask, 1/sqrt(num_codebooks+1) scale for semantic tokens)
//   Fast input rows        src/s2_model.cpp:1139-1157 ([hidden ; fast_emb[prefix]],
//       no per-codebook offset)
//   sample_token           src/s2_sampler.cpp:42-99 (exp via det_expf, the
//       normaliser of the T=1 softmax summed in double and rounded once, so
//       the CPU oracle reproduces the same draw)
//   frame loop             src/s2_generate.cpp:57-183 (semantic mask, im_end
//       blocking before min_tokens_before_end, RAS: window 10, resample at
//       T=1.0 / top-p 0.9 when a semantic token repeats, sem_code clamp)
#include "s2k_common.cuh"
#include "s2k_kernels.h"
#include "s2k_device.h"

#include <algorithm>
#include <climits>

namespace s2k {

__device__ __forceinline__ float deq_elem(const DevMat &w, long long row, int col) {
    return tq_elem(w.w, w.type == 12 ? TW_Q4_K : (w.type == 14 ? TW_Q6_K : (w.type == 1 ? TW_F16 : TW_Q8_0)), w.cols,
                   row, col);
}

// grid T, block 256
__global__ void embed_slow_kernel(EmbedArgs a, DevMat E, DevMat C) {
    pdl_launch_dependents();
    pdl_wait();
    if (a.done && __ldcg(a.done)) return;
    const int t = blockIdx.x, dim = E.cols, stride = a.ncb + 1;
    const int *tokens = a.seqs ? a.seqs[t]->state.step_in : a.tokens + t * stride;
    int tok = __ldcg(tokens);
    if (tok < 0 || tok >= E.rows) {
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, ERR_BAD_TOKEN);
        tok = 0;
    }
    const bool sem = tok >= a.sem_begin && tok <= a.sem_end;
    int ids[16];
    bool ok = true;
    if (sem) {
        for (int cb = 0; cb < a.ncb; ++cb) {
            ids[cb] = __ldcg(tokens + 1 + cb) + cb * a.cb_size;
            if (ids[cb] < 0 || ids[cb] >= C.rows) ok = false;
        }
    }
    if (!ok) {
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, ERR_BAD_TOKEN);
        for (int cb = 0; cb < a.ncb; ++cb) ids[cb] = 0;
    }
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float e = deq_elem(E, tok, i);
        if (sem && a.ncb > 0) {
            float s = deq_elem(C, ids[0], i);
            for (int cb = 1; cb < a.ncb; ++cb) s = __fadd_rn(s, deq_elem(C, ids[cb], i));
            e = __fadd_rn(e, s);
        }
        if (a.scale_cb && sem) e = __fmul_rn(e, a.sem_scale);
        a.x[(size_t)t * dim + i] = e;
    }
}

cudaError_t launch_embed_slow(const EmbedArgs &a, cudaStream_t st) {
    if (tw_of(a.tok_emb->type) < 0 || (a.ncb > 0 && tw_of(a.cb_emb->type) < 0) || a.ncb > 16)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.T);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    DevMat C = a.ncb > 0 ? *a.cb_emb : DevMat();
    return cudaLaunchKernelEx(&cfg, embed_slow_kernel, a, *a.tok_emb, C);
}

__global__ void embed_fast_kernel(DevMat F, const float *hidden, const int *codes, int code0, float *x, int dim,
                                  const int *done, int *err) {
    pdl_launch_dependents();
    pdl_wait();
    if (done && __ldcg(done)) return;
    const int r = blockIdx.x;
    if (hidden && r == 0) {
        for (int i = threadIdx.x; i < dim; i += blockDim.x) x[i] = __ldcg(hidden + i);
        return;
    }
    int c = __ldcg(codes + code0 + r - (hidden ? 1 : 0));
    if (c < 0 || c >= F.rows) {
        if (threadIdx.x == 0 && err) atomicOr(err, ERR_BAD_TOKEN);
        c = 0;
    }
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)r * dim + i] = deq_elem(F, c, i);
}

// grid n_rows (pass 0: 2n, else n), block 256
__global__ void embed_fast_batch_kernel(DevMat F, SeqDev *const *seqs, int pass, float *x, int dim, int *err) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x;
    const int b = pass == 0 ? r >> 1 : r;
    const SeqDev *sd = seqs[b];
    if (pass == 0 && (r & 1) == 0) {
        const float *h = sd->hidden;
        for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)r * dim + i] = __ldcg(h + i);
        return;
    }
    int c = __ldcg(&sd->state.codes[pass]);
    if (c < 0 || c >= F.rows) {
        if (threadIdx.x == 0 && err) atomicOr(err, ERR_BAD_TOKEN);
        c = 0;
    }
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)r * dim + i] = deq_elem(F, c, i);
}

cudaError_t launch_embed_fast_batch(const DevMat *fast_emb, SeqDev *const *seqs, int n, int pass, float *x, int dim,
                                    int *err, cudaStream_t st) {
    if (tw_of(fast_emb->type) < 0 || n < 1 || pass < 0 || pass >= 16) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pass == 0 ? 2 * n : n);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, embed_fast_batch_kernel, *fast_emb, seqs, pass, x, dim, err);
}

cudaError_t launch_embed_fast(const DevMat *fast_emb, const float *hidden, const int *codes, int code0, int n_rows,
                              float *x, int dim, const int *done, int *err, cudaStream_t st) {
    if (tw_of(fast_emb->type) < 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_rows);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, embed_fast_kernel, *fast_emb, hidden, codes, code0, x, dim, done, err);
}

// ---------------------------------------------------------------------------
// sampler: one CTA of 1024 threads
// ---------------------------------------------------------------------------
constexpr int kSampThreads = 1024;
constexpr int kSampMax = 8192;

struct SampSmem {
    float key[kSampMax];
    int idx[kSampMax];
    float rf[32];
    int ri[32];
    double rd[32];
    int result;
};

__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

// cand(i, v, ix) gives candidate i's logit and token index.
template <class F>
__device__ int block_sample(SampSmem &sm, int n, F cand, float temp, float top_p, int top_k, double u, int *err) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
    if (temp <= 0.f) {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int i = tid; i < n; i += nt) {
            float v;
            int ix;
            cand(i, v, ix);
            if (better(v, ix, bv, bi)) { bv = v; bi = ix; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { sm.rf[warp] = bv; sm.ri[warp] = bi; }
        __syncthreads();
        if (warp == 0) {
            bv = lane < nw ? sm.rf[lane] : -INFINITY;
            bi = lane < nw ? sm.ri[lane] : INT_MAX;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) {
                if (bi == INT_MAX) {  // no finite candidate: fall back to candidate 0
                    float v;
                    int ix;
                    cand(0, v, ix);
                    bi = ix;
                    if (err) atomicOr(err, ERR_SAMPLER);
                }
                sm.result = bi;
            }
        }
        __syncthreads();
        const int r = sm.result;
        __syncthreads();
        return r;
    }
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = tid; i < P; i += nt) {
        if (i < n) {
            cand(i, sm.key[i], sm.idx[i]);
        } else {
            sm.key[i] = -INFINITY;
            sm.idx[i] = INT_MAX;
        }
    }
    __syncthreads();
    // bitonic sort into "better first" order
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < P; i += nt) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const float a = sm.key[i], b = sm.key[ixj];
                    const int ia = sm.idx[i], ib = sm.idx[ixj];
                    const bool sw = ((i & k) == 0) ? better(b, ib, a, ia) : better(a, ia, b, ib);
                    if (sw) {
                        sm.key[i] = b; sm.key[ixj] = a;
                        sm.idx[i] = ib; sm.idx[ixj] = ia;
                    }
                }
            }
            __syncthreads();
        }
    }
    const float mx = sm.key[0];
    double part = 0.0;
    for (int i = tid; i < n; i += nt) part += (double)det_expf(__fsub_rn(sm.key[i], mx));
    part = warp_sum_d(part);
    if (lane == 0) sm.rd[warp] = part;
    __syncthreads();
    if (tid == 0) {
        double Sd = 0.0;
        for (int w = 0; w < nw; ++w) Sd += sm.rd[w];
        const float S = (float)Sd;
        const int k = top_k > 0 ? min(top_k, n) : n;
        const float tp = fminf(fmaxf(top_p, 0.f), 1.f);
        float cum = 0.f;
        int nf = 0;
        for (int i = 0; i < k; ++i) {
            float p = det_expf(__fsub_rn(sm.key[i], mx));
            if (S > 0.f) p = __fdiv_rn(p, S);
            cum = __fadd_rn(cum, p);
            if (i > 0 && cum > tp) break;
            nf = i + 1;
        }
        if (nf == 0) nf = 1;
        const float m2 = sm.key[0];
        float s = 0.f;
        for (int i = 0; i < nf; ++i) s = __fadd_rn(s, det_expf(__fdiv_rn(__fsub_rn(sm.key[i], m2), temp)));
        float sp = 0.f;
        for (int i = 0; i < nf; ++i) {
            float e = det_expf(__fdiv_rn(__fsub_rn(sm.key[i], m2), temp));
            if (s > 0.f) e = __fdiv_rn(e, s);
            sp = __fadd_rn(sp, e);
        }
        int pick = 0;
        if (sp > 0.f) {
            double tot = 0.0;
            for (int i = 0; i < nf; ++i) {
                float e = det_expf(__fdiv_rn(__fsub_rn(sm.key[i], m2), temp));
                if (s > 0.f) e = __fdiv_rn(e, s);
                tot += (double)__fdiv_rn(e, sp);
            }
            pick = nf - 1;
            double c = 0.0;
            for (int i = 0; i < nf - 1; ++i) {
                float e = det_expf(__fdiv_rn(__fsub_rn(sm.key[i], m2), temp));
                if (s > 0.f) e = __fdiv_rn(e, s);
                c += (double)__fdiv_rn(e, sp) / tot;
                if (c >= u) { pick = i; break; }
            }
        }
        int r = sm.idx[pick];
        if (r == INT_MAX) {
            float v;
            cand(0, v, r);
            if (err) atomicOr(err, ERR_SAMPLER);
        }
        sm.result = r;
    }
    __syncthreads();
    const int r = sm.result;
    __syncthreads();
    return r;
}

// Philox4x32-10 (Salmon et al., SC'11); 53-bit uniform from outputs 0 and 1.
__device__ double philox_uniform(unsigned long long seed, unsigned frame, unsigned purpose, unsigned seq) {
    unsigned c0 = frame, c1 = purpose, c2 = seq, c3 = 0x53324b30u;
    unsigned k0 = (unsigned)seed, k1 = (unsigned)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const unsigned long long p0 = 0xD2511F53ull * c0, p1 = 0xCD9E8D57ull * c2;
        const unsigned n0 = (unsigned)(p1 >> 32) ^ c1 ^ k0, n2 = (unsigned)(p0 >> 32) ^ c3 ^ k1;
        c1 = (unsigned)p1;
        c3 = (unsigned)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    const unsigned long long a = c0 >> 5, b = c1 >> 6;
    return (double)(a * 67108864ull + b) * (1.0 / 9007199254740992.0);
}

enum { RNG_MAIN = 0, RNG_RAS = 1, RNG_FAST0 = 2 };

// Frame-loop state is written by the previous kernels of the same PDL chain:
// read it through L2 (ld.global.cg), never from a possibly stale L1 line.
__device__ __forceinline__ SampleCfg load_cfg(const SampleCfg *p) {
    SampleCfg c;
    const int *w = reinterpret_cast<const int *>(p);
    int *o = reinterpret_cast<int *>(&c);
#pragma unroll
    for (int i = 0; i < (int)(sizeof(SampleCfg) / 4); ++i) o[i] = __ldcg(w + i);
    return c;
}

struct SlowCand {
    const float *logits;
    int sem_begin, nsem, im_end, extra, block;
    __device__ void operator()(int i, float &v, int &ix) const {
        if (i < nsem) {
            ix = sem_begin + i;
            v = (block && ix == im_end) ? -INFINITY : __ldcg(logits + ix);
        } else {
            ix = im_end;
            v = block ? -INFINITY : __ldcg(logits + im_end);
        }
    }
};

struct DenseCand {
    const float *logits;
    __device__ void operator()(int i, float &v, int &ix) const {
        ix = i;
        v = __ldcg(logits + i);
    }
};

__device__ __forceinline__ SlowCand make_slow_cand(const float *logits, const SampleCfg &c, int block) {
    SlowCand sc;
    sc.logits = logits;
    sc.sem_begin = c.sem_begin;
    const int se = min(c.sem_end, c.vocab - 1);
    sc.nsem = max(0, se - c.sem_begin + 1);
    sc.im_end = c.im_end;
    sc.extra = (c.im_end >= 0 && c.im_end < c.vocab && !(c.im_end >= c.sem_begin && c.im_end <= se)) ? 1 : 0;
    sc.block = block;
    return sc;
}

__device__ void sample_main_body(SampSmem &sm, const float *logits, SeqDev *sd, int *err) {
    volatile SeqState &st = sd->state;
    const SampleCfg c = load_cfg(&sd->cfg);
    if (st.done) return;
    const int f = st.n_frames;
    const int block = f < c.min_tokens_before_end;
    const SlowCand cand = make_slow_cand(logits, c, block);
    const int n = cand.nsem + cand.extra;
    int tok = block_sample(sm, n, cand, c.temperature, c.top_p, c.top_k,
                           philox_uniform(c.seed, (unsigned)f, RNG_MAIN, c.seq_id), err);
    if (tok == c.im_end || f >= c.max_new_tokens) {
        if (threadIdx.x == 0) {
            st.main_token = tok;
            st.done = 1;
            HostStatus *hs = (HostStatus *)__ldcg((const unsigned long long *)&sd->host);
            if (hs) {
                hs->n_frames = f;
                __threadfence_system();
                hs->done = 1;
            }
        }
        return;
    }
    // repetition-aware sampling (src/s2_generate.cpp:99-121)
    bool in_win = false;
    for (int i = 0; i < st.n_ras; ++i) in_win |= (st.ras[i] == tok);
    if (st.n_ras > 0 && in_win && tok >= c.sem_begin && tok <= c.sem_end) {
        tok = block_sample(sm, n, cand, 1.0f, 0.9f, c.top_k, philox_uniform(c.seed, (unsigned)f, RNG_RAS, c.seq_id),
                           err);
    }
    if (threadIdx.x == 0) {
        if (st.n_ras == 10) {
            for (int i = 0; i < 9; ++i) st.ras[i] = st.ras[i + 1];
            st.n_ras = 9;
        }
        st.ras[st.n_ras++] = tok;
        int sem = tok - c.sem_begin;
        sem = sem < 0 ? 0 : (sem >= c.cb_size ? c.cb_size - 1 : sem);
        st.main_token = tok;
        st.codes[0] = sem;
    }
}

__global__ void __launch_bounds__(kSampThreads) sample_main_kernel(const float *logits, SeqDev *sd, int *err) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(smem_raw);
    pdl_launch_dependents();
    pdl_wait();
    sample_main_body(sm, logits, sd, err);
}

// grid n: CTA b samples sequence b's main token from logits row b after
// storing hidden row b as the sequence's hidden state.
__global__ void __launch_bounds__(kSampThreads) sample_main_batch_kernel(const float *logits, size_t ld,
                                                                         SeqDev *const *seqs, const float *hidden,
                                                                         int dim, int *err) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(smem_raw);
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    SeqDev *sd = seqs[b];
    float *dst = sd->hidden;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) dst[i] = __ldcg(hidden + (size_t)b * dim + i);
    sample_main_body(sm, logits + (size_t)b * ld, sd, err);
}

__device__ void sample_fast_body(SampSmem &sm, const float *logits, SeqDev *sd, int cb, int *err) {
    volatile SeqState &st = sd->state;
    const SampleCfg c = load_cfg(&sd->cfg);
    if (st.done) return;
    DenseCand cand{logits};
    const int tok = block_sample(sm, c.cb_size, cand, c.temperature, c.top_p, c.top_k,
                                 philox_uniform(c.seed, (unsigned)st.n_frames, RNG_FAST0 + cb, c.seq_id), err);
    if (threadIdx.x == 0) st.codes[cb] = tok;
}

__global__ void __launch_bounds__(kSampThreads) sample_fast_kernel(const float *logits, SeqDev *sd, int cb, int *err) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(smem_raw);
    pdl_launch_dependents();
    pdl_wait();
    sample_fast_body(sm, logits, sd, cb, err);
}

__global__ void __launch_bounds__(kSampThreads) sample_fast_batch_kernel(const float *logits, size_t ld,
                                                                         SeqDev *const *seqs, int cb, int *err) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(smem_raw);
    pdl_launch_dependents();
    pdl_wait();
    sample_fast_body(sm, logits + (size_t)blockIdx.x * ld, seqs[blockIdx.x], cb, err);
}

__device__ void frame_commit_body(SeqDev *sd) {
    volatile SeqState &st = sd->state;
    const SampleCfg c = load_cfg(&sd->cfg);
    if (st.done) return;
    const int f = st.n_frames;
    const int i = threadIdx.x;
    HostStatus *hs = (HostStatus *)__ldcg((const unsigned long long *)&sd->host);
    if (i < c.ncb) {
        const int code = st.codes[i];
        c.codes_out[(size_t)i * c.codes_ld + f] = code;
        st.step_in[1 + i] = code;
        if (hs) {
            // streaming hand-off: the frame's codes into the host ring before its count
            hs->ring[f % kFrameRing][i] = code;
            __threadfence_system();
        }
    }
    __syncthreads();
    if (i == 0) {
        st.step_in[0] = st.main_token;
        st.n_frames = f + 1;
        if (hs) {
            __threadfence_system();
            hs->n_frames = f + 1;
        }
    }
}

__global__ void frame_commit_kernel(SeqDev *sd) {
    pdl_launch_dependents();
    pdl_wait();
    frame_commit_body(sd);
}

// grid n, block 32
__global__ void frame_commit_batch_kernel(SeqDev *const *seqs) {
    pdl_launch_dependents();
    pdl_wait();
    frame_commit_body(seqs[blockIdx.x]);
}

// one thread per sequence
__global__ void advance_batch_kernel(SeqDev *const *seqs, int n, int T) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    volatile SeqState &st = seqs[b]->state;
    if (!st.done) st.n_past = st.n_past + T;
}

__global__ void advance_kernel(SeqDev *sd, int T, const int *done) {
    pdl_launch_dependents();
    pdl_wait();
    if (done && __ldcg(done)) return;
    volatile SeqState &st = sd->state;
    st.n_past = st.n_past + T;
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

cudaError_t sampler_setup() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(sample_main_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(SampSmem))))
        return e;
    if ((e = cudaFuncSetAttribute(sample_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(SampSmem))))
        return e;
    if ((e = cudaFuncSetAttribute(sample_main_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  sizeof(SampSmem))))
        return e;
    if ((e = cudaFuncSetAttribute(sample_fast_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  sizeof(SampSmem))))
        return e;
    return cudaSuccess;
}

cudaError_t launch_sample_main(const float *logits, SeqDev *sd, int *err, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(kSampThreads), sizeof(SampSmem), st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, sample_main_kernel, logits, sd, err);
}

cudaError_t launch_sample_fast(const float *logits, SeqDev *sd, int cb, int *err, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(kSampThreads), sizeof(SampSmem), st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, sample_fast_kernel, logits, sd, cb, err);
}

cudaError_t launch_frame_commit(SeqDev *sd, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(32), 0, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, frame_commit_kernel, sd);
}

cudaError_t launch_sample_main_batch(const float *logits, size_t ld, SeqDev *const *seqs, int n, const float *hidden,
                                     int dim, int *err, cudaStream_t st) {
    if (n < 1) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(n), dim3(kSampThreads), sizeof(SampSmem), st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, sample_main_batch_kernel, logits, ld, seqs, hidden, dim, err);
}

cudaError_t launch_sample_fast_batch(const float *logits, size_t ld, SeqDev *const *seqs, int n, int cb, int *err,
                                     cudaStream_t st) {
    if (n < 1) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(n), dim3(kSampThreads), sizeof(SampSmem), st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, sample_fast_batch_kernel, logits, ld, seqs, cb, err);
}

cudaError_t launch_frame_commit_batch(SeqDev *const *seqs, int n, cudaStream_t st) {
    if (n < 1) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(n), dim3(32), 0, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, frame_commit_batch_kernel, seqs);
}

cudaError_t launch_advance_batch(SeqDev *const *seqs, int n, int T, cudaStream_t st) {
    if (n < 1) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3((n + 127) / 128), dim3(128), 0, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, advance_batch_kernel, seqs, n, T);
}

cudaError_t launch_advance(SeqDev *sd, int T, const int *done, cudaStream_t st) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(1), 0, st, attr);
    count_launch();
    return cudaLaunchKernelEx(&cfg, advance_kernel, sd, T, done);
}

// get_rows: out[r][c] = dequantized table row ids[r] (grid n, block 256).
// Invalid ids set ERR_BAD_TOKEN and give a zero row.
__global__ void gather_rows_kernel(DevMat E, const int *ids, int n, float *out, int *err) {
    const int r = blockIdx.x;
    const int id = __ldg(ids + r);
    const bool ok = id >= 0 && id < E.rows;
    if (!ok && threadIdx.x == 0) atomicOr(err, ERR_BAD_TOKEN);
    for (int c = threadIdx.x; c < E.cols; c += blockDim.x)
        out[(size_t)r * E.cols + c] = ok ? deq_elem(E, id, c) : 0.0f;
}

cudaError_t launch_gather_rows(const DevMat *E, const int *ids, int n, float *out, int *err, cudaStream_t st) {
    if (n < 1 || tw_of(E->type) < 0) return cudaErrorInvalidValue;
    count_launch();
    gather_rows_kernel<<<n, 256, 0, st>>>(*E, ids, n, out, err);
    return cudaGetLastError();
}

// standalone sampler (s2k_sample)
__global__ void __launch_bounds__(kSampThreads) sample_one_kernel(const float *logits, int n, float temperature,
                                                                  float top_p, int top_k, double u, int *out,
                                                                  int *err) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampSmem &sm = *reinterpret_cast<SampSmem *>(smem_raw);
    DenseCand cand{logits};
    const int r = block_sample(sm, n, cand, temperature, top_p, top_k, u, err);
    if (threadIdx.x == 0) *out = r;
}

cudaError_t launch_sample_one(const float *logits, int n, float temperature, float top_p, int top_k, double u,
                              int *out, int *err, cudaStream_t st) {
    if (n <= 0 || n > kSampMax) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(sample_one_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         sizeof(SampSmem));
    if (e != cudaSuccess) return e;
    count_launch();
    sample_one_kernel<<<1, kSampThreads, sizeof(SampSmem), st>>>(logits, n, temperature, top_p, top_k, u, out, err);
    return cudaGetLastError();
}

// det_expf over an array (the exp every kernel shares with the CPU oracle).
__global__ void det_expf_kernel(const float *x, float *y, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = det_expf(x[i]);
}

cudaError_t launch_det_expf(const float *x, float *y, long long n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148 * 8);
    det_expf_kernel<<<blocks, 256, 0, st>>>(x, y, n);
    return cudaGetLastError();
}

}  // namespace s2k
