// s2k_api.cu -- the C ABI of include/s2k.h: model and weight upload,
// sequences with a paged f16 KV cache, the eval_cached / fast_decode entry
// points, and the on-device frame loop captured as one CUDA graph per frame.
#include "../../include/s2k.h"
#include "s2k_common.cuh"
#include "s2k_device.h"
#include "s2k_kernels.h"
#include "s2k_mega.h"
#include "s2k_model.h"

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace s2k {

static std::atomic<unsigned long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

thread_local std::string g_err;
s2k_status fail(s2k_status code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}


}  // namespace s2k

using namespace s2k;


// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
int cuda_set(int dev) { return cudaSetDevice(dev) == cudaSuccess ? 0 : -1; }

s2k_status check_err_word(s2k_model *m) {
    int h = 0;
    CU(cudaMemcpy(&h, m->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        CU(cudaMemset(m->d_err, 0, sizeof(int)));
        if (h & (ERR_WAIT_FULL | ERR_WAIT_EMPTY | ERR_GRID))
            return fail(S2K_ERR_TIMEOUT, "device wait timed out (flags 0x%x)", h);
        return fail(S2K_ERR_ARG, "device reported invalid input (flags 0x%x)", h);
    }
    return S2K_OK;
}

// T: tokens per call; L: longest key range (positions) a call attends over.
// prefill: the Slow work, whose prompt-sized calls use the tensor-core GEMM.
cudaError_t work_alloc(s2k_model *m, Work &w, int T, int L, int dim, int H, int Hkv, int hd, int ff,
                              int n_layers, bool prefill, int flash_rows) {
    w.T = T;
    w.L = L;
    w.dim = dim;
    w.qs = H * hd;
    w.kvs = Hkv * hd;
    w.ff = ff;
    w.H = H;
    const size_t tn = (size_t)std::max(T, 1);
    cudaError_t e;
    if ((e = m->alloc(&w.x, tn * dim))) return e;
    if ((e = m->alloc(&w.h, tn * dim))) return e;
    if ((e = m->alloc(&w.qkv, tn * (w.qs + 2 * w.kvs)))) return e;
    if ((e = m->alloc(&w.attn, tn * w.qs))) return e;
    if ((e = m->alloc(&w.ff_buf, tn * 2 * ff))) return e;
    if ((e = m->alloc(&w.kcur, tn * w.kvs))) return e;
    if ((e = m->alloc(&w.vcur, tn * w.kvs))) return e;
    if ((e = m->alloc(&w.scores, tn * H * (size_t)L))) return e;
    // persistent-kernel buffers (its calls have at most kMegaTokens tokens)
    w.Tm = std::min(T, kMegaTokens);
    const size_t tm = (size_t)std::max(w.Tm, 1);
    w.n_split_max = (L + kAttnSplit - 1) / kAttnSplit;
    const size_t units = tm * Hkv * (size_t)w.n_split_max;
    if ((e = m->alloc(&w.part, units * (H / Hkv) * hd))) return e;
    if ((e = m->alloc(&w.part_ms, units * (H / Hkv) * 2))) return e;
    // split arrival counters per (layer, token, kv head, head block): no reuse within a launch
    const size_t n_counters = (size_t)n_layers * tm * Hkv * kAttnMaxGroup;
    if ((e = m->alloc(&w.counters, n_counters))) return e;
    if ((e = cudaMemset(w.counters, 0, n_counters * sizeof(int)))) return e;
    if ((e = m->alloc(&w.lx, tm * dim))) return e;
    if ((e = m->alloc(&w.lh, tm * dim))) return e;
    if ((e = m->alloc(&w.lqkv, tm * (w.qs + 2 * w.kvs)))) return e;
    if ((e = m->alloc(&w.lattn, tm * w.qs))) return e;
    if ((e = m->alloc(&w.lff, tm * ff))) return e;
    // tag 0 is never a launch's tag (epochs start at 1)
    if ((e = cudaMemset(w.lx, 0, tm * dim * 8))) return e;
    if ((e = cudaMemset(w.lh, 0, tm * dim * 8))) return e;
    if ((e = cudaMemset(w.lqkv, 0, tm * (w.qs + 2 * w.kvs) * 8))) return e;
    if ((e = cudaMemset(w.lattn, 0, tm * w.qs * 8))) return e;
    if ((e = cudaMemset(w.lff, 0, tm * ff * 8))) return e;
    if (flash_rows > 0) {
        w.fl_T = std::min(flash_rows, T);
        w.fl_nsp = (L + kAttnSplit - 1) / kAttnSplit;
        const size_t units = (size_t)w.fl_T * Hkv * w.fl_nsp * (H / Hkv);
        if ((e = m->alloc(&w.fl_part, units * hd))) return e;
        if ((e = m->alloc(&w.fl_ms, units * 2))) return e;
        if ((e = m->alloc(&w.fl_counters, (size_t)w.fl_T * Hkv))) return e;
        if ((e = cudaMemset(w.fl_counters, 0, (size_t)w.fl_T * Hkv * sizeof(int)))) return e;
    }
    if (prefill && T >= kPrefillMinT && m->prefill_mma) {
        const int kmax = std::max(std::max(dim, w.qs), ff);
        // Q8_K rows of a Q6_K GEMM are twice as wide (zero-padded sub-blocks)
        if ((e = m->alloc(&w.pf_xq, tn * kmax * 2))) return e;
        if ((e = m->alloc(&w.pf_xh, tn * kmax))) return e;
        if ((e = m->alloc(&w.pf_dx, tn * kmax * 2 / 32))) return e;
        // stream-K partials (one CTA per SM), and K-tile
        // counters for every (row block, token tile) of the largest GEMM
        w.pf_part_n = prefill_part_doubles(m->num_sms);
        if ((e = m->alloc(&w.pf_part, w.pf_part_n))) return e;
        const int max_rows = std::max({w.qs + 2 * w.kvs, 2 * ff, dim, m->hp.vocab_size, m->hp.codebook_size});
        const int tt = (T + 15) / 16;
        w.pf_n_counters = (size_t)(max_rows / 128 + 1) * tt;
        if ((e = m->alloc(&w.pf_counters, w.pf_n_counters))) return e;
        if ((e = cudaMemset(w.pf_counters, 0, w.pf_n_counters * sizeof(int)))) return e;
    }
    return cudaSuccess;
}

void work_free(s2k_model *m, Work &w) {
    for (void *p : {(void *)w.x, (void *)w.h, (void *)w.qkv, (void *)w.attn, (void *)w.ff_buf, (void *)w.kcur,
                    (void *)w.vcur, (void *)w.scores, (void *)w.part, (void *)w.part_ms, (void *)w.counters,
                    (void *)w.pf_xq, (void *)w.pf_dx, (void *)w.pf_part, (void *)w.pf_counters, (void *)w.pf_xh,
                    (void *)w.fl_part,
                    (void *)w.fl_ms, (void *)w.fl_counters, (void *)w.lx,
                    (void *)w.lh, (void *)w.lqkv, (void *)w.lattn, (void *)w.lff})
        m->release(p);
    w = Work();
}

s2k_status ensure_slow_work(s2k_model *m, int T, int L) {
    if (m->sw.T >= T && m->sw.L >= L) return S2K_OK;
    T = std::max(T, m->sw.T);
    L = std::max(L, m->sw.L);
    work_free(m, m->sw);
    m->ws_gen++;
    const s2k_hparams &hp = m->hp;
    const cudaError_t e = work_alloc(m, m->sw, T, L, hp.embedding_length, hp.head_count, hp.head_count_kv, hp.head_dim,
                                     hp.feed_forward_length, hp.block_count, true, 1);
    if (e != cudaSuccess) {
        // no half-built workspace stays behind: the next call allocates it again
        work_free(m, m->sw);
        return fail(e == cudaErrorMemoryAllocation ? S2K_ERR_OOM : S2K_ERR_CUDA,
                    "Slow workspace for %d tokens x %d positions: %s", T, L, cudaGetErrorString(e));
    }
    return S2K_OK;
}

// RoPE (ggml_rope_ext mode 0, freq_scale 1, ext_factor 0, attn_factor 1) as
// ggml's CPU path evaluates it (ggml_rope_cache_init): theta starts at the
// position and is multiplied by base^(-2/n_dims) once per pair; cos/sin are
// the libm float functions of that theta.  Stored as (cos, sin) per
// [position][pair] and uploaded once, so every kernel reads the same bits the
// CPU computes.
static s2k_status upload_rope(s2k_model *m, float2 **dst, int *n_out, int n_pos, int hd, float base) {
    std::vector<float2> tab((size_t)n_pos * (hd / 2));
    const float ts = powf(base, -2.0f / (float)hd);
    for (int p = 0; p < n_pos; ++p) {
        float theta = (float)p;
        for (int i = 0; i < hd / 2; ++i) {
            tab[(size_t)p * (hd / 2) + i] = make_float2(cosf(theta), sinf(theta));
            theta *= ts;
        }
    }
    CU(m->alloc(dst, tab.size()));
    CU(cudaMemcpy(*dst, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
    *n_out = n_pos;
    return S2K_OK;
}

// ---------------------------------------------------------------------------
// stacks
// ---------------------------------------------------------------------------

// One stack GEMM: prompt-sized Slow calls on Q8_0 weights go through the
// tensor cores (activation rows quantized once, then tcgen05 int8 MMAs,
// s2k_prefill.cu); everything else through the tile GEMV.
cudaError_t stack_gemm(s2k_model *m, Work &w, const GemvArgs &g, bool prefill, bool f16) {
    if (f16 && m->prefill_f16 && w.pf_xh && g.M >= kPrefillMinT && g.M <= w.T && prefill_f16_ok(*g.w, g.M)) {
        const DevMat &W = *g.w;
        cudaError_t e;
        if ((e = launch_rows_f16(g.x, g.ldx, g.M, W.cols, g.in_mode == IN_RMSNORM ? g.norm_w : nullptr, g.eps, w.pf_xh,
                                 g.act_out, m->stream)))
            return e;
        return launch_prefill_f16_gemm(W.w, W.rows, W.cols, g.M, w.pf_xh, g.epi, g.y, g.ldy, g.res, g.ldres,
                                       m->num_sms, m->d_err, m->stream);
    }
    if (prefill && m->prefill_mma && w.pf_xq && g.M >= kPrefillMinT && g.M <= w.T && prefill_ok(*g.w, g.M)) {
        const float *nw = g.in_mode == IN_RMSNORM ? g.norm_w : nullptr;
        cudaError_t e = g.w->type == S2K_TYPE_Q8_0
                            ? launch_quant_rows_q8(g.x, g.ldx, g.M, g.w->cols, nw, g.eps, w.pf_xq, w.pf_dx, g.act_out,
                                                   m->stream)
                            : launch_quant_rows_q8k(g.x, g.ldx, g.M, g.w->cols, nw, g.eps, g.w->type, w.pf_xq, w.pf_dx,
                                                    g.act_out, m->stream);
        if (e != cudaSuccess) return e;
        PrefillArgs a;
        a.w = g.w;
        a.T = g.M;
        a.xq = w.pf_xq;
        a.dx = w.pf_dx;
        a.epi = g.epi;
        a.y = g.y;
        a.ldy = g.ldy;
        a.res = g.res;
        a.ldres = g.ldres;
        a.part = w.pf_part;
        a.part_doubles = w.pf_part_n;
        a.counters = w.pf_counters;
        a.n_counters = w.pf_n_counters;
        a.num_sms = m->num_sms;
        a.err = m->d_err;
        return launch_prefill_gemm(a, m->stream);
    }
    return launch_gemv(g, m->num_sms, m->stream);
}

// Builds layer il's int8 prefill copies (its K-quant matrices) into layer
// slot il % 2.  A plain launch: it starts once every earlier kernel of the
// stream has finished, so layer il - 2's GEMMs, the slot's last readers, are
// done; layer il's GEMMs come a whole layer later.
cudaError_t kq_layer_build(s2k_model *m, int il) {
    Layer &L = m->layers[(size_t)il];
    for (DevMat *dm : {&L.wqkv, &L.wo, &L.w13, &L.w2}) {
        if (!dm->pf) continue;
        cudaError_t e = launch_build_kq_prefill(*dm, m->stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t run_stack(s2k_model *m, const StackCall &c) {
    const s2k_hparams &hp = m->hp;
    Work &w = c.w ? *c.w : (c.fast ? m->fw : m->sw);
    const std::vector<Layer> &layers = c.fast ? m->fast_layers : m->layers;
    const int H = c.fast ? hp.fast_head_count : hp.head_count;
    const int Hkv = c.fast ? hp.fast_head_count_kv : hp.head_count_kv;
    const int hd = c.fast ? hp.fast_head_dim : hp.head_dim;
    const float eps = c.fast ? hp.fast_rms_norm_eps : hp.rms_norm_eps;
    const int qkvs = w.qs + 2 * w.kvs;
    const int dim = w.dim;
    cudaStream_t st = m->stream;
    cudaError_t e;
    // K-quant matrices on the tensor cores read int8 copies built here, one
    // layer ahead, into two alternating layer slots (kq_layer_build)
    const bool kq_build = !c.fast && c.mma && m->kq_slot_bytes > 0 && c.T >= kPrefillKqMinT;
    if (kq_build && (e = kq_layer_build(m, 0))) return e;
    for (size_t il = 0; il < layers.size(); ++il) {
        const Layer &L = layers[il];
        if (kq_build && il + 1 < layers.size() && (e = kq_layer_build(m, (int)il + 1))) return e;
        GemvArgs g;
        g.w = &L.wqkv;
        g.x = w.x;
        g.ldx = dim;
        g.M = c.T;
        g.in_mode = IN_RMSNORM;
        g.norm_w = L.attn_norm;
        g.eps = eps;
        g.y = w.qkv;
        g.ldy = qkvs;
        g.done = c.done;
        g.err = m->d_err;
        if ((e = stack_gemm(m, w, g, c.mma, c.f16mma))) return e;

        QkPrepArgs q;
        q.qkv = w.qkv;
        q.ldqkv = qkvs;
        q.T = c.T;
        q.H = H;
        q.Hkv = Hkv;
        q.hd = hd;
        q.q_norm = L.q_norm;
        q.k_norm = L.k_norm;
        q.eps = eps;
        q.rope = c.fast ? m->rope_fast : m->rope_slow;
        q.rope_positions = c.fast ? m->rope_fast_n : m->rope_slow_n;
        q.pos_base = c.pos_base;
        q.pos_add = c.pos_add;
        q.kcur = c.fast ? (c.fk ? c.fk[il] : m->fkcur[il]) : w.kcur;
        q.vcur = c.fast ? (c.fv ? c.fv[il] : m->fvcur[il]) : w.vcur;
        q.rows = c.rows;
        q.seqs = c.seqs;
        q.cur_base = c.cur_base;
        q.kv = c.kv;
        q.layer = (int)il;
        q.done = c.done;
        q.err = m->d_err;
        if ((e = launch_qk_prep(q, st))) return e;

        AttnArgs a;
        a.q = w.qkv;
        a.ldq = qkvs;
        a.T = c.T;
        a.H = H;
        a.Hkv = Hkv;
        a.hd = hd;
        a.scale = 1.0f / sqrtf((float)hd);
        a.n_cached = c.fast ? nullptr : c.pos_base;
        a.rows = c.rows;
        a.seqs = c.seqs;
        a.kv = c.kv;
        a.layer = (int)il;
        a.kcur = q.kcur;
        a.vcur = q.vcur;
        a.cur_base = c.cur_base;
        a.max_keys = c.max_keys;
        if (c.T <= w.fl_T) {
            a.fl_part = w.fl_part;
            a.fl_ms = w.fl_ms;
            a.fl_counters = w.fl_counters;
            a.fl_nsp = w.fl_nsp;
        }
        a.num_sms = m->num_sms;
        a.scores = w.scores;
        a.ld_scores = w.L;
        a.out = w.attn;
        a.done = c.done;
        a.err = m->d_err;
        if ((e = launch_attention(a, st))) return e;

        GemvArgs o = g;
        o.w = &L.wo;
        o.x = w.attn;
        o.ldx = w.qs;
        o.in_mode = IN_PLAIN;
        o.norm_w = nullptr;
        o.y = w.h;
        o.ldy = dim;
        o.res = w.x;
        o.ldres = dim;
        if ((e = stack_gemm(m, w, o, c.mma, c.f16mma))) return e;

        GemvArgs f1 = g;
        f1.w = &L.w13;
        f1.x = w.h;
        f1.ldx = dim;
        f1.in_mode = IN_RMSNORM;
        f1.norm_w = L.ffn_norm;
        f1.epi = EPI_SWIGLU;
        f1.y = w.ff_buf;
        f1.ldy = w.ff;
        if ((e = stack_gemm(m, w, f1, c.mma, c.f16mma))) return e;

        GemvArgs f2 = g;
        f2.w = &L.w2;
        f2.x = w.ff_buf;
        f2.ldx = w.ff;
        f2.in_mode = IN_PLAIN;
        f2.norm_w = nullptr;
        f2.y = w.x;
        f2.ldy = dim;
        f2.res = w.h;
        f2.ldres = dim;
        if ((e = stack_gemm(m, w, f2, c.mma, c.f16mma))) return e;
    }
    return cudaSuccess;
}

// Slow step over T tokens already in `tokens_dev` ([T][ncb+1]): embedding,
// 36 layers, final norm + tied LM head on the last token, n_past += T.
cudaError_t enqueue_slow(s2k_model *m, s2k_seq *s, int T, const int *tokens_dev, const int *done) {
    const s2k_hparams &hp = m->hp;
    cudaStream_t st = m->stream;
    cudaError_t e;
    EmbedArgs ea;
    ea.tok_emb = &m->embed;
    ea.cb_emb = &m->cb_embed;
    ea.tokens = tokens_dev;
    ea.T = T;
    ea.ncb = hp.num_codebooks;
    ea.cb_size = hp.codebook_size;
    ea.sem_begin = hp.semantic_begin_id;
    ea.sem_end = hp.semantic_end_id;
    ea.scale_cb = hp.scale_codebook_embeddings;
    ea.sem_scale = 1.0f / sqrtf((float)(hp.num_codebooks + 1));
    ea.x = m->sw.x;
    ea.done = done;
    ea.err = m->d_err;
    if ((e = launch_embed_slow(ea, st))) return e;
    StackCall c;
    c.fast = false;
    c.mma = true;
    c.f16mma = T >= kPrefillMinT;  // prompt prefill (decode steps stay on the exact GEMV)
    c.T = T;
    c.pos_base = &s->dev->state.n_past;
    c.pos_add = 0;
    c.cur_base = 0;
    c.kv = s->kv();
    c.max_keys = m->sw.L;
    c.done = done;
    if ((e = run_stack(m, c))) return e;
    GemvArgs hd;
    hd.w = &m->embed;
    hd.x = m->sw.x + (size_t)(T - 1) * hp.embedding_length;
    hd.ldx = hp.embedding_length;
    hd.M = 1;
    hd.in_mode = IN_RMSNORM;
    hd.norm_w = m->norm;
    hd.eps = hp.rms_norm_eps;
    hd.y = m->logits;
    hd.ldy = hp.vocab_size;
    hd.act_out = m->hidden;
    hd.done = done;
    hd.err = m->d_err;
    if ((e = launch_gemv(hd, m->num_sms, st))) return e;
    return launch_advance(s->dev, T, done, st);
}

// One Fast-AR pass over rows already in fw.x.
static cudaError_t enqueue_fast(s2k_model *m, int T, int pos_add, const int *done) {
    const s2k_hparams &hp = m->hp;
    cudaError_t e;
    StackCall c;
    c.fast = true;
    c.T = T;
    c.pos_base = nullptr;
    c.pos_add = pos_add;
    c.cur_base = pos_add;
    c.max_keys = pos_add + T;
    c.done = done;
    if ((e = run_stack(m, c))) return e;
    GemvArgs hd;
    hd.w = &m->fast_out;
    hd.x = m->fw.x + (size_t)(T - 1) * hp.fast_embedding_length;
    hd.ldx = hp.fast_embedding_length;
    hd.M = 1;
    hd.in_mode = IN_RMSNORM;
    hd.norm_w = m->fast_norm;
    hd.eps = hp.fast_rms_norm_eps;
    hd.y = m->flogits;
    hd.ldy = hp.codebook_size;
    hd.done = done;
    hd.err = m->d_err;
    return launch_gemv(hd, m->num_sms, m->stream);
}

// All device work of one frame after its main token is known
// (src/s2_generate.cpp:123-182): 9 Fast-AR passes + samples, commit, Slow step,
// main-token sampling for the next frame.
static cudaError_t enqueue_frame(s2k_model *m, s2k_seq *s) {
    const s2k_hparams &hp = m->hp;
    cudaStream_t st = m->stream;
    const int *done = &s->dev->state.done;
    const int *codes = s->dev->state.codes;
    cudaError_t e;
    for (int p = 0; p + 1 < hp.num_codebooks; ++p) {
        if (p == 0) {
            if ((e = launch_embed_fast(&m->fast_embed, m->hidden, codes, 0, 2, m->fw.x, hp.fast_embedding_length, done,
                                       m->d_err, st)))
                return e;
            if ((e = enqueue_fast(m, 2, 0, done))) return e;
        } else {
            if ((e = launch_embed_fast(&m->fast_embed, nullptr, codes, p, 1, m->fw.x, hp.fast_embedding_length, done,
                                       m->d_err, st)))
                return e;
            if ((e = enqueue_fast(m, 1, p + 1, done))) return e;
        }
        if ((e = launch_sample_fast(m->flogits, s->dev, p + 1, m->d_err, st))) return e;
    }
    if ((e = launch_frame_commit(s->dev, st))) return e;
    if ((e = enqueue_slow(m, s, 1, s->dev->state.step_in, done))) return e;
    return launch_sample_main(m->logits, s->dev, m->d_err, st);
}

// ---------------------------------------------------------------------------
// tensor names
// ---------------------------------------------------------------------------
enum Slot { SL_NONE, SL_EMBED, SL_CB, SL_NORM, SL_FEMB, SL_FNORM, SL_FOUT, SL_ATTN_NORM, SL_FFN_NORM, SL_QN, SL_KN,
            SL_WQKV, SL_WO, SL_W1, SL_W2, SL_W3 };

static Slot parse_name(const s2k_model *m, const char *name, bool *fast, int *il) {
    *fast = false;
    *il = -1;
    if (!strcmp(name, "embeddings.weight")) return SL_EMBED;
    if (!strcmp(name, "codebook_embeddings.weight")) return SL_CB;
    if (!strcmp(name, "norm.weight")) return SL_NORM;
    if (!strcmp(name, "fast_embeddings.weight")) return SL_FEMB;
    if (!strcmp(name, "fast_norm.weight")) return SL_FNORM;
    if (!strcmp(name, "fast_output.weight")) return SL_FOUT;
    int off = 0;
    if (sscanf(name, "layers.%d.%n", il, &off) == 1 && off > 0) {
        *fast = false;
    } else if (sscanf(name, "fast_layers.%d.%n", il, &off) == 1 && off > 0) {
        *fast = true;
    } else {
        return SL_NONE;
    }
    const int nl = *fast ? m->hp.fast_block_count : m->hp.block_count;
    if (*il < 0 || *il >= nl) return SL_NONE;
    const char *s = name + off;
    if (!strcmp(s, "attention_norm.weight")) return SL_ATTN_NORM;
    if (!strcmp(s, "ffn_norm.weight")) return SL_FFN_NORM;
    if (!strcmp(s, "attention.q_norm.weight")) return SL_QN;
    if (!strcmp(s, "attention.k_norm.weight")) return SL_KN;
    if (!strcmp(s, "attention.wqkv.weight")) return SL_WQKV;
    if (!strcmp(s, "attention.wo.weight")) return SL_WO;
    if (!strcmp(s, "feed_forward.w1.weight")) return SL_W1;
    if (!strcmp(s, "feed_forward.w2.weight")) return SL_W2;
    if (!strcmp(s, "feed_forward.w3.weight")) return SL_W3;
    return SL_NONE;
}

bool s2k_model_binds(const s2k_model *m, const char *name) {
    bool fast = false;
    int il = -1;
    const Slot sl = parse_name(m, name, &fast, &il);
    if (sl == SL_NONE) return false;
    const bool fast_slot = fast || sl == SL_FEMB || sl == SL_FNORM || sl == SL_FOUT;
    return !fast_slot || m->hp.has_fast_decoder;
}

static s2k_status upload_vec(s2k_model *m, float **dst, int type, const int64_t ne[4], const void *host, size_t nbytes,
                             int64_t expect, const char *name) {
    if (type != S2K_TYPE_F32) return fail(S2K_ERR_UNSUPPORTED, "%s: norm weights must be F32 (type %d)", name, type);
    if (ne[0] != expect || (ne[1] > 1) || nbytes != (size_t)expect * 4)
        return fail(S2K_ERR_ARG, "%s: expected [%lld] f32, got ne0=%lld bytes=%zu", name, (long long)expect,
                    (long long)ne[0], nbytes);
    if (!*dst) CU(m->alloc(dst, (size_t)expect));
    CU(cudaMemcpyAsync(*dst, host, nbytes, cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return S2K_OK;
}

static s2k_status ensure_mat(s2k_model *m, DevMat &dm, int type, int rows, int cols) {
    if (dm.w) {
        if (dm.rows != rows || dm.cols != cols || dm.type != type) return fail(S2K_ERR_ARG, "matrix shape changed");
        return S2K_OK;
    }
    if (rows % kTR != 0 || cols % kTK != 0)
        return fail(S2K_ERR_UNSUPPORTED, "matrix [%d x %d]: rows must be a multiple of %d and columns of %d", rows,
                    cols, kTR, kTK);
    dm.type = type;
    dm.rows = rows;
    dm.cols = cols;
    CU(m->alloc(&dm.w, dm.bytes()));
    return S2K_OK;
}

static s2k_status upload_mat(s2k_model *m, DevMat &dm, int type, const int64_t ne[4], const void *host, size_t nbytes,
                             int64_t expect_in, int64_t expect_out, int dst_rows, int row_stride, int row_offset,
                             const char *name) {
    if (type != S2K_TYPE_Q8_0 && type != S2K_TYPE_Q4_K && type != S2K_TYPE_Q6_K && type != S2K_TYPE_F16)
        return fail(S2K_ERR_UNSUPPORTED, "%s: ggml type %d not supported for matrices (F16, Q8_0, Q4_K, Q6_K)", name,
                    type);
    if (ne[0] != expect_in || ne[1] != expect_out)
        return fail(S2K_ERR_ARG, "%s: expected ne [%lld, %lld], got [%lld, %lld]", name, (long long)expect_in,
                    (long long)expect_out, (long long)ne[0], (long long)ne[1]);
    if (ne[0] % 256 != 0) return fail(S2K_ERR_UNSUPPORTED, "%s: row length %lld not a multiple of 256", name, (long long)ne[0]);
    const size_t row_bytes = type == S2K_TYPE_F16    ? (size_t)ne[0] * 2
                             : type == S2K_TYPE_Q8_0 ? (size_t)ne[0] / 32 * 34
                                                     : (size_t)ne[0] / 256 * (type == S2K_TYPE_Q4_K ? 144 : 210);
    if (nbytes != row_bytes * (size_t)ne[1])
        return fail(S2K_ERR_ARG, "%s: %zu bytes, expected %zu", name, nbytes, row_bytes * (size_t)ne[1]);
    s2k_status rc = ensure_mat(m, dm, type, dst_rows, (int)ne[0]);
    if (rc) return rc;
    const size_t chunk_rows = std::max<size_t>(1, (size_t)(256u << 20) / row_bytes);
    if (!m->staging) {
        m->staging_bytes = chunk_rows * row_bytes;
        CU(m->alloc(&m->staging, m->staging_bytes));
    }
    const size_t rows_per = std::max<size_t>(1, m->staging_bytes / row_bytes);
    for (size_t r0 = 0; r0 < (size_t)ne[1]; r0 += rows_per) {
        const size_t nr = std::min(rows_per, (size_t)ne[1] - r0);
        CU(cudaMemcpyAsync(m->staging, (const uint8_t *)host + r0 * row_bytes, nr * row_bytes, cudaMemcpyHostToDevice,
                           m->stream));
        CU(launch_relayout(m->staging, (int)r0, (int)nr, (int)ne[0], &dm, row_stride, row_offset, m->stream));
        CU(cudaStreamSynchronize(m->stream));
    }
    return S2K_OK;
}

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

S2K_API int32_t s2k_abi_version(void) { return S2K_ABI_VERSION; }

S2K_API const char *s2k_last_error(void) { return g_err.c_str(); }

S2K_API uint64_t s2k_launch_count(int32_t reset) {
    return reset ? g_launches.exchange(0) : g_launches.load();
}

S2K_API s2k_status s2k_device_count(int32_t *count) {
    if (!count) return fail(S2K_ERR_ARG, "count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        return fail(S2K_ERR_NO_DEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *count = n;
    return S2K_OK;
}

S2K_API s2k_status s2k_model_create(int32_t device, const s2k_hparams *hp, s2k_model **out) {
    if (!hp || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(S2K_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= n) return fail(S2K_ERR_ARG, "device %d out of range (%d devices)", device, n);
    if (hp->embedding_length <= 0 || hp->block_count <= 0 || hp->head_count <= 0 || hp->head_count_kv <= 0 ||
        hp->head_dim != 128 || hp->head_count % hp->head_count_kv != 0 || hp->head_count / hp->head_count_kv > 8 ||
        hp->vocab_size <= 0 || hp->num_codebooks < 0 || hp->num_codebooks > 15 || hp->feed_forward_length <= 0)
        return fail(S2K_ERR_UNSUPPORTED, "unsupported hparams (head_dim must be 128, GQA group <= 8, <= 15 codebooks)");
    if (hp->has_fast_decoder &&
        (hp->fast_head_dim != 128 || hp->fast_head_count % hp->fast_head_count_kv != 0 ||
         hp->fast_head_count / hp->fast_head_count_kv > 8 || hp->fast_embedding_length != hp->embedding_length ||
         hp->fast_has_project_in))
        return fail(S2K_ERR_UNSUPPORTED, "unsupported Fast-AR hparams (fast_dim must equal dim, no project_in)");
    if (cudaSetDevice(device) != cudaSuccess) return fail(S2K_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    s2k_model *m = new s2k_model();
    m->hp = *hp;
    m->device = device;
    cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete m;
        return fail(S2K_ERR_CUDA, "stream create failed");
    }
    m->layers.resize(hp->block_count);
    m->fast_layers.resize(hp->has_fast_decoder ? hp->fast_block_count : 0);
    const unsigned epoch1 = 1;
    if (m->alloc(&m->d_err, kErrBlockInts) != cudaSuccess ||
        cudaMemset(m->d_err, 0, kErrBlockInts * sizeof(int)) != cudaSuccess ||
        m->alloc(&m->d_epoch, 1) != cudaSuccess ||
        cudaMemcpy(m->d_epoch, &epoch1, sizeof(unsigned), cudaMemcpyHostToDevice) != cudaSuccess) {
        s2k_model_free(m);
        return fail(S2K_ERR_OOM, "device allocation failed");
    }
    *out = m;
    return S2K_OK;
}

S2K_API void s2k_model_free(s2k_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    batch_free(m);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

S2K_API s2k_status s2k_model_get_hparams(const s2k_model *m, s2k_hparams *out) {
    if (!m || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = m->hp;
    return S2K_OK;
}

S2K_API size_t s2k_model_weight_bytes(const s2k_model *m) {
    if (!m) return 0;
    size_t b = m->embed.bytes() + m->cb_embed.bytes() + m->fast_embed.bytes() + m->fast_out.bytes();
    for (const auto &L : m->layers) b += L.wqkv.bytes() + L.wo.bytes() + L.w13.bytes() + L.w2.bytes();
    for (const auto &L : m->fast_layers) b += L.wqkv.bytes() + L.wo.bytes() + L.w13.bytes() + L.w2.bytes();
    return b;
}

S2K_API void *s2k_model_stream(s2k_model *m) { return m ? (void *)m->stream : nullptr; }

S2K_API s2k_status s2k_model_upload_tensor(s2k_model *m, const char *name, int32_t type, const int64_t ne[4],
                                           const void *host, size_t nbytes) {
    if (!m || !name || !ne || !host) return fail(S2K_ERR_ARG, "NULL argument");
    if (m->finalized) return fail(S2K_ERR_STATE, "model already finalized");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_hparams &hp = m->hp;
    bool fast = false;
    int il = -1;
    const Slot sl = parse_name(m, name, &fast, &il);
    if (sl == SL_NONE) return fail(S2K_ERR_ARG, "unknown tensor name '%s'", name);
    if (fast && !hp.has_fast_decoder) return fail(S2K_ERR_ARG, "'%s' but the model has no fast decoder", name);
    const int dim = hp.embedding_length;
    const int ff = fast ? hp.fast_feed_forward_length : hp.feed_forward_length;
    const int H = fast ? hp.fast_head_count : hp.head_count;
    const int Hkv = fast ? hp.fast_head_count_kv : hp.head_count_kv;
    const int hd = fast ? hp.fast_head_dim : hp.head_dim;
    Layer *L = il >= 0 ? (fast ? &m->fast_layers[il] : &m->layers[il]) : nullptr;
    switch (sl) {
    case SL_EMBED: return upload_mat(m, m->embed, type, ne, host, nbytes, dim, hp.vocab_size, hp.vocab_size, 1, 0, name);
    case SL_CB:
        return upload_mat(m, m->cb_embed, type, ne, host, nbytes, dim, (int64_t)hp.num_codebooks * hp.codebook_size,
                          hp.num_codebooks * hp.codebook_size, 1, 0, name);
    case SL_NORM: return upload_vec(m, &m->norm, type, ne, host, nbytes, dim, name);
    case SL_FEMB:
        return upload_mat(m, m->fast_embed, type, ne, host, nbytes, dim, hp.codebook_size, hp.codebook_size, 1, 0, name);
    case SL_FNORM: return upload_vec(m, &m->fast_norm, type, ne, host, nbytes, dim, name);
    case SL_FOUT:
        return upload_mat(m, m->fast_out, type, ne, host, nbytes, dim, hp.codebook_size, hp.codebook_size, 1, 0, name);
    case SL_ATTN_NORM: return upload_vec(m, &L->attn_norm, type, ne, host, nbytes, dim, name);
    case SL_FFN_NORM: return upload_vec(m, &L->ffn_norm, type, ne, host, nbytes, dim, name);
    case SL_QN: return upload_vec(m, &L->q_norm, type, ne, host, nbytes, hd, name);
    case SL_KN: return upload_vec(m, &L->k_norm, type, ne, host, nbytes, hd, name);
    case SL_WQKV: {
        const int rows = (H + 2 * Hkv) * hd;
        return upload_mat(m, L->wqkv, type, ne, host, nbytes, dim, rows, rows, 1, 0, name);
    }
    case SL_WO: return upload_mat(m, L->wo, type, ne, host, nbytes, (int64_t)H * hd, dim, dim, 1, 0, name);
    case SL_W1: {
        s2k_status rc = upload_mat(m, L->w13, type, ne, host, nbytes, dim, ff, 2 * ff, 2, 0, name);
        if (!rc) L->has_w1 = true;
        return rc;
    }
    case SL_W3: {
        s2k_status rc = upload_mat(m, L->w13, type, ne, host, nbytes, dim, ff, 2 * ff, 2, 1, name);
        if (!rc) L->has_w3 = true;
        return rc;
    }
    case SL_W2: return upload_mat(m, L->w2, type, ne, host, nbytes, ff, dim, dim, 1, 0, name);
    default: return fail(S2K_ERR_ARG, "unhandled tensor '%s'", name);
    }
}

S2K_API s2k_status s2k_model_finalize(s2k_model *m) {
    if (!m) return fail(S2K_ERR_ARG, "NULL model");
    if (m->finalized) return S2K_OK;
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_hparams &hp = m->hp;
    if (!m->embed.w) return fail(S2K_ERR_STATE, "missing tensor: embeddings.weight");
    if (hp.num_codebooks > 0 && !m->cb_embed.w) return fail(S2K_ERR_STATE, "missing tensor: codebook_embeddings.weight");
    if (!m->norm) return fail(S2K_ERR_STATE, "missing tensor: norm.weight");
    auto check_layers = [&](std::vector<Layer> &ls, bool fast) -> s2k_status {
        const int qkn = fast ? hp.fast_attention_qk_norm : hp.attention_qk_norm;
        for (size_t i = 0; i < ls.size(); ++i) {
            Layer &L = ls[i];
            const char *pre = fast ? "fast_layers" : "layers";
            if (!L.attn_norm) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.attention_norm.weight", pre, i);
            if (!L.ffn_norm) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.ffn_norm.weight", pre, i);
            if (!L.wqkv.w) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.attention.wqkv.weight", pre, i);
            if (!L.wo.w) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.attention.wo.weight", pre, i);
            if (!L.has_w1) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.feed_forward.w1.weight", pre, i);
            if (!L.has_w3) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.feed_forward.w3.weight", pre, i);
            if (!L.w2.w) return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.feed_forward.w2.weight", pre, i);
            if (qkn && (!L.q_norm || !L.k_norm))
                return fail(S2K_ERR_STATE, "missing tensor: %s.%zu.attention.q_norm/k_norm.weight", pre, i);
            if (!qkn) {
                L.q_norm = nullptr;
                L.k_norm = nullptr;
            }
        }
        return S2K_OK;
    };
    s2k_status rc = check_layers(m->layers, false);
    if (rc) return rc;
    if (hp.has_fast_decoder) {
        if (!m->fast_embed.w) return fail(S2K_ERR_STATE, "missing tensor: fast_embeddings.weight");
        if (!m->fast_norm) return fail(S2K_ERR_STATE, "missing tensor: fast_norm.weight");
        if (!m->fast_out.w) return fail(S2K_ERR_STATE, "missing tensor: fast_output.weight");
        rc = check_layers(m->fast_layers, true);
        if (rc) return rc;
    }
    CU(gemv_setup());
    CU(sampler_setup());
    CU(mega_setup());
    CU(attn_setup());
    m->prefill_mma = prefill_setup() == cudaSuccess;
    m->prefill_f16 = m->prefill_mma && prefill_f16_setup() == cudaSuccess;
    cudaGetLastError();  // a device without the tensor-map entry point keeps the GEMV path
    if (m->prefill_mma) {
        // int8 copies of the Slow stack's K-quant matrices for the tensor-core
        // prefill: two layer slots, layer il's copies in slot il % 2, built
        // by run_stack one layer ahead of their GEMMs (kq_layer_build)
        auto al = [](size_t b) { return (b + 255) / 256 * 256; };
        size_t slot = 0;
        for (Layer &L : m->layers) {
            size_t per = 0;
            for (DevMat *dm : {&L.wqkv, &L.wo, &L.w13, &L.w2}) {
                size_t side = 0;
                const size_t nb = kq_prefill_bytes(*dm, &side);
                if (nb) per += al(nb) + al(side);
            }
            slot = std::max(slot, per);
        }
        if (slot > 0) {
            CU(m->alloc(&m->kq_slots[0], slot));
            CU(m->alloc(&m->kq_slots[1], slot));
            for (size_t il = 0; il < m->layers.size(); ++il) {
                uint8_t *base = m->kq_slots[il % 2];
                size_t off = 0;
                for (DevMat *dm : {&m->layers[il].wqkv, &m->layers[il].wo, &m->layers[il].w13, &m->layers[il].w2}) {
                    size_t side = 0;
                    const size_t nb = kq_prefill_bytes(*dm, &side);
                    if (nb == 0) continue;
                    dm->pf = base + off;
                    off += al(nb);
                    dm->pf_side = base + off;
                    off += al(side);
                }
            }
            m->kq_slot_bytes = slot;
        }
    }
    if (m->staging) {
        m->release(m->staging);
        m->staging = nullptr;
        m->staging_bytes = 0;
    }
    CU(m->alloc(&m->logits, (size_t)hp.vocab_size));
    CU(m->alloc(&m->hidden, (size_t)hp.embedding_length));
    rc = upload_rope(m, &m->rope_slow, &m->rope_slow_n, std::max(hp.context_length, 1), hp.head_dim,
                     hp.rope_freq_base);
    if (rc) return rc;
    if (hp.has_fast_decoder) {
        rc = upload_rope(m, &m->rope_fast, &m->rope_fast_n,
                         std::max(hp.fast_context_length, hp.num_codebooks + 1), hp.fast_head_dim,
                         hp.fast_rope_freq_base);
        if (rc) return rc;
    }
    rc = ensure_slow_work(m, 16, 64);
    if (rc) return rc;
    if (hp.has_fast_decoder) {
        const int Tf = std::max(hp.num_codebooks, 2);
        CU(work_alloc(m, m->fw, Tf, Tf, hp.fast_embedding_length, hp.fast_head_count, hp.fast_head_count_kv,
                      hp.fast_head_dim, hp.fast_feed_forward_length, hp.fast_block_count, false, Tf));
        const int fkvs = hp.fast_head_count_kv * hp.fast_head_dim;
        m->fkcur.assign(hp.fast_block_count, nullptr);
        m->fvcur.assign(hp.fast_block_count, nullptr);
        for (int i = 0; i < hp.fast_block_count; ++i) {
            CU(m->alloc(&m->fkcur[i], (size_t)Tf * fkvs));
            CU(m->alloc(&m->fvcur[i], (size_t)Tf * fkvs));
        }
        CU(m->alloc(&m->flogits, (size_t)hp.codebook_size));
        CU(m->alloc(&m->fhidden, (size_t)hp.embedding_length));
        CU(m->alloc(&m->fcodes, 16));
    }
    CU(cudaStreamSynchronize(m->stream));
    m->finalized = true;
    return S2K_OK;
}

// The sequence's KV pages and hidden-state buffer as the batched-frame
// kernels read them from its device state.
s2k_status seq_publish(s2k_seq *s) {
    const KvPaged kv = s->kv();
    CU(cudaMemcpy(&s->dev->kv, &kv, sizeof(KvPaged), cudaMemcpyHostToDevice));
    CU(cudaMemcpy(&s->dev->hidden, &s->hidden, sizeof(float *), cudaMemcpyHostToDevice));
    return S2K_OK;
}

S2K_API s2k_status s2k_seq_create(s2k_model *m, int32_t max_seq_len, s2k_seq **out) {
    if (!m || !out || max_seq_len <= 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (max_seq_len > m->rope_slow_n)
        return fail(S2K_ERR_ARG, "max_seq_len %d exceeds context_length %d", max_seq_len, m->rope_slow_n);
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    *out = nullptr;
    s2k_seq *s = new s2k_seq();
    s->m = m;
    s->max_seq_len = max_seq_len;
    s->n_pages = (max_seq_len + kPage - 1) / kPage;
    const s2k_hparams &hp = m->hp;
    const size_t page_elems = (size_t)hp.block_count * hp.head_count_kv * kPage * hp.head_dim;
    auto cleanup = [&](s2k_status code, const char *what) {
        s2k_seq_free(s);
        return fail(code, "s2k_seq_create: %s", what);
    };
    if (m->alloc(&s->k, page_elems * s->n_pages) || m->alloc(&s->v, page_elems * s->n_pages))
        return cleanup(S2K_ERR_OOM, "KV pages");
    std::vector<int> bt(s->n_pages);
    for (int i = 0; i < s->n_pages; ++i) bt[i] = i;
    if (m->alloc(&s->block_table, (size_t)s->n_pages) ||
        cudaMemcpy(s->block_table, bt.data(), bt.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
        return cleanup(S2K_ERR_OOM, "block table");
    if (m->alloc(&s->hidden, (size_t)hp.embedding_length)) return cleanup(S2K_ERR_OOM, "hidden state");
    if (m->alloc(&s->dev, 1) || cudaMemset(s->dev, 0, sizeof(SeqDev)) != cudaSuccess)
        return cleanup(S2K_ERR_OOM, "sequence state");
    if (seq_publish(s) != S2K_OK) return cleanup(S2K_ERR_CUDA, "sequence state");
    if (cudaHostAlloc((void **)&s->hstat, sizeof(HostStatus), cudaHostAllocMapped) != cudaSuccess)
        return cleanup(S2K_ERR_OOM, "host status");
    memset((void *)s->hstat, 0, sizeof(HostStatus));
    if (cudaHostGetDevicePointer((void **)&s->hstat_dev, (void *)s->hstat, 0) != cudaSuccess)
        return cleanup(S2K_ERR_CUDA, "host status mapping");
    *out = s;
    return S2K_OK;
}

S2K_API s2k_status s2k_seq_reset(s2k_seq *s) {
    if (!s) return fail(S2K_ERR_ARG, "NULL sequence");
    if (cuda_set(s->m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    CU(cudaMemsetAsync(&s->dev->state, 0, sizeof(SeqState), s->m->stream));
    CU(cudaStreamSynchronize(s->m->stream));
    s->n_past = 0;
    return S2K_OK;
}

S2K_API void s2k_seq_free(s2k_seq *s) {
    if (!s) return;
    s2k_model *m = s->m;
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    if (s->frame_exec) cudaGraphExecDestroy(s->frame_exec);
    if (!s->pooled) {
        m->release(s->k);
        m->release(s->v);
    }
    m->release(s->hidden);
    m->release(s->block_table);
    m->release(s->dev);
    m->release(s->codes);
    m->release(s->prompt);
    m->release(s->mega_ops);
    m->release(s->mega_ctl);
    m->release(s->eval_ops);
    m->release(s->eval_ctl);
    m->release(s->eval_tokens);
    if (s->hstat) cudaFreeHost((void *)s->hstat);
    delete s;
}

S2K_API int32_t s2k_seq_n_past(const s2k_seq *s) { return s ? s->n_past : -1; }

s2k_status check_tokens_host(const s2k_model *m, const int32_t *flat, int32_t T) {
    const s2k_hparams &hp = m->hp;
    const int stride = hp.num_codebooks + 1;
    for (int t = 0; t < T; ++t) {
        const int tok = flat[t * stride];
        if (tok < 0 || tok >= hp.vocab_size) return fail(S2K_ERR_ARG, "token %d at %d out of range", tok, t);
        if (tok >= hp.semantic_begin_id && tok <= hp.semantic_end_id)
            for (int cb = 0; cb < hp.num_codebooks; ++cb) {
                const int c = flat[t * stride + 1 + cb];
                if (c < 0 || c >= hp.codebook_size) return fail(S2K_ERR_ARG, "code %d (cb %d, token %d) out of range", c, cb, t);
            }
    }
    return S2K_OK;
}

static s2k_status ensure_eval_program(s2k_model *m, s2k_seq *s);

S2K_API s2k_status s2k_eval(s2k_model *m, s2k_seq *s, const int32_t *flat, int32_t T, float *hidden_out,
                            float *logits_out) {
    if (!m || !s || !flat || T <= 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (s->m != m) return fail(S2K_ERR_ARG, "sequence belongs to another model");
    if (s->n_past + T > s->max_seq_len)
        return fail(S2K_ERR_KV_FULL, "KV cache overflow (%d + %d > %d)", s->n_past, T, s->max_seq_len);
    s2k_status rc = check_tokens_host(m, flat, T);
    if (rc) return rc;
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    rc = ensure_slow_work(m, T, s->max_seq_len);
    if (rc) return rc;
    const int stride = m->hp.num_codebooks + 1;
    bool on_mega = false;
    if (T == 1 && !s->pooled) {
        // one token: the whole step as one persistent-kernel launch
        rc = ensure_eval_program(m, s);
        if (rc) return rc;
        on_mega = s->eval_ok;
    }
    if (on_mega) {
        CU(cudaMemcpyAsync(s->eval_tokens, flat, (size_t)stride * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        CU(cudaMemsetAsync(s->eval_ctl, 0, sizeof(MegaCtl), m->stream));
        CU(launch_mega(s->eval_ops, s->eval_len, 1, s->eval_ctl, nullptr, m->d_err, m->num_sms, m->stream, m->d_epoch,
                       s->eval_q8));
    } else {
        if (m->tokens_cap < T * stride) {
            m->release(m->tokens);
            m->tokens = nullptr;
            CU(m->alloc(&m->tokens, (size_t)T * stride));
            m->tokens_cap = T * stride;
        }
        CU(cudaMemcpyAsync(m->tokens, flat, (size_t)T * stride * sizeof(int), cudaMemcpyHostToDevice, m->stream));
        CU(enqueue_slow(m, s, T, m->tokens, nullptr));
    }
    if (hidden_out)
        CU(cudaMemcpyAsync(hidden_out, m->hidden, (size_t)m->hp.embedding_length * 4, cudaMemcpyDeviceToHost, m->stream));
    if (logits_out)
        CU(cudaMemcpyAsync(logits_out, m->logits, (size_t)m->hp.vocab_size * 4, cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    rc = check_err_word(m);
    if (rc) return rc;
    s->n_past += T;
    return S2K_OK;
}

S2K_API s2k_status s2k_fast_decode(s2k_model *m, const float *hidden, const int32_t *prefix, int32_t n_prefix,
                                   float *logits_out) {
    if (!m || !hidden || !logits_out || n_prefix < 0 || (n_prefix > 0 && !prefix)) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    const s2k_hparams &hp = m->hp;
    if (!hp.has_fast_decoder) return fail(S2K_ERR_STATE, "model has no fast decoder");
    if (n_prefix >= hp.num_codebooks)
        return fail(S2K_ERR_ARG, "prefix too long (%d >= %d)", n_prefix, hp.num_codebooks);
    for (int i = 0; i < n_prefix; ++i)
        if (prefix[i] < 0 || prefix[i] >= hp.codebook_size) return fail(S2K_ERR_ARG, "prefix code %d out of range", prefix[i]);
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const int T = n_prefix + 1;
    CU(cudaMemcpyAsync(m->fhidden, hidden, (size_t)hp.embedding_length * 4, cudaMemcpyHostToDevice, m->stream));
    if (n_prefix > 0)
        CU(cudaMemcpyAsync(m->fcodes, prefix, (size_t)n_prefix * 4, cudaMemcpyHostToDevice, m->stream));
    CU(launch_embed_fast(&m->fast_embed, m->fhidden, m->fcodes, 0, T, m->fw.x, hp.fast_embedding_length, nullptr,
                         m->d_err, m->stream));
    CU(enqueue_fast(m, T, 0, nullptr));
    CU(cudaMemcpyAsync(logits_out, m->flogits, (size_t)hp.codebook_size * 4, cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return check_err_word(m);
}

S2K_API s2k_status s2k_sample(s2k_model *m, const float *logits, int32_t n, float temperature, float top_p,
                              int32_t top_k, double u, int32_t *token_out) {
    if (!m || !logits || !token_out || n <= 0 || n > 8192) return fail(S2K_ERR_ARG, "bad argument (n <= 8192)");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    if (m->samp_cap < n) {
        m->release(m->samp_logits);
        m->samp_logits = nullptr;
        CU(m->alloc(&m->samp_logits, (size_t)n));
        m->samp_cap = n;
    }
    if (!m->samp_out) CU(m->alloc(&m->samp_out, 1));
    CU(cudaMemcpyAsync(m->samp_logits, logits, (size_t)n * 4, cudaMemcpyHostToDevice, m->stream));
    CU(launch_sample_one(m->samp_logits, n, temperature, top_p, top_k, u, m->samp_out, m->d_err, m->stream));
    CU(cudaMemcpyAsync(token_out, m->samp_out, 4, cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return check_err_word(m);
}

// ---------------------------------------------------------------------------
// allocation-free sampler entry: fixed per-device scratch in a static
// __device__ array -- [0, 4*max) logits row, then the token slot and, 16
// bytes in, the error block (error word and wait limit, the part that must
// start at zero: cleared every call).
// ---------------------------------------------------------------------------
static_assert(S2K_SAMPLE_NOALLOC_MAX_N <= 8192, "the sampler kernel takes at most 8192 logits");
constexpr size_t kNoAllocTokOff = (size_t)S2K_SAMPLE_NOALLOC_MAX_N * sizeof(float);
constexpr size_t kNoAllocErrOff = kNoAllocTokOff + 16;
static __device__ __align__(256) unsigned char g_sample_scratch[kNoAllocTokOff + 256];
static_assert(kNoAllocErrOff + kErrBlockInts * sizeof(int) <= sizeof(g_sample_scratch), "scratch layout");
constexpr int kNoAllocMaxDevices = 64;
// Per device: the array's device address and the context it was looked up
// in.  A device reset gives the device a new context, and the address is
// looked up again there.
struct NoAllocScratch {
    void *ptr = nullptr;
    void *ctx = nullptr;
};
static NoAllocScratch g_sample_scratch_at[kNoAllocMaxDevices];
static std::mutex g_sample_scratch_mu;

// The current context (cuCtxGetCurrent through the runtime's driver entry
// point, so the library needs no link against libcuda), or null.
static void *current_context() {
    typedef int (*CtxGetCurrent)(void **);
    static CtxGetCurrent fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrent>(p);
    }();
    void *ctx = nullptr;
    if (!fn || fn(&ctx) != 0) return nullptr;
    return ctx;
}

S2K_API s2k_status s2k_sample_noalloc(s2k_model *m, const float *logits, int32_t n, float temperature, float top_p,
                                      int32_t top_k, double u, int32_t *token_out) {
    if (!m || !logits || !token_out) return fail(S2K_ERR_ARG, "bad argument");
    if (n <= 0 || n > S2K_SAMPLE_NOALLOC_MAX_N)
        return fail(S2K_ERR_ARG, "s2k_sample_noalloc: n = %d outside its fixed scratch (1..%d logits)", n,
                    S2K_SAMPLE_NOALLOC_MAX_N);
    if (m->device < 0 || m->device >= kNoAllocMaxDevices) return fail(S2K_ERR_ARG, "device %d out of range", m->device);
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_sample_scratch_mu);
        NoAllocScratch &sc = g_sample_scratch_at[m->device];
        void *ctx = current_context();
        if (!sc.ptr || ctx != sc.ctx) {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_sample_scratch);
            if (e != cudaSuccess || !p)
                return fail(S2K_ERR_CUDA, "cudaGetSymbolAddress(sampler scratch) failed: %s", cudaGetErrorString(e));
            sc.ptr = p;
            sc.ctx = ctx;
        }
        base = sc.ptr;
    }
    float *d_logits = static_cast<float *>(base);
    int *d_tok = reinterpret_cast<int *>(static_cast<unsigned char *>(base) + kNoAllocTokOff);
    int *d_err = reinterpret_cast<int *>(static_cast<unsigned char *>(base) + kNoAllocErrOff);
    int h_tok = 0, h_err = 0;
    CU(cudaMemsetAsync(d_err, 0, kErrBlockInts * sizeof(int), m->stream));
    CU(cudaMemcpyAsync(d_logits, logits, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, m->stream));
    CU(launch_sample_one(d_logits, n, temperature, top_p, top_k, u, d_tok, d_err, m->stream));
    CU(cudaMemcpyAsync(&h_tok, d_tok, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    CU(cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    if (h_err) return fail(S2K_ERR_ARG, "device reported invalid input (flags 0x%x)", h_err);
    *token_out = h_tok;
    return S2K_OK;
}

// ---------------------------------------------------------------------------
// persistent-kernel frame program
// ---------------------------------------------------------------------------
// A GEMV op of the persistent kernel.  ll says which of x / res / y are
// tagged activation words; the tags are the segment-relative indices of the
// ops that write them (the kernel adds the launch epoch).
static MegaOp mk_gemv(const DevMat &w, const void *x, int ldx, int M, int in_mode, const float *nw, float eps,
                      int epi, void *y, int ldy, const void *res, int ldres, float *act_out, int ll = 0,
                      int x_tag = 0, int res_tag = 0, int y_tag = 0) {
    MegaOp o;
    memset(&o, 0, sizeof(o));
    o.kind = MK_GEMV;
    o.g.ll = ll;
    o.g.x_tag = (uint32_t)x_tag;
    o.g.res_tag = (uint32_t)res_tag;
    o.g.y_tag = (uint32_t)y_tag;
    o.g.w = w.w;
    o.g.wtype = tw_of(w.type);
    o.g.R = w.rows;
    o.g.K = w.cols;
    o.g.x = static_cast<const float *>(x);
    o.g.ldx = ldx;
    o.g.M = M;
    o.g.in_mode = in_mode;
    o.g.norm_w = nw;
    o.g.eps = eps;
    o.g.epi = epi;
    o.g.y = static_cast<float *>(y);
    o.g.ldy = ldy;
    o.g.res = static_cast<const float *>(res);
    o.g.ldres = ldres;
    o.g.act_out = act_out;
    return o;
}

// One transformer stack (a4-a11 of the reference step) as persistent-kernel ops.
// One transformer stack (a4-a11 of the reference step) as persistent-kernel
// ops on the tagged activation buffers.  start: the segment's first op;
// x_op: segment-relative index of the op that last wrote x (updated).
static bool add_layers(s2k_model *m, s2k_seq *s, bool fast, int T, int pos_add, std::vector<MegaOp> &ops, int start,
                       int &x_op) {
    const s2k_hparams &hp = m->hp;
    Work &w = fast ? m->fw : m->sw;
    const std::vector<Layer> &layers = fast ? m->fast_layers : m->layers;
    const int H = fast ? hp.fast_head_count : hp.head_count;
    const int Hkv = fast ? hp.fast_head_count_kv : hp.head_count_kv;
    const int hd = fast ? hp.fast_head_dim : hp.head_dim;
    const float eps = fast ? hp.fast_rms_norm_eps : hp.rms_norm_eps;
    const int qkvs = w.qs + 2 * w.kvs, dim = w.dim;
    const size_t tn = (size_t)std::max(w.Tm, 1);
    if (T > w.Tm) return false;
    for (size_t il = 0; il < layers.size(); ++il) {
        const Layer &L = layers[il];
        const int q_op = (int)ops.size() - start, a_op = q_op + 1, o_op = q_op + 2, f_op = q_op + 3, d_op = q_op + 4;
        ops.push_back(mk_gemv(L.wqkv, w.lx, dim, T, IN_RMSNORM, L.attn_norm, eps, EPI_STORE, w.lqkv, qkvs, nullptr, 0,
                              nullptr, LL_X | LL_Y, x_op, 0, q_op));
        MegaOp a;
        memset(&a, 0, sizeof(a));
        a.kind = MK_ATTN;
        a.a.qkv = w.lqkv;
        a.a.in_tag = (uint32_t)q_op;
        a.a.out_tag = (uint32_t)a_op;
        a.a.ldqkv = qkvs;
        a.a.T = T;
        a.a.H = H;
        a.a.Hkv = Hkv;
        a.a.hd = hd;
        a.a.q_norm = L.q_norm;
        a.a.k_norm = L.k_norm;
        a.a.eps = eps;
        a.a.scale = 1.0f / sqrtf((float)hd);
        a.a.rope = fast ? m->rope_fast : m->rope_slow;
        a.a.rope_positions = fast ? m->rope_fast_n : m->rope_slow_n;
        a.a.pos_base = fast ? nullptr : &s->dev->state.n_past;
        a.a.pos_add = pos_add;
        a.a.n_cached_from_pos_base = fast ? 0 : 1;
        a.a.kcur = fast ? m->fkcur[il] : w.kcur;
        a.a.vcur = fast ? m->fvcur[il] : w.vcur;
        a.a.cur_base = fast ? pos_add : 0;
        if (!fast) {
            a.a.kv_k = s->k;
            a.a.kv_v = s->v;
            a.a.block_table = s->block_table;
            a.a.kv_layers = hp.block_count;
            a.a.kv_pages = s->n_pages;
        }
        a.a.layer = (int)il;
        a.a.part = w.part;
        a.a.part_ms = w.part_ms;
        a.a.counters = w.counters + il * tn * Hkv * kAttnMaxGroup;  // per layer: none is reused within a launch
        a.a.n_split_max = w.n_split_max;
        a.a.out = w.lattn;
        if (T * H > w.Tm * w.H || !mega_attn_ok(a.a, fast ? pos_add + T : s->max_seq_len)) return false;
        ops.push_back(a);
        ops.push_back(mk_gemv(L.wo, w.lattn, w.qs, T, IN_PLAIN, nullptr, eps, EPI_STORE, w.lh, dim, w.lx, dim, nullptr,
                              LL_X | LL_RES | LL_Y, a_op, x_op, o_op));
        ops.push_back(mk_gemv(L.w13, w.lh, dim, T, IN_RMSNORM, L.ffn_norm, eps, EPI_SWIGLU, w.lff, w.ff, nullptr, 0,
                              nullptr, LL_X | LL_Y, o_op, 0, f_op));
        ops.push_back(mk_gemv(L.w2, w.lff, w.ff, T, IN_PLAIN, nullptr, eps, EPI_STORE, w.lx, dim, w.lh, dim, nullptr,
                              LL_X | LL_RES | LL_Y, f_op, o_op, d_op));
        x_op = d_op;
    }
    return true;
}

// The Slow-AR step over one token (eval_cached with n_tokens = 1,
// src/s2_model.cpp:860-1097) as persistent-kernel ops appended to `ops`:
// embedding of the token row at `tokens` ([num_codebooks+1] ints in device
// memory), the layers, the final norm + tied LM head (logits, post-norm
// hidden), then n_past += 1.  False when a shape falls outside the kernel's
// limits.
static bool push_slow_step(s2k_model *m, s2k_seq *s, const int *tokens, std::vector<MegaOp> &ops) {
    const s2k_hparams &hp = m->hp;
    const int start = (int)ops.size();
    MegaOp e;
    memset(&e, 0, sizeof(e));
    e.kind = MK_EMBED_SLOW;
    e.es.e = m->embed.w;
    e.es.etype = tw_of(m->embed.type);
    e.es.ctype = hp.num_codebooks > 0 ? tw_of(m->cb_embed.type) : 0;
    e.es.e_rows = m->embed.rows;
    e.es.dim = hp.embedding_length;
    e.es.c = hp.num_codebooks > 0 ? m->cb_embed.w : nullptr;
    e.es.c_rows = hp.num_codebooks > 0 ? m->cb_embed.rows : 0;
    e.es.tokens = tokens;
    e.es.T = 1;
    e.es.ncb = hp.num_codebooks;
    e.es.cb_size = hp.codebook_size;
    e.es.sem_begin = hp.semantic_begin_id;
    e.es.sem_end = hp.semantic_end_id;
    e.es.scale_cb = hp.scale_codebook_embeddings;
    e.es.sem_scale = 1.0f / sqrtf((float)(hp.num_codebooks + 1));
    e.es.x = m->sw.lx;
    e.es.tag = 0;
    ops.push_back(e);
    int x_op = 0;
    if (!add_layers(m, s, false, 1, 0, ops, start, x_op)) return false;
    ops.push_back(mk_gemv(m->embed, m->sw.lx, hp.embedding_length, 1, IN_RMSNORM, m->norm, hp.rms_norm_eps,
                          EPI_STORE, m->logits, hp.vocab_size, nullptr, 0, m->hidden, LL_X, x_op));
    MegaOp adv;
    memset(&adv, 0, sizeof(adv));
    adv.kind = MK_ADVANCE;
    adv.adv.n_past = &s->dev->state.n_past;
    adv.adv.T = 1;
    ops.push_back(adv);
    for (size_t i = (size_t)start; i < ops.size(); ++i)
        if (ops[i].kind == MK_GEMV && !mega_gemv_ok(ops[i].g)) return false;
    if ((int)ops.size() - start > 255) return false;  // op indices are the low 8 bits of the activation tags
    return hp.num_codebooks <= 16;  // the persistent kernel's embedding sums at most 16 codebooks
}

// A single-token s2k_eval on the persistent kernel: the Slow step segment
// reading its token row from the sequence's eval_tokens, built once per
// sequence and workspace generation.
static s2k_status ensure_eval_program(s2k_model *m, s2k_seq *s) {
    if (s->eval_gen == m->ws_gen) return S2K_OK;
    if (!s->eval_tokens) CU(m->alloc(&s->eval_tokens, 32));
    if (!s->eval_ctl) CU(m->alloc(&s->eval_ctl, 1));
    std::vector<MegaOp> ops;
    s->eval_ok = push_slow_step(m, s, s->eval_tokens, ops);
    s->eval_q8 = true;
    for (const MegaOp &o : ops)
        if (o.kind == MK_GEMV && o.g.wtype != TW_Q8_0) s->eval_q8 = false;
    m->release(s->eval_ops);
    s->eval_ops = nullptr;
    s->eval_len = 0;
    if (s->eval_ok) {
        CU(m->alloc(&s->eval_ops, ops.size()));
        CU(cudaMemcpy(s->eval_ops, ops.data(), ops.size() * sizeof(MegaOp), cudaMemcpyHostToDevice));
        s->eval_len = (int)ops.size();
    }
    s->eval_gen = m->ws_gen;
    return S2K_OK;
}

// Builds the segments of one frame: 9 Fast-AR passes and the Slow step.
// Returns false (and the caller uses the per-op kernels) when a shape falls
// outside the persistent kernel's limits.
static s2k_status build_mega(s2k_model *m, s2k_seq *s) {
    const s2k_hparams &hp = m->hp;
    std::vector<MegaOp> ops;
    s->seg_start.clear();
    s->seg_len.clear();
    s->seg_mt.clear();
    bool ok = true;
    for (int p = 0; p + 1 < hp.num_codebooks; ++p) {
        const int T = p == 0 ? 2 : 1, pos_add = p == 0 ? 0 : p + 1;
        const int start = (int)ops.size();
        MegaOp e;
        memset(&e, 0, sizeof(e));
        e.kind = MK_EMBED_FAST;
        e.ef.f = m->fast_embed.w;
        e.ef.ftype = tw_of(m->fast_embed.type);
        e.ef.f_rows = m->fast_embed.rows;
        e.ef.hidden = p == 0 ? m->hidden : nullptr;
        e.ef.codes = s->dev->state.codes;
        e.ef.code0 = p;
        e.ef.n_rows = T;
        e.ef.dim = hp.fast_embedding_length;
        e.ef.x = m->fw.lx;
        e.ef.tag = 0;
        ops.push_back(e);
        int x_op = 0;
        ok = ok && add_layers(m, s, true, T, pos_add, ops, start, x_op);
        ops.push_back(mk_gemv(m->fast_out, m->fw.lx + (size_t)(T - 1) * hp.fast_embedding_length,
                              hp.fast_embedding_length, 1, IN_RMSNORM, m->fast_norm, hp.fast_rms_norm_eps, EPI_STORE,
                              m->flogits, hp.codebook_size, nullptr, 0, nullptr, LL_X, x_op));
        s->seg_start.push_back(start);
        s->seg_len.push_back((int)ops.size() - start);
        s->seg_mt.push_back(T);
    }
    {
        const int start = (int)ops.size();
        ok = ok && push_slow_step(m, s, s->dev->state.step_in, ops);
        s->seg_start.push_back(start);
        s->seg_len.push_back((int)ops.size() - start);
        s->seg_mt.push_back(1);
    }
    for (const MegaOp &o : ops)
        if (o.kind == MK_GEMV && !mega_gemv_ok(o.g)) ok = false;
    for (size_t i = 0; i < s->seg_len.size(); ++i)
        if (s->seg_len[i] > 255) ok = false;  // op indices are the low 8 bits of the activation tags
    if (hp.num_codebooks > 16) ok = false;  // the persistent kernel's embedding sums at most 16 codebooks
    s->use_mega = ok;
    if (!ok) return S2K_OK;
    s->mega_q8 = true;  // every GEMV Q8_0: the kernel variant with that consumer only
    for (const MegaOp &o : ops)
        if (o.kind == MK_GEMV && o.g.wtype != TW_Q8_0) s->mega_q8 = false;
    m->release(s->mega_ops);
    s->mega_ops = nullptr;
    CU(m->alloc(&s->mega_ops, ops.size()));
    CU(cudaMemcpy(s->mega_ops, ops.data(), ops.size() * sizeof(MegaOp), cudaMemcpyHostToDevice));
    if (!s->mega_ctl) CU(m->alloc(&s->mega_ctl, 16));
    return S2K_OK;
}

// The frame with the persistent kernel: one cooperative launch per segment,
// the samplers between them.
static cudaError_t enqueue_frame_mega(s2k_model *m, s2k_seq *s) {
    const s2k_hparams &hp = m->hp;
    cudaStream_t st = m->stream;
    const int *done = &s->dev->state.done;
    const int nseg = (int)s->seg_start.size();
    cudaError_t e;
    if ((e = cudaMemsetAsync(s->mega_ctl, 0, sizeof(MegaCtl) * nseg, st))) return e;
    for (int p = 0; p + 1 < hp.num_codebooks; ++p) {
        if ((e = launch_mega(s->mega_ops + s->seg_start[p], s->seg_len[p], s->seg_mt[p], s->mega_ctl + p, done,
                             m->d_err, m->num_sms, st, m->d_epoch, s->mega_q8)))
            return e;
        if ((e = launch_sample_fast(m->flogits, s->dev, p + 1, m->d_err, st))) return e;
    }
    if ((e = launch_frame_commit(s->dev, st))) return e;
    const int last = nseg - 1;
    if ((e = launch_mega(s->mega_ops + s->seg_start[last], s->seg_len[last], s->seg_mt[last], s->mega_ctl + last, done,
                         m->d_err, m->num_sms, st, m->d_epoch, s->mega_q8)))
        return e;
    return launch_sample_main(m->logits, s->dev, m->d_err, st);
}

// Frame graph: captured once per sequence; it reads everything that changes
// per frame or per call (positions, tokens, sampling parameters, output
// pointer) from the sequence's device state.
static s2k_status ensure_frame_graph(s2k_model *m, s2k_seq *s) {
    if (s->frame_exec && s->frame_gen == m->ws_gen) return S2K_OK;
    if (s->frame_exec) {
        cudaGraphExecDestroy(s->frame_exec);
        s->frame_exec = nullptr;
    }
    cudaGraph_t g = nullptr;
    const unsigned long long before = g_launches.load();
    s2k_status brc = build_mega(m, s);
    if (brc) return brc;
    CU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = s->use_mega ? enqueue_frame_mega(m, s) : enqueue_frame(m, s);
    cudaError_t e2 = cudaStreamEndCapture(m->stream, &g);
    g_launches.store(before);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return fail(S2K_ERR_CUDA, "frame capture failed: %s / %s", cudaGetErrorString(e), cudaGetErrorString(e2));
    }
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    s->frame_nodes = n;
    e = cudaGraphInstantiate(&s->frame_exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        s->frame_exec = nullptr;
        return fail(S2K_ERR_CUDA, "frame graph instantiate: %s", cudaGetErrorString(e));
    }
    s->frame_gen = m->ws_gen;
    return S2K_OK;
}

void fill_sample_cfg(const s2k_model *m, const s2k_gen_params *gp, int *d_codes, int codes_ld, SampleCfg *out) {
    const s2k_hparams &hp = m->hp;
    SampleCfg c;
    memset(&c, 0, sizeof(c));
    c.temperature = gp->temperature;
    c.top_p = gp->top_p;
    c.top_k = gp->top_k;
    c.min_tokens_before_end = gp->min_tokens_before_end;
    c.im_end = gp->im_end_id;
    c.max_new_tokens = gp->max_new_tokens;
    c.seed = gp->seed;
    c.seq_id = gp->seq_id;
    c.sem_begin = hp.semantic_begin_id;
    c.sem_end = hp.semantic_end_id;
    c.cb_size = hp.codebook_size;
    c.ncb = std::max(hp.num_codebooks, 1);
    c.vocab = hp.vocab_size;
    c.codes_out = d_codes;
    c.codes_ld = codes_ld;
    *out = c;
}

// The frame loop of generate() (src/s2_generate.cpp:57-183) on the device.
// Each frame is one graph launch; up to kLookahead frames run ahead of the
// host.  Frame f's codes reach the host ring (HostStatus::ring) when its
// frame_commit kernel ends, and on_frame (if any) is called for it as soon
// as the host sees them, while later frames run.  A zero return stops
// launching frames: the frames already in flight finish on the device, the
// result keeps frames 0..f, and n_past ends at cols + f, where the reference
// model stands when it breaks before step() (src/s2_generate.cpp:150-163).
static s2k_status generate_core(s2k_model *m, s2k_seq *s, const int32_t *d_prompt_tm, int32_t cols,
                                const s2k_gen_params *gp, int32_t *d_codes, int32_t codes_ld, int32_t *n_frames_out,
                                s2k_frame_callback on_frame, void *user) {
    const s2k_hparams &hp = m->hp;
    if (cols <= 0 || gp->max_new_tokens < 0) return fail(S2K_ERR_ARG, "bad prompt length / max_new_tokens");
    if (cols + gp->max_new_tokens > s->max_seq_len)
        return fail(S2K_ERR_KV_FULL, "sequence holds %d positions, need %d", s->max_seq_len, cols + gp->max_new_tokens);
    if (!hp.has_fast_decoder && hp.num_codebooks > 1) return fail(S2K_ERR_STATE, "model has no fast decoder");
    s2k_status rc = ensure_slow_work(m, cols, s->max_seq_len);
    if (rc) return rc;
    SampleCfg c;
    fill_sample_cfg(m, gp, d_codes, codes_ld, &c);
    const int ncb = c.ncb;
    // the Pipeline clears and re-inits the KV cache per synthesis (src/s2_pipeline.cpp:838-851)
    CU(cudaMemsetAsync(&s->dev->state, 0, sizeof(SeqState), m->stream));
    CU(cudaMemcpyAsync(&s->dev->cfg, &c, sizeof(SampleCfg), cudaMemcpyHostToDevice, m->stream));
    HostStatus *hs_dev = s->hstat_dev;
    CU(cudaMemcpyAsync(&s->dev->host, &hs_dev, sizeof(HostStatus *), cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    volatile HostStatus *hs = s->hstat;
    hs->n_frames = 0;
    hs->done = 0;
    s->n_past = 0;
    // the reference's [Metrics] split (src/s2_generate.cpp:185-199), timed on the device
    cudaEvent_t tev[3];
    for (int i = 0; i < 3; ++i) CU(cudaEventCreate(&tev[i]));
    struct EventGuard {
        cudaEvent_t *e;
        ~EventGuard() {
            for (int i = 0; i < 3; ++i) cudaEventDestroy(e[i]);
        }
    } tev_guard{tev};
    nvtxRangePushA("s2k generate: prefill");
    // prefill (generate(): prefill_fast of the whole prompt, src/s2_generate.cpp:51)
    CU(cudaEventRecord(tev[0], m->stream));
    CU(enqueue_slow(m, s, cols, d_prompt_tm, nullptr));
    CU(launch_sample_main(m->logits, s->dev, m->d_err, m->stream));
    CU(cudaEventRecord(tev[1], m->stream));
    nvtxRangePop();
    rc = ensure_frame_graph(m, s);
    if (rc) return rc;
    nvtxRangePushA("s2k generate: frame loop");
    constexpr int kLookahead = 4;
    static_assert(kLookahead < kFrameRing, "frames in flight must not overwrite ring slots the host has not read");
    cudaEvent_t ev[kLookahead];
    for (int i = 0; i < kLookahead; ++i) CU(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
    s2k_status out_rc = S2K_OK;
    int launched = 0, delivered = 0;
    bool aborted = false;
    // hand frames [delivered, upto) to on_frame; false once it asks to stop
    auto deliver = [&](int upto) -> bool {
        for (; delivered < upto; ++delivered) {
            if (!on_frame) continue;
            int codes[16];
            for (int cb = 0; cb < ncb; ++cb) codes[cb] = hs->ring[delivered % kFrameRing][cb];
            if (!on_frame(codes, delivered, delivered + 1, ncb, user)) {
                ++delivered;
                return false;
            }
        }
        return true;
    };
    for (;;) {
        const int landed = hs->n_frames;
        std::atomic_thread_fence(std::memory_order_acquire);
        if (!deliver(landed)) {
            aborted = true;
            break;
        }
        if (hs->done) {
            // the stop was decided after the last frame landed: nothing more comes
            std::atomic_thread_fence(std::memory_order_acquire);
            if (!deliver(hs->n_frames)) aborted = true;
            break;
        }
        if (launched < gp->max_new_tokens && launched - delivered < kLookahead) {
            cudaError_t e = cudaGraphLaunch(s->frame_exec, m->stream);
            if (e == cudaSuccess) e = cudaEventRecord(ev[launched % kLookahead], m->stream);
            if (e != cudaSuccess) {
                out_rc = fail(S2K_ERR_CUDA, "frame %d launch: %s", launched, cudaGetErrorString(e));
                break;
            }
            count_launch((int)s->frame_nodes);
            ++launched;
            continue;
        }
        if (launched == delivered) break;  // every launched frame handed over, none left to launch
        // wait for the graph of the oldest frame the host has not seen
        cudaError_t e = cudaEventSynchronize(ev[delivered % kLookahead]);
        if (e != cudaSuccess) {
            out_rc = fail(S2K_ERR_CUDA, "frame %d: %s", delivered, cudaGetErrorString(e));
            break;
        }
        if (hs->n_frames <= delivered && !hs->done) {
            out_rc = fail(S2K_ERR_STATE, "frame %d ended without codes", delivered);
            break;
        }
    }
    cudaEventRecord(tev[2], m->stream);
    cudaError_t e = cudaStreamSynchronize(m->stream);
    nvtxRangePop();
    for (int i = 0; i < kLookahead; ++i) cudaEventDestroy(ev[i]);
    if (out_rc) return out_rc;
    if (e != cudaSuccess) return fail(S2K_ERR_CUDA, "generate: %s", cudaGetErrorString(e));
    rc = check_err_word(m);
    if (rc) return rc;
    {
        float pre = 0.f, loop = 0.f;
        cudaEventElapsedTime(&pre, tev[0], tev[1]);
        cudaEventElapsedTime(&loop, tev[1], tev[2]);
        s2k_gen_metrics &gm = s->metrics;
        gm.prefill_ms = pre;
        gm.loop_ms = loop;
        gm.total_ms = (double)pre + (double)loop;
        gm.n_frames = aborted ? delivered : hs->n_frames;
        gm.prompt_tokens = cols;
        gm.ms_per_frame = gm.n_frames > 0 ? gm.loop_ms / gm.n_frames : 0.0;
    }
    if (aborted) {
        // the reference breaks before step() of the aborted frame
        const int n_past = cols + delivered - 1;
        CU(cudaMemcpy(&s->dev->state.n_past, &n_past, sizeof(int), cudaMemcpyHostToDevice));
        *n_frames_out = delivered;
        s->n_past = n_past;
        return S2K_OK;
    }
    *n_frames_out = hs->n_frames;
    s->n_past = cols + *n_frames_out;
    return S2K_OK;
}

S2K_API s2k_status s2k_generate_device(s2k_model *m, s2k_seq *s, const int32_t *d_prompt_tm, int32_t cols,
                                       const s2k_gen_params *gp, int32_t *d_codes_out, int32_t *n_frames_out) {
    if (!m || !s || !d_prompt_tm || !gp || !d_codes_out || !n_frames_out) return fail(S2K_ERR_ARG, "NULL argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (s->m != m) return fail(S2K_ERR_ARG, "sequence belongs to another model");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    return generate_core(m, s, d_prompt_tm, cols, gp, d_codes_out, std::max(gp->max_new_tokens, 1), n_frames_out,
                         nullptr, nullptr);
}

S2K_API s2k_status s2k_generate(s2k_model *m, s2k_seq *s, const int32_t *prompt, int32_t cols,
                                const s2k_gen_params *gp, int32_t *codes_out, int32_t *n_frames_out,
                                s2k_frame_callback on_frame, void *user) {
    if (!m || !s || !prompt || !gp || !codes_out || !n_frames_out || cols <= 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (s->m != m) return fail(S2K_ERR_ARG, "sequence belongs to another model");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_hparams &hp = m->hp;
    const int rows = hp.num_codebooks + 1;
    const int ncb = std::max(hp.num_codebooks, 1);
    // PromptTensor [rows][cols] -> token-major, as generate() does (src/s2_generate.cpp:37-44)
    std::vector<int32_t> tm((size_t)rows * cols);
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) tm[(size_t)c * rows + r] = prompt[(size_t)r * cols + c];
    s2k_status rc = check_tokens_host(m, tm.data(), cols);
    if (rc) return rc;
    if (s->prompt_cap < rows * cols) {
        m->release(s->prompt);
        s->prompt = nullptr;
        CU(m->alloc(&s->prompt, (size_t)rows * cols));
        s->prompt_cap = rows * cols;
    }
    const int ld = std::max(gp->max_new_tokens, 1);
    if (s->codes_cap < ld) {
        m->release(s->codes);
        s->codes = nullptr;
        CU(m->alloc(&s->codes, (size_t)ncb * ld));
        s->codes_cap = ld;
    }
    CU(cudaMemcpyAsync(s->prompt, tm.data(), tm.size() * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
    int32_t nf = 0;
    rc = generate_core(m, s, s->prompt, cols, gp, s->codes, ld, &nf, on_frame, user);
    if (rc) return rc;
    // compaction (src/s2_generate.cpp:201-213)
    for (int cb = 0; cb < ncb && nf > 0; ++cb)
        CU(cudaMemcpyAsync(codes_out + (size_t)cb * nf, s->codes + (size_t)cb * ld, (size_t)nf * sizeof(int32_t),
                           cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    *n_frames_out = nf;
    return S2K_OK;
}

S2K_API s2k_status s2k_profile_gemv(s2k_model *m, int32_t reps, double *bytes_per_pass, double *ms_per_pass,
                                    int32_t *launches_per_pass) {
    if (!m || reps <= 0 || !bytes_per_pass || !ms_per_pass || !launches_per_pass) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_hparams &hp = m->hp;
    Work &w = m->sw;
    double bytes = 0;
    int launches = 0;
    auto pass = [&](bool count) -> cudaError_t {
        cudaError_t e;
        for (const Layer &L : m->layers) {
            GemvArgs g;
            g.M = 1;
            g.err = m->d_err;
            g.eps = hp.rms_norm_eps;
            g.w = &L.wqkv; g.x = w.x; g.ldx = w.dim; g.in_mode = IN_RMSNORM; g.norm_w = L.attn_norm;
            g.y = w.qkv; g.ldy = w.qs + 2 * w.kvs;
            if ((e = launch_gemv(g, m->num_sms, m->stream))) return e;
            GemvArgs o = g;
            o.w = &L.wo; o.x = w.attn; o.ldx = w.qs; o.in_mode = IN_PLAIN; o.norm_w = nullptr; o.y = w.h; o.ldy = w.dim;
            o.res = w.x; o.ldres = w.dim;
            if ((e = launch_gemv(o, m->num_sms, m->stream))) return e;
            GemvArgs f1 = g;
            f1.w = &L.w13; f1.x = w.h; f1.ldx = w.dim; f1.norm_w = L.ffn_norm; f1.epi = EPI_SWIGLU; f1.y = w.ff_buf;
            f1.ldy = w.ff;
            if ((e = launch_gemv(f1, m->num_sms, m->stream))) return e;
            GemvArgs f2 = g;
            f2.w = &L.w2; f2.x = w.ff_buf; f2.ldx = w.ff; f2.in_mode = IN_PLAIN; f2.norm_w = nullptr; f2.y = w.x;
            f2.ldy = w.dim; f2.res = w.h; f2.ldres = w.dim;
            if ((e = launch_gemv(f2, m->num_sms, m->stream))) return e;
            if (count) {
                bytes += (double)(L.wqkv.bytes() + L.wo.bytes() + L.w13.bytes() + L.w2.bytes());
                launches += 4;
            }
        }
        GemvArgs hd;
        hd.w = &m->embed; hd.x = w.x; hd.ldx = w.dim; hd.M = 1; hd.in_mode = IN_RMSNORM; hd.norm_w = m->norm;
        hd.eps = hp.rms_norm_eps; hd.y = m->logits; hd.ldy = hp.vocab_size; hd.err = m->d_err;
        if ((e = launch_gemv(hd, m->num_sms, m->stream))) return e;
        if (count) {
            bytes += (double)m->embed.bytes();
            launches += 1;
        }
        return cudaSuccess;
    };
    // deterministic finite activations
    CU(cudaMemsetAsync(w.x, 0, (size_t)w.dim * sizeof(float), m->stream));
    CU(cudaMemsetAsync(w.attn, 0, (size_t)w.qs * sizeof(float), m->stream));
    CU(pass(true));  // warm-up
    cudaEvent_t e0, e1;
    CU(cudaEventCreate(&e0));
    CU(cudaEventCreate(&e1));
    CU(cudaEventRecord(e0, m->stream));
    for (int r = 0; r < reps; ++r) CU(pass(false));
    CU(cudaEventRecord(e1, m->stream));
    CU(cudaEventSynchronize(e1));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *bytes_per_pass = bytes;
    *ms_per_pass = ms / reps;
    *launches_per_pass = launches;
    return check_err_word(m);
}

S2K_API s2k_status s2k_profile_frame(s2k_model *m, s2k_seq *s, int32_t reps, double *ms_slow, double *ms_fast,
                                     double *bytes_slow, double *bytes_fast) {
    if (!m || !s || reps <= 0 || reps > 64 || !ms_slow || !ms_fast || !bytes_slow || !bytes_fast)
        return fail(S2K_ERR_ARG, "bad argument (1 <= reps <= 64)");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    if (!s->frame_exec || s->frame_gen != m->ws_gen || !s->use_mega || s->seg_start.size() < 2)
        return fail(S2K_ERR_STATE, "no persistent-kernel frame program for this sequence (run generate first)");
    if (s->n_past >= s->max_seq_len)
        return fail(S2K_ERR_KV_FULL, "profiling writes position n_past = %d; the sequence holds %d", s->n_past,
                    s->max_seq_len);
    const s2k_hparams &hp = m->hp;
    const int nseg = (int)s->seg_start.size();
    const int fseg = nseg > 2 ? 1 : 0, sseg = nseg - 1;
    // the Slow segment ends with the n_past advance: leave it out
    const int slow_len = s->seg_len[sseg] - 1;
    double bs = (double)m->embed.bytes(), bf = (double)m->fast_out.bytes();
    for (const Layer &L : m->layers) bs += (double)(L.wqkv.bytes() + L.wo.bytes() + L.w13.bytes() + L.w2.bytes());
    for (const Layer &L : m->fast_layers) bf += (double)(L.wqkv.bytes() + L.wo.bytes() + L.w13.bytes() + L.w2.bytes());
    bs += (double)s->n_past * hp.block_count * 2.0 * hp.head_count_kv * hp.head_dim * sizeof(__half);
    std::vector<cudaEvent_t> ev(4 * (size_t)reps, nullptr);
    for (auto &e : ev) CU(cudaEventCreate(&e));
    cudaError_t err = cudaSuccess;
    for (int r = 0; r < reps && err == cudaSuccess; ++r) {
        MegaCtl *cf = s->mega_ctl + fseg, *cs = s->mega_ctl + sseg;
        if ((err = cudaMemsetAsync(cf, 0, sizeof(MegaCtl), m->stream))) break;
        if ((err = cudaEventRecord(ev[4 * r], m->stream))) break;
        if ((err = launch_mega(s->mega_ops + s->seg_start[fseg], s->seg_len[fseg], s->seg_mt[fseg], cf, nullptr,
                               m->d_err, m->num_sms, m->stream, m->d_epoch, s->mega_q8)))
            break;
        if ((err = cudaEventRecord(ev[4 * r + 1], m->stream))) break;
        if ((err = cudaMemsetAsync(cs, 0, sizeof(MegaCtl), m->stream))) break;
        if ((err = cudaEventRecord(ev[4 * r + 2], m->stream))) break;
        if ((err = launch_mega(s->mega_ops + s->seg_start[sseg], slow_len, s->seg_mt[sseg], cs, nullptr, m->d_err,
                               m->num_sms, m->stream, m->d_epoch, s->mega_q8)))
            break;
        err = cudaEventRecord(ev[4 * r + 3], m->stream);
    }
    if (err == cudaSuccess) err = cudaStreamSynchronize(m->stream);
    double tf = 0, ts = 0;
    for (int r = 0; r < reps && err == cudaSuccess; ++r) {
        float a = 0, b = 0;
        cudaEventElapsedTime(&a, ev[4 * r], ev[4 * r + 1]);
        cudaEventElapsedTime(&b, ev[4 * r + 2], ev[4 * r + 3]);
        tf += a;
        ts += b;
    }
    for (auto &e : ev) cudaEventDestroy(e);
    CU(err);
    *ms_fast = tf / reps;
    *ms_slow = ts / reps;
    *bytes_fast = bf;
    *bytes_slow = bs;
    return check_err_word(m);
}

// Runs `reps` traced launches of one frame-program segment (the Slow step
// without its n_past advance) and returns the stamps of every launch,
// [rep][op][cta][kTraceSlots] (launch_mega's trace layout).
static s2k_status trace_segment(s2k_model *m, s2k_seq *s, int segment, int reps, std::vector<unsigned long long> &tr,
                                int *len_out, std::vector<int> *kinds) {
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    if (!s->frame_exec || s->frame_gen != m->ws_gen || !s->use_mega || s->seg_start.empty())
        return fail(S2K_ERR_STATE, "no persistent-kernel frame program for this sequence (run generate first)");
    const int nseg = (int)s->seg_start.size();
    if (segment < 0 || segment >= nseg) return fail(S2K_ERR_ARG, "segment %d outside 0..%d", segment, nseg - 1);
    if (s->n_past >= s->max_seq_len)
        return fail(S2K_ERR_KV_FULL, "profiling writes position n_past = %d; the sequence holds %d", s->n_past,
                    s->max_seq_len);
    // the Slow segment ends with the n_past advance: leave it out
    const int len = s->seg_len[segment] - (segment == nseg - 1 ? 1 : 0);
    if (kinds) {
        std::vector<MegaOp> hops((size_t)len);
        CU(cudaMemcpy(hops.data(), s->mega_ops + s->seg_start[segment], (size_t)len * sizeof(MegaOp),
                      cudaMemcpyDeviceToHost));
        kinds->resize((size_t)len);
        for (int i = 0; i < len; ++i) (*kinds)[(size_t)i] = hops[(size_t)i].kind;
    }
    const size_t per = (size_t)(len + 1) * m->num_sms * kTraceSlots;
    unsigned long long *d_tr = nullptr;
    CU(m->alloc(&d_tr, (size_t)reps * per));
    CU(cudaMemsetAsync(d_tr, 0, (size_t)reps * per * sizeof(unsigned long long), m->stream));
    MegaCtl *ctl = s->mega_ctl + segment;
    cudaError_t err = cudaSuccess;
    for (int r = 0; r < reps && err == cudaSuccess; ++r) {
        if ((err = cudaMemsetAsync(ctl, 0, sizeof(MegaCtl), m->stream))) break;
        err = launch_mega(s->mega_ops + s->seg_start[segment], len, s->seg_mt[segment], ctl, nullptr, m->d_err,
                          m->num_sms, m->stream, m->d_epoch, s->mega_q8, d_tr + (size_t)r * per);
    }
    tr.assign((size_t)reps * per, 0ull);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(tr.data(), d_tr, tr.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                              m->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(m->stream);
    m->release(d_tr);
    CU(err);
    *len_out = len;
    return check_err_word(m);
}

S2K_API s2k_status s2k_profile_ops(s2k_model *m, s2k_seq *s, int32_t segment, int32_t reps, double *op_us,
                                   int32_t *op_kind, int32_t cap, int32_t *n_ops) {
    if (!m || !s || reps <= 0 || reps > 64 || !op_us || !op_kind || cap <= 0 || !n_ops)
        return fail(S2K_ERR_ARG, "bad argument (1 <= reps <= 64)");
    std::vector<unsigned long long> tr;
    std::vector<int> kinds;
    int len = 0;
    s2k_status rc = trace_segment(m, s, segment, reps, tr, &len, &kinds);
    if (rc) return rc;
    if (len > cap) return fail(S2K_ERR_ARG, "segment %d has %d ops, capacity %d", segment, len, cap);
    const size_t G = (size_t)m->num_sms, per = (size_t)(len + 1) * G * kTraceSlots;
    for (int i = 0; i < len; ++i) {
        double t = 0;
        for (int r = 0; r < reps; ++r) {
            const unsigned long long *b = tr.data() + (size_t)r * per;
            t += (double)(b[(size_t)(i + 1) * G * kTraceSlots] - b[(size_t)i * G * kTraceSlots]);  // CTA 0 starts
        }
        op_us[i] = t / reps / 1e3;
        op_kind[i] = kinds[(size_t)i];
    }
    *n_ops = len;
    return S2K_OK;
}

S2K_API s2k_status s2k_profile_trace(s2k_model *m, s2k_seq *s, int32_t segment, uint64_t *stamps, size_t cap,
                                     int32_t *n_ops, int32_t *n_ctas) {
    if (!m || !s || !stamps || !n_ops || !n_ctas) return fail(S2K_ERR_ARG, "NULL argument");
    std::vector<unsigned long long> tr;
    int len = 0;
    s2k_status rc = trace_segment(m, s, segment, 2, tr, &len, nullptr);  // the first launch warms up
    if (rc) return rc;
    const size_t per = tr.size() / 2;
    if (per > cap) return fail(S2K_ERR_ARG, "trace needs %zu entries, capacity %zu", per, cap);
    memcpy(stamps, tr.data() + per, per * sizeof(uint64_t));
    *n_ops = len;
    *n_ctas = m->num_sms;
    return S2K_OK;
}

S2K_API s2k_status s2k_debug_copy(s2k_model *m, s2k_seq *s, const char *name, void *host, size_t nbytes,
                                  size_t *copied) {
    if (!m || !name || !host || !copied) return fail(S2K_ERR_ARG, "NULL argument");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_hparams &hp = m->hp;
    const void *src = nullptr;
    size_t bytes = 0;
    const Work &w = m->sw, &f = m->fw;
    const std::string n(name);
    auto pick = [&](const void *p, size_t b) { src = p; bytes = b; };
    if (n == "x") pick(w.x, (size_t)w.T * w.dim * 4);
    else if (n == "h") pick(w.h, (size_t)w.T * w.dim * 4);
    else if (n == "qkv") pick(w.qkv, (size_t)w.T * (w.qs + 2 * w.kvs) * 4);
    else if (n == "attn") pick(w.attn, (size_t)w.T * w.qs * 4);
    else if (n == "ff") pick(w.ff_buf, (size_t)w.T * w.ff * 4);
    else if (n == "kcur") pick(w.kcur, (size_t)w.T * w.kvs * 4);
    else if (n == "vcur") pick(w.vcur, (size_t)w.T * w.kvs * 4);
    else if (n == "logits") pick(m->logits, (size_t)hp.vocab_size * 4);
    else if (n == "hidden") pick(m->hidden, (size_t)hp.embedding_length * 4);
    else if (n == "fx") pick(f.x, (size_t)f.T * f.dim * 4);
    else if (n == "fh") pick(f.h, (size_t)f.T * f.dim * 4);
    else if (n == "fqkv") pick(f.qkv, (size_t)f.T * (f.qs + 2 * f.kvs) * 4);
    else if (n == "fattn") pick(f.attn, (size_t)f.T * f.qs * 4);
    else if (n == "fff") pick(f.ff_buf, (size_t)f.T * f.ff * 4);
    else if (n == "flogits") pick(m->flogits, (size_t)hp.codebook_size * 4);
    else if ((n == "kv_k" || n == "kv_v") && s) {
        const size_t page_elems = (size_t)hp.block_count * hp.head_count_kv * kPage * hp.head_dim;
        pick(n == "kv_k" ? (const void *)s->k : (const void *)s->v, page_elems * s->n_pages * 2);
    } else {
        return fail(S2K_ERR_ARG, "unknown buffer '%s'", name);
    }
    if (!src) return fail(S2K_ERR_STATE, "buffer '%s' not allocated", name);
    const size_t nb = std::min(nbytes, bytes);
    CU(cudaStreamSynchronize(m->stream));
    CU(cudaMemcpy(host, src, nb, cudaMemcpyDeviceToHost));
    *copied = nb;
    return S2K_OK;
}


// ---------------------------------------------------------------------------
// KV restore, get_rows, and the failure-injection / bounded-wait hooks
// ---------------------------------------------------------------------------
S2K_API s2k_status s2k_seq_load_kv(s2k_seq *s, const uint16_t *k, const uint16_t *v, int32_t n_pos) {
    if (!s || !k || !v || n_pos < 0) return fail(S2K_ERR_ARG, "bad argument");
    if (s->pooled) return fail(S2K_ERR_ARG, "sequence belongs to a scheduler's page pool");
    if (n_pos > s->max_seq_len) return fail(S2K_ERR_KV_FULL, "%d positions, the sequence holds %d", n_pos, s->max_seq_len);
    s2k_model *m = s->m;
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const s2k_hparams &hp = m->hp;
    const int L = hp.block_count, Hkv = hp.head_count_kv, hd = hp.head_dim;
    const size_t kvs = (size_t)Hkv * hd;
    const size_t page_elems = (size_t)L * Hkv * kPage * hd;
    const int np = (n_pos + kPage - 1) / kPage;
    if (np > 0) {
        // [layer][pos][kv_head][hd] -> pages [page][layer][kv_head][slot][hd]; the
        // sequence's own block table is the identity (s2k_seq_create)
        std::vector<uint16_t> pk((size_t)np * page_elems, 0), pv((size_t)np * page_elems, 0);
        for (int l = 0; l < L; ++l)
            for (int pos = 0; pos < n_pos; ++pos) {
                const int pg = pos / kPage, slot = pos % kPage;
                for (int g = 0; g < Hkv; ++g) {
                    const size_t src = ((size_t)l * n_pos + pos) * kvs + (size_t)g * hd;
                    const size_t dst = ((((size_t)pg * L + l) * Hkv + g) * kPage + slot) * hd;
                    memcpy(&pk[dst], k + src, (size_t)hd * 2);
                    memcpy(&pv[dst], v + src, (size_t)hd * 2);
                }
            }
        CU(cudaMemcpy(s->k, pk.data(), pk.size() * 2, cudaMemcpyHostToDevice));
        CU(cudaMemcpy(s->v, pv.data(), pv.size() * 2, cudaMemcpyHostToDevice));
    }
    CU(cudaStreamSynchronize(m->stream));
    CU(cudaMemsetAsync(&s->dev->state, 0, sizeof(SeqState), m->stream));
    CU(cudaMemcpyAsync(&s->dev->state.n_past, &n_pos, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    s->n_past = n_pos;
    return S2K_OK;
}

S2K_API s2k_status s2k_get_rows(s2k_model *m, const char *table, const int32_t *ids, int32_t n, float *out) {
    if (!m || !table || !ids || !out || n <= 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    const std::string t(table);
    const DevMat *E = t == "embeddings.weight" ? &m->embed
                      : t == "codebook_embeddings.weight" ? &m->cb_embed
                      : t == "fast_embeddings.weight" ? &m->fast_embed
                      : t == "fast_output.weight" ? &m->fast_out
                                                   : nullptr;
    if (!E || !E->w) return fail(S2K_ERR_ARG, "no table '%s'", table);
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= E->rows) return fail(S2K_ERR_ARG, "row %d out of range (%d rows)", ids[i], E->rows);
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    int *d_ids = nullptr;
    float *d_out = nullptr;
    CU(m->alloc(&d_ids, (size_t)n));
    if (m->alloc(&d_out, (size_t)n * E->cols) != cudaSuccess) {
        m->release(d_ids);
        return fail(S2K_ERR_OOM, "get_rows output");
    }
    cudaError_t e = cudaMemcpyAsync(d_ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = launch_gather_rows(E, d_ids, n, d_out, m->d_err, m->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(out, d_out, (size_t)n * E->cols * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    m->release(d_ids);
    m->release(d_out);
    CU(e);
    return check_err_word(m);
}

S2K_API s2k_status s2k_model_set_wait_limit(s2k_model *m, int64_t cycles) {
    if (!m || cycles < 0) return fail(S2K_ERR_ARG, "bad argument");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    const long long c = cycles;
    CU(cudaStreamSynchronize(m->stream));
    CU(cudaMemcpy(m->d_err + 2, &c, sizeof(c), cudaMemcpyHostToDevice));
    return S2K_OK;
}

S2K_API s2k_status s2k_debug_wait_probe(s2k_model *m) {
    if (!m) return fail(S2K_ERR_ARG, "NULL model");
    if (!m->finalized || !m->sw.lx) return fail(S2K_ERR_STATE, "model not finalized");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    CU(launch_wait_probe(m->sw.lx, m->d_err, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return check_err_word(m);
}

S2K_API s2k_status s2k_debug_det_expf(int32_t device, const float *x, float *y, int64_t n) {
    if (n < 0 || (n > 0 && (!x || !y))) return fail(S2K_ERR_ARG, "bad argument");
    if (n == 0) return S2K_OK;
    if (cuda_set(device)) return fail(S2K_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    float *d = nullptr;
    CU(cudaMalloc(&d, (size_t)n * 2 * sizeof(float)));
    cudaError_t e = cudaMemcpy(d, x, (size_t)n * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_det_expf(d, d + n, n, 0);
    if (e == cudaSuccess) e = cudaMemcpy(y, d + n, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(d);
    CU(e);
    return S2K_OK;
}

S2K_API s2k_status s2k_debug_fail_alloc(s2k_model *m, int64_t after) {
    if (!m) return fail(S2K_ERR_ARG, "NULL model");
    m->fail_alloc_at = after < 0 ? -1 : after;
    return S2K_OK;
}

S2K_API size_t s2k_model_device_bytes(const s2k_model *m) { return m ? m->dev_bytes : 0; }

S2K_API s2k_status s2k_device_mem_info(int32_t device, size_t *free_bytes, size_t *total_bytes) {
    if (!free_bytes || !total_bytes) return fail(S2K_ERR_ARG, "NULL argument");
    if (cuda_set(device)) return fail(S2K_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    CU(cudaMemGetInfo(free_bytes, total_bytes));
    return S2K_OK;
}

S2K_API s2k_status s2k_seq_last_metrics(const s2k_seq *s, s2k_gen_metrics *out) {
    if (!s || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = s->metrics;
    return S2K_OK;
}
