// s2k_batch.cu -- continuous batching over independent utterances: batched
// frames (every live sequence's Fast-AR passes and Slow step as one set of
// kernels, weights streamed once per frame for the whole batch) and a host
// scheduler that admits, prefills and retires requests between frames over a
// shared paged f16 KV pool.
//
// The reference runs one synthesis at a time (src/s2_pipeline.cpp:781,810,
// src/s2_server.cpp:715); batching changes no arithmetic.  A batched row
// computes exactly what the single-sequence frame computes for that sequence
// (same kernels' arithmetic, same counter-based sampling draws keyed by
// (seed, frame, stream, seq_id)), so every request's codes equal those of
// s2k_generate on the same prompt and parameters.
//
// Frame of n sequences (src/s2_generate.cpp:123-182 per sequence):
//   Fast-AR pass p = 0 .. ncb-2: rows [hidden_b ; fast_emb[c_b0]] (p = 0) or
//     fast_emb[c_bp]; 4 layers over BatchRow descriptors (positions 0..9 of
//     each sequence's own f32 K/V rows); fast_norm + fast_output on each
//     sequence's last row; per-sequence sampling of codebook p+1
//   commit the frame (codes, step input)
//   Slow step: n rows (one per sequence, at its own n_past, attending to its
//     own KV pages); final norm + tied LM head; n_past += 1; main-token
//     sampling (semantic mask, stop, RAS) and the hidden state per sequence.
// GEMMs with >= 8 rows run on the tensor cores (s2k_prefill.cu), smaller ones
// on the tile GEMV.  One CUDA graph per batch size n.
#include "s2k_model.h"

#include <algorithm>
#include <cstring>
#include <deque>
#include <map>
#include <vector>

namespace s2k {

struct BatchGraph {
    cudaGraphExec_t exec = nullptr;
    size_t nodes = 0;
};

struct BatchState {
    int cap = 0;  // sequences per frame
    int L = 0;    // longest key range of a Slow row (positions)
    int S = 0;    // Fast-AR positions per frame (num_codebooks)
    Work slow, fast;
    std::vector<float *> fk, fv;  // Fast-AR K/V rows per layer [cap * S][Hkv][hd]
    float *logits = nullptr, *hidden = nullptr, *flogits = nullptr;
    SeqDev **seqs = nullptr;         // device [cap]
    SeqDev **seqs_host = nullptr;    // pinned staging of the same
    BatchRow *rows_slow = nullptr;   // [cap]
    BatchRow *rows_fast = nullptr;   // pass 0 [2 cap], then pass p [cap] for p = 1 .. S-2
    std::map<int, BatchGraph> graphs;
};

static void batch_release(s2k_model *m) {
    BatchState *b = m->batch;
    if (!b) return;
    for (auto &kv : b->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    b->graphs.clear();
    work_free(m, b->slow);
    work_free(m, b->fast);
    for (float *p : b->fk) m->release(p);
    for (float *p : b->fv) m->release(p);
    for (void *p : {(void *)b->logits, (void *)b->hidden, (void *)b->flogits, (void *)b->seqs, (void *)b->rows_slow,
                    (void *)b->rows_fast})
        m->release(p);
    if (b->seqs_host) cudaFreeHost(b->seqs_host);
    delete b;
    m->batch = nullptr;
}

// Buffers for frames of up to cap sequences whose Slow rows attend over at
// most L positions.
static s2k_status ensure_batch(s2k_model *m, int cap, int L) {
    if (m->batch && m->batch->cap >= cap && m->batch->L >= L) return S2K_OK;
    if (m->batch) {
        cap = std::max(cap, m->batch->cap);
        L = std::max(L, m->batch->L);
    }
    CU(cudaStreamSynchronize(m->stream));
    batch_release(m);
    const s2k_hparams &hp = m->hp;
    BatchState *b = new BatchState();
    m->batch = b;
    b->cap = cap;
    b->L = L;
    b->S = std::max(hp.num_codebooks, 2);
    const int S = b->S;
    CU(work_alloc(m, b->slow, cap, L, hp.embedding_length, hp.head_count, hp.head_count_kv, hp.head_dim,
                  hp.feed_forward_length, hp.block_count, true, cap));
    CU(m->alloc(&b->logits, (size_t)cap * hp.vocab_size));
    CU(m->alloc(&b->hidden, (size_t)cap * hp.embedding_length));
    CU(m->alloc(&b->seqs, (size_t)cap));
    CU(cudaHostAlloc((void **)&b->seqs_host, (size_t)cap * sizeof(SeqDev *), cudaHostAllocDefault));
    std::vector<BatchRow> rs(cap);
    for (int i = 0; i < cap; ++i) rs[i] = BatchRow{i, 0, i, i};
    CU(m->alloc(&b->rows_slow, (size_t)cap));
    CU(cudaMemcpy(b->rows_slow, rs.data(), rs.size() * sizeof(BatchRow), cudaMemcpyHostToDevice));
    if (hp.has_fast_decoder) {
        CU(work_alloc(m, b->fast, 2 * cap, S, hp.fast_embedding_length, hp.fast_head_count, hp.fast_head_count_kv,
                      hp.fast_head_dim, hp.fast_feed_forward_length, hp.fast_block_count, true, 2 * cap));
        const size_t fkvs = (size_t)hp.fast_head_count_kv * hp.fast_head_dim;
        b->fk.assign(hp.fast_block_count, nullptr);
        b->fv.assign(hp.fast_block_count, nullptr);
        for (int i = 0; i < hp.fast_block_count; ++i) {
            CU(m->alloc(&b->fk[i], (size_t)cap * S * fkvs));
            CU(m->alloc(&b->fv[i], (size_t)cap * S * fkvs));
        }
        CU(m->alloc(&b->flogits, (size_t)cap * hp.codebook_size));
        // Fast rows: sequence i holds K/V rows [i*S, i*S + S); position 0 is
        // the hidden state, position p + 1 codebook p's embedding.
        std::vector<BatchRow> rf((size_t)2 * cap + (size_t)std::max(S - 2, 0) * cap);
        for (int i = 0; i < cap; ++i) {
            rf[2 * i] = BatchRow{i, 0, i * S, i * S};
            rf[2 * i + 1] = BatchRow{i, 1, i * S, i * S + 1};
        }
        for (int p = 1; p <= S - 2; ++p)
            for (int i = 0; i < cap; ++i)
                rf[(size_t)2 * cap + (size_t)(p - 1) * cap + i] = BatchRow{i, p + 1, i * S, i * S + p + 1};
        CU(m->alloc(&b->rows_fast, rf.size()));
        CU(cudaMemcpy(b->rows_fast, rf.data(), rf.size() * sizeof(BatchRow), cudaMemcpyHostToDevice));
    }
    return S2K_OK;
}

// All device work of one batched frame over the n sequences in b->seqs.
static cudaError_t enqueue_batch_frame(s2k_model *m, int n) {
    const s2k_hparams &hp = m->hp;
    BatchState *b = m->batch;
    cudaStream_t st = m->stream;
    cudaError_t e;
    const int dim = hp.embedding_length;
    for (int p = 0; p + 1 < hp.num_codebooks; ++p) {
        const int fdim = hp.fast_embedding_length;
        if ((e = launch_embed_fast_batch(&m->fast_embed, b->seqs, n, p, b->fast.x, fdim, m->d_err, st))) return e;
        StackCall c;
        c.fast = true;
        c.T = p == 0 ? 2 * n : n;
        c.rows = p == 0 ? b->rows_fast : b->rows_fast + (size_t)2 * b->cap + (size_t)(p - 1) * b->cap;
        c.w = &b->fast;
        c.fk = b->fk.data();
        c.fv = b->fv.data();
        c.max_keys = b->S;
        c.mma = true;
        if ((e = run_stack(m, c))) return e;
        GemvArgs hd;
        hd.w = &m->fast_out;
        hd.x = b->fast.x + (p == 0 ? fdim : 0);
        hd.ldx = (p == 0 ? 2 : 1) * fdim;
        hd.M = n;
        hd.in_mode = IN_RMSNORM;
        hd.norm_w = m->fast_norm;
        hd.eps = hp.fast_rms_norm_eps;
        hd.y = b->flogits;
        hd.ldy = hp.codebook_size;
        hd.err = m->d_err;
        if ((e = stack_gemm(m, b->fast, hd, true))) return e;
        if ((e = launch_sample_fast_batch(b->flogits, hp.codebook_size, b->seqs, n, p + 1, m->d_err, st))) return e;
    }
    if ((e = launch_frame_commit_batch(b->seqs, n, st))) return e;
    EmbedArgs ea;
    ea.tok_emb = &m->embed;
    ea.cb_emb = &m->cb_embed;
    ea.seqs = b->seqs;
    ea.T = n;
    ea.ncb = hp.num_codebooks;
    ea.cb_size = hp.codebook_size;
    ea.sem_begin = hp.semantic_begin_id;
    ea.sem_end = hp.semantic_end_id;
    ea.scale_cb = hp.scale_codebook_embeddings;
    ea.sem_scale = 1.0f / sqrtf((float)(hp.num_codebooks + 1));
    ea.x = b->slow.x;
    ea.err = m->d_err;
    if ((e = launch_embed_slow(ea, st))) return e;
    StackCall c;
    c.fast = false;
    c.T = n;
    c.rows = b->rows_slow;
    c.seqs = b->seqs;
    c.w = &b->slow;
    c.max_keys = b->L;
    c.mma = true;
    if ((e = run_stack(m, c))) return e;
    GemvArgs hd;
    hd.w = &m->embed;
    hd.x = b->slow.x;
    hd.ldx = dim;
    hd.M = n;
    hd.in_mode = IN_RMSNORM;
    hd.norm_w = m->norm;
    hd.eps = hp.rms_norm_eps;
    hd.y = b->logits;
    hd.ldy = hp.vocab_size;
    hd.act_out = b->hidden;
    hd.err = m->d_err;
    if ((e = stack_gemm(m, b->slow, hd, true))) return e;
    if ((e = launch_advance_batch(b->seqs, n, 1, st))) return e;
    return launch_sample_main_batch(b->logits, hp.vocab_size, b->seqs, n, b->hidden, dim, m->d_err, st);
}

static s2k_status batch_graph(s2k_model *m, int n, BatchGraph **out) {
    BatchState *b = m->batch;
    auto it = b->graphs.find(n);
    if (it != b->graphs.end()) {
        *out = &it->second;
        return S2K_OK;
    }
    cudaGraph_t g = nullptr;
    const unsigned long long before = s2k_launch_count(0);
    CU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_batch_frame(m, n);
    cudaError_t e2 = cudaStreamEndCapture(m->stream, &g);
    const unsigned long long after = s2k_launch_count(0);
    count_launch(-(int)(after - before));
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return fail(S2K_ERR_CUDA, "batched frame capture failed: %s / %s", cudaGetErrorString(e),
                    cudaGetErrorString(e2));
    }
    BatchGraph bg;
    cudaGraphGetNodes(g, nullptr, &bg.nodes);
    e = cudaGraphInstantiate(&bg.exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(S2K_ERR_CUDA, "batched frame graph instantiate: %s", cudaGetErrorString(e));
    *out = &(b->graphs[n] = bg);
    return S2K_OK;
}

// Prompt prefill and first main token of one sequence (generate():
// src/s2_generate.cpp:51-60), leaving it ready for batched frames.
// d_prompt_tm: token-major [cols][ncb+1] in device memory; d_codes:
// [ncb][codes_ld] frame codes.
static s2k_status seq_begin_core(s2k_model *m, s2k_seq *s, const int32_t *d_prompt_tm, int cols,
                                 const s2k_gen_params *gp, int *d_codes, int codes_ld) {
    const s2k_hparams &hp = m->hp;
    if (cols <= 0 || gp->max_new_tokens < 0) return fail(S2K_ERR_ARG, "bad prompt length / max_new_tokens");
    // one position of slack: a sequence that stops while others run may see
    // one more Slow step before it leaves the batch
    if (cols + gp->max_new_tokens + 1 > s->max_seq_len)
        return fail(S2K_ERR_KV_FULL, "sequence holds %d positions, need %d", s->max_seq_len,
                    cols + gp->max_new_tokens + 1);
    if (!hp.has_fast_decoder && hp.num_codebooks > 1) return fail(S2K_ERR_STATE, "model has no fast decoder");
    if (hp.num_codebooks < 2) return fail(S2K_ERR_STATE, "batched frames need num_codebooks >= 2");
    s2k_status rc = ensure_slow_work(m, cols, s->max_seq_len);
    if (rc) return rc;
    SampleCfg c;
    fill_sample_cfg(m, gp, d_codes, codes_ld, &c);
    CU(cudaMemsetAsync(&s->dev->state, 0, sizeof(SeqState), m->stream));
    CU(cudaMemcpyAsync(&s->dev->cfg, &c, sizeof(SampleCfg), cudaMemcpyHostToDevice, m->stream));
    HostStatus *hs = s->hstat_dev;
    CU(cudaMemcpyAsync(&s->dev->host, &hs, sizeof(HostStatus *), cudaMemcpyHostToDevice, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    s->hstat->n_frames = 0;
    s->hstat->done = 0;
    s->n_past = 0;
    CU(enqueue_slow(m, s, cols, d_prompt_tm, nullptr));
    CU(launch_sample_main(m->logits, s->dev, m->d_err, m->stream));
    CU(cudaMemcpyAsync(s->hidden, m->hidden, (size_t)hp.embedding_length * sizeof(float), cudaMemcpyDeviceToDevice,
                       m->stream));
    s->n_past = cols;
    return S2K_OK;
}

// One batched frame over n begun, unfinished sequences of model m.
static s2k_status batch_frame_core(s2k_model *m, s2k_seq *const *seqs, int n) {
    int L = 0;
    for (int i = 0; i < n; ++i) L = std::max(L, seqs[i]->max_seq_len);
    s2k_status rc = ensure_batch(m, n, L);
    if (rc) return rc;
    BatchState *b = m->batch;
    BatchGraph *g = nullptr;
    rc = batch_graph(m, n, &g);
    if (rc) return rc;
    for (int i = 0; i < n; ++i) b->seqs_host[i] = seqs[i]->dev;
    CU(cudaMemcpyAsync(b->seqs, b->seqs_host, (size_t)n * sizeof(SeqDev *), cudaMemcpyHostToDevice, m->stream));
    CU(cudaGraphLaunch(g->exec, m->stream));
    count_launch((int)g->nodes);
    CU(cudaStreamSynchronize(m->stream));
    rc = check_err_word(m);
    if (rc) return rc;
    for (int i = 0; i < n; ++i) seqs[i]->n_past++;  // every row's Slow step advanced its sequence
    return S2K_OK;
}

static s2k_status upload_prompt(s2k_model *m, s2k_seq *s, const int32_t *prompt, int cols) {
    const int rows = m->hp.num_codebooks + 1;
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
    CU(cudaMemcpy(s->prompt, tm.data(), tm.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
    return S2K_OK;
}

static s2k_status ensure_codes(s2k_model *m, s2k_seq *s, int frames) {
    const int ld = std::max(frames, 1);
    if (s->codes_cap >= ld) return S2K_OK;
    m->release(s->codes);
    s->codes = nullptr;
    CU(m->alloc(&s->codes, (size_t)std::max(m->hp.num_codebooks, 1) * ld));
    s->codes_cap = ld;
    return S2K_OK;
}

// Frame codes of a sequence so far, compacted cb-major [ncb][n_frames].
static s2k_status seq_codes(s2k_model *m, s2k_seq *s, int32_t *codes_out, int cap, int *n_frames) {
    const int ncb = std::max(m->hp.num_codebooks, 1);
    const int nf = s->hstat->n_frames;
    *n_frames = nf;
    if (!codes_out || nf == 0) return S2K_OK;
    if (cap < nf) return fail(S2K_ERR_ARG, "codes capacity %d < %d frames", cap, nf);
    for (int cb = 0; cb < ncb; ++cb)
        CU(cudaMemcpyAsync(codes_out + (size_t)cb * nf, s->codes + (size_t)cb * s->codes_cap, (size_t)nf * sizeof(int32_t),
                           cudaMemcpyDeviceToHost, m->stream));
    CU(cudaStreamSynchronize(m->stream));
    return S2K_OK;
}

}  // namespace s2k

void batch_free(s2k_model *m) { s2k::batch_release(m); }

// ---------------------------------------------------------------------------
// low-level batched frames
// ---------------------------------------------------------------------------
S2K_API s2k_status s2k_seq_begin(s2k_model *m, s2k_seq *s, const int32_t *prompt, int32_t cols,
                                 const s2k_gen_params *gp) {
    if (!m || !s || !prompt || !gp || cols <= 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (s->m != m) return fail(S2K_ERR_ARG, "sequence belongs to another model");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    s2k_status rc = upload_prompt(m, s, prompt, cols);
    if (!rc) rc = ensure_codes(m, s, gp->max_new_tokens);
    if (!rc) rc = seq_begin_core(m, s, s->prompt, cols, gp, s->codes, s->codes_cap);
    if (!rc) {
        CU(cudaStreamSynchronize(m->stream));
        rc = check_err_word(m);
    }
    return rc;
}

S2K_API s2k_status s2k_batch_frame(s2k_model *m, s2k_seq *const *seqs, int32_t n, int32_t *n_live) {
    if (!m || (n > 0 && !seqs) || n < 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    std::vector<s2k_seq *> live;
    for (int i = 0; i < n; ++i) {
        if (!seqs[i] || seqs[i]->m != m) return fail(S2K_ERR_ARG, "sequence %d is NULL or belongs to another model", i);
        if (!seqs[i]->hstat->done) live.push_back(seqs[i]);
    }
    for (size_t i = 0; i < live.size(); ++i)
        for (size_t j = i + 1; j < live.size(); ++j)
            if (live[i] == live[j]) return fail(S2K_ERR_ARG, "sequence listed twice");
    s2k_status rc = live.empty() ? S2K_OK : batch_frame_core(m, live.data(), (int)live.size());
    if (rc) return rc;
    if (n_live) {
        int k = 0;
        for (s2k_seq *s : live) k += !s->hstat->done;
        *n_live = k;
    }
    return S2K_OK;
}

S2K_API s2k_status s2k_seq_frames(s2k_seq *s, int32_t *codes_out, int32_t cap_frames, int32_t *n_frames,
                                  int32_t *done) {
    if (!s || !n_frames) return fail(S2K_ERR_ARG, "bad argument");
    if (cuda_set(s->m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    int nf = 0;
    s2k_status rc = seq_codes(s->m, s, codes_out, cap_frames, &nf);
    if (rc) return rc;
    *n_frames = nf;
    if (done) *done = s->hstat->done;
    return S2K_OK;
}

// ---------------------------------------------------------------------------
// scheduler
// ---------------------------------------------------------------------------
namespace {

struct Req {
    std::vector<int32_t> prompt_tm;  // token-major [cols][ncb+1]
    int cols = 0;
    s2k_gen_params gp{};
    int state = S2K_REQ_WAITING;
    s2k_status status = S2K_OK;  // why a failed request failed
    int slot = -1;
    int delivered = 0;  // frames handed to the frame callback
    std::vector<int32_t> codes;  // [ncb][n_frames] once finished
    int n_frames = 0;
};

struct Slot {
    s2k_seq *seq = nullptr;
    int req = -1;
    std::vector<int> pages;
};

}  // namespace

struct s2k_sched {
    s2k_model *m = nullptr;
    int max_batch = 0, max_seq_len = 0, pool_pages = 0, max_pages = 0;
    __half *k = nullptr, *v = nullptr;  // page pool [pool_pages][layer][kv_head][16][head_dim]
    std::vector<int> free_pages;
    std::vector<Slot> slots;
    std::vector<Req> reqs;
    std::deque<int> waiting;
    int32_t *prompt_dev = nullptr;
    size_t prompt_cap = 0;
    s2k_sched_stats stats{};
    s2k_sched_frame_callback on_frame = nullptr;
    void *on_frame_user = nullptr;
};

static void sched_release(s2k_sched *sc) {
    if (!sc) return;
    s2k_model *m = sc->m;
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    for (Slot &sl : sc->slots)
        if (sl.seq) s2k_seq_free(sl.seq);
    m->release(sc->k);
    m->release(sc->v);
    m->release(sc->prompt_dev);
    delete sc;
}

S2K_API void s2k_sched_free(s2k_sched *sc) { sched_release(sc); }

S2K_API s2k_status s2k_sched_create(s2k_model *m, int32_t max_batch, int32_t max_seq_len, int32_t pool_pages,
                                    s2k_sched **out) {
    if (!m || !out || max_batch <= 0 || max_seq_len <= 0 || pool_pages < 0) return fail(S2K_ERR_ARG, "bad argument");
    if (!m->finalized) return fail(S2K_ERR_STATE, "model not finalized");
    const s2k_hparams &hp = m->hp;
    if (hp.num_codebooks < 2 || !hp.has_fast_decoder) return fail(S2K_ERR_STATE, "batched frames need the Fast-AR decoder");
    if (max_seq_len > m->rope_slow_n)
        return fail(S2K_ERR_ARG, "max_seq_len %d exceeds context_length %d", max_seq_len, m->rope_slow_n);
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    *out = nullptr;
    s2k_sched *sc = new s2k_sched();
    sc->m = m;
    sc->max_batch = max_batch;
    sc->max_seq_len = max_seq_len;
    sc->max_pages = (max_seq_len + kPage - 1) / kPage;
    sc->pool_pages = pool_pages > 0 ? pool_pages : max_batch * sc->max_pages;
    const size_t page_elems = (size_t)hp.block_count * hp.head_count_kv * kPage * hp.head_dim;
    auto bail = [&](s2k_status code, const char *what) {
        std::string msg = std::string("s2k_sched_create: ") + what + ": " + s2k_last_error();
        sched_release(sc);
        return fail(code, "%s", msg.c_str());
    };
    if (m->alloc(&sc->k, page_elems * sc->pool_pages) || m->alloc(&sc->v, page_elems * sc->pool_pages))
        return bail(S2K_ERR_OOM, "KV page pool");
    sc->free_pages.resize(sc->pool_pages);
    for (int i = 0; i < sc->pool_pages; ++i) sc->free_pages[i] = sc->pool_pages - 1 - i;
    sc->slots.resize(max_batch);
    for (int i = 0; i < max_batch; ++i) {
        // a sequence whose pages come from the pool: its own block table, the
        // pool's K / V storage
        s2k_seq *s = new s2k_seq();
        s->m = m;
        s->pooled = true;
        s->k = sc->k;
        s->v = sc->v;
        s->max_seq_len = 0;
        s->n_pages = 0;
        sc->slots[i].seq = s;
        if (m->alloc(&s->block_table, (size_t)sc->max_pages) || m->alloc(&s->hidden, (size_t)hp.embedding_length) ||
            m->alloc(&s->dev, 1) || cudaMemset(s->dev, 0, sizeof(SeqDev)) != cudaSuccess)
            return bail(S2K_ERR_OOM, "sequence slots");
        if (cudaHostAlloc((void **)&s->hstat, sizeof(HostStatus), cudaHostAllocMapped) != cudaSuccess ||
            cudaHostGetDevicePointer((void **)&s->hstat_dev, (void *)s->hstat, 0) != cudaSuccess)
            return bail(S2K_ERR_OOM, "host status");
        memset((void *)s->hstat, 0, sizeof(HostStatus));
    }
    s2k_status rc = ensure_batch(m, max_batch, sc->max_pages * kPage);
    if (rc) return bail(rc, "batch buffers");
    *out = sc;
    return S2K_OK;
}

S2K_API s2k_status s2k_sched_submit(s2k_sched *sc, const int32_t *prompt, int32_t cols, const s2k_gen_params *gp,
                                    int32_t *req_id) {
    if (!sc || !prompt || !gp || cols <= 0 || gp->max_new_tokens < 0) return fail(S2K_ERR_ARG, "bad argument");
    s2k_model *m = sc->m;
    const int rows = m->hp.num_codebooks + 1;
    if (cols + gp->max_new_tokens + 1 > sc->max_seq_len)
        return fail(S2K_ERR_KV_FULL, "request needs %d positions, the scheduler's sequences hold %d",
                    cols + gp->max_new_tokens + 1, sc->max_seq_len);
    const int pages = (cols + gp->max_new_tokens + 1 + kPage - 1) / kPage;
    if (pages > sc->pool_pages) return fail(S2K_ERR_KV_FULL, "request needs %d pages, the pool has %d", pages, sc->pool_pages);
    Req r;
    r.cols = cols;
    r.gp = *gp;
    r.prompt_tm.resize((size_t)rows * cols);
    for (int q = 0; q < rows; ++q)
        for (int c = 0; c < cols; ++c) r.prompt_tm[(size_t)c * rows + q] = prompt[(size_t)q * cols + c];
    s2k_status rc = check_tokens_host(m, r.prompt_tm.data(), cols);
    if (rc) return rc;
    sc->reqs.push_back(std::move(r));
    const int id = (int)sc->reqs.size() - 1;
    sc->waiting.push_back(id);
    if (req_id) *req_id = id;
    return S2K_OK;
}

// Retire the request in slot i: copy its codes out, return its pages.
static s2k_status sched_retire(s2k_sched *sc, int i, int final_state = S2K_REQ_DONE) {
    s2k_model *m = sc->m;
    Slot &sl = sc->slots[i];
    Req &r = sc->reqs[sl.req];
    const int ncb = m->hp.num_codebooks;
    int nf = 0;
    const int nf0 = sl.seq->hstat->n_frames;
    r.codes.assign((size_t)ncb * std::max(nf0, 0), 0);
    s2k_status rc = seq_codes(m, sl.seq, r.codes.data(), (int)(r.codes.size() / std::max(ncb, 1)), &nf);
    if (rc) return rc;
    r.n_frames = nf;
    r.state = final_state;
    r.slot = -1;
    if (final_state == S2K_REQ_DONE) sc->stats.finished++;
    else sc->stats.cancelled++;
    for (int p : sl.pages) sc->free_pages.push_back(p);
    sl.pages.clear();
    sl.req = -1;
    return S2K_OK;
}

// Map request r's pages into sequence s, prefill its prompt and sample its
// first main token.
static s2k_status admit_one(s2k_sched *sc, Req &r, s2k_seq *s, const std::vector<int> &pages) {
    s2k_model *m = sc->m;
    const int need = (int)pages.size();
    CU(cudaMemcpy(s->block_table, pages.data(), (size_t)need * sizeof(int), cudaMemcpyHostToDevice));
    s->n_pages = need;
    s->max_seq_len = need * kPage;
    s2k_status rc = seq_publish(s);
    if (rc) return rc;
    rc = ensure_codes(m, s, r.gp.max_new_tokens);
    if (rc) return rc;
    const size_t ptoks = r.prompt_tm.size();
    if (sc->prompt_cap < ptoks) {
        m->release(sc->prompt_dev);
        sc->prompt_dev = nullptr;
        sc->prompt_cap = 0;
        CU(m->alloc(&sc->prompt_dev, ptoks));
        sc->prompt_cap = ptoks;
    }
    CU(cudaMemcpyAsync(sc->prompt_dev, r.prompt_tm.data(), ptoks * sizeof(int32_t), cudaMemcpyHostToDevice,
                       m->stream));
    rc = seq_begin_core(m, s, sc->prompt_dev, r.cols, &r.gp, s->codes, s->codes_cap);
    if (rc) return rc;
    CU(cudaStreamSynchronize(m->stream));
    return check_err_word(m);
}

// Admit waiting requests (FIFO) while a slot and their pages are free:
// map pages, prefill, sample the first main token.
static s2k_status sched_admit(s2k_sched *sc) {
    while (!sc->waiting.empty()) {
        const int id = sc->waiting.front();
        Req &r = sc->reqs[id];
        const int need = (r.cols + r.gp.max_new_tokens + 1 + kPage - 1) / kPage;
        int si = -1;
        for (int i = 0; i < sc->max_batch; ++i)
            if (sc->slots[i].req < 0) {
                si = i;
                break;
            }
        if (si < 0 || (int)sc->free_pages.size() < need) break;
        sc->waiting.pop_front();
        Slot &sl = sc->slots[si];
        s2k_seq *s = sl.seq;
        sl.pages.assign(sc->free_pages.end() - need, sc->free_pages.end());
        sc->free_pages.resize(sc->free_pages.size() - need);
        s2k_status rc = admit_one(sc, r, s, sl.pages);
        if (rc) {
            for (int pg : sl.pages) sc->free_pages.push_back(pg);
            sl.pages.clear();
            if (rc == S2K_ERR_CUDA || rc == S2K_ERR_TIMEOUT) {
                // the device failed, not the request: it goes back to the head of the queue
                sc->waiting.push_front(id);
                return rc;
            }
            // this request cannot run (no memory for it, bad input): it fails
            // alone and the others carry on
            r.state = S2K_REQ_FAILED;
            r.status = rc;
            sc->stats.failed++;
            continue;
        }
        sl.req = id;
        r.slot = si;
        r.state = S2K_REQ_LIVE;
        sc->stats.admitted++;
        sc->stats.prefill_tokens += r.cols;
        if (s->hstat->done) {
            rc = sched_retire(sc, si);
            if (rc) return rc;
        }
    }
    return S2K_OK;
}

S2K_API s2k_status s2k_sched_step(s2k_sched *sc, int32_t *n_live, int32_t *n_waiting) {
    if (!sc) return fail(S2K_ERR_ARG, "NULL scheduler");
    s2k_model *m = sc->m;
    if (cuda_set(m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    s2k_status rc = sched_admit(sc);
    if (rc) return rc;
    std::vector<s2k_seq *> live;
    std::vector<int> live_slots;
    for (int i = 0; i < sc->max_batch; ++i)
        if (sc->slots[i].req >= 0) {
            live.push_back(sc->slots[i].seq);
            live_slots.push_back(i);
        }
    if (!live.empty()) {
        for (s2k_seq *s : live) sc->stats.kv_positions += s->n_past;
        rc = batch_frame_core(m, live.data(), (int)live.size());
        if (rc) return rc;
        sc->stats.steps++;
        sc->stats.max_live = std::max<int32_t>(sc->stats.max_live, (int32_t)live.size());
        for (size_t j = 0; j < live.size(); ++j) {
            s2k_seq *s = live[j];
            Req &r = sc->reqs[sc->slots[live_slots[j]].req];
            bool cancel = false;
            if (sc->on_frame) {
                // the frame this step produced, from the sequence's host ring
                const int nf = s->hstat->n_frames;
                const int ncb = std::max(m->hp.num_codebooks, 1);
                int codes[16];
                for (; r.delivered < nf && !cancel; ++r.delivered) {
                    for (int cb = 0; cb < ncb; ++cb) codes[cb] = s->hstat->ring[r.delivered % kFrameRing][cb];
                    cancel = !sc->on_frame(sc->slots[live_slots[j]].req, codes, r.delivered, ncb, sc->on_frame_user);
                }
            }
            if (cancel) {
                rc = sched_retire(sc, live_slots[j], S2K_REQ_CANCELLED);
                if (rc) return rc;
            } else if (s->hstat->done) {
                rc = sched_retire(sc, live_slots[j]);
                if (rc) return rc;
            }
        }
        int64_t frames = 0;
        for (Req &r : sc->reqs)
            if (r.state == S2K_REQ_LIVE) frames += sc->slots[r.slot].seq->hstat->n_frames;
            else if (r.state == S2K_REQ_DONE || r.state == S2K_REQ_CANCELLED) frames += r.n_frames;
        sc->stats.frames = frames;
    }
    int nl = 0;
    for (const Slot &sl : sc->slots) nl += sl.req >= 0;
    if (n_live) *n_live = nl;
    if (n_waiting) *n_waiting = (int32_t)sc->waiting.size();
    return S2K_OK;
}

S2K_API s2k_status s2k_sched_run(s2k_sched *sc) {
    if (!sc) return fail(S2K_ERR_ARG, "NULL scheduler");
    for (;;) {
        int32_t nl = 0, nw = 0;
        s2k_status rc = s2k_sched_step(sc, &nl, &nw);
        if (rc) return rc;
        if (nl == 0 && nw == 0) return S2K_OK;
        if (nl == 0 && nw > 0) return fail(S2K_ERR_KV_FULL, "waiting requests that no slot can take");
    }
}

S2K_API s2k_status s2k_sched_poll(s2k_sched *sc, int32_t req_id, int32_t *state, int32_t *n_frames) {
    return s2k_sched_poll_status(sc, req_id, state, n_frames, nullptr);
}

S2K_API s2k_status s2k_sched_poll_status(s2k_sched *sc, int32_t req_id, int32_t *state, int32_t *n_frames,
                                         s2k_status *req_status) {
    if (!sc || req_id < 0 || req_id >= (int32_t)sc->reqs.size()) return fail(S2K_ERR_ARG, "bad request id");
    const Req &r = sc->reqs[req_id];
    if (state) *state = r.state;
    if (req_status) *req_status = r.status;
    if (n_frames) *n_frames = r.state == S2K_REQ_LIVE ? sc->slots[r.slot].seq->hstat->n_frames : r.n_frames;
    return S2K_OK;
}

S2K_API s2k_status s2k_sched_result(s2k_sched *sc, int32_t req_id, int32_t *codes_out, int32_t cap_frames,
                                    int32_t *n_frames) {
    if (!sc || req_id < 0 || req_id >= (int32_t)sc->reqs.size() || !n_frames) return fail(S2K_ERR_ARG, "bad argument");
    const Req &r = sc->reqs[req_id];
    if (r.state != S2K_REQ_DONE && r.state != S2K_REQ_CANCELLED)
        return fail(S2K_ERR_STATE, "request %d has no result (state %d)", req_id, r.state);
    *n_frames = r.n_frames;
    if (codes_out) {
        if (cap_frames < r.n_frames) return fail(S2K_ERR_ARG, "codes capacity %d < %d frames", cap_frames, r.n_frames);
        std::copy(r.codes.begin(), r.codes.end(), codes_out);
    }
    return S2K_OK;
}

S2K_API s2k_status s2k_sched_get_stats(const s2k_sched *sc, s2k_sched_stats *out) {
    if (!sc || !out) return fail(S2K_ERR_ARG, "NULL argument");
    *out = sc->stats;
    out->free_pages = (int32_t)sc->free_pages.size();
    out->pool_pages = sc->pool_pages;
    return S2K_OK;
}

S2K_API s2k_status s2k_sched_cancel(s2k_sched *sc, int32_t req_id) {
    if (!sc || req_id < 0 || req_id >= (int32_t)sc->reqs.size()) return fail(S2K_ERR_ARG, "bad request id");
    if (cuda_set(sc->m->device)) return fail(S2K_ERR_CUDA, "cudaSetDevice failed");
    Req &r = sc->reqs[req_id];
    if (r.state == S2K_REQ_WAITING) {
        auto it = std::find(sc->waiting.begin(), sc->waiting.end(), req_id);
        if (it != sc->waiting.end()) sc->waiting.erase(it);
        r.state = S2K_REQ_CANCELLED;
        r.n_frames = 0;
        r.codes.clear();
        sc->stats.cancelled++;
        return S2K_OK;
    }
    if (r.state == S2K_REQ_LIVE) {
        // between frames nothing of the scheduler runs on the device: the
        // request keeps the frames it has, its pages go back to the pool
        return sched_retire(sc, r.slot, S2K_REQ_CANCELLED);
    }
    return S2K_OK;  // finished, failed or cancelled already: nothing to stop
}

S2K_API s2k_status s2k_sched_set_frame_callback(s2k_sched *sc, s2k_sched_frame_callback cb, void *user) {
    if (!sc) return fail(S2K_ERR_ARG, "NULL scheduler");
    sc->on_frame = cb;
    sc->on_frame_user = user;
    return S2K_OK;
}
