// s2k_model.h -- the model and sequence objects behind the C ABI and the
// host-side pieces the single-sequence and batched entry points share
// (internal).
#pragma once

#include "../../include/s2k.h"
#include "s2k_common.cuh"
#include "s2k_device.h"
#include "s2k_kernels.h"
#include "s2k_mega.h"

#include <algorithm>
#include <cstddef>
#include <string>
#include <vector>

namespace s2k {

s2k_status fail(s2k_status code, const char *fmt, ...);

#define CU(expr)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (expr);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            return fail(e_ == cudaErrorMemoryAllocation ? S2K_ERR_OOM : S2K_ERR_CUDA, "%s: %s (%s:%d)", #expr, \
                        cudaGetErrorString(e_), __FILE__, __LINE__);                               \
    } while (0)

struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    DevMat wqkv, wo, w13, w2;
    bool has_w1 = false, has_w3 = false;
};

// Activations of one transformer stack for up to T tokens.
struct Work {
    int T = 0, L = 0, dim = 0, qs = 0, kvs = 0, ff = 0, H = 0;
    int Tm = 0;  // tokens the persistent-kernel buffers below hold (min(T, kMegaTokens))
    float *x = nullptr, *h = nullptr, *qkv = nullptr, *attn = nullptr, *ff_buf = nullptr;
    float *kcur = nullptr, *vcur = nullptr, *scores = nullptr;
    // persistent-kernel attention: per (token, kv head, split) the split's
    // O_i [G][hd] and (m_i, S_i) [G][2]; arrival counters per (token, kv head)
    double *part = nullptr, *part_ms = nullptr;
    int *counters = nullptr;
    int n_split_max = 0;
    // persistent kernel: tagged-word copies of x, h, qkv, attention output and
    // SwiGLU output (8 bytes per value), written and read only inside it
    uint64_t *lx = nullptr, *lh = nullptr, *lqkv = nullptr, *lattn = nullptr, *lff = nullptr;
    // tensor-core prefill: quantized activation rows, their block scales,
    // split-K partials and arrival counters (Slow work only)
    int8_t *pf_xq = nullptr;
    double *pf_dx = nullptr, *pf_part = nullptr;
    size_t pf_part_n = 0, pf_n_counters = 0;
    int *pf_counters = nullptr;
    __half *pf_xh = nullptr;  // fp16 activation rows of the fp16 tensor-core prefill [T][kmax]
    // split-parallel attention (calls of up to fl_T rows): per-split partials
    double *fl_part = nullptr, *fl_ms = nullptr;
    int *fl_counters = nullptr;
    int fl_T = 0, fl_nsp = 0;
};

// Tokens per call from which the Slow stack's Q8_0 GEMMs run on the tensor
// cores (s2k_prefill.cu) instead of the tile GEMV.
#ifndef S2K_PREFILL_MIN_T
#define S2K_PREFILL_MIN_T 8
#endif
constexpr int kPrefillMinT = S2K_PREFILL_MIN_T;
// Tokens per call from which K-quant GEMMs run on the tensor cores (their
// 64-token tiles; s2k_prefill.cu prefill_ok).
constexpr int kPrefillKqMinT = 64;
// Most tokens of one persistent-kernel call (the first Fast-AR pass: hidden + code 0).
constexpr int kMegaTokens = 2;

struct BatchState;  // batched frames over independent sequences (s2k_batch.cu)

}  // namespace s2k

using namespace s2k;  // internal header: the ABI objects below use the library's types

struct s2k_model {
    s2k_hparams hp{};
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    DevMat embed, cb_embed, fast_embed, fast_out;
    float *norm = nullptr, *fast_norm = nullptr;
    std::vector<Layer> layers, fast_layers;
    std::vector<void *> allocs;
    std::vector<size_t> alloc_bytes;  // size of allocs[i]
    size_t dev_bytes = 0;             // device bytes this model holds
    long long fail_alloc_at = -1;     // test hook: the allocation this many allocations ahead fails (once)
    bool finalized = false;
    bool prefill_mma = false;  // the tensor-core prefill path could be set up on this device
    bool prefill_f16 = false;  // the fp16 tensor-core prefill GEMM (F16 models) could be set up
    // K-quant tensor-core prefill: two layer slots of int8 copies (layer il in slot il % 2)
    uint8_t *kq_slots[2] = {nullptr, nullptr};
    size_t kq_slot_bytes = 0;
    int *d_err = nullptr;
    unsigned *d_epoch = nullptr;  // tag epoch of the persistent kernel's activations (starts at 1)
    // staging for uploads
    uint8_t *staging = nullptr;
    size_t staging_bytes = 0;
    // Slow workspace (ws_gen changes whenever it is reallocated: captured
    // frame graphs hold its pointers)
    Work sw;
    int ws_gen = 0;
    float *logits = nullptr, *hidden = nullptr;
    int *tokens = nullptr;
    int tokens_cap = 0;
    // Fast workspace (T <= num_codebooks)
    Work fw;
    std::vector<float *> fkcur, fvcur;
    float *flogits = nullptr, *fhidden = nullptr;
    int *fcodes = nullptr;
    // RoPE cos/sin tables [positions][head_dim/2]
    float2 *rope_slow = nullptr, *rope_fast = nullptr;
    int rope_slow_n = 0, rope_fast_n = 0;
    // standalone sampler scratch
    float *samp_logits = nullptr;
    int samp_cap = 0;
    int *samp_out = nullptr;
    // batched frames (s2k_batch.cu)
    BatchState *batch = nullptr;

    template <class T>
    cudaError_t alloc(T **p, size_t n) {
        if (fail_alloc_at >= 0 && fail_alloc_at-- == 0) return cudaErrorMemoryAllocation;
        void *v = nullptr;
        const size_t bytes = std::max<size_t>(n, 1) * sizeof(T);
        cudaError_t e = cudaMalloc(&v, bytes);
        if (e == cudaSuccess) {
            allocs.push_back(v);
            alloc_bytes.push_back(bytes);
            dev_bytes += bytes;
            *p = reinterpret_cast<T *>(v);
        }
        return e;
    }
    void release(void *p) {
        if (!p) return;
        auto it = std::find(allocs.begin(), allocs.end(), p);
        if (it != allocs.end()) {
            const size_t i = (size_t)(it - allocs.begin());
            dev_bytes -= alloc_bytes[i];
            alloc_bytes.erase(alloc_bytes.begin() + (std::ptrdiff_t)i);
            allocs.erase(it);
        }
        cudaFree(p);
    }
};

struct s2k_seq {
    s2k_model *m = nullptr;
    int max_seq_len = 0, n_pages = 0;
    __half *k = nullptr, *v = nullptr;
    int *block_table = nullptr;
    SeqDev *dev = nullptr;
    HostStatus *hstat = nullptr;      // mapped pinned
    HostStatus *hstat_dev = nullptr;  // device alias
    int n_past = 0;                   // host mirror
    float *hidden = nullptr;          // Slow hidden state that feeds the next Fast-AR pass (batched frames)
    bool pooled = false;              // k / v belong to a scheduler's page pool
    int *codes = nullptr;             // [ncb][codes_cap]
    int codes_cap = 0;
    int *prompt = nullptr;
    int prompt_cap = 0;
    cudaGraphExec_t frame_exec = nullptr;
    size_t frame_nodes = 0;
    int frame_gen = -1;
    // persistent-kernel frame program: segments of ops in device memory
    MegaOp *mega_ops = nullptr;
    MegaCtl *mega_ctl = nullptr;
    std::vector<int> seg_start, seg_len, seg_mt;
    bool use_mega = false;
    bool mega_q8 = false;  // every GEMV op of the frame program is Q8_0
    // single-token s2k_eval on the persistent kernel (its own token row and counters)
    MegaOp *eval_ops = nullptr;
    MegaCtl *eval_ctl = nullptr;
    int *eval_tokens = nullptr;
    int eval_len = 0, eval_gen = -1;
    bool eval_ok = false, eval_q8 = false;
    s2k_gen_metrics metrics{};  // of the last s2k_generate / s2k_generate_device
    KvPaged kv() const {
        KvPaged p;
        p.k = k;
        p.v = v;
        p.block_table = block_table;
        p.n_layers = m->hp.block_count;
        p.n_kv_heads = m->hp.head_count_kv;
        p.head_dim = m->hp.head_dim;
        p.n_pages = n_pages;
        return p;
    }
};

namespace s2k {

struct StackCall {
    bool fast = false;
    int T = 1;
    const int *pos_base = nullptr;  // device n_past (Slow) or null
    int pos_add = 0;
    int cur_base = 0;
    KvPaged kv;        // Slow only
    int max_keys = 0;  // upper bound of any token's key range
    const int *done = nullptr;
    // batched calls over independent sequences: per-row descriptors and the
    // call's sequences (Slow: their n_past and KV pages; null in the Fast stack)
    const BatchRow *rows = nullptr;
    SeqDev *const *seqs = nullptr;
    Work *w = nullptr;            // activations (default: the model's Slow / Fast work)
    float *const *fk = nullptr;   // Fast stack: per-layer K/V rows of the call (default m->fkcur / fvcur)
    float *const *fv = nullptr;
    bool mma = false;             // Q8_0 GEMMs of T >= kPrefillMinT rows may use the tensor cores
    bool f16mma = false;          // prompt prefill: F16 GEMMs may use the fp16 tensor-core GEMM
};

}  // namespace s2k

// Host-side pieces shared by the single-sequence and batched entry points
// (s2k_api.cu, s2k_batch.cu).
int cuda_set(int dev);
s2k_status check_err_word(s2k_model *m);
// T: tokens per call; L: longest key range (positions) a call attends over.
// prefill: also the buffers of the tensor-core GEMM path (T >= kPrefillMinT).
// flash_rows: calls of up to this many rows use the split-parallel attention.
cudaError_t work_alloc(s2k_model *m, Work &w, int T, int L, int dim, int H, int Hkv, int hd, int ff, int n_layers,
                       bool prefill, int flash_rows = 0);
void work_free(s2k_model *m, Work &w);
s2k_status ensure_slow_work(s2k_model *m, int T, int L);
// exact: Q8_0 GEMMs of 8+ rows on the tensor cores (the decode arithmetic);
// f16: F16 GEMMs of 8+ rows on the fp16 tensor-core GEMM (prefill).
cudaError_t stack_gemm(s2k_model *m, Work &w, const GemvArgs &g, bool exact, bool f16 = false);
cudaError_t run_stack(s2k_model *m, const StackCall &c);
cudaError_t enqueue_slow(s2k_model *m, s2k_seq *s, int T, const int *tokens_dev, const int *done);
s2k_status check_tokens_host(const s2k_model *m, const int32_t *flat, int32_t T);
void fill_sample_cfg(const s2k_model *m, const s2k_gen_params *gp, int *d_codes, int codes_ld, SampleCfg *c);
void batch_free(s2k_model *m);
s2k_status seq_publish(s2k_seq *s);
// Whether `name` is a tensor the model binds (the GGUF names SlowARModel
// reads, src/s2_model.cpp:374-423; Fast-AR tensors only with a fast decoder).
bool s2k_model_binds(const s2k_model *m, const char *name);
