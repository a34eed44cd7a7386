// s2k_kernels.h -- host-side launchers of the decode kernels (internal).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "s2k_tgemv.cuh"

namespace s2k {

struct SeqDev;  // s2k_device.h

// One token row of a batched call over independent sequences (continuous
// batching).  The rows of one sequence are contiguous and in position order.
struct BatchRow {
    int slot;    // the row's sequence: index into the call's sequence array
    int off;     // position = base + off; base = the sequence's n_past (Slow stack) or 0 (Fast stack)
    int cur_lo;  // this call's keys of the row: K/V rows [cur_lo, cur_hi] of kcur / vcur
    int cur_hi;  // the row's own K/V row in kcur / vcur
};

// ---------------------------------------------------------------------------
// Weight matrix in device layout: 32 x 512 tiles (s2k_tgemv.cuh) of
//   Q8_0 : int8 quants + fp16 scales,
//   Q4_K / Q6_K : GGUF super-blocks split into quant / scale planes;
// rows % 32 == 0 and cols % 512 == 0.
// ---------------------------------------------------------------------------
struct DevMat {
    int type = -1;  // ggml type id
    int rows = 0, cols = 0;
    uint8_t *w = nullptr;
    // Q4_K / Q6_K matrices of the Slow stack: the int8 copy the tensor-core
    // prefill reads and its (d, dmin) side array (s2k_prefill.cu); null when
    // absent
    uint8_t *pf = nullptr;
    uint8_t *pf_side = nullptr;
    size_t bytes() const;
};

struct GemvArgs {
    const DevMat *w = nullptr;
    const float *x = nullptr;  // [M][ldx]
    int ldx = 0;
    int M = 1;
    int in_mode = IN_PLAIN;
    const float *norm_w = nullptr;
    float eps = 0.f;
    int epi = EPI_STORE;
    float *y = nullptr;  // [M][ldy]
    int ldy = 0;
    const float *res = nullptr;  // optional residual [M][ldres], y = res + W.x
    int ldres = 0;
    float *act_out = nullptr;  // optional: CTA 0 stores the (normed) f32 activation [M][K]
    const int *done = nullptr;  // optional early-exit flag (frame loop)
    int *err = nullptr;
};

// Launch with programmatic-dependent-launch attribute on `st`.
cudaError_t launch_gemv(const GemvArgs &a, int num_sms, cudaStream_t st);
// smem bytes a gemv launch for (K, M) needs (to set the function attribute once).
cudaError_t gemv_setup();

// Q8_0 GGUF blocks (34 B) of rows [row0, row0 + rows) in device staging ->
// tiles of dst; source row r lands in dst row r * row_stride + row_offset
// (row_stride 2 interleaves w1/w3).
cudaError_t launch_relayout_q8_0(const uint8_t *src, int row0, int rows, int cols, DevMat *dst, int row_stride,
                                 int row_offset, cudaStream_t st);
// Same for any tile type (dst->type: ggml Q8_0, Q4_K or Q6_K blocks in src).
cudaError_t launch_relayout(const uint8_t *src, int row0, int rows, int cols, DevMat *dst, int row_stride,
                            int row_offset, cudaStream_t st);
// Tile-engine weight type (TWType) of a ggml type id, -1 if not a tile type.
int tw_of(int ggml_type);

// ---------------------------------------------------------------------------
// Prefill GEMM on the tensor cores (s2k_prefill.cu): y[T][R] (+ res, or
// SwiGLU of interleaved rows) from activations already quantized by
// launch_quant_rows_q8 (Q8_0 weights) or launch_quant_rows_q8k (Q4_K / Q6_K
// weights through their prefill copy, 64+ tokens).
// ---------------------------------------------------------------------------
struct PrefillArgs {
    const DevMat *w = nullptr;
    int T = 0;
    const int8_t *xq = nullptr;  // [T][K] int8
    const double *dx = nullptr;  // [T][K/32] block scales
    int epi = EPI_STORE;
    float *y = nullptr;
    int ldy = 0;
    const float *res = nullptr;
    int ldres = 0;
    double *part = nullptr;  // stream-K partials (>= prefill_part_doubles(num_sms))
    size_t part_doubles = 0;
    int *counters = nullptr;  // >= (R/128) * ceil(T/16) ints, zero between launches
    size_t n_counters = 0;
    int num_sms = 148;
    int *err = nullptr;
};
cudaError_t prefill_setup();
size_t prefill_part_doubles(int ctas);
bool prefill_ok(const DevMat &w, int T);
cudaError_t launch_prefill_gemm(const PrefillArgs &a, cudaStream_t st);
// Prefill GEMM on the tensor cores for F16 matrices (s2k_prefill_f16.cu);
// fp32 accumulation (prefill only: not the decode arithmetic).
cudaError_t prefill_f16_setup();
bool prefill_f16_ok(const DevMat &w, int T);
cudaError_t launch_rows_f16(const float *x, int ldx, int T, int K, const float *norm_w, float eps, __half *xh,
                            float *act_out, cudaStream_t st);
cudaError_t launch_prefill_f16_gemm(const uint8_t *wtiles, int R, int K, int T, const __half *xh, int epi, float *y,
                                    int ldy, const float *res, int ldres, int num_sms, int *err, cudaStream_t st);
// K-quant prefill copy of a Q4_K / Q6_K matrix: bytes of its int8 tiles (0
// when the matrix cannot have one) and of its side array; the launch fills
// w.pf / w.pf_side (allocated by the caller) from the decode tiles w.w.
size_t kq_prefill_bytes(const DevMat &w, size_t *side_bytes);
cudaError_t launch_build_kq_prefill(const DevMat &w, cudaStream_t st);
// x [T][ldx] (optional RMSNorm) -> Q8_K rows for the K-quant GEMM of a matrix
// of ggml type ggml_type: xq [T][Ke] int8 and slots [T][Ke/32], Ke = K (Q4_K)
// or 2K (Q6_K, each 16 values followed by 16 zeros).
cudaError_t launch_quant_rows_q8k(const float *x, int ldx, int T, int K, const float *norm_w, float eps, int ggml_type,
                                  int8_t *xq, double *slots, float *act_out, cudaStream_t st);
// x [T][ldx] (optional RMSNorm with norm_w, eps) -> xq [T][K] int8, dx [T][K/32]
cudaError_t launch_quant_rows_q8(const float *x, int ldx, int T, int K, const float *norm_w, float eps, int8_t *xq,
                                 double *dx, float *act_out, cudaStream_t st);

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------
struct KvPaged {
    __half *k = nullptr, *v = nullptr;  // [page][layer][kv_head][16][head_dim]
    const int *block_table = nullptr;   // logical page -> physical page
    int n_layers = 0, n_kv_heads = 0, head_dim = 0, n_pages = 0;
};
constexpr int kPage = 16;

struct QkPrepArgs {
    float *qkv = nullptr;  // [T][ldqkv] raw projections, q rotated in place
    int ldqkv = 0;
    int T = 1, H = 0, Hkv = 0, hd = 128;
    const float *q_norm = nullptr, *k_norm = nullptr;  // null: no qk-norm
    float eps = 0.f;
    const float2 *rope = nullptr;  // [rope_positions][hd/2] (cos, sin)
    int rope_positions = 0;
    const int *pos_base = nullptr;  // device: position of token 0 (n_past); null = 0
    int pos_add = 0;                // added to *pos_base
    float *kcur = nullptr, *vcur = nullptr;  // f32 [*][Hkv][hd] at index cur_base + t
    int cur_base = 0;
    KvPaged kv;  // if kv.k: also store f16 K/V of (layer) at the token's position
    int layer = 0;
    // batched call: row t is rows[t]; position, K/V row and (with seqs) the
    // KV pages it stores to come from the descriptor and its sequence
    const BatchRow *rows = nullptr;
    SeqDev *const *seqs = nullptr;
    const int *done = nullptr;
    int *err = nullptr;
};
cudaError_t launch_qk_prep(const QkPrepArgs &a, cudaStream_t st);

struct AttnArgs {
    const float *q = nullptr;  // [T][ldq] rotated queries (head h at h*hd)
    int ldq = 0;
    int T = 1, H = 0, Hkv = 0, hd = 128;
    float scale = 1.f;
    const int *n_cached = nullptr;  // device: # positions held in the paged cache (null = 0)
    KvPaged kv;
    int layer = 0;
    const float *kcur = nullptr, *vcur = nullptr;  // f32 [*][Hkv][hd], position n_cached + j at index j
    int cur_base = 0;  // token t attends to cur indices [0, cur_base + t]
    int max_keys = 0;  // upper bound of any token's key range (sizes the split-maxima buffer)
    float *scores = nullptr;  // scratch [T][H][ld_scores]
    int ld_scores = 0;        // >= longest key range of the call
    float *out = nullptr;     // [T][H*hd]
    // batched call: row t attends to its sequence's cached positions (with
    // seqs; none without) and to kcur / vcur rows [cur_lo, cur_hi] of rows[t]
    const BatchRow *rows = nullptr;
    SeqDev *const *seqs = nullptr;
    // split-parallel path (one CTA per (split, kv head, row)): per-split
    // partials O_i [T][Hkv][fl_nsp][G][hd] and (m_i, S_i) [T][Hkv][fl_nsp][G][2],
    // arrival counters [T][Hkv] (zero between launches); null = one CTA per
    // (kv head, row)
    double *fl_part = nullptr, *fl_ms = nullptr;
    int *fl_counters = nullptr;
    int fl_nsp = 0;
    int num_sms = 148;
    const int *done = nullptr;
    int *err = nullptr;
};
// keys per attention split (the CPU oracle splits the same way)
constexpr int kAttnSplit = 64;
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st);
cudaError_t attn_setup();  // once per device before the first launch_attention

// ---------------------------------------------------------------------------
// Embeddings / sampling / frame bookkeeping
// ---------------------------------------------------------------------------
struct EmbedArgs {
    const DevMat *tok_emb = nullptr;  // embeddings (Slow) or fast_embeddings (Fast)
    const DevMat *cb_emb = nullptr;   // codebook_embeddings (Slow only)
    const int *tokens = nullptr;      // Slow: [T][ncb+1]; Fast: codes
    int T = 1;
    int ncb = 0, cb_size = 0, sem_begin = 0, sem_end = -1;
    int scale_cb = 0;
    float sem_scale = 1.f;
    float *x = nullptr;  // [T][dim]
    SeqDev *const *seqs = nullptr;  // batched frame: row t's tokens are seqs[t]'s next step input
    const int *done = nullptr;
    int *err = nullptr;
};
cudaError_t launch_embed_slow(const EmbedArgs &a, cudaStream_t st);
// Fast-AR input rows: row r (r < n_rows) of x = (r == 0 && hidden) ? hidden : fast_emb[codes[code0 + r - (hidden?1:0)]]
cudaError_t launch_embed_fast(const DevMat *fast_emb, const float *hidden, const int *codes, int code0,
                              int n_rows, float *x, int dim, const int *done, int *err, cudaStream_t st);

// Fast-AR input rows of pass `pass` of a batched frame over n sequences:
// pass 0 rows (2b, 2b+1) = (hidden of b, fast_emb[codes_b[0]]); pass p > 0
// row b = fast_emb[codes_b[p]].
cudaError_t launch_embed_fast_batch(const DevMat *fast_emb, SeqDev *const *seqs, int n, int pass, float *x, int dim,
                                    int *err, cudaStream_t st);

// Frame-loop launchers (state structs in s2k_device.h).
cudaError_t sampler_setup();
// After a Slow step (or the prefill): sample the main token of the next frame
// with the semantic mask, stop test, RAS, window push, codes[0].
cudaError_t launch_sample_main(const float *logits, SeqDev *sd, int *err, cudaStream_t st);
// After the Fast-AR pass for codebook cb: sample codes[cb].
cudaError_t launch_sample_fast(const float *logits, SeqDev *sd, int cb, int *err, cudaStream_t st);
// End of the Fast-AR loop: store the frame's codes, n_frames++, step input.
cudaError_t launch_frame_commit(SeqDev *sd, cudaStream_t st);
// After the Slow step kernels: n_past += T.
cudaError_t launch_advance(SeqDev *sd, int T, const int *done, cudaStream_t st);
// Batched frame over n sequences (one CTA per sequence): logits row b
// belongs to seqs[b].  sample_main also stores hidden row b as the
// sequence's hidden state.
cudaError_t launch_sample_main_batch(const float *logits, size_t ld, SeqDev *const *seqs, int n, const float *hidden,
                                     int dim, int *err, cudaStream_t st);
cudaError_t launch_sample_fast_batch(const float *logits, size_t ld, SeqDev *const *seqs, int n, int cb, int *err,
                                     cudaStream_t st);
cudaError_t launch_frame_commit_batch(SeqDev *const *seqs, int n, cudaStream_t st);
cudaError_t launch_advance_batch(SeqDev *const *seqs, int n, int T, cudaStream_t st);
// get_rows of a (tiled) weight matrix: out [n][E->cols] f32 (s2k_get_rows).
cudaError_t launch_gather_rows(const DevMat *E, const int *ids, int n, float *out, int *err, cudaStream_t st);
// Standalone sampler (s2k_sample)
cudaError_t launch_sample_one(const float *logits, int n, float temperature, float top_p, int top_k,
                              double u, int *out, int *err, cudaStream_t st);
// det_expf of n floats (s2k_debug_det_expf)
cudaError_t launch_det_expf(const float *x, float *y, long long n, cudaStream_t st);

// launch accounting
void count_launch(int n = 1);

}  // namespace s2k
