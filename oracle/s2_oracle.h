/*
 * s2_oracle.h -- CPU restatement of s2.cpp's per-frame dual-AR decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in s2.cpp_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product never links it.
 *
 * What it restates (file:line are paths inside the s2.cpp project):
 *   - SlowARModel::eval_cached      src/s2_model.cpp:860-1097
 *   - SlowARModel::fast_decode      src/s2_model.cpp:1099-1255
 *   - sample_token                  src/s2_sampler.cpp:42-99
 *   - generate (frame loop, RAS)    src/s2_generate.cpp:11-216
 *   - hparam keys / defaults        src/s2_model.cpp:245-288
 * and the ggml arithmetic those call sites reach (ggml is an un-vendored
 * submodule of s2.cpp; its published CPU algorithms are restated here):
 *   - Q8_0 / Q4_K / Q6_K block layouts and dequantize_row_*      (pinned
 *     bit-exact against gguf-py 0.19.0 gguf/quants.py in tests/)
 *   - activation quantization of the CPU mat-vec: Q8_0 (x86 AVX2 form:
 *     id = 127/amax, round-half-even) and Q8_K (nearest_int, -127/max)
 *   - vec_dot_q8_0_q8_0, vec_dot_q4_K_q8_K, vec_dot_q6_K_q8_K, f16 dot
 *   - rms_norm (double accumulation), rope mode 0 with the cumulative
 *     theta *= theta_scale recurrence, soft_max, swiglu.
 *
 * Rounding convention (shared with the CUDA kernels): every reduction that
 * feeds an activation quantizer is evaluated as exactly-formed terms summed
 * in double and rounded to float once, and exp is so_det_expf.  ggml's own
 * float accumulation order is implementation-defined (SIMD width, thread
 * split); this convention is the order-free limit of it, and it lets the GPU
 * and this oracle agree bit for bit, which a Q8_0-quantized network needs:
 * any 1-ulp difference can flip an int8 activation and is then amplified
 * layer by layer.
 *
 * Pinning: the block formats are pinned (gguf-py known-answer vectors).  The
 * model-level math (eval / fast_decode / generate) is parity unpinned: the
 * reference's ggml backend cannot be built here and the reference ships no
 * golden vectors, so the restatement is checked by its own semantic tests
 * (prefill vs incremental, sampler rules, stop rules) and the CUDA path is
 * checked bit for bit against it.
 *
 * RNG: the reference draws from a thread_local mt19937 seeded by
 * std::random_device (src/s2_sampler.cpp:94), which no test can pin.  Both
 * this oracle and the CUDA sampler instead draw u ~ U[0,1) from Philox4x32-10
 * (Salmon et al., SC'11) keyed by a user seed and countered by
 * (frame, purpose, seq) -- see so_philox_uniform().
 */
#ifndef S2_ORACLE_H
#define S2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids used by the GGUF files s2.cpp loads */
enum {
    SO_TYPE_F32 = 0,
    SO_TYPE_F16 = 1,
    SO_TYPE_Q8_0 = 8,
    SO_TYPE_Q4_K = 12,
    SO_TYPE_Q6_K = 14,
    SO_TYPE_Q8_K = 15,
};

/* Mirrors s2::ModelHParams (include/s2_model.h:38-69). */
typedef struct so_hparams {
    int32_t context_length;
    int32_t vocab_size;
    int32_t embedding_length;
    int32_t feed_forward_length;
    int32_t block_count;
    int32_t head_count;
    int32_t head_count_kv;
    int32_t head_dim;
    int32_t codebook_size;
    int32_t num_codebooks;
    int32_t semantic_begin_id;
    int32_t semantic_end_id;
    float rope_freq_base;
    float rms_norm_eps;
    int32_t tie_word_embeddings;
    int32_t attention_qk_norm;
    int32_t scale_codebook_embeddings;
    int32_t fast_context_length;
    int32_t fast_embedding_length;
    int32_t fast_feed_forward_length;
    int32_t fast_block_count;
    int32_t fast_head_count;
    int32_t fast_head_count_kv;
    int32_t fast_head_dim;
    float fast_rope_freq_base;
    float fast_rms_norm_eps;
    int32_t fast_attention_qk_norm;
    int32_t fast_has_project_in;
    int32_t has_fast_decoder;
} so_hparams;

typedef struct so_model so_model;

/* ---- primitives (pinned by tests against gguf-py and hand KATs) ---- */
int64_t so_row_bytes(int type, int64_t n);
int so_dequant_row(int type, const void *src, float *dst, int64_t n);
/* ggml-cpu x86 quantize_row_q8_0: 34-byte blocks (fp16 d, 32 x int8) */
void so_quantize_act_q8_0(const float *x, int64_t n, uint8_t *out);
/* ggml quantize_row_q8_K_ref: 292-byte blocks (f32 d, 256 x int8, 16 x int16 bsums) */
void so_quantize_act_q8_K(const float *x, int64_t n, uint8_t *out);
/* one weight row (GGUF-native blocks) dotted with an activation row quantized
 * to the vec_dot type ggml pairs with it (Q8_0 -> Q8_0, K-quants -> Q8_K,
 * F16 -> F16, F32 -> F32) */
float so_vec_dot(int type, const void *wrow, const void *act, int64_t n);
/* y[r] = W[r,:] . x for a [rows x n] GGUF-native matrix, x f32; n_threads<=0: all */
void so_matvec(int type, const void *w, int64_t rows, int64_t n, const float *x, float *y);
uint16_t so_fp32_to_fp16(float f);
/* exp(x) by a fixed float operation sequence shared with the CUDA kernels */
float so_det_expf(float x);
float so_pow2_scale(float p, int k);
void so_det_expf_array(const float *x, float *y, int64_t n);
int64_t so_check_pow2_scale(int64_t n, uint32_t seed);
float so_det_sinf(float x);
float so_fp16_to_fp32(uint16_t h);
void so_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
double so_philox_uniform(uint64_t seed, uint32_t frame, uint32_t purpose, uint32_t seq);

/* ---- model ---- */
so_model *so_model_create(const so_hparams *hp);
void so_model_free(so_model *m);
/* Tensor data is referenced, not copied: keep it alive while the model lives.
 * name / ne follow the GGUF tensor names and ggml ne order [in, out]. */
int so_model_set_tensor(so_model *m, const char *name, int type, const int64_t ne[4],
                        const void *data, size_t nbytes);
int so_model_check(so_model *m);                 /* all required tensors bound? */
int so_kv_init(so_model *m, int32_t max_seq_len); /* init_kv_cache */
void so_kv_clear(so_model *m);                    /* clear_kv_cache */
/* restore n_pos cached positions, f16 [layer][pos][kv_head][head_dim]; n_past = n_pos */
int so_kv_load(so_model *m, const uint16_t *k, const uint16_t *v, int32_t n_pos);
int32_t so_n_past(const so_model *m);
/* eval_cached: flat_tokens is [n_tokens][num_codebooks+1] token-major */
int so_eval(so_model *m, const int32_t *flat_tokens, int32_t n_tokens, float *hidden_out,
            float *logits_out);
/* fast_decode: hidden[dim], prefix[n_prefix] (n_prefix < num_codebooks) */
int so_fast_decode(so_model *m, const float *hidden, const int32_t *prefix, int32_t n_prefix,
                   float *logits_out);

/* sample_token with lowest-index tie break and a supplied uniform u */
int32_t so_sample_token(const float *logits, int32_t n, float temperature, float top_p,
                        int32_t top_k, double u);

typedef struct so_gen_params {
    int32_t max_new_tokens;
    float temperature;
    float top_p;
    int32_t top_k;
    int32_t min_tokens_before_end;
    int32_t im_end_id;
    uint64_t seed;
    uint32_t seq_id;
} so_gen_params;

/* generate(): prompt is [rows = num_codebooks+1][cols] row-major (PromptTensor).
 * codes_out: [num_codebooks][max_new_tokens] cb-major, compacted to n_frames like
 * the reference (src/s2_generate.cpp:201-213). */
int so_generate(so_model *m, const int32_t *prompt, int32_t cols, const so_gen_params *gp,
                int32_t *codes_out, int32_t *n_frames_out);
/* The same with the reference's [Metrics] split (src/s2_generate.cpp:185-199):
 * wall-clock prefill and frame-loop milliseconds. */
int so_generate_timed(so_model *m, const int32_t *prompt, int32_t cols, const so_gen_params *gp,
                      int32_t *codes_out, int32_t *n_frames_out, double *prefill_ms, double *loop_ms);

/* Philox purposes, shared with the CUDA sampler */
enum { SO_RNG_MAIN = 0, SO_RNG_RAS = 1, SO_RNG_FAST0 = 2 };

void so_set_threads(int n);

/* ---- codec decode (s2_codec_oracle.c): AudioCodec::decode, src/s2_codec.cpp:1297-1447 ---- */
typedef struct so_codec_hparams {
    int32_t sample_rate, hop_length;
    int32_t latent_dim, decoder_dim;
    int32_t n_decoder_rates, decoder_rates[8];
    int32_t quantizer_input_dim, quantizer_codebook_dim;
    int32_t quantizer_residual_codebooks, quantizer_residual_codebook_size, quantizer_semantic_codebook_size;
    int32_t n_downsample, quantizer_downsample_factor[8];
    int32_t rvq_window_size, rvq_block_size, rvq_n_layer, rvq_n_local_heads, rvq_head_dim, rvq_dim;
    float rvq_rope_base, rvq_norm_eps;
} so_codec_hparams;
typedef struct so_codec so_codec;
so_codec *so_codec_create(const so_codec_hparams *hp);
void so_codec_free(so_codec *c);
/* F32 or F16 tensor under its GGUF name (the "c." prefix is optional); copied */
int so_codec_set_tensor(so_codec *c, const char *name, int type, const int64_t ne[4], const void *data);
int64_t so_codec_samples(const so_codec *c, int32_t n_frames);
/* codes [num_codebooks][n_frames] cb-major -> audio [*n_samples] (capacity cap) */
int so_codec_decode(const so_codec *c, const int32_t *codes, int32_t n_frames, float *audio, int64_t cap,
                    int64_t *n_samples);
/* 1: the decode's dot products accumulate in float, in sequence, instead of
 * double (a second accumulation order, for measuring the graph's own drift) */
void so_codec_set_f32_accum(int on);

#ifdef __cplusplus
}
#endif
#endif
