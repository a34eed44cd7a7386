/*
 * s2k.h -- C ABI of the B200-native dual-AR decode path for s2.cpp.
 *
 * This is the thin layer that replaces the ggml graph inside
 * s2::SlowARModel (src/s2_model.cpp) and the per-frame work of s2::generate
 * (src/s2_generate.cpp).  Plain C types only: pointers, sizes, status codes.
 * Every entry point below names the reference interface it stands in for.
 *
 * Threading: one host thread per model handle at a time, like the reference
 * (SlowARModel keeps n_past_ and its graph buffers as members,
 * include/s2_model.h:147-151; Pipeline serialises synthesis with
 * synthesize_mutex_, include/s2_pipeline.h:111).
 *
 * Errors: every call returns s2k_status (0 = OK, negative = error) and sets a
 * thread-local message readable with s2k_last_error().  No exception crosses
 * this boundary (the reference's model layer also reports bool + stderr,
 * src/s2_model.cpp:863-875, 1064-1086).
 */
#ifndef S2K_H
#define S2K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define S2K_API __declspec(dllexport)
#else
#define S2K_API __attribute__((visibility("default")))
#endif

#define S2K_ABI_VERSION 1

typedef int32_t s2k_status;
enum {
    S2K_OK = 0,
    S2K_ERR_ARG = -1,         /* bad argument / shape / name */
    S2K_ERR_OOM = -2,         /* device or pinned allocation failed */
    S2K_ERR_CUDA = -3,        /* CUDA runtime error */
    S2K_ERR_KV_FULL = -4,     /* n_past + n_tokens > max_seq_len (src/s2_model.cpp:870-875) */
    S2K_ERR_STATE = -5,       /* missing tensors, model not finalized, ... */
    S2K_ERR_TIMEOUT = -6,     /* a bounded device-side wait gave up */
    S2K_ERR_UNSUPPORTED = -7, /* quant type / shape not supported */
    S2K_ERR_NO_DEVICE = -8    /* no CUDA device visible */
};

/* ggml type ids accepted by s2k_model_upload_tensor */
enum {
    S2K_TYPE_F32 = 0,
    S2K_TYPE_F16 = 1,
    S2K_TYPE_Q8_0 = 8,
    S2K_TYPE_Q4_K = 12,
    S2K_TYPE_Q6_K = 14
};

/* Mirrors s2::ModelHParams (include/s2_model.h:38-69) plus head_dim, which the
 * reference derives from q_norm / wo (src/s2_model.cpp:879-884). */
typedef struct s2k_hparams {
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
} s2k_hparams;

/* Mirrors s2::GenerateParams (include/s2_generate.h:23-32) and the
 * TokenizerConfig::im_end_id generate() reads (src/s2_generate.cpp:26).
 * seed / seq_id key the counter-based sampler RNG that replaces the
 * reference's std::random_device-seeded mt19937 (src/s2_sampler.cpp:94). */
typedef struct s2k_gen_params {
    int32_t max_new_tokens;
    float temperature;
    float top_p;
    int32_t top_k;
    int32_t min_tokens_before_end;
    int32_t im_end_id;
    uint64_t seed;
    uint32_t seq_id;
} s2k_gen_params;

/* Mirrors s2::FrameCallbackData + FrameCallback (include/s2_generate.h:14-21):
 * return non-zero to continue, 0 to abort generation. */
typedef int32_t (*s2k_frame_callback)(const int32_t *codes, int32_t frame_index,
                                      int32_t total_frames, int32_t num_codebooks, void *user);

typedef struct s2k_model s2k_model;
typedef struct s2k_seq s2k_seq;

S2K_API int32_t s2k_abi_version(void);
S2K_API const char *s2k_last_error(void);
S2K_API s2k_status s2k_device_count(int32_t *count);

/* Replaces SlowARModel::load_shared's ggml context, backends and schedulers
 * (src/s2_model.cpp:204-608): creates the model on CUDA device `device`. */
S2K_API s2k_status s2k_model_create(int32_t device, const s2k_hparams *hp, s2k_model **out);

/* Replaces the ggml_backend_tensor_set of one model tensor in
 * read_all_tensor_data (src/s2_pipeline.cpp:326-343).  `host` holds the GGUF
 * tensor bytes exactly as stored on disk (ggml ne order [in, out]); the
 * blocks are re-laid out on the device for coalesced 128-bit loads.  Names
 * are the GGUF names SlowARModel binds (src/s2_model.cpp:374-423). */
S2K_API s2k_status s2k_model_upload_tensor(s2k_model *m, const char *name, int32_t ggml_type,
                                           const int64_t ne[4], const void *host, size_t nbytes);

/* ---- GGUF files without ggml.  The reference reads the hyper-parameters
 * with gguf_get_val_* under the keys and defaults of SlowARModel::load_shared
 * (src/s2_model.cpp:245-288: "<general.architecture>.*" and "fish_speech.*")
 * and copies each model tensor's bytes from data_offset + offset
 * (read_all_tensor_data, src/s2_pipeline.cpp:306-389).  These do the same
 * with a reader of their own (GGUF v2 / v3). */

/* The model hyper-parameters of a GGUF file (host only, no device needed).
 * head_dim comes from layer 0's q_norm or wo shape (src/s2_model.cpp:879-884). */
S2K_API s2k_status s2k_gguf_read_hparams(const char *path, s2k_hparams *out);
/* Tensor `index` of a GGUF file: name (NUL-terminated, capacity name_cap),
 * ggml type, ne (unused dimensions 1), absolute file offset of its data and
 * its size in bytes (0 for a ggml type this path does not read).  Any output
 * may be NULL; *n_tensors gets the file's tensor count (index -1: count only). */
S2K_API s2k_status s2k_gguf_tensor_info(const char *path, int32_t index, char *name, size_t name_cap,
                                        int32_t *type, int64_t ne[4], uint64_t *offset, uint64_t *nbytes,
                                        int32_t *n_tensors);
/* Creates the model on `device` from a GGUF file: hyper-parameters as
 * s2k_gguf_read_hparams, every tensor the model binds uploaded (the codec's
 * and other tensors are skipped, as the reference leaves them to the codec),
 * then s2k_model_finalize. */
S2K_API s2k_status s2k_model_load_gguf(int32_t device, const char *path, s2k_model **out);

/* Checks every required tensor is bound (the req_t checks of
 * src/s2_model.cpp:366-428) and prepares the decode kernels.  For models with
 * Q4_K / Q6_K matrices in the Slow stack it also reserves two layer slots for
 * the int8 copies the tensor-core prefill reads (rebuilt one layer ahead
 * during each prefill of 64+ tokens): about two layers' weights in extra
 * device memory (twice that for Q6_K); s2k_model_weight_bytes does not count
 * them. */
S2K_API s2k_status s2k_model_finalize(s2k_model *m);
S2K_API void s2k_model_free(s2k_model *m);
/* SlowARModel::hparams (include/s2_model.h:130) */
S2K_API s2k_status s2k_model_get_hparams(const s2k_model *m, s2k_hparams *out);
/* Device bytes of the re-laid-out weights. */
S2K_API size_t s2k_model_weight_bytes(const s2k_model *m);
/* The cudaStream_t all of this model's work runs on (for event timing). */
S2K_API void *s2k_model_stream(s2k_model *m);

/* SlowARModel::init_kv_cache (src/s2_model.cpp:717-765): a sequence owning a
 * paged f16 KV cache (16-token pages) for up to max_seq_len positions. */
S2K_API s2k_status s2k_seq_create(s2k_model *m, int32_t max_seq_len, s2k_seq **out);
/* SlowARModel::reset (src/s2_model.cpp:767-769): n_past = 0. */
S2K_API s2k_status s2k_seq_reset(s2k_seq *s);
/* SlowARModel::clear_kv_cache (src/s2_model.cpp:771-787). */
S2K_API void s2k_seq_free(s2k_seq *s);
S2K_API int32_t s2k_seq_n_past(const s2k_seq *s);

/* Restores the sequence's KV cache from host memory: k and v hold n_pos
 * positions in the reference's cache layout, f16 [layer][pos][kv_head][head_dim]
 * (src/s2_model.cpp:746-747, with max_seq_len = n_pos), and n_past becomes
 * n_pos, as if those positions had been prefilled (the state prefill_fast
 * leaves, src/s2_model.cpp:788-791).  For a cached voice-clone prefix, and for
 * a step over a given cache.  Not for sequences of a scheduler. */
S2K_API s2k_status s2k_seq_load_kv(s2k_seq *s, const uint16_t *k, const uint16_t *v, int32_t n_pos);

/* SlowARModel::eval_cached, reached through prefill_fast / step
 * (src/s2_model.cpp:788-791, 855-1097).  flat_tokens is [n_tokens][num_codebooks+1]
 * token-major.  hidden_out [embedding_length] and logits_out [vocab_size] are
 * host buffers (either may be NULL). */
S2K_API s2k_status s2k_eval(s2k_model *m, s2k_seq *s, const int32_t *flat_tokens,
                            int32_t n_tokens, float *hidden_out, float *logits_out);

/* SlowARModel::fast_decode (src/s2_model.cpp:1099-1255): hidden [embedding_length],
 * prefix [n_prefix] codebook values, n_prefix < num_codebooks; logits_out
 * [codebook_size]. */
S2K_API s2k_status s2k_fast_decode(s2k_model *m, const float *hidden, const int32_t *prefix,
                                   int32_t n_prefix, float *logits_out);

/* s2::generate (src/s2_generate.cpp:11-216) with the frame loop on the device:
 * prompt is the PromptTensor grid [num_codebooks+1][cols] row-major
 * (include/s2_prompt.h:11-15); codes_out receives [num_codebooks][n_frames]
 * cb-major, compacted like src/s2_generate.cpp:201-213 (capacity
 * num_codebooks * max_new_tokens).  The sequence is reset first (the
 * clear/init_kv_cache the Pipeline does, src/s2_pipeline.cpp:838-851) and
 * must hold cols + max_new_tokens positions.
 * on_frame (may be NULL) is called on the calling thread for each frame as
 * soon as its codes reach host memory, while up to 3 later frames decode on
 * the device (src/s2_generate.cpp:150-163).  Returning 0 stops generation:
 * no further frame is launched, codes_out holds frames 0..frame_index, and
 * n_past is cols + frame_index, as in the reference, which breaks before the
 * aborted frame's step(). */
S2K_API s2k_status s2k_generate(s2k_model *m, s2k_seq *s, const int32_t *prompt, int32_t cols,
                                const s2k_gen_params *gp, int32_t *codes_out,
                                int32_t *n_frames_out, s2k_frame_callback on_frame, void *user);

/* The [Metrics] line generate() prints when verbose (src/s2_generate.cpp:185-199):
 * device time of the last s2k_generate / s2k_generate_device call on this
 * sequence (CUDA events on the model stream) -- prompt prefill, frame loop,
 * their sum and the loop time per frame -- with its frame and prompt counts.
 * The same calls also mark "s2k generate: prefill" and "s2k generate: frame
 * loop" as NVTX ranges for a profiler's timeline. */
typedef struct s2k_gen_metrics {
    double prefill_ms, loop_ms, total_ms, ms_per_frame;
    int32_t n_frames, prompt_tokens;
} s2k_gen_metrics;
S2K_API s2k_status s2k_seq_last_metrics(const s2k_seq *s, s2k_gen_metrics *out);

/* Same as s2k_generate with device-resident buffers: d_prompt_tm is the
 * token-major [cols][num_codebooks+1] prompt and d_codes_out the
 * [num_codebooks][max_new_tokens] (uncompacted) codes, both device pointers. */
S2K_API s2k_status s2k_generate_device(s2k_model *m, s2k_seq *s, const int32_t *d_prompt_tm,
                                       int32_t cols, const s2k_gen_params *gp,
                                       int32_t *d_codes_out, int32_t *n_frames_out);

/* Tokenizer callback for s2k_build_prompt: writes the token ids of `text`
 * (at most cap of them; ids may be NULL with cap 0 to ask for the count) and
 * returns how many the text encodes to, or a negative value on failure
 * (the reference's Tokenizer::encode, src/s2_tokenizer.cpp). */
typedef int32_t (*s2k_encode_fn)(const char *text, int32_t *ids, int32_t cap, void *user);

/* s2::build_prompt (src/s2_prompt.cpp:5-103): the PromptTensor grid
 * [num_codebooks+1][cols] row-major for a synthesis of `text`, voice-cloned
 * from a reference clip when prompt_codes ([num_codebooks][T_prompt]
 * cb-major), T_prompt > 0 and a non-empty prompt_text (its transcript) are
 * given: the system / user / assistant turns encoded by `encode`, the
 * reference codes under their semantic tokens (codebook 0 + semantic_begin_id)
 * and code rows that are zero elsewhere.  *rows / *cols get the grid shape;
 * with out NULL only the shape is computed (a size query). */
S2K_API s2k_status s2k_build_prompt(s2k_encode_fn encode, void *user, const char *text, const char *prompt_text,
                                    const int32_t *prompt_codes, int32_t num_codebooks, int32_t T_prompt,
                                    int32_t im_end_id, int32_t voice_id, int32_t semantic_begin_id, int32_t *out,
                                    size_t cap, int32_t *rows, int32_t *cols);

/* Sampler on the device for one logits row already in device memory
 * (s2::sample_token, src/s2_sampler.cpp:42-99; tie break = lowest index).
 * u is the uniform draw used when temperature > 0.  Host logits in, token out. */
S2K_API s2k_status s2k_sample(s2k_model *m, const float *logits, int32_t n, float temperature,
                              float top_p, int32_t top_k, double u, int32_t *token_out);

/* Largest logits row s2k_sample_noalloc accepts (its fixed device scratch). */
#define S2K_SAMPLE_NOALLOC_MAX_N 8192

/* Allocation-free variant of s2k_sample; it has no counterpart in the
 * reference.  Same arguments, result and tie break as s2k_sample, but it
 * allocates no device memory: the logits staging row, the result slot and
 * the error word live in one fixed file-scope device array of
 * S2K_SAMPLE_NOALLOC_MAX_N floats + 256 bytes (32.25 KiB) per device, which
 * every device that loads the library holds until exit.
 * n > S2K_SAMPLE_NOALLOC_MAX_N is rejected with S2K_ERR_ARG.
 * The first call on a device (and the first after a device reset) looks up
 * that array's address with that device current (set-up); make that first
 * call before any stream capture.  Every call copies the logits in, samples
 * and synchronizes the model stream to read the token.  The error word is
 * cleared on the model stream at the start of every call.  The scratch is
 * shared by every model on the device: calls that overlap in time (other
 * threads, other models on the same device) race on it and must be
 * serialised by the caller. */
S2K_API s2k_status s2k_sample_noalloc(s2k_model *m, const float *logits, int32_t n, float temperature,
                                      float top_p, int32_t top_k, double u, int32_t *token_out);

/* ggml_get_rows of a weight table on the device (the embedding gathers of
 * src/s2_model.cpp:941-962, 1150-1157): out [n][embedding_length] f32 gets
 * rows ids[0..n) of `table` ("embeddings.weight", "codebook_embeddings.weight",
 * "fast_embeddings.weight", "fast_output.weight") dequantized exactly as the
 * decode kernels read them (ggml dequantize_row_* per block). */
S2K_API s2k_status s2k_get_rows(s2k_model *m, const char *table, const int32_t *ids, int32_t n, float *out);

/* ---- Failure detection (no reference counterpart: the reference's ggml
 * waits have no bound).  Every wait of a kernel on data another CTA, copy
 * engine or launch produces is bounded; when the bound passes, the kernel
 * records the failure in the model's error word and returns, and the call
 * returns S2K_ERR_TIMEOUT with the model still usable. */

/* Bound of every device-side wait of this model's kernels, in SM clock cycles
 * (0 = the default, 4e9, about 2 s).  Takes effect for launches after it. */
S2K_API s2k_status s2k_model_set_wait_limit(s2k_model *m, int64_t cycles);
/* Launches one warp that waits, with the persistent kernel's bounded wait, for
 * an activation tag nobody writes.  Returns S2K_ERR_TIMEOUT once the wait
 * limit has passed (the path every timed-out wait takes). */
S2K_API s2k_status s2k_debug_wait_probe(s2k_model *m);
/* Test hook: y[i] = the device exp (det_expf, the exp of every softmax, SiLU
 * and sampler kernel) of x[i], i < n, on `device`; host arrays.  The CPU
 * oracle's so_det_expf returns the same bits. */
S2K_API s2k_status s2k_debug_det_expf(int32_t device, const float *x, float *y, int64_t n);
/* Test hook: the device allocation `after` allocations from now fails once
 * (as an out-of-memory error); a negative value disarms it. */
S2K_API s2k_status s2k_debug_fail_alloc(s2k_model *m, int64_t after);
/* Device bytes the model holds (weights, workspaces, sequences, schedulers). */
S2K_API size_t s2k_model_device_bytes(const s2k_model *m);
/* cudaMemGetInfo of a device. */
S2K_API s2k_status s2k_device_mem_info(int32_t device, size_t *free_bytes, size_t *total_bytes);

/* Profiling hook for the dominant kernel (no reference counterpart): launches
 * every Slow-step weight GEMV (per layer wqkv, wo, w1|w3, w2, then the LM head)
 * `reps` times back to back on the model stream, as the decode step issues
 * them, and reports the mean device time per pass and the weight bytes one
 * pass streams.  Activations are scratch; KV and sequences are untouched. */
S2K_API s2k_status s2k_profile_gemv(s2k_model *m, int32_t reps, double *bytes_per_pass,
                                    double *ms_per_pass, int32_t *launches_per_pass);

/* Profiling hook for the persistent decode kernel (no reference counterpart).
 * Needs a sequence that has run s2k_generate / s2k_generate_device (its frame
 * program is built) with n_past < max_seq_len.  Launches `reps` times (1..64)
 * the kernel's Fast-AR pass segment for codebook 1 and its Slow-step segment
 * without the n_past advance, each bracketed by CUDA events on the model
 * stream, and reports the mean device time of each and the algorithmic bytes
 * each streams (weights at 34/32 B per Q8_0 weight; the Slow segment adds the
 * f16 K/V of n_past cached positions).  The Slow segment rewrites the cache
 * slot at n_past, which the next step writes anyway; n_past is unchanged. */
S2K_API s2k_status s2k_profile_frame(s2k_model *m, s2k_seq *s, int32_t reps, double *ms_slow,
                                     double *ms_fast, double *bytes_slow, double *bytes_fast);

/* Profiling hook for the persistent decode kernel (no reference counterpart).
 * Same preconditions as s2k_profile_frame.  Launches segment `segment` of the
 * sequence's frame program `reps` times (1..64; segments 0..num_codebooks-2 are
 * the Fast-AR passes, the last is the Slow step without its n_past advance)
 * with an in-kernel trace: op i's time is from the grid barrier that releases
 * it to the one that releases op i+1, as CTA 0 sees them (globaltimer), so it
 * includes that op's barrier.  op_us[i] gets the mean in microseconds and
 * op_kind[i] the op kind (1 GEMV, 2 attention, 3 Slow embedding, 4 Fast
 * embedding); *n_ops the number of ops (at most cap). */
S2K_API s2k_status s2k_profile_ops(s2k_model *m, s2k_seq *s, int32_t segment, int32_t reps, double *op_us,
                                   int32_t *op_kind, int32_t cap, int32_t *n_ops);

/* Profiling hook for the persistent decode kernel (no reference counterpart).
 * Same preconditions as s2k_profile_ops.  Launches segment `segment` twice
 * with the in-kernel trace and returns the second launch's stamps:
 * stamps[((op * n_ctas) + cta) * 12 + k], globaltimer nanoseconds (0 where a
 * stamp does not apply), for op = 0..n_ops (the entry at op = n_ops is the
 * end of the launch, k = 0 only) and k = 0 op start (its grid barrier
 * released), 1 GEMV activation prologue done, 2 op work done; GEMV ops: 3 the
 * CTA's producer warp issued the op's last weight tile, 4 RMSNorm partial sums
 * formed, 5 RMSNorm scale known, 6 first weight tile ready, 7 activation
 * quantized (before the CTA barrier that ends the prologue); attention ops
 * (first unit of the CTA): 3 split arrival counted, 4 keys / values in shared
 * memory, 5 scores, 6 split softmax, 7 split values, 8 queries and this
 * call's keys rotated, 9 CTA barrier after them, 10 split partials written.
 * cap is the capacity of stamps in entries. */
S2K_API s2k_status s2k_profile_trace(s2k_model *m, s2k_seq *s, int32_t segment, uint64_t *stamps, size_t cap,
                                     int32_t *n_ops, int32_t *n_ctas);

/* Debugging aid (no reference counterpart): copies up to nbytes of a named
 * device buffer to host memory.  Names: "x", "h", "qkv", "attn", "ff",
 * "kcur", "vcur", "logits", "hidden" (Slow workspace), "fx", "fh", "fqkv",
 * "fattn", "fff", "flogits" (Fast workspace), "kv_k", "kv_v" (the sequence's
 * f16 KV pages, [page][layer][kv_head][16][head_dim]).  *copied gets the
 * number of bytes written. */
S2K_API s2k_status s2k_debug_copy(s2k_model *m, s2k_seq *s, const char *name, void *host,
                                  size_t nbytes, size_t *copied);

/* ---- Continuous batching (no reference counterpart: the reference runs one
 * synthesis at a time, src/s2_pipeline.cpp:781,810).  Sequences decode
 * together one frame per call: every live sequence's Fast-AR passes and Slow
 * step run as one set of batched kernels, so the weights stream once per
 * frame for the whole batch.  Batching changes no arithmetic: each
 * sequence's codes are the ones s2k_generate gives for the same prompt and
 * parameters (the sampling draws are keyed by seed, frame and seq_id). */

/* Prefill + first main token of s (generate(), src/s2_generate.cpp:37-60),
 * leaving it ready for s2k_batch_frame.  prompt / cols / gp as s2k_generate;
 * s must hold cols + max_new_tokens + 1 positions. */
S2K_API s2k_status s2k_seq_begin(s2k_model *m, s2k_seq *s, const int32_t *prompt, int32_t cols,
                                 const s2k_gen_params *gp);
/* One frame (src/s2_generate.cpp:123-182) for each unfinished sequence of
 * seqs[0..n) (sequences begun with s2k_seq_begin; finished ones are
 * skipped), as batched kernels.  *n_live (may be NULL) gets the number still
 * unfinished afterwards. */
S2K_API s2k_status s2k_batch_frame(s2k_model *m, s2k_seq *const *seqs, int32_t n, int32_t *n_live);
/* Codes of s so far, cb-major [num_codebooks][*n_frames] (capacity
 * cap_frames frames; codes_out may be NULL), and whether it finished. */
S2K_API s2k_status s2k_seq_frames(s2k_seq *s, int32_t *codes_out, int32_t cap_frames, int32_t *n_frames,
                                  int32_t *done);

/* A continuous-batching scheduler over independent utterances: a FIFO of
 * requests, up to max_batch live sequences decoded together, and one paged
 * f16 KV pool (16-token pages, pool_pages of them; 0 = max_batch full-length
 * sequences) shared by all of them.  A request is admitted when a slot and
 * the pages for its prompt + max_new_tokens + 1 positions are free, is
 * prefilled, joins the next batched frame, and leaves the batch (its pages
 * back in the pool) when it stops (im_end or max_new_tokens). */
typedef struct s2k_sched s2k_sched;
/* Request states.  FAILED: admission failed for this request alone (no
 * memory for it, bad input; s2k_sched_poll_status gives the status) and the
 * scheduler went on with the others.  CANCELLED: stopped by s2k_sched_cancel
 * or by the frame callback; it keeps the frames it had. */
enum { S2K_REQ_WAITING = 0, S2K_REQ_LIVE = 1, S2K_REQ_DONE = 2, S2K_REQ_FAILED = 3, S2K_REQ_CANCELLED = 4 };
typedef struct {
    int64_t steps;           /* batched frames run */
    int64_t frames;          /* frames produced, all requests */
    int64_t prefill_tokens;  /* prompt positions prefilled */
    int64_t admitted, finished;
    int64_t kv_positions;    /* cached positions the batched Slow steps attended over */
    int32_t max_live;        /* largest batch so far */
    int32_t free_pages, pool_pages;
    int32_t pad_;
    int64_t cancelled, failed;
} s2k_sched_stats;
/* Called after each batched frame for each frame a live request produced
 * (the streaming hand-off of src/s2_generate.cpp:150-163 per request);
 * returning 0 cancels that request. */
typedef int32_t (*s2k_sched_frame_callback)(int32_t req_id, const int32_t *codes, int32_t frame_index,
                                            int32_t num_codebooks, void *user);
S2K_API s2k_status s2k_sched_create(s2k_model *m, int32_t max_batch, int32_t max_seq_len, int32_t pool_pages,
                                    s2k_sched **out);
S2K_API void s2k_sched_free(s2k_sched *sc);
/* Queue a request (prompt / cols / gp as s2k_generate); *req_id numbers
 * requests 0, 1, ... in submission order. */
S2K_API s2k_status s2k_sched_submit(s2k_sched *sc, const int32_t *prompt, int32_t cols, const s2k_gen_params *gp,
                                    int32_t *req_id);
/* Admit what fits, run one batched frame over the live requests, retire the
 * finished ones. */
S2K_API s2k_status s2k_sched_step(s2k_sched *sc, int32_t *n_live, int32_t *n_waiting);
/* s2k_sched_step until no request is live or waiting. */
S2K_API s2k_status s2k_sched_run(s2k_sched *sc);
S2K_API s2k_status s2k_sched_poll(s2k_sched *sc, int32_t req_id, int32_t *state, int32_t *n_frames);
/* s2k_sched_poll plus the status a FAILED request failed with (S2K_OK otherwise). */
S2K_API s2k_status s2k_sched_poll_status(s2k_sched *sc, int32_t req_id, int32_t *state, int32_t *n_frames,
                                         s2k_status *req_status);
/* Stops a request between frames (the reference cancels through on_frame,
 * src/s2_pipeline.cpp:1102-1105): a waiting one leaves the queue, a live one
 * leaves the batch with the frames it has and its KV pages go back to the
 * pool.  A finished request is left as it is. */
S2K_API s2k_status s2k_sched_cancel(s2k_sched *sc, int32_t req_id);
/* Per-frame hand-off for every request (cb may be NULL to turn it off). */
S2K_API s2k_status s2k_sched_set_frame_callback(s2k_sched *sc, s2k_sched_frame_callback cb, void *user);
/* Codes of a finished (or cancelled) request, cb-major [num_codebooks][*n_frames]. */
S2K_API s2k_status s2k_sched_result(s2k_sched *sc, int32_t req_id, int32_t *codes_out, int32_t cap_frames,
                                    int32_t *n_frames);
S2K_API s2k_status s2k_sched_get_stats(const s2k_sched *sc, s2k_sched_stats *out);

/* Counts kernel launches issued by the library since the last reset. */
S2K_API uint64_t s2k_launch_count(int32_t reset);

/* ---- codec decode: codes -> audio (s2::AudioCodec, include/s2_codec.h) ----
 *
 * The DAC-style decoder the reference runs after generation: RVQ lookup and
 * projection, the windowed post-module transformer, ConvTranspose + ConvNeXt
 * upsampling, and the snake / residual-unit decoder
 * (src/s2_codec.cpp:264-522, AudioCodec::decode :1297-1447).  Matrices are
 * F16 as the reference's GGUF exports keep them; the arithmetic follows the
 * reference's ggml graph (fp16-rounded operands for the F16 matrix products
 * and the im2col convolutions, f32 for the transposed convolutions) with f32
 * accumulation on the tensor cores, so audio agrees with the CPU oracle to a
 * floating-point tolerance, not bit for bit. */

/* The fish_speech.codec.* keys AudioCodec::load_shared reads
 * (src/s2_codec.cpp:813-858); n_local_heads < 1 means n_head. */
typedef struct s2k_codec_hparams {
    int32_t sample_rate, hop_length;
    int32_t latent_dim, decoder_dim;
    int32_t n_decoder_rates, decoder_rates[8];
    int32_t quantizer_input_dim, quantizer_codebook_dim;
    int32_t quantizer_residual_codebooks, quantizer_residual_codebook_size, quantizer_semantic_codebook_size;
    int32_t n_downsample, quantizer_downsample_factor[8];
    int32_t rvq_window_size, rvq_block_size, rvq_n_layer, rvq_n_local_heads, rvq_head_dim, rvq_dim;
    float rvq_rope_base, rvq_norm_eps;
} s2k_codec_hparams;

typedef struct s2k_codec s2k_codec;

/* AudioCodec construction: s2k_codec_create + one upload per tensor (GGUF
 * name, with or without the combined file's "c." prefix; F16 or F32; the
 * bytes are copied) + s2k_codec_finalize, which builds the device layouts. */
S2K_API s2k_status s2k_codec_create(int32_t device, const s2k_codec_hparams *hp, s2k_codec **out);
S2K_API s2k_status s2k_codec_upload_tensor(s2k_codec *c, const char *name, int32_t ggml_type, const int64_t ne[4],
                                           const void *data, size_t nbytes);
S2K_API s2k_status s2k_codec_finalize(s2k_codec *c);
/* AudioCodec::load (src/s2_codec.cpp:698-900): hyper-parameters and the
 * codec tensors of a combined ("fish-speech", "c." names) or codec-only
 * ("fish-speech-codec") GGUF. */
S2K_API s2k_status s2k_codec_load_gguf(int32_t device, const char *path, s2k_codec **out);
S2K_API void s2k_codec_free(s2k_codec *c);
S2K_API s2k_status s2k_codec_get_hparams(const s2k_codec *c, s2k_codec_hparams *out);
/* AudioCodec::samples_per_code_frame / streaming_history_frames / num_codebooks
 * (include/s2_codec.h:40-45, src/s2_codec.cpp:858-874) */
S2K_API int32_t s2k_codec_samples_per_frame(const s2k_codec *c);
S2K_API int32_t s2k_codec_history_frames(const s2k_codec *c);
S2K_API int32_t s2k_codec_num_codebooks(const s2k_codec *c);
/* Frames before the first sample a window emits that the decoder stages
 * (everything after the post-module transformer) must see for that sample to
 * equal a decode of the whole window; derived from the kernel sizes,
 * dilations and strides at finalize. */
S2K_API int32_t s2k_codec_receptive_frames(const s2k_codec *c);

/* AudioCodec::decode (src/s2_codec.cpp:1297-1447): codes [num_codebooks]
 * [n_frames] cb-major (clamped into each codebook as sanitize_decode_codes
 * does) -> n_frames * samples_per_frame samples in audio (capacity cap). */
S2K_API s2k_status s2k_codec_decode(s2k_codec *c, const int32_t *codes, int32_t n_frames, float *audio, size_t cap,
                                    int64_t *n_samples);
/* One window of the windowed decode: the samples of frames
 * [emit_begin, emit_end) of a decode of the n_frames-frame window, into
 * audio.  Only what those samples depend on is computed: the transformer over
 * frames [0, emit_end) (it is causal) and the decoder stages from
 * emit_begin - receptive_frames on; the samples are those of the whole-window
 * decode. */
S2K_API s2k_status s2k_codec_decode_range(s2k_codec *c, const int32_t *codes, int32_t n_frames, int32_t emit_begin,
                                          int32_t emit_end, float *audio, size_t cap, int64_t *n_samples);
/* decode_codes_windowed (src/s2_pipeline.cpp:198-289), the offline
 * synthesis decode: windows every stride_frames (<= 0: 16) frames with
 * context_frames_override (< 0: s2k_codec_history_frames) frames of history;
 * codes [num_codebooks][total_frames].  decode_ms: device time of the window
 * decodes; decode_batches: windows decoded (either may be NULL). */
S2K_API s2k_status s2k_codec_decode_windowed(s2k_codec *c, const int32_t *codes, int32_t total_frames,
                                             int32_t num_codebooks, int32_t stride_frames,
                                             int32_t context_frames_override, float *audio, size_t cap,
                                             int64_t *n_samples, double *decode_ms, int32_t *decode_batches);

/* Streaming decode (decode_window_and_emit and the on_frame trigger of
 * Pipeline::synthesize_stream, src/s2_pipeline.cpp:1011-1115): frames are
 * pushed one at a time as generation produces them; a window is decoded
 * once stride_frames (<= 0: 4) frames arrived since the last decode, holding
 * back holdback_frames (< 0: the context) frames, with context_frames
 * (< 0: s2k_codec_history_frames) of history.  push / finish return the PCM
 * the window released (possibly none). */
typedef struct s2k_codec_stream s2k_codec_stream;
S2K_API s2k_status s2k_codec_stream_create(s2k_codec *c, int32_t stride_frames, int32_t context_frames,
                                           int32_t holdback_frames, s2k_codec_stream **out);
S2K_API void s2k_codec_stream_free(s2k_codec_stream *s);
/* frame_codes: [num_codebooks] codes of one frame (the on_frame payload) */
S2K_API s2k_status s2k_codec_stream_push(s2k_codec_stream *s, const int32_t *frame_codes, float *pcm, size_t cap,
                                         int64_t *n_pcm);
S2K_API s2k_status s2k_codec_stream_finish(s2k_codec_stream *s, float *pcm, size_t cap, int64_t *n_pcm);
/* PCM samples the next push / finish can release at most (capacity to give). */
S2K_API int64_t s2k_codec_stream_max_release(const s2k_codec_stream *s);

#ifdef __cplusplus
}
#endif
#endif /* S2K_H */
