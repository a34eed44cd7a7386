// s2k_mega.h -- op descriptors of the persistent decode kernel (internal).
//
// A "segment" is a list of ops (a Fast-AR pass, or the Slow-AR step) run by
// one cooperative launch of mega_kernel: one CTA per SM, a producer warp that
// streams the weights of every GEMV op of the segment in order through a
// shared-memory ring, and consumer warps that run the ops one after another
// with a grid barrier between them.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "s2k_kernels.h"

namespace s2k {

enum MegaKind : int {
    MK_GEMV = 1,
    MK_ATTN = 2,
    MK_EMBED_SLOW = 3,
    MK_EMBED_FAST = 4,
    MK_ADVANCE = 5,
};

using MegaGemv = TGemv;  // s2k_tgemv.cuh

// Most query heads per kv head the persistent kernel's attention takes; its
// split arrival counters are kept per (layer, token, kv head, head block of
// up to this many blocks).
constexpr int kAttnMaxGroup = 4;

// Activations the persistent kernel passes between ops (x, h, qkv, attention
// output, SwiGLU output) are tagged 8-byte words (s2k_tgemv.cuh ll_pack);
// the *_tag fields hold the index, within the segment, of the op that writes
// the words an op reads or writes (the kernel adds the launch epoch).
struct MegaAttn {
    void *qkv;   // [T][ldqkv] raw projections (tagged words)
    uint32_t in_tag, out_tag;
    int ldqkv, T, H, Hkv, hd;
    const float *q_norm, *k_norm;
    float eps, scale;
    const float2 *rope;
    int rope_positions;
    const int *pos_base;  // device n_past (Slow) or null
    int pos_add;          // position of token 0 = *pos_base + pos_add
    int n_cached_from_pos_base;  // 1: keys < *pos_base come from the paged cache
    float *kcur, *vcur;   // f32 [positions][Hkv][hd]; index = cur_base + t
    int cur_base;
    __half *kv_k, *kv_v;  // paged f16 cache [page][layer][kv_head][16][hd] (Slow only)
    const int *block_table;
    int kv_layers, kv_pages;
    int layer;
    // split partials: per (token, kv head, split) O_i [group][hd] and
    // (m_i, S_i) [group][2], kAttnSplit keys per split; arrival counters per
    // (token, kv head), zero between ops (the combining unit resets them)
    double *part, *part_ms;
    int *counters;
    int n_split_max;
    void *out;            // [T][H*hd] (tagged words)
};

struct MegaEmbedSlow {
    const uint8_t *e;  // token embeddings (tiles of weight type etype), [e_rows][dim]
    int etype, e_rows, dim;
    const uint8_t *c;  // codebook embeddings (tiles of weight type ctype), [c_rows][dim]
    int ctype, c_rows;
    const int *tokens;  // [T][ncb+1]
    int T, ncb, cb_size, sem_begin, sem_end, scale_cb;
    float sem_scale;
    void *x;  // tagged words
    uint32_t tag;
};

struct MegaEmbedFast {
    const uint8_t *f;  // fast_embeddings (tiles of weight type ftype), [f_rows][dim]
    int ftype, f_rows;
    const float *hidden;  // null: no hidden row
    const int *codes;
    int code0, n_rows, dim;
    void *x;  // tagged words
    uint32_t tag;
};

struct MegaAdvance {
    int *n_past;
    int T;
};

struct MegaOp {
    int kind;
    int pad_;
    union {
        MegaGemv g;
        MegaAttn a;
        MegaEmbedSlow es;
        MegaEmbedFast ef;
        MegaAdvance adv;
    };
};

// Counters of one segment launch (zeroed before the launch): count = CTAs
// that finished (the last one advances the model's tag epoch), pad[0] = CTAs
// that reached the n_past advance.
struct MegaCtl {
    unsigned int count;
    unsigned int pad[31];
};

cudaError_t mega_setup();
// Launch one segment: ops in device memory, ctl zeroed on `st` before.
// trace (optional, (n_ops + 1) x grid x kTraceSlots entries): per op and CTA
// the globaltimer (ns) at [0] op start (the grid barrier after the previous op
// has released), [1] GEMV prologue done, [2] op work done, [3] the producer's
// last weight tile of the op issued, [4] RMSNorm partial sums formed (the
// activation loads have landed), [5] RMSNorm scale known, [6] first weight
// tile ready for the consumers, [7] activation quantized (before the CTA
// barrier that ends the prologue); attention ops use [3..10] for their phases
// (see mega_attn); entry [n_ops][cta][0] is taken after a final
// grid barrier.  Slots a launch does not reach stay as they were.
constexpr int kTraceSlots = 12;
cudaError_t launch_mega(const MegaOp *d_ops, int n_ops, int mt, MegaCtl *ctl, const int *done, int *err, int num_sms,
                        cudaStream_t st, unsigned *epoch, bool q8, unsigned long long *trace = nullptr);
// Tiles per CTA the producer keeps in flight into L2 beyond its ring.
int mega_l2_ahead();
// Host-side validation of a GEMV op for the persistent kernel.
bool mega_gemv_ok(const MegaGemv &g);
// One warp waits (bounded by the model's wait limit) for a tag nobody writes
// on the tagged words at `words` (32-byte aligned, read only); sets ERR_GRID.
cudaError_t launch_wait_probe(const uint64_t *words, int *err, cudaStream_t st);
// Host-side validation of an attention op; max_keys bounds any token's key range.
bool mega_attn_ok(const MegaAttn &a, int max_keys);

}  // namespace s2k
