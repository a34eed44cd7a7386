// s2k_mega.cu -- persistent decode kernel: one cooperative launch runs a whole
// segment of the decode step (a Fast-AR pass, or the Slow-AR step) on one CTA
// per SM.
//
// Why: at batch 1 every op is a short, memory-bound GEMV (1.6-8 us of HBM
// time for the per-layer matrices).  Launched as separate kernels, each op
// pays launch, dependency and prologue latency while HBM idles.  Here a
// producer warp per CTA streams the CTA's rows of every GEMV of the segment,
// back to back, as 17 KB weight tiles through a 10-stage shared-memory ring
// (cp.async.bulk + mbarriers); it runs ahead across op boundaries, so HBM keeps streaming while
// the consumer warps wait at a grid barrier, normalize and quantize the next
// activation, or run attention.
//
// Arithmetic is identical to the standalone kernels (s2k_gemv.cu,
// s2k_attn.cu): Q8_0 activation quantization, exact block terms summed in
// double, exact softmax with det_expf -- so results match the CPU oracle bit
// for bit.
#include "s2k_common.cuh"
#include "s2k_kernels.h"
#include "s2k_mega.h"

#include <algorithm>
#include <cstddef>
#include <cstdlib>

namespace s2k {

// 8 consumer warps (the tile engine's mapping, s2k_tgemv.cuh) + the producer warp + a helper warp.
constexpr int kMW = kTW;                   // consumer warps
constexpr int kMNC = kMW * 32;             // consumer threads
constexpr int kMThreads = kMNC + 64;       // + producer warp + helper warp (attention K/V prefetch)
constexpr int kMStages = 10;               // ring of 17 KB weight tiles
constexpr int kMaxPL = 4;                  // tiles the producer warp issues per group (one per lane)
constexpr int kMKMax = 10240;
constexpr int kMaxT = 2;
constexpr int kHD = 128;
constexpr int kPtab = 512;                 // cached pages whose ids are staged in shared memory
constexpr int kMPC = 5;                    // 8-value activation chunks per consumer thread per prologue pass

bool mega_gemv_ok(const MegaGemv &g) {
    if (g.wtype != TW_Q8_0 && g.wtype != TW_Q4_K && g.wtype != TW_Q6_K && g.wtype != TW_F16) return false;
    if (!tg_shape_ok(g.R, g.K, g.M, g.in_mode, g.epi, g.res != nullptr, kMKMax, kMaxT)) return false;
    if (g.in_mode == IN_RMSNORM && g.norm_w == nullptr) return false;
    // one-pass RMSNorm prologue; 32-byte activation and norm-weight loads
    if (g.in_mode == IN_RMSNORM && g.M * g.K > 8 * kMPC * kMNC) return false;
    if (g.ldx % 8 != 0 || reinterpret_cast<uintptr_t>(g.x) % 32 != 0) return false;
    if (g.act_out != nullptr && reinterpret_cast<uintptr_t>(g.act_out) % 16 != 0) return false;
    if (g.norm_w != nullptr && reinterpret_cast<uintptr_t>(g.norm_w) % 32 != 0) return false;
    return true;
}

constexpr int kAG = kAttnMaxGroup;  // most query heads per kv head (register arrays of a unit)
constexpr int kAF32 = 32;  // most f32 key rows of a unit (Fast-AR context)
constexpr int kCombineFast = 8;  // splits the combining unit reads in one round trip

// Attention unit buffers: the split's keys and values (f16 cache pages of the
// Slow step, or f32 rows of the Fast-AR), this call's rotated keys/values
// (Slow), the group's rotated queries as doubles (quarter rows padded so the
// four quarters of a key read different banks), the split's
// scores and exponentials, and the upper-half value partials.
struct AttnSm {
    union KV {
        __half h[kAttnSplit][kHD];
        float f[kAF32][kHD];
    };
    alignas(128) KV k;
    alignas(128) KV v;
    alignas(16) float kc[kMaxT][kHD];
    alignas(16) float vc[kMaxT][kHD];
    alignas(16) double q[kAG][4][34];  // quarter rows padded to 34: 16-byte loads, four banks apart
    float s[kAG][kAttnSplit];
    alignas(16) double e[kAttnSplit][kAG];  // exponentials, the group's heads side by side
    double o[kAG][kHD];
    float m[kAG];
    double S[kAG];
    int last;
};

bool mega_attn_ok(const MegaAttn &a, int max_keys) {
    if (a.hd != kHD || a.Hkv < 1 || a.H % a.Hkv != 0 || a.H / a.Hkv > kAG || a.T < 1 || a.T > kMaxT) return false;
    if (a.part == nullptr || a.part_ms == nullptr || a.counters == nullptr) return false;
    if ((max_keys + kAttnSplit - 1) / kAttnSplit > a.n_split_max) return false;
    if (a.kv_k == nullptr) {  // Fast-AR: every key an f32 row of one split
        if (a.cur_base + a.T > kAF32 || a.cur_base + a.T > kAttnSplit || a.n_cached_from_pos_base) return false;
    } else if (a.cur_base != 0) {
        return false;
    }
    return true;
}

struct GemvSm {
    // quantized activation (int8), or the fp16 activation of F16 weights
    // (2 bytes per value, spilling over xd / xbs, which F16 does not use)
    alignas(16) int8_t xq[kMaxT * kMKMax];
    float xd[kMaxT * kMKMax / 32];  // Q8_0 block scales, or Q8_K super-block scales
    int16_t xbs[kMaxT * kMKMax / 16];  // Q8_K block sums
    int8_t xh_rest[kMaxT * kMKMax * 3 / 4];  // the rest of the fp16 activation
};
static_assert(offsetof(GemvSm, xd) == kMaxT * kMKMax && offsetof(GemvSm, xh_rest) + sizeof(GemvSm::xh_rest) >=
                                                            (size_t)2 * kMaxT * kMKMax,
              "fp16 activation fits xq .. xh_rest");

struct MSmem {
    uint8_t ring[kMStages][kTileBytes];
    uint64_t full[kMStages], empty[kMStages];
    uint64_t abar;  // K/V page copies of an attention unit
    alignas(128) union {
        GemvSm g;
        AttnSm a;
    } u;
    double tok[kMW][kMaxT];
    int ptab[kPtab];  // page ids of the sequence's first kPtab pages (Slow segment)
    int ptab_ready;
    int cur_op;  // op the consumers are running (written by consumer thread 0, read by the helper warp)
};

static_assert(sizeof(MSmem) <= 227 * 1024, "persistent kernel shared memory exceeds the per-CTA limit");
// shared arrays read with vector loads or written by bulk copies
static_assert(offsetof(MSmem, ring) % 16 == 0 && kTileBytes % 16 == 0, "ring alignment");
static_assert(offsetof(MSmem, u) % 128 == 0, "activation / key buffer alignment");
static_assert(sizeof(AttnSm::KV) == kAttnSplit * kHD * sizeof(__half) && kAttnSplit % kPage == 0,
              "a split's cache pages fill the key buffer");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Units of an attention op: one per (token, kv head, head block, split of
// kAttnSplit keys).  A head block is nh query heads of the kv head's group:
// the fewest heads per unit (1, 2 or the whole group) that still give every
// unit a CTA of its own, so a short context spreads over more SMs and each
// unit does less of the double-precision score and value work.  Every head's
// arithmetic is the same whatever the block size (scores, split softmax and
// split partials are per head).  All CTAs of a launch read the same n_past
// (it advances only after every CTA has finished the segment's ops), so they
// agree on the plan.
struct AttnPlan {
    int nc, pos0, nspl, nh, nhb, units;
};

__device__ __forceinline__ AttnPlan attn_plan(const MegaAttn &a, int G) {
    AttnPlan p;
    const int base = a.pos_base ? __ldcg(a.pos_base) : 0;
    p.nc = a.n_cached_from_pos_base ? base : 0;
    p.pos0 = base + a.pos_add;
    p.nspl = (p.nc + a.cur_base + a.T + kAttnSplit - 1) / kAttnSplit;
    const int grp = a.H / a.Hkv;
    const int per = a.T * a.Hkv * p.nspl;  // units per head block
    if (per * grp <= G) {
        p.nh = 1;
    } else if (grp % 2 == 0 && per * (grp / 2) <= G) {
        p.nh = 2;
    } else {
        p.nh = grp;
    }
    p.nhb = grp / p.nh;
    p.units = per * p.nhb;
    return p;
}

struct AttnUnit {
    int t, g, hb, i;
};

__device__ __forceinline__ AttnUnit attn_unit_of(const MegaAttn &a, const AttnPlan &p, int u) {
    AttnUnit x;
    const int per_t = a.Hkv * p.nhb * p.nspl, per_g = p.nhb * p.nspl;
    x.t = u / per_t;
    int r = u - x.t * per_t;
    x.g = r / per_g;
    r -= x.g * per_g;
    x.hb = r / p.nspl;
    x.i = r - x.hb * p.nspl;
    return x;
}

// 4 tagged activation words at element i of base (32-byte aligned), polled
// until their tags are current (see ll_load8).
__device__ __forceinline__ float4 ll_wait4(const void *base, size_t i, uint32_t tag, int *err) {
    const uint64_t *q = reinterpret_cast<const uint64_t *>(base) + i;
    uint64_t w0, w1, w2, w3;
    auto load = [&]() {
        asm volatile("ld.global.cg.v4.u64 {%0,%1,%2,%3}, [%4];" : "=l"(w0), "=l"(w1), "=l"(w2), "=l"(w3) : "l"(q));
        return (uint32_t)(w0 >> 32) == tag && (uint32_t)(w1 >> 32) == tag && (uint32_t)(w2 >> 32) == tag &&
               (uint32_t)(w3 >> 32) == tag;
    };
    if (!load()) {
        const long long t0 = clock64(), lim = wait_limit(err);
        for (unsigned it = 1; !load(); ++it) {
            if (clock64() - t0 > lim ||
                (it % kErrPollEvery == 0 && (*reinterpret_cast<volatile int *>(err) & ERR_GRID))) {
                atomicOr(err, ERR_GRID);
                break;
            }
        }
    }
    return make_float4(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1), __uint_as_float((uint32_t)w2),
                       __uint_as_float((uint32_t)w3));
}

// ---------------------------------------------------------------------------
// producer: the weight tiles of every GEMV op of the segment, in op order
// ---------------------------------------------------------------------------
// Walks this CTA's weight tiles of a segment in the order the consumers use
// them (GEMV ops in op order, each op's tile range in address order).
struct TileCursor {
    int op = -1;
    long long u = 0, u1 = 0;
    const uint8_t *w = nullptr;
    uint32_t bytes = 0;  // tile size of the current op's weight type

    __device__ __forceinline__ const uint8_t *next(const MegaOp *ops, int n_ops, int cta, int G) {
        while (u >= u1) {
            if (++op >= n_ops) return nullptr;
            if (ops[op].kind != MK_GEMV) continue;
            tg_range(ops[op].g.R, ops[op].g.K, ops[op].g.wtype, cta, G, &u, &u1);
            w = ops[op].g.w;
            bytes = (uint32_t)tile_bytes(ops[op].g.wtype);
        }
        return w + (size_t)(u++) * bytes;
    }
};

// The ring holds kMStages tiles; a second cursor runs `l2_ahead` tiles past
// the ring's head and pulls those tiles into L2 with bulk prefetches, so HBM
// keeps streaming while the consumers sit in a grid barrier, an activation
// prologue or attention (the ring alone covers ~4 us of HBM time per SM).
//
// Run by the whole producer warp, in groups of up to `lanes` tiles: lane 0
// walks the cursors and checks the ring once per group (it waits for the
// group's last slot to be free, which frees the earlier ones too, since the
// consumers release tiles in order), then lanes 0..n-1 each arm one slot and
// issue its bulk copy in the same instruction.  One lane issuing every copy
// alone held a CTA to ~560 SM cycles per 17 KB tile even with the tiles in
// L2; four lanes per group bring it to ~450, where the consumer warps'
// shared-memory reads and block arithmetic bound it.
__device__ void mega_producer(const MegaOp *ops, int n_ops, MSmem &sm, int cta, int G, int l2_ahead, int depth,
                              int lanes, int *err, unsigned long long *trace) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = policy_evict_first();
    if (n_ops > 0 && ops[0].kind == MK_EMBED_SLOW) {
        // The Slow step's embedding gathers rows the sampler chose an instant
        // ago (three dependent memory round trips); 25 MB of weight tiles issued
        // at launch would queue ahead of each of them.  Start the stream once
        // the consumers have moved on to the first GEMV.
        const volatile int *cur = &sm.cur_op;
        const long long t0 = clock64(), lim = wait_limit(err);
        while (*cur < 1) {
            if (clock64() - t0 > lim) return;  // the consumers stopped (their error is reported)
            __nanosleep(64);
        }
    }
    // a group never needs a slot whose previous tile is in the same group
    const int gmax = max(1, min(min(lanes, kMaxPL), depth));
    TileCursor ld, pf;
    long long pf_n = 0;  // tiles the prefetch cursor has passed
    // the first kMStages tiles go straight into the empty ring
    if (lane == 0)
        for (int i = 0; i < kMStages && pf.next(ops, n_ops, cta, G); ++i) ++pf_n;
    for (long long ps = 0;;) {
        const uint8_t *srcs[kMaxPL];
        uint32_t bytes[kMaxPL];
        int endop[kMaxPL];  // op whose last tile is tile j of the group, or -1 (trace)
#pragma unroll
        for (int j = 0; j < kMaxPL; ++j) {
            srcs[j] = nullptr;
            bytes[j] = 0;
            endop[j] = -1;
        }
        int n = 0;  // tiles in this group
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < kMaxPL; ++j) {
                if (j < gmax && n == j && (srcs[j] = ld.next(ops, n_ops, cta, G)) != nullptr) {
                    bytes[j] = ld.bytes;
                    ++n;
                    if (ld.u == ld.u1) endop[j] = ld.op;
                }
            }
            for (const uint8_t *p; pf_n < ps + n - 1 + kMStages + l2_ahead && (p = pf.next(ops, n_ops, cta, G)) != nullptr;
                 ++pf_n)
                bulk_prefetch_l2(p, pf.bytes);
        }
        n = __shfl_sync(0xffffffffu, n, 0);
        if (n == 0) return;
        // at most `depth` tiles in flight: tile ps + j may start once tile
        // ps + j - depth has been consumed; waiting for the group's last such
        // tile covers the others
        const long long q = ps + n - 1 - depth;
        int ok = 1;
        if (q >= 0 && lane == 0)
            ok = mbar_wait(&sm.empty[q % kMStages], (uint32_t)(q / kMStages) & 1u, err, ERR_WAIT_EMPTY);
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
        const uint8_t *src = nullptr;
        uint32_t nb = 0;
#pragma unroll
        for (int j = 0; j < kMaxPL; ++j) {
            const uint8_t *s = reinterpret_cast<const uint8_t *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(srcs[j]), 0));
            const uint32_t b = __shfl_sync(0xffffffffu, bytes[j], 0);
            if (lane == j) {
                src = s;
                nb = b;
            }
        }
        if (lane < n) {
            const int slot = (int)((ps + lane) % kMStages);
            mbar_arrive_expect_tx(&sm.full[slot], nb);
            bulk_g2s(sm.ring[slot], src, nb, &sm.full[slot], pol);
        }
        if (trace != nullptr && lane == 0) {
            const unsigned long long now = globaltimer_ns();
#pragma unroll
            for (int j = 0; j < kMaxPL; ++j)
                if (endop[j] >= 0) trace[((size_t)endop[j] * G + cta) * kTraceSlots + 3] = now;
        }
        ps += n;
    }
}

// ---------------------------------------------------------------------------
// helper warp: K/V pages of the next attention op -> L2
// ---------------------------------------------------------------------------
// The cache pages an attention unit reads do not depend on the layer's QKV
// projection, only the current token's row does.  When the consumers start
// the op before a Slow attention op (its QKV GEMV), one lane pulls the pages
// of this CTA's attention units into L2, so the unit's bulk copies do not
// queue behind the weight stream in HBM.
__device__ void mega_kv_prefetch(const MegaOp *ops, int n_ops, MSmem &sm, int cta, int G, const int *err) {
    volatile int *cur = &sm.cur_op;
    const long long lim = wait_limit(err);
    for (int j = 1; j < n_ops; ++j) {
        if (ops[j].kind != MK_ATTN || ops[j].a.kv_k == nullptr) continue;
        const long long t0 = clock64();
        while (*cur < j - 1) {
            if (clock64() - t0 > lim) return;  // the consumers stopped (their error is reported)
            __nanosleep(256);
        }
        const MegaAttn &a = ops[j].a;
        const AttnPlan pl = attn_plan(a, G);
        const int nc = pl.nc;
        for (int u = cta; u < pl.units; u += G) {
            const AttnUnit un = attn_unit_of(a, pl, u);
            const int t = un.t, g = un.g, i = un.i;
            const int j0 = i * kAttnSplit, cnt = min(kAttnSplit, nc + a.cur_base + t + 1 - j0);
            const int ncp = max(0, min(cnt, nc - j0));
            for (int p = 0; p < (ncp + kPage - 1) / kPage; ++p) {
                const int page = __ldcg(a.block_table + j0 / kPage + p);
                const size_t off = (((size_t)page * a.kv_layers + a.layer) * a.Hkv + g) * kPage * kHD;
                bulk_prefetch_l2(a.kv_k + off, kPage * kHD * sizeof(__half));
                bulk_prefetch_l2(a.kv_v + off, kPage * kHD * sizeof(__half));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// GEMV op (consumer side): activation prologue, then this CTA's tiles
// ---------------------------------------------------------------------------
// Q8: every GEMV of the launch is Q8_0 (the kernel then carries only that
// consumer, which keeps its code compact).
template <int MT, bool Q8>
__device__ void mega_gemv(const MegaGemv &gref, const F8 (&nw)[kMPC], MSmem &sm, int cta, int G, int &slot,
                          uint32_t &phase, int *err, unsigned long long *tr, uint32_t ep8) {
    MegaGemv g = gref;  // op fields in registers; the op list holds producer op indices, the launch its epoch
    g.x_tag |= ep8;
    g.res_tag |= ep8;
    g.y_tag |= ep8;
    long long u0, u1;
    tg_range(g.R, g.K, g.wtype, cta, G, &u0, &u1);
    if (u0 == u1) return;  // no row tile of this op here (R / 32 < G)
    // the CTA owning row tile 0 stores act_out
    tg_prologue8<MT, kMNC, kMPC, Q8>(g, nw, sm.u.g.xq, sm.u.g.xd, sm.u.g.xbs, &sm.tok[0][0], kMaxT, u0 == 0, 1,
                                 tr != nullptr ? tr + 4 : nullptr, err);
    named_sync(1, kMNC);
    if (tr != nullptr && threadIdx.x == 0) tr[1] = globaltimer_ns();
    if constexpr (Q8)
        tg_consume<MT>(g, &sm.ring[0][0], sm.full, sm.empty, kMStages, slot, phase, sm.u.g.xq, sm.u.g.xd, cta, G, err,
                       tr != nullptr ? tr + 6 : nullptr);
    else
        tg_consume_any<MT>(g, &sm.ring[0][0], sm.full, sm.empty, kMStages, slot, phase, sm.u.g.xq, sm.u.g.xd,
                           sm.u.g.xbs, cta, G, err, tr != nullptr ? tr + 6 : nullptr);
}

// ---------------------------------------------------------------------------
// attention op: one CTA per (token, kv head, split of kAttnSplit keys) unit
// ---------------------------------------------------------------------------
// Restates src/s2_model.cpp:979-1039 for the whole query-head group of one kv
// head (GQA h -> h / (H / Hkv)): per-head qk-norm, RoPE mode 0, past keys and
// values from the f16 cache, this call's keys and values un-rounded f32, and
// softmax . V in the split convention the CPU oracle shares:
//   s_j = float(sum_d double(k_j[d]) * double(q[d])) * scale
//   split i: m_i = max s_j, e_j = det_expf(s_j - m_i),
//            S_i = sum double(e_j), O_i[d] = sum double(v_j[d]) * double(e_j)
//   out = float((sum_i O_i[d] * double(w_i)) / (sum_i S_i * double(w_i))),
//         w_i = det_expf(m_i - max_i m_i)
// A single-split unit writes out directly; otherwise each unit stores its
// (O_i, m_i, S_i) and the last unit of the (token, kv head) to arrive combines
// the splits in order.
//
// Latency plan: the split's cache pages are bulk-copied into shared memory at
// the start of the unit, while warps 0..G-1 normalize and rotate the queries
// and warps 4..7 this call's keys and values.  Scores use four threads per
// key (32 dims each), values two threads per output dim (even / odd keys).

// One 128-dim head vector held as 4 dims per lane (dims 4*lane..4*lane+3):
// optional RMSNorm (w = this lane's norm weights) and RoPE with cs = this
// lane's two (cos, sin) pairs, with the arithmetic of rms_norm_weighted and
// ggml_rope_ext mode 0.
__device__ __forceinline__ float4 head_norm_rope_warp(float4 x, bool has_norm, float4 w, float eps, float4 cs) {
    if (has_norm) {
        double s = (double)__fmul_rn(x.x, x.x) + (double)__fmul_rn(x.y, x.y) + (double)__fmul_rn(x.z, x.z) +
                   (double)__fmul_rn(x.w, x.w);
        s = warp_sum_d(s);
        const float mean = (float)(s / (double)kHD);
        const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        x = make_float4(__fmul_rn(__fmul_rn(x.x, sc), w.x), __fmul_rn(__fmul_rn(x.y, sc), w.y),
                        __fmul_rn(__fmul_rn(x.z, sc), w.z), __fmul_rn(__fmul_rn(x.w, sc), w.w));
    }
    const float y0 = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
    const float y1 = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    const float y2 = __fsub_rn(__fmul_rn(x.z, cs.z), __fmul_rn(x.w, cs.w));
    const float y3 = __fadd_rn(__fmul_rn(x.z, cs.w), __fmul_rn(x.w, cs.z));
    return make_float4(y0, y1, y2, y3);
}

// Norm weights and (cos, sin) pairs a consumer thread needs in its first
// attention unit (unit = cta): warps 0..nh-1 normalize the unit's query
// heads, warps 4 and 6 this call's keys of tokens 0 and 1.  None of it
// depends on the previous op, so the loads are issued before the op's input
// is polled.
struct AttnPre {
    float4 nw, cs;
};

__device__ __forceinline__ const float2 *rope_row(const MegaAttn &a, int pos) {
    return a.rope + (size_t)min(max(pos, 0), a.rope_positions - 1) * (kHD / 2);
}

__device__ __forceinline__ AttnPre attn_preload(const MegaAttn &a, int u, int G) {
    AttnPre p;
    p.nw = p.cs = make_float4(0.f, 0.f, 0.f, 0.f);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnPlan pl = attn_plan(a, G);
    if (u >= pl.units) return p;
    const int t = attn_unit_of(a, pl, u).t;
    int pos = -1;
    const float *nw = nullptr;
    if (warp < pl.nh) {
        pos = pl.pos0 + t;
        nw = a.q_norm;
    } else if (warp >= 4 && ((warp - 4) & 1) == 0 && ((warp - 4) >> 1) <= t) {
        pos = pl.pos0 + ((warp - 4) >> 1);
        nw = a.k_norm;
    }
    if (nw != nullptr) p.nw = __ldg(reinterpret_cast<const float4 *>(nw) + lane);
    if (pos >= 0) p.cs = __ldg(reinterpret_cast<const float4 *>(rope_row(a, pos)) + lane);
    return p;
}

// One attention unit (src/s2_model.cpp:979-1039 for query heads h0..h0+nh-1
// of kv head g; GQA h -> h / (H / Hkv)): per-head qk-norm, RoPE mode 0, past
// keys and values from the f16 cache, this call's keys and values un-rounded
// f32, and softmax . V in the split convention the CPU oracle shares:
//   s_j = float(sum_d double(k_j[d]) * double(q[d])) * scale
//   split i: m_i = max s_j, e_j = det_expf(s_j - m_i),
//            S_i = sum double(e_j), O_i[d] = sum double(v_j[d]) * double(e_j)
//   out = float((sum_i O_i[d] * double(w_i)) / (sum_i S_i * double(w_i))),
//         w_i = det_expf(m_i - max_i m_i)
// A single-split unit writes out directly; otherwise each unit stores its
// (O_i, m_i, S_i) and the last unit of the (token, kv head, head block) to
// arrive combines the splits in order.  HPU bounds nh (register arrays).
//
// Latency plan: the split's cache pages are bulk-copied into shared memory at
// the start of the unit, while warps 0..nh-1 normalize and rotate the queries
// and warps 4..7 this call's keys and values.  Scores use four threads per
// key (32 dims each), values two threads per output dim (even / odd keys).
template <int HPU>
__device__ void attn_unit(const MegaAttn &a, const AttnPlan &pl, const AttnUnit &un, const AttnPre &pre, bool first,
                          MSmem &sm, int cta, int *err, unsigned long long *tr, uint32_t &apar, uint32_t in_tag,
                          uint32_t out_tag) {
    AttnSm &as = sm.u.a;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = a.H / a.Hkv;
    const int nh = pl.nh;  // <= HPU
    const bool slow = a.kv_k != nullptr;
    const int nc = pl.nc, pos0 = pl.pos0;
    const int t = un.t, g = un.g, hb = un.hb, i = un.i, h0 = hb * nh;
    auto mark = [&](int k) {
        if (tr != nullptr && first && tid == 0) tr[k] = globaltimer_ns();
    };
    const int Lk = nc + a.cur_base + t + 1;  // keys of token t
    const int nsp = (Lk + kAttnSplit - 1) / kAttnSplit;
    if (i >= nsp) return;  // CTA-uniform
    const int j0 = i * kAttnSplit, cnt = min(kAttnSplit, Lk - j0);
    const int ncp = slow ? max(0, min(cnt, nc - j0)) : 0;  // cached keys of the split
    const int npg = (ncp + kPage - 1) / kPage;
    // ---- A. the split's cache pages -> shared memory (bulk copies) ----
    // Warp 7 (this call's v of token 1: idle at T = 1) issues them, one page's
    // keys or values per lane in the same instruction (one lane issuing them
    // one after another serializes the issue, as in the weight producer).
    static_assert(2 * (kAttnSplit / kPage) <= 32, "a lane per page copy");
    if (npg > 0 && warp == kMW - 1) {
        if (lane == 0) mbar_arrive_expect_tx(&sm.abar, (uint32_t)(2 * npg * kPage * kHD * sizeof(__half)));
        __syncwarp();
        if (lane < 2 * npg) {
            const int p = lane >> 1, pg = j0 / kPage + p;
            const int page = pg < kPtab ? sm.ptab[pg] : __ldcg(a.block_table + pg);
            const size_t off = (((size_t)page * a.kv_layers + a.layer) * a.Hkv + g) * kPage * kHD;
            fence_proxy_async_smem();
            if (lane & 1)
                bulk_g2s_plain(&as.v.h[p * kPage][0], a.kv_v + off, kPage * kHD * sizeof(__half), &sm.abar);
            else
                bulk_g2s_plain(&as.k.h[p * kPage][0], a.kv_k + off, kPage * kHD * sizeof(__half), &sm.abar);
        }
    }
    // ---- B. queries (warps 0..nh-1), this call's keys / values (warps 4..7) ----
    const bool has_cur = j0 + cnt > nc + a.cur_base;  // the split reaches this call's tokens
    const bool own = (nc + a.cur_base + t) / kAttnSplit == i && hb == 0;  // this unit stores token t's K/V
    if (warp < nh) {
        const int h = g * grp + h0 + warp;
        const int pos = pos0 + t;
        if (pos >= a.rope_positions && lane == 0) atomicOr(err, ERR_BAD_POS);
        const float4 x = ll_wait4(a.qkv, (size_t)t * a.ldqkv + (size_t)h * kHD + 4 * lane, in_tag, err);
        const float4 y = head_norm_rope_warp(x, a.q_norm != nullptr, pre.nw, a.eps, pre.cs);
        double *qd = &as.q[warp][lane >> 3][4 * (lane & 7)];  // 16-byte aligned: 34-double rows
        qd[0] = (double)y.x;
        qd[1] = (double)y.y;
        qd[2] = (double)y.z;
        qd[3] = (double)y.w;
    } else if (warp >= 4 && has_cur) {
        const int tt = (warp - 4) >> 1, isv = (warp - 4) & 1;
        if (tt <= t) {
            const int pos = pos0 + tt;
            float4 x = ll_wait4(a.qkv, (size_t)tt * a.ldqkv + (size_t)(a.H + (isv ? a.Hkv : 0) + g) * kHD + 4 * lane,
                                in_tag, err);
            if (!isv) x = head_norm_rope_warp(x, a.k_norm != nullptr, pre.nw, a.eps, pre.cs);
            float *dst = slow ? (isv ? as.vc[tt] : as.kc[tt]) : (isv ? as.v.f[a.cur_base + tt] : as.k.f[a.cur_base + tt]);
            reinterpret_cast<float4 *>(dst)[lane] = x;
            if (tt == t && own) {
                // token t's K/V: f32 for the later calls of this frame, f16 into the cache (Slow)
                float *cur = (isv ? a.vcur : a.kcur) + ((size_t)(a.cur_base + t) * a.Hkv + g) * kHD;
                reinterpret_cast<float4 *>(cur)[lane] = x;
                if (slow) {
                    const int pg = pos / kPage, slot = pos - pg * kPage;
                    if (pos >= 0 && pg < a.kv_pages) {
                        const int page = __ldcg(a.block_table + pg);
                        __half *c = (isv ? a.kv_v : a.kv_k) +
                                    ((((size_t)page * a.kv_layers + a.layer) * a.Hkv + g) * kPage + slot) * kHD;
                        __half2 *c2 = reinterpret_cast<__half2 *>(c) + 2 * lane;
                        c2[0] = __floats2half2_rn(x.x, x.y);
                        c2[1] = __floats2half2_rn(x.z, x.w);
                    } else if (lane == 0) {
                        atomicOr(err, ERR_BAD_POS);
                    }
                }
            }
        }
    }
    mark(8);
    if (!slow) {
        // earlier Fast-AR positions of this frame: f32 rows written by the previous passes
        for (int idx = tid; idx < a.cur_base * 64; idx += kMNC) {
            const int row = idx >> 6, isv = (idx >> 5) & 1, c4 = idx & 31;
            const float4 x = __ldcg(reinterpret_cast<const float4 *>((isv ? a.vcur : a.kcur) +
                                                                     ((size_t)row * a.Hkv + g) * kHD) + c4);
            reinterpret_cast<float4 *>(isv ? as.v.f[row] : as.k.f[row])[c4] = x;
        }
    }
    named_sync(3, kMNC);
    mark(9);
    if (npg > 0) {
        mbar_wait(&sm.abar, apar, err, ERR_WAIT_FULL);
        apar ^= 1u;
    }
    mark(4);
    // ---- C. scores: thread (key jj = tid / 4, quarter c = tid % 4) over 32 dims ----
    {
        const int jj = tid >> 2, c = tid & 3;
        double acc[HPU];
#pragma unroll
        for (int h = 0; h < HPU; ++h) acc[h] = 0.0;
        if (jj < cnt) {
            const int j = j0 + jj;
            if (j < nc) {
                const uint4 *kp = reinterpret_cast<const uint4 *>(&as.k.h[jj][32 * c]);
#pragma unroll
                for (int qd = 0; qd < 4; ++qd) {
                    const uint4 raw = kp[qd];
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const float2 f = __half22float2(hh[p]);
                        const double k0 = (double)f.x, k1 = (double)f.y;
#pragma unroll
                        for (int h = 0; h < HPU; ++h) {
                            const double2 qq = *reinterpret_cast<const double2 *>(&as.q[h][c][8 * qd + 2 * p]);
                            acc[h] += k0 * qq.x + k1 * qq.y;
                        }
                    }
                }
            } else {
                const float *kr = slow ? &as.kc[j - nc][32 * c] : &as.k.f[jj][32 * c];
#pragma unroll
                for (int d4 = 0; d4 < 8; ++d4) {
                    const float4 f = reinterpret_cast<const float4 *>(kr)[d4];
#pragma unroll
                    for (int h = 0; h < HPU; ++h) {
                        const double2 q0 = *reinterpret_cast<const double2 *>(&as.q[h][c][4 * d4]);
                        const double2 q1 = *reinterpret_cast<const double2 *>(&as.q[h][c][4 * d4 + 2]);
                        acc[h] += (double)f.x * q0.x + (double)f.y * q0.y + (double)f.z * q1.x + (double)f.w * q1.y;
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < HPU; ++h) {
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
            acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
        }
        if (c == 0 && jj < cnt)
#pragma unroll
            for (int h = 0; h < HPU; ++h)
                if (h < nh) as.s[h][jj] = __fmul_rn((float)acc[h], a.scale);
    }
    named_sync(3, kMNC);
    mark(5);
    // ---- D. the split's softmax statistics: warp h for head h ----
    if (warp < nh) {
        const float s0 = lane < cnt ? as.s[warp][lane] : -INFINITY;
        const float s1 = lane + 32 < cnt ? as.s[warp][lane + 32] : -INFINITY;
        const float mx = warp_max(fmaxf(s0, s1));
        const float e0 = lane < cnt ? det_expf(__fsub_rn(s0, mx)) : 0.f;
        const float e1 = lane + 32 < cnt ? det_expf(__fsub_rn(s1, mx)) : 0.f;
        as.e[lane][warp] = (double)e0;
        as.e[lane + 32][warp] = (double)e1;
        const double S = warp_sum_d((double)e0 + (double)e1);
        if (lane == 0) {
            as.m[warp] = mx;
            as.S[warp] = S;
        }
    }
    named_sync(3, kMNC);
    mark(6);
    // ---- E. values: thread (dim d = tid % 128, key parity kh = tid / 128) ----
    const int d = tid & (kHD - 1), kh = tid >> 7;
    double o[HPU];
#pragma unroll
    for (int h = 0; h < HPU; ++h) o[h] = 0.0;
#pragma unroll 4
    for (int jj = kh; jj < cnt; jj += 2) {
        const int j = j0 + jj;
        const double vd = j < nc ? (double)__half2float(as.v.h[jj][d])
                                 : (double)(slow ? as.vc[j - nc][d] : as.v.f[jj][d]);
        if constexpr (HPU == 1) {
            o[0] += vd * as.e[jj][0];
        } else {
            const double2 e01 = *reinterpret_cast<const double2 *>(&as.e[jj][0]);
            o[0] += vd * e01.x;
            o[1] += vd * e01.y;
            if constexpr (HPU == 4) {
                const double2 e23 = *reinterpret_cast<const double2 *>(&as.e[jj][2]);
                o[2] += vd * e23.x;
                o[3] += vd * e23.y;
            }
        }
    }
    if (kh == 1)
#pragma unroll
        for (int h = 0; h < HPU; ++h) as.o[h][d] = o[h];
    named_sync(3, kMNC);
    mark(7);
    if (kh == 0)
#pragma unroll
        for (int h = 0; h < HPU; ++h) o[h] += as.o[h][d];
    const size_t out_row = (size_t)t * a.H * kHD + (size_t)(g * grp + h0) * kHD;
    if (nsp == 1) {
        if (kh == 0)
#pragma unroll
            for (int h = 0; h < HPU; ++h)
                if (h < nh) ll_store(a.out, out_row + (size_t)h * kHD + d, (float)(o[h] / as.S[h]), out_tag);
        named_sync(3, kMNC);  // the unit's shared buffers are free for the next unit
        return;
    }
    const size_t pu = ((size_t)t * a.Hkv + g) * a.n_split_max;
    if (kh == 0)
#pragma unroll
        for (int h = 0; h < HPU; ++h)
            if (h < nh) a.part[((pu + i) * grp + h0 + h) * kHD + d] = o[h];
    if (tid < nh) {
        a.part_ms[((pu + i) * grp + h0 + tid) * 2] = (double)as.m[tid];
        a.part_ms[((pu + i) * grp + h0 + tid) * 2 + 1] = as.S[tid];
    }
    named_sync(3, kMNC);
    int *counter = a.counters + ((size_t)t * a.Hkv + g) * kAG + hb;
    if (tid == 0) {
        mark(10);
        // release: the CTA's partials (ordered before this thread by the CTA
        // barrier) become visible before the count; acquire: the other
        // units' partials are visible to this CTA after the next barrier
        unsigned old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
        as.last = (int)old == nsp - 1;
        mark(3);
    }
    named_sync(3, kMNC);
    if (as.last) {
        // combine in split order; (m_k, S_k) staged in shared memory, weights
        // w_k = det_expf(m_k - M); thread (d, kh) sums local heads kh, kh + 2
        if (nsp <= kCombineFast) {
            // one round trip: (m_k, S_k) staged by threads p < nh * nsp while every
            // thread loads its own O_k[h][d] of heads kh, kh + 2 into registers;
            // then the same threads form each split's weight w_k once (one
            // det_expf per (head, split), not one per output dim: the unit's
            // code stays small, which the instruction cache rewards)
            double ov[2][kCombineFast];
#pragma unroll
            for (int x = 0; x < 2; ++x)
#pragma unroll
                for (int k = 0; k < kCombineFast; ++k)
                    ov[x][k] = (kh + 2 * x < nh && k < nsp)
                                   ? __ldcg(a.part + ((pu + k) * grp + h0 + kh + 2 * x) * kHD + d)
                                   : 0.0;
            if (tid < nh * nsp) {
                const int h = tid / nsp, k = tid - h * nsp;
                const double2 ms = __ldcg(reinterpret_cast<const double2 *>(a.part_ms + ((pu + k) * grp + h0 + h) * 2));
                as.s[h][k] = (float)ms.x;
                as.e[k][h] = ms.y;
            }
            named_sync(3, kMNC);
            if (tid < nh * nsp) {
                const int h = tid / nsp, k = tid - h * nsp;
                float M = as.s[h][0];
                for (int k2 = 1; k2 < nsp; ++k2) M = fmaxf(M, as.s[h][k2]);
                as.o[h][k] = (double)det_expf(__fsub_rn(as.s[h][k], M));
            }
            named_sync(3, kMNC);
#pragma unroll
            for (int x = 0; x < 2; ++x) {
                const int h = kh + 2 * x;
                if (h < nh) {
                    double acc = 0.0, S = 0.0;
#pragma unroll
                    for (int k = 0; k < kCombineFast; ++k)
                        if (k < nsp) {
                            const double w = as.o[h][k];
                            acc += ov[x][k] * w;
                            S += as.e[k][h] * w;
                        }
                    ll_store(a.out, out_row + (size_t)h * kHD + d, (float)(acc / S), out_tag);
                }
            }
            if (tid == 0) *counter = 0;
            named_sync(3, kMNC);
            return;
        }
        const int nch = (nsp + kAttnSplit - 1) / kAttnSplit;
        auto stage = [&](int kb, int kn) {
            for (int p = tid; p < nh * kn; p += kMNC) {
                const int h = p / kn, k = p - h * kn;
                const double2 ms = __ldcg(reinterpret_cast<const double2 *>(a.part_ms + ((pu + kb + k) * grp + h0 + h) * 2));
                as.s[h][k] = (float)ms.x;
                as.e[k][h] = ms.y;
            }
            named_sync(3, kMNC);
        };
        for (int c = 0; c < nch; ++c) {
            const int kb = c * kAttnSplit, kn = min(kAttnSplit, nsp - kb);
            stage(kb, kn);
            if (warp < nh) {
                float mx = fmaxf(lane < kn ? as.s[warp][lane] : -INFINITY,
                                 lane + 32 < kn ? as.s[warp][lane + 32] : -INFINITY);
                mx = warp_max(mx);
                if (lane == 0) as.m[warp] = c == 0 ? mx : fmaxf(as.m[warp], mx);
            }
            named_sync(3, kMNC);
        }
        double acc[2] = {0.0, 0.0}, S[2] = {0.0, 0.0};
        for (int c = 0; c < nch; ++c) {
            const int kb = c * kAttnSplit, kn = min(kAttnSplit, nsp - kb);
            if (nch > 1) stage(kb, kn);  // one chunk: still staged from the max pass
            for (int p = tid; p < nh * kn; p += kMNC) {
                const int h = p / kn, k = p - h * kn;
                as.o[h][k] = (double)det_expf(__fsub_rn(as.s[h][k], as.m[h]));
            }
            named_sync(3, kMNC);
#pragma unroll
            for (int x = 0; x < 2; ++x) {
                const int h = kh + 2 * x;
                if (h < nh) {
                    const double *src = a.part + ((pu + kb) * grp + h0 + h) * kHD + d;
#pragma unroll 8
                    for (int k = 0; k < kn; ++k) {
                        acc[x] += __ldcg(src + (size_t)k * grp * kHD) * as.o[h][k];
                        S[x] += as.e[k][h] * as.o[h][k];
                    }
                }
            }
            named_sync(3, kMNC);
        }
#pragma unroll
        for (int x = 0; x < 2; ++x) {
            const int h = kh + 2 * x;
            if (h < nh) ll_store(a.out, out_row + (size_t)h * kHD + d, (float)(acc[x] / S[x]), out_tag);
        }
        if (tid == 0) *counter = 0;
    }
    named_sync(3, kMNC);  // the unit's shared buffers are free for the next unit
}

__device__ void mega_attn(const MegaAttn &a, const AttnPre &pre, MSmem &sm, int cta, int G, int *err,
                          unsigned long long *tr, uint32_t &apar, uint32_t ep8) {
    const uint32_t in_tag = ep8 | a.in_tag, out_tag = ep8 | a.out_tag;
    const int tid = threadIdx.x;
    const bool slow = a.kv_k != nullptr;
    const AttnPlan pl = attn_plan(a, G);
    if (slow && cta < pl.units && !sm.ptab_ready) {
        // the block table and n_past do not change within a segment: stage the
        // page ids once, at the first attention op this CTA runs
        const int npg = min((pl.nc + kPage - 1) / kPage, kPtab);
        for (int i = tid; i < npg; i += kMNC) sm.ptab[i] = __ldcg(a.block_table + i);
        named_sync(3, kMNC);
        if (tid == 0) sm.ptab_ready = 1;
    }
    for (int u = cta; u < pl.units; u += G) {
        const AttnUnit un = attn_unit_of(a, pl, u);
        const AttnPre pp = u == cta ? pre : attn_preload(a, u, G);
        if (pl.nh == 1)
            attn_unit<1>(a, pl, un, pp, u == cta, sm, cta, err, tr, apar, in_tag, out_tag);
        else if (pl.nh == 2)
            attn_unit<2>(a, pl, un, pp, u == cta, sm, cta, err, tr, apar, in_tag, out_tag);
        else
            attn_unit<kAG>(a, pl, un, pp, u == cta, sm, cta, err, tr, apar, in_tag, out_tag);
    }
}


// Every load a thread needs is issued before any is used (token id, the
// codebook ids, then all rows' quants and scales), so the op costs about three
// memory round trips; the codebook sum keeps the reference's order cb0..cb9.
constexpr int kMaxCb = 16;

__device__ void mega_embed_slow(const MegaEmbedSlow &e, int cta, int G, int *err, uint32_t ep8) {
    const int stride = e.ncb + 1;
    for (long long idx = (long long)cta * kMNC + threadIdx.x; idx < (long long)e.T * e.dim; idx += (long long)G * kMNC) {
        const int t = (int)(idx / e.dim), i = (int)(idx - (long long)t * e.dim);
        int tok = __ldcg(e.tokens + t * stride);
        int ids[kMaxCb];
#pragma unroll
        for (int cb = 0; cb < kMaxCb; ++cb) ids[cb] = cb < e.ncb ? __ldcg(e.tokens + t * stride + 1 + cb) : 0;
        if (tok < 0 || tok >= e.e_rows) {
            if (i == 0) atomicOr(err, ERR_BAD_TOKEN);
            tok = 0;
        }
        const bool sem = tok >= e.sem_begin && tok <= e.sem_end;
        float x = tq_elem(e.e, e.etype, e.dim, tok, i);
        if (sem && e.ncb > 0) {
            float r[kMaxCb];
#pragma unroll
            for (int cb = 0; cb < kMaxCb; ++cb) {
                r[cb] = 0.f;
                if (cb < e.ncb) {
                    int id = ids[cb] + cb * e.cb_size;
                    if (id < 0 || id >= e.c_rows) {
                        if (i == 0) atomicOr(err, ERR_BAD_TOKEN);
                        id = 0;
                    }
                    r[cb] = tq_elem(e.c, e.ctype, e.dim, id, i);
                }
            }
            float s = r[0];
#pragma unroll
            for (int cb = 1; cb < kMaxCb; ++cb)
                if (cb < e.ncb) s = __fadd_rn(s, r[cb]);
            x = __fadd_rn(x, s);
        }
        if (e.scale_cb && sem) x = __fmul_rn(x, e.sem_scale);
        ll_store(e.x, (size_t)t * e.dim + i, x, ep8 | e.tag);
    }
}

__device__ void mega_embed_fast(const MegaEmbedFast &e, int cta, int G, int *err, uint32_t ep8) {
    const int hrow = e.hidden ? 1 : 0;
    for (long long idx = (long long)cta * kMNC + threadIdx.x; idx < (long long)e.n_rows * e.dim;
         idx += (long long)G * kMNC) {
        const int r = (int)(idx / e.dim), i = (int)(idx - (long long)r * e.dim);
        float x;
        if (r < hrow) {
            x = __ldcg(e.hidden + i);
        } else {
            int c = __ldcg(e.codes + e.code0 + r - hrow);
            if (c < 0 || c >= e.f_rows) {
                if (i == 0) atomicOr(err, ERR_BAD_TOKEN);
                c = 0;
            }
            x = tq_elem(e.f, e.ftype, e.dim, c, i);
        }
        ll_store(e.x, (size_t)r * e.dim + i, x, ep8 | e.tag);
    }
}

// 10 warps per CTA, dealt to the SM's four sub-partitions round robin: two
// of them hold three warps, so their 16K registers cap a thread at 168 (the
// launch bound keeps the kernel there; 200 registers would not launch).
template <int MT, bool Q8>
__global__ void __launch_bounds__(kMThreads, 1)
    mega_kernel(const MegaOp *__restrict__ ops, int n_ops, MegaCtl *ctl, const int *done, int *err, int l2_ahead,
                unsigned long long *trace, int flags, unsigned *epoch) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    MSmem &sm = *reinterpret_cast<MSmem *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (done != nullptr && __ldcg(done) != 0) return;  // finished sequence: the whole grid exits
    // Tags of this launch's activations: (epoch << 8) | producing op.  The
    // epoch only changes when the last CTA of a launch exits, so every CTA of
    // a launch reads the same value here.
    const uint32_t ep8 = __ldcg(epoch) << 8;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kMW);
        }
        mbar_init(&sm.abar, 1);
        fence_mbar_init();
        sm.ptab_ready = 0;
        sm.cur_op = 0;
    }
    __syncthreads();
    if (warp == kMW) {
        const int depth = ((flags >> 8) & 255) > 0 ? min((flags >> 8) & 255, kMStages) : kMStages;
        const int lanes = ((flags >> 16) & 15) > 0 ? (flags >> 16) & 15 : kMaxPL;
        mega_producer(ops, n_ops, sm, cta, G, l2_ahead, depth, lanes, err, trace);
        return;
    }
    if (warp == kMW + 1) {
        if (lane == 0) mega_kv_prefetch(ops, n_ops, sm, cta, G, err);
        return;
    }
    // trace: per op and CTA, [start, prologue done, work done, producer's last tile issued]
    auto stamp = [&](int i, int k) {
        if (trace != nullptr && threadIdx.x == 0) trace[((size_t)i * G + cta) * kTraceSlots + k] = globaltimer_ns();
    };
    int cslot = 0;  // ring position of the consumers
    uint32_t cphase = 0;
    uint32_t apar = 0;  // phase of the attention page barrier
    for (int i = 0; i < n_ops; ++i) {
        const int kind = ops[i].kind;
        // RMSNorm weights of the next GEMV do not depend on the previous op: load them before the barrier
        F8 nw[kMPC];
        AttnPre ap;
        if (kind == MK_GEMV) tg_norm_preload<kMPC, kMNC>(ops[i].g, nw);
        if (kind == MK_ATTN) ap = attn_preload(ops[i].a, cta, G);
        // no grid barrier: each op's readers poll the tags of the words they read
        named_sync(1, kMNC);  // the previous op's shared buffers are free
        if (threadIdx.x == 0) *reinterpret_cast<volatile int *>(&sm.cur_op) = i;
        stamp(i, 0);
        stamp(i, 1);
        switch (kind) {
        case MK_GEMV:
            mega_gemv<MT, Q8>(ops[i].g, nw, sm, cta, G, cslot, cphase, err,
                          trace != nullptr ? trace + ((size_t)i * G + cta) * kTraceSlots : nullptr, ep8);
            break;
        case MK_ATTN:
            mega_attn(ops[i].a, ap, sm, cta, G, err,
                      trace != nullptr ? trace + ((size_t)i * G + cta) * kTraceSlots : nullptr, apar, ep8);
            break;
        case MK_EMBED_SLOW: mega_embed_slow(ops[i].es, cta, G, err, ep8); break;
        case MK_EMBED_FAST: mega_embed_fast(ops[i].ef, cta, G, err, ep8); break;
        case MK_ADVANCE:
            // n_past is read by every attention op of the launch: advance it
            // only once every CTA has finished all earlier ops (a CTA with no
            // work in the last ops would get here early)
            if (threadIdx.x == 0) {
                __threadfence();
                atomicAdd(&ctl->pad[0], 1u);
                if (cta == 0) {
                    const long long t0 = clock64(), lim = wait_limit(err);
                    while (ld_acquire_u32(&ctl->pad[0]) < (unsigned)G) {
                        if (clock64() - t0 > lim) {
                            atomicOr(err, ERR_GRID);
                            break;
                        }
                    }
                    volatile int *np = ops[i].adv.n_past;
                    *np = *np + ops[i].adv.T;
                }
            }
            break;
        default: break;
        }
        stamp(i, 2);
    }
    stamp(n_ops, 0);
    // the last CTA to finish moves the epoch on (the next launch's tags)
    named_sync(1, kMNC);
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&ctl->count, 1u) == (unsigned)G - 1) atomicAdd(epoch, 1u);
    }
}

// Tiles per CTA the producer prefetches into L2 beyond its ring (148 CTAs x
// 24 tiles x 17 KB would be 62 MB of the 126 MB L2).  Off by default: a
// run-ahead of 8-64 tiles measured no faster.  S2K_L2_AHEAD (read at each
// launch or graph capture) sets it, up to 64.
int mega_l2_ahead() {
    const char *e = getenv("S2K_L2_AHEAD");
    const int d = e ? atoi(e) : 0;
    return d < 0 ? 0 : (d > 64 ? 64 : d);
}

cudaError_t mega_setup() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(mega_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem))))
        return e;
    if ((e = cudaFuncSetAttribute(mega_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem))))
        return e;
    if ((e = cudaFuncSetAttribute(mega_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem))))
        return e;
    return cudaFuncSetAttribute(mega_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem));
}

cudaError_t launch_mega(const MegaOp *d_ops, int n_ops, int mt, MegaCtl *ctl, const int *done, int *err, int num_sms,
                        cudaStream_t st, unsigned *epoch, bool q8, unsigned long long *trace) {
    if (mt < 1 || mt > kMaxT) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kMThreads);
    cfg.dynamicSmemBytes = sizeof(MSmem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    const int ahead = mega_l2_ahead();
    // S2K_MEGA_FLAGS (tuning and measurement; 0 = defaults): bits 8-15 the
    // most tiles in flight per CTA (1..kMStages), bits 16-19 the producer
    // lanes per group of tiles (1..kMaxPL)
    const char *fe = getenv("S2K_MEGA_FLAGS");
    const int flags = fe ? atoi(fe) : 0;
    if (q8) {
        if (mt == 1)
            return cudaLaunchKernelEx(&cfg, mega_kernel<1, true>, d_ops, n_ops, ctl, done, err, ahead, trace, flags, epoch);
        return cudaLaunchKernelEx(&cfg, mega_kernel<2, true>, d_ops, n_ops, ctl, done, err, ahead, trace, flags, epoch);
    }
    if (mt == 1)
        return cudaLaunchKernelEx(&cfg, mega_kernel<1, false>, d_ops, n_ops, ctl, done, err, ahead, trace, flags, epoch);
    return cudaLaunchKernelEx(&cfg, mega_kernel<2, false>, d_ops, n_ops, ctl, done, err, ahead, trace, flags, epoch);
}

// Bounded-wait probe: one warp polls four tagged activation words for a tag
// that no launch writes (epoch 2^24 - 1 is never reached), through the same
// wait the persistent kernel's consumers use.  It returns once the model's
// wait limit has passed, with ERR_GRID set in *err.  Only reads `words`.
__global__ void wait_probe_kernel(const uint64_t *words, int *err) {
    const float4 v = ll_wait4(words, 0, 0xFFFFFFFFu, err);
    (void)v;
}

cudaError_t launch_wait_probe(const uint64_t *words, int *err, cudaStream_t st) {
    if (words == nullptr || reinterpret_cast<uintptr_t>(words) % 32 != 0) return cudaErrorInvalidValue;
    count_launch();
    wait_probe_kernel<<<1, 32, 0, st>>>(words, err);
    return cudaGetLastError();
}

}  // namespace s2k
