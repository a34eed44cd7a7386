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

// 8 consumer warps (the tile engine's mapping, s2k_tgemv.cuh) + 1 producer.
constexpr int kMW = kTW;                   // consumer warps
constexpr int kMNC = kMW * 32;             // consumer threads
constexpr int kMThreads = kMNC + 32;       // + producer warp
constexpr int kMStages = 10;               // ring of 17 KB weight tiles
constexpr int kMKMax = 10240;
constexpr int kMaxT = 2;
constexpr int kHD = 128;
constexpr int kPtab = 512;                 // cached pages whose ids are staged in shared memory
constexpr int kAttnKeys = 1024;            // longest key range whose scores stay on chip
constexpr int kMPC = 5;                    // 8-value activation chunks per consumer thread per prologue pass

bool mega_gemv_ok(const MegaGemv &g) {
    if (!tg_shape_ok(g.R, g.K, g.M, g.in_mode, g.epi, g.res != nullptr, kMKMax, kMaxT)) return false;
    if (g.in_mode == IN_RMSNORM && g.norm_w == nullptr) return false;
    // one-pass RMSNorm prologue; 32-byte activation and norm-weight loads
    if (g.in_mode == IN_RMSNORM && g.M * g.K > 8 * kMPC * kMNC) return false;
    if (g.ldx % 8 != 0 || reinterpret_cast<uintptr_t>(g.x) % 32 != 0) return false;
    if (g.act_out != nullptr && reinterpret_cast<uintptr_t>(g.act_out) % 16 != 0) return false;
    if (g.norm_w != nullptr && reinterpret_cast<uintptr_t>(g.norm_w) % 32 != 0) return false;
    return true;
}

struct MSmem {
    uint8_t ring[kMStages][kTileBytes];
    uint64_t full[kMStages], empty[kMStages];
    int8_t xq[kMaxT * kMKMax];  // quantized activation (GEMV)
    float xd[kMaxT * kMKMax / 32];
    float nw[kNormMax];  // norm weights (GEMV); probabilities (attention)
    double tok[kMW][kMaxT];
    float scale[kMaxT];
    // attention
    float aq[kHD];
    double aqd[kHD];  // q as doubles for the score loops
    alignas(16) float ak[kMaxT][kHD];  // read as float4
    alignas(16) float av[kMaxT][kHD];
    double vpart[kMW][kHD];
    float red_f[kMW];
    double red_d[kMW];
    int ptab[kPtab];  // page ids of the sequence's first kPtab pages (Slow segment)
    int ptab_ready;
};

static_assert(sizeof(MSmem) <= 227 * 1024, "persistent kernel shared memory exceeds the per-CTA limit");
static_assert(kAttnKeys <= kNormMax, "attention probabilities live in the norm-weight buffer");
// shared arrays read with 16-byte vector loads
static_assert(offsetof(MSmem, ring) % 16 == 0 && kTileBytes % 16 == 0, "ring alignment");
static_assert(offsetof(MSmem, xq) % 16 == 0 && offsetof(MSmem, nw) % 16 == 0, "activation buffer alignment");
static_assert(offsetof(MSmem, ak) % 16 == 0 && offsetof(MSmem, av) % 16 == 0, "key / value row alignment");
static_assert(kAttnKeys % kMNC == 0, "keys per thread");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// consumer-only grid barrier halves
__device__ __forceinline__ void grid_arrive(MegaCtl *ctl, int flags) {
    named_sync(1, kMNC);
    if (threadIdx.x == 0) {
        if (flags & 1) {
            // release-add: orders this CTA's writes (seen through the named barrier) before the count
            asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(&ctl->count), "r"(1u) : "memory");
        } else {
            __threadfence();
            atomicAdd(&ctl->count, 1u);
        }
    }
}

__device__ __forceinline__ void grid_wait(MegaCtl *ctl, unsigned target, int *err) {
    if (threadIdx.x == 0) {
        if (ld_acquire_u32(&ctl->count) < target &&
            !(*reinterpret_cast<volatile int *>(err) & (ERR_WAIT_FULL | ERR_WAIT_EMPTY | ERR_GRID))) {
            const long long t0 = clock64();
            while (ld_acquire_u32(&ctl->count) < target) {
                if (clock64() - t0 > kWaitLimitCycles) {
                    atomicOr(err, ERR_GRID);
                    break;
                }
            }
        }
    }
    named_sync(1, kMNC);
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

    __device__ __forceinline__ const uint8_t *next(const MegaOp *ops, int n_ops, int cta, int G) {
        while (u >= u1) {
            if (++op >= n_ops) return nullptr;
            if (ops[op].kind != MK_GEMV) continue;
            tg_range(ops[op].g.R, ops[op].g.K, cta, G, &u, &u1);
            w = ops[op].g.w;
        }
        return w + (size_t)(u++) * kTileBytes;
    }
};

// The ring holds kMStages tiles; a second cursor runs `l2_ahead` tiles past
// the ring's head and pulls those tiles into L2 with bulk prefetches, so HBM
// keeps streaming while the consumers sit in a grid barrier, an activation
// prologue or attention (the ring alone covers ~4 us of HBM time per SM).
__device__ void mega_producer(const MegaOp *ops, int n_ops, MSmem &sm, int cta, int G, int l2_ahead, int *err,
                              unsigned long long *trace) {
    const uint64_t pol = policy_evict_first();
    TileCursor ld, pf;
    long long pf_n = 0;  // tiles the prefetch cursor has passed
    // the first kMStages tiles go straight into the empty ring
    for (int i = 0; i < kMStages && pf.next(ops, n_ops, cta, G); ++i) ++pf_n;
    const uint8_t *src;
    for (long long ps = 0; (src = ld.next(ops, n_ops, cta, G)) != nullptr; ++ps) {
        for (const uint8_t *p; pf_n < ps + kMStages + l2_ahead && (p = pf.next(ops, n_ops, cta, G)) != nullptr; ++pf_n)
            bulk_prefetch_l2(p, kTileBytes);
        const int slot = (int)(ps % kMStages);
        if (ps >= kMStages && !mbar_wait(&sm.empty[slot], (uint32_t)((ps / kMStages) - 1) & 1u, err, ERR_WAIT_EMPTY))
            return;
        mbar_arrive_expect_tx(&sm.full[slot], kTileBytes);
        bulk_g2s(sm.ring[slot], src, kTileBytes, &sm.full[slot], pol);
        if (trace != nullptr && ld.u == ld.u1) trace[((size_t)ld.op * G + cta) * kTraceSlots + 3] = globaltimer_ns();
    }
}

// ---------------------------------------------------------------------------
// GEMV op (consumer side): activation prologue, then this CTA's tiles
// ---------------------------------------------------------------------------
template <int MT>
__device__ void mega_gemv(const MegaGemv &gref, const F8 (&nw)[kMPC], MSmem &sm, int cta, int G, int &slot,
                          uint32_t &phase, int *err, unsigned long long *tr) {
    const MegaGemv g = gref;  // op fields in registers
    long long u0, u1;
    tg_range(g.R, g.K, cta, G, &u0, &u1);
    if (u0 == u1) return;  // no row tile of this op here (R / 32 < G)
    // the CTA owning row tile 0 stores act_out
    tg_prologue8<MT, kMNC, kMPC>(g, nw, sm.xq, sm.xd, &sm.tok[0][0], kMaxT, u0 == 0, 1,
                                 tr != nullptr ? tr + 4 : nullptr);
    named_sync(1, kMNC);
    if (tr != nullptr && threadIdx.x == 0) tr[1] = globaltimer_ns();
    tg_consume<MT>(g, &sm.ring[0][0], sm.full, sm.empty, kMStages, slot, phase, sm.xq, sm.xd, cta, G, err,
                   tr != nullptr ? tr + 6 : nullptr);
}

// ---------------------------------------------------------------------------
// attention op: one CTA per (token, query head) unit
// ---------------------------------------------------------------------------
// x0/x1 = pair (2i, 2i+1) of a head vector held by 64 consecutive threads
// (i = index in the group); optional per-head RMSNorm (nw0/nw1 = the pair's
// norm weights, prefetched; reduction over the 64 threads of warps w0, w0+1,
// partial sums in red_d[red_slot..+1]) then RoPE with the prefetched (cos,
// sin) of the pair.  Every consumer thread must call it (one named barrier).
__device__ __forceinline__ void head_norm_rope(float &x0, float &x1, bool has_norm, float nw0, float nw1, float eps,
                                               float2 cs, int red_slot, MSmem &sm, bool active) {
    if (has_norm) {
        double s = active ? (double)__fmul_rn(x0, x0) + (double)__fmul_rn(x1, x1) : 0.0;
        s = warp_sum_d(s);
        if ((threadIdx.x & 31) == 0 && active) sm.red_d[red_slot + ((threadIdx.x >> 5) & 1)] = s;
    }
    named_sync(3, kMNC);
    if (active) {
        if (has_norm) {
            const double tot = sm.red_d[red_slot] + sm.red_d[red_slot + 1];
            const float mean = (float)(tot / (double)kHD);
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
            x0 = __fmul_rn(__fmul_rn(x0, sc), nw0);
            x1 = __fmul_rn(__fmul_rn(x1, sc), nw1);
        }
        const float y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
        const float y1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
        x0 = y0;
        x1 = y1;
    }
}

__device__ __forceinline__ const float *key_ptr_f32(const MegaAttn &a, MSmem &sm, int c, int g, bool value) {
    // current-call key index c (positions >= n_cached): persistent f32 buffer or this op's tokens
    if (c < a.cur_base) return (value ? a.vcur : a.kcur) + ((size_t)c * a.Hkv + g) * kHD;
    return value ? sm.av[c - a.cur_base] : sm.ak[c - a.cur_base];
}

// Row of cached key/value position j for kv head g in the paged f16 cache;
// ptab holds the first kPtab page ids of the sequence (staged per segment).
__device__ __forceinline__ const __half *kv_row(const MegaAttn &a, const __half *base, const int *ptab, int g, int j) {
    const int pg = j / kPage, slot = j - pg * kPage;
    const int page = pg < kPtab ? ptab[pg] : __ldcg(a.block_table + pg);
    return base + ((((size_t)page * a.kv_layers + a.layer) * a.Hkv + g) * kPage + slot) * kHD;
}

// Dot product of a cached f16 key row (16 x 16 bytes, already loaded) with q.
__device__ __forceinline__ float key_score(const uint4 (&raw)[kHD / 8], const double *aq, float scale) {
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
#pragma unroll
    for (int c = 0; c < kHD / 8; ++c) {
        const int d = 8 * c;
        const __half2 *hh = reinterpret_cast<const __half2 *>(&raw[c]);
        const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
        const float2 f2 = __half22float2(hh[2]), f3 = __half22float2(hh[3]);
        s0 += (double)f0.x * aq[d] + (double)f0.y * aq[d + 1];
        s1 += (double)f1.x * aq[d + 2] + (double)f1.y * aq[d + 3];
        s2 += (double)f2.x * aq[d + 4] + (double)f2.y * aq[d + 5];
        s3 += (double)f3.x * aq[d + 6] + (double)f3.y * aq[d + 7];
    }
    return __fmul_rn((float)((s0 + s1) + (s2 + s3)), scale);
}

// Attention of one (token t, query head h) unit per CTA (restates
// src/s2_model.cpp:979-1039: qk-norm, RoPE mode 0, f16 cache of past
// positions + f32 keys/values of this call, GQA h -> h / (H / Hkv), exact
// softmax, weighted value sum).
//
// Latency plan: every global load that does not depend on another is issued
// at the start of the unit -- q / k / v of this call, norm weights, RoPE
// (cos, sin) -- together with L2 prefetches of the cached key and value rows,
// so the key and value loads after the q / k normalization hit L2.  Scores stay in registers and the
// probabilities in shared memory (up to kAttnKeys keys; longer contexts go
// through the global score scratch).
__device__ void mega_attn(const MegaAttn &a, MSmem &sm, int cta, int G, int *err, unsigned long long *tr) {
    // tr (profiling, first unit only): [4] q/k/v normed and stored, [5] scores, [6] softmax, [7] values
    auto mark = [&](int u, int k) {
        if (tr != nullptr && u == cta && threadIdx.x == 0) tr[k] = globaltimer_ns();
    };
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int units = a.T * a.H;
    const int grp = a.H / a.Hkv;
    float *const pbuf = sm.nw;  // probabilities (the GEMV norm buffer is idle during attention)
    if (a.kv_k && cta < units && !sm.ptab_ready) {
        // the block table and n_past do not change within a segment: stage the
        // page ids once, at the first attention op this CTA runs
        const int nc = a.n_cached_from_pos_base && a.pos_base ? __ldcg(a.pos_base) : 0;
        const int npg = min((nc + kPage - 1) / kPage, kPtab);
        for (int i = tid; i < npg; i += kMNC) sm.ptab[i] = __ldcg(a.block_table + i);
        named_sync(3, kMNC);
        if (tid == 0) sm.ptab_ready = 1;
    }
    for (int u = cta; u < units; u += G) {
        const int t = u / a.H, h = u - t * a.H, g = h / grp;
        const int base = a.pos_base ? __ldcg(a.pos_base) : 0;
        const int nc = a.n_cached_from_pos_base ? base : 0;
        const int pos0 = base + a.pos_add;
        const int Lk = nc + a.cur_base + t + 1;
        const bool in_smem = Lk <= kAttnKeys;
        if (pos0 + t >= a.rope_positions && tid == 0) atomicOr(err, ERR_BAD_POS);
        // ---- A. independent loads ----
        const int i = tid & 63;
        const bool grp_q = tid < 64, grp_k = tid >= 64 && tid < 128, grp_v = tid >= 128 && tid < 192;
        float qx0 = 0.f, qx1 = 0.f, qn0 = 0.f, qn1 = 0.f;
        float2 qcs = make_float2(0.f, 0.f);
        float kx0[kMaxT], kx1[kMaxT], vx0[kMaxT], vx1[kMaxT];
        float2 kcs[kMaxT];
        float kn0 = 0.f, kn1 = 0.f;
        if (grp_q) {
            const float *src = a.qkv + (size_t)t * a.ldqkv + (size_t)h * kHD;
            qx0 = __ldcg(src + 2 * i);
            qx1 = __ldcg(src + 2 * i + 1);
            if (a.q_norm) {
                qn0 = __ldg(a.q_norm + 2 * i);
                qn1 = __ldg(a.q_norm + 2 * i + 1);
            }
            qcs = __ldg(a.rope + (size_t)min(pos0 + t, a.rope_positions - 1) * (kHD / 2) + i);
        }
#pragma unroll
        for (int tt = 0; tt < kMaxT; ++tt) {
            kx0[tt] = kx1[tt] = vx0[tt] = vx1[tt] = 0.f;
            kcs[tt] = make_float2(0.f, 0.f);
            if (tt <= t) {
                const float *row = a.qkv + (size_t)tt * a.ldqkv;
                if (grp_k) {
                    kx0[tt] = __ldcg(row + (size_t)(a.H + g) * kHD + 2 * i);
                    kx1[tt] = __ldcg(row + (size_t)(a.H + g) * kHD + 2 * i + 1);
                    kcs[tt] = __ldg(a.rope + (size_t)min(pos0 + tt, a.rope_positions - 1) * (kHD / 2) + i);
                }
                if (grp_v) {
                    vx0[tt] = __ldcg(row + (size_t)(a.H + a.Hkv + g) * kHD + 2 * i);
                    vx1[tt] = __ldcg(row + (size_t)(a.H + a.Hkv + g) * kHD + 2 * i + 1);
                }
            }
        }
        if (grp_k && a.k_norm) {
            kn0 = __ldg(a.k_norm + 2 * i);
            kn1 = __ldg(a.k_norm + 2 * i + 1);
        }
        // cached key and value rows -> L2 while q and k are normalized
        for (int j = tid; j < nc; j += kMNC) {
            const char *kp = reinterpret_cast<const char *>(kv_row(a, a.kv_k, sm.ptab, g, j));
            const char *vp = reinterpret_cast<const char *>(kv_row(a, a.kv_v, sm.ptab, g, j));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kp));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kp + 128));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(vp));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(vp + 128));
        }
        // ---- B. q: norm + RoPE ----
        head_norm_rope(qx0, qx1, a.q_norm != nullptr, qn0, qn1, a.eps, qcs, 0, sm, grp_q);
        if (grp_q) {
            sm.aq[2 * i] = qx0;
            sm.aq[2 * i + 1] = qx1;
            sm.aqd[2 * i] = (double)qx0;
            sm.aqd[2 * i + 1] = (double)qx1;
        }
        // ---- C. k, v of this call's tokens 0..t ----
        for (int tt = 0; tt <= t; ++tt) {
            float x0 = kx0[0], x1 = kx1[0];
            float2 cs = kcs[0];
#pragma unroll
            for (int q = 1; q < kMaxT; ++q)
                if (q == tt) {
                    x0 = kx0[q];
                    x1 = kx1[q];
                    cs = kcs[q];
                }
            // k pairs sit on threads 64..127 (warps 2, 3): reduction slots 2, 3
            head_norm_rope(x0, x1, a.k_norm != nullptr, kn0, kn1, a.eps, cs, 2, sm, grp_k);
            if (grp_k) {
                sm.ak[tt][2 * i] = x0;
                sm.ak[tt][2 * i + 1] = x1;
            }
            if (grp_v) {
                float v0 = vx0[0], v1 = vx1[0];
#pragma unroll
                for (int q = 1; q < kMaxT; ++q)
                    if (q == tt) {
                        v0 = vx0[q];
                        v1 = vx1[q];
                    }
                sm.av[tt][2 * i] = v0;
                sm.av[tt][2 * i + 1] = v1;
            }
        }
        named_sync(3, kMNC);
        // the first query head of the group stores token t's K/V
        if (h % grp == 0 && tid < kHD) {
            const size_t ci = ((size_t)(a.cur_base + t) * a.Hkv + g) * kHD + tid;
            a.kcur[ci] = sm.ak[t][tid];
            a.vcur[ci] = sm.av[t][tid];
            if (a.kv_k) {
                const int pos = pos0 + t, pg = pos / kPage, slot = pos % kPage;
                if (pos >= 0 && pg < a.kv_pages) {
                    const int page = __ldcg(a.block_table + pg);
                    const size_t off = ((((size_t)page * a.kv_layers + a.layer) * a.Hkv + g) * kPage + slot) * kHD + tid;
                    a.kv_k[off] = __float2half_rn(sm.ak[t][tid]);
                    a.kv_v[off] = __float2half_rn(sm.av[t][tid]);
                } else if (tid == 0) {
                    atomicOr(err, ERR_BAD_POS);
                }
            }
        }
        mark(u, 4);
        // ---- D. scores -> sc (pbuf in shared memory when the keys fit) ----
        float *const sc = in_smem ? pbuf : a.scores + (size_t)u * a.ld_scores;
        // cached keys: one f16 row per thread (rows were prefetched into L2)
        for (int j = tid; j < nc; j += kMNC) {
            const uint4 *kp = reinterpret_cast<const uint4 *>(kv_row(a, a.kv_k, sm.ptab, g, j));
            uint4 raw[kHD / 8];
#pragma unroll
            for (int c = 0; c < kHD / 8; ++c) raw[c] = __ldcg(kp + c);
            sc[j] = key_score(raw, sm.aqd, a.scale);
        }
        // keys of this call (f32 rows): one warp per key, lane = 4 dims
        for (int c = warp; c < Lk - nc; c += kMW) {
            const bool gl = c < a.cur_base;
            const float4 k4 = gl ? __ldcg(reinterpret_cast<const float4 *>(key_ptr_f32(a, sm, c, g, false)) + lane)
                                 : reinterpret_cast<const float4 *>(key_ptr_f32(a, sm, c, g, false))[lane];
            double p = (double)k4.x * sm.aqd[4 * lane] + (double)k4.y * sm.aqd[4 * lane + 1] +
                       (double)k4.z * sm.aqd[4 * lane + 2] + (double)k4.w * sm.aqd[4 * lane + 3];
            p = warp_sum_d(p);
            if (lane == 0) sc[nc + c] = __fmul_rn((float)p, a.scale);
        }
        named_sync(3, kMNC);
        mark(u, 5);
        // ---- E. exact softmax: max, sum in double, p' = exp(s - max) * (1 / sum) ----
        float mx = -INFINITY;
        for (int j = tid; j < Lk; j += kMNC) mx = fmaxf(mx, sc[j]);
        mx = warp_max(mx);
        if (lane == 0) sm.red_f[warp] = mx;
        named_sync(3, kMNC);
        mx = sm.red_f[0];
        for (int w = 1; w < kMW; ++w) mx = fmaxf(mx, sm.red_f[w]);
        double sum = 0.0;
        for (int j = tid; j < Lk; j += kMNC) sum += (double)det_expf(__fsub_rn(sc[j], mx));
        sum = warp_sum_d(sum);
        if (lane == 0) sm.red_d[warp] = sum;
        named_sync(3, kMNC);
        double tot = 0.0;
        for (int w = 0; w < kMW; ++w) tot += sm.red_d[w];
        const float inv = (float)(1.0 / tot);
        for (int j = tid; j < Lk; j += kMNC) sc[j] = __fmul_rn(det_expf(__fsub_rn(sc[j], mx)), inv);
        float *const pr = sc;
        named_sync(3, kMNC);
        mark(u, 6);
        // ---- F. values: warp w takes keys w, w + kMW, ...; lane takes dims 4*lane..4*lane+3;
        // kVU keys per warp are loaded before any is used (rows were prefetched into L2) ----
        {
            constexpr int kVU = 16;
            double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
            int j = warp;
            for (; j + (kVU - 1) * kMW < nc; j += kVU * kMW) {
                uint2 raw[kVU];
#pragma unroll
                for (int q = 0; q < kVU; ++q)
                    raw[q] = __ldcg(reinterpret_cast<const uint2 *>(kv_row(a, a.kv_v, sm.ptab, g, j + q * kMW) + 4 * lane));
#pragma unroll
                for (int q = 0; q < kVU; ++q) {
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&raw[q]);
                    const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                    const double pd = (double)pr[j + q * kMW];
                    acc0 += (double)f0.x * pd;
                    acc1 += (double)f0.y * pd;
                    acc2 += (double)f1.x * pd;
                    acc3 += (double)f1.y * pd;
                }
            }
            for (; j < nc; j += kMW) {
                const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(kv_row(a, a.kv_v, sm.ptab, g, j) + 4 * lane));
                const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
                const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                const double pd = (double)pr[j];
                acc0 += (double)f0.x * pd;
                acc1 += (double)f0.y * pd;
                acc2 += (double)f1.x * pd;
                acc3 += (double)f1.y * pd;
            }
            // keys of this call (f32): j = nc + c
            for (int c = warp; c < Lk - nc; c += kMW) {
                const float *vp = key_ptr_f32(a, sm, c, g, true) + 4 * lane;
                const bool gl = c < a.cur_base;
                const float v0 = gl ? __ldcg(vp) : vp[0], v1 = gl ? __ldcg(vp + 1) : vp[1];
                const float v2 = gl ? __ldcg(vp + 2) : vp[2], v3 = gl ? __ldcg(vp + 3) : vp[3];
                const double pd = (double)pr[nc + c];
                acc0 += (double)v0 * pd;
                acc1 += (double)v1 * pd;
                acc2 += (double)v2 * pd;
                acc3 += (double)v3 * pd;
            }
            sm.vpart[warp][4 * lane] = acc0;
            sm.vpart[warp][4 * lane + 1] = acc1;
            sm.vpart[warp][4 * lane + 2] = acc2;
            sm.vpart[warp][4 * lane + 3] = acc3;
        }
        named_sync(3, kMNC);
        mark(u, 7);
        if (tid < kHD) {
            double o = sm.vpart[0][tid];
            for (int k = 1; k < kMW; ++k) o += sm.vpart[k][tid];
            a.out[(size_t)t * a.H * kHD + (size_t)h * kHD + tid] = (float)o;
        }
        named_sync(3, kMNC);
    }
}

__device__ void mega_embed_slow(const MegaEmbedSlow &e, int cta, int G, int *err) {
    const int stride = e.ncb + 1;
    for (long long idx = (long long)cta * kMNC + threadIdx.x; idx < (long long)e.T * e.dim; idx += (long long)G * kMNC) {
        const int t = (int)(idx / e.dim), i = (int)(idx - (long long)t * e.dim);
        int tok = __ldcg(e.tokens + t * stride);
        if (tok < 0 || tok >= e.e_rows) {
            if (i == 0) atomicOr(err, ERR_BAD_TOKEN);
            tok = 0;
        }
        const bool sem = tok >= e.sem_begin && tok <= e.sem_end;
        float x = tq_elem(e.e, e.dim, tok, i);
        if (sem && e.ncb > 0) {
            float s = 0.f;
            for (int cb = 0; cb < e.ncb; ++cb) {
                int id = __ldcg(e.tokens + t * stride + 1 + cb) + cb * e.cb_size;
                if (id < 0 || id >= e.c_rows) {
                    if (i == 0) atomicOr(err, ERR_BAD_TOKEN);
                    id = 0;
                }
                const float r = tq_elem(e.c, e.dim, id, i);
                s = cb == 0 ? r : __fadd_rn(s, r);
            }
            x = __fadd_rn(x, s);
        }
        if (e.scale_cb && sem) x = __fmul_rn(x, e.sem_scale);
        e.x[(size_t)t * e.dim + i] = x;
    }
}

__device__ void mega_embed_fast(const MegaEmbedFast &e, int cta, int G, int *err) {
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
            x = tq_elem(e.f, e.dim, c, i);
        }
        e.x[(size_t)r * e.dim + i] = x;
    }
}

template <int MT>
__global__ void __launch_bounds__(kMThreads, 1)
    mega_kernel(const MegaOp *__restrict__ ops, int n_ops, MegaCtl *ctl, const int *done, int *err, int l2_ahead,
                unsigned long long *trace, int flags) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    MSmem &sm = *reinterpret_cast<MSmem *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (done != nullptr && __ldcg(done) != 0) return;  // finished sequence: the whole grid exits
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kMW);
        }
        fence_mbar_init();
        sm.ptab_ready = 0;
    }
    __syncthreads();
    if (warp == kMW) {
        if (lane == 0) mega_producer(ops, n_ops, sm, cta, G, l2_ahead, err, trace);
        return;
    }
    // trace: per op and CTA, [start, prologue done, work done, producer's last tile issued]
    auto stamp = [&](int i, int k) {
        if (trace != nullptr && threadIdx.x == 0) trace[((size_t)i * G + cta) * kTraceSlots + k] = globaltimer_ns();
    };
    int cslot = 0;  // ring position of the consumers
    uint32_t cphase = 0;
    for (int i = 0; i < n_ops; ++i) {
        const int kind = ops[i].kind;
        // RMSNorm weights of the next GEMV do not depend on the previous op: load them before the barrier
        F8 nw[kMPC];
        if (kind == MK_GEMV) tg_norm_preload<kMPC, kMNC>(ops[i].g, nw);
        if (i > 0) grid_wait(ctl, (unsigned)(i * G), err);
        stamp(i, 0);
        stamp(i, 1);
        switch (kind) {
        case MK_GEMV:
            mega_gemv<MT>(ops[i].g, nw, sm, cta, G, cslot, cphase, err,
                          trace != nullptr ? trace + ((size_t)i * G + cta) * kTraceSlots : nullptr);
            break;
        case MK_ATTN:
            mega_attn(ops[i].a, sm, cta, G, err, trace != nullptr ? trace + ((size_t)i * G + cta) * kTraceSlots : nullptr);
            break;
        case MK_EMBED_SLOW: mega_embed_slow(ops[i].es, cta, G, err); break;
        case MK_EMBED_FAST: mega_embed_fast(ops[i].ef, cta, G, err); break;
        case MK_ADVANCE:
            if (cta == 0 && threadIdx.x == 0) {
                volatile int *np = ops[i].adv.n_past;
                *np = *np + ops[i].adv.T;
            }
            break;
        default: break;
        }
        stamp(i, 2);
        grid_arrive(ctl, flags);
    }
    if (trace != nullptr) {
        grid_wait(ctl, (unsigned)(n_ops * G), err);
        stamp(n_ops, 0);
    }
}

// Tiles per CTA the producer prefetches into L2 beyond its ring: 148 CTAs x
// 24 tiles x 17 KB = 62 MB of the 126 MB L2.  S2K_L2_AHEAD (read at each
// launch or graph capture) overrides it; 0 turns the run-ahead off.
int mega_l2_ahead() {
    const char *e = getenv("S2K_L2_AHEAD");
    const int d = e ? atoi(e) : 0;
    return d < 0 ? 0 : (d > 64 ? 64 : d);
}

cudaError_t mega_setup() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(mega_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem))))
        return e;
    return cudaFuncSetAttribute(mega_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem));
}

cudaError_t launch_mega(const MegaOp *d_ops, int n_ops, int mt, MegaCtl *ctl, const int *done, int *err, int num_sms,
                        cudaStream_t st, unsigned long long *trace) {
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
    const char *fe = getenv("S2K_MEGA_FLAGS");
    const int flags = fe ? atoi(fe) : 0;
    if (mt == 1) return cudaLaunchKernelEx(&cfg, mega_kernel<1>, d_ops, n_ops, ctl, done, err, ahead, trace, flags);
    return cudaLaunchKernelEx(&cfg, mega_kernel<2>, d_ops, n_ops, ctl, done, err, ahead, trace, flags);
}

}  // namespace s2k
