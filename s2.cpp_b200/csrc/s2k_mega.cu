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

namespace s2k {

// 8 consumer warps (the tile engine's mapping, s2k_tgemv.cuh) + 1 producer.
constexpr int kMW = kTW;                   // consumer warps
constexpr int kMNC = kMW * 32;             // consumer threads
constexpr int kMThreads = kMNC + 32;       // + producer warp
constexpr int kMStages = 10;               // ring of 17 KB weight tiles
constexpr int kMKMax = 10240;
constexpr int kMaxT = 2;
constexpr int kHD = 128;
constexpr int kPtabMax = kMaxT * kMKMax / (int)sizeof(int);  // cached pages whose ids fit the staged table

bool mega_gemv_ok(const MegaGemv &g) {
    if (!tg_shape_ok(g.R, g.K, g.M, g.in_mode, g.epi, g.res != nullptr, kMKMax, kMaxT)) return false;
    if (g.in_mode == IN_RMSNORM && g.norm_w == nullptr) return false;
    return true;
}

struct MSmem {
    uint8_t ring[kMStages][kTileBytes];
    uint64_t full[kMStages], empty[kMStages];
    int8_t xq[kMaxT * kMKMax];  // quantized activation (GEMV); page table (attention)
    float xd[kMaxT * kMKMax / 32];
    float nw[kNormMax];
    double tok[kMW][kMaxT];
    float scale[kMaxT];
    // attention
    float aq[kHD];
    float ak[kMaxT][kHD], av[kMaxT][kHD];
    double vpart[kMW][kHD];
    float red_f[kMW];
    double red_d[kMW];
};

static_assert(sizeof(MSmem) <= 227 * 1024, "persistent kernel shared memory exceeds the per-CTA limit");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// consumer-only grid barrier halves
__device__ __forceinline__ void grid_arrive(MegaCtl *ctl) {
    named_sync(1, kMNC);
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(&ctl->count, 1u);
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
__device__ void mega_producer(const MegaOp *ops, int n_ops, MSmem &sm, int cta, int G, int *err) {
    const uint64_t pol = policy_evict_first();
    int ps = 0;
    for (int i = 0; i < n_ops; ++i) {
        if (ops[i].kind != MK_GEMV) continue;
        const MegaGemv g = ops[i].g;
        long long u0, u1;
        tg_range(g.R, g.K, cta, G, &u0, &u1);
        for (long long u = u0; u < u1; ++u, ++ps) {
            const int slot = ps % kMStages;
            if (ps >= kMStages && !mbar_wait(&sm.empty[slot], ((ps / kMStages) - 1) & 1, err, ERR_WAIT_EMPTY))
                return;
            mbar_arrive_expect_tx(&sm.full[slot], kTileBytes);
            bulk_g2s(sm.ring[slot], g.w + (size_t)u * kTileBytes, kTileBytes, &sm.full[slot], pol);
        }
    }
}

// ---------------------------------------------------------------------------
// GEMV op (consumer side): activation prologue, then this CTA's tiles
// ---------------------------------------------------------------------------
template <int MT>
__device__ void mega_gemv(const MegaGemv &gref, MSmem &sm, int cta, int G, int &slot, uint32_t &phase, int *err) {
    const MegaGemv g = gref;  // op fields in registers
    long long u0, u1;
    tg_range(g.R, g.K, cta, G, &u0, &u1);
    if (u0 == u1) return;  // no row tile of this op here (R / 32 < G)
    // the CTA owning row tile 0 stores act_out
    tg_prologue<MT, kMNC>(g, sm.xq, sm.xd, sm.nw, &sm.tok[0][0], kMaxT, sm.scale, u0 == 0, 1);
    named_sync(1, kMNC);
    tg_consume<MT>(g, &sm.ring[0][0], sm.full, sm.empty, kMStages, slot, phase, sm.xq, sm.xd, cta, G, err);
}

// ---------------------------------------------------------------------------
// attention op: one CTA per (token, query head) unit
// ---------------------------------------------------------------------------
// x0/x1 = pair (2i, 2i+1) of a head vector held by 64 threads (i = thread);
// optional per-head RMSNorm (reduction over the 64 threads of warps w0, w0+1)
// then RoPE from the table.
__device__ __forceinline__ void head_norm_rope(float &x0, float &x1, const float *nw, float eps, const float2 *rope,
                                               int pos, int i, int red_slot, MSmem &sm, bool active) {
    if (nw) {
        double s = active ? (double)__fmul_rn(x0, x0) + (double)__fmul_rn(x1, x1) : 0.0;
        s = warp_sum_d(s);
        if ((threadIdx.x & 31) == 0 && threadIdx.x < 64) sm.red_d[red_slot + (threadIdx.x >> 5)] = s;
    }
    named_sync(3, kMNC);
    if (active) {
        if (nw) {
            const double tot = sm.red_d[red_slot] + sm.red_d[red_slot + 1];
            const float mean = (float)(tot / (double)kHD);
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
            x0 = __fmul_rn(__fmul_rn(x0, sc), nw[2 * i]);
            x1 = __fmul_rn(__fmul_rn(x1, sc), nw[2 * i + 1]);
        }
        const float2 cs = rope[(size_t)pos * (kHD / 2) + i];
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

// Row of cached key/value position j for kv head g in the paged f16 cache.
__device__ __forceinline__ const __half *kv_row(const MegaAttn &a, const __half *base, const int *ptab, int g, int j) {
    const int pg = j / kPage, slot = j - pg * kPage;
    const int page = pg < kPtabMax ? ptab[pg] : __ldcg(a.block_table + pg);
    return base + ((((size_t)page * a.kv_layers + a.layer) * a.Hkv + g) * kPage + slot) * kHD;
}

__device__ void mega_attn(const MegaAttn &a, MSmem &sm, int cta, int G, int *err) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int *const ptab = reinterpret_cast<int *>(sm.xq);
    const int units = a.T * a.H;
    const int grp = a.H / a.Hkv;
    for (int u = cta; u < units; u += G) {
        const int t = u / a.H, h = u - t * a.H, g = h / grp;
        const int base = a.pos_base ? __ldcg(a.pos_base) : 0;
        const int nc = a.n_cached_from_pos_base ? base : 0;
        const int pos0 = base + a.pos_add;
        // page table of the cached keys, staged in the (idle) GEMV activation buffer
        const int npg = a.kv_k ? (nc + kPage - 1) / kPage : 0;
        for (int i = tid; i < min(npg, kPtabMax); i += kMNC) ptab[i] = __ldcg(a.block_table + i);
        // 1. q of (t, h): threads 0..63 (pair i)
        {
            const bool act = tid < 64;
            const int i = tid & 63;
            float x0 = 0.f, x1 = 0.f;
            if (act) {
                const float *src = a.qkv + (size_t)t * a.ldqkv + (size_t)h * kHD;
                x0 = __ldcg(src + 2 * i);
                x1 = __ldcg(src + 2 * i + 1);
            }
            if (pos0 + t >= a.rope_positions) {
                if (tid == 0) atomicOr(err, ERR_BAD_POS);
            }
            head_norm_rope(x0, x1, a.q_norm, a.eps, a.rope, min(pos0 + t, a.rope_positions - 1), i,
                           0, sm, act);
            if (act) {
                sm.aq[2 * i] = x0;
                sm.aq[2 * i + 1] = x1;
            }
        }
        // 2. k, v of the op's tokens 0..t for kv head g
        for (int tt = 0; tt <= t; ++tt) {
            const bool actk = tid < 64, actv = tid >= 64 && tid < 128;
            const int i = tid & 63;
            const float *row = a.qkv + (size_t)tt * a.ldqkv;
            float x0 = 0.f, x1 = 0.f;
            if (actk) {
                x0 = __ldcg(row + (size_t)(a.H + g) * kHD + 2 * i);
                x1 = __ldcg(row + (size_t)(a.H + g) * kHD + 2 * i + 1);
            }
            head_norm_rope(x0, x1, a.k_norm, a.eps, a.rope, min(pos0 + tt, a.rope_positions - 1), i, 2, sm, actk);
            if (actk) {
                sm.ak[tt][2 * i] = x0;
                sm.ak[tt][2 * i + 1] = x1;
            }
            if (actv) {
                sm.av[tt][2 * i] = __ldcg(row + (size_t)(a.H + a.Hkv + g) * kHD + 2 * i);
                sm.av[tt][2 * i + 1] = __ldcg(row + (size_t)(a.H + a.Hkv + g) * kHD + 2 * i + 1);
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
        // 3. scores
        const int Lk = nc + a.cur_base + t + 1;
        float *sc = a.scores + (size_t)u * a.ld_scores;
        float mx = -INFINITY;
        for (int j = tid; j < Lk; j += kMNC) {
            double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
            if (j < nc) {
                // the whole 256-byte key row in flight at once
                const uint4 *kp = reinterpret_cast<const uint4 *>(kv_row(a, a.kv_k, ptab, g, j));
                uint4 raw[kHD / 8];
#pragma unroll
                for (int c = 0; c < kHD / 8; ++c) raw[c] = __ldcg(kp + c);
#pragma unroll
                for (int c = 0; c < kHD / 8; ++c) {
                    const int d = 8 * c;
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&raw[c]);
                    const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                    const float2 f2 = __half22float2(hh[2]), f3 = __half22float2(hh[3]);
                    s0 += (double)f0.x * (double)sm.aq[d] + (double)f0.y * (double)sm.aq[d + 1];
                    s1 += (double)f1.x * (double)sm.aq[d + 2] + (double)f1.y * (double)sm.aq[d + 3];
                    s2 += (double)f2.x * (double)sm.aq[d + 4] + (double)f2.y * (double)sm.aq[d + 5];
                    s3 += (double)f3.x * (double)sm.aq[d + 6] + (double)f3.y * (double)sm.aq[d + 7];
                }
            } else {
                const int c = j - nc;
                const float *kp = key_ptr_f32(a, sm, c, g, false);
                const bool gl = c < a.cur_base;
#pragma unroll 4
                for (int d = 0; d < kHD; d += 4) {
                    const float k0 = gl ? __ldcg(kp + d) : kp[d], k1 = gl ? __ldcg(kp + d + 1) : kp[d + 1];
                    const float k2 = gl ? __ldcg(kp + d + 2) : kp[d + 2], k3 = gl ? __ldcg(kp + d + 3) : kp[d + 3];
                    s0 += (double)k0 * (double)sm.aq[d];
                    s1 += (double)k1 * (double)sm.aq[d + 1];
                    s2 += (double)k2 * (double)sm.aq[d + 2];
                    s3 += (double)k3 * (double)sm.aq[d + 3];
                }
            }
            const float s = __fmul_rn((float)((s0 + s1) + (s2 + s3)), a.scale);
            sc[j] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        if (lane == 0) sm.red_f[warp] = mx;
        named_sync(3, kMNC);
        mx = sm.red_f[0];
        for (int w = 1; w < kMW; ++w) mx = fmaxf(mx, sm.red_f[w]);
        double sum = 0.0;
        for (int j = tid; j < Lk; j += kMNC) sum += (double)det_expf(__fsub_rn(sc[j], mx));
        sum = warp_sum_d(sum);
        named_sync(3, kMNC);  // red_f reads done before red_d / red_f reuse
        if (lane == 0) sm.red_d[warp] = sum;
        named_sync(3, kMNC);
        double tot = 0.0;
        for (int w = 0; w < kMW; ++w) tot += sm.red_d[w];
        const float inv = (float)(1.0 / tot);
        for (int j = tid; j < Lk; j += kMNC) sc[j] = __fmul_rn(det_expf(__fsub_rn(sc[j], mx)), inv);
        named_sync(3, kMNC);
        // 4. values: warp w takes keys w, w + kMW, ...; lane takes dims 4*lane..4*lane+3.
        // kVU keys per warp are loaded before any is used.
        {
            constexpr int kVU = 8;
            double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0;
            int j = warp;
            for (; j + (kVU - 1) * kMW < nc; j += kVU * kMW) {
                uint2 raw[kVU];
                float pr[kVU];
#pragma unroll
                for (int q = 0; q < kVU; ++q) {
                    const int jj = j + q * kMW;
                    raw[q] = __ldcg(reinterpret_cast<const uint2 *>(kv_row(a, a.kv_v, ptab, g, jj) + 4 * lane));
                    pr[q] = sc[jj];
                }
#pragma unroll
                for (int q = 0; q < kVU; ++q) {
                    const __half2 *hh = reinterpret_cast<const __half2 *>(&raw[q]);
                    const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                    const double pd = (double)pr[q];
                    acc0 += (double)f0.x * pd;
                    acc1 += (double)f0.y * pd;
                    acc2 += (double)f1.x * pd;
                    acc3 += (double)f1.y * pd;
                }
            }
            for (; j < nc; j += kMW) {
                const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(kv_row(a, a.kv_v, ptab, g, j) + 4 * lane));
                const __half2 *hh = reinterpret_cast<const __half2 *>(&raw);
                const float2 f0 = __half22float2(hh[0]), f1 = __half22float2(hh[1]);
                const double pd = (double)sc[j];
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
                const double pd = (double)sc[nc + c];
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
    mega_kernel(const MegaOp *__restrict__ ops, int n_ops, MegaCtl *ctl, const int *done, int *err) {
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
    }
    __syncthreads();
    if (warp == kMW) {
        if (lane == 0) mega_producer(ops, n_ops, sm, cta, G, err);
        return;
    }
    int cslot = 0;  // ring position of the consumers
    uint32_t cphase = 0;
    for (int i = 0; i < n_ops; ++i) {
        const int kind = ops[i].kind;
        if (i > 0) grid_wait(ctl, (unsigned)(i * G), err);
        switch (kind) {
        case MK_GEMV: mega_gemv<MT>(ops[i].g, sm, cta, G, cslot, cphase, err); break;
        case MK_ATTN: mega_attn(ops[i].a, sm, cta, G, err); break;
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
        grid_arrive(ctl);
    }
}

cudaError_t mega_setup() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(mega_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem))))
        return e;
    return cudaFuncSetAttribute(mega_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MSmem));
}

cudaError_t launch_mega(const MegaOp *d_ops, int n_ops, int mt, MegaCtl *ctl, const int *done, int *err, int num_sms,
                        cudaStream_t st) {
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
    if (mt == 1) return cudaLaunchKernelEx(&cfg, mega_kernel<1>, d_ops, n_ops, ctl, done, err);
    return cudaLaunchKernelEx(&cfg, mega_kernel<2>, d_ops, n_ops, ctl, done, err);
}

}  // namespace s2k
