// s2k_mega.cu -- persistent decode kernel: one cooperative launch runs a whole
// segment of the decode step (a Fast-AR pass, or the Slow-AR step) on one CTA
// per SM.
//
// Why: at batch 1 every op is a short, memory-bound GEMV (1.6-8 us of HBM
// time for the per-layer matrices).  Launched as separate kernels, each op
// pays launch, dependency and prologue latency while HBM idles.  Here a
// producer warp per CTA streams the CTA's rows of every GEMV of the segment,
// back to back, through a 7-stage shared-memory ring (cp.async.bulk +
// mbarriers); it runs ahead across op boundaries, so HBM keeps streaming while
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

// 12 consumer warps + 1 producer: at most 4 warps per SM sub-partition, so
// each thread can hold 128 registers.
constexpr int kMW = 12;                    // consumer warps
constexpr int kMNC = kMW * 32;             // consumer threads
constexpr int kMThreads = kMNC + 32;       // + producer warp
constexpr int kMStages = 4;
constexpr int kMSlot = 40 * 1024;
constexpr int kCPL = 5;                    // 16-byte weight chunks per lane per row slice
constexpr int kMKMax = 10240;
constexpr int kMNormMax = 4096;
constexpr int kMMaxRows = 64;
constexpr int kMaxT = 2;
constexpr int kHD = 128;
constexpr int kPtabMax = kMaxT * kMKMax / (int)sizeof(int);  // cached pages whose ids fit the staged table

struct MStage {
    int S, WPR, BPL;
};

// S rows per stage and WPR warps per row with S * WPR = kMW; BPL = 16-byte
// chunks per lane of a row slice.
__host__ __device__ inline MStage mega_stage(int K) {
    const int row_bytes = K + K / 16;
    const int cand[6] = {12, 6, 4, 3, 2, 1};
    int S = 1;
    for (int i = 0; i < 6; ++i)
        if (cand[i] * row_bytes <= kMSlot) {
            S = cand[i];
            break;
        }
    MStage r;
    r.S = S;
    r.WPR = kMW / S;
    const int NC = K / 16;
    const int CPS = (NC + r.WPR - 1) / r.WPR;
    r.BPL = (CPS + 31) / 32;
    return r;
}

bool mega_gemv_ok(const MegaGemv &g) {
    if (g.K % 256 != 0 || g.K > kMKMax || g.M < 1 || g.M > kMaxT || g.R <= 0) return false;
    const MStage st = mega_stage(g.K);
    if (st.S * (g.K + g.K / 16) > kMSlot || st.BPL > kCPL) return false;
    if (g.in_mode == IN_RMSNORM && g.K > kMNormMax) return false;
    if (g.epi == EPI_SWIGLU && (g.R % 2 != 0 || g.res != nullptr)) return false;
    return true;
}

struct MSmem {
    uint8_t ring[kMStages][kMSlot];
    uint64_t full[kMStages], empty[kMStages];
    int8_t xq[kMaxT * kMKMax];
    float xd[kMaxT * kMKMax / 32];
    float nw[kMNormMax];
    float res[kMaxT * kMMaxRows];
    double rowacc[kMStages][kMW][kMaxT];  // cross-warp row partials of a stage
    int rowcnt[kMStages][kMW];            // arrivals per row (unit) of a stage
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
        if (ld_acquire_u32(&ctl->count) < target) {
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

__device__ __forceinline__ void gemv_rows(const MegaGemv &g, int cta, int G, int *r0, int *r1) {
    const int unit = g.epi == EPI_SWIGLU ? 2 : 1;
    const int NU = g.R / unit;
    *r0 = unit * (int)(((long long)NU * cta) / G);
    *r1 = unit * (int)(((long long)NU * (cta + 1)) / G);
}

// ---------------------------------------------------------------------------
// producer: the weight stream of every GEMV op of the segment
// ---------------------------------------------------------------------------
__device__ void mega_producer(const MegaOp *ops, int n_ops, MSmem &sm, int cta, int G, int *err) {
    const uint64_t pol = policy_evict_first();
    int ps = 0;
    for (int i = 0; i < n_ops; ++i) {
        if (ops[i].kind != MK_GEMV) continue;
        const MegaGemv g = ops[i].g;
        int r0, r1;
        gemv_rows(g, cta, G, &r0, &r1);
        const MStage st = mega_stage(g.K);
        for (int rb = r0; rb < r1; rb += st.S, ++ps) {
            const int slot = ps % kMStages;
            if (ps >= kMStages && !mbar_wait(&sm.empty[slot], ((ps / kMStages) - 1) & 1, err, ERR_WAIT_EMPTY))
                return;
            const int rows = min(st.S, r1 - rb);
            const uint32_t qb = (uint32_t)rows * (uint32_t)g.K;
            const uint32_t db = (uint32_t)rows * (uint32_t)(g.K / 16);
            mbar_arrive_expect_tx(&sm.full[slot], qb + db);
            bulk_g2s(sm.ring[slot], g.wq + (size_t)rb * g.K, qb, &sm.full[slot], pol);
            bulk_g2s(sm.ring[slot] + (size_t)st.S * g.K, reinterpret_cast<const uint8_t *>(g.wd) + (size_t)rb * (g.K / 16),
                     db, &sm.full[slot], pol);
        }
    }
}

__device__ __forceinline__ int dot_block8(const int4 &w0, const int4 &w1, const int (&xb)[8]) {
    int s0 = dp4a(w0.x, xb[0], 0);
    int s1 = dp4a(w1.x, xb[4], 0);
    s0 = dp4a(w0.y, xb[1], s0);
    s1 = dp4a(w1.y, xb[5], s1);
    s0 = dp4a(w0.z, xb[2], s0);
    s1 = dp4a(w1.z, xb[6], s1);
    s0 = dp4a(w0.w, xb[3], s0);
    s1 = dp4a(w1.w, xb[7], s1);
    return s0 + s1;
}

// ---------------------------------------------------------------------------
// GEMV op (consumer side)
// ---------------------------------------------------------------------------
// Lane 0 of a warp holding a row slice's sum: combine the row's slices (and
// the gate/up pair) in shared memory; the last warp to arrive writes the
// output.  The terms are exact, so the arrival order does not change the
// rounded result.
template <int MT>
__device__ __forceinline__ void combine_row(MSmem &sm, int slot, int row_local, int unit, int need, int M,
                                            const double (&acc)[MT], int epi, float *y, int ldy, int rb, int r0,
                                            const float *res) {
    if (need == 1) {
        const int r = rb + row_local;
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (m < M) {
                const float val = (float)acc[m];
                y[(size_t)m * ldy + r] = res ? sm.res[m * kMMaxRows + (r - r0)] + val : val;
            }
        return;
    }
    const int grp = row_local / unit;
#pragma unroll
    for (int m = 0; m < MT; ++m)
        if (m < M) atomicAdd(&sm.rowacc[slot][row_local][m], acc[m]);
    __threadfence_block();
    if (atomicAdd(&sm.rowcnt[slot][grp], 1) != need - 1) return;
    __threadfence_block();
    volatile double *ra = &sm.rowacc[slot][0][0];
    if (epi == EPI_SWIGLU) {
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (m < M) {
                const double gg = ra[(2 * grp) * kMaxT + m], up = ra[(2 * grp + 1) * kMaxT + m];
                y[(size_t)m * ldy + rb / 2 + grp] = __fmul_rn(silu((float)gg), (float)up);
                ra[(2 * grp) * kMaxT + m] = 0.0;
                ra[(2 * grp + 1) * kMaxT + m] = 0.0;
            }
    } else {
        const int r = rb + row_local;
#pragma unroll
        for (int m = 0; m < MT; ++m)
            if (m < M) {
                const float val = (float)ra[row_local * kMaxT + m];
                y[(size_t)m * ldy + r] = res ? sm.res[m * kMMaxRows + (r - r0)] + val : val;
                ra[row_local * kMaxT + m] = 0.0;
            }
    }
    sm.rowcnt[slot][grp] = 0;
}

template <int MT>
__device__ void mega_gemv(const MegaGemv &gref, MSmem &sm, int cta, int G, int &cs, int *err) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // op fields in registers (stores through y must not force re-reads of the op)
    const int K = gref.K, R = gref.R, M = gref.M, ldx = gref.ldx, ldy = gref.ldy, ldres = gref.ldres;
    const int in_mode = gref.in_mode, epi = gref.epi;
    const float eps = gref.eps;
    const float *const x = gref.x;
    const float *const res = gref.res;
    const float *const norm_w = gref.norm_w;
    float *const y = gref.y;
    float *const act_out = gref.act_out;
    const int NB = K >> 5;
    const int unit = epi == EPI_SWIGLU ? 2 : 1;
    const int NU = R / unit;
    const int r0 = unit * (int)(((long long)NU * cta) / G);
    const int r1 = unit * (int)(((long long)NU * (cta + 1)) / G);
    if (r1 <= r0) return;
    const MStage st = mega_stage(K);

    if (in_mode == IN_RMSNORM)
        for (int i = tid; i < K / 4; i += kMNC)
            reinterpret_cast<float4 *>(sm.nw)[i] = __ldg(reinterpret_cast<const float4 *>(norm_w) + i);
    const int nrows = r1 - r0;
    if (res != nullptr)
        for (int i = tid; i < M * nrows; i += kMNC) {
            const int m = i / nrows, r = i - m * nrows;
            sm.res[m * kMMaxRows + r] = __ldcg(res + (size_t)m * ldres + r0 + r);
        }

    // activation -> Q8_0 blocks in shared memory; one block per thread
    const int items = M * NB;
    const bool single = items <= kMNC;
    {
        float4 v[8];
        if (in_mode == IN_RMSNORM) {
            double tk[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) tk[m] = 0.0;
            for (int it = tid; it < items; it += kMNC) {
                const int m = it / NB, b = it - m * NB;
                const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)m * ldx + b * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + j);
                double s = 0.0;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    s += (double)__fmul_rn(v[j].x, v[j].x) + (double)__fmul_rn(v[j].y, v[j].y) +
                         (double)__fmul_rn(v[j].z, v[j].z) + (double)__fmul_rn(v[j].w, v[j].w);
#pragma unroll
                for (int mm = 0; mm < MT; ++mm)
                    if (mm == m) tk[mm] += s;
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const double t = warp_sum_d(tk[m]);
                if (lane == 0) sm.tok[warp][m] = t;
            }
            named_sync(1, kMNC);
            if (tid < M) {
                double tot = 0.0;
                for (int w = 0; w < kMW; ++w) tot += sm.tok[w][tid];
                const float mean = (float)(tot / (double)K);
                sm.scale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
            }
            named_sync(1, kMNC);
        }
        for (int it = tid; it < items; it += kMNC) {
            const int m = it / NB, b = it - m * NB;
            if (!(single && in_mode == IN_RMSNORM)) {
                const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)m * ldx + b * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + j);
            }
            if (in_mode == IN_RMSNORM) {
                const float sc = sm.scale[m];
                const float4 *nw = reinterpret_cast<const float4 *>(sm.nw + b * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 w4 = nw[j];
                    v[j].x = __fmul_rn(__fmul_rn(v[j].x, sc), w4.x);
                    v[j].y = __fmul_rn(__fmul_rn(v[j].y, sc), w4.y);
                    v[j].z = __fmul_rn(__fmul_rn(v[j].z, sc), w4.z);
                    v[j].w = __fmul_rn(__fmul_rn(v[j].w, sc), w4.w);
                }
            }
            if (act_out != nullptr && cta == 0) {
                float4 *dst = reinterpret_cast<float4 *>(act_out + (size_t)m * K + b * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) dst[j] = v[j];
            }
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                amax = fmaxf(fmaxf(fmaxf(amax, fabsf(v[j].x)), fmaxf(fabsf(v[j].y), fabsf(v[j].z))), fabsf(v[j].w));
            const float d = __fdiv_rn(amax, 127.f);
            const float id = amax != 0.0f ? __fdiv_rn(127.f, amax) : 0.0f;
            int pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int q0 = __float2int_rn(__fmul_rn(v[j].x, id)), q1 = __float2int_rn(__fmul_rn(v[j].y, id));
                const int q2 = __float2int_rn(__fmul_rn(v[j].z, id)), q3 = __float2int_rn(__fmul_rn(v[j].w, id));
                pk[j] = (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
            }
            int4 *dq = reinterpret_cast<int4 *>(sm.xq + m * K + b * 32);
            dq[0] = make_int4(pk[0], pk[1], pk[2], pk[3]);
            dq[1] = make_int4(pk[4], pk[5], pk[6], pk[7]);
            sm.xd[m * NB + b] = __half2float(__float2half_rn(d));
        }
    }
    named_sync(1, kMNC);

    // warp -> (row in stage, K slice); lane -> 16-byte chunks c0 + lane + 32j of
    // the slice (consecutive lanes read consecutive 16 bytes: no bank
    // conflicts).  A chunk is half a Q8_0 block; its term s_half * (d_w * d_x)
    // is exact in double, so halves need not be paired before accumulating.
    // The lane's activation chunks are the same for every row: registers.
    const int S = st.S, WPR = st.WPR;
    const int row_local = warp / WPR, slice = warp - row_local * WPR;
    const int NC = K >> 4;
    const int CPS = (NC + WPR - 1) / WPR;
    const int c_begin = slice * CPS, c_end = min(NC, c_begin + CPS);
    int cj[kCPL];
    bool cv[kCPL];
#pragma unroll
    for (int j = 0; j < kCPL; ++j) {
        const int c = c_begin + lane + 32 * j;
        cv[j] = c < c_end;
        cj[j] = cv[j] ? c : c_begin;
    }
    int xr[MT][kCPL][4];
    float xs[MT][kCPL];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int j = 0; j < kCPL; ++j) {
            const int mm = m < M ? m : 0;
            const int4 a = *reinterpret_cast<const int4 *>(sm.xq + mm * K + cj[j] * 16);
            xr[m][j][0] = a.x;
            xr[m][j][1] = a.y;
            xr[m][j][2] = a.z;
            xr[m][j][3] = a.w;
            xs[m][j] = sm.xd[mm * NB + (cj[j] >> 1)];
        }
    // arrivals a row group (one row, or one gate/up pair) collects before it is finalized
    const int need = WPR * unit;

    for (int rb = r0; rb < r1; rb += S, ++cs) {
        const int slot = cs % kMStages;
        const int rows = min(S, r1 - rb);
        mbar_wait(&sm.full[slot], (cs / kMStages) & 1, err, ERR_WAIT_FULL);
        double acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = 0.0;
        const bool have = row_local < rows;
        if (have) {
            const int8_t *sq = reinterpret_cast<const int8_t *>(sm.ring[slot]);
            const int8_t *wrow = sq + (size_t)row_local * K;
            const __half *drow = reinterpret_cast<const __half *>(sq + (size_t)S * K) + (size_t)row_local * NB;
            int4 wv[kCPL];
            float dw[kCPL];
#pragma unroll
            for (int j = 0; j < kCPL; ++j)
                if (cv[j]) {
                    wv[j] = *reinterpret_cast<const int4 *>(wrow + cj[j] * 16);
                    dw[j] = __half2float(drow[cj[j] >> 1]);
                }
#pragma unroll
            for (int j = 0; j < kCPL; ++j)
                if (cv[j]) {
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        if (m < M) {
                            int sh = dp4a(wv[j].x, xr[m][j][0], 0);
                            sh = dp4a(wv[j].y, xr[m][j][1], sh);
                            sh = dp4a(wv[j].z, xr[m][j][2], sh);
                            sh = dp4a(wv[j].w, xr[m][j][3], sh);
                            acc[m] += (double)sh * (double)(dw[j] * xs[m][j]);
                        }
                }
        }
        __syncwarp();
        if (!have) {
            if (lane == 0) mbar_arrive(&sm.empty[slot]);
            continue;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = warp_sum_d(acc[m]);
        if (lane == 0) {
            combine_row<MT>(sm, slot, row_local, unit, need, M, acc, epi, y, ldy, rb, r0, res);
            // release the slot only after the combine: its row accumulators are
            // reused when the slot comes round again
            mbar_arrive(&sm.empty[slot]);
        }
    }
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

__device__ __forceinline__ float deq_row(const int8_t *q, const __half *d, int cols, long long row, int col) {
    return (float)q[row * cols + col] * __half2float(d[row * (cols >> 5) + (col >> 5)]);
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
        float x = deq_row(e.eq, e.ed, e.dim, tok, i);
        if (sem && e.ncb > 0) {
            float s = 0.f;
            for (int cb = 0; cb < e.ncb; ++cb) {
                int id = __ldcg(e.tokens + t * stride + 1 + cb) + cb * e.cb_size;
                if (id < 0 || id >= e.c_rows) {
                    if (i == 0) atomicOr(err, ERR_BAD_TOKEN);
                    id = 0;
                }
                const float r = deq_row(e.cq, e.cd, e.dim, id, i);
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
            x = deq_row(e.fq, e.fd, e.dim, c, i);
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
    for (int i = threadIdx.x; i < kMStages * kMW * kMaxT; i += blockDim.x) (&sm.rowacc[0][0][0])[i] = 0.0;
    for (int i = threadIdx.x; i < kMStages * kMW; i += blockDim.x) (&sm.rowcnt[0][0])[i] = 0;
    __syncthreads();
    if (warp == kMW) {
        if (lane == 0) mega_producer(ops, n_ops, sm, cta, G, err);
        return;
    }
    int cs = 0;
    for (int i = 0; i < n_ops; ++i) {
        const int kind = ops[i].kind;
        if (i > 0) grid_wait(ctl, (unsigned)(i * G), err);
        switch (kind) {
        case MK_GEMV: mega_gemv<MT>(ops[i].g, sm, cta, G, cs, err); break;
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
