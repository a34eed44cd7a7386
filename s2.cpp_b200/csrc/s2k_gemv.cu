// s2k_gemv.cu -- standalone fused (RMSNorm | SwiGLU | residual) + Q8_0
// activation quantization + dequant-GEMV for 1..8 tokens on sm_100a, and the
// upload-time re-layout of GGUF Q8_0 blocks into tiles.
//
// Reference semantics (s2.cpp reaches these through ggml's CPU mat-vec):
//   mul_mat(W, x) with W Q8_0 quantizes each activation row to Q8_0 blocks
//   (ggml-cpu quantize_row_q8_0, x86 form) and computes, per output row,
//   sum_b (int sum_b) * (d_w * d_x)      (vec_dot_q8_0_q8_0)
//   The RMSNorm prologue restates rms_norm_weighted (src/s2_model.cpp:46-55);
//   the SwiGLU epilogue (rows interleaved gate/up) restates ggml_swiglu_split
//   (src/s2_model.cpp:1047), so W2 reads silu(gate)*up directly.
//
// This kernel runs the GEMVs of s2k_eval (prompt prefill, single steps) and
// s2k_fast_decode; the frame loop uses the same tile engine inside the
// persistent kernel (s2k_mega.cu).  One CTA per SM: warp 8 streams the CTA's
// tiles through a shared-memory ring with cp.async.bulk + mbarriers, starting
// BEFORE griddepcontrol.wait, so with programmatic dependent launch the
// weights stream while the previous kernel finishes; warps 0-7 wait for the
// previous kernel, quantize the activation into shared memory and consume the
// tiles (s2k_tgemv.cuh).
#include "s2k_common.cuh"
#include "s2k_kernels.h"

#include <algorithm>
#include <cstddef>
#include <cstdint>

namespace s2k {

constexpr int kThreads = kTNC + 32;  // consumers + producer warp
constexpr int kMaxMT = 8;
constexpr int kMaxK = 10240;

template <int MT>
struct GemvCfg {
    static constexpr int NS = MT <= 2 ? 9 : (MT <= 4 ? 7 : 5);  // ring stages
};

constexpr int kPC = 5;  // 8-value activation chunks per consumer thread per prologue pass
constexpr int kGemvPL = 4;  // tiles the producer warp issues per group (one per lane)
constexpr int kMaxMTF16 = 4;  // tokens per launch on F16 weights (their activation takes 2 B per value)

template <int MT>
struct GemvSmem {
    uint8_t ring[GemvCfg<MT>::NS][kTileBytes];
    uint64_t full[GemvCfg<MT>::NS], empty[GemvCfg<MT>::NS];
    // quantized activation (int8), or the fp16 activation of F16 weights (2 B
    // per value over xq, xd, xbs and xh_rest; MT <= kMaxMTF16)
    alignas(16) int8_t xq[MT * kMaxK];
    float xd[MT * kMaxK / 32];      // Q8_0 block scales, or Q8_K super-block scales
    int16_t xbs[MT * kMaxK / 16];   // Q8_K block sums
    int8_t xh_rest[MT <= kMaxMTF16 ? MT * kMaxK * 3 / 4 : 16];
    double tok[kTW][MT];
    int abort_flag;
};
static_assert(offsetof(GemvSmem<4>, xh_rest) + sizeof(GemvSmem<4>::xh_rest) - offsetof(GemvSmem<4>, xq) >=
                  (size_t)2 * 4 * kMaxK,
              "fp16 activation fits xq .. xh_rest");
static_assert(sizeof(GemvSmem<8>) <= 227 * 1024, "gemv shared memory");
static_assert(sizeof(GemvSmem<4>) <= 227 * 1024, "gemv shared memory");
static_assert(sizeof(GemvSmem<2>) <= 227 * 1024, "gemv shared memory");

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) tgemv_kernel(TGemv g, const int *done, int *err) {
    constexpr int NS = GemvCfg<MT>::NS;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    GemvSmem<MT> &sm = *reinterpret_cast<GemvSmem<MT> *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    long long u0, u1;
    tg_range(g.R, g.K, g.wtype, blockIdx.x, gridDim.x, &u0, &u1);
    const int ntiles = (int)(u1 - u0);
    const uint32_t tb = (uint32_t)tile_bytes(g.wtype);
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kTW);
        }
        fence_mbar_init();
        // A finished frame (done already visible) issues no weight traffic.
        const bool early = done != nullptr && *reinterpret_cast<const volatile int *>(done) != 0;
        sm.abort_flag = early ? 2 : 0;
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kTW) {  // ---------------- producer ----------------
        // Tiles go out in groups of up to kGemvPL, one bulk copy per lane in
        // the same instruction (one lane issuing every copy bounds a CTA's
        // tile rate).  Lane 0 checks the ring once per group: tile t reuses
        // the slot of tile t - NS, and the consumers release tiles in order,
        // so waiting for the group's last such tile covers the others.  The
        // first NS tiles, which an aborting consumer drains, are issued
        // without a check, so no group straddles tile NS.
        if (__shfl_sync(0xffffffffu, sm.abort_flag, 0) == 0) {
            const uint64_t pol = policy_evict_first();
            for (int t = 0; t < ntiles;) {
                const int n = min(min(kGemvPL, ntiles - t), t < NS ? NS - t : kGemvPL);
                if (t + n - 1 >= NS) {
                    int stop = 0;
                    if (lane == 0) {
                        const int q = t + n - 1 - NS;
                        stop = !mbar_wait(&sm.empty[q % NS], (q / NS) & 1, err, ERR_WAIT_EMPTY) ||
                               *reinterpret_cast<volatile int *>(&sm.abort_flag) != 0;
                    }
                    if (__shfl_sync(0xffffffffu, stop, 0)) break;
                }
                if (lane < n) {
                    const int slot = (t + lane) % NS;
                    mbar_arrive_expect_tx(&sm.full[slot], tb);
                    bulk_g2s(sm.ring[slot], g.w + (size_t)(u0 + t + lane) * tb, tb, &sm.full[slot], pol);
                }
                t += n;
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    F8 nw[kPC];  // norm weights do not depend on the previous kernel: load them before waiting for it
    tg_norm_preload<kPC, kTNC>(g, nw);
    pdl_wait();
    const bool early = sm.abort_flag == 2;
    if (early || (done != nullptr && *reinterpret_cast<const volatile int *>(done) != 0)) {
        // Drain what the producer may have issued before it sees the flag.
        if (tid == 0) sm.abort_flag = 1;
        named_sync(1, kTNC);
        const int cap = early ? 0 : min(ntiles, NS);
        for (int t = 0; t < cap; ++t) {
            const int slot = t % NS;
            mbar_wait(&sm.full[slot], (t / NS) & 1, err, ERR_WAIT_FULL);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[slot]);
        }
        return;
    }
    if (ntiles == 0) return;
    // the CTA owning row tile 0 stores act_out
    tg_prologue8<MT, kTNC, kPC>(g, nw, sm.xq, sm.xd, sm.xbs, &sm.tok[0][0], MT, u0 == 0, 1);
    named_sync(1, kTNC);
    int slot = 0;
    uint32_t phase = 0;
    tg_consume_any<MT>(g, &sm.ring[0][0], sm.full, sm.empty, NS, slot, phase, sm.xq, sm.xd, sm.xbs, blockIdx.x,
                       gridDim.x, err);
}

int tw_of(int ggml_type) {
    return ggml_type == 12 ? TW_Q4_K
                           : (ggml_type == 14 ? TW_Q6_K : (ggml_type == 8 ? TW_Q8_0 : (ggml_type == 1 ? TW_F16 : -1)));
}

size_t DevMat::bytes() const {
    const int tw = tw_of(type);
    if (tw < 0) return 0;
    return (size_t)(rows / kTR) * (size_t)(cols / tile_cols(tw)) * tile_bytes(tw);
}

cudaError_t gemv_setup() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(tgemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(GemvSmem<1>))))
        return e;
    if ((e = cudaFuncSetAttribute(tgemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(GemvSmem<2>))))
        return e;
    if ((e = cudaFuncSetAttribute(tgemv_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(GemvSmem<4>))))
        return e;
    return cudaFuncSetAttribute(tgemv_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(GemvSmem<8>));
}

template <int MT>
static cudaError_t launch_one(const GemvArgs &a, int m0, int M, int grid, cudaStream_t st) {
    const DevMat &w = *a.w;
    TGemv g;
    g.w = w.w;
    g.wtype = tw_of(w.type);
    g.ll = 0;  // plain float activations
    g.x_tag = g.res_tag = g.y_tag = 0;
    g.R = w.rows;
    g.K = w.cols;
    g.x = a.x + (size_t)m0 * a.ldx;
    g.ldx = a.ldx;
    g.M = M;
    g.in_mode = a.in_mode;
    g.norm_w = a.norm_w;
    g.eps = a.eps;
    g.epi = a.epi;
    g.y = a.y + (size_t)m0 * a.ldy;
    g.ldy = a.ldy;
    g.res = a.res ? a.res + (size_t)m0 * a.ldres : nullptr;
    g.ldres = a.ldres;
    g.act_out = a.act_out ? a.act_out + (size_t)m0 * w.cols : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(GemvSmem<MT>);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, tgemv_kernel<MT>, g, a.done, a.err);
}

cudaError_t launch_gemv(const GemvArgs &a, int num_sms, cudaStream_t st) {
    const DevMat &w = *a.w;
    if (tw_of(w.type) < 0 || !w.w) return cudaErrorInvalidValue;
    if (a.ldx % 8 != 0 || reinterpret_cast<uintptr_t>(a.x) % 32 != 0) return cudaErrorInvalidValue;
    if (a.in_mode == IN_RMSNORM && reinterpret_cast<uintptr_t>(a.norm_w) % 32 != 0) return cudaErrorInvalidValue;
    if (!tg_shape_ok(w.rows, w.cols, std::min(a.M, kMaxMT), a.in_mode, a.epi, a.res != nullptr, kMaxK, kMaxMT))
        return cudaErrorInvalidValue;
    if (a.in_mode == IN_RMSNORM && a.norm_w == nullptr) return cudaErrorInvalidValue;
    const int grid = std::min(num_sms, w.rows / kTR);
    const int mt_max = w.type == 1 ? kMaxMTF16 : kMaxMT;
    for (int m0 = 0; m0 < a.M; m0 += mt_max) {
        const int M = std::min(mt_max, a.M - m0);
        cudaError_t e;
        if (M == 1) e = launch_one<1>(a, m0, M, grid, st);
        else if (M == 2) e = launch_one<2>(a, m0, M, grid, st);
        else if (M <= 4) e = launch_one<4>(a, m0, M, grid, st);
        else e = launch_one<8>(a, m0, M, grid, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------------------
// GGUF Q8_0 blocks -> tiles
// ---------------------------------------------------------------------------
// One thread per 34-byte source block (fp16 d, 32 int8 q): block b of source
// row r goes to destination row dr = r * row_stride + row_offset, tile
// (dr / 32, b / 16), quants at (dr % 32) * 512 + (b % 16) * 32, scale at
// (dr % 32) * 16 + b % 16 of the tile's scale table.
__global__ void relayout_q8_0_kernel(const uint8_t *__restrict__ src, int row0, int rows, int cols,
                                     uint8_t *__restrict__ dst, int row_stride, int row_offset) {
    const int nb = cols / 32, nkt = cols / kTK;
    const long long total = (long long)rows * nb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int rr = (int)(i / nb), b = (int)(i - (long long)rr * nb);
        const uint8_t *blk = src + i * 34;
        const long long dr = (long long)(row0 + rr) * row_stride + row_offset;
        uint8_t *tile = dst + ((size_t)(dr / kTR) * nkt + (size_t)(b / (kTK / 32))) * kTileBytes;
        const int rl = (int)(dr % kTR), bl = b % (kTK / 32);
        tile[kTileQ + (rl * (kTK / 32) + bl) * 2] = blk[0];
        tile[kTileQ + (rl * (kTK / 32) + bl) * 2 + 1] = blk[1];
        uint8_t *qd = tile + rl * kTK + bl * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) qd[j] = blk[2 + j];
    }
}

cudaError_t launch_relayout_q8_0(const uint8_t *src, int row0, int rows, int cols, DevMat *dst, int row_stride,
                                 int row_offset, cudaStream_t st) {
    const long long total = (long long)rows * (cols / 32);
    const int block = 256;
    const int grid = (int)std::min<long long>((total + block - 1) / block, 148 * 16);
    count_launch();
    relayout_q8_0_kernel<<<grid, block, 0, st>>>(src, row0, rows, cols, dst->w, row_stride, row_offset);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// GGUF Q4_K / Q6_K super-blocks -> tiles
// ---------------------------------------------------------------------------
// One thread per source super-block: super-block b of source row r goes to
// destination row dr = r * row_stride + row_offset, tile (dr / 32, b / 2),
// super-block slot sb = b % 2 of row dr % 32 (layout in s2k_tgemv.cuh).
__global__ void relayout_k_kernel(const uint8_t *__restrict__ src, int row0, int rows, int cols, int wtype,
                                  uint8_t *__restrict__ dst, int row_stride, int row_offset) {
    const int nsb = cols / 256, nkt = cols / kTK;
    const int sbb = wtype == TW_Q4_K ? 144 : 210;
    const long long total = (long long)rows * nsb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int rr = (int)(i / nsb), b = (int)(i - (long long)rr * nsb);
        const uint8_t *blk = src + i * sbb;
        const long long dr = (long long)(row0 + rr) * row_stride + row_offset;
        uint8_t *tile = dst + ((size_t)(dr / kTR) * nkt + (size_t)(b / 2)) * tile_bytes(wtype);
        const int rb = (int)(dr % kTR) * 2 + (b & 1);
        if (wtype == TW_Q4_K) {  // d dmin scales[12] | qs[128]
            for (int j = 0; j < 16; ++j) tile[kQ4kHdr + rb * 16 + j] = blk[j];
            for (int j = 0; j < 128; ++j) tile[rb * 128 + j] = blk[16 + j];
        } else {  // ql[128] qh[64] scales[16] d
            for (int j = 0; j < 128; ++j) tile[rb * 128 + j] = blk[j];
            for (int j = 0; j < 64; ++j) tile[kQ6kQh + rb * 64 + j] = blk[128 + j];
            for (int j = 0; j < 16; ++j) tile[kQ6kSc + rb * 16 + j] = blk[192 + j];
            tile[kQ6kD + rb * 2] = blk[208];
            tile[kQ6kD + rb * 2 + 1] = blk[209];
        }
    }
}

// ---------------------------------------------------------------------------
// GGUF F16 rows -> tiles of 32 x 256 halves: one thread per 16-byte chunk
// (8 halves); chunk c of source row r lands in destination row dr = r *
// row_stride + row_offset, tile (dr / 32, c / 32), at (dr % 32, 8 (c % 32)).
// ---------------------------------------------------------------------------
__global__ void relayout_f16_kernel(const uint8_t *__restrict__ src, int row0, int rows, int cols,
                                    uint8_t *__restrict__ dst, int row_stride, int row_offset) {
    const int nc = cols / 8, nkt = cols / kTKH;
    const long long total = (long long)rows * nc;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int rr = (int)(i / nc), c = (int)(i - (long long)rr * nc);
        const long long dr = (long long)(row0 + rr) * row_stride + row_offset;
        uint8_t *tile = dst + ((size_t)(dr / kTR) * nkt + (size_t)(c / (kTKH / 8))) * kTileBytesF16;
        *reinterpret_cast<uint4 *>(tile + ((dr % kTR) * kTKH + 8 * (c % (kTKH / 8))) * 2) =
            *reinterpret_cast<const uint4 *>(src + i * 16);
    }
}

cudaError_t launch_relayout(const uint8_t *src, int row0, int rows, int cols, DevMat *dst, int row_stride,
                            int row_offset, cudaStream_t st) {
    const int tw = tw_of(dst->type);
    if (tw == TW_Q8_0) return launch_relayout_q8_0(src, row0, rows, cols, dst, row_stride, row_offset, st);
    if (tw < 0) return cudaErrorInvalidValue;
    if (tw == TW_F16) {
        if (reinterpret_cast<uintptr_t>(src) % 16 != 0 || cols % kTKH != 0) return cudaErrorInvalidValue;
        const long long total = (long long)rows * (cols / 8);
        const int block = 256;
        const int grid = (int)std::min<long long>((total + block - 1) / block, 148 * 16);
        count_launch();
        relayout_f16_kernel<<<grid, block, 0, st>>>(src, row0, rows, cols, dst->w, row_stride, row_offset);
        return cudaGetLastError();
    }
    const long long total = (long long)rows * (cols / 256);
    const int block = 256;
    const int grid = (int)std::min<long long>((total + block - 1) / block, 148 * 16);
    count_launch();
    relayout_k_kernel<<<grid, block, 0, st>>>(src, row0, rows, cols, tw, dst->w, row_stride, row_offset);
    return cudaGetLastError();
}

}  // namespace s2k
