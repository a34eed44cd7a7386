// tile_ring.cu -- microbenchmark of the weight-tile ring that the persistent
// decode kernel (s2k_mega.cu) and the standalone GEMV (s2k_gemv.cu) stream
// through: 148 CTAs, each with a 10-slot ring of 17 KB Q8_0 tiles filled by
// bulk copies (cp.async.bulk + mbarriers) and drained by 8 consumer warps
// (4 rows each, the tile engine's dp4a block sums in double).  It measures SM
// cycles per tile for
//   - the producer issuing every copy from one lane, or groups of four tiles
//     from four lanes (one bulk copy per lane in the same instruction);
//   - the consumers' work alone (the producer arms the slots without copies)
//     and the copies alone (the consumers only hand slots back);
// with the tiles in L2 (64 tiles cycled) or streamed from HBM (4 GB).
//
// Build and run (one GPU):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -o tile_ring s2.cpp_b200/microbench/tile_ring.cu && ./tile_ring
//
// Every wait is bounded (a timed-out wait sets an error flag and returns).
#include "../csrc/s2k_common.cuh"

#include <cstdio>
#include <cstdlib>
#include <vector>

using namespace s2k;

namespace {

constexpr int TR = 32, TK = 512, TQ = TR * TK, TB = TQ + TR * (TK / 32) * 2;  // 17,408-byte tiles
constexpr int NS = 10, K = 2560, NKT = K / TK, NB = K / 32;
constexpr int NW = 8, NT = NW * 32 + 32;  // 8 consumer warps + the producer warp
constexpr long long kLimit = 2000000000LL;  // ~1 s of SM cycles per wait

struct Smem {
    uint8_t ring[NS][TB];
    uint64_t full[NS], empty[NS];
    alignas(16) int8_t xq[K];
    float xd[NB];
};

__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_test(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_test(bar, parity))
        if (clock64() - t0 > kLimit) {
            atomicOr(err, 1);
            return false;
        }
    return true;
}

enum Mode { kFull = 0, kCopyOnly = 1, kComputeOnly = 2 };

// PL: producer lanes per group of tiles (1 = one lane issues every copy).
template <int PL, int MODE>
__global__ void __launch_bounds__(NT, 1)
    ring_kernel(const uint8_t *src, long long nsrc, int T, const int8_t *xq_g, const float *xd_g, double *out,
                long long *cyc, int *err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cta = blockIdx.x;
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], NW);
        }
        fence_mbar_init();
    }
    for (int i = tid; i < K; i += NT) sm.xq[i] = xq_g[i];
    for (int i = tid; i < NB; i += NT) sm.xd[i] = xd_g[i];
    __syncthreads();
    if (warp == NW) {  // producer
        const uint64_t pol = policy_evict_first();
        for (int ps0 = 0; ps0 < T; ps0 += PL) {
            // tiles ps0 .. ps0 + PL - 1 reuse the slots of tiles ps0 - NS ..: wait for the last of those
            const int q = ps0 + PL - 1 - NS;
            int ok = 1;
            if (q >= 0 && lane == 0) ok = wait_bounded(&sm.empty[q % NS], (uint32_t)(q / NS) & 1u, err);
            if (!__shfl_sync(0xffffffffu, ok, 0)) return;
            const int ps = ps0 + lane;
            if (lane < PL && ps < T) {
                const int slot = ps % NS;
                if (MODE == kComputeOnly) {
                    mbar_arrive(&sm.full[slot]);
                } else {
                    mbar_arrive_expect_tx(&sm.full[slot], TB);
                    bulk_g2s(sm.ring[slot], src + (((long long)cta * T + ps) % nsrc) * TB, TB, &sm.full[slot], pol);
                }
            }
        }
        return;
    }
    const long long c0 = clock64();
    int slot = 0;
    uint32_t phase = 0;
    const int rbase = warp * 4;
    double total = 0.0;
    for (int rt = 0; rt < T / NKT; ++rt) {
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        for (int kt = 0; kt < NKT; ++kt) {
            const int4 xa = *reinterpret_cast<const int4 *>(sm.xq + lane * 16 + kt * TK);
            const float xs = sm.xd[kt * 16 + (lane >> 1)];
            if (!wait_bounded(&sm.full[slot], phase, err)) return;
            const uint8_t *t = sm.ring[slot];
            int4 wv[4];
            float dw[4];
            if (MODE != kCopyOnly) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    wv[i] = *reinterpret_cast<const int4 *>(t + (rbase + i) * TK + lane * 16);
                    dw[i] = __half2float(reinterpret_cast<const __half *>(t + TQ)[(rbase + i) * 16 + (lane >> 1)]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[slot]);
            if (++slot == NS) {
                slot = 0;
                phase ^= 1u;
            }
            if (MODE != kCopyOnly) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    int sh = dp4a(wv[i].x, xa.x, 0);
                    sh = dp4a(wv[i].y, xa.y, sh);
                    sh = dp4a(wv[i].z, xa.z, sh);
                    sh = dp4a(wv[i].w, xa.w, sh);
                    acc[i] += (double)sh * (double)__fmul_rn(dw[i], xs);
                }
            } else {
                acc[0] += xs;
            }
        }
        total += acc[0] + acc[1] + acc[2] + acc[3];
    }
    out[(size_t)cta * NT + tid] = total;
    __syncwarp();
    if (tid == 0) cyc[cta] = clock64() - c0;
}

void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
        exit(1);
    }
}

template <int PL, int MODE>
void run(const char *name, const uint8_t *src, long long nsrc, int G, int T, const int8_t *xq, const float *xd,
         double *out, long long *cyc, int *err) {
    const size_t smem = sizeof(Smem) + 1024;
    check(cudaFuncSetAttribute(ring_kernel<PL, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem), "attr");
    for (int r = 0; r < 3; ++r) ring_kernel<PL, MODE><<<G, NT, smem>>>(src, nsrc, T, xq, xd, out, cyc, err);
    check(cudaDeviceSynchronize(), name);
    int herr = 0;
    check(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost), "err");
    std::vector<long long> h(G);
    check(cudaMemcpy(h.data(), cyc, G * sizeof(long long), cudaMemcpyDeviceToHost), "cycles");
    long long mx = 0, sum = 0;
    for (long long c : h) {
        mx = c > mx ? c : mx;
        sum += c;
    }
    printf("%-44s %s  SM cycles per tile: mean %.0f, slowest CTA %.0f%s\n", name,
           nsrc > 64 ? "HBM" : "L2 ", (double)sum / G / T, (double)mx / T, herr ? "  (a wait timed out)" : "");
}

}  // namespace

int main() {
    const long long nbig = (4LL << 30) / TB;  // 4 GB of tiles
    uint8_t *src = nullptr;
    check(cudaMalloc(&src, (size_t)nbig * TB), "tiles");
    {
        std::vector<uint8_t> h((size_t)4096 * TB);
        uint32_t s = 12345;
        for (size_t t = 0; t < 4096; ++t) {
            uint8_t *p = h.data() + t * TB;
            for (int i = 0; i < TQ; ++i) {
                s = s * 1664525u + 1013904223u;
                p[i] = (uint8_t)(int8_t)((int)((s >> 24) % 255) - 127);
            }
            uint16_t *d = reinterpret_cast<uint16_t *>(p + TQ);
            for (int i = 0; i < TR * 16; ++i) {
                s = s * 1664525u + 1013904223u;
                d[i] = (uint16_t)(0x1000 + (s >> 20) % 0x1800);  // fp16 scales 2^-11 .. 2^-5
            }
        }
        for (long long t = 0; t < nbig; t += 4096) {
            const long long n = nbig - t < 4096 ? nbig - t : 4096;
            check(cudaMemcpy(src + t * TB, h.data(), (size_t)n * TB, cudaMemcpyHostToDevice), "fill");
        }
    }
    const int G = 148;
    int8_t *xq = nullptr;
    float *xd = nullptr;
    double *out = nullptr;
    long long *cyc = nullptr;
    int *err = nullptr;
    check(cudaMalloc(&xq, K), "xq");
    check(cudaMalloc(&xd, NB * sizeof(float)), "xd");
    check(cudaMalloc(&out, (size_t)G * NT * sizeof(double)), "out");
    check(cudaMalloc(&cyc, G * sizeof(long long)), "cyc");
    check(cudaMalloc(&err, sizeof(int)), "err");
    check(cudaMemset(err, 0, sizeof(int)), "err0");
    {
        std::vector<int8_t> hx(K);
        std::vector<float> hd(NB);
        for (int i = 0; i < K; ++i) hx[i] = (int8_t)((i * 37) % 255 - 127);
        for (int i = 0; i < NB; ++i) hd[i] = 0.0078125f * (1 + i % 7);
        check(cudaMemcpy(xq, hx.data(), K, cudaMemcpyHostToDevice), "xq");
        check(cudaMemcpy(xd, hd.data(), NB * sizeof(float), cudaMemcpyHostToDevice), "xd");
    }
    const int T = 4000;
    run<1, kFull>("one producer lane", src, 64, G, T, xq, xd, out, cyc, err);
    run<4, kFull>("four producer lanes per group", src, 64, G, T, xq, xd, out, cyc, err);
    run<1, kCopyOnly>("copies only, one producer lane", src, 64, G, T, xq, xd, out, cyc, err);
    run<4, kCopyOnly>("copies only, four producer lanes", src, 64, G, T, xq, xd, out, cyc, err);
    run<4, kComputeOnly>("consumers only (slots armed without copies)", src, 64, G, T, xq, xd, out, cyc, err);
    run<1, kFull>("one producer lane", src, nbig, G, 1000, xq, xd, out, cyc, err);
    run<4, kFull>("four producer lanes per group", src, nbig, G, 1000, xq, xd, out, cyc, err);
    return 0;
}
