// gemm_sm100_pair.cu -- prefill grouped expert GEMM on CTA pairs: one
// tcgen05.mma.cta_group::2 of M=256 spans two SMs of a cluster.
//
// Same arithmetic as the one-SM kernel in gemm_sm100.cu (the gather_mm path
// of ESExperts::sparseForward, aptransformer/ESExperts.mm:50-57, with the
// GeGLU fused into the gate_up epilogue), on 256-row m-tiles:
//   each CTA stages its own 128 activation rows and HALF of the weight tile
//   (gate_up: the leader the gate rows, the peer the matching up rows; down:
//   one half of the output columns each), so per flop a CTA pulls half the
//   weight bytes through L2 -> shared memory that a one-SM tile of the same
//   N does.  That ingest was what bounded the one-SM kernel.
//
// Roles (192 threads per CTA, one CTA per SM, clusters of 2):
//   warp 0      both CTAs: TMA producer of the CTA's A and B halves into its
//               own ring; the bytes are credited to the LEADER's `full`
//               barrier (the leader posts the expected count for both)
//   warp 1      TMEM owner in both CTAs (pair allocation, 512 columns = two
//               accumulators of N <= 256); the leader's lane 0 issues the
//               MMAs and commits to `empty` / `tfull` of both CTAs
//   warps 2..5  both CTAs: epilogue of the CTA's 128 accumulator rows; each
//               thread arrives on the leader's `tempty` (count 256)
// Accumulator rows of CTA c are tile rows c*128 .. c*128+127.  Every wait is
// bounded and records an error code on expiry.  Before leaving, each producer
// drains its `empty` ring so no commit targets a CTA that has exited, and the
// pair meets at a cluster barrier before releasing TMEM.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "moe_internal.h"
#include "launch_util.h"
#include "sm100_ptx.cuh"
#include "gemm_epilogue.cuh"

namespace apt {

namespace {

using namespace sm100;

constexpr int kBM = 256;                 // rows per pair tile
constexpr int kHM = 128;                 // rows per CTA
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kAccStride = 256;
constexpr long long kWaitLimit = 4000000000LL;
constexpr int kMaxGroups = 256;
constexpr int kStageC = 4 * 2 * 4096;    // down: 2 x 4 KB store boxes per epilogue warp

enum { EPI_GATEUP = 0, EPI_DOWN = 1 };

__device__ __forceinline__ void record_error(int32_t *err, int code, int where) {
    if (atomicCAS(err, 0, code) == 0) err[1] = where;
}

__device__ __forceinline__ void decode_tile(int t, int NT, const int *mtp, int E, int &e, int &mloc,
                                            int &nt) {
    const int mt = t / NT;
    nt = t - mt * NT;
    int lo = 0, hi = E - 1;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (mtp[mid + 1] > mt) hi = mid;
        else lo = mid + 1;
    }
    e = lo;
    mloc = mt - mtp[e];
}

// N = MMA width (both CTAs' B halves); NH = N/2 weight rows staged per CTA.
template <int EPI, int N, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const int32_t *__restrict__ counts, const int32_t *__restrict__ offsets, int E,
                     int Kdim, int I, int H, uint16_t *__restrict__ out, int out_ld,
                     int32_t *__restrict__ err, const int32_t *__restrict__ g2e) {
    constexpr int NH = N / 2;
    constexpr int A_BYTES = kHM * kBK * 2, B_BYTES = NH * kBK * 2;
    constexpr uint32_t IDESC = idesc_bf16_f32(kBM, N);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    uint8_t *sC = sB + STAGES * B_BYTES;  // down: per-epilogue-warp store staging
    uint64_t *full = reinterpret_cast<uint64_t *>(sC + (EPI == EPI_DOWN ? kStageC : 0));
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    int *mtp = reinterpret_cast<int *>(tmem_slot + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * 128);
        }
        fence_barrier_init();
        tma_prefetch(&tmA);
        tma_prefetch(&tmB);
    }
    pdl_wait();
    if (warp == 0 && lane == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            mtp[e] = acc;
            acc += (counts[e] + kBM - 1) / kBM;
        }
        mtp[E] = acc;
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    fence_proxy_async();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();
    const int NT = (EPI == EPI_GATEUP) ? (I + NH - 1) / NH : H / N;
    const int tiles = mtp[E] * NT;
    const int KB = Kdim / kBK;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (warp == 0) {
        if (lane == 0) {
            int g = 0;
            for (int t = pair; t < tiles; t += npairs) {
                int e, mloc, nt;
                decode_tile(t, NT, mtp, E, e, mloc, nt);
                const int row0 = offsets[e] + mloc * kBM + (int)rank * kHM;
                const int ew = g2e ? g2e[e] : e;
                const int brow = (EPI == EPI_GATEUP) ? ew * 2 * I + (int)rank * I + nt * NH
                                                     : ew * H + nt * N + (int)rank * NH;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, kWaitLimit)) {
                        record_error(err, 11, t);
                        goto producer_done;
                    }
                    const uint32_t fb = cluster_addr(&full[s], 0);
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * (A_BYTES + B_BYTES));
                    tma_load_2d_pair(sA + s * A_BYTES, &tmA, fb, kb * kBK, row0);
                    tma_load_2d_pair(sB + s * B_BYTES, &tmB, fb, kb * kBK, brow);
                }
            }
            // drain: every stage's last commit has arrived here before exit
            for (int j = 0; j < STAGES; ++j, ++g) {
                if (!mbar_wait(&empty[g % STAGES], ((g / STAGES) & 1) ^ 1, kWaitLimit)) {
                    record_error(err, 12, j);
                    break;
                }
            }
        producer_done:;
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            int g = 0, i = 0;
            for (int t = pair; t < tiles; t += npairs, ++i) {
                const int buf = i & 1;
                const uint32_t use = i >> 1;
                if (!mbar_wait_cluster(&tempty[buf], (use & 1) ^ 1, kWaitLimit)) {
                    record_error(err, 13, t);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + buf * kAccStride;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, kWaitLimit)) {
                        record_error(err, 14, t);
                        goto mma_done;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_bf16_pair(d, smem_desc_sw128(a0 + kk * 32),
                                      smem_desc_sw128(b0 + kk * 32), IDESC, (kb | kk) != 0);
                    mma_commit_pair(&empty[s], 0x3);
                }
                mma_commit_pair(&tfull[buf], 0x3);
            }
        mma_done:;
        }
    } else {
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t te0 = cluster_addr(&tempty[0], 0), te1 = cluster_addr(&tempty[1], 0);
        int i = 0, bufsel = 0;
        for (int t = pair; t < tiles; t += npairs, ++i) {
            int e, mloc, nt;
            decode_tile(t, NT, mtp, E, e, mloc, nt);
            const int base = mloc * kBM + (int)rank * kHM;
            const int nvalid = counts[e] - base;
            const int row = offsets[e] + base + r;
            const int buf = i & 1;
            const uint32_t use = i >> 1;
            if (!mbar_wait(&tfull[buf], use & 1, kWaitLimit)) {
                record_error(err, 15, t);
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + buf * kAccStride + ((uint32_t)(q * 32) << 16);
            if constexpr (EPI == EPI_GATEUP)
                epilogue_geglu(taddr, NH, min(NH, I - nt * NH), r < nvalid,
                               out + (size_t)row * out_ld + nt * NH);
            else if (q * 32 + 32 <= nvalid)
                epilogue_bf16_tma<N>(taddr, sC + q * 8192, bufsel, &tmC, nt * N, row - lane, lane);
            else if (q * 32 < nvalid)
                epilogue_bf16<N>(taddr, r < nvalid, out + (size_t)row * out_ld + nt * N);
            tc_fence_before();
            mbar_arrive_cluster(buf ? te1 : te0);
        }
        if (EPI == EPI_DOWN && lane == 0) bulk_wait<0>();  // stores complete before exit
    }
    __syncthreads();
    cluster_sync();  // the peer is done with this CTA's barriers and TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------- host side

bool make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
    return bf16_map_2d(m, base, inner, rows, kBK, box_rows, true);
}

template <int EPI, int N, int STAGES>
constexpr size_t smem_bytes() {
    return 1024 + (size_t)STAGES * (kHM * kBK * 2 + (N / 2) * kBK * 2) +
           (EPI == EPI_DOWN ? kStageC : 0) + 8 * (2 * STAGES + 4) + 16 + 4 * (kMaxGroups + 1);
}

template <int EPI, int N, int STAGES>
cudaError_t set_attr() {
    return cudaFuncSetAttribute(moe_gemm_pair_kernel<EPI, N, STAGES>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes<EPI, N, STAGES>());
}

template <int EPI, int N, int STAGES>
cudaError_t launch(const CUtensorMap &a, const CUtensorMap &b, const Dispatch &d, int E, int Kdim,
                   int I, int H, uint16_t *out, int out_ld, int32_t *err, cudaStream_t s,
                   const int32_t *g2e, const CUtensorMap *c = nullptr) {
    auto kern = moe_gemm_pair_kernel<EPI, N, STAGES>;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes<EPI, N, STAGES>();
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    // as many pairs as can be resident at once (not every SM need be paired)
    static int pairs[8] = {0};
    const int dev = current_device();
    if (dev < 0 || dev >= 8) return cudaErrorInvalidDevice;
    if (!pairs[dev]) {
        cfg.gridDim = dim3(2 * num_sms(dev));
        int n = 0;
        cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        if (e != cudaSuccess || n < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
        pairs[dev] = n;
    }
    cfg.gridDim = dim3(2 * pairs[dev]);
    return cudaLaunchKernelEx(&cfg, kern, a, b, c ? *c : a, d.counts, d.offsets, E, Kdim, I, H, out, out_ld, err,
                              g2e);
}

constexpr int kStages = 6;

}  // namespace

cudaError_t gemm_pair_init() {
    cudaError_t e;
    if ((e = set_attr<EPI_GATEUP, 256, kStages>())) return e;
    if ((e = set_attr<EPI_GATEUP, 176, 7>())) return e;
    return set_attr<EPI_DOWN, 256, kStages>();
}

// Pair kernels apply to H % 256 == 0 (down halves of 128 columns) and
// I % 128 == 0 or I % 88 == 0 (gate_up halves); the caller checks
// gemm_pair_supported first.
bool gemm_pair_supported(int H, int I) { return H % 256 == 0 && I % 64 == 0; }

cudaError_t launch_gemm_pair_gateup(const uint16_t *xp, const Dispatch &d, const int32_t *g2e,
                                    const ExpertWeights &w, int rows_cap, int H, int I, int E_w,
                                    int G, uint16_t *yp, int32_t *err, cudaStream_t s,
                                    int *launches) {
    if (G > kMaxGroups) return cudaErrorInvalidValue;
    static const int pref = [] {
        const char *v = getenv("APT_PAIR_GATEUP_N");
        return v ? atoi(v) : 0;
    }();
    const int n = (pref == 176 && I % 88 == 0) ? 176 : 256;
    CUtensorMap a, b;
    if (!make_map(&a, xp, H, rows_cap, kHM) || !make_map(&b, w.gu, H, (uint64_t)E_w * 2 * I, n / 2))
        return cudaErrorInvalidValue;
    cudaError_t e = (n == 176)
        ? launch<EPI_GATEUP, 176, 7>(a, b, d, G, H, I, H, yp, I, err, s, g2e)
        : launch<EPI_GATEUP, 256, kStages>(a, b, d, G, H, I, H, yp, I, err, s, g2e);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemm_pair_down(const uint16_t *yp, const Dispatch &d, const int32_t *g2e,
                                  const ExpertWeights &w, int rows_cap, int H, int I, int E_w,
                                  int G, uint16_t *out, int32_t *err, cudaStream_t s,
                                  int *launches) {
    if (G > kMaxGroups) return cudaErrorInvalidValue;
    CUtensorMap a, b, c;
    if (!make_map(&a, yp, I, rows_cap, kHM) || !make_map(&b, w.dn, I, (uint64_t)E_w * H, 128) ||
        !bf16_map_2d(&c, out, H, rows_cap, 64, 32, true))
        return cudaErrorInvalidValue;
    cudaError_t e = launch<EPI_DOWN, 256, kStages>(a, b, d, G, I, I, H, out, H, err, s, g2e, &c);
    if (launches) ++*launches;
    return e;
}

}  // namespace apt
