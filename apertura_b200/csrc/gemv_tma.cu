// gemv_tma.cu -- decode-sized grouped expert GEMV with TMA-streamed weights
// (bf16 experts).
//
// Same arithmetic as gemv.cu (gather_mm path of ESExperts::sparseForward,
// aptransformer/ESExperts.mm:44-60, with the reference's rounding points):
//   gate_up: y_j = bf16(bf16(gelu(bf16(x.Wg_j))) * bf16(x.Wu_j))
//   down:    o_h = bf16(y.Wd_h)
// but the weights do not pass through registers on their way in: a producer
// warp streams the CTA's weight rows into a STAGES-deep shared-memory ring
// with 2-D TMA copies, so every CTA keeps STAGES x 16 KB (gate_up) or 8 KB
// (down) of HBM reads in flight regardless of register pressure, and four
// compute warps consume the ring with conflict-free 128-bit shared loads.
//
// CTA = one active expert x one block of output rows:
//   gate_up: 16 intermediate columns j = 32 weight rows (16 gate, 16 up),
//            K chunks of 256; a warp owns 4 j (8 rows), its 32 lanes split K.
//   down:    64 hidden rows, K chunks of 64; a warp owns 16 rows as 4
//            row-groups of 8 lanes, each lane 4 rows.
// The expert's tokens are staged as bf16 in shared memory, up to NTMAX per
// pass (the compile-time bound picked from the call's T), by 1-D bulk copies
// the producer issues ahead of the compute warps into a double buffer, so
// consecutive items of a CTA follow without a memory round trip between them.  All mbarrier waits
// are bounded; on expiry the kernel records an error code and returns.
#include <cuda.h>

#include "common.cuh"
#include "moe_internal.h"
#include "launch_util.h"
#include "sm100_ptx.cuh"

namespace apt {

namespace {

using namespace sm100;

constexpr int kComputeWarps = 4;
constexpr int kThreads = (kComputeWarps + 1) * 32;  // + producer warp
constexpr long long kWaitLimit = 4000000000LL;
enum { GATEUP = 0, DOWN = 1 };

template <int EPI>
struct Shape;
template <>
struct Shape<GATEUP> {
    static constexpr int ROWS = 32, KC = 256, STAGE_BYTES = ROWS * KC * 2;
};
template <>
struct Shape<DOWN> {
    static constexpr int ROWS = 64, KC = 64, STAGE_BYTES = ROWS * KC * 2;
};

__device__ __forceinline__ void record_error(int32_t *err, int code, int where) {
    if (atomicCAS(err, 0, code) == 0) err[1] = where;
}

__device__ __forceinline__ float dot8f(const float (&w)[8], const float (&x)[8]) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s = fmaf(w[j], x[j], s);
    return s;
}

template <int NT, int R>
__device__ __forceinline__ float pick(const float (&acc)[R][NT], int r, int t) {
    float v = 0.f;
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
        if (tt == t) v = acc[r][tt];
    return v;
}

struct Args {
    const uint16_t *in;  // x [T,H] (gate_up, rows via perm/K) or yp [rows,I] (down)
    const int32_t *perm, *offsets, *counts, *active, *n_active;
    uint16_t *out;
    int32_t *err;
    int K, H, I;
};

// One pass over the K chunks for up to NT staged tokens.  `g` is the ring
// position shared (in lockstep) with the producer.
template <int NT, int STAGES>
__device__ __forceinline__ bool gateup_pass(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                            const uint16_t *xs, const Args &a, int g, int w,
                                            int lane, int j0, int nt, int row0) {
    constexpr int ST = Shape<GATEUP>::STAGE_BYTES;
    const int NK = a.H / 256;
    float acc[8][NT];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % STAGES;
        if (!mbar_wait(&full[s], (g / STAGES) & 1, kWaitLimit)) {
            record_error(a.err, 11, kc);
            return false;
        }
        const uint8_t *st = ring + s * ST;
        float wf[8][8];  // weights unpacked once per stage, reused by every token
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            unpack8(*reinterpret_cast<const uint4 *>(st + (4 * w + q) * 512 + lane * 16), wf[q]);
            unpack8(*reinterpret_cast<const uint4 *>(st + (16 + 4 * w + q) * 512 + lane * 16),
                    wf[4 + q]);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + t * a.H + kc * 256 + lane * 8), xf);
#pragma unroll
            for (int r = 0; r < 8; ++r) acc[r][t] += dot8f(wf[r], xf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = warp_sum(acc[r][t]);
    if (lane < nt) {
        uint16_t *dst = a.out + (size_t)(row0 + lane) * a.I + j0 + 4 * w;
        float y[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            y[q] = geglu_bf16(rbf(pick<NT, 8>(acc, q, lane)), rbf(pick<NT, 8>(acc, 4 + q, lane)));
        uint2 v;
        v.x = pack_bf2(y[0], y[1]);
        v.y = pack_bf2(y[2], y[3]);
        *reinterpret_cast<uint2 *>(dst) = v;
    }
    return true;
}

template <int NT, int STAGES>
__device__ __forceinline__ bool down_pass(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                          const uint16_t *xs, const Args &a, int g, int w,
                                          int lane, int h0, int nt, int row0) {
    constexpr int ST = Shape<DOWN>::STAGE_BYTES;
    const int NK = a.I / 64;
    const int gq = lane >> 3, c = lane & 7;
    const int rbase = 16 * w + 4 * gq;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % STAGES;
        if (!mbar_wait(&full[s], (g / STAGES) & 1, kWaitLimit)) {
            record_error(a.err, 12, kc);
            return false;
        }
        const uint8_t *st = ring + s * ST;
        float wf[4][8];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            unpack8(*reinterpret_cast<const uint4 *>(st + (rbase + r) * 128 + c * 16), wf[r]);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + t * a.I + kc * 64 + c * 8), xf);
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][t] += dot8f(wf[r], xf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float v = acc[r][t];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            acc[r][t] = v;
        }
    if (c < nt) {
        uint16_t *dst = a.out + (size_t)(row0 + c) * a.H + h0 + rbase;
        uint2 v;
        v.x = pack_bf2(pick<NT, 4>(acc, 0, c), pick<NT, 4>(acc, 1, c));
        v.y = pack_bf2(pick<NT, 4>(acc, 2, c), pick<NT, 4>(acc, 3, c));
        *reinterpret_cast<uint2 *>(dst) = v;
    }
    return true;
}

// Persistent: each CTA walks work items (active expert u, row block rb),
// u-major so neighbouring CTAs share an expert's token rows in L2.  The
// producer warp runs ahead across item boundaries, so the weight stream never
// drains between items; the compute warps restage the item's tokens behind a
// named barrier of their own.
template <int EPI, int NTMAX, int STAGES>
__global__ void __launch_bounds__(kThreads)
gemv_tma_kernel(const __grid_constant__ CUtensorMap tmW, Args a) {
    using S = Shape<EPI>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *ring = smem_align(smem_raw, 1024);
    const int LEN = (EPI == GATEUP) ? a.H : a.I;
    // token rows per unit (item x token pass), double-buffered, fetched by the
    // producer with 1-D bulk copies ahead of the compute warps
    uint16_t *xs0 = reinterpret_cast<uint16_t *>(ring + STAGES * S::STAGE_BYTES);
    uint64_t *full = reinterpret_cast<uint64_t *>(xs0 + 2 * NTMAX * LEN);
    uint64_t *empty = full + STAGES;
    uint64_t *ufull = empty + STAGES;
    uint64_t *uempty = ufull + 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows_per_blk = (EPI == GATEUP) ? S::ROWS / 2 : S::ROWS;  // j or h per item
    const int NRB = ((EPI == GATEUP) ? a.I : a.H) / rows_per_blk;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kComputeWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ufull[b], 1);
            mbar_init(&uempty[b], kComputeWarps);
        }
        fence_barrier_init();
        tma_prefetch(&tmW);
    }
    __syncthreads();  // barriers initialised
    const int NK = LEN / S::KC;
    int g = 0, u = 0;
    // one weight stage of unit (e, blk0) into the ring (producer lane only)
    auto stage = [&](int e, int blk0, int kc, int item) -> bool {
        const int s = g % STAGES;
        if (!mbar_wait(&empty[s], ((g / STAGES) & 1) ^ 1, kWaitLimit)) {
            record_error(a.err, 10, item);
            return false;
        }
        mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
        uint8_t *dst = ring + s * S::STAGE_BYTES;
        if (EPI == GATEUP) {
            const int r0 = e * 2 * a.I + blk0;
            tma_load_2d(dst, &tmW, &full[s], kc * S::KC, r0);
            tma_load_2d(dst + S::STAGE_BYTES / 2, &tmW, &full[s], kc * S::KC, r0 + a.I);
        } else {
            tma_load_2d(dst, &tmW, &full[s], kc * S::KC, e * a.H + blk0);
        }
        ++g;
        return true;
    };
    // Launch order: gate_up lets its dependent (this kernel's DOWN form) start
    // only after its own wait, i.e. once the routing and dispatch are
    // complete.  DOWN may then read the dispatch and stream the first weight
    // stages of its first item while gate_up is still running; it waits for
    // gate_up's output (its token rows) before loading any of them.
    int items, pre = 0;  // pre: weight stages of the first unit already issued
    if constexpr (EPI == GATEUP) {
        pdl_wait();  // the dispatch this kernel reads is complete
        pdl_trigger();
        items = *a.n_active * NRB;
    } else {
        pdl_trigger();
        items = *a.n_active * NRB;
        if (warp == kComputeWarps && lane == 0 && (int)blockIdx.x < items) {
            const int item = blockIdx.x;
            const int e = a.active[item / NRB], blk0 = (item % NRB) * rows_per_blk;
            const int lead = NK < STAGES ? NK : STAGES;
            for (; pre < lead; ++pre)
                if (!stage(e, blk0, pre, item)) {
                    pre = -1;
                    break;
                }
        }
        pdl_wait();  // gate_up's rows (this kernel's operands) are complete
    }
    if (warp == kComputeWarps) {
        if (lane != 0 || pre < 0) return;
        for (int item = blockIdx.x; item < items; item += gridDim.x) {
            const int e = a.active[item / NRB], blk0 = (item % NRB) * rows_per_blk;
            const int n = a.counts[e], base = a.offsets[e];
            for (int tc = 0; tc < n; tc += NTMAX, ++u) {
                // the weight stream first (it needs only e); the unit's operands
                // need the dispatch order, one more dependent load
                const int lead = NK < STAGES ? NK : STAGES;
                for (int kc = pre; kc < lead; ++kc)
                    if (!stage(e, blk0, kc, item)) return;
                pre = 0;  // only the first unit was started early
                const int b = u & 1;
                if (!mbar_wait(&uempty[b], ((u >> 1) & 1) ^ 1, kWaitLimit)) {
                    record_error(a.err, 13, item);
                    return;
                }
                const int nt = min(NTMAX, n - tc);
                uint16_t *xs = xs0 + b * NTMAX * LEN;
                mbar_arrive_expect_tx(&ufull[b], nt * LEN * 2);
                if (EPI == GATEUP) {
                    for (int r = 0; r < nt; ++r)
                        bulk_load(xs + r * LEN, a.in + (size_t)(a.perm[base + tc + r] / a.K) * a.H,
                                  LEN * 2, &ufull[b]);
                } else {
                    bulk_load(xs, a.in + (size_t)(base + tc) * a.I, nt * LEN * 2, &ufull[b]);
                }
                for (int kc = lead; kc < NK; ++kc)
                    if (!stage(e, blk0, kc, item)) return;
            }
        }
        return;
    }
    // compute warps (128 threads)
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int e = a.active[item / NRB], blk0 = (item % NRB) * rows_per_blk;
        const int n = a.counts[e], base = a.offsets[e];
        for (int tc = 0; tc < n; tc += NTMAX, g += NK, ++u) {
            const int nt = min(NTMAX, n - tc);
            const int b = u & 1;
            if (!mbar_wait(&ufull[b], (u >> 1) & 1, kWaitLimit)) {
                record_error(a.err, 14, item);
                return;
            }
            const uint16_t *xs = xs0 + b * NTMAX * LEN;
            bool ok = true;
            if (EPI == GATEUP) {
                if (nt == 1) ok = gateup_pass<1, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc);
                else if (nt == 2) { if constexpr (NTMAX >= 2) ok = gateup_pass<2, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc); }
                else if (nt <= 4) { if constexpr (NTMAX >= 4) ok = gateup_pass<4, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc); }
                else { if constexpr (NTMAX >= 8) ok = gateup_pass<8, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc); }
            } else {
                if (nt == 1) ok = down_pass<1, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc);
                else if (nt == 2) { if constexpr (NTMAX >= 2) ok = down_pass<2, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc); }
                else if (nt <= 4) { if constexpr (NTMAX >= 4) ok = down_pass<4, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc); }
                else { if constexpr (NTMAX >= 8) ok = down_pass<8, STAGES>(ring, full, empty, xs, a, g, warp, lane, blk0, nt, base + tc); }
            }
            // A timed-out wait leaves the ring inconsistent: every compute warp
            // waits on the same barriers, so all of them expire; leave at once.
            if (!ok) return;
            __syncwarp();
            if (lane == 0) mbar_arrive(&uempty[b]);  // this warp is done with the unit's rows
        }
    }
}

// ---------------------------------------------------------------- host side

bool make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint32_t kc,
              uint32_t box_rows) {
    return bf16_map_2d(m, base, inner, rows, kc, box_rows, false);
}

// Ring depth: about 64-96 KB of weights in flight per CTA (a CTA's stream is
// bounded by bytes in flight over the load latency), within the shared memory
// that still lets two CTAs share an SM at small token counts.
template <int EPI, int NTMAX>
constexpr int stages_for() {
    return EPI == DOWN ? 8 : (NTMAX <= 2 ? 6 : 4);
}

template <int EPI, int NTMAX>
size_t smem_bytes(int len) {
    constexpr int kStages = stages_for<EPI, NTMAX>();
    return 1024 + (size_t)kStages * Shape<EPI>::STAGE_BYTES + 2 * (size_t)NTMAX * len * 2 +
           16 * kStages + 32 + 64;
}

template <int EPI, int NTMAX>
cudaError_t set_attr() {
    return cudaFuncSetAttribute(gemv_tma_kernel<EPI, NTMAX, stages_for<EPI, NTMAX>()>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

// Grid: one CTA per possible work item, capped at the number that fit on the
// GPU at once (the kernel is persistent beyond that).
template <int EPI, int NTMAX>
cudaError_t launch_one(const CUtensorMap &m, const Args &a, int max_items, int len,
                       cudaStream_t s) {
    const size_t smem = smem_bytes<EPI, NTMAX>(len);
    const int dev = current_device();
    static int occ_cache[64][4] = {};  // per device, keyed by the token-row length class
    const int slot = len >= 2048 ? 0 : len >= 1024 ? 1 : len >= 512 ? 2 : 3;
    int &occ = occ_cache[dev & 63][slot];
    if (!occ) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ,
                                                      gemv_tma_kernel<EPI, NTMAX, stages_for<EPI, NTMAX>()>,
                                                      kThreads, smem);
        if (occ < 1) occ = 1;
    }
    int grid = grid_sms(dev) * occ;
    if (max_items < grid) grid = max_items;
    if (grid < 1) grid = 1;
    return launch_ex(gemv_tma_kernel<EPI, NTMAX, stages_for<EPI, NTMAX>()>, dim3(grid),
                     dim3(kThreads), smem, s,
                     true, m, a);
}

template <int EPI>
cudaError_t launch_ntmax(const CUtensorMap &m, const Args &a, int max_items, int len,
                         int max_rows, cudaStream_t s) {
    if (max_rows <= 1) return launch_one<EPI, 1>(m, a, max_items, len, s);
    if (max_rows <= 2) return launch_one<EPI, 2>(m, a, max_items, len, s);
    if (max_rows <= 4) return launch_one<EPI, 4>(m, a, max_items, len, s);
    return launch_one<EPI, 8>(m, a, max_items, len, s);
}

}  // namespace

cudaError_t gemv_tma_init() {
    cudaError_t e;
    if ((e = set_attr<GATEUP, 1>()) || (e = set_attr<GATEUP, 2>()) || (e = set_attr<GATEUP, 4>()) ||
        (e = set_attr<GATEUP, 8>()) || (e = set_attr<DOWN, 1>()) || (e = set_attr<DOWN, 2>()) ||
        (e = set_attr<DOWN, 4>()) || (e = set_attr<DOWN, 8>()))
        return e;
    return cudaSuccess;
}

bool gemv_tma_supported(int H, int I) {
    return encode_tiled_fn() != nullptr && H % 256 == 0 && H % 64 == 0 && I % 64 == 0 && I % 16 == 0;
}

cudaError_t launch_gemv_tma_gateup(const uint16_t *x, int K, const Dispatch &d,
                                   const ExpertWeights &w, int H, int I, int E, int max_rows,
                                   uint16_t *yp, int32_t *err, cudaStream_t s, int *launches) {
    CUtensorMap m;
    if (!make_map(&m, w.gu, H, (uint64_t)E * 2 * I, 256, 16)) return cudaErrorInvalidValue;
    Args a{x, d.perm, d.offsets, d.counts, d.active, d.n_active, yp, err, K, H, I};
    const int max_active = min(E, max_rows * K > 0 ? max_rows * K : E);
    cudaError_t e = launch_ntmax<GATEUP>(m, a, max_active * (I / 16), H, max_rows, s);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemv_tma_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                                 int H, int I, int E, int max_k, int max_rows, uint16_t *op, int32_t *err,
                                 cudaStream_t s, int *launches) {
    CUtensorMap m;
    if (!make_map(&m, w.dn, I, (uint64_t)E * H, 64, 64)) return cudaErrorInvalidValue;
    Args a{yp, d.perm, d.offsets, d.counts, d.active, d.n_active, op, err, 0, H, I};
    const int max_active = min(E, max_rows * max_k);
    cudaError_t e = launch_ntmax<DOWN>(m, a, max_active * (H / 64), I, max_rows, s);
    if (launches) ++*launches;
    return e;
}

}  // namespace apt
