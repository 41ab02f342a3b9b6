// gemv_tma_q.cu -- decode-sized grouped expert GEMV over MLX affine 4/8-bit
// experts, with the packed weights streamed by TMA.
//
// Restates the gather_qmm path of ESExperts::sparseForward
// (aptransformer/ESExperts.mm:50-57) for decode-sized token groups.  Each
// 64-element group of a weight row dequantises as w = scale*q + bias
// (mx::quantize affine layout: 32/bits values per uint32, low bits first); a
// lane's slice of 8 elements lies inside one group, so its contribution is
// scale*sum(q*x) + bias*sum(x) in f32.  Rounding points as in gemv_tma.cu:
// gate/up -> bf16, GeGLU in f32 -> bf16, y -> bf16, down -> bf16.
//
// Same structure as the bf16 TMA GEMV: persistent CTAs over (active expert,
// row block) items; a producer warp streams the packed rows into a deep
// shared-memory ring (4-bit rows are a quarter of the bf16 bytes, so the ring
// has more, smaller stages).  The producer also fetches each unit's operands
// ahead of the compute warps, into one of two buffers: the item's (scale,
// bias) pairs by a 2-D TMA copy, its token rows by 1-D bulk copies.  The
// compute warps never wait on a global load of their own, so a CTA's items
// follow one another without a memory round trip in between.  Waits are
// bounded; expiry records an error.
#include <cuda.h>

#include "common.cuh"
#include "launch_util.h"
#include "moe_internal.h"
#include "sm100_ptx.cuh"

namespace apt {

namespace {

using namespace sm100;

constexpr int kComputeWarps = 4;
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr long long kWaitLimit = 4000000000LL;
enum { GATEUP = 0, DOWN = 1 };

template <int EPI, int BITS>
struct QShape {
    static constexpr int ROWS = EPI == GATEUP ? 32 : 64;   // weight rows per item
    static constexpr int KC = EPI == GATEUP ? 256 : 64;    // elements per row per stage
    static constexpr int ROW_WORDS = KC * BITS / 32;       // packed words per row per stage
    static constexpr int STAGE_BYTES = ROWS * ROW_WORDS * 4;
    static constexpr int STAGES = STAGE_BYTES <= 2048 ? 16 : 8;
    static constexpr int LANE_WORDS = 8 * BITS / 32;       // words holding a lane's 8 elements
};

__device__ __forceinline__ void record_error(int32_t *err, int code, int where) {
    if (atomicCAS(err, 0, code) == 0) err[1] = where;
}

// Packed unsigned q -> f32 without the int-to-float unit: OR-ing q into the
// mantissa of 2^23 gives exactly 2^23 + q, and subtracting 2^23 leaves q.
template <int BITS>
__device__ __forceinline__ void unpack_q8(const uint32_t *w, float (&q)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
        q[i] = __fsub_rn(__uint_as_float(((w[i * BITS / 32] >> ((i * BITS) & 31)) &
                                          ((1u << BITS) - 1u)) |
                                         0x4B000000u),
                         8388608.0f);
}

template <int NT, int R>
__device__ __forceinline__ float pick(const float (&acc)[R][NT], int r, int t) {
    float v = 0.f;
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
        if (tt == t) v = acc[r][tt];
    return v;
}

struct QArgs {
    const uint16_t *in;
    const int32_t *perm, *offsets, *counts, *active, *n_active;
    const uint32_t *sb;  // [E*rows, gp] (scale | bias << 16) pairs, rows padded to gp
    uint16_t *out;
    int32_t *err;
    int K, H, I;
    int gp;              // groups per row, rounded up to 4 (16-byte rows)
};

template <int NT, int BITS>
__device__ __forceinline__ bool gateup_pass_q(const uint8_t *ring, uint64_t *full,
                                              uint64_t *empty, const uint16_t *xs,
                                              const uint32_t *sbp, const QArgs &a, int g, int w,
                                              int lane, int j0, int nt, int row0) {
    using S = QShape<GATEUP, BITS>;
    const int NK = a.H / S::KC, G = a.gp;
    float acc[8][NT];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S::STAGES;
        if (!mbar_wait(&full[s], (g / S::STAGES) & 1, kWaitLimit)) {
            record_error(a.err, 21, kc);
            return false;
        }
        const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + s * S::STAGE_BYTES);
        const int grp = kc * (S::KC / 64) + (lane >> 3);
        float qf[8][8], sr[8], br[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int row = (q < 4) ? 4 * w + q : 16 + 4 * w + (q - 4);
            uint32_t wd[S::LANE_WORDS];
#pragma unroll
            for (int k = 0; k < S::LANE_WORDS; ++k)
                wd[k] = st[row * S::ROW_WORDS + lane * S::LANE_WORDS + k];
            unpack_q8<BITS>(wd, qf[q]);
            const uint32_t pv = sbp[row * G + grp];
            sr[q] = bf_lo(pv);
            br[q] = bf_hi(pv);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + t * a.H + kc * S::KC + lane * 8), xf);
            float xsum = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) xsum += xf[i];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                float qx = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) qx = fmaf(qf[r][i], xf[i], qx);
                acc[r][t] += fmaf(sr[r], qx, br[r] * xsum);
            }
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

template <int NT, int BITS>
__device__ __forceinline__ bool down_pass_q(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                            const uint16_t *xs, const uint32_t *sbp,
                                            const QArgs &a, int g, int w, int lane, int h0, int nt,
                                            int row0) {
    using S = QShape<DOWN, BITS>;
    const int NK = a.I / S::KC, G = a.gp;
    const int gq = lane >> 3, c = lane & 7;
    const int rbase = 16 * w + 4 * gq;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S::STAGES;
        if (!mbar_wait(&full[s], (g / S::STAGES) & 1, kWaitLimit)) {
            record_error(a.err, 22, kc);
            return false;
        }
        const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + s * S::STAGE_BYTES);
        float qf[4][8], sr[4], br[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t wd[S::LANE_WORDS];
#pragma unroll
            for (int k = 0; k < S::LANE_WORDS; ++k)
                wd[k] = st[(rbase + r) * S::ROW_WORDS + c * S::LANE_WORDS + k];
            unpack_q8<BITS>(wd, qf[r]);
            const uint32_t pv = sbp[(rbase + r) * G + kc];
            sr[r] = bf_lo(pv);
            br[r] = bf_hi(pv);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + t * a.I + kc * S::KC + c * 8), xf);
            float xsum = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) xsum += xf[i];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float qx = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) qx = fmaf(qf[r][i], xf[i], qx);
                acc[r][t] += fmaf(sr[r], qx, br[r] * xsum);
            }
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

template <int EPI, int BITS, int NTMAX>
__global__ void __launch_bounds__(kThreads)
gemv_tma_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmSB,
                  QArgs a) {
    using S = QShape<EPI, BITS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    const int LEN = (EPI == GATEUP) ? a.H : a.I;
    const int Gp = a.gp;
    // per unit (item x token pass), double-buffered: token rows, (scale, bias)
    uint16_t *xs0 = reinterpret_cast<uint16_t *>(ring + S::STAGES * S::STAGE_BYTES);
    uint32_t *sb0 = reinterpret_cast<uint32_t *>(
        (reinterpret_cast<uintptr_t>(xs0 + 2 * NTMAX * LEN) + 127) & ~uintptr_t(127));
    uint64_t *full = reinterpret_cast<uint64_t *>(sb0 + 2 * S::ROWS * Gp);
    uint64_t *empty = full + S::STAGES;
    uint64_t *ufull = empty + S::STAGES;
    uint64_t *uempty = ufull + 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows_per_blk = (EPI == GATEUP) ? S::ROWS / 2 : S::ROWS;
    const int NRB = ((EPI == GATEUP) ? a.I : a.H) / rows_per_blk;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kComputeWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ufull[b], 1);
            mbar_init(&uempty[b], kComputeWarps);
        }
        fence_barrier_init();
        tma_prefetch(&tmQ);
        tma_prefetch(&tmSB);
    }
    pdl_trigger();
    pdl_wait();
    const int items = *a.n_active * NRB;
    __syncthreads();
    const int NK = LEN / S::KC;
    if (warp == kComputeWarps) {
        if (lane != 0) return;
        int g = 0, u = 0;
        // one weight stage of unit (e, blk0) into the ring
        auto stage = [&](int e, int blk0, int kc, int item) -> bool {
            const int s = g % S::STAGES;
            if (!mbar_wait(&empty[s], ((g / S::STAGES) & 1) ^ 1, kWaitLimit)) {
                record_error(a.err, 20, item);
                return false;
            }
            mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
            uint8_t *dst = ring + s * S::STAGE_BYTES;
            if (EPI == GATEUP) {
                const int r0 = e * 2 * a.I + blk0;
                tma_load_2d(dst, &tmQ, &full[s], kc * S::ROW_WORDS, r0);
                tma_load_2d(dst + S::STAGE_BYTES / 2, &tmQ, &full[s], kc * S::ROW_WORDS, r0 + a.I);
            } else {
                tma_load_2d(dst, &tmQ, &full[s], kc * S::ROW_WORDS, e * a.H + blk0);
            }
            ++g;
            return true;
        };
        for (int item = blockIdx.x; item < items; item += gridDim.x) {
            const int e = a.active[item / NRB], blk0 = (item % NRB) * rows_per_blk;
            const int n = a.counts[e], base = a.offsets[e];
            for (int tc = 0; tc < n; tc += NTMAX, ++u) {
                // the weight stream first (it needs only e); the unit's operands
                // need the dispatch order, one more dependent load
                const int lead = NK < S::STAGES ? NK : S::STAGES;
                for (int kc = 0; kc < lead; ++kc)
                    if (!stage(e, blk0, kc, item)) return;
                const int b = u & 1;
                if (!mbar_wait(&uempty[b], ((u >> 1) & 1) ^ 1, kWaitLimit)) {
                    record_error(a.err, 23, item);
                    return;
                }
                const int nt = min(NTMAX, n - tc);
                uint16_t *xs = xs0 + b * NTMAX * LEN;
                uint32_t *sbp = sb0 + b * S::ROWS * Gp;
                mbar_arrive_expect_tx(&ufull[b], S::ROWS * Gp * 4 + nt * LEN * 2);
                if (EPI == GATEUP) {
                    const int r0 = e * 2 * a.I + blk0;
                    tma_load_2d(sbp, &tmSB, &ufull[b], 0, r0);
                    tma_load_2d(sbp + (S::ROWS / 2) * Gp, &tmSB, &ufull[b], 0, r0 + a.I);
                    for (int r = 0; r < nt; ++r)
                        bulk_load(xs + r * LEN, a.in + (size_t)(a.perm[base + tc + r] / a.K) * a.H,
                                  LEN * 2, &ufull[b]);
                } else {
                    tma_load_2d(sbp, &tmSB, &ufull[b], 0, e * a.H + blk0);
                    bulk_load(xs, a.in + (size_t)(base + tc) * a.I, nt * LEN * 2, &ufull[b]);
                }
                for (int kc = lead; kc < NK; ++kc)
                    if (!stage(e, blk0, kc, item)) return;
            }
        }
        return;
    }
    int g = 0, u = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int e = a.active[item / NRB], blk0 = (item % NRB) * rows_per_blk;
        const int n = a.counts[e], base = a.offsets[e];
        for (int tc = 0; tc < n; tc += NTMAX, g += NK, ++u) {
            const int nt = min(NTMAX, n - tc);
            const int b = u & 1;
            if (!mbar_wait(&ufull[b], (u >> 1) & 1, kWaitLimit)) {
                record_error(a.err, 24, item);
                return;
            }
            const uint16_t *xs = xs0 + b * NTMAX * LEN;
            const uint32_t *sbp = sb0 + b * S::ROWS * Gp;
            bool ok = true;
            if (EPI == GATEUP) {
                if (nt == 1) ok = gateup_pass_q<1, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc);
                else if (nt == 2) { if constexpr (NTMAX >= 2) ok = gateup_pass_q<2, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc); }
                else if (nt <= 4) { if constexpr (NTMAX >= 4) ok = gateup_pass_q<4, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc); }
                else { if constexpr (NTMAX >= 8) ok = gateup_pass_q<8, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc); }
            } else {
                if (nt == 1) ok = down_pass_q<1, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc);
                else if (nt == 2) { if constexpr (NTMAX >= 2) ok = down_pass_q<2, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc); }
                else if (nt <= 4) { if constexpr (NTMAX >= 4) ok = down_pass_q<4, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc); }
                else { if constexpr (NTMAX >= 8) ok = down_pass_q<8, BITS>(ring, full, empty, xs, sbp, a, g, warp, lane, blk0, nt, base + tc); }
            }
            // A timed-out wait leaves the rings inconsistent: every compute warp
            // waits on the same barriers, so all of them expire; leave at once.
            if (!ok) return;
            __syncwarp();
            if (lane == 0) mbar_arrive(&uempty[b]);  // this warp is done with the unit's operands
        }
    }
}

// ---------------------------------------------------------------- host side

// packed [rows, words] uint32 tensor, box {box_words, box_rows}, no swizzle
bool make_qmap(CUtensorMap *m, const void *base, uint64_t words, uint64_t rows,
               uint32_t box_words, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {words, rows};
    cuuint64_t strides[1] = {words * 4};
    cuuint32_t box[2] = {box_words, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

template <int EPI, int BITS, int NTMAX>
size_t qsmem_bytes(int len, int gp) {
    using S = QShape<EPI, BITS>;
    return 1024 + (size_t)S::STAGES * S::STAGE_BYTES + 2 * (size_t)NTMAX * len * 2 + 128 +
           2 * (size_t)S::ROWS * gp * 4 + 16 * S::STAGES + 32 + 64;
}

template <int EPI, int BITS, int NTMAX>
cudaError_t qlaunch_one(const CUtensorMap &m, const CUtensorMap &sbm, const QArgs &a,
                        int max_items, int len, cudaStream_t s) {
    const size_t smem = qsmem_bytes<EPI, BITS, NTMAX>(len, a.gp);
    static int occ_cache[64] = {};
    const int dev = current_device();
    int &occ = occ_cache[dev & 63];
    if (!occ) {
        cudaFuncSetAttribute(gemv_tma_q_kernel<EPI, BITS, NTMAX>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_tma_q_kernel<EPI, BITS, NTMAX>,
                                                      kThreads, smem);
        if (occ < 1) occ = 1;
    }
    int grid = grid_sms(dev) * occ;
    if (max_items < grid) grid = max_items;
    if (grid < 1) grid = 1;
    return launch_ex(gemv_tma_q_kernel<EPI, BITS, NTMAX>, dim3(grid), dim3(kThreads), smem, s,
                     true, m, sbm, a);
}

template <int EPI, int BITS>
cudaError_t qlaunch(const CUtensorMap &m, const CUtensorMap &sbm, const QArgs &a, int max_items,
                    int len, int max_rows, cudaStream_t s) {
    if (max_rows <= 1) return qlaunch_one<EPI, BITS, 1>(m, sbm, a, max_items, len, s);
    if (max_rows <= 2) return qlaunch_one<EPI, BITS, 2>(m, sbm, a, max_items, len, s);
    if (max_rows <= 4) return qlaunch_one<EPI, BITS, 4>(m, sbm, a, max_items, len, s);
    return qlaunch_one<EPI, BITS, 8>(m, sbm, a, max_items, len, s);
}

}  // namespace

bool gemv_tma_q_supported(int H, int I, int bits) {
    return encode_tiled_fn() != nullptr && (bits == 4 || bits == 8) && H % 256 == 0 &&
           I % 64 == 0;
}

cudaError_t launch_gemv_tma_q_gateup(const uint16_t *x, int K, const Dispatch &d,
                                     const ExpertWeights &w, int H, int I, int E, int max_rows,
                                     uint16_t *yp, int32_t *err, cudaStream_t s, int *launches) {
    CUtensorMap m, sbm;
    const uint32_t row_words = 256 * w.bits / 32;
    const int gp = sb_row_words(H);
    if (!make_qmap(&m, w.gu_q, (uint64_t)H * w.bits / 32, (uint64_t)E * 2 * I, row_words, 16) ||
        !make_qmap(&sbm, w.gu_sb, gp, (uint64_t)E * 2 * I, gp, 16))
        return cudaErrorInvalidValue;
    QArgs a{x, d.perm, d.offsets, d.counts, d.active, d.n_active, w.gu_sb, yp, err, K, H, I, gp};
    const int max_items = min(E, max_rows * K) * (I / 16);
    cudaError_t e = (w.bits == 4) ? qlaunch<GATEUP, 4>(m, sbm, a, max_items, H, max_rows, s)
                                  : qlaunch<GATEUP, 8>(m, sbm, a, max_items, H, max_rows, s);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemv_tma_q_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                                   int H, int I, int E, int max_k, int max_rows, uint16_t *op,
                                   int32_t *err, cudaStream_t s, int *launches) {
    CUtensorMap m, sbm;
    const uint32_t row_words = 64 * w.bits / 32;
    const int gp = sb_row_words(I);
    if (!make_qmap(&m, w.dn_q, (uint64_t)I * w.bits / 32, (uint64_t)E * H, row_words, 64) ||
        !make_qmap(&sbm, w.dn_sb, gp, (uint64_t)E * H, gp, 64))
        return cudaErrorInvalidValue;
    QArgs a{yp, d.perm, d.offsets, d.counts, d.active, d.n_active, w.dn_sb, op, err, 0, H, I, gp};
    const int max_items = min(E, max_rows * max_k) * (H / 64);
    cudaError_t e = (w.bits == 4) ? qlaunch<DOWN, 4>(m, sbm, a, max_items, I, max_rows, s)
                                  : qlaunch<DOWN, 8>(m, sbm, a, max_items, I, max_rows, s);
    if (launches) ++*launches;
    return e;
}

}  // namespace apt
