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
    // ~64 KB of packed weights in flight per CTA (a CTA's stream is bounded by
    // bytes in flight over the load latency)
    static constexpr int STAGES = (65536 / STAGE_BYTES) < 4 ? 4 : (65536 / STAGE_BYTES) > 32 ? 32
                                                                 : (65536 / STAGE_BYTES);
    static constexpr int LANE_WORDS = 8 * BITS / 32;       // words holding a lane's 8 elements
};

__device__ __forceinline__ void record_error(int32_t *err, int code, int where) {
    if (atomicCAS(err, 0, code) == 0) err[1] = where;
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

// ---------------------------------------------------------------- 4-bit on the tensor cores
//
// For 4-bit codes the SIMT pass above is issue-bound (about five instructions
// per weight to unpack and multiply).  This variant turns two codes into a
// bf16 pair with three integer instructions and lets mma.sync.m16n8k16 do the
// multiplies for all (up to 8) tokens at once.  A code q becomes the bf16
// value 128 + q exactly (0x4300 | q: exponent of 128, q in the low mantissa
// bits), so a 16x16 weight tile times the tokens' x gives
//   D = sum (128 + q) x = sum q x + 128 sum x
// with exact products and f32 sums; per 64-element group the affine
// dequantisation then adds  s * D + (b - 128 s) * sum x,  i.e. the same
// s * sum q x + b * sum x  as the SIMT pass, in a different summation order.
// (mma.sync rather than tcgen05: at T <= 8 the multiply is a small part of
// the work and the operands are built in registers; a tcgen05 MMA would need
// them written to shared memory first.)

// gate_up, 32 rows (16 gate + 16 up) x one 256-wide stage per pass step;
// warp w takes the stage's group w (k = 64w .. 64w+63) for both row halves.
// Partial sums meet in shared memory at the end of the item.
template <int NT>
__device__ __forceinline__ bool gateup_pass_mma(const uint8_t *ring, uint64_t *full,
                                                uint64_t *empty, const uint16_t *xs,
                                                const uint32_t *sbp, const float *xsum,
                                                float *red, const QArgs &a, int g, int w,
                                                int lane, int j0, int nt, int row0) {
    using S = QShape<GATEUP, 4>;
    const int NK = a.H / S::KC, G = a.gp, LEN = a.H;
    const int gid = lane >> 2, t = lane & 3;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S::STAGES;
        if (!mbar_wait(&full[s], (g / S::STAGES) & 1, kWaitLimit)) {
            record_error(a.err, 25, kc);
            return false;
        }
        const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + s * S::STAGE_BYTES);
        const int grp = kc * (S::KC / 64) + w;  // this warp's group of the row
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 16-wide chunks of the group
            const int k0 = w * 64 + c * 16;  // within the stage
            uint32_t b0 = 0u, b1 = 0u;
            if (gid < nt) {
                const uint16_t *xr = xs + gid * LEN + kc * S::KC + k0 + 2 * t;
                b0 = *reinterpret_cast<const uint32_t *>(xr);
                b1 = *reinterpret_cast<const uint32_t *>(xr + 8);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // gate rows 0..15, up rows 16..31
                const uint32_t *r0 = st + (h * 16 + gid) * S::ROW_WORDS + k0 / 8;
                const uint32_t *r1 = r0 + 8 * S::ROW_WORDS;
                uint32_t af[4];
                q4_pair(r0[0], r0[1], t, af[0], af[2]);
                q4_pair(r1[0], r1[1], t, af[1], af[3]);
                mma_bf16_16816(d[h], af, b0, b1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        // affine dequantisation of this group: s*D + (b - 128 s)*sum(x)
        const float xs0 = (2 * t < nt) ? xsum[(2 * t) * G + grp] : 0.f;
        const float xs1 = (2 * t + 1 < nt) ? xsum[(2 * t + 1) * G + grp] : 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t p0 = sbp[(h * 16 + gid) * G + grp];
            const uint32_t p1 = sbp[(h * 16 + gid + 8) * G + grp];
            const float s0 = bf_lo(p0), c0 = fmaf(-128.f, s0, bf_hi(p0));
            const float s1 = bf_lo(p1), c1 = fmaf(-128.f, s1, bf_hi(p1));
            acc[h][0] += fmaf(s0, d[h][0], c0 * xs0);
            acc[h][1] += fmaf(s0, d[h][1], c0 * xs1);
            acc[h][2] += fmaf(s1, d[h][2], c1 * xs0);
            acc[h][3] += fmaf(s1, d[h][3], c1 * xs1);
        }
    }
    // red[w][row 0..31][tok 0..7]
    float *rw = red + w * 256;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        rw[(h * 16 + gid) * 8 + 2 * t] = acc[h][0];
        rw[(h * 16 + gid) * 8 + 2 * t + 1] = acc[h][1];
        rw[(h * 16 + gid + 8) * 8 + 2 * t] = acc[h][2];
        rw[(h * 16 + gid + 8) * 8 + 2 * t + 1] = acc[h][3];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32));
    {
        const int j = threadIdx.x >> 3, tok = threadIdx.x & 7;  // 16 j x 8 tokens
        if (tok < nt) {
            float gsum = 0.f, usum = 0.f;
#pragma unroll
            for (int q = 0; q < kComputeWarps; ++q) {
                gsum += red[q * 256 + j * 8 + tok];
                usum += red[q * 256 + (16 + j) * 8 + tok];
            }
            a.out[(size_t)(row0 + tok) * a.I + j0 + j] = f2bf(geglu_bf16(rbf(gsum), rbf(usum)));
        }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32));  // red free for the next item
    return true;
}

// down, 64 rows x one 64-wide stage (= one group); warp w owns rows 16w..16w+15.
template <int NT>
__device__ __forceinline__ bool down_pass_mma(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                              const uint16_t *xs, const uint32_t *sbp,
                                              const float *xsum, const QArgs &a, int g, int w,
                                              int lane, int h0, int nt, int row0) {
    using S = QShape<DOWN, 4>;
    const int NK = a.I / S::KC, G = a.gp, LEN = a.I;
    const int gid = lane >> 2, t = lane & 3;
    const int rb = 16 * w;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S::STAGES;
        if (!mbar_wait(&full[s], (g / S::STAGES) & 1, kWaitLimit)) {
            record_error(a.err, 26, kc);
            return false;
        }
        const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + s * S::STAGE_BYTES);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t b0 = 0u, b1 = 0u;
            if (gid < nt) {
                const uint16_t *xr = xs + gid * LEN + kc * S::KC + c * 16 + 2 * t;
                b0 = *reinterpret_cast<const uint32_t *>(xr);
                b1 = *reinterpret_cast<const uint32_t *>(xr + 8);
            }
            const uint32_t *r0 = st + (rb + gid) * S::ROW_WORDS + c * 2;
            const uint32_t *r1 = r0 + 8 * S::ROW_WORDS;
            uint32_t af[4];
            q4_pair(r0[0], r0[1], t, af[0], af[2]);
            q4_pair(r1[0], r1[1], t, af[1], af[3]);
            mma_bf16_16816(d, af, b0, b1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        const float xs0 = (2 * t < nt) ? xsum[(2 * t) * G + kc] : 0.f;
        const float xs1 = (2 * t + 1 < nt) ? xsum[(2 * t + 1) * G + kc] : 0.f;
        const uint32_t p0 = sbp[(rb + gid) * G + kc];
        const uint32_t p1 = sbp[(rb + gid + 8) * G + kc];
        const float s0 = bf_lo(p0), c0 = fmaf(-128.f, s0, bf_hi(p0));
        const float s1 = bf_lo(p1), c1 = fmaf(-128.f, s1, bf_hi(p1));
        acc[0] += fmaf(s0, d[0], c0 * xs0);
        acc[1] += fmaf(s0, d[1], c0 * xs1);
        acc[2] += fmaf(s1, d[2], c1 * xs0);
        acc[3] += fmaf(s1, d[3], c1 * xs1);
    }
    // rows rb+gid, rb+gid+8; tokens 2t, 2t+1
    if (2 * t < nt) {
        a.out[(size_t)(row0 + 2 * t) * a.H + h0 + rb + gid] = f2bf(acc[0]);
        a.out[(size_t)(row0 + 2 * t) * a.H + h0 + rb + gid + 8] = f2bf(acc[2]);
    }
    if (2 * t + 1 < nt) {
        a.out[(size_t)(row0 + 2 * t + 1) * a.H + h0 + rb + gid] = f2bf(acc[1]);
        a.out[(size_t)(row0 + 2 * t + 1) * a.H + h0 + rb + gid + 8] = f2bf(acc[3]);
    }
    return true;
}

template <int EPI, int BITS, int NTMAX, bool MMA = false>
__global__ void __launch_bounds__(kThreads)
gemv_tma_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmSB,
                  QArgs a) {
    using S = QShape<EPI, BITS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *ring = smem_align(smem_raw, 1024);
    const int LEN = (EPI == GATEUP) ? a.H : a.I;
    const int Gp = a.gp;
    // per unit (item x token pass), double-buffered: token rows, (scale, bias)
    uint16_t *xs0 = reinterpret_cast<uint16_t *>(ring + S::STAGES * S::STAGE_BYTES);
    uint32_t *sb0 = reinterpret_cast<uint32_t *>(
        smem_align(reinterpret_cast<uint8_t *>(xs0 + 2 * NTMAX * LEN), 128));
    // MMA variant: per-unit sums of x over each group, and gate_up's
    // cross-warp partial sums
    float *xsum = reinterpret_cast<float *>(sb0 + 2 * S::ROWS * Gp);
    float *red = xsum + (MMA ? NTMAX * Gp : 0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem_align(
        reinterpret_cast<uint8_t *>(red + (MMA && EPI == GATEUP ? kComputeWarps * 256 : 0)), 8));
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
            if constexpr (MMA && BITS == 4) {
                // sum of x over every 64-element group, per token of the unit
                asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32));  // old sums read
                const int G = LEN / 64;
                for (int v = threadIdx.x; v < nt * G; v += kComputeWarps * 32) {
                    const int tok = v / G, gi = v - tok * G;
                    const uint4 *xp = reinterpret_cast<const uint4 *>(xs + tok * LEN + gi * 64);
                    float sum = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        float f[8];
                        unpack8(xp[q], f);
#pragma unroll
                        for (int i = 0; i < 8; ++i) sum += f[i];
                    }
                    xsum[tok * Gp + gi] = sum;
                }
                asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32));
                if (EPI == GATEUP)
                    ok = gateup_pass_mma<NTMAX>(ring, full, empty, xs, sbp, xsum, red, a, g, warp,
                                                lane, blk0, nt, base + tc);
                else
                    ok = down_pass_mma<NTMAX>(ring, full, empty, xs, sbp, xsum, a, g, warp, lane,
                                              blk0, nt, base + tc);
            } else if (EPI == GATEUP) {
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

template <int EPI, int BITS, int NTMAX, bool MMA>
size_t qsmem_bytes(int len, int gp) {
    using S = QShape<EPI, BITS>;
    return 1024 + (size_t)S::STAGES * S::STAGE_BYTES + 2 * (size_t)NTMAX * len * 2 + 128 +
           2 * (size_t)S::ROWS * gp * 4 + (MMA ? (size_t)NTMAX * gp * 4 : 0) +
           (MMA && EPI == GATEUP ? (size_t)kComputeWarps * 256 * 4 : 0) + 8 + 16 * S::STAGES +
           32 + 64;
}

template <int EPI, int BITS, int NTMAX, bool MMA>
cudaError_t qlaunch_one(const CUtensorMap &m, const CUtensorMap &sbm, const QArgs &a,
                        int max_items, int len, cudaStream_t s) {
    const size_t smem = qsmem_bytes<EPI, BITS, NTMAX, MMA>(len, a.gp);
    static int occ_cache[64] = {};
    const int dev = current_device();
    int &occ = occ_cache[dev & 63];
    if (!occ) {
        cudaFuncSetAttribute(gemv_tma_q_kernel<EPI, BITS, NTMAX, MMA>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_tma_q_kernel<EPI, BITS, NTMAX, MMA>,
                                                      kThreads, smem);
        if (occ < 1) occ = 1;
    }
    int grid = grid_sms(dev) * occ;
    if (max_items < grid) grid = max_items;
    if (grid < 1) grid = 1;
    return launch_ex(gemv_tma_q_kernel<EPI, BITS, NTMAX, MMA>, dim3(grid), dim3(kThreads), smem, s,
                     true, m, sbm, a);
}

template <int EPI, int BITS>
cudaError_t qlaunch(const CUtensorMap &m, const CUtensorMap &sbm, const QArgs &a, int max_items,
                    int len, int max_rows, cudaStream_t s) {
    // 4-bit codes on the tensor cores (mma passes), 8-bit on the SIMT passes
    constexpr bool M = (BITS == 4);
    if (max_rows <= 1) return qlaunch_one<EPI, BITS, 1, M>(m, sbm, a, max_items, len, s);
    if (max_rows <= 2) return qlaunch_one<EPI, BITS, 2, M>(m, sbm, a, max_items, len, s);
    if (max_rows <= 4) return qlaunch_one<EPI, BITS, 4, M>(m, sbm, a, max_items, len, s);
    return qlaunch_one<EPI, BITS, 8, M>(m, sbm, a, max_items, len, s);
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
