// gemm_sm100.cu -- prefill grouped expert GEMM on the 5th-generation tensor
// cores (tcgen05 + TMEM), fed by TMA.
//
// Restates the gather_mm path of ESExperts::sparseForward
// (aptransformer/ESExperts.mm:50-57) for prefill-sized token groups, after
// the dispatch grouped the (token, k) rows by expert:
//   gate_up: yp[r, j] = bf16( bf16(gelu(bf16(xp_r . Wg_j))) * bf16(xp_r . Wu_j) )
//   down:    op[r, h] = bf16( yp_r . Wd_h )
// with f32 accumulation in TMEM and the GeGLU fused into the epilogue.
//
// One persistent CTA per SM walks a static tile list (m-tile of 128 rows of
// one expert x n-tile of the weights, n fastest) with three warp roles:
//   warp 0      TMA producer: A (activation rows) and B (weight rows) tiles,
//               128-byte swizzled, into a STAGES-deep shared-memory ring
//   warp 1      owns TMEM (512 columns = two accumulators) and issues
//               tcgen05.mma (M=128, N=BN, K=16) from one thread
//   warps 2..5  epilogue: tcgen05.ld from TMEM, GeGLU / bf16 rounding,
//               stores; overlaps the next tile's MMAs (double buffer)
// For gate_up a B tile is BN2 gate rows followed by the BN2 matching up rows
// (two TMA boxes), so each accumulator row holds g and u for the same j.
// Every mbarrier wait is bounded; on expiry the kernel records an error code
// and leaves through the normal exit (TMEM released).  Every TMA load is a
// plain per-CTA load from this GPU's own memory.
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "moe_internal.h"
#include "launch_util.h"
#include "sm100_ptx.cuh"
#include "gemm_epilogue.cuh"

namespace apt {

namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;                  // one 128-byte swizzle atom of bf16
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kAccStride = 256;          // TMEM columns between the two accumulators
constexpr long long kWaitLimit = 4000000000LL;  // cycles (~2 s) before giving up
constexpr int kMaxExperts = 256;
constexpr int kStageC = 4 * 2 * 4096;    // down: 2 x 4 KB store boxes per epilogue warp
// QB = 4 (MLX affine 4-bit experts, 64-element groups): eight more warps
// dequantise each stage's packed codes into the bf16 B tile
constexpr int kDqThreads = 256;
constexpr int kBRing = 3;  // dequantised B tiles in flight (QB)

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z),
                 "r"(w)
                 : "memory");
}

// EPI_GATEUP_G: gate_up whose A rows are gathered from the token rows by the
// TMA (tile::gather4, 4 rows per copy) through the dispatch permutation, so no
// expert-sorted copy of the activations is materialised.  Used for small row
// counts per expert: a full 128-row stage takes 32 gather copies, which the
// TMA issues far slower than one tiled copy (measured 2.8x slower gate_up at
// 512 rows per expert), while a tile of a few rows takes one or two.
enum { EPI_GATEUP = 0, EPI_DOWN = 1, EPI_F32 = 2, EPI_GATEUP_G = 3 };

template <int BN>
struct Smem {
    static constexpr int A_BYTES = kBM * kBK * 2;
    static constexpr int B_BYTES = BN * kBK * 2;
};

__device__ __forceinline__ void record_error(int32_t *err, int code, int where) {
    if (atomicCAS(err, 0, code) == 0) err[1] = where;
}

// Tile t -> (expert, m-tile within expert, n-tile).  mtp = m-tile prefix.
__device__ __forceinline__ void decode_tile(int t, int NT, const int *mtp, int E, int &e, int &mloc,
                                            int &nt) {
    const int mt = t / NT;
    nt = t - mt * NT;
    int lo = 0, hi = E - 1;  // first e with mtp[e+1] > mt
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (mtp[mid + 1] > mt) hi = mid;
        else lo = mid + 1;
    }
    e = lo;
    mloc = mt - mtp[e];
}

// AROWS: rows of A staged per stage.  128 in general; 64 for decode-sized
// groups (at most 64 rows per expert), which frees shared memory for more
// weight stages in flight.  The M = 128 MMA then reads rows 64..127 from
// whatever follows the stage (never stored rows: D rows are independent).
//
// QB = 4: the expert weights are MLX affine 4-bit codes (ESExperts.mm:51,56
// gather_qmm, 64-element groups).  The producer streams a stage's codes
// (BN rows x 8 words, tmB / tmC) and its rows' (scale | bias << 16) words
// (a 4-group box, tmS / tmSt) next to the A tile, through the STAGES-deep
// ring; warps 6..13 turn them into the bf16 B tile w = bf16(scale * q + bias)
// -- the rounding of MLX's dequantise and of dequant_active_kernel -- written
// in the 128-byte-swizzled layout a TMA copy would produce into a separate
// kBRing-deep ring of B tiles, then fence.proxy.async and arrive on bfull.
// The MMA thread waits on full (A) and bfull (B) and commits to empty (the A /
// code stage: its codes were consumed before B was complete) and to bempty
// (the B tile), which the dequantising warps wait on before rewriting it.
template <int EPI, int BN, int BN2, int STAGES, int AROWS = 128, int QB = 0>
__global__ void __launch_bounds__(QB ? kThreads + kDqThreads : kThreads, 1)
moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const int32_t *__restrict__ counts, const int32_t *__restrict__ offsets, int E,
                int Kdim, int I, int H, uint16_t *__restrict__ out, int out_ld,
                int32_t *__restrict__ err, const int32_t *__restrict__ g2e,
                const int32_t *__restrict__ gperm, int gk, int a_rows,
                const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmSt) {
    constexpr bool GU = (EPI == EPI_GATEUP || EPI == EPI_GATEUP_G);
    constexpr int A_BYTES = AROWS * kBK * 2, B_BYTES = Smem<BN>::B_BYTES;
    constexpr int Q_BYTES = QB ? BN * kBK * QB / 8 : 0;  // packed codes of a stage
    constexpr int S_BYTES = QB ? BN * 16 : 0;            // 4 (scale, bias) words per row
    constexpr bool STAGE_C = (EPI == EPI_DOWN && AROWS == kBM);  // TMA-store epilogue
    constexpr uint32_t IDESC = idesc_bf16_f32(kBM, BN);
    static_assert(QB == 0 || (QB == 4 && (EPI == EPI_GATEUP || EPI == EPI_DOWN) && AROWS == kBM &&
                              BN <= kDqThreads),
                  "quantised B: 4-bit, tiled A, one dequantising thread per B row");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_align(smem_raw, 1024);
    constexpr int BSTAGES = QB ? kBRing : STAGES;  // B tiles: own ring when dequantised
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * A_BYTES;
    uint8_t *sC = sB + BSTAGES * B_BYTES;  // down: per-epilogue-warp store staging
    uint8_t *sQ = sC + (STAGE_C ? kStageC : 0);
    uint8_t *sS = sQ + STAGES * Q_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(sS + STAGES * S_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *bfull = tempty + 2;          // QB: B tile dequantised
    uint64_t *bempty = bfull + kBRing;     // QB: B tile read by the MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bempty + (QB ? kBRing : 0));
    int *mtp = reinterpret_cast<int *>(tmem_slot + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 128);
        }
        if (QB)
            for (int b = 0; b < kBRing; ++b) {
                mbar_init(&bfull[b], kDqThreads);
                mbar_init(&bempty[b], 1);
            }
        fence_barrier_init();
        tma_prefetch(&tmA);
        tma_prefetch(&tmB);
        if (QB) tma_prefetch(&tmS);
    }
    pdl_wait();  // dispatch / gather / gate_up output this kernel reads is complete
    // EPI_F32 (router scores) has one group of gk = T rows at offset 0 and no
    // count arrays
    auto grp_cnt = [&](int e) { return EPI == EPI_F32 ? gk : counts[e]; };
    auto grp_off = [&](int e) { return EPI == EPI_F32 ? 0 : offsets[e]; };
    if (warp == 0 && lane == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            mtp[e] = acc;
            acc += (grp_cnt(e) + kBM - 1) / kBM;
        }
        mtp[E] = acc;
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    fence_proxy_async();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();
    // EPI_F32 (router scores): one "expert", N = H outputs, K = I; the B
    // operand is the folded two-term weights [H, 2*I], and the n-tiles run
    // over (term, column block): term 0 multiplies the token rows by the
    // first I-wide half of B, term 1 by the second, each into its own score
    // plane, so that twice as many CTAs share the T / 128 m-tiles.
    const int NCB = H / BN;  // column blocks (EPI_F32)
    const int NT = GU ? (I + BN2 - 1) / BN2 : EPI == EPI_F32 ? 2 * NCB : H / BN;
    const int tiles = mtp[E] * NT;
    const int KB = Kdim / kBK;
    // gate_up: the last n-tile covers TW = I - (NT-1)*BN2 columns; when that is
    // less than BN2 it runs as a narrower tile (N = 2*TW MMAs, B rows through
    // the TW-row tensor map tmC) instead of computing padding
    const int TW = GU ? I - (NT - 1) * BN2 : BN2;

    if (EPI == EPI_GATEUP_G && warp == 0) {
        // all 32 lanes: lane l gathers tile rows 4l..4l+3 of every A stage
        int g = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            int e, mloc, nt;
            decode_tile(t, NT, mtp, E, e, mloc, nt);
            const int row0 = offsets[e] + mloc * kBM;
            const int nvalid = counts[e] - mloc * kBM;
            // rows past the group's end read the group's first token (never stored)
            const int first = gperm[row0] / gk;
            int tok[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int rr = lane * 4 + j;
                tok[j] = rr < nvalid ? gperm[row0 + rr] / gk : first;
            }
            const int ew = g2e ? g2e[e] : e;
            const int gate_row = ew * 2 * I + nt * BN2;
            const bool tail = nt == NT - 1 && TW < BN2;
            const int wrows = tail ? TW : BN2;
            const CUtensorMap *mb = tail ? &tmC : &tmB;
            // only the 4-row groups holding valid rows are fetched; the rest of
            // the A stage keeps stale data, which only feeds accumulator rows
            // that are never stored (rows of D are independent)
            const int nact = min(AROWS / 4, (nvalid + 3) >> 2);
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int s = g % STAGES;
                const uint32_t ph = (g / STAGES) & 1;
                int ok = 1;
                if (lane == 0) ok = mbar_wait(&empty[s], ph ^ 1, kWaitLimit);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) record_error(err, 1, t);
                    goto done;
                }
                if (lane == 0) mbar_arrive_expect_tx(&full[s], nact * 512 + 2 * wrows * kBK * 2);
                __syncwarp();
                if (lane < nact)
                    tma_gather4(sA + s * A_BYTES + lane * 512, &tmA, &full[s], kb * kBK, tok[0],
                            tok[1], tok[2], tok[3]);
                if (lane == 0) {
                    tma_load_2d(sB + s * B_BYTES, mb, &full[s], kb * kBK, gate_row);
                    tma_load_2d(sB + s * B_BYTES + wrows * kBK * 2, mb, &full[s], kb * kBK,
                                gate_row + I);
                }
            }
        }
    } else if (warp == 0) {
        if (lane == 0) {
            int g = 0;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
                int e, mloc, nt;
                decode_tile(t, NT, mtp, E, e, mloc, nt);
                const int row0 = grp_off(e) + mloc * kBM;
                const bool tail = GU && nt == NT - 1 && TW < BN2;
                const int wrows = tail ? TW : BN2;
                const CUtensorMap *mb = tail ? &tmC : &tmB;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, kWaitLimit)) {
                        record_error(err, 1, t);
                        goto done;
                    }
                    // a_rows: A box height (decode-sized groups stage fewer rows;
                    // the rest of the stage is never stored)
                    const int brows = GU ? 2 * wrows : BN;
                    mbar_arrive_expect_tx(&full[s], a_rows * kBK * 2 +
                                                        (QB ? brows * (kBK * QB / 8 + 16)
                                                            : GU ? 2 * wrows * kBK * 2 : B_BYTES));
                    tma_load_2d(sA + s * A_BYTES, &tmA, &full[s], kb * kBK, row0);
                    if constexpr (QB != 0) {
                        // codes: kBK * QB / 32 words of each B row; (scale, bias):
                        // the 4-word (16-byte) box holding group kb
                        const int ew = g2e ? g2e[e] : e;
                        const int cx = kb * (kBK * QB / 32), sx = kb & ~3;
                        if (GU) {
                            const int gate_row = ew * 2 * I + nt * BN2;
                            const CUtensorMap *ms = tail ? &tmSt : &tmS;
                            tma_load_2d(sQ + s * Q_BYTES, mb, &full[s], cx, gate_row);
                            tma_load_2d(sQ + s * Q_BYTES + wrows * (kBK * QB / 8), mb, &full[s],
                                        cx, gate_row + I);
                            tma_load_2d(sS + s * S_BYTES, ms, &full[s], sx, gate_row);
                            tma_load_2d(sS + s * S_BYTES + wrows * 16, ms, &full[s], sx,
                                        gate_row + I);
                        } else {
                            tma_load_2d(sQ + s * Q_BYTES, &tmB, &full[s], cx, ew * H + nt * BN);
                            tma_load_2d(sS + s * S_BYTES, &tmS, &full[s], sx, ew * H + nt * BN);
                        }
                    } else if (EPI == EPI_GATEUP) {
                        // g2e: row group -> expert (grouped entry point); else identity
                        const int ew = g2e ? g2e[e] : e;
                        const int gate_row = ew * 2 * I + nt * BN2;
                        tma_load_2d(sB + s * B_BYTES, mb, &full[s], kb * kBK, gate_row);
                        tma_load_2d(sB + s * B_BYTES + wrows * kBK * 2, mb, &full[s], kb * kBK,
                                    gate_row + I);
                    } else if (EPI == EPI_F32) {
                        tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], kb * kBK + (nt / NCB) * I,
                                    (nt % NCB) * BN);
                    } else {
                        const int ew = g2e ? g2e[e] : e;
                        tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], kb * kBK, ew * H + nt * BN);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int g = 0, i = 0;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
                const int buf = i & 1;
                const uint32_t use = i >> 1;
                if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, kWaitLimit)) {
                    record_error(err, 2, t);
                    goto done;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + buf * kAccStride;
                const bool tail = GU && t % NT == NT - 1 && TW < BN2;
                // a gate_up m-tile with at most 64 rows (an expert group's
                // last, or a decode-sized group) runs M = 64 MMAs: half the
                // tensor work (down tiles keep M = 128 and their TMA-store
                // epilogue, which matters more for their short K loop)
                int e_, mloc_, nt_;
                decode_tile(t, NT, mtp, E, e_, mloc_, nt_);
                const int mrows = (GU && grp_cnt(e_) - mloc_ * kBM <= 64) ? 64 : kBM;
                const uint32_t idesc = tail ? idesc_bf16_f32(mrows, 2 * TW)
                                            : (mrows == kBM ? IDESC : idesc_bf16_f32(64, BN));
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % STAGES;
                    const uint32_t ph = (g / STAGES) & 1;
                    const int bs = QB ? g % kBRing : s;
                    if (!mbar_wait(&full[s], ph, kWaitLimit) ||
                        (QB && !mbar_wait(&bfull[bs], (g / kBRing) & 1, kWaitLimit))) {
                        record_error(err, 3, t);
                        goto done;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + bs * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_bf16(d, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                                 idesc, (kb | kk) != 0);
                    mma_commit(&empty[s]);  // frees the stage once these MMAs finish
                    if (QB) mma_commit(&bempty[bs]);
                }
                mma_commit(&tfull[buf]);    // accumulator ready for the epilogue
            }
        }
    } else if (QB && warp >= kThreads / 32) {
        // dequantising warps: thread r owns B row r of every stage
        const int r = threadIdx.x - kThreads;
        int g = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const int nt = t % NT;
            const bool tail = GU && nt == NT - 1 && TW < BN2;
            const int brows = GU ? 2 * (tail ? TW : BN2) : BN;
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int s = g % STAGES;
                const uint32_t ph = (g / STAGES) & 1;
                const int bs = g % kBRing;
                if (!mbar_wait(&full[s], ph, kWaitLimit) ||
                    !mbar_wait(&bempty[bs], ((g / kBRing) & 1) ^ 1, kWaitLimit)) {
                    record_error(err, 5, t);
                    goto done;
                }
                if (r < brows) {
                    // the two 16-byte halves of the row in an order that
                    // spreads a warp's loads over all banks
                    const uint32_t qr = smem_u32(sQ + s * Q_BYTES + r * 32);
                    const int h0 = (r >> 2) & 1;
                    const uint4 qa = lds128(qr + 16 * h0), qb = lds128(qr + 16 * (h0 ^ 1));
                    const uint4 q0 = h0 ? qb : qa, q1 = h0 ? qa : qb;
                    const uint32_t sbw = lds32(smem_u32(sS + s * S_BYTES + r * 16 + (kb & 3) * 4));
                    const float2 sc2 = make_float2(bf_lo(sbw), bf_lo(sbw));
                    const float2 bi2 = make_float2(bf_hi(sbw), bf_hi(sbw));
                    const float2 m23 = make_float2(-8388608.f, -8388608.f);
                    const uint32_t wds[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                    const uint32_t dst = smem_u32(sB + bs * B_BYTES + r * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        // 16-byte chunk c = elements 8c..8c+7 = code word c:
                        // element 2i is byte i of the low nibbles, 2i+1 of the
                        // high ones; a byte permute puts each under the
                        // exponent of 2^23 (exactly 2^23 + q as an f32)
                        const uint32_t lo = wds[c] & 0x0F0F0F0Fu, hi = (wds[c] >> 4) & 0x0F0F0F0Fu;
                        uint32_t o[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            // packed f32x2 arithmetic: (2^23 + q) - 2^23 = q
                            // exactly, then fma(scale, q, bias) per lane
                            const uint32_t sel = (uint32_t)i | 0x7440u;
                            const float2 q = __fadd2_rn(
                                make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, sel)),
                                            __uint_as_float(__byte_perm(hi, 0x4B000000u, sel))),
                                m23);
                            const float2 f = __ffma2_rn(sc2, q, bi2);
                            o[i] = pack_bf2(f.x, f.y);
                        }
                        sts128(dst + ((c ^ (r & 7)) << 4), o[0], o[1], o[2], o[3]);
                    }
                }
                fence_proxy_async();  // generic-proxy stores -> the tensor core's reads
                mbar_arrive(&bfull[bs]);
            }
        }
    } else {
        const int q = warp & 3;             // TMEM lane quarter this warp may read
        int i = 0, bufsel = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            int e, mloc, nt;
            decode_tile(t, NT, mtp, E, e, mloc, nt);
            const int nvalid = grp_cnt(e) - mloc * kBM;
            // accumulator row of this thread: lane q*32 + lane holds row
            // q*32 + lane of an M = 128 tile, and row q*16 + lane (lanes < 16)
            // of an M = 64 tile
            const bool m64 = GU && nvalid <= 64;
            const int r = m64 ? q * 16 + lane : q * 32 + lane;
            const bool rvalid = r < nvalid && (!m64 || lane < 16);
            const int row = grp_off(e) + mloc * kBM + r;
            const int buf = i & 1;
            const uint32_t use = i >> 1;
            if (!mbar_wait(&tfull[buf], use & 1, kWaitLimit)) {
                record_error(err, 4, t);
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem_base + buf * kAccStride + ((uint32_t)(q * 32) << 16);
            if constexpr (GU) {
                // a narrow last tile holds g in columns [0, TW), u in [TW, 2*TW)
                const int w = min(BN2, I - nt * BN2);
                epilogue_geglu(taddr, w, w, rvalid, out + (size_t)row * out_ld + nt * BN2);
            } else if constexpr (EPI == EPI_F32) {
                // plane nt / NCB of [2][gk = T][out_ld]
                float *dst = reinterpret_cast<float *>(out) + (size_t)(nt / NCB) * gk * out_ld +
                             (size_t)row * out_ld + (nt % NCB) * BN;
#pragma unroll 1
                for (int c = 0; c < BN / 8; ++c) {
                    uint32_t a[8];
                    tmem_ld8(taddr + c * 8, a);
                    tmem_ld_wait();
                    if (r < nvalid) {
                        float4 *d4 = reinterpret_cast<float4 *>(dst + c * 8);
                        d4[0] = make_float4(__uint_as_float(a[0]), __uint_as_float(a[1]),
                                            __uint_as_float(a[2]), __uint_as_float(a[3]));
                        d4[1] = make_float4(__uint_as_float(a[4]), __uint_as_float(a[5]),
                                            __uint_as_float(a[6]), __uint_as_float(a[7]));
                    }
                }
            } else if (STAGE_C && !m64 && q * 32 + 32 <= nvalid) {
                epilogue_bf16_tma<BN>(taddr, sC + q * 8192, bufsel, &tmC, nt * BN, row - lane,
                                      lane);
            } else if ((m64 ? q * 16 : q * 32) < nvalid) {
                epilogue_bf16<BN>(taddr, rvalid, out + (size_t)row * out_ld + nt * BN);
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
        }
        if (STAGE_C && lane == 0) bulk_wait<0>();  // stores complete before exit
    }
done:
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------- host side

// 2-D bf16 row-major [rows, inner] tensor, box {64, box_rows}, 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
    return bf16_map_2d(m, base, inner, rows, kBK, box_rows, true);
}

template <int EPI, int BN, int BN2, int STAGES, int AROWS = 128, int QB = 0>
constexpr size_t smem_bytes() {
    return 1024 +
           (size_t)STAGES * (AROWS * kBK * 2 + (QB ? BN * kBK * QB / 8 + BN * 16
                                                   : Smem<BN>::B_BYTES)) +
           (QB ? (size_t)kBRing * Smem<BN>::B_BYTES : 0) +
           ((EPI == EPI_DOWN && AROWS == kBM) ? kStageC : 0) +
           8 * (2 * STAGES + 4 + (QB ? 2 * kBRing : 0)) + 16 + 4 * (kMaxExperts + 1);
}

template <int EPI, int BN, int BN2, int STAGES, int AROWS = 128, int QB = 0>
cudaError_t set_attr() {
    static_assert(smem_bytes<EPI, BN, BN2, STAGES, AROWS, QB>() <= 232448, "shared memory");
    return cudaFuncSetAttribute(moe_gemm_kernel<EPI, BN, BN2, STAGES, AROWS, QB>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem_bytes<EPI, BN, BN2, STAGES, AROWS, QB>());
}

// sq / sqt (QB only): the (scale, bias) word maps of the full and the narrow
// last gate_up tile.
template <int EPI, int BN, int BN2, int STAGES, int AROWS = 128, int QB = 0>
cudaError_t launch(const CUtensorMap &a, const CUtensorMap &b, const Dispatch &d, int E, int Kdim,
                   int I, int H, uint16_t *out, int out_ld, int32_t *err, cudaStream_t s,
                   const int32_t *g2e = nullptr, const CUtensorMap *c = nullptr,
                   const int32_t *gperm = nullptr, int gk = 1, int a_rows = kBM,
                   const CUtensorMap *sq = nullptr, const CUtensorMap *sqt = nullptr) {
    const int sms = grid_sms(current_device());
    return launch_ex(moe_gemm_kernel<EPI, BN, BN2, STAGES, AROWS, QB>, dim3(sms),
                     dim3(QB ? kThreads + kDqThreads : kThreads),
                     smem_bytes<EPI, BN, BN2, STAGES, AROWS, QB>(), s, true, a, b, c ? *c : a,
                     d.counts, d.offsets, E, Kdim, I, H, out, out_ld, err, g2e, gperm, gk, a_rows,
                     sq ? *sq : a, sqt ? *sqt : (sq ? *sq : a));
}

// gate_up tile: BN2 gate + BN2 up rows; down tile: BN rows of W_down.
constexpr int kGuStages = 5, kDnStages = 4, kRtStages = 6;
// QB: A + codes + (scale, bias) stages of 28 KB, plus kBRing 32 KB B tiles
constexpr int kQ4GuStages = 4, kQ4DnStages = 3;

}  // namespace

cudaError_t gemm_init() {
    cudaError_t e;
    if ((e = set_attr<EPI_F32, 64, 0, kRtStages>())) return e;
    if ((e = set_attr<EPI_F32, 128, 0, kRtStages>())) return e;
    if ((e = set_attr<EPI_GATEUP, 176, 88, kGuStages>())) return e;
    if ((e = set_attr<EPI_GATEUP, 256, 128, kDnStages>())) return e;
    if ((e = set_attr<EPI_GATEUP, 128, 64, kGuStages>())) return e;
    if ((e = set_attr<EPI_GATEUP_G, 176, 88, kGuStages>())) return e;
    if ((e = set_attr<EPI_GATEUP_G, 176, 88, 7, 64>())) return e;
    if ((e = set_attr<EPI_DOWN, 256, 0, 5, 64>())) return e;
    if ((e = set_attr<EPI_GATEUP_G, 256, 128, kDnStages>())) return e;
    if ((e = set_attr<EPI_GATEUP_G, 128, 64, kGuStages>())) return e;
    if ((e = set_attr<EPI_DOWN, 256, 0, kDnStages>())) return e;
    if ((e = set_attr<EPI_GATEUP, 256, 128, kQ4GuStages, kBM, 4>())) return e;
    if ((e = set_attr<EPI_DOWN, 256, 0, kQ4DnStages, kBM, 4>())) return e;
    return set_attr<EPI_DOWN, 128, 0, kDnStages>();
}

bool gemm_supported(int H, int I) {
    return encode_tiled_fn() != nullptr && H % 128 == 0 && (I % 88 == 0 || I % 64 == 0) && I % 64 == 0;
}

// Tensor map of the narrow last gate_up tile (TW = I mod bn2 rows per box);
// a copy of the main B map when I is a multiple of bn2 (never read then).
bool tail_map(CUtensorMap *c, const CUtensorMap &b, const uint16_t *gu, int H, int I, int E_w,
              int bn2) {
    const int tw = I % bn2;
    if (!tw) {
        *c = b;
        return true;
    }
    return bf16_map_2d(c, gu, H, (uint64_t)E_w * 2 * I, kBK, tw, true);
}

cudaError_t launch_gemm_gateup(const uint16_t *xp, const Dispatch &d, const ExpertWeights &w,
                               int rows_cap, int H, int I, int E, uint16_t *yp, int32_t *err,
                               cudaStream_t s, int *launches) {
    if (E > kMaxExperts) return cudaErrorInvalidValue;
    // Prefill (many rows per expert, tensor-bound): 128 gate + 128 up columns
    // per tile, fewer staged bytes per flop; the last tile of I=704 is half
    // used.  Decode-sized calls are HBM-bound, so they use exact 88+88 tiles
    // that read no padding.  APT_GATEUP_BN2 (88 / 128) overrides.
    static const int pref = [] {
        const char *v = getenv("APT_GATEUP_BN2");
        return v ? atoi(v) : 0;
    }();
    const int want = pref ? pref : (rows_cap > 4096 ? 128 : 88);
    const int bn2 = (want == 88 && I % 88 == 0) ? 88 : (I >= 128 ? 128 : 64);
    CUtensorMap a, b;
    CUtensorMap c;
    if (!make_map(&a, xp, H, rows_cap, kBM) || !make_map(&b, w.gu, H, (uint64_t)E * 2 * I, bn2) ||
        !tail_map(&c, b, w.gu, H, I, E, bn2))
        return cudaErrorInvalidValue;
    cudaError_t e = (bn2 == 88)
        ? launch<EPI_GATEUP, 176, 88, kGuStages>(a, b, d, E, H, I, H, yp, I, err, s, nullptr, &c)
        : (bn2 == 128)
        ? launch<EPI_GATEUP, 256, 128, kDnStages>(a, b, d, E, H, I, H, yp, I, err, s, nullptr, &c)
        : launch<EPI_GATEUP, 128, 64, kGuStages>(a, b, d, E, H, I, H, yp, I, err, s, nullptr, &c);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemm_gateup_gather(const uint16_t *x, int T, int Kp, const Dispatch &d,
                                      const ExpertWeights &w, int rows_cap, int H, int I, int E,
                                      uint16_t *yp, int32_t *err, cudaStream_t s, int *launches) {
    if (E > kMaxExperts || T <= 0) return cudaErrorInvalidValue;
    static const int pref = [] {
        const char *v = getenv("APT_GATEUP_BN2");
        return v ? atoi(v) : 0;
    }();
    const int want = pref ? pref : (rows_cap > 4096 ? 128 : 88);
    const int bn2 = (want == 88 && I % 88 == 0) ? 88 : (I >= 128 ? 128 : 64);
    CUtensorMap a, b;
    // token rows [T, H], one-row boxes: each tile::gather4 copy fetches 4 rows
    CUtensorMap c;
    if (!bf16_map_2d(&a, x, H, T, kBK, 1, true) ||
        !make_map(&b, w.gu, H, (uint64_t)E * 2 * I, bn2) || !tail_map(&c, b, w.gu, H, I, E, bn2))
        return cudaErrorInvalidValue;
    const int32_t *perm = d.perm;
    cudaError_t e = (bn2 == 88)
        ? (T <= 64  // at most 64 rows per expert: 64-row A stages, 7 weight stages
               ? launch<EPI_GATEUP_G, 176, 88, 7, 64>(a, b, d, E, H, I, H, yp, I, err, s,
                                                      nullptr, &c, perm, Kp)
               : launch<EPI_GATEUP_G, 176, 88, kGuStages>(a, b, d, E, H, I, H, yp, I, err, s,
                                                         nullptr, &c, perm, Kp))
        : (bn2 == 128)
        ? launch<EPI_GATEUP_G, 256, 128, kDnStages>(a, b, d, E, H, I, H, yp, I, err, s, nullptr,
                                                   &c, perm, Kp)
        : launch<EPI_GATEUP_G, 128, 64, kGuStages>(a, b, d, E, H, I, H, yp, I, err, s, nullptr,
                                                  &c, perm, Kp);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemm_gateup_grouped(const uint16_t *rows, const Dispatch &d,
                                       const int32_t *g2e, const ExpertWeights &w, int rows_cap,
                                       int H, int I, int E_w, int G, uint16_t *yp, int32_t *err,
                                       cudaStream_t s, int *launches) {
    if (G > kMaxExperts) return cudaErrorInvalidValue;
    const int bn2 = (rows_cap > 4096 || I % 88) ? (I >= 128 ? 128 : 64) : 88;
    CUtensorMap a, b;
    CUtensorMap c;
    if (!make_map(&a, rows, H, rows_cap, kBM) ||
        !make_map(&b, w.gu, H, (uint64_t)E_w * 2 * I, bn2) || !tail_map(&c, b, w.gu, H, I, E_w, bn2))
        return cudaErrorInvalidValue;
    cudaError_t e = (bn2 == 88)
        ? launch<EPI_GATEUP, 176, 88, kGuStages>(a, b, d, G, H, I, H, yp, I, err, s, g2e, &c)
        : (bn2 == 128)
        ? launch<EPI_GATEUP, 256, 128, kDnStages>(a, b, d, G, H, I, H, yp, I, err, s, g2e, &c)
        : launch<EPI_GATEUP, 128, 64, kGuStages>(a, b, d, G, H, I, H, yp, I, err, s, g2e, &c);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemm_down_grouped(const uint16_t *yp, const Dispatch &d, const int32_t *g2e,
                                     const ExpertWeights &w, int rows_cap, int H, int I, int E_w,
                                     int G, uint16_t *out, int32_t *err, cudaStream_t s,
                                     int *launches) {
    if (G > kMaxExperts) return cudaErrorInvalidValue;
    const int bn = (H % 256 == 0) ? 256 : 128;
    CUtensorMap a, b, c;
    if (!make_map(&a, yp, I, rows_cap, kBM) || !make_map(&b, w.dn, I, (uint64_t)E_w * H, bn) ||
        !bf16_map_2d(&c, out, H, rows_cap, 64, 32, true))
        return cudaErrorInvalidValue;
    cudaError_t e = (bn == 256)
        ? launch<EPI_DOWN, 256, 0, kDnStages>(a, b, d, G, I, I, H, out, H, err, s, g2e, &c)
        : launch<EPI_DOWN, 128, 0, kDnStages>(a, b, d, G, I, I, H, out, H, err, s, g2e, &c);
    if (launches) ++*launches;
    return e;
}

// 4-bit MLX affine experts (64-element groups) on the tensor cores: the
// gate_up / down GEMMs with the B tiles dequantised in shared memory from the
// packed codes and the interleaved (scale, bias) words (QB = 4 above); no
// bf16 copy of the weights is made.
bool gemm_q4_supported(int H, int I) {
    return gemm_supported(H, I) && H % 256 == 0 && I % 64 == 0 && I >= 128;
}

cudaError_t launch_gemm_gateup_q4(const uint16_t *xp, const Dispatch &d, const ExpertWeights &w,
                                  int rows_cap, int H, int I, int E, uint16_t *yp, int32_t *err,
                                  cudaStream_t s, int *launches) {
    if (E > kMaxExperts || w.bits != 4 || !w.gu_q || !w.gu_sb) return cudaErrorInvalidValue;
    const int bn2 = 128, tw = I % bn2 ? I % bn2 : bn2;
    const uint64_t rows = (uint64_t)E * 2 * I;
    CUtensorMap a, b, c, sq, sqt;
    if (!make_map(&a, xp, H, rows_cap, kBM) ||
        !map_2d(&b, w.gu_q, H / 8, rows, 8, bn2, false, true) ||
        !map_2d(&c, w.gu_q, H / 8, rows, 8, tw, false, true) ||
        !map_2d(&sq, w.gu_sb, sb_row_words(H), rows, 4, bn2, false, true) ||
        !map_2d(&sqt, w.gu_sb, sb_row_words(H), rows, 4, tw, false, true))
        return cudaErrorInvalidValue;
    cudaError_t e = launch<EPI_GATEUP, 256, 128, kQ4GuStages, kBM, 4>(
        a, b, d, E, H, I, H, yp, I, err, s, nullptr, &c, nullptr, 1, kBM, &sq, &sqt);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemm_down_q4(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                                int rows_cap, int H, int I, int E, uint16_t *op, int32_t *err,
                                cudaStream_t s, int *launches) {
    if (E > kMaxExperts || w.bits != 4 || !w.dn_q || !w.dn_sb) return cudaErrorInvalidValue;
    const uint64_t rows = (uint64_t)E * H;
    CUtensorMap a, b, c, sq;
    if (!make_map(&a, yp, I, rows_cap, kBM) ||
        !map_2d(&b, w.dn_q, I / 8, rows, 8, 256, false, true) ||
        !map_2d(&sq, w.dn_sb, sb_row_words(I), rows, 4, 256, false, true) ||
        !bf16_map_2d(&c, op, H, rows_cap, 64, 32, true))
        return cudaErrorInvalidValue;
    cudaError_t e = launch<EPI_DOWN, 256, 0, kQ4DnStages, kBM, 4>(
        a, b, d, E, I, I, H, op, H, err, s, nullptr, &c, nullptr, 1, kBM, &sq, nullptr);
    if (launches) ++*launches;
    return e;
}

cudaError_t launch_gemm_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                             int rows_cap, int H, int I, int E, uint16_t *op, int32_t *err,
                             cudaStream_t s, int *launches, int max_group_rows) {
    if (E > kMaxExperts) return cudaErrorInvalidValue;
    // Decode-sized groups (a few rows per expert): A boxes only as tall as the
    // largest group (rounded to 16); the rest of each A stage is never stored.
    // (128-column tiles were tried for a finer spread and were slower: half
    // the bytes in flight per stage.)
    const bool small = max_group_rows > 0 && max_group_rows <= 64;
    const int a_rows = small ? ((max_group_rows + 15) / 16) * 16 : kBM;
    const int bn = (H % 256 == 0) ? 256 : 128;
    CUtensorMap a, b, c;
    if (!make_map(&a, yp, I, rows_cap, a_rows) || !make_map(&b, w.dn, I, (uint64_t)E * H, bn) ||
        !bf16_map_2d(&c, op, H, rows_cap, 64, 32, true))
        return cudaErrorInvalidValue;
    cudaError_t e = (bn == 256)
        ? (small  // 64-row A stages, 5 weight stages, plain-store epilogue
               ? launch<EPI_DOWN, 256, 0, 5, 64>(a, b, d, E, I, I, H, op, H, err, s, nullptr, &c,
                                                 nullptr, 1, a_rows)
               : launch<EPI_DOWN, 256, 0, kDnStages>(a, b, d, E, I, I, H, op, H, err, s, nullptr,
                                                     &c, nullptr, 1, a_rows))
        : launch<EPI_DOWN, 128, 0, kDnStages>(a, b, d, E, I, I, H, op, H, err, s, nullptr, &c,
                                              nullptr, 1, a_rows);
    if (launches) ++*launches;
    return e;
}

}  // namespace apt

namespace apt {

// Router scores on the tensor cores, before the per-token RMS factor, as two
// planes scores[term] [T,E] f32 = x [T, H] . w_term^T, where (w1 | w2)
// [E, 2H] is the two-term bf16 split of (scale * H^-1/2) * proj folded at
// load; x is bf16, the products are exact and accumulate in f32, so
// plane 0 + plane 1 matches the f32 dot product to ~2^-17 relative per term.
cudaError_t launch_gemm_router(const uint16_t *x, const uint16_t *projw, int T, int H, int E,
                               float *scores, int32_t *err, cudaStream_t s, int *launches) {
    const int bn = E % 128 == 0 ? 128 : 64;
    CUtensorMap a, b;
    if (!make_map(&a, x, H, T, kBM) || !make_map(&b, projw, 2 * (uint64_t)H, E, bn))
        return cudaErrorInvalidValue;
    Dispatch d{};
    float *o = scores;
    cudaError_t e =
        bn == 128 ? launch<EPI_F32, 128, 0, kRtStages>(a, b, d, 1, H, H, E,
                                                       reinterpret_cast<uint16_t *>(o), E, err, s,
                                                       nullptr, nullptr, nullptr, T)
                  : launch<EPI_F32, 64, 0, kRtStages>(a, b, d, 1, H, H, E,
                                                      reinterpret_cast<uint16_t *>(o), E, err, s,
                                                      nullptr, nullptr, nullptr, T);
    if (launches) ++*launches;
    return e;
}

}  // namespace apt
