// decode_fused.cu -- the whole MoE block for decode-sized calls (T <= 8, bf16
// experts) as ONE persistent kernel: ESRouter::routeTopK
// (aptransformer/ESRouter.mm:14-32), ESExperts::sparseForward's gate_up /
// GeGLU / down (ESExperts.mm:44-57) and the weighted k-order combine
// (ESExperts.mm:58-59), with the reference's rounding points.
//
// Why one kernel: at T = 1 the block moves ~96 MB of expert weights, 15 us of
// HBM time, but as a chain of launches (router -> gate_up -> down ->
// combine) every hand-over drains the weight stream and the GEMVs run only
// 2-3 work items per SM.  Here one CTA per SM does:
//   1. router: CTA e computes expert e's scores for all T tokens (its proj
//      row, the token rows, scale and per_expert_scale arrive by bulk
//      copies), stores them and adds one to a count (release); every CTA
//      waits for the count to reach E (acquire), reads the T x E scores and
//      runs softmax, top-K and the dispatch itself in shared
//      memory (same inputs, same arithmetic, same result in every CTA); CTA 0
//      writes idx, w and the dispatch out for the caller.
//   2. experts: equal-size work items, 32 gate_up rows x H (16 intermediate
//      columns) or 128 down rows x I, both 11 x 16 KB weight stages; every
//      gate_up item precedes every down item in the global order, and CTAs
//      claim items from an atomic counter (a down item only ever waits on
//      items already claimed by running CTAs).  A producer warp streams each
//      claimed item's weights through a TMA ring without waiting on anything
//      but ring slots, so a down item's weights are in flight while its
//      expert's gate_up items finish elsewhere; eight compute warps do the
//      dot products (f32).  Hand-overs between CTAs carry no flags: GeGLU
//      and down rows are stored as 64-bit words tagged with the call's count
//      (two bf16 values + the count), and a reader polls the words
//      themselves, so readiness and value arrive in one load.  A stager warp
//      loads a down item's GeGLU rows this way into a double buffer.
//   3. combine: the down item (u, hb) of each token's last expert in claim
//      order -- whose other experts' down items were all claimed before it
//      -- has its signal warp read the token's K tagged down rows of row
//      block hb, sum bf16(w * row) in k order (f32) and store the slice,
//      rounded once.
// The two counters (next work item, scores published) come in two sets used
// by calls of even and odd count; each call zeroes the set the previous call
// used, so the kernel can be replayed (CUDA graphs) without host resets or a
// reset step at its end.  The router hand-over needs the whole grid
// resident: one CTA per SM, grid = SMs.
// Every wait is bounded; on expiry the kernel records an error code in the
// handle's error word and returns (apt_moe_sync reports APT_ERR_TIMEOUT).
#include <cuda.h>

#include "common.cuh"
#include "launch_util.h"
#include "moe_internal.h"
#include "router_select.cuh"
#include "sm100_ptx.cuh"

namespace apt {

namespace {

using namespace sm100;

constexpr int kCW = 8;                 // compute warps
constexpr int kProdWarp = kCW;         // TMA producer warp
constexpr int kStagerWarp = kCW + 1;   // GeGLU-row stager warp
constexpr int kSignalWarp = kCW + 2;   // completion counts and the combine
constexpr int kThreads = (kCW + 3) * 32;
constexpr int kStageBytes = 16384;
// ring depth by the call's largest per-expert token count: the smaller the
// staged token rows, the more 16 KB weight stages fit (bytes in flight per SM)
// Quantised experts (BITS = 4 or 8, MLX affine, 64-element groups): the same
// items, with packed codes streamed in stages of 32 gate_up rows x 256 or 128
// down rows x 64 columns (1 KB x BITS either way), and each item's (scale,
// bias) pairs in a ring of kSB slots.
template <int BITS>
constexpr int stage_bytes() { return BITS ? 1024 * BITS : kStageBytes; }
// ring stages (4-bit: the most whole-item slots; their number depends on H, I)
template <int NTMAX, int BITS = 0>
constexpr int stages_for() {
    return BITS == 0 ? (NTMAX <= 2 ? 12 : NTMAX <= 4 ? 10 : 8)
           : BITS == 4 ? 4
                       : (NTMAX <= 4 ? 144 * 1024 : 112 * 1024) / stage_bytes<BITS>();
}
template <int NTMAX, int BITS>
constexpr int ring_bytes() {
    return BITS == 4 ? (NTMAX <= 4 ? 150 : 100) * 1024 : stages_for<NTMAX, BITS>() * stage_bytes<BITS>();
}
// 4-bit experts run their multiplies on mma.sync (codes become bf16 128 + q,
// exact; tokens are the n = 8 dimension).  Extra shared memory: the gate_up
// partial sums of the eight compute warps [8][32 rows][8 tokens], per-token
// sums of x over 32-column blocks [T][H/32], and per-token sums of the staged
// GeGLU rows over 64-element groups [2][NTMAX][I/64].
constexpr int kRedFloats = kCW * 32 * 8;
constexpr int kSB = 4;  // (scale, bias) slots: items in flight between the producer and the rest
// words of one (scale, bias) slot: 32 gate_up rows x gp(H) or 128 down rows x gp(I)
__host__ __device__ inline int sb_slot_words(int H, int I) {
    const int gu = 32 * (((H / 64) + 3) / 4 * 4), dn = 128 * (((I / 64) + 3) / 4 * 4);
    return ((gu > dn ? gu : dn) + 31) / 32 * 32;
}
constexpr int kMaxT = 8;
constexpr int kMaxPairs = 64;          // T * K
constexpr int kGuCols = 16;            // intermediate columns per gate_up item
constexpr int kDnRows = 128;           // hidden rows per down item
constexpr int kQ = 8;                  // claimed-item queue between the producer and the rest
constexpr long long kWait = 4000000000LL;
constexpr int kMaxGrid = 256;          // per-CTA call counters in the sync words
// dynamic shared memory cap: 227 KB per CTA less the kernel's static arrays
constexpr int kMaxDynSmem = 214 * 1024;

// Phase timestamps (%globaltimer, one thread per CTA) for tuning builds
// compiled with -DAPT_FUSED_TRACE; absent from the library build.
#ifdef APT_FUSED_TRACE
__device__ unsigned long long g_ftrace[1024][16];
__device__ unsigned long long g_itrace[1024][16][8];
#define FT_ITEM(slot, j, v)                                                \
    do {                                                                   \
        unsigned long long t_;                                             \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));             \
        if ((j) < 16) { g_itrace[blockIdx.x][j][slot] = t_; if (slot == 0) g_itrace[blockIdx.x][j][3] = (v); } \
    } while (0)
#define FT_STAMP(i)                                                        \
    do {                                                                   \
        unsigned long long t_;                                             \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));             \
        g_ftrace[blockIdx.x][i] = t_;                                      \
    } while (0)
#else
#define FT_ITEM(slot, j, v) \
    do {                    \
    } while (0)
#define FT_STAMP(i) \
    do {            \
    } while (0)
#endif

// Sync words (int32, zeroed once when the handle is created):
//   [0, kMaxGrid)  per-CTA call count: CTA b increments word b at the start of
//                  every call; all CTAs run in every call, so all agree on it
//   two counter sets, used by calls of even / odd count: [0] next work item,
//                  [1] CTAs whose scores are published; a call zeroes the
//                  other parity's set, which the previous call used, for the
//                  next call (no reset step at the end of a call)
//   tagged rows    from word kTagWord (8-byte aligned), u64 each: the call
//                  count in the high half, two bf16 values in the low half;
//                  GeGLU rows [kMaxPairs][I/2], then down rows [kMaxPairs][H/2].
//                  A reader polls a word until it carries this call's count:
//                  the value and its readiness arrive in one load.
constexpr int kSetWords = 2;
constexpr int kTagWord = kMaxGrid + 2 * kSetWords;

struct FusedArgs {
    const uint16_t *xr, *xe;            // router input, expert input [T, H]
    const uint16_t *scale, *pes, *proj; // router weights
    int T, H, E, K, I;
    float eps, root;
    float *scores;                      // [T, E] scratch
    int32_t *idx;                       // [T, K]
    uint16_t *w;                        // [T, K]
    Dispatch d;
    unsigned long long *yq;             // [kMaxPairs][I/2] GeGLU rows, sorted order, tagged
    unsigned long long *oq;             // [kMaxPairs][H/2] down rows, sorted order, tagged
    uint16_t *out;                      // [T, H]
    int32_t *sync;                      // see the sync-word layout above set_words()
    int32_t *err;
    const uint32_t *gq, *dq, *gsb, *dsb;  // 4-bit: fragment-ordered codes, (scale, bias) rows
};

__device__ __forceinline__ void record_error(int32_t *err, int code, int where) {
    if (atomicCAS(err, 0, code) == 0) err[1] = where;
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_gpu_v2u64(unsigned long long *p, unsigned long long v0,
                                                     unsigned long long v1) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(v0), "l"(v1)
                 : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Load NW tagged words per lane (p[q], q < n) and wait (bounded) until every
// word of the warp carries call count `epoch`: each retry reloads all the
// words not yet current at once, so a retry costs one round trip.
template <int NW>
__device__ __forceinline__ void tagged_load(unsigned long long (&x)[NW],
                                            const unsigned long long *const (&p)[NW], int n,
                                            uint32_t epoch, int32_t *err, int code, int where) {
#pragma unroll
    for (int q = 0; q < NW; ++q) x[q] = q < n ? ld_relaxed_gpu_u64(p[q]) : 0ull;
    const long long t0 = clock64();
    for (;;) {
        bool ok = true;
#pragma unroll
        for (int q = 0; q < NW; ++q) ok &= q >= n || (uint32_t)(x[q] >> 32) == epoch;
        if (__all_sync(0xffffffffu, ok)) return;
        if (clock64() - t0 > kWait) {
            record_error(err, code, where);
            return;
        }
        __nanosleep(64);
#pragma unroll
        for (int q = 0; q < NW; ++q)
            if (q < n && (uint32_t)(x[q] >> 32) != epoch) x[q] = ld_relaxed_gpu_u64(p[q]);
    }
}

__device__ __forceinline__ void red_add_release_gpu(int32_t *p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_cta_shared(const int *p) {
    int v;
    asm volatile("ld.acquire.cta.shared.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}

__device__ __forceinline__ void red_add_release_cta_shared(int *p, int v) {
    asm volatile("red.release.cta.shared.add.s32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ float dot8(const float (&w)[8], const float (&x)[8]) {
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

// gate_up item: 16 intermediate columns = 16 gate + 16 up rows x H; warp w
// owns columns j0+2w, j0+2w+1 (2 gate and 2 up rows), lanes split each
// 256-column stage; tokens read from the staged rows.
template <int NT, int S>
__device__ bool gateup_item(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                            const uint16_t *xs, const int *toks, int nt, const FusedArgs &a,
                            int &g, int w, int lane, unsigned long long *ydst,
                            unsigned long long tag) {
    const int NK = a.H / 256;
    int toff[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) toff[t] = (t < nt ? toks[t] : toks[0]) * a.H + lane * 8;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S;
        if (!mbar_wait(&full[s], (g / S) & 1, kWait)) {
            record_error(a.err, 71, kc);
            return false;
        }
        const uint8_t *st = ring + s * kStageBytes;
        float wf[4][8];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            unpack8(*reinterpret_cast<const uint4 *>(st + (2 * w + q) * 512 + lane * 16), wf[q]);
            unpack8(*reinterpret_cast<const uint4 *>(st + (kGuCols + 2 * w + q) * 512 + lane * 16),
                    wf[2 + q]);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + toff[t] + kc * 256), xf);
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][t] += dot8(wf[r], xf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = warp_sum(acc[r][t]);
    if (lane < nt) {
        const float y0 = geglu_bf16(rbf(pick<NT, 4>(acc, 0, lane)), rbf(pick<NT, 4>(acc, 2, lane)));
        const float y1 = geglu_bf16(rbf(pick<NT, 4>(acc, 1, lane)), rbf(pick<NT, 4>(acc, 3, lane)));
        st_relaxed_gpu_u64(ydst + (size_t)lane * (a.I / 2) + w, tag | pack_bf2(y0, y1));
    }
    return true;
}

// down item: 128 hidden rows; warp w owns rows 16w..16w+15 as 4 groups of 8
// lanes, each lane 4 rows x 8 columns of every 64-column stage.
template <int NT, int S>
__device__ bool down_item(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                          const uint16_t *ys, int nt, const FusedArgs &a, int &g, int w, int lane,
                          unsigned long long *odst, unsigned long long tag) {
    const int NK = a.I / 64;
    const int gq = lane >> 3, c = lane & 7;
    const int rbase = 16 * w + 4 * gq;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S;
        if (!mbar_wait(&full[s], (g / S) & 1, kWait)) {
            record_error(a.err, 72, kc);
            return false;
        }
        const uint8_t *st = ring + s * kStageBytes;
        float wf[4][8];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            unpack8(*reinterpret_cast<const uint4 *>(st + (rbase + r) * 128 + c * 16), wf[r]);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float yf[8];
            unpack8(*reinterpret_cast<const uint4 *>(ys + t * a.I + kc * 64 + c * 8), yf);
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][t] += dot8(wf[r], yf);
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
    if (c < nt)
        st_relaxed_gpu_v2u64(odst + (size_t)c * (a.H / 2) + rbase / 2,
                             tag | pack_bf2(pick<NT, 4>(acc, 0, c), pick<NT, 4>(acc, 1, c)),
                             tag | pack_bf2(pick<NT, 4>(acc, 2, c), pick<NT, 4>(acc, 3, c)));
    return true;
}

template <int NTMAX, int S>
__device__ bool run_gateup(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                           const uint16_t *xs, const int *toks, int nt, const FusedArgs &a,
                           int &g, int w, int lane, unsigned long long *ydst,
                           unsigned long long tag) {
    if (nt == 1) return gateup_item<1, S>(ring, full, empty, xs, toks, nt, a, g, w, lane, ydst, tag);
    if constexpr (NTMAX >= 2)
        if (nt == 2) return gateup_item<2, S>(ring, full, empty, xs, toks, nt, a, g, w, lane, ydst, tag);
    if constexpr (NTMAX >= 4)
        if (nt <= 4) return gateup_item<4, S>(ring, full, empty, xs, toks, nt, a, g, w, lane, ydst, tag);
    if constexpr (NTMAX >= 8)
        return gateup_item<8, S>(ring, full, empty, xs, toks, nt, a, g, w, lane, ydst, tag);
    return false;
}

template <int NTMAX, int S>
__device__ bool run_down(const uint8_t *ring, uint64_t *full, uint64_t *empty, const uint16_t *ys,
                         int nt, const FusedArgs &a, int &g, int w, int lane,
                         unsigned long long *odst, unsigned long long tag) {
    if (nt == 1) return down_item<1, S>(ring, full, empty, ys, nt, a, g, w, lane, odst, tag);
    if constexpr (NTMAX >= 2)
        if (nt == 2) return down_item<2, S>(ring, full, empty, ys, nt, a, g, w, lane, odst, tag);
    if constexpr (NTMAX >= 4)
        if (nt <= 4) return down_item<4, S>(ring, full, empty, ys, nt, a, g, w, lane, odst, tag);
    if constexpr (NTMAX >= 8) return down_item<8, S>(ring, full, empty, ys, nt, a, g, w, lane, odst, tag);
    return false;
}

// Quantised gate_up item: the rows and lanes of gateup_item; a lane's 8
// codes of a row lie in one 64-element group, so its contribution is
// s * sum(q x) + b * sum(x) in f32, with (s, b) from the item's slot `sbs`
// ([32 rows][gp] (scale | bias << 16) words).
template <int NT, int S, int BITS>
__device__ bool gateup_item_q(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                              const uint16_t *xs, const uint32_t *sbs, int gp, const int *toks,
                              int nt, const FusedArgs &a, int &g, int w, int lane,
                              unsigned long long *ydst, unsigned long long tag) {
    constexpr int SBY = stage_bytes<BITS>();
    constexpr int RW = 256 * BITS / 32;  // words per row per stage
    constexpr int LW = BITS / 4;         // words per lane per row
    const int NK = a.H / 256;
    int toff[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) toff[t] = (t < nt ? toks[t] : toks[0]) * a.H + lane * 8;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S;
        if (!mbar_wait(&full[s], (g / S) & 1, kWait)) {
            record_error(a.err, 71, kc);
            return false;
        }
        const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + s * SBY);
        const int grp = kc * 4 + (lane >> 3);
        float qf[4][8], sr[4], br[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int row = (q < 2 ? 0 : kGuCols) + 2 * w + (q & 1);
            uint32_t wd[LW];
#pragma unroll
            for (int k = 0; k < LW; ++k) wd[k] = st[row * RW + lane * LW + k];
            unpack_q8<BITS>(wd, qf[q]);
            const uint32_t pv = sbs[row * gp + grp];
            sr[q] = bf_lo(pv);
            br[q] = bf_hi(pv);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + toff[t] + kc * 256), xf);
            float xsum = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) xsum += xf[i];
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][t] += fmaf(sr[r], dot8(qf[r], xf), br[r] * xsum);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = warp_sum(acc[r][t]);
    if (lane < nt) {
        const float y0 = geglu_bf16(rbf(pick<NT, 4>(acc, 0, lane)), rbf(pick<NT, 4>(acc, 2, lane)));
        const float y1 = geglu_bf16(rbf(pick<NT, 4>(acc, 1, lane)), rbf(pick<NT, 4>(acc, 3, lane)));
        st_relaxed_gpu_u64(ydst + (size_t)lane * (a.I / 2) + w, tag | pack_bf2(y0, y1));
    }
    return true;
}

// Quantised down item: the rows and lanes of down_item; a stage is one
// 64-element group of the 128 rows.
template <int NT, int S, int BITS>
__device__ bool down_item_q(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                            const uint16_t *ys, const uint32_t *sbs, int gp, int nt,
                            const FusedArgs &a, int &g, int w, int lane, unsigned long long *odst,
                            unsigned long long tag) {
    constexpr int SBY = stage_bytes<BITS>();
    constexpr int RW = 64 * BITS / 32;
    constexpr int LW = BITS / 4;
    const int NK = a.I / 64;
    const int gq = lane >> 3, c = lane & 7;
    const int rbase = 16 * w + 4 * gq;
    float acc[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    for (int kc = 0; kc < NK; ++kc, ++g) {
        const int s = g % S;
        if (!mbar_wait(&full[s], (g / S) & 1, kWait)) {
            record_error(a.err, 72, kc);
            return false;
        }
        const uint32_t *st = reinterpret_cast<const uint32_t *>(ring + s * SBY);
        float qf[4][8], sr[4], br[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t wd[LW];
#pragma unroll
            for (int k = 0; k < LW; ++k) wd[k] = st[(rbase + r) * RW + c * LW + k];
            unpack_q8<BITS>(wd, qf[r]);
            const uint32_t pv = sbs[(rbase + r) * gp + kc];
            sr[r] = bf_lo(pv);
            br[r] = bf_hi(pv);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float yf[8];
            unpack8(*reinterpret_cast<const uint4 *>(ys + t * a.I + kc * 64 + c * 8), yf);
            float ysum = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) ysum += yf[i];
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][t] += fmaf(sr[r], dot8(qf[r], yf), br[r] * ysum);
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
    if (c < nt)
        st_relaxed_gpu_v2u64(odst + (size_t)c * (a.H / 2) + rbase / 2,
                             tag | pack_bf2(pick<NT, 4>(acc, 0, c), pick<NT, 4>(acc, 1, c)),
                             tag | pack_bf2(pick<NT, 4>(acc, 2, c), pick<NT, 4>(acc, 3, c)));
    return true;
}

// 4-bit gate_up item on mma.sync: warp w multiplies columns 32w..32w+31 of
// every 256-column stage for all 32 rows (two 16-row tiles: gate, up) with the
// item's tokens (n = token slot, x rows from the staged token rows), then adds
// the affine terms of that 64-element group: s * D + (b - 128 s) * sum(x).
// The eight warps' partial sums meet in `red`; warps 0-1 reduce them (in warp
// order), apply GeGLU and store the tagged GeGLU words.  The hand-offs use
// mbarriers with bounded waits: redfull (all 8 warps wrote), redfree (the
// reduction has read `red`).
// 4-bit items arrive whole: one ring slot holds an item's packed rows (gate_up:
// 16 gate + 16 up rows of H/8 words; down: 128 rows of I/8 words), copied as
// contiguous runs by 1-D bulk copies, followed by its (scale, bias) rows.
// One bf16 fragment pair (128 + q, 128 + q') from a fragment-ordered code
// word (repack_q4_decode_kernel, quant.cu): pair p sits at bits 4p and 16 + 4p.
__device__ __forceinline__ uint32_t q4_frag(uint32_t w, int p) {
    return ((w >> (4 * p)) & 0x000F000Fu) | 0x43004300u;
}

__host__ __device__ inline int q4_code_words(int H, int I) {
    const int gu = 32 * (H / 8), dn = kDnRows * (I / 8);
    return gu > dn ? gu : dn;
}
__host__ __device__ inline size_t q4_slot_bytes(int H, int I) {
    return ((size_t)q4_code_words(H, I) + sb_slot_words(H, I)) * 4;
}

// 4-bit gate_up item on mma.sync: warp w multiplies columns 32w..32w+31 of
// every 256-column block for all 32 rows (two 16-row tiles: gate, up) with the
// item's tokens (n = token slot, x rows from the staged token rows), then adds
// the affine terms of that 64-element group: s * D + (b - 128 s) * sum(x).
// The eight warps' partial sums meet in `red`; warps 0-1 reduce them (in warp
// order), apply GeGLU and store the tagged GeGLU words.  The hand-offs use
// mbarriers with bounded waits: redfull (all 8 warps wrote), redfree (the
// reduction has read `red`).
__device__ bool gateup_item_q4(const uint32_t *codes, const uint32_t *sbs, int gp,
                               const uint16_t *xs, const float *xsum32, const int *toks, int nt,
                               float *red, uint64_t *redfull, uint64_t *redfree, int &gi,
                               const FusedArgs &a, int w, int lane, unsigned long long *ydst,
                               unsigned long long tag) {
    const int NK = a.H / 256, HB = a.H / 32, RW = a.H / 8;
    const int gid = lane >> 2, t = lane & 3;
    const uint16_t *xrow = xs + (size_t)(gid < nt ? toks[gid] : toks[0]) * a.H;
    const int n0 = 2 * t, n1 = 2 * t + 1;
    const float *xs0 = xsum32 + (size_t)(n0 < nt ? toks[n0] : toks[0]) * HB;
    const float *xs1 = xsum32 + (size_t)(n1 < nt ? toks[n1] : toks[0]) * HB;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    (void)RW;
    for (int kc = 0; kc < NK; ++kc) {
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        // this lane's codes of the step, fragment-ordered: gate rows g, g + 8,
        // up rows g, g + 8 (one conflict-free 16-byte load)
        const uint4 q = *reinterpret_cast<const uint4 *>(codes + ((kc * 8 + w) * 32 + lane) * 4);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int k0 = kc * 256 + 32 * w + 16 * c;  // column within the row
            uint32_t b0 = 0u, b1 = 0u;
            if (gid < nt) {
                b0 = *reinterpret_cast<const uint32_t *>(xrow + k0 + 2 * t);
                b1 = *reinterpret_cast<const uint32_t *>(xrow + k0 + 2 * t + 8);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t wa = h ? q.z : q.x, wb = h ? q.w : q.y;
                const uint32_t af[4] = {q4_frag(wa, 2 * c), q4_frag(wb, 2 * c),
                                        q4_frag(wa, 2 * c + 1), q4_frag(wb, 2 * c + 1)};
                mma_bf16_16816(d[h], af, b0, b1);
            }
        }
        const int grp = kc * 4 + (w >> 1);
        const float x0 = n0 < nt ? xs0[kc * 8 + w] : 0.f;
        const float x1 = n1 < nt ? xs1[kc * 8 + w] : 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t p0 = sbs[(h * 16 + gid) * gp + grp];
            const uint32_t p1 = sbs[(h * 16 + gid + 8) * gp + grp];
            const float s0 = bf_lo(p0), c0 = fmaf(-128.f, s0, bf_hi(p0));
            const float s1 = bf_lo(p1), c1 = fmaf(-128.f, s1, bf_hi(p1));
            acc[h][0] += fmaf(s0, d[h][0], c0 * x0);
            acc[h][1] += fmaf(s0, d[h][1], c0 * x1);
            acc[h][2] += fmaf(s1, d[h][2], c1 * x0);
            acc[h][3] += fmaf(s1, d[h][3], c1 * x1);
        }
    }
    // partial sums -> red[w][row][token], once the previous item's reduction has read red
    if (gi > 0 && !mbar_wait(redfree, (gi - 1) & 1, kWait)) {
        record_error(a.err, 84, gi);
        return false;
    }
    float *rw = red + w * 256;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        rw[(h * 16 + gid) * 8 + n0] = acc[h][0];
        rw[(h * 16 + gid) * 8 + n1] = acc[h][1];
        rw[(h * 16 + gid + 8) * 8 + n0] = acc[h][2];
        rw[(h * 16 + gid + 8) * 8 + n1] = acc[h][3];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(redfull);
    if (w < 2) {
        if (!mbar_wait(redfull, gi & 1, kWait)) {
            record_error(a.err, 85, gi);
            return false;
        }
        const int tid = w * 32 + lane, jp = tid >> 3, n = tid & 7;  // column pair, token
        if (n < nt) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};  // gate 2jp, 2jp+1, up 2jp, 2jp+1
#pragma unroll
            for (int q = 0; q < kCW; ++q) {
                const float *rq = red + q * 256;
                v[0] += rq[(2 * jp) * 8 + n];
                v[1] += rq[(2 * jp + 1) * 8 + n];
                v[2] += rq[(16 + 2 * jp) * 8 + n];
                v[3] += rq[(16 + 2 * jp + 1) * 8 + n];
            }
            const float y0 = geglu_bf16(rbf(v[0]), rbf(v[2]));
            const float y1 = geglu_bf16(rbf(v[1]), rbf(v[3]));
            st_relaxed_gpu_u64(ydst + (size_t)n * (a.I / 2) + jp, tag | pack_bf2(y0, y1));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(redfree);
    }
    ++gi;
    return true;
}

// 4-bit down item on mma.sync: warp w owns rows 16w..16w+15 of the item's 128
// and all columns, one 64-element group per step: s * D + (b - 128 s) * sum(y).
__device__ void down_item_q4(const uint32_t *codes, const uint32_t *sbs, int gp,
                             const uint16_t *ys, const float *ysum, int nt, const FusedArgs &a,
                             int w, int lane, unsigned long long *odst, unsigned long long tag) {
    const int NK = a.I / 64, RW = a.I / 8;
    const int gid = lane >> 2, t = lane & 3;
    const int n0 = 2 * t, n1 = 2 * t + 1;
    const uint16_t *yrow = ys + (size_t)(gid < nt ? gid : 0) * a.I;
    (void)RW;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kc = 0; kc < NK; ++kc) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        // this lane's codes of the group, fragment-ordered: rows g, g + 8 of
        // the first 32 columns, then of the second (one 16-byte load)
        const uint4 q = *reinterpret_cast<const uint4 *>(codes + ((kc * 8 + w) * 32 + lane) * 4);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t b0 = 0u, b1 = 0u;
            if (gid < nt) {
                b0 = *reinterpret_cast<const uint32_t *>(yrow + kc * 64 + 16 * c + 2 * t);
                b1 = *reinterpret_cast<const uint32_t *>(yrow + kc * 64 + 16 * c + 2 * t + 8);
            }
            const uint32_t wa = (c >> 1) ? q.z : q.x, wb = (c >> 1) ? q.w : q.y;
            const int p = 2 * (c & 1);
            const uint32_t af[4] = {q4_frag(wa, p), q4_frag(wb, p), q4_frag(wa, p + 1),
                                    q4_frag(wb, p + 1)};
            mma_bf16_16816(d, af, b0, b1);
        }
        const float y0 = n0 < nt ? ysum[n0 * NK + kc] : 0.f;
        const float y1 = n1 < nt ? ysum[n1 * NK + kc] : 0.f;
        const uint32_t p0 = sbs[(16 * w + gid) * gp + kc];
        const uint32_t p1 = sbs[(16 * w + gid + 8) * gp + kc];
        const float s0 = bf_lo(p0), c0 = fmaf(-128.f, s0, bf_hi(p0));
        const float s1 = bf_lo(p1), c1 = fmaf(-128.f, s1, bf_hi(p1));
        acc[0] += fmaf(s0, d[0], c0 * y0);
        acc[1] += fmaf(s0, d[1], c0 * y1);
        acc[2] += fmaf(s1, d[2], c1 * y0);
        acc[3] += fmaf(s1, d[3], c1 * y1);
    }
    // rows (16w + gid, +1) pair up across lanes gid, gid + 1 (lane + 4)
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_down_sync(0xffffffffu, acc[i], 4);
    if ((gid & 1) == 0) {
        const int r = 16 * w + gid;
        if (n0 < nt) {
            st_relaxed_gpu_u64(odst + (size_t)n0 * (a.H / 2) + r / 2, tag | pack_bf2(acc[0], p[0]));
            st_relaxed_gpu_u64(odst + (size_t)n0 * (a.H / 2) + (r + 8) / 2, tag | pack_bf2(acc[2], p[2]));
        }
        if (n1 < nt) {
            st_relaxed_gpu_u64(odst + (size_t)n1 * (a.H / 2) + r / 2, tag | pack_bf2(acc[1], p[1]));
            st_relaxed_gpu_u64(odst + (size_t)n1 * (a.H / 2) + (r + 8) / 2, tag | pack_bf2(acc[3], p[3]));
        }
    }
}

template <int NTMAX, int S, int BITS>
__device__ bool run_gateup_q(const uint8_t *ring, uint64_t *full, uint64_t *empty,
                             const uint16_t *xs, const uint32_t *sbs, int gp, const int *toks,
                             int nt, const FusedArgs &a, int &g, int w, int lane,
                             unsigned long long *ydst, unsigned long long tag) {
    if (nt == 1)
        return gateup_item_q<1, S, BITS>(ring, full, empty, xs, sbs, gp, toks, nt, a, g, w, lane, ydst, tag);
    if constexpr (NTMAX >= 2)
        if (nt == 2)
            return gateup_item_q<2, S, BITS>(ring, full, empty, xs, sbs, gp, toks, nt, a, g, w, lane, ydst, tag);
    if constexpr (NTMAX >= 4)
        if (nt <= 4)
            return gateup_item_q<4, S, BITS>(ring, full, empty, xs, sbs, gp, toks, nt, a, g, w, lane, ydst, tag);
    if constexpr (NTMAX >= 8)
        return gateup_item_q<8, S, BITS>(ring, full, empty, xs, sbs, gp, toks, nt, a, g, w, lane, ydst, tag);
    return false;
}

template <int NTMAX, int S, int BITS>
__device__ bool run_down_q(const uint8_t *ring, uint64_t *full, uint64_t *empty, const uint16_t *ys,
                           const uint32_t *sbs, int gp, int nt, const FusedArgs &a, int &g, int w,
                           int lane, unsigned long long *odst, unsigned long long tag) {
    if (nt == 1) return down_item_q<1, S, BITS>(ring, full, empty, ys, sbs, gp, nt, a, g, w, lane, odst, tag);
    if constexpr (NTMAX >= 2)
        if (nt == 2)
            return down_item_q<2, S, BITS>(ring, full, empty, ys, sbs, gp, nt, a, g, w, lane, odst, tag);
    if constexpr (NTMAX >= 4)
        if (nt <= 4)
            return down_item_q<4, S, BITS>(ring, full, empty, ys, sbs, gp, nt, a, g, w, lane, odst, tag);
    if constexpr (NTMAX >= 8)
        return down_item_q<8, S, BITS>(ring, full, empty, ys, sbs, gp, nt, a, g, w, lane, odst, tag);
    return false;
}

template <int NTMAX, int BITS>
__global__ void __launch_bounds__(kThreads, 1)
decode_fused_kernel(const __grid_constant__ CUtensorMap tmGU,
                    const __grid_constant__ CUtensorMap tmDN,
                    const __grid_constant__ CUtensorMap tmSG,
                    const __grid_constant__ CUtensorMap tmSD, FusedArgs a) {
    constexpr int S = stages_for<NTMAX, BITS>();
    constexpr int SBY = stage_bytes<BITS>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *ring = smem_align(smem_raw, 1024);
    uint16_t *xs = reinterpret_cast<uint16_t *>(ring + ring_bytes<NTMAX, BITS>());  // [T][H]
    uint16_t *ys = xs + (size_t)a.T * a.H;                                           // [2][NTMAX][I]
    // 8-bit experts: kSB (scale, bias) slots, 128-byte aligned
    uint32_t *sbq = reinterpret_cast<uint32_t *>(ys + 2 * NTMAX * a.I);
    const int slotw = sb_slot_words(a.H, a.I);
    // 4-bit experts: whole-item slots in the ring
    const size_t q4slot = (q4_slot_bytes(a.H, a.I) + 127) & ~size_t(127);
    const int ns = BITS == 4 ? (int)(ring_bytes<NTMAX, BITS>() / q4slot) : S;
    const int gpH = ((a.H / 64) + 3) / 4 * 4, gpI = ((a.I / 64) + 3) / 4 * 4;
    // 4-bit: gate_up partial sums, x sums per 32 columns, GeGLU-row sums per group
    float *red = reinterpret_cast<float *>(sbq + (BITS == 8 ? kSB * slotw : 0));
    float *xsum32 = red + (BITS == 4 ? kRedFloats : 0);
    float *ysum = xsum32 + (BITS == 4 ? a.T * (a.H / 32) : 0);
    const int GI = a.I / 64;
    uint64_t *bars = reinterpret_cast<uint64_t *>(
        smem_align(reinterpret_cast<uint8_t *>(ysum + (BITS == 4 ? 2 * NTMAX * GI : 0)), 8));
    uint64_t *full = bars, *empty = bars + S;
    uint64_t *yfull = bars + 2 * S, *yempty = yfull + 2, *xbar = yempty + 2;
    uint64_t *sbfull = xbar + 1, *sbempty = sbfull + kSB;
    uint64_t *redfull = sbempty + kSB, *redfree = redfull + 1;
    __shared__ float s_r[kMaxT];
    __shared__ float s_part[kThreads / 32][kMaxT];
    __shared__ int s_U, s_skip;
    __shared__ uint32_t s_epoch;
    __shared__ int s_idx[kMaxPairs];
    __shared__ int s_rank[kMaxPairs], s_lt[kMaxPairs], s_cnt[kMaxPairs];
    __shared__ int s_act[kMaxPairs], s_n[kMaxPairs], s_off[kMaxPairs];
    __shared__ int s_tok[kMaxPairs][kMaxT];
    __shared__ int s_idone;
    __shared__ int s_q[kQ];
    __shared__ __align__(8) uint64_t s_qfull[kQ], s_qempty[kQ];
    __shared__ int s_inv[kMaxPairs];
    __shared__ float s_wsel[kMaxPairs];
    __shared__ int s_slot[kEpMaxExperts];
    __shared__ int s_ulast[kMaxT];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, H = a.H, E = a.E, K = a.K, I = a.I;
    const int P = T * K;
    const bool has_e = (int)blockIdx.x < E;
    const bool same_x = a.xr == a.xe;
    // router staging in the ring (dead once the dispatch is built): x_router
    // rows (when distinct from the expert input), this CTA's proj row, scale,
    // per_expert_scale, then all the scores [T][E] f32
    uint16_t *xr_s = same_x ? xs : reinterpret_cast<uint16_t *>(ring);
    uint16_t *p_s = reinterpret_cast<uint16_t *>(ring) + (same_x ? 0 : (size_t)T * H);
    uint16_t *sc_s = p_s + H;
    uint16_t *pes_s = sc_s + H;
    float *s_all = reinterpret_cast<float *>(pes_s + ((E + 7) / 8) * 8);
    const int NDN = H / kDnRows;
    const int SW = kSetWords;

    // ---- 1. router: CTA e computes expert e's scores for all T tokens
    if (tid == 0) FT_STAMP(0);
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&yfull[b], 1);
            mbar_init(&yempty[b], kCW);
        }
        mbar_init(xbar, 1);
        if (BITS)
            for (int q = 0; q < kSB; ++q) {
                mbar_init(&sbfull[q], 1);
                mbar_init(&sbempty[q], kCW);
            }
        if (BITS == 4) {
            mbar_init(redfull, kCW);
            mbar_init(redfree, 2);
        }
        for (int q = 0; q < kQ; ++q) {
            mbar_init(&s_qfull[q], 1);
            mbar_init(&s_qempty[q], kCW + 2);  // compute warps, stager, signal warp
        }
        fence_barrier_init();
        s_idone = 0;
        s_skip = 0;
        s_epoch = (uint32_t)a.sync[blockIdx.x] + 1u;  // this call's count
        a.sync[blockIdx.x] = (int32_t)s_epoch;
        const uint32_t row = (uint32_t)H * 2;
        uint32_t bytes = (uint32_t)T * row + (uint32_t)E * 2;
        if (!same_x) bytes += (uint32_t)T * row;
        if (has_e) bytes += 2 * row;
        mbar_arrive_expect_tx(xbar, bytes);
        bulk_load(xs, a.xe, (uint32_t)T * row, xbar);
        if (!same_x) bulk_load(xr_s, a.xr, (uint32_t)T * row, xbar);
        if (has_e) {
            bulk_load(p_s, a.proj + (size_t)blockIdx.x * H, row, xbar);
            bulk_load(sc_s, a.scale, row, xbar);
        }
        bulk_load(pes_s, a.pes, (uint32_t)E * 2, xbar);
        tma_prefetch(&tmGU);
        tma_prefetch(&tmDN);
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    int32_t *set = a.sync + kMaxGrid + (epoch & 1u) * SW;
    int32_t *work = set;
    int32_t *scnt = set + 1;
    const unsigned long long tag = (unsigned long long)epoch << 32;
    {  // the other parity's counters, used by the previous call, for the next one
        int32_t *other = a.sync + kMaxGrid + ((epoch & 1u) ^ 1u) * SW;
        for (int i = blockIdx.x * kThreads + tid; i < SW; i += gridDim.x * kThreads) other[i] = 0;
    }
    if (!mbar_wait(xbar, 0, kWait) && tid == 0) {
        record_error(a.err, 70, blockIdx.x);
        s_skip = 1;
    }
    if (tid == 0) FT_STAMP(1);
    if constexpr (BITS == 4) {  // sums of each token's x over 32-column blocks
        const int HB = H / 32;
        for (int i = tid; i < T * HB; i += kThreads) {
            const uint4 *src = reinterpret_cast<const uint4 *>(xs + (size_t)(i / HB) * H + (i % HB) * 32);
            float sum = 0.f;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                float f[8];
                unpack8(src[v], f);
#pragma unroll
                for (int j = 0; j < 8; ++j) sum += f[j];
            }
            xsum32[i] = sum;
        }
    }
    if (has_e) {
        for (int t = warp; t < T; t += kThreads / 32) {
            float ss = 0.f;
            for (int c = lane; c < H / 8; c += 32) {
                float f[8];
                unpack8(*reinterpret_cast<const uint4 *>(xr_s + (size_t)t * H + c * 8), f);
#pragma unroll
                for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) s_r[t] = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)H), a.eps));
        }
        __syncthreads();
        float acc[NTMAX];
#pragma unroll
        for (int t = 0; t < NTMAX; ++t) acc[t] = 0.f;
        for (int c = tid; c < H / 8; c += kThreads) {
            float sf[8], pf[8];
            unpack8(*reinterpret_cast<const uint4 *>(sc_s + c * 8), sf);
            unpack8(*reinterpret_cast<const uint4 *>(p_s + c * 8), pf);
#pragma unroll
            for (int t = 0; t < NTMAX; ++t) {
                if (t >= T) break;
                float f[8];
                unpack8(*reinterpret_cast<const uint4 *>(xr_s + (size_t)t * H + c * 8), f);
                const float r = s_r[t];
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[t] = fmaf(pf[j], router_h(f[j], r, sf[j], a.root), acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < NTMAX; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0) s_part[warp][t] = v;
        }
        __syncthreads();
        if (tid < T) {
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < kThreads / 32; ++q) v += s_part[q][tid];
            a.scores[(size_t)tid * E + blockIdx.x] = v;
        }
    }
    if (tid == 0) FT_STAMP(2);
    // ---- hand-over: each scoring CTA adds one to the count (release, after
    // its scores); every CTA waits until all E have (acquire), then reads them
    __syncthreads();
    if (tid == 0) {
        if (has_e) red_add_release_gpu(scnt, 1);
        const long long t0 = clock64();
        while (ld_acquire_gpu(scnt) < E) {
            if (clock64() - t0 > kWait) {
                record_error(a.err, 73, blockIdx.x);
                s_skip = 1;
                break;
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < T * E; i += kThreads) s_all[i] = __ldcg(a.scores + i);
    __syncthreads();
    if (tid == 0) FT_STAMP(3);
    // ---- every CTA selects the top-K and builds the dispatch itself, in
    // shared memory (same inputs and arithmetic, so the same result in every
    // CTA); CTA 0 also writes idx, w and the dispatch out for the caller.
    // Selection: one warp per token (select_core: softmax, top-K in
    // descending probability with lower id on ties, k-order sum), then the
    // routing weights p_k / sum * per_expert_scale.
    for (int t = warp; t < T; t += kThreads / 32) {
        int e;
        float sel_p, sum;
        const float *pt = s_all + t * E;
        if (E <= 128) {
            float p[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) p[j] = lane + 32 * j < E ? pt[lane + 32 * j] : -INFINITY;
            select_core<4>(p, E, K, lane, e, sel_p, sum);
        } else {
            float p[kMaxPerLane];
#pragma unroll
            for (int j = 0; j < kMaxPerLane; ++j) p[j] = lane + 32 * j < E ? pt[lane + 32 * j] : -INFINITY;
            select_core<kMaxPerLane>(p, E, K, lane, e, sel_p, sum);
        }
        if (lane < K) {
            if ((unsigned)e >= (unsigned)E) e = 0;  // all-NaN scores: stay in range
            const uint16_t wb = f2bf(__fmul_rn(__fdiv_rn(sel_p, sum), bf2f(pes_s[e])));
            s_idx[t * K + lane] = e;
            s_wsel[t * K + lane] = bf2f(wb);
            if (blockIdx.x == 0) {
                a.idx[(size_t)t * K + lane] = e;
                a.w[(size_t)t * K + lane] = wb;
            }
        }
    }
    __syncthreads();
    if (tid == 0) FT_STAMP(8);
    // dispatch position: pairs sorted by expert, stable (pair order inside an
    // expert); the expert's group offset, size and this pair's rank in it
    if (tid < P) {
        const int e = s_idx[tid];
        int lt = 0, before = 0, n = 0;
        for (int j = 0; j < P; ++j) {
            const int ej = s_idx[j];
            lt += ej < e;
            n += ej == e;
            before += (ej == e) & (j < tid);
        }
        s_inv[tid] = lt + before;
        s_rank[tid] = before;
        s_lt[tid] = lt;
        s_cnt[tid] = n;
        if (blockIdx.x == 0) {
            a.d.perm[lt + before] = tid;
            a.d.inv[tid] = lt + before;
        }
    }
    // active experts (ascending id): the first pair of each expert takes slot
    // #{first pairs of smaller experts}
    const int nact = __syncthreads_count(tid < P && s_rank[tid] == 0);
    if (tid == 0) FT_STAMP(9);
    if (tid < P && s_rank[tid] == 0) {
        const int e = s_idx[tid];
        int u = 0;
        for (int j = 0; j < P; ++j) u += (s_rank[j] == 0) & (s_idx[j] < e);
        s_slot[e] = u;
        s_act[u] = e;
        s_n[u] = s_cnt[tid];
        s_off[u] = s_lt[tid];
        if (blockIdx.x == 0) a.d.active[u] = e;
    }
    if (blockIdx.x == 0) {  // the dispatch's per-expert counts and offsets
        for (int e = tid; e < E; e += kThreads) {
            int lt = 0, n = 0;
            for (int j = 0; j < P; ++j) {
                lt += s_idx[j] < e;
                n += s_idx[j] == e;
            }
            a.d.counts[e] = n;
            a.d.offsets[e] = lt;
        }
        if (tid == 0) {
            a.d.offsets[E] = P;
            *a.d.n_active = nact;
        }
    }
    if (tid == 0) s_U = nact;
    __syncthreads();
    if (tid == 0) FT_STAMP(10);
    if (tid < P) s_tok[s_slot[s_idx[tid]]][s_rank[tid]] = tid / K;
    if (tid < T) {  // each token's last expert in claim order (highest active slot)
        int ul = 0;
        for (int k = 0; k < K; ++k) ul = max(ul, s_slot[s_idx[tid * K + k]]);
        s_ulast[tid] = ul;
    }
    __syncthreads();  // the router's staging in the ring is dead from here on
    const int U = s_U;
    if (tid == 0) FT_STAMP(4);

    // ---- 2. expert items
    const int NGU = I / kGuCols;
    const int Ngu = U * NGU, N = U * (NGU + NDN);
    auto producer = [&]() {
        int g = 0, qi = 0, it = 0;
        for (;;) {
            // claim the next item (global order: every gate_up item before any
            // down item, so a down item only waits on items already claimed)
            int i = atomicAdd(work, 1);
            if (i >= N) i = -1;
            const int slot = qi % kQ;
            if (!mbar_wait(&s_qempty[slot], ((qi / kQ) & 1) ^ 1, kWait)) {
                record_error(a.err, 79, qi);
                return;
            }
            s_q[slot] = i;
            FT_ITEM(0, qi, i + 1);
            mbar_arrive(&s_qfull[slot]);
            ++qi;
            if (i < 0) break;
            int r0, nk;
            const bool gu = i < Ngu;
            if (gu) {
                const int u = i / NGU, blk = i - u * NGU;
                r0 = s_act[u] * 2 * I + blk * kGuCols;
                nk = H / 256;
            } else {
                const int j = i - Ngu, u = j / NDN, hb = j - u * NDN;
                r0 = s_act[u] * H + hb * kDnRows;
                nk = I / 64;
            }
            if constexpr (BITS == 4) {  // the whole item into one slot: 2-4 bulk copies
                const int sl = it % ns;
                if (!mbar_wait(&empty[sl], ((it / ns) & 1) ^ 1, kWait)) {
                    record_error(a.err, 74, i);
                    return;
                }
                uint32_t *dc = reinterpret_cast<uint32_t *>(ring + sl * q4slot);
                uint32_t *ds = dc + q4_code_words(H, I);
                const uint32_t rwH = (uint32_t)H / 8, rwI = (uint32_t)I / 8;
                if (gu) {
                    // codes: the item's fragment-ordered block (32 rows x H/8 words)
                    const int u = i / NGU, blk = i - u * NGU;
                    const size_t item = (size_t)s_act[u] * NGU + blk;
                    mbar_arrive_expect_tx(&full[sl], 2u * 16 * (rwH + gpH) * 4);
                    bulk_load(dc, a.gq + item * 32 * rwH, 32 * rwH * 4, &full[sl]);
                    bulk_load(ds, a.gsb + (size_t)r0 * gpH, 16u * gpH * 4, &full[sl]);
                    bulk_load(ds + 16 * gpH, a.gsb + (size_t)(r0 + I) * gpH, 16u * gpH * 4, &full[sl]);
                } else {
                    // codes: the item's fragment-ordered block (128 rows x I/8 words)
                    const int j = i - Ngu, u = j / NDN, hb = j - u * NDN;
                    const size_t item = (size_t)s_act[u] * NDN + hb;
                    mbar_arrive_expect_tx(&full[sl], (uint32_t)kDnRows * (rwI + gpI) * 4);
                    bulk_load(dc, a.dq + item * kDnRows * rwI, kDnRows * rwI * 4, &full[sl]);
                    bulk_load(ds, a.dsb + (size_t)r0 * gpI, (uint32_t)kDnRows * gpI * 4, &full[sl]);
                }
                ++it;
                FT_ITEM(6, qi - 1, 0);
                continue;
            }
            if constexpr (BITS > 0) {  // the item's (scale, bias) pairs
                const int sl = it % kSB;
                if (!mbar_wait(&sbempty[sl], ((it / kSB) & 1) ^ 1, kWait)) {
                    record_error(a.err, 82, i);
                    return;
                }
                uint32_t *dsb = sbq + sl * slotw;
                if (gu) {
                    mbar_arrive_expect_tx(&sbfull[sl], 2u * 16 * gpH * 4);
                    tma_load_2d(dsb, &tmSG, &sbfull[sl], 0, r0);
                    tma_load_2d(dsb + 16 * gpH, &tmSG, &sbfull[sl], 0, r0 + I);
                } else {
                    mbar_arrive_expect_tx(&sbfull[sl], (uint32_t)kDnRows * gpI * 4);
                    tma_load_2d(dsb, &tmSD, &sbfull[sl], 0, r0);
                }
                ++it;
            }
            for (int kc = 0; kc < nk; ++kc, ++g) {
                const int s = g % S;
                if (!mbar_wait(&empty[s], ((g / S) & 1) ^ 1, kWait)) {
                    record_error(a.err, 74, i);
                    return;
                }
                mbar_arrive_expect_tx(&full[s], SBY);
                uint8_t *dst = ring + s * SBY;
                // coordinates in elements: bf16 values, or u32 words of codes
                constexpr int GU_X = BITS ? 256 * BITS / 32 : 256, DN_X = BITS ? 64 * BITS / 32 : 64;
                if (gu) {
                    tma_load_2d(dst, &tmGU, &full[s], kc * GU_X, r0);
                    tma_load_2d(dst + SBY / 2, &tmGU, &full[s], kc * GU_X, r0 + I);
                } else {
                    tma_load_2d(dst, &tmDN, &full[s], kc * DN_X, r0);
                }
            }
            FT_ITEM(6, qi - 1, 0);
        }
    };
    int qi = 0;
    auto next = [&]() -> int {  // the next claimed item, -1 at the end, -2 on a timeout
        const int slot = qi % kQ;
        if (!mbar_wait(&s_qfull[slot], (qi / kQ) & 1, kWait)) {
            if (lane == 0) record_error(a.err, 80, qi);
            return -2;
        }
        const int i = s_q[slot];
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_qempty[slot]);
        ++qi;
        return i;
    };
    auto stager = [&]() {
        // a down item's GeGLU rows: poll the tagged words (up to kYB loads in
        // flight per lane) until every one carries this call's count, then
        // hand the rows to the compute warps through a double buffer
        constexpr int kYB = 12;
        int ub = 0;
        for (int i = next(); i >= 0; i = next()) {
            if (i < Ngu) continue;
            const int u = (i - Ngu) / NDN;
            const int b = ub & 1;
            if (!mbar_wait(&yempty[b], ((ub >> 1) & 1) ^ 1, kWait)) {
                if (lane == 0) record_error(a.err, 76, i);
                return;
            }
            const int nw = s_n[u] * (I / 2);
            const unsigned long long *src = a.yq + (size_t)s_off[u] * (I / 2);
            uint32_t *dst = reinterpret_cast<uint32_t *>(ys + (size_t)b * NTMAX * I);
            for (int v0 = 0; v0 < nw; v0 += 32 * kYB) {
                unsigned long long x[kYB];
                const unsigned long long *ptr[kYB];
                int n = 0;
#pragma unroll
                for (int q = 0; q < kYB; ++q) {
                    const int v = v0 + q * 32 + lane;
                    ptr[q] = src + (v < nw ? v : 0);
                    n += v < nw;
                }
                tagged_load<kYB>(x, ptr, n, epoch, a.err, 75, u);
#pragma unroll
                for (int q = 0; q < kYB; ++q)
                    if (q < n) dst[v0 + q * 32 + lane] = (uint32_t)x[q];
            }
            if constexpr (BITS == 4) {  // sums of each staged row over 64-element groups
                __syncwarp();
                const uint16_t *yb = ys + (size_t)b * NTMAX * I;
                float *sb = ysum + b * NTMAX * GI;
                for (int k = lane; k < s_n[u] * GI; k += 32) {
                    const uint4 *src = reinterpret_cast<const uint4 *>(yb + (size_t)(k / GI) * I + (k % GI) * 64);
                    float sum = 0.f;
#pragma unroll
                    for (int v = 0; v < 8; ++v) {
                        float f[8];
                        unpack8(src[v], f);
#pragma unroll
                        for (int j = 0; j < 8; ++j) sum += f[j];
                    }
                    sb[k] = sum;
                }
            }
            if (lane == 0) FT_ITEM(5, qi - 1, 0);
            __syncwarp();
            if (lane == 0) mbar_arrive(&yfull[b]);
            ++ub;
        }
    };
    auto signal = [&]() {
        // The combine, off the compute warps' path: the down item (u, hb) of
        // each token's last expert in claim order (the highest active slot;
        // its other experts' down items were claimed before it) sums
        // bf16(w * row) in k order (f32) over the token's K down rows of row
        // block hb and stores the output slice, rounded once.  The rows are
        // read as tagged words; those of other CTAs are almost always ready.
        int j = 0;
        for (int i = next(); i >= 0; i = next(), ++j) {
            if (i < Ngu) continue;
            {  // every lane acquires the compute warps' stores of this item
                const long long t0 = clock64();
                while (ld_acquire_cta_shared(&s_idone) < kCW * (j + 1)) {
                    if (clock64() - t0 > kWait) {
                        if (lane == 0) record_error(a.err, 78, i);
                        break;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) FT_ITEM(2, j, 0);
            const int jj = i - Ngu, u = jj / NDN, hb = jj - u * NDN;
            const int n = s_n[u];
            unsigned fin = __ballot_sync(0xffffffffu, lane < n && s_ulast[s_tok[u][lane < n ? lane : 0]] == u);
            while (fin) {
                const int r = __ffs(fin) - 1;
                fin &= fin - 1;
                const int tt = s_tok[u][r];
                const int w0 = hb * (kDnRows / 2) + lane * 2;  // 4 hidden columns per lane
                float acc[4] = {0, 0, 0, 0};
                for (int k0 = 0; k0 < K; k0 += 8) {
                    unsigned long long x[16];
                    const unsigned long long *ptr[16];
                    const int nk = min(8, K - k0);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const unsigned long long *src =
                            a.oq + (size_t)s_inv[tt * K + k0 + (q < nk ? q : 0)] * (H / 2) + w0;
                        ptr[2 * q] = src;
                        ptr[2 * q + 1] = src + 1;
                    }
                    tagged_load<16>(x, ptr, 2 * nk, epoch, a.err, 81, tt);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        if (q >= nk) continue;
                        const uint32_t lo = (uint32_t)x[2 * q], hi = (uint32_t)x[2 * q + 1];
                        const float f[4] = {bf2f((uint16_t)lo), bf2f((uint16_t)(lo >> 16)),
                                            bf2f((uint16_t)hi), bf2f((uint16_t)(hi >> 16))};
                        const float wk = s_wsel[tt * K + k0 + q];
#pragma unroll
                        for (int c = 0; c < 4; ++c) acc[c] = __fadd_rn(acc[c], rbf(__fmul_rn(wk, f[c])));
                    }
                }
                uint2 o;
                o.x = pack_bf2(acc[0], acc[1]);
                o.y = pack_bf2(acc[2], acc[3]);
                *reinterpret_cast<uint2 *>(a.out + (size_t)tt * H + 2 * w0) = o;
            }
        }
        if (lane == 0) FT_STAMP(6);
    };
    auto compute = [&]() {
    int g = 0, ub = 0, it = 0, gi = 0;
    for (int i = next(); i >= 0; i = next()) {
        const uint32_t *sbs = nullptr, *codes = nullptr;
        int sl = 0;
        if constexpr (BITS == 4) {  // the item's slot: codes, then (scale, bias) rows
            sl = it % ns;
            if (!mbar_wait(&full[sl], (it / ns) & 1, kWait)) {
                if (lane == 0) record_error(a.err, 83, i);
                return;
            }
            codes = reinterpret_cast<const uint32_t *>(ring + sl * q4slot);
            sbs = codes + q4_code_words(H, I);
            ++it;
        } else if constexpr (BITS > 0) {  // the item's (scale, bias) pairs
            sl = it % kSB;
            if (!mbar_wait(&sbfull[sl], (it / kSB) & 1, kWait)) {
                if (lane == 0) record_error(a.err, 83, i);
                return;
            }
            sbs = sbq + sl * slotw;
            ++it;
        }
        if (i < Ngu) {
            const int u = i / NGU, blk = i - u * NGU;
            unsigned long long *ydst = a.yq + (size_t)s_off[u] * (I / 2) + blk * (kGuCols / 2);
            bool ok;
            if constexpr (BITS == 4)
                ok = gateup_item_q4(codes, sbs, gpH, xs, xsum32, s_tok[u], s_n[u], red, redfull,
                                    redfree, gi, a, warp, lane, ydst, tag);
            else if constexpr (BITS > 0)
                ok = run_gateup_q<NTMAX, S, BITS>(ring, full, empty, xs, sbs, gpH, s_tok[u], s_n[u],
                                                  a, g, warp, lane, ydst, tag);
            else
                ok = run_gateup<NTMAX, S>(ring, full, empty, xs, s_tok[u], s_n[u], a, g, warp,
                                          lane, ydst, tag);
            if (!ok) return;
        } else {
            const int jj = i - Ngu, u = jj / NDN, hb = jj - u * NDN;
            const int b = ub & 1;
            if (!mbar_wait(&yfull[b], (ub >> 1) & 1, kWait)) {
                if (lane == 0) record_error(a.err, 77, i);
                return;
            }
            if (tid == 0) FT_ITEM(4, qi - 1, 0);
            unsigned long long *odst = a.oq + (size_t)s_off[u] * (H / 2) + hb * (kDnRows / 2);
            bool ok;
            if constexpr (BITS == 4) {
                down_item_q4(codes, sbs, gpI, ys + (size_t)b * NTMAX * I, ysum + b * NTMAX * GI,
                             s_n[u], a, warp, lane, odst, tag);
                ok = true;
            }
            else if constexpr (BITS > 0)
                ok = run_down_q<NTMAX, S, BITS>(ring, full, empty, ys + (size_t)b * NTMAX * I, sbs,
                                                gpI, s_n[u], a, g, warp, lane, odst, tag);
            else
                ok = run_down<NTMAX, S>(ring, full, empty, ys + (size_t)b * NTMAX * I, s_n[u], a, g,
                                        warp, lane, odst, tag);
            if (!ok) return;
            __syncwarp();
            if (lane == 0) mbar_arrive(&yempty[b]);
            ++ub;
        }
        __syncwarp();  // the warp's stores of this item, then one release
        if (lane == 0) {
            red_add_release_cta_shared(&s_idone, 1);
            if (BITS == 4) mbar_arrive(&empty[sl]);
            else if (BITS) mbar_arrive(&sbempty[sl]);
        }
        if (tid == 0) FT_ITEM(1, qi - 1, 0);
    }
    if (tid == 0) FT_STAMP(5);
    };
    if (!s_skip) {
        if (warp == kProdWarp) {
            if (lane == 0) producer();
        } else if (warp == kStagerWarp) {
            stager();
        } else if (warp == kSignalWarp) {
            signal();
        } else {
            compute();
        }
    }
#ifdef APT_FUSED_TRACE
    __syncthreads();
    if (tid == 0) FT_STAMP(7);
#endif
}

template <int NTMAX, int BITS>
size_t fused_smem(int T, int H, int I) {
    constexpr int S = stages_for<NTMAX, BITS>();
    return 1024 + (size_t)ring_bytes<NTMAX, BITS>() + (size_t)T * H * 2 +
           2 * (size_t)NTMAX * I * 2 + (BITS == 8 ? (size_t)kSB * sb_slot_words(H, I) * 4 : 0) +
           (BITS == 4 ? 4 * ((size_t)kRedFloats + (size_t)T * (H / 32) + 2 * (size_t)NTMAX * (I / 64)) + 8
                      : 0) +
           8 * (2 * S + 5 + 2 * kSB + 2) + 64;
}

template <int NTMAX, int BITS>
cudaError_t fused_attr() {
    return cudaFuncSetAttribute(decode_fused_kernel<NTMAX, BITS>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
}

template <int NTMAX, int BITS>
cudaError_t launch_fused_nt(const CUtensorMap (&m)[4], const FusedArgs &a, cudaStream_t s) {
    const int dev = current_device();
    static int occ_cache[64][12] = {};
    const int slot = (NTMAX == 1 ? 0 : NTMAX == 2 ? 1 : NTMAX == 4 ? 2 : 3) + 4 * (BITS / 4);
    int &occ = occ_cache[dev & 63][slot];
    if (!occ) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_fused_kernel<NTMAX, BITS>,
                                                      kThreads,
                                                      fused_smem<NTMAX, BITS>(NTMAX, a.H, a.I));
        if (occ < 1) return cudaErrorInvalidConfiguration;
    }
    // every CTA waits on the scores of the CTAs < E: the grid must be
    // resident at once, one CTA per SM
    const int grid = grid_sms(dev);
    if (grid < a.E) return cudaErrorInvalidConfiguration;
    return launch_ex(decode_fused_kernel<NTMAX, BITS>, dim3(grid), dim3(kThreads),
                     fused_smem<NTMAX, BITS>(a.T, a.H, a.I), s, false, m[0], m[1], m[2], m[3], a);
}

template <int BITS>
size_t fused_smem_T(int T, int H, int I) {
    return T <= 1 ? fused_smem<1, BITS>(T, H, I) : T <= 2 ? fused_smem<2, BITS>(T, H, I)
         : T <= 4 ? fused_smem<4, BITS>(T, H, I) : fused_smem<8, BITS>(T, H, I);
}

template <int BITS>
size_t ring_T(int T) {
    return T <= 2 ? ring_bytes<2, BITS>() : T <= 4 ? ring_bytes<4, BITS>() : ring_bytes<8, BITS>();
}

template <int BITS>
cudaError_t launch_bits(const CUtensorMap (&m)[4], const FusedArgs &a, cudaStream_t s) {
    // the largest per-expert token count is at most T
    const int T = a.T;
    return T <= 1   ? launch_fused_nt<1, BITS>(m, a, s)
           : T <= 2 ? launch_fused_nt<2, BITS>(m, a, s)
           : T <= 4 ? launch_fused_nt<4, BITS>(m, a, s)
                    : launch_fused_nt<8, BITS>(m, a, s);
}

}  // namespace

cudaError_t decode_fused_init() {
    cudaError_t e;
    if ((e = fused_attr<1, 0>()) || (e = fused_attr<2, 0>()) || (e = fused_attr<4, 0>()) ||
        (e = fused_attr<8, 0>()) || (e = fused_attr<1, 4>()) || (e = fused_attr<2, 4>()) ||
        (e = fused_attr<4, 4>()) || (e = fused_attr<8, 4>()) || (e = fused_attr<1, 8>()) ||
        (e = fused_attr<2, 8>()) || (e = fused_attr<4, 8>()) || (e = fused_attr<8, 8>()))
        return e;
    return cudaSuccess;
}

bool decode_fused_supported(int T, int H, int I, int E, int K, bool same_x, int bits, int gs) {
    if (T < 1 || T > kMaxT) return false;
    if (bits != 0 && !((bits == 4 || bits == 8) && gs == 64)) return false;
    const size_t ring = bits == 0 ? ring_T<0>(T) : bits == 4 ? ring_T<4>(T) : ring_T<8>(T);
    // 4-bit: at least two whole-item slots (one in use, one filling)
    if (bits == 4 && ring / ((q4_slot_bytes(H, I) + 127) & ~size_t(127)) < 2) return false;
    const size_t smem = bits == 0 ? fused_smem_T<0>(T, H, I)
                        : bits == 4 ? fused_smem_T<4>(T, H, I) : fused_smem_T<8>(T, H, I);
    const size_t router = (same_x ? 0 : (size_t)T * H * 2) + (size_t)H * 4 +
                          (size_t)(E + 7) / 8 * 16 + (size_t)T * E * 4;
    return T * K <= kMaxPairs && K <= 32 && E <= kEpMaxExperts && E % 8 == 0 &&
           E <= grid_sms(current_device()) && grid_sms(current_device()) <= kMaxGrid &&
           router <= ring && H % 256 == 0 && H % kDnRows == 0 && I % 64 == 0 &&
           I % kGuCols == 0 && smem <= kMaxDynSmem && encode_tiled_fn() != nullptr;
}

size_t decode_fused_sync_words(int E, int H, int I) {
    (void)E;
    return kTagWord + 2 * (size_t)kMaxPairs * (size_t)(I + H) / 2;
}

cudaError_t launch_decode_fused(const uint16_t *xr, const uint16_t *xe, const uint16_t *proj,
                                const uint16_t *scale, const uint16_t *pes, int T, int H, int E,
                                int K, int I, float eps, float *scores, int32_t *idx, uint16_t *w,
                                const Dispatch &d, const ExpertWeights &wt, uint16_t *out,
                                int32_t *sync, int32_t *err, cudaStream_t s, int *launches) {
    unsigned long long *yq = reinterpret_cast<unsigned long long *>(sync + kTagWord);
    unsigned long long *oq = yq + (size_t)kMaxPairs * (I / 2);
    CUtensorMap m[4];
    const int bits = wt.bits;
    if (bits == 0) {
        if (!bf16_map_2d(&m[0], wt.gu, H, (uint64_t)E * 2 * I, 256, kGuCols, false) ||
            !bf16_map_2d(&m[1], wt.dn, I, (uint64_t)E * H, 64, kDnRows, false))
            return cudaErrorInvalidValue;
        m[2] = m[0];  // unused
        m[3] = m[1];
    } else {
        // packed codes [rows][len * bits / 32] u32 and (scale, bias) words
        // [rows][gp], gp = groups rounded up to 4
        const int gpH = ((H / 64) + 3) / 4 * 4, gpI = ((I / 64) + 3) / 4 * 4;
        if (!map_2d(&m[0], wt.gu_q, (uint64_t)H * bits / 32, (uint64_t)E * 2 * I, 256 * bits / 32,
                    kGuCols, false, true) ||
            !map_2d(&m[1], wt.dn_q, (uint64_t)I * bits / 32, (uint64_t)E * H, 64 * bits / 32,
                    kDnRows, false, true) ||
            !map_2d(&m[2], wt.gu_sb, gpH, (uint64_t)E * 2 * I, gpH, kGuCols, false, true) ||
            !map_2d(&m[3], wt.dn_sb, gpI, (uint64_t)E * H, gpI, kDnRows, false, true))
            return cudaErrorInvalidValue;
    }
    FusedArgs a{xr, xe, scale, pes, proj, T, H, E, K, I, eps, (float)(1.0 / sqrt((double)H)),
                scores, idx, w, d, yq, oq, out, sync, err,
                bits == 4 ? wt.gu_qd : wt.gu_q, bits == 4 ? wt.dn_qd : wt.dn_q, wt.gu_sb,
                wt.dn_sb};
    const cudaError_t e = bits == 0   ? launch_bits<0>(m, a, s)
                          : bits == 4 ? launch_bits<4>(m, a, s)
                                      : launch_bits<8>(m, a, s);
    if (launches) ++*launches;
    return e;
}

}  // namespace apt

#ifdef APT_FUSED_TRACE
extern "C" int apt_fused_trace_read(unsigned long long *host) {
    return (int)cudaMemcpyFromSymbol(host, apt::g_ftrace, sizeof(apt::g_ftrace));
}
extern "C" int apt_fused_itrace_read(unsigned long long *host) {
    return (int)cudaMemcpyFromSymbol(host, apt::g_itrace, sizeof(apt::g_itrace));
}
#endif
