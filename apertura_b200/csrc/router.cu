// router.cu -- ESRouter::routeTopK / routeWeights on sm_100a.
//
// Restates aptransformer/ESRouter.mm:14-40:
//   xf = f32(x); ms = mean(xf^2); h = xf * rsqrt(ms + eps)
//   h  = (h * f32(scale)) * H^-1/2                       (each product rounded in f32)
//   scores = h . f32(proj)^T                             (f32 accumulate)
//   probs  = softmax(scores) (max-subtracted, f32)
//   idx    = argsort(-probs)[:K]   (descending; lower expert id first on exact ties)
//   w      = probs[idx] / sum(probs[idx]) * f32(per_expert_scale[idx]) -> bf16
//
// Two score kernels: a warp-per-expert kernel for decode-sized T (every CTA
// streams a few proj rows once, all 128 experts spread over 32 CTAs) and a
// register-tiled f32 kernel for prefill-sized T (proj and x tiles reused from
// shared memory).  The selection kernel runs one warp per token.
#include "common.cuh"
#include "launch_util.h"
#include "moe_internal.h"
#include "router_select.cuh"
#include "sm100_ptx.cuh"

namespace apt {

namespace {

constexpr int kSmallTok = 8;     // tokens staged per CTA in the decode kernel
constexpr int kSmallWarps = 4;   // experts per CTA in the decode kernel
constexpr int kSmallThreads = 256;  // 8 warps per decode router CTA

// Phase timestamps (%globaltimer, thread 0 of each CTA) for tuning builds
// compiled with -DAPT_ROUTER_TRACE; absent from the library build.
#ifdef APT_ROUTER_TRACE
__device__ unsigned long long g_rtrace[1024][12];
__device__ long long g_rclock[1024][12];
#define RT_STAMP(i)                                                                    \
    do {                                                                               \
        if (threadIdx.x == 0) {                                                        \
            unsigned long long t_;                                                     \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                     \
            g_rtrace[blockIdx.y * gridDim.x + blockIdx.x][i] = t_;                     \
            g_rclock[blockIdx.y * gridDim.x + blockIdx.x][i] = clock64();              \
        }                                                                              \
    } while (0)
#else
#define RT_STAMP(i) \
    do {            \
    } while (0)
#endif

// r_t = 1/sqrt(mean(x_t^2) + eps) for one token, computed by one warp.
__device__ __forceinline__ float token_rrms(const uint16_t *xr, int H, float eps, int lane) {
    float s = 0.f;
    for (int i = lane * 8; i < H; i += 256) {
        uint4 v = *reinterpret_cast<const uint4 *>(xr + i);
        float f[8];
        unpack8(v, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) s = fmaf(f[j], f[j], s);
    }
    s = warp_sum(s);
    float ms = __fmul_rn(s, 1.0f / (float)H);
    return 1.0f / sqrtf(__fadd_rn(ms, eps));
}


// Scores of experts [blockIdx.x*4, +4) for tokens [blockIdx.y*8, +8).  The
// chunk's token rows, the CTA's 4 proj rows and the scale vector arrive in
// shared memory by bulk copies issued at entry (one memory round trip).  Each
// thread then owns 8-element slices of the hidden axis: it reads every staged
// row once (16-byte, conflict-free), forms h = ((x r) scale) root for the
// chunk's tokens in registers and keeps all 4 x 8 partial dot products; a warp
// sum and a sum over the 8 warps finish them.  Shared-memory reads are one
// pass over 13 rows, where a warp-per-(expert, token-group) mapping re-reads
// every staged h row once per expert.
// Dynamic shared memory: (min(T, 8) + kSmallWarps + 1) rows of H bf16.
constexpr int kMaxVec = 12;  // H <= 12 * 256
constexpr long long kRouterWaitLimit = 4000000000LL;

__host__ __device__ constexpr size_t scores_small_smem(int T, int H) {
    return (size_t)((T < kSmallTok ? T : kSmallTok) + kSmallWarps + 1) * H * 2;
}

__device__ __forceinline__ void scores_small_block(const uint16_t *__restrict__ x,
                                                   const uint16_t *__restrict__ proj,
                                                   const uint16_t *__restrict__ scale, int T,
                                                   int H, int E, float eps, float root,
                                                   float *__restrict__ scores, uint16_t *sm,
                                                   const uint16_t *__restrict__ pre_w = nullptr,
                                                   uint16_t *__restrict__ xn = nullptr,
                                                   int32_t *__restrict__ err = nullptr) {
    __shared__ __align__(8) uint64_t s_bar;
    __shared__ float s_part[kSmallThreads / 32][kSmallWarps * kSmallTok];
    __shared__ float s_r[kSmallTok];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * kSmallWarps;
    const int ne = min(kSmallWarps, E - e0);
    const int t0 = blockIdx.y * kSmallTok;
    const int nt = min(kSmallTok, T - t0);
    const int nts = min(T, kSmallTok);  // staged token rows
    uint16_t *s_x = sm;                      // [nts][H]
    uint16_t *s_p = sm + (size_t)nts * H;    // [kSmallWarps][H]
    uint16_t *s_scale = s_p + (size_t)kSmallWarps * H;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&s_bar, 1);
        sm100::fence_barrier_init();
        const uint32_t row_bytes = (uint32_t)H * 2;
        sm100::mbar_arrive_expect_tx(&s_bar, (uint32_t)(nt + ne + 1) * row_bytes);
        sm100::bulk_load(s_scale, scale, row_bytes, &s_bar);
        sm100::bulk_load(s_p, proj + (size_t)e0 * H, (uint32_t)ne * row_bytes, &s_bar);
        sm100::bulk_load(s_x, x + (size_t)t0 * H, (uint32_t)nt * row_bytes, &s_bar);
    }
    __syncthreads();  // barrier initialised
    if (!sm100::mbar_wait(&s_bar, 0, kRouterWaitLimit) && err && threadIdx.x == 0)
        atomicCAS(err, 0, 30);  // rows never arrived: the scores of this call are invalid
    RT_STAMP(7);
    const int nch = H / 8;  // 8-element slices
    // r_t = 1/sqrt(mean(x_t^2) + eps): warp w sums token w
    if (warp < nt) {
        float ss = 0.f;
        for (int c = lane; c < nch; c += 32) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4 *>(s_x + (size_t)warp * H + c * 8), f);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) s_r[warp] = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)H), eps));
    }
    __syncthreads();
    float acc[kSmallWarps][kSmallTok];
#pragma unroll
    for (int q = 0; q < kSmallWarps; ++q)
#pragma unroll
        for (int t = 0; t < kSmallTok; ++t) acc[q][t] = 0.f;
    const bool wxn = xn && blockIdx.x == 0;  // pre_ff_ln_2(x1), once per token
    for (int c = threadIdx.x; c < nch; c += blockDim.x) {
        float sf[8], p[kSmallWarps][8];
        unpack8(*reinterpret_cast<const uint4 *>(s_scale + c * 8), sf);
#pragma unroll
        for (int q = 0; q < kSmallWarps; ++q)
            if (q < ne) unpack8(*reinterpret_cast<const uint4 *>(s_p + (size_t)q * H + c * 8), p[q]);
#pragma unroll
        for (int t = 0; t < kSmallTok; ++t) {
            if (t >= nt) break;
            float f[8], hv[8];
            unpack8(*reinterpret_cast<const uint4 *>(s_x + (size_t)t * H + c * 8), f);
            const float r = s_r[t];
#pragma unroll
            for (int j = 0; j < 8; ++j) hv[j] = router_h(f[j], r, sf[j], root);
#pragma unroll
            for (int q = 0; q < kSmallWarps; ++q)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[q][t] = fmaf(p[q][j], hv[j], acc[q][t]);
            if (wxn) {
                float wf[8];
                unpack8(__ldg(reinterpret_cast<const uint4 *>(pre_w + c * 8)), wf);
                uint4 o;
                o.x = pack_bf2(__fmul_rn(__fmul_rn(f[0], r), wf[0]), __fmul_rn(__fmul_rn(f[1], r), wf[1]));
                o.y = pack_bf2(__fmul_rn(__fmul_rn(f[2], r), wf[2]), __fmul_rn(__fmul_rn(f[3], r), wf[3]));
                o.z = pack_bf2(__fmul_rn(__fmul_rn(f[4], r), wf[4]), __fmul_rn(__fmul_rn(f[5], r), wf[5]));
                o.w = pack_bf2(__fmul_rn(__fmul_rn(f[6], r), wf[6]), __fmul_rn(__fmul_rn(f[7], r), wf[7]));
                *reinterpret_cast<uint4 *>(xn + (size_t)(t0 + t) * H + c * 8) = o;
            }
        }
    }
    // sum the partials: over the warp's lanes, then over the 8 warps
#pragma unroll
    for (int q = 0; q < kSmallWarps; ++q)
#pragma unroll
        for (int t = 0; t < kSmallTok; ++t) {
            const float v = warp_sum(acc[q][t]);
            if (lane == 0) s_part[warp][q * kSmallTok + t] = v;
        }
    __syncthreads();
    if (threadIdx.x < kSmallWarps * kSmallTok) {
        const int q = threadIdx.x / kSmallTok, t = threadIdx.x % kSmallTok;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kSmallThreads / 32; ++w) v += s_part[w][threadIdx.x];
        if (q < ne && t < nt) scores[(size_t)(t0 + t) * E + e0 + q] = v;
    }
}

__global__ void __launch_bounds__(kSmallThreads)
router_scores_small(const uint16_t *__restrict__ x, const uint16_t *__restrict__ proj,
                    const uint16_t *__restrict__ scale, int T, int H, int E, float eps,
                    float root, float *__restrict__ scores, int32_t *__restrict__ err) {
    extern __shared__ __align__(16) uint16_t rs_smem[];
    scores_small_block(x, proj, scale, T, H, E, eps, root, scores, rs_smem, nullptr, nullptr, err);
}

// Register-tiled f32 GEMM: CTA = 64 tokens x 64 experts, 256 threads, each
// thread a 4x4 micro-tile, K staged in chunks of 32.
constexpr int kTT = 64, kEB = 64, kKC = 32;

__global__ void __launch_bounds__(256)
router_scores_tiled(const uint16_t *__restrict__ x, const uint16_t *__restrict__ proj,
                    const uint16_t *__restrict__ scale, int T, int H, int E, float eps,
                    float root, float *__restrict__ scores) {
    __shared__ float As[kKC][kTT + 4];
    __shared__ float Bs[kKC][kEB + 4];
    __shared__ float rs[kTT];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.y * kTT, e0 = blockIdx.x * kEB;
    for (int t = warp; t < kTT; t += 8) {
        float r = 0.f;
        if (t0 + t < T) r = token_rrms(x + (size_t)(t0 + t) * H, H, eps, lane);
        if (lane == 0) rs[t] = r;
    }
    __syncthreads();
    const int ty = tid / 16, tx = tid % 16;  // 16 x 16 threads, 4x4 each
    float acc[4][4] = {};
    for (int k0 = 0; k0 < H; k0 += kKC) {
        // stage A: 64 tokens x 32 k (as 64*4 vectors of 8) and B: 64 experts x 32 k
        {
            const int row = tid / 4, kv = (tid % 4) * 8;
            float f[8], sf[8];
            const int t = t0 + row;
            if (t < T) {
                unpack8(*reinterpret_cast<const uint4 *>(x + (size_t)t * H + k0 + kv), f);
                unpack8(*reinterpret_cast<const uint4 *>(scale + k0 + kv), sf);
#pragma unroll
                for (int j = 0; j < 8; ++j) As[kv + j][row] = router_h(f[j], rs[row], sf[j], root);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) As[kv + j][row] = 0.f;
            }
            const int e = e0 + row;
            if (e < E) {
                unpack8(*reinterpret_cast<const uint4 *>(proj + (size_t)e * H + k0 + kv), f);
#pragma unroll
                for (int j = 0; j < 8; ++j) Bs[kv + j][row] = f[j];
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) Bs[kv + j][row] = 0.f;
            }
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kKC; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + tx * 4 + j;
            if (e < E) scores[(size_t)t * E + e] = acc[i][j];
        }
    }
}

// Softmax, top-K (descending prob, lower id on ties), renormalise and
// per-expert scale for one token, by one warp.  Lanes k < K return the k-th
// choice in (sel_e, wk); other lanes return sel_e = -1.
// One token's scores row into p (lane + 32 j), -inf past E.
template <int NP>
__device__ __forceinline__ void load_scores(const float *__restrict__ sr, int E, int lane,
                                            float (&p)[NP]) {
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? __ldcg(sr + e) : -INFINITY;  // written by other CTAs
    }
}

// sr2 (optional): a second partial-score row added to sr's; rs: per-token
// factor applied to the (summed) scores -- the RMS factor when the scores
// were computed from the un-normalised token row.
template <int NP>
__device__ __forceinline__ void select_token(const float *__restrict__ sr,
                                             const uint16_t *__restrict__ pes, int E, int K,
                                             int lane, int &sel_e_out, float &wk_out,
                                             const float *__restrict__ sr2 = nullptr,
                                             float rs = 1.f) {
    float p[NP];
    load_scores<NP>(sr, E, lane, p);
    if (sr2) {
        float p2[NP];
        load_scores<NP>(sr2, E, lane, p2);
#pragma unroll
        for (int j = 0; j < NP; ++j) p[j] = __fmul_rn(__fadd_rn(p[j], p2[j]), rs);
    }
    int sel_e;
    float sel_p, sum;
    select_core<NP>(p, E, K, lane, sel_e, sel_p, sum);
    wk_out = 0.f;
    sel_e_out = -1;
    if (lane < K) {
        wk_out = __fmul_rn(__fdiv_rn(sel_p, sum), bf2f(pes[sel_e]));
        sel_e_out = sel_e;
    }
}

// One warp per token.  Slots in the experts' groups are claimed per block:
// shared-memory atomics give each pair its place among the block's pairs of
// the same expert, then one global atomic per (block, expert) reserves the
// block's range -- under skewed routing most pairs go to a few experts, and
// one global atomic per pair would serialise on those counters.
constexpr int kSelectWarps = 32;

template <int NP>
__global__ void __launch_bounds__(kSelectWarps * 32)
router_select(const float *__restrict__ scores, const uint16_t *__restrict__ pes, int T, int E,
              int K, int32_t *__restrict__ idx, uint16_t *__restrict__ w,
              int32_t *__restrict__ counts, int32_t *__restrict__ rank,
              const int32_t *__restrict__ err, const uint16_t *__restrict__ xr, int H,
              float eps) {
    __shared__ int s_cnt[kMaxPerLane * 32];
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    pdl_trigger();
    pdl_wait();
    // xr: the scores are two planes [2][T][E] of partial x . (scale * H^-1/2
    // * proj) of the raw token rows; they are summed and the RMS factor
    // r = 1 / sqrt(mean(x^2) + eps) of ESRouter.mm:18-20 is applied here
    float rs = 1.f;
    if (xr && warp < T) {
        const uint16_t *row = xr + (size_t)warp * H;
        float ss = 0.f;
        for (int i = lane * 8; i < H; i += 256) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4 *>(row + i), f);
#pragma unroll
            for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
        }
        ss = warp_sum(ss);
        rs = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)H), eps));
    }
    int e = -1, local = 0;
    float wk = 0.f;
    if (err && __ldcg(err) != 0) {  // the scores of this call never arrived: mark it invalid
        if (warp < T && lane < K) {
            idx[(size_t)warp * K + lane] = -1;
            w[(size_t)warp * K + lane] = 0;
        }
        return;
    }
    if (warp < T) {
        select_token<NP>(scores + (size_t)warp * E, pes, E, K, lane, e, wk,
                         xr ? scores + ((size_t)T + warp) * E : nullptr, rs);
        if (lane < K) {
            idx[(size_t)warp * K + lane] = e;
            w[(size_t)warp * K + lane] = f2bf(wk);
        }
    }
    if (!counts) return;  // uniform over the block
    __syncthreads();  // s_cnt zeroed
    if (e >= 0) local = atomicAdd(&s_cnt[e], 1);
    __syncthreads();
    for (int x = threadIdx.x; x < E; x += blockDim.x) {
        const int c = s_cnt[x];
        s_cnt[x] = c > 0 ? atomicAdd(counts + x, c) : 0;  // base of this block's range
    }
    __syncthreads();
    if (e >= 0 && rank) rank[(size_t)warp * K + lane] = s_cnt[e] + local;
}

// Decode-sized fused routing: the scores of router_scores_small; the last CTA
// of each 8-token chunk (threadfence + per-chunk counter) selects the top-K of
// the chunk's tokens, one warp per token; the last chunk to finish builds the
// whole dispatch -- counts, offsets, active-expert list and the stable sorted
// order -- in shared memory.  Counters live in `done` ([0] chunks, [1+c] CTAs
// of chunk c) and are reset by the kernel itself.
// Requires T <= 64, T*K <= kFusedMaxPairs, E <= 256.
constexpr int kFusedMaxPairs = 512;


__global__ void __launch_bounds__(kSmallThreads, 2)
router_dispatch_small(const uint16_t *__restrict__ x, const uint16_t *__restrict__ proj,
                      const uint16_t *__restrict__ scale, const uint16_t *__restrict__ pes, int T,
                      int H, int E, int K, float eps, float root, float *__restrict__ scores,
                      int32_t *__restrict__ idx, uint16_t *__restrict__ w, Dispatch d,
                      int32_t *__restrict__ done, const uint16_t *__restrict__ pre_w,
                      uint16_t *__restrict__ xn, int32_t *__restrict__ err) {
    extern __shared__ __align__(16) uint16_t rs_smem[];
    __shared__ int s_last;
    __shared__ int s_idx[kFusedMaxPairs];
    __shared__ int s_cnt[256];
    __shared__ int s_off[257];
    __shared__ float s_pes[256];
    RT_STAMP(0);
    pdl_trigger();
    pdl_wait();  // launched early behind the stream's previous kernel; x may be its output
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // per_expert_scale for the select phase, fetched while the scores run
    for (int e = tid; e < E; e += blockDim.x) s_pes[e] = bf2f(pes[e]);
    scores_small_block(x, proj, scale, T, H, E, eps, root, scores, rs_smem, pre_w, xn, err);
    RT_STAMP(1);
    // level 1: the last CTA of this token chunk selects the chunk's tokens
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(done + 1 + blockIdx.y, 1);
        s_last = (prev == (int)gridDim.x - 1);
    }
    __syncthreads();
    RT_STAMP(2);
    if (!s_last) return;
    __threadfence();
    const bool single = gridDim.y == 1;  // one chunk: this CTA also builds the dispatch
    {
        const int t = blockIdx.y * kSmallTok + warp;  // 8 warps, 8 tokens per chunk
        if (t < T) {
            int e;
            float sel_p, sum;
            if (E <= 128) {
                float p[4];
                load_scores<4>(scores + (size_t)t * E, E, lane, p);
                select_core<4>(p, E, K, lane, e, sel_p, sum);
            } else {
                float p[kMaxPerLane];
                load_scores<kMaxPerLane>(scores + (size_t)t * E, E, lane, p);
                select_core<kMaxPerLane>(p, E, K, lane, e, sel_p, sum);
            }
            if (lane < K) {
                idx[(size_t)t * K + lane] = e;
                w[(size_t)t * K + lane] = f2bf(__fmul_rn(__fdiv_rn(sel_p, sum), s_pes[e]));
                if (single) s_idx[t * K + lane] = e;
            }
        }
    }
    RT_STAMP(3);
    if (tid == 0) done[1 + blockIdx.y] = 0;  // ready for the next call
    if (!single) {
        // level 2: the last chunk builds the dispatch for all tokens
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const int prev = atomicAdd(done, 1);
            s_last = (prev == (int)gridDim.y - 1);
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
    }
    RT_STAMP(4);
    for (int e = tid; e < E; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    const int P = T * K;
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = single ? s_idx[p] : __ldcg(idx + p);  // else written by other CTAs
        s_idx[p] = e;
        atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the counts, 8 experts per lane
        int loc[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane * 8 + j;
            loc[j] = (e < E) ? s_cnt[e] : 0;
            sum += loc[j];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - sum;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane * 8 + j;
            if (e < E) {
                s_off[e] = run;
                d.counts[e] = loc[j];
                d.offsets[e] = run;
            }
            run += loc[j];
        }
        if (lane == 31) d.offsets[E] = incl;
        // active list: experts with nonzero count, ascending
        int na = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const bool act = e < E && s_cnt[e] > 0;
            const unsigned m = __ballot_sync(0xffffffffu, act);
            if (act) d.active[na + __popc(m & ((1u << lane) - 1u))] = e;
            na += __popc(m);
        }
        if (lane == 0) {
            *d.n_active = na;
            if (!single) *done = 0;  // ready for the next call
        }
    }
    __syncthreads();
    RT_STAMP(5);
    // placement: each pair claims the next slot of its expert's group.  The
    // order inside a group is arbitrary; every row is computed independently
    // and found again through inv, so results do not depend on it.
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = s_idx[p];
        const int pos = atomicAdd(&s_off[e], 1);
        d.perm[pos] = p;
        d.inv[p] = pos;
    }
    RT_STAMP(6);
}

// Router weights for the tensor-core score GEMM, folded once at load:
// w = (scale[h] * H^-1/2) * proj[e, h] in f32, stored as the two-term bf16
// split pw[e] = (w1 | w2) [E, 2H], w1 = bf16(w), w2 = bf16(w - w1), so that
// x . w1 + x . w2 reproduces x . w to ~2^-17 relative per term (x is bf16,
// the products are exact, the accumulation f32).
__global__ void router_fold_split(const uint16_t *__restrict__ proj,
                                  const uint16_t *__restrict__ scale, int H, int E, float root,
                                  uint16_t *__restrict__ pw) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)E * H) return;
    const size_t e = i / H, c = i - e * H;
    const float wv = __fmul_rn(__fmul_rn(bf2f(scale[c]), root), bf2f(proj[i]));
    const float w1 = rbf(wv);
    pw[e * 2 * H + c] = f2bf(w1);
    pw[e * 2 * H + H + c] = f2bf(__fsub_rn(wv, w1));
}

// Standalone RMSNorm with weight (ESRMSNorm.mm:14-28), one warp per row.
__global__ void rmsnorm_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ wgt,
                               int T, int H, float eps, uint16_t *__restrict__ out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    pdl_wait();
    if (warp >= T) return;
    const uint16_t *xr = x + (size_t)warp * H;
    float ss = 0.f;
    for (int i = lane * 8; i < H; i += 256) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4 *>(xr + i), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)H), eps));
    for (int i = lane * 8; i < H; i += 256) {
        float f[8], wf[8], o[8];
        unpack8(*reinterpret_cast<const uint4 *>(xr + i), f);
        unpack8(*reinterpret_cast<const uint4 *>(wgt + i), wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(__fmul_rn(f[j], r), wf[j]);
        uint4 v;
        v.x = pack_bf2(o[0], o[1]); v.y = pack_bf2(o[2], o[3]);
        v.z = pack_bf2(o[4], o[5]); v.w = pack_bf2(o[6], o[7]);
        *reinterpret_cast<uint4 *>(out + (size_t)warp * H + i) = v;
    }
}

__global__ void scatter_dense(const int32_t *__restrict__ idx, const uint16_t *__restrict__ w,
                              int T, int E, int K, uint16_t *__restrict__ W) {
    const int t = blockIdx.x;
    for (int e = threadIdx.x; e < E; e += blockDim.x) W[(size_t)t * E + e] = 0;
    __syncthreads();
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int e = idx[(size_t)t * K + k];
        if (e >= 0 && e < E) W[(size_t)t * E + e] = w[(size_t)t * K + k];
    }
}

// Dense W -> per-token pair list in expert order; zero weights are skipped
// (they contribute exactly zero to ESExperts::forward's sum).
__global__ void dense_to_pairs(const uint16_t *__restrict__ W, int T, int E,
                               int32_t *__restrict__ idx2, uint16_t *__restrict__ w2,
                               int32_t *__restrict__ counts) {
    const int t = blockIdx.x;
    if (threadIdx.x != 0) return;
    int n = 0;
    for (int e = 0; e < E; ++e) {
        const uint16_t v = W[(size_t)t * E + e];
        if ((v & 0x7fff) != 0) {
            idx2[(size_t)t * E + n] = e;
            w2[(size_t)t * E + n] = v;
            ++n;
            atomicAdd(counts + e, 1);
        }
    }
    for (int k = n; k < E; ++k) {
        idx2[(size_t)t * E + k] = -1;
        w2[(size_t)t * E + k] = 0;
    }
}

}  // namespace

cudaError_t router_init() {
    cudaError_t e = cudaFuncSetAttribute(router_scores_small,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e) return e;
    return cudaFuncSetAttribute(router_dispatch_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
}

bool router_dispatch_fusable(int T, int H, int E, int K) {
    return T >= 1 && T <= 64 && T * K <= kFusedMaxPairs && E <= 256 && H % 256 == 0 &&
           H <= 256 * kMaxVec;
}

cudaError_t launch_router_dispatch(const uint16_t *x, const uint16_t *proj, const uint16_t *scale,
                                   const uint16_t *pes, int T, int H, int E, int K, float eps,
                                   float *scores, int32_t *idx, uint16_t *w, const Dispatch &d,
                                   int32_t *done, cudaStream_t s, int *launches,
                                   const uint16_t *pre_w, uint16_t *xn, int32_t *err) {
    const float root = (float)(1.0 / sqrt((double)H));
    const size_t smem = scores_small_smem(T, H);
    dim3 grid((E + kSmallWarps - 1) / kSmallWarps, (T + kSmallTok - 1) / kSmallTok);
    cudaError_t r = launch_ex(router_dispatch_small, grid, dim3(kSmallThreads), smem, s, true,
                              x, proj, scale, pes, T, H, E, K, eps, root, scores, idx, w, d,
                              done, pre_w, xn, err);
    if (launches) ++*launches;
    return r;
}

cudaError_t launch_router_scores(const uint16_t *x, const uint16_t *proj, const uint16_t *scale,
                                 int T, int H, int E, float eps, float *scores, cudaStream_t s,
                                 int *launches, int32_t *err) {
    const float root = (float)(1.0 / sqrt((double)H));
    if (T <= 64 && H % 256 == 0 && H <= 256 * kMaxVec) {
        const size_t smem = scores_small_smem(T, H);
        dim3 grid((E + kSmallWarps - 1) / kSmallWarps, (T + kSmallTok - 1) / kSmallTok);
        router_scores_small<<<grid, kSmallThreads, smem, s>>>(x, proj, scale, T, H, E, eps,
                                                                 root, scores, err);
    } else {
        dim3 grid((E + kEB - 1) / kEB, (T + kTT - 1) / kTT);
        router_scores_tiled<<<grid, 256, 0, s>>>(x, proj, scale, T, H, E, eps, root, scores);
    }
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *w, int T, int H, float eps,
                          uint16_t *out, cudaStream_t s, int *launches) {
    const int wpb = 8;
    cudaError_t err = launch_ex(rmsnorm_kernel, dim3((T + wpb - 1) / wpb), dim3(wpb * 32), 0, s,
                                true, x, w, T, H, eps, out);
    if (launches) ++*launches;
    return err;
}

cudaError_t launch_router_fold_split(const uint16_t *proj, const uint16_t *scale, int H, int E,
                                     uint16_t *pw, cudaStream_t s) {
    const float root = (float)(1.0 / sqrt((double)H));
    const size_t n = (size_t)E * H;
    router_fold_split<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(proj, scale, H, E, root, pw);
    return cudaGetLastError();
}

cudaError_t launch_router_select(const float *scores, const uint16_t *pes, int T, int E, int K,
                                 int32_t *idx, uint16_t *w, int32_t *counts, cudaStream_t s,
                                 int *launches, int32_t *rank, const int32_t *err,
                                 const uint16_t *x, int H, float eps) {
    dim3 grid((T + kSelectWarps - 1) / kSelectWarps);
    cudaError_t r = launch_ex(E <= 128 ? router_select<4> : router_select<kMaxPerLane>, grid,
                              dim3(kSelectWarps * 32), 0, s, true,
                              (const float *)scores, pes, T, E, K, idx, w, counts, rank, err,
                              x, H, eps);
    if (launches) ++*launches;
    return r;
}

cudaError_t launch_scatter_dense(const int32_t *idx, const uint16_t *w, int T, int E, int K,
                                 uint16_t *W, cudaStream_t s, int *launches) {
    scatter_dense<<<T, 128, 0, s>>>(idx, w, T, E, K, W);
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_dense_to_pairs(const uint16_t *W, int T, int E, int32_t *idx2, uint16_t *w2,
                                  int32_t *counts, cudaStream_t s, int *launches) {
    dense_to_pairs<<<T, 32, 0, s>>>(W, T, E, idx2, w2, counts);
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace apt
