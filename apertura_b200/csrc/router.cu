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
#include "moe_internal.h"

namespace apt {

namespace {

constexpr int kSmallTok = 8;     // tokens staged per CTA in the decode kernel
constexpr int kSmallWarps = 4;   // experts per CTA in the decode kernel

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

// h = ((x * r) * scale) * root, element-wise, f32 rounding at every step.
__device__ __forceinline__ float router_h(float x, float r, float sc, float root) {
    return __fmul_rn(__fmul_rn(__fmul_rn(x, r), sc), root);
}

__global__ void __launch_bounds__(kSmallWarps * 32)
router_scores_small(const uint16_t *__restrict__ x, const uint16_t *__restrict__ proj,
                    const uint16_t *__restrict__ scale, int T, int H, int E, float eps,
                    float root, float *__restrict__ scores) {
    extern __shared__ float hs[];  // [kSmallTok][H]
    __shared__ float rs[kSmallTok];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kSmallWarps + warp;
    const uint16_t *pr = proj + (size_t)(e < E ? e : 0) * H;
    for (int t0 = 0; t0 < T; t0 += kSmallTok) {
        const int nt = min(kSmallTok, T - t0);
        for (int t = warp; t < nt; t += kSmallWarps)
            {
                float r = token_rrms(x + (size_t)(t0 + t) * H, H, eps, lane);
                if (lane == 0) rs[t] = r;
            }
        __syncthreads();
        const int vecs = H / 8;
        for (int v = threadIdx.x; v < nt * vecs; v += blockDim.x) {
            const int t = v / vecs, i = (v - t * vecs) * 8;
            uint4 xv = *reinterpret_cast<const uint4 *>(x + (size_t)(t0 + t) * H + i);
            uint4 sv = *reinterpret_cast<const uint4 *>(scale + i);
            float xf[8], sf[8];
            unpack8(xv, xf);
            unpack8(sv, sf);
            float *dst = hs + t * H + i;
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = router_h(xf[j], rs[t], sf[j], root);
        }
        __syncthreads();
        if (e < E) {
            float acc[kSmallTok];
#pragma unroll
            for (int t = 0; t < kSmallTok; ++t) acc[t] = 0.f;
            for (int i = lane * 8; i < H; i += 256) {
                float p[8];
                unpack8(*reinterpret_cast<const uint4 *>(pr + i), p);
#pragma unroll
                for (int t = 0; t < kSmallTok; ++t) {
                    if (t < nt) {
                        const float4 a = *reinterpret_cast<const float4 *>(hs + t * H + i);
                        const float4 b = *reinterpret_cast<const float4 *>(hs + t * H + i + 4);
                        acc[t] = fmaf(p[0], a.x, acc[t]);
                        acc[t] = fmaf(p[1], a.y, acc[t]);
                        acc[t] = fmaf(p[2], a.z, acc[t]);
                        acc[t] = fmaf(p[3], a.w, acc[t]);
                        acc[t] = fmaf(p[4], b.x, acc[t]);
                        acc[t] = fmaf(p[5], b.y, acc[t]);
                        acc[t] = fmaf(p[6], b.z, acc[t]);
                        acc[t] = fmaf(p[7], b.w, acc[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < kSmallTok; ++t) {
                float s = warp_sum(acc[t]);
                if (lane == 0 && t < nt) scores[(size_t)(t0 + t) * E + e] = s;
            }
        }
        __syncthreads();
    }
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

constexpr int kMaxPerLane = 8;  // E <= 256

// One warp per token: softmax, top-K (descending prob, lower id on ties),
// renormalise, per-expert scale, bf16.
__global__ void router_select(const float *__restrict__ scores, const uint16_t *__restrict__ pes,
                              int T, int E, int K, int32_t *__restrict__ idx,
                              uint16_t *__restrict__ w, int32_t *__restrict__ counts) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float *sr = scores + (size_t)warp * E;
    float p[kMaxPerLane];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? sr[e] : -INFINITY;
        m = fmaxf(m, p[j]);
    }
    m = warp_max(m);
    float den = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? expf(__fsub_rn(p[j], m)) : 0.f;
        den += p[j];
    }
    den = warp_sum(den);
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? __fdiv_rn(p[j], den) : -1.f;  // -1: never selected
    }
    float sum = 0.f;
    float sel_p = 0.f;
    int sel_e = 0;
    unsigned taken = 0;
    for (int k = 0; k < K; ++k) {
        // lane-local best among untaken
        float bp = -2.f;
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kMaxPerLane; ++j) {
            const int e = lane + 32 * j;
            if (!((taken >> j) & 1u) && (p[j] > bp)) {
                bp = p[j];
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xffffffffu, bp, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (op > bp || (op == bp && oe < be)) {
                bp = op;
                be = oe;
            }
        }
        if ((be & 31) == lane) taken |= 1u << (be >> 5);
        sum = __fadd_rn(sum, bp);  // sequential in k order, every lane the same
        if (lane == k) {
            sel_p = bp;
            sel_e = be;
        }
    }
    if (lane < K) {
        float wk = __fdiv_rn(sel_p, sum);
        wk = __fmul_rn(wk, bf2f(pes[sel_e]));
        idx[(size_t)warp * K + lane] = sel_e;
        w[(size_t)warp * K + lane] = f2bf(wk);
        if (counts) atomicAdd(counts + sel_e, 1);
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
    return cudaFuncSetAttribute(router_scores_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
}

cudaError_t launch_router_scores(const uint16_t *x, const uint16_t *proj, const uint16_t *scale,
                                 int T, int H, int E, float eps, float *scores, cudaStream_t s,
                                 int *launches) {
    const float root = (float)(1.0 / sqrt((double)H));
    if (T <= 64) {
        const size_t smem = (size_t)kSmallTok * H * sizeof(float);
        dim3 grid((E + kSmallWarps - 1) / kSmallWarps);
        router_scores_small<<<grid, kSmallWarps * 32, smem, s>>>(x, proj, scale, T, H, E, eps,
                                                                 root, scores);
    } else {
        dim3 grid((E + kEB - 1) / kEB, (T + kTT - 1) / kTT);
        router_scores_tiled<<<grid, 256, 0, s>>>(x, proj, scale, T, H, E, eps, root, scores);
    }
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_router_select(const float *scores, const uint16_t *pes, int T, int E, int K,
                                 int32_t *idx, uint16_t *w, int32_t *counts, cudaStream_t s,
                                 int *launches) {
    const int warps_per_block = 8;
    dim3 grid((T + warps_per_block - 1) / warps_per_block);
    router_select<<<grid, warps_per_block * 32, 0, s>>>(scores, pes, T, E, K, idx, w, counts);
    if (launches) ++*launches;
    return cudaGetLastError();
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
