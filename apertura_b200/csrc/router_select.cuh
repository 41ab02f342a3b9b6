// router_select.cuh -- the parts of ESRouter::routeTopK (aptransformer/ESRouter.mm:14-32)
// shared by the router kernels (router.cu) and the fused decode kernel
// (decode_fused.cu): the router input h, and softmax + top-K + renormalise of
// one token's scores by one warp.
#pragma once

#include "common.cuh"

namespace apt {

// h = ((x * r) * scale) * root, element-wise, f32 rounding at every step.
__device__ __forceinline__ float router_h(float x, float r, float sc, float root) {
    return __fmul_rn(__fmul_rn(__fmul_rn(x, r), sc), root);
}

constexpr int kMaxPerLane = 8;  // E <= 256

// Softmax and top-K (descending prob, lower id on ties) of one token's scores
// p[j] = score of expert lane + 32 j (-inf past E), by one warp.  Lane k < K
// returns the k-th choice (sel_e, sel_p); every lane returns the k-order sum
// of the K chosen probabilities.
// Order-preserving map of f32 to u32 (for single-instruction warp max).
__device__ __forceinline__ unsigned fkey(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Softmax of one token's scores in place, by one warp: p[j] (expert
// lane + 32 j) becomes exp(s - max) / sum, rounded as the f32 ops round;
// slots past E become -1 (never selected).
template <int NP>
__device__ __forceinline__ void softmax_core(float (&p)[NP], int E, int lane) {
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NP; ++j) m = fmaxf(m, p[j]);
    m = fkey_inv(__reduce_max_sync(0xffffffffu, fkey(m)));
    float den = 0.f;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? expf(__fsub_rn(p[j], m)) : 0.f;
        den += p[j];
    }
    den = warp_sum(den);
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const int e = lane + 32 * j;
        p[j] = (e < E) ? __fdiv_rn(p[j], den) : -1.f;  // -1: never selected
    }
}

// NP = scores per lane (E <= 32 NP); E <= 128 scans 4 slots per lane per round.
template <int NP>
__device__ __forceinline__ void select_core(float (&p)[NP], int E, int K, int lane,
                                            int &sel_e, float &sel_p, float &sum) {
    softmax_core<NP>(p, E, lane);
    sum = 0.f;
    sel_p = 0.f;
    sel_e = -1;
    unsigned taken = 0;
    for (int k = 0; k < K; ++k) {
        float bp = -2.f;  // lane-local best among untaken (lowest id on ties)
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < NP; ++j) {
            const int e = lane + 32 * j;
            if (!((taken >> j) & 1u) && (p[j] > bp)) {
                bp = p[j];
                be = e;
            }
        }
        // warp-wide: the largest probability, then the lowest id holding it
        const unsigned kb = fkey(bp);
        const unsigned mk = __reduce_max_sync(0xffffffffu, kb);
        const int we = (int)__reduce_min_sync(0xffffffffu, kb == mk ? (unsigned)be : 0xffffffffu);
        const float wp = fkey_inv(mk);
        if ((we & 31) == lane) taken |= 1u << (we >> 5);
        sum = __fadd_rn(sum, wp);  // sequential in k order, every lane the same
        if (lane == k) {
            sel_p = wp;
            sel_e = we;
        }
    }
}

}  // namespace apt
