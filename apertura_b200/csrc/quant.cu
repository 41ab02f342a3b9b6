// quant.cu -- MLX-format affine quantisation of expert weights on the device.
//
// The reference quantises the bf16 expert banks once at load when quantBits > 0
// (aptransformer/ESExperts.mm:13-18, via mx::quantize, ml-explore/mlx @ 057cdc9ec).
// This kernel applies MLX's published affine scheme per group of `gs` values
// along the input axis:
//   scale = (max - min) / (2^bits - 1)  (clamped below at 1e-7), bias = min,
//   both stored as bf16; q = clamp(rint((w - bias) / scale), 0, 2^bits - 1)
//   computed against the stored bf16 scale and bias; 32/bits values per uint32,
//   element i at bit (i*bits) % 32 of word i*bits/32 (low bits first).
#include "common.cuh"
#include "moe_internal.h"

namespace apt {

namespace {

__global__ void quantize_affine_kernel(const uint16_t *__restrict__ w, int64_t rows, int cols,
                                       int gs, int bits, uint32_t *__restrict__ q,
                                       uint16_t *__restrict__ sc, uint16_t *__restrict__ bi) {
    const int ng = cols / gs;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * ng) return;
    const int64_t r = gid / ng;
    const int g = (int)(gid - r * ng);
    const uint16_t *src = w + r * cols + (int64_t)g * gs;
    float mn = bf2f(src[0]), mx = mn;
    for (int i = 1; i < gs; ++i) {
        const float v = bf2f(src[i]);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    const int qmax = (1 << bits) - 1;
    float s = __fdiv_rn(__fsub_rn(mx, mn), (float)qmax);
    if (s < 1e-7f) s = 1e-7f;
    const uint16_t sb = f2bf(s), bb = f2bf(mn);
    sc[r * ng + g] = sb;
    bi[r * ng + g] = bb;
    const float sq = bf2f(sb), bq = bf2f(bb);
    const int per_word = 32 / bits;
    uint32_t *dst = q + (r * cols + (int64_t)g * gs) / per_word;
    for (int i = 0; i < gs; i += per_word) {
        uint32_t word = 0;
        for (int l = 0; l < per_word; ++l) {
            int qi = __float2int_rn(__fdiv_rn(__fsub_rn(bf2f(src[i + l]), bq), sq));
            qi = qi < 0 ? 0 : (qi > qmax ? qmax : qi);
            word |= ((uint32_t)qi) << (l * bits);
        }
        dst[i / per_word] = word;
    }
}

}  // namespace

cudaError_t launch_quantize_affine(const uint16_t *w, int64_t rows, int cols, int gs, int bits,
                                   uint32_t *q, uint16_t *sc, uint16_t *bi, cudaStream_t s) {
    const int64_t groups = rows * (cols / gs);
    const int threads = 256;
    const int64_t blocks = (groups + threads - 1) / threads;
    quantize_affine_kernel<<<(unsigned)blocks, threads, 0, s>>>(w, rows, cols, gs, bits, q, sc, bi);
    return cudaGetLastError();
}

}  // namespace apt
