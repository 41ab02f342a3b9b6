// quant.cu -- MLX-format affine quantisation of expert weights on the device.
//
// The reference quantises the bf16 expert banks once at load when quantBits > 0
// (aptransformer/ESExperts.mm:13-18, via mx::quantize, ml-explore/mlx @ 057cdc9ec).
// This kernel applies MLX's affine rule (mlx/fast.cpp `affine_quantize` at that
// commit) per group of `gs` values along the input axis, in f32:
//   n = 2^bits - 1; mask = |min| > |max|
//   scale = max((max - min) / n, 1e-7), negated when !mask
//   edge = mask ? min : max;  q0 = rint(edge / scale)
//   if q0 != 0: scale = edge / q0 (zero becomes a code);  bias = q0 ? edge : 0
//   q = clamp(rint((w - bias) / scale), 0, n) with the f32 scale and bias,
// then scale and bias are stored as bf16; 32/bits values per uint32, element i
// at bit (i*bits) % 32 of word i*bits/32 (low bits first).
#include "common.cuh"
#include "launch_util.h"
#include "moe_internal.h"
#include "sm100_ptx.cuh"

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
    const bool mask = fabsf(mn) > fabsf(mx);
    float s = __fdiv_rn(__fsub_rn(mx, mn), (float)qmax);
    if (s < 1e-7f) s = 1e-7f;
    if (!mask) s = -s;
    const float edge = mask ? mn : mx;
    const float q0 = rintf(__fdiv_rn(edge, s));
    if (q0 != 0.f) s = __fdiv_rn(edge, q0);
    const float bq = q0 == 0.f ? 0.f : edge;
    const float sq = s;
    sc[r * ng + g] = f2bf(sq);
    bi[r * ng + g] = f2bf(bq);
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

// Dequantise the rows of every active expert into a bf16 bank with the same
// [E, rows, cols] layout as the original weights: w = bf16(scale*q + bias).
// The prefill path runs the bf16 tensor-core GEMM on this bank.  Each thread
// expands 8 consecutive elements: one code word (4-bit) or two (8-bit), one
// (scale, bias) pair, one 16-byte store; 32-bit index arithmetic (an
// expert's rows * cols / 8 fits easily).
__global__ void __launch_bounds__(256)
dequant_active_kernel(const uint32_t *__restrict__ q, const uint16_t *__restrict__ sc,
                      const uint16_t *__restrict__ bi, int rows, int cols, int bits,
                      const int32_t *__restrict__ active, const int32_t *__restrict__ n_active,
                      uint16_t *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    if ((int)blockIdx.y >= *n_active) return;
    const int e = active[blockIdx.y];
    const int nvec = rows * (cols / 8);  // 8-element vectors of this expert
    const int gpr = cols / 64;           // groups per row
    const size_t ebase = (size_t)e * rows * cols;
    const uint32_t *qe = q + ebase * bits / 32;
    const uint16_t *se = sc + (size_t)e * rows * gpr, *be = bi + (size_t)e * rows * gpr;
    uint4 *oe = reinterpret_cast<uint4 *>(out + ebase);
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += gridDim.x * blockDim.x) {
        const int g = v >> 3;  // row-major 64-element groups: 8 vectors each
        const float s = bf2f(__ldg(se + g)), b = bf2f(__ldg(be + g));
        float f[8];
        if (bits == 4) {
            const uint32_t w = __ldg(qe + v);
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = fmaf(s, (float)((w >> (4 * i)) & 15u), b);
        } else {
            const uint2 w = __ldg(reinterpret_cast<const uint2 *>(qe) + v);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                f[i] = fmaf(s, (float)((w.x >> (8 * i)) & 255u), b);
                f[4 + i] = fmaf(s, (float)((w.y >> (8 * i)) & 255u), b);
            }
        }
        uint4 o;
        o.x = pack_bf2(f[0], f[1]);
        o.y = pack_bf2(f[2], f[3]);
        o.z = pack_bf2(f[4], f[5]);
        o.w = pack_bf2(f[6], f[7]);
        oe[v] = o;
    }
}

// 4-bit codes of one MLX row-major bank (low nibble first) in the order the
// one-kernel decode block's mma.sync m16n8k16 A fragments read them
// (decode_fused.cu).  An item is one contiguous block of words
// [k-step][warp 0..7][lane 0..31][4]; lane (g, t) = (lane >> 2, lane & 3)
// finds in each of its 4 words the codes of one row at
// k = base + 2t + 8p and base + 2t + 8p + 1 for p = 0..3, at bits 4p and
// 16 + 4p, so that ((word >> 4p) & 0x000F000F) | 0x43004300 is its bf16
// fragment pair (128 + q, 128 + q') -- the same values the MLX layout gives.
//   gate_up item (expert e, 16-column block b, H/256 k-steps of 256 columns):
//     warp w covers columns 256 kc + 32 w; words (gate row g, gate row g + 8,
//     up row g, up row g + 8) of the block; base = 256 kc + 32 w.
//   down item (expert e, 128-row block hb, I/64 k-steps of one 64-column
//     group): warp w covers rows 16 w .. 16 w + 15; words (row 16w + g, base
//     64 kc), (row 16w + g + 8, same), (row 16w + g, base 64 kc + 32),
//     (row 16w + g + 8, same).
__global__ void repack_q4_decode_kernel(const uint32_t *__restrict__ q, int E, int H, int I,
                                        int down, uint32_t *__restrict__ out) {
    const int cols = down ? I : H;
    const int64_t item_words = down ? 16LL * I : 4LL * H;
    const int per_expert = down ? H / 128 : I / 16;
    const int64_t total = (int64_t)E * per_expert * item_words;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t item = idx / item_words;
        const int within = (int)(idx - item * item_words);
        const int kc = within >> 10, w = (within >> 7) & 7, lane = (within >> 2) & 31, j = within & 3;
        const int g = lane >> 2, t = lane & 3;
        const int e = (int)(item / per_expert), b = (int)(item - (int64_t)e * per_expert);
        int64_t row;
        int base;
        if (!down) {
            const int h = j >> 1, rs = j & 1;
            row = (int64_t)e * 2 * I + (h ? I : 0) + b * 16 + g + 8 * rs;
            base = 256 * kc + 32 * w;
        } else {
            const int rs = j & 1, ch = j >> 1;
            row = (int64_t)e * H + b * 128 + 16 * w + g + 8 * rs;
            base = 64 * kc + 32 * ch;
        }
        const uint32_t *qr = q + row * (cols / 8);
        uint32_t word = 0;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int k = base + 2 * t + 8 * p;
            const uint32_t c0 = (qr[k >> 3] >> (4 * (k & 7))) & 15u;
            const uint32_t c1 = (qr[(k + 1) >> 3] >> (4 * ((k + 1) & 7))) & 15u;
            word |= (c0 << (4 * p)) | (c1 << (16 + 4 * p));
        }
        out[idx] = word;
    }
}

// Repack scales/biases [rows, groups] x2 into one [rows, groups] uint32 array
// of (scale | bias << 16) pairs: a row's pairs are contiguous (groups*4 bytes),
// so a kernel stages a block of rows with plain 16-byte loads.
// (scale | bias << 16) per group, rows of g groups padded with zeros to gp
// (a multiple of 4, so every row starts on 16 bytes for the TMA).
__global__ void interleave_sb_kernel(const uint16_t *__restrict__ sc,
                                     const uint16_t *__restrict__ bi, int64_t rows, int g, int gp,
                                     uint32_t *__restrict__ out) {
    const int64_t n = rows * gp;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / gp;
        const int c = (int)(i - r * gp);
        out[i] = c < g ? ((uint32_t)sc[r * g + c] | ((uint32_t)bi[r * g + c] << 16)) : 0u;
    }
}

}  // namespace

cudaError_t launch_interleave_sb(const uint16_t *sc, const uint16_t *bi, int64_t rows, int g,
                                 uint32_t *out, cudaStream_t s) {
    interleave_sb_kernel<<<1024, 256, 0, s>>>(sc, bi, rows, g, sb_row_words(g * 64), out);
    return cudaGetLastError();
}

cudaError_t launch_repack_q4_decode(const uint32_t *gu_q, const uint32_t *dn_q, int E, int H, int I,
                                    uint32_t *gu_qd, uint32_t *dn_qd, cudaStream_t s) {
    repack_q4_decode_kernel<<<2048, 256, 0, s>>>(gu_q, E, H, I, 0, gu_qd);
    cudaError_t e = cudaGetLastError();
    if (e) return e;
    repack_q4_decode_kernel<<<2048, 256, 0, s>>>(dn_q, E, H, I, 1, dn_qd);
    return cudaGetLastError();
}

cudaError_t launch_dequant_active(const uint32_t *q, const uint16_t *sc, const uint16_t *bi,
                                  int rows, int cols, int bits, const Dispatch &d, int E,
                                  uint16_t *out, cudaStream_t s, int *launches) {
    dim3 grid(64, E);
    cudaError_t err = launch_ex(dequant_active_kernel, grid, dim3(256), 0, s, true, q, sc, bi,
                                rows, cols, bits, (const int32_t *)d.active,
                                (const int32_t *)d.n_active, out);
    if (launches) ++*launches;
    return err;
}

cudaError_t launch_quantize_affine(const uint16_t *w, int64_t rows, int cols, int gs, int bits,
                                   uint32_t *q, uint16_t *sc, uint16_t *bi, cudaStream_t s) {
    const int64_t groups = rows * (cols / gs);
    const int threads = 256;
    const int64_t blocks = (groups + threads - 1) / threads;
    quantize_affine_kernel<<<(unsigned)blocks, threads, 0, s>>>(w, rows, cols, gs, bits, q, sc, bi);
    return cudaGetLastError();
}

}  // namespace apt

namespace apt {

namespace {

// One thread waits on an mbarrier nothing arrives on, through the same bounded
// wait every pipeline of the library uses; on expiry it records `code` in the
// error word and returns (the context stays usable).
__global__ void selftest_wait_kernel(long long limit_cycles, int32_t *err, int code) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        sm100::fence_barrier_init();
        if (!sm100::mbar_wait(&bar, 0, limit_cycles) && atomicCAS(err, 0, code) == 0) err[1] = -1;
    }
}

}  // namespace

cudaError_t launch_selftest_wait(long long limit_cycles, int32_t *err, cudaStream_t s) {
    selftest_wait_kernel<<<1, 32, 0, s>>>(limit_cycles, err, 99);
    return cudaGetLastError();
}

}  // namespace apt
