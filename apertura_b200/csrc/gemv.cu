// gemv.cu -- decode-sized grouped expert GEMV (HBM streaming): bf16 and MLX
// affine 4/8-bit expert weights.
//
// Restates the gather_mm / gather_qmm path of ESExperts::sparseForward
// (aptransformer/ESExperts.mm:44-60) for decode-sized token groups:
//   gate_up: g = bf16(x . Wg_j), u = bf16(x . Wu_j)          (f32 accumulate)
//            y_j = bf16(bf16(gelu_f32(g)) * u)               (ESExperts.mm:53-54, ESOps.h:29-37)
//   down:    o_h = bf16(y . Wd_h)                             (ESExperts.mm:55-57)
// Quantised rows dequantise as w = scale*q + bias per group of 64; the dot is
// taken as scale*sum(q*x) + bias*sum(x) per group, the same value in f32.
// Each active expert's weights stream from HBM once for all of its tokens
// (the dispatch grouped them) instead of once per (token, k) pair.
//
// Work decomposition.  A CTA owns one active expert and a block of output rows.
// Inside a warp, lanes form 4 row-groups of 8 lanes; the 8 lanes of a group
// split the reduction dimension into EPL-element slices (one 16-byte load of
// bf16, or EPL*bits/8 bytes of packed weights per lane and step), so each warp
// load instruction reads 4 fully-used contiguous segments.  The expert's
// tokens are staged in shared memory as f32 in a lane-permuted layout
// (conflict-free 128-bit reads, broadcast across the 4 row-groups) and
// processed in chunks of up to 8; the chunk's token count selects a
// specialised inner loop.
#include "common.cuh"
#include "launch_util.h"
#include "moe_internal.h"

namespace apt {

namespace {

constexpr int kWarps = 4;
constexpr int kTokChunk = 8;

// Staged-token layout for a lane slice of EPL elements: element k sits at
// step = k / (8*EPL), lane c = (k / EPL) % 8, r = k % EPL ->
// float index ((step*(EPL/4) + r/4)*8 + c)*4 + r%4.
template <int EPL>
__device__ __forceinline__ int xs_index(int k) {
    const int step = k / (8 * EPL), c = (k / EPL) & 7, r = k % EPL;
    return ((step * (EPL / 4) + (r >> 2)) * 8 + c) * 4 + (r & 3);
}

template <int EPL>
__device__ __forceinline__ void stage_rows(float *xs, const uint16_t *const *src_rows, int nt,
                                           int len) {
    const int vecs = len / 8;
    for (int v = threadIdx.x; v < nt * vecs; v += blockDim.x) {
        const int r = v / vecs, k = (v - r * vecs) * 8;
        float f[8];
        unpack8(*reinterpret_cast<const uint4 *>(src_rows[r] + k), f);
        float *d = xs + r * len;
        *reinterpret_cast<float4 *>(d + xs_index<EPL>(k)) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4 *>(d + xs_index<EPL>(k + 4)) = make_float4(f[4], f[5], f[6], f[7]);
    }
}

// ---------------------------------------------------------------- weight formats

// bf16 rows: 8 elements (one uint4) per lane and step.
struct FmtBf16 {
    static constexpr int EPL = 8;
    struct Row {
        const uint16_t *p;  // this lane's slice of step 0
    };
    __device__ static Row row(const uint16_t *w, const uint32_t *, const uint16_t *,
                              const uint16_t *, int64_t r, int len, int c) {
        return Row{w + r * len + c * EPL};
    }
    struct Frag {
        uint4 v;
    };
    __device__ static Frag load(const Row &rw, int step) {
        return Frag{ldg_stream(rw.p + (size_t)step * 8 * EPL)};
    }
    // dot of the fragment with EPL staged x values (xf); xsum unused
    __device__ static float dot(const Frag &f, const float *xf, float /*xsum*/) {
        float s = 0.f;
        s = fmaf(bf_lo(f.v.x), xf[0], s);
        s = fmaf(bf_hi(f.v.x), xf[1], s);
        s = fmaf(bf_lo(f.v.y), xf[2], s);
        s = fmaf(bf_hi(f.v.y), xf[3], s);
        s = fmaf(bf_lo(f.v.z), xf[4], s);
        s = fmaf(bf_hi(f.v.z), xf[5], s);
        s = fmaf(bf_lo(f.v.w), xf[6], s);
        s = fmaf(bf_hi(f.v.w), xf[7], s);
        return s;
    }
    static constexpr bool kNeedsXsum = false;
};

// MLX affine rows: EPL elements = EPL*BITS/32 words per lane and step, plus
// the (scale, bias) of the 64-group the slice lies in.
template <int BITS, int EPL_>
struct FmtQ {
    static constexpr int EPL = EPL_;
    static constexpr int WORDS = EPL * BITS / 32;
    static_assert(64 % EPL == 0, "a lane slice must lie inside one group");
    struct Row {
        const uint32_t *q;
        const uint16_t *s, *b;
        int c;
    };
    __device__ static Row row(const uint16_t *, const uint32_t *q, const uint16_t *s,
                              const uint16_t *b, int64_t r, int len, int c) {
        return Row{q + r * (len * BITS / 32) + c * WORDS, s + r * (len / 64), b + r * (len / 64),
                   c};
    }
    struct Frag {
        uint32_t w[WORDS];
        float s, b;
    };
    __device__ static Frag load(const Row &rw, int step) {
        Frag f;
        const uint32_t *p = rw.q + (size_t)step * 8 * WORDS;
        if constexpr (WORDS == 4) {
            const uint4 v = ldg_stream(p);
            f.w[0] = v.x; f.w[1] = v.y; f.w[2] = v.z; f.w[3] = v.w;
        } else if constexpr (WORDS == 2) {
            const uint2 v = __ldg(reinterpret_cast<const uint2 *>(p));
            f.w[0] = v.x; f.w[1] = v.y;
        } else {
            f.w[0] = __ldg(p);
        }
        const int g = (step * 8 * EPL + rw.c * EPL) >> 6;
        f.s = bf2f(__ldg(rw.s + g));
        f.b = bf2f(__ldg(rw.b + g));
        return f;
    }
    __device__ static float dot(const Frag &f, const float *xf, float xsum) {
        float qx = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const uint32_t qi = (f.w[i * BITS / 32] >> ((i * BITS) & 31)) & ((1u << BITS) - 1u);
            qx = fmaf((float)qi, xf[i], qx);
        }
        return fmaf(f.s, qx, f.b * xsum);
    }
    static constexpr bool kNeedsXsum = true;
};

// acc[r][t] += W_r . x_t over `nsteps` steps of 8*EPL elements.  U steps of
// weight loads are in flight before they are consumed.
template <class F, int NT, int R, int U>
__device__ __forceinline__ void accumulate(const typename F::Row (&rows)[R], int nsteps,
                                           const float *xs, int ld, int c, float (&acc)[R][NT]) {
    constexpr int EPL = F::EPL;
    for (int s0 = 0; s0 < nsteps; s0 += U) {
        typename F::Frag fr[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (s0 + u < nsteps) fr[u][r] = F::load(rows[r], s0 + u);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (s0 + u < nsteps) {
                const int base = ((s0 + u) * (EPL / 4) * 8 + c) * 4;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float xf[EPL];
#pragma unroll
                    for (int v = 0; v < EPL / 4; ++v) {
                        const float4 a = *reinterpret_cast<const float4 *>(xs + t * ld + base + v * 32);
                        xf[4 * v] = a.x; xf[4 * v + 1] = a.y; xf[4 * v + 2] = a.z; xf[4 * v + 3] = a.w;
                    }
                    float xsum = 0.f;
                    if constexpr (F::kNeedsXsum) {
#pragma unroll
                        for (int i = 0; i < EPL; ++i) xsum += xf[i];
                    }
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r][t] += F::dot(fr[u][r], xf, xsum);
                }
            }
        }
    }
}

// Sum over the 8 lanes of a row-group (lane bits 0..2).
template <int NT, int R>
__device__ __forceinline__ void group_reduce(float (&acc)[R][NT]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float v = acc[r][t];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            acc[r][t] = v;
        }
}

template <int NT, int R>
__device__ __forceinline__ float pick(const float (&acc)[R][NT], int r, int t) {
    float v = 0.f;
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
        if (tt == t) v = acc[r][tt];
    return v;
}

struct GemvArgs {
    const uint16_t *w;                    // bf16 bank
    const uint32_t *q;                    // packed bank
    const uint16_t *s, *b;                // scales / biases
    const int32_t *perm, *offsets, *counts, *active, *n_active;
    const uint16_t *in;                   // x [T,H] (gate_up) or yp [rows,I] (down)
    uint16_t *out;                        // yp [rows,I] (gate_up) or op [rows,H] (down)
    int K, H, I, tok_chunk;
};

// ---------------------------------------------------------------- gate_up

// RJ intermediate columns per row-group; rows per lane = 2*RJ (gate j.., up j..)
template <class F, int NT, int RJ, int U>
__device__ __forceinline__ void gateup_chunk(const GemvArgs &a, int e, int j0, const float *xs,
                                             int c, int nt, int row0) {
    constexpr int R = 2 * RJ;
    typename F::Row rows[R];
    const int64_t rb = (int64_t)e * 2 * a.I;
#pragma unroll
    for (int q = 0; q < RJ; ++q) {
        rows[q] = F::row(a.w, a.q, a.s, a.b, rb + j0 + q, a.H, c);
        rows[RJ + q] = F::row(a.w, a.q, a.s, a.b, rb + a.I + j0 + q, a.H, c);
    }
    float acc[R][NT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    accumulate<F, NT, R, U>(rows, a.H / (8 * F::EPL), xs, a.H, c, acc);
    group_reduce<NT, R>(acc);
    if (c < nt) {
        uint16_t *dst = a.out + (size_t)(row0 + c) * a.I + j0;
#pragma unroll
        for (int q = 0; q < RJ; ++q) {
            const float g = rbf(pick<NT, R>(acc, q, c));
            const float u = rbf(pick<NT, R>(acc, RJ + q, c));
            dst[q] = f2bf(geglu_bf16(g, u));
        }
    }
}

template <class F, int RJ, int U, int NTMAX>
__global__ void __launch_bounds__(kWarps * 32) gemv_gateup(GemvArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float xs[];
    __shared__ const uint16_t *src[kTokChunk];
    if ((int)blockIdx.y >= *a.n_active) return;
    const int e = a.active[blockIdx.y];
    const int n = a.counts[e], base = a.offsets[e];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, c = lane & 7;
    const int j0 = (blockIdx.x * kWarps + warp) * 4 * RJ + g * RJ;
    constexpr int U2 = U > 2 ? 2 : U;
    for (int tc = 0; tc < n; tc += a.tok_chunk) {
        const int nt = min(a.tok_chunk, n - tc);
        if ((int)threadIdx.x < nt)
            src[threadIdx.x] = a.in + (size_t)(a.perm[base + tc + threadIdx.x] / a.K) * a.H;
        __syncthreads();
        stage_rows<F::EPL>(xs, src, nt, a.H);
        __syncthreads();
        // only the token counts this launch can see are instantiated, so the
        // register budget follows the call's T, not the worst case
        if (nt == 1) {
            gateup_chunk<F, 1, RJ, U>(a, e, j0, xs, c, nt, base + tc);
        } else if (nt == 2) {
            if constexpr (NTMAX >= 2) gateup_chunk<F, 2, RJ, U>(a, e, j0, xs, c, nt, base + tc);
        } else if (nt <= 4) {
            if constexpr (NTMAX >= 4) gateup_chunk<F, 4, RJ, U2>(a, e, j0, xs, c, nt, base + tc);
        } else {
            if constexpr (NTMAX >= 8) gateup_chunk<F, 8, RJ, U2>(a, e, j0, xs, c, nt, base + tc);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- down

template <class F, int NT, int R, int U>
__device__ __forceinline__ void down_chunk(const GemvArgs &a, int e, int h0, const float *ys,
                                           int c, int nt, int row0) {
    typename F::Row rows[R];
    const int64_t rb = (int64_t)e * a.H;
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = F::row(a.w, a.q, a.s, a.b, rb + h0 + r, a.I, c);
    float acc[R][NT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.f;
    accumulate<F, NT, R, U>(rows, a.I / (8 * F::EPL), ys, a.I, c, acc);
    group_reduce<NT, R>(acc);
    if (c < nt) {
        uint16_t *dst = a.out + (size_t)(row0 + c) * a.H + h0;
#pragma unroll
        for (int r = 0; r < R; ++r) dst[r] = f2bf(pick<NT, R>(acc, r, c));
    }
}

template <class F, int R, int U, int NTMAX>
__global__ void __launch_bounds__(kWarps * 32) gemv_down(GemvArgs a) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float ys[];
    __shared__ const uint16_t *src[kTokChunk];
    if ((int)blockIdx.y >= *a.n_active) return;
    const int e = a.active[blockIdx.y];
    const int n = a.counts[e], base = a.offsets[e];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 3, c = lane & 7;
    const int h0 = (blockIdx.x * kWarps + warp) * 4 * R + g * R;
    constexpr int U2 = U > 2 ? 2 : U;
    for (int tc = 0; tc < n; tc += a.tok_chunk) {
        const int nt = min(a.tok_chunk, n - tc);
        if ((int)threadIdx.x < nt) src[threadIdx.x] = a.in + (size_t)(base + tc + threadIdx.x) * a.I;
        __syncthreads();
        stage_rows<F::EPL>(ys, src, nt, a.I);
        __syncthreads();
        if (nt == 1) {
            down_chunk<F, 1, R, U>(a, e, h0, ys, c, nt, base + tc);
        } else if (nt == 2) {
            if constexpr (NTMAX >= 2) down_chunk<F, 2, R, U>(a, e, h0, ys, c, nt, base + tc);
        } else if (nt <= 4) {
            if constexpr (NTMAX >= 4) down_chunk<F, 4, R, U2>(a, e, h0, ys, c, nt, base + tc);
        } else {
            if constexpr (NTMAX >= 8) down_chunk<F, 8, R, U2>(a, e, h0, ys, c, nt, base + tc);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- launch plumbing

template <class F, int RJ, int U, int NTMAX>
cudaError_t set_gateup_attr() {
    return cudaFuncSetAttribute(gemv_gateup<F, RJ, U, NTMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
}
template <class F, int R, int U, int NTMAX>
cudaError_t set_down_attr() {
    return cudaFuncSetAttribute(gemv_down<F, R, U, NTMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                200 * 1024);
}

// Two shapes per format: small groups (<= 2 rows per expert) spread the rows
// thinly over many lanes with deep prefetch; larger groups give each lane more
// rows so one staged x value feeds more FMAs.
template <class F>
cudaError_t init_fmt() {
    cudaError_t e;
    if ((e = set_gateup_attr<F, 1, 4, 1>())) return e;
    if ((e = set_gateup_attr<F, 1, 4, 2>())) return e;
    if ((e = set_gateup_attr<F, 2, 2, 4>())) return e;
    if ((e = set_gateup_attr<F, 2, 2, 8>())) return e;
    if ((e = set_down_attr<F, 1, 4, 1>())) return e;
    if ((e = set_down_attr<F, 1, 4, 2>())) return e;
    if ((e = set_down_attr<F, 4, 2, 4>())) return e;
    return set_down_attr<F, 4, 2, 8>();
}

template <class F>
void launch_gateup_fmt(const GemvArgs &a, int E, int max_rows, size_t smem, cudaStream_t s) {
    if (max_rows <= 2) {
        dim3 grid(a.I / (kWarps * 4 * 1), E);
        if (max_rows <= 1) launch_ex(gemv_gateup<F, 1, 4, 1>, grid, dim3(kWarps * 32), smem, s, true, a);
        else launch_ex(gemv_gateup<F, 1, 4, 2>, grid, dim3(kWarps * 32), smem, s, true, a);
    } else {
        dim3 grid(a.I / (kWarps * 4 * 2), E);
        if (max_rows <= 4) launch_ex(gemv_gateup<F, 2, 2, 4>, grid, dim3(kWarps * 32), smem, s, true, a);
        else launch_ex(gemv_gateup<F, 2, 2, 8>, grid, dim3(kWarps * 32), smem, s, true, a);
    }
}

template <class F>
void launch_down_fmt(const GemvArgs &a, int E, int max_rows, size_t smem, cudaStream_t s) {
    if (max_rows <= 2) {
        dim3 grid(a.H / (kWarps * 4 * 1), E);
        if (max_rows <= 1) launch_ex(gemv_down<F, 1, 4, 1>, grid, dim3(kWarps * 32), smem, s, true, a);
        else launch_ex(gemv_down<F, 1, 4, 2>, grid, dim3(kWarps * 32), smem, s, true, a);
    } else {
        dim3 grid(a.H / (kWarps * 4 * 4), E);
        if (max_rows <= 4) launch_ex(gemv_down<F, 4, 2, 4>, grid, dim3(kWarps * 32), smem, s, true, a);
        else launch_ex(gemv_down<F, 4, 2, 8>, grid, dim3(kWarps * 32), smem, s, true, a);
    }
}

// Token rows staged per pass: the power of two the kernel is specialised for
// (1, 2, 4 or 8), so every specialised inner loop stays inside the staged rows.
int tok_chunk_for(int max_rows) {
    return max_rows <= 1 ? 1 : max_rows <= 2 ? 2 : max_rows <= 4 ? 4 : kTokChunk;
}

}  // namespace

cudaError_t gemv_init() {
    cudaError_t e;
    if ((e = init_fmt<FmtBf16>())) return e;
    if ((e = init_fmt<FmtQ<4, 32>>())) return e;
    if ((e = init_fmt<FmtQ<4, 8>>())) return e;
    if ((e = init_fmt<FmtQ<8, 16>>())) return e;
    return init_fmt<FmtQ<8, 8>>();
}

cudaError_t launch_gemv_gateup(const uint16_t *x, int K, const Dispatch &d, const ExpertWeights &w,
                               int H, int I, int E, int max_rows, uint16_t *yp, cudaStream_t s,
                               int *launches) {
    GemvArgs a{w.gu, w.gu_q, w.gu_s, w.gu_b, d.perm, d.offsets, d.counts, d.active, d.n_active,
               x, yp, K, H, I, tok_chunk_for(max_rows)};
    const size_t smem = (size_t)a.tok_chunk * H * sizeof(float);
    if (w.bits == 0) {
        launch_gateup_fmt<FmtBf16>(a, E, max_rows, smem, s);
    } else if (w.bits == 4) {
        if (H % 256 == 0) launch_gateup_fmt<FmtQ<4, 32>>(a, E, max_rows, smem, s);
        else launch_gateup_fmt<FmtQ<4, 8>>(a, E, max_rows, smem, s);
    } else if (w.bits == 8) {
        if (H % 128 == 0) launch_gateup_fmt<FmtQ<8, 16>>(a, E, max_rows, smem, s);
        else launch_gateup_fmt<FmtQ<8, 8>>(a, E, max_rows, smem, s);
    } else {
        return cudaErrorInvalidValue;
    }
    if (launches) ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_gemv_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w, int H,
                             int I, int E, int max_rows, uint16_t *op, cudaStream_t s,
                             int *launches) {
    GemvArgs a{w.dn, w.dn_q, w.dn_s, w.dn_b, d.perm, d.offsets, d.counts, d.active, d.n_active,
               yp, op, 0, H, I, tok_chunk_for(max_rows)};
    const size_t smem = (size_t)a.tok_chunk * I * sizeof(float);
    if (w.bits == 0) launch_down_fmt<FmtBf16>(a, E, max_rows, smem, s);
    else if (w.bits == 4) launch_down_fmt<FmtQ<4, 8>>(a, E, max_rows, smem, s);
    else if (w.bits == 8) launch_down_fmt<FmtQ<8, 8>>(a, E, max_rows, smem, s);
    else return cudaErrorInvalidValue;
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace apt
