// common.cuh -- shared device helpers for the MoE block kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace apt {

// ---------------------------------------------------------------- bf16 bits

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// Round-to-nearest-even f32 -> bf16 (the hardware conversion; NaN preserved).
__device__ __forceinline__ uint16_t f2bf(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }
// Two round-to-nearest-even conversions (lo in the low half) as one paired
// conversion instruction.
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Unpack 8 bf16 held in a uint4 into f32.
__device__ __forceinline__ void unpack8(const uint4 &v, float *f) {
    f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
    f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
    f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
    f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
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

// m16n8k16 bf16 MMA, f32 accumulate (D += A B) and the 4-bit code -> bf16
// fragment packing used with it (128 + q is exact in bf16).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The A fragment of one 16x16 tile (rows g and g + 8, k = 2t, 2t+1, 2t+8,
// 2t+9 of the tile) from the two packed words (k 0..7, k 8..15) of each row.
__device__ __forceinline__ void q4_pair(uint32_t w0, uint32_t w1, int t, uint32_t &lo,
                                        uint32_t &hi) {
    // byte t of w0 (codes k=2t, 2t+1) and byte t of w1 (k=2t+8, 2t+9)
    const uint32_t x = __byte_perm(w0, w1, (uint32_t)(t | ((4 + t) << 4))) & 0xFFFFu;
    lo = ((x | (x << 12)) & 0x000F000Fu) | 0x43004300u;         // (128+q0, 128+q1)
    hi = (((x >> 8) | (x << 4)) & 0x000F000Fu) | 0x43004300u;  // (128+q8, 128+q9)
}

// Streaming 16-byte global load that does not allocate in L1 (weights are
// read once per launch).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// ---------------------------------------------------------------- gelu

// gelu_pytorch_tanh in f32 with the reference op order (aptransformer/ESOps.h:29-37):
//   x3 = (x*x)*x; inner = c0*(x + c1*x3); y = (0.5*x)*(1 + tanh(inner)).
// Contraction into FMAs is disabled so every step rounds like the reference.
__device__ __forceinline__ float gelu_tanh_f32(float x) {
    float x3 = __fmul_rn(__fmul_rn(x, x), x);
    float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// y = bf16( bf16(gelu(g)) * u ) for bf16-valued g and u (ESExperts.mm:53-54).
__device__ __forceinline__ float geglu_bf16(float g_bf, float u_bf) {
    float ge = rbf(gelu_tanh_f32(g_bf));
    return rbf(__fmul_rn(ge, u_bf));
}

// ---------------------------------------------------------------- PDL

// Programmatic dependent launch: wait until the preceding kernel on the
// stream has completed and its writes are visible (no-op when this kernel
// was launched without the attribute), and let the next kernel start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- warp helpers

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace apt
