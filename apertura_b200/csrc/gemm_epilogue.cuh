// gemm_epilogue.cuh -- TMEM -> registers -> global epilogues shared by the
// one-CTA and CTA-pair expert GEMMs.  One thread owns one accumulator row
// (TMEM lane); it pulls 32-column chunks with tcgen05.ld.32x32b.x32 and
// waits once per 64 columns, so the TMEM load latency is paid a few times
// per tile rather than once per 8 columns.
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace apt {

__device__ __forceinline__ void store_bf16x32(uint16_t *dst, const float *y) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 v;
        v.x = pack_bf2(y[8 * q + 0], y[8 * q + 1]);
        v.y = pack_bf2(y[8 * q + 2], y[8 * q + 3]);
        v.z = pack_bf2(y[8 * q + 4], y[8 * q + 5]);
        v.w = pack_bf2(y[8 * q + 6], y[8 * q + 7]);
        reinterpret_cast<uint4 *>(dst)[q] = v;
    }
}

__device__ __forceinline__ void store_bf16x8(uint16_t *dst, const float *y) {
    uint4 v;
    v.x = pack_bf2(y[0], y[1]);
    v.y = pack_bf2(y[2], y[3]);
    v.z = pack_bf2(y[4], y[5]);
    v.w = pack_bf2(y[6], y[7]);
    *reinterpret_cast<uint4 *>(dst) = v;
}

// gate_up: accumulator columns [0, half) hold g_j, [half, 2*half) hold u_j;
// writes y_j = bf16(bf16(gelu(bf16 g)) * bf16 u) for j < ncols (ncols % 8 == 0).
__device__ __forceinline__ void epilogue_geglu(uint32_t taddr, int half, int ncols, bool valid,
                                               uint16_t *dst) {
    int c = 0;
#pragma unroll 1
    for (; c + 32 <= ncols; c += 32) {
        uint32_t g[32], u[32];
        sm100::tmem_ld32(taddr + c, g);
        sm100::tmem_ld32(taddr + half + c, u);
        sm100::tmem_ld_wait();
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
            y[j] = geglu_bf16(rbf(__uint_as_float(g[j])), rbf(__uint_as_float(u[j])));
        if (valid) store_bf16x32(dst + c, y);
    }
#pragma unroll 1
    for (; c < ncols; c += 8) {
        uint32_t g[8], u[8];
        sm100::tmem_ld8(taddr + c, g);
        sm100::tmem_ld8(taddr + half + c, u);
        sm100::tmem_ld_wait();
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            y[j] = geglu_bf16(rbf(__uint_as_float(g[j])), rbf(__uint_as_float(u[j])));
        if (valid) store_bf16x8(dst + c, y);
    }
}

// down: bf16 rounding of N columns (N % 64 == 0).
template <int N>
__device__ __forceinline__ void epilogue_bf16(uint32_t taddr, bool valid, uint16_t *dst) {
    static_assert(N % 64 == 0, "64-column chunks");
#pragma unroll 1
    for (int c = 0; c < N; c += 64) {
        uint32_t a[32], b[32];
        sm100::tmem_ld32(taddr + c, a);
        sm100::tmem_ld32(taddr + c + 32, b);
        sm100::tmem_ld_wait();
        if (valid) {
            float y[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) y[j] = __uint_as_float(a[j]);
            store_bf16x32(dst + c, y);
#pragma unroll
            for (int j = 0; j < 32; ++j) y[j] = __uint_as_float(b[j]);
            store_bf16x32(dst + c + 32, y);
        }
    }
}

// down, through shared memory and TMA stores: the warp's 32 rows x 64
// columns go to a 4 KB staging box (128-byte swizzle, as the tensor map
// expects) and leave as one bulk store of whole 128-byte lines, instead of
// 32 rows x 16-byte scattered stores per instruction.  `stage` = two
// 1024-aligned 4 KB buffers owned by this warp; `bufsel` alternates them
// across calls.  Only for warps whose 32 rows are all valid.
template <int N>
__device__ __forceinline__ void epilogue_bf16_tma(uint32_t taddr, uint8_t *stage, int &bufsel,
                                                  const CUtensorMap *map, int col0, int row0,
                                                  int lane) {
    static_assert(N % 64 == 0, "64-column chunks");
#pragma unroll 1
    for (int c = 0; c < N; c += 64) {
        uint32_t a[32], b[32];
        sm100::tmem_ld32(taddr + c, a);
        sm100::tmem_ld32(taddr + c + 32, b);
        sm100::tmem_ld_wait();
        uint8_t *buf = stage + bufsel * 4096;
        if (lane == 0) sm100::bulk_wait_read<1>();  // this buffer's previous store has read it
        __syncwarp();
        uint8_t *rowp = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t *src = (j < 4) ? a + 8 * j : b + 8 * (j - 4);
            uint4 v;
            v.x = pack_bf2(__uint_as_float(src[0]), __uint_as_float(src[1]));
            v.y = pack_bf2(__uint_as_float(src[2]), __uint_as_float(src[3]));
            v.z = pack_bf2(__uint_as_float(src[4]), __uint_as_float(src[5]));
            v.w = pack_bf2(__uint_as_float(src[6]), __uint_as_float(src[7]));
            *reinterpret_cast<uint4 *>(rowp + ((j ^ (lane & 7)) << 4)) = v;
        }
        sm100::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            sm100::tma_store_2d(map, buf, col0 + c, row0);
            sm100::bulk_commit();
        }
        bufsel ^= 1;
    }
}

}  // namespace apt
