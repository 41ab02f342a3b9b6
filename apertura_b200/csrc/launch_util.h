// launch_util.h -- host-side launch helpers shared by the kernel files:
// cached device properties, a cache of TMA tensor maps (encoding one costs
// microseconds of host time, and the weight and workspace pointers a handle
// passes are stable between calls), and programmatic dependent launch.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

namespace apt {

inline int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

inline int num_sms(int dev) {
    static int cache[64] = {0};
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int v = 148;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v;
    }
    return cache[dev];
}

// SMs the persistent kernels of the current call may fill: all of them, or a
// per-handle cap (apt_moe_set_sm_limit) that leaves room for kernels running
// beside them, e.g. NCCL's during an expert-parallel exchange.  Set by the
// entry point at the start of each call on the calling thread.
inline int &sm_cap() {
    static thread_local int cap = 0;
    return cap;
}

inline int grid_sms(int dev) {
    const int n = num_sms(dev), c = sm_cap();
    return (c > 0 && c < n) ? c : n;
}

// ---------------------------------------------------------------- tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D row-major [rows, inner] tensor of 2-byte (bf16) or 4-byte (u32)
// elements, box {box_inner, box_rows}.  Returns false if the driver entry
// point is missing or encoding fails.  Results are cached by all their
// parameters (a small direct-mapped cache).
inline bool map_2d(CUtensorMap *out, const void *base, uint64_t inner, uint64_t rows,
                   uint32_t box_inner, uint32_t box_rows, bool swizzle128, bool u32) {
    struct Entry {
        const void *base;
        uint64_t inner, rows;
        uint32_t bi, br;
        bool sw, u32;
        bool valid;
        CUtensorMap map;
    };
    static Entry cache[64];
    static std::mutex mu;
    const uint64_t key = (reinterpret_cast<uintptr_t>(base) >> 8) ^ (inner * 31) ^ (rows * 131) ^
                         (box_inner * 7) ^ (box_rows * 13) ^ (swizzle128 ? 1 : 0) ^ (u32 ? 2 : 0);
    Entry &slot = cache[key % 64];
    {
        std::lock_guard<std::mutex> lock(mu);
        if (slot.valid && slot.base == base && slot.inner == inner && slot.rows == rows &&
            slot.bi == box_inner && slot.br == box_rows && slot.sw == swizzle128 && slot.u32 == u32) {
            *out = slot.map;
            return true;
        }
    }
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    const uint64_t esize = u32 ? 4 : 2;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * esize};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    if (fn(&m, u32 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
           const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    std::lock_guard<std::mutex> lock(mu);
    slot = Entry{base, inner, rows, box_inner, box_rows, swizzle128, u32, true, m};
    *out = m;
    return true;
}

inline bool bf16_map_2d(CUtensorMap *out, const void *base, uint64_t inner, uint64_t rows,
                        uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
    return map_2d(out, base, inner, rows, box_inner, box_rows, swizzle128, false);
}

// ---------------------------------------------------------------- launches

// Launch with programmatic dependent launch allowed when `pdl`: the kernel may
// start while the previous kernel on the stream finishes; it must execute
// griddepcontrol.wait before touching that kernel's outputs.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t s, bool pdl, Args &&...args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace apt
