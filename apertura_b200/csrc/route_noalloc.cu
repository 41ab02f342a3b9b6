// route_noalloc.cu -- apt_moe_route_noalloc: the router entry point for
// callers that may not allocate device memory (see include/apt_moe.h).
//
// The router's only scratch, the [T,E] f32 scores between the score kernel and
// the top-k selection kernel, lives in a file-scope device array instead of a
// handle's workspace.  Host code cannot use the array's name as a device
// address, so the address is looked up once per device with
// cudaGetSymbolAddress and passed to the kernels.  Nothing here calls
// cudaMalloc, cudaFree or any allocating library routine.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/apt_moe.h"
#include "moe_internal.h"

namespace {

// Shared by every call on a device; the score kernel writes every element the
// selection kernel reads, so nothing has to start at zero.
static __device__ __align__(256) float g_noalloc_scores[APT_NOALLOC_MAX_SCORES];
// Error word of the score kernel's bounded wait (30 = its staged rows never
// arrived).  Cleared at the start of every call; the selection kernel reads it
// and then marks the whole call invalid (every idx -1, every w 0).
static __device__ __align__(16) int32_t g_noalloc_err;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float *g_scores_ptr[kMaxDevices] = {};
int32_t *g_err_ptr[kMaxDevices] = {};

// Per-device set-up with that device current: resolve the arrays' device
// addresses once (they stay valid for the life of the CUDA context; calls
// after a cudaDeviceReset on that device are not supported).
apt_status setup_device(int dev, float **scores, int32_t **err) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scores_ptr[dev]) {
        void *p = nullptr, *q = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scores);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_noalloc_err);
        if (e != cudaSuccess) {
            fprintf(stderr, "apt_moe_route_noalloc: cudaGetSymbolAddress failed: %s\n",
                    cudaGetErrorString(e));
            return APT_ERR_CUDA;
        }
        g_err_ptr[dev] = static_cast<int32_t *>(q);
        g_scores_ptr[dev] = static_cast<float *>(p);
    }
    *scores = g_scores_ptr[dev];
    *err = g_err_ptr[dev];
    return APT_OK;
}

}  // namespace

extern "C" apt_status apt_moe_route_noalloc(const uint16_t *x, int T, const uint16_t *proj,
                                            const uint16_t *scale, const uint16_t *pes, int H,
                                            int E, int K, float eps, int32_t *idx, uint16_t *w,
                                            void *stream) {
    if (T < 0 || H <= 0 || E <= 0 || K <= 0) return APT_ERR_INVALID;
    if (H % 64 || E > 256 || K > 32 || K > E) return APT_ERR_UNSUPPORTED;
    if ((long long)T * E > APT_NOALLOC_MAX_SCORES) {
        fprintf(stderr,
                "apt_moe_route_noalloc: T*num_experts = %lld exceeds the fixed scratch of %d "
                "scores; split the call or use apt_moe_route\n",
                (long long)T * E, APT_NOALLOC_MAX_SCORES);
        return APT_ERR_UNSUPPORTED;
    }
    if (T == 0) return APT_OK;
    if (!x || !proj || !scale || !pes || !idx || !w) return APT_ERR_INVALID;
    // the score kernels read x, proj and scale with 16-byte vector and bulk loads
    if (((uintptr_t)x | (uintptr_t)proj | (uintptr_t)scale) & 15) {
        fprintf(stderr, "apt_moe_route_noalloc: x, proj and scale must be 16-byte aligned\n");
        return APT_ERR_INVALID;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return APT_ERR_CUDA;
    float *scores = nullptr;
    int32_t *err = nullptr;
    apt_status st = setup_device(dev, &scores, &err);
    if (st) return st;
    // per call: sets the score kernel's shared-memory limit (no allocation)
    if (apt::router_init() != cudaSuccess) return APT_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(err, 0, sizeof(int32_t), s) != cudaSuccess) return APT_ERR_CUDA;
    if (apt::launch_router_scores(x, proj, scale, T, H, E, eps, scores, s, nullptr, err) !=
        cudaSuccess)
        return APT_ERR_CUDA;
    if (apt::launch_router_select(scores, pes, T, E, K, idx, w, nullptr, s, nullptr, nullptr,
                                  err) != cudaSuccess)
        return APT_ERR_CUDA;
    return APT_OK;
}
