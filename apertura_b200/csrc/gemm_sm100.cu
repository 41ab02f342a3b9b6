// gemm_sm100.cu -- prefill grouped expert GEMM (tcgen05 / TMEM / TMA).  [in progress]
#include "common.cuh"
#include "moe_internal.h"

namespace apt {

cudaError_t gemm_init() { return cudaSuccess; }
bool gemm_supported(int, int) { return false; }
cudaError_t launch_gemm_gateup(const uint16_t *, const Dispatch &, const ExpertWeights &, int, int,
                               int, int, uint16_t *, int32_t *, cudaStream_t, int *) {
    return cudaErrorNotSupported;
}
cudaError_t launch_gemm_down(const uint16_t *, const Dispatch &, const ExpertWeights &, int, int,
                             int, int, uint16_t *, int32_t *, cudaStream_t, int *) {
    return cudaErrorNotSupported;
}

}  // namespace apt
