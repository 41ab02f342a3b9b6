// ep_p2p.cu -- the expert-parallel exchange over NVLink peer memory: the
// dispatch and the combine of the all-to-all are done by this library's own
// kernels with stores to and loads from the other GPUs' memory (CUDA IPC
// mappings), with no host round trip inside a step.
//
// Every rank owns one region that all ranks map:
//   flags  [3N+2] u32: count flags (by source), push flags, done flags, a
//                      CTA counter for this rank's push kernel, an error word
//   table  [2][N][E] i32: per-source routed-row counts (new expert ids)
//   recv   [2][max_recv][H] bf16: rows other ranks push for this rank's experts
//   out    [2][max_recv][H] bf16: this rank's expert outputs for those rows
// indexed by the step's parity, so a step never overwrites what a slower
// rank may still read from the step before.  Flags carry the step number
// (epoch) and only grow, so nothing is reset between steps.
//
// A step (rank `me`, parity p, epoch s):
//   push kernel  -- CTA 0 writes this rank's counts into every rank's table[p]
//                   and release-stores count flag s there; every CTA waits for
//                   all count flags, derives where each of its cold rows lands
//                   in its owner's recv[p] (owner layout: expert-major, then
//                   source rank), copies the rows there with 16-byte stores
//                   and records for every (token, k) pair the address its
//                   result will have (hot rows: this rank's own output); the
//                   last CTA release-stores push flag s at every rank
//   wait kernel  -- the owner waits for every push flag s and writes its
//                   experts' group counts for the grouped GEMM
//   (grouped tcgen05 GEMM on recv[p] -> out[p], apt_moe_experts_grouped)
//   done kernel  -- release-stores done flag s at every rank
//   combine      -- waits for every done flag s, then out[t] = sum_k
//                   bf16(w * row) in k order (ESExperts.mm:58-59), reading
//                   each remote row straight from its owner's out[p]
// Every wait is bounded (~1 s); on expiry the kernel records code 60..63 in
// the error word and carries on, so the step ends with garbage and
// apt_moe_ep_sync reports APT_ERR_TIMEOUT instead of hanging the GPU.
// No load here uses multicast; remote rows are plain 16-byte loads/stores.
#include "common.cuh"
#include "moe_internal.h"

namespace apt {

namespace {

constexpr long long kEpWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *flag has reached epoch (wrap-safe); false after the bound.
__device__ bool wait_epoch(const uint32_t *flag, uint32_t epoch) {
    const long long t0 = clock64();
    while ((int32_t)(ld_acquire_sys(flag) - epoch) < 0) {
        if (clock64() - t0 > kEpWaitCycles) return false;
        __nanosleep(64);
    }
    return true;
}

__device__ __forceinline__ void ep_error(const EpP2PArgs &a, int code) {
    atomicCAS(reinterpret_cast<int *>(a.peers[a.me].flags + a.ERR()), 0, code);
}

__device__ __forceinline__ const int32_t *table_of(const EpP2PArgs &a, int rank) {
    return a.peers[rank].table + (size_t)a.parity * a.N * a.E;
}

constexpr int kPushThreads = 256;

__global__ void __launch_bounds__(kPushThreads) ep_push_kernel(EpP2PArgs a) {
    __shared__ int s_off[kEpMaxExperts + 1];
    __shared__ int s_dst[kEpMaxExperts];  // first recv row of (this rank, cold expert e), -1: overflow
    __shared__ int s_last;
    pdl_wait();
    const int tid = threadIdx.x;
    const EpPeer *P = a.peers;
    // 1. CTA 0 publishes this rank's counts into table[p] of every rank
    if (blockIdx.x == 0) {
        for (int i = tid; i < a.N * a.E; i += blockDim.x) {
            const int d = i / a.E, e = i - d * a.E;
            P[d].table[(size_t)a.parity * a.N * a.E + (size_t)a.me * a.E + e] = a.counts[e];
        }
        __syncthreads();
        if (tid < a.N) {
            __threadfence_system();
            st_release_sys(P[tid].flags + a.CNT() + a.me, a.epoch);
        }
    }
    // 2. every rank's counts
    if (tid < a.N && !wait_epoch(P[a.me].flags + a.CNT() + tid, a.epoch)) ep_error(a, 60);
    __syncthreads();
    for (int e = tid; e <= a.E; e += blockDim.x) s_off[e] = a.offsets[e];
    const int32_t *tab = table_of(a, a.me);
    for (int e = a.R + tid; e < a.E; e += blockDim.x) {
        const int d = (e - a.R) / a.C, j = (e - a.R) - d * a.C;
        const int e0 = a.R + d * a.C;
        int base = 0, total = 0, mine = 0;
        for (int src = 0; src < a.N; ++src) {
            const int32_t *row = tab + (size_t)src * a.E;
            for (int jj = 0; jj < a.C; ++jj) {
                const int c = row[e0 + jj];
                total += c;
                if (jj < j) base += c;
            }
            if (src < a.me) mine += row[e];
        }
        s_dst[e] = total <= a.max_recv ? base + mine : -1;
        if (total > a.max_recv) ep_error(a, 61);
    }
    __syncthreads();
    // 3. one warp per sorted row
    const int lane = tid & 31;
    const int rows = s_off[a.E];
    const size_t slot = (size_t)a.parity * a.max_recv * a.H;
    const int nv = a.H / 8;  // 16-byte vectors per row
    for (int i = (blockIdx.x * blockDim.x + tid) >> 5; i < rows;
         i += (gridDim.x * blockDim.x) >> 5) {
        int lo = 0, hi = a.E;  // expert e with s_off[e] <= i < s_off[e+1]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_off[mid] <= i) lo = mid;
            else hi = mid;
        }
        const int e = lo;
        const int pair = a.perm[i];
        if (e < a.R) {
            if (lane == 0) a.rowptr[pair] = a.back + (size_t)i * a.H;
            continue;
        }
        const int d = (e - a.R) / a.C;
        const int base = s_dst[e];
        if (base < 0) {
            if (lane == 0) a.rowptr[pair] = a.back + (size_t)i * a.H;  // rejected step
            continue;
        }
        const size_t r = (size_t)base + (i - s_off[e]);
        const uint4 *src = reinterpret_cast<const uint4 *>(a.rows + (size_t)i * a.H);
        uint4 *dst = reinterpret_cast<uint4 *>(P[d].recv + slot + r * a.H);
        for (int v = lane; v < nv; v += 32) dst[v] = __ldcs(src + v);
        if (lane == 0) a.rowptr[pair] = P[d].out + slot + r * a.H;
    }
    // 4. the last CTA tells every rank that this rank's rows are in place
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        const unsigned prev = atomicAdd(P[a.me].flags + a.CTR(), 1u);
        s_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
        if (tid == 0) P[a.me].flags[a.CTR()] = 0;
        if (tid < a.N) {
            __threadfence_system();
            st_release_sys(P[tid].flags + a.PUSH() + a.me, a.epoch);
        }
    }
}

// Owner side: every source's rows have arrived; group counts per local expert.
__global__ void ep_wait_recv_kernel(EpP2PArgs a) {
    pdl_wait();
    const int tid = threadIdx.x;
    if (tid < a.N && !wait_epoch(a.peers[a.me].flags + a.PUSH() + tid, a.epoch)) ep_error(a, 62);
    __syncthreads();
    const int32_t *tab = table_of(a, a.me);
    for (int j = tid; j < a.C; j += blockDim.x) {
        int n = 0;
        for (int src = 0; src < a.N; ++src) n += tab[(size_t)src * a.E + a.R + a.me * a.C + j];
        a.grp[j] = n;
    }
}

// Owner side: this rank's expert outputs for the step are complete.
__global__ void ep_done_kernel(EpP2PArgs a) {
    pdl_wait();
    if (threadIdx.x < a.N) {
        __threadfence_system();
        st_release_sys(a.peers[threadIdx.x].flags + a.DONE() + a.me, a.epoch);
    }
}

constexpr int kCombThreads = 128;

// out[t] = sum_k bf16(w[t,k] * row(t,k)) in k order, f32 accumulation, one
// bf16 rounding (the arithmetic of combine_kernel); rows local or remote.
__global__ void __launch_bounds__(kCombThreads) ep_combine_kernel(EpP2PArgs a,
                                                                  const uint16_t *__restrict__ w,
                                                                  int T, int K,
                                                                  uint16_t *__restrict__ out) {
    __shared__ const uint16_t *s_ptr[kEpMaxK];
    __shared__ float s_w[kEpMaxK];
    pdl_wait();
    const int tid = threadIdx.x;
    if (tid < a.N && !wait_epoch(a.peers[a.me].flags + a.DONE() + tid, a.epoch)) ep_error(a, 63);
    __syncthreads();
    const int nv = a.H / 8;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
        __syncthreads();
        for (int k = tid; k < K; k += blockDim.x) {
            s_ptr[k] = a.rowptr[(size_t)t * K + k];
            s_w[k] = bf2f(w[(size_t)t * K + k]);
        }
        __syncthreads();
        for (int v = tid; v < nv; v += blockDim.x) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            constexpr int B = 8;
            for (int k0 = 0; k0 < K; k0 += B) {
                uint4 o[B];
#pragma unroll
                for (int j = 0; j < B; ++j)
                    if (k0 + j < K) o[j] = __ldcg(reinterpret_cast<const uint4 *>(s_ptr[k0 + j]) + v);
#pragma unroll
                for (int j = 0; j < B; ++j) {
                    if (k0 + j >= K) continue;
                    float f[8];
                    unpack8(o[j], f);
                    const float wk = s_w[k0 + j];
#pragma unroll
                    for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], rbf(__fmul_rn(wk, f[q])));
                }
            }
            uint4 r;
            r.x = pack_bf2(acc[0], acc[1]);
            r.y = pack_bf2(acc[2], acc[3]);
            r.z = pack_bf2(acc[4], acc[5]);
            r.w = pack_bf2(acc[6], acc[7]);
            reinterpret_cast<uint4 *>(out + (size_t)t * a.H)[v] = r;
        }
    }
}

}  // namespace

cudaError_t launch_ep_push(const EpP2PArgs &a, int grid, cudaStream_t s) {
    ep_push_kernel<<<grid, kPushThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait_recv(const EpP2PArgs &a, cudaStream_t s) {
    ep_wait_recv_kernel<<<1, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_done(const EpP2PArgs &a, cudaStream_t s) {
    ep_done_kernel<<<1, 32, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const EpP2PArgs &a, const uint16_t *w, int T, int K, uint16_t *out,
                              int grid, cudaStream_t s) {
    if (K > kEpMaxK) return cudaErrorInvalidValue;
    ep_combine_kernel<<<grid, kCombThreads, 0, s>>>(a, w, T, K, out);
    return cudaGetLastError();
}

}  // namespace apt
