// moe_internal.h -- kernel launchers shared between the .cu files of libapt_moe.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

struct apt_moe_handle;

namespace apt {

// Routing / dispatch state of one call, all device pointers.
struct Dispatch {
    int32_t *counts;    // [E]   tokens routed to each expert
    int32_t *offsets;   // [E+1] exclusive scan of counts (offsets[E] = rows)
    int32_t *perm;      // [P]   sorted row -> pair id (t*K + k)
    int32_t *inv;       // [P]   pair id -> sorted row
    int32_t *active;    // [E]   experts with counts > 0, ascending
    int32_t *n_active;  // [1]
};

// Per-device one-time kernel attribute set-up (called with the device current).
cudaError_t router_init();
cudaError_t gemv_init();
cudaError_t gemm_init();

// ---- router (router.cu)
// scores [T,E] f32 = (((x*rsqrt(mean(x^2)+eps))*scale)*H^-1/2) . proj^T
// err (optional): set to 30 by the T <= 64 kernel when its staged rows never arrive
cudaError_t launch_router_scores(const uint16_t *x, const uint16_t *proj, const uint16_t *scale,
                                 int T, int H, int E, float eps, float *scores,
                                 cudaStream_t s, int *launches, int32_t *err = nullptr);
// softmax + top-K + renorm + per-expert scale; optional per-expert counts
// rank (optional, needs counts): each pair's slot in its expert group (atomic)
// err (optional): when the word is non-zero (the score kernel's bounded wait
// gave up), every idx of the call is written as -1 and every w as 0
cudaError_t launch_router_select(const float *scores, const uint16_t *pes, int T, int E, int K,
                                 int32_t *idx, uint16_t *w, int32_t *counts, cudaStream_t s,
                                 int *launches, int32_t *rank = nullptr,
                                 const int32_t *err = nullptr, const uint16_t *x = nullptr,
                                 int H = 0, float eps = 0.f);
// Decode-sized fused router + dispatch (one launch): writes idx/w and the full
// Dispatch.  `done` is a zero-initialised device counter the kernel resets.
bool router_dispatch_fusable(int T, int H, int E, int K);
cudaError_t launch_router_dispatch(const uint16_t *x, const uint16_t *proj, const uint16_t *scale,
                                   const uint16_t *pes, int T, int H, int E, int K, float eps,
                                   float *scores, int32_t *idx, uint16_t *w, const Dispatch &d,
                                   int32_t *done, cudaStream_t s, int *launches,
                                   const uint16_t *pre_w = nullptr, uint16_t *xn = nullptr,
                                   int32_t *err = nullptr);
// Tensor-core router path: (scale * H^-1/2 * proj) folded at load into a
// two-term bf16 split [E, 2H]; the f32-output tcgen05 GEMM reads the token
// rows directly (gemm_sm100.cu) and router_select applies the RMS factor
// (launch_router_select with x).
cudaError_t launch_router_fold_split(const uint16_t *proj, const uint16_t *scale, int H, int E,
                                     uint16_t *pw, cudaStream_t s);
// out = RMSNorm(x) * w (ESRMSNorm.mm:14-28), one warp per row
// idx[i] = 0, w[i] = bf16 1.0 for i < n: every row to the single "expert"
// of a dense GeGLU MLP handle
cudaError_t launch_fill_mlp_routing(int32_t *idx, uint16_t *w, int n, cudaStream_t s,
                                    int *launches);
cudaError_t launch_rmsnorm(const uint16_t *x, const uint16_t *w, int T, int H, float eps,
                          uint16_t *out, cudaStream_t s, int *launches);
cudaError_t launch_gemm_router(const uint16_t *x, const uint16_t *projw, int T, int H, int E,
                               float *scores, int32_t *err, cudaStream_t s, int *launches);
// dense routeWeights scatter: W [T,E] = 0 except W[t, idx[t,k]] = w[t,k]
cudaError_t launch_scatter_dense(const int32_t *idx, const uint16_t *w, int T, int E, int K,
                                 uint16_t *W, cudaStream_t s, int *launches);
// dense W [T,E] -> pair lists idx2/w2 [T,E] (nonzero experts in index order, rest -1)
cudaError_t launch_dense_to_pairs(const uint16_t *W, int T, int E, int32_t *idx2, uint16_t *w2,
                                  int32_t *counts, cudaStream_t s, int *launches);

// ---- dispatch (dispatch.cu)
cudaError_t launch_count(const int32_t *idx, int P, int E, int32_t *counts, cudaStream_t s,
                         int *launches);
cudaError_t launch_dispatch(const int32_t *idx, int P, int E, const Dispatch &d, cudaStream_t s,
                            int *launches);
// Dispatch from per-pair slots (router_select's rank output): offsets,
// active list, perm and inv in one launch
cudaError_t launch_place(const int32_t *idx, const int32_t *rank, int P, int E, const Dispatch &d,
                         cudaStream_t s, int *launches);
// xp[row] = x[perm[row] / K] for row < offsets[E].  With the routing (idx, T)
// and a bounded-wait error sink, prefill-sized calls run token-major on bulk
// copies (each x row read once).
cudaError_t launch_gather_rows(const uint16_t *x, int H, int K, int E, const Dispatch &d,
                               int max_rows, uint16_t *xp, cudaStream_t s, int *launches,
                               const int32_t *idx = nullptr, int T = 0, int32_t *err = nullptr);
// dst[0, bytes) = src[0, bytes) by a kernel (bytes % 16 == 0, both 16-byte
// aligned; src may be mapped pinned host memory)
cudaError_t launch_copy16(const void *src, void *dst, size_t bytes, cudaStream_t s,
                          int *launches);
// Optional norms around the MoE output, applied by the combine
// (ESDecoderLayer.mm:66-78).  post_w alone: out = post_ff_ln_2(moe).  With
// mlp (+ mlp_w, ff_w, resid): out = resid + post_ff_ln(post_ff_ln_1(mlp) +
// post_ff_ln_2(moe)).  All weights [H] bf16 on the device.
struct CombineTail {
    const uint16_t *post_w;  // post_ff_ln_2
    const uint16_t *mlp;     // dense MLP output [T,H]
    const uint16_t *mlp_w;   // post_ff_ln_1
    const uint16_t *ff_w;    // post_ff_ln
    const uint16_t *resid;   // x1 [T,H]
    float eps;
};
// out[t] = bf16( sum_k f32(bf16(w[t,k] * op[inv[t*K+k]])) ), then the tail.  With
// err (bounded-wait error sink) and T >= 2 x SMs the bulk-copy form runs.
cudaError_t launch_combine(const uint16_t *op, const int32_t *idx, const uint16_t *w,
                           const Dispatch &d, int T, int K, int H, uint16_t *out,
                           cudaStream_t s, int *launches, const CombineTail *tail = nullptr,
                           int32_t *err = nullptr);

// ---- decode GEMV (gemv.cu).  Weight formats: bits == 0 -> bf16, else affine.
struct ExpertWeights {
    const uint16_t *gu, *dn;                // bf16 [E,2I,H], [E,H,I]
    const uint32_t *gu_q, *dn_q;            // packed
    const uint16_t *gu_s, *gu_b, *dn_s, *dn_b;
    const uint32_t *gu_sb, *dn_sb;          // interleaved (scale, bias) pairs
    const uint32_t *gu_qd, *dn_qd;          // 4-bit codes in the decode block's fragment order
    int bits, gs;
};
// max_rows_per_expert bounds counts[e] for this call (T for top-k routing).
cudaError_t launch_gemv_gateup(const uint16_t *x, int K, const Dispatch &d, const ExpertWeights &w,
                               int H, int I, int E, int max_rows_per_expert, uint16_t *yp,
                               cudaStream_t s, int *launches);
cudaError_t launch_gemv_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w, int H,
                             int I, int E, int max_rows_per_expert, uint16_t *op, cudaStream_t s,
                             int *launches);

// ---- decode GEMV with TMA-streamed bf16 weights (gemv_tma.cu)
cudaError_t gemv_tma_init();
bool gemv_tma_supported(int H, int I);
cudaError_t launch_gemv_tma_gateup(const uint16_t *x, int K, const Dispatch &d,
                                   const ExpertWeights &w, int H, int I, int E, int max_rows,
                                   uint16_t *yp, int32_t *err, cudaStream_t s, int *launches);
cudaError_t launch_gemv_tma_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                                 int H, int I, int E, int max_k, int max_rows, uint16_t *op, int32_t *err,
                                 cudaStream_t s, int *launches);

// ---- decode GEMV with TMA-streamed MLX affine 4/8-bit weights (gemv_tma_q.cu)
bool gemv_tma_q_supported(int H, int I, int bits);
cudaError_t launch_gemv_tma_q_gateup(const uint16_t *x, int K, const Dispatch &d,
                                     const ExpertWeights &w, int H, int I, int E, int max_rows,
                                     uint16_t *yp, int32_t *err, cudaStream_t s, int *launches);
cudaError_t launch_gemv_tma_q_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                                   int H, int I, int E, int max_k, int max_rows, uint16_t *op,
                                   int32_t *err, cudaStream_t s, int *launches);

// ---- prefill grouped GEMM (gemm_sm100.cu), bf16 tcgen05 tiles
struct GemmPlan;  // opaque, owns tensor maps
bool gemm_supported(int H, int I);
cudaError_t launch_gemm_gateup(const uint16_t *xp, const Dispatch &d, const ExpertWeights &w,
                               int rows_cap, int H, int I, int E, uint16_t *yp, int32_t *err,
                               cudaStream_t s, int *launches);
// gate_up with A rows gathered by the TMA from x [T, H] through d.perm (no
// separate gather launch); same results as gather + launch_gemm_gateup.
cudaError_t launch_gemm_gateup_gather(const uint16_t *x, int T, int Kp, const Dispatch &d,
                                      const ExpertWeights &w, int rows_cap, int H, int I, int E,
                                      uint16_t *yp, int32_t *err, cudaStream_t s, int *launches);
// max_group_rows: bound on rows per expert for this call (0 = unknown)
cudaError_t launch_gemm_down(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                             int rows_cap, int H, int I, int E, uint16_t *op, int32_t *err,
                             cudaStream_t s, int *launches, int max_group_rows = 0);

// Grouped variants: G row groups (counts/offsets in d), group g uses the
// weights of expert g2e[g]; rows are consumed in place (no gather).
cudaError_t launch_gemm_gateup_grouped(const uint16_t *rows, const Dispatch &d,
                                       const int32_t *g2e, const ExpertWeights &w, int rows_cap,
                                       int H, int I, int E_w, int G, uint16_t *yp, int32_t *err,
                                       cudaStream_t s, int *launches);
cudaError_t launch_gemm_down_grouped(const uint16_t *yp, const Dispatch &d, const int32_t *g2e,
                                     const ExpertWeights &w, int rows_cap, int H, int I, int E_w,
                                     int G, uint16_t *out, int32_t *err, cudaStream_t s,
                                     int *launches);

// offsets = exclusive scan of G group counts (one CTA); offsets[G] = total
cudaError_t launch_group_offsets(const int32_t *counts, int G, int32_t *offsets, cudaStream_t s,
                                 int *launches);

// ---- quantisation (quant.cu)
cudaError_t launch_quantize_affine(const uint16_t *w, int64_t rows, int cols, int gs, int bits,
                                   uint32_t *q, uint16_t *sc, uint16_t *bi, cudaStream_t s);
// (scale, bias) pairs interleaved per group: [rows, groups] uint32
// Self-test of the bounded device wait: expires after limit_cycles and records
// error code 99 (quant.cu).
cudaError_t launch_selftest_wait(long long limit_cycles, int32_t *err, cudaStream_t s);

// Interleaved (scale, bias) pairs of `rows` rows of g groups each, rows padded
// to sb_row_words(g * 64) words (zeros), for the quantised TMA GEMV.
inline int sb_row_words(int len) { return ((len / 64) + 3) / 4 * 4; }
// 4-bit experts on the tensor cores, B tiles dequantised in shared memory
// (gemm_sm100.cu); A rows tiled (the expert-sorted copy xp / yp).
bool gemm_q4_supported(int H, int I);
cudaError_t launch_gemm_gateup_q4(const uint16_t *xp, const Dispatch &d, const ExpertWeights &w,
                                  int rows_cap, int H, int I, int E, uint16_t *yp, int32_t *err,
                                  cudaStream_t s, int *launches);
cudaError_t launch_gemm_down_q4(const uint16_t *yp, const Dispatch &d, const ExpertWeights &w,
                                int rows_cap, int H, int I, int E, uint16_t *op, int32_t *err,
                                cudaStream_t s, int *launches);
cudaError_t launch_interleave_sb(const uint16_t *sc, const uint16_t *bi, int64_t rows, int g,
                                 uint32_t *out, cudaStream_t s);
// bf16 copy of the active experts' quantised rows (prefill path)
// 4-bit codes re-ordered for the one-kernel decode block (quant.cu):
// gate_up items of 16 intermediate columns (32 rows x H) and down items of
// 128 rows x I, each one contiguous block in its mma.sync fragment order.
cudaError_t launch_repack_q4_decode(const uint32_t *gu_q, const uint32_t *dn_q, int E, int H, int I,
                                    uint32_t *gu_qd, uint32_t *dn_qd, cudaStream_t s);
cudaError_t launch_dequant_active(const uint32_t *q, const uint16_t *sc, const uint16_t *bi,
                                  int rows, int cols, int bits, const Dispatch &d, int E,
                                  uint16_t *out, cudaStream_t s, int *launches);

// ---- expert parallelism over NVLink peer memory (ep_p2p.cu)
constexpr int kEpMaxExperts = 256;
constexpr int kEpMaxK = 32;
constexpr int kEpMaxRanks = 16;
// One rank's shared region as seen from this process (own or IPC-mapped).
struct EpPeer {
    uint32_t *flags;  // [3N+2]
    int32_t *table;   // [2][N][E]
    uint16_t *recv;   // [2][max_recv][H]
    uint16_t *out;    // [2][max_recv][H]
};
struct EpP2PArgs {
    const EpPeer *peers;  // device array [N]
    int N, me, R, C, E, H, max_recv, parity;
    uint32_t epoch;
    const int32_t *counts, *offsets, *perm;  // this rank's dispatch (new expert ids)
    const uint16_t *rows;                    // sorted routed rows [P, H]
    uint16_t *back;                          // hot-expert outputs [P, H] (sorted rows)
    const uint16_t **rowptr;                 // [P] pair -> address of its expert output
    int32_t *grp;                            // [C] group counts of this rank's experts
    __host__ __device__ int CNT() const { return 0; }
    __host__ __device__ int PUSH() const { return N; }
    __host__ __device__ int DONE() const { return 2 * N; }
    __host__ __device__ int CTR() const { return 3 * N; }
    __host__ __device__ int ERR() const { return 3 * N + 1; }
};
cudaError_t launch_ep_push(const EpP2PArgs &a, int grid, cudaStream_t s);
cudaError_t launch_ep_wait_recv(const EpP2PArgs &a, cudaStream_t s);
cudaError_t launch_ep_done(const EpP2PArgs &a, cudaStream_t s);
cudaError_t launch_ep_combine(const EpP2PArgs &a, const uint16_t *w, int T, int K, uint16_t *out,
                              int grid, cudaStream_t s);
// ---- the whole decode block in one persistent kernel (decode_fused.cu):
// router, dispatch, gate_up, down and combine for T <= 8; bf16 experts, or
// 4/8-bit MLX affine experts with 64-element groups (wt.bits, wt.gs).
// sync: decode_fused_sync_words(E, H, I) int32 (counters and the tagged
// GeGLU / down rows), zeroed once before the first call; the kernel keeps it
// consistent from call to call itself.
cudaError_t decode_fused_init();
bool decode_fused_supported(int T, int H, int I, int E, int K, bool same_x, int bits, int gs);
size_t decode_fused_sync_words(int E, int H, int I);
cudaError_t launch_decode_fused(const uint16_t *xr, const uint16_t *xe, const uint16_t *proj,
                                const uint16_t *scale, const uint16_t *pes, int T, int H, int E,
                                int K, int I, float eps, float *scores, int32_t *idx, uint16_t *w,
                                const Dispatch &d, const ExpertWeights &wt, uint16_t *out,
                                int32_t *sync, int32_t *err, cudaStream_t s, int *launches);

// The dispatch (counts, offsets, perm, inv) of the last routing call on h.
Dispatch handle_dispatch(apt_moe_handle *h);

}  // namespace apt
