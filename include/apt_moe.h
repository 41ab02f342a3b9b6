/*
 * apt_moe.h -- C ABI of the B200-native Gemma-4 MoE block (ESRouter + ESExperts).
 *
 * Drop-in boundary for the reference's MoE section of ESDecoderLayer::forward
 * (aptransformer/ESDecoderLayer.mm:67-75).  The reference has no FFI: its
 * callers use the C++ classes es::ESRouter (aptransformer/ESRouter.h:17-34)
 * and es::ESExperts (aptransformer/ESExperts.h:17-41).  Each entry point below
 * replaces one of their members; the mapping is given beside it.
 *
 * Conventions
 *   - Every function returns apt_status (0 = APT_OK) and never throws.  The
 *     message of the last failure on a handle is apt_moe_last_error(h).
 *   - bf16 tensors are passed as uint16_t* holding raw bf16 bits, row-major.
 *   - Pointers marked "device" are CUDA device pointers on the handle's
 *     device; "host" pointers are ordinary host memory (pinned for speed).
 *   - Activation buffers ([T,H] / [rows,H] inputs and outputs) and norm
 *     weights must be 16-byte aligned (any CUDA allocation is); a misaligned
 *     one is refused with APT_ERR_INVALID.  Weights given to the loaders are
 *     copied and have no such requirement.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream).  All
 *     compute entry points are stream-ordered and asynchronous.
 *   - A handle is not re-entrant: callers serialise calls per handle.
 *   - Shapes: T tokens, H hidden_size, E num_experts, K top_k_experts,
 *     I moe_intermediate_size.
 */
#ifndef APT_MOE_H
#define APT_MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define APT_API __attribute__((visibility("default")))
#else
#define APT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int apt_status;
enum {
    APT_OK = 0,
    APT_ERR_INVALID = 1,      /* bad argument / shape                        */
    APT_ERR_UNSUPPORTED = 2,  /* unsupported bits / group size / shape       */
    APT_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed        */
    APT_ERR_NCCL = 4,         /* an NCCL call failed                         */
    APT_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up          */
    APT_ERR_STATE = 6         /* weights not loaded / wrong call order       */
};

typedef struct apt_moe_handle apt_moe_handle;

/*
 * MoE subset of ESModelConfig (aptransformer/ESModelConfig.h:135-157; parsed
 * from config.json text_config at ESModelConfig.mm:46-49).
 */
typedef struct apt_moe_config {
    int hidden_size;            /* H  (text_config.hidden_size)                */
    int num_experts;            /* E  (text_config.num_experts)                */
    int top_k_experts;          /* K  (text_config.top_k_experts)              */
    int moe_intermediate_size;  /* I  (text_config.moe_intermediate_size)      */
    float rms_norm_eps;         /* router RMSNorm eps (text_config.rms_norm_eps) */
    int enable_moe_block;       /* text_config.enable_moe_block                */
    int moe_sparse;             /* runtime: 1 = top-k gather path, 0 = dense    */
    int quant_bits;             /* runtime: 0 = bf16 experts, 4 or 8 = affine   */
    int quant_group_size;       /* runtime: affine group size (64)              */
    int max_tokens;             /* largest T per call; sizes the workspace      */
    int device;                 /* CUDA device ordinal                          */
} apt_moe_config;

/* Fill *cfg from the text of an HF config.json (top level or text_config).
 * Runtime knobs get the reference defaults: moe_sparse=0, quant_bits=0,
 * quant_group_size=64; max_tokens=8192, device=0.
 * Replaces ESModelConfig::fromConfigJSON (ESModelConfig.h:69) for these keys. */
APT_API apt_status apt_moe_config_from_json(const char *json_text, apt_moe_config *cfg);

/* Create a handle: validates the config, allocates the workspace for
 * max_tokens on cfg->device.  No weights yet.  hidden_size must be a multiple
 * of 64; moe_intermediate_size a multiple of 64, or of 8 for bf16 experts (the
 * handle then pads the experts with zero rows / columns to the next multiple
 * of 64, which leaves every output unchanged). */
APT_API apt_status apt_moe_create(const apt_moe_config *cfg, apt_moe_handle **out);
APT_API apt_status apt_moe_destroy(apt_moe_handle *h);

/*
 * A second handle on the same device weights (ESExperts / ESRouter instances
 * sharing mx::arrays, as several sessions of one model do): its own
 * workspace, streams, settings and error state, the weights shared and
 * read-only.  cfg may be NULL (same config) or differ from the source's only
 * in max_tokens, moe_sparse, rms_norm_eps and enable_moe_block.  Loading
 * weights into either handle afterwards returns APT_ERR_STATE.  The weights
 * are freed with the last handle that holds them; destroy order is free.
 */
APT_API apt_status apt_moe_clone_shared(apt_moe_handle *src, const apt_moe_config *cfg,
                                        apt_moe_handle **out);
APT_API const char *apt_moe_last_error(const apt_moe_handle *h);
/* Library version string (static). */
APT_API const char *apt_moe_version(void);

/*
 * Router weights (ESRouter ctor, ESRouter.mm:8-12): proj [E,H], scale [H],
 * per_expert_scale [E], bf16.  src_on_device: 0 = host pointers, 1 = device.
 */
APT_API apt_status apt_moe_load_router(apt_moe_handle *h, const uint16_t *proj, const uint16_t *scale,
                               const uint16_t *per_expert_scale, int src_on_device);

/*
 * bf16 expert weights in HF layout (ESExperts ctor, ESExperts.mm:8-19):
 * gate_up [E,2I,H] (gate = rows 0..I-1, up = rows I..2I-1), down [E,H,I].
 * If cfg.quant_bits > 0 the weights are quantised on the device (MLX affine,
 * group cfg.quant_group_size) exactly as the reference quantises at load.
 */
APT_API apt_status apt_moe_load_experts_bf16(apt_moe_handle *h, const uint16_t *gate_up,
                                     const uint16_t *down, int src_on_device);

/*
 * Pre-quantised expert weights in MLX affine format (ESExperts bundle ctor,
 * ESExperts.mm:21-26; esMakeExperts, ESWeightLoader.mm:145-154):
 *   gate_up: q [E,2I,H*bits/32] u32, scales/biases [E,2I,H/gs] bf16
 *   down:    q [E,H,I*bits/32]  u32, scales/biases [E,H,I/gs]  bf16
 * bits in {4,8}; gs = 64.  Values are adopted verbatim.
 */
APT_API apt_status apt_moe_load_experts_quant(apt_moe_handle *h, const uint32_t *gu_q,
                                      const uint16_t *gu_scales, const uint16_t *gu_biases,
                                      const uint32_t *dn_q, const uint16_t *dn_scales,
                                      const uint16_t *dn_biases, int bits, int group_size,
                                      int src_on_device);

/*
 * ESRouter::routeTopK (ESRouter.mm:14-32).  x [T,H] bf16 (device) ->
 * idx [T,K] int32 (descending probability), w [T,K] bf16 (device).
 */
APT_API apt_status apt_moe_route(apt_moe_handle *h, const uint16_t *x, int T, int32_t *idx,
                         uint16_t *w, void *stream);

/*
 * ESRouter::routeWeights (ESRouter.mm:34-40).  x [T,H] (device) ->
 * W [T,E] bf16 dense (device), zero except at the top-k experts.
 */
APT_API apt_status apt_moe_route_weights(apt_moe_handle *h, const uint16_t *x, int T, uint16_t *W,
                                 void *stream);

/*
 * ESExperts::sparseForward (ESExperts.mm:44-60).  x [T,H], idx [T,K] int32,
 * w [T,K] bf16 -> out [T,H] bf16; all device.  idx entries < 0 are skipped.
 */
APT_API apt_status apt_moe_experts(apt_moe_handle *h, const uint16_t *x, const int32_t *idx,
                           const uint16_t *w, int T, uint16_t *out, void *stream);

/*
 * ESExperts::forward (ESExperts.mm:28-42), the dense path: out[t] =
 * sum_e bf16(W[t,e] * expert_e(x[t])).  W [T,E] bf16 (device).  Experts with
 * W[t,e] == 0 contribute exactly zero and are not evaluated.
 */
APT_API apt_status apt_moe_experts_dense(apt_moe_handle *h, const uint16_t *x, const uint16_t *W,
                                 int T, uint16_t *out, void *stream);

/*
 * The MoE section of ESDecoderLayer::forward (ESDecoderLayer.mm:70-73):
 * router reads x_router (the raw residual x1), experts read x_experts
 * (pre_ff_ln_2(x1)); pass the same pointer for both in a block harness.
 * Honours cfg.moe_sparse (sparse vs dense dispatch) and the loaded weight
 * format.  idx_out / w_out (device, [T,K]) may be NULL.
 */
APT_API apt_status apt_moe_forward(apt_moe_handle *h, const uint16_t *x_router,
                           const uint16_t *x_experts, int T, uint16_t *out, int32_t *idx_out,
                           uint16_t *w_out, void *stream);

/*
 * The MoE half of ESDecoderLayer::forward with its norms (ESDecoderLayer.mm:
 * 69-74): out = post_ff_ln_2( experts( pre_ff_ln_2(x1), router(x1) ) ).
 * pre_ff_ln_2_w / post_ff_ln_2_w are the two RMSNorm weights [H] bf16
 * (device); eps = cfg.rms_norm_eps (ESRMSNorm.mm:14-28).  The pre-norm is
 * computed by the router kernels from the same sum of squares the router
 * uses; the post-norm is applied in the combine kernel.  (The dense MLP path
 * and post_ff_ln_1 that the layer adds to this are outside this library.)
 */
APT_API apt_status apt_moe_layer_forward(apt_moe_handle *h, const uint16_t *x1,
                                         const uint16_t *pre_ff_ln_2_w,
                                         const uint16_t *post_ff_ln_2_w, int T, uint16_t *out,
                                         void *stream);

/*
 * The whole feed-forward tail of an MoE decoder layer (ESDecoderLayer.mm:
 * 61-78) given the dense MLP output hmlp = mlp(pre_ff_ln(x1)):
 *   x2 = x1 + post_ff_ln( post_ff_ln_1(hmlp) + post_ff_ln_2(MoE(x1)) )
 * with the MoE block as in apt_moe_layer_forward.  Every RMSNorm is f32 with
 * one bf16 rounding (ESRMSNorm.mm:19-26), every add is bf16 + bf16 -> bf16.
 * The three trailing norms and the residual add run inside the combine
 * kernel.  x1, hmlp, x2 [T,H] bf16 on the device; x2 may not alias x1 or
 * hmlp.  The four weights are [H] bf16 on the device.
 */
APT_API apt_status apt_moe_decoder_ff(apt_moe_handle *h, const uint16_t *x1, const uint16_t *hmlp,
                                      const uint16_t *pre_ff_ln_2_w,
                                      const uint16_t *post_ff_ln_1_w,
                                      const uint16_t *post_ff_ln_2_w,
                                      const uint16_t *post_ff_ln_w, int T, uint16_t *x2,
                                      void *stream);

/*
 * The dense GeGLU MLP of the same layer (ESMLPBlock::forward, ESMLPBlock.mm:
 * 11-15): down(gelu(gate(x)) * up(x)) with the same rounding points as an
 * expert.  The handle is made with num_experts = top_k_experts = 1 and
 * moe_intermediate_size = the MLP's intermediate_size, and loaded with
 * apt_moe_load_experts_bf16 / _quant using gate_up = [gate_proj ; up_proj]
 * ([1, 2I, H]) and down = down_proj ([1, H, I]).  x, out [T, H] bf16 (device).
 */
APT_API apt_status apt_moe_mlp_forward(apt_moe_handle *h, const uint16_t *x, int T,
                                       uint16_t *out, void *stream);

/*
 * The whole feed-forward half of an MoE decoder layer (ESDecoderLayer.mm:
 * 61-78) with the dense MLP computed too:
 *   x2 = x1 + post_ff_ln( post_ff_ln_1(mlp(pre_ff_ln(x1)))
 *                         + post_ff_ln_2(MoE(pre_ff_ln_2(x1), router(x1))) )
 * `mlp` is an MLP handle (see apt_moe_mlp_forward) on the same device.
 */
APT_API apt_status apt_moe_decoder_ff_full(apt_moe_handle *moe, apt_moe_handle *mlp,
                                           const uint16_t *x1, const uint16_t *pre_ff_ln_w,
                                           const uint16_t *pre_ff_ln_2_w,
                                           const uint16_t *post_ff_ln_1_w,
                                           const uint16_t *post_ff_ln_2_w,
                                           const uint16_t *post_ff_ln_w, int T, uint16_t *x2,
                                           void *stream);

/*
 * Same as apt_moe_forward with HOST buffers: copies x to the device, runs
 * the block, copies out back and synchronises the stream.  x_host [T,H],
 * out_host [T,H] bf16.  Pinned (page-locked, hence device-mapped) 16-byte
 * aligned buffers are moved by kernels: x is read from the host buffer by a
 * staging kernel and the combine stores the result directly into out_host
 * (sparse configurations); other buffers go through cudaMemcpyAsync.  With
 * pinned buffers the sequence is captured once per
 * (T, x_host, out_host) as a CUDA graph and replayed on later calls, so a
 * pinned buffer passed here must stay allocated and pinned while the handle
 * is used with it (a freed buffer's address reused for pageable memory is
 * not detected).  Loading weights or changing a setting drops the graphs;
 * environment APT_NO_GRAPH=1 disables them.
 */
APT_API apt_status apt_moe_forward_host(apt_moe_handle *h, const uint16_t *x_host, int T,
                                uint16_t *out_host, void *stream);

/*
 * apt_moe_forward_host without the final synchronisation: the copy in, the
 * block and the copy out are queued on `stream` (x_host must stay unchanged
 * and out_host unread until the stream reaches that point, e.g. after
 * cudaStreamSynchronize or an event).  Consecutive calls on one handle are
 * ordered; a decode engine can queue several and wait once.
 */
APT_API apt_status apt_moe_forward_host_async(apt_moe_handle *h, const uint16_t *x_host, int T,
                                              uint16_t *out_host, void *stream);

/*
 * Expert parallelism (no reference counterpart: the reference is one device).
 * The block splits at the token exchange:
 *   apt_moe_ep_dispatch: router + top-K + dispatch on this rank's tokens, and the
 *     routed rows gathered in expert order into rows_out [T*K, H] (device);
 *     counts_out [E] (device) receives the per-expert row counts.  With experts
 *     numbered so that each rank owns a contiguous id range, rows_out is already
 *     grouped by destination rank: it is the all-to-all send buffer.
 *   (remote) apt_moe_experts on a handle holding the rank's local experts, with
 *     idx = local expert id, w = 1, K = 1, returns the unweighted expert rows.
 *   apt_moe_ep_combine: rows [T*K, H] returned in the same order as rows_out ->
 *     out [T,H] = sum_k bf16(w * row), in k order (ESExperts.mm:58-59), using
 *     the dispatch of the last apt_moe_ep_dispatch on this handle.
 */
APT_API apt_status apt_moe_ep_dispatch(apt_moe_handle *h, const uint16_t *x, int T, int32_t *idx,
                                       uint16_t *w, uint16_t *rows_out, int32_t *counts_out,
                                       void *stream);
APT_API apt_status apt_moe_ep_combine(apt_moe_handle *h, const uint16_t *rows, const int32_t *idx,
                                      const uint16_t *w, int T, uint16_t *out, void *stream);

/*
 * Expert-parallel remote compute on rows that arrive already grouped: R rows
 * [R,H] (device) in G consecutive groups of group_counts[g] rows (device,
 * int32 [G]); group g runs expert group_expert[g] (device, int32 [G]) of this
 * handle's bank.  out [R,H] receives the unweighted expert outputs in the
 * same row order.  No gather and no combine: the rows are consumed in place.
 * Requires R <= max_tokens * top_k_experts and G <= 256.
 */
APT_API apt_status apt_moe_experts_grouped(apt_moe_handle *h, const uint16_t *rows, int R,
                                           const int32_t *group_counts,
                                           const int32_t *group_expert, int G, uint16_t *out,
                                           void *stream);

/* Synchronise the handle's device and report any pending CUDA error. */
APT_API apt_status apt_moe_sync(apt_moe_handle *h);

/*
 * Self-test of the failure path: launches one thread that waits on a device
 * barrier nothing signals, through the same bounded wait the kernels use,
 * for about `microseconds`; it then records a timeout in the handle's error
 * word and returns.  The next apt_moe_sync reports APT_ERR_TIMEOUT (and clears
 * it); the context stays usable.
 */
APT_API apt_status apt_moe_selftest_wait(apt_moe_handle *h, int microseconds, void *stream);

/*
 * Introspection for tests and the bench: per-expert token counts of the last
 * dispatch (device -> host copy, synchronous), and kernel launch count of the
 * last compute call.
 */
APT_API apt_status apt_moe_last_counts(apt_moe_handle *h, int32_t *counts_host);
APT_API int apt_moe_last_launches(const apt_moe_handle *h);

/*
 * Path selection: the grouped expert kernels run as HBM-streaming GEMV when
 * T <= gemv_max_tokens and as tcgen05 tensor-core tiles otherwise.
 * Default 8.  Set to 0 to force the tensor-core path, to a huge value to
 * force the GEMV path (used by the parity tests).
 */
APT_API apt_status apt_moe_set_gemv_max_tokens(apt_moe_handle *h, int t);

/*
 * Decode form for T <= gemv_max_tokens (<= 8) with bf16 experts: 1 (default)
 * = the whole block -- router, dispatch, gate_up, down and the k-order
 * combine -- in one persistent kernel; 0 = the chain of router, GEMV and
 * combine kernels.  Same rounding points either way.  Calls with the layer
 * norms (apt_moe_layer_forward / decoder_ff) use the chain.
 */
APT_API apt_status apt_moe_set_fused_decode(apt_moe_handle *h, int on);

/*
 * Tensor-core form of 4-bit (group 64) experts above the decode sizes
 * (gather_qmm, aptransformer/ESExperts.mm:51,56): 1 (default) = the grouped
 * GEMMs dequantise each B tile in shared memory from the packed codes and
 * (scale, bias) pairs; 0 = every call first expands the experts it touches
 * to a bf16 scratch bank and runs the bf16 GEMMs on it.  Both feed the tensor
 * cores the same bf16 values w = bf16(scale * q + bias), so the outputs are
 * bitwise equal.  8-bit experts always use the expansion.
 */
APT_API apt_status apt_moe_set_q4_gemm(apt_moe_handle *h, int on);

/*
 * Cap on the SMs this handle's persistent kernels fill (0 = all, the
 * default).  Leaves room for kernels that must run beside them, e.g. NCCL's
 * all-to-all while the replicated experts of an expert-parallel step run.
 */
APT_API apt_status apt_moe_set_sm_limit(apt_moe_handle *h, int n);

/*
 * Per-stage timing for measurement: when enabled, every compute call records
 * a CUDA event pair on its stream around each stage's kernel;
 * apt_moe_stage_times fills ms[APT_STAGE_COUNT] with the last call's
 * durations (-1 for stages that did not run), synchronising on the events.
 * A stage that launched several times in one call reports its last launch.
 */
enum {
    APT_STAGE_ROUTER_SCORES = 0,
    APT_STAGE_ROUTER_SELECT = 1,
    APT_STAGE_DISPATCH_COUNT = 2,
    APT_STAGE_DISPATCH = 3,
    APT_STAGE_GATHER = 4,
    APT_STAGE_GATE_UP = 5,
    APT_STAGE_DOWN = 6,
    APT_STAGE_COMBINE = 7,
    APT_STAGE_COUNT = 8
};
APT_API apt_status apt_moe_set_timing(apt_moe_handle *h, int enable);
APT_API apt_status apt_moe_stage_times(apt_moe_handle *h, float *ms);

/*
 * Router without any allocation.  This entry point has no counterpart in the
 * reference: it exists for callers that may not allocate device memory while
 * they run -- code between a CUDA-graph-style memory plan and its replay, a
 * host runtime whose memory pool owns every device byte, or an embedding
 * (an FFI binding, a plugin) that receives only the buffers its host hands it.
 * It computes exactly what apt_moe_route computes, with the same kernels, but
 * takes every weight as a caller pointer and needs no handle.
 *
 * All pointers are device pointers: x [T,H] bf16, proj [E,H], scale [H],
 * per_expert_scale [E] bf16 -> idx [T,K] int32, w [T,K] bf16.
 * Its only scratch (the [T,E] f32 router scores) lives in a fixed array
 * compiled into the library, APT_NOALLOC_MAX_SCORES floats (64 KiB) per GPU,
 * held by every GPU that loads the library until the process exits; calls
 * with T * num_experts above that limit return APT_ERR_UNSUPPORTED (and print
 * the limit to stderr).  The first call on each device looks up that array's
 * device address (no allocation); make that first call outside any stream
 * capture.  Every call shares the array, so two calls that overlap on the GPU
 * (different streams, or different host threads) race; serialise them.
 * x, proj and scale must be 16-byte aligned (else APT_ERR_INVALID, nothing
 * launched).  If the score kernel's bounded wait for its staged rows runs
 * out, every idx of the call is written as -1 and every w as 0.  Calls made
 * after a cudaDeviceReset of the device are not supported.
 * Requires hidden_size % 64 == 0, num_experts <= 256, top_k <= min(32, E).
 */
#define APT_NOALLOC_MAX_SCORES 16384
APT_API apt_status apt_moe_route_noalloc(const uint16_t *x, int T, const uint16_t *proj,
                                         const uint16_t *scale, const uint16_t *per_expert_scale,
                                         int hidden_size, int num_experts, int top_k, float eps,
                                         int32_t *idx, uint16_t *w, void *stream);

/*
 * Expert parallelism as one C-ABI handle per GPU (no reference
 * counterpart): the hottest `replicate_hot` experts (by expected_loads, [E]
 * tokens per expert; NULL = uniform) are held by every rank, the others are
 * spread over the ranks by longest-processing-time placement; each forward
 * routes the rank's tokens, computes the replicated experts at home beside
 * the exchange of the other rows, computes the rank's own experts on the
 * rows it receives, returns the results and combines in k order.  The result
 * equals the single-GPU block on the same tokens (up to router ties, which
 * the relabelled expert ids may break the other way).  bf16 experts only.
 *
 * Two transports.  APT_EP_P2P (the default when every rank could map every
 * other rank's buffers through CUDA IPC at create): the library's own kernels
 * store the routed rows straight into their owners' memory over NVLink and
 * the combine loads the results straight from there, synchronised by
 * per-step flags in device memory -- no host synchronisation inside a step.
 * APT_EP_NCCL: NCCL send/recv with one host synchronisation per step for the
 * split sizes.  NCCL (resolved at run time, libnccl.so.2) also makes the
 * communicator that create and destroy use in both modes.
 *
 *   apt_moe_nccl_unique_id: 128-byte id for the ranks' communicator (rank 0
 *     makes it, the host distributes it)
 *   apt_moe_create_ep: cfg.max_tokens = tokens per rank per call; the
 *     communicator is created from nccl_id (collective over the ranks)
 *   apt_moe_ep_load_router / _experts_bf16: the FULL router and expert banks
 *     (every rank passes the same tensors; each keeps what it needs)
 *   apt_moe_ep_forward: x, out [T, H] bf16 on this rank's device
 *   apt_moe_ep_placement: the placement alone, perm[new id] = original id
 *   apt_moe_ep_stats: rows received / computed at home in the last forward
 *     (synchronises the device)
 *   apt_moe_ep_set_transport / _get_transport: APT_EP_P2P or APT_EP_NCCL
 *   apt_moe_ep_sync: synchronises the device; APT_ERR_TIMEOUT when a bounded
 *     wait of the peer-memory exchange (about 1 s) gave up -- that step's
 *     output is invalid (the error is then cleared)
 * apt_moe_ep_destroy is collective with the P2P transport (a rank's buffers
 * stay mapped by the others until all ranks destroy).
 */
#define APT_EP_NCCL 0
#define APT_EP_P2P 1
typedef struct apt_moe_ep apt_moe_ep;
APT_API apt_status apt_moe_nccl_unique_id(void *id_out);
APT_API apt_status apt_moe_create_ep(const apt_moe_config *cfg, const void *nccl_id, int rank,
                                     int nranks, const float *expected_loads, int replicate_hot,
                                     apt_moe_ep **out);
APT_API apt_status apt_moe_ep_destroy(apt_moe_ep *ep);
APT_API const char *apt_moe_ep_last_error(const apt_moe_ep *ep);
APT_API apt_status apt_moe_ep_load_router(apt_moe_ep *ep, const uint16_t *proj,
                                          const uint16_t *scale, const uint16_t *pes,
                                          int on_device);
APT_API apt_status apt_moe_ep_load_experts_bf16(apt_moe_ep *ep, const uint16_t *gate_up,
                                                const uint16_t *down, int on_device);
APT_API apt_status apt_moe_ep_forward(apt_moe_ep *ep, const uint16_t *x, int T, uint16_t *out,
                                      void *stream);
APT_API apt_status apt_moe_ep_placement(const float *loads, int E, int nranks, int n_hot,
                                        int32_t *perm_out);
APT_API apt_status apt_moe_ep_stats(apt_moe_ep *ep, int *recv_rows, int *hot_rows);
APT_API apt_status apt_moe_ep_set_transport(apt_moe_ep *ep, int transport);
APT_API apt_status apt_moe_ep_get_transport(const apt_moe_ep *ep, int *transport);
APT_API apt_status apt_moe_ep_sync(apt_moe_ep *ep);

#ifdef __cplusplus
}
#endif

#endif /* APT_MOE_H */
