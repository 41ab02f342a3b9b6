// api.cu -- the C ABI (include/apt_moe.h): handle, weights, workspace, and the
// ESRouter / ESExperts entry points.
//
// Reference interface each entry point replaces (paths within the reference):
//   apt_moe_route          ESRouter::routeTopK       aptransformer/ESRouter.mm:14-32
//   apt_moe_route_weights  ESRouter::routeWeights    aptransformer/ESRouter.mm:34-40
//   apt_moe_experts        ESExperts::sparseForward  aptransformer/ESExperts.mm:44-60
//   apt_moe_experts_dense  ESExperts::forward        aptransformer/ESExperts.mm:28-42
//   apt_moe_forward        MoE section of ESDecoderLayer::forward, ESDecoderLayer.mm:67-75
//   apt_moe_load_*         ESRouter / ESExperts ctors, esMakeExperts (ESWeightLoader.mm:145-154)
//   apt_moe_config_from_json  ESModelConfig::fromConfigJSON MoE keys (ESModelConfig.mm:46-49)
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <memory>
#include <initializer_list>
#include <vector>

#include "../../include/apt_moe.h"
#include "moe_internal.h"
#include "launch_util.h"

using namespace apt;

// Device weight buffers shared by handles made with apt_moe_clone_shared: freed
// when the last handle holding them is destroyed.
struct WeightOwner {
    int device = 0;
    std::vector<void *> ptrs;
    ~WeightOwner() {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        for (void *p : ptrs) cudaFree(p);
        if (prev >= 0) cudaSetDevice(prev);
    }
};

struct apt_moe_handle {
    apt_moe_config cfg{};
    std::string err;
    int launches = 0;
    int gemv_max_tokens = 8;
    int sm_limit = 0;      // cap on SMs for persistent grids (0: all)
    bool gemv_tma = true;  // TMA-streamed bf16 GEMV (else the register-prefetch GEMV)
    bool fused_decode = true;  // whole decode block in one kernel (decode_fused.cu)
    bool q4_gemm = true;       // 4-bit experts: dequantise B tiles inside the tcgen05 GEMMs
    // moe_intermediate_size as given when it is not a multiple of 64: the
    // handle then runs I rounded up to 64, the extra gate / up rows and down
    // columns zero (GeGLU of a zero row is exactly 0, and a zero column adds
    // exactly 0), so the outputs are those of the given I
    int I_user = 0;

    // per-stage CUDA-event timing (apt_moe_set_timing / apt_moe_stage_times)
    bool timing = false;
    cudaEvent_t ev[APT_STAGE_COUNT][2] = {};

    // apt_moe_forward_host replays a CUDA graph of (copy in, block, copy out)
    // per (T, host buffers): one launch instead of a copy, ~5 kernels and a
    // copy.  Captured on a private stream (the legacy default stream cannot
    // be captured) and launched on the caller's; any change of weights or
    // settings drops the cache.
    struct HostGraph {
        int T;
        const void *x;
        void *out;
        cudaGraphExec_t exec;
        int launches;
    };
    std::vector<HostGraph> graphs;
    cudaStream_t gstream = nullptr;
    bool ev_used[APT_STAGE_COUNT] = {};

    // router
    uint16_t *proj = nullptr, *scale = nullptr, *pes = nullptr;
    // (scale * H^-1/2 * proj) as a two-term bf16 split [E, 2H], folded at load
    // for the tensor-core router (T > 64)
    uint16_t *projw = nullptr;
    // experts, bf16 (kept when quantised from bf16 so the dense path works)
    uint16_t *gu = nullptr, *dn = nullptr;
    // per-call bf16 expansion of the touched quantised experts for the
    // tensor-core path (scratch of this handle, allocated at first use)
    uint16_t *dq_gu = nullptr, *dq_dn = nullptr;
    // experts, affine quantised
    uint32_t *gu_q = nullptr, *dn_q = nullptr;
    uint16_t *gu_s = nullptr, *gu_b = nullptr, *dn_s = nullptr, *dn_b = nullptr;
    uint32_t *gu_sb = nullptr, *dn_sb = nullptr;  // (scale, bias) pairs, per-row contiguous
    // 4-bit codes re-ordered for the one-kernel decode block's mma.sync
    // fragments (repack_q4_decode_kernel); the MLX-format gu_q / dn_q stay the
    // source of every other path
    uint32_t *gu_qd = nullptr, *dn_qd = nullptr;
    int qbits = 0, qgs = 64;
    // set when the weights above are shared with other handles (read-only then)
    std::shared_ptr<WeightOwner> wowner;

    // workspace
    int Tm = 0, Pcap = 0;
    float *scores = nullptr;     // [Tm, E] (tensor-core router: two planes [2][T][E])
    int32_t *idx_i = nullptr;
    uint16_t *w_i = nullptr;
    int32_t *counts = nullptr, *offsets = nullptr, *perm = nullptr, *inv = nullptr;
    int32_t *active = nullptr, *n_active = nullptr, *errflag = nullptr;
    int32_t *done = nullptr;    // fused decode router's completion counter (self-resetting)
    int32_t *fsync = nullptr;   // one-kernel decode block's counters (self re-arming)
    // router rows x of the current call when h->scores holds the tensor-core
    // router's raw x . (scale * H^-1/2 * proj) (router_select applies the RMS
    // factor); nullptr when the scores are final
    const uint16_t *rs_x = nullptr;
    uint16_t *xp = nullptr, *yp = nullptr, *op = nullptr;
    uint16_t *Wd = nullptr;     // dense routing matrix [Tm,E]
    int32_t *idx2 = nullptr;    // dense pair lists [Pcap]
    uint16_t *w2 = nullptr;
    uint16_t *xin = nullptr, *xout = nullptr;  // host-API staging [Tm,H]
    uint16_t *xn = nullptr;                    // pre_ff_ln_2(x1) [Tm,H] (layer entry point)
    CombineTail cur_tail{};                    // norms the current call's combine applies

    Dispatch disp() const { return Dispatch{counts, offsets, perm, inv, active, n_active}; }
};

namespace {

apt_status fail(apt_moe_handle *h, apt_status code, const char *fmt, ...) {
    if (h) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        h->err = buf;
    }
    return code;
}

#define CUDA_TRY(h, expr)                                                                    \
    do {                                                                                     \
        cudaError_t e_ = (expr);                                                             \
        if (e_ != cudaSuccess)                                                               \
            return fail((h), APT_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_),  \
                        __FILE__, __LINE__);                                                 \
    } while (0)

template <class T>
cudaError_t dalloc(T **p, size_t n) {
    return cudaMalloc(reinterpret_cast<void **>(p), n * sizeof(T) + 256);
}

void dfree(void *p) {
    if (p) cudaFree(p);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

apt_status copy_in(apt_moe_handle *h, void *dst, const void *src, size_t bytes, int on_device) {
    CUDA_TRY(h, cudaMemcpy(dst, src, bytes, on_device ? cudaMemcpyDeviceToDevice
                                                      : cudaMemcpyHostToDevice));
    return APT_OK;
}

ExpertWeights weights_for(const apt_moe_handle *h, bool quant) {
    ExpertWeights w{};
    w.gu = h->gu;
    w.dn = h->dn;
    if (quant) {
        w.gu_q = h->gu_q;
        w.dn_q = h->dn_q;
        w.gu_s = h->gu_s;
        w.gu_b = h->gu_b;
        w.dn_s = h->dn_s;
        w.dn_b = h->dn_b;
        w.gu_sb = h->gu_sb;
        w.dn_sb = h->dn_sb;
        w.gu_qd = h->gu_qd;
        w.dn_qd = h->dn_qd;
        w.bits = h->qbits;
        w.gs = h->qgs;
    }
    return w;
}

struct StageScope {
    apt_moe_handle *h;
    int id;
    cudaStream_t s;
    StageScope(apt_moe_handle *h_, int id_, cudaStream_t s_) : h(h_), id(id_), s(s_) {
        if (h->timing) cudaEventRecord(h->ev[id][0], s);
    }
    ~StageScope() {
        if (h->timing) {
            cudaEventRecord(h->ev[id][1], s);
            h->ev_used[id] = true;
        }
    }
};

// Run one launch inside a timed stage scope.
#define STAGE(h, id, s, expr)                    \
    do {                                         \
        StageScope sc_((h), (id), (s));          \
        CUDA_TRY((h), (expr));                   \
    } while (0)

// The handle's weight buffers (what apt_moe_clone_shared shares).
std::vector<void **> weight_fields(apt_moe_handle *h) {
    return {reinterpret_cast<void **>(&h->proj),  reinterpret_cast<void **>(&h->scale),
            reinterpret_cast<void **>(&h->pes),   reinterpret_cast<void **>(&h->gu),
            reinterpret_cast<void **>(&h->dn),    reinterpret_cast<void **>(&h->gu_q),
            reinterpret_cast<void **>(&h->dn_q),  reinterpret_cast<void **>(&h->gu_s),
            reinterpret_cast<void **>(&h->gu_b),  reinterpret_cast<void **>(&h->dn_s),
            reinterpret_cast<void **>(&h->dn_b),  reinterpret_cast<void **>(&h->gu_sb),
            reinterpret_cast<void **>(&h->dn_sb), reinterpret_cast<void **>(&h->projw),
            reinterpret_cast<void **>(&h->gu_qd), reinterpret_cast<void **>(&h->dn_qd)};
}

void drop_graphs(apt_moe_handle *h) {
    for (auto &g : h->graphs) cudaGraphExecDestroy(g.exec);
    h->graphs.clear();
}

// Activations and norm weights are read and written with 16-byte vector
// accesses and bulk copies, so each such device pointer must be 16-byte
// aligned (what any allocator returns).  Checked at the entry points.
bool aligned16(std::initializer_list<const void *> ps) {
    for (const void *p : ps)
        if (reinterpret_cast<uintptr_t>(p) & 15) return false;
    return true;
}

#define CHECK_ALIGNED(h, ...)                                                                \
    do {                                                                                     \
        if (!aligned16({__VA_ARGS__}))                                                       \
            return fail((h), APT_ERR_INVALID, "activation / norm buffers must be 16-byte aligned"); \
    } while (0)

void begin_call(apt_moe_handle *h) {
    h->launches = 0;
    sm_cap() = h->sm_limit;
    for (int i = 0; i < APT_STAGE_COUNT; ++i) h->ev_used[i] = false;
}

// ---- tiny config.json reader (MoE keys only)

const char *find_key(const char *begin, const char *end, const char *key) {
    std::string pat = std::string("\"") + key + "\"";
    const char *p = begin;
    while (p < end) {
        const char *q = strstr(p, pat.c_str());
        if (!q || q >= end) return nullptr;
        const char *c = q + pat.size();
        while (c < end && (*c == ' ' || *c == '\t' || *c == '\n' || *c == '\r')) ++c;
        if (c < end && *c == ':') {
            ++c;
            while (c < end && (*c == ' ' || *c == '\t' || *c == '\n' || *c == '\r')) ++c;
            return c;
        }
        p = q + 1;
    }
    return nullptr;
}

bool read_num(const char *b, const char *e, const char *key, double *out) {
    const char *v = find_key(b, e, key);
    if (!v) return false;
    if (!strncmp(v, "true", 4)) { *out = 1; return true; }
    if (!strncmp(v, "false", 5)) { *out = 0; return true; }
    if (!strncmp(v, "null", 4)) return false;
    char *endp = nullptr;
    double d = strtod(v, &endp);
    if (endp == v) return false;
    *out = d;
    return true;
}

}  // namespace

// ------------------------------------------------------------------ config

extern "C" apt_status apt_moe_config_from_json(const char *json, apt_moe_config *cfg) {
    if (!json || !cfg) return APT_ERR_INVALID;
    memset(cfg, 0, sizeof *cfg);
    cfg->rms_norm_eps = 1e-6f;
    cfg->quant_group_size = 64;
    cfg->max_tokens = 8192;
    const char *b = json, *e = json + strlen(json);
    // prefer the text_config object when present (multimodal Gemma-4 configs)
    const char *tc = find_key(b, e, "text_config");
    if (tc && *tc == '{') {
        int depth = 0;
        const char *p = tc;
        for (; p < e; ++p) {
            if (*p == '{') ++depth;
            else if (*p == '}' && --depth == 0) break;
        }
        b = tc;
        e = p;
    }
    double v;
    if (read_num(b, e, "hidden_size", &v)) cfg->hidden_size = (int)v;
    if (read_num(b, e, "num_experts", &v)) cfg->num_experts = (int)v;
    if (read_num(b, e, "top_k_experts", &v)) cfg->top_k_experts = (int)v;
    if (read_num(b, e, "moe_intermediate_size", &v)) cfg->moe_intermediate_size = (int)v;
    if (read_num(b, e, "rms_norm_eps", &v)) cfg->rms_norm_eps = (float)v;
    if (read_num(b, e, "enable_moe_block", &v)) cfg->enable_moe_block = v != 0.0;
    return APT_OK;
}

extern "C" const char *apt_moe_version(void) { return "apt_moe 0.1 (sm_100a)"; }

// ------------------------------------------------------------------ lifecycle

extern "C" apt_status apt_moe_create(const apt_moe_config *cfg, apt_moe_handle **out) {
    if (!cfg || !out) return APT_ERR_INVALID;
    *out = nullptr;
    const int H = cfg->hidden_size, E = cfg->num_experts, K = cfg->top_k_experts,
              I = cfg->moe_intermediate_size;
    if (H <= 0 || E <= 0 || K <= 0 || I <= 0 || cfg->max_tokens <= 0) return APT_ERR_INVALID;
    const bool pad_i = I % 64 != 0;
    if (H % 64 || (pad_i && (I % 8 || cfg->quant_bits)) || E > 256 || K > 32 || K > E)
        return APT_ERR_UNSUPPORTED;
    if (cfg->quant_bits && !((cfg->quant_bits == 4 || cfg->quant_bits == 8) &&
                             cfg->quant_group_size == 64))
        return APT_ERR_UNSUPPORTED;
    apt_moe_handle *h = new apt_moe_handle();
    h->cfg = *cfg;
    if (pad_i) {
        h->I_user = I;
        h->cfg.moe_intermediate_size = (I + 63) / 64 * 64;
    }
    if (cfg->max_tokens > (1 << 24) / K) {
        delete h;
        return APT_ERR_UNSUPPORTED;
    }
    DeviceGuard g(cfg->device);
    h->Tm = cfg->max_tokens;
    h->Pcap = h->Tm * K;
    cudaError_t e1 = cudaSuccess;
#define ALLOC(p, n) if (e1 == cudaSuccess) e1 = dalloc(&h->p, (size_t)(n))
    ALLOC(scores, 2 * (size_t)h->Tm * E);  // two partial planes on the tensor-core router
    ALLOC(idx_i, h->Pcap);
    ALLOC(w_i, h->Pcap);
    ALLOC(counts, E);
    ALLOC(offsets, E + 1);
    ALLOC(perm, h->Pcap);
    ALLOC(inv, h->Pcap);
    ALLOC(active, E);
    ALLOC(n_active, 1);
    ALLOC(errflag, 4);
    ALLOC(done, 16);
    ALLOC(xp, (size_t)h->Pcap * H);
    ALLOC(yp, (size_t)h->Pcap * I);
    ALLOC(op, (size_t)h->Pcap * H);
    ALLOC(Wd, (size_t)h->Tm * E);
    ALLOC(idx2, h->Pcap);
    ALLOC(w2, h->Pcap);
    ALLOC(xin, (size_t)h->Tm * H);
    ALLOC(xout, (size_t)h->Tm * H);
    ALLOC(xn, (size_t)h->Tm * H);
    ALLOC(fsync, decode_fused_sync_words(E, H, h->cfg.moe_intermediate_size));
#undef ALLOC
    if (e1 == cudaSuccess) e1 = router_init();
    if (e1 == cudaSuccess) e1 = gemv_init();
    if (e1 == cudaSuccess) e1 = gemm_init();
    if (e1 == cudaSuccess) e1 = gemv_tma_init();
    if (e1 == cudaSuccess) e1 = decode_fused_init();
    if (e1 == cudaSuccess)
        e1 = cudaMemset(h->fsync, 0, sizeof(int32_t) * decode_fused_sync_words(E, H, h->cfg.moe_intermediate_size));
    if (e1 == cudaSuccess) e1 = cudaMemset(h->errflag, 0, 16);
    if (e1 == cudaSuccess) e1 = cudaMemset(h->done, 0, 16 * sizeof(int32_t));
    for (int i = 0; i < APT_STAGE_COUNT && e1 == cudaSuccess; ++i)
        for (int j = 0; j < 2 && e1 == cudaSuccess; ++j) e1 = cudaEventCreate(&h->ev[i][j]);
    if (e1 != cudaSuccess) {
        apt_moe_destroy(h);
        return APT_ERR_CUDA;
    }
    *out = h;
    return APT_OK;
}

extern "C" apt_status apt_moe_destroy(apt_moe_handle *h) {
    if (!h) return APT_OK;
    DeviceGuard g(h->cfg.device);
    if (h->wowner) {  // shared weights: freed by their owner with the last handle
        for (void **f : weight_fields(h))
            for (void *p : h->wowner->ptrs)
                if (*f == p) *f = nullptr;
        h->wowner.reset();
    }
    void *ptrs[] = {h->proj, h->scale, h->pes, h->gu, h->dn, h->gu_q, h->dn_q, h->gu_s, h->gu_b,
                    h->dn_s, h->dn_b, h->scores, h->idx_i, h->w_i, h->counts, h->offsets,
                    h->perm, h->inv, h->active, h->n_active, h->errflag, h->done, h->projw, h->xp, h->yp, h->op,
                    h->Wd, h->idx2, h->w2, h->xin, h->xout, h->dq_gu, h->dq_dn, h->gu_sb, h->dn_sb, h->xn, h->fsync, h->gu_qd, h->dn_qd};
    for (void *p : ptrs) dfree(p);
    drop_graphs(h);
    if (h->gstream) cudaStreamDestroy(h->gstream);
    for (int i = 0; i < APT_STAGE_COUNT; ++i)
        for (int j = 0; j < 2; ++j)
            if (h->ev[i][j]) cudaEventDestroy(h->ev[i][j]);
    delete h;
    return APT_OK;
}

extern "C" apt_status apt_moe_clone_shared(apt_moe_handle *src, const apt_moe_config *cfg,
                                           apt_moe_handle **out) {
    if (!src || !out) return APT_ERR_INVALID;
    *out = nullptr;
    if (!src->proj) return fail(src, APT_ERR_STATE, "router weights not loaded");
    apt_moe_config c = src->cfg;
    if (cfg) {  // the clone may differ in workspace size and sparse/dense switch only
        if (cfg->hidden_size != c.hidden_size || cfg->num_experts != c.num_experts ||
            cfg->top_k_experts != c.top_k_experts ||
            cfg->moe_intermediate_size != c.moe_intermediate_size ||
            cfg->quant_bits != c.quant_bits || cfg->device != c.device)
            return fail(src, APT_ERR_INVALID, "clone config differs in shape, format or device");
        c.max_tokens = cfg->max_tokens;
        c.moe_sparse = cfg->moe_sparse;
        c.rms_norm_eps = cfg->rms_norm_eps;
        c.enable_moe_block = cfg->enable_moe_block;
    }
    apt_moe_handle *h = nullptr;
    if (apt_status st = apt_moe_create(&c, &h)) return st;
    DeviceGuard g(src->cfg.device);
    if (!src->wowner) {  // hand the source's weight buffers to a shared owner
        src->wowner = std::make_shared<WeightOwner>();
        src->wowner->device = src->cfg.device;
        for (void **f : weight_fields(src))
            if (*f) src->wowner->ptrs.push_back(*f);
    }
    h->wowner = src->wowner;
    std::vector<void **> to = weight_fields(h), from = weight_fields(src);
    for (size_t i = 0; i < to.size(); ++i) {
        bool shared = false;
        for (void *p : src->wowner->ptrs) shared |= (*from[i] == p);
        *to[i] = shared ? *from[i] : nullptr;  // the dequantised cache stays per handle
    }
    h->qbits = src->qbits;
    h->qgs = src->qgs;
    *out = h;
    return APT_OK;
}

extern "C" const char *apt_moe_last_error(const apt_moe_handle *h) {
    return h ? h->err.c_str() : "null handle";
}

extern "C" apt_status apt_moe_set_gemv_max_tokens(apt_moe_handle *h, int t) {
    if (!h) return APT_ERR_INVALID;
    drop_graphs(h);
    h->gemv_max_tokens = t;
    return APT_OK;
}

extern "C" apt_status apt_moe_set_sm_limit(apt_moe_handle *h, int n) {
    if (!h || n < 0) return APT_ERR_INVALID;
    drop_graphs(h);
    h->sm_limit = n;
    return APT_OK;
}

extern "C" apt_status apt_moe_set_fused_decode(apt_moe_handle *h, int on) {
    if (!h || on < 0 || on > 1) return APT_ERR_INVALID;
    drop_graphs(h);
    h->fused_decode = on != 0;
    return APT_OK;
}

extern "C" apt_status apt_moe_set_q4_gemm(apt_moe_handle *h, int on) {
    if (!h || on < 0 || on > 1) return APT_ERR_INVALID;
    drop_graphs(h);
    h->q4_gemm = on != 0;
    return APT_OK;
}

extern "C" apt_status apt_moe_set_timing(apt_moe_handle *h, int enable) {
    if (!h) return APT_ERR_INVALID;
    drop_graphs(h);
    h->timing = enable != 0;
    return APT_OK;
}

extern "C" apt_status apt_moe_stage_times(apt_moe_handle *h, float *ms) {
    if (!h || !ms) return APT_ERR_INVALID;
    DeviceGuard g(h->cfg.device);
    for (int i = 0; i < APT_STAGE_COUNT; ++i) {
        ms[i] = -1.f;
        if (!h->ev_used[i]) continue;
        CUDA_TRY(h, cudaEventSynchronize(h->ev[i][1]));
        CUDA_TRY(h, cudaEventElapsedTime(&ms[i], h->ev[i][0], h->ev[i][1]));
    }
    return APT_OK;
}

extern "C" int apt_moe_last_launches(const apt_moe_handle *h) { return h ? h->launches : -1; }

extern "C" apt_status apt_moe_last_counts(apt_moe_handle *h, int32_t *counts_host) {
    if (!h || !counts_host) return APT_ERR_INVALID;
    DeviceGuard g(h->cfg.device);
    CUDA_TRY(h, cudaDeviceSynchronize());
    CUDA_TRY(h, cudaMemcpy(counts_host, h->counts, sizeof(int32_t) * h->cfg.num_experts,
                           cudaMemcpyDeviceToHost));
    return APT_OK;
}

extern "C" apt_status apt_moe_sync(apt_moe_handle *h) {
    if (!h) return APT_ERR_INVALID;
    DeviceGuard g(h->cfg.device);
    CUDA_TRY(h, cudaDeviceSynchronize());
    int32_t ef[4] = {0, 0, 0, 0};
    CUDA_TRY(h, cudaMemcpy(ef, h->errflag, sizeof ef, cudaMemcpyDeviceToHost));
    if (ef[0]) {
        cudaMemset(h->errflag, 0, sizeof ef);
        return fail(h, APT_ERR_TIMEOUT, "device wait gave up (code %d, at %d)", ef[0], ef[1]);
    }
    return APT_OK;
}

extern "C" apt_status apt_moe_selftest_wait(apt_moe_handle *h, int microseconds, void *stream) {
    if (!h || microseconds <= 0 || microseconds > 10000000) return APT_ERR_INVALID;
    DeviceGuard g(h->cfg.device);
    int khz = 0;
    CUDA_TRY(h, cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, h->cfg.device));
    const long long cycles = (long long)khz * microseconds / 1000;  // at the rated clock
    CUDA_TRY(h, launch_selftest_wait(cycles, h->errflag, (cudaStream_t)stream));
    return APT_OK;
}

// ------------------------------------------------------------------ weights

namespace {
apt_status build_sb(apt_moe_handle *h) {
    const size_t H = h->cfg.hidden_size, E = h->cfg.num_experts, I = h->cfg.moe_intermediate_size;
    const size_t gu_rows = E * 2 * I, dn_rows = E * H;
    dfree(h->gu_sb);
    dfree(h->dn_sb);
    h->gu_sb = h->dn_sb = nullptr;
    CUDA_TRY(h, dalloc(&h->gu_sb, gu_rows * sb_row_words((int)H)));
    CUDA_TRY(h, dalloc(&h->dn_sb, dn_rows * sb_row_words((int)I)));
    CUDA_TRY(h, launch_interleave_sb(h->gu_s, h->gu_b, (int64_t)gu_rows, (int)H / 64, h->gu_sb, 0));
    CUDA_TRY(h, launch_interleave_sb(h->dn_s, h->dn_b, (int64_t)dn_rows, (int)I / 64, h->dn_sb, 0));
    dfree(h->gu_qd);
    dfree(h->dn_qd);
    h->gu_qd = h->dn_qd = nullptr;
    if (h->qbits == 4 && h->qgs == 64 && H % 256 == 0 && H % 128 == 0 && I % 64 == 0) {
        // the decode block's fragment-ordered copy of the codes (same size as gu_q / dn_q)
        CUDA_TRY(h, dalloc(&h->gu_qd, gu_rows * H / 8));
        CUDA_TRY(h, dalloc(&h->dn_qd, dn_rows * I / 8));
        CUDA_TRY(h, launch_repack_q4_decode(h->gu_q, h->dn_q, (int)E, (int)H, (int)I, h->gu_qd,
                                            h->dn_qd, 0));
    }
    CUDA_TRY(h, cudaDeviceSynchronize());
    return APT_OK;
}
}  // namespace

extern "C" apt_status apt_moe_load_router(apt_moe_handle *h, const uint16_t *proj,
                                          const uint16_t *scale, const uint16_t *pes,
                                          int on_device) {
    if (!h || !proj || !scale || !pes) return fail(h, APT_ERR_INVALID, "null router weight");
    DeviceGuard g(h->cfg.device);
    drop_graphs(h);
    if (h->wowner)
        return fail(h, APT_ERR_STATE, "weights are shared with another handle (read-only)");
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts;
    if (!h->proj) {
        CUDA_TRY(h, dalloc(&h->proj, (size_t)E * H));
        CUDA_TRY(h, dalloc(&h->scale, (size_t)H));
        CUDA_TRY(h, dalloc(&h->pes, (size_t)E));
        CUDA_TRY(h, dalloc(&h->projw, (size_t)E * 2 * H));
    }
    apt_status st;
    if ((st = copy_in(h, h->proj, proj, sizeof(uint16_t) * E * H, on_device))) return st;
    if ((st = copy_in(h, h->scale, scale, sizeof(uint16_t) * H, on_device))) return st;
    if ((st = copy_in(h, h->pes, pes, sizeof(uint16_t) * E, on_device))) return st;
    CUDA_TRY(h, launch_router_fold_split(h->proj, h->scale, H, E, h->projw, 0));
    CUDA_TRY(h, cudaDeviceSynchronize());
    return APT_OK;
}

extern "C" apt_status apt_moe_load_experts_bf16(apt_moe_handle *h, const uint16_t *gate_up,
                                                const uint16_t *down, int on_device) {
    if (!h || !gate_up || !down) return fail(h, APT_ERR_INVALID, "null expert weight");
    DeviceGuard g(h->cfg.device);
    drop_graphs(h);
    if (h->wowner)
        return fail(h, APT_ERR_STATE, "weights are shared with another handle (read-only)");
    const size_t H = h->cfg.hidden_size, E = h->cfg.num_experts, I = h->cfg.moe_intermediate_size;
    if (!h->gu) {
        CUDA_TRY(h, dalloc(&h->gu, E * 2 * I * H));
        CUDA_TRY(h, dalloc(&h->dn, E * H * I));
    }
    apt_status st;
    if (h->I_user) {
        // [E, 2*Iu, H] and [E, H, Iu] into the zero-padded [E, 2*I, H], [E, H, I]
        const size_t Iu = h->I_user;
        CUDA_TRY(h, cudaMemset(h->gu, 0, sizeof(uint16_t) * E * 2 * I * H));
        CUDA_TRY(h, cudaMemset(h->dn, 0, sizeof(uint16_t) * E * H * I));
        for (size_t e = 0; e < E; ++e)
            for (size_t half = 0; half < 2; ++half)
                CUDA_TRY(h, cudaMemcpy(h->gu + (e * 2 * I + half * I) * H,
                                       gate_up + (e * 2 * Iu + half * Iu) * H,
                                       sizeof(uint16_t) * Iu * H, cudaMemcpyDefault));
        CUDA_TRY(h, cudaMemcpy2D(h->dn, I * 2, down, Iu * 2, Iu * 2, E * H, cudaMemcpyDefault));
        CUDA_TRY(h, cudaDeviceSynchronize());
    } else {
        if ((st = copy_in(h, h->gu, gate_up, sizeof(uint16_t) * E * 2 * I * H, on_device)))
            return st;
        if ((st = copy_in(h, h->dn, down, sizeof(uint16_t) * E * H * I, on_device))) return st;
    }
    if (h->cfg.quant_bits) {
        // ESExperts ctor with quantBits > 0 (ESExperts.mm:13-18): quantise at load,
        // keep bf16 for the dense path.
        const int bits = h->cfg.quant_bits, gs = h->cfg.quant_group_size;
        if (!h->gu_q) {
            CUDA_TRY(h, dalloc(&h->gu_q, E * 2 * I * H * bits / 32));
            CUDA_TRY(h, dalloc(&h->dn_q, E * H * I * bits / 32));
            CUDA_TRY(h, dalloc(&h->gu_s, E * 2 * I * H / gs));
            CUDA_TRY(h, dalloc(&h->gu_b, E * 2 * I * H / gs));
            CUDA_TRY(h, dalloc(&h->dn_s, E * H * I / gs));
            CUDA_TRY(h, dalloc(&h->dn_b, E * H * I / gs));
        }
        CUDA_TRY(h, launch_quantize_affine(h->gu, (int64_t)E * 2 * I, (int)H, gs, bits, h->gu_q,
                                           h->gu_s, h->gu_b, 0));
        CUDA_TRY(h, launch_quantize_affine(h->dn, (int64_t)E * H, (int)I, gs, bits, h->dn_q,
                                           h->dn_s, h->dn_b, 0));
        CUDA_TRY(h, cudaDeviceSynchronize());
        h->qbits = bits;
        h->qgs = gs;
        if (apt_status st = build_sb(h)) return st;
    }
    return APT_OK;
}

extern "C" apt_status apt_moe_load_experts_quant(apt_moe_handle *h, const uint32_t *gu_q,
                                                 const uint16_t *gu_s, const uint16_t *gu_b,
                                                 const uint32_t *dn_q, const uint16_t *dn_s,
                                                 const uint16_t *dn_b, int bits, int gs,
                                                 int on_device) {
    if (!h || !gu_q || !gu_s || !gu_b || !dn_q || !dn_s || !dn_b)
        return fail(h, APT_ERR_INVALID, "null quantised expert weight");
    if (h->I_user)
        return fail(h, APT_ERR_UNSUPPORTED, "quantised experts need moe_intermediate_size % 64 == 0");
    if (!((bits == 4 || bits == 8) && gs == 64))
        return fail(h, APT_ERR_UNSUPPORTED, "bits=%d group=%d (need bits 4|8, group 64)", bits, gs);
    DeviceGuard g(h->cfg.device);
    drop_graphs(h);
    if (h->wowner)
        return fail(h, APT_ERR_STATE, "weights are shared with another handle (read-only)");
    const size_t H = h->cfg.hidden_size, E = h->cfg.num_experts, I = h->cfg.moe_intermediate_size;
    dfree(h->gu_q); dfree(h->dn_q); dfree(h->gu_s); dfree(h->gu_b); dfree(h->dn_s); dfree(h->dn_b);
    h->gu_q = h->dn_q = nullptr;
    h->gu_s = h->gu_b = h->dn_s = h->dn_b = nullptr;
    CUDA_TRY(h, dalloc(&h->gu_q, E * 2 * I * H * bits / 32));
    CUDA_TRY(h, dalloc(&h->dn_q, E * H * I * bits / 32));
    CUDA_TRY(h, dalloc(&h->gu_s, E * 2 * I * H / gs));
    CUDA_TRY(h, dalloc(&h->gu_b, E * 2 * I * H / gs));
    CUDA_TRY(h, dalloc(&h->dn_s, E * H * I / gs));
    CUDA_TRY(h, dalloc(&h->dn_b, E * H * I / gs));
    apt_status st;
    if ((st = copy_in(h, h->gu_q, gu_q, 4 * E * 2 * I * H * bits / 32, on_device))) return st;
    if ((st = copy_in(h, h->dn_q, dn_q, 4 * E * H * I * bits / 32, on_device))) return st;
    if ((st = copy_in(h, h->gu_s, gu_s, 2 * E * 2 * I * H / gs, on_device))) return st;
    if ((st = copy_in(h, h->gu_b, gu_b, 2 * E * 2 * I * H / gs, on_device))) return st;
    if ((st = copy_in(h, h->dn_s, dn_s, 2 * E * H * I / gs, on_device))) return st;
    if ((st = copy_in(h, h->dn_b, dn_b, 2 * E * H * I / gs, on_device))) return st;
    // a bundle carries no bf16 experts (ESExperts.mm:21-26): dense path unavailable
    dfree(h->gu);
    dfree(h->dn);
    h->gu = h->dn = nullptr;
    h->qbits = bits;
    h->qgs = gs;
    return build_sb(h);
}

// ------------------------------------------------------------------ compute

namespace {

// Routed rows (T*K) up to which gate_up gathers its A rows itself.
constexpr int kGatherInGemmRows = 4096;

apt_status check_T(apt_moe_handle *h, int T) {
    if (T < 0 || T > h->Tm)
        return fail(h, APT_ERR_INVALID, "T=%d outside [0, max_tokens=%d]", T, h->Tm);
    return APT_OK;
}

// Router scores [T,E] f32 into h->scores: tensor-core GEMM on the folded
// weights for prefill-sized T (raw scores; h->rs_x = x tells router_select to
// apply the RMS factor), f32 SIMT kernels otherwise (final scores).
apt_status router_scores(apt_moe_handle *h, const uint16_t *x, int T, cudaStream_t s,
                         const uint16_t *pre_w = nullptr) {
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts;
    if (pre_w)
        STAGE(h, APT_STAGE_ROUTER_SCORES, s,
              launch_rmsnorm(x, pre_w, T, H, h->cfg.rms_norm_eps, h->xn, s, &h->launches));
    if (T > 64 && E % 64 == 0 && gemm_supported(H, h->cfg.moe_intermediate_size)) {
        STAGE(h, APT_STAGE_ROUTER_SCORES, s,
              launch_gemm_router(x, h->projw, T, H, E, h->scores, h->errflag, s, &h->launches));
        h->rs_x = x;
        return APT_OK;
    }
    h->rs_x = nullptr;
    STAGE(h, APT_STAGE_ROUTER_SCORES, s,
          launch_router_scores(x, h->proj, h->scale, T, H, E, h->cfg.rms_norm_eps, h->scores, s,
                               &h->launches));
    return APT_OK;
}

// Grouped experts over an already-dispatched pair list, then the combine.
// idx/w: [T, Kp] pair lists (Kp = K for sparse, E for dense).
apt_status run_experts(apt_moe_handle *h, const uint16_t *x, const int32_t *idx,
                       const uint16_t *w, int T, int Kp, bool quant, uint16_t *out,
                       cudaStream_t s, bool dispatched = false) {
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts, I = h->cfg.moe_intermediate_size;
    const int P = T * Kp;
    Dispatch d = h->disp();
    if (!dispatched)
        STAGE(h, APT_STAGE_DISPATCH, s, launch_dispatch(idx, P, E, d, s, &h->launches));
    ExpertWeights ew = weights_for(h, quant);
    const int max_rows = T;  // an expert appears at most once per token
    const bool gemm = T > h->gemv_max_tokens && gemm_supported(H, I);
    // 4-bit experts: the GEMMs dequantise their B tiles in shared memory
    const bool q4 = gemm && quant && h->qbits == 4 && h->qgs == 64 && h->q4_gemm &&
                    gemm_q4_supported(H, I);
    if (gemm && quant && !q4) {
        // The bf16 GEMM on the dequantised experts (w = scale*q + bias, rounded
        // to bf16 as MLX's dequantise does).  Every call expands the experts
        // it touches (the dispatch's active list) into a scratch bank laid out
        // like the bf16 weights, then runs the bf16 GEMM on it; the scratch is
        // allocated at the first tensor-core-sized call (1.5 GB at the
        // Gemma-4 shape) and nothing of it is reused between calls.
        if (!h->dq_gu) {
            CUDA_TRY(h, dalloc(&h->dq_gu, (size_t)E * 2 * I * H));
            CUDA_TRY(h, dalloc(&h->dq_dn, (size_t)E * H * I));
        }
        STAGE(h, APT_STAGE_GATHER, s,
              launch_dequant_active(h->gu_q, h->gu_s, h->gu_b, 2 * I, H, h->qbits, d, E,
                                    h->dq_gu, s, &h->launches));
        STAGE(h, APT_STAGE_GATHER, s,
              launch_dequant_active(h->dn_q, h->dn_s, h->dn_b, H, I, h->qbits, d, E,
                                    h->dq_dn, s, &h->launches));
        ew.gu = h->dq_gu;
        ew.dn = h->dq_dn;
    }
    if (gemm) {
        const int rows_cap = P < h->Pcap ? P : h->Pcap;
        // Few rows per expert: A rows gathered inside the GEMM (tile::gather4);
        // prefill-sized groups: one gather pass, then full-tile TMA copies.
        const bool gather_in_gemm = rows_cap <= kGatherInGemmRows && !q4;
        if (!gather_in_gemm)
            STAGE(h, APT_STAGE_GATHER, s,
                  launch_gather_rows(x, H, Kp, E, d, rows_cap, h->xp, s, &h->launches, idx, T,
                                     h->errflag));
        if (q4) {
            STAGE(h, APT_STAGE_GATE_UP, s,
                  launch_gemm_gateup_q4(h->xp, d, ew, rows_cap, H, I, E, h->yp, h->errflag, s,
                                        &h->launches));
            STAGE(h, APT_STAGE_DOWN, s,
                  launch_gemm_down_q4(h->yp, d, ew, rows_cap, H, I, E, h->op, h->errflag, s,
                                      &h->launches));
        } else if (gather_in_gemm)
            STAGE(h, APT_STAGE_GATE_UP, s,
                  launch_gemm_gateup_gather(x, T, Kp, d, ew, rows_cap, H, I, E, h->yp,
                                            h->errflag, s, &h->launches));
        else
            STAGE(h, APT_STAGE_GATE_UP, s,
                  launch_gemm_gateup(h->xp, d, ew, rows_cap, H, I, E, h->yp, h->errflag, s,
                                     &h->launches));
        if (!q4)
            STAGE(h, APT_STAGE_DOWN, s,
                  launch_gemm_down(h->yp, d, ew, rows_cap, H, I, E, h->op, h->errflag, s,
                                   &h->launches, max_rows));
    } else if (quant && h->gemv_tma && gemv_tma_q_supported(H, I, h->qbits)) {
        STAGE(h, APT_STAGE_GATE_UP, s,
              launch_gemv_tma_q_gateup(x, Kp, d, ew, H, I, E, max_rows, h->yp, h->errflag, s,
                                       &h->launches));
        STAGE(h, APT_STAGE_DOWN, s,
              launch_gemv_tma_q_down(h->yp, d, ew, H, I, E, Kp, max_rows, h->op, h->errflag, s,
                                     &h->launches));
    } else if (!quant && h->gemv_tma && gemv_tma_supported(H, I)) {
        STAGE(h, APT_STAGE_GATE_UP, s, launch_gemv_tma_gateup(x, Kp, d, ew, H, I, E, max_rows, h->yp,
                                                              h->errflag, s, &h->launches));
        STAGE(h, APT_STAGE_DOWN, s, launch_gemv_tma_down(h->yp, d, ew, H, I, E, Kp, max_rows, h->op,
                                                         h->errflag, s, &h->launches));
    } else {
        STAGE(h, APT_STAGE_GATE_UP, s, launch_gemv_gateup(x, Kp, d, ew, H, I, E, max_rows, h->yp, s, &h->launches));
        STAGE(h, APT_STAGE_DOWN, s, launch_gemv_down(h->yp, d, ew, H, I, E, max_rows, h->op, s, &h->launches));
    }
    STAGE(h, APT_STAGE_COMBINE, s,
          launch_combine(h->op, idx, w, d, T, Kp, H, out, s, &h->launches,
                         h->cur_tail.post_w ? &h->cur_tail : nullptr, h->errflag));
    return APT_OK;
}

apt_status experts_sparse(apt_moe_handle *h, const uint16_t *x, const int32_t *idx,
                          const uint16_t *w, int T, uint16_t *out, cudaStream_t s,
                          bool counts_ready) {
    const int E = h->cfg.num_experts, K = h->cfg.top_k_experts;
    const bool quant = h->qbits > 0;
    if (!quant && !h->gu) return fail(h, APT_ERR_STATE, "expert weights not loaded");
    if (quant && !h->gu_q) return fail(h, APT_ERR_STATE, "quantised expert weights not loaded");
    if (!counts_ready) {
        CUDA_TRY(h, cudaMemsetAsync(h->counts, 0, sizeof(int32_t) * E, s));
        STAGE(h, APT_STAGE_DISPATCH_COUNT, s, launch_count(idx, T * K, E, h->counts, s, &h->launches));
    }
    return run_experts(h, x, idx, w, T, K, quant, out, s);
}

apt_status experts_dense(apt_moe_handle *h, const uint16_t *x, const uint16_t *W, int T,
                         uint16_t *out, cudaStream_t s) {
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts;
    if (!h->gu)
        return fail(h, APT_ERR_STATE,
                    "dense expert path needs bf16 experts (unavailable from a quantised bundle)");
    // chunks small enough that even a fully dense W fits the pair workspace
    const int chunk = h->Pcap / E > 0 ? h->Pcap / E : 1;
    for (int t0 = 0; t0 < T; t0 += chunk) {
        const int tc = T - t0 < chunk ? T - t0 : chunk;
        CUDA_TRY(h, cudaMemsetAsync(h->counts, 0, sizeof(int32_t) * E, s));
        STAGE(h, APT_STAGE_DISPATCH_COUNT, s, launch_dense_to_pairs(W + (size_t)t0 * E, tc, E, h->idx2, h->w2, h->counts, s,
                                          &h->launches));
        apt_status st = run_experts(h, x + (size_t)t0 * H, h->idx2, h->w2, tc, E, false,
                                    out + (size_t)t0 * H, s);
        if (st) return st;
    }
    return APT_OK;
}

}  // namespace

extern "C" apt_status apt_moe_route(apt_moe_handle *h, const uint16_t *x, int T, int32_t *idx,
                                    uint16_t *w, void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (!h->proj) return fail(h, APT_ERR_STATE, "router weights not loaded");
    if (T == 0) return APT_OK;
    if (!x || !idx || !w) return fail(h, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(h, x);
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    begin_call(h);
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts, K = h->cfg.top_k_experts;
    (void)H;
    if (apt_status st = router_scores(h, x, T, s)) return st;
    STAGE(h, APT_STAGE_ROUTER_SELECT, s, launch_router_select(h->scores, h->pes, T, E, K, idx, w, nullptr, s,
                                     &h->launches, nullptr, nullptr, h->rs_x, H,
                                     h->cfg.rms_norm_eps));
    return APT_OK;
}

extern "C" apt_status apt_moe_route_weights(apt_moe_handle *h, const uint16_t *x, int T,
                                            uint16_t *W, void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!W) return fail(h, APT_ERR_INVALID, "null pointer");
    apt_status st = apt_moe_route(h, x, T, h->idx_i, h->w_i, stream);
    if (st) return st;
    DeviceGuard g(h->cfg.device);
    STAGE(h, APT_STAGE_ROUTER_SELECT, (cudaStream_t)stream, launch_scatter_dense(h->idx_i, h->w_i, T, h->cfg.num_experts,
                                     h->cfg.top_k_experts, W, (cudaStream_t)stream,
                                     &h->launches));
    return APT_OK;
}

extern "C" apt_status apt_moe_experts(apt_moe_handle *h, const uint16_t *x, const int32_t *idx,
                                      const uint16_t *w, int T, uint16_t *out, void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x || !idx || !w || !out) return fail(h, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(h, x, out);
    DeviceGuard g(h->cfg.device);
    begin_call(h);
    return experts_sparse(h, x, idx, w, T, out, (cudaStream_t)stream, false);
}

extern "C" apt_status apt_moe_experts_dense(apt_moe_handle *h, const uint16_t *x,
                                            const uint16_t *W, int T, uint16_t *out,
                                            void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x || !W || !out) return fail(h, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(h, x, out);
    DeviceGuard g(h->cfg.device);
    begin_call(h);
    return experts_dense(h, x, W, T, out, (cudaStream_t)stream);
}

namespace {
// The MoE section of ESDecoderLayer::forward.  With pre_w, the expert input is
// pre_ff_ln_2(x_router) computed on the way (x_experts ignored); with a tail,
// the norms after the block (post_ff_ln_2, and optionally post_ff_ln_1 of the
// dense MLP, post_ff_ln and the residual add) are fused into the combine.
apt_status forward_impl(apt_moe_handle *h, const uint16_t *x_router, const uint16_t *x_experts,
                        int T, uint16_t *out, int32_t *idx_out, uint16_t *w_out, void *stream,
                        const uint16_t *pre_w, const CombineTail *tail) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x_router || !out) return fail(h, APT_ERR_INVALID, "null pointer");
    if (!x_experts) x_experts = x_router;
    CHECK_ALIGNED(h, x_router, x_experts, out, pre_w);
    if (!h->proj) return fail(h, APT_ERR_STATE, "router weights not loaded");
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    begin_call(h);
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts, K = h->cfg.top_k_experts;
    int32_t *idx = idx_out ? idx_out : h->idx_i;
    uint16_t *w = w_out ? w_out : h->w_i;
    if (pre_w) x_experts = h->xn;
    if (tail) h->cur_tail = *tail;
    struct ClearPost {
        apt_moe_handle *h;
        ~ClearPost() { h->cur_tail = CombineTail{}; }
    } clear_post{h};
    const bool fq = h->qbits > 0;
    if (h->cfg.moe_sparse && h->fused_decode && !pre_w && !tail &&
        (fq ? h->gu_q && h->gu_sb && h->dn_sb && (h->qbits != 4 || h->gu_qd)
            : h->gu != nullptr) &&
        T <= h->gemv_max_tokens &&
        decode_fused_supported(T, H, h->cfg.moe_intermediate_size, E, K, x_router == x_experts,
                               h->qbits, h->qgs)) {
        // decode: the whole block (router .. combine) in one persistent kernel
        STAGE(h, APT_STAGE_GATE_UP, s,
              launch_decode_fused(x_router, x_experts, h->proj, h->scale, h->pes, T, H, E, K,
                                  h->cfg.moe_intermediate_size, h->cfg.rms_norm_eps, h->scores,
                                  idx, w, h->disp(), weights_for(h, fq), out, h->fsync,
                                  h->errflag, s, &h->launches));
        return APT_OK;
    }
    if (h->cfg.moe_sparse && router_dispatch_fusable(T, H, E, K)) {
        // decode: router + top-k + dispatch in one launch
        const bool quant = h->qbits > 0;
        if (!quant && !h->gu) return fail(h, APT_ERR_STATE, "expert weights not loaded");
        if (quant && !h->gu_q) return fail(h, APT_ERR_STATE, "quantised expert weights not loaded");
        STAGE(h, APT_STAGE_ROUTER_SCORES, s,
              launch_router_dispatch(x_router, h->proj, h->scale, h->pes, T, H, E, K,
                                     h->cfg.rms_norm_eps, h->scores, idx, w, h->disp(), h->done,
                                     s, &h->launches, pre_w, pre_w ? h->xn : nullptr,
                                     h->errflag));
        return run_experts(h, x_experts, idx, w, T, K, quant, out, s, true);
    }
    if (apt_status st = router_scores(h, x_router, T, s, pre_w)) return st;
    if (h->cfg.moe_sparse) {
        CUDA_TRY(h, cudaMemsetAsync(h->counts, 0, sizeof(int32_t) * E, s));
        // slots claimed at selection; one parallel placement replaces the
        // per-expert scan of the dispatch kernel
        STAGE(h, APT_STAGE_ROUTER_SELECT, s,
              launch_router_select(h->scores, h->pes, T, E, K, idx, w, h->counts, s,
                                   &h->launches, h->idx2, nullptr, h->rs_x, H,
                                   h->cfg.rms_norm_eps));
        STAGE(h, APT_STAGE_DISPATCH, s,
              launch_place(idx, h->idx2, T * K, E, h->disp(), s, &h->launches));
        const bool quant = h->qbits > 0;
        if (!quant && !h->gu) return fail(h, APT_ERR_STATE, "expert weights not loaded");
        if (quant && !h->gu_q) return fail(h, APT_ERR_STATE, "quantised expert weights not loaded");
        return run_experts(h, x_experts, idx, w, T, K, quant, out, s, true);
    }
    // dense (reference default): routeWeights then ESExperts::forward
    STAGE(h, APT_STAGE_ROUTER_SELECT, s, launch_router_select(h->scores, h->pes, T, E, K, idx, w, nullptr, s,
                                     &h->launches, nullptr, nullptr, h->rs_x, H,
                                     h->cfg.rms_norm_eps));
    STAGE(h, APT_STAGE_ROUTER_SELECT, s, launch_scatter_dense(idx, w, T, E, K, h->Wd, s, &h->launches));
    return experts_dense(h, x_experts, h->Wd, T, out, s);
}

}  // namespace

extern "C" apt_status apt_moe_forward(apt_moe_handle *h, const uint16_t *x_router,
                                      const uint16_t *x_experts, int T, uint16_t *out,
                                      int32_t *idx_out, uint16_t *w_out, void *stream) {
    return forward_impl(h, x_router, x_experts, T, out, idx_out, w_out, stream, nullptr, nullptr);
}

extern "C" apt_status apt_moe_layer_forward(apt_moe_handle *h, const uint16_t *x1,
                                            const uint16_t *pre_ff_ln_2_w,
                                            const uint16_t *post_ff_ln_2_w, int T, uint16_t *out,
                                            void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (!pre_ff_ln_2_w || !post_ff_ln_2_w) return fail(h, APT_ERR_INVALID, "null norm weight");
    if (h->cfg.hidden_size % 8) return fail(h, APT_ERR_UNSUPPORTED, "hidden_size % 8");
    CHECK_ALIGNED(h, pre_ff_ln_2_w, post_ff_ln_2_w);
    CombineTail tail{};
    tail.post_w = post_ff_ln_2_w;
    tail.eps = h->cfg.rms_norm_eps;
    return forward_impl(h, x1, nullptr, T, out, nullptr, nullptr, stream, pre_ff_ln_2_w, &tail);
}

extern "C" apt_status apt_moe_decoder_ff(apt_moe_handle *h, const uint16_t *x1,
                                         const uint16_t *hmlp, const uint16_t *pre_ff_ln_2_w,
                                         const uint16_t *post_ff_ln_1_w,
                                         const uint16_t *post_ff_ln_2_w,
                                         const uint16_t *post_ff_ln_w, int T, uint16_t *x2,
                                         void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (!x1 || !hmlp || !x2) return fail(h, APT_ERR_INVALID, "null pointer");
    if (!pre_ff_ln_2_w || !post_ff_ln_1_w || !post_ff_ln_2_w || !post_ff_ln_w)
        return fail(h, APT_ERR_INVALID, "null norm weight");
    CHECK_ALIGNED(h, x1, hmlp, x2, pre_ff_ln_2_w, post_ff_ln_1_w, post_ff_ln_2_w, post_ff_ln_w);
    if (h->cfg.hidden_size % 8) return fail(h, APT_ERR_UNSUPPORTED, "hidden_size % 8");
    if (x2 == x1 || x2 == hmlp)
        return fail(h, APT_ERR_INVALID, "x2 must not alias x1 or hmlp");
    CombineTail tail{};
    tail.post_w = post_ff_ln_2_w;
    tail.mlp = hmlp;
    tail.mlp_w = post_ff_ln_1_w;
    tail.ff_w = post_ff_ln_w;
    tail.resid = x1;
    tail.eps = h->cfg.rms_norm_eps;
    return forward_impl(h, x1, nullptr, T, x2, nullptr, nullptr, stream, pre_ff_ln_2_w, &tail);
}

namespace apt {
Dispatch handle_dispatch(apt_moe_handle *h) { return h->disp(); }
}  // namespace apt

// ---- expert-parallel halves: the routing + dispatch before the all-to-all,
// and the combine after it (the remote expert compute is apt_moe_experts on a
// handle holding the rank's local experts).

extern "C" apt_status apt_moe_ep_dispatch(apt_moe_handle *h, const uint16_t *x, int T,
                                          int32_t *idx, uint16_t *w, uint16_t *rows_out,
                                          int32_t *counts_out, void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x || !idx || !w || !rows_out || !counts_out)
        return fail(h, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(h, x, rows_out);
    if (!h->proj) return fail(h, APT_ERR_STATE, "router weights not loaded");
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    begin_call(h);
    const int H = h->cfg.hidden_size, E = h->cfg.num_experts, K = h->cfg.top_k_experts;
    Dispatch d = h->disp();
    if (router_dispatch_fusable(T, H, E, K)) {
        STAGE(h, APT_STAGE_ROUTER_SCORES, s,
              launch_router_dispatch(x, h->proj, h->scale, h->pes, T, H, E, K,
                                     h->cfg.rms_norm_eps, h->scores, idx, w, d, h->done, s,
                                     &h->launches, nullptr, nullptr, h->errflag));
    } else {
        if (apt_status st = router_scores(h, x, T, s)) return st;
        CUDA_TRY(h, cudaMemsetAsync(h->counts, 0, sizeof(int32_t) * E, s));
        STAGE(h, APT_STAGE_ROUTER_SELECT, s,
              launch_router_select(h->scores, h->pes, T, E, K, idx, w, h->counts, s,
                                   &h->launches, h->idx2, nullptr, h->rs_x, H,
                                   h->cfg.rms_norm_eps));
        STAGE(h, APT_STAGE_DISPATCH, s, launch_place(idx, h->idx2, T * K, E, d, s, &h->launches));
    }
    STAGE(h, APT_STAGE_GATHER, s,
          launch_gather_rows(x, H, K, E, d, T * K, rows_out, s, &h->launches, idx, T,
                             h->errflag));
    CUDA_TRY(h, cudaMemcpyAsync(counts_out, h->counts, sizeof(int32_t) * E,
                                cudaMemcpyDeviceToDevice, s));
    return APT_OK;
}

extern "C" apt_status apt_moe_ep_combine(apt_moe_handle *h, const uint16_t *rows,
                                         const int32_t *idx, const uint16_t *w, int T,
                                         uint16_t *out, void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!rows || !idx || !w || !out) return fail(h, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(h, rows, out);
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    STAGE(h, APT_STAGE_COMBINE, s,
          launch_combine(rows, idx, w, h->disp(), T, h->cfg.top_k_experts, h->cfg.hidden_size,
                         out, s, &h->launches, nullptr, h->errflag));
    return APT_OK;
}

extern "C" apt_status apt_moe_experts_grouped(apt_moe_handle *h, const uint16_t *rows, int R,
                                              const int32_t *group_counts,
                                              const int32_t *group_expert, int G, uint16_t *out,
                                              void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (R < 0 || R > h->Pcap)
        return fail(h, APT_ERR_INVALID, "R=%d outside [0, max_tokens*top_k=%d]", R, h->Pcap);
    if (R == 0) return APT_OK;
    if (!rows || !group_counts || !group_expert || !out || G <= 0 || G > 256)
        return fail(h, APT_ERR_INVALID, "bad grouped-experts arguments");
    CHECK_ALIGNED(h, rows, out);
    if (!h->gu) return fail(h, APT_ERR_STATE, "bf16 expert weights not loaded");
    const int H = h->cfg.hidden_size, I = h->cfg.moe_intermediate_size, E = h->cfg.num_experts;
    if (!gemm_supported(H, I)) return fail(h, APT_ERR_UNSUPPORTED, "shape not covered by the GEMM");
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    begin_call(h);
    Dispatch d{};
    d.counts = const_cast<int32_t *>(group_counts);
    // group offsets go to the offsets workspace, or to the (larger) perm
    // workspace when there are more groups than this handle has experts
    d.offsets = (G > E) ? h->perm : h->offsets;
    ExpertWeights ew = weights_for(h, false);
    CUDA_TRY(h, launch_group_offsets(group_counts, G, d.offsets, s, &h->launches));
    STAGE(h, APT_STAGE_GATE_UP, s,
          launch_gemm_gateup_grouped(rows, d, group_expert, ew, R, H, I, E, G, h->yp,
                                     h->errflag, s, &h->launches));
    STAGE(h, APT_STAGE_DOWN, s,
          launch_gemm_down_grouped(h->yp, d, group_expert, ew, R, H, I, E, G, out, h->errflag,
                                   s, &h->launches));
    return APT_OK;
}

extern "C" apt_status apt_moe_mlp_forward(apt_moe_handle *h, const uint16_t *x, int T,
                                          uint16_t *out, void *stream) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x || !out) return fail(h, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(h, x, out);
    if (h->cfg.num_experts != 1 || h->cfg.top_k_experts != 1)
        return fail(h, APT_ERR_STATE, "an MLP handle has num_experts = top_k_experts = 1");
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    begin_call(h);
    // down(gelu(gate(x)) * up(x)) = the expert pipeline with one expert and
    // weight 1 (the combine's bf16(1 * y) is exact)
    CUDA_TRY(h, launch_fill_mlp_routing(h->idx_i, h->w_i, T, s, &h->launches));
    return experts_sparse(h, x, h->idx_i, h->w_i, T, out, s, false);
}

extern "C" apt_status apt_moe_decoder_ff_full(apt_moe_handle *moe, apt_moe_handle *mlp,
                                              const uint16_t *x1, const uint16_t *pre_ff_ln_w,
                                              const uint16_t *pre_ff_ln_2_w,
                                              const uint16_t *post_ff_ln_1_w,
                                              const uint16_t *post_ff_ln_2_w,
                                              const uint16_t *post_ff_ln_w, int T, uint16_t *x2,
                                              void *stream) {
    if (!moe || !mlp) return APT_ERR_INVALID;
    if (check_T(mlp, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x1 || !x2 || !pre_ff_ln_w) return fail(moe, APT_ERR_INVALID, "null pointer");
    CHECK_ALIGNED(moe, x1, x2, pre_ff_ln_w);
    if (mlp->cfg.device != moe->cfg.device || mlp->cfg.hidden_size != moe->cfg.hidden_size)
        return fail(moe, APT_ERR_INVALID, "MLP and MoE handles differ in device or hidden size");
    {
        DeviceGuard g(mlp->cfg.device);
        cudaStream_t s = (cudaStream_t)stream;
        begin_call(mlp);
        // hmlp = mlp(pre_ff_ln(x1)) in the MLP handle's workspace
        CUDA_TRY(mlp, launch_rmsnorm(x1, pre_ff_ln_w, T, mlp->cfg.hidden_size,
                                     mlp->cfg.rms_norm_eps, mlp->xn, s, &mlp->launches));
        CUDA_TRY(mlp, launch_fill_mlp_routing(mlp->idx_i, mlp->w_i, T, s, &mlp->launches));
        if (apt_status st = experts_sparse(mlp, mlp->xn, mlp->idx_i, mlp->w_i, T, mlp->xout, s,
                                           false))
            return st;
    }
    return apt_moe_decoder_ff(moe, x1, mlp->xout, pre_ff_ln_2_w, post_ff_ln_1_w, post_ff_ln_2_w,
                              post_ff_ln_w, T, x2, stream);
}

namespace {

// Device address of a pinned host buffer, or null for pageable memory: under
// unified addressing page-locked host memory is mapped into the device's
// address space, so kernels may read and write it directly.
void *mapped_host_ptr(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

apt_status forward_host_impl(apt_moe_handle *h, const uint16_t *x_host, int T,
                             uint16_t *out_host, void *stream, bool sync) {
    if (!h) return APT_ERR_INVALID;
    if (check_T(h, T)) return APT_ERR_INVALID;
    if (T == 0) return APT_OK;
    if (!x_host || !out_host) return fail(h, APT_ERR_INVALID, "null pointer");
    DeviceGuard g(h->cfg.device);
    cudaStream_t s = (cudaStream_t)stream;
    const size_t bytes = sizeof(uint16_t) * (size_t)T * h->cfg.hidden_size;
    static const bool no_graph = [] {
        const char *v = getenv("APT_NO_GRAPH");
        return v && atoi(v) != 0;
    }();
    // Pinned buffers (sparse path, 16-byte aligned): x is staged in by a kernel
    // that reads the host buffer and the combine writes the result straight
    // into out_host, so no copy-engine transfer sits between the step's
    // kernels.  Pageable buffers go through cudaMemcpyAsync.
    const uint16_t *x_map = nullptr;
    uint16_t *out_map = nullptr;
    if (h->cfg.moe_sparse && h->cfg.hidden_size % 8 == 0) {
        x_map = static_cast<const uint16_t *>(mapped_host_ptr(x_host));
        out_map = static_cast<uint16_t *>(mapped_host_ptr(out_host));
        if (!x_map || !out_map ||
            ((reinterpret_cast<uintptr_t>(x_map) | reinterpret_cast<uintptr_t>(out_map)) & 15))
            x_map = nullptr, out_map = nullptr;
    }
    // the whole step on stream `cs`: copy in, block, copy out
    auto enqueue = [&](cudaStream_t cs, int *launches) -> apt_status {
        if (x_map) {
            CUDA_TRY(h, launch_copy16(x_map, h->xin, bytes, cs, nullptr));
            apt_status st = apt_moe_forward(h, h->xin, h->xin, T, out_map, nullptr, nullptr, cs);
            h->launches += 1;  // the staging kernel (the call's counter starts in the forward)
            if (launches) *launches = h->launches;
            return st;
        }
        CUDA_TRY(h, cudaMemcpyAsync(h->xin, x_host, bytes, cudaMemcpyHostToDevice, cs));
        apt_status st = apt_moe_forward(h, h->xin, h->xin, T, h->xout, nullptr, nullptr, cs);
        if (launches) *launches = h->launches;
        if (st) return st;
        CUDA_TRY(h, cudaMemcpyAsync(out_host, h->xout, bytes, cudaMemcpyDeviceToHost, cs));
        return APT_OK;
    };
    auto direct = [&]() -> apt_status {
        if (apt_status st = enqueue(s, nullptr)) return st;
        if (sync) CUDA_TRY(h, cudaStreamSynchronize(s));
        return APT_OK;
    };
    if (no_graph || h->timing) return direct();
    apt_moe_handle::HostGraph *hg = nullptr;
    for (auto &e : h->graphs)
        if (e.T == T && e.x == x_host && e.out == out_host) hg = &e;
    if (!hg) {
        if (!h->gstream) {
            CUDA_TRY(h, cudaStreamCreateWithFlags(&h->gstream, cudaStreamNonBlocking));
        }
        // capture; anything the capture refuses (pageable host memory, ...)
        // leaves the graph unset and the call runs the same kernels directly
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        apt_status st = APT_OK;
        int launches = 0;
        if (cudaStreamBeginCapture(h->gstream, cudaStreamCaptureModeRelaxed) == cudaSuccess) {
            st = enqueue(h->gstream, &launches);
            const cudaError_t e2 = cudaStreamEndCapture(h->gstream, &graph);
            if (st == APT_OK && e2 == cudaSuccess && graph &&
                cudaGraphInstantiateWithFlags(&exec, graph, 0) != cudaSuccess)
                exec = nullptr;
            if (graph) cudaGraphDestroy(graph);
        }
        (void)cudaGetLastError();  // clear the (non-sticky) error a refused capture leaves
        if (st != APT_OK) return st;
        if (!exec) return direct();
        if (h->graphs.size() >= 8) {
            cudaGraphExecDestroy(h->graphs.front().exec);
            h->graphs.erase(h->graphs.begin());
        }
        h->graphs.push_back({T, x_host, out_host, exec, launches});
        hg = &h->graphs.back();
    }
    begin_call(h);
    // captured on the private stream, replayed on the caller's (any stream,
    // the legacy default one included, may launch a graph)
    CUDA_TRY(h, cudaGraphLaunch(hg->exec, s));
    h->launches = hg->launches;
    if (sync) CUDA_TRY(h, cudaStreamSynchronize(s));
    return APT_OK;
}

}  // namespace

extern "C" apt_status apt_moe_forward_host(apt_moe_handle *h, const uint16_t *x_host, int T,
                                           uint16_t *out_host, void *stream) {
    return forward_host_impl(h, x_host, T, out_host, stream, true);
}

extern "C" apt_status apt_moe_forward_host_async(apt_moe_handle *h, const uint16_t *x_host, int T,
                                                 uint16_t *out_host, void *stream) {
    return forward_host_impl(h, x_host, T, out_host, stream, false);
}
