// ep.cu -- the expert-parallel MoE block in C++ over NCCL: one handle per GPU,
// the hottest experts replicated on every GPU, the others sharded.
//
// The reference runs on one device; this mode is new.  It is the C-ABI form of
// the host flow in apertura_b200/ep.py (same placement, same steps), for hosts
// that drive the library from C or C++:
//   1. route + top-K + dispatch + row gather        (router handle, all experts)
//   2. NCCL exchange of per-expert counts
//   3. replicated experts on a side stream, straight into the return buffer;
//      one host sync for the splits
//   4. NCCL exchange of the cold rows to their owners
//   5. owned experts on the received rows, grouped by (source rank, expert)
//   6. NCCL exchange of the result rows back
//   7. weighted k-order combine on the home rank (ESExperts.mm:58-59)
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy the
// process has already loaded) so the library links no NCCL of its own.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/apt_moe.h"
#include "moe_internal.h"

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

const NcclApi &nccl() {
    static NcclApi api = [] {
        NcclApi a;
        void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return a;
#define APT_NCCL_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(lib, name))
        APT_NCCL_SYM(get_unique_id, "ncclGetUniqueId");
        APT_NCCL_SYM(comm_init_rank, "ncclCommInitRank");
        APT_NCCL_SYM(comm_destroy, "ncclCommDestroy");
        APT_NCCL_SYM(group_start, "ncclGroupStart");
        APT_NCCL_SYM(group_end, "ncclGroupEnd");
        APT_NCCL_SYM(send, "ncclSend");
        APT_NCCL_SYM(recv, "ncclRecv");
        APT_NCCL_SYM(all_gather, "ncclAllGather");
        APT_NCCL_SYM(error_string, "ncclGetErrorString");
#undef APT_NCCL_SYM
        a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.group_start &&
               a.group_end && a.send && a.recv && a.all_gather && a.error_string;
        return a;
    }();
    return api;
}

}  // namespace

struct apt_moe_ep {
    apt_moe_config cfg{};
    int rank = 0, nranks = 1, n_hot = 0, n_cold = 0, c_loc = 0;
    std::vector<int32_t> perm;  // perm[new id] = original expert id
    ncclComm_t comm = nullptr;
    apt_moe_handle *router = nullptr, *hot = nullptr, *cold = nullptr;
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    int Tm = 0, max_recv = 0;
    // device buffers
    int32_t *idx = nullptr, *counts = nullptr, *recv_counts = nullptr, *hot_ge = nullptr,
            *cold_ge = nullptr;
    uint16_t *w = nullptr, *rows = nullptr, *back = nullptr, *recv_rows = nullptr,
             *out_rows = nullptr;
    // pinned host copies of the counts
    int32_t *h_counts = nullptr, *h_recv = nullptr;
    int last_recv = 0, last_hot = 0;
    // NVLink peer-memory transport (ep_p2p.cu): this rank's shared region,
    // the IPC mappings of the others', and the per-step epoch
    int transport = 0;  // APT_EP_NCCL or APT_EP_P2P
    bool p2p_ready = false;
    uint8_t *region = nullptr;
    size_t region_bytes = 0;
    std::vector<void *> mapped;  // peer regions opened through CUDA IPC
    apt::EpPeer *d_peers = nullptr;
    const uint16_t **rowptr = nullptr;
    int32_t *grp = nullptr, *grp_ge = nullptr;
    uint32_t epoch = 0;
    int sms = 148;
    std::string err;
};

namespace {

apt_status ep_fail(apt_moe_ep *ep, apt_status st, const char *fmt, ...) {
    if (ep) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ep->err = buf;
    }
    return st;
}

#define EP_CUDA(ep, call)                                                                   \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return ep_fail(ep, APT_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_));       \
    } while (0)

#define EP_NCCL(ep, call)                                                                   \
    do {                                                                                    \
        ncclResult_t r_ = (call);                                                           \
        if (r_ != ncclSuccess)                                                              \
            return ep_fail(ep, APT_ERR_NCCL, "%s: %s", #call, nccl().error_string(r_));      \
    } while (0)

#define EP_APT(ep, h, call)                                                                 \
    do {                                                                                    \
        apt_status s_ = (call);                                                             \
        if (s_ != APT_OK) return ep_fail(ep, s_, "%s: %s", #call, apt_moe_last_error(h));  \
    } while (0)

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

template <typename T>
cudaError_t dalloc(T **p, size_t n) {
    return cudaMalloc(reinterpret_cast<void **>(p), n * sizeof(T) + 16);
}

// Longest-processing-time placement, n_ranks equal shares; the same rule
// (and tie-breaking) as lpt_placement in apertura_b200/ep.py.
std::vector<int> lpt(const std::vector<double> &loads, int n_ranks) {
    const int E = (int)loads.size(), cap = E / n_ranks;
    std::vector<int> order(E);
    for (int e = 0; e < E; ++e) order[e] = e;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
        return loads[a] > loads[b] || (loads[a] == loads[b] && a < b);
    });
    std::vector<double> rload(n_ranks, 0.0);
    std::vector<std::vector<int>> members(n_ranks);
    for (int e : order) {
        int best = -1;
        for (int r = 0; r < n_ranks; ++r)
            if ((int)members[r].size() < cap && (best < 0 || rload[r] < rload[best])) best = r;
        members[best].push_back(e);
        rload[best] += loads[e];
    }
    std::vector<int> perm;
    for (int r = 0; r < n_ranks; ++r) {
        std::sort(members[r].begin(), members[r].end());
        perm.insert(perm.end(), members[r].begin(), members[r].end());
    }
    return perm;
}

}  // namespace

extern "C" apt_status apt_moe_ep_placement(const float *loads, int E, int nranks, int n_hot,
                                           int32_t *perm_out) {
    if (E <= 0 || nranks <= 0 || !perm_out || n_hot < 0 || n_hot >= E || (E - n_hot) % nranks)
        return APT_ERR_INVALID;
    std::vector<double> l(E, 1.0);
    if (loads)
        for (int e = 0; e < E; ++e) l[e] = loads[e];
    std::vector<int> order(E);
    for (int e = 0; e < E; ++e) order[e] = e;
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return l[a] > l[b] || (l[a] == l[b] && a < b); });
    std::vector<int> hot(order.begin(), order.begin() + n_hot), cold(order.begin() + n_hot, order.end());
    std::sort(hot.begin(), hot.end());
    std::sort(cold.begin(), cold.end());
    std::vector<double> cl;
    for (int e : cold) cl.push_back(l[e]);
    const std::vector<int> sub = lpt(cl, nranks);
    int k = 0;
    for (int e : hot) perm_out[k++] = e;
    for (int i : sub) perm_out[k++] = cold[i];
    return APT_OK;
}

extern "C" apt_status apt_moe_nccl_unique_id(void *id_out) {
    if (!id_out) return APT_ERR_INVALID;
    if (!nccl().ok) return APT_ERR_UNSUPPORTED;
    ncclUniqueId id;
    if (nccl().get_unique_id(&id) != ncclSuccess) return APT_ERR_NCCL;
    memcpy(id_out, &id, sizeof id);
    return APT_OK;
}

namespace {
apt_status ep_barrier(apt_moe_ep *ep);
}

extern "C" apt_status apt_moe_ep_destroy(apt_moe_ep *ep) {
    if (!ep) return APT_OK;
    DevGuard g(ep->cfg.device);
    if (ep->side) cudaStreamSynchronize(ep->side);
    if (ep->p2p_ready) {
        // peers may still read this rank's region until they are done too
        cudaDeviceSynchronize();
        ep_barrier(ep);
        for (void *m : ep->mapped)
            if (m) cudaIpcCloseMemHandle(m);
    }
    if (ep->region) cudaFree(ep->region);
    if (ep->d_peers) cudaFree(ep->d_peers);
    if (ep->rowptr) cudaFree(ep->rowptr);
    if (ep->grp) cudaFree(ep->grp);
    if (ep->grp_ge) cudaFree(ep->grp_ge);
    apt_moe_destroy(ep->router);
    apt_moe_destroy(ep->hot);
    apt_moe_destroy(ep->cold);
    void *ptrs[] = {ep->idx, ep->counts, ep->recv_counts, ep->hot_ge, ep->cold_ge, ep->w,
                    ep->rows, ep->back, ep->recv_rows, ep->out_rows};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    if (ep->h_counts) cudaFreeHost(ep->h_counts);
    if (ep->h_recv) cudaFreeHost(ep->h_recv);
    if (ep->ev_fork) cudaEventDestroy(ep->ev_fork);
    if (ep->ev_join) cudaEventDestroy(ep->ev_join);
    if (ep->side) cudaStreamDestroy(ep->side);
    if (ep->comm && nccl().ok) nccl().comm_destroy(ep->comm);
    delete ep;
    return APT_OK;
}

extern "C" const char *apt_moe_ep_last_error(const apt_moe_ep *ep) {
    return ep ? ep->err.c_str() : "null handle";
}

namespace {

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// All ranks reach this point before any returns (one tiny NCCL all-gather).
apt_status ep_barrier(apt_moe_ep *ep) {
    uint8_t *b = nullptr;
    EP_CUDA(ep, cudaMalloc(&b, 16 * (size_t)ep->nranks));
    ncclResult_t r = nccl().all_gather(b + 16 * ep->rank, b, 16, ncclChar, ep->comm, 0);
    cudaError_t e = cudaStreamSynchronize(0);
    cudaFree(b);
    if (r != ncclSuccess) return ep_fail(ep, APT_ERR_NCCL, "barrier: %s", nccl().error_string(r));
    if (e != cudaSuccess) return ep_fail(ep, APT_ERR_CUDA, "barrier: %s", cudaGetErrorString(e));
    return APT_OK;
}

// The peer-memory transport: one region per rank, mapped by every other rank
// through CUDA IPC (handles exchanged with one NCCL all-gather).  Collective.
// Any failure leaves the NCCL transport in place.
apt_status setup_p2p(apt_moe_ep *ep) {
    const int N = ep->nranks, E = ep->cfg.num_experts, H = ep->cfg.hidden_size;
    const int K = ep->cfg.top_k_experts;
    if (N > apt::kEpMaxRanks || E > apt::kEpMaxExperts || K > apt::kEpMaxK || H % 8)
        return APT_ERR_UNSUPPORTED;
    const size_t flags_b = align256(sizeof(uint32_t) * (3 * N + 2));
    const size_t table_b = align256(sizeof(int32_t) * 2 * N * E);
    const size_t rows_b = align256((size_t)2 * ep->max_recv * H * 2);
    ep->region_bytes = flags_b + table_b + 2 * rows_b;
    EP_CUDA(ep, cudaMalloc(&ep->region, ep->region_bytes));
    EP_CUDA(ep, cudaMemset(ep->region, 0, flags_b + table_b));
    EP_CUDA(ep, dalloc(&ep->rowptr, (size_t)ep->Tm * K));
    EP_CUDA(ep, dalloc(&ep->grp, (size_t)ep->c_loc));
    EP_CUDA(ep, dalloc(&ep->grp_ge, (size_t)ep->c_loc));
    std::vector<int32_t> ge(ep->c_loc);
    for (int j = 0; j < ep->c_loc; ++j) ge[j] = j;
    EP_CUDA(ep, cudaMemcpy(ep->grp_ge, ge.data(), sizeof(int32_t) * ep->c_loc,
                           cudaMemcpyHostToDevice));
    EP_CUDA(ep, cudaDeviceSynchronize());
    // exchange the IPC handles
    cudaIpcMemHandle_t mine;
    cudaError_t ie = cudaIpcGetMemHandle(&mine, ep->region);
    uint8_t *hb = nullptr;
    EP_CUDA(ep, cudaMalloc(&hb, sizeof(cudaIpcMemHandle_t) * N + 16));
    // a rank that could not export its region sends zeros; every rank then
    // sees the failure and stays on NCCL
    std::vector<uint8_t> h(sizeof(cudaIpcMemHandle_t) * N, 0);
    if (ie == cudaSuccess) memcpy(h.data() + sizeof mine * ep->rank, &mine, sizeof mine);
    cudaMemcpy(hb, h.data(), h.size(), cudaMemcpyHostToDevice);
    ncclResult_t r = nccl().all_gather(hb + sizeof mine * ep->rank, hb, sizeof mine, ncclChar,
                                       ep->comm, 0);
    cudaStreamSynchronize(0);
    cudaMemcpy(h.data(), hb, h.size(), cudaMemcpyDeviceToHost);
    cudaFree(hb);
    if (r != ncclSuccess) return ep_fail(ep, APT_ERR_NCCL, "handle exchange failed");
    bool ok = true;
    for (int d = 0; d < N; ++d) {
        bool zero = true;
        for (size_t i = 0; i < sizeof mine; ++i) zero &= h[sizeof mine * d + i] == 0;
        ok &= !zero;
    }
    std::vector<apt::EpPeer> peers(N);
    ep->mapped.assign(N, nullptr);
    for (int d = 0; d < N && ok; ++d) {
        uint8_t *base = ep->region;
        if (d != ep->rank) {
            cudaIpcMemHandle_t hd;
            memcpy(&hd, h.data() + sizeof hd * d, sizeof hd);
            void *p = nullptr;
            if (cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = false;
                break;
            }
            ep->mapped[d] = p;
            base = static_cast<uint8_t *>(p);
        }
        peers[d].flags = reinterpret_cast<uint32_t *>(base);
        peers[d].table = reinterpret_cast<int32_t *>(base + flags_b);
        peers[d].recv = reinterpret_cast<uint16_t *>(base + flags_b + table_b);
        peers[d].out = reinterpret_cast<uint16_t *>(base + flags_b + table_b + rows_b);
    }
    // every rank must have mapped every other rank's region
    int32_t *okb = nullptr;
    EP_CUDA(ep, dalloc(&okb, (size_t)N * 4));
    std::vector<int32_t> oks(N * 4, 0);
    oks[ep->rank * 4] = ok ? 1 : 0;
    cudaMemcpy(okb, oks.data(), sizeof(int32_t) * N * 4, cudaMemcpyHostToDevice);
    r = nccl().all_gather(okb + ep->rank * 4, okb, 4, ncclInt32, ep->comm, 0);
    cudaStreamSynchronize(0);
    cudaMemcpy(oks.data(), okb, sizeof(int32_t) * N * 4, cudaMemcpyDeviceToHost);
    cudaFree(okb);
    for (int d = 0; d < N; ++d) ok &= oks[d * 4] == 1;
    if (r != ncclSuccess || !ok) {
        for (void *m : ep->mapped)
            if (m) cudaIpcCloseMemHandle(m);
        ep->mapped.clear();
        return ep_fail(ep, APT_ERR_UNSUPPORTED, "peer-memory transport unavailable; using NCCL");
    }
    EP_CUDA(ep, dalloc(&ep->d_peers, (size_t)N));
    EP_CUDA(ep, cudaMemcpy(ep->d_peers, peers.data(), sizeof(apt::EpPeer) * N,
                           cudaMemcpyHostToDevice));
    ep->p2p_ready = true;
    return APT_OK;
}

}  // namespace

extern "C" apt_status apt_moe_create_ep(const apt_moe_config *cfg, const void *nccl_id, int rank,
                                        int nranks, const float *expected_loads, int replicate_hot,
                                        apt_moe_ep **out) {
    if (!cfg || !nccl_id || !out || nranks <= 0 || rank < 0 || rank >= nranks)
        return APT_ERR_INVALID;
    *out = nullptr;
    if (!nccl().ok) return APT_ERR_UNSUPPORTED;
    const int E = cfg->num_experts, K = cfg->top_k_experts, H = cfg->hidden_size;
    int R = nranks > 1 ? replicate_hot : 0;
    if (R < 0 || R >= E || (E - R) % nranks) R = 0;
    if (E % nranks && (E - R) % nranks) return APT_ERR_UNSUPPORTED;
    if (cfg->quant_bits) return APT_ERR_UNSUPPORTED;  // bf16 experts only
    apt_moe_ep *ep = new apt_moe_ep();
    ep->cfg = *cfg;
    ep->cfg.moe_sparse = 1;
    ep->rank = rank;
    ep->nranks = nranks;
    ep->n_hot = R;
    ep->n_cold = E - R;
    ep->c_loc = (E - R) / nranks;
    ep->Tm = cfg->max_tokens;
    ep->max_recv = 4 * cfg->max_tokens * K;
    ep->perm.resize(E);
    DevGuard g(cfg->device);
    auto bail = [&](apt_status st) {
        apt_moe_ep_destroy(ep);
        return st;
    };
    if (apt_moe_ep_placement(expected_loads, E, nranks, R, ep->perm.data())) return bail(APT_ERR_INVALID);
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof id);
    if (nccl().comm_init_rank(&ep->comm, nranks, id, rank) != ncclSuccess) return bail(APT_ERR_NCCL);
    // handles: router over all experts, replicated bank, owned bank
    apt_moe_config c = ep->cfg;
    if (apt_moe_create(&c, &ep->router)) return bail(APT_ERR_CUDA);
    apt_moe_config cb = ep->cfg;
    cb.top_k_experts = 1;
    if (R) {
        cb.num_experts = R;
        cb.max_tokens = ep->Tm * K;
        if (apt_moe_create(&cb, &ep->hot)) return bail(APT_ERR_CUDA);
    }
    cb.num_experts = ep->c_loc;
    cb.max_tokens = ep->max_recv;
    if (apt_moe_create(&cb, &ep->cold)) return bail(APT_ERR_CUDA);
    // device buffers
    const size_t P = (size_t)ep->Tm * K;
    cudaError_t e1 = cudaSuccess;
    if (!e1) e1 = dalloc(&ep->idx, P);
    if (!e1) e1 = dalloc(&ep->w, P);
    if (!e1) e1 = dalloc(&ep->counts, (size_t)E);
    if (!e1) e1 = dalloc(&ep->recv_counts, (size_t)nranks * ep->c_loc);
    if (!e1) e1 = dalloc(&ep->hot_ge, (size_t)R + 1);
    if (!e1) e1 = dalloc(&ep->cold_ge, (size_t)nranks * ep->c_loc);
    if (!e1) e1 = dalloc(&ep->rows, P * H);
    if (!e1) e1 = dalloc(&ep->back, P * H);
    if (!e1) e1 = dalloc(&ep->recv_rows, (size_t)ep->max_recv * H);
    if (!e1) e1 = dalloc(&ep->out_rows, (size_t)ep->max_recv * H);
    if (!e1) e1 = cudaMallocHost(reinterpret_cast<void **>(&ep->h_counts), sizeof(int32_t) * E);
    if (!e1)
        e1 = cudaMallocHost(reinterpret_cast<void **>(&ep->h_recv),
                            sizeof(int32_t) * nranks * ep->c_loc);
    if (!e1) e1 = cudaStreamCreateWithFlags(&ep->side, cudaStreamNonBlocking);
    if (!e1) e1 = cudaEventCreateWithFlags(&ep->ev_fork, cudaEventDisableTiming);
    if (!e1) e1 = cudaEventCreateWithFlags(&ep->ev_join, cudaEventDisableTiming);
    if (e1) return bail(APT_ERR_CUDA);
    std::vector<int32_t> ge(std::max(R, nranks * ep->c_loc) + 1);
    for (int i = 0; i < R; ++i) ge[i] = i;
    if (R && cudaMemcpy(ep->hot_ge, ge.data(), sizeof(int32_t) * R, cudaMemcpyHostToDevice))
        return bail(APT_ERR_CUDA);
    for (int i = 0; i < nranks * ep->c_loc; ++i) ge[i] = i % ep->c_loc;
    if (cudaMemcpy(ep->cold_ge, ge.data(), sizeof(int32_t) * nranks * ep->c_loc,
                   cudaMemcpyHostToDevice))
        return bail(APT_ERR_CUDA);
    // the replicated experts leave SMs to NCCL while they run beside the exchange
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device);
    if (ep->hot) apt_moe_set_sm_limit(ep->hot, sms > 32 ? sms - 24 : sms);
    ep->sms = sms;
    ep->transport = APT_EP_NCCL;
    if (setup_p2p(ep) == APT_OK) ep->transport = APT_EP_P2P;
    *out = ep;
    return APT_OK;
}

namespace {

// rows[perm[i]] of src (rows of `row_elems` bf16) -> dst row i, i < n.
apt_status gather_rows(apt_moe_ep *ep, uint16_t *dst, const uint16_t *src, const int32_t *ids,
                       int n, size_t row_elems, int on_device) {
    for (int i = 0; i < n; ++i)
        EP_CUDA(ep, cudaMemcpy(dst + (size_t)i * row_elems, src + (size_t)ids[i] * row_elems,
                               row_elems * 2, on_device ? cudaMemcpyDeviceToDevice
                                                        : cudaMemcpyHostToDevice));
    return APT_OK;
}

}  // namespace

extern "C" apt_status apt_moe_ep_load_router(apt_moe_ep *ep, const uint16_t *proj,
                                             const uint16_t *scale, const uint16_t *pes,
                                             int on_device) {
    if (!ep || !proj || !scale || !pes) return APT_ERR_INVALID;
    DevGuard g(ep->cfg.device);
    const int E = ep->cfg.num_experts, H = ep->cfg.hidden_size;
    // proj rows and per_expert_scale in the relabelled expert order
    uint16_t *p = nullptr, *e = nullptr, *sc = nullptr;
    EP_CUDA(ep, dalloc(&p, (size_t)E * H));
    EP_CUDA(ep, dalloc(&e, (size_t)E));
    EP_CUDA(ep, dalloc(&sc, (size_t)H));
    apt_status st = gather_rows(ep, p, proj, ep->perm.data(), E, H, on_device);
    if (!st) st = gather_rows(ep, e, pes, ep->perm.data(), E, 1, on_device);
    if (!st && cudaMemcpy(sc, scale, (size_t)H * 2,
                          on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice))
        st = ep_fail(ep, APT_ERR_CUDA, "scale copy failed");
    if (!st) {
        st = apt_moe_load_router(ep->router, p, sc, e, 1);
        if (st) ep_fail(ep, st, "router: %s", apt_moe_last_error(ep->router));
    }
    cudaFree(p);
    cudaFree(e);
    cudaFree(sc);
    return st;
}

extern "C" apt_status apt_moe_ep_load_experts_bf16(apt_moe_ep *ep, const uint16_t *gate_up,
                                                   const uint16_t *down, int on_device) {
    if (!ep || !gate_up || !down) return APT_ERR_INVALID;
    DevGuard g(ep->cfg.device);
    const size_t H = ep->cfg.hidden_size, I = ep->cfg.moe_intermediate_size;
    const int R = ep->n_hot, C = ep->c_loc;
    auto load = [&](apt_moe_handle *h, const int32_t *ids, int n) -> apt_status {
        uint16_t *gu = nullptr, *dn = nullptr;
        EP_CUDA(ep, dalloc(&gu, (size_t)n * 2 * I * H));
        EP_CUDA(ep, dalloc(&dn, (size_t)n * H * I));
        apt_status st = gather_rows(ep, gu, gate_up, ids, n, 2 * I * H, on_device);
        if (!st) st = gather_rows(ep, dn, down, ids, n, H * I, on_device);
        if (!st) {
            st = apt_moe_load_experts_bf16(h, gu, dn, 1);
            if (st) ep_fail(ep, st, "experts: %s", apt_moe_last_error(h));
        }
        cudaFree(gu);
        cudaFree(dn);
        return st;
    };
    if (R)
        if (apt_status st = load(ep->hot, ep->perm.data(), R)) return st;
    return load(ep->cold, ep->perm.data() + R + ep->rank * C, C);
}

namespace {

// One step over the peer-memory transport (ep_p2p.cu): no host
// synchronisation; every exchange is a kernel.
apt_status ep_forward_p2p(apt_moe_ep *ep, const uint16_t *x, int T, uint16_t *out, void *stream) {
    cudaStream_t s = (cudaStream_t)stream;
    const int N = ep->nranks, C = ep->c_loc, R = ep->n_hot, K = ep->cfg.top_k_experts;
    const int E = ep->cfg.num_experts, H = ep->cfg.hidden_size;
    EP_APT(ep, ep->router,
           apt_moe_ep_dispatch(ep->router, x, T, ep->idx, ep->w, ep->rows, ep->counts, stream));
    const apt::Dispatch d = apt::handle_dispatch(ep->router);
    ++ep->epoch;
    if (ep->epoch == 0) ep->epoch = 1;  // flags start at 0
    apt::EpP2PArgs a{};
    a.peers = ep->d_peers;
    a.N = N;
    a.me = ep->rank;
    a.R = R;
    a.C = C;
    a.E = E;
    a.H = H;
    a.max_recv = ep->max_recv;
    a.parity = (int)(ep->epoch & 1);
    a.epoch = ep->epoch;
    a.counts = d.counts;
    a.offsets = d.offsets;
    a.perm = d.perm;
    a.rows = ep->rows;
    a.back = ep->back;
    a.rowptr = ep->rowptr;
    a.grp = ep->grp;
    if (R) {  // replicated experts beside the exchange
        EP_CUDA(ep, cudaEventRecord(ep->ev_fork, s));
        EP_CUDA(ep, cudaStreamWaitEvent(ep->side, ep->ev_fork, 0));
        EP_APT(ep, ep->hot,
               apt_moe_experts_grouped(ep->hot, ep->rows, T * K, ep->counts, ep->hot_ge, R,
                                       ep->back, ep->side));
    }
    EP_CUDA(ep, apt::launch_ep_push(a, 2 * ep->sms, s));
    EP_CUDA(ep, apt::launch_ep_wait_recv(a, s));
    const size_t slot = (size_t)a.parity * ep->max_recv * H;
    const size_t flags_b = align256(sizeof(uint32_t) * (3 * N + 2));
    const size_t table_b = align256(sizeof(int32_t) * 2 * N * E);
    const size_t rows_b = align256((size_t)2 * ep->max_recv * H * 2);
    uint16_t *recv = reinterpret_cast<uint16_t *>(ep->region + flags_b + table_b) + slot;
    uint16_t *res = reinterpret_cast<uint16_t *>(ep->region + flags_b + table_b + rows_b) + slot;
    EP_APT(ep, ep->cold,
           apt_moe_experts_grouped(ep->cold, recv, ep->max_recv, ep->grp, ep->grp_ge, C, res,
                                   stream));
    EP_CUDA(ep, apt::launch_ep_done(a, s));
    if (R) {
        EP_CUDA(ep, cudaEventRecord(ep->ev_join, ep->side));
        EP_CUDA(ep, cudaStreamWaitEvent(s, ep->ev_join, 0));
    }
    EP_CUDA(ep, apt::launch_ep_combine(a, ep->w, T, K, out, std::min(T, 4 * ep->sms), s));
    ep->last_recv = -1;  // counted on demand (apt_moe_ep_stats)
    ep->last_hot = -1;
    return APT_OK;
}

}  // namespace

extern "C" apt_status apt_moe_ep_forward(apt_moe_ep *ep, const uint16_t *x, int T, uint16_t *out,
                                         void *stream) {
    if (!ep) return APT_ERR_INVALID;
    if (T < 0 || T > ep->Tm) return ep_fail(ep, APT_ERR_INVALID, "T=%d outside [0, %d]", T, ep->Tm);
    if (T == 0) return APT_OK;
    if (!x || !out) return ep_fail(ep, APT_ERR_INVALID, "null pointer");
    if (((uintptr_t)x | (uintptr_t)out) & 15)
        return ep_fail(ep, APT_ERR_INVALID, "x and out must be 16-byte aligned");
    DevGuard g(ep->cfg.device);
    if (ep->transport == APT_EP_P2P) return ep_forward_p2p(ep, x, T, out, stream);
    cudaStream_t s = (cudaStream_t)stream;
    const NcclApi &nc = nccl();
    const int N = ep->nranks, C = ep->c_loc, R = ep->n_hot, K = ep->cfg.top_k_experts;
    const int E = ep->cfg.num_experts;
    const size_t H = ep->cfg.hidden_size;
    // 1. route, dispatch, gather: rows sorted [hot | cold by destination rank]
    EP_APT(ep, ep->router,
           apt_moe_ep_dispatch(ep->router, x, T, ep->idx, ep->w, ep->rows, ep->counts, stream));
    // 2. counts of the cold experts, exchanged first (a small NCCL op that must
    //    not queue behind the replicated experts for SMs)
    EP_NCCL(ep, nc.group_start());
    for (int r = 0; r < N; ++r) {
        EP_NCCL(ep, nc.send(ep->counts + R + r * C, C, ncclInt32, r, ep->comm, s));
        EP_NCCL(ep, nc.recv(ep->recv_counts + r * C, C, ncclInt32, r, ep->comm, s));
    }
    EP_NCCL(ep, nc.group_end());
    // 3. replicated experts beside the exchange (hot rows open the buffer)
    if (R) {
        EP_CUDA(ep, cudaEventRecord(ep->ev_fork, s));
        EP_CUDA(ep, cudaStreamWaitEvent(ep->side, ep->ev_fork, 0));
        EP_APT(ep, ep->hot,
               apt_moe_experts_grouped(ep->hot, ep->rows, T * K, ep->counts, ep->hot_ge, R,
                                       ep->back, ep->side));
    }
    // one host sync for the splits
    EP_CUDA(ep, cudaMemcpyAsync(ep->h_counts, ep->counts, sizeof(int32_t) * E,
                                cudaMemcpyDeviceToHost, s));
    EP_CUDA(ep, cudaMemcpyAsync(ep->h_recv, ep->recv_counts, sizeof(int32_t) * N * C,
                                cudaMemcpyDeviceToHost, s));
    EP_CUDA(ep, cudaStreamSynchronize(s));
    int hot_rows = 0;
    for (int e = 0; e < R; ++e) hot_rows += ep->h_counts[e];
    std::vector<size_t> soff(N + 1, 0), roff(N + 1, 0);
    for (int r = 0; r < N; ++r) {
        size_t sn = 0, rn = 0;
        for (int j = 0; j < C; ++j) {
            sn += ep->h_counts[R + r * C + j];
            rn += ep->h_recv[r * C + j];
        }
        soff[r + 1] = soff[r] + sn;
        roff[r + 1] = roff[r] + rn;
    }
    const int recv = (int)roff[N];
    if (recv > ep->max_recv)
        return ep_fail(ep, APT_ERR_UNSUPPORTED, "rank %d receives %d rows > capacity %d", ep->rank,
                       recv, ep->max_recv);
    uint16_t *send_base = ep->rows + (size_t)hot_rows * H;
    uint16_t *back_base = ep->back + (size_t)hot_rows * H;
    // 4. cold rows to their owners
    EP_NCCL(ep, nc.group_start());
    for (int r = 0; r < N; ++r) {
        EP_NCCL(ep, nc.send(send_base + soff[r] * H, (soff[r + 1] - soff[r]) * H, ncclBfloat16, r,
                            ep->comm, s));
        EP_NCCL(ep, nc.recv(ep->recv_rows + roff[r] * H, (roff[r + 1] - roff[r]) * H,
                            ncclBfloat16, r, ep->comm, s));
    }
    EP_NCCL(ep, nc.group_end());
    // 5. owned experts on the received rows, in place
    EP_APT(ep, ep->cold,
           apt_moe_experts_grouped(ep->cold, ep->recv_rows, recv, ep->recv_counts, ep->cold_ge,
                                   N * C, ep->out_rows, stream));
    // 6. results back, in the send order
    EP_NCCL(ep, nc.group_start());
    for (int r = 0; r < N; ++r) {
        EP_NCCL(ep, nc.send(ep->out_rows + roff[r] * H, (roff[r + 1] - roff[r]) * H, ncclBfloat16,
                            r, ep->comm, s));
        EP_NCCL(ep, nc.recv(back_base + soff[r] * H, (soff[r + 1] - soff[r]) * H, ncclBfloat16, r,
                            ep->comm, s));
    }
    EP_NCCL(ep, nc.group_end());
    if (R) {
        EP_CUDA(ep, cudaEventRecord(ep->ev_join, ep->side));
        EP_CUDA(ep, cudaStreamWaitEvent(s, ep->ev_join, 0));
    }
    // 7. weighted k-order combine on the home rank
    EP_APT(ep, ep->router, apt_moe_ep_combine(ep->router, ep->back, ep->idx, ep->w, T, out, stream));
    ep->last_recv = recv;
    ep->last_hot = hot_rows;
    return APT_OK;
}

extern "C" apt_status apt_moe_ep_stats(apt_moe_ep *ep, int *recv_rows, int *hot_rows) {
    if (!ep) return APT_ERR_INVALID;
    if (ep->last_recv < 0) {  // peer-memory step: read the group counts back
        DevGuard g(ep->cfg.device);
        std::vector<int32_t> grp(ep->c_loc), cnt(ep->cfg.num_experts);
        EP_CUDA(ep, cudaDeviceSynchronize());
        EP_CUDA(ep, cudaMemcpy(grp.data(), ep->grp, sizeof(int32_t) * ep->c_loc,
                               cudaMemcpyDeviceToHost));
        EP_CUDA(ep, cudaMemcpy(cnt.data(), ep->counts, sizeof(int32_t) * cnt.size(),
                               cudaMemcpyDeviceToHost));
        ep->last_recv = 0;
        for (int v : grp) ep->last_recv += v;
        ep->last_hot = 0;
        for (int e = 0; e < ep->n_hot; ++e) ep->last_hot += cnt[e];
    }
    if (recv_rows) *recv_rows = ep->last_recv;
    if (hot_rows) *hot_rows = ep->last_hot;
    return APT_OK;
}

extern "C" apt_status apt_moe_ep_set_transport(apt_moe_ep *ep, int transport) {
    if (!ep || (transport != APT_EP_NCCL && transport != APT_EP_P2P)) return APT_ERR_INVALID;
    if (transport == APT_EP_P2P && !ep->p2p_ready)
        return ep_fail(ep, APT_ERR_UNSUPPORTED, "peer-memory transport was not set up");
    ep->transport = transport;
    return APT_OK;
}

extern "C" apt_status apt_moe_ep_get_transport(const apt_moe_ep *ep, int *transport) {
    if (!ep || !transport) return APT_ERR_INVALID;
    *transport = ep->transport;
    return APT_OK;
}

extern "C" apt_status apt_moe_ep_sync(apt_moe_ep *ep) {
    if (!ep) return APT_ERR_INVALID;
    DevGuard g(ep->cfg.device);
    EP_CUDA(ep, cudaDeviceSynchronize());
    apt_status st = APT_OK;
    if (ep->p2p_ready) {
        const int N = ep->nranks;
        uint32_t *errw = reinterpret_cast<uint32_t *>(ep->region) + 3 * N + 1;
        uint32_t code = 0;
        EP_CUDA(ep, cudaMemcpy(&code, errw, sizeof code, cudaMemcpyDeviceToHost));
        if (code) {
            EP_CUDA(ep, cudaMemset(errw, 0, sizeof code));
            st = ep_fail(ep, APT_ERR_TIMEOUT, "peer-memory exchange: error code %u", code);
        }
    }
    apt_moe_handle *hs[] = {ep->router, ep->hot, ep->cold};
    for (apt_moe_handle *h : hs) {
        if (!h) continue;
        apt_status hs_st = apt_moe_sync(h);
        if (hs_st && !st) st = ep_fail(ep, hs_st, "%s", apt_moe_last_error(h));
    }
    return st;
}
