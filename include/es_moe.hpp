// es_moe.hpp -- the reference's es::ESRouter / es::ESExperts pair
// (aptransformer/ESRouter.h:19-27, aptransformer/ESExperts.h:20-32) and
// esMakeExperts (ESWeightLoader.mm:145-154) as C++ classes over this
// library's C ABI (apt_moe.h), for C++ hosts.  Header-only; link
// libapt_moe.so and the CUDA runtime.
//
// Where the reference passes mx::array, these classes take es::Array: a
// tensor in host or device memory (dtype, shape, pointer), owning its storage
// or viewing the caller's.  Weights may be given on either side (they are
// copied into the handle); activations are device arrays, and results come
// back as device arrays the Array owns.  Calls are stream-ordered on
// `stream()` (the legacy default stream unless set).  Errors throw
// std::runtime_error with the library's message, as the reference's
// constructors and loader report failures.
//
// Beyond the reference signatures each class takes trailing runtime options
// (largest T per call, top-k for the experts' workspace, device), which
// MLX needs no equivalent of because it allocates per call; this library
// sizes its workspace once.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "apt_moe.h"
#include "es_weight_loader.hpp"

namespace es {

struct Array {
    Dtype dtype = Dtype::bfloat16;
    std::vector<int64_t> shape;
    void *data = nullptr;
    bool on_device = false;
    std::shared_ptr<void> owner;  // keeps owned storage alive (empty for views)

    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
    size_t nbytes() const { return (size_t)numel() * dtype_size(dtype); }
    int64_t dim(int i) const { return shape.at(i < 0 ? shape.size() + i : i); }

    // a view of caller memory
    static Array view(void *p, Dtype dt, std::vector<int64_t> shape, bool on_device) {
        Array a;
        a.data = p;
        a.dtype = dt;
        a.shape = std::move(shape);
        a.on_device = on_device;
        return a;
    }
    // a host array holding a loader tensor (shares its bytes)
    static Array from_host(HostTensor t) {
        auto keep = std::make_shared<HostTensor>(std::move(t));
        Array a = view(keep->bytes.data(), keep->dtype, keep->shape, false);
        a.owner = keep;
        return a;
    }
    // new device storage
    static Array device(Dtype dt, std::vector<int64_t> shape) {
        Array a;
        a.dtype = dt;
        a.shape = std::move(shape);
        a.on_device = true;
        void *p = nullptr;
        if (cudaMalloc(&p, a.nbytes() ? a.nbytes() : 16) != cudaSuccess)
            throw std::runtime_error("es::Array: cudaMalloc failed");
        a.data = p;
        a.owner = std::shared_ptr<void>(p, [](void *q) { cudaFree(q); });
        return a;
    }
    // copies to / from the device
    Array to_device() const {
        if (on_device) return *this;
        Array d = device(dtype, shape);
        if (cudaMemcpy(d.data, data, nbytes(), cudaMemcpyHostToDevice) != cudaSuccess)
            throw std::runtime_error("es::Array: copy to device failed");
        return d;
    }
    std::vector<uint8_t> to_host_bytes() const {
        std::vector<uint8_t> out(nbytes());
        if (cudaMemcpy(out.data(), data, out.size(),
                       on_device ? cudaMemcpyDeviceToHost : cudaMemcpyHostToHost) != cudaSuccess)
            throw std::runtime_error("es::Array: copy to host failed");
        return out;
    }
};

namespace detail {
inline void check(apt_status st, apt_moe_handle *h, const char *what) {
    if (st != APT_OK)
        throw std::runtime_error(std::string(what) + ": " +
                                 (h ? apt_moe_last_error(h) : ("status " + std::to_string(st))));
}
inline void need(const Array &a, Dtype dt, size_t rank, const char *what) {
    if (a.dtype != dt || a.shape.size() != rank)
        throw std::runtime_error(std::string(what) + ": unexpected dtype or rank");
}
struct HandleDeleter {
    void operator()(apt_moe_handle *h) const { apt_moe_destroy(h); }
};
using HandlePtr = std::shared_ptr<apt_moe_handle>;
inline HandlePtr make_handle(const apt_moe_config &cfg) {
    apt_moe_handle *h = nullptr;
    check(apt_moe_create(&cfg, &h), nullptr, "apt_moe_create");
    return HandlePtr(h, HandleDeleter());
}
}  // namespace detail

// Gemma4TextRouter: weightless RMSNorm, x scale x H^-1/2, proj, softmax,
// top-k, renormalise, x per_expert_scale (ESRouter.mm:14-40).
class ESRouter {
public:
    struct TopK {
        Array idx;  // [T, K] int32, device
        Array w;    // [T, K] bf16, device
    };

    ESRouter(Array projWeight, Array scale, Array perExpertScale, int numExperts, int topK,
             int hiddenSize, float eps, Dtype computeDtype, int maxTokens = 8192, int device = 0)
        : E_(numExperts), K_(topK), H_(hiddenSize) {
        if (computeDtype != Dtype::bfloat16)
            throw std::runtime_error("ESRouter: the CUDA path computes in bf16");
        detail::need(projWeight, Dtype::bfloat16, 2, "ESRouter proj");
        if (scale.dtype != Dtype::bfloat16 || perExpertScale.dtype != Dtype::bfloat16)
            throw std::runtime_error("ESRouter: scale and per_expert_scale must be bf16");
        if (projWeight.dim(0) != E_ || projWeight.dim(1) != H_ || scale.numel() != H_ ||
            perExpertScale.numel() != E_)
            throw std::runtime_error("ESRouter: weight shapes do not match E, H");
        apt_moe_config c{};
        c.hidden_size = H_;
        c.num_experts = E_;
        c.top_k_experts = K_;
        c.moe_intermediate_size = 64;  // no expert weights in this handle
        c.rms_norm_eps = eps;
        c.enable_moe_block = 1;
        c.moe_sparse = 1;
        c.quant_group_size = 64;
        c.max_tokens = maxTokens;
        c.device = device;
        h_ = detail::make_handle(c);
        // the loader accepts host or device pointers, but not a mix
        const bool dev = projWeight.on_device;
        const Array s = dev ? scale.to_device() : scale, p = dev ? perExpertScale.to_device()
                                                                 : perExpertScale;
        if (!dev && (scale.on_device || perExpertScale.on_device))
            throw std::runtime_error("ESRouter: router weights must all be host or all device");
        detail::check(apt_moe_load_router(h_.get(), static_cast<const uint16_t *>(projWeight.data),
                                          static_cast<const uint16_t *>(s.data),
                                          static_cast<const uint16_t *>(p.data), dev ? 1 : 0),
                      h_.get(), "ESRouter");
    }

    TopK routeTopK(const Array &x) const {
        const int T = check_x(x);
        TopK r{Array::device(Dtype::int32, {T, K_}), Array::device(Dtype::bfloat16, {T, K_})};
        detail::check(apt_moe_route(h_.get(), static_cast<const uint16_t *>(x.data), T,
                                    static_cast<int32_t *>(r.idx.data),
                                    static_cast<uint16_t *>(r.w.data), stream_),
                      h_.get(), "ESRouter::routeTopK");
        return r;
    }

    // dense [T, E] bf16: the top-k weights, 0 elsewhere
    Array routeWeights(const Array &x) const {
        const int T = check_x(x);
        Array W = Array::device(Dtype::bfloat16, {T, E_});
        detail::check(apt_moe_route_weights(h_.get(), static_cast<const uint16_t *>(x.data), T,
                                            static_cast<uint16_t *>(W.data), stream_),
                      h_.get(), "ESRouter::routeWeights");
        return W;
    }

    void setStream(void *s) { stream_ = s; }
    void *stream() const { return stream_; }
    apt_moe_handle *raw() const { return h_.get(); }

private:
    int check_x(const Array &x) const {
        detail::need(x, Dtype::bfloat16, 2, "ESRouter input");
        if (!x.on_device || x.dim(1) != H_) throw std::runtime_error("ESRouter: x must be [T, H] on the device");
        return (int)x.dim(0);
    }
    int E_, K_, H_;
    detail::HandlePtr h_;
    void *stream_ = nullptr;
};

// Gemma4TextExperts: E GeGLU MLPs, gate_up [E, 2I, H], down [E, H, I]
// (ESExperts.mm:8-60).
class ESExperts {
public:
    // bf16 banks; quantBits > 0 quantises them at load (MLX affine, groupSize)
    ESExperts(Array gateUp, Array down, int quantBits = 0, int groupSize = 64, int topK = 8,
              int maxTokens = 8192, int device = 0) {
        detail::need(gateUp, Dtype::bfloat16, 3, "ESExperts gate_up");
        detail::need(down, Dtype::bfloat16, 3, "ESExperts down");
        E_ = (int)gateUp.dim(0);
        I_ = (int)gateUp.dim(1) / 2;
        H_ = (int)gateUp.dim(2);
        if (down.dim(0) != E_ || down.dim(1) != H_ || down.dim(2) != I_)
            throw std::runtime_error("ESExperts: down is not [E, H, I]");
        if (gateUp.on_device != down.on_device)
            throw std::runtime_error("ESExperts: weights must both be host or both device");
        create(quantBits, groupSize, topK, maxTokens, device);
        detail::check(apt_moe_load_experts_bf16(h_.get(), static_cast<const uint16_t *>(gateUp.data),
                                                static_cast<const uint16_t *>(down.data),
                                                gateUp.on_device ? 1 : 0),
                      h_.get(), "ESExperts");
    }

    // already quantised (a bundle): packed codes and bf16 scales / biases
    // adopted verbatim; the dense forward() is unavailable then
    ESExperts(Array gateUpQ, Array gateUpS, Array gateUpB, Array downQ, Array downS, Array downB,
              int bits, int groupSize, int topK = 8, int maxTokens = 8192, int device = 0) {
        // packed codes: u32 (MLX) or the same bits stored as i32
        if (gateUpQ.dtype == Dtype::int32) gateUpQ.dtype = Dtype::uint32;
        if (downQ.dtype == Dtype::int32) downQ.dtype = Dtype::uint32;
        detail::need(gateUpQ, Dtype::uint32, 3, "ESExperts gate_up codes");
        detail::need(downQ, Dtype::uint32, 3, "ESExperts down codes");
        E_ = (int)gateUpQ.dim(0);
        I_ = (int)gateUpQ.dim(1) / 2;
        H_ = (int)(gateUpQ.dim(2) * 32 / bits);
        const bool dev = gateUpQ.on_device;
        for (const Array *a : {&gateUpS, &gateUpB, &downQ, &downS, &downB})
            if (a->on_device != dev)
                throw std::runtime_error("ESExperts: quantised tensors must all be host or all device");
        for (const Array *a : {&gateUpS, &gateUpB, &downS, &downB})
            if (a->dtype != Dtype::bfloat16)
                throw std::runtime_error("ESExperts: scales and biases must be bf16");
        create(bits, groupSize, topK, maxTokens, device);
        detail::check(apt_moe_load_experts_quant(
                          h_.get(), static_cast<const uint32_t *>(gateUpQ.data),
                          static_cast<const uint16_t *>(gateUpS.data),
                          static_cast<const uint16_t *>(gateUpB.data),
                          static_cast<const uint32_t *>(downQ.data),
                          static_cast<const uint16_t *>(downS.data),
                          static_cast<const uint16_t *>(downB.data), bits, groupSize, dev ? 1 : 0),
                      h_.get(), "ESExperts (quantised)");
    }

    // dense: every expert, combined by W [T, E] (0 = unchosen)
    Array forward(const Array &x, const Array &W) const {
        const int T = check_x(x);
        if (!W.on_device || W.dim(0) != T || W.dim(1) != E_)
            throw std::runtime_error("ESExperts::forward: W must be [T, E] on the device");
        Array out = Array::device(Dtype::bfloat16, {T, H_});
        detail::check(apt_moe_experts_dense(h_.get(), static_cast<const uint16_t *>(x.data),
                                            static_cast<const uint16_t *>(W.data), T,
                                            static_cast<uint16_t *>(out.data), stream_),
                      h_.get(), "ESExperts::forward");
        return out;
    }

    // sparse: only the experts in idx [T, K] (int32), weighted by w [T, K]
    Array sparseForward(const Array &x, const Array &idx, const Array &w) const {
        const int T = check_x(x);
        if (!idx.on_device || !w.on_device || idx.dim(0) != T || w.dim(0) != T ||
            idx.dim(1) != K_ || w.dim(1) != K_)
            throw std::runtime_error("ESExperts::sparseForward: idx, w must be [T, K] on the device");
        Array out = Array::device(Dtype::bfloat16, {T, H_});
        detail::check(apt_moe_experts(h_.get(), static_cast<const uint16_t *>(x.data),
                                      static_cast<const int32_t *>(idx.data),
                                      static_cast<const uint16_t *>(w.data), T,
                                      static_cast<uint16_t *>(out.data), stream_),
                      h_.get(), "ESExperts::sparseForward");
        return out;
    }

    void setStream(void *s) { stream_ = s; }
    apt_moe_handle *raw() const { return h_.get(); }
    int numExperts() const { return E_; }
    int hiddenSize() const { return H_; }
    int intermediateSize() const { return I_; }

private:
    void create(int bits, int gs, int topK, int maxTokens, int device) {
        K_ = topK;
        apt_moe_config c{};
        c.hidden_size = H_;
        c.num_experts = E_;
        c.top_k_experts = topK;
        c.moe_intermediate_size = I_;
        c.rms_norm_eps = 1e-6f;
        c.enable_moe_block = 1;
        c.moe_sparse = 1;
        c.quant_bits = bits;
        c.quant_group_size = gs;
        c.max_tokens = maxTokens;
        c.device = device;
        h_ = detail::make_handle(c);
    }
    int check_x(const Array &x) const {
        detail::need(x, Dtype::bfloat16, 2, "ESExperts input");
        if (!x.on_device || x.dim(1) != H_) throw std::runtime_error("ESExperts: x must be [T, H] on the device");
        return (int)x.dim(0);
    }
    int E_ = 0, I_ = 0, H_ = 0, K_ = 8;
    detail::HandlePtr h_;
    void *stream_ = nullptr;
};

// esMakeExperts (ESWeightLoader.mm:145-154): pre-quantised from the bundle
// when "<gateUpName>.scales" exists (bits and group size from its manifest),
// else the bf16 banks (quantised now iff quantBits > 0).
inline ESExperts esMakeExperts(const ESWeightLoader &w, const std::string &gateUpName,
                               const std::string &downName, int quantBits, int groupSize,
                               int topK = 8, int maxTokens = 8192, int device = 0) {
    if (w.hasQuantized(gateUpName)) {
        auto g = w.quantized(gateUpName);
        auto d = w.quantized(downName);
        return ESExperts(Array::from_host(std::move(g.weight)), Array::from_host(std::move(g.scales)),
                         Array::from_host(std::move(g.biases)), Array::from_host(std::move(d.weight)),
                         Array::from_host(std::move(d.scales)), Array::from_host(std::move(d.biases)),
                         w.bundleBits(), w.bundleGroupSize(), topK, maxTokens, device);
    }
    return ESExperts(Array::from_host(w.get(gateUpName)), Array::from_host(w.get(downName)),
                     quantBits, groupSize, topK, maxTokens, device);
}

// The router of decoder layer `layer` (ESDecoderLayer.mm:35-37's keys).
inline ESRouter esMakeRouter(const ESWeightLoader &w, int layer, int numExperts, int topK,
                             int hiddenSize, float eps, int maxTokens = 8192, int device = 0) {
    return ESRouter(Array::from_host(w.layer(layer, "router.proj.weight")),
                    Array::from_host(w.layer(layer, "router.scale")),
                    Array::from_host(w.layer(layer, "router.per_expert_scale")), numExperts, topK,
                    hiddenSize, eps, Dtype::bfloat16, maxTokens, device);
}

}  // namespace es
