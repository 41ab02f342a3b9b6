// es_moe_cuda.hpp -- C++ wrapper over the C ABI (apt_moe.h) with the shape of
// the reference's es::ESRouter / es::ESExperts pair (aptransformer/ESRouter.h,
// aptransformer/ESExperts.h): what an Objective-C++ ESDecoderLayer would hold.
// Header-only; link libapt_moe.so.  Errors become std::runtime_error, as the
// reference's loader reports them (ESWeightLoader.mm:56-59).
#pragma once

#include <stdexcept>
#include <string>

#include "apt_moe.h"

namespace es {

class ESMoECuda {
public:
    // config.json text (top level or text_config) + runtime knobs
    ESMoECuda(const std::string &config_json, int max_tokens, bool moe_sparse = true,
              int quant_bits = 0, int device = 0) {
        apt_moe_config cfg{};
        check(apt_moe_config_from_json(config_json.c_str(), &cfg), "config");
        cfg.max_tokens = max_tokens;
        cfg.moe_sparse = moe_sparse ? 1 : 0;
        cfg.quant_bits = quant_bits;
        cfg.device = device;
        cfg_ = cfg;
        check(apt_moe_create(&cfg, &h_), "create");
    }
    ESMoECuda(const ESMoECuda &) = delete;
    ESMoECuda &operator=(const ESMoECuda &) = delete;
    ~ESMoECuda() { apt_moe_destroy(h_); }

    const apt_moe_config &config() const { return cfg_; }

    // ESRouter ctor: router.proj.weight [E,H], router.scale [H], router.per_expert_scale [E]
    void loadRouter(const uint16_t *proj, const uint16_t *scale, const uint16_t *pes,
                    bool on_device = false) {
        check(apt_moe_load_router(h_, proj, scale, pes, on_device), "load_router");
    }
    // ESExperts ctor: experts.gate_up_proj [E,2I,H], experts.down_proj [E,H,I]
    void loadExperts(const uint16_t *gate_up, const uint16_t *down, bool on_device = false) {
        check(apt_moe_load_experts_bf16(h_, gate_up, down, on_device), "load_experts");
    }
    // ESRouter::routeTopK on device pointers
    void routeTopK(const uint16_t *x, int T, int32_t *idx, uint16_t *w, void *stream = nullptr) {
        check(apt_moe_route(h_, x, T, idx, w, stream), "route");
    }
    // ESExperts::sparseForward on device pointers
    void sparseForward(const uint16_t *x, const int32_t *idx, const uint16_t *w, int T,
                       uint16_t *out, void *stream = nullptr) {
        check(apt_moe_experts(h_, x, idx, w, T, out, stream), "experts");
    }
    // MoE section of ESDecoderLayer::forward (router on x1, experts on pre_ff_ln_2(x1))
    void forward(const uint16_t *x1, const uint16_t *expert_in, int T, uint16_t *out,
                 void *stream = nullptr) {
        check(apt_moe_forward(h_, x1, expert_in, T, out, nullptr, nullptr, stream), "forward");
    }
    // MoE half with its norms: post_ff_ln_2(experts(pre_ff_ln_2(x1), router(x1)))
    void layerForward(const uint16_t *x1, const uint16_t *preFFLN2, const uint16_t *postFFLN2,
                      int T, uint16_t *out, void *stream = nullptr) {
        check(apt_moe_layer_forward(h_, x1, preFFLN2, postFFLN2, T, out, stream), "layer_forward");
    }
    // feed-forward tail of an MoE layer given the dense MLP output hmlp:
    // x2 = x1 + post_ff_ln(post_ff_ln_1(hmlp) + post_ff_ln_2(MoE(x1)))
    void decoderFF(const uint16_t *x1, const uint16_t *hmlp, const uint16_t *preFFLN2,
                   const uint16_t *postFFLN1, const uint16_t *postFFLN2, const uint16_t *postFFLN,
                   int T, uint16_t *x2, void *stream = nullptr) {
        check(apt_moe_decoder_ff(h_, x1, hmlp, preFFLN2, postFFLN1, postFFLN2, postFFLN, T, x2,
                                 stream),
              "decoder_ff");
    }
    // the whole feed-forward half with the dense MLP too (see ESMLPCuda)
    void decoderFFFull(apt_moe_handle *mlp, const uint16_t *x1, const uint16_t *preFFLN,
                       const uint16_t *preFFLN2, const uint16_t *postFFLN1,
                       const uint16_t *postFFLN2, const uint16_t *postFFLN, int T, uint16_t *x2,
                       void *stream = nullptr) {
        check(apt_moe_decoder_ff_full(h_, mlp, x1, preFFLN, preFFLN2, postFFLN1, postFFLN2,
                                      postFFLN, T, x2, stream),
              "decoder_ff_full");
    }
    apt_moe_handle *raw() { return h_; }
    // host buffers in and out (copies included)
    void forwardHost(const uint16_t *x_host, int T, uint16_t *out_host) {
        check(apt_moe_forward_host(h_, x_host, T, out_host, nullptr), "forward_host");
    }

private:
    void check(apt_status st, const char *what) {
        if (st != APT_OK)
            throw std::runtime_error(std::string("apt_moe ") + what + ": " +
                                     (h_ ? apt_moe_last_error(h_) : "status " + std::to_string(st)));
    }
    apt_moe_handle *h_ = nullptr;
    apt_moe_config cfg_{};
};

// ESMLPBlock (ESMLPBlock.mm:11-15) on the expert kernels: one-expert handle.
class ESMLPCuda {
public:
    ESMLPCuda(int hidden_size, int intermediate_size, int max_tokens, float rms_norm_eps = 1e-6f,
              int quant_bits = 0, int device = 0) {
        apt_moe_config cfg{};
        cfg.hidden_size = hidden_size;
        cfg.num_experts = 1;
        cfg.top_k_experts = 1;
        cfg.moe_intermediate_size = intermediate_size;
        cfg.rms_norm_eps = rms_norm_eps;
        cfg.enable_moe_block = 1;
        cfg.moe_sparse = 1;
        cfg.quant_bits = quant_bits;
        cfg.quant_group_size = 64;
        cfg.max_tokens = max_tokens;
        cfg.device = device;
        if (apt_moe_create(&cfg, &h_) != APT_OK) throw std::runtime_error("apt_moe mlp: create");
    }
    ESMLPCuda(const ESMLPCuda &) = delete;
    ESMLPCuda &operator=(const ESMLPCuda &) = delete;
    ~ESMLPCuda() { apt_moe_destroy(h_); }
    // gate_up = [gate_proj ; up_proj] as [1, 2I, H], down = down_proj as [1, H, I]
    void load(const uint16_t *gate_up, const uint16_t *down, bool on_device = false) {
        if (apt_moe_load_experts_bf16(h_, gate_up, down, on_device) != APT_OK)
            throw std::runtime_error(std::string("apt_moe mlp: ") + apt_moe_last_error(h_));
    }
    void forward(const uint16_t *x, int T, uint16_t *out, void *stream = nullptr) {
        if (apt_moe_mlp_forward(h_, x, T, out, stream) != APT_OK)
            throw std::runtime_error(std::string("apt_moe mlp: ") + apt_moe_last_error(h_));
    }
    apt_moe_handle *raw() { return h_; }

private:
    apt_moe_handle *h_ = nullptr;
};

}  // namespace es
