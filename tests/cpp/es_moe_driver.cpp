// Drives the MoE block of one decoder layer from C++ the way ESDecoderLayer's
// constructor and forward do (ESDecoderLayer.mm:35-43, :67-75), through
// include/es_weight_loader.hpp and include/es_moe.hpp.
//
//   es_moe_driver list <dir> <layer>
//       CPU only: loads the layer's MoE tensors and prints, per tensor, its
//       name, dtype, shape and a byte checksum (the loader's behaviour).
//   es_moe_driver run <dir> <layer> <T> <x.bin> <out_prefix> [quant_bits]
//       GPU: ESRouter + esMakeExperts from the checkpoint or bundle in <dir>,
//       config from <dir>/config.json; x.bin holds [T, H] bf16.  Writes
//       <out_prefix>.idx (int32 [T,K]), .w (bf16 [T,K]), .sparse (bf16
//       [T,H], sparseForward) and, for bf16 experts, .dense (bf16 [T,H],
//       routeWeights + the dense forward).
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "es_weight_loader.hpp"

#ifndef ES_DRIVER_CPU_ONLY
#include "es_moe.hpp"
#endif

static const char *dtype_name(es::Dtype d) {
    switch (d) {
        case es::Dtype::bfloat16: return "bf16";
        case es::Dtype::float16: return "f16";
        case es::Dtype::float32: return "f32";
        case es::Dtype::uint32: return "u32";
        case es::Dtype::int32: return "i32";
        default: return "u8";
    }
}

[[maybe_unused]] static void write_bytes(const std::string &path, const void *p, size_t n) {
    std::ofstream f(path, std::ios::binary);
    f.write(static_cast<const char *>(p), (std::streamsize)n);
}

int main(int argc, char **argv) {
    if (argc < 4) {
        std::cerr << "usage: es_moe_driver list <dir> <layer> | run <dir> <layer> <T> <x.bin> "
                     "<out_prefix> [quant_bits]\n";
        return 2;
    }
    try {
        const std::string mode = argv[1], dir = argv[2];
        const int layer = std::atoi(argv[3]);
        es::ESWeightLoader w(dir);
        if (mode == "list") {
            const char *sufs[] = {"router.proj.weight", "router.scale", "router.per_expert_scale",
                                  "experts.gate_up_proj", "experts.down_proj"};
            for (const char *suf : sufs) {
                std::vector<std::string> names{w.layerKey(layer, suf)};
                if (std::string(suf).rfind("experts.", 0) == 0 && w.hasQuantized(names[0])) {
                    names.push_back(names[0] + ".scales");
                    names.push_back(names[0] + ".biases");
                }
                for (const std::string &n : names) {
                    es::HostTensor t = w.get(n);
                    unsigned long long sum = 0;
                    for (uint8_t b : t.bytes) sum = sum * 1099511628211ull + b;
                    std::printf("%s %s", n.c_str(), dtype_name(t.dtype));
                    for (int64_t d : t.shape) std::printf(" %lld", (long long)d);
                    std::printf(" %llu\n", sum);
                }
            }
            std::printf("bundle=%d bits=%d group=%d quantized=%d\n", w.isBundle() ? 1 : 0,
                        w.bundleBits(), w.bundleGroupSize(),
                        w.hasQuantized(w.layerKey(layer, "experts.gate_up_proj")) ? 1 : 0);
            return 0;
        }
#ifdef ES_DRIVER_CPU_ONLY
        std::cerr << "built without the CUDA classes\n";
        return 2;
#else
        if (mode != "run" || argc < 7) {
            std::cerr << "bad arguments\n";
            return 2;
        }
        const int T = std::atoi(argv[4]);
        const std::string out = argv[6];
        const int qbits = argc > 7 ? std::atoi(argv[7]) : 0;
        const es::Json cfg = es::Json::parse(es::read_file(es::join_path(dir, "config.json")));
        const es::Json &tc = cfg.find("text_config") ? cfg.at("text_config") : cfg;
        const int H = (int)tc.at("hidden_size").num, E = (int)tc.at("num_experts").num;
        const int K = (int)tc.at("top_k_experts").num;
        const float eps = tc.find("rms_norm_eps") ? (float)tc.at("rms_norm_eps").num : 1e-6f;
        es::ESRouter router = es::esMakeRouter(w, layer, E, K, H, eps, T);
        es::ESExperts experts = es::esMakeExperts(w, w.layerKey(layer, "experts.gate_up_proj"),
                                                  w.layerKey(layer, "experts.down_proj"), qbits,
                                                  64, K, T);
        std::string xs = es::read_file(argv[5]);
        if (xs.size() != (size_t)T * H * 2) throw std::runtime_error("x.bin is not [T, H] bf16");
        es::Array x = es::Array::view(&xs[0], es::Dtype::bfloat16, {T, H}, false).to_device();
        auto tk = router.routeTopK(x);
        es::Array sparse = experts.sparseForward(x, tk.idx, tk.w);
        const auto ib = tk.idx.to_host_bytes(), wb = tk.w.to_host_bytes(),
                   sb = sparse.to_host_bytes();
        write_bytes(out + ".idx", ib.data(), ib.size());
        write_bytes(out + ".w", wb.data(), wb.size());
        write_bytes(out + ".sparse", sb.data(), sb.size());
        if (!w.hasQuantized(w.layerKey(layer, "experts.gate_up_proj"))) {
            es::Array W = router.routeWeights(x);
            es::Array dense = experts.forward(x, W);
            const auto db = dense.to_host_bytes();
            write_bytes(out + ".dense", db.data(), db.size());
        }
        // an error path: a token count above the workspace must throw
        try {
            es::Array big = es::Array::device(es::Dtype::bfloat16, {T + 1, H});
            router.routeTopK(big);
            std::cerr << "expected an error for T > max_tokens\n";
            return 3;
        } catch (const std::runtime_error &) {
        }
        std::printf("ok T=%d H=%d E=%d K=%d\n", T, H, E, K);
        return 0;
#endif
    } catch (const std::exception &e) {
        std::cerr << e.what() << "\n";
        return 1;
    }
}
