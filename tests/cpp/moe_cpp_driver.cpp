// Drives the MoE block from C++ through include/es_moe_cuda.hpp: reads
// weights and tokens from raw files, runs forwardHost, writes the output.
// Usage: moe_cpp_driver <config.json> <dir> <T>
//   dir holds proj.bin scale.bin pes.bin gate_up.bin down.bin x.bin (bf16)
#include <cstdio>
#include <fstream>
#include <iostream>
#include <sstream>
#include <vector>

#include "es_moe_cuda.hpp"

static std::vector<uint16_t> read_bf16(const std::string &path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open " + path);
    const std::streamsize n = f.tellg();
    f.seekg(0);
    std::vector<uint16_t> v(n / 2);
    f.read(reinterpret_cast<char *>(v.data()), n);
    return v;
}

int main(int argc, char **argv) {
    if (argc != 4) {
        std::cerr << "usage: moe_cpp_driver <config.json> <dir> <T>\n";
        return 2;
    }
    try {
        std::ifstream cf(argv[1]);
        std::stringstream ss;
        ss << cf.rdbuf();
        const std::string dir = argv[2];
        const int T = std::atoi(argv[3]);
        es::ESMoECuda moe(ss.str(), T, /*moe_sparse=*/true);
        auto proj = read_bf16(dir + "/proj.bin"), scale = read_bf16(dir + "/scale.bin"),
             pes = read_bf16(dir + "/pes.bin"), gu = read_bf16(dir + "/gate_up.bin"),
             dn = read_bf16(dir + "/down.bin"), x = read_bf16(dir + "/x.bin");
        moe.loadRouter(proj.data(), scale.data(), pes.data());
        moe.loadExperts(gu.data(), dn.data());
        std::vector<uint16_t> out((size_t)T * moe.config().hidden_size);
        moe.forwardHost(x.data(), T, out.data());
        std::ofstream of(dir + "/out.bin", std::ios::binary);
        of.write(reinterpret_cast<const char *>(out.data()), out.size() * 2);
        // an error path: T above max_tokens must raise
        try {
            moe.forwardHost(x.data(), T + 1, out.data());
            std::cerr << "expected an error for T > max_tokens\n";
            return 3;
        } catch (const std::runtime_error &) {
        }
        std::printf("ok T=%d H=%d\n", T, moe.config().hidden_size);
        return 0;
    } catch (const std::exception &e) {
        std::cerr << e.what() << "\n";
        return 1;
    }
}
