// es_weight_loader.hpp -- the MoE-relevant part of es::ESWeightLoader
// (aptransformer/ESWeightLoader.h, ESWeightLoader.mm:24-61, :77-110, :143-154)
// in plain C++17 for hosts of this library: HF safetensors checkpoints
// (sharded through model.safetensors.index.json, or one model.safetensors)
// and Apertura .apml bundles (manifest.json -> default variant -> files).
//
//   HF:     keys under the text prefix "model.language_model." are kept with
//           the prefix stripped; floating-point tensors are cast to bf16 (the
//           compute dtype) when read, as ESWeightLoader.mm:52 casts them.
//   bundle: tensors are adopted verbatim (packed uint32 stays uint32); bits,
//           group size and embed bits come from the default variant's
//           "quantization" object.
//   hasQuantized(name): "<name>.scales" exists (ESWeightLoader.h:46).
//
// Header-only, no CUDA and no third-party dependency: a small JSON reader
// (objects, arrays, strings, numbers, literals) parses the safetensors
// headers, the index and the manifest.  Tensors are read from their files on
// first use (a checkpoint's MoE layer is read without loading the rest).
// Errors throw std::runtime_error, as the reference's loader does.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace es {

// ---------------------------------------------------------------- JSON

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json *find(const std::string &k) const {
        for (const auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
    const Json &at(const std::string &k) const {
        const Json *j = find(k);
        if (!j) throw std::runtime_error("json: missing key '" + k + "'");
        return *j;
    }

    static Json parse(const std::string &text) {
        size_t i = 0;
        Json j = value(text, i);
        ws(text, i);
        if (i != text.size()) throw std::runtime_error("json: trailing characters");
        return j;
    }

private:
    static void ws(const std::string &s, size_t &i) {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    static std::string string_lit(const std::string &s, size_t &i) {
        if (s[i] != '"') throw std::runtime_error("json: expected a string");
        std::string out;
        for (++i; i < s.size() && s[i] != '"'; ++i) {
            if (s[i] != '\\') {
                out += s[i];
                continue;
            }
            if (++i >= s.size()) break;
            switch (s[i]) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {  // code point -> UTF-8 (surrogate pairs are not needed for keys here)
                    if (i + 4 >= s.size()) throw std::runtime_error("json: bad \\u escape");
                    const unsigned cp = (unsigned)std::stoul(s.substr(i + 1, 4), nullptr, 16);
                    i += 4;
                    if (cp < 0x80) {
                        out += (char)cp;
                    } else if (cp < 0x800) {
                        out += (char)(0xC0 | (cp >> 6));
                        out += (char)(0x80 | (cp & 0x3F));
                    } else {
                        out += (char)(0xE0 | (cp >> 12));
                        out += (char)(0x80 | ((cp >> 6) & 0x3F));
                        out += (char)(0x80 | (cp & 0x3F));
                    }
                    break;
                }
                default: out += s[i];
            }
        }
        if (i >= s.size()) throw std::runtime_error("json: unterminated string");
        ++i;
        return out;
    }
    static Json value(const std::string &s, size_t &i) {
        ws(s, i);
        if (i >= s.size()) throw std::runtime_error("json: unexpected end");
        Json j;
        const char c = s[i];
        if (c == '{') {
            j.kind = Object;
            ++i;
            ws(s, i);
            if (s[i] == '}') {
                ++i;
                return j;
            }
            for (;;) {
                ws(s, i);
                std::string k = string_lit(s, i);
                ws(s, i);
                if (s[i] != ':') throw std::runtime_error("json: expected ':'");
                ++i;
                j.obj.emplace_back(std::move(k), value(s, i));
                ws(s, i);
                if (s[i] == ',') {
                    ++i;
                    continue;
                }
                if (s[i] == '}') {
                    ++i;
                    return j;
                }
                throw std::runtime_error("json: expected ',' or '}'");
            }
        }
        if (c == '[') {
            j.kind = Array;
            ++i;
            ws(s, i);
            if (s[i] == ']') {
                ++i;
                return j;
            }
            for (;;) {
                j.arr.push_back(value(s, i));
                ws(s, i);
                if (s[i] == ',') {
                    ++i;
                    continue;
                }
                if (s[i] == ']') {
                    ++i;
                    return j;
                }
                throw std::runtime_error("json: expected ',' or ']'");
            }
        }
        if (c == '"') {
            j.kind = String;
            j.str = string_lit(s, i);
            return j;
        }
        if (s.compare(i, 4, "true") == 0) {
            j.kind = Bool;
            j.b = true;
            i += 4;
            return j;
        }
        if (s.compare(i, 5, "false") == 0) {
            j.kind = Bool;
            i += 5;
            return j;
        }
        if (s.compare(i, 4, "null") == 0) {
            i += 4;
            return j;
        }
        size_t n = 0;
        j.kind = Number;
        j.num = std::stod(s.substr(i, 64), &n);
        if (!n) throw std::runtime_error("json: bad value");
        i += n;
        return j;
    }
};

inline std::string read_file(const std::string &path) {
    std::unique_ptr<FILE, int (*)(FILE *)> f(std::fopen(path.c_str(), "rb"), &std::fclose);
    if (!f) throw std::runtime_error("cannot open " + path);
    std::string out;
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f.get())) > 0) out.append(buf, n);
    return out;
}

inline bool file_exists(const std::string &path) {
    FILE *f = std::fopen(path.c_str(), "rb");
    if (f) std::fclose(f);
    return f != nullptr;
}

inline std::string join_path(const std::string &a, const std::string &b) {
    if (a.empty()) return b;
    return a.back() == '/' ? a + b : a + "/" + b;
}

// ---------------------------------------------------------------- tensors

enum class Dtype { bfloat16, float16, float32, uint32, int32, uint8 };

inline size_t dtype_size(Dtype d) {
    switch (d) {
        case Dtype::bfloat16:
        case Dtype::float16: return 2;
        case Dtype::uint8: return 1;
        default: return 4;
    }
}

// A tensor in host memory: dtype, shape and its bytes.
struct HostTensor {
    Dtype dtype = Dtype::bfloat16;
    std::vector<int64_t> shape;
    std::vector<uint8_t> bytes;
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
    template <typename T>
    const T *data() const { return reinterpret_cast<const T *>(bytes.data()); }
};

// float -> bf16 bits, round to nearest even (the compute-dtype cast)
inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

inline float f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t u;
    if (e == 0) {
        if (m == 0) {
            u = s;
        } else {  // subnormal: normalise
            int ee = -1;
            uint32_t mm = m;
            do {
                ++ee;
                mm <<= 1;
            } while (!(mm & 0x400u));
            u = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// One safetensors file: its header (name -> dtype, shape, byte range) and
// on-demand reads of single tensors.
class SafetensorsFile {
public:
    struct Entry {
        Dtype dtype;
        std::vector<int64_t> shape;
        uint64_t begin, end;  // absolute file offsets
    };

    explicit SafetensorsFile(std::string path) : path_(std::move(path)) {
        std::unique_ptr<FILE, int (*)(FILE *)> f(std::fopen(path_.c_str(), "rb"), &std::fclose);
        if (!f) throw std::runtime_error("cannot open " + path_);
        uint8_t lenb[8];
        if (std::fread(lenb, 1, 8, f.get()) != 8) throw std::runtime_error(path_ + ": short file");
        uint64_t n = 0;
        for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];  // little-endian
        if (n > (1ull << 30)) throw std::runtime_error(path_ + ": implausible header size");
        std::string hdr(n, '\0');
        if (std::fread(&hdr[0], 1, n, f.get()) != n) throw std::runtime_error(path_ + ": short header");
        const Json j = Json::parse(hdr);
        for (const auto &kv : j.obj) {
            if (kv.first == "__metadata__") continue;
            Entry e;
            const std::string dt = kv.second.at("dtype").str;
            if (dt == "BF16") e.dtype = Dtype::bfloat16;
            else if (dt == "F16") e.dtype = Dtype::float16;
            else if (dt == "F32") e.dtype = Dtype::float32;
            else if (dt == "U32") e.dtype = Dtype::uint32;
            else if (dt == "I32") e.dtype = Dtype::int32;
            else if (dt == "U8") e.dtype = Dtype::uint8;
            else throw std::runtime_error(path_ + ": unsupported dtype " + dt + " of " + kv.first);
            for (const Json &d : kv.second.at("shape").arr) e.shape.push_back((int64_t)d.num);
            const Json &off = kv.second.at("data_offsets");
            e.begin = 8 + n + (uint64_t)off.arr.at(0).num;
            e.end = 8 + n + (uint64_t)off.arr.at(1).num;
            entries_.emplace(kv.first, std::move(e));
        }
    }

    const std::map<std::string, Entry> &entries() const { return entries_; }

    HostTensor read(const std::string &name) const {
        auto it = entries_.find(name);
        if (it == entries_.end()) throw std::runtime_error(path_ + ": no tensor " + name);
        const Entry &e = it->second;
        HostTensor t;
        t.dtype = e.dtype;
        t.shape = e.shape;
        if ((uint64_t)(t.numel() * (int64_t)dtype_size(e.dtype)) != e.end - e.begin)
            throw std::runtime_error(path_ + ": size mismatch for " + name);
        t.bytes.resize(e.end - e.begin);
        std::unique_ptr<FILE, int (*)(FILE *)> f(std::fopen(path_.c_str(), "rb"), &std::fclose);
        if (!f || std::fseek(f.get(), (long)e.begin, SEEK_SET) != 0 ||
            std::fread(t.bytes.data(), 1, t.bytes.size(), f.get()) != t.bytes.size())
            throw std::runtime_error(path_ + ": cannot read " + name);
        return t;
    }

private:
    std::string path_;
    std::map<std::string, Entry> entries_;
};

// ---------------------------------------------------------------- loader

class ESWeightLoader {
public:
    // dir: an HF snapshot (config.json, shards, index) or an .apml bundle
    // (manifest.json present)
    explicit ESWeightLoader(const std::string &dir) {
        if (file_exists(join_path(dir, "manifest.json"))) loadBundle(dir);
        else loadHF(dir);
    }

    bool has(const std::string &name) const { return where_.count(name) > 0; }
    size_t count() const { return where_.size(); }

    // The tensor `name` (text-decoder relative), read from its file now; HF
    // floating-point tensors come back as bf16, bundle tensors verbatim.
    HostTensor get(const std::string &name) const {
        auto it = where_.find(name);
        if (it == where_.end()) throw std::runtime_error("ESWeightLoader: missing tensor '" + name + "'");
        HostTensor t = files_.at(it->second.first)->read(it->second.second);
        return isBundle_ ? t : to_compute_dtype(std::move(t));
    }
    HostTensor layer(int idx, const std::string &suffix) const { return get(layerKey(idx, suffix)); }
    std::string layerKey(int idx, const std::string &suffix) const {
        return "layers." + std::to_string(idx) + "." + suffix;
    }

    bool isBundle() const { return isBundle_; }
    bool hasQuantized(const std::string &name) const { return has(name + ".scales"); }
    struct QuantTriple {
        HostTensor weight, scales, biases;
    };
    QuantTriple quantized(const std::string &name) const {
        return {get(name), get(name + ".scales"), get(name + ".biases")};
    }
    int bundleBits() const { return bundleBits_; }
    int bundleGroupSize() const { return bundleGroupSize_; }
    int bundleEmbedBits() const { return bundleEmbedBits_; }

private:
    static constexpr const char *kTextPrefix = "model.language_model.";

    static HostTensor to_compute_dtype(HostTensor t) {
        if (t.dtype == Dtype::float32 || t.dtype == Dtype::float16) {
            const int64_t n = t.numel();
            std::vector<uint8_t> out((size_t)n * 2);
            uint16_t *o = reinterpret_cast<uint16_t *>(out.data());
            for (int64_t i = 0; i < n; ++i) {
                float f;
                if (t.dtype == Dtype::float32) std::memcpy(&f, t.bytes.data() + 4 * i, 4);
                else f = f16_to_f32(reinterpret_cast<const uint16_t *>(t.bytes.data())[i]);
                o[i] = f32_to_bf16(f);
            }
            t.bytes.swap(out);
            t.dtype = Dtype::bfloat16;
        }
        return t;
    }

    int file_index(const std::string &path) {
        auto it = file_ids_.find(path);
        if (it != file_ids_.end()) return it->second;
        files_.push_back(std::make_unique<SafetensorsFile>(path));
        return file_ids_[path] = (int)files_.size() - 1;
    }

    void add_file_keys(const std::string &path, bool strip_prefix) {
        const int id = file_index(path);
        const std::string pre = kTextPrefix;
        for (const auto &kv : files_[id]->entries()) {
            if (strip_prefix) {
                if (kv.first.compare(0, pre.size(), pre) != 0) continue;  // vision / audio
                where_[kv.first.substr(pre.size())] = {id, kv.first};
            } else {
                where_[kv.first] = {id, kv.first};
            }
        }
    }

    void loadHF(const std::string &dir) {
        const std::string idx = join_path(dir, "model.safetensors.index.json");
        if (file_exists(idx)) {
            const Json j = Json::parse(read_file(idx));
            const std::string pre = kTextPrefix;
            std::map<std::string, std::string> shard_of;
            for (const auto &kv : j.at("weight_map").obj)
                if (kv.first.compare(0, pre.size(), pre) == 0) shard_of[kv.first] = kv.second.str;
            for (const auto &kv : shard_of) {
                const int id = file_index(join_path(dir, kv.second));
                where_[kv.first.substr(pre.size())] = {id, kv.first};
            }
        } else {
            const std::string single = join_path(dir, "model.safetensors");
            if (!file_exists(single))
                throw std::runtime_error("ESWeightLoader: no model.safetensors(.index.json) in " + dir);
            add_file_keys(single, true);
        }
    }

    void loadBundle(const std::string &dir) {
        isBundle_ = true;
        const Json m = Json::parse(read_file(join_path(dir, "manifest.json")));
        const Json *kind = m.find("kind");
        if (kind && kind->kind == Json::String && kind->str != "apertura-model")
            throw std::runtime_error("ESWeightLoader: " + dir + " is not an Apertura model bundle");
        const std::string def = m.at("default_variant").str;
        const Json *variant = nullptr;
        for (const Json &v : m.at("variants").arr)
            if (v.find("id") && v.at("id").str == def) variant = &v;
        if (!variant) throw std::runtime_error("ESWeightLoader: default_variant not found in manifest");
        if (const Json *q = variant->find("quantization")) {
            if (const Json *b = q->find("bits")) bundleBits_ = (int)b->num;
            if (const Json *g = q->find("group_size")) bundleGroupSize_ = (int)g->num;
            if (const Json *e = q->find("embed_bits")) bundleEmbedBits_ = (int)e->num;
        }
        const std::string base = join_path(dir, variant->at("path").str);
        for (const Json &f : variant->at("files").arr) add_file_keys(join_path(base, f.str), false);
    }

    std::vector<std::unique_ptr<SafetensorsFile>> files_;
    std::unordered_map<std::string, int> file_ids_;
    std::unordered_map<std::string, std::pair<int, std::string>> where_;  // key -> (file, stored name)
    bool isBundle_ = false;
    int bundleBits_ = 0, bundleGroupSize_ = 64, bundleEmbedBits_ = 0;
};

}  // namespace es
