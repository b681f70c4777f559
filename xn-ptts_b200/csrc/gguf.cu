// GGUF checkpoints (host code): the reader, the reference's key remap and ptts_b200_load_gguf.
//
// Format (GGUF v2/v3, the published ggml spec): magic "GGUF", u32 version, u64 tensor count,
// u64 metadata count; metadata entries (string key, u32 type, value; arrays nest a u32 element
// type and a u64 count); tensor infos (string name, u32 n_dims, u64 dims[n_dims] innermost
// first, u32 ggml type, u64 offset into the data section); the data section starts at the next
// multiple of general.alignment (32 by default). Strings are a u64 length and the bytes.
// Element types read here: F32 (0), F16 (1), Q8_0 (8: blocks of an f16 scale and 32 int8) and
// BF16 (30). Every length and offset is checked against the file before it is used.
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "host.h"
#include "ptts_b200.h"

bool ptts_b200_flow_wants(const ptts_b200_flow* flow, const std::string& name);

namespace {

using namespace ptts::host;

constexpr uint32_t kF32 = 0, kF16 = 1, kQ8_0 = 8, kBF16 = 30;

struct Tensor {
    std::vector<uint64_t> dims;  // innermost first
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t numel() const {
        uint64_t n = 1;
        for (uint64_t d : dims) n *= d;
        return n;
    }
};

struct Reader {
    const std::vector<unsigned char>& b;
    size_t at = 0;
    const unsigned char* take(size_t n) {
        require(n <= b.size() && at <= b.size() - n, PTTS_B200_ERR_ARG, "GGUF file is truncated");
        const unsigned char* p = b.data() + at;
        at += n;
        return p;
    }
    template <class T>
    T get() {
        T v;
        std::memcpy(&v, take(sizeof(T)), sizeof(T));
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        require(n < (1u << 20), PTTS_B200_ERR_ARG, "GGUF string too long");
        const unsigned char* p = take((size_t)n);
        return std::string(reinterpret_cast<const char*>(p), (size_t)n);
    }
    // Skips one metadata value of `type`; returns it as an integer when it is one.
    uint64_t value(uint32_t type, int depth = 0) {
        require(depth < 4, PTTS_B200_ERR_ARG, "GGUF metadata nests too deep");
        switch (type) {
            case 0: case 1: case 7: return take(1)[0];
            case 2: case 3: return get<uint16_t>();
            case 4: case 5: return get<uint32_t>();
            case 6: take(4); return 0;
            case 8: str(); return 0;
            case 10: case 11: return get<uint64_t>();
            case 12: take(8); return 0;
            case 9: {
                const uint32_t et = get<uint32_t>();
                const uint64_t n = get<uint64_t>();
                require(n <= b.size(), PTTS_B200_ERR_ARG, "GGUF array too long");
                for (uint64_t i = 0; i < n; ++i) value(et, depth + 1);
                return 0;
            }
            default: fail(PTTS_B200_ERR_ARG, "GGUF metadata type " + std::to_string(type) + " is unknown");
        }
    }
};

// loader.rs:15-39: drop the tensors the runtime has no use for, rename the rest (every
// occurrence, the more specific names first).
bool remap_key(std::string& name) {
    if (name.find("flow.w_s_t") != std::string::npos || name.find("quantizer.vq") != std::string::npos ||
        name.find("quantizer.logvar_proj") != std::string::npos)
        return false;
    static const char* const kRules[][2] = {
        {"flow_lm.condition_provider.conditioners.speaker_wavs.output_proj.weight", "flow_lm.speaker_proj_weight"},
        {"flow_lm.condition_provider.conditioners.transcript_in_segment.", "flow_lm.conditioner."},
        {"flow_lm.backbone.", "flow_lm.transformer."},
        {"flow_lm.flow.", "flow_lm.flow_net."},
        {"mimi.model.", "mimi."},
    };
    for (const auto& r : kRules) {
        const std::string from = r[0], to = r[1];
        for (size_t p = name.find(from); p != std::string::npos; p = name.find(from, p + to.size()))
            name.replace(p, from.size(), to);
    }
    return true;
}

struct Gguf {
    std::vector<unsigned char> bytes;
    size_t data = 0;
    std::map<std::string, Tensor> tensors;  // remapped names

    void open(const char* path) {
        FILE* f = std::fopen(path, "rb");
        require(f != nullptr, PTTS_B200_ERR_ARG, std::string("cannot open ") + path);
        std::fseek(f, 0, SEEK_END);
        const long size = std::ftell(f);
        std::fseek(f, 0, SEEK_SET);
        bytes.resize(size > 0 ? (size_t)size : 0);
        const size_t got = bytes.empty() ? 0 : std::fread(bytes.data(), 1, bytes.size(), f);
        std::fclose(f);
        require(got == bytes.size(), PTTS_B200_ERR_ARG, std::string("cannot read ") + path);
        Reader r{bytes};
        require(r.get<uint32_t>() == 0x46554747u, PTTS_B200_ERR_ARG, "not a GGUF file (magic)");
        const uint32_t version = r.get<uint32_t>();
        require(version == 2 || version == 3, PTTS_B200_ERR_UNSUPPORTED,
                "GGUF version " + std::to_string(version) + " (2 and 3 are read)");
        const uint64_t n_tensors = r.get<uint64_t>(), n_meta = r.get<uint64_t>();
        require(n_tensors <= bytes.size() && n_meta <= bytes.size(), PTTS_B200_ERR_ARG, "GGUF counts are too large");
        uint64_t alignment = 32;
        for (uint64_t i = 0; i < n_meta; ++i) {
            const std::string key = r.str();
            const uint32_t type = r.get<uint32_t>();
            const uint64_t v = r.value(type);
            if (key == "general.alignment") alignment = v;
        }
        require(alignment > 0 && alignment <= 4096 && (alignment & (alignment - 1)) == 0, PTTS_B200_ERR_ARG,
                "GGUF alignment must be a power of two");
        for (uint64_t i = 0; i < n_tensors; ++i) {
            std::string name = r.str();
            Tensor t;
            const uint32_t nd = r.get<uint32_t>();
            require(nd >= 1 && nd <= 4, PTTS_B200_ERR_ARG, name + ": " + std::to_string(nd) + " dimensions");
            for (uint32_t d = 0; d < nd; ++d) {
                t.dims.push_back(r.get<uint64_t>());
                require(t.dims.back() >= 1 && t.dims.back() <= (1ull << 31), PTTS_B200_ERR_ARG,
                        name + ": a dimension is out of range");
            }
            require(t.numel() <= (1ull << 40), PTTS_B200_ERR_ARG, name + ": too many elements");
            t.type = r.get<uint32_t>();
            t.offset = r.get<uint64_t>();
            if (remap_key(name)) tensors[name] = t;
        }
        data = (r.at + alignment - 1) / alignment * alignment;
        require(data <= bytes.size(), PTTS_B200_ERR_ARG, "GGUF data section is missing");
    }

    const Tensor& find(const std::string& name) const {
        auto it = tensors.find(name);
        require(it != tensors.end(), PTTS_B200_ERR_STATE, "GGUF tensor missing: " + name);
        return it->second;
    }

    // The tensor's bytes, checked against the expected dims (innermost first) and the file's end.
    const unsigned char* bytes_of(const std::string& name, const std::vector<uint64_t>& want) const {
        const Tensor& t = find(name);
        std::vector<uint64_t> have = t.dims;
        while (have.size() > want.size() && have.back() == 1) have.pop_back();
        std::string shape;
        for (uint64_t d : want) shape += (shape.empty() ? "" : ", ") + std::to_string(d);
        require(have == want, PTTS_B200_ERR_ARG, name + ": expected dims (" + shape + ")");
        const uint64_t n = t.numel();
        uint64_t bytes_needed = 0;
        switch (t.type) {
            case kF32: bytes_needed = 4 * n; break;
            case kF16: case kBF16: bytes_needed = 2 * n; break;
            case kQ8_0:
                require(t.dims[0] % 32 == 0, PTTS_B200_ERR_ARG, name + ": q8_0 rows must be a multiple of 32");
                bytes_needed = n / 32 * 34;
                break;
            default:
                fail(PTTS_B200_ERR_UNSUPPORTED, name + ": ggml type " + std::to_string(t.type) +
                                                    " (F32, F16, BF16 and Q8_0 are read)");
        }
        require(t.offset <= bytes.size() - data && bytes_needed <= bytes.size() - data - t.offset,
                PTTS_B200_ERR_ARG, name + ": data past the end of the file");
        return bytes.data() + data + t.offset;
    }

    // The q8_0 blocks of a tensor stored as q8_0 (checked as above), else nullptr.
    const unsigned char* q8_0(const std::string& name, const std::vector<uint64_t>& want) const {
        return find(name).type == kQ8_0 ? bytes_of(name, want) : nullptr;
    }

    // The tensor as f32, checked against the expected dims (innermost first).
    std::vector<float> f32(const std::string& name, const std::vector<uint64_t>& want) const {
        const Tensor& t = find(name);
        const unsigned char* p = bytes_of(name, want);
        const uint64_t n = t.numel();
        std::vector<float> out(n);
        if (t.type == kF32) {
            std::memcpy(out.data(), p, 4 * n);
        } else if (t.type == kF16) {
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                out[i] = f16_value(h);
            }
        } else if (t.type == kBF16) {
            for (uint64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, p + 2 * i, 2);
                const uint32_t u = (uint32_t)h << 16;
                std::memcpy(&out[i], &u, 4);
            }
        } else {  // q8_0: W = q * d per block of 32 (exact in f32)
            for (uint64_t blk = 0; blk < n / 32; ++blk) {
                uint16_t d16;
                std::memcpy(&d16, p + 34 * blk, 2);
                const float d = f16_value(d16);
                for (int j = 0; j < 32; ++j) out[blk * 32 + j] = (float)(int8_t)p[34 * blk + 2 + j] * d;
            }
        }
        return out;
    }
};

void check_rc(int rc) {
    if (rc != PTTS_B200_OK) fail(rc, ptts_b200_last_error());
}

}  // namespace

extern "C" int ptts_b200_gguf_remap_key(const char* name, char* out, int out_size) {
    if (!name || !out || out_size <= 0) return PTTS_B200_ERR_ARG;
    std::string n(name);
    if (!remap_key(n)) return 0;
    if ((int)n.size() + 1 > out_size) return PTTS_B200_ERR_ARG;
    std::memcpy(out, n.c_str(), n.size() + 1);
    return 1;
}

extern "C" int ptts_b200_load_gguf(ptts_b200_model* model, ptts_b200_flow* flow, const char* path) {
    return guarded([&] {
        require(model && path, PTTS_B200_ERR_ARG, "NULL argument");
        ptts_b200_config c;
        check_rc(ptts_b200_model_config(model, &c));
        Gguf g;
        g.open(path);
        const uint64_t dm = c.d_model, hd = (uint64_t)c.num_heads * c.head_dim;
        const uint64_t nqkv = hd + 2ull * c.num_kv_heads * c.head_dim, ff = c.dim_feedforward;
        for (int l = 0; l < c.num_layers; ++l) {
            const std::string p = "flow_lm.transformer.layers." + std::to_string(l) + ".";
            // q8_0 linears (the reference's model.q8.gguf) keep their blocks: the layer then
            // holds the int8 values and block scales beside the exact f16 planes.
            const unsigned char* b_qkv = g.q8_0(p + "self_attn.in_proj.weight", {dm, nqkv});
            const unsigned char* b_out = g.q8_0(p + "self_attn.out_proj.weight", {hd, dm});
            const unsigned char* b_1 = g.q8_0(p + "linear1.weight", {dm, ff});
            const unsigned char* b_2 = g.q8_0(p + "linear2.weight", {ff, dm});
            const auto n1w = g.f32(p + "norm1.weight", {dm}), n1b = g.f32(p + "norm1.bias", {dm});
            const auto n2w = g.f32(p + "norm2.weight", {dm}), n2b = g.f32(p + "norm2.bias", {dm});
            if (b_qkv && b_out && b_1 && b_2) {
                ptts_b200_layer_weights_q8_0 q{b_qkv, b_out, b_1, b_2, n1w.data(), n1b.data(), n2w.data(), n2b.data()};
                check_rc(ptts_b200_model_load_layer_q8_0(model, l, &q));
                continue;
            }
            const auto qkv = g.f32(p + "self_attn.in_proj.weight", {dm, nqkv});
            const auto out = g.f32(p + "self_attn.out_proj.weight", {hd, dm});
            const auto l1 = g.f32(p + "linear1.weight", {dm, ff});
            const auto l2 = g.f32(p + "linear2.weight", {ff, dm});
            ptts_b200_layer_weights_f32 w{qkv.data(), out.data(), l1.data(), l2.data(),
                                          n1w.data(), n1b.data(), n2w.data(), n2b.data()};
            check_rc(ptts_b200_model_load_layer_f32(model, l, &w));
        }
        if (!flow) return;
        const std::string pre = "flow_lm.";
        for (const auto& kv : g.tensors) {
            if (kv.first.compare(0, pre.size(), pre) != 0) continue;
            const std::string name = kv.first.substr(pre.size());
            if (!ptts_b200_flow_wants(flow, name)) continue;  // conditioner, emb_mean, ... belong elsewhere
            const std::vector<float> v = g.f32(kv.first, kv.second.dims);
            check_rc(ptts_b200_flow_set_tensor(flow, name.c_str(), v.data(), (int64_t)v.size()));
        }
        check_rc(ptts_b200_flow_finish(flow));
    });
}
