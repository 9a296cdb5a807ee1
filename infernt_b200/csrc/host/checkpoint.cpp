// checkpoint.cpp — INFT v1 checkpoints: CheckpointLoader (the reference's
// loader/checkpoint_loader.cpp:42-161 interface, include/checkpoint_loader.h)
// and the C entry points infernt_checkpoint_* (include/infernt_capi.h).
//
// model.bin is read one tensor at a time (a payload is converted and placed
// before the next is read, so host memory holds one tensor at most): every
// recognised tensor goes to its slot of the plan's weight order [embedding,
// final_norm, lm_head, per layer attn_norm, q, k, v, o, ffn_norm, gate, up,
// down], norms and embedding FP32, projections and lm_head in the
// configured weight dtype (bf16 rounded to nearest even, as
// infernt_round_bf16).  Unlike the reference, element counts are checked
// against the configuration and reads are checked for truncation.  A tensor
// the file lacks stays empty in CheckpointLoader::load_weights (as in the
// reference); infernt_checkpoint_load, which feeds an engine, requires every
// tensor but lm_head.
#include <cuda_runtime.h>

#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <new>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../../include/checkpoint_loader.h"
#include "../../../include/infernt_capi.h"
#include "../../../include/infernt_seed.h"
#include "../internal.h"

namespace {

constexpr uint32_t kMagic = 0x494E4654u;  // "INFT"
constexpr uint32_t kVersion = 1;

// ---- config.json: the scalar members of the top-level object ----

struct JsonScalars {
    std::map<std::string, std::string> strings;
    std::map<std::string, double> numbers;
};

void skip_ws(const std::string& s, size_t& i) {
    while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
}

std::string parse_string(const std::string& s, size_t& i) {
    // s[i] == '"'; escapes kept literally except \" and \\ (names and
    // architectures carry no others)
    std::string out;
    ++i;
    while (i < s.size() && s[i] != '"') {
        if (s[i] == '\\' && i + 1 < s.size()) ++i;
        out.push_back(s[i++]);
    }
    if (i >= s.size()) throw std::runtime_error("config.json: unterminated string");
    ++i;
    return out;
}

// Skips a nested object or array starting at s[i] ('{' or '[').
void skip_nested(const std::string& s, size_t& i) {
    int depth = 0;
    while (i < s.size()) {
        const char c = s[i];
        if (c == '"') {
            parse_string(s, i);
            continue;
        }
        if (c == '{' || c == '[') ++depth;
        if (c == '}' || c == ']') {
            --depth;
            if (depth == 0) {
                ++i;
                return;
            }
        }
        ++i;
    }
    throw std::runtime_error("config.json: unbalanced brackets");
}

JsonScalars parse_top_level(const std::string& s) {
    JsonScalars out;
    size_t i = 0;
    skip_ws(s, i);
    if (i >= s.size() || s[i] != '{') throw std::runtime_error("config.json: not a JSON object");
    ++i;
    for (;;) {
        skip_ws(s, i);
        if (i < s.size() && s[i] == '}') break;
        if (i >= s.size() || s[i] != '"') throw std::runtime_error("config.json: expected a key");
        const std::string key = parse_string(s, i);
        skip_ws(s, i);
        if (i >= s.size() || s[i] != ':') throw std::runtime_error("config.json: expected ':' after \"" + key + "\"");
        ++i;
        skip_ws(s, i);
        if (i >= s.size()) throw std::runtime_error("config.json: truncated");
        if (s[i] == '"') {
            out.strings[key] = parse_string(s, i);
        } else if (s[i] == '{' || s[i] == '[') {
            skip_nested(s, i);
        } else {
            const size_t j = i;
            while (i < s.size() && s[i] != ',' && s[i] != '}' && !std::isspace(static_cast<unsigned char>(s[i]))) ++i;
            const std::string tok = s.substr(j, i - j);
            char* end = nullptr;
            const double v = std::strtod(tok.c_str(), &end);
            if (end && *end == '\0' && !tok.empty()) out.numbers[key] = v;  // true / false / null are skipped
        }
        skip_ws(s, i);
        if (i < s.size() && s[i] == ',') {
            ++i;
            continue;
        }
        if (i < s.size() && s[i] == '}') break;
        throw std::runtime_error("config.json: expected ',' or '}' after \"" + key + "\"");
    }
    return out;
}

ModelConfig config_from_json(const std::string& path) {
    std::ifstream f(path);
    if (!f.is_open()) throw std::runtime_error("Failed to open config file: " + path);
    std::stringstream buf;
    buf << f.rdbuf();
    const JsonScalars js = parse_top_level(buf.str());
    auto num = [&](const char* k, double dflt) {
        auto it = js.numbers.find(k);
        return it == js.numbers.end() ? dflt : it->second;
    };
    ModelConfig c;
    auto arch = js.strings.find("architecture");
    c.architecture = arch == js.strings.end() || arch->second.empty() ? "LlamaForCausalLM" : arch->second;
    c.vocab_size = static_cast<int>(num("vocab_size", 0));
    c.hidden_size = static_cast<int>(num("hidden_size", 0));
    c.num_layers = static_cast<int>(num("num_layers", 0));
    c.num_attention_heads = static_cast<int>(num("num_attention_heads", 0));
    c.num_key_value_heads = static_cast<int>(num("num_key_value_heads", 0));
    c.intermediate_size = static_cast<int>(num("intermediate_size", 0));
    c.max_seq_len = static_cast<int>(num("max_seq_len", 2048));
    c.head_dim = static_cast<int>(num("head_dim", 0));
    c.rms_norm_eps = static_cast<float>(num("rms_norm_eps", 1e-5));
    c.rope_theta = static_cast<float>(num("rope_theta", 10000.0));
    auto wd = js.strings.find("weight_dtype");
    if (wd != js.strings.end()) {
        if (wd->second == "bf16" || wd->second == "bfloat16")
            c.weight_dtype = DType::BF16;
        else if (wd->second == "fp32" || wd->second == "float32")
            c.weight_dtype = DType::FP32;
        else
            throw std::runtime_error("config.json: weight_dtype \"" + wd->second + "\" (bf16 or fp32)");
    }
    c.derive_computed_fields();
    c.validate();
    return c;
}

// ---- model.bin ----

// Slot of a tensor name in the weight order, or -1 for a name the model
// does not use.
int slot_of(const std::string& name, int num_layers) {
    if (name == "model.embed_tokens.weight") return 0;
    if (name == "model.norm.weight") return 1;
    if (name == "lm_head.weight") return 2;
    static const char* kPrefix = "model.layers.";
    const size_t np = std::strlen(kPrefix);
    if (name.compare(0, np, kPrefix) != 0) return -1;
    size_t i = np;
    if (i >= name.size() || !std::isdigit(static_cast<unsigned char>(name[i]))) return -1;
    long layer = 0;
    while (i < name.size() && std::isdigit(static_cast<unsigned char>(name[i]))) {
        layer = layer * 10 + (name[i] - '0');
        if (layer > (1 << 20)) return -1;
        ++i;
    }
    if (i >= name.size() || name[i] != '.' || layer >= num_layers) return -1;
    static const char* kSub[9] = {"input_layernorm.weight",          "self_attn.q_proj.weight",
                                  "self_attn.k_proj.weight",         "self_attn.v_proj.weight",
                                  "self_attn.o_proj.weight",         "post_attention_layernorm.weight",
                                  "mlp.gate_proj.weight",            "mlp.up_proj.weight",
                                  "mlp.down_proj.weight"};
    const std::string sub = name.substr(i + 1);
    for (int k = 0; k < 9; ++k)
        if (sub == kSub[k]) return 3 + 9 * static_cast<int>(layer) + k;
    return -1;
}

// Element count and storage dtype of each slot for a configuration.
struct SlotSpec {
    int64_t elements;
    bool projection;  // stored in weight_dtype (else FP32)
};

SlotSpec slot_spec(const ModelConfig& c, int slot) {
    const int64_t H = c.hidden_size, V = c.vocab_size, I = c.intermediate_size;
    const int64_t qs = (int64_t)c.num_attention_heads * c.head_dim, kvs = (int64_t)c.num_key_value_heads * c.head_dim;
    if (slot == 0) return {V * H, false};
    if (slot == 1) return {H, false};
    if (slot == 2) return {V * H, true};
    switch ((slot - 3) % 9) {
        case 0: return {H, false};
        case 1: return {qs * H, true};
        case 2: return {kvs * H, true};
        case 3: return {kvs * H, true};
        case 4: return {H * qs, true};
        case 5: return {H, false};
        case 6: return {I * H, true};
        case 7: return {I * H, true};
        default: return {H * I, true};
    }
}

const char* slot_name(int slot) {
    static const char* kTop[3] = {"model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"};
    static const char* kLayer[9] = {"input_layernorm", "q_proj", "k_proj", "v_proj", "o_proj",
                                    "post_attention_layernorm", "gate_proj", "up_proj", "down_proj"};
    return slot < 3 ? kTop[slot] : kLayer[(slot - 3) % 9];
}

// Reads model.bin and hands every recognised tensor to sink(slot, shape,
// payload) (FP32 values; the sink may take the vector's contents).
void scan_model_bin(const std::string& path, const ModelConfig& c,
                    const std::function<void(int, const std::vector<int>&, std::vector<float>&)>& sink) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Failed to open weights file: " + path);
    auto read = [&](void* dst, size_t n, const char* what) {
        f.read(static_cast<char*>(dst), static_cast<std::streamsize>(n));
        if (static_cast<size_t>(f.gcount()) != n)
            throw std::runtime_error(std::string("model.bin truncated while reading ") + what);
    };
    uint32_t head[3];
    read(head, sizeof(head), "the header");
    if (head[0] != kMagic) throw std::runtime_error("Invalid model binary magic number");
    if (head[1] != kVersion) throw std::runtime_error("Unsupported model binary version");
    std::vector<float> payload;
    for (uint32_t t = 0; t < head[2]; ++t) {
        int32_t name_len = 0;
        read(&name_len, 4, "a name length");
        if (name_len < 0 || name_len > 4096) throw std::runtime_error("model.bin: name length out of range");
        std::string name(static_cast<size_t>(name_len), '\0');
        read(&name[0], static_cast<size_t>(name_len), "a tensor name");
        int32_t ndim = 0;
        read(&ndim, 4, "a dimension count");
        if (ndim < 0 || ndim > 8) throw std::runtime_error("model.bin: " + name + " has " + std::to_string(ndim) + " dims");
        std::vector<int> shape(static_cast<size_t>(ndim));
        int64_t prod = 1;
        for (int d = 0; d < ndim; ++d) {
            int32_t v = 0;
            read(&v, 4, "a dimension");
            if (v < 0) throw std::runtime_error("model.bin: " + name + " has a negative dimension");
            shape[static_cast<size_t>(d)] = v;
            prod *= v;
        }
        int64_t n = 0;
        read(&n, 8, "an element count");
        if (n < 0 || n != prod)
            throw std::runtime_error("model.bin: " + name + " holds " + std::to_string(n) + " elements, its dims " +
                                     std::to_string(prod));
        const int slot = slot_of(name, c.num_layers);
        if (slot < 0) {
            f.seekg(n * 4, std::ios::cur);  // not a tensor of this model
            if (!f) throw std::runtime_error("model.bin truncated in " + name);
            continue;
        }
        const SlotSpec spec = slot_spec(c, slot);
        if (n != spec.elements)
            throw std::runtime_error("model.bin: " + name + " holds " + std::to_string(n) + " elements, the config " +
                                     std::to_string(spec.elements));
        payload.resize(static_cast<size_t>(n));
        read(payload.data(), static_cast<size_t>(n) * 4, name.c_str());
        sink(slot, shape, payload);
    }
}

std::vector<uint16_t> to_bf16(const std::vector<float>& v) {
    std::vector<uint16_t> out(v.size());
    for (size_t i = 0; i < v.size(); ++i) {
        const float r = infernt_round_bf16(v[i]);
        uint32_t u;
        std::memcpy(&u, &r, 4);
        out[i] = static_cast<uint16_t>(u >> 16);
    }
    return out;
}

}  // namespace

ModelConfig CheckpointLoader::load_config(const std::string& config_path) { return config_from_json(config_path); }

void CheckpointLoader::load_weights(const std::string& weights_path, const ModelConfig& config, ModelWeights& weights,
                                    Device target_device) {
    const int L = config.num_layers, nslots = 3 + 9 * L;
    std::vector<Tensor> slots(static_cast<size_t>(nslots));
    std::vector<bool> seen(static_cast<size_t>(nslots), false);
    const bool bf16 = config.weight_dtype == DType::BF16;
    auto place = [&](int slot, const std::vector<int>& shape, const std::vector<float>& v) {
        const bool as_bf16 = bf16 && slot_spec(config, slot).projection;
        Tensor host(shape, as_bf16 ? DType::BF16 : DType::FP32, Device::CPU);
        if (as_bf16) {
            const std::vector<uint16_t> b = to_bf16(v);
            std::memcpy(host.data_ptr(), b.data(), b.size() * 2);
        } else {
            std::memcpy(host.data_ptr(), v.data(), v.size() * 4);
        }
        slots[static_cast<size_t>(slot)] = target_device == Device::CUDA ? host.to(Device::CUDA) : std::move(host);
        seen[static_cast<size_t>(slot)] = true;
    };
    std::vector<float> embedding_copy;
    std::vector<int> embedding_shape;
    scan_model_bin(weights_path, config, [&](int slot, const std::vector<int>& shape, std::vector<float>& v) {
        if (slot == 0) {
            embedding_copy = v;  // the lm_head stand-in if the file has none
            embedding_shape = shape;
        }
        place(slot, shape, v);
    });
    if (!seen[2] && seen[0]) place(2, embedding_shape, embedding_copy);
    // a tensor the file does not hold stays empty (is_valid() false), as in
    // the reference's loader; the engine's C entry point requires them all
    weights.embedding = std::move(slots[0]);
    weights.final_norm = std::move(slots[1]);
    weights.lm_head = std::move(slots[2]);
    weights.layers.clear();
    weights.layers.resize(static_cast<size_t>(L));
    for (int l = 0; l < L; ++l) {
        TransformerLayerWeights& w = weights.layers[static_cast<size_t>(l)];
        Tensor* s = &slots[static_cast<size_t>(3 + 9 * l)];
        w.attn_norm = std::move(s[0]);
        w.q_proj = std::move(s[1]);
        w.k_proj = std::move(s[2]);
        w.v_proj = std::move(s[3]);
        w.o_proj = std::move(s[4]);
        w.ffn_norm = std::move(s[5]);
        w.gate_proj = std::move(s[6]);
        w.up_proj = std::move(s[7]);
        w.down_proj = std::move(s[8]);
    }
}

// ---------------------------------------------------------------- C ABI

struct infernt_checkpoint {
    bool on_device = false;
    std::vector<void*> ptrs;
    ~infernt_checkpoint() {
        for (void* p : ptrs) {
            if (on_device)
                cudaFree(p);
            else
                std::free(p);
        }
    }
};

namespace {

ModelConfig to_model_config(const infernt_llama_config& c) {
    ModelConfig m;
    m.architecture = "LlamaForCausalLM";
    m.vocab_size = c.vocab_size;
    m.hidden_size = c.hidden_size;
    m.num_layers = c.num_layers;
    m.num_attention_heads = c.num_attention_heads;
    m.num_key_value_heads = c.num_key_value_heads;
    m.intermediate_size = c.intermediate_size;
    m.max_seq_len = c.max_seq_len;
    m.head_dim = c.head_dim;
    m.rms_norm_eps = c.rms_norm_eps;
    m.rope_theta = c.rope_theta;
    m.weight_dtype = c.weight_dtype == INFERNT_DTYPE_BF16 ? DType::BF16 : DType::FP32;
    m.derive_computed_fields();
    return m;
}

}  // namespace

extern "C" {

int infernt_checkpoint_read_config(const char* config_json, infernt_llama_config* out) {
    INFERNT_REQUIRE(config_json && out, "checkpoint_read_config: null argument");
    try {
        const ModelConfig c = config_from_json(config_json);
        out->vocab_size = c.vocab_size;
        out->hidden_size = c.hidden_size;
        out->num_layers = c.num_layers;
        out->num_attention_heads = c.num_attention_heads;
        out->num_key_value_heads = c.num_key_value_heads;
        out->intermediate_size = c.intermediate_size;
        out->max_seq_len = c.max_seq_len;
        out->head_dim = c.head_dim;
        out->rms_norm_eps = c.rms_norm_eps;
        out->rope_theta = c.rope_theta;
        out->weight_dtype = c.weight_dtype == DType::BF16 ? INFERNT_DTYPE_BF16 : INFERNT_DTYPE_F32;
    } catch (const std::exception& ex) {
        return infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "%s", ex.what());
    }
    return INFERNT_OK;
}

int infernt_checkpoint_load(const char* model_bin, const infernt_llama_config* cfg, int device,
                            infernt_checkpoint** out) {
    INFERNT_REQUIRE(model_bin && cfg && out, "checkpoint_load: null argument");
    INFERNT_REQUIRE(device == 0 || device == 1, "checkpoint_load: device %d (0 host, 1 CUDA)", device);
    INFERNT_REQUIRE(cfg->num_layers >= 1 && cfg->num_layers <= 4096, "checkpoint_load: %d layers", cfg->num_layers);
    *out = nullptr;
    infernt_checkpoint* ck = new (std::nothrow) infernt_checkpoint();
    INFERNT_REQUIRE(ck, "checkpoint_load: host allocation failed");
    ck->on_device = device == 1;
    int status = INFERNT_OK;
    try {
        const ModelConfig c = to_model_config(*cfg);
        c.validate();
        const int nslots = 3 + 9 * c.num_layers;
        ck->ptrs.assign(static_cast<size_t>(nslots), nullptr);
        const bool bf16 = c.weight_dtype == DType::BF16;
        auto place = [&](int slot, const std::vector<float>& v) {
            const bool as_bf16 = bf16 && slot_spec(c, slot).projection;
            std::vector<uint16_t> b;
            const void* src = v.data();
            size_t bytes = v.size() * 4;
            if (as_bf16) {
                b = to_bf16(v);
                src = b.data();
                bytes = b.size() * 2;
            }
            void*& dst = ck->ptrs[static_cast<size_t>(slot)];
            if (dst) throw std::runtime_error(std::string("model.bin: ") + slot_name(slot) + " appears twice");
            if (ck->on_device) {
                cudaError_t e = cudaMalloc(&dst, bytes);
                if (e == cudaSuccess) e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
                if (e != cudaSuccess) throw std::runtime_error(std::string("checkpoint upload: ") + cudaGetErrorString(e));
            } else {
                dst = std::malloc(bytes);
                if (!dst) throw std::runtime_error("checkpoint: host allocation failed");
                std::memcpy(dst, src, bytes);
            }
        };
        std::vector<float> embedding_copy;
        scan_model_bin(model_bin, c, [&](int slot, const std::vector<int>&, std::vector<float>& v) {
            if (slot == 0) embedding_copy = v;
            place(slot, v);
        });
        if (!ck->ptrs[2] && ck->ptrs[0]) place(2, embedding_copy);
        for (int s = 0; s < nslots; ++s)
            if (!ck->ptrs[static_cast<size_t>(s)])
                throw std::runtime_error(std::string("model.bin: missing ") + slot_name(s) +
                                         (s >= 3 ? " of layer " + std::to_string((s - 3) / 9) : std::string()));
    } catch (const std::exception& ex) {
        status = infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "%s", ex.what());
    }
    if (status) {
        delete ck;
        return status;
    }
    *out = ck;
    return INFERNT_OK;
}

int infernt_checkpoint_weights(const infernt_checkpoint* ck, const void** out, int n) {
    INFERNT_REQUIRE(ck && out, "checkpoint_weights: null argument");
    INFERNT_REQUIRE(n == static_cast<int>(ck->ptrs.size()), "checkpoint_weights: %d pointers, the checkpoint has %d", n,
                    static_cast<int>(ck->ptrs.size()));
    for (int i = 0; i < n; ++i) out[i] = ck->ptrs[static_cast<size_t>(i)];
    return INFERNT_OK;
}

int infernt_checkpoint_free(infernt_checkpoint* ck) {
    delete ck;
    return INFERNT_OK;
}

}  // extern "C"
