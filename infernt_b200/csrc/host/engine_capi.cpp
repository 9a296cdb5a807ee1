// engine_capi.cpp — C entry points over the C++ InferenceEngine
// (infernt_engine_* in include/infernt_capi.h), for ctypes / cgo / JNI
// hosts.  The engine is built with seeded synthetic weights generated on
// the device (include/infernt_seed.h streams; norms 1.0).
#include "../../../include/checkpoint_loader.h"
#include <cuda_runtime.h>

#include <cstring>
#include <exception>
#include <new>
#include <stdexcept>
#include <string>

#include "../../../include/infernt_seed.h"
#include "../internal.h"
#include "engine.h"

struct infernt_engine {
    InferenceEngine engine;
};

namespace {

int guard(const std::exception& e) { return infernt::fail(INFERNT_ERR_CUDA, "%s", e.what()); }

Tensor seeded(const std::vector<int>& shape, DType dt, uint64_t seed, uint64_t stream, float std_dev) {
    Tensor t(shape, dt, Device::CUDA);
    int s = infernt_fill_normal(t.data_ptr(), (size_t)t.num_elements(),
                                dt == DType::BF16 ? INFERNT_DTYPE_BF16 : INFERNT_DTYPE_F32, seed, stream, std_dev,
                                nullptr);
    if (s) throw std::runtime_error(std::string("seeded fill: ") + infernt_last_error());
    return t;
}

Tensor ones(int n) {
    Tensor t({n}, DType::FP32, Device::CUDA);
    if (infernt_fill_const(t.data_as_float(), (size_t)n, 1.0f, nullptr))
        throw std::runtime_error(std::string("const fill: ") + infernt_last_error());
    return t;
}

}  // namespace

extern "C" {

int infernt_engine_create_seeded(const infernt_llama_config* c, uint64_t seed, float std_dev,
                                 infernt_engine** out) {
    INFERNT_REQUIRE(c && out, "engine_create_seeded: null argument");
    *out = nullptr;
    try {
        ModelConfig mc;
        mc.architecture = "LlamaForCausalLM";
        mc.vocab_size = c->vocab_size;
        mc.hidden_size = c->hidden_size;
        mc.num_layers = c->num_layers;
        mc.num_attention_heads = c->num_attention_heads;
        mc.num_key_value_heads = c->num_key_value_heads;
        mc.intermediate_size = c->intermediate_size;
        mc.max_seq_len = c->max_seq_len;
        mc.head_dim = c->head_dim;
        mc.rms_norm_eps = c->rms_norm_eps;
        mc.rope_theta = c->rope_theta;
        mc.weight_dtype = c->weight_dtype == INFERNT_DTYPE_BF16 ? DType::BF16 : DType::FP32;
        mc.derive_computed_fields();
        mc.validate();
        const DType wd = mc.weight_dtype;
        const int H = mc.hidden_size, I = mc.intermediate_size;
        const int qs = mc.num_attention_heads * mc.head_dim, ks = mc.num_key_value_heads * mc.head_dim;
        ModelWeights w;
        w.embedding = seeded({mc.vocab_size, H}, DType::FP32, seed, INFERNT_STREAM_EMBEDDING, std_dev);
        w.final_norm = ones(H);
        w.lm_head = seeded({mc.vocab_size, H}, wd, seed, INFERNT_STREAM_LM_HEAD, std_dev);
        for (int l = 0; l < mc.num_layers; ++l) {
            TransformerLayerWeights lw;
            lw.attn_norm = ones(H);
            lw.q_proj = seeded({qs, H}, wd, seed, INFERNT_STREAM_LAYER(l, 0), std_dev);
            lw.k_proj = seeded({ks, H}, wd, seed, INFERNT_STREAM_LAYER(l, 1), std_dev);
            lw.v_proj = seeded({ks, H}, wd, seed, INFERNT_STREAM_LAYER(l, 2), std_dev);
            lw.o_proj = seeded({H, qs}, wd, seed, INFERNT_STREAM_LAYER(l, 3), std_dev);
            lw.ffn_norm = ones(H);
            lw.gate_proj = seeded({I, H}, wd, seed, INFERNT_STREAM_LAYER(l, 4), std_dev);
            lw.up_proj = seeded({I, H}, wd, seed, INFERNT_STREAM_LAYER(l, 5), std_dev);
            lw.down_proj = seeded({H, I}, wd, seed, INFERNT_STREAM_LAYER(l, 6), std_dev);
            w.layers.push_back(std::move(lw));
        }
        if (cudaDeviceSynchronize() != cudaSuccess)
            return infernt::fail(INFERNT_ERR_CUDA, "engine_create_seeded: weight fill failed");
        auto* e = new infernt_engine();
        e->engine.initialize(mc, std::move(w), Tokenizer());
        *out = e;
        return INFERNT_OK;
    } catch (const std::bad_alloc&) {
        return infernt::fail(INFERNT_ERR_OUT_OF_MEMORY, "engine_create_seeded: host allocation failed");
    } catch (const std::exception& ex) {
        std::string m = ex.what();
        if (m.find("allocation failed") != std::string::npos)
            return infernt::fail(INFERNT_ERR_OUT_OF_MEMORY, "%s", m.c_str());
        return infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "%s", m.c_str());
    }
}

int infernt_engine_destroy(infernt_engine* e) {
    delete e;
    return INFERNT_OK;
}

int infernt_engine_set_mode(infernt_engine* e, int mode) {
    INFERNT_REQUIRE(e, "engine_set_mode: null engine");
    INFERNT_REQUIRE(mode >= INFERNT_MODE_EAGER && mode <= INFERNT_MODE_PERSISTENT, "engine_set_mode: mode %d", mode);
    e->engine.architecture().set_decode_mode(mode);
    return INFERNT_OK;
}

int infernt_engine_mode(infernt_engine* e, int* mode) {
    INFERNT_REQUIRE(e && mode, "engine_mode: null argument");
    *mode = e->engine.architecture().decode_mode();
    return INFERNT_OK;
}

int infernt_engine_trace_chain(infernt_engine* e, int token, int position, int steps, unsigned long long* host_out,
                               size_t n) {
    INFERNT_REQUIRE(e && host_out && steps > 0, "engine_trace_chain: bad arguments");
    try {
        infernt_plan* plan = e->engine.architecture().plan_for(e->engine.weights(), e->engine.kv_cache());
        const size_t need = infernt_plan_trace_entries(plan, steps);
        INFERNT_REQUIRE(need > 0, "engine_trace_chain: the plan does not run the persistent kernel");
        INFERNT_REQUIRE(n >= need, "engine_trace_chain: need %zu entries", need);
        unsigned long long* dev = nullptr;
        INFERNT_CUDA_TRY(cudaMalloc(&dev, need * sizeof(unsigned long long)));
        cudaMemset(dev, 0, need * sizeof(unsigned long long));
        int s = infernt_plan_set_trace(plan, dev);
        if (!s) e->engine.decode_chain(token, position, steps, nullptr);
        infernt_plan_set_trace(plan, nullptr);
        cudaError_t ce = cudaMemcpy(host_out, dev, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        cudaFree(dev);
        if (s) return s;
        INFERNT_CUDA_TRY(ce);
    } catch (const std::exception& ex) {
        return infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "%s", ex.what());
    }
    return INFERNT_OK;
}

int infernt_engine_reset(infernt_engine* e) {
    INFERNT_REQUIRE(e, "engine_reset: null engine");
    try {
        e->engine.reset();
    } catch (const std::exception& ex) {
        return guard(ex);
    }
    return INFERNT_OK;
}

int infernt_engine_forward_token(infernt_engine* e, int token, int position, int* next_token) {
    INFERNT_REQUIRE(e && next_token, "engine_forward_token: null argument");
    try {
        *next_token = e->engine.forward_token(token, position);
    } catch (const std::exception& ex) {
        return infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "%s", ex.what());
    }
    return INFERNT_OK;
}

int infernt_engine_load_model(const char* model_dir, int weight_dtype, infernt_engine** out) {
    INFERNT_REQUIRE(model_dir && out, "engine_load_model: null argument");
    INFERNT_REQUIRE(weight_dtype == INFERNT_DTYPE_F32 || weight_dtype == INFERNT_DTYPE_BF16 || weight_dtype < 0,
                    "engine_load_model: weight_dtype %d", weight_dtype);
    *out = nullptr;
    try {
        const std::string dir(model_dir);
        ModelConfig mc = CheckpointLoader::load_config(dir + "/config.json");
        if (weight_dtype >= 0) mc.weight_dtype = weight_dtype == INFERNT_DTYPE_BF16 ? DType::BF16 : DType::FP32;
        auto* e = new infernt_engine();
        try {
            e->engine.load_model(mc, dir + "/model.bin", dir + "/tokenizer.bin");
        } catch (...) {
            delete e;
            throw;
        }
        *out = e;
        return INFERNT_OK;
    } catch (const std::bad_alloc&) {
        return infernt::fail(INFERNT_ERR_OUT_OF_MEMORY, "engine_load_model: host allocation failed");
    } catch (const std::exception& ex) {
        return infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "engine_load_model: %s", ex.what());
    }
}

int infernt_engine_set_step_temperature(infernt_engine* e, float temperature) {
    INFERNT_REQUIRE(e, "engine_set_step_temperature: null engine");
    try {
        e->engine.set_step_temperature(temperature);
    } catch (const std::exception& ex) {
        return infernt::fail(INFERNT_ERR_CUDA, "engine_set_step_temperature: %s", ex.what());
    }
    return INFERNT_OK;
}

int infernt_engine_set_device_sampling(infernt_engine* e, int on, uint64_t seed) {
    INFERNT_REQUIRE(e, "engine_set_device_sampling: null engine");
    e->engine.set_device_sampling(on != 0, seed);
    return INFERNT_OK;
}

int infernt_engine_sample_next_token(infernt_engine* e, float temperature, int* token) {
    INFERNT_REQUIRE(e && token, "engine_sample_next_token: null argument");
    try {
        *token = e->engine.sample_next_token(temperature);
    } catch (const std::exception& ex) {
        return guard(ex);
    }
    return INFERNT_OK;
}

int infernt_engine_logits(infernt_engine* e, float* host) {
    INFERNT_REQUIRE(e && host, "engine_logits: null argument");
    const Tensor& l = e->engine.logits();
    INFERNT_CUDA_TRY(cudaMemcpy(host, l.data_ptr(), l.size_bytes(), cudaMemcpyDeviceToHost));
    return INFERNT_OK;
}

int infernt_engine_fill_kv(infernt_engine* e, uint64_t seed, int n_pos, float std_dev) {
    INFERNT_REQUIRE(e, "engine_fill_kv: null engine");
    const ModelConfig& c = e->engine.config();
    KVCache& kv = e->engine.kv_cache();
    std::vector<float*> k, v;
    for (int l = 0; l < c.num_layers; ++l) {
        k.push_back(kv.k_cache[l].data_as_float());
        v.push_back(kv.v_cache[l].data_as_float());
    }
    int s = infernt_fill_kv(k.data(), v.data(), c.num_layers, c.num_key_value_heads, c.max_seq_len, c.head_dim,
                            n_pos, seed, std_dev, nullptr);
    if (s) return s;
    INFERNT_CUDA_TRY(cudaDeviceSynchronize());
    return INFERNT_OK;
}

int infernt_engine_decode_chain(infernt_engine* e, int token, int position, int steps, int* tokens_host,
                                float* ms) {
    INFERNT_REQUIRE(e, "engine_decode_chain: null engine");
    try {
        std::vector<int> toks;
        const float t = e->engine.decode_chain(token, position, steps, tokens_host ? &toks : nullptr);
        if (tokens_host) std::memcpy(tokens_host, toks.data(), sizeof(int) * toks.size());
        if (ms) *ms = t;
    } catch (const std::exception& ex) {
        return infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, "%s", ex.what());
    }
    return INFERNT_OK;
}

int infernt_engine_weight_ptrs(infernt_engine* e, const void** ptrs, int n) {
    INFERNT_REQUIRE(e && ptrs, "engine_weight_ptrs: null argument");
    ModelWeights& w = e->engine.weights();
    const int need = 3 + 9 * (int)w.layers.size();
    INFERNT_REQUIRE(n >= need, "engine_weight_ptrs: need %d entries", need);
    int i = 0;
    ptrs[i++] = w.embedding.data_ptr();
    ptrs[i++] = w.final_norm.data_ptr();
    ptrs[i++] = w.lm_head.data_ptr();
    for (auto& lw : w.layers) {
        ptrs[i++] = lw.attn_norm.data_ptr();
        ptrs[i++] = lw.q_proj.data_ptr();
        ptrs[i++] = lw.k_proj.data_ptr();
        ptrs[i++] = lw.v_proj.data_ptr();
        ptrs[i++] = lw.o_proj.data_ptr();
        ptrs[i++] = lw.ffn_norm.data_ptr();
        ptrs[i++] = lw.gate_proj.data_ptr();
        ptrs[i++] = lw.up_proj.data_ptr();
        ptrs[i++] = lw.down_proj.data_ptr();
    }
    return INFERNT_OK;
}

int infernt_engine_kv_ptrs(infernt_engine* e, float** k, float** v, int n) {
    INFERNT_REQUIRE(e && k && v, "engine_kv_ptrs: null argument");
    KVCache& kv = e->engine.kv_cache();
    INFERNT_REQUIRE(n >= (int)kv.k_cache.size(), "engine_kv_ptrs: need %zu entries", kv.k_cache.size());
    for (size_t l = 0; l < kv.k_cache.size(); ++l) {
        k[l] = kv.k_cache[l].data_as_float();
        v[l] = kv.v_cache[l].data_as_float();
    }
    return INFERNT_OK;
}

}  // extern "C"
