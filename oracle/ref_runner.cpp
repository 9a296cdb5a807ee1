// ref_runner.cpp — drives the UNMODIFIED INFERNT sources (compiled from the
// reference checkout by oracle/Makefile into oracle/_ref/libinfernt_ref.so)
// through the reference's own public C++ API.  TEST/BENCH INFRASTRUCTURE:
// it is the reference arm of the benchmark and the source of the
// reference-generated golden logits; the product never links it.
//
// Two handles:
//   * "arch" handle  — ModelWeights + CublasWrapper + LlamaArchitecture +
//     KVCache, driven as the reference's own tests drive it
//     (src/main.cpp:479-531): returns logits of LlamaArchitecture::forward.
//   * "engine" handle — InferenceEngine::initialize + forward_token +
//     sample_next_token (src/engine.cpp:33-105): the decode loop of
//     InferenceEngine::generate (src/engine.cpp:135-154) without the
//     tokenizer and stdout work.
//
// Weights are the seeded synthetic weights of include/infernt_seed.h,
// generated on the host and uploaded with Tensor::to (as the reference's
// checkpoint loader does, loader/checkpoint_loader.cpp:112-114).
#include "architecture.h"
#include "checkpoint_loader.h"
#include "config.h"
#include "cublas_wrapper.h"
#include "cuda_utils.h"
#include "engine.h"
#include "kernels.h"
#include "kv_cache.h"
#include "tensor.h"
#include "tokenizer.h"
#include "weights.h"

#include "../include/infernt_seed.h"

#include <cuda_runtime.h>
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

struct RefArch {
    ModelConfig cfg;
    ModelWeights weights;
    std::unique_ptr<CublasWrapper> cublas;
    std::unique_ptr<LlamaArchitecture> arch;
    KVCache kv;
    Tensor input;
    Tensor logits;
    Tensor token;
};

struct RefEngine {
    ModelConfig cfg;
    InferenceEngine engine;
};

ModelConfig make_config(const int* ci, const float* cf) {
    ModelConfig c;
    c.architecture = "LlamaForCausalLM";
    c.vocab_size = ci[0];
    c.hidden_size = ci[1];
    c.num_layers = ci[2];
    c.num_attention_heads = ci[3];
    c.num_key_value_heads = ci[4];
    c.intermediate_size = ci[5];
    c.max_seq_len = ci[6];
    c.head_dim = ci[7];
    c.rms_norm_eps = cf[0];
    c.rope_theta = cf[1];
    c.derive_computed_fields();
    c.validate();
    return c;
}

void fill_normal_host(float* out, size_t n, uint64_t seed, uint64_t stream, float std_dev,
                      int round_bf16) {
    uint64_t key = infernt_stream_key(seed, stream);
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (n < (1u << 16)) nt = 1;
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t) {
        size_t b = n * t / nt, e = n * (t + 1) / nt;
        th.emplace_back([=] {
            for (size_t i = b; i < e; ++i) {
                float v = infernt_normal_std(key, i, std_dev);
                out[i] = round_bf16 ? infernt_round_bf16(v) : v;
            }
        });
    }
    for (auto& t : th) t.join();
}

Tensor seeded(const std::vector<int>& shape, uint64_t seed, uint64_t stream, float std_dev,
              int round_bf16) {
    Tensor cpu = Tensor::zeros(shape, DType::FP32, Device::CPU);
    fill_normal_host(cpu.data_as_float(), (size_t)cpu.num_elements(), seed, stream, std_dev,
                     round_bf16);
    return cpu.to(Device::CUDA);
}

Tensor ones(const std::vector<int>& shape) {
    Tensor cpu = Tensor::zeros(shape, DType::FP32, Device::CPU);
    float* p = cpu.data_as_float();
    for (int64_t i = 0; i < cpu.num_elements(); ++i) p[i] = 1.0f;
    return cpu.to(Device::CUDA);
}

ModelWeights make_weights(const ModelConfig& c, uint64_t seed, float std_dev, int round_bf16) {
    ModelWeights w;
    int qs = c.num_attention_heads * c.head_dim;
    int ks = c.num_key_value_heads * c.head_dim;
    // the embedding stays FP32 under round_bf16 (the bf16-weight variant
    // rounds the projections and the LM head only, as the engine stores them)
    w.embedding = seeded({c.vocab_size, c.hidden_size}, seed, INFERNT_STREAM_EMBEDDING, std_dev, 0);
    w.final_norm = ones({c.hidden_size});
    w.lm_head = seeded({c.vocab_size, c.hidden_size}, seed, INFERNT_STREAM_LM_HEAD, std_dev,
                       round_bf16);
    for (int l = 0; l < c.num_layers; ++l) {
        TransformerLayerWeights lw;
        lw.attn_norm = ones({c.hidden_size});
        lw.q_proj = seeded({qs, c.hidden_size}, seed, INFERNT_STREAM_LAYER(l, 0), std_dev, round_bf16);
        lw.k_proj = seeded({ks, c.hidden_size}, seed, INFERNT_STREAM_LAYER(l, 1), std_dev, round_bf16);
        lw.v_proj = seeded({ks, c.hidden_size}, seed, INFERNT_STREAM_LAYER(l, 2), std_dev, round_bf16);
        lw.o_proj = seeded({c.hidden_size, qs}, seed, INFERNT_STREAM_LAYER(l, 3), std_dev, round_bf16);
        lw.ffn_norm = ones({c.hidden_size});
        lw.gate_proj = seeded({c.intermediate_size, c.hidden_size}, seed, INFERNT_STREAM_LAYER(l, 4),
                              std_dev, round_bf16);
        lw.up_proj = seeded({c.intermediate_size, c.hidden_size}, seed, INFERNT_STREAM_LAYER(l, 5),
                            std_dev, round_bf16);
        lw.down_proj = seeded({c.hidden_size, c.intermediate_size}, seed, INFERNT_STREAM_LAYER(l, 6),
                              std_dev, round_bf16);
        w.layers.push_back(std::move(lw));
    }
    return w;
}

thread_local char g_err[512];

void set_err(const char* m) { std::snprintf(g_err, sizeof(g_err), "%s", m); }

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err; }

// ---------------------------------------------------------------- arch ---
void* ref_arch_create(const int* ci, const float* cf, unsigned long long seed, float std_dev,
                      int round_bf16) {
    try {
        auto* r = new RefArch();
        r->cfg = make_config(ci, cf);
        r->weights = make_weights(r->cfg, seed, std_dev, round_bf16);
        r->cublas = std::make_unique<CublasWrapper>();
        r->arch = std::make_unique<LlamaArchitecture>(*r->cublas);
        r->arch->allocate_activations(r->cfg, 1);
        r->kv.allocate(r->cfg);
        r->kv.reset();
        r->input = Tensor::zeros({1, r->cfg.hidden_size}, DType::FP32, Device::CUDA);
        r->logits = Tensor::zeros({1, r->cfg.vocab_size}, DType::FP32, Device::CUDA);
        r->token = Tensor::zeros({1}, DType::FP32, Device::CUDA);
        return r;
    } catch (const std::exception& e) {
        set_err(e.what());
        return nullptr;
    }
}

void ref_arch_destroy(void* h) { delete static_cast<RefArch*>(h); }

int ref_arch_reset(void* h) {
    static_cast<RefArch*>(h)->kv.reset();
    return 0;
}

// One token at `position` through launch_embedding_lookup +
// LlamaArchitecture::forward + launch_argmax; copies logits to the host.
int ref_arch_decode(void* h, int token, int position, float* logits_host) {
    auto* r = static_cast<RefArch*>(h);
    try {
        launch_embedding_lookup(r->input.data_as_float(), r->weights.embedding.data_as_float(),
                                token, r->cfg.hidden_size);
        r->arch->forward(r->input, r->weights, r->kv, position, r->logits);
        launch_argmax(reinterpret_cast<int*>(r->token.data_as_float()), r->logits.data_as_float(),
                      r->cfg.vocab_size);
        if (cudaDeviceSynchronize() != cudaSuccess) return -1;
        int tok = 0;
        cudaMemcpy(&tok, r->token.data_as_float(), sizeof(int), cudaMemcpyDeviceToHost);
        if (logits_host)
            cudaMemcpy(logits_host, r->logits.data_as_float(), sizeof(float) * r->cfg.vocab_size,
                       cudaMemcpyDeviceToHost);
        return tok;
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1;
    }
}

// Fill every layer's K and V cache rows [0, n_pos) with seeded N(0, std).
int ref_arch_prefill_kv(void* h, unsigned long long seed, int n_pos, float std_dev) {
    auto* r = static_cast<RefArch*>(h);
    const ModelConfig& c = r->cfg;
    size_t per = (size_t)c.num_key_value_heads * c.max_seq_len * c.head_dim;
    std::vector<float> buf(per);
    // element (layer l, head hh, position p, dim d) is element
    // ((l * Nkv + hh) * 2^20 + p) * D + d of the K (or V) stream, so the
    // values do not depend on max_seq_len.
    for (int l = 0; l < c.num_layers; ++l) {
        for (int which = 0; which < 2; ++which) {
            uint64_t key = infernt_stream_key(seed, which == 0 ? INFERNT_STREAM_KV_K : INFERNT_STREAM_KV_V);
            for (int hh = 0; hh < c.num_key_value_heads; ++hh)
                for (int p = 0; p < c.max_seq_len; ++p)
                    for (int d = 0; d < c.head_dim; ++d) {
                        size_t i = ((size_t)hh * c.max_seq_len + p) * c.head_dim + d;
                        uint64_t gi = ((((uint64_t)l * c.num_key_value_heads + hh) << 20) + p) *
                                          (uint64_t)c.head_dim + d;
                        buf[i] = p < n_pos ? infernt_normal_std(key, gi, std_dev) : 0.0f;
                    }
            Tensor& t = which == 0 ? r->kv.k_cache[l] : r->kv.v_cache[l];
            cudaMemcpy(t.data_ptr(), buf.data(), sizeof(float) * per, cudaMemcpyHostToDevice);
        }
    }
    return 0;
}

// -------------------------------------------------------------- engine ---
void* ref_engine_create(const int* ci, const float* cf, unsigned long long seed, float std_dev) {
    try {
        auto* r = new RefEngine();
        r->cfg = make_config(ci, cf);
        r->engine.initialize(r->cfg, make_weights(r->cfg, seed, std_dev, 0), Tokenizer());
        return r;
    } catch (const std::exception& e) {
        set_err(e.what());
        return nullptr;
    }
}

void ref_engine_destroy(void* h) { delete static_cast<RefEngine*>(h); }

int ref_engine_forward_token(void* h, int token, int position) {
    try {
        return static_cast<RefEngine*>(h)->engine.forward_token(token, position);
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1;
    }
}

int ref_engine_sample_next_token(void* h) {
    try {
        return static_cast<RefEngine*>(h)->engine.sample_next_token(0.0f);
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1;
    }
}

// The decode loop of InferenceEngine::generate (src/engine.cpp:135-154) for
// `steps` tokens starting at (token, position): forward_token then
// sample_next_token each step, exactly as generate() calls them.  Device
// time of the whole loop from CUDA events on the legacy default stream (the
// stream every reference launch uses), in milliseconds.
float ref_engine_decode_loop(void* h, int token, int position, int steps, int* tokens_out) {
    auto* r = static_cast<RefEngine*>(h);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaDeviceSynchronize();
    cudaEventRecord(a, 0);
    int next = token;
    try {
        for (int s = 0; s < steps; ++s) {
            r->engine.forward_token(next, position + s);
            next = r->engine.sample_next_token(0.0f);
            if (tokens_out) tokens_out[s] = next;
        }
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1.0f;
    }
    cudaEventRecord(b, 0);
    cudaEventSynchronize(b);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return ms;
}

// The reference's CheckpointLoader on the host (Device::CPU): config.json
// into ci [vocab, hidden, layers, q heads, kv heads, intermediate, max_seq,
// head_dim] and cf [eps, theta]; model.bin into out[slot] (3 + 9 layers
// caller arrays of FP32, the order of ModelWeights: embedding, final_norm,
// lm_head, per layer attn_norm, q, k, v, o, ffn_norm, gate, up, down), each
// of out_n[slot] floats.  Returns 0, or -1 with ref_last_error() set when
// the reference throws.
int ref_checkpoint_load_cpu(const char* config_json, const char* model_bin, int* ci, float* cf, int n_slots,
                            float* const* out, const long long* out_n) {
    try {
        ModelConfig c = CheckpointLoader::load_config(config_json);
        ci[0] = c.vocab_size;
        ci[1] = c.hidden_size;
        ci[2] = c.num_layers;
        ci[3] = c.num_attention_heads;
        ci[4] = c.num_key_value_heads;
        ci[5] = c.intermediate_size;
        ci[6] = c.max_seq_len;
        ci[7] = c.head_dim;
        cf[0] = c.rms_norm_eps;
        cf[1] = c.rope_theta;
        if (!model_bin) return 0;
        ModelWeights w;
        CheckpointLoader::load_weights(model_bin, c, w, Device::CPU);
        std::vector<const Tensor*> ts = {&w.embedding, &w.final_norm, &w.lm_head};
        for (const auto& l : w.layers)
            for (const Tensor* x : {&l.attn_norm, &l.q_proj, &l.k_proj, &l.v_proj, &l.o_proj, &l.ffn_norm,
                                    &l.gate_proj, &l.up_proj, &l.down_proj})
                ts.push_back(x);
        if ((int)ts.size() != n_slots) throw std::runtime_error("slot count mismatch");
        for (int s = 0; s < n_slots; ++s) {
            if (!ts[s]->is_valid() || ts[s]->num_elements() != out_n[s])
                throw std::runtime_error("tensor " + std::to_string(s) + " missing or of another size");
            std::memcpy(out[s], ts[s]->data_as_float(), sizeof(float) * (size_t)out_n[s]);
        }
        return 0;
    } catch (const std::exception& e) {
        set_err(e.what());
        return -1;
    }
}

}  // extern "C"
