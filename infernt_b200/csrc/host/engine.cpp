// engine.cpp — InferenceEngine (include/engine.h) over LlamaArchitecture.
// Decode loop semantics follow src/engine.cpp:107-169 of the reference:
// token-by-token prefill, greedy or temperature sampling, EOS / max_seq
// stop, wall-clock GenerationStats.
#include "engine.h"
#include "checkpoint_loader.h"
#include "infernt_capi.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <iostream>
#include <random>
#include <stdexcept>

InferenceEngine::InferenceEngine() : last_token_(0), is_loaded_(false) {}
InferenceEngine::~InferenceEngine() = default;

// A converted checkpoint directory (src/engine.cpp:14-31): config.json,
// model.bin (INFT v1, host/checkpoint.cpp) and tokenizer.bin.
void InferenceEngine::load_model(const std::string& model_dir) {
    load_model(CheckpointLoader::load_config(model_dir + "/config.json"), model_dir + "/model.bin",
               model_dir + "/tokenizer.bin");
}

void InferenceEngine::load_model(const ModelConfig& config, const std::string& weights_path,
                                 const std::string& tokenizer_path) {
    Tokenizer tok;
    if (!tok.load(tokenizer_path)) throw std::runtime_error("Failed to load tokenizer from: " + tokenizer_path);
    ModelWeights w;
    CheckpointLoader::load_weights(weights_path, config, w, Device::CUDA);
    initialize(config, std::move(w), std::move(tok));
}

void InferenceEngine::set_step_temperature(float temperature) {
    if (!is_loaded_) throw std::runtime_error("Engine model is not loaded");
    infernt_plan* plan = architecture_->plan_for(weights_, kv_cache_);
    const float t = (device_sampling_ && temperature > 0.0f) ? temperature : 0.0f;
    if (t > 0.0f && infernt_plan_set_sampling(plan, t, sample_seed_) == INFERNT_OK) {
        step_temperature_ = t;
        return;
    }
    if (infernt_plan_set_sampling(plan, 0.0f, sample_seed_) != INFERNT_OK)
        throw std::runtime_error(std::string("set_step_temperature: ") + infernt_last_error());
    step_temperature_ = 0.0f;
}

void InferenceEngine::set_device_sampling(bool on, uint64_t seed) {
    device_sampling_ = on;
    sample_seed_ = seed;
    if (is_loaded_ && step_temperature_ > 0.0f) set_step_temperature(on ? step_temperature_ : 0.0f);
}

void InferenceEngine::initialize(const ModelConfig& config, ModelWeights weights, Tokenizer tokenizer) {
    config.validate();
    config_ = config;
    weights_ = std::move(weights);
    tokenizer_ = std::move(tokenizer);
    cublas_ = std::make_unique<CublasWrapper>();
    architecture_ = std::make_unique<LlamaArchitecture>(*cublas_);
    architecture_->allocate_activations(config_, 1);
    kv_cache_.allocate(config_);
    logits_ = Tensor::zeros({1, config_.vocab_size}, DType::FP32, Device::CUDA);
    tokens_dev_ = Tensor::zeros({config_.max_seq_len}, DType::INT32, Device::CUDA);
    is_loaded_ = true;
}

int InferenceEngine::forward_token(int token_id, int position) {
    if (!is_loaded_) throw std::runtime_error("Engine model is not loaded");
    architecture_->forward_token(token_id, weights_, kv_cache_, position, logits_);
    last_token_ = architecture_->last_token();
    last_position_ = position;
    draws_at_position_ = 0;
    return last_token_;
}

int InferenceEngine::sample_next_token(float temperature) {
    if (!is_loaded_) throw std::runtime_error("Engine model is not loaded");
    // the token the step already chose: greedy, or its first draw at this
    // temperature (a further call at the same position draws afresh, as the
    // reference's sampler does)
    if (temperature <= 0.0f && step_temperature_ <= 0.0f) return last_token_;
    if (temperature > 0.0f && temperature == step_temperature_ && draws_at_position_ == 0) {
        draws_at_position_ = 1;
        return last_token_;
    }
    if (device_sampling_ || temperature <= 0.0f) {
        // one kernel over the step's logits (sample.cu; T <= 0 is its greedy
        // argmax): one int crosses to the host
        if (!sample_ws_.is_valid()) {
            const int bytes = (int)infernt_sample_workspace_bytes(1);
            sample_ws_ = Tensor::zeros({bytes}, DType::UINT8, Device::CUDA);
            sample_out_ = Tensor::zeros({1}, DType::INT32, Device::CUDA);
        }
        const int s = infernt_sample_tokens(static_cast<const float*>(logits_.data_ptr()), 0, 1, config_.vocab_size,
                                            temperature, sample_seed_,
                                            (uint64_t)(unsigned)last_position_ | ((uint64_t)draws_at_position_ << 32),
                                            static_cast<int*>(sample_out_.data_ptr()), sample_ws_.data_ptr(), nullptr);
        if (s) throw std::runtime_error(std::string("sample_next_token: ") + infernt_last_error());
        if (temperature > 0.0f) ++draws_at_position_;
        int tok = 0;
        if (cudaMemcpy(&tok, sample_out_.data_ptr(), sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
            throw std::runtime_error("sample_next_token: device-to-host copy failed");
        return tok;
    }
    Tensor cpu = logits_.to(Device::CPU);
    const float* l = cpu.data_as_float();
    float mx = -1e30f;
    for (int i = 0; i < config_.vocab_size; ++i)
        if (l[i] > mx) mx = l[i];
    std::vector<float> probs(config_.vocab_size);
    float sum = 0.0f;
    for (int i = 0; i < config_.vocab_size; ++i) {
        probs[i] = std::exp((l[i] - mx) / temperature);
        sum += probs[i];
    }
    static std::mt19937 gen(1337);
    std::uniform_real_distribution<float> dis(0.0f, sum);
    const float r = dis(gen);
    float cum = 0.0f;
    for (int i = 0; i < config_.vocab_size; ++i) {
        cum += probs[i];
        if (r <= cum) return i;
    }
    return config_.vocab_size - 1;
}

float InferenceEngine::decode_chain(int token_id, int position, int steps, std::vector<int>* tokens_out) {
    if (!is_loaded_) throw std::runtime_error("Engine model is not loaded");
    if (steps <= 0) return 0.0f;
    cudaStream_t st = architecture_->stream();
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, st);
    architecture_->decode_chain(token_id, position, steps, weights_, kv_cache_, static_cast<int*>(tokens_dev_.data_ptr()));
    cudaEventRecord(b, st);
    last_token_ = architecture_->last_token();
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (tokens_out) {
        tokens_out->resize(steps);
        if (cudaMemcpy(tokens_out->data(), tokens_dev_.data_ptr(), sizeof(int) * steps, cudaMemcpyDeviceToHost) !=
            cudaSuccess)
            throw std::runtime_error("decode_chain: token copy failed");
    }
    return ms;
}

void InferenceEngine::reset() { kv_cache_.reset(); }

std::vector<int> InferenceEngine::generate_tokens(const std::vector<int>& prompt, const GenerationConfig& gc,
                                                  GenerationStats* stats) {
    if (!is_loaded_) throw std::runtime_error("Engine model is not loaded");
    std::vector<int> tokens = prompt;
    if (tokens.empty()) tokens.push_back(tokenizer_.bos_id());
    // draw inside the decode kernel at the generation's temperature (restored
    // to greedy afterwards)
    set_step_temperature(gc.temperature);
    struct Restore {
        InferenceEngine* e;
        ~Restore() {
            try {
                e->set_step_temperature(0.0f);
            } catch (...) {
            }
        }
    } restore{this};
    auto t0 = std::chrono::high_resolution_clock::now();
    kv_cache_.reset();
    for (size_t pos = 0; pos < tokens.size(); ++pos) forward_token(tokens[pos], (int)pos);
    auto t1 = std::chrono::high_resolution_clock::now();
    int next = sample_next_token(gc.temperature);
    std::vector<int> out;
    for (int step = 0; step < gc.max_new_tokens; ++step) {
        if (next == tokenizer_.eos_id()) break;
        out.push_back(next);
        const int pos = (int)tokens.size() + step;
        if (pos >= config_.max_seq_len - 1) break;
        forward_token(next, pos);
        next = sample_next_token(gc.temperature);
    }
    auto t2 = std::chrono::high_resolution_clock::now();
    if (stats) {
        stats->prompt_tokens = (int)tokens.size();
        stats->generated_tokens = (int)out.size();
        stats->prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
        stats->decode_ms = std::chrono::duration<double, std::milli>(t2 - t1).count();
        stats->total_ms = std::chrono::duration<double, std::milli>(t2 - t0).count();
        stats->tokens_per_second =
            (!out.empty() && stats->decode_ms > 0) ? out.size() / (stats->decode_ms / 1000.0) : 0.0;
    }
    return out;
}

std::string InferenceEngine::generate(const std::string& prompt, const GenerationConfig& gc, GenerationStats* stats) {
    std::vector<int> out = generate_tokens(tokenizer_.encode(prompt, true, false), gc, stats);
    std::string text;
    for (int t : out) {
        std::string piece = tokenizer_.decode(t);
        text += piece;
        if (gc.stream_stdout) std::cout << piece << std::flush;
    }
    return text;
}

const ModelConfig& InferenceEngine::config() const { return config_; }
const Tokenizer& InferenceEngine::tokenizer() const { return tokenizer_; }
bool InferenceEngine::is_loaded() const { return is_loaded_; }
ModelWeights& InferenceEngine::weights() { return weights_; }
KVCache& InferenceEngine::kv_cache() { return kv_cache_; }
const Tensor& InferenceEngine::logits() const { return logits_; }
LlamaArchitecture& InferenceEngine::architecture() { return *architecture_; }
