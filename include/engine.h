// engine.h — the inference engine of the reference's include/engine.h:1-66:
// owns weights, KV cache and the architecture; all buffers are allocated in
// initialize() (zero-allocation decode loop).  forward_token() is one launch
// of the persistent decode kernel (embedding, every layer, final norm, LM
// head and argmax; a CUDA graph of fused kernels for shapes that kernel does
// not take) plus a 4-byte device-to-host copy of the next token.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "architecture.h"
#include "config.h"
#include "cublas_wrapper.h"
#include "kv_cache.h"
#include "tokenizer.h"
#include "weights.h"

struct GenerationConfig {
    int max_new_tokens = 64;
    float temperature = 0.0f;
    int top_k = 1;
    bool stream_stdout = true;
};

struct GenerationStats {
    int prompt_tokens = 0;
    int generated_tokens = 0;
    double prefill_ms = 0.0;
    double decode_ms = 0.0;
    double total_ms = 0.0;
    double tokens_per_second = 0.0;
};

class InferenceEngine {
public:
    InferenceEngine();
    ~InferenceEngine();

    // A converted checkpoint directory (config.json, model.bin in INFT v1,
    // tokenizer.bin), as the reference's src/engine.cpp:14-31; the weights
    // go through CheckpointLoader (include/checkpoint_loader.h).
    void load_model(const std::string& model_dir);
    void load_model(const ModelConfig& config, const std::string& weights_path,
                    const std::string& tokenizer_path);

    void initialize(const ModelConfig& config, ModelWeights weights, Tokenizer tokenizer);

    std::string generate(const std::string& prompt, const GenerationConfig& gen_config = GenerationConfig(),
                         GenerationStats* stats = nullptr);
    // The same loop over token IDs (no tokenizer); returns the generated IDs.
    std::vector<int> generate_tokens(const std::vector<int>& prompt_tokens,
                                     const GenerationConfig& gen_config = GenerationConfig(),
                                     GenerationStats* stats = nullptr);

    // One decode step at `position`: returns the next token, greedy, or
    // drawn at the step temperature (set_step_temperature) inside the step.
    int forward_token(int token_id, int position);
    // temperature <= 0: the greedy token of the last step.  temperature > 0:
    // a draw from softmax(logits / temperature) — on the GPU by Gumbel-max
    // (the default): the token the step itself drew when the temperature
    // equals the step temperature (no further kernel), else one sampling
    // kernel over the step's logits; with set_device_sampling(false), the
    // reference's host sampler (src/engine.cpp:78-104: softmax on the host, a
    // draw from a static mt19937(1337)).  GPU draws are keyed by (seed, the
    // step's position, the draw's count since the step), so every call draws
    // afresh and runs are reproducible; they follow the distribution of the
    // reference's draws, not its mt19937 sequence.
    int sample_next_token(float temperature = 0.0f);
    // Not in the reference: `on` (the default) samples on the GPU as above,
    // off restores the reference's host sampler.
    void set_device_sampling(bool on, uint64_t seed = 1337);
    // Not in the reference: the temperature at which forward_token draws the
    // next token inside the decode kernel's LM-head phase (0: greedy, the
    // default).  Needs the persistent decode kernel and device sampling;
    // otherwise the step stays greedy and sample_next_token samples after it.
    // generate() sets it to its temperature for the generation.
    void set_step_temperature(float temperature);

    // `steps` greedy steps chained on the device from (token_id, position);
    // writes the produced tokens to tokens_out and returns the device time in ms.
    float decode_chain(int token_id, int position, int steps, std::vector<int>* tokens_out);
    // Zero the KV cache.
    void reset();

    const ModelConfig& config() const;
    const Tokenizer& tokenizer() const;
    bool is_loaded() const;

    ModelWeights& weights();
    KVCache& kv_cache();
    const Tensor& logits() const;
    LlamaArchitecture& architecture();

private:
    ModelConfig config_;
    ModelWeights weights_;
    Tokenizer tokenizer_;
    std::unique_ptr<CublasWrapper> cublas_;
    std::unique_ptr<LlamaArchitecture> architecture_;
    KVCache kv_cache_;

    Tensor logits_;
    Tensor tokens_dev_;
    int last_token_;
    bool is_loaded_;
    bool device_sampling_ = true;
    uint64_t sample_seed_ = 1337;
    float step_temperature_ = 0.0f;  // temperature the last steps drew at inside the kernel (0: greedy)
    int last_position_ = 0;
    uint64_t draws_at_position_ = 0;  // GPU draws sample_next_token made since the last step
    Tensor sample_ws_, sample_out_;
};
