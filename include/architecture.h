// architecture.h — the model-architecture interface of the reference's
// include/architecture.h:9-61.  LlamaArchitecture keeps its constructor
// and virtual methods; underneath, forward() runs the fused B200 decode step
// (infernt_plan_* in include/infernt_capi.h) on the stream of the
// CublasWrapper it was built with: one launch of the persistent decode
// kernel (a CUDA graph of fused kernels for shapes that kernel does not
// take).
#pragma once

#include <vector>

#include "config.h"
#include "cublas_wrapper.h"
#include "infernt_capi.h"
#include "kv_cache.h"
#include "tensor.h"
#include "weights.h"

class ModelArchitecture {
public:
    virtual ~ModelArchitecture() = default;

    virtual void allocate_activations(const ModelConfig& config, int max_batch_size) = 0;

    virtual void forward(const Tensor& input_embeddings, const ModelWeights& weights, KVCache& kv_cache,
                         int position, Tensor& logits) = 0;
};

class LlamaArchitecture : public ModelArchitecture {
public:
    explicit LlamaArchitecture(CublasWrapper& cublas);
    ~LlamaArchitecture() override;

    LlamaArchitecture(const LlamaArchitecture&) = delete;
    LlamaArchitecture& operator=(const LlamaArchitecture&) = delete;

    // Records the configuration; the decode-step scratch is allocated on the
    // first forward (once per weights / cache binding).  Batch 1 only, as the
    // reference's single-position forward (throws std::invalid_argument otherwise).
    void allocate_activations(const ModelConfig& config, int max_batch_size) override;

    // input_embeddings [1, h] at `position` -> logits [1, V]; also computes the
    // greedy token (last_token()).  Asynchronous on stream().
    void forward(const Tensor& input_embeddings, const ModelWeights& weights, KVCache& kv_cache,
                 int position, Tensor& logits) override;

    // Embedding lookup of token_id + forward + argmax, asynchronously.
    void forward_token(int token_id, const ModelWeights& weights, KVCache& kv_cache, int position,
                       Tensor& logits);

    // `steps` chained decode steps on the device from (token_id, position);
    // tokens_dev (device int[steps]) receives each produced token.
    void decode_chain(int token_id, int position, int steps, const ModelWeights& weights,
                      KVCache& kv_cache, int* tokens_dev);

    // Synchronises stream() and returns the greedy token of the last step.
    int last_token();

    cudaStream_t stream() const;
    // Kernels per decode step (launch accounting).
    int kernels_per_step() const;

    // The decode plan bound to these weights and this cache (created on first use).
    infernt_plan* plan_for(const ModelWeights& weights, KVCache& kv_cache) { return bind(weights, kv_cache, true); }

    // INFERNT_MODE_* for the following steps (rebinds the plan).
    void set_decode_mode(int mode);
    // The mode in use: the bound plan's, or the requested one before any step.
    int decode_mode() const;

private:
    // token_input: the plan will look tokens up in weights.embedding (else
    // only forward(), which takes the input embedding, runs on it)
    infernt_plan* bind(const ModelWeights& weights, KVCache& kv_cache, bool token_input);

    CublasWrapper& cublas_;
    ModelConfig config_;
    int max_batch_size_;
    int mode_;
    infernt_plan* plan_;
    std::vector<const void*> bound_weights_;
    std::vector<float*> bound_k_;
    std::vector<float*> bound_v_;
};
