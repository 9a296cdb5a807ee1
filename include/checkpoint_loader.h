// checkpoint_loader.h — INFT v1 checkpoints (config.json + model.bin), the
// same interface as the reference's include/checkpoint_loader.h:7-14
// (loader/checkpoint_loader.cpp).  Format of model.bin (little-endian):
//   uint32 magic 0x494E4654 ("INFT"), uint32 version 1, uint32 tensor count;
//   per tensor: int32 name length, UTF-8 name, int32 dim count, int32 dims[],
//   int64 element count, element count x FP32 payload.
// Names follow the Hugging Face Llama layout (model.embed_tokens.weight,
// model.norm.weight, lm_head.weight, model.layers.<i>.{input_layernorm,
// self_attn.{q,k,v,o}_proj, post_attention_layernorm,
// mlp.{gate,up,down}_proj}.weight); other names are skipped.
#pragma once

#include <string>

#include "config.h"
#include "weights.h"

class CheckpointLoader {
public:
    // Keys as the reference reads them (architecture, vocab_size, hidden_size,
    // num_layers, num_attention_heads, num_key_value_heads, intermediate_size,
    // max_seq_len = 2048, rms_norm_eps = 1e-5, rope_theta = 10000 when absent);
    // optional head_dim, and weight_dtype "bf16" / "fp32" (default fp32).
    // Throws std::runtime_error if the file cannot be read or the config is
    // invalid.
    static ModelConfig load_config(const std::string& config_path);
    // Fills `weights` (norms and embedding FP32; projections and lm_head in
    // config.weight_dtype, bf16 rounded to nearest even) on target_device.
    // A missing lm_head is a copy of the embedding, any other tensor the file
    // lacks stays empty (both as the reference).  Throws std::runtime_error
    // on a bad magic or version, a truncated file, or a tensor whose element
    // count does not match the config.
    static void load_weights(const std::string& weights_path, const ModelConfig& config, ModelWeights& weights,
                             Device target_device = Device::CUDA);
};
