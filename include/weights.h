// weights.h — weight containers, as the reference's include/weights.h:8-25.
// Projection matrices are row-major [out, in]; norms and the embedding are
// FP32, projections and lm_head have ModelConfig::weight_dtype.
#pragma once

#include <vector>

#include "config.h"
#include "tensor.h"

struct TransformerLayerWeights {
    Tensor attn_norm;
    Tensor q_proj;
    Tensor k_proj;
    Tensor v_proj;
    Tensor o_proj;
    Tensor ffn_norm;
    Tensor gate_proj;
    Tensor up_proj;
    Tensor down_proj;
};

struct ModelWeights {
    Tensor embedding;
    std::vector<TransformerLayerWeights> layers;
    Tensor final_norm;
    Tensor lm_head;
};
