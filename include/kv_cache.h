// kv_cache.h — per-layer K and V caches, [num_kv_heads, max_seq_len,
// head_dim] FP32 each (the reference's include/kv_cache.h:7-15 layout).
#pragma once

#include <vector>

#include "config.h"
#include "tensor.h"

struct KVCache {
    std::vector<Tensor> k_cache;
    std::vector<Tensor> v_cache;
    int current_seq_len = 0;
    int max_seq_len = 0;

    // One zero-filled [Nkv, max_seq_len, D] FP32 tensor per layer for K and V.
    void allocate(const ModelConfig& config);
    // Zero every cache tensor (src/kv_cache.cpp:22-30 semantics).
    void reset();
};
