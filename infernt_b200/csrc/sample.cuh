// sample.cuh — the Gumbel-max score shared by the standalone sampler
// (sample.cu) and the batched engine's argmax kernels (batch.cu): for logit
// x of vocabulary index i, x / T + g with g = -ln(-ln u), u a 24-bit uniform
// in (0, 1) hashed from (key, i) (splitmix64, include/infernt_seed.h).  The
// index with the largest score is a draw from softmax(logits / T).
#pragma once

#include <stdint.h>

#include "../../include/infernt_seed.h"

namespace infernt {

__device__ __forceinline__ float gumbel_score(float logit, float inv_t, uint64_t key, uint64_t i) {
    const uint64_t h = infernt_splitmix64(key + i);
    const float u = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    return fmaf(logit, inv_t, -logf(-logf(u)));
}

}  // namespace infernt
