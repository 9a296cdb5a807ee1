// attention.cuh — argument block and launcher of the decode attention kernel
// (attention.cu).
#pragma once

#include "common.cuh"

namespace infernt {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnTile = 64;
constexpr int kAttnMaxD = 128;
constexpr int kAttnMaxGroup = 16;
constexpr int kAttnMinChunk = 32;

struct AttnArgs {
    const float* qkv;  // [Nq*D | Nkv*D | Nkv*D], before RoPE
    float* k_cache;    // [Nkv, max_seq, D]
    float* v_cache;
    float* out;        // [Nq*D]
    float* part;       // [Nkv][splits][G][D + 2]
    unsigned* counter; // [Nkv], zero between launches
    const int* pos_ptr;  // device position, or NULL to use pos
    int pos;
    int nq, nkv, D, max_seq, splits;
    float theta, scale;
    unsigned* err;
};

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t stream, bool pdl);
int attention_shape_check(int nq, int nkv, int D, int splits);
size_t attention_workspace_bytes(int nq, int nkv, int D, int splits);

}  // namespace infernt
