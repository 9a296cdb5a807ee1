// sample.cu — temperature sampling on the GPU.  The reference samples on the
// host (src/engine.cpp:78-104): softmax of logits / T, one uniform draw from
// a mt19937 seeded 1337, inverse-CDF walk over the vocabulary.  Here the
// same distribution is drawn on the device by the Gumbel-max method
// (Gumbel 1954; e.g. Maddison et al. 2014): with g_i = -ln(-ln u_i) for
// independent uniforms u_i, argmax_i (logit_i / T + g_i) is distributed as
// softmax(logit / T), so sampling is an argmax pass over the logits with no
// normalisation and no host round trip.  u_i is a counter-based hash of
// (seed, counter, i) (splitmix64, include/infernt_seed.h), 24 bits, in
// (0, 1); the draws are reproducible for a given (seed, counter).  T <= 0
// is the greedy argmax.  Ties go to the lowest index, NaN never wins.
//
// Rows are independent samples: row r reads logits + r * ld (ld = 0: every
// row samples the same logits) with counter + r.  Per row kChunks CTAs scan
// a slice each; the last CTA of the row to finish (ticket, left at 0)
// combines the candidates in slice order.
#include <cstdint>

#include "../../include/infernt_seed.h"
#include "common.cuh"
#include "internal.h"
#include "sample.cuh"

namespace infernt {
namespace {

constexpr int kChunks = 16;
constexpr int kThreads = 256;

struct SampleWs {
    unsigned* tickets;  // [rows]
    int2* cand;         // [rows][kChunks] (score bits, index)
};

__global__ void __launch_bounds__(kThreads) sample_gumbel(const float* logits, long long ld, int V, float inv_t,
                                                          bool greedy, uint64_t seed, uint64_t counter, int* out,
                                                          SampleWs ws) {
    __shared__ float bv[kThreads / 32];
    __shared__ int bi[kThreads / 32];
    const int chunk = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
    const float* lr = logits + (size_t)row * (size_t)ld;
    const uint64_t key = infernt_stream_key(seed, counter + (uint64_t)row);
    const int i0 = (int)((long long)V * chunk / kChunks), i1 = (int)((long long)V * (chunk + 1) / kChunks);
    float v = -INFINITY;
    int id = 0x7fffffff;
    for (int i = i0 + tid; i < i1; i += kThreads) {
        float s = lr[i];
        if (!greedy) s = gumbel_score(s, inv_t, key, (uint64_t)i);
        if (argmax_better(s, i, v, id)) {
            v = s;
            id = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, id, o);
        if (argmax_better(ov, oi, v, id)) {
            v = ov;
            id = oi;
        }
    }
    if ((tid & 31) == 0) {
        bv[tid >> 5] = v;
        bi[tid >> 5] = id;
    }
    __syncthreads();
    if (tid != 0) return;
    for (int w = 1; w < kThreads / 32; ++w)
        if (argmax_better(bv[w], bi[w], v, id)) {
            v = bv[w];
            id = bi[w];
        }
    int2* cr = ws.cand + (size_t)row * kChunks;
    cr[chunk] = make_int2(__float_as_int(v), id);
    __threadfence();
    const unsigned done = atomicAdd(ws.tickets + row, 1u) + 1u;
    if (done != (unsigned)kChunks) return;
    ws.tickets[row] = 0u;
    __threadfence();
    v = -INFINITY;
    id = 0x7fffffff;
    for (int c = 0; c < kChunks; ++c) {
        const int2 x = __ldcg(cr + c);
        if (argmax_better(__int_as_float(x.x), x.y, v, id)) {
            v = __int_as_float(x.x);
            id = x.y;
        }
    }
    out[row] = id == 0x7fffffff ? 0 : id;  // every score NaN: token 0
}

}  // namespace
}  // namespace infernt

extern "C" size_t infernt_sample_workspace_bytes(int rows) {
    if (rows < 1) return 0;
    const size_t t = ((size_t)rows * sizeof(unsigned) + 255) / 256 * 256;
    return t + (size_t)rows * infernt::kChunks * sizeof(int2);
}

extern "C" int infernt_sample_tokens(const float* logits, long long ld, int rows, int vocab_size, float temperature,
                                     uint64_t seed, uint64_t counter, int* out_tokens, void* workspace,
                                     void* stream) {
    using namespace infernt;
    INFERNT_REQUIRE(logits && out_tokens && workspace, "sample_tokens: null pointer");
    INFERNT_REQUIRE(rows >= 1 && rows <= 65535 && vocab_size >= 1 && ld >= 0, "sample_tokens: %d rows of %d, ld %lld",
                    rows, vocab_size, ld);
    INFERNT_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15u) == 0, "sample_tokens: workspace not 16-byte aligned");
    SampleWs ws;
    ws.tickets = static_cast<unsigned*>(workspace);
    ws.cand = reinterpret_cast<int2*>(static_cast<char*>(workspace) +
                                      ((size_t)rows * sizeof(unsigned) + 255) / 256 * 256);
    const bool greedy = !(temperature > 0.0f);
    sample_gumbel<<<dim3(kChunks, rows), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        logits, ld, vocab_size, greedy ? 1.0f : 1.0f / temperature, greedy, seed, counter, out_tokens, ws);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}
