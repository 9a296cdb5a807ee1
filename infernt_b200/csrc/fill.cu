// fill.cu — seeded synthetic weights and KV prefill on the device, using
// the same counter-based generator as the host (include/infernt_seed.h), so
// device-filled tensors are bit-identical to host-filled ones.
#include "../../include/infernt_seed.h"
#include "common.cuh"
#include "internal.h"

namespace infernt {
namespace {

__global__ void fill_normal_f32(float* dst, size_t n, uint64_t key, float std_dev) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = infernt_normal_std(key, i, std_dev);
}

__global__ void fill_normal_bf16(__nv_bfloat16* dst, size_t n, uint64_t key, float std_dev) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(infernt_normal_std(key, i, std_dev));
}

// dst [rows][ld_dst] = the window (row0.., col0..) of a seeded matrix with
// src_ld columns; columns cols..ld_dst-1 are zero (padding)
template <typename T>
__global__ void fill_window(T* dst, int rows, int cols, int ld_dst, uint64_t src_ld, uint64_t row0, uint64_t col0,
                            uint64_t key, float std_dev) {
    const size_t n = (size_t)rows * ld_dst;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / ld_dst), c = (int)(i % ld_dst);
        const float v = c < cols ? infernt_normal_std(key, (row0 + r) * src_ld + col0 + c, std_dev) : 0.0f;
        if constexpr (sizeof(T) == 2)
            dst[i] = __float2bfloat16_rn(v);
        else
            dst[i] = v;
    }
}

__global__ void fill_const_f32(float* dst, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = v;
}

// one layer's [Nkv, max_seq, D] cache; rows >= n_pos are zero
__global__ void fill_kv_layer(float* dst, int layer, int nkv, int max_seq, int D, int n_pos, uint64_t key,
                              float std_dev) {
    const size_t n = (size_t)nkv * max_seq * D;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int p = (int)((i / D) % max_seq);
        const int h = (int)(i / ((size_t)D * max_seq));
        const uint64_t gi = ((((uint64_t)layer * nkv + h) << 20) + (uint64_t)p) * (uint64_t)D + d;
        dst[i] = p < n_pos ? infernt_normal_std(key, gi, std_dev) : 0.0f;
    }
}

int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)sm_count() * 16;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace infernt

using namespace infernt;

extern "C" {

int infernt_fill_normal(void* dst, size_t n, int dtype, uint64_t seed, uint64_t stream_id, float std_dev,
                        void* stream) {
    INFERNT_REQUIRE(dst, "fill_normal: null destination");
    if (n == 0) return INFERNT_OK;
    const uint64_t key = infernt_stream_key(seed, stream_id);
    if (dtype == INFERNT_DTYPE_BF16)
        fill_normal_bf16<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(static_cast<__nv_bfloat16*>(dst), n,
                                                                        key, std_dev);
    else if (dtype == INFERNT_DTYPE_F32)
        fill_normal_f32<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(static_cast<float*>(dst), n, key,
                                                                       std_dev);
    else
        return fail(INFERNT_ERR_INVALID_ARGUMENT, "fill_normal: dtype %d", dtype);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int infernt_fill_normal_window(void* dst, int rows, int cols, int ld_dst, uint64_t src_ld, uint64_t row0,
                               uint64_t col0, int dtype, uint64_t seed, uint64_t stream_id, float std_dev,
                               void* stream) {
    INFERNT_REQUIRE(dst && rows >= 0 && cols >= 0 && ld_dst >= cols && col0 + (uint64_t)cols <= src_ld,
                    "fill_normal_window: bad window");
    const size_t n = (size_t)rows * ld_dst;
    if (n == 0) return INFERNT_OK;
    const uint64_t key = infernt_stream_key(seed, stream_id);
    if (dtype == INFERNT_DTYPE_BF16)
        fill_window<__nv_bfloat16><<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(
            static_cast<__nv_bfloat16*>(dst), rows, cols, ld_dst, src_ld, row0, col0, key, std_dev);
    else if (dtype == INFERNT_DTYPE_F32)
        fill_window<float><<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(static_cast<float*>(dst), rows, cols,
                                                                           ld_dst, src_ld, row0, col0, key, std_dev);
    else
        return fail(INFERNT_ERR_INVALID_ARGUMENT, "fill_normal_window: dtype %d", dtype);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int infernt_fill_const(float* dst, size_t n, float value, void* stream) {
    INFERNT_REQUIRE(dst, "fill_const: null destination");
    if (n == 0) return INFERNT_OK;
    fill_const_f32<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(dst, n, value);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int infernt_fill_prompt(int* out_host, int n, uint64_t seed, int lo, int hi) {
    INFERNT_REQUIRE(out_host && n >= 0 && lo < hi, "fill_prompt: bad arguments");
    const uint64_t key = infernt_stream_key(seed, INFERNT_STREAM_PROMPT);
    for (int i = 0; i < n; ++i) out_host[i] = infernt_uniform_int(key, (uint64_t)i, lo, hi);
    return INFERNT_OK;
}

int infernt_fill_kv(float* const* k_cache, float* const* v_cache, int num_layers, int num_kv_heads,
                    int max_seq_len, int head_dim, int n_pos, uint64_t seed, float std_dev, void* stream) {
    INFERNT_REQUIRE(k_cache && v_cache && num_layers > 0 && num_kv_heads > 0 && max_seq_len > 0 && head_dim > 0,
                    "fill_kv: bad arguments");
    INFERNT_REQUIRE(n_pos >= 0 && n_pos <= max_seq_len && max_seq_len <= (1 << 20), "fill_kv: n_pos %d", n_pos);
    const uint64_t kk = infernt_stream_key(seed, INFERNT_STREAM_KV_K);
    const uint64_t vk = infernt_stream_key(seed, INFERNT_STREAM_KV_V);
    const size_t n = (size_t)num_kv_heads * max_seq_len * head_dim;
    for (int l = 0; l < num_layers; ++l) {
        fill_kv_layer<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(k_cache[l], l, num_kv_heads, max_seq_len,
                                                                     head_dim, n_pos, kk, std_dev);
        fill_kv_layer<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(v_cache[l], l, num_kv_heads, max_seq_len,
                                                                     head_dim, n_pos, vk, std_dev);
    }
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

}  // extern "C"
