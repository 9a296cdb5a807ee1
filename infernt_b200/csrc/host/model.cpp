// model.cpp — ModelConfig, KVCache, CublasWrapper, device init and the
// kernels.h launch_* functions (include/config.h, kv_cache.h,
// cublas_wrapper.h, cuda_utils.h, kernels.h).
#include <cuda_runtime.h>

#include <cstdio>
#include <stdexcept>
#include <string>

#include "config.h"
#include "cublas_wrapper.h"
#include "cuda_utils.h"
#include "infernt_capi.h"
#include "kernels.h"
#include "kv_cache.h"

namespace {
void check(int status, const char* what) {
    if (status != INFERNT_OK)
        throw std::runtime_error(std::string(what) + ": " + infernt_status_string(status) + " (" +
                                 infernt_last_error() + ")");
}
}  // namespace

// ------------------------------------------------------------ ModelConfig --
const char* activation_name(ActivationType a) {
    switch (a) {
        case ActivationType::SILU: return "SiLU";
        case ActivationType::GELU: return "GELU";
        case ActivationType::RELU: return "ReLU";
    }
    return "UNKNOWN";
}

const char* norm_type_name(NormType n) { return n == NormType::RMSNORM ? "RMSNorm" : "LayerNorm"; }

const char* position_embedding_name(PositionEmbeddingType p) {
    switch (p) {
        case PositionEmbeddingType::ROPE: return "RoPE";
        case PositionEmbeddingType::ABSOLUTE: return "Absolute";
        case PositionEmbeddingType::ALIBI: return "ALiBi";
    }
    return "UNKNOWN";
}

void ModelConfig::derive_computed_fields() {
    if (num_attention_heads > 0 && hidden_size > 0 && head_dim == 0) head_dim = hidden_size / num_attention_heads;
}

int ModelConfig::num_kv_groups() const {
    return num_key_value_heads == 0 ? 1 : num_attention_heads / num_key_value_heads;
}

void ModelConfig::validate() const {
    if (vocab_size <= 0) throw std::runtime_error("Invalid vocab_size");
    if (hidden_size <= 0) throw std::runtime_error("Invalid hidden_size");
    if (num_layers <= 0) throw std::runtime_error("Invalid num_layers");
    if (num_attention_heads <= 0) throw std::runtime_error("Invalid num_attention_heads");
    if (num_key_value_heads <= 0) throw std::runtime_error("Invalid num_key_value_heads");
    if (intermediate_size <= 0) throw std::runtime_error("Invalid intermediate_size");
    if (max_seq_len <= 0) throw std::runtime_error("Invalid max_seq_len");
    if (head_dim <= 0) throw std::runtime_error("Invalid head_dim");
    if (num_attention_heads % num_key_value_heads != 0)
        throw std::runtime_error("num_attention_heads must be divisible by num_key_value_heads");
    if (weight_dtype != DType::FP32 && weight_dtype != DType::BF16)
        throw std::runtime_error("weight_dtype must be FP32 or BF16");
}

void ModelConfig::print() const {
    std::printf("=== Model Configuration ===\n");
    std::printf("  Architecture:        %s\n", architecture.c_str());
    std::printf("  Vocab size:          %d\n", vocab_size);
    std::printf("  Hidden size:         %d\n", hidden_size);
    std::printf("  Num layers:          %d\n", num_layers);
    std::printf("  Attention heads:     %d\n", num_attention_heads);
    std::printf("  KV heads:            %d\n", num_key_value_heads);
    std::printf("  KV groups:           %d\n", num_kv_groups());
    std::printf("  Intermediate size:   %d\n", intermediate_size);
    std::printf("  Max seq len:         %d\n", max_seq_len);
    std::printf("  Head dim:            %d\n", head_dim);
    std::printf("  RMSNorm eps:         %.1e\n", rms_norm_eps);
    std::printf("  RoPE theta:          %.1f\n", rope_theta);
    std::printf("  Activation:          %s\n", activation_name(activation));
    std::printf("  Normalization:       %s\n", norm_type_name(norm_type));
    std::printf("  Position embedding:  %s\n", position_embedding_name(position_embedding));
    std::printf("  Weight dtype:        %s\n", dtype_name(weight_dtype));
    std::printf("===========================\n");
}

// ---------------------------------------------------------------- KVCache --
void KVCache::allocate(const ModelConfig& config) {
    max_seq_len = config.max_seq_len;
    current_seq_len = 0;
    k_cache.clear();
    v_cache.clear();
    for (int l = 0; l < config.num_layers; ++l) {
        k_cache.push_back(Tensor::zeros({config.num_key_value_heads, max_seq_len, config.head_dim}, DType::FP32,
                                        Device::CUDA));
        v_cache.push_back(Tensor::zeros({config.num_key_value_heads, max_seq_len, config.head_dim}, DType::FP32,
                                        Device::CUDA));
    }
}

void KVCache::reset() {
    current_seq_len = 0;
    for (auto& t : k_cache)
        if (cudaMemset(t.data_ptr(), 0, t.size_bytes()) != cudaSuccess) throw std::runtime_error("KV reset failed");
    for (auto& t : v_cache)
        if (cudaMemset(t.data_ptr(), 0, t.size_bytes()) != cudaSuccess) throw std::runtime_error("KV reset failed");
}

// ---------------------------------------------------------- CublasWrapper --
CublasWrapper::CublasWrapper() : stream_(nullptr) {}
CublasWrapper::~CublasWrapper() = default;

void CublasWrapper::gemm(const float* A, const float* B, float* C, int M, int N, int K, float alpha, float beta,
                         bool trans_a, bool trans_b) {
    check(infernt_gemm_f32(A, B, C, M, N, K, alpha, beta, trans_a, trans_b, stream_), "CublasWrapper::gemm");
}

void CublasWrapper::batched_gemm(const float* A, const float* B, float* C, int M, int N, int K, int batch_count,
                                 int stride_a, int stride_b, int stride_c, float alpha, float beta, bool trans_a,
                                 bool trans_b) {
    for (int b = 0; b < batch_count; ++b)
        gemm(A + (size_t)b * stride_a, B + (size_t)b * stride_b, C + (size_t)b * stride_c, M, N, K, alpha, beta,
             trans_a, trans_b);
}

void CublasWrapper::set_stream(cudaStream_t stream) { stream_ = stream; }
cublasHandle_t CublasWrapper::handle() const { return nullptr; }
cudaStream_t CublasWrapper::stream() const { return stream_; }

// ------------------------------------------------------------ device init --
void cuda_init(int device_id) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) throw std::runtime_error("No CUDA-capable GPU detected");
    if (device_id < 0 || device_id >= n) throw std::runtime_error("Requested CUDA device does not exist");
    if (cudaSetDevice(device_id) != cudaSuccess) throw std::runtime_error("cudaSetDevice failed");
}

GPUInfo cuda_get_device_info(int device_id) {
    GPUInfo info = {};
    info.device_id = device_id;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device_id) != cudaSuccess)
        throw std::runtime_error("cudaGetDeviceProperties failed");
    std::snprintf(info.name, sizeof(info.name), "%s", prop.name);
    info.total_memory = prop.totalGlobalMem;
    info.compute_major = prop.major;
    info.compute_minor = prop.minor;
    info.sm_count = prop.multiProcessorCount;
    info.max_threads_per_block = prop.maxThreadsPerBlock;
    info.warp_size = prop.warpSize;
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    info.free_memory = free_b;
    return info;
}

void cuda_print_device_info(const GPUInfo& info) {
    std::printf("=== GPU Device Info ===\n");
    std::printf("  Device ID:           %d\n", info.device_id);
    std::printf("  Name:                %s\n", info.name);
    std::printf("  Total Memory:        %.2f GB\n", info.total_memory / (1024.0 * 1024.0 * 1024.0));
    std::printf("  Free Memory:         %.2f GB\n", info.free_memory / (1024.0 * 1024.0 * 1024.0));
    std::printf("  Compute Capability:  %d.%d\n", info.compute_major, info.compute_minor);
    std::printf("  SM Count:            %d\n", info.sm_count);
    std::printf("=======================\n");
}

size_t cuda_get_free_memory() {
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    return free_b;
}

// ------------------------------------------------------- kernels.h shims --
void launch_rmsnorm(float* o, const float* i, const float* w, int b, int h, float eps, cudaStream_t s) {
    check(infernt_rmsnorm(o, i, w, b, h, eps, s), "launch_rmsnorm");
}
void launch_residual_add(float* o, const float* a, const float* b, int n, cudaStream_t s) {
    check(infernt_residual_add(o, a, b, n, s), "launch_residual_add");
}
void launch_rope(float* q, float* k, int b, int nq, int nkv, int d, int pos, float theta, cudaStream_t s) {
    check(infernt_rope(q, k, b, nq, nkv, d, pos, theta, s), "launch_rope");
}
void launch_softmax(float* o, const float* i, int b, int n, cudaStream_t s) {
    check(infernt_softmax(o, i, b, n, s), "launch_softmax");
}
void launch_softmax_with_mask(float* o, const float* i, int h, int n, int total, cudaStream_t s) {
    check(infernt_softmax_with_mask(o, i, h, n, total, s), "launch_softmax_with_mask");
}
void launch_kv_cache_append(float* kc, float* vc, const float* kn, const float* vn, int nkv, int d, int max_seq,
                            int pos, cudaStream_t s) {
    check(infernt_kv_cache_append(kc, vc, kn, vn, nkv, d, max_seq, pos, s), "launch_kv_cache_append");
}
void launch_attention_scores(float* sc, const float* q, const float* kc, int nq, int nkv, int d, int seq,
                             int max_seq, float scale, cudaStream_t s) {
    check(infernt_attention_scores(sc, q, kc, nq, nkv, d, seq, max_seq, scale, s), "launch_attention_scores");
}
void launch_attention_values(float* o, const float* sc, const float* vc, int nq, int nkv, int d, int seq,
                             int max_seq, cudaStream_t s) {
    check(infernt_attention_values(o, sc, vc, nq, nkv, d, seq, max_seq, s), "launch_attention_values");
}
void launch_silu_mul(float* o, const float* g, const float* u, int n, cudaStream_t s) {
    check(infernt_silu_mul(o, g, u, n, s), "launch_silu_mul");
}
void launch_embedding_lookup(float* o, const float* t, int tok, int h, cudaStream_t s) {
    check(infernt_embedding_lookup(o, t, tok, h, s), "launch_embedding_lookup");
}
void launch_argmax(int* o, const float* l, int v, cudaStream_t s) { check(infernt_argmax(o, l, v, s), "launch_argmax"); }
