// kernels.h — the reference's kernel entry points (include/kernels.h:5-49),
// same signatures, running the B200 kernels of the C ABI
// (include/infernt_capi.h).  A failed launch throws std::runtime_error
// (the reference's launches are unchecked).
#pragma once

#include <cuda_runtime.h>

void launch_rmsnorm(float* output, const float* input, const float* weight, int batch_size,
                    int hidden_size, float eps, cudaStream_t stream = nullptr);

void launch_residual_add(float* output, const float* a, const float* b, int num_elements,
                         cudaStream_t stream = nullptr);

void launch_rope(float* q, float* k, int batch_size, int num_q_heads, int num_kv_heads, int head_dim,
                 int position, float theta, cudaStream_t stream = nullptr);

void launch_softmax(float* output, const float* input, int batch_size, int seq_len,
                    cudaStream_t stream = nullptr);

void launch_softmax_with_mask(float* output, const float* input, int num_heads, int seq_len,
                              int total_seq_len, cudaStream_t stream = nullptr);

void launch_kv_cache_append(float* k_cache, float* v_cache, const float* k_new, const float* v_new,
                            int num_kv_heads, int head_dim, int max_seq_len, int position,
                            cudaStream_t stream = nullptr);

void launch_attention_scores(float* scores, const float* q, const float* k_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int seq_len, int max_seq_len, float scale,
                             cudaStream_t stream = nullptr);

void launch_attention_values(float* output, const float* scores, const float* v_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int seq_len, int max_seq_len,
                             cudaStream_t stream = nullptr);

void launch_silu_mul(float* out, const float* gate, const float* up, int num_elements,
                     cudaStream_t stream = nullptr);

void launch_embedding_lookup(float* output, const float* table, int token_id, int hidden_size,
                             cudaStream_t stream = nullptr);

void launch_argmax(int* out_token, const float* logits, int vocab_size, cudaStream_t stream = nullptr);
