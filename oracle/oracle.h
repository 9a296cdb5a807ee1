/*
 * oracle.h — CPU oracle for INFERNT's decode step (TEST INFRASTRUCTURE).
 *
 * This is a scalar C restatement of the reference engine's FP32 decode
 * math, written to check the CUDA path.  It is test infrastructure only:
 * the tests, the smoke check and the benchmark's CPU-baseline leg may call
 * it; the product library never links or calls it.
 *
 * Parity pins: the per-op functions are checked against the known-answer
 * tests of the reference's self-test suite (src/main.cpp:108-681, fixtures
 * in tests/golden/kat.json), and the full forward against logits produced
 * by the reference's own CUDA build (tests/golden/ref_forward_*.npz).
 *
 * Reductions (dot products, sums of squares, softmax sums) accumulate in
 * double; every intermediate tensor is stored as float, as the reference's
 * buffers are.  Element-wise formulas keep the reference's float
 * expressions (RoPE angle, SiLU, softmax exp) so the result is the exact
 * math the reference intends, rounded once per stored tensor.
 */
#ifndef INFERNT_ORACLE_H
#define INFERNT_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int vocab_size;
    int hidden_size;
    int num_layers;
    int num_attention_heads;
    int num_key_value_heads;
    int intermediate_size;
    int max_seq_len;
    int head_dim;
    float rms_norm_eps;
    float rope_theta;
} oracle_config;

/* Worker threads used by the matrix-vector products (default 1). */
void oracle_set_threads(int n);
/* Batched-decode variant: round activations to bf16 where they enter a
 * projection, and K/V rows before they enter the cache (default off). */
void oracle_set_act_bf16(int on);
int oracle_get_threads(void);

/* ---- synthetic inputs (same values as the device initialiser) ---- */
void oracle_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream,
                        float std_dev, int round_bf16);
/* Elements [start, start + n) of a stream. */
void oracle_fill_normal_range(float* out, size_t n, uint64_t seed, uint64_t stream,
                              float std_dev, int round_bf16, uint64_t start);
void oracle_fill_const(float* out, size_t n, float value);
void oracle_fill_prompt(int* out, int n, uint64_t seed, int lo, int hi);

/* ---- per-op restatements (reference file:line in oracle.c) ---- */
void oracle_rmsnorm(float* out, const float* in, const float* w, int batch,
                    int hidden, float eps);
void oracle_residual_add(float* out, const float* a, const float* b, int n);
void oracle_rope(float* q, float* k, int batch, int num_q_heads,
                 int num_kv_heads, int head_dim, int position, float theta);
void oracle_softmax(float* out, const float* in, int rows, int seq_len);
void oracle_softmax_with_mask(float* out, const float* in, int heads,
                              int seq_len, int total_seq_len);
void oracle_kv_cache_append(float* k_cache, float* v_cache, const float* k_new,
                            const float* v_new, int num_kv_heads, int head_dim,
                            int max_seq_len, int position);
void oracle_attention_scores(float* scores, const float* q, const float* k_cache,
                             int num_q_heads, int num_kv_heads, int head_dim,
                             int seq_len, int max_seq_len, float scale);
void oracle_attention_values(float* out, const float* scores,
                             const float* v_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int seq_len,
                             int max_seq_len);
void oracle_silu_mul(float* out, const float* gate, const float* up, int n);
void oracle_embedding_lookup(float* out, const float* table, int token_id,
                             int hidden);
/* Lowest index among the maximal values; NaN never wins; start (-1e30, 0). */
int oracle_argmax(const float* logits, int vocab_size);
/* The reference kernel's own tie order (256-thread stride + tree). */
int oracle_argmax_ref_order(const float* logits, int vocab_size);
/* Row-major C[M,N] = alpha * op(A)[M,K] . op(B)[K,N] + beta * C. */
void oracle_gemm(const float* A, const float* B, float* C, int M, int N, int K,
                 float alpha, float beta, int trans_a, int trans_b);

/* ---- the decode step ----
 * weights: flat array of 3 + 9*L float pointers:
 *   [0] embedding [V,h]  [1] final_norm [h]  [2] lm_head [V,h]
 *   [3 + 9*l + j], j = attn_norm, q, k, v, o, ffn_norm, gate, up, down
 * kv_k / kv_v: num_layers * num_kv_heads * max_seq_len * head_dim floats
 * (layer-major, [N_kv, max_seq, D] per layer).
 */
void oracle_llama_forward(const oracle_config* cfg, const float* const* weights,
                          float* kv_k, float* kv_v, int position,
                          const float* input_embedding, float* logits);
/* One decode step: embedding lookup + forward + argmax (lowest index). */
int oracle_decode_token(const oracle_config* cfg, const float* const* weights,
                        float* kv_k, float* kv_v, int token, int position,
                        float* logits);
/* Forward only layers [0, n_layers) (no final norm / head); writes the
 * residual stream after them to hidden_out.  For truncated spot checks. */
void oracle_llama_layers(const oracle_config* cfg, const float* const* weights,
                         float* kv_k, float* kv_v, int position,
                         const float* input_embedding, int n_layers,
                         float* hidden_out);

#ifdef __cplusplus
}
#endif
#endif /* INFERNT_ORACLE_H */
