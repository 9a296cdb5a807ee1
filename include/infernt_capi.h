/*
 * infernt_capi.h — the C ABI of the B200 decode engine.
 *
 * Every entry point takes plain pointers and sizes, an explicit CUDA stream
 * (`void*` holding a cudaStream_t; NULL = the legacy default stream, the
 * stream every reference launch uses) and returns an int status (0 = OK).
 * Nothing here calls exit().  Kernel launches are asynchronous: a 0 status
 * means the launch was accepted; device-side faults detected by the kernels
 * themselves (wait timeouts, out-of-range positions or token ids) are
 * reported by the synchronising calls (infernt_plan_read_token and the
 * engine calls) as INFERNT_ERR_DEVICE.
 *
 * Each function names the reference interface it replaces (paths relative
 * to the INFERNT repository).  All device pointers must come from
 * cudaMalloc (256-byte aligned) or be offsets into such memory that keep
 * the alignment each function states.
 */
#ifndef INFERNT_CAPI_H
#define INFERNT_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INFERNT_API __attribute__((visibility("default")))

/* ------------------------------------------------------------- status --- */
enum {
    INFERNT_OK = 0,
    INFERNT_ERR_INVALID_ARGUMENT = 1, /* shape, pointer or range check failed */
    INFERNT_ERR_UNSUPPORTED = 2,      /* valid but not implemented on this path */
    INFERNT_ERR_CUDA = 3,             /* a CUDA runtime call failed */
    INFERNT_ERR_OUT_OF_MEMORY = 4,
    INFERNT_ERR_DEVICE = 5,           /* a kernel reported an error word */
    INFERNT_ERR_NO_DEVICE = 6         /* no sm_100 device is visible */
};

INFERNT_API const char* infernt_status_string(int status);
/* Detail of the last failing call on this host thread ("" if none). */
INFERNT_API const char* infernt_last_error(void);
INFERNT_API int infernt_version(void);

/* ---------------------------------------- include/kernels.h mirrors ---
 * Same argument meaning as the reference's launch_* functions.          */

/* kernels.h:5-7 (cuda/rmsnorm.cu:29-35): out[b] = in[b] * rsqrt(mean(in[b]^2) + eps) * w */
INFERNT_API int infernt_rmsnorm(float* out, const float* in, const float* weight, int batch,
                                int hidden, float eps, void* stream);
/* kernels.h:9-10 (cuda/residual.cu:12-17): out = a + b (out may alias a or b) */
INFERNT_API int infernt_residual_add(float* out, const float* a, const float* b, int n,
                                     void* stream);
/* kernels.h:12-15 (cuda/rope.cu:37-46): split-half RoPE of q [Nq, D] and k [Nkv, D] in place */
INFERNT_API int infernt_rope(float* q, float* k, int batch, int num_q_heads, int num_kv_heads,
                             int head_dim, int position, float theta, void* stream);
/* kernels.h:17-19 (cuda/softmax.cu:101-106): row softmax of [rows, seq_len], in place allowed */
INFERNT_API int infernt_softmax(float* out, const float* in, int rows, int seq_len, void* stream);
/* kernels.h:21-23 (cuda/softmax.cu:108-115): softmax of the first seq_len entries of rows of
 * total_seq_len, tail zeroed */
INFERNT_API int infernt_softmax_with_mask(float* out, const float* in, int num_heads,
                                          int seq_len, int total_seq_len, void* stream);
/* kernels.h:25-29 (cuda/kv_cache.cu:16-26): cache[h][position][:] = new[h][:] for K and V */
INFERNT_API int infernt_kv_cache_append(float* k_cache, float* v_cache, const float* k_new,
                                        const float* v_new, int num_kv_heads, int head_dim,
                                        int max_seq_len, int position, void* stream);
/* kernels.h:31-34 (cuda/attention.cu:45-53): scores[qh][p] = scale * q[qh].K[kvh][p],
 * kvh = qh / (Nq/Nkv), row stride seq_len; every position is computed (no 1024 cap) */
INFERNT_API int infernt_attention_scores(float* scores, const float* q, const float* k_cache,
                                         int num_q_heads, int num_kv_heads, int head_dim,
                                         int seq_len, int max_seq_len, float scale,
                                         void* stream);
/* kernels.h:36-39 (cuda/attention.cu:55-64): out[qh][d] = sum_p P[qh][p] V[kvh][p][d] */
INFERNT_API int infernt_attention_values(float* out, const float* scores, const float* v_cache,
                                         int num_q_heads, int num_kv_heads, int head_dim,
                                         int seq_len, int max_seq_len, void* stream);
/* kernels.h:41-42 (cuda/activation.cu:13-17): out = g / (1 + exp(-g)) * u */
INFERNT_API int infernt_silu_mul(float* out, const float* gate, const float* up, int n,
                                 void* stream);
/* kernels.h:44-46 (cuda/embedding.cu:10-14): out = table[token_id] (row of hidden) */
INFERNT_API int infernt_embedding_lookup(float* out, const float* table, int token_id,
                                         int hidden, void* stream);
/* kernels.h:48-49 (cuda/sampling.cu:38-40): *out_token = argmax(logits), one pass over all
 * SMs whose last block reduces the per-block winners.  Ties -> lowest index; NaN never wins;
 * all values <= -1e30 -> 0.  Uses a small per-device workspace allocated on the first call
 * on each device (make that first call outside stream capture). */
INFERNT_API int infernt_argmax(int* out_token, const float* logits, int vocab_size,
                               void* stream);

/* -------------------------------- include/cublas_wrapper.h:23-26 mirror ---
 * Row-major C[M,N] = alpha * op(A)[M,K] . op(B)[K,N] + beta * C with
 * lda = trans_a ? M : K, ldb = trans_b ? K : N, ldc = N
 * (gemm/cublas_wrapper.cu:21-40).  FP32 arithmetic (no TF32).             */
INFERNT_API int infernt_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K,
                                 float alpha, float beta, int trans_a, int trans_b,
                                 void* stream);

/* --------------------------------------------------- fused decode ops ---
 * Building blocks of the decode step, each one kernel.  `weight_dtype`:
 * INFERNT_DTYPE_F32 (float weights) or INFERNT_DTYPE_BF16 (bf16 weights,
 * fp32 accumulation).  Weights are row-major [out, in] (the HF layout the
 * reference multiplies with trans_b = true, llama_layer.cpp:18-69).
 * The fast path (TMA-staged weight streaming) needs `in` % 512 == 0 and
 * 16-byte aligned rows; other shapes run a plain-load kernel.
 * These kernels and infernt_attention_decode launch with programmatic
 * dependent launch: one may start while the previous kernel on the stream
 * is finishing and stream its weights then, but it reads every other input
 * and writes its outputs only after that kernel has completed.  So the
 * weights must not be written by the kernel launched just before.       */
enum { INFERNT_DTYPE_F32 = 0, INFERNT_DTYPE_BF16 = 1 };

/* y[n] = sum_k W[n][k] * xn[k] with xn = rmsnorm(x, norm_w, eps) when norm_w != NULL
 * (llama_layer.cpp:11-23 with the rmsnorm fused).  Rows of W0, W1, W2 (any of W1/W2 NULL)
 * are stacked: y = [W0 x ; W1 x ; W2 x] (the Q, K, V projections in one pass). */
INFERNT_API int infernt_rmsnorm_gemv(float* y, const void* W0, int n0, const void* W1, int n1,
                                     const void* W2, int n2, int in_features, int weight_dtype,
                                     const float* x, const float* norm_w, float eps,
                                     void* stream);
/* out[n] = res[n] + sum_k W[n][k] x[k] (llama_layer.cpp:51-55 and :68-72; out may alias res) */
INFERNT_API int infernt_gemv_residual(float* out, const float* res, const void* W, int n,
                                      int in_features, int weight_dtype, const float* x,
                                      void* stream);
/* out[i] = silu(gate_i) * up_i with gate = Wg xn, up = Wu xn, xn = rmsnorm(x, norm_w)
 * (llama_layer.cpp:57-66) */
INFERNT_API int infernt_rmsnorm_gate_up_silu(float* out, const void* Wg, const void* Wu, int n,
                                             int in_features, int weight_dtype, const float* x,
                                             const float* norm_w, float eps, void* stream);
/* RoPE of q and k at `position`, KV append, and split-KV GQA attention with online softmax
 * over positions [0, position] (llama_layer.cpp:25-48; cuda/rope.cu, kv_cache.cu,
 * attention.cu, softmax.cu).  qkv = [q (Nq*D) | k (Nkv*D) | v (Nkv*D)] before RoPE; out =
 * attention output [Nq*D].  workspace: infernt_attention_workspace_bytes() bytes, zeroed
 * once before first use (the kernel leaves its counters at zero). */
INFERNT_API size_t infernt_attention_workspace_bytes(int num_q_heads, int num_kv_heads,
                                                     int head_dim, int splits);
INFERNT_API int infernt_attention_decode(float* out, const float* qkv, float* k_cache,
                                         float* v_cache, int num_q_heads, int num_kv_heads,
                                         int head_dim, int max_seq_len, int position,
                                         float theta, int splits, void* workspace,
                                         void* stream);
/* No counterpart in the reference.  infernt_attention_decode without the workspace argument,
 * for callers that cannot allocate device memory for it: the kernel and its results are the
 * same, but the split partials and tickets live in a fixed 512 KiB static device array inside
 * this library, so the call allocates nothing (no cudaMalloc / cudaFree, no allocating
 * library routine).  Limits and rules:
 *  - a shape whose infernt_attention_workspace_bytes() exceeds 512 KiB is rejected with
 *    INFERNT_ERR_INVALID_ARGUMENT (lower `splits`);
 *  - the tickets in that array must be zero when a call starts: static storage starts
 *    zeroed and every completed call leaves them at zero;
 *  - there is one array per device: calls that overlap in time on one device (different
 *    streams, or different host threads without ordering) race on it and give wrong
 *    results.  Issue them on one stream, or order them;
 *  - the first call on each device looks up the array's address (cudaGetSymbolAddress);
 *    make that first call before any stream capture on the device. */
INFERNT_API int infernt_attention_decode_noalloc(float* out, const float* qkv, float* k_cache,
                                                 float* v_cache, int num_q_heads,
                                                 int num_kv_heads, int head_dim,
                                                 int max_seq_len, int position, float theta,
                                                 int splits, void* stream);
/* logits = W rmsnorm(x, norm_w); *out_token = argmax(logits) (llama_model.cpp:58-64 +
 * cuda/sampling.cu).  workspace: infernt_lm_head_workspace_bytes() bytes, zeroed once. */
INFERNT_API size_t infernt_lm_head_workspace_bytes(void);
INFERNT_API int infernt_rmsnorm_lm_head_argmax(float* logits, int* out_token, const void* W,
                                               int vocab_size, int in_features,
                                               int weight_dtype, const float* x,
                                               const float* norm_w, float eps,
                                               void* workspace, void* stream);
/* Batched projection on the tensor cores (CublasWrapper::gemm with M = batch,
 * gemm/cublas_wrapper.cu:21-40 as called by llama_layer.cpp:18-23 for an
 * activation batch [B, h]): for T tokens X [T][K] and row-major weights
 * W [N][K], both bf16, partials[s][t][n] = the FP32 sum over split s's share
 * of K of X[t][k] W[n][k]; the caller adds the `splits` partials (in order
 * for a deterministic result).  N a multiple of 128, K a multiple of 64,
 * 1 <= T <= 256, 1 <= splits <= K / 64, W and X 16-byte aligned.  err (or
 * NULL): bit 0 set by the device if a wait timed out. */
INFERNT_API int infernt_bgemm_bf16(const void* W, int N, int K, const void* X, int T,
                                   float* partials, int splits, unsigned* err, void* stream);
/* Prefill projection on the tensor cores (CublasWrapper::gemm with M = the
 * prompt tokens of a chunk, gemm/cublas_wrapper.cu:21-40; the reference
 * instead runs M = 1 per prompt token, src/engine.cpp:124-126): Y[t][n] =
 * the FP32 sum over k of X[t][k] W[n][k] for X [T][K] and W [N][K] bf16,
 * one accumulation over the whole K per element; Y rows ldy floats apart
 * (columns [0, N) written).  N a multiple of 128, K a multiple of 64,
 * T >= 1, ldy >= N, W and X 16-byte aligned.  err as infernt_bgemm_bf16. */
INFERNT_API int infernt_pgemm_bf16(const void* W, int N, int K, const void* X, int T, float* Y,
                                   int ldy, unsigned* err, void* stream);
/* The gate/up projection of a prompt chunk with SwiGLU in its epilogue
 * (llama_layer.cpp:61-66, cuda/activation.cu:7-9): W_gate_up [2 I][K] bf16
 * (gate rows, then up rows), act[t][i] = bf16(silu(g) u) for the FP32 sums
 * g = X[t] . W_gate[i], u = X[t] . W_up[i]; act rows ld_act elements apart.
 * I a multiple of 128; otherwise as infernt_pgemm_bf16. */
INFERNT_API int infernt_pgemm_swiglu_bf16(const void* W_gate_up, int I, int K, const void* X, int T,
                                          void* act, int ld_act, unsigned* err, void* stream);
/* Causal attention of a prompt chunk (cuda/attention.cu:9-42 and
 * cuda/softmax.cu:13-48 per query row): q [n_tokens][nq][D] bf16 with RoPE
 * applied, the sequence's caches [nkv][max_seq][D] bf16 holding positions
 * [0, start_pos + n_tokens); token t (position start_pos + t) of query head
 * h attends to positions [0, start_pos + t] of KV head h / (nq / nkv);
 * attn [n_tokens][nq][D] bf16.  Queries and probabilities enter the tensor
 * cores as bf16 (FP32 scores, softmax and sums), so each output is within
 * 2^-8 of the largest |V| of its head (bf16 probabilities, bf16 output).
 * D in {64, 128}; nq / nkv in {1, 2, 4, 8}; all pointers 16-byte aligned
 * device memory; asynchronous on `stream`.  tensor_cores != 0: the tcgen05
 * kernel (S and O in tensor memory; err, or NULL, gets bit 0 if one of its
 * bounded waits ran out); 0: the mma.sync kernel. */
INFERNT_API int infernt_prefill_attention(const void* q, const void* k_cache, const void* v_cache,
                                          int n_tokens, int start_pos, int nq, int nkv,
                                          int head_dim, int max_seq, void* attn, unsigned* err,
                                          int tensor_cores, void* stream);

/* ------------------------------------------------- the decode plan ---
 * One decoder of a LLaMA-family model over caller-owned weights and KV
 * cache (the state LlamaArchitecture::forward works on,
 * architectures/llama/llama_model.cpp:45-65).  The plan owns its scratch
 * activations (allocated once at creation: the zero-allocation decode
 * loop).  Execution modes:
 *   INFERNT_MODE_EAGER       5 kernels per layer + 1, launched per step;
 *   INFERNT_MODE_GRAPH       the same kernels replayed as one CUDA graph;
 *   INFERNT_MODE_PERSISTENT  one cooperative launch of the persistent decode
 *                            kernel per call (a whole chain of steps too);
 *                            falls back to GRAPH when the shapes do not allow
 *                            it (projection inputs not multiples of 512,
 *                            weights or caches not 16-byte aligned, head_dim
 *                            not a multiple of 4).                        */
enum { INFERNT_MODE_EAGER = 0, INFERNT_MODE_GRAPH = 1, INFERNT_MODE_PERSISTENT = 2 };
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
    int weight_dtype; /* INFERNT_DTYPE_F32 or INFERNT_DTYPE_BF16 */
} infernt_llama_config;

typedef struct infernt_plan infernt_plan;

/* weights: 3 + 9*num_layers device pointers in the order
 *   embedding [V,h], final_norm [h], lm_head [V,h], then per layer
 *   attn_norm [h], q [Nq*D,h], k [Nkv*D,h], v [Nkv*D,h], o [h,Nq*D], ffn_norm [h],
 *   gate [I,h], up [I,h], down [h,I]
 * (include/weights.h:8-25).  Norm weights and the embedding are always float; the seven
 * projection matrices and lm_head have weight_dtype.  k_cache / v_cache: num_layers device
 * pointers to float [Nkv, max_seq_len, D] (include/kv_cache.h:7-15). */
INFERNT_API int infernt_plan_create(const infernt_llama_config* cfg, const void* const* weights,
                                    float* const* k_cache, float* const* v_cache, int mode,
                                    infernt_plan** out);
INFERNT_API int infernt_plan_destroy(infernt_plan* plan);
/* The mode the plan runs in (PERSISTENT may have fallen back to GRAPH). */
INFERNT_API int infernt_plan_mode(const infernt_plan* plan);
/* ModelArchitecture::forward (include/architecture.h:15-19): input_embedding [h] at
 * `position`; writes logits [V] (NULL: the plan's own buffer) and the greedy token
 * (read it with infernt_plan_read_token). */
INFERNT_API int infernt_plan_forward(infernt_plan* plan, const float* input_embedding,
                                     int position, float* logits, void* stream);
/* InferenceEngine::forward_token's device work (src/engine.cpp:53-66): embedding of
 * `token` + forward + argmax, asynchronously. */
INFERNT_API int infernt_plan_decode(infernt_plan* plan, int token, int position, float* logits,
                                    void* stream);
/* `steps` decode steps chained on the device: step s consumes the token step s-1
 * produced, starting from (token, position).  tokens_dev (device int[steps], may be NULL)
 * receives each produced token.  No host round trip between steps. */
INFERNT_API int infernt_plan_decode_chain(infernt_plan* plan, int token, int position,
                                          int steps, int* tokens_dev, void* stream);
/* Synchronises `stream`, checks the kernels' error word, copies the last greedy token. */
INFERNT_API int infernt_plan_read_token(infernt_plan* plan, int* token_host, void* stream);
/* Device pointer of the plan's logits buffer [V]. */
INFERNT_API float* infernt_plan_logits(infernt_plan* plan);
/* Number of kernels one decode step launches (for launch accounting). */
INFERNT_API int infernt_plan_kernels_per_step(const infernt_plan* plan);
/* Phase timeline of the persistent decode kernel.  Phases per step:
 * 5 per layer (qkv, attention, o, gate/up, down) + the LM head.  With a
 * device buffer of infernt_plan_trace_entries(plan, steps) uint64 set, the
 * following launches record, for every CTA per (step, phase): [phase start,
 * input loaded, work done, grid barrier passed, producer issued the phase's
 * last slot] as %globaltimer nanoseconds, then the SM cycles the first
 * consumer thread waited for weight slots and the SM cycles the producer
 * waited for free slots; layout [cta][step][phase][7] over
 * infernt_persistent_ctas() CTAs.  In attention phases a CTA with an item
 * records instead: field 1 its inputs landed, 4 its partial computed, 5 its
 * split ticket taken, 6 the merge done (when it merged).  NULL turns it off.
 * PERSISTENT mode only. */
INFERNT_API size_t infernt_plan_trace_entries(const infernt_plan* plan, int steps);
INFERNT_API int infernt_plan_set_trace(infernt_plan* plan, unsigned long long* trace_dev);
/* Token choice of the following steps: temperature <= 0 greedy (the
 * default), otherwise the LM-head phase of the persistent decode kernel
 * draws the token from softmax(logits / temperature) by Gumbel-max (the
 * argmax of logit / T + g_i, g_i = -ln(-ln u_i), u_i hashed from (seed, the
 * step's position, i)): the token infernt_sample_tokens(logits, ..., seed,
 * counter = position) draws from the same logits.  Logits stay the raw
 * values.  Returns INFERNT_ERR_UNSUPPORTED for T > 0 on a plan that does
 * not run the persistent kernel.  No counterpart in the reference (its
 * sampler runs on the host, src/engine.cpp:78-104). */
INFERNT_API int infernt_plan_set_sampling(infernt_plan* plan, float temperature, uint64_t seed);
/* CTAs of the persistent decode kernel on the current device (one per SM). */
INFERNT_API int infernt_persistent_ctas(void);

/* ------------------------------------------------ batched decode ---
 * T sequences decoding together, one token each per step (the reference's
 * LlamaArchitecture keeps [B, h] activations, architectures/llama/
 * llama_model.cpp:8-43, but decodes B = 1): bf16 projection weights on the
 * tensor cores (infernt_bgemm_bf16), activations rounded to bf16 where they
 * enter a projection, per-sequence bf16 KV caches [N_kv, max_seq, D] per
 * layer, FP32 residual stream, norms and attention arithmetic.  Seeded
 * synthetic weights as infernt_engine_create_seeded; hidden, heads x
 * head_dim, intermediate and vocabulary multiples of 128, head_dim 64 or
 * 128, query groups up to 16, 1 <= batch <= 256.  attn_splits: KV splits per
 * (sequence, KV head) of the attention, 0 for automatic. */
typedef struct infernt_batch_engine infernt_batch_engine;
INFERNT_API int infernt_batch_engine_create_seeded(const infernt_llama_config* cfg, int batch,
                                                   uint64_t seed, float std_dev, int attn_splits,
                                                   infernt_batch_engine** out);
/* One rank of a tensor-parallel batched decoder over `world` GPUs, one
 * process per GPU (the reference decodes on one GPU; this splits
 * LlamaArchitecture::forward, architectures/llama/llama_model.cpp:45-65,
 * Megatron-style): rank r holds query heads [r Nq/world, ..), KV heads
 * [r Nkv/world, ..) with their caches, gate/up rows and down columns
 * [r I/world, ..), the matching O columns and LM-head vocabulary rows
 * [V r/world, V (r+1)/world), each the window of the seeded matrices a
 * single-GPU engine of the same seed holds.  Per layer the O and down
 * partial sums are all-reduced over the ranks (ncclAllReduce, FP32 [batch,
 * hidden]) and the greedy token is agreed through an all-gather of every
 * rank's (value, id) candidates (the lowest id wins among equal values);
 * every rank then holds the same tokens.  nccl_id: the 128-byte
 * ncclUniqueId from infernt_nccl_unique_id on one rank, passed to all (NULL
 * for world = 1).  All ranks create, step and destroy together; the
 * process's libnccl.so.2 is used (the one already loaded, else the system
 * one).  Nkv, and the per-rank Q|K|V rows, O and down K must split into
 * tensor-core tiles (rows multiples of 128, K multiples of 64).  Prefill is
 * single-rank only. */
INFERNT_API int infernt_batch_engine_create_tp(const infernt_llama_config* cfg, int batch, uint64_t seed,
                                               float std_dev, int attn_splits, int rank, int world,
                                               const void* nccl_id, infernt_batch_engine** out);
/* A new ncclUniqueId (n >= 128 bytes) for infernt_batch_engine_create_tp. */
INFERNT_API int infernt_nccl_unique_id(void* out, size_t n);
/* This rank's vocabulary rows [*v0, *v0 + *vl) (the whole vocabulary on one
 * rank). */
INFERNT_API int infernt_batch_engine_vocab_range(infernt_batch_engine* e, int* v0, int* vl);
INFERNT_API int infernt_batch_engine_destroy(infernt_batch_engine* e);
/* Rows [0, n_pos) of sequence seq's KV caches from the seeded KV streams
 * (the values infernt_fill_kv writes), rounded to bf16. */
INFERNT_API int infernt_batch_engine_fill_kv(infernt_batch_engine* e, int seq, uint64_t seed, int n_pos,
                                             float std_dev);
/* One step: tokens[t] at positions[t] for every sequence; next_tokens[t]
 * the greedy tokens (host arrays of `batch` ints; synchronous). */
INFERNT_API int infernt_batch_engine_step(infernt_batch_engine* e, const int* tokens,
                                          const int* positions, int* next_tokens);
/* `steps` chained steps on the device from (tokens, positions); tokens_out
 * [steps][batch] (or NULL); *ms the device time of the steps (or NULL). */
INFERNT_API int infernt_batch_engine_decode(infernt_batch_engine* e, const int* tokens,
                                            const int* positions, int steps, int* tokens_out,
                                            float* ms);
/* The last step's logits [batch][vl] of this rank's vocabulary rows
 * (infernt_batch_engine_vocab_range; n = batch x vl floats). */
INFERNT_API int infernt_batch_engine_logits(infernt_batch_engine* e, float* logits_host, size_t n);
/* Prompt prefill of sequence seq: tokens[0, n_tokens) (host array) at
 * positions [start_pos, start_pos + n_tokens), in chunks of `chunk` tokens
 * (0: 4096; at most 16384) that pass through every layer at once, replacing the
 * reference's sequential single-token forwards (src/engine.cpp:124-126,
 * the same arithmetic per token: architectures/llama/llama_layer.cpp:11-72).
 * The projections run as dense tensor-core GEMMs (infernt_pgemm_bf16), the
 * attention causally over the sequence's cache (infernt_prefill_attention);
 * the sequence's K/V rows of every prompt position are written.  Then the LM
 * head and greedy argmax of the last prompt token: *next_token (or NULL),
 * its logits into logits_host [vocab] (or NULL), and *ms the device time
 * of the prefill (or NULL).  Synchronous.  The first call (and a later call
 * with a larger chunk) allocates the prefill scratch: about chunk x (hidden
 * x 10 + max(Q|K|V rows, 2 x intermediate) x 4 + intermediate x 2) bytes.
 * Tensor-parallel engines (infernt_batch_engine_create_tp): every rank calls
 * it with the same arguments; each runs its shards of the heads,
 * intermediate rows and vocabulary, ncclAllReduce sums the O and down
 * projections' partial rows of a chunk, every rank returns the same token,
 * and logits_host receives this rank's vocabulary rows
 * (infernt_batch_engine_vocab_range) at its start. */
INFERNT_API int infernt_batch_engine_prefill(infernt_batch_engine* e, int seq, const int* tokens,
                                             int n_tokens, int start_pos, int chunk, int* next_token,
                                             float* logits_host, float* ms);
/* Rows [0, n_pos) of sequence seq's K and V caches of one layer into host
 * arrays [nkv][n_pos][head_dim] of bf16 bits (uint16). */
INFERNT_API int infernt_batch_engine_read_kv(infernt_batch_engine* e, int seq, int layer, int n_pos,
                                             void* k_host, void* v_host);
/* Token choice of the following steps (and of prefill's first token):
 * temperature 0 greedy (the default; InferenceEngine's temperature <= 0
 * path), otherwise a draw from softmax(logits / temperature) per sequence
 * (src/engine.cpp:78-104 samples that distribution on the host) by
 * Gumbel-max inside the argmax kernels: the token with the largest logit /
 * T + g_i, g_i = -ln(-ln u_i), u_i hashed from (seed, the sequence's
 * position, i) as infernt_sample_tokens(..., seed, counter = position)
 * draws it.  Reproducible per seed; not the reference's mt19937 sequence.
 * The step graph is captured again at the next step. */
INFERNT_API int infernt_batch_engine_set_sampling(infernt_batch_engine* e, float temperature,
                                                  uint64_t seed);
/* How a tensor-parallel batched engine adds the ranks' O and down sums:
 * INFERNT_TP_EXCHANGE_PEER (the default) pushes each rank's sums into every
 * rank's exchange region over NVLink (CUDA IPC mappings made at creation)
 * as tagged words that the residual + RMSNorm kernel of every rank adds in
 * rank order (no NCCL call on the data path; waits bounded, reported as
 * INFERNT_ERR_DEVICE); INFERNT_TP_EXCHANGE_NCCL runs ncclAllReduce (the
 * baseline).  Every rank must use the same mode.  No counterpart in the
 * reference. */
enum { INFERNT_TP_EXCHANGE_PEER = 1, INFERNT_TP_EXCHANGE_NCCL = 0 };
INFERNT_API int infernt_batch_engine_set_tp_exchange(infernt_batch_engine* e, int mode);
/* K splits of the Q|K|V, O, gate|up, down and LM-head projections and the
 * attention's KV splits (6 ints). */
INFERNT_API int infernt_batch_engine_splits(infernt_batch_engine* e, int* out);
/* Attention work split: `splits` KV splits per (sequence, KV head), each at
 * least min_chunk positions, and `stages` copy stages per warp (2 to 4 at
 * head_dim 64, 2 or 3 at 128).  Results do not depend on these; the step
 * graph is captured again at the next step. */
INFERNT_API int infernt_batch_engine_set_attention(infernt_batch_engine* e, int splits, int min_chunk,
                                                   int stages);

/* ------------------------------------------ paged KV, continuous batching ---
 * Not in the reference (its README lists paged KV and continuous batching as
 * future work; it keeps one KVCache [N_kv, max_seq, D] per layer for one
 * sequence, include/kv_cache.h:7-15).
 *
 * A batched engine whose caches are pools of pages: per layer K and V pools
 * [num_pages][N_kv][page_size][head_dim] bf16, and a block table [batch]
 * [max_pages] (max_pages = ceil(max_seq_len / page_size)): position p of
 * sequence t lives in page table[t][p / page_size] at row p % page_size.
 * Slots whose position is -1 in a step are empty (not read, not written,
 * their position stays -1).  Everything else as infernt_batch_engine_create_
 * seeded, with query groups of at most 8 heads.  Prefill runs on contiguous
 * staging caches ([N_kv][max_seq_len][head_dim] per layer, allocated by the
 * first prefill) and copies the written rows into the pages. */
INFERNT_API int infernt_batch_engine_create_paged(const infernt_llama_config* cfg, int batch, int page_size,
                                                  int num_pages, uint64_t seed, float std_dev,
                                                  int attn_splits, infernt_batch_engine** out);
/* Pages of sequence seq: pages[0, n_pages) for its positions [0, n_pages x
 * page_size); the rest of its row is cleared.  Each in [0, num_pages); the
 * caller keeps live sequences' pages disjoint.  A step, prefill or fill_kv
 * needs pages for every position it touches (checked on the host). */
INFERNT_API int infernt_batch_engine_set_pages(infernt_batch_engine* e, int seq, const int* pages,
                                               int n_pages);
/* page_size, num_pages and max_pages per sequence (all 0: contiguous). */
INFERNT_API int infernt_batch_engine_paging(infernt_batch_engine* e, int* page_size, int* num_pages,
                                            int* max_pages);
/* Per-sequence sampling salts (`batch` values, e.g. request ids; NULL: none):
 * temperature draws of sequence t are keyed by (infernt_stream_key(seed,
 * salts[t]), position), so sequences at one position draw independently. */
INFERNT_API int infernt_batch_engine_set_salts(infernt_batch_engine* e, const uint64_t* salts);

/* Iteration-level scheduler over `slots` sequence slots and a pool of
 * num_pages pages of page_size positions (host logic, no GPU).  Requests
 * (prompt, max_new_tokens, eos) queue first-come first-served; a request is
 * admitted when a slot is free and the pool holds pages for its known tokens
 * plus the next position; each admitted request is prefilled once, then
 * takes one position per step in the batched decode beside the others.  A
 * running request that needs a page when the pool is empty preempts the
 * most recently admitted request (its pages are freed; it goes back to the
 * head of the queue and is prefilled again later with its prompt and the
 * tokens generated so far: recomputation).  A request finishes after
 * max_new_tokens tokens, or at the eos token (included). */
typedef struct infernt_scheduler infernt_scheduler;
typedef struct infernt_sched_plan {
    int n_prefill;              /* requests to prefill this step */
    const int* prefill_slot;    /* [n_prefill] their slots */
    const int* prefill_offset;  /* [n_prefill] start of each one's tokens in prefill_tokens */
    const int* prefill_len;     /* [n_prefill] tokens to prefill (positions [0, len)) */
    const int* prefill_tokens;
    int n_decode;               /* slots in this step's batched decode */
    const int* tokens;          /* [slots] token per slot (0 where empty) */
    const int* positions;       /* [slots] position per slot, -1: not decoding this step */
    int n_changed;              /* slots whose pages changed since the last plan */
    const int* changed_slot;    /* [n_changed] */
    const int* pages;           /* [slots][max_pages] page table, -1 past a slot's pages */
    const int* n_pages;         /* [slots] pages per slot */
    int max_pages;
    int n_preempted;            /* requests this plan preempted */
} infernt_sched_plan;
typedef struct infernt_sched_stats {
    int waiting, running, finished, free_pages;
    long long steps, preemptions, prefill_tokens, decode_tokens;
} infernt_sched_stats;
enum {
    INFERNT_REQUEST_WAITING = 0,
    INFERNT_REQUEST_RUNNING = 1,
    INFERNT_REQUEST_FINISHED = 2,
    INFERNT_REQUEST_CANCELLED = 3
};
INFERNT_API int infernt_scheduler_create(int slots, int page_size, int num_pages, int max_seq_len,
                                         infernt_scheduler** out);
INFERNT_API int infernt_scheduler_destroy(infernt_scheduler* s);
/* Queue a request: prompt[0, n) with 1 <= n, max_new_tokens >= 1, n +
 * max_new_tokens <= max_seq_len and pages for them within the pool; eos < 0
 * for none.  *id: the request's id (increasing from 1). */
INFERNT_API int infernt_scheduler_submit(infernt_scheduler* s, const int* prompt, int n, int max_new_tokens,
                                         int eos, int64_t* id);
/* Drop a waiting or running request (its pages and slot are freed). */
INFERNT_API int infernt_scheduler_cancel(infernt_scheduler* s, int64_t id);
/* The next step's work: preemptions, page growth and admissions applied.
 * The arrays stay valid until the next plan or commit. */
INFERNT_API int infernt_scheduler_plan(infernt_scheduler* s, infernt_sched_plan* plan);
/* The step's results: prefill_next [n_prefill] the token after each prefill,
 * decode_next [slots] the token after each decoding slot (others ignored). */
INFERNT_API int infernt_scheduler_commit(infernt_scheduler* s, const int* prefill_next, const int* decode_next);
/* Request id: *state (INFERNT_REQUEST_*), *n generated tokens so far, the
 * first min(cap, *n) of them into tokens (may be NULL when cap is 0),
 * *preemptions how often it was preempted (or NULL). */
INFERNT_API int infernt_scheduler_result(infernt_scheduler* s, int64_t id, int* tokens, int cap, int* n,
                                         int* state, int* preemptions);
/* Forget a finished or cancelled request's record. */
INFERNT_API int infernt_scheduler_release(infernt_scheduler* s, int64_t id);
INFERNT_API int infernt_scheduler_stats(infernt_scheduler* s, infernt_sched_stats* out);

/* Continuous-batching server: the scheduler above driving a paged batched
 * engine of `slots` sequences (seeded weights as infernt_batch_engine_create_
 * paged).  A step: the plan's page tables into the engine, each admitted
 * request's prefill, one batched decode step of the running requests, the
 * results into the scheduler. */
typedef struct infernt_server infernt_server;
INFERNT_API int infernt_server_create_seeded(const infernt_llama_config* cfg, int slots, int page_size,
                                             int num_pages, uint64_t seed, float std_dev,
                                             infernt_server** out);
INFERNT_API int infernt_server_destroy(infernt_server* srv);
INFERNT_API int infernt_server_submit(infernt_server* srv, const int* prompt, int n, int max_new_tokens,
                                      int eos, int64_t* id);
/* One step; *n_finished (or NULL) the requests it finished. */
INFERNT_API int infernt_server_step(infernt_server* srv, int* n_finished);
/* Steps until no request waits or runs; *ms (or NULL) the host time. */
INFERNT_API int infernt_server_run(infernt_server* srv, double* ms);
INFERNT_API int infernt_server_result(infernt_server* srv, int64_t id, int* tokens, int cap, int* n, int* state,
                                      int* preemptions);
INFERNT_API int infernt_server_stats(infernt_server* srv, infernt_sched_stats* out);
/* Temperature sampling of the following steps (0: greedy), keyed per
 * request: draws of request r at position p use (infernt_stream_key(seed,
 * r), p). */
INFERNT_API int infernt_server_set_sampling(infernt_server* srv, float temperature, uint64_t seed);
/* The server's engine (logits of the last decode step, attention settings);
 * owned by the server. */
INFERNT_API int infernt_server_engine(infernt_server* srv, infernt_batch_engine** out);

/* Attention of T decoding sequences over bf16 caches (the batched engine's
 * kernels; cuda/attention.cu:9-42 per sequence and query head): q [T][nq][D]
 * FP32 (RoPE applied), caches [T][nkv][max_seq][D] bf16, sequence t
 * attends to positions [0, positions[t]]; attn [T][nq][D] bf16 (rounded to
 * nearest even) and, when attn_f32 is not NULL, the FP32 values.  splits
 * KV splits per (t, KV head) of at least min_chunk positions, `stages` copy
 * stages (2 to 4 at D = 64, 2 or 3 at 128; ignored for 16 query heads per
 * KV head); partials holds T x nkv x splits x (nq / nkv) x (D + 2) floats.
 * D in {64, 128}; nq / nkv from 1 to 8, or 16 at D = 64.  positions[t] in
 * [0, max_seq) (a sequence outside is not read; its output is undefined).
 * Device pointers; asynchronous on `stream`. */
INFERNT_API int infernt_batch_attention(const float* q, const void* k_cache, const void* v_cache,
                                        const int* positions, int T, int nq, int nkv, int head_dim,
                                        int max_seq, int splits, int min_chunk, int stages,
                                        float* partials, void* attn, float* attn_f32, void* stream);

/* ----------------------------------------- tensor parallelism ---
 * The 8B-class configuration decoded by tp_size GPUs, one process per GPU
 * (the reference has a single-GPU engine only; this extends
 * LlamaArchitecture::forward, architectures/llama/llama_model.cpp:45-65,
 * Megatron-style).  Rank t of T holds
 *   q/k/v: the rows of its Nq/T query heads and Nkv/T KV heads,
 *   o:     the columns of its query heads, [h, Nq*D/T],
 *   gate/up: rows [t*I/T, (t+1)*I/T),
 *   down:  the matching columns, [h, Ip] with Ip = I/T rounded up to 512 and
 *          the extra columns zero,
 *   lm_head: vocabulary rows [V*t/T, V*(t+1)/T), the embedding in full,
 * and its KV heads' caches [Nkv/T, max_seq, D].  The O and down products are
 * all-reduced inside the persistent decode kernel: each rank writes its
 * partial rows into every rank's exchange region over NVLink (peer memory
 * mapped by CUDA IPC) as tagged words, and the next phase polls them and
 * adds the partials in rank order, so every rank holds bit-identical
 * activations.  The greedy token is agreed the same way.  Every rank must
 * run the same calls in the same order.
 *
 * infernt_tp_shard_dims: dims[6] = {Nq/T, Nkv/T, I/T, Ip, first vocabulary
 * row, vocabulary rows} of rank t.  infernt_plan_create_tp: `cfg` is the
 * whole model's; weights/caches are the rank's shards in the order of
 * infernt_plan_create.  Then exchange the ranks' 64-byte handles
 * (infernt_plan_xchg_handle) by any host channel and pass all of them, in
 * rank order, to infernt_plan_set_peers before the first decode call.
 * Decode calls (forward, decode, decode_chain) then work as for a single
 * GPU; logits hold the rank's vocabulary rows. */
#define INFERNT_IPC_HANDLE_BYTES 64
INFERNT_API int infernt_tp_shard_dims(const infernt_llama_config* cfg, int tp_rank, int tp_size,
                                      int* dims);
INFERNT_API int infernt_plan_create_tp(const infernt_llama_config* cfg, const void* const* weights,
                                       float* const* k_cache, float* const* v_cache, int tp_rank,
                                       int tp_size, infernt_plan** out);
INFERNT_API int infernt_plan_xchg_handle(infernt_plan* plan, void* handle_out);
INFERNT_API int infernt_plan_set_peers(infernt_plan* plan, const void* handles);
/* Bytes of a tensor-parallel plan's exchange region. */
INFERNT_API int infernt_plan_xchg_bytes(const infernt_plan* plan, size_t* bytes);
/* In place of infernt_plan_set_peers: every rank's exchange region as a
 * device pointer this process can read and write (regions[tp_rank] must be
 * the plan's own), for callers that map peer memory themselves (a symmetric
 * heap, a virtual-memory mapping).  Each region holds
 * infernt_plan_xchg_bytes bytes. */
INFERNT_API int infernt_plan_set_peer_regions(infernt_plan* plan, void* const* regions);
/* The own exchange region (device pointer). */
INFERNT_API void* infernt_plan_xchg_region(infernt_plan* plan);
/* Time budget of every wait inside the persistent decode kernel (ring
 * slots, tagged activations, peers' partials, the step hand-off), in
 * microseconds at the maximum SM clock; default 2 000 000 (2 s).  A wait
 * that runs out sets the wait-timeout bit of the error word, every CTA of
 * the launch returns, and the next synchronising call reports
 * INFERNT_ERR_DEVICE; the plan stays usable. */
INFERNT_API int infernt_plan_set_wait_budget(infernt_plan* plan, long long microseconds);
/* Weight-stream slots (16 KB each) the persistent decode kernel keeps in
 * flight per SM: the producer issues a slot's bulk copy only when the slot
 * `slots` earlier has landed.  Landed slots still fill the whole ring ahead
 * of the consumers; the limit only bounds the copies queued in the memory
 * system, behind which the reads of tagged activations at a phase boundary
 * wait.  0 or more than the ring: no limit beyond the ring.  Plans of the
 * other modes accept and ignore it.  No reference counterpart (the
 * reference streams its weights through cuBLAS). */
INFERNT_API int infernt_plan_set_stream_depth(infernt_plan* plan, int slots);
/* The in-flight limit and the ring size in slots. */
INFERNT_API int infernt_plan_stream_depth(const infernt_plan* plan, int* slots, int* ring_slots);

/* One rank of a tensor-parallel decoder with seeded synthetic weights: the
 * rank's shards are windows of the matrices infernt_engine_create_seeded
 * generates for the same seed (norms 1.0), its KV caches start at zero.
 * Exchange handles and set peers as for the plan; forward_token runs one
 * greedy step (every rank returns the same token); decode_chain runs
 * `steps` chained steps and reports their device time (CUDA events);
 * logits copies the rank's vocabulary rows (dims: infernt_tp_shard_dims). */
typedef struct infernt_tp_engine infernt_tp_engine;
INFERNT_API int infernt_tp_engine_create_seeded(const infernt_llama_config* cfg, uint64_t seed,
                                                float std_dev, int tp_rank, int tp_size,
                                                infernt_tp_engine** out);
INFERNT_API int infernt_tp_engine_destroy(infernt_tp_engine* e);
INFERNT_API int infernt_tp_engine_xchg_handle(infernt_tp_engine* e, void* handle_out);
INFERNT_API int infernt_tp_engine_set_peers(infernt_tp_engine* e, const void* handles);
INFERNT_API int infernt_tp_engine_forward_token(infernt_tp_engine* e, int token, int position,
                                                int* next_token);
INFERNT_API int infernt_tp_engine_decode_chain(infernt_tp_engine* e, int token, int position,
                                               int steps, int* tokens_host, float* ms);
INFERNT_API int infernt_tp_engine_logits(infernt_tp_engine* e, float* logits_host, int n);
INFERNT_API int infernt_tp_engine_dims(infernt_tp_engine* e, int* dims);
/* The engine's tensor-parallel plan (owned by the engine). */
INFERNT_API int infernt_tp_engine_plan(infernt_tp_engine* e, infernt_plan** plan);
/* decode_chain with the phase timeline of infernt_plan_set_trace recorded into host_out
 * (infernt_plan_trace_entries entries). */
INFERNT_API int infernt_tp_engine_trace_chain(infernt_tp_engine* e, int token, int position,
                                              int steps, unsigned long long* host_out, size_t n);

/* ------------------------------------------------ synthetic weights ---
 * Fill device memory with the seeded values of include/infernt_seed.h
 * (bit-identical to the host generator).  dtype selects float or bf16
 * output; bf16 values are the float values rounded to nearest even.     */
INFERNT_API int infernt_fill_normal(void* dst, size_t n, int dtype, uint64_t seed,
                                    uint64_t stream_id, float std_dev, void* stream);
/* dst [rows][ld_dst] = rows row0.. and columns col0..col0+cols-1 of the seeded matrix with
 * src_ld columns that infernt_fill_normal(seed, stream_id) would produce (its element
 * (r, c) has index r*src_ld + c); columns cols..ld_dst-1 are zero.  For weight shards. */
INFERNT_API int infernt_fill_normal_window(void* dst, int rows, int cols, int ld_dst,
                                           uint64_t src_ld, uint64_t row0, uint64_t col0,
                                           int dtype, uint64_t seed, uint64_t stream_id,
                                           float std_dev, void* stream);
INFERNT_API int infernt_fill_const(float* dst, size_t n, float value, void* stream);
/* Host: n seeded token ids uniform in [lo, hi) (the prompt stream of
 * include/infernt_seed.h; the synthetic prompts of the benchmarks). */
INFERNT_API int infernt_fill_prompt(int* out_host, int n, uint64_t seed, int lo, int hi);
/* KV prefill: rows [0, n_pos) of every layer's K and V cache get N(0, std) from the
 * KV streams (element (l, h, p, d) = index ((l*Nkv + h) * 2^20 + p) * D + d). */
INFERNT_API int infernt_fill_kv(float* const* k_cache, float* const* v_cache, int num_layers,
                                int num_kv_heads, int max_seq_len, int head_dim, int n_pos,
                                uint64_t seed, float std_dev, void* stream);

/* --------------------------------------------------- the engine ---
 * C entry points over the C++ InferenceEngine (include/engine.h), for
 * hosts that cannot call C++ (ctypes, cgo, JNI).  The engine owns seeded
 * synthetic weights (weights ~ N(0, std), norms 1.0).                  */
typedef struct infernt_engine infernt_engine;
INFERNT_API int infernt_engine_create_seeded(const infernt_llama_config* cfg, uint64_t seed,
                                             float std_dev, infernt_engine** out);
INFERNT_API int infernt_engine_destroy(infernt_engine* e);
/* Decode execution mode (INFERNT_MODE_*) for the following steps; the default is
 * PERSISTENT, or the INFERNT_DECODE_MODE environment variable (eager | graph |
 * persistent) when set.  infernt_engine_mode reports the mode in use (after a step). */
INFERNT_API int infernt_engine_set_mode(infernt_engine* e, int mode);
INFERNT_API int infernt_engine_mode(infernt_engine* e, int* mode);
/* A device-chained decode of `steps` steps with the phase timeline recorded
 * (infernt_plan_set_trace layout) into host_out (n entries). */
INFERNT_API int infernt_engine_trace_chain(infernt_engine* e, int token, int position, int steps,
                                           unsigned long long* host_out, size_t n);
/* KVCache::reset (src/kv_cache.cpp:22-30). */
INFERNT_API int infernt_engine_reset(infernt_engine* e);
/* InferenceEngine::forward_token (src/engine.cpp:53-66): returns the greedy next token in
 * *next_token (host). */
INFERNT_API int infernt_engine_forward_token(infernt_engine* e, int token, int position,
                                             int* next_token);
/* InferenceEngine::load_model(model_dir) (src/engine.cpp:14-31): config.json,
 * model.bin (INFT v1) and tokenizer.bin of a converted checkpoint;
 * weight_dtype INFERNT_DTYPE_F32 / _BF16 overrides config.json's (negative:
 * keep it). */
INFERNT_API int infernt_engine_load_model(const char* model_dir, int weight_dtype, infernt_engine** out);
/* on != 0 (the default, seed 1337): the engine's sample_next_token(T > 0)
 * draws on the GPU by Gumbel-max as infernt_sample_tokens(..., seed, counter
 * = position | k << 32) for its k-th draw since the last step (k = 0: the
 * draw a step at that temperature makes inside the kernel); on == 0
 * restores the reference's host mt19937 sampler.  No counterpart in the
 * reference. */
INFERNT_API int infernt_engine_set_device_sampling(infernt_engine* e, int on, uint64_t seed);
/* InferenceEngine::set_step_temperature: following steps (forward_token,
 * decode_chain) draw their token at this temperature inside the persistent
 * decode kernel's LM-head phase (0: greedy).  Without the persistent kernel
 * or with host sampling the steps stay greedy.  No counterpart in the
 * reference. */
INFERNT_API int infernt_engine_set_step_temperature(infernt_engine* e, float temperature);
/* InferenceEngine::sample_next_token (src/engine.cpp:68-105). */
INFERNT_API int infernt_engine_sample_next_token(infernt_engine* e, float temperature,
                                                 int* token);
/* Copies the last step's logits [V] to host memory. */
INFERNT_API int infernt_engine_logits(infernt_engine* e, float* logits_host);
/* Prefill of KV rows [0, n_pos) with seeded values (benchmark set-up). */
INFERNT_API int infernt_engine_fill_kv(infernt_engine* e, uint64_t seed, int n_pos,
                                       float std_dev);
/* Device-chained decode loop (as infernt_plan_decode_chain) on the engine's stream; writes
 * `steps` tokens to tokens_host and the device time of the loop (CUDA events) to *ms. */
INFERNT_API int infernt_engine_decode_chain(infernt_engine* e, int token, int position,
                                            int steps, int* tokens_host, float* ms);
/* Device pointers of the engine's weights (3 + 9L, order of infernt_plan_create) and
 * KV cache (L each), for tests that drive the per-op entry points. */
INFERNT_API int infernt_engine_weight_ptrs(infernt_engine* e, const void** ptrs, int n);
INFERNT_API int infernt_engine_kv_ptrs(infernt_engine* e, float** k, float** v, int n);

/* ------------------------------------------------ temperature sampling ---
 * InferenceEngine::sample_next_token(temperature) samples softmax(logits / T)
 * on the host (src/engine.cpp:78-104, mt19937 seeded 1337).  This draws the
 * same distribution on the GPU by the Gumbel-max method: row r's token is
 * argmax_i (logits[r][i] / T + g_i), g_i = -ln(-ln u_i), u_i a 24-bit
 * uniform in (0, 1) hashed from (seed, counter + r, i) — reproducible per
 * (seed, counter), not the reference's mt19937 sequence.  T <= 0: greedy
 * argmax.  Ties go to the lowest index; NaN never wins.  logits rows are ld
 * floats apart (ld = 0: every row samples the same logits); out_tokens
 * [rows] device ints; workspace: infernt_sample_workspace_bytes(rows) bytes
 * of device memory, zeroed once before the first call (calls leave it
 * zeroed; calls that share it must not overlap).  Asynchronous. */
INFERNT_API size_t infernt_sample_workspace_bytes(int rows);
INFERNT_API int infernt_sample_tokens(const float* logits, long long ld, int rows, int vocab_size,
                                      float temperature, uint64_t seed, uint64_t counter,
                                      int* out_tokens, void* workspace, void* stream);

/* ------------------------------------------------ INFT v1 checkpoints ---
 * The reference's CheckpointLoader (include/checkpoint_loader.h:7-14,
 * loader/checkpoint_loader.cpp:42-161; the C++ class is in
 * include/checkpoint_loader.h).  config.json: the keys the reference reads
 * (with its defaults), optional head_dim and weight_dtype ("bf16" / "fp32"). */
INFERNT_API int infernt_checkpoint_read_config(const char* config_json, infernt_llama_config* out);
/* model.bin (magic 0x494E4654, version 1, FP32 payloads) for cfg: every
 * tensor in its own buffer, device 0 = host memory, 1 = the current CUDA
 * device; norms and embedding FP32, projections and lm_head in
 * cfg->weight_dtype (bf16 rounded to nearest even).  A missing lm_head is a
 * copy of the embedding (as the reference); a bad magic or version, a
 * truncated file, an element count that does not match cfg or a missing
 * tensor is INFERNT_ERR_INVALID_ARGUMENT (the reference does not check). */
typedef struct infernt_checkpoint infernt_checkpoint;
INFERNT_API int infernt_checkpoint_load(const char* model_bin, const infernt_llama_config* cfg, int device,
                                        infernt_checkpoint** out);
/* The 3 + 9 num_layers buffers in the order of infernt_plan_create. */
INFERNT_API int infernt_checkpoint_weights(const infernt_checkpoint* ck, const void** out, int n);
INFERNT_API int infernt_checkpoint_free(infernt_checkpoint* ck);

#ifdef __cplusplus
}
#endif
#endif /* INFERNT_CAPI_H */
