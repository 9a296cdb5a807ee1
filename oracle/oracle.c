/*
 * oracle.c — CPU oracle for INFERNT's decode step (TEST INFRASTRUCTURE;
 * only the tests, the smoke check and the benchmark's CPU-baseline leg use
 * it).  Each function cites the reference source it restates; paths are
 * relative to the INFERNT repository.
 */
#include "oracle.h"
#include "../include/infernt_seed.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static int g_threads = 1;

void oracle_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

/* Batched-decode variant (infernt_batch_engine_*): activations rounded to
 * bf16 where they enter a projection (normed inputs, attention output,
 * SiLU*up) and K/V rows rounded to bf16 before they enter the cache. */
static int g_act_bf16 = 0;
void oracle_set_act_bf16(int on) { g_act_bf16 = on != 0; }

static void round_vec(float* x, int n) {
    if (!g_act_bf16) return;
    for (int i = 0; i < n; ++i) x[i] = infernt_round_bf16(x[i]);
}
int oracle_get_threads(void) { return g_threads; }

/* ------------------------------------------------------------------ */
/* synthetic inputs                                                    */
/* ------------------------------------------------------------------ */

typedef struct {
    float* out;
    size_t begin, end;
    uint64_t key;
    uint64_t start;
    float std_dev;
    int round_bf16;
} fill_job;

static void* fill_worker(void* arg) {
    fill_job* j = (fill_job*)arg;
    for (size_t i = j->begin; i < j->end; ++i) {
        float v = infernt_normal_std(j->key, j->start + (uint64_t)i, j->std_dev);
        j->out[i] = j->round_bf16 ? infernt_round_bf16(v) : v;
    }
    return NULL;
}

void oracle_fill_normal(float* out, size_t n, uint64_t seed, uint64_t stream,
                        float std_dev, int round_bf16) {
    oracle_fill_normal_range(out, n, seed, stream, std_dev, round_bf16, 0);
}

void oracle_fill_normal_range(float* out, size_t n, uint64_t seed, uint64_t stream,
                              float std_dev, int round_bf16, uint64_t start) {
    uint64_t key = infernt_stream_key(seed, stream);
    int t = g_threads;
    if (n < (1u << 16)) t = 1;
    pthread_t th[256];
    fill_job jobs[256];
    for (int i = 0; i < t; ++i) {
        jobs[i].out = out;
        jobs[i].begin = n * (size_t)i / (size_t)t;
        jobs[i].end = n * (size_t)(i + 1) / (size_t)t;
        jobs[i].key = key;
        jobs[i].start = start;
        jobs[i].std_dev = std_dev;
        jobs[i].round_bf16 = round_bf16;
    }
    for (int i = 1; i < t; ++i) pthread_create(&th[i], NULL, fill_worker, &jobs[i]);
    fill_worker(&jobs[0]);
    for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

void oracle_fill_const(float* out, size_t n, float value) {
    for (size_t i = 0; i < n; ++i) out[i] = value;
}

void oracle_fill_prompt(int* out, int n, uint64_t seed, int lo, int hi) {
    uint64_t key = infernt_stream_key(seed, INFERNT_STREAM_PROMPT);
    for (int i = 0; i < n; ++i) out[i] = infernt_uniform_int(key, (uint64_t)i, lo, hi);
}

/* ------------------------------------------------------------------ */
/* per-op restatements                                                 */
/* ------------------------------------------------------------------ */

/* cuda/rmsnorm.cu:4-27 — o = x * rsqrt(sum(x^2)/h + eps) * w, per row. */
void oracle_rmsnorm(float* out, const float* in, const float* w, int batch,
                    int hidden, float eps) {
    for (int r = 0; r < batch; ++r) {
        const float* x = in + (size_t)r * hidden;
        float* o = out + (size_t)r * hidden;
        double ss = 0.0;
        for (int i = 0; i < hidden; ++i) ss += (double)x[i] * (double)x[i];
        float rms = (float)(1.0 / sqrt(ss / (double)hidden + (double)eps));
        for (int i = 0; i < hidden; ++i) o[i] = x[i] * rms * w[i];
    }
}

/* cuda/residual.cu:4-10 — out = a + b. */
void oracle_residual_add(float* out, const float* a, const float* b, int n) {
    for (int i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* cuda/rope.cu:5-35 — split-half rotation of pairs (d, d + D/2);
 * freq = 1 / powf(theta, 2d/D), angle = position * freq (float). */
void oracle_rope(float* q, float* k, int batch, int num_q_heads,
                 int num_kv_heads, int head_dim, int position, float theta) {
    (void)batch; /* the reference kernel ignores batch (rope.cu:37-45) */
    int half = head_dim / 2;
    int heads = num_q_heads > num_kv_heads ? num_q_heads : num_kv_heads;
    for (int h = 0; h < heads; ++h) {
        for (int d = 0; d < half; ++d) {
            float freq = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
            float angle = (float)position * freq;
            float c = cosf(angle), s = sinf(angle);
            if (h < num_q_heads) {
                float* p = q + (size_t)h * head_dim;
                float a = p[d], b = p[d + half];
                p[d] = a * c - b * s;
                p[d + half] = b * c + a * s;
            }
            if (h < num_kv_heads) {
                float* p = k + (size_t)h * head_dim;
                float a = p[d], b = p[d + half];
                p[d] = a * c - b * s;
                p[d + half] = b * c + a * s;
            }
        }
    }
}

/* cuda/softmax.cu:5-49 — max-subtracted softmax per row of seq_len. */
void oracle_softmax(float* out, const float* in, int rows, int seq_len) {
    for (int r = 0; r < rows; ++r) {
        const float* x = in + (size_t)r * seq_len;
        float* o = out + (size_t)r * seq_len;
        float m = -3.402823466e38f;
        for (int i = 0; i < seq_len; ++i) m = fmaxf(m, x[i]);
        double sum = 0.0;
        for (int i = 0; i < seq_len; ++i) sum += (double)expf(x[i] - m);
        double inv = 1.0 / (sum > 0.0 ? sum : 1.0);
        for (int i = 0; i < seq_len; ++i) o[i] = (float)((double)expf(x[i] - m) * inv);
    }
}

/* cuda/softmax.cu:51-99 — softmax over the first seq_len entries of rows of
 * length total_seq_len; the tail [seq_len, total) is zeroed. */
void oracle_softmax_with_mask(float* out, const float* in, int heads,
                              int seq_len, int total_seq_len) {
    for (int r = 0; r < heads; ++r) {
        const float* x = in + (size_t)r * total_seq_len;
        float* o = out + (size_t)r * total_seq_len;
        float m = -3.402823466e38f;
        for (int i = 0; i < seq_len; ++i) m = fmaxf(m, x[i]);
        double sum = 0.0;
        for (int i = 0; i < seq_len; ++i) sum += (double)expf(x[i] - m);
        double inv = 1.0 / (sum > 0.0 ? sum : 1.0);
        for (int i = 0; i < total_seq_len; ++i)
            o[i] = i < seq_len ? (float)((double)expf(x[i] - m) * inv) : 0.0f;
    }
}

/* cuda/kv_cache.cu:4-26 — cache[h][pos][d] = new[h][d] for K and V. */
void oracle_kv_cache_append(float* k_cache, float* v_cache, const float* k_new,
                            const float* v_new, int num_kv_heads, int head_dim,
                            int max_seq_len, int position) {
    for (int h = 0; h < num_kv_heads; ++h) {
        size_t dst = ((size_t)h * max_seq_len + position) * head_dim;
        memcpy(k_cache + dst, k_new + (size_t)h * head_dim, sizeof(float) * head_dim);
        memcpy(v_cache + dst, v_new + (size_t)h * head_dim, sizeof(float) * head_dim);
    }
}

/* cuda/attention.cu:4-23 — scores[qh][p] = (q[qh] . K[kvh][p]) * scale with
 * kvh = qh / (Nq / Nkv); row stride seq_len.  All seq_len positions are
 * computed (the reference computes only the first 1024, attention.cu:49). */
void oracle_attention_scores(float* scores, const float* q, const float* k_cache,
                             int num_q_heads, int num_kv_heads, int head_dim,
                             int seq_len, int max_seq_len, float scale) {
    int group = num_q_heads / num_kv_heads;
    for (int qh = 0; qh < num_q_heads; ++qh) {
        int kvh = qh / group;
        const float* qv = q + (size_t)qh * head_dim;
        for (int p = 0; p < seq_len; ++p) {
            const float* kv = k_cache + ((size_t)kvh * max_seq_len + p) * head_dim;
            double dot = 0.0;
            for (int d = 0; d < head_dim; ++d) dot += (double)qv[d] * (double)kv[d];
            scores[(size_t)qh * seq_len + p] = (float)dot * scale;
        }
    }
}

/* cuda/attention.cu:25-43 — out[qh][d] = sum_p P[qh][p] * V[kvh][p][d]. */
void oracle_attention_values(float* out, const float* scores,
                             const float* v_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int seq_len,
                             int max_seq_len) {
    int group = num_q_heads / num_kv_heads;
    for (int qh = 0; qh < num_q_heads; ++qh) {
        int kvh = qh / group;
        const float* s = scores + (size_t)qh * seq_len;
        for (int d = 0; d < head_dim; ++d) {
            double acc = 0.0;
            for (int p = 0; p < seq_len; ++p)
                acc += (double)s[p] *
                       (double)v_cache[((size_t)kvh * max_seq_len + p) * head_dim + d];
            out[(size_t)qh * head_dim + d] = (float)acc;
        }
    }
}

/* cuda/activation.cu:4-11 — out = g / (1 + expf(-g)) * u. */
void oracle_silu_mul(float* out, const float* gate, const float* up, int n) {
    for (int i = 0; i < n; ++i) {
        float g = gate[i];
        float silu = g / (1.0f + expf(-g));
        out[i] = silu * up[i];
    }
}

/* cuda/embedding.cu:3-8 — out = table[token * h : (token + 1) * h]. */
void oracle_embedding_lookup(float* out, const float* table, int token_id,
                             int hidden) {
    memcpy(out, table + (size_t)token_id * hidden, sizeof(float) * hidden);
}

/* cuda/sampling.cu:3-36 — argmax starting from (-1e30, 0) with strict '>',
 * so NaN never wins.  Ties resolve to the lowest index (the defined
 * tie-break of the new engine). */
int oracle_argmax(const float* logits, int vocab_size) {
    float best = -1e30f;
    int idx = 0;
    for (int i = 0; i < vocab_size; ++i) {
        if (logits[i] > best) {
            best = logits[i];
            idx = i;
        }
    }
    return idx;
}

/* cuda/sampling.cu:3-36 — the reference kernel's exact tie order: a
 * 256-thread strided scan then a halving tree, both with strict '>'. */
int oracle_argmax_ref_order(const float* logits, int vocab_size) {
    float smax[256];
    int sidx[256];
    for (int t = 0; t < 256; ++t) {
        float m = -1e30f;
        int id = 0;
        for (int i = t; i < vocab_size; i += 256)
            if (logits[i] > m) { m = logits[i]; id = i; }
        smax[t] = m;
        sidx[t] = id;
    }
    for (int s = 128; s > 0; s >>= 1)
        for (int t = 0; t < s; ++t)
            if (smax[t + s] > smax[t]) { smax[t] = smax[t + s]; sidx[t] = sidx[t + s]; }
    return sidx[0];
}

/* gemm/cublas_wrapper.cu:21-40 — row-major C = alpha op(A) op(B) + beta C,
 * lda = trans_a ? M : K, ldb = trans_b ? K : N. */
void oracle_gemm(const float* A, const float* B, float* C, int M, int N, int K,
                 float alpha, float beta, int trans_a, int trans_b) {
    for (int i = 0; i < M; ++i) {
        for (int j = 0; j < N; ++j) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                double a = trans_a ? A[(size_t)k * M + i] : A[(size_t)i * K + k];
                double b = trans_b ? B[(size_t)j * K + k] : B[(size_t)k * N + j];
                acc += a * b;
            }
            float prev = beta != 0.0f ? C[(size_t)i * N + j] : 0.0f;
            C[(size_t)i * N + j] = (float)((double)alpha * acc + (double)beta * prev);
        }
    }
}

/* ------------------------------------------------------------------ */
/* threaded y = W x  (W row-major [N, K]); the model's trans_b=true GEMM */
/* ------------------------------------------------------------------ */

typedef struct {
    const float* W;
    const float* x;
    float* y;
    int K;
    int r0, r1;
} gemv_job;

static void* gemv_worker(void* arg) {
    gemv_job* j = (gemv_job*)arg;
    for (int r = j->r0; r < j->r1; ++r) {
        const float* w = j->W + (size_t)r * j->K;
        double acc = 0.0;
        for (int k = 0; k < j->K; ++k) acc += (double)w[k] * (double)j->x[k];
        j->y[r] = (float)acc;
    }
    return NULL;
}

static void gemv(const float* W, const float* x, float* y, int N, int K) {
    int t = g_threads;
    if ((size_t)N * (size_t)K < (1u << 18)) t = 1;
    if (t > N) t = N;
    if (t < 1) t = 1;
    pthread_t th[256];
    gemv_job jobs[256];
    for (int i = 0; i < t; ++i) {
        jobs[i].W = W;
        jobs[i].x = x;
        jobs[i].y = y;
        jobs[i].K = K;
        jobs[i].r0 = (int)((long long)N * i / t);
        jobs[i].r1 = (int)((long long)N * (i + 1) / t);
    }
    for (int i = 1; i < t; ++i) pthread_create(&th[i], NULL, gemv_worker, &jobs[i]);
    gemv_worker(&jobs[0]);
    for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------ */
/* decoder layer and model                                             */
/* ------------------------------------------------------------------ */

typedef struct {
    float *xn, *q, *k, *v, *scores, *attn, *o, *gate, *up, *act, *mlp;
} scratch;

static void scratch_alloc(scratch* s, const oracle_config* c) {
    int qs = c->num_attention_heads * c->head_dim;
    int ks = c->num_key_value_heads * c->head_dim;
    s->xn = malloc(sizeof(float) * c->hidden_size);
    s->q = malloc(sizeof(float) * qs);
    s->k = malloc(sizeof(float) * ks);
    s->v = malloc(sizeof(float) * ks);
    s->scores = malloc(sizeof(float) * (size_t)c->num_attention_heads * c->max_seq_len);
    s->attn = malloc(sizeof(float) * qs);
    s->o = malloc(sizeof(float) * c->hidden_size);
    s->gate = malloc(sizeof(float) * c->intermediate_size);
    s->up = malloc(sizeof(float) * c->intermediate_size);
    s->act = malloc(sizeof(float) * c->intermediate_size);
    s->mlp = malloc(sizeof(float) * c->hidden_size);
}

static void scratch_free(scratch* s) {
    free(s->xn); free(s->q); free(s->k); free(s->v); free(s->scores);
    free(s->attn); free(s->o); free(s->gate); free(s->up); free(s->act); free(s->mlp);
}

/* architectures/llama/llama_layer.cpp:5-73 — one decoder layer, in place on
 * the residual stream h: norm, Q/K/V, RoPE, KV append, scores, softmax,
 * values, O, h += o, norm, gate/up, SiLU*up, down, h += mlp. */
static void layer_forward(const oracle_config* c, const float* const* lw,
                          float* kv_k, float* kv_v, int position, float* h,
                          scratch* s) {
    int H = c->hidden_size, D = c->head_dim, I = c->intermediate_size;
    int qs = c->num_attention_heads * D, ks = c->num_key_value_heads * D;
    oracle_rmsnorm(s->xn, h, lw[0], 1, H, c->rms_norm_eps);
    round_vec(s->xn, H);
    gemv(lw[1], s->xn, s->q, qs, H);
    gemv(lw[2], s->xn, s->k, ks, H);
    gemv(lw[3], s->xn, s->v, ks, H);
    oracle_rope(s->q, s->k, 1, c->num_attention_heads, c->num_key_value_heads, D,
                position, c->rope_theta);
    round_vec(s->k, ks);
    round_vec(s->v, ks);
    oracle_kv_cache_append(kv_k, kv_v, s->k, s->v, c->num_key_value_heads, D,
                           c->max_seq_len, position);
    int seq_len = position + 1;
    float scale = 1.0f / sqrtf((float)D); /* llama_layer.cpp:38 */
    oracle_attention_scores(s->scores, s->q, kv_k, c->num_attention_heads,
                            c->num_key_value_heads, D, seq_len, c->max_seq_len, scale);
    oracle_softmax(s->scores, s->scores, c->num_attention_heads, seq_len);
    oracle_attention_values(s->attn, s->scores, kv_v, c->num_attention_heads,
                            c->num_key_value_heads, D, seq_len, c->max_seq_len);
    round_vec(s->attn, qs);
    gemv(lw[4], s->attn, s->o, H, qs);
    oracle_residual_add(h, h, s->o, H);
    oracle_rmsnorm(s->xn, h, lw[5], 1, H, c->rms_norm_eps);
    round_vec(s->xn, H);
    gemv(lw[6], s->xn, s->gate, I, H);
    gemv(lw[7], s->xn, s->up, I, H);
    oracle_silu_mul(s->act, s->gate, s->up, I);
    round_vec(s->act, I);
    gemv(lw[8], s->act, s->mlp, H, I);
    oracle_residual_add(h, h, s->mlp, H);
}

static size_t kv_layer_elems(const oracle_config* c) {
    return (size_t)c->num_key_value_heads * c->max_seq_len * c->head_dim;
}

void oracle_llama_layers(const oracle_config* c, const float* const* w,
                         float* kv_k, float* kv_v, int position,
                         const float* input_embedding, int n_layers,
                         float* hidden_out) {
    scratch s;
    scratch_alloc(&s, c);
    memcpy(hidden_out, input_embedding, sizeof(float) * c->hidden_size);
    size_t kvl = kv_layer_elems(c);
    for (int l = 0; l < n_layers; ++l)
        layer_forward(c, w + 3 + 9 * l, kv_k + kvl * l, kv_v + kvl * l, position,
                      hidden_out, &s);
    scratch_free(&s);
}

/* architectures/llama/llama_model.cpp:45-65 — layers, final RMSNorm, LM head. */
void oracle_llama_forward(const oracle_config* c, const float* const* w,
                          float* kv_k, float* kv_v, int position,
                          const float* input_embedding, float* logits) {
    float* h = malloc(sizeof(float) * c->hidden_size);
    float* xn = malloc(sizeof(float) * c->hidden_size);
    oracle_llama_layers(c, w, kv_k, kv_v, position, input_embedding, c->num_layers, h);
    oracle_rmsnorm(xn, h, w[1], 1, c->hidden_size, c->rms_norm_eps);
    round_vec(xn, c->hidden_size);
    gemv(w[2], xn, logits, c->vocab_size, c->hidden_size);
    free(h);
    free(xn);
}

/* src/engine.cpp:53-76 — embedding lookup, forward, greedy argmax. */
int oracle_decode_token(const oracle_config* c, const float* const* w,
                        float* kv_k, float* kv_v, int token, int position,
                        float* logits) {
    float* emb = malloc(sizeof(float) * c->hidden_size);
    oracle_embedding_lookup(emb, w[0], token, c->hidden_size);
    oracle_llama_forward(c, w, kv_k, kv_v, position, emb, logits);
    free(emb);
    return oracle_argmax(logits, c->vocab_size);
}
