// plan.cu — the decode step: 5 kernels per decoder layer + 1 for the head.
//
//   qkv     RMSNorm(attn_norm) + [Wq;Wk;Wv] x          (layer 0: embedding row of the token)
//   attn    RoPE + KV append + split-KV GQA attention   -> attn_out
//   o       hidden += Wo attn_out
//   gateup  RMSNorm(ffn_norm) + SiLU(Wg x) * (Wu x)     -> act
//   down    hidden += Wd act
//   head    RMSNorm(final_norm) + logits = Wlm x + argmax -> token, state advanced
//
// (architectures/llama/llama_layer.cpp:5-73, llama_model.cpp:45-65,
// src/engine.cpp:53-76).  The residual stream is updated in place, so the
// reference's 23 hidden-state copies per token (llama_model.cpp:48, :55)
// disappear.  Token, position and step live in a small device state block:
// the attention kernel reads the position from it and the head kernel
// writes the next token and position into it, so a chain of steps needs no
// host round trip.  Every kernel is launched with programmatic stream
// serialisation, so the next kernel's CTAs start streaming their weights
// while the previous kernel drains; the step is captured once into a CUDA
// graph and replayed.
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "attention.cuh"
#include "gemv.cuh"
#include "internal.h"

namespace infernt {

__global__ void set_state_kernel(int* state, int token, int pos) {
    state[0] = token;
    state[1] = pos;
    state[2] = 0;
}

struct LmWs {
    float val[kArgmaxMaxBlocks];
    int idx[kArgmaxMaxBlocks];
    unsigned counter;
    unsigned pad[3];
};

}  // namespace infernt

using namespace infernt;

struct infernt_plan {
    infernt_llama_config cfg;
    std::vector<const void*> w;
    std::vector<float*> kc, vc;
    int qs = 0, kvs = 0, splits = 1;
    void* scratch = nullptr;
    float* qkv = nullptr;
    float* attn = nullptr;
    float* act = nullptr;
    float* hidden = nullptr;
    float* logits = nullptr;
    int* state = nullptr;     // {token, position, step, last token}
    unsigned* err = nullptr;
    float* attn_part = nullptr;
    unsigned* attn_counter = nullptr;
    LmWs* lm_ws = nullptr;
    bool use_graph = true;
    cudaStream_t cap_stream = nullptr;
    struct Entry {
        int mode;
        const float* input;
        float* logits;
        int* hist;
        cudaGraphExec_t exec;
    };
    std::vector<Entry> graphs;
};

namespace {

const int kModeInput = 0;  // layer 0 reads an input embedding vector
const int kModeToken = 1;  // layer 0 reads the embedding row of state[0]

int record_step(infernt_plan* p, cudaStream_t st, int mode, const float* input, float* logits,
                int* hist) {
    const infernt_llama_config& c = p->cfg;
    const int H = c.hidden_size, I = c.intermediate_size, L = c.num_layers;
    const int dt = c.weight_dtype;
    for (int l = 0; l < L; ++l) {
        const void* const* lw = p->w.data() + 3 + 9 * l;
        // qkv
        GemvArgs a;
        memset(&a, 0, sizeof(a));
        a.seg_ptr[0] = lw[1];
        a.seg_ptr[1] = lw[2];
        a.seg_ptr[2] = lw[3];
        a.seg_rows[0] = p->qs;
        a.seg_rows[1] = p->kvs;
        a.seg_rows[2] = p->kvs;
        a.nseg = 3;
        a.units = p->qs + 2 * p->kvs;
        a.K = H;
        if (l == 0) {
            a.x = mode == kModeInput ? input : nullptr;
            a.emb = static_cast<const float*>(p->w[0]);
            a.token = p->state;
            a.vocab = c.vocab_size;
            a.x_copy = p->hidden;
        } else {
            a.x = p->hidden;
        }
        a.norm_w = static_cast<const float*>(lw[0]);
        a.eps = c.rms_norm_eps;
        a.out = p->qkv;
        a.err = p->err;
        INFERNT_CUDA_TRY(launch_gemv(a, dt, kEpiStore, st, true, nullptr));

        // attention
        AttnArgs at;
        memset(&at, 0, sizeof(at));
        at.qkv = p->qkv;
        at.k_cache = p->kc[l];
        at.v_cache = p->vc[l];
        at.out = p->attn;
        at.part = p->attn_part;
        at.counter = p->attn_counter;
        at.pos_ptr = p->state + 1;
        at.nq = c.num_attention_heads;
        at.nkv = c.num_key_value_heads;
        at.D = c.head_dim;
        at.max_seq = c.max_seq_len;
        at.splits = p->splits;
        at.theta = c.rope_theta;
        at.scale = 1.0f / sqrtf((float)c.head_dim);
        at.err = p->err;
        INFERNT_CUDA_TRY(launch_attention_decode(at, st, true));

        // o projection + residual
        memset(&a, 0, sizeof(a));
        a.seg_ptr[0] = lw[4];
        a.seg_rows[0] = H;
        a.nseg = 1;
        a.units = H;
        a.K = p->qs;
        a.x = p->attn;
        a.out = p->hidden;
        a.res = p->hidden;
        a.err = p->err;
        INFERNT_CUDA_TRY(launch_gemv(a, dt, kEpiResidual, st, true, nullptr));

        // gate/up + SiLU
        memset(&a, 0, sizeof(a));
        a.seg_ptr[0] = lw[6];
        a.seg_ptr[1] = lw[7];
        a.seg_rows[0] = a.seg_rows[1] = I;
        a.nseg = 2;
        a.units = I;
        a.K = H;
        a.x = p->hidden;
        a.norm_w = static_cast<const float*>(lw[5]);
        a.eps = c.rms_norm_eps;
        a.out = p->act;
        a.err = p->err;
        INFERNT_CUDA_TRY(launch_gemv(a, dt, kEpiSwiGLU, st, true, nullptr));

        // down + residual
        memset(&a, 0, sizeof(a));
        a.seg_ptr[0] = lw[8];
        a.seg_rows[0] = H;
        a.nseg = 1;
        a.units = H;
        a.K = I;
        a.x = p->act;
        a.out = p->hidden;
        a.res = p->hidden;
        a.err = p->err;
        INFERNT_CUDA_TRY(launch_gemv(a, dt, kEpiResidual, st, true, nullptr));
    }
    // final norm + LM head + argmax
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.seg_ptr[0] = p->w[2];
    a.seg_rows[0] = c.vocab_size;
    a.nseg = 1;
    a.units = c.vocab_size;
    a.K = H;
    a.x = p->hidden;
    a.norm_w = static_cast<const float*>(p->w[1]);
    a.eps = c.rms_norm_eps;
    a.out = logits;
    a.am_val = p->lm_ws->val;
    a.am_idx = p->lm_ws->idx;
    a.am_counter = &p->lm_ws->counter;
    a.am_out = p->state + 3;
    a.state = p->state;
    a.token_hist = hist;
    a.err = p->err;
    INFERNT_CUDA_TRY(launch_gemv(a, dt, kEpiArgmax, st, true, nullptr));
    return INFERNT_OK;
}

int run_step(infernt_plan* p, cudaStream_t st, int mode, const float* input, float* logits, int* hist) {
    if (!logits) logits = p->logits;
    if (!p->use_graph) return record_step(p, st, mode, input, logits, hist);
    for (auto& e : p->graphs)
        if (e.mode == mode && e.input == input && e.logits == logits && e.hist == hist) {
            INFERNT_CUDA_TRY(cudaGraphLaunch(e.exec, st));
            return INFERNT_OK;
        }
    if (!p->cap_stream) INFERNT_CUDA_TRY(cudaStreamCreateWithFlags(&p->cap_stream, cudaStreamNonBlocking));
    INFERNT_CUDA_TRY(cudaStreamBeginCapture(p->cap_stream, cudaStreamCaptureModeThreadLocal));
    int s = record_step(p, p->cap_stream, mode, input, logits, hist);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(p->cap_stream, &g);
    if (s) {
        if (g) cudaGraphDestroy(g);
        return s;
    }
    INFERNT_CUDA_TRY(e);
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    INFERNT_CUDA_TRY(e);
    if (p->graphs.size() >= 8) {
        cudaGraphExecDestroy(p->graphs.front().exec);
        p->graphs.erase(p->graphs.begin());
    }
    p->graphs.push_back({mode, input, logits, hist, exec});
    INFERNT_CUDA_TRY(cudaGraphLaunch(exec, st));
    return INFERNT_OK;
}

int validate_config(const infernt_llama_config* c) {
    INFERNT_REQUIRE(c, "plan: null config");
    INFERNT_REQUIRE(c->vocab_size > 0 && c->hidden_size > 0 && c->num_layers > 0 &&
                        c->num_attention_heads > 0 && c->num_key_value_heads > 0 &&
                        c->intermediate_size > 0 && c->max_seq_len > 0 && c->head_dim > 0,
                    "plan: every dimension must be positive");
    INFERNT_REQUIRE(c->hidden_size % 4 == 0 && c->intermediate_size % 4 == 0,
                    "plan: hidden %d and intermediate %d must be multiples of 4", c->hidden_size,
                    c->intermediate_size);
    INFERNT_REQUIRE(c->weight_dtype == INFERNT_DTYPE_F32 || c->weight_dtype == INFERNT_DTYPE_BF16,
                    "plan: weight_dtype %d", c->weight_dtype);
    INFERNT_REQUIRE(c->vocab_size <= 1 << 30 && (long long)c->max_seq_len * c->head_dim < (1ll << 31),
                    "plan: shape too large");
    return attention_shape_check(c->num_attention_heads, c->num_key_value_heads, c->head_dim, 1);
}

}  // namespace

extern "C" {

int infernt_plan_create(const infernt_llama_config* cfg, const void* const* weights,
                        float* const* k_cache, float* const* v_cache, int use_graph,
                        infernt_plan** out) {
    INFERNT_REQUIRE(out, "plan_create: null output");
    *out = nullptr;
    if (int s = validate_config(cfg)) return s;
    INFERNT_REQUIRE(weights && k_cache && v_cache, "plan_create: null weights or cache");
    const int L = cfg->num_layers;
    for (int i = 0; i < 3 + 9 * L; ++i)
        INFERNT_REQUIRE(weights[i], "plan_create: weight pointer %d is null", i);
    for (int l = 0; l < L; ++l) INFERNT_REQUIRE(k_cache[l] && v_cache[l], "plan_create: cache layer %d null", l);
    INFERNT_CUDA_TRY(gemv_prepare());

    infernt_plan* p = new (std::nothrow) infernt_plan();
    INFERNT_REQUIRE(p, "plan_create: host allocation failed");
    p->cfg = *cfg;
    p->w.assign(weights, weights + 3 + 9 * L);
    p->kc.assign(k_cache, k_cache + L);
    p->vc.assign(v_cache, v_cache + L);
    p->qs = cfg->num_attention_heads * cfg->head_dim;
    p->kvs = cfg->num_key_value_heads * cfg->head_dim;
    p->use_graph = use_graph != 0;
    int splits = sm_count() / cfg->num_key_value_heads;
    p->splits = splits < 1 ? 1 : splits;

    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t b_qkv = al(sizeof(float) * (p->qs + 2 * p->kvs));
    const size_t b_attn = al(sizeof(float) * p->qs);
    const size_t b_act = al(sizeof(float) * cfg->intermediate_size);
    const size_t b_hid = al(sizeof(float) * cfg->hidden_size);
    const size_t b_log = al(sizeof(float) * cfg->vocab_size);
    const size_t b_state = 256;
    const size_t b_aws = attention_workspace_bytes(cfg->num_attention_heads, cfg->num_key_value_heads,
                                                   cfg->head_dim, p->splits);
    const size_t b_lm = al(sizeof(LmWs));
    const size_t total = b_qkv + b_attn + b_act + b_hid + b_log + b_state + b_aws + b_lm;
    cudaError_t e = cudaMalloc(&p->scratch, total);
    if (e != cudaSuccess) {
        delete p;
        return cuda_fail(e, "cudaMalloc(plan scratch)");
    }
    e = cudaMemset(p->scratch, 0, total);
    if (e != cudaSuccess) {
        cudaFree(p->scratch);
        delete p;
        return cuda_fail(e, "cudaMemset(plan scratch)");
    }
    char* b = static_cast<char*>(p->scratch);
    p->qkv = reinterpret_cast<float*>(b); b += b_qkv;
    p->attn = reinterpret_cast<float*>(b); b += b_attn;
    p->act = reinterpret_cast<float*>(b); b += b_act;
    p->hidden = reinterpret_cast<float*>(b); b += b_hid;
    p->logits = reinterpret_cast<float*>(b); b += b_log;
    p->state = reinterpret_cast<int*>(b);
    p->err = reinterpret_cast<unsigned*>(b + 64);
    b += b_state;
    const size_t part = (size_t)cfg->num_key_value_heads * p->splits *
                        (cfg->num_attention_heads / cfg->num_key_value_heads) * (cfg->head_dim + 2) * 4;
    p->attn_part = reinterpret_cast<float*>(b);
    p->attn_counter = reinterpret_cast<unsigned*>(b + al(part));
    b += b_aws;
    p->lm_ws = reinterpret_cast<LmWs*>(b);
    *out = p;
    return INFERNT_OK;
}

int infernt_plan_destroy(infernt_plan* p) {
    if (!p) return INFERNT_OK;
    for (auto& e : p->graphs) cudaGraphExecDestroy(e.exec);
    if (p->cap_stream) cudaStreamDestroy(p->cap_stream);
    cudaFree(p->scratch);
    delete p;
    return INFERNT_OK;
}

int infernt_plan_forward(infernt_plan* p, const float* input_embedding, int position, float* logits,
                         void* stream) {
    INFERNT_REQUIRE(p && input_embedding, "plan_forward: null argument");
    INFERNT_REQUIRE(position >= 0 && position < p->cfg.max_seq_len,
                    "plan_forward: position %d outside [0, %d)", position, p->cfg.max_seq_len);
    cudaStream_t st = (cudaStream_t)stream;
    set_state_kernel<<<1, 1, 0, st>>>(p->state, 0, position);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return run_step(p, st, kModeInput, input_embedding, logits, nullptr);
}

int infernt_plan_decode(infernt_plan* p, int token, int position, float* logits, void* stream) {
    INFERNT_REQUIRE(p, "plan_decode: null plan");
    INFERNT_REQUIRE(token >= 0 && token < p->cfg.vocab_size, "plan_decode: token %d outside [0, %d)", token,
                    p->cfg.vocab_size);
    INFERNT_REQUIRE(position >= 0 && position < p->cfg.max_seq_len,
                    "plan_decode: position %d outside [0, %d)", position, p->cfg.max_seq_len);
    cudaStream_t st = (cudaStream_t)stream;
    set_state_kernel<<<1, 1, 0, st>>>(p->state, token, position);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return run_step(p, st, kModeToken, nullptr, logits, nullptr);
}

int infernt_plan_decode_chain(infernt_plan* p, int token, int position, int steps, int* tokens_dev,
                              void* stream) {
    INFERNT_REQUIRE(p, "plan_decode_chain: null plan");
    INFERNT_REQUIRE(token >= 0 && token < p->cfg.vocab_size, "plan_decode_chain: token %d", token);
    INFERNT_REQUIRE(steps >= 0 && position >= 0 && (long long)position + steps <= p->cfg.max_seq_len,
                    "plan_decode_chain: positions [%d, %d) exceed max_seq_len %d", position,
                    position + steps, p->cfg.max_seq_len);
    cudaStream_t st = (cudaStream_t)stream;
    set_state_kernel<<<1, 1, 0, st>>>(p->state, token, position);
    INFERNT_CUDA_TRY(cudaGetLastError());
    for (int s = 0; s < steps; ++s)
        if (int r = run_step(p, st, kModeToken, nullptr, nullptr, tokens_dev)) return r;
    return INFERNT_OK;
}

int infernt_plan_read_token(infernt_plan* p, int* token_host, void* stream) {
    INFERNT_REQUIRE(p && token_host, "plan_read_token: null argument");
    cudaStream_t st = (cudaStream_t)stream;
    int buf[4];
    unsigned err = 0;
    INFERNT_CUDA_TRY(cudaMemcpyAsync(buf, p->state, sizeof(buf), cudaMemcpyDeviceToHost, st));
    INFERNT_CUDA_TRY(cudaMemcpyAsync(&err, p->err, sizeof(err), cudaMemcpyDeviceToHost, st));
    INFERNT_CUDA_TRY(cudaStreamSynchronize(st));
    if (err) {
        cudaMemsetAsync(p->err, 0, sizeof(unsigned), st);
        return fail(INFERNT_ERR_DEVICE, "decode kernels reported error word 0x%x (1: wait timeout, 2: position, "
                    "4: token id)", err);
    }
    *token_host = buf[3];
    return INFERNT_OK;
}

float* infernt_plan_logits(infernt_plan* p) { return p ? p->logits : nullptr; }

int infernt_plan_kernels_per_step(const infernt_plan* p) { return p ? 5 * p->cfg.num_layers + 1 : 0; }

}  // extern "C"
