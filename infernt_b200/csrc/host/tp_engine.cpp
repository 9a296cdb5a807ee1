// tp_engine.cpp — one rank of a tensor-parallel decoder with seeded
// synthetic weights (infernt_tp_engine_* in include/infernt_capi.h): the
// rank's weight shards are generated on the device as windows of the full
// seeded matrices (the values a single-GPU engine of the same seed holds),
// its KV caches allocated for its KV heads, and the tensor-parallel plan
// built over them.  Every allocation happens here, at creation.
#include <cuda_runtime.h>

#include <cstring>
#include <new>
#include <vector>

#include "../../../include/infernt_capi.h"
#include "../../../include/infernt_seed.h"
#include "../internal.h"

struct infernt_tp_engine {
    infernt_llama_config cfg;
    int rank = 0, size = 1;
    int dims[6] = {0, 0, 0, 0, 0, 0};
    std::vector<void*> bufs;
    std::vector<const void*> w;
    std::vector<float*> kc, vc;
    infernt_plan* plan = nullptr;
    cudaStream_t stream = nullptr;
    int* tokens_dev = nullptr;
    int tokens_cap = 0;
    cudaEvent_t ev[2] = {nullptr, nullptr};

    ~infernt_tp_engine() {
        infernt_plan_destroy(plan);
        if (ev[0]) cudaEventDestroy(ev[0]);
        if (ev[1]) cudaEventDestroy(ev[1]);
        cudaFree(tokens_dev);
        for (void* b : bufs) cudaFree(b);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

using infernt::fail;

int alloc(infernt_tp_engine* e, size_t bytes, void** out) {
    void* p = nullptr;
    INFERNT_CUDA_TRY(cudaMalloc(&p, bytes));
    e->bufs.push_back(p);
    *out = p;
    return INFERNT_OK;
}

// a [rows][ld] shard: rows row0.. and columns col0..col0+cols-1 of the seeded
// [*, src_ld] matrix of `stream_id`, zero past cols
int shard(infernt_tp_engine* e, int rows, int cols, int ld, long long src_ld, long long row0, long long col0,
          int dtype, uint64_t seed, uint64_t stream_id, float std_dev, const void** out) {
    void* p = nullptr;
    const size_t eb = dtype == INFERNT_DTYPE_BF16 ? 2 : 4;
    if (int s = alloc(e, (size_t)rows * ld * eb, &p)) return s;
    if (int s = infernt_fill_normal_window(p, rows, cols, ld, (uint64_t)src_ld, (uint64_t)row0, (uint64_t)col0,
                                           dtype, seed, stream_id, std_dev, e->stream))
        return s;
    *out = p;
    return INFERNT_OK;
}

int ones(infernt_tp_engine* e, int n, const void** out) {
    void* p = nullptr;
    if (int s = alloc(e, (size_t)n * 4, &p)) return s;
    if (int s = infernt_fill_const(static_cast<float*>(p), (size_t)n, 1.0f, e->stream)) return s;
    *out = p;
    return INFERNT_OK;
}

int build(infernt_tp_engine* e, uint64_t seed, float std_dev) {
    const infernt_llama_config& c = e->cfg;
    const int t = e->rank;
    const int H = c.hidden_size, V = c.vocab_size, D = c.head_dim, L = c.num_layers;
    const int nq = e->dims[0], nkv = e->dims[1], il = e->dims[2], ip = e->dims[3];
    const int v0 = e->dims[4], vl = e->dims[5];
    const int qs = c.num_attention_heads * D, kvs = c.num_key_value_heads * D;
    const int qsl = nq * D, kvsl = nkv * D;
    const int wd = c.weight_dtype, f32 = INFERNT_DTYPE_F32;
    INFERNT_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    e->w.assign(3 + 9 * L, nullptr);
    if (int s = shard(e, V, H, H, H, 0, 0, f32, seed, INFERNT_STREAM_EMBEDDING, std_dev, &e->w[0])) return s;
    if (int s = ones(e, H, &e->w[1])) return s;
    if (int s = shard(e, vl, H, H, H, v0, 0, wd, seed, INFERNT_STREAM_LM_HEAD, std_dev, &e->w[2])) return s;
    for (int l = 0; l < L; ++l) {
        const void** lw = e->w.data() + 3 + 9 * l;
        if (int s = ones(e, H, &lw[0])) return s;
        if (int s = shard(e, qsl, H, H, H, (long long)t * qsl, 0, wd, seed, INFERNT_STREAM_LAYER(l, 0), std_dev,
                          &lw[1]))
            return s;
        if (int s = shard(e, kvsl, H, H, H, (long long)t * kvsl, 0, wd, seed, INFERNT_STREAM_LAYER(l, 1), std_dev,
                          &lw[2]))
            return s;
        if (int s = shard(e, kvsl, H, H, H, (long long)t * kvsl, 0, wd, seed, INFERNT_STREAM_LAYER(l, 2), std_dev,
                          &lw[3]))
            return s;
        if (int s = shard(e, H, qsl, qsl, qs, 0, (long long)t * qsl, wd, seed, INFERNT_STREAM_LAYER(l, 3), std_dev,
                          &lw[4]))
            return s;
        if (int s = ones(e, H, &lw[5])) return s;
        if (int s = shard(e, il, H, H, H, (long long)t * il, 0, wd, seed, INFERNT_STREAM_LAYER(l, 4), std_dev,
                          &lw[6]))
            return s;
        if (int s = shard(e, il, H, H, H, (long long)t * il, 0, wd, seed, INFERNT_STREAM_LAYER(l, 5), std_dev,
                          &lw[7]))
            return s;
        if (int s = shard(e, H, il, ip, c.intermediate_size, 0, (long long)t * il, wd, seed,
                          INFERNT_STREAM_LAYER(l, 6), std_dev, &lw[8]))
            return s;
    }
    (void)kvs;
    const size_t cache = (size_t)nkv * c.max_seq_len * D * sizeof(float);
    for (int l = 0; l < L; ++l) {
        void* k = nullptr;
        void* v = nullptr;
        if (int s = alloc(e, cache, &k)) return s;
        if (int s = alloc(e, cache, &v)) return s;
        INFERNT_CUDA_TRY(cudaMemsetAsync(k, 0, cache, e->stream));
        INFERNT_CUDA_TRY(cudaMemsetAsync(v, 0, cache, e->stream));
        e->kc.push_back(static_cast<float*>(k));
        e->vc.push_back(static_cast<float*>(v));
    }
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    INFERNT_CUDA_TRY(cudaEventCreate(&e->ev[0]));
    INFERNT_CUDA_TRY(cudaEventCreate(&e->ev[1]));
    return infernt_plan_create_tp(&e->cfg, e->w.data(), e->kc.data(), e->vc.data(), t, e->size, &e->plan);
}

}  // namespace

extern "C" {

int infernt_tp_engine_create_seeded(const infernt_llama_config* cfg, uint64_t seed, float std_dev, int tp_rank,
                                    int tp_size, infernt_tp_engine** out) {
    INFERNT_REQUIRE(cfg && out, "tp_engine_create_seeded: null argument");
    *out = nullptr;
    infernt_tp_engine* e = new (std::nothrow) infernt_tp_engine();
    INFERNT_REQUIRE(e, "tp_engine_create_seeded: host allocation failed");
    e->cfg = *cfg;
    e->rank = tp_rank;
    e->size = tp_size;
    int s = infernt_tp_shard_dims(cfg, tp_rank, tp_size, e->dims);
    if (!s) s = build(e, seed, std_dev);
    if (s) {
        delete e;
        return s;
    }
    *out = e;
    return INFERNT_OK;
}

int infernt_tp_engine_destroy(infernt_tp_engine* e) {
    delete e;
    return INFERNT_OK;
}

int infernt_tp_engine_xchg_handle(infernt_tp_engine* e, void* handle_out) {
    INFERNT_REQUIRE(e, "tp_engine_xchg_handle: null engine");
    return infernt_plan_xchg_handle(e->plan, handle_out);
}

int infernt_tp_engine_set_peers(infernt_tp_engine* e, const void* handles) {
    INFERNT_REQUIRE(e, "tp_engine_set_peers: null engine");
    return infernt_plan_set_peers(e->plan, handles);
}

int infernt_tp_engine_forward_token(infernt_tp_engine* e, int token, int position, int* next_token) {
    INFERNT_REQUIRE(e && next_token, "tp_engine_forward_token: null argument");
    if (int s = infernt_plan_decode(e->plan, token, position, nullptr, e->stream)) return s;
    return infernt_plan_read_token(e->plan, next_token, e->stream);
}

int infernt_tp_engine_decode_chain(infernt_tp_engine* e, int token, int position, int steps, int* tokens_host,
                                   float* ms) {
    INFERNT_REQUIRE(e && steps > 0, "tp_engine_decode_chain: bad arguments");
    if (steps > e->tokens_cap) {
        cudaFree(e->tokens_dev);
        e->tokens_dev = nullptr;
        e->tokens_cap = 0;
        INFERNT_CUDA_TRY(cudaMalloc(&e->tokens_dev, sizeof(int) * steps));
        e->tokens_cap = steps;
    }
    INFERNT_CUDA_TRY(cudaEventRecord(e->ev[0], e->stream));
    if (int s = infernt_plan_decode_chain(e->plan, token, position, steps, e->tokens_dev, e->stream)) return s;
    INFERNT_CUDA_TRY(cudaEventRecord(e->ev[1], e->stream));
    int last = 0;
    if (int s = infernt_plan_read_token(e->plan, &last, e->stream)) return s;
    if (ms) INFERNT_CUDA_TRY(cudaEventElapsedTime(ms, e->ev[0], e->ev[1]));
    if (tokens_host)
        INFERNT_CUDA_TRY(cudaMemcpy(tokens_host, e->tokens_dev, sizeof(int) * steps, cudaMemcpyDeviceToHost));
    return INFERNT_OK;
}

int infernt_tp_engine_logits(infernt_tp_engine* e, float* logits_host, int n) {
    INFERNT_REQUIRE(e && logits_host && n == e->dims[5], "tp_engine_logits: need the rank's %d vocabulary rows",
                    e ? e->dims[5] : 0);
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    INFERNT_CUDA_TRY(
        cudaMemcpy(logits_host, infernt_plan_logits(e->plan), sizeof(float) * n, cudaMemcpyDeviceToHost));
    return INFERNT_OK;
}

int infernt_tp_engine_trace_chain(infernt_tp_engine* e, int token, int position, int steps,
                                  unsigned long long* host_out, size_t n) {
    INFERNT_REQUIRE(e && host_out && steps > 0, "tp_engine_trace_chain: bad arguments");
    const size_t need = infernt_plan_trace_entries(e->plan, steps);
    INFERNT_REQUIRE(n >= need, "tp_engine_trace_chain: need %zu entries", need);
    unsigned long long* dev = nullptr;
    INFERNT_CUDA_TRY(cudaMalloc(&dev, need * sizeof(unsigned long long)));
    cudaMemset(dev, 0, need * sizeof(unsigned long long));
    int s = infernt_plan_set_trace(e->plan, dev);
    if (!s) s = infernt_tp_engine_decode_chain(e, token, position, steps, nullptr, nullptr);
    infernt_plan_set_trace(e->plan, nullptr);
    const cudaError_t ce = cudaMemcpy(host_out, dev, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (s) return s;
    INFERNT_CUDA_TRY(ce);
    return INFERNT_OK;
}

int infernt_tp_engine_plan(infernt_tp_engine* e, infernt_plan** plan) {
    INFERNT_REQUIRE(e && plan, "tp_engine_plan: null argument");
    *plan = e->plan;
    return INFERNT_OK;
}

int infernt_tp_engine_dims(infernt_tp_engine* e, int* dims) {
    INFERNT_REQUIRE(e && dims, "tp_engine_dims: null argument");
    memcpy(dims, e->dims, sizeof(e->dims));
    return INFERNT_OK;
}

}  // extern "C"
