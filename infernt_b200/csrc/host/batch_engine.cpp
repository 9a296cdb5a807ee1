// batch_engine.cpp — batched decode of T sequences with seeded synthetic
// weights (infernt_batch_engine_* in include/infernt_capi.h): bf16
// projection weights (the Q|K|V and gate|up matrices stacked so each is one
// tensor-core projection), FP32 embedding and norms, per-sequence bf16 KV
// caches [T][N_kv][max_seq][D] per layer.  A step is a fixed sequence of
// launches (bgemm.cu, batch.cu) captured once into a CUDA graph and
// replayed; tokens and positions live on the device and the argmax kernel
// advances them, so chained steps need no host round trip.  Decode
// allocates nothing after creation; prompt prefill (prefill.cu, pgemm in
// bgemm.cu) allocates its chunk scratch at its first call.  With world > 1
// the engine is one rank of a tensor-parallel decoder (NCCL all-reduce of
// the O and down sums, all-gather of the argmax candidates).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "../../../include/infernt_capi.h"
#include "../../../include/infernt_seed.h"
#include "../internal.h"

namespace infernt {
int bgemm_ctas_per_sm(int tp);
int bgemm_launch(const void* W, int N, int K, const void* X, int T, float* part, int splits, unsigned* err,
                 cudaStream_t st);
int bt_swiglu_launch(const float* part, int splits, int T, int I, uint16_t* act, cudaStream_t st);
int bt_rope_table_launch(float2* tab, int max_seq, int D, float theta, cudaStream_t st);
int bt_embed_norm_launch(const float* emb, const int* tokens, int vocab, int T, int H, const float* norm_w, float eps,
                         float* h, uint16_t* xb, unsigned* err, cudaStream_t st);
int bt_resid_norm_launch(const float* part, int splits, int T, int H, float* h, const float* norm_w, float eps,
                         uint16_t* xb, cudaStream_t st);
int bt_qkv_finish_launch(const float* part, int splits, int T, int nq, int nkv, int D, const int* positions,
                         const float2* rope, int max_seq, float* q, uint16_t* kc, uint16_t* vc, unsigned* err,
                         cudaStream_t st);
int bt_attention_launch(const float* q, const uint16_t* kc, const uint16_t* vc, const int* positions, int T, int nq,
                        int nkv, int D, int max_seq, int S, int min_chunk, int stages, float* part, uint16_t* attn,
                        cudaStream_t st, float* attn_f32 = nullptr);
int bt_attention_fused_launch(const float* qkv_part, int qkv_splits, const float2* rope, uint16_t* kc, uint16_t* vc,
                              const int* positions, int T, int nq, int nkv, int D, int max_seq, int S, int min_chunk,
                              int stages, float* part, uint16_t* attn, unsigned* err, unsigned* tickets,
                              cudaStream_t st, const int* block_table, int page_size, int max_pages);
int bt_fill_kv_launch(uint16_t* cache, int seq, int layer, int nkv, int max_seq, int D, int n_pos, uint64_t key,
                      float std_dev, int h0, int nkv_all, cudaStream_t st, const int* pages, int page_size);
int bt_page_copy_launch(uint16_t* pool, uint16_t* flat, const int* pages, int page_size, int nkv, int max_seq, int D,
                        int p0, int p1, bool to_pages, cudaStream_t st);
int bt_argmax_launch(const float* logits, int T, int V, int* tokens, int* positions, int* hist, float* cand_v,
                     int* cand_i, unsigned* tickets, float inv_t, uint64_t seed, cudaStream_t st,
                     const uint64_t* salts);
int pgemm_launch(const void* W, int N, int K, const void* X, int T, float* Y, int ldy, unsigned* err,
                 cudaStream_t st);
int pgemm_swiglu_launch(const void* W_gu, int I, int K, const void* X, int T, uint16_t* act, int ldy, unsigned* err,
                        cudaStream_t st);
int pf_qkv_rope_launch(const float* y, int C, int p0, int nq, int nkv, int D, const float2* rope, int max_seq,
                       uint16_t* q, uint16_t* kc, uint16_t* vc, cudaStream_t st);
int pf_attention_launch(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int C, int p0, int nq, int nkv,
                        int D, int max_seq, uint16_t* attn, unsigned* err, int tensor_cores, cudaStream_t st);
int tp_sum_splits_launch(const float* part, int splits, int T, int N, float* y, cudaStream_t st);
int bt_epoch_advance_launch(unsigned* epoch, cudaStream_t st);
int tp_push_launch(const float* part, int splits, int T, int N, unsigned long long* const* peers, int rank, int world,
                   const unsigned* epoch, int per_step, int idx, cudaStream_t st);
int bt_resid_norm_tp_launch(const unsigned long long* own, int world, int T, int H, float* h, const float* norm_w,
                            float eps, uint16_t* xb, const unsigned* epoch, int per_step, int idx, unsigned* err,
                            long long budget, cudaStream_t st);
int tp_argmax_local_launch(const float* logits, int T, int ld, int vl, int v0, int2* cand, const int* positions,
                           float inv_t, uint64_t seed, cudaStream_t st);
int tp_argmax_pick_launch(const int2* cand_all, int world, int T, int* tokens, int* positions, cudaStream_t st);
}  // namespace infernt

namespace {

// NCCL entry points of the process's libnccl.so.2, resolved at run time: the
// one already loaded (by the framework that set up the ranks) when there is
// one, so that the process holds a single NCCL; the library itself does not
// link NCCL.
struct NcclApi {
    decltype(&ncclGetUniqueId) get_id = nullptr;
    decltype(&ncclCommInitRank) init = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGetErrorString) err_str = nullptr;
};

NcclApi load_nccl() {
    NcclApi api;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (h) {
        api.get_id = reinterpret_cast<decltype(api.get_id)>(dlsym(h, "ncclGetUniqueId"));
        api.init = reinterpret_cast<decltype(api.init)>(dlsym(h, "ncclCommInitRank"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
        api.err_str = reinterpret_cast<decltype(api.err_str)>(dlsym(h, "ncclGetErrorString"));
    }
    return api;
}

const NcclApi* nccl_api() {
    static const NcclApi api = load_nccl();  // resolved once, thread-safe initialisation
    const bool ok = api.get_id && api.init && api.all_reduce && api.all_gather && api.destroy && api.err_str;
    return ok ? &api : nullptr;
}

}  // namespace

struct infernt_batch_engine {
    infernt_llama_config cfg;
    int T = 0, S = 1;            // sequences, attention splits
    int min_chunk = 64, stages = 3;  // attention: least positions per split, cp.async stages per warp
    // weights
    const float* emb = nullptr;
    const float* final_norm = nullptr;
    const void* lm = nullptr;
    struct Layer {
        const float *attn_norm, *ffn_norm;
        const void *qkv, *o, *gu, *down;
    };
    std::vector<Layer> layers;
    std::vector<uint16_t*> kc, vc;
    // splits of the projections
    int sp_qkv = 1, sp_o = 1, sp_gu = 1, sp_down = 1, sp_lm = 1;
    // state and scratch
    int* tokens = nullptr;
    int* positions = nullptr;
    unsigned* err = nullptr;
    float* h = nullptr;
    uint16_t* xb = nullptr;
    uint16_t* attn = nullptr;
    uint16_t* act = nullptr;
    float* q = nullptr;
    float* part = nullptr;
    float* apart = nullptr;
    unsigned* tickets = nullptr;     // [T][nkv] split tickets of the attention (zero between launches)
    unsigned* am_tickets = nullptr;  // [T] chunk tickets of the argmax
    float* cand_v = nullptr;         // [T][8] argmax candidates per vocabulary chunk
    int* cand_i = nullptr;
    float2* rope = nullptr;
    std::vector<void*> bufs;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int* hist = nullptr;  // tokens of chained steps (grown on demand)
    size_t hist_cap = 0;
    // prefill scratch, allocated by the first prefill call for its chunk size
    // (grown by a later call with a larger chunk): prompt tokens [max_seq],
    // residual stream h [C][H] FP32, projection inputs x [C][max(H, Nq D, I)]
    // bf16 (also the attention output), queries q [C][Nq D] bf16, SwiGLU
    // activations act [C][I] bf16, projection outputs y [C][max(Q|K|V, 2 I,
    // H)] FP32 (at least the vocabulary: the last token's logits), (token,
    // position) of the greedy pick and its argmax ticket
    int pf_cap = 0;
    int* pf_tokens = nullptr;
    float* pf_h = nullptr;
    uint16_t* pf_x = nullptr;
    uint16_t* pf_q = nullptr;
    uint16_t* pf_act = nullptr;  // [C][I] bf16 SwiGLU activations (the gate/up projection's output)
    float* pf_y = nullptr;
    int* pf_tok = nullptr;
    unsigned* pf_ticket = nullptr;
    // tensor parallelism over `world` ranks (one process per GPU): this rank
    // holds query heads [rank nq_l, ..), KV heads [rank nkv_l, ..),
    // intermediate rows [rank il, ..) and vocabulary rows [v0, v0 + vl) of the
    // LM head (padded with zero rows to vlp, a multiple of 128); world = 1
    // holds everything.  comm: the NCCL communicator of the ranks; ysum
    // [T][H] a rank's O / down sums, all-reduced in place; cand [T] and
    // cand_all [world][T] the (value, id) argmax candidates.
    int rank = 0, world = 1;
    int nq_l = 0, nkv_l = 0, il = 0, v0 = 0, vl = 0, vlp = 0;
    void* comm = nullptr;
    float* ysum = nullptr;
    int2* cand = nullptr;
    int2* cand_all = nullptr;
    // the sums after O and down cross the ranks by the peer-memory exchange
    // (tp_peer, the default: tp_push into every rank's region over NVLink,
    // bt_resid_norm_tp adds them) or by ncclAllReduce (the baseline).  xch:
    // this rank's region [2][world][T][H] tagged words; peer_tab [world]:
    // every rank's region mapped here (CUDA IPC); epoch: step counter of the
    // exchange tags
    bool tp_peer = true;
    unsigned long long* xch = nullptr;
    unsigned long long** peer_tab = nullptr;
    std::vector<void*> opened;
    unsigned* epoch = nullptr;
    long long wait_cycles = 4000000000ll;  // about 2 s at the maximum SM clock
    // token choice: greedy (sample_inv_t = 0) or temperature sampling by
    // Gumbel-max inside the argmax kernels, keyed by (sample_seed, position)
    float sample_inv_t = 0.0f;
    uint64_t sample_seed = 0;
    // paged KV caches (page_size > 0): kc / vc of a layer are pools
    // [num_pages][nkv][page_size][D]; sequence t's position p lives in page
    // table[t][p / page_size] (table [T][max_pages], -1: no page; the host
    // copy is uploaded before a step once it changed).  A sequence at
    // position -1 is an empty slot.  Prefill runs on contiguous staging
    // caches st_k / st_v [nkv][max_seq][D] per layer (allocated by the first
    // paged prefill) and copies the rows into the pages.  salts [T]: the
    // per-sequence sampling keys (set_salts), or none.
    int page_size = 0, num_pages = 0, max_pages = 0;
    int* table = nullptr;
    std::vector<int> table_host;
    bool table_dirty = false;
    std::vector<uint16_t*> st_k, st_v;
    uint64_t* salts = nullptr;

    ~infernt_batch_engine() {
        if (graph) cudaGraphExecDestroy(graph);  // before the communicator its NCCL nodes use
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : opened) cudaIpcCloseMemHandle(p);
        if (comm) {
            if (const NcclApi* n = nccl_api()) n->destroy(static_cast<ncclComm_t>(comm));
        }
        cudaFree(hist);
        if (ev[0]) cudaEventDestroy(ev[0]);
        if (ev[1]) cudaEventDestroy(ev[1]);
        for (void* b : bufs) cudaFree(b);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

using infernt::fail;

int alloc(infernt_batch_engine* e, size_t bytes, void** out) {
    void* p = nullptr;
    INFERNT_CUDA_TRY(cudaMalloc(&p, bytes));
    e->bufs.push_back(p);
    *out = p;
    return INFERNT_OK;
}

// K splits of a projection: tiles x splits CTAs of ceil(nk / splits) weight
// stages each.  The busiest SM streams ceil(ctas / sms) CTAs' stages, and
// every wave of resident CTAs adds a fixed cost (pipeline fill, epilogue) of
// about two stages; the split count with the least such cost wins (ties go
// to fewer partials).  At most 8 splits: the finishing kernels add the
// partials in one round of loads (fewer registers than 16).
int pick_splits(int N, int K, int T) {
    const int tiles = N / 128, nk = K / 64, sms = infernt::sm_count();
    const int slots = sms * infernt::bgemm_ctas_per_sm((T + 15) / 16 * 16);
    int best = 1;
    long best_cost = -1;
    for (int s = 1; s <= 8 && s <= nk; ++s) {
        const long ctas = (long)tiles * s;
        const long cost = (ctas + sms - 1) / sms * ((nk + s - 1) / s) + 2 * ((ctas + slots - 1) / slots);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

int fill_bf16(infernt_batch_engine* e, void* dst, size_t n, uint64_t seed, uint64_t stream_id, float std_dev) {
    return infernt_fill_normal(dst, n, INFERNT_DTYPE_BF16, seed, stream_id, std_dev, e->stream);
}

// The rank's shard of the seeded model (the values a single-GPU engine of
// the same seed holds, as windows of the full matrices): Q|K|V rows of its
// query and KV heads stacked, the matching O columns, its gate and up rows
// stacked, the matching down columns, LM-head rows [v0, v0 + vl) (zero rows
// up to vlp); the embedding and norms whole.
int build(infernt_batch_engine* e, uint64_t seed, float std_dev) {
    const infernt_llama_config& c = e->cfg;
    const int H = c.hidden_size, V = c.vocab_size, D = c.head_dim, L = c.num_layers, I = c.intermediate_size;
    const int T = e->T, r = e->rank;
    const int nq = e->nq_l, nkv = e->nkv_l, il = e->il;
    const int qs = c.num_attention_heads * D, qsl = nq * D, kvsl = nkv * D, nqkv = qsl + 2 * kvsl;
    const int bf = INFERNT_DTYPE_BF16;
    INFERNT_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    auto window = [&](void* dst, int rows, int cols, int ld, long long src_ld, long long row0, long long col0,
                      uint64_t stream_id) {
        return infernt_fill_normal_window(dst, rows, cols, ld, (uint64_t)src_ld, (uint64_t)row0, (uint64_t)col0, bf,
                                          seed, stream_id, std_dev, e->stream);
    };
    void* p = nullptr;
    // embedding (FP32) and norms
    if (int s = alloc(e, sizeof(float) * (size_t)V * H, &p)) return s;
    if (int s = infernt_fill_normal(p, (size_t)V * H, INFERNT_DTYPE_F32, seed, INFERNT_STREAM_EMBEDDING, std_dev,
                                    e->stream))
        return s;
    e->emb = static_cast<const float*>(p);
    float* ones = nullptr;
    if (int s = alloc(e, sizeof(float) * H, reinterpret_cast<void**>(&ones))) return s;
    if (int s = infernt_fill_const(ones, H, 1.0f, e->stream)) return s;
    e->final_norm = ones;  // every norm weight is 1.0 in the seeded model
    if (int s = alloc(e, (size_t)e->vlp * H * 2, &p)) return s;
    INFERNT_CUDA_TRY(cudaMemsetAsync(p, 0, (size_t)e->vlp * H * 2, e->stream));
    if (int s = window(p, e->vl, H, H, H, e->v0, 0, INFERNT_STREAM_LM_HEAD)) return s;
    e->lm = p;
    for (int l = 0; l < L; ++l) {
        infernt_batch_engine::Layer ly;
        ly.attn_norm = ones;
        ly.ffn_norm = ones;
        char* qkv = nullptr;
        if (int s = alloc(e, (size_t)nqkv * H * 2, reinterpret_cast<void**>(&qkv))) return s;
        if (int s = window(qkv, qsl, H, H, H, (long long)r * qsl, 0, INFERNT_STREAM_LAYER(l, 0))) return s;
        if (int s = window(qkv + (size_t)qsl * H * 2, kvsl, H, H, H, (long long)r * kvsl, 0, INFERNT_STREAM_LAYER(l, 1)))
            return s;
        if (int s = window(qkv + (size_t)(qsl + kvsl) * H * 2, kvsl, H, H, H, (long long)r * kvsl, 0,
                           INFERNT_STREAM_LAYER(l, 2)))
            return s;
        ly.qkv = qkv;
        if (int s = alloc(e, (size_t)H * qsl * 2, &p)) return s;
        if (int s = window(p, H, qsl, qsl, qs, 0, (long long)r * qsl, INFERNT_STREAM_LAYER(l, 3))) return s;
        ly.o = p;
        char* gu = nullptr;
        if (int s = alloc(e, (size_t)2 * il * H * 2, reinterpret_cast<void**>(&gu))) return s;
        if (int s = window(gu, il, H, H, H, (long long)r * il, 0, INFERNT_STREAM_LAYER(l, 4))) return s;
        if (int s = window(gu + (size_t)il * H * 2, il, H, H, H, (long long)r * il, 0, INFERNT_STREAM_LAYER(l, 5)))
            return s;
        ly.gu = gu;
        if (int s = alloc(e, (size_t)H * il * 2, &p)) return s;
        if (int s = window(p, H, il, il, I, 0, (long long)r * il, INFERNT_STREAM_LAYER(l, 6))) return s;
        ly.down = p;
        e->layers.push_back(ly);
        const size_t cache = e->page_size ? (size_t)e->num_pages * nkv * e->page_size * D * 2
                                          : (size_t)T * nkv * c.max_seq_len * D * 2;
        void* k = nullptr;
        void* v = nullptr;
        if (int s = alloc(e, cache, &k)) return s;
        if (int s = alloc(e, cache, &v)) return s;
        INFERNT_CUDA_TRY(cudaMemsetAsync(k, 0, cache, e->stream));
        INFERNT_CUDA_TRY(cudaMemsetAsync(v, 0, cache, e->stream));
        e->kc.push_back(static_cast<uint16_t*>(k));
        e->vc.push_back(static_cast<uint16_t*>(v));
    }
    e->sp_qkv = pick_splits(nqkv, H, T);
    e->sp_o = pick_splits(H, qsl, T);
    e->sp_gu = pick_splits(2 * il, H, T);
    e->sp_down = pick_splits(H, il, T);
    e->sp_lm = 1;  // the argmax reads whole logits
    size_t part = 0;
    auto need = [&](int sp, int N) {
        const size_t b = (size_t)sp * T * N;
        if (b > part) part = b;
    };
    need(e->sp_qkv, nqkv);
    need(e->sp_o, H);
    need(e->sp_gu, 2 * il);
    need(e->sp_down, H);
    need(e->sp_lm, e->vlp);
    const int kmax = H > qsl ? (H > il ? H : il) : (qsl > il ? qsl : il);
    if (int s = alloc(e, sizeof(int) * T, reinterpret_cast<void**>(&e->tokens))) return s;
    if (int s = alloc(e, sizeof(int) * T, reinterpret_cast<void**>(&e->positions))) return s;
    if (int s = alloc(e, 256, reinterpret_cast<void**>(&e->err))) return s;
    INFERNT_CUDA_TRY(cudaMemsetAsync(e->err, 0, 256, e->stream));
    if (int s = alloc(e, sizeof(float) * (size_t)T * H, reinterpret_cast<void**>(&e->h))) return s;
    if (int s = alloc(e, (size_t)T * kmax * 2, reinterpret_cast<void**>(&e->xb))) return s;
    if (int s = alloc(e, (size_t)T * qsl * 2, reinterpret_cast<void**>(&e->attn))) return s;
    if (int s = alloc(e, (size_t)T * il * 2, reinterpret_cast<void**>(&e->act))) return s;
    if (int s = alloc(e, sizeof(float) * (size_t)T * qsl, reinterpret_cast<void**>(&e->q))) return s;
    if (int s = alloc(e, sizeof(float) * part, reinterpret_cast<void**>(&e->part))) return s;
    const int G = nq / nkv;
    if (int s = alloc(e, sizeof(float) * (size_t)T * nkv * e->S * G * (D + 2), reinterpret_cast<void**>(&e->apart)))
        return s;
    if (int s = alloc(e, sizeof(unsigned) * (size_t)T * nkv, reinterpret_cast<void**>(&e->tickets))) return s;
    INFERNT_CUDA_TRY(cudaMemsetAsync(e->tickets, 0, sizeof(unsigned) * (size_t)T * nkv, e->stream));
    if (int s = alloc(e, sizeof(unsigned) * T, reinterpret_cast<void**>(&e->am_tickets))) return s;
    INFERNT_CUDA_TRY(cudaMemsetAsync(e->am_tickets, 0, sizeof(unsigned) * T, e->stream));
    if (int s = alloc(e, sizeof(float) * T * 8, reinterpret_cast<void**>(&e->cand_v))) return s;
    if (int s = alloc(e, sizeof(int) * T * 8, reinterpret_cast<void**>(&e->cand_i))) return s;
    if (e->world > 1) {
        const size_t xb_bytes = sizeof(unsigned long long) * 2 * (size_t)e->world * T * H;
        if (int s = alloc(e, xb_bytes, reinterpret_cast<void**>(&e->xch))) return s;
        INFERNT_CUDA_TRY(cudaMemsetAsync(e->xch, 0, xb_bytes, e->stream));
        if (int s = alloc(e, 256, reinterpret_cast<void**>(&e->epoch))) return s;
        INFERNT_CUDA_TRY(cudaMemsetAsync(e->epoch, 0, 256, e->stream));
        if (int s = alloc(e, sizeof(void*) * (size_t)e->world, reinterpret_cast<void**>(&e->peer_tab))) return s;
        if (int s = alloc(e, sizeof(float) * (size_t)T * H, reinterpret_cast<void**>(&e->ysum))) return s;
        if (int s = alloc(e, sizeof(int2) * (size_t)T, reinterpret_cast<void**>(&e->cand))) return s;
        if (int s = alloc(e, sizeof(int2) * (size_t)T * e->world, reinterpret_cast<void**>(&e->cand_all))) return s;
    }
    if (e->page_size) {
        e->max_pages = (c.max_seq_len + e->page_size - 1) / e->page_size;
        const size_t tb = sizeof(int) * (size_t)T * e->max_pages;
        if (int s = alloc(e, tb, reinterpret_cast<void**>(&e->table))) return s;
        INFERNT_CUDA_TRY(cudaMemsetAsync(e->table, 0xff, tb, e->stream));
        e->table_host.assign((size_t)T * e->max_pages, -1);
    }
    if (int s = alloc(e, sizeof(float2) * (size_t)c.max_seq_len * (D / 2), reinterpret_cast<void**>(&e->rope)))
        return s;
    if (int s = infernt::bt_rope_table_launch(e->rope, c.max_seq_len, D, c.rope_theta, e->stream)) return s;
    INFERNT_CUDA_TRY(cudaEventCreate(&e->ev[0]));
    INFERNT_CUDA_TRY(cudaEventCreate(&e->ev[1]));
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    return INFERNT_OK;
}

// The sum over the ranks of y [T][H] in place (tensor parallelism).
int all_reduce(infernt_batch_engine* e, float* y, cudaStream_t st, size_t count = 0) {
    const NcclApi* n = nccl_api();
    if (!count) count = (size_t)e->T * e->cfg.hidden_size;
    const ncclResult_t r = n->all_reduce(y, y, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(e->comm), st);
    return r == ncclSuccess ? INFERNT_OK : fail(INFERNT_ERR_CUDA, "ncclAllReduce: %s", n->err_str(r));
}

// Residual add + RMSNorm of an O or down projection (the step's idx-th
// exchange): its split partials summed in order (one rank), or summed per
// rank and then over the ranks (peer-memory exchange, or NCCL).
int resid_norm(infernt_batch_engine* e, int splits, const float* norm_w, int idx, cudaStream_t st) {
    const infernt_llama_config& c = e->cfg;
    const int H = c.hidden_size, T = e->T;
    using namespace infernt;
    if (e->world == 1) return bt_resid_norm_launch(e->part, splits, T, H, e->h, norm_w, c.rms_norm_eps, e->xb, st);
    if (e->tp_peer) {
        const int per_step = 2 * c.num_layers;
        if (int s = tp_push_launch(e->part, splits, T, H, e->peer_tab, e->rank, e->world, e->epoch, per_step, idx, st))
            return s;
        return bt_resid_norm_tp_launch(e->xch, e->world, T, H, e->h, norm_w, c.rms_norm_eps, e->xb, e->epoch, per_step,
                                       idx, e->err, e->wait_cycles, st);
    }
    if (int s = tp_sum_splits_launch(e->part, splits, T, H, e->ysum, st)) return s;
    if (int s = all_reduce(e, e->ysum, st)) return s;
    return bt_resid_norm_launch(e->ysum, 1, T, H, e->h, norm_w, c.rms_norm_eps, e->xb, st);
}

// One decode step of every sequence (launches only; the caller synchronises).
int record_step(infernt_batch_engine* e, cudaStream_t st) {
    const infernt_llama_config& c = e->cfg;
    const int H = c.hidden_size, V = c.vocab_size, D = c.head_dim, L = c.num_layers;
    const int nq = e->nq_l, nkv = e->nkv_l, il = e->il, T = e->T;
    const int qsl = nq * D, nqkv = qsl + 2 * nkv * D;
    const float eps = c.rms_norm_eps;
    using namespace infernt;
    if (e->world > 1 && e->tp_peer)
        if (int s = bt_epoch_advance_launch(e->epoch, st)) return s;
    if (int s = bt_embed_norm_launch(e->emb, e->tokens, V, T, H, e->layers[0].attn_norm, eps, e->h, e->xb, e->err, st))
        return s;
    for (int l = 0; l < L; ++l) {
        const auto& ly = e->layers[l];
        if (int s = bgemm_launch(ly.qkv, nqkv, H, e->xb, T, e->part, e->sp_qkv, e->err, st)) return s;
        if (nq / nkv <= 8) {
            // Q|K|V finishing inside the tensor-core attention
            if (int s = bt_attention_fused_launch(e->part, e->sp_qkv, e->rope, e->kc[l], e->vc[l], e->positions, T, nq,
                                                  nkv, D, c.max_seq_len, e->S, e->min_chunk, e->stages, e->apart,
                                                  e->attn, e->err, e->tickets, st, e->table, e->page_size,
                                                  e->max_pages))
                return s;
        } else {
            if (int s = bt_qkv_finish_launch(e->part, e->sp_qkv, T, nq, nkv, D, e->positions, e->rope, c.max_seq_len,
                                             e->q, e->kc[l], e->vc[l], e->err, st))
                return s;
            if (int s = bt_attention_launch(e->q, e->kc[l], e->vc[l], e->positions, T, nq, nkv, D, c.max_seq_len, e->S,
                                            e->min_chunk, e->stages, e->apart, e->attn, st))
                return s;
        }
        if (int s = bgemm_launch(ly.o, H, qsl, e->attn, T, e->part, e->sp_o, e->err, st)) return s;
        if (int s = resid_norm(e, e->sp_o, ly.ffn_norm, 2 * l, st)) return s;
        if (int s = bgemm_launch(ly.gu, 2 * il, H, e->xb, T, e->part, e->sp_gu, e->err, st)) return s;
        if (int s = bt_swiglu_launch(e->part, e->sp_gu, T, il, e->act, st)) return s;
        if (int s = bgemm_launch(ly.down, H, il, e->act, T, e->part, e->sp_down, e->err, st)) return s;
        const float* next_norm = l + 1 < L ? e->layers[l + 1].attn_norm : e->final_norm;
        if (int s = resid_norm(e, e->sp_down, next_norm, 2 * l + 1, st)) return s;
    }
    if (int s = bgemm_launch(e->lm, e->vlp, H, e->xb, T, e->part, e->sp_lm, e->err, st)) return s;
    // the LM head runs unsplit: part[0] holds the logits [T][vlp]
    if (e->world == 1)
        return bt_argmax_launch(e->part, T, V, e->tokens, e->positions, nullptr, e->cand_v, e->cand_i, e->am_tickets,
                                e->sample_inv_t, e->sample_seed, st, e->salts);
    if (int s = tp_argmax_local_launch(e->part, T, e->vlp, e->vl, e->v0, e->cand, e->positions, e->sample_inv_t,
                                       e->sample_seed, st))
        return s;
    const NcclApi* n = nccl_api();
    const ncclResult_t r =
        n->all_gather(e->cand, e->cand_all, (size_t)2 * T, ncclInt32, static_cast<ncclComm_t>(e->comm), st);
    if (r != ncclSuccess) return fail(INFERNT_ERR_CUDA, "ncclAllGather: %s", n->err_str(r));
    return tp_argmax_pick_launch(e->cand_all, e->world, T, e->tokens, e->positions, st);
}

int ensure_graph(infernt_batch_engine* e) {
    if (e->graph) return INFERNT_OK;
    cudaStream_t cap = nullptr;
    INFERNT_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    cudaError_t ce = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    int s = ce == cudaSuccess ? record_step(e, cap) : INFERNT_ERR_CUDA;
    cudaGraph_t g = nullptr;
    const cudaError_t ee = cudaStreamEndCapture(cap, &g);
    cudaStreamDestroy(cap);
    if (ce != cudaSuccess) return infernt::cuda_fail(ce, "batch engine: stream capture");
    if (s) {
        if (g) cudaGraphDestroy(g);
        return s;
    }
    INFERNT_CUDA_TRY(ee);
    const cudaError_t ie = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    INFERNT_CUDA_TRY(ie);
    return INFERNT_OK;
}

// Every rank's exchange region mapped into this process: the CUDA IPC
// handles gathered over the ranks' NCCL communicator at creation.
int map_peers(infernt_batch_engine* e, const NcclApi* nccl) {
    const int W = e->world;
    cudaIpcMemHandle_t h;
    INFERNT_CUDA_TRY(cudaIpcGetMemHandle(&h, e->xch));
    char* d_h = nullptr;
    if (int s = alloc(e, sizeof(h) * (size_t)(W + 1), reinterpret_cast<void**>(&d_h))) return s;
    INFERNT_CUDA_TRY(cudaMemcpy(d_h, &h, sizeof(h), cudaMemcpyHostToDevice));
    const ncclResult_t r = nccl->all_gather(d_h, d_h + sizeof(h), sizeof(h), ncclUint8,
                                            static_cast<ncclComm_t>(e->comm), e->stream);
    if (r != ncclSuccess) return fail(INFERNT_ERR_CUDA, "ncclAllGather (exchange handles): %s", nccl->err_str(r));
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    std::vector<cudaIpcMemHandle_t> all(W);
    INFERNT_CUDA_TRY(cudaMemcpy(all.data(), d_h + sizeof(h), sizeof(h) * (size_t)W, cudaMemcpyDeviceToHost));
    std::vector<unsigned long long*> tab(W, nullptr);
    for (int q = 0; q < W; ++q) {
        if (q == e->rank) {
            tab[q] = e->xch;
            continue;
        }
        void* ptr = nullptr;
        INFERNT_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, all[q], cudaIpcMemLazyEnablePeerAccess));
        e->opened.push_back(ptr);
        tab[q] = static_cast<unsigned long long*>(ptr);
    }
    INFERNT_CUDA_TRY(cudaMemcpy(e->peer_tab, tab.data(), sizeof(void*) * (size_t)W, cudaMemcpyHostToDevice));
    return INFERNT_OK;
}

int check_err(infernt_batch_engine* e) {
    unsigned err = 0;
    INFERNT_CUDA_TRY(cudaMemcpyAsync(&err, e->err, sizeof(err), cudaMemcpyDeviceToHost, e->stream));
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if (err) {
        cudaMemsetAsync(e->err, 0, sizeof(unsigned), e->stream);
        cudaStreamSynchronize(e->stream);
        return fail(INFERNT_ERR_DEVICE, "batched decode reported error word 0x%x (1: wait timeout, 2: position, "
                                        "4: token id)", err);
    }
    return INFERNT_OK;
}

void release(infernt_batch_engine* e, void* p) {
    if (!p) return;
    for (auto it = e->bufs.begin(); it != e->bufs.end(); ++it)
        if (*it == p) {
            e->bufs.erase(it);
            break;
        }
    cudaFree(p);
}

// Prefill scratch for chunks of up to C tokens.
int grow_prefill(infernt_batch_engine* e, int C) {
    if (C <= e->pf_cap) return INFERNT_OK;
    const infernt_llama_config& c = e->cfg;
    const int H = c.hidden_size, I = c.intermediate_size, D = c.head_dim;
    const int qs = c.num_attention_heads * D, nqkv = qs + 2 * c.num_key_value_heads * D;
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    release(e, e->pf_h);
    release(e, e->pf_x);
    release(e, e->pf_q);
    release(e, e->pf_act);
    release(e, e->pf_y);
    e->pf_h = nullptr;
    e->pf_x = e->pf_q = e->pf_act = nullptr;
    e->pf_y = nullptr;
    e->pf_cap = 0;
    if (!e->pf_tokens) {
        if (int s = alloc(e, sizeof(int) * (size_t)c.max_seq_len, reinterpret_cast<void**>(&e->pf_tokens))) return s;
        if (int s = alloc(e, 256, reinterpret_cast<void**>(&e->pf_tok))) return s;
        if (int s = alloc(e, 256, reinterpret_cast<void**>(&e->pf_ticket))) return s;
        INFERNT_CUDA_TRY(cudaMemsetAsync(e->pf_ticket, 0, 256, e->stream));
    }
    const size_t kx = (size_t)(H > qs ? (H > I ? H : I) : (qs > I ? qs : I));
    size_t ny = (size_t)(nqkv > 2 * I ? nqkv : 2 * I);
    if ((size_t)H > ny) ny = H;
    size_t y_floats = (size_t)C * ny;
    if (y_floats < (size_t)c.vocab_size) y_floats = c.vocab_size;
    if (int s = alloc(e, sizeof(float) * (size_t)C * H, reinterpret_cast<void**>(&e->pf_h))) return s;
    if (int s = alloc(e, (size_t)C * kx * 2, reinterpret_cast<void**>(&e->pf_x))) return s;
    if (int s = alloc(e, (size_t)C * qs * 2, reinterpret_cast<void**>(&e->pf_q))) return s;
    if (int s = alloc(e, (size_t)C * I * 2, reinterpret_cast<void**>(&e->pf_act))) return s;
    if (int s = alloc(e, sizeof(float) * y_floats, reinterpret_cast<void**>(&e->pf_y))) return s;
    e->pf_cap = C;
    return INFERNT_OK;
}

// Staging caches of a paged engine's prefill: [nkv][max_seq][D] K and V per
// layer.
int grow_staging(infernt_batch_engine* e) {
    if (!e->st_k.empty()) return INFERNT_OK;
    const infernt_llama_config& c = e->cfg;
    const size_t bytes = (size_t)e->nkv_l * c.max_seq_len * c.head_dim * 2;
    for (int l = 0; l < c.num_layers; ++l) {
        void* k = nullptr;
        void* v = nullptr;
        if (int s = alloc(e, bytes, &k)) return s;
        if (int s = alloc(e, bytes, &v)) return s;
        e->st_k.push_back(static_cast<uint16_t*>(k));
        e->st_v.push_back(static_cast<uint16_t*>(v));
    }
    return INFERNT_OK;
}

// Rows [p0, p1) of sequence seq, every layer, from its pages into the
// staging caches (to_pages false) or back.
int stage_rows(infernt_batch_engine* e, int seq, int p0, int p1, bool to_pages) {
    const infernt_llama_config& c = e->cfg;
    const int* pages = e->table + (size_t)seq * e->max_pages;
    for (int l = 0; l < c.num_layers; ++l) {
        if (int s = infernt::bt_page_copy_launch(e->kc[l], e->st_k[l], pages, e->page_size, e->nkv_l, c.max_seq_len,
                                                 c.head_dim, p0, p1, to_pages, e->stream))
            return s;
        if (int s = infernt::bt_page_copy_launch(e->vc[l], e->st_v[l], pages, e->page_size, e->nkv_l, c.max_seq_len,
                                                 c.head_dim, p0, p1, to_pages, e->stream))
            return s;
    }
    return INFERNT_OK;
}

// Prefill of sequence `seq`: prompt tokens pf_tokens[0, n) at positions
// [start, start + n) in chunks of C, every layer per chunk; then the LM head
// and argmax of the last token (its logits in pf_y[0, V), the greedy token
// in pf_tok[0]).  A tensor-parallel rank runs its shards (query and KV
// heads, intermediate rows, vocabulary rows) and sums the O and down
// projections' partial rows [m][H] over the ranks with ncclAllReduce before
// each residual add (the chunk's rows are too many for the decode step's
// peer-memory exchange region); the last token's argmax candidates of every
// rank meet by ncclAllGather, as in the decode step.  Every rank must call
// it with the same arguments.  Launches only.
int record_prefill(infernt_batch_engine* e, int seq, int n, int start, int C, cudaStream_t st) {
    const infernt_llama_config& c = e->cfg;
    const int H = c.hidden_size, V = c.vocab_size, D = c.head_dim, L = c.num_layers, I = e->il;
    const int nq = e->nq_l, nkv = e->nkv_l, S = c.max_seq_len;
    const int qs = nq * D, nqkv = qs + 2 * nkv * D;
    const bool tp = e->world > 1;
    const float eps = c.rms_norm_eps;
    // the sequence's contiguous caches: its rows of [T][nkv][S][D], or the
    // staging caches of a paged engine
    const bool paged = e->page_size > 0;
    const size_t seq_off = paged ? 0 : (size_t)seq * nkv * S * D;
    const std::vector<uint16_t*>& kcs = paged ? e->st_k : e->kc;
    const std::vector<uint16_t*>& vcs = paged ? e->st_v : e->vc;
    using namespace infernt;
    int m = 0;
    for (int c0 = 0; c0 < n; c0 += C) {
        m = n - c0 < C ? n - c0 : C;
        const int p0 = start + c0;
        if (int s = bt_embed_norm_launch(e->emb, e->pf_tokens + c0, V, m, H, e->layers[0].attn_norm, eps, e->pf_h,
                                         e->pf_x, e->err, st))
            return s;
        for (int l = 0; l < L; ++l) {
            const auto& ly = e->layers[l];
            uint16_t* kc = kcs[l] + seq_off;
            uint16_t* vc = vcs[l] + seq_off;
            if (int s = pgemm_launch(ly.qkv, nqkv, H, e->pf_x, m, e->pf_y, nqkv, e->err, st)) return s;
            if (int s = pf_qkv_rope_launch(e->pf_y, m, p0, nq, nkv, D, e->rope, S, e->pf_q, kc, vc, st)) return s;
            if (int s = pf_attention_launch(e->pf_q, kc, vc, m, p0, nq, nkv, D, S, e->pf_x, e->err, 1, st)) return s;
            if (int s = pgemm_launch(ly.o, H, qs, e->pf_x, m, e->pf_y, H, e->err, st)) return s;
            if (tp)
                if (int s = all_reduce(e, e->pf_y, st, (size_t)m * H)) return s;
            if (int s = bt_resid_norm_launch(e->pf_y, 1, m, H, e->pf_h, ly.ffn_norm, eps, e->pf_x, st)) return s;
            // gate/up with SwiGLU in its epilogue: bf16 activations, no FP32 gate/up rows
            if (int s = pgemm_swiglu_launch(ly.gu, I, H, e->pf_x, m, e->pf_act, I, e->err, st)) return s;
            if (int s = pgemm_launch(ly.down, H, I, e->pf_act, m, e->pf_y, H, e->err, st)) return s;
            if (tp)
                if (int s = all_reduce(e, e->pf_y, st, (size_t)m * H)) return s;
            const float* next_norm = l + 1 < L ? e->layers[l + 1].attn_norm : e->final_norm;
            if (int s = bt_resid_norm_launch(e->pf_y, 1, m, H, e->pf_h, next_norm, eps, e->pf_x, st)) return s;
        }
    }
    // the last token's final-normed row is row m - 1 of the last chunk
    if (!tp) {
        if (int s = bgemm_launch(e->lm, V, H, e->pf_x + (size_t)(m - 1) * H, 1, e->pf_y, 1, e->err, st)) return s;
        return bt_argmax_launch(e->pf_y, 1, V, e->pf_tok, e->pf_tok + 1, nullptr, e->cand_v, e->cand_i, e->pf_ticket,
                                e->sample_inv_t, e->sample_seed, st, e->salts ? e->salts + seq : nullptr);
    }
    // this rank's vocabulary rows (zero-padded to vlp), its candidate, then
    // the winner over the ranks' candidates
    if (int s = bgemm_launch(e->lm, e->vlp, H, e->pf_x + (size_t)(m - 1) * H, 1, e->pf_y, 1, e->err, st)) return s;
    if (int s = tp_argmax_local_launch(e->pf_y, 1, e->vlp, e->vl, e->v0, e->cand, e->pf_tok + 1, e->sample_inv_t,
                                       e->sample_seed, st))
        return s;
    const NcclApi* nc = nccl_api();
    const ncclResult_t r =
        nc->all_gather(e->cand, e->cand_all, (size_t)2, ncclInt32, static_cast<ncclComm_t>(e->comm), st);
    if (r != ncclSuccess) return fail(INFERNT_ERR_CUDA, "ncclAllGather: %s", nc->err_str(r));
    return tp_argmax_pick_launch(e->cand_all, e->world, 1, e->pf_tok, e->pf_tok + 1, st);
}

// Whether the block table gives sequence t pages for positions [0, last].
bool pages_cover(const infernt_batch_engine* e, int t, int last) {
    const int* row = e->table_host.data() + (size_t)t * e->max_pages;
    for (int i = 0; i <= last / e->page_size; ++i)
        if (row[i] < 0) return false;
    return true;
}

// The host block table on the device (before a step that reads it).
int upload_table(infernt_batch_engine* e) {
    if (!e->page_size || !e->table_dirty) return INFERNT_OK;
    INFERNT_CUDA_TRY(cudaMemcpyAsync(e->table, e->table_host.data(), sizeof(int) * e->table_host.size(),
                                     cudaMemcpyHostToDevice, e->stream));
    e->table_dirty = false;
    return INFERNT_OK;
}

// Token and position per sequence for the next steps (`steps` of them);
// a paged engine takes position -1 for an empty slot and needs pages
// through the last position the steps write.
int set_inputs(infernt_batch_engine* e, const int* tokens, const int* positions, int steps = 1) {
    const bool paged = e->page_size > 0;
    for (int t = 0; t < e->T; ++t) {
        INFERNT_REQUIRE(tokens[t] >= 0 && tokens[t] < e->cfg.vocab_size, "batch engine: token %d of sequence %d",
                        tokens[t], t);
        if (paged && positions[t] == -1) continue;
        INFERNT_REQUIRE(positions[t] >= 0 && positions[t] < e->cfg.max_seq_len,
                        "batch engine: position %d of sequence %d outside [0, %d)", positions[t], t,
                        e->cfg.max_seq_len);
        INFERNT_REQUIRE(!paged || pages_cover(e, t, positions[t] + steps - 1),
                        "batch engine: sequence %d has no page for a position in [0, %d]", t,
                        positions[t] + steps - 1);
    }
    if (int s = upload_table(e)) return s;
    INFERNT_CUDA_TRY(cudaMemcpyAsync(e->tokens, tokens, sizeof(int) * e->T, cudaMemcpyHostToDevice, e->stream));
    INFERNT_CUDA_TRY(cudaMemcpyAsync(e->positions, positions, sizeof(int) * e->T, cudaMemcpyHostToDevice, e->stream));
    return INFERNT_OK;
}

// An engine of `batch` sequences: contiguous caches (page_size 0) or pools
// of num_pages pages of page_size positions.
int create_engine(const infernt_llama_config* cfg, int batch, uint64_t seed, float std_dev, int attn_splits, int rank,
                  int world, const void* nccl_id, int page_size, int num_pages, infernt_batch_engine** out) {
    INFERNT_REQUIRE(cfg && out, "batch_engine_create: null argument");
    *out = nullptr;
    INFERNT_REQUIRE(cfg->weight_dtype == INFERNT_DTYPE_BF16, "batch engine: bf16 weights only");
    INFERNT_REQUIRE(batch >= 1 && batch <= 256, "batch engine: batch %d outside [1, 256]", batch);
    INFERNT_REQUIRE(world >= 1 && world <= 64 && rank >= 0 && rank < world, "batch engine: rank %d of %d", rank, world);
    INFERNT_REQUIRE(world == 1 || nccl_id, "batch engine: %d ranks need an NCCL unique id", world);
    const int D = cfg->head_dim;
    INFERNT_REQUIRE(D == 64 || D == 128, "batch engine: head_dim %d (64 or 128)", D);
    INFERNT_REQUIRE(cfg->num_attention_heads % cfg->num_key_value_heads == 0 &&
                        cfg->num_attention_heads / cfg->num_key_value_heads <= 16,
                    "batch engine: query group size above 16");
    const int qs = cfg->num_attention_heads * D, kvs = cfg->num_key_value_heads * D;
    INFERNT_REQUIRE(cfg->hidden_size % 128 == 0 && qs % 128 == 0 && (qs + 2 * kvs) % 128 == 0 &&
                        cfg->intermediate_size % 128 == 0 && cfg->vocab_size % 128 == 0,
                    "batch engine: hidden, heads x head_dim, Q|K|V rows, intermediate and vocabulary must be "
                    "multiples of 128");
    INFERNT_REQUIRE(cfg->max_seq_len <= (1 << 20), "batch engine: max_seq_len above 2^20");
    // a rank's shard must keep the tensor-core tile shapes: Q|K|V and gate|up
    // rows multiples of 128, O and down K multiples of 64
    const int nq_l = cfg->num_attention_heads / world, nkv_l = cfg->num_key_value_heads / world;
    const int il = cfg->intermediate_size / world;
    INFERNT_REQUIRE(cfg->num_key_value_heads % world == 0 && (nq_l + 2 * nkv_l) * D % 128 == 0 &&
                        nq_l * D % 64 == 0 && cfg->intermediate_size % world == 0 && il % 64 == 0,
                    "batch engine: %d ranks do not split the KV heads, Q|K|V rows or intermediate rows into "
                    "tensor-core tiles",
                    world);
    const NcclApi* nccl = nullptr;
    if (world > 1) {
        nccl = nccl_api();
        INFERNT_REQUIRE(nccl, "batch engine: libnccl.so.2 is not loadable (needed for %d ranks)", world);
    }
    infernt_batch_engine* e = new (std::nothrow) infernt_batch_engine();
    INFERNT_REQUIRE(e, "batch_engine_create: host allocation failed");
    e->cfg = *cfg;
    e->T = batch;
    e->rank = rank;
    e->world = world;
    e->nq_l = nq_l;
    e->nkv_l = nkv_l;
    e->il = il;
    e->v0 = (int)((long long)cfg->vocab_size * rank / world);
    e->vl = (int)((long long)cfg->vocab_size * (rank + 1) / world) - e->v0;
    e->vlp = (e->vl + 127) / 128 * 128;
    int S = attn_splits;
    if (S <= 0) {
        // one split (no merge) once the (sequence, KV head) pairs fill the
        // SMs; otherwise about two CTAs per SM
        const int pairs = batch * nkv_l, sms = infernt::sm_count();
        S = pairs >= sms ? 1 : (2 * sms + pairs - 1) / pairs;
        if (S > 64) S = 64;
    }
    e->S = S < 1 ? 1 : S;
    e->page_size = page_size;
    e->num_pages = num_pages;
    int s = build(e, seed, std_dev);
    if (!s && world > 1) {
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        ncclComm_t comm = nullptr;
        const ncclResult_t r = nccl->init(&comm, world, id, rank);
        if (r != ncclSuccess)
            s = fail(INFERNT_ERR_CUDA, "ncclCommInitRank (rank %d of %d): %s", rank, world, nccl->err_str(r));
        else
            e->comm = comm;
        if (!s) s = map_peers(e, nccl);
    }
    if (s) {
        delete e;
        return s;
    }
    *out = e;
    return INFERNT_OK;
}

}  // namespace

extern "C" {

int infernt_batch_engine_create_tp(const infernt_llama_config* cfg, int batch, uint64_t seed, float std_dev,
                                   int attn_splits, int rank, int world, const void* nccl_id,
                                   infernt_batch_engine** out) {
    return create_engine(cfg, batch, seed, std_dev, attn_splits, rank, world, nccl_id, 0, 0, out);
}

int infernt_batch_engine_create_seeded(const infernt_llama_config* cfg, int batch, uint64_t seed, float std_dev,
                                       int attn_splits, infernt_batch_engine** out) {
    return create_engine(cfg, batch, seed, std_dev, attn_splits, 0, 1, nullptr, 0, 0, out);
}

int infernt_batch_engine_create_paged(const infernt_llama_config* cfg, int batch, int page_size, int num_pages,
                                      uint64_t seed, float std_dev, int attn_splits, infernt_batch_engine** out) {
    INFERNT_REQUIRE(cfg && out, "batch_engine_create_paged: null argument");
    *out = nullptr;
    INFERNT_REQUIRE(page_size >= 1 && page_size <= cfg->max_seq_len && num_pages >= 1,
                    "batch_engine_create_paged: %d pages of %d positions (max_seq_len %d)", num_pages, page_size,
                    cfg->max_seq_len);
    INFERNT_REQUIRE(cfg->num_key_value_heads >= 1 && cfg->num_attention_heads % cfg->num_key_value_heads == 0 &&
                        cfg->num_attention_heads / cfg->num_key_value_heads <= 8,
                    "batch_engine_create_paged: paged caches need query groups of at most 8 heads");
    INFERNT_REQUIRE((long long)num_pages * cfg->num_key_value_heads * page_size <= (1ll << 40),
                    "batch_engine_create_paged: pool of %d pages too large", num_pages);
    return create_engine(cfg, batch, seed, std_dev, attn_splits, 0, 1, nullptr, page_size, num_pages, out);
}

int infernt_batch_engine_set_pages(infernt_batch_engine* e, int seq, const int* pages, int n_pages) {
    INFERNT_REQUIRE(e, "batch_engine_set_pages: null engine");
    INFERNT_REQUIRE(e->page_size > 0, "batch_engine_set_pages: the engine's caches are not paged");
    INFERNT_REQUIRE(seq >= 0 && seq < e->T, "batch_engine_set_pages: sequence %d outside [0, %d)", seq, e->T);
    INFERNT_REQUIRE(n_pages >= 0 && n_pages <= e->max_pages && (n_pages == 0 || pages),
                    "batch_engine_set_pages: %d pages (at most %d per sequence)", n_pages, e->max_pages);
    for (int i = 0; i < n_pages; ++i)
        INFERNT_REQUIRE(pages[i] >= 0 && pages[i] < e->num_pages, "batch_engine_set_pages: page %d outside [0, %d)",
                        pages[i], e->num_pages);
    int* row = e->table_host.data() + (size_t)seq * e->max_pages;
    for (int i = 0; i < e->max_pages; ++i) row[i] = i < n_pages ? pages[i] : -1;
    e->table_dirty = true;
    return INFERNT_OK;
}

int infernt_batch_engine_paging(infernt_batch_engine* e, int* page_size, int* num_pages, int* max_pages) {
    INFERNT_REQUIRE(e && page_size && num_pages && max_pages, "batch_engine_paging: null argument");
    *page_size = e->page_size;
    *num_pages = e->num_pages;
    *max_pages = e->max_pages;
    return INFERNT_OK;
}

int infernt_batch_engine_set_salts(infernt_batch_engine* e, const uint64_t* salts) {
    INFERNT_REQUIRE(e, "batch_engine_set_salts: null engine");
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if (!salts) {
        if (e->salts) {
            release(e, e->salts);
            e->salts = nullptr;
            if (e->graph) {
                cudaGraphExecDestroy(e->graph);
                e->graph = nullptr;  // captured again at the next step
            }
        }
        return INFERNT_OK;
    }
    if (!e->salts) {
        if (int s = alloc(e, sizeof(uint64_t) * (size_t)e->T, reinterpret_cast<void**>(&e->salts))) return s;
        if (e->graph) {
            cudaGraphExecDestroy(e->graph);
            e->graph = nullptr;
        }
    }
    INFERNT_CUDA_TRY(cudaMemcpy(e->salts, salts, sizeof(uint64_t) * (size_t)e->T, cudaMemcpyHostToDevice));
    return INFERNT_OK;
}

int infernt_nccl_unique_id(void* out, size_t n) {
    INFERNT_REQUIRE(out && n >= sizeof(ncclUniqueId), "nccl_unique_id: need %zu bytes", sizeof(ncclUniqueId));
    const NcclApi* nccl = nccl_api();
    INFERNT_REQUIRE(nccl, "nccl_unique_id: libnccl.so.2 is not loadable");
    ncclUniqueId id;
    const ncclResult_t r = nccl->get_id(&id);
    if (r != ncclSuccess) return fail(INFERNT_ERR_CUDA, "ncclGetUniqueId: %s", nccl->err_str(r));
    std::memcpy(out, &id, sizeof(id));
    return INFERNT_OK;
}

int infernt_batch_engine_vocab_range(infernt_batch_engine* e, int* v0, int* vl) {
    INFERNT_REQUIRE(e && v0 && vl, "batch_engine_vocab_range: null argument");
    *v0 = e->v0;
    *vl = e->vl;
    return INFERNT_OK;
}

int infernt_batch_engine_destroy(infernt_batch_engine* e) {
    delete e;
    return INFERNT_OK;
}

int infernt_batch_engine_fill_kv(infernt_batch_engine* e, int seq, uint64_t seed, int n_pos, float std_dev) {
    INFERNT_REQUIRE(e && seq >= 0 && seq < e->T && n_pos >= 0 && n_pos <= e->cfg.max_seq_len,
                    "batch_engine_fill_kv: bad arguments");
    const int* pages = nullptr;
    if (e->page_size && n_pos > 0) {
        INFERNT_REQUIRE(pages_cover(e, seq, n_pos - 1), "batch_engine_fill_kv: sequence %d has no page for a position "
                        "below %d", seq, n_pos);
        if (int s = upload_table(e)) return s;
        pages = e->table + (size_t)seq * e->max_pages;
    }
    const uint64_t kk = infernt_stream_key(seed, INFERNT_STREAM_KV_K), vk = infernt_stream_key(seed, INFERNT_STREAM_KV_V);
    for (int l = 0; l < e->cfg.num_layers; ++l) {
        if (int s = infernt::bt_fill_kv_launch(e->kc[l], seq, l, e->nkv_l, e->cfg.max_seq_len, e->cfg.head_dim, n_pos,
                                               kk, std_dev, e->rank * e->nkv_l, e->cfg.num_key_value_heads, e->stream,
                                               pages, e->page_size))
            return s;
        if (int s = infernt::bt_fill_kv_launch(e->vc[l], seq, l, e->nkv_l, e->cfg.max_seq_len, e->cfg.head_dim, n_pos,
                                               vk, std_dev, e->rank * e->nkv_l, e->cfg.num_key_value_heads, e->stream,
                                               pages, e->page_size))
            return s;
    }
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    return INFERNT_OK;
}

int infernt_batch_engine_step(infernt_batch_engine* e, const int* tokens, const int* positions, int* next_tokens) {
    INFERNT_REQUIRE(e && tokens && positions && next_tokens, "batch_engine_step: null argument");
    if (int s = set_inputs(e, tokens, positions)) return s;
    if (int s = ensure_graph(e)) return s;
    INFERNT_CUDA_TRY(cudaGraphLaunch(e->graph, e->stream));
    INFERNT_CUDA_TRY(cudaMemcpyAsync(next_tokens, e->tokens, sizeof(int) * e->T, cudaMemcpyDeviceToHost, e->stream));
    return check_err(e);
}

int infernt_batch_engine_decode(infernt_batch_engine* e, const int* tokens, const int* positions, int steps,
                                int* tokens_out, float* ms) {
    INFERNT_REQUIRE(e && tokens && positions && steps > 0, "batch_engine_decode: bad arguments");
    for (int t = 0; t < e->T; ++t)
        INFERNT_REQUIRE((long long)positions[t] + steps <= e->cfg.max_seq_len,
                        "batch_engine_decode: sequence %d would pass max_seq_len", t);
    if (int s = set_inputs(e, tokens, positions, steps)) return s;
    if (int s = ensure_graph(e)) return s;
    int* hist = nullptr;
    if (tokens_out) {
        const size_t n = (size_t)steps * e->T;
        if (n > e->hist_cap) {
            cudaFree(e->hist);
            e->hist = nullptr;
            e->hist_cap = 0;
            INFERNT_CUDA_TRY(cudaMalloc(&e->hist, sizeof(int) * n));
            e->hist_cap = n;
        }
        hist = e->hist;
    }
    INFERNT_CUDA_TRY(cudaEventRecord(e->ev[0], e->stream));
    for (int s = 0; s < steps; ++s) {
        INFERNT_CUDA_TRY(cudaGraphLaunch(e->graph, e->stream));
        if (hist)
            INFERNT_CUDA_TRY(cudaMemcpyAsync(hist + (size_t)s * e->T, e->tokens, sizeof(int) * e->T,
                                             cudaMemcpyDeviceToDevice, e->stream));
    }
    INFERNT_CUDA_TRY(cudaEventRecord(e->ev[1], e->stream));
    if (hist)
        INFERNT_CUDA_TRY(cudaMemcpyAsync(tokens_out, hist, sizeof(int) * (size_t)steps * e->T, cudaMemcpyDeviceToHost,
                                         e->stream));
    const int s = check_err(e);
    if (ms) cudaEventElapsedTime(ms, e->ev[0], e->ev[1]);
    return s;
}

int infernt_batch_engine_logits(infernt_batch_engine* e, float* logits_host, size_t n) {
    INFERNT_REQUIRE(e && logits_host && n == (size_t)e->T * e->vl, "batch_engine_logits: need %d x %d floats",
                    e ? e->T : 0, e ? e->vl : 0);
    INFERNT_REQUIRE(e->sp_lm == 1, "batch_engine_logits: the LM head runs split; logits are partial sums");
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    INFERNT_CUDA_TRY(cudaMemcpy2D(logits_host, sizeof(float) * e->vl, e->part, sizeof(float) * e->vlp,
                                  sizeof(float) * e->vl, e->T, cudaMemcpyDeviceToHost));
    return INFERNT_OK;
}

int infernt_batch_engine_set_attention(infernt_batch_engine* e, int splits, int min_chunk, int stages) {
    INFERNT_REQUIRE(e, "batch_engine_set_attention: null engine");
    const int D = e->cfg.head_dim, nkv = e->nkv_l, G = e->nq_l / nkv;
    INFERNT_REQUIRE(splits >= 1 && splits <= 64, "batch_engine_set_attention: splits %d outside [1, 64]", splits);
    INFERNT_REQUIRE(min_chunk >= 1, "batch_engine_set_attention: min_chunk %d", min_chunk);
    INFERNT_REQUIRE(stages >= 2 && stages <= (D == 64 ? 4 : 3), "batch_engine_set_attention: %d stages at head_dim %d",
                    stages, D);
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if (splits > e->S) {
        // the partial buffer holds [T][Nkv][S][G][D + 2]
        for (auto it = e->bufs.begin(); it != e->bufs.end(); ++it)
            if (*it == e->apart) {
                e->bufs.erase(it);
                break;
            }
        cudaFree(e->apart);
        e->apart = nullptr;
        void* p = nullptr;
        if (int s = alloc(e, sizeof(float) * (size_t)e->T * nkv * splits * G * (D + 2), &p)) return s;
        e->apart = static_cast<float*>(p);
    }
    e->S = splits;
    e->min_chunk = min_chunk;
    e->stages = stages;
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;  // captured again at the next step
    }
    return INFERNT_OK;
}

int infernt_batch_engine_prefill(infernt_batch_engine* e, int seq, const int* tokens, int n_tokens, int start_pos,
                                 int chunk, int* next_token, float* logits_host, float* ms) {
    INFERNT_REQUIRE(e && tokens, "batch_engine_prefill: null argument");
    const infernt_llama_config& c = e->cfg;
    INFERNT_REQUIRE(seq >= 0 && seq < e->T, "batch_engine_prefill: sequence %d outside [0, %d)", seq, e->T);
    INFERNT_REQUIRE(n_tokens >= 1 && start_pos >= 0 && (long long)start_pos + n_tokens <= c.max_seq_len,
                    "batch_engine_prefill: %d tokens at position %d pass max_seq_len %d", n_tokens, start_pos,
                    c.max_seq_len);
    INFERNT_REQUIRE(chunk >= 0 && chunk <= 16384, "batch_engine_prefill: chunk %d outside [0, 16384]", chunk);
    for (int i = 0; i < n_tokens; ++i)
        INFERNT_REQUIRE(tokens[i] >= 0 && tokens[i] < c.vocab_size, "batch_engine_prefill: token %d at index %d",
                        tokens[i], i);
    int C = chunk > 0 ? chunk : 4096;
    if (C > n_tokens) C = n_tokens;
    const bool paged = e->page_size > 0;
    if (paged) {
        INFERNT_REQUIRE(pages_cover(e, seq, start_pos + n_tokens - 1),
                        "batch_engine_prefill: sequence %d has no page for a position in [0, %d]", seq,
                        start_pos + n_tokens - 1);
        if (int s = grow_staging(e)) return s;
        if (int s = upload_table(e)) return s;
        // earlier rows of the sequence into the staging caches
        if (int s = stage_rows(e, seq, 0, start_pos, false)) return s;
    }
    if (int s = grow_prefill(e, C)) return s;
    INFERNT_CUDA_TRY(
        cudaMemcpyAsync(e->pf_tokens, tokens, sizeof(int) * (size_t)n_tokens, cudaMemcpyHostToDevice, e->stream));
    const int tp[2] = {0, start_pos + n_tokens - 1};  // the argmax advances the position to start + n
    INFERNT_CUDA_TRY(cudaMemcpyAsync(e->pf_tok, tp, sizeof(tp), cudaMemcpyHostToDevice, e->stream));
    INFERNT_CUDA_TRY(cudaEventRecord(e->ev[0], e->stream));
    if (int s = record_prefill(e, seq, n_tokens, start_pos, C, e->stream)) return s;
    if (paged)
        if (int s = stage_rows(e, seq, start_pos, start_pos + n_tokens, true)) return s;
    INFERNT_CUDA_TRY(cudaEventRecord(e->ev[1], e->stream));
    int out[2] = {0, 0};
    INFERNT_CUDA_TRY(cudaMemcpyAsync(out, e->pf_tok, sizeof(out), cudaMemcpyDeviceToHost, e->stream));
    if (logits_host)
        INFERNT_CUDA_TRY(cudaMemcpyAsync(logits_host, e->pf_y, sizeof(float) * (size_t)e->vl, cudaMemcpyDeviceToHost,
                                         e->stream));
    const int s = check_err(e);
    if (s) return s;
    if (next_token) *next_token = out[0];
    if (ms) cudaEventElapsedTime(ms, e->ev[0], e->ev[1]);
    return INFERNT_OK;
}

int infernt_batch_engine_read_kv(infernt_batch_engine* e, int seq, int layer, int n_pos, void* k_host,
                                 void* v_host) {
    INFERNT_REQUIRE(e && k_host && v_host, "batch_engine_read_kv: null argument");
    const infernt_llama_config& c = e->cfg;
    INFERNT_REQUIRE(seq >= 0 && seq < e->T && layer >= 0 && layer < c.num_layers && n_pos >= 0 &&
                        n_pos <= c.max_seq_len,
                    "batch_engine_read_kv: sequence %d, layer %d, %d positions", seq, layer, n_pos);
    const int nkv = e->nkv_l, D = c.head_dim, S = c.max_seq_len;
    const size_t row = (size_t)n_pos * D * 2;
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if (e->page_size) {
        // page by page: rows [i P, min(n_pos, (i + 1) P)) of each KV head
        const int P = e->page_size;
        INFERNT_REQUIRE(n_pos == 0 || pages_cover(e, seq, n_pos - 1),
                        "batch_engine_read_kv: sequence %d has no page for a position below %d", seq, n_pos);
        const int* tab = e->table_host.data() + (size_t)seq * e->max_pages;
        for (int h = 0; h < nkv; ++h)
            for (int p0 = 0; p0 < n_pos; p0 += P) {
                const int rows = n_pos - p0 < P ? n_pos - p0 : P;
                const size_t src = (((size_t)tab[p0 / P] * nkv + h) * P) * D;
                const size_t dst = (size_t)h * row + (size_t)p0 * D * 2;
                INFERNT_CUDA_TRY(cudaMemcpy(static_cast<char*>(k_host) + dst, e->kc[layer] + src,
                                            (size_t)rows * D * 2, cudaMemcpyDeviceToHost));
                INFERNT_CUDA_TRY(cudaMemcpy(static_cast<char*>(v_host) + dst, e->vc[layer] + src,
                                            (size_t)rows * D * 2, cudaMemcpyDeviceToHost));
            }
        return INFERNT_OK;
    }
    for (int h = 0; h < nkv; ++h) {
        const size_t off = ((size_t)seq * nkv + h) * S * D;
        INFERNT_CUDA_TRY(cudaMemcpy(static_cast<char*>(k_host) + h * row, e->kc[layer] + off, row,
                                    cudaMemcpyDeviceToHost));
        INFERNT_CUDA_TRY(cudaMemcpy(static_cast<char*>(v_host) + h * row, e->vc[layer] + off, row,
                                    cudaMemcpyDeviceToHost));
    }
    return INFERNT_OK;
}

int infernt_batch_engine_set_sampling(infernt_batch_engine* e, float temperature, uint64_t seed) {
    INFERNT_REQUIRE(e, "batch_engine_set_sampling: null engine");
    INFERNT_REQUIRE(!(temperature < 0.0f) && temperature == temperature, "batch_engine_set_sampling: temperature %g",
                    (double)temperature);
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    e->sample_inv_t = temperature > 0.0f ? 1.0f / temperature : 0.0f;
    e->sample_seed = seed;
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;  // captured again at the next step
    }
    return INFERNT_OK;
}

int infernt_batch_engine_set_tp_exchange(infernt_batch_engine* e, int mode) {
    INFERNT_REQUIRE(e, "batch_engine_set_tp_exchange: null engine");
    INFERNT_REQUIRE(mode == INFERNT_TP_EXCHANGE_PEER || mode == INFERNT_TP_EXCHANGE_NCCL,
                    "batch_engine_set_tp_exchange: mode %d", mode);
    INFERNT_CUDA_TRY(cudaStreamSynchronize(e->stream));
    e->tp_peer = mode == INFERNT_TP_EXCHANGE_PEER;
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;  // captured again at the next step
    }
    return INFERNT_OK;
}

int infernt_batch_engine_splits(infernt_batch_engine* e, int* out) {
    INFERNT_REQUIRE(e && out, "batch_engine_splits: null argument");
    out[0] = e->sp_qkv;
    out[1] = e->sp_o;
    out[2] = e->sp_gu;
    out[3] = e->sp_down;
    out[4] = e->sp_lm;
    out[5] = e->S;
    return INFERNT_OK;
}

}  // extern "C"
