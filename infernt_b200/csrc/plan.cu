// plan.cu — the decode step over caller-owned weights and KV cache.
//
// Two executions of the same step (architectures/llama/llama_layer.cpp:5-73,
// llama_model.cpp:45-65, src/engine.cpp:53-76):
//
// * persistent (default when the shapes allow it): one cooperative launch
//   of the persistent decode kernel (decode_kernel.cu) runs every layer and
//   the LM head, and a chain of steps, with the weight stream never stopping
//   at phase boundaries;
// * kernel sequence: 5 kernels per layer + 1 for the head, chained with
//   programmatic dependent launch and replayed as a CUDA graph:
//     qkv     RMSNorm(attn_norm) + [Wq;Wk;Wv] x      (layer 0: embedding row of the token)
//     attn    RoPE + KV append + split-KV GQA attention
//     o       hidden += Wo attn_out
//     gateup  RMSNorm(ffn_norm) + SiLU(Wg x) * (Wu x)
//     down    hidden += Wd act
//     head    RMSNorm(final_norm) + logits = Wlm x + argmax
//
// The residual stream is updated in place, so the reference's 23 hidden-
// state copies per token (llama_model.cpp:48, :55) disappear.  Token,
// position and step live in a small device state block: attention reads the
// position from it and the head writes the next token and position into it,
// so a chain of steps needs no host round trip.
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "decode_kernel.cuh"
#include "gemv.cuh"
#include "internal.h"

namespace infernt {

// (cos, sin) RoPE factors for every position and pair, with the same device
// functions the attention would otherwise evaluate per step.
__global__ void rope_table_kernel(float2* tab, int max_seq, int D, float theta) {
    const int half = D / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)max_seq * half;
         i += (long long)gridDim.x * blockDim.x)
        tab[i] = rope_factors((int)(i % half), D, (int)(i / half), theta);
}

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
    float2* rope = nullptr;  // (cos, sin) table [max_seq][D/2]
    int* state = nullptr;  // {token, position, step, last token}
    unsigned* err = nullptr;  // 64 bytes after state
    int* host_rb = nullptr;   // pinned host copy of state .. err (one readback per step)
    float* attn_part = nullptr;
    unsigned* attn_counter = nullptr;
    LmWs* lm_ws = nullptr;
    int mode = INFERNT_MODE_PERSISTENT;
    // kernel-sequence path
    cudaStream_t cap_stream = nullptr;
    struct Entry {
        int mode;
        const float* input;
        float* logits;
        int* hist;
        cudaGraphExec_t exec;
    };
    std::vector<Entry> graphs;
    // persistent path
    void* mega_mem = nullptr;
    MegaParams mega;
    int mega_ctas = 0;
    unsigned tag_base = 0;   // phase instances run so far (tags of tagged activations)
    void* ll_mem = nullptr;  // tagged activation buffers of the persistent kernel
    // tensor parallelism (tp_size 1: none).  cfg holds this rank's shapes:
    // its heads, its gate/up rows padded to a multiple of 512 (down's K), its
    // vocabulary rows
    int tp_rank = 0, tp_size = 1;
    int vocab_global = 0;  // embedding rows (token ids)
    int iloc = 0;          // gate/up rows of this rank (<= cfg.intermediate_size)
    int v0 = 0;            // first vocabulary row of this rank
    float* hmid = nullptr;  // residual stream after the O all-reduce
    void* xch_mem = nullptr;  // this rank's exchange region
    size_t xch_bytes = 0;
    std::vector<void*> opened;  // peers' regions mapped into this process
    unsigned char** peer_tab = nullptr;  // device copy of the region pointers
    bool peers_set = false;
};

namespace {

// SM clock cycles of `us` microseconds at the device's maximum SM clock.
long long wait_cycles_for(long long us) {
    int dev = 0, khz = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev) != cudaSuccess ||
        khz <= 0) {
        cudaGetLastError();
        khz = 2000000;
    }
    return us * (long long)khz / 1000;
}

const int kInputVector = 0;  // layer 0 reads an input embedding vector
const int kInputToken = 1;   // layer 0 reads the embedding row of state[0]

int record_step(infernt_plan* p, cudaStream_t st, int mode, const float* input, float* logits, int* hist) {
    const infernt_llama_config& c = p->cfg;
    const int H = c.hidden_size, I = c.intermediate_size, L = c.num_layers;
    const int dt = c.weight_dtype;
    for (int l = 0; l < L; ++l) {
        const void* const* lw = p->w.data() + 3 + 9 * l;
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
            a.x = mode == kInputVector ? input : nullptr;
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
        at.rope = p->rope;
        INFERNT_CUDA_TRY(launch_attention_decode(at, st, true));

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

int run_graph_step(infernt_plan* p, cudaStream_t st, int mode, const float* input, float* logits, int* hist) {
    if (p->mode == INFERNT_MODE_EAGER) return record_step(p, st, mode, input, logits, hist);
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

// `steps` decode steps from the current device state.
// Steps of the plan from the device state; (token, position) with
// position >= 0 set the first step's instead (the persistent kernel takes
// them as launch parameters, the kernel sequences from set_state_kernel).
int run_steps(infernt_plan* p, cudaStream_t st, int mode, const float* input, float* logits, int* hist, int steps,
              int token = 0, int position = -1) {
    if (!logits) logits = p->logits;
    if (p->mode != INFERNT_MODE_PERSISTENT && position >= 0) {
        set_state_kernel<<<1, 1, 0, st>>>(p->state, token, position);
        INFERNT_CUDA_TRY(cudaGetLastError());
    }
    if (p->mode == INFERNT_MODE_PERSISTENT) {
        INFERNT_REQUIRE(p->tp_size == 1 || p->peers_set,
                        "tensor-parallel plan: infernt_plan_set_peers has not been called");
        MegaParams m = p->mega;
        m.input = mode == kInputVector ? input : nullptr;
        m.logits = logits;
        m.hist = hist;
        m.steps = steps;
        m.init_token = token;
        m.init_pos = position;
        // every phase instance has its own tag (the same sequence on every
        // rank); 32-bit tags bound a plan's lifetime
        const unsigned long long used = (unsigned long long)steps * (unsigned long long)m.nphases;
        INFERNT_REQUIRE((unsigned long long)p->tag_base + used < 0xffffffffull,
                        "persistent plan: %u phase instances run, the tag space is spent; recreate the plan",
                        p->tag_base);
        m.tag_base = p->tag_base;
        p->tag_base += (unsigned)used;
        if (p->tp_size > 1) m.peers = p->peer_tab;
        INFERNT_CUDA_TRY(launch_mega(m, p->cfg.weight_dtype, p->mega_ctas, st));
        return INFERNT_OK;
    }
    for (int s = 0; s < steps; ++s)
        if (int r = run_graph_step(p, st, mode, input, logits, hist)) return r;
    return INFERNT_OK;
}

int validate_config(const infernt_llama_config* c) {
    INFERNT_REQUIRE(c, "plan: null config");
    INFERNT_REQUIRE(c->vocab_size > 0 && c->hidden_size > 0 && c->num_layers > 0 && c->num_attention_heads > 0 &&
                        c->num_key_value_heads > 0 && c->intermediate_size > 0 && c->max_seq_len > 0 &&
                        c->head_dim > 0,
                    "plan: every dimension must be positive");
    INFERNT_REQUIRE(c->hidden_size % 4 == 0 && c->intermediate_size % 4 == 0,
                    "plan: hidden %d and intermediate %d must be multiples of 4", c->hidden_size, c->intermediate_size);
    INFERNT_REQUIRE(c->weight_dtype == INFERNT_DTYPE_F32 || c->weight_dtype == INFERNT_DTYPE_BF16,
                    "plan: weight_dtype %d", c->weight_dtype);
    INFERNT_REQUIRE(c->vocab_size <= 1 << 30 && (long long)c->max_seq_len * c->head_dim < (1ll << 31),
                    "plan: shape too large");
    return attention_shape_check(c->num_attention_heads, c->num_key_value_heads, c->head_dim, 1);
}

// Whether the persistent kernel applies: projection inputs in 512-column
// blocks, 16-byte aligned weights, and the shared memory budget.
bool mega_eligible(const infernt_plan* p) {
    const infernt_llama_config& c = p->cfg;
    if (c.hidden_size % kPiece || p->qs % kPiece || c.intermediate_size % kPiece) return false;
    for (const void* w : p->w)
        if (!aligned16(w)) return false;
    // attention inputs arrive by bulk copies: whole rows of 16-byte multiples
    if (c.head_dim % 4) return false;
    for (int l = 0; l < c.num_layers; ++l)
        if (!aligned16(p->kc[l]) || !aligned16(p->vc[l])) return false;
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, current_device());
    return coop != 0;
}

int build_mega(infernt_plan* p) {
    const infernt_llama_config& c = p->cfg;
    const int H = c.hidden_size, I = c.intermediate_size, L = c.num_layers, V = c.vocab_size;
    const int dt = c.weight_dtype;
    const int G = c.num_attention_heads / c.num_key_value_heads;
    const bool tp = p->tp_size > 1;
    const int T = p->tp_size;
    // exchange buffers of the O and down partials, tagged words [T][H]
    const int off_o = kXchData, off_d = kXchData + T * H * 8;

    // tagged activations: Q|K|V rows, split partials, attention output, the
    // residual stream (hA: layer input / after down, hB: after O), act
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t w8 = sizeof(unsigned long long);
    const size_t n_qkv = (size_t)p->qs + 2 * p->kvs;
    const size_t n_part = (size_t)c.num_key_value_heads * p->splits * G * (c.head_dim + 2);
    const size_t b_qkv = al(w8 * n_qkv), b_part = al(w8 * n_part), b_attn = al(w8 * p->qs), b_h = al(w8 * H),
                 b_act = al(w8 * I);
    const size_t ll_total = b_qkv + b_part + b_attn + 2 * b_h + b_act;
    INFERNT_CUDA_TRY(cudaMalloc(&p->ll_mem, ll_total));
    INFERNT_CUDA_TRY(cudaMemset(p->ll_mem, 0, ll_total));
    char* lb = static_cast<char*>(p->ll_mem);
    auto take = [&](size_t bytes) {
        unsigned long long* r = reinterpret_cast<unsigned long long*>(lb);
        lb += bytes;
        return r;
    };
    unsigned long long* ll_qkv = take(b_qkv);
    unsigned long long* ll_part = take(b_part);
    unsigned long long* ll_attn = take(b_attn);
    unsigned long long* hA = take(b_h);
    unsigned long long* hB = take(b_h);
    unsigned long long* ll_act = take(b_act);

    std::vector<MegaPhase> ph;

    // a GEMV phase over the matrices `mats` stacked in the row space (ns ==
    // 2: gate, up), input x written by phase x_ph of the step
    auto gemv = [&](int epi, int ns, std::initializer_list<const void*> mats, std::initializer_list<int> rows,
                    int units, int K, const unsigned long long* x, int x_ph, const float* norm,
                    unsigned long long* out) -> MegaPhase& {
        MegaPhase P;
        memset(&P, 0, sizeof(P));
        P.kind = kPhGemv;
        P.epi = epi;
        P.ns = ns;
        P.nseg = (int)mats.size();
        int i = 0;
        for (const void* m : mats) P.w[i++] = m;
        i = 0;
        for (int r : rows) P.seg_rows[i++] = r;
        P.units = units;
        P.K = K;
        P.kx = K;
        P.cb = K / kPiece;
        P.x = x;
        P.x_ph = x_ph;
        P.norm_w = norm;
        P.eps = c.rms_norm_eps;
        P.out = out;
        P.xch_off = -1;
        ph.push_back(P);
        return ph.back();
    };
    // with tensor parallelism the input after an all-reduce is the sum of
    // this CTA's share of the residual stream and every rank's partial
    // (published at xout), then the whole of xout
    auto summed = [&](MegaPhase& P, const unsigned long long* base, int base_ph, int off, int sum_ph,
                      unsigned long long* xout) {
        P.nsum = T;
        P.xbase = base;
        P.xbase_ph = base_ph;
        P.sum_off = off;
        P.sum_ph = sum_ph;
        P.xout = xout;
    };
    const int Iu = p->iloc;  // gate/up rows (down's K may be padded past them)
    for (int l = 0; l < L; ++l) {
        const void* const* lw = p->w.data() + 3 + 9 * l;
        const int q = 5 * l;       // this layer's phases: q, q+1 (attention), q+2 (O), q+3 (gate/up), q+4 (down)
        const int dprev = q - 1;   // the previous layer's down phase
        const float* attn_norm = static_cast<const float*>(lw[0]);
        MegaPhase& Q = gemv(kEpiStore, 1, {lw[1], lw[2], lw[3]}, {p->qs, p->kvs, p->kvs}, p->qs + 2 * p->kvs, H,
                            (l == 0 || tp) ? nullptr : hA, dprev, attn_norm, ll_qkv);
        if (l == 0)
            Q.xout = hA;  // the embedding row starts the residual stream
        else if (tp)
            summed(Q, hB, dprev - 1, off_d, dprev, hA);
        // the attention phase's caches: prefetched into L2 while Q|K|V runs
        Q.kc = p->kc[l];
        Q.vc = p->vc[l];
        MegaPhase A;
        memset(&A, 0, sizeof(A));
        A.kind = kPhAttn;
        A.layer = l;
        A.kc = p->kc[l];
        A.vc = p->vc[l];
        A.x_ph = q;
        A.xch_off = -1;
        ph.push_back(A);
        if (tp) {
            gemv(kEpiExchange, 1, {lw[4]}, {H}, H, p->qs, ll_attn, q + 1, nullptr, nullptr).xch_off = off_o;
            MegaPhase& U = gemv(kEpiSwiGLU, 2, {lw[6], lw[7]}, {Iu, Iu}, Iu, H, nullptr, 0,
                                static_cast<const float*>(lw[5]), ll_act);
            summed(U, hA, q, off_o, q + 2, hB);
            MegaPhase& Dn = gemv(kEpiExchange, 1, {lw[8]}, {H}, H, I, ll_act, q + 3, nullptr, nullptr);
            Dn.xch_off = off_d;
            Dn.kx = Iu;  // the padding columns past this rank's gate/up rows
        } else {
            MegaPhase& O = gemv(kEpiResidual, 1, {lw[4]}, {H}, H, p->qs, ll_attn, q + 1, nullptr, hB);
            O.res = hA;
            O.res_ph = l == 0 ? 0 : dprev;
            gemv(kEpiSwiGLU, 2, {lw[6], lw[7]}, {Iu, Iu}, Iu, H, hB, q + 2, static_cast<const float*>(lw[5]),
                 ll_act);
            MegaPhase& Dn = gemv(kEpiResidual, 1, {lw[8]}, {H}, H, I, ll_act, q + 3, nullptr, hA);
            Dn.res = hB;
            Dn.res_ph = q + 2;
        }
    }
    const int dlast = 5 * L - 1;
    MegaPhase& LM = gemv(kEpiArgmax, 1, {p->w[2]}, {V}, V, H, tp ? nullptr : hA, dlast,
                         static_cast<const float*>(p->w[1]), nullptr);
    LM.row_base = p->v0;
    if (tp) summed(LM, hB, dlast - 1, off_d, dlast, hA);

    // input vector + the norm weights behind it (RMSNorm phases), or the
    // attention scratch, whichever is larger
    int x_floats = 2 * H;
    if (p->qs > x_floats) x_floats = p->qs;
    if (I > x_floats) x_floats = I;
    // attention scratch, then the merge's split weights [G][splits] and [G]
    const int af = attn_bulk_smem_floats(G, c.head_dim) + G * (p->splits + 1);
    if (af > x_floats) x_floats = af;
    x_floats = (x_floats + 3) / 4 * 4;

    INFERNT_CUDA_TRY(mega_prepare());
    int optin = 0;
    INFERNT_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, current_device()));
    int slots = mega_max_ring_slots();
    const int budget = optin - mega_static_smem(dt) - 256;
    while (slots >= 4 && mega_smem_bytes(slots, x_floats) > budget) --slots;
    slots &= ~1;  // the two consumer teams own alternate slots: an even ring keeps each slot with one team
    INFERNT_REQUIRE(slots >= 4, "persistent decode: shared memory budget too small");
    const int smem = mega_smem_bytes(slots, x_floats);
    const int per_sm = mega_occupancy(dt, smem);
    INFERNT_REQUIRE(per_sm >= 1, "persistent decode: kernel does not fit on an SM");
    const int ctas = sm_count();

    // device memory: phases | argmax partials | argmax ticket
    const size_t b_ph = al(sizeof(MegaPhase) * ph.size());
    const size_t b_am = al(sizeof(float) * ctas) + al(sizeof(int) * ctas) + 256;
    const size_t total = b_ph + b_am;
    INFERNT_CUDA_TRY(cudaMalloc(&p->mega_mem, total));
    INFERNT_CUDA_TRY(cudaMemset(p->mega_mem, 0, total));
    char* b = static_cast<char*>(p->mega_mem);
    MegaPhase* d_ph = reinterpret_cast<MegaPhase*>(b);
    INFERNT_CUDA_TRY(cudaMemcpy(d_ph, ph.data(), sizeof(MegaPhase) * ph.size(), cudaMemcpyHostToDevice));
    b += b_ph;
    float* d_amv = reinterpret_cast<float*>(b);
    b += al(sizeof(float) * ctas);
    int* d_ami = reinterpret_cast<int*>(b);
    b += al(sizeof(int) * ctas);
    unsigned* d_amc = reinterpret_cast<unsigned*>(b);

    MegaParams& m = p->mega;
    memset(&m, 0, sizeof(m));
    m.phases = d_ph;
    m.nphases = (int)ph.size();
    m.emb = static_cast<const float*>(p->w[0]);
    m.vocab = p->vocab_global;  // embedding rows (V is this rank's LM-head rows)
    m.ll_qkv = ll_qkv;
    m.ll_part = ll_part;
    m.ll_attn = ll_attn;
    m.attn.nq = c.num_attention_heads;
    m.attn.nkv = c.num_key_value_heads;
    m.attn.D = c.head_dim;
    m.attn.max_seq = c.max_seq_len;
    m.attn.splits = p->splits;
    m.attn.theta = c.rope_theta;
    m.attn.scale = 1.0f / sqrtf((float)c.head_dim);
    m.attn.err = p->err;
    m.attn.rope = p->rope;
    m.state = p->state;
    m.err = p->err;
    m.am_val = d_amv;
    m.am_idx = d_ami;
    m.am_cnt = d_amc;
    m.ring_slots = slots;
    m.x_floats = x_floats;
    m.tp_rank = p->tp_rank;
    m.tp_size = p->tp_size;
    m.peers = p->peer_tab;  // set by infernt_plan_set_peers (tensor parallelism)
    m.wait_cycles = wait_cycles_for(2000000);
    m.inv_temp = 0.0f;  // greedy until infernt_plan_set_sampling
    m.sample_seed = 0;
    // 8 slots in flight (128 KB per SM) keep HBM saturated; a deeper queue
    // only lengthens the phase boundaries' reads (TinyLlama FP32 1.009 ->
    // 0.993 ms per step, 8B bf16 3.227 -> 3.187; 6 to 10 slots all equal)
    m.stream_depth = slots < 8 ? slots : 8;
    // rows narrower than a slot other than 2048 / 4096 columns: the kernel
    // instantiation with the narrow-row paths
    const int pt = dt == INFERNT_DTYPE_BF16 ? 16 : 8;
    m.narrow = 0;
    for (const MegaPhase& P : ph)
        if (P.kind == kPhGemv && P.cb < pt && P.cb != 4 && P.cb != 8) m.narrow = 1;
    p->mega_ctas = ctas;
    return INFERNT_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Tensor-parallel rank description for plan_create_impl (rank 0 of 1: none).
struct TpShard {
    int rank = 0, size = 1;
    int vocab_global = 0, iloc = 0, v0 = 0;
};

int plan_create_impl(const infernt_llama_config* cfg, const void* const* weights, float* const* k_cache,
                     float* const* v_cache, int mode, const TpShard& tp, infernt_plan** out) {
    const int L = cfg->num_layers;
    for (int i = 0; i < 3 + 9 * L; ++i) INFERNT_REQUIRE(weights[i], "plan_create: weight pointer %d is null", i);
    for (int l = 0; l < L; ++l) INFERNT_REQUIRE(k_cache[l] && v_cache[l], "plan_create: cache layer %d null", l);
    INFERNT_CUDA_TRY(gemv_prepare());

    infernt_plan* p = new (std::nothrow) infernt_plan();
    INFERNT_REQUIRE(p, "plan_create: host allocation failed");
    p->cfg = *cfg;
    p->tp_rank = tp.rank;
    p->tp_size = tp.size;
    p->vocab_global = tp.vocab_global;
    p->iloc = tp.iloc;
    p->v0 = tp.v0;
    p->w.assign(weights, weights + 3 + 9 * L);
    p->kc.assign(k_cache, k_cache + L);
    p->vc.assign(v_cache, v_cache + L);
    p->qs = cfg->num_attention_heads * cfg->head_dim;
    p->kvs = cfg->num_key_value_heads * cfg->head_dim;
    p->mode = mode;
    const int splits = sm_count() / cfg->num_key_value_heads;
    // at most 64 splits per KV head (the persistent kernel's merge bound)
    p->splits = splits < 1 ? 1 : (splits > 64 ? 64 : splits);

    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t b_qkv = al(sizeof(float) * (p->qs + 2 * p->kvs));
    const size_t b_attn = al(sizeof(float) * p->qs);
    const size_t b_act = al(sizeof(float) * cfg->intermediate_size);
    const size_t b_hid = al(sizeof(float) * cfg->hidden_size);
    const size_t b_log = al(sizeof(float) * cfg->vocab_size);
    const size_t b_state = 256;
    const size_t b_aws =
        attention_workspace_bytes(cfg->num_attention_heads, cfg->num_key_value_heads, cfg->head_dim, p->splits);
    const size_t b_lm = al(sizeof(LmWs));
    const size_t b_rope = al(sizeof(float2) * (size_t)cfg->max_seq_len * (cfg->head_dim / 2));
    const size_t total = b_qkv + b_attn + b_act + 2 * b_hid + b_log + b_state + b_aws + b_lm + b_rope;
    cudaError_t e = cudaMalloc(&p->scratch, total);
    if (e == cudaSuccess) e = cudaMemset(p->scratch, 0, total);
    if (e != cudaSuccess) {
        cudaFree(p->scratch);
        delete p;
        return cuda_fail(e, "plan scratch allocation");
    }
    char* b = static_cast<char*>(p->scratch);
    p->qkv = reinterpret_cast<float*>(b);
    b += b_qkv;
    p->attn = reinterpret_cast<float*>(b);
    b += b_attn;
    p->act = reinterpret_cast<float*>(b);
    b += b_act;
    p->hidden = reinterpret_cast<float*>(b);
    b += b_hid;
    p->hmid = reinterpret_cast<float*>(b);
    b += b_hid;
    p->logits = reinterpret_cast<float*>(b);
    b += b_log;
    p->state = reinterpret_cast<int*>(b);
    p->err = reinterpret_cast<unsigned*>(b + 64);
    b += b_state;
    if (cudaHostAlloc(reinterpret_cast<void**>(&p->host_rb), 128, cudaHostAllocDefault) != cudaSuccess) {
        cudaGetLastError();
        p->host_rb = nullptr;  // read_token falls back to pageable copies
    }
    const size_t part = (size_t)cfg->num_key_value_heads * p->splits *
                        (cfg->num_attention_heads / cfg->num_key_value_heads) * (cfg->head_dim + 2) * 4;
    p->attn_part = reinterpret_cast<float*>(b);
    p->attn_counter = reinterpret_cast<unsigned*>(b + al(part));
    b += b_aws;
    p->lm_ws = reinterpret_cast<LmWs*>(b);
    b += b_lm;
    p->rope = reinterpret_cast<float2*>(b);
    rope_table_kernel<<<sm_count() * 4, 256>>>(p->rope, cfg->max_seq_len, cfg->head_dim, cfg->rope_theta);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        infernt_plan_destroy(p);
        return cuda_fail(e, "RoPE table");
    }

    if (p->tp_size > 1) {
        // the all-reduces run inside the persistent kernel only
        if (p->mode != INFERNT_MODE_PERSISTENT || !mega_eligible(p)) {
            infernt_plan_destroy(p);
            return fail(INFERNT_ERR_UNSUPPORTED, "tensor-parallel plan: shapes not eligible for the persistent "
                                                 "kernel (K multiples of 512, 16-byte aligned, head_dim %% 4)");
        }
        p->xch_bytes = kXchData + 2 * (size_t)p->tp_size * cfg->hidden_size * sizeof(unsigned long long);
        e = cudaMalloc(&p->xch_mem, p->xch_bytes);
        if (e == cudaSuccess) e = cudaMemset(p->xch_mem, 0, p->xch_bytes);
        if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&p->peer_tab), sizeof(void*) * kMaxTp);
        if (e != cudaSuccess) {
            infernt_plan_destroy(p);
            return cuda_fail(e, "tensor-parallel exchange region");
        }
    }
    if (p->mode == INFERNT_MODE_PERSISTENT) {
        if (mega_eligible(p)) {
            if (int s = build_mega(p)) {
                infernt_plan_destroy(p);
                return s;
            }
        } else {
            p->mode = INFERNT_MODE_GRAPH;
        }
    }
    *out = p;
    return INFERNT_OK;
}

}  // namespace

extern "C" {

int infernt_plan_create(const infernt_llama_config* cfg, const void* const* weights, float* const* k_cache,
                        float* const* v_cache, int mode, infernt_plan** out) {
    INFERNT_REQUIRE(out, "plan_create: null output");
    *out = nullptr;
    if (int s = validate_config(cfg)) return s;
    INFERNT_REQUIRE(weights && k_cache && v_cache, "plan_create: null weights or cache");
    INFERNT_REQUIRE(mode >= INFERNT_MODE_EAGER && mode <= INFERNT_MODE_PERSISTENT, "plan_create: mode %d", mode);
    TpShard tp;
    tp.vocab_global = cfg->vocab_size;
    tp.iloc = cfg->intermediate_size;
    return plan_create_impl(cfg, weights, k_cache, v_cache, mode, tp, out);
}

int infernt_tp_shard_dims(const infernt_llama_config* cfg, int tp_rank, int tp_size, int* dims) {
    INFERNT_REQUIRE(cfg && dims, "tp_shard_dims: null argument");
    if (int s = validate_config(cfg)) return s;
    INFERNT_REQUIRE(tp_size >= 1 && tp_size <= kMaxTp && tp_rank >= 0 && tp_rank < tp_size,
                    "tp_shard_dims: rank %d of %d (at most %d ranks)", tp_rank, tp_size, kMaxTp);
    INFERNT_REQUIRE(cfg->num_key_value_heads % tp_size == 0 && cfg->intermediate_size % tp_size == 0,
                    "tp_shard_dims: %d KV heads and intermediate %d must divide among %d ranks",
                    cfg->num_key_value_heads, cfg->intermediate_size, tp_size);
    const int il = cfg->intermediate_size / tp_size;
    dims[0] = cfg->num_attention_heads / tp_size;
    dims[1] = cfg->num_key_value_heads / tp_size;
    dims[2] = il;
    dims[3] = (il + kPiece - 1) / kPiece * kPiece;
    dims[4] = (int)((long long)cfg->vocab_size * tp_rank / tp_size);
    dims[5] = (int)((long long)cfg->vocab_size * (tp_rank + 1) / tp_size) - dims[4];
    return INFERNT_OK;
}

int infernt_plan_create_tp(const infernt_llama_config* cfg, const void* const* weights, float* const* k_cache,
                           float* const* v_cache, int tp_rank, int tp_size, infernt_plan** out) {
    INFERNT_REQUIRE(out, "plan_create_tp: null output");
    *out = nullptr;
    int d[6];
    if (int s = infernt_tp_shard_dims(cfg, tp_rank, tp_size, d)) return s;
    INFERNT_REQUIRE(weights && k_cache && v_cache, "plan_create_tp: null weights or cache");
    infernt_llama_config local = *cfg;
    local.num_attention_heads = d[0];
    local.num_key_value_heads = d[1];
    local.intermediate_size = d[3];
    local.vocab_size = d[5];
    if (int s = validate_config(&local)) return s;
    INFERNT_REQUIRE(cfg->vocab_size <= (1 << 24), "plan_create_tp: vocabulary of %d above 2^24 ids",
                    cfg->vocab_size);
    TpShard tp;
    tp.rank = tp_rank;
    tp.size = tp_size;
    tp.vocab_global = cfg->vocab_size;
    tp.iloc = d[2];
    tp.v0 = d[4];
    return plan_create_impl(&local, weights, k_cache, v_cache, INFERNT_MODE_PERSISTENT, tp, out);
}

int infernt_plan_xchg_handle(infernt_plan* p, void* handle_out) {
    INFERNT_REQUIRE(p && handle_out, "plan_xchg_handle: null argument");
    INFERNT_REQUIRE(p->tp_size > 1 && p->xch_mem, "plan_xchg_handle: not a tensor-parallel plan");
    cudaIpcMemHandle_t h;
    INFERNT_CUDA_TRY(cudaIpcGetMemHandle(&h, p->xch_mem));
    static_assert(sizeof(h) == INFERNT_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return INFERNT_OK;
}

int infernt_plan_set_peers(infernt_plan* p, const void* handles) {
    INFERNT_REQUIRE(p && handles, "plan_set_peers: null argument");
    INFERNT_REQUIRE(p->tp_size > 1 && p->xch_mem, "plan_set_peers: not a tensor-parallel plan");
    INFERNT_REQUIRE(!p->peers_set, "plan_set_peers: peers are already set");
    std::vector<unsigned char*> tab(kMaxTp, nullptr);
    for (int r = 0; r < p->tp_size; ++r) {
        if (r == p->tp_rank) {
            tab[r] = static_cast<unsigned char*>(p->xch_mem);
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + (size_t)r * INFERNT_IPC_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        INFERNT_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        p->opened.push_back(ptr);
        tab[r] = static_cast<unsigned char*>(ptr);
    }
    INFERNT_CUDA_TRY(cudaMemcpy(p->peer_tab, tab.data(), sizeof(void*) * kMaxTp, cudaMemcpyHostToDevice));
    p->peers_set = true;
    return INFERNT_OK;
}

int infernt_plan_xchg_bytes(const infernt_plan* p, size_t* bytes) {
    INFERNT_REQUIRE(p && bytes, "plan_xchg_bytes: null argument");
    INFERNT_REQUIRE(p->tp_size > 1 && p->xch_mem, "plan_xchg_bytes: not a tensor-parallel plan");
    *bytes = p->xch_bytes;
    return INFERNT_OK;
}

void* infernt_plan_xchg_region(infernt_plan* p) { return p ? p->xch_mem : nullptr; }

int infernt_plan_set_peer_regions(infernt_plan* p, void* const* regions) {
    INFERNT_REQUIRE(p && regions, "plan_set_peer_regions: null argument");
    INFERNT_REQUIRE(p->tp_size > 1 && p->xch_mem, "plan_set_peer_regions: not a tensor-parallel plan");
    INFERNT_REQUIRE(!p->peers_set, "plan_set_peer_regions: peers are already set");
    INFERNT_REQUIRE(regions[p->tp_rank] == p->xch_mem, "plan_set_peer_regions: regions[%d] is not this plan's own",
                    p->tp_rank);
    std::vector<unsigned char*> tab(kMaxTp, nullptr);
    for (int r = 0; r < p->tp_size; ++r) {
        INFERNT_REQUIRE(regions[r] && aligned16(regions[r]), "plan_set_peer_regions: region %d null or unaligned", r);
        tab[r] = static_cast<unsigned char*>(regions[r]);
    }
    INFERNT_CUDA_TRY(cudaMemcpy(p->peer_tab, tab.data(), sizeof(void*) * kMaxTp, cudaMemcpyHostToDevice));
    p->peers_set = true;
    return INFERNT_OK;
}

int infernt_plan_set_wait_budget(infernt_plan* p, long long microseconds) {
    INFERNT_REQUIRE(p, "plan_set_wait_budget: null plan");
    INFERNT_REQUIRE(microseconds > 0 && microseconds <= 600000000ll,
                    "plan_set_wait_budget: %lld us outside (0, 600 s]", microseconds);
    p->mega.wait_cycles = wait_cycles_for(microseconds);
    return INFERNT_OK;
}

int infernt_plan_set_stream_depth(infernt_plan* p, int slots) {
    INFERNT_REQUIRE(p, "plan_set_stream_depth: null plan");
    INFERNT_REQUIRE(slots >= 0, "plan_set_stream_depth: %d slots", slots);
    if (p->mode != INFERNT_MODE_PERSISTENT) return INFERNT_OK;  // only the persistent kernel streams
    p->mega.stream_depth = slots == 0 || slots > p->mega.ring_slots ? p->mega.ring_slots : slots;
    return INFERNT_OK;
}

int infernt_plan_stream_depth(const infernt_plan* p, int* slots, int* ring_slots) {
    INFERNT_REQUIRE(p && slots && ring_slots, "plan_stream_depth: null argument");
    *slots = p->mega.stream_depth;
    *ring_slots = p->mega.ring_slots;
    return INFERNT_OK;
}

int infernt_plan_set_sampling(infernt_plan* p, float temperature, uint64_t seed) {
    INFERNT_REQUIRE(p, "plan_set_sampling: null plan");
    INFERNT_REQUIRE(temperature == temperature, "plan_set_sampling: temperature is NaN");
    if (temperature <= 0.0f) {
        p->mega.inv_temp = 0.0f;
        return INFERNT_OK;
    }
    if (p->mode != INFERNT_MODE_PERSISTENT)
        return fail(INFERNT_ERR_UNSUPPORTED, "plan_set_sampling: temperature sampling inside the step needs the "
                                             "persistent decode kernel (this plan runs mode %d)", p->mode);
    p->mega.inv_temp = 1.0f / temperature;
    p->mega.sample_seed = seed;
    return INFERNT_OK;
}

int infernt_plan_destroy(infernt_plan* p) {
    if (!p) return INFERNT_OK;
    for (auto& e : p->graphs) cudaGraphExecDestroy(e.exec);
    if (p->cap_stream) cudaStreamDestroy(p->cap_stream);
    for (void* ptr : p->opened) cudaIpcCloseMemHandle(ptr);
    cudaFree(p->peer_tab);
    cudaFree(p->xch_mem);
    cudaFree(p->mega_mem);
    cudaFree(p->ll_mem);
    cudaFree(p->scratch);
    if (p->host_rb) cudaFreeHost(p->host_rb);
    delete p;
    return INFERNT_OK;
}

int infernt_plan_mode(const infernt_plan* p) { return p ? p->mode : -1; }

int infernt_plan_forward(infernt_plan* p, const float* input_embedding, int position, float* logits, void* stream) {
    INFERNT_REQUIRE(p && input_embedding, "plan_forward: null argument");
    INFERNT_REQUIRE(position >= 0 && position < p->cfg.max_seq_len, "plan_forward: position %d outside [0, %d)",
                    position, p->cfg.max_seq_len);
    INFERNT_REQUIRE(aligned16(input_embedding), "plan_forward: input must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    return run_steps(p, st, kInputVector, input_embedding, logits, nullptr, 1, 0, position);
}

int infernt_plan_decode(infernt_plan* p, int token, int position, float* logits, void* stream) {
    INFERNT_REQUIRE(p, "plan_decode: null plan");
    INFERNT_REQUIRE(token >= 0 && token < p->vocab_global, "plan_decode: token %d outside [0, %d)", token,
                    p->vocab_global);
    INFERNT_REQUIRE(position >= 0 && position < p->cfg.max_seq_len, "plan_decode: position %d outside [0, %d)",
                    position, p->cfg.max_seq_len);
    cudaStream_t st = (cudaStream_t)stream;
    return run_steps(p, st, kInputToken, nullptr, logits, nullptr, 1, token, position);
}

int infernt_plan_decode_chain(infernt_plan* p, int token, int position, int steps, int* tokens_dev, void* stream) {
    INFERNT_REQUIRE(p, "plan_decode_chain: null plan");
    INFERNT_REQUIRE(token >= 0 && token < p->vocab_global, "plan_decode_chain: token %d", token);
    INFERNT_REQUIRE(steps >= 0 && position >= 0 && (long long)position + steps <= p->cfg.max_seq_len,
                    "plan_decode_chain: positions [%d, %d) exceed max_seq_len %d", position, position + steps,
                    p->cfg.max_seq_len);
    if (steps == 0) return INFERNT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    return run_steps(p, st, kInputToken, nullptr, nullptr, tokens_dev, steps, token, position);
}

int infernt_plan_read_token(infernt_plan* p, int* token_host, void* stream) {
    INFERNT_REQUIRE(p && token_host, "plan_read_token: null argument");
    cudaStream_t st = (cudaStream_t)stream;
    int buf[4];
    unsigned err = 0;
    if (p->host_rb) {
        // state and error word in one copy into pinned memory (the error
        // word sits 64 bytes after the state)
        INFERNT_CUDA_TRY(cudaMemcpyAsync(p->host_rb, p->state, 68, cudaMemcpyDeviceToHost, st));
        INFERNT_CUDA_TRY(cudaStreamSynchronize(st));
        memcpy(buf, p->host_rb, sizeof(buf));
        memcpy(&err, reinterpret_cast<const char*>(p->host_rb) + 64, sizeof(err));
    } else {
        INFERNT_CUDA_TRY(cudaMemcpyAsync(buf, p->state, sizeof(buf), cudaMemcpyDeviceToHost, st));
        INFERNT_CUDA_TRY(cudaMemcpyAsync(&err, p->err, sizeof(err), cudaMemcpyDeviceToHost, st));
        INFERNT_CUDA_TRY(cudaStreamSynchronize(st));
    }
    if (err) {
        cudaMemsetAsync(p->err, 0, sizeof(unsigned), st);
        cudaStreamSynchronize(st);
        return fail(INFERNT_ERR_DEVICE,
                    "decode kernels reported error word 0x%x (1: wait timeout, 2: position, 4: token id)", err);
    }
    *token_host = buf[3];
    return INFERNT_OK;
}

float* infernt_plan_logits(infernt_plan* p) { return p ? p->logits : nullptr; }

size_t infernt_plan_trace_entries(const infernt_plan* p, int steps) {
    if (!p || p->mode != INFERNT_MODE_PERSISTENT || steps <= 0) return 0;
    return (size_t)p->mega_ctas * steps * p->mega.nphases * kTraceFields;
}

int infernt_plan_set_trace(infernt_plan* p, unsigned long long* trace_dev) {
    INFERNT_REQUIRE(p, "plan_set_trace: null plan");
    INFERNT_REQUIRE(p->mode == INFERNT_MODE_PERSISTENT || !trace_dev, "plan_set_trace: persistent mode only");
    p->mega.trace = trace_dev;
    return INFERNT_OK;
}

int infernt_persistent_ctas(void) { return sm_count(); }

int infernt_plan_kernels_per_step(const infernt_plan* p) {
    if (!p) return 0;
    return p->mode == INFERNT_MODE_PERSISTENT ? 1 : 5 * p->cfg.num_layers + 1;
}

}  // extern "C"
