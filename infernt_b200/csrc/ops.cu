// ops.cu — the kernels.h entry points (include/kernels.h:5-49) as sm_100a
// kernels behind the C ABI, plus the general FP32 GEMM behind
// CublasWrapper::gemm (gemm/cublas_wrapper.cu:21-40).
//
// These are the per-op building blocks a caller of the reference's
// launch_* functions gets; the decode step itself runs the fused kernels
// of gemv.cu / attention.cu.  Reductions use fixed orders (deterministic);
// the reference's rmsnorm uses a shared-memory atomicAdd whose order varies
// run to run (cuda/rmsnorm.cu:19).
#include <cfloat>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "gemv.cuh"
#include "internal.h"

namespace infernt {
namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ float block_sum(float v, float* sh) {
    // fixed order: xor-shuffle within warps, then warps 0..7 in order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = 0.0f;
    const int nw = blockDim.x >> 5;
    for (int w = 0; w < nw; ++w) t += sh[w];
    return t;
}

__device__ __forceinline__ float block_max(float v, float* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = -FLT_MAX;
    const int nw = blockDim.x >> 5;
    for (int w = 0; w < nw; ++w) t = fmaxf(t, sh[w]);
    return t;
}

// cuda/rmsnorm.cu:4-27
__global__ void rmsnorm_kernel(float* out, const float* in, const float* w, int hidden, float eps) {
    __shared__ float sh[32];
    const float* x = in + (size_t)blockIdx.x * hidden;
    float* o = out + (size_t)blockIdx.x * hidden;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum(ss, sh);
    const float rms = rsqrtf(ss / (float)hidden + eps);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = x[i] * rms * w[i];
}

// cuda/residual.cu:4-10
__global__ void residual_kernel(float* out, const float* a, const float* b, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
}

// cuda/activation.cu:4-11
__global__ void silu_mul_kernel(float* out, const float* g, const float* u, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = silu_mul(g[i], u[i]);
}

// cuda/embedding.cu:3-8
__global__ void embedding_kernel(float* out, const float* table, int token, int hidden) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        out[i] = table[(size_t)token * hidden + i];
}

// cuda/rope.cu:5-35, applied to every batch row (the reference kernel
// rotates only the first row whatever batch_size is, rope.cu:37-45)
__global__ void rope_kernel(float* q, float* k, int nq, int nkv, int D, int pos, float theta) {
    const int b = blockIdx.y, head = blockIdx.x, half = D / 2;
    for (int d = threadIdx.x; d < half; d += blockDim.x) {
        const float freq = 1.0f / powf(theta, (float)(2 * d) / (float)D);
        const float angle = (float)pos * freq;
        const float c = cosf(angle), s = sinf(angle);
        if (head < nq) {
            float* p = q + ((size_t)b * nq + head) * D;
            const float a0 = p[d], a1 = p[d + half];
            p[d] = a0 * c - a1 * s;
            p[d + half] = a1 * c + a0 * s;
        }
        if (head < nkv) {
            float* p = k + ((size_t)b * nkv + head) * D;
            const float a0 = p[d], a1 = p[d + half];
            p[d] = a0 * c - a1 * s;
            p[d + half] = a1 * c + a0 * s;
        }
    }
}

// cuda/softmax.cu:5-49 (row stride = seq_len) and :51-99 (row stride = total,
// tail zeroed); one block per row, max / sum / normalise passes.
__global__ void softmax_kernel(float* out, const float* in, int seq_len, int total) {
    __shared__ float sh[32];
    const float* x = in + (size_t)blockIdx.x * total;
    float* o = out + (size_t)blockIdx.x * total;
    float m = -FLT_MAX;
    for (int i = threadIdx.x; i < seq_len; i += blockDim.x) m = fmaxf(m, x[i]);
    m = block_max(m, sh);
    float s = 0.0f;
    for (int i = threadIdx.x; i < seq_len; i += blockDim.x) s += expf(x[i] - m);
    s = block_sum(s, sh);
    const float inv = 1.0f / (s > 0.0f ? s : 1.0f);
    for (int i = threadIdx.x; i < total; i += blockDim.x)
        o[i] = i < seq_len ? expf(x[i] - m) * inv : 0.0f;
}

// cuda/kv_cache.cu:4-14, K and V in one launch
__global__ void kv_append_kernel(float* kc, float* vc, const float* kn, const float* vn, int D,
                                 int max_seq, int pos) {
    const int h = blockIdx.x;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const size_t dst = ((size_t)h * max_seq + pos) * D + d;
        kc[dst] = kn[(size_t)h * D + d];
        vc[dst] = vn[(size_t)h * D + d];
    }
}

// cuda/attention.cu:4-23: one warp per (q head, position); d in increasing
// order, then the product with scale.  Covers every position.
__global__ void attn_scores_kernel(float* scores, const float* q, const float* kc, int nq, int nkv,
                                   int D, int seq, int max_seq, float scale) {
    const int qh = blockIdx.x, lane = threadIdx.x & 31;
    const int p = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (p >= seq) return;
    const int kvh = qh / (nq / nkv);
    const float* qv = q + (size_t)qh * D;
    const float* kv = kc + ((size_t)kvh * max_seq + p) * D;
    // lane-contiguous partial sums over d, summed in lane order on lane 0
    float part = 0.0f;
    for (int d = lane; d < D; d += 32) part = fmaf(qv[d], kv[d], part);
    part = warp_sum(part);
    if (lane == 0) scores[(size_t)qh * seq + p] = part * scale;
}

// cuda/attention.cu:25-43: 8 warps split the positions of one (q head,
// 32-dim slice); partial sums combined in warp order.
__global__ void attn_values_kernel(float* out, const float* sc, const float* vc, int nq, int nkv,
                                   int D, int seq, int max_seq) {
    __shared__ float part[8][32];
    const int qh = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int d = blockIdx.y * 32 + lane;
    const int kvh = qh / (nq / nkv);
    float acc = 0.0f;
    if (d < D)
        for (int p = warp; p < seq; p += 8)
            acc = fmaf(sc[(size_t)qh * seq + p], vc[((size_t)kvh * max_seq + p) * D + d], acc);
    part[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && d < D) {
        float t = 0.0f;
        for (int w = 0; w < 8; ++w) t += part[w][lane];
        out[(size_t)qh * D + d] = t;
    }
}

// cuda/sampling.cu:3-36 as a grid-wide pass: per-block winner, the last
// block reduces winners in block order.  Ties -> lowest index.
struct ArgmaxWorkspace {
    float val[kArgmaxMaxBlocks];
    int idx[kArgmaxMaxBlocks];
    unsigned counter;
};

__global__ void argmax_kernel(int* out, const float* logits, int n, ArgmaxWorkspace* ws) {
    __shared__ float sv[kBlock / 32];
    __shared__ int si[kBlock / 32];
    __shared__ int s_last;
    float bv = -1e30f;
    int bi = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        if (argmax_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = -1e30f;
        int id = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
            if (argmax_better(sv[w], si[w], v, id)) { v = sv[w]; id = si[w]; }
        ws->val[blockIdx.x] = v;
        ws->idx[blockIdx.x] = id;
        __threadfence();
        s_last = atomicAdd(&ws->counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    float v = -1e30f;
    int id = 0;
    for (unsigned b = 0; b < gridDim.x; ++b) {
        const float pv = __ldcg(ws->val + b);
        const int pi = __ldcg(ws->idx + b);
        if (argmax_better(pv, pi, v, id)) { v = pv; id = pi; }
    }
    *out = id;
    ws->counter = 0u;
}

// Row-major FP32 GEMM, C = alpha op(A) op(B) + beta C (64x64 tile, 4x4 per
// thread, K in steps of 16).  Fixed summation order per output.
constexpr int TM = 64, TN = 64, TK = 16;
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* A, const float* B, float* C,
                                                       int M, int N, int K, float alpha, float beta,
                                                       int ta, int tb) {
    __shared__ float As[TK][TM + 1];
    __shared__ float Bs[TK][TN + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int i = threadIdx.x; i < TK * TM; i += 256) {
            const int kk = i / TM, mm = i % TM;
            const int gm = m0 + mm, gk = k0 + kk;
            float v = 0.0f;
            if (gm < M && gk < K) v = ta ? A[(size_t)gk * M + gm] : A[(size_t)gm * K + gk];
            As[kk][mm] = v;
        }
        for (int i = threadIdx.x; i < TK * TN; i += 256) {
            const int kk = i / TN, nn = i % TN;
            const int gn = n0 + nn, gk = k0 + kk;
            float v = 0.0f;
            if (gn < N && gk < K) v = tb ? B[(size_t)gn * K + gk] : B[(size_t)gk * N + gn];
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(As[kk][ty * 4 + i], Bs[kk][tx * 4 + j], acc[i][j]);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
            if (gm < M && gn < N) {
                float r = alpha * acc[i][j];
                if (beta != 0.0f) r += beta * C[(size_t)gm * N + gn];
                C[(size_t)gm * N + gn] = r;
            }
        }
}

int elementwise_grid(int n) {
    int g = (n + kBlock - 1) / kBlock;
    const int cap = sm_count() * 8;
    return g < 1 ? 1 : (g > cap ? cap : g);
}

// The argmax partials live in the module's own device memory (zeroed when
// the module loads on a device), so launch_argmax allocates nothing: the
// reference's kernels never allocate.  The last block resets the ticket, so
// the workspace is ready for the next launch; launches that overlap on one
// device (different streams) share it and must be ordered by the caller.
__device__ ArgmaxWorkspace g_argmax_ws_dev;

std::mutex g_ws_mu;
ArgmaxWorkspace* g_argmax_ws[64] = {nullptr};

int argmax_workspace(ArgmaxWorkspace** out) {
    const int d = current_device();
    INFERNT_REQUIRE(d >= 0 && d < 64, "argmax: device ordinal %d out of range", d);
    std::lock_guard<std::mutex> lk(g_ws_mu);
    if (!g_argmax_ws[d]) {
        void* p = nullptr;
        INFERNT_CUDA_TRY(cudaGetSymbolAddress(&p, g_argmax_ws_dev));
        g_argmax_ws[d] = static_cast<ArgmaxWorkspace*>(p);
    }
    *out = g_argmax_ws[d];
    return INFERNT_OK;
}

}  // namespace
}  // namespace infernt

using namespace infernt;

#define LAUNCH_CHECK() INFERNT_CUDA_TRY(cudaGetLastError())

extern "C" {

int infernt_rmsnorm(float* out, const float* in, const float* weight, int batch, int hidden,
                    float eps, void* stream) {
    INFERNT_REQUIRE(out && in && weight, "rmsnorm: null pointer");
    INFERNT_REQUIRE(batch >= 0 && hidden > 0, "rmsnorm: batch %d hidden %d", batch, hidden);
    if (batch == 0) return INFERNT_OK;
    rmsnorm_kernel<<<batch, kBlock, 0, (cudaStream_t)stream>>>(out, in, weight, hidden, eps);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_residual_add(float* out, const float* a, const float* b, int n, void* stream) {
    INFERNT_REQUIRE(out && a && b && n >= 0, "residual_add: bad arguments");
    if (n == 0) return INFERNT_OK;
    residual_kernel<<<elementwise_grid(n), kBlock, 0, (cudaStream_t)stream>>>(out, a, b, n);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_rope(float* q, float* k, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                 int position, float theta, void* stream) {
    INFERNT_REQUIRE(q && k, "rope: null pointer");
    INFERNT_REQUIRE(batch >= 0 && num_q_heads > 0 && num_kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0,
                    "rope: bad shape");
    if (batch == 0) return INFERNT_OK;
    const int heads = num_q_heads > num_kv_heads ? num_q_heads : num_kv_heads;
    rope_kernel<<<dim3(heads, batch), 64, 0, (cudaStream_t)stream>>>(q, k, num_q_heads, num_kv_heads,
                                                                     head_dim, position, theta);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_softmax(float* out, const float* in, int rows, int seq_len, void* stream) {
    INFERNT_REQUIRE(out && in && rows >= 0 && seq_len > 0, "softmax: bad arguments");
    if (rows == 0) return INFERNT_OK;
    softmax_kernel<<<rows, kBlock, 0, (cudaStream_t)stream>>>(out, in, seq_len, seq_len);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_softmax_with_mask(float* out, const float* in, int num_heads, int seq_len,
                              int total_seq_len, void* stream) {
    INFERNT_REQUIRE(out && in && num_heads >= 0 && seq_len > 0 && total_seq_len >= seq_len,
                    "softmax_with_mask: bad arguments");
    if (num_heads == 0) return INFERNT_OK;
    softmax_kernel<<<num_heads, kBlock, 0, (cudaStream_t)stream>>>(out, in, seq_len, total_seq_len);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_kv_cache_append(float* k_cache, float* v_cache, const float* k_new, const float* v_new,
                            int num_kv_heads, int head_dim, int max_seq_len, int position,
                            void* stream) {
    INFERNT_REQUIRE(k_cache && v_cache && k_new && v_new, "kv_cache_append: null pointer");
    INFERNT_REQUIRE(num_kv_heads > 0 && head_dim > 0, "kv_cache_append: bad shape");
    INFERNT_REQUIRE(position >= 0 && position < max_seq_len,
                    "kv_cache_append: position %d outside [0, %d)", position, max_seq_len);
    kv_append_kernel<<<num_kv_heads, 128, 0, (cudaStream_t)stream>>>(k_cache, v_cache, k_new, v_new,
                                                                      head_dim, max_seq_len, position);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_attention_scores(float* scores, const float* q, const float* k_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int seq_len, int max_seq_len,
                             float scale, void* stream) {
    INFERNT_REQUIRE(scores && q && k_cache, "attention_scores: null pointer");
    INFERNT_REQUIRE(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0 && head_dim > 0,
                    "attention_scores: bad head shape");
    INFERNT_REQUIRE(seq_len > 0 && seq_len <= max_seq_len, "attention_scores: seq_len %d max %d", seq_len,
                    max_seq_len);
    attn_scores_kernel<<<dim3(num_q_heads, (seq_len + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
        scores, q, k_cache, num_q_heads, num_kv_heads, head_dim, seq_len, max_seq_len, scale);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_attention_values(float* out, const float* scores, const float* v_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int seq_len, int max_seq_len,
                             void* stream) {
    INFERNT_REQUIRE(out && scores && v_cache, "attention_values: null pointer");
    INFERNT_REQUIRE(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0 && head_dim > 0,
                    "attention_values: bad head shape");
    INFERNT_REQUIRE(seq_len > 0 && seq_len <= max_seq_len, "attention_values: seq_len %d max %d", seq_len,
                    max_seq_len);
    attn_values_kernel<<<dim3(num_q_heads, (head_dim + 31) / 32), 256, 0, (cudaStream_t)stream>>>(
        out, scores, v_cache, num_q_heads, num_kv_heads, head_dim, seq_len, max_seq_len);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_silu_mul(float* out, const float* gate, const float* up, int n, void* stream) {
    INFERNT_REQUIRE(out && gate && up && n >= 0, "silu_mul: bad arguments");
    if (n == 0) return INFERNT_OK;
    silu_mul_kernel<<<elementwise_grid(n), kBlock, 0, (cudaStream_t)stream>>>(out, gate, up, n);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_embedding_lookup(float* out, const float* table, int token_id, int hidden, void* stream) {
    INFERNT_REQUIRE(out && table && hidden > 0 && token_id >= 0, "embedding_lookup: bad arguments");
    embedding_kernel<<<elementwise_grid(hidden), kBlock, 0, (cudaStream_t)stream>>>(out, table, token_id,
                                                                                   hidden);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_argmax(int* out_token, const float* logits, int vocab_size, void* stream) {
    INFERNT_REQUIRE(out_token && logits && vocab_size > 0, "argmax: bad arguments");
    ArgmaxWorkspace* ws = nullptr;
    if (int s = argmax_workspace(&ws)) return s;
    int grid = (vocab_size + kBlock * 4 - 1) / (kBlock * 4);
    const int cap = sm_count() * 2;
    if (grid > cap) grid = cap;
    if (grid > kArgmaxMaxBlocks) grid = kArgmaxMaxBlocks;
    if (grid < 1) grid = 1;
    argmax_kernel<<<grid, kBlock, 0, (cudaStream_t)stream>>>(out_token, logits, vocab_size, ws);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

int infernt_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K, float alpha,
                     float beta, int trans_a, int trans_b, void* stream) {
    INFERNT_REQUIRE(A && B && C, "gemm: null pointer");
    INFERNT_REQUIRE(M > 0 && N > 0 && K > 0, "gemm: M %d N %d K %d", M, N, K);
    if (M == 1 && trans_b && alpha == 1.0f && beta == 0.0f) {
        // the decode-step projection: y[n] = sum_k B[n][k] A[k] -> weight streaming
        return infernt_rmsnorm_gemv(C, B, N, nullptr, 0, nullptr, 0, K, INFERNT_DTYPE_F32, A, nullptr,
                                    0.0f, stream);
    }
    dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM);
    gemm_f32_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(A, B, C, M, N, K, alpha, beta, trans_a,
                                                            trans_b);
    LAUNCH_CHECK();
    return INFERNT_OK;
}

}  // extern "C"
