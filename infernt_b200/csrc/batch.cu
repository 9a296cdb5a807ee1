// batch.cu — the element-wise, attention and reduction kernels of batched
// decode (T sequences, one token each per step), around the tensor-core
// projections of bgemm.cu.  Per step and layer:
//
//   xb = bf16(RMSNorm(h))                       bt_resid_norm (or bt_embed_norm)
//   part = xb W_qkv^T                           bgemm (split-K partials)
//   q = RoPE(sum part), K/V rows appended       bt_qkv_finish
//   attention partials per (seq, KV head, split) bt_attn_partial
//   attn = bf16(merge of the splits)            bt_attn_merge
//   part = attn W_o^T; h += sum part; xb = ...  bgemm, bt_resid_norm
//   part = xb [W_gate; W_up]^T; act = bf16(silu(g) u)   bgemm, bt_swiglu
//   part = act W_down^T; h += sum part; xb = bf16(RMSNorm(h)) with the next norm
//   logits = xb W_lm^T, argmax per sequence     bgemm, bt_argmax
//
// The algorithms are the reference's decode step (architectures/llama/
// llama_layer.cpp:11-72, llama_model.cpp:45-65) applied to every sequence;
// activations enter the tensor cores as bf16 (rounded to nearest even) and
// the KV cache holds bf16 rows.  Partials are added in split order, so
// results do not depend on timing.
#include <cstdint>

#include "../../include/infernt_seed.h"
#include "attention.cuh"
#include "common.cuh"
#include "internal.h"

namespace infernt {

namespace {

__device__ __forceinline__ uint16_t bf16_bits(float v) {
    return (uint16_t)(__float_as_uint(infernt_round_bf16(v)) >> 16);
}
__device__ __forceinline__ float bf16_float(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// sum over the splits of part[s][t][j] (in split order)
__device__ __forceinline__ float sum_parts(const float* part, int splits, size_t stride, size_t off) {
    float v = part[off];
    for (int s = 1; s < splits; ++s) v += part[(size_t)s * stride + off];
    return v;
}

// RMSNorm of the row x[0, H) (cuda/rmsnorm.cu:10-26) into bf16 xb; block-wide.
__device__ void norm_row_bf16(const float* x, const float* w, int H, float eps, uint16_t* xb, float* red) {
    const int tid = threadIdx.x, nt = blockDim.x;
    float ss = 0.0f;
    for (int i = tid; i < H; i += nt) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int w8 = 0; w8 < nt / 32; ++w8) t += red[w8];
        red[32] = rsqrtf(t / (float)H + eps);
    }
    __syncthreads();
    const float rms = red[32];
    for (int i = tid; i < H; i += nt) xb[i] = bf16_bits(x[i] * rms * w[i]);
}

// h[t] = embedding row of tokens[t]; xb[t] = bf16(RMSNorm(h[t])).
__global__ void bt_embed_norm(const float* emb, const int* tokens, int vocab, int H, const float* norm_w, float eps,
                              float* h, uint16_t* xb, unsigned* err) {
    __shared__ float red[33];
    const int t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, kErrToken);
        tok = 0;
    }
    float* ht = h + (size_t)t * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ht[i] = emb[(size_t)tok * H + i];
    __syncthreads();
    norm_row_bf16(ht, norm_w, H, eps, xb + (size_t)t * H, red);
}

// h[t] += sum of the partials; xb[t] = bf16(RMSNorm(h[t], norm_w)).
__global__ void bt_resid_norm(const float* part, int splits, int T, int H, float* h, const float* norm_w, float eps,
                              uint16_t* xb) {
    __shared__ float red[33];
    const int t = blockIdx.x;
    float* ht = h + (size_t)t * H;
    const size_t stride = (size_t)T * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ht[i] += sum_parts(part, splits, stride, (size_t)t * H + i);
    __syncthreads();
    norm_row_bf16(ht, norm_w, H, eps, xb + (size_t)t * H, red);
}

// Q|K|V of token t: q rows RoPE'd into q (FP32), K (RoPE'd) and V rows
// rounded to bf16 and appended at the sequence's position
// (cuda/rope.cu:13-34, cuda/kv_cache.cu:4-14).  Cache [T][Nkv][max_seq][D].
__global__ void bt_qkv_finish(const float* part, int splits, int T, int nq, int nkv, int D, const int* positions,
                              const float2* rope, int max_seq, float* q, uint16_t* kc, uint16_t* vc, unsigned* err) {
    const int t = blockIdx.x;
    const int N = (nq + 2 * nkv) * D, half = D / 2;
    const size_t stride = (size_t)T * N, row = (size_t)t * N;
    const int pos = positions[t];
    if (pos < 0 || pos >= max_seq) {
        if (threadIdx.x == 0) atomicOr(err, kErrPosition);
        return;
    }
    const float2* rp = rope + (size_t)pos * half;
    // q and k pairs (d, d + D/2) of every head
    for (int i = threadIdx.x; i < (nq + nkv) * half; i += blockDim.x) {
        const int hd = i / half, d = i % half;
        const size_t j = (size_t)hd * D + d;
        float a = sum_parts(part, splits, stride, row + j), b = sum_parts(part, splits, stride, row + j + half);
        rope_apply(a, b, rp[d]);
        if (hd < nq) {
            q[(size_t)t * nq * D + j] = a;
            q[(size_t)t * nq * D + j + half] = b;
        } else {
            const int kh = hd - nq;
            uint16_t* dst = kc + (((size_t)t * nkv + kh) * max_seq + pos) * D;
            dst[d] = bf16_bits(a);
            dst[d + half] = bf16_bits(b);
        }
    }
    for (int i = threadIdx.x; i < nkv * D; i += blockDim.x) {
        const int kh = i / D, d = i % D;
        const float v = sum_parts(part, splits, stride, row + (size_t)(nq + nkv) * D + i);
        vc[(((size_t)t * nkv + kh) * max_seq + pos) * D + d] = bf16_bits(v);
    }
}

// act[t][i] = bf16(silu(gate) * up) from the partials of the stacked
// [gate; up] projection (cuda/activation.cu:7-9).
__global__ void bt_swiglu(const float* part, int splits, int T, int I, uint16_t* act) {
    const int t = blockIdx.x;
    const size_t N = (size_t)2 * I, stride = (size_t)T * N, row = (size_t)t * N;
    for (int i = threadIdx.x; i < I; i += blockDim.x) {
        const float g = sum_parts(part, splits, stride, row + i);
        const float u = sum_parts(part, splits, stride, row + I + i);
        act[(size_t)t * I + i] = bf16_bits(silu_mul(g, u));
    }
}

// Positions per attention tile and the chunk of a split.
constexpr int kBtTile = 32;
constexpr int kBtMinChunk = 64;

__device__ __forceinline__ void bt_chunk(int seq, int splits, int& chunk, int& active) {
    chunk = (seq + splits - 1) / splits;
    if (chunk < kBtMinChunk) chunk = kBtMinChunk;
    active = (seq + chunk - 1) / chunk;
}

// Partial attention of (sequence t, KV head kvh, split) over its positions
// (cuda/attention.cu:9-22, :30-42 with online softmax): G query heads,
// D = 32 DL.  Warp w takes heads w, w + 4, ...; in the score pass lane p
// takes position p of a 32-position tile, in the value pass lane l takes
// columns l, l + 32, ....  The next tile's bf16 rows are loaded into
// registers while the current tile is used.  Partials [T][Nkv][S][G][D + 2].
template <int DL, int HW>
__global__ void __launch_bounds__(128) bt_attn_partial(const float* q, const uint16_t* kc, const uint16_t* vc,
                                                       const int* positions, int nq, int nkv, int max_seq, int S,
                                                       float scale, float* part) {
    constexpr int D = 32 * DL, T = kBtTile, NW = 4;
    constexpr int CPR = D / 8;                 // 16-byte chunks per row
    constexpr int CH = (T * CPR + 127) / 128;  // chunks per thread per tile (K or V)
    __shared__ float qs[16 * D];
    __shared__ float kt[T][D + 1];
    __shared__ float vt[T][D];
    __shared__ float ps[16][T];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = nq / nkv;
    const int item = blockIdx.x;
    const int split = item % S, kvh = (item / S) % nkv, t = item / (S * nkv);
    const int seq = positions[t] + 1;
    int chunk, active;
    bt_chunk(seq, S, chunk, active);
    if (split >= active) return;
    const int c0 = split * chunk, c1 = min(seq, c0 + chunk);
    const uint16_t* kb = kc + ((size_t)t * nkv + kvh) * max_seq * D;
    const uint16_t* vb = vc + ((size_t)t * nkv + kvh) * max_seq * D;
    for (int i = tid; i < G * D; i += 128) qs[i] = q[((size_t)t * nq + (size_t)kvh * G) * D + i];

    uint4 kr[CH], vr[CH];
    auto load = [&](int p0, int n) {
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int e = tid + c * 128, r = e / CPR, cc = e % CPR;
            if (e < T * CPR && r < n) {
                kr[c] = *reinterpret_cast<const uint4*>(kb + (size_t)(p0 + r) * D + cc * 8);
                vr[c] = *reinterpret_cast<const uint4*>(vb + (size_t)(p0 + r) * D + cc * 8);
            }
        }
    };
    float m_run[HW], l_run[HW], o_run[HW][DL];
#pragma unroll
    for (int j = 0; j < HW; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < DL; ++i) o_run[j][i] = 0.0f;
    }
    int tl = min(T, c1 - c0);
    load(c0, tl);
    for (int p0 = c0; p0 < c1; p0 += T) {
        __syncthreads();  // the previous tile's readers are done
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int e = tid + c * 128, r = e / CPR, cc = e % CPR;
            if (e < T * CPR && r < tl) {
                const uint16_t* kk = reinterpret_cast<const uint16_t*>(&kr[c]);
                const uint16_t* vv = reinterpret_cast<const uint16_t*>(&vr[c]);
#pragma unroll
                for (int x = 0; x < 8; ++x) {
                    kt[r][cc * 8 + x] = bf16_float(kk[x]);
                    vt[r][cc * 8 + x] = bf16_float(vv[x]);
                }
            }
        }
        __syncthreads();
        const int cur = tl;
        const int nxt = p0 + T;
        if (nxt < c1) {
            tl = min(T, c1 - nxt);
            load(nxt, tl);
        }
#pragma unroll
        for (int j = 0; j < HW; ++j) {
            const int h = warp + j * NW;
            if (h < G) {
                float s = -INFINITY;
                if (lane < cur) {
                    float d0 = 0.0f, d1 = 0.0f;
                    const float* qh = qs + h * D;
#pragma unroll 8
                    for (int d = 0; d < D; d += 2) {
                        d0 = fmaf(qh[d], kt[lane][d], d0);
                        d1 = fmaf(qh[d + 1], kt[lane][d + 1], d1);
                    }
                    s = (d0 + d1) * scale;
                }
                const float m_new = fmaxf(m_run[j], warp_max(s));
                const float alpha = expf(m_run[j] - m_new);
                const float pe = lane < cur ? expf(s - m_new) : 0.0f;
                ps[h][lane] = pe;
                l_run[j] = l_run[j] * alpha + warp_sum(pe);
                m_run[j] = m_new;
                __syncwarp();
                float acc[DL];
#pragma unroll
                for (int i = 0; i < DL; ++i) acc[i] = o_run[j][i] * alpha;
#pragma unroll 4
                for (int p = 0; p < cur; ++p) {
                    const float pp = ps[h][p];
#pragma unroll
                    for (int i = 0; i < DL; ++i) acc[i] = fmaf(pp, vt[p][lane + 32 * i], acc[i]);
                }
#pragma unroll
                for (int i = 0; i < DL; ++i) o_run[j][i] = acc[i];
            }
        }
    }
#pragma unroll
    for (int j = 0; j < HW; ++j) {
        const int h = warp + j * NW;
        if (h < G) {
            float* pp = part + ((((size_t)t * nkv + kvh) * S + split) * G + h) * (D + 2);
            if (lane == 0) {
                pp[0] = m_run[j];
                pp[1] = l_run[j];
            }
#pragma unroll
            for (int i = 0; i < DL; ++i) pp[2 + lane + 32 * i] = o_run[j][i];
        }
    }
}

// Merge of the active splits of (t, kvh) in split order; output bf16
// attn[t][(kvh G + h) D + d].
__global__ void bt_attn_merge(const float* part, const int* positions, int nq, int nkv, int D, int S,
                              uint16_t* attn) {
    const int t = blockIdx.x / nkv, kvh = blockIdx.x % nkv;
    const int G = nq / nkv;
    int chunk, active;
    bt_chunk(positions[t] + 1, S, chunk, active);
    const float* pk = part + ((size_t)t * nkv + kvh) * S * G * (D + 2);
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
        const int h = e / D, d = e % D;
        float M = -INFINITY;
        for (int s = 0; s < active; ++s) M = fmaxf(M, pk[((size_t)s * G + h) * (D + 2)]);
        float L = 0.0f, acc = 0.0f;
        for (int s = 0; s < active; ++s) {
            const float* pp = pk + ((size_t)s * G + h) * (D + 2);
            const float w = expf(pp[0] - M);
            L = fmaf(pp[1], w, L);
            acc = fmaf(pp[2 + d], w, acc);
        }
        attn[(size_t)t * nq * D + (size_t)kvh * G * D + e] = bf16_bits(acc / L);
    }
}

// Greedy next token of sequence t (lowest index among equal maxima;
// cuda/sampling.cu:3-40), then position + 1.
__global__ void bt_argmax(const float* logits, int V, int* tokens, int* positions, int* hist) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* lt = logits + (size_t)t * V;
    float v = -INFINITY;
    int id = 0;
    for (int i = tid; i < V; i += blockDim.x)
        if (argmax_better(lt[i], i, v, id)) {
            v = lt[i];
            id = i;
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, id, o);
        if (argmax_better(ov, oi, v, id)) {
            v = ov;
            id = oi;
        }
    }
    if ((tid & 31) == 0) {
        bv[tid >> 5] = v;
        bi[tid >> 5] = id;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)blockDim.x / 32; ++w)
            if (argmax_better(bv[w], bi[w], v, id)) {
                v = bv[w];
                id = bi[w];
            }
        tokens[t] = id;
        if (hist) hist[t] = id;
        positions[t] += 1;
    }
}

// Rows [0, n_pos) of sequence `seq`'s cache of one layer, [T][Nkv][max_seq][D]
// bf16: element (layer, h, p, d) of the seeded KV stream (include/infernt_seed.h),
// the values infernt_fill_kv writes in FP32, rounded to bf16.
__global__ void bt_fill_kv(uint16_t* cache, int seq, int layer, int nkv, int max_seq, int D, int n_pos,
                           uint64_t key, float std_dev) {
    const size_t n = (size_t)nkv * n_pos * D;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int p = (int)((i / D) % n_pos);
        const int h = (int)(i / ((size_t)D * n_pos));
        const uint64_t gi = ((((uint64_t)layer * nkv + h) << 20) + (uint64_t)p) * (uint64_t)D + d;
        cache[(((size_t)seq * nkv + h) * max_seq + p) * D + d] = bf16_bits(infernt_normal_std(key, gi, std_dev));
    }
}

__global__ void bt_rope_table(float2* tab, int max_seq, int D, float theta) {
    const int half = D / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)max_seq * half;
         i += (long long)gridDim.x * blockDim.x)
        tab[i] = rope_factors((int)(i % half), D, (int)(i / half), theta);
}

}  // namespace

// ------------------------------------------------------------ host side

int bt_rope_table_launch(float2* tab, int max_seq, int D, float theta, cudaStream_t st) {
    bt_rope_table<<<256, 256, 0, st>>>(tab, max_seq, D, theta);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_embed_norm_launch(const float* emb, const int* tokens, int vocab, int T, int H, const float* norm_w, float eps,
                         float* h, uint16_t* xb, unsigned* err, cudaStream_t st) {
    bt_embed_norm<<<T, 256, 0, st>>>(emb, tokens, vocab, H, norm_w, eps, h, xb, err);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_resid_norm_launch(const float* part, int splits, int T, int H, float* h, const float* norm_w, float eps,
                         uint16_t* xb, cudaStream_t st) {
    bt_resid_norm<<<T, 256, 0, st>>>(part, splits, T, H, h, norm_w, eps, xb);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_qkv_finish_launch(const float* part, int splits, int T, int nq, int nkv, int D, const int* positions,
                         const float2* rope, int max_seq, float* q, uint16_t* kc, uint16_t* vc, unsigned* err,
                         cudaStream_t st) {
    bt_qkv_finish<<<T, 256, 0, st>>>(part, splits, T, nq, nkv, D, positions, rope, max_seq, q, kc, vc, err);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_swiglu_launch(const float* part, int splits, int T, int I, uint16_t* act, cudaStream_t st) {
    bt_swiglu<<<T, 256, 0, st>>>(part, splits, T, I, act);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

// Attention of every sequence: partials over `S` splits per (t, KV head),
// then the merge.  D in {64, 128}, G = nq / nkv <= 16.
int bt_attention_launch(const float* q, const uint16_t* kc, const uint16_t* vc, const int* positions, int T, int nq,
                        int nkv, int D, int max_seq, int S, float* part, uint16_t* attn, cudaStream_t st) {
    const int G = nq / nkv;
    INFERNT_REQUIRE(G >= 1 && G <= 16 && nq % nkv == 0, "batched attention: group size %d", G);
    const float scale = 1.0f / sqrtf((float)D);
    const int items = T * nkv * S;
    if (D == 64) {
        if (G <= 4)
            bt_attn_partial<2, 1><<<items, 128, 0, st>>>(q, kc, vc, positions, nq, nkv, max_seq, S, scale, part);
        else if (G <= 8)
            bt_attn_partial<2, 2><<<items, 128, 0, st>>>(q, kc, vc, positions, nq, nkv, max_seq, S, scale, part);
        else
            bt_attn_partial<2, 4><<<items, 128, 0, st>>>(q, kc, vc, positions, nq, nkv, max_seq, S, scale, part);
    } else if (D == 128) {
        if (G <= 4)
            bt_attn_partial<4, 1><<<items, 128, 0, st>>>(q, kc, vc, positions, nq, nkv, max_seq, S, scale, part);
        else if (G <= 8)
            bt_attn_partial<4, 2><<<items, 128, 0, st>>>(q, kc, vc, positions, nq, nkv, max_seq, S, scale, part);
        else
            bt_attn_partial<4, 4><<<items, 128, 0, st>>>(q, kc, vc, positions, nq, nkv, max_seq, S, scale, part);
    } else {
        return fail(INFERNT_ERR_UNSUPPORTED, "batched attention: head_dim %d (64 or 128)", D);
    }
    INFERNT_CUDA_TRY(cudaGetLastError());
    bt_attn_merge<<<T * nkv, 128, 0, st>>>(part, positions, nq, nkv, D, S, attn);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_fill_kv_launch(uint16_t* cache, int seq, int layer, int nkv, int max_seq, int D, int n_pos, uint64_t key,
                      float std_dev, cudaStream_t st) {
    if (n_pos <= 0) return INFERNT_OK;
    bt_fill_kv<<<256, 256, 0, st>>>(cache, seq, layer, nkv, max_seq, D, n_pos, key, std_dev);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_argmax_launch(const float* logits, int T, int V, int* tokens, int* positions, int* hist, cudaStream_t st) {
    bt_argmax<<<T, 256, 0, st>>>(logits, V, tokens, positions, hist);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

}  // namespace infernt
