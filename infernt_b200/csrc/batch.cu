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
#include "sample.cuh"
#include "warp_mma.cuh"

namespace infernt {

namespace {

constexpr int kMaxSplits = 8;   // K splits of a batched projection (bgemm partials)

// Sum over the splits of part[s][t][off .. off + 3] (in split order): every
// split's 16 bytes are loaded first, so a thread waits one round trip, not
// one per split.
__device__ __forceinline__ float4 sum_parts4(const float* part, int splits, size_t stride, size_t off) {
    float4 w[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s)
        if (s < splits) w[s] = *reinterpret_cast<const float4*>(part + (size_t)s * stride + off);
    float4 v = w[0];
#pragma unroll
    for (int s = 1; s < kMaxSplits; ++s)
        if (s < splits) {
            v.x += w[s].x;
            v.y += w[s].y;
            v.z += w[s].z;
            v.w += w[s].w;
        }
    return v;
}

// RMSNorm (cuda/rmsnorm.cu:10-26) of a row of H = 4 x blockDim.x values,
// thread i holding elements [4 i, 4 i + 4) in v, into bf16 xb.
__device__ void norm_row_bf16(float4 v, const float* w, int H, float eps, uint16_t* xb, float* red) {
    const int tid = threadIdx.x, nt = blockDim.x;
    float ss = v.x * v.x;
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
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
    const float4 g = *reinterpret_cast<const float4*>(w + 4 * tid);
    const uint32_t lo = (uint32_t)bf16_bits(v.x * rms * g.x) | ((uint32_t)bf16_bits(v.y * rms * g.y) << 16);
    const uint32_t hi = (uint32_t)bf16_bits(v.z * rms * g.z) | ((uint32_t)bf16_bits(v.w * rms * g.w) << 16);
    *reinterpret_cast<uint2*>(xb + 4 * tid) = make_uint2(lo, hi);
}

// h[t] = embedding row of tokens[t]; xb[t] = bf16(RMSNorm(h[t])).  H / 4 threads.
__global__ void bt_embed_norm(const float* emb, const int* tokens, int vocab, int H, const float* norm_w, float eps,
                              float* h, uint16_t* xb, unsigned* err) {
    pdl_wait();  // the previous kernel of the step has completed
    pdl_launch_dependents();
    __shared__ float red[33];
    const int t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, kErrToken);
        tok = 0;
    }
    const float4 v = *reinterpret_cast<const float4*>(emb + (size_t)tok * H + 4 * threadIdx.x);
    *reinterpret_cast<float4*>(h + (size_t)t * H + 4 * threadIdx.x) = v;
    norm_row_bf16(v, norm_w, H, eps, xb + (size_t)t * H, red);
}

// h[t] += sum of the partials; xb[t] = bf16(RMSNorm(h[t], norm_w)).  H / 4 threads.
__global__ void bt_resid_norm(const float* part, int splits, int T, int H, float* h, const float* norm_w, float eps,
                              uint16_t* xb) {
    pdl_wait();  // the previous kernel of the step has completed
    pdl_launch_dependents();
    __shared__ float red[33];
    const int t = blockIdx.x;
    float4* hp = reinterpret_cast<float4*>(h + (size_t)t * H + 4 * threadIdx.x);
    const float4 y = sum_parts4(part, splits, (size_t)T * H, (size_t)t * H + 4 * threadIdx.x);
    float4 v = *hp;
    v.x += y.x;
    v.y += y.y;
    v.z += y.z;
    v.w += y.w;
    *hp = v;
    norm_row_bf16(v, norm_w, H, eps, xb + (size_t)t * H, red);
}

// Q|K|V of token t: q rows RoPE'd into q (FP32), K (RoPE'd) and V rows
// rounded to bf16 and appended at the sequence's position
// (cuda/rope.cu:13-34, cuda/kv_cache.cu:4-14).  Cache [T][Nkv][max_seq][D].
__global__ void bt_qkv_finish(const float* part, int splits, int T, int nq, int nkv, int D, const int* positions,
                              const float2* rope, int max_seq, float* q, uint16_t* kc, uint16_t* vc, unsigned* err) {
    pdl_wait();  // the previous kernel of the step has completed
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const int N = (nq + 2 * nkv) * D, half = D / 2;
    const size_t stride = (size_t)T * N, row = (size_t)t * N;
    const int pos = positions[t];
    if (pos < 0 || pos >= max_seq) {
        if (threadIdx.x == 0) atomicOr(err, kErrPosition);
        return;
    }
    const float2* rp = rope + (size_t)pos * half;
    // q and k: four pairs (d .. d + 3, d + D/2 .. d + D/2 + 3) per unit
    const int qk_units = (nq + nkv) * (half / 4);
    for (int u = threadIdx.x; u < qk_units; u += blockDim.x) {
        const int hd = u / (half / 4), d = (u % (half / 4)) * 4;
        const size_t j = (size_t)hd * D + d;
        const float4 a4 = sum_parts4(part, splits, stride, row + j), b4 = sum_parts4(part, splits, stride, row + j + half);
        float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) rope_apply(a[e], b[e], rp[d + e]);
        if (hd < nq) {
            float* qd = q + (size_t)t * nq * D + j;
            *reinterpret_cast<float4*>(qd) = make_float4(a[0], a[1], a[2], a[3]);
            *reinterpret_cast<float4*>(qd + half) = make_float4(b[0], b[1], b[2], b[3]);
        } else {
            const int kh = hd - nq;
            uint16_t* dst = kc + (((size_t)t * nkv + kh) * max_seq + pos) * D;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                dst[d + e] = bf16_bits(a[e]);
                dst[d + half + e] = bf16_bits(b[e]);
            }
        }
    }
    for (int u = threadIdx.x; u < nkv * D / 4; u += blockDim.x) {
        const int i = 4 * u, kh = i / D, d = i % D;
        const float4 v = sum_parts4(part, splits, stride, row + (size_t)(nq + nkv) * D + i);
        uint16_t* dst = vc + (((size_t)t * nkv + kh) * max_seq + pos) * D + d;
        dst[0] = bf16_bits(v.x);
        dst[1] = bf16_bits(v.y);
        dst[2] = bf16_bits(v.z);
        dst[3] = bf16_bits(v.w);
    }
}

// act[t][i] = bf16(silu(gate) * up) from the partials of the stacked
// [gate; up] projection (cuda/activation.cu:7-9).
__global__ void bt_swiglu(const float* part, int splits, int T, int I, uint16_t* act) {
    pdl_wait();  // the previous kernel of the step has completed
    pdl_launch_dependents();
    const int t = blockIdx.y;
    const size_t N = (size_t)2 * I, stride = (size_t)T * N, row = (size_t)t * N;
    const int i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= I) return;
    const float4 g = sum_parts4(part, splits, stride, row + i), u = sum_parts4(part, splits, stride, row + I + i);
    const uint32_t lo = (uint32_t)bf16_bits(silu_mul(g.x, u.x)) | ((uint32_t)bf16_bits(silu_mul(g.y, u.y)) << 16);
    const uint32_t hi = (uint32_t)bf16_bits(silu_mul(g.z, u.z)) | ((uint32_t)bf16_bits(silu_mul(g.w, u.w)) << 16);
    *reinterpret_cast<uint2*>(act + (size_t)t * I + i) = make_uint2(lo, hi);
}

// The chunk of a split: seq / splits positions, at least min_chunk; the
// splits past the sequence's last chunk are inactive.
__device__ __forceinline__ void bt_chunk(int seq, int splits, int min_chunk, int& chunk, int& active) {
    chunk = (seq + splits - 1) / splits;
    if (chunk < min_chunk) chunk = min_chunk;
    active = (seq + chunk - 1) / chunk;
}

// Partial attention of (sequence t, KV head kvh, split) over its positions
// (cuda/attention.cu:9-22, :30-42 with online softmax), G query heads,
// D = 32 DL.  Each warp takes 32 positions at a time: in the score pass lane
// p holds position p and scores it against all G heads (q in shared memory,
// the key row read once, 16 dimensions at a time); after the per-head online
// softmax update the value pass gives lane l the DL columns [DL l, DL l +
// DL) of every head.  The four warps' (m, l, o) are merged in shared memory
// in warp order into the split's partial [T][Nkv][S][G][D + 2].
template <int DL, int G>
__global__ void __launch_bounds__(128) bt_attn_partial(const float* q, const uint16_t* kc, const uint16_t* vc,
                                                       const int* positions, int nq, int nkv, int max_seq, int S,
                                                       int min_chunk, float scale, float* part) {
    pdl_wait();
    pdl_launch_dependents();
    constexpr int D = 32 * DL, NW = 4;
    __shared__ __align__(16) float qs[G * D];
    __shared__ __align__(16) float ps[NW][32][G];     // probabilities of the warp's 32 positions
    __shared__ float wm[NW][G], wl[NW][G];
    __shared__ float wo[NW][G][D];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int item = blockIdx.x;
    const int split = item % S, kvh = (item / S) % nkv, t = item / (S * nkv);
    const int seq = positions[t] + 1;
    int chunk, active;
    bt_chunk(seq, S, min_chunk, chunk, active);
    if (split >= active || seq > max_seq) return;  // positions past the cache are not read
    const int c0 = split * chunk, c1 = min(seq, c0 + chunk);
    const uint16_t* kb = kc + ((size_t)t * nkv + kvh) * max_seq * D;
    const uint16_t* vb = vc + ((size_t)t * nkv + kvh) * max_seq * D;
    for (int i = tid; i < G * D; i += 128) qs[i] = q[((size_t)t * nq + (size_t)kvh * G) * D + i];
    __syncthreads();

    float m_run[G], l_run[G], o_run[G][DL];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
#pragma unroll
        for (int i = 0; i < DL; ++i) o_run[h][i] = 0.0f;
    }
    for (int p0 = c0 + warp * 32; p0 < c1; p0 += NW * 32) {
        const int n = min(32, c1 - p0);
        const int p = p0 + lane;
        // scores of position p against every head
        float sc[G];
#pragma unroll
        for (int h = 0; h < G; ++h) sc[h] = 0.0f;
        if (lane < n) {
            const uint4* kr = reinterpret_cast<const uint4*>(kb + (size_t)p * D);
#pragma unroll
            for (int c = 0; c < D / 16; ++c) {
                const uint4 k0 = kr[2 * c], k1 = kr[2 * c + 1];
                const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
                float kf[16];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    kf[2 * e] = __uint_as_float(kw[e] << 16);
                    kf[2 * e + 1] = __uint_as_float(kw[e] & 0xffff0000u);
                }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float4* qh = reinterpret_cast<const float4*>(qs + h * D + 16 * c);
                    float acc = sc[h];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float4 qq = qh[e];
                        acc = fmaf(qq.x, kf[4 * e], acc);
                        acc = fmaf(qq.y, kf[4 * e + 1], acc);
                        acc = fmaf(qq.z, kf[4 * e + 2], acc);
                        acc = fmaf(qq.w, kf[4 * e + 3], acc);
                    }
                    sc[h] = acc;
                }
            }
        }
        // online softmax per head over the warp's positions
        float alpha[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float s = lane < n ? sc[h] * scale : -INFINITY;
            const float m_new = fmaxf(m_run[h], warp_max(s));
            alpha[h] = expf(m_run[h] - m_new);
            const float pe = lane < n ? expf(s - m_new) : 0.0f;
            ps[warp][lane][h] = pe;
            l_run[h] = l_run[h] * alpha[h] + warp_sum(pe);
            m_run[h] = m_new;
        }
        __syncwarp();
        // values: lane l takes columns [DL l, DL l + DL) of every head
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
            for (int i = 0; i < DL; ++i) o_run[h][i] *= alpha[h];
        // the sub-tile's value rows (DL bf16 columns per lane) are loaded
        // together before they are used
        uint32_t vw[32][DL / 2];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < n) {
                const uint16_t* vr = vb + (size_t)(p0 + j) * D + DL * lane;
                if (DL == 2) {
                    vw[j][0] = *reinterpret_cast<const uint32_t*>(vr);
                } else {
                    const uint2 w = *reinterpret_cast<const uint2*>(vr);
                    vw[j][0] = w.x;
                    vw[j][(DL / 2) - 1] = w.y;
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (j < n) {
                float vf[DL];
#pragma unroll
                for (int i = 0; i < DL / 2; ++i) {
                    vf[2 * i] = __uint_as_float(vw[j][i] << 16);
                    vf[2 * i + 1] = __uint_as_float(vw[j][i] & 0xffff0000u);
                }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float pj = ps[warp][j][h];
#pragma unroll
                    for (int i = 0; i < DL; ++i) o_run[h][i] = fmaf(pj, vf[i], o_run[h][i]);
                }
            }
        }
        __syncwarp();
    }
    // merge the warps' states (warp order) into the split's partial
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
            wm[warp][h] = m_run[h];
            wl[warp][h] = l_run[h];
        }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int i = 0; i < DL; ++i) wo[warp][h][DL * lane + i] = o_run[h][i];
    __syncthreads();
    for (int e = tid; e < G * D; e += 128) {
        const int h = e / D, d = e % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][h]);
        float L = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float f = wm[w][h] == -INFINITY ? 0.0f : expf(wm[w][h] - M);
            L = fmaf(wl[w][h], f, L);
            acc = fmaf(wo[w][h][d], f, acc);
        }
        float* pp = part + ((((size_t)t * nkv + kvh) * S + split) * G + h) * (D + 2);
        if (d == 0) {
            pp[0] = M;
            pp[1] = L;
        }
        pp[2 + d] = acc;
    }
}

// ---- attention partials on the tensor cores (mma.sync m16n8k16, bf16)
//
// The same partial as bt_attn_partial for head groups of up to 8 query
// heads, with the two dot products on the tensor cores.  The bf16 keys and
// values are exact MMA operands; the FP32 queries and probabilities are
// split into three bf16 terms x = hi + mid + lo (hi = bf16(x), mid =
// bf16(x - hi), lo = bf16(x - hi - mid): 24 mantissa bits, as FP32) and two
// MMAs take them: rows 0-7 of the first A operand hold the hi terms of the
// group's heads and rows 8-15 the mid terms, rows 0-7 of the second the lo
// terms (rows 8-15 zero), both into one accumulator, so a head's value is
// the sum of its two accumulator rows.
//   scores  S[16 x 8 positions] = Qsplit[16 x D] K^T      (2 D / 16 MMAs)
//   output  O[16 x D]         += Psplit[16 x 16 pos] V     (2 D / 8 MMAs)
// Each warp streams 32-position tiles of K and V into its own ring of
// attn_stages<D>() shared-memory stages with 16-byte cp.async copies (rows past
// the split's end are zero-filled), the 16-byte chunks of a row stored at
// chunk ^ (row & 7) so that ldmatrix reads are conflict-free.  Warp w takes
// tiles w, w + 4, ...; online softmax per warp (quad shuffles for the row
// maxima), then the four warps' (m, l, o) are merged in warp order into the
// split's partial [T][Nkv][S][G][D + 2] exactly as bt_attn_partial does.
constexpr int kAttnTile = 32;

template <int D, int NST>
constexpr int attn_smem_bytes() {
    return 4 * NST * 2 * kAttnTile * D * 2;
}

// Arguments of the tensor-core attention.  Standalone: q [T][nq][D] FP32
// with RoPE applied and caches already holding every position.  Fused
// (qkv_part set): the Q|K|V projection's split partials part[s][t][(nq +
// 2 nkv) D]; the kernel sums them in split order, applies RoPE to q and k
// (the table rope[pos][D / 2]) and appends the bf16 K and V rows at
// positions[t] (what bt_qkv_finish does, bit for bit).  With S == 1 the
// kernel writes attn (and attn_f32) itself; otherwise the split partials,
// and with tickets given the last split CTA of each (t, KV head) to finish
// merges them (in split order, as bt_attn_merge) and leaves its ticket at 0.
struct BtAttnArgs {
    const float* q;
    const float* qkv_part;
    int qkv_splits;
    const float2* rope;
    uint16_t* kc;
    uint16_t* vc;
    const int* positions;
    int T, nq, nkv, G, max_seq, S, min_chunk;
    float scale;
    float* part;
    uint16_t* attn;
    float* attn_f32;
    unsigned* err;
    unsigned* tickets;  // [T][nkv] zeros, or NULL (S > 1: a separate merge launch)
    // paged caches (block_table set): kc / vc are pools of pages
    // [page][nkv][page_size][D]; position p of sequence t lives in page
    // block_table[t][p / page_size] at row p % page_size.  A sequence at
    // position -1 is an empty slot: skipped without an error.
    const int* block_table;
    int page_size, max_pages;
};

// Address of cache row p of (sequence t, KV head kvh): contiguous
// [T][nkv][max_seq][D], or its page (paged caches).
template <int D>
__device__ __forceinline__ size_t bt_row_off(const BtAttnArgs& a, int t, int kvh, int p) {
    if (!a.block_table) return (((size_t)t * a.nkv + kvh) * a.max_seq + p) * D;
    const int page = a.block_table[(size_t)t * a.max_pages + p / a.page_size];
    return (((size_t)page * a.nkv + kvh) * a.page_size + p % a.page_size) * D;
}

template <int D>
constexpr int attn_extra_bytes() {
    return 8 * D * 4 + 2 * D * 2;  // q of up to 8 heads (FP32), the new K and V rows (bf16)
}

template <int D, int NST, bool FUSED>
__global__ void __launch_bounds__(128) bt_attn_mma(const BtAttnArgs a) {
    constexpr int NW = 4;
    constexpr int ROWB = D * 2, CH = ROWB / 16;           // bytes and 16-byte chunks per cache row
    constexpr int TILEB = kAttnTile * ROWB;              // one K (or V) tile
    constexpr int KC = D / 16, DB = D / 8;               // k-steps of the scores, d-blocks of the output
    extern __shared__ __align__(128) unsigned char att_smem[];
    float* qs = reinterpret_cast<float*>(att_smem + attn_smem_bytes<D, NST>());   // [8][D]
    uint16_t* newk = reinterpret_cast<uint16_t*>(qs + 8 * D);                     // [D]
    uint16_t* newv = newk + D;                                                      // [D]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int S = a.S, nkv = a.nkv, nq = a.nq, G = a.G, max_seq = a.max_seq;
    const int item = blockIdx.x;
    const int split = item % S, kvh = (item / S) % nkv, t = item / (S * nkv);
    // positions are final before the step's first kernel, and the cache rows
    // below them were written by kernels that have completed: the tile
    // copies may start before the projection this kernel depends on
    const int pos = a.positions[t];
    if (pos < 0 || pos >= max_seq) {
        if (FUSED && tid == 0 && a.err && !(a.block_table && pos == -1)) atomicOr(a.err, kErrPosition);
        return;
    }
    const int seq = pos + 1;
    int chunk, active;
    bt_chunk(seq, S, a.min_chunk, chunk, active);
    if (split >= active) return;
    const int c0 = split * chunk, c1 = min(seq, c0 + chunk);
    const bool own_row = FUSED && split == active - 1;  // this split holds position pos
    const int ntiles = (c1 - c0 + kAttnTile - 1) / kAttnTile;
    const unsigned char* kb = reinterpret_cast<const unsigned char*>(a.kc);
    const unsigned char* vb = reinterpret_cast<const unsigned char*>(a.vc);
    const uint32_t ring = smem_addr(att_smem) + (uint32_t)warp * NST * 2 * TILEB;

    // this warp's tile i of the split -> stage i % NST (K at +0, V at +TILEB).
    // Row of position p: off0 + p below `bound`, else off1 + p — one base
    // for contiguous caches, and for pages of at least a tile the tile's
    // one or two pages (looked up once per tile); smaller pages look up
    // every row.  Rows past the split (ok false) copy nothing from p0's row.
    const bool row_pages = a.block_table && a.page_size < kAttnTile;
    auto issue = [&](int i) {
        const int tile = warp + NW * i;
        if (tile < ntiles) {
            const int p0 = c0 + tile * kAttnTile;
            const uint32_t st = ring + (uint32_t)(i % NST) * 2 * TILEB;
            long long off0 = ((long long)t * nkv + kvh) * max_seq, off1 = off0;
            int bound = max_seq;
            if (a.block_table && !row_pages) {
                const int P = a.page_size, pi = p0 / P, last = min(p0 + kAttnTile, c1) - 1;
                const int* tab = a.block_table + (size_t)t * a.max_pages;
                bound = (pi + 1) * P;
                off0 = ((long long)tab[pi] * nkv + kvh) * P - (long long)pi * P;
                if (last >= bound) off1 = ((long long)tab[pi + 1] * nkv + kvh) * P - (long long)bound;
            }
#pragma unroll
            for (int e = 0; e < kAttnTile * CH / 32; ++e) {
                const int idx = e * 32 + lane, row = idx / CH, ch = idx % CH;
                const bool ok = p0 + row < c1;
                const int pp = ok ? p0 + row : p0;
                const size_t r = row_pages ? bt_row_off<D>(a, t, kvh, pp) / D
                                           : (size_t)((pp < bound ? off0 : off1) + pp);
                const size_t off = r * ROWB + (size_t)ch * 16;
                const uint32_t dst = st + (uint32_t)(row * ROWB + ((ch ^ (row & 7)) << 4));
                cp_async16(dst, kb + off, ok ? 16u : 0u);
                cp_async16(dst + TILEB, vb + off, ok ? 16u : 0u);
            }
        }
        cp_async_commit();
    };
    const int my_tiles = ntiles > warp ? (ntiles - warp + NW - 1) / NW : 0;
#pragma unroll
    for (int i = 0; i < NST - 1; ++i) issue(i);  // row pos of a fused step is patched in below
    pdl_wait();

    // queries of the group (and the new K / V rows) into shared memory
    if (FUSED) {
        const int N = (nq + 2 * nkv) * D, half = D / 2;
        const size_t stride = (size_t)a.T * N;
        const float* pr = a.qkv_part + (size_t)t * N;
        const float2* rp = a.rope + (size_t)pos * half;
        // the split partials of columns col and col + half: every split's
        // value is loaded before the in-order sums (one round trip)
        auto sum2 = [&](int col, float& x, float& y) {
            float wx[kMaxSplits], wy[kMaxSplits];
#pragma unroll
            for (int s = 0; s < kMaxSplits; ++s)
                if (s < a.qkv_splits) {
                    wx[s] = pr[(size_t)s * stride + col];
                    wy[s] = pr[(size_t)s * stride + col + half];
                }
            x = wx[0];
            y = wy[0];
#pragma unroll
            for (int s = 1; s < kMaxSplits; ++s)
                if (s < a.qkv_splits) {
                    x += wx[s];
                    y += wy[s];
                }
        };
        for (int e = tid; e < G * half; e += 128) {
            const int h = e / half, d = e % half;
            float x, y;
            sum2((kvh * G + h) * D + d, x, y);
            rope_apply(x, y, rp[d]);
            qs[h * D + d] = x;
            qs[h * D + d + half] = y;
        }
        if (own_row && tid < half) {
            // thread d: k pair (d, d + half) with RoPE, v elements d and d + half
            float x, y, u, w;
            sum2((nq + kvh) * D + tid, x, y);
            sum2((nq + nkv + kvh) * D + tid, u, w);
            rope_apply(x, y, rp[tid]);
            newk[tid] = bf16_bits(x);
            newk[tid + half] = bf16_bits(y);
            newv[tid] = bf16_bits(u);
            newv[tid + half] = bf16_bits(w);
        }
        __syncthreads();
        if (own_row && tid < 2 * CH) {
            // the rows for later steps (16 bytes per thread)
            const uint16_t* src = tid < CH ? newk : newv;
            uint16_t* dst = (tid < CH ? a.kc : a.vc) + bt_row_off<D>(a, t, kvh, pos);
            const int c = tid % CH;
            *reinterpret_cast<uint4*>(dst + 8 * c) = *reinterpret_cast<const uint4*>(src + 8 * c);
        }
    } else {
        const float* qg = a.q + ((size_t)t * nq + (size_t)kvh * G) * D;
        for (int e = tid; e < G * D; e += 128) qs[e] = qg[e];
        __syncthreads();
    }

    // query fragments: qa rows g / g + 8 = hi / mid terms of head g, ql row
    // g = its lo terms (rows g + 8 of the second operand are zero)
    uint32_t qa[KC][4], ql[KC][4];
#pragma unroll
    for (int k = 0; k < KC; ++k) {
        float2 lo2 = make_float2(0.f, 0.f), hi2 = make_float2(0.f, 0.f);
        if (g < G) {
            lo2 = *reinterpret_cast<const float2*>(qs + g * D + 16 * k + 2 * tig);
            hi2 = *reinterpret_cast<const float2*>(qs + g * D + 16 * k + 2 * tig + 8);
        }
        split3_bf16x2(lo2.x, lo2.y, qa[k][0], qa[k][1], ql[k][0]);
        split3_bf16x2(hi2.x, hi2.y, qa[k][2], qa[k][3], ql[k][2]);
        ql[k][1] = ql[k][3] = 0u;
    }
    float m_run = -INFINITY, l_run = 0.0f;
    float acc[DB][4];
#pragma unroll
    for (int b = 0; b < DB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.0f;

    for (int i = 0; i < my_tiles; ++i) {
        issue(i + NST - 1);  // the stage it fills was read in iteration i - 1 (synced below)
        cp_async_wait<NST - 1>();
        __syncwarp();
        const uint32_t kt = ring + (uint32_t)(i % NST) * 2 * TILEB, vt = kt + TILEB;
        const int p0 = c0 + (warp + NW * i) * kAttnTile;
        if (own_row && pos < p0 + kAttnTile) {
            // the new row replaces what the copy read at position pos
            if (lane < 2 * CH) {
                const int r = pos - p0, c = lane % CH;
                const uint32_t dst = (lane < CH ? kt : vt) + (uint32_t)(r * ROWB + ((c ^ (r & 7)) << 4));
                const uint4 v = *reinterpret_cast<const uint4*>((lane < CH ? newk : newv) + 8 * c);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z),
                             "r"(v.w)
                             : "memory");
            }
            __syncwarp();
        }
        // scores: hi / mid terms in sc, lo terms in sl (two shorter MMA chains)
        float sc[4][4], sl[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[j][e] = sl[j][e] = 0.0f;
#pragma unroll
        for (int k = 0; k < KC; ++k)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int m = lane >> 3, row = 8 * (2 * jj + (m >> 1)) + (lane & 7), ch = 2 * k + (m & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kt + (uint32_t)(row * ROWB + ((ch ^ (row & 7)) << 4)), b0, b1, b2, b3);
                mma_bf16_16816(sc[2 * jj], qa[k], b0, b1);
                mma_bf16_16816(sl[2 * jj], ql[k], b0, b1);
                mma_bf16_16816(sc[2 * jj + 1], qa[k], b2, b3);
                mma_bf16_16816(sl[2 * jj + 1], ql[k], b2, b3);
            }
        // online softmax of head g over the tile (each quad holds one head)
        float sv[4][2], mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int p = p0 + 8 * j + 2 * tig + e;
                sv[j][e] = p < c1 ? ((sc[j][e] + sc[j][e + 2]) + sl[j][e]) * a.scale : -INFINITY;
                mx = fmaxf(mx, sv[j][e]);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = expf(m_run - m_new);
        m_run = m_new;
        float lsum = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sv[j][e] = expf(sv[j][e] - m_new);
                lsum += sv[j][e];
            }
        l_run = l_run * alpha + lsum;
#pragma unroll
        for (int b = 0; b < DB; ++b)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[b][e] *= alpha;
        // output: probabilities of 16 positions per k-step as the A operand
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            uint32_t pa[4], pl[4];
            split3_bf16x2(sv[2 * kk][0], sv[2 * kk][1], pa[0], pa[1], pl[0]);
            split3_bf16x2(sv[2 * kk + 1][0], sv[2 * kk + 1][1], pa[2], pa[3], pl[2]);
            pl[1] = pl[3] = 0u;
#pragma unroll
            for (int b2 = 0; b2 < DB / 2; ++b2) {
                const int m = lane >> 3, row = 16 * kk + 8 * (m & 1) + (lane & 7), ch = 2 * b2 + (m >> 1);
                uint32_t v0, v1, v2, v3;
                ldsm_x4_trans(vt + (uint32_t)(row * ROWB + ((ch ^ (row & 7)) << 4)), v0, v1, v2, v3);
                mma_bf16_16816(acc[2 * b2], pa, v0, v1);
                mma_bf16_16816(acc[2 * b2], pl, v0, v1);
                mma_bf16_16816(acc[2 * b2 + 1], pa, v2, v3);
                mma_bf16_16816(acc[2 * b2 + 1], pl, v2, v3);
            }
        }
        __syncwarp();  // every lane has read the stage before it is refilled
    }
    cp_async_wait<0>();
    // the next kernel's CTAs may start once every CTA is past its main loop
    // (earlier, they would hold SM slots the second wave of this grid needs)
    pdl_launch_dependents();
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    __syncthreads();  // the rings are reused for the merge
    float* wm = reinterpret_cast<float*>(att_smem);      // [NW][8]
    float* wl = wm + NW * 8;                              // [NW][8]
    float* wo = wl + NW * 8;                              // [NW][8][D]
    if (tig == 0) {
        wm[warp * 8 + g] = m_run;
        wl[warp * 8 + g] = l_run;
    }
#pragma unroll
    for (int b = 0; b < DB; ++b) {
        float* o = wo + ((size_t)warp * 8 + g) * D + 8 * b + 2 * tig;
        o[0] = acc[b][0] + acc[b][2];
        o[1] = acc[b][1] + acc[b][3];
    }
    __syncthreads();
    for (int e = tid; e < G * D; e += 128) {
        const int h = e / D, d = e % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w * 8 + h]);
        float L = 0.0f, acc_o = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float mw = wm[w * 8 + h];
            const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
            L = fmaf(wl[w * 8 + h], f, L);
            acc_o = fmaf(wo[((size_t)w * 8 + h) * D + d], f, acc_o);
        }
        if (S == 1) {
            const size_t o = (size_t)t * nq * D + (size_t)kvh * G * D + e;
            a.attn[o] = bf16_bits(acc_o / L);
            if (a.attn_f32) a.attn_f32[o] = acc_o / L;
        } else {
            float* pp = a.part + ((((size_t)t * nkv + kvh) * S + split) * G + h) * (D + 2);
            if (d == 0) {
                pp[0] = M;
                pp[1] = L;
            }
            pp[2 + d] = acc_o;
        }
    }
    if (S == 1 || !a.tickets) return;
    // the last split of (t, kvh) to finish merges the active splits
    __shared__ unsigned s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned* tk = a.tickets + (size_t)t * nkv + kvh;
        const unsigned done = atomicAdd(tk, 1u) + 1u;
        s_last = done == (unsigned)active;
        if (s_last) *tk = 0u;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* pk = a.part + ((size_t)t * nkv + kvh) * S * G * (D + 2);
    for (int e = tid; e < G * D; e += 128) {
        const int h = e / D, d = e % D;
        float M = -INFINITY;
        for (int sp = 0; sp < active; ++sp) M = fmaxf(M, __ldcg(pk + ((size_t)sp * G + h) * (D + 2)));
        float L = 0.0f, acc_o = 0.0f;
        for (int sp = 0; sp < active; ++sp) {
            const float* pp = pk + ((size_t)sp * G + h) * (D + 2);
            const float w = expf(__ldcg(pp) - M);
            L = fmaf(__ldcg(pp + 1), w, L);
            acc_o = fmaf(__ldcg(pp + 2 + d), w, acc_o);
        }
        const size_t o = (size_t)t * nq * D + (size_t)kvh * G * D + e;
        a.attn[o] = bf16_bits(acc_o / L);
        if (a.attn_f32) a.attn_f32[o] = acc_o / L;
    }
}

// Merge of the active splits of (t, kvh) in split order; output bf16
// attn[t][(kvh G + h) D + d] (and the FP32 value in attn_f32 when given).
__global__ void bt_attn_merge(const float* part, const int* positions, int nq, int nkv, int D, int S,
                              int min_chunk, uint16_t* attn, float* attn_f32) {
    pdl_wait();  // the previous kernel of the step has completed
    pdl_launch_dependents();
    const int t = blockIdx.x / nkv, kvh = blockIdx.x % nkv;
    const int G = nq / nkv;
    int chunk, active;
    bt_chunk(positions[t] + 1, S, min_chunk, chunk, active);
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
        const size_t o = (size_t)t * nq * D + (size_t)kvh * G * D + e;
        attn[o] = bf16_bits(acc / L);
        if (attn_f32) attn_f32[o] = acc / L;
    }
}

// Greedy next token of sequence t (lowest index among equal maxima;
// cuda/sampling.cu:3-40), then position + 1.  Grid (kArgChunks, T): CTA
// (c, t) reduces chunk c of the vocabulary (every thread's float4 loads in
// flight at once) to a candidate; the last chunk CTA of t to finish (split
// ticket, left at 0) combines the candidates in chunk order.
constexpr int kArgChunks = 8;

__global__ void __launch_bounds__(256) bt_argmax(const float* logits, int V, int* tokens, int* positions, int* hist,
                                                 float* cand_v, int* cand_i, unsigned* tickets, float inv_t,
                                                 uint64_t seed, const uint64_t* salts) {
    pdl_wait();  // the previous kernel of the step has completed
    pdl_launch_dependents();
    __shared__ float bv[8];
    __shared__ int bi[8];
    const int chunk = blockIdx.x, t = blockIdx.y, tid = threadIdx.x;
    const int n4 = V / 4;
    const int c0 = (int)((long long)n4 * chunk / kArgChunks), c1 = (int)((long long)n4 * (chunk + 1) / kArgChunks);
    const float4* lt = reinterpret_cast<const float4*>(logits + (size_t)t * V);
    // temperature sampling (inv_t > 0): Gumbel scores keyed by (seed, the
    // sequence's position), so chained steps draw fresh noise without a host
    // counter; every chunk reads the position before the last one advances it.
    // With salts (a value per sequence, e.g. its request id) the key is
    // (stream_key(seed, salt), position): sequences at one position draw
    // independent noise
    const bool sample = inv_t > 0.0f;
    const uint64_t base = salts ? infernt_stream_key(seed, salts[t]) : seed;
    const uint64_t key = sample ? infernt_stream_key(base, (uint64_t)positions[t]) : 0;
    float v = -INFINITY;
    int id = 4 * c0;  // equal to the old single-pass start (index 0) once chunks combine in order
#pragma unroll 4
    for (int i = c0 + tid; i < c1; i += 256) {
        const float4 x = lt[i];
        float xs[4] = {x.x, x.y, x.z, x.w};
        if (sample)
#pragma unroll
            for (int e = 0; e < 4; ++e) xs[e] = gumbel_score(xs[e], inv_t, key, (uint64_t)(4 * i + e));
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (argmax_better(xs[e], 4 * i + e, v, id)) {
                v = xs[e];
                id = 4 * i + e;
            }
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
    if (tid != 0) return;
    for (int w = 1; w < 8; ++w)
        if (argmax_better(bv[w], bi[w], v, id)) {
            v = bv[w];
            id = bi[w];
        }
    cand_v[(size_t)t * kArgChunks + chunk] = v;
    cand_i[(size_t)t * kArgChunks + chunk] = id;
    __threadfence();
    const unsigned done = atomicAdd(tickets + t, 1u) + 1u;
    if (done != (unsigned)kArgChunks) return;
    tickets[t] = 0u;
    __threadfence();
    v = __ldcg(cand_v + (size_t)t * kArgChunks);
    id = __ldcg(cand_i + (size_t)t * kArgChunks);
    for (int c = 1; c < kArgChunks; ++c) {
        const float cv = __ldcg(cand_v + (size_t)t * kArgChunks + c);
        const int ci = __ldcg(cand_i + (size_t)t * kArgChunks + c);
        if (argmax_better(cv, ci, v, id)) {
            v = cv;
            id = ci;
        }
    }
    tokens[t] = id;
    if (hist) hist[t] = id;
    if (positions[t] >= 0) positions[t] += 1;  // an empty slot (position -1) stays empty
}

// Rows [0, n_pos) of sequence `seq`'s cache of one layer, [T][Nkv][max_seq][D]
// bf16: element (layer, h0 + h, p, d) of the seeded KV stream of a model with
// nkv_all KV heads (include/infernt_seed.h; h0 > 0 on a tensor-parallel rank
// holding heads [h0, h0 + nkv)), the values infernt_fill_kv writes in FP32,
// rounded to bf16.  Paged caches (pages set): the pool [page][Nkv][P][D],
// position p in page pages[p / P] at row p % P.
__global__ void bt_fill_kv(uint16_t* cache, int seq, int layer, int nkv, int max_seq, int D, int n_pos,
                           uint64_t key, float std_dev, int h0, int nkv_all, const int* pages, int page_size) {
    const size_t n = (size_t)nkv * n_pos * D;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int p = (int)((i / D) % n_pos);
        const int h = (int)(i / ((size_t)D * n_pos));
        const uint64_t gi = ((((uint64_t)layer * nkv_all + h0 + h) << 20) + (uint64_t)p) * (uint64_t)D + d;
        const size_t row = pages ? ((size_t)pages[p / page_size] * nkv + h) * page_size + p % page_size
                                 : ((size_t)seq * nkv + h) * max_seq + p;
        cache[row * D + d] = bf16_bits(infernt_normal_std(key, gi, std_dev));
    }
}

// Rows [p0, p1) of one sequence between a contiguous cache [Nkv][max_seq][D]
// and its pages of a pool [page][Nkv][P][D] (to_pages: contiguous -> pages),
// 16 bytes per thread and step.
__global__ void bt_page_copy(uint16_t* pool, uint16_t* flat, const int* pages, int page_size, int nkv, int max_seq,
                             int D, int p0, int p1, int to_pages) {
    const int ch = D / 8;  // 16-byte chunks per row
    const size_t n = (size_t)nkv * (p1 - p0) * ch;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % ch);
        const int p = p0 + (int)((i / ch) % (p1 - p0));
        const int h = (int)(i / ((size_t)ch * (p1 - p0)));
        uint4* a = reinterpret_cast<uint4*>(flat + ((size_t)h * max_seq + p) * D) + c;
        uint4* b = reinterpret_cast<uint4*>(
                       pool + (((size_t)pages[p / page_size] * nkv + h) * page_size + p % page_size) * D) + c;
        if (to_pages)
            *b = *a;
        else
            *a = *b;
    }
}

// ---------------------------------------------------- tensor parallelism
// y[t][n] = sum of the partials part[s][t][n] in split order: a rank's share
// of an O or down projection before the all-reduce over the ranks.
__global__ void tp_sum_splits(const float* part, int splits, int T, int N, float* y) {
    pdl_wait();
    pdl_launch_dependents();
    const size_t n4 = (size_t)T * N / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
        reinterpret_cast<float4*>(y)[i] = sum_parts4(part, splits, (size_t)T * N, 4 * i);
}

// ------------------------------------- peer-memory exchange of the sums
// In place of an NCCL all-reduce after the O and down projections, each
// rank pushes its sum of the split partials [T][N] into slot [rank] of every
// rank's exchange region (CUDA IPC mappings over NVLink) as tagged words
// (value | tag << 32, one 8-byte store each: a reader that sees the tag has
// the value), and the residual + RMSNorm kernel of every rank adds the
// world slots of its own region in rank order, so every rank holds the same
// bits.  A region is two buffers [2][world][T][N] taken in turn (buffer idx &
// 1 of the step's idx-th exchange), so a rank one exchange ahead never
// overwrites a slot a peer still reads.  Tags: epoch x per_step + idx + 1,
// the epoch advanced once per step on the device (bt_epoch_advance).

__device__ __forceinline__ void tp_st_sys2(unsigned long long* a, unsigned long long w0, unsigned long long w1) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(a), "l"(w0), "l"(w1) : "memory");
}

__device__ __forceinline__ ulonglong2 tp_ld_sys2(const unsigned long long* a) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(a) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long tp_pack(float v, unsigned tag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
}

__device__ __forceinline__ unsigned tp_tag(const unsigned* epoch, int per_step, int idx) {
    return *epoch * (unsigned)per_step + (unsigned)idx + 1u;
}

__global__ void bt_epoch_advance(unsigned* epoch) {
    pdl_wait();
    pdl_launch_dependents();
    ++*epoch;
}

// This rank's sum of the split partials into slot [rank] of buffer idx & 1 of
// every rank's region (peers[r] = rank r's region, own included).
__global__ void tp_push(const float* part, int splits, int T, int N, unsigned long long* const* peers, int rank,
                        int world, const unsigned* epoch, int per_step, int idx) {
    pdl_wait();
    pdl_launch_dependents();
    const unsigned tag = tp_tag(epoch, per_step, idx);
    const size_t n = (size_t)T * N;
    const size_t base = ((size_t)(idx & 1) * world + rank) * n;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n / 4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = sum_parts4(part, splits, n, 4 * i);
        const unsigned long long w0 = tp_pack(v.x, tag), w1 = tp_pack(v.y, tag), w2 = tp_pack(v.z, tag),
                                 w3 = tp_pack(v.w, tag);
        for (int r = 0; r < world; ++r) {
            unsigned long long* d = peers[r] + base + 4 * i;
            tp_st_sys2(d, w0, w1);
            tp_st_sys2(d + 2, w2, w3);
        }
    }
}

// h[t] += the world ranks' sums (rank order) from this rank's region;
// xb[t] = bf16(RMSNorm(h[t], norm_w)).  H / 4 threads.  Waits for the
// peers' words at most `budget` SM cycles (then kErrWaitTimeout).
__global__ void bt_resid_norm_tp(const unsigned long long* own, int world, int T, int H, float* h,
                                 const float* norm_w, float eps, uint16_t* xb, const unsigned* epoch, int per_step,
                                 int idx, unsigned* err, long long budget) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float red[33];
    const int t = blockIdx.x;
    const unsigned tag = tp_tag(epoch, per_step, idx);
    const size_t n = (size_t)T * H;
    const unsigned long long* b = own + (size_t)(idx & 1) * world * n + (size_t)t * H + 4 * threadIdx.x;
    float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const long long t0 = clock64();
    bool late = false;
    for (int r = 0; r < world; ++r) {
        const unsigned long long* a = b + (size_t)r * n;
        ulonglong2 lo = tp_ld_sys2(a), hi = tp_ld_sys2(a + 2);
        auto ok = [&]() {
            return (unsigned)(lo.x >> 32) == tag && (unsigned)(lo.y >> 32) == tag && (unsigned)(hi.x >> 32) == tag &&
                   (unsigned)(hi.y >> 32) == tag;
        };
        while (!ok() && !late) {
            if (clock64() - t0 > budget) {
                atomicOr(err, kErrWaitTimeout);
                late = true;
                break;
            }
            lo = tp_ld_sys2(a);
            hi = tp_ld_sys2(a + 2);
        }
        y.x += __uint_as_float((unsigned)lo.x);
        y.y += __uint_as_float((unsigned)lo.y);
        y.z += __uint_as_float((unsigned)hi.x);
        y.w += __uint_as_float((unsigned)hi.y);
    }
    float4* hp = reinterpret_cast<float4*>(h + (size_t)t * H + 4 * threadIdx.x);
    float4 v = *hp;
    v.x += y.x;
    v.y += y.y;
    v.z += y.z;
    v.w += y.w;
    *hp = v;
    norm_row_bf16(v, norm_w, H, eps, xb + (size_t)t * H, red);
}

// Greedy pick of sequence t over this rank's vocabulary rows: logits [T][ld]
// (rows [0, vl) valid, vocabulary ids v0 + row) -> cand[t] = (value, id).
// The lowest id wins among equal values; NaN never wins.
__global__ void __launch_bounds__(256) tp_argmax_local(const float* logits, int ld, int vl, int v0, int2* cand,
                                                       const int* positions, float inv_t, uint64_t seed) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float bv[8];
    __shared__ int bi[8];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* row = logits + (size_t)t * ld;
    const bool sample = inv_t > 0.0f;  // Gumbel scores over global vocabulary ids, as bt_argmax
    const uint64_t key = sample ? infernt_stream_key(seed, (uint64_t)positions[t]) : 0;
    float v = -INFINITY;
    int id = v0;
    for (int i = tid; i < vl; i += 256) {
        const float x = sample ? gumbel_score(row[i], inv_t, key, (uint64_t)(v0 + i)) : row[i];
        if (argmax_better(x, v0 + i, v, id)) {
            v = x;
            id = v0 + i;
        }
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
    if (tid != 0) return;
    for (int w = 1; w < 8; ++w)
        if (argmax_better(bv[w], bi[w], v, id)) {
            v = bv[w];
            id = bi[w];
        }
    cand[t] = make_int2(__float_as_int(v), id);
}

// Every rank's candidates cand_all [world][T] (gathered in rank order) ->
// the sequence's token (the same on every rank) and its next position.
__global__ void tp_argmax_pick(const int2* cand_all, int world, int T, int* tokens, int* positions) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    float v = -INFINITY;
    int id = 0x7fffffff;
    for (int r = 0; r < world; ++r) {
        const int2 c = cand_all[(size_t)r * T + t];
        if (argmax_better(__int_as_float(c.x), c.y, v, id)) {
            v = __int_as_float(c.x);
            id = c.y;
        }
    }
    if (id == 0x7fffffff) id = 0;  // every logit NaN
    tokens[t] = id;
    positions[t] += 1;
}

__global__ void bt_rope_table(float2* tab, int max_seq, int D, float theta) {
    const int half = D / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)max_seq * half;
         i += (long long)gridDim.x * blockDim.x)
        tab[i] = rope_factors((int)(i % half), D, (int)(i / half), theta);
}

// Launches k with programmatic dependent launch: it may start while the
// previous kernel of the stream finishes; it waits (griddepcontrol.wait)
// before it touches that kernel's outputs.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_smem(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
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
    INFERNT_REQUIRE(H % 128 == 0 && H / 4 <= 1024, "batched decode: hidden size %d", H);
    INFERNT_CUDA_TRY(launch_pdl(bt_embed_norm, dim3(T), dim3(H / 4), st, emb, tokens, vocab, H, norm_w, eps, h, xb, err));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_resid_norm_launch(const float* part, int splits, int T, int H, float* h, const float* norm_w, float eps,
                         uint16_t* xb, cudaStream_t st) {
    INFERNT_REQUIRE(H % 128 == 0 && H / 4 <= 1024 && splits <= kMaxSplits, "batched decode: hidden %d, splits %d", H,
                    splits);
    INFERNT_CUDA_TRY(launch_pdl(bt_resid_norm, dim3(T), dim3(H / 4), st, part, splits, T, H, h, norm_w, eps, xb));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_qkv_finish_launch(const float* part, int splits, int T, int nq, int nkv, int D, const int* positions,
                         const float2* rope, int max_seq, float* q, uint16_t* kc, uint16_t* vc, unsigned* err,
                         cudaStream_t st) {
    INFERNT_REQUIRE(D % 8 == 0 && splits <= kMaxSplits, "batched decode: head_dim %d, splits %d", D, splits);
    INFERNT_CUDA_TRY(launch_pdl(bt_qkv_finish, dim3(T), dim3(256), st, part, splits, T, nq, nkv, D, positions, rope, max_seq, q, kc, vc, err));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_swiglu_launch(const float* part, int splits, int T, int I, uint16_t* act, cudaStream_t st) {
    INFERNT_REQUIRE(I % 4 == 0 && splits <= kMaxSplits, "batched decode: intermediate %d, splits %d", I, splits);
    INFERNT_CUDA_TRY(launch_pdl(bt_swiglu, dim3((I / 4 + 127) / 128, T), dim3(128), st, part, splits, T, I, act));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

namespace {

template <int D, int NST, bool FUSED>
int launch_attn_mma(const BtAttnArgs& a, int items, cudaStream_t st) {
    static bool raised = false;
    constexpr int smem = attn_smem_bytes<D, NST>() + attn_extra_bytes<D>();
    if (!raised) {
        INFERNT_CUDA_TRY(
            cudaFuncSetAttribute(bt_attn_mma<D, NST, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        raised = true;
    }
    INFERNT_CUDA_TRY(launch_pdl_smem(bt_attn_mma<D, NST, FUSED>, dim3(items), dim3(128), (size_t)smem, st, a));
    return INFERNT_OK;
}

template <bool FUSED>
int attn_mma_dispatch(const BtAttnArgs& a, int D, int stages, cudaStream_t st) {
    INFERNT_REQUIRE(stages >= 2 && stages <= (D == 64 ? 4 : 3), "batched attention: %d stages for head_dim %d", stages,
                    D);
    const int items = a.T * a.nkv * a.S;
    if (D == 64) {
        if (stages == 2) return launch_attn_mma<64, 2, FUSED>(a, items, st);
        if (stages == 3) return launch_attn_mma<64, 3, FUSED>(a, items, st);
        return launch_attn_mma<64, 4, FUSED>(a, items, st);
    }
    if (stages == 2) return launch_attn_mma<128, 2, FUSED>(a, items, st);
    return launch_attn_mma<128, 3, FUSED>(a, items, st);
}

int attn_merge(const BtAttnArgs& a, int D, cudaStream_t st) {
    if (a.S == 1 || a.tickets) return INFERNT_OK;  // the partial kernel wrote the output
    INFERNT_CUDA_TRY(launch_pdl(bt_attn_merge, dim3(a.T * a.nkv), dim3(128), st, (const float*)a.part, a.positions,
                                a.nq, a.nkv, D, a.S, a.min_chunk, a.attn, a.attn_f32));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

}  // namespace

// Attention of every sequence: partials over `S` splits per (t, KV head),
// each a chunk of at least min_chunk positions, then the merge (none for S =
// 1).  D in {64, 128}; groups of up to 8 query heads run on the tensor cores
// (bt_attn_mma, `stages` cp.async stages per warp), groups of 16 (D = 64) on
// CUDA cores (bt_attn_partial).
int bt_attention_launch(const float* q, const uint16_t* kc, const uint16_t* vc, const int* positions, int T, int nq,
                        int nkv, int D, int max_seq, int S, int min_chunk, int stages, float* part, uint16_t* attn,
                        cudaStream_t st, float* attn_f32) {
    const int G = nq / nkv;
    INFERNT_REQUIRE(G >= 1 && G <= 16 && nq % nkv == 0, "batched attention: group size %d", G);
    INFERNT_REQUIRE(S >= 1 && min_chunk >= 1, "batched attention: splits %d, min_chunk %d", S, min_chunk);
    const float scale = 1.0f / sqrtf((float)D);
    BtAttnArgs a = {};
    a.q = q;
    a.kc = const_cast<uint16_t*>(kc);
    a.vc = const_cast<uint16_t*>(vc);
    a.positions = positions;
    a.T = T;
    a.nq = nq;
    a.nkv = nkv;
    a.G = G;
    a.max_seq = max_seq;
    a.S = S;
    a.min_chunk = min_chunk;
    a.scale = scale;
    a.part = part;
    a.attn = attn;
    a.attn_f32 = attn_f32;
    if (G <= 8 && (D == 64 || D == 128)) {
        if (int s = attn_mma_dispatch<false>(a, D, stages, st)) return s;
        INFERNT_CUDA_TRY(cudaGetLastError());
        return attn_merge(a, D, st);
    }
    if (!(D == 64 && G == 16)) {
        if (D == 64 || D == 128)
            return fail(INFERNT_ERR_UNSUPPORTED, "batched attention: group size %d (1 to 8, or 16 at head_dim 64)", G);
        return fail(INFERNT_ERR_UNSUPPORTED, "batched attention: head_dim %d (64 or 128)", D);
    }
    const int items = T * nkv * S;
    INFERNT_CUDA_TRY(launch_pdl(bt_attn_partial<2, 16>, dim3(items), dim3(128), st, q, kc, vc, positions, nq, nkv,
                                max_seq, S, min_chunk, scale, part));
    INFERNT_CUDA_TRY(cudaGetLastError());
    a.S = S;
    // the CUDA-core partials always write partials: merge even for one split
    INFERNT_CUDA_TRY(launch_pdl(bt_attn_merge, dim3(T * nkv), dim3(128), st, (const float*)part, positions, nq, nkv, D,
                                S, min_chunk, attn, attn_f32));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

// The batched step's attention with the Q|K|V finishing folded in (groups of
// up to 8 query heads): q and the new K / V rows from the projection's
// partials, RoPE, the bf16 cache append, then the output (merged in-kernel
// by the last split with tickets [T][nkv], else by a merge launch).
int bt_attention_fused_launch(const float* qkv_part, int qkv_splits, const float2* rope, uint16_t* kc, uint16_t* vc,
                              const int* positions, int T, int nq, int nkv, int D, int max_seq, int S, int min_chunk,
                              int stages, float* part, uint16_t* attn, unsigned* err, unsigned* tickets,
                              cudaStream_t st, const int* block_table, int page_size, int max_pages) {
    const int G = nq / nkv;
    INFERNT_REQUIRE(!block_table || (page_size >= 1 && (long long)page_size * max_pages >= max_seq),
                    "fused batched attention: pages of %d positions, %d per sequence, max_seq %d", page_size,
                    max_pages, max_seq);
    INFERNT_REQUIRE(G >= 1 && G <= 8 && nq % nkv == 0 && (D == 64 || D == 128),
                    "fused batched attention: group size %d, head_dim %d", G, D);
    INFERNT_REQUIRE(S >= 1 && min_chunk >= 1 && qkv_splits >= 1 && qkv_splits <= kMaxSplits,
                    "fused batched attention: splits %d, Q|K|V splits %d", S, qkv_splits);
    BtAttnArgs a = {};
    a.qkv_part = qkv_part;
    a.qkv_splits = qkv_splits;
    a.rope = rope;
    a.kc = kc;
    a.vc = vc;
    a.positions = positions;
    a.T = T;
    a.nq = nq;
    a.nkv = nkv;
    a.G = G;
    a.max_seq = max_seq;
    a.S = S;
    a.min_chunk = min_chunk;
    a.scale = 1.0f / sqrtf((float)D);
    a.part = part;
    a.attn = attn;
    a.err = err;
    a.tickets = tickets;
    a.block_table = block_table;
    a.page_size = page_size;
    a.max_pages = max_pages;
    if (int s = attn_mma_dispatch<true>(a, D, stages, st)) return s;
    INFERNT_CUDA_TRY(cudaGetLastError());
    return attn_merge(a, D, st);
}

int bt_fill_kv_launch(uint16_t* cache, int seq, int layer, int nkv, int max_seq, int D, int n_pos, uint64_t key,
                      float std_dev, int h0, int nkv_all, cudaStream_t st, const int* pages, int page_size) {
    if (n_pos <= 0) return INFERNT_OK;
    bt_fill_kv<<<256, 256, 0, st>>>(cache, seq, layer, nkv, max_seq, D, n_pos, key, std_dev, h0, nkv_all, pages,
                                    page_size);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int bt_page_copy_launch(uint16_t* pool, uint16_t* flat, const int* pages, int page_size, int nkv, int max_seq, int D,
                        int p0, int p1, bool to_pages, cudaStream_t st) {
    INFERNT_REQUIRE(pool && flat && pages && page_size >= 1 && D % 8 == 0 && 0 <= p0 && p0 <= p1 && p1 <= max_seq,
                    "page copy: rows [%d, %d) of %d, pages of %d", p0, p1, max_seq, page_size);
    if (p0 == p1) return INFERNT_OK;
    bt_page_copy<<<2 * sm_count(), 256, 0, st>>>(pool, flat, pages, page_size, nkv, max_seq, D, p0, p1,
                                                 to_pages ? 1 : 0);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int tp_sum_splits_launch(const float* part, int splits, int T, int N, float* y, cudaStream_t st) {
    INFERNT_REQUIRE(N % 4 == 0 && splits >= 1 && splits <= kMaxSplits, "tensor-parallel sum: N %d, splits %d", N,
                    splits);
    const size_t n4 = (size_t)T * N / 4;
    const int blocks = (int)((n4 + 255) / 256 < 1184 ? (n4 + 255) / 256 : 1184);
    INFERNT_CUDA_TRY(launch_pdl(tp_sum_splits, dim3(blocks), dim3(256), st, part, splits, T, N, y));
    return INFERNT_OK;
}

int bt_epoch_advance_launch(unsigned* epoch, cudaStream_t st) {
    INFERNT_CUDA_TRY(launch_pdl(bt_epoch_advance, dim3(1), dim3(1), st, epoch));
    return INFERNT_OK;
}

int tp_push_launch(const float* part, int splits, int T, int N, unsigned long long* const* peers, int rank, int world,
                   const unsigned* epoch, int per_step, int idx, cudaStream_t st) {
    INFERNT_REQUIRE(N % 4 == 0 && splits >= 1 && splits <= kMaxSplits && world >= 1,
                    "tensor-parallel push: N %d, splits %d", N, splits);
    const size_t n4 = (size_t)T * N / 4;
    const int blocks = (int)((n4 + 255) / 256 < 1184 ? (n4 + 255) / 256 : 1184);
    INFERNT_CUDA_TRY(launch_pdl(tp_push, dim3(blocks), dim3(256), st, part, splits, T, N, peers, rank, world, epoch,
                                per_step, idx));
    return INFERNT_OK;
}

int bt_resid_norm_tp_launch(const unsigned long long* own, int world, int T, int H, float* h, const float* norm_w,
                            float eps, uint16_t* xb, const unsigned* epoch, int per_step, int idx, unsigned* err,
                            long long budget, cudaStream_t st) {
    INFERNT_REQUIRE(H % 4 == 0 && H / 4 <= 1024, "tensor-parallel residual: H %d", H);
    INFERNT_CUDA_TRY(launch_pdl(bt_resid_norm_tp, dim3(T), dim3(H / 4), st, own, world, T, H, h, norm_w, eps, xb,
                                epoch, per_step, idx, err, budget));
    return INFERNT_OK;
}

int tp_argmax_local_launch(const float* logits, int T, int ld, int vl, int v0, int2* cand, const int* positions,
                           float inv_t, uint64_t seed, cudaStream_t st) {
    INFERNT_CUDA_TRY(
        launch_pdl(tp_argmax_local, dim3(T), dim3(256), st, logits, ld, vl, v0, cand, positions, inv_t, seed));
    return INFERNT_OK;
}

int tp_argmax_pick_launch(const int2* cand_all, int world, int T, int* tokens, int* positions, cudaStream_t st) {
    INFERNT_CUDA_TRY(launch_pdl(tp_argmax_pick, dim3((T + 127) / 128), dim3(128), st, cand_all, world, T, tokens,
                                positions));
    return INFERNT_OK;
}

int bt_argmax_launch(const float* logits, int T, int V, int* tokens, int* positions, int* hist, float* cand_v,
                     int* cand_i, unsigned* tickets, float inv_t, uint64_t seed, cudaStream_t st,
                     const uint64_t* salts) {
    INFERNT_REQUIRE(V % 4 == 0 && V / 4 >= kArgChunks, "batched argmax: vocabulary %d", V);
    INFERNT_CUDA_TRY(launch_pdl(bt_argmax, dim3(kArgChunks, T), dim3(256), st, logits, V, tokens, positions, hist,
                                cand_v, cand_i, tickets, inv_t, seed, salts));
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

}  // namespace infernt

extern "C" int infernt_batch_attention(const float* q, const void* k_cache, const void* v_cache, const int* positions,
                                       int T, int nq, int nkv, int head_dim, int max_seq, int splits, int min_chunk,
                                       int stages, float* partials, void* attn, float* attn_f32, void* stream) {
    INFERNT_REQUIRE(q && k_cache && v_cache && positions && partials && attn, "batch_attention: null pointer");
    INFERNT_REQUIRE(T >= 1 && nq >= 1 && nkv >= 1 && max_seq >= 1, "batch_attention: bad sizes");
    INFERNT_REQUIRE(infernt::aligned16(k_cache) && infernt::aligned16(v_cache) && infernt::aligned16(q),
                    "batch_attention: q and the caches must be 16-byte aligned");
    return infernt::bt_attention_launch(q, static_cast<const uint16_t*>(k_cache), static_cast<const uint16_t*>(v_cache),
                                        positions, T, nq, nkv, head_dim, max_seq, splits, min_chunk, stages, partials,
                                        static_cast<uint16_t*>(attn), static_cast<cudaStream_t>(stream), attn_f32);
}
