// attention.cuh — decode-step attention as a device function: RoPE + KV
// append + one split of grouped-query flash-decoding + the last-split merge.
//
// Replaces the reference's launch_rope, launch_kv_cache_append,
// launch_attention_scores, launch_softmax and launch_attention_values
// sequence (llama_layer.cpp:25-48; cuda/rope.cu:5-35, cuda/kv_cache.cu:4-14,
// cuda/attention.cu:4-43, cuda/softmax.cu:5-49).
//
// Work item (kvh, split): a contiguous chunk of key positions of one KV
// head for all Nq/Nkv query heads that share it (GQA), so each K/V row is
// read from HBM once per group.  The chunk is walked in tiles of 64
// positions with an online softmax (running max m, running sum l,
// rescaled output o); (m, l, o) per head goes to the partial buffer.  The
// last item of a KV head to finish (atomic ticket, nothing spins) merges the
// partials in split order and writes the normalised output, so the merge
// is deterministic.  Only the item whose chunk ends at `position` appends
// the new K/V row; it uses its own copy for that row, so no item reads a
// row another item is writing.  Scores keep the reference's order: dot
// product over d in increasing d, then the product with scale
// (attention.cu:18-22).
//
// NT threads take part (a multiple of 32); they synchronise with named
// barrier 1, so the function runs inside a larger block whose other warps
// are busy elsewhere (the persistent decode kernel).
#pragma once

#include <math.h>

#include "common.cuh"

namespace infernt {

constexpr int kAttnTile = 64;
constexpr int kAttnMaxD = 128;
constexpr int kAttnMaxGroup = 16;
constexpr int kAttnMinChunk = 32;

struct AttnArgs {
    const float* qkv;  // [Nq*D | Nkv*D | Nkv*D], before RoPE
    float* k_cache;    // [Nkv, max_seq, D]
    float* v_cache;
    float* out;        // [Nq*D]
    float* part;       // [Nkv][splits][G][D + 2]
    unsigned* counter; // [Nkv], zero between uses
    const int* pos_ptr;  // device position, or NULL to use pos
    int pos;
    int nq, nkv, D, max_seq, splits;
    float theta, scale;
    unsigned* err;
    const float2* rope;  // optional (cos, sin) table [max_seq][D/2]; NULL: computed in place
};

// The (cos, sin) RoPE factors of pair d at `pos` (cuda/rope.cu:13-16).
__device__ __forceinline__ float2 rope_factors(int d, int D, int pos, float theta) {
    const float freq = 1.0f / powf(theta, (float)(2 * d) / (float)D);
    const float angle = (float)pos * freq;
    return make_float2(cosf(angle), sinf(angle));
}

// cuda/rope.cu:21-24 with precomputed factors.
__device__ __forceinline__ void rope_apply(float& a, float& b, float2 cs) {
    const float a0 = a, b0 = b;
    a = a0 * cs.x - b0 * cs.y;
    b = b0 * cs.x + a0 * cs.y;
}

__host__ __device__ inline int attn_smem_floats(int G, int D) {
    // q [G][D] | K tile [T][D+1] | V tile [T][D] | p [G][T] | k_new [D] | v_new [D] | flag
    return G * D + kAttnTile * (D + 1) + kAttnTile * D + G * kAttnTile + 2 * D + 4;
}

// Positions per K/V tile of the bulk-copy variant in the persistent kernel.
constexpr int kAttnBulkTile = 32;

__host__ __device__ inline int attn_bulk_smem_floats(int G, int D) {
    // q [G][D] | K tile [T][D] | V tile [T][D] | p [G][T] | RoPE row [D] | k_new [D] | v_new [D] | flag
    return G * D + 2 * kAttnBulkTile * D + G * kAttnBulkTile + 3 * D + 4;
}

__device__ __forceinline__ void rope_pair(float& a, float& b, int d, int D, int pos, float theta) {
    // cuda/rope.cu:13-16 and :21-24
    const float freq = 1.0f / powf(theta, (float)(2 * d) / (float)D);
    const float angle = (float)pos * freq;
    const float c = cosf(angle), s = sinf(angle);
    const float a0 = a, b0 = b;
    a = a0 * c - b0 * s;
    b = b0 * c + a0 * s;
}

// Chunk geometry of a split at sequence length seq.
__device__ __forceinline__ void attn_chunk(int seq, int splits, int& chunk, int& active) {
    chunk = (seq + splits - 1) / splits;
    if (chunk < kAttnMinChunk) chunk = kAttnMinChunk;
    active = (seq + chunk - 1) / chunk;
}

// One work item.  `pos` already validated (0 <= pos < max_seq); `split` <
// active.  `sm`: attn_smem_floats(G, D) floats of shared memory.
template <int NT>
__device__ void attention_item(const AttnArgs& a, int kvh, int split, int pos, float* sm, int tid) {
    constexpr int NW = NT / 32;
    constexpr int MAXH = (kAttnMaxGroup + NW - 1) / NW;
    constexpr int MAXDL = kAttnMaxD / 32;
    const int warp = tid >> 5, lane = tid & 31;
    const int D = a.D, G = a.nq / a.nkv, half = D / 2;
    const int seq = pos + 1;
    int chunk, active;
    attn_chunk(seq, a.splits, chunk, active);
    const int c0 = split * chunk;
    const int c1 = min(seq, c0 + chunk);
    const bool owns_new = (c1 == seq);

    float* qs = sm;                        // [G][D]
    float* ks = qs + G * D;                // [T][D+1]
    float* vs = ks + kAttnTile * (D + 1);  // [T][D]
    float* ps = vs + kAttnTile * D;        // [G][T]
    float* knew = ps + G * kAttnTile;      // [D]
    float* vnew = knew + D;                // [D]
    int* s_last = reinterpret_cast<int*>(vnew + D);

    // q heads of this group, rotated at `pos`
    const float* qsrc = a.qkv + (size_t)kvh * G * D;
    for (int i = tid; i < G * half; i += NT) {
        const int h = i / half, d = i % half;
        float x0 = __ldcg(qsrc + h * D + d), x1 = __ldcg(qsrc + h * D + d + half);
        rope_apply(x0, x1, a.rope ? __ldg(a.rope + (size_t)pos * half + d) : rope_factors(d, D, pos, a.theta));
        qs[h * D + d] = x0;
        qs[h * D + d + half] = x1;
    }
    if (owns_new) {
        const float* ksrc = a.qkv + (size_t)a.nq * D + (size_t)kvh * D;
        const float* vsrc = a.qkv + (size_t)a.nq * D + (size_t)a.nkv * D + (size_t)kvh * D;
        float* kdst = a.k_cache + ((size_t)kvh * a.max_seq + pos) * D;
        float* vdst = a.v_cache + ((size_t)kvh * a.max_seq + pos) * D;
        for (int d = tid; d < half; d += NT) {
            float x0 = __ldcg(ksrc + d), x1 = __ldcg(ksrc + d + half);
            rope_apply(x0, x1, a.rope ? __ldg(a.rope + (size_t)pos * half + d) : rope_factors(d, D, pos, a.theta));
            knew[d] = x0;
            knew[d + half] = x1;
            kdst[d] = x0;
            kdst[d + half] = x1;
        }
        for (int d = tid; d < D; d += NT) {
            const float v = __ldcg(vsrc + d);
            vnew[d] = v;
            vdst[d] = v;
        }
    }
    named_sync(1, NT);

    float m_run[MAXH], l_run[MAXH], o_run[MAXH][MAXDL];
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < MAXDL; ++i) o_run[j][i] = 0.0f;
    }

    const float* kbase = a.k_cache + (size_t)kvh * a.max_seq * D;
    const float* vbase = a.v_cache + (size_t)kvh * a.max_seq * D;
    for (int t0 = c0; t0 < c1; t0 += kAttnTile) {
        const int tl = min(kAttnTile, c1 - t0);
        // stage K and V rows of the tile (the row at `pos` comes from this item's copy)
        if ((D & 3) == 0) {
            const int n4 = tl * D / 4;
#pragma unroll 4
            for (int i = tid; i < n4; i += NT) {
                const int p = (4 * i) / D, d = (4 * i) % D;
                const int gp = t0 + p;
                float4 kv, vv;
                if (gp == pos) {
                    kv = make_float4(knew[d], knew[d + 1], knew[d + 2], knew[d + 3]);
                    vv = make_float4(vnew[d], vnew[d + 1], vnew[d + 2], vnew[d + 3]);
                } else {
                    kv = __ldcg(reinterpret_cast<const float4*>(kbase + (size_t)gp * D + d));
                    vv = __ldcg(reinterpret_cast<const float4*>(vbase + (size_t)gp * D + d));
                }
                float* kd = ks + p * (D + 1) + d;
                kd[0] = kv.x;
                kd[1] = kv.y;
                kd[2] = kv.z;
                kd[3] = kv.w;
                *reinterpret_cast<float4*>(vs + p * D + d) = vv;
            }
        } else {
            for (int i = tid; i < tl * D; i += NT) {
                const int p = i / D, d = i % D;
                const int gp = t0 + p;
                const float kv = gp == pos ? knew[d] : __ldcg(kbase + (size_t)gp * D + d);
                const float vv = gp == pos ? vnew[d] : __ldcg(vbase + (size_t)gp * D + d);
                ks[p * (D + 1) + d] = kv;
                vs[p * D + d] = vv;
            }
        }
        named_sync(1, NT);
#pragma unroll
        for (int j = 0; j < MAXH; ++j) {
            const int h = warp + j * NW;
            if (h < G) {
                float sc[kAttnTile / 32];
                float tmax = -INFINITY;
#pragma unroll
                for (int r = 0; r < kAttnTile / 32; ++r) {
                    const int p = lane + r * 32;
                    float s = -INFINITY;
                    if (p < tl) {
                        float dot = 0.0f;
                        const float* qh = qs + h * D;
                        const float* kr = ks + p * (D + 1);
                        for (int d = 0; d < D; ++d) dot = fmaf(qh[d], kr[d], dot);
                        s = dot * a.scale;
                    }
                    sc[r] = s;
                    tmax = fmaxf(tmax, s);
                }
                tmax = warp_max(tmax);
                const float m_new = fmaxf(m_run[j], tmax);
                const float alpha = expf(m_run[j] - m_new);
                float psum = 0.0f;
#pragma unroll
                for (int r = 0; r < kAttnTile / 32; ++r) {
                    const int p = lane + r * 32;
                    const float pe = (p < tl) ? expf(sc[r] - m_new) : 0.0f;
                    ps[h * kAttnTile + p] = pe;
                    psum += pe;
                }
                psum = warp_sum(psum);
                l_run[j] = l_run[j] * alpha + psum;
                m_run[j] = m_new;
                __syncwarp();
#pragma unroll
                for (int i = 0; i < MAXDL; ++i) {
                    const int d = lane + 32 * i;
                    if (d < D) {
                        float acc = o_run[j][i] * alpha;
                        for (int p = 0; p < tl; ++p) acc = fmaf(ps[h * kAttnTile + p], vs[p * D + d], acc);
                        o_run[j][i] = acc;
                    }
                }
            }
        }
        named_sync(1, NT);
    }

    // partial (m, l, o) of each head
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        const int h = warp + j * NW;
        if (h < G) {
            float* pp = a.part + (((size_t)kvh * a.splits + split) * G + h) * (D + 2);
            if (lane == 0) {
                pp[0] = m_run[j];
                pp[1] = l_run[j];
            }
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (lane + 32 * i < D) pp[2 + lane + 32 * i] = o_run[j][i];
        }
    }
    named_sync(1, NT);
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&a.counter[kvh], 1u);
        *s_last = (ticket == (unsigned)active - 1u);
    }
    named_sync(1, NT);
    if (*s_last) {
        __threadfence();
        // merge the active splits of this KV head: one warp per head, the
        // lanes load 32 splits' (m, l) at once (one round trip per 32 splits,
        // not one per split); every output element sums w_s o_s in split
        // order, the loads of eight splits in flight
        for (int h = warp; h < G; h += NW) {
            const float* ph = a.part + ((size_t)kvh * a.splits * G + h) * (D + 2);
            const size_t sstride = (size_t)G * (D + 2);
            float M = -INFINITY;
            for (int s0 = 0; s0 < active; s0 += 32)
                if (s0 + lane < active) M = fmaxf(M, __ldcg(ph + (size_t)(s0 + lane) * sstride));
            M = warp_max(M);
            float L = 0.0f;
            float acc[MAXDL];
#pragma unroll
            for (int i = 0; i < MAXDL; ++i) acc[i] = 0.0f;
            for (int s0 = 0; s0 < active; s0 += 32) {
                const int sl = s0 + lane;
                float w = 0.0f;
                if (sl < active) {
                    w = expf(__ldcg(ph + (size_t)sl * sstride) - M);
                    L = fmaf(__ldcg(ph + (size_t)sl * sstride + 1), w, L);
                }
                const int n = min(32, active - s0);
                for (int k0 = 0; k0 < n; k0 += 8) {
                    float ov[8][MAXDL];
#pragma unroll
                    for (int k = 0; k < 8; ++k)
#pragma unroll
                        for (int i = 0; i < MAXDL; ++i)
                            ov[k][i] = (k0 + k < n && lane + 32 * i < D)
                                           ? __ldcg(ph + (size_t)(s0 + k0 + k) * sstride + 2 + lane + 32 * i)
                                           : 0.0f;
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float wk = __shfl_sync(0xffffffffu, w, (k0 + k) & 31);
                        if (k0 + k < n)
#pragma unroll
                            for (int i = 0; i < MAXDL; ++i) acc[i] = fmaf(ov[k][i], wk, acc[i]);
                    }
                }
            }
            L = warp_sum(L);
            const float inv = 1.0f / L;
            float* o = a.out + ((size_t)kvh * G + h) * D;
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (lane + 32 * i < D) o[lane + 32 * i] = acc[i] * inv;
        }
        if (tid == 0) a.counter[kvh] = 0u;
    }
    named_sync(1, NT);
}

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t stream, bool pdl);
int attention_shape_check(int nq, int nkv, int D, int splits);
size_t attention_workspace_bytes(int nq, int nkv, int D, int splits);

}  // namespace infernt
