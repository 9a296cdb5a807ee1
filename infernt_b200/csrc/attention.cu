// attention.cu — decode-step attention: RoPE + KV append + split-KV
// grouped-query flash-decoding, one kernel.
//
// Replaces the reference's launch_rope, launch_kv_cache_append,
// launch_attention_scores, launch_softmax and launch_attention_values
// sequence (llama_layer.cpp:25-48; cuda/rope.cu:5-35, cuda/kv_cache.cu:4-14,
// cuda/attention.cu:4-43, cuda/softmax.cu:5-49).
//
// Grid (num_kv_heads, splits): CTA (kvh, s) owns a contiguous chunk of key
// positions of one KV head and all Nq/Nkv query heads that share it (GQA),
// so each K/V row is read from HBM once for the whole group.  Within the
// chunk it walks tiles of 64 positions with an online softmax (running max
// m, running sum l, rescaled output o) and writes (m, l, o) per head.  The
// last CTA of a KV head to finish (atomic ticket; nothing spins) merges the
// partials in split order and writes the normalised output, so the merge is
// deterministic.  Only the CTA whose chunk ends at `position` appends the
// new K/V row, and it uses its registers' copy rather than re-reading the
// cache, so no CTA reads a row another CTA is writing.
//
// Scores keep the reference's order: dot product over d in increasing d,
// then the product with scale (attention.cu:18-22).
#include <cmath>
#include <cstring>

#include "attention.cuh"
#include "gemv.cuh"
#include "internal.h"

namespace infernt {

__host__ __device__ inline int attn_smem_floats(int G, int D) {
    // q [G][D] | K tile [T][D+1] | V tile [T][D] | p [G][T] | k_new [D] | v_new [D]
    return G * D + kAttnTile * (D + 1) + kAttnTile * D + G * kAttnTile + 2 * D;
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

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int D = a.D, G = a.nq / a.nkv, half = D / 2;
    pdl_launch_dependents();
    pdl_wait();

    const int pos = a.pos_ptr ? *a.pos_ptr : a.pos;
    if (pos < 0 || pos >= a.max_seq) {
        if (tid == 0 && kvh == 0 && split == 0 && a.err) atomicOr(a.err, kErrPosition);
        return;
    }
    const int seq = pos + 1;
    int chunk = (seq + a.splits - 1) / a.splits;
    if (chunk < kAttnMinChunk) chunk = kAttnMinChunk;
    const int active = (seq + chunk - 1) / chunk;
    if (split >= active) return;
    const int c0 = split * chunk;
    const int c1 = min(seq, c0 + chunk);
    const bool owns_new = (c1 == seq);

    float* qs = sm;                          // [G][D]
    float* ks = qs + G * D;                  // [T][D+1]
    float* vs = ks + kAttnTile * (D + 1);    // [T][D]
    float* ps = vs + kAttnTile * D;          // [G][T]
    float* knew = ps + G * kAttnTile;        // [D]
    float* vnew = knew + D;                  // [D]

    // q heads of this group, rotated at `pos`
    const float* qsrc = a.qkv + (size_t)kvh * G * D;
    for (int i = tid; i < G * half; i += kAttnThreads) {
        const int h = i / half, d = i % half;
        float x0 = qsrc[h * D + d], x1 = qsrc[h * D + d + half];
        rope_pair(x0, x1, d, D, pos, a.theta);
        qs[h * D + d] = x0;
        qs[h * D + d + half] = x1;
    }
    if (owns_new) {
        const float* ksrc = a.qkv + (size_t)a.nq * D + (size_t)kvh * D;
        const float* vsrc = a.qkv + (size_t)a.nq * D + (size_t)a.nkv * D + (size_t)kvh * D;
        float* kdst = a.k_cache + ((size_t)kvh * a.max_seq + pos) * D;
        float* vdst = a.v_cache + ((size_t)kvh * a.max_seq + pos) * D;
        for (int d = tid; d < half; d += kAttnThreads) {
            float x0 = ksrc[d], x1 = ksrc[d + half];
            rope_pair(x0, x1, d, D, pos, a.theta);
            knew[d] = x0;
            knew[d + half] = x1;
            kdst[d] = x0;
            kdst[d + half] = x1;
        }
        for (int d = tid; d < D; d += kAttnThreads) {
            const float v = vsrc[d];
            vnew[d] = v;
            vdst[d] = v;
        }
    }
    __syncthreads();

    // running state of up to two heads per warp (G <= 16), D/32 dims per lane
    constexpr int MAXH = kAttnMaxGroup / kAttnWarps;  // 2
    constexpr int MAXDL = kAttnMaxD / 32;             // 4
    float m_run[MAXH], l_run[MAXH], o_run[MAXH][MAXDL];
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < MAXDL; ++i) o_run[j][i] = 0.0f;
    }
    const int ndl = D / 32;

    const float* kbase = a.k_cache + (size_t)kvh * a.max_seq * D;
    const float* vbase = a.v_cache + (size_t)kvh * a.max_seq * D;
    for (int t0 = c0; t0 < c1; t0 += kAttnTile) {
        const int tl = min(kAttnTile, c1 - t0);
        // stage K and V rows of the tile (the row at `pos` comes from registers)
        for (int i = tid; i < tl * D; i += kAttnThreads) {
            const int p = i / D, d = i % D;
            const int gp = t0 + p;
            float kv, vv;
            if (gp == pos) {
                kv = knew[d];
                vv = vnew[d];
            } else {
                kv = kbase[(size_t)gp * D + d];
                vv = vbase[(size_t)gp * D + d];
            }
            ks[p * (D + 1) + d] = kv;
            vs[p * D + d] = vv;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < MAXH; ++j) {
            const int h = warp + j * kAttnWarps;
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
                    if (i < ndl) {
                        const int d = lane + 32 * i;
                        float acc = o_run[j][i] * alpha;
                        for (int p = 0; p < tl; ++p) acc = fmaf(ps[h * kAttnTile + p], vs[p * D + d], acc);
                        o_run[j][i] = acc;
                    }
                }
            }
        }
        __syncthreads();
    }

    // partial (m, l, o) of each head
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        const int h = warp + j * kAttnWarps;
        if (h < G) {
            float* pp = a.part + (((size_t)kvh * a.splits + split) * G + h) * (D + 2);
            if (lane == 0) {
                pp[0] = m_run[j];
                pp[1] = l_run[j];
            }
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (i < ndl) pp[2 + lane + 32 * i] = o_run[j][i];
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&a.counter[kvh], 1u);
        s_last = (ticket == (unsigned)active - 1u);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // merge the active splits of this KV head, in split order
    for (int h = warp; h < G; h += kAttnWarps) {
        float M = -INFINITY;
        for (int s = 0; s < active; ++s)
            M = fmaxf(M, __ldcg(a.part + (((size_t)kvh * a.splits + s) * G + h) * (D + 2)));
        float L = 0.0f;
        float acc[MAXDL];
#pragma unroll
        for (int i = 0; i < MAXDL; ++i) acc[i] = 0.0f;
        for (int s = 0; s < active; ++s) {
            const float* pp = a.part + (((size_t)kvh * a.splits + s) * G + h) * (D + 2);
            const float w = expf(__ldcg(pp) - M);
            L = fmaf(__ldcg(pp + 1), w, L);
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (i < ndl) acc[i] = fmaf(__ldcg(pp + 2 + lane + 32 * i), w, acc[i]);
        }
        const float inv = 1.0f / L;
        float* o = a.out + ((size_t)kvh * G + h) * D;
#pragma unroll
        for (int i = 0; i < MAXDL; ++i)
            if (i < ndl) o[lane + 32 * i] = acc[i] * inv;
    }
    if (tid == 0) a.counter[kvh] = 0u;
}

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t stream, bool pdl) {
    cudaError_t e = gemv_prepare();
    if (e != cudaSuccess) return e;
    const int G = a.nq / a.nkv;
    const int smem = attn_smem_floats(G, a.D) * 4;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(a.nkv, a.splits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, attention_decode_kernel, a);
}

cudaError_t attention_prepare() {
    return cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kMaxDynSmem);
}

int attention_shape_check(int nq, int nkv, int D, int splits) {
    INFERNT_REQUIRE(nq > 0 && nkv > 0 && nq % nkv == 0, "attention: Nq %d must be a positive multiple of Nkv %d", nq, nkv);
    INFERNT_REQUIRE(nq / nkv <= kAttnMaxGroup, "attention: group size %d > %d", nq / nkv, kAttnMaxGroup);
    INFERNT_REQUIRE(D >= 32 && D <= kAttnMaxD && D % 32 == 0, "attention: head_dim %d must be 32, 64, 96 or 128", D);
    INFERNT_REQUIRE(splits >= 1 && splits <= 4096, "attention: splits %d out of range", splits);
    return INFERNT_OK;
}

size_t attention_workspace_bytes(int nq, int nkv, int D, int splits) {
    const size_t part = (size_t)nkv * splits * (nq / nkv) * (D + 2) * sizeof(float);
    const size_t cnt = (size_t)nkv * sizeof(unsigned);
    return ((part + 255) / 256) * 256 + ((cnt + 255) / 256) * 256 + 256;
}

}  // namespace infernt

using namespace infernt;

extern "C" {

size_t infernt_attention_workspace_bytes(int num_q_heads, int num_kv_heads, int head_dim, int splits) {
    if (num_kv_heads <= 0 || splits <= 0) return 0;
    return attention_workspace_bytes(num_q_heads, num_kv_heads, head_dim, splits);
}

int infernt_attention_decode(float* out, const float* qkv, float* k_cache, float* v_cache,
                             int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
                             int position, float theta, int splits, void* workspace, void* stream) {
    if (int s = attention_shape_check(num_q_heads, num_kv_heads, head_dim, splits)) return s;
    INFERNT_REQUIRE(out && qkv && k_cache && v_cache && workspace, "attention_decode: null pointer");
    INFERNT_REQUIRE(position >= 0 && position < max_seq_len,
                    "attention_decode: position %d outside [0, %d)", position, max_seq_len);
    const size_t part = (size_t)num_kv_heads * splits * (num_q_heads / num_kv_heads) * (head_dim + 2) * 4;
    AttnArgs a;
    memset(&a, 0, sizeof(a));
    a.qkv = qkv;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.out = out;
    a.part = static_cast<float*>(workspace);
    const size_t part_al = ((part + 255) / 256) * 256;
    const size_t cnt_al = (((size_t)num_kv_heads * 4 + 255) / 256) * 256;
    a.counter = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + part_al);
    a.err = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + part_al + cnt_al);
    a.pos = position;
    a.nq = num_q_heads;
    a.nkv = num_kv_heads;
    a.D = head_dim;
    a.max_seq = max_seq_len;
    a.splits = splits;
    a.theta = theta;
    a.scale = 1.0f / sqrtf((float)head_dim);
    INFERNT_CUDA_TRY(launch_attention_decode(a, (cudaStream_t)stream, false));
    return INFERNT_OK;
}

}  // extern "C"
