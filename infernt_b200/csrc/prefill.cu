// prefill.cu — the non-projection kernels of prompt prefill: a chunk of C
// consecutive prompt tokens of one sequence at positions [p0, p0 + C)
// through a layer at once.  The reference feeds a prompt as sequential
// single-token forwards (src/engine.cpp:124-126); the arithmetic per token is
// the same decode step (architectures/llama/llama_layer.cpp:11-72), with the
// projections as dense tensor-core contractions (pgemm_kernel, bgemm.cu):
//
//   Y = xb W_qkv^T                                   pgemm
//   q = bf16(RoPE(Y_q)); K/V rows appended (bf16)     pf_qkv_rope
//   attn = bf16(causal GQA attention)                pf_attn
//   Y = attn W_o^T; h += Y; xb = bf16(RMSNorm(h))     pgemm, bt_resid_norm
//   Y = xb [W_gate; W_up]^T; act = bf16(silu(g) u)    pgemm, bt_swiglu
//   Y = act W_down^T; h += Y; xb = ...                pgemm, bt_resid_norm
//
// The cache rows written here are the rows a decode step would append
// (cuda/rope.cu:13-34, cuda/kv_cache.cu:4-14: RoPE in FP32 from the table,
// then rounded to bf16).  Queries enter the attention's tensor cores as bf16
// and the probabilities as bf16 (FP32 scores, softmax statistics and
// accumulators).
#include <cmath>
#include <cstdint>

#include "attention.cuh"
#include "common.cuh"
#include "internal.h"
#include "warp_mma.cuh"

namespace infernt {

namespace {

// Q|K|V of prompt token t (position p0 + t) from the projection rows y[t]
// [(nq + 2 nkv) D] FP32: q rows RoPE'd and rounded into q [C][nq D] bf16; K
// (RoPE'd) and V rows rounded and written at the position in the
// sequence's caches [nkv][max_seq][D].  Four RoPE pairs (d .. d + 3, d + D/2
// .. d + D/2 + 3) per unit.
__global__ void pf_qkv_rope(const float* y, int p0, int nq, int nkv, int D, const float2* rope, int max_seq,
                            uint16_t* q, uint16_t* kc, uint16_t* vc) {
    const int t = blockIdx.x, pos = p0 + t, half = D / 2;
    const int N = (nq + 2 * nkv) * D;
    const float* row = y + (size_t)t * N;
    const float2* rp = rope + (size_t)pos * half;
    const int qk_units = (nq + nkv) * (half / 4);
    for (int u = threadIdx.x; u < qk_units; u += blockDim.x) {
        const int hd = u / (half / 4), d = (u % (half / 4)) * 4;
        const float4 a4 = *reinterpret_cast<const float4*>(row + (size_t)hd * D + d);
        const float4 b4 = *reinterpret_cast<const float4*>(row + (size_t)hd * D + d + half);
        float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) rope_apply(a[e], b[e], rp[d + e]);
        uint16_t* dst = hd < nq ? q + (size_t)t * nq * D + (size_t)hd * D
                                : kc + ((size_t)(hd - nq) * max_seq + pos) * D;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            dst[d + e] = bf16_bits(a[e]);
            dst[d + half + e] = bf16_bits(b[e]);
        }
    }
    for (int u = threadIdx.x; u < nkv * D / 4; u += blockDim.x) {
        const int i = 4 * u, kh = i / D, d = i % D;
        const float4 v = *reinterpret_cast<const float4*>(row + (size_t)(nq + nkv) * D + i);
        const uint32_t lo = (uint32_t)bf16_bits(v.x) | ((uint32_t)bf16_bits(v.y) << 16);
        const uint32_t hi = (uint32_t)bf16_bits(v.z) | ((uint32_t)bf16_bits(v.w) << 16);
        *reinterpret_cast<uint2*>(vc + ((size_t)kh * max_seq + pos) * D + d) = make_uint2(lo, hi);
    }
}

// Causal GQA attention of a prompt chunk (cuda/attention.cu:9-42 and
// cuda/softmax.cu:13-48 per query row, with online softmax): query token t
// of head h attends to cache positions [0, p0 + t] of KV head h / G.
//
// One CTA of 8 warps per (KV head, block of BQ = 16 x 8 / G tokens); warp w
// takes query head (w mod G) of the group and 16 consecutive tokens, so the
// CTA's 128 query rows share every K/V tile it loads.  Tiles of 64 keys
// stream through a ring of kPfStages stages (16-byte cp.async copies by all
// threads, chunk c of row r stored at c ^ (r & 7) for conflict-free
// ldmatrix; rows past the chunk's last position are zero-filled).  Per warp
// and tile, on mma.sync m16n8k16 (bf16 x bf16 -> FP32):
//   S[16 x 64] = Q[16 x D] K^T,  O[16 x D] += bf16(P)[16 x 64] V
// with the softmax in base 2 (scores scaled by log2(e) / sqrt(D)); a warp
// skips tiles that start after its last token's position.  Blocks are
// launched heaviest (latest tokens) first.
constexpr int kPfKeys = 64;
constexpr int kPfWarps = 8;
constexpr int kPfStages = 3;

template <int D>
constexpr int pf_smem_bytes() {
    return kPfStages * 2 * kPfKeys * D * 2;
}

struct PfAttnArgs {
    const uint16_t* q;   // [C][nq D] bf16, RoPE applied
    const uint16_t* kc;  // [nkv][max_seq][D] bf16, positions [0, p0 + C) written
    const uint16_t* vc;
    uint16_t* attn;      // [C][nq D] bf16
    int C, p0, nq, nkv, max_seq;
    float scale_log2;    // log2(e) / sqrt(D)
};

template <int D, int G>
__global__ void __launch_bounds__(256, D == 64 ? 2 : 1) pf_attn(const PfAttnArgs a) {
    constexpr int ROWB = D * 2, CH = ROWB / 16, TILEB = kPfKeys * ROWB;
    constexpr int KC = D / 16, DB = D / 8, NT = kPfKeys / 8;
    constexpr int BQ = 16 * (kPfWarps / G);
    extern __shared__ __align__(128) unsigned char pf_smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int C = a.C, nblocks = (C + BQ - 1) / BQ;
    const int kvh = blockIdx.x % a.nkv;
    const int qb = nblocks - 1 - (int)(blockIdx.x / a.nkv);
    const int hq = kvh * G + warp % G;
    const int ts = qb * BQ + (warp / G) * 16;  // first token of the warp
    const int t_end = min(C, (qb + 1) * BQ);  // tokens of the CTA: [qb BQ, t_end)
    const int kend = a.p0 + t_end;            // keys of the CTA: [0, kend)
    const int ntiles = (kend + kPfKeys - 1) / kPfKeys;
    const bool has_rows = ts < C;
    const int wpos_last = a.p0 + min(ts + 15, C - 1);
    const unsigned char* kb = reinterpret_cast<const unsigned char*>(a.kc + (size_t)kvh * a.max_seq * D);
    const unsigned char* vb = reinterpret_cast<const unsigned char*>(a.vc + (size_t)kvh * a.max_seq * D);
    const uint32_t ring = smem_addr(pf_smem);

    auto issue = [&](int i) {
        if (i < ntiles) {
            const int k0 = i * kPfKeys;
            const uint32_t st = ring + (uint32_t)(i % kPfStages) * 2 * TILEB;
#pragma unroll
            for (int e = 0; e < kPfKeys * CH / 256; ++e) {
                const int idx = e * 256 + tid, row = idx / CH, ch = idx % CH;
                const bool ok = k0 + row < kend;
                const size_t off = (size_t)(ok ? k0 + row : 0) * ROWB + (size_t)ch * 16;
                const uint32_t dst = st + (uint32_t)(row * ROWB + ((ch ^ (row & 7)) << 4));
                cp_async16(dst, kb + off, ok ? 16u : 0u);
                cp_async16(dst + TILEB, vb + off, ok ? 16u : 0u);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int i = 0; i < kPfStages - 1; ++i) issue(i);

    // query fragments of rows g (token ts + g) and g + 8 (token ts + g + 8)
    const int r0 = ts + g, r1 = ts + g + 8;
    uint32_t qa[KC][4];
    {
        const uint16_t* q0 = a.q + (size_t)r0 * a.nq * D + (size_t)hq * D + 2 * tig;
        const uint16_t* q1 = a.q + (size_t)r1 * a.nq * D + (size_t)hq * D + 2 * tig;
#pragma unroll
        for (int k = 0; k < KC; ++k) {
            qa[k][0] = r0 < C ? *reinterpret_cast<const uint32_t*>(q0 + 16 * k) : 0u;
            qa[k][1] = r1 < C ? *reinterpret_cast<const uint32_t*>(q1 + 16 * k) : 0u;
            qa[k][2] = r0 < C ? *reinterpret_cast<const uint32_t*>(q0 + 16 * k + 8) : 0u;
            qa[k][3] = r1 < C ? *reinterpret_cast<const uint32_t*>(q1 + 16 * k + 8) : 0u;
        }
    }
    // positions of the two rows (rows past the chunk take its last position:
    // never written, but free of NaN)
    const int pr0 = a.p0 + min(r0, C - 1), pr1 = a.p0 + min(r1, C - 1);
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    float acc[DB][4];
#pragma unroll
    for (int b = 0; b < DB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.0f;

    for (int i = 0; i < ntiles; ++i) {
        cp_async_wait<kPfStages - 2>();  // this thread's copies of tile i have landed
        __syncthreads();                 // everyone's have, and tile i - 1's stage is no longer read
        issue(i + kPfStages - 1);
        const int k0 = i * kPfKeys;
        if (!has_rows || k0 > wpos_last) continue;  // warp-uniform
        const uint32_t kt = ring + (uint32_t)(i % kPfStages) * 2 * TILEB, vt = kt + TILEB;
        float sc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
        for (int k = 0; k < KC; ++k)
#pragma unroll
            for (int jj = 0; jj < NT / 2; ++jj) {
                const int m = lane >> 3, row = 8 * (2 * jj + (m >> 1)) + (lane & 7), ch = 2 * k + (m & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kt + (uint32_t)(row * ROWB + ((ch ^ (row & 7)) << 4)), b0, b1, b2, b3);
                mma_bf16_16816(sc[2 * jj], qa[k], b0, b1);
                mma_bf16_16816(sc[2 * jj + 1], qa[k], b2, b3);
            }
        // causal mask and online softmax (base 2) of rows g and g + 8
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = k0 + 8 * j + 2 * tig + e;
                sc[j][e] = key <= pr0 ? sc[j][e] * a.scale_log2 : -INFINITY;
                sc[j][e + 2] = key <= pr1 ? sc[j][e + 2] * a.scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, sc[j][e]);
                mx1 = fmaxf(mx1, sc[j][e + 2]);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // every row's first tile holds key 0 <= its position, so the running
        // maxima are finite from the first tile on
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const float al0 = exp2f(m0 - n0), al1 = exp2f(m1 - n1);
        m0 = n0;
        m1 = n1;
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            sc[j][0] = exp2f(sc[j][0] - n0);
            sc[j][1] = exp2f(sc[j][1] - n0);
            sc[j][2] = exp2f(sc[j][2] - n1);
            sc[j][3] = exp2f(sc[j][3] - n1);
            s0 += sc[j][0] + sc[j][1];
            s1 += sc[j][2] + sc[j][3];
        }
        l0 = l0 * al0 + s0;
        l1 = l1 * al1 + s1;
#pragma unroll
        for (int b = 0; b < DB; ++b) {
            acc[b][0] *= al0;
            acc[b][1] *= al0;
            acc[b][2] *= al1;
            acc[b][3] *= al1;
        }
        // O += P V, 16 keys per k-step: the score fragments of two n-tiles
        // are the A fragment of the probabilities
#pragma unroll
        for (int kk = 0; kk < NT / 2; ++kk) {
            uint32_t pa[4];
            pa[0] = cvt_bf16x2(sc[2 * kk][0], sc[2 * kk][1]);
            pa[1] = cvt_bf16x2(sc[2 * kk][2], sc[2 * kk][3]);
            pa[2] = cvt_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
            pa[3] = cvt_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
            for (int b2 = 0; b2 < DB / 2; ++b2) {
                const int m = lane >> 3, row = 16 * kk + 8 * (m & 1) + (lane & 7), ch = 2 * b2 + (m >> 1);
                uint32_t v0, v1, v2, v3;
                ldsm_x4_trans(vt + (uint32_t)(row * ROWB + ((ch ^ (row & 7)) << 4)), v0, v1, v2, v3);
                mma_bf16_16816(acc[2 * b2], pa, v0, v1);
                mma_bf16_16816(acc[2 * b2 + 1], pa, v2, v3);
            }
        }
    }
    cp_async_wait<0>();
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (!has_rows) return;
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    uint16_t* o0 = a.attn + (size_t)r0 * a.nq * D + (size_t)hq * D + 2 * tig;
    uint16_t* o1 = a.attn + (size_t)r1 * a.nq * D + (size_t)hq * D + 2 * tig;
#pragma unroll
    for (int b = 0; b < DB; ++b) {
        if (r0 < C) *reinterpret_cast<uint32_t*>(o0 + 8 * b) = cvt_bf16x2(acc[b][0] * i0, acc[b][1] * i0);
        if (r1 < C) *reinterpret_cast<uint32_t*>(o1 + 8 * b) = cvt_bf16x2(acc[b][2] * i1, acc[b][3] * i1);
    }
}

template <int D, int G>
int launch_pf_attn(const PfAttnArgs& a, cudaStream_t st) {
    constexpr int smem = pf_smem_bytes<D>();
    static bool raised = false;
    if (!raised) {
        INFERNT_CUDA_TRY(cudaFuncSetAttribute(pf_attn<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        raised = true;
    }
    constexpr int BQ = 16 * (kPfWarps / G);
    const long long ctas = (long long)a.nkv * ((a.C + BQ - 1) / BQ);
    INFERNT_REQUIRE(ctas < (1ll << 31), "prefill attention: %lld blocks", ctas);
    pf_attn<D, G><<<(unsigned)ctas, 256, smem, st>>>(a);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

template <int D>
int pf_attn_group(const PfAttnArgs& a, int G, cudaStream_t st) {
    switch (G) {
        case 1: return launch_pf_attn<D, 1>(a, st);
        case 2: return launch_pf_attn<D, 2>(a, st);
        case 4: return launch_pf_attn<D, 4>(a, st);
        case 8: return launch_pf_attn<D, 8>(a, st);
        default: return fail(INFERNT_ERR_UNSUPPORTED, "prefill attention: group size %d (1, 2, 4 or 8)", G);
    }
}

}  // namespace

int pf_qkv_rope_launch(const float* y, int C, int p0, int nq, int nkv, int D, const float2* rope, int max_seq,
                       uint16_t* q, uint16_t* kc, uint16_t* vc, cudaStream_t st) {
    INFERNT_REQUIRE(D % 8 == 0 && C >= 1 && p0 >= 0 && (long long)p0 + C <= max_seq,
                    "prefill: head_dim %d, tokens %d at %d, max_seq %d", D, C, p0, max_seq);
    pf_qkv_rope<<<C, 128, 0, st>>>(y, p0, nq, nkv, D, rope, max_seq, q, kc, vc);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

int pf_attention_launch(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int C, int p0, int nq, int nkv,
                        int D, int max_seq, uint16_t* attn, cudaStream_t st) {
    INFERNT_REQUIRE(q && kc && vc && attn, "prefill attention: null pointer");
    INFERNT_REQUIRE(C >= 1 && p0 >= 0 && (long long)p0 + C <= max_seq, "prefill attention: %d tokens at %d, max_seq %d",
                    C, p0, max_seq);
    INFERNT_REQUIRE(nq >= 1 && nkv >= 1 && nq % nkv == 0, "prefill attention: %d query heads, %d KV heads", nq, nkv);
    INFERNT_REQUIRE(aligned16(q) && aligned16(kc) && aligned16(vc) && aligned16(attn),
                    "prefill attention: q, caches and attn must be 16-byte aligned");
    PfAttnArgs a;
    a.q = q;
    a.kc = kc;
    a.vc = vc;
    a.attn = attn;
    a.C = C;
    a.p0 = p0;
    a.nq = nq;
    a.nkv = nkv;
    a.max_seq = max_seq;
    a.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    const int G = nq / nkv;
    if (D == 64) return pf_attn_group<64>(a, G, st);
    if (D == 128) return pf_attn_group<128>(a, G, st);
    return fail(INFERNT_ERR_UNSUPPORTED, "prefill attention: head_dim %d (64 or 128)", D);
}

}  // namespace infernt

extern "C" int infernt_prefill_attention(const void* q, const void* k_cache, const void* v_cache, int n_tokens,
                                         int start_pos, int nq, int nkv, int head_dim, int max_seq, void* attn,
                                         void* stream) {
    return infernt::pf_attention_launch(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k_cache),
                                        static_cast<const uint16_t*>(v_cache), n_tokens, start_pos, nq, nkv, head_dim,
                                        max_seq, static_cast<uint16_t*>(attn), static_cast<cudaStream_t>(stream));
}
