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
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdint>

#include "attention.cuh"
#include "common.cuh"
#include "internal.h"
#include "warp_mma.cuh"

namespace infernt {

void* tensor_map_encoder();  // bgemm.cu

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

// ------------------------------------------------ tensor-core attention
// The same causal GQA attention for head_dim 64 or 128 on the 5th-generation
// tensor cores, S and O in tensor memory.  One CTA of 10 warps per (KV head,
// block of 128 / G tokens): its 128 query rows (token, head of the group)
// are the MMA's M.  Per 128-key tile i:
//   S_i[128 x 128] = Q K_i^T           tcgen05.mma (A = Q, B = K, both K-major)
//   P_i = bf16(exp2(S scale - m))      softmax warps: tcgen05.ld of S, P into
//                                      shared memory (128-byte swizzled K-major)
//   O[128 x 128] += P_i V_i            tcgen05.mma (A = P, B = V MN-major:
//                                      the cache's [key][d] rows as they are)
// Warp 0 (one thread) drives TMA: Q once through a 4-D map of q [C][Nkv][G][D]
// that yields the rows in (token, head) order, K and V tiles through 3-D maps
// of the caches bounded at the chunk's last position (rows past it read as
// zeros); two K/V stages.  Warp 1 (one thread) issues the MMAs: S_{i+1} into
// the other of two TMEM score buffers before P_i V_i, so the tensor pipe
// computes the next scores while the softmax warps work; the softmax computes
// P_i in registers while P_{i-1} V_{i-1} runs and stores it once that has
// completed.  Warps 2-9 run the softmax, two threads per query row
// (warps 2-5 keys and O columns 0-63, warps 6-9 64-127, each in its TMEM lane
// quarter; the two halves' row maxima and sums meet through shared memory
// and an mbarrier): base-2 online softmax whose reference maximum m moves
// only when a row's maximum exceeds it by more than 8 (probabilities stay
// below 2^8); then the row of O is rescaled in tensor memory (tcgen05.ld /
// st) after the previous P V has completed.  Tiles wholly below a warp's
// diagonal skip the causal mask.  The epilogue divides O by the row sums and
// writes bf16 rows.  Every wait is bounded; on expiry the CTA sets bit 0 of
// *err and returns once its copies have landed.
constexpr int kTcRows = 128;
constexpr int kTcKeys = 128;
constexpr uint32_t kTcBox = 16384;  // a [128][64] bf16 box
// Shared memory for head_dim D (D / 64 boxes per row block): Q, then two
// stages of K and V, then P (2 boxes: keys 0-63, 64-127).
template <int D>
struct TcLayout {
    static constexpr uint32_t kBoxes = D / 64;
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kStage0 = kBoxes * kTcBox;
    static constexpr uint32_t kStage = 2 * kBoxes * kTcBox;  // K boxes, then V boxes
    static constexpr uint32_t kP = kStage0 + 2 * kStage;
    static constexpr uint32_t kSmem = kP + 2 * kTcBox + 1024;
};
constexpr float kTcRescale = 8.0f;                     // log2 of the largest unnormalised probability
constexpr long long kTcWait = 2000000000ll;

struct PfTcArgs {
    uint16_t* attn;  // [C][nq D]
    unsigned* err;
    int C, p0, nq, nkv, G, tok_per_cta;
    float scale_log2;
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, bool& ok) {
    if (!ok) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kTcWait) {
            ok = false;
            return false;
        }
    return true;
}

// K-major operand, 128-byte swizzle: 128-byte rows, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3fffu) | (uint64_t)1u << 16 | (uint64_t)(1024u >> 4) << 32 |
           (uint64_t)1u << 46 | (uint64_t)2u << 61;
}

// MN-major operand, 128-byte swizzle: rows of 64 MN-contiguous elements (128
// bytes) per K index, atoms of 8 K rows 1024 bytes apart (stride byte
// offset), the next 64 MN elements `mn_block` bytes away (leading byte offset).
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t addr, uint32_t mn_block) {
    return (uint64_t)((addr >> 4) & 0x3fffu) | (uint64_t)((mn_block >> 4) & 0x3fffu) << 16 |
           (uint64_t)(1024u >> 4) << 32 | (uint64_t)1u << 46 | (uint64_t)2u << 61;
}

// D FP32, A and B bf16, M = 128, N = n; B MN-major when b_mn.
__device__ __forceinline__ uint32_t tc_idesc(bool b_mn, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// 2^x by the MUFU instruction (flush-to-zero; 2^-inf = 0)
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(dst),
        "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                       uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, "
        "%6}], [%2];" ::"r"(dst),
        "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

template <int D>
__global__ void __launch_bounds__(320, 1)
    pf_attn_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const PfTcArgs a) {
    using Lay = TcLayout<D>;
    constexpr uint32_t NB = Lay::kBoxes;
    constexpr uint32_t kTcQ = Lay::kQ, kTcStage0 = Lay::kStage0, kTcStage = Lay::kStage, kTcP = Lay::kP;
    constexpr int HALF = D / 2;  // O columns per softmax half
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    __shared__ uint64_t full_q, full_k[2], full_v[2], empty[2], bar_s[2], bar_p[2], bar_pv[2], bar_x[2], bar_l;
    __shared__ float red_max[2][2][kTcRows];  // [tile parity][half][row]
    __shared__ float red_l[2][kTcRows];
    __shared__ uint32_t tmem_base;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t base = (smem_addr(tc_smem_raw) + 1023u) & ~1023u;
    const int C = a.C, G = a.G;
    const int nblocks = (C + a.tok_per_cta - 1) / a.tok_per_cta;
    const int kvh = blockIdx.x % a.nkv;
    const int qb = nblocks - 1 - (int)(blockIdx.x / a.nkv);  // heaviest blocks first
    const int t0 = qb * a.tok_per_cta;
    const int t_end = min(C, t0 + a.tok_per_cta);
    const int kend = a.p0 + t_end;
    const int ntiles = (kend + kTcKeys - 1) / kTcKeys;

    if (tid == 0) {
        mbar_init(&full_q, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&full_k[s], 1);
            mbar_init(&full_v[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&bar_s[s], 1);
            mbar_init(&bar_p[s], 256);
            mbar_init(&bar_pv[s], 1);
            mbar_init(&bar_x[s], 256);
        }
        mbar_init(&bar_l, 256);
        mbar_fence_init();
        s_ok = 1;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // TMEM columns: S buffers at 0 and 128, O at 256
    const uint32_t tmem_o = tmem_base + 256;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(&full_q, NB * kTcBox);
            for (uint32_t b = 0; b < NB; ++b) tma_4d(base + kTcQ + b * kTcBox, &tm_q, 64 * b, 0, kvh, t0, &full_q);
            for (int i = 0; i < ntiles; ++i) {
                const int s = i & 1;
                if (i >= 2 && !tc_wait(&empty[s], ((i >> 1) - 1) & 1u, ok)) break;
                const uint32_t kb = base + kTcStage0 + (uint32_t)s * kTcStage, vb = kb + NB * kTcBox;
                mbar_arrive_expect_tx(&full_k[s], NB * kTcBox);
                for (uint32_t b = 0; b < NB; ++b) tma_3d(kb + b * kTcBox, &tm_k, 64 * b, i * kTcKeys, kvh, &full_k[s]);
                mbar_arrive_expect_tx(&full_v[s], NB * kTcBox);
                for (uint32_t b = 0; b < NB; ++b) tma_3d(vb + b * kTcBox, &tm_v, 64 * b, i * kTcKeys, kvh, &full_v[s]);
            }
            if (!ok) atomicExch(&s_ok, 0);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id_s = tc_idesc(false, kTcKeys), id_o = tc_idesc(true, D);
            // S_j = Q K_j^T into score buffer j % 2
            auto scores = [&](int j) {
                const int s = j & 1;
                const uint32_t kb = base + kTcStage0 + (uint32_t)s * kTcStage;
                if (!tc_wait(&full_k[s], (j >> 1) & 1u, ok)) return;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int b = 0; b < (int)NB; ++b)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma(tmem_base + 128u * (uint32_t)s, desc_k_sw128(base + kTcQ + b * kTcBox) + 2 * kk,
                               desc_k_sw128(kb + b * kTcBox) + 2 * kk, id_s, (b | kk) ? 1u : 0u);
                tc_commit(&bar_s[s]);
            };
            tc_wait(&full_q, 0u, ok);
            if (ok) scores(0);
            for (int i = 0; i < ntiles && ok; ++i) {
                const int s = i & 1;
                // the other score buffer was read by softmax i - 1 (bar_p waited last iteration)
                if (i + 1 < ntiles) scores(i + 1);
                if (!ok) break;
                if (!tc_wait(&bar_p[s], (i >> 1) & 1u, ok)) break;
                if (!tc_wait(&full_v[s], (i >> 1) & 1u, ok)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t vb = base + kTcStage0 + (uint32_t)s * kTcStage + NB * kTcBox;
                const uint32_t pb = base + kTcP;
#pragma unroll
                for (int b = 0; b < 2; ++b)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma(tmem_o, desc_k_sw128(pb + b * kTcBox) + 2 * kk,
                               desc_mn_sw128(vb + (uint32_t)(b * 4 + kk) * 2048u, kTcBox), id_o,
                               (i | b | kk) ? 1u : 0u);
                tc_commit(&bar_pv[s]);
                tc_commit(&empty[s]);
            }
            if (!ok) atomicExch(&s_ok, 0);
        }
    } else {
        // softmax: the thread of TMEM lane r and half h holds keys (and O
        // columns) [64 h, 64 h + 64) of query row r (token t0 + r / G, head r % G)
        const int half = (warp - 2) >> 2, quarter = warp & 3, r = 32 * quarter + lane;
        const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
        const int tl = r / G, g = r % G;
        const bool row_ok = t0 + tl < C;
        const int pos = a.p0 + min(t0 + tl, C - 1);
        const float sc = a.scale_log2;
        float m_ref = -INFINITY, l_half = 0.0f;  // m_ref in base-2 units (scores x sc)
        for (int i = 0; i < ntiles; ++i) {
            const int s = i & 1;
            tc_wait(&bar_s[s], (i >> 1) & 1u, ok);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float sv[64];
            const uint32_t sb = tmem_base + 128u * (uint32_t)s + lane_off + 64u * (uint32_t)half;
            tc_ld32(sb, *reinterpret_cast<float(*)[32]>(sv));
            tc_ld32(sb + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
            const int k0 = i * kTcKeys + 64 * half;
            float mx = -INFINITY;
            if (__all_sync(0xffffffffu, k0 + 63 <= pos)) {
#pragma unroll
                for (int j = 0; j < 64; ++j) mx = fmaxf(mx, sv[j]);
            } else {
#pragma unroll
                for (int j = 0; j < 64; ++j) {
                    sv[j] = k0 + j <= pos ? sv[j] : -INFINITY;
                    mx = fmaxf(mx, sv[j]);
                }
            }
            // the row maximum over both halves
            red_max[s][half][r] = mx;
            mbar_arrive(&bar_x[s]);
            tc_wait(&bar_x[s], (i >> 1) & 1u, ok);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            mx = fmaxf(red_max[s][0][r], red_max[s][1][r]) * sc;
            if (i == 0) {
                m_ref = mx;  // every row's first tile holds key 0 <= its position: finite
            } else {
                const bool grow = mx > m_ref + kTcRescale;
                if (__any_sync(0xffffffffu, grow)) {
                    // O must hold P_{i-1} V_{i-1} before it is rescaled
                    tc_wait(&bar_pv[(i - 1) & 1], ((i - 1) >> 1) & 1u, ok);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const float alpha = grow ? ex2_ftz(m_ref - mx) : 1.0f;
#pragma unroll
                    for (int c = 0; c < HALF / 32; ++c) {
                        float o[32];
                        const uint32_t oa = tmem_o + lane_off + (uint32_t)(HALF * half) + 32u * (uint32_t)c;
                        tc_ld32(oa, o);
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= alpha;
                        tc_st32(oa, o);
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    if (grow) {
                        l_half *= alpha;
                        m_ref = mx;
                    }
                }
            }
            // probabilities of the half row, packed as bf16 pairs
            float ls = 0.0f;
            uint32_t w[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float p0 = ex2_ftz(fmaf(sv[2 * j], sc, -m_ref)), p1 = ex2_ftz(fmaf(sv[2 * j + 1], sc, -m_ref));
                ls += p0 + p1;
                w[j] = cvt_bf16x2(p0, p1);
            }
            l_half += ls;
            if (i >= 1) {
                // P is read by P_{i-1} V_{i-1} until it completes
                tc_wait(&bar_pv[(i - 1) & 1], ((i - 1) >> 1) & 1u, ok);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
            }
            const uint32_t pb = base + kTcP + (uint32_t)half * kTcBox + (uint32_t)r * 128u;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t addr = pb + ((uint32_t)(c ^ (r & 7)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[4 * c]), "r"(w[4 * c + 1]),
                             "r"(w[4 * c + 2]), "r"(w[4 * c + 3])
                             : "memory");
            }
            fence_proxy_async_smem();
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            mbar_arrive(&bar_p[s]);
        }
        if (ok) {
            red_l[half][r] = l_half;
            mbar_arrive(&bar_l);
            tc_wait(&bar_l, 0u, ok);
            tc_wait(&bar_pv[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1u, ok);
            ok = __all_sync(0xffffffffu, ok);
        }
        if (ok) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const float inv = 1.0f / (red_l[0][r] + red_l[1][r]);
            uint16_t* out = a.attn + (size_t)(t0 + tl) * a.nq * D + (size_t)(kvh * G + g) * D + HALF * half;
#pragma unroll
            for (int c = 0; c < HALF / 32; ++c) {
                float o[32];
                tc_ld32(tmem_o + lane_off + (uint32_t)(HALF * half) + 32u * (uint32_t)c, o);
                if (row_ok) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 v;
                        v.x = cvt_bf16x2(o[8 * q + 0] * inv, o[8 * q + 1] * inv);
                        v.y = cvt_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv);
                        v.z = cvt_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv);
                        v.w = cvt_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv);
                        *reinterpret_cast<uint4*>(out + 32 * c + 8 * q) = v;
                    }
                }
            }
        }
        if (!ok) atomicExch(&s_ok, 0);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (!s_ok) {
        if (tid == 0 && a.err) atomicOr(a.err, 1u);
        const long long tw = clock64();
        while (clock64() - tw < 20000000ll) __nanosleep(1000);
    }
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512));
}

int encode_map(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
               const cuuint32_t* box) {
    auto fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    INFERNT_REQUIRE(fn, "prefill attention: cuTensorMapEncodeTiled is not available");
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    INFERNT_REQUIRE(r == CUDA_SUCCESS, "prefill attention: tensor map encoding failed (%d)", (int)r);
    return INFERNT_OK;
}

template <int D>
int launch_pf_attn_tc(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int C, int p0, int nq, int nkv,
                      int max_seq, uint16_t* attn, unsigned* err, cudaStream_t st) {
    const int G = nq / nkv;
    constexpr uint32_t kTcSmem = TcLayout<D>::kSmem;
    CUtensorMap mq, mk, mv;
    {
        const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)G, (cuuint64_t)nkv, (cuuint64_t)C};
        const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)G * D * 2, (cuuint64_t)nq * D * 2};
        const cuuint32_t box[4] = {64, (cuuint32_t)G, 1, (cuuint32_t)(kTcRows / G)};
        if (int s = encode_map(&mq, 4, q, dims, strides, box)) return s;
    }
    {
        const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)(p0 + C), (cuuint64_t)nkv};
        const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)max_seq * D * 2};
        const cuuint32_t box[3] = {64, (cuuint32_t)kTcKeys, 1};
        if (int s = encode_map(&mk, 3, kc, dims, strides, box)) return s;
        if (int s = encode_map(&mv, 3, vc, dims, strides, box)) return s;
    }
    // per launch (a driver attribute of the current device; prefill kernels run for milliseconds)
    INFERNT_CUDA_TRY(cudaFuncSetAttribute(pf_attn_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
    PfTcArgs a;
    a.attn = attn;
    a.err = err;
    a.C = C;
    a.p0 = p0;
    a.nq = nq;
    a.nkv = nkv;
    a.G = G;
    a.tok_per_cta = kTcRows / G;
    a.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    const long long ctas = (long long)nkv * ((C + a.tok_per_cta - 1) / a.tok_per_cta);
    INFERNT_REQUIRE(ctas < (1ll << 31), "prefill attention: %lld blocks", ctas);
    pf_attn_tc<D><<<(unsigned)ctas, 320, kTcSmem, st>>>(mq, mk, mv, a);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

template <int D, int G>
int launch_pf_attn(const PfAttnArgs& a, cudaStream_t st) {
    constexpr int smem = pf_smem_bytes<D>();
    INFERNT_CUDA_TRY(cudaFuncSetAttribute(pf_attn<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
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
                        int D, int max_seq, uint16_t* attn, unsigned* err, int tensor_cores, cudaStream_t st) {
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
    if (tensor_cores && (G == 1 || G == 2 || G == 4 || G == 8)) {
        if (D == 128) return launch_pf_attn_tc<128>(q, kc, vc, C, p0, nq, nkv, max_seq, attn, err, st);
        if (D == 64) return launch_pf_attn_tc<64>(q, kc, vc, C, p0, nq, nkv, max_seq, attn, err, st);
    }
    if (D == 64) return pf_attn_group<64>(a, G, st);
    if (D == 128) return pf_attn_group<128>(a, G, st);
    return fail(INFERNT_ERR_UNSUPPORTED, "prefill attention: head_dim %d (64 or 128)", D);
}

}  // namespace infernt

extern "C" int infernt_prefill_attention(const void* q, const void* k_cache, const void* v_cache, int n_tokens,
                                         int start_pos, int nq, int nkv, int head_dim, int max_seq, void* attn,
                                         unsigned* err, int tensor_cores, void* stream) {
    return infernt::pf_attention_launch(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k_cache),
                                        static_cast<const uint16_t*>(v_cache), n_tokens, start_pos, nq, nkv, head_dim,
                                        max_seq, static_cast<uint16_t*>(attn), err, tensor_cores,
                                        static_cast<cudaStream_t>(stream));
}
