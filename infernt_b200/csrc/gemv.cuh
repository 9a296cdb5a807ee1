// gemv.cuh — batch-1 projection kernels of the decode step.
//
// A decode-step projection is y = W x with W row-major [out, in] (the
// reference multiplies the HF layout with cublasSgemm and trans_b = true,
// gemm/cublas_wrapper.cu:21-40, llama_layer.cpp:18-69).  At batch 1 this
// is pure weight streaming: every weight byte is read once and used for
// one FMA, so the kernel is bound by HBM bandwidth and its job is to keep
// enough bytes in flight on every SM.
//
// Fast path (in % 512 == 0, 16-byte aligned rows): one CTA per SM, four
// producer threads (one per producer warp, taking turns slot by slot: a
// slot takes one bulk copy per row, so one thread issuing them all would
// cap the stream below the HBM rate) stream the CTA's contiguous block of
// rows into a ring of shared-memory slots with 1-D bulk copies
// (cp.async.bulk, the TMA engine) and mbarrier transaction counts; four
// consumer warps multiply the slots against the input vector held in
// shared memory (slot layout below).  The producer starts before griddepcontrol.wait, so under programmatic
// dependent launch a kernel's weights stream in while the previous kernel
// is still finishing.
//
// Every reduction has a fixed order (lane-strided partials, xor-shuffle
// tree, then warps 0..3 in order), so results are bit-reproducible run to
// run.
//
// Fused prologue: RMSNorm of the input vector (cuda/rmsnorm.cu:4-27,
// o = x * rsqrt(sum(x^2)/h + eps) * w), or the embedding row of a token
// read from device memory (cuda/embedding.cu:3-8).
// Fused epilogues: store; residual add (cuda/residual.cu:4-10);
// SiLU(gate) * up over paired rows (cuda/activation.cu:4-11); logits +
// argmax (cuda/sampling.cu:3-36) with the last CTA reducing the per-CTA
// winners.
#pragma once

#include "common.cuh"

namespace infernt {

// kEpiExchange (persistent kernel, tensor parallelism): the rows go to every
// rank's exchange buffer, to be summed by the next phase.
enum EpiKind : int { kEpiStore = 0, kEpiResidual = 1, kEpiSwiGLU = 2, kEpiArgmax = 3, kEpiExchange = 4 };

constexpr int kPiece = 512;          // weight elements per piece (one float4/bf16x4 per thread)
constexpr int kGemvConsumers = 128;  // four consumer warps
constexpr int kGemvProducers = 4;    // producer warps (lane 0 of each issues every fourth slot)
constexpr int kGemvThreads = kGemvConsumers + 32 * kGemvProducers;
constexpr int kSlotBytes = 16384;    // ring slot: one 512-column block of 8 FP32 / 16 bf16 rows
constexpr int kGemvStages = 8;       // ring depth of the standalone kernels (128 KB in flight per SM)
constexpr int kGemvStagesDeep = 12;  // when the input vector leaves room (192 KB in flight per SM)
constexpr int kArgmaxMaxBlocks = 1024;
constexpr int kPlainThreads = 256;
constexpr int kMaxDynSmem = 226 * 1024;  // dynamic shared memory the launchers plan with (opt-in 227 KB
                                         // minus room for the kernels' static shared memory)

struct GemvArgs {
    const void* seg_ptr[3];  // matrices stacked in one virtual row space (Q|K|V)
    int seg_rows[3];
    int nseg;
    int units;  // output rows; SwiGLU: (gate, up) pairs with seg 0 = gate, seg 1 = up
    int K;      // input features
    const float* x;      // input vector [K]; NULL selects the embedding row below
    const float* emb;    // embedding table [vocab, K]
    const int* token;    // device token id for the embedding row
    int vocab;
    const float* norm_w;  // RMSNorm weight [K] or NULL (no norm)
    float eps;
    float* x_copy;        // block 0 stores the raw input row here when non-NULL
    float* out;
    const float* res;     // residual input (out = res + y), may alias out
    // argmax epilogue
    float* am_val;        // [gridDim.x] per-CTA winners
    int* am_idx;
    unsigned* am_counter;  // zero before the launch; the last CTA resets it
    int* am_out;           // final token
    int* state;            // optional decode state {token, position, step}: advanced by the last CTA
    int* token_hist;       // optional history, written at state[2]
    unsigned* err;
};

// Resolve the input row (explicit vector or the embedding row of *token).
__device__ __forceinline__ const float* gemv_input(const GemvArgs& a) {
    if (a.x) return a.x;
    int t = *a.token;
    if (t < 0 || t >= a.vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && a.err) atomicOr(a.err, kErrToken);
        t = 0;
    }
    return a.emb + (size_t)t * (size_t)a.K;
}

// Shared epilogue for one output unit.
template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int u, float y0, float y1,
                                              float& am_v, int& am_i) {
    if (EPI == kEpiStore) {
        a.out[u] = y0;
    } else if (EPI == kEpiResidual) {
        a.out[u] = a.res[u] + y0;
    } else if (EPI == kEpiSwiGLU) {
        a.out[u] = silu_mul(y0, y1);
    } else {  // kEpiArgmax
        a.out[u] = y0;
        if (argmax_better(y0, u, am_v, am_i)) {
            am_v = y0;
            am_i = u;
        }
    }
}

// Final step of the argmax epilogue: block winner -> partial; the last
// block to finish reduces all partials in block order.  `bv/bi` must be the
// block's winner, called by one thread.
__device__ __forceinline__ void argmax_finish(const GemvArgs& a, float bv, int bi) {
    a.am_val[blockIdx.x] = bv;
    a.am_idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned ticket = atomicAdd(a.am_counter, 1u);
    if (ticket != gridDim.x - 1) return;
    __threadfence();
    float v = -1e30f;
    int i = 0;
    for (unsigned b = 0; b < gridDim.x; ++b) {
        const float pv = __ldcg(a.am_val + b);
        const int pi = __ldcg(a.am_idx + b);
        if (argmax_better(pv, pi, v, i)) {
            v = pv;
            i = pi;
        }
    }
    if (a.am_out) *a.am_out = i;
    if (a.state) {
        const int step = a.state[2];
        if (a.token_hist) a.token_hist[step] = i;
        a.state[0] = i;
        a.state[1] = a.state[1] + 1;
        a.state[2] = step + 1;
    }
    *a.am_counter = 0u;
}

// ---------------------------------------------------------------------------
// Fast path: TMA ring
//
// Work of one CTA: the contiguous units [ub, ue) (rows, or gate/up row
// pairs), taken in groups of G = R / NS units.  A ring slot holds one
// 512-column block j of every row of the group: piece i = s * G + g is row
// g of segment s (gate/up) at columns [512 j, 512 j + 512).  So a consumer
// thread loads one float4 of x per slot and R independent weight vectors,
// accumulating into R registers; a group's rows are reduced across the
// four warps once, after its last column block.  The producer issues one
// bulk copy per piece (2 KB FP32 / 1 KB bf16); slot bytes are R pieces.
// ---------------------------------------------------------------------------

template <typename WT>
struct TmaShape {
    static constexpr int EB = WeightTraits<WT>::kBytes;
    static constexpr int PB = kPiece * EB;                 // piece bytes
    static constexpr int R = kSlotBytes / PB;              // pieces (rows) per slot: 8 FP32, 16 bf16
};

// Global address of unit-row `row` of segment space `s` (SwiGLU: 0 gate, 1
// up; otherwise the stacked virtual row space).
template <typename WT>
__device__ __forceinline__ const unsigned char* tma_row(const GemvArgs& a, int ns, int s, int row) {
    const size_t rb = (size_t)a.K * WeightTraits<WT>::kBytes;
    if (ns == 2) return static_cast<const unsigned char*>(a.seg_ptr[s]) + (size_t)row * rb;
    int base = 0;
    for (int q = 0; q < a.nseg; ++q) {
        if (row < base + a.seg_rows[q])
            return static_cast<const unsigned char*>(a.seg_ptr[q]) + (size_t)(row - base) * rb;
        base += a.seg_rows[q];
    }
    return static_cast<const unsigned char*>(a.seg_ptr[0]);
}

__host__ __device__ inline int gemv_tma_smem_bytes(int K, int stages) {
    // ring | x [K] | reduction [2][4][16] | 2*stages mbarriers
    return stages * kSlotBytes + K * 4 + 2 * 4 * 16 * 4 + 2 * stages * 8;
}

__device__ __forceinline__ void dot_slot_piece(const float* wp, const float4& x, int t, float& acc) {
    const float4 w = reinterpret_cast<const float4*>(wp)[t];
    acc = fmaf(w.x, x.x, acc);
    acc = fmaf(w.y, x.y, acc);
    acc = fmaf(w.z, x.z, acc);
    acc = fmaf(w.w, x.w, acc);
}

__device__ __forceinline__ void dot_slot_piece(const __nv_bfloat16* wp, const float4& x, int t, float& acc) {
    const uint2 raw = reinterpret_cast<const uint2*>(wp)[t];
    const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    acc = fmaf(w01.x, x.x, acc);
    acc = fmaf(w01.y, x.y, acc);
    acc = fmaf(w23.x, x.z, acc);
    acc = fmaf(w23.y, x.w, acc);
}

template <typename WT, int EPI, int STAGES>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_tma_kernel(const GemvArgs a) {
    using S = TmaShape<WT>;
    constexpr int PB = S::PB;
    constexpr int R = S::R;
    constexpr int NS = (EPI == kEpiSwiGLU) ? 2 : 1;
    constexpr int G = R / NS;

    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + STAGES * kSlotBytes);
    float* red = xs + a.K;  // [2][4][16]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * 4 * 16);
    uint64_t* empty = full + STAGES;
    __shared__ float s_ss[4];
    __shared__ float s_amv[G];
    __shared__ int s_ami[G];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGemvConsumers / 32);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    const int ub = (int)((long long)a.units * blockIdx.x / gridDim.x);
    const int ue = (int)((long long)a.units * (blockIdx.x + 1) / gridDim.x);
    const int PPR = a.K / kPiece;

    if (warp >= kGemvConsumers / 32) {
        // ---------------- producers: weights do not depend on the previous
        // kernel.  Producer k arms the slots sl = k (mod kGemvProducers);
        // STAGES is a multiple of kGemvProducers, so every lap of a ring slot
        // belongs to one producer.
        static_assert(STAGES % kGemvProducers == 0, "producers divide the ring");
        const uint32_t k = (uint32_t)(warp - kGemvConsumers / 32);
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            uint32_t sl = 0;
            bool ok = true;
            for (int u0 = ub; u0 < ue && ok; u0 += G) {
                const int ng = min(G, ue - u0);
                for (int j = 0; j < PPR && ok; ++j, ++sl) {
                    if (sl % kGemvProducers != k) continue;
                    const int s = (int)(sl % STAGES);
                    const uint32_t use = sl / STAGES;
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1u, a.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], (uint32_t)(ng * NS * PB));
                    unsigned char* dst = ring + s * kSlotBytes;
#pragma unroll
                    for (int q = 0; q < NS; ++q)
                        for (int g = 0; g < ng; ++g)
                            bulk_g2s(dst + (q * G + g) * PB,
                                     tma_row<WT>(a, NS, q, u0 + g) + (size_t)j * PB, PB, &full[s], pol);
                }
            }
            if (!ok) {  // let every slot this producer armed land before the CTA can exit
                const uint32_t first = sl > (uint32_t)STAGES ? sl - STAGES : 0u;
                for (uint32_t q = first; q < sl; ++q)
                    if (q % kGemvProducers == k) mbar_wait(&full[q % STAGES], (q / STAGES) & 1u, a.err);
            }
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();
    const float* xsrc = gemv_input(a);
    float rms = 1.0f;
    if (a.norm_w) {
        float ss = 0.0f;
        for (int i = tid * 4; i < a.K; i += kGemvConsumers * 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(xsrc + i));
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) s_ss[warp] = ss;
        named_sync(1, kGemvConsumers);
        const float tot = ((s_ss[0] + s_ss[1]) + s_ss[2]) + s_ss[3];
        rms = rsqrtf(tot / (float)a.K + a.eps);
    }
    for (int i = tid * 4; i < a.K; i += kGemvConsumers * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(xsrc + i));
        float4 o = v;
        if (a.norm_w) {
            const float4 w = *reinterpret_cast<const float4*>(a.norm_w + i);
            o.x = v.x * rms * w.x;
            o.y = v.y * rms * w.y;
            o.z = v.z * rms * w.z;
            o.w = v.w * rms * w.w;
        }
        *reinterpret_cast<float4*>(xs + i) = o;
        if (a.x_copy && blockIdx.x == 0) *reinterpret_cast<float4*>(a.x_copy + i) = v;
    }
    named_sync(1, kGemvConsumers);

    uint32_t sl = 0;
    bool failed = false;
    int buf = 0;
    float am_v = -1e30f;
    int am_i = 0;
    for (int u0 = ub; u0 < ue; u0 += G) {
        const int ng = min(G, ue - u0);
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = 0.0f;
        for (int j = 0; j < PPR; ++j, ++sl) {
            const int s = (int)(sl % STAGES);
            if (!failed) failed = !mbar_wait(&full[s], (sl / STAGES) & 1u, a.err);
            const float4 xv = reinterpret_cast<const float4*>(xs + j * kPiece)[tid];
            const unsigned char* slot = ring + s * kSlotBytes;
#pragma unroll
            for (int i = 0; i < R; ++i)
                dot_slot_piece(reinterpret_cast<const WT*>(slot + i * PB), xv, tid, acc[i]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        float* rb = red + buf * 64;  // [4 warps][16]
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const float v = warp_sum(acc[i]);
            if (lane == 0) rb[warp * 16 + i] = v;
        }
        named_sync(1, kGemvConsumers);
        if (tid < ng) {
            float y[2] = {0.0f, 0.0f};
#pragma unroll
            for (int q = 0; q < NS; ++q) {
                const int i = q * G + tid;
                y[q] = ((rb[0 * 16 + i] + rb[1 * 16 + i]) + rb[2 * 16 + i]) + rb[3 * 16 + i];
            }
            gemv_epilogue<EPI>(a, u0 + tid, y[0], y[1], am_v, am_i);
        }
        buf ^= 1;
    }

    if (EPI == kEpiArgmax) {
        if (tid < G) {
            s_amv[tid] = am_v;
            s_ami[tid] = am_i;
        }
        named_sync(1, kGemvConsumers);
        if (tid == 0) {
            float bv = -1e30f;
            int bi = 0;
            for (int g = 0; g < G; ++g)
                if (argmax_better(s_amv[g], s_ami[g], bv, bi)) {
                    bv = s_amv[g];
                    bi = s_ami[g];
                }
            argmax_finish(a, bv, bi);
        }
    }
}


// ---------------------------------------------------------------------------
// Plain path: any K, scalar loads, one warp per output unit
// ---------------------------------------------------------------------------

template <typename WT>
__device__ __forceinline__ const WT* gemv_row_ptr(const GemvArgs& a, int seg_space, int row) {
    if (seg_space >= 0)  // SwiGLU: gate (0) or up (1)
        return static_cast<const WT*>(a.seg_ptr[seg_space]) + (size_t)row * a.K;
    int base = 0;
    for (int s = 0; s < a.nseg; ++s) {
        if (row < base + a.seg_rows[s])
            return static_cast<const WT*>(a.seg_ptr[s]) + (size_t)(row - base) * a.K;
        base += a.seg_rows[s];
    }
    return nullptr;
}

template <typename WT, int EPI>
__global__ void __launch_bounds__(kPlainThreads) gemv_plain_kernel(const GemvArgs a) {
    extern __shared__ float xs_plain[];
    __shared__ float s_red[kPlainThreads / 32];
    __shared__ float s_amv[kPlainThreads / 32];
    __shared__ int s_ami[kPlainThreads / 32];
    constexpr int NW = kPlainThreads / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_launch_dependents();
    pdl_wait();

    const float* xsrc = gemv_input(a);
    float rms = 1.0f;
    if (a.norm_w) {
        float ss = 0.0f;
        for (int i = tid; i < a.K; i += kPlainThreads) ss = fmaf(xsrc[i], xsrc[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = 0; w < NW; ++w) tot += s_red[w];
        rms = rsqrtf(tot / (float)a.K + a.eps);
    }
    for (int i = tid; i < a.K; i += kPlainThreads) {
        const float v = xsrc[i];
        xs_plain[i] = a.norm_w ? v * rms * a.norm_w[i] : v;
        if (a.x_copy && blockIdx.x == 0) a.x_copy[i] = v;
    }
    __syncthreads();

    float am_v = -1e30f;
    int am_i = 0;
    for (int u = blockIdx.x * NW + warp; u < a.units; u += gridDim.x * NW) {
        float y[2] = {0.0f, 0.0f};
        constexpr int NS = (EPI == kEpiSwiGLU) ? 2 : 1;
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            const WT* w = gemv_row_ptr<WT>(a, NS == 2 ? s : -1, u);
            float acc = 0.0f;
            for (int k = lane; k < a.K; k += 32) acc = fmaf(to_f32(w[k]), xs_plain[k], acc);
            y[s] = warp_sum(acc);
        }
        if (lane == 0) gemv_epilogue<EPI>(a, u, y[0], y[1], am_v, am_i);
    }
    if (EPI == kEpiArgmax) {
        if (lane == 0) {
            s_amv[warp] = am_v;
            s_ami[warp] = am_i;
        }
        __syncthreads();
        if (tid == 0) {
            float bv = -1e30f;
            int bi = 0;
            for (int w = 0; w < NW; ++w)
                if (argmax_better(s_amv[w], s_ami[w], bv, bi)) {
                    bv = s_amv[w];
                    bi = s_ami[w];
                }
            argmax_finish(a, bv, bi);
        }
    }
}

// Raises the dynamic shared-memory limit of every decode kernel on the
// current device (once per device; call outside stream capture).
cudaError_t gemv_prepare();
cudaError_t attention_prepare();
// Sets a kernel's dynamic shared-memory limit to the device's opt-in
// maximum minus the kernel's static shared memory.
cudaError_t raise_dynamic_smem_limit(const void* kernel);

// Host launcher (gemv.cu).  `weight_dtype` INFERNT_DTYPE_*, `epi` EpiKind.
// `pdl` enables programmatic dependent launch on the stream.
cudaError_t launch_gemv(const GemvArgs& a, int weight_dtype, int epi, cudaStream_t stream,
                        bool pdl, int* grid_out);
// Whether the TMA path applies to these arguments.
bool gemv_fast_path_ok(const GemvArgs& a, int weight_dtype, int epi);
// Grid the launcher would use (argmax workspace sizing).
int gemv_grid(const GemvArgs& a, int weight_dtype, int epi);

}  // namespace infernt
