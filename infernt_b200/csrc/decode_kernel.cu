// decode_kernel.cu — the persistent decode kernel.
//
// One CTA per SM runs every phase of a decode step (and of a chain of
// steps): per layer the fused RMSNorm + Q/K/V projection, attention (RoPE,
// KV append, split-KV GQA, merge), O projection + residual, RMSNorm +
// gate/up + SiLU, down projection + residual; then RMSNorm + LM head +
// argmax.  Phases are separated by a grid barrier among the consumer warps.
//
// Warp 4 of every CTA is the producer: lanes 0-3 stream the CTA's share of
// every GEMV phase's weights, tile by tile, into a ring of 16 KB shared-
// memory slots with 2-D TMA box loads (8 KB FP32 / 8 KB bf16 per
// instruction).  Weights do not depend on activations, so the producer runs
// ahead across phase boundaries and layers while the consumers wait at grid
// barriers or compute attention: HBM keeps streaming through every
// synchronisation point, which a sequence of separate kernels cannot do.
//
// A GEMV phase of T tiles (tile = R rows x 512 columns; R = 8 FP32, 16 bf16)
// gives CTA b the tiles [T b / P, T (b + 1) / P).  A row group split
// between CTAs is merged by the last contributor (atomic ticket) in CTA
// order, so results do not depend on timing.  Reductions inside a CTA are
// fixed-order as in gemv.cuh.
//
// Every wait (ring slots, grid barrier) is bounded by a clock budget; on
// expiry the CTA sets kErrWaitTimeout in the error word, marks itself
// aborted and runs the remaining control flow without waiting, so the
// kernel always terminates and the host reports INFERNT_ERR_DEVICE.
#include <cstring>

#include "decode_kernel.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "tensormap.h"

namespace infernt {

namespace {

constexpr int kMegaSlot = 16384;
constexpr int kMegaConsumers = 128;
constexpr int kMegaThreads = 160;
constexpr long long kWaitCycles = 4000000000ll;  // about 2 s at the maximum SM clock

template <typename WT>
struct MegaRows {
    static constexpr int EB = WeightTraits<WT>::kBytes;
    static constexpr int R = kMegaSlot / (kPiece * EB);  // 8 FP32, 16 bf16
};

struct MegaShared {
    int abort;
    int flag;
    float ss[4];
    float amv[16];
    int ami[16];
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait on an mbarrier phase; returns false (and marks the CTA
// aborted) when the budget runs out or the CTA has already aborted.
__device__ __forceinline__ bool mega_wait(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(err, kErrWaitTimeout);
            *abort = 1;
            return false;
        }
    }
}

// Grid barrier of the consumer warps (named barrier 1 inside the CTA).
__device__ __forceinline__ void grid_sync(const MegaParams& p, volatile int* abort, int tid) {
    named_sync(1, kMegaConsumers);
    if (tid == 0 && !*abort) {
        const unsigned gen = ld_acquire(p.bar + 32);
        __threadfence();
        const unsigned arrived = atomicAdd(p.bar, 1u);
        if (arrived == gridDim.x - 1) {
            atomicExch(p.bar, 0u);
            __threadfence();
            atomicAdd(p.bar + 32, 1u);
        } else {
            const long long t0 = clock64();
            while (ld_acquire(p.bar + 32) == gen) {
                __nanosleep(32);
                if ((ld_acquire(p.err) & kErrWaitTimeout) || clock64() - t0 > kWaitCycles) {
                    atomicOr(p.err, kErrWaitTimeout);
                    *abort = 1;
                    break;
                }
            }
        }
        __threadfence();
    }
    named_sync(1, kMegaConsumers);
}

__device__ __forceinline__ void tile_range(long long tiles, long long& t0, long long& t1) {
    t0 = tiles * blockIdx.x / gridDim.x;
    t1 = tiles * (blockIdx.x + 1) / gridDim.x;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Timeline slot of (step, phase) for CTA 0 and the last CTA; -1 otherwise.
__device__ __forceinline__ long long trace_base(const MegaParams& p, int step, int ph) {
    if (!p.trace || (blockIdx.x != 0 && blockIdx.x != gridDim.x - 1)) return -1;
    const long long who = blockIdx.x == 0 ? 0 : 1;
    return ((who * p.steps + step) * p.nphases + ph) * kTraceFields;
}

__device__ __forceinline__ void trace_mark(const MegaParams& p, long long base, int field) {
    if (base >= 0) p.trace[base + field] = global_ns();
}

// CTA whose tile range contains tile t.
__device__ __forceinline__ int cta_of(long long t, long long tiles) {
    return (int)(((t + 1) * (long long)gridDim.x - 1) / tiles);
}

// Segment and local group of group g in the stacked row space.
__device__ __forceinline__ int seg_of(const MegaPhase& P, int g, int& lg, int& rowbase) {
    int q = 0;
    lg = g;
    rowbase = 0;
    while (q < P.nseg - 1 && lg >= P.seg_groups[q]) {
        lg -= P.seg_groups[q];
        rowbase += P.seg_rows[q];
        ++q;
    }
    return q;
}

// -------------------------------------------------------------- consumers

template <typename WT, int NS>
__device__ __forceinline__ void tile_fma(const unsigned char* slot, const float4& xv, int tid, float* acc) {
    constexpr int R = MegaRows<WT>::R;
    constexpr int EB = MegaRows<WT>::EB;
    constexpr int BR = R / NS;
    const int h = tid >> 6;
    const unsigned char* base = slot + (size_t)(h * BR) * kBoxCols * EB + (size_t)(tid & 63) * 4 * EB;
#pragma unroll
    for (int a = 0; a < R; ++a) {
        const int s2 = a / BR, i = a % BR;
        const unsigned char* wp = base + (size_t)(s2 * 2 * BR + i) * kBoxCols * EB;
        if (EB == 4) {
            const float4 w = *reinterpret_cast<const float4*>(wp);
            acc[a] = fmaf(w.x, xv.x, acc[a]);
            acc[a] = fmaf(w.y, xv.y, acc[a]);
            acc[a] = fmaf(w.z, xv.z, acc[a]);
            acc[a] = fmaf(w.w, xv.w, acc[a]);
        } else {
            const uint2 raw = *reinterpret_cast<const uint2*>(wp);
            const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
            const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
            acc[a] = fmaf(w01.x, xv.x, acc[a]);
            acc[a] = fmaf(w01.y, xv.y, acc[a]);
            acc[a] = fmaf(w23.x, xv.z, acc[a]);
            acc[a] = fmaf(w23.y, xv.w, acc[a]);
        }
    }
}

// Input vector of a GEMV phase into shared memory (RMSNorm applied when set).
__device__ void load_x(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const float* src = P.x;
    if (!src) {
        src = p.input;
        if (!src) {
            int t = (int)ld_acquire(reinterpret_cast<const unsigned*>(p.state));
            if (t < 0 || t >= p.vocab) {
                if (tid == 0) atomicOr(p.err, kErrToken);
                t = 0;
            }
            src = p.emb + (size_t)t * P.K;
        }
    }
    float rms = 1.0f;
    if (P.norm_w) {
        float ss = 0.0f;
        for (int i = tid * 4; i < P.K; i += kMegaConsumers * 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + i));
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) sh.ss[warp] = ss;
        named_sync(1, kMegaConsumers);
        const float tot = ((sh.ss[0] + sh.ss[1]) + sh.ss[2]) + sh.ss[3];
        rms = rsqrtf(tot / (float)P.K + P.eps);
    }
    for (int i = tid * 4; i < P.K; i += kMegaConsumers * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + i));
        float4 o = v;
        if (P.norm_w) {
            const float4 w = *reinterpret_cast<const float4*>(P.norm_w + i);
            o.x = v.x * rms * w.x;
            o.y = v.y * rms * w.y;
            o.z = v.z * rms * w.z;
            o.w = v.w * rms * w.w;
        }
        *reinterpret_cast<float4*>(xs + i) = o;
        if (P.x_copy && blockIdx.x == 0) *reinterpret_cast<float4*>(P.x_copy + i) = v;
    }
    named_sync(1, kMegaConsumers);
}

// Cross-warp reduction of a group's R partial sums, split-K merge when the
// group is shared with other CTAs, then the phase epilogue.
template <typename WT, int NS>
__device__ void finish_group(const MegaParams& p, const MegaPhase& P, long long g, long long t0, long long t1,
                             const float* acc, float* red, float* yv, MegaShared& sh, int tid, float& am_v,
                             int& am_i) {
    constexpr int R = MegaRows<WT>::R;
    constexpr int BR = R / NS;
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int a = 0; a < R; ++a) {
        const float v = warp_sum(acc[a]);
        if (lane == 0) red[warp * 16 + a] = v;
    }
    named_sync(1, kMegaConsumers);
    const long long cb = P.cb;
    const bool whole = (g * cb >= t0) && ((g + 1) * cb <= t1);
    float y = 0.0f;
    if (tid < R) y = ((red[0 * 16 + tid] + red[1 * 16 + tid]) + red[2 * 16 + tid]) + red[3 * 16 + tid];
    bool emit = whole;
    if (whole) {
        if (tid < R) yv[tid] = y;
    } else {
        const int which = (g == t0 / cb) ? 0 : 1;
        if (tid < R) p.part[((size_t)blockIdx.x * 2 + which) * 16 + tid] = y;
        named_sync(1, kMegaConsumers);
        const int b_first = cta_of(g * cb, P.tiles);
        const int b_last = cta_of(g * cb + cb - 1, P.tiles);
        if (tid == 0) {
            // contributors: the non-empty tile ranges between b_first and b_last
            int n = 0;
            for (int b = b_first; b <= b_last; ++b)
                n += (P.tiles * (b + 1) / gridDim.x > P.tiles * b / gridDim.x) ? 1 : 0;
            __threadfence();
            const unsigned ticket = atomicAdd(&p.gcnt[g], 1u);
            sh.flag = (ticket == (unsigned)(n - 1));
        }
        named_sync(1, kMegaConsumers);
        emit = sh.flag != 0;
        if (emit) {
            __threadfence();
            if (tid < R) {
                float s = 0.0f;
                for (int b = b_first; b <= b_last; ++b) {
                    const long long bs = P.tiles * b / gridDim.x;  // first tile of CTA b
                    if (P.tiles * (b + 1) / gridDim.x == bs) continue;  // empty range
                    const int wb = (g == bs / cb) ? 0 : 1;
                    s += __ldcg(p.part + ((size_t)b * 2 + wb) * 16 + tid);
                }
                yv[tid] = s;
            }
            if (tid == 0) p.gcnt[g] = 0u;
        }
    }
    named_sync(1, kMegaConsumers);
    if (!emit) return;
    if (NS == 2) {
        if (tid < BR) {
            const long long unit = g * BR + tid;
            if (unit < P.units) P.out[unit] = silu_mul(yv[tid], yv[BR + tid]);
        }
        return;
    }
    if (tid < R) {
        int lg, rowbase;
        const int q = seg_of(P, (int)g, lg, rowbase);
        const int local = lg * R + tid;
        if (local < P.seg_rows[q]) {
            const int row = rowbase + local;
            const float v = yv[tid];
            if (P.epi == kEpiStore) {
                P.out[row] = v;
            } else if (P.epi == kEpiResidual) {
                P.out[row] = __ldcg(P.res + row) + v;
            } else {
                float* lo = P.out ? P.out : p.logits;
                lo[row] = v;
                if (argmax_better(v, row, am_v, am_i)) {
                    am_v = v;
                    am_i = row;
                }
            }
        }
    }
}

// Winner of the CTA -> partial; the last CTA reduces all partials in CTA
// order, writes the token and advances the decode state.
__device__ void argmax_phase_end(const MegaParams& p, MegaShared& sh, int tid, float am_v, int am_i, int R) {
    if (tid < R) {
        sh.amv[tid] = am_v;
        sh.ami[tid] = am_i;
    }
    named_sync(1, kMegaConsumers);
    if (tid != 0) return;
    float bv = -1e30f;
    int bi = 0;
    for (int i = 0; i < R; ++i)
        if (argmax_better(sh.amv[i], sh.ami[i], bv, bi)) {
            bv = sh.amv[i];
            bi = sh.ami[i];
        }
    p.am_val[blockIdx.x] = bv;
    p.am_idx[blockIdx.x] = bi;
    __threadfence();
    if (atomicAdd(p.am_cnt, 1u) != gridDim.x - 1) return;
    __threadfence();
    float v = -1e30f;
    int id = 0;
    for (unsigned b = 0; b < gridDim.x; ++b) {
        const float pv = __ldcg(p.am_val + b);
        const int pi = __ldcg(p.am_idx + b);
        if (argmax_better(pv, pi, v, id)) {
            v = pv;
            id = pi;
        }
    }
    const int step = __ldcg(p.state + 2);
    if (p.hist) p.hist[step] = id;
    p.state[3] = id;
    p.state[0] = id;
    p.state[1] = __ldcg(p.state + 1) + 1;
    p.state[2] = step + 1;
    *p.am_cnt = 0u;
}

template <typename WT, int NS>
__device__ void gemv_phase(const MegaParams& p, const MegaPhase& P, unsigned char* ring, uint64_t* full,
                           uint64_t* empty, uint32_t& sl, float* xs, float* red, float* yv, MegaShared& sh,
                           int tid, long long tb) {
    constexpr int R = MegaRows<WT>::R;
    const int lane = tid & 31;
    const int slots = p.ring_slots;
    load_x(p, P, xs, sh, tid);
    if (tid == 0) trace_mark(p, tb, 1);
    long long t0, t1;
    tile_range(P.tiles, t0, t1);
    float acc[R];
#pragma unroll
    for (int a = 0; a < R; ++a) acc[a] = 0.0f;
    float am_v = -1e30f;
    int am_i = 0;
    long long g = t0 / P.cb;
    int j = (int)(t0 - g * P.cb);
    for (long long t = t0; t < t1; ++t, ++sl) {
        const int s = (int)(sl % slots);
        mega_wait(&full[s], (sl / slots) & 1u, &sh.abort, p.err);
        const float4 xv = reinterpret_cast<const float4*>(xs + j * kPiece)[tid];
        tile_fma<WT, NS>(ring + (size_t)s * kMegaSlot, xv, tid, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (j == P.cb - 1 || t == t1 - 1) {
            finish_group<WT, NS>(p, P, g, t0, t1, acc, red, yv, sh, tid, am_v, am_i);
#pragma unroll
            for (int a = 0; a < R; ++a) acc[a] = 0.0f;
        }
        if (++j == P.cb) {
            j = 0;
            ++g;
        }
    }
    if (P.epi == kEpiArgmax) argmax_phase_end(p, sh, tid, am_v, am_i, R);
}

__device__ void attention_phase(const MegaParams& p, const MegaPhase& P, float* xs, int tid) {
    const int pos = (int)ld_acquire(reinterpret_cast<const unsigned*>(p.state + 1));
    if (pos < 0 || pos >= p.attn.max_seq) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(p.err, kErrPosition);
        return;
    }
    AttnArgs a = p.attn;
    a.k_cache = p.kc[P.layer];
    a.v_cache = p.vc[P.layer];
    int chunk, active;
    attn_chunk(pos + 1, a.splits, chunk, active);
    const int items = a.nkv * a.splits;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int kvh = it / a.splits, split = it % a.splits;
        if (split < active) attention_item<kMegaConsumers>(a, kvh, split, pos, xs, tid);
    }
}

// ---------------------------------------------------------------- producer

template <typename WT>
__device__ void produce(const MegaParams& p, unsigned char* ring, uint64_t* full, uint64_t* empty,
                        volatile int* abort, int lane) {
    constexpr int R = MegaRows<WT>::R;
    constexpr int EB = MegaRows<WT>::EB;
    const int slots = p.ring_slots;
    const uint64_t pol = l2_evict_first_policy();
    uint32_t sl = 0;
    int ok = 1;
    for (int step = 0; step < p.steps && ok; ++step) {
        for (int ph = 0; ph < p.nphases && ok; ++ph) {
            const MegaPhase& P = p.phases[ph];
            if (P.kind != kPhGemv) continue;
            const int ns = P.ns;
            const int BR = R / ns;
            long long t0, t1;
            tile_range(P.tiles, t0, t1);
            long long g = t0 / P.cb;
            int j = (int)(t0 - g * P.cb);
            for (long long t = t0; t < t1 && ok; ++t, ++sl) {
                const int s = (int)(sl % slots);
                const uint32_t use = sl / slots;
                if (lane == 0) {
                    if (use > 0 && !mega_wait(&empty[s], (use - 1) & 1u, abort, p.err))
                        ok = 0;
                    else
                        mbar_arrive_expect_tx(&full[s], kMegaSlot);
                }
                ok = __shfl_sync(0xFu, ok, 0);
                if (ok) {
                    unsigned char* dst = ring + (size_t)s * kMegaSlot;
                    if (ns == 1) {
                        if (lane < 2) {
                            int lg, rowbase;
                            const int q = seg_of(P, (int)g, lg, rowbase);
                            tma_load_2d(dst + (size_t)lane * R * kBoxCols * EB, &p.maps[P.map[q]],
                                        j * kPiece + lane * kBoxCols, lg * R, &full[s], pol);
                        }
                    } else {
                        const int s2 = lane >> 1, h = lane & 1;
                        tma_load_2d(dst + (size_t)(s2 * 2 + h) * BR * kBoxCols * EB, &p.maps[P.map[s2]],
                                    j * kPiece + h * kBoxCols, (int)g * BR, &full[s], pol);
                    }
                }
                __syncwarp(0xFu);
                if (++j == P.cb) {
                    j = 0;
                    ++g;
                }
            }
            if (lane == 0) trace_mark(p, trace_base(p, step, ph), 4);
        }
    }
    if (!ok && lane == 0) {
        // slot sl - 1 was not armed; let the copies of every armed slot land
        // before the CTA can exit
        const uint32_t failed = sl - 1;
        const uint32_t first = failed > (uint32_t)slots ? failed - slots : 0u;
        volatile int no_abort = 0;
        for (uint32_t q = first; q < failed; ++q) mega_wait(&full[q % slots], (q / slots) & 1u, &no_abort, p.err);
    }
}

template <typename WT>
__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(const MegaParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ MegaShared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slots = p.ring_slots;
    unsigned char* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)slots * kMegaSlot);
    float* red = xs + p.x_floats;  // [4][16]
    float* yv = red + 64;          // [16]
    uint64_t* full = reinterpret_cast<uint64_t*>(yv + 16);
    uint64_t* empty = full + slots;
    if (tid == 0) {
        for (int s = 0; s < slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMegaConsumers / 32);
        }
        mbar_fence_init();
        sh.abort = 0;
        sh.flag = 0;
    }
    __syncthreads();

    if (warp == kMegaConsumers / 32) {
        if (lane < 4) produce<WT>(p, ring, full, empty, &sh.abort, lane);
        return;
    }

    uint32_t sl = 0;
    for (int step = 0; step < p.steps; ++step) {
        for (int ph = 0; ph < p.nphases; ++ph) {
            const MegaPhase& P = p.phases[ph];
            // every consumer thread takes the same branches here (no branch on the
            // abort flag, which the producer may set at any moment): the phases
            // contain named barriers
            const long long tb = tid == 0 ? trace_base(p, step, ph) : -1;
            trace_mark(p, tb, 0);
            if (P.kind == kPhAttn) {
                attention_phase(p, P, xs, tid);
            } else if (P.ns == 2) {
                gemv_phase<WT, 2>(p, P, ring, full, empty, sl, xs, red, yv, sh, tid, tb);
            } else {
                gemv_phase<WT, 1>(p, P, ring, full, empty, sl, xs, red, yv, sh, tid, tb);
            }
            trace_mark(p, tb, 2);
            grid_sync(p, &sh.abort, tid);
            trace_mark(p, tb, 3);
        }
    }
}

}  // namespace

int mega_smem_bytes(int ring_slots, int x_floats) {
    return ring_slots * kMegaSlot + x_floats * 4 + (64 + 16) * 4 + 2 * ring_slots * 8;
}

cudaError_t mega_prepare() {
    cudaError_t e = raise_dynamic_smem_limit(reinterpret_cast<const void*>(decode_mega_kernel<float>));
    if (e != cudaSuccess) return e;
    return raise_dynamic_smem_limit(reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16>));
}

int mega_occupancy(int weight_dtype, int smem_bytes) {
    int n = 0;
    const void* k = weight_dtype == INFERNT_DTYPE_BF16
                        ? reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16>)
                        : reinterpret_cast<const void*>(decode_mega_kernel<float>);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kMegaThreads, smem_bytes) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

cudaError_t launch_mega(const MegaParams& p, int weight_dtype, int ctas, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kMegaThreads);
    cfg.dynamicSmemBytes = mega_smem_bytes(p.ring_slots, p.x_floats);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (weight_dtype == INFERNT_DTYPE_BF16) return cudaLaunchKernelEx(&cfg, decode_mega_kernel<__nv_bfloat16>, p);
    return cudaLaunchKernelEx(&cfg, decode_mega_kernel<float>, p);
}

}  // namespace infernt
