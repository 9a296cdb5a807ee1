// decode_kernel.cu — the persistent decode kernel.
//
// One CTA per SM runs every phase of a decode step (and of a chain of
// steps): per layer the fused RMSNorm + Q/K/V projection, attention (RoPE,
// KV append, split-KV GQA, merge), O projection + residual, RMSNorm +
// gate/up + SiLU, down projection + residual; then RMSNorm + LM head +
// argmax.  Phases are separated by a grid barrier among the consumer warps.
//
// Warps 0-3 consume; lane 0 of warp 4 produces: it streams the CTA's share
// of every GEMV phase's weights into a ring of 16 KB shared-memory slots with
// 1-D bulk copies (cp.async.bulk).  A GEMV phase gives CTA b the output units
// [U b / P, U (b + 1) / P), whose weight rows are contiguous in row-major
// memory, so every slot is one contiguous 16 KB run of HBM (two runs where
// it straddles a matrix or gate/up boundary): the access pattern that
// streams fastest, and a split balanced to one row per CTA.  Weights do not
// depend on activations, so the producer runs ahead across phase boundaries
// and layers while the consumers wait at grid barriers or compute attention.
//
// Consumers walk the stream in 512-element pieces, each thread covering 4
// columns of every piece, in batches of R rows (R = 8 FP32 / 16 bf16; for
// gate/up R / 2 units, gate rows then up rows), which fill exactly K / 512
// slots.  Each thread adds a row's pieces in column order into one
// accumulator per row; for the usual widths the (row, column block) of every
// piece of a batch is known at compile time and the input columns stay in
// registers.  Row sums are reduced over the warp by a reduce-scatter (per
// slot in that case, else once per batch), and the four warps' row sums are
// added in warp order in the batches' epilogue.
// Every output is reduced inside one CTA in a fixed order, so results do
// not depend on timing and no cross-CTA merge sits on the critical path.
//
// Every wait (ring slots, grid barrier, bulk copies) is bounded by a clock
// budget; on expiry the CTA sets kErrWaitTimeout in the error word, marks
// itself aborted and runs the remaining control flow without waiting, so the
// kernel always terminates and the host reports INFERNT_ERR_DEVICE.
#include <cstring>

#include "decode_kernel.cuh"
#include "gemv.cuh"
#include "internal.h"

namespace infernt {

namespace {

constexpr int kMegaSlot = 16384;
constexpr int kMegaConsumers = 128;
constexpr int kProducerWarp = 4;
constexpr int kMegaThreads = 160;  // 4 consumer warps and the producer warp
constexpr long long kWaitCycles = 4000000000ll;  // about 2 s at the maximum SM clock
constexpr int kResRows = 128;                    // residual rows a CTA stages per phase
constexpr int kMergeChunk = 8;                   // attention splits merged per round of loads
constexpr int kMergeRounds = 8;                  // lanes x rounds bound the splits of a KV head (256)

template <typename WT>
struct MegaRows {
    static constexpr int EB = WeightTraits<WT>::kBytes;
    static constexpr int R = kMegaSlot / (kPiece * EB);  // rows per batch: 8 FP32, 16 bf16
    static constexpr int PB = kPiece * EB;               // bytes per 512-element piece
    static constexpr int PT = kMegaSlot / PB;            // pieces per slot (= R)
};

constexpr int kGroupBatch = 16;  // batches whose row sums are held before their epilogue runs
constexpr int kMaxRingSlots = 14;

struct MegaShared {
    int abort;
    float ss[4];
    float amv[4];  // LM-head candidate of each consumer warp
    int ami[4];
    int res_base;  // first staged residual row
    int res_n;     // staged rows
    float res[kResRows];
    float gpart[4][kGroupBatch][16];  // per-warp row sums of up to kGroupBatch batches
    unsigned long long xe;            // tensor parallelism: epoch of the phase's exchange
    uint64_t xbar;                    // completion of the input-vector bulk copy
    uint64_t pbar;                   // completion of the next phase descriptor's bulk copy
};

// Position in the shared-memory ring: slot and the parity of its current
// lap (advanced without division).
struct RingPos {
    int s;
    uint32_t ph;
    __device__ __forceinline__ void advance(int slots) {
        if (++s == slots) {
            s = 0;
            ph ^= 1u;
        }
    }
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

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Publishes exchange epoch e to every rank (after this rank's data writes,
// which the caller has fenced at system scope) and waits, bounded, until
// every rank has published e.  Returns false on timeout.
__device__ bool exchange_flags(const MegaParams& p, unsigned long long e, volatile int* abort) {
    for (int r = 0; r < p.tp_size; ++r)
        st_release_sys64(reinterpret_cast<unsigned long long*>(p.peers[r] + kXchFlags) + p.tp_rank, e);
    const unsigned long long* own = reinterpret_cast<const unsigned long long*>(p.peers[p.tp_rank] + kXchFlags);
    const long long t0 = clock64();
    for (int r = 0; r < p.tp_size; ++r) {
        while (ld_acquire_sys64(own + r) < e) {
            if (*abort || (ld_acquire(p.err) & kErrWaitTimeout) || clock64() - t0 > kWaitCycles) {
                atomicOr(p.err, kErrWaitTimeout);
                *abort = 1;
                return false;
            }
        }
    }
    return true;
}

// Grid barrier of the consumer warps: every CTA adds 1 (release) to a 64-bit
// counter that only grows, and polls (acquire) until it reaches `target`
// (the launch's base plus gridDim.x per barrier passed).  One atomic per
// CTA, no reset and no last-arriver hop.  The named barrier orders the other
// consumer threads' writes before thread 0's release, which is cumulative,
// so no separate fence is needed.
//
// After an exchange phase (xe > 0) the barrier also crosses the GPUs: once
// every local CTA has arrived (each fenced its writes into the peers'
// regions at system scope first), CTA 0 publishes epoch xe to every rank,
// waits for every rank's, and adds one more arrival; the other CTAs wait for
// that one too (target counts it).
__device__ __forceinline__ void grid_sync(const MegaParams& p, volatile int* abort, int tid,
                                          unsigned long long target, unsigned long long xe = 0) {
    named_sync(1, kMegaConsumers);
    if (tid == 0 && !*abort) {
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p.bar) : "memory");
        if (xe && blockIdx.x == 0) {
            const long long t0 = clock64();
            while (ld_acquire64(p.bar) < target - 1) {
                if ((ld_acquire(p.err) & kErrWaitTimeout) || clock64() - t0 > kWaitCycles) {
                    atomicOr(p.err, kErrWaitTimeout);
                    *abort = 1;
                    break;
                }
            }
            if (!*abort) {
                __threadfence_system();
                exchange_flags(p, xe, abort);
            }
            // the extra arrival is made even after a failure, so no CTA waits
            // on it in vain
            asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p.bar) : "memory");
        }
        if (ld_acquire64(p.bar) < target) {
            const long long t0 = clock64();
            while (ld_acquire64(p.bar) < target) {
                __nanosleep(20);
                if ((ld_acquire(p.err) & kErrWaitTimeout) || clock64() - t0 > kWaitCycles) {
                    atomicOr(p.err, kErrWaitTimeout);
                    *abort = 1;
                    break;
                }
            }
        }
    }
    named_sync(1, kMegaConsumers);
}

// Output units [u0, u1) of this CTA: [U b / P, U (b + 1) / P).
__device__ __forceinline__ void unit_range(const MegaPhase& P, int& u0, int& u1) {
    u0 = (int)((long long)P.units * blockIdx.x / gridDim.x);
    u1 = (int)((long long)P.units * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Timeline slot of (step, phase) for this CTA; -1 when tracing is off.
__device__ __forceinline__ long long trace_base(const MegaParams& p, int step, int ph) {
    if (!p.trace) return -1;
    return (((long long)blockIdx.x * p.steps + step) * p.nphases + ph) * kTraceFields;
}

__device__ __forceinline__ void trace_mark(const MegaParams& p, long long base, int field) {
    if (base >= 0) p.trace[base + field] = global_ns();
}

// -------------------------------------------------------------- consumers

// The dot product of 4 weights at wp with 4 inputs, in element order.
template <typename WT>
__device__ __forceinline__ float piece_dot(const unsigned char* wp, const float4& xv) {
    float acc = 0.0f;
    if (WeightTraits<WT>::kBytes == 4) {
        const float4 w = *reinterpret_cast<const float4*>(wp);
        acc = fmaf(w.x, xv.x, acc);
        acc = fmaf(w.y, xv.y, acc);
        acc = fmaf(w.z, xv.z, acc);
        acc = fmaf(w.w, xv.w, acc);
    } else {
        // a bf16 value is the top half of the FP32 with the same bits, so
        // widening is a shift (low element) or a mask (high element)
        const uint2 raw = *reinterpret_cast<const uint2*>(wp);
        acc = fmaf(__uint_as_float(raw.x << 16), xv.x, acc);
        acc = fmaf(__uint_as_float(raw.x & 0xffff0000u), xv.y, acc);
        acc = fmaf(__uint_as_float(raw.y << 16), xv.z, acc);
        acc = fmaf(__uint_as_float(raw.y & 0xffff0000u), xv.w, acc);
    }
    return acc;
}

// Input vector of a GEMV phase into shared memory (RMSNorm applied when set).
// Residual phases also stage the residual rows of the CTA's units in sh.res,
// so the epilogue needs no L2 round trip.
__device__ void load_x(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid, int u0, int u1,
                       uint32_t& xphase, int tok) {
    const int warp = tid >> 5, lane = tid & 31;
    const float* src = P.x;
    if (!src) {
        src = p.input;
        if (!src) {
            int t = tok;
            if (t < 0 || t >= p.vocab) {
                if (tid == 0) atomicOr(p.err, kErrToken);
                t = 0;
            }
            src = p.emb + (size_t)t * P.K;
        }
    }
    // the input vector (and the norm weights behind it) in one bulk copy
    // each, issued first so the residual loads below overlap them; the
    // vector was written by generic stores (after the grid barrier's
    // acquire), read here through the async proxy.  A summed input (tensor
    // parallelism) is formed by the threads instead.
    const bool sum = P.nsum > 0;
    const uint32_t vbytes = (uint32_t)P.K * 4u;
    const uint32_t bytes = (sum ? 0u : vbytes) + (P.norm_w ? vbytes : 0u);
    if (tid == 0 && bytes) {
        fence_proxy_async_global();
        mbar_arrive_expect_tx(&sh.xbar, bytes);
        if (!sum) bulk_g2s_plain(xs, src, vbytes, &sh.xbar);
        if (P.norm_w) bulk_g2s_plain(xs + P.K, P.norm_w, vbytes, &sh.xbar);
    }
    if (sum) {
        // x = src + the ranks' partials in rank order (every rank forms the
        // same sum); this CTA also stores its share of the result for later
        // phases' residual reads
        const int s0 = (int)((long long)P.K * blockIdx.x / gridDim.x);
        const int s1 = (int)((long long)P.K * (blockIdx.x + 1) / gridDim.x);
        for (int i = tid * 4; i < P.K; i += kMegaConsumers * 4) {
            float4 v = __ldcg(reinterpret_cast<const float4*>(src + i));
            for (int r = 0; r < P.nsum; ++r) {
                const float4 w = __ldcg(reinterpret_cast<const float4*>(P.xsum + (size_t)r * P.K + i));
                v.x += w.x;
                v.y += w.y;
                v.z += w.z;
                v.w += w.w;
            }
            *reinterpret_cast<float4*>(xs + i) = v;
            if (P.xout) {
                const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (i + j >= s0 && i + j < s1) P.xout[i + j] = e[j];
            }
        }
    }
    int staged = 0;
    const int staged_base = u0;
    if (P.epi == kEpiResidual && u1 - u0 <= kResRows) {
        for (int i = tid; i < u1 - u0; i += kMegaConsumers) sh.res[i] = __ldcg(P.res + u0 + i);
        staged = u1 - u0;
    }
    if (tid == 0) {  // one writer; read after the named barrier at the end
        sh.res_n = staged;
        sh.res_base = staged_base;
    }
    if (bytes) {
        mega_wait(&sh.xbar, xphase & 1u, &sh.abort, p.err);
        ++xphase;
    }
    constexpr int STRIDE = kMegaConsumers * 4;
    if (P.x_copy && blockIdx.x == 0)
        for (int i = tid * 4; i < P.K; i += STRIDE)
            *reinterpret_cast<float4*>(P.x_copy + i) = *reinterpret_cast<const float4*>(xs + i);
    if (P.norm_w) {
        float ss = 0.0f;
        for (int i = tid * 4; i < P.K; i += STRIDE) {
            const float4 v = *reinterpret_cast<const float4*>(xs + i);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) sh.ss[warp] = ss;
        named_sync(1, kMegaConsumers);
        const float tot = ((sh.ss[0] + sh.ss[1]) + sh.ss[2]) + sh.ss[3];
        const float rms = rsqrtf(tot / (float)P.K + P.eps);
        // each thread scales the elements it summed
        for (int i = tid * 4; i < P.K; i += STRIDE) {
            float4 v = *reinterpret_cast<const float4*>(xs + i);
            const float4 w = *reinterpret_cast<const float4*>(xs + P.K + i);
            v.x = v.x * rms * w.x;
            v.y = v.y * rms * w.y;
            v.z = v.z * rms * w.z;
            v.w = v.w * rms * w.w;
            *reinterpret_cast<float4*>(xs + i) = v;
        }
    }
    named_sync(1, kMegaConsumers);
}

// Warp sums of N per-lane values by a reduce-scatter butterfly (N - 1
// exchanges that halve the values held per lane, then the remaining xor
// steps on one value): lane L returns the warp sum of value L / (32 / N).
// Every value is added along the same xor tree as a full butterfly (16, 8,
// 4, 2, 1), for N - 1 + log2(32 / N) shuffles instead of 5 N.
template <int N>
__device__ __forceinline__ float warp_reduce_scatter(const float* in, int lane) {
    float a[N];
#pragma unroll
    for (int i = 0; i < N; ++i) a[i] = in[i];
    int o = 16;
#pragma unroll
    for (int n = N; n > 1; n >>= 1, o >>= 1) {
        const bool hi = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = hi ? a[i] : a[i + n / 2];
            const float keep = hi ? a[i + n / 2] : a[i];
            a[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
#pragma unroll
    for (; o > 0; o >>= 1) a[0] += __shfl_xor_sync(0xffffffffu, a[0], o);
    return a[0];
}

// Epilogue of n batches whose first unit is ub (their row sums in gpart
// slots [0, n)), units below u1: the four warps' sums added in warp order,
// then store / residual add / SwiGLU / logits + argmax candidate.  All
// consumer threads take part; called between named barriers.  Units of a
// Q|K|V phase are rows of the stacked [q | k | v] output, so the stacked row
// is the output index.
template <typename WT, int NS>
__device__ void combine_batches(const MegaParams& p, const MegaPhase& P, MegaShared& sh, int ub, int n, int u1,
                                int tid, float& am_v, int& am_i) {
    constexpr int BU = MegaRows<WT>::R / NS;
    for (int idx = tid; idx < n * BU; idx += kMegaConsumers) {
        const int sl = idx / BU, i = idx % BU;
        const int row = ub + idx;
        if (row >= u1) continue;
        const float v = ((sh.gpart[0][sl][i] + sh.gpart[1][sl][i]) + sh.gpart[2][sl][i]) + sh.gpart[3][sl][i];
        if (NS == 2) {
            const int u = BU + i;
            const float yu = ((sh.gpart[0][sl][u] + sh.gpart[1][sl][u]) + sh.gpart[2][sl][u]) + sh.gpart[3][sl][u];
            P.out[row] = silu_mul(v, yu);
        } else if (P.epi == kEpiStore) {
            P.out[row] = v;
        } else if (P.epi == kEpiResidual) {
            const int ri = row - sh.res_base;
            const float r = (ri >= 0 && ri < sh.res_n) ? sh.res[ri] : __ldcg(P.res + row);
            P.out[row] = r + v;
        } else if (P.epi == kEpiExchange) {
            // this rank's partial of the row, into every rank's slot for it
            for (int r = 0; r < p.tp_size; ++r)
                reinterpret_cast<float*>(p.peers[r] + P.xch_off)[(size_t)p.tp_rank * P.units + row] = v;
        } else {
            float* lo = P.out ? P.out : p.logits;
            lo[row] = v;
            const int id = P.row_base + row;
            if (argmax_better(v, id, am_v, am_i)) {
                am_v = v;
                am_i = id;
            }
        }
    }
}

// Winner of the CTA -> partial; the last CTA reduces all partials in CTA
// order, writes the token and advances the decode state.
__device__ void argmax_phase_end(const MegaParams& p, MegaShared& sh, int tid, float am_v, int am_i) {
    const int warp = tid >> 5, lane = tid & 31;
    // the order is total, so any reduction tree picks the same winner
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, am_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, am_i, o);
        if (argmax_better(ov, oi, am_v, am_i)) {
            am_v = ov;
            am_i = oi;
        }
    }
    if (lane == 0) {
        sh.amv[warp] = am_v;
        sh.ami[warp] = am_i;
    }
    named_sync(1, kMegaConsumers);
    if (warp != 0) return;
    int last = 0;
    if (lane == 0) {
        float bv = -1e30f;
        int bi = 0;
        for (int w = 0; w < kMegaConsumers / 32; ++w)
            if (argmax_better(sh.amv[w], sh.ami[w], bv, bi)) {
                bv = sh.amv[w];
                bi = sh.ami[w];
            }
        p.am_val[blockIdx.x] = bv;
        p.am_idx[blockIdx.x] = bi;
        last = atom_add_acq_rel(p.am_cnt, 1u) == gridDim.x - 1;
    }
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    // the last CTA: every lane scans a strided share of the partials, then a
    // shuffle tree picks the winner (the order is total, so the result does
    // not depend on the tree's shape)
    float v = -1e30f;
    int id = 0;
    for (unsigned b = lane; b < gridDim.x; b += 32) {
        const float pv = __ldcg(p.am_val + b);
        const int pi = __ldcg(p.am_idx + b);
        if (argmax_better(pv, pi, v, id)) {
            v = pv;
            id = pi;
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
    if (lane != 0) return;
    if (p.tp_size > 1) {
        // this rank's winner (over its vocabulary rows) to every rank, then
        // the winner of all ranks' (the order is total: every rank agrees)
        const unsigned long long mine =
            (unsigned long long)__float_as_uint(v) | ((unsigned long long)(unsigned)id << 32);
        for (int r = 0; r < p.tp_size; ++r)
            reinterpret_cast<unsigned long long*>(p.peers[r] + kXchArgmax)[p.tp_rank] = mine;
        __threadfence_system();
        if (exchange_flags(p, sh.xe, &sh.abort)) {
            const unsigned long long* slots =
                reinterpret_cast<const unsigned long long*>(p.peers[p.tp_rank] + kXchArgmax);
            for (int r = 0; r < p.tp_size; ++r) {
                const unsigned long long s = __ldcg(slots + r);
                const float rv = __uint_as_float((unsigned)(s & 0xffffffffull));
                const int ri = (int)(unsigned)(s >> 32);
                if (argmax_better(rv, ri, v, id)) {
                    v = rv;
                    id = ri;
                }
            }
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

// A consumer's view of the ring: the next slot to take, and the wait
// accounting of the phase timeline.
struct SlotReader {
    unsigned char* ring;
    uint64_t* full;
    uint64_t* empty;
    RingPos* rp;
    int slots;
    volatile int* abort;
    unsigned* err;
    bool timed;
    long long waited;

    // Waits for the next slot; returns this thread's first byte in it.
    __device__ __forceinline__ const unsigned char* take(int tid, int eb) {
        if (timed) {
            const long long c0 = clock64();
            mega_wait(&full[rp->s], rp->ph, abort, err);
            waited += clock64() - c0;
        } else {
            mega_wait(&full[rp->s], rp->ph, abort, err);
        }
        return ring + (size_t)rp->s * kMegaSlot + (size_t)tid * 4 * eb;
    }
    // Hands the slot back to the producer (after the warp's last read of it).
    __device__ __forceinline__ void release(int lane) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[rp->s]);
        rp->advance(slots);
    }
};

// Stream row s of a batch of nb units -> its accumulator: gate rows first,
// then up rows (NS == 2).
template <int NS, int BU>
__device__ __forceinline__ int stream_row_acc(int s, int nb) {
    return (NS == 2 && s >= nb) ? BU + (s - nb) : s;
}

// acc[k] = v with k only known at run time, without indexing the register
// array dynamically.
template <int R>
__device__ __forceinline__ void acc_set(float* acc, int k, float v) {
#pragma unroll
    for (int m = 0; m < R; ++m)
        if (m == k) acc[m] = v;
}

// A batch when CB = K / 512 divides the pieces of a slot: every slot holds
// RS = PT / CB whole rows and the same column blocks in the same places, so
// the input columns stay in registers (xr) and a slot's rows are summed with
// compile-time indexing.  Each slot's RS row sums are reduced over the warp
// at once (the same xor tree as a reduction of the whole batch, so the same
// bits) and land in the warp's row-sum slots `gp`, indexed by accumulator.
// The slot loop stays rolled: its body is one slot, small enough for the
// instruction cache (an unrolled batch stalled the warps on instruction
// fetch).  The warp reduction of a slot runs one slot late, beside the next
// slot's loads and products, so the latency of its shuffle chain is hidden.
// Rows past `rows` (a short last batch) are not in the stream; the tail of
// its last slot is computed and dropped.
template <typename WT, int CB>
__device__ __forceinline__ void slot_row_sums(const unsigned char* wp, const float4* xr, float* v) {
    constexpr int PT = MegaRows<WT>::PT, PB = MegaRows<WT>::PB;
    constexpr int RS = PT / CB;
    float pv[PT];
#pragma unroll
    for (int i = 0; i < PT; ++i) pv[i] = piece_dot<WT>(wp + i * PB, xr[i % CB]);
#pragma unroll
    for (int k = 0; k < RS; ++k) {
        float t = 0.0f;
#pragma unroll
        for (int c = 0; c < CB; ++c) t += pv[k * CB + c];
        v[k] = t;
    }
}

template <typename WT, int NS, int CB>
__device__ __forceinline__ void batch_regs(SlotReader& rd, const float4* xr, float* gp, int rows, int nb, int tid,
                                           int lane) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, EB = MegaRows<WT>::EB;
    constexpr int RS = PT / CB;    // rows per slot
    constexpr int LPR = 32 / RS;   // lanes per row after the reduce-scatter
    static_assert(PT % CB == 0, "CB divides the slot");
    const int nslots = (rows + RS - 1) / RS;
    const int srow = lane / LPR;   // this lane's row within a slot after the reduction
    const bool writer = lane % LPR == 0;
    float v[RS];
    slot_row_sums<WT, CB>(rd.take(tid, EB), xr, v);
    rd.release(lane);
#pragma unroll 1
    for (int j = 1; j < nslots; ++j) {
        const unsigned char* wp = rd.take(tid, EB);
        float vn[RS];
        slot_row_sums<WT, CB>(wp, xr, vn);
        const float r = warp_reduce_scatter<RS>(v, lane);  // slot j - 1
        const int s = (j - 1) * RS + srow;
        if (writer && s < rows) gp[stream_row_acc<NS, BU>(s, nb)] = r;
        rd.release(lane);
#pragma unroll
        for (int k = 0; k < RS; ++k) v[k] = vn[k];
    }
    const float r = warp_reduce_scatter<RS>(v, lane);
    const int s = (nslots - 1) * RS + srow;
    if (writer && s < rows) gp[stream_row_acc<NS, BU>(s, nb)] = r;
}

// A batch when K / 512 >= the pieces of a slot: a slot holds the end of one
// row and at most the start of the next.  Both partial sums are formed
// without branches (pieces in column order), the running row sum carries
// over slots, and a finished row goes to its accumulator.  The input columns
// are read from shared memory.
template <typename WT, int NS>
__device__ __forceinline__ void batch_split(SlotReader& rd, const float* xt, int cb, int rows, int nb, float* acc,
                                            int tid, int lane) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, PB = MegaRows<WT>::PB, EB = MegaRows<WT>::EB;
    const int npieces = rows * cb;
    int q0 = 0;  // column block of the slot's first piece
    int s = 0;   // stream row of the slot's first piece
    float run = 0.0f;
    for (int p0 = 0; p0 < npieces; p0 += PT) {
        const unsigned char* wp = rd.take(tid, EB);
        const int n = min(PT, npieces - p0);
        const int split = cb - q0;  // pieces of row s in this slot (>= 1)
        float pv[PT];
#pragma unroll
        for (int i = 0; i < PT; ++i) {
            const int q = q0 + i >= cb ? q0 + i - cb : q0 + i;
            pv[i] = piece_dot<WT>(wp + i * PB, *reinterpret_cast<const float4*>(xt + q * kPiece));
        }
        rd.release(lane);
        float nxt = 0.0f;
#pragma unroll
        for (int i = 0; i < PT; ++i) {
            const float v = i < n ? pv[i] : 0.0f;
            if (i < split)
                run += v;
            else
                nxt += v;
        }
        if (split <= n) {  // row s ends in this slot
            acc_set<R>(acc, stream_row_acc<NS, BU>(s, nb), run);
            run = nxt;
            ++s;
            q0 = n - split;
        } else {
            q0 += n;
        }
    }
}

// Any batch, any cb: the pieces of each slot as independent products, added
// to a running row sum in stream order; a finished row moves to its
// accumulator.  Pieces past the batch's end (a short last batch) are not
// in the stream.
template <typename WT, int NS>
__device__ void batch_generic(SlotReader& rd, const float* xt, int cb, int nb, float* acc, int tid, int lane) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, PB = MegaRows<WT>::PB, EB = MegaRows<WT>::EB;
    const int npieces = (NS == 2 ? 2 * nb : nb) * cb;
    int q = 0;  // column block of the next piece
    int r = 0;  // row (stream order) of the next piece
    float racc = 0.0f;
    for (int p0 = 0; p0 < npieces; p0 += PT) {
        const unsigned char* wp = rd.take(tid, EB);
        const int n = min(PT, npieces - p0);
        float pv[PT];
        int qi = q;
#pragma unroll
        for (int i = 0; i < PT; ++i) {
            // bytes past n are stale but inside the slot: read, then dropped
            const float d = piece_dot<WT>(wp + i * PB, *reinterpret_cast<const float4*>(xt + qi * kPiece));
            pv[i] = i < n ? d : 0.0f;
            if (++qi == cb) qi = 0;
        }
        rd.release(lane);
#pragma unroll
        for (int i = 0; i < PT; ++i) {
            if (i < n) {
                racc += pv[i];
                if (++q == cb) {
                    acc_set<R>(acc, stream_row_acc<NS, BU>(r, nb), racc);
                    racc = 0.0f;
                    q = 0;
                    ++r;
                }
            }
        }
    }
}

template <typename WT, int NS, int CB>
__device__ void gemv_body(const MegaParams& p, const MegaPhase& P, SlotReader& rd, const float* xs, MegaShared& sh,
                          int tid, int u0, int u1) {
    constexpr int R = MegaRows<WT>::R;
    constexpr int BU = R / NS;  // units per batch
    static_assert(MegaRows<WT>::PT == R, "a batch of R rows fills whole slots");
    const int warp = tid >> 5, lane = tid & 31;
    const float* xt = xs + tid * 4;  // this thread's 4 columns of every piece
    constexpr int NXR = CB > 0 ? CB : 1;
    float4 xr[NXR];
    if (CB > 0) {
#pragma unroll
        for (int c = 0; c < NXR; ++c) xr[c] = *reinterpret_cast<const float4*>(xt + c * kPiece);
    }
    const bool split = CB == 0 && P.cb >= MegaRows<WT>::PT;
    float am_v = -1e30f;
    int am_i = 0;
    int bi = 0;  // batches finished in this phase
    for (int ub = u0; ub < u1; ub += BU) {
        const int nb = min(BU, u1 - ub);
        const int rows = NS * nb;  // stream rows of the batch
        float* gp = sh.gpart[warp][bi % kGroupBatch];
        if (CB > 0) {
            batch_regs<WT, NS, NXR>(rd, xr, gp, rows, nb, tid, lane);
        } else {
            float acc[R];
#pragma unroll
            for (int a = 0; a < R; ++a) acc[a] = 0.0f;
            if (split)
                batch_split<WT, NS>(rd, xt, P.cb, rows, nb, acc, tid, lane);
            else
                batch_generic<WT, NS>(rd, xt, P.cb, nb, acc, tid, lane);
            // the warp's sum of each row; lane L holds row L / (32 / R)
            const float v = warp_reduce_scatter<R>(acc, lane);
            constexpr int kLanesPerRow = 32 / R;
            if (lane % kLanesPerRow == 0) gp[lane / kLanesPerRow] = v;
        }
        // kGroupBatch batches held: every warp has summed them (all walk the
        // same rows); run their epilogue before the slots are reused
        if (++bi % kGroupBatch == 0) {
            named_sync(1, kMegaConsumers);
            combine_batches<WT, NS>(p, P, sh, u0 + (bi - kGroupBatch) * BU, kGroupBatch, u1, tid, am_v, am_i);
            named_sync(1, kMegaConsumers);
        }
    }
    const int rest = bi % kGroupBatch;
    if (rest) {
        named_sync(1, kMegaConsumers);
        combine_batches<WT, NS>(p, P, sh, u0 + (bi - rest) * BU, rest, u1, tid, am_v, am_i);
    }
    if (P.epi == kEpiArgmax) argmax_phase_end(p, sh, tid, am_v, am_i);
}

template <typename WT, int NS>
__device__ void gemv_phase(const MegaParams& p, const MegaPhase& P, unsigned char* ring, uint64_t* full,
                           uint64_t* empty, RingPos& rp, uint32_t& xphase, float* xs, MegaShared& sh, int tid,
                           long long tb, int tok) {
    int u0, u1;
    unit_range(P, u0, u1);
    load_x(p, P, xs, sh, tid, u0, u1, xphase, tok);
    if (tid == 0) trace_mark(p, tb, 1);
    SlotReader rd{ring, full, empty, &rp, p.ring_slots, &sh.abort, p.err, tb >= 0, 0};
    // widths that divide a slot's pieces keep their input columns in
    // registers (every thread takes the same branch: P is shared)
    switch (P.cb) {
        case 4: gemv_body<WT, NS, 4>(p, P, rd, xs, sh, tid, u0, u1); break;
        case 8: gemv_body<WT, NS, 8>(p, P, rd, xs, sh, tid, u0, u1); break;
        default: gemv_body<WT, NS, 0>(p, P, rd, xs, sh, tid, u0, u1); break;
    }
    if (tb >= 0) p.trace[tb + 5] = (unsigned long long)rd.waited;
}

__device__ void attention_merge(const AttnArgs& a, int kvh, int active, float* sm, int tid);

// One (KV head, split) item of decode attention inside the persistent
// kernel: the same computation as attention_item (attention.cuh), with its
// inputs brought in by bulk copies on the input-vector mbarrier, so the
// query rows, the RoPE row, the new K/V rows and the first K/V tile arrive
// in one round trip.  Tiles hold kAttnBulkTile positions (one per lane in
// the score pass).  A split that covers the whole sequence writes the
// normalised output directly; otherwise partials are merged by the last
// split of the head, as in attention_item.
//
// Scores: lane p walks the D/4 float4 chunks of its key row starting at
// chunk p mod (D/4), which keeps the unpadded [T][D] tile free of bank
// conflicts; the sum order per lane is fixed, so results are deterministic.
__device__ void attention_item_bulk(const AttnArgs& a, int kvh, int split, int pos, float* sm, MegaShared& sh,
                                    int tid, uint32_t& xphase, unsigned* err, unsigned long long* tr, long long tb) {
    // timeline marks of an attention phase (thread 0, tracing on)
    auto mark = [&](int f) {
        if (tb >= 0) tr[tb + f] = global_ns();
    };
    constexpr int T = kAttnBulkTile;
    constexpr int NW = kMegaConsumers / 32;
    constexpr int MAXH = (kAttnMaxGroup + NW - 1) / NW;
    constexpr int MAXDL = kAttnMaxD / 32;
    const int warp = tid >> 5, lane = tid & 31;
    const int D = a.D, G = a.nq / a.nkv, half = D / 2, nc = D / 4;
    const int seq = pos + 1;
    int chunk, active;
    attn_chunk(seq, a.splits, chunk, active);
    const int c0 = split * chunk;
    const int c1 = min(seq, c0 + chunk);
    const bool owns_new = (c1 == seq);

    float* qs = sm;                        // [G][D]
    float* kt = qs + G * D;                // [T][D]
    float* vt = kt + T * D;                // [T][D]
    float* ps = vt + T * D;                // [G][T]
    float* rope = ps + G * T;              // [D/2] (cos, sin)
    float* knew = rope + D;                // [D]
    float* vnew = knew + D;                // [D]
    int* s_last = reinterpret_cast<int*>(vnew + D);

    const float* kbase = a.k_cache + (size_t)kvh * a.max_seq * D;
    const float* vbase = a.v_cache + (size_t)kvh * a.max_seq * D;
    const uint32_t row_bytes = (uint32_t)D * 4u;

    // first round: q rows, RoPE row, new K/V rows, first K/V tile
    int t0 = c0, tl = min(T, c1 - c0);
    if (tid == 0) {
        fence_proxy_async_global();
        uint32_t bytes = (uint32_t)G * row_bytes + row_bytes + 2u * (uint32_t)tl * row_bytes;
        if (owns_new) bytes += 2u * row_bytes;
        mbar_arrive_expect_tx(&sh.xbar, bytes);
        bulk_g2s_plain(qs, a.qkv + (size_t)kvh * G * D, (uint32_t)G * row_bytes, &sh.xbar);
        bulk_g2s_plain(rope, a.rope + (size_t)pos * half, row_bytes, &sh.xbar);
        if (owns_new) {
            bulk_g2s_plain(knew, a.qkv + (size_t)a.nq * D + (size_t)kvh * D, row_bytes, &sh.xbar);
            bulk_g2s_plain(vnew, a.qkv + (size_t)(a.nq + a.nkv) * D + (size_t)kvh * D, row_bytes, &sh.xbar);
        }
        bulk_g2s_plain(kt, kbase + (size_t)t0 * D, (uint32_t)tl * row_bytes, &sh.xbar);
        bulk_g2s_plain(vt, vbase + (size_t)t0 * D, (uint32_t)tl * row_bytes, &sh.xbar);
    }
    mega_wait(&sh.xbar, xphase & 1u, &sh.abort, err);
    ++xphase;
    mark(1);

    // RoPE (cuda/rope.cu:13-24 with the tabulated factors) on q and the new
    // key; append the new K/V row (cuda/kv_cache.cu:4-14)
    const float2* rp = reinterpret_cast<const float2*>(rope);
    for (int i = tid; i < G * half; i += kMegaConsumers) {
        const int h = i / half, d = i % half;
        rope_apply(qs[h * D + d], qs[h * D + d + half], rp[d]);
    }
    if (owns_new) {
        float* kdst = a.k_cache + ((size_t)kvh * a.max_seq + pos) * D;
        float* vdst = a.v_cache + ((size_t)kvh * a.max_seq + pos) * D;
        for (int d = tid; d < half; d += kMegaConsumers) {
            rope_apply(knew[d], knew[d + half], rp[d]);
            kdst[d] = knew[d];
            kdst[d + half] = knew[d + half];
        }
        for (int d = tid; d < D; d += kMegaConsumers) vdst[d] = vnew[d];
    }
    named_sync(1, kMegaConsumers);

    // this warp's heads h = warp + j NW (warp-uniform validity)
    bool hv[MAXH];
    float m_run[MAXH], l_run[MAXH], o_run[MAXH][MAXDL];
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        hv[j] = warp + j * NW < G;
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < MAXDL; ++i) o_run[j][i] = 0.0f;
    }
    const int cstart = lane % nc;
    while (true) {
        // the cached row at `pos` is stale: use this item's rotated copy
        if (owns_new && pos >= t0 && pos < t0 + tl) {
            for (int d = tid; d < D; d += kMegaConsumers) {
                kt[(pos - t0) * D + d] = knew[d];
                vt[(pos - t0) * D + d] = vnew[d];
            }
            named_sync(1, kMegaConsumers);
        }
        // scores of key row `lane` against every head of the warp: each key
        // chunk is read once for all of them; two partial sums per head
        // (even / odd chunks) halve the dependent FMA chain
        float dd[MAXH][2];
#pragma unroll
        for (int j = 0; j < MAXH; ++j) dd[j][0] = dd[j][1] = 0.0f;
        if (lane < tl) {
            const float* kr = kt + lane * D;
            int c = cstart;
            auto chunk = [&](int e) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * c);
#pragma unroll
                for (int j = 0; j < MAXH; ++j) {
                    if (hv[j]) {
                        const float4 q4 = *reinterpret_cast<const float4*>(qs + (warp + j * NW) * D + 4 * c);
                        float t = dd[j][e];
                        t = fmaf(q4.x, k4.x, t);
                        t = fmaf(q4.y, k4.y, t);
                        t = fmaf(q4.z, k4.z, t);
                        t = fmaf(q4.w, k4.w, t);
                        dd[j][e] = t;
                    }
                }
                if (++c == nc) c = 0;
            };
            int n = 0;
            for (; n + 2 <= nc; n += 2) {
                chunk(0);
                chunk(1);
            }
            if (n < nc) chunk(0);
        }
        // online softmax of each head over the tile's positions
        float alpha[MAXH];
#pragma unroll
        for (int j = 0; j < MAXH; ++j) {
            alpha[j] = 1.0f;
            if (hv[j]) {
                const float s = lane < tl ? (dd[j][0] + dd[j][1]) * a.scale : -INFINITY;
                const float m_new = fmaxf(m_run[j], warp_max(s));
                alpha[j] = expf(m_run[j] - m_new);
                const float pe = lane < tl ? expf(s - m_new) : 0.0f;
                ps[(warp + j * NW) * T + lane] = pe;
                l_run[j] = l_run[j] * alpha[j] + warp_sum(pe);
                m_run[j] = m_new;
            }
        }
        __syncwarp();
        // P V: each value row is read once for all heads; every output
        // column's sum runs over the positions in order
        float acc[MAXH][MAXDL];
#pragma unroll
        for (int j = 0; j < MAXH; ++j)
#pragma unroll
            for (int i = 0; i < MAXDL; ++i) acc[j][i] = o_run[j][i] * alpha[j];
#pragma unroll 4
        for (int q = 0; q < tl; ++q) {
            float vq[MAXDL];
#pragma unroll
            for (int i = 0; i < MAXDL; ++i) vq[i] = lane + 32 * i < D ? vt[q * D + lane + 32 * i] : 0.0f;
#pragma unroll
            for (int j = 0; j < MAXH; ++j) {
                if (hv[j]) {
                    const float pq = ps[(warp + j * NW) * T + q];
#pragma unroll
                    for (int i = 0; i < MAXDL; ++i) acc[j][i] = fmaf(pq, vq[i], acc[j][i]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < MAXH; ++j)
#pragma unroll
            for (int i = 0; i < MAXDL; ++i) o_run[j][i] = acc[j][i];
        t0 += tl;
        if (t0 >= c1) break;
        // next tile: every thread's reads of the tile come before the copies
        tl = min(T, c1 - t0);
        fence_proxy_async_smem();
        named_sync(1, kMegaConsumers);
        if (tid == 0) {
            mbar_arrive_expect_tx(&sh.xbar, 2u * (uint32_t)tl * row_bytes);
            bulk_g2s_plain(kt, kbase + (size_t)t0 * D, (uint32_t)tl * row_bytes, &sh.xbar);
            bulk_g2s_plain(vt, vbase + (size_t)t0 * D, (uint32_t)tl * row_bytes, &sh.xbar);
        }
        mega_wait(&sh.xbar, xphase & 1u, &sh.abort, err);
        ++xphase;
    }

    mark(4);
    if (active == 1) {
        // the only split: normalised output (cuda/attention.cu:30-43 after softmax)
#pragma unroll
        for (int j = 0; j < MAXH; ++j) {
            if (hv[j]) {
                const float inv = 1.0f / l_run[j];
                float* o = a.out + ((size_t)kvh * G + warp + j * NW) * D;
#pragma unroll
                for (int i = 0; i < MAXDL; ++i)
                    if (lane + 32 * i < D) o[lane + 32 * i] = o_run[j][i] * inv;
            }
        }
        return;
    }

    // partial (m, l, o) of each head; the last split of the head merges
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        if (hv[j]) {
            float* pp = a.part + (((size_t)kvh * a.splits + split) * G + warp + j * NW) * (D + 2);
            if (lane == 0) {
                pp[0] = m_run[j];
                pp[1] = l_run[j];
            }
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (lane + 32 * i < D) pp[2 + lane + 32 * i] = o_run[j][i];
        }
    }
    named_sync(1, kMegaConsumers);
    if (tid == 0) {
        // release: this CTA's partials (ordered by the named barrier) before
        // the ticket; acquire: the other splits' partials before the merge
        const unsigned ticket = atom_add_acq_rel(&a.counter[kvh], 1u);
        *s_last = (ticket == (unsigned)active - 1u);
    }
    named_sync(1, kMegaConsumers);
    mark(5);
    if (*s_last) {
        attention_merge(a, kvh, active, sm, tid);
        mark(6);
    }
}

// The flash-decoding merge of the active splits of KV head kvh by the last
// split to finish: out = sum_s w_s o_s / sum_s w_s l_s with w_s = exp(m_s -
// M).  This is the attention phase's critical path, so it is arranged for
// few dependent L2 round trips: every thread owns output elements (head,
// column) and issues the loads of its elements' partial rows for
// kMergeChunk splits at once, the first chunk before the weights are
// known; meanwhile each warp forms the split weights of its heads (lanes
// over splits) into shared memory after the item's scratch.  Sums run over
// the splits in order, so the result does not depend on timing.
__device__ void attention_merge(const AttnArgs& a, int kvh, int active, float* sm, int tid) {
    constexpr int NW = kMegaConsumers / 32;
    constexpr int MAXH = (kAttnMaxGroup + NW - 1) / NW;
    constexpr int SC = kMergeChunk;
    constexpr int OPT = 4;  // output elements per thread per pass
    const int warp = tid >> 5, lane = tid & 31;
    const int D = a.D, G = a.nq / a.nkv, S = a.splits;
    const size_t sstride = (size_t)G * (D + 2);
    const float* pk = a.part + (size_t)kvh * S * sstride;
    float* wtab = sm + attn_bulk_smem_floats(G, D);  // [G][S] split weights
    float* linv = wtab + (size_t)G * S;               // [G] 1 / sum_s w_s l_s
    const int nout = G * D;

    float ov[OPT][SC];
    auto load_chunk = [&](int o0, int s0) {
#pragma unroll
        for (int k = 0; k < OPT; ++k) {
            const int e = o0 + k * kMegaConsumers;
            const int h = e / D, d = e - h * D;
#pragma unroll
            for (int q = 0; q < SC; ++q)
                ov[k][q] = (e < nout && s0 + q < active)
                               ? __ldcg(pk + (s0 + q) * sstride + (size_t)h * (D + 2) + 2 + d)
                               : 0.0f;
        }
    };
    load_chunk(tid, 0);

    // split weights of this warp's heads
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        const int h = warp + j * NW;
        if (h >= G) continue;
        const float* ph = pk + (size_t)h * (D + 2);
        float mr[kMergeRounds], lr[kMergeRounds];
#pragma unroll
        for (int r = 0; r < kMergeRounds; ++r) {
            const int s = lane + 32 * r;
            mr[r] = s < active ? __ldcg(ph + s * sstride) : -INFINITY;
            lr[r] = s < active ? __ldcg(ph + s * sstride + 1) : 0.0f;
        }
        float M = mr[0];
#pragma unroll
        for (int r = 1; r < kMergeRounds; ++r) M = fmaxf(M, mr[r]);
        M = warp_max(M);
        float L = 0.0f;
#pragma unroll
        for (int r = 0; r < kMergeRounds; ++r) {
            const int s = lane + 32 * r;
            if (s < active) {
                const float w = expf(mr[r] - M);
                wtab[h * S + s] = w;
                L = fmaf(lr[r], w, L);
            }
        }
        L = warp_sum(L);
        if (lane == 0) linv[h] = 1.0f / L;
    }
    named_sync(1, kMegaConsumers);

    for (int o0 = tid; o0 < nout; o0 += OPT * kMegaConsumers) {
        float acc[OPT];
#pragma unroll
        for (int k = 0; k < OPT; ++k) acc[k] = 0.0f;
        for (int s0 = 0; s0 < active; s0 += SC) {
            if (o0 != tid || s0 != 0) load_chunk(o0, s0);
#pragma unroll
            for (int k = 0; k < OPT; ++k) {
                const int e = o0 + k * kMegaConsumers;
                const int h = e < nout ? e / D : 0;
#pragma unroll
                for (int q = 0; q < SC; ++q)
                    if (s0 + q < active) acc[k] = fmaf(ov[k][q], wtab[h * S + s0 + q], acc[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < OPT; ++k) {
            const int e = o0 + k * kMegaConsumers;
            if (e < nout) a.out[(size_t)kvh * nout + e] = acc[k] * linv[e / D];
        }
    }
    if (tid == 0) a.counter[kvh] = 0u;
}

__device__ void attention_phase(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid, long long tb,
                                uint32_t& xphase, int pos) {
    if (pos < 0 || pos >= p.attn.max_seq) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(p.err, kErrPosition);
        return;
    }
    AttnArgs a = p.attn;
    a.k_cache = P.kc;
    a.v_cache = P.vc;
    int chunk, active;
    attn_chunk(pos + 1, a.splits, chunk, active);
    const int items = a.nkv * a.splits;
    bool first = true;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int kvh = it / a.splits, split = it % a.splits;
        if (split >= active) continue;
        if (!first) {
            // the previous item's shared-memory use comes before this one's copies
            fence_proxy_async_smem();
            named_sync(1, kMegaConsumers);
        }
        first = false;
        attention_item_bulk(a, kvh, split, pos, xs, sh, tid, xphase, p.err, p.trace, tb);
    }
}

// ---------------------------------------------------------------- producer

// A CTA's weight stream of one GEMV phase as consecutive byte ranges of the
// weight matrices, in the order the consumers walk the rows: NS == 1, the
// rows [u0, u1) of the stacked matrices (one range per matrix crossed);
// NS == 2, per batch of bu units, the batch's gate rows then its up rows.
// Scalar fields only (no arrays indexed at run time), so it stays in
// registers.
struct StreamRanges {
    const unsigned char *w0, *w1, *w2;
    int r0, r1;  // rows of the first two stacked matrices
    int ns, bu;
    long long rowbytes;
    int u, u1;  // next unit (NS == 2: first unit of the batch), end of the CTA's units
    bool up;    // NS == 2: the next range is the batch's up rows
    const unsigned char* addr;  // rest of the current range
    long long left;

    __device__ void start(const MegaPhase& P, int eb, int u0, int uend, int units_per_batch) {
        w0 = static_cast<const unsigned char*>(P.w[0]);
        w1 = static_cast<const unsigned char*>(P.w[1]);
        w2 = static_cast<const unsigned char*>(P.w[2]);
        r0 = P.nseg > 1 ? P.seg_rows[0] : P.units;
        r1 = P.nseg > 2 ? P.seg_rows[1] : P.units;
        ns = P.ns;
        bu = units_per_batch;
        rowbytes = (long long)P.K * eb;
        u = u0;
        u1 = uend;
        up = false;
        addr = nullptr;
        left = 0;
    }
    // Moves to the next range; false when the phase's stream has ended.
    __device__ bool next() {
        if (u >= u1) return false;
        if (ns == 1) {
            // stacked rows: [0, r0) of w0, [r0, r0 + r1) of w1, the rest of w2
            const unsigned char* w;
            int first, end;
            if (u < r0) {
                w = w0;
                first = 0;
                end = r0;
            } else if (u < r0 + r1) {
                w = w1;
                first = r0;
                end = r0 + r1;
            } else {
                w = w2;
                first = r0 + r1;
                end = u1;
            }
            end = min(end, u1);
            addr = w + (long long)(u - first) * rowbytes;
            left = (long long)(end - u) * rowbytes;
            u = end;
            return true;
        }
        const int nb = min(bu, u1 - u);
        addr = (up ? w1 : w0) + (long long)u * rowbytes;
        left = (long long)nb * rowbytes;
        if (up) u += nb;
        up = !up;
        return true;
    }
};

// Position in this CTA's weight stream: the GEMV phases of every step, in
// consumer order, as byte ranges; `pos` counts the bytes passed since the
// launch started.
template <typename WT>
struct StreamCursor {
    int step, ph;
    long long left;  // bytes left in the current phase
    long long pos;
    bool done;
    StreamRanges st;

    __device__ void start(const MegaParams& p) {
        step = 0;
        ph = -1;
        pos = 0;
        left = 0;
        done = false;
        next_phase(p);
    }
    // Moves to the next GEMV phase with units for this CTA.
    __device__ void next_phase(const MegaParams& p) {
        while (true) {
            if (++ph == p.nphases) {
                ph = 0;
                if (++step >= p.steps) {
                    done = true;
                    left = 0;
                    return;
                }
            }
            const MegaPhase& P = p.phases[ph];
            if (P.kind != kPhGemv) continue;
            int u0, u1;
            unit_range(P, u0, u1);
            if (u0 >= u1) continue;
            st.start(P, MegaRows<WT>::EB, u0, u1, MegaRows<WT>::R / P.ns);
            left = (long long)(u1 - u0) * st.rowbytes * P.ns;
            return;
        }
    }
    // The next contiguous run of at most `max` bytes of the current phase;
    // false at the end of the phase's ranges.
    __device__ bool chunk(uint32_t max, const unsigned char*& addr, uint32_t& n) {
        if (st.left == 0 && !st.next()) return false;
        n = (uint32_t)(st.left < (long long)max ? st.left : (long long)max);
        addr = st.addr;
        st.addr += n;
        st.left -= n;
        left -= n;
        pos += n;
        return true;
    }
};

// One thread streams every GEMV phase's weights of this CTA, across phases
// and steps, into the ring: each slot takes the next min(16 KB, rest of the
// phase) bytes with one or more bulk copies (a slot straddles at most a
// matrix or gate/up boundary), completing on the slot's full barrier; a
// phase starts a new slot.  From the second lap on it waits until the
// consumers released the slot.  (Prefetching the stream further ahead into
// L2 while the ring is full was measured slower: the extra queueing
// lengthens the latency-bound synchronisation between phases.)
template <typename WT>
__device__ void produce(const MegaParams& p, unsigned char* ring, uint64_t* full, uint64_t* empty, MegaShared& sh) {
    volatile int* abort = &sh.abort;
    const int slots = p.ring_slots;
    const uint64_t pol = l2_evict_first_policy();
    uint32_t sl = 0;  // slots armed so far
    bool ok = true;
    RingPos wp{0, 0u};
    StreamCursor<WT> lc;
    lc.start(p);
    long long pwait = 0;  // cycles waited for free slots in the phase (trace)
    while (!lc.done && ok) {
        const uint32_t sb = (uint32_t)(lc.left < kMegaSlot ? lc.left : kMegaSlot);
        const long long c0 = clock64();
        if (sl >= (uint32_t)slots && !mega_wait(&empty[wp.s], wp.ph ^ 1u, abort, p.err)) {
            ok = false;
            break;
        }
        pwait += clock64() - c0;
        mbar_arrive_expect_tx(&full[wp.s], sb);
        unsigned char* dst = ring + (size_t)wp.s * kMegaSlot;
        uint32_t fill = 0;
        while (fill < sb) {
            const unsigned char* a;
            uint32_t n;
            if (!lc.chunk(sb - fill, a, n)) {
                // the ranges ended before the phase's byte count (a
                // descriptor error): the slot's consumers time out
                atomicOr(p.err, kErrWaitTimeout);
                *abort = 1;
                ok = false;
                break;
            }
            bulk_g2s(dst + fill, a, n, &full[wp.s], pol);
            fill += n;
        }
        ++sl;
        wp.advance(slots);
        if (lc.left == 0) {
            const long long tbp = trace_base(p, lc.step, lc.ph);
            trace_mark(p, tbp, 4);
            if (tbp >= 0) p.trace[tbp + 6] = (unsigned long long)pwait;
            pwait = 0;
            lc.next_phase(p);
        }
    }
    if (!ok) {
        // the next slot was not armed; let the copies of every armed slot
        // land before the CTA can exit
        const uint32_t first = sl > (uint32_t)slots ? sl - slots : 0u;
        volatile int no_abort = 0;
        for (uint32_t q = first; q < sl; ++q) mega_wait(&full[q % slots], (q / slots) & 1u, &no_abort, p.err);
    }
}

template <typename WT>
__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(const MegaParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ MegaShared sh;
    __shared__ MegaPhase sP[2];  // descriptors of the current and the next phase
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slots = p.ring_slots;
    unsigned char* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)slots * kMegaSlot);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + p.x_floats);
    uint64_t* empty = full + slots;
    if (tid == 0) {
        for (int s = 0; s < slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMegaConsumers / 32);
        }
        mbar_init(&sh.xbar, 1);
        mbar_init(&sh.pbar, 1);
        mbar_fence_init();
        sP[0] = p.phases[0];
        sP[1] = p.phases[p.nphases > 1 ? 1 : 0];
        sh.abort = 0;
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        if (lane == 0) produce<WT>(p, ring, full, empty, sh);
        return;
    }

    RingPos rp{0, 0u};
    uint32_t xphase = 0, pphase = 0;
    unsigned long long xe = p.xe_base;  // exchange epochs so far
    unsigned long long target = p.bar_base;
    int cur = 0;
    long long n = 0;  // phases started so far
    const long long total = (long long)p.steps * p.nphases;
    for (int step = 0; step < p.steps; ++step) {
        // this step's token and position (written by the previous step's
        // LM-head phase before the grid barrier)
        const unsigned long long st = ld_acquire64(reinterpret_cast<const unsigned long long*>(p.state));
        const int tok = (int)(unsigned)(st & 0xffffffffull), pos = (int)(unsigned)(st >> 32);
        for (int ph = 0; ph < p.nphases; ++ph) {
            const long long tb = tid == 0 ? trace_base(p, step, ph) : -1;
            trace_mark(p, tb, 0);
            // this phase's descriptor was prefetched into sP[cur] (the first
            // two were copied at the start)
            if (n >= 2) {
                mega_wait(&sh.pbar, pphase & 1u, &sh.abort, p.err);
                ++pphase;
            }
            // the previous phase's shared-memory accesses (sP[cur ^ 1]
            // included) come before this phase's bulk copies into them
            fence_proxy_async_smem();
            named_sync(1, kMegaConsumers);
            if (tid == 0 && n >= 1 && n + 1 < total) {
                const int nph = ph + 1 == p.nphases ? 0 : ph + 1;
                mbar_arrive_expect_tx(&sh.pbar, (uint32_t)sizeof(MegaPhase));
                bulk_g2s_plain(&sP[cur ^ 1], p.phases + nph, (uint32_t)sizeof(MegaPhase), &sh.pbar);
            }
            const MegaPhase& P = sP[cur];
            // tensor parallelism: the partial-sum phases and the LM head
            // exchange with the other ranks, each under a new epoch
            const bool xdata = p.tp_size > 1 && P.kind == kPhGemv && P.xch_off >= 0;
            if (xdata || (p.tp_size > 1 && P.kind == kPhGemv && P.epi == kEpiArgmax)) ++xe;
            if (tid == 0) sh.xe = xe;
            // every consumer thread takes the same branches here (no branch on the
            // abort flag, which the producer may set at any moment): the phases
            // contain named barriers
            if (P.kind == kPhAttn) {
                attention_phase(p, P, xs, sh, tid, tb, xphase, pos);
            } else if (P.ns == 2) {
                gemv_phase<WT, 2>(p, P, ring, full, empty, rp, xphase, xs, sh, tid, tb, tok);
            } else {
                gemv_phase<WT, 1>(p, P, ring, full, empty, rp, xphase, xs, sh, tid, tb, tok);
            }
            trace_mark(p, tb, 2);
            if (xdata) __threadfence_system();  // this CTA's writes into the peers' regions
            target += gridDim.x + (xdata ? 1 : 0);
            grid_sync(p, &sh.abort, tid, target, xdata ? xe : 0);
            trace_mark(p, tb, 3);
            cur ^= 1;
            ++n;
        }
    }
    if (tid == 0 && *reinterpret_cast<volatile int*>(&sh.abort)) {
        // waits were cut short: give bulk copies still in flight into this
        // CTA's shared memory time to land before it exits
        const long long t0 = clock64();
        while (clock64() - t0 < 20000000ll) __nanosleep(1000);
    }
}

}  // namespace

int mega_smem_bytes(int ring_slots, int x_floats) {
    return ring_slots * kMegaSlot + x_floats * 4 + 2 * ring_slots * 8;
}

int mega_max_ring_slots() { return kMaxRingSlots; }

int mega_static_smem(int weight_dtype) {
    cudaFuncAttributes fa;
    const void* k = weight_dtype == INFERNT_DTYPE_BF16
                        ? reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16>)
                        : reinterpret_cast<const void*>(decode_mega_kernel<float>);
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) {
        cudaGetLastError();
        return 48 * 1024;
    }
    return (int)fa.sharedSizeBytes;
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
