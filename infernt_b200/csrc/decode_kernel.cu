// decode_kernel.cu — the persistent decode kernel.
//
// One CTA per SM runs every phase of a decode step (and of a chain of
// steps): per layer the fused RMSNorm + Q/K/V projection, attention (RoPE,
// KV append, split-KV GQA, merge), O projection + residual, RMSNorm +
// gate/up + SiLU, down projection + residual; then RMSNorm + LM head +
// argmax.  Phases hand their outputs to the next phase as tagged words
// (below), with no grid barrier.
//
// Warps 0-7 consume, as two teams of four warps; lane 0 of warp 8 produces:
// it streams the CTA's share of every GEMV phase's weights into a ring of
// 16 KB shared-memory slots with 1-D bulk copies (cp.async.bulk).  A GEMV
// phase gives CTA b the output units [U b / P, U (b + 1) / P), whose weight
// rows are contiguous in row-major memory, so every slot is one contiguous
// 16 KB run of HBM (two runs where it straddles a matrix or gate/up
// boundary): the access pattern that streams fastest, and a split balanced
// to one row per CTA.  Weights do not depend on activations, so the
// producer runs ahead across phase boundaries and layers while the
// consumers wait for inputs or compute attention.  Warps 9-11 only complete
// the producer's warpgroup and leave at once.
//
// Consumers walk the stream in 512-element pieces, each thread of a team
// covering 4 columns of every piece, in batches of R rows (R = 8 FP32 / 16
// bf16; for gate/up R / 2 units, gate rows then up rows), which fill exactly
// K / 512 slots.  The teams take turns: when a slot holds whole rows (K / 512
// divides the pieces of a slot) the even slots of a phase go to team 0 and
// the odd ones to team 1, otherwise the even batches to team 0 and the odd
// ones to team 1; a team steps over the other's slots without waiting.  Two
// teams keep two slots in flight per SM, so after any wait for inputs the
// consumers drain the ring faster than HBM refills it.  Each thread adds a
// row's pieces in column order into one accumulator per row; for the usual
// widths the (row, column block) of every piece of a batch is known at
// compile time and the input columns stay in registers.  Row sums are
// reduced over the warp by a reduce-scatter (per slot in that case, else
// once per batch), and the owning team's four warp sums are added in warp
// order in the batches' epilogue.  Every output is reduced inside one CTA
// in a fixed order, so results do not depend on timing and no cross-CTA
// merge sits on the critical path.
//
// Every wait (ring slots, tagged words, bulk copies) is bounded by a clock
// budget (MegaParams::wait_cycles, about 2 s by default); on expiry the CTA
// sets kErrWaitTimeout in the error word, marks itself aborted and runs the
// remaining control flow without waiting, so the kernel always terminates
// and the host reports INFERNT_ERR_DEVICE.
#include <array>
#include <cstring>

#include "decode_kernel.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "sample.cuh"

namespace infernt {

namespace {

constexpr int kMegaSlot = 16384;
constexpr int kMegaConsumers = 256;  // two teams of four consumer warps
constexpr int kTeamThreads = 128;    // a team covers the 512 columns of a piece, 4 per thread
constexpr int kTeamWarps = kTeamThreads / 32;
constexpr int kConsumerWarps = kMegaConsumers / 32;
constexpr int kProducerWarp = 8;     // lane 0 streams the weights; warps 9-11 leave at once
constexpr int kMegaThreads = 384;    // three warpgroups
// Register split (setmaxnreg): the kernel is compiled for 384 threads at
// kLaunchRegs each; the producer's warpgroup hands registers to the two
// consumer warpgroups.  The split must not exceed what the launch holds.
constexpr int kLaunchRegs = 168;
constexpr int kConsumerRegs = 232;
constexpr int kProducerRegs = 40;
static_assert(2 * 128 * kConsumerRegs + 128 * kProducerRegs <= kMegaThreads * kLaunchRegs,
              "register split exceeds the launch's registers");
// Clock budget of every wait in this CTA (MegaParams::wait_cycles, set by
// thread 0 before the first barrier).
__shared__ long long s_wait_cycles;
constexpr int kResRows = 128;                    // residual rows a CTA stages per phase
constexpr int kMergeChunk = 8;                   // attention splits merged per round of loads
constexpr int kMergeRounds = 2;                  // lanes x rounds bound the splits of a KV head (64)

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
    float ss[kConsumerWarps];
    float amv[kConsumerWarps];  // LM-head candidate of each consumer warp
    int ami[kConsumerWarps];
    int res_base;  // first staged residual row
    int res_n;     // staged rows
    float res[kResRows];
    float gpart[2][kTeamWarps][kGroupBatch][16];  // row sums per team and warp of up to kGroupBatch batches
    unsigned long long skey;          // Gumbel key of the step (temperature sampling)
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
        if (clock64() - t0 > s_wait_cycles) {
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

// ------------------------------------------------------------ tagged words
//
// Activations travel between CTAs (and, with tensor parallelism, between
// GPUs) as 8-byte words: the FP32 value in the low half, in the high half
// the tag of the phase instance that wrote it (launch tag base + step x
// phases + phase + 1, the same on every rank).  An aligned 8-byte store is
// single-copy atomic, so a reader that sees the tag it expects has that
// instance's value: consumers poll the data words themselves, and a phase
// boundary costs one L2 round trip instead of a grid barrier followed by a
// load.  Reuse of a buffer is safe because every phase needs the whole of
// its predecessor's output: no CTA can overwrite a word of phase k's output
// before every reader of it has passed phase k + 1.

__device__ __forceinline__ unsigned long long ll_pack(float v, unsigned tag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
}

__device__ __forceinline__ void st_ll(unsigned long long* a, float v, unsigned tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(ll_pack(v, tag)) : "memory");
}

// into another GPU's memory (tensor parallelism)
__device__ __forceinline__ void st_ll_sys(unsigned long long* a, float v, unsigned tag) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(ll_pack(v, tag)) : "memory");
}

template <bool SYS>
__device__ __forceinline__ ulonglong2 ld_ll2(const unsigned long long* a) {
    ulonglong2 v;
    if (SYS)
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(a) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(a) : "memory");
    return v;
}

template <bool SYS>
__device__ __forceinline__ unsigned long long ld_ll1(const unsigned long long* a) {
    unsigned long long v;
    if (SYS)
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

__device__ __forceinline__ bool ll_is(unsigned long long w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(unsigned long long w) { return __uint_as_float((unsigned)w); }

// Bounded re-reading of words not yet current.  On timeout (or when another
// CTA has already timed out) the CTA is marked aborted, the error word set,
// and the stale value returned: control flow continues without waiting.
struct LLWait {
    unsigned* err;
    volatile int* abort;
    // called once per failed polling round: checks the time budget
    __device__ __forceinline__ bool give_up(long long t0, unsigned& spins) const {
        if (*abort) return true;
        if ((++spins & 63u) == 0u) {
            if ((ld_acquire(err) & kErrWaitTimeout) || clock64() - t0 > s_wait_cycles) {
                atomicOr(err, kErrWaitTimeout);
                *abort = 1;
                return true;
            }
        }
        return false;
    }
    template <bool SYS>
    __device__ __forceinline__ unsigned long long one(const unsigned long long* a, unsigned long long w,
                                                      unsigned tag) const {
        if (ll_is(w, tag)) return w;
        const long long t0 = clock64();
        unsigned spins = 0;
        do {
            if (give_up(t0, spins)) break;
            w = ld_ll1<SYS>(a);
        } while (!ll_is(w, tag));
        return w;
    }
    template <bool SYS>
    __device__ __forceinline__ float2 two(const unsigned long long* a, ulonglong2 w, unsigned tag) const {
        if (!(ll_is(w.x, tag) && ll_is(w.y, tag))) {
            const long long t0 = clock64();
            unsigned spins = 0;
            do {
                if (give_up(t0, spins)) break;
                w = ld_ll2<SYS>(a);
            } while (!(ll_is(w.x, tag) && ll_is(w.y, tag)));
        }
        return make_float2(ll_val(w.x), ll_val(w.y));
    }
};

// Polls words w[0, n) (loaded from addr(k)) until each carries `tag`:
// every round re-reads all stale words at once, so a round costs one round
// trip however many words are late.
template <int N, bool SYS, typename Addr>
__device__ __forceinline__ void ll_poll(unsigned long long (&w)[N], int n, Addr addr, unsigned tag,
                                        const LLWait& wt) {
    const long long t0 = clock64();
    unsigned spins = 0;
    while (true) {
        bool ok = true;
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (k < n && !ll_is(w[k], tag)) ok = false;
        if (ok || wt.give_up(t0, spins)) return;
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (k < n && !ll_is(w[k], tag)) w[k] = ld_ll1<SYS>(addr(k));
    }
}

constexpr int kLLBatch = 16;  // word pairs a thread has in flight when reading a vector

// dst[0, n) = the values of the tagged words src[0, n) of phase instance
// `tag` (src 16-byte aligned), read by the consumer threads in
// batches of kLLBatch pairs each (one round trip per batch).  Not inlined:
// its registers for the loads in flight do not add to its callers'.
template <bool SYS>
__device__ __noinline__ void ll_read_vec(const unsigned long long* src, float* dst, int n, unsigned tag, int tid,
                                         const LLWait wt) {
    constexpr int STEP = kMegaConsumers * 2;
    for (int base = tid * 2; base < n; base += STEP * kLLBatch) {
        ulonglong2 w[kLLBatch];
#pragma unroll
        for (int k = 0; k < kLLBatch; ++k) {
            const int i = base + k * STEP;
            if (i + 1 < n) w[k] = ld_ll2<SYS>(src + i);
        }
        // re-read the stale pairs of the batch together until all are current
        const long long t0 = clock64();
        unsigned spins = 0;
        while (true) {
            bool ok = true;
#pragma unroll
            for (int k = 0; k < kLLBatch; ++k) {
                const int i = base + k * STEP;
                if (i + 1 < n && !(ll_is(w[k].x, tag) && ll_is(w[k].y, tag))) ok = false;
            }
            if (ok || wt.give_up(t0, spins)) break;
#pragma unroll
            for (int k = 0; k < kLLBatch; ++k) {
                const int i = base + k * STEP;
                if (i + 1 < n && !(ll_is(w[k].x, tag) && ll_is(w[k].y, tag))) w[k] = ld_ll2<SYS>(src + i);
            }
        }
#pragma unroll
        for (int k = 0; k < kLLBatch; ++k) {
            const int i = base + k * STEP;
            if (i + 1 < n) *reinterpret_cast<float2*>(dst + i) = make_float2(ll_val(w[k].x), ll_val(w[k].y));
        }
    }
    if ((n & 1) && tid == 0) dst[n - 1] = ll_val(wt.one<SYS>(src + n - 1, ld_ll1<SYS>(src + n - 1), tag));
}

// A run of tagged words src[0, n) read into dst[0, n) (n even, src 16-byte
// and dst 8-byte aligned).
struct LLSeg {
    const unsigned long long* src;
    float* dst;
    int n;
};

// ll_read_vec over three runs at once: the word pairs of all three are
// loaded in the same batches, so runs that land together cost one round
// trip instead of one each.  Batches of kSegBatch pairs per thread (the
// attention inputs are a few thousand words at most).
constexpr int kSegBatch = 4;
__device__ __noinline__ void ll_read_segs(const LLSeg s0, const LLSeg s1, const LLSeg s2, unsigned tag, int tid,
                                          const LLWait wt) {
    constexpr int STEP = kMegaConsumers * 2;
    const int n01 = s0.n + s1.n, total = n01 + s2.n;
    auto src_of = [&](int i) {
        return i < s0.n ? s0.src + i : (i < n01 ? s1.src + (i - s0.n) : s2.src + (i - n01));
    };
    auto dst_of = [&](int i) {
        return i < s0.n ? s0.dst + i : (i < n01 ? s1.dst + (i - s0.n) : s2.dst + (i - n01));
    };
    for (int base = tid * 2; base < total; base += STEP * kSegBatch) {
        ulonglong2 w[kSegBatch];
#pragma unroll
        for (int k = 0; k < kSegBatch; ++k)
            if (base + k * STEP < total) w[k] = ld_ll2<false>(src_of(base + k * STEP));
        const long long t0 = clock64();
        unsigned spins = 0;
        while (true) {
            bool ok = true;
#pragma unroll
            for (int k = 0; k < kSegBatch; ++k)
                if (base + k * STEP < total && !(ll_is(w[k].x, tag) && ll_is(w[k].y, tag))) ok = false;
            if (ok || wt.give_up(t0, spins)) break;
#pragma unroll
            for (int k = 0; k < kSegBatch; ++k)
                if (base + k * STEP < total && !(ll_is(w[k].x, tag) && ll_is(w[k].y, tag)))
                    w[k] = ld_ll2<false>(src_of(base + k * STEP));
        }
#pragma unroll
        for (int k = 0; k < kSegBatch; ++k)
            if (base + k * STEP < total)
                *reinterpret_cast<float2*>(dst_of(base + k * STEP)) = make_float2(ll_val(w[k].x), ll_val(w[k].y));
    }
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

// (a.x, a.y) = (fma(w0, x0, a.x), fma(w1, x1, a.y)): one packed FP32 FMA
// (two lanes, each rounded as fmaf).  The consumers are bound by issue
// latency, so halving their FMA instructions shortens every slot.
__device__ __forceinline__ void fma2(float2& a, float w0, float w1, float x0, float x1) {
    asm("{\n\t.reg .b64 pw, px, pa;\n\t"
        "mov.b64 pw, {%2, %3};\n\t"
        "mov.b64 px, {%4, %5};\n\t"
        "mov.b64 pa, {%0, %1};\n\t"
        "fma.rn.f32x2 pa, pw, px, pa;\n\t"
        "mov.b64 {%0, %1}, pa;\n\t}"
        : "+f"(a.x), "+f"(a.y)
        : "f"(w0), "f"(w1), "f"(x0), "f"(x1));
}

// The 4 weights at wp (FP32, or bf16 widened: a bf16 value is the top half
// of the FP32 with the same bits, so widening is a shift for the low
// element and a mask for the high one), multiplied into the two lanes of a:
// lane 0 takes elements 0 and 2, lane 1 elements 1 and 3.
template <typename WT>
__device__ __forceinline__ void piece_fma2(float2& a, const unsigned char* wp, const float4& xv) {
    if (WeightTraits<WT>::kBytes == 4) {
        const float4 w = *reinterpret_cast<const float4*>(wp);
        fma2(a, w.x, w.y, xv.x, xv.y);
        fma2(a, w.z, w.w, xv.z, xv.w);
    } else {
        const uint2 raw = *reinterpret_cast<const uint2*>(wp);
        fma2(a, __uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u), xv.x, xv.y);
        fma2(a, __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u), xv.z, xv.w);
    }
}

// The dot product of 4 weights at wp with 4 inputs: (w0 x0 + w2 x2) +
// (w1 x1 + w3 x3), each lane of the packed FMA rounded as fmaf.
template <typename WT>
__device__ __forceinline__ float piece_dot(const unsigned char* wp, const float4& xv) {
    float2 a = make_float2(0.0f, 0.0f);
    piece_fma2<WT>(a, wp, xv);
    return a.x + a.y;
}

// RMSNorm folded into the GEMV: for the widths whose input columns stay in
// registers (K = 2048, 4096) the phase reads the raw input, each thread
// multiplies its columns by the norm weights and sums their squares, and the
// epilogue scales every row sum by rsqrt(sum x^2 / K + eps):
// W (x * w * r) = r (W (x * w)) (cuda/rmsnorm.cu:10-26, with the factor r
// applied once per output instead of once per input element).  This takes
// the norm's two barriers and passes over the input off the critical path
// at the phase start.
__device__ __forceinline__ bool norm_folded(const MegaPhase& P) {
    return P.norm_w != nullptr && (P.cb == 4 || P.cb == 8);
}


// Input vector of a GEMV phase into shared memory (RMSNorm applied when
// set, unless folded), `ts` the tag of phase 0 of this step, `tag` this
// phase's.
//
// * Tagged input (P.x): read as it lands (phase P.x_ph's tag).
// * Layer 0: the embedding row of the step's token (or the launch's input
//   vector) by bulk copy; its raw values are also published as this CTA's
//   share [K b / P, K (b + 1) / P) of the residual stream at P.xout.
// * Tensor parallelism (P.nsum > 0): first this CTA's share of base +
//   the ranks' partials (rank order, the same sum on every rank), published
//   at P.xout; then the whole vector from every CTA's share.
// Residual phases also stage the (tagged) residual rows of the CTA's units
// in sh.res.
__device__ void load_x(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid, int u0, int u1,
                       uint32_t& xphase, int tok, unsigned ts, unsigned tag, long long tb) {
    const int warp = tid >> 5, lane = tid & 31;
    const LLWait wt{p.err, &sh.abort};
    const int K = P.K;
    const int s0 = (int)((long long)K * blockIdx.x / gridDim.x);
    const int s1 = (int)((long long)K * (blockIdx.x + 1) / gridDim.x);
    const float* plain = nullptr;
    if (!P.x && P.nsum == 0) {
        plain = p.input;
        if (!plain) {
            int t = tok;
            if (t < 0 || t >= p.vocab) {
                if (tid == 0) atomicOr(p.err, kErrToken);
                t = 0;
            }
            plain = p.emb + (size_t)t * K;
        }
    }
    // constant inputs (norm weights, the embedding row, the launch's input
    // vector) by bulk copy, issued first so the tagged reads below overlap
    // them; nothing in this launch writes them, so no proxy fence is needed
    const uint32_t vbytes = (uint32_t)K * 4u;
    const uint32_t bytes = (plain ? vbytes : 0u) + (P.norm_w ? vbytes : 0u);
    if (tid == 0 && bytes) {
        mbar_arrive_expect_tx(&sh.xbar, bytes);
        if (plain) bulk_g2s_plain(xs, plain, vbytes, &sh.xbar);
        if (P.norm_w) bulk_g2s_plain(xs + K, P.norm_w, vbytes, &sh.xbar);
    }
    // the residual rows of the CTA's units (residual phases): loaded now,
    // checked after the input vector, so the two reads overlap
    static_assert(kResRows <= kMegaConsumers, "one residual row per thread");
    const bool stage = P.res && u1 - u0 <= kResRows;
    const bool my_res = stage && tid < u1 - u0;
    unsigned long long res_w = 0;
    if (my_res) res_w = ld_ll1<false>(P.res + u0 + tid);
    if (tid == 0) {  // one writer; read after the named barrier at the end
        sh.res_n = stage ? u1 - u0 : 0;
        sh.res_base = u0;
    }
    if (P.nsum > 0) {
        // this CTA's share: base + partial 0 + partial 1 + ...
        const unsigned bt = ts + (unsigned)P.xbase_ph, pt = ts + (unsigned)P.sum_ph;
        const unsigned long long* parts =
            reinterpret_cast<const unsigned long long*>(p.peers[p.tp_rank] + P.sum_off);
        for (int i = s0 + tid; i < s1; i += kMegaConsumers) {
            // the own share was stored by this CTA (current at once)
            const float base = ll_val(wt.one<false>(P.xbase + i, ld_ll1<false>(P.xbase + i), bt));
            unsigned long long w[kMaxTp];
#pragma unroll
            for (int r = 0; r < kMaxTp; ++r)
                if (r < P.nsum) w[r] = ld_ll1<true>(parts + (size_t)r * K + i);
            ll_poll<kMaxTp, true>(w, P.nsum, [&](int r) { return parts + (size_t)r * K + i; }, pt, wt);
            float v = base;
#pragma unroll
            for (int r = 0; r < kMaxTp; ++r)
                if (r < P.nsum) v += ll_val(w[r]);
            st_ll(P.xout + i, v, tag);
        }
        ll_read_vec<false>(P.xout, xs, K, tag, tid, wt);
    } else if (P.x) {
        ll_read_vec<false>(P.x, xs, P.kx, ts + (unsigned)P.x_ph, tid, wt);
        for (int i = P.kx + tid; i < K; i += kMegaConsumers) xs[i] = 0.0f;
    }
    if (my_res) sh.res[tid] = ll_val(wt.one<false>(P.res + u0 + tid, res_w, ts + (unsigned)P.res_ph));
    trace_mark(p, tb, 7);
    if (bytes) {
        mega_wait(&sh.xbar, xphase & 1u, &sh.abort, p.err);
        ++xphase;
    }
    named_sync(1, kMegaConsumers);  // every thread's tagged reads into xs
    trace_mark(p, tb, 8);
    if (plain && P.xout)
        for (int i = s0 + tid; i < s1; i += kMegaConsumers) st_ll(P.xout + i, xs[i], tag);
    // widths whose input columns stay in registers fold RMSNorm into the
    // GEMV (norm_folded): xs keeps the raw input, nothing more to do here
    if (norm_folded(P)) return;
    constexpr int STRIDE = kMegaConsumers * 4;
    if (P.norm_w) {
        float ss = 0.0f;
        for (int i = tid * 4; i < K; i += STRIDE) {
            const float4 v = *reinterpret_cast<const float4*>(xs + i);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) sh.ss[warp] = ss;
        named_sync(1, kMegaConsumers);
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) tot += sh.ss[w];
        const float rms = rsqrtf(tot / (float)K + P.eps);
        // each thread scales the elements it summed
        for (int i = tid * 4; i < K; i += STRIDE) {
            float4 v = *reinterpret_cast<const float4*>(xs + i);
            const float4 w = *reinterpret_cast<const float4*>(xs + K + i);
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

// Sum of the warp row sums of accumulator a of batch slot sl: the four
// warps of team 0 in warp order, then (TWO: rows whose pieces both teams
// summed) the four of team 1.
template <bool TWO>
__device__ __forceinline__ float gpart_sum(const MegaShared& sh, int sl, int a) {
    float v = ((sh.gpart[0][0][sl][a] + sh.gpart[0][1][sl][a]) + sh.gpart[0][2][sl][a]) + sh.gpart[0][3][sl][a];
    if (TWO) v = (((v + sh.gpart[1][0][sl][a]) + sh.gpart[1][1][sl][a]) + sh.gpart[1][2][sl][a]) + sh.gpart[1][3][sl][a];
    return v;
}

// Epilogue of n batches whose first unit is ub (their row sums in gpart
// slots [0, n)), units below u1: the warps' sums added in a fixed order
// (gpart_sum), then store / residual add / SwiGLU / logits + argmax
// candidate.  All consumer threads take part; called between named
// barriers.  Units of a Q|K|V phase are rows of the stacked [q | k | v]
// output, so the stacked row is the output index.
template <typename WT, int NS, bool TWO, bool FOLD>
__device__ void combine_batches(const MegaParams& p, const MegaPhase& P, MegaShared& sh, int ub, int n, int u1,
                                int tid, float& am_v, int& am_i, unsigned ts, unsigned tag) {
    constexpr int BU = MegaRows<WT>::R / NS;
    // folded RMSNorm (norm_folded): the factor from team 0's sums of squares
    float r = 1.0f;
    if (FOLD && P.norm_w)
        r = rsqrtf((((sh.ss[0] + sh.ss[1]) + sh.ss[2]) + sh.ss[3]) / (float)P.K + P.eps);
    for (int idx = tid; idx < n * BU; idx += kMegaConsumers) {
        const int sl = idx / BU, i = idx % BU;
        const int row = ub + idx;
        if (row >= u1) continue;
        const float v = gpart_sum<TWO>(sh, sl, i) * r;
        if (NS == 2) {
            const int u = BU + i;
            const float yu = gpart_sum<TWO>(sh, sl, u) * r;
            st_ll(P.out + row, silu_mul(v, yu), tag);
        } else if (P.epi == kEpiStore) {
            st_ll(P.out + row, v, tag);
        } else if (P.epi == kEpiResidual) {
            const int ri = row - sh.res_base;
            float r;
            if (ri >= 0 && ri < sh.res_n) {
                r = sh.res[ri];
            } else {
                const LLWait wt{p.err, &sh.abort};
                r = ll_val(wt.one<false>(P.res + row, ld_ll1<false>(P.res + row), ts + (unsigned)P.res_ph));
            }
            st_ll(P.out + row, r + v, tag);
        } else if (P.epi == kEpiExchange) {
            // this rank's partial of the row, into every rank's slot for it
            for (int r = 0; r < p.tp_size; ++r)
                st_ll_sys(reinterpret_cast<unsigned long long*>(p.peers[r] + P.xch_off) + (size_t)p.tp_rank * P.units +
                              row,
                          v, tag);
        } else {
            p.logits[row] = v;
            const int id = P.row_base + row;
            // greedy: the logit; sampling: its Gumbel score (global id, so
            // every rank of a tensor-parallel run draws the same noise)
            const float sc = p.inv_temp > 0.0f ? gumbel_score(v, p.inv_temp, sh.skey, (uint64_t)id) : v;
            if (argmax_better(sc, id, am_v, am_i)) {
                am_v = sc;
                am_i = id;
            }
        }
    }
}

// Winner of the CTA -> partial; the last CTA reduces all partials in CTA
// order, writes the token and advances the decode state.
__device__ void argmax_phase_end(const MegaParams& p, MegaShared& sh, int tid, float am_v, int am_i,
                                 unsigned tag) {
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
        // this rank's winner (over its vocabulary rows) into every rank's
        // slot for it: value bits | id << 32 | a step mark << 56 (ids below
        // 2^24; the mark is the step's count since the plan was built, low 7
        // bits, with the top bit set so that zeroed memory never matches);
        // then the winner of all ranks' slots once every slot carries this
        // step's mark (the order is total: every rank agrees)
        const unsigned t8 = (((tag - 1u) / (unsigned)p.nphases) & 0x7fu) | 0x80u;
        const unsigned long long mine = (unsigned long long)__float_as_uint(v) |
                                        ((unsigned long long)((unsigned)id & 0xffffffu) << 32) |
                                        ((unsigned long long)t8 << 56);
        for (int r = 0; r < p.tp_size; ++r)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(
                             reinterpret_cast<unsigned long long*>(p.peers[r] + kXchArgmax) + p.tp_rank),
                         "l"(mine)
                         : "memory");
        const unsigned long long* slots = reinterpret_cast<const unsigned long long*>(p.peers[p.tp_rank] + kXchArgmax);
        const LLWait wt{p.err, &sh.abort};
        unsigned long long ws[kMaxTp];
        for (int r = 0; r < p.tp_size; ++r) ws[r] = ld_ll1<true>(slots + r);
        const long long t0 = clock64();
        unsigned spins = 0;
        while (true) {  // re-read the stale slots together
            bool ok = true;
            for (int r = 0; r < p.tp_size; ++r)
                if ((unsigned)(ws[r] >> 56) != t8) ok = false;
            if (ok || wt.give_up(t0, spins)) break;
            for (int r = 0; r < p.tp_size; ++r)
                if ((unsigned)(ws[r] >> 56) != t8) ws[r] = ld_ll1<true>(slots + r);
        }
        for (int r = 0; r < p.tp_size; ++r) {
            const unsigned long long w = ws[r];
            const float rv = __uint_as_float((unsigned)w);
            const int ri = (int)((unsigned)(w >> 32) & 0xffffffu);
            if (argmax_better(rv, ri, v, id)) {
                v = rv;
                id = ri;
            }
        }
    }
    // the next step's (token, position) is published last, with release
    // semantics: every CTA acquires it before the step, and with it this
    // step's KV-cache rows and the state below
    const int step = __ldcg(p.state + 2);
    const int pos = __ldcg(p.state + 1);
    if (p.hist) p.hist[step] = id;
    p.state[3] = id;
    p.state[2] = step + 1;
    *p.am_cnt = 0u;
    const unsigned long long nst = (unsigned long long)(unsigned)id | ((unsigned long long)(unsigned)(pos + 1) << 32);
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(reinterpret_cast<unsigned long long*>(p.state)),
                 "l"(nst)
                 : "memory");
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
    // Steps over n slots that the other team consumes (no wait, no release).
    __device__ __forceinline__ void skip(int n) {
        for (int i = 0; i < n; ++i) rp->advance(slots);
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
    // packed FMAs: per row two accumulators (even / odd pieces), two lanes each
    float2 a[RS][2];
#pragma unroll
    for (int k = 0; k < RS; ++k) a[k][0] = a[k][1] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < PT; ++i) piece_fma2<WT>(a[i / CB][(i % CB) & 1], wp + i * PB, xr[i % CB]);
#pragma unroll
    for (int k = 0; k < RS; ++k) v[k] = (a[k][0].x + a[k][0].y) + (a[k][1].x + a[k][1].y);
}

template <typename WT, int NS, int CB>
__device__ __forceinline__ void batch_regs(SlotReader& rd, const float4* xr, float* gp, int rows, int nb, int ctid,
                                           int lane, int par) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, EB = MegaRows<WT>::EB;
    constexpr int RS = PT / CB;    // rows per slot
    constexpr int LPR = 32 / RS;   // lanes per row after the reduce-scatter
    static_assert(PT % CB == 0, "CB divides the slot");
    const int nslots = (rows + RS - 1) / RS;
    // this team's slots of the batch: par, par + 2, ... (par = 0 or 1)
    if (par >= nslots) {
        rd.skip(nslots);
        return;
    }
    const int srow = lane / LPR;   // this lane's row within a slot after the reduction
    const bool writer = lane % LPR == 0;
    rd.skip(par);
    float v[RS];
    slot_row_sums<WT, CB>(rd.take(ctid, EB), xr, v);
    rd.release(lane);
    int jl = par;  // the batch slot whose row sums v holds
#pragma unroll 1
    for (int j = par + 2; j < nslots; j += 2) {
        rd.skip(1);  // the other team's slot j - 1
        const unsigned char* wp = rd.take(ctid, EB);
        float vn[RS];
        slot_row_sums<WT, CB>(wp, xr, vn);
        const float r = warp_reduce_scatter<RS>(v, lane);  // slot jl
        const int s = jl * RS + srow;
        if (writer && s < rows) gp[stream_row_acc<NS, BU>(s, nb)] = r;
        rd.release(lane);
#pragma unroll
        for (int k = 0; k < RS; ++k) v[k] = vn[k];
        jl = j;
    }
    const float r = warp_reduce_scatter<RS>(v, lane);
    const int s = jl * RS + srow;
    if (writer && s < rows) gp[stream_row_acc<NS, BU>(s, nb)] = r;
    rd.skip(nslots - 1 - jl);  // the other team's slots after this team's last
}

// A batch when K / 512 >= the pieces of a slot: a slot holds the end of one
// row and at most the start of the next.  The teams take alternate slots
// (slot g of the ring belongs to team g & 1), so each forms its partial sum
// of every row over the pieces in its own slots: both partial sums of a
// slot are formed without branches (pieces in column order), the running
// row sum carries over slots, and at a row's end the partial goes to its
// accumulator; a slot of the other team contributes nothing but moves the
// row and column bookkeeping along.  The input columns are read from
// shared memory.
template <typename WT, int NS>
__device__ __forceinline__ void batch_split(SlotReader& rd, const float* xt, int cb, int rows, int nb, float* acc,
                                            int ctid, int lane, int team) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, PB = MegaRows<WT>::PB, EB = MegaRows<WT>::EB;
    const int npieces = rows * cb;
    int q0 = 0;  // column block of the slot's first piece
    int s = 0;   // stream row of the slot's first piece
    float run = 0.0f;
#pragma unroll 1
    for (int p0 = 0; p0 < npieces; p0 += PT) {
        const int n = min(PT, npieces - p0);
        const int split = cb - q0;  // pieces of row s in this slot (>= 1)
        float nxt = 0.0f;
        if ((rd.rp->s & 1) == team) {
            const unsigned char* wp = rd.take(ctid, EB);
            // inputs of piece i: column block q0 + i of row s (i < split),
            // else block i - split of row s + 1; each an immediate offset
            // from one of two bases.  Pieces past n (the batch's last slot,
            // where row s is the batch's last row and split == n) are stale
            // and land in nxt, which is not used after that slot.
            const float* xa = xt + q0 * kPiece;
            const float* xb = xt - split * kPiece;
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                const float* xp = i < split ? xa + i * kPiece : xb + i * kPiece;
                const float d = piece_dot<WT>(wp + i * PB, *reinterpret_cast<const float4*>(xp));
                if (i < split)
                    run += d;
                else
                    nxt += d;
            }
            rd.release(lane);
        } else {
            // the other team's slot: nothing to add, only the row bookkeeping
            rd.skip(1);
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

// A batch when the slot holds pieces of up to MB + 1 rows (MB row ends:
// MB x K / 512 >= the pieces of a slot, K / 512 smaller than them): the
// shape of batch_split with MB + 1 running sums.  Piece i belongs to row
// s + k, k the row ends before it (b0 = K / 512 - q0, b0 + K / 512, ...), and
// reads column block q0 + i - k K / 512; the sums are kept in stream order
// and each finished row's goes to its accumulator.  Stale pieces of a
// batch's last slot (past its last row end) land in a later sum, which is
// not used.
template <typename WT, int NS, int MB>
__device__ __forceinline__ void batch_rows(SlotReader& rd, const float* xt, int cb, int rows, int nb, float* acc,
                                           int ctid, int lane, int team) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, PB = MegaRows<WT>::PB, EB = MegaRows<WT>::EB;
    const int npieces = rows * cb;
    int q0 = 0;  // column block of the slot's first piece
    int s = 0;   // stream row of the slot's first piece
    float run = 0.0f;
#pragma unroll 1
    for (int p0 = 0; p0 < npieces; p0 += PT) {
        const int n = min(PT, npieces - p0);
        const int b0 = cb - q0;  // pieces of row s in this slot (>= 1)
        float sum[MB + 1];
        sum[0] = run;
#pragma unroll
        for (int e = 1; e <= MB; ++e) sum[e] = 0.0f;
        if ((rd.rp->s & 1) == team) {
            const unsigned char* wp = rd.take(ctid, EB);
            const float* xq = xt + q0 * kPiece;
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                int k = 0;
#pragma unroll
                for (int e = 0; e < MB; ++e) k += i >= b0 + e * cb ? 1 : 0;
                const float d =
                    piece_dot<WT>(wp + i * PB, *reinterpret_cast<const float4*>(xq + (i - k * cb) * kPiece));
#pragma unroll
                for (int e = 0; e <= MB; ++e)
                    if (k == e) sum[e] += d;
            }
            rd.release(lane);
        } else {
            // the other team's slot: nothing to add, only the row bookkeeping
            rd.skip(1);
        }
        int ends = 0;  // rows that end in this slot
#pragma unroll
        for (int e = 0; e < MB; ++e)
            if (b0 + e * cb <= n) ends = e + 1;
#pragma unroll
        for (int e = 0; e < MB; ++e)
            if (e < ends) acc_set<R>(acc, stream_row_acc<NS, BU>(s + e, nb), sum[e]);
        float nr = sum[0];
#pragma unroll
        for (int e = 1; e <= MB; ++e)
            if (e == ends) nr = sum[e];
        run = nr;
        q0 = ends ? n - (b0 + (ends - 1) * cb) : q0 + n;
        s += ends;
    }
}

// Any batch, any cb: the pieces of each slot as independent products, added
// to a running row sum in stream order; a finished row moves to its
// accumulator.  Pieces past the batch's end (a short last batch) are not
// in the stream.  As in batch_split, each team sums the pieces of its own
// slots (the other team's count as zero).
template <typename WT, int NS>
__device__ void batch_generic(SlotReader& rd, const float* xt, int cb, int nb, float* acc, int ctid, int lane,
                              int team) {
    constexpr int R = MegaRows<WT>::R, BU = R / NS;
    constexpr int PT = MegaRows<WT>::PT, PB = MegaRows<WT>::PB, EB = MegaRows<WT>::EB;
    const int npieces = (NS == 2 ? 2 * nb : nb) * cb;
    int q = 0;  // column block of the next piece
    int r = 0;  // row (stream order) of the next piece
    float racc = 0.0f;
    for (int p0 = 0; p0 < npieces; p0 += PT) {
        const int n = min(PT, npieces - p0);
        float pv[PT];
        if ((rd.rp->s & 1) == team) {
            const unsigned char* wp = rd.take(ctid, EB);
            int qi = q;
#pragma unroll
            for (int i = 0; i < PT; ++i) {
                // bytes past n are stale but inside the slot: read, then dropped
                const float d = piece_dot<WT>(wp + i * PB, *reinterpret_cast<const float4*>(xt + qi * kPiece));
                pv[i] = i < n ? d : 0.0f;
                if (++qi == cb) qi = 0;
            }
            rd.release(lane);
        } else {
#pragma unroll
            for (int i = 0; i < PT; ++i) pv[i] = 0.0f;
            rd.skip(1);
        }
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

template <typename WT, int NS, int CB, bool NARROW>
__device__ void gemv_body(const MegaParams& p, const MegaPhase& P, SlotReader& rd, const float* xs, MegaShared& sh,
                          int tid, int u0, int u1, unsigned ts, unsigned tag) {
    constexpr int R = MegaRows<WT>::R, PT = MegaRows<WT>::PT;
    constexpr int BU = R / NS;  // units per batch
    static_assert(PT == R, "a batch of R rows fills whole slots");
    static_assert(kGroupBatch % 2 == 0, "both teams' batches of a group");
    const int warp = tid >> 5, lane = tid & 31;
    const int team = warp / kTeamWarps, cwarp = warp % kTeamWarps, ctid = tid % kTeamThreads;
    const float* xt = xs + ctid * 4;  // this thread's 4 columns of every piece
    constexpr int NXR = CB > 0 ? CB : 1;
    float4 xr[NXR];
    if (CB > 0) {
#pragma unroll
        for (int c = 0; c < NXR; ++c) xr[c] = *reinterpret_cast<const float4*>(xt + c * kPiece);
        if ((CB == 4 || CB == 8) && P.norm_w) {
            // folded RMSNorm: a team covers every column once; team 0's warps
            // publish their sums of squares for the epilogue's factor
            const float* wn = xs + P.K + ctid * 4;
            float ss = 0.0f;
#pragma unroll
            for (int c = 0; c < NXR; ++c) {
                const float4 w = *reinterpret_cast<const float4*>(wn + c * kPiece);
                float4& v = xr[c];
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
                v.x *= w.x;
                v.y *= w.y;
                v.z *= w.z;
                v.w *= w.w;
            }
            ss = warp_sum(ss);
            if (team == 0 && lane == 0) sh.ss[cwarp] = ss;
        }
    }
    const bool split = CB == 0 && P.cb >= PT;
    float am_v = -1e30f;
    int am_i = 0;
    int bi = 0;  // batches finished in this phase
    for (int ub = u0; ub < u1; ub += BU) {
        const int nb = min(BU, u1 - ub);
        const int rows = NS * nb;  // stream rows of the batch
        // slot g of the ring belongs to team g & 1 (the ring has an even
        // number of slots, so a team's slot one lap earlier was its own)
        if (CB > 0) {
            // whole rows per slot: the owning team's warp sums, team-0 entries
            batch_regs<WT, NS, NXR>(rd, xr, sh.gpart[0][cwarp][bi % kGroupBatch], rows, nb, ctid, lane,
                                    (team ^ rd.rp->s) & 1);
        } else {
            // rows across slots: both teams' partial sums of every row
            float* gp = sh.gpart[team][cwarp][bi % kGroupBatch];
            float acc[R];
#pragma unroll
            for (int a = 0; a < R; ++a) acc[a] = 0.0f;
            if (split)
                batch_split<WT, NS>(rd, xt, P.cb, rows, nb, acc, ctid, lane, team);
            else if (NARROW && 2 * P.cb >= PT)
                batch_rows<WT, NS, 2>(rd, xt, P.cb, rows, nb, acc, ctid, lane, team);
            else if (NARROW && 3 * P.cb >= PT)
                batch_rows<WT, NS, 3>(rd, xt, P.cb, rows, nb, acc, ctid, lane, team);
            else
                batch_generic<WT, NS>(rd, xt, P.cb, nb, acc, ctid, lane, team);
            // the warp's sum of each row; lane L holds row L / (32 / R)
            const float v = warp_reduce_scatter<R>(acc, lane);
            constexpr int kLanesPerRow = 32 / R;
            if (lane % kLanesPerRow == 0) gp[lane / kLanesPerRow] = v;
        }
        // kGroupBatch batches held: both teams have summed their rows; run
        // their epilogue before the row-sum slots are reused
        if (++bi % kGroupBatch == 0) {
            named_sync(1, kMegaConsumers);
            combine_batches<WT, NS, CB == 0, CB == 4 || CB == 8>(p, P, sh, u0 + (bi - kGroupBatch) * BU,
                                                                 kGroupBatch, u1, tid, am_v, am_i, ts, tag);
            named_sync(1, kMegaConsumers);
        }
    }
    const int rest = bi % kGroupBatch;
    if (rest) {
        named_sync(1, kMegaConsumers);
        combine_batches<WT, NS, CB == 0, CB == 4 || CB == 8>(p, P, sh, u0 + (bi - rest) * BU, rest, u1, tid, am_v,
                                                             am_i, ts, tag);
    }
    if (P.epi == kEpiArgmax) argmax_phase_end(p, sh, tid, am_v, am_i, tag);
}

// The cached K/V rows of this CTA's items in the attention phase that
// follows (caches P.kc / P.vc), and the RoPE row of `pos`, into L2: issued
// when the Q|K|V phase starts, so the attention phase's bulk copies of them
// hit L2 instead of waiting for HBM behind the weight stream.
__device__ void attention_prefetch(const MegaParams& p, const MegaPhase& P, int pos) {
    const AttnArgs& a = p.attn;
    if (pos < 0 || pos >= a.max_seq) return;
    int chunk, active;
    attn_chunk(pos + 1, a.splits, chunk, active);
    const uint32_t row_bytes = (uint32_t)a.D * 4u;
    bool any = false;
    for (int it = blockIdx.x; it < a.nkv * a.splits; it += gridDim.x) {
        const int kvh = it / a.splits, split = it % a.splits;
        if (split >= active) continue;
        any = true;
        const int c0 = split * chunk, c1 = min(pos, c0 + chunk);  // row pos is this step's
        if (c1 <= c0) continue;
        const size_t off = ((size_t)kvh * a.max_seq + c0) * a.D;
        bulk_prefetch_l2(P.kc + off, (uint32_t)(c1 - c0) * row_bytes);
        bulk_prefetch_l2(P.vc + off, (uint32_t)(c1 - c0) * row_bytes);
    }
    if (any && a.rope) bulk_prefetch_l2(a.rope + (size_t)pos * (a.D / 2), row_bytes);
}

template <typename WT, int NS, bool NARROW>
__device__ void gemv_phase(const MegaParams& p, const MegaPhase& P, unsigned char* ring, uint64_t* full,
                           uint64_t* empty, RingPos& rp, uint32_t& xphase, float* xs, MegaShared& sh, int tid,
                           long long tb, int tok, int pos, unsigned ts, unsigned tag) {
    if (P.kc && tid == 0) attention_prefetch(p, P, pos);
    int u0, u1;
    unit_range(P, u0, u1);
    load_x(p, P, xs, sh, tid, u0, u1, xphase, tok, ts, tag, tb);
    if (tid == 0) trace_mark(p, tb, 1);
    SlotReader rd{ring, full, empty, &rp, p.ring_slots, &sh.abort, p.err, tb >= 0, 0};
    // widths that divide a slot's pieces keep their input columns in
    // registers (every thread takes the same branch: P is shared)
    if constexpr (NARROW) {
        switch (P.cb) {
            case 1: gemv_body<WT, NS, 1, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
            case 2: gemv_body<WT, NS, 2, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
            case 4: gemv_body<WT, NS, 4, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
            case 8: gemv_body<WT, NS, 8, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
            default: gemv_body<WT, NS, 0, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
        }
    } else {
        switch (P.cb) {
            case 4: gemv_body<WT, NS, 4, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
            case 8: gemv_body<WT, NS, 8, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
            default: gemv_body<WT, NS, 0, NARROW>(p, P, rd, xs, sh, tid, u0, u1, ts, tag); break;
        }
    }
    if (tb >= 0) p.trace[tb + 5] = (unsigned long long)rd.waited;
}

// Tagged buffers and tags of an attention phase.
struct AttnLL {
    const unsigned long long* qkv;  // [Nq D | Nkv D | Nkv D], written by the Q|K|V phase (tag tin)
    unsigned long long* part;       // split partials [Nkv][splits][G][D + 2]
    unsigned long long* out;        // [Nq D]
    unsigned tin, tag;
};

__device__ void attention_slice_merge(const AttnArgs& a, const AttnLL& ll, int kvh, int split, int active, float* sm,
                                      int tid, const LLWait& wt);

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
__device__ void attention_item_bulk(const AttnArgs& a, const AttnLL& ll, int kvh, int split, int pos, float* sm,
                                    MegaShared& sh, int tid, uint32_t& xphase, unsigned* err, unsigned long long* tr,
                                    long long tb, const LLWait& wt) {
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

    const float* kbase = a.k_cache + (size_t)kvh * a.max_seq * D;
    const float* vbase = a.v_cache + (size_t)kvh * a.max_seq * D;
    const uint32_t row_bytes = (uint32_t)D * 4u;

    // first round: the RoPE row and the first K/V tile by bulk copy, while
    // the threads read the tagged q rows and new K/V rows as they land
    // (the cached rows were written by generic stores of earlier steps; the
    // proxy fence after the step's acquire orders them before these copies)
    int t0 = c0, tl = min(T, c1 - c0);
    if (tid == 0) {
        const uint32_t bytes = row_bytes + 2u * (uint32_t)tl * row_bytes;
        mbar_arrive_expect_tx(&sh.xbar, bytes);
        bulk_g2s_plain(rope, a.rope + (size_t)pos * half, row_bytes, &sh.xbar);
        bulk_g2s_plain(kt, kbase + (size_t)t0 * D, (uint32_t)tl * row_bytes, &sh.xbar);
        bulk_g2s_plain(vt, vbase + (size_t)t0 * D, (uint32_t)tl * row_bytes, &sh.xbar);
    }
    // the group's q rows and (last split) the new K and V rows, in one round
    const int nn = owns_new ? D : 0;
    ll_read_segs(LLSeg{ll.qkv + (size_t)kvh * G * D, qs, G * D},
                 LLSeg{ll.qkv + (size_t)a.nq * D + (size_t)kvh * D, knew, nn},
                 LLSeg{ll.qkv + (size_t)(a.nq + a.nkv) * D + (size_t)kvh * D, vnew, nn}, ll.tin, tid, wt);
    mega_wait(&sh.xbar, xphase & 1u, &sh.abort, err);
    ++xphase;
    named_sync(1, kMegaConsumers);
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
    mark(7);

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
        if (t0 == c0) mark(8);
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
                unsigned long long* o = ll.out + ((size_t)kvh * G + warp + j * NW) * D;
#pragma unroll
                for (int i = 0; i < MAXDL; ++i)
                    if (lane + 32 * i < D) st_ll(o + lane + 32 * i, o_run[j][i] * inv, ll.tag);
            }
        }
        return;
    }
    // partial (m, l, o) of each head, tagged; every split then merges its
    // slice of the head group's output (attention_slice_merge)
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
        if (hv[j]) {
            unsigned long long* pp = ll.part + (((size_t)kvh * a.splits + split) * G + warp + j * NW) * (D + 2);
            if (lane == 0) {
                st_ll(pp, m_run[j], ll.tag);
                st_ll(pp + 1, l_run[j], ll.tag);
            }
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (lane + 32 * i < D) st_ll(pp + 2 + lane + 32 * i, o_run[j][i], ll.tag);
        }
    }
}

// The flash-decoding merge of KV head kvh's active splits, shared by the
// splits: split `split` forms output elements [G D split / active, G D
// (split + 1) / active) of the head group, out = sum_s w_s o_s / sum_s w_s
// l_s with w_s = exp(m_s - M), reading the tagged partials as they land (no
// ticket, no single merging CTA).  Each thread owns an element and issues
// the loads of its kMergeChunk splits' values before the weights are known;
// each warp forms the weights of a head of the slice (lanes over splits)
// in shared memory after the item's scratch.  Sums run over the splits in
// order, so results do not depend on timing.
__device__ void attention_slice_merge(const AttnArgs& a, const AttnLL& ll, int kvh, int split, int active, float* sm,
                                      int tid, const LLWait& wt) {
    constexpr int NW = kMegaConsumers / 32;
    constexpr int SC = kMergeChunk;
    const int warp = tid >> 5, lane = tid & 31;
    const int D = a.D, G = a.nq / a.nkv, S = a.splits;
    const int nout = G * D;
    const int e0 = (int)((long long)nout * split / active), e1 = (int)((long long)nout * (split + 1) / active);
    const int h0 = e0 / D, h1 = (e1 - 1) / D;
    const size_t sstride = (size_t)G * (D + 2);
    const unsigned long long* pk = ll.part + (size_t)kvh * S * sstride;
    float* wtab = sm + attn_bulk_smem_floats(G, D);  // [G][S] split weights
    float* linv = wtab + (size_t)G * S;               // [G] 1 / sum_s w_s l_s

    unsigned long long ow[SC];
    auto issue = [&](int e, int c0) {
        const int h = e / D, d = e - h * D;
#pragma unroll
        for (int q = 0; q < SC; ++q)
            if (c0 + q < active) ow[q] = ld_ll1<false>(pk + (c0 + q) * sstride + (size_t)h * (D + 2) + 2 + d);
    };
    if (e0 + tid < e1) issue(e0 + tid, 0);

    for (int h = h0 + warp; h <= h1; h += NW) {
        const unsigned long long* ph = pk + (size_t)h * (D + 2);
        unsigned long long mw[kMergeRounds], lw[kMergeRounds];
#pragma unroll
        for (int r = 0; r < kMergeRounds; ++r) {
            const int s = lane + 32 * r;
            if (s < active) {
                mw[r] = ld_ll1<false>(ph + s * sstride);
                lw[r] = ld_ll1<false>(ph + s * sstride + 1);
            }
        }
        const int nr = active > lane ? (active - lane + 31) / 32 : 0;  // this lane's rounds
        ll_poll<kMergeRounds, false>(mw, nr, [&](int r) { return ph + (lane + 32 * r) * sstride; }, ll.tag, wt);
        ll_poll<kMergeRounds, false>(lw, nr, [&](int r) { return ph + (lane + 32 * r) * sstride + 1; }, ll.tag, wt);
        float mr[kMergeRounds], lr[kMergeRounds];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMergeRounds; ++r) {
            mr[r] = r < nr ? ll_val(mw[r]) : -INFINITY;
            lr[r] = r < nr ? ll_val(lw[r]) : 0.0f;
            M = fmaxf(M, mr[r]);
        }
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

    for (int e = e0 + tid; e < e1; e += kMegaConsumers) {
        const int h = e / D, d = e - h * D;
        float acc = 0.0f;
        for (int c0 = 0; c0 < active; c0 += SC) {
            if (e != e0 + tid || c0 != 0) issue(e, c0);
            ll_poll<SC, false>(ow, active - c0,
                               [&](int q) { return pk + (c0 + q) * sstride + (size_t)h * (D + 2) + 2 + d; }, ll.tag,
                               wt);
#pragma unroll
            for (int q = 0; q < SC; ++q)
                if (c0 + q < active) acc = fmaf(ll_val(ow[q]), wtab[h * S + c0 + q], acc);
        }
        st_ll(ll.out + (size_t)kvh * nout + e, acc * linv[h], ll.tag);
    }
}

__device__ void attention_phase(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid, long long tb,
                                uint32_t& xphase, int pos, unsigned ts, unsigned tag) {
    if (pos < 0 || pos >= p.attn.max_seq) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(p.err, kErrPosition);
        return;
    }
    AttnArgs a = p.attn;
    a.k_cache = P.kc;
    a.v_cache = P.vc;
    const AttnLL ll{p.ll_qkv, p.ll_part, p.ll_attn, ts + (unsigned)P.x_ph, tag};
    const LLWait wt{p.err, &sh.abort};
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
        attention_item_bulk(a, ll, kvh, split, pos, xs, sh, tid, xphase, p.err, p.trace, tb, wt);
    }
    // every partial of this CTA is stored before it waits on other splits'
    if (active > 1) {
        for (int it = blockIdx.x; it < items; it += gridDim.x) {
            const int kvh = it / a.splits, split = it % a.splits;
            if (split >= active) continue;
            named_sync(1, kMegaConsumers);
            if (tb >= 0) p.trace[tb + 5] = global_ns();
            attention_slice_merge(a, ll, kvh, split, active, xs, tid, wt);
            if (tb >= 0) p.trace[tb + 6] = global_ns();
        }
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
    const int depth = p.stream_depth > 0 && p.stream_depth < slots ? p.stream_depth : slots;
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
        // at most `depth` slots in flight: slot sl - depth must have landed
        // (its full barrier is not re-armed before slot sl - depth + slots)
        if (depth < slots && sl >= (uint32_t)depth) {
            const uint32_t q = sl - (uint32_t)depth;
            if (!mega_wait(&full[q % (uint32_t)slots], (q / (uint32_t)slots) & 1u, abort, p.err)) {
                ok = false;
                break;
            }
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

// NARROW: the instantiation for plans with rows narrower than a slot other
// than the widths 2048 and 4096 (tensor-parallel shards, small models): it
// adds register-resident inputs for rows of 512 and 1024 columns and the
// slots holding several row ends (batch_rows).  The plain instantiation
// goes without them, so their code and registers do not weigh on the other
// plans' loops.
template <typename WT, bool NARROW>
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
            mbar_init(&empty[s], kTeamWarps);  // released by the owning team's warps
        }
        mbar_init(&sh.xbar, 1);
        mbar_init(&sh.pbar, 1);
        mbar_fence_init();
        sP[0] = p.phases[0];
        sP[1] = p.phases[p.nphases > 1 ? 1 : 0];
        sh.abort = 0;
        s_wait_cycles = p.wait_cycles;
    }
    __syncthreads();

    if (warp >= kProducerWarp) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
        if (warp == kProducerWarp && lane == 0) produce<WT>(p, ring, full, empty, sh);
        return;
    }
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));

    RingPos rp{0, 0u};
    uint32_t xphase = 0, pphase = 0;
    int cur = 0;
    long long n = 0;  // phases started so far
    const long long total = (long long)p.steps * p.nphases;
    const unsigned long long* stw = reinterpret_cast<const unsigned long long*>(p.state);
    // the first step's (token, position): launch parameters, or the state
    // a previous launch or kernel left
    const unsigned long long st0 =
        p.init_pos >= 0 ? ((unsigned long long)(unsigned)p.init_token | ((unsigned long long)(unsigned)p.init_pos << 32))
                        : ld_acquire64(stw);
    if (p.init_pos >= 0 && blockIdx.x == 0 && tid == 0) {
        // the state the LM-head phase reads and advances; ordered before its
        // reads through the argmax ticket every CTA takes
        p.state[0] = p.init_token;
        p.state[1] = p.init_pos;
        p.state[2] = 0;
    }
    const int pos0 = (int)(unsigned)(st0 >> 32);
    for (int step = 0; step < p.steps; ++step) {
        // this step's token and position: published (release) by the last
        // CTA of the previous step's LM-head phase; acquiring them also makes
        // that step's KV-cache rows visible
        unsigned long long st = st0;
        if (step > 0) {
            st = ld_acquire64(stw);
            const long long t0 = clock64();
            unsigned spins = 0;
            const LLWait wt{p.err, &sh.abort};
            while ((int)(unsigned)(st >> 32) != pos0 + step && !wt.give_up(t0, spins)) st = ld_acquire64(stw);
        }
        const int tok = (int)(unsigned)(st & 0xffffffffull), pos = (int)(unsigned)(st >> 32);
        // the KV-cache rows of earlier steps (generic stores, made visible by
        // the acquire) before this step's bulk copies of them: thread 0
        // issues every attention copy of the CTA
        if (tid == 0) fence_proxy_async_global();
        // read after the first phase's opening barrier, so no thread of the
        // previous step still uses the old key
        if (tid == 0) sh.skey = infernt_stream_key(p.sample_seed, (uint64_t)(unsigned)pos);
        const unsigned ts = p.tag_base + (unsigned)step * (unsigned)p.nphases + 1u;  // tag of phase 0
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
            const unsigned tag = ts + (unsigned)ph;
            // every consumer thread takes the same branches here (no branch on the
            // abort flag, which the producer may set at any moment): the phases
            // contain named barriers
            if (P.kind == kPhAttn) {
                attention_phase(p, P, xs, sh, tid, tb, xphase, pos, ts, tag);
            } else if (P.ns == 2) {
                gemv_phase<WT, 2, NARROW>(p, P, ring, full, empty, rp, xphase, xs, sh, tid, tb, tok, pos, ts, tag);
            } else {
                gemv_phase<WT, 1, NARROW>(p, P, ring, full, empty, rp, xphase, xs, sh, tid, tb, tok, pos, ts, tag);
            }
            trace_mark(p, tb, 2);
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

// Both instantiations of a weight type (the plan's limits hold for either).
std::array<const void*, 2> mega_kernels(int weight_dtype) {
    if (weight_dtype == INFERNT_DTYPE_BF16)
        return {reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16, false>),
                reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16, true>)};
    return {reinterpret_cast<const void*>(decode_mega_kernel<float, false>),
            reinterpret_cast<const void*>(decode_mega_kernel<float, true>)};
}

int mega_smem_bytes(int ring_slots, int x_floats) {
    return ring_slots * kMegaSlot + x_floats * 4 + 2 * ring_slots * 8;
}

int mega_max_ring_slots() { return kMaxRingSlots; }

int mega_static_smem(int weight_dtype) {
    int most = 0;
    for (const void* k : mega_kernels(weight_dtype)) {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) {
            cudaGetLastError();
            return 48 * 1024;
        }
        if ((int)fa.sharedSizeBytes > most) most = (int)fa.sharedSizeBytes;
    }
    return most;
}

cudaError_t mega_prepare() {
    // the register split assumes the launch holds kLaunchRegs per thread: a
    // build that allocated fewer could not satisfy setmaxnreg.inc, so it is
    // refused here rather than launched
    for (const void* k : {reinterpret_cast<const void*>(decode_mega_kernel<float, false>),
                          reinterpret_cast<const void*>(decode_mega_kernel<float, true>),
                          reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16, false>),
                          reinterpret_cast<const void*>(decode_mega_kernel<__nv_bfloat16, true>)}) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, k);
        if (e != cudaSuccess) return e;
        if (fa.numRegs * kMegaThreads < 2 * 128 * kConsumerRegs + 128 * kProducerRegs)
            return cudaErrorInvalidKernelImage;
        e = raise_dynamic_smem_limit(k);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int mega_occupancy(int weight_dtype, int smem_bytes) {
    int least = 1 << 30;
    for (const void* k : mega_kernels(weight_dtype)) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kMegaThreads, smem_bytes) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        if (n < least) least = n;
    }
    return least;
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
    if (weight_dtype == INFERNT_DTYPE_BF16)
        return p.narrow ? cudaLaunchKernelEx(&cfg, decode_mega_kernel<__nv_bfloat16, true>, p)
                        : cudaLaunchKernelEx(&cfg, decode_mega_kernel<__nv_bfloat16, false>, p);
    return p.narrow ? cudaLaunchKernelEx(&cfg, decode_mega_kernel<float, true>, p)
                    : cudaLaunchKernelEx(&cfg, decode_mega_kernel<float, false>, p);
}

}  // namespace infernt
