// decode_kernel.cu — the persistent decode kernel.
//
// One CTA per SM runs every phase of a decode step (and of a chain of
// steps): per layer the fused RMSNorm + Q/K/V projection, attention (RoPE,
// KV append, split-KV GQA, merge), O projection + residual, RMSNorm +
// gate/up + SiLU, down projection + residual; then RMSNorm + LM head +
// argmax.  Phases are separated by a grid barrier among the consumer warps.
//
// Warps 0-3 consume; warp 4 produces: lanes 0-3 stream the CTA's share of
// every GEMV phase's weights, tile by tile, into a ring of 16 KB shared-
// memory slots with 2-D TMA box loads (8 KB per instruction).  Weights do
// not depend on activations, so the producer runs ahead across phase
// boundaries and layers while the consumers wait at grid barriers or compute
// attention.  Warp 5 keeps an L2 prefetch window (cp.async.bulk.prefetch
// .tensor) a fixed number of tiles ahead of the producer, so HBM keeps
// streaming for longer than the shared-memory ring alone could buffer.
//
// A GEMV phase of G row groups (R rows each, R = 8 FP32 / 16 bf16; a tile is
// one 512-column block of a group) gives CTA b the groups
// [G b / P, G (b + 1) / P): every group is reduced inside one CTA, in a
// fixed order, so results do not depend on timing and no cross-CTA merge
// sits on the critical path.
//
// Every wait (ring slots, grid barrier, prefetch pacing) is bounded by a
// clock budget; on expiry the CTA sets kErrWaitTimeout in the error word,
// marks itself aborted and runs the remaining control flow without waiting,
// so the kernel always terminates and the host reports INFERNT_ERR_DEVICE.
#include <cstring>

#include "decode_kernel.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "tensormap.h"

namespace infernt {

namespace {

constexpr int kMegaSlot = 16384;
constexpr int kMegaConsumers = 128;
constexpr int kProducerWarp = 4;
constexpr int kPrefetchWarp = 5;
constexpr int kMegaThreads = 192;  // 4 consumer warps, the producer warp, the L2 prefetch warp
constexpr long long kWaitCycles = 4000000000ll;  // about 2 s at the maximum SM clock
constexpr int kResRows = 128;                    // residual rows a CTA stages per phase

template <typename WT>
struct MegaRows {
    static constexpr int EB = WeightTraits<WT>::kBytes;
    static constexpr int R = kMegaSlot / (kPiece * EB);  // 8 FP32, 16 bf16
};

constexpr int kGroupSlots = 16;  // group hand-off slots (> ring slots, see finish_group)
constexpr int kMaxRingSlots = 14;

struct MegaShared {
    int abort;
    unsigned loaded;  // tiles the producer has issued (paces the prefetch warp)
    int producer_done;
    float ss[4];
    float amv[64];  // LM-head candidates [warp][lane < R]
    int ami[64];
    int res_base;  // first staged residual row
    int res_n;     // staged rows
    float res[kResRows];
    int gcnt[kGroupSlots];           // warps that have deposited a group's partials
    float gred[kGroupSlots][4][16];  // per-warp partial sums of a group's rows
    uint64_t xbar;                   // completion of the input-vector bulk copy
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

// Grid barrier of the consumer warps: every CTA adds 1 (release) to a 64-bit
// counter that only grows, and polls (acquire) until it reaches `target`
// (the launch's base plus gridDim.x per barrier passed).  One atomic per
// CTA, no reset and no last-arriver hop.  The named barrier orders the other
// consumer threads' writes before thread 0's release, which is cumulative,
// so no separate fence is needed.
__device__ __forceinline__ void grid_sync(const MegaParams& p, volatile int* abort, int tid,
                                          unsigned long long target) {
    named_sync(1, kMegaConsumers);
    if (tid == 0 && !*abort) {
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p.bar) : "memory");
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

// Tiles [t0, t1) of this CTA: whole row groups [G b / P, G (b + 1) / P).
__device__ __forceinline__ void phase_range(const MegaPhase& P, long long& t0, long long& t1) {
    const long long g0 = (long long)P.groups * blockIdx.x / gridDim.x;
    const long long g1 = (long long)P.groups * (blockIdx.x + 1) / gridDim.x;
    t0 = g0 * P.cb;
    t1 = g1 * P.cb;
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
// Residual phases also stage the residual rows of the CTA's row groups
// (R rows per group) in sh.res, so the epilogue needs no L2 round trip.
__device__ void load_x(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid, int R,
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
    if (tid == 0) {
        // the input vector (and the norm weights behind it) in one bulk copy
        // each, issued first so the residual loads below overlap them; the
        // vector was written by generic stores (after the grid barrier's
        // acquire), read here through the async proxy
        fence_proxy_async_global();
        const uint32_t bytes = (uint32_t)P.K * 4u;
        mbar_arrive_expect_tx(&sh.xbar, P.norm_w ? 2u * bytes : bytes);
        bulk_g2s_plain(xs, src, bytes, &sh.xbar);
        if (P.norm_w) bulk_g2s_plain(xs + P.K, P.norm_w, bytes, &sh.xbar);
    }
    int staged = 0, staged_base = 0;
    if (P.epi == kEpiResidual) {
        long long t0, t1;
        phase_range(P, t0, t1);
        if (t1 > t0) {
            const long long r0 = (t0 / P.cb) * R;
            long long r1 = (t1 / P.cb) * R;
            if (r1 > P.units) r1 = P.units;
            const int n = (int)(r1 - r0);
            if (n > 0 && n <= kResRows) {
                for (int i = tid; i < n; i += kMegaConsumers) sh.res[i] = __ldcg(P.res + r0 + i);
                staged = n;
                staged_base = (int)r0;
            }
        }
    }
    if (tid == 0) {  // one writer; read after the named barrier at the end
        sh.res_n = staged;
        sh.res_base = staged_base;
    }
    mega_wait(&sh.xbar, xphase & 1u, &sh.abort, p.err);
    ++xphase;
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

// A warp's share of a finished group: its R row sums (xor-shuffle trees)
// go to the group's hand-off slot; the fourth warp to deposit adds the four
// shares in warp order and runs the epilogue.  No CTA-wide barrier, so the
// warps keep streaming tiles.  A slot is reused kGroupSlots groups later,
// and no warp runs more than the ring's slot count of tiles (at least one
// tile per group) ahead of the slowest warp, so kGroupSlots > ring slots
// keeps a slot's readers ahead of its next writers.
template <typename WT, int NS>
__device__ __forceinline__ void finish_group(const MegaParams& p, const MegaPhase& P, long long g, const float* acc,
                             MegaShared& sh, int gslot, int tid, float& am_v, int& am_i) {
    constexpr int R = MegaRows<WT>::R;
    constexpr int BR = R / NS;
    const int warp = tid >> 5, lane = tid & 31;
    float(*slot)[16] = sh.gred[gslot];
#pragma unroll
    for (int a = 0; a < R; ++a) {
        const float v = warp_sum(acc[a]);
        if (lane == a) slot[warp][a] = v;
    }
    __threadfence_block();
    int ticket = 0;
    if (lane == 0) ticket = atomicAdd(&sh.gcnt[gslot], 1);
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != kMegaConsumers / 32 - 1) return;
    __threadfence_block();
    if (NS == 2) {
        if (lane < BR) {
            const float yg = ((slot[0][lane] + slot[1][lane]) + slot[2][lane]) + slot[3][lane];
            const int u = BR + lane;
            const float yu = ((slot[0][u] + slot[1][u]) + slot[2][u]) + slot[3][u];
            const long long unit = g * BR + lane;
            if (unit < P.units) P.out[unit] = silu_mul(yg, yu);
        }
    } else if (lane < R) {
        const float v = ((slot[0][lane] + slot[1][lane]) + slot[2][lane]) + slot[3][lane];
        int lg, rowbase;
        const int q = seg_of(P, (int)g, lg, rowbase);
        const int local = lg * R + lane;
        if (local < P.seg_rows[q]) {
            const int row = rowbase + local;
            if (P.epi == kEpiStore) {
                P.out[row] = v;
            } else if (P.epi == kEpiResidual) {
                const int ri = row - sh.res_base;
                const float r = (ri >= 0 && ri < sh.res_n) ? sh.res[ri] : __ldcg(P.res + row);
                P.out[row] = r + v;
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
    __syncwarp();
    if (lane == 0) sh.gcnt[gslot] = 0;
}

// Winner of the CTA -> partial; the last CTA reduces all partials in CTA
// order, writes the token and advances the decode state.
__device__ void argmax_phase_end(const MegaParams& p, MegaShared& sh, int tid, float am_v, int am_i, int R) {
    const int warp = tid >> 5, lane = tid & 31;
    if (lane < R) {
        sh.amv[warp * 16 + lane] = am_v;
        sh.ami[warp * 16 + lane] = am_i;
    }
    named_sync(1, kMegaConsumers);
    if (warp != 0) return;
    int last = 0;
    if (lane == 0) {
        float bv = -1e30f;
        int bi = 0;
        for (int w = 0; w < kMegaConsumers / 32; ++w)
            for (int i = 0; i < R; ++i)
                if (argmax_better(sh.amv[w * 16 + i], sh.ami[w * 16 + i], bv, bi)) {
                    bv = sh.amv[w * 16 + i];
                    bi = sh.ami[w * 16 + i];
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
                           uint64_t* empty, RingPos& rp, uint32_t& gcount, uint32_t& xphase, float* xs,
                           MegaShared& sh, int tid, long long tb, int tok) {
    constexpr int R = MegaRows<WT>::R;
    const int lane = tid & 31;
    const int slots = p.ring_slots;
    load_x(p, P, xs, sh, tid, R, xphase, tok);
    if (tid == 0) trace_mark(p, tb, 1);
    long long t0, t1;
    phase_range(P, t0, t1);
    float acc[R];
#pragma unroll
    for (int a = 0; a < R; ++a) acc[a] = 0.0f;
    float am_v = -1e30f;
    int am_i = 0;
    long long g = t0 / P.cb;
    int j = 0;
    long long waited = 0;
    for (long long t = t0; t < t1; ++t, rp.advance(slots)) {
        const int s = rp.s;
        if (tb >= 0) {
            const long long c0 = clock64();
            mega_wait(&full[s], rp.ph, &sh.abort, p.err);
            waited += clock64() - c0;
        } else {
            mega_wait(&full[s], rp.ph, &sh.abort, p.err);
        }
        const float4 xv = reinterpret_cast<const float4*>(xs + j * kPiece)[tid];
        tile_fma<WT, NS>(ring + (size_t)s * kMegaSlot, xv, tid, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++j == P.cb) {
            finish_group<WT, NS>(p, P, g, acc, sh, (int)(gcount++ % kGroupSlots), tid, am_v, am_i);
#pragma unroll
            for (int a = 0; a < R; ++a) acc[a] = 0.0f;
            j = 0;
            ++g;
        }
    }
    if (tb >= 0) p.trace[tb + 5] = (unsigned long long)waited;
    if (P.epi == kEpiArgmax) argmax_phase_end(p, sh, tid, am_v, am_i, R);
}

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
                                    int tid, uint32_t& xphase, unsigned* err) {
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

    float m_run[MAXH], l_run[MAXH], o_run[MAXH][MAXDL];
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
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
#pragma unroll
        for (int j = 0; j < MAXH; ++j) {
            const int h = warp + j * NW;
            if (h < G) {
                float s = -INFINITY;
                if (lane < tl) {
                    const float* qh = qs + h * D;
                    const float* kr = kt + lane * D;
                    float dot = 0.0f;
                    int c = cstart;
                    for (int n = 0; n < nc; ++n) {
                        const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * c);
                        const float4 q4 = *reinterpret_cast<const float4*>(qh + 4 * c);
                        dot = fmaf(q4.x, k4.x, dot);
                        dot = fmaf(q4.y, k4.y, dot);
                        dot = fmaf(q4.z, k4.z, dot);
                        dot = fmaf(q4.w, k4.w, dot);
                        if (++c == nc) c = 0;
                    }
                    s = dot * a.scale;
                }
                const float m_new = fmaxf(m_run[j], warp_max(s));
                const float alpha = expf(m_run[j] - m_new);
                const float pe = lane < tl ? expf(s - m_new) : 0.0f;
                ps[h * T + lane] = pe;
                l_run[j] = l_run[j] * alpha + warp_sum(pe);
                m_run[j] = m_new;
                __syncwarp();
#pragma unroll
                for (int i = 0; i < MAXDL; ++i) {
                    const int d = lane + 32 * i;
                    if (d < D) {
                        float acc = o_run[j][i] * alpha;
                        for (int q = 0; q < tl; ++q) acc = fmaf(ps[h * T + q], vt[q * D + d], acc);
                        o_run[j][i] = acc;
                    }
                }
            }
        }
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

    if (active == 1) {
        // the only split: normalised output (cuda/attention.cu:30-43 after softmax)
#pragma unroll
        for (int j = 0; j < MAXH; ++j) {
            const int h = warp + j * NW;
            if (h < G) {
                const float inv = 1.0f / l_run[j];
                float* o = a.out + ((size_t)kvh * G + h) * D;
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
    named_sync(1, kMegaConsumers);
    if (tid == 0) {
        // release: this CTA's partials (ordered by the named barrier) before
        // the ticket; acquire: the other splits' partials before the merge
        const unsigned ticket = atom_add_acq_rel(&a.counter[kvh], 1u);
        *s_last = (ticket == (unsigned)active - 1u);
    }
    named_sync(1, kMegaConsumers);
    if (*s_last) {
        for (int h = warp; h < G; h += NW) {
            const float* ph = a.part + ((size_t)kvh * a.splits * G + h) * (D + 2);
            const size_t sstride = (size_t)G * (D + 2);
            float M = -INFINITY;
            for (int s = lane; s < active; s += 32) M = fmaxf(M, __ldcg(ph + s * sstride));
            M = warp_max(M);
            float L = 0.0f;
            float acc[MAXDL];
#pragma unroll
            for (int i = 0; i < MAXDL; ++i) acc[i] = 0.0f;
#pragma unroll 4
            for (int s = 0; s < active; ++s) {
                const float* pp = ph + s * sstride;
                const float w = expf(__ldcg(pp) - M);
                L = fmaf(__ldcg(pp + 1), w, L);
#pragma unroll
                for (int i = 0; i < MAXDL; ++i)
                    if (lane + 32 * i < D) acc[i] = fmaf(__ldcg(pp + 2 + lane + 32 * i), w, acc[i]);
            }
            const float inv = 1.0f / L;
            float* o = a.out + ((size_t)kvh * G + h) * D;
#pragma unroll
            for (int i = 0; i < MAXDL; ++i)
                if (lane + 32 * i < D) o[lane + 32 * i] = acc[i] * inv;
        }
        if (tid == 0) a.counter[kvh] = 0u;
    }
}

__device__ void attention_phase(const MegaParams& p, const MegaPhase& P, float* xs, MegaShared& sh, int tid,
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
        attention_item_bulk(a, kvh, split, pos, xs, sh, tid, xphase, p.err);
    }
}

// ---------------------------------------------------------------- producer

// Position in a CTA's weight stream: (step, phase, tile) over the GEMV
// phases, in the order the consumers use them.  The phase's fields the
// producer needs are cached in registers when the cursor enters a phase,
// so a tile costs no global-memory reads.
struct TileCursor {
    int step, ph;
    long long t, t1;
    int g, j, cb, ns, q, lg;
    int segg[3];
    const CUtensorMap* m[3];
    bool done;

    __device__ void start(const MegaParams& p) {
        step = 0;
        ph = -1;
        done = false;
        next_phase(p);
    }
    __device__ void next_phase(const MegaParams& p) {
        while (true) {
            if (++ph == p.nphases) {
                ph = 0;
                if (++step >= p.steps) {
                    done = true;
                    return;
                }
            }
            const MegaPhase& P = p.phases[ph];
            if (P.kind != kPhGemv) continue;
            long long t0;
            phase_range(P, t0, t1);
            if (t0 == t1) continue;
            t = t0;
            cb = P.cb;
            ns = P.ns;
            g = (int)(t0 / cb);
            j = 0;
            const int nm = ns == 2 ? 2 : P.nseg;
            for (int i = 0; i < 3; ++i) {
                segg[i] = P.seg_groups[i];
                m[i] = &p.maps[P.map[i < nm ? i : 0]];
            }
            q = 0;
            lg = g;
            if (ns == 1)
                while (q < P.nseg - 1 && lg >= segg[q]) {
                    lg -= segg[q];
                    ++q;
                }
            return;
        }
    }
    __device__ __forceinline__ void next(const MegaParams& p) {
        ++t;
        if (++j == cb) {
            j = 0;
            ++g;
            if (++lg == segg[q] && ns == 1) {
                ++q;
                lg = 0;
            }
        }
        if (t == t1) next_phase(p);
    }
};

// Box `box` (0..3) of the tile at cursor c: tensor map and coordinates.
template <typename WT>
__device__ __forceinline__ const CUtensorMap* tile_box(const TileCursor& c, int box, int& x, int& y) {
    constexpr int R = MegaRows<WT>::R;
    x = c.j * kPiece + (box & 1) * kBoxCols;
    if (c.ns == 1) {
        y = c.lg * R;
        return c.m[c.q];
    }
    y = c.g * (R / 2);
    return c.m[box >> 1];
}

template <typename WT>
__device__ void produce(const MegaParams& p, unsigned char* ring, uint64_t* full, uint64_t* empty,
                        MegaShared& sh, int lane) {
    constexpr int R = MegaRows<WT>::R;
    constexpr int EB = MegaRows<WT>::EB;
    volatile int* abort = &sh.abort;
    const int slots = p.ring_slots;
    const uint64_t pol = l2_evict_first_policy();
    TileCursor ld;
    ld.start(p);
    uint32_t sl = 0;
    int ok = 1;
    RingPos wp{0, 0u};
    long long pwait = 0;  // cycles waited for free slots in the current phase (trace)
    while (!ld.done && ok) {
        const int s = wp.s;
        if (lane == 0) {
            // from the second lap on, wait until the consumers released the slot
            const long long c0 = clock64();
            if (sl >= (uint32_t)slots && !mega_wait(&empty[s], wp.ph ^ 1u, abort, p.err))
                ok = 0;
            else
                mbar_arrive_expect_tx(&full[s], kMegaSlot);
            pwait += clock64() - c0;
        }
        ok = __shfl_sync(0xFu, ok, 0);
        if (ok) {
            // ns == 1: box h at h*R rows; ns == 2: box (s2, h) at (s2*2 + h)*(R/2) rows
            const int BR = R / ld.ns;
            if (lane < (ld.ns == 1 ? 2 : 4)) {
                int x, y;
                const CUtensorMap* m = tile_box<WT>(ld, lane, x, y);
                tma_load_2d(ring + (size_t)s * kMegaSlot + (size_t)lane * BR * kBoxCols * EB, m, x, y, &full[s], pol);
            }
            const int ph_before = ld.ph, step_before = ld.step;
            ld.next(p);
            ++sl;
            wp.advance(slots);
            if (lane == 0) {
                *reinterpret_cast<volatile unsigned*>(&sh.loaded) = sl;
                if (ld.done || ld.ph != ph_before || ld.step != step_before)
                {
                    const long long tbp = trace_base(p, step_before, ph_before);
                    trace_mark(p, tbp, 4);
                    if (tbp >= 0) p.trace[tbp + 6] = (unsigned long long)pwait;
                    pwait = 0;
                }
            }
        }
        __syncwarp(0xFu);
    }
    if (lane == 0) *reinterpret_cast<volatile int*>(&sh.producer_done) = 1;
    if (!ok && lane == 0) {
        // slot sl was not armed; let the copies of every armed slot land
        // before the CTA can exit
        const uint32_t first = sl > (uint32_t)slots ? sl - slots : 0u;
        volatile int no_abort = 0;
        for (uint32_t q = first; q < sl; ++q) mega_wait(&full[q % slots], (q / slots) & 1u, &no_abort, p.err);
    }
}

// L2 prefetch window: tile n of the stream is prefetched once the producer
// has issued tile n - window.  Prefetches have no completion to wait for.
template <typename WT>
__device__ void prefetch_l2(const MegaParams& p, MegaShared& sh) {
    const int window = p.l2_prefetch_tiles;
    if (window <= 0) return;
    volatile unsigned* loaded = &sh.loaded;
    volatile int* done = &sh.producer_done;
    volatile int* abort = &sh.abort;
    TileCursor pf;
    pf.start(p);
    unsigned n = 0;
    while (!pf.done) {
        if (n >= *loaded + (unsigned)window) {
            const long long t0 = clock64();
            while (n >= *loaded + (unsigned)window) {
                if (*done || *abort || clock64() - t0 > kWaitCycles) return;
                __nanosleep(200);
            }
        }
        const int nb = pf.ns == 1 ? 2 : 4;
        for (int b = 0; b < nb; ++b) {
            int x, y;
            const CUtensorMap* m = tile_box<WT>(pf, b, x, y);
            tma_prefetch_l2_2d(m, x, y);
        }
        pf.next(p);
        ++n;
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
        sh.loaded = 0;
        sh.producer_done = 0;
        for (int i = 0; i < kGroupSlots; ++i) sh.gcnt[i] = 0;
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        if (lane < 4) produce<WT>(p, ring, full, empty, sh, lane);
        return;
    }
    if (warp == kPrefetchWarp) {
        if (lane == 0) prefetch_l2<WT>(p, sh);
        return;
    }

    RingPos rp{0, 0u};
    uint32_t gcount = 0, xphase = 0, pphase = 0;
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
            // every consumer thread takes the same branches here (no branch on the
            // abort flag, which the producer may set at any moment): the phases
            // contain named barriers
            if (P.kind == kPhAttn) {
                attention_phase(p, P, xs, sh, tid, xphase, pos);
            } else if (P.ns == 2) {
                gemv_phase<WT, 2>(p, P, ring, full, empty, rp, gcount, xphase, xs, sh, tid, tb, tok);
            } else {
                gemv_phase<WT, 1>(p, P, ring, full, empty, rp, gcount, xphase, xs, sh, tid, tb, tok);
            }
            trace_mark(p, tb, 2);
            target += gridDim.x;
            grid_sync(p, &sh.abort, tid, target);
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
