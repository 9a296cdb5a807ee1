// bgemm.cu — the projections of batched decode on the 5th-generation tensor
// cores: Y[t][n] = sum_k X[t][k] W[n][k] for T tokens (a batch of decoding
// sequences) and row-major bf16 weights W[N][K], FP32 accumulation.
//
// The weights are the MMA's A operand (M = 128 output rows per tile, K-major
// as stored) and the tokens its B operand (N = T padded to 16, K-major), so a
// tile's accumulator is D[128 rows][T] FP32 in tensor memory.  Decode is
// weight-bandwidth bound (2 T FLOP per weight element), so every SM must
// stream weights: the K range of a row tile is split over `splits` CTAs, each
// writing its partial D to part[split][t][n]; the consumer of the projection
// adds the partials in split order (deterministic).
//
// Per CTA (128 threads): thread 0 of warp 0 drives TMA (tiled 2-D loads of a
// [128 x 64] weight box and a [T x 64] token box per stage, 128-byte swizzle,
// into a ring of kStages stages with full / empty mbarriers); thread 0 of warp
// 1 issues tcgen05.mma (kind::f16, bf16 x bf16 -> FP32, four K = 16 steps per
// stage) and frees each stage with tcgen05.commit; after the last stage's
// commit all four warps read their 32 accumulator lanes with tcgen05.ld and
// store the partial.  Every wait is bounded; on expiry the kernel sets bit 0
// of *err and returns after its copies have landed.  Launched with
// programmatic dependent launch: the weight boxes of the first stages are
// requested before the kernel waits for the previous one (griddepcontrol),
// so the weight stream overlaps the previous kernel's tail.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "../../include/infernt_seed.h"
#include "common.cuh"
#include "internal.h"

namespace infernt {
namespace {

constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kBK = 64;         // K per stage: one 128-byte swizzle row of bf16
constexpr int kStages = 6;       // most stages (fewer for large token counts)
constexpr int kSmemLimit = 225 * 1024;  // dynamic shared memory (the static part stays below 2 KB)
constexpr int kThreads = 128;
constexpr int kMaxTokens = 256;  // MMA N limit
constexpr uint32_t kTileW = kBM * kBK * 2;  // 16 KB
constexpr long long kWaitCycles = 2000000000ll;

struct BgemmArgs {
    float* part;      // [splits][T][N]
    unsigned* err;    // bit 0: a wait timed out (may be NULL)
    int N, K, T, tp, splits, stages;
};

__device__ __forceinline__ bool bg_wait(uint64_t* bar, uint32_t parity, bool& ok) {
    if (!ok) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            ok = false;
            return false;
        }
    }
    return true;
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 128 bytes, 8-row swizzle atoms of 1024 bytes (stride byte offset),
// descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3fffu);      // start address
    d |= (uint64_t)1u << 16;                          // leading byte offset (unused with swizzle)
    d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1u << 46;                          // version
    d |= (uint64_t)2u << 61;                          // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor: D FP32, A and B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t bf16_idesc(int n) {
    return (1u << 4)                      // D format F32
           | (1u << 7)                    // A format BF16
           | (1u << 10)                   // B format BF16
           | ((uint32_t)(n >> 3) << 17)   // N / 8
           | ((uint32_t)(kBM >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__global__ void __launch_bounds__(kThreads, 2)
    bgemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, BgemmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ uint64_t full[kStages], empty[kStages], done;
    __shared__ uint32_t tmem_base;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // 1024-byte aligned stages: [W tile | X tile]
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t tile_x = (uint32_t)a.tp * kBK * 2;
    const uint32_t stage_bytes = kTileW + tile_x;

    const int tiles_n = a.N / kBM;
    const int tile = blockIdx.x / a.splits, split = blockIdx.x % a.splits;
    const int n0 = tile * kBM;
    const int nk = a.K / kBK;
    const int k0 = (int)((long long)nk * split / a.splits), k1 = (int)((long long)nk * (split + 1) / a.splits);
    const int cols = a.tp < 32 ? 32 : (a.tp <= 32 ? 32 : (a.tp <= 64 ? 64 : (a.tp <= 128 ? 128 : 256)));
    (void)tiles_n;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        mbar_fence_init();
        s_ok = 1;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    bool ok = true;
    pdl_launch_dependents();
    if (warp == 0 && lane == 0) {
        // producer: the weight boxes of the first stages do not depend on the
        // previous kernel, so they are requested before waiting for it
        // (programmatic dependent launch); the token boxes after
        const int first = (k1 - k0) < a.stages ? (k1 - k0) : a.stages;
        for (int j = 0; j < first; ++j) {
            mbar_arrive_expect_tx(&full[j], stage_bytes);
            tma_load_2d(smem + (size_t)j * stage_bytes, &tm_w, (k0 + j) * kBK, n0, &full[j]);
        }
        pdl_wait();
        for (int j = 0; j < first; ++j)
            tma_load_2d(smem + (size_t)j * stage_bytes + kTileW, &tm_x, (k0 + j) * kBK, 0, &full[j]);
        for (int i = k0 + first; i < k1; ++i) {
            const int j = i - k0, s = j % a.stages;
            if (!bg_wait(&empty[s], ((j / a.stages) - 1) & 1u, ok)) break;
            unsigned char* st = smem + (size_t)s * stage_bytes;
            mbar_arrive_expect_tx(&full[s], stage_bytes);
            tma_load_2d(st, &tm_w, i * kBK, n0, &full[s]);
            tma_load_2d(st + kTileW, &tm_x, i * kBK, 0, &full[s]);
        }
        if (!ok) atomicExch(&s_ok, 0);
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        const uint32_t idesc = bf16_idesc(a.tp);
        for (int i = k0; i < k1; ++i) {
            const int j = i - k0, s = j % a.stages;
            if (!bg_wait(&full[s], (j / a.stages) & 1u, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t wa = smem_addr(smem + (size_t)s * stage_bytes);
            const uint64_t da = sw128_desc(wa), db = sw128_desc(wa + kTileW);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
                // K = 16 bf16 = 32 bytes further along the swizzled rows
                const uint64_t adv = (uint64_t)((kk * 32) >> 4);
                const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
                    "l"(da + adv), "l"(db + adv), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
            }
            // the stage is free once these MMAs have read it
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(&empty[s]))
                         : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_addr(&done))
                     : "memory");
        if (!ok) atomicExch(&s_ok, 0);
    }
    __syncwarp();
    // epilogue: every thread waits for the accumulator, then warp w reads
    // lanes [32 w, 32 w + 32) = output rows n0 + 32 w + lane
    bool eok = true;
    bg_wait(&done, 0u, eok);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int n = n0 + warp * 32 + lane;
    float* out = a.part + (size_t)split * a.T * a.N;
    for (int c = 0; c < a.tp; c += 16) {
        uint32_t r[16];
        const uint32_t addr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(addr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int q = 0; q < 16; ++q)
            if (c + q < a.T) out[(size_t)(c + q) * a.N + n] = __uint_as_float(r[q]);
    }
    if (!eok) atomicExch(&s_ok, 0);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (!s_ok) {
        if (tid == 0 && a.err) atomicOr(a.err, 1u);
        // copies still in flight into shared memory land before the CTA exits
        const long long t0 = clock64();
        while (clock64() - t0 < 20000000ll) __nanosleep(1000);
    }
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols));
}

// ---------------------------------------------------------------- prefill
// Y[t][n] = sum_k X[t][k] W[n][k] for a prompt chunk of T tokens: a dense
// contraction (2 x 128 x 256 FLOP per pair of 16 KB weight and 32 KB token
// boxes), so every tile keeps its whole K range in tensor memory.  One CTA
// per (128 weight rows, tp tokens) tile, tp = 256 (fewer for a short
// chunk); the token tile varies fastest along the grid, so the CTAs that
// share a weight tile run in the same wave and the weights cross HBM once
// per chunk while the chunk's token tiles stay in L2.  The same roles as
// bgemm_kernel: one thread drives TMA into a ring of stages, one issues
// tcgen05.mma (M = 128, N = tp, K = 16 per instruction) and frees stages with
// tcgen05.commit, then four warps read the accumulator with tcgen05.ld and
// store FP32 rows of Y (ldy floats apart).
//
// SWIGLU: W is the stacked [gate; up] matrix [2 N][K]; a tile loads the
// gate rows [n0, n0 + 128) and the up rows [N + n0, ..) per stage into two
// accumulators (2 tp TMEM columns) and its epilogue stores
// act[t][n] = bf16(silu(gate) up) (cuda/activation.cu:7-9; the rounding of
// bt_swiglu), so the FP32 gate/up rows never reach memory.
constexpr int kPStagesMax = 8;

struct PgemmArgs {
    float* y;           // FP32 output (plain)
    uint16_t* act;      // bf16 output (SWIGLU)
    unsigned* err;
    int N, K, T, tp, tiles_t, ldy, stages;
};

__device__ __forceinline__ uint16_t pg_bf16_bits(float v) {
    return (uint16_t)(__float_as_uint(infernt_round_bf16(v)) >> 16);
}

template <bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 2)
    pgemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, PgemmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ uint64_t full[kPStagesMax], empty[kPStagesMax], done;
    __shared__ uint32_t tmem_base;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t kW = SWIGLU ? 2 * kTileW : kTileW;  // weight bytes per stage
    const uint32_t stage_bytes = kW + (uint32_t)a.tp * kBK * 2;
    const int tile_t = blockIdx.x % a.tiles_t, tile_n = blockIdx.x / a.tiles_t;
    const int n0 = tile_n * kBM, t0 = tile_t * a.tp;
    const int nk = a.K / kBK;
    const int acc_cols = a.tp <= 32 ? 32 : (a.tp <= 64 ? 64 : (a.tp <= 128 ? 128 : 256));
    const int cols = SWIGLU ? 2 * acc_cols : acc_cols;

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        mbar_fence_init();
        s_ok = 1;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    bool ok = true;
    if (warp == 0 && lane == 0) {
        for (int i = 0; i < nk; ++i) {
            const int s = i % a.stages;
            if (i >= a.stages && !bg_wait(&empty[s], ((i / a.stages) - 1) & 1u, ok)) break;
            unsigned char* st = smem + (size_t)s * stage_bytes;
            mbar_arrive_expect_tx(&full[s], stage_bytes);
            tma_load_2d(st, &tm_w, i * kBK, n0, &full[s]);
            if (SWIGLU) tma_load_2d(st + kTileW, &tm_w, i * kBK, a.N + n0, &full[s]);
            tma_load_2d(st + kW, &tm_x, i * kBK, t0, &full[s]);
        }
        if (!ok) atomicExch(&s_ok, 0);
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = bf16_idesc(a.tp);
        for (int i = 0; i < nk; ++i) {
            const int s = i % a.stages;
            if (!bg_wait(&full[s], (i / a.stages) & 1u, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t wa = smem_addr(smem + (size_t)s * stage_bytes);
            const uint64_t da = sw128_desc(wa), db = sw128_desc(wa + kW), du = sw128_desc(wa + kTileW);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
                const uint64_t adv = (uint64_t)((kk * 32) >> 4);
                const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
                    "l"(da + adv), "l"(db + adv), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
                if (SWIGLU)
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
                            tmem + (uint32_t)acc_cols),
                        "l"(du + adv), "l"(db + adv), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(&empty[s]))
                         : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_addr(&done))
                     : "memory");
        if (!ok) atomicExch(&s_ok, 0);
    }
    __syncwarp();
    bool eok = true;
    bg_wait(&done, 0u, eok);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int n = n0 + warp * 32 + lane;
    const int tn = a.T - t0 < a.tp ? a.T - t0 : a.tp;  // tokens of this tile
    auto ld16 = [&](uint32_t addr, uint32_t (&r)[16]) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(addr));
    };
    for (int c = 0; c < tn; c += 16) {
        uint32_t r[16];
        const uint32_t addr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c;
        ld16(addr, r);
        if (SWIGLU) {
            uint32_t u[16];
            ld16(addr + (uint32_t)acc_cols, u);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            uint16_t* ac = a.act + (size_t)(t0 + c) * a.ldy + n;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                if (c + q < tn)
                    ac[(size_t)q * a.ldy] = pg_bf16_bits(silu_mul(__uint_as_float(r[q]), __uint_as_float(u[q])));
        } else {
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            float* yc = a.y + (size_t)(t0 + c) * a.ldy + n;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                if (c + q < tn) yc[(size_t)q * a.ldy] = __uint_as_float(r[q]);
        }
    }
    if (!eok) atomicExch(&s_ok, 0);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (!s_ok) {
        if (tid == 0 && a.err) atomicOr(a.err, 1u);
        const long long tw = clock64();
        while (clock64() - tw < 20000000ll) __nanosleep(1000);
    }
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols));
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// A [rows][K] bf16 row-major matrix as 2-D boxes of [box_rows][64].
int make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    auto fn = encode_fn();
    INFERNT_REQUIRE(fn, "bgemm: cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    INFERNT_REQUIRE(r == CUDA_SUCCESS, "bgemm: tensor map encoding failed (%d)", (int)r);
    return INFERNT_OK;
}

}  // namespace

// The cuTensorMapEncodeTiled entry point for other kernels' tensor maps
// (NULL if the driver has none).
void* tensor_map_encoder() { return reinterpret_cast<void*>(encode_fn()); }

// Two CTAs share an SM when at least kPairStages stages fit in half of its
// shared memory (their weight streams and epilogues then overlap); otherwise
// one CTA per SM with as many stages as fit.
constexpr int kPairSmem = 112 * 1024;
constexpr int kPairStages = 3;

int bgemm_ctas_per_sm(int tp) {
    const int per = kTileW + tp * kBK * 2;
    return (kPairSmem - 1024) / per >= kPairStages ? 2 : 1;
}

int bgemm_stages(int tp) {
    const int per = kTileW + tp * kBK * 2;
    const int n = ((bgemm_ctas_per_sm(tp) == 2 ? kPairSmem : kSmemLimit) - 1024) / per;
    return n < kStages ? n : kStages;
}

int bgemm_smem_bytes(int tp) { return bgemm_stages(tp) * (kTileW + tp * kBK * 2) + 1024; }

// Host side of one batched projection (plan code calls this with maps it
// built once; the C entry point builds them per call).
int bgemm_launch(const void* W, int N, int K, const void* X, int T, float* part, int splits, unsigned* err,
                 cudaStream_t st) {
    INFERNT_REQUIRE(W && X && part, "bgemm: null pointer");
    INFERNT_REQUIRE(N > 0 && N % kBM == 0, "bgemm: N = %d must be a positive multiple of %d", N, kBM);
    INFERNT_REQUIRE(K > 0 && K % kBK == 0, "bgemm: K = %d must be a positive multiple of %d", K, kBK);
    INFERNT_REQUIRE(T >= 1 && T <= kMaxTokens, "bgemm: T = %d outside [1, %d]", T, kMaxTokens);
    INFERNT_REQUIRE(splits >= 1 && splits <= K / kBK, "bgemm: splits = %d outside [1, K / %d]", splits, kBK);
    INFERNT_REQUIRE(aligned16(W) && aligned16(X), "bgemm: W and X must be 16-byte aligned");
    const int tp = (T + 15) / 16 * 16;
    CUtensorMap mw, mx;
    if (int s = make_map(&mw, W, N, K, kBM)) return s;
    if (int s = make_map(&mx, X, T, K, tp)) return s;
    const int smem = bgemm_smem_bytes(tp);
    static bool raised = false;
    if (!raised) {
        INFERNT_CUDA_TRY(cudaFuncSetAttribute(bgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
        raised = true;
    }
    BgemmArgs args;
    args.part = part;
    args.err = err;
    args.N = N;
    args.K = K;
    args.T = T;
    args.tp = tp;
    args.splits = splits;
    args.stages = bgemm_stages(tp);
    // programmatic dependent launch: the CTAs may start (and fetch their
    // first weight boxes) while the previous kernel of the stream finishes
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((N / kBM) * splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    INFERNT_CUDA_TRY(cudaLaunchKernelEx(&cfg, bgemm_kernel, mw, mx, args));
    return INFERNT_OK;
}

// Host side of one prefill projection: Y [T][ldy] FP32 (columns [0, N)) =
// X [T][K] bf16 times W [N][K] bf16 transposed; any T >= 1.
namespace {

// One prefill projection: plain (Y FP32 [T][ldy], W [N][K]) or SWIGLU (act
// bf16 [T][ldy], W the stacked [gate; up] matrix [2 N][K]).
int pgemm_run(bool swiglu, const void* W, int N, int K, const void* X, int T, float* Y, uint16_t* act, int ldy,
              unsigned* err, cudaStream_t st) {
    INFERNT_REQUIRE(W && X && (swiglu ? (const void*)act : (const void*)Y), "pgemm: null pointer");
    INFERNT_REQUIRE(N > 0 && N % kBM == 0, "pgemm: N = %d must be a positive multiple of %d", N, kBM);
    INFERNT_REQUIRE(K > 0 && K % kBK == 0, "pgemm: K = %d must be a positive multiple of %d", K, kBK);
    INFERNT_REQUIRE(T >= 1, "pgemm: T = %d", T);
    INFERNT_REQUIRE(ldy >= N, "pgemm: ldy = %d below N = %d", ldy, N);
    INFERNT_REQUIRE(aligned16(W) && aligned16(X), "pgemm: W and X must be 16-byte aligned");
    // two CTAs per SM, two 48 KB stages each: one CTA's epilogue (tcgen05.ld
    // and stores) and pipeline fill run under the other's MMAs; the SwiGLU
    // variant takes 128 tokens per tile so its two accumulators fit in half
    // of the tensor memory
    const int tmax = swiglu ? 128 : kMaxTokens;
    const int tp = T >= tmax ? tmax : (T + 15) / 16 * 16;
    const int tiles_t = (T + tp - 1) / tp;
    const long long ctas = (long long)(N / kBM) * tiles_t;
    INFERNT_REQUIRE(ctas < (1ll << 31), "pgemm: %lld tiles", ctas);
    const int per = (swiglu ? 2 : 1) * kTileW + tp * kBK * 2;
    int stages = (kSmemLimit / 2 - 1024 - 1024) / per;  // half of the SM per CTA (static part included)
    if (stages < 2) stages = 2;
    if (stages > kPStagesMax) stages = kPStagesMax;
    CUtensorMap mw, mx;
    if (int s = make_map(&mw, W, swiglu ? 2 * N : N, K, kBM)) return s;
    if (int s = make_map(&mx, X, T, K, tp)) return s;
    // per launch: the attribute belongs to the current device
    if (swiglu)
        INFERNT_CUDA_TRY(cudaFuncSetAttribute(pgemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    else
        INFERNT_CUDA_TRY(
            cudaFuncSetAttribute(pgemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    PgemmArgs args;
    args.y = Y;
    args.act = act;
    args.err = err;
    args.N = N;
    args.K = K;
    args.T = T;
    args.tp = tp;
    args.tiles_t = tiles_t;
    args.ldy = ldy;
    args.stages = stages;
    if (swiglu)
        pgemm_kernel<true><<<(unsigned)ctas, kThreads, stages * per + 1024, st>>>(mw, mx, args);
    else
        pgemm_kernel<false><<<(unsigned)ctas, kThreads, stages * per + 1024, st>>>(mw, mx, args);
    INFERNT_CUDA_TRY(cudaGetLastError());
    return INFERNT_OK;
}

}  // namespace

int pgemm_launch(const void* W, int N, int K, const void* X, int T, float* Y, int ldy, unsigned* err,
                 cudaStream_t st) {
    return pgemm_run(false, W, N, K, X, T, Y, nullptr, ldy, err, st);
}

// act [T][ldy] bf16 = silu(X W_gate^T) (X W_up^T) for the stacked W_gu [2 I][K].
int pgemm_swiglu_launch(const void* W_gu, int I, int K, const void* X, int T, uint16_t* act, int ldy, unsigned* err,
                        cudaStream_t st) {
    return pgemm_run(true, W_gu, I, K, X, T, nullptr, act, ldy, err, st);
}

}  // namespace infernt

extern "C" int infernt_bgemm_bf16(const void* W, int N, int K, const void* X, int T, float* partials, int splits,
                                  unsigned* err, void* stream) {
    return infernt::bgemm_launch(W, N, K, X, T, partials, splits, err, static_cast<cudaStream_t>(stream));
}

extern "C" int infernt_pgemm_bf16(const void* W, int N, int K, const void* X, int T, float* Y, int ldy,
                                  unsigned* err, void* stream) {
    return infernt::pgemm_launch(W, N, K, X, T, Y, ldy, err, static_cast<cudaStream_t>(stream));
}

extern "C" int infernt_pgemm_swiglu_bf16(const void* W_gate_up, int I, int K, const void* X, int T, void* act,
                                         int ld_act, unsigned* err, void* stream) {
    return infernt::pgemm_swiglu_launch(W_gate_up, I, K, X, T, static_cast<uint16_t*>(act), ld_act, err,
                                        static_cast<cudaStream_t>(stream));
}
