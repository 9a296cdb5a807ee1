// decode_kernel.cuh — the persistent decode kernel: argument blocks and host
// entry points (decode_kernel.cu).
#pragma once

#include "attention.cuh"

namespace infernt {

enum MegaKind : int { kPhGemv = 0, kPhAttn = 1 };

// One phase of a decode step.  A GEMV phase gives CTA b the output units
// [units b / P, units (b + 1) / P) and streams the weight rows of those units
// (contiguous in row-major memory) through the shared-memory ring in 16 KB
// slots: one to three byte ranges for a stacked Q|K|V phase, two ranges per
// batch of units for gate/up.
struct alignas(16) MegaPhase {
    int kind;           // MegaKind
    int epi;            // EpiKind (gemv.cuh)
    int ns;             // 1, or 2 for paired gate/up
    int nseg;           // matrices stacked in the row space (Q|K|V = 3); ns == 2: gate, up
    const void* w[3];   // the matrices, row-major [seg_rows][K]
    int seg_rows[3];
    int units;          // output rows (ns == 2: gate/up pairs)
    int K;              // input features, a multiple of 512
    int cb;             // K / 512
    const float* x;     // input vector; NULL: the per-launch input (layer 0)
    const float* norm_w;  // RMSNorm weight or NULL
    float eps;
    float* out;         // NULL: the per-launch logits (LM head)
    const float* res;   // residual source (out = res + y)
    float* x_copy;      // layer 0: the raw input row is copied here (residual stream)
    int layer;          // attention phases: KV-cache layer
    float* kc;          // attention phases: the layer's K and V caches [N_kv, max_seq, D]
    float* vc;
    // tensor parallelism
    int nsum;           // > 0: the input vector is x + the nsum partial vectors at xsum (rank order)
    int xch_off;        // >= 0: epilogue writes its rows to every rank's exchange region at this
                        // byte offset, slot [this rank][units]; -1: none
    const float* xsum;  // [nsum][K] partials of the previous exchange (this rank's region)
    float* xout;        // the summed input's rows [K b/P, K (b+1)/P) are written here (or NULL)
    int row_base;       // LM head: global index of the first local row (argmax ids)
    int pad_;
};
// descriptors are bulk-copied into shared memory ahead of their phase
static_assert(sizeof(MegaPhase) % 16 == 0, "MegaPhase must be a multiple of 16 bytes");

struct MegaParams {
    const MegaPhase* phases;
    int nphases;
    // per launch
    const float* input;  // NULL: embedding row of the state's token
    float* logits;
    int* hist;           // token history (chained steps) or NULL
    int steps;
    // model
    const float* emb;
    int vocab;
    AttnArgs attn;       // qkv, out, part, counter, shape, theta, scale (caches per phase)
    // scratch
    int* state;          // {token, position, step, last token}
    unsigned* err;
    unsigned long long* bar;       // grid-barrier arrivals (only ever grows)
    unsigned long long bar_base;   // its value when this launch starts
    float* am_val;       // LM-head argmax partials [gridDim]
    int* am_idx;
    unsigned* am_cnt;
    int ring_slots;
    int x_floats;        // shared floats for the input vector / attention scratch
    // tensor parallelism over tp_size GPUs (tp_size 1: none): every rank's
    // exchange region (flags at kXchFlags, argmax slots at kXchArgmax, the
    // partial buffers at the phases' xch_off), mapped into this process
    int tp_rank, tp_size;
    unsigned char* const* peers;   // [tp_size] region base pointers (own included)
    unsigned long long xe_base;    // exchange epoch before this launch's first exchange    // optional phase timeline (nanoseconds, %globaltimer): for CTA 0 and the
    // last CTA, per (step, phase): [phase start, input loaded, work done,
    // barrier passed, producer issued the phase's last slot, SM cycles
    // consumer warp 0 waited for full slots, SM cycles the producer waited
    // for free slots while issuing the phase's slots]
    unsigned long long* trace;
};

constexpr int kTraceFields = 7;

// Exchange region layout (one per rank, cudaMalloc'd, shared by IPC):
// flags [8] u64 (the last exchange epoch each rank has published), argmax
// slots [8] u64 (float value bits | index << 32), then the partial buffers.
constexpr int kMaxTp = 8;
constexpr int kXchFlags = 0;
constexpr int kXchArgmax = 256;
constexpr int kXchData = 512;

// Rows of a consumer batch: 8 FP32 / 16 bf16 (a batch is whole 16 KB slots).
inline int mega_batch_rows(int weight_dtype) { return weight_dtype == 1 ? 16 : 8; }

// Dynamic shared memory of the persistent kernel.
int mega_smem_bytes(int ring_slots, int x_floats);
// Largest ring the kernel uses.
int mega_max_ring_slots();
// Static shared memory of the kernel instantiation.
int mega_static_smem(int weight_dtype);

// Launches the cooperative persistent kernel (grid = `ctas`).
cudaError_t launch_mega(const MegaParams& p, int weight_dtype, int ctas, cudaStream_t stream);
// Raises the dynamic shared-memory limit of both instantiations.
cudaError_t mega_prepare();
// Largest CTAs-per-SM count at this shared-memory size (0: does not fit).
int mega_occupancy(int weight_dtype, int smem_bytes);

}  // namespace infernt
