// decode_kernel.cuh — the persistent decode kernel: argument blocks and host
// entry points (decode_kernel.cu).
#pragma once

#include <cuda.h>

#include "attention.cuh"

namespace infernt {

enum MegaKind : int { kPhGemv = 0, kPhAttn = 1 };

// One phase of a decode step.  GEMV phases stream their weights through the
// shared-memory ring as tiles of (R rows x 512 columns); R = 8 FP32 / 16
// bf16 (gate/up tiles carry R/2 rows of each).
struct MegaPhase {
    int kind;           // MegaKind
    int epi;            // EpiKind (gemv.cuh)
    int ns;             // 1, or 2 for paired gate/up
    int nseg;           // segments stacked in the row space (Q|K|V = 3)
    int map[3];         // tensor-map index of each segment (ns == 2: gate, up)
    int seg_groups[3];  // tile rows groups per segment (ns == 1)
    int seg_rows[3];
    int units;          // output rows (ns == 2: gate/up pairs)
    int K;              // input features, a multiple of 512
    int cb;             // K / 512
    int groups;
    long long tiles;    // groups * cb
    const float* x;     // input vector; NULL: the per-launch input (layer 0)
    const float* norm_w;  // RMSNorm weight or NULL
    float eps;
    float* out;         // NULL: the per-launch logits (LM head)
    const float* res;   // residual source (out = res + y)
    float* x_copy;      // layer 0: the raw input row is copied here (residual stream)
    int layer;          // attention phases: KV-cache layer
};

struct MegaParams {
    const MegaPhase* phases;
    int nphases;
    const CUtensorMap* maps;
    // per launch
    const float* input;  // NULL: embedding row of the state's token
    float* logits;
    int* hist;           // token history (chained steps) or NULL
    int steps;
    // model
    const float* emb;
    int vocab;
    float* const* kc;    // device array of per-layer K caches
    float* const* vc;
    AttnArgs attn;       // qkv, out, part, counter, shape, theta, scale (caches per layer)
    // scratch
    int* state;          // {token, position, step, last token}
    unsigned* err;
    unsigned* bar;       // grid barrier: [0] arrivals, [32] generation
    float* part;         // split-K partials [gridDim][2][16]
    unsigned* gcnt;      // split-K group tickets
    float* am_val;       // LM-head argmax partials [gridDim]
    int* am_idx;
    unsigned* am_cnt;
    int ring_slots;
    int x_floats;        // shared floats for the input vector / attention scratch
    // optional phase timeline (nanoseconds, %globaltimer): for CTA 0 and the
    // last CTA, per (step, phase): [phase start, input loaded, work done,
    // barrier passed, producer issued the phase's last tile]
    unsigned long long* trace;
};

constexpr int kTraceFields = 5;

// Rows per tile for a weight type.
inline int mega_tile_rows(int weight_dtype) { return weight_dtype == 1 ? 16 : 8; }

// Dynamic shared memory of the persistent kernel.
int mega_smem_bytes(int ring_slots, int x_floats);

// Launches the cooperative persistent kernel (grid = `ctas`).
cudaError_t launch_mega(const MegaParams& p, int weight_dtype, int ctas, cudaStream_t stream);
// Raises the dynamic shared-memory limit of both instantiations.
cudaError_t mega_prepare();
// Largest CTAs-per-SM count at this shared-memory size (0: does not fit).
int mega_occupancy(int weight_dtype, int smem_bytes);

}  // namespace infernt
