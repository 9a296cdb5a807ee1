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
    int kx;             // input columns written by the producing phase (<= K; the rest, down's
                        // padding under tensor parallelism, reads as zero)
    // activations are tagged words (decode_kernel.cu): value | phase tag << 32
    const unsigned long long* x;  // input vector, written by phase x_ph of the step; NULL: the
                                  // per-launch input or embedding row (layer 0), or the summed input
    int x_ph;                     // attention phases: the Q|K|V phase
    const float* norm_w;  // RMSNorm weight or NULL
    float eps;
    unsigned long long* out;        // NULL: the per-launch logits (LM head, plain FP32)
    const unsigned long long* res;  // residual rows (out = res + y), written by phase res_ph
    int res_ph;
    unsigned long long* xout;       // this CTA's share [K b/P, K (b+1)/P) of the input (layer 0's raw
                                    // embedding row, or the summed input) is published here, or NULL
    int layer;          // attention phases: KV-cache layer
    float* kc;          // attention phases: the layer's K and V caches [N_kv, max_seq, D]; the
    float* vc;          // Q|K|V phase before one: the same caches, whose cached rows the CTAs
                        // owning attention items prefetch into L2 when the phase starts
    // tensor parallelism
    int nsum;           // > 0: x = the xout vector of shares xbase + the nsum partials (rank order)
    const unsigned long long* xbase;  // this CTA's earlier share of the residual stream (phase xbase_ph)
    int xbase_ph;
    int sum_off;        // the partials [nsum][K] in this rank's exchange region, written by phase sum_ph
    int sum_ph;
    int xch_off;        // >= 0: epilogue writes its rows to every rank's exchange region at this
                        // byte offset, slot [this rank][units]; -1: none
    int row_base;       // LM head: global index of the first local row (argmax ids)
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
    int* state;          // {token, position, step, last token}; (token, position) published with release
    unsigned* err;
    unsigned tag_base;   // tag of this launch's first phase instance, minus 1
    unsigned long long* ll_qkv;   // tagged Q|K|V rows, split partials and attention output
    unsigned long long* ll_part;
    unsigned long long* ll_attn;
    float* am_val;       // LM-head argmax partials [gridDim]
    int* am_idx;
    unsigned* am_cnt;
    int ring_slots;
    int x_floats;        // shared floats for the input vector / attention scratch
    // tensor parallelism over tp_size GPUs (tp_size 1: none): every rank's
    // exchange region (argmax slots at kXchArgmax, the partial buffers at
    // the phases' xch_off), mapped into this process
    int tp_rank, tp_size;
    unsigned char* const* peers;   // [tp_size] region base pointers (own included)
    // optional phase timeline (nanoseconds, %globaltimer): for every CTA,
    // per (step, phase): [phase start, input loaded, work done, phase end,
    // producer issued the phase's last slot, SM cycles consumer warp 0
    // waited for full slots, SM cycles the producer waited for free slots
    // while issuing the phase's slots, GEMV phases: thread 0's tagged input
    // words current, every thread's input and the bulk-copied constants in
    // shared memory (before RMSNorm)]; attention phases record the item's
    // inputs landed (1), partial computed (4), merge start and end (5, 6),
    // RoPE and cache append done (7), first tile's softmax done (8)
    unsigned long long* trace;
    // SM clock cycles any single wait may take before the kernel gives up
    // (kErrWaitTimeout in the error word, every CTA returns)
    long long wait_cycles;
    // token choice of the LM-head phase: inv_temp 0 greedy, else a draw from
    // softmax(logits * inv_temp) by Gumbel-max with noise keyed by
    // (sample_seed, the step's position, the vocabulary id)
    float inv_temp;
    unsigned long long sample_seed;
    // weight-stream slots the producer keeps in flight (issued, not yet
    // landed); ring_slots: no limit beyond the ring
    int stream_depth;
    // the first step's token and position (init_pos >= 0): taken from here
    // instead of the state word, which CTA 0 initialises; -1: read the state
    int init_token, init_pos;
    // 1: some GEMV phase has rows narrower than a slot other than 2048 and
    // 4096 columns: launch the instantiation with the narrow-row paths
    int narrow;
};

constexpr int kTraceFields = 9;

// Exchange region layout (one per rank, cudaMalloc'd, shared by IPC):
// argmax slots [8] u64 (float value bits | index << 32 | tag << 56), then
// the tagged partial buffers.
constexpr int kMaxTp = 8;
constexpr int kXchArgmax = 0;
constexpr int kXchData = 256;

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
