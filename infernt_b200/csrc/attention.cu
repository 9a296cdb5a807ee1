// attention.cu — standalone launcher of the decode attention (one CTA per
// (KV head, split) work item; the device code is attention.cuh).
#include <cmath>
#include <cstring>
#include <mutex>

#include "attention.cuh"
#include "gemv.cuh"
#include "internal.h"

namespace infernt {

constexpr int kAttnThreads = 256;

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    pdl_launch_dependents();
    pdl_wait();
    const int pos = a.pos_ptr ? *a.pos_ptr : a.pos;
    if (pos < 0 || pos >= a.max_seq) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && a.err) atomicOr(a.err, kErrPosition);
        return;
    }
    int chunk, active;
    attn_chunk(pos + 1, a.splits, chunk, active);
    if ((int)blockIdx.y >= active) return;
    attention_item<kAttnThreads>(a, blockIdx.x, blockIdx.y, pos, sm, threadIdx.x);
}

cudaError_t launch_attention_decode(const AttnArgs& a, cudaStream_t stream, bool pdl) {
    cudaError_t e = gemv_prepare();
    if (e != cudaSuccess) return e;
    const int G = a.nq / a.nkv;
    const int smem = attn_smem_floats(G, a.D) * 4;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(a.nkv, a.splits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, attention_decode_kernel, a);
}

cudaError_t attention_prepare() {
    return raise_dynamic_smem_limit(reinterpret_cast<const void*>(attention_decode_kernel));
}

int attention_shape_check(int nq, int nkv, int D, int splits) {
    INFERNT_REQUIRE(nq > 0 && nkv > 0 && nq % nkv == 0, "attention: Nq %d must be a positive multiple of Nkv %d", nq, nkv);
    INFERNT_REQUIRE(nq / nkv <= kAttnMaxGroup, "attention: group size %d > %d", nq / nkv, kAttnMaxGroup);
    INFERNT_REQUIRE(D >= 2 && D <= kAttnMaxD && D % 2 == 0, "attention: head_dim %d must be even and at most %d", D,
                    kAttnMaxD);
    INFERNT_REQUIRE(splits >= 1 && splits <= 4096, "attention: splits %d out of range", splits);
    return INFERNT_OK;
}

size_t attention_workspace_bytes(int nq, int nkv, int D, int splits) {
    const size_t part = (size_t)nkv * splits * (nq / nkv) * (D + 2) * sizeof(float);
    const size_t cnt = (size_t)nkv * sizeof(unsigned);
    return ((part + 255) / 256) * 256 + ((cnt + 255) / 256) * 256 + 256;
}

}  // namespace infernt

// Scratch of infernt_attention_decode_noalloc: the per-KV-head tickets (up
// to 64 heads) at a fixed place at the start, so calls of different shapes
// find them where the previous call left them at zero; then the kernel's
// error word (written by the device only: the host validates the position
// and shape before the launch, so it stays clear; it is not read back); then
// the split partials from offset 512.  512 KiB covers every split
// count up to the SM count for the usual LLaMA shapes (TinyLlama: 313 KB of
// partials at 37 splits; Llama-3-8B: 300 KB at 18).  Static storage starts
// zeroed when the module loads, which is what the tickets need; each
// completed call leaves them at zero again.  The partials need no zeroing.
static constexpr size_t kAttnStaticScratchBytes = 512 * 1024;
static constexpr int kAttnStaticTickets = 64;
static constexpr size_t kAttnStaticPartOffset = 512;
static __device__ __align__(256) unsigned char g_attn_static_scratch[kAttnStaticScratchBytes];

namespace infernt {
namespace {

std::mutex g_static_mu;
void* g_static_addr[64] = {nullptr};

// Device address of the static scratch on the current device, looked up
// once per device and kept for the process: after cudaDeviceReset the
// module reloads and the address may change, so a process that resets a
// device must not call infernt_attention_decode_noalloc on it again.
int attn_static_scratch(void** out) {
    const int d = current_device();
    INFERNT_REQUIRE(d >= 0 && d < 64, "attention_decode_noalloc: device ordinal %d out of range", d);
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_addr[d]) {
        void* p = nullptr;
        INFERNT_CUDA_TRY(cudaGetSymbolAddress(&p, g_attn_static_scratch));
        g_static_addr[d] = p;
    }
    *out = g_static_addr[d];
    return INFERNT_OK;
}

}  // namespace
}  // namespace infernt

using namespace infernt;

extern "C" {

size_t infernt_attention_workspace_bytes(int num_q_heads, int num_kv_heads, int head_dim, int splits) {
    if (num_kv_heads <= 0 || splits <= 0) return 0;
    return attention_workspace_bytes(num_q_heads, num_kv_heads, head_dim, splits);
}

int infernt_attention_decode(float* out, const float* qkv, float* k_cache, float* v_cache, int num_q_heads,
                             int num_kv_heads, int head_dim, int max_seq_len, int position, float theta, int splits,
                             void* workspace, void* stream) {
    if (int s = attention_shape_check(num_q_heads, num_kv_heads, head_dim, splits)) return s;
    INFERNT_REQUIRE(out && qkv && k_cache && v_cache && workspace, "attention_decode: null pointer");
    INFERNT_REQUIRE(position >= 0 && position < max_seq_len, "attention_decode: position %d outside [0, %d)", position,
                    max_seq_len);
    const size_t part = (size_t)num_kv_heads * splits * (num_q_heads / num_kv_heads) * (head_dim + 2) * 4;
    const size_t part_al = ((part + 255) / 256) * 256;
    const size_t cnt_al = (((size_t)num_kv_heads * 4 + 255) / 256) * 256;
    AttnArgs a;
    memset(&a, 0, sizeof(a));
    a.qkv = qkv;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.out = out;
    a.part = static_cast<float*>(workspace);
    a.counter = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + part_al);
    a.err = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + part_al + cnt_al);
    a.pos = position;
    a.nq = num_q_heads;
    a.nkv = num_kv_heads;
    a.D = head_dim;
    a.max_seq = max_seq_len;
    a.splits = splits;
    a.theta = theta;
    a.scale = 1.0f / sqrtf((float)head_dim);
    INFERNT_CUDA_TRY(launch_attention_decode(a, (cudaStream_t)stream, true));
    return INFERNT_OK;
}

int infernt_attention_decode_noalloc(float* out, const float* qkv, float* k_cache, float* v_cache, int num_q_heads,
                                     int num_kv_heads, int head_dim, int max_seq_len, int position, float theta,
                                     int splits, void* stream) {
    if (int s = attention_shape_check(num_q_heads, num_kv_heads, head_dim, splits)) return s;
    const size_t need = attention_workspace_bytes(num_q_heads, num_kv_heads, head_dim, splits);
    INFERNT_REQUIRE(num_kv_heads <= kAttnStaticTickets && need <= kAttnStaticScratchBytes,
                    "attention_decode_noalloc: %d KV heads x %d splits need %zu bytes of scratch, the static "
                    "scratch holds %zu (and tickets for %d KV heads); use fewer splits or "
                    "infernt_attention_decode with a workspace",
                    num_kv_heads, splits, need, kAttnStaticScratchBytes, kAttnStaticTickets);
    INFERNT_REQUIRE(out && qkv && k_cache && v_cache, "attention_decode_noalloc: null pointer");
    INFERNT_REQUIRE(position >= 0 && position < max_seq_len,
                    "attention_decode_noalloc: position %d outside [0, %d)", position, max_seq_len);
    void* ws = nullptr;
    if (int s = attn_static_scratch(&ws)) return s;
    char* base = static_cast<char*>(ws);
    AttnArgs a;
    memset(&a, 0, sizeof(a));
    a.qkv = qkv;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.out = out;
    a.counter = reinterpret_cast<unsigned*>(base);
    a.err = reinterpret_cast<unsigned*>(base + kAttnStaticTickets * sizeof(unsigned));
    a.part = reinterpret_cast<float*>(base + kAttnStaticPartOffset);
    a.pos = position;
    a.nq = num_q_heads;
    a.nkv = num_kv_heads;
    a.D = head_dim;
    a.max_seq = max_seq_len;
    a.splits = splits;
    a.theta = theta;
    a.scale = 1.0f / sqrtf((float)head_dim);
    INFERNT_CUDA_TRY(launch_attention_decode(a, (cudaStream_t)stream, true));
    return INFERNT_OK;
}

}  // extern "C"
