// gemv.cu — launchers and C entry points of the fused projection kernels.
#include <cstring>

#include <atomic>

#include "gemv.cuh"
#include "internal.h"

namespace infernt {

namespace {

template <typename WT, int EPI>
cudaError_t launch_one(const GemvArgs& a, bool fast, int grid, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(grid);
    cfg.stream = stream;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    if (fast) {
        cfg.blockDim = dim3(kGemvThreads);
        if (gemv_tma_smem_bytes(a.K, kGemvStagesDeep) <= kMaxDynSmem) {
            cfg.dynamicSmemBytes = gemv_tma_smem_bytes(a.K, kGemvStagesDeep);
            return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<WT, EPI, kGemvStagesDeep>, a);
        }
        cfg.dynamicSmemBytes = gemv_tma_smem_bytes(a.K, kGemvStages);
        return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<WT, EPI, kGemvStages>, a);
    }
    cfg.blockDim = dim3(kPlainThreads);
    cfg.dynamicSmemBytes = a.K * 4;
    return cudaLaunchKernelEx(&cfg, gemv_plain_kernel<WT, EPI>, a);
}

template <typename WT, int EPI>
cudaError_t set_max_smem() {
    cudaError_t e =
        raise_dynamic_smem_limit(reinterpret_cast<const void*>(gemv_tma_kernel<WT, EPI, kGemvStages>));
    if (e != cudaSuccess) return e;
    e = raise_dynamic_smem_limit(reinterpret_cast<const void*>(gemv_tma_kernel<WT, EPI, kGemvStagesDeep>));
    if (e != cudaSuccess) return e;
    return raise_dynamic_smem_limit(reinterpret_cast<const void*>(gemv_plain_kernel<WT, EPI>));
}

std::atomic<bool> g_prepared[64] = {};  // first calls on a device may race: set once, idempotent

template <typename WT>
cudaError_t launch_dtype(const GemvArgs& a, int epi, bool fast, int grid, cudaStream_t s, bool pdl) {
    switch (epi) {
        case kEpiStore: return launch_one<WT, kEpiStore>(a, fast, grid, s, pdl);
        case kEpiResidual: return launch_one<WT, kEpiResidual>(a, fast, grid, s, pdl);
        case kEpiSwiGLU: return launch_one<WT, kEpiSwiGLU>(a, fast, grid, s, pdl);
        default: return launch_one<WT, kEpiArgmax>(a, fast, grid, s, pdl);
    }
}

}  // namespace

cudaError_t raise_dynamic_smem_limit(const void* kernel) {
    int optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, current_device());
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                optin - (int)fa.sharedSizeBytes);
}

bool gemv_fast_path_ok(const GemvArgs& a, int weight_dtype, int epi) {
    (void)weight_dtype;
    if (a.K <= 0 || a.K % kPiece != 0) return false;
    if (gemv_tma_smem_bytes(a.K, kGemvStages) > kMaxDynSmem) return false;
    const int nseg = epi == kEpiSwiGLU ? 2 : a.nseg;
    for (int s = 0; s < nseg; ++s)
        if (!aligned16(a.seg_ptr[s])) return false;
    if (a.x && !aligned16(a.x)) return false;
    if (!a.x && !aligned16(a.emb)) return false;
    if (a.norm_w && !aligned16(a.norm_w)) return false;
    if (a.x_copy && !aligned16(a.x_copy)) return false;
    return true;
}

int gemv_grid(const GemvArgs& a, int weight_dtype, int epi) {
    const int sms = sm_count();
    if (gemv_fast_path_ok(a, weight_dtype, epi)) return a.units < sms ? a.units : sms;
    int g = (a.units + kPlainThreads / 32 - 1) / (kPlainThreads / 32);
    if (g > sms * 4) g = sms * 4;
    return g < 1 ? 1 : g;
}

cudaError_t gemv_prepare() {
    const int d = current_device();
    if (d >= 0 && d < 64 && g_prepared[d].load(std::memory_order_acquire)) return cudaSuccess;
    cudaError_t e;
    if ((e = set_max_smem<float, kEpiStore>()) != cudaSuccess) return e;
    if ((e = set_max_smem<float, kEpiResidual>()) != cudaSuccess) return e;
    if ((e = set_max_smem<float, kEpiSwiGLU>()) != cudaSuccess) return e;
    if ((e = set_max_smem<float, kEpiArgmax>()) != cudaSuccess) return e;
    if ((e = set_max_smem<__nv_bfloat16, kEpiStore>()) != cudaSuccess) return e;
    if ((e = set_max_smem<__nv_bfloat16, kEpiResidual>()) != cudaSuccess) return e;
    if ((e = set_max_smem<__nv_bfloat16, kEpiSwiGLU>()) != cudaSuccess) return e;
    if ((e = set_max_smem<__nv_bfloat16, kEpiArgmax>()) != cudaSuccess) return e;
    if ((e = attention_prepare()) != cudaSuccess) return e;
    if (d >= 0 && d < 64) g_prepared[d].store(true, std::memory_order_release);
    return cudaSuccess;
}

cudaError_t launch_gemv(const GemvArgs& a, int weight_dtype, int epi, cudaStream_t stream, bool pdl,
                        int* grid_out) {
    cudaError_t pe = gemv_prepare();
    if (pe != cudaSuccess) return pe;
    const bool fast = gemv_fast_path_ok(a, weight_dtype, epi);
    const int grid = gemv_grid(a, weight_dtype, epi);
    if (grid_out) *grid_out = grid;
    if (weight_dtype == INFERNT_DTYPE_BF16)
        return launch_dtype<__nv_bfloat16>(a, epi, fast, grid, stream, pdl);
    return launch_dtype<float>(a, epi, fast, grid, stream, pdl);
}

}  // namespace infernt

using namespace infernt;

namespace {

int check_dtype(int d) {
    if (d != INFERNT_DTYPE_F32 && d != INFERNT_DTYPE_BF16)
        return fail(INFERNT_ERR_INVALID_ARGUMENT, "weight_dtype %d is not F32 (0) or BF16 (1)", d);
    return INFERNT_OK;
}

GemvArgs base_args() {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    return a;
}

struct LmHeadWorkspace {
    float val[kArgmaxMaxBlocks];
    int idx[kArgmaxMaxBlocks];
    unsigned counter;
    unsigned err;
};

}  // namespace

extern "C" {

int infernt_rmsnorm_gemv(float* y, const void* W0, int n0, const void* W1, int n1, const void* W2,
                         int n2, int in_features, int weight_dtype, const float* x,
                         const float* norm_w, float eps, void* stream) {
    if (int s = check_dtype(weight_dtype)) return s;
    INFERNT_REQUIRE(y && W0 && x && n0 > 0 && in_features > 0, "rmsnorm_gemv: null pointer or empty shape");
    INFERNT_REQUIRE((W1 == nullptr) == (n1 == 0) && (W2 == nullptr) == (n2 == 0),
                    "rmsnorm_gemv: W1/W2 pointer and row count disagree");
    GemvArgs a = base_args();
    a.seg_ptr[0] = W0;
    a.seg_rows[0] = n0;
    a.nseg = 1;
    if (W1) { a.seg_ptr[a.nseg] = W1; a.seg_rows[a.nseg++] = n1; }
    if (W2) { a.seg_ptr[a.nseg] = W2; a.seg_rows[a.nseg++] = n2; }
    a.units = n0 + n1 + n2;
    a.K = in_features;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out = y;
    INFERNT_CUDA_TRY(launch_gemv(a, weight_dtype, kEpiStore, (cudaStream_t)stream, true, nullptr));
    return INFERNT_OK;
}

int infernt_gemv_residual(float* out, const float* res, const void* W, int n, int in_features,
                          int weight_dtype, const float* x, void* stream) {
    if (int s = check_dtype(weight_dtype)) return s;
    INFERNT_REQUIRE(out && res && W && x && n > 0 && in_features > 0,
                    "gemv_residual: null pointer or empty shape");
    GemvArgs a = base_args();
    a.seg_ptr[0] = W;
    a.seg_rows[0] = n;
    a.nseg = 1;
    a.units = n;
    a.K = in_features;
    a.x = x;
    a.out = out;
    a.res = res;
    INFERNT_CUDA_TRY(launch_gemv(a, weight_dtype, kEpiResidual, (cudaStream_t)stream, true, nullptr));
    return INFERNT_OK;
}

int infernt_rmsnorm_gate_up_silu(float* out, const void* Wg, const void* Wu, int n, int in_features,
                                 int weight_dtype, const float* x, const float* norm_w, float eps,
                                 void* stream) {
    if (int s = check_dtype(weight_dtype)) return s;
    INFERNT_REQUIRE(out && Wg && Wu && x && n > 0 && in_features > 0,
                    "gate_up_silu: null pointer or empty shape");
    GemvArgs a = base_args();
    a.seg_ptr[0] = Wg;
    a.seg_ptr[1] = Wu;
    a.seg_rows[0] = a.seg_rows[1] = n;
    a.nseg = 2;
    a.units = n;
    a.K = in_features;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out = out;
    INFERNT_CUDA_TRY(launch_gemv(a, weight_dtype, kEpiSwiGLU, (cudaStream_t)stream, true, nullptr));
    return INFERNT_OK;
}

size_t infernt_lm_head_workspace_bytes(void) { return sizeof(LmHeadWorkspace); }

int infernt_rmsnorm_lm_head_argmax(float* logits, int* out_token, const void* W, int vocab_size,
                                   int in_features, int weight_dtype, const float* x,
                                   const float* norm_w, float eps, void* workspace, void* stream) {
    if (int s = check_dtype(weight_dtype)) return s;
    INFERNT_REQUIRE(logits && out_token && W && x && workspace && vocab_size > 0 && in_features > 0,
                    "lm_head_argmax: null pointer or empty shape");
    auto* ws = static_cast<LmHeadWorkspace*>(workspace);
    GemvArgs a = base_args();
    a.seg_ptr[0] = W;
    a.seg_rows[0] = vocab_size;
    a.nseg = 1;
    a.units = vocab_size;
    a.K = in_features;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.out = logits;
    a.am_val = ws->val;
    a.am_idx = ws->idx;
    a.am_counter = &ws->counter;
    a.am_out = out_token;
    a.err = &ws->err;
    INFERNT_REQUIRE(gemv_grid(a, weight_dtype, kEpiArgmax) <= kArgmaxMaxBlocks, "lm_head_argmax: grid too large");
    INFERNT_CUDA_TRY(launch_gemv(a, weight_dtype, kEpiArgmax, (cudaStream_t)stream, true, nullptr));
    return INFERNT_OK;
}

}  // extern "C"
