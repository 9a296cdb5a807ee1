// cublas_wrapper.h — the GEMM interface of the reference's
// include/cublas_wrapper.h:15-39, kept under its class name so callers that
// construct a CublasWrapper and pass it to LlamaArchitecture compile
// unchanged.  There is no cuBLAS underneath: gemm() runs the engine's own
// FP32 kernels (weight-streaming GEMV for M = 1, tiled SIMT otherwise).
#pragma once

#include <cuda_runtime.h>

// The reference's handle type, declared as cuBLAS declares it (struct
// cublasContext*), so handle() keeps its signature without a cuBLAS
// dependency; a caller that also includes cublas_v2.h sees the same type.
struct cublasContext;
typedef struct cublasContext* cublasHandle_t;

class CublasWrapper {
public:
    CublasWrapper();
    ~CublasWrapper();

    CublasWrapper(const CublasWrapper&) = delete;
    CublasWrapper& operator=(const CublasWrapper&) = delete;

    // Row-major C[M,N] = alpha * op(A) . op(B) + beta * C (gemm/cublas_wrapper.cu:21-40).
    void gemm(const float* A, const float* B, float* C, int M, int N, int K, float alpha = 1.0f,
              float beta = 0.0f, bool trans_a = false, bool trans_b = false);

    // batch_count independent GEMMs at the given element strides.
    void batched_gemm(const float* A, const float* B, float* C, int M, int N, int K, int batch_count,
                      int stride_a, int stride_b, int stride_c, float alpha = 1.0f, float beta = 0.0f,
                      bool trans_a = false, bool trans_b = false);

    void set_stream(cudaStream_t stream);
    // The reference's accessor (include/cublas_wrapper.h:35).  No cuBLAS
    // handle exists underneath: always nullptr.
    cublasHandle_t handle() const;
    // The stream this wrapper launches on.
    cudaStream_t stream() const;

private:
    cudaStream_t stream_;
};
