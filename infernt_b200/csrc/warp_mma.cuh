// warp_mma.cuh — warp-level helpers shared by the attention kernels of
// batched decode (batch.cu) and prefill (prefill.cu): bf16 rounding,
// mma.sync m16n8k16 (bf16 x bf16 -> FP32), ldmatrix and cp.async copies.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/infernt_seed.h"

namespace infernt {

// bf16 bits of v rounded to nearest even, and back
__device__ __forceinline__ uint16_t bf16_bits(float v) {
    return (uint16_t)(__float_as_uint(infernt_round_bf16(v)) >> 16);
}
__device__ __forceinline__ float bf16_float(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// bf16x2 of (a, b), each rounded to nearest even; a in the low half
__device__ __forceinline__ uint32_t cvt_bf16x2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}

// x = hi + mid + lo as bf16 pairs (elements a, b of consecutive k); every
// difference is exact in FP32
__device__ __forceinline__ void split3_bf16x2(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
    hi = cvt_bf16x2(a, b);
    const float ar = a - __uint_as_float(hi << 16), br = b - __uint_as_float(hi & 0xffff0000u);
    mid = cvt_bf16x2(ar, br);
    lo = cvt_bf16x2(ar - __uint_as_float(mid << 16), br - __uint_as_float(mid & 0xffff0000u));
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// 16 bytes global -> shared; src_bytes 0 writes zeros (src is not read)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace infernt
