// internal.h — host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/infernt_capi.h"

namespace infernt {

// Records a formatted detail message for infernt_last_error() and returns status.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Maps a CUDA error to INFERNT_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t e, const char* what);
// Clears the detail message (successful calls leave it untouched).
void clear_error();

// Streaming multiprocessors of the current device (cached per device).
int sm_count();
// Current device ordinal.
int current_device();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace infernt

#define INFERNT_CUDA_TRY(expr)                                   \
    do {                                                         \
        cudaError_t e__ = (expr);                                \
        if (e__ != cudaSuccess) return ::infernt::cuda_fail(e__, #expr); \
    } while (0)

#define INFERNT_REQUIRE(cond, ...)                                              \
    do {                                                                        \
        if (!(cond)) return ::infernt::fail(INFERNT_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)
