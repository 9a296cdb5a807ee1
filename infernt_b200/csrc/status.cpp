// status.cpp — status strings, per-thread error detail, device queries.
#include <cstdarg>
#include <cstdio>

#include "internal.h"

namespace infernt {

namespace {
thread_local char g_detail[1024] = "";
int g_sm_count[64] = {0};
}  // namespace

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_detail, sizeof(g_detail), fmt, ap);
    va_end(ap);
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    // the error is reported here; clear the runtime's last-error slot so a
    // later launch check does not report it a second time
    cudaGetLastError();
    if (e == cudaErrorMemoryAllocation)
        return fail(INFERNT_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
        return fail(INFERNT_ERR_NO_DEVICE, "%s: %s", what, cudaGetErrorString(e));
    return fail(INFERNT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void clear_error() { g_detail[0] = '\0'; }

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

int sm_count() {
    int d = current_device();
    if (d < 0 || d >= 64) d = 0;
    if (g_sm_count[d] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
        g_sm_count[d] = n > 0 ? n : 1;
    }
    return g_sm_count[d];
}

}  // namespace infernt

extern "C" {

const char* infernt_status_string(int status) {
    switch (status) {
        case INFERNT_OK: return "ok";
        case INFERNT_ERR_INVALID_ARGUMENT: return "invalid argument";
        case INFERNT_ERR_UNSUPPORTED: return "unsupported";
        case INFERNT_ERR_CUDA: return "CUDA error";
        case INFERNT_ERR_OUT_OF_MEMORY: return "out of device memory";
        case INFERNT_ERR_DEVICE: return "device-side error";
        case INFERNT_ERR_NO_DEVICE: return "no usable CUDA device";
    }
    return "unknown status";
}

const char* infernt_last_error(void) { return infernt::g_detail; }

int infernt_version(void) { return 100; }

}  // extern "C"
