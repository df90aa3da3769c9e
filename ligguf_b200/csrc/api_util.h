// api_util.h - host-side plumbing shared by the library's C-ABI translation units: the one-line error
// reason of the calling thread (ligguf_cuda_attn_last_error), CUDA status checks that turn into
// LIGGUF_ATTN_ECUDA, and a scoped switch of the current device.
#pragma once

#include <cuda_runtime.h>

#include "ligguf_cuda_attn.h"

namespace lgapi {

// Records a printf-style reason for the calling thread and returns `code`.
int fail(int code, const char* fmt, ...);
// The reason recorded last on the calling thread ("" if none).
const char* last_error();

struct DeviceGuard {
    int prev = -1;
    bool switched = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) switched = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (switched) cudaSetDevice(prev);
    }
};

}  // namespace lgapi

#define LG_CUDA(expr)                                                                          \
    do {                                                                                       \
        const cudaError_t e_ = (expr);                                                         \
        if (e_ != cudaSuccess) {                                                               \
            (void)cudaGetLastError(); /* do not leave it pending for unrelated calls */       \
            return lgapi::fail(LIGGUF_ATTN_ECUDA, "%s failed: %s (%s:%d)", #expr,              \
                               cudaGetErrorString(e_), __FILE__, __LINE__);                    \
        }                                                                                      \
    } while (0)
