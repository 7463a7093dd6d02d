// host_util.h - error reporting and device scoping shared by the host files of
// libprism_moe.so.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

// Records the message for prism_last_error_string() on this thread; returns code.
int set_error(int code, const char* fmt, ...);

// Makes `d` the current device for the scope, restoring the caller's device after.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int d) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != d) cudaSetDevice(d);
    }
    ~DeviceGuard() {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Per-context scratch of the encoder / decoder passes (codec_tc.cu).
void* codec_scratch_new();
void codec_scratch_free(void* p);

// [off, off + n) inside [0, limit)?
inline bool in_range(int64_t off, int64_t n, size_t limit) {
    return off >= 0 && n >= 0 && (uint64_t)(off + n) <= (uint64_t)limit;
}

}  // namespace prism

// the context struct behind the opaque prism_ctx handle
struct prism_ctx {
    int device;
    int sm_count;
    uint32_t* err = nullptr;  // device error word of the per-pass kernels that wait (prism_ctx_status)
    void* codec = nullptr;    // repacked weights of the encoder / decoder passes, per kind
};
