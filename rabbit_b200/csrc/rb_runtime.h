// rb_runtime.h -- host runtime shared by the C ABI translation units:
// per-device context (stream, SM count, error word, pinned staging),
// thread-local error text, CUDA-call checking.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "../../include/rabbit_cuda.h"

namespace rb {

// Set the calling thread's error text and return `code`.
int fail(int code, const char *fmt, ...);
// Clear the calling thread's error text; returns RABBIT_CUDA_OK.
int ok();
// Turn a CUDA error into RABBIT_CUDA_ERR_DEVICE with context.
int cuda_fail(cudaError_t e, const char *what);

#define RB_CUDA(call)                                              \
    do {                                                           \
        cudaError_t rb_e_ = (call);                                \
        if (rb_e_ != cudaSuccess) return ::rb::cuda_fail(rb_e_, #call); \
    } while (0)

constexpr int kMaxDevices = 16;
constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in per CTA on sm_100

struct DevCtx {
    int device = -1;
    int sm_count = 0;
    cudaStream_t stream = nullptr;  // library stream for host-buffer entry points
    int *d_err = nullptr;           // device error word (RB_ERR_*), 0 = clean
    // pinned host staging for host-buffer entry points
    void *pin = nullptr;
    size_t pin_cap = 0;
    // device scratch for stateless entry points (raw blob, x, y)
    void *dscratch = nullptr;
    size_t dscratch_cap = 0;
    std::mutex mu;  // serialises host-buffer calls on this device
};

// Current thread's device (set by rabbit_cuda_set_device, default 0).
int current_device();
// Lazily created context for `device`; nullptr + error text on failure.
DevCtx *dev_ctx(int device, int *status);
// Grow pinned / device scratch of ctx (caller holds ctx->mu).
int ensure_pinned(DevCtx *c, size_t bytes);
int ensure_dscratch(DevCtx *c, size_t bytes);
// Device wait limit in ns for bounded spins.
uint64_t wait_limit_ns();
// Read and clear the device error word of ctx after synchronising `s`.
int check_device_error(DevCtx *c, cudaStream_t s, const char *what);

// A NULL stream argument is the default (legacy) stream, as in CUDA itself,
// so a caller's stream-0 work and ours stay ordered.
inline cudaStream_t as_stream(void *s, DevCtx *) { return static_cast<cudaStream_t>(s); }

}  // namespace rb
