// rb_runtime.cu -- per-device contexts, error text, library-level entry points.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "rb_device.cuh"
#include "rb_runtime.h"

namespace rb {

static thread_local std::string t_err;
static thread_local int t_device = 0;
static std::atomic<uint64_t> g_wait_ns{2000ull * 1000 * 1000};
static DevCtx g_ctx[kMaxDevices];
static std::mutex g_ctx_mu;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

int ok() {
    t_err.clear();
    return RABBIT_CUDA_OK;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(RABBIT_CUDA_ERR_DEVICE, "%s: %s (%s)", what, cudaGetErrorString(e),
                cudaGetErrorName(e));
}

int current_device() { return t_device; }

uint64_t wait_limit_ns() { return g_wait_ns.load(); }

DevCtx *dev_ctx(int device, int *status) {
    if (device < 0 || device >= kMaxDevices) {
        *status = fail(RABBIT_CUDA_ERR_ARGS, "device %d out of range", device);
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_ctx_mu);
    DevCtx *c = &g_ctx[device];
    if (c->device == device) {
        *status = RABBIT_CUDA_OK;
        if (cudaSetDevice(device) != cudaSuccess) {
            *status = fail(RABBIT_CUDA_ERR_DEVICE, "cudaSetDevice(%d) failed", device);
            return nullptr;
        }
        return c;
    }
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || device >= n) {
        *status = fail(RABBIT_CUDA_ERR_DEVICE, "no CUDA device %d (count %d: %s)", device, n,
                       cudaGetErrorString(e));
        return nullptr;
    }
    if ((e = cudaSetDevice(device)) != cudaSuccess) {
        *status = cuda_fail(e, "cudaSetDevice");
        return nullptr;
    }
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
        *status = cuda_fail(e, "cudaGetDeviceProperties");
        return nullptr;
    }
    if (prop.major < 10) {
        *status = fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                       "device %d is sm_%d%d; this build targets sm_100a (B200)", device,
                       prop.major, prop.minor);
        return nullptr;
    }
    c->sm_count = prop.multiProcessorCount;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMalloc(&c->d_err, sizeof(int))) != cudaSuccess ||
        (e = cudaMemset(c->d_err, 0, sizeof(int))) != cudaSuccess) {
        *status = cuda_fail(e, "device context setup");
        return nullptr;
    }
    c->device = device;
    *status = RABBIT_CUDA_OK;
    return c;
}

int ensure_pinned(DevCtx *c, size_t bytes) {
    if (bytes <= c->pin_cap) return RABBIT_CUDA_OK;
    if (c->pin) cudaFreeHost(c->pin);
    c->pin = nullptr;
    c->pin_cap = 0;
    size_t cap = bytes < 4096 ? 4096 : bytes;
    RB_CUDA(cudaMallocHost(&c->pin, cap));
    c->pin_cap = cap;
    return RABBIT_CUDA_OK;
}

int ensure_dscratch(DevCtx *c, size_t bytes) {
    if (bytes <= c->dscratch_cap) return RABBIT_CUDA_OK;
    if (c->dscratch) cudaFree(c->dscratch);
    c->dscratch = nullptr;
    c->dscratch_cap = 0;
    size_t cap = bytes < 4096 ? 4096 : bytes;
    RB_CUDA(cudaMalloc(&c->dscratch, cap));
    c->dscratch_cap = cap;
    return RABBIT_CUDA_OK;
}

int check_device_error(DevCtx *c, cudaStream_t s, const char *what) {
    RB_CUDA(cudaStreamSynchronize(s));
    int h = 0;
    RB_CUDA(cudaMemcpyAsync(&h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RB_CUDA(cudaStreamSynchronize(s));
    if (h != 0) {
        RB_CUDA(cudaMemsetAsync(c->d_err, 0, sizeof(int), s));
        RB_CUDA(cudaStreamSynchronize(s));
        if (h == RB_ERR_TIMEOUT)
            return fail(RABBIT_CUDA_ERR_TIMEOUT, "%s: a bounded device wait ran out", what);
        return fail(RABBIT_CUDA_ERR_DEVICE, "%s: device error code %d", what, h);
    }
    return RABBIT_CUDA_OK;
}

}  // namespace rb

extern "C" {

const char *rabbit_cuda_version(void) { return "rabbit-b200 0.1.0 (sm_100a)"; }

const char *rabbit_cuda_last_error(void) { return rb::t_err.c_str(); }

int rabbit_cuda_device_count(int *count) {
    if (!count) return rb::fail(RABBIT_CUDA_ERR_ARGS, "count is NULL");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
    *count = n;
    return rb::ok();
}

int rabbit_cuda_set_device(int device) {
    int st;
    if (!rb::dev_ctx(device, &st)) return st;
    rb::t_device = device;
    return rb::ok();
}

int rabbit_cuda_set_wait_limit_ms(int ms) {
    if (ms <= 0) return rb::fail(RABBIT_CUDA_ERR_ARGS, "wait limit must be positive");
    rb::g_wait_ns.store(static_cast<uint64_t>(ms) * 1000ull * 1000ull);
    return rb::ok();
}

int rabbit_cuda_set_wait_limit_us(int us) {
    if (us <= 0) return rb::fail(RABBIT_CUDA_ERR_ARGS, "wait limit must be positive");
    rb::g_wait_ns.store(static_cast<uint64_t>(us) * 1000ull);
    return rb::ok();
}

}  // extern "C"
