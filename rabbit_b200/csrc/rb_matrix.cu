// rb_matrix.cu -- C ABI: stateless quant drop-ins and resident int4 matrices.
#include <string.h>

#include <vector>

#include "rb_gemv.cuh"
#include "rb_runtime.h"

struct rabbit_cuda_matrix {
    int device;
    int rows, in_dim;
    uint32_t group_size;
    bool fast;             // tiled layout + streaming kernel
    uint8_t *tiles;        // fast: plan.til.ntiles tiles of plan.til.tile_stride bytes
    uint8_t *raw;          // flat: verbatim blob
    size_t blob_bytes;     // bytes of the .rabbit blob
    rb::G32Plan plan;
};

namespace rb {

static bool g_attr_set[kMaxDevices];

// One launch over n matrices of plan p's tiling (n == 1: a single GEMV).
static int launch_g32(const G32Plan &p, int n, const uint8_t *const *tiles,
                      const float *const *x, float *const *y, DevCtx *c, cudaStream_t s) {
    if (!g_attr_set[c->device]) {
        for (int J = 1; J <= 2; ++J)
            RB_CUDA(cudaFuncSetAttribute(gemv_g32_kernel(J),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem));
        g_attr_set[c->device] = true;
    }
    G32Plan pb;
    if (!plan_g32_batch(p, n, c->sm_count, &pb))
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED, "gemv: no launch plan for %d matrices", n);
    G32Args a;
    a.nmat = n;
    a.shared_x = 1;
    for (int m = 0; m < n; ++m) {
        a.tiles[m] = tiles[m];
        a.x[m] = x[m];
        a.y[m] = y[m];
        if (x[m] != x[0]) a.shared_x = 0;
    }
    a.til = pb.til;
    a.KS = pb.KS;
    a.NG = pb.NG;
    a.ROWS = pb.ROWS;
    a.nslots = pb.nslots;
    a.tiles_cta_max = pb.tiles_cta_max;
    a.err = c->d_err;
    a.wait_ns = wait_limit_ns();
    // Programmatic dependent launch: this GEMV may start (and stream its
    // weights) while the kernel before it on the stream finishes; it waits
    // for that kernel before reading x or writing y.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pb.grid);
    cfg.blockDim = dim3(pb.block);
    cfg.dynamicSmemBytes = pb.smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&a};
    RB_CUDA(cudaLaunchKernelExC(&cfg, gemv_g32_kernel(pb.J), args));
    return RABBIT_CUDA_OK;
}

static int launch_g32(const G32Plan &p, const uint8_t *tiles, const float *x, float *y, DevCtx *c,
                      cudaStream_t s) {
    return launch_g32(p, 1, &tiles, &x, &y, c, s);
}

static int launch_flat(const uint8_t *blob, const float *x, float *y, int out_dim, int in_dim,
                       cudaStream_t s) {
    const int warps = 8;
    k_gemv_flat<<<(out_dim + warps - 1) / warps, warps * 32, 0, s>>>(blob, x, y, out_dim, in_dim);
    RB_CUDA(cudaGetLastError());
    return RABBIT_CUDA_OK;
}

static bool blob_bytes(int out_dim, int in_dim, uint32_t gs, size_t *out) {
    const long long n = (long long)out_dim * in_dim;
    if (n <= 0 || n > 0x7fffffffLL) return false;  // the format indexes with int
    const long long g = gs ? gs : 32;
    *out = (size_t)(4 + 4 * ((n + g - 1) / g) + (n + 1) / 2);
    return true;
}

}  // namespace rb

using namespace rb;

extern "C" {

int rabbit_cuda_gemv_int4_grouped(const uint8_t *W, const float *x, float *y, int out_dim,
                                  int in_dim) {
    if (!W || !x || !y || out_dim <= 0 || in_dim <= 0)
        return fail(RABBIT_CUDA_ERR_ARGS, "gemv: NULL pointer or non-positive size");
    uint32_t gs;
    memcpy(&gs, W, 4);
    if (gs == 0 || gs > 4096) {  // quant.c:158-161
        memset(y, 0, sizeof(float) * (size_t)out_dim);
        return ok();
    }
    size_t nbytes;
    if (!blob_bytes(out_dim, in_dim, gs, &nbytes))
        return fail(RABBIT_CUDA_ERR_ARGS, "gemv: out_dim*in_dim exceeds the format's int range");
    int st;
    DevCtx *c = dev_ctx(current_device(), &st);
    if (!c) return st;
    std::lock_guard<std::mutex> g(c->mu);
    const size_t xb = align_up((size_t)in_dim * 4, 256), yb = align_up((size_t)out_dim * 4, 256);
    G32Plan p;
    const bool fast = gs == 32 && plan_g32(out_dim, in_dim, c->sm_count, &p);
    const size_t tb = fast ? (size_t)p.til.ntiles * p.til.tile_stride : 0;
    const size_t wb = fast ? align_up(tb, 256) : align_up(nbytes, 256);
    if ((st = ensure_dscratch(c, wb + xb + yb)) != RABBIT_CUDA_OK) return st;
    uint8_t *dw = static_cast<uint8_t *>(c->dscratch);
    float *dx = reinterpret_cast<float *>(dw + wb);
    float *dy = reinterpret_cast<float *>(dw + wb + xb);
    cudaStream_t s = c->stream;
    RB_CUDA(cudaMemcpyAsync(dx, x, (size_t)in_dim * 4, cudaMemcpyHostToDevice, s));
    if (fast) {
        // tile on the host into pinned memory, one copy to the device
        if ((st = ensure_pinned(c, tb)) != RABBIT_CUDA_OK) return st;
        RB_CUDA(cudaStreamSynchronize(s));  // pinned buffer is free
        tile_blob_host(W, p.til, static_cast<uint8_t *>(c->pin));
        RB_CUDA(cudaMemcpyAsync(dw, c->pin, tb, cudaMemcpyHostToDevice, s));
        if ((st = launch_g32(p, dw, dx, dy, c, s)) != RABBIT_CUDA_OK) return st;
    } else {
        RB_CUDA(cudaMemcpyAsync(dw, W, nbytes, cudaMemcpyHostToDevice, s));
        if ((st = launch_flat(dw, dx, dy, out_dim, in_dim, s)) != RABBIT_CUDA_OK) return st;
    }
    RB_CUDA(cudaMemcpyAsync(y, dy, (size_t)out_dim * 4, cudaMemcpyDeviceToHost, s));
    if ((st = check_device_error(c, s, "gemv")) != RABBIT_CUDA_OK) return st;
    return ok();
}

int rabbit_cuda_dequant_int4_grouped_dev(const uint8_t *d_blob, float *d_dst, int n,
                                         void *stream) {
    if (!d_blob || !d_dst || n <= 0)
        return fail(RABBIT_CUDA_ERR_ARGS, "dequant: NULL pointer or non-positive n");
    int st;
    DevCtx *c = dev_ctx(current_device(), &st);
    if (!c) return st;
    cudaStream_t s = as_stream(stream, c);
    uint32_t gs = 0;
    RB_CUDA(cudaMemcpyAsync(&gs, d_blob, 4, cudaMemcpyDeviceToHost, s));
    RB_CUDA(cudaStreamSynchronize(s));
    if (gs == 0 || gs > 4096)  // quant.c:128
        return fail(RABBIT_CUDA_ERR_FORMAT, "dequant: invalid group_size %u", gs);
    const int threads = 256;
    long long blocks = ((long long)n + threads - 1) / threads;
    if (blocks > 4L * c->sm_count * 8) blocks = 4L * c->sm_count * 8;
    k_dequant_flat<<<(int)blocks, threads, 0, s>>>(d_blob, d_dst, n, gs);
    RB_CUDA(cudaGetLastError());
    return ok();
}

int rabbit_cuda_gemv_int4_grouped_dev(const uint8_t *d_blob, const float *d_x, float *d_y,
                                      int out_dim, int in_dim, void *stream) {
    if (!d_blob || !d_x || !d_y || out_dim <= 0 || in_dim <= 0)
        return fail(RABBIT_CUDA_ERR_ARGS, "gemv_dev: NULL pointer or non-positive size");
    int st;
    DevCtx *c = dev_ctx(current_device(), &st);
    if (!c) return st;
    if ((st = launch_flat(d_blob, d_x, d_y, out_dim, in_dim, as_stream(stream, c))) !=
        RABBIT_CUDA_OK)
        return st;
    return ok();
}

int rabbit_cuda_matrix_upload(const uint8_t *blob, int out_dim, int in_dim,
                              rabbit_cuda_matrix **out) {
    if (!blob || !out || out_dim <= 0 || in_dim <= 0)
        return fail(RABBIT_CUDA_ERR_ARGS, "matrix_upload: NULL pointer or non-positive size");
    *out = nullptr;
    uint32_t gs;
    memcpy(&gs, blob, 4);
    size_t nbytes;
    if (!blob_bytes(out_dim, in_dim, gs, &nbytes))
        return fail(RABBIT_CUDA_ERR_ARGS, "matrix_upload: out_dim*in_dim exceeds int range");
    int st;
    DevCtx *c = dev_ctx(current_device(), &st);
    if (!c) return st;
    rabbit_cuda_matrix *m = new rabbit_cuda_matrix();
    m->device = c->device;
    m->rows = out_dim;
    m->in_dim = in_dim;
    m->group_size = gs;
    m->blob_bytes = nbytes;
    m->fast = gs == 32 && plan_g32(out_dim, in_dim, c->sm_count, &m->plan);
    cudaError_t e;
    if (m->fast) {
        const size_t tb = (size_t)m->plan.til.ntiles * m->plan.til.tile_stride;
        std::vector<uint8_t> img(tb);
        tile_blob_host(blob, m->plan.til, img.data());
        if ((e = cudaMalloc(&m->tiles, tb)) != cudaSuccess ||
            (e = cudaMemcpy(m->tiles, img.data(), tb, cudaMemcpyHostToDevice)) != cudaSuccess) {
            rabbit_cuda_matrix_free(m);
            return cuda_fail(e, "matrix_upload (tiles)");
        }
    } else {
        if ((e = cudaMalloc(&m->raw, nbytes)) != cudaSuccess ||
            (e = cudaMemcpy(m->raw, blob, nbytes, cudaMemcpyHostToDevice)) != cudaSuccess) {
            rabbit_cuda_matrix_free(m);
            return cuda_fail(e, "matrix_upload (raw)");
        }
    }
    *out = m;
    return ok();
}

int rabbit_cuda_matrix_free(rabbit_cuda_matrix *m) {
    if (!m) return ok();
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    if (m->tiles) cudaFree(m->tiles);
    if (m->raw) cudaFree(m->raw);
    cudaSetDevice(prev);
    delete m;
    return ok();
}

int rabbit_cuda_matrix_gemv_batch_dev(const rabbit_cuda_matrix *const *m, int n,
                                      const float *const *d_x, float *const *d_y, void *stream) {
    if (!m || !d_x || !d_y || n < 1 || n > kMaxBatch)
        return fail(RABBIT_CUDA_ERR_ARGS, "matrix_gemv_batch_dev: need 1..%d matrices", kMaxBatch);
    for (int i = 0; i < n; ++i) {
        if (!m[i] || !d_x[i] || !d_y[i])
            return fail(RABBIT_CUDA_ERR_ARGS, "matrix_gemv_batch_dev: NULL entry %d", i);
        if (m[i]->device != m[0]->device || m[i]->rows != m[0]->rows ||
            m[i]->in_dim != m[0]->in_dim || m[i]->fast != m[0]->fast ||
            m[i]->group_size != m[0]->group_size)
            return fail(RABBIT_CUDA_ERR_ARGS,
                        "matrix_gemv_batch_dev: matrix %d differs in device, shape or format", i);
    }
    if (!m[0]->fast) {  // one flat-index launch per matrix
        for (int i = 0; i < n; ++i) {
            const int st = rabbit_cuda_matrix_gemv_dev(m[i], d_x[i], d_y[i], stream);
            if (st != RABBIT_CUDA_OK) return st;
        }
        return ok();
    }
    int st;
    DevCtx *c = dev_ctx(m[0]->device, &st);
    if (!c) return st;
    const uint8_t *tiles[kMaxBatch];
    for (int i = 0; i < n; ++i) {
        if ((reinterpret_cast<uintptr_t>(d_x[i]) & 15) != 0)
            return fail(RABBIT_CUDA_ERR_ARGS, "matrix_gemv_batch_dev: x must be 16-byte aligned");
        tiles[i] = m[i]->tiles;
    }
    st = launch_g32(m[0]->plan, n, tiles, d_x, d_y, c, as_stream(stream, c));
    return st == RABBIT_CUDA_OK ? ok() : st;
}

int rabbit_cuda_matrix_gemv_dev(const rabbit_cuda_matrix *m, const float *d_x, float *d_y,
                                void *stream) {
    if (!m || !d_x || !d_y) return fail(RABBIT_CUDA_ERR_ARGS, "matrix_gemv_dev: NULL argument");
    int st;
    DevCtx *c = dev_ctx(m->device, &st);
    if (!c) return st;
    cudaStream_t s = as_stream(stream, c);
    if (m->fast) {
        if ((reinterpret_cast<uintptr_t>(d_x) & 15) != 0)
            return fail(RABBIT_CUDA_ERR_ARGS, "matrix_gemv_dev: x must be 16-byte aligned");
        st = launch_g32(m->plan, m->tiles, d_x, d_y, c, s);
    } else if (m->group_size == 0 || m->group_size > 4096) {
        RB_CUDA(cudaMemsetAsync(d_y, 0, (size_t)m->rows * 4, s));
        st = RABBIT_CUDA_OK;
    } else {
        st = launch_flat(m->raw, d_x, d_y, m->rows, m->in_dim, s);
    }
    return st == RABBIT_CUDA_OK ? ok() : st;
}

int rabbit_cuda_matrix_gemv(const rabbit_cuda_matrix *m, const float *x, float *y) {
    if (!m || !x || !y) return fail(RABBIT_CUDA_ERR_ARGS, "matrix_gemv: NULL argument");
    int st;
    DevCtx *c = dev_ctx(m->device, &st);
    if (!c) return st;
    std::lock_guard<std::mutex> g(c->mu);
    const size_t xb = align_up((size_t)m->in_dim * 4, 256), yb = (size_t)m->rows * 4;
    if ((st = ensure_dscratch(c, xb + yb)) != RABBIT_CUDA_OK) return st;
    if ((st = ensure_pinned(c, xb + yb)) != RABBIT_CUDA_OK) return st;
    float *dx = static_cast<float *>(c->dscratch);
    float *dy = reinterpret_cast<float *>(static_cast<uint8_t *>(c->dscratch) + xb);
    float *px = static_cast<float *>(c->pin);
    float *py = reinterpret_cast<float *>(static_cast<uint8_t *>(c->pin) + xb);
    memcpy(px, x, (size_t)m->in_dim * 4);
    cudaStream_t s = c->stream;
    RB_CUDA(cudaMemcpyAsync(dx, px, (size_t)m->in_dim * 4, cudaMemcpyHostToDevice, s));
    if ((st = rabbit_cuda_matrix_gemv_dev(m, dx, dy, s)) != RABBIT_CUDA_OK) return st;
    RB_CUDA(cudaMemcpyAsync(py, dy, yb, cudaMemcpyDeviceToHost, s));
    if ((st = check_device_error(c, s, "matrix_gemv")) != RABBIT_CUDA_OK) return st;
    memcpy(y, py, yb);
    return ok();
}

uint64_t rabbit_cuda_matrix_bytes(const rabbit_cuda_matrix *m) {
    if (!m) return 0;
    return (uint64_t)m->blob_bytes + 4ull * (uint64_t)m->in_dim + 4ull * (uint64_t)m->rows;
}

}  // extern "C"
