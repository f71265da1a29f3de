// rb_legacy.cu -- C ABI: the legacy per-tensor expert of src/moe.c:119-224
// (apply_expert) on the GPU, for models whose expert_quant is the older
// per-tensor int4 / int8 format (one fp32 scale per matrix).
//
// The record is read the way apply_expert reads it:
//   * three matrices (gate [I, H], up [I, H], down [H, I]) of [f32 scale |
//     payload], payload (I H + 1) / 2 bytes for quant 4 (int4, row o at
//     o (in + 1) / 2 bytes: element 2j the low nibble of byte j, 2j + 1 the
//     high one, value nibble - 8) and I H bytes otherwise (int8, quant 0
//     included); a stored scale that is not a positive finite number reads as
//     1/127 (moe.c:137-143); I = expert_dim, 2 H when 0, 2 H when above 4 H;
//     hidden += down(silu(gate) * up) with each matrix's
//     y[o] += weight * (sum_i w x_i) * scale (moe.c:7-35, weight 1 for gate
//     and up);
//   * a record too small for that: one square [H, H] matrix after an
//     optional scale, times weight * 0.05, or -- int8 only -- the matrix from
//     byte 0 with scale 1/127, or the first bytes as (b - 128) / 128 * 0.1
//     * weight (moe.c:183-220).
// Sums run over lanes and warps (fp32), not left to right: results agree
// with the reference within fp32 rounding, not bit for bit.
#include <math.h>
#include <string.h>

#include "rb_device.cuh"
#include "rb_runtime.h"

namespace rb {
namespace {

struct LegacyGemv {
    const uint8_t *W;        // row 0
    const uint8_t *scale_at; // the stored scale, or nullptr: 1/127
    const float *x;
    float *y;                // y[o] += weight * sum * scale
    int out_dim, in_dim, int4;
    float weight;
};

// moe.c:137-143 (bytes may sit at any alignment)
__device__ __forceinline__ float legacy_scale(const uint8_t *p) {
    if (!p) return 1.0f / 127.0f;
    const uint32_t u = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                       ((uint32_t)p[3] << 24);
    const float s = __uint_as_float(u);
    return (s > 0.0f && isfinite(s)) ? s : 1.0f / 127.0f;
}

// One warp per output row; 8 warps a CTA.
__global__ void __launch_bounds__(256) k_legacy_gemv(LegacyGemv g) {
    const int lane = threadIdx.x & 31;
    const int o = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (o >= g.out_dim) return;
    float sum = 0.f;
    if (g.int4) {
        const int in_bytes = (g.in_dim + 1) / 2;
        const uint8_t *row = g.W + (size_t)o * in_bytes;
        for (int j = lane; j < in_bytes; j += 32) {
            const uint32_t b = row[j];
            sum = fmaf((float)((int)(b & 15u) - 8), g.x[2 * j], sum);
            if (2 * j + 1 < g.in_dim) sum = fmaf((float)((int)(b >> 4) - 8), g.x[2 * j + 1], sum);
        }
    } else {
        const int8_t *row = reinterpret_cast<const int8_t *>(g.W) + (size_t)o * g.in_dim;
        for (int i = lane; i < g.in_dim; i += 32) sum = fmaf((float)row[i], g.x[i], sum);
    }
    sum = warp_sum(sum);
    if (lane == 0) g.y[o] += g.weight * sum * legacy_scale(g.scale_at);
}

// moe.c:162-166: mid = (g * sigmoid(g)) * up
__global__ void __launch_bounds__(256) k_legacy_silu(const float *gate, const float *up,
                                                     float *mid, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float gv = gate[i];
    const float sg = 1.0f / (1.0f + expf(-gv));
    mid[i] = (gv * sg) * up[i];
}

// moe.c:211-216: the first `usable` bytes as the expert's output
__global__ void __launch_bounds__(256) k_legacy_bytes(const uint8_t *bytes, int usable,
                                                      float weight, float *delta) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= usable) return;
    const float v = ((float)bytes[i] - 128.0f) / 128.0f;
    delta[i] = weight * v * 0.1f;
}

__global__ void __launch_bounds__(256) k_legacy_add(float *hidden, const float *delta, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) hidden[i] += delta[i];
}

cudaError_t gemv(const uint8_t *W, const uint8_t *scale_at, const float *x, float *y, int out_dim,
                 int in_dim, bool int4, float weight, cudaStream_t s) {
    LegacyGemv g{W, scale_at, x, y, out_dim, in_dim, int4 ? 1 : 0, weight};
    k_legacy_gemv<<<(out_dim + 7) / 8, 256, 0, s>>>(g);
    return cudaGetLastError();
}

// The body of both entry points: record and hidden in device memory.
int apply_dev(const uint8_t *rec, uint64_t size, int quant, int H, int expert_dim, float *hidden,
              float weight, cudaStream_t s) {
    const bool int4 = quant == 4;
    int inter = expert_dim > 0 ? expert_dim : H * 2;  // moe.c:126-128
    if (inter > H * 4) inter = H * 2;
    if (inter < 1) inter = H;
    const uint64_t mat = (uint64_t)inter * (uint64_t)H;
    const uint64_t payload3 = int4 ? (mat + 1) / 2 : mat;
    const bool swiglu = size >= 3 * (4 + payload3);
    // scratch: delta [H], and gate / up / mid [I] for the three-matrix form
    float *scr = nullptr;
    const size_t nscr = (size_t)H + (swiglu ? 3 * (size_t)inter : 0);
    RB_CUDA(cudaMallocAsync(reinterpret_cast<void **>(&scr), sizeof(float) * nscr, s));
    float *delta = scr;
    cudaError_t e = cudaMemsetAsync(scr, 0, sizeof(float) * nscr, s);
    if (e == cudaSuccess && swiglu) {  // moe.c:135-181
        float *gate = scr + H, *up = gate + inter, *mid = up + inter;
        const uint8_t *p = rec;
        const uint8_t *sc[3], *W[3];
        for (int part = 0; part < 3; ++part) {
            sc[part] = nullptr;
            if (size - (uint64_t)(p - rec) >= 4) {
                sc[part] = p;
                p += 4;
            }
            W[part] = p;
            p += payload3;
        }
        // int4 rows of an odd width run past their matrix's (I H + 1) / 2
        // bytes, as in the reference; past the record's end they are refused
        const uint64_t rg = int4 ? (uint64_t)(H + 1) / 2 : (uint64_t)H;
        const uint64_t rd = int4 ? (uint64_t)(inter + 1) / 2 : (uint64_t)inter;
        if ((uint64_t)(W[0] - rec) + inter * rg > size || (uint64_t)(W[1] - rec) + inter * rg > size ||
            (uint64_t)(W[2] - rec) + (uint64_t)H * rd > size) {
            cudaFreeAsync(scr, s);
            return fail(RABBIT_CUDA_ERR_FORMAT,
                        "legacy_apply_expert: int4 rows of odd width run past the record's end");
        }
        e = gemv(W[0], sc[0], hidden, gate, inter, H, int4, 1.0f, s);
        if (e == cudaSuccess) e = gemv(W[1], sc[1], hidden, up, inter, H, int4, 1.0f, s);
        if (e == cudaSuccess) {
            k_legacy_silu<<<(inter + 255) / 256, 256, 0, s>>>(gate, up, mid, inter);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = gemv(W[2], sc[2], mid, delta, H, inter, int4, weight, s);
    } else if (e == cudaSuccess) {  // moe.c:183-220
        const uint8_t *scale_at = nullptr, *W = rec;
        uint64_t payload = size;
        if (size >= 4 + (uint64_t)H) {
            scale_at = rec;
            W = rec + 4;
            payload = size - 4;
        }
        const float w = weight * 0.05f;
        const uint64_t sq = (uint64_t)H * (uint64_t)H;
        if (int4) {
            if (payload >= (uint64_t)H * (uint64_t)((H + 1) / 2))
                e = gemv(W, scale_at, hidden, delta, H, H, true, w, s);
        } else if (payload >= sq) {
            e = gemv(W, scale_at, hidden, delta, H, H, false, w, s);
        } else if (size >= sq) {
            e = gemv(rec, nullptr, hidden, delta, H, H, false, w, s);
        } else {
            const int usable = (int)(size < (uint64_t)H ? size : (uint64_t)H);
            if (usable > 0) {
                k_legacy_bytes<<<(usable + 255) / 256, 256, 0, s>>>(rec, usable, weight, delta);
                e = cudaGetLastError();
            }
        }
    }
    if (e == cudaSuccess) {
        k_legacy_add<<<(H + 255) / 256, 256, 0, s>>>(hidden, delta, H);
        e = cudaGetLastError();
    }
    const cudaError_t e2 = cudaFreeAsync(scr, s);
    if (e != cudaSuccess) return cuda_fail(e, "legacy_apply_expert");
    if (e2 != cudaSuccess) return cuda_fail(e2, "legacy_apply_expert: scratch");
    return RABBIT_CUDA_OK;
}

}  // namespace
}  // namespace rb

extern "C" {

int rabbit_cuda_legacy_apply_expert_dev(const void *d_record, uint64_t expert_size,
                                        int expert_quant, int hidden_dim, int expert_dim,
                                        float *d_hidden, float weight, void *stream) {
    if (!d_record || !d_hidden || hidden_dim <= 0)
        return rb::fail(RABBIT_CUDA_ERR_ARGS, "legacy_apply_expert: NULL record or hidden");
    int st = RABBIT_CUDA_OK;
    if (!rb::dev_ctx(rb::current_device(), &st)) return st;
    RB_CUDA(cudaSetDevice(rb::current_device()));
    st = rb::apply_dev(static_cast<const uint8_t *>(d_record), expert_size, expert_quant,
                       hidden_dim, expert_dim, d_hidden, weight,
                       static_cast<cudaStream_t>(stream));
    return st ? st : rb::ok();
}

int rabbit_cuda_legacy_apply_expert(const void *record, uint64_t expert_size, int expert_quant,
                                    int hidden_dim, int expert_dim, float *hidden, float weight) {
    if (!record || !hidden || hidden_dim <= 0)
        return rb::fail(RABBIT_CUDA_ERR_ARGS, "legacy_apply_expert: NULL record or hidden");
    int st = RABBIT_CUDA_OK;
    rb::DevCtx *ctx = rb::dev_ctx(rb::current_device(), &st);
    if (!ctx) return st;
    std::lock_guard<std::mutex> g(ctx->mu);
    RB_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const size_t hb = sizeof(float) * (size_t)hidden_dim;
    const size_t rb_bytes = (expert_size + 15) / 16 * 16;
    if ((st = rb::ensure_dscratch(ctx, rb_bytes + hb)) != RABBIT_CUDA_OK) return st;
    uint8_t *d_rec = static_cast<uint8_t *>(ctx->dscratch);
    float *d_h = reinterpret_cast<float *>(d_rec + rb_bytes);
    RB_CUDA(cudaMemcpyAsync(d_rec, record, expert_size, cudaMemcpyHostToDevice, s));
    RB_CUDA(cudaMemcpyAsync(d_h, hidden, hb, cudaMemcpyHostToDevice, s));
    st = rb::apply_dev(d_rec, expert_size, expert_quant, hidden_dim, expert_dim, d_h, weight, s);
    if (st) return st;
    RB_CUDA(cudaMemcpyAsync(hidden, d_h, hb, cudaMemcpyDeviceToHost, s));
    RB_CUDA(cudaStreamSynchronize(s));
    return rb::ok();
}

}  // extern "C"
