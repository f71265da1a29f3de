// rb_gemv.cu -- group-32 int4 GEMV on B200.
//
// Streaming kernel (k_gemv_g32), one persistent CTA per SM, contiguous row
// range per CTA:
//   warp CW (producer): one lane issues cp.async.bulk copies of row chunks
//       (nibbles + scales) into a ring of shared-memory stages, gated by
//       full/empty mbarriers; x is bulk-copied once.
//   warps 0..CW-1 (consumers): warp w owns k-slice w % KS (lane = one group
//       of 32 inputs, x for that group held in 32 registers for the whole
//       kernel) and row subset w / KS. Each lane computes its group's dot
//       product on packed fp32, scales it, and eight rows at a time are
//       reduced across the warp with a transposed butterfly. Partials per
//       (row, k-slice) go to shared memory and are summed once at the end.
// Arithmetic: per group, sum_i (q_i/64) x_i, times 64*scale; rows summed over
// groups in a fixed order (within tolerance of the reference's serial fp32
// sum, quant.c:181-184).
#include "rb_gemv.cuh"
#include "rb_runtime.h"

namespace rb {

bool plan_g32(int rows, int in_dim, int sm_count, G32Plan *p) {
    if (rows <= 0 || !g32_ok(in_dim)) return false;
    const int G = in_dim / 32;
    p->rows = rows;
    p->in_dim = in_dim;
    p->units = (rows + 3) / 4;
    p->KS = (G + 31) / 32;
    p->RS = p->KS >= 8 ? 1 : 8 / p->KS;
    const size_t row_bytes = (size_t)in_dim / 2 + (size_t)in_dim / 8;
    int cr = (int)((32 * 1024) / row_bytes) / 4 * 4;
    if (cr < 4) cr = 4;
    if (cr > 64) cr = 64;
    p->CR = cr;
    p->slot_bytes = (uint32_t)align_up((size_t)cr * row_bytes, 128);
    p->grid = p->units < sm_count ? p->units : sm_count;
    p->rows_cta_max = 4 * ((p->units + p->grid - 1) / p->grid);
    const int CW = p->KS * p->RS;
    p->block = (CW + 1) * 32;
    const size_t fixed = align_up((size_t)in_dim * 4, 128) +
                         align_up((size_t)p->rows_cta_max * p->KS * 4, 16);
    int ns = (int)((kMaxDynSmem - fixed - 8 * 64) / p->slot_bytes);
    if (ns > 16) ns = 16;
    if (ns < 2) return false;
    p->nslots = ns;
    p->smem = fixed + (size_t)ns * p->slot_bytes + 8 * (2 * ns + 1);
    return p->smem <= (size_t)kMaxDynSmem;
}

__global__ void __launch_bounds__(17 * 32, 1) k_gemv_g32(G32Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int CW = a.KS * a.RS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int in = a.in_dim, G = in >> 5;
    const int half = in >> 1;  // nibble bytes per row

    float *xs = reinterpret_cast<float *>(smem);
    uint8_t *ring = smem + align_up((size_t)in * 4, 128);
    float *part = reinterpret_cast<float *>(ring + (size_t)a.nslots * a.slot_bytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(
        reinterpret_cast<uint8_t *>(part) + align_up((size_t)a.rows_cta_max * a.KS * 4, 16));
    uint64_t *empty = full + a.nslots;
    uint64_t *xbar = empty + a.nslots;

    const int u0 = (int)((long long)blockIdx.x * a.units / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * a.units / gridDim.x);
    const int r0 = 4 * u0, r1 = 4 * u1, nrows = r1 - r0;
    const int nchunks = (nrows + a.CR - 1) / a.CR;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init(xbar, 1);
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == CW) {  // ---------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            mbar_arrive_expect_tx(xbar, (uint32_t)in * 4);
            bulk_g2s(xs, a.x, (uint32_t)in * 4, xbar, pol_x);
            int issued = 0;
            for (int i = 0; i < nchunks; ++i) {
                const int s = i % a.nslots, n = i / a.nslots;
                if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.wait_ns, a.err)) break;
                const int row0 = r0 + i * a.CR;
                const int rows = min(a.CR, r1 - row0);
                const uint32_t nb = (uint32_t)rows * half, sb = (uint32_t)rows * (in >> 3);
                uint8_t *dst = ring + (size_t)s * a.slot_bytes;
                mbar_arrive_expect_tx(&full[s], nb + sb);
                bulk_g2s(dst, a.nib + (size_t)row0 * half, nb, &full[s], pol_w);
                bulk_g2s(dst + (size_t)a.CR * half, a.sc + (size_t)row0 * G, sb, &full[s], pol_w);
                ++issued;
            }
            // Never leave the CTA while a copy we issued may still be landing.
            mbar_wait(xbar, 0, a.wait_ns, a.err);
            for (int i = issued > a.nslots ? issued - a.nslots : 0; i < issued; ++i)
                mbar_wait(&full[i % a.nslots], (i / a.nslots) & 1, a.wait_ns, a.err);
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int ks = warp % a.KS, rsub = warp / a.KS;
    const int g = ks * 32 + lane;
    const bool active = g < G;
    // A wait that runs out marks the CTA failed; every consumer still reaches
    // the named barrier below (a warp that left would stall the others).
    bool good = __all_sync(0xffffffffu, mbar_wait(xbar, 0, a.wait_ns, a.err));
    float xr[32];
    if (active) {
        const float4 *xp = reinterpret_cast<const float4 *>(xs + g * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 t = xp[j];
            xr[4 * j] = t.x;
            xr[4 * j + 1] = t.y;
            xr[4 * j + 2] = t.z;
            xr[4 * j + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) xr[j] = 0.f;
    }

    for (int i = 0; good && i < nchunks; ++i) {
        const int s = i % a.nslots, n = i / a.nslots;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], n & 1, a.wait_ns, a.err))) {
            good = false;
            break;
        }
        const int row0 = r0 + i * a.CR;
        const int rows = min(a.CR, r1 - row0);
        const uint8_t *sn = ring + (size_t)s * a.slot_bytes;
        const float *ss = reinterpret_cast<const float *>(sn + (size_t)a.CR * half);
        for (int rb = rsub; rb < rows; rb += 8 * a.RS) {
            float v[8];
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const int r = rb + b * a.RS;
                v[b] = 0.f;
                if (active && r < rows) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(sn + (size_t)r * half + g * 16);
                    const float sc64 = ss[r * G + g] * 64.f;
                    v[b] = dot32_q64(w, xr) * sc64;
                }
            }
            const float tot = warp_reduce8(v);
            if ((lane & 3) == 0) {
                const int r = rb + (lane >> 2) * a.RS;
                if (r < rows) part[(row0 - r0 + r) * a.KS + ks] = tot;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    named_sync(1, CW * 32);
    if (!good) return;
    for (int lr = threadIdx.x; lr < nrows; lr += CW * 32) {
        const int row = r0 + lr;
        if (row < a.rows) {
            float acc = 0.f;
            for (int k = 0; k < a.KS; ++k) acc += part[lr * a.KS + k];
            a.y[row] = acc;
        }
    }
}

// --------------------------------------------------------- flat kernels --
__device__ __forceinline__ uint32_t ld_u32_any(const uint8_t *p) {
    if ((reinterpret_cast<uintptr_t>(p) & 3) == 0) return *reinterpret_cast<const uint32_t *>(p);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
           ((uint32_t)p[3] << 24);
}

// One warp per output row; element order and group index follow the flat
// row-major index exactly as quant.c:171-185 does, so groups may straddle
// rows and n may be odd.
__global__ void k_gemv_flat(const uint8_t *blob, const float *x, float *y, int out_dim,
                            int in_dim) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= out_dim) return;
    const uint32_t gs = ld_u32_any(blob);
    if (gs == 0 || gs > 4096) {
        if (lane == 0) y[row] = 0.f;
        return;
    }
    const long long n = (long long)out_dim * in_dim;
    const long long ng = (n + gs - 1) / gs;
    const uint8_t *scales = blob + 4;
    const uint8_t *nib = blob + 4 + 4 * ng;
    float acc = 0.f;
    for (int i = lane; i < in_dim; i += 32) {
        const long long flat = (long long)row * in_dim + i;
        const uint8_t b = nib[flat >> 1];
        const int q = (int)((flat & 1) ? (b >> 4) : (b & 15)) - 8;
        const float s = __uint_as_float(ld_u32_any(scales + 4 * (flat / gs)));
        acc += __fmul_rn((float)q, s) * x[i];
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

// dst[i] = (float)q_i * scale[i / gs], rounded once (bit-identical to
// quant.c:134-140).
__global__ void k_dequant_flat(const uint8_t *blob, float *dst, long long n, uint32_t gs) {
    const long long ng = (n + gs - 1) / gs;
    const uint8_t *scales = blob + 4;
    const uint8_t *nib = blob + 4 + 4 * ng;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const uint8_t b = nib[i >> 1];
        const int q = (int)((i & 1) ? (b >> 4) : (b & 15)) - 8;
        dst[i] = __fmul_rn((float)q, __uint_as_float(ld_u32_any(scales + 4 * (i / gs))));
    }
}

}  // namespace rb
