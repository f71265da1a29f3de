// rb_gemv.cu -- group-32 int4 GEMV on B200.
//
// Streaming kernel (k_gemv_g32), one persistent CTA per SM, a contiguous
// range of row tiles per CTA (tile = TR rows of nibbles + scales, one
// contiguous block in HBM):
//   warp CW (producer): one lane issues one cp.async.bulk per tile into a
//       ring of shared-memory stages, gated by full/empty mbarriers.
//   warps 0..CW-1 (consumers, at most eight): warp w owns k-slice w % KS
//       (lane = J groups of 32 inputs, held as integer planes in registers
//       for the whole kernel) and ROWS rows of every tile from
//       (w / KS) * ROWS. ROWS and J are compile-time, so a warp does exactly
//       its ROWS x J dots per tile: it loads them, releases the stage, then
//       computes, and the ROWS values are reduced across the warp together
//       with a transposed butterfly.
//       Partials per (row, k-slice) go to shared memory and are summed once
//       at the end.
// Arithmetic: per group an exact integer dot of the nibbles with the
// activations' 23-bit block-floating-point planes (dp4a), times the group
// scale; rows summed over groups in a fixed order (within tolerance of the
// reference's serial fp32 sum, quant.c:181-184).
#include <string.h>

#include <algorithm>

#include "rb_gemv.cuh"
#include "rb_runtime.h"

namespace rb {

#ifdef RB_PHASE_TIMERS
// Diagnostic build only: for CTA 0 of each launch, %globaltimer at kernel
// start, after the wait for the preceding kernel, at the first tile and at
// the end; a ring of 64 launches.
__device__ uint64_t g_gemv_ns[64 * 4];
__device__ unsigned g_gemv_launch;
#define RB_GEMV_STAMP(slot, k)                                              \
    do {                                                                    \
        if (blockIdx.x == 0 && threadIdx.x == 0)                            \
            g_gemv_ns[((slot) & 63) * 4 + (k)] = globaltimer_ns();          \
    } while (0)
#else
#define RB_GEMV_STAMP(slot, k) \
    do {                       \
    } while (0)
#endif

// Per-SM streaming rate and fixed cost of one bulk copy issued by one
// thread, used to size tiles (measured on B200: 16-40 KB single copies stream
// at 6.6-7 TB/s; 8 KB copies from one issuing thread at ~3.3 TB/s, i.e.
// ~0.35 us per copy per SM).
constexpr double kSmBytesPerUs = 44.0e3;
constexpr double kCopyUs = 0.35;
// Consumer-side fixed work per tile (wait, release, cross-lane reduction,
// partial stores), not hidden behind the copies.
constexpr double kTileFixedUs = 0.15;
const double kTileSmBytesPerUs = kSmBytesPerUs, kTileCopyUs = kCopyUs;

int choose_rows(int rows, int mats, bool spread, int ctas, size_t row_bytes, int NG, int max_rows,
                size_t max_bytes) {
    int best = 1;
    double best_cost = 1e30;
    for (int R = 1; R <= max_rows; R *= 2) {
        const int TR = NG * R;
        if (R > 1 && (size_t)TR * row_bytes > max_bytes) break;
        const long long tiles = (rows + TR - 1) / TR;
        const long long per =
            spread ? (mats * tiles + ctas - 1) / ctas : mats * ((tiles + ctas - 1) / ctas);
        const double cost = std::max((double)per * TR * row_bytes / kSmBytesPerUs, per * kCopyUs) +
                             per * kTileFixedUs;
        if (cost < best_cost * 0.98 || (cost <= best_cost * 1.02 && R > best)) {
            if (cost < best_cost) best_cost = cost;
            best = R;
        }
    }
    return best;
}

void tile_blob_host(const uint8_t *blob, const Tiling &t, uint8_t *dst) {
    const size_t n = (size_t)t.rows * t.in_dim;
    const size_t half = t.in_dim / 2, scb = t.in_dim / 8;  // bytes per row
    const size_t chalf = t.cols / 2, cscb = t.cols / 8;    // bytes per row of one chunk
    const uint8_t *sc = blob + 4;
    const uint8_t *nib = blob + 4 + n / 32 * 4;
    for (int c = 0; c < t.KC; ++c)
        for (int ti = 0; ti < t.rtiles; ++ti) {
            uint8_t *d = dst + (size_t)(c * t.rtiles + ti) * t.tile_stride;
            const int r0 = ti * t.TR, nr = std::min(t.TR, t.rows - r0);
            memset(d, 0, t.tile_stride);
            if (t.KC == 1) {
                memcpy(d, nib + (size_t)r0 * half, (size_t)nr * half);
                memcpy(d + (size_t)t.TR * half, sc + (size_t)r0 * scb, (size_t)nr * scb);
                continue;
            }
            for (int r = 0; r < nr; ++r) {
                memcpy(d + (size_t)r * chalf, nib + (size_t)(r0 + r) * half + c * chalf, chalf);
                memcpy(d + (size_t)t.TR * chalf + (size_t)r * cscb,
                       sc + (size_t)(r0 + r) * scb + c * cscb, cscb);
            }
        }
}

void tile_pair_host(const uint8_t *a, const uint8_t *b, const Tiling &t2, uint8_t *dst) {
    const size_t n = (size_t)t2.rows * t2.in_dim;
    const size_t half = t2.in_dim / 2, scb = t2.in_dim / 8;
    const uint8_t *srcs[2] = {a, b};
    for (int ti = 0; ti < t2.ntiles; ++ti) {
        uint8_t *d = dst + (size_t)ti * t2.tile_stride;
        const int r0 = ti * t2.TR, nr = std::min(t2.TR, t2.rows - r0);
        memset(d, 0, t2.tile_stride);
        for (int m = 0; m < 2; ++m) {
            const uint8_t *sc = srcs[m] + 4;
            const uint8_t *nib = srcs[m] + 4 + n / 32 * 4;
            memcpy(d + (size_t)m * t2.TR * half, nib + (size_t)r0 * half, (size_t)nr * half);
            memcpy(d + 2 * (size_t)t2.TR * half + (size_t)m * t2.TR * scb, sc + (size_t)r0 * scb,
                   (size_t)nr * scb);
        }
    }
}

bool plan_g32(int rows, int in_dim, int sm_count, G32Plan *p) {
    if (rows <= 0 || !g32_ok(in_dim)) return false;
    const int G = in_dim / 32;
    p->J = lane_groups(G);
    p->KS = kslices(G, p->J);
    p->NG = std::max(1, kConsumerWarps / p->KS);
    const size_t row_bytes = (size_t)in_dim / 2 + (size_t)in_dim / 8;
    p->ROWS = choose_rows(rows, 1, true, sm_count, row_bytes, p->NG, 8 / p->J, 48 * 1024);
    const int TR = p->NG * p->ROWS;
    p->til = make_tiling(rows, in_dim, TR);
    return plan_g32_batch(*p, 1, sm_count, p);
}

bool plan_g32_batch(const G32Plan &one, int nmat, int sm_count, G32Plan *p) {
    *p = one;
    const long long total = (long long)nmat * p->til.ntiles;
    p->grid = total < sm_count ? (int)total : sm_count;
    p->tiles_cta_max = (int)((total + p->grid - 1) / p->grid);
    const int CW = p->KS * p->NG, TR = p->til.TR;
    p->block = (CW + 1) * 32;
    const size_t part = align_up((size_t)p->tiles_cta_max * TR * p->KS * 4, 16);
    // J == 1: two CTAs per SM (consecutive launches overlap), 113 KB each
    const long long cap = p->J == 1 ? 113 * 1024 : kMaxDynSmem;
    long long ns = (cap - (long long)part - 16 * 24 - 128) / p->til.tile_stride;
    if (ns > 24) ns = 24;
    if (ns < 2) return false;
    p->nslots = (int)ns;
    p->smem = (size_t)ns * p->til.tile_stride + part + 16 * (size_t)ns + 4 * 32;
    return p->smem <= (size_t)cap;
}

// The consumer loop of one warp over the CTA's tiles [t0, t0 + nt) of the
// launch's matrix-major tile range: ROWS rows of every tile starting at
// rbase, J groups per lane, x planes (re)built when the matrix changes (once
// if x is shared). False when a wait ran out.
template <int J, int ROWS>
__device__ __forceinline__ bool gemv_tiles(const G32Args &a, const uint8_t *ring, float *part,
                                           uint64_t *full, uint64_t *empty, uint32_t *sink,
                                           int t0, int nt, int ks, int rbase, int g0,
                                           const bool (&act)[J]) {
    const int G = a.til.in_dim >> 5, half = a.til.in_dim >> 1, TR = a.til.TR, KS = a.KS;
    const uint32_t stride = a.til.tile_stride;
    XPlanes xg[J];
    int mcur = -1, m = t0 / a.til.ntiles, tin = t0 - m * a.til.ntiles;
    for (int i = 0; i < nt; ++i, ++tin) {
        if (tin == a.til.ntiles) {
            tin = 0;
            ++m;
        }
        if (m != mcur && (mcur < 0 || !a.shared_x)) {
#pragma unroll
            for (int j = 0; j < J; ++j)
                load_xplanes_global(xg[j], a.x[m] + (size_t)(g0 + 32 * j) * 32, act[j]);
        }
        mcur = m;
        const int s = i % a.nslots, n = i / a.nslots;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], n & 1, a.wait_ns, a.err))) return false;
        const int lb = i * TR + rbase;
        chunk_dot<1, ROWS, J>(ring + (size_t)s * stride, TR, rbase, half, G, g0, act, xg,
                              [=](int, int r) { return (lb + r) * KS + ks; }, part, &empty[s],
                              1u, sink);
    }
    return true;
}

// J == 1 (rows up to 8192 inputs): two CTAs per SM (<= 113 KB of shared
// memory, <= 113 registers a thread), so a launch that follows this one on
// the stream can stream its weights while this one finishes.
template <int J>
__global__ void __launch_bounds__((kConsumerWarps + 1) * 32, J == 1 ? 2 : 1) k_gemv_g32(G32Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int CW = a.KS * a.NG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.til.in_dim >> 5;
#ifdef RB_PHASE_TIMERS
    unsigned slot = 0;
    if (blockIdx.x == 0 && threadIdx.x == 0) slot = atomicAdd(&g_gemv_launch, 1u);
#endif
    RB_GEMV_STAMP(slot, 0);
    const int TR = a.til.TR;
    const uint32_t stride = a.til.tile_stride;

    uint8_t *ring = smem;
    float *part = reinterpret_cast<float *>(ring + (size_t)a.nslots * stride);
    uint64_t *full = reinterpret_cast<uint64_t *>(
        reinterpret_cast<uint8_t *>(part) + align_up((size_t)a.tiles_cta_max * TR * a.KS * 4, 16));
    uint64_t *empty = full + a.nslots;
    uint32_t *sink = reinterpret_cast<uint32_t *>(empty + a.nslots);  // one word per warp

    const long long total = (long long)a.nmat * a.til.ntiles;  // matrix-major tile range
    const int t0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int t1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    const int nt = t1 - t0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);  // every consumer warp releases every stage
        }
        mbar_init_fence();
    }
    // The next kernel on the stream may launch now; it waits for this one to
    // complete before it touches its own x / y (wait_prerequisite below).
    launch_dependents();
    __syncthreads();

    if (warp == CW) {  // ---------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int issued = 0;
            int m = t0 / a.til.ntiles, tin = t0 - m * a.til.ntiles;
            for (int i = 0; i < nt; ++i, ++tin) {
                if (tin == a.til.ntiles) {
                    tin = 0;
                    ++m;
                }
                const int s = i % a.nslots, n = i / a.nslots;
                if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.wait_ns, a.err, 0)) break;
                mbar_arrive_expect_tx(&full[s], a.til.tile_bytes);
                bulk_g2s(ring + (size_t)s * stride, a.tiles[m] + (size_t)tin * stride,
                         a.til.tile_bytes, &full[s], pol);
                ++issued;
            }
            // Never leave the CTA while a copy we issued may still be landing.
            for (int i = issued > a.nslots ? issued - a.nslots : 0; i < issued; ++i)
                mbar_wait(&full[i % a.nslots], (i / a.nslots) & 1, a.wait_ns, a.err);
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    // Warp group q = warp / KS (KS warps cover one row, J groups of 32
    // inputs per lane) takes rows [q*ROWS, (q+1)*ROWS) of every tile. Every
    // consumer waits for and releases every stage, so the ring's phases stay
    // in step.
    const int ks = warp % a.KS, grp = warp / a.KS;
    const int g0 = ks * 32 * J + lane;
    bool act[J];
#pragma unroll
    for (int j = 0; j < J; ++j) act[j] = g0 + 32 * j < G;
    // x may be the output of the preceding kernel, and y may still be read by
    // it: nothing below touches either before that kernel has completed. The
    // weights (uploaded by copies, not written by a kernel) are already
    // streaming in.
    wait_prerequisite();
    RB_GEMV_STAMP(slot, 1);
    const int rbase = grp * a.ROWS;
    // A wait that runs out marks the CTA failed; every consumer still reaches
    // the named barrier below (a warp that left would stall the others).
    bool good;
    switch (a.ROWS) {
        case 1: good = gemv_tiles<J, 1>(a, ring, part, full, empty, sink + warp, t0, nt, ks, rbase, g0, act); break;
        case 2: good = gemv_tiles<J, 2>(a, ring, part, full, empty, sink + warp, t0, nt, ks, rbase, g0, act); break;
        case 4: good = gemv_tiles<J, 4>(a, ring, part, full, empty, sink + warp, t0, nt, ks, rbase, g0, act); break;
        // ROWS * J <= 8 (the planner never asks for more)
        default: good = gemv_tiles<J, 8 / J>(a, ring, part, full, empty, sink + warp, t0, nt, ks, rbase, g0, act); break;
    }
    RB_GEMV_STAMP(slot, 2);
    named_sync(1, CW * 32);
    if (!good) return;
    for (int lr = threadIdx.x; lr < nt * TR; lr += CW * 32) {
        const int gt = t0 + lr / TR, m = gt / a.til.ntiles;
        const int row = (gt - m * a.til.ntiles) * TR + lr % TR;
        if (row < a.til.rows) {
            float acc = 0.f;
            for (int k = 0; k < a.KS; ++k) acc += part[lr * a.KS + k];
            a.y[m][row] = acc;
        }
    }
    RB_GEMV_STAMP(slot, 3);
}

#ifdef RB_PHASE_TIMERS
}  // namespace rb
extern "C" __attribute__((visibility("default"))) int rabbit_cuda_debug_gemv_ns(uint64_t *out) {
    return cudaMemcpyFromSymbol(out, rb::g_gemv_ns, sizeof(uint64_t) * 256) == cudaSuccess ? 0 : 6;
}
namespace rb {
#endif

const void *gemv_g32_kernel(int J) {
    return J == 2 ? (const void *)k_gemv_g32<2> : (const void *)k_gemv_g32<1>;
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
