// rb_moe_kernels.cu -- MoE decode on B200: one token through one layer's
// routed + shared SwiGLU experts (forward_v2.c:280-402).
//
// Fused group-32 kernel (k_moe_decode_g32), cooperative launch, one CTA per SM:
//   A. every CTA: rmsnorm(h) -> xn in shared memory; CTA c computes router
//      rows c, c+grid, ... -> scores.            [grid barrier 1]
//      every CTA: top-k + softmax on the scores (identical in all CTAs), the
//      active slot list (routed in rank order, then shared experts).
//   B. gate/up: the active slots' GU tiles (TRb rows of gate and of up,
//      nibbles + scales, one contiguous block) dealt out evenly over the
//      CTAs; the producer warp bulk-copies them into the shared-memory ring;
//      eight consumer warps dot them against xn held in registers (JB groups
//      of 32 per lane, ROWSb rows per warp group and tile, both fixed at
//      compile time); mid = silu(gate) * up goes to global scratch.
//   C. down + combine: each CTA owns D tiles (TRc rows of the H outputs) for
//      every active slot; the producer keeps issuing these W2 chunks as soon as
//      ring stages free up -- before and during grid barrier 2 -- so the down
//      weights are in flight while the last gate/up rows finish. Consumers
//      reload x = mid[slot] per slot and combine h_out = h + sum_j w_j down_j
//      in slot order (forward_v2.c:356-357, 398-399).
// Every wait (mbarrier or grid barrier) is bounded by a %globaltimer limit;
// a timeout records RB_ERR_TIMEOUT and the CTA drains its copies and exits.
#include "rb_gemv.cuh"
#include "rb_moe.cuh"

namespace rb {

#ifdef RB_PHASE_TIMERS
// Diagnostic build only: per-CTA %globaltimer stamps at phase boundaries, and
// for CTA 0 the producer's issue time and consumer warp 0's wait / ready /
// done times of each of the first 64 chunks.
__device__ uint64_t g_phase_ns[1024 * 8];
__device__ uint64_t g_chunk_ns[4 * 64];
#define RB_CHUNK(kind, i)                                                              \
    do {                                                                               \
        if (blockIdx.x == 0 && (i) < 64) g_chunk_ns[(kind) * 64 + (i)] = globaltimer_ns(); \
    } while (0)
#define RB_STAMP(i)                                                        \
    do {                                                                   \
        if (threadIdx.x == 0) g_phase_ns[blockIdx.x * 8 + (i)] = globaltimer_ns(); \
    } while (0)
#else
#define RB_STAMP(i) \
    do {            \
    } while (0)
#define RB_CHUNK(kind, i) \
    do {                  \
    } while (0)
#endif

// ---------------------------------------------------------- grid barrier --
// One thread per CTA. *count is a monotonic 64-bit arrival counter (zeroed at
// pool creation and after any failed wait); every barrier adds exactly
// gridDim.x, so the round ends at the next multiple of nblocks. One
// release-atomic to arrive, acquire loads to wait: a single L2 round trip on
// the critical path.
__device__ bool grid_barrier(unsigned long long *count, unsigned nblocks, uint64_t wait_ns,
                             int *err) {
    unsigned long long old;
    asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(count) : "memory");
    const unsigned long long target = old - old % nblocks + nblocks;
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 0;; ++it) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(count) : "memory");
        if (v >= target) return true;
        if ((it & 15u) == 15u && globaltimer_ns() - t0 > wait_ns) {
            set_error(err, RB_ERR_TIMEOUT);
            return false;
        }
    }
}

// --------------------------------------------------------------- top-k ----
// forward_v2.c:248-278: insertion into a descending list seeded (-1, -1e30),
// strict '>' (lower index wins ties, NaN never enters), softmax over the k.
__device__ void topk_softmax(const float *scores, int E, int k, int *ids, float *w) {
    for (int i = 0; i < k; ++i) {
        ids[i] = -1;
        w[i] = -1e30f;
    }
    for (int e = 0; e < E; ++e) {
        const float s = scores[e];
        int slot = 0;
        while (slot < k && !(s > w[slot])) ++slot;
        if (slot == k) continue;
        for (int j = k - 1; j > slot; --j) {
            ids[j] = ids[j - 1];
            w[j] = w[j - 1];
        }
        ids[slot] = e;
        w[slot] = s;
    }
    float m = w[0];
    for (int i = 1; i < k; ++i)
        if (w[i] > m) m = w[i];
    float z = 0.f;
    for (int i = 0; i < k; ++i) {
        w[i] = expf(w[i] - m);
        z += w[i];
    }
    if (z > 0.f)
        for (int i = 0; i < k; ++i) w[i] = w[i] / z;
}

// Active slot list: routed experts in rank order, then shared experts with
// weight 1 (forward_v2.c:384-396). Returns the count.
__device__ int build_slots(const int *ids, const float *w, int k, int E, int S, int rec_base,
                           int n_local, int usable, int *rec, float *wt) {
    int n = 0;
    if (!usable) return 0;
    for (int i = 0; i < k; ++i)
        if (ids[i] >= 0 && ids[i] < n_local) {
            rec[n] = rec_base + ids[i];
            wt[n] = w[i];
            ++n;
        }
    for (int s = 0; s < S; ++s)
        if (E + s < n_local) {
            rec[n] = rec_base + E + s;
            wt[n] = 1.0f;
            ++n;
        }
    return n;
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float sg = 1.0f / (1.0f + expf(-g));  // forward_v2.c:327-331
    return (g * sg) * u;
}

// Release a stage this warp has no rows of (its wait has completed).
__device__ __forceinline__ void release_stage(uint64_t *empty) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive_cnt(empty, 1);
}

// Phase B for one consumer warp: the CTA's units [ub0, ub1) (slot, GU tile),
// ROWS rows of gate and of up per tile from rbase. `i` counts ring stages.
template <int J, int ROWS>
__device__ __forceinline__ bool moe_gate_up(const MoeFusedArgs &a, const uint8_t *ring,
                                            float *part, uint64_t *full, uint64_t *empty,
                                            uint32_t *sink, int ub0, int ub1, int &i, int ks,
                                            int rbase, bool mine, int g0, const bool (&act)[J],
                                            const XPlanes (&xg)[J]) {
    const int KS = a.KSb, TRb = a.tb.TR, Hh = a.H >> 1, Gb = a.H >> 5;
    for (int u = ub0; u < ub1; ++u, ++i) {
        const int s = i % a.nslots, n = i / a.nslots;
        if (threadIdx.x == 0) RB_CHUNK(1, i);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], n & 1, a.wait_ns, a.err))) return false;
        if (threadIdx.x == 0) RB_CHUNK(2, i);
        const int lb = (u - ub0) * TRb + rbase;
        if (mine)
            chunk_dot<2, ROWS, J>(ring + (size_t)s * a.slot_bytes, TRb, rbase, Hh, Gb, g0, act, xg,
                                  [=](int m, int r) { return ((lb + r) * 2 + m) * KS + ks; },
                                  part, &empty[s], 1u, sink);
        else
            release_stage(&empty[s]);
        if (threadIdx.x == 0) RB_CHUNK(3, i);
    }
    return true;
}

// Phase C for one consumer warp: for every active slot, the CTA's D tiles
// [c0, c1), ROWS rows of each from rbase, x = mid of the slot.
template <int J, int ROWS>
__device__ __forceinline__ bool moe_down(const MoeFusedArgs &a, const uint8_t *ring, float *part,
                                         uint64_t *full, uint64_t *empty, uint32_t *sink,
                                         int nact, int c0, int c1, int &i, int ks, int rbase,
                                         bool mine, int g0, const bool (&act)[J]) {
    const int KS = a.KSc, TRc = a.tc.TR, Ih = a.I >> 1, Gc = a.I >> 5;
    XPlanes xg[J];
    for (int j = 0; j < nact; ++j) {
        // x = mid of this slot (written by all CTAs before grid barrier 2)
#pragma unroll
        for (int q = 0; q < J; ++q)
            load_xplanes_global(xg[q], a.mid + (size_t)j * a.I + (size_t)(g0 + 32 * q) * 32, act[q]);
        for (int t = c0; t < c1; ++t, ++i) {
            const int s = i % a.nslots, n = i / a.nslots;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[s], n & 1, a.wait_ns, a.err)))
                return false;
            const int lb = (t - c0) * TRc + rbase;
            if (mine)
                chunk_dot<1, ROWS, J>(ring + (size_t)s * a.slot_bytes, TRc, rbase, Ih, Gc, g0, act,
                                      xg, [=](int, int r) { return ((lb + r) * nact + j) * KS + ks; },
                                      part, &empty[s], 1u, sink);
            else
                release_stage(&empty[s]);
        }
    }
    return true;
}

template <int JB, int JC>
__global__ void __launch_bounds__((kConsumerWarps + 1) * 32, 1) k_moe_decode_g32(MoeFusedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nthr = blockDim.x;
    const int H = a.H, I = a.I, CW = a.CW;
    const int Gb = H >> 5, Gc = I >> 5;

    size_t off = 0;
    float *xn = reinterpret_cast<float *>(smem);  // padded: 33 floats per group of 32
    off = align_up((size_t)Gb * 33 * 4, 128);
    float *red = reinterpret_cast<float *>(smem + off);
    off += 128;
    int *s_rec = reinterpret_cast<int *>(smem + off);
    off += kMaxSlots * 4;
    float *s_w = reinterpret_cast<float *>(smem + off);
    off += kMaxSlots * 4;
    int *s_misc = reinterpret_cast<int *>(smem + off);  // [0] nact [1] abort A [2] abort B
    off = align_up(off + 16, 128);
    float *s_sc = reinterpret_cast<float *>(smem + off);  // router scores for top-k
    off = align_up(off + (size_t)a.E * 4, 128);
    uint8_t *ring = smem + off;
    off += (size_t)a.nslots * a.slot_bytes;
    float *part = reinterpret_cast<float *>(smem + off);
    off += align_up((size_t)a.part_floats * 4, 16);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + off);
    uint64_t *empty = full + a.nslots;
    uint32_t *sink = reinterpret_cast<uint32_t *>(empty + a.nslots);  // one word per warp

    RB_STAMP(0);
    if (tid == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);  // every consumer warp releases every stage
        }
        mbar_init_fence();
    }

    // ------------------------------------------------ A: rmsnorm + router --
    float ss = 0.f;
    for (int i = tid; i < H; i += nthr) {
        const float v = a.h_in[i];
        ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < (nthr >> 5); ++w) t += red[w];
        t /= (float)H;
        red[31] = 1.0f / sqrtf(t + 1e-5f);  // forward_v2.c:61-69
    }
    __syncthreads();
    const float inv = red[31];
    for (int i = tid; i < H; i += nthr) xn[xpad(i)] = (a.h_in[i] * inv) * a.rms[i];
    __syncthreads();
    for (int e = blockIdx.x; e < a.E; e += gridDim.x) {
        const float *wr = a.router + (size_t)e * H;
        float d = 0.f;
        for (int i = tid; i < H; i += nthr) d += wr[i] * xn[xpad(i)];
        d = warp_sum(d);
        if (lane == 0) red[warp] = d;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int w = 0; w < (nthr >> 5); ++w) t += red[w];
            a.scores[e] = t;
        }
        __syncthreads();
    }
    RB_STAMP(1);
    if (tid == 0) {
        s_misc[1] = grid_barrier(a.bar, gridDim.x, a.wait_ns, a.err) ? 0 : 1;
        s_misc[2] = 0;
    }
    __syncthreads();
    if (s_misc[1]) return;  // nothing in flight yet
    for (int e = tid; e < a.E; e += nthr) s_sc[e] = __ldcg(a.scores + e);
    __syncthreads();
    if (tid == 0) {
        int ids[8];
        float w[8];
        topk_softmax(s_sc, a.E, a.k, ids, w);
        if (blockIdx.x == 0) {
            for (int i = 0; i < a.k; ++i) {
                a.ids_out[i] = ids[i];
                a.w_out[i] = w[i];
            }
        }
        s_misc[0] = build_slots(ids, w, a.k, a.E, a.S, a.rec_base, a.n_local, a.usable, s_rec, s_w);
    }
    __syncthreads();
    RB_STAMP(2);
    const int nact = s_misc[0];
    if (nact == 0) {
        for (int i = blockIdx.x * nthr + tid; i < H; i += gridDim.x * nthr) a.h_out[i] = a.h_in[i];
        return;
    }

    const int ntb = a.tb.ntiles, TRb = a.tb.TR, ntc = a.tc.ntiles, TRc = a.tc.TR;
    const int UB = nact * ntb;  // phase B units: (slot, GU tile)
    const int ub0 = (int)((long long)blockIdx.x * UB / gridDim.x);
    const int ub1 = (int)((long long)(blockIdx.x + 1) * UB / gridDim.x);
    const int c0 = (int)((long long)blockIdx.x * ntc / gridDim.x);  // phase C: D tiles over H
    const int c1 = (int)((long long)(blockIdx.x + 1) * ntc / gridDim.x);
    const uint32_t sb = a.tb.tile_stride, sc = a.tc.tile_stride;

    if (warp == CW) {  // -------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int i = 0;
            bool okp = true;
            for (int u = ub0; okp && u < ub1; ++u, ++i) {
                const int s = i % a.nslots, n = i / a.nslots;
                if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.wait_ns, a.err, 0)) {
                    okp = false;
                    break;
                }
                const int slot = u / ntb, t = u - slot * ntb;
                const uint8_t *src = a.pool + (size_t)s_rec[slot] * a.rec_stride + (size_t)t * sb;
                RB_CHUNK(0, i);
                mbar_arrive_expect_tx(&full[s], a.tb.tile_bytes);
                bulk_g2s(ring + (size_t)s * a.slot_bytes, src, a.tb.tile_bytes, &full[s], pol);
            }
            for (int j = 0; okp && j < nact; ++j) {
                const uint8_t *rec = a.pool + (size_t)s_rec[j] * a.rec_stride + a.off_d;
                for (int t = c0; t < c1; ++t, ++i) {
                    const int s = i % a.nslots, n = i / a.nslots;
                    if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.wait_ns, a.err, 0)) {
                        okp = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], a.tc.tile_bytes);
                    bulk_g2s(ring + (size_t)s * a.slot_bytes, rec + (size_t)t * sc, a.tc.tile_bytes,
                             &full[s], pol);
                }
            }
            // drain: the last use of every stage must have landed before exit
            for (int t = i > a.nslots ? i - a.nslots : 0; t < i; ++t)
                mbar_wait(&full[t % a.nslots], (t / a.nslots) & 1, a.wait_ns, a.err);
        }
        return;
    }

    // ---------------------------------------------------------- consumers --
    // Warp group q = warp / KS covers one row (KS warps, J groups of 32 inputs
    // per lane) and takes rows [q*ROWS, (q+1)*ROWS) of every tile; warps past
    // the phase's NG groups only release. Every consumer waits for and
    // releases every stage (weight 1), so the ring's phases stay in step
    // across both phases.
    bool good = true;
    int i = 0;
    {  // B: gate + up
        const int ks = warp % a.KSb, grp = warp / a.KSb;
        const int g0 = ks * 32 * JB + lane;
        const bool mine = grp < a.NGb;
        bool act[JB];
        XPlanes xg[JB];
#pragma unroll
        for (int q = 0; q < JB; ++q) {
            act[q] = mine && g0 + 32 * q < Gb;
            load_xplanes_padded(xg[q], xn, g0 + 32 * q, act[q]);
        }
        const int rbase = grp * a.ROWSb;
        switch (a.ROWSb) {
            case 1: good = moe_gate_up<JB, 1>(a, ring, part, full, empty, sink + warp, ub0, ub1, i, ks, rbase, mine, g0, act, xg); break;
            case 2: good = moe_gate_up<JB, 2>(a, ring, part, full, empty, sink + warp, ub0, ub1, i, ks, rbase, mine, g0, act, xg); break;
            default: good = moe_gate_up<JB, 4>(a, ring, part, full, empty, sink + warp, ub0, ub1, i, ks, rbase, mine, g0, act, xg); break;
        }
    }
    named_sync(1, CW * 32);
    if (good) {
        const int nrb = (ub1 - ub0) * TRb;
        for (int lr = tid; lr < nrb; lr += CW * 32) {
            const int u = ub0 + lr / TRb;
            const int slot = u / ntb, row = (u - slot * ntb) * TRb + lr % TRb;
            if (row >= I) continue;
            float gs = 0.f, us = 0.f;
            for (int k = 0; k < a.KSb; ++k) {
                gs += part[(lr * 2) * a.KSb + k];
                us += part[(lr * 2 + 1) * a.KSb + k];
            }
            a.mid[(size_t)slot * I + row] = silu_mul(gs, us);
        }
    }
    __threadfence();
    named_sync(1, CW * 32);
    RB_STAMP(3);
    if (tid == 0) s_misc[2] = grid_barrier(a.bar, gridDim.x, a.wait_ns, a.err) ? 0 : 1;
    named_sync(1, CW * 32);
    RB_STAMP(4);
    good = good && !s_misc[2];

    if (good) {  // C: down + combine
        const int ks = warp % a.KSc, grp = warp / a.KSc;
        const int g0 = ks * 32 * JC + lane;
        const bool mine = grp < a.NGc;
        bool act[JC];
#pragma unroll
        for (int q = 0; q < JC; ++q) act[q] = mine && g0 + 32 * q < Gc;
        const int rbase = grp * a.ROWSc;
        switch (a.ROWSc) {
            case 1: good = moe_down<JC, 1>(a, ring, part, full, empty, sink + warp, nact, c0, c1, i, ks, rbase, mine, g0, act); break;
            case 2: good = moe_down<JC, 2>(a, ring, part, full, empty, sink + warp, nact, c0, c1, i, ks, rbase, mine, g0, act); break;
            case 4: good = moe_down<JC, 4>(a, ring, part, full, empty, sink + warp, nact, c0, c1, i, ks, rbase, mine, g0, act); break;
            default: good = moe_down<JC, 8>(a, ring, part, full, empty, sink + warp, nact, c0, c1, i, ks, rbase, mine, g0, act); break;
        }
    }
    named_sync(1, CW * 32);
    RB_STAMP(5);
    if (!good) return;
    for (int lr = tid; lr < (c1 - c0) * TRc; lr += CW * 32) {
        const int row = c0 * TRc + lr;
        if (row >= H) continue;
        float delta = 0.f;
        for (int j = 0; j < nact; ++j) {
            float d = 0.f;
            for (int k = 0; k < a.KSc; ++k) d += part[(lr * nact + j) * a.KSc + k];
            delta += s_w[j] * d;
        }
        a.h_out[row] = a.h_in[row] + delta;
    }
    RB_STAMP(6);
}

const void *moe_fused_kernel(int JB, int JC) {
    if (JB == 2)
        return JC == 2 ? (const void *)k_moe_decode_g32<2, 2> : (const void *)k_moe_decode_g32<2, 1>;
    return JC == 2 ? (const void *)k_moe_decode_g32<1, 2> : (const void *)k_moe_decode_g32<1, 1>;
}

#ifdef RB_PHASE_TIMERS
}  // namespace rb
extern "C" __attribute__((visibility("default"))) int rabbit_cuda_debug_phase_ns(uint64_t *out,
                                                                                 int n) {
    return cudaMemcpyFromSymbol(out, rb::g_phase_ns, sizeof(uint64_t) * n) == cudaSuccess ? 0 : 6;
}
extern "C" __attribute__((visibility("default"))) int rabbit_cuda_debug_dot_ns(uint64_t *out) {
    int z = 0;
    cudaMemcpyToSymbol(rb::rb_dbg_i, &z, sizeof(int));
    return cudaMemcpyFromSymbol(out, rb::rb_dbg_ns, sizeof(uint64_t) * 128) == cudaSuccess ? 0 : 6;
}
extern "C" __attribute__((visibility("default"))) int rabbit_cuda_debug_chunk_ns(uint64_t *out) {
    return cudaMemcpyFromSymbol(out, rb::g_chunk_ns, sizeof(uint64_t) * 256) == cudaSuccess ? 0 : 6;
}
namespace rb {
#endif

// ======================================================= generic path ====
__device__ __forceinline__ uint32_t ldu32(const uint8_t *p) {
    if ((reinterpret_cast<uintptr_t>(p) & 3) == 0) return *reinterpret_cast<const uint32_t *>(p);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
           ((uint32_t)p[3] << 24);
}

__device__ __forceinline__ int nbytes_g32(long long n) {
    return (int)(4 + 4 * ((n + 31) / 32) + (n + 1) / 2);
}

// Lane partial of row `row` of an [out, in] matrix in expert format `quant`
// starting at `m` (quant 4: grouped blob; 0: fp32; else: f32 scale + int8).
__device__ float row_dot_lane(const uint8_t *m, int quant, int row, int out_dim, int in_dim,
                              const float *x, bool *zero) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    *zero = false;
    if (quant == 0) {
        const float *w = reinterpret_cast<const float *>(m) + (size_t)row * in_dim;
        for (int i = lane; i < in_dim; i += 32) acc += w[i] * x[i];
    } else if (quant == 4) {
        const uint32_t gs = ldu32(m);
        if (gs == 0 || gs > 4096) {  // quant.c:158-161
            *zero = true;
            return 0.f;
        }
        const long long n = (long long)out_dim * in_dim;
        const uint8_t *sc = m + 4;
        const uint8_t *nib = m + 4 + 4 * ((n + gs - 1) / gs);
        for (int i = lane; i < in_dim; i += 32) {
            const long long f = (long long)row * in_dim + i;
            const uint8_t b = nib[f >> 1];
            const int q = (int)((f & 1) ? (b >> 4) : (b & 15)) - 8;
            acc += __fmul_rn((float)q, __uint_as_float(ldu32(sc + 4 * (f / gs)))) * x[i];
        }
    } else {
        const int8_t *w = reinterpret_cast<const int8_t *>(m + 4) + (size_t)row * in_dim;
        for (int i = lane; i < in_dim; i += 32) acc += (float)w[i] * x[i];
    }
    return acc;
}

__device__ __forceinline__ float row_finish(const uint8_t *m, int quant, float sum) {
    if (quant == 0 || quant == 4) return sum;
    return sum * __uint_as_float(ldu32(m));  // int8: scale after the dot (forward_v2.c:88)
}

// Offsets of gate / up / down inside a record (forward_v2.c:303-353).
__device__ void mat_offsets(int quant, int H, int I, size_t *og, size_t *ou, size_t *od) {
    const size_t mat = (size_t)H * I;
    if (quant == 0) {
        *og = 0;
        *ou = mat * 4;
        *od = 2 * mat * 4;
    } else if (quant == 4) {
        const size_t nb = (size_t)nbytes_g32((long long)mat);
        *og = 0;
        *ou = nb;
        *od = 2 * nb;
    } else {
        *og = 0;
        *ou = 4 + mat;
        *od = 2 * (4 + mat);
    }
}

// One block: rmsnorm, router scores, top-k, slot list.
__global__ void k_moe_route(MoeGenericArgs a) {
    __shared__ float red[32];
    __shared__ float inv_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
    float ss = 0.f;
    for (int i = tid; i < a.H; i += nthr) ss += a.h_in[i] * a.h_in[i];
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < (nthr >> 5); ++w) t += red[w];
        t /= (float)a.H;
        inv_s = 1.0f / sqrtf(t + 1e-5f);
    }
    __syncthreads();
    for (int i = tid; i < a.H; i += nthr) a.xn[i] = (a.h_in[i] * inv_s) * a.rms[i];
    __syncthreads();
    for (int e = warp; e < a.E; e += nthr >> 5) {
        float d = 0.f;
        for (int i = lane; i < a.H; i += 32) d += a.router[(size_t)e * a.H + i] * a.xn[i];
        d = warp_sum(d);
        if (lane == 0) a.scores[e] = d;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_block();
        int ids[8];
        float w[8];
        topk_softmax(a.scores, a.E, a.k, ids, w);
        for (int i = 0; i < a.k; ++i) {
            a.ids_out[i] = ids[i];
            a.w_out[i] = w[i];
        }
        a.route->nact =
            build_slots(ids, w, a.k, a.E, a.S, a.rec_base, a.n_local, a.usable, a.route->rec,
                        a.route->w);
    }
}

// grid (ceil(I / warps), slots): warp per row of gate and up -> mid.
__global__ void k_moe_up_generic(MoeGenericArgs a) {
    const int j = blockIdx.y;
    if (j >= a.route->nact) return;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= a.I) return;
    const uint8_t *rec = a.pool + (size_t)a.route->rec[j] * a.rec_stride;
    size_t og, ou, od;
    mat_offsets(a.quant, a.H, a.I, &og, &ou, &od);
    bool zg, zu;
    float g = warp_sum(row_dot_lane(rec + og, a.quant, row, a.I, a.H, a.xn, &zg));
    float u = warp_sum(row_dot_lane(rec + ou, a.quant, row, a.I, a.H, a.xn, &zu));
    g = zg ? 0.f : row_finish(rec + og, a.quant, g);
    u = zu ? 0.f : row_finish(rec + ou, a.quant, u);
    if ((threadIdx.x & 31) == 0) a.mid[(size_t)j * a.I + row] = silu_mul(g, u);
}

// grid (ceil(H / warps), slots): warp per row of down.
__global__ void k_moe_down_generic(MoeGenericArgs a) {
    const int j = blockIdx.y;
    if (j >= a.route->nact) return;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= a.H) return;
    const uint8_t *rec = a.pool + (size_t)a.route->rec[j] * a.rec_stride;
    size_t og, ou, od;
    mat_offsets(a.quant, a.H, a.I, &og, &ou, &od);
    bool z;
    float d = warp_sum(row_dot_lane(rec + od, a.quant, row, a.H, a.I, a.mid + (size_t)j * a.I, &z));
    d = z ? 0.f : row_finish(rec + od, a.quant, d);
    if ((threadIdx.x & 31) == 0) a.down[(size_t)j * a.H + row] = d;
}

__global__ void k_moe_combine(MoeGenericArgs a) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.H) return;
    float delta = 0.f;
    const int n = a.route->nact;
    for (int j = 0; j < n; ++j) delta += a.route->w[j] * a.down[(size_t)j * a.H + r];
    a.h_out[r] = a.h_in[r] + delta;
}

}  // namespace rb
