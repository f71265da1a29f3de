// rb_device.cuh -- device-side building blocks for sm_100a.
//
//  * mbarrier + cp.async.bulk (1-D bulk copy, no tensor map, no multicast)
//    for staging weight rows into shared memory;
//  * bounded waits: every spin checks %globaltimer against a limit and, when
//    it runs out, records RB_ERR_TIMEOUT in a device error word and returns
//    false so the caller can drain and exit;
//  * the group-32 int4 dot product on integer dp4a over activation planes.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define RB_ERR_TIMEOUT 7
#define RB_ERR_ARGS 5

namespace rb {

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void set_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive with a weight: `count` of the barrier's expected arrivals at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// try_wait with a suspend-time hint: a waiting warp sleeps in hardware until
// the phase completes (or the hint expires) instead of spinning, so waiting
// warps do not take issue slots from the warps that compute.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Non-blocking: has phase `parity` of `bar` completed?
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false (and *err set) after
// `limit_ns` nanoseconds. Consumers back off with __nanosleep (doubling up to
// `max_sleep_ns`) so warps that wait do not spin on the issue slots of the
// warps that compute; the producer passes 0 and re-polls at once.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                          int *err, uint32_t max_sleep_ns = 256) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t sleep = 32;
    for (uint32_t it = 1;; ++it) {
        if (max_sleep_ns) {
            __nanosleep(sleep);
            sleep = sleep * 2 > max_sleep_ns ? max_sleep_ns : sleep * 2;
        }
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 7u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            set_error(err, RB_ERR_TIMEOUT);
            return false;
        }
    }
}

// Activations staged in shared memory padded to 33 floats per group of 32:
// lane l reading element j of group l hits bank (l + j) % 32, conflict-free.
__device__ __forceinline__ int xpad(int i) { return (i >> 5) * 33 + (i & 31); }

// --------------------------------------------------------------- bulk copy --
// 1-D global -> shared bulk copy completing on `bar`. Both addresses 16-byte
// aligned, bytes a multiple of 16. evict_first: weights are streamed once.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch. `launch_dependents`: this CTA no longer
// holds back the launch of the next kernel on the stream (it launches once
// every CTA has said so or exited). `wait_prerequisite`: block until the
// preceding kernel on the stream has completed and its memory is visible.
// Both are no-ops for a launch without the programmatic-serialization
// attribute.
__device__ __forceinline__ void launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_prerequisite() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Named barrier among `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------- int4 dot product --
// The 32 activations of one group are turned into a 23-bit block-floating-
// point integer vector: X_i = rint(x_i * 2^(22-e)) with 2^e > max|x_i|, so
// |X_i| <= 2^22 and the rounding error is at most 2^(e-23) per element. The
// planes are the bytes of X_i's two's-complement form:
//   X = B2 * 2^16 + B1 * 2^8 + B0,  B0, B1 = bytes 0, 1 (unsigned, 0..255),
//   B2 = X >> 16 = byte 2 read as a signed int8 (in [-64, 64]).
// The weights stay unsigned nibbles (bias 8): w & 0x0F0F0F0F holds the even
// elements of a word as bytes, (w >> 4) & 0x0F0F0F0F the odd ones, and dp4a
// accumulates exact plane sums S_p = sum nib_i * B_p,i (u8 x u8 for planes 0
// and 1, |S| <= 122400; u8 x s8 for plane 2, |S2| <= 30720). Then
//   sum_i q_i X_i = S0 + 256 S1 + 65536 S2 - 8 sum_i X_i,
// |sum_i q_i X_i| <= 32 * 8 * 2^22 = 2^30: the sum is formed in 32-bit
// wrap-around arithmetic (terms may leave the int32 range, the result cannot,
// so it is exact), converted to float once and scaled by unit = 2^(e-22).
struct XPlanes {
    uint32_t lo[3][4];  // plane p, word j: byte p of X for elements 8j, 8j+2, 8j+4, 8j+6
    uint32_t hi[3][4];  // plane p, word j: byte p of X for elements 8j+1, 8j+3, 8j+5, 8j+7
    int m8sum;          // -8 * sum_i X_i  (|.| <= 2^30)
    float unit;         // 2^(e-22)
};

// Planes 0..2 of four integers a, b, c, d (bytes p of each, a in the low
// byte): seven byte permutes for the three planes.
__device__ __forceinline__ void planes4(int a, int b, int c, int d, uint32_t &p0, uint32_t &p1,
                                        uint32_t &p2) {
    const uint32_t ab = __byte_perm((uint32_t)a, (uint32_t)b, 0x5140u);  // a0 b0 a1 b1
    const uint32_t cd = __byte_perm((uint32_t)c, (uint32_t)d, 0x5140u);  // c0 d0 c1 d1
    p0 = __byte_perm(ab, cd, 0x5410u);
    p1 = __byte_perm(ab, cd, 0x7632u);
    const uint32_t ab2 = __byte_perm((uint32_t)a, (uint32_t)b, 0x0062u);  // a2 b2
    const uint32_t cd2 = __byte_perm((uint32_t)c, (uint32_t)d, 0x0062u);  // c2 d2
    p2 = __byte_perm(ab2, cd2, 0x5410u);
}

__device__ __forceinline__ void make_xplanes(XPlanes &g, const float (&x)[32]) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    // e with 2^e > amax; clamped so 2^(22-e) stays finite for tiny groups
    int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
    if (e < -100) e = -100;
    const float scale = __int_as_float((127 + 22 - e) << 23);  // 2^(22-e)
    g.unit = __int_as_float((127 - 22 + e) << 23);             // 2^(e-22)
    int X[32];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        // rint via the 1.5*2^23 shift: exact for |x*scale| <= 2^22
        X[i] = __float_as_int(fmaf(x[i], scale, 12582912.0f)) - 0x4B400000;
        sum += X[i];
    }
    g.m8sum = -8 * sum;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        planes4(X[8 * j], X[8 * j + 2], X[8 * j + 4], X[8 * j + 6], g.lo[0][j], g.lo[1][j],
                g.lo[2][j]);
        planes4(X[8 * j + 1], X[8 * j + 3], X[8 * j + 5], X[8 * j + 7], g.hi[0][j], g.hi[1][j],
                g.hi[2][j]);
    }
}

__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// sum_{i<32} q_i * x_i for one 16-byte group (element 2b = low nibble of byte
// b, 2b+1 = high nibble), q = nib - 8, x as planes.
__device__ __forceinline__ float dot32(const uint4 w, const XPlanes &g) {
    int s0 = 0, s1 = 0, s2 = 0;
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = wv[j] & 0x0F0F0F0Fu;
        const uint32_t hi = (wv[j] >> 4) & 0x0F0F0F0Fu;
        s0 = dp4a_uu(lo, g.lo[0][j], s0);
        s1 = dp4a_uu(lo, g.lo[1][j], s1);
        s2 = dp4a_us(lo, g.lo[2][j], s2);
        s0 = dp4a_uu(hi, g.hi[0][j], s0);
        s1 = dp4a_uu(hi, g.hi[1][j], s1);
        s2 = dp4a_us(hi, g.hi[2][j], s2);
    }
    const uint32_t t = (uint32_t)s0 + ((uint32_t)s1 << 8) + ((uint32_t)s2 << 16) +
                       (uint32_t)g.m8sum;
    return (float)(int)t * g.unit;
}

// x staged in shared memory padded to 33 floats per group of 32, so lane l
// reading element j of group l hits bank (l + j) % 32: conflict-free.
__device__ __forceinline__ void load_xplanes_padded(XPlanes &g, const float *xp, int grp,
                                                    bool act) {
    float xr[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) xr[j] = act ? xp[grp * 33 + j] : 0.f;
    make_xplanes(g, xr);
}

// Lane's 32 activations straight from global memory (128 contiguous bytes,
// 16-byte aligned), through L2 only (written by other CTAs earlier).
__device__ __forceinline__ void load_xplanes_global(XPlanes &g, const float *src, bool act) {
    float xr[32];
    const float4 *p = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 t = act ? __ldcg(p + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[4 * q] = t.x;
        xr[4 * q + 1] = t.y;
        xr[4 * q + 2] = t.z;
        xr[4 * q + 3] = t.w;
    }
    make_xplanes(g, xr);
}

// Sum 8 per-lane values across the warp; afterwards lane l with (l & 3) == 0
// holds the total of value (l >> 2) & 7. Every lane must call it.
__device__ __forceinline__ float warp_reduce8(float (&v)[8]) {
    const int lane = threadIdx.x & 31;
    float a[4];
    {
        const bool up = lane & 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float send = up ? v[i] : v[i + 4];
            const float keep = up ? v[i + 4] : v[i];
            a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
    }
    float b[2];
    {
        const bool up = lane & 8;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float send = up ? a[i] : a[i + 2];
            const float keep = up ? a[i + 2] : a[i];
            b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
    }
    float c;
    {
        const bool up = lane & 4;
        const float send = up ? b[0] : b[1];
        const float keep = up ? b[1] : b[0];
        c = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// Sum 4 per-lane values across the warp; afterwards lane l with (l & 7) == 0
// holds the total of value (l >> 3) & 3.
__device__ __forceinline__ float warp_reduce4(float (&v)[4]) {
    const int lane = threadIdx.x & 31;
    float a[2];
    {
        const bool up = lane & 16;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float send = up ? v[i] : v[i + 2];
            const float keep = up ? v[i + 2] : v[i];
            a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
    }
    float c;
    {
        const bool up = lane & 8;
        const float send = up ? a[0] : a[1];
        const float keep = up ? a[1] : a[0];
        c = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    c += __shfl_xor_sync(0xffffffffu, c, 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Store `token` (all lanes, one word per warp) and then, from lane 0, arrive
// on `bar` with weight `count`. The store reads the token, so the arrive --
// a release that is ordered after the store -- executes only once the loads
// that produced the token have returned.
__device__ __forceinline__ void mbar_arrive_dep(uint64_t *bar, uint32_t count, uint32_t token,
                                                uint32_t *sink) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(smem_u32(sink)), "r"(token) : "memory");
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive_cnt(bar, count);
}

#ifdef RB_PHASE_TIMERS
__device__ uint64_t rb_dbg_ns[128];
__device__ int rb_dbg_i;
#endif

// One staged tile holding NMAT matrices x TR rows, seen by one warp of the
// group that takes tile rows [rbase, rbase + ROWS). Tile layout: nibbles of
// matrix m at st + m*TR*half (row r at + r*half), then scales of matrix m at
// st + NMAT*TR*half + m*TR*G*4. The lane owns input groups g0 + 32*j
// (j < J; act[j]: group in range) with activations xg[j]. All of the warp's
// loads are issued first; once they have returned the warp releases the stage
// (arrive on `empty` with weight `wgt`) and computes and reduces while the
// producer refills it. Rows past the matrix end are zero in the tile (scale 0)
// and contribute 0. Each (m, r) value is written by one lane to part[pidx(m, r)].
template <int NMAT, int ROWS, int J, typename PIdx>
__device__ __forceinline__ void chunk_dot(const uint8_t *st, int TR, int rbase, int half, int G,
                                          int g0, const bool (&act)[J],
                                          const XPlanes (&xg)[J], PIdx pidx, float *part,
                                          uint64_t *empty, uint32_t wgt, uint32_t *sink) {
    constexpr int V = NMAT * ROWS;  // values per warp: 1..8
    static_assert(V >= 1 && V * J <= 8, "at most 8 dots per lane and tile");
    const int lane = threadIdx.x & 31;
    const float *scb = reinterpret_cast<const float *>(st + (size_t)NMAT * TR * half);
    uint4 w[V][J];
    float s[V][J];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const int m = v / ROWS, r = rbase + v % ROWS;
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const int g = g0 + 32 * j;
            if (act[j]) {
                w[v][j] = *reinterpret_cast<const uint4 *>(st + (size_t)(m * TR + r) * half + g * 16);
                s[v][j] = scb[(m * TR + r) * G + g];
            } else {
                w[v][j] = make_uint4(0u, 0u, 0u, 0u);
                s[v][j] = 0.f;
            }
        }
    }
    // Release the stage once the loads have *returned*: the token reads one
    // register of every load and the arrive is ordered after its store (an
    // arrive issued right after the loads let a refill race the reads).
    uint32_t tok = 0;
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < J; ++j) tok ^= w[v][j].x ^ __float_as_uint(s[v][j]);
    mbar_arrive_dep(empty, wgt, tok, sink);
    float val[V <= 4 ? 4 : 8];
#pragma unroll
    for (int v = 0; v < (V <= 4 ? 4 : 8); ++v) {
        float acc = 0.f;
        if (v < V) {
#pragma unroll
            for (int j = 0; j < J; ++j) acc = fmaf(s[v][j], dot32(w[v][j], xg[j]), acc);
        }
        val[v] = acc;
    }
    float tot;
    int b;
    if (V <= 4) {
        tot = warp_reduce4(*reinterpret_cast<float(*)[4]>(val));
        b = (lane & 7) == 0 ? (lane >> 3) : 8;
    } else {
        tot = warp_reduce8(*reinterpret_cast<float(*)[8]>(val));
        b = (lane & 3) == 0 ? (lane >> 2) : 8;
    }
    if (b < V) part[pidx(b / ROWS, b % ROWS)] = tot;
}

}  // namespace rb
