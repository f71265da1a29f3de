// rb_device.cuh -- device-side building blocks for sm_100a.
//
//  * mbarrier + cp.async.bulk (1-D bulk copy, no tensor map, no multicast)
//    for staging weight rows into shared memory;
//  * bounded waits: every spin checks %globaltimer against a limit and, when
//    it runs out, records RB_ERR_TIMEOUT in a device error word and returns
//    false so the caller can drain and exit;
//  * the group-32 int4 dot product on packed fp32 (FFMA2/FADD2).
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

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false (and *err set) after
// `limit_ns` nanoseconds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                          int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            set_error(err, RB_ERR_TIMEOUT);
            return false;
        }
    }
}

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

// Named barrier among `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------- int4 dot product --
// Two nibble-derived floats per byte: __byte_perm places the nibble (low 4
// bits of a byte) into mantissa bits 16..19 under the exponent byte 0x40, so
// the float is exactly 2 + nib/64. Subtracting 2.125 (exact, Sterbenz) gives
// (nib - 8)/64 = q/64. The caller multiplies the group sum by 64*scale.
__device__ __forceinline__ float nib_f(uint32_t bytes4, uint32_t sel) {
    return __uint_as_float(__byte_perm(bytes4, 0x40000000u, sel));
}

// sum_{i<32} (q_i / 64) * x[i] for one 16-byte group (element 2b = low
// nibble of byte b, 2b+1 = high nibble), x in registers.
__device__ __forceinline__ float dot32_q64(const uint4 w, const float (&x)[32]) {
    const float2 off = make_float2(-2.125f, -2.125f);
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = wv[j] & 0x0F0F0F0Fu;         // elements 8j + 0,2,4,6
        const uint32_t hi = (wv[j] >> 4) & 0x0F0F0F0Fu;  // elements 8j + 1,3,5,7
        // selectors: byte b of `lo`/`hi` into byte 2, constant bytes elsewhere
        float2 q0 = __fadd2_rn(make_float2(nib_f(lo, 0x7054u), nib_f(hi, 0x7054u)), off);
        float2 q1 = __fadd2_rn(make_float2(nib_f(lo, 0x7154u), nib_f(hi, 0x7154u)), off);
        float2 q2 = __fadd2_rn(make_float2(nib_f(lo, 0x7254u), nib_f(hi, 0x7254u)), off);
        float2 q3 = __fadd2_rn(make_float2(nib_f(lo, 0x7354u), nib_f(hi, 0x7354u)), off);
        acc0 = __ffma2_rn(q0, make_float2(x[8 * j + 0], x[8 * j + 1]), acc0);
        acc1 = __ffma2_rn(q1, make_float2(x[8 * j + 2], x[8 * j + 3]), acc1);
        acc0 = __ffma2_rn(q2, make_float2(x[8 * j + 4], x[8 * j + 5]), acc0);
        acc1 = __ffma2_rn(q3, make_float2(x[8 * j + 6], x[8 * j + 7]), acc1);
    }
    return (acc0.x + acc0.y) + (acc1.x + acc1.y);
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace rb
