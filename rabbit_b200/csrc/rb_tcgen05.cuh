// rb_tcgen05.cuh -- sm_100a tensor-core building blocks: tensor memory
// (TMEM) allocation, tcgen05.mma of kind::i8 with A in TMEM and B in shared
// memory, its commit to an mbarrier, TMEM loads / stores, and the tiled TMA
// copy (cp.async.bulk.tensor, no multicast) that stages weight rows.
//
// Conventions used throughout (PTX ISA, tcgen05 chapter):
//  * a TMEM address is (lane << 16) | column; a warp may touch only the 32
//    lanes 32 * (warp % 4) .. + 31;
//  * for M = 128 (cta_group::1) row m of A and of the accumulator D is TMEM
//    lane m; A's K bytes are packed four to a 32-bit column in K order, D's
//    column n is output column n (one s32 each);
//  * B is read from shared memory through a matrix descriptor; here always
//    the K-major layout without swizzle: 8-row x 16-byte core matrices of 128
//    contiguous bytes, the two 16-byte K halves of a 32-byte K step LBO = 128
//    bytes apart and consecutive 8-row groups SBO = 256 bytes apart.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "rb_device.cuh"

namespace rb {

// Instruction descriptor of tcgen05.mma.kind::i8: s32 accumulator, A and B
// signed 8-bit, both K-major, M = 128, N (a multiple of 16, <= 256).
__host__ __device__ constexpr uint32_t i8_idesc(int N) {
    return (2u << 4)                       // D format: s32
           | (1u << 7)                     // A: s8
           | (1u << 10)                    // B: s8
           | ((uint32_t)(N >> 3) << 17)    // N / 8
           | ((uint32_t)(128 >> 4) << 24); // M / 16
}

// Shared-memory matrix descriptor, K-major, no swizzle, LBO 128, SBO 256.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4)  // start address / 16
           | ((uint64_t)(128 >> 4) << 16)            // leading byte offset / 16
           | ((uint64_t)(256 >> 4) << 32)            // stride byte offset / 16
           | (1ull << 46);                           // descriptor version (sm_100)
}

// ------------------------------------------------------------------ TMEM --
// Allocate `cols` columns (a power of two, 32..512); the whole warp calls it.
// The address lands in *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Eight 32-bit columns of this thread's lane (32x32b shape: lane = the
// warp's lane quarter + laneid).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 and 8 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16], int o) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr + (uint32_t)o)
        : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&v)[8], int o) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7])
        : "r"(taddr + (uint32_t)o)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// D[128 x N] = A[128 x 32] * B[N x 32]^T, s8 x s8 -> s32 (accumulate: D +=).
// A in TMEM at a_tmem, B in shared memory (descriptor), D in TMEM. Issued by
// one thread.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}
// The mbarrier gets one arrival once every tcgen05.mma this thread issued
// before has completed (and its shared-memory operands may be overwritten).
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// ----------------------------------------------------------- tiled TMA --
// Box of a 4-D / 5-D tensor map into shared memory, completing on `bar`.
// The innermost coordinate c0 is a byte offset and a multiple of 16 at every
// call site (128 * chunk).
__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_load_5d(void *smem_dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
        "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------ int4 -> A operand --
// The 16 nibble bytes of one 32-input group (words w0..w3, element 2b of a
// word = low nibble of its byte b, 2b + 1 = high nibble) as the MMA's A
// row: 8 words of 16 q (q = nibble - 8) as signed bytes,
//   word 2j     = 16 q of elements 8j, 8j+2, 8j+4, 8j+6   (K = 8j .. 8j+3)
//   word 2j + 1 = 16 q of elements 8j+1, 8j+3, 8j+5, 8j+7 (K = 8j+4 .. 8j+7)
// (nibble << 4) ^ 0x80 is the two's-complement byte of 16 (nibble - 8).
// The activation rows use the same K order (tc_k_element).
__device__ __forceinline__ void nibbles_to_a(const uint4 w, uint32_t (&a)[8]) {
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        a[2 * j] = ((wv[j] << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
        a[2 * j + 1] = (wv[j] & 0xF0F0F0F0u) ^ 0x80808080u;
    }
}
// Element of a group held at K index kk of an A / B row.
__host__ __device__ __forceinline__ int tc_k_element(int kk) {
    return (kk & ~7) + 2 * (kk & 3) + ((kk >> 2) & 1);
}

}  // namespace rb
