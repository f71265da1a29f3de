// rb_gemv.cuh -- group-32 int4 GEMV kernels shared by the matrix and MoE paths.
#pragma once
#include <stdint.h>

#include "rb_device.cuh"

namespace rb {

// ------------------------------------------------------------------ plans --
// Streaming GEMV launch plan for a [rows, in] group-32 matrix in the plane
// layout: nibbles [rows_pad][in/2], scales [rows_pad][in/32], rows_pad a
// multiple of 4 (pad rows are zero).
struct G32Plan {
    int rows, in_dim, units;  // units of 4 rows
    int KS;                   // k-slices: warps that split one row (32 groups each)
    int RS;                   // row subsets: warps that split a chunk's rows
    int CR;                   // rows per chunk (multiple of 4)
    int nslots;               // ring stages
    uint32_t slot_bytes;
    int rows_cta_max;
    int grid, block;
    size_t smem;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Fast path eligibility: group 32, whole groups per row, at most 16 k-slices.
inline bool g32_ok(int in_dim) { return in_dim > 0 && in_dim % 32 == 0 && in_dim <= 16384; }

bool plan_g32(int rows, int in_dim, int sm_count, G32Plan *p);

struct G32Args {
    const uint8_t *nib;
    const float *sc;
    const float *x;
    float *y;
    int rows, in_dim, units;
    int KS, RS, CR, nslots;
    uint32_t slot_bytes;
    int rows_cta_max;
    int *err;
    uint64_t wait_ns;
};

__global__ void k_gemv_g32(G32Args a);

// Flat-index kernels over a raw .rabbit blob (any shape / alignment).
__global__ void k_gemv_flat(const uint8_t *blob, const float *x, float *y, int out_dim,
                            int in_dim);
__global__ void k_dequant_flat(const uint8_t *blob, float *dst, long long n, uint32_t gs);

}  // namespace rb
