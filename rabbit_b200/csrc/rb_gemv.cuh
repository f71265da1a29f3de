// rb_gemv.cuh -- group-32 int4 GEMV kernels shared by the matrix and MoE paths.
#pragma once
#include <stdint.h>

#include "rb_device.cuh"

namespace rb {

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// --------------------------------------------------------------- tiling --
// A matrix [rows, in] in HBM as tiles of TR rows x cols = in / KC inputs
// (KC column chunks, 1 unless stated): tile (c, t), at index c * rtiles + t,
// holds rows [t*TR, t*TR + TR) of input columns [c*cols, (c+1)*cols): the
// packed nibbles (TR x cols/2 bytes, row-major) followed by the group scales
// (TR x cols/32 fp32). Tiles sit tile_stride bytes apart; rows past the end
// of the matrix are zero. One tile is one bulk copy.
struct Tiling {
    int rows, in_dim, TR, ntiles;
    int KC, cols, rtiles;  // column chunks, inputs per chunk, row tiles per chunk
    uint32_t tile_bytes;   // TR * (cols/2 + cols/8)
    uint32_t tile_stride;  // tile_bytes rounded up to 128
};

__host__ __device__ inline Tiling make_tiling(int rows, int in_dim, int TR, int KC = 1) {
    Tiling t;
    t.rows = rows;
    t.in_dim = in_dim;
    t.TR = TR;
    t.KC = KC;
    t.cols = in_dim / KC;
    t.rtiles = (rows + TR - 1) / TR;
    t.ntiles = t.rtiles * KC;
    t.tile_bytes = (uint32_t)((size_t)TR * ((size_t)t.cols / 2 + (size_t)t.cols / 8));
    t.tile_stride = (uint32_t)align_up(t.tile_bytes, 128);
    return t;
}

// Re-lay a .rabbit group-32 blob (u32 gs | f32 scales | nibbles, flat row
// major) into tiles on the host. `dst` must hold ntiles * tile_stride bytes.
void tile_blob_host(const uint8_t *blob, const Tiling &t, uint8_t *dst);
// Same for a pair of matrices of equal shape interleaved per tile as
// [a nibbles | b nibbles | a scales | b scales] (tile_bytes of the pair).
void tile_pair_host(const uint8_t *a, const uint8_t *b, const Tiling &t2, uint8_t *dst);

// Warp layout over a row of G = in/32 groups: each lane holds J groups (1,
// or 2 for rows longer than 8192 inputs) and KS warps cover one row.
__host__ __device__ inline int lane_groups(int G) { return G > 256 ? 2 : 1; }
__host__ __device__ inline int kslices(int G, int J) { return (G + 32 * J - 1) / (32 * J); }
constexpr int kConsumerWarps = 8;  // consumer warps per CTA (two per SM sub-partition)

// Rows per warp group per tile (1, 2, 4 or 8, at most max_rows) for NG warp
// groups: minimises the per-CTA time max(bytes / per-SM bandwidth, copies *
// per-copy cost) + tiles * fixed consumer work per tile, with tiles of
// NG*ROWS rows at most max_bytes. `mats`
// matrices of `rows` rows each: spread = their tiles are dealt out over the
// CTAs together; otherwise every CTA takes its share of every matrix.
int choose_rows(int rows, int mats, bool spread, int ctas, size_t row_bytes, int NG, int max_rows,
                size_t max_bytes);
// The same cost model's constants (per-SM bytes per microsecond, us per copy).
extern const double kTileSmBytesPerUs, kTileCopyUs;

// Fast path eligibility: group 32, whole groups per row, at most 16 k-slices.
inline bool g32_ok(int in_dim) { return in_dim > 0 && in_dim % 32 == 0 && in_dim <= 16384; }

// Streaming GEMV launch plan.
struct G32Plan {
    Tiling til;
    int J;     // groups of 32 inputs per lane
    int KS;    // k-slices: warps that split one row
    int NG;    // warp groups; group q takes rows [q*ROWS, (q+1)*ROWS) of every tile
    int ROWS;  // rows per warp group per tile (1, 2, 4, 8)
    int nslots;
    int tiles_cta_max;
    int grid, block;
    size_t smem;
};

bool plan_g32(int rows, int in_dim, int sm_count, G32Plan *p);
// The same tiling and warp layout for a launch over `nmat` matrices.
bool plan_g32_batch(const G32Plan &one, int nmat, int sm_count, G32Plan *p);

constexpr int kMaxBatch = 32;  // matrices of one shape per GEMV launch

// One launch: y[m] = W[m] x[m] for nmat matrices of one tiling, their tiles
// dealt out to the CTAs as one range (matrix-major).
struct G32Args {
    const uint8_t *tiles[kMaxBatch];
    const float *x[kMaxBatch];
    float *y[kMaxBatch];
    int nmat;
    int shared_x;  // 1: every x[m] is x[0], planes are built once
    Tiling til;
    int KS, NG, ROWS, nslots, tiles_cta_max;
    int *err;
    uint64_t wait_ns;
};

// k_gemv_g32<J> for J groups of 32 per lane (1 or 2); launched with one
// G32Args argument.
const void *gemv_g32_kernel(int J);

// Flat-index kernels over a raw .rabbit blob (any shape / alignment).
__global__ void k_gemv_flat(const uint8_t *blob, const float *x, float *y, int out_dim,
                            int in_dim);
__global__ void k_dequant_flat(const uint8_t *blob, float *dst, long long n, uint32_t gs);

}  // namespace rb
