// rb_moe.cuh -- MoE decode kernels (fused group-32 path and generic path).
#pragma once
#include <stdint.h>

#include "rb_device.cuh"
#include "rb_gemv.cuh"

struct rabbit_cuda_moe;

namespace rb {

constexpr int kMaxSlots = 72;  // top-k (<= 8) + shared (<= 64)
constexpr int kPartRing = 8;   // partial-sum regions between consumers and epilogue
constexpr int kMaxGrid = 1024; // CTAs of the fused kernel (one per SM)
constexpr int kMoeConsumerWarps = 8;  // consumer warps of the fused kernel (2 per SM sub-partition)

// Routing result shared by the generic kernels (device memory).
struct Route {
    int nact;                  // active slots
    int rec[kMaxSlots];        // global record id per slot
    float w[kMaxSlots];        // combine weight per slot
};

struct MoeFusedArgs {
    const float *h_in;
    float *h_out;
    int *ids_out;     // [k]
    float *w_out;     // [k]
    const float *rms;     // [H]
    const float *router;  // [E, H]
    const uint8_t *pool;
    uint64_t rec_stride;
    uint64_t off_d;  // record = [GU tiles (gate+up pairs over I rows)] [D tiles over H rows]
    Tiling tb;       // GU tiling: rows I, in H, tile_bytes/stride of the gate+up pair
    Tiling tc;       // D tiling: rows H, in I, KC column chunks
    int rec_base;  // global record of local expert 0 in this layer
    int n_local;   // local ids >= n_local have no record (skipped)
    int H, E, k, I, S;
    int usable;    // 0: records too small, experts add nothing (forward_v2.c:319-322)
    int route_local;  // 1: every CTA computes all router rows from shared memory
    int route_stage;  // route_local == 0: 1 = each CTA's own rows staged in shared memory
    unsigned long long *scores;  // [E] tagged router scores (route_local == 0)
    // scratch shared between CTAs, every value tagged {float, seq} (64-bit)
    unsigned long long *mid;   // [k+S][I]
    unsigned long long *down;  // [k+S][tc.KC][H]: down rows per slot and column chunk
    unsigned *flags;           // [grid]: seq once the CTA has read h
    unsigned seq;              // this launch's tag (never 0)
    int *err;
    uint64_t wait_ns;
    // plan: CW consumer warps; phase B (gate/up, in = H) uses KSb warps per
    // row, NGb warp groups of ROWSb rows per tile, JB groups per lane; phase C
    // (down, in = I) likewise with KSc, NGc, ROWSc, JC
    int CW, KSb, NGb, ROWSb, JB, KSc, NGc, ROWSc, JC, nslots;
    uint32_t slot_bytes;
    int part_floats;  // floats per partial region
};

// k_moe_decode_g32<JB, JC, PACKED> for JB / JC groups of 32 per lane in
// phases B / C (1 or 2 each) and the combine's batching (PACKED: fewer than 8
// column chunks of W2); one CTA per SM, all resident, one MoeFusedArgs
// argument.
const void *moe_fused_kernel(int JB, int JC, bool packed);
inline bool combine_packed(int KC) { return KC < 8; }

// ------------------------------------------------------- multi-token path --
// T tokens through one layer's MoE block, each as moe_step (forward_v2.c:
// 362-402) would take it alone, with every active expert's tiles read once for
// all the tokens routed to it:
//   k_batch_route   grid (token, router slice): rmsnorm, the slice's router
//                   rows; the token's last CTA to finish: top-k, slots;
//   k_batch_bucket  one CTA: per local record, the (token, slot) pairs that
//                   use it, in token order (bitmask ranks: deterministic),
//                   cut into units of at most kBatchTokChunk pairs;
//   k_batch_xplanes xn as activation planes (the integer MMA's B operand);
//   k_batch_gu      (unit, GU tile) items: mid = silu(gate) * up for the
//                   unit's tokens, integer tensor-core MMAs per group;
//   k_batch_mplanes mid as activation planes;
//   k_batch_down    (unit, D tile) items: each column chunk's down rows per
//                   pair, integer tensor-core MMAs per group;
//   k_batch_combine h_out = h + sum_j w_j sum_c down_jc, slots and chunks in
//                   order (forward_v2.c:356-357, 398-399).
constexpr int kMaxBatchTokens = 256;
constexpr int kBatchTokChunk = 16;  // tokens per work unit (two n8 blocks of the MMA)
constexpr int kBatchThreads = 512;  // threads of k_batch_gu / k_batch_down
// The activation planes of the multi-token kernels, kept in the order the
// integer MMA (m16n8k32, B operand) reads them. For work unit u, group g of
// 32 activations and 8-column block nb, lane l = 4 i + t of a warp loads
// three uint2 at bfrag[((u G + g) 2 + nb) 32 + l]: planes 0..2 of
// X = rint(x 2^(22-e)) of column 8 nb + i, each as (bytes of the even
// elements 8t, 8t+2, 8t+4, 8t+6 ; bytes of the odd ones) -- the k order of
// the nibble operand (see make_xplanes). The readout terms of column c,
// (-8 sum X, the unit 2^(e-22) as float bits), are at rfrag[(u G + g) 16 + c].
constexpr int kFragCols = 16;  // columns of one unit (= kBatchTokChunk)
// One multi-token work item of `rows` weight rows staged in shared memory.
// Banded (when a band's nibble rows fill at least 4 KB, so its copies stay
// large): 8 bands of u = 2 ceil(rows / 16) consecutive rows, nibble rows at
// stride ns within a band and bands at a stride bs = 16 (mod 128) bytes, so
// the 8 rows a tensor-core fragment reads (one per band) start in distinct
// banks; the scale rows banded the same way when every band's (and tile's)
// scale rows are a whole number of 16-byte units (sc_band), else the tiles'
// scale blocks back to back. Otherwise the rows in order (fragment rows g and
// g + 8 of block mb are rows 16 mb + g and + 8), two copies per tile.
struct StageGeom {
    int u;             // rows per band
    uint32_t ns, bs;   // nibble row stride, band stride (bytes)
    uint32_t ss, sbs;  // scale row stride, band stride (sc_band)
    uint32_t sc_off;   // scales' offset
    uint32_t bytes;    // the item's buffer, 128-byte aligned
    bool banded, sc_band, ok;  // ok: every copy a whole number of 16-byte units
};
__host__ __device__ inline StageGeom stage_geom(int rows, int tile_rows, int nib_bytes, int sc_bytes) {
    StageGeom g;
    g.u = 2 * ((rows + 15) / 16);
    g.banded = (size_t)g.u * nib_bytes >= 4096;
    g.ns = (uint32_t)nib_bytes;
    g.bs = g.banded ? (uint32_t)align_up((size_t)g.u * nib_bytes, 128) + 16 : 0u;
    g.sc_band = g.banded && ((size_t)g.u * sc_bytes) % 16 == 0 &&
                ((size_t)tile_rows * sc_bytes) % 16 == 0;
    g.ss = (uint32_t)sc_bytes;
    g.sbs = g.sc_band ? (uint32_t)align_up((size_t)g.u * sc_bytes, 128) + 16 : 0u;
    g.sc_off = g.banded ? 8 * g.bs : (uint32_t)align_up((size_t)rows * nib_bytes, 16);
    g.bytes = (uint32_t)align_up(
        (size_t)g.sc_off + (g.sc_band ? 8 * (size_t)g.sbs : (size_t)rows * sc_bytes), 128);
    g.ok = nib_bytes % 16 == 0 && (g.sc_band || ((size_t)tile_rows * sc_bytes) % 16 == 0) &&
           (g.banded || ((size_t)tile_rows * nib_bytes) % 16 == 0);
    return g;
}
// Most work-item buffers of a multi-token GEMM kernel. Measured on the
// DeepSeek- and Mixtral-8x22B-shaped chunks: 2 (one item in flight while one
// is computed) beat 3, 4 and 8 buffers by 1-3%.
constexpr int kTcMaxBuf = 2;
// Warp partial sums of the multi-token tensor-core tiles: per warp two 16-row
// blocks x two 8-column blocks of 16x8 fragments.
constexpr int kTcRedFloats = (kBatchThreads / 32) * 2 * (kBatchTokChunk / 8) * 128;

struct MoeBatchArgs {
    const float *h_in;
    float *h_out;
    int T;
    int *ids_out;    // [T][k] or nullptr
    float *w_out;    // [T][k] or nullptr
    const float *rms, *router;
    const uint8_t *pool;
    uint64_t rec_stride, off_d;
    int rec_base, n_local, H, E, k, I, S, usable;
    Tiling tb, tc;   // GU tiles (gate + up pair), D tiles (column chunks)
    int gu_tpi;                // GU tiles per work item (2 TR gu_tpi <= 64)
    int dn_tpi;                // D row tiles of one chunk per work item (TR dn_tpi <= 64)
    int gu_nbuf, dn_nbuf;      // staged items per CTA: one computed, the rest in flight
    int *err;                  // device error word (RB_ERR_TIMEOUT)
    uint64_t wait_ns;          // bound of every wait
    // scratch
    float *xn;       // [T][H]
    int *srec;       // [T][kMaxSlots] global record per slot
    float *sw;       // [T][kMaxSlots] combine weight per slot
    int *nslot;      // [T]
    int *pidx;       // [T][kMaxSlots] pair index of (token, slot)
    int *pair_t;     // [P] token of pair
    int *act, *act_off, *act_cnt;  // [units] work units (record, <= kBatchTokChunk of its
                                   // pairs): global record id, first pair, pairs
    int *n_act;      // [2] units, pairs
    float *scores;   // [T][E] router scores
    unsigned *tcount;  // [T] router CTAs done per token (zero between launches)
    int route_split;   // router rows per CTA of k_batch_route
    int ep_rank, ep_size;  // expert-parallel share (1 rank: the whole layer)
    float *mid;      // [P][I]
    float *down;     // [P][tc.KC][H]
    int *pair_u;     // [P] unit * 16 + column of pair
    uint2 *xbf;      // [units][H / 32][2][32][3] planes of xn per unit column (see kFragCols)
    int2 *xrf;       // [units][H / 32][16] their readout terms
    uint2 *mbf;      // [units][I / 32][2][32][3] planes of mid
    int2 *mrf;       // [units][I / 32][16]
};
// The five kernels (same translation unit as the fused kernel).
const void *moe_batch_kernel(int i);  // 0 route, 1 bucket, 2 gu, 3 down, 4 combine, 5 planes

// ---- generic path (any quant / shape): route, up (gate+up+silu), down, combine
struct MoeGenericArgs {
    const float *h_in;
    float *h_out;
    int *ids_out;
    float *w_out;
    const float *rms;
    const float *router;
    const uint8_t *pool;  // raw records at rec_stride
    uint64_t rec_stride;
    uint64_t expert_size;
    int rec_base, n_local;
    int H, E, k, I, S, quant, usable;
    float *xn;     // [H]
    float *scores; // [E]
    float *mid;    // [slots][I]
    float *down;   // [slots][H]
    Route *route;
};

__global__ void k_moe_route(MoeGenericArgs a);
__global__ void k_moe_up_generic(MoeGenericArgs a);
__global__ void k_moe_down_generic(MoeGenericArgs a);
__global__ void k_moe_combine(MoeGenericArgs a);

// Device, layer count and hidden size of a pool (for code that runs a pool's
// layers as part of a larger model).
void moe_shape(const struct ::rabbit_cuda_moe *p, int *device, int *n_layers, int *hidden);

}  // namespace rb
