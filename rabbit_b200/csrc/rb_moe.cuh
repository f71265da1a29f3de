// rb_moe.cuh -- MoE decode kernels (fused group-32 path and generic path).
#pragma once
#include <stdint.h>

#include <cuda.h>

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
    int withhold_row;          // test hook: router row no CTA publishes (-1: none)
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
// 362-402) would take it alone, with every active expert's tiles read once
// per work unit for all the pairs routed to it:
//   k_batch_route   grid (token, router slice): rmsnorm, the slice's router
//                   rows; the token's last CTA to finish: top-k, slots;
//   k_batch_bucket  one CTA: per local record, the (token, slot) pairs that
//                   use it, in token order (bitmask ranks: deterministic),
//                   cut into units of at most unit_cap pairs;
//   k_tc_images     xn as the tensor-core MMA's B rows, per unit;
//   k_tc_gemm<1>    (unit, 128 rows of W1 and of W3) items: mid = silu(gate)
//                   * up for the unit's pairs (tcgen05, kind::i8);
//   k_tc_images     mid as B rows;
//   k_tc_gemm<0>    (unit, W2 column chunk, 256 rows) items: each chunk's
//                   down rows per pair;
//   k_batch_combine h_out = h + sum_j w_j sum_c down_jc, slots and chunks in
//                   order (forward_v2.c:356-357, 398-399).
constexpr int kMaxBatchTokens = 256;
constexpr int kTcMaxUnit = 32;       // widest work unit (pairs); pair_u = unit * kTcMaxUnit + column
constexpr int kTcMinUnit = 16;       // narrowest (bounds the number of units)
constexpr int kTcRows = 256;         // weight rows per work item (two M = 128 MMAs)
// The tensor-core GEMMs in two configurations, picked per launch by how many
// pairs an expert can expect:
//   wide    one CTA per SM: units of up to 32 pairs, 3 staged chunks, 8 A
//           slots, up to 8 D buffers, 512 tensor-memory columns;
//   narrow  two CTAs per SM (each 256 columns, 89 KB of shared memory, 10
//           warps of at most 96 registers), so one CTA's hand-off latencies
//           overlap the other's work: units of up to 16 pairs, 2 stages, 4 A
//           slots, up to 4 D buffers. Experts drawing more pairs than that
//           are read once per unit.
// Warps: TMA, MMA, 4 unpack, then kReadoutWarps readout warps (8: one item
// row per thread; 4: two, one in each 128-row half).
struct TcWide {
    static constexpr int kUnit = 32, kStages = 3, kASlots = 8, kMaxDBufs = 8, kTmemCols = 512,
                         kCtasPerSm = 1, kReadoutWarps = 8, kThreads = (6 + kReadoutWarps) * 32;
};
struct TcNarrow {
    static constexpr int kUnit = 16, kStages = 2, kASlots = 4, kMaxDBufs = 4, kTmemCols = 256,
                         kCtasPerSm = 2, kReadoutWarps = 4, kThreads = (6 + kReadoutWarps) * 32;
};
inline int tc_threads(bool wide) { return wide ? TcWide::kThreads : TcNarrow::kThreads; }
// MMA N of a unit of n pairs: three digit rows per pair, rounded up to 16.
__host__ __device__ inline int tc_n_of(int n) { return (3 * n + 15) / 16 * 16; }

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
    int *err;                  // device error word (RB_ERR_TIMEOUT)
    uint64_t wait_ns;          // bound of every wait
    // scratch
    float *xn;       // [T][H]
    int *srec;       // [T][kMaxSlots] global record per slot
    float *sw;       // [T][kMaxSlots] combine weight per slot
    int *nslot;      // [T]
    int *pidx;       // [T][kMaxSlots] pair index of (token, slot)
    int *pair_t;     // [P] token of pair
    int unit_cap;    // pairs per work unit of this launch (the GEMMs' configuration)
    int *act, *act_off, *act_cnt;  // [units] work units (record, <= unit_cap of its
                                   // pairs): global record id, first pair, pairs
    int *img_off;    // [units] B rows of the units before this one (sum of tc_n_of)
    int *n_act;      // [2] units, pairs
    float *scores;   // [T][E] router scores
    unsigned *tcount;  // [T] router CTAs done per token (zero between launches)
    int route_split;   // router rows per CTA of k_batch_route
    int ep_rank, ep_size;  // expert-parallel share (1 rank: the whole layer)
    float *mid;      // [P][I]
    float *down;     // [P][tc.KC][H]
    int *pair_u;     // [P] unit * kTcMaxUnit + column of pair
    // B rows of the units: unit u's image holds, per group g of 32 inputs,
    // N_u = tc_n_of(n_u) rows of 32 bytes (row 3c + p = digit p of pair c) as
    // 8-row x 16-byte core matrices, at (img_off[u] G + g N_u) 32 bytes
    uint8_t *xim;    // xn rows (G = H / 32)
    uint8_t *mim;    // mid rows (G = I / 32)
    float *xunit;    // [P] 2^(e-22) of the pair's xn row
    float *munit;    // [P] same for its mid row
    // expert-parallel exchange (rabbit_cuda_moe_set_ep): ep_mode 0 none or
    // all-reduce (the kernels then see a plain share), 2 all-to-all. In
    // all-to-all mode the first T_own tokens are this rank's own; tokens
    // T_own .. T - 1 are the rows received from the peers, peer index
    // qi (ranks other than this one, in rank order) at rows qi * ep_cap ..,
    // each one pair (token, slot) of a peer's token routed to an expert here
    int ep_mode, T_own, ep_cap;
    int *rt_ids;      // [T_own][k] full routing of the own tokens (-1: none)
    float *rt_w;      // [T_own][k]
    int *pos_tab;     // [T_own][k] the pair's row in the owner peer's list (-1: local)
    int4 *send_meta;  // [size-1][cap] {token, slot, local record, valid} sent to peer qi
    int4 *recv_meta;  // [size-1][cap] the same, received from peer qi
    float *send_x;    // [size-1][cap][H] xn rows sent (received ones land in xn)
    float *ret_send;  // [size-1][cap][H] expert outputs of the received rows
    float *ret_recv;  // [size-1][cap][H] expert outputs of the rows sent
};
// route, bucket, combine (same translation unit as the fused kernel); with
// all-to-all exchange 2 pack, 3 return
const void *moe_batch_kernel(int i);  // 0 route, 1 bucket, 2 pack, 3 return, 4 combine

// The tensor-core kernels (rb_moe_tc.cu): one launch argument each, the
// GEMMs with a tensor map over the pool's nibble rows of their phase.
struct alignas(64) TcGemmArgs {
    CUtensorMap tmap;
    MoeBatchArgs b;
};
// 0 x images, 1 gate/up GEMM, 2 mid images, 3 down GEMM; wide: TcWide, else TcNarrow
const void *moe_tc_kernel(int i, bool wide);
size_t tc_gemm_smem(bool wide);  // dynamic shared memory of a GEMM launch
// Tensor maps over a pool's GU and D nibble rows (boxes of 256 rows x 128
// bytes, 128-byte swizzle): 0 built, 1 the tiling does not fit the kernels'
// boxes, 2 the driver's tensor-map encoder is missing or refused.
int tc_tensor_maps(const uint8_t *pool, uint64_t pool_bytes, uint64_t rec_stride, uint64_t off_d,
                   const Tiling &tb, const Tiling &tc, int H, CUtensorMap *gu, CUtensorMap *dn);
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float sg = 1.0f / (1.0f + expf(-g));  // forward_v2.c:327-331
    return (g * sg) * u;
}

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
