// rb_moe_tc.cu -- the multi-token MoE GEMMs on the sm_100a tensor cores
// (tcgen05.mma, kind::i8, accumulators in tensor memory).
//
// T tokens through one layer (rabbit_cuda_moe_prefill[_dev]): every expert
// the chunk touches is streamed from HBM once per work unit (up to kTcUnit of
// the (token, slot) pairs routed to it), and each 32-input group of a weight row
// is multiplied exactly, in integers, as the decode path does it:
//
//   * the weights stay group-32 int4: the warps that unpack a staged tile
//     turn a group's 16 nibble bytes into the MMA's A row, 32 signed bytes
//     16 q (q = nibble - 8), and store it into tensor memory;
//   * each activation row x (one pair's xn or mid) is scaled once by a power
//     of two, X = rint(x 2^(22-e)) with 2^e > max|x|, and split into three
//     signed digits, X = D0 + 256 D1 + 65536 D2 (D0, D1 in [-128, 127], D2 in
//     [-64, 64]); the three digit rows of a pair are three consecutive rows
//     of the MMA's B operand (k_tc_images);
//   * one tcgen05.mma (M = 128 weight rows, N = 3 x pairs rounded up to 16,
//     K = 32) per group and 128-row tile gives the exact plane sums
//     S_p = sum 16 q D_p (|S_p| <= 2^19, multiples of 16) in s32; the readout
//     warps combine them exactly in s32, sum q X = S0 / 16 + 16 S1 + 4096 S2
//     (|sum q X| <= 32 * 8 * 2^22 = 2^30), convert that once to fp32 and
//     accumulate scale_g * it over the groups in order; the row's result is
//     acc * 2^(e-22).
//
// Rounding: the activation's quantisation error is at most 2^(e-23) per
// element (e from the row's largest |x|), the per-group sums are exact, and
// the fp32 accumulation runs over the groups in order -- the same arithmetic
// as the decode kernels' dp4a form, on the tensor pipe.
//
// Work items are (unit, 256 weight rows): for gate/up 128 rows of W1 and the
// same 128 rows of W3 (the pool's GU tiles interleave TRb rows of each), for
// down 256 rows of one column chunk of W2. In the narrow configuration two
// CTAs share an SM (each half the SM's tensor memory, 91 KB of shared memory,
// 10 warps of at most 96 registers a thread), so one CTA's hand-off latencies
// overlap the other's work; the wide one has one CTA of 14 warps per SM. A CTA
// takes a contiguous run of items whose summed cost (a fixed part per group plus the
// readout's 8-pair blocks) is 1 / grid of the launch's, and runs it through a
// warp-specialised pipeline:
//   warp 0       TMA: each 8-group chunk of the item's 256 nibble rows (one
//                cp.async.bulk.tensor box, 128-byte swizzle) and the unit's
//                B rows of those 8 groups (one bulk copy) into a ring of
//                kTcStages stages;
//   warp 1       allocates tensor memory; one lane issues the MMAs (two per
//                group: rows 0..127 and 128..255) and commits them once per
//                group (gdone[g % kTcASlots]: the group's A slot is free and
//                its D buffer full);
//   warps 2..5   unpack: two weight rows per thread (one of each 128-row
//                half), nibbles -> A in TMEM;
//   warps 6..    readout (C::kReadoutWarps: 8 with one weight row per
//                thread, or 4 with two, one in each 128-row half, so the
//                per-group wait, fences and arrival serve both), accumulators in
//                registers; the item's outputs at its end (gate/up: mid =
//                silu(gate) * up, the partner row in the same warp, taken
//                by a shuffle; down: the chunk's rows of each pair).
// A takes kTcASlots slots of 16 columns; the D buffers form a ring of
// nD <= kTcASlots buffers of 2 x NW columns
// (NW: the widest MMA N among the CTA's items), as many as tensor memory holds
// past the A slots, so small units keep more groups in flight. A group's
// gdone phase cannot be overtaken before both its readers have seen it: the
// MMA of group g + kTcASlots needs that group's A, which its unpack writes
// only after seeing group g done, and a D buffer that only the readout of
// group g or a later one frees (nD <= kTcASlots).
// Every wait is bounded; on a timeout the CTA drains its copies and MMAs,
// frees its tensor memory and leaves with RB_ERR_TIMEOUT in the error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "rb_moe.cuh"
#include "rb_tcgen05.cuh"

namespace rb {

namespace {

constexpr int kWarpReadout = 6;  // first readout warp
constexpr uint32_t kNibBytes = kTcRows * 128;  // one stage's nibble box
constexpr uint32_t kColA = 0;                  // A slots: 16 columns each

// The layout a configuration C (TcWide / TcNarrow) implies.
template <class C>
struct TcPlan {
    static constexpr int kMaxN = 3 * C::kUnit;               // MMA N of a full unit
    static constexpr uint32_t kBBytes = 8 * kMaxN * 32;      // one stage's B rows
    static constexpr uint32_t kStageBytes = kNibBytes + kBBytes;
    static constexpr uint32_t kColD = C::kASlots * 16;       // the D ring after the A slots
    static_assert(kColD + 2 * 2 * kMaxN <= (uint32_t)C::kTmemCols,
                  "tensor memory plan: two full buffers");
    static_assert(C::kMaxDBufs <= C::kASlots,
                  "a group's gdone phase is read before it can recur");
    static_assert(kStageBytes % 1024 == 0, "stages stay 1024-byte aligned (128-byte swizzle)");
};

template <class C>
struct TcSmem {
    uint64_t full[C::kStages], empty[C::kStages];
    uint64_t afull[C::kASlots], gdone[C::kASlots];
    uint64_t dempty[C::kMaxDBufs];
    uint64_t mdone;
    uint32_t tmem;
    int abort;
};

// Bounded wait on phase `parity` of `bar` that also gives up once another
// role of the CTA has given up (abort); false then.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, const TcGemmArgs &a,
                                        volatile int *abort, bool sleep) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (sleep) __nanosleep(64);
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > a.b.wait_ns) {
                set_error(a.b.err, RB_ERR_TIMEOUT);
                *abort = 1;
                return false;
            }
        }
    }
}

// The same for every lane of a warp: the lanes agree on the outcome and are
// converged afterwards (the tcgen05 loads and stores that follow are
// warp-collective).
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, const TcGemmArgs &a,
                                             volatile int *abort) {
    const bool ok = tc_wait(bar, parity, a, abort, true);
    return __all_sync(0xffffffffu, ok);
}

// One work item, decoded the same way by every role.
struct Item {
    int u, rec, t0, c;       // unit, global record, first tile of the box, W2 column chunk
    int n, off, N;           // pairs of the unit, first pair, MMA N (3 n rounded up to 16)
    int G;                   // 32-input groups of the item's rows
    int nchunks;             // 8-group chunks
    const uint8_t *img;      // the unit's B rows of group 0 of the item
};

template <bool GU>
__device__ __forceinline__ Item item_of(const TcGemmArgs &a, int item) {
    const MoeBatchArgs &b = a.b;
    Item it;
    if (GU) {
        const int nrb = (b.I + 127) / 128;
        it.u = item / nrb;
        const int rb = item - it.u * nrb;
        it.t0 = rb * (128 / b.tb.TR);
        it.c = 0;
        it.G = b.H / 32;
    } else {
        const int nrb = (b.H + kTcRows - 1) / kTcRows, per = b.tc.KC * nrb;
        it.u = item / per;
        const int d = item - it.u * per;
        it.c = d / nrb;
        it.t0 = (d - it.c * nrb) * (kTcRows / b.tc.TR);
        it.G = b.tc.cols / 32;
    }
    it.rec = b.act[it.u];
    it.off = b.act_off[it.u];
    it.n = b.act_cnt[it.u];
    it.N = tc_n_of(it.n);
    it.nchunks = (it.G + 7) / 8;
    const int Gimg = GU ? b.H / 32 : b.I / 32;  // groups of one B row of the unit's image
    const uint8_t *im = GU ? b.xim : b.mim;
    it.img = im + ((size_t)b.img_off[it.u] * Gimg + (size_t)it.c * it.G * it.N) * 32;
    return it;
}

// The staged row (0..255) that item row m -- TMEM lane m of tile m / 128 --
// holds. Down items: row m. Gate/up items: the item's GU tiles hold TRb gate
// rows then the same TRb up rows, and a lane's gate row and up row must sit
// in one warp, TRh = min(TRb, 16) lanes apart, so the readout can pair them
// by a shuffle: within warp w (m = 32 w + l), lanes l with bit TRh clear take
// gate rows, the others the up rows of the same outputs p = 16 w + (l /
// (2 TRh)) TRh + l % TRh. For TRb <= 16 that is row m itself. *p_out gets p
// (the item's output row), *h_out 0 for gate and 1 for up.
__device__ __forceinline__ int gu_row(int m, int TRb, int *p_out, int *h_out) {
    const int TRh = TRb < 16 ? TRb : 16;
    const int w = m >> 5, l = m & 31, h = (l / TRh) & 1;
    const int p = 16 * w + (l / (2 * TRh)) * TRh + l % TRh;
    *p_out = p;
    *h_out = h;
    return (p / TRb) * 2 * TRb + h * TRb + p % TRb;
}

template <bool GU>
__device__ __forceinline__ int items_per_unit(const MoeBatchArgs &b) {
    return GU ? (b.I + 127) / 128 : b.tc.KC * ((b.H + kTcRows - 1) / kTcRows);
}

// Relative cost of one item of a unit of n pairs: a fixed part per group
// (staging, unpack, MMA, hand-offs) and the readout's 8-pair blocks.
__device__ __forceinline__ long long item_cost(int n) { return 2 + ((n + 7) >> 3); }

// The first item (units in order, items_per_unit each) whose cost-weighted
// start s satisfies s * grid >= T; n_items if none.
template <bool GU>
__device__ int first_item_from(const MoeBatchArgs &b, long long T, int grid) {
    const int U = b.n_act[0], ipu = items_per_unit<GU>(b);
    long long pre = 0;
    for (int u = 0; u < U; ++u) {
        const long long c = item_cost(b.act_cnt[u]);
        const long long end = pre + (long long)ipu * c;
        if (end * grid > T) {  // some item of this unit starts at or past T / grid
            const long long num = T - pre * grid, den = c * grid;
            const long long k = num <= 0 ? 0 : (num + den - 1) / den;
            if (k < ipu) return u * ipu + (int)k;
        }
        pre = end;
    }
    return U * ipu;
}

// This CTA's items: a contiguous run whose summed cost is about 1 / grid of
// the launch's, so CTAs that draw the wide units (e.g. the shared experts,
// routed every token) take fewer of them.
template <bool GU>
__device__ void cta_items(const MoeBatchArgs &b, int bx, int grid, int *i0, int *i1) {
    const int U = b.n_act[0], ipu = items_per_unit<GU>(b);
    long long total = 0;
    for (int u = 0; u < U; ++u) total += (long long)ipu * item_cost(b.act_cnt[u]);
    *i0 = first_item_from<GU>(b, total * bx, grid);
    *i1 = first_item_from<GU>(b, total * (bx + 1), grid);
}

}  // namespace

template <bool GU, class C>
__global__ void __launch_bounds__(C::kThreads, C::kCtasPerSm)
    k_tc_gemm(const __grid_constant__ TcGemmArgs a) {
    using P = TcPlan<C>;
    constexpr int kTcUnit = C::kUnit, kTcStages = C::kStages, kTcASlots = C::kASlots;
    constexpr int kTcMaxDBufs = C::kMaxDBufs;
    constexpr uint32_t kTmemCols = C::kTmemCols, kStageBytes = P::kStageBytes, kColD = P::kColD;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ TcSmem<C> ss;
    // stages at the first 1024-byte boundary of the dynamic block
    uint8_t *stages = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const MoeBatchArgs &b = a.b;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int *abort = &ss.abort;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&ss.full[s], 1);
            mbar_init(&ss.empty[s], 4 + 1);  // the unpack warps + the MMA commit
        }
        for (int j = 0; j < kTcASlots; ++j) {
            mbar_init(&ss.afull[j], 4);
            mbar_init(&ss.gdone[j], 1);
        }
        for (int d = 0; d < kTcMaxDBufs; ++d) {
            mbar_init(&ss.dempty[d], C::kReadoutWarps);
        }
        mbar_init(&ss.mdone, 1);
        ss.abort = 0;
        mbar_init_fence();
        tma_prefetch_map(&a.tmap);
    }
    if (warp == 1) tmem_alloc(&ss.tmem, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ss.tmem;
    launch_dependents();
    wait_prerequisite();

    int i0, i1;
    cta_items<GU>(b, (int)blockIdx.x, (int)gridDim.x, &i0, &i1);
    int nmax = 1;
    {
        const int ipu = items_per_unit<GU>(b);
        for (int item = i0; item < i1; ++item) nmax = max(nmax, b.act_cnt[item / ipu]);
    }
    // the readout loads 24 columns per 8 pairs, up to OV columns past an
    // item's NW-column half (garbage for pairs past n, never used): the ring
    // leaves that much room at its end
    const int NW = tc_n_of(nmax), OV = max(0, 24 * ((nmax + 7) / 8) - NW);
    const int nD = min(kTcMaxDBufs, (int)(kTmemCols - kColD - OV) / (2 * NW));

    if (warp == 0) {
        // ---------------------------------------------------------- TMA --
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int kc = 0;
            bool ok = true;
            for (int item = i0; item < i1 && ok; ++item) {
                const Item it = item_of<GU>(a, item);
                for (int ch = 0; ch < it.nchunks; ++ch, ++kc) {
                    const int s = kc % kTcStages, use = kc / kTcStages;
                    if (use > 0 && !(ok = tc_wait(&ss.empty[s], (use - 1) & 1, a, abort, false)))
                        break;
                    const int g0 = ch * 8, ng = min(8, it.G - g0);
                    const uint32_t bbytes = (uint32_t)ng * it.N * 32;
                    uint8_t *st = stages + (size_t)s * kStageBytes;
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_expect_tx(&ss.full[s], kNibBytes + bbytes);
                    tma_load_5d(st, &a.tmap, ch * 128, 0, it.t0, it.c, it.rec, &ss.full[s], pol);
                    bulk_g2s(st + kNibBytes, it.img + (size_t)g0 * it.N * 32, bbytes, &ss.full[s],
                             policy_evict_last());
                }
            }
            // let every copy still in flight land before the CTA can leave
            for (int q = max(0, kc - kTcStages); q < kc; ++q)
                mbar_wait(&ss.full[q % kTcStages], (q / kTcStages) & 1, b.wait_ns, b.err, 0);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA --
        if (lane == 0) {
            int kc = 0, g = 0;
            int d = 0;
            uint32_t dph = 0;
            bool wrapped = false;
            bool ok = true;
            for (int item = i0; item < i1 && ok; ++item) {
                const Item it = item_of<GU>(a, item);
                const uint32_t idesc = i8_idesc(it.N);
                for (int ch = 0; ch < it.nchunks && ok; ++ch, ++kc) {
                    const int s = kc % kTcStages;
                    if (!(ok = tc_wait(&ss.full[s], (kc / kTcStages) & 1, a, abort, false))) break;
                    const uint32_t bsm = smem_u32(stages + (size_t)s * kStageBytes + kNibBytes);
                    const int ng = min(8, it.G - ch * 8);
                    for (int gi = 0; gi < ng; ++gi, ++g) {
                        const int j = g % kTcASlots;
                        if (!(ok = tc_wait(&ss.afull[j], (g / kTcASlots) & 1, a, abort, false)))
                            break;
                        if (wrapped && !(ok = tc_wait(&ss.dempty[d], dph ^ 1u, a, abort, false)))
                            break;
                        tc_fence_after();
                        const uint64_t bd = kmajor_desc(bsm + (uint32_t)(gi * it.N * 32));
#pragma unroll
                        for (int t = 0; t < 2; ++t)
                            mma_i8_ts(tmem + kColD + (uint32_t)((2 * d + t) * NW),
                                      tmem + kColA + (uint32_t)(j * 16 + t * 8), bd, idesc, 0u);
                        mma_commit(&ss.gdone[j]);
                        if (++d == nD) {
                            d = 0;
                            dph ^= 1u;
                            wrapped = true;
                        }
                    }
                    if (ok) mma_commit(&ss.empty[s]);
                }
            }
            // every MMA issued has completed before the tensor memory is freed
            mma_commit(&ss.mdone);
            mbar_wait(&ss.mdone, 0, b.wait_ns, b.err, 0);
        }
        __syncwarp();
    } else if (warp < kWarpReadout) {
        // ------------------------------------------------------- unpack --
        const int q = warp & 3;
        // the TMEM rows this thread fills: lane q * 32 + lane of both halves
        const int m0 = q * 32 + lane, m1 = 128 + q * 32 + lane;
        int sr0 = m0, sr1 = m1;  // the staged rows they take
        if (GU) {
            int p, h;
            sr0 = gu_row(m0, b.tb.TR, &p, &h);
            sr1 = gu_row(m1, b.tb.TR, &p, &h);
        }
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        int kc = 0, g = 0;
        bool ok = true;
        for (int item = i0; item < i1 && ok; ++item) {
            const Item it = item_of<GU>(a, item);
            for (int ch = 0; ch < it.nchunks && ok; ++ch, ++kc) {
                const int s = kc % kTcStages;
                if (!(ok = tc_wait_warp(&ss.full[s], (kc / kTcStages) & 1, a, abort))) break;
                const uint8_t *row0 = stages + (size_t)s * kStageBytes + (size_t)sr0 * 128;
                const uint8_t *row1 = stages + (size_t)s * kStageBytes + (size_t)sr1 * 128;
                const int ng = min(8, it.G - ch * 8);
                for (int gi = 0; gi < ng; ++gi, ++g) {
                    const int j = g % kTcASlots;
                    if (g >= kTcASlots &&
                        !(ok = tc_wait_warp(&ss.gdone[j], ((g / kTcASlots) - 1) & 1, a, abort)))
                        break;
                    // 128-byte swizzle: 16-byte unit gi of row m sits at unit gi ^ (m % 8)
                    const uint4 w0 = *reinterpret_cast<const uint4 *>(row0 + ((gi ^ (sr0 & 7)) << 4));
                    const uint4 w1 = *reinterpret_cast<const uint4 *>(row1 + ((gi ^ (sr1 & 7)) << 4));
                    uint32_t av[8];
                    nibbles_to_a(w0, av);
                    tmem_st8(tmem + lane_base + kColA + (uint32_t)(j * 16), av);
                    nibbles_to_a(w1, av);
                    tmem_st8(tmem + lane_base + kColA + (uint32_t)(j * 16 + 8), av);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ss.afull[j]);
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&ss.empty[s]);
            }
        }
    } else {
        // ------------------------------------------------------ readout --
        // RPT item rows per thread: with 8 readout warps one (warps 6..9 the
        // rows 0..127, warps 10..13 the rows 128..255), with 4 two, one in
        // each 128-row half, so the per-group waits, fences and arrivals are
        // paid once for both.
        constexpr int RPT = 8 / C::kReadoutWarps;
        const int w = warp - kWarpReadout, q = warp & 3;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        int g = 0;
        int d = 0;
        uint32_t dph = 0;
        bool ok = true;
        for (int item = i0; item < i1 && ok; ++item) {
            const Item it = item_of<GU>(a, item);
            // each row's scales and output position
            int out_row[RPT], gate[RPT];
            bool valid[RPT];
            const float *srow[RPT];
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                const int t = RPT == 1 ? w >> 2 : r;
                const int m = t * 128 + q * 32 + lane;  // the item row
                gate[r] = 0;
                if (GU) {
                    const int TR = b.tb.TR;
                    int p, h;
                    const int sr = gu_row(m, TR, &p, &h);
                    gate[r] = h == 0;
                    const int tile = it.t0 + sr / (2 * TR);
                    const int j = sr % (2 * TR);  // row of the tile: gate rows, then up rows
                    out_row[r] = it.t0 * TR + p;
                    valid[r] = tile < b.tb.ntiles && out_row[r] < b.I;
                    srow[r] = reinterpret_cast<const float *>(
                        b.pool + (size_t)it.rec * b.rec_stride + (size_t)tile * b.tb.tile_stride +
                        (size_t)TR * b.H + (size_t)j * (b.H / 8));
                } else {
                    const int TR = b.tc.TR;
                    const int tile = it.t0 + m / TR;
                    const int j = m % TR;
                    out_row[r] = tile * TR + j;
                    valid[r] = tile < b.tc.rtiles && out_row[r] < b.H;
                    srow[r] = reinterpret_cast<const float *>(
                        b.pool + (size_t)it.rec * b.rec_stride + b.off_d +
                        (size_t)(it.c * b.tc.rtiles + tile) * b.tc.tile_stride +
                        (size_t)TR * (b.tc.cols / 2) + (size_t)j * (b.tc.cols / 8));
                }
            }
            float acc[RPT][kTcUnit];
#pragma unroll
            for (int r = 0; r < RPT; ++r)
#pragma unroll
                for (int c = 0; c < kTcUnit; ++c) acc[r][c] = 0.f;
            const int nblk = (it.n + 7) >> 3;
            // the group's scales, fetched one group ahead
            float s_next[RPT];
#pragma unroll
            for (int r = 0; r < RPT; ++r) s_next[r] = valid[r] ? __ldg(srow[r]) : 0.f;
            for (int ch = 0; ch < it.nchunks && ok; ++ch) {
                const int ng = min(8, it.G - ch * 8);
#pragma unroll 1
                for (int gi = 0; gi < ng; ++gi) {
                    float s[RPT];
                    const int gn = ch * 8 + gi + 1;
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        s[r] = s_next[r];
                        s_next[r] = valid[r] && gn < it.G ? __ldg(srow[r] + gn) : 0.f;
                    }
                    if (!(ok = tc_wait_warp(&ss.gdone[g % kTcASlots], (g / kTcASlots) & 1, a, abort)))
                        break;
                    tc_fence_after();
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        const int t = RPT == 1 ? w >> 2 : r;
                        const uint32_t dt =
                            tmem + lane_base + kColD + (uint32_t)((2 * d + t) * NW);
#pragma unroll
                        for (int blk = 0; blk < kTcUnit / 8; ++blk) {
                            if (blk < nblk) {
                                int v16[16], v8[8];
                                tmem_ld16(dt, v16, blk * 24);
                                tmem_ld8(dt, v8, blk * 24 + 16);
                                tmem_wait_ld();
                                int v[24];
#pragma unroll
                                for (int i = 0; i < 16; ++i) v[i] = v16[i];
#pragma unroll
                                for (int i = 0; i < 8; ++i) v[16 + i] = v8[i];
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    const int qx = (v[3 * i] >> 4) + v[3 * i + 1] * 16 +
                                                   v[3 * i + 2] * 4096;
                                    acc[r][blk * 8 + i] =
                                        fmaf(s[r], (float)qx, acc[r][blk * 8 + i]);
                                }
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ss.dempty[d]);
                    ++g;
                    if (++d == nD) {
                        d = 0;
                        dph ^= 1u;
                    }
                }
            }
            if (!ok) break;
            // the item's outputs: acc * 2^(e-22) per pair
            const float *unit = GU ? b.xunit : b.munit;
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
#pragma unroll
                for (int c = 0; c < kTcUnit; ++c) {
                    if (c >= it.n) break;
                    const float v = acc[r][c] * unit[it.off + c];
                    if (GU) {
                        const int TRh = b.tb.TR < 16 ? b.tb.TR : 16;
                        const float up = __shfl_xor_sync(0xffffffffu, v, TRh);
                        if (valid[r] && gate[r])
                            b.mid[(size_t)(it.off + c) * b.I + out_row[r]] = silu_mul(v, up);
                    } else if (valid[r]) {
                        b.down[((size_t)(it.off + c) * b.tc.KC + it.c) * b.H + out_row[r]] = v;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Activation rows of one pair (one CTA per pair; pairs past the chunk's
// count leave at once) as the MMA's B rows: the row's exponent e (2^e >
// max|x|), unit[pair] = 2^(e-22), and for every group of 32 the three digit
// rows 3c, 3c + 1, 3c + 2 (c = the pair's column in its unit) of the unit's
// image, in the K order of nibbles_to_a, laid out as 8-row x 16-byte core
// matrices (see rb_tcgen05.cuh).
template <bool MID>
__global__ void __launch_bounds__(256) k_tc_images(MoeBatchArgs a) {
    __shared__ float red[8];
    launch_dependents();
    wait_prerequisite();
    const int pr = blockIdx.x;
    if (pr >= a.n_act[1]) return;
    const int K = MID ? a.I : a.H, G = K / 32;
    const float *x = MID ? a.mid + (size_t)pr * a.I : a.xn + (size_t)a.pair_t[pr] * a.H;
    const int tid = threadIdx.x;
    float mx = 0.f;
    for (int i = tid * 4; i < K; i += 256 * 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + i));
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 126;  // 2^e > max|x|
    if (e < -100) e = -100;
    const float scale = __int_as_float((127 + 22 - e) << 23);  // 2^(22-e)
    if (tid == 0) (MID ? a.munit : a.xunit)[pr] = __int_as_float((127 - 22 + e) << 23);
    const int uc = a.pair_u[pr], u = uc / kTcMaxUnit, c = uc - u * kTcMaxUnit;
    const int N = tc_n_of(a.act_cnt[u]);
    uint8_t *img = (MID ? a.mim : a.xim) + (size_t)a.img_off[u] * G * 32;
    for (int g = tid; g < G; g += 256) {
        const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)g * 32);
        int X[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = __ldcg(x4 + i);
            const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)  // rint via the 1.5 * 2^23 shift (|x 2^(22-e)| <= 2^22)
                X[4 * i + r] = __float_as_int(fmaf(f[r], scale, 12582912.0f)) - 0x4B400000;
        }
        // digits in K order: D0 = X mod 256 in [-128, 127], then the rest
        uint32_t wd[3][8];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                const int v = X[tc_k_element(4 * w + bb)];
                const int d0 = ((v + 128) & 255) - 128;
                const int v1 = (v - d0) >> 8;
                const int d1 = ((v1 + 128) & 255) - 128;
                const int d2 = (v1 - d1) >> 8;
                b0 |= (uint32_t)(d0 & 255) << (8 * bb);
                b1 |= (uint32_t)(d1 & 255) << (8 * bb);
                b2 |= (uint32_t)(d2 & 255) << (8 * bb);
            }
            wd[0][w] = b0;
            wd[1][w] = b1;
            wd[2][w] = b2;
        }
        uint8_t *gb = img + (size_t)g * N * 32;
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            const int r = 3 * c + p;
#pragma unroll
            for (int kh = 0; kh < 2; ++kh)
                *reinterpret_cast<uint4 *>(gb + ((r >> 3) * 2 + kh) * 128 + (r & 7) * 16) =
                    make_uint4(wd[p][4 * kh], wd[p][4 * kh + 1], wd[p][4 * kh + 2],
                               wd[p][4 * kh + 3]);
        }
    }
}

const void *moe_tc_kernel(int i, bool wide) {
    switch (i) {
        case 0: return (const void *)k_tc_images<false>;
        case 1: return wide ? (const void *)k_tc_gemm<true, TcWide>
                            : (const void *)k_tc_gemm<true, TcNarrow>;
        case 2: return (const void *)k_tc_images<true>;
        case 3: return wide ? (const void *)k_tc_gemm<false, TcWide>
                            : (const void *)k_tc_gemm<false, TcNarrow>;
        default: return nullptr;
    }
}

size_t tc_gemm_smem(bool wide) {
    return wide ? 1024 + (size_t)TcWide::kStages * TcPlan<TcWide>::kStageBytes
                : 1024 + (size_t)TcNarrow::kStages * TcPlan<TcNarrow>::kStageBytes;
}

// ----------------------------------------------------------- tensor maps --
namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}
}  // namespace

int tc_tensor_maps(const uint8_t *pool, uint64_t pool_bytes, uint64_t rec_stride, uint64_t off_d,
                   const Tiling &tb, const Tiling &tc, int H, CUtensorMap *gu, CUtensorMap *dn) {
    if (rec_stride == 0 || tb.TR > 64 || 128 % tb.TR || tc.TR > 256 || kTcRows % tc.TR) return 1;
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return 2;
    const uint64_t R = pool_bytes / rec_stride;
    const cuuint32_t es[5] = {1, 1, 1, 1, 1};
    {   // GU nibble rows: [record][tile][2 TRb rows][H / 2 bytes]
        const cuuint64_t dims[5] = {(cuuint64_t)H / 2, (cuuint64_t)2 * tb.TR,
                                    (cuuint64_t)tb.ntiles, 1, R};
        const cuuint64_t strides[4] = {(cuuint64_t)H / 2, tb.tile_stride,
                                       (cuuint64_t)tb.tile_stride * tb.ntiles, rec_stride};
        const cuuint32_t box[5] = {128, (cuuint32_t)(2 * tb.TR), (cuuint32_t)(128 / tb.TR), 1, 1};
        if (enc(gu, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<uint8_t *>(pool), dims, strides,
                box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return 2;
    }
    {   // D nibble rows: [record][chunk][tile][TRc rows][cols / 2 bytes], from off_d
        const cuuint64_t dims[5] = {(cuuint64_t)tc.cols / 2, (cuuint64_t)tc.TR,
                                    (cuuint64_t)tc.rtiles, (cuuint64_t)tc.KC, R};
        const cuuint64_t strides[4] = {(cuuint64_t)tc.cols / 2, tc.tile_stride,
                                       (cuuint64_t)tc.tile_stride * tc.rtiles, rec_stride};
        const cuuint32_t box[5] = {128, (cuuint32_t)tc.TR, (cuuint32_t)(kTcRows / tc.TR), 1, 1};
        if (enc(dn, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<uint8_t *>(pool + off_d), dims,
                strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
            CUDA_SUCCESS)
            return 2;
    }
    return 0;
}

}  // namespace rb
