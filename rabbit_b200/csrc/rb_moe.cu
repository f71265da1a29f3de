// rb_moe.cu -- C ABI: HBM-resident expert pool + MoE decode entry points.
//
// The pool replaces the reference's expert cache / mmap fetch
// (memory.c:94-253, moe.c:73-117): every record of the .rabbit expert table
// lives in HBM for the life of the pool. Records are read from the host map,
// copied into one of two pinned staging buffers, and moved with
// cudaMemcpyAsync on a side stream (double buffered: the host fills one
// buffer while the other is in flight).
//
// Group-32 int4 records are re-laid out on the way in -- the packed values
// are the same bytes, only moved -- into row tiles the kernels fetch with one
// bulk copy each: [GU tiles: TRb rows of gate nibbles | up nibbles | gate
// scales | up scales] over the I rows, then [D tiles: TRc rows of down
// nibbles | scales] over the H rows. Other formats are kept verbatim.
#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <condition_variable>
#include <mutex>
#include <numeric>
#include <thread>
#include <vector>

#include "rb_ep.h"
#include "rb_gemv.cuh"
#include "rb_moe.cuh"
#include "rb_runtime.h"

namespace {

constexpr size_t kPinChunk = 32ull << 20;  // bytes per pinned staging buffer
constexpr int kIoSlots = 3;                 // pinned record buffers of the file reader
constexpr uint64_t kIoAlign = 4096;         // O_DIRECT offset / length / buffer alignment

inline uint64_t nbytes_g32(uint64_t n) { return 4 + 4 * ((n + 31) / 32) + (n + 1) / 2; }

// A pre-tiled record (RABBIT_CUDA_QUANT_INT4_TILED) is the pool's tiled
// record (rec_stride bytes) followed by kTileTrailer bytes: a magic word and
// the tile plan it was laid out for, so a pool planned otherwise refuses it.
constexpr uint64_t kTileTrailer = 256;
constexpr char kTileMagic[8] = {'R', 'B', '2', 'T', 'I', 'L', 'E', '1'};
struct TileTrailer {
    char magic[8];
    uint32_t trb, trc, kc, h, inter;
    uint64_t rec_stride;
};

inline uint64_t mix_host(uint64_t seed, uint64_t r) {
    uint64_t z = seed * 0x100000001B3ull + r * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 33)) * 0xFF51AFD7ED558CCDull;
    return z ^ (z >> 33);
}

}  // namespace

struct rabbit_cuda_moe {
    int device = -1;
    rb::DevCtx *ctx = nullptr;
    // model
    int L = 0, H = 0, E = 0, k = 0, I = 0, S = 0, quant = 4;
    uint64_t expert_size = 0;
    int n_records = 0, epl = 0, shared_table = 0;
    const uint8_t *host_map = nullptr;
    bool usable = false, fast = false;
    bool pretiled = false;  // records arrive in the tiled layout (RABBIT_CUDA_QUANT_INT4_TILED)
    // Windowed pools (rabbit_cuda_moe_create_window): HBM blocks of epl records
    // for `window` layers, reassigned least recently used first; 0: every
    // layer has its own block. pool_records = the records HBM holds.
    int window = 0, pool_records = 0;
    std::vector<int> layer_block, block_layer;
    std::vector<uint64_t> block_use;
    uint64_t use_clock = 0;
    std::vector<cudaEvent_t> block_ev, block_up_ev;  // last kernel reading / last copy into a block
    // pool
    uint8_t *pool = nullptr;
    uint64_t rec_stride = 0, pool_bytes = 0;
    uint64_t off_d = 0;  // GU tiles at 0, D tiles at off_d (group-32 layout)
    std::vector<uint8_t> resident;
    // dense per-layer inputs
    float *rms = nullptr, *router = nullptr;
    // scratch
    float *scores = nullptr, *mid = nullptr, *xn = nullptr, *down = nullptr;
    // host-buffer decode: h_in, and one block [h_out (H) | ids (8) | weights
    // (8) | error word (4)] that comes back to the host in one copy
    float *h_in = nullptr, *h_out = nullptr, *w_int = nullptr;
    int *ids_int = nullptr, *err_io = nullptr;
    uint8_t *dio = nullptr;
    size_t dio_bytes = 0;
    unsigned *flags = nullptr;  // fused path: per-CTA "h read" tags
    unsigned seq = 1;           // tag of the next fused launch (never 0)
    rb::Route *route = nullptr;
    // upload machinery
    cudaStream_t up = nullptr;
    void *pin[2] = {nullptr, nullptr};
    uint64_t pin_cap = 0;  // bytes per pinned staging buffer
    cudaEvent_t pin_ev[2] = {nullptr, nullptr};
    int pin_next = 0;
    // host-buffer decode staging
    float *pin_io = nullptr;
    float *pin_io_dev = nullptr;  // the same pinned block as the device addresses it
    // fused plan
    rb::MoeFusedArgs plan{};
    int grid = 0, block = 0;
    size_t smem = 0;
    // multi-token scratch (rabbit_cuda_moe_prefill*), grown on demand
    int bt_cap = 0;          // tokens the scratch holds
    void *bt_block = nullptr;  // one allocation, carved below
    rb::MoeBatchArgs bt{};   // scratch pointers of the block
    float *bt_h = nullptr;   // [bt_cap][H] device copy of host tokens
    int *bt_ids = nullptr;   // [bt_cap][8] routing of host-buffer calls
    float *bt_w = nullptr;   // [bt_cap][8]
    float *bt_pin = nullptr; // pinned [bt_cap][H] + ids/weights
    int ep_rank = 0, ep_size = 1;  // expert-parallel share of the multi-token path
    // exchange of that share (rabbit_cuda_moe_set_ep): the communicator, the
    // mode, and the all-to-all buffers for ep_tcap own tokens
    rabbit_cuda_ep *ep = nullptr;
    int ep_mode = 0;
    void *ep_block = nullptr;
    int ep_tcap = 0;
    int withhold_row = -1;  // test hook for the next fused launch (see rabbit_cuda_moe_debug_*)
    // tensor maps of the multi-token GEMMs over the pool's GU and D nibble
    // rows (tc_ok: built; otherwise the multi-token path runs per token)
    CUtensorMap tm_gu{}, tm_dn{};
    bool tc_ok = false;
    // counters (rabbit_cuda_moe_stats[_ex]): kernel calls served from HBM,
    // calls refused because their layer was not resident, records uploaded,
    // records dropped from a window block taken for another layer, bytes moved
    uint64_t hbm_hits = 0, uploads = 0, h2d_bytes = 0;
    mutable uint64_t misses = 0;
    uint64_t evictions = 0;
    std::vector<uint8_t> img;  // host image of one record in the tiled layout
    // file-backed upload (rabbit_cuda_moe_upload_file): pinned record buffers
    // the reader thread fills, and pinned tiled images (group-32 pools), each
    // with the event of the last copy that reads it
    uint8_t *io_raw[kIoSlots] = {};
    uint8_t *io_img[2] = {};
    cudaEvent_t io_raw_ev[kIoSlots] = {}, io_img_ev[2] = {};
    uint64_t io_raw_cap = 0;
};

namespace rb {

static bool g_moe_attr[kMaxDevices];

static int layer_map(const rabbit_cuda_moe *p, int layer, int *base, int *n_local) {
    if (layer < 0 || layer >= p->L) return fail(RABBIT_CUDA_ERR_ARGS, "layer %d out of range", layer);
    if (p->window) {  // the layer's block, if it holds one
        const int b = p->layer_block[layer];
        if (b < 0) {
            p->misses++;
            return fail(RABBIT_CUDA_ERR_ARGS, "layer %d not uploaded (not in the pool's window)", layer);
        }
        *base = b * p->epl;
        *n_local = std::min(p->epl, p->n_records - layer * p->epl);
        return RABBIT_CUDA_OK;
    }
    if (p->shared_table) {
        *base = 0;
        *n_local = p->n_records;
    } else {
        *base = layer * p->epl;
        *n_local = std::min(p->epl, p->n_records - *base);
        if (*n_local < 0) *n_local = 0;
    }
    return RABBIT_CUDA_OK;
}

// The pool records of `layer` for an upload: its block in a windowed pool
// (taking the least recently used block, and dropping the layer it held, when
// the layer has none: the side stream first waits for the last kernel that
// read that block), else its place in the table. *src_base is the layer's
// first record in the model's expert table.
static int layer_slot(rabbit_cuda_moe *p, int layer, int *base, int *n_local, int *src_base) {
    if (!p->window) {
        const int st = layer_map(p, layer, base, n_local);
        *src_base = *base;
        return st;
    }
    if (layer < 0 || layer >= p->L) return fail(RABBIT_CUDA_ERR_ARGS, "layer %d out of range", layer);
    int b = p->layer_block[layer];
    if (b < 0) {
        b = 0;
        for (int i = 1; i < p->window; ++i)
            if (p->block_use[i] < p->block_use[b]) b = i;
        if (p->block_layer[b] >= 0) p->layer_block[p->block_layer[b]] = -1;
        for (int r = 0; r < p->epl; ++r) p->evictions += p->resident[(size_t)b * p->epl + r];
        std::fill(p->resident.begin() + (size_t)b * p->epl, p->resident.begin() + (size_t)(b + 1) * p->epl, 0);
        RB_CUDA(cudaStreamWaitEvent(p->up, p->block_ev[b], 0));
        p->block_layer[b] = layer;
        p->layer_block[layer] = b;
    }
    p->block_use[b] = ++p->use_clock;
    *base = b * p->epl;
    *n_local = std::min(p->epl, p->n_records - layer * p->epl);
    *src_base = layer * p->epl;
    return RABBIT_CUDA_OK;
}

// Windowed pools: kernels on `s` that read the layer's block wait for the
// copies into it, and later copies into the block wait for them.
static int window_enter(rabbit_cuda_moe *p, int layer, cudaStream_t s) {
    if (!p->window || layer < 0 || layer >= p->L || p->layer_block[layer] < 0) return RABBIT_CUDA_OK;
    RB_CUDA(cudaStreamWaitEvent(s, p->block_up_ev[p->layer_block[layer]], 0));
    return RABBIT_CUDA_OK;
}
static int window_leave(rabbit_cuda_moe *p, int layer, cudaStream_t s) {
    if (!p->window || layer < 0 || layer >= p->L || p->layer_block[layer] < 0) return RABBIT_CUDA_OK;
    const int b = p->layer_block[layer];
    RB_CUDA(cudaEventRecord(p->block_ev[b], s));
    p->block_use[b] = ++p->use_clock;
    return RABBIT_CUDA_OK;
}

// Bytes per element of the mid / down scratch: the fused kernel tags every
// value with its launch ({float, seq}, 8 bytes); the generic kernels use
// plain floats.
static size_t scratch_elt(const rabbit_cuda_moe *p) { return p->fast ? 8 : 4; }
static size_t mid_bytes(const rabbit_cuda_moe *p) {
    return scratch_elt(p) * (size_t)std::max(1, p->k + p->S) * p->I;
}
static size_t down_bytes(const rabbit_cuda_moe *p) {
    return scratch_elt(p) * (size_t)std::max(1, p->k + p->S) * (p->fast ? p->plan.tc.KC : 1) *
           p->H;
}

// The next launch tag. Tags never repeat while the scratch lives: on wrap the
// tagged buffers are cleared (on the launch's stream) and tags restart at 1.
static unsigned next_seq(unsigned *seq, void *tagged[], const size_t bytes[], int n,
                         cudaStream_t s) {
    if (*seq == 0) *seq = 1;  // 0 is the tag of zeroed memory
    if (*seq == 0xFFFFFFFFu) {
        for (int i = 0; i < n; ++i) cudaMemsetAsync(tagged[i], 0, bytes[i], s);
        *seq = 1;
    }
    return (*seq)++;
}

// The fused decode tags what its CTAs share with a number the host picks at
// call time (next_seq). A launch recorded into a CUDA graph would keep that
// number on every replay, so a replay could accept values an earlier replay
// left behind; calls made while their stream is capturing are refused.
static int refuse_capture(cudaStream_t s, const char *who) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const cudaError_t e = cudaStreamIsCapturing(s, &cs);
    if (e != cudaSuccess) return cuda_fail(e, who);
    if (cs != cudaStreamCaptureStatusNone)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "%s: the stream is being captured; each launch needs a tag chosen when it "
                    "is issued, so this call cannot be recorded into a graph",
                    who);
    return RABBIT_CUDA_OK;
}

// One fused decode launch, programmatic-dependent: it may start while the
// kernel before it on the stream finishes (it waits for that kernel before it
// reads h or touches scratch), which hides the launch gap between layers.
// Its CTAs wait on one another's data, so all of them must be resident: the
// grid is one CTA per SM and the shared memory admits exactly one per SM
// (checked at pool creation), and the next launch on the stream starts only
// after every CTA of this one has started. The cooperative-launch attribute
// would state that guarantee but keeps consecutive launches from overlapping;
// if the device is shared and some CTAs cannot be placed, the bounded waits
// end the launch with RABBIT_CUDA_ERR_TIMEOUT.
static cudaError_t launch_fused(const rabbit_cuda_moe *p, MoeFusedArgs &a, cudaStream_t s) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(p->block);
    cfg.dynamicSmemBytes = p->smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&a};
    return cudaLaunchKernelExC(&cfg, moe_fused_kernel(a.JB, a.JC, combine_packed(a.tc.KC)), args);
}

// Shared-memory bytes in front of the ring, in the order k_moe_decode_g32
// carves them: xn, reduction scratch, slot records/weights, flags, scores.
static size_t fused_head_bytes(int H, int E) {
    size_t off = align_up((size_t)(H / 32) * 33 * 4, 128);
    off += 128 + 2 * (size_t)kMaxSlots * 4;
    off = align_up(off + 16, 128);
    off = align_up(off + (size_t)E * 4, 128);
    return off;
}

static bool plan_fused(rabbit_cuda_moe *p, int sm_count) {
    const int H = p->H, I = p->I;
    if (!g32_ok(H) || !g32_ok(I)) return false;
    MoeFusedArgs &a = p->plan;
    a.JB = lane_groups(H / 32);
    a.KSb = kslices(H / 32, a.JB);
    a.NGb = std::max(1, kMoeConsumerWarps / a.KSb);  // warp groups in phase B
    // W2 is split into column chunks of CG groups: the largest divisor of I/32
    // up to 32 (1024 inputs), at most 16 chunks. A CTA then needs only its
    // chunk of mid, not all of it.
    const int Gc = I / 32;
    int CG = 0;
    for (int g = std::min(Gc, 32); g >= 1 && !CG; --g)
        if (Gc % g == 0) CG = g;
    const int KCc = Gc / CG;
    if (KCc > 16) return false;
    a.JC = lane_groups(CG);
    a.KSc = kslices(CG, a.JC);
    a.NGc = std::max(1, kMoeConsumerWarps / a.KSc);  // warp groups in phase C
    const int CW = std::max(a.KSb * a.NGb, a.KSc * a.NGc);
    a.CW = CW;

    const int slots = std::max(1, p->k + p->S);
    const int G = sm_count;
    const size_t rb_b = (size_t)H / 2 + (size_t)H / 8;  // bytes per row, one matrix
    const size_t rb_c = (size_t)CG * 32 / 2 + (size_t)CG * 32 / 8;  // one chunk row
    // gate+up tiles: the slots' tiles are dealt out over the CTAs; at most 8
    // dots per lane and tile (rows * 2 matrices * groups per lane)
    a.ROWSb = choose_rows(I, slots, true, G, 2 * rb_b, a.NGb, 4 / a.JB, 48 * 1024);
    // down tiles: the slots' tiles are dealt out over the CTAs as well
    a.ROWSc = choose_rows(H, slots * KCc, true, G, rb_c, a.NGc, 8 / a.JC, 48 * 1024);
    const int TRb = a.NGb * a.ROWSb, TRc = a.NGc * a.ROWSc;
    const int KSb = a.KSb, KSc = a.KSc;
    a.tb = make_tiling(I, H, TRb);
    a.tb.tile_bytes *= 2;  // a GU tile holds gate and up rows
    a.tb.tile_stride = (uint32_t)align_up(a.tb.tile_bytes, 128);
    a.tc = make_tiling(H, I, TRc, KCc);
    const size_t slot = std::max(a.tb.tile_stride, a.tc.tile_stride);
    a.slot_bytes = (uint32_t)slot;
    // one partial region holds one unit's per-(row, k-slice) sums
    a.part_floats = std::max(TRb * 2 * KSb, TRc * KSc);
    const size_t head = fused_head_bytes(H, p->E);
    // partial regions, then two staging buffers for chunks of mid (padded)
    const size_t tail = align_up((size_t)kPartRing * a.part_floats * 4, 16) +
                        align_up((size_t)2 * (CG * 33) * 4, 16);
    // ring barriers (16 per stage), one sink word per warp (128), the two
    // staging barriers (16), the partial-region barriers (16 per region),
    // the mid staging barriers (32)
    const size_t bars = 128 + 16 + 16 * (size_t)kPartRing + 32;
    long long ns =
        ((long long)kMaxDynSmem - (long long)(head + tail + bars) - 16 * 24) / (long long)slot;
    if (ns > 24) ns = 24;
    if (ns < 2) return false;
    a.nslots = (int)ns;
    p->smem = head + (size_t)ns * slot + tail + 16 * (size_t)ns + bars;
    // Until routing is done the ring is idle and stages h and the norm
    // weights (8 H bytes); routers up to 256 KB that fit in front of them are
    // staged too and scored by every CTA; larger ones are split over the CTAs,
    // which publish the scores as tagged values.
    const size_t ring = (size_t)ns * slot, router_bytes = (size_t)p->E * H * 4;
    if ((size_t)8 * H > ring) return false;
    a.route_local =
        router_bytes <= 256 * 1024 && align_up(router_bytes, 128) + (size_t)8 * H <= ring ? 1 : 0;
    // split routing: a CTA scores ceil(E / grid) rows at most (one when E <
    // grid); they are staged with h before the wait for the kernel before
    const size_t own_rows = p->E < G ? 1 : (size_t)(p->E + G - 1) / G;
    a.route_stage =
        !a.route_local && align_up(own_rows * H * 4, 128) + (size_t)8 * H <= ring ? 1 : 0;
    if (p->smem > (size_t)kMaxDynSmem) return false;
    p->block = (CW + 3) * 32;  // consumers, producer, epilogue, scout
    if (G > kMaxGrid) return false;
    p->grid = G;
    a.withhold_row = -1;
    p->off_d = align_up((size_t)a.tb.ntiles * a.tb.tile_stride, 256);
    p->rec_stride = p->off_d + align_up((size_t)a.tc.ntiles * a.tc.tile_stride, 256);
    return true;
}

static void free_pool(rabbit_cuda_moe *p) {
    if (p->device >= 0) cudaSetDevice(p->device);
    if (p->up) cudaStreamSynchronize(p->up);
    void *bufs[] = {p->pool,  p->rms,  p->router, p->scores,  p->mid, p->xn,  p->down,
                    p->h_in,  p->dio,   p->route,   p->flags};
    for (void *b : bufs)
        if (b) cudaFree(b);
    for (int i = 0; i < 2; ++i) {
        if (p->pin[i]) cudaFreeHost(p->pin[i]);
        if (p->pin_ev[i]) cudaEventDestroy(p->pin_ev[i]);
    }
    if (p->pin_io) cudaFreeHost(p->pin_io);
    for (cudaEvent_t ev : p->block_ev)
        if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : p->block_up_ev)
        if (ev) cudaEventDestroy(ev);
    for (int i = 0; i < kIoSlots; ++i) {
        if (p->io_raw[i]) cudaFreeHost(p->io_raw[i]);
        if (p->io_raw_ev[i]) cudaEventDestroy(p->io_raw_ev[i]);
    }
    for (int i = 0; i < 2; ++i) {
        if (p->io_img[i]) cudaFreeHost(p->io_img[i]);
        if (p->io_img_ev[i]) cudaEventDestroy(p->io_img_ev[i]);
    }
    if (p->bt_block) cudaFree(p->bt_block);
    if (p->bt_pin) cudaFreeHost(p->bt_pin);
    if (p->ep_block) cudaFree(p->ep_block);
    if (p->up) cudaStreamDestroy(p->up);
    delete p;
}

// Copy `n` host bytes to device memory through the two pinned staging
// buffers on the side stream (the host fills one while the other is in flight).
static int stage_h2d(rabbit_cuda_moe *p, uint8_t *dst, const uint8_t *src, uint64_t n) {
    for (uint64_t done = 0; done < n;) {
        const uint64_t m = std::min<uint64_t>(p->pin_cap, n - done);
        const int b = p->pin_next;
        p->pin_next ^= 1;
        RB_CUDA(cudaEventSynchronize(p->pin_ev[b]));  // buffer b free again
        memcpy(p->pin[b], src + done, m);
        RB_CUDA(cudaMemcpyAsync(dst + done, p->pin[b], m, cudaMemcpyHostToDevice, p->up));
        RB_CUDA(cudaEventRecord(p->pin_ev[b], p->up));
        p->h2d_bytes += m;
        done += m;
    }
    return RABBIT_CUDA_OK;
}

static void fill_trailer(const rabbit_cuda_moe *p, uint8_t *rec) {
    TileTrailer t = {};
    memcpy(t.magic, kTileMagic, 8);
    t.trb = (uint32_t)p->plan.tb.TR;
    t.trc = (uint32_t)p->plan.tc.TR;
    t.kc = (uint32_t)p->plan.tc.KC;
    t.h = (uint32_t)p->H;
    t.inter = (uint32_t)p->I;
    t.rec_stride = p->rec_stride;
    memset(rec + p->rec_stride, 0, kTileTrailer);
    memcpy(rec + p->rec_stride, &t, sizeof(t));
}

// A pre-tiled record's trailer must name this pool's tile plan.
static int check_trailer(const rabbit_cuda_moe *p, const uint8_t *rec, int gid) {
    TileTrailer t;
    memcpy(&t, rec + p->rec_stride, sizeof(t));
    if (memcmp(t.magic, kTileMagic, 8) != 0 || t.trb != (uint32_t)p->plan.tb.TR ||
        t.trc != (uint32_t)p->plan.tc.TR || t.kc != (uint32_t)p->plan.tc.KC ||
        t.h != (uint32_t)p->H || t.inter != (uint32_t)p->I || t.rec_stride != p->rec_stride)
        return fail(RABBIT_CUDA_ERR_FORMAT,
                    "moe_upload: record %d was not tiled for this pool's plan (tiles of %u / %u "
                    "rows, %u chunks here)", gid, (unsigned)p->plan.tb.TR, (unsigned)p->plan.tc.TR,
                    (unsigned)p->plan.tc.KC);
    return RABBIT_CUDA_OK;
}

// Record gid of the host map into pool record `pos`.
static int upload_record(rabbit_cuda_moe *p, int gid, int pos) {
    const uint8_t *src = p->host_map + (uint64_t)gid * p->expert_size;
    uint8_t *dst = p->pool + (uint64_t)pos * p->rec_stride;
    int st;
    if (p->pretiled) {
        if ((st = check_trailer(p, src, gid)) != RABBIT_CUDA_OK) return st;
        st = stage_h2d(p, dst, src, p->rec_stride);
    } else if (p->fast) {
        // gate / up / down blobs -> [GU tiles][D tiles] in a host image
        const uint64_t nb = nbytes_g32((uint64_t)p->H * p->I);
        p->img.resize(p->rec_stride);
        Tiling t2 = p->plan.tb;
        tile_pair_host(src, src + nb, t2, p->img.data());
        tile_blob_host(src + 2 * nb, p->plan.tc, p->img.data() + p->off_d);
        st = stage_h2d(p, dst, p->img.data(), p->rec_stride);
    } else {
        st = stage_h2d(p, dst, src, p->expert_size);
    }
    if (st != RABBIT_CUDA_OK) return st;
    p->resident[pos] = 1;
    p->uploads++;
    return RABBIT_CUDA_OK;
}

// splitmix64: a stateless hash of (seed, index) for device-side random init.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform random bytes (two uniform nibbles each) over [dst, dst + n).
__global__ void k_fill_bytes(uint8_t *dst, uint64_t n, uint64_t seed) {
    const uint64_t n8 = n / 8;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8;
         i += (uint64_t)gridDim.x * blockDim.x)
        reinterpret_cast<uint64_t *>(dst)[i] = mix64(seed ^ (i * 0xD1B54A32D192ED03ull));
}

// |N(0, sigma)| / 7 per scale (Box-Muller on two hashed uniforms); the scales
// of tile t are n_per_tile floats at base + t*stride + off.
__global__ void k_fill_scales(uint8_t *base, int ntiles, uint32_t stride, uint32_t off,
                              uint32_t n_per_tile, uint64_t seed, float sigma) {
    const uint64_t n = (uint64_t)ntiles * n_per_tile;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        float *dst = reinterpret_cast<float *>(base + (i / n_per_tile) * stride + off) +
                     i % n_per_tile;
        const uint64_t h = mix64(seed ^ (i * 0xA24BAED4963EE407ull));
        const float u1 = ((uint32_t)(h >> 40) + 1) * (1.0f / 16777217.0f);
        const float u2 = (uint32_t)(h & 0xFFFFFF) * (1.0f / 16777216.0f);
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        *dst = fabsf(z) * sigma / 7.0f;
    }
}

}  // namespace rb

namespace rb {
void moe_shape(const rabbit_cuda_moe *p, int *device, int *n_layers, int *hidden) {
    *device = p->device;
    *n_layers = p->L;
    *hidden = p->H;
}
}  // namespace rb

using namespace rb;

extern "C" {

}  // extern "C"

static int create_pool(const rabbit_cuda_moe_desc *d, int device, int window, rabbit_cuda_moe **out) {
    if (!d || !out) return fail(RABBIT_CUDA_ERR_ARGS, "moe_create: NULL argument");
    *out = nullptr;
    if (d->n_layers <= 0 || d->hidden <= 0 || d->n_experts <= 0 || d->inter <= 0 ||
        d->expert_size == 0 || d->n_records <= 0 || !d->rms_ffn || !d->w_router)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_create: incomplete model description");
    for (int l = 0; l < d->n_layers; ++l)
        if (!d->rms_ffn[l] || !d->w_router[l])
            return fail(RABBIT_CUDA_ERR_ARGS, "moe_create: layer %d has no norm/router", l);
    int st;
    DevCtx *c = dev_ctx(device, &st);
    if (!c) return st;

    rabbit_cuda_moe *p = new rabbit_cuda_moe();
    p->device = device;
    p->ctx = c;
    p->L = d->n_layers;
    p->H = d->hidden;
    p->E = d->n_experts;
    p->I = d->inter;
    int k = d->experts_per_token > 0 ? d->experts_per_token : 2;  // forward_v2.c:113
    k = std::min(k, p->E);
    k = std::min(k, 8);  // forward_v2.c:366-367
    p->k = k;
    p->S = (d->n_shared > 0 && d->n_shared <= 64) ? d->n_shared : 0;  // forward_v2.c:392
    p->quant = d->expert_quant;
    if (p->quant == RABBIT_CUDA_QUANT_INT4_TILED) {  // group-32 int4, already tiled
        p->pretiled = true;
        p->quant = 4;
    }
    p->expert_size = d->expert_size;
    p->n_records = d->n_records;
    p->epl = d->experts_per_layer > 0 ? d->experts_per_layer : d->n_experts;
    p->shared_table = d->experts_shared ? 1 : 0;
    p->host_map = static_cast<const uint8_t *>(d->expert_map);
    if (window > 0 && window < p->L) {
        if (p->shared_table) {
            delete p;
            return fail(RABBIT_CUDA_ERR_ARGS,
                        "moe_create_window: a table shared by every layer has no per-layer blocks");
        }
        p->window = window;
    }

    const uint64_t mat = (uint64_t)p->H * p->I;
    uint64_t need;
    if (p->quant == 0)
        need = (2 * mat + mat) * 4;
    else if (p->quant == 4)
        need = 2 * nbytes_g32(mat) + nbytes_g32(mat);
    else
        need = 3 * (4 + mat);
    p->usable = p->expert_size >= need;  // forward_v2.c:299,319,335: else experts add nothing
    if (p->pretiled) p->usable = true;  // checked against the plan below

    // Fast layout only when every blob carries group 32.
    p->fast = p->quant == 4 && p->usable && mat <= 0x7fffffffull;
    if (p->fast && p->host_map && !p->pretiled) {
        const uint64_t nb = nbytes_g32(mat);
        for (int r = 0; r < p->n_records && p->fast; ++r) {
            const uint8_t *rec = p->host_map + (uint64_t)r * p->expert_size;
            for (int m = 0; m < 3; ++m) {
                uint32_t gs;
                memcpy(&gs, rec + m * nb, 4);
                if (gs != 32) {
                    p->fast = false;
                    break;
                }
            }
        }
    }
    if (p->fast && !plan_fused(p, c->sm_count)) p->fast = false;
    if (p->pretiled && (!p->fast || p->expert_size != p->rec_stride + kTileTrailer)) {
        const unsigned long long want = p->fast ? p->rec_stride + kTileTrailer : 0;
        delete p;
        return fail(RABBIT_CUDA_ERR_FORMAT,
                    "moe_create: pre-tiled records of %llu bytes do not match this device's tile "
                    "plan (%llu bytes)", (unsigned long long)d->expert_size, want);
    }

    cudaError_t e = cudaSuccess;
    if (!p->fast) p->rec_stride = align_up(p->expert_size, 256);  // verbatim records
    p->pool_records = p->window ? p->window * p->epl : p->n_records;
    p->pool_bytes = p->rec_stride * (uint64_t)p->pool_records;
    p->resident.assign(p->pool_records, 0);
    if (p->window) {
        p->layer_block.assign(p->L, -1);
        p->block_layer.assign(p->window, -1);
        p->block_use.assign(p->window, 0);
        p->block_ev.assign(p->window, nullptr);
        p->block_up_ev.assign(p->window, nullptr);
        for (int b = 0; b < p->window; ++b)
            if ((e = cudaEventCreateWithFlags(&p->block_ev[b], cudaEventDisableTiming)) != cudaSuccess ||
                (e = cudaEventCreateWithFlags(&p->block_up_ev[b], cudaEventDisableTiming)) != cudaSuccess) {
                free_pool(p);
                return cuda_fail(e, "moe_create: window events");
            }
    }

    const size_t HE = (size_t)p->H * p->E;
    if ((e = cudaMalloc(&p->pool, p->pool_bytes)) != cudaSuccess) {
        free_pool(p);
        return fail(RABBIT_CUDA_ERR_MEM, "moe_create: cannot allocate %.2f GB expert pool: %s",
                    p->pool_bytes / 1e9, cudaGetErrorString(e));
    }
    if ((e = cudaMalloc(&p->rms, sizeof(float) * (size_t)p->H * p->L)) != cudaSuccess ||
        (e = cudaMalloc(&p->router, sizeof(float) * HE * p->L)) != cudaSuccess ||
        (e = cudaMalloc(&p->scores, sizeof(unsigned long long) * p->E)) != cudaSuccess ||
        (e = cudaMalloc(&p->mid, mid_bytes(p))) != cudaSuccess ||
        (e = cudaMemset(p->mid, 0, mid_bytes(p))) != cudaSuccess ||
        (e = cudaMalloc(&p->xn, sizeof(float) * p->H)) != cudaSuccess ||
        (e = cudaMalloc(&p->down, down_bytes(p))) != cudaSuccess ||
        (e = cudaMemset(p->down, 0, down_bytes(p))) != cudaSuccess ||
        (e = cudaMalloc(&p->flags, sizeof(unsigned) * kMaxGrid)) != cudaSuccess ||
        (e = cudaMemset(p->flags, 0, sizeof(unsigned) * kMaxGrid)) != cudaSuccess ||
        (e = cudaMalloc(&p->h_in, sizeof(float) * p->H)) != cudaSuccess ||
        (e = cudaMalloc(&p->dio, p->dio_bytes = sizeof(float) * (size_t)p->H + 80)) !=
            cudaSuccess ||
        (e = cudaMemset(p->dio, 0, p->dio_bytes)) != cudaSuccess ||
        (e = cudaMalloc(&p->route, sizeof(Route))) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&p->up, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMallocHost(&p->pin_io, sizeof(float) * (2 * (size_t)p->H + 32))) !=
            cudaSuccess ||
        (e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&p->pin_io_dev), p->pin_io, 0)) !=
            cudaSuccess) {
        free_pool(p);
        return cuda_fail(e, "moe_create: scratch");
    }
    if (p->fast) {
        const int tm = tc_tensor_maps(p->pool, p->pool_bytes, p->rec_stride, p->off_d, p->plan.tb,
                                      p->plan.tc, p->H, &p->tm_gu, &p->tm_dn);
        if (tm == 2) {
            free_pool(p);
            return fail(RABBIT_CUDA_ERR_DEVICE,
                        "moe_create: the driver could not encode the expert pool's tensor maps");
        }
        p->tc_ok = tm == 0;
    }
    p->h_out = reinterpret_cast<float *>(p->dio);
    p->ids_int = reinterpret_cast<int *>(p->dio + sizeof(float) * (size_t)p->H);
    p->w_int = reinterpret_cast<float *>(p->ids_int + 8);
    p->err_io = reinterpret_cast<int *>(p->w_int + 8);
    // staging holds up to one record image (verbatim or tiled, whichever is larger)
    const uint64_t pin_bytes =
        std::min<uint64_t>(kPinChunk, align_up(std::max<uint64_t>(p->expert_size, p->rec_stride), 4096));
    p->pin_cap = pin_bytes;
    for (int i = 0; i < 2; ++i) {
        if ((e = cudaMallocHost(&p->pin[i], pin_bytes)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&p->pin_ev[i], cudaEventDisableTiming)) !=
                cudaSuccess ||
            (e = cudaEventRecord(p->pin_ev[i], p->up)) != cudaSuccess) {
            free_pool(p);
            return cuda_fail(e, "moe_create: pinned staging");
        }
    }
    for (int l = 0; l < p->L; ++l) {
        if ((e = cudaMemcpy(p->rms + (size_t)l * p->H, d->rms_ffn[l], sizeof(float) * p->H,
                            cudaMemcpyHostToDevice)) != cudaSuccess ||
            (e = cudaMemcpy(p->router + HE * l, d->w_router[l], sizeof(float) * HE,
                            cudaMemcpyHostToDevice)) != cudaSuccess) {
            free_pool(p);
            return cuda_fail(e, "moe_create: router/norm upload");
        }
    }
    if (p->fast && !g_moe_attr[device]) {
        for (const void *k :
             {moe_fused_kernel(1, 1, false), moe_fused_kernel(1, 2, false),
              moe_fused_kernel(2, 1, false), moe_fused_kernel(2, 2, false),
              moe_fused_kernel(1, 1, true), moe_fused_kernel(1, 2, true),
              moe_fused_kernel(2, 1, true), moe_fused_kernel(2, 2, true)})
            if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kMaxDynSmem)) != cudaSuccess) {
                free_pool(p);
                return cuda_fail(e, "moe_create: smem attribute");
            }
        g_moe_attr[device] = true;
    }
    if (p->fast) {
        int per_sm = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                 &per_sm, moe_fused_kernel(p->plan.JB, p->plan.JC, combine_packed(p->plan.tc.KC)),
                 p->block, p->smem)) !=
                cudaSuccess ||
            per_sm < 1) {
            free_pool(p);
            return fail(RABBIT_CUDA_ERR_UNSUPPORTED, "moe_create: fused kernel does not fit an SM");
        }
    }
    *out = p;
    return ok();
}

extern "C" {

int rabbit_cuda_moe_create(const rabbit_cuda_moe_desc *d, int device, rabbit_cuda_moe **out) {
    return create_pool(d, device, 0, out);
}

int rabbit_cuda_moe_create_window(const rabbit_cuda_moe_desc *d, int device, int window_layers,
                                  rabbit_cuda_moe **out) {
    if (window_layers < 1) return fail(RABBIT_CUDA_ERR_ARGS, "moe_create_window: window of %d layers", window_layers);
    return create_pool(d, device, window_layers, out);
}

int rabbit_cuda_moe_upload(rabbit_cuda_moe *p, int layer_begin, int layer_end) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload: NULL pool");
    if (layer_begin < 0 || layer_end > p->L || layer_begin >= layer_end)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload: bad layer range [%d, %d)", layer_begin,
                    layer_end);
    if (!p->host_map)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload: pool was created without a host map");
    if (p->window && layer_end - layer_begin > p->window)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload: %d layers exceed the pool's window of %d",
                    layer_end - layer_begin, p->window);
    RB_CUDA(cudaSetDevice(p->device));
    for (int l = layer_begin; l < layer_end; ++l) {
        int base, n, src;
        int st = layer_slot(p, l, &base, &n, &src);
        if (st) return st;
        for (int r = 0; r < n; ++r)
            if (!p->resident[base + r] && (st = upload_record(p, src + r, base + r)) != RABBIT_CUDA_OK)
                return st;
        if (p->window) RB_CUDA(cudaEventRecord(p->block_up_ev[p->layer_block[l]], p->up));
    }
    return ok();
}

}  // extern "C"

namespace rb {

// Pinned buffers of the file reader, allocated on first use and kept with
// the pool: kIoSlots record buffers (a record plus O_DIRECT alignment slack)
// and, for group-32 pools, two tiled images.
static int ensure_io(rabbit_cuda_moe *p) {
    const uint64_t cap = align_up(p->expert_size, kIoAlign) + 2 * kIoAlign;
    cudaError_t e;
    if (p->io_raw_cap < cap) {
        for (int i = 0; i < kIoSlots; ++i) {
            if (p->io_raw_ev[i]) RB_CUDA(cudaEventSynchronize(p->io_raw_ev[i]));
            if (p->io_raw[i]) cudaFreeHost(p->io_raw[i]);
            p->io_raw[i] = nullptr;
        }
        p->io_raw_cap = 0;
        for (int i = 0; i < kIoSlots; ++i)
            if ((e = cudaMallocHost(&p->io_raw[i], cap)) != cudaSuccess)
                return cuda_fail(e, "moe_upload_file: pinned record buffers");
        p->io_raw_cap = cap;
    }
    for (int i = 0; i < kIoSlots; ++i)
        if (!p->io_raw_ev[i]) {
            if ((e = cudaEventCreateWithFlags(&p->io_raw_ev[i], cudaEventDisableTiming)) != cudaSuccess ||
                (e = cudaEventRecord(p->io_raw_ev[i], p->up)) != cudaSuccess)
                return cuda_fail(e, "moe_upload_file: events");
        }
    if (p->fast && !p->pretiled)
        for (int i = 0; i < 2; ++i)
            if (!p->io_img[i]) {
                if ((e = cudaMallocHost(&p->io_img[i], p->rec_stride)) != cudaSuccess ||
                    (e = cudaEventCreateWithFlags(&p->io_img_ev[i], cudaEventDisableTiming)) != cudaSuccess ||
                    (e = cudaEventRecord(p->io_img_ev[i], p->up)) != cudaSuccess)
                    return cuda_fail(e, "moe_upload_file: pinned images");
            }
    return RABBIT_CUDA_OK;
}

// Read [off, off + n) of fd into buf. With O_DIRECT the read starts at the
// aligned offset below off and covers whole blocks (the file's end may cut
// the last one short); *data is where byte `off` landed. False on an I/O
// error or a file that ends before off + n.
static bool read_record(int fd, bool direct, uint64_t off, uint64_t n, uint8_t *buf, uint8_t **data,
                        int *err) {
    const uint64_t a0 = direct ? off / kIoAlign * kIoAlign : off;
    const uint64_t len = direct ? align_up(off + n, kIoAlign) - a0 : n;
    const uint64_t need = off + n - a0;
    uint64_t got = 0;
    while (got < len) {
        const ssize_t r = pread(fd, buf + got, (size_t)(len - got), (off_t)(a0 + got));
        if (r < 0) {
            if (errno == EINTR) continue;
            *err = errno;
            return false;
        }
        if (r == 0) break;  // end of file
        got += (uint64_t)r;
        if (direct && got % kIoAlign != 0) break;  // a short direct read ends at the file's end
    }
    *data = buf + (off - a0);
    if (got < need) *err = 0;
    return got >= need;
}

// The body of rabbit_cuda_moe_upload_file: the records of `gids`, read by a
// reader thread into the pinned ring while this thread lays them out and
// queues their copies.
static int upload_from_file(rabbit_cuda_moe *p, const char *path, uint64_t expert_offset,
                            const std::vector<int> &gids, const std::vector<int> &dsts) {
    int st = ensure_io(p);
    if (st) return st;
    int fd = open(path, O_RDONLY | O_DIRECT);
    bool direct = fd >= 0;
    if (fd < 0) fd = open(path, O_RDONLY);
    if (fd < 0) return fail(RABBIT_CUDA_ERR_IO, "moe_upload_file: cannot open %s (%s)", path, strerror(errno));

    const int n = (int)gids.size();
    std::mutex mu;
    std::condition_variable cv;
    int produced = 0, consumed = 0, io_err = -1, bad = -1;  // bad: first record that failed
    bool stop = false;
    uint8_t *data[kIoSlots] = {};
    const int device = p->device;
    std::thread reader([&] {
        cudaSetDevice(device);
        for (int i = 0; i < n; ++i) {
            const int s = i % kIoSlots;
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return stop || i - consumed < kIoSlots; });
                if (stop) return;
            }
            cudaEventSynchronize(p->io_raw_ev[s]);  // the last copy out of this buffer is done
            const uint64_t off = expert_offset + (uint64_t)gids[i] * p->expert_size;
            int err = 0;
            uint8_t *d = nullptr;
            bool ok = read_record(fd, direct, off, p->expert_size, p->io_raw[s], &d, &err);
            if (!ok && direct && err == EINVAL) {  // this file system refuses O_DIRECT reads
                direct = false;
                ok = read_record(fd, false, off, p->expert_size, p->io_raw[s], &d, &err);
            }
            std::lock_guard<std::mutex> lk(mu);
            if (!ok) {
                io_err = err;
                bad = i;
                cv.notify_all();
                return;
            }
            data[s] = d;
            produced = i + 1;
            cv.notify_all();
        }
    });
    const uint64_t nb = nbytes_g32((uint64_t)p->H * p->I);
    for (int i = 0; i < n && st == RABBIT_CUDA_OK; ++i) {
        const int s = i % kIoSlots, gid = gids[i], pos = dsts[i];
        uint8_t *rec;
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return produced > i || bad >= 0; });
            if (produced <= i) {
                st = io_err > 0 ? fail(RABBIT_CUDA_ERR_IO, "moe_upload_file: reading record %d of %s: %s",
                                       gid, path, strerror(io_err))
                                : fail(RABBIT_CUDA_ERR_IO,
                                       "moe_upload_file: %s ends inside record %d (offset %llu)", path,
                                       gid, (unsigned long long)(expert_offset + (uint64_t)gid * p->expert_size));
                break;
            }
            rec = data[s];
        }
        uint8_t *dst = p->pool + (uint64_t)pos * p->rec_stride;
        cudaError_t e = cudaSuccess;
        if (p->pretiled && (st = check_trailer(p, rec, gid)) != RABBIT_CUDA_OK) break;
        if (p->fast && !p->pretiled) {
            for (int m = 0; m < 3 && st == RABBIT_CUDA_OK; ++m) {
                uint32_t gs;
                memcpy(&gs, rec + m * nb, 4);
                if (gs != 32)
                    st = fail(RABBIT_CUDA_ERR_FORMAT,
                              "moe_upload_file: record %d blob %d has group size %u; the pool was "
                              "planned for group-32 records", gid, m, gs);
            }
            if (st) break;
            const int b = i & 1;
            if ((e = cudaEventSynchronize(p->io_img_ev[b])) != cudaSuccess) {
                st = cuda_fail(e, "moe_upload_file");
                break;
            }
            tile_pair_host(rec, rec + nb, p->plan.tb, p->io_img[b]);
            tile_blob_host(rec + 2 * nb, p->plan.tc, p->io_img[b] + p->off_d);
            if ((e = cudaMemcpyAsync(dst, p->io_img[b], p->rec_stride, cudaMemcpyHostToDevice, p->up)) !=
                    cudaSuccess ||
                (e = cudaEventRecord(p->io_img_ev[b], p->up)) != cudaSuccess) {
                st = cuda_fail(e, "moe_upload_file");
                break;
            }
            p->h2d_bytes += p->rec_stride;
        } else {  // verbatim (or pre-tiled) records: copied straight from the record buffer
            const uint64_t bytes = p->pretiled ? p->rec_stride : p->expert_size;
            if ((e = cudaMemcpyAsync(dst, rec, bytes, cudaMemcpyHostToDevice, p->up)) != cudaSuccess ||
                (e = cudaEventRecord(p->io_raw_ev[s], p->up)) != cudaSuccess) {
                st = cuda_fail(e, "moe_upload_file");
                break;
            }
            p->h2d_bytes += bytes;
        }
        p->resident[pos] = 1;
        p->uploads++;
        std::lock_guard<std::mutex> lk(mu);
        consumed = i + 1;  // the record buffer may be refilled (after its copy, for verbatim pools)
        cv.notify_all();
    }
    {
        std::lock_guard<std::mutex> lk(mu);
        stop = true;
        cv.notify_all();
    }
    reader.join();
    close(fd);
    return st;
}

}  // namespace rb

extern "C" {

int rabbit_cuda_moe_upload_file(rabbit_cuda_moe *p, const char *path, uint64_t expert_offset,
                                int layer_begin, int layer_end) {
    if (!p || !path) return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload_file: NULL argument");
    if (layer_begin < 0 || layer_end > p->L || layer_begin >= layer_end)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload_file: bad layer range [%d, %d)", layer_begin,
                    layer_end);
    if (p->window && layer_end - layer_begin > p->window)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_upload_file: %d layers exceed the pool's window of %d",
                    layer_end - layer_begin, p->window);
    RB_CUDA(cudaSetDevice(p->device));
    std::vector<int> gids, dsts;  // model record -> pool record
    for (int l = layer_begin; l < layer_end; ++l) {
        int base, n, src;
        const int st = layer_slot(p, l, &base, &n, &src);
        if (st) return st;
        for (int r = 0; r < n; ++r)
            if (!p->resident[base + r] &&
                std::find(dsts.begin(), dsts.end(), base + r) == dsts.end()) {
                gids.push_back(src + r);
                dsts.push_back(base + r);
            }
    }
    int st = gids.empty() ? RABBIT_CUDA_OK : rb::upload_from_file(p, path, expert_offset, gids, dsts);
    if (p->window)
        for (int l = layer_begin; l < layer_end; ++l)
            if (p->layer_block[l] >= 0) RB_CUDA(cudaEventRecord(p->block_up_ev[p->layer_block[l]], p->up));
    return st == RABBIT_CUDA_OK ? ok() : st;
}

int rabbit_cuda_moe_sync(rabbit_cuda_moe *p) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_sync: NULL pool");
    RB_CUDA(cudaSetDevice(p->device));
    RB_CUDA(cudaStreamSynchronize(p->up));
    return ok();
}

int rabbit_cuda_moe_fill_synthetic(rabbit_cuda_moe *p, uint64_t seed, float scale_sigma) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_fill_synthetic: NULL pool");
    if (!p->fast)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_fill_synthetic: pool is not in the group-32 layout");
    if (p->window)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED, "moe_fill_synthetic: windowed pools load layers on demand");
    RB_CUDA(cudaSetDevice(p->device));
    const int blocks = p->ctx->sm_count * 8;
    const Tiling &tb = p->plan.tb, &tc = p->plan.tc;
    for (int r = 0; r < p->n_records; ++r) {
        uint8_t *rec = p->pool + (uint64_t)r * p->rec_stride;
        const uint64_t s0 = mix_host(seed, (uint64_t)r);
        // nibbles everywhere (uniform bytes), then the scale blocks of each tile
        k_fill_bytes<<<blocks, 256, 0, p->up>>>(rec, p->rec_stride, s0);
        k_fill_scales<<<blocks, 256, 0, p->up>>>(rec, tb.ntiles, tb.tile_stride,
                                                 (uint32_t)(2 * (size_t)tb.TR * (p->H / 2)),
                                                 2 * tb.TR * (p->H / 32), s0 + 1, scale_sigma);
        k_fill_scales<<<blocks, 256, 0, p->up>>>(rec + p->off_d, tc.ntiles, tc.tile_stride,
                                                 (uint32_t)((size_t)tc.TR * (tc.cols / 2)),
                                                 tc.TR * (tc.cols / 32), s0 + 2, scale_sigma);
        p->resident[r] = 1;
    }
    RB_CUDA(cudaGetLastError());
    RB_CUDA(cudaStreamSynchronize(p->up));
    return ok();
}

int rabbit_cuda_moe_free(rabbit_cuda_moe *p) {
    if (p) free_pool(p);
    return ok();
}

}  // extern "C"

namespace rb {
// The body of rabbit_cuda_moe_decode_dev; `err` is the device word the fused
// kernel records a failed wait in.
static int decode_launch(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out,
                         int *d_ids, float *d_weights, cudaStream_t s, int *err);
// Host-buffer decode helpers: h from pinned host memory into HBM (one CTA,
// float4 over PCIe), and the device error word into the pinned block (then
// cleared for the next call).
__global__ void __launch_bounds__(256) k_h_in(const float *src, float *dst, int n) {
    const int n4 = n >> 2;  // both 16-byte aligned: a page of pinned memory, cudaMalloc
    for (int i = threadIdx.x; i < n4; i += blockDim.x)
        reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(src)[i];
    for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}
__global__ void k_err_out(int *d_err, int *h_err) {
    if (threadIdx.x == 0) {
        const int e = *reinterpret_cast<volatile int *>(d_err);
        *reinterpret_cast<volatile int *>(h_err) = e;
        if (e) *d_err = 0;
    }
}

static int decode_impl(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out,
                       int *d_ids, float *d_weights, cudaStream_t s, int *err) {
    int st = window_enter(p, layer, s);
    if (st == RABBIT_CUDA_OK) st = decode_launch(p, layer, d_h_in, d_h_out, d_ids, d_weights, s, err);
    const int st2 = window_leave(p, layer, s);
    return st ? st : st2;
}
static int decode_launch(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out,
                         int *d_ids, float *d_weights, cudaStream_t s, int *err) {
    if (p->ep_size > 1)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_decode: expert-parallel pools run the multi-token path");
    int base, n_local;
    int st = layer_map(p, layer, &base, &n_local);
    if (st) return st;
    for (int r = 0; r < n_local; ++r)
        if (!p->resident[base + r])
        {
            p->misses++;
            return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode: layer %d not uploaded", layer);
        }
    RB_CUDA(cudaSetDevice(p->device));
    int *ids = d_ids ? d_ids : p->ids_int;
    float *w = d_weights ? d_weights : p->w_int;
    const float *rms = p->rms + (size_t)layer * p->H;
    const float *router = p->router + (size_t)layer * p->H * p->E;
    if (p->fast) {
        if ((reinterpret_cast<uintptr_t>(d_h_in) & 15) || (reinterpret_cast<uintptr_t>(d_h_out) & 15))
            return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode: h must be 16-byte aligned");
        MoeFusedArgs a = p->plan;
        a.h_in = d_h_in;
        a.h_out = d_h_out;
        a.ids_out = ids;
        a.w_out = w;
        a.rms = rms;
        a.router = router;
        a.pool = p->pool;
        a.rec_stride = p->rec_stride;
        a.off_d = p->off_d;
        a.rec_base = base;
        a.n_local = n_local;
        a.H = p->H;
        a.E = p->E;
        a.k = p->k;
        a.I = p->I;
        a.S = p->S;
        a.usable = p->usable ? 1 : 0;
        a.scores = reinterpret_cast<unsigned long long *>(p->scores);
        a.mid = reinterpret_cast<unsigned long long *>(p->mid);
        a.down = reinterpret_cast<unsigned long long *>(p->down);
        a.flags = p->flags;
        a.err = err;
        {
            void *tagged[] = {p->mid, p->down, p->flags, p->scores};
            const size_t bytes[] = {mid_bytes(p), down_bytes(p), sizeof(unsigned) * kMaxGrid,
                                    sizeof(unsigned long long) * p->E};
            a.seq = next_seq(&p->seq, tagged, bytes, 4, s);
        }
        a.wait_ns = wait_limit_ns();
        a.withhold_row = p->withhold_row;
        p->withhold_row = -1;
        RB_CUDA(launch_fused(p, a, s));
    } else {
        MoeGenericArgs a;
        a.h_in = d_h_in;
        a.h_out = d_h_out;
        a.ids_out = ids;
        a.w_out = w;
        a.rms = rms;
        a.router = router;
        a.pool = p->pool;
        a.rec_stride = p->rec_stride;
        a.expert_size = p->expert_size;
        a.rec_base = base;
        a.n_local = n_local;
        a.H = p->H;
        a.E = p->E;
        a.k = p->k;
        a.I = p->I;
        a.S = p->S;
        a.quant = p->quant;
        a.usable = p->usable ? 1 : 0;
        a.xn = p->xn;
        a.scores = p->scores;
        a.mid = p->mid;
        a.down = p->down;
        a.route = p->route;
        const int slots = std::max(1, p->k + p->S);
        k_moe_route<<<1, 512, 0, s>>>(a);
        k_moe_up_generic<<<dim3((p->I + 7) / 8, slots), 256, 0, s>>>(a);
        k_moe_down_generic<<<dim3((p->H + 7) / 8, slots), 256, 0, s>>>(a);
        k_moe_combine<<<(p->H + 255) / 256, 256, 0, s>>>(a);
        RB_CUDA(cudaGetLastError());
    }
    p->hbm_hits++;
    return ok();
}
}  // namespace rb

extern "C" {

int rabbit_cuda_moe_decode_dev(rabbit_cuda_moe *p, int layer, const float *d_h_in,
                               float *d_h_out, int *d_ids, float *d_weights, void *stream) {
    if (!p || !d_h_in || !d_h_out) return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode: NULL argument");
    if (int st = refuse_capture(as_stream(stream, p->ctx), "moe_decode_dev")) return st;
    return decode_impl(p, layer, d_h_in, d_h_out, d_ids, d_weights, as_stream(stream, p->ctx),
                       p->ctx->d_err);
}

// ------------------------------------------------------- no-alloc decode --
// Scratch for rabbit_cuda_moe_decode_dev_noalloc, in a fixed array of this
// module instead of the pool: [0, 256) routed ids at 64 and weights at 128
// when the caller passes none; then the per-CTA flags; the router scores (E
// tagged values, 8 bytes each); mid ((k + S) x I tagged
// values, 8 bytes each); the down rows per column chunk of W2 ((k + S) x KC
// x H tagged values), each part 256-aligned. Every
// device that loads the library holds these bytes until the process exits.
constexpr size_t kNoAllocScratchBytes = 2u << 20;  // 2 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static unsigned g_noalloc_seq[kMaxDevices] = {};  // next launch tag per device (0: unset)
// g_noalloc_scratch names the array only on the host side; its device address
// on each device, looked up once per device with that device current.
static uint8_t *g_noalloc_ptr[kMaxDevices];
static std::mutex g_noalloc_mu;

static int noalloc_scratch(int device, uint8_t **out) {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void *ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "moe_decode_noalloc: scratch address");
        g_noalloc_ptr[device] = static_cast<uint8_t *>(ptr);
    }
    *out = g_noalloc_ptr[device];
    return RABBIT_CUDA_OK;
}

int rabbit_cuda_moe_decode_dev_noalloc(rabbit_cuda_moe *p, int layer, const float *d_h_in,
                                       float *d_h_out, int *d_ids, float *d_weights,
                                       void *stream) {
    if (!p || !d_h_in || !d_h_out)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode_noalloc: NULL argument");
    if (int st = refuse_capture(as_stream(stream, p->ctx), "moe_decode_noalloc")) return st;
    if (!p->fast)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_decode_noalloc: pool is not in the group-32 fused layout");
    if (p->ep_size > 1)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_decode_noalloc: expert-parallel pools run the multi-token path");
    if ((reinterpret_cast<uintptr_t>(d_h_in) & 15) || (reinterpret_cast<uintptr_t>(d_h_out) & 15))
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode_noalloc: h must be 16-byte aligned");
    const size_t off_flags = 256;
    const size_t off_scores = off_flags + align_up(sizeof(unsigned) * kMaxGrid, 256);
    const size_t off_mid = off_scores + align_up((size_t)p->E * 8, 256);
    const size_t off_down = off_mid + align_up(mid_bytes(p), 256);
    const size_t need = off_down + down_bytes(p);
    if (need > kNoAllocScratchBytes)
        return fail(RABBIT_CUDA_ERR_ARGS,
                    "moe_decode_noalloc: this model needs %zu bytes of scratch, more than the "
                    "%zu-byte limit",
                    need, kNoAllocScratchBytes);
    int base, n_local;
    int st = layer_map(p, layer, &base, &n_local);
    if (st) return st;
    for (int r = 0; r < n_local; ++r)
        if (!p->resident[base + r])
        {
            p->misses++;
            return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode_noalloc: layer %d not uploaded", layer);
        }
    RB_CUDA(cudaSetDevice(p->device));
    uint8_t *scratch = nullptr;
    if ((st = noalloc_scratch(p->device, &scratch)) != RABBIT_CUDA_OK) return st;
    cudaStream_t s = as_stream(stream, p->ctx);
    // Values shared between CTAs are tagged with the call's sequence number,
    // which is new on every call on this device: what an earlier call left in
    // the array is never read.
    MoeFusedArgs a = p->plan;
    a.h_in = d_h_in;
    a.h_out = d_h_out;
    a.ids_out = d_ids ? d_ids : reinterpret_cast<int *>(scratch + 64);
    a.w_out = d_weights ? d_weights : reinterpret_cast<float *>(scratch + 128);
    a.rms = p->rms + (size_t)layer * p->H;
    a.router = p->router + (size_t)layer * p->H * p->E;
    a.pool = p->pool;
    a.rec_stride = p->rec_stride;
    a.off_d = p->off_d;
    a.rec_base = base;
    a.n_local = n_local;
    a.H = p->H;
    a.E = p->E;
    a.k = p->k;
    a.I = p->I;
    a.S = p->S;
    a.usable = p->usable ? 1 : 0;
    a.scores = reinterpret_cast<unsigned long long *>(scratch + off_scores);
    a.mid = reinterpret_cast<unsigned long long *>(scratch + off_mid);
    a.down = reinterpret_cast<unsigned long long *>(scratch + off_down);
    a.flags = reinterpret_cast<unsigned *>(scratch + off_flags);
    {
        std::lock_guard<std::mutex> g(g_noalloc_mu);
        void *tagged[] = {scratch + off_flags};
        const size_t bytes[] = {kNoAllocScratchBytes - off_flags};
        a.seq = next_seq(&g_noalloc_seq[p->device], tagged, bytes, 1, s);
    }
    a.err = p->ctx->d_err;
    a.wait_ns = wait_limit_ns();
    if ((st = window_enter(p, layer, s)) != RABBIT_CUDA_OK) return st;
    RB_CUDA(launch_fused(p, a, s));
    if ((st = window_leave(p, layer, s)) != RABBIT_CUDA_OK) return st;
    p->hbm_hits++;
    return ok();
}

int rabbit_cuda_moe_debug_withhold_score(rabbit_cuda_moe *p, int expert) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_debug_withhold_score: NULL pool");
    if (!p->fast || p->plan.route_local)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_debug_withhold_score: this pool's fused decode scores every router row "
                    "in every CTA (no scores are published)");
    if (expert < 0 || expert >= p->E)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_debug_withhold_score: expert %d of %d", expert,
                    p->E);
    p->withhold_row = expert;
    return ok();
}

int rabbit_cuda_moe_check(rabbit_cuda_moe *p, void *stream) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_check: NULL pool");
    RB_CUDA(cudaSetDevice(p->device));
    cudaStream_t s = as_stream(stream, p->ctx);
    int st = check_device_error(p->ctx, s, "moe_decode");
    // after a wait that gave up, scratch needs no cleaning: everything the
    // CTAs share is tagged, and the next launch has a new tag
    return st != RABBIT_CUDA_OK ? st : ok();
}

int rabbit_cuda_moe_decode(rabbit_cuda_moe *p, int layer, const float *h_in, float *h_out,
                           int *ids, float *weights, int *k_out) {
    if (!p || !h_in || !h_out) return fail(RABBIT_CUDA_ERR_ARGS, "moe_decode: NULL argument");
    std::lock_guard<std::mutex> g(p->ctx->mu);
    RB_CUDA(cudaSetDevice(p->device));
    cudaStream_t s = p->ctx->stream;
    const size_t hb = sizeof(float) * p->H;
    // pinned, mapped: [h_in (H)] [h_out (H) | ids (8) | weights (8) | error word].
    // One small kernel brings h into HBM over PCIe, the decode writes h_out,
    // ids and weights straight into the pinned block, and a last one-thread
    // kernel moves the error word there (and clears it): no copy engine
    // transfers, one synchronisation.
    float *pin_h = p->pin_io;
    uint8_t *pin_o = reinterpret_cast<uint8_t *>(p->pin_io + p->H);
    uint8_t *dev_o = reinterpret_cast<uint8_t *>(p->pin_io_dev + p->H);
    int *dev_err = reinterpret_cast<int *>(dev_o + (p->dio_bytes - 16));
    memcpy(pin_h, h_in, hb);
    k_h_in<<<1, 256, 0, s>>>(p->pin_io_dev, p->h_in, p->H);
    RB_CUDA(cudaGetLastError());
    int st = decode_impl(p, layer, p->h_in, reinterpret_cast<float *>(dev_o),
                         reinterpret_cast<int *>(dev_o + hb),
                         reinterpret_cast<float *>(dev_o + hb + 32), s, p->err_io);
    if (st) return st;
    k_err_out<<<1, 32, 0, s>>>(p->err_io, dev_err);
    RB_CUDA(cudaGetLastError());
    RB_CUDA(cudaStreamSynchronize(s));
    const int err = *reinterpret_cast<const volatile int *>(pin_o + (p->dio_bytes - 16));
    if (err != 0) {
        if (err == RB_ERR_TIMEOUT)
            return fail(RABBIT_CUDA_ERR_TIMEOUT, "moe_decode: a bounded device wait ran out");
        return fail(RABBIT_CUDA_ERR_DEVICE, "moe_decode: device error code %d", err);
    }
    memcpy(h_out, pin_o, hb);
    if (ids) memcpy(ids, pin_o + hb, sizeof(int) * p->k);
    if (weights) memcpy(weights, pin_o + hb + 32, sizeof(float) * p->k);
    if (k_out) *k_out = p->k;
    return ok();
}

}  // extern "C"

namespace rb {
static bool g_batch_attr[kMaxDevices];

// Records a layer can have (the bucket's range).
static int max_local(const rabbit_cuda_moe *p) { return p->shared_table ? p->n_records : p->epl; }

// Grow the multi-token scratch to T tokens (caller holds no stream work on it).
static int ensure_batch(rabbit_cuda_moe *p, int T) {
    if (T <= p->bt_cap) return RABBIT_CUDA_OK;
    const int cap = std::max(T, std::min(kMaxBatchTokens, 2 * p->bt_cap));
    const int slots = std::max(1, std::min(kMaxSlots, p->k + p->S));
    const size_t P = (size_t)cap * slots, R = (size_t)std::max(1, max_local(p));
    const int KC = p->plan.tc.KC;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off = align_up(off + bytes, 256); return o; };
    const size_t o_xn = take(sizeof(float) * cap * p->H);
    const size_t o_srec = take(sizeof(int) * cap * kMaxSlots);
    const size_t o_sw = take(sizeof(float) * cap * kMaxSlots);
    const size_t o_ns = take(sizeof(int) * cap);
    const size_t o_pidx = take(sizeof(int) * cap * kMaxSlots);
    const size_t o_pt = take(sizeof(int) * P);
    // work units: each record's pairs in runs of at most the unit cap (the
    // narrowest is kTcMinUnit), so at most one per kTcMinUnit pairs plus one
    // partial run per record
    const size_t U = P / kTcMinUnit + R;
    const size_t o_act = take(sizeof(int) * U * 4 + 2 * sizeof(int));
    const size_t o_pu = take(sizeof(int) * P);
    // B rows of the units: three per pair, each unit padded by at most 15; a
    // row holds one byte per input
    const size_t rows = 3 * P + 15 * U;
    const size_t o_xim = take(rows * (size_t)p->H), o_mim = take(rows * (size_t)p->I);
    const size_t o_xu = take(sizeof(float) * P), o_mu = take(sizeof(float) * P);
    const size_t o_sc = take(sizeof(float) * cap * p->E);
    const size_t o_tc = take(sizeof(unsigned) * cap);
    const size_t o_mid = take(sizeof(float) * P * p->I);
    const size_t o_down = take(sizeof(float) * P * KC * p->H);
    const size_t o_h = take(sizeof(float) * cap * p->H);
    const size_t o_ids = take(sizeof(int) * cap * 8);
    const size_t o_w = take(sizeof(float) * cap * 8);
    void *blk = nullptr;
    float *pin = nullptr;
    cudaError_t e = cudaMalloc(&blk, off);
    if (e != cudaSuccess) return cuda_fail(e, "moe_prefill: scratch");
    // the router arrival counts start at zero; the B rows too (a unit's rows
    // past its pairs' are multiplied, their results never read)
    if ((e = cudaMemset(static_cast<uint8_t *>(blk) + o_tc, 0, sizeof(unsigned) * cap)) !=
            cudaSuccess ||
        (e = cudaMemset(static_cast<uint8_t *>(blk) + o_xim, 0, o_xu - o_xim)) != cudaSuccess) {
        cudaFree(blk);
        return cuda_fail(e, "moe_prefill: scratch");
    }
    if ((e = cudaMallocHost(&pin, sizeof(float) * ((size_t)cap * p->H + 2 * (size_t)cap * 8))) !=
        cudaSuccess) {
        cudaFree(blk);
        return cuda_fail(e, "moe_prefill: pinned staging");
    }
    if (p->bt_block) cudaFree(p->bt_block);
    if (p->bt_pin) cudaFreeHost(p->bt_pin);
    p->bt_block = blk;
    p->bt_pin = pin;
    uint8_t *b = static_cast<uint8_t *>(blk);
    MoeBatchArgs &a = p->bt;
    a.xn = reinterpret_cast<float *>(b + o_xn);
    a.srec = reinterpret_cast<int *>(b + o_srec);
    a.sw = reinterpret_cast<float *>(b + o_sw);
    a.nslot = reinterpret_cast<int *>(b + o_ns);
    a.pidx = reinterpret_cast<int *>(b + o_pidx);
    a.pair_t = reinterpret_cast<int *>(b + o_pt);
    a.act = reinterpret_cast<int *>(b + o_act);
    a.act_off = a.act + U;
    a.act_cnt = a.act_off + U;
    a.img_off = a.act_cnt + U;
    a.n_act = a.img_off + U;
    a.pair_u = reinterpret_cast<int *>(b + o_pu);
    a.xim = b + o_xim;
    a.mim = b + o_mim;
    a.xunit = reinterpret_cast<float *>(b + o_xu);
    a.munit = reinterpret_cast<float *>(b + o_mu);
    a.scores = reinterpret_cast<float *>(b + o_sc);
    a.tcount = reinterpret_cast<unsigned *>(b + o_tc);
    a.mid = reinterpret_cast<float *>(b + o_mid);
    a.down = reinterpret_cast<float *>(b + o_down);
    p->bt_h = reinterpret_cast<float *>(b + o_h);
    p->bt_ids = reinterpret_cast<int *>(b + o_ids);
    p->bt_w = reinterpret_cast<float *>(b + o_w);
    p->bt_cap = cap;
    return RABBIT_CUDA_OK;
}

// All-to-all rows per peer for T own tokens: a token sends a peer at most
// one pair per expert that peer holds, and at most k.
static int ep_rows(const rabbit_cuda_moe *p, int T) {
    return T * std::max(1, std::min(p->k, p->E / std::max(1, p->ep_size)));
}
// Tokens the batch scratch must hold for T own tokens: T, plus the rows the
// peers may send in all-to-all mode.
// All-to-all exchange in force (one rank alone has nothing to exchange).
static bool ep_a2a(const rabbit_cuda_moe *p) {
    return p->ep && p->ep_mode == RABBIT_CUDA_EP_ALLTOALL && p->ep_size > 1;
}
static int batch_tokens(const rabbit_cuda_moe *p, int T) {
    return ep_a2a(p) ? T + (p->ep_size - 1) * ep_rows(p, T) : T;
}

// All-to-all buffers for T own tokens (after ensure_batch, whose block they
// join in p->bt).
static int ensure_ep(rabbit_cuda_moe *p, int T) {
    if (T <= p->ep_tcap) return RABBIT_CUDA_OK;
    const size_t peers = (size_t)p->ep_size - 1, cap = (size_t)ep_rows(p, T);
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off = align_up(off + bytes, 256); return o; };
    const size_t o_ids = take(sizeof(int) * T * p->k), o_w = take(sizeof(float) * T * p->k);
    const size_t o_pos = take(sizeof(int) * T * p->k);
    const size_t o_sm = take(sizeof(int4) * peers * cap), o_rm = take(sizeof(int4) * peers * cap);
    const size_t rows = sizeof(float) * peers * cap * p->H;
    const size_t o_sx = take(rows), o_rs = take(rows), o_rr = take(rows);
    void *blk = nullptr;
    cudaError_t e = cudaMalloc(&blk, off);
    if (e != cudaSuccess) return cuda_fail(e, "moe_prefill: exchange buffers");
    if (p->ep_block) cudaFree(p->ep_block);
    p->ep_block = blk;
    uint8_t *b = static_cast<uint8_t *>(blk);
    MoeBatchArgs &a = p->bt;
    a.rt_ids = reinterpret_cast<int *>(b + o_ids);
    a.rt_w = reinterpret_cast<float *>(b + o_w);
    a.pos_tab = reinterpret_cast<int *>(b + o_pos);
    a.send_meta = reinterpret_cast<int4 *>(b + o_sm);
    a.recv_meta = reinterpret_cast<int4 *>(b + o_rm);
    a.send_x = reinterpret_cast<float *>(b + o_sx);
    a.ret_send = reinterpret_cast<float *>(b + o_rs);
    a.ret_recv = reinterpret_cast<float *>(b + o_rr);
    p->ep_tcap = T;
    return RABBIT_CUDA_OK;
}

// One list exchanged with every other rank: n_per_peer elements of dtype per
// peer, peer index qi (rank qi, or qi + 1 from this rank on) at qi * n_per_peer.
struct EpList {
    const void *send;
    void *recv;
    size_t n_per_peer;
    int dtype;
    size_t elem_bytes;
};
// Every list of one exchange step in one NCCL group (a single launch on s).
static int ep_swap(rabbit_cuda_moe *p, const Nccl *n, const EpList *lists, int n_lists,
                   cudaStream_t s) {
    int r = n->group_start();
    for (int qi = 0; r == 0 && qi < p->ep_size - 1; ++qi) {
        const int q = qi < p->ep_rank ? qi : qi + 1;
        for (int l = 0; r == 0 && l < n_lists; ++l) {
            const EpList &L = lists[l];
            const size_t o = (size_t)qi * L.n_per_peer * L.elem_bytes;
            r = n->send(static_cast<const uint8_t *>(L.send) + o, L.n_per_peer, L.dtype, q,
                        p->ep->comm, s);
            if (r == 0)
                r = n->recv(static_cast<uint8_t *>(L.recv) + o, L.n_per_peer, L.dtype, q,
                            p->ep->comm, s);
        }
    }
    const int r2 = n->group_end();
    if (r) return nccl_fail(r, "moe_prefill: exchange");
    if (r2) return nccl_fail(r2, "moe_prefill: exchange (group end)");
    return RABBIT_CUDA_OK;
}

static cudaError_t launch_batch(int which, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                MoeBatchArgs &a) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&a};
    return cudaLaunchKernelExC(&cfg, moe_batch_kernel(which), args);
}

// The batch kernels' static shared memory stays under 1 KB: dynamic sizes
// leave that room.
constexpr size_t kBatchDynMax = (size_t)kMaxDynSmem - 1024;

static cudaError_t launch_tc(int which, bool wide, dim3 grid, dim3 block, size_t smem,
                             cudaStream_t s, void *arg) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {arg};
    return cudaLaunchKernelExC(&cfg, moe_tc_kernel(which, wide), args);
}

// The body of rabbit_cuda_moe_prefill_dev.
static int prefill_launch(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out,
                          int T, int *d_ids, float *d_w, cudaStream_t s);
static int prefill_impl(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out, int T,
                        int *d_ids, float *d_w, cudaStream_t s) {
    int st = window_enter(p, layer, s);
    if (st == RABBIT_CUDA_OK) st = prefill_launch(p, layer, d_h_in, d_h_out, T, d_ids, d_w, s);
    const int st2 = window_leave(p, layer, s);
    return st ? st : st2;
}
static int prefill_launch(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out,
                          int T, int *d_ids, float *d_w, cudaStream_t s) {
    int base, n_local;
    int st = layer_map(p, layer, &base, &n_local);
    if (st) return st;
    for (int r = 0; r < n_local; ++r)
        if (!p->resident[base + r])
        {
            p->misses++;
            return fail(RABBIT_CUDA_ERR_ARGS, "moe_prefill: layer %d not uploaded", layer);
        }
    RB_CUDA(cudaSetDevice(p->device));
    const bool batch = p->tc_ok;
    if (!batch && p->ep_size > 1)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_prefill: expert-parallel pools need the group-32 layout");
    if (!batch) {  // other record formats and shapes: the per-token decode, token by token
        for (int t = 0; t < T; ++t) {
            st = decode_impl(p, layer, d_h_in + (size_t)t * p->H, d_h_out + (size_t)t * p->H,
                             d_ids ? d_ids + (size_t)t * p->k : nullptr,
                             d_w ? d_w + (size_t)t * p->k : nullptr, s, p->ctx->d_err);
            if (st) return st;
        }
        return ok();
    }
    // all-to-all: V tokens = the T own ones and the rows the peers may send
    const bool a2a = ep_a2a(p);
    const int V = batch_tokens(p, T);
    if ((st = ensure_batch(p, V)) != RABBIT_CUDA_OK) return st;
    if (a2a && (st = ensure_ep(p, T)) != RABBIT_CUDA_OK) return st;
    const Nccl *nc = nullptr;
    if (p->ep && p->ep_mode && !(nc = nccl_lib())) return RABBIT_CUDA_ERR_UNSUPPORTED;
    const int sms = p->ctx->sm_count, R = std::max(1, n_local), W = (V + 31) / 32;
    const size_t bucket_smem = sizeof(uint32_t) * (size_t)R * W + 3 * sizeof(int) * R;
    if (bucket_smem > kBatchDynMax)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED, "moe_prefill: layer too wide for the batch kernels");
    if (!g_batch_attr[p->device]) {
        for (int i : {0, 1})
            RB_CUDA(cudaFuncSetAttribute(moe_batch_kernel(i),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kBatchDynMax));
        for (int i : {1, 3})
            for (bool wide : {true, false})
                RB_CUDA(cudaFuncSetAttribute(moe_tc_kernel(i, wide),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)tc_gemm_smem(wide)));
        g_batch_attr[p->device] = true;
    }
    MoeBatchArgs a = p->bt;
    a.h_in = d_h_in;
    a.h_out = d_h_out;
    a.T = T;
    a.ids_out = d_ids;
    a.w_out = d_ids ? d_w : nullptr;
    a.rms = p->rms + (size_t)layer * p->H;
    a.router = p->router + (size_t)layer * p->H * p->E;
    a.pool = p->pool;
    a.rec_stride = p->rec_stride;
    a.off_d = p->off_d;
    a.rec_base = base;
    a.n_local = n_local;
    a.H = p->H;
    a.E = p->E;
    a.k = p->k;
    a.I = p->I;
    a.S = p->S;
    a.usable = p->usable ? 1 : 0;
    a.tb = p->plan.tb;
    a.tc = p->plan.tc;
    a.err = p->ctx->d_err;
    a.wait_ns = wait_limit_ns();
    a.route_split = 8;  // router rows per CTA: E / 8 CTAs per token
    a.ep_rank = p->ep_rank;
    a.ep_size = p->ep_size;
    a.ep_mode = a2a ? RABBIT_CUDA_EP_ALLTOALL : 0;
    // GEMM configuration: the narrow one (two CTAs per SM, 16-pair units) when
    // the layer's gate/up work can fill two CTAs per SM -- the experts the
    // batch can touch here (this rank's routed records, at most the batch's
    // routed pairs, plus the shared ones) times the 128-row items of each --
    // else the wide one (one CTA per SM, an expert read once for up to 32
    // pairs), whose single CTA per SM does not share the SM when work is
    // scarce (one expert per rank in 8-way expert parallelism)
    const int tokens_all = a2a ? T * p->ep_size : T;
    const long long routed_local = std::max(0, n_local - p->S);
    const long long touched =
        std::min(routed_local, (long long)tokens_all * p->k) + std::min(p->S, n_local);
    const bool wide = touched * ((p->I + 127) / 128) < 2ll * sms;
    a.unit_cap = wide ? TcWide::kUnit : TcNarrow::kUnit;
    const int gemm_ctas = (wide ? TcWide::kCtasPerSm : TcNarrow::kCtasPerSm) * sms;
    a.T_own = T;
    a.ep_cap = a2a ? ep_rows(p, T) : 0;
    const size_t cap = (size_t)a.ep_cap, H = (size_t)p->H;
    // per-call timing marks of the exchange (nullptr: timing off); a mode
    // without a first or second exchange records that pair back to back
    EpMarks *mk = p->ep && p->ep_mode ? ep_begin(p->ep, s) : nullptr;
    auto mark = [&](int i) {
        if (mk) cudaEventRecord(mk->ev[i], s);
    };
    RB_CUDA(launch_batch(0, dim3(T, (p->E + a.route_split - 1) / a.route_split), dim3(256),
                         sizeof(float) * (size_t)std::max(p->E, p->H), s, a));
    if (a2a) {  // dispatch: the pairs routed to the peers' experts, with their xn rows
        RB_CUDA(launch_batch(2, dim3(T, p->k), dim3(256), 0, s, a));
        mark(1);
        const EpList lists[2] = {{a.send_meta, a.recv_meta, 4 * cap, kNcclInt32, 4},
                                 {a.send_x, a.xn + (size_t)T * H, cap * H, kNcclFloat32, 4}};
        if ((st = ep_swap(p, nc, lists, 2, s))) return st;
        a.T = V;
    } else {
        mark(1);
    }
    mark(2);
    RB_CUDA(launch_batch(1, dim3(1), dim3(1024), bucket_smem, s, a));
    // B rows: one CTA per pair (pairs counted on the device; the rest leave)
    const unsigned pairs_max = (unsigned)V * std::max(1, std::min(kMaxSlots, p->k + p->S));
    TcGemmArgs ga;
    ga.b = a;
    ga.tmap = p->tm_gu;
    RB_CUDA(launch_tc(0, wide, dim3(pairs_max), dim3(256), 0, s, &a));
    RB_CUDA(launch_tc(1, wide, dim3(gemm_ctas), dim3(tc_threads(wide)), tc_gemm_smem(wide), s, &ga));
    RB_CUDA(launch_tc(2, wide, dim3(pairs_max), dim3(256), 0, s, &a));
    ga.tmap = p->tm_dn;
    RB_CUDA(launch_tc(3, wide, dim3(gemm_ctas), dim3(tc_threads(wide)), tc_gemm_smem(wide), s, &ga));
    if (a2a) {  // combine, first half: the received pairs' outputs go back to their senders
        if (V > T) RB_CUDA(launch_batch(3, dim3(V - T, (p->H + 255) / 256), dim3(256), 0, s, a));
        mark(3);
        const EpList back = {a.ret_send, a.ret_recv, cap * H, kNcclFloat32, 4};
        if ((st = ep_swap(p, nc, &back, 1, s))) return st;
        mark(4);
    }
    RB_CUDA(launch_batch(4, dim3(T, (p->H + 255) / 256), dim3(256), 0, s, a));
    if (p->ep && p->ep_mode == RABBIT_CUDA_EP_ALLREDUCE) {  // the ranks' shares summed
        mark(3);
        const int r = nc->all_reduce(d_h_out, d_h_out, (size_t)T * H, kNcclFloat32, kNcclSum,
                                     p->ep->comm, s);
        if (r) return nccl_fail(r, "moe_prefill: all-reduce");
        mark(4);
    }
    mark(5);
    p->hbm_hits += T;
    return ok();
}
}  // namespace rb

extern "C" {

int rabbit_cuda_moe_prefill_dev(rabbit_cuda_moe *p, int layer, const float *d_h_in, float *d_h_out,
                                int n_tokens, int *d_ids, float *d_weights, void *stream) {
    if (!p || !d_h_in || !d_h_out) return fail(RABBIT_CUDA_ERR_ARGS, "moe_prefill: NULL argument");
    if (n_tokens < 1 || n_tokens > kMaxBatchTokens)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_prefill: n_tokens must be 1..%d", kMaxBatchTokens);
    if ((d_ids == nullptr) != (d_weights == nullptr))
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_prefill: pass both ids and weights, or neither");
    return prefill_impl(p, layer, d_h_in, d_h_out, n_tokens, d_ids, d_weights,
                        as_stream(stream, p->ctx));
}

int rabbit_cuda_moe_set_expert_parallel(rabbit_cuda_moe *p, int rank, int size) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_set_expert_parallel: NULL pool");
    if (size < 1 || rank < 0 || rank >= size)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_set_expert_parallel: rank %d of %d", rank, size);
    if (size > 1 && (p->E % size || p->shared_table || p->epl != p->E / size + p->S))
        return fail(RABBIT_CUDA_ERR_ARGS,
                    "moe_set_expert_parallel: need E (%d) a multiple of %d and %d records per "
                    "layer (E / size routed + %d shared)",
                    p->E, size, p->E / std::max(size, 1) + p->S, p->S);
    p->ep_rank = rank;
    p->ep_size = size;
    return ok();
}

int rabbit_cuda_moe_set_ep(rabbit_cuda_moe *p, rabbit_cuda_ep *ep, int mode) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_set_ep: NULL pool");
    if (!ep || mode == 0) {
        p->ep = nullptr;
        p->ep_mode = 0;
        return ok();
    }
    if (mode != RABBIT_CUDA_EP_ALLREDUCE && mode != RABBIT_CUDA_EP_ALLTOALL)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_set_ep: unknown mode %d", mode);
    if (!ep->comm) return fail(RABBIT_CUDA_ERR_ARGS, "moe_set_ep: the exchange was aborted");
    if (ep->device != p->device)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_set_ep: pool on device %d, exchange on %d", p->device,
                    ep->device);
    if (!p->tc_ok)
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED,
                    "moe_set_ep: expert-parallel pools need the group-32 layout");
    const int st = rabbit_cuda_moe_set_expert_parallel(p, ep->rank, ep->size);
    if (st) return st;
    std::lock_guard<std::mutex> g(p->ctx->mu);
    if (p->ep_block) {  // sized for another rank count
        RB_CUDA(cudaSetDevice(p->device));
        RB_CUDA(cudaDeviceSynchronize());
        cudaFree(p->ep_block);
        p->ep_block = nullptr;
    }
    p->ep_tcap = 0;
    p->ep = ep;
    p->ep_mode = mode;
    return ok();
}

int rabbit_cuda_moe_prefill(rabbit_cuda_moe *p, int layer, const float *h_in, float *h_out,
                            int n_tokens, int *ids, float *weights) {
    if (!p || !h_in || !h_out) return fail(RABBIT_CUDA_ERR_ARGS, "moe_prefill: NULL argument");
    if (n_tokens < 1 || n_tokens > kMaxBatchTokens)
        return fail(RABBIT_CUDA_ERR_ARGS, "moe_prefill: n_tokens must be 1..%d", kMaxBatchTokens);
    std::lock_guard<std::mutex> g(p->ctx->mu);
    RB_CUDA(cudaSetDevice(p->device));
    cudaStream_t s = p->ctx->stream;
    // sized for the whole call up front: the staging below lives in the block
    int st = ensure_batch(p, batch_tokens(p, n_tokens));
    if (st) return st;
    // pinned staging: [h (cap H)] [ids (cap 8)] [weights (cap 8)]; the device
    // copy of h is bt_h, ids / weights go to bt_ids / bt_w
    const size_t hb = sizeof(float) * (size_t)n_tokens * p->H;
    const size_t kb = sizeof(float) * (size_t)n_tokens * p->k;
    int *pin_ids = reinterpret_cast<int *>(p->bt_pin + (size_t)p->bt_cap * p->H);
    float *pin_w = p->bt_pin + (size_t)p->bt_cap * p->H + (size_t)p->bt_cap * 8;
    memcpy(p->bt_pin, h_in, hb);
    RB_CUDA(cudaMemcpyAsync(p->bt_h, p->bt_pin, hb, cudaMemcpyHostToDevice, s));
    const bool want = ids || weights;
    st = prefill_impl(p, layer, p->bt_h, p->bt_h, n_tokens, want ? p->bt_ids : nullptr,
                      want ? p->bt_w : nullptr, s);
    if (st) return st;
    RB_CUDA(cudaMemcpyAsync(p->bt_pin, p->bt_h, hb, cudaMemcpyDeviceToHost, s));
    if (want) {
        RB_CUDA(cudaMemcpyAsync(pin_ids, p->bt_ids, kb, cudaMemcpyDeviceToHost, s));
        RB_CUDA(cudaMemcpyAsync(pin_w, p->bt_w, kb, cudaMemcpyDeviceToHost, s));
    }
    if ((st = check_device_error(p->ctx, s, "moe_prefill")) != RABBIT_CUDA_OK) return st;
    memcpy(h_out, p->bt_pin, hb);
    if (ids) memcpy(ids, pin_ids, kb);
    if (weights) memcpy(weights, pin_w, kb);
    return ok();
}

int rabbit_cuda_moe_stats(const rabbit_cuda_moe *p, uint64_t *hbm_hits, uint64_t *uploads,
                          uint64_t *h2d_bytes, int *resident_records, uint64_t *pool_bytes) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_stats: NULL pool");
    if (hbm_hits) *hbm_hits = p->hbm_hits;
    if (uploads) *uploads = p->uploads;
    if (h2d_bytes) *h2d_bytes = p->h2d_bytes;
    if (resident_records) {
        int n = 0;
        for (uint8_t r : p->resident) n += r;
        *resident_records = n;
    }
    if (pool_bytes) *pool_bytes = p->pool_bytes;
    return ok();
}

int rabbit_cuda_moe_stats_ex(const rabbit_cuda_moe *p, uint64_t *hits, uint64_t *misses,
                             uint64_t *inserts, uint64_t *evictions, uint64_t *bytes_copied,
                             int *n_slots, int *n_pinned) {
    if (!p) return fail(RABBIT_CUDA_ERR_ARGS, "moe_stats_ex: NULL pool");
    if (hits) *hits = p->hbm_hits;
    if (misses) *misses = p->misses;
    if (inserts) *inserts = p->uploads;
    if (evictions) *evictions = p->evictions;
    if (bytes_copied) *bytes_copied = p->h2d_bytes;
    if (n_slots) *n_slots = p->pool_records;
    if (n_pinned) {  // a pool without a window never drops a record it holds
        int n = 0;
        if (!p->window)
            for (uint8_t r : p->resident) n += r;
        *n_pinned = n;
    }
    return ok();
}

uint64_t rabbit_cuda_moe_decode_bytes(const rabbit_cuda_moe *p) {
    if (!p) return 0;
    const uint64_t mat = (uint64_t)p->H * p->I;
    uint64_t per;
    if (p->quant == 0)
        per = 3 * mat * 4;
    else if (p->quant == 4)
        per = 3 * nbytes_g32(mat);
    else
        per = 3 * (4 + mat);
    return 4ull * p->E * p->H + (uint64_t)(p->k + p->S) * per;
}

}  // extern "C"

extern "C" int rabbit_cuda_tile_records(const rabbit_cuda_moe_desc *d, int sm_count, const void *src,
                                        int n_records, void *dst, uint64_t *tiled_size) {
    if (!d || !tiled_size || sm_count <= 0 || n_records < 0 || (n_records > 0 && !src && dst))
        return fail(RABBIT_CUDA_ERR_ARGS, "tile_records: bad arguments");
    if (d->expert_quant != 4 || d->hidden <= 0 || d->inter <= 0 || d->n_experts <= 0)
        return fail(RABBIT_CUDA_ERR_ARGS, "tile_records: needs a group-int4 (expert_quant 4) model");
    // the pool's own planning, on the host only (no device is touched)
    rabbit_cuda_moe q;
    q.H = d->hidden;
    q.I = d->inter;
    q.E = d->n_experts;
    int k = d->experts_per_token > 0 ? d->experts_per_token : 2;
    q.k = std::min(std::min(k, q.E), 8);
    q.S = (d->n_shared > 0 && d->n_shared <= 64) ? d->n_shared : 0;
    q.expert_size = d->expert_size;
    const uint64_t mat = (uint64_t)q.H * q.I, nb = nbytes_g32(mat);
    if (d->expert_size < 3 * nb || mat > 0x7fffffffull || !rb::plan_fused(&q, sm_count))
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED, "tile_records: no tiled layout for this shape");
    const uint64_t rec = q.rec_stride + kTileTrailer;
    *tiled_size = rec;
    if (!dst) return ok();
    const uint8_t *in = static_cast<const uint8_t *>(src);
    uint8_t *out = static_cast<uint8_t *>(dst);
    for (int r = 0; r < n_records; ++r) {
        const uint8_t *blob = in + (uint64_t)r * d->expert_size;
        for (int m = 0; m < 3; ++m) {
            uint32_t gs;
            memcpy(&gs, blob + m * nb, 4);
            if (gs != 32)
                return fail(RABBIT_CUDA_ERR_FORMAT, "tile_records: record %d blob %d has group size %u",
                            r, m, gs);
        }
        uint8_t *o = out + (uint64_t)r * rec;
        memset(o, 0, q.rec_stride);
        rb::tile_pair_host(blob, blob + nb, q.plan.tb, o);
        rb::tile_blob_host(blob + 2 * nb, q.plan.tc, o + q.off_d);
        rb::fill_trailer(&q, o);
    }
    return ok();
}
