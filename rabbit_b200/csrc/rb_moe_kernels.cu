// rb_moe_kernels.cu -- MoE decode on B200: one token through one layer's
// routed + shared SwiGLU experts (forward_v2.c:280-402).
//
// Fused group-32 kernel (k_moe_decode_g32), one CTA per SM, all resident:
//   A. every CTA: rmsnorm(h) -> xn in shared memory; router scores: for
//      routers up to 256 KB every CTA computes all E rows itself (same code
//      and order everywhere, so the same scores); larger routers are split
//      over the CTAs and published as tagged values (below).
//      every CTA: top-k + softmax on the scores (identical in all CTAs), the
//      active slot list (routed in rank order, then shared experts).
//   B. gate/up: the active slots' GU tiles (TRb rows of gate and of up,
//      nibbles + scales, one contiguous block) dealt out round-robin over the
//      CTAs (in reverse CTA order); the producer warp bulk-copies them into the shared-memory ring;
//      eight consumer warps dot them against xn held in registers (JB groups
//      of 32 per lane, ROWSb rows per warp group and tile, both fixed at
//      compile time) and leave per-k-slice partials in shared memory; the
//      epilogue warp stores mid = silu(gate) * up to global scratch, each
//      value tagged with the launch's sequence number.
//   C. down: W2 is tiled as (column chunk of up to 1024 inputs, row tile of
//      TRc rows); the active slots' tiles are dealt out in contiguous ranges
//      over the CTAs in (slot, chunk, row tile) order, so a CTA reads only one
//      or two chunks of mid. The producer issues them right after the CTA's
//      gate/up tiles, so the down
//      weights are in flight while the last gate/up rows finish. A scout warp
//      reads the CTA's chunks of mid once all their values carry this
//      launch's tag and stages them in shared memory; consumers build x
//      planes from there when (slot, chunk) changes; the epilogue warp stores
//      the tagged partial down rows per chunk.
//      combine: row tile t is owned by CTA t % grid, which reads its partials
//      once tagged: down_j = the sum of its chunks in chunk order, h_out =
//      h + sum_j w_j down_j in slot order (forward_v2.c:356-357, 398-399).
// There are no grid barriers: CTAs wait only for the data they read.
// Every wait (mbarrier or tagged value) is bounded by a %globaltimer limit;
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
#ifndef RB_CHUNK_CTA
#define RB_CHUNK_CTA 0
#endif
#define RB_CHUNK(kind, i)                                                     \
    do {                                                                      \
        if (blockIdx.x == RB_CHUNK_CTA && (i) < 64)                           \
            g_chunk_ns[(kind) * 64 + (i)] = globaltimer_ns();                 \
    } while (0)
#define RB_STAMP(i)                                                        \
    do {                                                                   \
        if (threadIdx.x == 0) g_phase_ns[blockIdx.x * 8 + (i)] = globaltimer_ns(); \
    } while (0)
#define RB_DBG(k)                                                                  \
    do {                                                                           \
        if (blockIdx.x == RB_CHUNK_CTA && threadIdx.x == 0) rb_dbg_ns[(k)] = globaltimer_ns(); \
    } while (0)
#else
#define RB_DBG(k) \
    do {          \
    } while (0)
#define RB_STAMP(i) \
    do {            \
    } while (0)
#define RB_CHUNK(kind, i) \
    do {                  \
    } while (0)
#endif

// --------------------------------------------------------------- top-k ----
// Softmax over the k selected scores in place (max-subtracted, expf).
__device__ __forceinline__ void softmax_k(float *w, int k) {
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
    softmax_k(w, k);
}

// forward_v2.c:248-278 by a whole CTA: an expert with a score above the
// -1e30 seed (NaN never qualifies) takes place r = the number of qualifying
// experts with a larger score, or an equal score and a lower index -- the
// order the strict-'>' insertion builds. Places past the qualifying count
// keep (-1, -1e30). One thread per expert, the scores read as float4 from
// shared memory (16-byte aligned); ids / w in shared memory. Every thread
// calls it; thread 0 softmaxes the list last (no sync after that).
__device__ void topk_softmax_block(const float *scores, int E, int k, int *ids, float *w) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    if (tid < k) {
        ids[tid] = -1;
        w[tid] = -1e30f;
    }
    __syncthreads();
    const float4 *s4 = reinterpret_cast<const float4 *>(scores);
    const int E4 = E >> 2;
    for (int e = tid; e < E; e += nthr) {
        const float s = scores[e];
        if (!(s > -1e30f)) continue;
        int r = 0;
#pragma unroll 4
        for (int f4 = 0; f4 < E4; ++f4) {
            const float4 t = s4[f4];
            const int f = 4 * f4;
            r += (t.x > s || (t.x == s && f < e)) ? 1 : 0;
            r += (t.y > s || (t.y == s && f + 1 < e)) ? 1 : 0;
            r += (t.z > s || (t.z == s && f + 2 < e)) ? 1 : 0;
            r += (t.w > s || (t.w == s && f + 3 < e)) ? 1 : 0;
        }
        for (int f = 4 * E4; f < E; ++f) {
            const float t = scores[f];
            r += (t > s || (t == s && f < e)) ? 1 : 0;
        }
        if (r < k) {
            ids[r] = e;
            w[r] = s;
        }
    }
    __syncthreads();
    if (tid == 0) softmax_k(w, k);
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


// Release a stage this warp has no rows of (its wait has completed).
__device__ __forceinline__ void release_stage(uint64_t *empty) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive_cnt(empty, 1);
}

// Values shared between CTAs carry the launch's sequence number: {value,
// seq} in one 64-bit word, stored and loaded as one aligned relaxed 64-bit
// access (single-copy atomic). A reader takes a value once its tag matches
// the current launch -- no counter, no fence. Buffers start zeroed and
// sequence numbers start at 1.
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, unsigned seq) {
    const unsigned long long w = ((unsigned long long)seq << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ __forceinline__ bool tag_ok(unsigned long long w, unsigned seq) {
    return (unsigned)(w >> 32) == seq;
}

__device__ __forceinline__ float tag_val(unsigned long long w) {
    return __uint_as_float((unsigned)w);
}

// Wait until every CTA has published seq in flags[0, n) (every lane polls).
__device__ __forceinline__ bool wait_flags(const unsigned *flags, int n, unsigned seq,
                                           uint64_t limit_ns, int *err) {
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 0;; ++it) {
        bool ok = true;
        for (int b = threadIdx.x & 31; b < n; b += 32) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + b) : "memory");
            ok = ok && v == seq;
        }
        if (__all_sync(0xffffffffu, ok)) return true;
        if ((it & 7u) == 7u && globaltimer_ns() - t0 > limit_ns) {
            set_error(err, RB_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(128);
    }
}

// Partial sums of one unit go to part region i % kPartRing; the warp first
// waits until the epilogue warp has emptied that region (unit i - kPartRing),
// and signals `done` when its partials are written.
__device__ __forceinline__ bool part_acquire(uint64_t *pfree, int i, const MoeFusedArgs &a) {
    if (i < kPartRing) return true;
    return __all_sync(0xffffffffu, mbar_wait(&pfree[i % kPartRing], ((i / kPartRing) - 1) & 1,
                                             a.wait_ns, a.err));
}

__device__ __forceinline__ void part_done(uint64_t *done, int i) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&done[i % kPartRing]);
}

// Phase B for one consumer warp: the CTA's gate/up units u = blockIdx.x +
// n * gridDim.x (n < nB), ROWS rows of gate and of up per tile from rbase.
// `i` counts the CTA's units (ring stages and partial regions).
template <int J, int ROWS>
__device__ __forceinline__ bool moe_gate_up(const MoeFusedArgs &a, const uint8_t *ring,
                                            float *part, uint64_t *full, uint64_t *empty,
                                            uint64_t *done, uint64_t *pfree, uint32_t *sink,
                                            int nB, int &i, int ks, int rbase, bool mine, int g0,
                                            const bool (&act)[J], const XPlanes (&xg)[J]) {
    const int KS = a.KSb, TRb = a.tb.TR, Hh = a.H >> 1, Gb = a.H >> 5;
    for (int n = 0; n < nB; ++n, ++i) {
        const int s = i % a.nslots, ph = i / a.nslots;
        if (threadIdx.x == 0) RB_CHUNK(1, i);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph & 1, a.wait_ns, a.err))) return false;
        if (threadIdx.x == 0) RB_CHUNK(2, i);
        if (!part_acquire(pfree, i, a)) return false;
        float *pp = part + (size_t)(i % kPartRing) * a.part_floats;
        if (mine)
            chunk_dot<2, ROWS, J>(ring + (size_t)s * a.slot_bytes, TRb, rbase, Hh, Gb, g0, act, xg,
                                  [=](int m, int r) { return ((rbase + r) * 2 + m) * KS + ks; },
                                  pp, &empty[s], 1u, sink);
        else
            release_stage(&empty[s]);
        part_done(done, i);
        if (threadIdx.x == 0) RB_CHUNK(3, i);
    }
    return true;
}

// Phase C for one consumer warp: the CTA's units [uc0, uc1), unit u = slot
// u / ntiles, tile u % ntiles of the slot's W2 (column chunk c, row tile t);
// ROWS rows of each tile from rbase. x = the chunk's slice of the slot's mid,
// staged in shared memory by the scout warp (buffer kk & 1 for the CTA's
// kk-th (slot, chunk) key); planes are rebuilt when the key changes (units
// run in key order, so once or twice per CTA).
template <int J, int ROWS>
__device__ __forceinline__ bool moe_down(const MoeFusedArgs &a, const uint8_t *ring, float *part,
                                         uint64_t *full, uint64_t *empty, uint64_t *done,
                                         uint64_t *pfree, uint32_t *sink, const float *xbuf,
                                         int xb, uint64_t *xfull, uint64_t *xfree, int key0,
                                         int uc0, int uc1, int &i, int ks, int rbase, bool mine,
                                         int g0, const bool (&act)[J]) {
    const int KS = a.KSc, TRc = a.tc.TR, ntc = a.tc.ntiles, rt = a.tc.rtiles;
    const int cols = a.tc.cols, Gk = cols >> 5, half = cols >> 1;
    XPlanes xg[J];
    int cur = -1;
    RB_DBG(5);
    // (slot, chunk) key of unit u, relative to the CTA's first, tracked
    // incrementally: units run in (slot, chunk, row tile) order
    int kk = 0, t_in_key = (uc0 % ntc) % rt;
    for (int u = uc0; u < uc1; ++u, ++i) {
        if (u > uc0 && ++t_in_key == rt) {
            t_in_key = 0;
            ++kk;
        }
        if (kk != cur) {
            cur = kk;
            const int b = kk & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&xfull[b], (kk >> 1) & 1, a.wait_ns, a.err)))
                return false;
#pragma unroll
            for (int q = 0; q < J; ++q) load_xplanes_padded(xg[q], xbuf + b * xb, g0 + 32 * q, act[q]);
            __syncwarp();
            if ((threadIdx.x & 31) == 0) mbar_arrive(&xfree[b]);
            RB_DBG(6);
        }
        const int s = i % a.nslots, ph = i / a.nslots;
        if (threadIdx.x == 0) RB_CHUNK(1, i);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph & 1, a.wait_ns, a.err))) return false;
        if (threadIdx.x == 0) RB_CHUNK(2, i);
        if (!part_acquire(pfree, i, a)) return false;
        float *pp = part + (size_t)(i % kPartRing) * a.part_floats;
        if (mine)
            chunk_dot<1, ROWS, J>(ring + (size_t)s * a.slot_bytes, TRc, rbase, half, Gk, g0, act,
                                  xg, [=](int, int r) { return (rbase + r) * KS + ks; }, pp,
                                  &empty[s], 1u, sink);
        else
            release_stage(&empty[s]);
        part_done(done, i);
        if (threadIdx.x == 0) RB_CHUNK(3, i);
    }
    return true;
}

template <int JB, int JC, bool PACKED>
__global__ void __launch_bounds__((kMoeConsumerWarps + 3) * 32, 1) k_moe_decode_g32(MoeFusedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nthr = blockDim.x;
    const int H = a.H, I = a.I, CW = a.CW;
    const int Gb = H >> 5;

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
    float *part = reinterpret_cast<float *>(smem + off);  // kPartRing regions
    off += align_up((size_t)kPartRing * a.part_floats * 4, 16);
    const int xb = (a.tc.cols >> 5) * 33;  // one padded chunk of mid
    float *xbuf = reinterpret_cast<float *>(smem + off);  // [2][xb]
    off += align_up((size_t)2 * xb * 4, 16);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + off);
    uint64_t *empty = full + a.nslots;
    uint32_t *sink = reinterpret_cast<uint32_t *>(empty + a.nslots);  // one word per warp
    uint64_t *rbar = reinterpret_cast<uint64_t *>(sink + 32);  // router staging barrier
    uint64_t *hbar = rbar + 1;                                  // h / rms staging barrier
    uint64_t *done = hbar + 1;                                  // [kPartRing] partials written
    uint64_t *pfree = done + kPartRing;                         // [kPartRing] partials consumed
    uint64_t *xfull = pfree + kPartRing;                        // [2] chunk of mid staged
    uint64_t *xfree = xfull + 2;                                // [2] its planes taken
    const uint32_t router_bytes = (uint32_t)a.E * (uint32_t)H * 4u;
    // Split routing: this CTA scores rows r_e0, r_e0 + grid, ... (r_n rows;
    // r_e0 = CTA % E when E < grid, so every row has several CTAs).
    const int r_e0 = a.E < (int)gridDim.x ? (int)blockIdx.x % a.E : (int)blockIdx.x;
    const int r_n = a.route_local || r_e0 >= a.E ? 0 : (a.E - r_e0 + (int)gridDim.x - 1) / (int)gridDim.x;
    // the ring is idle until routing is done: [router rows] [h] [rms], the
    // router rows being the whole router (route_local) or this CTA's rows
    // (route_stage), else none
    const uint32_t staged =
        a.route_local ? router_bytes : (a.route_stage ? (uint32_t)r_n * (uint32_t)H * 4u : 0u);
    float *hs = reinterpret_cast<float *>(ring + align_up(staged, 128));
    float *rs = hs + H;

    RB_STAMP(0);
    if (tid == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);  // every consumer warp releases every stage
        }
        mbar_init(rbar, 1);
        mbar_init(hbar, 1);
        for (int d = 0; d < kPartRing; ++d) {
            mbar_init(&done[d], CW);  // every consumer warp, after its partials
            mbar_init(&pfree[d], 1);  // the epilogue warp
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&xfull[b], 1);   // the scout warp
            mbar_init(&xfree[b], CW);  // every consumer warp, after its planes
        }
        mbar_init_fence();
        // The norm weights and (small routers) the router block go to the
        // idle ring at once: they are weights, not written by the kernel
        // before this one on the stream. h is: its copy waits for that kernel
        // (programmatic dependent launch; a no-op for a plain launch).
        const uint64_t pol_h = policy_evict_last();
        mbar_arrive_expect_tx(hbar, 8u * (uint32_t)H);
        bulk_g2s(rs, a.rms, 4u * (uint32_t)H, hbar, pol_h);
        if (a.route_local) {
            mbar_arrive_expect_tx(rbar, router_bytes);
            const uint64_t pol = policy_evict_last();  // every CTA reads it
            for (uint32_t o = 0; o < router_bytes; o += 32768u)
                bulk_g2s(ring + o, reinterpret_cast<const uint8_t *>(a.router) + o,
                         router_bytes - o < 32768u ? router_bytes - o : 32768u, rbar, pol);
        } else if (staged) {
            mbar_arrive_expect_tx(rbar, staged);
            const uint64_t pol = policy_evict_last();  // read again every token
            const uint32_t rowb = (uint32_t)H * 4u;
            for (int n = 0; n < r_n; ++n) {
                const uint8_t *src =
                    reinterpret_cast<const uint8_t *>(a.router + (size_t)(r_e0 + n * (int)gridDim.x) * H);
                for (uint32_t o = 0; o < rowb; o += 32768u)
                    bulk_g2s(ring + (size_t)n * rowb + o, src + o,
                             rowb - o < 32768u ? rowb - o : 32768u, rbar, pol);
            }
        }
        wait_prerequisite();
        bulk_g2s(hs, a.h_in, 4u * (uint32_t)H, hbar, pol_h);
    }
    // The next kernel on the stream may launch now (it waits for this one
    // before it reads h or touches scratch).
    launch_dependents();

    // ------------------------------------------------ A: rmsnorm + router --
    // no thread may touch a barrier before thread 0 has initialised it
    __syncthreads();
    RB_DBG(0);
    {
        const bool okh = mbar_wait(hbar, 0, a.wait_ns, a.err);
        if (__syncthreads_or(!okh)) {
            if (!okh) mbar_wait(hbar, 0, a.wait_ns, a.err);  // let the copies land first
            if (staged) mbar_wait(rbar, 0, a.wait_ns, a.err);
            return;
        }
    }
    RB_DBG(1);
    // rmsnorm (forward_v2.c:61-69): x * (1 / sqrt(mean(x^2) + 1e-5)) * w
    const float4 *hs4 = reinterpret_cast<const float4 *>(hs);
    const float4 *rs4 = reinterpret_cast<const float4 *>(rs);
    float ss = 0.f;
    for (int i4 = tid; i4 < (H >> 2); i4 += nthr) {
        const float4 v = hs4[i4];
        ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float t = lane < (nthr >> 5) ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[31] = 1.0f / sqrtf(t / (float)H + 1e-5f);
    }
    __syncthreads();
    const float inv = red[31];
    for (int i4 = tid; i4 < (H >> 2); i4 += nthr) {
        const float4 v = hs4[i4], w = rs4[i4];
        float *xp = xn + xpad(i4 * 4);  // four floats of one group
        xp[0] = (v.x * inv) * w.x;
        xp[1] = (v.y * inv) * w.y;
        xp[2] = (v.z * inv) * w.z;
        xp[3] = (v.w * inv) * w.w;
    }
    __syncthreads();
    RB_DBG(2);
    if (a.route_local) {
        // Every CTA scores every expert itself from the staged router: warp w
        // takes rows w, w + 11, ...; lane l sums inputs 4l + 128t in four
        // chains, then a fixed butterfly. The code and order are the same in every
        // CTA, so every CTA gets the same scores and the same top-k, and no
        // grid barrier is needed.
        const bool okr = mbar_wait(rbar, 0, a.wait_ns, a.err);
        if (__syncthreads_or(!okr)) {
            if (!okr) mbar_wait(rbar, 0, a.wait_ns, a.err);  // let the copy land first
            return;
        }
        RB_DBG(3);
        const float *rt = reinterpret_cast<const float *>(ring);
        // lane l reads inputs 4l + 128t (t < nq): padded xn index xpad(4l) + 132t
        const float *xl = xn + xpad(4 * lane);
        const int nq = (H >> 2) > lane ? ((H >> 2) - lane + 31) >> 5 : 0;
        for (int e = warp; e < a.E; e += nthr >> 5) {
            const float4 *wr = reinterpret_cast<const float4 *>(rt + (size_t)e * H) + lane;
            const float *xp = xl;
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;  // four independent chains
#pragma unroll 4
            for (int t = 0; t < nq; ++t, wr += 32, xp += 132) {
                const float4 w = *wr;
                d0 = fmaf(w.x, xp[0], d0);
                d1 = fmaf(w.y, xp[1], d1);
                d2 = fmaf(w.z, xp[2], d2);
                d3 = fmaf(w.w, xp[3], d3);
            }
            const float d = warp_sum((d0 + d1) + (d2 + d3));
            if (lane == 0) s_sc[e] = d;
        }
        if (tid == 0) s_misc[2] = 0;
        __syncthreads();
        RB_STAMP(1);
    } else {
        // Larger routers: the rows are spread over the CTAs -- rows b, b + G,
        // ... for CTA b when E >= G, else row b % E, so every row has several
        // CTAs and the first of them to finish publishes it -- each score
        // stored tagged with this launch. Every CTA then reads all E scores
        // once their tags match: no grid barrier, no counter. Each copy of a
        // row comes from the same code in the same order, so copies agree bit
        // for bit.
        const int G = (int)gridDim.x;
        const int nw = nthr >> 5;
        if (staged) {
            const bool okr = mbar_wait(rbar, 0, a.wait_ns, a.err);
            if (__syncthreads_or(!okr)) {
                if (!okr) mbar_wait(rbar, 0, a.wait_ns, a.err);  // let the copies land first
                return;
            }
        }
        for (int n = 0; n < r_n; ++n) {
            const int e = r_e0 + n * G;
            const float4 *wr =
                staged ? reinterpret_cast<const float4 *>(ring + (size_t)n * H * 4)
                       : reinterpret_cast<const float4 *>(a.router + (size_t)e * H);
            float d = 0.f;
            for (int i4 = tid; i4 < (H >> 2); i4 += nthr) {
                const float4 w = wr[i4];
                const float *xp = xn + xpad(i4 * 4);  // four floats of one group
                d = fmaf(w.x, xp[0], d);
                d = fmaf(w.y, xp[1], d);
                d = fmaf(w.z, xp[2], d);
                d = fmaf(w.w, xp[3], d);
            }
            d = warp_sum(d);
            if (lane == 0) red[warp] = d;
            __syncthreads();
            if (tid == 0 && e != a.withhold_row) {
                float t = 0.f;
                for (int w = 0; w < nw; ++w) t += red[w];
                st_tagged(a.scores + e, t, a.seq);
            }
            __syncthreads();
        }
        RB_STAMP(1);
        bool okr = true;
        for (int e = tid; okr && e < a.E; e += nthr) {
            const uint64_t t0 = globaltimer_ns();
            for (unsigned it = 0;; ++it) {
                const unsigned long long w = ld_tagged(a.scores + e);
                if (tag_ok(w, a.seq)) {
                    s_sc[e] = tag_val(w);
                    break;
                }
                if ((it & 7u) == 7u && globaltimer_ns() - t0 > a.wait_ns) {
                    set_error(a.err, RB_ERR_TIMEOUT);
                    okr = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        if (tid == 0) s_misc[2] = 0;
        if (__syncthreads_or(!okr)) return;  // nothing in flight yet
        RB_STAMP(6);
    }
    RB_DBG(4);
    // top-k lists in shared memory (the norm's reduction words are free by
    // now)
    topk_softmax_block(s_sc, a.E, a.k, reinterpret_cast<int *>(red), red + 8);
    RB_STAMP(7);
    RB_DBG(8);
    if (tid == 0) {
        const int *ids = reinterpret_cast<const int *>(red);
        const float *w = red + 8;
        if (blockIdx.x == 0) {
            for (int i = 0; i < a.k; ++i) {
                a.ids_out[i] = ids[i];
                a.w_out[i] = w[i];
            }
        }
        s_misc[0] = build_slots(ids, w, a.k, a.E, a.S, a.rec_base, a.n_local, a.usable, s_rec, s_w);
        RB_DBG(9);
    }
    __syncthreads();
    RB_STAMP(2);
    const int nact = s_misc[0];
    if (nact == 0) {
        for (int i = blockIdx.x * nthr + tid; i < H; i += gridDim.x * nthr) a.h_out[i] = a.h_in[i];
        return;
    }

    const int ntb = a.tb.ntiles, TRb = a.tb.TR, ntc = a.tc.ntiles, TRc = a.tc.TR;
    const int G = (int)gridDim.x, bx = (int)blockIdx.x;
    const int UB = nact * ntb;  // gate/up units (slot, GU tile), dealt round-robin
    // gate/up unit n of this CTA is vb + n * G with vb = G - 1 - bx: the last,
    // partial round goes to the highest CTAs, which hold the down units of the
    // last chunks of mid -- the CTAs that finish gate/up last are the ones
    // that would wait for those chunks anyway
    const int vb = G - 1 - bx;
    const int nB = UB > vb ? (UB - vb + G - 1) / G : 0;
    const int UC = nact * ntc;  // down units (slot, chunk, row tile), contiguous ranges
    const int uc0 = bx * UC / G;  // bx * UC < 2^31: UC <= 72 * 16 * 16384 / 1
    const int uc1 = (bx + 1) * UC / G;
    const uint32_t sb = a.tb.tile_stride, sc = a.tc.tile_stride;

    if (warp == CW) {  // -------------------------------------------- producer
        if (lane == 0) {
            // the ring may have held the router, read through the generic proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const uint64_t pol = policy_evict_first();
            int i = 0;
            bool okp = true;
            for (int n = 0; okp && n < nB; ++n, ++i) {
                const int s = i % a.nslots, ph = i / a.nslots;
                if (ph > 0 && !mbar_wait(&empty[s], (ph - 1) & 1, a.wait_ns, a.err, 0)) {
                    okp = false;
                    break;
                }
                const int u = vb + n * G, slot = u / ntb, t = u - slot * ntb;
                const uint8_t *src = a.pool + (size_t)s_rec[slot] * a.rec_stride + (size_t)t * sb;
                RB_CHUNK(0, i);
                mbar_arrive_expect_tx(&full[s], a.tb.tile_bytes);
                bulk_g2s(ring + (size_t)s * a.slot_bytes, src, a.tb.tile_bytes, &full[s], pol);
            }
            for (int u = uc0; okp && u < uc1; ++u, ++i) {
                const int s = i % a.nslots, ph = i / a.nslots;
                if (ph > 0 && !mbar_wait(&empty[s], (ph - 1) & 1, a.wait_ns, a.err, 0)) {
                    okp = false;
                    break;
                }
                const int slot = u / ntc, t = u - slot * ntc;
                const uint8_t *src =
                    a.pool + (size_t)s_rec[slot] * a.rec_stride + a.off_d + (size_t)t * sc;
                RB_CHUNK(0, i);
                mbar_arrive_expect_tx(&full[s], a.tc.tile_bytes);
                bulk_g2s(ring + (size_t)s * a.slot_bytes, src, a.tc.tile_bytes, &full[s], pol);
            }
            // drain: the last use of every stage must have landed before exit
            for (int t = i > a.nslots ? i - a.nslots : 0; t < i; ++t)
                mbar_wait(&full[t % a.nslots], (t / a.nslots) & 1, a.wait_ns, a.err);
        }
        return;
    }

    const int KC = a.tc.KC;
    const int rt_c = a.tc.rtiles;
    // (slot, chunk) key of down unit u; the CTA's keys are key0 .. key of uc1-1
    auto key_of = [&](int u) { const int j = u / ntc; return j * KC + (u - j * ntc) / rt_c; };
    const int key0 = uc0 < uc1 ? key_of(uc0) : 0;

    if (warp == CW + 2) {  // --------------------------------------------- scout
        // For each of the CTA's (slot, chunk) keys in order: once the
        // consumers have taken the planes of key kk - 2 from staging buffer
        // kk & 1, read that chunk of mid until every value carries this
        // launch's tag and copy the values there in the padded layout (33
        // floats per group). Runs while the CTA is still on its gate/up
        // units, so the down units find x ready.
        if (uc0 >= uc1) return;
        const int nkeys = key_of(uc1 - 1) - key0 + 1;
        const int cols = a.tc.cols;
        for (int kk = 0; kk < nkeys; ++kk) {
            const int key = key0 + kk, b = kk & 1;
            if (kk >= 2 &&
                !__all_sync(0xffffffffu, mbar_wait(&xfree[b], ((kk >> 1) - 1) & 1, a.wait_ns, a.err)))
                return;
            // poll the chunk until every value carries this launch's tag
            const unsigned long long *src =
                a.mid + (size_t)(key / KC) * I + (size_t)(key % KC) * cols;
            float *dst = xbuf + b * xb;
            const uint64_t t0 = globaltimer_ns();
            for (int e0 = 0; e0 < cols; e0 += 32 * 16) {
                for (unsigned it = 0;; ++it) {
                    unsigned long long w[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        const int e = e0 + lane + 32 * q;
                        w[q] = e < cols ? ld_tagged(src + e) : (unsigned long long)a.seq << 32;
                    }
                    bool ok = true;
#pragma unroll
                    for (int q = 0; q < 16; ++q) ok = ok && tag_ok(w[q], a.seq);
                    if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const int e = e0 + lane + 32 * q;
                            if (e < cols) dst[xpad(e)] = tag_val(w[q]);
                        }
                        break;
                    }
                    if ((it & 7u) == 7u && globaltimer_ns() - t0 > a.wait_ns) {
                        set_error(a.err, RB_ERR_TIMEOUT);
                        return;
                    }
                    __nanosleep(128);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xfull[b]);
        }
        return;
    }

    if (warp == CW + 1) {  // ------------------------------------------ epilogue
        // Unit by unit, in the consumers' order: sum the KS partials of each
        // row and store mid (gate/up units) or the chunk's down rows (down
        // units) tagged with this launch, then free the partial region. Then
        // combine the row tiles this CTA owns (t = blockIdx.x, + grid, ...):
        // h_out = h + sum_j w_j sum_c down_jc, slots and chunks in order
        // (forward_v2.c:356-357, 398-399), reading each partial once its tag
        // matches and once every CTA has read h (h_out may be h_in).
        // This CTA has read h_in (its copy landed before the norm), and
        // h_out may be h_in: tell the combine owners.
        if (lane == 0)
            asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.flags + blockIdx.x),
                         "r"(a.seq)
                         : "memory");
        const int rt = a.tc.rtiles;
        const int nU = nB + (uc1 - uc0);
        for (int i = 0; i < nU; ++i) {
            const int d = i % kPartRing;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&done[d], (i / kPartRing) & 1, a.wait_ns, a.err)))
                return;
            const float *pp = part + (size_t)d * a.part_floats;
            if (i < nB) {
                const int u = vb + i * G, slot = u / ntb, t = u - slot * ntb;
                for (int r = lane; r < TRb; r += 32) {
                    const int row = t * TRb + r;
                    if (row >= I) continue;
                    float gs = 0.f, us = 0.f;
                    for (int k = 0; k < a.KSb; ++k) {
                        gs += pp[(r * 2) * a.KSb + k];
                        us += pp[(r * 2 + 1) * a.KSb + k];
                    }
                    st_tagged(a.mid + (size_t)slot * I + row, silu_mul(gs, us), a.seq);
                }
            } else {
                const int u = uc0 + (i - nB);
                const int slot = u / ntc, ti = u - slot * ntc, c = ti / rt, t = ti - c * rt;
                for (int r = lane; r < TRc; r += 32) {
                    const int row = t * TRc + r;
                    if (row >= H) continue;
                    float dsum = 0.f;
                    for (int k = 0; k < a.KSc; ++k) dsum += pp[r * a.KSc + k];
                    st_tagged(a.down + ((size_t)slot * KC + c) * H + row, dsum, a.seq);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfree[d]);
        }
        bool flags_seen = false;
        for (int t = bx; t < rt; t += G) {
            if (!flags_seen) {
                if (!wait_flags(a.flags, G, a.seq, a.wait_ns, a.err)) return;
                flags_seen = true;
            }
            const uint64_t t0 = globaltimer_ns();
            // Each of the lane's rows r = lane + 32 m: down_j = the sum of its
            // chunks in chunk order, delta += w_j down_j in slot order, h_out =
            // h + delta. PACKED (fewer than 8 chunks per slot): the row's
            // (slot, chunk) values 16 at a time; else one slot's chunks at a
            // time. Every load of a batch is in flight at once. (The two are
            // separate kernels: either form slows the other's shapes.)
            for (int r = lane; r < TRc; r += 32) {
                const int row = t * TRc + r;
                if (row >= H) break;
                float delta = 0.f;
                if constexpr (PACKED) {
                    const int per_row = nact * KC;
                    float dj = 0.f;
                    int fj = 0, fc = 0;
                    for (int q0 = 0; q0 < per_row; q0 += 16) {
                        unsigned long long w[16];
                        for (unsigned it = 0;; ++it) {
                            int j = fj, c = fc;
#pragma unroll
                            for (int qq = 0; qq < 16; ++qq) {
                                w[qq] = (unsigned long long)a.seq << 32;
                                if (q0 + qq < per_row) {
                                    w[qq] = ld_tagged(a.down + ((size_t)j * KC + c) * H + row);
                                    if (++c == KC) {
                                        c = 0;
                                        ++j;
                                    }
                                }
                            }
                            bool all = true;
#pragma unroll
                            for (int qq = 0; qq < 16; ++qq) all = all && tag_ok(w[qq], a.seq);
                            if (all) break;
                            if ((it & 7u) == 7u && globaltimer_ns() - t0 > a.wait_ns) {
                                set_error(a.err, RB_ERR_TIMEOUT);
                                return;
                            }
                            __nanosleep(128);
                        }
#pragma unroll
                        for (int qq = 0; qq < 16; ++qq) {
                            if (q0 + qq >= per_row) break;
                            dj += tag_val(w[qq]);
                            if (++fc == KC) {
                                fc = 0;
                                delta += s_w[fj] * dj;
                                dj = 0.f;
                                ++fj;
                            }
                        }
                    }
                } else {
                    for (int j = 0; j < nact; ++j) {
                        const unsigned long long *dp = a.down + (size_t)j * KC * H + row;
                        unsigned long long w[16];  // KC <= 16: all loads in flight at once
                        for (unsigned it = 0;; ++it) {
                            bool all = true;
#pragma unroll
                            for (int cc = 0; cc < 16; ++cc) {
                                w[cc] = cc < KC ? ld_tagged(dp + (size_t)cc * H)
                                                : (unsigned long long)a.seq << 32;
                                all = all && tag_ok(w[cc], a.seq);
                            }
                            if (all) break;
                            if ((it & 7u) == 7u && globaltimer_ns() - t0 > a.wait_ns) {
                                set_error(a.err, RB_ERR_TIMEOUT);
                                return;
                            }
                            __nanosleep(128);
                        }
                        float dj = 0.f;
#pragma unroll
                        for (int cc = 0; cc < 16; ++cc)
                            if (cc < KC) dj += tag_val(w[cc]);
                        delta += s_w[j] * dj;
                    }
                }
                a.h_out[row] = a.h_in[row] + delta;
            }
        }
#ifdef RB_PHASE_TIMERS
        if (lane == 0) g_phase_ns[blockIdx.x * 8 + 5] = globaltimer_ns();
#endif
        return;
    }

    // ---------------------------------------------------------- consumers --
    // Warp group q = warp / KS covers one row (KS warps, J groups of 32 inputs
    // per lane) and takes rows [q*ROWS, (q+1)*ROWS) of every tile; warps past
    // the phase's NG groups only release. Every consumer waits for and
    // releases every stage (weight 1), so the ring's phases stay in step
    // across both phases.
    int i = 0;
    bool good;
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
        RB_DBG(7);
        const int rbase = grp * a.ROWSb;
        switch (a.ROWSb) {
            // ROWS * 2 matrices * JB <= 8 (the planner never asks for more)
            case 1: good = moe_gate_up<JB, 1>(a, ring, part, full, empty, done, pfree, sink + warp, nB, i, ks, rbase, mine, g0, act, xg); break;
            case 2: good = moe_gate_up<JB, 2>(a, ring, part, full, empty, done, pfree, sink + warp, nB, i, ks, rbase, mine, g0, act, xg); break;
            default: good = moe_gate_up<JB, 4 / JB>(a, ring, part, full, empty, done, pfree, sink + warp, nB, i, ks, rbase, mine, g0, act, xg); break;
        }
    }
    RB_STAMP(3);
    if (!good) return;
    {  // C: down
        const int ks = warp % a.KSc, grp = warp / a.KSc;
        const int g0 = ks * 32 * JC + lane;
        const bool mine = grp < a.NGc;
        bool act[JC];
#pragma unroll
        for (int q = 0; q < JC; ++q) act[q] = mine && g0 + 32 * q < (a.tc.cols >> 5);
        const int rbase = grp * a.ROWSc;
        switch (a.ROWSc) {
            case 1: moe_down<JC, 1>(a, ring, part, full, empty, done, pfree, sink + warp, xbuf, xb, xfull, xfree, key0, uc0, uc1, i, ks, rbase, mine, g0, act); break;
            case 2: moe_down<JC, 2>(a, ring, part, full, empty, done, pfree, sink + warp, xbuf, xb, xfull, xfree, key0, uc0, uc1, i, ks, rbase, mine, g0, act); break;
            case 4: moe_down<JC, 4>(a, ring, part, full, empty, done, pfree, sink + warp, xbuf, xb, xfull, xfree, key0, uc0, uc1, i, ks, rbase, mine, g0, act); break;
            // ROWS * JC <= 8 (the planner never asks for more)
            default: moe_down<JC, 8 / JC>(a, ring, part, full, empty, done, pfree, sink + warp, xbuf, xb, xfull, xfree, key0, uc0, uc1, i, ks, rbase, mine, g0, act); break;
        }
    }
    RB_STAMP(4);
}

const void *moe_fused_kernel(int JB, int JC, bool packed) {
    if (packed) {
        if (JB == 2)
            return JC == 2 ? (const void *)k_moe_decode_g32<2, 2, true>
                           : (const void *)k_moe_decode_g32<2, 1, true>;
        return JC == 2 ? (const void *)k_moe_decode_g32<1, 2, true>
                       : (const void *)k_moe_decode_g32<1, 1, true>;
    }
    if (JB == 2)
        return JC == 2 ? (const void *)k_moe_decode_g32<2, 2, false>
                       : (const void *)k_moe_decode_g32<2, 1, false>;
    return JC == 2 ? (const void *)k_moe_decode_g32<1, 2, false>
                   : (const void *)k_moe_decode_g32<1, 1, false>;
}

// ======================================================= multi-token path ==
// Grid (T, ceil(E / route_split)): CTA (t, y) scores router rows
// [y route_split, (y + 1) route_split) of token t; the token's last CTA to
// finish ranks all E scores and writes the slot list.
__global__ void __launch_bounds__(256) k_batch_route(MoeBatchArgs a) {
    extern __shared__ __align__(16) float s_sc[];  // [E] router scores (last CTA)
    __shared__ float red[32];
    __shared__ int s_rec[kMaxSlots];
    __shared__ float s_w[kMaxSlots];
    __shared__ bool last;
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int t = blockIdx.x, H = a.H;
    const float *h = a.h_in + (size_t)t * H;
    float *xn = a.xn + (size_t)t * H;
    // rmsnorm (forward_v2.c:61-69), in every CTA of the token; CTA 0 stores xn
    float ss = 0.f;
    for (int i = tid; i < H; i += nthr) ss += h[i] * h[i];
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float v = lane < (nthr >> 5) ? red[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) red[31] = 1.0f / sqrtf(v / (float)H + 1e-5f);
    }
    __syncthreads();
    const float inv = red[31];
    float *xs = s_sc;  // xn staged here first ([H] fits: the launch gives max(E, H) floats)
    for (int i = tid; i < H; i += nthr) {
        const float v = (h[i] * inv) * a.rms[i];
        xs[i] = v;
        if (blockIdx.y == 0) xn[i] = v;
    }
    __syncthreads();
    // this CTA's router rows (forward_v2.c:71-79, :378): a warp per row, 16
    // float4 loads per lane in flight
    const int e0 = blockIdx.y * a.route_split, e1 = min(a.E, e0 + a.route_split);
    for (int e = e0 + warp; e < e1; e += nthr >> 5) {
        const float4 *wr = reinterpret_cast<const float4 *>(a.router + (size_t)e * H);
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        float d = 0.f;
        for (int b = lane; b < (H >> 2); b += 32 * 16) {
            float4 w[16];
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (b + 32 * u < (H >> 2)) w[u] = __ldg(wr + b + 32 * u);
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (b + 32 * u < (H >> 2)) {
                    const float4 x = x4[b + 32 * u];
                    d = fmaf(w[u].x, x.x, d);
                    d = fmaf(w[u].y, x.y, d);
                    d = fmaf(w[u].z, x.z, d);
                    d = fmaf(w[u].w, x.w, d);
                }
        }
        d = warp_sum(d);
        if (lane == 0) a.scores[(size_t)t * a.E + e] = d;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.tcount + t, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int e = tid; e < a.E; e += nthr) s_sc[e] = __ldcg(a.scores + (size_t)t * a.E + e);
    __syncthreads();
    int *ids = reinterpret_cast<int *>(red);
    float *w = red + 8;
    topk_softmax_block(s_sc, a.E, a.k, ids, w);
    if (tid == 0) {
        if (a.ids_out)
            for (int i = 0; i < a.k; ++i) {
                a.ids_out[(size_t)t * a.k + i] = ids[i];
                a.w_out[(size_t)t * a.k + i] = w[i];
            }
        int n = 0;
        if (a.ep_size <= 1) {
            n = build_slots(ids, w, a.k, a.E, a.S, a.rec_base, a.n_local, a.usable, s_rec, s_w);
        } else if (a.ep_mode == 2) {
            // all-to-all: the token's full routing is kept for the dispatch
            // and the combine; local slots are its experts on this rank
            // (local record e / ep_size), then every shared expert
            for (int i = 0; i < a.k; ++i) {
                a.rt_ids[(size_t)t * a.k + i] = a.usable ? ids[i] : -1;
                a.rt_w[(size_t)t * a.k + i] = w[i];
            }
            if (a.usable) {
                for (int i = 0; i < a.k; ++i)
                    if (ids[i] >= 0 && ids[i] % a.ep_size == a.ep_rank) {
                        s_rec[n] = a.rec_base + ids[i] / a.ep_size;
                        s_w[n] = w[i];
                        ++n;
                    }
                const int e_loc = a.E / a.ep_size;
                for (int sh = 0; sh < a.S; ++sh)
                    if (e_loc + sh < a.n_local) {
                        s_rec[n] = a.rec_base + e_loc + sh;
                        s_w[n] = 1.0f;
                        ++n;
                    }
            }
        } else if (a.usable) {
            // expert-parallel: this rank holds routed experts e = ep_rank (mod
            // ep_size) as local records e / ep_size, then the shared experts;
            // rank 0 alone applies the shared ones
            const int e_loc = a.E / a.ep_size;
            for (int i = 0; i < a.k; ++i)
                if (ids[i] >= 0 && ids[i] % a.ep_size == a.ep_rank && ids[i] / a.ep_size < a.n_local) {
                    s_rec[n] = a.rec_base + ids[i] / a.ep_size;
                    s_w[n] = w[i];
                    ++n;
                }
            if (a.ep_rank == 0)
                for (int sh = 0; sh < a.S; ++sh)
                    if (e_loc + sh < a.n_local) {
                        s_rec[n] = a.rec_base + e_loc + sh;
                        s_w[n] = 1.0f;
                        ++n;
                    }
        }
        a.nslot[t] = n;
        for (int j = 0; j < n; ++j) {
            a.srec[(size_t)t * kMaxSlots + j] = s_rec[j];
            a.sw[(size_t)t * kMaxSlots + j] = s_w[j];
        }
        a.tcount[t] = 0u;  // ready for the next launch
    }
}

// One CTA. Ranks come from per-record token bitmasks, so the pair order is
// token order whatever order the atomics land in.
__global__ void __launch_bounds__(1024) k_batch_bucket(MoeBatchArgs a) {
    extern __shared__ __align__(16) uint32_t bm[];  // [R][W] bits, then cnt[R], off[R], uf[R]
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int R = a.n_local, W = (a.T + 31) >> 5;
    int *cnt = reinterpret_cast<int *>(bm + (size_t)R * W), *off = cnt + R, *uf = off + R;
    for (int i = tid; i < R * W; i += nthr) bm[i] = 0u;
    if (a.ep_mode == 2) {
        // all-to-all: each received row is a token of one slot, the local
        // record its sender named (padding rows: no slot)
        for (int v = a.T_own + tid; v < a.T; v += nthr) {
            const int4 m = a.recv_meta[v - a.T_own];
            const bool used = m.w != 0 && m.z >= 0 && m.z < R;
            a.nslot[v] = used ? 1 : 0;
            if (used) {
                a.srec[(size_t)v * kMaxSlots] = a.rec_base + m.z;
                a.sw[(size_t)v * kMaxSlots] = 1.0f;
            }
        }
    }
    __syncthreads();
    const int Q = a.T * kMaxSlots;
    for (int q = tid; q < Q; q += nthr) {
        const int t = q / kMaxSlots, j = q - t * kMaxSlots;
        if (j < a.nslot[t]) {
            const int r = a.srec[q] - a.rec_base;
            atomicOr(&bm[r * W + (t >> 5)], 1u << (t & 31));
        }
    }
    __syncthreads();
    for (int r = tid; r < R; r += nthr) {
        int c = 0;
        for (int x = 0; x < W; ++x) c += __popc(bm[r * W + x]);
        cnt[r] = c;
    }
    __syncthreads();
    const int cap = a.unit_cap;
    if (tid == 0) {  // units: each record's pairs cut into runs of <= unit_cap
        int o = 0, nu = 0, rows = 0;
        for (int r = 0; r < R; ++r) {
            off[r] = o;
            uf[r] = nu;  // the record's first unit
            for (int c0 = 0; c0 < cnt[r]; c0 += cap) {
                const int n = min(cap, cnt[r] - c0);
                a.act[nu] = a.rec_base + r;
                a.act_off[nu] = o + c0;
                a.act_cnt[nu] = n;
                a.img_off[nu] = rows;  // the unit's B rows follow the earlier units'
                rows += tc_n_of(n);
                ++nu;
            }
            o += cnt[r];
        }
        a.n_act[0] = nu;
        a.n_act[1] = o;  // pairs
    }
    __syncthreads();
    for (int q = tid; q < Q; q += nthr) {
        const int t = q / kMaxSlots, j = q - t * kMaxSlots;
        if (j < a.nslot[t]) {
            const int r = a.srec[q] - a.rec_base;
            int rank = 0;
            for (int x = 0; x < (t >> 5); ++x) rank += __popc(bm[r * W + x]);
            rank += __popc(bm[r * W + (t >> 5)] & ((1u << (t & 31)) - 1u));
            const int pos = off[r] + rank;
            a.pair_t[pos] = t;
            a.pair_u[pos] = (uf[r] + rank / cap) * kTcMaxUnit + rank % cap;
            a.pidx[q] = pos;
        }
    }
}

// h_out = h + sum_j w_j down_j, down_j = the sum of its chunks in chunk order
// (forward_v2.c:356-357, 398-399); grid (T, ceil(H / 256)).
__global__ void __launch_bounds__(256) k_batch_combine(MoeBatchArgs a) {
    launch_dependents();
    wait_prerequisite();
    const int t = blockIdx.x, row = blockIdx.y * blockDim.x + threadIdx.x;
    if (row >= a.H) return;
    const int ns = a.nslot[t], KC = a.tc.KC;
    float delta = 0.f;
    if (a.ep_mode == 2) {
        // all-to-all: the token's routed slots in order, each from its local
        // pair or from the row its owner sent back, then the shared experts
        // (local): the same terms in the same order as one pool's combine
        int jl = 0;
        for (int i = 0; i < a.k; ++i) {
            const int e = a.rt_ids[(size_t)t * a.k + i];
            if (e < 0) continue;
            float dj = 0.f;
            const int q = e % a.ep_size;
            if (q == a.ep_rank) {
                const int pj = a.pidx[(size_t)t * kMaxSlots + jl++];
                for (int c = 0; c < KC; ++c) dj += a.down[((size_t)pj * KC + c) * a.H + row];
            } else {
                const int qi = q < a.ep_rank ? q : q - 1;
                const int r = a.pos_tab[(size_t)t * a.k + i];
                dj = a.ret_recv[((size_t)qi * a.ep_cap + r) * a.H + row];
            }
            delta += a.rt_w[(size_t)t * a.k + i] * dj;
        }
        for (; jl < ns; ++jl) {
            const int pj = a.pidx[(size_t)t * kMaxSlots + jl];
            float dj = 0.f;
            for (int c = 0; c < KC; ++c) dj += a.down[((size_t)pj * KC + c) * a.H + row];
            delta += a.sw[(size_t)t * kMaxSlots + jl] * dj;
        }
        a.h_out[(size_t)t * a.H + row] = a.h_in[(size_t)t * a.H + row] + delta;
        return;
    }
    for (int j = 0; j < ns; ++j) {
        const int pj = a.pidx[(size_t)t * kMaxSlots + j];
        float dj = 0.f;
        for (int c = 0; c < KC; ++c) dj += a.down[((size_t)pj * KC + c) * a.H + row];
        delta += a.sw[(size_t)t * kMaxSlots + j] * dj;
    }
    // expert-parallel ranks other than 0 leave their share only; the ranks'
    // outputs then sum to h + delta
    const float base = a.ep_rank == 0 ? a.h_in[(size_t)t * a.H + row] : 0.f;
    a.h_out[(size_t)t * a.H + row] = base + delta;
}

// All-to-all dispatch, grid (T_own, k): CTA (t, i) places pair (token t,
// slot i) in the list of the rank that owns its expert (e % ep_size), when
// that is another rank: its row there is the number of earlier pairs (token
// major, slot minor) with the same owner, so every list is in token order
// whatever order the CTAs run in. The row gets the token's xn row and
// {t, i, local record e / ep_size, 1}; CTA (0, 0) marks each list's rows
// past its count unused.
__global__ void __launch_bounds__(256) k_ep_pack(MoeBatchArgs a) {
    __shared__ int s_pos;
    launch_dependents();
    wait_prerequisite();
    const int t = blockIdx.x, i = blockIdx.y, tid = threadIdx.x, nthr = blockDim.x;
    const int K = a.k, size = a.ep_size, rank = a.ep_rank, cap = a.ep_cap;
    const int n = a.T_own * K;
    if (t == 0 && i == 0) {
        for (int qi = 0; qi < size - 1; ++qi) {
            const int q = qi < rank ? qi : qi + 1;
            int c = 0;
            for (int x0 = 0; x0 < n; x0 += nthr) {
                const int x = x0 + tid;
                const int e = x < n ? a.rt_ids[x] : -1;
                c += __syncthreads_count(e >= 0 && e % size == q);
            }
            for (int r = c + tid; r < cap; r += nthr)
                a.send_meta[(size_t)qi * cap + r] = make_int4(0, 0, 0, 0);
        }
    }
    const int me = t * K + i, e = a.rt_ids[me];
    if (e < 0 || e % size == rank) {
        if (tid == 0) a.pos_tab[me] = -1;
        return;
    }
    const int q = e % size, qi = q < rank ? q : q - 1;
    int c = 0;
    for (int x0 = 0; x0 < me; x0 += nthr) {
        const int x = x0 + tid;
        const int ex = x < me ? a.rt_ids[x] : -1;
        c += __syncthreads_count(ex >= 0 && ex % size == q);
    }
    if (tid == 0) {
        s_pos = c;
        a.pos_tab[me] = c;
        a.send_meta[(size_t)qi * cap + c] = make_int4(t, i, e / size, 1);
    }
    __syncthreads();
    const float4 *src = reinterpret_cast<const float4 *>(a.xn + (size_t)t * a.H);
    float4 *dst = reinterpret_cast<float4 *>(a.send_x + ((size_t)qi * cap + s_pos) * a.H);
    for (int j = tid; j < (a.H >> 2); j += nthr) dst[j] = src[j];
}

// All-to-all return, grid (T - T_own, ceil(H / 256)): each received pair's
// expert output (its down row: the column chunks summed in order) into the
// list that goes back to its sender, at the row it came in.
__global__ void __launch_bounds__(256) k_ep_return(MoeBatchArgs a) {
    launch_dependents();
    wait_prerequisite();
    const int v = a.T_own + blockIdx.x, row = blockIdx.y * blockDim.x + threadIdx.x;
    if (row >= a.H || a.nslot[v] == 0) return;
    const int KC = a.tc.KC, pj = a.pidx[(size_t)v * kMaxSlots];
    float dj = 0.f;
    for (int c = 0; c < KC; ++c) dj += a.down[((size_t)pj * KC + c) * a.H + row];
    a.ret_send[(size_t)blockIdx.x * a.H + row] = dj;
}

const void *moe_batch_kernel(int i) {
    switch (i) {
        case 0: return (const void *)k_batch_route;
        case 1: return (const void *)k_batch_bucket;
        case 2: return (const void *)k_ep_pack;
        case 3: return (const void *)k_ep_return;
        case 4: return (const void *)k_batch_combine;
        default: return nullptr;
    }
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
