// rb_moe_kernels.cu -- MoE decode on B200: one token through one layer's
// routed + shared SwiGLU experts (forward_v2.c:280-402).
//
// Fused group-32 kernel (k_moe_decode_g32), cooperative launch, one CTA per SM:
//   A. every CTA: rmsnorm(h) -> xn in shared memory; CTA c computes router
//      rows c, c+grid, ... -> scores.            [grid barrier 1]
//      every CTA: top-k + softmax on the scores (identical in all CTAs), the
//      active slot list (routed in rank order, then shared experts).
//   B. gate/up: the active slots' gate and up rows, flattened and split evenly
//      over CTAs in units of 4 rows; the producer warp bulk-copies chunks of
//      gate+up rows (nibbles + scales) into the shared-memory ring; consumer
//      warps dot them against xn held in registers (one group of 32 per lane);
//      mid = silu(gate) * up goes to global scratch.
//   C. down + combine: each CTA owns 4-row units of the H outputs for every
//      active slot; the producer keeps issuing these W2 chunks as soon as
//      ring stages free up -- before and during grid barrier 2 -- so the down
//      weights are in flight while the last gate/up rows finish. Consumers
//      reload x = mid[slot] per slot and combine h_out = h + sum_j w_j down_j
//      in slot order (forward_v2.c:356-357, 398-399).
// Every wait (mbarrier or grid barrier) is bounded by a %globaltimer limit;
// a timeout records RB_ERR_TIMEOUT and the CTA drains its copies and exits.
#include "rb_gemv.cuh"
#include "rb_moe.cuh"

namespace rb {

// ---------------------------------------------------------- grid barrier --
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread per CTA. bar[0] counts arrivals, bar[1] is the generation.
__device__ bool grid_barrier(unsigned *bar, unsigned nblocks, uint64_t wait_ns, int *err) {
    const unsigned gen = ld_acquire_u32(bar + 1);
    __threadfence();
    const unsigned prev = atomicAdd(bar, 1u);
    if (prev == nblocks - 1) {
        atomicExch(bar, 0u);
        __threadfence();
        st_release_u32(bar + 1, gen + 1);
        return true;
    }
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 1;; ++it) {
        if (ld_acquire_u32(bar + 1) != gen) return true;
        if ((it & 31u) == 0 && globaltimer_ns() - t0 > wait_ns) {
            set_error(err, RB_ERR_TIMEOUT);
            return false;
        }
    }
}

// --------------------------------------------------------------- top-k ----
// forward_v2.c:248-278: insertion into a descending list seeded (-1, -1e30),
// strict '>' (lower index wins ties, NaN never enters), softmax over the k.
__device__ void topk_softmax(const float *scores, int E, int k, int *ids, float *w) {
    for (int i = 0; i < k; ++i) {
        ids[i] = -1;
        w[i] = -1e30f;
    }
    for (int e = 0; e < E; ++e) {
        const float s = __ldcg(scores + e);
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

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float sg = 1.0f / (1.0f + expf(-g));  // forward_v2.c:327-331
    return (g * sg) * u;
}

// Phase-B cursor: 4-row units over the flattened (slot, row) space of I rows
// per slot; a chunk never crosses a slot boundary.
__device__ __forceinline__ bool next_b(int &u, int ub1, int I, int CR, int &slot, int &r,
                                       int &rows) {
    if (u >= ub1) return false;
    const int per = I >> 2;
    slot = u / per;
    r = (u - slot * per) * 4;
    rows = min(CR, min(4 * (ub1 - u), I - r));
    u += rows >> 2;
    return true;
}

__device__ __forceinline__ void load_x32(float (&xr)[32], const float *src, bool act, bool l2) {
    if (act) {
        const float4 *p = reinterpret_cast<const float4 *>(src);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 t = l2 ? __ldcg(p + j) : p[j];
            xr[4 * j] = t.x;
            xr[4 * j + 1] = t.y;
            xr[4 * j + 2] = t.z;
            xr[4 * j + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) xr[j] = 0.f;
    }
}

__global__ void __launch_bounds__(17 * 32, 1) k_moe_decode_g32(MoeFusedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nthr = blockDim.x;
    const int H = a.H, I = a.I, CW = a.CW;
    const int Hh = H >> 1, Ih = I >> 1, Gb = H >> 5, Gc = I >> 5;

    size_t off = 0;
    float *xn = reinterpret_cast<float *>(smem);
    off = align_up((size_t)H * 4, 128);
    float *red = reinterpret_cast<float *>(smem + off);
    off += 128;
    int *s_rec = reinterpret_cast<int *>(smem + off);
    off += kMaxSlots * 4;
    float *s_w = reinterpret_cast<float *>(smem + off);
    off += kMaxSlots * 4;
    int *s_misc = reinterpret_cast<int *>(smem + off);  // [0] nact [1] abort A [2] abort B
    off = align_up(off + 16, 128);
    uint8_t *ring = smem + off;
    off += (size_t)a.nslots * a.slot_bytes;
    float *part = reinterpret_cast<float *>(smem + off);
    off += align_up((size_t)a.part_floats * 4, 16);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + off);
    uint64_t *empty = full + a.nslots;

    if (tid == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init_fence();
    }

    // ------------------------------------------------ A: rmsnorm + router --
    float ss = 0.f;
    for (int i = tid; i < H; i += nthr) {
        const float v = a.h_in[i];
        ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < (nthr >> 5); ++w) t += red[w];
        t /= (float)H;
        red[31] = 1.0f / sqrtf(t + 1e-5f);  // forward_v2.c:61-69
    }
    __syncthreads();
    const float inv = red[31];
    for (int i = tid; i < H; i += nthr) xn[i] = (a.h_in[i] * inv) * a.rms[i];
    __syncthreads();
    for (int e = blockIdx.x; e < a.E; e += gridDim.x) {
        const float *wr = a.router + (size_t)e * H;
        float d = 0.f;
        for (int i = tid; i < H; i += nthr) d += wr[i] * xn[i];
        d = warp_sum(d);
        if (lane == 0) red[warp] = d;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int w = 0; w < (nthr >> 5); ++w) t += red[w];
            a.scores[e] = t;
        }
        __syncthreads();
    }
    if (tid == 0) {
        __threadfence();
        s_misc[1] = grid_barrier(a.bar, gridDim.x, a.wait_ns, a.err) ? 0 : 1;
        s_misc[2] = 0;
        if (!s_misc[1]) {
            int ids[8];
            float w[8];
            topk_softmax(a.scores, a.E, a.k, ids, w);
            if (blockIdx.x == 0) {
                for (int i = 0; i < a.k; ++i) {
                    a.ids_out[i] = ids[i];
                    a.w_out[i] = w[i];
                }
            }
            s_misc[0] =
                build_slots(ids, w, a.k, a.E, a.S, a.rec_base, a.n_local, a.usable, s_rec, s_w);
        }
    }
    __syncthreads();
    if (s_misc[1]) return;  // nothing in flight yet
    const int nact = s_misc[0];
    if (nact == 0) {
        for (int i = blockIdx.x * nthr + tid; i < H; i += gridDim.x * nthr) a.h_out[i] = a.h_in[i];
        return;
    }

    const int UB = nact * (I >> 2);
    const int ub0 = (int)((long long)blockIdx.x * UB / gridDim.x);
    const int ub1 = (int)((long long)(blockIdx.x + 1) * UB / gridDim.x);
    const int UC = H >> 2;
    const int uc0 = (int)((long long)blockIdx.x * UC / gridDim.x);
    const int uc1 = (int)((long long)(blockIdx.x + 1) * UC / gridDim.x);
    const int c0 = 4 * uc0, c1 = 4 * uc1;

    if (warp == CW) {  // -------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int i = 0;
            bool okp = true;
            int u = ub0, slot, r, rows;
            while (okp && next_b(u, ub1, I, a.CRb, slot, r, rows)) {
                const int s = i % a.nslots, n = i / a.nslots;
                if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.wait_ns, a.err)) {
                    okp = false;
                    break;
                }
                const uint8_t *rec = a.pool + (size_t)s_rec[slot] * a.rec_stride;
                const uint32_t nb = (uint32_t)rows * Hh, sb = (uint32_t)rows * (H >> 3);
                uint8_t *dst = ring + (size_t)s * a.slot_bytes;
                const size_t cn = (size_t)a.CRb * Hh, cs = (size_t)a.CRb * (H >> 3);
                mbar_arrive_expect_tx(&full[s], 2 * (nb + sb));
                bulk_g2s(dst, rec + a.off_gnib + (size_t)r * Hh, nb, &full[s], pol);
                bulk_g2s(dst + cn, rec + a.off_unib + (size_t)r * Hh, nb, &full[s], pol);
                bulk_g2s(dst + 2 * cn, rec + a.off_gsc + (size_t)r * (H >> 3), sb, &full[s], pol);
                bulk_g2s(dst + 2 * cn + cs, rec + a.off_usc + (size_t)r * (H >> 3), sb, &full[s],
                         pol);
                ++i;
            }
            for (int j = 0; okp && j < nact; ++j) {
                const uint8_t *rec = a.pool + (size_t)s_rec[j] * a.rec_stride;
                for (int rr = c0; rr < c1; rr += a.CRc) {
                    const int s = i % a.nslots, n = i / a.nslots;
                    if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.wait_ns, a.err)) {
                        okp = false;
                        break;
                    }
                    const int rws = min(a.CRc, c1 - rr);
                    const uint32_t nb = (uint32_t)rws * Ih, sb = (uint32_t)rws * (I >> 3);
                    uint8_t *dst = ring + (size_t)s * a.slot_bytes;
                    mbar_arrive_expect_tx(&full[s], nb + sb);
                    bulk_g2s(dst, rec + a.off_dnib + (size_t)rr * Ih, nb, &full[s], pol);
                    bulk_g2s(dst + (size_t)a.CRc * Ih, rec + a.off_dsc + (size_t)rr * (I >> 3), sb,
                             &full[s], pol);
                    ++i;
                }
            }
            // drain: the last use of every stage must have landed before exit
            for (int t = i > a.nslots ? i - a.nslots : 0; t < i; ++t)
                mbar_wait(&full[t % a.nslots], (t / a.nslots) & 1, a.wait_ns, a.err);
        }
        return;
    }

    // ---------------------------------------------------------- consumers --
    bool good = true;
    int i = 0;
    {  // B: gate + up
        const int ks = warp % a.KSb, rsub = warp / a.KSb;
        const int g = ks * 32 + lane;
        const bool wact = rsub < a.RSb;
        const bool act = wact && g < Gb;
        float xr[32];
        load_x32(xr, xn + g * 32, act, false);
        const size_t cn = (size_t)a.CRb * Hh, cs = (size_t)a.CRb * (H >> 3);
        int u = ub0, slot, r, rows;
        while (next_b(u, ub1, I, a.CRb, slot, r, rows)) {
            const int s = i % a.nslots, n = i / a.nslots;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[s], n & 1, a.wait_ns, a.err))) {
                good = false;
                break;
            }
            const uint8_t *st = ring + (size_t)s * a.slot_bytes;
            const float *gsc = reinterpret_cast<const float *>(st + 2 * cn);
            const float *usc = reinterpret_cast<const float *>(st + 2 * cn + cs);
            const int lbase = slot * I + r - 4 * ub0;
            if (wact) {
                for (int rb = rsub; rb < rows; rb += 4 * a.RSb) {
                    float v[8];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int rr = rb + b * a.RSb;
                        v[b] = 0.f;
                        v[b + 4] = 0.f;
                        if (act && rr < rows) {
                            const uint4 wg =
                                *reinterpret_cast<const uint4 *>(st + (size_t)rr * Hh + g * 16);
                            const uint4 wu =
                                *reinterpret_cast<const uint4 *>(st + cn + (size_t)rr * Hh + g * 16);
                            v[b] = dot32_q64(wg, xr) * (gsc[rr * Gb + g] * 64.f);
                            v[b + 4] = dot32_q64(wu, xr) * (usc[rr * Gb + g] * 64.f);
                        }
                    }
                    const float tot = warp_reduce8(v);
                    if ((lane & 3) == 0) {
                        const int idx = lane >> 2;  // 0..3 gate rows, 4..7 up rows
                        const int rr = rb + (idx & 3) * a.RSb;
                        if (rr < rows)
                            part[((lbase + rr) * 2 + (idx >> 2)) * a.KSb + ks] = tot;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ++i;
        }
    }
    named_sync(1, CW * 32);
    if (good) {
        const int nrb = 4 * (ub1 - ub0);
        for (int lr = tid; lr < nrb; lr += CW * 32) {
            float gs = 0.f, us = 0.f;
            for (int k = 0; k < a.KSb; ++k) {
                gs += part[(lr * 2) * a.KSb + k];
                us += part[(lr * 2 + 1) * a.KSb + k];
            }
            a.mid[4 * ub0 + lr] = silu_mul(gs, us);
        }
    }
    __threadfence();
    named_sync(1, CW * 32);
    if (tid == 0) s_misc[2] = grid_barrier(a.bar, gridDim.x, a.wait_ns, a.err) ? 0 : 1;
    named_sync(1, CW * 32);
    good = good && !s_misc[2];

    {  // C: down + combine
        const int ks = warp % a.KSc, rsub = warp / a.KSc;
        const int g = ks * 32 + lane;
        const bool wact = rsub < a.RSc;
        const bool act = wact && g < Gc;
        float xr[32];
        const size_t cn = (size_t)a.CRc * Ih;
        for (int j = 0; good && j < nact; ++j) {
            load_x32(xr, a.mid + (size_t)j * I + g * 32, act, true);
            for (int rr0 = c0; rr0 < c1; rr0 += a.CRc) {
                const int rows = min(a.CRc, c1 - rr0);
                const int s = i % a.nslots, n = i / a.nslots;
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], n & 1, a.wait_ns, a.err))) {
                    good = false;
                    break;
                }
                const uint8_t *st = ring + (size_t)s * a.slot_bytes;
                const float *dsc = reinterpret_cast<const float *>(st + cn);
                if (wact) {
                    for (int rb = rsub; rb < rows; rb += 8 * a.RSc) {
                        float v[8];
#pragma unroll
                        for (int b = 0; b < 8; ++b) {
                            const int rr = rb + b * a.RSc;
                            v[b] = 0.f;
                            if (act && rr < rows) {
                                const uint4 w =
                                    *reinterpret_cast<const uint4 *>(st + (size_t)rr * Ih + g * 16);
                                v[b] = dot32_q64(w, xr) * (dsc[rr * Gc + g] * 64.f);
                            }
                        }
                        const float tot = warp_reduce8(v);
                        if ((lane & 3) == 0) {
                            const int rr = rb + (lane >> 2) * a.RSc;
                            if (rr < rows)
                                part[((rr0 - c0 + rr) * nact + j) * a.KSc + ks] = tot;
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                ++i;
            }
        }
    }
    named_sync(1, CW * 32);
    if (!good) return;
    for (int lr = tid; lr < c1 - c0; lr += CW * 32) {
        float delta = 0.f;
        for (int j = 0; j < nact; ++j) {
            float d = 0.f;
            for (int k = 0; k < a.KSc; ++k) d += part[(lr * nact + j) * a.KSc + k];
            delta += s_w[j] * d;
        }
        a.h_out[c0 + lr] = a.h_in[c0 + lr] + delta;
    }
}

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
