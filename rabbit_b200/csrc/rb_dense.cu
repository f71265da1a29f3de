// rb_dense.cu -- dense fp32 kernels of a ref-v2 decode step on B200.
//
// Every kernel is launched programmatic-dependent: it lets the next kernel on
// the stream launch at once and waits for the one before it before it reads
// anything that kernel writes, so the ~65 launches of a token overlap their
// launch latency. All of them stream fp32 weights once per token and are
// HBM-bound; the dot products sum in a different order from the reference's
// serial loops (results agree within fp32 rounding).
#include <math.h>

#include "rb_dense.cuh"
#include "rb_device.cuh"

namespace rb {

__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();  // red may still be read from an earlier call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ float block_max(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? red[lane] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// ------------------------------------------------------------ fp32 GEMV --
__device__ __forceinline__ void fma4(float &acc, const float4 w, const float4 x) {
    acc = fmaf(w.x, x.x, acc);
    acc = fmaf(w.y, x.y, acc);
    acc = fmaf(w.z, x.z, acc);
    acc = fmaf(w.w, x.w, acc);
}

__device__ __forceinline__ const float4 *gemv_row_ptr(const GemvF32Args &a, int r) {
    int m = 0;
    while (r >= a.rows[m]) r -= a.rows[m++];
    return reinterpret_cast<const float4 *>(a.W[m] + (size_t)r * a.in_dim);
}

template <int XK>
__global__ void __launch_bounds__(kGemvF32Threads, XK >= 4 ? 1 : 2) k_gemv_f32(GemvF32Args a) {
    // rows per group: 8 float4 loads per thread in flight (16 for XK = 8),
    // at least 2 so that a RoPE pair never straddles two groups
    constexpr int RG = kGemvF32Rows / XK < 2 ? 2 : kGemvF32Rows / XK;
    constexpr int NW = kGemvF32Threads / 32, NB = 4;
    __shared__ float part[NB][NW][kGemvF32Rows];  // per-warp row sums, a ring of NB groups
    __shared__ __align__(8) uint64_t full[NB], empty[NB];
    __shared__ float red[NW];
    __shared__ float2 rope_cs[512];  // (cos, sin) per pair index, head_dim <= 1024
    launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int in = a.in_dim, in4 = in >> 2;
    int total = 0;
    for (int m = 0; m < a.nmat; ++m) total += a.rows[m];
    int r0 = (int)((long long)blockIdx.x * total / gridDim.x);
    int r1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    if (a.rope_nmat > 0) {  // RoPE pairs stay within a CTA (total is even)
        r0 &= ~1;
        r1 &= ~1;
    }
    float4 w[RG][XK];
    auto load_group = [&](int rb) {
#pragma unroll
        for (int u = 0; u < RG; ++u) {
            const float4 *p = rb + u < r1 ? gemv_row_ptr(a, rb + u) : nullptr;
#pragma unroll
            for (int k = 0; k < XK; ++k) {
                const int c = tid + k * kGemvF32Threads;
                w[u][k] = p && c < in4 ? __ldcs(p + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
    if (r0 < r1) load_group(r0);
    if (tid == 0) {
        for (int b = 0; b < NB; ++b) {
            mbar_init(&full[b], NW);  // every warp posts every group
            mbar_init(&empty[b], 1);  // warp 0, once the group is stored
        }
    }
    if (a.rope_nmat > 0)  // this position's rotation (forward_v2.c:92-104)
        for (int i = tid; i < a.rope_hd / 2; i += kGemvF32Threads) {
            const float freq = 1.0f / powf(10000.0f, (float)i / (float)(a.rope_hd / 2));
            const float angle = (float)a.rope_pos * freq;
            rope_cs[i] = make_float2(cosf(angle), sinf(angle));
        }
    wait_prerequisite();
    if (r0 >= r1 && !(a.embed && blockIdx.x == 0)) return;
    const float *x = a.x;
    if (a.embed) {
        int t = a.idp ? *a.idp : a.id;
        t %= a.V;
        if (t < 0) t = 0;
        x = a.embed + (size_t)t * in;
    }
    const float4 *x4g = reinterpret_cast<const float4 *>(x);
    float4 xv[XK];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < XK; ++k) {
        const int c = tid + k * kGemvF32Threads;
        xv[k] = c < in4 ? x4g[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss += (xv[k].x * xv[k].x + xv[k].y * xv[k].y) + (xv[k].z * xv[k].z + xv[k].w * xv[k].w);
        if (a.embed && blockIdx.x == 0 && c < in4) reinterpret_cast<float4 *>(a.h)[c] = xv[k];
    }
    // one barrier: the sum of squares, and the barriers / table above
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (a.norm_w) {
        float t = 0.f;
#pragma unroll
        for (int wi = 0; wi < NW; ++wi) t += red[wi];
        const float inv = 1.0f / sqrtf(t / (float)in + 1e-5f);
        const float4 *n4 = reinterpret_cast<const float4 *>(a.norm_w);
#pragma unroll
        for (int k = 0; k < XK; ++k) {
            const int c = tid + k * kGemvF32Threads;
            if (c < in4) {
                const float4 nw = n4[c];
                xv[k].x = (xv[k].x * inv) * nw.x;
                xv[k].y = (xv[k].y * inv) * nw.y;
                xv[k].z = (xv[k].z * inv) * nw.z;
                xv[k].w = (xv[k].w * inv) * nw.w;
            }
        }
    }
    // warp 0: sum group g's partials, rotate, store; lane u < RG has row rb + u
    auto finish = [&](int g) -> bool {
        const int b = g % NB, rb = r0 + g * RG;
        if (!mbar_wait(&full[b], (g / NB) & 1, a.wait_ns, a.err)) return false;
        float sum = 0.f;
        if (lane < RG) {
#pragma unroll
            for (int wi = 0; wi < NW; ++wi) sum += part[b][wi][lane];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[b]);
        const int r = rb + lane;
        const bool mine = lane < RG && r < r1;
        int m = 0, row = r;
        if (mine)
            while (row >= a.rows[m]) row -= a.rows[m++];
        float val = mine && a.res[m] ? a.res[m][row] + sum : sum;
        // RoPE: rows 2i, 2i + 1 of a head are lanes 2i', 2i' + 1 here (even
        // group starts, even matrix sizes)
        const float other = __shfl_xor_sync(0xffffffffu, val, 1);
        if (mine) {
            if (m < a.rope_nmat) {
                const float2 cs = rope_cs[(row % a.rope_hd) / 2];
                const float x0 = (row & 1) ? other : val, x1 = (row & 1) ? val : other;
                val = (row & 1) ? x0 * cs.y + x1 * cs.x : x0 * cs.x - x1 * cs.y;
            }
            a.y[m][row] = val;
            if (a.cache[m]) a.cache[m][row] = val;
        }
        return true;
    };
    const int ng = (r1 - r0 + RG - 1) / RG;
    for (int g = 0; g < ng; ++g) {
        if (g > 0) load_group(r0 + g * RG);
        if (warp == 0 && g > 0 && !finish(g - 1)) return;
        float v[kGemvF32Rows];
#pragma unroll
        for (int u = 0; u < kGemvF32Rows; ++u) {
            float acc = 0.f;
            if (u < RG) {
#pragma unroll
                for (int k = 0; k < XK; ++k) fma4(acc, w[u][k], xv[k]);
            }
            v[u] = acc;
        }
        const float tot = warp_reduce8(v);  // lane 4u holds row u's warp sum
        const int b = g % NB;
        if (g >= NB && !mbar_wait(&empty[b], (g / NB - 1) & 1, a.wait_ns, a.err)) return;
        if ((lane & 3) == 0) part[b][warp][lane >> 2] = tot;
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[b]);
    }
    if (warp == 0 && ng > 0) finish(ng - 1);
}

const void *gemv_f32_kernel(int in) {
    const int xk = (in / 4 + kGemvF32Threads - 1) / kGemvF32Threads;
    switch (xk) {
        case 1: return (const void *)k_gemv_f32<1>;
        case 2: return (const void *)k_gemv_f32<2>;
        case 3: case 4: return (const void *)k_gemv_f32<4>;
        case 5: case 6: case 7: case 8: return (const void *)k_gemv_f32<8>;
        default: return nullptr;
    }
}

// ------------------------------------------------------------ attention --
// Positions [p0, p1) of split `split` out of `splits` over len.
__device__ __forceinline__ void split_range(int len, int split, int splits, int &p0, int &p1) {
    p0 = (int)((long long)split * len / splits);
    p1 = (int)((long long)(split + 1) * len / splits);
}

// The last CTA of a head merges the splits' (max m_s, sum l_s, values o_s):
// out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s, M = max m_s. Every
// thread of the CTA calls it after storing its split's values; false for the
// CTAs that are not last.
__device__ bool merge_splits(const AttnArgs &a, int head, bool *last) {
    const int tid = threadIdx.x, nthr = blockDim.x, hd = a.hd;
    __threadfence();
    __syncthreads();
    if (tid == 0) *last = atomicAdd(a.count + head, 1u) == (unsigned)a.splits - 1;
    __syncthreads();
    if (!*last) return false;
    __threadfence();
    const float *ph = a.part + (size_t)head * kAttnMaxSplits * (hd + 2);
    float M = -INFINITY;
    for (int s2 = 0; s2 < a.splits; ++s2) M = fmaxf(M, __ldcg(ph + (size_t)s2 * (hd + 2) + hd));
    float L = 0.f;
    for (int s2 = 0; s2 < a.splits; ++s2) {
        const float *q2 = ph + (size_t)s2 * (hd + 2);
        L += __ldcg(q2 + hd + 1) * expf(__ldcg(q2 + hd) - M);
    }
    for (int i = tid; i < hd; i += nthr) {
        float o = 0.f;
        for (int s2 = 0; s2 < a.splits; ++s2) {
            const float *q2 = ph + (size_t)s2 * (hd + 2);
            o = fmaf(__ldcg(q2 + i), expf(__ldcg(q2 + hd) - M), o);
        }
        a.out[(size_t)head * hd + i] = L > 0.f ? o / L : o;
    }
    if (tid == 0) a.count[head] = 0u;  // ready for the next launch
    return true;
}

// Any even head_dim: scores by a warp per position, values by (group,
// column) threads, two block reductions.
__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    __shared__ bool last;
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int nwarp = nthr >> 5;
    const int head = blockIdx.x, split = blockIdx.y, hd = a.hd, kvd = a.nkv * hd;
    const int j = head / (a.nh / a.nkv);  // nh is a multiple of nkv (checked at creation)
    const int groups = hd < nthr ? nthr / hd : 1;
    int p0, p1;
    split_range(a.len, split, a.splits, p0, p1);
    const int n = p1 - p0;
    float *qs = sm;            // [hd]
    float *sc = qs + hd;       // [n]
    float *pv = sc + n;        // [groups][hd]
    for (int i = tid; i < hd; i += nthr) qs[i] = a.q[(size_t)head * hd + i];
    __syncthreads();
    const float *kb = a.kc + (size_t)j * hd, *vb = a.vc + (size_t)j * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int t0 = warp * 4; t0 < n; t0 += nwarp * 4) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const float *kt[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) kt[u] = kb + (size_t)(p0 + min(t0 + u, n - 1)) * kvd;
        for (int i = lane; i < hd; i += 32) {
            const float qi = qs[i];
#pragma unroll
            for (int u = 0; u < 4; ++u) d[u] = fmaf(qi, kt[u][i], d[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float v = warp_sum(d[u]);
            if (lane == 0 && t0 + u < n) sc[t0 + u] = v * scale;
        }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int t = tid; t < n; t += nthr) mx = fmaxf(mx, sc[t]);
    mx = block_max(mx, red);
    float sum = 0.f;
    for (int t = tid; t < n; t += nthr) {
        const float e = expf(sc[t] - mx);
        sc[t] = e;
        sum += e;
    }
    sum = block_sum(sum, red);  // ends with a barrier: sc is complete
    for (int c = tid; c < groups * hd; c += nthr) {
        const int g = c / hd, i = c - g * hd;
        float acc = 0.f;
#pragma unroll 4
        for (int t = g; t < n; t += groups) acc = fmaf(sc[t], vb[(size_t)(p0 + t) * kvd + i], acc);
        pv[c] = acc;
    }
    __syncthreads();
    if (a.splits == 1) {
        for (int i = tid; i < hd; i += nthr) {
            float o = 0.f;
            for (int g = 0; g < groups; ++g) o += pv[g * hd + i];
            a.out[(size_t)head * hd + i] = sum > 0.f ? o / sum : o;
        }
        return;
    }
    float *mine = a.part + ((size_t)head * kAttnMaxSplits + split) * (hd + 2);
    for (int i = tid; i < hd; i += nthr) {
        float o = 0.f;
        for (int g = 0; g < groups; ++g) o += pv[g * hd + i];
        mine[i] = o;
    }
    if (tid == 0) {
        mine[hd] = mx;
        mine[hd + 1] = sum;
    }
    merge_splits(a, head, &last);
}

// VPL consecutive floats (aligned to min(VPL, 4) floats) as vector loads.
template <int VPL>
__device__ __forceinline__ void load_vec(float (&d)[VPL], const float *p) {
    if constexpr (VPL % 4 == 0) {
#pragma unroll
        for (int v = 0; v < VPL; v += 4) {
            const float4 t = *reinterpret_cast<const float4 *>(p + v);
            d[v] = t.x;
            d[v + 1] = t.y;
            d[v + 2] = t.z;
            d[v + 3] = t.w;
        }
    } else if constexpr (VPL == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(p);
        d[0] = t.x;
        d[1] = t.y;
    } else {
        d[0] = p[0];
    }
}

// head_dim = 32 VPL: lane l holds elements [l VPL, (l + 1) VPL) of q and of
// every k / v row. Each of the four warps takes batches of PB positions
// (batch b: positions p0 + b PB ..., warp b % 4), loads their k and v rows
// at once (2 PB VPL floats per lane in flight), and folds them into its
// running (max, sum, values); the warps are then merged in shared memory.
template <int VPL, int NWA>
__global__ void __launch_bounds__(NWA * 32) k_attention_reg(AttnArgs a) {
    constexpr int HD = 32 * VPL, PB = 32 / VPL < 8 ? 32 / VPL : 8;
    __shared__ float wm[NWA], wl[NWA];
    __shared__ __align__(16) float wo[NWA][HD];
    __shared__ bool last;
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int head = blockIdx.x, split = blockIdx.y, kvd = a.nkv * HD;
    const int j = head / (a.nh / a.nkv);
    int p0, p1;
    split_range(a.len, split, a.splits, p0, p1);
    float q[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) q[v] = a.q[(size_t)head * HD + lane * VPL + v];
    const float *kb = a.kc + (size_t)j * HD + lane * VPL, *vb = a.vc + (size_t)j * HD + lane * VPL;
    const float scale = 1.0f / sqrtf((float)HD);
    float m = -INFINITY, l = 0.f, o[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) o[v] = 0.f;
    for (int t0 = p0 + warp * PB; t0 < p1; t0 += NWA * PB) {
        float kr[PB][VPL], vr[PB][VPL];
#pragma unroll
        for (int u = 0; u < PB; ++u) {
            const int t = min(t0 + u, p1 - 1);
            load_vec<VPL>(kr[u], kb + (size_t)t * kvd);
            load_vec<VPL>(vr[u], vb + (size_t)t * kvd);
        }
        float s[PB], bm = -INFINITY;
#pragma unroll
        for (int u = 0; u < PB; ++u) {
            float d = 0.f;
#pragma unroll
            for (int v = 0; v < VPL; ++v) d = fmaf(q[v], kr[u][v], d);
            d = warp_sum(d);
            s[u] = t0 + u < p1 ? d * scale : -INFINITY;
            bm = fmaxf(bm, s[u]);
        }
        const float mn = fmaxf(m, bm);
        const float corr = expf(m - mn);  // 0 while m is -inf
        l *= corr;
#pragma unroll
        for (int v = 0; v < VPL; ++v) o[v] *= corr;
#pragma unroll
        for (int u = 0; u < PB; ++u) {
            const float pu = expf(s[u] - mn);  // 0 past p1
            l += pu;
#pragma unroll
            for (int v = 0; v < VPL; ++v) o[v] = fmaf(pu, vr[u][v], o[v]);
        }
        m = mn;
    }
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
#pragma unroll
    for (int v = 0; v < VPL; ++v) wo[warp][lane * VPL + v] = o[v];
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < NWA; ++w2) M = fmaxf(M, wm[w2]);
    float L = 0.f, f[NWA];
#pragma unroll
    for (int w2 = 0; w2 < NWA; ++w2) {
        f[w2] = wl[w2] > 0.f ? expf(wm[w2] - M) : 0.f;  // warps without positions add 0
        L += wl[w2] * f[w2];
    }
    if (a.splits == 1) {
        for (int i = tid; i < HD; i += NWA * 32) {
            float acc = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < NWA; ++w2) acc = fmaf(wo[w2][i], f[w2], acc);
            a.out[(size_t)head * HD + i] = L > 0.f ? acc / L : acc;
        }
        return;
    }
    float *mine = a.part + ((size_t)head * kAttnMaxSplits + split) * (HD + 2);
    for (int i = tid; i < HD; i += NWA * 32) {
        float acc = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < NWA; ++w2) acc = fmaf(wo[w2][i], f[w2], acc);
        mine[i] = acc;
    }
    if (tid == 0) {
        mine[HD] = M;
        mine[HD + 1] = L;
    }
    merge_splits(a, head, &last);
}

const void *attention_reg_kernel(int hd) {
    switch (hd) {
        case 32: return (const void *)k_attention_reg<1, kAttnRegThreads / 32>;
        case 64: return (const void *)k_attention_reg<2, kAttnRegThreads / 32>;
        case 128: return (const void *)k_attention_reg<4, kAttnRegThreads / 32>;
        case 256: return (const void *)k_attention_reg<8, kAttnRegThreads / 32>;
        default: return nullptr;
    }
}

// -------------------------------------------------------------- lm_head --
__global__ void __launch_bounds__(256) k_lm_head_partial(LmHeadArgs a) {
    extern __shared__ __align__(16) float xs[];  // rows_per_chunk
    __shared__ float red[32];
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, nthr = blockDim.x;
    float ss = 0.f;
    for (int i = tid; i < a.H; i += nthr) ss += a.h[i] * a.h[i];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)a.H + 1e-5f);  // final norm, forward_v2.c:475-479
    const int r0 = blockIdx.y * a.rows_per_chunk;
    const int r1 = min(a.H, r0 + a.rows_per_chunk);
    for (int i = r0 + tid; i < r1; i += nthr) xs[i - r0] = (a.h[i] * inv) * a.norm_w[i];
    if (a.hidden && blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = tid; i < a.H; i += nthr) a.hidden[i] = (a.h[i] * inv) * a.norm_w[i];
    __syncthreads();
    const int v0 = (blockIdx.x * nthr + tid) * 4;
    if (v0 >= a.V) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if ((a.V & 3) == 0) {
        const float *col = a.lm_head + v0;
        int i = r0;
        for (; i + 7 < r1; i += 8) {
            float4 w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                w[u] = __ldcs(reinterpret_cast<const float4 *>(col + (size_t)(i + u) * a.V));
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float x = xs[i + u - r0];
                acc[0] = fmaf(w[u].x, x, acc[0]);
                acc[1] = fmaf(w[u].y, x, acc[1]);
                acc[2] = fmaf(w[u].z, x, acc[2]);
                acc[3] = fmaf(w[u].w, x, acc[3]);
            }
        }
        for (; i < r1; ++i) {
            const float4 w = __ldcs(reinterpret_cast<const float4 *>(col + (size_t)i * a.V));
            const float x = xs[i - r0];
            acc[0] = fmaf(w.x, x, acc[0]);
            acc[1] = fmaf(w.y, x, acc[1]);
            acc[2] = fmaf(w.z, x, acc[2]);
            acc[3] = fmaf(w.w, x, acc[3]);
        }
    } else {
        for (int i = r0; i < r1; ++i) {
            const float x = xs[i - r0];
            for (int q = 0; q < 4 && v0 + q < a.V; ++q)
                acc[q] = fmaf(a.lm_head[(size_t)i * a.V + v0 + q], x, acc[q]);
        }
    }
    float *p = a.partial + (size_t)blockIdx.y * a.V + v0;
    for (int q = 0; q < 4 && v0 + q < a.V; ++q) p[q] = acc[q];
}

// (value, index) better: larger value, or an equal value at a smaller index
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void block_best(float *sv, int *si) {
    const int tid = threadIdx.x;
    __syncthreads();
    for (int o = blockDim.x >> 1; o > 0; o >>= 1) {
        if (tid < o && better(sv[tid + o], si[tid + o], sv[tid], si[tid])) {
            sv[tid] = sv[tid + o];
            si[tid] = si[tid + o];
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(256) k_logits_argmax(const float *partial, int nchunk, int V,
                                                       float *logits, int *block_best_out,
                                                       float *block_val, int *argmax_out,
                                                       unsigned *done_ctr) {
    __shared__ float sv[256];
    __shared__ int si[256];
    __shared__ bool last;
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, v = blockIdx.x * blockDim.x + tid;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    if (v < V) {
        float s = 0.f;
        for (int c = 0; c < nchunk; ++c) s += partial[(size_t)c * V + v];
        if (logits) logits[v] = s;
        bv = s;
        bi = v;
    }
    sv[tid] = bv;
    si[tid] = bi;
    block_best(sv, si);
    if (tid == 0) {
        block_val[blockIdx.x] = sv[0];
        block_best_out[blockIdx.x] = si[0];
        __threadfence();
        last = atomicAdd(done_ctr, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int b = tid; b < (int)gridDim.x; b += blockDim.x) {
        const float x = __ldcg(block_val + b);
        const int xi = __ldcg(block_best_out + b);
        if (better(x, xi, bv, bi)) {
            bv = x;
            bi = xi;
        }
    }
    sv[tid] = bv;
    si[tid] = bi;
    block_best(sv, si);
    if (tid == 0) {
        *argmax_out = si[0] == 0x7fffffff ? 0 : si[0];
        *done_ctr = 0u;  // ready for the next launch
    }
}

// ----------------------------------------------------------------- fill --
__device__ __forceinline__ uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_fill_f32(float *p, size_t n, uint64_t seed, float sigma, float value) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        if (sigma == 0.f) {
            p[i] = value;
            continue;
        }
        const uint64_t h = mix64(seed ^ (i * 0x9E3779B97F4A7C15ull));
        const float u = ((uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
        p[i] = (2.0f * u - 1.0f) * sigma * 1.7320508f;                          // var sigma^2
    }
}

}  // namespace rb
