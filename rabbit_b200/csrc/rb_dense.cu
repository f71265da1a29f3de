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
__global__ void __launch_bounds__(kGemvF32Threads, XK >= 8 ? 1 : 2) k_gemv_f32(GemvF32Args a) {
    // rows per group: 8 float4 loads per thread in flight whatever XK
    constexpr int RG = kGemvF32Rows / XK, NW = kGemvF32Threads / 32;
    __shared__ float part[2][NW][kGemvF32Rows];  // per-warp row sums, double-buffered
    __shared__ float red[32];
    launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int in = a.in_dim, in4 = in >> 2;
    int total = 0;
    for (int m = 0; m < a.nmat; ++m) total += a.rows[m];
    const int r0 = (int)((long long)blockIdx.x * total / gridDim.x);
    const int r1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
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
    if (a.norm_w) {
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)in + 1e-5f);
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
    int buf = 0;
    for (int rb = r0; rb < r1; rb += RG, buf ^= 1) {
        if (rb != r0) load_group(rb);
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
        if ((lane & 3) == 0) part[buf][warp][lane >> 2] = tot;
        __syncthreads();
        if (tid < RG && rb + tid < r1) {
            float sum = 0.f;
#pragma unroll
            for (int wi = 0; wi < NW; ++wi) sum += part[buf][wi][tid];
            int m = 0, row = rb + tid;
            while (row >= a.rows[m]) row -= a.rows[m++];
            a.y[m][row] = (a.res[m] ? a.res[m][row] : 0.f) + sum;
        }
    }
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
__device__ __forceinline__ void rope_pairs(float *x, int hd, int pos) {
    // forward_v2.c:92-104
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float freq = 1.0f / powf(10000.0f, (float)i / (float)half);
        const float angle = (float)pos * freq;
        const float c = cosf(angle), s = sinf(angle);
        const float x0 = x[2 * i], x1 = x[2 * i + 1];
        x[2 * i] = x0 * c - x1 * s;
        x[2 * i + 1] = x0 * s + x1 * c;
    }
}

__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    __shared__ bool last;
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int nwarp = nthr >> 5;
    const int head = blockIdx.x, split = blockIdx.y, hd = a.hd, kvd = a.nkv * hd;
    const int rep = a.nh / a.nkv;  // nh is a multiple of nkv (checked at creation)
    const int j = head / rep;
    const int groups = hd < nthr ? nthr / hd : 1;
    float *qs = sm;                // [hd]
    float *ks = qs + hd;           // [hd] this token's k (RoPE applied)
    float *sc = ks + hd;           // [max_len]
    float *pv = sc + a.max_len;    // [groups][hd]
    for (int i = tid; i < hd; i += nthr) {
        qs[i] = a.q[(size_t)head * hd + i];
        ks[i] = a.k[(size_t)j * hd + i];
    }
    __syncthreads();
    rope_pairs(qs, hd, a.pos);
    rope_pairs(ks, hd, a.pos);
    __syncthreads();
    const bool append = a.len < a.max_len;
    const int len = append ? a.len + 1 : a.len;
    const float *vnew = a.v + (size_t)j * hd;
    if (append && head % rep == 0 && split == 0)
        for (int i = tid; i < hd; i += nthr) {
            a.kc[(size_t)a.len * kvd + (size_t)j * hd + i] = ks[i];
            a.vc[(size_t)a.len * kvd + (size_t)j * hd + i] = vnew[i];
        }
    // this CTA's positions [p0, p1); the appended one reads this CTA's own
    // k / v (another CTA writes the cache row)
    const int p0 = (int)((long long)split * len / a.splits);
    const int p1 = (int)((long long)(split + 1) * len / a.splits);
    const int n = p1 - p0;
    const float scale = 1.0f / sqrtf((float)hd);
    // scores: a warp per position, lanes across the head, four at a time
    for (int t0 = warp * 4; t0 < n; t0 += nwarp * 4) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const float *kt[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = p0 + min(t0 + u, n - 1);
            kt[u] = append && t == a.len ? ks : a.kc + (size_t)t * kvd + (size_t)j * hd;
        }
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
    // values: thread (g, i) sums positions g, g + groups, ... of column i
    for (int c = tid; c < groups * hd; c += nthr) {
        const int g = c / hd, i = c - g * hd;
        float acc = 0.f;
#pragma unroll 4
        for (int t = g; t < n; t += groups) {
            const int tp = p0 + t;
            const float vt = append && tp == a.len ? vnew[i]
                                                  : a.vc[(size_t)tp * kvd + (size_t)j * hd + i];
            acc = fmaf(sc[t], vt, acc);
        }
        pv[c] = acc;
    }
    __syncthreads();
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
    // the last CTA of this head merges the splits:
    // out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.count + head, 1u) == (unsigned)a.splits - 1;
    __syncthreads();
    if (!last) return;
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
