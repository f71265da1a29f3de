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
// One warp per row, grid-stride over the rows of all matrices; lanes read
// the row as float4 (eight loads in flight each) against x staged in shared
// memory.
__global__ void __launch_bounds__(512, 2) k_gemv_f32(GemvF32Args a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[32];
    launch_dependents();
    wait_prerequisite();
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int in = a.in_dim, in4 = in >> 2;
    for (int i = tid; i < in; i += nthr) xs[i] = a.x[i];
    if (a.norm_w) {
        __syncthreads();
        float ss = 0.f;
        for (int i = tid; i < in; i += nthr) ss += xs[i] * xs[i];
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)in + 1e-5f);
        for (int i = tid; i < in; i += nthr) xs[i] = (xs[i] * inv) * a.norm_w[i];
    }
    __syncthreads();
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    int total = 0;
    for (int m = 0; m < a.nmat; ++m) total += a.rows[m];
    const int nw = nthr >> 5;
    for (int r = blockIdx.x * nw + warp; r < total; r += gridDim.x * nw) {
        int m = 0, row = r;
        while (row >= a.rows[m]) row -= a.rows[m++];
        const float4 *w4 = reinterpret_cast<const float4 *>(a.W[m] + (size_t)row * in);
        float acc = 0.f;
        int j = lane;
        for (; j + 7 * 32 < in4; j += 8 * 32) {
            float4 w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) w[u] = __ldcs(w4 + j + 32 * u);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float4 x = x4[j + 32 * u];
                acc = fmaf(w[u].x, x.x, acc);
                acc = fmaf(w[u].y, x.y, acc);
                acc = fmaf(w[u].z, x.z, acc);
                acc = fmaf(w[u].w, x.w, acc);
            }
        }
        for (; j < in4; j += 32) {
            const float4 w = __ldcs(w4 + j), x = x4[j];
            acc = fmaf(w.x, x.x, acc);
            acc = fmaf(w.y, x.y, acc);
            acc = fmaf(w.z, x.z, acc);
            acc = fmaf(w.w, x.w, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) a.y[m][row] = (a.res[m] ? a.res[m][row] : 0.f) + acc;
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

__global__ void __launch_bounds__(256) k_attention(AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[32];
    launch_dependents();
    wait_prerequisite();
    const int j = blockIdx.x, hd = a.hd, kv_dim = a.nkv * hd;
    const int rep = a.nh / a.nkv;  // nh is a multiple of nkv (checked at creation)
    float *qs = sm;       // [hd]
    float *sc = sm + hd;  // [max_len]
    float *kh = a.k + (size_t)j * hd;
    rope_pairs(kh, hd, a.pos);
    __syncthreads();
    const int len = a.len < a.max_len ? a.len + 1 : a.len;
    if (a.len < a.max_len)
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            a.kc[(size_t)a.len * kv_dim + (size_t)j * hd + i] = kh[i];
            a.vc[(size_t)a.len * kv_dim + (size_t)j * hd + i] = a.v[(size_t)j * hd + i];
        }
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)hd);
    for (int r = 0; r < rep; ++r) {
        const int head = j * rep + r;
        float *qh = a.q + (size_t)head * hd;
        rope_pairs(qh, hd, a.pos);
        __syncthreads();
        for (int i = threadIdx.x; i < hd; i += blockDim.x) qs[i] = qh[i];
        __syncthreads();
        for (int t = threadIdx.x; t < len; t += blockDim.x) {
            const float *kt = a.kc + (size_t)t * kv_dim + (size_t)j * hd;
            float dot = 0.f;
            for (int i = 0; i < hd; ++i) dot += qs[i] * kt[i];
            sc[t] = dot * scale;
        }
        __syncthreads();
        float mx = -INFINITY;
        for (int t = threadIdx.x; t < len; t += blockDim.x) mx = fmaxf(mx, sc[t]);
        mx = block_max(mx, red);
        float sum = 0.f;
        for (int t = threadIdx.x; t < len; t += blockDim.x) {
            const float e = expf(sc[t] - mx);
            sc[t] = e;
            sum += e;
        }
        sum = block_sum(sum, red);
        if (sum > 0.f)
            for (int t = threadIdx.x; t < len; t += blockDim.x) sc[t] = sc[t] / sum;
        __syncthreads();
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            float acc = 0.f;
            for (int t = 0; t < len; ++t) acc += sc[t] * a.vc[(size_t)t * kv_dim + (size_t)j * hd + i];
            a.out[(size_t)head * hd + i] = acc;
        }
        __syncthreads();
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

// ---------------------------------------------------------------- embed --
__global__ void k_embed(const float *embed, int V, int H, const int *idp, int id, float *h) {
    launch_dependents();
    wait_prerequisite();
    int t = idp ? *idp : id;
    t %= V;
    if (t < 0) t = 0;
    const float *e = embed + (size_t)t * H;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) h[i] = e[i];
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
