// rb_dense.cuh -- the dense (fp32) part of a ref-v2 decode step on B200:
// embedding, fused rmsnorm + projections, RoPE + KV append + attention,
// final norm + lm_head + argmax (forward_v2.c:61-79, 92-104, 171-246, 404-421).
#pragma once
#include <stdint.h>

namespace rb {

constexpr int kMaxGemvMats = 4;

// y_m = W_m x for up to 4 row-major fp32 matrices [rows_m, in] sharing x.
// norm_w != nullptr: x is first replaced by rmsnorm(x) * norm_w
// (forward_v2.c:61-69). res_m != nullptr: y_m = res_m + W_m x (res_m may be y_m).
struct GemvF32Args {
    const float *W[kMaxGemvMats];
    float *y[kMaxGemvMats];
    const float *res[kMaxGemvMats];
    int rows[kMaxGemvMats];
    int nmat, in_dim;
    const float *x;
    const float *norm_w;
};

__global__ void k_gemv_f32(GemvF32Args a);

// One CTA per KV head: RoPE on its k, append k / v at position `len` of the
// cache when len < max_len, then for each of its query heads RoPE on q,
// scores over the cache, softmax, weighted sum of values (forward_v2.c:171-246).
struct AttnArgs {
    float *q;             // [nh * hd] (RoPE applied in place)
    float *k;             // [nkv * hd] (RoPE applied in place)
    const float *v;       // [nkv * hd]
    float *kc, *vc;       // cache [max_len, nkv * hd]
    float *out;           // [nh * hd]
    int nh, nkv, hd, pos, len, max_len;
};

__global__ void k_attention(AttnArgs a);

// Final rmsnorm + lm_head partial sums: partial[c][v] = sum over rows i of
// chunk c of lm_head[i, v] * xn[i], lm_head row-major [H, V] (forward_v2.c:404-413).
struct LmHeadArgs {
    const float *h, *norm_w, *lm_head;
    float *partial;  // [nchunk, V]
    float *hidden;   // the normalised h, written by CTA (0, 0) (may be nullptr)
    int H, V, rows_per_chunk;
};

__global__ void k_lm_head_partial(LmHeadArgs a);

// logits[v] = sum_c partial[c][v] (chunks in order); the argmax keeps the
// lowest index among equal maxima (forward_v2.c:415-421). The last block to
// finish reduces the per-block results into *argmax_out and re-zeroes
// *done_ctr for the next launch.
__global__ void k_logits_argmax(const float *partial, int nchunk, int V, float *logits,
                                int *block_best, float *block_val, int *argmax_out,
                                unsigned *done_ctr);

// h = embed[id % V] (id < 0 -> 0; forward_v2.c:459-461). id from *idp when
// idp != nullptr, else `id`.
__global__ void k_embed(const float *embed, int V, int H, const int *idp, int id, float *h);

// Seeded synthetic fill: p[i] uniform with standard deviation `sigma`
// (sigma == 0: every element = `value`).
__global__ void k_fill_f32(float *p, size_t n, uint64_t seed, float sigma, float value);

}  // namespace rb
