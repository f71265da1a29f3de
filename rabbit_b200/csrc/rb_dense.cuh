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
// embed != nullptr: x is row id % V of embed [V, in] (id from *idp, or `id`
// when idp is nullptr; negative -> row 0, forward_v2.c:459-461), and the raw
// row is also written to h (the token's residual stream).
// rope_nmat > 0: matrices m < rope_nmat are heads of rope_hd rows whose
// (2i, 2i + 1) row pairs are rotated for position rope_pos
// (forward_v2.c:92-104) before they are stored. cache[m] != nullptr: y_m is
// also stored there (the KV-cache row of this position).
//
// CTA b owns the stacked rows [b R / G, (b + 1) R / G) rounded down to even
// (R rows, G CTAs; R and every matrix even when rope_nmat > 0) and walks
// them in groups of max(2, 8 / XK); thread t owns the float4 columns t,
// t + 512, ... (XK of them) of x, held in registers, so each row is one
// fully coalesced sweep of the CTA. The loads of the first group go out
// before the wait for the kernel before (weights are not written by it).
// Warps do not wait for one another per group: each posts its row partials
// to a ring of shared buffers (mbarrier arrivals) and streams on; warp 0
// sums, rotates and stores group g while its own loads of g + 1 are in
// flight.
constexpr int kGemvF32Threads = 512;
constexpr int kGemvF32Rows = 8;  // float4 loads per thread and group
struct GemvF32Args {
    const float *W[kMaxGemvMats];
    float *y[kMaxGemvMats];
    const float *res[kMaxGemvMats];
    int rows[kMaxGemvMats];
    int nmat, in_dim;
    const float *x;
    const float *norm_w;
    const float *embed;
    const int *idp;
    int id, V;
    float *h;
    int rope_nmat, rope_hd, rope_pos;
    float *cache[kMaxGemvMats];
    int *err;          // device error word (RB_ERR_TIMEOUT when a wait ran out)
    uint64_t wait_ns;  // bound of every wait
};

// The kernel for rows of `in` floats: XK = ceil(in / 4 / 512) float4 columns
// per thread rounded up to 1, 2, 4 or 8 (in <= 16384); nullptr past that.
const void *gemv_f32_kernel(int in);


// Grid (nh, splits): CTA (h, s) takes query head h and the s-th of `splits`
// equal ranges of the len cached positions -- q already rotated, the cache
// already holding this token's k / v row (the Q/K/V projection stores them).
// Each CTA keeps a running max, sum of exponentials and weighted values over
// its positions (an online softmax); with several splits it leaves them in
// `part` and the last CTA of the head to finish merges them into out
// (forward_v2.c:171-246: scores scaled by 1/sqrt(hd), softmax, weighted sum
// of values). head_dim 32, 64, 128 or 256: k_attention_reg, rows held in
// registers; any other even head_dim: k_attention.
constexpr int kAttnMaxSplits = 8;
constexpr int kAttnThreads = 256;     // k_attention
constexpr int kAttnRegThreads = 256;  // k_attention_reg: eight warps
struct AttnArgs {
    const float *q;       // [nh * hd], RoPE applied
    const float *kc, *vc; // cache [max_len, nkv * hd], this token's row included
    float *out;           // [nh * hd]
    float *part;          // [nh][kAttnMaxSplits][hd + 2]
    unsigned *count;      // [nh] arrivals, zero between launches
    int nh, nkv, hd, len, splits;
};

// Splits for n cached positions: ranges of >= 32.
inline int attention_splits(int n) {
    const int s = (n + 31) / 32;
    return s < 1 ? 1 : (s > kAttnMaxSplits ? kAttnMaxSplits : s);
}
// Dynamic shared memory of k_attention (none for k_attention_reg).
inline size_t attention_smem(int hd, int max_len) {
    const int groups = hd < kAttnThreads ? kAttnThreads / hd : 1;
    return sizeof(float) * (size_t)(hd + max_len + groups * hd);
}
// k_attention_reg for head_dim hd, nullptr when hd is not 32, 64, 128, 256.
const void *attention_reg_kernel(int hd);

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

// Seeded synthetic fill: p[i] uniform with standard deviation `sigma`
// (sigma == 0: every element = `value`).
__global__ void k_fill_f32(float *p, size_t n, uint64_t seed, float sigma, float value);

}  // namespace rb
