// rb_refv2.cu -- C ABI: the incremental ref-v2 decode context
// (RabbitRefV2Ctx, src/rabbit.h:160-167) with every weight and the KV cache
// resident in HBM.
//
// One token is one stream of programmatic-dependent launches on the device
// context's stream: embed; per layer the fused rmsnorm + Q/K/V projections,
// attention (RoPE, KV append, softmax, values), the O projection with the
// residual, and the fused MoE decode of the layer; then the final norm +
// lm_head partial sums and the logits / argmax reduction (forward_v2.c:457-484).
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "rb_dense.cuh"
#include "rb_moe.cuh"
#include "rb_runtime.h"

namespace {
constexpr int kMaxNew = 4096;       // tokens per rabbit_cuda_refv2_generate call
constexpr int kLmRowsPerChunk = 128;  // lm_head rows per partial-sum chunk
}  // namespace

struct rabbit_cuda_refv2 {
    int device = -1;
    rb::DevCtx *ctx = nullptr;
    rabbit_cuda_moe *moe = nullptr;
    int L = 0, H = 0, V = 0, nh = 0, nkv = 0, hd = 0, qd = 0, kvd = 0, max_ctx = 0;
    // dense weights, one block: embed | lm_head | final_norm | per layer
    // [rms_attn | w_q | w_k | w_v | w_o]
    float *w = nullptr;
    size_t w_floats = 0, layer_floats = 0;
    float *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;
    float *kc = nullptr, *vc = nullptr;  // [L][max_ctx][kvd]
    // activations and outputs
    float *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *hidden = nullptr, *logits = nullptr, *partial = nullptr, *bval = nullptr;
    int *bbest = nullptr, *ids = nullptr;  // ids[kMaxNew + 1]: argmax chain
    unsigned *done = nullptr;
    float *apart = nullptr;     // attention split partials [nh][kAttnMaxSplits][hd + 2]
    unsigned *acount = nullptr; // attention arrivals per head [nh]
    float *pin = nullptr;  // host staging: logits | hidden | argmax
    int nchunk = 0, lm_blocks = 0, am_blocks = 0;
    const void *gemv_h = nullptr, *gemv_q = nullptr;  // projection kernels, rows of H / q_dim
    const void *attn_reg = nullptr;  // register attention for this head_dim (or nullptr)
    int pos = 0, len = 0;
    bool stepped = false;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;  // around the kernels of the last call
    float last_ms = 0.f;

    float *rms_attn(int l) const { return w + off_layers() + (size_t)l * layer_floats; }
    float *w_q(int l) const { return rms_attn(l) + H; }
    float *w_k(int l) const { return w_q(l) + (size_t)qd * H; }
    float *w_v(int l) const { return w_k(l) + (size_t)kvd * H; }
    float *w_o(int l) const { return w_v(l) + (size_t)kvd * H; }
    size_t off_layers() const { return 2 * (size_t)V * H + H; }
};

namespace rb {


static void free_refv2(rabbit_cuda_refv2 *c) {
    if (c->device >= 0) cudaSetDevice(c->device);
    void *bufs[] = {c->w,      c->kc,      c->vc,   c->h,    c->q,     c->k,    c->v,
                    c->att,    c->hidden,  c->logits, c->partial, c->bval, c->bbest, c->ids,
                    c->done,   c->apart,   c->acount};
    for (void *b : bufs)
        if (b) cudaFree(b);
    if (c->pin) cudaFreeHost(c->pin);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    delete c;
}

static cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                  cudaLaunchAttribute *attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

static cudaError_t launch_pdl_ptr(const void *kern, dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t s, void **args) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(grid, block, smem, s, attr);
    return cudaLaunchKernelExC(&cfg, kern, args);
}

template <typename... Args>
static cudaError_t launch_pdl(void (*kern)(Args...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(grid, block, smem, s, attr);
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Enqueue one token on `s`: its id from *idp (device) when idp != nullptr,
// else `id`; its argmax to *argmax_out (device). 4 L + 2 launches: per layer
// the Q/K/V projections (with the embedding lookup in layer 0), attention,
// the O projection and the MoE block; then lm_head and the argmax.
static int enqueue_step(rabbit_cuda_refv2 *c, const int *idp, int id, int *argmax_out,
                        bool want_hidden, cudaStream_t s) {
    const int sms = c->ctx->sm_count;
    const uint64_t wait_ns = wait_limit_ns();
    const int kv_after = c->len < c->max_ctx ? c->len + 1 : c->len;
    // register attention: one CTA per head covers the whole window (<= 256
    // positions: a round or four of 64 per CTA); the shared-memory kernel
    // splits the window over CTAs of 32 positions and more
    const int splits = c->attn_reg ? 1 : attention_splits(kv_after);
    for (int l = 0; l < c->L; ++l) {
        GemvF32Args g = {};
        g.nmat = 3;
        g.W[0] = c->w_q(l);
        g.W[1] = c->w_k(l);
        g.W[2] = c->w_v(l);
        g.y[0] = c->q;
        g.y[1] = c->k;
        g.y[2] = c->v;
        g.rows[0] = c->qd;
        g.rows[1] = c->kvd;
        g.rows[2] = c->kvd;
        g.in_dim = c->H;
        g.x = c->h;
        g.norm_w = c->rms_attn(l);
        g.err = c->ctx->d_err;
        g.wait_ns = wait_ns;
        if (l == 0) {  // h = embed[id % V] (forward_v2.c:459-461)
            g.embed = c->embed;
            g.idp = idp;
            g.id = id;
            g.V = c->V;
            g.h = c->h;
        }
        // q and k rotated for this position; k / v rows appended to the cache
        // while it has room (forward_v2.c:190-202)
        g.rope_nmat = 2;
        g.rope_hd = c->hd;
        g.rope_pos = c->pos;
        float *kc_l = c->kc + (size_t)l * c->max_ctx * c->kvd;
        float *vc_l = c->vc + (size_t)l * c->max_ctx * c->kvd;
        if (c->len < c->max_ctx) {
            g.cache[1] = kc_l + (size_t)c->len * c->kvd;
            g.cache[2] = vc_l + (size_t)c->len * c->kvd;
        }
        void *ga[] = {&g};
        RB_CUDA(launch_pdl_ptr(c->gemv_h, dim3(2 * sms), dim3(kGemvF32Threads), 0, s, ga));
        AttnArgs at;
        at.q = c->q;
        at.kc = kc_l;
        at.vc = vc_l;
        at.out = c->att;
        at.part = c->apart;
        at.count = c->acount;
        at.nh = c->nh;
        at.nkv = c->nkv;
        at.hd = c->hd;
        at.len = kv_after;
        at.splits = splits;
        void *aa[] = {&at};
        if (c->attn_reg)
            RB_CUDA(launch_pdl_ptr(c->attn_reg, dim3(c->nh, splits), dim3(kAttnRegThreads), 0, s, aa));
        else
            RB_CUDA(launch_pdl(k_attention, dim3(c->nh, splits), dim3(kAttnThreads),
                               attention_smem(c->hd, c->max_ctx), s, at));
        GemvF32Args o = {};
        o.nmat = 1;
        o.W[0] = c->w_o(l);
        o.y[0] = c->h;
        o.res[0] = c->h;
        o.rows[0] = c->H;
        o.in_dim = c->qd;
        o.x = c->att;
        o.err = c->ctx->d_err;
        o.wait_ns = wait_ns;
        void *oa[] = {&o};
        RB_CUDA(launch_pdl_ptr(c->gemv_q, dim3(2 * sms), dim3(kGemvF32Threads), 0, s, oa));
        const int st = rabbit_cuda_moe_decode_dev(c->moe, l, c->h, c->h, nullptr, nullptr, s);
        if (st != RABBIT_CUDA_OK) return st;
    }
    LmHeadArgs lm;
    lm.h = c->h;
    lm.norm_w = c->final_norm;
    lm.lm_head = c->lm_head;
    lm.partial = c->partial;
    lm.hidden = want_hidden ? c->hidden : nullptr;
    lm.H = c->H;
    lm.V = c->V;
    lm.rows_per_chunk = kLmRowsPerChunk;
    RB_CUDA(launch_pdl(k_lm_head_partial, dim3(c->lm_blocks, c->nchunk), dim3(256),
                       sizeof(float) * (size_t)kLmRowsPerChunk, s, lm));
    RB_CUDA(launch_pdl(k_logits_argmax, dim3(c->am_blocks), dim3(256), 0, s,
                       (const float *)c->partial, c->nchunk, c->V, c->logits, c->bbest, c->bval,
                       argmax_out, c->done));
    ++c->pos;
    if (c->len < c->max_ctx) ++c->len;
    c->stepped = true;
    return RABBIT_CUDA_OK;
}

// Copy the requested outputs of the last step to the host and check errors.
static int finish(rabbit_cuda_refv2 *c, cudaStream_t s, float *logits, float *hidden,
                  int *argmax) {
    float *pl = c->pin, *ph = c->pin + c->V;
    int *pa = reinterpret_cast<int *>(ph + c->H);
    RB_CUDA(cudaEventRecord(c->ev1, s));
    if (logits)
        RB_CUDA(cudaMemcpyAsync(pl, c->logits, sizeof(float) * c->V, cudaMemcpyDeviceToHost, s));
    if (hidden)
        RB_CUDA(cudaMemcpyAsync(ph, c->hidden, sizeof(float) * c->H, cudaMemcpyDeviceToHost, s));
    RB_CUDA(cudaMemcpyAsync(pa, c->ids, sizeof(int), cudaMemcpyDeviceToHost, s));
    const int st = check_device_error(c->ctx, s, "refv2");
    if (st != RABBIT_CUDA_OK) return st;
    RB_CUDA(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
    if (logits) memcpy(logits, pl, sizeof(float) * c->V);
    if (hidden) memcpy(hidden, ph, sizeof(float) * c->H);
    if (argmax) *argmax = *pa;
    return RABBIT_CUDA_OK;
}

}  // namespace rb

using namespace rb;

extern "C" {

int rabbit_cuda_refv2_create(const rabbit_cuda_dense_desc *d, rabbit_cuda_moe *moe,
                             rabbit_cuda_refv2 **out) {
    if (!d || !moe || !out) return fail(RABBIT_CUDA_ERR_ARGS, "refv2_create: NULL argument");
    *out = nullptr;
    int device, mL, mH;
    moe_shape(moe, &device, &mL, &mH);
    if (d->n_layers < 1 || d->hidden < 4 || (d->hidden & 3) || d->vocab < 1 || d->n_heads < 1 ||
        d->n_kv_heads < 1 || d->n_heads % d->n_kv_heads || d->head_dim < 2 || (d->head_dim & 1) ||
        d->head_dim > 1024 || ((d->n_heads * d->head_dim) & 3) || d->max_ctx < 1 ||
        d->max_ctx > 256)
        return fail(RABBIT_CUDA_ERR_ARGS,
                    "refv2_create: need hidden and n_heads*head_dim multiples of 4, n_heads a "
                    "multiple of n_kv_heads, an even head_dim <= 1024, max_ctx in 1..256");
    if (mL != d->n_layers || mH != d->hidden)
        return fail(RABBIT_CUDA_ERR_ARGS, "refv2_create: the MoE pool has %d layers of hidden %d",
                    mL, mH);
    if (!gemv_f32_kernel(d->hidden) || !gemv_f32_kernel(d->n_heads * d->head_dim))
        return fail(RABBIT_CUDA_ERR_UNSUPPORTED, "refv2_create: hidden / q width above 16384");
    int st;
    DevCtx *ctx = dev_ctx(device, &st);
    if (!ctx) return st;
    auto *c = new rabbit_cuda_refv2();
    c->device = device;
    c->ctx = ctx;
    c->moe = moe;
    c->L = d->n_layers;
    c->H = d->hidden;
    c->V = d->vocab;
    c->nh = d->n_heads;
    c->nkv = d->n_kv_heads;
    c->hd = d->head_dim;
    c->qd = c->nh * c->hd;
    c->kvd = c->nkv * c->hd;
    c->max_ctx = d->max_ctx;
    c->layer_floats = (size_t)c->H + (size_t)c->qd * c->H + 2 * (size_t)c->kvd * c->H +
                      (size_t)c->H * c->qd;
    c->w_floats = c->off_layers() + (size_t)c->L * c->layer_floats;
    c->nchunk = (c->H + kLmRowsPerChunk - 1) / kLmRowsPerChunk;
    c->lm_blocks = (c->V + 1023) / 1024;
    c->am_blocks = (c->V + 255) / 256;
    cudaError_t e = cudaSetDevice(device);
    const size_t kv = (size_t)c->L * c->max_ctx * c->kvd;
    if (e == cudaSuccess &&
        ((e = cudaMalloc(&c->w, sizeof(float) * c->w_floats)) != cudaSuccess ||
         (e = cudaMalloc(&c->kc, sizeof(float) * kv)) != cudaSuccess ||
         (e = cudaMalloc(&c->vc, sizeof(float) * kv)) != cudaSuccess ||
         (e = cudaMalloc(&c->h, sizeof(float) * c->H)) != cudaSuccess ||
         (e = cudaMalloc(&c->q, sizeof(float) * c->qd)) != cudaSuccess ||
         (e = cudaMalloc(&c->k, sizeof(float) * c->kvd)) != cudaSuccess ||
         (e = cudaMalloc(&c->v, sizeof(float) * c->kvd)) != cudaSuccess ||
         (e = cudaMalloc(&c->att, sizeof(float) * c->qd)) != cudaSuccess ||
         (e = cudaMalloc(&c->hidden, sizeof(float) * c->H)) != cudaSuccess ||
         (e = cudaMalloc(&c->logits, sizeof(float) * c->V)) != cudaSuccess ||
         (e = cudaMalloc(&c->partial, sizeof(float) * (size_t)c->nchunk * c->V)) != cudaSuccess ||
         (e = cudaMalloc(&c->bval, sizeof(float) * c->am_blocks)) != cudaSuccess ||
         (e = cudaMalloc(&c->bbest, sizeof(int) * c->am_blocks)) != cudaSuccess ||
         (e = cudaMalloc(&c->ids, sizeof(int) * (kMaxNew + 1))) != cudaSuccess ||
         (e = cudaMalloc(&c->done, sizeof(unsigned))) != cudaSuccess ||
         (e = cudaMemset(c->done, 0, sizeof(unsigned))) != cudaSuccess ||
         (e = cudaMalloc(&c->apart, sizeof(float) * (size_t)c->nh * kAttnMaxSplits *
                                        (c->hd + 2))) != cudaSuccess ||
         (e = cudaMalloc(&c->acount, sizeof(unsigned) * c->nh)) != cudaSuccess ||
         (e = cudaMemset(c->acount, 0, sizeof(unsigned) * c->nh)) != cudaSuccess ||
         (e = cudaMemset(c->ids, 0, sizeof(int) * (kMaxNew + 1))) != cudaSuccess ||
         (e = cudaMallocHost(&c->pin, sizeof(float) * ((size_t)c->V + c->H + 4))) !=
             cudaSuccess ||
         (e = cudaEventCreate(&c->ev0)) != cudaSuccess ||
         (e = cudaEventCreate(&c->ev1)) != cudaSuccess)) {
    }
    if (e != cudaSuccess) {
        free_refv2(c);
        return cuda_fail(e, "refv2_create: device memory");
    }
    c->embed = c->w;
    c->lm_head = c->w + (size_t)c->V * c->H;
    c->final_norm = c->lm_head + (size_t)c->H * c->V;
    c->gemv_h = gemv_f32_kernel(c->H);
    c->gemv_q = gemv_f32_kernel(c->qd);
    c->attn_reg = attention_reg_kernel(c->hd);
    if (d->embed) {  // host weights -> the device block
        if (!d->lm_head || !d->final_norm || !d->rms_attn || !d->w_q || !d->w_k || !d->w_v ||
            !d->w_o) {
            free_refv2(c);
            return fail(RABBIT_CUDA_ERR_ARGS, "refv2_create: incomplete dense weights");
        }
        struct Part {
            float *dst;
            const float *src;
            size_t n;
        };
        std::vector<Part> parts = {{c->embed, d->embed, (size_t)c->V * c->H},
                                   {c->lm_head, d->lm_head, (size_t)c->H * c->V},
                                   {c->final_norm, d->final_norm, (size_t)c->H}};
        for (int l = 0; l < c->L; ++l) {
            parts.push_back({c->rms_attn(l), d->rms_attn[l], (size_t)c->H});
            parts.push_back({c->w_q(l), d->w_q[l], (size_t)c->qd * c->H});
            parts.push_back({c->w_k(l), d->w_k[l], (size_t)c->kvd * c->H});
            parts.push_back({c->w_v(l), d->w_v[l], (size_t)c->kvd * c->H});
            parts.push_back({c->w_o(l), d->w_o[l], (size_t)c->H * c->qd});
        }
        for (const Part &p : parts) {
            if (!p.src || (e = cudaMemcpy(p.dst, p.src, sizeof(float) * p.n,
                                          cudaMemcpyHostToDevice)) != cudaSuccess) {
                free_refv2(c);
                return p.src ? cuda_fail(e, "refv2_create: weight upload")
                             : fail(RABBIT_CUDA_ERR_ARGS, "refv2_create: NULL layer weight");
            }
        }
    }
    *out = c;
    return ok();
}

int rabbit_cuda_refv2_fill_synthetic(rabbit_cuda_refv2 *c, uint64_t seed, float sigma) {
    if (!c) return fail(RABBIT_CUDA_ERR_ARGS, "refv2_fill_synthetic: NULL context");
    RB_CUDA(cudaSetDevice(c->device));
    const int blocks = c->ctx->sm_count * 8;
    cudaStream_t s = c->ctx->stream;
    std::lock_guard<std::mutex> g(c->ctx->mu);
    auto fill = [&](float *p, size_t n, float sg, float val, uint64_t k) {
        k_fill_f32<<<blocks, 256, 0, s>>>(p, n, seed * 0x9E3779B97F4A7C15ull + k, sg, val);
    };
    fill(c->embed, (size_t)c->V * c->H, sigma, 0.f, 1);
    fill(c->lm_head, (size_t)c->H * c->V, sigma, 0.f, 2);
    fill(c->final_norm, c->H, 0.f, 1.f, 3);
    for (int l = 0; l < c->L; ++l) {
        fill(c->rms_attn(l), c->H, 0.f, 1.f, 16 + 8 * l);
        fill(c->w_q(l), (size_t)c->qd * c->H, sigma, 0.f, 17 + 8 * l);
        fill(c->w_k(l), (size_t)c->kvd * c->H, sigma, 0.f, 18 + 8 * l);
        fill(c->w_v(l), (size_t)c->kvd * c->H, sigma, 0.f, 19 + 8 * l);
        fill(c->w_o(l), (size_t)c->H * c->qd, sigma, 0.f, 20 + 8 * l);
    }
    RB_CUDA(cudaGetLastError());
    RB_CUDA(cudaStreamSynchronize(s));
    return ok();
}

int rabbit_cuda_refv2_free(rabbit_cuda_refv2 *c) {
    if (c) free_refv2(c);
    return ok();
}

int rabbit_cuda_refv2_reset(rabbit_cuda_refv2 *c) {
    if (!c) return fail(RABBIT_CUDA_ERR_ARGS, "refv2_reset: NULL context");
    c->pos = 0;
    c->len = 0;
    c->stepped = false;
    return ok();
}

int rabbit_cuda_refv2_position(const rabbit_cuda_refv2 *c) { return c ? c->pos : -1; }

int rabbit_cuda_refv2_step(rabbit_cuda_refv2 *c, int token_id, float *logits, float *hidden,
                           int *argmax) {
    return rabbit_cuda_refv2_prefill(c, &token_id, 1, logits, hidden, argmax);
}

int rabbit_cuda_refv2_prefill(rabbit_cuda_refv2 *c, const int *token_ids, int n_tokens,
                              float *logits, float *hidden, int *argmax) {
    if (!c || !token_ids || n_tokens < 1)
        return fail(RABBIT_CUDA_ERR_ARGS, "refv2_prefill: NULL context/ids or no tokens");
    std::lock_guard<std::mutex> g(c->ctx->mu);
    RB_CUDA(cudaSetDevice(c->device));
    cudaStream_t s = c->ctx->stream;
    RB_CUDA(cudaEventRecord(c->ev0, s));
    for (int t = 0; t < n_tokens; ++t) {
        const int st = enqueue_step(c, nullptr, token_ids[t], c->ids, t == n_tokens - 1 && hidden, s);
        if (st != RABBIT_CUDA_OK) return st;
    }
    const int st = finish(c, s, logits, hidden, argmax);
    return st == RABBIT_CUDA_OK ? ok() : st;
}

int rabbit_cuda_refv2_generate(rabbit_cuda_refv2 *c, int n_new, int *out_ids) {
    if (!c || !out_ids || n_new < 1 || n_new > kMaxNew)
        return fail(RABBIT_CUDA_ERR_ARGS, "refv2_generate: need 1..%d tokens", kMaxNew);
    if (!c->stepped) return fail(RABBIT_CUDA_ERR_ARGS, "refv2_generate: no step before it");
    std::lock_guard<std::mutex> g(c->ctx->mu);
    RB_CUDA(cudaSetDevice(c->device));
    cudaStream_t s = c->ctx->stream;
    // ids[0] holds the last step's argmax; step i reads ids[i], writes ids[i + 1]
    RB_CUDA(cudaEventRecord(c->ev0, s));
    for (int i = 0; i < n_new; ++i) {
        const int st = enqueue_step(c, c->ids + i, 0, c->ids + i + 1, false, s);
        if (st != RABBIT_CUDA_OK) return st;
    }
    RB_CUDA(cudaEventRecord(c->ev1, s));
    RB_CUDA(cudaMemcpyAsync(c->ids, c->ids + n_new, sizeof(int), cudaMemcpyDeviceToDevice, s));
    int *pin_ids = reinterpret_cast<int *>(c->pin);
    const int chunk = std::min(n_new, c->V + c->H);  // staging capacity in ints
    int st = RABBIT_CUDA_OK;
    for (int i = 0; i < n_new && st == RABBIT_CUDA_OK; i += chunk) {
        const int m = std::min(chunk, n_new - i);
        RB_CUDA(cudaMemcpyAsync(pin_ids, c->ids + 1 + i, sizeof(int) * m, cudaMemcpyDeviceToHost, s));
        st = check_device_error(c->ctx, s, "refv2_generate");
        if (st == RABBIT_CUDA_OK) memcpy(out_ids + i, pin_ids, sizeof(int) * m);
    }
    if (st == RABBIT_CUDA_OK) RB_CUDA(cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1));
    return st == RABBIT_CUDA_OK ? ok() : st;
}

int rabbit_cuda_refv2_device_ms(const rabbit_cuda_refv2 *c, float *ms) {
    if (!c || !ms) return fail(RABBIT_CUDA_ERR_ARGS, "refv2_device_ms: NULL argument");
    *ms = c->last_ms;
    return ok();
}

}  // extern "C"
