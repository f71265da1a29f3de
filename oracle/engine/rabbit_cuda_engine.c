/* rabbit_cuda_engine.c -- the engine side of the drop-in boundary, built the
 * way a maintainer of the reference engine would add it: this file is
 * appended (#include) to a build-time copy of the engine's src/forward_v2.c,
 * so it sees RefV2Weights, parse_weights, rabbit_v2_max_ctx; patch_engine.py
 * adds one hook call at the top of moe_step (forward_v2.c:362) and one at the
 * top of rabbit_ref_v2_greedy (forward_v2.c:495), and nothing else changes.
 *
 *   moe_step            -> rabbit_cuda_moe_decode on a pool of the model's
 *                          experts (host h in and out, as moe_step's h);
 *   RabbitRefV2Ctx      -> rabbit_cuda_refv2_* (rabbit.h:160-167, declared
 *                          but not implemented by the reference);
 *   rabbit_ref_v2_greedy-> with RABBIT_CUDA_CTX set: the prompt ids made as the
 *                          reference makes them (forward_v2.c:502-511), one
 *                          context prefill and a greedy continuation on the
 *                          device, instead of a re-forward per token.
 * RABBIT_CUDA_OFF set: the hooks step aside (the engine's own C path).
 * Test infrastructure: built by oracle/engine/Makefile into oracle/_ref;
 * nothing here is part of librabbit_cuda. */
#include "rabbit_cuda.h"

static rabbit_cuda_moe *rc_pool;
static const RabbitModel *rc_pool_model;

/* One pool per model: every layer's records uploaded once, from the model's
 * host map of the expert table. */
static rabbit_cuda_moe *rabbit_cuda_pool_for(const RabbitModel *m, const RefV2Weights *w) {
    if (rc_pool && rc_pool_model == m) return rc_pool;
    if (rc_pool) {
        rabbit_cuda_moe_free(rc_pool);
        rc_pool = NULL;
    }
    uint32_t n_shared = 0;
    memcpy(&n_shared, m->hdr.reserved + 12, 4);
    rabbit_cuda_moe_desc d;
    memset(&d, 0, sizeof d);
    d.n_layers = w->n_layers;
    d.hidden = w->hidden;
    d.n_experts = w->n_experts;
    d.experts_per_token = w->top_k;
    d.inter = w->inter;
    d.n_shared = (n_shared > 0 && n_shared <= 64) ? (int)n_shared : 0;
    d.expert_quant = (int)m->hdr.expert_quant;
    d.expert_size = m->expert_size;
    d.n_records = m->n_expert_records;
    d.experts_per_layer = m->experts_per_layer;
    d.experts_shared = m->experts_shared;
    d.expert_map = m->expert_map;
    d.rms_ffn = w->rms_ffn;
    d.w_router = w->w_router;
    rabbit_cuda_moe *p = NULL;
    int st = rabbit_cuda_moe_create(&d, 0, &p);
    if (st == RABBIT_CUDA_OK) st = rabbit_cuda_moe_upload(p, 0, w->n_layers);
    if (st == RABBIT_CUDA_OK) st = rabbit_cuda_moe_sync(p);
    if (st != RABBIT_CUDA_OK) {
        fprintf(stderr, "rabbit_cuda: expert pool: %s\n", rabbit_cuda_last_error());
        rabbit_cuda_moe_free(p);
        return NULL;
    }
    rc_pool = p;
    rc_pool_model = m;
    return p;
}

/* moe_step's hook: 1 when the block ran on the GPU (h += experts), 0 to let
 * the C body run. */
static int rabbit_cuda_hook_moe_step(const RabbitModel *m, const RefV2Weights *w, int layer,
                                     float *h) {
    if (getenv("RABBIT_CUDA_OFF")) return 0;
    rabbit_cuda_moe *p = rabbit_cuda_pool_for(m, w);
    if (!p) return 0;
    if (rabbit_cuda_moe_decode(p, layer, h, h, NULL, NULL, NULL) != RABBIT_CUDA_OK) {
        fprintf(stderr, "rabbit_cuda: moe_step layer %d: %s\n", layer, rabbit_cuda_last_error());
        return 0;
    }
    return 1;
}

/* ---------------------------------------------------- RabbitRefV2Ctx -- */
struct RabbitRefV2Ctx {
    rabbit_cuda_moe *pool;
    rabbit_cuda_refv2 *dev;
    int vocab;
};

RabbitRefV2Ctx *rabbit_ref_v2_ctx_create(RabbitModel *m) {
    RefV2Weights w;
    memset(&w, 0, sizeof w);
    if (!m || parse_weights(m, &w) != 0) return NULL;
    RabbitRefV2Ctx *c = (RabbitRefV2Ctx *)calloc(1, sizeof *c);
    if (!c) return NULL;
    c->pool = rabbit_cuda_pool_for(m, &w);
    rabbit_cuda_dense_desc d;
    memset(&d, 0, sizeof d);
    d.n_layers = w.n_layers;
    d.hidden = w.hidden;
    d.vocab = w.vocab;
    d.n_heads = w.n_heads;
    d.n_kv_heads = w.n_kv_heads;
    d.head_dim = w.head_dim;
    d.max_ctx = rabbit_v2_max_ctx();
    d.embed = w.embed;
    d.lm_head = w.lm_head;
    d.final_norm = w.final_norm;
    d.rms_attn = (const float *const *)w.rms_attn;
    d.w_q = (const float *const *)w.w_q;
    d.w_k = (const float *const *)w.w_k;
    d.w_v = (const float *const *)w.w_v;
    d.w_o = (const float *const *)w.w_o;
    if (!c->pool || rabbit_cuda_refv2_create(&d, c->pool, &c->dev) != RABBIT_CUDA_OK) {
        fprintf(stderr, "rabbit_cuda: ref-v2 context: %s\n", rabbit_cuda_last_error());
        free(c);
        return NULL;
    }
    c->vocab = w.vocab;
    return c;
}

void rabbit_ref_v2_ctx_free(RabbitRefV2Ctx *c) {
    if (!c) return;
    rabbit_cuda_refv2_free(c->dev); /* the pool stays: it belongs to the model */
    free(c);
}

void rabbit_ref_v2_ctx_reset(RabbitRefV2Ctx *c) {
    if (c) rabbit_cuda_refv2_reset(c->dev);
}

int rabbit_ref_v2_ctx_prefill(RabbitRefV2Ctx *c, const int *ids, int n, float *out_logits) {
    if (!c) return -1;
    return rabbit_cuda_refv2_prefill(c->dev, ids, n, out_logits, NULL, NULL) == RABBIT_CUDA_OK
               ? 0
               : -1;
}

int rabbit_ref_v2_ctx_step(RabbitRefV2Ctx *c, int id, float *out_logits) {
    if (!c) return -1;
    return rabbit_cuda_refv2_step(c->dev, id, out_logits, NULL, NULL) == RABBIT_CUDA_OK ? 0 : -1;
}

/* rabbit_ref_v2_greedy's hook: with RABBIT_CUDA_CTX set, the ids through the
 * context (the same ids while prompt + n_new <= max_ctx: the positions and
 * the KV cache are those of the re-forward); -2 to let the C body run. */
static int rabbit_cuda_hook_greedy(RabbitModel *m, const char *prompt, int n_new, int *out_ids,
                                   int max_ids) {
    if (!getenv("RABBIT_CUDA_CTX") || getenv("RABBIT_CUDA_OFF")) return -2;
    if (!m || !prompt || !out_ids || max_ids < 1) return -1;
    RefV2Weights w;
    memset(&w, 0, sizeof w);
    if (parse_weights(m, &w) != 0) return -1;
    int n = rabbit_tokenize(prompt, out_ids, max_ids - n_new - 1);
    if (n <= 0) {
        out_ids[0] = 1;
        n = 1;
    }
    for (int i = 0; i < n; i++) {
        if (out_ids[i] < 0) out_ids[i] = 0;
        out_ids[i] %= w.vocab;
    }
    int take = n_new < max_ids - n ? n_new : max_ids - n;
    if (take <= 0) return n;
    RabbitRefV2Ctx *c = rabbit_ref_v2_ctx_create(m);
    if (!c) return -1;
    int am = -1, st = rabbit_cuda_refv2_prefill(c->dev, out_ids, n, NULL, NULL, &am);
    if (st == RABBIT_CUDA_OK) {
        out_ids[n] = am;  /* the first new id: argmax after the prompt */
        if (take > 1) st = rabbit_cuda_refv2_generate(c->dev, take - 1, out_ids + n + 1);
    }
    if (st != RABBIT_CUDA_OK) {
        fprintf(stderr, "rabbit_cuda: greedy: %s\n", rabbit_cuda_last_error());
        rabbit_ref_v2_ctx_free(c);
        return -1;
    }
    rabbit_ref_v2_ctx_free(c);
    return n + take;
}
