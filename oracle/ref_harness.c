/*
 * ref_harness.c -- exposes the reference engine's own routines for pinning.
 *
 * TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile into oracle/_ref/ from
 * the reference sources where they lie (nothing is copied into this repo).
 * forward_v2.c keeps rmsnorm, select_top_k, expert_swiglu, moe_step and
 * attention_step `static`, so this translation unit #includes that file and
 * wraps those functions behind plain-pointer entry points (ref_*), the same
 * shapes as the oracle's orc_* functions. quant.c's public functions
 * (rabbit_gemv_int4_grouped, rabbit_dequant_int4_grouped, ...) are linked
 * from the reference object directly.
 */
#include REF_FORWARD_V2_C

void ref_rmsnorm(const float *x, const float *w, float *out, int n) { rmsnorm(x, w, out, n); }

void ref_gemv_f32(const float *W, const float *x, float *y, int out_dim, int in_dim) {
    gemv_f32(W, x, y, out_dim, in_dim);
}

void ref_select_top_k(const float *scores, int n, int k, int *ids, float *weights) {
    select_top_k(scores, n, k, ids, weights);
}

void ref_apply_rope_head(float *x, int head_dim, int pos) { apply_rope_head(x, head_dim, pos); }

/* A RabbitModel view over one layer's records: experts_per_layer = E + S,
 * n_layers = 1, so rabbit_expert_ptr_layer(m, 0, id) = records + id*size. */
static void ref_model_view(RabbitModel *m, int H, int E, int top_k, int inter, int n_shared,
                           int quant, int n_records, size_t expert_size, const uint8_t *records) {
    memset(m, 0, sizeof(*m));
    m->hdr.hidden_dim = (uint32_t)H;
    m->hdr.n_experts = (uint32_t)E;
    m->hdr.experts_per_token = (uint32_t)top_k;
    m->hdr.expert_dim = (uint32_t)inter;
    m->hdr.expert_quant = (uint32_t)quant;
    m->hdr.n_layers = 1;
    uint32_t s = (uint32_t)n_shared;
    memcpy(m->hdr.reserved + 12, &s, 4);
    m->n_layers = 1;
    m->hidden_dim = H;
    m->num_experts = E;
    m->experts_per_token = top_k;
    m->expert_size = expert_size;
    m->n_expert_records = n_records;
    m->experts_per_layer = n_records;
    m->experts_shared = 0;
    m->expert_fd = -1;
    m->expert_map = (void *)records;
}

void ref_expert_swiglu(const uint8_t *record, size_t expert_size, int quant, const float *xn,
                       float *delta, int H, int inter, float weight) {
    RabbitModel m;
    ref_model_view(&m, H, 1, 1, inter, 0, quant, 1, expert_size, record);
    expert_swiglu(&m, 0, 0, xn, delta, H, inter, weight);
}

void ref_moe_step(int H, int E, int top_k, int inter, int n_shared, int quant, int n_records,
                  size_t expert_size, const uint8_t *records, const float *rms_ffn,
                  const float *w_router, float *h) {
    RabbitModel m;
    ref_model_view(&m, H, E, top_k, inter, n_shared, quant, n_records, expert_size, records);
    RefV2Weights w;
    memset(&w, 0, sizeof(w));
    w.n_layers = 1;
    w.hidden = H;
    w.n_experts = E;
    w.top_k = top_k > 0 ? top_k : 2;
    w.inter = inter;
    w.rms_ffn[0] = rms_ffn;
    w.w_router[0] = w_router;
    moe_step(&m, &w, 0, h);
}

void ref_attention_step(int H, int nh, int nkv, int hd, const float *rms_attn, const float *w_q,
                        const float *w_k, const float *w_v, const float *w_o, float *h,
                        float *kv_k, float *kv_v, int *kv_len, int kv_max, int pos) {
    RefV2Weights w;
    memset(&w, 0, sizeof(w));
    w.n_layers = 1;
    w.hidden = H;
    w.n_heads = nh;
    w.n_kv_heads = nkv;
    w.head_dim = hd;
    w.q_dim = nh * hd;
    w.kv_dim = nkv * hd;
    w.rms_attn[0] = rms_attn;
    w.w_q[0] = w_q;
    w.w_k[0] = w_k;
    w.w_v[0] = w_v;
    w.w_o[0] = w_o;
    RefV2KV kv = {kv_k, kv_v, *kv_len, kv_max};
    attention_step(&w, 0, h, &kv, pos);
    *kv_len = kv.len;
}

void ref_logits(const float *lm_head, const float *h, float *logits, int H, int V) {
    RefV2Weights w;
    memset(&w, 0, sizeof(w));
    w.hidden = H;
    w.vocab = V;
    w.lm_head = lm_head;
    logits_from_hidden(&w, h, logits);
}
