/*
 * rabbit_oracle.h -- CPU oracle for the routed-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * engine's (Stanley03-arch/Rabbit v0.4.28) arithmetic for the group-32 int4
 * matvec, the SwiGLU expert FFN, top-k routing and the surrounding ref-v2
 * decode step. It keeps the reference's fp32 operation order, so with the same
 * compiler flags its outputs are bit-identical to the reference's.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
 * it, and only as the checker. The product library never links it.
 */
#ifndef RABBIT_ORACLE_H
#define RABBIT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_INT4_GROUP 32
#define ORC_EPS 1e-5f

/* quant.c:190-195 */
int  orc_int4_grouped_nbytes(int n, int group_size);
/* quant.c:76-121 */
int  orc_pack_int4_grouped(const float *src, int n, int group_size, uint8_t *dst, int dst_cap);
/* quant.c:123-142 */
int  orc_dequant_int4_grouped(const uint8_t *blob, float *dst, int n);
/* quant.c:152-188 */
void orc_gemv_int4_grouped(const uint8_t *W, const float *x, float *y, int out_dim, int in_dim);

/* forward_v2.c:61-69 */
void orc_rmsnorm(const float *x, const float *w, float *out, int n);
/* forward_v2.c:71-79 */
void orc_gemv_f32(const float *W, const float *x, float *y, int out_dim, int in_dim);
/* forward_v2.c:248-278 (same algorithm as moe.c:37-71) */
void orc_select_top_k(const float *scores, int n, int k, int *ids, float *weights);

/* forward_v2.c:280-360: adds weight * W2(silu(W1 xn) * (W3 xn)) into delta.
 * Returns 1 if the expert contributed, 0 if the record was too small. */
int  orc_expert_swiglu(const uint8_t *record, size_t expert_size, int quant,
                       const float *xn, float *delta, int H, int inter, float weight);

/* One layer's MoE block, as moe_step sees it (forward_v2.c:362-402). */
typedef struct {
    int hidden;             /* H */
    int n_experts;          /* routed experts E (router width) */
    int experts_per_token;  /* header value; <=0 means 2 (forward_v2.c:113) */
    int inter;              /* expert FFN width I */
    int n_shared;           /* reserved[12..15]; used when 0 < S <= 64 */
    int quant;              /* expert_quant: 0 f32, 4 group-int4, else int8 */
    int n_records;          /* records present for this layer (ids >= are skipped) */
    size_t expert_size;     /* bytes per record */
    const uint8_t *records; /* this layer's records, E routed then S shared */
    const float *rms_ffn;   /* [H] */
    const float *w_router;  /* [E, H] */
} orc_moe_layer;

/* forward_v2.c:362-402. h is updated in place. ids/weights (8 each, may be
 * NULL) receive the routing decision; returns k actually used. */
int  orc_moe_step(const orc_moe_layer *L, float *h, int *ids_out, float *weights_out);

/* forward_v2.c:92-104 */
void orc_apply_rope_head(float *x, int head_dim, int pos);

/* Dense per-layer attention weights (forward_v2.c:159-167 layout). */
typedef struct {
    int hidden, n_heads, n_kv_heads, head_dim;
    const float *rms_attn;  /* [H] */
    const float *w_q;       /* [nh*hd, H] */
    const float *w_k;       /* [nkv*hd, H] */
    const float *w_v;       /* [nkv*hd, H] */
    const float *w_o;       /* [H, nh*hd] */
} orc_attn_layer;

/* KV cache for one layer: k, v are [max_len, kv_dim]. */
typedef struct {
    float *k;
    float *v;
    int len;
    int max_len;
} orc_kv;

/* forward_v2.c:171-246 */
void orc_attention_step(const orc_attn_layer *A, float *h, orc_kv *kv, int pos);

/* forward_v2.c:404-413: logits[v] = sum_i lm_head[i*V+v] * h[i] */
void orc_logits(const float *lm_head, const float *h, float *logits, int H, int V);

/* forward_v2.c:415-421 */
int  orc_argmax(const float *x, int n);

/* The legacy per-tensor expert of moe.c:119-224 (apply_expert): a record of
 * three [f32 scale | int4 or int8 payload] matrices (gate, up, down; quant 4
 * is int4 with rows of (in + 1) / 2 bytes, any other value int8), or, for a
 * record too small for that, the square fallback (moe.c:183-220). Adds the
 * expert's output times `weight` into hidden[hidden_dim]. expert_dim is the
 * header's expert_dim (0: 2 * hidden_dim, moe.c:126-128). */
void orc_legacy_apply_expert(const uint8_t *record, size_t expert_size, int quant, int hidden_dim,
                             int expert_dim, float *hidden, float weight);

#ifdef __cplusplus
}
#endif
#endif
