/*
 * rabbit_oracle.c -- CPU oracle for the routed-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Each function restates one reference routine of Stanley03-arch/Rabbit
 * v0.4.28, cited by file:line, keeping its fp32 evaluation order: every sum is
 * a left-to-right serial fp32 sum, products are rounded before they are added
 * (build with -ffp-contract=off), and libm's expf/sqrtf/powf/cosf/sinf are
 * called exactly where the reference calls them.
 */
#include "rabbit_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ int4 -- */

/* quant.c:190-195: header word + one fp32 scale per group + two nibbles/byte. */
int orc_int4_grouped_nbytes(int n, int group_size) {
    if (n <= 0) return 0;
    int gs = group_size > 0 ? group_size : ORC_INT4_GROUP;
    int groups = (n + gs - 1) / gs;
    return 4 + 4 * groups + (n + 1) / 2;
}

static int orc_clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* quant.c:76-121: scale = max|x|/7 + 1e-8 per group; q = clamp(rint(x/s), -8, 7);
 * byte = (q_even + 8) | (q_odd + 8) << 4. */
int orc_pack_int4_grouped(const float *src, int n, int group_size, uint8_t *dst, int dst_cap) {
    if (!src || !dst || n <= 0) return -1;
    int gs = group_size > 0 ? group_size : ORC_INT4_GROUP;
    int groups = (n + gs - 1) / gs;
    int total = 4 + 4 * groups + (n + 1) / 2;
    if (dst_cap < total) return -1;

    uint32_t gs_word = (uint32_t)gs;
    memcpy(dst, &gs_word, 4);
    float *scale = (float *)(dst + 4);
    uint8_t *nib = dst + 4 + 4 * groups;

    for (int g = 0; g < groups; g++) {
        int end = (g + 1) * gs < n ? (g + 1) * gs : n;
        float amax = 0.0f;
        for (int i = g * gs; i < end; i++) {
            float a = fabsf(src[i]);
            if (a > amax) amax = a;
        }
        scale[g] = amax / 7.0f + 1e-8f;
    }
    for (int i = 0; i < n; i += 2) {
        int q0 = orc_clampi((int)lrintf(src[i] / scale[i / gs]), -8, 7);
        int q1 = 0;
        if (i + 1 < n) q1 = orc_clampi((int)lrintf(src[i + 1] / scale[(i + 1) / gs]), -8, 7);
        nib[i / 2] = (uint8_t)((q0 + 8) | ((q1 + 8) << 4));
    }
    return total;
}

/* Element i of a grouped blob: nibble (i odd -> high half), minus the +8 bias. */
static inline int orc_nibble_q(const uint8_t *nib, int i) {
    uint8_t b = nib[i >> 1];
    return (int)((i & 1) ? (b >> 4) : (b & 0x0F)) - 8;
}

/* quant.c:123-142: dst[i] = (float)q_i * scale[i / group_size]; group_size
 * must be 1..4096 else -1. */
int orc_dequant_int4_grouped(const uint8_t *blob, float *dst, int n) {
    if (!blob || !dst || n <= 0) return -1;
    uint32_t gs;
    memcpy(&gs, blob, 4);
    if (gs == 0 || gs > 4096) return -1;
    int groups = (n + (int)gs - 1) / (int)gs;
    const float *scale = (const float *)(blob + 4);
    const uint8_t *nib = blob + 4 + 4 * groups;
    for (int i = 0; i < n; i++) dst[i] = (float)orc_nibble_q(nib, i) * scale[i / (int)gs];
    return 0;
}

/* quant.c:152-188: per output row, dequantise the row (flat index o*in+i, so
 * groups may straddle rows when in % group_size != 0), then a serial fp32 dot.
 * An invalid group size writes zeros. */
void orc_gemv_int4_grouped(const uint8_t *W, const float *x, float *y, int out_dim, int in_dim) {
    if (!W || !x || !y || out_dim <= 0 || in_dim <= 0) return;
    uint32_t gs;
    memcpy(&gs, W, 4);
    if (gs == 0 || gs > 4096) {
        memset(y, 0, sizeof(float) * (size_t)out_dim);
        return;
    }
    int n = out_dim * in_dim;
    int groups = (n + (int)gs - 1) / (int)gs;
    const float *scale = (const float *)(W + 4);
    const uint8_t *nib = W + 4 + 4 * groups;
    float *w_row = (float *)malloc(sizeof(float) * (size_t)in_dim);
    if (!w_row) return;
    for (int o = 0; o < out_dim; o++) {
        int base = o * in_dim;
        for (int i = 0; i < in_dim; i++) {
            int flat = base + i;
            w_row[i] = (float)orc_nibble_q(nib, flat) * scale[flat / (int)gs];
        }
        float acc = 0.0f;
        for (int i = 0; i < in_dim; i++) acc += w_row[i] * x[i];
        y[o] = acc;
    }
    free(w_row);
}

/* ------------------------------------------------------------ fp32 bits -- */

/* forward_v2.c:61-69 */
void orc_rmsnorm(const float *x, const float *w, float *out, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss /= (float)n;
    float r = 1.0f / sqrtf(ss + ORC_EPS);
    for (int i = 0; i < n; i++) out[i] = x[i] * r * w[i];
}

/* forward_v2.c:71-79 */
void orc_gemv_f32(const float *W, const float *x, float *y, int out_dim, int in_dim) {
    for (int o = 0; o < out_dim; o++) {
        const float *w = W + (size_t)o * (size_t)in_dim;
        float acc = 0.0f;
        for (int i = 0; i < in_dim; i++) acc += w[i] * x[i];
        y[o] = acc;
    }
}

/* forward_v2.c:81-90: int8 rows, per-matrix scale applied after the dot. */
static void orc_gemv_int8(const int8_t *W, float scale, const float *x, float *y,
                          int out_dim, int in_dim) {
    for (int o = 0; o < out_dim; o++) {
        const int8_t *w = W + (size_t)o * (size_t)in_dim;
        float acc = 0.0f;
        for (int i = 0; i < in_dim; i++) acc += (float)w[i] * x[i];
        y[o] = acc * scale;
    }
}

/* forward_v2.c:248-278: keep a descending list seeded with (-1, -1e30); an
 * expert is inserted before the first entry it strictly beats, so on ties the
 * lower index stays first. Then softmax over the k kept scores. */
void orc_select_top_k(const float *scores, int n, int k, int *ids, float *weights) {
    for (int i = 0; i < k; i++) {
        ids[i] = -1;
        weights[i] = -1e30f;
    }
    for (int e = 0; e < n; e++) {
        float s = scores[e];
        int slot = 0;
        while (slot < k && !(s > weights[slot])) slot++;
        if (slot == k) continue;
        for (int j = k - 1; j > slot; j--) {
            ids[j] = ids[j - 1];
            weights[j] = weights[j - 1];
        }
        ids[slot] = e;
        weights[slot] = s;
    }
    float m = weights[0];
    for (int i = 1; i < k; i++)
        if (weights[i] > m) m = weights[i];
    float z = 0.0f;
    for (int i = 0; i < k; i++) {
        weights[i] = expf(weights[i] - m);
        z += weights[i];
    }
    if (z > 0.0f)
        for (int i = 0; i < k; i++) weights[i] /= z;
}

/* ------------------------------------------------------------- experts -- */

/* forward_v2.c:327-331: mid = (g * sigmoid(g)) * up */
static void orc_silu_mul(const float *gate, const float *up, float *mid, int n) {
    for (int i = 0; i < n; i++) {
        float g = gate[i];
        float sg = 1.0f / (1.0f + expf(-g));
        mid[i] = (g * sg) * up[i];
    }
}

/* forward_v2.c:280-360. Record = gate [I,H] | up [I,H] | down [H,I]. */
int orc_expert_swiglu(const uint8_t *rec, size_t expert_size, int quant,
                      const float *xn, float *delta, int H, int inter, float weight) {
    if (!rec) return 0;
    size_t mat = (size_t)inter * (size_t)H;
    float *gate = (float *)calloc((size_t)inter, sizeof(float));
    float *up = (float *)calloc((size_t)inter, sizeof(float));
    float *mid = (float *)calloc((size_t)inter, sizeof(float));
    float *down = (float *)calloc((size_t)H, sizeof(float));
    int used = 0;
    if (!gate || !up || !mid || !down) goto done;

    if (quant == 0) {
        if (expert_size < (2 * mat + (size_t)H * (size_t)inter) * sizeof(float)) goto done;
        const float *w = (const float *)rec;
        orc_gemv_f32(w, xn, gate, inter, H);
        orc_gemv_f32(w + mat, xn, up, inter, H);
        orc_silu_mul(gate, up, mid, inter);
        orc_gemv_f32(w + 2 * mat, mid, down, H, inter);
    } else if (quant == 4) {
        /* offsets assume the default group of 32, as the reference does */
        int nb_gu = orc_int4_grouped_nbytes((int)mat, ORC_INT4_GROUP);
        int nb_d = orc_int4_grouped_nbytes(H * inter, ORC_INT4_GROUP);
        if (expert_size < (size_t)(2 * nb_gu + nb_d)) goto done;
        orc_gemv_int4_grouped(rec, xn, gate, inter, H);
        orc_gemv_int4_grouped(rec + nb_gu, xn, up, inter, H);
        orc_silu_mul(gate, up, mid, inter);
        orc_gemv_int4_grouped(rec + 2 * (size_t)nb_gu, mid, down, H, inter);
    } else {
        size_t one = 4 + mat; /* f32 scale + int8 payload */
        if (expert_size < 3 * one) goto done;
        float sg, su, sd;
        memcpy(&sg, rec, 4);
        orc_gemv_int8((const int8_t *)(rec + 4), sg, xn, gate, inter, H);
        memcpy(&su, rec + one, 4);
        orc_gemv_int8((const int8_t *)(rec + one + 4), su, xn, up, inter, H);
        orc_silu_mul(gate, up, mid, inter);
        memcpy(&sd, rec + 2 * one, 4);
        orc_gemv_int8((const int8_t *)(rec + 2 * one + 4), sd, mid, down, H, inter);
    }
    for (int i = 0; i < H; i++) delta[i] += weight * down[i];
    used = 1;
done:
    free(gate);
    free(up);
    free(mid);
    free(down);
    return used;
}

/* forward_v2.c:362-402 */
int orc_moe_step(const orc_moe_layer *L, float *h, int *ids_out, float *weights_out) {
    int H = L->hidden, E = L->n_experts;
    int k = L->experts_per_token > 0 ? L->experts_per_token : 2;
    if (k > E) k = E;
    if (k > 8) k = 8;
    float *xn = (float *)malloc(sizeof(float) * (size_t)H);
    float *scores = (float *)malloc(sizeof(float) * (size_t)(E > 0 ? E : 1));
    float *delta = (float *)calloc((size_t)H, sizeof(float));
    int ids[8];
    float wts[8];
    if (!xn || !scores || !delta) {
        k = 0;
        goto done;
    }
    orc_rmsnorm(h, L->rms_ffn, xn, H);
    orc_gemv_f32(L->w_router, xn, scores, E, H);
    orc_select_top_k(scores, E, k, ids, wts);

    for (int i = 0; i < k; i++) {
        int id = ids[i];
        if (id < 0 || id >= L->n_records) continue;
        orc_expert_swiglu(L->records + (size_t)id * L->expert_size, L->expert_size, L->quant,
                          xn, delta, H, L->inter, wts[i]);
    }
    if (L->n_shared > 0 && L->n_shared <= 64) {
        for (int s = 0; s < L->n_shared; s++) {
            int id = E + s;
            if (id >= L->n_records) continue;
            orc_expert_swiglu(L->records + (size_t)id * L->expert_size, L->expert_size,
                              L->quant, xn, delta, H, L->inter, 1.0f);
        }
    }
    for (int i = 0; i < H; i++) h[i] += delta[i];
    if (ids_out)
        for (int i = 0; i < k; i++) ids_out[i] = ids[i];
    if (weights_out)
        for (int i = 0; i < k; i++) weights_out[i] = wts[i];
done:
    free(xn);
    free(scores);
    free(delta);
    return k;
}

/* ----------------------------------------------------------- attention -- */

/* forward_v2.c:92-104: rotate interleaved pairs (2i, 2i+1) by pos * 10000^(-i/half). */
void orc_apply_rope_head(float *x, int head_dim, int pos) {
    int half = head_dim / 2;
    for (int i = 0; i < half; i++) {
        float inv_freq = 1.0f / powf(10000.0f, (float)i / (float)half);
        float ang = (float)pos * inv_freq;
        float c = cosf(ang), s = sinf(ang);
        float a = x[2 * i], b = x[2 * i + 1];
        x[2 * i] = a * c - b * s;
        x[2 * i + 1] = a * s + b * c;
    }
}

/* forward_v2.c:171-246 */
void orc_attention_step(const orc_attn_layer *A, float *h, orc_kv *kv, int pos) {
    int H = A->hidden, nh = A->n_heads, nkv = A->n_kv_heads, hd = A->head_dim;
    int qd = nh * hd, kvd = nkv * hd;
    int group = nh / nkv;
    if (group < 1) group = 1;
    float *xn = (float *)malloc(sizeof(float) * (size_t)H);
    float *q = (float *)malloc(sizeof(float) * (size_t)qd);
    float *k = (float *)malloc(sizeof(float) * (size_t)kvd);
    float *v = (float *)malloc(sizeof(float) * (size_t)kvd);
    float *ctx = (float *)calloc((size_t)qd, sizeof(float));
    float *o = (float *)malloc(sizeof(float) * (size_t)H);
    float *p = (float *)malloc(sizeof(float) * (size_t)(kv->max_len > 0 ? kv->max_len : 1));
    if (!xn || !q || !k || !v || !ctx || !o || !p) goto done;

    orc_rmsnorm(h, A->rms_attn, xn, H);
    orc_gemv_f32(A->w_q, xn, q, qd, H);
    orc_gemv_f32(A->w_k, xn, k, kvd, H);
    orc_gemv_f32(A->w_v, xn, v, kvd, H);
    for (int hh = 0; hh < nh; hh++) orc_apply_rope_head(q + hh * hd, hd, pos);
    for (int hh = 0; hh < nkv; hh++) orc_apply_rope_head(k + hh * hd, hd, pos);

    if (kv->len < kv->max_len) { /* a full window silently stops appending */
        memcpy(kv->k + (size_t)kv->len * kvd, k, sizeof(float) * (size_t)kvd);
        memcpy(kv->v + (size_t)kv->len * kvd, v, sizeof(float) * (size_t)kvd);
        kv->len++;
    }
    float scale = 1.0f / sqrtf((float)hd);
    for (int hh = 0; hh < nh; hh++) {
        const float *qh = q + hh * hd;
        int off = (hh / group) * hd;
        for (int t = 0; t < kv->len; t++) {
            const float *kt = kv->k + (size_t)t * kvd + off;
            float d = 0.0f;
            for (int i = 0; i < hd; i++) d += qh[i] * kt[i];
            p[t] = d * scale;
        }
        float m = p[0];
        for (int t = 1; t < kv->len; t++)
            if (p[t] > m) m = p[t];
        float z = 0.0f;
        for (int t = 0; t < kv->len; t++) {
            p[t] = expf(p[t] - m);
            z += p[t];
        }
        if (z > 0.0f)
            for (int t = 0; t < kv->len; t++) p[t] /= z;
        float *ch = ctx + hh * hd;
        for (int t = 0; t < kv->len; t++) {
            const float *vt = kv->v + (size_t)t * kvd + off;
            for (int i = 0; i < hd; i++) ch[i] += p[t] * vt[i];
        }
    }
    orc_gemv_f32(A->w_o, ctx, o, H, qd);
    for (int i = 0; i < H; i++) h[i] += o[i];
done:
    free(xn);
    free(q);
    free(k);
    free(v);
    free(ctx);
    free(o);
    free(p);
}

/* forward_v2.c:404-413 (lm_head stored [H, V]) */
void orc_logits(const float *lm_head, const float *h, float *logits, int H, int V) {
    for (int v = 0; v < V; v++) {
        float acc = 0.0f;
        for (int i = 0; i < H; i++) acc += lm_head[(size_t)i * (size_t)V + v] * h[i];
        logits[v] = acc;
    }
}

/* forward_v2.c:415-421: first maximum wins */
int orc_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

/* ------------------------------------------------ legacy per-tensor experts -- */

/* moe.c:7-16: y[o] += weight * (sum_i row[i] x[i]) * scale */
static void orc_legacy_gemv_int8(const int8_t *W, float scale, const float *x, float *y,
                                 int out_dim, int in_dim, float weight) {
    for (int o = 0; o < out_dim; o++) {
        const int8_t *row = W + (size_t)o * in_dim;
        float sum = 0.0f;
        for (int i = 0; i < in_dim; i++) sum += (float)row[i] * x[i];
        y[o] += weight * sum * scale;
    }
}

/* moe.c:18-35: rows of (in_dim + 1) / 2 bytes, element 2j = low nibble of
 * byte j, 2j + 1 = its high nibble, value nibble - 8 */
static void orc_legacy_gemv_int4(const uint8_t *W, float scale, const float *x, float *y,
                                 int out_dim, int in_dim, float weight) {
    const int in_bytes = (in_dim + 1) / 2;
    for (int o = 0; o < out_dim; o++) {
        const uint8_t *row = W + (size_t)o * in_bytes;
        float sum = 0.0f;
        for (int i = 0; i < in_dim; i += 2) {
            const uint8_t b = row[i / 2];
            sum += (float)((int)(b & 0x0F) - 8) * x[i];
            if (i + 1 < in_dim) sum += (float)((int)((b >> 4) & 0x0F) - 8) * x[i + 1];
        }
        y[o] += weight * sum * scale;
    }
}

/* moe.c:137-143: a stored scale that is not a positive finite number reads as 1/127 */
static float orc_legacy_scale(const uint8_t *p) {
    float s;
    memcpy(&s, p, 4);
    return (s > 0.0f && isfinite(s)) ? s : 1.0f / 127.0f;
}

/* moe.c:119-224 */
void orc_legacy_apply_expert(const uint8_t *bytes, size_t size, int quant, int hidden_dim,
                             int expert_dim, float *hidden, float weight) {
    if (!bytes || !hidden || hidden_dim <= 0) return;
    const int H = hidden_dim;
    float *delta = (float *)calloc((size_t)H, sizeof(float));
    if (!delta) return;
    int inter = expert_dim > 0 ? expert_dim : H * 2;       /* moe.c:126-128 */
    if (inter > H * 4) inter = H * 2;
    if (inter < 1) inter = H;
    const size_t mat = (size_t)inter * (size_t)H;
    const size_t payload3 = quant == 4 ? (mat + 1) / 2 : mat;
    if (size >= 3 * (4 + payload3) && inter > 0) {          /* moe.c:135-181 */
        float *gate = (float *)calloc((size_t)inter, sizeof(float));
        float *up = (float *)calloc((size_t)inter, sizeof(float));
        float *mid = (float *)calloc((size_t)inter, sizeof(float));
        const uint8_t *p = bytes;
        if (gate && up && mid) {
            for (int part = 0; part < 3; part++) {
                float scale = 1.0f / 127.0f;
                if (size - (size_t)(p - bytes) >= 4) {
                    scale = orc_legacy_scale(p);
                    p += 4;
                }
                const uint8_t *W = p;
                p += payload3;
                if (part < 2) {
                    float *y = part == 0 ? gate : up;
                    if (quant == 4) orc_legacy_gemv_int4(W, scale, hidden, y, inter, H, 1.0f);
                    else orc_legacy_gemv_int8((const int8_t *)W, scale, hidden, y, inter, H, 1.0f);
                } else {
                    orc_silu_mul(gate, up, mid, inter);
                    if (quant == 4) orc_legacy_gemv_int4(W, scale, mid, delta, H, inter, weight);
                    else orc_legacy_gemv_int8((const int8_t *)W, scale, mid, delta, H, inter, weight);
                }
            }
            for (int i = 0; i < H; i++) hidden[i] += delta[i];
        }
        free(gate);
        free(up);
        free(mid);
        free(delta);
        return;
    }
    /* moe.c:183-220: one square matrix, or the raw bytes */
    float scale = 1.0f / 127.0f;
    const uint8_t *W = bytes;
    size_t payload = size;
    if (size >= 4 + (size_t)H) {
        scale = orc_legacy_scale(bytes);
        W = bytes + 4;
        payload = size - 4;
    }
    const float w = weight * 0.05f;
    if (quant == 4) {
        if (payload >= (size_t)H * (size_t)((H + 1) / 2))
            orc_legacy_gemv_int4(W, scale, hidden, delta, H, H, w);
    } else {
        const size_t need = (size_t)H * (size_t)H;
        if (payload >= need) {
            orc_legacy_gemv_int8((const int8_t *)W, scale, hidden, delta, H, H, w);
        } else if (size >= need) {
            orc_legacy_gemv_int8((const int8_t *)bytes, 1.0f / 127.0f, hidden, delta, H, H, w);
        } else {
            const int usable = (int)(size < (size_t)H ? size : (size_t)H);
            for (int i = 0; i < usable; i++) {
                const float v = ((float)bytes[i] - 128.0f) / 128.0f;
                delta[i] = weight * v * 0.1f;
            }
        }
    }
    for (int i = 0; i < H; i++) hidden[i] += delta[i];
    free(delta);
}
