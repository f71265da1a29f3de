/*
 * ref_harness_moe.c -- exposes the reference engine's legacy per-tensor
 * expert (src/moe.c:119-224, apply_expert, `static` there) for pinning.
 *
 * TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile into oracle/_ref/ from
 * the reference sources where they lie (nothing is copied into this repo):
 * this translation unit #includes moe.c and calls apply_expert on a
 * RabbitModel view that carries only what it reads.
 */
#include REF_MOE_C

void ref_legacy_apply_expert(const uint8_t *record, size_t expert_size, int quant, int hidden_dim,
                             int expert_dim, float *hidden, float weight) {
    RabbitModel m;
    memset(&m, 0, sizeof m);
    m.expert_size = expert_size;
    m.hdr.expert_quant = (uint32_t)quant;
    m.hdr.expert_dim = (uint32_t)(expert_dim > 0 ? expert_dim : 0);
    apply_expert(&m, record, hidden, hidden_dim, weight);
}
