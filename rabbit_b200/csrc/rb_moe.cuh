// rb_moe.cuh -- MoE decode kernels (fused group-32 path and generic path).
#pragma once
#include <stdint.h>

#include "rb_device.cuh"

namespace rb {

constexpr int kMaxSlots = 72;  // top-k (<= 8) + shared (<= 64)

// Routing result shared by the generic kernels (device memory).
struct Route {
    int nact;                  // active slots
    int rec[kMaxSlots];        // global record id per slot
    float w[kMaxSlots];        // combine weight per slot
};

struct MoeFusedArgs {
    const float *h_in;
    float *h_out;
    int *ids_out;     // [k]
    float *w_out;     // [k]
    const float *rms;     // [H]
    const float *router;  // [E, H]
    const uint8_t *pool;
    uint64_t rec_stride;
    uint64_t off_gnib, off_unib, off_dnib, off_gsc, off_usc, off_dsc;
    int rec_base;  // global record of local expert 0 in this layer
    int n_local;   // local ids >= n_local have no record (skipped)
    int H, E, k, I, S;
    int usable;    // 0: records too small, experts add nothing (forward_v2.c:319-322)
    float *scores; // scratch [E]
    float *mid;    // scratch [k+S][I]
    unsigned *bar; // scratch [2]: arrival count, generation
    int *err;
    uint64_t wait_ns;
    // plan
    int CW, KSb, RSb, CRb, KSc, RSc, CRc, nslots;
    uint32_t slot_bytes;
    int part_floats;
};

__global__ void k_moe_decode_g32(MoeFusedArgs a);

// ---- generic path (any quant / shape): route, up (gate+up+silu), down, combine
struct MoeGenericArgs {
    const float *h_in;
    float *h_out;
    int *ids_out;
    float *w_out;
    const float *rms;
    const float *router;
    const uint8_t *pool;  // raw records at rec_stride
    uint64_t rec_stride;
    uint64_t expert_size;
    int rec_base, n_local;
    int H, E, k, I, S, quant, usable;
    float *xn;     // [H]
    float *scores; // [E]
    float *mid;    // [slots][I]
    float *down;   // [slots][H]
    Route *route;
};

__global__ void k_moe_route(MoeGenericArgs a);
__global__ void k_moe_up_generic(MoeGenericArgs a);
__global__ void k_moe_down_generic(MoeGenericArgs a);
__global__ void k_moe_combine(MoeGenericArgs a);

}  // namespace rb
