// rb_ep.h -- expert-parallel exchange owned by the library: an NCCL
// communicator (libnccl.so.2 loaded at run time) and the per-call timing of
// its exchange steps, used by the multi-token MoE path (rb_moe.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "rb_runtime.h"

namespace rb {

// The part of NCCL's C ABI (nccl.h, NCCL 2.x) used here: an opaque
// communicator, the 128-byte unique id passed by value, ncclResult_t /
// ncclDataType_t / ncclRedOp_t as int.
struct NcclComm;
typedef NcclComm *nccl_comm_t;
struct NcclUniqueId {
    char internal[RABBIT_CUDA_EP_ID_BYTES];
};
constexpr int kNcclInt32 = 2, kNcclFloat32 = 7, kNcclSum = 0;

struct Nccl {
    int version = 0;
    int (*get_unique_id)(NcclUniqueId *) = nullptr;
    int (*comm_init_rank)(nccl_comm_t *, int, NcclUniqueId, int) = nullptr;
    int (*comm_destroy)(nccl_comm_t) = nullptr;
    int (*comm_abort)(nccl_comm_t) = nullptr;
    int (*all_reduce)(const void *, void *, size_t, int, int, nccl_comm_t, cudaStream_t) = nullptr;
    int (*send)(const void *, size_t, int, int, nccl_comm_t, cudaStream_t) = nullptr;
    int (*recv)(void *, size_t, int, int, nccl_comm_t, cudaStream_t) = nullptr;
    int (*group_start)() = nullptr;
    int (*group_end)() = nullptr;
    const char *(*error_string)(int) = nullptr;
};

// libnccl.so.2, loaded once (RABBIT_NCCL_LIB names another file); nullptr +
// error text when it cannot be loaded.
const Nccl *nccl_lib();
// An NCCL result as a library status (RABBIT_CUDA_ERR_DEVICE with the text).
int nccl_fail(int r, const char *what);

// Events of one exchanged call: [0] start, [1] / [2] first exchange, [3] /
// [4] second exchange, [5] end.
struct EpMarks {
    cudaEvent_t ev[6] = {};
};

}  // namespace rb

struct rabbit_cuda_ep {
    rb::nccl_comm_t comm = nullptr;
    int rank = 0, size = 1, device = 0;
    // timing (rabbit_cuda_ep_set_timing): a ring of recorded calls, folded
    // into the sums by rabbit_cuda_ep_stats
    bool timing = false;
    std::vector<rb::EpMarks> ring;
    size_t head = 0, count = 0;
    uint64_t calls = 0;
    double total_ms = 0.0, exchange_ms = 0.0;
};

namespace rb {
// Start of an exchanged call on stream s: the marks to record into, or
// nullptr when timing is off.
EpMarks *ep_begin(rabbit_cuda_ep *ep, cudaStream_t s);
}  // namespace rb
