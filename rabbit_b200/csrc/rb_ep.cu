// rb_ep.cu -- C ABI: the expert-parallel exchange's communicator. NCCL is
// loaded at run time (dlopen), so the library links no NCCL and a process
// that already holds one (a torch process) shares it.
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <new>

#include "rb_ep.h"

namespace rb {

namespace {

std::mutex g_nccl_mu;
Nccl g_nccl;
bool g_nccl_tried = false, g_nccl_ok = false;
char g_nccl_why[256];

template <typename F>
bool sym(void *h, const char *name, F *dst) {
    *dst = reinterpret_cast<F>(dlsym(h, name));
    return *dst != nullptr;
}

}  // namespace

const Nccl *nccl_lib() {
    std::lock_guard<std::mutex> g(g_nccl_mu);
    if (!g_nccl_tried) {
        g_nccl_tried = true;
        const char *env = getenv("RABBIT_NCCL_LIB");
        void *h = nullptr;
        if (env && *env) {
            h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
        } else {
            // the copy the process already holds, else the loader's search
            h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
            if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        }
        if (!h) {
            snprintf(g_nccl_why, sizeof g_nccl_why, "cannot load NCCL: %s", dlerror());
        } else {
            int (*get_version)(int *) = nullptr;
            Nccl n;
            const bool all =
                sym(h, "ncclGetVersion", &get_version) && sym(h, "ncclGetUniqueId", &n.get_unique_id) &&
                sym(h, "ncclCommInitRank", &n.comm_init_rank) &&
                sym(h, "ncclCommDestroy", &n.comm_destroy) && sym(h, "ncclCommAbort", &n.comm_abort) &&
                sym(h, "ncclAllReduce", &n.all_reduce) && sym(h, "ncclSend", &n.send) &&
                sym(h, "ncclRecv", &n.recv) && sym(h, "ncclGroupStart", &n.group_start) &&
                sym(h, "ncclGroupEnd", &n.group_end) && sym(h, "ncclGetErrorString", &n.error_string);
            if (!all) {
                snprintf(g_nccl_why, sizeof g_nccl_why, "NCCL library lacks a needed symbol");
            } else if (get_version(&n.version) != 0 || n.version < 21800) {
                // grouped point-to-point calls and ncclCommAbort as used here
                snprintf(g_nccl_why, sizeof g_nccl_why, "NCCL %d is older than 2.18", n.version);
            } else {
                g_nccl = n;
                g_nccl_ok = true;
            }
        }
    }
    if (!g_nccl_ok) {
        fail(RABBIT_CUDA_ERR_UNSUPPORTED, "%s", g_nccl_why);
        return nullptr;
    }
    return &g_nccl;
}

int nccl_fail(int r, const char *what) {
    const char *s = g_nccl_ok && g_nccl.error_string ? g_nccl.error_string(r) : "?";
    return fail(RABBIT_CUDA_ERR_DEVICE, "%s: NCCL error %d (%s)", what, r, s);
}

// Fold the oldest recorded call into the sums (waits for its last event).
static int ep_fold_one(rabbit_cuda_ep *ep) {
    EpMarks &m = ep->ring[ep->head];
    cudaError_t e = cudaEventSynchronize(m.ev[5]);
    float t = 0.f, x1 = 0.f, x2 = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&t, m.ev[0], m.ev[5]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&x1, m.ev[1], m.ev[2]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&x2, m.ev[3], m.ev[4]);
    ep->head = (ep->head + 1) % ep->ring.size();
    ep->count--;
    if (e != cudaSuccess) return cuda_fail(e, "ep_stats: events");
    ep->calls++;
    ep->total_ms += t;
    ep->exchange_ms += (double)x1 + (double)x2;
    return RABBIT_CUDA_OK;
}

EpMarks *ep_begin(rabbit_cuda_ep *ep, cudaStream_t s) {
    if (!ep || !ep->timing || ep->ring.empty()) return nullptr;
    if (ep->count == ep->ring.size() && ep_fold_one(ep) != RABBIT_CUDA_OK) return nullptr;
    EpMarks *m = &ep->ring[(ep->head + ep->count) % ep->ring.size()];
    ep->count++;
    cudaEventRecord(m->ev[0], s);
    return m;
}

}  // namespace rb

extern "C" {

int rabbit_cuda_ep_unique_id(unsigned char id[RABBIT_CUDA_EP_ID_BYTES]) {
    if (!id) return rb::fail(RABBIT_CUDA_ERR_ARGS, "ep_unique_id: NULL id");
    const rb::Nccl *n = rb::nccl_lib();
    if (!n) return RABBIT_CUDA_ERR_UNSUPPORTED;
    rb::NcclUniqueId u;
    const int r = n->get_unique_id(&u);
    if (r) return rb::nccl_fail(r, "ncclGetUniqueId");
    memcpy(id, u.internal, sizeof u.internal);
    return rb::ok();
}

rabbit_cuda_ep *rabbit_cuda_ep_create(const unsigned char id[RABBIT_CUDA_EP_ID_BYTES], int rank,
                                      int size, int device) {
    if (!id || size < 1 || rank < 0 || rank >= size) {
        rb::fail(RABBIT_CUDA_ERR_ARGS, "ep_create: rank %d of %d", rank, size);
        return nullptr;
    }
    const rb::Nccl *n = rb::nccl_lib();
    if (!n) return nullptr;
    int st = RABBIT_CUDA_OK;
    if (!rb::dev_ctx(device, &st)) return nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        rb::fail(RABBIT_CUDA_ERR_DEVICE, "ep_create: device %d", device);
        return nullptr;
    }
    rabbit_cuda_ep *ep = new (std::nothrow) rabbit_cuda_ep();
    if (!ep) {
        rb::fail(RABBIT_CUDA_ERR_MEM, "ep_create: out of host memory");
        return nullptr;
    }
    rb::NcclUniqueId u;
    memcpy(u.internal, id, sizeof u.internal);
    const int r = n->comm_init_rank(&ep->comm, size, u, rank);
    if (r) {
        rb::nccl_fail(r, "ncclCommInitRank");
        delete ep;
        return nullptr;
    }
    ep->rank = rank;
    ep->size = size;
    ep->device = device;
    rb::ok();
    return ep;
}

static void ep_release(rabbit_cuda_ep *ep) {
    cudaSetDevice(ep->device);
    for (rb::EpMarks &m : ep->ring)
        for (cudaEvent_t &e : m.ev)
            if (e) cudaEventDestroy(e);
    ep->ring.clear();
    delete ep;
}

void rabbit_cuda_ep_free(rabbit_cuda_ep *ep) {
    if (!ep) return;
    const rb::Nccl *n = rb::nccl_lib();
    if (n && ep->comm) n->comm_destroy(ep->comm);
    ep_release(ep);
}

int rabbit_cuda_ep_abort(rabbit_cuda_ep *ep) {
    if (!ep) return rb::fail(RABBIT_CUDA_ERR_ARGS, "ep_abort: NULL");
    const rb::Nccl *n = rb::nccl_lib();
    if (!n) return RABBIT_CUDA_ERR_UNSUPPORTED;
    if (ep->comm) {
        const int r = n->comm_abort(ep->comm);
        ep->comm = nullptr;
        if (r) return rb::nccl_fail(r, "ncclCommAbort");
    }
    return rb::ok();
}

int rabbit_cuda_ep_set_timing(rabbit_cuda_ep *ep, int on) {
    if (!ep) return rb::fail(RABBIT_CUDA_ERR_ARGS, "ep_set_timing: NULL");
    RB_CUDA(cudaSetDevice(ep->device));
    if (on && ep->ring.empty()) {
        ep->ring.resize(512);
        for (rb::EpMarks &m : ep->ring)
            for (cudaEvent_t &e : m.ev) RB_CUDA(cudaEventCreate(&e));
    }
    ep->timing = on != 0;
    return rb::ok();
}

int rabbit_cuda_ep_stats(rabbit_cuda_ep *ep, uint64_t *calls, double *total_ms,
                         double *exchange_ms, int reset) {
    if (!ep) return rb::fail(RABBIT_CUDA_ERR_ARGS, "ep_stats: NULL");
    RB_CUDA(cudaSetDevice(ep->device));
    int st = RABBIT_CUDA_OK;
    while (ep->count && st == RABBIT_CUDA_OK) st = rb::ep_fold_one(ep);
    if (calls) *calls = ep->calls;
    if (total_ms) *total_ms = ep->total_ms;
    if (exchange_ms) *exchange_ms = ep->exchange_ms;
    if (reset) {
        ep->calls = 0;
        ep->total_ms = ep->exchange_ms = 0.0;
    }
    return st ? st : rb::ok();
}

}  // extern "C"
