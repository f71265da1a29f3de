// rb_cache.cu -- C ABI: the reference's expert cache (src/memory.c:12-193,
// declared at src/rabbit.h:123-134) with HBM slots as its backing store.
//
// Same signatures (prefixed rabbit_cuda_), same argument meaning, same
// return conventions (NULL / -1, no status code) and the same replacement
// rule and counters:
//   * create(n_slots): n_slots <= 0 means 4, at most 64
//     (RABBIT_MAX_CACHE_SLOTS); every slot starts empty;
//   * set_expert_size: sizes every slot (here: one HBM allocation of
//     n_slots * size on the calling thread's device);
//   * get: a hit bumps the slot's LRU clock and returns its record, a miss
//     counts and returns NULL;
//   * put / pin: a resident id is bumped (pin also pins it); otherwise the
//     victim is the first empty slot, else the least recently used unpinned
//     one (none: NULL / -1); replacing a resident record counts an eviction;
//     the record is copied in (inserts += 1, bytes_copied += size);
//   * stats / stats_ex: the counters, n_slots and the pinned slots that hold
//     a record.
// The difference is where the bytes live: get / put / pin return DEVICE
// pointers to the slot in HBM (16-byte aligned), and put / pin copy the
// caller's HOST record into it (through pinned staging on a stream of the
// cache's own; the call returns once the record is in HBM). Calls on one
// cache are not thread safe, as in the reference.
#include <string.h>

#include <algorithm>

#include "rb_runtime.h"

namespace {

constexpr int kMaxCacheSlots = 64;  // RABBIT_MAX_CACHE_SLOTS, src/rabbit.h:11

struct Slot {
    int expert_id = -1;  // -1 = empty
    int last_used = 0;   // LRU clock
    int pinned = 0;      // never evicted when set
};

}  // namespace

struct rabbit_cuda_cache {
    Slot slots[kMaxCacheSlots];
    int clock = 0;
    int n_slots = 0;
    size_t expert_size = 0;
    uint64_t hits = 0, misses = 0, inserts = 0, evictions = 0, bytes_copied = 0;
    // HBM backing store
    int device = -1;
    uint8_t *hbm = nullptr;      // n_slots * stride bytes
    size_t stride = 0;           // expert_size rounded up to 256
    cudaStream_t stream = nullptr;
    void *pin = nullptr;         // pinned staging (one record, at most 32 MB)
    size_t pin_cap = 0;
};

namespace {

uint8_t *slot_data(rabbit_cuda_cache *c, int i) { return c->hbm + (size_t)i * c->stride; }

// First empty slot, else the least recently used unpinned one, else -1
// (src/memory.c:118-137).
int find_victim(rabbit_cuda_cache *c) {
    for (int i = 0; i < c->n_slots; i++)
        if (c->slots[i].expert_id < 0) return i;
    int victim = -1, oldest = 0x7fffffff;
    for (int i = 0; i < c->n_slots; i++) {
        if (c->slots[i].pinned) continue;
        if (c->slots[i].last_used < oldest) {
            oldest = c->slots[i].last_used;
            victim = i;
        }
    }
    return victim;
}

// Host record -> the slot in HBM, in staging-sized pieces; 0 on success.
int copy_in(rabbit_cuda_cache *c, int slot, const void *src) {
    if (cudaSetDevice(c->device) != cudaSuccess) return -1;
    const uint8_t *s = static_cast<const uint8_t *>(src);
    uint8_t *d = slot_data(c, slot);
    for (size_t off = 0; off < c->expert_size; off += c->pin_cap) {
        const size_t n = std::min(c->pin_cap, c->expert_size - off);
        memcpy(c->pin, s + off, n);
        cudaError_t e = cudaMemcpyAsync(d + off, c->pin, n, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) {
            rb::cuda_fail(e, "cache: record copy");
            return -1;
        }
    }
    return 0;
}

// Bring `expert_id` into a victim slot (put / pin); the slot or -1.
int insert(rabbit_cuda_cache *c, int expert_id, const void *src, int pinned) {
    const int victim = find_victim(c);
    if (victim < 0) return -1;  // all slots pinned and full
    if (c->slots[victim].expert_id >= 0) c->evictions++;
    // the slot is taken over before the copy, as the reference does
    c->slots[victim].expert_id = -1;
    if (copy_in(c, victim, src) != 0) return -1;
    c->slots[victim].expert_id = expert_id;
    c->slots[victim].last_used = ++c->clock;
    c->slots[victim].pinned = pinned;
    c->inserts++;
    c->bytes_copied += c->expert_size;
    return victim;
}

void release_store(rabbit_cuda_cache *c) {
    if (c->device >= 0) cudaSetDevice(c->device);
    if (c->hbm) cudaFree(c->hbm);
    if (c->pin) cudaFreeHost(c->pin);
    c->hbm = nullptr;
    c->pin = nullptr;
    c->pin_cap = 0;
}

}  // namespace

extern "C" {

rabbit_cuda_cache *rabbit_cuda_cache_create(int n_slots) {
    if (n_slots <= 0) n_slots = 4;
    if (n_slots > kMaxCacheSlots) n_slots = kMaxCacheSlots;
    int st = RABBIT_CUDA_OK;
    const int dev = rb::current_device();
    rb::DevCtx *ctx = rb::dev_ctx(dev, &st);
    if (!ctx) return nullptr;
    rabbit_cuda_cache *c = new (std::nothrow) rabbit_cuda_cache();
    if (!c) {
        rb::fail(RABBIT_CUDA_ERR_MEM, "cache_create: out of host memory");
        return nullptr;
    }
    c->n_slots = n_slots;
    c->device = dev;
    if (cudaSetDevice(dev) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        rb::fail(RABBIT_CUDA_ERR_DEVICE, "cache_create: stream");
        delete c;
        return nullptr;
    }
    rb::ok();
    return c;
}

void rabbit_cuda_cache_free(rabbit_cuda_cache *c) {
    if (!c) return;
    release_store(c);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

void rabbit_cuda_cache_set_expert_size(rabbit_cuda_cache *c, size_t size) {
    if (!c) return;
    // the slots' records are dropped with their storage when the size changes
    if (c->hbm && size != c->expert_size) {
        release_store(c);
        for (int i = 0; i < c->n_slots; i++) c->slots[i] = Slot();
    }
    c->expert_size = size;
    if (size == 0 || c->hbm) return;
    // every slot is allocated up front, so put never allocates (memory.c:44-58)
    c->stride = (size + 255) / 256 * 256;
    c->pin_cap = std::min<size_t>(size, 32u << 20);
    cudaError_t e = cudaSetDevice(c->device);
    if (e == cudaSuccess) e = cudaMalloc(&c->hbm, c->stride * (size_t)c->n_slots);
    if (e == cudaSuccess) e = cudaMallocHost(&c->pin, c->pin_cap);
    if (e != cudaSuccess) {
        release_store(c);
        rb::cuda_fail(e, "cache_set_expert_size: HBM slots");
    }
}

void *rabbit_cuda_cache_get(rabbit_cuda_cache *c, int expert_id) {
    if (!c) return nullptr;
    for (int i = 0; i < c->n_slots; i++) {
        if (c->slots[i].expert_id == expert_id) {
            c->slots[i].last_used = ++c->clock;
            c->hits++;
            return slot_data(c, i);
        }
    }
    c->misses++;
    return nullptr;
}

void *rabbit_cuda_cache_put(rabbit_cuda_cache *c, int expert_id, const void *src) {
    if (!c || !src || c->expert_size == 0 || !c->hbm) return nullptr;
    for (int i = 0; i < c->n_slots; i++) {  // already resident
        if (c->slots[i].expert_id == expert_id) {
            c->slots[i].last_used = ++c->clock;
            return slot_data(c, i);
        }
    }
    const int v = insert(c, expert_id, src, 0);
    return v < 0 ? nullptr : slot_data(c, v);
}

int rabbit_cuda_cache_pin(rabbit_cuda_cache *c, int expert_id, const void *src_or_null) {
    if (!c || expert_id < 0) return -1;
    for (int i = 0; i < c->n_slots; i++) {  // already present: just pin
        if (c->slots[i].expert_id == expert_id) {
            c->slots[i].pinned = 1;
            c->slots[i].last_used = ++c->clock;
            return 0;
        }
    }
    if (!src_or_null || c->expert_size == 0 || !c->hbm) return -1;
    return insert(c, expert_id, src_or_null, 1) < 0 ? -1 : 0;
}

void rabbit_cuda_cache_stats(const rabbit_cuda_cache *c, uint64_t *hits, uint64_t *misses,
                             uint64_t *inserts) {
    if (hits) *hits = c ? c->hits : 0;
    if (misses) *misses = c ? c->misses : 0;
    if (inserts) *inserts = c ? c->inserts : 0;
}

void rabbit_cuda_cache_stats_ex(const rabbit_cuda_cache *c, uint64_t *hits, uint64_t *misses,
                                uint64_t *inserts, uint64_t *evictions, uint64_t *bytes_copied,
                                int *n_slots, int *n_pinned) {
    rabbit_cuda_cache_stats(c, hits, misses, inserts);
    if (evictions) *evictions = c ? c->evictions : 0;
    if (bytes_copied) *bytes_copied = c ? c->bytes_copied : 0;
    if (n_slots) *n_slots = c ? c->n_slots : 0;
    if (n_pinned) {
        int p = 0;
        if (c)
            for (int i = 0; i < c->n_slots; i++)
                if (c->slots[i].pinned && c->slots[i].expert_id >= 0) p++;
        *n_pinned = p;
    }
}

}  // extern "C"
