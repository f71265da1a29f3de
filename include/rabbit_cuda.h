/*
 * rabbit_cuda.h -- C ABI of the B200 (sm_100a) routed-expert hot path.
 *
 * Plain C: pointers, sizes and status codes only. A CUDA stream is passed as
 * `void *` (a cudaStream_t / CUstream; NULL = the default stream). Entry
 * points that take HOST buffers use a stream of the library's own and return
 * after the result is on the host.
 * Every entry point returns a rabbit_cuda_status; on failure
 * rabbit_cuda_last_error() holds a one-line explanation for the calling
 * thread. Nothing here calls exit(); nothing falls back to the CPU.
 *
 * Reference interfaces replaced (Stanley03-arch/Rabbit v0.4.28):
 *   rabbit_gemv_int4_grouped        src/quant.c:152-188, src/rabbit.h:178-179
 *   rabbit_dequant_int4_grouped     src/quant.c:123-142, src/rabbit.h:177
 *   moe_step / expert_swiglu /
 *     select_top_k (static)         src/forward_v2.c:248-402
 *   expert cache + mmap fetch       src/memory.c:94-253, src/moe.c:73-117
 *   rabbit_cache_* (HBM slots)      src/rabbit.h:123-134, src/memory.c:12-193
 *   rabbit_cache_stats_ex           src/rabbit.h:132-134
 */
#ifndef RABBIT_CUDA_H
#define RABBIT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported even when the library is built with -fvisibility=hidden. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define RABBIT_CUDA_ABI_VERSION 1

/* The first six values are rabbit_status (src/rabbit.h:16-23). */
typedef enum {
    RABBIT_CUDA_OK = 0,
    RABBIT_CUDA_ERR_IO = 1,
    RABBIT_CUDA_ERR_MEM = 2,
    RABBIT_CUDA_ERR_FORMAT = 3,
    RABBIT_CUDA_ERR_UNSUPPORTED = 4,
    RABBIT_CUDA_ERR_ARGS = 5,
    RABBIT_CUDA_ERR_DEVICE = 6,  /* a CUDA call failed (message has the CUDA error) */
    RABBIT_CUDA_ERR_TIMEOUT = 7  /* a bounded device-side wait gave up */
} rabbit_cuda_status;

/* ------------------------------------------------------------- library -- */

/* "rabbit-b200 <version>" */
const char *rabbit_cuda_version(void);
/* Text of the last failure on this thread ("" if none). */
const char *rabbit_cuda_last_error(void);
/* Number of visible CUDA devices (0 without a GPU; never fails on a host). */
int rabbit_cuda_device_count(int *count);
/* Select the device later calls on this thread use (default 0). */
int rabbit_cuda_set_device(int device);
/* Device-side wait limit in milliseconds for mbarrier / inter-CTA spins
 * (default 2000). A wait that runs out sets RABBIT_CUDA_ERR_TIMEOUT. */
int rabbit_cuda_set_wait_limit_ms(int ms);
/* The same limit in microseconds (for tests of the timeout path). */
int rabbit_cuda_set_wait_limit_us(int us);

/* --------------------------------------------- stateless quant drop-ins -- */

/* Drop-in for rabbit_gemv_int4_grouped (src/quant.c:152-188): y = W x with W a
 * group-scaled int4 blob (u32 group_size | f32 scales | packed nibbles) over
 * the flat row-major index, any shape. HOST buffers; W is copied to the device
 * each call. An invalid group_size (0 or > 4096) writes zeros, as the
 * reference does. Returns ARGS for NULL pointers or non-positive sizes (the
 * reference returns silently there). */
int rabbit_cuda_gemv_int4_grouped(const uint8_t *W, const float *x, float *y,
                                  int out_dim, int in_dim);

/* Device-buffer dequant (src/quant.c:123-142): dst[i] = (float)q_i * scale.
 * d_blob may have any alignment. Returns FORMAT for an invalid group size. */
int rabbit_cuda_dequant_int4_grouped_dev(const uint8_t *d_blob, float *d_dst, int n,
                                         void *stream);

/* Device-buffer GEMV over a raw blob already in device memory (any shape,
 * any alignment), same arithmetic contract as rabbit_gemv_int4_grouped. */
int rabbit_cuda_gemv_int4_grouped_dev(const uint8_t *d_blob, const float *d_x, float *d_y,
                                      int out_dim, int in_dim, void *stream);

/* ------------------------------------------------- resident int4 matrix -- */

/* One group-32 int4 matrix kept in HBM in the GEMV layout (16-byte aligned
 * nibble plane [rows][in/2] and scale plane [rows][in/32]). */
typedef struct rabbit_cuda_matrix rabbit_cuda_matrix;

/* Upload a host blob (.rabbit matrix format). Shapes with in_dim % 32 != 0 or
 * group_size != 32 are kept verbatim and served by the flat-index kernel. */
int rabbit_cuda_matrix_upload(const uint8_t *blob, int out_dim, int in_dim,
                              rabbit_cuda_matrix **out);
int rabbit_cuda_matrix_free(rabbit_cuda_matrix *m);
/* y = W x with device x / y (16-byte aligned), on `stream`. */
int rabbit_cuda_matrix_gemv_dev(const rabbit_cuda_matrix *m, const float *d_x, float *d_y,
                                void *stream);
/* Same with HOST x / y: copies in, GEMV, copies out, synchronises. */
int rabbit_cuda_matrix_gemv(const rabbit_cuda_matrix *m, const float *x, float *y);
/* n independent GEMVs in one launch (no counterpart in the reference, which
 * calls rabbit_gemv_int4_grouped once per matrix): d_y[i] = m[i] d_x[i] for
 * 1 <= n <= 32 resident matrices of one device, shape and format, e.g. the
 * projections that share one input. The matrices' tiles stream back to back
 * through every SM, so the fixed cost of a launch and of its dependency on
 * the previous kernel is paid once; x planes are built once when every d_x[i]
 * is the same pointer. Same conventions as rabbit_cuda_matrix_gemv_dev. */
int rabbit_cuda_matrix_gemv_batch_dev(const rabbit_cuda_matrix *const *m, int n,
                                      const float *const *d_x, float *const *d_y, void *stream);
/* Algorithmic bytes one GEMV streams: the blob (4 + 4*ceil(n/32) + n/2)
 * plus x and y in fp32. */
uint64_t rabbit_cuda_matrix_bytes(const rabbit_cuda_matrix *m);

/* --------------------------------------------- HBM-resident expert pool -- */

/* Model description for the MoE block. Mirrors the fields moe_step reads from
 * RabbitModel / RefV2Weights (src/rabbit.h:28-97, src/forward_v2.c:106-169,
 * src/model.c:152-189). All pointers are HOST pointers and are read only
 * during rabbit_cuda_moe_create / rabbit_cuda_moe_upload. */
typedef struct {
    int n_layers;
    int hidden;             /* H */
    int n_experts;          /* routed experts per layer, E (router width) */
    int experts_per_token;  /* header top-k; <= 0 means 2 (forward_v2.c:113) */
    int inter;              /* expert FFN width I */
    int n_shared;           /* always-on shared experts S (reserved[12..15]); 0..64 */
    int expert_quant;       /* 0 f32, 4 group-int4, 8 int8 (forward_v2.c:297-354) */
    uint64_t expert_size;   /* bytes per record */
    int n_records;          /* records in expert_map */
    int experts_per_layer;  /* records per layer (E or E+S) */
    int experts_shared;     /* 1: one table for every layer (memory.c:230-238) */
    const void *expert_map; /* host pointer to record 0 (e.g. the mmap'd file);
                               NULL: records come from rabbit_cuda_moe_fill_synthetic */
    const float *const *rms_ffn;  /* [n_layers] -> H floats */
    const float *const *w_router; /* [n_layers] -> E*H floats */
} rabbit_cuda_moe_desc;

typedef struct rabbit_cuda_moe rabbit_cuda_moe;

/* expert_quant code of records already in this library's tiled group-32
 * layout, as rabbit_cuda_tile_records writes them (no counterpart in the
 * reference, whose codes are 0, 4 and 8; a converter that writes such a file
 * marks it with this code so readers of the group-32 format never see it).
 * A pool of such records uploads them without re-laying them out. */
#define RABBIT_CUDA_QUANT_INT4_TILED 36

/* Re-lay n_records group-32 int4 expert records (gate | up | down blobs,
 * src/forward_v2.c:314-332; desc's shapes, expert_quant 4, records
 * desc->expert_size apart) into the tiled layout a pool uses on a GPU with
 * sm_count SMs (148 on a B200), each followed by a 256-byte trailer that names
 * the tile plan: the converter side of RABBIT_CUDA_QUANT_INT4_TILED
 * (convert_hf_stream.py:56-73 writes the group-32 blobs). Host only: touches no
 * GPU. *tiled_size gets the bytes of one tiled record -- the expert_size the
 * converted file declares; dst (n_records * *tiled_size bytes) may be NULL to
 * query it. A pool on a GPU whose plan differs refuses the records
 * (RABBIT_CUDA_ERR_FORMAT). */
int rabbit_cuda_tile_records(const rabbit_cuda_moe_desc *desc, int sm_count, const void *src,
                             int n_records, void *dst, uint64_t *tiled_size);

/* Create the pool on `device`: allocates HBM for every record (the pool is the
 * whole expert table, resident), plus router/norm weights and scratch. */
int rabbit_cuda_moe_create(const rabbit_cuda_moe_desc *desc, int device,
                           rabbit_cuda_moe **out);
/* A pool for models larger than HBM (no counterpart in the reference, whose
 * expert LRU cache, src/memory.c:94-193, holds at most 64 single records):
 * HBM holds the records of `window_layers` layers at a time, one block per
 * layer. Uploading a layer that has no block (rabbit_cuda_moe_upload or
 * _upload_file, at most window_layers layers per call) takes the least
 * recently used block, dropping the layer it held; the copies wait on the
 * pool's side stream for the last kernel that read the block, and kernels on
 * any stream wait for the copies into their layer's block, so an engine can
 * upload layer l + 1 while layer l computes. Decoding a layer without a block
 * returns RABBIT_CUDA_ERR_ARGS ("not uploaded"). window_layers >= n_layers is
 * rabbit_cuda_moe_create. Tables shared by every layer (experts_shared) and
 * rabbit_cuda_moe_fill_synthetic are not supported. */
int rabbit_cuda_moe_create_window(const rabbit_cuda_moe_desc *desc, int device, int window_layers,
                                  rabbit_cuda_moe **out);
/* Stage records of layers [layer_begin, layer_end) host -> pinned -> HBM on the
 * pool's side stream (asynchronous; returns once queued). */
int rabbit_cuda_moe_upload(rabbit_cuda_moe *p, int layer_begin, int layer_end);
/* Stage records of layers [layer_begin, layer_end) straight from the model
 * file instead of a host map -- the reference's pread fallback
 * (rabbit_expert_pread, src/memory.c:255-279, record gid at expert_offset +
 * gid * expert_size). A reader thread preads records (O_DIRECT when the file
 * system allows it, else buffered) into a ring of pinned buffers while the
 * caller's thread re-lays group-32 records into tiles and queues their copies
 * on the pool's side stream, so file reads, host re-layout and PCIe copies
 * overlap. `expert_offset` is the file offset of record 0 (the .rabbit
 * header, then the dense block, then the expert table: src/model.c:324-339);
 * it is an argument because the reference never sets expert_file_offset
 * (src/model.c:236-348) and its pread path reads from offset 0. Resident
 * records are skipped. Returns once the copies are queued (see
 * rabbit_cuda_moe_sync). RABBIT_CUDA_ERR_IO: the file cannot be opened, a
 * read fails, or the file ends inside a record; RABBIT_CUDA_ERR_FORMAT: a
 * record of a pool planned for group-32 records carries another group size.
 * Records read before an error stay resident. */
int rabbit_cuda_moe_upload_file(rabbit_cuda_moe *p, const char *path, uint64_t expert_offset,
                                int layer_begin, int layer_end);
/* Wait until every queued upload has landed. */
int rabbit_cuda_moe_sync(rabbit_cuda_moe *p);
/* Fill every record of a group-32 int4 pool on the device with seeded
 * synthetic weights (nibbles uniform on [-8, 7], one scale |N(0, sigma)|/7 per
 * 32 inputs) and mark them resident. For benchmarks and tests of models too
 * large to stage from host memory; desc.expert_map may be NULL then.
 * UNSUPPORTED for pools that are not in the group-32 layout. */
int rabbit_cuda_moe_fill_synthetic(rabbit_cuda_moe *p, uint64_t seed, float scale_sigma);
int rabbit_cuda_moe_free(rabbit_cuda_moe *p);

/* One token through one layer's MoE block (moe_step, forward_v2.c:362-402):
 * xn = rmsnorm(h); scores = W_router xn; top-k (strict '>', lower id wins
 * ties) + softmax; h_out = h + sum_j w_j * SwiGLU_j(xn) + sum_shared SwiGLU(xn).
 * HOST buffers: h_in/h_out [H] (may alias), ids/weights [k] (may be NULL).
 * Returns the k used through *k_out (may be NULL). */
int rabbit_cuda_moe_decode(rabbit_cuda_moe *p, int layer, const float *h_in, float *h_out,
                           int *ids, float *weights, int *k_out);
/* Same on DEVICE buffers, asynchronous on `stream` (16-byte aligned h). The
 * values the kernel's CTAs share are tagged with a number the host picks for
 * each call, so a call made while `stream` is capturing a CUDA graph (whose
 * replays would all reuse one tag) returns RABBIT_CUDA_ERR_UNSUPPORTED. */
int rabbit_cuda_moe_decode_dev(rabbit_cuda_moe *p, int layer, const float *d_h_in,
                               float *d_h_out, int *d_ids, float *d_weights, void *stream);
/* No counterpart in the reference (its moe_step runs on the CPU). The same
 * decode as rabbit_cuda_moe_decode_dev, for callers that must not allocate
 * device memory while they decode: an engine that has already split the
 * device's memory between its own arenas, or a serving loop that cannot take
 * the device-wide synchronisation a cudaMalloc/cudaFree brings. The call
 * allocates nothing and frees nothing; its scratch (router scores, the SwiGLU
 * activations, the down-projection rows and per-CTA flags) is a fixed 2 MiB
 * array inside this library, present on every device that loads it until the
 * process exits. A model fits when
 *   256 + 4096 + A(E * 8) + A((k + S) * I * 8) + (k + S) * C * H * 8
 * is at most 2 MiB, with A(x) = x rounded up to a multiple of 256 and C the
 * number of column chunks of W2 (the I / 32 groups of a W2 row split into
 * chunks of the largest divisor of I / 32 up to 32; C = I / 1024 when I is a
 * multiple of 1024); larger models are rejected with RABBIT_CUDA_ERR_ARGS,
 * pools not in the group-32 layout with RABBIT_CUDA_ERR_UNSUPPORTED. The
 * first call on each device looks up the array's device address (once, with
 * that device current); make that first call before any stream capture. As
 * for rabbit_cuda_moe_decode_dev, a call made while `stream` is capturing
 * returns RABBIT_CUDA_ERR_UNSUPPORTED. Every call uses the same array, which
 * keeps what the last call left there: the values its CTAs share carry a tag
 * new to each call, so leftovers are never read. Calls that overlap on the GPU
 * (other streams, other pools on the same device) race on the array and give
 * wrong results. d_ids / d_weights may be NULL. Errors surface through
 * rabbit_cuda_moe_check as for rabbit_cuda_moe_decode_dev. */
int rabbit_cuda_moe_decode_dev_noalloc(rabbit_cuda_moe *p, int layer, const float *d_h_in,
                                       float *d_h_out, int *d_ids, float *d_weights,
                                       void *stream);
/* T tokens through one layer's MoE block at once (the multi-token "prefill"
 * form of moe_step, forward_v2.c:362-402): each token is routed on its own
 * (rmsnorm, router, top-k, softmax, shared experts with weight 1) and gets the
 * same result as rabbit_cuda_moe_decode would give it alone, but each expert
 * the chunk touches is read from HBM once for all the tokens routed to it.
 * DEVICE buffers, asynchronous on `stream`: h_in / h_out [T][H] (may alias),
 * ids / weights [T][k] (both or neither may be NULL). 1 <= n_tokens <= 256.
 * Pools outside the group-32 layout run the per-token decode, token by token. */
int rabbit_cuda_moe_prefill_dev(rabbit_cuda_moe *p, int layer, const float *d_h_in,
                                float *d_h_out, int n_tokens, int *d_ids, float *d_weights,
                                void *stream);
/* Same on HOST buffers; synchronous. */
int rabbit_cuda_moe_prefill(rabbit_cuda_moe *p, int layer, const float *h_in, float *h_out,
                            int n_tokens, int *ids, float *weights);
/* Expert parallelism for the multi-token path (no counterpart in the
 * reference): this pool holds rank `rank`'s share of a layer whose E routed
 * experts are spread over `size` ranks -- expert e lives on rank e % size as
 * local record e / size of each layer -- followed by the S shared experts,
 * so experts_per_layer must be E / size + S. Routing is computed in full on
 * every rank; rabbit_cuda_moe_prefill[_dev] then writes rank 0: h + its
 * experts' share (shared experts included), other ranks: their experts'
 * share only, so the sum of the ranks' outputs (an all-reduce) is the layer
 * output. ids / weights report the full routing. size 1 (the default) is the
 * whole layer. Decode calls on a pool with size > 1 are refused. */
int rabbit_cuda_moe_set_expert_parallel(rabbit_cuda_moe *p, int rank, int size);

/* ------------------------------------- expert-parallel exchange (NCCL) --
 * No counterpart in the reference (a single-process engine): the exchange
 * between expert-parallel ranks done inside the library, over an NCCL
 * communicator (libnccl.so.2, loaded when the first exchange object is made;
 * RABBIT_NCCL_LIB names another file), so a C engine gets expert
 * parallelism without torch. One process per GPU; every rank makes the same
 * calls in the same order. */
#define RABBIT_CUDA_EP_ID_BYTES 128
typedef struct rabbit_cuda_ep rabbit_cuda_ep;
/* A new communicator id (one rank makes it and hands the bytes to the others
 * out of band: a file, a socket, MPI). */
int rabbit_cuda_ep_unique_id(unsigned char id[RABBIT_CUDA_EP_ID_BYTES]);
/* Join the communicator `id` as `rank` of `size` on `device`; collective (all
 * ranks call it, each blocks until all have). NULL on failure. */
rabbit_cuda_ep *rabbit_cuda_ep_create(const unsigned char id[RABBIT_CUDA_EP_ID_BYTES], int rank,
                                      int size, int device);
/* Destroy (ep_abort first if a peer is gone: it ends the communicator's
 * pending work instead of waiting for it). Pools that use it must be freed,
 * or given another exchange, first. */
void rabbit_cuda_ep_free(rabbit_cuda_ep *ep);
int rabbit_cuda_ep_abort(rabbit_cuda_ep *ep);
/* Per-call timing (CUDA events on the call's stream, off by default):
 * rabbit_cuda_ep_stats then synchronises them and reports the exchanged
 * calls timed, their total time on the stream and the part spent in the
 * exchange steps (collective wait included), in ms. Any pointer may be NULL;
 * reset != 0 zeroes the sums afterwards. */
int rabbit_cuda_ep_set_timing(rabbit_cuda_ep *ep, int on);
int rabbit_cuda_ep_stats(rabbit_cuda_ep *ep, uint64_t *calls, double *total_ms,
                         double *exchange_ms, int reset);

/* Exchange modes of rabbit_cuda_moe_set_ep. */
#define RABBIT_CUDA_EP_ALLREDUCE 1 /* every rank passes the same tokens; the ranks'
                                      shares are summed (ncclAllReduce) so every
                                      rank gets the layer output */
#define RABBIT_CUDA_EP_ALLTOALL 2  /* every rank passes its OWN n_tokens tokens (the
                                      same n_tokens on every rank) and gets their
                                      layer output; pairs routed to another rank's
                                      experts go there and come back (grouped
                                      ncclSend / ncclRecv) */
/* Give the pool's multi-token path (rabbit_cuda_moe_prefill[_dev]) an
 * exchange: the pool holds rank ep.rank's share as in
 * rabbit_cuda_moe_set_expert_parallel(p, ep.rank, ep.size) (same record rule),
 * and each call also does the exchange of `mode` on its stream, so its output
 * is the whole layer's. ALLTOALL outputs equal the single-pool outputs bit for
 * bit (each token's slots combine in the same order). ep NULL (or mode 0)
 * goes back to no exchange. The pool's device must be ep's. */
int rabbit_cuda_moe_set_ep(rabbit_cuda_moe *p, rabbit_cuda_ep *ep, int mode);
/* Test hook (no counterpart in the reference): in the next fused decode of
 * this pool, no CTA publishes router row `expert`, so every CTA's bounded
 * wait for that score runs out (RABBIT_CUDA_ERR_TIMEOUT through
 * rabbit_cuda_moe_check) with no copy in flight; the launch after it is
 * normal. UNSUPPORTED for pools whose decode scores every router row in
 * every CTA (routers up to 256 KB). */
int rabbit_cuda_moe_debug_withhold_score(rabbit_cuda_moe *p, int expert);
/* Check the device error word after work on `stream` finished (TIMEOUT if a
 * bounded wait gave up). Synchronises `stream`. */
int rabbit_cuda_moe_check(rabbit_cuda_moe *p, void *stream);

/* Counters in the spirit of rabbit_cache_stats_ex (src/memory.c:74-92):
 * decode calls served from HBM, records uploaded, bytes moved host->device,
 * records resident, pool bytes. */
int rabbit_cuda_moe_stats(const rabbit_cuda_moe *p, uint64_t *hbm_hits, uint64_t *uploads,
                          uint64_t *h2d_bytes, int *resident_records, uint64_t *pool_bytes);
/* The counters of rabbit_cache_stats_ex (src/rabbit.h:132-134,
 * src/memory.c:74-92) for the pool: hits = kernel calls served from HBM,
 * misses = calls refused because their layer was not resident, inserts =
 * records uploaded, evictions = resident records dropped when a window block
 * was taken for another layer, bytes_copied = bytes moved host -> device,
 * n_slots = records HBM holds, n_pinned = records that cannot be dropped
 * (every resident record of a pool without a window; 0 with one). Any
 * pointer may be NULL. */
int rabbit_cuda_moe_stats_ex(const rabbit_cuda_moe *p, uint64_t *hits, uint64_t *misses,
                             uint64_t *inserts, uint64_t *evictions, uint64_t *bytes_copied,
                             int *n_slots, int *n_pinned);
/* Algorithmic bytes of one decode (router + selected + shared experts). */
uint64_t rabbit_cuda_moe_decode_bytes(const rabbit_cuda_moe *p);

/* ------------------------------------------------- HBM expert cache -- */

/* The reference's expert cache (src/rabbit.h:123-134, src/memory.c:12-193)
 * with its slots in HBM: the same signatures, argument meaning, return
 * conventions (NULL / -1; rabbit_cuda_last_error() says why where a CUDA call
 * failed), replacement rule (a resident id is bumped; else the first empty
 * slot, else the least recently used unpinned one) and counters. get / put /
 * pin return DEVICE pointers to the record's slot (256-byte aligned); put /
 * pin copy the caller's HOST record in and return once it is in HBM. The
 * cache lives on the calling thread's device (rabbit_cuda_set_device). Not
 * thread safe, as in the reference. */
typedef struct rabbit_cuda_cache rabbit_cuda_cache;
/* n_slots <= 0 means 4; at most 64 (RABBIT_MAX_CACHE_SLOTS). NULL on failure. */
rabbit_cuda_cache *rabbit_cuda_cache_create(int n_slots);
void rabbit_cuda_cache_free(rabbit_cuda_cache *c);
/* Allocates every slot in HBM (n_slots x size); a new size empties the cache. */
void rabbit_cuda_cache_set_expert_size(rabbit_cuda_cache *c, size_t size);
void *rabbit_cuda_cache_get(rabbit_cuda_cache *c, int expert_id);
void *rabbit_cuda_cache_put(rabbit_cuda_cache *c, int expert_id, const void *src);
/* Pin an already-cached or about-to-be-cached expert so LRU will not evict
 * it; 0 on success, -1 otherwise. */
int rabbit_cuda_cache_pin(rabbit_cuda_cache *c, int expert_id, const void *src_or_null);
void rabbit_cuda_cache_stats(const rabbit_cuda_cache *c, uint64_t *hits, uint64_t *misses,
                             uint64_t *inserts);
void rabbit_cuda_cache_stats_ex(const rabbit_cuda_cache *c, uint64_t *hits, uint64_t *misses,
                                uint64_t *inserts, uint64_t *evictions, uint64_t *bytes_copied,
                                int *n_slots, int *n_pinned);

/* ----------------------------------------- legacy per-tensor experts -- */

/* The legacy expert of src/moe.c:119-224 (apply_expert), for records in the
 * older per-tensor format (expert_quant 4: int4, any other value: int8; one
 * fp32 scale per matrix): hidden[hidden_dim] += the expert's output times
 * `weight`, the record read exactly as apply_expert reads it -- three
 * [scale | payload] matrices (gate, up, down; I = expert_dim, 2 H when 0 or
 * above 4 H; scales that are not positive finite numbers read as 1/127) with
 * SwiGLU between them, or, for a record too small for three, its square-matrix
 * and raw-byte fallbacks (moe.c:183-220). HOST record and hidden; synchronous.
 * Sums are reordered across lanes: outputs match the reference within fp32
 * rounding. A record whose odd-width int4 rows would run past its end (the
 * reference reads beyond the buffer there) returns RABBIT_CUDA_ERR_FORMAT. */
int rabbit_cuda_legacy_apply_expert(const void *record, uint64_t expert_size, int expert_quant,
                                    int hidden_dim, int expert_dim, float *hidden, float weight);
/* Same on DEVICE record and hidden (e.g. a slot of rabbit_cuda_cache_put),
 * asynchronous on `stream`. */
int rabbit_cuda_legacy_apply_expert_dev(const void *d_record, uint64_t expert_size,
                                        int expert_quant, int hidden_dim, int expert_dim,
                                        float *d_hidden, float weight, void *stream);

/* ------------------------------------- incremental ref-v2 decode context -- */

/* The dense (fp32) weights of a ref-v2 model, in the layout parse_weights
 * reads from the .rabbit dense block (src/forward_v2.c:106-169). HOST
 * pointers, read only during rabbit_cuda_refv2_create; embed == NULL: every
 * dense weight is left for rabbit_cuda_refv2_fill_synthetic. */
typedef struct {
    int n_layers, hidden, vocab;
    int n_heads, n_kv_heads, head_dim;  /* n_heads * head_dim may differ from hidden */
    int max_ctx;                        /* KV window, 1..256 (forward_v2.c:16-26) */
    const float *embed;                 /* [vocab, hidden] */
    const float *lm_head;               /* [hidden, vocab] */
    const float *final_norm;            /* [hidden] */
    const float *const *rms_attn;       /* [n_layers] -> [hidden] */
    const float *const *w_q;            /* [n_layers] -> [n_heads * head_dim, hidden] */
    const float *const *w_k;            /* [n_layers] -> [n_kv_heads * head_dim, hidden] */
    const float *const *w_v;            /* [n_layers] -> [n_kv_heads * head_dim, hidden] */
    const float *const *w_o;            /* [n_layers] -> [hidden, n_heads * head_dim] */
} rabbit_cuda_dense_desc;

typedef struct rabbit_cuda_refv2 rabbit_cuda_refv2;

/* The device-resident form of RabbitRefV2Ctx (src/rabbit.h:160-167, declared
 * but not implemented in the reference): dense weights and a per-layer KV
 * cache in HBM, the MoE blocks from `moe` (a pool of the same model on the
 * same device; it must outlive the context). One decode step follows
 * rabbit_ref_v2_forward's per-token loop (forward_v2.c:457-471):
 * h = embed[id % vocab]; per layer attention_step then moe_step; then the
 * final rmsnorm and logits = lm_head^T h (forward_v2.c:404-413, 473-484).
 * The KV cache stops growing at max_ctx, as attention_step does. */
int rabbit_cuda_refv2_create(const rabbit_cuda_dense_desc *desc, rabbit_cuda_moe *moe,
                             rabbit_cuda_refv2 **out);
/* Seeded synthetic dense weights on the device: embed, projections, lm_head
 * uniform with standard deviation `sigma`, norms 1. */
int rabbit_cuda_refv2_fill_synthetic(rabbit_cuda_refv2 *c, uint64_t seed, float sigma);
int rabbit_cuda_refv2_free(rabbit_cuda_refv2 *c);
/* Empty the KV cache and restart at position 0 (rabbit_ref_v2_ctx_reset). */
int rabbit_cuda_refv2_reset(rabbit_cuda_refv2 *c);
/* One token at the next position (rabbit_ref_v2_ctx_step). HOST outputs, each
 * may be NULL: logits [vocab], hidden [hidden] (the final-normed h, as
 * rabbit_ref_v2_forward's out_hidden), argmax (lowest index among equal
 * maxima, forward_v2.c:415-421). Synchronous. */
int rabbit_cuda_refv2_step(rabbit_cuda_refv2 *c, int token_id, float *logits, float *hidden,
                           int *argmax);
/* n tokens in order (rabbit_ref_v2_ctx_prefill); outputs as for the last one. */
int rabbit_cuda_refv2_prefill(rabbit_cuda_refv2 *c, const int *token_ids, int n_tokens,
                              float *logits, float *hidden, int *argmax);
/* Greedy continuation (as rabbit_ref_v2_greedy, without re-running the
 * prefix): n_new tokens, each the argmax of the previous step, chained on the
 * device with no host round trip; out_ids[n_new] (host). Needs a step before
 * it; n_new <= 4096. */
int rabbit_cuda_refv2_generate(rabbit_cuda_refv2 *c, int n_new, int *out_ids);
/* Tokens processed since the last reset. */
int rabbit_cuda_refv2_position(const rabbit_cuda_refv2 *c);
/* Device time (CUDA events on the context's stream) from the first kernel to
 * the last one of the latest successful prefill / step / generate call, in ms;
 * the copies of its outputs to the host are outside it. */
int rabbit_cuda_refv2_device_ms(const rabbit_cuda_refv2 *c, float *ms);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* RABBIT_CUDA_H */
