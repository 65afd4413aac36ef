/*
 * kvm_recall.h — C ABI of the B200 history-recall path.
 *
 * The path scores every page of a paged KV history against the current
 * queries (page-softmax mass under GQA), selects the top-k pages with pinned
 * keep-pages, plans the residency delta, and stages the selected pages' K/V
 * bytes from mapped pinned host memory into a device paged cache.
 *
 * Conventions
 *  - Plain C: opaque handles, plain pointers and sizes, no exceptions.
 *  - Every entry point returns a kvm_status. Work is enqueued on the
 *    caller's CUDA stream (`stream` is a cudaStream_t; NULL = legacy default).
 *  - Device-side failures (a non-finite score, a bounded wait that ran out)
 *    are recorded in the context and reported by kvm_ctx_status().
 *  - One context per execution state; a context is never used by two host
 *    threads at once (the reference rule, src/adapter/llama-kvmem-hooks.h:54-57).
 *  - Device pointers must belong to the context's device.
 */
#ifndef KVM_RECALL_H
#define KVM_RECALL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 1..8 follow kvmem::MemoryErrorCode in order
 * (kvmem/include/kvmem/memory_contract.hpp:14-17); the rest stand for the
 * reference's std::invalid_argument / std::length_error / CUDA runtime_error. */
typedef enum kvm_status {
    KVM_OK = 0,
    KVM_ERR_INVALID_PLAN = 1,
    KVM_ERR_UNSUPPORTED = 2,
    KVM_ERR_BUDGET_EXCEEDED = 3,
    KVM_ERR_STALE = 4,
    KVM_ERR_PENDING = 5,
    KVM_ERR_TRANSFER_FAILED = 6,
    KVM_ERR_DISCONNECTED = 7,
    KVM_ERR_INVALID_SESSION = 8,
    KVM_ERR_INVALID_ARGUMENT = 9, /* geometry / operand rejected (std::invalid_argument) */
    KVM_ERR_LENGTH = 10,          /* exceeds workspace or launch range (std::length_error) */
    KVM_ERR_CUDA = 11,            /* CUDA runtime failure (std::runtime_error) */
    KVM_ERR_TIMEOUT = 12,         /* a bounded wait ran out */
    KVM_ERR_NONFINITE = 13        /* non-finite / negative score or non-finite FP16 operand
                                     (the reference's std::invalid_argument for those) */
} kvm_status;

/* Element / block encodings. */
typedef enum kvm_type {
    KVM_F32 = 0,
    KVM_F16 = 1,
    KVM_BF16 = 2,
    KVM_Q8_0 = 3, /* GGUF block of 32: {fp16 d; int8 qs[32]}              34 B */
    KVM_Q4_0 = 4, /* GGUF block of 32: {fp16 d; uint8 qs[16]} (nibble-8)  18 B */
    KVM_Q5_0 = 5  /* GGUF block of 32: {fp16 d; uint8 qh[4]; uint8 qs[16]} 22 B */
} kvm_type;

typedef struct kvm_ctx kvm_ctx;
typedef struct kvm_pool kvm_pool;

/* Current-step queries: element (l, r, h, d) at
 * data + l*layer_stride + r*row_stride + h*head_stride + d*sizeof(type).
 * type F32, F16 or BF16; device memory; data and strides 2-byte aligned.
 *
 * Sampled rows (the reference's `rows` list of
 * llama_kvmem_attention_cuda::score, src/adapter/llama-kvmem-attention-cuda.cu:146-190):
 * with row_ids != NULL, scored row i (i < rows) is query row row_ids[i] of the
 * tensor and reads mask row row_ids[i]; outputs are indexed by i. row_ids is a
 * HOST array of at most 512 entries, each below row_count (the rows the tensor
 * holds, the reference's q->ne[1]), else KVM_ERR_INVALID_ARGUMENT. Only
 * kvm_score_pages and kvm_score_pages_noalloc take a row list (others return
 * KVM_ERR_UNSUPPORTED). The listed query rows, and their mask rows, are packed
 * densely into the scoring workspace first: it then needs, beyond
 * kvm_score_workspace_bytes, layers*rows*q_heads*head_dim*sizeof(type) plus,
 * with a mask, rows*tokens*sizeof(mask type) bytes, each rounded up to 256. */
typedef struct kvm_query {
    const void* data;
    int32_t type;
    uint32_t rows;
    uint64_t layer_stride, row_stride, head_stride;
    const uint32_t* row_ids; /* optional host u32 [rows]; NULL = rows 0 .. rows-1 */
    uint32_t row_count;      /* rows held by the tensor (used with row_ids) */
    uint32_t reserved;
} kvm_query;

/* K history in HBM, token-major rows as in the engine's K cache view
 * [D, T, Hkv] (src/adapter/llama-kvmem-attention-cuda.cu:76): row (l, t, kvh)
 * at data + l*layer_stride + t*token_stride + kvh*head_stride.
 * The scorer needs the dense layout
 *   head_stride = row_bytes(type, D), token_stride = kv_heads * head_stride,
 * whole pages allocated (capacity_tokens >= pages * page_tokens) and 16-byte
 * aligned layer bases; anything else returns KVM_ERR_UNSUPPORTED, as the
 * reference's score() returns false for inputs it does not handle. */
typedef struct kvm_kcache {
    const void* data;
    int32_t type;
    uint32_t reserved;
    uint64_t layer_stride, token_stride, head_stride;
    uint64_t capacity_tokens;
} kvm_kcache;

/* One scoring problem. */
typedef struct kvm_score_desc {
    uint32_t layers, q_heads, kv_heads, head_dim;
    uint64_t tokens;      /* visible history: token t takes part iff t < tokens */
    uint32_t page_tokens; /* tokens per page ("block") */
    uint32_t groups;      /* 1: mass averaged over all query heads (reference `average`);
                             kv_heads: averaged over the query heads of each KV head */
    float scale;          /* logit scale; 0 selects 1/sqrt(head_dim) */
    float softcap;        /* > 0: logit = softcap * tanh(logit / softcap) */
    const void* mask;     /* optional device bias per (row, token), type mask_type (F32/F16);
                             a non-finite bias hides the token */
    int32_t mask_type;
    uint32_t reserved;
    uint64_t mask_row_stride; /* bytes between rows of the mask */
} kvm_score_desc;

/* ---------------------------------------------------------------- context */

/* Replaces the lazily created device/stream state of llama_kvmem_attention_cuda
 * (src/adapter/llama-kvmem-attention-cuda.cu:131-156) and of PageSoftmaxCuda
 * (kvmem/src/cuda/page_softmax.cu:156-175). */
int kvm_ctx_create(int device, kvm_ctx** out);
int kvm_ctx_destroy(kvm_ctx* ctx);
int kvm_ctx_device(const kvm_ctx* ctx);

/* Reads and clears the device-side status word (synchronises `stream`).
 * Replaces the exceptions the reference throws from inside score()/pick. */
int kvm_ctx_status(kvm_ctx* ctx, void* stream);

/* Workspace: bytes of device scratch kvm_score_pages needs for `rows` query
 * rows; the context grows its own allocation on demand unless a workspace has
 * been bound. Binding mirrors PageSoftmaxCuda's borrowed-workspace constructor
 * (kvmem/include/kvmem/page_softmax_cuda.hpp:13-15): the pointer must be
 * 256-byte aligned device memory of the context's device, and a later call
 * that would need more returns KVM_ERR_LENGTH before any launch
 * (kvmem/src/cuda/page_softmax.cu:34). */
size_t kvm_score_workspace_bytes(const kvm_score_desc* desc, uint32_t rows);
int kvm_ctx_bind_workspace(kvm_ctx* ctx, void* workspace, size_t bytes);
size_t kvm_ctx_device_bytes(const kvm_ctx* ctx);

/* ------------------------------------------------------------ page scoring */

/* Per-token page mass. Replaces llama_kvmem_attention_cuda::score
 * (src/adapter/llama-kvmem-attention-cuda.cu:146-193; kernels page_lse /
 * normalize / average at :59-121):
 *   lse[l,r,h,p]   = log sum_{t in p, t < tokens} exp(scale*<q_lrh, K_l,t,h/G> [softcap] + bias_rt)
 *   prob[l,r,h,p]  = exp(lse - M_lrh) / Z_lrh,  M, Z over all pages of layer l
 *   mass_rows[l,g,r,p] = mean over the query heads h of group g of prob[l,r,h,p]
 *   mass_mean[l,g,p]   = mean over r of mass_rows[l,g,r,p]
 * Outputs are device f32 arrays (either may be NULL):
 *   mass_rows [layers][groups][rows][pages], mass_mean [layers][groups][pages].
 * q8_0 / q4_0 / q5_0 keys are dequantised in registers. */
int kvm_score_pages(kvm_ctx* ctx, const kvm_score_desc* desc, const kvm_query* q, const kvm_kcache* k,
                    float* mass_rows, float* mass_mean, void* stream);

/* Page mass without allocating device memory. This entry point has no
 * counterpart in the reference. It computes exactly what kvm_score_pages
 * computes, but needs no context: its scratch (a status word and the page
 * log-sum-exp buffer) is a fixed 8 MiB array that the CUDA driver reserves on
 * each GPU that loads this library and keeps until the process exits. It is
 * meant for callers that must not call cudaMalloc while they score, such as an
 * engine whose device memory is all handed out up front by its own pool, or a
 * plugin host that forbids new device allocations after start-up.
 *  - Runs on the current device. The first call on a device looks up the
 *    array's device address; make that first call before any stream capture.
 *    The address is kept for the life of the process: after cudaDeviceReset
 *    (or anything else that tears down the device's primary context) it is
 *    stale, so do not call this entry point on that device again.
 *  - Needs layers * rows * q_heads * pages * 4 bytes (rounded up to 256) of
 *    scratch, plus the packed rows of a row list (see kvm_query), at most
 *    8 MiB - 256 B in all; larger problems return KVM_ERR_LENGTH before any
 *    launch.
 *  - Every call uses the same array; the status word is cleared on each call,
 *    the rest is fully rewritten. Calls that overlap on the GPU (two streams,
 *    two threads) race on it: order them on one stream.
 *  - A bounded device wait that runs out leaves the outputs undefined; this
 *    variant has no status read-back. */
int kvm_score_pages_noalloc(const kvm_score_desc* desc, const kvm_query* q, const kvm_kcache* k,
                            float* mass_rows, float* mass_mean, void* stream);

/* ------------------------------------------------------------ score frame */

/* The Query recall's score frame. Replaces kvmem::query_score_frame
 * (kvmem/src/host/graph_recall.cpp:269-293), host code (no device work):
 *   n = ceil(accepted / block_tokens) pages; page i starts at token
 *   i*block_tokens and holds min(block_tokens, accepted - start) tokens;
 *   score_mask[i] = 1, except that when n > budget and sink + recent < n the
 *   first `sink` and last `recent` pages are 0 (they are kept, not scored);
 *   transport_mask[i] = (n > budget), except 0 for every `fixed` page.
 * Outputs are host arrays of at least `capacity` entries (each may be NULL);
 * *n_out = n. block_tokens or budget 0, or a fixed page >= n, is
 * KVM_ERR_INVALID_ARGUMENT (the reference's std::invalid_argument); n above
 * capacity or UINT32_MAX is KVM_ERR_LENGTH. score_mask feeds kvm_meank_score
 * and kvm_layerwise_accumulate; the fixed pages are the pickers' keep list. */
int kvm_query_score_frame(uint64_t accepted, uint32_t block_tokens, uint32_t budget, uint32_t sink, uint32_t recent,
                          const uint32_t* fixed, uint32_t nfixed, uint64_t capacity, uint64_t* starts,
                          uint32_t* counts, uint8_t* score_mask, uint8_t* transport_mask, uint64_t* n_out);

/* The keep set of a Query selection. Replaces KvMemStore::query_fixed_blocks
 * (kvmem/src/host/kvmem_store.cpp:381-405), host code (no device work), for a
 * store of ceil(total_tokens / block_tokens) pages:
 *   budget 0 or pages <= budget: every page; else, each page with its whole
 *   media group (the closure of scored_media_group, ranges as in
 *   kvm_select_topk_media): the first `sink` pages, the page of the newest
 *   media range (the last of `ranges`, when it starts before total_tokens)
 *   and every `mandatory` page (required: a group that does not fit the
 *   budget is KVM_ERR_BUDGET_EXCEEDED, a page past the end
 *   KVM_ERR_INVALID_ARGUMENT), then the last `recent` pages, newest first,
 *   while they fit. out: host u32 [capacity], ascending; *n_out its length
 *   (KVM_ERR_LENGTH when capacity is too small). The result is the keep list
 *   of kvm_select_topk / kvm_select_topk_media. */
int kvm_query_fixed_blocks(uint64_t total_tokens, uint32_t block_tokens, uint32_t budget, uint32_t sink,
                           uint32_t recent, const uint32_t* ranges, uint32_t nranges, const uint32_t* mandatory,
                           uint32_t nmandatory, uint32_t* out, uint32_t capacity, uint32_t* n_out);

/* ------------------------------------------------------------------ top-k */

/* Budgeted top-k with keep pages, one selection per score row. Replaces
 * KvMemStore::pick_scored_blocks (kvmem/src/host/kvmem_store.cpp:418-451)
 * for candidates = all pages of the row and no media groups:
 *   keep pages first (an out-of-range keep is KVM_ERR_INVALID_ARGUMENT, more
 *   distinct keeps than `budget` is KVM_ERR_BUDGET_EXCEEDED, both before any
 *   launch), then pages by (score desc, page id desc) until `budget` pages are
 *   kept; output ascending.
 * scores: device f32 [nrows][score_stride]; keep: host u32 [nkeep].
 * out_ids: device u32 [nrows][out_stride], out_n: device u32 [nrows].
 * A non-finite score, or a negative one without signed_scores, sets
 * KVM_ERR_NONFINITE in the context status and that row's out_n to 0. */
int kvm_select_topk(kvm_ctx* ctx, const float* scores, uint32_t nrows, uint32_t pages, uint32_t score_stride,
                    const uint32_t* keep, uint32_t nkeep, uint32_t budget, int signed_scores,
                    uint32_t* out_ids, uint32_t* out_n, uint32_t out_stride, void* stream);

/* kvm_select_topk with the store's media groups. Replaces
 * KvMemStore::pick_scored_blocks (kvmem/src/host/kvmem_store.cpp:418-451)
 * with its media-group closure scored_media_group (:18-32), candidates = all
 * pages of the row: a page is admitted only together with its whole group (the
 * pages covered by a chain of overlapping media ranges, or the page alone).
 *   ranges: host u32 [nranges][2], token ranges [begin, end) of the media
 *   items; block_tokens: tokens per page.
 *   Keep pages first, each with its group, in the given order (an
 *   out-of-range keep is KVM_ERR_INVALID_ARGUMENT, groups that overflow
 *   `budget` KVM_ERR_BUDGET_EXCEEDED, both before any launch); then groups in
 *   the order of their best page by (score desc, page id desc), each kept if
 *   it still fits the budget and skipped otherwise; output ascending.
 * pages <= 16384 (else KVM_ERR_LENGTH). Other arguments, outputs and the
 * non-finite rule as kvm_select_topk. */
int kvm_select_topk_media(kvm_ctx* ctx, const float* scores, uint32_t nrows, uint32_t pages, uint32_t score_stride,
                          const uint32_t* keep, uint32_t nkeep, uint32_t budget, int signed_scores,
                          uint32_t block_tokens, const uint32_t* ranges, uint32_t nranges, uint32_t* out_ids,
                          uint32_t* out_n, uint32_t out_stride, void* stream);

/* ------------------------------------------------ post-scoring fusion */

/* Attention-feedback graph (kvmem::GraphSnapshot, kvmem/include/kvmem/graph_recall.hpp:47-99)
 * as plain arrays: rows in chunk order, each row's edges [edge_begin, edge_begin + edge_count),
 * positions are page-start tokens. has_messages = 0: no message spans (span coefficient 1). */
typedef struct kvm_graph_row {
    uint64_t source;
    uint64_t samples;
    uint32_t edge_begin;
    uint32_t edge_count;
} kvm_graph_row;
typedef struct kvm_graph_edge {
    uint64_t target;
    double mass;
} kvm_graph_edge;
typedef struct kvm_graph_span {
    uint64_t begin, end;
    uint32_t end_known;
    uint32_t reserved;
} kvm_graph_span;
typedef struct kvm_graph {
    uint32_t block_tokens;
    int32_t has_messages;
    uint64_t accepted_through, completed_through;
    const kvm_graph_row* rows;
    uint32_t nrows;
    uint32_t nedges;
    const kvm_graph_edge* edges;
    const kvm_graph_span* spans;
    uint32_t nspans;
    uint32_t reserved;
} kvm_graph;

/* One-hop propagation of positive score mass over the graph, on the device.
 * Replaces propagate_query_scores (kvmem/src/host/graph_recall.cpp:494-551):
 *   total = sum of max(raw, 0) over transport pages, seed = max(raw, 0) / total,
 *   each transport page sends total*seed*alpha/4*span_coefficient to its
 *   neighbour pages (start -+ block_tokens) and total*seed*alpha/2*mass/den
 *   along the edges of its completed graph row, out = max(min(raw, 0), result).
 * The transfer weights depend only on the graph and the frame: the host side
 * of this call builds them, the device applies them to the scores in double
 * precision. raw / out: device f32 [n]; starts / transport_mask: host [n]
 * (the frame of query_score_frame). Invalid inputs (alpha / cross outside
 * [0, 1], a graph of another accepted prefix, duplicate or unaligned starts, a
 * negative or non-finite edge mass) return KVM_ERR_INVALID_ARGUMENT before any
 * launch; a non-finite raw score sets KVM_ERR_NONFINITE in the context status
 * and out = raw. raw and out may be the same buffer; n <= 8192. The weights
 * are uploaded from pageable memory, so the call waits for `stream` to reach
 * the upload; they live in the context until its next propagation. */
int kvm_propagate_scores(kvm_ctx* ctx, const float* raw, uint32_t n, const uint64_t* starts,
                         const uint8_t* transport_mask, uint64_t accepted_through, const kvm_graph* graph,
                         double alpha, double cross, float* out, void* stream);

/* LRFU preview on the device. Replaces LrfuHistory::preview (kvmem/include/kvmem/lrfu.hpp:57-79):
 *   threshold = the value of rank min(n-1, floor((1-fraction)*n)) in ascending order
 *               (no gate when fraction == 1),
 *   out[i] = lambda * prev[i] (0 for i >= n_prev) + (s[i] >= threshold ? s[i] : min(s[i], 0)).
 * scores / out: device f32 [n]; prev: device f32 [n_prev] (the committed
 * history; NULL when n_prev = 0). lambda in [0, 1], fraction in (0, 1], else
 * KVM_ERR_INVALID_ARGUMENT; a non-finite score sets KVM_ERR_NONFINITE and
 * leaves out unwritten. Rank the result with kvm_select_topk(signed_scores = 1). */
int kvm_lrfu_preview(kvm_ctx* ctx, const float* scores, uint32_t n, const float* prev, uint32_t n_prev,
                     double lambda, double fraction, float* out, void* stream);

/* -------------------------------------------------------- residency + stage-in */

/* Device residency table for `rows` independent selections (one per layer or
 * per (layer, KV head)), each over `pages` logical pages and `slots` cache
 * slots. Holds the resident set that plan_residency consumes
 * (kvmem/src/host/memory_contract.cpp:135-150). All slots start free. */
int kvm_pool_create(kvm_ctx* ctx, uint32_t rows, uint32_t pages, uint32_t slots, kvm_pool** out);
int kvm_pool_destroy(kvm_pool* pool);
int kvm_pool_reset(kvm_pool* pool, void* stream);

/* Stage-in geometry: page (row i, page p) of plane j (0 = K, 1 = V; `planes`
 * of them) is `bytes[j]` contiguous bytes at host_base[j] + i*host_row_stride[j]
 * + p*host_page_stride[j] in mapped pinned host memory (cudaHostAlloc /
 * cudaHostRegister), written to dev_base[j] + i*dev_row_stride[j] +
 * slot*dev_slot_stride[j] in device memory. Replaces write_block_to_gpu's
 * destination arithmetic (src/adapter/llama-memory-kvmem.cpp:4475-4486). */
typedef struct kvm_stage_layout {
    uint32_t planes;
    uint32_t reserved;
    const void* host_base[2];
    uint64_t host_row_stride[2], host_page_stride[2];
    void* dev_base[2];
    uint64_t dev_row_stride[2], dev_slot_stride[2];
    uint64_t bytes[2];
} kvm_stage_layout;

/* Residency delta on the device for every row: evict = resident \ selected,
 * retain = resident ∩ selected, restore = selected \ resident (all resident /
 * all selected when force_reload), the plan_residency rule
 * (kvmem/src/host/memory_contract.cpp:135-150). Restored pages take the freed
 * slots in ascending page / slot order; the table is updated in place and the
 * restore list is kept for kvm_stagein_pool. sel_ids / sel_n are the outputs
 * of kvm_select_topk (device). Optional device outputs (may be NULL):
 * n_restore[rows], n_evict[rows]. */
int kvm_plan_residency(kvm_ctx* ctx, kvm_pool* pool, const uint32_t* sel_ids, const uint32_t* sel_n,
                       uint32_t sel_stride, int force_reload, uint32_t* n_restore, uint32_t* n_evict,
                       void* stream);

/* Device-initiated gather of every planned restore from mapped pinned host
 * memory into the device cache (replaces kvmem_stagein_enqueue_v +
 * kvmem_stagein_flush, src/adapter/llama-kvmem-stagein.cu:673-881, without
 * the pinned slab and the per-item D2D copies). `ctas` bounds the SMs the
 * gather occupies (0 = default). Asynchronous on `stream`. */
int kvm_stagein_pool(kvm_ctx* ctx, kvm_pool* pool, const kvm_stage_layout* layout, uint32_t ctas, void* stream);

/* Explicit copy list (the form of kvmem_stagein_enqueue_v / kvmem_d2d_batched,
 * src/adapter/llama-kvmem-stagein.cu:861,1006): n host ops {src, dst, bytes};
 * src may be mapped pinned host or device memory, dst device memory.
 * Asynchronous on `stream`: the ops are copied into one of the context's two
 * mapped pinned lists (the caller's array may be reused on return); a call
 * waits only when both lists are still read by gathers in flight (bounded:
 * KVM_ERR_TIMEOUT after 30 s). */
typedef struct kvm_copy {
    const void* src;
    void* dst;
    uint64_t bytes;
} kvm_copy;
int kvm_stagein_copies(kvm_ctx* ctx, const kvm_copy* ops, uint32_t n, uint32_t ctas, void* stream);

/* Bounded host wait for everything enqueued on `stream`; returns
 * KVM_ERR_TIMEOUT after timeout_us, else the context status
 * (replaces kvmem_stagein_sync_checked, src/adapter/llama-kvmem-stagein.cu:656). */
int kvm_stagein_wait(kvm_ctx* ctx, void* stream, uint64_t timeout_us);

/* ----------------------------------------------------------------- stage-out */

/* Device page bytes (K / V rows of a filled block) gathered into one of two
 * pinned host slots, alternately, so the host writes one batch into its store
 * while the GPU fills the other. Replaces the reverse slab of
 * src/adapter/llama-kvmem-stagein.h:48-55 (stagein.cu:883-1004), whose gather
 * kernel packs the regions into a 32 MiB device buffer and then copies it to
 * the slot with one D2H memcpy: here one kernel writes straight into the
 * mapped pinned slot. A handle is owned by one execution state, like a
 * kvm_ctx. */
typedef struct kvm_stageout kvm_stageout;

/* Two mapped pinned slots of slot_bytes (a multiple of 16; the reference uses
 * 32 MiB) and room for max_items regions per batch (the reference's
 * GATHER_MAX is 8192). */
int kvm_stageout_create(int device, uint64_t slot_bytes, uint32_t max_items, kvm_stageout** out);
int kvm_stageout_destroy(kvm_stageout* so);

/* Queues nbytes of device memory at dev_src for the next submit and returns
 * its byte offset in the slot (kvmem_stageout_enqueue, stagein.cu:883).
 * Offsets are rounded up to 16 bytes (the reference packs back to back), and
 * kvm_stageout_used() is the next item's offset, so a caller that reads the
 * offset from kvm_stageout_used() before enqueueing, as the reference's
 * harvest does (src/adapter/llama-memory-kvmem.cpp:4033-4036), finds its
 * bytes there. KVM_ERR_LENGTH when the batch is full (bytes or items): submit
 * and retry, as the reference's caller flushes its slab. */
int kvm_stageout_enqueue(kvm_stageout* so, const void* dev_src, uint64_t nbytes, uint64_t* offset);
uint64_t kvm_stageout_used(const kvm_stageout* so);

/* Enqueues the gather of the queued regions into the current slot on
 * `stream`, records the slot's event and switches to the other slot
 * (kvmem_stageout_submit, stagein.cu:907-973). *slot = the slot filled, or
 * -1 when nothing was queued. If the slot's previous batch is still in
 * flight, waits for it first (bounded: KVM_ERR_TIMEOUT after 30 s). `ctas`
 * bounds the SMs the gather occupies (0 = 32). */
int kvm_stageout_submit(kvm_stageout* so, uint32_t ctas, void* stream, int* slot);

/* Bounded host wait for a submitted slot (kvmem_stageout_wait,
 * stagein.cu:975-990): KVM_OK once its bytes are in host memory, KVM_OK for
 * slot -1, KVM_ERR_TIMEOUT after timeout_us. */
int kvm_stageout_wait(kvm_stageout* so, int slot, uint64_t timeout_us);

/* Host address of slot 0 or 1 (kvmem_stageout_slot_base, stagein.cu:992),
 * NULL otherwise. */
const uint8_t* kvm_stageout_slot_base(const kvm_stageout* so, int slot);

/* Drops the queued, not yet submitted regions (kvmem_stageout_clear,
 * stagein.cu:999-1004). */
int kvm_stageout_clear(kvm_stageout* so);

/* Pool introspection (tests): copies the device tables to host arrays
 * slot_of[rows][pages] (-1 = not resident) and page_of[rows][slots]. */
int kvm_pool_read(kvm_pool* pool, int32_t* slot_of, int32_t* page_of, void* stream);

/* ------------------------------------------------- working-set transfers */

/* A working-set transfer over a pool, the GPU side of kvmem::MemoryTransfer
 * (kvmem/include/kvmem/memory_contract.hpp:171-185) as kvmem::MemorySession
 * drives it (kvmem/src/host/memory_contract.cpp:245-365):
 *   prepare  -> start_spill -> poll until KVM_OK -> start_restore -> poll until
 *   KVM_OK -> publish, or abort at any point.
 * prepare reserves everything the transfer needs and plans the residency delta
 * (plan_residency, memory_contract.cpp:135-150) into a shadow copy of the
 * pool's tables: on any error nothing was started and the published view is
 * intact (the strong guarantee of MemoryBackend::prepare). One transfer per
 * pool at a time (KVM_ERR_PENDING otherwise); kvm_plan_residency and
 * kvm_stagein_pool must not be used on the pool while it is pending. */
typedef struct kvm_transfer kvm_transfer;
int kvm_transfer_prepare(kvm_ctx* ctx, kvm_pool* pool, const uint32_t* sel_ids, const uint32_t* sel_n,
                         uint32_t sel_stride, int force_reload, void* stream, kvm_transfer** out);

/* Spill: evicted pages whose host copy is stale (device u8 stale[rows][pages]
 * != 0; NULL = every host copy is current, nothing to copy) are written from
 * their device slots back to their host records (layout: host_base = mapped
 * pinned records, dev_base = the cache), before any slot is reused
 * (MemoryTransfer::start_spill; "start_spill cannot reclaim source pages"). */
int kvm_transfer_start_spill(kvm_transfer* t, const kvm_stage_layout* layout, const uint8_t* stale, uint32_t ctas,
                             void* stream);

/* Non-blocking poll of the current step (MemoryTransfer::poll): KVM_OK when it
 * is complete, KVM_ERR_PENDING while it runs, KVM_ERR_TRANSFER_FAILED on a CUDA
 * failure, KVM_ERR_INVALID_SESSION after an abort. */
int kvm_transfer_poll(kvm_transfer* t);

/* Restore: the planned pages are gathered from their host records into their
 * new slots (MemoryTransfer::start_restore, "called only after spill
 * completes": KVM_ERR_PENDING while the spill runs, KVM_ERR_INVALID_PLAN out of
 * order). From here on an abort cannot preserve the previous view. */
int kvm_transfer_start_restore(kvm_transfer* t, const kvm_stage_layout* layout, uint32_t ctas, void* stream);

/* Publish: once the restore is complete, the shadow tables become the pool's
 * view (MemoryTransfer::publish); synchronises `stream`. KVM_ERR_PENDING before
 * the restore completes; KVM_ERR_TRANSFER_FAILED (or KVM_ERR_BUDGET_EXCEEDED for a
 * selection larger than the pool) when a device step failed. */
int kvm_transfer_publish(kvm_transfer* t, void* stream);

/* Abort (MemoryTransfer::abort): drains every step already issued (bounded by
 * timeout_us, KVM_ERR_TIMEOUT otherwise) before anything is released, then
 * drops the transfer. *previous_view_preserved = 1 when no restore had started
 * (bytes and tables of the previous view intact:
 * AbortResult::PreviousViewPreserved), else 0 (SessionInvalidated). */
int kvm_transfer_abort(kvm_transfer* t, uint64_t timeout_us, int* previous_view_preserved);

/* Frees a published or aborted transfer (a pending one is aborted first);
 * KVM_ERR_TIMEOUT and nothing freed when device work could not be drained. */
int kvm_transfer_destroy(kvm_transfer* t);

/* Raw-K restore transform of stage-in, fused: each item's `tokens` packed K
 * rows (q8_0 or q4_0, n_head * head_dim elements per row, rows contiguous)
 * are dequantised, rotated by NeoX RoPE on the first n_rot dims of every head
 * at position pos0 + token (angle = position * theta[i], i < n_rot / 2),
 * Walsh-Hadamard transformed over every nrot-element chunk (scaled by
 * 1/sqrt(nrot); nrot = 0: no transform) and requantised into dst in the same
 * format. Replaces kvmem_stagein_enqueue_k + kvmem_stagein_flush
 * (src/adapter/llama-kvmem-stagein.cu:104-234, 499-671, 673-858): one launch
 * for all items, no f32 scratch, src may be mapped pinned host memory.
 * items / theta: host arrays; src / dst: device-accessible. type must be
 * KVM_Q8_0 or KVM_Q4_0 (else KVM_ERR_UNSUPPORTED); nrot in {0, 64, 128, 256,
 * 512} dividing n_head * head_dim, n_rot even and <= head_dim, head_dim a
 * multiple of 32, else KVM_ERR_INVALID_ARGUMENT. */
typedef struct kvm_restore_item {
    const void* src;
    void* dst;
    uint32_t tokens;
    int32_t pos0;
} kvm_restore_item;
int kvm_restore_k(kvm_ctx* ctx, int type, const kvm_restore_item* items, uint32_t n_items, uint32_t n_head,
                  uint32_t head_dim, uint32_t n_rot, const float* theta, uint32_t nrot, void* stream);

/* -------------------------------------------------------------- Mean-K path */

/* Mean-K producer: per-page K sums kept in HBM. Adds the K rows of tokens
 * [tok0, tok0 + n) of layers [0, layers) of `k` into
 *   sums[l][page][kv_heads*head_dim] (device f32, page = token / page_tokens,
 *   `pages` pages per layer), one f32 add per (token, element) in token order,
 * and the number of tokens added to each page into counts[page] (device u32,
 * once per page, not per layer). Replaces kvmem_meank_add + kvmem_meank_d2h +
 * kvmem_meank_zero (src/adapter/llama-kvmem-stagein.cu:270-316, 1072-1114),
 * which keep one open-block sum per layer that the host copies out on block
 * fill and uploads again on every scoring call (kvmem/src/cuda/page_softmax.cu:239-248):
 * here the table is directly the `sums` / `counts` input of kvm_meank_score.
 * Key types as the reference's producer (f32, f16, bf16) plus q8_0 / q4_0 /
 * q5_0 decoded as its key() (llama-kvmem-attention-cuda.cu:39-58). n = 0 is a
 * no-op; tokens past k->capacity_tokens or pages past `pages` are rejected. */
int kvm_meank_add(kvm_ctx* ctx, const kvm_kcache* k, uint32_t layers, uint32_t kv_heads, uint32_t head_dim,
                  uint64_t tok0, uint32_t n, uint32_t page_tokens, float* sums, uint32_t pages, uint32_t* counts,
                  void* stream);

/* Mean-K page softmax over device-resident per-page K sums. Replaces
 * PageSoftmaxCuda::score (kvmem/src/cuda/page_softmax.cu:202-280):
 *   mean[l,p]  = fp16(sum[l,p] * (1/count[p]))           (raw_kv_store.cpp:606-614, recall_fp16)
 *   logit      = scale * <fp16(q_lrh), mean[l,p,h/G]>    over pages with score_mask[p]
 *   Mean:  out[p] += prob / (active_layers * Hq)          (page_softmax.cu:88-96)
 *   Max:   out[p] += (max_{h in group} prob) / mass / (active_layers * Hkv)  (:100-133)
 * sums: device f32 [layers][pages][kv_heads*head_dim]; counts: device u32 [pages];
 * q: device f32 [layers][rows][q_heads*head_dim]; layer_rows: host u32 [layers]
 * (0 = absent layer); score_mask: host u8 [pages]; out: device f32 [pages]
 * (overwritten; disabled pages get 0). A non-finite or FP16-overflowing
 * operand returns KVM_ERR_NONFINITE (this call synchronises `stream` to read
 * the operand flag, as the reference does at page_softmax.cu:372-375). */
int kvm_meank_score(kvm_ctx* ctx, const float* sums, const uint32_t* counts, const float* q,
                    const uint32_t* layer_rows, uint32_t layers, uint32_t rows, uint32_t q_heads,
                    uint32_t kv_heads, uint32_t head_dim, uint32_t pages, const uint8_t* score_mask,
                    int aggregation, float scale, float* out, void* stream);

/* -------------------------------------------------- layerwise tile accumulation */

/* The layerwise (current-layer Query) recall scores a prefill's query rows in
 * tiles against one frozen page frame and sums the tiles' page masses (no mean
 * over rows): kvmem/src/host/layerwise_selection.cpp (layerwise_tile_scores
 * :32-75, LayerwiseQuerySelection::accumulate :283-296 and finish :298-309).
 * The accumulator is device FP64 [pages * (keep_halves ? 2 : 1)], zeroed by the
 * caller before the first tile.
 *
 * kvm_layerwise_accumulate adds one tile: tile is device f32 [pages * halves],
 * the scorer's masses over the frame (halves = 1) or over its half-page frame
 * (halves = 2: Mean-K records of half a page; elements 2i, 2i+1 are page i's
 * halves), e.g. the output of kvm_meank_score for the tile's rows of one layer.
 * With halves = 2 the halves are summed (left + right, in FP64) unless
 * keep_halves, which keeps both until kvm_layerwise_finish (keep_halves needs
 * halves = 2, else KVM_ERR_INVALID_ARGUMENT). score_mask: device u8 [pages].
 * Checks, all made before anything is added (a failure sets the context status
 * and leaves accum as it was): halves >= 0 with a finite sum and 0 on pages
 * outside the score mask (KVM_ERR_INVALID_ARGUMENT, the reference's
 * std::invalid_argument); every value finite, >= 0, keeping the sum finite and 0
 * outside the mask (KVM_ERR_INVALID_PLAN, the reference's MemoryError InvalidPlan).
 *
 * kvm_layerwise_finish writes scores[i] (device f32 [pages]) = accum[i], or with
 * keep_halves the larger of page i's halves (layerwise_max_page_scores :24-30),
 * ready for kvm_select_topk. */
int kvm_layerwise_accumulate(kvm_ctx* ctx, const float* tile, uint32_t pages, uint32_t halves, int keep_halves,
                             const uint8_t* score_mask, double* accum, void* stream);
int kvm_layerwise_finish(kvm_ctx* ctx, const double* accum, uint32_t pages, int keep_halves, float* scores,
                         void* stream);

/* ------------------------------------------------------------ fused step */

/* One decode-step recall: score -> per-row top-k -> residency plan -> stage-in,
 * pipelined over layer chunks so the stage-in of chunk i (side stream, PCIe)
 * overlaps the scoring of chunk i+1 (HBM). Selection rows are (layer, group)
 * pairs; the keep list applies to every row. When the stage-in of a step takes
 * longer than its scoring, the step ends about one first chunk's scoring after
 * the stage-in alone would: first_layers (< layers) makes the first chunk that
 * small and splits the other layers into chunks - 1 chunks.
 *   mass_mean: device f32 [layers*groups][pages]
 *   sel_ids: device u32 [layers*groups][budget], sel_n: device u32 [layers*groups]
 *   pool: residency table with rows = layers*groups (NULL: select only)
 *   layout: stage-in geometry for the pool (NULL: plan without copying)
 * Returns after enqueueing; completion is ordered on `stream`. */
typedef struct kvm_step_desc {
    const kvm_score_desc* score;
    const kvm_query* q;
    const kvm_kcache* k;
    const uint32_t* keep;
    uint32_t nkeep;
    uint32_t budget;
    uint32_t chunks;     /* layer chunks (0 = 4) */
    uint32_t stage_ctas; /* CTAs (128 threads each) of each gather launch (0 = 64) */
    int force_reload;    /* stage every selected page (cold worst case) */
    uint32_t first_layers; /* layers of the first chunk (0: all chunks equal) */
} kvm_step_desc;
int kvm_recall_step(kvm_ctx* ctx, const kvm_step_desc* step, kvm_pool* pool, const kvm_stage_layout* layout,
                    float* mass_mean, uint32_t* sel_ids, uint32_t* sel_n, void* stream);

/* --------------------------------------------------- page-range sharding */

/* One history partitioned by contiguous page ranges over several GPUs (the
 * reference has no multi-GPU selection): each rank scores its range and two
 * all-gathers merge. Per decode step, on every rank:
 *   1. kvm_shard_score_partial: page LSE of the rank's pages [page0, page0 +
 *      local_pages) (k: that range's K, dense as in kvm_kcache; desc->tokens is
 *      the GLOBAL visible token count) into the context workspace, and its
 *      softmax statistics stats[layers][rows][q_heads] = {max, sum exp(lse-max)}
 *      (device f32 pairs). All-gather stats over the ranks (rank order).
 *   2. kvm_shard_merge_stats: gathered [ranks][count] pairs -> global
 *      [count] {max, 1/sum}.
 *   3. kvm_shard_score_finish: local page masses normalised by the global
 *      statistics (outputs as kvm_score_pages, over local_pages). Nothing else
 *      may score on the context between steps 1 and 3 (the LSE stays in its
 *      workspace); KVM_ERR_STALE when no partial pass left one.
 *   4. kvm_shard_candidates: per score row the top-k local pages that are not
 *      keep pages (keep = GLOBAL page ids), as (score, global id) in
 *      cand_scores / cand_ids [nrows][k], padded with (-inf, 0xffffffff).
 *      All-gather both over the ranks.
 *   5. kvm_shard_merge: gathered [ranks][nrows][k] candidates -> per row the
 *      (budget - keeps) best by (score desc, id desc) plus the keep pages,
 *      ascending ids (out_ids [nrows][out_stride], out_n [nrows]): the same set
 *      as kvm_select_topk over the whole row when k >= budget - keeps. */
int kvm_shard_score_partial(kvm_ctx* ctx, const kvm_score_desc* desc, const kvm_query* q, const kvm_kcache* k,
                            uint32_t page0, uint32_t local_pages, float* stats, void* stream);
int kvm_shard_merge_stats(kvm_ctx* ctx, const float* gathered, uint32_t ranks, uint32_t count, float* global_stats,
                          void* stream);
int kvm_shard_score_finish(kvm_ctx* ctx, const kvm_score_desc* desc, uint32_t rows, uint32_t local_pages,
                           const float* global_stats, float* mass_rows, float* mass_mean, void* stream);
int kvm_shard_candidates(kvm_ctx* ctx, const float* scores, uint32_t nrows, uint32_t local_pages, uint32_t score_stride,
                         uint32_t page0, const uint32_t* keep, uint32_t nkeep, uint32_t k, float* cand_scores,
                         uint32_t* cand_ids, void* stream);
int kvm_shard_merge(kvm_ctx* ctx, const float* cand_scores, const uint32_t* cand_ids, uint32_t ranks, uint32_t nrows,
                    uint32_t k, const uint32_t* keep, uint32_t nkeep, uint32_t budget, uint32_t* out_ids,
                    uint32_t* out_n, uint32_t out_stride, void* stream);

/* One collective per step instead of two: every rank all-gathers the page LSE
 * of its range and finishes the whole rows itself with the single-GPU kernels.
 *   kvm_shard_page_lse: page LSE of the rank's pages [page0, page0 +
 *     local_pages) into lse (device f32 [layers][rows][q_heads][local_pages];
 *     k and desc as kvm_shard_score_partial). All-gather lse over the ranks
 *     and lay the ranges side by side in page order:
 *     [layers][rows][q_heads][pages of the whole history].
 *   kvm_page_mass_from_lse: softmax over the pages and the head / row means
 *     of a whole-history LSE (device f32 [layers][rows][q_heads][pages],
 *     pages = ceil(desc->tokens / desc->page_tokens)) -> mass_rows / mass_mean
 *     exactly as kvm_score_pages writes them. Then kvm_select_topk over the
 *     mean rows gives every rank the unsharded selection.
 * The gathered LSE is layers * rows * q_heads * pages * 4 bytes (config 2,
 * one layer: 48 KiB); no counterpart in the reference. */
int kvm_shard_page_lse(kvm_ctx* ctx, const kvm_score_desc* desc, const kvm_query* q, const kvm_kcache* k,
                       uint32_t page0, uint32_t local_pages, float* lse, void* stream);
int kvm_page_mass_from_lse(kvm_ctx* ctx, const kvm_score_desc* desc, uint32_t rows, const float* lse,
                           float* mass_rows, float* mass_mean, void* stream);

/* Stage-in of one rank's page range, to the owning decode GPU. The ranks of
 * a page-range partition keep identical residency tables (each plans the same
 * merged selection with kvm_plan_residency: the plan is deterministic), and
 * each rank gathers only the planned restores whose page lies in
 * [page0, page0 + page_count), from its own range's records over its own PCIe
 * link: page p of row i is at host_base[j] + i*host_row_stride[j] +
 * (p - page0)*host_page_stride[j]. dev_base[j] is the decode GPU's cache: on
 * the decode GPU its own memory, on the other ranks a peer mapping of it
 * (kvm_ipc_open), written over NVLink. Every writer fences its stores at system
 * scope before the gather completes, so a collective enqueued after it on
 * `stream` (on every rank) tells the decode GPU that its cache is complete.
 * No counterpart in the reference (its stage-in has one GPU,
 * src/adapter/llama-kvmem-stagein.cu:673-881). Asynchronous on `stream`. */
int kvm_shard_stagein(kvm_ctx* ctx, kvm_pool* pool, const kvm_stage_layout* layout, uint32_t page0,
                      uint32_t page_count, uint32_t ctas, void* stream);

/* Device memory shared between the processes of one node (one per GPU):
 * kvm_ipc_export writes an opaque handle (KVM_IPC_HANDLE_BYTES) naming dev_ptr
 * (any address inside a device allocation: the handle carries the offset);
 * kvm_ipc_open maps it in another process for `device`, with peer access
 * enabled, and returns the same address's mapping; kvm_ipc_close(device, that
 * pointer) unmaps it. Plain CUDA IPC (no multicast). */
#define KVM_IPC_HANDLE_BYTES 72
int kvm_ipc_export(const void* dev_ptr, void* handle);
int kvm_ipc_open(int device, const void* handle, void** dev_ptr);
int kvm_ipc_close(int device, void* dev_ptr);

/* ------------------------------------------- prefill page-LSE capture */

/* Causal prompt attention with the page LSE of sampled prompt rows captured in
 * the same pass. Replaces the engine's prompt attention with capture,
 * causal_softmax_attention_with_page_lse / try_dense_prompt_page_lse
 * (backends/patches/ninfer-prefill-page-lse-kv-coverage.patch:30-83, the
 * capture itself PromptPageLseRows in prompt_page_lse_tile.cuh, :891-1006 of
 * that patch), for fp16 / bf16 operands (the engine's FP8 KV row codec is not
 * part of the reference).
 *   Prompt row i (0 <= i < width) sits at position base + i and attends to
 *   cache keys 0 .. base + i (K and V of the prompt rows already appended).
 *   out[i][h]          = softmax_t(scale * <q_ih, K_t,h/G>) . V_t,h/G
 *   page_lse[s][h][p]  = log sum_{t in page p, t <= base + rows[s]} exp(scale * <q_rows[s],h, K_t,h/G>)
 *                        (-inf for a page with no visible key; natural log)
 * q: device [width] rows of q_heads x head_dim elements of `type`, rows
 * q_row_stride bytes apart, heads q_head_stride apart; k, v: the cache's K and
 * V views (kvm_kcache: token_stride, head_stride; the layer fields are
 * unused), capacity_tokens >= base + width; out: device, like q. page_lse:
 * device f32 [samples][q_heads][pages] (pages >= ceil((base + width) /
 * page_tokens)), or NULL with samples = 0 (attention only). sample_rows: host,
 * strictly ascending, < width, at most KVM_PREFILL_MAX_SAMPLES (the engine's
 * first capture took 64 rows in its launch parameters; its dynamic-sample form,
 * ninfer-prefill-page-lse-dynamic-samples.patch:22-35, takes as many as the
 * scratch holds, from device memory, as this one does above 64 rows: that
 * table is staged from the host array, which waits for the stream's earlier
 * work; up to 64 rows travel in the launch and need no copy). head_dim 128 or
 * 256; page_tokens 16, 32 or a multiple of 64; all base pointers and strides
 * 16-byte aligned. kvm_page_mass_from_lse(desc = {layers 1, q_heads, kv_heads,
 * page_tokens, tokens = pages * page_tokens, groups 1}, rows = samples) turns
 * page_lse into the reference's attention_page_mass_from_lse output (softmax
 * over pages, mean over heads). Long histories split each row tile's keys
 * into chunks merged by a second pass whose partial rows live in the context's
 * scoring workspace (as kvm_score_pages's LSE does). Asynchronous on `stream`. */
#define KVM_PREFILL_MAX_SAMPLES 4096
typedef struct kvm_prefill_desc {
    uint32_t q_heads, kv_heads, head_dim;
    int32_t type;         /* KVM_F16 or KVM_BF16: q, k, v and out */
    uint64_t base;        /* cache tokens before prompt row 0 */
    uint32_t width;       /* prompt rows */
    float scale;          /* logit scale; 0 selects 1/sqrt(head_dim) */
    uint32_t page_tokens; /* capture page size */
    uint32_t pages;       /* capture columns per (sample, head) */
    uint32_t samples;     /* sampled rows (0: no capture) */
    uint32_t reserved;
    const uint32_t* sample_rows;
} kvm_prefill_desc;
int kvm_prefill_attention(kvm_ctx* ctx, const kvm_prefill_desc* desc, const void* q, uint64_t q_row_stride,
                          uint64_t q_head_stride, const kvm_kcache* k, const kvm_kcache* v, void* out,
                          uint64_t out_row_stride, uint64_t out_head_stride, float* page_lse, void* stream);

/* Bytes of one D-element row of `type` (0 for an unknown type). */
uint64_t kvm_row_bytes(int type, uint32_t dim);

/* Kernel launches this context has issued (for launch accounting). */
uint64_t kvm_ctx_launches(const kvm_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif
