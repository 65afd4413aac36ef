// C ABI of the B200 history-recall path (declarations: include/kvm_recall.h).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "layerwise.cuh"
#include "lse_launch.cuh"
#include "page_mass_tc.cuh"
#include "meank.cuh"
#include "page_norm.cuh"
#include "post.cuh"
#include "prefill_attn.cuh"
#include "restore.cuh"
#include "rows.cuh"
#include "select.cuh"
#include "shard.cuh"
#include "stagein.cuh"

using namespace kvmb;

struct kvm_transfer;

struct kvm_pool {
    kvm_ctx* ctx = nullptr;
    PoolView view{};
    void* mem = nullptr;
    kvm_transfer* pending = nullptr;  // the prepared, not yet published or aborted transfer
};

// A working-set transfer over a pool (kvm_transfer_*): the plan, the restore
// lists and the new residency tables live in a shadow copy until publish.
struct kvm_transfer {
    kvm_ctx* ctx = nullptr;
    kvm_pool* pool = nullptr;
    void* mem = nullptr;  // shadow tables, same layout as the pool's
    PoolView shadow{};
    int force = 0;
    enum Phase { Prepared, Spilling, Restoring, Published, Aborted } phase = Prepared;
    bool restore_started = false;
    bool drained = true;  // false when an abort could not drain the device work
    cudaEvent_t planned = nullptr, spill_done = nullptr, restore_done = nullptr;
    // The transfer's own device status word (inside `mem`): its plan reports
    // there, so unrelated work on the context neither fails nor is hidden by it.
    kvmb::DeviceStatus* status = nullptr;
};

namespace {

struct DeviceGuard {
    int previous = -1;
    bool ok = false;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&previous) != cudaSuccess) return;
        ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (previous >= 0) cudaSetDevice(previous);
    }
};

#define KVM_CUDA(call)               \
    do {                             \
        if ((call) != cudaSuccess) { \
            cudaGetLastError();      \
            return KVM_ERR_CUDA;     \
        }                            \
    } while (0)

#define KVM_TRY(call)                  \
    do {                               \
        const int rc_ = (call);        \
        if (rc_ != KVM_OK) return rc_; \
    } while (0)

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

// Defined with the transfer entry points below (inside their extern "C" block).
extern "C" {
namespace {
int transfer_drain(kvm_transfer* t, uint64_t timeout_us);
}
}

namespace {

int ensure_ws(kvm_ctx* c, size_t bytes) {
    if (bytes <= c->ws_bytes) return KVM_OK;
    if (c->ws_borrowed) return KVM_ERR_LENGTH;
    if (c->ws) {
        cudaDeviceSynchronize();
        cudaFree(c->ws);
        c->ws = nullptr;
        c->ws_bytes = 0;
    }
    KVM_CUDA(cudaMalloc(&c->ws, bytes));
    c->ws_bytes = bytes;
    return KVM_OK;
}

int ensure_small(kvm_ctx* c, size_t bytes) {
    if (bytes <= c->small_bytes) return KVM_OK;
    if (c->small) {
        cudaDeviceSynchronize();
        cudaFree(c->small);
        c->small = nullptr;
        c->small_bytes = 0;
        c->keep_valid = false;
    }
    const size_t want = std::max<size_t>(bytes, 1 << 16);
    KVM_CUDA(cudaMalloc(&c->small, want));
    c->small_bytes = want;
    return KVM_OK;
}

// The per-call table buffer is rewritten by the next call that needs one: first
// wait (host side) until the last kernel that read it has finished, so calls on
// different streams never overwrite a table still in use.
int ensure_aux(kvm_ctx* c, size_t bytes) {
    if (!c->aux_done) KVM_CUDA(cudaEventCreateWithFlags(&c->aux_done, cudaEventDisableTiming));
    if (c->aux_pending) {
        KVM_CUDA(cudaEventSynchronize(c->aux_done));
        c->aux_pending = false;
    }
    if (bytes <= c->aux_bytes) return KVM_OK;
    if (c->aux) {
        cudaDeviceSynchronize();
        cudaFree(c->aux);
        c->aux = nullptr;
        c->aux_bytes = 0;
    }
    const size_t want = std::max<size_t>(align256(bytes), 1 << 16);
    KVM_CUDA(cudaMalloc(&c->aux, want));
    c->aux_bytes = want;
    return KVM_OK;
}

// Marks the table buffer in use until the work enqueued on `s` so far is done.
int aux_release(kvm_ctx* c, cudaStream_t s) {
    KVM_CUDA(cudaEventRecord(c->aux_done, s));
    c->aux_pending = true;
    return KVM_OK;
}

// span_coefficient (kvmem/src/host/graph_recall.cpp:234-246).
double span_coefficient(const kvm_graph* g, uint64_t a, uint64_t b, double cross) {
    if (!g->has_messages) return 1.0;
    const uint64_t begin = std::min(a, b), end = std::max(a, b) + g->block_tokens;
    for (uint32_t i = 0; i < g->nspans; ++i)
        if (g->spans[i].begin <= begin && end <= g->spans[i].end) return 1.0;
    for (uint32_t i = 0; i < g->nspans; ++i) {
        const auto& sp = g->spans[i];
        if ((begin < sp.begin && sp.begin < end) || (sp.end_known && begin < sp.end && sp.end < end)) return cross;
    }
    return 1.0;
}

// The keep list lives at the start of the small scratch (first 4 KiB + list);
// it is re-uploaded only when it changes, by a synchronous copy, so the host
// array may be reused as soon as the call returns.
size_t keep_area(const kvm_ctx* c) { return align256(4096 + c->keep_cached.size() * 4); }

int upload_keep(kvm_ctx* c, const uint32_t* keep, uint32_t nkeep) {
    if (c->keep_valid && c->keep_cached.size() == nkeep &&
        (nkeep == 0 || std::memcmp(c->keep_cached.data(), keep, size_t(nkeep) * 4) == 0))
        return KVM_OK;
    KVM_TRY(ensure_small(c, align256(4096 + size_t(nkeep) * 4)));
    if (nkeep) {
        cudaDeviceSynchronize();  // no launch may still read the previous list
        KVM_CUDA(cudaMemcpy(c->small, keep, size_t(nkeep) * 4, cudaMemcpyHostToDevice));
    }
    c->keep_cached.assign(keep, keep + nkeep);
    c->keep_valid = true;
    return KVM_OK;
}

struct LseConfig {
    uint32_t lpr = 0, tpc = 0, chunk_bytes = 0, chunks = 0, row_bytes = 0, stage_stride = 0;
    size_t smem = 0;
    // Tensor-core scorer (fp16 / q8_0 / q4_0 keys, 1/2/4/8 KV heads), when usable.
    bool mma = false;
    uint32_t mma_tpc = 0, mma_chunk_bytes = 0, mma_chunks = 0, mma_stage_stride = 0, mma_stages = 0, mma_slot = 0;
    size_t mma_smem = 0;
    // Quantised-key scorer (q8_0 / q4_0, page_mass_q.cuh), when usable.
    bool q = false;
    uint32_t q_tpc = 0, q_chunks = 0, q_slot = 0, q_hpg = 0, q_groups = 0, q_stage_stride = 0, q_stages = 0, q_tx = 0;
    size_t q_smem = 0;
    // tcgen05 scorer (fp16 keys, 16..160 query vectors per KV head), when usable.
    bool tc = false;
    bool head_major = false;  // K is a head-major mirror (only the tcgen05 scorer reads it)
    int tc_ka = 0, tc_lm = 0;
    uint32_t tc_stages = 0, tc_pass_nv = 0;  // tc_pass_nv: vectors per launch (the last may have fewer)
    size_t tc_smem = 0;
};

// Scorer selection: KVM_SCORER=simt forces the FP32 SIMT kernel and
// KVM_SCORER=mma the mma.sync kernel wherever it applies; KVM_SCORER=tc
// requires the tcgen05 kernel (KVM_ERR_UNSUPPORTED where it does not apply);
// KVM_SCORER=mma_generic scores q8_0 / q4_0 keys with the fp16 mma.sync kernel
// instead of the integer-tensor-core one. The tests use them to check every
// kernel against the oracle; anything else picks the tcgen05 kernel, then the
// quantised-key kernel, then the mma.sync kernel, wherever they apply.
bool scorer_is(const char* name) {
    const char* e = std::getenv("KVM_SCORER");
    return e && std::strcmp(e, name) == 0;
}
bool force_simt() { return scorer_is("simt"); }

// tcgen05 scorer: fp16 K, head_dim 64 / 128 / 256, 16 or more query vectors
// per KV head (rows x group), pages of 32 / 64 / 128 tokens or multiples of
// 128, a token range addressable by 32-bit TMA coordinates, and room for at
// least two K stages next to the query tiles. One launch scores up to 160
// vectors (128 at head_dim 256, whose query operand leaves no shared memory
// for a packed second tile); more are split into equal passes, each reading K
// once, so a batch of sampled rows costs ceil(vectors / 160) reads of K rather
// than the mma.sync kernel's ceil(vectors / 8).
void plan_tc(const kvm_score_desc* d, const kvm_query* q, const kvm_kcache* k, LseConfig* cfg) {
    if (force_simt() || scorer_is("mma")) return;
    if (k->type != KVM_F16 || (d->head_dim != 64 && d->head_dim != 128 && d->head_dim != 256)) return;
    const uint64_t nv = uint64_t(q->rows) * (d->q_heads / d->kv_heads);
    if (nv < 16) return;
    const uint32_t pt = d->page_tokens;
    if (pt % 32 || (pt < 128 && 128 % pt) || (pt > 128 && pt % 128)) return;
    const uint64_t pages = (d->tokens + pt - 1) / pt;
    if (pages * pt + 128 > 0x7fffffffull) return;
    const int ka = int(d->head_dim / 64);
    const uint64_t per_launch = ka == 4 ? uint64_t(kTcTile) : uint64_t(kTcMaxVectors);
    const uint64_t passes = (nv + per_launch - 1) / per_launch;
    const uint32_t pass_nv = uint32_t((nv + passes - 1) / passes);
    const int lm = tc_layout_for(pass_nv);
    const size_t fixed = tc_smem_bytes(ka, lm, 0);
    const size_t stage = size_t(ka) * kTcAtomBytes;
    if (fixed + 2 * stage > kTcSmemMax) return;
    const uint32_t stages = uint32_t(std::min<size_t>(kTcMaxStages, (kTcSmemMax - fixed) / stage));
    cfg->tc = true;
    cfg->tc_ka = ka;
    cfg->tc_lm = lm;
    cfg->tc_pass_nv = pass_nv;
    cfg->tc_stages = stages;
    cfg->tc_smem = tc_smem_bytes(ka, lm, stages);
}

void plan_mma(const kvm_score_desc* d, const kvm_kcache* k, LseConfig* cfg) {
    if (force_simt()) return;
    if (k->type != KVM_F16 && k->type != KVM_Q8_0 && k->type != KVM_Q4_0) return;
    if (8 % d->kv_heads) return;
    const uint64_t row_all = k->token_stride;  // bytes of one token across KV heads
    // Every consumer warp needs an octet of one KV head in every chunk.
    uint32_t tpc = std::max<uint32_t>(8, 64 / d->kv_heads);
    while (tpc <= d->page_tokens && (d->page_tokens % tpc || (uint64_t(tpc) * row_all) % 16)) tpc <<= 1;
    if (tpc > d->page_tokens || d->page_tokens % tpc) return;
    while (tpc * 2 <= d->page_tokens && d->page_tokens % (tpc * 2) == 0 && uint64_t(tpc) * 2 * row_all <= 16384)
        tpc <<= 1;
    const uint64_t cb = uint64_t(tpc) * row_all;
    if (cb > 65536) return;
    // Quantised keys: one shared-memory slot per token, its stride 16 bytes past a
    // multiple of 128 so the 8 tokens of an octet start in different bank groups.
    uint64_t slot = row_all;
    if (k->type != KVM_F16) {
        if (row_all % 16) return;  // per-token bulk copies need 16-byte multiples
        slot = (row_all + 127) / 128 * 128 + 16;
        if (slot - 128 >= row_all) slot -= 128;
    }
    const uint64_t stage_bytes = k->type != KVM_F16 ? uint64_t(tpc) * slot : cb;
    cfg->mma = true;
    cfg->mma_tpc = tpc;
    cfg->mma_chunk_bytes = uint32_t(cb);
    cfg->mma_chunks = d->page_tokens / tpc;
    cfg->mma_slot = uint32_t(slot);
    cfg->mma_stage_stride = uint32_t((stage_bytes + 16 + 127) / 128 * 128);
    cfg->mma_stages = uint32_t(std::max<uint64_t>(2, std::min<uint64_t>(kMmaMaxStages, (110 * 1024) / cfg->mma_stage_stride)));
    cfg->mma_smem = size_t(cfg->mma_stages) * cfg->mma_stage_stride + 2 * kMmaMaxStages * sizeof(uint64_t) +
                    2 * 2 * kLseConsumerWarps * 8 * sizeof(float) + 16;
}

// Quantised-key scorer: the K heads of a token are split into the largest
// groups of hpg heads whose row bytes are a multiple of 16 and fit one TMA box
// row (<= 255 u64 elements with the pad) -- normally all heads of a token, one
// ring, so each chunk is one contiguous run of token rows in HBM; each group
// has its own ring, its rows land in shared memory at a stride of an odd
// number of 16-byte units (pad = 0 or 16 zero-filled bytes). A chunk is the
// largest of 32, 16 or 8 tokens per warp of a KV head whose stage stays within
// 40 KiB with two stages fitting; the rings and the kernel's other shared
// memory fill ~112 KiB so two CTAs share an SM. (Config 3, q8_0 D 256 x 4 KV
// heads: one ring of two 32-token, 35 KiB stages reads K at 0.99 of the
// measured copy bandwidth, where four per-head rings of 16-token stages read it
// at 0.74 and one ring of five 16-token stages at 0.78.)
void plan_q(const kvm_score_desc* d, const kvm_kcache* k, LseConfig* cfg) {
    if (force_simt() || scorer_is("mma_generic")) return;
    if (k->type != KVM_Q8_0 && k->type != KVM_Q4_0) return;
    const uint32_t kvh = d->kv_heads;
    if (kvh == 0 || 8 % kvh) return;
    const uint64_t rb = row_bytes_of(k->type, d->head_dim);
    uint32_t hpg = 0, pad = 0;
    for (uint32_t h = 1; h <= kvh; h <<= 1) {
        const uint64_t gb = h * rb;
        if (kvh % h || gb % 16) continue;
        const uint32_t pd = (gb / 16) % 2 ? 0 : 16;
        if ((gb + pd) / 8 > 255) break;
        hpg = h;
        pad = pd;
    }
    if (!hpg) return;
    const uint32_t slot = uint32_t(hpg * rb + pad), groups = kvh / hpg;
    const uint64_t budget = 112 * 1024 - q_smem_extra();
    auto stages_for = [&](uint32_t tpc) {
        const uint32_t stride = uint32_t((uint64_t(tpc) * slot + 127) / 128 * 128);
        return uint32_t(std::min<uint64_t>(kMmaMaxStages, budget / (uint64_t(groups) * stride)));
    };
    // Chunks of 4, 2 or 1 octets per warp: the largest whose stages stay within
    // 40 KiB and of which two fit (fewer, larger chunks mean fewer barrier
    // round trips and refills per byte).
    const uint32_t base = 8 * (kLseConsumerWarps / kvh);
    uint32_t tpc = base;
    for (uint32_t mult = 4; mult >= 2; mult /= 2) {
        const uint32_t t = mult * base;
        if (d->page_tokens % t == 0 && t <= 256 && uint64_t(t) * slot <= 40 * 1024 && stages_for(t) >= 2) {
            tpc = t;
            break;
        }
    }
    if (d->page_tokens % tpc || tpc > 256 || groups > uint32_t(kQMaxGroups)) return;
    const uint64_t stage = uint64_t(tpc) * slot;
    const uint32_t stride = uint32_t((stage + 127) / 128 * 128);
    const uint32_t stages = stages_for(tpc);
    if (stages < 2) return;
    cfg->q = true;
    cfg->q_tpc = tpc;
    cfg->q_chunks = d->page_tokens / tpc;
    cfg->q_slot = slot;
    cfg->q_hpg = hpg;
    cfg->q_groups = groups;
    cfg->q_stage_stride = stride;
    cfg->q_stages = stages;
    cfg->q_tx = uint32_t(stage);
    cfg->q_smem = size_t(groups) * stages * stride + q_smem_extra();
}

bool supported_type(int t) { return t >= KVM_F32 && t <= KVM_Q5_0; }

int validate_score(const kvm_score_desc* d, const kvm_query* q, const kvm_kcache* k, LseConfig* cfg) {
    if (!d || !q || !k || !q->data || !k->data) return KVM_ERR_INVALID_ARGUMENT;
    if (!d->layers || !d->q_heads || !d->kv_heads || !d->head_dim || !d->page_tokens || !q->rows ||
        d->q_heads % d->kv_heads)
        return KVM_ERR_INVALID_ARGUMENT;
    if (d->groups != 1 && d->groups != d->kv_heads) return KVM_ERR_INVALID_ARGUMENT;
    if (q->type != KVM_F32 && q->type != KVM_F16 && q->type != KVM_BF16) return KVM_ERR_UNSUPPORTED;
    if (!supported_type(k->type)) return KVM_ERR_UNSUPPORTED;
    if (d->mask && d->mask_type != KVM_F32 && d->mask_type != KVM_F16) return KVM_ERR_UNSUPPORTED;
    const uint32_t D = d->head_dim;
    if (D != 64 && D != 128 && D != 256) return KVM_ERR_UNSUPPORTED;
    const uint32_t lpr = D / 8;
    const uint32_t ng = kLseConsumerWarps * 32 / lpr;
    if (ng % d->kv_heads) return KVM_ERR_UNSUPPORTED;
    const uint64_t rb = row_bytes_of(k->type, D);
    const uint64_t pages = (d->tokens + d->page_tokens - 1) / d->page_tokens;
    if (!pages) return KVM_ERR_INVALID_ARGUMENT;
    if (k->capacity_tokens < pages * d->page_tokens) return KVM_ERR_UNSUPPORTED;
    // Token-major (the engine's cache view) for every scorer; head-major (each KV
    // head's rows contiguous, a score mirror) for the tcgen05 scorer.
    const bool token_major = k->head_stride == rb && k->token_stride == rb * d->kv_heads;
    const bool head_major = !token_major && d->kv_heads > 1 && k->token_stride == rb && !(k->head_stride & 15) &&
                            k->head_stride >= k->capacity_tokens * rb;
    if (!token_major && !head_major) return KVM_ERR_UNSUPPORTED;
    const uint64_t page_bytes = uint64_t(d->page_tokens) * k->token_stride;
    if ((reinterpret_cast<uintptr_t>(k->data) & 15) || (k->layer_stride & 15) || (page_bytes & 15))
        return KVM_ERR_UNSUPPORTED;
    const uint64_t layer_span = head_major ? d->kv_heads * k->head_stride : pages * page_bytes;
    if (d->layers > 1 && k->layer_stride < layer_span) return KVM_ERR_INVALID_ARGUMENT;
    cfg->head_major = head_major;
    if (pages > 0x7fffffffull || uint64_t(d->layers) * pages > 0x7fffffffull) return KVM_ERR_LENGTH;
    if (q->rows * uint64_t(d->q_heads / d->kv_heads) > 0x7fffffffull) return KVM_ERR_LENGTH;
    // Tokens per ring chunk: the largest power of two dividing page_tokens whose
    // chunk is a multiple of 16 bytes and stays within 16 KiB (32 KiB when a
    // single token row set is that large).
    uint32_t tpc = 0;
    for (uint32_t t = 1; t <= d->page_tokens; t <<= 1) {
        if (d->page_tokens % t) break;
        const uint64_t cb = uint64_t(t) * k->token_stride;
        if (cb > 32768) break;
        if (cb % 16 == 0 && (tpc == 0 || cb <= 16384)) tpc = t;
    }
    if (!tpc) return KVM_ERR_UNSUPPORTED;
    cfg->lpr = lpr;
    cfg->tpc = tpc;
    cfg->chunk_bytes = uint32_t(uint64_t(tpc) * k->token_stride);
    cfg->chunks = d->page_tokens / tpc;
    cfg->row_bytes = uint32_t(rb);
    cfg->stage_stride = uint32_t((cfg->chunk_bytes + 16 + 127) / 128 * 128);
    cfg->smem = size_t(kLseStages) * cfg->stage_stride + 2 * kLseStages * sizeof(uint64_t) +
                2 * 2 * size_t(ng) * 8 * sizeof(float) + 16;
    if (!head_major) {
        plan_mma(d, k, cfg);
        plan_q(d, k, cfg);
    }
    plan_tc(d, q, k, cfg);
    if (scorer_is("tc") && !cfg->tc) return KVM_ERR_UNSUPPORTED;  // strict: the tcgen05 kernel or nothing
    if (head_major && !cfg->tc) return KVM_ERR_UNSUPPORTED;       // only the tcgen05 scorer reads head-major K
    return KVM_OK;
}

size_t lse_bytes(const kvm_score_desc* d, uint32_t layers, uint32_t rows) {
    const uint64_t pages = (d->tokens + d->page_tokens - 1) / d->page_tokens;
    return align256(size_t(layers) * rows * d->q_heads * pages * sizeof(float));
}

int launch_lse_mma(kvm_ctx* c, int kt, const LseParams& p, int kk, size_t smem, cudaStream_t s) {
    switch (kt) {
        case KVM_F16: return launch_lse_mma_kt<KVM_F16>(c, p, kk, smem, s);
        case KVM_Q8_0: return launch_lse_mma_kt<KVM_Q8_0>(c, p, kk, smem, s);
        case KVM_Q4_0: return launch_lse_mma_kt<KVM_Q4_0>(c, p, kk, smem, s);
        default: return KVM_ERR_UNSUPPORTED;
    }
}

// cuTensorMapEncodeTiled from the driver (the library links only the runtime).
using TensorMapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                       const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

TensorMapEncodeFn tensor_map_encoder() {
    static TensorMapEncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TensorMapEncodeFn>(ptr);
        else
            cudaGetLastError();
    });
    return fn;
}

// cuMemGetAddressRange from the driver: the allocation that holds a device
// pointer (CUDA IPC handles name whole allocations).
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddressRangeFn>(ptr);
        else
            cudaGetLastError();
    });
    return fn;
}

// Peer mappings opened by kvm_ipc_open: returned pointer -> mapped allocation base.
std::mutex& ipc_mutex() {
    static std::mutex m;
    return m;
}
std::unordered_map<void*, void*>& ipc_bases() {
    static std::unordered_map<void*, void*> m;
    return m;
}

// 4-D tensor map of fp16 K of layers [0, nl) from `base`: dims (head_dim,
// kv_heads, tokens, layers), box 64 dims x 1 head x 128 tokens x 1 layer, or
// for a head-major mirror (head_dim, tokens, kv_heads, layers), box 64 dims x
// 128 tokens x 1 head x 1 layer (strides increase in both); 128-byte swizzle;
// reads past the allocated tokens fill zeros.
int encode_k_map(const kvm_score_desc* d, const kvm_kcache* k, const void* base, uint32_t nl, bool head_major,
                 CUtensorMap* map) {
    TensorMapEncodeFn enc = tensor_map_encoder();
    if (!enc) return KVM_ERR_CUDA;
    uint64_t cap = std::min<uint64_t>(k->capacity_tokens, 0x7fffffffull);
    if (head_major) cap = std::min<uint64_t>(cap, k->head_stride / k->token_stride);  // heads never overlap
    else if (nl > 1) cap = std::min<uint64_t>(cap, k->layer_stride / k->token_stride);  // layers never overlap
    const uint64_t span = head_major ? uint64_t(d->kv_heads) * k->head_stride : cap * k->token_stride;
    const uint64_t lstride = nl > 1 ? k->layer_stride : span;
    cuuint64_t dims[4] = {d->head_dim, d->kv_heads, cap, nl};
    cuuint64_t strides[3] = {k->head_stride, k->token_stride, lstride};
    cuuint32_t box[4] = {64, 1, uint32_t(kTcTile), 1};
    if (head_major) {
        dims[1] = cap, dims[2] = d->kv_heads;
        strides[0] = k->token_stride, strides[1] = k->head_stride;
        box[1] = uint32_t(kTcTile), box[2] = 1;
    }
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? KVM_OK : KVM_ERR_CUDA;
}

// 4-D tensor map of quantised K of layers [0, nl) from `base`, in u64 units:
// dims (group row bytes / 8, head groups, tokens, layers), box (row + pad
// columns, 1 group, tpc tokens, 1 layer); the pad columns lie past the
// group's row and read as zeros.
int encode_q_map(const kvm_score_desc* d, const kvm_kcache* k, const void* base, uint32_t nl, const LseConfig& cfg,
                 CUtensorMap* map) {
    TensorMapEncodeFn enc = tensor_map_encoder();
    if (!enc) return KVM_ERR_CUDA;
    const uint64_t gb = uint64_t(cfg.q_hpg) * k->head_stride;
    uint64_t cap = std::min<uint64_t>(k->capacity_tokens, 0x7fffffffull);
    if (nl > 1) cap = std::min<uint64_t>(cap, k->layer_stride / k->token_stride);
    const cuuint64_t dims[4] = {gb / 8, cfg.q_groups, cap, nl};
    const uint64_t lstride = nl > 1 ? k->layer_stride : cap * k->token_stride;
    const cuuint64_t strides[3] = {cfg.q_groups > 1 ? gb : k->token_stride, k->token_stride, lstride};
    const cuuint32_t box[4] = {cfg.q_slot / 8, 1, cfg.q_tpc, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? KVM_OK : KVM_ERR_CUDA;
}

int launch_lse_q(kvm_ctx* c, int kt, const CUtensorMap& map, const LseParams& p, int kk, size_t smem,
                 cudaStream_t s) {
    switch (kt) {
        case KVM_Q8_0: return launch_lse_q_kt<KVM_Q8_0>(c, map, p, kk, smem, s);
        case KVM_Q4_0: return launch_lse_q_kt<KVM_Q4_0>(c, map, p, kk, smem, s);
        default: return KVM_ERR_UNSUPPORTED;
    }
}

int launch_lse(kvm_ctx* c, int kt, const LseParams& p, int lpr, int vp, size_t smem, cudaStream_t s) {
    switch (kt) {
        case KVM_F32: return launch_lse_kt<KVM_F32>(c, p, lpr, vp, smem, s);
        case KVM_F16: return launch_lse_kt<KVM_F16>(c, p, lpr, vp, smem, s);
        case KVM_BF16: return launch_lse_kt<KVM_BF16>(c, p, lpr, vp, smem, s);
        case KVM_Q8_0: return launch_lse_kt<KVM_Q8_0>(c, p, lpr, vp, smem, s);
        case KVM_Q4_0: return launch_lse_kt<KVM_Q4_0>(c, p, lpr, vp, smem, s);
        default: return launch_lse_kt<KVM_Q5_0>(c, p, lpr, vp, smem, s);
    }
}

// Page LSE of layers [l0, l0+nl) into `lse` ([nl][rows][Hq][pages]); token t
// takes part iff t < visible (pages and visible are the caller's: the whole
// history for kvm_score_pages, one rank's page range for sharded scoring).
int lse_layers(kvm_ctx* c, const kvm_score_desc* d, const kvm_query* q, const kvm_kcache* k, const LseConfig& cfg,
               uint32_t l0, uint32_t nl, uint32_t pages, uint64_t visible, float* lse, cudaStream_t s) {
    const uint32_t G = d->q_heads / d->kv_heads;
    const uint32_t nvt = q->rows * G;
    int vp = 1;
    while (vp < int(nvt) && vp < 8) vp <<= 1;
    LseParams p{};
    p.k = static_cast<const uint8_t*>(k->data) + uint64_t(l0) * k->layer_stride;
    p.k_layer = k->layer_stride;
    p.page_bytes = uint64_t(d->page_tokens) * k->token_stride;
    p.chunk_bytes = cfg.chunk_bytes;
    p.chunks = cfg.chunks;
    p.tpc = cfg.tpc;
    p.kv_heads = d->kv_heads;
    p.row_bytes = cfg.row_bytes;
    p.pages = pages;
    p.layers = nl;
    p.page_tokens = d->page_tokens;
    p.tokens = visible;
    p.q = static_cast<const uint8_t*>(q->data) + uint64_t(l0) * q->layer_stride;
    p.q_type = q->type;
    p.rows = q->rows;
    p.q_layer = q->layer_stride;
    p.q_row = q->row_stride;
    p.q_head = q->head_stride;
    p.group = G;
    p.q_heads = d->q_heads;
    p.scale = d->scale > 0.f ? d->scale : 1.f / std::sqrt(float(d->head_dim));
    p.softcap = d->softcap;
    p.mask = static_cast<const uint8_t*>(d->mask);
    p.mask_type = d->mask_type;
    p.mask_row = d->mask_row_stride;
    p.lse = lse;
    p.status = c->status;
    p.stage_stride = cfg.stage_stride;
    if (cfg.tc) {
        // The query vectors of a KV head in passes of tc_pass_nv (one or two M
        // tiles each); a smaller last pass may use the one-tile layout.
        CUtensorMap map;
        KVM_TRY(encode_k_map(d, k, p.k, nl, cfg.head_major, &map));
        p.head_major = cfg.head_major;
        p.stages = cfg.tc_stages;
        for (uint32_t v0 = 0; v0 < nvt; v0 += cfg.tc_pass_nv) {
            p.v0 = v0;
            p.nv = std::min<uint32_t>(cfg.tc_pass_nv, nvt - v0);
            const int lm = tc_layout_for(p.nv);
            KVM_TRY(launch_lse_tc(c, map, p, cfg.tc_ka, lm, tc_smem_bytes(cfg.tc_ka, lm, cfg.tc_stages), s));
        }
        return KVM_OK;
    }
    if (cfg.q) {
        // Passes of up to 8 query vectors, as the mma.sync kernel below.
        CUtensorMap map;
        KVM_TRY(encode_q_map(d, k, p.k, nl, cfg, &map));
        p.chunk_bytes = cfg.q_tx;
        p.chunks = cfg.q_chunks;
        p.tpc = cfg.q_tpc;
        p.stage_stride = cfg.q_stage_stride;
        p.stages = cfg.q_stages;
        p.slot_stride = cfg.q_slot;
        p.hpg = cfg.q_hpg;
        p.groups_tma = cfg.q_groups;
        for (uint32_t v0 = 0; v0 < nvt; v0 += 8) {
            p.v0 = v0;
            p.nv = std::min<uint32_t>(8, nvt - v0);
            KVM_TRY(launch_lse_q(c, k->type, map, p, int(d->head_dim / 32), cfg.q_smem, s));
        }
        return KVM_OK;
    }
    if (cfg.mma) {
        // Passes of up to 8 query vectors (the 16 rows of the mma's A tile hold
        // their fp16 hi and lo parts).
        p.chunk_bytes = cfg.mma_chunk_bytes;
        p.chunks = cfg.mma_chunks;
        p.tpc = cfg.mma_tpc;
        p.stage_stride = cfg.mma_stage_stride;
        p.stages = cfg.mma_stages;
        p.row_set = uint32_t(k->token_stride);
        p.slot_stride = cfg.mma_slot;
        for (uint32_t v0 = 0; v0 < nvt; v0 += 8) {
            p.v0 = v0;
            p.nv = std::min<uint32_t>(8, nvt - v0);
            KVM_TRY(launch_lse_mma(c, k->type, p, int(d->head_dim / 32), cfg.mma_smem, s));
        }
    } else {
        for (uint32_t v0 = 0; v0 < nvt; v0 += vp) {
            p.v0 = v0;
            p.nv = std::min<uint32_t>(vp, nvt - v0);
            KVM_TRY(launch_lse(c, k->type, p, int(cfg.lpr), vp, cfg.smem, s));
        }
    }
    return KVM_OK;
}

// Softmax over pages and the head / row means of layers [l0, l0+nl), with the
// statistics computed here or (`given`, sharded scoring) supplied.
int normalize_layers(kvm_ctx* c, const kvm_score_desc* d, uint32_t rows, uint32_t l0, uint32_t nl, uint32_t pages,
                     const float* lse, const float2* given, float* mass_rows, float* mass_mean, cudaStream_t s) {
    const uint32_t G = d->q_heads / d->kv_heads;
    const uint32_t heads_per = d->groups == 1 ? d->q_heads : G;
    const size_t nsmem = size_t(rows) * heads_per * sizeof(float2);
    if (nsmem > 200 * 1024) return KVM_ERR_LENGTH;
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(page_mass_normalize_kernel), 200 * 1024));
    page_mass_normalize_kernel<<<nl * d->groups, 256, nsmem, s>>>(lse, rows, d->q_heads, G, d->groups, pages,
                                                                 mass_rows, mass_mean, l0, given);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

// Scores layers [l0, l0+nl) into mass rows / means whose layer index starts at
// l0 (absolute), using `lse` ([nl][rows][Hq][pages]) as scratch.
int score_layers(kvm_ctx* c, const kvm_score_desc* d, const kvm_query* q, const kvm_kcache* k, const LseConfig& cfg,
                 uint32_t l0, uint32_t nl, float* lse, float* mass_rows, float* mass_mean, cudaStream_t s) {
    const uint32_t pages = uint32_t((d->tokens + d->page_tokens - 1) / d->page_tokens);
    KVM_TRY(lse_layers(c, d, q, k, cfg, l0, nl, pages, d->tokens, lse, s));
    return normalize_layers(c, d, q->rows, l0, nl, pages, lse, nullptr, mass_rows, mass_mean, s);
}

// Workspace bytes of a sampled-row call's packed query rows and mask rows
// (both 0 without a row list); validates the list and the alignment the
// packing kernels need.
int row_pack_bytes(const kvm_score_desc* d, const kvm_query* q, size_t* qbytes, size_t* mbytes) {
    *qbytes = *mbytes = 0;
    if (!q->row_ids) return KVM_OK;
    if (q->rows > kMaxRowIds) return KVM_ERR_LENGTH;
    for (uint32_t i = 0; i < q->rows; ++i)
        if (q->row_ids[i] >= q->row_count) return KVM_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(q->data) | q->layer_stride | q->row_stride | q->head_stride) & 1)
        return KVM_ERR_INVALID_ARGUMENT;
    *qbytes = align256(size_t(d->layers) * q->rows * d->q_heads * d->head_dim * type_bytes(q->type));
    if (d->mask) {
        if ((reinterpret_cast<uintptr_t>(d->mask) | d->mask_row_stride) & 1) return KVM_ERR_INVALID_ARGUMENT;
        const uint64_t rb = d->tokens * type_bytes(d->mask_type);
        if (rb > 0x7fffffffull) return KVM_ERR_LENGTH;
        *mbytes = align256(size_t(q->rows) * rb);
    }
    return KVM_OK;
}

// Packs the listed query rows (and their mask rows) densely at `dst` (query
// rows first, `qbytes` of them, then mask rows) and points `dd` / `qq` at the
// copies, so the scorers see rows 0 .. n-1.
int pack_rows(kvm_ctx* c, const kvm_score_desc* d, const kvm_query* q, uint8_t* dst, size_t qbytes,
              kvm_score_desc* dd, kvm_query* qq, cudaStream_t s) {
    RowIds ids{};
    ids.n = q->rows;
    for (uint32_t i = 0; i < q->rows; ++i) ids.id[i] = q->row_ids[i];
    const uint32_t head_bytes = d->head_dim * type_bytes(q->type);
    const uint64_t chunks = uint64_t(d->layers) * q->rows * d->q_heads;
    const uint32_t grid = uint32_t(std::min<uint64_t>(chunks, uint64_t(c->num_sms) * 8));
    pack_query_rows_kernel<<<grid, 128, 0, s>>>(static_cast<const uint8_t*>(q->data), q->layer_stride,
                                                q->row_stride, q->head_stride, d->q_heads, head_bytes, d->layers,
                                                ids, dst);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    *qq = *q;
    qq->data = dst;
    qq->row_ids = nullptr;
    qq->row_count = q->rows;
    qq->head_stride = head_bytes;
    qq->row_stride = uint64_t(d->q_heads) * head_bytes;
    qq->layer_stride = uint64_t(q->rows) * qq->row_stride;
    *dd = *d;
    if (d->mask) {
        const uint32_t rb = uint32_t(d->tokens * type_bytes(d->mask_type));
        uint8_t* mdst = dst + qbytes;
        const dim3 mgrid(std::max<uint32_t>(1, std::min<uint32_t>((rb / 2 + 255) / 256, 64)), q->rows);
        pack_mask_rows_kernel<<<mgrid, 256, 0, s>>>(static_cast<const uint8_t*>(d->mask), d->mask_row_stride, rb,
                                                    ids, mdst);
        ++c->launches;
        KVM_CUDA(cudaGetLastError());
        dd->mask = mdst;
        dd->mask_row_stride = rb;
    }
    return KVM_OK;
}

int select_rows(kvm_ctx* c, const float* scores, uint32_t nrows, uint32_t pages, uint32_t score_stride,
                const uint32_t* keep, uint32_t nkeep, uint32_t budget, int signed_scores, uint32_t* out_ids,
                uint32_t* out_n, uint32_t out_stride, cudaStream_t s) {
    if (!scores || !out_ids || !out_n || !nrows || !pages || !budget) return KVM_ERR_INVALID_ARGUMENT;
    if (nkeep && !keep) return KVM_ERR_INVALID_ARGUMENT;
    if (pages > 196608) return KVM_ERR_LENGTH;
    if (score_stride < pages || out_stride < std::min(budget, pages)) return KVM_ERR_INVALID_ARGUMENT;
    std::vector<uint8_t> seen(pages, 0);
    uint32_t distinct = 0;
    for (uint32_t i = 0; i < nkeep; ++i) {
        if (keep[i] >= pages) return KVM_ERR_INVALID_ARGUMENT;
        distinct += !seen[keep[i]];
        seen[keep[i]] = 1;
    }
    if (distinct > budget) return KVM_ERR_BUDGET_EXCEEDED;
    KVM_TRY(upload_keep(c, keep, nkeep));
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(select_topk_kernel), 200 * 1024));
    select_topk_kernel<<<nrows, kSelectThreads, pages, s>>>(scores, pages, score_stride,
                                                             static_cast<const uint32_t*>(c->small), nkeep, budget,
                                                             signed_scores, out_ids, out_n, out_stride, c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int plan_rows(kvm_ctx* c, kvm_pool* pool, uint32_t row0, uint32_t nrows, const uint32_t* sel_ids,
              const uint32_t* sel_n, uint32_t sel_stride, int force, uint32_t* n_restore, uint32_t* n_evict,
              cudaStream_t s, DeviceStatus* status = nullptr) {
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(plan_residency_kernel), 200 * 1024));
    plan_residency_kernel<<<nrows, kPlanThreads, pool->view.pages, s>>>(pool->view, row0, sel_ids, sel_n, sel_stride,
                                                                         force, n_restore, n_evict,
                                                                         status ? status : c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int gather_layout(const kvm_stage_layout* L, GatherLayout* g) {
    if (!L || L->planes < 1 || L->planes > 2) return KVM_ERR_INVALID_ARGUMENT;
    g->planes = L->planes;
    for (uint32_t j = 0; j < 2; ++j) {
        g->host_base[j] = static_cast<const uint8_t*>(L->host_base[j]);
        g->host_row_stride[j] = L->host_row_stride[j];
        g->host_page_stride[j] = L->host_page_stride[j];
        g->dev_base[j] = static_cast<uint8_t*>(L->dev_base[j]);
        g->dev_row_stride[j] = L->dev_row_stride[j];
        g->dev_slot_stride[j] = L->dev_slot_stride[j];
        g->bytes[j] = L->bytes[j];
        if (j < L->planes) {
            if (!L->host_base[j] || !L->dev_base[j] || !L->bytes[j]) return KVM_ERR_INVALID_ARGUMENT;
            if (L->host_page_stride[j] < L->bytes[j] || L->dev_slot_stride[j] < L->bytes[j])
                return KVM_ERR_INVALID_ARGUMENT;
        }
    }
    return KVM_OK;
}

int gather_rows(kvm_ctx* c, kvm_pool* pool, uint32_t row0, uint32_t nrows, const GatherLayout& g, uint32_t ctas,
                cudaStream_t s, uint32_t page0 = 0, uint32_t page_end = 0xffffffffu, int fence_sys = 0) {
    const uint32_t grid = ctas ? ctas : kGatherDefaultCtas;
    stagein_gather_kernel<<<grid, kGatherThreads, 0, s>>>(pool->view, row0, nrows, g, page0, page_end, fence_sys);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

}  // namespace

extern "C" {

uint64_t kvm_row_bytes(int type, uint32_t dim) { return supported_type(type) ? row_bytes_of(type, dim) : 0; }

int kvm_ctx_create(int device, kvm_ctx** out) {
    if (!out) return KVM_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int count = 0;
    KVM_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(device);
    if (!guard.ok) return KVM_ERR_CUDA;
    auto* c = new (std::nothrow) kvm_ctx;
    if (!c) return KVM_ERR_CUDA;
    c->device = device;
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->side_done, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&c->status, sizeof(DeviceStatus)) != cudaSuccess ||
        cudaMallocHost(&c->status_host, sizeof(DeviceStatus)) != cudaSuccess ||
        cudaMemset(c->status, 0, sizeof(DeviceStatus)) != cudaSuccess) {
        cudaGetLastError();
        kvm_ctx_destroy(c);
        return KVM_ERR_CUDA;
    }
    *out = c;
    return KVM_OK;
}

int kvm_ctx_destroy(kvm_ctx* c) {
    if (!c) return KVM_OK;
    DeviceGuard guard(c->device);
    cudaDeviceSynchronize();
    for (auto e : c->events) cudaEventDestroy(e);
    if (c->side_done) cudaEventDestroy(c->side_done);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->status) cudaFree(c->status);
    if (c->status_host) cudaFreeHost(c->status_host);
    if (c->ws && !c->ws_borrowed) cudaFree(c->ws);
    if (c->small) cudaFree(c->small);
    if (c->aux) cudaFree(c->aux);
    if (c->aux_done) cudaEventDestroy(c->aux_done);
    for (auto& L : c->copy_lists) {
        if (L.done) cudaEventDestroy(L.done);
        if (L.host) cudaFreeHost(L.host);
    }
    delete c;
    return KVM_OK;
}

int kvm_ctx_device(const kvm_ctx* c) { return c ? c->device : -1; }
uint64_t kvm_ctx_launches(const kvm_ctx* c) { return c ? c->launches : 0; }

int kvm_ctx_status(kvm_ctx* c, void* stream) {
    if (!c) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_CUDA(cudaMemcpyAsync(c->status_host, c->status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost, s));
    KVM_CUDA(cudaStreamSynchronize(s));
    const int code = c->status_host->code;
    if (code) {
        KVM_CUDA(cudaMemsetAsync(c->status, 0, sizeof(DeviceStatus), s));
        KVM_CUDA(cudaStreamSynchronize(s));
    }
    return code;
}

size_t kvm_score_workspace_bytes(const kvm_score_desc* d, uint32_t rows) {
    if (!d || !d->page_tokens) return 0;
    return lse_bytes(d, d->layers, rows);
}

int kvm_ctx_bind_workspace(kvm_ctx* c, void* ws, size_t bytes) {
    if (!c || !ws || (reinterpret_cast<uintptr_t>(ws) & 255)) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, ws) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_INVALID_ARGUMENT;
    }
    if (a.type != cudaMemoryTypeDevice || a.device != c->device) return KVM_ERR_INVALID_ARGUMENT;
    if (c->ws && !c->ws_borrowed) {
        cudaDeviceSynchronize();
        cudaFree(c->ws);
    }
    c->ws = ws;
    c->ws_bytes = bytes;
    c->ws_borrowed = true;
    return KVM_OK;
}

size_t kvm_ctx_device_bytes(const kvm_ctx* c) {
    return c ? (c->ws_borrowed ? 0 : c->ws_bytes) + c->small_bytes : 0;
}

int kvm_score_pages(kvm_ctx* c, const kvm_score_desc* d, const kvm_query* q, const kvm_kcache* k, float* mass_rows,
                    float* mass_mean, void* stream) {
    if (!c) return KVM_ERR_INVALID_ARGUMENT;
    LseConfig cfg;
    KVM_TRY(validate_score(d, q, k, &cfg));
    size_t qb = 0, mb = 0;
    KVM_TRY(row_pack_bytes(d, q, &qb, &mb));
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    const size_t lb = lse_bytes(d, d->layers, q->rows);
    KVM_TRY(ensure_ws(c, lb + qb + mb));
    kvm_score_desc dd = *d;
    kvm_query qq = *q;
    if (q->row_ids) KVM_TRY(pack_rows(c, d, q, static_cast<uint8_t*>(c->ws) + lb, qb, &dd, &qq, s));
    return score_layers(c, &dd, &qq, k, cfg, 0, d->layers, static_cast<float*>(c->ws), mass_rows, mass_mean, s);
}

int kvm_select_topk(kvm_ctx* c, const float* scores, uint32_t nrows, uint32_t pages, uint32_t score_stride,
                    const uint32_t* keep, uint32_t nkeep, uint32_t budget, int signed_scores, uint32_t* out_ids,
                    uint32_t* out_n, uint32_t out_stride, void* stream) {
    if (!c) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    return select_rows(c, scores, nrows, pages, score_stride, keep, nkeep, budget, signed_scores, out_ids, out_n,
                       out_stride, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {

// Media groups of a row of `pages` pages: each range [first, second) covers pages
// [first / block, ceil(second / block)) clipped to the row; chains of strictly
// overlapping spans merge into one group, which is the fixed point that
// scored_media_group (kvmem/src/host/kvmem_store.cpp:18-32) reaches from any page
// inside them. gb[p] / ge[p]: first page / one past the last page of p's group
// (p alone when no range covers it).
void media_group_table(uint32_t pages, uint32_t block_tokens, const uint32_t* ranges, uint32_t nranges,
                       std::vector<uint32_t>& gb, std::vector<uint32_t>& ge) {
    std::vector<std::pair<uint32_t, uint32_t>> spans;
    for (uint32_t i = 0; i < nranges; ++i) {
        const uint32_t lo = ranges[2 * i] / block_tokens;
        const uint32_t hi =
            uint32_t(std::min<uint64_t>(pages, (uint64_t(ranges[2 * i + 1]) + block_tokens - 1) / block_tokens));
        if (lo < hi) spans.emplace_back(lo, hi);
    }
    std::sort(spans.begin(), spans.end());
    gb.resize(pages);
    ge.resize(pages);
    for (uint32_t p = 0; p < pages; ++p) gb[p] = p, ge[p] = p + 1;
    for (size_t i = 0; i < spans.size();) {
        uint32_t b = spans[i].first, e = spans[i].second;
        size_t j = i + 1;
        for (; j < spans.size() && spans[j].first < e; ++j) e = std::max(e, spans[j].second);
        for (uint32_t p = b; p < e; ++p) gb[p] = b, ge[p] = e;
        i = j;
    }
}

}  // namespace

extern "C" {

int kvm_query_fixed_blocks(uint64_t total_tokens, uint32_t block_tokens, uint32_t budget, uint32_t sink,
                           uint32_t recent, const uint32_t* ranges, uint32_t nranges, const uint32_t* mandatory,
                           uint32_t nmandatory, uint32_t* out, uint32_t capacity, uint32_t* n_out) {
    if (!block_tokens || !out || !n_out || (nranges && !ranges) || (nmandatory && !mandatory))
        return KVM_ERR_INVALID_ARGUMENT;
    const uint64_t n64 = total_tokens / block_tokens + (total_tokens % block_tokens != 0);
    if (n64 > UINT32_MAX) return KVM_ERR_LENGTH;
    const uint32_t n = uint32_t(n64);
    std::vector<uint8_t> kept(n, 0);
    if (!budget || n <= budget) {
        std::fill(kept.begin(), kept.end(), 1);
    } else {
        std::vector<uint32_t> gb, ge;
        media_group_table(n, block_tokens, ranges, nranges, gb, ge);
        uint32_t count = 0;
        // One page with its whole group; a required one that does not fit is an error.
        auto keep = [&](uint32_t id, bool required) -> int {
            if (id >= n) return KVM_ERR_INVALID_ARGUMENT;
            uint32_t need = 0;
            for (uint32_t b = gb[id]; b < ge[id]; ++b) need += !kept[b];
            if (count + need > budget) return required ? KVM_ERR_BUDGET_EXCEEDED : KVM_OK;
            for (uint32_t b = gb[id]; b < ge[id]; ++b) kept[b] = 1;
            count += need;
            return KVM_OK;
        };
        for (uint32_t i = 0; i < std::min(n, sink); ++i) KVM_TRY(keep(i, true));
        if (nranges && uint64_t(ranges[2 * (nranges - 1)]) < total_tokens)
            KVM_TRY(keep(ranges[2 * (nranges - 1)] / block_tokens, true));  // the newest media item
        for (uint32_t i = 0; i < nmandatory; ++i) KVM_TRY(keep(mandatory[i], true));
        for (uint32_t i = 0; i < std::min(n, recent); ++i) KVM_TRY(keep(n - 1 - i, false));
    }
    uint32_t m = 0;
    for (uint32_t p = 0; p < n; ++p) m += kept[p];
    if (m > capacity) return KVM_ERR_LENGTH;
    m = 0;
    for (uint32_t p = 0; p < n; ++p)
        if (kept[p]) out[m++] = p;
    *n_out = m;
    return KVM_OK;
}

int kvm_query_score_frame(uint64_t accepted, uint32_t block_tokens, uint32_t budget, uint32_t sink, uint32_t recent,
                          const uint32_t* fixed, uint32_t nfixed, uint64_t capacity, uint64_t* starts,
                          uint32_t* counts, uint8_t* score_mask, uint8_t* transport_mask, uint64_t* n_out) {
    if (!block_tokens || !budget || (nfixed && !fixed)) return KVM_ERR_INVALID_ARGUMENT;
    const uint64_t n = accepted / block_tokens + (accepted % block_tokens != 0);
    if (n > UINT32_MAX || n > capacity) return KVM_ERR_LENGTH;
    for (uint32_t i = 0; i < nfixed; ++i)
        if (fixed[i] >= n) return KVM_ERR_INVALID_ARGUMENT;
    const bool transported = n > budget;
    const bool trim = transported && uint64_t(sink) + recent < n;  // sink + recent < n <= UINT32_MAX
    for (uint64_t i = 0; i < n; ++i) {
        const uint64_t start = i * block_tokens;
        if (starts) starts[i] = start;
        if (counts) counts[i] = uint32_t(std::min<uint64_t>(block_tokens, accepted - start));
        if (score_mask) score_mask[i] = (trim && (i < sink || i >= n - recent)) ? 0 : 1;
        if (transport_mask) transport_mask[i] = transported ? 1 : 0;
    }
    if (transport_mask)
        for (uint32_t i = 0; i < nfixed; ++i) transport_mask[fixed[i]] = 0;
    if (n_out) *n_out = n;
    return KVM_OK;
}

int kvm_select_topk_media(kvm_ctx* c, const float* scores, uint32_t nrows, uint32_t pages, uint32_t score_stride,
                          const uint32_t* keep, uint32_t nkeep, uint32_t budget, int signed_scores,
                          uint32_t block_tokens, const uint32_t* ranges, uint32_t nranges, uint32_t* out_ids,
                          uint32_t* out_n, uint32_t out_stride, void* stream) {
    if (!c || !scores || !out_ids || !out_n || !nrows || !pages || !budget || !block_tokens)
        return KVM_ERR_INVALID_ARGUMENT;
    if ((nkeep && !keep) || (nranges && !ranges)) return KVM_ERR_INVALID_ARGUMENT;
    if (pages > kMediaMaxPages) return KVM_ERR_LENGTH;
    if (score_stride < pages || out_stride < std::min(budget, pages)) return KVM_ERR_INVALID_ARGUMENT;
    std::vector<uint32_t> gb, ge;
    media_group_table(pages, block_tokens, ranges, nranges, gb, ge);
    std::vector<uint32_t> group(pages);
    for (uint32_t p = 0; p < pages; ++p) group[p] = gb[p] | (ge[p] << 15);
    // Keep pages first, each with its whole group, in the caller's order.
    uint32_t count = 0;
    for (uint32_t i = 0; i < nkeep; ++i) {
        if (keep[i] >= pages) return KVM_ERR_INVALID_ARGUMENT;
        const uint32_t b = group[keep[i]] & 0x7fffu, e = (group[keep[i]] >> 15) & 0x7fffu;
        uint32_t need = 0;
        for (uint32_t p = b; p < e; ++p) need += !(group[p] >> 30);
        if (count + need > budget) return KVM_ERR_BUDGET_EXCEEDED;
        for (uint32_t p = b; p < e; ++p) group[p] |= 1u << 30;
        count += need;
    }
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_TRY(ensure_aux(c, size_t(pages) * 4));
    KVM_CUDA(cudaMemcpyAsync(c->aux, group.data(), size_t(pages) * 4, cudaMemcpyHostToDevice, s));
    const size_t smem = media_smem_bytes(pages);
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(select_topk_media_kernel), int(media_smem_bytes(kMediaMaxPages))));
    select_topk_media_kernel<<<nrows, kMediaThreads, smem, s>>>(scores, pages, score_stride,
                                                                static_cast<const uint32_t*>(c->aux), count, budget,
                                                                signed_scores, out_ids, out_n, out_stride, c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return aux_release(c, s);
}

int kvm_pool_create(kvm_ctx* c, uint32_t rows, uint32_t pages, uint32_t slots, kvm_pool** out) {
    if (!c || !out || !rows || !pages || !slots || pages > 196608) return KVM_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    DeviceGuard guard(c->device);
    auto* p = new (std::nothrow) kvm_pool;
    if (!p) return KVM_ERR_CUDA;
    p->ctx = c;
    const size_t a = align256(size_t(rows) * pages * 4), b = align256(size_t(rows) * slots * 4),
                 n = align256(size_t(rows) * 4);
    if (cudaMalloc(&p->mem, a + 3 * b + n) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return KVM_ERR_CUDA;
    }
    auto* base = static_cast<uint8_t*>(p->mem);
    p->view.slot_of = reinterpret_cast<int32_t*>(base);
    p->view.page_of = reinterpret_cast<int32_t*>(base + a);
    p->view.restore = reinterpret_cast<uint32_t*>(base + a + b);
    p->view.restore_slot = reinterpret_cast<uint32_t*>(base + a + 2 * b);
    p->view.n_restore = reinterpret_cast<uint32_t*>(base + a + 3 * b);
    p->view.rows = rows;
    p->view.pages = pages;
    p->view.slots = slots;
    int rc = kvm_pool_reset(p, nullptr);
    if (rc == KVM_OK && cudaDeviceSynchronize() != cudaSuccess) rc = KVM_ERR_CUDA;
    if (rc != KVM_OK) {
        kvm_pool_destroy(p);
        return rc;
    }
    *out = p;
    return KVM_OK;
}

int kvm_pool_destroy(kvm_pool* p) {
    if (!p) return KVM_OK;
    if (p->pending) return KVM_ERR_PENDING;  // destroy (or abort) the transfer first
    DeviceGuard guard(p->ctx->device);
    cudaDeviceSynchronize();
    if (p->mem) cudaFree(p->mem);
    delete p;
    return KVM_OK;
}

int kvm_pool_reset(kvm_pool* p, void* stream) {
    if (!p) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(p->ctx->device);
    if (p->pending) {
        // An aborted transfer that could not drain: wait for its copies first.
        if (p->pending->phase != kvm_transfer::Aborted) return KVM_ERR_PENDING;
        KVM_TRY(transfer_drain(p->pending, 30ull * 1000 * 1000));
    }
    auto s = static_cast<cudaStream_t>(stream);
    const auto& v = p->view;
    KVM_CUDA(cudaMemsetAsync(v.slot_of, 0xff, size_t(v.rows) * v.pages * 4, s));
    KVM_CUDA(cudaMemsetAsync(v.page_of, 0xff, size_t(v.rows) * v.slots * 4, s));
    KVM_CUDA(cudaMemsetAsync(v.n_restore, 0, size_t(v.rows) * 4, s));
    return KVM_OK;
}

namespace {

// Bounded host wait for an event: KVM_OK, KVM_ERR_TIMEOUT or KVM_ERR_CUDA.
int event_wait(cudaEvent_t e, uint64_t timeout_us) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t r = cudaEventQuery(e);
        if (r == cudaSuccess) return KVM_OK;
        if (r != cudaErrorNotReady) {
            cudaGetLastError();
            return KVM_ERR_CUDA;
        }
        const auto us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (uint64_t(us) >= timeout_us) return KVM_ERR_TIMEOUT;
    }
}

int event_ready(cudaEvent_t e) {
    const cudaError_t r = cudaEventQuery(e);
    if (r == cudaSuccess) return KVM_OK;
    if (r == cudaErrorNotReady) return KVM_ERR_PENDING;
    cudaGetLastError();
    return KVM_ERR_TRANSFER_FAILED;
}

void transfer_free(kvm_transfer* t) {
    if (t->planned) cudaEventDestroy(t->planned);
    if (t->spill_done) cudaEventDestroy(t->spill_done);
    if (t->restore_done) cudaEventDestroy(t->restore_done);
    if (t->mem) cudaFree(t->mem);
    delete t;
}

// Waits (bounded) for every step of an aborted transfer that had not drained;
// once it has, the transfer releases its pool.
int transfer_drain(kvm_transfer* t, uint64_t timeout_us) {
    for (cudaEvent_t e : {t->planned, t->spill_done, t->restore_done}) {
        const int w = event_wait(e, timeout_us);
        if (w != KVM_OK) return w;
    }
    t->drained = true;
    if (t->pool && t->pool->pending == t) t->pool->pending = nullptr;
    return KVM_OK;
}

}  // namespace

int kvm_transfer_prepare(kvm_ctx* c, kvm_pool* pool, const uint32_t* sel_ids, const uint32_t* sel_n,
                         uint32_t sel_stride, int force_reload, void* stream, kvm_transfer** out) {
    if (!out) return KVM_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (!c || !pool || pool->ctx != c || !sel_ids || !sel_n || !sel_stride) return KVM_ERR_INVALID_ARGUMENT;
    if (pool->pending) return KVM_ERR_PENDING;
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    auto* t = new (std::nothrow) kvm_transfer;
    if (!t) return KVM_ERR_CUDA;
    t->ctx = c;
    t->pool = pool;
    t->force = force_reload;
    const auto& v = pool->view;
    const size_t a = align256(size_t(v.rows) * v.pages * 4), b = align256(size_t(v.rows) * v.slots * 4),
                 n = align256(size_t(v.rows) * 4);
    // Everything the transfer needs is reserved here; the pool's tables are only read.
    if (cudaMalloc(&t->mem, a + 3 * b + n + 256) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->planned, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->spill_done, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->restore_done, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        transfer_free(t);
        return KVM_ERR_CUDA;
    }
    auto* base = static_cast<uint8_t*>(t->mem);
    t->shadow = v;
    t->shadow.slot_of = reinterpret_cast<int32_t*>(base);
    t->shadow.page_of = reinterpret_cast<int32_t*>(base + a);
    t->shadow.restore = reinterpret_cast<uint32_t*>(base + a + b);
    t->shadow.restore_slot = reinterpret_cast<uint32_t*>(base + a + 2 * b);
    t->shadow.n_restore = reinterpret_cast<uint32_t*>(base + a + 3 * b);
    t->status = reinterpret_cast<DeviceStatus*>(base + a + 3 * b + n);
    int rc = KVM_OK;
    if (cudaMemsetAsync(t->status, 0, sizeof(DeviceStatus), s) != cudaSuccess ||
        cudaMemcpyAsync(t->shadow.slot_of, v.slot_of, size_t(v.rows) * v.pages * 4, cudaMemcpyDeviceToDevice, s) !=
            cudaSuccess ||
        cudaMemcpyAsync(t->shadow.page_of, v.page_of, size_t(v.rows) * v.slots * 4, cudaMemcpyDeviceToDevice, s) !=
            cudaSuccess) {
        cudaGetLastError();
        rc = KVM_ERR_CUDA;
    }
    if (rc == KVM_OK) {
        kvm_pool shadow_pool;
        shadow_pool.ctx = c;
        shadow_pool.view = t->shadow;
        rc = plan_rows(c, &shadow_pool, 0, v.rows, sel_ids, sel_n, sel_stride, force_reload, nullptr, nullptr, s,
                       t->status);
    }
    if (rc == KVM_OK && cudaEventRecord(t->planned, s) != cudaSuccess) {
        cudaGetLastError();
        rc = KVM_ERR_CUDA;
    }
    if (rc != KVM_OK) {
        cudaStreamSynchronize(s);  // nothing may still read the shadow when it is freed
        cudaGetLastError();
        transfer_free(t);
        return rc;
    }
    pool->pending = t;
    *out = t;
    return KVM_OK;
}

int kvm_transfer_start_spill(kvm_transfer* t, const kvm_stage_layout* layout, const uint8_t* stale, uint32_t ctas,
                             void* stream) {
    if (!t) return KVM_ERR_INVALID_ARGUMENT;
    if (t->phase != kvm_transfer::Prepared) return KVM_ERR_INVALID_PLAN;
    DeviceGuard guard(t->ctx->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_CUDA(cudaStreamWaitEvent(s, t->planned, 0));
    if (stale) {
        GatherLayout g{};
        KVM_TRY(gather_layout(layout, &g));
        const auto& v = t->pool->view;
        spill_gather_kernel<<<ctas ? ctas : kGatherDefaultCtas, kGatherThreads, 0, s>>>(v.page_of, t->shadow.slot_of, stale, v.rows,
                                                                        v.pages, v.slots, t->force, g);
        ++t->ctx->launches;
        KVM_CUDA(cudaGetLastError());
    }
    KVM_CUDA(cudaEventRecord(t->spill_done, s));
    t->phase = kvm_transfer::Spilling;
    return KVM_OK;
}

int kvm_transfer_poll(kvm_transfer* t) {
    if (!t) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(t->ctx->device);
    switch (t->phase) {
        case kvm_transfer::Prepared: return event_ready(t->planned);
        case kvm_transfer::Spilling: return event_ready(t->spill_done);
        case kvm_transfer::Restoring: return event_ready(t->restore_done);
        case kvm_transfer::Published: return KVM_OK;
        default: return KVM_ERR_INVALID_SESSION;
    }
}

int kvm_transfer_start_restore(kvm_transfer* t, const kvm_stage_layout* layout, uint32_t ctas, void* stream) {
    if (!t) return KVM_ERR_INVALID_ARGUMENT;
    if (t->phase != kvm_transfer::Spilling) return KVM_ERR_INVALID_PLAN;
    GatherLayout g{};
    KVM_TRY(gather_layout(layout, &g));
    DeviceGuard guard(t->ctx->device);
    const int ready = event_ready(t->spill_done);  // slots of evicted pages are reused only after the spill
    if (ready != KVM_OK) return ready;
    auto s = static_cast<cudaStream_t>(stream);
    kvm_pool shadow_pool;
    shadow_pool.ctx = t->ctx;
    shadow_pool.view = t->shadow;
    t->restore_started = true;
    KVM_TRY(gather_rows(t->ctx, &shadow_pool, 0, t->shadow.rows, g, ctas, s));
    KVM_CUDA(cudaEventRecord(t->restore_done, s));
    t->phase = kvm_transfer::Restoring;
    return KVM_OK;
}

int kvm_transfer_publish(kvm_transfer* t, void* stream) {
    if (!t) return KVM_ERR_INVALID_ARGUMENT;
    if (t->phase != kvm_transfer::Restoring) return KVM_ERR_PENDING;
    DeviceGuard guard(t->ctx->device);
    const int ready = event_ready(t->restore_done);
    if (ready != KVM_OK) return ready;
    auto s = static_cast<cudaStream_t>(stream);
    // A device-side failure of the plan fails the transfer; its restore has
    // already reused slots, so the previous view is not preserved. Only the
    // transfer's own status word is read: the context's is left to its owner.
    DeviceStatus st{};
    KVM_CUDA(cudaMemcpyAsync(&st, t->status, sizeof(st), cudaMemcpyDeviceToHost, s));
    KVM_CUDA(cudaStreamSynchronize(s));
    if (st.code != KVM_OK) return st.code == KVM_ERR_BUDGET_EXCEEDED ? st.code : KVM_ERR_TRANSFER_FAILED;
    const auto& v = t->pool->view;
    const auto& w = t->shadow;
    KVM_CUDA(cudaMemcpyAsync(v.slot_of, w.slot_of, size_t(v.rows) * v.pages * 4, cudaMemcpyDeviceToDevice, s));
    KVM_CUDA(cudaMemcpyAsync(v.page_of, w.page_of, size_t(v.rows) * v.slots * 4, cudaMemcpyDeviceToDevice, s));
    KVM_CUDA(cudaMemcpyAsync(v.restore, w.restore, size_t(v.rows) * v.slots * 4, cudaMemcpyDeviceToDevice, s));
    KVM_CUDA(cudaMemcpyAsync(v.restore_slot, w.restore_slot, size_t(v.rows) * v.slots * 4, cudaMemcpyDeviceToDevice,
                             s));
    KVM_CUDA(cudaMemcpyAsync(v.n_restore, w.n_restore, size_t(v.rows) * 4, cudaMemcpyDeviceToDevice, s));
    KVM_CUDA(cudaStreamSynchronize(s));  // the new view is in place before the call returns
    t->phase = kvm_transfer::Published;
    t->pool->pending = nullptr;
    return KVM_OK;
}

int kvm_transfer_abort(kvm_transfer* t, uint64_t timeout_us, int* previous_view_preserved) {
    if (previous_view_preserved) *previous_view_preserved = 0;
    if (!t) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(t->ctx->device);
    if (t->phase == kvm_transfer::Published) {
        if (previous_view_preserved) *previous_view_preserved = 0;  // the new view is the current one
        return KVM_OK;
    }
    // Drain every recorded step before anything is released.
    int rc = KVM_OK;
    for (cudaEvent_t e : {t->planned, t->spill_done, t->restore_done}) {
        const int w = event_wait(e, timeout_us);
        if (w != KVM_OK) rc = w;
    }
    t->drained = rc == KVM_OK;
    if (previous_view_preserved) *previous_view_preserved = (!t->restore_started && t->drained) ? 1 : 0;
    t->phase = kvm_transfer::Aborted;
    // A transfer whose copies may still write the pool's slots keeps the pool
    // blocked (prepare returns KVM_ERR_PENDING) until a later drain succeeds:
    // kvm_transfer_destroy or kvm_pool_reset.
    if (t->drained && t->pool->pending == t) t->pool->pending = nullptr;
    return rc;
}

int kvm_transfer_destroy(kvm_transfer* t) {
    if (!t) return KVM_OK;
    DeviceGuard guard(t->ctx->device);
    if (t->phase != kvm_transfer::Published && t->phase != kvm_transfer::Aborted) {
        int preserved = 0;
        kvm_transfer_abort(t, 30ull * 1000 * 1000, &preserved);
    }
    if (!t->drained) KVM_TRY(transfer_drain(t, 30ull * 1000 * 1000));
    if (!t->drained) return KVM_ERR_TIMEOUT;  // device work may still use the buffers: keep them
    transfer_free(t);
    return KVM_OK;
}

int kvm_pool_read(kvm_pool* p, int32_t* slot_of, int32_t* page_of, void* stream) {
    if (!p) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(p->ctx->device);
    auto s = static_cast<cudaStream_t>(stream);
    const auto& v = p->view;
    if (slot_of)
        KVM_CUDA(cudaMemcpyAsync(slot_of, v.slot_of, size_t(v.rows) * v.pages * 4, cudaMemcpyDeviceToHost, s));
    if (page_of)
        KVM_CUDA(cudaMemcpyAsync(page_of, v.page_of, size_t(v.rows) * v.slots * 4, cudaMemcpyDeviceToHost, s));
    KVM_CUDA(cudaStreamSynchronize(s));
    return KVM_OK;
}

int kvm_plan_residency(kvm_ctx* c, kvm_pool* pool, const uint32_t* sel_ids, const uint32_t* sel_n, uint32_t sel_stride,
                       int force_reload, uint32_t* n_restore, uint32_t* n_evict, void* stream) {
    if (!c || !pool || !sel_ids || !sel_n || pool->ctx != c) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    return plan_rows(c, pool, 0, pool->view.rows, sel_ids, sel_n, sel_stride, force_reload, n_restore, n_evict,
                     static_cast<cudaStream_t>(stream));
}

int kvm_stagein_pool(kvm_ctx* c, kvm_pool* pool, const kvm_stage_layout* layout, uint32_t ctas, void* stream) {
    if (!c || !pool || pool->ctx != c) return KVM_ERR_INVALID_ARGUMENT;
    GatherLayout g{};
    KVM_TRY(gather_layout(layout, &g));
    DeviceGuard guard(c->device);
    return gather_rows(c, pool, 0, pool->view.rows, g, ctas, static_cast<cudaStream_t>(stream));
}

int kvm_shard_stagein(kvm_ctx* c, kvm_pool* pool, const kvm_stage_layout* layout, uint32_t page0,
                      uint32_t page_count, uint32_t ctas, void* stream) {
    if (!c || !pool || pool->ctx != c || !page_count) return KVM_ERR_INVALID_ARGUMENT;
    if (uint64_t(page0) + page_count > pool->view.pages) return KVM_ERR_INVALID_ARGUMENT;
    GatherLayout g{};
    KVM_TRY(gather_layout(layout, &g));
    DeviceGuard guard(c->device);
    return gather_rows(c, pool, 0, pool->view.rows, g, ctas, static_cast<cudaStream_t>(stream), page0,
                       page0 + page_count, 1);
}

int kvm_ipc_export(const void* dev_ptr, void* handle) {
    if (!dev_ptr || !handle) return KVM_ERR_INVALID_ARGUMENT;
    static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(uint64_t) <= KVM_IPC_HANDLE_BYTES, "IPC handle size");
    AddressRangeFn range = address_range_fn();
    if (!range) return KVM_ERR_CUDA;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return KVM_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h{};
    KVM_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    const uint64_t offset = reinterpret_cast<uintptr_t>(dev_ptr) - base;
    std::memset(handle, 0, KVM_IPC_HANDLE_BYTES);
    std::memcpy(handle, &h, sizeof(h));
    std::memcpy(static_cast<uint8_t*>(handle) + sizeof(h), &offset, sizeof(offset));
    return KVM_OK;
}

int kvm_ipc_open(int device, const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return KVM_ERR_INVALID_ARGUMENT;
    *dev_ptr = nullptr;
    DeviceGuard guard(device);
    if (!guard.ok) return KVM_ERR_CUDA;
    cudaIpcMemHandle_t h{};
    uint64_t offset = 0;
    std::memcpy(&h, handle, sizeof(h));
    std::memcpy(&offset, static_cast<const uint8_t*>(handle) + sizeof(h), sizeof(offset));
    void* base = nullptr;
    KVM_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr = static_cast<uint8_t*>(base) + offset;
    std::lock_guard<std::mutex> lock(ipc_mutex());
    ipc_bases()[*dev_ptr] = base;
    return KVM_OK;
}

int kvm_ipc_close(int device, void* dev_ptr) {
    if (!dev_ptr) return KVM_OK;
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(ipc_mutex());
        auto it = ipc_bases().find(dev_ptr);
        if (it == ipc_bases().end()) return KVM_ERR_INVALID_ARGUMENT;
        base = it->second;
        ipc_bases().erase(it);
    }
    DeviceGuard guard(device);
    KVM_CUDA(cudaIpcCloseMemHandle(base));
    return KVM_OK;
}

int kvm_stagein_copies(kvm_ctx* c, const kvm_copy* ops, uint32_t n, uint32_t ctas, void* stream) {
    if (!c || (n && !ops)) return KVM_ERR_INVALID_ARGUMENT;
    if (!n) return KVM_OK;
    for (uint32_t i = 0; i < n; ++i)
        if (!ops[i].src || !ops[i].dst || !ops[i].bytes) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    static_assert(sizeof(CopyOp) == sizeof(kvm_copy), "copy op layout");
    // The list is copied into one of two mapped pinned lists that the gather reads
    // directly, so the caller's array may be reused on return and nothing waits for
    // the device unless both lists are still in flight.
    auto& L = c->copy_lists[c->copy_next];
    if (L.pending) {
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            const cudaError_t e = cudaEventQuery(L.done);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady) {
                cudaGetLastError();
                return KVM_ERR_CUDA;
            }
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(30)) return KVM_ERR_TIMEOUT;
        }
        L.pending = false;
    }
    if (!L.done) KVM_CUDA(cudaEventCreateWithFlags(&L.done, cudaEventDisableTiming));
    if (L.cap < n) {
        if (L.host) cudaFreeHost(L.host);
        L.host = nullptr;
        L.cap = 0;
        const uint32_t cap = std::max<uint32_t>(256, n);
        KVM_CUDA(cudaHostAlloc(&L.host, size_t(cap) * sizeof(CopyOp), cudaHostAllocMapped | cudaHostAllocPortable));
        L.cap = cap;
    }
    std::memcpy(L.host, ops, size_t(n) * sizeof(CopyOp));
    CopyOp* dev_ops = nullptr;
    KVM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev_ops), L.host, 0));
    const uint32_t grid = std::min<uint32_t>(n, ctas ? ctas : kGatherDefaultCtas);
    copy_ops_kernel<<<grid, kGatherThreads, 0, s>>>(dev_ops, n);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    KVM_CUDA(cudaEventRecord(L.done, s));
    L.pending = true;
    c->copy_next ^= 1;
    return KVM_OK;
}

int kvm_stagein_wait(kvm_ctx* c, void* stream, uint64_t timeout_us) {
    if (!c) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) {
            cudaGetLastError();
            return KVM_ERR_CUDA;
        }
        const auto us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (uint64_t(us) >= timeout_us) return KVM_ERR_TIMEOUT;
    }
    return kvm_ctx_status(c, stream);
}

int kvm_restore_k(kvm_ctx* c, int type, const kvm_restore_item* items, uint32_t n_items, uint32_t n_head,
                  uint32_t head_dim, uint32_t n_rot, const float* theta, uint32_t nrot, void* stream) {
    if (!c || (n_items && !items)) return KVM_ERR_INVALID_ARGUMENT;
    if (type != KVM_Q8_0 && type != KVM_Q4_0) return KVM_ERR_UNSUPPORTED;
    if (!n_head || !head_dim || head_dim % 32 || n_rot % 2 || n_rot > head_dim || (n_rot && !theta))
        return KVM_ERR_INVALID_ARGUMENT;
    const uint64_t n_embd = uint64_t(n_head) * head_dim;
    if (nrot && ((nrot != 64 && nrot != 128 && nrot != 256 && nrot != 512) || n_embd % nrot))
        return KVM_ERR_INVALID_ARGUMENT;
    if (n_embd > 16384) return KVM_ERR_LENGTH;
    std::vector<RestoreItem> its(std::max<uint32_t>(n_items, 1));
    std::vector<uint64_t> base(n_items + 1, 0);
    for (uint32_t i = 0; i < n_items; ++i) {
        if (!items[i].src || !items[i].dst) return KVM_ERR_INVALID_ARGUMENT;
        its[i] = RestoreItem{static_cast<const uint8_t*>(items[i].src), static_cast<uint8_t*>(items[i].dst),
                             items[i].tokens, items[i].pos0};
        base[i + 1] = base[i] + items[i].tokens;
    }
    if (!base[n_items]) return KVM_OK;
    const uint32_t half = n_rot / 2;
    const size_t o_items = 0, o_base = align256(its.size() * sizeof(RestoreItem)),
                 o_theta = o_base + align256(base.size() * 8), total = o_theta + align256(std::max<uint32_t>(half, 1) * 4);
    std::vector<uint8_t> host(total, 0);
    std::memcpy(host.data() + o_items, its.data(), its.size() * sizeof(RestoreItem));
    std::memcpy(host.data() + o_base, base.data(), base.size() * 8);
    if (half) std::memcpy(host.data() + o_theta, theta, half * 4);
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_TRY(ensure_aux(c, total));
    auto* a = static_cast<uint8_t*>(c->aux);
    KVM_CUDA(cudaMemcpyAsync(a, host.data(), total, cudaMemcpyHostToDevice, s));
    const float scale = nrot ? 1.0f / std::sqrt(float(nrot)) : 1.0f;
    const uint32_t grid = uint32_t(std::min<uint64_t>(base[n_items], uint64_t(c->num_sms) * 8));
    const size_t smem = n_embd * 4;
    const auto* di = reinterpret_cast<const RestoreItem*>(a + o_items);
    const auto* db = reinterpret_cast<const uint64_t*>(a + o_base);
    const auto* dt = reinterpret_cast<const float*>(a + o_theta);
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(restore_k_kernel<KVM_Q8_0>), 64 * 1024));
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(restore_k_kernel<KVM_Q4_0>), 64 * 1024));
    if (type == KVM_Q8_0)
        restore_k_kernel<KVM_Q8_0><<<grid, kRestoreThreads, smem, s>>>(di, n_items, db, n_head, head_dim, n_rot, dt,
                                                                       nrot, scale);
    else
        restore_k_kernel<KVM_Q4_0><<<grid, kRestoreThreads, smem, s>>>(di, n_items, db, n_head, head_dim, n_rot, dt,
                                                                       nrot, scale);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return aux_release(c, s);
}

int kvm_propagate_scores(kvm_ctx* c, const float* raw, uint32_t n, const uint64_t* starts,
                         const uint8_t* transport_mask, uint64_t accepted_through, const kvm_graph* g, double alpha,
                         double cross, float* out, void* stream) {
    if (!c || !raw || !out || !starts || !transport_mask || !g) return KVM_ERR_INVALID_ARGUMENT;
    if (!(std::isfinite(alpha) && alpha >= 0 && alpha <= 1) || !(std::isfinite(cross) && cross >= 0 && cross <= 1))
        return KVM_ERR_INVALID_ARGUMENT;
    if (!g->block_tokens || g->accepted_through != accepted_through) return KVM_ERR_INVALID_ARGUMENT;
    if ((g->nrows && !g->rows) || (g->nedges && !g->edges) || (g->has_messages && g->nspans && !g->spans))
        return KVM_ERR_INVALID_ARGUMENT;
    if (n == 0) return KVM_OK;
    if (n > 8u * kPostThreads) return KVM_ERR_LENGTH;
    const uint64_t block = g->block_tokens;
    // Frame index of each transport page, by its start.
    std::unordered_map<uint64_t, uint32_t> where;
    std::unordered_map<uint64_t, uint32_t> seen;
    uint32_t nallowed = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (starts[i] % block || !seen.emplace(starts[i], i).second) return KVM_ERR_INVALID_ARGUMENT;
        if (transport_mask[i]) {
            where.emplace(starts[i], i);
            ++nallowed;
        }
    }
    // Transfers (source, target, weight) in the reference's order: neighbours of
    // every transport page, then the completed graph rows.
    std::vector<uint32_t> ts, td;
    std::vector<double> tw;
    if (alpha > 0 && nallowed > 1) {
        for (uint32_t i = 0; i < n; ++i) {
            if (!transport_mask[i]) continue;
            const uint64_t src = starts[i];
            for (int dir = -1; dir <= 1; dir += 2) {
                if (dir < 0 && src < block) continue;
                if (dir > 0 && src > UINT64_MAX - block) continue;
                const uint64_t tgt = dir < 0 ? src - block : src + block;
                const auto it = where.find(tgt);
                if (it == where.end()) continue;
                ts.push_back(i);
                td.push_back(it->second);
                tw.push_back(alpha * .25 * span_coefficient(g, src, tgt, cross));
            }
        }
        for (uint32_t r = 0; r < g->nrows; ++r) {
            const kvm_graph_row& row = g->rows[r];
            const auto sit = where.find(row.source);
            if (sit == where.end() || !row.samples || row.source + block > g->completed_through) continue;
            if (uint64_t(row.edge_begin) + row.edge_count > g->nedges) return KVM_ERR_INVALID_ARGUMENT;
            double den = 0;
            for (uint32_t e = row.edge_begin; e < row.edge_begin + row.edge_count; ++e) {
                const kvm_graph_edge& edge = g->edges[e];
                if (!(std::isfinite(edge.mass) && edge.mass >= 0)) return KVM_ERR_INVALID_ARGUMENT;
                if (edge.target != row.source && where.count(edge.target)) den += edge.mass;
            }
            if (!den) continue;
            for (uint32_t e = row.edge_begin; e < row.edge_begin + row.edge_count; ++e) {
                const kvm_graph_edge& edge = g->edges[e];
                const auto tit = where.find(edge.target);
                if (tit == where.end() || edge.target == row.source) continue;
                ts.push_back(sit->second);
                td.push_back(tit->second);
                tw.push_back(alpha * .5 * edge.mass / den);
            }
        }
    }
    // By source and by target, each in transfer order (counting sort).
    const size_t m = tw.size();
    std::vector<uint32_t> out_off(n + 1, 0), in_off(n + 1, 0), in_src(std::max<size_t>(m, 1));
    std::vector<double> out_w(std::max<size_t>(m, 1)), in_w(std::max<size_t>(m, 1));
    for (size_t k = 0; k < m; ++k) {
        ++out_off[ts[k] + 1];
        ++in_off[td[k] + 1];
    }
    for (uint32_t i = 0; i < n; ++i) {
        out_off[i + 1] += out_off[i];
        in_off[i + 1] += in_off[i];
    }
    {
        std::vector<uint32_t> po(out_off.begin(), out_off.end() - 1), pi(in_off.begin(), in_off.end() - 1);
        for (size_t k = 0; k < m; ++k) {
            out_w[po[ts[k]]++] = tw[k];
            in_src[pi[td[k]]] = ts[k];
            in_w[pi[td[k]]++] = tw[k];
        }
    }
    // One upload: allowed | out_off | in_off | in_src | out_w | in_w.
    const size_t o_allowed = 0, o_outoff = align256(n), o_inoff = o_outoff + align256((n + 1) * 4ull),
                 o_insrc = o_inoff + align256((n + 1) * 4ull), o_outw = o_insrc + align256(in_src.size() * 4),
                 o_inw = o_outw + align256(out_w.size() * 8), total = o_inw + align256(in_w.size() * 8);
    std::vector<uint8_t> host(total, 0);
    std::memcpy(host.data() + o_allowed, transport_mask, n);
    std::memcpy(host.data() + o_outoff, out_off.data(), (n + 1) * 4ull);
    std::memcpy(host.data() + o_inoff, in_off.data(), (n + 1) * 4ull);
    std::memcpy(host.data() + o_insrc, in_src.data(), in_src.size() * 4);
    std::memcpy(host.data() + o_outw, out_w.data(), out_w.size() * 8);
    std::memcpy(host.data() + o_inw, in_w.data(), in_w.size() * 8);
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_TRY(ensure_aux(c, total));
    auto* a = static_cast<uint8_t*>(c->aux);
    KVM_CUDA(cudaMemcpyAsync(a, host.data(), total, cudaMemcpyHostToDevice, s));
    // No transfer at all (alpha 0, one transport page): the scores pass through.
    propagate_kernel<<<1, kPostThreads, 0, s>>>(
        raw, n, a + o_allowed, m ? nallowed : 0, reinterpret_cast<const uint32_t*>(a + o_outoff),
        reinterpret_cast<const double*>(a + o_outw), reinterpret_cast<const uint32_t*>(a + o_inoff),
        reinterpret_cast<const uint32_t*>(a + o_insrc), reinterpret_cast<const double*>(a + o_inw), out, c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return aux_release(c, s);  // a pageable upload is staged before cudaMemcpyAsync returns: `host` may go
}

int kvm_lrfu_preview(kvm_ctx* c, const float* scores, uint32_t n, const float* prev, uint32_t n_prev, double lambda,
                     double fraction, float* out, void* stream) {
    if (!c || !scores || !out || (n_prev && !prev)) return KVM_ERR_INVALID_ARGUMENT;
    if (!(std::isfinite(lambda) && lambda >= 0 && lambda <= 1) ||
        !(std::isfinite(fraction) && fraction > 0 && fraction <= 1))
        return KVM_ERR_INVALID_ARGUMENT;
    if (n == 0) return KVM_OK;
    uint32_t rank = 0xffffffffu;
    if (fraction < 1) {
        const size_t r = static_cast<size_t>((1 - fraction) * n);  // lrfu.hpp:66-67
        rank = uint32_t(std::min<size_t>(n - 1, r));
    }
    DeviceGuard guard(c->device);
    lrfu_preview_kernel<<<1, kPostThreads, 0, static_cast<cudaStream_t>(stream)>>>(scores, n, prev, n_prev, lambda,
                                                                                   rank, out, c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_meank_add(kvm_ctx* c, const kvm_kcache* k, uint32_t layers, uint32_t kv_heads, uint32_t head_dim,
                  uint64_t tok0, uint32_t n, uint32_t page_tokens, float* sums, uint32_t pages, uint32_t* counts,
                  void* stream) {
    if (!c || !k || !k->data || !sums || !counts) return KVM_ERR_INVALID_ARGUMENT;
    if (!layers || !kv_heads || !head_dim || !page_tokens || !pages) return KVM_ERR_INVALID_ARGUMENT;
    if (!supported_type(k->type)) return KVM_ERR_UNSUPPORTED;
    if (k->type >= KVM_Q8_0 && head_dim % 32) return KVM_ERR_UNSUPPORTED;
    if (n == 0) return KVM_OK;
    const uint64_t rb = row_bytes_of(k->type, head_dim);
    if (k->head_stride < rb || k->token_stride < k->head_stride * kv_heads) return KVM_ERR_INVALID_ARGUMENT;
    if (layers > 1 && k->layer_stride < k->token_stride * k->capacity_tokens) return KVM_ERR_INVALID_ARGUMENT;
    const uint64_t end = tok0 + n;
    if (end > k->capacity_tokens) return KVM_ERR_LENGTH;
    const uint64_t p0 = tok0 / page_tokens, p1 = (end - 1) / page_tokens;
    if (p1 >= pages) return KVM_ERR_LENGTH;
    const uint64_t n_embd = uint64_t(kv_heads) * head_dim;
    if (n_embd > 0xffffffffull || p1 - p0 + 1 > 65535 || layers > 65535) return KVM_ERR_LENGTH;
    DeviceGuard g(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    const dim3 grid(uint32_t((n_embd + 255) / 256), uint32_t(p1 - p0 + 1), layers);
    const auto* kb = static_cast<const uint8_t*>(k->data);
    switch (k->type) {
#define KVM_MEANK_ADD(T)                                                                                          \
    case T:                                                                                                      \
        meank_add_kernel<T><<<grid, 256, 0, s>>>(kb, k->layer_stride, k->token_stride, k->head_stride, head_dim, \
                                                 uint32_t(n_embd), tok0, end, page_tokens, uint32_t(p0), sums,   \
                                                 pages, counts);                                                 \
        break;
        KVM_MEANK_ADD(KVM_F32)
        KVM_MEANK_ADD(KVM_F16)
        KVM_MEANK_ADD(KVM_BF16)
        KVM_MEANK_ADD(KVM_Q8_0)
        KVM_MEANK_ADD(KVM_Q4_0)
        KVM_MEANK_ADD(KVM_Q5_0)
#undef KVM_MEANK_ADD
        default: return KVM_ERR_UNSUPPORTED;
    }
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_meank_score(kvm_ctx* c, const float* sums, const uint32_t* counts, const float* q, const uint32_t* layer_rows,
                    uint32_t layers, uint32_t rows, uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
                    uint32_t pages, const uint8_t* score_mask, int aggregation, float scale, float* out,
                    void* stream) {
    if (!c || !sums || !counts || !q || !layer_rows || !score_mask || !out) return KVM_ERR_INVALID_ARGUMENT;
    if (aggregation != 0 && aggregation != 1) return KVM_ERR_INVALID_ARGUMENT;
    if (!layers || !rows || !q_heads || !kv_heads || !head_dim || q_heads % kv_heads || !pages)
        return KVM_ERR_INVALID_ARGUMENT;
    std::vector<uint32_t> enabled, active, pairs, pair_slot;
    for (uint32_t p = 0; p < pages; ++p)
        if (score_mask[p]) enabled.push_back(p);
    for (uint32_t l = 0; l < layers; ++l) {
        if (layer_rows[l] > rows) return KVM_ERR_INVALID_ARGUMENT;
        if (!layer_rows[l]) continue;
        for (uint32_t r = 0; r < layer_rows[l]; ++r) {
            pairs.push_back(l);
            pairs.push_back(r);
            pair_slot.push_back(uint32_t(active.size()));
        }
        active.push_back(l);
    }
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_CUDA(cudaMemsetAsync(out, 0, size_t(pages) * 4, s));
    if (enabled.empty() || active.empty()) return KVM_OK;
    const uint32_t n = uint32_t(enabled.size()), nact = uint32_t(active.size());
    const uint32_t npairs = uint32_t(pair_slot.size());
    const uint64_t kw = uint64_t(kv_heads) * head_dim, qw = uint64_t(q_heads) * head_dim;
    const uint64_t dists = uint64_t(npairs) * q_heads;
    if (dists > 65535) return KVM_ERR_LENGTH;  // grid.y of the logits launch
    const uint32_t group = q_heads / kv_heads;
    // Workspace: means_h | qh | logits | norms | group_inv | bad
    const size_t b_means = align256(size_t(nact) * n * kw * 2), b_q = align256(size_t(npairs) * qw * 2),
                 b_logits = align256(size_t(dists) * n * 4), b_norms = align256(size_t(dists) * 8),
                 b_group = align256(size_t(dists / group) * 4), b_bad = 256;
    KVM_TRY(ensure_ws(c, b_means + b_q + b_logits + b_norms + b_group + b_bad));
    auto* w = static_cast<uint8_t*>(c->ws);
    auto* means_h = reinterpret_cast<__half*>(w);
    auto* qh = reinterpret_cast<__half*>(w + b_means);
    auto* logits = reinterpret_cast<float*>(w + b_means + b_q);
    auto* norms = reinterpret_cast<float2*>(w + b_means + b_q + b_logits);
    auto* ginv = reinterpret_cast<float*>(w + b_means + b_q + b_logits + b_norms);
    auto* bad = reinterpret_cast<uint32_t*>(w + b_means + b_q + b_logits + b_norms + b_group);
    // Host tables: enabled | active | pairs | pair_slot
    std::vector<uint32_t> host;
    host.insert(host.end(), enabled.begin(), enabled.end());
    host.insert(host.end(), active.begin(), active.end());
    host.insert(host.end(), pairs.begin(), pairs.end());
    host.insert(host.end(), pair_slot.begin(), pair_slot.end());
    const size_t tbl = host.size() * 4;
    const size_t off = keep_area(c);
    KVM_TRY(ensure_small(c, off + tbl));
    auto* t = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(c->small) + off);
    KVM_CUDA(cudaDeviceSynchronize());
    KVM_CUDA(cudaMemcpy(t, host.data(), tbl, cudaMemcpyHostToDevice));
    const uint32_t* d_enabled = t;
    const uint32_t* d_active = t + enabled.size();
    const uint32_t* d_pairs = d_active + active.size();
    const uint32_t* d_slot = d_pairs + pairs.size();
    KVM_CUDA(cudaMemsetAsync(bad, 0, 4, s));
    const uint32_t pack_grid = uint32_t(std::max(1, c->num_sms * 4));
    meank_pack_means_kernel<<<pack_grid, 256, 0, s>>>(sums, counts, d_enabled, d_active, nact, pages, n, uint32_t(kw),
                                                      means_h, bad);
    meank_pack_query_kernel<<<pack_grid, 256, 0, s>>>(q, d_pairs, npairs, rows, uint32_t(qw), qh, bad);
    c->launches += 2;
    KVM_CUDA(cudaGetLastError());
    KVM_CUDA(cudaMemcpyAsync(c->status_host, bad, 4, cudaMemcpyDeviceToHost, s));
    KVM_CUDA(cudaStreamSynchronize(s));
    if (c->status_host->code) return KVM_ERR_NONFINITE;
    const float sc = scale > 0.f ? scale : 1.f / std::sqrt(float(head_dim));
    meank_logits_kernel<<<dim3((n + 7) / 8, uint32_t(dists)), 256, 0, s>>>(qh, means_h, d_slot, q_heads, kv_heads,
                                                                           head_dim, n, sc, logits);
    meank_normalize_kernel<<<uint32_t((dists + 7) / 8), 256, 0, s>>>(logits, n, uint32_t(dists), norms);
    c->launches += 2;
    if (aggregation == 1) {
        const uint32_t ngroups = uint32_t(dists / group);
        meank_group_mass_kernel<<<(ngroups + 7) / 8, 256, 0, s>>>(logits, norms, n, group, ngroups, ginv);
        ++c->launches;
    }
    const float weight = aggregation == 0 ? 1.f / (float(nact) * q_heads) : 1.f / (float(nact) * kv_heads);
    meank_accumulate_kernel<<<(n + 255) / 256, 256, 0, s>>>(logits, norms, ginv, d_enabled, n, uint32_t(dists), group,
                                                            aggregation, weight, out);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_layerwise_accumulate(kvm_ctx* c, const float* tile, uint32_t pages, uint32_t halves, int keep_halves,
                             const uint8_t* score_mask, double* accum, void* stream) {
    if (!c || !tile || !score_mask || !accum || !pages) return KVM_ERR_INVALID_ARGUMENT;
    if (halves != 1 && halves != 2) return KVM_ERR_INVALID_ARGUMENT;
    if (keep_halves && halves != 2) return KVM_ERR_INVALID_ARGUMENT;  // needs two Mean-K records per page
    DeviceGuard guard(c->device);
    layerwise_accumulate_kernel<<<1, kLayerwiseThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        tile, pages, halves, keep_halves, score_mask, accum, c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_layerwise_finish(kvm_ctx* c, const double* accum, uint32_t pages, int keep_halves, float* scores,
                         void* stream) {
    if (!c || !accum || !scores || !pages) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    const uint32_t grid = std::min<uint32_t>((pages + 255) / 256, uint32_t(c->num_sms));
    layerwise_finish_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(accum, pages, keep_halves, scores);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_recall_step(kvm_ctx* c, const kvm_step_desc* st, kvm_pool* pool, const kvm_stage_layout* layout,
                    float* mass_mean, uint32_t* sel_ids, uint32_t* sel_n, void* stream) {
    if (!c || !st || !st->score || !mass_mean || !sel_ids || !sel_n || !st->budget) return KVM_ERR_INVALID_ARGUMENT;
    const kvm_score_desc* d = st->score;
    if (st->q && st->q->row_ids) return KVM_ERR_UNSUPPORTED;  // decode rows are dense
    LseConfig cfg;
    KVM_TRY(validate_score(d, st->q, st->k, &cfg));
    const uint32_t pages = uint32_t((d->tokens + d->page_tokens - 1) / d->page_tokens);
    const uint32_t srows = d->layers * d->groups;
    GatherLayout g{};
    if (pool) {
        if (pool->ctx != c || pool->view.rows != srows || pool->view.pages != pages) return KVM_ERR_INVALID_ARGUMENT;
        if (pool->view.slots < std::min(st->budget, pages)) return KVM_ERR_BUDGET_EXCEEDED;
        if (layout) KVM_TRY(gather_layout(layout, &g));
    }
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    // Layer chunks: [l0, l0 + nl) each; a small first chunk when asked for.
    const uint32_t nch = std::max<uint32_t>(1, std::min(st->chunks ? st->chunks : 4u, d->layers));
    std::vector<std::pair<uint32_t, uint32_t>> parts;
    uint32_t l0 = 0;
    if (st->first_layers && st->first_layers < d->layers && nch > 1) {
        parts.push_back({0, st->first_layers});
        l0 = st->first_layers;
    }
    const uint32_t rest_chunks = parts.empty() ? nch : nch - 1;
    const uint32_t per = (d->layers - l0 + rest_chunks - 1) / rest_chunks;
    for (; l0 < d->layers; l0 += per) parts.push_back({l0, std::min(per, d->layers - l0)});
    const uint32_t chunks = uint32_t(parts.size());
    uint32_t widest = 0;
    for (const auto& pc : parts) widest = std::max(widest, pc.second);
    KVM_TRY(ensure_ws(c, lse_bytes(d, widest, st->q->rows)));
    while (c->events.size() < chunks) {
        cudaEvent_t e;
        KVM_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        c->events.push_back(e);
    }
    const uint32_t out_stride = st->budget;
    bool staged = false;
    for (uint32_t ci = 0; ci < chunks; ++ci) {
        const uint32_t l0 = parts[ci].first, nl = parts[ci].second;
        KVM_TRY(score_layers(c, d, st->q, st->k, cfg, l0, nl, static_cast<float*>(c->ws), nullptr, mass_mean, s));
        const uint32_t r0 = l0 * d->groups, nr = nl * d->groups;
        KVM_TRY(select_rows(c, mass_mean + size_t(r0) * pages, nr, pages, pages, st->keep, st->nkeep, st->budget, 0,
                            sel_ids + size_t(r0) * out_stride, sel_n + r0, out_stride, s));
        if (!pool) continue;
        KVM_TRY(plan_rows(c, pool, r0, nr, sel_ids + size_t(r0) * out_stride, sel_n + r0, out_stride,
                          st->force_reload, nullptr, nullptr, s));
        if (!layout) continue;
        KVM_CUDA(cudaEventRecord(c->events[ci], s));
        KVM_CUDA(cudaStreamWaitEvent(c->side, c->events[ci], 0));
        KVM_TRY(gather_rows(c, pool, r0, nr, g, st->stage_ctas, c->side));
        staged = true;
    }
    if (staged) {
        KVM_CUDA(cudaEventRecord(c->side_done, c->side));
        KVM_CUDA(cudaStreamWaitEvent(s, c->side_done, 0));
    }
    return KVM_OK;
}

}  // extern "C"

// ------------------------------------------------- scoring without device allocation
//
// kvm_score_pages needs a page log-sum-exp buffer that the context allocates
// (or that the caller binds). kvm_score_pages_noalloc below is the same
// computation for callers that cannot allocate device memory when they score:
// its scratch is this fixed array, which the CUDA driver reserves on every GPU
// that loads the library and keeps until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 256 B status word + page LSE buffer
constexpr size_t kNoAllocStatusBytes = 256;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_base[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
// The host symbol is only a stand-in; the address is looked up once per device.
int noalloc_scratch(int device, void** base) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_base[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return KVM_ERR_CUDA;
        }
        g_noalloc_base[device] = p;
    }
    *base = g_noalloc_base[device];
    return KVM_OK;
}

}  // namespace

extern "C" int kvm_score_pages_noalloc(const kvm_score_desc* d, const kvm_query* q, const kvm_kcache* k,
                                       float* mass_rows, float* mass_mean, void* stream) {
    LseConfig cfg;
    KVM_TRY(validate_score(d, q, k, &cfg));
    size_t qb = 0, mb = 0;
    KVM_TRY(row_pack_bytes(d, q, &qb, &mb));
    const size_t lb = lse_bytes(d, d->layers, q->rows);
    if (kNoAllocStatusBytes + lb + qb + mb > kNoAllocScratchBytes) return KVM_ERR_LENGTH;
    int device = -1;
    KVM_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kNoAllocMaxDevices) return KVM_ERR_UNSUPPORTED;
    void* base = nullptr;
    KVM_TRY(noalloc_scratch(device, &base));
    auto s = static_cast<cudaStream_t>(stream);
    // A context on the stack: it carries the device, SM count and the status
    // word (inside the fixed scratch); it owns no memory.
    kvm_ctx c;
    c.device = device;
    KVM_CUDA(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, device));
    c.status = static_cast<DeviceStatus*>(base);
    KVM_CUDA(cudaMemsetAsync(base, 0, sizeof(DeviceStatus), s));
    uint8_t* lse = static_cast<uint8_t*>(base) + kNoAllocStatusBytes;
    kvm_score_desc dd = *d;
    kvm_query qq = *q;
    if (q->row_ids) KVM_TRY(pack_rows(&c, d, q, lse + lb, qb, &dd, &qq, s));
    return score_layers(&c, &dd, &qq, k, cfg, 0, d->layers, reinterpret_cast<float*>(lse), mass_rows, mass_mean, s);
}

// ------------------------------------------------------------- page-range sharding
namespace {

// Copies the keep list without duplicates into `out` (validation of range is the caller's).
std::vector<uint32_t> distinct(const uint32_t* keep, uint32_t nkeep) {
    std::vector<uint32_t> v(keep, keep + nkeep);
    std::sort(v.begin(), v.end());
    v.erase(std::unique(v.begin(), v.end()), v.end());
    return v;
}

}  // namespace

extern "C" {

int kvm_shard_score_partial(kvm_ctx* c, const kvm_score_desc* desc, const kvm_query* q, const kvm_kcache* k,
                            uint32_t page0, uint32_t local_pages, float* stats, void* stream) {
    if (!c || !desc || !q || !stats || !local_pages) return KVM_ERR_INVALID_ARGUMENT;
    if (q->row_ids) return KVM_ERR_UNSUPPORTED;
    // Validate and plan with the local slice; visibility follows the global token count.
    kvm_score_desc local = *desc;
    local.tokens = uint64_t(local_pages) * desc->page_tokens;
    LseConfig cfg;
    KVM_TRY(validate_score(&local, q, k, &cfg));
    const uint64_t first = uint64_t(page0) * desc->page_tokens;
    const uint64_t visible = desc->tokens > first ? std::min<uint64_t>(desc->tokens - first, local.tokens) : 0;
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    KVM_TRY(ensure_ws(c, lse_bytes(&local, local.layers, q->rows)));
    float* lse = static_cast<float*>(c->ws);
    KVM_TRY(lse_layers(c, &local, q, k, cfg, 0, local.layers, local_pages, visible, lse, s));
    const uint32_t nrows = local.layers * q->rows * local.q_heads;
    lse_stats_kernel<<<(nrows + 7) / 8, 256, 0, s>>>(lse, nrows, local_pages, reinterpret_cast<float2*>(stats));
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_shard_page_lse(kvm_ctx* c, const kvm_score_desc* desc, const kvm_query* q, const kvm_kcache* k,
                       uint32_t page0, uint32_t local_pages, float* lse, void* stream) {
    if (!c || !desc || !q || !lse || !local_pages) return KVM_ERR_INVALID_ARGUMENT;
    if (q->row_ids) return KVM_ERR_UNSUPPORTED;
    kvm_score_desc local = *desc;
    local.tokens = uint64_t(local_pages) * desc->page_tokens;
    LseConfig cfg;
    KVM_TRY(validate_score(&local, q, k, &cfg));
    const uint64_t first = uint64_t(page0) * desc->page_tokens;
    const uint64_t visible = desc->tokens > first ? std::min<uint64_t>(desc->tokens - first, local.tokens) : 0;
    DeviceGuard guard(c->device);
    return lse_layers(c, &local, q, k, cfg, 0, local.layers, local_pages, visible, lse,
                      static_cast<cudaStream_t>(stream));
}

int kvm_page_mass_from_lse(kvm_ctx* c, const kvm_score_desc* desc, uint32_t rows, const float* lse, float* mass_rows,
                           float* mass_mean, void* stream) {
    if (!c || !desc || !lse || !rows || !desc->layers || !desc->page_tokens || !desc->kv_heads ||
        desc->q_heads % desc->kv_heads)
        return KVM_ERR_INVALID_ARGUMENT;
    if (desc->groups != 1 && desc->groups != desc->kv_heads) return KVM_ERR_INVALID_ARGUMENT;
    if (!mass_rows && !mass_mean) return KVM_OK;
    const uint32_t pages = uint32_t((desc->tokens + desc->page_tokens - 1) / desc->page_tokens);
    if (!pages) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    return normalize_layers(c, desc, rows, 0, desc->layers, pages, lse, nullptr, mass_rows, mass_mean,
                            static_cast<cudaStream_t>(stream));
}

int kvm_shard_merge_stats(kvm_ctx* c, const float* gathered, uint32_t ranks, uint32_t count, float* global_stats,
                          void* stream) {
    if (!c || !gathered || !global_stats || !ranks || !count) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    auto s = static_cast<cudaStream_t>(stream);
    stats_merge_kernel<<<(count + 255) / 256, 256, 0, s>>>(reinterpret_cast<const float2*>(gathered), ranks, count,
                                                          reinterpret_cast<float2*>(global_stats));
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_shard_score_finish(kvm_ctx* c, const kvm_score_desc* desc, uint32_t rows, uint32_t local_pages,
                           const float* global_stats, float* mass_rows, float* mass_mean, void* stream) {
    if (!c || !desc || !global_stats || !rows || !local_pages) return KVM_ERR_INVALID_ARGUMENT;
    if (desc->groups != 1 && desc->groups != desc->kv_heads) return KVM_ERR_INVALID_ARGUMENT;
    kvm_score_desc local = *desc;
    local.tokens = uint64_t(local_pages) * desc->page_tokens;
    if (lse_bytes(&local, local.layers, rows) > c->ws_bytes) return KVM_ERR_STALE;  // no partial pass ran
    DeviceGuard guard(c->device);
    return normalize_layers(c, &local, rows, 0, local.layers, local_pages, static_cast<const float*>(c->ws),
                            reinterpret_cast<const float2*>(global_stats), mass_rows, mass_mean,
                            static_cast<cudaStream_t>(stream));
}

int kvm_shard_candidates(kvm_ctx* c, const float* scores, uint32_t nrows, uint32_t local_pages, uint32_t score_stride,
                         uint32_t page0, const uint32_t* keep, uint32_t nkeep, uint32_t k, float* cand_scores,
                         uint32_t* cand_ids, void* stream) {
    if (!c || !scores || !nrows || !local_pages || !k || !cand_scores || !cand_ids || (nkeep && !keep))
        return KVM_ERR_INVALID_ARGUMENT;
    if (local_pages > 196608 || score_stride < local_pages) return KVM_ERR_LENGTH;
    const auto kd = distinct(keep, nkeep);
    DeviceGuard guard(c->device);
    KVM_TRY(upload_keep(c, kd.data(), uint32_t(kd.size())));
    auto s = static_cast<cudaStream_t>(stream);
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(shard_candidates_kernel), 200 * 1024));
    shard_candidates_kernel<<<nrows, kSelectThreads, local_pages, s>>>(
        scores, local_pages, score_stride, page0, static_cast<const uint32_t*>(c->small), uint32_t(kd.size()), k,
        cand_scores, cand_ids, c->status);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_shard_merge(kvm_ctx* c, const float* cand_scores, const uint32_t* cand_ids, uint32_t ranks, uint32_t nrows,
                    uint32_t k, const uint32_t* keep, uint32_t nkeep, uint32_t budget, uint32_t* out_ids,
                    uint32_t* out_n, uint32_t out_stride, void* stream) {
    if (!c || !cand_scores || !cand_ids || !ranks || !nrows || !k || !budget || !out_ids || !out_n ||
        (nkeep && !keep))
        return KVM_ERR_INVALID_ARGUMENT;
    if (uint64_t(ranks) * k > kMergeMax) return KVM_ERR_LENGTH;
    const auto kd = distinct(keep, nkeep);
    if (kd.size() > budget) return KVM_ERR_BUDGET_EXCEEDED;
    if (out_stride < budget) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(c->device);
    KVM_TRY(upload_keep(c, kd.data(), uint32_t(kd.size())));
    auto s = static_cast<cudaStream_t>(stream);
    const size_t smem = size_t(ranks) * k * 8 + (size_t(budget) + kd.size()) * 4;
    if (smem > 200 * 1024) return KVM_ERR_LENGTH;
    KVM_CUDA(smem_attr(reinterpret_cast<const void*>(shard_merge_kernel), 200 * 1024));
    shard_merge_kernel<<<nrows, kSelectThreads, smem, s>>>(cand_scores, cand_ids, ranks, k, nrows,
                                                            static_cast<const uint32_t*>(c->small),
                                                            uint32_t(kd.size()), budget, out_ids, out_n, out_stride);
    ++c->launches;
    KVM_CUDA(cudaGetLastError());
    return KVM_OK;
}

int kvm_prefill_attention(kvm_ctx* c, const kvm_prefill_desc* d, const void* q, uint64_t q_row_stride,
                          uint64_t q_head_stride, const kvm_kcache* k, const kvm_kcache* v, void* out,
                          uint64_t out_row_stride, uint64_t out_head_stride, float* page_lse, void* stream) {
    if (!c || !d || !q || !k || !v || !out || !k->data || !v->data) return KVM_ERR_INVALID_ARGUMENT;
    if (d->head_dim != 128 && d->head_dim != 256) return KVM_ERR_UNSUPPORTED;
    if (d->type != KVM_F16 && d->type != KVM_BF16) return KVM_ERR_UNSUPPORTED;
    if (k->type != d->type || v->type != d->type) return KVM_ERR_INVALID_ARGUMENT;
    if (!d->q_heads || !d->kv_heads || d->q_heads % d->kv_heads) return KVM_ERR_INVALID_ARGUMENT;
    if (!(d->scale >= 0.f) || !std::isfinite(d->scale)) return KVM_ERR_INVALID_ARGUMENT;
    if (!d->width) return KVM_OK;
    const uint64_t keys = d->base + d->width;
    if (keys > 0x7fffffffull || keys > k->capacity_tokens || keys > v->capacity_tokens) return KVM_ERR_LENGTH;
    const uint64_t rb = uint64_t(d->head_dim) * 2;
    auto al16 = [](uint64_t x) { return (x & 15) == 0; };
    auto p16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!p16(q) || !p16(out) || !p16(k->data) || !p16(v->data) || !al16(q_row_stride) || !al16(q_head_stride) ||
        !al16(out_row_stride) || !al16(out_head_stride) || !al16(k->token_stride) || !al16(k->head_stride) ||
        !al16(v->token_stride) || !al16(v->head_stride))
        return KVM_ERR_UNSUPPORTED;
    if (q_head_stride < rb || out_head_stride < rb || k->head_stride < rb || v->head_stride < rb ||
        k->token_stride < rb || v->token_stride < rb || q_row_stride < rb || out_row_stride < rb)
        return KVM_ERR_INVALID_ARGUMENT;
    if (d->samples > KVM_PREFILL_MAX_SAMPLES) return KVM_ERR_LENGTH;
    kvmb::PrefillParams p{};
    if (d->samples) {
        if (!page_lse || !d->sample_rows || !d->page_tokens) return KVM_ERR_INVALID_ARGUMENT;
        if (d->page_tokens != 16 && d->page_tokens != 32 && d->page_tokens % kvmb::kPfKeys) return KVM_ERR_UNSUPPORTED;
        if (uint64_t(d->pages) * d->page_tokens < keys) return KVM_ERR_LENGTH;
        for (uint32_t i = 0; i < d->samples; ++i)
            if (d->sample_rows[i] >= d->width || (i && d->sample_rows[i] <= d->sample_rows[i - 1]))
                return KVM_ERR_INVALID_ARGUMENT;
        p.lse = page_lse;
        p.pages = d->pages;
        p.page_tokens = d->page_tokens;
        p.samples = d->samples;
    }
    TensorMapEncodeFn enc = tensor_map_encoder();
    if (!enc) return KVM_ERR_CUDA;
    const CUtensorMapDataType dt =
        d->type == KVM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap maps[2];
    const kvm_kcache* kv[2] = {k, v};
    for (int i = 0; i < 2; ++i) {
        const cuuint64_t dims[3] = {d->head_dim, d->kv_heads, std::min<uint64_t>(kv[i]->capacity_tokens, 0x7fffffffull)};
        const cuuint64_t strides[2] = {kv[i]->head_stride, kv[i]->token_stride};
        const cuuint32_t box[3] = {64, 1, uint32_t(kvmb::kPfKeys)};
        if (enc(&maps[i], dt, 3, const_cast<void*>(kv[i]->data), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KVM_ERR_CUDA;
    }
    p.q = static_cast<const uint8_t*>(q);
    p.q_row = q_row_stride;
    p.q_head = q_head_stride;
    p.q_heads = d->q_heads;
    p.kv_heads = d->kv_heads;
    p.width = d->width;
    p.q_tiles = (d->width + kvmb::kPfRows - 1) / kvmb::kPfRows;
    p.base = uint32_t(d->base);
    const float scale = d->scale > 0.f ? d->scale : 1.f / std::sqrt(float(d->head_dim));
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = static_cast<uint8_t*>(out);
    p.out_row = out_row_stride;
    p.out_head = out_head_stride;
    p.status = c->status;
    DeviceGuard guard(c->device);
    // Key-range split: one CTA per SM, so the (row tile, head) pairs run in waves of num_sms;
    // cutting each pair's key tiles into S chunks (whole capture pages each) fills the last
    // wave at the price of a merge pass over S partial rows. S minimises the modelled time
    // (waves x (tiles per chunk x ~1.1 us + ~6 us per CTA) + merge bytes at ~6 TB/s);
    // KVM_PREFILL_SPLITS overrides it (tests use it to reach the merge on small problems).
    p.granule = d->samples && d->page_tokens > uint32_t(kvmb::kPfKeys) ? d->page_tokens / kvmb::kPfKeys : 1;
    const uint64_t pairs = uint64_t(p.q_tiles) * d->q_heads;
    const uint64_t tiles = (keys + kvmb::kPfKeys - 1) / kvmb::kPfKeys;
    const uint64_t row_bytes_f32 = uint64_t(d->width) * d->q_heads * (uint64_t(d->head_dim) * 4 + 8);
    uint32_t splits = 1;
    double best = 0;
    for (uint32_t sp = 1; sp <= 16; ++sp) {
        const uint64_t chunk = ((tiles + sp - 1) / sp + p.granule - 1) / p.granule * p.granule;
        if (sp > 1 && (sp - 1) * chunk >= tiles) break;  // an empty chunk: no finer split helps
        const uint64_t waves = (pairs * sp + c->num_sms - 1) / c->num_sms;
        const double t = double(waves) * (double(chunk) * 1.1 + 6.0) +
                         (sp > 1 ? 4.0 + double(sp + 1) * double(row_bytes_f32) / 6e6 : 0.0);
        if (sp == 1 || t < best) best = t, splits = sp;
    }
    if (const char* e = std::getenv("KVM_PREFILL_SPLITS")) {
        const long v = std::strtol(e, nullptr, 10);
        if (v >= 1 && v <= 64) splits = uint32_t(v);
    }
    p.splits = splits;
    if (splits > 1) {
        const size_t rows = size_t(splits) * d->width * d->q_heads;
        const size_t ml_off = (rows * d->head_dim * 4 + 255) / 256 * 256;
        if (ensure_ws(c, ml_off + rows * 8) != KVM_OK) {
            p.splits = 1;  // a bound workspace too small for the partial rows
        } else {
            p.part_o = static_cast<float*>(c->ws);
            p.part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(c->ws) + ml_off);
        }
    }
    auto s = static_cast<cudaStream_t>(stream);
    const bool table = d->samples > uint32_t(kvmb::kPfInlineSamples);
    if (table) {
        // More rows than the launch parameters carry: a device table in the context's per-call
        // table buffer, reused once the kernels that read it are done.
        KVM_TRY(ensure_aux(c, size_t(d->samples) * 4));
        KVM_CUDA(cudaMemcpyAsync(c->aux, d->sample_rows, size_t(d->samples) * 4, cudaMemcpyHostToDevice, s));
        p.rows = static_cast<const uint32_t*>(c->aux);
    } else {
        p.rows = nullptr;
        for (uint32_t i = 0; i < d->samples; ++i) p.rows_inline[i] = d->sample_rows[i];
    }
    KVM_TRY(kvmb::launch_prefill(c, maps, p, d->head_dim, d->type == KVM_BF16, s));
    return table ? aux_release(c, s) : KVM_OK;
}

}  // extern "C"
