// CPU ORACLE BUILD SUPPORT — test infrastructure only.
//
// extern "C" entry points over the reference's own GPU scorers, compiled from
// the reference's sources by oracle/Makefile (target `refcuda`) into
// oracle/_ref/libkvref_cuda.so, so the tests can check this repository's
// restatement and kernels against numbers the reference itself produces, and
// bench.py can time the reference's GPU path on the same box:
//
//  * llama_kvmem_attention_cuda::score — the per-token page mass
//    (src/adapter/llama-kvmem-attention-cuda.cu:146-193, kernels page_lse /
//    normalize / average at :59-121), built against oracle/ggml_stub;
//  * kvmem::PageSoftmaxCuda::score — the Mean-K page softmax
//    (kvmem/src/cuda/page_softmax.cu:202-280) over a RawKvStore of per-page
//    K sums;
//  * kvmem_stagein_enqueue_k / _v + kvmem_stagein_flush — the stage-in route
//    with the raw-K restore transform (src/adapter/llama-kvmem-stagein.cu:
//    104-234, 673-881), run on this thread's own execution state.
//
// The product never links this file. Exceptions become status codes:
// 0 ok, 1 std::invalid_argument, 2 any other exception, 3 score() returned
// false (an input the reference does not handle).
#include "ggml-backend.h"
#include "ggml.h"
#include "llama-kvmem-attention-cuda.h"
#include "llama-kvmem-execution.h"
#include "llama-kvmem-stagein.h"

#include "kvmem/graph_recall.hpp"
#include "kvmem/page_softmax_cuda.hpp"
#include "kvmem/raw_kv_store.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <vector>

namespace {

template <class F> int guarded(F&& f) {
    try {
        return f();
    } catch (const std::invalid_argument&) {
        return 1;
    } catch (...) {
        return 2;
    }
}

// This repository's element / block encodings (include/kvm_recall.h kvm_type)
// as ggml types.
ggml_type to_ggml(int t) {
    switch (t) {
        case 0: return GGML_TYPE_F32;
        case 1: return GGML_TYPE_F16;
        case 2: return GGML_TYPE_BF16;
        case 3: return GGML_TYPE_Q8_0;
        case 4: return GGML_TYPE_Q4_0;
        case 5: return GGML_TYPE_Q5_0;
    }
    throw std::invalid_argument("element type");
}

// One reference scorer object per device, reused across calls (it keeps its
// stream and buffers, as the reference's AttentionSampler::Device does).
std::map<int, std::unique_ptr<llama_kvmem_attention_cuda>>& attention_scorers() {
    static std::map<int, std::unique_ptr<llama_kvmem_attention_cuda>> m;
    return m;
}
std::map<int, std::unique_ptr<kvmem::PageSoftmaxCuda>>& meank_scorers() {
    static std::map<int, std::unique_ptr<kvmem::PageSoftmaxCuda>> m;
    return m;
}

}  // namespace

extern "C" {

size_t ggml_row_size(enum ggml_type type, int64_t ne) {
    switch (type) {
        case GGML_TYPE_F32: return size_t(ne) * 4;
        case GGML_TYPE_F16:
        case GGML_TYPE_BF16: return size_t(ne) * 2;
        case GGML_TYPE_Q8_0: return size_t(ne / 32) * 34;
        case GGML_TYPE_Q4_0: return size_t(ne / 32) * 18;
        case GGML_TYPE_Q5_0: return size_t(ne / 32) * 22;
        default: return 0;
    }
}

void ggml_backend_tensor_get(const struct ggml_tensor* tensor, void* data, size_t offset, size_t size) {
    std::memcpy(data, static_cast<const uint8_t*>(tensor->data) + offset, size);
}

// llama_kvmem_attention_cuda::score over ggml views of device memory:
//   q:    element (d, r, h) at q + r*q_row_stride + h*q_head_stride (ne = [dim, q_rows, heads])
//   k:    row (t, kvh) at k + t*k_token_stride + kvh*k_head_stride (ne = [dim, tokens, kv_heads])
//   mask: element (t, r) at mask + r*mask_row_stride (ne = [tokens, q_rows]); device or host memory
// out: host f32 [nrows][pages], pages = ceil(tokens / block). *ms (optional):
// host wall time of the score() call, which synchronises its own stream.
int kvref_attention_score(const void* q, int q_type, uint32_t dim, uint32_t q_rows, uint32_t heads,
                          uint64_t q_row_stride, uint64_t q_head_stride, const void* k, int k_type, uint64_t tokens,
                          uint32_t kv_heads, uint64_t k_token_stride, uint64_t k_head_stride, const void* mask,
                          int mask_type, uint64_t mask_row_stride, float scale, float softcap, uint32_t block,
                          const uint32_t* rows, uint32_t nrows, float* out, double* ms) {
    return guarded([&] {
        ggml_tensor tq{}, tk{}, tm{};
        tq.type = to_ggml(q_type);
        tq.ne[0] = dim, tq.ne[1] = q_rows, tq.ne[2] = heads, tq.ne[3] = 1;
        tq.nb[0] = ggml_row_size(tq.type, 1), tq.nb[1] = q_row_stride, tq.nb[2] = q_head_stride;
        tq.nb[3] = q_head_stride * heads;
        tq.data = const_cast<void*>(q);
        tk.type = to_ggml(k_type);
        tk.ne[0] = dim, tk.ne[1] = int64_t(tokens), tk.ne[2] = kv_heads, tk.ne[3] = 1;
        tk.nb[0] = 0, tk.nb[1] = k_token_stride, tk.nb[2] = k_head_stride, tk.nb[3] = k_head_stride * kv_heads;
        tk.data = const_cast<void*>(k);
        tm.type = to_ggml(mask_type);
        tm.ne[0] = int64_t(tokens), tm.ne[1] = q_rows, tm.ne[2] = 1, tm.ne[3] = 1;
        tm.nb[0] = ggml_row_size(tm.type, 1), tm.nb[1] = mask_row_stride, tm.nb[2] = mask_row_stride * q_rows;
        tm.nb[3] = tm.nb[2];
        tm.data = const_cast<void*>(mask);
        int device = 0;
        if (cudaGetDevice(&device) != cudaSuccess) throw std::runtime_error("device");
        auto& scorer = attention_scorers()[device];
        if (!scorer) scorer = std::make_unique<llama_kvmem_attention_cuda>();
        std::vector<std::vector<float>> result;
        const auto t0 = std::chrono::steady_clock::now();
        const bool ok = scorer->score(&tq, &tk, &tm, scale, softcap, block, std::vector<uint32_t>(rows, rows + nrows),
                                      result);
        const auto t1 = std::chrono::steady_clock::now();
        if (ms) *ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
        if (!ok) return 3;
        const size_t pages = (tokens + block - 1) / block;
        for (uint32_t i = 0; i < nrows; ++i) std::memcpy(out + size_t(i) * pages, result[i].data(), pages * 4);
        return 0;
    });
}

// kvmem::PageSoftmaxCuda::score on `device` over a RawKvStore filled with
// per-page F32 K sums (the store kvref_page_softmax_scores builds), with the
// frame of query_score_frame(accepted, block, budget, sink, recent, fixed).
// Arguments and output as kvref_page_softmax_scores; *ms (optional): host
// wall time of the score() call (it synchronises its own stream).
int kvref_page_softmax_cuda(int device, const float* sums, const uint32_t* counts, const float* q,
                            const uint32_t* layer_rows, uint32_t layers, uint32_t rows, uint32_t heads,
                            uint32_t kv_heads, uint32_t dim, uint32_t block, uint64_t accepted, uint32_t budget,
                            uint32_t sink, uint32_t recent, const uint32_t* fixed, uint32_t nfixed, int aggregation,
                            float scale, double* out, uint64_t capacity, double* ms) {
    return guarded([&] {
        const uint32_t kw = kv_heads * dim;
        kvmem::RawKvStore keys({layers, kw, 0, block});
        auto frame = kvmem::query_score_frame(accepted, block, budget, sink, recent,
                                              std::vector<uint32_t>(fixed, fixed + nfixed));
        const size_t pages = frame.starts.size();
        if (pages > capacity) throw std::invalid_argument("capacity");
        for (uint32_t l = 0; l < layers; ++l)
            for (size_t p = 0; p < pages; ++p)
                keys.write_layer_mean_sum(uint32_t(p * block), counts[p], l, sums + (size_t(l) * pages + p) * kw);
        kvmem::PageQueryView view{q, layer_rows, layers, rows, heads, kv_heads, dim, nullptr, scale};
        auto& scorer = meank_scorers()[device];
        if (!scorer) scorer = std::make_unique<kvmem::PageSoftmaxCuda>(device);
        const auto t0 = std::chrono::steady_clock::now();
        const auto r = scorer->score(keys, view, frame,
                                     aggregation ? kvmem::GqaScoreAggregation::Max : kvmem::GqaScoreAggregation::Mean);
        const auto t1 = std::chrono::steady_clock::now();
        if (ms) *ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
        std::memcpy(out, r.data(), r.size() * sizeof(double));
        return 0;
    });
}

// Drops the cached reference scorers (their device memory and streams).
void kvref_cuda_release(void) {
    attention_scorers().clear();
    meank_scorers().clear();
}

int64_t ggml_time_us(void) {
    return std::chrono::duration_cast<std::chrono::microseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

void ggml_backend_tensor_set(struct ggml_tensor* tensor, const void* data, size_t offset, size_t size) {
    std::memcpy(static_cast<uint8_t*>(tensor->data) + offset, data, size);
}

bool ggml_backend_buffer_is_host(ggml_backend_buffer_t) { return true; }

// The reference's stage-in route for one batch of K items (raw-K restore:
// dequant -> NeoX RoPE -> Walsh-Hadamard -> requant into dst) and V items
// (byte copies): enqueue each, flush, synchronise. k_src / v_src are host bytes
// (the reference copies them into its pinned slab), dst device memory. type:
// 3 = q8_0, 4 = q4_0 (this repository's kvm_type). Returns 0, or 3 when the
// reference refused an item or a step failed.
int kvref_stagein(int type, uint32_t n_k, const uint8_t* const* k_src, const uint64_t* k_bytes,
                  uint8_t* const* k_dst, const int64_t* k_tokens, const int32_t* k_pos0, int64_t n_embd, int nrot,
                  int n_head, int n_embd_head, int n_rot_rope, const float* theta, int n_theta, uint32_t n_v,
                  const uint8_t* const* v_src, const uint64_t* v_bytes, uint8_t* const* v_dst) {
    return guarded([&] {
        const ggml_type ty = type == 3 ? GGML_TYPE_Q8_0 : GGML_TYPE_Q4_0;
        // The engine sizes the route's scratch before it enqueues a block
        // (src/adapter/llama-memory-kvmem.cpp:4470-4473): f32 rows of the
        // largest item, packed bytes of the largest record (at least one
        // 32 MiB slab, which also pins the two host slabs).
        int64_t max_tokens = 1;
        uint64_t max_bytes = 1;
        for (uint32_t i = 0; i < n_k; ++i) {
            max_tokens = std::max(max_tokens, k_tokens[i]);
            max_bytes = std::max(max_bytes, k_bytes[i]);
        }
        for (uint32_t i = 0; i < n_v; ++i) max_bytes = std::max(max_bytes, v_bytes[i]);
        if (!kvmem_stagein_gpu_ready(size_t(max_tokens) * size_t(n_embd), size_t(max_bytes))) return 3;
        for (uint32_t i = 0; i < n_k; ++i)
            if (!kvmem_stagein_enqueue_k(ty, k_src[i], k_bytes[i], k_dst[i], k_tokens[i], n_embd, nrot, n_head,
                                         n_embd_head, n_rot_rope, k_pos0[i], theta, n_theta, nullptr, nullptr,
                                         nullptr, nullptr))
                return 3;
        for (uint32_t i = 0; i < n_v; ++i)
            if (!kvmem_stagein_enqueue_v(v_src[i], v_bytes[i], v_dst[i], nullptr)) return 3;
        if (!kvmem_stagein_flush(nullptr, nullptr, nullptr, nullptr)) return 3;
        return kvmem_stagein_sync_checked() ? 0 : 3;
    });
}

}  // extern "C"

// The engine's side of the execution state, as the stage-in code reaches it:
// one state per host thread here, with its GPU staging created on first use.
struct kvmem_conv_pool {};
llama_kvmem_execution_state::llama_kvmem_execution_state() = default;
llama_kvmem_execution_state::~llama_kvmem_execution_state() = default;
llama_kvmem_execution_state& kvmem_current_execution() {
    static thread_local llama_kvmem_execution_state state;
    if (!state.gpu) state.gpu = kvmem_gpu_state_create();
    return state;
}
void kvmem_record_transfer(int, uint64_t) {}
