// kvmem::PageSoftmaxCuda over the B200 recall library.
//
// Implements the reference's class (kvmem/include/kvmem/page_softmax_cuda.hpp:10-31)
// with kvm_meank_score in place of the kernels of kvmem/src/cuda/page_softmax.cu.
// Argument meaning and errors are the reference's: std::invalid_argument for
// geometry, stale frames and non-finite or FP16-overflowing operands,
// std::length_error for launch-range or workspace overflow, std::runtime_error for
// CUDA failures. The page means are read from the RawKvStore as the reference
// reads them (mean_k) and handed to the library as sums over a count of 1, so the
// FP16 operands the device forms are the reference's recall_fp16(mean) exactly.
//
// Workspace. Constructed with a device only, the scorer lets the library size its
// own device memory and scores every layer in one call. With a borrowed
// workspace it allocates nothing in score(): it works one layer and one batch of
// at most 64 query rows at a time (the reference's batch rule) inside the
// borrowed bytes, whose size workspace_bytes() gives for the declared geometry,
// and adds the batches' masses on the host.
// A KVMem build compiles this file instead of page_softmax.cu and links libkvm_b200.so.
#include "kvmem/page_softmax_cuda.hpp"

#include "kvmem/raw_kv_store.hpp"
#include "kvm_recall.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <climits>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace kvmem {
namespace {

constexpr size_t kLogitsLimit = 64u << 20;  // the reference's per-batch logits budget

void checked(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("page softmax CUDA: ") + cudaGetErrorString(e));
}

struct DeviceBinding {
    int previous = -1;
    explicit DeviceBinding(int device) {
        checked(cudaGetDevice(&previous));
        checked(cudaSetDevice(device));
    }
    ~DeviceBinding() { cudaSetDevice(previous); }
};

size_t aligned(size_t bytes) {
    if (bytes > SIZE_MAX - 255) throw std::length_error("page softmax workspace overflow");
    return (bytes + 255) / 256 * 256;
}

void throw_status(int rc) {
    if (rc == KVM_OK) return;
    if (rc == KVM_ERR_NONFINITE) throw std::invalid_argument("page softmax operand is not finite or exceeds FP16");
    if (rc == KVM_ERR_INVALID_ARGUMENT) throw std::invalid_argument("page softmax CUDA geometry mismatch");
    if (rc == KVM_ERR_LENGTH) throw std::length_error("page softmax exceeds its planned device workspace");
    throw std::runtime_error("page softmax CUDA: library status " + std::to_string(rc));
}

// Query rows per call for `blocks` enabled pages (the reference's batch rule).
uint32_t batch_rows(size_t blocks, uint32_t heads) {
    return uint32_t(std::min<size_t>(64, kLogitsLimit / (std::max<size_t>(blocks, 1) * heads * sizeof(float))));
}

// The adapter's operands of one call (f32 means, u32 counts, f32 queries, f32
// output) and the library's own scratch of one kvm_meank_score call over one
// layer and `batch` rows, in that order.
struct Plan {
    size_t sums, counts, queries, out, lib;
    size_t total() const { return sums + counts + queries + out + lib; }
};

Plan plan(size_t blocks, uint32_t heads, uint32_t kvheads, uint32_t dim, size_t batch) {
    const size_t kw = size_t(kvheads) * dim, qw = size_t(heads) * dim, dists = batch * heads;
    Plan p{};
    p.sums = aligned(blocks * kw * 4);
    p.counts = aligned(blocks * 4);
    p.queries = aligned(batch * qw * 4);
    p.out = aligned(blocks * 4);
    p.lib = aligned(blocks * kw * 2) + aligned(batch * qw * 2) + aligned(dists * blocks * 4) + aligned(dists * 8) +
            aligned(dists / (heads / kvheads) * 4) + 256;
    return p;
}

}  // namespace

struct PageSoftmaxCuda::Impl {
    int device = -1;
    kvm_ctx* ctx = nullptr;
    cudaStream_t stream = nullptr;
    bool borrowed = false;
    uint8_t* ws = nullptr;  // the borrowed workspace
    size_t ws_bytes = 0;
    uint32_t max_blocks = 0, heads = 0, kvheads = 0, dim = 0;
    // Owned operand buffers (not borrowed).
    void* buf = nullptr;
    size_t buf_bytes = 0;

    explicit Impl(int dev) : device(dev) {
        DeviceBinding binding(device);
        if (kvm_ctx_create(device, &ctx) != KVM_OK) throw std::runtime_error("page softmax CUDA: context");
        checked(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    }
    ~Impl() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (buf) cudaFree(buf);
        if (stream) cudaStreamDestroy(stream);
        kvm_ctx_destroy(ctx);
    }
    uint8_t* operands(size_t bytes) {
        if (borrowed) {
            if (bytes > ws_bytes) throw std::length_error("page softmax exceeds its planned device workspace");
            return ws;
        }
        if (bytes > buf_bytes) {
            if (buf) checked(cudaFree(buf));
            buf = nullptr;
            buf_bytes = 0;
            checked(cudaMalloc(&buf, bytes));
            buf_bytes = bytes;
        }
        return static_cast<uint8_t*>(buf);
    }
};

PageSoftmaxCuda::PageSoftmaxCuda(int device) : impl_(std::make_unique<Impl>(device)) {}

size_t PageSoftmaxCuda::workspace_bytes(uint32_t blocks, uint32_t heads, uint32_t kvheads, uint32_t dim) {
    if (!blocks || !heads || !kvheads || !dim || heads % kvheads ||
        uint64_t(blocks) * heads * sizeof(float) > kLogitsLimit)
        throw std::invalid_argument("invalid planned page softmax geometry");
    return plan(blocks, heads, kvheads, dim, batch_rows(blocks, heads)).total();
}

PageSoftmaxCuda::PageSoftmaxCuda(int device, void* workspace, size_t bytes, uint32_t blocks, uint32_t heads,
                                 uint32_t kvheads, uint32_t dim)
    : PageSoftmaxCuda(device) {
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 ||
        bytes < workspace_bytes(blocks, heads, kvheads, dim))
        throw std::invalid_argument("page softmax borrowed workspace is missing, unaligned or too small");
    auto& w = *impl_;
    const Plan p = plan(blocks, heads, kvheads, dim, batch_rows(blocks, heads));
    const size_t ops = p.total() - p.lib;
    w.borrowed = true;
    w.ws = static_cast<uint8_t*>(workspace);
    w.ws_bytes = ops;
    w.max_blocks = blocks, w.heads = heads, w.kvheads = kvheads, w.dim = dim;
    DeviceBinding binding(device);
    throw_status(kvm_ctx_bind_workspace(w.ctx, w.ws + ops, bytes - ops));
    // One call at the planned geometry now, so that the library's host-table
    // upload area exists before score() runs (score() allocates nothing).
    const uint32_t batch = batch_rows(blocks, heads);
    checked(cudaMemsetAsync(w.ws, 0, ops, w.stream));
    const auto* base = w.ws;
    std::vector<uint8_t> mask(blocks, 1);
    const uint32_t rows[1] = {batch};
    std::vector<uint32_t> ones(blocks, 1);
    checked(cudaMemcpyAsync(w.ws + p.sums, ones.data(), blocks * 4, cudaMemcpyHostToDevice, w.stream));
    throw_status(kvm_meank_score(w.ctx, reinterpret_cast<const float*>(base), reinterpret_cast<const uint32_t*>(base + p.sums),
                                 reinterpret_cast<const float*>(base + p.sums + p.counts), rows, 1, batch, heads, kvheads,
                                 dim, blocks, mask.data(), 0, 0.f,
                                 reinterpret_cast<float*>(w.ws + p.sums + p.counts + p.queries), w.stream));
    checked(cudaStreamSynchronize(w.stream));
}

PageSoftmaxCuda::~PageSoftmaxCuda() = default;

size_t PageSoftmaxCuda::device_bytes() const {
    const auto& w = *impl_;
    return w.borrowed ? w.ws_bytes + kvm_ctx_device_bytes(w.ctx) : w.buf_bytes + kvm_ctx_device_bytes(w.ctx);
}

std::vector<double> PageSoftmaxCuda::score(const RawKvStore& keys, PageQueryView q, const QueryScoreFrame& frame,
                                           GqaScoreAggregation aggregation) {
    if (aggregation != GqaScoreAggregation::Mean && aggregation != GqaScoreAggregation::Max)
        throw std::invalid_argument("invalid page softmax CUDA aggregation");
    if ((!q.data && !q.layer_data) || !q.layer_rows || !q.rows || !q.layers || !q.head_dim || !q.kv_heads ||
        !q.query_heads || q.query_heads % q.kv_heads || q.layers != keys.config().n_layer ||
        uint64_t(q.kv_heads) * q.head_dim != keys.config().n_embd_k ||
        frame.starts.size() != frame.counts.size() || frame.starts.size() != frame.score_mask.size())
        throw std::invalid_argument("page softmax CUDA geometry mismatch");
    std::vector<size_t> enabled;
    for (size_t i = 0; i < frame.starts.size(); ++i)
        if (frame.score_mask[i]) enabled.push_back(i);
    std::vector<double> result(frame.starts.size(), 0);
    uint32_t active = 0;
    for (uint32_t l = 0; l < q.layers; ++l) {
        if (q.layer_rows[l] > q.rows) throw std::invalid_argument("page softmax CUDA row coverage mismatch");
        active += q.layer_rows[l] != 0;
    }
    if (enabled.empty() || !active) return result;
    if (enabled.size() > INT_MAX || q.query_heads > INT_MAX || q.head_dim > INT_MAX)
        throw std::length_error("page softmax CUDA geometry exceeds launch addressing");
    const size_t blocks = enabled.size(), kw = size_t(q.kv_heads) * q.head_dim, qw = size_t(q.query_heads) * q.head_dim;
    if (blocks * q.query_heads * sizeof(float) > kLogitsLimit)
        throw std::length_error("page softmax CUDA needs a larger per-row logits budget");
    const uint32_t block_tokens = keys.config().block_tokens;
    for (size_t j = 0; j < blocks; ++j) {
        const auto i = enabled[j];
        const auto begin = frame.starts[i];
        if (begin % block_tokens || begin >= frame.accepted_through || !frame.counts[i] ||
            frame.counts[i] > frame.accepted_through - begin || begin / block_tokens > UINT32_MAX ||
            !keys.has_block(uint32_t(begin / block_tokens)))
            throw std::invalid_argument("page softmax CUDA stale index extent");
    }
    auto& w = *impl_;
    DeviceBinding binding(w.device);
    checked(cudaStreamSynchronize(w.stream));
    const int agg = aggregation == GqaScoreAggregation::Max ? 1 : 0;
    const std::vector<uint8_t> mask(blocks, 1);
    const std::vector<uint32_t> ones(blocks, 1);
    std::vector<float> key(kw), scores(blocks);
    auto layer_means = [&](uint32_t l, float* dst) {
        for (size_t j = 0; j < blocks; ++j)
            keys.mean_k(uint32_t(frame.starts[enabled[j]] / block_tokens), l, dst + j * kw);
    };
    auto layer_query = [&](uint32_t l) -> const float* {
        const float* base = q.layer_data ? q.layer_data[l] : q.data + size_t(l) * q.rows * qw;
        if (!base) throw std::invalid_argument("page softmax CUDA missing active layer storage");
        return base;
    };
    if (!w.borrowed) {
        // Every layer in one library call.
        const Plan p = plan(blocks, q.query_heads, q.kv_heads, q.head_dim, q.rows);
        const size_t sums_b = aligned(size_t(q.layers) * blocks * kw * 4), q_b = aligned(size_t(q.layers) * q.rows * qw * 4);
        uint8_t* ops = w.operands(sums_b + p.counts + q_b + p.out);
        std::vector<float> hs(size_t(q.layers) * blocks * kw, 0.f), hq(size_t(q.layers) * q.rows * qw, 0.f);
        for (uint32_t l = 0; l < q.layers; ++l) {
            if (!q.layer_rows[l]) continue;
            layer_means(l, hs.data() + size_t(l) * blocks * kw);
            std::memcpy(hq.data() + size_t(l) * q.rows * qw, layer_query(l), size_t(q.layer_rows[l]) * qw * 4);
        }
        auto* d_sums = reinterpret_cast<float*>(ops);
        auto* d_counts = reinterpret_cast<uint32_t*>(ops + sums_b);
        auto* d_q = reinterpret_cast<float*>(ops + sums_b + p.counts);
        auto* d_out = reinterpret_cast<float*>(ops + sums_b + p.counts + q_b);
        checked(cudaMemcpyAsync(d_sums, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, w.stream));
        checked(cudaMemcpyAsync(d_counts, ones.data(), blocks * 4, cudaMemcpyHostToDevice, w.stream));
        checked(cudaMemcpyAsync(d_q, hq.data(), hq.size() * 4, cudaMemcpyHostToDevice, w.stream));
        throw_status(kvm_meank_score(w.ctx, d_sums, d_counts, d_q, q.layer_rows, q.layers, q.rows, q.query_heads,
                                     q.kv_heads, q.head_dim, uint32_t(blocks), mask.data(), agg, q.attention_scale,
                                     d_out, w.stream));
        checked(cudaMemcpyAsync(scores.data(), d_out, blocks * 4, cudaMemcpyDeviceToHost, w.stream));
        checked(cudaStreamSynchronize(w.stream));
        for (size_t j = 0; j < blocks; ++j) result[enabled[j]] = scores[j];
        return result;
    }
    // Borrowed workspace: one layer and at most `batch` rows per call, inside the plan.
    if (blocks > w.max_blocks || q.query_heads != w.heads || q.kv_heads != w.kvheads || q.head_dim != w.dim)
        throw std::length_error("page softmax exceeds its planned device workspace");
    const uint32_t batch = batch_rows(w.max_blocks, w.heads);
    const Plan p = plan(w.max_blocks, w.heads, w.kvheads, w.dim, batch);
    auto* d_sums = reinterpret_cast<float*>(w.ws);
    auto* d_counts = reinterpret_cast<uint32_t*>(w.ws + p.sums);
    auto* d_q = reinterpret_cast<float*>(w.ws + p.sums + p.counts);
    auto* d_out = reinterpret_cast<float*>(w.ws + p.sums + p.counts + p.queries);
    std::vector<float> hs(blocks * kw);
    checked(cudaMemcpyAsync(d_counts, ones.data(), blocks * 4, cudaMemcpyHostToDevice, w.stream));
    std::vector<double> total(blocks, 0.0);
    for (uint32_t l = 0; l < q.layers; ++l) {
        if (!q.layer_rows[l]) continue;
        checked(cudaStreamSynchronize(w.stream));  // host staging arrays are reused
        layer_means(l, hs.data());
        checked(cudaMemcpyAsync(d_sums, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, w.stream));
        const float* base = layer_query(l);
        for (uint32_t first = 0; first < q.layer_rows[l]; first += batch) {
            const uint32_t rows = std::min(batch, q.layer_rows[l] - first);
            checked(cudaMemcpyAsync(d_q, base + size_t(first) * qw, size_t(rows) * qw * 4, cudaMemcpyHostToDevice,
                                    w.stream));
            const uint32_t lr[1] = {rows};
            throw_status(kvm_meank_score(w.ctx, d_sums, d_counts, d_q, lr, 1, rows, q.query_heads, q.kv_heads,
                                         q.head_dim, uint32_t(blocks), mask.data(), agg, q.attention_scale, d_out,
                                         w.stream));
            checked(cudaMemcpyAsync(scores.data(), d_out, blocks * 4, cudaMemcpyDeviceToHost, w.stream));
            checked(cudaStreamSynchronize(w.stream));
            // One call weighs its masses by 1 / (one active layer x heads): rescale to `active` layers.
            for (size_t j = 0; j < blocks; ++j) total[j] += double(scores[j]) / active;
        }
    }
    for (size_t j = 0; j < blocks; ++j) result[enabled[j]] = total[j];
    return result;
}

std::vector<double> PageSoftmaxCuda::score_current_layer(const RawKvStore& keys, NativeCurrentLayerQuery q,
                                                         const QueryScoreFrame& frame, void* producer_stream) {
    validate_native_layer_query(q);
    const auto n = frame.starts.size();
    const auto block_tokens = keys.config().block_tokens;
    if (q.layer >= keys.config().n_layer || !block_tokens || uint64_t(q.kv_heads) * q.head_dim != keys.config().n_embd_k ||
        frame.counts.size() != n || frame.score_mask.size() != n || frame.transport_mask.size() != n ||
        uintptr_t(q.data) > UINTPTR_MAX - q.bytes)
        throw std::invalid_argument("native CUDA Query or score frame geometry mismatch");
    std::vector<size_t> enabled;
    for (size_t i = 0; i < n; ++i) {
        const auto start = frame.starts[i], count = uint64_t(frame.counts[i]);
        if (!count || count > block_tokens || start % block_tokens || start > frame.accepted_through ||
            count > frame.accepted_through - start || start / block_tokens > UINT32_MAX ||
            keys.mean_k_tokens(uint32_t(start / block_tokens), q.layer) != count)
            throw std::invalid_argument("native CUDA target-layer Mean-K coverage differs from frozen frame");
        if (frame.score_mask[i]) enabled.push_back(i);
    }
    auto& w = *impl_;
    DeviceBinding binding(w.device);
    auto stream = static_cast<cudaStream_t>(producer_stream);
    int stream_device = -1;
    checked(cudaStreamGetDevice(stream, &stream_device));
    if (stream_device != w.device) throw std::invalid_argument("native Query stream belongs to a different device");
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    checked(cudaStreamIsCapturing(stream, &capture));
    if (capture != cudaStreamCaptureStatusNone)
        throw std::invalid_argument("native Query selection requires an eager CUDA boundary");
    cudaPointerAttributes attributes{};
    checked(cudaPointerGetAttributes(&attributes, q.data));
    if (attributes.type != cudaMemoryTypeDevice || attributes.device != w.device)
        throw std::invalid_argument("native Query is not stored on its scoring CUDA device");
    std::vector<double> result(n, 0);
    if (enabled.empty()) return result;
    // The native rows, in their scalar type and strides, become dense f32 rows on
    // the host (f16 and bf16 widen exactly), then one call per batch of rows.
    std::vector<uint8_t> raw(q.bytes);
    checked(cudaMemcpyAsync(raw.data(), q.data, q.bytes, cudaMemcpyDeviceToHost, stream));
    checked(cudaStreamSynchronize(stream));
    const size_t qw = size_t(q.query_heads) * q.head_dim;
    std::vector<float> dense(size_t(q.rows) * qw);
    for (uint32_t r = 0; r < q.rows; ++r)
        for (uint32_t h = 0; h < q.query_heads; ++h)
            for (uint32_t d = 0; d < q.head_dim; ++d) {
                const uint8_t* e = raw.data() + size_t(r) * q.row_stride + size_t(h) * q.head_stride +
                                   size_t(d) * q.dimension_stride;
                float v;
                if (q.scalar == NativeQueryScalar::Float32) {
                    std::memcpy(&v, e, 4);
                } else {
                    uint16_t bits;
                    std::memcpy(&bits, e, 2);
                    if (q.scalar == NativeQueryScalar::Float16) {
                        __half_raw hr;
                        hr.x = bits;
                        v = __half2float(__half(hr));
                    } else {
                        const uint32_t u = uint32_t(bits) << 16;
                        std::memcpy(&v, &u, 4);
                    }
                }
                dense[(size_t(r) * q.query_heads + h) * q.head_dim + d] = v;
            }
    // The layer's Mean-K operands in a one-layer view of the store's geometry.
    std::vector<uint32_t> layer_rows(keys.config().n_layer, 0);
    layer_rows[q.layer] = q.rows;
    PageQueryView view{};
    std::vector<const float*> layer_data(keys.config().n_layer, nullptr);
    layer_data[q.layer] = dense.data();
    view.layer_data = layer_data.data();
    view.layer_rows = layer_rows.data();
    view.layers = keys.config().n_layer;
    view.rows = q.rows;
    view.query_heads = q.query_heads;
    view.kv_heads = q.kv_heads;
    view.head_dim = q.head_dim;
    view.attention_scale = q.attention_scale;
    return score(keys, view, frame, GqaScoreAggregation::Mean);
}

}  // namespace kvmem
