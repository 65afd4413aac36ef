// ShardedRecallStep: see kvm_sharded_step.hpp.
#include "kvm_sharded_step.hpp"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace kvm_adapter {

namespace {

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void check_kvm(int rc, const char* what) {
    if (rc != KVM_OK) throw std::runtime_error(std::string(what) + ": kvm status " + std::to_string(rc));
}

// Restores the caller's current device on scope exit.
struct DeviceScope {
    int saved = -1;
    explicit DeviceScope(int device) {
        cudaGetDevice(&saved);
        check_cuda(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceScope() {
        if (saved >= 0) cudaSetDevice(saved);
    }
};

}  // namespace

ShardedRecallStep::ShardedRecallStep(ShardedStepOptions opts) : o_(std::move(opts)) {
    if (o_.world < 1 || o_.rank < 0 || o_.rank >= o_.world || int(o_.ranges.size()) != o_.world ||
        o_.chunks.empty() || !o_.budget || !o_.layers || !o_.total_pages || !o_.slots)
        throw std::invalid_argument("ShardedRecallStep: incomplete geometry");
    if (o_.world > 1 && !o_.comm) throw std::invalid_argument("ShardedRecallStep: no communicator");
    uint32_t covered = 0;
    for (const auto& r : o_.ranges) {
        if (r.first != covered || r.second <= r.first) throw std::invalid_argument("ShardedRecallStep: page ranges");
        covered = r.second;
        widest_ = std::max(widest_, r.second - r.first);
    }
    if (covered != o_.total_pages) throw std::invalid_argument("ShardedRecallStep: page ranges");
    DeviceScope scope(o_.device);
    try {
        check_kvm(kvm_ctx_create(o_.device, &ctx_), "kvm_ctx_create");
        uint32_t widest_chunk = 0;
        for (const auto& c : o_.chunks) {
            widest_chunk = std::max(widest_chunk, c.second);
            kvm_pool* p = nullptr;
            check_kvm(kvm_pool_create(ctx_, c.second * o_.groups, o_.total_pages, o_.slots, &p), "kvm_pool_create");
            pools_.push_back(p);
            kvm_stage_layout l = o_.layout;  // the chunk's rows: layer c.first onwards
            for (uint32_t j = 0; j < l.planes; ++j) {
                l.host_base[j] = static_cast<const uint8_t*>(l.host_base[j]) +
                                 uint64_t(c.first) * o_.groups * l.host_row_stride[j];
                l.dev_base[j] = static_cast<uint8_t*>(l.dev_base[j]) + uint64_t(c.first) * o_.groups * l.dev_row_stride[j];
            }
            layouts_.push_back(l);
            cudaEvent_t e;
            check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
            events_.push_back(e);
        }
        check_cuda(cudaEventCreateWithFlags(&side_done_, cudaEventDisableTiming), "cudaEventCreate");
        check_cuda(cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking), "cudaStreamCreate");
        const size_t heads = size_t(widest_chunk) * o_.rows * o_.q_heads;
        check_cuda(cudaMalloc(&lse_send_, heads * widest_ * sizeof(float)), "cudaMalloc");
        check_cuda(cudaMalloc(&lse_recv_, heads * widest_ * o_.world * sizeof(float)), "cudaMalloc");
        check_cuda(cudaMalloc(&lse_full_, heads * o_.total_pages * sizeof(float)), "cudaMalloc");
        const size_t srows = size_t(o_.layers) * o_.groups;
        check_cuda(cudaMalloc(&mass_, srows * o_.total_pages * sizeof(float)), "cudaMalloc");
        check_cuda(cudaMalloc(&ids_, srows * o_.budget * sizeof(uint32_t)), "cudaMalloc");
        check_cuda(cudaMalloc(&n_, srows * sizeof(uint32_t)), "cudaMalloc");
        check_cuda(cudaMalloc(&flag_, sizeof(int32_t)), "cudaMalloc");
        check_cuda(cudaMemset(flag_, 0, sizeof(int32_t)), "cudaMemset");
    } catch (...) {
        release();
        throw;
    }
}

ShardedRecallStep::~ShardedRecallStep() { release(); }

void ShardedRecallStep::release() noexcept {
    int saved = -1;
    cudaGetDevice(&saved);
    cudaSetDevice(o_.device);
    if (side_) cudaStreamSynchronize(side_);
    for (auto* p : pools_) kvm_pool_destroy(p);
    pools_.clear();
    for (auto e : events_) cudaEventDestroy(e);
    events_.clear();
    if (side_done_) cudaEventDestroy(side_done_);
    if (side_) cudaStreamDestroy(side_);
    for (void* p : {static_cast<void*>(lse_send_), static_cast<void*>(lse_recv_), static_cast<void*>(lse_full_),
                    static_cast<void*>(mass_), static_cast<void*>(ids_), static_cast<void*>(n_),
                    static_cast<void*>(flag_)})
        if (p) cudaFree(p);
    lse_send_ = lse_recv_ = lse_full_ = mass_ = nullptr;
    ids_ = n_ = nullptr;
    flag_ = nullptr;
    side_done_ = nullptr;
    side_ = nullptr;
    if (ctx_) kvm_ctx_destroy(ctx_);
    ctx_ = nullptr;
    if (saved >= 0) cudaSetDevice(saved);
}

int ShardedRecallStep::step(const kvm_score_desc& desc, const kvm_query& q, const kvm_kcache& k, cudaStream_t stream) {
    if (desc.layers != o_.layers || desc.q_heads != o_.q_heads || desc.kv_heads != o_.kv_heads ||
        desc.groups != o_.groups || q.rows != o_.rows)
        return KVM_ERR_INVALID_ARGUMENT;
    int saved = -1;
    cudaGetDevice(&saved);
    if (cudaSetDevice(o_.device) != cudaSuccess) return KVM_ERR_CUDA;
    const uint32_t page0 = o_.ranges[o_.rank].first, local = o_.ranges[o_.rank].second - page0;
    const uint32_t P = o_.total_pages;
    int rc = KVM_OK;
    for (size_t ci = 0; ci < o_.chunks.size() && rc == KVM_OK; ++ci) {
        const uint32_t l0 = o_.chunks[ci].first, nl = o_.chunks[ci].second;
        kvm_score_desc d = desc;
        d.layers = nl;
        kvm_query qc = q;
        qc.data = static_cast<const uint8_t*>(q.data) + uint64_t(l0) * q.layer_stride;
        kvm_kcache kc = k;
        kc.data = static_cast<const uint8_t*>(k.data) + uint64_t(l0) * k.layer_stride;
        const uint64_t heads = uint64_t(nl) * o_.rows * o_.q_heads;
        // 1. this rank's page LSE, then every rank's, laid out [heads][all pages]
        if ((rc = kvm_shard_page_lse(ctx_, &d, &qc, &kc, page0, local, lse_send_, stream)) != KVM_OK) break;
        float* gathered = lse_send_;
        if (o_.world > 1) {
            if (ncclAllGather(lse_send_, lse_recv_, heads * widest_, ncclFloat, o_.comm, stream) != ncclSuccess) {
                rc = KVM_ERR_CUDA;
                break;
            }
            gathered = lse_recv_;
        }
        float* full = lse_send_;
        if (o_.world > 1) {
            full = lse_full_;
            for (int w = 0; w < o_.world && rc == KVM_OK; ++w) {
                const uint32_t b = o_.ranges[w].first, lp = o_.ranges[w].second - b;
                if (cudaMemcpy2DAsync(full + b, size_t(P) * sizeof(float), gathered + size_t(w) * heads * widest_,
                                      size_t(lp) * sizeof(float), size_t(lp) * sizeof(float), heads,
                                      cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
                    rc = KVM_ERR_CUDA;
            }
            if (rc != KVM_OK) break;
        }
        // 2. whole-row masses and the selection of the chunk's rows (the same on every rank)
        const uint32_t r0 = l0 * o_.groups, nr = nl * o_.groups;
        float* mass = mass_ + size_t(r0) * P;
        uint32_t* ids = ids_ + size_t(r0) * o_.budget;
        uint32_t* n = n_ + r0;
        if ((rc = kvm_page_mass_from_lse(ctx_, &d, o_.rows, full, nullptr, mass, stream)) != KVM_OK) break;
        if ((rc = kvm_select_topk(ctx_, mass, nr, P, P, o_.keep.data(), uint32_t(o_.keep.size()), o_.budget, 0, ids,
                                  n, o_.budget, stream)) != KVM_OK)
            break;
        // 3. the plan on this rank's copy of the pool, and the gather of this rank's range
        if ((rc = kvm_plan_residency(ctx_, pools_[ci], ids, n, o_.budget, 0, nullptr, nullptr, stream)) != KVM_OK)
            break;
        if (cudaEventRecord(events_[ci], stream) != cudaSuccess ||
            cudaStreamWaitEvent(side_, events_[ci], 0) != cudaSuccess) {
            rc = KVM_ERR_CUDA;
            break;
        }
        rc = kvm_shard_stagein(ctx_, pools_[ci], &layouts_[ci], page0, local, o_.stage_ctas, side_);
    }
    if (rc == KVM_OK) {
        if (cudaEventRecord(side_done_, side_) != cudaSuccess || cudaStreamWaitEvent(stream, side_done_, 0) != cudaSuccess)
            rc = KVM_ERR_CUDA;
        else if (o_.world > 1 &&
                 ncclAllReduce(flag_, flag_, 1, ncclInt32, ncclMax, o_.comm, stream) != ncclSuccess)
            rc = KVM_ERR_CUDA;
    }
    if (saved >= 0) cudaSetDevice(saved);
    return rc;
}

}  // namespace kvm_adapter
