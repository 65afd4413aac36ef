// kvmem::MemoryBackend / MemoryTransfer over the kvm_transfer_* C ABI (see the
// header). Each contract operation is one C-ABI call; the catalog, stamp and
// resident set follow the rules kvmem::plan_working_set checks
// (kvmem/src/host/memory_contract.cpp:150-225).
#include "kvm_memory_backend.hpp"

#include <algorithm>
#include <stdexcept>

namespace kvm_adapter {
namespace {

using kvmem::MemoryError;
using kvmem::MemoryErrorCode;

// Binds the backend's device for the scope and restores the caller's.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
        if (prev_ != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        if (prev_ >= 0) cudaSetDevice(prev_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int prev_ = -1;
};

void check(int status, const char* what) {
    if (status != KVM_OK) throw_status(status, what);
}

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw MemoryError(MemoryErrorCode::TransferFailed, std::string(what) + ": " + cudaGetErrorString(e));
    }
}

}  // namespace

[[noreturn]] void throw_status(int status, const std::string& what) {
    const std::string msg = what + ": kvm status " + std::to_string(status);
    if (status >= KVM_ERR_INVALID_PLAN && status <= KVM_ERR_INVALID_SESSION)
        throw MemoryError(static_cast<MemoryErrorCode>(status - KVM_ERR_INVALID_PLAN), msg);
    if (status == KVM_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    if (status == KVM_ERR_LENGTH) throw std::length_error(msg);
    throw MemoryError(MemoryErrorCode::TransferFailed, msg);
}

// One prepared working-set transfer. Owns its kvm_transfer; the backend
// outlives it (MemorySession keeps the backend while a transfer is pending).
class B200Transfer final : public kvmem::MemoryTransfer {
public:
    B200Transfer(B200MemoryBackend& backend, kvm_transfer* t, const kvmem::WorkingSetPlan& plan)
        : be_(backend), t_(t), plan_(plan) {}
    ~B200Transfer() override {
        DeviceGuard guard(be_.opt_.device);
        kvm_transfer_destroy(t_);  // aborts a still pending transfer first
        be_.released();
    }

    void start_spill() override {
        DeviceGuard guard(be_.opt_.device);
        // Only evicted blocks without a current host copy are written back.
        const uint8_t* stale = plan_.spill.empty() ? nullptr : be_.d_stale_;
        check(kvm_transfer_start_spill(t_, &be_.opt_.layout, stale, be_.opt_.ctas, be_.stream_), "start_spill");
    }

    kvmem::TransferPoll poll() override {
        DeviceGuard guard(be_.opt_.device);
        const int rc = kvm_transfer_poll(t_);
        if (rc == KVM_ERR_PENDING) return {kvmem::TransferStatus::Pending, ""};
        if (rc == KVM_OK) return {kvmem::TransferStatus::Complete, ""};
        return {kvmem::TransferStatus::Failed, "kvm_transfer_poll: kvm status " + std::to_string(rc)};
    }

    void start_restore() override {
        DeviceGuard guard(be_.opt_.device);
        check(kvm_transfer_start_restore(t_, &be_.opt_.layout, be_.opt_.ctas, be_.stream_), "start_restore");
    }

    void publish(const kvmem::ExecutionView& view) override {
        DeviceGuard guard(be_.opt_.device);
        check(kvm_transfer_publish(t_, be_.stream_), "publish");
        be_.published(plan_, view);
    }

    kvmem::AbortResult abort() noexcept override {
        DeviceGuard guard(be_.opt_.device);
        int kept = 0;
        const int rc = kvm_transfer_abort(t_, be_.opt_.drain_timeout_us, &kept);
        return rc == KVM_OK && kept ? kvmem::AbortResult::PreviousViewPreserved
                                    : kvmem::AbortResult::SessionInvalidated;
    }

private:
    B200MemoryBackend& be_;
    kvm_transfer* t_;
    kvmem::WorkingSetPlan plan_;
};

B200MemoryBackend::B200MemoryBackend(const B200BackendOptions& options) : opt_(options) {
    if (!opt_.layers || !opt_.max_blocks || !opt_.slots || !opt_.block_tokens || opt_.slots > opt_.max_blocks)
        throw std::invalid_argument("B200MemoryBackend: layers, blocks, slots and block tokens must be positive");
    if (opt_.layout.planes != 2 || !opt_.layout.bytes[0] || !opt_.layout.bytes[1])
        throw std::invalid_argument("B200MemoryBackend: the layout needs a key and a value plane");
    DeviceGuard guard(opt_.device);
    try {
        check(kvm_ctx_create(opt_.device, &ctx_), "kvm_ctx_create");
        check(kvm_pool_create(ctx_, opt_.layers, opt_.max_blocks, opt_.slots, &pool_), "kvm_pool_create");
        check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        check_cuda(cudaMalloc(&d_ids_, size_t(opt_.layers) * opt_.slots * sizeof(uint32_t)), "cudaMalloc");
        check_cuda(cudaMalloc(&d_n_, size_t(opt_.layers) * sizeof(uint32_t)), "cudaMalloc");
        check_cuda(cudaMalloc(&d_stale_, size_t(opt_.layers) * opt_.max_blocks), "cudaMalloc");
    } catch (...) {
        cudaFree(d_stale_);
        cudaFree(d_n_);
        cudaFree(d_ids_);
        if (stream_) cudaStreamDestroy(stream_);
        if (pool_) kvm_pool_destroy(pool_);
        if (ctx_) kvm_ctx_destroy(ctx_);
        throw;
    }
    h_ids_.assign(size_t(opt_.layers) * opt_.slots, 0u);
    h_n_.assign(opt_.layers, 0u);
    h_stale_.assign(size_t(opt_.layers) * opt_.max_blocks, 0u);
}

B200MemoryBackend::~B200MemoryBackend() {
    DeviceGuard guard(opt_.device);
    cudaStreamSynchronize(stream_);
    cudaFree(d_stale_);
    cudaFree(d_n_);
    cudaFree(d_ids_);
    kvm_pool_destroy(pool_);
    kvm_ctx_destroy(ctx_);
    cudaStreamDestroy(stream_);
}

kvmem::MemoryDescriptor B200MemoryBackend::descriptor() const {
    kvmem::MemoryDescriptor d;
    d.identity = opt_.identity;
    auto& L = d.layout;
    L.format = "kvm-b200/page-record";
    L.version = 1;
    L.block_tokens = opt_.block_tokens;
    L.alignment = 16;
    uint64_t off = 0;
    for (uint32_t l = 0; l < opt_.layers; ++l)
        for (uint32_t j = 0; j < 2; ++j) {
            kvmem::PayloadPlane p;
            p.layer = l;
            p.kind = j == 0 ? kvmem::PayloadPlaneKind::Key : kvmem::PayloadPlaneKind::Value;
            p.offset = off;
            p.bytes = opt_.layout.bytes[j];
            p.alignment = 16;
            // Token rows of a page record are contiguous when the page divides evenly.
            p.token_stride = p.bytes % opt_.block_tokens == 0 ? p.bytes / opt_.block_tokens : 0;
            L.planes.push_back(p);
            off += (p.bytes + 15) / 16 * 16;
        }
    L.record_bytes = off;
    auto& c = d.capabilities;
    c.page_tokens = opt_.block_tokens;
    c.max_position = uint64_t(opt_.max_blocks) * opt_.block_tokens;
    c.native_payload = true;
    c.sparse_view = true;
    c.original_rope_positions = true;  // pages are restored byte-exact at their original positions
    c.asynchronous_transfer = true;
    return d;
}

kvmem::MemorySnapshot B200MemoryBackend::snapshot() const {
    kvmem::MemorySnapshot s;
    s.stamp = stamp_;
    s.blocks = blocks_;
    s.resident = resident_;
    return s;
}

kvmem::MemoryStamp B200MemoryBackend::stamp() const noexcept { return stamp_; }

void B200MemoryBackend::invalidate() noexcept { stamp_.valid = false; }

void B200MemoryBackend::begin_session(uint64_t id, uint64_t incarnation) {
    if (pending_) throw MemoryError(MemoryErrorCode::Pending, "a working-set transfer is pending");
    if (!id || !incarnation) throw std::invalid_argument("begin_session: session id and incarnation are nonzero");
    DeviceGuard guard(opt_.device);
    check(kvm_pool_reset(pool_, stream_), "kvm_pool_reset");
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    blocks_.clear();
    resident_.clear();
    stamp_ = kvmem::MemoryStamp{};
    stamp_.valid = true;
    stamp_.session = {id, incarnation};
    stamp_.history_revision = 1;
    stamp_.execution_history = 1;
}

uint64_t B200MemoryBackend::commit_block(uint32_t valid_tokens, bool host_copy_current) {
    if (!stamp_.valid) throw MemoryError(MemoryErrorCode::InvalidSession, "commit_block: no valid session");
    if (pending_) throw MemoryError(MemoryErrorCode::Pending, "commit_block: a working-set transfer is pending");
    if (!valid_tokens || valid_tokens > opt_.block_tokens || blocks_.size() >= opt_.max_blocks)
        throw std::invalid_argument("commit_block: block size or catalog capacity exceeded");
    if (!blocks_.empty() && blocks_.back().block.valid_tokens != opt_.block_tokens)
        throw std::invalid_argument("commit_block: the previous block is still partial");
    kvmem::BlockCopies c;
    c.block.session = stamp_.session;
    c.block.id = blocks_.size() + 1;
    c.block.original_start = stamp_.frontier;
    c.block.valid_tokens = valid_tokens;
    c.block.content_version = 1;
    c.block.statistics_version = 1;
    c.host_version = host_copy_current ? 1 : 0;
    blocks_.push_back(c);
    stamp_.frontier += valid_tokens;
    ++stamp_.history_revision;
    return c.block.id;
}

void B200MemoryBackend::device_wrote(uint64_t id) {
    if (pending_) throw MemoryError(MemoryErrorCode::Pending, "device_wrote: a working-set transfer is pending");
    if (!id || id > blocks_.size() || !std::binary_search(resident_.begin(), resident_.end(), id))
        throw std::invalid_argument("device_wrote: the block is not resident");
    ++blocks_[id - 1].block.content_version;
    ++stamp_.history_revision;
}

std::unique_ptr<kvmem::MemoryTransfer> B200MemoryBackend::prepare(const kvmem::WorkingSetPlan& plan) {
    if (!stamp_.valid) throw MemoryError(MemoryErrorCode::InvalidSession, "prepare: session invalidated");
    if (pending_) throw MemoryError(MemoryErrorCode::Pending, "prepare: a working-set transfer is pending");
    if (!(plan.expected == stamp_)) throw MemoryError(MemoryErrorCode::Stale, "prepare: plan of another stamp");
    std::vector<uint32_t> pages;
    for (const auto& vb : plan.next.blocks) {
        const uint64_t id = vb.block.id;
        if (!id || id > blocks_.size() || !(blocks_[id - 1].block == vb.block))
            throw MemoryError(MemoryErrorCode::Stale, "prepare: view block is not in the catalog");
        pages.push_back(uint32_t(id - 1));
    }
    std::sort(pages.begin(), pages.end());
    if (std::adjacent_find(pages.begin(), pages.end()) != pages.end())
        throw MemoryError(MemoryErrorCode::InvalidPlan, "prepare: duplicate view block");
    if (pages.size() > opt_.slots)
        throw MemoryError(MemoryErrorCode::BudgetExceeded, "prepare: selection exceeds the device slots");
    std::fill(h_stale_.begin(), h_stale_.end(), uint8_t(0));
    for (const auto& b : plan.spill) {
        if (!b.id || b.id > blocks_.size())
            throw MemoryError(MemoryErrorCode::InvalidPlan, "prepare: unknown spill block");
        for (uint32_t l = 0; l < opt_.layers; ++l) h_stale_[size_t(l) * opt_.max_blocks + (b.id - 1)] = 1;
    }
    for (uint32_t l = 0; l < opt_.layers; ++l) {
        std::copy(pages.begin(), pages.end(), h_ids_.begin() + size_t(l) * opt_.slots);
        h_n_[l] = uint32_t(pages.size());
    }
    DeviceGuard guard(opt_.device);
    check_cuda(cudaMemcpyAsync(d_ids_, h_ids_.data(), h_ids_.size() * sizeof(uint32_t), cudaMemcpyHostToDevice,
                               stream_),
               "cudaMemcpyAsync");
    check_cuda(cudaMemcpyAsync(d_n_, h_n_.data(), h_n_.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_),
               "cudaMemcpyAsync");
    check_cuda(cudaMemcpyAsync(d_stale_, h_stale_.data(), h_stale_.size(), cudaMemcpyHostToDevice, stream_),
               "cudaMemcpyAsync");
    kvm_transfer* t = nullptr;
    check(kvm_transfer_prepare(ctx_, pool_, d_ids_, d_n_, opt_.slots, 0, stream_, &t), "kvm_transfer_prepare");
    pending_ = true;
    try {
        return std::make_unique<B200Transfer>(*this, t, plan);
    } catch (...) {
        kvm_transfer_destroy(t);
        pending_ = false;
        throw;
    }
}

void B200MemoryBackend::published(const kvmem::WorkingSetPlan& plan, const kvmem::ExecutionView& view) {
    resident_.clear();
    for (const auto& vb : view.blocks) resident_.push_back(vb.block.id);
    std::sort(resident_.begin(), resident_.end());
    for (const auto& b : plan.spill) blocks_[b.id - 1].host_version = blocks_[b.id - 1].block.content_version;
    stamp_ = view.stamp;
}

}  // namespace kvm_adapter
