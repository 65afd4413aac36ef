// kvmem::MemoryBackend over the kvm_transfer_* C ABI: the adapter a KVMem build
// links to put its native working set (a paged KV cache on one B200 whose page
// records live in mapped pinned host memory) behind the reference's
// memory-backend contract (kvmem/include/kvmem/memory_contract.hpp:171-195),
// driven unchanged by kvmem::MemorySession (kvmem/src/host/memory_contract.cpp:245-365).
//
// One logical block = one page of every layer: block id b (1-based) is page
// b - 1 of every pool row, and a working set selects the same blocks in every
// layer. The engine-side calls (begin_session, commit_block, device_wrote)
// stand for the engine's commit path: they keep the block catalog and the
// stamp the contract plans against.
//
// Compiles against the reference's `kvmem/memory_contract.hpp`, this
// repository's `include/kvm_recall.h` and the CUDA runtime headers; links
// libkvm_b200.so and the CUDA runtime.
#pragma once

#include "kvm_recall.h"
#include "kvmem/memory_contract.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace kvm_adapter {

struct B200BackendOptions {
    int device = 0;
    uint32_t layers = 0;        // pool rows: one selection per layer
    uint32_t max_blocks = 0;    // pool pages: blocks the history can hold
    uint32_t slots = 0;         // device cache slots per layer
    uint32_t block_tokens = 0;  // tokens per block (one native page)
    uint32_t ctas = 0;          // SMs the gathers may occupy (0 = library default)
    uint64_t drain_timeout_us = 5'000'000;
    kvm_stage_layout layout{};  // page (layer, block) <-> (host record, device slot), K and V planes
    kvmem::BackendIdentity identity;
};

// Throws the reference's exception for a kvm status: MemoryError with the same
// code for 1..8 (kvmem::MemoryErrorCode in order), std::invalid_argument /
// std::length_error for 9 / 10, MemoryError(TransferFailed) for CUDA failures
// and bounded waits that ran out.
[[noreturn]] void throw_status(int status, const std::string& what);

class B200MemoryBackend final : public kvmem::MemoryBackend {
public:
    explicit B200MemoryBackend(const B200BackendOptions& options);
    ~B200MemoryBackend() override;
    B200MemoryBackend(const B200MemoryBackend&) = delete;
    B200MemoryBackend& operator=(const B200MemoryBackend&) = delete;

    // kvmem::MemoryBackend
    kvmem::MemoryDescriptor descriptor() const override;
    kvmem::MemorySnapshot snapshot() const override;
    kvmem::MemoryStamp stamp() const noexcept override;
    std::unique_ptr<kvmem::MemoryTransfer> prepare(const kvmem::WorkingSetPlan& plan) override;
    void invalidate() noexcept override;

    // Engine side. A new session (empty catalog, nothing resident).
    void begin_session(uint64_t id, uint64_t incarnation);
    // Appends the next block of `valid_tokens` tokens; `host_copy_current` when
    // its host record already holds the block's bytes. Returns the block id.
    uint64_t commit_block(uint32_t valid_tokens, bool host_copy_current);
    // The device copy of a resident block changed: its host record is stale.
    void device_wrote(uint64_t id);

    kvm_pool* pool() const noexcept { return pool_; }
    cudaStream_t stream() const noexcept { return stream_; }
    const B200BackendOptions& options() const noexcept { return opt_; }

private:
    friend class B200Transfer;
    void published(const kvmem::WorkingSetPlan& plan, const kvmem::ExecutionView& view);
    void released() noexcept { pending_ = false; }

    B200BackendOptions opt_;
    kvm_ctx* ctx_ = nullptr;
    kvm_pool* pool_ = nullptr;
    cudaStream_t stream_ = nullptr;
    // Reserved at construction, so prepare allocates no selection scratch.
    uint32_t* d_ids_ = nullptr;  // [layers][slots]
    uint32_t* d_n_ = nullptr;    // [layers]
    uint8_t* d_stale_ = nullptr; // [layers][max_blocks]
    std::vector<uint32_t> h_ids_, h_n_;
    std::vector<uint8_t> h_stale_;
    std::vector<kvmem::BlockCopies> blocks_;
    std::vector<uint64_t> resident_;
    kvmem::MemoryStamp stamp_;
    bool pending_ = false;
};

}  // namespace kvm_adapter
