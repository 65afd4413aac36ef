// One decode-step recall over a history partitioned by page range across the
// GPUs of one box, in C++ over the kvm_* C ABI and NCCL: the host side a KVMem
// build uses when one history is larger than one GPU (the reference scores on
// one GPU only). Every rank runs the same step on its own stream:
//
//   per layer chunk: page LSE of the rank's page range (kvm_shard_page_lse),
//   one ncclAllGather of it, the ranges laid side by side (one 2-D copy per
//   rank), whole-row masses (kvm_page_mass_from_lse) and the top-k
//   (kvm_select_topk) -- the unsharded selection, identical on every rank --,
//   the residency plan on the rank's copy of the pool (kvm_plan_residency), and
//   on a side stream the gather of the planned restores that lie in the rank's
//   range from its own pinned records into the decode GPU's cache
//   (kvm_shard_stagein); the gather of chunk i overlaps the scoring of chunk
//   i + 1. One ncclAllReduce enqueued after the gathers ends the step: when it
//   completes on the decode rank, every rank's pages are in its cache.
//
// The decode rank's cache is `layout.dev_base`: its own memory on the decode
// rank, a peer pointer on the others (peer access between devices of one
// process, or a kvm_ipc_open mapping across processes). Compiles against
// include/kvm_recall.h, nccl.h and the CUDA runtime; links libkvm_b200.so,
// NCCL and the CUDA runtime.
#pragma once

#include "kvm_recall.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstdint>
#include <utility>
#include <vector>

namespace kvm_adapter {

struct ShardedStepOptions {
    int device = 0;
    int rank = 0, world = 1;
    ncclComm_t comm = nullptr;      // one rank per GPU, rank order = page-range order
    uint32_t layers = 0, rows = 1, q_heads = 0, kv_heads = 0, groups = 1;
    uint32_t total_pages = 0;       // pages of the whole history per layer
    std::vector<std::pair<uint32_t, uint32_t>> ranges;  // [begin, end) page range of every rank
    std::vector<std::pair<uint32_t, uint32_t>> chunks;  // (first layer, layers) of each chunk, in order
    uint32_t budget = 0;            // pages per selection row, keep pages included
    std::vector<uint32_t> keep;     // global page ids kept in every row
    uint32_t slots = 0;             // decode-cache slots per selection row
    kvm_stage_layout layout{};      // this rank's records (host_base at its first page) -> decode cache
    uint32_t stage_ctas = 0;        // CTAs of each gather launch (0 = library default)
};

class ShardedRecallStep {
public:
    // Creates the context, the chunks' residency pools and the step's buffers on
    // opts.device. Throws std::runtime_error on a CUDA or library failure.
    explicit ShardedRecallStep(ShardedStepOptions opts);
    ~ShardedRecallStep();
    ShardedRecallStep(const ShardedRecallStep&) = delete;
    ShardedRecallStep& operator=(const ShardedRecallStep&) = delete;

    // Enqueues one step on `stream` (a stream of opts.device). desc: the whole
    // step's scoring problem (desc.tokens = the GLOBAL visible token count);
    // q: the step's queries for all layers; k: this rank's K range for all
    // layers. Returns a kvm_status (the first failing call's; NCCL failures are
    // KVM_ERR_CUDA).
    int step(const kvm_score_desc& desc, const kvm_query& q, const kvm_kcache& k, cudaStream_t stream);

    // Device results of the last step: ids [layers*groups][budget] (ascending
    // page ids), counts [layers*groups]; identical on every rank.
    const uint32_t* ids() const { return ids_; }
    const uint32_t* counts() const { return n_; }
    kvm_ctx* context() const { return ctx_; }
    kvm_pool* pool(size_t chunk) const { return pools_[chunk]; }

private:
    ShardedStepOptions o_;
    kvm_ctx* ctx_ = nullptr;
    std::vector<kvm_pool*> pools_;
    std::vector<kvm_stage_layout> layouts_;
    std::vector<cudaEvent_t> events_;
    cudaEvent_t side_done_ = nullptr;
    cudaStream_t side_ = nullptr;
    uint32_t widest_ = 0;  // pages of the widest range (the all-gather slice)
    float* lse_send_ = nullptr;
    float* lse_recv_ = nullptr;
    float* lse_full_ = nullptr;
    float* mass_ = nullptr;
    uint32_t* ids_ = nullptr;
    uint32_t* n_ = nullptr;
    int32_t* flag_ = nullptr;
    void release() noexcept;
};

}  // namespace kvm_adapter
