// GPU test: the reference's own kvmem::MemorySession (kvmem/src/host/memory_contract.cpp:245-365,
// linked from the reference build in oracle/_ref) drives the B200 memory backend
// (kvmem_b200/adapter) through whole working-set transfers on one GPU:
//   A  a first working set: restores land byte-exact in their slots;
//   B  device-written blocks: the evicted one is spilled to its host record before
//      its slot is reused, the retained one keeps the device bytes;
//   C  abort during the spill: previous view (tables, bytes, stamp) preserved;
//   D  a plan against a stale stamp and a second prepare while one is pending are
//      refused by the session;
//   E  a selection larger than the device slots: the backend refuses it with the
//      strong guarantee and the next transfer goes through;
//   F  abort after the restore started: the session is invalidated.
// Exit status 0 when every check holds.
#include "kvm_memory_backend.hpp"

#include <chrono>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr uint32_t kLayers = 3, kBlocks = 40, kSlots = 8, kBlockTokens = 16;
constexpr uint64_t kKBytes = 4096, kVBytes = 2048;  // per page record and layer
constexpr uint32_t kLastTokens = 9;                 // the last block is partial

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

#define REQUIRE(cond)                                                                             \
    do {                                                                                          \
        if (!(cond)) throw Failure(std::string("line ") + std::to_string(__LINE__) + ": " #cond); \
    } while (0)

void cuda(cudaError_t e) {
    if (e != cudaSuccess) throw Failure(std::string("CUDA: ") + cudaGetErrorString(e));
}

struct Store {
    uint8_t* hk = nullptr;  // host records [layer][block][kKBytes], mapped pinned
    uint8_t* hv = nullptr;
    uint8_t* dk = nullptr;  // device cache [layer][slot][kKBytes]
    uint8_t* dv = nullptr;
    Store() {
        cuda(cudaHostAlloc(reinterpret_cast<void**>(&hk), kLayers * kBlocks * kKBytes,
                           cudaHostAllocMapped | cudaHostAllocPortable));
        cuda(cudaHostAlloc(reinterpret_cast<void**>(&hv), kLayers * kBlocks * kVBytes,
                           cudaHostAllocMapped | cudaHostAllocPortable));
        cuda(cudaMalloc(&dk, kLayers * kSlots * kKBytes));
        cuda(cudaMalloc(&dv, kLayers * kSlots * kVBytes));
        cuda(cudaMemset(dk, 0, kLayers * kSlots * kKBytes));
        cuda(cudaMemset(dv, 0, kLayers * kSlots * kVBytes));
        uint64_t x = 0x9E3779B97F4A7C15ull;
        auto fill = [&](uint8_t* p, uint64_t n) {
            for (uint64_t i = 0; i < n; ++i) {
                x = x * 6364136223846793005ull + 1442695040888963407ull;
                p[i] = uint8_t(x >> 56);
            }
        };
        fill(hk, kLayers * kBlocks * kKBytes);
        fill(hv, kLayers * kBlocks * kVBytes);
    }
    ~Store() {
        cudaFreeHost(hk);
        cudaFreeHost(hv);
        cudaFree(dk);
        cudaFree(dv);
    }
    kvm_stage_layout layout() const {
        kvm_stage_layout L{};
        L.planes = 2;
        L.host_base[0] = hk;
        L.host_base[1] = hv;
        L.host_row_stride[0] = kBlocks * kKBytes;
        L.host_row_stride[1] = kBlocks * kVBytes;
        L.host_page_stride[0] = kKBytes;
        L.host_page_stride[1] = kVBytes;
        L.dev_base[0] = dk;
        L.dev_base[1] = dv;
        L.dev_row_stride[0] = kSlots * kKBytes;
        L.dev_row_stride[1] = kSlots * kVBytes;
        L.dev_slot_stride[0] = kKBytes;
        L.dev_slot_stride[1] = kVBytes;
        L.bytes[0] = kKBytes;
        L.bytes[1] = kVBytes;
        return L;
    }
    std::vector<uint8_t> cache_k() const {
        std::vector<uint8_t> v(kLayers * kSlots * kKBytes);
        cuda(cudaMemcpy(v.data(), dk, v.size(), cudaMemcpyDeviceToHost));
        return v;
    }
    std::vector<uint8_t> cache_v() const {
        std::vector<uint8_t> v(kLayers * kSlots * kVBytes);
        cuda(cudaMemcpy(v.data(), dv, v.size(), cudaMemcpyDeviceToHost));
        return v;
    }
};

struct Tables {
    std::vector<int32_t> slot_of, page_of;
    bool operator==(const Tables& o) const { return slot_of == o.slot_of && page_of == o.page_of; }
};

Tables read_tables(kvm_adapter::B200MemoryBackend& be) {
    Tables t{std::vector<int32_t>(kLayers * kBlocks), std::vector<int32_t>(kLayers * kSlots)};
    const int rc = kvm_pool_read(be.pool(), t.slot_of.data(), t.page_of.data(), be.stream());
    if (rc != KVM_OK) kvm_adapter::throw_status(rc, "kvm_pool_read");
    return t;
}

kvmem::MemoryBudget budget() {
    kvmem::MemoryBudget b;
    b.selected_tokens = 9 * kBlockTokens;
    b.device_tokens = 16 * kBlockTokens;
    b.host_payload_bytes = uint64_t(1) << 30;
    return b;
}

// prepare -> advance until Ready (bounded) -> publish.
kvmem::ExecutionView cycle(kvmem::MemorySession& s, kvm_adapter::B200MemoryBackend& be,
                           const std::vector<uint64_t>& sel, const std::vector<uint64_t>& mandatory,
                           size_t expect_spill = size_t(-1)) {
    const auto& plan = s.prepare(be.stamp(), sel, mandatory, budget());
    if (expect_spill != size_t(-1)) REQUIRE(plan.spill.size() == expect_spill);
    for (int i = 0; i < 200000 && s.phase() != kvmem::MemoryPhase::Ready; ++i) {
        s.advance();
        if (s.phase() != kvmem::MemoryPhase::Ready) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    REQUIRE(s.phase() == kvmem::MemoryPhase::Ready);
    return s.publish();
}

// Every selected block is resident in every layer and its slot holds the
// host record's bytes (or `dev_byte` for blocks listed in `device_newer`).
void verify(kvm_adapter::B200MemoryBackend& be, const Store& st, const std::vector<uint64_t>& sel,
            const std::vector<uint64_t>& device_newer = {}, uint8_t dev_byte = 0) {
    const Tables t = read_tables(be);
    const auto ck = st.cache_k(), cv = st.cache_v();
    for (uint32_t l = 0; l < kLayers; ++l) {
        uint32_t resident = 0;
        for (uint32_t p = 0; p < kBlocks; ++p) resident += t.slot_of[l * kBlocks + p] >= 0;
        REQUIRE(resident == sel.size());
        for (uint64_t id : sel) {
            const uint32_t p = uint32_t(id - 1);
            const int32_t slot = t.slot_of[l * kBlocks + p];
            REQUIRE(slot >= 0 && slot < int32_t(kSlots));
            REQUIRE(t.page_of[l * kSlots + slot] == int32_t(p));
            const uint8_t* k = ck.data() + (size_t(l) * kSlots + slot) * kKBytes;
            const uint8_t* v = cv.data() + (size_t(l) * kSlots + slot) * kVBytes;
            bool newer = false;
            for (uint64_t d : device_newer) newer |= d == id;
            if (newer) {
                for (uint64_t i = 0; i < kKBytes; ++i) REQUIRE(k[i] == dev_byte);
                for (uint64_t i = 0; i < kVBytes; ++i) REQUIRE(v[i] == dev_byte);
            } else {
                REQUIRE(std::memcmp(k, st.hk + (size_t(l) * kBlocks + p) * kKBytes, kKBytes) == 0);
                REQUIRE(std::memcmp(v, st.hv + (size_t(l) * kBlocks + p) * kVBytes, kVBytes) == 0);
            }
        }
    }
}

template <class F>
kvmem::MemoryErrorCode thrown_code(F&& f) {
    try {
        f();
    } catch (const kvmem::MemoryError& e) {
        return e.code();
    }
    throw Failure("expected a kvmem::MemoryError");
}

void run() {
    cuda(cudaSetDevice(0));
    Store st;
    kvm_adapter::B200BackendOptions opt;
    opt.device = 0;
    opt.layers = kLayers;
    opt.max_blocks = kBlocks;
    opt.slots = kSlots;
    opt.block_tokens = kBlockTokens;
    opt.ctas = 4;
    opt.layout = st.layout();
    opt.identity = {"kvmem-b200", "1", "synthetic", "paged-record-v1"};
    auto be = std::make_shared<kvm_adapter::B200MemoryBackend>(opt);
    be->begin_session(7, 1);
    for (uint32_t b = 0; b < kBlocks; ++b) be->commit_block(b + 1 == kBlocks ? kLastTokens : kBlockTokens, true);
    kvmem::MemorySession s(be);

    // A: first working set (sink + recent mandatory), everything restored.
    const std::vector<uint64_t> selA = {1, 2, 3, 10, 20, 30, 39, 40};
    const auto viewA = cycle(s, *be, selA, {1, 40}, 0);
    REQUIRE(s.phase() == kvmem::MemoryPhase::Published);
    REQUIRE(viewA.blocks.size() == selA.size());
    REQUIRE(viewA.visible_tokens == 7 * kBlockTokens + kLastTokens);
    REQUIRE(be->stamp() == viewA.stamp);
    verify(*be, st, selA);

    // B: blocks 10 and 20 are rewritten on the device; 10 is evicted (spilled), 20 retained.
    {
        const Tables t = read_tables(*be);
        for (uint32_t l = 0; l < kLayers; ++l)
            for (uint64_t id : {10u, 20u}) {
                const int32_t slot = t.slot_of[l * kBlocks + (id - 1)];
                cuda(cudaMemset(st.dk + (size_t(l) * kSlots + slot) * kKBytes, 0xA5, kKBytes));
                cuda(cudaMemset(st.dv + (size_t(l) * kSlots + slot) * kVBytes, 0xA5, kVBytes));
            }
        cuda(cudaDeviceSynchronize());
        be->device_wrote(10);
        be->device_wrote(20);
    }
    const std::vector<uint64_t> selB = {1, 2, 3, 5, 6, 20, 39, 40};
    cycle(s, *be, selB, {1, 40}, 1);
    verify(*be, st, selB, {20}, 0xA5);
    for (uint32_t l = 0; l < kLayers; ++l) {
        const uint8_t* k = st.hk + (size_t(l) * kBlocks + 9) * kKBytes;
        const uint8_t* v = st.hv + (size_t(l) * kBlocks + 9) * kVBytes;
        for (uint64_t i = 0; i < kKBytes; ++i) REQUIRE(k[i] == 0xA5);
        for (uint64_t i = 0; i < kVBytes; ++i) REQUIRE(v[i] == 0xA5);
    }
    // The spilled block's host copy is current again.
    REQUIRE(be->snapshot().blocks[9].host_version == be->snapshot().blocks[9].block.content_version);

    // C: abort during the spill keeps tables, bytes and stamp.
    {
        const Tables t0 = read_tables(*be);
        const auto k0 = st.cache_k(), v0 = st.cache_v();
        const auto stamp0 = be->stamp();
        s.prepare(be->stamp(), {4, 7, 8, 9, 11, 12, 13, 14}, {}, budget());
        s.advance();  // start_spill
        REQUIRE(s.abort() == kvmem::AbortResult::PreviousViewPreserved);
        REQUIRE(s.phase() == kvmem::MemoryPhase::Idle);
        REQUIRE(read_tables(*be) == t0);
        REQUIRE(st.cache_k() == k0 && st.cache_v() == v0);
        REQUIRE(be->stamp() == stamp0);
    }

    // D: a stale expected stamp, then a second prepare while one is pending.
    {
        auto old = be->stamp();
        old.view_version += 5;
        REQUIRE(thrown_code([&] { s.prepare(old, selB, {}, budget()); }) == kvmem::MemoryErrorCode::Stale);
        s.prepare(be->stamp(), selA, {}, budget());
        REQUIRE(thrown_code([&] { s.prepare(be->stamp(), selA, {}, budget()); }) ==
                kvmem::MemoryErrorCode::Pending);
        REQUIRE(s.abort() == kvmem::AbortResult::PreviousViewPreserved);
    }

    // E: nine blocks for eight slots: the backend refuses, nothing changes, the next transfer works.
    {
        const Tables t0 = read_tables(*be);
        const auto stamp0 = be->stamp();
        REQUIRE(thrown_code([&] { s.prepare(be->stamp(), {1, 2, 3, 4, 5, 6, 7, 8, 9}, {}, budget()); }) ==
                kvmem::MemoryErrorCode::BudgetExceeded);
        REQUIRE(s.phase() == kvmem::MemoryPhase::Idle);
        REQUIRE(read_tables(*be) == t0);
        REQUIRE(be->stamp() == stamp0);
        const std::vector<uint64_t> selE = {1, 10, 11, 12, 13, 20, 39, 40};
        cycle(s, *be, selE, {1, 40}, 0);
        // block 10's record holds the spilled device bytes, block 20 kept its slot
        verify(*be, st, selE, {10, 20}, 0xA5);
    }

    // F: abort once the restore has started: the previous view cannot be kept.
    {
        s.prepare(be->stamp(), {2, 3, 4, 5, 6, 7, 8, 9}, {}, budget());
        for (int i = 0; i < 200000 && s.phase() != kvmem::MemoryPhase::Restoring &&
                        s.phase() != kvmem::MemoryPhase::Ready;
             ++i)
            s.advance();
        REQUIRE(s.phase() == kvmem::MemoryPhase::Restoring || s.phase() == kvmem::MemoryPhase::Ready);
        REQUIRE(s.abort() == kvmem::AbortResult::SessionInvalidated);
        REQUIRE(s.phase() == kvmem::MemoryPhase::Invalid);
        REQUIRE(!be->stamp().valid);
        REQUIRE(thrown_code([&] { s.prepare(be->stamp(), selA, {}, budget()); }) ==
                kvmem::MemoryErrorCode::InvalidSession);
    }
}

}  // namespace

int main() {
    try {
        run();
    } catch (const std::exception& e) {
        std::fprintf(stderr, "memory_session_test: FAILED: %s\n", e.what());
        return 1;
    }
    std::printf("memory_session_test: OK\n");
    return 0;
}
