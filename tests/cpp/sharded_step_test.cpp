// C++ GPU test of kvm_adapter::ShardedRecallStep on two devices of one process
// (one thread and one NCCL rank per device, communicators from ncclCommInitAll;
// device 1 writes device 0's cache through peer access). A watchdog on the main
// thread aborts both communicators when a rank fails or the ranks have not
// finished within 120 s, so a rank that stops early never leaves the other's
// collective waiting. A 4-layer fp16 history of 40 pages is split 20 / 20;
// over three steps with different queries every rank must hold the selection
// that kvm_score_pages + kvm_select_topk give over the whole history on one
// device, and device 0's cache must hold, in the slots its pools assign, exactly
// the host records of the selected pages (K and V). Exit code 77: fewer than two
// devices (skipped); 0: pass; 1: fail.
#include "kvm_sharded_step.hpp"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>
#include <atomic>
#include <exception>
#include <chrono>
#include <random>
#include <thread>
#include <vector>

using kvm_adapter::ShardedRecallStep;
using kvm_adapter::ShardedStepOptions;

namespace {

constexpr uint32_t L = 4, HQ = 8, HKV = 2, D = 128, PT = 64, P = 40, BUDGET = 10, STEPS = 3;
constexpr uint32_t T = P * PT, RB = D * 2, PAGE_K = PT * HKV * RB, PAGE_V = 160;

#define CHECK(x)                                                                   \
    do {                                                                           \
        if (!(x)) {                                                                \
            std::fprintf(stderr, "check failed: %s (line %d)\n", #x, __LINE__); \
            return 1;                                                              \
        }                                                                          \
    } while (0)

struct Problem {
    std::vector<uint8_t> k;                // [L][T][HKV][RB] fp16 bytes (token-major)
    std::vector<uint8_t> v;                // [L][P][PAGE_V]
    std::vector<std::vector<float>> q;     // per step [L][HQ][D]
};

Problem make_problem() {
    Problem pr;
    std::mt19937 gen(7);
    std::normal_distribution<float> nd(0.f, 1.f);
    pr.k.resize(size_t(L) * T * HKV * RB);
    auto* k16 = reinterpret_cast<__half*>(pr.k.data());
    for (size_t i = 0; i < pr.k.size() / 2; ++i) k16[i] = __float2half(nd(gen));
    pr.v.resize(size_t(L) * P * PAGE_V);
    for (auto& b : pr.v) b = uint8_t(gen());
    for (uint32_t s = 0; s < STEPS; ++s) {
        std::vector<float> q(size_t(L) * HQ * D);
        for (auto& x : q) x = nd(gen);
        pr.q.push_back(q);
    }
    return pr;
}

kvm_score_desc make_desc() {
    kvm_score_desc d{};
    d.layers = L, d.q_heads = HQ, d.kv_heads = HKV, d.head_dim = D, d.tokens = T, d.page_tokens = PT, d.groups = 1;
    return d;
}

kvm_query make_query(const float* q) {
    kvm_query x{};
    x.data = q, x.type = KVM_F32, x.rows = 1;
    x.layer_stride = uint64_t(HQ) * D * 4, x.row_stride = uint64_t(HQ) * D * 4, x.head_stride = D * 4;
    return x;
}

// The unsharded selection of every step on device 0.
int reference(const Problem& pr, std::vector<std::vector<uint32_t>>& sel) {
    cudaSetDevice(0);
    kvm_ctx* ctx = nullptr;
    CHECK(kvm_ctx_create(0, &ctx) == KVM_OK);
    void *k = nullptr, *q = nullptr, *mass = nullptr, *ids = nullptr, *n = nullptr;
    CHECK(cudaMalloc(&k, pr.k.size()) == cudaSuccess);
    CHECK(cudaMemcpy(k, pr.k.data(), pr.k.size(), cudaMemcpyHostToDevice) == cudaSuccess);
    CHECK(cudaMalloc(&q, pr.q[0].size() * 4) == cudaSuccess);
    CHECK(cudaMalloc(&mass, size_t(L) * P * 4) == cudaSuccess);
    CHECK(cudaMalloc(&ids, size_t(L) * BUDGET * 4) == cudaSuccess);
    CHECK(cudaMalloc(&n, size_t(L) * 4) == cudaSuccess);
    kvm_kcache kc{};
    kc.data = k, kc.type = KVM_F16, kc.layer_stride = uint64_t(T) * HKV * RB, kc.token_stride = HKV * RB,
    kc.head_stride = RB, kc.capacity_tokens = T;
    const kvm_score_desc d = make_desc();
    const uint32_t keep[2] = {0, P - 1};
    for (uint32_t s = 0; s < STEPS; ++s) {
        CHECK(cudaMemcpy(q, pr.q[s].data(), pr.q[s].size() * 4, cudaMemcpyHostToDevice) == cudaSuccess);
        const kvm_query qq = make_query(static_cast<const float*>(q));
        CHECK(kvm_score_pages(ctx, &d, &qq, &kc, nullptr, static_cast<float*>(mass), nullptr) == KVM_OK);
        CHECK(kvm_select_topk(ctx, static_cast<float*>(mass), L, P, P, keep, 2, BUDGET, 0, static_cast<uint32_t*>(ids),
                              static_cast<uint32_t*>(n), BUDGET, nullptr) == KVM_OK);
        std::vector<uint32_t> hi(size_t(L) * BUDGET), hn(L);
        CHECK(cudaMemcpy(hi.data(), ids, hi.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
        CHECK(cudaMemcpy(hn.data(), n, hn.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
        std::vector<uint32_t> out;
        for (uint32_t l = 0; l < L; ++l) {
            out.push_back(hn[l]);
            for (uint32_t i = 0; i < hn[l]; ++i) out.push_back(hi[size_t(l) * BUDGET + i]);
        }
        sel.push_back(out);
    }
    CHECK(kvm_ctx_status(ctx, nullptr) == KVM_OK);
    for (void* p : {k, q, mass, ids, n}) cudaFree(p);
    kvm_ctx_destroy(ctx);
    return 0;
}

struct RankResult {
    int rc = 1;
    std::vector<std::vector<uint32_t>> sel;  // per step: for each layer n, ids...
    std::vector<int32_t> slot_of;           // rank 0: [L][P] after the last step
};

int run_rank(int rank, const Problem& pr, ncclComm_t comm, uint8_t* cache_k, uint8_t* cache_v, RankResult& res) {
    const int dev = rank;
    CHECK(cudaSetDevice(dev) == cudaSuccess);
    const uint32_t p0 = rank == 0 ? 0 : P / 2, p1 = rank == 0 ? P / 2 : P, lp = p1 - p0;
    // This rank's K range on its device and its page records in mapped pinned host memory.
    void* k = nullptr;
    CHECK(cudaMalloc(&k, size_t(L) * lp * PT * HKV * RB) == cudaSuccess);
    uint8_t *hk = nullptr, *hv = nullptr;
    CHECK(cudaHostAlloc(&hk, size_t(L) * lp * PAGE_K, cudaHostAllocMapped) == cudaSuccess);
    CHECK(cudaHostAlloc(&hv, size_t(L) * lp * PAGE_V, cudaHostAllocMapped) == cudaSuccess);
    for (uint32_t l = 0; l < L; ++l) {
        const uint8_t* src = pr.k.data() + (size_t(l) * T + size_t(p0) * PT) * HKV * RB;
        std::memcpy(hk + size_t(l) * lp * PAGE_K, src, size_t(lp) * PAGE_K);
        CHECK(cudaMemcpy(static_cast<uint8_t*>(k) + size_t(l) * lp * PAGE_K, src, size_t(lp) * PAGE_K,
                         cudaMemcpyHostToDevice) == cudaSuccess);
        std::memcpy(hv + size_t(l) * lp * PAGE_V, pr.v.data() + (size_t(l) * P + p0) * PAGE_V, size_t(lp) * PAGE_V);
    }
    ShardedStepOptions o;
    o.device = dev, o.rank = rank, o.world = 2, o.comm = comm;
    o.layers = L, o.rows = 1, o.q_heads = HQ, o.kv_heads = HKV, o.groups = 1, o.total_pages = P;
    o.ranges = {{0, P / 2}, {P / 2, P}};
    o.chunks = {{0, 1}, {1, L - 1}};
    o.budget = BUDGET, o.keep = {0, P - 1}, o.slots = BUDGET, o.stage_ctas = 4;
    o.layout.planes = 2;
    o.layout.host_base[0] = hk, o.layout.host_row_stride[0] = uint64_t(lp) * PAGE_K, o.layout.host_page_stride[0] = PAGE_K;
    o.layout.dev_base[0] = cache_k, o.layout.dev_row_stride[0] = uint64_t(BUDGET) * PAGE_K,
    o.layout.dev_slot_stride[0] = PAGE_K, o.layout.bytes[0] = PAGE_K;
    o.layout.host_base[1] = hv, o.layout.host_row_stride[1] = uint64_t(lp) * PAGE_V, o.layout.host_page_stride[1] = PAGE_V;
    o.layout.dev_base[1] = cache_v, o.layout.dev_row_stride[1] = uint64_t(BUDGET) * PAGE_V,
    o.layout.dev_slot_stride[1] = PAGE_V, o.layout.bytes[1] = PAGE_V;
    {
        ShardedRecallStep step(o);
        cudaStream_t s;
        CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess);
        void* q = nullptr;
        CHECK(cudaMalloc(&q, pr.q[0].size() * 4) == cudaSuccess);
        kvm_kcache kc{};
        kc.data = k, kc.type = KVM_F16, kc.layer_stride = uint64_t(lp) * PT * HKV * RB, kc.token_stride = HKV * RB,
        kc.head_stride = RB, kc.capacity_tokens = uint64_t(lp) * PT;
        const kvm_score_desc d = make_desc();
        for (uint32_t st = 0; st < STEPS; ++st) {
            CHECK(cudaMemcpyAsync(q, pr.q[st].data(), pr.q[st].size() * 4, cudaMemcpyHostToDevice, s) == cudaSuccess);
            const kvm_query qq = make_query(static_cast<const float*>(q));
            CHECK(step.step(d, qq, kc, s) == KVM_OK);
            CHECK(cudaStreamSynchronize(s) == cudaSuccess);
            std::vector<uint32_t> hi(size_t(L) * BUDGET), hn(L);
            CHECK(cudaMemcpy(hi.data(), step.ids(), hi.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
            CHECK(cudaMemcpy(hn.data(), step.counts(), hn.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
            std::vector<uint32_t> out;
            for (uint32_t l = 0; l < L; ++l) {
                out.push_back(hn[l]);
                for (uint32_t i = 0; i < hn[l]; ++i) out.push_back(hi[size_t(l) * BUDGET + i]);
            }
            res.sel.push_back(out);
        }
        CHECK(kvm_ctx_status(step.context(), s) == KVM_OK);
        if (rank == 0) {  // the residency after the last step: layer 0 in chunk 0, layers 1.. in chunk 1
            res.slot_of.assign(size_t(L) * P, -1);
            CHECK(kvm_pool_read(step.pool(0), res.slot_of.data(), nullptr, s) == KVM_OK);
            CHECK(kvm_pool_read(step.pool(1), res.slot_of.data() + P, nullptr, s) == KVM_OK);
        }
        cudaFree(q);
        cudaStreamDestroy(s);
    }
    cudaFree(k);
    cudaFreeHost(hk);
    cudaFreeHost(hv);
    res.rc = 0;
    return 0;
}

}  // namespace

int main() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n < 2) {
        std::printf("skipped: needs two devices\n");
        return 77;
    }
    int can = 0;
    cudaDeviceCanAccessPeer(&can, 1, 0);
    if (!can) {
        std::printf("skipped: device 1 cannot access device 0\n");
        return 77;
    }
    const Problem pr = make_problem();
    std::vector<std::vector<uint32_t>> want;
    if (reference(pr, want)) return 1;
    cudaSetDevice(1);
    cudaDeviceEnablePeerAccess(0, 0);
    cudaGetLastError();
    cudaSetDevice(0);
    uint8_t *cache_k = nullptr, *cache_v = nullptr;
    CHECK(cudaMalloc(&cache_k, size_t(L) * BUDGET * PAGE_K) == cudaSuccess);
    CHECK(cudaMalloc(&cache_v, size_t(L) * BUDGET * PAGE_V) == cudaSuccess);
    CHECK(cudaMemset(cache_k, 0, size_t(L) * BUDGET * PAGE_K) == cudaSuccess);
    CHECK(cudaMemset(cache_v, 0, size_t(L) * BUDGET * PAGE_V) == cudaSuccess);
    ncclComm_t comms[2];
    const int devs[2] = {0, 1};
    CHECK(ncclCommInitAll(comms, 2, devs) == ncclSuccess);
    RankResult r[2];
    std::atomic<int> finished{0}, failed{0};
    auto body = [&](int rank) {
        try {
            run_rank(rank, pr, comms[rank], cache_k, cache_v, r[rank]);
        } catch (const std::exception& e) {
            std::fprintf(stderr, "rank %d: %s\n", rank, e.what());
        }
        if (r[rank].rc) failed = 1;
        ++finished;
    };
    std::thread t0(body, 0), t1(body, 1);
    const auto until = std::chrono::steady_clock::now() + std::chrono::seconds(120);
    while (finished < 2 && !failed && std::chrono::steady_clock::now() < until)
        std::this_thread::sleep_for(std::chrono::milliseconds(10));
    const bool abort = finished < 2;
    if (abort) {
        std::fprintf(stderr, "a rank failed or the ranks did not finish: aborting the communicators\n");
        for (auto c : comms) ncclCommAbort(c);
    }
    t0.join();
    t1.join();
    if (!abort)
        for (auto c : comms) ncclCommDestroy(c);
    CHECK(!abort);
    RankResult &r0 = r[0], &r1 = r[1];
    CHECK(r0.rc == 0 && r1.rc == 0);
    CHECK(r0.sel == want);
    CHECK(r1.sel == want);
    // Device 0's cache after the last step: every selected page in its slot, byte for byte.
    cudaSetDevice(0);
    std::vector<uint8_t> ck(size_t(L) * BUDGET * PAGE_K), cv(size_t(L) * BUDGET * PAGE_V);
    CHECK(cudaMemcpy(ck.data(), cache_k, ck.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(cudaMemcpy(cv.data(), cache_v, cv.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    const auto& last = want.back();
    size_t pos = 0, checked = 0;
    for (uint32_t l = 0; l < L; ++l) {
        const uint32_t cnt = last[pos++];
        for (uint32_t i = 0; i < cnt; ++i) {
            const uint32_t p = last[pos++];
            const int32_t slot = r0.slot_of[size_t(l) * P + p];
            CHECK(slot >= 0 && uint32_t(slot) < BUDGET);
            const uint8_t* kpage = pr.k.data() + (size_t(l) * T + size_t(p) * PT) * HKV * RB;
            CHECK(std::memcmp(ck.data() + (size_t(l) * BUDGET + slot) * PAGE_K, kpage, PAGE_K) == 0);
            CHECK(std::memcmp(cv.data() + (size_t(l) * BUDGET + slot) * PAGE_V,
                              pr.v.data() + (size_t(l) * P + p) * PAGE_V, PAGE_V) == 0);
            ++checked;
        }
    }
    cudaFree(cache_k);
    cudaFree(cache_v);
    std::printf("sharded step ok: %u steps, selections equal on both ranks and to the unsharded pick, %zu pages "
                "checked in device 0's cache\n",
                STEPS, checked);
    return 0;
}
