// Context definition shared by the library's translation units, and the
// templated launcher of the page log-sum-exp kernel (instantiated once per key
// type in lse_<type>.cu so the variants compile in parallel).
#pragma once
#include <algorithm>
#include <cuda.h>
#include <mutex>
#include <vector>

#include "page_mass.cuh"
#include "page_mass_mma.cuh"
#include "page_mass_q.cuh"

struct kvm_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t side = nullptr;  // stage-in stream of kvm_recall_step
    std::vector<cudaEvent_t> events;
    cudaEvent_t side_done = nullptr;
    kvmb::DeviceStatus* status = nullptr;       // device
    kvmb::DeviceStatus* status_host = nullptr;  // pinned
    void* ws = nullptr;                         // scoring workspace
    size_t ws_bytes = 0;
    bool ws_borrowed = false;
    void* small = nullptr;  // device copy of short host-built tables
    size_t small_bytes = 0;
    void* aux = nullptr;  // device copy of per-call host-built tables (propagation weights)
    size_t aux_bytes = 0;
    cudaEvent_t aux_done = nullptr;  // recorded after the last kernel that read `aux`
    bool aux_pending = false;
    std::vector<uint32_t> keep_cached;
    bool keep_valid = false;
    uint64_t launches = 0;
    // kvm_stagein_copies: two op lists in mapped pinned memory, used in turn; a list
    // is rewritten only after the gather that read it (its event) is done.
    struct CopyList {
        void* host = nullptr;  // kvmb::CopyOp[cap], mapped
        uint32_t cap = 0;
        cudaEvent_t done = nullptr;
        bool pending = false;
    } copy_lists[2];
    int copy_next = 0;
};

namespace kvmb {

template <int KT, int LPR, int VP, bool MASK>
int launch_lse_t(kvm_ctx* c, const LseParams& p, size_t smem, cudaStream_t s) {
    auto fn = page_lse_kernel<KT, LPR, VP, MASK>;
    if (smem_attr(reinterpret_cast<const void*>(fn), 200 * 1024) != cudaSuccess) return KVM_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kLseThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    if (per_sm < 1) return KVM_ERR_UNSUPPORTED;
    const uint32_t units = p.layers * p.pages;
    const uint32_t grid = std::min<uint32_t>(units, uint32_t(c->num_sms * per_sm));
    fn<<<grid, kLseThreads, smem, s>>>(p);
    ++c->launches;
    if (cudaGetLastError() != cudaSuccess) return KVM_ERR_CUDA;
    return KVM_OK;
}

template <int KT, int LPR, int VP>
int launch_lse_m(kvm_ctx* c, const LseParams& p, size_t smem, cudaStream_t s) {
    return p.mask ? launch_lse_t<KT, LPR, VP, true>(c, p, smem, s) : launch_lse_t<KT, LPR, VP, false>(c, p, smem, s);
}

template <int KT, int LPR>
int launch_lse_v(kvm_ctx* c, const LseParams& p, int vp, size_t smem, cudaStream_t s) {
    switch (vp) {
        case 1: return launch_lse_m<KT, LPR, 1>(c, p, smem, s);
        case 2: return launch_lse_m<KT, LPR, 2>(c, p, smem, s);
        case 4: return launch_lse_m<KT, LPR, 4>(c, p, smem, s);
        default: return launch_lse_m<KT, LPR, 8>(c, p, smem, s);
    }
}

template <int KT>
int launch_lse_kt(kvm_ctx* c, const LseParams& p, int lpr, int vp, size_t smem, cudaStream_t s) {
    switch (lpr) {
        case 8: return launch_lse_v<KT, 8>(c, p, vp, smem, s);
        case 16: return launch_lse_v<KT, 16>(c, p, vp, smem, s);
        default: return launch_lse_v<KT, 32>(c, p, vp, smem, s);
    }
}

template <int KT, int KK, bool MASK>
int launch_lse_mma_t(kvm_ctx* c, const LseParams& p, size_t smem, cudaStream_t s) {
    auto fn = page_lse_mma_kernel<KT, KK, MASK>;
    if (smem_attr(reinterpret_cast<const void*>(fn), 200 * 1024) != cudaSuccess) return KVM_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kLseThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    if (per_sm < 1) return KVM_ERR_UNSUPPORTED;
    const uint32_t units = p.layers * p.pages;
    const uint32_t grid = std::min<uint32_t>(units, uint32_t(c->num_sms * per_sm));
    fn<<<grid, kLseThreads, smem, s>>>(p);
    ++c->launches;
    if (cudaGetLastError() != cudaSuccess) return KVM_ERR_CUDA;
    return KVM_OK;
}

// Tensor-core scorer for fp16 / q8_0 / q4_0 keys; kk = head_dim / 32.
template <int KT>
int launch_lse_mma_kt(kvm_ctx* c, const LseParams& p, int kk, size_t smem, cudaStream_t s) {
    if constexpr (KT == KVM_F16 || KT == KVM_Q8_0 || KT == KVM_Q4_0) {
        const bool m = p.mask != nullptr;
        switch (kk) {
            case 2: return m ? launch_lse_mma_t<KT, 2, true>(c, p, smem, s) : launch_lse_mma_t<KT, 2, false>(c, p, smem, s);
            case 4: return m ? launch_lse_mma_t<KT, 4, true>(c, p, smem, s) : launch_lse_mma_t<KT, 4, false>(c, p, smem, s);
            case 8: return m ? launch_lse_mma_t<KT, 8, true>(c, p, smem, s) : launch_lse_mma_t<KT, 8, false>(c, p, smem, s);
        }
    }
    return KVM_ERR_UNSUPPORTED;
}

template <int KT, int KK, int KVH, bool MASK>
int launch_lse_q_t(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, size_t smem, cudaStream_t s) {
    auto fn = page_lse_q_kernel<KT, KK, KVH, MASK>;
    if (smem_attr(reinterpret_cast<const void*>(fn), 200 * 1024) != cudaSuccess) return KVM_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kQThreads, smem) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    if (per_sm < 1) return KVM_ERR_UNSUPPORTED;
    const uint32_t units = p.layers * p.pages;
    const uint32_t grid = std::min<uint32_t>(units, uint32_t(c->num_sms * per_sm));
    fn<<<grid, kQThreads, smem, s>>>(map, p);
    ++c->launches;
    if (cudaGetLastError() != cudaSuccess) return KVM_ERR_CUDA;
    return KVM_OK;
}

template <int KT, int KK>
int launch_lse_q_kk(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, size_t smem, cudaStream_t s) {
    const bool m = p.mask != nullptr;
    switch (p.kv_heads) {
        case 1: return m ? launch_lse_q_t<KT, KK, 1, true>(c, map, p, smem, s) : launch_lse_q_t<KT, KK, 1, false>(c, map, p, smem, s);
        case 2: return m ? launch_lse_q_t<KT, KK, 2, true>(c, map, p, smem, s) : launch_lse_q_t<KT, KK, 2, false>(c, map, p, smem, s);
        case 4: return m ? launch_lse_q_t<KT, KK, 4, true>(c, map, p, smem, s) : launch_lse_q_t<KT, KK, 4, false>(c, map, p, smem, s);
        case 8: return m ? launch_lse_q_t<KT, KK, 8, true>(c, map, p, smem, s) : launch_lse_q_t<KT, KK, 8, false>(c, map, p, smem, s);
    }
    return KVM_ERR_UNSUPPORTED;
}

// Tensor-core scorer for q8_0 / q4_0 keys (page_mass_q.cuh); kk = head_dim / 32.
template <int KT>
int launch_lse_q_kt(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, int kk, size_t smem, cudaStream_t s) {
    if constexpr (KT == KVM_Q8_0 || KT == KVM_Q4_0) {
        switch (kk) {
            case 2: return launch_lse_q_kk<KT, 2>(c, map, p, smem, s);
            case 4: return launch_lse_q_kk<KT, 4>(c, map, p, smem, s);
            case 8: return launch_lse_q_kk<KT, 8>(c, map, p, smem, s);
        }
    }
    return KVM_ERR_UNSUPPORTED;
}

// Tensor-core (tcgen05) scorer of fp16 keys, in lse_tc.cu: ka = head_dim / 64
// (1 or 2), lm = query-tile layout (1: <= 128 vectors per KV head, 2: 129..160
// with a packed second tile); `map` is the 4-D TMA tensor map of the K cache
// built by the caller.
int launch_lse_tc(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, int ka, int lm, size_t smem,
                  cudaStream_t s);

// Causal prompt attention with page-LSE capture (prefill_attn.cu): maps =
// the 3-D TMA tensor maps of K and V built by the caller; head_dim 128 or
// 256; fp16 (bf16 = false) or bf16 operands.
struct PrefillParams;
int launch_prefill(kvm_ctx* c, const CUtensorMap* maps, const PrefillParams& p, uint32_t head_dim, bool bf16,
                   cudaStream_t s);

// Instantiated once each in lse_<type>.cu.
extern template int launch_lse_kt<KVM_F32>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
extern template int launch_lse_kt<KVM_F16>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
extern template int launch_lse_kt<KVM_BF16>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
extern template int launch_lse_kt<KVM_Q8_0>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
extern template int launch_lse_kt<KVM_Q4_0>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
extern template int launch_lse_kt<KVM_Q5_0>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
extern template int launch_lse_mma_kt<KVM_F16>(kvm_ctx*, const LseParams&, int, size_t, cudaStream_t);
extern template int launch_lse_mma_kt<KVM_Q8_0>(kvm_ctx*, const LseParams&, int, size_t, cudaStream_t);
extern template int launch_lse_mma_kt<KVM_Q4_0>(kvm_ctx*, const LseParams&, int, size_t, cudaStream_t);
extern template int launch_lse_q_kt<KVM_Q8_0>(kvm_ctx*, const CUtensorMap&, const LseParams&, int, size_t,
                                              cudaStream_t);
extern template int launch_lse_q_kt<KVM_Q4_0>(kvm_ctx*, const CUtensorMap&, const LseParams&, int, size_t,
                                              cudaStream_t);

}  // namespace kvmb
