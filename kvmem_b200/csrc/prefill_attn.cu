// Launcher of the causal prompt-attention kernel with page-LSE capture
// (prefill_attn.cuh) and, for a split key range, its merge pass: head_dim 128 /
// 256, fp16 or bf16 operands.
#include "lse_launch.cuh"
#include "prefill_attn.cuh"

namespace kvmb {

namespace {

template <int KA, bool BF16>
int launch_pf_t(kvm_ctx* c, const CUtensorMap* maps, const PrefillParams& p, cudaStream_t s) {
    auto fn = prefill_attn_kernel<KA, BF16>;
    const size_t smem = pf_smem_bytes(KA);
    if (smem_attr(reinterpret_cast<const void*>(fn), int(smem)) != cudaSuccess) return KVM_ERR_CUDA;
    const uint64_t grid = uint64_t(p.q_tiles) * p.q_heads * p.splits;
    if (!grid) return KVM_OK;
    if (grid > 0x7fffffffull) return KVM_ERR_LENGTH;
    fn<<<uint32_t(grid), kPfThreads, smem, s>>>(maps[0], maps[1], p);
    ++c->launches;
    if (cudaGetLastError() != cudaSuccess) return KVM_ERR_CUDA;
    if (p.splits > 1) {
        const uint64_t threads = uint64_t(p.width) * p.q_heads * 32;
        prefill_combine_kernel<KA * 64, BF16><<<uint32_t((threads + 255) / 256), 256, 0, s>>>(p);
        ++c->launches;
        if (cudaGetLastError() != cudaSuccess) return KVM_ERR_CUDA;
    }
    return KVM_OK;
}

}  // namespace

int launch_prefill(kvm_ctx* c, const CUtensorMap* maps, const PrefillParams& p, uint32_t head_dim, bool bf16,
                   cudaStream_t s) {
    if (head_dim == 128) return bf16 ? launch_pf_t<2, true>(c, maps, p, s) : launch_pf_t<2, false>(c, maps, p, s);
    if (head_dim == 256) return bf16 ? launch_pf_t<4, true>(c, maps, p, s) : launch_pf_t<4, false>(c, maps, p, s);
    return KVM_ERR_UNSUPPORTED;
}

}  // namespace kvmb
