// Launcher of the tcgen05 page log-sum-exp kernel (page_mass_tc.cuh):
// head_dim 64 / 128 / 256 (one, two or four 64-dim swizzle atoms), query-tile
// layout 1 / 2 (one M tile, plus a packed second tile; head_dim 256 has layout
// 1 only), with or without an additive attention mask.
#include "lse_launch.cuh"
#include "page_mass_tc.cuh"

namespace kvmb {

namespace {

template <int KA, int LM, bool MASK>
int launch_tc_t(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, size_t smem, cudaStream_t s) {
    auto fn = page_lse_tc_kernel<KA, LM, MASK>;
    if (smem_attr(reinterpret_cast<const void*>(fn), int(kTcSmemMax)) != cudaSuccess) return KVM_ERR_CUDA;
    if (smem > kTcSmemMax) return KVM_ERR_UNSUPPORTED;
    const uint64_t units = uint64_t(p.layers) * p.kv_heads * tc_units_per_head(p.pages, p.page_tokens);
    if (!units) return KVM_OK;
    const uint32_t grid = uint32_t(std::min<uint64_t>(units, uint64_t(c->num_sms)));
    fn<<<grid, tc_threads(LM), smem, s>>>(map, p);
    ++c->launches;
    if (cudaGetLastError() != cudaSuccess) return KVM_ERR_CUDA;
    return KVM_OK;
}

template <int KA, int LM>
int launch_tc_m(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, size_t smem, cudaStream_t s) {
    return p.mask ? launch_tc_t<KA, LM, true>(c, map, p, smem, s) : launch_tc_t<KA, LM, false>(c, map, p, smem, s);
}

template <int KA>
int launch_tc_l(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, int lm, size_t smem, cudaStream_t s) {
    switch (lm) {
        case 1: return launch_tc_m<KA, 1>(c, map, p, smem, s);
        case 2: return launch_tc_m<KA, 2>(c, map, p, smem, s);
    }
    return KVM_ERR_UNSUPPORTED;
}

}  // namespace

int launch_lse_tc(kvm_ctx* c, const CUtensorMap& map, const LseParams& p, int ka, int lm, size_t smem,
                  cudaStream_t s) {
    if (ka == 1) return launch_tc_l<1>(c, map, p, lm, smem, s);
    if (ka == 2) return launch_tc_l<2>(c, map, p, lm, smem, s);
    if (ka == 4 && lm == 1) return launch_tc_m<4, 1>(c, map, p, smem, s);  // head_dim 256: one M tile only
    return KVM_ERR_UNSUPPORTED;
}

}  // namespace kvmb
