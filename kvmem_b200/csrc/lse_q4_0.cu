// Page log-sum-exp launchers for q4_0 keys (one translation unit per key type).
#include "lse_launch.cuh"

namespace kvmb {
template int launch_lse_kt<KVM_Q4_0>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
template int launch_lse_mma_kt<KVM_Q4_0>(kvm_ctx*, const LseParams&, int, size_t, cudaStream_t);
template int launch_lse_q_kt<KVM_Q4_0>(kvm_ctx*, const CUtensorMap&, const LseParams&, int, size_t, cudaStream_t);
}  // namespace kvmb
