// Page log-sum-exp launchers for f32 keys (one translation unit per key type).
#include "lse_launch.cuh"

namespace kvmb {
template int launch_lse_kt<KVM_F32>(kvm_ctx*, const LseParams&, int, int, size_t, cudaStream_t);
}  // namespace kvmb
