// Shared device helpers for the recall kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <utility>

#include "kvm_recall.h"

namespace kvmb {

// Raises the dynamic shared-memory limit of kernel `fn` to `bytes` on the
// current device, once per (kernel, device). The attribute belongs to the
// device, so a process that drives several GPUs sets it on each of them.
inline cudaError_t smem_attr(const void* fn, int bytes) {
    int device = -1;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    static std::mutex m;
    static std::set<std::pair<const void*, int>> done;
    std::lock_guard<std::mutex> lock(m);
    if (done.count({fn, device})) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({fn, device});
    else cudaGetLastError();
    return e;
}

// Upper bound on polls of one mbarrier / flag before a kernel gives up,
// records KVM_ERR_TIMEOUT and unwinds (a few seconds at the longest).
constexpr uint32_t kSpinLimit = 1u << 22;

// Device status word shared by all kernels of a context: the first error
// code wins; `where` names the kernel that set it.
struct DeviceStatus {
    int32_t code;
    int32_t where;
};

__device__ __forceinline__ void record_error(DeviceStatus* st, int code, int where) {
    if (atomicCAS(&st->code, 0, code) == 0) st->where = where;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// L2 policy for a stream read exactly once (the K history).
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// One bulk (non-tensor) TMA copy global -> this CTA's shared memory, completing
// `bytes` transactions on `bar`. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Tiled 4-D TMA load of one box into this CTA's shared memory (this CTA only).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float fast_log2(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Named barrier over the first `threads` threads of the CTA.
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Four signed int8 in a word -> four floats, exactly: place (b ^ 0x80) in the
// low mantissa of 2^23 and subtract 2^23 + 128.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float* f) {
    const uint32_t x = w ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440)) - 8388736.f;
    f[1] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7441)) - 8388736.f;
    f[2] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7442)) - 8388736.f;
    f[3] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7443)) - 8388736.f;
}

// Four unsigned bytes minus `bias - 2^23` -> floats, exactly (bias = 2^23 + offset).
__device__ __forceinline__ void u8x4_to_f32(uint32_t x, float bias, float* f) {
    f[0] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440)) - bias;
    f[1] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7441)) - bias;
    f[2] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7442)) - bias;
    f[3] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7443)) - bias;
}

__device__ __forceinline__ float load_scalar(const uint8_t* p, int type) {
    if (type == KVM_F32) return *reinterpret_cast<const float*>(p);
    if (type == KVM_F16) return __half2float(*reinterpret_cast<const __half*>(p));
    return __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t*>(p)) << 16);
}

__host__ __device__ __forceinline__ uint32_t type_bytes(int type) { return type == KVM_F32 ? 4u : 2u; }

__host__ __device__ __forceinline__ uint64_t row_bytes_of(int type, uint32_t dim) {
    switch (type) {
        case KVM_F32: return 4ull * dim;
        case KVM_F16:
        case KVM_BF16: return 2ull * dim;
        case KVM_Q8_0: return uint64_t(dim / 32) * 34;
        case KVM_Q4_0: return uint64_t(dim / 32) * 18;
        case KVM_Q5_0: return uint64_t(dim / 32) * 22;
    }
    return 0;
}

// Block-wide exclusive scan of one u32 per thread (blockDim a multiple of 32);
// returns the block total. Contains __syncthreads: call from every thread.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums, uint32_t* out_prefix) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) warp_sums[lane] = w;  // inclusive
    }
    __syncthreads();
    const uint32_t base = warp ? warp_sums[warp - 1] : 0;
    const uint32_t total = warp_sums[nw - 1];
    *out_prefix = base + x - v;
    __syncthreads();
    return total;
}

}  // namespace kvmb
