// Stage-out: device page bytes gathered into a double-buffered pair of pinned
// host slots (declarations: include/kvm_recall.h, "stage-out").
//
// The reference (src/adapter/llama-kvmem-stagein.cu:883-1004) packs the
// queued device regions into a device staging buffer with a copy kernel, then
// copies that buffer to the current pinned slot with one D2H memcpy and
// records the slot's event. Here the gather kernel writes straight into the
// mapped pinned slot over PCIe / C2C (16-byte stores of whole 128-byte lines
// per warp), so there is no device staging buffer and no second copy. The two
// slots alternate exactly as the reference's `out_cur`, so the host can write
// one batch into the store while the GPU fills the other.
#include <algorithm>
#include <chrono>
#include <new>
#include <vector>

#include "common.cuh"

namespace {

constexpr uint32_t kOutThreads = 256;
constexpr uint32_t kOutUnroll = 8;
constexpr uint64_t kOutChunk = 64 * 1024;  // bytes of one work unit
constexpr uint32_t kOutDefaultCtas = 32;

struct OutOp {
    const uint8_t* src;  // device
    uint8_t* dst;        // mapped pinned host (device view)
    uint64_t bytes;
    uint64_t first_chunk;  // index of this op's first kOutChunk unit
};

// Unit u = (op, chunk): CTAs take units round-robin; each CTA's units rise, so
// its op cursor only moves forward.
__global__ void __launch_bounds__(kOutThreads) stageout_gather_kernel(const OutOp* __restrict__ ops, uint32_t n,
                                                                      uint64_t units) {
    uint32_t op = 0;
    for (uint64_t u = blockIdx.x; u < units; u += gridDim.x) {
        while (op + 1 < n && ops[op + 1].first_chunk <= u) ++op;
        const OutOp o = ops[op];
        const uint64_t off = (u - o.first_chunk) * kOutChunk;
        if (off >= o.bytes) continue;
        const uint64_t len = min(kOutChunk, o.bytes - off);
        const uint8_t* src = o.src + off;
        uint8_t* dst = o.dst + off;
        if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0) {
            const uint4* s4 = reinterpret_cast<const uint4*>(src);
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            const uint64_t n4 = len >> 4;
            uint64_t i = threadIdx.x;
            for (; i + uint64_t(kOutUnroll - 1) * kOutThreads < n4; i += uint64_t(kOutThreads) * kOutUnroll) {
                uint4 v[kOutUnroll];
#pragma unroll
                for (uint32_t k = 0; k < kOutUnroll; ++k) v[k] = __ldcs(s4 + i + uint64_t(k) * kOutThreads);
#pragma unroll
                for (uint32_t k = 0; k < kOutUnroll; ++k) d4[i + uint64_t(k) * kOutThreads] = v[k];
            }
            for (; i < n4; i += kOutThreads) d4[i] = __ldcs(s4 + i);
            for (uint64_t b = (n4 << 4) + threadIdx.x; b < len; b += kOutThreads) dst[b] = src[b];
        } else {
            for (uint64_t b = threadIdx.x; b < len; b += kOutThreads) dst[b] = src[b];
        }
    }
}

struct DeviceGuard {
    int previous = -1;
    bool ok = false;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&previous) != cudaSuccess) return;
        ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (previous >= 0) cudaSetDevice(previous);
    }
};

int bounded_event_wait(cudaEvent_t e, uint64_t timeout_us) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t r = cudaEventQuery(e);
        if (r == cudaSuccess) return KVM_OK;
        if (r != cudaErrorNotReady) {
            cudaGetLastError();
            return KVM_ERR_CUDA;
        }
        const auto us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (uint64_t(us) >= timeout_us) return KVM_ERR_TIMEOUT;
    }
}

}  // namespace

struct kvm_stageout {
    int device = 0;
    uint64_t slot_bytes = 0;
    uint32_t max_items = 0;
    uint8_t* slot[2] = {nullptr, nullptr};      // pinned, mapped
    OutOp* host_ops[2] = {nullptr, nullptr};    // pinned: the op list of each slot's last submit
    OutOp* dev_ops[2] = {nullptr, nullptr};     // device copies of those lists
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool pending[2] = {false, false};           // submitted, event not yet observed
    int cur = 0;                                // slot the next submit fills
    uint64_t used = 0;
    std::vector<OutOp> queued;
};

namespace {

void release(kvm_stageout* s) {
    for (int i = 0; i < 2; ++i) {
        if (s->done[i]) cudaEventSynchronize(s->done[i]);
        if (s->done[i]) cudaEventDestroy(s->done[i]);
        if (s->slot[i]) cudaFreeHost(s->slot[i]);
        if (s->host_ops[i]) cudaFreeHost(s->host_ops[i]);
        if (s->dev_ops[i]) cudaFree(s->dev_ops[i]);
    }
    cudaGetLastError();
    delete s;
}

}  // namespace

extern "C" {

int kvm_stageout_create(int device, uint64_t slot_bytes, uint32_t max_items, kvm_stageout** out) {
    if (!out) return KVM_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (slot_bytes == 0 || max_items == 0 || slot_bytes % 16) return KVM_ERR_INVALID_ARGUMENT;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    if (device < 0 || device >= count) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(device);
    if (!guard.ok) return KVM_ERR_CUDA;
    auto* s = new (std::nothrow) kvm_stageout;
    if (!s) return KVM_ERR_CUDA;
    s->device = device;
    s->slot_bytes = slot_bytes;
    s->max_items = max_items;
    for (int i = 0; i < 2; ++i) {
        if (cudaHostAlloc(reinterpret_cast<void**>(&s->slot[i]), slot_bytes,
                          cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
            cudaHostAlloc(reinterpret_cast<void**>(&s->host_ops[i]), size_t(max_items) * sizeof(OutOp),
                          cudaHostAllocDefault) != cudaSuccess ||
            cudaMalloc(&s->dev_ops[i], size_t(max_items) * sizeof(OutOp)) != cudaSuccess ||
            cudaEventCreateWithFlags(&s->done[i], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            release(s);
            return KVM_ERR_CUDA;
        }
    }
    s->queued.reserve(max_items);
    *out = s;
    return KVM_OK;
}

int kvm_stageout_destroy(kvm_stageout* s) {
    if (!s) return KVM_OK;
    DeviceGuard guard(s->device);
    release(s);
    return KVM_OK;
}

int kvm_stageout_enqueue(kvm_stageout* s, const void* dev_src, uint64_t nbytes, uint64_t* offset) {
    if (!s || !dev_src || nbytes == 0) return KVM_ERR_INVALID_ARGUMENT;
    if (nbytes > s->slot_bytes || s->queued.size() >= s->max_items || s->used + nbytes > s->slot_bytes)
        return KVM_ERR_LENGTH;
    OutOp o{};
    o.src = static_cast<const uint8_t*>(dev_src);
    o.dst = reinterpret_cast<uint8_t*>(s->used);  // slot offset until submit
    o.bytes = nbytes;
    s->queued.push_back(o);
    if (offset) *offset = s->used;
    s->used = std::min(s->slot_bytes, (s->used + nbytes + 15) / 16 * 16);
    return KVM_OK;
}

uint64_t kvm_stageout_used(const kvm_stageout* s) { return s ? s->used : 0; }

int kvm_stageout_submit(kvm_stageout* s, uint32_t ctas, void* stream, int* slot_out) {
    if (!s || !slot_out) return KVM_ERR_INVALID_ARGUMENT;
    *slot_out = -1;
    if (s->queued.empty()) return KVM_OK;
    DeviceGuard guard(s->device);
    if (!guard.ok) return KVM_ERR_CUDA;
    const int slot = s->cur;
    // The slot's previous gather may still read its op list; the host owns the
    // slot's bytes again once that gather is done.
    if (s->pending[slot]) {
        const int rc = bounded_event_wait(s->done[slot], 30ull * 1000 * 1000);
        if (rc != KVM_OK) return rc;
        s->pending[slot] = false;
    }
    uint8_t* base = nullptr;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&base), s->slot[slot], 0) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    const uint32_t n = uint32_t(s->queued.size());
    uint64_t units = 0;
    for (uint32_t i = 0; i < n; ++i) {
        OutOp o = s->queued[i];
        o.dst = base + reinterpret_cast<uintptr_t>(o.dst);
        o.first_chunk = units;
        units += (o.bytes + kOutChunk - 1) / kOutChunk;
        s->host_ops[slot][i] = o;
    }
    auto st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(s->dev_ops[slot], s->host_ops[slot], size_t(n) * sizeof(OutOp), cudaMemcpyHostToDevice,
                        st) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    const uint64_t grid = std::min<uint64_t>(units, ctas ? ctas : kOutDefaultCtas);
    stageout_gather_kernel<<<unsigned(grid), kOutThreads, 0, st>>>(s->dev_ops[slot], n, units);
    if (cudaGetLastError() != cudaSuccess || cudaEventRecord(s->done[slot], st) != cudaSuccess) {
        cudaGetLastError();
        return KVM_ERR_CUDA;
    }
    s->pending[slot] = true;
    s->queued.clear();
    s->used = 0;
    s->cur = 1 - slot;
    *slot_out = slot;
    return KVM_OK;
}

int kvm_stageout_wait(kvm_stageout* s, int slot, uint64_t timeout_us) {
    if (!s) return KVM_ERR_INVALID_ARGUMENT;
    if (slot < 0) return KVM_OK;
    if (slot > 1) return KVM_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(s->device);
    if (!guard.ok) return KVM_ERR_CUDA;
    const int rc = bounded_event_wait(s->done[slot], timeout_us);
    if (rc == KVM_OK) s->pending[slot] = false;
    return rc;
}

const uint8_t* kvm_stageout_slot_base(const kvm_stageout* s, int slot) {
    if (!s || slot < 0 || slot > 1) return nullptr;
    return s->slot[slot];
}

int kvm_stageout_clear(kvm_stageout* s) {
    if (!s) return KVM_ERR_INVALID_ARGUMENT;
    s->queued.clear();
    s->used = 0;
    return KVM_OK;
}

}  // extern "C"
