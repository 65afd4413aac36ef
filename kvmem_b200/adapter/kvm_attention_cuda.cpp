// llama_kvmem_attention_cuda over the B200 recall library.
//
// Implements the reference's class (src/adapter/llama-kvmem-attention-cuda.h:9-18)
// with the body of its score() (src/adapter/llama-kvmem-attention-cuda.cu:146-193)
// replaced by one kvm_score_pages call over every sampled row (kvm_query.row_ids):
// the K history is read once for the whole batch, where the reference's page_lse
// kernel reads it once per query head. The argument meaning and error behaviour are
// the reference's: false for inputs outside what the kernel handles (the caller then
// builds its ggml graph), std::runtime_error on a CUDA failure or a device change.
// A KVMem build compiles this file instead of llama-kvmem-attention-cuda.cu and links
// libkvm_b200.so.
#include "llama-kvmem-attention-cuda.h"

#include "ggml-backend.h"
#include "kvm_recall.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>

namespace {

int kvm_type_of(ggml_type t) {
    switch (t) {
        case GGML_TYPE_F32: return KVM_F32;
        case GGML_TYPE_F16: return KVM_F16;
        case GGML_TYPE_BF16: return KVM_BF16;
        case GGML_TYPE_Q8_0: return KVM_Q8_0;
        case GGML_TYPE_Q4_0: return KVM_Q4_0;
        case GGML_TYPE_Q5_0: return KVM_Q5_0;
        default: return -1;
    }
}

// As the reference's device_pointer (cu:123-128): device or managed memory, and its device.
bool device_pointer(const void* data, int& device) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, data) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) return false;
    device = attr.device;
    return true;
}

// End of the device allocation that holds `p` (0 when it cannot be found): the
// scorer reads whole pages, so a K view whose last page is partial is scored only
// when that page still lies inside the allocation (tokens past ne[1] are hidden).
uintptr_t allocation_end(const void* p) {
    using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return RangeFn(nullptr);
        }
        return reinterpret_cast<RangeFn>(f);
    }();
    CUdeviceptr base = 0;
    size_t size = 0;
    if (!fn || fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return 0;
    return uintptr_t(base) + size;
}

void checked(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("KVMem attention CUDA: ") + what + ": " +
                                                   cudaGetErrorString(e));
}

struct DeviceGuard {
    int previous = -1;
    explicit DeviceGuard(int device) {
        checked(cudaGetDevice(&previous), "cudaGetDevice");
        checked(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceGuard() { cudaSetDevice(previous); }
};

}  // namespace

struct llama_kvmem_attention_cuda::Impl {
    int device = -1;
    kvm_ctx* ctx = nullptr;
    cudaStream_t stream = nullptr;
    void* mask = nullptr;  // device copy of a host mask's sampled rows
    size_t mask_bytes = 0;
    void* out = nullptr;  // device [rows][pages]
    size_t out_bytes = 0;
    ~Impl() {
        if (device < 0) return;
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (mask) cudaFree(mask);
        if (out) cudaFree(out);
        if (stream) cudaStreamDestroy(stream);
        kvm_ctx_destroy(ctx);
    }
    void reserve(void** p, size_t* have, size_t bytes) {
        if (bytes <= *have) return;
        if (*p) checked(cudaFree(*p), "cudaFree");
        *p = nullptr;
        *have = 0;
        checked(cudaMalloc(p, bytes), "cudaMalloc");
        *have = bytes;
    }
};

llama_kvmem_attention_cuda::llama_kvmem_attention_cuda() : impl(std::make_unique<Impl>()) {}
llama_kvmem_attention_cuda::~llama_kvmem_attention_cuda() = default;

bool llama_kvmem_attention_cuda::score(ggml_tensor* q, ggml_tensor* k, ggml_tensor* mask, float scale,
                                       float softcap, uint32_t block, const std::vector<uint32_t>& rows,
                                       std::vector<std::vector<float>>& output) {
    const int qt = kvm_type_of(q->type), kt = kvm_type_of(k->type), mt = kvm_type_of(mask->type);
    // The reference's domain (cu:150-151): f32/f16/bf16 Q and mask, head_dim <= 256 and a multiple of 32.
    if (qt < 0 || qt > KVM_BF16 || kt < 0 || mt < 0 || mt > KVM_BF16 || q->ne[0] > 256 || q->ne[0] % 32) return false;
    if (mt == KVM_BF16) return false;  // the library takes f32 / f16 masks
    int device = -1, key_device = -1, mask_device = -1;
    if (!device_pointer(q->data, device) || !device_pointer(k->data, key_device) || device != key_device) return false;
    if (rows.size() > 512) return false;  // one call scores at most 512 sampled rows
    DeviceGuard guard(device);
    if (impl->device < 0) {
        if (kvm_ctx_create(device, &impl->ctx) != KVM_OK) throw std::runtime_error("KVMem attention CUDA: context");
        impl->device = device;
        checked(cudaStreamCreateWithFlags(&impl->stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
    }
    if (impl->device != device) throw std::runtime_error("KVMem attention workspace changed device");
    const uint64_t tokens = uint64_t(k->ne[1]);
    const uint32_t pages = uint32_t((tokens + block - 1) / block);
    output.assign(rows.size(), std::vector<float>(pages));
    if (rows.empty()) return true;
    // A mask that is not device memory of this device: its sampled rows are staged first (cu:159,172-178).
    const size_t mask_row = size_t(tokens) * (mt == KVM_F32 ? 4 : 2);
    const bool staged = !device_pointer(mask->data, mask_device) || mask_device != device;
    const void* mask_data = mask->data;
    uint64_t mask_stride = mask->nb[1];
    if (staged) {
        std::vector<uint8_t> host(rows.size() * mask_row);
        for (size_t i = 0; i < rows.size(); ++i)
            ggml_backend_tensor_get(mask, host.data() + i * mask_row, size_t(rows[i]) * mask->nb[1], mask_row);
        impl->reserve(&impl->mask, &impl->mask_bytes, host.size());
        checked(cudaMemcpyAsync(impl->mask, host.data(), host.size(), cudaMemcpyHostToDevice, impl->stream),
                "mask upload");
        mask_data = impl->mask;
        mask_stride = mask_row;
    }
    kvm_kcache kc{};
    kc.data = k->data;
    kc.type = kt;
    kc.layer_stride = 0;
    kc.token_stride = k->nb[1];
    kc.head_stride = k->nb[2];
    kc.capacity_tokens = tokens;
    if (tokens % block) {
        const uint64_t whole = uint64_t(pages) * block;
        const uintptr_t need = reinterpret_cast<uintptr_t>(k->data) + (whole - 1) * k->nb[1] +
                               uint64_t(k->ne[2]) * k->nb[2];
        if (need <= allocation_end(k->data)) kc.capacity_tokens = whole;  // else: scored only if aligned
    }
    kvm_score_desc d{};
    d.layers = 1;
    d.q_heads = uint32_t(q->ne[2]);
    d.kv_heads = uint32_t(k->ne[2]);
    d.head_dim = uint32_t(q->ne[0]);
    d.tokens = tokens;
    d.page_tokens = block;
    d.groups = 1;
    d.scale = scale;
    d.softcap = softcap;
    d.mask = mask_data;
    d.mask_type = mt;
    d.mask_row_stride = mask_stride;
    // Query row rows[i] and mask row rows[i] are scored as output row i (kvm_query.row_ids).
    kvm_query qq{};
    qq.data = q->data;
    qq.type = qt;
    qq.layer_stride = 0;
    qq.row_stride = q->nb[1];
    qq.head_stride = q->nb[2];
    qq.rows = uint32_t(rows.size());
    qq.row_ids = rows.data();
    qq.row_count = uint32_t(q->ne[1]);
    impl->reserve(&impl->out, &impl->out_bytes, rows.size() * size_t(pages) * sizeof(float));
    if (staged) {
        // The staged mask holds the sampled rows in list order, not at their row ids: one call
        // per sampled row, each with its own staged mask row (the uncommon host-mask case).
        for (size_t i = 0; i < rows.size(); ++i) {
            kvm_query one = qq;
            one.data = static_cast<const uint8_t*>(q->data) + size_t(rows[i]) * q->nb[1];
            one.rows = 1;
            one.row_ids = nullptr;
            d.mask = static_cast<const uint8_t*>(impl->mask) + i * mask_row;
            const int rc = kvm_score_pages(impl->ctx, &d, &one, &kc,
                                           static_cast<float*>(impl->out) + i * pages, nullptr, impl->stream);
            if (rc == KVM_ERR_UNSUPPORTED) return false;
            if (rc != KVM_OK) throw std::runtime_error("KVMem attention CUDA: kvm_score_pages " + std::to_string(rc));
        }
    } else {
        const int rc = kvm_score_pages(impl->ctx, &d, &qq, &kc, static_cast<float*>(impl->out), nullptr,
                                       impl->stream);
        if (rc == KVM_ERR_UNSUPPORTED) return false;  // e.g. head_dim 96 or non-dense K strides
        if (rc != KVM_OK) throw std::runtime_error("KVMem attention CUDA: kvm_score_pages " + std::to_string(rc));
    }
    std::vector<float> host(rows.size() * size_t(pages));
    checked(cudaMemcpyAsync(host.data(), impl->out, host.size() * sizeof(float), cudaMemcpyDeviceToHost,
                            impl->stream),
            "result download");
    const int st = kvm_ctx_status(impl->ctx, impl->stream);  // synchronises the stream
    if (st != KVM_OK) throw std::runtime_error("KVMem attention CUDA: device status " + std::to_string(st));
    for (size_t i = 0; i < rows.size(); ++i) std::memcpy(output[i].data(), host.data() + i * pages, pages * 4);
    return true;
}
