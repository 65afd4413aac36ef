// Sampled query rows. The reference scores a list of rows of its captured
// query batch (llama_kvmem_attention_cuda::score's `rows`,
// src/adapter/llama-kvmem-attention-cuda.cu:146-190, whose page_lse kernel
// reads query row rows[i] and mask row rows[i] at :66-67). Here the listed
// rows, and their mask rows, are first packed densely into the workspace, so
// every scorer sees rows 0 .. n-1 and one pass over K serves all of them.
#pragma once
#include "common.cuh"

namespace kvmb {

constexpr uint32_t kMaxRowIds = 512;

// The row list travels as a kernel parameter (2 KiB): no upload, no sync.
struct RowIds {
    uint32_t n;
    uint32_t id[kMaxRowIds];
};

// dst[(l*n + i)*heads + h] (head_bytes each) <- q + l*q_layer + id[i]*q_row + h*q_head.
// head_bytes even, source addresses 2-byte aligned (checked by the host).
__global__ void __launch_bounds__(128) pack_query_rows_kernel(const uint8_t* __restrict__ q, uint64_t q_layer,
                                                              uint64_t q_row, uint64_t q_head, uint32_t heads,
                                                              uint32_t head_bytes, uint32_t layers, RowIds ids,
                                                              uint8_t* __restrict__ dst) {
    const uint64_t chunks = uint64_t(layers) * ids.n * heads;
    for (uint64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
        const uint32_t h = uint32_t(c % heads);
        const uint64_t li = c / heads;
        const uint32_t i = uint32_t(li % ids.n), l = uint32_t(li / ids.n);
        const uint8_t* src = q + l * q_layer + uint64_t(ids.id[i]) * q_row + uint64_t(h) * q_head;
        uint8_t* d = dst + c * head_bytes;
        for (uint32_t b = threadIdx.x * 2; b < head_bytes; b += blockDim.x * 2)
            *reinterpret_cast<uint16_t*>(d + b) = *reinterpret_cast<const uint16_t*>(src + b);
    }
}

// dst[i][0 .. row_bytes) <- mask + id[i]*mask_row (row_bytes = tokens * element size, even).
__global__ void __launch_bounds__(256) pack_mask_rows_kernel(const uint8_t* __restrict__ mask, uint64_t mask_row,
                                                             uint32_t row_bytes, RowIds ids,
                                                             uint8_t* __restrict__ dst) {
    const uint32_t i = blockIdx.y;
    const uint8_t* src = mask + uint64_t(ids.id[i]) * mask_row;
    uint8_t* d = dst + uint64_t(i) * row_bytes;
    for (uint32_t b = (blockIdx.x * blockDim.x + threadIdx.x) * 2; b < row_bytes; b += gridDim.x * blockDim.x * 2)
        *reinterpret_cast<uint16_t*>(d + b) = *reinterpret_cast<const uint16_t*>(src + b);
}

}  // namespace kvmb
