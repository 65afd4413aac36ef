// Layerwise tile accumulation on the device.
//
// The reference's layerwise (current-layer Query) recall scores the query rows
// of a prefill in tiles against one frozen page frame and sums the tiles' page
// masses (no mean over rows); when the Mean-K records are half pages, each
// tile is scored over the half-page frame and either collapsed (left + right)
// or kept as halves until the end, where each page takes the larger half
// (kvmem/src/host/layerwise_selection.cpp: layerwise_tile_scores :32-75,
// LayerwiseQuerySelection::accumulate :283-296, finish :298-309,
// layerwise_max_page_scores :24-30). Here the tile masses stay on the device,
// the accumulator is FP64 as the reference's, and every check the reference
// makes before it adds a tile is made before anything is added.
#pragma once
#include "common.cuh"

namespace kvmb {

constexpr int kLayerwiseThreads = 1024;

// accum[s] += the tile's value of slot s, for every slot, or nothing when any
// value fails the reference's checks:
//   halves = 2: left = tile[2i], right = tile[2i+1] must be >= 0 with a finite
//     sum, and a page outside the score mask must sum to 0
//     (layerwise_tile_scores :61-63; else KVM_ERR_INVALID_ARGUMENT);
//     keep_halves keeps (left, right), otherwise the slot is left + right;
//   every slot value must be finite, >= 0, keep accum finite, and be 0 on a page
//   outside the score mask (accumulate :288-293; else KVM_ERR_INVALID_PLAN).
__global__ void __launch_bounds__(kLayerwiseThreads) layerwise_accumulate_kernel(const float* __restrict__ tile,
                                                                                 uint32_t pages, uint32_t halves,
                                                                                 int keep_halves,
                                                                                 const uint8_t* __restrict__ mask,
                                                                                 double* __restrict__ accum,
                                                                                 DeviceStatus* status) {
    __shared__ int bad_half, bad_slot;
    if (threadIdx.x == 0) bad_half = bad_slot = 0;
    __syncthreads();
    const uint32_t per = keep_halves ? 2u : 1u;
    for (int pass = 0; pass < 2; ++pass) {
        for (uint32_t i = threadIdx.x; i < pages; i += blockDim.x) {
            double v[2];
            if (halves == 2) {
                const double left = tile[2 * i], right = tile[2 * i + 1], sum = left + right;
                if (pass == 0 && (left < 0 || right < 0 || !isfinite(sum) || (!mask[i] && sum != 0)))
                    atomicOr(&bad_half, 1);
                v[0] = keep_halves ? left : sum;
                v[1] = right;
            } else {
                v[0] = tile[i];
                v[1] = 0;
            }
            for (uint32_t j = 0; j < per; ++j) {
                const uint64_t s = uint64_t(i) * per + j;
                if (pass == 0) {
                    if (!isfinite(v[j]) || v[j] < 0 || !isfinite(accum[s] + v[j]) || (!mask[i] && v[j] != 0))
                        atomicOr(&bad_slot, 1);
                } else {
                    accum[s] += v[j];
                }
            }
        }
        __syncthreads();
        if (bad_half || bad_slot) {
            if (threadIdx.x == 0) record_error(status, bad_half ? KVM_ERR_INVALID_ARGUMENT : KVM_ERR_INVALID_PLAN, 40);
            return;
        }
    }
}

// scores[i] = keep_halves ? max(accum[2i], accum[2i+1]) : accum[i], as f32 for the picker.
__global__ void layerwise_finish_kernel(const double* __restrict__ accum, uint32_t pages, int keep_halves,
                                        float* __restrict__ scores) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < pages; i += gridDim.x * blockDim.x)
        scores[i] = float(keep_halves ? fmax(accum[2 * i], accum[2 * i + 1]) : accum[i]);
}

}  // namespace kvmb
