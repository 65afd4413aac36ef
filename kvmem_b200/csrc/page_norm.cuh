// Per-token page mass, second pass: softmax over pages and head / row means.
#pragma once
#include "page_mass.cuh"

namespace kvmb {

// Per (layer, group): softmax statistics of every (row, head) over all pages,
// then mass_rows = mean over the group's heads, mass_mean = mean over rows.
// Mirrors the reference's normalize + average
// (src/adapter/llama-kvmem-attention-cuda.cu:98-121): max, 1/sum(exp(lse-max)),
// then sum_h exp(lse-max)*inv / heads. A (row, head) whose pages are all
// empty has max = -inf and yields NaN, as the reference's normaliser does.
// With `given` (sharded scoring) the statistics are not computed but read:
// given[(l*rows + r)*q_heads + h] = (global max, 1/global sum).
__global__ void __launch_bounds__(256) page_mass_normalize_kernel(const float* lse, uint32_t rows, uint32_t q_heads,
                                                                  uint32_t group, uint32_t groups, uint32_t pages,
                                                                  float* mass_rows, float* mass_mean,
                                                                  uint32_t out_layer0, const float2* given) {
    extern __shared__ float2 stats[];  // [rows * heads_per]
    const uint32_t l = blockIdx.x / groups, g = blockIdx.x % groups;
    const uint32_t heads_per = groups == 1 ? q_heads : group;
    const uint32_t h0 = groups == 1 ? 0 : g * group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nrow = rows * heads_per;
    for (uint32_t idx = warp; idx < nrow; idx += 8) {
        const uint32_t r = idx / heads_per, h = h0 + idx % heads_per;
        if (given) {
            if (lane == 0) stats[idx] = given[(uint64_t(l) * rows + r) * q_heads + h];
            continue;
        }
        const float* row = lse + ((uint64_t(l) * rows + r) * q_heads + h) * pages;
        float M = -INFINITY;
        for (uint32_t p = lane; p < pages; p += 32) M = fmaxf(M, row[p]);
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float S = 0.f;
        for (uint32_t p = lane; p < pages; p += 32) S += fast_exp2((row[p] - M) * kLog2e);
#pragma unroll
        for (int o = 16; o; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
        if (lane == 0) stats[idx] = make_float2(M, 1.f / S);
    }
    __syncthreads();
    const float inv_heads = 1.f / float(heads_per), inv_rows = 1.f / float(rows);
    const uint64_t orow = uint64_t(out_layer0 + l) * groups + g;
    for (uint32_t p = threadIdx.x; p < pages; p += blockDim.x) {
        float mean = 0.f;
        for (uint32_t r = 0; r < rows; ++r) {
            float v = 0.f;
            for (uint32_t hh = 0; hh < heads_per; ++hh) {
                const float2 st = stats[r * heads_per + hh];
                const float x = lse[((uint64_t(l) * rows + r) * q_heads + h0 + hh) * pages + p];
                v += fast_exp2((x - st.x) * kLog2e) * st.y;
            }
            v *= inv_heads;
            if (mass_rows) mass_rows[(orow * rows + r) * pages + p] = v;
            mean += v;
        }
        if (mass_mean) mass_mean[orow * pages + p] = mean * inv_rows;
    }
}

}  // namespace kvmb
