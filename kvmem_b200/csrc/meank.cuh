// Mean-K page softmax over device-resident per-page K sums.
//
// Same formula as PageSoftmaxCuda::score (kvmem/src/cuda/page_softmax.cu:58-133,
// 202-280) and its FP64 reference page_softmax_scores
// (kvmem/src/host/graph_recall.cpp:322-394), without the host mean loop and the
// per-call upload: the per-page K sums live in HBM, the mean is formed on the
// device as sum * (1/count) in f32 (raw_kv_store.cpp:606-614), and both
// operands cross the explicit FP16 boundary (recall_fp16,
// graph_recall.cpp:295-320: round-to-nearest-even, rejecting non-finite values
// and values that round to infinity).
//
// Kernels: pack (means + queries -> fp16, operand flag), logits (one warp per
// (page, distribution row), lane-strided fp32 dot), normalize (warp per row:
// max, 1/sum), Max-aggregation group mass (per (layer, row, KV group) the page
// mass of the per-page max probability) and accumulate (per page, the sum of
// every distribution row's contribution).
#pragma once
#include "common.cuh"

namespace kvmb {

__device__ __forceinline__ __half recall_half(float x, uint32_t* bad) {
    const __half h = __float2half_rn(x);
    if (!isfinite(x) || __hisinf(h)) atomicExch(bad, 1u);
    return h;
}

// means_h[slot][j][kw] = fp16(sums[layer[slot]][enabled[j]][kw] * (1/counts[enabled[j]]))
// for the active layers only (an absent layer's statistics are never read,
// graph_recall.cpp:354).
__global__ void meank_pack_means_kernel(const float* sums, const uint32_t* counts, const uint32_t* enabled,
                                        const uint32_t* active_layers, uint32_t nactive, uint32_t pages, uint32_t n,
                                        uint32_t kw, __half* means_h, uint32_t* bad) {
    const uint64_t total = uint64_t(nactive) * n * kw;
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total; i += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t d = i % kw, j = (i / kw) % n, slot = i / (uint64_t(kw) * n);
        const uint32_t p = enabled[j];
        const float inv = 1.0f / float(counts[p]);
        means_h[i] = recall_half(sums[(uint64_t(active_layers[slot]) * pages + p) * kw + d] * inv, bad);
    }
}

// qh[i][Hq*D] = fp16(q[layer][row][Hq*D]) for every present (layer, row) pair i;
// pair_lr holds the pairs as consecutive u32 (layer, row).
__global__ void meank_pack_query_kernel(const float* q, const uint32_t* pair_lr, uint32_t npairs, uint32_t rows,
                                        uint32_t qw, __half* qh, uint32_t* bad) {
    const uint64_t total = uint64_t(npairs) * qw;
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total; i += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t e = i % qw, pi = i / qw;
        const uint32_t l = pair_lr[2 * pi], r = pair_lr[2 * pi + 1];
        qh[i] = recall_half(q[(uint64_t(l) * rows + r) * qw + e], bad);
    }
}

// logits[dist][j], dist = pair*Hq + h.
__global__ void meank_logits_kernel(const __half* qh, const __half* means_h, const uint32_t* pair_slot,
                                    uint32_t heads, uint32_t kv_heads, uint32_t dim, uint32_t n, float scale,
                                    float* logits) {
    const uint32_t dist = blockIdx.y;
    const uint32_t j = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (j >= n) return;
    const uint32_t h = dist % heads, pair = dist / heads;
    const uint32_t slot = pair_slot[pair];
    const uint32_t kvh = h / (heads / kv_heads);
    const __half* qv = qh + uint64_t(dist) * dim;
    const __half* kv = means_h + (uint64_t(slot) * n + j) * (uint64_t(kv_heads) * dim) + uint64_t(kvh) * dim;
    float dot = 0.f;
    for (uint32_t d = lane; d < dim; d += 32) dot = fmaf(__half2float(qv[d]), __half2float(kv[d]), dot);
#pragma unroll
    for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) logits[uint64_t(dist) * n + j] = dot * scale;
}

// norms[dist] = (max, 1/sum exp(logit - max)), one warp per distribution row.
__global__ void meank_normalize_kernel(const float* logits, uint32_t n, uint32_t dists, float2* norms) {
    const uint32_t dist = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (dist >= dists) return;
    const float* row = logits + uint64_t(dist) * n;
    float M = -INFINITY;
    for (uint32_t j = lane; j < n; j += 32) M = fmaxf(M, row[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float S = 0.f;
    for (uint32_t j = lane; j < n; j += 32) S += expf(row[j] - M);
#pragma unroll
    for (int o = 16; o; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (lane == 0) norms[dist] = make_float2(M, 1.f / S);
}

// Max aggregation: per (pair, KV group) the inverse page mass of the per-page
// max probability over the group's heads (page_softmax.cu:100-122).
__global__ void meank_group_mass_kernel(const float* logits, const float2* norms, uint32_t n, uint32_t group,
                                        uint32_t groups_total, float* group_inv_mass) {
    const uint32_t gid = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gid >= groups_total) return;
    const uint32_t base = gid * group;  // first distribution row of the group
    float sum = 0.f;
    for (uint32_t j = lane; j < n; j += 32) {
        float mx = 0.f;
        for (uint32_t h = 0; h < group; ++h) {
            const float2 st = norms[base + h];
            mx = fmaxf(mx, expf(logits[uint64_t(base + h) * n + j] - st.x) * st.y);
        }
        sum += mx;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) group_inv_mass[gid] = 1.f / sum;
}

// out[enabled[j]] = weight * sum over distribution rows of the row's contribution.
__global__ void meank_accumulate_kernel(const float* logits, const float2* norms, const float* group_inv_mass,
                                        const uint32_t* enabled, uint32_t n, uint32_t dists, uint32_t group, int max_agg,
                                        float weight, float* out) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float acc = 0.f;
    if (!max_agg) {
        for (uint32_t d = 0; d < dists; ++d) {
            const float2 st = norms[d];
            acc += expf(logits[uint64_t(d) * n + j] - st.x) * st.y;
        }
    } else {
        for (uint32_t g = 0; g * group < dists; ++g) {
            float mx = 0.f;
            for (uint32_t h = 0; h < group; ++h) {
                const uint32_t d = g * group + h;
                const float2 st = norms[d];
                mx = fmaxf(mx, expf(logits[uint64_t(d) * n + j] - st.x) * st.y);
            }
            acc += mx * group_inv_mass[g];
        }
    }
    out[enabled[j]] = acc * weight;
}

// Element d of one K row (head slice) as float, as the reference's key()
// (src/adapter/llama-kvmem-attention-cuda.cu:39-58): f32 / f16 / bf16 values,
// GGUF q8_0 / q4_0 / q5_0 codes times the block's fp16 scale as one rounded
// f32 product (__fmul_rn: never contracted into the caller's add).
template <int KT>
__device__ __forceinline__ float key_elem(const uint8_t* row, uint32_t d) {
    const uint32_t at = d % 32;
    if constexpr (KT == KVM_F32) return reinterpret_cast<const float*>(row)[d];
    if constexpr (KT == KVM_F16) return __half2float(reinterpret_cast<const __half*>(row)[d]);
    if constexpr (KT == KVM_BF16) return __uint_as_float(uint32_t(reinterpret_cast<const uint16_t*>(row)[d]) << 16);
    if constexpr (KT == KVM_Q8_0) {
        const uint8_t* b = row + (d / 32) * 34u;
        return __fmul_rn(float(int8_t(b[2 + at])), __half2float(*reinterpret_cast<const __half*>(b)));
    }
    if constexpr (KT == KVM_Q4_0) {
        const uint8_t* b = row + (d / 32) * 18u;
        const int code = (b[2 + at % 16] >> (at < 16 ? 0 : 4)) & 15;
        return __fmul_rn(float(code - 8), __half2float(*reinterpret_cast<const __half*>(b)));
    }
    if constexpr (KT == KVM_Q5_0) {
        const uint8_t* b = row + (d / 32) * 22u;
        const int low = (b[6 + at % 16] >> (at < 16 ? 0 : 4)) & 15;
        const int high = (b[2 + at / 8] >> (at % 8)) & 1;
        return __fmul_rn(float((low | (high << 4)) - 16), __half2float(*reinterpret_cast<const __half*>(b)));
    }
    return 0.f;
}

// Mean-K producer: sums[l][page][e] += K[l][t][e] for the tokens t of
// [tok0, tok_end) in page `page0 + blockIdx.y`, in token order, one f32 add per
// (token, element) as the reference's meank_add_* kernels
// (src/adapter/llama-kvmem-stagein.cu:270-316); e = kv_head * D + dim. Block
// (x = 0, layer 0) of each page also adds the page's new tokens to counts.
// Grid: x = ceil(n_embd / blockDim), y = pages touched, z = layers.
template <int KT>
__global__ void __launch_bounds__(256) meank_add_kernel(const uint8_t* k, uint64_t k_layer, uint64_t k_token,
                                                        uint64_t k_head, uint32_t D, uint32_t n_embd, uint64_t tok0,
                                                        uint64_t tok_end, uint32_t page_tokens, uint32_t page0,
                                                        float* sums, uint32_t pages, uint32_t* counts) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t p = page0 + blockIdx.y, l = blockIdx.z;
    const uint64_t pb = uint64_t(p) * page_tokens;
    const uint64_t t0 = tok0 > pb ? tok0 : pb;
    const uint64_t t1 = tok_end < pb + page_tokens ? tok_end : pb + page_tokens;
    if (l == 0 && blockIdx.x == 0 && threadIdx.x == 0 && t1 > t0) counts[p] += uint32_t(t1 - t0);
    if (e >= n_embd) return;
    const uint32_t h = e / D, d = e % D;
    float* dst = sums + (uint64_t(l) * pages + p) * n_embd + e;
    float s = *dst;
    const uint8_t* base = k + l * k_layer + h * k_head;
    for (uint64_t t = t0; t < t1; ++t) s += key_elem<KT>(base + t * k_token, d);
    *dst = s;
}

}  // namespace kvmb
