// Post-scoring fusion on the device, between the page scorer and the top-k:
// one-hop propagation of positive score mass over the attention-feedback
// graph, and the LRFU preview (decayed history plus gated current scores).
// Both run as one CTA: a frame has at most a few thousand pages.
#pragma once
#include "common.cuh"
#include "select.cuh"

namespace kvmb {

constexpr int kPostThreads = 1024;

// Deterministic block sum of one double per thread (fixed tree for a fixed
// block size). Contains __syncthreads: call from every thread.
__device__ __forceinline__ double block_sum_f64(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double w = lane < nw ? red[lane] : 0.0;
#pragma unroll
        for (int o = 16; o; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    const double total = red[32];
    __syncthreads();
    return total;
}

// Propagation (kvmem/src/host/graph_recall.cpp:494-551) with the transfer
// weights prepared by the host: page i sends total*seed[i]*out_w[k] for k in
// [out_off[i], out_off[i+1]) and receives total*seed[in_src[k]]*in_w[k] for k
// in [in_off[i], in_off[i+1]), seed = max(raw, 0)/total over transport pages.
__global__ void __launch_bounds__(kPostThreads) propagate_kernel(
    const float* raw, uint32_t n, const uint8_t* allowed, uint32_t nallowed, const uint32_t* out_off,
    const double* out_w, const uint32_t* in_off, const uint32_t* in_src, const double* in_w, float* out,
    DeviceStatus* status) {
    __shared__ double red[33];
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    double part = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = raw[i];
        if (!isfinite(v)) bad = 1;
        if (allowed[i] && v > 0.f) part += double(v);
    }
    const double total = block_sum_f64(part, red);  // the barrier inside also publishes `bad`
    if (bad || !isfinite(total)) {
        if (threadIdx.x == 0) record_error(status, KVM_ERR_NONFINITE, 60);
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = raw[i];
        return;
    }
    const bool pass = nallowed <= 1 || total == 0.0;
    // Every thread reads all of raw before any thread writes out (raw may alias out).
    float res[8];
    int cnt = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x, ++cnt) {
        const double ri = double(raw[i]);
        double v = ri;
        if (!pass) {
            const double si = allowed[i] && ri > 0.0 ? ri / total : 0.0;
            for (uint32_t k = out_off[i]; k < out_off[i + 1]; ++k) v -= total * si * out_w[k];
            for (uint32_t k = in_off[i]; k < in_off[i + 1]; ++k) {
                const double rs = double(raw[in_src[k]]);
                const double ss = rs > 0.0 ? rs / total : 0.0;
                v += total * ss * in_w[k];
            }
            const double residual = ri < 0.0 ? ri : 0.0;
            if (!isfinite(v) || v < residual - 1e-12 * (total > 1.0 ? total : 1.0))
                record_error(status, KVM_ERR_INVALID_ARGUMENT, 61);
            v = v > residual ? v : residual;
        }
        if (cnt < 8) res[cnt] = float(v);
    }
    __syncthreads();
    cnt = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x, ++cnt) out[i] = res[cnt];
}

// LRFU preview (kvmem/include/kvmem/lrfu.hpp:57-79): the ascending rank-th
// score as the gate (rank = UINT32_MAX: no gate), found by a 4-pass 8-bit
// radix select on order-preserving keys; then lambda*prev + gated score in
// double, rounded to f32.
__global__ void __launch_bounds__(kPostThreads) lrfu_preview_kernel(const float* scores, uint32_t n, const float* prev,
                                                                    uint32_t n_prev, double lambda, uint32_t rank,
                                                                    float* out, DeviceStatus* status) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sh_prefix, sh_need;
    __shared__ int bad;
    const int tid = threadIdx.x;
    if (tid == 0) bad = 0;
    __syncthreads();
    for (uint32_t i = tid; i < n; i += blockDim.x)
        if (!isfinite(scores[i])) bad = 1;
    __syncthreads();
    if (bad) {
        if (tid == 0) record_error(status, KVM_ERR_NONFINITE, 62);
        return;
    }
    float threshold = -INFINITY;
    if (rank != 0xffffffffu) {
        uint32_t prefix = 0, mask = 0, need = rank;
        for (int pass = 3; pass >= 0; --pass) {
            const int shift = pass * 8;
            for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
            __syncthreads();
            for (uint32_t i = tid; i < n; i += blockDim.x) {
                const uint32_t key = order_key(scores[i]);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                uint32_t acc = 0;
                int digit = 0;
                for (; digit < 255; ++digit) {
                    if (acc + hist[digit] > need) break;
                    acc += hist[digit];
                }
                sh_prefix = prefix | (uint32_t(digit) << shift);
                sh_need = need - acc;
            }
            __syncthreads();
            prefix = sh_prefix;
            need = sh_need;
            mask |= 255u << shift;
            __syncthreads();
        }
        // The score whose key is the selected one.
        const uint32_t key = prefix;
        threshold = __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
    }
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const double s = double(scores[i]);
        const double gated = scores[i] >= threshold ? s : (s < 0.0 ? s : 0.0);
        const double h = i < n_prev ? double(prev[i]) : 0.0;
        out[i] = float(lambda * h + gated);
    }
}

}  // namespace kvmb
