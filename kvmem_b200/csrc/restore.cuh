// Raw-K restore transform of stage-in, fused into one kernel: packed q8_0 /
// q4_0 K rows -> f32 -> NeoX RoPE at the tokens' original positions ->
// Walsh-Hadamard transform over nrot-element chunks -> requantised into the
// device cache. The reference runs it as five launches through an f32 scratch
// buffer after a slab H2D copy (src/adapter/llama-kvmem-stagein.cu:104-234,
// 499-671, 673-811); here one CTA per token reads the packed row (device or
// mapped pinned host memory), keeps it in shared memory and writes the
// requantised row. Every f32 operation is rounded as written (no contraction),
// so the result is reproducible and equals the C restatement except where
// sincosf and the host's sinf / cosf differ in the last bits.
#pragma once
#include "common.cuh"

namespace kvmb {

struct RestoreItem {
    const uint8_t* src;
    uint8_t* dst;
    uint32_t tokens;
    int32_t pos0;
};

constexpr int kRestoreThreads = 256;

// One token of one item per CTA iteration. token_base: [n_items + 1] prefix
// sums of the items' token counts; theta: [n_rot / 2].
template <int KT>
__global__ void __launch_bounds__(kRestoreThreads) restore_k_kernel(const RestoreItem* items, uint32_t n_items,
                                                                    const uint64_t* token_base, uint32_t n_head,
                                                                    uint32_t D, uint32_t n_rot, const float* theta,
                                                                    uint32_t nrot, float fwht_scale) {
    static_assert(KT == KVM_Q8_0 || KT == KVM_Q4_0, "restore keys are q8_0 or q4_0");
    constexpr uint32_t kBlock = KT == KVM_Q8_0 ? 34 : 18;
    extern __shared__ float row[];  // [n_embd]
    const uint32_t n_embd = n_head * D, nblk = n_embd / 32, rb = nblk * kBlock;
    const uint64_t total = token_base[n_items];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    for (uint64_t gt = blockIdx.x; gt < total; gt += gridDim.x) {
        uint32_t lo = 0, hi = n_items;  // last item whose base <= gt
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) / 2;
            if (token_base[mid] <= gt) lo = mid;
            else hi = mid;
        }
        const RestoreItem it = items[lo];
        const uint64_t t = gt - token_base[lo];
        const uint8_t* src = it.src + t * rb;
        uint8_t* dst = it.dst + t * rb;
        // Dequantise (llama-kvmem-stagein.cu:134-160).
        for (uint32_t e = tid; e < n_embd; e += blockDim.x) {
            const uint8_t* b = src + (e / 32) * kBlock;
            const uint32_t j = e % 32;
            const float d = __half2float(__ushort_as_half(uint16_t(b[0] | (b[1] << 8))));
            float code;
            if constexpr (KT == KVM_Q8_0) code = float(int8_t(b[2 + j]));
            else code = float(int((b[2 + j % 16] >> (j < 16 ? 0 : 4)) & 15) - 8);
            row[e] = __fmul_rn(code, d);
        }
        __syncthreads();
        // NeoX RoPE on the first n_rot dims of every head (:162-180).
        if (n_rot) {
            const uint32_t half = n_rot / 2;
            const float pos = float(int32_t(it.pos0 + int32_t(t)));
            for (uint32_t idx = tid; idx < n_head * half; idx += blockDim.x) {
                const uint32_t h = idx / half, i = idx % half;
                float s, c;
                sincosf(__fmul_rn(pos, theta[i]), &s, &c);
                float* r = row + h * D;
                const float x0 = r[i], x1 = r[i + half];
                r[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
                r[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
            }
            __syncthreads();
        }
        // Walsh-Hadamard transform of every nrot-element chunk (:104-130).
        if (nrot) {
            for (uint32_t e = tid; e < n_embd; e += blockDim.x) row[e] = __fmul_rn(row[e], fwht_scale);
            __syncthreads();
            const uint32_t pairs = n_embd / 2, half_chunk = nrot / 2;
            for (uint32_t h = 1; h < nrot; h *= 2) {
                for (uint32_t p = tid; p < pairs; p += blockDim.x) {
                    const uint32_t c0 = (p / half_chunk) * nrot, q = p % half_chunk;
                    const uint32_t i = c0 + (q / h) * 2 * h + (q % h);
                    const float a = row[i], b = row[i + h];
                    row[i] = __fadd_rn(a, b);
                    row[i + h] = __fsub_rn(a, b);
                }
                __syncthreads();
            }
        }
        // Requantise, one warp per 32-element block (:182-234).
        for (uint32_t blk = warp; blk < nblk; blk += nwarps) {
            const float v = row[blk * 32 + lane];
            uint8_t* b = dst + blk * kBlock;
            if constexpr (KT == KVM_Q8_0) {
                float amax = fabsf(v);
#pragma unroll
                for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
                // The fp16 scale as one 16-bit store (blocks of 34 / 18 bytes keep it 2-byte aligned).
                if (lane == 0) *reinterpret_cast<uint16_t*>(b) = __half_as_ushort(__float2half_rn(d));
                b[2 + lane] = uint8_t(int8_t(roundf(__fmul_rn(v, id))));
            } else {
                // The first element (lowest index) of largest magnitude, as the
                // reference's sequential strict-greater scan.
                float best = fabsf(v);
                int at = lane;
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
                    const int oa = __shfl_xor_sync(0xffffffffu, at, o);
                    if (ob > best || (ob == best && oa < at)) {
                        best = ob;
                        at = oa;
                    }
                }
                const float vmax = __shfl_sync(0xffffffffu, v, at);
                const float d = __fdiv_rn(vmax, -8.0f);
                const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.0f;
                int xi = int(__fadd_rn(__fmul_rn(v, id), 8.5f));
                if (xi > 15) xi = 15;
                const int other = __shfl_down_sync(0xffffffffu, xi, 16);
                if (lane == 0) *reinterpret_cast<uint16_t*>(b) = __half_as_ushort(__float2half_rn(d));
                if (lane < 16) b[2 + lane] = uint8_t((xi & 15) | ((other & 15) << 4));
            }
        }
        __syncthreads();
    }
}

}  // namespace kvmb
