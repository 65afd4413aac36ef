// Per-token page mass, first pass, on the tensor cores: page log-sum-exp of
// up to 8 query vectors that share a KV head, for fp16 / q8_0 / q4_0 keys.
//
// Same result as page_lse_kernel (page_mass.cuh); the dot products of the
// query vectors with the page's K rows run as mma.sync m16n8k16 (fp16 inputs,
// fp32 accumulation) instead of FP32 FMAs:
//  * A (16 x 16, row-major) = the query vectors: rows 0..7 hold the fp16 "hi"
//    part of vectors 0..7, rows 8..15 their fp16 "lo" residual
//    (q' = hi + lo to ~2^-22 relative), after an exact power-of-two prescale
//    per vector that keeps |q'| <= 2^14 (no fp16 overflow). An f16 query has
//    lo = 0. C rows g and g+8 are then added: dot = hi.K + lo.K.
//  * B (16 x 8, col-major) = 8 K rows (tokens) of one KV head: a B fragment
//    is exactly one 16-byte load per lane from the staged K row (lane = token
//    n*4 + c holds dims 8c..8c+7 of a 32-dim chunk), because the k index of
//    the mma is permuted the same way for A: within chunk kk, k-step s, the
//    mma's k = 2c+j and 2c+8+j map to dims kk*32 + 8c + 4s + j and + 2 + j.
//  * q8_0 / q4_0 codes are exact in fp16; each 32-dim block is one chunk, its
//    partial dots are scaled by the token's block scale in fp32 and summed.
//    For these keys lane c takes codes 4c..4c+3 and 16+4c..16+4c+3 of a block
//    (two 32-bit words of q8_0 codes, one word of q4_0 nibbles) and the producer
//    copies every token into its own shared-memory slot whose stride is 16
//    bytes past a multiple of 128: the 8 tokens of an octet then start in 8
//    different bank groups and every quantised load is conflict-free.
//  * the K pages stream into shared memory through the same bulk-TMA mbarrier
//    ring as the SIMT kernel; each consumer warp owns octets of 8 tokens of
//    one KV head, keeps an online (max, sum) per (vector, token pair) and the
//    lanes / warps that share a vector are merged at the end of the page.
#pragma once
#include <type_traits>

#include "page_mass.cuh"

namespace kvmb {

constexpr int kMmaMaxStages = 8;

// Calls f(std::integral_constant<int, kk>) for kk = 0 .. N-1 (compile-time chunk index).
template <int N, int I = 0, class F>
__device__ __forceinline__ void unroll_kk(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        unroll_kk<N, I + 1>(f);
    }
}

__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Four signed int8 codes -> two half2 words, exactly (magic 1024 + 128 + c).
__device__ __forceinline__ void s8x4_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t x = w ^ 0x80808080u;
    const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152
    uint32_t a = __byte_perm(x, 0x64646464u, 0x5140), b = __byte_perm(x, 0x64646464u, 0x5342);
    __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias), hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
    lo = *reinterpret_cast<uint32_t*>(&ha);
    hi = *reinterpret_cast<uint32_t*>(&hb);
}

// Four nibble bytes (values 0..15) -> two half2 words of (v - offset), exactly.
__device__ __forceinline__ void u4x4_to_h2(uint32_t x, uint16_t offset_bits, uint32_t& lo, uint32_t& hi) {
    const __half2 bias = __half2half2(__ushort_as_half(offset_bits));
    uint32_t a = __byte_perm(x, 0x64646464u, 0x5140), b = __byte_perm(x, 0x64646464u, 0x5342);
    __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias), hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
    lo = *reinterpret_cast<uint32_t*>(&ha);
    hi = *reinterpret_cast<uint32_t*>(&hb);
}

// B fragments of one 32-dim chunk for this lane (token row `row`, lane part c):
// b[0..1] for k-step 0, b[2..3] for k-step 1.
//  fp16: dims 8c..8c+7 of the chunk, one 16-byte load.
//  q8_0 / q4_0: codes 4c..4c+3 (k-step 0) and 16+4c..16+4c+3 (k-step 1) of block kk.
template <int KT, int KK_INDEX>
__device__ __forceinline__ void load_b_chunk(const uint8_t* row, int c, uint32_t* b) {
    constexpr int kk = KK_INDEX;
    if constexpr (KT == KVM_F16) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + kk * 64 + c * 16);
        b[0] = w.x; b[1] = w.y; b[2] = w.z; b[3] = w.w;
    } else {
        constexpr int kBlock = KT == KVM_Q8_0 ? 34 : 18;
        // Rows start 4-byte aligned; a block's codes start 2 + 34kk (18kk) bytes in,
        // so the lane's words are aligned exactly when kk is odd.
        constexpr bool aligned = (kBlock * kk + 2) % 4 == 0;
        const uint8_t* src = row + kBlock * kk + 2 + 4 * c;
        uint32_t w0, w1 = 0;
        if constexpr (aligned) {
            w0 = *reinterpret_cast<const uint32_t*>(src);
            if constexpr (KT == KVM_Q8_0) w1 = *reinterpret_cast<const uint32_t*>(src + 16);
        } else {
            const uint32_t* a = reinterpret_cast<const uint32_t*>(src - 2);
            w0 = __funnelshift_r(a[0], a[1], 16);
            if constexpr (KT == KVM_Q8_0) w1 = __funnelshift_r(a[4], a[5], 16);
        }
        if constexpr (KT == KVM_Q8_0) {
            s8x4_to_h2(w0, b[0], b[1]);
            s8x4_to_h2(w1, b[2], b[3]);
        } else {
            u4x4_to_h2(w0 & 0x0F0F0F0Fu, 0x6408 /* 1032 */, b[0], b[1]);
            u4x4_to_h2((w0 >> 4) & 0x0F0F0F0Fu, 0x6408, b[2], b[3]);
        }
    }
}

template <int KT>
__device__ __forceinline__ float block_scale(const uint8_t* row, int kk) {
    constexpr int kBlock = KT == KVM_Q8_0 ? 34 : 18;
    return __half2float(*reinterpret_cast<const __half*>(row + kBlock * kk));
}

// KK = head_dim / 32 chunks per row.
template <int KT, int KK, bool MASK>
__global__ void __launch_bounds__(kLseThreads, 2) page_lse_mma_kernel(const LseParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = kLseConsumerWarps;
    constexpr bool QUANT = KT != KVM_F16;
    const uint32_t S = P.stages;
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * P.stage_stride);
    uint64_t* empty = full + kMmaMaxStages;
    float* red_m = reinterpret_cast<float*>(empty + kMmaMaxStages);  // [2][NW][8]
    float* red_s = red_m + 2 * NW * 8;
    int* abort_flag = reinterpret_cast<int*>(red_s + 2 * NW * 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    // Each CTA scores a contiguous range of (layer, page) units, so the query
    // registers are reloaded only when its range crosses a layer.
    const uint32_t units = P.layers * P.pages;
    const uint32_t per_cta = (units + gridDim.x - 1) / gridDim.x;
    const uint32_t unit_begin = min(units, blockIdx.x * per_cta), unit_end = min(units, unit_begin + per_cta);

    if (warp == NW) {
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            uint32_t it = 0, issued = 0;
            for (uint32_t unit = unit_begin; unit < unit_end; ++unit) {
                const uint32_t l = unit / P.pages, p = unit % P.pages;
                const uint8_t* src = P.k + l * P.k_layer + uint64_t(p) * P.page_bytes;
                for (uint32_t c = 0; c < P.chunks; ++c, ++it) {
                    const uint32_t s = it % S, round = it / S;
                    if (*reinterpret_cast<volatile int*>(abort_flag)) continue;
                    if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) {
                        record_error(P.status, KVM_ERR_TIMEOUT, 4);
                        *reinterpret_cast<volatile int*>(abort_flag) = 1;
                        continue;
                    }
                    mbar_arrive_expect_tx(&full[s], P.chunk_bytes);
                    if constexpr (QUANT) {
                        // One copy per token into its padded slot.
                        for (uint32_t t = 0; t < P.tpc; ++t)
                            bulk_g2s(stages + s * P.stage_stride + t * P.slot_stride,
                                     src + uint64_t(c) * P.chunk_bytes + uint64_t(t) * P.row_set, P.row_set, &full[s],
                                     policy);
                    } else {
                        bulk_g2s(stages + s * P.stage_stride, src + uint64_t(c) * P.chunk_bytes, P.chunk_bytes,
                                 &full[s], policy);
                    }
                    issued = it + 1;
                }
            }
            for (uint32_t s = 0; s < S && s < issued; ++s) {
                const uint32_t last_round = (issued - 1 - s) / S;
                if (!mbar_wait(&full[s], last_round & 1)) record_error(P.status, KVM_ERR_TIMEOUT, 5);
            }
        }
        return;
    }

    // Consumers: lane = g*4 + c. g is the query vector (A row) and the token
    // (B column) this lane loads; c the 8-dim part of each 32-dim chunk.
    const int g = lane >> 2, c = lane & 3;
    const uint32_t kvh = uint32_t(warp) % P.kv_heads;
    const uint32_t items = P.kv_heads * (P.tpc / 8);  // octets per chunk, a multiple of NW
    const bool gvalid = g < int(P.nv);
    const uint32_t myr = gvalid ? (P.v0 + g) / P.group : 0;
    const float scale_l2 = P.scale * kLog2e;

    uint32_t qa[KK][2][4];  // A fragments: [chunk][k-step][a0..a3]
    float qinv = 1.f;       // 2^-shift of this lane's vector prescale
    uint32_t it = 0, ucount = 0, qlayer = 0xffffffffu;
    for (uint32_t unit = unit_begin; unit < unit_end; ++unit, ++ucount) {
        const uint32_t l = unit / P.pages, p = unit % P.pages;
        if (l != qlayer) {
            qlayer = l;
            // Query vector g of this KV head (8 dims per chunk), prescaled by 2^shift.
            float qv[KK][8];
            float amax = 0.f;
            const uint32_t vg = P.v0 + g, r = gvalid ? vg / P.group : 0, gg = gvalid ? vg % P.group : 0;
            const uint8_t* qp = P.q + l * P.q_layer + r * P.q_row + (kvh * P.group + gg) * P.q_head;
            const uint32_t esz = type_bytes(P.q_type);
            // Dims of this lane's 8 values in chunk kk: fp16 keys 8c..8c+7;
            // quantised keys 4c..4c+3 and 16+4c..16+4c+3 (see load_b_chunk).
#pragma unroll
            for (int kk = 0; kk < KK; ++kk)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int dim = QUANT ? kk * 32 + (i < 4 ? 4 * c + i : 16 + 4 * c + i - 4) : kk * 32 + c * 8 + i;
                    qv[kk][i] = gvalid ? load_scalar(qp + dim * esz, P.q_type) : 0.f;
                    amax = fmaxf(amax, fabsf(qv[kk][i]));
                }
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            int shift = 0;
            if (amax > 0.f) {
                const int e = int((__float_as_uint(amax) >> 23) & 255) - 127;  // floor(log2(amax))
                shift = min(100, max(-100, 13 - e));
            }
            const float qs = ldexpf(1.f, shift);
            qinv = ldexpf(1.f, -shift);
#pragma unroll
            for (int kk = 0; kk < KK; ++kk)
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    float h[4], lo[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float x = qv[kk][4 * s + j] * qs;
                        h[j] = __half2float(__float2half_rn(x));
                        lo[j] = x - h[j];
                    }
                    qa[kk][s][0] = pack_half2(h[0], h[1]);
                    qa[kk][s][1] = pack_half2(lo[0], lo[1]);
                    qa[kk][s][2] = pack_half2(h[2], h[3]);
                    qa[kk][s][3] = pack_half2(lo[2], lo[3]);
                }
        }
        float m = -INFINITY, ssum = 0.f;  // online state of (vector g, this lane's token pairs)
        const uint64_t tok0 = uint64_t(p) * P.page_tokens;

        for (uint32_t ch = 0; ch < P.chunks; ++ch, ++it) {
            const uint32_t s = it % S, round = it / S;
            bool ok = !*reinterpret_cast<volatile int*>(abort_flag);
            if (ok && !mbar_wait(&full[s], round & 1)) {
                record_error(P.status, KVM_ERR_TIMEOUT, 6);
                *reinterpret_cast<volatile int*>(abort_flag) = 1;
                ok = false;
            }
            if (ok) {
                const uint8_t* stage = stages + s * P.stage_stride;
                for (uint32_t item = warp; item < items; item += NW) {
                    const uint32_t oct = item / P.kv_heads;  // kv head of `item` is kvh
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
                    if constexpr (!QUANT) {
                        const uint8_t* brow = stage + ((oct * 8 + g) * P.kv_heads + kvh) * P.row_bytes;
                        uint32_t b[KK][4];
                        unroll_kk<KK>([&](auto kkc) {
                            constexpr int kk = decltype(kkc)::value;
                            load_b_chunk<KT, kk>(brow, c, b[kk]);
                        });
#pragma unroll
                        for (int kk = 0; kk < KK; ++kk) {
                            mma_16816(acc, qa[kk][0], b[kk][0], b[kk][1]);
                            mma_16816(acc, qa[kk][1], b[kk][2], b[kk][3]);
                        }
                    } else {
                        const uint8_t* brow = stage + (oct * 8 + g) * P.slot_stride + kvh * P.row_bytes;
                        const uint8_t* crow0 = stage + (oct * 8 + 2 * c) * P.slot_stride + kvh * P.row_bytes;
                        const uint8_t* crow1 = crow0 + P.slot_stride;
                        unroll_kk<KK>([&](auto kkc) {
                            constexpr int kk = decltype(kkc)::value;
                            uint32_t b[4];
                            load_b_chunk<KT, kk>(brow, c, b);
                            float blk[4] = {0.f, 0.f, 0.f, 0.f};
                            mma_16816(blk, qa[kk][0], b[0], b[1]);
                            mma_16816(blk, qa[kk][1], b[2], b[3]);
                            const float d0 = block_scale<KT>(crow0, kk), d1 = block_scale<KT>(crow1, kk);
                            acc[0] = fmaf(blk[0], d0, acc[0]);
                            acc[1] = fmaf(blk[1], d1, acc[1]);
                            acc[2] = fmaf(blk[2], d0, acc[2]);
                            acc[3] = fmaf(blk[3], d1, acc[3]);
                        });
                    }
                    // Tokens 2c and 2c+1 of the octet for vector g.
                    const uint64_t t0 = tok0 + uint64_t(ch) * P.tpc + oct * 8 + 2 * c;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const float dot = (acc[j] + acc[2 + j]) * qinv;
                        float x;
                        if (P.softcap > 0.f) x = P.softcap * tanhf(dot * P.scale / P.softcap) * kLog2e;
                        else x = dot * scale_l2;
                        const uint64_t t = t0 + j;
                        bool visible = gvalid && t < P.tokens;
                        if constexpr (MASK) {
                            if (visible) {
                                const float bias = load_scalar(
                                    P.mask + myr * P.mask_row + t * type_bytes(P.mask_type), P.mask_type);
                                visible = isfinite(bias);
                                x += bias * kLog2e;
                            }
                        }
                        if (visible) {
                            if (x > m) {
                                ssum = ssum * fast_exp2(m - x) + 1.f;
                                m = x;
                            } else {
                                ssum += fast_exp2(x - m);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // Merge the four lanes of vector g, then the warps of the KV head.
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, ssum, o);
            const float M = fmaxf(m, m2);
            float Sx = 0.f;
            if (M != -INFINITY) {
                if (ssum > 0.f) Sx += ssum * fast_exp2(m - M);
                if (s2 > 0.f) Sx += s2 * fast_exp2(m2 - M);
            }
            m = M;
            ssum = Sx;
        }
        const int buf = ucount & 1;
        if (c == 0) {
            red_m[(buf * NW + warp) * 8 + g] = m;
            red_s[(buf * NW + warp) * 8 + g] = ssum;
        }
        named_sync(1, NW * 32);
        if (tid < int(P.kv_heads) * 8) {
            const uint32_t h_kv = tid / 8, v = tid % 8;
            float M = -INFINITY;
            for (uint32_t w2 = h_kv; w2 < NW; w2 += P.kv_heads) M = fmaxf(M, red_m[(buf * NW + w2) * 8 + v]);
            float Sx = 0.f;
            if (M != -INFINITY)
                for (uint32_t w2 = h_kv; w2 < NW; w2 += P.kv_heads) {
                    const int at = (buf * NW + w2) * 8 + v;
                    if (red_s[at] > 0.f) Sx += red_s[at] * fast_exp2(red_m[at] - M);
                }
            if (v < P.nv) {
                const uint32_t vg = P.v0 + v, r = vg / P.group, gg = vg % P.group;
                const uint32_t h = h_kv * P.group + gg;
                P.lse[((uint64_t(l) * P.rows + r) * P.q_heads + h) * P.pages + p] =
                    Sx > 0.f ? (M + fast_log2(Sx)) * kLn2 : -INFINITY;
            }
        }
    }
}

}  // namespace kvmb
