// Per-token page mass, first pass: page log-sum-exp over the K history.
//
// Restates the computation of the reference's page_lse kernel
// (src/adapter/llama-kvmem-attention-cuda.cu:59-97) with a B200 layout:
//  * one work unit = (layer, page): page_tokens x kv_heads K rows, contiguous
//    in the token-major cache, streamed into shared memory by bulk TMA copies
//    (cp.async.bulk) through an S-stage mbarrier ring fed by one producer warp;
//  * each KV head's rows are read once for every query vector that shares it
//    (up to 8 per pass: the GQA group times the query rows), with the query
//    vectors held in registers;
//  * each row is split over LPR = head_dim/8 lanes (8 elements, 16 bytes of
//    fp16 per lane); partial dots of all query vectors are combined by a
//    transposed warp-shuffle reduction (VP/2 + VP/4 + ... shuffles) after
//    which each lane owns one query vector's dot and keeps its online
//    (max, sum) in the log2 domain;
//  * q8_0 / q4_0 / q5_0 blocks are decoded in registers from shared memory.
#pragma once
#include "common.cuh"

namespace kvmb {

constexpr int kLseConsumerWarps = 8;
constexpr int kLseThreads = (kLseConsumerWarps + 1) * 32;
constexpr int kLseStages = 6;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct LseParams {
    const uint8_t* k;       // K base of layer 0
    uint64_t k_layer;       // bytes between layers
    uint64_t page_bytes;    // page_tokens * kv_heads * row_bytes
    uint32_t chunk_bytes;   // tokens_per_chunk * kv_heads * row_bytes
    uint32_t chunks;        // chunks per page
    uint32_t tpc;           // tokens per chunk
    uint32_t kv_heads;
    uint32_t row_bytes;     // bytes of one (token, head) row
    uint32_t pages;
    uint32_t layers;
    uint32_t page_tokens;
    uint64_t tokens;        // visible tokens
    const uint8_t* q;
    int32_t q_type;
    uint32_t rows;          // query rows R
    uint64_t q_layer, q_row, q_head;
    uint32_t group;         // query heads per KV head (G)
    uint32_t q_heads;
    uint32_t v0;            // first query vector (r*G + g) of this pass
    uint32_t nv;            // query vectors in this pass (<= VP)
    float scale;
    float softcap;
    const uint8_t* mask;
    int32_t mask_type;
    uint64_t mask_row;
    float* lse;             // [layers][rows][q_heads][pages], natural log
    DeviceStatus* status;
    uint32_t stage_stride;  // bytes per ring stage in shared memory
    uint32_t stages;        // ring stages (tensor-core kernel; the SIMT kernel uses kLseStages)
    uint32_t row_set;       // bytes of one token across KV heads (kv_heads * row_bytes)
    uint32_t slot_stride;   // tensor-core kernel, quantised keys: padded shared-memory stride per token
    uint32_t hpg;           // quantised-key kernel: KV heads per TMA head group
    uint32_t groups_tma;    // quantised-key kernel: head groups (one tiled TMA box each per chunk)
    uint32_t head_major;    // tcgen05 kernel: K rows of one KV head are contiguous (head-major mirror)
};

// Decode the lane's 8 consecutive elements of one K row held in shared
// memory. Returns the block scale (1 for plain float types) that multiplies
// the lane's partial dot; kf receives the element values (codes for quants).
template <int KT>
__device__ __forceinline__ float load_k8(const uint8_t* row, int lig, float* kf) {
    if constexpr (KT == KVM_F16) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + lig * 16);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[i]));
            kf[2 * i] = f.x;
            kf[2 * i + 1] = f.y;
        }
        return 1.f;
    } else if constexpr (KT == KVM_BF16) {
        const uint4 w = *reinterpret_cast<const uint4*>(row + lig * 16);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            kf[2 * i] = __uint_as_float(ws[i] << 16);
            kf[2 * i + 1] = __uint_as_float(ws[i] & 0xffff0000u);
        }
        return 1.f;
    } else if constexpr (KT == KVM_F32) {
        const uint4 a = *reinterpret_cast<const uint4*>(row + lig * 32);
        const uint4 b = *reinterpret_cast<const uint4*>(row + lig * 32 + 16);
        kf[0] = __uint_as_float(a.x); kf[1] = __uint_as_float(a.y);
        kf[2] = __uint_as_float(a.z); kf[3] = __uint_as_float(a.w);
        kf[4] = __uint_as_float(b.x); kf[5] = __uint_as_float(b.y);
        kf[6] = __uint_as_float(b.z); kf[7] = __uint_as_float(b.w);
        return 1.f;
    } else {
        // GGUF blocks of 32: four lanes per block, lane j holds elements 8j..8j+7.
        const int b = lig >> 2, j = lig & 3;
        constexpr int kBlock = KT == KVM_Q8_0 ? 34 : (KT == KVM_Q4_0 ? 18 : 22);
        const uint8_t* blk = row + kBlock * b;
        const float d = __half2float(*reinterpret_cast<const __half*>(blk));
        const uint8_t* src;
        if constexpr (KT == KVM_Q8_0) src = blk + 2 + 8 * j;
        else if constexpr (KT == KVM_Q4_0) src = blk + 2 + 8 * (j & 1);
        else src = blk + 6 + 8 * (j & 1);
        // 8 bytes at a 2-byte aligned address: three aligned words + funnel shift.
        // (Each ring stage carries 16 bytes of slack, so the third word of the
        // last row stays inside the stage.)
        const uintptr_t addr = reinterpret_cast<uintptr_t>(src);
        const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~uintptr_t(3));
        const uint32_t sh = uint32_t(addr & 3) * 8;
        const uint32_t w0 = base[0], w1 = base[1], w2 = base[2];
        const uint32_t lo = __funnelshift_r(w0, w1, sh), hi = __funnelshift_r(w1, w2, sh);
        if constexpr (KT == KVM_Q8_0) {
            s8x4_to_f32(lo, kf);
            s8x4_to_f32(hi, kf + 4);
        } else {
            const uint32_t shift = 4 * (j >> 1);
            uint32_t nlo = (lo >> shift) & 0x0F0F0F0Fu, nhi = (hi >> shift) & 0x0F0F0F0Fu;
            float off = 8388616.f;  // 2^23 + 8
            if constexpr (KT == KVM_Q5_0) {
                const uint32_t qh = blk[2 + j];
                auto spread = [](uint32_t x) {
                    return ((x & 1u) | ((x & 2u) << 7) | ((x & 4u) << 14) | ((x & 8u) << 21)) << 4;
                };
                nlo |= spread(qh & 15u);
                nhi |= spread(qh >> 4);
                off = 8388624.f;  // 2^23 + 16
            }
            u8x4_to_f32(nlo, off, kf);
            u8x4_to_f32(nhi, off, kf + 4);
        }
        return d;
    }
}

template <int KT, int LPR, int VP, bool MASK>
__global__ void __launch_bounds__(kLseThreads, 2) page_lse_kernel(const LseParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = kLseConsumerWarps;
    constexpr int NG = NW * 32 / LPR;  // lane groups
    uint8_t* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kLseStages * P.stage_stride);
    uint64_t* empty = full + kLseStages;
    float* red_m = reinterpret_cast<float*>(empty + kLseStages);  // [2][NG*VP]
    float* red_s = red_m + 2 * NG * VP;
    int* abort_flag = reinterpret_cast<int*>(red_s + 2 * NG * VP);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kLseStages; ++s) {
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
        // Producer warp: one elected lane streams page chunks into the ring.
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            uint32_t it = 0, issued = 0;  // issued chunks form a prefix of the sequence
            for (uint32_t unit = unit_begin; unit < unit_end; ++unit) {
                const uint32_t l = unit / P.pages, p = unit % P.pages;
                const uint8_t* src = P.k + l * P.k_layer + uint64_t(p) * P.page_bytes;
                for (uint32_t c = 0; c < P.chunks; ++c, ++it) {
                    const uint32_t s = it % kLseStages, round = it / kLseStages;
                    if (*reinterpret_cast<volatile int*>(abort_flag)) continue;
                    if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) {
                        record_error(P.status, KVM_ERR_TIMEOUT, 1);
                        *reinterpret_cast<volatile int*>(abort_flag) = 1;
                        continue;
                    }
                    mbar_arrive_expect_tx(&full[s], P.chunk_bytes);
                    bulk_g2s(stages + s * P.stage_stride, src + uint64_t(c) * P.chunk_bytes, P.chunk_bytes, &full[s],
                             policy);
                    issued = it + 1;
                }
            }
            // Never leave the CTA with a copy in flight.
            for (uint32_t s = 0; s < kLseStages && s < issued; ++s) {
                const uint32_t last_round = (issued - 1 - s) / kLseStages;
                if (!mbar_wait(&full[s], last_round & 1)) record_error(P.status, KVM_ERR_TIMEOUT, 2);
            }
        }
        return;
    }

    // Consumers.
    const int gi = tid / LPR, lig = tid % LPR;
    const uint32_t kvh = gi % P.kv_heads, tsub = gi / P.kv_heads, nsub = NG / P.kv_heads;

    // Query vector owned by this lane after the transposed reduction.
    int myv = 0;
    {
        int c = VP;
#pragma unroll
        for (int s = LPR / 2; s >= 1; s >>= 1) {
            if (c > 1) {
                if (lig & s) myv += c / 2;
                c /= 2;
            }
        }
    }
    const bool rep = (lig & (LPR / VP - 1)) == 0;
    const float scale_l2 = P.scale * kLog2e;

    float qv[VP][8];
    uint32_t it = 0, ucount = 0, qlayer = 0xffffffffu;
    for (uint32_t unit = unit_begin; unit < unit_end; ++unit, ++ucount) {
        const uint32_t l = unit / P.pages, p = unit % P.pages;
        // Query vectors of this KV head for layer l, as f32 registers.
        if (l != qlayer) {
        qlayer = l;
#pragma unroll
        for (int v = 0; v < VP; ++v) {
            const uint32_t vg = P.v0 + v;
            const bool ok = v < int(P.nv);
            const uint32_t r = ok ? vg / P.group : 0, g = ok ? vg % P.group : 0;
            const uint8_t* qp = P.q + l * P.q_layer + r * P.q_row + (kvh * P.group + g) * P.q_head;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                qv[v][i] = ok ? load_scalar(qp + (lig * 8 + i) * type_bytes(P.q_type), P.q_type) : 0.f;
        }
        }
        // Row of this lane's query vector; lanes that own a padding vector
        // (myv >= nv) read row 0 so their mask reads stay in bounds.
        const uint32_t myr = myv < int(P.nv) ? (P.v0 + myv) / P.group : 0;
        float m = -INFINITY, ssum = 0.f;
        const uint64_t tok0 = uint64_t(p) * P.page_tokens;

        for (uint32_t c = 0; c < P.chunks; ++c, ++it) {
            const uint32_t s = it % kLseStages, round = it / kLseStages;
            bool ok = !*reinterpret_cast<volatile int*>(abort_flag);
            if (ok && !mbar_wait(&full[s], round & 1)) {
                record_error(P.status, KVM_ERR_TIMEOUT, 3);
                *reinterpret_cast<volatile int*>(abort_flag) = 1;
                ok = false;
            }
            if (ok) {
                const uint8_t* stage = stages + s * P.stage_stride;
                const uint64_t ctok = tok0 + uint64_t(c) * P.tpc;
#pragma unroll 2
                for (uint32_t tt = tsub; tt < P.tpc; tt += nsub) {
                    const uint8_t* row = stage + (tt * P.kv_heads + kvh) * P.row_bytes;
                    float kf[8];
                    const float d = load_k8<KT>(row, lig, kf);
                    float vals[VP];
#pragma unroll
                    for (int v = 0; v < VP; ++v) {
                        float a = 0.f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) a = fmaf(qv[v][i], kf[i], a);
                        vals[v] = (KT == KVM_Q8_0 || KT == KVM_Q4_0 || KT == KVM_Q5_0) ? a * d : a;
                    }
                    // Transposed reduction over the LPR lanes of this row.
#pragma unroll
                    for (int step = 0, sft = LPR / 2; sft >= 1; ++step, sft >>= 1) {
                        const int cnt = VP >> step;
                        if (cnt > 1) {
                            const bool up = lig & sft;
#pragma unroll
                            for (int j = 0; j < cnt / 2; ++j) {
                                const float send = up ? vals[j] : vals[j + cnt / 2];
                                const float keep = up ? vals[j + cnt / 2] : vals[j];
                                vals[j] = keep + __shfl_xor_sync(0xffffffffu, send, sft);
                            }
                        } else {
                            vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], sft);
                        }
                    }
                    const uint64_t t = ctok + tt;
                    float x;
                    if (P.softcap > 0.f) x = P.softcap * tanhf(vals[0] * P.scale / P.softcap) * kLog2e;
                    else x = vals[0] * scale_l2;
                    bool visible = t < P.tokens;
                    if constexpr (MASK) {
                        if (visible) {
                            const float bias = load_scalar(P.mask + myr * P.mask_row + t * type_bytes(P.mask_type),
                                                           P.mask_type);
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
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // Combine the lane groups that share a KV head.
        const int buf = ucount & 1;
        if (rep) {
            red_m[buf * NG * VP + gi * VP + myv] = m;
            red_s[buf * NG * VP + gi * VP + myv] = ssum;
        }
        named_sync(1, NW * 32);
        if (tid < int(P.kv_heads) * VP) {
            const uint32_t h_kv = tid / VP, v = tid % VP;
            float M = -INFINITY;
            for (uint32_t sub = 0; sub < nsub; ++sub)
                M = fmaxf(M, red_m[buf * NG * VP + (sub * P.kv_heads + h_kv) * VP + v]);
            float S = 0.f;
            if (M != -INFINITY)
                for (uint32_t sub = 0; sub < nsub; ++sub) {
                    const int at = buf * NG * VP + (sub * P.kv_heads + h_kv) * VP + v;
                    if (red_s[at] > 0.f) S += red_s[at] * fast_exp2(red_m[at] - M);
                }
            if (v < P.nv) {
                const uint32_t vg = P.v0 + v, r = vg / P.group, g = vg % P.group;
                const uint32_t h = h_kv * P.group + g;
                P.lse[((uint64_t(l) * P.rows + r) * P.q_heads + h) * P.pages + p] =
                    S > 0.f ? (M + fast_log2(S)) * kLn2 : -INFINITY;
            }
        }
    }
}

}  // namespace kvmb
