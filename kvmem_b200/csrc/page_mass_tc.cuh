// Per-token page mass, first pass, on the 5th-generation tensor cores
// (tcgen05): page log-sum-exp of 16..256 query vectors per KV head (query
// replay / multi-lane batching turn the scoring into a real Q.K^T contraction),
// fp16 keys, head_dim 64 or 128.
//
// Same result as page_lse_kernel (page_mass.cuh) and page_lse_mma_kernel
// (page_mass_mma.cuh). One CTA per SM walks a contiguous range of units
// (layer, KV head, tile group); per 128-token tile:
//  * warp 0 (one thread) loads the tile's K rows of the KV head with tiled TMA
//    (a 4-D tensor map over [layers][tokens][kv_heads][head_dim], box
//    1 x 128 tokens x 1 x 64 dims, 128-byte swizzle) into a ring of
//    shared-memory stages, one 16 KiB atom per 64 dims;
//  * warp 1 owns the tensor-memory allocation, (re)builds the query tiles in
//    shared memory whenever its range crosses to another (layer, KV head), and
//    one of its threads issues tcgen05.mma kind::f16: A = query vectors
//    (M = 128 rows per M tile, K-major, 128-byte swizzle), B = the tile's K rows
//    (N = 128 tokens, K-major), D = fp32 in tensor memory, double buffered.
//    Each f32 query vector is prescaled by an exact power of two (|q'| <= 2^14)
//    and split into fp16 hi + lo parts (q' = hi + lo to ~2^-22 relative); the
//    two products accumulate into the same D, so the dot keeps ~f32 accuracy;
//  * warps 2.. read D with tcgen05.ld (one thread per query vector = one TMEM
//    lane, 32 tokens per load) and keep an online (max, sum) in the log2
//    domain per (vector, page), writing the page's natural-log LSE when the
//    page ends. A page larger than a tile spans consecutive tiles of one unit.
// Every wait is bounded: a timeout records KVM_ERR_TIMEOUT, raises the CTA's
// abort flag, lets the in-flight copies and MMAs finish and frees the tensor
// memory before the CTA exits.
#pragma once
#include <cuda.h>

#include "page_mass.cuh"

namespace kvmb {

constexpr int kTcTile = 128;            // tokens per MMA tile (N) and rows per M tile
constexpr int kTcAtomBytes = 128 * 128; // 128 rows x 64 fp16 dims (one swizzle atom column)
constexpr int kTcMaxStages = 8;

// Shared-memory matrix descriptor of a K-major operand in the canonical
// 128-byte-swizzle layout: rows of 128 bytes, 8-row groups 1024 bytes apart
// (stride byte offset), descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16 instruction descriptor: fp32 D (bits 4-5 = 1), fp16 A and B
// (formats 0), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t M, uint32_t N) {
    return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread is complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32*(w%4)..+31).
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Waits for this thread's tcgen05.ld results; the registers are in/out
// operands so no use of them can be scheduled before the wait.
__device__ __forceinline__ void tc_wait_ld(uint32_t* r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// Tiled 4-D TMA load of one box into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Power-of-two prescale exponent of a query vector: |q| * 2^shift < 2^14.
__device__ __forceinline__ int tc_shift_of(float amax) {
    if (!(amax > 0.f)) return 0;
    const int e = int((__float_as_uint(amax) >> 23) & 255) - 127;  // floor(log2(amax))
    return min(100, max(-100, 13 - e));
}

// Largest |element| of query vector `qp` (D elements of `type`).
__device__ __forceinline__ float tc_query_amax(const uint8_t* qp, int type, uint32_t D) {
    float amax = 0.f;
    if (type == KVM_F32 && (reinterpret_cast<uintptr_t>(qp) & 15) == 0) {
        const float4* q4 = reinterpret_cast<const float4*>(qp);
#pragma unroll 8
        for (uint32_t i = 0; i < D / 4; ++i) {
            const float4 x = q4[i];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
    } else {
        const uint32_t esz = type_bytes(type);
#pragma unroll 8
        for (uint32_t i = 0; i < D; ++i) amax = fmaxf(amax, fabsf(load_scalar(qp + i * esz, type)));
    }
    return amax;
}

// Byte offset of (row, k) in a 128-row x 64-dim fp16 swizzle atom: 16-byte
// chunk index XOR (row mod 8), as the 128-byte TMA swizzle writes it.
__device__ __forceinline__ uint32_t tc_sw128_offset(uint32_t row, uint32_t k) {
    const uint32_t byte = k * 2;
    return row * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15));
}

// Shared-memory bytes of the query tiles (hi and lo parts of MT M tiles).
__host__ __device__ constexpr uint32_t tc_q_bytes(int KA, int MT) { return uint32_t(MT) * 2 * KA * kTcAtomBytes; }

// Dynamic shared memory of the kernel: alignment pad, query tiles, K stages,
// mbarriers (2 x kTcMaxStages + 4), TMEM address slot and abort flag.
constexpr size_t kTcSmemMax = 227 * 1024;
__host__ __device__ constexpr size_t tc_smem_bytes(int KA, int MT, uint32_t stages) {
    return 1024 + tc_q_bytes(KA, MT) + size_t(stages) * KA * kTcAtomBytes + (2 * kTcMaxStages + 4) * 8 + 16;
}

// Units per (layer, KV head): one 128-token tile when pages are <= 128 tokens,
// one page (page_tokens / 128 tiles) when they are larger.
__host__ __device__ inline uint32_t tc_units_per_head(uint32_t pages, uint32_t page_tokens) {
    const uint64_t unit_tokens = page_tokens > uint32_t(kTcTile) ? page_tokens : uint32_t(kTcTile);
    return uint32_t((uint64_t(pages) * page_tokens + unit_tokens - 1) / unit_tokens);
}

template <int KA, int MT, bool MASK>
__global__ void __launch_bounds__(64 + 128 * MT, 1) page_lse_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                       const LseParams P) {
    constexpr uint32_t D = KA * 64;
    constexpr uint32_t kQBytes = tc_q_bytes(KA, MT);
    constexpr uint32_t kStageBytes = KA * kTcAtomBytes;
    constexpr uint32_t kCols = MT == 1 ? 256 : 512;  // 2 buffers x MT tiles x 128 fp32 columns
    constexpr uint32_t E = D / 32;                   // query dims per lane while building tiles
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* qsm = smem_raw + pad;
    uint8_t* ksm = qsm + kQBytes;
    const uint32_t S = P.stages;
    uint64_t* kfull = reinterpret_cast<uint64_t*>(ksm + S * kStageBytes);
    uint64_t* kempty = kfull + kTcMaxStages;
    uint64_t* tfull = kempty + kTcMaxStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t V = P.nv;                   // query vectors per KV head (rows * group)
    const uint32_t active_warps = (V + 31) / 32;  // epilogue warps that own at least one vector
    if (tid == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&kfull[s], 1);
            mbar_init(&kempty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], active_warps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Units: (layer, KV head, u); a unit is one tile (pages of <= 128 tokens:
    // 128 / page_tokens pages) or the `ut` tiles of one page (larger pages).
    const uint32_t ut = P.page_tokens > uint32_t(kTcTile) ? P.page_tokens / kTcTile : 1;
    const uint32_t upl = tc_units_per_head(P.pages, P.page_tokens);
    const uint64_t units = uint64_t(P.layers) * P.kv_heads * upl;
    const uint64_t ub = units * blockIdx.x / gridDim.x, ue = units * (blockIdx.x + 1) / gridDim.x;
    const uint32_t G = P.group;

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();
            uint32_t it = 0, issued = 0;
            for (uint64_t u = ub; u < ue && !*abort_flag; ++u) {
                const uint32_t lh = uint32_t(u / upl), j = uint32_t(u % upl);
                const int l = int(lh / P.kv_heads), h = int(lh % P.kv_heads);
                for (uint32_t t = 0; t < ut; ++t, ++it) {
                    const uint32_t s = it % S, round = it / S;
                    if (*abort_flag) break;
                    if (round > 0 && !mbar_wait(&kempty[s], (round - 1) & 1)) {
                        record_error(P.status, KVM_ERR_TIMEOUT, 40);
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&kfull[s], kStageBytes);
                    const int tok = int((uint64_t(j) * ut + t) * kTcTile);
#pragma unroll
                    for (int a = 0; a < KA; ++a)
                        tma_load_4d(ksm + s * kStageBytes + a * kTcAtomBytes, &kmap, a * 64, h, tok, l, &kfull[s],
                                    policy);
                    issued = it + 1;
                }
            }
            // Every issued copy lands before the CTA frees its shared memory.
            for (uint32_t s = 0; s < S && s < issued; ++s) {
                const uint32_t last_round = (issued - 1 - s) / S;
                if (!mbar_wait(&kfull[s], last_round & 1)) record_error(P.status, KVM_ERR_TIMEOUT, 41);
            }
        }
    } else if (warp == 1) {
        // ---- query tiles + MMA issue ----
        constexpr uint32_t idesc = tc_idesc(kTcTile, kTcTile);
        uint32_t it = 0, issued = 0, qlh = 0xffffffffu;
        for (uint64_t u = ub; u < ue; ++u) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;  // warp-uniform
            const uint32_t lh = uint32_t(u / upl);
            if (lh != qlh) {
                // The previous query tiles stay until every MMA reading them is done.
                int ok = 1;
                if (lane == 0 && issued > 0) ok = mbar_wait(&tfull[(issued - 1) & 1], ((issued - 1) >> 1) & 1);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) record_error(P.status, KVM_ERR_TIMEOUT, 42);
                    *abort_flag = 1;
                    break;
                }
                qlh = lh;
                const uint32_t l = lh / P.kv_heads, h = lh % P.kv_heads;
                // 16 vectors per pass (loads first, then the amax reductions, so
                // their latencies overlap); lane holds dims lane*E .. lane*E+E-1.
                for (uint32_t v0 = 0; v0 < uint32_t(MT) * kTcTile; v0 += 16) {
                    float x[16][E], am[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const uint32_t v = v0 + i;
                        am[i] = 0.f;
#pragma unroll
                        for (uint32_t k = 0; k < E; ++k) x[i][k] = 0.f;
                        if (v < V) {
                            const uint32_t r = v / G, hq = h * G + v % G;
                            const uint8_t* qp = P.q + l * P.q_layer + r * P.q_row + hq * P.q_head;
                            bool vec = false;
                            if constexpr (E == 4) {
                                if (P.q_type == KVM_F32 && (reinterpret_cast<uintptr_t>(qp) & 15) == 0) {
                                    const float4 f = reinterpret_cast<const float4*>(qp)[lane];
                                    x[i][0] = f.x;
                                    x[i][1] = f.y;
                                    x[i][2] = f.z;
                                    x[i][3] = f.w;
                                    vec = true;
                                }
                            }
                            if (!vec) {
                                const uint32_t esz = type_bytes(P.q_type);
#pragma unroll
                                for (uint32_t k = 0; k < E; ++k) x[i][k] = load_scalar(qp + (lane * E + k) * esz, P.q_type);
                            }
#pragma unroll
                            for (uint32_t k = 0; k < E; ++k) am[i] = fmaxf(am[i], fabsf(x[i][k]));
                        }
                    }
#pragma unroll
                    for (int o = 16; o; o >>= 1)
#pragma unroll
                        for (int i = 0; i < 16; ++i) am[i] = fmaxf(am[i], __shfl_xor_sync(0xffffffffu, am[i], o));
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const uint32_t v = v0 + i;
                        const float qs = ldexpf(1.f, tc_shift_of(am[i]));
                        const uint32_t mt = v / kTcTile, row = v % kTcTile;
                        const uint32_t d0 = lane * E, a = d0 / 64, k0 = d0 % 64;
                        uint32_t hw[E / 2], lw[E / 2];
#pragma unroll
                        for (uint32_t k = 0; k < E; k += 2) {
                            const float x0 = x[i][k] * qs, x1 = x[i][k + 1] * qs;
                            const float h0 = __half2float(__float2half_rn(x0)), h1 = __half2float(__float2half_rn(x1));
                            hw[k / 2] = pack_half2(h0, h1);
                            lw[k / 2] = pack_half2(x0 - h0, x1 - h1);
                        }
                        const uint32_t off = tc_sw128_offset(row, k0);
                        uint8_t* hi = qsm + ((mt * 2 + 0) * KA + a) * kTcAtomBytes + off;
                        uint8_t* lo = qsm + ((mt * 2 + 1) * KA + a) * kTcAtomBytes + off;
                        if constexpr (E == 4) {
                            *reinterpret_cast<uint2*>(hi) = make_uint2(hw[0], hw[1]);
                            *reinterpret_cast<uint2*>(lo) = make_uint2(lw[0], lw[1]);
                        } else {
                            *reinterpret_cast<uint32_t*>(hi) = hw[0];
                            *reinterpret_cast<uint32_t*>(lo) = lw[0];
                        }
                    }
                }
                // Generic-proxy stores -> visible to the tensor cores (async proxy).
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            for (uint32_t t = 0; t < ut; ++t, ++it) {
                int ok = 1;
                if (lane == 0) {
                    const uint32_t b = it & 1, s = it % S;
                    if (*abort_flag) ok = 0;
                    if (ok && it >= 2 && !mbar_wait(&tempty[b], ((it >> 1) - 1) & 1)) {
                        record_error(P.status, KVM_ERR_TIMEOUT, 43);
                        ok = 0;
                    }
                    if (ok && !mbar_wait(&kfull[s], (it / S) & 1)) {
                        record_error(P.status, KVM_ERR_TIMEOUT, 44);
                        ok = 0;
                    }
                    if (ok) {
                        tc_fence_after();
                        const uint32_t kbase = smem_u32(ksm + s * kStageBytes);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            const uint32_t dcol = tmem + (b * MT + mt) * kTcTile;
                            const uint32_t qhi = smem_u32(qsm + (mt * 2 + 0) * KA * kTcAtomBytes);
                            const uint32_t qlo = smem_u32(qsm + (mt * 2 + 1) * KA * kTcAtomBytes);
#pragma unroll
                            for (int a = 0; a < KA; ++a)
#pragma unroll
                                for (int kk = 0; kk < 4; ++kk) {
                                    const uint32_t koff = a * kTcAtomBytes + kk * 32;
                                    const uint64_t bd = tc_desc_sw128(kbase + koff);
                                    tc_mma(dcol, tc_desc_sw128(qhi + koff), bd, idesc, (a | kk) != 0);
                                    tc_mma(dcol, tc_desc_sw128(qlo + koff), bd, idesc, 1);
                                }
                        }
                        tc_commit(&kempty[s]);  // K stage reusable once these MMAs have read it
                        tc_commit(&tfull[b]);   // accumulator ready for the epilogue
                        issued = it + 1;
                    } else {
                        *abort_flag = 1;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
        // No MMA may still write tensor memory when it is freed.
        if (lane == 0 && issued > 0 && !mbar_wait(&tfull[(issued - 1) & 1], ((issued - 1) >> 1) & 1))
            record_error(P.status, KVM_ERR_TIMEOUT, 45);
    } else {
        // ---- epilogue: one thread per query vector ----
        const int e = warp - 2, mt = e / 4, sp = warp % 4;
        const uint32_t v = uint32_t(mt) * kTcTile + 32 * sp + lane;
        const bool warp_active = uint32_t(mt) * kTcTile + 32 * sp < V;
        if (warp_active) {
            const bool vvalid = v < V;
            const uint32_t r = vvalid ? v / G : 0, gsub = vvalid ? v % G : 0;
            const float scale_l2 = P.scale * kLog2e;
            uint32_t it = 0, qlh = 0xffffffffu;
            float cvt = 0.f, qinv = 1.f;
            float m = -INFINITY, ssum = 0.f;
            bool stop = false;
            for (uint64_t u = ub; u < ue && !stop; ++u) {
                const uint32_t lh = uint32_t(u / upl), j = uint32_t(u % upl);
                const uint32_t l = lh / P.kv_heads, h = lh % P.kv_heads;
                const uint32_t hq = h * G + gsub;
                if (lh != qlh) {
                    qlh = lh;
                    float amax = 0.f;
                    if (vvalid) amax = tc_query_amax(P.q + l * P.q_layer + r * P.q_row + hq * P.q_head, P.q_type, D);
                    qinv = ldexpf(1.f, -tc_shift_of(amax));
                    cvt = qinv * scale_l2;
                }
                for (uint32_t t = 0; t < ut; ++t, ++it) {
                    const uint32_t b = it & 1;
                    int ok = 1;
                    if (lane == 0) {
                        if (*abort_flag) ok = 0;
                        else if (!mbar_wait(&tfull[b], (it >> 1) & 1)) {
                            record_error(P.status, KVM_ERR_TIMEOUT, 46);
                            *abort_flag = 1;
                            ok = 0;
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t tok0 = (uint64_t(j) * ut + t) * kTcTile;
                    const uint32_t tbase = tmem + (uint32_t(32 * sp) << 16) + (b * MT + mt) * kTcTile;
#pragma unroll 1
                    for (int ch = 0; ch < kTcTile / 32; ++ch) {
                        uint32_t acc[32];
                        tc_ld32(tbase + ch * 32, acc);
                        tc_wait_ld(acc);
                        const uint64_t t0 = tok0 + uint64_t(ch) * 32;
                        if (vvalid) {
                            if (!MASK && !(P.softcap > 0.f) && t0 + 32 <= P.tokens) {
                                float mx = __uint_as_float(acc[0]);
#pragma unroll
                                for (int i = 1; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(acc[i]));
                                const float mn = fmaxf(m, mx * cvt);
                                float add = 0.f;
#pragma unroll
                                for (int i = 0; i < 32; ++i) add += fast_exp2(fmaf(__uint_as_float(acc[i]), cvt, -mn));
                                ssum = ssum * fast_exp2(m - mn) + add;
                                m = mn;
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i) {
                                    const uint64_t tt = t0 + i;
                                    if (tt >= P.tokens) continue;
                                    const float dot = __uint_as_float(acc[i]) * qinv;
                                    float x;
                                    if (P.softcap > 0.f) x = P.softcap * tanhf(dot * P.scale / P.softcap) * kLog2e;
                                    else x = dot * scale_l2;
                                    if constexpr (MASK) {
                                        const float bias =
                                            load_scalar(P.mask + r * P.mask_row + tt * type_bytes(P.mask_type),
                                                        P.mask_type);
                                        if (!isfinite(bias)) continue;
                                        x += bias * kLog2e;
                                    }
                                    if (x > m) {
                                        ssum = ssum * fast_exp2(m - x) + 1.f;
                                        m = x;
                                    } else {
                                        ssum += fast_exp2(x - m);
                                    }
                                }
                            }
                            if ((t0 + 32) % P.page_tokens == 0) {
                                const uint64_t p = t0 / P.page_tokens;
                                if (p < P.pages)
                                    P.lse[((uint64_t(l) * P.rows + r) * P.q_heads + hq) * P.pages + p] =
                                        ssum > 0.f ? (m + fast_log2(ssum)) * kLn2 : -INFINITY;
                                m = -INFINITY;
                                ssum = 0.f;
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[b]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
    }
}

}  // namespace kvmb
