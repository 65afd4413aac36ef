// Causal prompt (prefill) attention with the page log-sum-exp of sampled rows
// captured in the same pass, on the 5th-generation tensor cores (tcgen05).
//
// The engine's prefill attention already computes every logit of every prompt
// row; the page statistics KVMem needs for a few sampled rows (per (row, query
// head, page): log sum over the page's visible keys of exp(scale * q.k)) are a
// by-product of its online softmax. The reference captures them inside its FP8
// prompt kernels (backends/patches/ninfer-prefill-page-lse-kv-coverage.patch:
// prompt_page_lse_tile.cuh, PromptPageLseRows at :953-984 and the -inf
// clear of unvisited pages at :925-928, :945-947) instead of a second Q.K^T pass
// over the sampled rows. This kernel does the same on B200 for fp16 / bf16
// caches:
//
//  * one CTA per (128 prompt rows, key chunk, query head); K and V tiles of 64
//    keys of the head's KV head (GQA) are loaded by TMA (3-D maps over
//    [tokens][kv_heads][head_dim], 64-dim boxes, 128-byte swizzle) into rings
//    of 3 (head_dim 256) or 6 (head_dim 128) stages. The query tile lives in
//    tensor memory (the MMA's A operand), written once by the softmax threads,
//    which leaves the shared memory to the K / V rings: with two stages the
//    load of tile j + 2 only starts when tile j's MMA ends, and its latency
//    set the pace;
//  * one thread issues tcgen05.mma kind::f16: S = Q.K^T (M = 128 rows, N = 64
//    keys, fp32 in tensor memory, double buffered), then O += P.V (M = 128,
//    N = head_dim, K = 64 keys; V is the MN-major operand straight from its
//    token-major tile). S of tile j + 2 is issued right after P.V of tile j,
//    so the tensor core works on one tile while the softmax warps read the
//    next;
//  * four softmax warps own one row each per thread (tensor-memory lane =
//    row): causal mask, online max in the log2 domain with lazy rescaling (the
//    O accumulator in tensor memory is rescaled only when a row's max grows by
//    more than 2^8), P = exp2(x - m) written as fp16 / bf16 into a swizzled
//    shared-memory tile for the P.V MMA, and for a sampled row the page sums
//    of P, flushed as natural-log page LSE when a page ends;
//  * the epilogue divides O by the row sum and stores fp16 / bf16 rows, or,
//    when the row tile's keys are split into chunks (to fill the last wave of
//    CTAs on long histories), stores the chunk's unnormalised rows and (max,
//    sum) for prefill_combine_kernel.
// Every wait is bounded: a timeout records KVM_ERR_TIMEOUT, raises the CTA's
// abort flag, lets in-flight copies and MMAs finish and frees the tensor
// memory before the CTA exits.
#pragma once
#include <cuda.h>

#include "page_mass_tc.cuh"

namespace kvmb {

constexpr int kPfRows = 128;         // prompt rows per CTA (M)
constexpr int kPfKeys = 64;          // keys per tile
constexpr int kPfMaxSamples = 4096;  // sampled rows per call (the reference's scratch decides; 64 by default)
constexpr int kPfInlineSamples = 64; // up to this many travel in the launch parameters
constexpr int kPfThreads = 256;      // warp 0: K loads, 1: MMA, 2: V loads, 3: idle, 4-7: softmax
constexpr float kPfRescale = 8.f;    // lazy rescale threshold (log2 units)

struct PrefillParams {
    const uint8_t* q;     // prompt rows: element (i, h, d) at q + i*q_row + h*q_head + 2*d
    uint64_t q_row, q_head;
    uint32_t q_heads, kv_heads, width, q_tiles;
    uint32_t base;        // cache tokens before prompt row 0 (row i sits at base + i)
    float scale_log2;     // logit scale * log2(e)
    uint8_t* out;
    uint64_t out_row, out_head;
    float* lse;           // [samples][q_heads][pages] or null
    uint32_t pages, page_tokens, samples;
    // Key-range split: each (row tile, head) pair's key tiles in `splits` chunks of
    // whole capture pages (`granule` tiles); with splits > 1 every chunk writes its
    // unnormalised rows to part_o [splits][width][q_heads][head_dim] and its (max,
    // sum) to part_ml [splits][width][q_heads], merged by prefill_combine_kernel.
    uint32_t splits, granule;
    float* part_o;
    float2* part_ml;
    // Sampled prompt rows, ascending: in rows_inline when samples <= kPfInlineSamples
    // (no copy, no synchronisation), else in the device table `rows`.
    const uint32_t* rows;
    uint32_t rows_inline[kPfInlineSamples];
    DeviceStatus* status;
};

__host__ __device__ constexpr uint32_t pf_kv_stage(int KA) { return uint32_t(KA) * kPfKeys * 128; }
__host__ __device__ constexpr uint32_t pf_stages(int KA) { return KA == 4 ? 3u : 6u; }  // per K and per V ring
__host__ __device__ constexpr uint32_t pf_p_bytes() { return kPfRows * 128; }
__host__ __device__ constexpr size_t pf_smem_bytes(int KA) {
    return 1024 + 2 * pf_stages(KA) * pf_kv_stage(KA) + 2 * pf_p_bytes() + 512;
}
// Tensor-memory columns: S double buffer (2 x 64), O (head_dim), Q (head_dim / 2:
// two 16-bit elements per column).
constexpr uint32_t kPfTmemCols = 512;

// Shared-memory descriptor of an MN-major operand in the 128-byte-swizzle
// layout: for each K index a row of 64 contiguous MN elements (128 bytes),
// 8-row groups 1024 bytes apart (stride byte offset), consecutive 64-element
// MN blocks `lbo` bytes apart (leading byte offset).
__device__ __forceinline__ uint64_t pf_desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16 instruction descriptor: fp32 D, A and B both fp16 (fmt 0) or both
// bf16 (fmt 1), A K-major, B K-major or MN-major (bit 16), N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t pf_idesc(uint32_t M, uint32_t N, bool bf16, bool b_mn) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn ? 1u : 0u) << 16) |
           ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Tiled 3-D TMA load of one box into this CTA's shared memory (this CTA only).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// All lanes poll the barrier (each gets the acquire), then agree.
__device__ __forceinline__ bool pf_warp_wait(uint64_t* bar, uint32_t parity) {
    const bool ok = mbar_wait(bar, parity);
    return __all_sync(0xffffffffu, ok);
}

// Three-input max (sm_100).
__device__ __forceinline__ float pf_max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// (d0, d1) = (a0, a1) * b + c, one packed f32x2 FMA (sm_100), rounded as two FMAs.
__device__ __forceinline__ void pf_fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\t"
        "mov.b64 rc, {%5, %5};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

// (s0, s1) += (a0, a1), one packed f32x2 add (sm_100).
__device__ __forceinline__ void pf_add2(float& s0, float& s1, float a0, float a1) {
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "+f"(s0), "+f"(s1)
        : "f"(a0), "f"(a1));
}

// Max of 64 values in a tree of three-input maxes (32 instructions, depth 4).
__device__ __forceinline__ float pf_max64(const float* x) {
    float t[22], u[8];
#pragma unroll
    for (int i = 0; i < 21; ++i) t[i] = pf_max3(x[3 * i], x[3 * i + 1], x[3 * i + 2]);
    t[21] = x[63];
#pragma unroll
    for (int i = 0; i < 7; ++i) u[i] = pf_max3(t[3 * i], t[3 * i + 1], t[3 * i + 2]);
    u[7] = t[21];
    return pf_max3(pf_max3(u[0], u[1], u[2]), pf_max3(u[3], u[4], u[5]), fmaxf(u[6], u[7]));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pf_pack2(float a, float b) {
    if constexpr (BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

template <int KA, bool BF16>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const PrefillParams P) {
    constexpr uint32_t D = KA * 64;
    constexpr uint32_t kStage = pf_kv_stage(KA), kP = pf_p_bytes(), S = pf_stages(KA);
    constexpr uint32_t kAtomKV = kPfKeys * 128;
    constexpr uint32_t kCols = kPfTmemCols;
    constexpr uint32_t kColO = 2 * kPfKeys, kColQ = kColO + D;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* ksm = smem_raw + pad;    // [S] stages
    uint8_t* vsm = ksm + S * kStage;  // [S] stages
    uint8_t* psm = vsm + S * kStage;  // [2] P tiles
    uint64_t* bars = reinterpret_cast<uint64_t*>(psm + 2 * kP);
    uint64_t* q_full = bars;        // query tile written to tensor memory (128 arrivals)
    uint64_t* k_full = bars + 1;    // [S]
    uint64_t* k_empty = bars + 7;   // [S]
    uint64_t* v_full = bars + 13;   // [S]
    uint64_t* v_empty = bars + 19;  // [S]
    uint64_t* s_full = bars + 25;   // [2]
    uint64_t* p_full = bars + 27;   // [2]
    uint64_t* pv_done = bars + 29;  // [2]
    uint64_t* fin = bars + 31;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 32);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Unit = (row tile, key chunk, query head), query heads fastest so the heads of one KV
    // head read the same K / V tiles at about the same time; heaviest (last) row tiles first.
    const uint32_t h = blockIdx.x % P.q_heads;
    const uint32_t rest = blockIdx.x / P.q_heads;
    const uint32_t split = rest % P.splits;
    const uint32_t qt = P.q_tiles - 1 - rest / P.splits;
    const uint32_t kvh = h / (P.q_heads / P.kv_heads);
    const uint32_t r0 = qt * kPfRows, r1 = min(P.width, r0 + kPfRows);
    const uint32_t n_all = (P.base + r1 + kPfKeys - 1) / kPfKeys;  // key tiles the row tile sees
    const uint32_t chunk = (((n_all + P.splits - 1) / P.splits + P.granule - 1) / P.granule) * P.granule;
    const uint32_t jb = min(n_all, split * chunk), je = min(n_all, jb + chunk);
    const uint32_t n = je - jb;                 // key tiles this unit visits
    const uint32_t unmasked = P.base + r0 + 1;  // keys every row of the tile sees

    if (tid == 0) {
        mbar_init(q_full, 128);
        for (uint32_t i = 0; i < S; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 128);
            mbar_init(&pv_done[i], 1);
        }
        mbar_init(fin, 1);
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

    if (warp == 0 || warp == 2) {
        // ---- TMA producers: warp 0 K, warp 2 V ----
        if (lane == 0) {
            const bool is_k = warp == 0;
            uint8_t* ring = is_k ? ksm : vsm;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* empty = is_k ? k_empty : v_empty;
            const CUtensorMap* map = is_k ? &kmap : &vmap;
            uint32_t issued = 0;
            for (uint32_t j = 0; j < n; ++j) {
                if (*abort_flag) break;
                const uint32_t s = j % S;
                if (j >= S && !mbar_wait(&empty[s], ((j - S) / S) & 1)) {
                    record_error(P.status, KVM_ERR_TIMEOUT, is_k ? 70 : 71);
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], kStage);
#pragma unroll
                for (int a = 0; a < KA; ++a)
                    tma_load_3d(ring + s * kStage + a * kAtomKV, map, a * 64, int(kvh), int((jb + j) * kPfKeys),
                                &full[s]);
                issued = j + 1;
            }
            // Every issued copy lands before the CTA frees its shared memory.
            for (uint32_t j = issued > S ? issued - S : 0; j < issued; ++j)
                if (!mbar_wait(&full[j % S], (j / S) & 1)) record_error(P.status, KVM_ERR_TIMEOUT, 72);
        }
    } else if (warp == 1) {
        // ---- MMA issue: one thread ----
        if (lane == 0) {
            constexpr uint32_t idesc_qk = pf_idesc(kPfRows, kPfKeys, BF16, false);
            constexpr uint32_t idesc_pv = pf_idesc(kPfRows, D, BF16, true);
            int err = 0;
            auto issue_s = [&](uint32_t j) -> bool {
                const uint32_t s = j % S, b = j & 1;
                if (!mbar_wait(&k_full[s], (j / S) & 1)) return false;
                tc_fence_after();
                const uint32_t kb = smem_u32(ksm + s * kStage);
#pragma unroll
                for (int a = 0; a < KA; ++a)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)  // A: 16 query elements = 8 tensor-memory columns per k-step
                        tc_mma_ts(tmem + b * kPfKeys, tmem + kColQ + (a * 4 + kk) * 8,
                                  tc_desc_sw128(kb + a * kAtomKV + kk * 32), idesc_qk, (a | kk) != 0);
                tc_commit(&s_full[b]);
                tc_commit(&k_empty[s]);
                return true;
            };
            if (!mbar_wait(q_full, 0)) err = 80;
            tc_fence_after();
            if (!err && n > 0 && !issue_s(0)) err = 81;
            if (!err && n > 1 && !issue_s(1)) err = 81;
            for (uint32_t j = 0; j < n && !err; ++j) {
                if (*abort_flag) {
                    err = -1;
                    break;
                }
                const uint32_t b = j & 1, vs = j % S;
                if (!mbar_wait(&p_full[b], (j >> 1) & 1) || !mbar_wait(&v_full[vs], (j / S) & 1)) {
                    err = 82;
                    break;
                }
                tc_fence_after();
                const uint32_t pb = smem_u32(psm + b * kP), vb = smem_u32(vsm + vs * kStage);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc_mma(tmem + kColO, tc_desc_sw128(pb + kk * 32), pf_desc_mn_sw128(vb + kk * 2048, kAtomKV),
                           idesc_pv, (j | kk) != 0);
                tc_commit(&pv_done[b]);
                tc_commit(&v_empty[vs]);
                if (j + 2 < n && !issue_s(j + 2)) {
                    err = 81;
                    break;
                }
            }
            if (err > 0) {
                record_error(P.status, KVM_ERR_TIMEOUT, err);
                *abort_flag = 1;
            }
            // Every MMA this thread issued is complete before the tensor memory is freed.
            tc_commit(fin);
            if (!mbar_wait(fin, 0)) record_error(P.status, KVM_ERR_TIMEOUT, 83);
        }
    } else if (warp >= 4) {
        // ---- softmax, page capture and epilogue: thread = row = tensor-memory lane ----
        const uint32_t row = uint32_t(tid - 128);
        const uint32_t lane_addr = tmem + ((32u * uint32_t(warp & 3)) << 16);
        const uint32_t r = r0 + row;
        const uint32_t pos = P.base + min(r, P.width - 1);  // last key this row sees
        {
            // The query row into tensor memory (zeros past the prompt): the A operand of S = Q.K^T.
            const uint4* qp = reinterpret_cast<const uint4*>(P.q + size_t(r) * P.q_row + size_t(h) * P.q_head);
            const bool valid = r < P.width;
#pragma unroll
            for (uint32_t d0 = 0; d0 < D; d0 += 64) {
                uint32_t w[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint4 v = valid ? __ldg(qp + d0 / 8 + i) : make_uint4(0, 0, 0, 0);
                    w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
                }
                tc_st32(lane_addr + kColQ + d0 / 2, w);
            }
            tc_wait_st();
            tc_fence_before();
            mbar_arrive(q_full);
        }
        // Sampled slot of this row (binary search of the ascending list), -1 if none.
        int slot = -1;
        if (P.lse && r < P.width) {
            uint32_t lo = 0, hi = P.samples;
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if ((P.rows ? __ldg(P.rows + mid) : P.rows_inline[mid]) < r) lo = mid + 1;
                else hi = mid;
            }
            if (lo < P.samples && (P.rows ? __ldg(P.rows + lo) : P.rows_inline[lo]) == r) slot = int(lo);
        }
        float* lse_row = slot >= 0 ? P.lse + (size_t(slot) * P.q_heads + h) * P.pages : nullptr;
        const uint32_t pt = P.page_tokens;
        const float c = P.scale_log2;
        float m_used = -INFINITY, l = 0.f, page_acc = 0.f;
        bool ok = true;
        for (uint32_t j = 0; j < n; ++j) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) {
                ok = false;
                break;
            }
            const uint32_t b = j & 1;
            if (!pf_warp_wait(&s_full[b], (j >> 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[kPfKeys];
            {
                uint32_t u[kPfKeys];
                tc_ld32(lane_addr + b * kPfKeys, u);
                tc_ld32(lane_addr + b * kPfKeys + 32, u + 32);
                tc_wait_ld(u);
                tc_wait_ld(u + 32);
#pragma unroll
                for (int k = 0; k < kPfKeys; ++k) x[k] = __uint_as_float(u[k]);
            }
            const uint32_t k0 = (jb + j) * kPfKeys;
            if (k0 + kPfKeys > unmasked) {
#pragma unroll
                for (int k = 0; k < kPfKeys; ++k)
                    if (k0 + k > pos) x[k] = -INFINITY;
            }
            const float mt = pf_max64(x) * c;  // this tile's max in log2 units (-inf: nothing visible)
            float alpha = 1.f;
            if (j == 0) {
                // A finite floor for rows that see no key of this chunk's first tile (a chunk
                // past key 0): their P stays 0 until a visible key raises the max.
                m_used = fmaxf(mt, -1e30f);
            } else {
                const bool need = mt > m_used + kPfRescale;
                if (__any_sync(0xffffffffu, need)) {
                    if (need) {
                        alpha = fast_exp2(m_used - mt);
                        m_used = mt;
                        l *= alpha;
                        page_acc *= alpha;
                    }
                    // O holds P.V of tiles < j once that MMA is done; rescale this warp's rows.
                    if (!pf_warp_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (uint32_t cc = 0; cc < D; cc += 32) {
                        uint32_t o[32];
                        tc_ld32(lane_addr + kColO + cc, o);
                        tc_wait_ld(o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tc_st32(lane_addr + kColO + cc, o);
                    }
                    tc_wait_st();
                }
            }
            const float mneg = -m_used;
            float q2[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // pair sums per 16 keys
#pragma unroll
            for (int k = 0; k < kPfKeys; k += 2) {
                pf_fma2(x[k], x[k + 1], x[k], x[k + 1], c, mneg);
                x[k] = fast_exp2(x[k]);
                x[k + 1] = fast_exp2(x[k + 1]);
                pf_add2(q2[2 * (k >> 4)], q2[2 * (k >> 4) + 1], x[k], x[k + 1]);
            }
            // sums of P over keys 0-15, 16-31, 32-47, 48-63
            const float q16[4] = {q2[0] + q2[1], q2[2] + q2[3], q2[4] + q2[5], q2[6] + q2[7]};
            const float tsum = (q16[0] + q16[1]) + (q16[2] + q16[3]);
            l += tsum;
            if (lse_row) {
                // Page sums of this tile's P; a page's LSE is written when it ends.
                if (pt >= uint32_t(kPfKeys)) {
                    page_acc += tsum;
                    const uint32_t kend = k0 + kPfKeys;
                    if (kend % pt == 0 || jb + j + 1 == je) {
                        const uint32_t pg = k0 / pt;
                        if (pg < P.pages)
                            lse_row[pg] = page_acc > 0.f ? (m_used + fast_log2(page_acc)) * kLn2 : -INFINITY;
                        page_acc = 0.f;
                    }
                } else {
                    // Pages of 16 or 32 keys: four or two per tile.
                    const float part[4] = {pt == 16 ? q16[0] : q16[0] + q16[1], pt == 16 ? q16[1] : q16[2] + q16[3],
                                           q16[2], q16[3]};
                    const uint32_t per = uint32_t(kPfKeys) / pt;
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i) {
                        const uint32_t pg = k0 / pt + i;
                        if (i < per && pg < P.pages)
                            lse_row[pg] = part[i] > 0.f ? (m_used + fast_log2(part[i])) * kLn2 : -INFINITY;
                    }
                }
            }
            // P tile b is free once P.V of tile j - 2 is done.
            if (j >= 2 && !pf_warp_wait(&pv_done[b], ((j - 2) >> 1) & 1)) {
                ok = false;
                break;
            }
            uint8_t* prow = psm + b * kP + row * 128;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                uint4 v;
                v.x = pf_pack2<BF16>(x[8 * cc + 0], x[8 * cc + 1]);
                v.y = pf_pack2<BF16>(x[8 * cc + 2], x[8 * cc + 3]);
                v.z = pf_pack2<BF16>(x[8 * cc + 4], x[8 * cc + 5]);
                v.w = pf_pack2<BF16>(x[8 * cc + 6], x[8 * cc + 7]);
                *reinterpret_cast<uint4*>(prow + ((uint32_t(cc) ^ (row & 7)) << 4)) = v;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&p_full[b]);
        }
        if (lse_row && split + 1 == P.splits) {
            // Pages past the row tile's last key tile: no visible key, zero probability.
            const uint32_t first = (n_all * kPfKeys + pt - 1) / pt;
            for (uint32_t pg = first; pg < P.pages; ++pg) lse_row[pg] = -INFINITY;
        }
        const bool go = __shfl_sync(0xffffffffu, (ok && !*abort_flag) ? 1 : 0, 0) != 0;
        if (go && n == 0) {
            // An empty chunk: nothing to merge.
            if (r < P.width) P.part_ml[(size_t(split) * P.width + r) * P.q_heads + h] = make_float2(-1e30f, 0.f);
        } else if (go && P.splits > 1) {
            // ---- epilogue of one chunk: unnormalised rows and (max, sum) for the merge ----
            if (pf_warp_wait(&pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1)) {
                tc_fence_after();
                const size_t row_id = (size_t(split) * P.width + r) * P.q_heads + h;
                float* orow = P.part_o + row_id * D;
#pragma unroll 1
                for (uint32_t cc = 0; cc < D; cc += 32) {
                    uint32_t o[32];
                    tc_ld32(lane_addr + kColO + cc, o);
                    tc_wait_ld(o);
                    if (r < P.width) {
                        float4* dst = reinterpret_cast<float4*>(orow + cc);
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            dst[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                                 __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
                    }
                }
                if (r < P.width) P.part_ml[row_id] = make_float2(m_used, l);
            } else {
                record_error(P.status, KVM_ERR_TIMEOUT, 84);
                *abort_flag = 1;
            }
        } else if (go) {
            // ---- epilogue: O / l ----
            if (pf_warp_wait(&pv_done[(n - 1) & 1], ((n - 1) >> 1) & 1)) {
                tc_fence_after();
                const float inv = 1.f / l;
                uint8_t* orow = P.out + size_t(r) * P.out_row + size_t(h) * P.out_head;
#pragma unroll 1
                for (uint32_t cc = 0; cc < D; cc += 32) {
                    uint32_t o[32];
                    tc_ld32(lane_addr + kColO + cc, o);
                    tc_wait_ld(o);
                    if (r < P.width) {
                        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 2);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint4 v;
                            v.x = pf_pack2<BF16>(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
                            v.y = pf_pack2<BF16>(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
                            v.z = pf_pack2<BF16>(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
                            v.w = pf_pack2<BF16>(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
                            dst[i] = v;
                        }
                    }
                }
            } else {
                record_error(P.status, KVM_ERR_TIMEOUT, 84);
                *abort_flag = 1;
            }
        } else if (!ok) {
            record_error(P.status, KVM_ERR_TIMEOUT, 85);
            *abort_flag = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// Merge of the key chunks of one (prompt row, query head) per warp: rows scaled by
// 2^(m_c - max m) and divided by the merged sum; chunks with a zero sum are skipped.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) prefill_combine_kernel(const PrefillParams P) {
    const uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= P.width * P.q_heads) return;
    const size_t stride = size_t(P.width) * P.q_heads;
    float m = -INFINITY;
    for (uint32_t c = 0; c < P.splits; ++c) {
        const float2 ml = P.part_ml[c * stride + w];
        if (ml.y > 0.f) m = fmaxf(m, ml.x);
    }
    constexpr int E = D / 32;  // elements per lane
    float acc[E];
#pragma unroll
    for (int i = 0; i < E; ++i) acc[i] = 0.f;
    float lsum = 0.f;
    for (uint32_t c = 0; c < P.splits; ++c) {
        const float2 ml = P.part_ml[c * stride + w];
        if (!(ml.y > 0.f)) continue;
        const float a = exp2f(ml.x - m);
        lsum += a * ml.y;
        const float4* src = reinterpret_cast<const float4*>(P.part_o + (c * stride + w) * D) + lane * (E / 4);
#pragma unroll
        for (int i = 0; i < E / 4; ++i) {
            const float4 v = src[i];
            acc[4 * i] += a * v.x;
            acc[4 * i + 1] += a * v.y;
            acc[4 * i + 2] += a * v.z;
            acc[4 * i + 3] += a * v.w;
        }
    }
    const float inv = 1.f / lsum;
    const uint32_t r = w / P.q_heads, h = w % P.q_heads;
    uint8_t* orow = P.out + size_t(r) * P.out_row + size_t(h) * P.out_head + size_t(lane) * E * 2;
    uint32_t packed[E / 2];
#pragma unroll
    for (int i = 0; i < E / 2; ++i) packed[i] = pf_pack2<BF16>(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    if constexpr (E == 8) {
        *reinterpret_cast<uint4*>(orow) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    } else {
        *reinterpret_cast<uint2*>(orow) = make_uint2(packed[0], packed[1]);
    }
}

}  // namespace kvmb
