// Budgeted top-k with keep pages, one CTA per score row.
//
// Same result as KvMemStore::pick_scored_blocks
// (kvmem/src/host/kvmem_store.cpp:418-451) with candidates = every page of
// the row and no media groups:
//   kept = keep pages; then pages ranked by (score desc, page id desc) fill the
//   budget; output ascending.
// Implementation: 4-pass 8-bit radix select over order-preserving 32-bit keys
// of the non-kept scores finds the threshold key T with
//   count(key > T) < need <= count(key >= T);
// every key > T is taken, and among keys == T the highest page ids
// (a descending-id ballot scan) fill the remainder. The output is an
// ascending compaction of the kept flags.
#pragma once
#include "common.cuh"

namespace kvmb {

constexpr int kSelectThreads = 512;

__device__ __forceinline__ uint32_t order_key(float s) {
    if (s == 0.f) s = 0.f;  // -0 == +0, as the reference's double comparison
    const uint32_t u = __float_as_uint(s);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kSelectThreads) select_topk_kernel(
    const float* scores, uint32_t pages, uint32_t score_stride, const uint32_t* keep, uint32_t nkeep, uint32_t budget,
    int signed_scores, uint32_t* out_ids, uint32_t* out_n, uint32_t out_stride, DeviceStatus* status) {
    extern __shared__ uint8_t kept[];  // [pages]
    __shared__ uint32_t hist[256];
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t sh_prefix, sh_need, sh_bad, sh_count;

    const uint32_t row = blockIdx.x;
    const float* sc = scores + uint64_t(row) * score_stride;
    const int tid = threadIdx.x;

    if (tid == 0) {
        sh_bad = 0;
        sh_count = 0;
    }
    for (uint32_t p = tid; p < pages; p += blockDim.x) kept[p] = 0;
    __syncthreads();
    for (uint32_t p = tid; p < pages; p += blockDim.x) {
        const float s = sc[p];
        if (!isfinite(s) || (!signed_scores && s < 0.f)) sh_bad = 1;
    }
    for (uint32_t i = tid; i < nkeep; i += blockDim.x) kept[keep[i]] = 1;
    __syncthreads();
    if (sh_bad) {
        if (tid == 0) {
            record_error(status, KVM_ERR_NONFINITE, 10);
            out_n[row] = 0;
        }
        return;
    }
    // Distinct keeps.
    uint32_t nk = 0;
    for (uint32_t p = tid; p < pages; p += blockDim.x) nk += kept[p];
    if (nk) atomicAdd(&sh_count, nk);
    __syncthreads();
    const uint32_t kept_n = sh_count;
    const uint32_t target = budget < pages ? budget : pages;
    uint32_t need = target > kept_n ? target - kept_n : 0;

    if (need > 0) {
        // Radix select of the need-th largest key among non-kept pages.
        uint32_t prefix = 0, prefix_mask = 0;
        for (int pass = 3; pass >= 0; --pass) {
            const int shift = pass * 8;
            for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
            __syncthreads();
            for (uint32_t p = tid; p < pages; p += blockDim.x) {
                if (kept[p]) continue;
                const uint32_t key = order_key(sc[p]);
                if ((key & prefix_mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                uint32_t acc = 0;
                int digit = 255;
                for (; digit > 0; --digit) {
                    if (acc + hist[digit] >= need) break;
                    acc += hist[digit];
                }
                sh_prefix = prefix | (uint32_t(digit) << shift);
                sh_need = need - acc;  // still needed from keys matching the new prefix
            }
            __syncthreads();
            prefix = sh_prefix;
            need = sh_need;
            prefix_mask |= 255u << shift;
            __syncthreads();
        }
        const uint32_t T = prefix;  // threshold key; `need` = how many keys == T to take
        for (uint32_t p = tid; p < pages; p += blockDim.x)
            if (!kept[p] && order_key(sc[p]) > T) kept[p] = 2;
        __syncthreads();
        // Among keys == T take the `need` highest page ids.
        if (tid < 32) {
            uint32_t taken = 0;
            for (int64_t base = int64_t(pages) - 1; base >= 0 && taken < need; base -= 32) {
                const int64_t p = base - tid;
                const bool tie = p >= 0 && kept[p] == 0 && order_key(sc[p]) == T;
                const uint32_t ball = __ballot_sync(0xffffffffu, tie);
                const uint32_t before = __popc(ball & ((1u << tid) - 1u));
                if (tie && taken + before < need) kept[p] = 2;
                taken += __popc(ball);
            }
        }
        __syncthreads();
    }

    // Ascending compaction.
    uint32_t written = 0;
    for (uint32_t base = 0; base < pages; base += blockDim.x) {
        const uint32_t p = base + tid;
        const uint32_t f = (p < pages && kept[p]) ? 1u : 0u;
        uint32_t pre;
        const uint32_t tot = block_exclusive_scan(f, warp_sums, &pre);
        if (f) out_ids[uint64_t(row) * out_stride + written + pre] = p;
        written += tot;
    }
    if (tid == 0) out_n[row] = written;
}

// ---------------------------------------------------------------- media groups
//
// Same result as KvMemStore::pick_scored_blocks (kvmem_store.cpp:418-451)
// with candidates = every page of the row and the store's media ranges: a page
// is admitted only together with its whole media group (the closure
// scored_media_group, kvmem_store.cpp:18-32, computes it: the pages covered by
// a chain of overlapping media ranges, or the page alone). Groups are disjoint
// intervals, so a group is decided once, at its best-ranked page: kept when it
// still fits the budget, skipped for good otherwise (its later pages find the
// same need and a count that only grew).
//
// group[p] (host-built): bits 0-14 first page of p's group, bits 15-29 one past
// its last page, bit 30 set when a keep page's group covers p (the host admits
// those groups first, in keep order, and rejects a list that overflows the
// budget before any launch). One CTA per row: a bitonic sort of the 64-bit
// keys (order_key(score) << 32 | page id, descending = score desc then id
// desc; kept pages get key 0, which no finite score produces) in shared memory,
// then one thread walks the ranked pages until the budget is full, and the
// block writes the kept pages in ascending order.
constexpr uint32_t kMediaMaxPages = 16384;
constexpr int kMediaThreads = 512;

__host__ __device__ inline size_t media_smem_bytes(uint32_t pages) {
    uint32_t n = 1;
    while (n < pages) n <<= 1;
    return size_t(n) * 8 + pages;
}

__global__ void __launch_bounds__(kMediaThreads) select_topk_media_kernel(
    const float* scores, uint32_t pages, uint32_t score_stride, const uint32_t* group, uint32_t kept0,
    uint32_t budget, int signed_scores, uint32_t* out_ids, uint32_t* out_n, uint32_t out_stride,
    DeviceStatus* status) {
    extern __shared__ uint64_t keys[];  // [npow2], then kept flags [pages]
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t sh_bad;
    uint32_t npow2 = 1;
    while (npow2 < pages) npow2 <<= 1;
    uint8_t* kept = reinterpret_cast<uint8_t*>(keys + npow2);  // 0 no, 1 kept, 2 group skipped (at its first page)
    const uint32_t row = blockIdx.x;
    const float* sc = scores + uint64_t(row) * score_stride;
    const int tid = threadIdx.x;
    if (tid == 0) sh_bad = 0;
    __syncthreads();
    for (uint32_t p = tid; p < npow2; p += blockDim.x) {
        uint64_t key = 0;
        if (p < pages) {
            const float s = sc[p];
            if (!isfinite(s) || (!signed_scores && s < 0.f)) sh_bad = 1;
            const bool k = (group[p] >> 30) & 1u;
            kept[p] = k ? 1 : 0;
            if (!k) key = (uint64_t(order_key(s)) << 32) | p;
        }
        keys[p] = key;
    }
    __syncthreads();
    if (sh_bad) {
        if (tid == 0) {
            record_error(status, KVM_ERR_NONFINITE, 11);
            out_n[row] = 0;
        }
        return;
    }
    // Bitonic sort, descending.
    for (uint32_t k = 2; k <= npow2; k <<= 1)
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t i = tid; i < npow2; i += blockDim.x) {
                const uint32_t ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t a = keys[i], b = keys[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? a < b : a > b) {
                        keys[i] = b;
                        keys[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    if (tid == 0) {
        uint32_t count = kept0;
        for (uint32_t i = 0; i < pages && count < budget; ++i) {
            const uint64_t key = keys[i];
            if (key == 0) break;  // only kept pages (and padding) remain
            const uint32_t p = uint32_t(key & 0xffffffffu), g = group[p];
            const uint32_t b = g & 0x7fffu, e = (g >> 15) & 0x7fffu;
            if (kept[b] != 0) continue;  // the group was decided at a better-ranked page
            const uint32_t need = e - b;
            if (count + need <= budget) {
                for (uint32_t q = b; q < e; ++q) kept[q] = 1;
                count += need;
            } else {
                kept[b] = 2;
            }
        }
    }
    __syncthreads();
    uint32_t written = 0;
    for (uint32_t base = 0; base < pages; base += blockDim.x) {
        const uint32_t p = base + tid;
        const uint32_t f = (p < pages && kept[p] == 1) ? 1u : 0u;
        uint32_t pre;
        const uint32_t tot = block_exclusive_scan(f, warp_sums, &pre);
        if (f) out_ids[uint64_t(row) * out_stride + written + pre] = p;
        written += tot;
    }
    if (tid == 0) out_n[row] = written;
}

}  // namespace kvmb
