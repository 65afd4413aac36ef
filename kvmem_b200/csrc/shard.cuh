// Page-range sharding of one history over several GPUs (ranks).
//
// The softmax over pages spans every page of a layer, so a rank that holds
// pages [page0, page0 + local_pages) cannot normalise alone. The exchange is
// two all-gathers of small tensors between these kernels:
//   1. lse_stats_kernel: per (layer, row, head) the local max and sum of
//      exp(lse - max) over the local pages (the rank's softmax statistics);
//      all-gather; stats_merge_kernel: the global (max, 1/sum) per row.
//   2. page_mass_normalize_kernel with the global statistics gives the local
//      page masses; shard_candidates_kernel proposes each row's top-B local
//      pages that are not keep pages, as (score, global page id); all-gather;
//      shard_merge_kernel takes the B best of all candidates by
//      (score desc, page id desc), adds the keep pages and writes ascending ids.
// Any page of the global top-B is in the top-B of its own rank (fewer of its
// rank's pages can beat it), so the merge equals pick_scored_blocks over the
// whole row (kvmem/src/host/kvmem_store.cpp:418-451).
#pragma once
#include "common.cuh"
#include "page_mass.cuh"
#include "select.cuh"

namespace kvmb {

// stats[row] = (max_p lse[row][p], sum_p exp(lse - max)) over `pages` local pages.
__global__ void lse_stats_kernel(const float* lse, uint32_t nrows, uint32_t pages, float2* stats) {
    const uint32_t row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= nrows) return;
    const float* x = lse + uint64_t(row) * pages;
    float M = -INFINITY;
    for (uint32_t p = lane; p < pages; p += 32) M = fmaxf(M, x[p]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float S = 0.f;
    if (M != -INFINITY)
        for (uint32_t p = lane; p < pages; p += 32) S += fast_exp2((x[p] - M) * kLog2e);
#pragma unroll
    for (int o = 16; o; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (lane == 0) stats[row] = make_float2(M, S);
}

// gathered: [ranks][n] local (max, sum); global: [n] (max, 1/sum).
__global__ void stats_merge_kernel(const float2* gathered, uint32_t ranks, uint32_t n, float2* global) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float M = -INFINITY;
    for (uint32_t r = 0; r < ranks; ++r) M = fmaxf(M, gathered[uint64_t(r) * n + i].x);
    float S = 0.f;
    for (uint32_t r = 0; r < ranks; ++r) {
        const float2 g = gathered[uint64_t(r) * n + i];
        if (g.y > 0.f) S += g.y * fast_exp2((g.x - M) * kLog2e);
    }
    global[i] = make_float2(M, 1.f / S);  // an all-empty row gives (-inf, inf) -> NaN masses, as unsharded
}

// Per row: the top-`k` local pages that are not keep pages, as (score, page0 + p)
// in ascending page order, padded with (-inf, 0xffffffff).
__global__ void __launch_bounds__(kSelectThreads) shard_candidates_kernel(
    const float* scores, uint32_t pages, uint32_t score_stride, uint32_t page0, const uint32_t* keep, uint32_t nkeep,
    uint32_t k, float* cand_scores, uint32_t* cand_ids, DeviceStatus* status) {
    extern __shared__ uint8_t flag[];  // [pages] 1 = keep (excluded), 2 = selected
    __shared__ uint32_t hist[256];
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t sh_prefix, sh_need, sh_bad, sh_excl;
    const uint32_t row = blockIdx.x;
    const float* sc = scores + uint64_t(row) * score_stride;
    const int tid = threadIdx.x;
    if (tid == 0) {
        sh_bad = 0;
        sh_excl = 0;
    }
    for (uint32_t p = tid; p < pages; p += blockDim.x) flag[p] = 0;
    __syncthreads();
    for (uint32_t p = tid; p < pages; p += blockDim.x) {
        const float s = sc[p];
        if (!isfinite(s) || s < 0.f) sh_bad = 1;
    }
    // The keep list is distinct (the host removes duplicates).
    for (uint32_t i = tid; i < nkeep; i += blockDim.x) {
        const uint32_t g = keep[i];
        if (g >= page0 && g < page0 + pages) {
            flag[g - page0] = 1;
            atomicAdd(&sh_excl, 1u);
        }
    }
    __syncthreads();
    float* out_s = cand_scores + uint64_t(row) * k;
    uint32_t* out_i = cand_ids + uint64_t(row) * k;
    for (uint32_t i = tid; i < k; i += blockDim.x) {
        out_s[i] = -INFINITY;
        out_i[i] = 0xffffffffu;
    }
    if (sh_bad) {
        if (tid == 0) record_error(status, KVM_ERR_NONFINITE, 30);
        return;
    }
    const uint32_t avail = pages - min(pages, sh_excl);
    uint32_t need = min(k, avail);
    if (need > 0) {
        uint32_t prefix = 0, prefix_mask = 0;
        for (int pass = 3; pass >= 0; --pass) {
            const int shift = pass * 8;
            for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
            __syncthreads();
            for (uint32_t p = tid; p < pages; p += blockDim.x) {
                if (flag[p]) continue;
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
                sh_need = need - acc;
            }
            __syncthreads();
            prefix = sh_prefix;
            need = sh_need;
            prefix_mask |= 255u << shift;
            __syncthreads();
        }
        const uint32_t T = prefix;
        for (uint32_t p = tid; p < pages; p += blockDim.x)
            if (!flag[p] && order_key(sc[p]) > T) flag[p] = 2;
        __syncthreads();
        if (tid < 32) {
            uint32_t taken = 0;
            for (int64_t base = int64_t(pages) - 1; base >= 0 && taken < need; base -= 32) {
                const int64_t p = base - tid;
                const bool tie = p >= 0 && flag[p] == 0 && order_key(sc[p]) == T;
                const uint32_t ball = __ballot_sync(0xffffffffu, tie);
                const uint32_t before = __popc(ball & ((1u << tid) - 1u));
                if (tie && taken + before < need) flag[p] = 2;
                taken += __popc(ball);
            }
        }
        __syncthreads();
    }
    uint32_t written = 0;
    for (uint32_t base = 0; base < pages; base += blockDim.x) {
        const uint32_t p = base + tid;
        const uint32_t f = (p < pages && flag[p] == 2) ? 1u : 0u;
        uint32_t pre;
        const uint32_t tot = block_exclusive_scan(f, warp_sums, &pre);
        if (f) {
            out_s[written + pre] = sc[p];
            out_i[written + pre] = page0 + p;
        }
        written += tot;
    }
}

// Per row: the `budget - distinct keeps` best candidates of all ranks by
// (score desc, global id desc), plus the keep pages, as ascending ids.
// n = ranks * k candidates, at most kMergeMax.
constexpr uint32_t kMergeMax = 8192;

__global__ void __launch_bounds__(kSelectThreads) shard_merge_kernel(
    const float* cand_scores, const uint32_t* cand_ids, uint32_t ranks, uint32_t k, uint32_t nrows,
    const uint32_t* keep, uint32_t nkeep, uint32_t budget, uint32_t* out_ids, uint32_t* out_n, uint32_t out_stride) {
    extern __shared__ uint64_t keys[];  // [ranks * k], then chosen ids
    __shared__ uint32_t sh_keep_n, sh_nsel;
    const uint32_t row = blockIdx.x;
    const uint32_t n = ranks * k;
    uint32_t* chosen = reinterpret_cast<uint32_t*>(keys + n);  // [budget + nkeep]
    const int tid = threadIdx.x;
    // The keep list is distinct (the host removes duplicates).
    for (uint32_t i = tid; i < nkeep; i += blockDim.x) chosen[i] = keep[i];
    if (tid == 0) sh_keep_n = nkeep;
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const uint32_t r = i / k, j = i % k;
        const uint64_t at = (uint64_t(r) * nrows + row) * k + j;
        const uint32_t id = cand_ids[at];
        keys[i] = id == 0xffffffffu ? 0ull : (uint64_t(order_key(cand_scores[at])) << 32) | id;
    }
    __syncthreads();
    const uint32_t kn = sh_keep_n;
    const uint32_t want = budget > kn ? budget - kn : 0;
    // Rank of each valid candidate = number of larger keys (keys are distinct: ids are).
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const uint64_t key = keys[i];
        if (!key) continue;
        uint32_t rank = 0;
        for (uint32_t j = 0; j < n; ++j) rank += keys[j] > key;
        if (rank < want) chosen[kn + rank] = uint32_t(key & 0xffffffffu);
    }
    if (tid == 0) {
        uint32_t valid = 0;
        for (uint32_t j = 0; j < n; ++j) valid += keys[j] != 0;
        sh_nsel = kn + min(want, valid);
    }
    __syncthreads();
    const uint32_t total = sh_nsel;
    // Ascending output: position of each chosen id = number of smaller chosen ids.
    for (uint32_t i = tid; i < total; i += blockDim.x) {
        const uint32_t id = chosen[i];
        uint32_t pos = 0;
        for (uint32_t j = 0; j < total; ++j) pos += chosen[j] < id;
        out_ids[uint64_t(row) * out_stride + pos] = id;
    }
    if (tid == 0) out_n[row] = total;
}

}  // namespace kvmb
