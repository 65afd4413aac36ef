// Residency plan and device-initiated stage-in.
//
// plan_residency_kernel: one CTA per selection row. Follows plan_residency
// (kvmem/src/host/memory_contract.cpp:135-150) on the device:
//   evict   = resident \ selected     (every resident page when force_reload)
//   retain  = resident ∩ selected
//   restore = selected \ resident     (every selected page when force_reload)
// Restored pages (ascending) take the free slots (ascending); the table
// slot_of[row][page] / page_of[row][slot] is updated in place and the
// (page, slot) restore list is written for the gather.
//
// stagein_gather_kernel: every CTA walks the rows' restore lists and copies
// its share of (row, restore, plane) items from mapped pinned host memory to
// the device cache with 16-byte loads, several in flight per thread, so a few
// CTAs keep the PCIe / C2C link busy while the rest of the GPU scores.
#pragma once
#include "common.cuh"

namespace kvmb {

constexpr int kPlanThreads = 512;
// 128 threads and no shared memory per gather CTA: small enough to sit on an SM
// beside the two CTAs of the page scorer (2 x 288 threads x 96 registers, ~220 KB
// of shared memory), so a stage-in on a side stream runs during scoring instead
// of waiting for the scorer's persistent CTAs to exit.
constexpr int kGatherThreads = 128;
constexpr int kGatherDefaultCtas = 64;
constexpr int kGatherUnroll = 8;

struct PoolView {
    int32_t* slot_of;        // [rows][pages], -1 = not resident
    int32_t* page_of;        // [rows][slots], -1 = free
    uint32_t* restore;       // [rows][slots] restored pages of the last plan
    uint32_t* restore_slot;  // [rows][slots] their slots
    uint32_t* n_restore;     // [rows]
    uint32_t rows, pages, slots;
};

__global__ void __launch_bounds__(kPlanThreads) plan_residency_kernel(PoolView pool, uint32_t row0,
                                                                      const uint32_t* sel_ids, const uint32_t* sel_n,
                                                                      uint32_t sel_stride, int force_reload,
                                                                      uint32_t* n_restore_out, uint32_t* n_evict_out,
                                                                      DeviceStatus* status) {
    extern __shared__ uint8_t sel[];  // [pages]
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t sh_evict;
    const uint32_t row = row0 + blockIdx.x;
    const int tid = threadIdx.x;
    int32_t* slot_of = pool.slot_of + uint64_t(row) * pool.pages;
    int32_t* page_of = pool.page_of + uint64_t(row) * pool.slots;
    uint32_t* rest = pool.restore + uint64_t(row) * pool.slots;
    uint32_t* rest_slot = pool.restore_slot + uint64_t(row) * pool.slots;
    const uint32_t n = sel_n[blockIdx.x];
    const uint32_t* ids = sel_ids + uint64_t(blockIdx.x) * sel_stride;

    if (tid == 0) sh_evict = 0;
    for (uint32_t p = tid; p < pool.pages; p += blockDim.x) sel[p] = 0;
    __syncthreads();
    if (n > pool.slots) {
        if (tid == 0) {
            record_error(status, KVM_ERR_BUDGET_EXCEEDED, 20);
            pool.n_restore[row] = 0;
            if (n_restore_out) n_restore_out[blockIdx.x] = 0;
            if (n_evict_out) n_evict_out[blockIdx.x] = 0;
        }
        return;
    }
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const uint32_t p = ids[i];
        if (p < pool.pages) sel[p] = 1;
    }
    __syncthreads();
    // Evict.
    uint32_t ev = 0;
    for (uint32_t s = tid; s < pool.slots; s += blockDim.x) {
        const int32_t pg = page_of[s];
        if (pg >= 0 && (force_reload || !sel[pg])) {
            page_of[s] = -1;
            slot_of[pg] = -1;
            ++ev;
        }
    }
    if (ev) atomicAdd(&sh_evict, ev);
    __syncthreads();
    // Restore list (ascending pages) and free slots (ascending) paired in order.
    uint32_t written = 0;
    for (uint32_t base = 0; base < pool.pages; base += blockDim.x) {
        const uint32_t p = base + tid;
        const uint32_t f = (p < pool.pages && sel[p] && slot_of[p] < 0) ? 1u : 0u;
        uint32_t pre;
        const uint32_t tot = block_exclusive_scan(f, warp_sums, &pre);
        if (f) rest[written + pre] = p;
        written += tot;
    }
    uint32_t freed = 0;
    for (uint32_t base = 0; base < pool.slots && freed < written; base += blockDim.x) {
        const uint32_t s = base + tid;
        const uint32_t f = (s < pool.slots && page_of[s] < 0) ? 1u : 0u;
        uint32_t pre;
        const uint32_t tot = block_exclusive_scan(f, warp_sums, &pre);
        if (f && freed + pre < written) rest_slot[freed + pre] = s;
        freed += tot;
    }
    __syncthreads();
    for (uint32_t i = tid; i < written; i += blockDim.x) {
        const uint32_t p = rest[i], s = rest_slot[i];
        slot_of[p] = int32_t(s);
        page_of[s] = int32_t(p);
    }
    if (tid == 0) {
        pool.n_restore[row] = written;
        if (n_restore_out) n_restore_out[blockIdx.x] = written;
        if (n_evict_out) n_evict_out[blockIdx.x] = sh_evict;
    }
}

struct GatherLayout {
    uint32_t planes;
    const uint8_t* host_base[2];
    uint64_t host_row_stride[2], host_page_stride[2];
    uint8_t* dev_base[2];
    uint64_t dev_row_stride[2], dev_slot_stride[2];
    uint64_t bytes[2];
};

__device__ __forceinline__ void copy_item(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t bytes) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | bytes) & 15u) == 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        const uint64_t n4 = bytes >> 4;
        const uint64_t step = uint64_t(blockDim.x) * kGatherUnroll;
        uint64_t i = threadIdx.x;
        for (; i + uint64_t(kGatherUnroll - 1) * blockDim.x < n4; i += step) {
            uint4 v[kGatherUnroll];
#pragma unroll
            for (int u = 0; u < kGatherUnroll; ++u) v[u] = __ldcs(s4 + i + uint64_t(u) * blockDim.x);
#pragma unroll
            for (int u = 0; u < kGatherUnroll; ++u) __stcg(d4 + i + uint64_t(u) * blockDim.x, v[u]);
        }
        for (; i < n4; i += blockDim.x) __stcg(d4 + i, __ldcs(s4 + i));
    } else {
        for (uint64_t i = threadIdx.x; i < bytes; i += blockDim.x) dst[i] = src[i];
    }
}

// Restores of rows [row0, row0 + nrows) whose page lies in [page0, page_end)
// (the whole row: 0 and pages). The host records start at page page0: page p of
// row r is at host_base + r*host_row_stride + (p - page0)*host_page_stride, so a
// rank of a page-range partition passes only its own range's records. With
// `fence_sys`, every thread fences its writes at system scope before it exits:
// the destination may be another GPU's memory (a peer mapping), and the
// collective that follows the gather on the stream must find them in place.
__global__ void __launch_bounds__(kGatherThreads, 8) stagein_gather_kernel(PoolView pool, uint32_t row0, uint32_t nrows,
                                                                        GatherLayout lay, uint32_t page0,
                                                                        uint32_t page_end, int fence_sys) {
    uint64_t item = 0;
    for (uint32_t r = row0; r < row0 + nrows; ++r) {
        const uint32_t n = pool.n_restore[r];
        const uint32_t* rest = pool.restore + uint64_t(r) * pool.slots;
        const uint32_t* rest_slot = pool.restore_slot + uint64_t(r) * pool.slots;
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t p = rest[i], s = rest_slot[i];
            if (p < page0 || p >= page_end) continue;
            for (uint32_t j = 0; j < lay.planes; ++j, ++item) {
                if (item % gridDim.x != blockIdx.x) continue;
                const uint8_t* src = lay.host_base[j] + uint64_t(r) * lay.host_row_stride[j] +
                                     uint64_t(p - page0) * lay.host_page_stride[j];
                uint8_t* dst = lay.dev_base[j] + uint64_t(r) * lay.dev_row_stride[j] + uint64_t(s) * lay.dev_slot_stride[j];
                copy_item(src, dst, lay.bytes[j]);
            }
        }
    }
    if (fence_sys) __threadfence_system();
}

// Write-back before a restore may reuse slots (the spill of a working-set
// transfer): for every (row, slot, plane) whose published page p is evicted by
// the new plan (not at that slot in new_slot_of, or force_reload) and whose host
// copy is stale (stale[row][p] != 0), the device slot's bytes are copied to the
// page's host record (mapped pinned memory). Items are spread over the CTAs.
__global__ void __launch_bounds__(kGatherThreads, 8) spill_gather_kernel(const int32_t* old_page_of,
                                                                       const int32_t* new_slot_of,
                                                                       const uint8_t* stale, uint32_t rows,
                                                                       uint32_t pages, uint32_t slots, int force,
                                                                       GatherLayout lay) {
    const uint64_t items = uint64_t(rows) * slots * lay.planes;
    for (uint64_t item = blockIdx.x; item < items; item += gridDim.x) {
        const uint32_t j = uint32_t(item % lay.planes);
        const uint64_t rs = item / lay.planes;
        const uint32_t r = uint32_t(rs / slots), s = uint32_t(rs % slots);
        const int32_t p = old_page_of[rs];
        if (p < 0 || uint32_t(p) >= pages) continue;
        const uint64_t rp = uint64_t(r) * pages + uint32_t(p);
        if (!(force || new_slot_of[rp] != int32_t(s)) || !stale[rp]) continue;
        const uint8_t* src = lay.dev_base[j] + uint64_t(r) * lay.dev_row_stride[j] + uint64_t(s) * lay.dev_slot_stride[j];
        uint8_t* dst = const_cast<uint8_t*>(lay.host_base[j]) + uint64_t(r) * lay.host_row_stride[j] +
                       uint64_t(p) * lay.host_page_stride[j];
        copy_item(src, dst, lay.bytes[j]);
    }
}

struct CopyOp {
    const uint8_t* src;
    uint8_t* dst;
    uint64_t bytes;
};

__global__ void __launch_bounds__(kGatherThreads, 8) copy_ops_kernel(const CopyOp* ops, uint32_t n) {
    for (uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
        const CopyOp op = ops[i];
        if (op.src && op.dst && op.bytes) copy_item(op.src, op.dst, op.bytes);
    }
}

}  // namespace kvmb
