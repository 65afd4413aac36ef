// Per-token page mass, first pass, on the 5th-generation tensor cores
// (tcgen05): page log-sum-exp of 16..256 query vectors per KV head (query
// replay / multi-lane batching turn the scoring into a real Q.K^T contraction),
// fp16 keys, head_dim 64, 128 or 256 (256: up to 128 vectors per launch).
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
//    lane, 32 tokens per load; the packed second tile of 129..160 vectors
//    with 16x256b loads, four threads per vector) and keep an online
//    (max, sum) in the log2 domain per (vector, page), writing the page's
//    natural-log LSE when the page ends. A page larger than a tile spans
//    consecutive tiles of one unit. Each TMEM lane quadrant (= SM
//    sub-partition) gets the same share of the exponentials.
// Every wait is bounded: a timeout records KVM_ERR_TIMEOUT, raises the CTA's
// abort flag, lets the in-flight copies and MMAs finish and frees the tensor
// memory before the CTA exits.
#pragma once
#include <cuda.h>

#include "page_mass.cuh"
#include "page_mass_mma.cuh"  // pack_half2

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

// Query-tile layouts (LM): 1 = one M tile (16..128 vectors per KV head);
// 2 = plus a packed second M tile for vectors 128..159: in lane quadrant q,
// rows 32q+g hold the fp16 hi part and rows 32q+8+g the lo part of vector
// 128+8q+g (g < 8), so one MMA pass covers them and a 16x256b TMEM load hands
// each thread hi and lo of the same (vector, token) (lanes g and g+8).
__host__ __device__ constexpr int tc_layout_for(uint32_t nv) { return nv <= 128 ? 1 : 2; }
constexpr uint32_t kTcMaxVectors = 160;

// Tensor-memory columns (512 allocated). Layout 1: tile-0 accumulators triple
// buffered at [0, 384) and the tile-0 query operand (fp16 hi at [384, 384 + D/2),
// lo after it) at the top; at head_dim 256 the operand takes 256 columns, so the
// accumulators are double buffered at [0, 256) and the operand sits at
// [256, 512). Layout 2: tile-0 accumulators double buffered at [0, 256), the
// packed tile's accumulators double buffered at [256, 384) and [384, 512); the
// tile-0 query operand lives in shared memory.
constexpr uint32_t kTcColPacked = 256;
__host__ __device__ constexpr uint32_t tc_col_q(int KA) { return KA <= 2 ? 384u : 256u; }
// Tile-0 accumulator buffers.
__host__ __device__ constexpr uint32_t tc_acc_buffers(int KA, int LM) { return LM == 1 && KA <= 2 ? 3u : 2u; }

// Shared memory of the query operands of layout 2: the packed tile (KA atoms),
// then the tile-0 hi parts (KA atoms) and lo parts (KA atoms).
__host__ __device__ constexpr uint32_t tc_q_bytes(int KA, int LM) {
    return LM == 2 ? 3u * uint32_t(KA) * kTcAtomBytes : 0u;
}

// Dynamic shared memory of the kernel: alignment pad, packed query tile, K
// stages, mbarriers (2 x kTcMaxStages + 10), TMEM address slot and abort flag.
constexpr size_t kTcSmemMax = 227 * 1024;
__host__ __device__ constexpr size_t tc_smem_bytes(int KA, int LM, uint32_t stages) {
    return 1024 + tc_q_bytes(KA, LM) + size_t(stages) * KA * kTcAtomBytes + (2 * kTcMaxStages + 12) * 8 + 16;
}

// Threads per CTA: producer warp, MMA warp, two sets of tile-0 epilogue
// warps (one warp per TMEM lane quadrant each; the sets take alternate units),
// and (layout 2) one packed-tile epilogue warp per quadrant. At 448 threads
// (four warps on two SM sub-partitions) each thread may use 128 registers.
__host__ __device__ constexpr int tc_threads(int LM) { return LM == 1 ? 320 : 448; }

// Units per (layer, KV head): one 128-token tile when pages are <= 128 tokens,
// one page (page_tokens / 128 tiles) when they are larger.
__host__ __device__ inline uint32_t tc_units_per_head(uint32_t pages, uint32_t page_tokens) {
    const uint64_t unit_tokens = page_tokens > uint32_t(kTcTile) ? page_tokens : uint32_t(kTcTile);
    return uint32_t((uint64_t(pages) * page_tokens + unit_tokens - 1) / unit_tokens);
}

// tcgen05.mma kind::f16 with A in tensor memory (lane = row, two fp16 per
// 32-bit column along K) and B from shared memory.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane <- r.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
        "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// tcgen05.wait::ld that also takes the running (max, sum) as operands, so the
// arithmetic of the chunk before it cannot be moved after it (which would
// expose the next load's latency).
__device__ __forceinline__ void tc_wait_ld_after(uint32_t* r, float& m, float& s) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+f"(m), "+f"(s)
                 :
                 : "memory");
}

// fp16 hi / lo parts of 2 prescaled query values, packed.
__device__ __forceinline__ void tc_split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const float h0 = __half2float(__float2half_rn(x0)), h1 = __half2float(__float2half_rn(x1));
    hi = pack_half2(h0, h1);
    lo = pack_half2(x0 - h0, x1 - h1);
}

// 8 columns x 16 lanes per repetition, 8 repetitions (64 columns): thread t
// gets r[4i + j] = (lane t/4, column 8i + 2(t%4) + j) and r[4i + 2 + j] =
// (lane t/4 + 8, same column), j = 0, 1 (lanes relative to the warp's quadrant base).
__device__ __forceinline__ void tc_ld16x256x8(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// Online log2-domain (max, sum) of one query vector over a page's tokens.
struct TcLse {
    float m = -INFINITY, s = 0.f;

    // N dots (raw accumulators) that are all visible, unmasked, no softcap: x = acc * cvt.
    template <int N>
    __device__ __forceinline__ void add_fast(const float* a, float cvt) {
        float t[N / 2];
#pragma unroll
        for (int i = 0; i < N / 2; ++i) t[i] = fmaxf(a[i], a[i + N / 2]);
#pragma unroll
        for (int w = N / 4; w >= 1; w >>= 1)
#pragma unroll
            for (int i = 0; i < w; ++i) t[i] = fmaxf(t[i], t[i + w]);
        const float mn = fmaxf(m, t[0] * cvt);
        float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < N; ++i) p[i & 3] += fast_exp2(fmaf(a[i], cvt, -mn));
        s = s * fast_exp2(m - mn) + ((p[0] + p[1]) + (p[2] + p[3]));
        m = mn;
    }

    // One log2-domain logit x (already scaled, masked and capped).
    __device__ __forceinline__ void add_one(float x) {
        if (x > m) {
            s = s * fast_exp2(m - x) + 1.f;
            m = x;
        } else {
            s += fast_exp2(x - m);
        }
    }

    // Merge with another partial state (lanes sharing a vector).
    __device__ __forceinline__ void merge(float m2, float s2) {
        const float M = fmaxf(m, m2);
        float S = 0.f;
        if (M != -INFINITY) {
            if (s > 0.f) S += s * fast_exp2(m - M);
            if (s2 > 0.f) S += s2 * fast_exp2(m2 - M);
        }
        m = M;
        s = S;
    }

    __device__ __forceinline__ float lse_nat() const { return s > 0.f ? (m + fast_log2(s)) * kLn2 : -INFINITY; }
};

// Fields of the rare per-token path (mask, softcap, tokens past the visible end).
struct TcSlowArgs {
    uint64_t tokens;
    float scale, softcap;
    const uint8_t* mask;
    int32_t mask_type;
    uint64_t mask_row;
};

// The rare path of one 32-token chunk (a mask, a softcap, or tokens past the
// visible end): reloads the chunk's dots from tensor memory and folds them
// into (m, s) token by token. Called by the whole warp (the TMEM load is
// warp-collective); lanes without a valid vector return (m, s) unchanged.
// PACKED: 16x256b layout (dots hi + lo of the 8 tokens t0 + 8i + 2c4 + j of
// group grp); else 32x32b (token t0 + i). Kept out of line so the hot loop
// stays small, and so no register array of the hot loop is ever addressed.
template <bool MASK, bool PACKED>
__device__ __noinline__ float2 tc_fold_slow(const TcSlowArgs a, float m, float s, uint32_t taddr, int grp,
                                            uint64_t t0, int c4, float qinv, uint32_t r, bool valid) {
    uint32_t rr[32];
    if constexpr (PACKED) tc_ld16x256x8(taddr, rr);
    else tc_ld32(taddr, rr);
    tc_wait_ld(rr);
    TcLse st;
    st.m = m;
    st.s = s;
    if (!valid) return make_float2(m, s);
    constexpr int N = PACKED ? 8 : 32;
#pragma unroll
    for (int i = 0; i < N; ++i) {
        float dot;
        uint64_t t;
        if constexpr (PACKED) {
            const int ii = 4 * grp + i / 2, j = i & 1;
            dot = __uint_as_float(rr[4 * ii + j]) + __uint_as_float(rr[4 * ii + 2 + j]);
            t = t0 + 8 * (i >> 1) + 2 * c4 + j;
        } else {
            dot = __uint_as_float(rr[i]);
            t = t0 + i;
        }
        if (t >= a.tokens) continue;
        dot *= qinv;
        float x;
        if (a.softcap > 0.f) x = a.softcap * tanhf(dot * a.scale / a.softcap) * kLog2e;
        else x = dot * (a.scale * kLog2e);
        if constexpr (MASK) {
            const float bias = load_scalar(a.mask + r * a.mask_row + t * type_bytes(a.mask_type), a.mask_type);
            if (!isfinite(bias)) continue;
            x += bias * kLog2e;
        }
        st.add_one(x);
    }
    return make_float2(st.m, st.s);
}

// Writes this lane's query vector (prescaled by 2^shift, zeros when !valid)
// as fp16 hi parts at TMEM columns [qbase, qbase + D/2) and lo parts at
// [qbase + D/2, qbase + D) of the lane's row. Warp-collective; out of line
// (it runs once per (layer, KV head)).
template <uint32_t D>
__device__ __noinline__ bool tc_write_query_row(uint32_t qbase, const uint8_t* qp, int q_type, int shift, bool valid) {
    const float qs = ldexpf(1.f, shift);
    const uint32_t esz = type_bytes(q_type);
    uint32_t lo_bits = 0;
#pragma unroll
    for (uint32_t d0 = 0; d0 < D; d0 += 64) {
        uint32_t hw[32], lw[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            float x0 = 0.f, x1 = 0.f;
            if (valid) {
                x0 = load_scalar(qp + (d0 + 2 * i) * esz, q_type) * qs;
                x1 = load_scalar(qp + (d0 + 2 * i + 1) * esz, q_type) * qs;
            }
            tc_split2(x0, x1, hw[i], lw[i]);
            lo_bits |= lw[i] & 0x7FFF7FFFu;  // -0 counts as zero
        }
        tc_st32(qbase + d0 / 2, hw);
        tc_st32(qbase + D / 2 + d0 / 2, lw);
    }
    return lo_bits != 0;
}

// Walks units (layer, KV head, u) in order without 64-bit divisions per step.
struct TcUnit {
    uint32_t l, h, j, upl, heads;
    __device__ TcUnit(uint64_t u0, uint32_t upl_, uint32_t heads_) : upl(upl_), heads(heads_) {
        const uint64_t lh = u0 / upl_;
        j = uint32_t(u0 % upl_);
        l = uint32_t(lh / heads_);
        h = uint32_t(lh % heads_);
    }
    __device__ __forceinline__ void next() {
        if (++j == upl) {
            j = 0;
            if (++h == heads) {
                h = 0;
                ++l;
            }
        }
    }
};

template <int KA, int LM, bool MASK>
__global__ void __launch_bounds__(tc_threads(LM), 1) page_lse_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                             const LseParams P) {
    constexpr uint32_t D = KA * 64;
    constexpr uint32_t kQBytes = tc_q_bytes(KA, LM);
    constexpr uint32_t kStageBytes = KA * kTcAtomBytes;
    constexpr uint32_t kCols = 512;
    // Tile-0 accumulator buffers: three when neither a packed tile nor a
    // head_dim-256 query operand needs their columns.
    constexpr uint32_t NB = tc_acc_buffers(KA, LM);
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t* qsm = smem_raw + pad;                 // packed query tile (layout 2)
    uint8_t* q0hi = qsm + KA * kTcAtomBytes;       // tile-0 query operand, hi parts (layout 2)
    uint8_t* q0lo = q0hi + KA * kTcAtomBytes;      // tile-0 query operand, lo parts (layout 2)
    uint8_t* ksm = qsm + kQBytes;
    const uint32_t S = P.stages;
    uint64_t* kfull = reinterpret_cast<uint64_t*>(ksm + S * kStageBytes);
    uint64_t* kempty = kfull + kTcMaxStages;
    uint64_t* tfull = kempty + kTcMaxStages;  // [NB] tile-0 accumulators written
    uint64_t* tempty = tfull + 3;             // [NB] tile-0 accumulators read
    uint64_t* pfull = tempty + 3;             // [2] packed accumulators written
    uint64_t* pempty = pfull + 2;             // [2] packed accumulators read
    uint64_t* qfree = pempty + 2;             // MMAs reading the tile-0 query operand are done
    uint64_t* qready = qfree + 1;             // tile-0 query operand written
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qready + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // Set by the tile-0 query writers when any lo part of the (layer, KV head)'s
    // operand is nonzero; read and cleared by the MMA issuer after qready.
    volatile uint32_t* lo_any = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t V = P.nv;  // query vectors per KV head in this pass (vectors P.v0 .. P.v0 + V - 1)
    const uint32_t warps0 = (min(V, 128u) + 31) / 32;                  // active tile-0 epilogue warps
    const uint32_t warps1 = LM == 2 ? (V - 128 + 7) / 8 : 0;          // active packed epilogue warps
    if (tid == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&kfull[s], 1);
            mbar_init(&kempty[s], 1);
        }
        for (uint32_t b = 0; b < NB; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], warps0);
        }
        for (int pb = 0; pb < 2; ++pb) {
            mbar_init(&pfull[pb], 1);
            mbar_init(&pempty[pb], warps1 ? warps1 : 1);
        }
        mbar_init(qfree, 1);
        mbar_init(qready, warps0 + warps1);
        *abort_flag = 0;
        *lo_any = 0;
        mbar_fence_init();
    }
    if constexpr (LM == 2) {
        // Rows of the query tiles that no vector uses stay zero.
        uint4* z = reinterpret_cast<uint4*>(qsm);
        for (uint32_t i = tid; i < kQBytes / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
            uint32_t it = 0, issued = 0, s = 0, phase = 0;
            TcUnit un(ub, upl, P.kv_heads);
            for (uint64_t u = ub; u < ue && !*abort_flag; ++u, un.next()) {
                for (uint32_t t = 0; t < ut; ++t, ++it) {
                    if (*abort_flag) break;
                    if (it >= S && !mbar_wait(&kempty[s], phase ^ 1)) {
                        record_error(P.status, KVM_ERR_TIMEOUT, 40);
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&kfull[s], kStageBytes);
                    const int tok = int((uint64_t(un.j) * ut + t) * kTcTile);
#pragma unroll
                    for (int a = 0; a < KA; ++a)  // map dims: (D, heads, tokens) or, head-major, (D, tokens, heads)
                        tma_load_4d(ksm + s * kStageBytes + a * kTcAtomBytes, &kmap, a * 64,
                                    P.head_major ? tok : int(un.h), P.head_major ? int(un.h) : tok, int(un.l),
                                    &kfull[s], policy);
                    issued = it + 1;
                    if (++s == S) {
                        s = 0;
                        phase ^= 1;
                    }
                }
            }
            // Every issued copy lands before the CTA frees its shared memory.
            for (uint32_t s2 = 0; s2 < S && s2 < issued; ++s2) {
                const uint32_t last_round = (issued - 1 - s2) / S;
                if (!mbar_wait(&kfull[s2], last_round & 1)) record_error(P.status, KVM_ERR_TIMEOUT, 41);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue: one thread, nothing but barrier waits and MMAs ----
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc(kTcTile, kTcTile);
            uint32_t it = 0, ks = 0, kphase = 0, nq = 0, tb = 0, tround = 0;
            // Last tile whose K-stage commit was issued (that commit covers every
            // earlier MMA of this thread); the packed-tile MMAs of a tile are
            // issued one tile late so they never hold up the next tile-0 MMAs.
            int64_t last = -1;
            uint32_t pend_it = 0, pend_s = 0;
            bool pend = false, use_lo = true;
            int err = 0;
            auto issue_packed = [&]() -> bool {
                // Packed accumulator pend_it % 2, free once the epilogue read its use two tiles ago.
                const uint32_t pb = pend_it & 1;
                if (pend_it >= 2 && !mbar_wait(&pempty[pb], ((pend_it - 2) >> 1) & 1)) return false;
                tc_fence_after();
                const uint32_t kbase = smem_u32(ksm + pend_s * kStageBytes), qp0 = smem_u32(qsm);
#pragma unroll
                for (int a = 0; a < KA; ++a)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t off = a * kTcAtomBytes + kk * 32;
                        tc_mma(tmem + kTcColPacked + pb * kTcTile, tc_desc_sw128(qp0 + off), tc_desc_sw128(kbase + off), idesc,
                               (a | kk) != 0);
                    }
                tc_commit(&pfull[pb]);
                tc_commit(&kempty[pend_s]);
                last = pend_it;
                pend = false;
                return true;
            };
            TcUnit un(ub, upl, P.kv_heads);
            for (uint64_t u = ub; u < ue && !err; ++u, un.next()) {
                if (u == ub || un.j == 0) {
                    // New (layer, KV head): once every MMA reading the old query
                    // operands is done, the epilogue warps rewrite them.
                    if (LM == 2 && pend && !issue_packed()) {
                        err = 48;
                        break;
                    }
                    if (last >= 0 && !mbar_wait(&kempty[uint32_t(last) % S], (uint32_t(last) / S) & 1)) {
                        err = 42;
                        break;
                    }
                    tc_fence_before();
                    mbar_arrive(qfree);
                    if (!mbar_wait(qready, nq & 1)) {
                        err = 47;
                        break;
                    }
                    ++nq;
                    tc_fence_after();
                    use_lo = *lo_any != 0;  // all-zero lo parts (fp16 queries): skip their MMAs
                    *lo_any = 0;
                }
                for (uint32_t t = 0; t < ut; ++t, ++it) {
                    const uint32_t b = tb, s = ks;
                    if (*abort_flag) {
                        err = -1;
                        break;
                    }
                    if (tround >= 1 && !mbar_wait(&tempty[b], (tround - 1) & 1)) {
                        err = 43;
                        break;
                    }
                    if (!mbar_wait(&kfull[s], kphase)) {
                        err = 44;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t kbase = smem_u32(ksm + s * kStageBytes);
                    const uint32_t d0 = tmem + b * kTcTile;
                    if constexpr (LM == 1) {
                        const uint32_t qhi = tmem + tc_col_q(KA), qlo = tmem + tc_col_q(KA) + D / 2;
#pragma unroll
                        for (int a = 0; a < KA; ++a)
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint64_t bd = tc_desc_sw128(kbase + a * kTcAtomBytes + kk * 32);
                                const uint32_t acol = (a * 4 + kk) * 8;  // 16 fp16 = 8 columns per k-step
                                tc_mma_ts(d0, qhi + acol, bd, idesc, (a | kk) != 0);
                                if (use_lo) tc_mma_ts(d0, qlo + acol, bd, idesc, 1);
                            }
                    } else {
                        const uint32_t qh = smem_u32(q0hi), ql = smem_u32(q0lo);
#pragma unroll
                        for (int a = 0; a < KA; ++a)
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint32_t off = a * kTcAtomBytes + kk * 32;
                                const uint64_t bd = tc_desc_sw128(kbase + off);
                                tc_mma(d0, tc_desc_sw128(qh + off), bd, idesc, (a | kk) != 0);
                                if (use_lo) tc_mma(d0, tc_desc_sw128(ql + off), bd, idesc, 1);
                            }
                    }
                    tc_commit(&tfull[b]);  // tile-0 accumulator ready for the epilogue
                    if constexpr (LM == 2) {
                        if (pend && !issue_packed()) {
                            err = 48;
                            break;
                        }
                        pend = true;
                        pend_it = it;
                        pend_s = s;
                    } else {
                        tc_commit(&kempty[s]);  // K stage reusable once these MMAs have read it
                        last = it;
                    }
                    if (++ks == S) {
                        ks = 0;
                        kphase ^= 1;
                    }
                    if (++tb == NB) {
                        tb = 0;
                        ++tround;
                    }
                }
            }
            if (!err && LM == 2 && pend && !issue_packed()) err = 48;
            if (err) {
                if (err > 0) record_error(P.status, KVM_ERR_TIMEOUT, err);
                *abort_flag = 1;
            }
            // No MMA may still write tensor memory when it is freed.
            if (last >= 0 && !mbar_wait(&kempty[uint32_t(last) % S], (uint32_t(last) / S) & 1))
                record_error(P.status, KVM_ERR_TIMEOUT, 45);
        }
    } else {
        // ---- epilogue ----
        // Warps 2..5 and 6..9: tile 0, one thread per query vector (TMEM lane),
        // all 128 columns of a tile; the two sets take alternate units (whole
        // pages), so each has two tiles' time per tile and no page is split
        // between warps. Warps 2..5 also write the tile-0 query operand of their
        // vectors. Warps 10..13 (layout 2): the packed vectors 128+8q+g, four
        // threads per vector (token pairs 2(t%4)+j of every 8 columns), and the
        // packed query rows.
        const int q = warp % 4;
        const bool packed = warp >= 10;
        const uint32_t set = (!packed && warp >= 6) ? 1u : 0u;
        const int g = packed ? lane >> 2 : lane, c4 = lane & 3;
        const uint32_t v = packed ? kTcTile + 8 * q + g : 32 * q + lane;
        const bool warp_active = packed ? kTcTile + 8 * q < V : 32u * q < V;
        if (warp_active) {
            const bool vvalid = v < V;
            // This pass's vector v is vector P.v0 + v = (row r, head gsub of the group).
            const uint32_t r = vvalid ? (P.v0 + v) / G : 0, gsub = vvalid ? (P.v0 + v) % G : 0;
            const TcSlowArgs sa{P.tokens, P.scale, P.softcap, P.mask, P.mask_type, P.mask_row};
            // Page ends: pages of <= 128 tokens end every cpp = page_tokens / 32
            // chunks (a power of two) inside a tile; larger pages at the last
            // chunk of the unit's last tile.
            const bool small_pages = P.page_tokens <= uint32_t(kTcTile);
            const uint32_t cpp_log = small_pages ? (P.page_tokens == 32 ? 0 : P.page_tokens == 64 ? 1 : 2) : 2;
            const uint32_t ppt = small_pages ? kTcTile / P.page_tokens : 1;
            const uint32_t qbase = tmem + (uint32_t(32 * q) << 16) + tc_col_q(KA);
            uint32_t it = 0, nq = 0, tb = 0, tround = 0;
            float cvt = 0.f, qinv = 1.f;
            TcLse st;
            float* lse_row = P.lse;
            TcUnit un(ub, upl, P.kv_heads);
            bool stop = false;
            uint32_t k = 0;  // unit ordinal in this CTA (its parity picks the tile-0 set)
            for (uint64_t u = ub; u < ue && !stop; ++u, un.next(), ++k) {
                const bool mine = packed || (k & 1u) == set;
                if (u == ub || un.j == 0) {
                    const uint32_t hq = un.h * G + gsub;
                    const uint8_t* qp = P.q + un.l * P.q_layer + r * P.q_row + hq * P.q_head;
                    const float amax = vvalid ? tc_query_amax(qp, P.q_type, D) : 0.f;
                    const int shift = tc_shift_of(amax);
                    qinv = ldexpf(1.f, -shift);
                    cvt = qinv * P.scale * kLog2e;
                    lse_row = P.lse + ((uint64_t(un.l) * P.rows + r) * P.q_heads + hq) * P.pages;
                    if (packed) {
                        // This quadrant's rows of the packed query tile: vector
                        // 128+8q+g, hi at row 32q+g and lo at row 32q+8+g; lane c4
                        // writes dims [c4*D/4, (c4+1)*D/4) as 16-byte swizzled pieces.
                        int ok = 1;
                        if (lane == 0) ok = mbar_wait(qfree, nq & 1);
                        ok = __shfl_sync(0xffffffffu, ok, 0);
                        ++nq;
                        if (!ok) {
                            if (lane == 0) record_error(P.status, KVM_ERR_TIMEOUT, 51);
                            *abort_flag = 1;
                            break;
                        }
                        if (vvalid) {
                            const float qs = ldexpf(1.f, shift);
                            const uint32_t esz = type_bytes(P.q_type);
                            constexpr uint32_t DL = D / 4;  // dims per lane
#pragma unroll
                            for (uint32_t p8 = 0; p8 < DL; p8 += 8) {
                                const uint32_t dim0 = c4 * DL + p8, a = dim0 / 64, k0 = dim0 % 64;
                                uint32_t hw[4], lw[4];
#pragma unroll
                                for (int i = 0; i < 4; ++i)
                                    tc_split2(load_scalar(qp + (dim0 + 2 * i) * esz, P.q_type) * qs,
                                              load_scalar(qp + (dim0 + 2 * i + 1) * esz, P.q_type) * qs, hw[i], lw[i]);
                                uint8_t* base = qsm + a * kTcAtomBytes;
                                *reinterpret_cast<uint4*>(base + tc_sw128_offset(32 * q + g, k0)) =
                                    make_uint4(hw[0], hw[1], hw[2], hw[3]);
                                *reinterpret_cast<uint4*>(base + tc_sw128_offset(32 * q + 8 + g, k0)) =
                                    make_uint4(lw[0], lw[1], lw[2], lw[3]);
                            }
                        }
                        // Generic-proxy stores -> visible to the tensor cores (async proxy).
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mbar_arrive(qready);
                    }
                    if (!packed && set == 0) {
                        // Tile-0 query operand of this lane's vector (zeros past V),
                        // once the MMAs reading the previous one are done.
                        int ok = 1;
                        if (lane == 0) ok = mbar_wait(qfree, nq & 1);
                        ok = __shfl_sync(0xffffffffu, ok, 0);
                        ++nq;
                        if (!ok) {
                            if (lane == 0) record_error(P.status, KVM_ERR_TIMEOUT, 49);
                            *abort_flag = 1;
                            break;
                        }
                        bool lo_nz = false;
                        if constexpr (LM == 1) {
                            tc_fence_after();
                            lo_nz = tc_write_query_row<D>(qbase, qp, P.q_type, shift, vvalid);
                            tc_wait_st();
                            tc_fence_before();
                        } else {
                            // Row v of the shared-memory tile-0 operand: hi and lo parts,
                            // 16-byte swizzled pieces (zeros when !vvalid).
                            const float qs = ldexpf(1.f, shift);
                            const uint32_t esz = type_bytes(P.q_type);
#pragma unroll 1
                            for (uint32_t d8 = 0; d8 < D; d8 += 8) {
                                const uint32_t at = d8 / 64, k0 = d8 % 64;
                                uint32_t hw[4], lw[4];
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    float x0 = 0.f, x1 = 0.f;
                                    if (vvalid) {
                                        x0 = load_scalar(qp + (d8 + 2 * i) * esz, P.q_type) * qs;
                                        x1 = load_scalar(qp + (d8 + 2 * i + 1) * esz, P.q_type) * qs;
                                    }
                                    tc_split2(x0, x1, hw[i], lw[i]);
                                }
                                const uint32_t off = at * kTcAtomBytes + tc_sw128_offset(v, k0);
                                *reinterpret_cast<uint4*>(q0hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                                *reinterpret_cast<uint4*>(q0lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                                lo_nz |= ((lw[0] | lw[1] | lw[2] | lw[3]) & 0x7FFF7FFFu) != 0;
                            }
                            // Generic-proxy stores -> visible to the tensor cores (async proxy).
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        }
                        if (__any_sync(0xffffffffu, lo_nz) && lane == 0) atomicOr(const_cast<uint32_t*>(lo_any), 1u);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(qready);
                    }
                }
                for (uint32_t t = 0; t < ut; ++t, ++it) {
                    const uint32_t b = tb;
                    if (++tb == NB) {
                        tb = 0;
                        ++tround;
                    }
                    if (!mine) continue;  // the other tile-0 set's unit
                    uint64_t* full = packed ? &pfull[it & 1] : &tfull[b];
                    const uint32_t parity = packed ? (it >> 1) & 1 : ((it - b) / NB) & 1;
                    int ok = 1;
                    if (lane == 0) {
                        if (*abort_flag) ok = 0;
                        else if (!mbar_wait(full, parity)) {
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
                    const uint64_t tok0 = (uint64_t(un.j) * ut + t) * kTcTile;
                    const uint32_t tbase =
                        tmem + (uint32_t(32 * q) << 16) + (packed ? kTcColPacked + (it & 1) * kTcTile : b * kTcTile);
                    const bool fast = !MASK && !(P.softcap > 0.f) && tok0 + kTcTile <= P.tokens;
                    const bool last_tile = t + 1 == ut;
                    // Folds one 32-token chunk `ch` of this tile (n dots of this thread, or,
                    // off the fast path, the chunk reloaded from `slow_taddr` / group
                    // `slow_grp`) and closes the page if it ends there.
                    auto chunk = [&](const float* dots, int n, int ch, bool shared4, uint32_t slow_taddr,
                                     int slow_grp) {
                        if (fast) {
                            if (vvalid) {
                                if (n == 32) st.add_fast<32>(dots, cvt);
                                else st.add_fast<8>(dots, cvt);
                            }
                        } else {
                            const float2 ms =
                                shared4 ? tc_fold_slow<MASK, true>(sa, st.m, st.s, slow_taddr, slow_grp, tok0 + 32 * ch,
                                                                    c4, qinv, r, vvalid)
                                        : tc_fold_slow<MASK, false>(sa, st.m, st.s, slow_taddr, 0, tok0 + 32 * ch, c4,
                                                                     qinv, r, vvalid);
                            st.m = ms.x;
                            st.s = ms.y;
                        }
                        const bool ends =
                            small_pages ? ((ch + 1) & ((1 << cpp_log) - 1)) == 0 : (last_tile && ch == 3);
                        if (ends) {
                            if (shared4) {
                                // The page's four partial states of this vector -> one.
#pragma unroll
                                for (int o = 1; o <= 2; o <<= 1) {
                                    const float m2 = __shfl_xor_sync(0xffffffffu, st.m, o);
                                    const float s2 = __shfl_xor_sync(0xffffffffu, st.s, o);
                                    st.merge(m2, s2);
                                }
                            }
                            const uint32_t p = small_pages ? un.j * ppt + (uint32_t(ch) >> cpp_log) : un.j;
                            if (vvalid && (!shared4 || c4 == 0) && p < P.pages) lse_row[p] = st.lse_nat();
                            st = TcLse{};
                        }
                    };
                    uint32_t ra[32];
                    if (!packed) {
                        if constexpr (LM == 1) {
                            // Four 32-column chunks, each loaded while the one before is folded.
                            uint32_t rb[32];
                            tc_ld32(tbase, ra);
                            tc_wait_ld(ra);
#pragma unroll 1
                            for (int ch = 0; ch < 4; ch += 2) {
                                tc_ld32(tbase + (ch + 1) * 32, rb);
                                chunk(reinterpret_cast<const float*>(ra), 32, ch, false, tbase + ch * 32, 0);
                                tc_wait_ld_after(rb, st.m, st.s);
                                if (ch + 2 < 4) tc_ld32(tbase + (ch + 2) * 32, ra);
                                chunk(reinterpret_cast<const float*>(rb), 32, ch + 1, false, tbase + (ch + 1) * 32,
                                      0);
                                if (ch + 2 < 4) tc_wait_ld_after(ra, st.m, st.s);
                            }
                        } else {
                            // 128 registers per thread at 448 threads: one chunk at a time (the
                            // other tile-0 set and the packed warp cover the load latency).
#pragma unroll 1
                            for (int ch = 0; ch < 4; ++ch) {
                                tc_ld32(tbase + ch * 32, ra);
                                tc_wait_ld_after(ra, st.m, st.s);
                                chunk(reinterpret_cast<const float*>(ra), 32, ch, false, tbase + ch * 32, 0);
                            }
                        }
                    } else {
                        // 16x256b loads of 64 columns; hi (lane g) + lo (lane g+8) per dot.
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
                            tc_ld16x256x8(tbase + hh * 64, ra);
                            tc_wait_ld_after(ra, st.m, st.s);
#pragma unroll
                            for (int grp = 0; grp < 2; ++grp) {
                                float dots[8];
#pragma unroll
                                for (int i = 0; i < 4; ++i)
#pragma unroll
                                    for (int jj = 0; jj < 2; ++jj)
                                        dots[2 * i + jj] = __uint_as_float(ra[4 * (4 * grp + i) + jj]) +
                                                           __uint_as_float(ra[4 * (4 * grp + i) + 2 + jj]);
                                chunk(dots, 8, 2 * hh + grp, true, tbase + hh * 64, grp);
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(packed ? &pempty[it & 1] : &tempty[b]);
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
