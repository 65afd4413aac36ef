// Per-token page mass, first pass, for quantised keys (q8_0 / q4_0) on the
// integer tensor cores: the page log-sum-exp of up to 8 query vectors that
// share a KV head.
//
// The K codes enter mma.sync m16n8k32 (s8 x s8 -> s32; q4_0 nibbles as u8)
// exactly as they are stored, so no key element is ever converted. The query
// vectors are the A operand as two int8 digits per element: each 32-element
// block of a vector is scaled by its own power of two so that its largest
// magnitude lies in [2^13, 2^15), rounded to an integer q and split as
// q = 256*hi + lo (rows 0..7: hi of vectors 0..7, rows 8..15: lo). The block's
// dots are exact integers; the mma's C operand starts at the bit pattern of
// M = 1.5 * 2^(23+k) (k = the row's power of two; q4_0 also subtracts
// 8 * the row's digit sum for the nibble offset), so the s32 result read as a
// float is M + dot * 2^k exactly and one FADD of M recovers the scaled dot.
// Each block's dot is then scaled by the token's fp16 block scale in fp32.
// The query keeps 15-16 significant bits per block (relative error <= 2^-15 of
// the block's largest element), within the 1e-3 relative bound on page scores.
//
// Instruction stream of the consumer warps:
//  * the KV-head count, block geometry and row bytes are template constants,
//    each warp serves one KV head and a fixed set of octets (8 tokens), and
//    its shared-memory addresses advance by a constant per octet;
//  * blocks whose codes start 2 bytes off a 32-bit word (every other block:
//    the 34- / 18-byte blocks alternate) are read as the aligned words that
//    hold codes 2..29 (q8_0; nibble bytes 2..13 for q4_0) plus one word
//    spliced (byte permute) from the halves of the block's first and last
//    words: lane c holds the aligned words 1+c and 5+c, lane 3's second word
//    is {30, 31, 0, 1}. The mma's k index follows the same lane-dependent
//    order for the query digits, so every element is counted once;
//  * each chunk arrives as one tiled TMA box per group of KV heads whose
//    inner extent runs 16 bytes past the group's row bytes into zero-filled
//    out-of-bounds columns, so token rows land in shared memory at a stride
//    of an odd number of 16-byte units: the 8 tokens of an octet start in 8
//    different bank groups and every 32-bit load is conflict-free;
//  * a chunk that is fully visible, unmasked and without softcap takes a
//    branchless online (max, sum) update per token pair; everything else
//    takes the general per-token path.
#pragma once
#include "page_mass_mma.cuh"

namespace kvmb {

// Element (0..31) of a block held in position i (0..7) of lane c's B
// fragment for block kk: positions 0..3 form k-step 0, 4..7 k-step 1.
template <int KT>
__host__ __device__ constexpr int q_dim(int kk, int c, int i) {
    const bool aligned = (kk & 1) != 0;  // codes start on a word boundary
    if constexpr (KT == KVM_Q8_0) {
        if (aligned) return i < 4 ? 4 * c + i : 16 + 4 * c + (i - 4);
        if (i < 4) return 4 * c + 2 + i;
        if (c < 3) return 4 * c + 18 + (i - 4);
        return (i - 4) < 2 ? 30 + (i - 4) : (i - 4) - 2;
    } else {  // q4_0: byte j holds elements j (low nibble) and 16 + j (high nibble)
        const int j = i & 3;
        int byte;
        if (aligned) byte = 4 * c + j;
        else if (c < 3) byte = 4 * c + 2 + j;
        else byte = j < 2 ? 14 + j : j - 2;
        return i < 4 ? byte : 16 + byte;
    }
}

// B fragments of block kk for this lane from its token's row, as the mma
// takes them: b[0] = positions 0..3 (k 4c..4c+3), b[1] = positions 4..7
// (k 16+4c..16+4c+3); q8_0 codes as s8, q4_0 nibbles as u8 (0..15).
template <int KT, int kk>
__device__ __forceinline__ void q_b_frag(const uint8_t* row, int c, uint32_t splice, uint32_t* b) {
    constexpr int kBlock = KT == KVM_Q8_0 ? 34 : 18;
    const uint8_t* blk = row + kBlock * kk;
    if constexpr (KT == KVM_Q8_0) {
        if constexpr (kk & 1) {
            b[0] = *reinterpret_cast<const uint32_t*>(blk + 2 + 4 * c);
            b[1] = *reinterpret_cast<const uint32_t*>(blk + 18 + 4 * c);
        } else {
            b[0] = *reinterpret_cast<const uint32_t*>(blk + 4 + 4 * c);
            const uint32_t r = *reinterpret_cast<const uint32_t*>(blk + 20 + 4 * c);
            const uint32_t h = *reinterpret_cast<const uint32_t*>(blk);
            b[1] = __byte_perm(r, h, splice);
        }
    } else {
        uint32_t w;
        if constexpr (kk & 1) {
            w = *reinterpret_cast<const uint32_t*>(blk + 2 + 4 * c);
        } else {
            const uint32_t r = *reinterpret_cast<const uint32_t*>(blk + 4 + 4 * c);
            const uint32_t h = *reinterpret_cast<const uint32_t*>(blk);
            w = __byte_perm(r, h, splice);
        }
        b[0] = w & 0x0F0F0F0Fu;
        b[1] = (w >> 4) & 0x0F0F0F0Fu;
    }
}

// d (s32) = a (16 x 32 s8, row-major) . b (32 x 8, s8 or u8) + c.
template <int KT>
__device__ __forceinline__ void imma_16832(int* d, const uint32_t* a, const uint32_t* b, const int4& c) {
    if constexpr (KT == KVM_Q8_0) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(c.x), "r"(c.y), "r"(c.z),
              "r"(c.w));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(c.x), "r"(c.y), "r"(c.z),
              "r"(c.w));
    }
}

// Power of two of one query block: |q| * 2^s <= 32639 (two int8 digits),
// with the largest element at 2^14 or above when that fits, else 2^13.
__device__ __forceinline__ int q_block_shift(float amax) {
    if (!(amax > 0.f)) return 0;
    const int e = int((__float_as_uint(amax) >> 23) & 255) - 127;  // floor(log2(amax)) for normals
    int sh = 14 - e;
    if (ldexpf(amax, sh) > 32639.f) sh = 13 - e;
    return min(140, max(-96, sh));
}

constexpr int kQThreads = kLseConsumerWarps * 32;  // no producer warp: 16 warps per SM at 2 CTAs
// Per-page merge buffers: warps are at most (stages) chunks apart, so a buffer
// is reused only after the page that last used it has been merged.
constexpr int kQPageBufs = kMmaMaxStages + 2;
constexpr int kQMaxGroups = 8;      // head groups, each with its own ring
constexpr int kQCounterBytes = 1280;  // barriers and counters

// Shared memory of page_lse_q_kernel beyond its S ring stages.
__host__ __device__ constexpr size_t q_smem_extra() {
    return kQCounterBytes +                                       // barriers and counters
           kLseConsumerWarps * 8 * 8 * 8 * sizeof(float) +        // per-warp mma C / magic values [kk][g][8]
           kLseConsumerWarps * 2 * 64 * sizeof(float) +           // per-warp scale tables (double buffered)
           2 * kQPageBufs * kLseConsumerWarps * 8 * sizeof(float) +  // per-page merge buffers
           16;                                                    // abort flag
}

// KK = head_dim / 32 blocks per row; KVH = KV heads (1, 2, 4 or 8).
//
// Ring protocol: thread 0 fills the first S stages; afterwards the warp that
// releases a stage last (a shared-memory count of releases per stage) issues
// the stage's next chunk, S chunks ahead. There is no producer warp, so the
// SM holds 16 warps of two CTAs and each thread may use 128 registers.
template <int KT, int KK, int KVH, bool MASK>
__global__ void __launch_bounds__(kQThreads, 2) page_lse_q_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                  const LseParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NW = kLseConsumerWarps;
    constexpr int WPH = NW / KVH;  // warps per KV head
    constexpr int kBlock = KT == KVM_Q8_0 ? 34 : 18;
    constexpr uint32_t kRow = uint32_t(kBlock * KK);
    static_assert(NW % KVH == 0 && (NW & (NW - 1)) == 0, "warps per KV head");
    const uint32_t S = P.stages;
    const uint32_t NG = P.groups_tma;  // head groups: one ring of S stages each
    uint8_t* stages = smem;            // [NG][S] stages of stage_stride bytes
    // After the rings (128-byte aligned): barriers and counters, then 16-byte
    // aligned float arrays.
    uint8_t* extra = smem + NG * S * P.stage_stride;
    uint64_t* full = reinterpret_cast<uint64_t*>(extra);  // [kQMaxGroups][kMmaMaxStages]
    uint32_t* released = reinterpret_cast<uint32_t*>(full + kQMaxGroups * kMmaMaxStages);
    uint32_t* issued = released + kQMaxGroups * kMmaMaxStages;
    uint32_t* arrived = issued + kQMaxGroups * kMmaMaxStages;  // [kQPageBufs]
    static_assert(kQMaxGroups * kMmaMaxStages * 16 + kQPageBufs * 4 <= kQCounterBytes, "counter area");
    float* cstart = reinterpret_cast<float*>(extra + kQCounterBytes);  // [NW][8][8][8]
    float* tables = cstart + NW * 8 * 8 * 8;                        // [NW][2][8][8]
    float* red_m = tables + NW * 2 * 64;                            // [kQPageBufs][NW][8]
    float* red_s = red_m + kQPageBufs * NW * 8;
    int* abort_flag = reinterpret_cast<int*>(red_s + kQPageBufs * NW * 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t units = P.layers * P.pages;
    const uint32_t per_cta = (units + gridDim.x - 1) / gridDim.x;
    const uint32_t unit_begin = min(units, blockIdx.x * per_cta), unit_end = min(units, unit_begin + per_cta);
    const uint32_t total = (unit_end - unit_begin) * P.chunks;  // chunks of this CTA
    const uint64_t policy = policy_evict_first();

    // Chunk ch of page unit_begin + u of head group gi into its stage s: one
    // tiled box, tokens x (the group's row bytes [+ zero-filled pad columns]).
    auto issue = [&](uint32_t gi, uint32_t s, uint32_t u, uint32_t ch) {
        const uint32_t unit = unit_begin + u;
        const uint32_t l = unit / P.pages, p = unit - l * P.pages;
        const int tok = int(p * P.page_tokens + ch * P.tpc);
        const uint32_t at = gi * kMmaMaxStages + s;
        mbar_arrive_expect_tx(&full[at], P.chunk_bytes);
        tma_load_4d(stages + (gi * S + s) * P.stage_stride, &kmap, 0, int(gi), tok, int(l), &full[at], policy);
        ++issued[at];
    };

    if (tid == 0) {
        for (uint32_t gi = 0; gi < NG; ++gi)
            for (uint32_t s = 0; s < S; ++s) {
                mbar_init(&full[gi * kMmaMaxStages + s], 1);
                released[gi * kMmaMaxStages + s] = 0;
                issued[gi * kMmaMaxStages + s] = 0;
            }
        for (int b = 0; b < kQPageBufs; ++b) arrived[b] = 0;
        *abort_flag = 0;
        mbar_fence_init();
        for (uint32_t gi = 0; gi < NG; ++gi)
            for (uint32_t i = 0; i < S && i < total; ++i) issue(gi, i, i / P.chunks, i % P.chunks);
    }
    __syncthreads();

    // lane = g*4 + c; warp serves KV head kvh and octets wsub, wsub + WPH, ... of each chunk.
    const int g = lane >> 2, c = lane & 3;
    const uint32_t kvh = uint32_t(warp) % KVH, wsub = uint32_t(warp) / KVH;
    const uint32_t splice = c == 3 ? 0x7610u : 0x3210u;
    const bool gvalid = g < int(P.nv);
    const uint32_t myr = gvalid ? (P.v0 + g) / P.group : 0;
    const uint32_t slot = P.slot_stride;
    const uint32_t nj = P.tpc / (8 * WPH);
    const uint32_t gi = kvh / P.hpg;                 // this warp's head group (ring)
    const uint32_t gwarps = WPH * P.hpg;             // warps that release each stage of the ring
    uint8_t* ring = stages + gi * S * P.stage_stride;
    uint64_t* gfull = full + gi * kMmaMaxStages;
    uint32_t* greleased = released + gi * kMmaMaxStages;
    const uint32_t head_off = (kvh % P.hpg) * kRow;
    const uint32_t lane_b = (wsub * 8 + g) * slot + head_off;             // code row: token g of the octet
    const uint32_t tab_row = (wsub * 8 + (lane & 7)) * slot + head_off;  // scale-table fill: token lane % 8
    const uint32_t jstep = WPH * 8 * slot;
    float* tab = tables + warp * 2 * 64;
    float* cw = cstart + warp * 8 * 8 * 8;

    uint32_t qa[KK][4];  // A fragments: int8 digits [block][a0..a3]
    const float sl2 = P.scale * kLog2e;
    uint32_t s = 0, phase = 0, pb = 0, qlayer = 0xffffffffu, tb = 0;
    // Refill cursor: the chunk S ahead of the one being consumed.
    uint32_t r_idx = S, r_u = S / P.chunks, r_ch = S % P.chunks;
    for (uint32_t unit = unit_begin; unit < unit_end; ++unit) {
        const uint32_t l = unit / P.pages, p = unit - l * P.pages;
        if (l != qlayer) {
            qlayer = l;
            const uint32_t vg = P.v0 + g, r = gvalid ? vg / P.group : 0, gg = gvalid ? vg % P.group : 0;
            const uint8_t* qp = P.q + l * P.q_layer + r * P.q_row + (kvh * P.group + gg) * P.q_head;
            const uint32_t esz = type_bytes(P.q_type);
            __syncwarp();
#pragma unroll
            for (int kk = 0; kk < KK; ++kk) {
                float qv[8];
                float amax = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int dim = kk * 32 + q_dim<KT>(kk, c, i);
                    qv[i] = gvalid ? load_scalar(qp + dim * esz, P.q_type) : 0.f;
                    amax = fmaxf(amax, fabsf(qv[i]));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                const int sh = q_block_shift(amax);
                uint32_t hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
                int dsum_hi = 0, dsum_lo = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int qi = __float2int_rn(ldexpf(qv[i], sh));  // |qi| <= 32639
                    const int h = (qi + 128) >> 8, lw = qi - (h << 8);  // h, lw in [-128, 127]
                    hi[i >> 2] |= uint32_t(h & 255) << (8 * (i & 3));
                    lo[i >> 2] |= uint32_t(lw & 255) << (8 * (i & 3));
                    dsum_hi += h;
                    dsum_lo += lw;
                }
                qa[kk][0] = hi[0];  // row g,   k 4c..4c+3
                qa[kk][1] = lo[0];  // row g+8, k 4c..4c+3
                qa[kk][2] = hi[1];  // row g,   k 16+4c..16+4c+3
                qa[kk][3] = lo[1];  // row g+8, k 16+4c..16+4c+3
                // C start (bits of M, minus 8 * digit sum for q4_0) and M of rows g / g+8.
                dsum_hi += __shfl_xor_sync(0xffffffffu, dsum_hi, 1);
                dsum_lo += __shfl_xor_sync(0xffffffffu, dsum_lo, 1);
                dsum_hi += __shfl_xor_sync(0xffffffffu, dsum_hi, 2);
                dsum_lo += __shfl_xor_sync(0xffffffffu, dsum_lo, 2);
                if (c == 0) {
                    const float mh = ldexpf(12582912.f, 8 - sh), ml = ldexpf(12582912.f, -sh);  // 1.5 * 2^(23+k)
                    const int off_h = KT == KVM_Q4_0 ? -8 * dsum_hi : 0, off_l = KT == KVM_Q4_0 ? -8 * dsum_lo : 0;
                    const int ch_ = int(__float_as_uint(mh)) + off_h, cl_ = int(__float_as_uint(ml)) + off_l;
                    *reinterpret_cast<int4*>(cw + (kk * 8 + g) * 8) = make_int4(ch_, ch_, cl_, cl_);
                    *reinterpret_cast<float4*>(cw + (kk * 8 + g) * 8 + 4) = make_float4(mh, ml, 0.f, 0.f);
                }
            }
            __syncwarp();
        }
        float m = -INFINITY, ssum = 0.f;
        const uint64_t tok0 = uint64_t(p) * P.page_tokens;

        for (uint32_t ch = 0; ch < P.chunks; ++ch) {
            bool ok = !*reinterpret_cast<volatile int*>(abort_flag);
            if (ok && !mbar_wait(&gfull[s], phase)) {
                record_error(P.status, KVM_ERR_TIMEOUT, 6);
                *reinterpret_cast<volatile int*>(abort_flag) = 1;
                ok = false;
            }
            if (ok) {
                const uint8_t* stage = ring + s * P.stage_stride;
                const uint64_t ctok = tok0 + uint64_t(ch) * P.tpc;
                const bool fast = !MASK && P.softcap <= 0.f && ctok + P.tpc <= P.tokens;
                for (uint32_t j = 0; j < nj; ++j) {
                    const uint8_t* brow = stage + lane_b + j * jstep;
                    // Block scales of the octet's 8 tokens as floats: tab[kk][token].
                    {
                        const uint8_t* trow = stage + tab_row + j * jstep;
                        float* t = tab + tb * 64;
#pragma unroll
                        for (int b = 0; b < (KK + 3) / 4; ++b) {
                            const int kk = (lane >> 3) + 4 * b;
                            if (kk < KK)
                                t[kk * 8 + (lane & 7)] =
                                    __half2float(*reinterpret_cast<const __half*>(trow + kBlock * kk));
                        }
                        __syncwarp();
                    }
                    const float* tsc = tab + tb * 64 + 2 * c;
                    tb ^= 1;
                    float acc[2] = {0.f, 0.f};  // tokens 2c, 2c+1 of the octet for vector g
                    unroll_kk<KK>([&](auto kkc) {
                        constexpr int kk = decltype(kkc)::value;
                        uint32_t b[2];
                        q_b_frag<KT, kk>(brow, c, splice, b);
                        const int4 cc = *reinterpret_cast<const int4*>(cw + (kk * 8 + g) * 8);
                        int dd[4];
                        imma_16832<KT>(dd, qa[kk], b, cc);
                        float mh, ml;
                        if constexpr (KT == KVM_Q8_0) {
                            mh = __int_as_float(cc.x);
                            ml = __int_as_float(cc.z);
                        } else {
                            const float2 mm = *reinterpret_cast<const float2*>(cw + (kk * 8 + g) * 8 + 4);
                            mh = mm.x;
                            ml = mm.y;
                        }
                        const float2 d = *reinterpret_cast<const float2*>(tsc + kk * 8);  // tokens 2c, 2c+1
                        acc[0] = fmaf(__int_as_float(dd[0]) - mh, d.x, acc[0]);
                        acc[1] = fmaf(__int_as_float(dd[1]) - mh, d.y, acc[1]);
                        acc[0] = fmaf(__int_as_float(dd[2]) - ml, d.x, acc[0]);
                        acc[1] = fmaf(__int_as_float(dd[3]) - ml, d.y, acc[1]);
                    });
                    if (fast) {
                        const float x0 = acc[0] * sl2, x1 = acc[1] * sl2;
                        const float mn = fmaxf(m, fmaxf(x0, x1));
                        ssum = fmaf(ssum, fast_exp2(m - mn), fast_exp2(x0 - mn) + fast_exp2(x1 - mn));
                        m = mn;
                    } else {
                        const uint64_t t0 = ctok + (wsub + j * WPH) * 8 + 2 * c;
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) {
                            const float dot = acc[jj];
                            float x;
                            if (P.softcap > 0.f) x = P.softcap * tanhf(dot * P.scale / P.softcap) * kLog2e;
                            else x = dot * P.scale * kLog2e;
                            const uint64_t t = t0 + jj;
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
            }
            // Release the stage; the last of the group's warps to release it refills it S chunks ahead.
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                const uint32_t before = atomicAdd(&greleased[s], 1u);
                if ((before & (gwarps - 1)) == gwarps - 1 && r_idx < total &&
                    !*reinterpret_cast<volatile int*>(abort_flag)) {
                    __threadfence_block();
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(gi, s, r_u, r_ch);
                }
            }
            ++r_idx;
            if (++r_ch == P.chunks) {
                r_ch = 0;
                ++r_u;
            }
            if (++s == S) {
                s = 0;
                phase ^= 1;
            }
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
        // The last warp to finish the page merges its KV heads' warps (no CTA barrier).
        if (c == 0) {
            red_m[(pb * NW + warp) * 8 + g] = m;
            red_s[(pb * NW + warp) * 8 + g] = ssum;
        }
        __syncwarp();
        uint32_t before = 0;
        if (lane == 0) {
            __threadfence_block();
            before = atomicAdd(&arrived[pb], 1u);
        }
        if ((__shfl_sync(0xffffffffu, before, 0) & (NW - 1)) == NW - 1) {
            __threadfence_block();
            for (int idx = lane; idx < KVH * 8; idx += 32) {
                const uint32_t h_kv = idx / 8, v = idx % 8;
                float M = -INFINITY;
#pragma unroll
                for (int w2 = 0; w2 < WPH; ++w2) M = fmaxf(M, red_m[(pb * NW + h_kv + w2 * KVH) * 8 + v]);
                float Sx = 0.f;
                if (M != -INFINITY)
#pragma unroll
                    for (int w2 = 0; w2 < WPH; ++w2) {
                        const int at = (pb * NW + h_kv + w2 * KVH) * 8 + v;
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
        if (++pb == kQPageBufs) pb = 0;
    }

    // After a timeout no copy may still be landing in this CTA's shared memory when it exits.
    __syncthreads();
    if (tid == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
        for (uint32_t gr = 0; gr < NG; ++gr)
            for (uint32_t st = 0; st < S; ++st) {
                const uint32_t at = gr * kMmaMaxStages + st;
                if (issued[at] && !mbar_wait(&full[at], (issued[at] - 1) & 1))
                    record_error(P.status, KVM_ERR_TIMEOUT, 5);
            }
    }
}

}  // namespace kvmb
