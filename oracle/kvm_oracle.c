/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the reference algorithms on the history-recall path.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load
 * this file's library, and only as the checker; the product (kvmem_b200) never
 * links or calls it.
 *
 * Pinned against: the reference's own known-answer tests
 * (kvmem/tests/graph_recall_test.cpp:22-106,242-253 and
 * kvmem/tests/kvmem_store_test.cpp:1085-1160, restated as fixtures under
 * tests/golden/) and the reference's CPU selection library compiled from its
 * own sources into oracle/_ref/ (page_softmax_scores, query_score_frame,
 * pick_scored_blocks, plan_residency). The per-token page mass has no
 * reference golden vector (its only check is a runtime FP64 self-test that
 * needs a model), so that part is pinned against the reference's FP64 oracle
 * formula restated here plus hand-computed known answers.
 *
 * Every function names the reference file:line whose behaviour it follows.
 * All arithmetic is FP64 except where the reference itself rounds (fp16
 * operand boundary, f32 mean = sum * (1/count)).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KVO_OK 0
#define KVO_ERR_INVALID 1 /* std::invalid_argument in the reference */
#define KVO_ERR_RUNTIME 2 /* std::runtime_error in the reference */

/* Scalar / block type codes: the same numbering as include/kvm_recall.h. */
enum { KVO_F32 = 0, KVO_F16 = 1, KVO_BF16 = 2, KVO_Q8_0 = 3, KVO_Q4_0 = 4, KVO_Q5_0 = 5 };

/* IEEE binary16 -> double, exact (every half is representable). */
double kvo_half_to_double(uint16_t h) {
    const int sign = (h >> 15) & 1, exp = (h >> 10) & 31, man = h & 1023;
    double v;
    if (exp == 0) v = ldexp((double)man, -24);
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = ldexp((double)(man | 1024), exp - 25);
    return sign ? -v : v;
}

static double bf16_to_double(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return (double)f;
}

/* Bytes of one D-element row of `type` (ggml row size; blocks of 32). */
uint64_t kvo_row_bytes(int type, uint32_t dim) {
    switch (type) {
    case KVO_F32: return 4ull * dim;
    case KVO_F16: case KVO_BF16: return 2ull * dim;
    case KVO_Q8_0: return (uint64_t)(dim / 32) * 34;
    case KVO_Q4_0: return (uint64_t)(dim / 32) * 18;
    case KVO_Q5_0: return (uint64_t)(dim / 32) * 22;
    }
    return 0;
}

/*
 * Decode element d of one row, as the reference's device `key()`/`scalar()`
 * (src/adapter/llama-kvmem-attention-cuda.cu:35-58) and ggml's to_float agree:
 *   q8_0 {half d; int8 qs[32]}            -> qs[i] * d
 *   q4_0 {half d; uint8 qs[16]}           -> ((qs[i%16] >> (i<16?0:4)) & 15) - 8) * d
 *   q5_0 {half d; uint8 qh[4]; uint8 qs[16]} -> (low | high<<4) - 16) * d
 * The product with the fp16 scale is formed in FP32 in the reference kernel;
 * every such product of an int in [-128,127] and a half is exact in FP32, so
 * FP64 here gives the same value.
 */
double kvo_decode(int type, const uint8_t* row, uint32_t d) {
    const uint32_t at = d % 32;
    switch (type) {
    case KVO_F32: { float f; memcpy(&f, row + 4ull * d, 4); return (double)f; }
    case KVO_F16: { uint16_t h; memcpy(&h, row + 2ull * d, 2); return kvo_half_to_double(h); }
    case KVO_BF16: { uint16_t h; memcpy(&h, row + 2ull * d, 2); return bf16_to_double(h); }
    case KVO_Q8_0: {
        const uint8_t* b = row + (d / 32) * 34ull;
        uint16_t h; memcpy(&h, b, 2);
        return (double)(int8_t)b[2 + at] * kvo_half_to_double(h);
    }
    case KVO_Q4_0: {
        const uint8_t* b = row + (d / 32) * 18ull;
        uint16_t h; memcpy(&h, b, 2);
        const int code = (b[2 + at % 16] >> (at < 16 ? 0 : 4)) & 15;
        return (double)(code - 8) * kvo_half_to_double(h);
    }
    case KVO_Q5_0: {
        const uint8_t* b = row + (d / 32) * 22ull;
        uint16_t h; memcpy(&h, b, 2);
        const int low = (b[6 + at % 16] >> (at < 16 ? 0 : 4)) & 15;
        const int high = (b[2 + at / 8] >> (at % 8)) & 1;
        return (double)((low | (high << 4)) - 16) * kvo_half_to_double(h);
    }
    }
    return NAN;
}

/*
 * Mean-K producer — restates the reference's meank_add_f32/_f16/_bf16 kernels
 * (src/adapter/llama-kvmem-stagein.cu:270-316: acc[d] += K[token][head][dim]
 * in token order, one f32 add each) applied per page into a per-page table:
 * sums[l][page][kv_heads*dim] += value, counts[page] += tokens added, for the
 * tokens [tok0, tok0+n) of layers [0, layers). Values are the f32 reading of
 * the key element (the reference's key(), llama-kvmem-attention-cuda.cu:39-58:
 * codes times the fp16 block scale as one f32 product for q8_0/q4_0/q5_0).
 * Returns 0, or 1 for a range outside the table.
 */
static float half_to_float(uint16_t h) { return (float)kvo_half_to_double(h); }

static float key_elem_f32(int type, const uint8_t* row, uint32_t d) {
    const uint32_t at = d % 32;
    switch (type) {
    case KVO_F32: { float f; memcpy(&f, row + 4ull * d, 4); return f; }
    case KVO_F16: { uint16_t h; memcpy(&h, row + 2ull * d, 2); return half_to_float(h); }
    case KVO_BF16: { uint16_t h; memcpy(&h, row + 2ull * d, 2); return (float)bf16_to_double(h); }
    case KVO_Q8_0: {
        const uint8_t* b = row + (d / 32) * 34ull;
        uint16_t h; memcpy(&h, b, 2);
        const float code = (float)(int8_t)b[2 + at];
        return code * half_to_float(h);
    }
    case KVO_Q4_0: {
        const uint8_t* b = row + (d / 32) * 18ull;
        uint16_t h; memcpy(&h, b, 2);
        const float code = (float)(((b[2 + at % 16] >> (at < 16 ? 0 : 4)) & 15) - 8);
        return code * half_to_float(h);
    }
    case KVO_Q5_0: {
        const uint8_t* b = row + (d / 32) * 22ull;
        uint16_t h; memcpy(&h, b, 2);
        const int low = (b[6 + at % 16] >> (at < 16 ? 0 : 4)) & 15;
        const int high = (b[2 + at / 8] >> (at % 8)) & 1;
        const float code = (float)((low | (high << 4)) - 16);
        return code * half_to_float(h);
    }
    }
    return NAN;
}

int kvo_meank_add(float* sums, uint32_t* counts, uint32_t pages, const uint8_t* k, int k_type, uint64_t k_layer,
                  uint64_t k_token, uint64_t k_head, uint32_t layers, uint32_t kv_heads, uint32_t dim, uint64_t tok0,
                  uint32_t n, uint32_t page_tokens) {
    if (n == 0) return 0;
    if ((tok0 + n - 1) / page_tokens >= pages) return 1;
    const uint64_t n_embd = (uint64_t)kv_heads * dim;
    for (uint64_t t = tok0; t < tok0 + n; ++t) counts[t / page_tokens] += 1;
    for (uint32_t l = 0; l < layers; ++l)
        for (uint64_t e = 0; e < n_embd; ++e) {
            const uint32_t h = (uint32_t)(e / dim), d = (uint32_t)(e % dim);
            for (uint64_t t = tok0; t < tok0 + n; ++t) {
                float* s = sums + ((uint64_t)l * pages + t / page_tokens) * n_embd + e;
                *s = *s + key_elem_f32(k_type, k + l * k_layer + t * k_token + h * k_head, d);
            }
        }
    return 0;
}

/*
 * One-hop score propagation — restates propagate_query_scores
 * (kvmem/src/host/graph_recall.cpp:494-551, span_coefficient :234-246) over a
 * graph given as arrays: rows (source position, samples, edges
 * [edge_begin, edge_begin + edge_count)), edges (target position, mass), and
 * optional message spans. Sources are visited in frame order (the reference
 * walks an unordered_map, so its own summation order is unspecified).
 * Returns 0, 1 for an invalid input (the reference's invalid_argument).
 */
static double span_coef(uint64_t a, uint64_t b, uint32_t block, const uint64_t* sb, const uint64_t* se,
                        const uint8_t* sk, uint32_t ns, int has_messages, double cross) {
    if (!has_messages) return 1;
    const uint64_t begin = a < b ? a : b, end = (a > b ? a : b) + block;
    for (uint32_t i = 0; i < ns; ++i)
        if (sb[i] <= begin && end <= se[i]) return 1;
    for (uint32_t i = 0; i < ns; ++i)
        if ((begin < sb[i] && sb[i] < end) || (sk[i] && begin < se[i] && se[i] < end)) return cross;
    return 1;
}

static int64_t frame_index(const uint64_t* starts, const uint8_t* allowed, uint32_t n, uint64_t pos) {
    for (uint32_t i = 0; i < n; ++i)
        if (starts[i] == pos) return allowed[i] ? (int64_t)i : -1;
    return -1;
}

int kvo_propagate_scores(const double* raw, uint32_t n, const uint64_t* starts, const uint8_t* transport_mask,
                         uint64_t frame_accepted, uint32_t block, uint64_t graph_accepted, uint64_t completed,
                         const uint64_t* row_source, const uint64_t* row_samples, const uint32_t* row_begin,
                         const uint32_t* row_count, uint32_t nrows, const uint64_t* edge_target,
                         const double* edge_mass, const uint64_t* span_begin, const uint64_t* span_end,
                         const uint8_t* span_end_known, uint32_t nspans, int has_messages, double alpha,
                         double cross, double* out) {
    if (!(isfinite(alpha) && alpha >= 0 && alpha <= 1) || !(isfinite(cross) && cross >= 0 && cross <= 1)) return 1;
    if (!block || graph_accepted != frame_accepted) return 1;
    double total = 0;
    uint32_t nallowed = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (!isfinite(raw[i]) || starts[i] % block) return 1;
        for (uint32_t j = 0; j < i; ++j)
            if (starts[j] == starts[i]) return 1;
        if (transport_mask[i]) {
            ++nallowed;
            total += raw[i] > 0 ? raw[i] : 0;
        }
    }
    if (!isfinite(total)) return 1;
    for (uint32_t i = 0; i < n; ++i) out[i] = raw[i];
    if (nallowed <= 1 || total == 0 || alpha == 0) return 0;
    double* seed = (double*)calloc(n, sizeof(double));
    if (!seed) return 2;
    for (uint32_t i = 0; i < n; ++i)
        if (transport_mask[i]) seed[i] = (raw[i] > 0 ? raw[i] : 0) / total;
    for (uint32_t i = 0; i < n; ++i) {
        if (!transport_mask[i]) continue;
        const uint64_t src = starts[i];
        for (int dir = -1; dir <= 1; dir += 2) {
            if (dir < 0 && src < block) continue;
            if (dir > 0 && src > UINT64_MAX - block) continue;
            const uint64_t tgt = dir < 0 ? src - block : src + block;
            const int64_t j = frame_index(starts, transport_mask, n, tgt);
            if (j < 0) continue;
            const double w = alpha * .25 *
                             span_coef(src, tgt, block, span_begin, span_end, span_end_known, nspans, has_messages, cross);
            const double delta = total * seed[i] * w;
            out[i] -= delta;
            out[j] += delta;
        }
    }
    for (uint32_t r = 0; r < nrows; ++r) {
        const int64_t i = frame_index(starts, transport_mask, n, row_source[r]);
        if (i < 0 || !row_samples[r] || row_source[r] + block > completed) continue;
        double den = 0;
        for (uint32_t e = row_begin[r]; e < row_begin[r] + row_count[r]; ++e) {
            if (!(isfinite(edge_mass[e]) && edge_mass[e] >= 0)) { free(seed); return 1; }
            if (edge_target[e] != row_source[r] && frame_index(starts, transport_mask, n, edge_target[e]) >= 0)
                den += edge_mass[e];
        }
        if (!den) continue;
        for (uint32_t e = row_begin[r]; e < row_begin[r] + row_count[r]; ++e) {
            const int64_t j = frame_index(starts, transport_mask, n, edge_target[e]);
            if (j < 0 || edge_target[e] == row_source[r]) continue;
            const double delta = total * seed[i] * (alpha * .5 * edge_mass[e] / den);
            out[i] -= delta;
            out[j] += delta;
        }
    }
    free(seed);
    for (uint32_t i = 0; i < n; ++i) {
        const double residual = raw[i] < 0 ? raw[i] : 0;
        if (!isfinite(out[i]) || out[i] < residual - 1e-12 * (total > 1 ? total : 1)) return 2;
        if (out[i] < residual) out[i] = residual;
    }
    return 0;
}

/*
 * LRFU preview — restates LrfuHistory::preview (kvmem/include/kvmem/lrfu.hpp:57-79):
 * threshold = the value of rank min(n-1, floor((1-fraction)*n)) in ascending
 * order (-inf when fraction == 1); out[i] = lambda*prev[i] (0 past n_prev) +
 * (score >= threshold ? score : min(score, 0)). Returns 1 for a non-finite
 * score or an invalid lambda / fraction.
 */
static int cmp_double(const void* a, const void* b) {
    const double x = *(const double*)a, y = *(const double*)b;
    return x < y ? -1 : x > y;
}

int kvo_lrfu_preview(const double* scores, uint32_t n, const double* prev, uint32_t n_prev, double lambda,
                     double fraction, double* out) {
    if (!(isfinite(lambda) && lambda >= 0 && lambda <= 1) || !(isfinite(fraction) && fraction > 0 && fraction <= 1))
        return 1;
    for (uint32_t i = 0; i < n; ++i)
        if (!isfinite(scores[i])) return 1;
    if (!n) return 0;
    double threshold = -INFINITY;
    if (fraction < 1) {
        double* ranked = (double*)malloc(n * sizeof(double));
        if (!ranked) return 2;
        memcpy(ranked, scores, n * sizeof(double));
        qsort(ranked, n, sizeof(double), cmp_double);
        size_t rank = (size_t)((1 - fraction) * n);
        if (rank > n - 1) rank = n - 1;
        threshold = ranked[rank];
        free(ranked);
    }
    for (uint32_t i = 0; i < n; ++i)
        out[i] = lambda * (i < n_prev ? prev[i] : 0) +
                 (scores[i] >= threshold ? scores[i] : (scores[i] < 0 ? scores[i] : 0));
    return 0;
}

/*
 * Raw-K restore transform — restates the reference's stage-in kernels
 * (src/adapter/llama-kvmem-stagein.cu: dequant_q8_0 / dequant_q4_0 :134-160,
 * rope_neox_kernel :162-180, fwht_kernel :104-130 with scale 1/sqrtf(nrot),
 * quant_q8_0 / quant_q4_0 :182-234) for `nt` contiguous rows of n_head*dim
 * elements, one f32 operation at a time (this file is built without
 * floating-point contraction). Angles use sinf / cosf. Returns 1 for an
 * invalid shape.
 */
static float h2f(const uint8_t* b) { uint16_t h; memcpy(&h, b, 2); return (float)kvo_half_to_double(h); }

static uint16_t f2h_rn(float f) {
    /* float -> IEEE half, round to nearest even (values here are finite). */
    uint32_t x; memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = (int32_t)((x >> 23) & 255) - 127 + 15;
    uint32_t man = x & 0x7fffffu;
    if (((x >> 23) & 255) == 0 && man == 0) return (uint16_t)sign;
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const uint32_t shift = (uint32_t)(14 - exp);
        uint32_t half_man = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_man & 1))) ++half_man;
        return (uint16_t)(sign | half_man);
    }
    uint32_t half_man = man >> 13;
    const uint32_t rem = man & 0x1fffu;
    uint32_t h = sign | ((uint32_t)exp << 10) | half_man;
    if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1))) ++h;
    return (uint16_t)h;
}

int kvo_restore_k(int type, const uint8_t* src, uint8_t* dst, uint32_t nt, uint32_t n_head, uint32_t dim,
                  uint32_t n_rot, int32_t pos0, const float* theta, uint32_t nrot) {
    if (type != KVO_Q8_0 && type != KVO_Q4_0) return 1;
    const uint32_t n_embd = n_head * dim, nblk = n_embd / 32, kb = type == KVO_Q8_0 ? 34 : 18;
    if (!n_embd || dim % 32 || n_rot % 2 || n_rot > dim) return 1;
    if (nrot && ((nrot != 64 && nrot != 128 && nrot != 256 && nrot != 512) || n_embd % nrot)) return 1;
    float* row = (float*)malloc(n_embd * sizeof(float));
    if (!row) return 2;
    const float scale = nrot ? 1.0f / sqrtf((float)nrot) : 1.0f;
    for (uint32_t t = 0; t < nt; ++t) {
        const uint8_t* s = src + (uint64_t)t * nblk * kb;
        uint8_t* o = dst + (uint64_t)t * nblk * kb;
        for (uint32_t e = 0; e < n_embd; ++e) {
            const uint8_t* b = s + (e / 32) * kb;
            const uint32_t j = e % 32;
            const float code = type == KVO_Q8_0 ? (float)(int8_t)b[2 + j]
                                                : (float)(((b[2 + j % 16] >> (j < 16 ? 0 : 4)) & 15) - 8);
            row[e] = code * h2f(b);
        }
        if (n_rot) {
            const uint32_t half = n_rot / 2;
            const float pos = (float)(int32_t)(pos0 + (int32_t)t);
            for (uint32_t h = 0; h < n_head; ++h)
                for (uint32_t i = 0; i < half; ++i) {
                    const float ang = pos * theta[i];
                    const float sn = sinf(ang), cs = cosf(ang);
                    float* r = row + h * dim;
                    const float x0 = r[i], x1 = r[i + half];
                    const float a0 = x0 * cs, a1 = x1 * sn, b0 = x0 * sn, b1 = x1 * cs;
                    r[i] = a0 - a1;
                    r[i + half] = b0 + b1;
                }
        }
        if (nrot) {
            for (uint32_t e = 0; e < n_embd; ++e) row[e] = row[e] * scale;
            for (uint32_t c0 = 0; c0 < n_embd; c0 += nrot)
                for (uint32_t h = 1; h < nrot; h *= 2)
                    for (uint32_t i = 0; i < nrot; i += 2 * h)
                        for (uint32_t j = 0; j < h; ++j) {
                            const float a = row[c0 + i + j], b = row[c0 + i + j + h];
                            row[c0 + i + j] = a + b;
                            row[c0 + i + j + h] = a - b;
                        }
        }
        for (uint32_t bi = 0; bi < nblk; ++bi) {
            const float* x = row + bi * 32;
            uint8_t* b = o + bi * kb;
            if (type == KVO_Q8_0) {
                float amax = 0.0f;
                for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
                const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
                const uint16_t hd = f2h_rn(d);
                memcpy(b, &hd, 2);
                for (int j = 0; j < 32; ++j) b[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
            } else {
                float amax = 0.0f, vmax = 0.0f;
                for (int j = 0; j < 32; ++j)
                    if (amax < fabsf(x[j])) { amax = fabsf(x[j]); vmax = x[j]; }
                const float d = vmax / -8.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
                const uint16_t hd = f2h_rn(d);
                memcpy(b, &hd, 2);
                for (int j = 0; j < 16; ++j) {
                    const float x0 = x[j] * id, x1 = x[j + 16] * id;
                    int xi0 = (int)(x0 + 8.5f), xi1 = (int)(x1 + 8.5f);
                    if (xi0 > 15) xi0 = 15;
                    if (xi1 > 15) xi1 = 15;
                    b[2 + j] = (uint8_t)((xi0 & 15) | ((xi1 & 15) << 4));
                }
            }
        }
    }
    free(row);
    return 0;
}

/*
 * Per-token page mass, FP64 — restates the reference's dense oracle
 * AttentionSampler::qualify (src/adapter/llama-kvmem-attention.cpp:61-94):
 *   logit_t = scale * <q_rh, K_t,kvh(h)>   (FP64 dot of decoded operands)
 *   softcap > 0:   logit_t = softcap * tanh(logit_t / softcap)      (:76)
 *   logit_t += bias_t; tokens whose bias is non-finite are skipped  (:71,:77)
 *   prob_t = exp(logit_t - max) / sum                               (:80)
 *   mass[page(t)] += prob_t / heads_in_group                         (:81)
 * with token visibility t < tokens as in the CUDA kernel
 * (src/adapter/llama-kvmem-attention-cuda.cu:73).
 *
 * Generalised only in its indexing: L layers with a byte layer stride, R query
 * rows, and `groups` aggregation groups (groups == 1: mean over all Hq heads,
 * the reference's `average` kernel; groups == Hkv: mean over the G heads that
 * share one KV head).
 *
 * q:    element (l, r, h, d) at q + l*q_layer + r*q_row + h*q_head + d*esize(q_type)
 * k:    row (l, t, kvh) at k + l*k_layer + t*k_row + kvh*k_head, `k_type` row of D
 * mask: optional f32 bias, element (r, t) at mask[r*mask_row + t] (NULL: zero bias)
 * out:  mass[((l*groups + g)*R + r)*pages + p], pages = ceil(tokens/page_tokens)
 * A (row, head) with no visible token yields NaN mass, as the reference's
 * normaliser does (max = -inf).
 */
int kvo_page_mass(const uint8_t* q, int q_type, uint64_t q_layer, uint64_t q_row, uint64_t q_head,
                  const uint8_t* k, int k_type, uint64_t k_layer, uint64_t k_row, uint64_t k_head,
                  const float* mask, uint64_t mask_row,
                  uint32_t layers, uint32_t rows, uint32_t heads, uint32_t kv_heads, uint32_t dim,
                  uint64_t tokens, uint32_t page_tokens, double scale, double softcap,
                  uint32_t groups, double* out) {
    if (!layers || !rows || !heads || !kv_heads || !dim || heads % kv_heads || !page_tokens ||
        (groups != 1 && groups != kv_heads))
        return KVO_ERR_INVALID;
    const uint64_t pages = (tokens + page_tokens - 1) / page_tokens;
    const uint32_t group = heads / kv_heads;
    const uint32_t per_group = groups == 1 ? heads : group;
    /* Each K row is decoded once and dotted with the `group` query heads that
     * share its KV head; every dot is the same FP64 sum in dimension order. */
    const uint64_t nt = tokens ? tokens : 1;
    double* logits = (double*)malloc(sizeof(double) * nt * group);
    double* qv = (double*)malloc(sizeof(double) * dim * group);
    double* kv = (double*)malloc(sizeof(double) * dim);
    double* maxima = (double*)malloc(sizeof(double) * group);
    if (!logits || !qv || !kv || !maxima) {
        free(logits); free(qv); free(kv); free(maxima);
        return KVO_ERR_RUNTIME;
    }
    memset(out, 0, sizeof(double) * layers * groups * rows * pages);
    for (uint32_t l = 0; l < layers; ++l)
        for (uint32_t r = 0; r < rows; ++r)
            for (uint32_t kvh = 0; kvh < kv_heads; ++kvh) {
                for (uint32_t g = 0; g < group; ++g) {
                    const uint8_t* qb = q + l * q_layer + r * q_row + (kvh * group + g) * q_head;
                    for (uint32_t d = 0; d < dim; ++d) qv[g * dim + d] = kvo_decode(q_type, qb, d);
                    maxima[g] = -INFINITY;
                }
                for (uint64_t t = 0; t < tokens; ++t) {
                    const double bias = mask ? (double)mask[r * mask_row + t] : 0.0;
                    if (!isfinite(bias)) {
                        for (uint32_t g = 0; g < group; ++g) logits[g * nt + t] = -INFINITY;
                        continue;
                    }
                    const uint8_t* kb = k + l * k_layer + t * k_row + kvh * k_head;
                    for (uint32_t d = 0; d < dim; ++d) kv[d] = kvo_decode(k_type, kb, d);
                    for (uint32_t g = 0; g < group; ++g) {
                        const double* qg = qv + g * dim;
                        double dot = 0;
                        for (uint32_t d = 0; d < dim; ++d) dot += qg[d] * kv[d];
                        dot *= scale;
                        if (softcap > 0) dot = softcap * tanh(dot / softcap);
                        const double logit = dot + bias;
                        logits[g * nt + t] = logit;
                        if (logit > maxima[g]) maxima[g] = logit;
                    }
                }
                for (uint32_t g = 0; g < group; ++g) {
                    double* lg = logits + g * nt;
                    double* row_out = out + (((uint64_t)l * groups + (groups == 1 ? 0 : kvh)) * rows + r) * pages;
                    if (maxima[g] == -INFINITY) {
                        for (uint64_t p = 0; p < pages; ++p) row_out[p] = NAN;
                        continue;
                    }
                    double denominator = 0;
                    for (uint64_t t = 0; t < tokens; ++t) denominator += lg[t] = exp(lg[t] - maxima[g]);
                    for (uint64_t t = 0; t < tokens; ++t)
                        row_out[t / page_tokens] += lg[t] / denominator / per_group;
                }
            }
    free(kv);
    free(maxima);
    free(logits);
    free(qv);
    return KVO_OK;
}

/*
 * Explicit FP16 operand boundary — restates recall_fp16
 * (kvmem/src/host/graph_recall.cpp:295-320): round-to-nearest-even to binary16,
 * rejecting non-finite input, exponents above 15 and values that round to
 * infinity. Returns KVO_ERR_INVALID for a rejected operand.
 */
int kvo_recall_fp16(float value, float* out) {
    if (!isfinite(value)) return KVO_ERR_INVALID;
    uint32_t bits;
    memcpy(&bits, &value, 4);
    const uint32_t sign = bits & 0x80000000u;
    const int exponent = (int)((bits >> 23) & 255) - 127;
    uint32_t rounded = 0;
    if (exponent >= -14) {
        if (exponent > 15) return KVO_ERR_INVALID;
        rounded = (bits & 0x7fffffffu) + 0xfffu + ((bits >> 13) & 1u);
        rounded &= 0x7fffe000u;
        if (rounded >= 0x47800000u) return KVO_ERR_INVALID;
    } else if (exponent >= -25) {
        const uint32_t mantissa = (bits & 0x7fffffu) | 0x800000u;
        const int shift = -exponent - 1;
        uint32_t half = mantissa >> shift;
        const uint32_t remainder = mantissa & ((1u << shift) - 1);
        const uint32_t halfway = 1u << (shift - 1);
        half += remainder > halfway || (remainder == halfway && (half & 1));
        float v = ldexpf((float)half, -24);
        *out = sign ? -v : v;
        return KVO_OK;
    }
    rounded |= sign;
    memcpy(out, &rounded, 4);
    return KVO_OK;
}

/*
 * Mean-K page softmax, FP64 — restates page_softmax_scores
 * (kvmem/src/host/graph_recall.cpp:322-394).
 *   means: f32 mean keys, element (l, page, kvh*D + d) at means[(l*pages + p)*Hkv*D + ...]
 *          (what RawKvStore::mean_k returns: sum * (1.0f/count), raw_kv_store.cpp:606-614)
 *   q:     f32 queries, element (l, t, h, d) at q[((l*rows + t)*Hq + h)*D + d]
 *   layer_rows[l]: active rows of layer l (0 = absent layer)
 *   score_mask[p]: page p takes part in the softmax domain (graph_recall.cpp:333-339)
 *   aggregation 0 = Mean (:378-380), 1 = Max (:381-389)
 *   out[p]: double score; disabled pages stay 0.
 * Both operands pass recall_fp16 (:359, :368); a rejected operand returns
 * KVO_ERR_INVALID like the reference's exception.
 */
int kvo_meank_scores(const float* means, const float* q, const uint32_t* layer_rows,
                     uint32_t layers, uint32_t rows, uint32_t heads, uint32_t kv_heads, uint32_t dim,
                     uint32_t pages, const uint8_t* score_mask, int aggregation, double scale,
                     double* out) {
    if (!layers || !rows || !heads || !kv_heads || !dim || heads % kv_heads || (aggregation != 0 && aggregation != 1))
        return KVO_ERR_INVALID;
    memset(out, 0, sizeof(double) * pages);
    uint32_t* enabled = (uint32_t*)malloc(sizeof(uint32_t) * (pages ? pages : 1));
    uint32_t n = 0;
    for (uint32_t p = 0; p < pages; ++p) if (score_mask[p]) enabled[n++] = p;
    uint32_t active = 0;
    for (uint32_t l = 0; l < layers; ++l) {
        if (layer_rows[l] > rows) { free(enabled); return KVO_ERR_INVALID; }
        active += layer_rows[l] != 0;
    }
    if (!n || !active) { free(enabled); return KVO_OK; }
    const uint64_t kw = (uint64_t)kv_heads * dim, qw = (uint64_t)heads * dim;
    const uint32_t group = heads / kv_heads;
    float* rep = (float*)malloc(sizeof(float) * n * kw);
    float* qrep = (float*)malloc(sizeof(float) * dim);
    double* logits = (double*)malloc(sizeof(double) * n);
    double* gmax = (double*)malloc(sizeof(double) * n);
    if (!scale) scale = 1.0 / sqrt((double)dim);
    int rc = KVO_OK;
    for (uint32_t l = 0; l < layers && rc == KVO_OK; ++l) {
        if (!layer_rows[l]) continue;
        for (uint32_t j = 0; j < n && rc == KVO_OK; ++j)
            for (uint64_t d = 0; d < kw && rc == KVO_OK; ++d)
                rc = kvo_recall_fp16(means[((uint64_t)l * pages + enabled[j]) * kw + d], &rep[j * kw + d]);
        for (uint32_t t = 0; t < layer_rows[l] && rc == KVO_OK; ++t)
            for (uint32_t h = 0; h < heads && rc == KVO_OK; ++h) {
                if (aggregation == 1 && h % group == 0) for (uint32_t j = 0; j < n; ++j) gmax[j] = 0;
                const float* row = q + ((uint64_t)l * rows + t) * qw + (uint64_t)h * dim;
                for (uint32_t d = 0; d < dim && rc == KVO_OK; ++d) rc = kvo_recall_fp16(row[d], &qrep[d]);
                if (rc != KVO_OK) break;
                const uint32_t kvh = h / group;
                double maximum = -INFINITY;
                for (uint32_t j = 0; j < n; ++j) {
                    double dot = 0;
                    for (uint32_t d = 0; d < dim; ++d) dot += (double)qrep[d] * rep[j * kw + kvh * dim + d];
                    logits[j] = dot * scale;
                    if (logits[j] > maximum) maximum = logits[j];
                }
                double denominator = 0;
                for (uint32_t j = 0; j < n; ++j) denominator += logits[j] = exp(logits[j] - maximum);
                if (aggregation == 0) {
                    for (uint32_t j = 0; j < n; ++j)
                        out[enabled[j]] += logits[j] / denominator / ((double)active * heads);
                } else {
                    for (uint32_t j = 0; j < n; ++j) {
                        const double v = logits[j] / denominator;
                        if (v > gmax[j]) gmax[j] = v;
                    }
                    if (h % group == group - 1) {
                        double mass = 0;
                        for (uint32_t j = 0; j < n; ++j) mass += gmax[j];
                        for (uint32_t j = 0; j < n; ++j)
                            out[enabled[j]] += gmax[j] / mass / ((double)active * kv_heads);
                    }
                }
            }
    }
    free(enabled); free(rep); free(qrep); free(logits); free(gmax);
    return rc;
}

/*
 * Score frame — restates query_score_frame (kvmem/src/host/graph_recall.cpp:269-293).
 * Outputs n = ceil(accepted/block) entries; returns n via *out_n.
 */
int kvo_query_score_frame(uint64_t accepted, uint32_t block, uint32_t budget, uint32_t sink, uint32_t recent,
                          const uint32_t* fixed, uint32_t nfixed, uint64_t capacity,
                          uint64_t* starts, uint32_t* counts, uint8_t* score_mask, uint8_t* transport_mask,
                          uint64_t* out_n) {
    if (!block || !budget) return KVO_ERR_INVALID;
    const uint64_t n = accepted / block + (accepted % block != 0);
    if (n > UINT32_MAX || n > capacity) return KVO_ERR_INVALID;
    for (uint64_t i = 0; i < n; ++i) {
        starts[i] = i * block;
        const uint64_t rest = accepted - i * block;
        counts[i] = (uint32_t)(rest < block ? rest : block);
        score_mask[i] = 1;
        transport_mask[i] = n > budget;
    }
    if (n > budget && (uint64_t)sink + recent < n) {
        for (uint64_t i = 0; i < (sink < n ? sink : n); ++i) score_mask[i] = 0;
        for (uint64_t i = n - (recent < n ? recent : n); i < n; ++i) score_mask[i] = 0;
    }
    for (uint32_t i = 0; i < nfixed; ++i) {
        if (fixed[i] >= n) return KVO_ERR_INVALID;
        transport_mask[fixed[i]] = 0;
    }
    *out_n = n;
    return KVO_OK;
}

/*
 * Media group closure — restates scored_media_group
 * (kvmem/src/host/kvmem_store.cpp:18-32). ranges: nr half-open token spans.
 */
static void media_group(uint32_t id, uint32_t n, uint32_t block, const uint32_t* ranges, uint32_t nr,
                        uint32_t* gb, uint32_t* ge) {
    uint32_t begin = id, end = id + 1;
    int changed;
    do {
        const uint32_t ob = begin, oe = end;
        for (uint32_t i = 0; i < nr; ++i) {
            const uint32_t lo = ranges[2 * i] / block;
            uint64_t hi64 = ((uint64_t)ranges[2 * i + 1] + block - 1) / block;
            const uint32_t hi = hi64 < n ? (uint32_t)hi64 : n;
            if (lo < end && begin < hi) { if (lo < begin) begin = lo; if (hi > end) end = hi; }
        }
        changed = ob != begin || oe != end;
    } while (changed);
    *gb = begin; *ge = end;
}

typedef struct { double score; uint32_t id; uint32_t index; } kvo_rank;
static int rank_cmp(const void* a, const void* b) {
    const kvo_rank* x = (const kvo_rank*)a; const kvo_rank* y = (const kvo_rank*)b;
    if (x->score != y->score) return x->score > y->score ? -1 : 1;
    return x->id > y->id ? -1 : (x->id < y->id ? 1 : 0);
}

/*
 * Budgeted top-k with keep pages — restates KvMemStore::pick_scored_blocks
 * (kvmem/src/host/kvmem_store.cpp:418-451): mandatory pages first (required:
 * a cold, incomplete or over-budget mandatory group is an error), then
 * candidates by (score desc, id desc), each admitted with its whole media group
 * only if it fits; output ascending. `n` is the store's block count.
 * Errors: KVO_ERR_INVALID for a bad frame / candidate (invalid_argument),
 * KVO_ERR_RUNTIME for an unsatisfiable mandatory page (runtime_error).
 */
int kvo_pick_scored(uint32_t n, const uint32_t* candidates, const double* scores, uint32_t ncand,
                    const uint32_t* mandatory, uint32_t nmand, uint32_t budget, int signed_scores,
                    uint32_t block_tokens, const uint32_t* ranges, uint32_t nranges,
                    uint32_t* out, uint32_t* out_n) {
    if (!budget) return KVO_ERR_INVALID;
    uint8_t* allowed = (uint8_t*)calloc(n ? n : 1, 1);
    uint8_t* kept = (uint8_t*)calloc(n ? n : 1, 1);
    kvo_rank* rank = (kvo_rank*)malloc(sizeof(kvo_rank) * (ncand ? ncand : 1));
    int rc = KVO_OK;
    uint32_t count = 0;
    for (uint32_t i = 0; i < ncand; ++i) {
        const uint32_t id = candidates[i];
        if (id >= n || allowed[id] || !isfinite(scores[i]) || (!signed_scores && scores[i] < 0)) { rc = KVO_ERR_INVALID; goto done; }
        allowed[id] = 1;
    }
    for (uint32_t m = 0; m < nmand; ++m) {
        const uint32_t id = mandatory[m];
        if (id >= n) { rc = KVO_ERR_INVALID; goto done; }
        uint32_t b, e, need = 0; int complete = 1;
        media_group(id, n, block_tokens, ranges, nranges, &b, &e);
        for (uint32_t x = b; x < e; ++x) { need += !kept[x]; complete &= allowed[x] != 0; }
        if (!complete || count + need > budget) { rc = KVO_ERR_RUNTIME; goto done; }
        for (uint32_t x = b; x < e; ++x) if (!kept[x]) { kept[x] = 1; ++count; }
    }
    for (uint32_t i = 0; i < ncand; ++i) { rank[i].score = scores[i]; rank[i].id = candidates[i]; rank[i].index = i; }
    qsort(rank, ncand, sizeof(kvo_rank), rank_cmp);
    for (uint32_t i = 0; i < ncand; ++i) {
        uint32_t b, e, need = 0; int complete = 1;
        media_group(rank[i].id, n, block_tokens, ranges, nranges, &b, &e);
        for (uint32_t x = b; x < e; ++x) { need += !kept[x]; complete &= allowed[x] != 0; }
        if (!complete || count + need > budget) continue;
        for (uint32_t x = b; x < e; ++x) if (!kept[x]) { kept[x] = 1; ++count; }
    }
    {
        uint32_t w = 0;
        for (uint32_t id = 0; id < n; ++id) if (kept[id]) out[w++] = id;
        *out_n = w;
    }
done:
    free(allowed); free(kept); free(rank);
    return rc;
}

static int u64_cmp(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/*
 * Residency delta — restates plan_residency (kvmem/src/host/memory_contract.cpp:135-150):
 * evict = resident \ selected (or all resident when force_reload),
 * retain = resident ∩ selected, restore = selected \ resident (or all selected
 * when force_reload); each ascending. Duplicates in either input are an error
 * (MemoryErrorCode::InvalidPlan).
 */
int kvo_plan_residency(const uint64_t* resident, uint32_t nres, const uint64_t* selected, uint32_t nsel,
                       int force_reload, uint64_t* evict, uint32_t* nevict, uint64_t* retain, uint32_t* nretain,
                       uint64_t* restore, uint32_t* nrestore) {
    uint64_t* a = (uint64_t*)malloc(sizeof(uint64_t) * (nres ? nres : 1));
    uint64_t* b = (uint64_t*)malloc(sizeof(uint64_t) * (nsel ? nsel : 1));
    memcpy(a, resident, sizeof(uint64_t) * nres);
    memcpy(b, selected, sizeof(uint64_t) * nsel);
    qsort(a, nres, sizeof(uint64_t), u64_cmp);
    qsort(b, nsel, sizeof(uint64_t), u64_cmp);
    int rc = KVO_OK;
    for (uint32_t i = 1; i < nres; ++i) if (a[i] == a[i - 1]) rc = KVO_ERR_INVALID;
    for (uint32_t i = 1; i < nsel; ++i) if (b[i] == b[i - 1]) rc = KVO_ERR_INVALID;
    if (rc == KVO_OK) {
        uint32_t ne = 0, nr = 0, ns = 0, i = 0, j = 0;
        for (i = 0; i < nres; ++i) {
            while (j < nsel && b[j] < a[i]) ++j;
            const int chosen = j < nsel && b[j] == a[i];
            if (force_reload || !chosen) evict[ne++] = a[i];
            else retain[nr++] = a[i];
        }
        j = 0;
        for (i = 0; i < nsel; ++i) {
            while (j < nres && a[j] < b[i]) ++j;
            const int current = j < nres && a[j] == b[i];
            if (force_reload || !current) restore[ns++] = b[i];
        }
        *nevict = ne; *nretain = nr; *nrestore = ns;
    }
    free(a); free(b);
    return rc;
}
