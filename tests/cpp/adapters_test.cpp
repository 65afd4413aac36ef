// GPU test of the reference-interface adapters (kvmem_b200/adapter): the
// reference's own classes llama_kvmem_attention_cuda
// (src/adapter/llama-kvmem-attention-cuda.h) and kvmem::PageSoftmaxCuda
// (kvmem/include/kvmem/page_softmax_cuda.hpp), implemented over libkvm_b200.so,
// driven as their callers drive them and compared with
//   * the FP64 per-token restatement (oracle/_ref/liboracle.so, kvo_page_mass)
//     within 1e-3 relative + 1e-6, and
//   * the reference's own CPU Mean-K scorer kvmem::page_softmax_scores (the
//     reference build, oracle/_ref/libkvref.so) within its qualification bound
//     2e-6 + 3e-5 * expected (kvmem/tests/graph_recall_cuda_test.cpp:43,52).
// Prints "ok" and exits 0, or names the first failure and exits 1.
#include "ggml-backend.h"
#include "ggml.h"
#include "llama-kvmem-attention-cuda.h"

#include "kvmem/graph_recall.hpp"
#include "kvmem/page_softmax_cuda.hpp"
#include "kvmem/raw_kv_store.hpp"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

extern "C" int kvo_page_mass(const uint8_t* q, int q_type, uint64_t q_layer, uint64_t q_row, uint64_t q_head,
                             const uint8_t* k, int k_type, uint64_t k_layer, uint64_t k_row, uint64_t k_head,
                             const float* mask, uint64_t mask_row, uint32_t layers, uint32_t rows, uint32_t heads,
                             uint32_t kv_heads, uint32_t dim, uint64_t tokens, uint32_t page_tokens, double scale,
                             double softcap, uint32_t groups, double* out);

// ggml's host read of a tensor's bytes, as the engine provides it (used for a host mask).
extern "C" void ggml_backend_tensor_get(const struct ggml_tensor* tensor, void* data, size_t offset, size_t size) {
    std::memcpy(data, static_cast<const uint8_t*>(tensor->data) + offset, size);
}
extern "C" size_t ggml_row_size(enum ggml_type type, int64_t ne) {
    return type == GGML_TYPE_F32 ? size_t(ne) * 4 : size_t(ne) * 2;
}

namespace {

void check(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error(what);
}
void cuda(cudaError_t e) { check(e == cudaSuccess, std::string("CUDA: ") + cudaGetErrorString(e)); }

template <class T> T* upload(const std::vector<T>& v) {
    T* d = nullptr;
    cuda(cudaMalloc(&d, v.size() * sizeof(T)));
    cuda(cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

void test_attention() {
    const int D = 128, Hq = 8, Hkv = 2, R = 5, T = 1000, page = 64;
    const int P = (T + page - 1) / page, alloc = P * page;  // the K allocation holds whole pages
    std::mt19937 g(3);
    std::normal_distribution<float> n01;
    std::vector<__half> k(size_t(alloc) * Hkv * D);
    for (auto& x : k) x = __float2half(n01(g));
    std::vector<float> q(size_t(R) * Hq * D), mask(size_t(R) * T, 0.f);
    for (auto& x : q) x = n01(g);
    for (int r = 0; r < R; ++r)
        for (int t = T - R + r + 1; t < T; ++t) mask[size_t(r) * T + t] = -INFINITY;  // causal rows
    __half* dk = upload(k);
    float* dq = upload(q);
    float* dm = upload(mask);
    ggml_tensor tq{}, tk{}, tm{}, th{};
    tq.type = GGML_TYPE_F32;
    tq.ne[0] = D, tq.ne[1] = R, tq.ne[2] = Hq, tq.ne[3] = 1;
    tq.nb[0] = 4, tq.nb[1] = size_t(Hq) * D * 4, tq.nb[2] = size_t(D) * 4;
    tq.data = dq;
    tk.type = GGML_TYPE_F16;
    tk.ne[0] = D, tk.ne[1] = T, tk.ne[2] = Hkv, tk.ne[3] = 1;
    tk.nb[0] = 2, tk.nb[1] = size_t(Hkv) * D * 2, tk.nb[2] = size_t(D) * 2;
    tk.data = dk;
    tm.type = GGML_TYPE_F32;
    tm.ne[0] = T, tm.ne[1] = R, tm.ne[2] = 1, tm.ne[3] = 1;
    tm.nb[0] = 4, tm.nb[1] = size_t(T) * 4;
    tm.data = dm;
    th = tm;
    th.data = mask.data();  // the same mask in host memory: staged by the adapter
    const float scale = 1.f / std::sqrt(float(D));
    std::vector<double> exp(size_t(R) * P);
    check(kvo_page_mass(reinterpret_cast<const uint8_t*>(q.data()), 0, 0, tq.nb[1], tq.nb[2],
                        reinterpret_cast<const uint8_t*>(k.data()), 1, 0, tk.nb[1], tk.nb[2], mask.data(), T, 1, R,
                        Hq, Hkv, D, T, page, scale, 0.0, 1, exp.data()) == 0,
          "oracle rejected its input");
    llama_kvmem_attention_cuda scorer;
    const std::vector<uint32_t> rows{4, 1, 2, 2};
    for (ggml_tensor* mt : {&tm, &th}) {
        std::vector<std::vector<float>> out;
        check(scorer.score(&tq, &tk, mt, scale, 0.f, page, rows, out), "score() refused a supported input");
        check(out.size() == rows.size(), "one output row per sampled row");
        for (size_t i = 0; i < rows.size(); ++i)
            for (int p = 0; p < P; ++p) {
                const double e = exp[size_t(rows[i]) * P + p], a = out[i][p];
                if (!(std::abs(a - e) <= 1e-6 + 1e-3 * std::abs(e)))
                    throw std::runtime_error("attention row " + std::to_string(rows[i]) + " page " +
                                             std::to_string(p) + ": " + std::to_string(a) + " vs " +
                                             std::to_string(e));
            }
    }
    // A K view whose partial last page runs past the end of its allocation cannot be read
    // page-wise: false (the caller builds its graph). Here the view's allocation ends at
    // token 1000 exactly.
    __half* tight = nullptr;
    cuda(cudaMalloc(&tight, size_t(T) * Hkv * D * 2));
    cuda(cudaMemcpy(tight, k.data(), size_t(T) * Hkv * D * 2, cudaMemcpyHostToDevice));
    ggml_tensor tt = tk;
    tt.data = tight;
    std::vector<std::vector<float>> out;
    check(!scorer.score(&tq, &tt, &tm, scale, 0.f, page, rows, out), "a partial page past the allocation");
    cudaFree(tight);
    // Outside the kernel's domain: false, as the reference (the caller builds its ggml graph).
    ggml_tensor t96 = tq;
    t96.ne[0] = 96;
    check(!scorer.score(&t96, &tk, &tm, scale, 0.f, page, rows, out), "head_dim 96 must return false");
    ggml_tensor tq8 = tq;
    tq8.type = GGML_TYPE_Q8_0;
    check(!scorer.score(&tq8, &tk, &tm, scale, 0.f, page, rows, out), "a q8_0 query must return false");
    cudaFree(dk), cudaFree(dq), cudaFree(dm);
}

void compare_meank(const std::vector<double>& got, const std::vector<double>& want, const char* what) {
    check(got.size() == want.size(), std::string(what) + ": size");
    for (size_t i = 0; i < got.size(); ++i)
        if (!(std::abs(got[i] - want[i]) <= 2e-6 + 3e-5 * std::abs(want[i])))
            throw std::runtime_error(std::string(what) + " page " + std::to_string(i) + ": " + std::to_string(got[i]) +
                                     " vs " + std::to_string(want[i]));
}

void test_page_softmax() {
    struct Shape { uint32_t blocks, rows, dim, qheads, kvheads; };
    for (const auto agg : {kvmem::GqaScoreAggregation::Mean, kvmem::GqaScoreAggregation::Max})
        for (const Shape s : {Shape{7, 129, 256, 8, 2}, Shape{300, 3, 64, 4, 1}}) {
            const uint32_t layers = 3, kw = s.kvheads * s.dim, qw = s.qheads * s.dim;
            kvmem::RawKvStoreConfig cfg;
            cfg.n_layer = layers, cfg.n_embd_k = kw, cfg.n_embd_v = 0, cfg.block_tokens = 4;
            kvmem::RawKvStore keys(cfg);
            std::vector<float> key(kw);
            for (uint32_t l = 0; l < layers; ++l)
                for (uint32_t b = 0; b < s.blocks; ++b) {
                    for (uint32_t d = 0; d < kw; ++d) key[d] = float(int((b * 13 + d * 7 + l * 11) % 101) - 50) / 16;
                    keys.write_layer_mean_sum(b * 4, 4, l, key.data());
                }
            std::vector<float> query(size_t(layers) * s.rows * qw);
            for (size_t d = 0; d < query.size(); ++d) query[d] = float(int((d * 17) % 127) - 63) / 32;
            const uint32_t counts[]{s.rows, 0, s.rows};  // layer 1 absent
            auto frame = kvmem::query_score_frame(uint64_t(s.blocks) * 4, 4, 3, 1, 1, {0, s.blocks - 1});
            kvmem::PageQueryView view{query.data(), counts, layers, s.rows, s.qheads, s.kvheads, s.dim};
            const auto want = kvmem::page_softmax_scores(keys, view, frame, agg);
            kvmem::PageSoftmaxCuda own(0);
            compare_meank(own.score(keys, view, frame, agg), want, "PageSoftmaxCuda(device)");
            // Borrowed workspace: planned for the geometry, score() works inside it.
            const auto bytes = kvmem::PageSoftmaxCuda::workspace_bytes(s.blocks, s.qheads, s.kvheads, s.dim);
            void* ws = nullptr;
            cuda(cudaMalloc(&ws, bytes));
            {
                kvmem::PageSoftmaxCuda borrowed(0, ws, bytes, s.blocks, s.qheads, s.kvheads, s.dim);
                compare_meank(borrowed.score(keys, view, frame, agg), want, "PageSoftmaxCuda(borrowed)");
                bool threw = false;
                try {
                    kvmem::PageSoftmaxCuda small(0, ws, bytes - 256, s.blocks, s.qheads, s.kvheads, s.dim);
                } catch (const std::invalid_argument&) {
                    threw = true;
                }
                check(threw, "a too-small borrowed workspace must be rejected");
            }
            cudaFree(ws);
            if (agg == kvmem::GqaScoreAggregation::Mean) {
                // score_current_layer: one layer's native FP16 Q on the producer's stream.
                const uint32_t layer = 2;
                std::vector<__half> native(size_t(s.rows) * qw);
                std::vector<float> widened(size_t(layers) * s.rows * qw, 0.f);
                for (size_t i = 0; i < native.size(); ++i) {
                    native[i] = __float2half(query[size_t(layer) * s.rows * qw + i]);
                    widened[size_t(layer) * s.rows * qw + i] = __half2float(native[i]);
                }
                const uint32_t only[]{0, 0, s.rows};
                kvmem::PageQueryView wview{widened.data(), only, layers, s.rows, s.qheads, s.kvheads, s.dim};
                const auto want_layer = kvmem::page_softmax_scores(keys, wview, frame, agg);
                __half* dq = upload(native);
                cudaStream_t st;
                cuda(cudaStreamCreate(&st));
                kvmem::NativeCurrentLayerQuery nq{};
                nq.data = dq;
                nq.bytes = native.size() * 2;
                nq.layer = layer, nq.rows = s.rows, nq.query_heads = s.qheads, nq.kv_heads = s.kvheads,
                nq.head_dim = s.dim;
                nq.scalar = kvmem::NativeQueryScalar::Float16;
                nq.row_stride = size_t(qw) * 2, nq.head_stride = size_t(s.dim) * 2, nq.dimension_stride = 2;
                compare_meank(own.score_current_layer(keys, nq, frame, st), want_layer, "score_current_layer");
                cudaStreamDestroy(st);
                cudaFree(dq);
            }
            // A non-finite operand is the reference's std::invalid_argument.
            std::vector<float> bad(query);
            bad[5] = INFINITY;
            kvmem::PageQueryView bview{bad.data(), counts, layers, s.rows, s.qheads, s.kvheads, s.dim};
            bool threw = false;
            try {
                own.score(keys, bview, frame, agg);
            } catch (const std::invalid_argument&) {
                threw = true;
            }
            check(threw, "a non-finite query must throw std::invalid_argument");
        }
}

}  // namespace

int main() {
    try {
        test_attention();
        test_page_softmax();
        std::printf("ok\n");
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FAILED: %s\n", e.what());
        return 1;
    }
}
