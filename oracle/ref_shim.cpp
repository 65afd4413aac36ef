// CPU ORACLE — test infrastructure only.
//
// extern "C" entry points over the reference's own CPU selection classes, so
// tests and bench.py's reference arm can call the unmodified reference code
// through ctypes. This file is compiled together with the reference sources
// (kvmem/src/host/*.cpp, listed in oracle/Makefile) into oracle/_ref/; the
// product never links it. Exceptions are mapped to status codes:
//   0 ok, 1 std::invalid_argument / MemoryError(InvalidPlan), 2 other exception.
#include "kvmem/graph_recall.hpp"
#include "kvmem/layerwise_selection.hpp"
#include "kvmem/kvmem_store.hpp"
#include "kvmem/memory_contract.hpp"
#include "kvmem/raw_kv_store.hpp"

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <vector>

namespace {
template <class F> int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument&) {
        return 1;
    } catch (const kvmem::MemoryError& e) {
        return e.code() == kvmem::MemoryErrorCode::InvalidPlan ? 1 : 2;
    } catch (...) {
        return 2;
    }
}
}  // namespace

extern "C" {

// query_score_frame (kvmem/src/host/graph_recall.cpp:269) into caller arrays.
int kvref_query_score_frame(uint64_t accepted, uint32_t block, uint32_t budget, uint32_t sink,
                            uint32_t recent, const uint32_t* fixed, uint32_t nfixed, uint64_t capacity,
                            uint64_t* starts, uint32_t* counts, uint8_t* score_mask,
                            uint8_t* transport_mask, uint64_t* out_n) {
    return guarded([&] {
        auto f = kvmem::query_score_frame(accepted, block, budget, sink, recent,
                                          std::vector<uint32_t>(fixed, fixed + nfixed));
        if (f.starts.size() > capacity) throw std::invalid_argument("capacity");
        std::memcpy(starts, f.starts.data(), f.starts.size() * sizeof(uint64_t));
        std::memcpy(counts, f.counts.data(), f.counts.size() * sizeof(uint32_t));
        std::memcpy(score_mask, f.score_mask.data(), f.score_mask.size());
        std::memcpy(transport_mask, f.transport_mask.data(), f.transport_mask.size());
        *out_n = f.starts.size();
    });
}

// page_softmax_scores (kvmem/src/host/graph_recall.cpp:322) over a RawKvStore
// filled with per-page F32 K sums through write_layer_mean_sum
// (kvmem/src/host/raw_kv_store.cpp:444), so mean_k returns sum * (1/count).
//   sums:   [layers][pages][kv_heads*dim] f32, counts: [pages] tokens per page
//   q:      [layers][rows][heads*dim] f32
//   frame:  from query_score_frame(accepted, block, budget, sink, recent, fixed)
int kvref_page_softmax_scores(const float* sums, const uint32_t* counts, const float* q,
                              const uint32_t* layer_rows, uint32_t layers, uint32_t rows,
                              uint32_t heads, uint32_t kv_heads, uint32_t dim, uint32_t block,
                              uint64_t accepted, uint32_t budget, uint32_t sink, uint32_t recent,
                              const uint32_t* fixed, uint32_t nfixed, int aggregation, float scale,
                              double* out, uint64_t capacity) {
    return guarded([&] {
        const uint32_t kw = kv_heads * dim;
        kvmem::RawKvStore keys({layers, kw, 0, block});
        auto frame = kvmem::query_score_frame(accepted, block, budget, sink, recent,
                                              std::vector<uint32_t>(fixed, fixed + nfixed));
        const size_t pages = frame.starts.size();
        if (pages > capacity) throw std::invalid_argument("capacity");
        for (uint32_t l = 0; l < layers; ++l)
            for (size_t p = 0; p < pages; ++p)
                keys.write_layer_mean_sum(uint32_t(p * block), counts[p], l, sums + (size_t(l) * pages + p) * kw);
        kvmem::PageQueryView view{q, layer_rows, layers, rows, heads, kv_heads, dim, nullptr, scale};
        const auto r = kvmem::page_softmax_scores(
            keys, view, frame, aggregation ? kvmem::GqaScoreAggregation::Max : kvmem::GqaScoreAggregation::Mean);
        std::memcpy(out, r.data(), r.size() * sizeof(double));
    });
}

// recall_fp16 (kvmem/src/host/graph_recall.cpp:295).
int kvref_recall_fp16(float value, float* out) {
    return guarded([&] { *out = kvmem::recall_fp16(value); });
}

// KvMemStore::pick_scored_blocks (kvmem/src/host/kvmem_store.cpp:418) on a
// store of n blocks of `block` tokens, with optional media ranges.
int kvref_pick_scored(uint32_t n, const uint32_t* candidates, const double* scores, uint32_t ncand,
                      const uint32_t* mandatory, uint32_t nmand, uint32_t budget, int signed_scores,
                      uint32_t block, const uint32_t* ranges, uint32_t nranges, uint32_t* out,
                      uint32_t* out_n) {
    return guarded([&] {
        kvmem::KvMemStoreConfig cfg;
        cfg.block_tokens = block;
        cfg.select_budget = budget * block;
        cfg.sink_blocks = 0;
        cfg.recent_blocks = 0;
        kvmem::KvMemStore store(cfg);
        store.register_append(n * block);
        std::vector<std::pair<uint32_t, uint32_t>> media;
        for (uint32_t i = 0; i < nranges; ++i) media.push_back({ranges[2 * i], ranges[2 * i + 1]});
        store.set_media_ranges(media);
        const auto r = store.pick_scored_blocks(std::vector<uint32_t>(candidates, candidates + ncand),
                                                std::vector<double>(scores, scores + ncand),
                                                std::vector<uint32_t>(mandatory, mandatory + nmand), budget,
                                                signed_scores != 0);
        std::memcpy(out, r.data(), r.size() * sizeof(uint32_t));
        *out_n = uint32_t(r.size());
    });
}

// KvMemStore::query_fixed_blocks (kvmem/src/host/kvmem_store.cpp:381) on a store
// of `total_tokens` appended tokens in blocks of `block`, a selection budget of
// `budget` blocks, sink / recent blocks and media ranges. Exceptions: 1 for
// std::invalid_argument, 2 for any other (the budget overflow).
int kvref_query_fixed_blocks(uint32_t total_tokens, uint32_t block, uint32_t budget, uint32_t sink, uint32_t recent,
                             const uint32_t* ranges, uint32_t nranges, const uint32_t* mandatory, uint32_t nmand,
                             uint32_t* out, uint32_t* out_n) {
    return guarded([&] {
        kvmem::KvMemStoreConfig cfg;
        cfg.block_tokens = block;
        cfg.select_budget = budget * block;
        cfg.sink_blocks = sink;
        cfg.recent_blocks = recent;
        kvmem::KvMemStore store(cfg);
        store.register_append(total_tokens);
        std::vector<std::pair<uint32_t, uint32_t>> media;
        for (uint32_t i = 0; i < nranges; ++i) media.push_back({ranges[2 * i], ranges[2 * i + 1]});
        store.set_media_ranges(media);
        const auto r = store.query_fixed_blocks(std::vector<uint32_t>(mandatory, mandatory + nmand));
        std::memcpy(out, r.data(), r.size() * sizeof(uint32_t));
        *out_n = uint32_t(r.size());
    });
}

// plan_residency (kvmem/src/host/memory_contract.cpp:135).
int kvref_plan_residency(const uint64_t* resident, uint32_t nres, const uint64_t* selected, uint32_t nsel,
                         int force_reload, uint64_t* evict, uint32_t* nevict, uint64_t* retain,
                         uint32_t* nretain, uint64_t* restore, uint32_t* nrestore) {
    return guarded([&] {
        const auto d = kvmem::plan_residency(std::vector<uint64_t>(resident, resident + nres),
                                             std::vector<uint64_t>(selected, selected + nsel), force_reload != 0);
        std::memcpy(evict, d.evict.data(), d.evict.size() * 8);
        std::memcpy(retain, d.retain.data(), d.retain.size() * 8);
        std::memcpy(restore, d.restore.data(), d.restore.size() * 8);
        *nevict = uint32_t(d.evict.size());
        *nretain = uint32_t(d.retain.size());
        *nrestore = uint32_t(d.restore.size());
    });
}

// propagate_query_scores (kvmem/src/host/graph_recall.cpp:494) on a
// GraphSnapshot assembled from arrays (one chunk holding every row; message
// spans when has_messages), a frame given by starts / transport_mask.
int kvref_propagate_scores(const double* raw, uint32_t n, const uint64_t* starts, const uint8_t* transport_mask,
                           uint64_t frame_accepted, uint32_t block, uint64_t graph_accepted, uint64_t completed,
                           const uint64_t* row_source, const uint64_t* row_samples, const uint32_t* row_begin,
                           const uint32_t* row_count, uint32_t nrows, const uint64_t* edge_target,
                           const double* edge_mass, const uint64_t* span_begin, const uint64_t* span_end,
                           const uint8_t* span_end_known, uint32_t nspans, int has_messages, double alpha,
                           double cross, double* out) {
    return guarded([&] {
        kvmem::QueryScoreFrame frame;
        frame.starts.assign(starts, starts + n);
        frame.counts.assign(n, block);
        frame.score_mask.assign(n, 1);
        frame.transport_mask.assign(transport_mask, transport_mask + n);
        frame.accepted_through = frame_accepted;
        kvmem::GraphSnapshot graph;
        graph.block_tokens = block;
        graph.accepted_through = graph_accepted;
        graph.completed_through = completed;
        auto rows = std::make_shared<std::vector<kvmem::GraphRow>>();
        for (uint32_t r = 0; r < nrows; ++r) {
            kvmem::GraphRow row;
            row.source = row_source[r];
            row.samples = row_samples[r];
            for (uint32_t e = row_begin[r]; e < row_begin[r] + row_count[r]; ++e)
                row.edges.push_back({edge_target[e], edge_mass[e]});
            rows->push_back(std::move(row));
        }
        if (nrows) graph.chunks.push_back(rows);
        if (has_messages) {
            auto spans = std::make_shared<std::vector<kvmem::GraphMessageSpan>>();
            for (uint32_t i = 0; i < nspans; ++i) spans->push_back({span_begin[i], span_end[i], span_end_known[i] != 0});
            graph.messages = spans;
        }
        const auto result = kvmem::propagate_query_scores(std::vector<double>(raw, raw + n), frame, graph, alpha, cross);
        std::memcpy(out, result.data(), n * sizeof(double));
    });
}

// LrfuHistory::preview (kvmem/include/kvmem/lrfu.hpp:57-79) after restoring a
// committed history `prev` and opening the next round; out = score(i).
int kvref_lrfu_preview(const double* scores, uint32_t n, const double* prev, uint32_t n_prev, double lambda,
                       double fraction, double* out) {
    return guarded([&] {
        kvmem::LrfuHistory history(lambda, fraction);
        kvmem::LrfuState state;
        state.scores = std::make_shared<const std::vector<double>>(prev, prev + n_prev);
        state.round = 1;
        state.committed = true;
        history.restore(state);
        history.begin_round();
        history.preview(std::vector<double>(scores, scores + n));
        for (uint32_t i = 0; i < n; ++i) out[i] = history.score(i);
    });
}

// layerwise_tile_scores (kvmem/src/host/layerwise_selection.cpp:32-75) over the
// frame of n pages (starts / counts / masks) with a scorer that returns the given
// masses (n_masses of them: n, or 2n for the half-page frame); out receives the
// tile's slot scores (*out_n of them).
int kvref_layerwise_tile_scores(const uint64_t* starts, const uint32_t* counts, const uint8_t* score_mask,
                                const uint8_t* transport_mask, uint64_t n, uint64_t accepted, uint32_t page_tokens,
                                uint32_t mean_tokens, int keep_halves, const double* masses, uint64_t n_masses,
                                double* out, uint64_t* out_n) {
    return guarded([&] {
        kvmem::QueryScoreFrame f;
        f.accepted_through = accepted;
        f.starts.assign(starts, starts + n);
        f.counts.assign(counts, counts + n);
        f.score_mask.assign(score_mask, score_mask + n);
        f.transport_mask.assign(transport_mask, transport_mask + n);
        const auto r = kvmem::layerwise_tile_scores(f, page_tokens, mean_tokens, keep_halves != 0,
                                                    [&](const kvmem::QueryScoreFrame& g) {
                                                        if (g.starts.size() != n_masses)
                                                            throw std::invalid_argument("mass count");
                                                        return std::vector<double>(masses, masses + n_masses);
                                                    });
        std::memcpy(out, r.data(), r.size() * sizeof(double));
        *out_n = r.size();
    });
}

// layerwise_max_page_scores (kvmem/src/host/layerwise_selection.cpp:24-30).
int kvref_layerwise_max_page_scores(const double* halves, uint64_t n, double* out) {
    return guarded([&] {
        const auto r = kvmem::layerwise_max_page_scores(std::vector<double>(halves, halves + n));
        std::memcpy(out, r.data(), r.size() * sizeof(double));
    });
}

}  // extern "C"
