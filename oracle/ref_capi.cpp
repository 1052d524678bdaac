// ref_capi.cpp -- TEST / BASELINE INFRASTRUCTURE ONLY.
//
// A thin C-ABI bridge, compiled together with the UNMODIFIED reference
// HillServe sources (policy/host_policy.cpp, policy/full_gqa_cpu.cpp,
// policy/gqa_policy.cpp, smartssd/adapter.cpp, policy/h2o_residency.cpp,
// storage/{file_store,segmented_store}.cpp and the header-only
// runtime/gqa_pack.hpp) into oracle/_ref/libhs_ref.so by oracle/Makefile.
// It lets the tests pin the C oracle against the reference's own code on
// seeded inputs, and lets bench.py time the reference CPU path.  Nothing in
// the product links it.
#include "policy/full_gqa_cpu.hpp"
#include "policy/gqa_policy.hpp"
#include "policy/host_policy.hpp"
#include "runtime/gqa_pack.hpp"
#include "policy/h2o_residency.hpp"
#include "runtime/full_gqa_contract.hpp"
#include "storage/file_store.hpp"
#include "storage/kv_checksum.hpp"
#include "storage/kv_read_plan.hpp"
#include "storage/segmented_store.hpp"

#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

namespace {
void copy_error(const std::exception& e, char* err, std::size_t errlen) {
    if (err && errlen) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = 0;
    }
}
}  // namespace

extern "C" {

float ref_half_value(std::uint16_t h) { return hillserve::half_value(h); }
std::uint16_t ref_half_bits(float f) { return hillserve::half_bits(f); }

// FullGqaCpuScorer(threads, implementation) -- policy/full_gqa_cpu.hpp:27-50.
// implementation: 0 automatic, 1 scalar, 2 avx2_f16c.
void* ref_scorer_create(unsigned threads, int implementation, char* err, std::size_t errlen) {
    try {
        return new hillserve::FullGqaCpuScorer(
            threads, static_cast<hillserve::FullGqaCpuImplementation>(implementation));
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return nullptr;
    }
}
void ref_scorer_destroy(void* scorer) { delete static_cast<hillserve::FullGqaCpuScorer*>(scorer); }
const char* ref_scorer_name(void* scorer) {
    return static_cast<hillserve::FullGqaCpuScorer*>(scorer)->implementation_name();
}

// score(query, views, output); views given as parallel arrays.  out receives
// 32*sum(tokens) scores, head-major.
int ref_scorer_score(void* scorer, const std::uint16_t* q, const std::uint16_t* const* data,
                     const std::size_t* tokens, const std::size_t* strides, std::size_t nviews,
                     std::uint16_t* out, std::size_t out_capacity, char* err, std::size_t errlen) {
    try {
        static thread_local std::vector<std::uint16_t> query, output;
        query.assign(q, q + 4096);
        std::vector<hillserve::FullGqaKeyView> views(nviews);
        for (std::size_t i = 0; i < nviews; ++i) views[i] = {data[i], tokens[i], strides[i]};
        static_cast<hillserve::FullGqaCpuScorer*>(scorer)->score(query, views, output);
        if (output.size() > out_capacity) throw std::runtime_error("bridge output capacity");
        std::memcpy(out, output.data(), output.size() * 2);
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}

// score_full_gqa_legacy_cpu -- policy/full_gqa_cpu.cpp:109-138
int ref_legacy_score(const std::uint16_t* q, const std::uint16_t* k, std::size_t n,
                     std::size_t stride, unsigned threads, std::uint16_t* out, char* err,
                     std::size_t errlen) {
    try {
        std::vector<std::uint16_t> query(q, q + 4096);
        auto result = hillserve::score_full_gqa_legacy_cpu(query, k, n, stride, threads);
        std::memcpy(out, result.data(), result.size() * 2);
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}

// The runtime's score scaling -- policy/full_gqa_runtime.cpp:571
void ref_scale(const std::uint16_t* raw, std::size_t count, std::uint16_t* out) {
    for (std::size_t i = 0; i < count; ++i)
        out[i] = hillserve::half_bits(hillserve::half_value(raw[i]) / std::sqrt(128.f));
}

// select_gqa_scores -- policy/gqa_policy.hpp:19-21.  ids is [heads][kcap].
int ref_select(const std::uint16_t* scaled, std::size_t heads, std::size_t stride,
               std::size_t valid, float alpha, float ratio, int fp32_counts, std::uint64_t* ids,
               std::size_t kcap, std::uint32_t* counts, std::size_t* k_out,
               std::size_t* tied_out, char* err, std::size_t errlen) {
    try {
        std::vector<std::uint16_t> scores(scaled, scaled + heads * stride);
        auto s = hillserve::policy::select_gqa_scores(scores, heads, stride, valid, alpha, ratio,
                                                      fp32_counts != 0);
        if (s.k > kcap) throw std::runtime_error("bridge ids capacity");
        for (std::size_t h = 0; h < heads; ++h) {
            counts[h] = s.counts[h];
            for (std::size_t j = 0; j < s.k; ++j) ids[h * kcap + j] = s.ids[h][j];
        }
        *k_out = s.k;
        *tied_out = s.boundary_tied_heads;
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}

// gqa_physical_union -- runtime/gqa_pack.hpp:12-22
int ref_union(const std::uint64_t* ids, std::size_t kstride, const std::size_t* sizes,
              std::size_t visible, std::uint64_t* physical, std::size_t* count, char* err,
              std::size_t errlen) {
    try {
        std::vector<std::vector<std::uint64_t>> heads(32);
        for (std::size_t h = 0; h < 32; ++h)
            heads[h].assign(ids + h * kstride, ids + h * kstride + sizes[h]);
        auto u = hillserve::gqa_physical_union(heads, visible);
        std::memcpy(physical, u.data(), u.size() * 8);
        *count = u.size();
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}

// pack_gqa_workspace -- runtime/gqa_pack.hpp:26-58
int ref_pack(const std::uint64_t* ids, std::size_t kstride, const std::size_t* sizes,
             const std::uint64_t* positions, std::size_t npos, const std::uint64_t* physical,
             std::size_t nphys, const std::uint8_t* payload, std::size_t payload_bytes,
             std::size_t count, std::uint16_t* k, std::uint16_t* v, float* mask, char* err,
             std::size_t errlen) {
    try {
        std::vector<std::vector<std::uint64_t>> heads(32);
        for (std::size_t h = 0; h < 32; ++h)
            heads[h].assign(ids + h * kstride, ids + h * kstride + sizes[h]);
        std::vector<std::uint64_t> pos(positions, positions + npos), phys(physical, physical + nphys);
        std::vector<std::uint8_t> bytes(payload, payload + payload_bytes);
        hillserve::pack_gqa_workspace(heads, pos, phys, bytes, count, k, v, mask);
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}

// H2OResidency -- policy/h2o_residency.hpp:16-77, the CPU consumer of the
// H2O group sums and the reference's CPU path for them (observe_attention).
void* ref_h2o_create(std::size_t layers, std::size_t query_heads, std::size_t kv_heads,
                     std::size_t prompt_tokens, std::size_t generated_capacity,
                     std::size_t prompt_resident_tokens_per_head, std::uint64_t budget, char* err,
                     std::size_t errlen) {
    try {
        hillserve::policy::H2OResidency::Config c;
        c.layers = layers;
        c.query_heads = query_heads;
        c.kv_heads = kv_heads;
        c.prompt_tokens = prompt_tokens;
        c.generated_capacity = generated_capacity;
        c.prompt_resident_tokens_per_head = prompt_resident_tokens_per_head;
        c.metadata_budget_bytes = budget;
        return new hillserve::policy::H2OResidency(c);
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return nullptr;
    }
}
void ref_h2o_destroy(void* h) { delete static_cast<hillserve::policy::H2OResidency*>(h); }
int ref_h2o_observe_attention(void* h, std::size_t layer, std::size_t first, std::size_t queries,
                              std::size_t keys, const float* p, std::size_t elements, char* err,
                              std::size_t errlen) {
    try {
        static_cast<hillserve::policy::H2OResidency*>(h)->observe_attention(layer, first, queries, keys, p,
                                                                            elements);
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
int ref_h2o_observe_group_sums(void* h, std::size_t layer, std::size_t first, std::size_t queries,
                               std::size_t keys, const float* sums, std::size_t elements, char* err,
                               std::size_t errlen) {
    try {
        static_cast<hillserve::policy::H2OResidency*>(h)->observe_group_sums(layer, first, queries, keys, sums,
                                                                             elements);
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
// importance(layer, head, position) for positions [0, count) of every KV head.
int ref_h2o_importance(void* h, std::size_t layer, std::size_t kv_heads, std::size_t count, float* out,
                       char* err, std::size_t errlen) {
    try {
        auto* r = static_cast<hillserve::policy::H2OResidency*>(h);
        for (std::size_t kh = 0; kh < kv_heads; ++kh)
            for (std::size_t k = 0; k < count; ++k) out[kh * count + k] = r->importance(layer, kh, k);
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
// resident_ids(layer): head h's IDs at out[h * stride ...], sizes[h].
int ref_h2o_resident_ids(void* h, std::size_t layer, std::uint64_t* out, std::size_t stride,
                         std::size_t* sizes, char* err, std::size_t errlen) {
    try {
        auto ids = static_cast<hillserve::policy::H2OResidency*>(h)->resident_ids(layer);
        for (std::size_t kh = 0; kh < ids.size(); ++kh) {
            if (ids[kh].size() > stride) throw std::runtime_error("bridge resident capacity");
            std::memcpy(out + kh * stride, ids[kh].data(), ids[kh].size() * 8);
            sizes[kh] = ids[kh].size();
        }
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}

// checksum -- storage/file_store.cpp:12-16
std::uint64_t ref_checksum(const void* data, std::size_t n) { return hillserve::checksum(data, n); }
// checksum_four -- storage/kv_checksum.hpp:11-23
int ref_checksum_four(const unsigned char* const* rows, std::size_t bytes, std::size_t count, std::uint64_t* out,
                      char* err, std::size_t errlen) {
    try {
        std::array<const unsigned char*, 4> r{};
        for (std::size_t i = 0; i < count && i < 4; ++i) r[i] = rows[i];
        const auto h = hillserve::storage::checksum_four(r, bytes, count);
        for (std::size_t i = 0; i < count; ++i) out[i] = h[i];
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
// plan_kv_reads -- storage/kv_read_plan.hpp:34-59; windows as 5 u64 each.
int ref_read_plan(const std::uint64_t* offsets, std::size_t count, std::uint64_t record_bytes,
                  std::uint64_t extent, std::size_t window_bytes, std::size_t gap_bytes, unsigned amplification,
                  std::uint64_t* windows, std::size_t capacity, std::size_t* n, char* err, std::size_t errlen) {
    try {
        std::vector<hillserve::storage::KVReadRecord> records(count);
        for (std::size_t i = 0; i < count; ++i) records[i] = {offsets[i], i};
        hillserve::storage::KVReadLimits limits;
        limits.window_bytes = window_bytes;
        limits.gap_bytes = gap_bytes;
        limits.max_amplification_permille = amplification;
        const auto w = hillserve::storage::plan_kv_reads(records, record_bytes, extent, limits);
        if (w.size() > capacity) throw std::runtime_error("bridge window capacity");
        for (std::size_t i = 0; i < w.size(); ++i) {
            windows[5 * i + 0] = w[i].begin;
            windows[5 * i + 1] = w[i].end;
            windows[5 * i + 2] = w[i].required_page_bytes;
            windows[5 * i + 3] = w[i].first_record;
            windows[5 * i + 4] = w[i].end_record;
        }
        *n = w.size();
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
// SegmentedKVStore (storage/segmented_store.cpp): creates the store file at
// `path`, appends per layer l the `counts[l]` records of payload rows
// payload[l] (record_bytes each, positions 0..), drains, then (optionally)
// XORs one byte of the file at mutate_offset (when >= 0) and fetches `nids`
// positions of `fetch_layer` into out.  The file stays for the caller.
int ref_segment_roundtrip(const char* path, std::uint64_t request, std::size_t layers, std::uint64_t positions,
                          std::size_t record_bytes, std::uint64_t quota, const unsigned char* const* payload,
                          const std::uint64_t* counts, long long mutate_offset, unsigned char mutate_xor,
                          std::size_t fetch_layer, const std::uint64_t* ids, std::size_t nids, unsigned char* out,
                          char* err, std::size_t errlen) {
    try {
        hillserve::SegmentedKVStore store(path, request, layers, positions, record_bytes, quota);
        for (std::size_t l = 0; l < layers; ++l) {
            if (!counts[l]) continue;
            std::vector<std::uint8_t> rows(payload[l], payload[l] + counts[l] * record_bytes);
            store.append(l, 0, rows);
        }
        store.drain();
        if (mutate_offset >= 0) {
            const int fd = open(path, O_RDWR | O_CLOEXEC);
            if (fd < 0) throw std::runtime_error("bridge reopen");
            unsigned char b = 0;
            const bool ok = pread(fd, &b, 1, mutate_offset) == 1 && (b ^= mutate_xor, pwrite(fd, &b, 1, mutate_offset) == 1);
            close(fd);
            if (!ok) throw std::runtime_error("bridge mutate");
        }
        if (nids) {
            std::vector<std::uint64_t> want(ids, ids + nids);
            const auto data = store.fetch(fetch_layer, want, nids * record_bytes);
            std::memcpy(out, data.data(), data.size());
        }
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
// The runtime's integrity loop (policy/full_gqa_runtime.cpp:394-408): the
// digests of `count` payloads at base + offsets[i], four at a time through
// checksum_four; bench.py times it as the reference's CPU cost.
void ref_checksum_records(const unsigned char* base, const std::uint64_t* offsets, std::size_t count,
                          std::size_t bytes, std::uint64_t* out) {
    for (std::size_t j = 0; j < count; j += 4) {
        const std::size_t n = std::min<std::size_t>(4, count - j);
        std::array<const unsigned char*, 4> rows{};
        for (std::size_t k = 0; k < n; ++k) rows[k] = base + offsets[j + k];
        const auto h = hillserve::storage::checksum_four(rows, bytes, n);
        for (std::size_t k = 0; k < n; ++k) out[j + k] = h[k];
    }
}
// plan_full_gqa_runtime's placement (runtime/full_gqa_contract.hpp:110-185)
// with budgets large enough to pass; writes hot_slot_by_position [capacity].
int ref_plan_hot_slots(std::uint64_t capacity, std::uint64_t prompt, std::uint64_t generated, double beta,
                       int allow_partial, std::int64_t* out, std::uint64_t* hot_tokens, char* err,
                       std::size_t errlen) {
    try {
        hillserve::runtime::FullGqaRuntimeSpec s;
        s.layers = 32;
        s.capacity = capacity;
        s.prompt_tokens = prompt;
        s.generated_capacity = generated;
        s.allow_partial_prompt = allow_partial != 0;
        s.beta = beta;
        s.hot_kv_budget_bytes = ~0ull >> 2;
        s.total_host_workspace_budget_bytes = ~0ull >> 1;
        s.fp32_selection_counts = capacity > 65536;
        const auto p = hillserve::runtime::plan_full_gqa_runtime(s);
        std::memcpy(out, p.hot_slot_by_position.data(), capacity * 8);
        *hot_tokens = p.prompt_hot_tokens;
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
}
