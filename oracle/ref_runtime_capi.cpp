// ref_runtime_capi.cpp -- TEST INFRASTRUCTURE ONLY (see hs_oracle.h).
//
// A C bridge to the reference's FullGqaRuntimePolicy, compiled unchanged from
// its sources by oracle/Makefile (policy/full_gqa_runtime.cpp and what it
// links: full_gqa_cpu, gqa_policy, host_policy, core/hkm, core/app_partition,
// storage/{segmented_store,file_store}, smartssd/adapter).  It drives one
// layer of one request through the reference's own decode protocol -- prompt
// append, then per step prepare_history (payload prefetch on, so the cover of
// full_gqa_runtime.cpp:299-344 is published as an artifact), the current
// token's append, select (:549-585) and fetch (:586-690) -- and records the
// cover and the final selections, so tests can pin the library's cover and
// decode history to the reference's outputs.  Files go to a caller-given
// scratch directory.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <memory>
#include <mutex>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "policy/full_gqa_runtime.hpp"
#include "runtime/full_gqa_contract.hpp"
#include "runtime/gqa_prefetch.hpp"
#include "storage/segmented_store.hpp"

namespace {
void put_error(const std::exception& e, char* err, std::size_t errlen) {
    if (err && errlen) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = 0;
    }
}
}  // namespace

extern "C" {
// rows: [capacity][2048] F16 bits (K[8][128] then V[8][128]) of `layer`.
// rehearsal: [steps][4096] F32 selection queries.  Per step s (position
// prompt + s): cover_bound[s] = the cover's per-head bound, cover_ids[s][32]
// [cap_max] its per-head lists, phys[s][phys_max] / phys_count[s] its sorted
// physical IDs, is_cold[s][phys_max] whether the policy reads them from the
// cold tier, final_k[s] and final_ids[s][32][k_max] the selection.
int ref_runtime_decode(const char* dir, std::size_t capacity, std::size_t prompt, std::size_t steps, int layer,
                       double beta, float alpha, const std::uint16_t* rows, const float* rehearsal,
                       std::uint64_t* cover_bound, std::uint64_t* cover_ids, std::size_t cap_max,
                       std::uint64_t* phys, std::uint64_t* phys_count, std::uint8_t* is_cold, std::size_t phys_max,
                       std::uint64_t* final_k, std::uint64_t* final_ids, std::size_t k_max, char* err,
                       std::size_t errlen) {
    using namespace hillserve;
    using namespace hillserve::policy;
    using namespace hillserve::runtime;
    try {
        const std::filesystem::path root(dir);
        std::filesystem::create_directories(root);
        const std::size_t layers = 32;
        const auto extent = full_gqa_align_page(4096 + layers * capacity * 4128ULL);
        SegmentedKVStore store(root / "kv", 4242, layers, capacity, 4096, extent);
        store.enable_direct_writes(root / "kv");
        FullGqaRuntimePolicy::Config c;
        c.layers = layers;
        c.capacity = capacity;
        c.prompt_tokens = prompt;
        c.generated_capacity = steps;
        c.beta = beta;
        c.selector_alpha = alpha;
        c.hot_kv_budget_bytes = layers * capacity * 4096ULL;
        c.total_host_workspace_budget_bytes = 8ULL << 30;
        c.chunk_tokens = 64;
        c.hot_threads = 1;
        c.cold_threads = 1;
        c.score_file = (root / "raw-k").string();
        c.payload_prefetch = true;
        c.full_kv_backing_path = (root / "kv").string();
        c.full_kv_io_fence = std::make_shared<GQAPrefetchIOFence>();
        FullGqaRuntimePolicy policy(c);
        auto append = [&](std::uint64_t first, std::size_t n) {
            std::vector<std::uint8_t> kv(n * 4096);
            std::memcpy(kv.data(), rows + first * 2048, kv.size());
            std::vector<std::uint16_t> keys(n * 1024);
            for (std::size_t t = 0; t < n; ++t) std::memcpy(keys.data() + t * 1024, rows + (first + t) * 2048, 2048);
            std::vector<std::uint64_t> positions(n);
            std::iota(positions.begin(), positions.end(), first);
            {
                std::lock_guard<std::mutex> lock(c.full_kv_io_fence->file_io);
                store.append(layer, first, kv);
            }
            policy.append(layer, positions, keys, kv);
        };
        append(0, prompt);
        for (std::size_t s = 0; s < steps; ++s) {
            const std::uint64_t position = prompt + s;
            const std::vector<float> q(rehearsal + s * 4096, rehearsal + (s + 1) * 4096);
            std::shared_ptr<const GQAPrefetchArtifact> artifact;
            std::mutex mu;
            policy.prepare_history(layer, position, q, [&](std::shared_ptr<const GQAPrefetchArtifact> a) {
                std::lock_guard<std::mutex> lock(mu);
                artifact = std::move(a);
            });
            append(position, 1);
            const auto selected = policy.select(layer, position, q);
            std::vector<std::uint64_t> physical;
            for (const auto& head : selected) physical.insert(physical.end(), head.begin(), head.end());
            std::sort(physical.begin(), physical.end());
            physical.erase(std::unique(physical.begin(), physical.end()), physical.end());
            policy.fetch(layer, physical, {});  // joins the payload read and the callback
            std::lock_guard<std::mutex> lock(mu);
            if (!artifact) throw std::runtime_error("bridge: no prefetch artifact was published");
            const std::size_t bound = artifact->per_head_ids.empty() ? 0 : artifact->per_head_ids[0].size();
            if (bound > cap_max || artifact->physical_ids.size() > phys_max)
                throw std::runtime_error("bridge: cover larger than the output buffers");
            cover_bound[s] = bound;
            for (std::size_t h = 0; h < 32; ++h) {
                const auto& ids = artifact->per_head_ids[h];
                if (ids.size() != bound) throw std::runtime_error("bridge: per-head cover sizes differ");
                std::copy(ids.begin(), ids.end(), cover_ids + (s * 32 + h) * cap_max);
            }
            phys_count[s] = artifact->physical_ids.size();
            for (std::size_t i = 0; i < artifact->physical_ids.size(); ++i) {
                phys[s * phys_max + i] = artifact->physical_ids[i];
                is_cold[s * phys_max + i] = policy.is_hot(layer, artifact->physical_ids[i]) ? 0 : 1;
            }
            const std::size_t k = selected.empty() ? 0 : selected[0].size();
            if (k > k_max) throw std::runtime_error("bridge: selection larger than the output buffer");
            final_k[s] = k;
            for (std::size_t h = 0; h < 32; ++h)
                std::copy(selected[h].begin(), selected[h].end(), final_ids + (s * 32 + h) * k_max);
        }
        policy.drain();
        store.drain();
        return 0;
    } catch (const std::exception& e) {
        put_error(e, err, errlen);
        return 1;
    }
}
}
