// Drop-in for the selector of policy/gqa_policy.hpp (:14-21): GQASelection and
// select_gqa_scores with the reference's semantics -- head-0 maximum
// broadcast, inclusive F16 threshold, F16 count/mean rounding (or the FP32
// count extension), ratio cap, per-query-head ordered IDs with original-ID
// ties -- computed by the sm_100a selector (hsb_select).  The legacy
// partial-key GQAPolicy class of the same header is not part of this path.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

namespace hillserve::policy {
struct GQASelection {
    std::vector<std::vector<std::uint64_t>> ids;
    std::vector<std::uint32_t> counts;
    std::size_t k = 0, boundary_tied_heads = 0;
};
// Synchronous.  Throws std::runtime_error with the reference's messages.
GQASelection select_gqa_scores(const std::vector<std::uint16_t>& scaled_scores, std::size_t heads,
                               std::size_t stride, std::size_t valid_tokens, float alpha, float cap_ratio,
                               bool fp32_counts = false);
}  // namespace hillserve::policy
