// The binary16 conversions of policy/host_policy.hpp (:7-8) that callers of
// the selected-KV path use: exact widening and round-to-nearest-even
// narrowing (overflow to infinity, canonical quiet NaN keeping the sign).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace hillserve {
float half_value(std::uint16_t);
std::uint16_t half_bits(float);

// The partial-key policy's interface (policy/host_policy.hpp:9-19). It is not
// part of the selected-KV path and this library does not implement it: the
// declarations are here, unchanged, so that code using it still compiles with
// this directory first on the include path, and its definitions stay in the
// reference's policy/host_policy.cpp.  That file also defines half_value and
// half_bits, the same conversions as the library's.
struct PolicySelection {
    std::size_t k = 0, boundary_tied_heads = 0;
    std::vector<std::uint64_t> ids;  // [q_head][k], original token IDs
    std::vector<std::uint32_t> above_threshold;
};
std::vector<std::uint16_t> host_partial_scores(const std::vector<std::uint16_t>& q,
                                               const std::vector<std::uint16_t>& keys, std::size_t heads,
                                               std::size_t tokens, std::size_t channels);
PolicySelection select_partial_scores(const std::vector<std::uint16_t>& scores, std::size_t heads,
                                      std::size_t tokens, float alpha, std::size_t cap, bool inclusive = false);
}  // namespace hillserve
