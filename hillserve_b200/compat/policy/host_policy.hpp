// The binary16 conversions of policy/host_policy.hpp (:7-8) that callers of
// the selected-KV path use: exact widening and round-to-nearest-even
// narrowing (overflow to infinity, canonical quiet NaN keeping the sign).
#pragma once
#include <cstdint>

namespace hillserve {
float half_value(std::uint16_t);
std::uint16_t half_bits(float);
}  // namespace hillserve
