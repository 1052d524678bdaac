// Drop-in for runtime/gqa_pack.hpp (:12-58): the physical union of the 32
// per-head selections and the packing of payload rows into the delivery
// layout K [slot][32][128], V [32][128][slot], mask [32][qpad][slot], computed
// on the GPU (hsb_union, hsb_pack) with the reference's bits, checks and
// std::invalid_argument messages.  k, v and mask are host buffers, as in the
// reference; use hsb_pack directly to keep them in device memory.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>
// The reference header defines these functions inline and so brings in the
// following standard headers; translation units written against it may rely
// on them.
#include <algorithm>
#include <cstring>
#include <limits>
#include <stdexcept>

namespace hillserve {
std::vector<std::uint64_t> gqa_physical_union(const std::vector<std::vector<std::uint64_t>>& ids,
                                               std::size_t visible);

void pack_gqa_workspace(const std::vector<std::vector<std::uint64_t>>& ids,
                        const std::vector<std::uint64_t>& positions, const std::vector<std::uint64_t>& physical,
                        const std::vector<std::uint8_t>& payload, std::size_t count, std::uint16_t* k,
                        std::uint16_t* v, float* mask);
}  // namespace hillserve
