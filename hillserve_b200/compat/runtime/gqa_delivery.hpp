// Drop-in for runtime/gqa_delivery.hpp (:10-19): owns the device K/V/mask
// workspace of `count` slots and the attention over it.  The reference packs
// on the host, uploads with ggml and runs a ggml graph; here the packing
// (hsb_pack) and the attention (hsb_attention_packed) are sm_100a kernels,
// so there is no ggml dependency.  verify_and_consume() returns its report
// as a JSON string (the reference returns an nlohmann::ordered_json).
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace hillserve {
struct GQADeliveryResult {
    double pack_ms = 0, upload_wall_ms = 0, cuda_copy_stream_interval_ms = 0;
    std::uint64_t gpu_ready_ns = 0, upload_bytes = 0;
};
class GQADeliveryWorkspace {
    struct Impl;
    std::unique_ptr<Impl> p;

public:
    GQADeliveryWorkspace(std::size_t count, const std::vector<float>& actual_attention_query);
    ~GQADeliveryWorkspace();
    GQADeliveryResult deliver(const std::vector<std::vector<std::uint64_t>>& ids, std::uint64_t query_position,
                              const std::vector<std::uint64_t>& physical, const std::vector<std::uint8_t>& payload);
    // Runs the attention and returns {"attention_output_checksum", ...} as JSON.
    std::string verify_and_consume();
    // The F32 [32][128] attention output of the last verify_and_consume().
    const std::vector<float>& output() const;
    std::uint64_t gpu_bytes() const;
};
}  // namespace hillserve
