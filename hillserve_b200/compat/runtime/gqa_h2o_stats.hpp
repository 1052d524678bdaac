// Drop-in for runtime/gqa_h2o_stats.hpp (:12-45): H2O residency statistics
// from the actual F32 softmax tensor, reduced on the GPU by the sm_100a
// group-sum kernels (hsb_h2o_group_sums) on the caller's attention stream,
// then copied to pinned host memory and waited for.  Same class, Result
// fields, buffer bounds (8 x capacity F32 on each side), validation order,
// exception type (std::runtime_error) and borrowing rules.
#pragma once
#include <array>
#include <cstddef>
#include <cstdint>
#include <memory>

namespace hillserve {

class GQAH2OStatsCuda {
    struct Impl;
    std::unique_ptr<Impl> impl_;

public:
    struct Result {
        const float* sums = nullptr;  // [8][valid_keys], valid until the next reduce()
        std::size_t elements = 0;
        std::uint64_t started_ns = 0;
        std::uint64_t ready_observed_ns = 0;
        std::uint64_t d2h_bytes = 0;
        double reduction_ms = 0;
        double d2h_ms = 0;
    };
    GQAH2OStatsCuda(const void* actual_gpu_pointer, std::size_t capacity_keys);
    ~GQAH2OStatsCuda();
    GQAH2OStatsCuda(const GQAH2OStatsCuda&) = delete;
    GQAH2OStatsCuda& operator=(const GQAH2OStatsCuda&) = delete;
    std::size_t gpu_bytes() const noexcept;
    std::size_t host_bytes() const noexcept;

    // ne = [key, query, Q head, stream] with ggml byte strides; B = 1 and
    // 32 query heads over 8 KV heads only.  Sums every valid query of the
    // four query heads of each KV head, in the reference's order.
    Result reduce(const void* probabilities, const std::array<std::int64_t, 4>& ne,
                  const std::array<std::size_t, 4>& byte_strides, std::size_t valid_keys,
                  std::size_t valid_queries, void* actual_attention_stream);
};

}  // namespace hillserve
