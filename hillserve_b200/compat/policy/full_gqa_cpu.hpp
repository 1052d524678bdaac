// Drop-in for policy/full_gqa_cpu.hpp of HillServe (policy/full_gqa_cpu.hpp:1-50):
// same namespace, types and member functions; the scoring runs on the B200
// through the C ABI of include/hsb.h (hsb_score_views) with identical bits.
//
// Views may point at host memory (as in the reference; the K rows are staged
// to the GPU per call) or at CUDA device memory (scored in place, no copy).
// Errors keep the reference's exception types and messages.
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

namespace hillserve {
// Fixed V3 scoring contract: 32 Q heads, 8 physical KV heads, 128 channels.
// F16 inputs; channels 0..127 accumulated in order in FP32 from +0; one final
// round-to-nearest-even F16 score; head-major output.
enum class FullGqaCpuImplementation { automatic, scalar, avx2_f16c };
inline constexpr char full_gqa_legacy_cpu_name[] = "legacy_software_half_per_call_threads";
// Same arithmetic as the pooled scorer; `threads` is validated (1..32) as the
// reference does and otherwise unused on the GPU.
std::vector<std::uint16_t> score_full_gqa_legacy_cpu(const std::vector<std::uint16_t>& query,
                                                     const std::uint16_t* input, std::size_t tokens,
                                                     std::size_t token_stride_words, unsigned threads);

struct FullGqaKeyView {
    const std::uint16_t* data = nullptr;
    std::size_t tokens = 0;
    std::size_t token_stride_words = 1024;
};

class FullGqaCpuScorer {
public:
    explicit FullGqaCpuScorer(unsigned threads,
                              FullGqaCpuImplementation implementation = FullGqaCpuImplementation::automatic);
    ~FullGqaCpuScorer();
    FullGqaCpuScorer(const FullGqaCpuScorer&) = delete;
    FullGqaCpuScorer& operator=(const FullGqaCpuScorer&) = delete;
    // Synchronous; calls on one instance are serialised.  Output is resized
    // to 32 * sum(tokens) scores, head-major.
    void score(const std::vector<std::uint16_t>& query, const std::vector<FullGqaKeyView>& views,
               std::vector<std::uint16_t>& output);
    unsigned threads() const noexcept;
    const char* implementation_name() const noexcept;
    // Device staging + host pinned bytes held between calls.
    std::size_t workspace_bytes() const noexcept;
    static bool avx2_f16c_available() noexcept;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};
}  // namespace hillserve
