// host_checks.cpp -- the argument checks of the path's C++ interfaces,
// exercised without a GPU.
//
// Built twice by tests/test_compat_host_checks.py from this one source: with
// hillserve_b200/compat first on the include path and linked to
// libhsb_compat, and against the reference's own headers and sources.  Every
// case passes arguments that the interface must reject before doing any
// work; the program prints one line per case -- the exception's class and
// message -- and the two builds' outputs must be identical.  (Valid calls
// would need a GPU in the drop-in build, so none is made.)
#include <cfenv>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

#include "policy/full_gqa_cpu.hpp"
#include "policy/gqa_policy.hpp"
#include "runtime/gqa_pack.hpp"

using namespace hillserve;

namespace {
int cases = 0;

void expect_throw(const char* name, const std::function<void()>& f) {
    ++cases;
    try {
        f();
        std::printf("%s|no exception\n", name);
    } catch (const std::invalid_argument& e) {
        std::printf("%s|invalid_argument|%s\n", name, e.what());
    } catch (const std::runtime_error& e) {
        std::printf("%s|runtime_error|%s\n", name, e.what());
    } catch (const std::exception& e) {
        std::printf("%s|exception|%s\n", name, e.what());
    }
}

using Ids = std::vector<std::vector<std::uint64_t>>;
}  // namespace

int main() {
    const float nan = std::numeric_limits<float>::quiet_NaN(), inf = std::numeric_limits<float>::infinity();
    const std::size_t big = std::numeric_limits<std::size_t>::max();

    // FullGqaCpuScorer construction (policy/full_gqa_cpu.cpp).
    expect_throw("scorer threads 0", [] { FullGqaCpuScorer s(0); });
    expect_throw("scorer threads 129", [] { FullGqaCpuScorer s(129); });
    expect_throw("scorer implementation 99",
                 [] { FullGqaCpuScorer s(1, static_cast<FullGqaCpuImplementation>(99)); });
    expect_throw("scorer threads 0 and implementation 99",
                 [] { FullGqaCpuScorer s(0, static_cast<FullGqaCpuImplementation>(99)); });
    std::fesetround(FE_DOWNWARD);
    expect_throw("scorer rounding mode", [] { FullGqaCpuScorer s(2); });
    expect_throw("scorer rounding mode and threads 0", [] { FullGqaCpuScorer s(0); });
    std::fesetround(FE_TONEAREST);

    // score_full_gqa_legacy_cpu.
    std::vector<std::uint16_t> q(32 * 128), short_q(100), keys(4 * 2048);
    expect_throw("legacy query size", [&] { score_full_gqa_legacy_cpu(short_q, keys.data(), 4, 1024, 1); });
    expect_throw("legacy null input", [&] { score_full_gqa_legacy_cpu(q, nullptr, 4, 1024, 1); });
    expect_throw("legacy zero tokens", [&] { score_full_gqa_legacy_cpu(q, keys.data(), 0, 1024, 1); });
    expect_throw("legacy stride 999", [&] { score_full_gqa_legacy_cpu(q, keys.data(), 4, 999, 1); });
    expect_throw("legacy threads 0", [&] { score_full_gqa_legacy_cpu(q, keys.data(), 4, 1024, 0); });
    expect_throw("legacy threads 33", [&] { score_full_gqa_legacy_cpu(q, keys.data(), 4, 2048, 33); });
    expect_throw("legacy extent overflow", [&] { score_full_gqa_legacy_cpu(q, keys.data(), big / 16, 1024, 1); });
    std::fesetround(FE_UPWARD);
    expect_throw("legacy rounding mode", [&] { score_full_gqa_legacy_cpu(q, keys.data(), 4, 1024, 1); });
    expect_throw("legacy rounding mode and stride 999",
                 [&] { score_full_gqa_legacy_cpu(q, keys.data(), 4, 999, 1); });
    std::fesetround(FE_TONEAREST);

    // select_gqa_scores (policy/gqa_policy.cpp:47-49).
    std::vector<std::uint16_t> scores(32 * 64, 0x3c00);
    using policy::select_gqa_scores;
    expect_throw("select heads 0", [&] { select_gqa_scores(scores, 0, 64, 64, 0.1f, 0.2f); });
    expect_throw("select heads 129", [&] { select_gqa_scores(scores, 129, 64, 64, 0.1f, 0.2f); });
    expect_throw("select valid 0", [&] { select_gqa_scores(scores, 32, 64, 0, 0.1f, 0.2f); });
    expect_throw("select valid above stride", [&] { select_gqa_scores(scores, 32, 64, 65, 0.1f, 0.2f); });
    expect_throw("select score size", [&] { select_gqa_scores(scores, 32, 63, 63, 0.1f, 0.2f); });
    expect_throw("select alpha NaN", [&] { select_gqa_scores(scores, 32, 64, 64, nan, 0.2f); });
    expect_throw("select alpha negative", [&] { select_gqa_scores(scores, 32, 64, 64, -0.5f, 0.2f); });
    expect_throw("select alpha infinite", [&] { select_gqa_scores(scores, 32, 64, 64, inf, 0.2f); });
    expect_throw("select ratio 0", [&] { select_gqa_scores(scores, 32, 64, 64, 0.1f, 0.0f); });
    expect_throw("select ratio above 1", [&] { select_gqa_scores(scores, 32, 64, 64, 0.1f, 1.5f); });
    expect_throw("select ratio NaN", [&] { select_gqa_scores(scores, 32, 64, 64, 0.1f, nan); });
    expect_throw("select shape and alpha NaN", [&] { select_gqa_scores(scores, 0, 64, 64, nan, 0.2f); });

    // gqa_physical_union / pack_gqa_workspace (runtime/gqa_pack.hpp).
    Ids ids(32, std::vector<std::uint64_t>{1, 2}), ids31(31, std::vector<std::uint64_t>{1});
    expect_throw("union 31 heads", [&] { gqa_physical_union(ids31, 8); });
    expect_throw("union visible 0", [&] { gqa_physical_union(ids, 0); });
    expect_throw("union visible 66049", [&] { gqa_physical_union(ids, 66049); });
    std::vector<std::uint64_t> positions{5}, physical{1, 2};
    std::vector<std::uint8_t> payload(2 * 4096);
    std::vector<std::uint16_t> k(8 * 4096), v(8 * 4096);
    std::vector<float> mask(8 * 64 * 32);
    auto pack = [&](const Ids& i, const std::vector<std::uint64_t>& pos, const std::vector<std::uint8_t>& pl,
                    std::size_t count) { pack_gqa_workspace(i, pos, physical, pl, count, k.data(), v.data(), mask.data()); };
    expect_throw("pack 31 heads", [&] { pack(ids31, positions, payload, 8); });
    expect_throw("pack no positions", [&] { pack(ids, {}, payload, 8); });
    expect_throw("pack 257 positions", [&] { pack(ids, std::vector<std::uint64_t>(257, 5), payload, 8); });
    expect_throw("pack last position 66048", [&] { pack(ids, {66048}, payload, 8); });
    expect_throw("pack count 0", [&] { pack(ids, positions, payload, 0); });
    expect_throw("pack count 66049", [&] { pack(ids, positions, payload, 66049); });
    expect_throw("pack payload size", [&] { pack(ids, positions, std::vector<std::uint8_t>(4096), 8); });

    std::printf("cases|%d\n", cases);
    return 0;
}
