// C++ drop-in tests: the reference's own interfaces (policy/full_gqa_cpu.hpp,
// policy/gqa_policy.hpp, runtime/gqa_pack.hpp, runtime/gqa_prefetch_cuda.hpp,
// runtime/gqa_delivery.hpp, runtime/gqa_h2o_stats.hpp), included by their
// reference paths and backed by the B200 kernels.  The checks follow the
// reference unit tests (tests/full_gqa_cpu_tests.cpp, tests/gqa_policy_tests.cpp,
// tests/gqa_pack_tests.cpp, tests/gqa_h2o_stats_tests.cu) with independent
// scalar oracles written here.
// Prints one JSON status line; exit code 0 on success.
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cfenv>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <limits>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "policy/full_gqa_cpu.hpp"
#include "policy/gqa_policy.hpp"
#include "policy/host_policy.hpp"
#include "runtime/gqa_delivery.hpp"
#include "runtime/gqa_h2o_stats.hpp"
#include "runtime/gqa_pack.hpp"
#include "runtime/gqa_prefetch_cuda.hpp"

using namespace hillserve;
using u16 = std::uint16_t;
using u64 = std::uint64_t;

namespace {
void need(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error("check failed: " + what);
}
template <class Ex, class F>
void throws(F f, const std::string& what) {
    bool hit = false;
    try {
        f();
    } catch (const Ex&) {
        hit = true;
    }
    need(hit, "expected exception: " + what);
}

// xorshift32 stream and random finite F16 values, as the reference scorer test draws them.
struct Xs {
    std::uint32_t s;
    std::uint32_t operator()() {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        return s;
    }
};
u16 finite_half(Xs& r) {
    static const u16 edge[] = {0, 0x8000, 1, 0x8001, 0x03ff, 0x83ff, 0x0400, 0x8400,
                               0x3c00, 0xbc00, 0x7bff, 0xfbff, 0x3555, 0xb555};
    const auto w = r();
    return w % 5 == 0 ? edge[(w >> 8) % 14] : u16((w & 0x83ff) | (((w >> 10) % 31) << 10));
}

// Scalar oracle: every product rounded, channels added in order from +0.
std::vector<u16> oracle_scores(const std::vector<u16>& q, const std::vector<const u16*>& rows) {
    const auto n = rows.size();
    std::vector<u16> out(32 * n);
    for (std::size_t h = 0; h < 32; ++h)
        for (std::size_t t = 0; t < n; ++t) {
            volatile float acc = 0.0f;
            for (std::size_t c = 0; c < 128; ++c) {
                volatile float p = half_value(q[h * 128 + c]) * half_value(rows[t][(h / 4) * 128 + c]);
                acc = acc + p;
            }
            out[h * n + t] = half_bits(acc);
        }
    return out;
}

std::size_t scorer_tests() {
    std::size_t compared = 0;
    Xs rng{0x7f123451u};
    for (unsigned threads : {1u, 2u, 7u}) {
        FullGqaCpuScorer scorer(threads);
        need(scorer.threads() == threads, "thread count");
        for (std::size_t n : {1u, 2u, 7u, 8u, 9u, 17u, 65u, 129u})
            for (std::size_t stride : {1024u, 2048u}) {
                std::vector<u16> q(4096), data(n * stride, 0x7e00);
                for (auto& x : q) x = finite_half(rng);
                for (std::size_t t = 0; t < n; ++t)
                    for (std::size_t c = 0; c < 1024; ++c) data[t * stride + c] = finite_half(rng);
                std::vector<const u16*> rows;
                for (std::size_t t = 0; t < n; ++t) rows.push_back(data.data() + t * stride);
                std::vector<u16> out;
                scorer.score(q, {{data.data(), n, stride}}, out);
                need(out == oracle_scores(q, rows), "scores n=" + std::to_string(n));
                compared += out.size();
                auto flipped = q;
                for (auto& x : flipped) x ^= 0x8000;
                scorer.score(flipped, {{data.data(), n, stride}}, out);
                need(out == oracle_scores(flipped, rows), "second call");
                if (n >= 9) {
                    std::vector<const u16*> mixed = {rows[7], rows[8], rows[0], rows[1], rows[2], rows[1]};
                    scorer.score(q, {{data.data() + 7 * stride, 2, stride}, {data.data(), 3, stride},
                                     {data.data() + stride, 1, stride}},
                                 out);
                    need(out == oracle_scores(q, mixed), "mixed views");
                }
            }
        // subnormal minimum, exact cancellation, overflow, negative zero
        std::vector<u16> q(4096, 1), data(9 * 1024, 1);
        std::vector<const u16*> rows;
        for (std::size_t t = 0; t < 9; ++t) rows.push_back(data.data() + t * 1024);
        std::vector<u16> out;
        scorer.score(q, {{data.data(), 9, 1024}}, out);
        need(out == oracle_scores(q, rows), "subnormals");
        for (std::size_t i = 0; i < q.size(); ++i) q[i] = i % 2 ? 0xfbff : 0x7bff;
        std::fill(data.begin(), data.end(), 0x7bff);
        scorer.score(q, {{data.data(), 9, 1024}}, out);
        need(out == oracle_scores(q, rows), "cancellation");
        std::fill(q.begin(), q.end(), 0x7bff);
        scorer.score(q, {{data.data(), 9, 1024}}, out);
        need(out == oracle_scores(q, rows), "overflow");
        std::fill(q.begin(), q.end(), 0x8000);
        scorer.score(q, {{data.data(), 9, 1024}}, out);
        need(out == oracle_scores(q, rows), "negative zero");
    }
    throws<std::invalid_argument>([] { FullGqaCpuScorer s(0); }, "0 threads");
    throws<std::invalid_argument>([] { FullGqaCpuScorer s(129); }, "129 threads");
    throws<std::invalid_argument>([] { FullGqaCpuScorer s(1, static_cast<FullGqaCpuImplementation>(99)); }, "impl");
    FullGqaCpuScorer scorer(2);
    std::vector<u16> q(4096), key(1024), out;
    throws<std::invalid_argument>([&] { scorer.score({}, {{key.data(), 1, 1024}}, out); }, "empty q");
    throws<std::invalid_argument>([&] { scorer.score(q, {}, out); }, "no views");
    throws<std::invalid_argument>([&] { scorer.score(q, {{nullptr, 1, 1024}}, out); }, "null view");
    throws<std::invalid_argument>([&] { scorer.score(q, {{key.data(), 0, 1024}}, out); }, "zero tokens");
    throws<std::invalid_argument>([&] { scorer.score(q, {{key.data(), 1, 1}}, out); }, "stride");
    throws<std::invalid_argument>(
        [&] { scorer.score(q, {{key.data(), std::numeric_limits<std::size_t>::max(), 1024}}, out); }, "extent");
    throws<std::invalid_argument>([&] { scorer.score(q, {{key.data(), 1, 1024}}, q); }, "alias");
    std::fesetround(FE_DOWNWARD);
    throws<std::invalid_argument>([] { FullGqaCpuScorer s(2); }, "rounding ctor");
    throws<std::invalid_argument>([&] { scorer.score(q, {{key.data(), 1, 1024}}, out); }, "rounding score");
    std::fesetround(FE_TONEAREST);
    // the legacy entry point computes the same bits
    std::vector<u16> qq(4096), kk(65 * 2048);
    for (auto& x : qq) x = finite_half(rng);
    for (auto& x : kk) x = finite_half(rng);
    std::vector<const u16*> rows;
    for (std::size_t t = 0; t < 65; ++t) rows.push_back(kk.data() + t * 2048);
    need(score_full_gqa_legacy_cpu(qq, kk.data(), 65, 2048, 4) == oracle_scores(qq, rows), "legacy");
    throws<std::invalid_argument>([&] { score_full_gqa_legacy_cpu(qq, kk.data(), 65, 2048, 33); }, "legacy threads");
    return compared;
}

void selector_tests() {
    using policy::select_gqa_scores;
    std::vector<u16> s;
    for (float x : {10.f, 9.f, 8.f, 7.f, 1.f, 1.f, 1.f, 1.f}) s.push_back(half_bits(x));
    auto r = select_gqa_scores(s, 2, 4, 4, 2.f, 1.f);
    need(r.counts == std::vector<std::uint32_t>({3, 0}) && r.k == 1, "head0 broadcast + inclusive");
    need(r.ids[0][0] == 0 && r.ids[1][0] == 0, "ID ties");
    std::vector<u16> pad(16, half_bits(1000));
    for (std::size_t h = 0; h < 2; ++h)
        for (std::size_t t = 0; t < 5; ++t) pad[h * 8 + t] = half_bits(float(t));
    r = select_gqa_scores(pad, 2, 8, 5, 10, .4f);
    need(r.k == 2 && r.ids[0] == std::vector<u64>({4, 3}), "padding excluded");
    std::vector<u16> many(2049, half_bits(0));
    r = select_gqa_scores(many, 1, 2049, 2049, 0, 1);
    need(r.counts[0] == 2049 && r.k == 2048, "F16 count 2049 -> 2048");
    need(select_gqa_scores(many, 1, 2049, 2049, 0, 1, true).k == 2049, "FP32 count extension");
    std::vector<u16> lng(131072, half_bits(-10));
    lng.back() = half_bits(1);
    r = select_gqa_scores(lng, 1, lng.size(), lng.size(), 0, 1);
    need(r.k == 1 && r.ids[0][0] == 131071, "long IDs");
    std::vector<u16> over(65520, half_bits(0));
    throws<std::runtime_error>([&] { select_gqa_scores(over, 1, over.size(), over.size(), 0, 1); }, "F16 overflow");
    r = select_gqa_scores(over, 1, over.size(), over.size(), 0, .2f, true);
    need(r.counts[0] == 65520 && r.k == 13104 && r.ids[0].front() == 0 && r.ids[0].back() == 13103, "FP32 cap");
    throws<std::runtime_error>([&] { select_gqa_scores(s, 0, 4, 4, 1, .2f); }, "heads 0");
    throws<std::runtime_error>([&] { select_gqa_scores(s, 2, 4, 4, -1, .2f); }, "alpha < 0");
    std::mt19937 rng(1741);
    for (int trial = 0; trial < 8; ++trial) {
        const std::size_t heads = 32, n = 257, stride = 288;
        std::vector<u16> in(heads * stride, half_bits(1000));
        for (std::size_t h = 0; h < heads; ++h)
            for (std::size_t t = 0; t < n; ++t)
                in[h * stride + t] = (t % 17 == 0) ? u16(t % 2 ? 0 : 0x8000)
                                                   : half_bits(float(int(rng() % 97) - 48) / 2);
        const auto sel = select_gqa_scores(in, heads, stride, n, 10, .2f);
        for (std::size_t h = 0; h < heads; ++h) {
            std::vector<u64> want(n);
            std::iota(want.begin(), want.end(), 0);
            std::stable_sort(want.begin(), want.end(), [&](u64 a, u64 b) {
                return half_value(in[h * stride + a]) > half_value(in[h * stride + b]);
            });
            want.resize(sel.k);
            need(want == sel.ids[h], "ordered IDs vs full sort");
        }
    }
}

void pack_tests() {
    std::vector<std::vector<u64>> ids(32, {8, 12});
    ids[4] = {12, 8};
    std::vector<u64> physical = {8, 12};
    std::vector<u16> raw(4096);
    for (std::size_t t = 0; t < 2; ++t)
        for (std::size_t h = 0; h < 8; ++h)
            for (std::size_t d = 0; d < 128; ++d) {
                raw[t * 2048 + h * 128 + d] = u16(1000 * t + 100 * h + d);
                raw[t * 2048 + 1024 + h * 128 + d] = u16(5000 + 1000 * t + 100 * h + d);
            }
    std::vector<std::uint8_t> payload(raw.size() * 2);
    std::memcpy(payload.data(), raw.data(), payload.size());
    std::vector<u16> k(32 * 4096), v(k.size());
    std::vector<float> mask(32 * 64 * 32);
    pack_gqa_workspace(ids, {10, 12}, physical, payload, 32, k.data(), v.data(), mask.data());
    need(k[0] == 0 && k[4096] == 1000 && k[4 * 128] == 1100 && k[4096 + 4 * 128] == 100, "K values");
    need(v[(4 * 128) * 32] == 6100 && v[(4 * 128) * 32 + 1] == 5100, "V values");
    need(k[2 * 4096 + 127] == 0 && v[127 * 32 + 2] == 0, "zero padding");
    need(mask[0] == 0 && std::isinf(mask[1]) && mask[32 + 1] == 0, "mask causal");
    need(std::isinf(mask[(4 * 64) * 32]) && mask[(4 * 64) * 32 + 1] == 0 && std::isinf(mask[2 * 32]), "mask head 4");
    auto bad = ids;
    bad[0] = {13};
    throws<std::invalid_argument>(
        [&] { pack_gqa_workspace(bad, {12}, physical, payload, 32, k.data(), v.data(), mask.data()); }, "future ID");
    std::mt19937 rng(781);
    for (int trial = 0; trial < 12; ++trial) {
        const std::size_t n = 65 + trial * 4, slots = (n + 31) / 32 * 32;
        std::vector<u64> rows(n);
        std::iota(rows.begin(), rows.end(), 0);
        std::shuffle(rows.begin(), rows.end(), rng);
        std::vector<std::uint8_t> bytes(n * 4096);
        for (auto& x : bytes) x = std::uint8_t(rng());
        std::vector<std::vector<u64>> sel(32);
        for (auto& head : sel) {
            head = rows;
            if (trial % 2) head.resize(1 + rng() % n);
            std::shuffle(head.begin(), head.end(), rng);
        }
        std::vector<u64> queries{n / 2, n - 1};
        std::vector<u16> gk(slots * 4096), gv(gk.size()), rk(gk.size(), 0), rv(gk.size(), 0);
        std::vector<float> gm(slots * 64 * 32), rm(gm.size(), -std::numeric_limits<float>::infinity());
        for (std::size_t h = 0; h < 32; ++h)
            for (std::size_t s = 0; s < sel[h].size(); ++s) {
                const auto id = sel[h][s];
                const auto row = std::size_t(std::find(rows.begin(), rows.end(), id) - rows.begin());
                const auto* src = bytes.data() + row * 4096;
                for (std::size_t d = 0; d < 128; ++d) {
                    std::memcpy(&rk[s * 4096 + h * 128 + d], src + (h / 4 * 128 + d) * 2, 2);
                    std::memcpy(&rv[(h * 128 + d) * slots + s], src + 2048 + (h / 4 * 128 + d) * 2, 2);
                }
                for (std::size_t qi = 0; qi < queries.size(); ++qi)
                    if (id <= queries[qi]) rm[(h * 64 + qi) * slots + s] = 0;
            }
        pack_gqa_workspace(sel, queries, rows, bytes, slots, gk.data(), gv.data(), gm.data());
        need(gk == rk && gv == rv && gm == rm, "random pack trial");
        auto u = gqa_physical_union(sel, n);
        std::vector<u64> want;
        for (const auto& h : sel) want.insert(want.end(), h.begin(), h.end());
        std::sort(want.begin(), want.end());
        want.erase(std::unique(want.begin(), want.end()), want.end());
        need(u == want, "union");
        sel[31].push_back(sel[31].front());
        throws<std::invalid_argument>([&] { gqa_physical_union(sel, n); }, "duplicate in head");
    }
}

void prefetch_and_delivery_tests() {
    const std::size_t rows = 40, count = 32;
    void* anchor = nullptr;
    need(cudaMalloc(&anchor, 256) == cudaSuccess, "device anchor");
    GQAPrefetchCuda pf(anchor, rows);
    std::mt19937 rng(5);
    std::vector<std::uint8_t> pre(20 * 4096), miss(5 * 4096);
    for (auto& x : pre) x = std::uint8_t(rng());
    for (auto& x : miss) x = std::uint8_t(rng());
    auto up = pf.stage(1, pre);
    need(up.bytes == pre.size(), "upload bytes");
    std::vector<std::int32_t> map(count * 32);
    for (auto& m : map) m = int(rng() % 26) - 6;  // -6..19: misses, padding, prefetched
    void *dk, *dv, *dm;
    need(cudaMalloc(&dk, count * 4096 * 2) == cudaSuccess && cudaMalloc(&dv, count * 4096 * 2) == cudaSuccess &&
             cudaMalloc(&dm, 4) == cudaSuccess,
         "outputs");
    cudaStream_t s;
    cudaStreamCreate(&s);
    pf.deliver(1, map, miss, nullptr, 0, count, dk, dv, dm, s);
    std::vector<u16> gk(count * 4096), gv(gk.size());
    cudaMemcpy(gk.data(), dk, gk.size() * 2, cudaMemcpyDeviceToHost);
    cudaMemcpy(gv.data(), dv, gv.size() * 2, cudaMemcpyDeviceToHost);
    for (std::size_t s2 = 0; s2 < count; ++s2)
        for (std::size_t h = 0; h < 32; ++h)
            for (std::size_t d = 0; d < 128; ++d) {
                const auto row = map[h * count + s2];
                u16 kv = 0, vv = 0;
                if (row != -1) {
                    const auto* src = reinterpret_cast<const u16*>(row >= 0 ? pre.data() + std::size_t(row) * 4096
                                                                            : miss.data() + std::size_t(-2 - row) * 4096);
                    kv = src[(h / 4) * 128 + d];
                    vv = src[1024 + (h / 4) * 128 + d];
                }
                need(gk[(s2 * 32 + h) * 128 + d] == kv && gv[(h * 128 + d) * count + s2] == vv, "gather map");
            }
    map[3] = 20;  // beyond the 20 uploaded rows
    throws<std::runtime_error>([&] { pf.deliver(1, map, miss, nullptr, 0, count, dk, dv, dm, s); }, "row bounds");
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dm);
    cudaFree(anchor);
    cudaStreamDestroy(s);

    std::vector<float> q(4096);
    for (auto& x : q) x = float(int(rng() % 200) - 100) / 100.f;
    GQADeliveryWorkspace ws(64, q);
    std::vector<std::vector<u64>> ids(32);
    std::vector<u64> physical = {1, 4, 7, 9};
    for (auto& h : ids) h = {9, 4, 1};
    std::vector<std::uint8_t> payload(physical.size() * 4096);
    std::vector<u16> words(payload.size() / 2);
    for (auto& w : words) w = half_bits(float(int(rng() % 100) - 50) / 50.f);
    std::memcpy(payload.data(), words.data(), payload.size());
    ws.deliver(ids, 9, physical, payload);
    const auto report = ws.verify_and_consume();
    need(report.find("attention_output_checksum") != std::string::npos, "report");
    for (float x : ws.output()) need(std::isfinite(x), "finite attention");
}

// tests/gqa_h2o_stats_tests.cu:39-95: a strided [11, 6, 32, 1] F32 tensor with
// holes between keys and NaN in every byte that is not a valid probability;
// blocks (first 0, 3 queries) and (first 3, 2 queries); the sums must equal a
// scalar F32 sum in (Q head, query) order, bit for bit.
void h2o_tests() {
    const std::array<std::int64_t, 4> ne{{11, 6, 32, 1}};
    const std::array<std::size_t, 4> nb{{8, 112, 704, 22528}};
    std::vector<float> storage(nb[3] / sizeof(float));
    void* gpu = nullptr;
    cudaStream_t stream = nullptr;
    if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&gpu, nb[3]) != cudaSuccess)
        throw std::runtime_error("H2O fixture allocation");
    struct Free {
        void* g;
        cudaStream_t s;
        ~Free() {
            cudaStreamSynchronize(s);
            cudaFree(g);
            cudaStreamDestroy(s);
        }
    } guard{gpu, stream};
    GQAH2OStatsCuda reducer(gpu, 7);
    need(reducer.gpu_bytes() == 8 * 7 * sizeof(float) && reducer.host_bytes() == 8 * 7 * sizeof(float),
         "H2O buffers bounded by 8 x capacity");
    for (std::size_t first : {0u, 3u}) {
        const std::size_t queries = first == 0 ? 3 : 2, keys = first + queries;
        std::fill(storage.begin(), storage.end(), std::numeric_limits<float>::quiet_NaN());
        std::vector<float> dense(32 * queries * keys, 0.f);
        for (std::size_t h = 0; h < 32; ++h)
            for (std::size_t q = 0; q < queries; ++q) {
                const std::size_t available = first + q + 1;
                double total = 0;
                for (std::size_t k = 0; k < available; ++k) total += 1 + (k + h / 4) % 5;
                for (std::size_t k = 0; k < keys; ++k) {
                    const float x = k < available ? float((1 + (k + h / 4) % 5) / total) : 0.f;
                    storage[(h * nb[2] + q * nb[1] + k * nb[0]) / sizeof(float)] = x;
                    dense[(h * queries + q) * keys + k] = x;
                }
            }
        if (cudaMemcpyAsync(gpu, storage.data(), nb[3], cudaMemcpyHostToDevice, stream) != cudaSuccess)
            throw std::runtime_error("H2O fixture upload");
        const auto r = reducer.reduce(gpu, ne, nb, keys, queries, stream);
        need(r.sums && r.elements == 8 * keys && r.d2h_bytes == 8 * keys * sizeof(float), "H2O result shape");
        need(r.ready_observed_ns >= r.started_ns && r.reduction_ms >= 0 && r.d2h_ms >= 0, "H2O timings");
        for (std::size_t kh = 0; kh < 8; ++kh)
            for (std::size_t k = 0; k < keys; ++k) {
                float want = 0.f;
                for (std::size_t lane = 0; lane < 4; ++lane)
                    for (std::size_t q = 0; q < queries; ++q) want += dense[((kh * 4 + lane) * queries + q) * keys + k];
                std::uint32_t a, b;
                std::memcpy(&a, &r.sums[kh * keys + k], 4);
                std::memcpy(&b, &want, 4);
                need(a == b, "H2O strided F32 group sum");
            }
    }
    auto heads = ne;
    heads[2] = 8;
    throws<std::runtime_error>([&] { reducer.reduce(gpu, heads, nb, 5, 2, stream); }, "non-GQA32 head shape");
    auto streams = ne;
    streams[3] = 2;
    throws<std::runtime_error>([&] { reducer.reduce(gpu, streams, nb, 5, 2, stream); }, "multi-sequence shape");
    throws<std::runtime_error>([&] { reducer.reduce(gpu, ne, nb, 8, 2, stream); }, "capacity overrun");
    throws<std::runtime_error>([&] { reducer.reduce(gpu, ne, nb, 5, 7, stream); }, "padding query overrun");
    throws<std::runtime_error>([&] { reducer.reduce(gpu, ne, nb, 5, 2, nullptr); }, "missing attention stream");
    std::vector<float> host(16);
    throws<std::runtime_error>([&] { GQAH2OStatsCuda bad(host.data(), 4); }, "host pointer as reference");
    throws<std::runtime_error>([&] { reducer.reduce(host.data(), ne, nb, 5, 2, stream); }, "host probabilities");
}
}  // namespace

int main() {
    try {
        const auto compared = scorer_tests();
        selector_tests();
        pack_tests();
        prefetch_and_delivery_tests();
        h2o_tests();
        std::cout << "{\"status\":\"passed\",\"bitwise_scores_compared\":" << compared << "}" << std::endl;
        return 0;
    } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
        return 1;
    }
}
