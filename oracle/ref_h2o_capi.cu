// ref_h2o_capi.cu -- TEST / BASELINE INFRASTRUCTURE ONLY.
//
// A C-ABI bridge to the reference's own GQAH2OStatsCuda
// (runtime/gqa_h2o_stats.{hpp,cu}), compiled UNMODIFIED from its sources for
// sm_100a by oracle/Makefile into oracle/_ref/libhs_ref_h2o.so.  bench.py
// times the reference's CUDA reduction beside the B200 kernels through it;
// nothing in the product links it.
#include "runtime/gqa_h2o_stats.hpp"

#include <array>
#include <cstdint>
#include <cstring>
#include <exception>

namespace {
void copy_error(const std::exception& e, char* err, std::size_t errlen) {
    if (err && errlen) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = 0;
    }
}
}  // namespace

extern "C" {
void* refh2o_create(const void* gpu_pointer, std::size_t capacity, char* err, std::size_t errlen) {
    try {
        return new hillserve::GQAH2OStatsCuda(gpu_pointer, capacity);
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return nullptr;
    }
}
void refh2o_destroy(void* r) { delete static_cast<hillserve::GQAH2OStatsCuda*>(r); }
// reduce(); copies the sums (8 * keys floats) to `sums` when non-null.
int refh2o_reduce(void* r, const void* probabilities, const std::int64_t* ne, const std::size_t* nb,
                  std::size_t keys, std::size_t queries, void* stream, float* sums, double* reduction_ms,
                  double* d2h_ms, char* err, std::size_t errlen) {
    try {
        const std::array<std::int64_t, 4> n{{ne[0], ne[1], ne[2], ne[3]}};
        const std::array<std::size_t, 4> b{{nb[0], nb[1], nb[2], nb[3]}};
        auto res = static_cast<hillserve::GQAH2OStatsCuda*>(r)->reduce(probabilities, n, b, keys, queries, stream);
        if (sums) std::memcpy(sums, res.sums, res.elements * sizeof(float));
        if (reduction_ms) *reduction_ms = res.reduction_ms;
        if (d2h_ms) *d2h_ms = res.d2h_ms;
        return 0;
    } catch (const std::exception& e) {
        copy_error(e, err, errlen);
        return -1;
    }
}
}
