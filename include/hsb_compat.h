/*
 * hsb_compat.h -- C handles over the C++ drop-in classes of libhsb_compat.so,
 * for C and ctypes callers that cannot hold a C++ object (the reference's
 * Python tooling).  Each call behaves exactly as the class method it wraps;
 * an exception becomes a nonzero return with its message copied to err.
 */
#ifndef HSB_COMPAT_H
#define HSB_COMPAT_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* hillserve::GQAH2OStatsCuda (runtime/gqa_h2o_stats.hpp:12-45). */
void* hsb_compat_h2o_create(const void* actual_gpu_pointer, size_t capacity_keys, char* err, size_t errlen);
void hsb_compat_h2o_destroy(void* reducer);
/* reduce(): on success *sums points at the pinned host sums (8 * valid_keys
 * floats, borrowed until the next reduce or destroy). */
int hsb_compat_h2o_reduce(void* reducer, const void* probabilities, const int64_t ne[4], const size_t nb[4],
                          size_t valid_keys, size_t valid_queries, void* actual_attention_stream,
                          const float** sums, double* reduction_ms, double* d2h_ms, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif
