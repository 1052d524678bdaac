/*
 * hs_oracle.h -- CPU ORACLE FOR TESTS ONLY.
 *
 * This is test infrastructure, not product code.  It restates, in plain C,
 * the reference HillServe algorithms of the selected-KV decode path so that
 * the CUDA implementation can be checked against them.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it, and
 * only as a checker.  Product code never links or calls it.
 *
 * Parity pinning: every function here is checked against (a) the known-answer
 * vectors of the reference's own tests and (b) outputs of the reference's own
 * C++ code compiled from its sources (oracle/Makefile -> oracle/_ref/), on
 * seeded inputs (tests/golden/make_golden.py).  The two functions whose
 * reference runs in ggml (attention, rehearsal GEMV+RoPE) are "parity
 * unpinned": they are double-precision restatements of the documented math.
 *
 * Citations are paths inside the reference project.
 */
#ifndef HS_ORACLE_H
#define HS_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Error codes.  Values equal the HSB_E* codes of include/hsb.h so tests can
 * compare them directly; each names the reference exception it stands for. */
enum {
    ORC_OK = 0,
    ORC_E_SCORE_SHAPE = 10,       /* full_gqa_cpu.cpp:214-222 */
    ORC_E_SEL_SHAPE = 20,         /* gqa_policy.cpp:48 "GQA selector shape" */
    ORC_E_SEL_PARAMS = 21,        /* gqa_policy.cpp:49 "GQA selector numeric parameters" */
    ORC_E_SEL_NONFINITE_HEAD0 = 22, /* gqa_policy.cpp:54 "nonfinite head0 score" */
    ORC_E_SEL_THRESHOLD = 23,     /* gqa_policy.cpp:55 "F16 threshold overflow" */
    ORC_E_SEL_NONFINITE = 24,     /* gqa_policy.cpp:57 "nonfinite GQA score" */
    ORC_E_SEL_U32 = 25,           /* gqa_policy.cpp:58 "threshold count exceeds u32" */
    ORC_E_SEL_COUNT_F16 = 26,     /* gqa_policy.cpp:59 "public F16 count overflow ..." */
    ORC_E_SEL_MEAN_F16 = 27,      /* gqa_policy.cpp:61 "public F16 mean overflow ..." */
    ORC_E_SEL_CAPACITY = 28,      /* oracle-only: ids buffer smaller than k */
    ORC_E_UNION_BOUNDS = 30,      /* gqa_pack.hpp:14 "GQA union bounds" */
    ORC_E_UNION_DUPLICATE = 31,   /* gqa_pack.hpp:17 "GQA duplicate/future selected ID" */
    ORC_E_PACK_SHAPE = 40,        /* gqa_pack.hpp:29-30 "GQA packing shape" */
    ORC_E_PACK_PHYSICAL = 41,     /* gqa_pack.hpp:33 "duplicate/future physical position" */
    ORC_E_PACK_SLOTS = 42,        /* gqa_pack.hpp:41 "per-head selection exceeds slots" */
    ORC_E_PACK_MISSING = 43,      /* gqa_pack.hpp:44 "future or missing selected KV" */
    ORC_E_MAP_GEOMETRY = 50,      /* gqa_prefetch_cuda.cu:217 */
    ORC_E_MAP_ROW = 51,           /* gqa_prefetch_cuda.cu:218 prefetch row outside payload */
    ORC_E_MAP_MISS = 52,          /* gqa_prefetch_cuda.cu:218 miss row outside payload */
    ORC_E_COVER_RANGE = 60,       /* full_gqa_runtime.cpp:316-317 */
    ORC_E_COVER_THRESHOLD = 61,   /* full_gqa_runtime.cpp:323 */
    ORC_E_COVER_COUNT = 62,       /* full_gqa_runtime.cpp:330 */
    ORC_E_COVER_MEAN = 63         /* full_gqa_runtime.cpp:333 */
};

/* binary16 <-> binary32, policy/host_policy.cpp:9-28 */
float orc_half_value(uint16_t h);
uint16_t orc_half_bits(float f);
/* policy/half_order.hpp:7-10 */
uint16_t orc_order_key(uint16_t bits);

/* V3 scoring, policy/full_gqa_cpu.cpp:23-37 (scalar tile) and the volatile
 * scalar oracle of tests/full_gqa_cpu_tests.cpp:28-44.  Scores tokens
 * [0,n) of one view whose token t starts at k + t*stride_words, writing
 * out[h*out_stride + col0 + t].  threads<=1 runs on the calling thread. */
int orc_score(const uint16_t* q, const uint16_t* k, size_t n, size_t stride_words,
              uint16_t* out, size_t out_stride, size_t col0, int threads);

/* F16 division by sqrtf(128), policy/full_gqa_runtime.cpp:571 */
void orc_scale(const uint16_t* raw, size_t count, uint16_t* scaled);

/* select_gqa_scores, policy/gqa_policy.cpp:47-70.  ids is [heads][kcap]. */
int orc_select(const uint16_t* scaled, size_t heads, size_t stride, size_t valid,
               float alpha, float ratio, int fp32_counts, uint64_t* ids, size_t kcap,
               uint32_t* counts, size_t* k_out, size_t* tied_heads_out);

/* gqa_physical_union, runtime/gqa_pack.hpp:12-22.  ids is [32][kstride]
 * with sizes[h] valid entries per head. */
int orc_union(const uint64_t* ids, size_t kstride, const size_t* sizes, size_t visible,
              uint64_t* physical, size_t* physical_count);

/* pack_gqa_workspace, runtime/gqa_pack.hpp:26-58 */
int orc_pack(const uint64_t* ids, size_t kstride, const size_t* sizes,
             const uint64_t* positions, size_t npositions,
             const uint64_t* physical, size_t nphysical,
             const uint8_t* payload, size_t payload_bytes, size_t count,
             uint16_t* k, uint16_t* v, float* mask);

/* gather_gqa + deliver's row checks, runtime/gqa_prefetch_cuda.cu:12-22,217-218 */
int orc_gather_map(const uint16_t* prefetched, size_t prefetched_rows,
                   const uint16_t* misses, size_t miss_rows,
                   const int32_t* map, size_t count, uint16_t* k, uint16_t* v);

/* prefetch cover, policy/full_gqa_runtime.cpp:299-344.  raw is the raw
 * (unscaled) score matrix [32][capacity]; per_head is [32][cap] where
 * cap=min(position, floor((position+1)*0.2f)). */
int orc_prefetch_cover(const uint16_t* raw, size_t capacity, size_t position,
                       float alpha, int fp32_counts, uint64_t* per_head, size_t* bound_out,
                       uint64_t* physical, size_t* physical_count);

/* Attention over the packed workspace (parity unpinned: ggml graph of
 * runtime/gqa_delivery.cpp:19-20), double precision.  k [count,32,128],
 * v [32,128,count], mask [32,qpad,count] (query row 0 is used), q [32,128]. */
void orc_attention_packed(const uint16_t* k, const uint16_t* v, const float* mask,
                          size_t count, size_t qpad, const float* q, double* out);

/* Attention over per-head compact slot lists (live slots only, no mask):
 * head h attends slots [0,lengths[h]) of the packed layout above. */
void orc_attention_compact(const uint16_t* k, const uint16_t* v, size_t count,
                           const uint32_t* lengths, const float* q, double* out);

/* Dense decode attention over a token-major cache (layers 0-1,
 * runtime/gqa_executor.cpp:174-176): K,V [n, 8, 128] at stride_words. */
void orc_attention_dense(const uint16_t* kc, const uint16_t* vc, size_t n,
                         size_t stride_words, const float* q, double* out);

/* Rehearsal query (parity unpinned: ggml mul_mat + rope_ext NORM mode,
 * patches/llama-b6000-round2.patch:308-314).  x bf16[4096],
 * w bf16[4096 out][4096 in], q_out[4096] = RoPE_pos(W x). */
void orc_rehearsal(const uint16_t* x_bf16, const uint16_t* w_bf16, uint64_t position,
                   double theta, double* q_out);

/* Timed CPU baseline only (stage 4 has no reference CPU code): float,
 * multithreaded ports of the ggml attention graph. */
void orc_attention_dense_f32(const uint16_t* kc, const uint16_t* vc, size_t n, size_t stride,
                             const float* q, float* out, int threads);
void orc_attention_packed_f32(const uint16_t* k, const uint16_t* v, const float* mask,
                              size_t count, size_t qpad, const float* q, float* out, int threads);

/* H2O residency statistics, runtime/gqa_h2o_stats.cu:41-57
 * (sum_actual_attention).  probabilities: bytes of an F32 tensor [key][query]
 * [Q head] with byte strides nb0, nb1, nb2; out[kv * keys + key] = F32 sum,
 * from +0, over Q heads 4kv..4kv+3 (outer) and queries 0..queries-1 (inner).
 * The same order as H2OResidency::observe_attention (h2o_residency.cpp:66-76). */
void orc_h2o_group_sums(const void* probabilities, size_t keys, size_t queries, size_t nb0, size_t nb1,
                        size_t nb2, float* out);

/* Cold-tier KV records (SegmentedKVStore v1).
 * FNV-1a 64, storage/file_store.cpp:12-16. */
uint64_t orc_fnv1a64(const void* data, size_t n);
/* The bytes SegmentedKVStore::append writes for records (layer, first + i),
 * storage/segmented_store.cpp:95-104: {digest, position, request, layer,
 * version 1} then the payload, count * (record_bytes + 32) bytes. */
void orc_kv_records_encode(const void* payload, size_t payload_stride, size_t count, size_t record_bytes,
                           uint64_t request, uint32_t layer, uint64_t first, void* records);
/* Checks records at window + offsets[i] and copies their payloads to
 * out + row * out_stride (row = out_rows ? out_rows[i] : i), walking the
 * reference's validation loop (policy/full_gqa_runtime.cpp:394-409):
 * records in validation groups (groups[i]; NULL: one per record), each
 * group's identity checks before its checksums.  Returns 0 or the first
 * error (90 identity, 91 checksum, 92 bounds) and its record index. */
int orc_kv_records_verify(const void* window, size_t window_bytes, const uint64_t* offsets,
                          const uint64_t* positions, const uint32_t* groups, size_t count, uint64_t request,
                          uint32_t layer, size_t record_bytes, void* out, size_t out_stride,
                          const uint32_t* out_rows, size_t out_capacity, uint32_t* error_index);

/* Synthetic benchmark inputs, restating the library's generator
 * (hsb_synth_normal_f16/_bf16, hsb_synth_keys in include/hsb.h) bit for bit:
 * splitmix64 counters, Box-Muller in double precision with series for ln,
 * e^x and sin/cos of 2 pi x, RNE to F32 then F16 / BF16.  Keys: heavy rows
 * by hash, NORM-mode RoPE by token position.  threads <= 128. */
void orc_synth_normal(uint16_t* out, size_t count, uint64_t seed, float stddev, int bf16, int threads);
void orc_synth_keys(uint16_t* rows, size_t tokens, size_t stride_words, uint64_t seed, float heavy_fraction,
                    float heavy_scale, int rope, float theta, int threads);

#ifdef __cplusplus
}
#endif
#endif
