// capi.cu -- the extern "C" boundary (include/hsb.h): argument validation in
// the reference's order and wording, the thread-local last-error string,
// device status read-back, and the fused selected-KV layer step.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cfenv>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"

namespace hsb {

namespace {
thread_local std::string g_last_error;

int fail(int status, const char* message) {
    g_last_error = message;
    return status;
}
int fail_cuda(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return HSB_E_CUDA;
}
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

std::mutex g_dev_mutex;
DeviceInfo g_devices[64];
// Set (release) once a device's entry is filled; a reader that sees it set
// (acquire) sees the whole entry.
std::atomic<bool> g_device_ready[64];
}  // namespace

int record_error(int status, const char* message) { return fail(status, message); }
int record_cuda_error(cudaError_t e, const char* what) { return fail_cuda(e, what); }

const DeviceInfo& device_info() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    DeviceInfo& d = g_devices[dev];
    if (!g_device_ready[dev].load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lock(g_dev_mutex);
        if (!g_device_ready[dev].load(std::memory_order_relaxed)) {
            cudaDeviceProp prop{};
            if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
                d.sms = prop.multiProcessorCount;
                d.major = prop.major;
                d.minor = prop.minor;
                d.smem_optin = prop.sharedMemPerBlockOptin;
            } else {
                d.sms = 148;
            }
            d.ordinal = dev;
            g_device_ready[dev].store(true, std::memory_order_release);
        }
    }
    return d;
}

}  // namespace hsb

using namespace hsb;

extern "C" {

int hsb_abi_version(void) { return HSB_ABI_VERSION; }
const char* hsb_last_error(void) { return g_last_error.c_str(); }

const char* hsb_status_message(int status) {
    switch (status) {
    case HSB_OK: return "";
    case HSB_E_INVALID: return "invalid argument";
    case HSB_E_CUDA: return "CUDA runtime error";
    case HSB_E_WORKSPACE: return "workspace missing or too small";
    case HSB_E_TIMEOUT: return "bounded device wait timed out";
    case HSB_E_NO_DEVICE: return "no sm_100 device";
    case HSB_E_SCORE_SHAPE: return "full GQA CPU key view shape/stride/extent";
    case HSB_E_SCORE_ALIAS: return "full GQA CPU output must not alias the query";
    case HSB_E_SCORE_V3_TOKENS: return "HS_FULL_GQA_PIPELINE_F16_V3 requires64<=N<=32768,N%64==0;no padding or fallback";
    case HSB_E_SEL_SHAPE: return "GQA selector shape";
    case HSB_E_SEL_PARAMS: return "GQA selector numeric parameters";
    case HSB_E_SEL_NONFINITE_HEAD0: return "nonfinite head0 score";
    case HSB_E_SEL_THRESHOLD: return "F16 threshold overflow";
    case HSB_E_SEL_NONFINITE: return "nonfinite GQA score";
    case HSB_E_SEL_U32: return "threshold count exceeds u32";
    case HSB_E_SEL_COUNT_F16: return "public F16 count overflow; long-count policy extension required";
    case HSB_E_SEL_MEAN_F16: return "public F16 mean overflow; long-count policy extension required";
    case HSB_E_SEL_CAPACITY: return "selected ID buffer smaller than min(floor(valid*ratio), valid)";
    case HSB_E_UNION_BOUNDS: return "GQA union bounds";
    case HSB_E_UNION_DUPLICATE: return "GQA duplicate/future selected ID";
    case HSB_E_PACK_SHAPE: return "GQA packing shape";
    case HSB_E_PACK_PHYSICAL: return "duplicate/future physical position";
    case HSB_E_PACK_SLOTS: return "per-head selection exceeds slots";
    case HSB_E_PACK_MISSING: return "future or missing selected KV";
    case HSB_E_MAP_GEOMETRY: return "prefetch CUDA delivery geometry/stream";
    case HSB_E_MAP_ROW: return "prefetch row outside uploaded payload";
    case HSB_E_MAP_MISS: return "prefetch miss row outside payload";
    case HSB_E_COVER_RANGE: return "payload prefetch historical cap/range mismatch";
    case HSB_E_COVER_THRESHOLD: return "prefetch threshold upper-bound requires finite historical threshold";
    case HSB_E_COVER_COUNT: return "prefetch count upper-bound exceeds original F16 range";
    case HSB_E_COVER_MEAN: return "prefetch mean upper-bound invalid";
    case HSB_E_ZERO_SELECTION: return "full GQA zero selection; no dense/current-token fallback";
    case HSB_E_H2O_ARGS: return "H2O reduction invalid pointer, actual CUDA stream or capacity";
    case HSB_E_H2O_SHAPE: return "H2O reduction requires [keys,queries,32,1] actual attention";
    case HSB_E_H2O_STRIDE: return "H2O reduction invalid F32 tensor stride";
    case HSB_E_H2O_OVERFLOW: return "H2O attention statistics address overflow";
    case HSB_E_H2O_ALIGN: return "H2O reduction requires aligned F32 tensor";
    case HSB_E_H2O_GRID: return "H2O reduction exceeds CUDA grid limit";
    case HSB_E_H2O_DEVICE: return "H2O softmax tensor is not on the expected CUDA device";
    case HSB_E_RECORD_IDENTITY: return "prefetch complete KV record layer/position/request mismatch";
    case HSB_E_RECORD_CHECKSUM: return "prefetch complete KV checksum mismatch";
    case HSB_E_RECORD_BOUNDS: return "complete KV record outside the uploaded window or output rows";
    case HSB_E_SEGMENT_GEOMETRY: return "bounded segmented geometry/quota";
    case HSB_E_READ_PLAN: return "invalid complete-KV read plan";
    case HSB_E_HISTORY_RESIDENCY: return "full GQA hot lookup on cold/unreserved token";
    case HSB_E_HISTORY_GEOMETRY: return "full GQA common store capacity must cover prompt+decode and align64";
    case HSB_E_HISTORY_PROTOCOL: return "full GQA history protocol violation";
    case HSB_E_HISTORY_QUERY: return "history Q/position differs from current same-query selection";
    case HSB_E_EXECUTOR_SHAPE: return "GQA current KV ABI mismatch";
    case HSB_E_EXECUTOR_NONFINITE_KV: return "GQA current model KV contains nonfinite F16";
    case HSB_E_EXECUTOR_REHEARSAL: return "full GQA rehearsal nonfinite";
    case HSB_E_EXECUTOR_REHEARSAL_F16: return "full GQA rehearsal F16 overflow";
    default: return "unknown hsb status";
    }
}

int hsb_status_check(const hsb_device_status* d_status, void* stream) {
    if (!d_status) return fail(HSB_E_INVALID, "null status");
    hsb_device_status h{};
    cudaError_t e = cudaMemcpyAsync(&h, d_status, sizeof(h), cudaMemcpyDeviceToHost, as_stream(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "status read-back");
    if (h.code) return fail(h.code, hsb_status_message(h.code));
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------------------------ stage 1
static int check_views(const hsb_key_view* views, size_t nviews, size_t* total) {
    // policy/full_gqa_cpu.cpp:214-227
    if (!views || nviews == 0) return fail(HSB_E_SCORE_SHAPE, "full GQA CPU query/views shape");
    size_t tokens = 0;
    for (size_t i = 0; i < nviews; ++i) {
        const hsb_key_view& v = views[i];
        if (!v.data || v.tokens == 0 || (v.stride_words != 1024 && v.stride_words != 2048) ||
            v.tokens > std::numeric_limits<size_t>::max() / v.stride_words ||
            v.tokens > std::numeric_limits<size_t>::max() / HSB_QUERY_HEADS - tokens)
            return fail(HSB_E_SCORE_SHAPE, "full GQA CPU key view shape/stride/extent");
        if (!aligned(v.data, 16)) return fail(HSB_E_INVALID, "key view must be 16-byte aligned");
        tokens += v.tokens;
    }
    *total = tokens;
    return HSB_OK;
}

int hsb_score_views(const uint16_t* d_q, const hsb_key_view* h_views, size_t nviews, uint16_t* d_scores,
                    void* stream) {
    if (!d_q) return fail(HSB_E_SCORE_SHAPE, "full GQA CPU query/views shape");
    if (d_scores == d_q) return fail(HSB_E_SCORE_ALIAS, "full GQA CPU output must not alias the query");
    size_t total = 0;
    int rc = check_views(h_views, nviews, &total);
    if (rc) return rc;
    if (!d_scores) return fail(HSB_E_INVALID, "null score output");
    size_t col = 0;
    for (size_t first = 0; first < nviews; first += HSB_MAX_VIEWS) {
        const size_t n = std::min<size_t>(HSB_MAX_VIEWS, nviews - first);
        cudaError_t e = launch_score(d_q, h_views + first, n, d_scores, total, col, nullptr, as_stream(stream));
        if (e != cudaSuccess) return fail_cuda(e, "score launch");
        for (size_t i = 0; i < n; ++i) col += h_views[first + i].tokens;
    }
    g_last_error.clear();
    return HSB_OK;
}

int hsb_score_v3(const uint16_t* d_q, const uint16_t* d_keys, size_t tokens, size_t stride_words,
                 uint16_t* d_scores, void* stream) {
    const hsb_key_view view{d_keys, tokens, stride_words};
    return hsb_score_views(d_q, &view, 1, d_scores, stream);
}

int hsb_score_pipeline_v3(const uint16_t* d_q, const uint16_t* d_keys, uint32_t tokens, uint16_t* d_scores,
                          void* stream) {
    // smartssd/adapter.hpp:97-104 and the kernel's own guard (kernel.cpp:237-253):
    // invalid counts are rejected before any memory access.
    if (tokens < 64 || tokens > 32768 || tokens % 64)
        return fail(HSB_E_SCORE_V3_TOKENS,
                    "HS_FULL_GQA_PIPELINE_F16_V3 requires64<=N<=32768,N%64==0;no padding or fallback");
    return hsb_score_v3(d_q, d_keys, tokens, 1024, d_scores, stream);
}

int hsb_score_with_keys(const uint16_t* d_q, const uint16_t* d_keys, size_t tokens, size_t stride_words,
                        uint16_t* d_scores, uint16_t* d_order_keys, void* stream) {
    if (!d_q) return fail(HSB_E_SCORE_SHAPE, "full GQA CPU query/views shape");
    if (d_scores == d_q || d_order_keys == d_q)
        return fail(HSB_E_SCORE_ALIAS, "full GQA CPU output must not alias the query");
    const hsb_key_view view{d_keys, tokens, stride_words};
    size_t total = 0;
    int rc = check_views(&view, 1, &total);
    if (rc) return rc;
    if (!d_scores || !d_order_keys) return fail(HSB_E_INVALID, "null score output");
    cudaError_t e = launch_score(d_q, &view, 1, d_scores, total, 0, nullptr, as_stream(stream), d_order_keys);
    if (e != cudaSuccess) return fail_cuda(e, "score launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_scale_scores(const uint16_t* d_raw, size_t count, uint16_t* d_out, void* stream) {
    if (!d_raw || !d_out) return fail(HSB_E_INVALID, "null score buffer");
    if (count == 0) return HSB_OK;
    cudaError_t e = launch_scale(d_raw, count, d_out, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "scale launch");
    return HSB_OK;
}

// ------------------------------------------------------------------ stage 2
size_t hsb_select_workspace_bytes(size_t heads, size_t stride, size_t valid, size_t kcap) {
    (void)stride;
    return select_workspace_bytes(heads, valid, kcap);
}

static int check_select(size_t heads, size_t stride, size_t valid, float alpha, float ratio) {
    // policy/gqa_policy.cpp:48-49
    if (!(heads > 0 && heads <= 128 && valid > 0 && valid <= stride))
        return fail(HSB_E_SEL_SHAPE, "GQA selector shape");
    if (!(std::isfinite(alpha) && alpha >= 0 && std::isfinite(ratio) && ratio > 0 && ratio <= 1))
        return fail(HSB_E_SEL_PARAMS, "GQA selector numeric parameters");
    if (valid > 0xffffffffull) return fail(HSB_E_SEL_SHAPE, "GQA selector shape (valid >= 2^32)");
    return HSB_OK;
}

static size_t select_kmax(size_t valid, float ratio) {
    const size_t cap = (size_t)std::floor((double)valid * (double)ratio);
    return std::min(cap, valid);
}

int hsb_select(const uint16_t* d_scores, int input_is_raw, size_t heads, size_t stride, size_t valid, float alpha,
               float ratio, int fp32_counts, uint32_t* d_ids, size_t kcap, uint32_t* d_counts,
               hsb_selection* d_result, void* d_workspace, size_t workspace_bytes, void* stream) {
    int rc = check_select(heads, stride, valid, alpha, ratio);
    if (rc) return rc;
    if (!d_scores || !d_ids || !d_result) return fail(HSB_E_INVALID, "null selector buffer");
    if (!aligned(d_result, 8)) return fail(HSB_E_INVALID, "selection result must be 8-byte aligned");
    if (kcap < select_kmax(valid, ratio)) return fail(HSB_E_SEL_CAPACITY, hsb_status_message(HSB_E_SEL_CAPACITY));
    if (!d_workspace || workspace_bytes < select_workspace_bytes(heads, valid, kcap) || !aligned(d_workspace, 256))
        return fail(HSB_E_WORKSPACE, "selector workspace missing or too small");
    SelectLaunch s{};
    s.scores = d_scores;
    s.raw = input_is_raw != 0;
    s.cover = 0;
    s.heads = (uint32_t)heads;
    s.stride = stride;
    s.valid = valid;
    s.alpha = alpha;
    s.ratio = ratio;
    s.fp32_counts = fp32_counts != 0;
    s.ids = d_ids;
    s.kcap = kcap;
    s.counts = d_counts;
    s.result = d_result;
    s.workspace = d_workspace;
    s.workspace_bytes = workspace_bytes;
    cudaError_t e = launch_select(s, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "select launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_select_keys(const uint16_t* d_order_keys, const uint16_t* d_raw, size_t heads, size_t stride, size_t valid,
                    float alpha, float ratio, int fp32_counts, uint32_t* d_ids, size_t kcap, uint32_t* d_counts,
                    hsb_selection* d_result, void* d_workspace, size_t workspace_bytes, void* stream) {
    int rc = check_select(heads, stride, valid, alpha, ratio);
    if (rc) return rc;
    if (!d_order_keys || !d_raw || !d_ids || !d_result) return fail(HSB_E_INVALID, "null selector buffer");
    if (!aligned(d_result, 8)) return fail(HSB_E_INVALID, "selection result must be 8-byte aligned");
    if (kcap < select_kmax(valid, ratio)) return fail(HSB_E_SEL_CAPACITY, hsb_status_message(HSB_E_SEL_CAPACITY));
    if (!d_workspace || workspace_bytes < select_workspace_bytes(heads, valid, kcap) || !aligned(d_workspace, 256))
        return fail(HSB_E_WORKSPACE, "selector workspace missing or too small");
    SelectLaunch s{};
    s.scores = d_order_keys;
    s.keys = 1;
    s.tie_raw = d_raw;
    s.heads = (uint32_t)heads;
    s.stride = stride;
    s.valid = valid;
    s.alpha = alpha;
    s.ratio = ratio;
    s.fp32_counts = fp32_counts != 0;
    s.ids = d_ids;
    s.kcap = kcap;
    s.counts = d_counts;
    s.result = d_result;
    s.workspace = d_workspace;
    s.workspace_bytes = workspace_bytes;
    cudaError_t e = launch_select(s, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "select launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_selection_read(const hsb_selection* d_result, hsb_selection* h_result, void* stream) {
    if (!d_result || !h_result) return fail(HSB_E_INVALID, "null selection");
    cudaError_t e = cudaMemcpyAsync(h_result, d_result, sizeof(*h_result), cudaMemcpyDeviceToHost, as_stream(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "selection read-back");
    if (h_result->status.code) return fail(h_result->status.code, hsb_status_message(h_result->status.code));
    g_last_error.clear();
    return HSB_OK;
}

int hsb_prefetch_cover(const uint16_t* d_raw, size_t capacity, size_t position, float alpha, int fp32_counts,
                       uint32_t* d_per_head, size_t cap, hsb_selection* d_result, void* d_workspace,
                       size_t workspace_bytes, void* stream) {
    // policy/full_gqa_runtime.cpp:314-317
    const size_t by_ratio = (size_t)std::floor((double)(position + 1) * (double)0.2f);
    const size_t want = std::min(position, by_ratio);
    if (!(position && position < capacity && want))
        return fail(HSB_E_COVER_RANGE, "payload prefetch historical cap/range mismatch");
    if (cap != want) return fail(HSB_E_INVALID, "per-head cover buffer stride must equal the cap");
    if (!d_raw || !d_per_head || !d_result) return fail(HSB_E_INVALID, "null cover buffer");
    if (!aligned(d_result, 8)) return fail(HSB_E_INVALID, "selection result must be 8-byte aligned");
    if (!d_workspace || workspace_bytes < select_workspace_bytes(HSB_QUERY_HEADS, position, cap) ||
        !aligned(d_workspace, 256))
        return fail(HSB_E_WORKSPACE, "cover workspace missing or too small");
    SelectLaunch s{};
    s.scores = d_raw;
    s.raw = 1;
    s.cover = 1;
    s.heads = HSB_QUERY_HEADS;
    s.stride = capacity;
    s.valid = position;
    s.alpha = alpha;
    s.ratio = 1.0f;
    s.fp32_counts = fp32_counts != 0;
    s.ids = d_per_head;
    s.kcap = cap;
    s.counts = nullptr;
    s.result = d_result;
    s.workspace = d_workspace;
    s.workspace_bytes = workspace_bytes;
    s.cover_cap = cap;
    cudaError_t e = launch_select(s, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "cover launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------------------------ stage 3
size_t hsb_union_workspace_bytes(size_t visible) { return union_workspace_bytes(visible); }

int hsb_union(const uint32_t* d_ids, size_t kstride, const uint32_t* d_sizes, size_t sizes_stride, size_t visible,
              uint32_t* d_physical, uint32_t* d_physical_count, hsb_device_status* d_status, void* d_workspace,
              size_t workspace_bytes, void* stream) {
    // runtime/gqa_pack.hpp:14
    if (!visible || visible > 66048) return fail(HSB_E_UNION_BOUNDS, "GQA union bounds");
    if (!d_ids || !d_sizes || !d_physical || !d_physical_count) return fail(HSB_E_INVALID, "null union buffer");
    if (d_status && !aligned(d_status, 8)) return fail(HSB_E_INVALID, "status must be 8-byte aligned");
    if (!d_workspace || workspace_bytes < union_workspace_bytes(visible))
        return fail(HSB_E_WORKSPACE, "union workspace missing or too small");
    cudaError_t e = launch_union(d_ids, kstride, d_sizes, sizes_stride, visible, d_physical, d_physical_count,
                                 d_status, d_workspace, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "union launch");
    g_last_error.clear();
    return HSB_OK;
}

size_t hsb_pack_workspace_bytes(uint64_t last_position) { return pack_workspace_bytes(last_position); }

int hsb_pack(const uint32_t* d_ids, size_t kstride, const uint32_t* d_sizes, size_t sizes_stride,
             const uint64_t* d_positions, size_t npositions, uint64_t last_position, const uint32_t* d_physical,
             size_t nphysical, const uint8_t* d_payload, size_t payload_bytes, size_t count, uint16_t* d_k,
             uint16_t* d_v, float* d_mask, hsb_device_status* d_status, void* d_workspace,
             size_t workspace_bytes, void* stream) {
    // runtime/gqa_pack.hpp:29-30
    if (npositions == 0 || npositions > 256 || last_position >= 66048 || !count || count > 66048 ||
        payload_bytes != nphysical * 4096)
        return fail(HSB_E_PACK_SHAPE, "GQA packing shape");
    if (!d_ids || !d_sizes || !d_k || !d_v || (nphysical && (!d_physical || !d_payload)) ||
        (d_mask && !d_positions))
        return fail(HSB_E_INVALID, "null pack buffer");
    if ((nphysical && !aligned(d_payload, 16)) || !aligned(d_k, 16) || (d_status && !aligned(d_status, 8)))
        return fail(HSB_E_INVALID, "pack buffers must be 16-byte aligned");
    if (!d_workspace || workspace_bytes < pack_workspace_bytes(last_position))
        return fail(HSB_E_WORKSPACE, "pack workspace missing or too small");
    cudaError_t e = launch_pack(d_ids, kstride, d_sizes, sizes_stride, d_positions, npositions, last_position,
                                d_physical, nphysical, d_payload, count, d_k, d_v, d_mask, d_status, d_workspace,
                                as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "pack launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_gather_map(const uint16_t* d_prefetched, size_t prefetched_rows, const uint16_t* d_misses, size_t miss_rows,
                   const int32_t* d_map, size_t count, uint16_t* d_k, uint16_t* d_v, hsb_device_status* d_status,
                   void* stream) {
    if (!d_map || !d_k || !d_v || count == 0) return fail(HSB_E_MAP_GEOMETRY, "prefetch CUDA delivery geometry/stream");
    if ((prefetched_rows && !aligned(d_prefetched, 16)) || (miss_rows && !aligned(d_misses, 16)) || !aligned(d_k, 16) ||
        (d_status && !aligned(d_status, 8)))
        return fail(HSB_E_INVALID, "gather buffers must be 16-byte aligned");
    cudaError_t e = launch_gather_map(d_prefetched, prefetched_rows, d_misses, miss_rows, d_map, count, d_k, d_v,
                                      d_status, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "gather launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_gather_cache(const uint32_t* d_ids, size_t kstride, const uint32_t* d_sizes, size_t sizes_stride,
                     const uint16_t* d_kcache, const uint16_t* d_vcache, size_t stride_words, size_t visible,
                     size_t count, int zero_padding, uint16_t* d_k, uint16_t* d_v, hsb_device_status* d_status,
                     void* stream) {
    if (!d_ids || !d_sizes || !d_kcache || !d_vcache || !d_k || !d_v || count == 0 || visible == 0 || kstride == 0)
        return fail(HSB_E_INVALID, "gather_cache arguments");
    if (stride_words % 8 || !aligned(d_kcache, 16) || !aligned(d_vcache, 16) || !aligned(d_k, 16) ||
        (d_status && !aligned(d_status, 8)))
        return fail(HSB_E_INVALID, "gather_cache buffers must be 16-byte aligned");
    cudaError_t e = launch_gather_cache(d_ids, kstride, d_sizes, sizes_stride, d_kcache, d_vcache, stride_words,
                                        visible, count, zero_padding, d_k, d_v, d_status, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "gather_cache launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_stage_rows(const uint8_t* d_rows, const uint32_t* d_physical, const uint32_t* d_count, size_t max_rows,
                   uint8_t* d_dst, void* stream) {
    if (!d_rows || !d_physical || !d_count || !d_dst) return fail(HSB_E_INVALID, "null staging buffer");
    if (!aligned(d_rows, 16) || !aligned(d_dst, 16)) return fail(HSB_E_INVALID, "staging buffers must be 16-byte aligned");
    if (max_rows == 0) return HSB_OK;
    // The row store may be device memory or pinned host memory; translate it
    // to the address the GPU uses and refuse memory the GPU cannot reach.
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, d_rows) != cudaSuccess || attr.devicePointer == nullptr) {
        cudaGetLastError();
        return fail(HSB_E_INVALID, "row store is neither device memory nor mapped pinned host memory");
    }
    const uint8_t* rows = static_cast<const uint8_t*>(attr.devicePointer);
    if (!aligned(rows, 16)) return fail(HSB_E_INVALID, "staging buffers must be 16-byte aligned");
    cudaError_t e = launch_stage_rows(rows, d_physical, d_count, max_rows, d_dst, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "stage launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------------------------ stage 4
size_t hsb_attention_workspace_bytes(size_t count) { return attention_workspace_bytes(count); }

int hsb_attention_packed(const float* d_q, const uint16_t* d_k, const uint16_t* d_v, size_t count, const float* d_mask,
                         size_t qpad, const uint32_t* d_sizes, size_t sizes_stride, float* d_out, void* d_workspace,
                         size_t workspace_bytes, void* stream) {
    if (!d_q || !d_k || !d_v || !d_out || count == 0 || (!d_mask && !d_sizes) || (d_mask && qpad == 0))
        return fail(HSB_E_INVALID, "attention arguments");
    if (!aligned(d_q, 16) || !aligned(d_k, 16) || !aligned(d_v, 16))
        return fail(HSB_E_INVALID, "attention buffers must be 16-byte aligned");
    if (!d_workspace || workspace_bytes < attention_workspace_bytes(count))
        return fail(HSB_E_WORKSPACE, "attention workspace missing or too small");
    cudaError_t e = launch_attention_packed(d_q, d_k, d_v, count, d_mask, qpad, d_sizes, sizes_stride, d_out,
                                            d_workspace, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "attention launch");
    g_last_error.clear();
    return HSB_OK;
}

size_t hsb_attention_dense_workspace_bytes(size_t tokens) { return attention_dense_workspace_bytes(tokens); }

int hsb_attention_dense(const float* d_q, const uint16_t* d_kcache, const uint16_t* d_vcache, size_t tokens,
                        size_t stride_words, float* d_out, void* d_workspace, size_t workspace_bytes, void* stream) {
    if (!d_q || !d_kcache || !d_vcache || !d_out || tokens == 0 || stride_words < 1024 || stride_words % 8)
        return fail(HSB_E_INVALID, "dense attention arguments");
    if (!aligned(d_kcache, 16) || !aligned(d_vcache, 16))
        return fail(HSB_E_INVALID, "dense attention caches must be 16-byte aligned");
    if (!d_workspace || workspace_bytes < attention_dense_workspace_bytes(tokens))
        return fail(HSB_E_WORKSPACE, "dense attention workspace missing or too small");
    cudaError_t e = launch_attention_dense(d_q, d_kcache, d_vcache, tokens, stride_words, d_out, d_workspace,
                                           as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "dense attention launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------------------- rehearsal
int hsb_rehearsal_query(const uint16_t* d_x, const uint16_t* d_w, uint64_t position, float theta, float* d_q_f32,
                        uint16_t* d_q_f16, void* stream) {
    if (!d_x || !d_w || (!d_q_f32 && !d_q_f16) || !(theta > 0.0f) || !std::isfinite(theta))
        return fail(HSB_E_INVALID, "rehearsal arguments");
    if (!aligned(d_w, 16) || !aligned(d_x, 16))
        return fail(HSB_E_INVALID, "rehearsal weights and activation must be 16-byte aligned");
    cudaError_t e = launch_rehearsal(d_x, d_w, position, theta, d_q_f32, d_q_f16, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "rehearsal launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------------------- layer step
// Layer-step workspace: selector | attention | order keys [32][valid].
static size_t align256(size_t b) { return (b + 255) / 256 * 256; }
// Layer workspace: selector | gather+attention | order keys [32][valid] |
// head-0 partials [kH0Partials].
namespace {
struct LayerLayout {
    size_t sel, att, keys, h0, total;
};
LayerLayout layer_layout(size_t valid, size_t count) {
    LayerLayout l{};
    l.sel = 0;
    l.att = align256(select_workspace_bytes(HSB_QUERY_HEADS, valid, count));
    l.keys = l.att + align256(gather_attention_workspace_bytes(count));
    l.h0 = l.keys + align256(HSB_QUERY_HEADS * valid * 2);
    l.total = l.h0 + kH0Partials * sizeof(uint32_t);
    return l;
}
}  // namespace

size_t hsb_layer_workspace_bytes(size_t valid, size_t count) { return layer_layout(valid, count).total; }

// The layer step whole, or split at the reference's prepare / select
// boundary (policy/full_gqa_runtime.cpp:493-516 scores the history ahead;
// :531-548 scores the current token inside select): kPrepare scores positions
// [0, valid - 1); kSelect scores position valid - 1 in the selector and
// completes the layer.
enum LayerPhase { kLayerWhole, kLayerPrepare, kLayerSelect };

static int layer_step(LayerPhase phase, const uint16_t* d_q16, const float* d_q32, const uint16_t* d_kcache,
                      const uint16_t* d_vcache, size_t stride_words, size_t valid, float alpha, float ratio,
                      size_t count, const hsb_layer_buffers* b, float* d_out, void* stream) {
    const bool selects = phase != kLayerPrepare;
    if (!b || !d_q16 || (selects && (!d_q32 || !d_out))) return fail(HSB_E_INVALID, "layer step arguments");
    int rc = check_select(HSB_QUERY_HEADS, valid, valid, alpha, ratio);
    if (rc) return rc;
    if (count < select_kmax(valid, ratio) || count == 0)
        return fail(HSB_E_SEL_CAPACITY, hsb_status_message(HSB_E_SEL_CAPACITY));
    if (phase != kLayerWhole && valid < 2)
        return fail(HSB_E_INVALID, "layer prepare / select: at least one history position before the current one");
    const LayerLayout lay = layer_layout(valid, count);
    if (!b->scores || !b->ids || !b->result || !b->k_packed || !b->v_packed || !b->workspace ||
        b->workspace_bytes < lay.total || !aligned(b->workspace, 256))
        return fail(HSB_E_WORKSPACE, "layer step buffers missing or too small");
    cudaStream_t s = as_stream(stream);
    const hsb_key_view view{d_kcache, valid, stride_words};
    size_t total = 0;
    if ((rc = check_views(&view, 1, &total))) return rc;
    // 16-byte row and query loads / packed stores.
    if (selects && (!d_vcache || !aligned(d_vcache, 16) || !aligned(d_q32, 16) || !aligned(b->k_packed, 16) ||
                    !aligned(b->v_packed, 16)))
        return fail(HSB_E_INVALID, "layer step: V cache, F32 query and packed buffers must be 16-byte aligned");
    if (phase == kLayerSelect && (!aligned(d_q16, 16) || !aligned(d_kcache, 16) || (stride_words * 2) % 16))
        return fail(HSB_E_INVALID, "layer select: the query and the key rows must be 16-byte aligned");
    if (phase == kLayerSelect && !select_cluster_available(valid))
        return fail(HSB_E_INVALID, "layer select: needs the cluster selector (at most 65536 positions)");
    unsigned char* ws = static_cast<unsigned char*>(b->workspace);
    uint16_t* keys = reinterpret_cast<uint16_t*>(ws + lay.keys);
    uint32_t* h0 = reinterpret_cast<uint32_t*>(ws + lay.h0);
    cudaError_t e;
    if (phase != kLayerSelect) {
        // The scorer clears what the later stages expect at zero (selector
        // header, result, attention counters) and leaves head-0 partials, so
        // the step has no memset nodes and the selector no pass over head 0's
        // row.  Prepare scores the history only: columns [0, valid - 1).
        ScoreExtras x{};
        x.h0 = h0;
        x.zero[0] = reinterpret_cast<uint32_t*>(ws + lay.sel);
        x.zero_words[0] = (unsigned)(select_header_bytes() / 4);
        x.zero[1] = reinterpret_cast<uint32_t*>(b->result);
        x.zero_words[1] = (unsigned)(sizeof(hsb_selection) / 4);
        x.zero[2] = reinterpret_cast<uint32_t*>(ws + lay.att);
        x.zero_words[2] = HSB_QUERY_HEADS;
        const hsb_key_view scored{d_kcache, phase == kLayerPrepare ? valid - 1 : valid, stride_words};
        if ((e = launch_score(d_q16, &scored, 1, b->scores, valid, 0, &b->result->status, s, keys, &x)) !=
            cudaSuccess)
            return fail_cuda(e, "score launch");
        if (phase == kLayerPrepare) {
            g_last_error.clear();
            return HSB_OK;
        }
    }
    SelectLaunch sl{};
    sl.scores = keys;
    sl.keys = 1;
    sl.tie_raw = b->scores;
    sl.raw = 0;
    sl.heads = HSB_QUERY_HEADS;
    sl.stride = valid;
    sl.valid = valid;
    sl.alpha = alpha;
    sl.ratio = ratio;
    sl.ids = b->ids;
    sl.kcap = count;
    sl.counts = b->counts;
    sl.result = b->result;
    sl.workspace = ws + lay.sel;
    sl.workspace_bytes = lay.att - lay.sel;
    sl.reset_result = 0;
    sl.reset_header = 0;
    sl.h0 = h0;
    sl.zero_is_error = 1;
    if (phase == kLayerSelect) {
        // Beside another layer's history scorer, a cooperative launch would
        // wait for the whole GPU; the selector's CTAs instead become resident
        // as that scorer's CTAs retire (which never wait on the selector), so
        // its bounded grid barrier completes without the attribute.
        sl.cooperative = 0;
        sl.cur_q = d_q16;
        sl.cur_k = d_kcache + (valid - 1) * stride_words;
        sl.cur_raw = b->scores;
    }
    // The cluster selector gathers and attends in its epilogue; otherwise a
    // separate gather + attention kernel follows.
    sl.ga.q = d_q32;
    sl.ga.kcache = d_kcache;
    sl.ga.vcache = d_vcache;
    sl.ga.stride_words = stride_words;
    sl.ga.kp = b->k_packed;
    sl.ga.vp = b->v_packed;
    sl.ga.count = count;
    sl.ga.out = d_out;
    sl.ga.scale = 1.0f / sqrtf(128.0f);
    int fused = 0;
    sl.ga_done = &fused;
    if ((e = launch_select(sl, s)) != cudaSuccess) return fail_cuda(e, "select launch");
    if (!fused &&
        (e = launch_gather_attention(d_q32, b->ids, count, &b->result->k, d_kcache, d_vcache, stride_words, valid,
                                     count, b->k_packed, b->v_packed, d_out, ws + lay.att, 0, &b->result->status,
                                     s)) != cudaSuccess)
        return fail_cuda(e, "gather-attention launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_layer_step(const uint16_t* d_q16, const float* d_q32, const uint16_t* d_kcache, const uint16_t* d_vcache,
                   size_t stride_words, size_t valid, float alpha, float ratio, size_t count,
                   const hsb_layer_buffers* b, float* d_out, void* stream) {
    return layer_step(kLayerWhole, d_q16, d_q32, d_kcache, d_vcache, stride_words, valid, alpha, ratio, count, b,
                      d_out, stream);
}

int hsb_layer_prepare(const uint16_t* d_q16, const uint16_t* d_kcache, size_t stride_words, size_t valid,
                      float alpha, float ratio, size_t count, const hsb_layer_buffers* b, void* stream) {
    return layer_step(kLayerPrepare, d_q16, nullptr, d_kcache, nullptr, stride_words, valid, alpha, ratio, count, b,
                      nullptr, stream);
}

int hsb_layer_select(const uint16_t* d_q16, const float* d_q32, const uint16_t* d_kcache, const uint16_t* d_vcache,
                     size_t stride_words, size_t valid, float alpha, float ratio, size_t count,
                     const hsb_layer_buffers* b, float* d_out, void* stream) {
    return layer_step(kLayerSelect, d_q16, d_q32, d_kcache, d_vcache, stride_words, valid, alpha, ratio, count, b,
                      d_out, stream);
}

// ------------------------------------------------------------ KV-head shards
size_t hsb_shard_head0_words(void) { return kH0Partials; }

static bool valid_kv_heads(int g) { return g == 1 || g == 2 || g == 4 || g == 8; }

int hsb_shard_score(const uint16_t* d_q, int kv_heads, const uint16_t* d_kshard, size_t tokens, size_t batch,
                    uint16_t* d_scores, uint16_t* d_order_keys, uint32_t* d_head0, void* stream) {
    if (!d_q || !d_kshard || !d_scores || !d_order_keys || !valid_kv_heads(kv_heads) || tokens == 0 || batch == 0 ||
        batch > 65535 || tokens * batch > 0x7fffffffull)
        return fail(HSB_E_INVALID, "shard score arguments");
    if (!aligned(d_kshard, 16)) return fail(HSB_E_INVALID, "key shard must be 16-byte aligned");
    ScoreExtras x{};
    x.h0 = d_head0;
    const cudaError_t e = launch_score_shard(d_q, kv_heads, d_kshard, tokens, (size_t)kv_heads * HSB_DIM, d_scores,
                                             d_order_keys, nullptr, &x, as_stream(stream), batch);
    if (e != cudaSuccess) return fail_cuda(e, "shard score launch");
    g_last_error.clear();
    return HSB_OK;
}

static int check_group(const hsb_peer_group* g);

int hsb_shard_score_push(const uint16_t* d_q, int kv_heads, const uint16_t* d_kshard, size_t tokens, size_t batch,
                         uint16_t* d_scores, uint16_t* d_order_keys, uint32_t* d_head0, float alpha,
                         const hsb_peer_group* group, void* stream) {
    if (!d_q || !d_kshard || !d_scores || !d_order_keys || !d_head0 || !valid_kv_heads(kv_heads) || tokens == 0 ||
        batch == 0 || batch > 65535 || tokens * batch > 0x7fffffffull)
        return fail(HSB_E_INVALID, "shard score arguments");
    if (!aligned(d_kshard, 16)) return fail(HSB_E_INVALID, "key shard must be 16-byte aligned");
    if (!(alpha >= 0.0f) || !std::isfinite(alpha)) return fail(HSB_E_SEL_PARAMS, "GQA selector numeric parameters");
    int rc = check_group(group);
    if (rc) return rc;
    if (group->rank != 0 || group->batch != batch || group->world * kv_heads != HSB_KV_HEADS)
        return fail(HSB_E_INVALID, "shard score push: rank 0 of a group of this batch, holding 8 / world KV heads");
    ThresholdPush push{};
    if (!threshold_push_params(group, alpha, &push)) return fail(HSB_E_INVALID, "shard score push: peer group");
    ScoreExtras x{};
    x.h0 = d_head0;
    const cudaError_t e = launch_score_shard(d_q, kv_heads, d_kshard, tokens, (size_t)kv_heads * HSB_DIM, d_scores,
                                             d_order_keys, nullptr, &x, as_stream(stream), batch, &push);
    if (e != cudaSuccess) return fail_cuda(e, "shard score launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_shard_threshold(const uint32_t* d_head0, size_t batch, float alpha, uint32_t* d_thr, void* stream) {
    if (!d_head0 || !d_thr || batch == 0 || batch > 65535) return fail(HSB_E_INVALID, "shard threshold arguments");
    if (!(alpha >= 0.0f) || !std::isfinite(alpha)) return fail(HSB_E_SEL_PARAMS, "GQA selector numeric parameters");
    const cudaError_t e = launch_shard_threshold(d_head0, batch, alpha, d_thr, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "shard threshold launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_shard_count(const uint16_t* d_order_keys, size_t heads, size_t tokens, size_t batch, const uint32_t* d_thr,
                    uint32_t* d_records, void* stream) {
    if (!d_order_keys || !d_thr || !d_records || heads == 0 || heads > 128 || tokens == 0 ||
        tokens > 0x7fffffffull || batch == 0 || heads * batch > 0x7fffffffull)
        return fail(HSB_E_INVALID, "shard count arguments");
    const cudaError_t e = launch_shard_count(d_order_keys, heads, tokens, batch, d_thr, d_records, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "shard count launch");
    g_last_error.clear();
    return HSB_OK;
}

size_t hsb_shard_select_workspace_bytes(int kv_heads, size_t tokens, size_t kcap, size_t batch) {
    return select_workspace_bytes((size_t)(valid_kv_heads(kv_heads) ? kv_heads : 8) * 4 * (batch ? batch : 1), tokens,
                                  kcap);
}

int hsb_shard_select(const uint16_t* d_order_keys, const uint16_t* d_raw, int kv_heads, size_t tokens, size_t batch,
                     const uint32_t* d_thr, const uint32_t* d_records, size_t heads_total, size_t head_base,
                     float alpha, float ratio, uint32_t* d_ids, size_t kcap, uint32_t* d_counts,
                     hsb_selection* d_result, const float* d_q32, const uint16_t* d_kshard, const uint16_t* d_vshard,
                     uint16_t* d_k_packed, uint16_t* d_v_packed, float* d_out, void* d_workspace,
                     size_t workspace_bytes, void* stream) {
    if (!valid_kv_heads(kv_heads)) return fail(HSB_E_INVALID, "shard select: kv_heads must be 1, 2, 4 or 8");
    const size_t heads = (size_t)kv_heads * 4;
    int rc = check_select(heads_total, tokens, tokens, alpha, ratio);
    if (rc) return rc;
    if (batch == 0 || batch * heads * 4 > 0x7fffffffull)
        return fail(HSB_E_INVALID, "shard select: batch out of range");
    if (heads_total % 4 || head_base % 4 || head_base + heads > heads_total)
        return fail(HSB_E_INVALID, "shard select: head range outside the query heads");
    if (!d_order_keys || !d_thr || !d_records || !d_ids || !d_result || !d_q32 || !d_kshard || !d_vshard ||
        !d_k_packed || !d_v_packed || !d_out)
        return fail(HSB_E_INVALID, "shard select arguments");
    if (kcap < select_kmax(tokens, ratio)) return fail(HSB_E_SEL_CAPACITY, hsb_status_message(HSB_E_SEL_CAPACITY));
    if (!aligned(d_q32, 16) || !aligned(d_kshard, 16) || !aligned(d_vshard, 16) || !aligned(d_k_packed, 16) ||
        !aligned(d_v_packed, 16))
        return fail(HSB_E_INVALID, "shard select: query, shards and packed buffers must be 16-byte aligned");
    if (!select_cluster_available(tokens))
        return fail(HSB_E_INVALID, "shard select: at most 65536 tokens per head on this device");
    if (!d_workspace || workspace_bytes < select_workspace_bytes(heads * batch, tokens, kcap))
        return fail(HSB_E_WORKSPACE, "shard select workspace missing or too small");
    cudaError_t e = cudaMemsetAsync(d_result, 0, batch * sizeof(hsb_selection), as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "result reset");
    SelectLaunch sl{};
    sl.scores = d_order_keys;
    sl.keys = 1;
    sl.tie_raw = d_raw;
    sl.heads = (uint32_t)heads;
    sl.stride = tokens;
    sl.valid = tokens;
    sl.alpha = alpha;
    sl.ratio = ratio;
    sl.ids = d_ids;
    sl.kcap = kcap;
    sl.counts = d_counts;
    sl.result = d_result;
    sl.workspace = d_workspace;
    sl.workspace_bytes = workspace_bytes;
    sl.zero_is_error = 1;
    sl.reset_result = 0;
    sl.ext = d_records;
    sl.ext_thr = d_thr;
    sl.head_base = (uint32_t)head_base;
    sl.heads_total = (uint32_t)heads_total;
    sl.batch = (uint32_t)batch;
    sl.seq_scores = (unsigned long long)heads * tokens;
    sl.ga.q = d_q32;
    sl.ga.kcache = d_kshard;
    sl.ga.vcache = d_vshard;
    sl.ga.stride_words = (size_t)kv_heads * HSB_DIM;
    sl.ga.kp = d_k_packed;
    sl.ga.vp = d_v_packed;
    sl.ga.count = kcap;
    sl.ga.out = d_out;
    sl.ga.scale = 1.0f / sqrtf(128.0f);
    sl.ga.heads = (unsigned)heads;
    e = launch_select(sl, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "shard select launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------- KV-head shards, peer memory
size_t hsb_mailbox_bytes(size_t batch) { return mailbox_bytes(batch); }

void hsb_mailbox_layout_of(size_t batch, hsb_mailbox_layout* out) {
    if (out) mailbox_offsets(batch, out);
}

int hsb_mailbox_create(size_t batch, void** d_mailbox, void* ipc_handle) {
    if (!d_mailbox || batch == 0 || batch > 65535) return fail(HSB_E_INVALID, "mailbox arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) == HSB_IPC_HANDLE_BYTES, "IPC handle size");
    void* p = nullptr;
    const size_t bytes = mailbox_bytes(batch);
    cudaError_t e = cudaMalloc(&p, bytes);  // a base pointer: its IPC handle maps the mailbox itself
    if (e != cudaSuccess) return fail_cuda(e, "mailbox allocation");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess && ipc_handle) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail_cuda(e, "mailbox set-up");
    }
    *d_mailbox = p;
    g_last_error.clear();
    return HSB_OK;
}

int hsb_mailbox_destroy(void* d_mailbox) {
    const cudaError_t e = cudaFree(d_mailbox);
    return e == cudaSuccess ? HSB_OK : fail_cuda(e, "mailbox release");
}

int hsb_mailbox_open(const void* ipc_handle, void** d_peer) {
    if (!ipc_handle || !d_peer) return fail(HSB_E_INVALID, "mailbox open arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof h);
    const cudaError_t e = cudaIpcOpenMemHandle(d_peer, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? HSB_OK : fail_cuda(e, "mailbox open");
}

int hsb_mailbox_close(void* d_peer) {
    const cudaError_t e = cudaIpcCloseMemHandle(d_peer);
    return e == cudaSuccess ? HSB_OK : fail_cuda(e, "mailbox close");
}

static int check_group(const hsb_peer_group* g) {
    if (!g || g->world < 1 || g->world > HSB_MAX_PEERS || HSB_KV_HEADS % g->world || g->rank < 0 ||
        g->rank >= g->world || g->batch == 0 || g->batch > 65535)
        return fail(HSB_E_INVALID, "peer group: world must divide the 8 KV heads, rank < world, batch 1..65535");
    for (int w = 0; w < g->world; ++w)
        if (!g->mailbox[w] || !aligned(g->mailbox[w], 256))
            return fail(HSB_E_INVALID, "peer group: every rank's mailbox must be mapped (256-byte aligned)");
    return HSB_OK;
}

int hsb_exchange_threshold(const uint32_t* d_head0, float alpha, const hsb_peer_group* g, void* stream) {
    int rc = check_group(g);
    if (rc) return rc;
    if (!d_head0) return fail(HSB_E_INVALID, "exchange threshold: head-0 partials");
    if (g->rank != 0) return fail(HSB_E_INVALID, "exchange threshold: rank 0 holds query head 0");
    if (!(alpha >= 0.0f) || !std::isfinite(alpha)) return fail(HSB_E_SEL_PARAMS, "GQA selector numeric parameters");
    const cudaError_t e = launch_exchange_threshold(d_head0, alpha, g, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "exchange threshold launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_exchange_count(const uint16_t* d_order_keys, size_t heads, size_t tokens, const hsb_peer_group* g,
                       void* stream) {
    int rc = check_group(g);
    if (rc) return rc;
    if (!d_order_keys || tokens == 0 || tokens > 0x7fffffffull || heads * (size_t)g->world != HSB_QUERY_HEADS)
        return fail(HSB_E_INVALID, "exchange count: keys [batch][32 / world][tokens]");
    const cudaError_t e = launch_exchange_count(d_order_keys, heads, tokens, g, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "exchange count launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_exchange_finish(const float* d_out, const hsb_selection* d_results, size_t heads, const hsb_peer_group* g,
                        void* stream) {
    int rc = check_group(g);
    if (rc) return rc;
    if (!d_out || !d_results || !aligned(d_out, 16) || heads * (size_t)g->world != HSB_QUERY_HEADS)
        return fail(HSB_E_INVALID, "exchange finish: outputs [batch][32 / world][128] (16-byte aligned), results");
    const cudaError_t e = launch_exchange_finish(d_out, d_results, heads, g, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "exchange finish launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------------------- synthetic
int hsb_synth_normal_f16(uint16_t* d_out, size_t count, uint64_t seed, float stddev, void* stream) {
    if (!d_out) return fail(HSB_E_INVALID, "null output");
    cudaError_t e = launch_synth_normal(d_out, count, seed, stddev, 0, as_stream(stream));
    return e == cudaSuccess ? HSB_OK : fail_cuda(e, "synth launch");
}
int hsb_synth_normal_bf16(uint16_t* d_out, size_t count, uint64_t seed, float stddev, void* stream) {
    if (!d_out) return fail(HSB_E_INVALID, "null output");
    cudaError_t e = launch_synth_normal(d_out, count, seed, stddev, 1, as_stream(stream));
    return e == cudaSuccess ? HSB_OK : fail_cuda(e, "synth launch");
}
int hsb_synth_keys(uint16_t* d_rows, size_t tokens, size_t stride_words, uint64_t seed, float heavy_fraction,
                   float heavy_scale, int rope, float theta, void* stream) {
    if (!d_rows || stride_words < 1024) return fail(HSB_E_INVALID, "synth keys arguments");
    cudaError_t e = launch_synth_keys(d_rows, tokens, stride_words, seed, heavy_fraction, heavy_scale, rope, theta,
                                      as_stream(stream));
    return e == cudaSuccess ? HSB_OK : fail_cuda(e, "synth launch");
}

// ------------------------------------------------------- H2O statistics
int hsb_h2o_group_sums(const void* d_probabilities, const int64_t ne[4], const size_t nb[4],
                       size_t valid_keys, size_t valid_queries, float* d_sums, size_t capacity_keys,
                       hsb_device_status* d_status, void* stream) {
    // runtime/gqa_h2o_stats.cu:110-133, in the reference's order.
    if (!d_probabilities || !d_sums || !ne || !nb || !valid_keys || !valid_queries || valid_keys > capacity_keys)
        return fail(HSB_E_H2O_ARGS, "H2O reduction invalid pointer, actual CUDA stream or capacity");
    if (!(ne[0] > 0 && ne[1] > 0 && ne[2] == 32 && ne[3] == 1 && valid_keys <= (uint64_t)ne[0] &&
          valid_queries <= (uint64_t)ne[1]))
        return fail(HSB_E_H2O_SHAPE, "H2O reduction requires [keys,queries,32,1] actual attention");
    const size_t extents[3] = {valid_keys, valid_queries, 32};
    size_t max_offset = 0;
    for (int axis = 0; axis < 3; ++axis) {
        if (nb[axis] < sizeof(float) || nb[axis] % alignof(float) != 0)
            return fail(HSB_E_H2O_STRIDE, "H2O reduction invalid F32 tensor stride");
        if (nb[axis] && extents[axis] - 1 > std::numeric_limits<size_t>::max() / nb[axis])
            return fail(HSB_E_H2O_OVERFLOW, "H2O attention statistics size overflow");
        const size_t offset = (extents[axis] - 1) * nb[axis];
        if (offset > std::numeric_limits<size_t>::max() - max_offset)
            return fail(HSB_E_H2O_OVERFLOW, "H2O attention statistics address overflow");
        max_offset += offset;
    }
    if (max_offset > std::numeric_limits<size_t>::max() - sizeof(float))
        return fail(HSB_E_H2O_OVERFLOW, "H2O attention statistics final address overflow");
    if (!aligned(d_probabilities, alignof(float)))
        return fail(HSB_E_H2O_ALIGN, "H2O reduction requires aligned F32 tensor");
    if ((valid_keys - 1) / 256 + 1 > 2147483647u)
        return fail(HSB_E_H2O_GRID, "H2O reduction exceeds CUDA grid limit");
    int device = -1;
    cudaPointerAttributes attributes{};
    if (cudaGetDevice(&device) != cudaSuccess || cudaPointerGetAttributes(&attributes, d_probabilities) != cudaSuccess) {
        cudaGetLastError();
        return fail(HSB_E_H2O_DEVICE, "H2O softmax tensor is not on the expected CUDA device");
    }
    if (attributes.type != cudaMemoryTypeDevice || attributes.device != device)
        return fail(HSB_E_H2O_DEVICE, "H2O softmax tensor is not on the expected CUDA device");
    cudaError_t e = launch_h2o_group_sums(d_probabilities, valid_keys, valid_queries, nb[0], nb[1], nb[2], d_sums,
                                          d_status, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "H2O attention reduction launch");
    g_last_error.clear();
    return HSB_OK;
}

// ------------------------------------------------- cold-tier KV records
static bool segment_geometry_ok(size_t layers, uint64_t positions, size_t record_bytes) {
    // storage/segmented_store.cpp:25
    return layers && layers <= 128 && positions && positions <= 66048 && record_bytes && record_bytes <= 65536;
}

uint64_t hsb_segment_extent_bytes(size_t layers, uint64_t positions, size_t record_bytes) {
    if (!segment_geometry_ok(layers, positions, record_bytes)) return 0;
    const uint64_t stride = (uint64_t)record_bytes + HSB_RECORD_HEADER_BYTES;
    return (HSB_SEGMENT_HEADER_BYTES + (uint64_t)layers * positions * stride + 4095) / 4096 * 4096;
}

int hsb_segment_header(void* header, uint64_t request, size_t layers, uint64_t positions, size_t record_bytes) {
    if (!header) return fail(HSB_E_INVALID, "null segment header");
    if (!segment_geometry_ok(layers, positions, record_bytes))
        return fail(HSB_E_SEGMENT_GEOMETRY, "bounded segmented geometry/quota");
    // segmented_store.cpp:30: 512 u64 words, the first eight set.
    uint64_t words[HSB_SEGMENT_HEADER_BYTES / 8] = {};
    words[0] = 0x48534b5653454731ull;  // "HSKVSEG1"
    words[1] = 1;
    words[2] = request;
    words[3] = layers;
    words[4] = positions;
    words[5] = record_bytes;
    words[6] = (uint64_t)record_bytes + HSB_RECORD_HEADER_BYTES;
    words[7] = hsb_segment_extent_bytes(layers, positions, record_bytes);
    std::memcpy(header, words, sizeof words);
    g_last_error.clear();
    return HSB_OK;
}

uint64_t hsb_fnv1a64(const void* data, size_t n) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

int hsb_kv_records_encode(const void* d_payload, size_t payload_stride, size_t count, size_t record_bytes,
                          uint64_t request, uint32_t layer, uint64_t first, void* d_records, void* stream) {
    if (!record_bytes || record_bytes > 65536)
        return fail(HSB_E_SEGMENT_GEOMETRY, "bounded segmented geometry/quota");
    // segmented_store.cpp:98: an empty append is rejected.
    if (!d_payload || !d_records || !count || payload_stride < record_bytes)
        return fail(HSB_E_INVALID, "append epoch/size/poisoned state");
    if (first > std::numeric_limits<uint64_t>::max() - count) return fail(HSB_E_INVALID, "append capacity");
    cudaError_t e = launch_records_encode(d_payload, payload_stride, count, record_bytes, request, layer, first,
                                          d_records, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "record encode launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_kv_records_verify(const void* d_window, size_t window_bytes, const uint64_t* d_offsets,
                          const uint64_t* d_positions, const uint32_t* d_groups, size_t count, uint64_t request,
                          uint32_t layer, size_t record_bytes, void* d_out, size_t out_stride,
                          const uint32_t* d_out_rows, size_t out_rows_capacity, hsb_device_status* d_status,
                          void* stream) {
    if (!record_bytes || record_bytes > 65536)
        return fail(HSB_E_SEGMENT_GEOMETRY, "bounded segmented geometry/quota");
    if (!d_status || out_stride < record_bytes || count > 0xffffffffull)
        return fail(HSB_E_INVALID, "record verify arguments");
    if (count == 0) {
        g_last_error.clear();
        return HSB_OK;
    }
    if (!d_window || !d_offsets || !d_positions || !d_out) return fail(HSB_E_INVALID, "record verify arguments");
    // The window is device memory, or pinned host memory the kernel reads in
    // place over the bus (mapped at the same address); never pageable memory.
    cudaPointerAttributes wa{};
    if (cudaPointerGetAttributes(&wa, d_window) != cudaSuccess) {
        cudaGetLastError();
        return fail(HSB_E_INVALID, "record window is not device or pinned host memory");
    }
    const bool device_window = wa.type == cudaMemoryTypeDevice || wa.type == cudaMemoryTypeManaged;
    const bool mapped_host = wa.type == cudaMemoryTypeHost && wa.devicePointer == d_window;
    if (!device_window && !mapped_host)
        return fail(HSB_E_INVALID, "record window is not device or pinned host memory");
    cudaError_t e = launch_records_verify(d_window, window_bytes, d_offsets, d_positions, d_groups, count, request,
                                          layer, record_bytes, d_out, out_stride, d_out_rows, out_rows_capacity,
                                          mapped_host ? 1 : 0, d_status, as_stream(stream));
    if (e != cudaSuccess) return fail_cuda(e, "record verify launch");
    g_last_error.clear();
    return HSB_OK;
}

int hsb_kv_read_plan(const uint64_t* offsets, size_t count, uint64_t record_bytes, uint64_t extent,
                     size_t window_bytes, size_t gap_bytes, unsigned amplification, hsb_kv_read_window* windows,
                     size_t windows_capacity, size_t* nwindows) {
    // storage/kv_read_plan.hpp:22-28 (limits), :37-39 (geometry), :41-59 (plan)
    if (window_bytes < 8192 || window_bytes > 1024 * 1024 || window_bytes % 4096 || gap_bytes > 64 * 1024 ||
        gap_bytes % 4096 || amplification < 1000 || amplification > 2000)
        return fail(HSB_E_READ_PLAN, "invalid bounded complete-KV read limits");
    if (!record_bytes || extent % 4096 || record_bytes > window_bytes - 4095)
        return fail(HSB_E_READ_PLAN, "invalid complete-KV record geometry");
    if (!nwindows || (count && (!offsets || !windows))) return fail(HSB_E_INVALID, "read plan arguments");
    size_t n = 0;
    uint64_t previous_end = 0, last_page_end = 0;
    for (size_t i = 0; i < count; ++i) {
        const uint64_t offset = offsets[i];
        if (offset > extent || record_bytes > extent - offset || (i && offset < previous_end))
            return fail(HSB_E_READ_PLAN, "unordered, overlapping or out-of-extent KV record");
        previous_end = offset + record_bytes;
        if (previous_end > std::numeric_limits<uint64_t>::max() - 4095)
            return fail(HSB_E_READ_PLAN, "complete-KV aligned offset overflow");
        const uint64_t begin = offset / 4096 * 4096, end = (previous_end + 4095) / 4096 * 4096;
        if (end > extent) return fail(HSB_E_READ_PLAN, "complete-KV aligned read exceeds extent");
        bool merged = false;
        if (n) {
            hsb_kv_read_window& w = windows[n - 1];
            const uint64_t required = w.required_page_bytes + end - std::max(begin, last_page_end);
            const uint64_t span = end - w.begin, gap = begin > w.end ? begin - w.end : 0;
            if (span <= window_bytes && gap <= gap_bytes && span * 1000 <= required * amplification) {
                w.end = end;
                w.required_page_bytes = required;
                w.end_record = i + 1;
                merged = true;
            }
        }
        if (!merged) {
            if (n == windows_capacity) return fail(HSB_E_INVALID, "read plan window capacity");
            windows[n++] = hsb_kv_read_window{begin, end, end - begin, i, i + 1};
        }
        last_page_end = end;
    }
    *nwindows = n;
    g_last_error.clear();
    return HSB_OK;
}

int hsb_kv_read_groups(const hsb_kv_read_window* windows, size_t nwindows, uint32_t* groups, size_t count) {
    if ((nwindows && !windows) || (count && !groups)) return fail(HSB_E_INVALID, "read group arguments");
    uint64_t next = 0, group = 0;
    for (size_t w = 0; w < nwindows; ++w) {
        if (windows[w].first_record != next || windows[w].end_record <= next || windows[w].end_record > count)
            return fail(HSB_E_READ_PLAN, "read windows do not cover the records in order");
        for (uint64_t j = windows[w].first_record; j < windows[w].end_record; j += 4, ++group)
            for (uint64_t k = j; k < std::min<uint64_t>(j + 4, windows[w].end_record); ++k) groups[k] = (uint32_t)group;
        next = windows[w].end_record;
    }
    if (next != count) return fail(HSB_E_READ_PLAN, "read windows do not cover the records in order");
    g_last_error.clear();
    return HSB_OK;
}

}  // extern "C"
