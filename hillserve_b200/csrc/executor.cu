// executor.cu -- the model-facing decode step of the layer executor
// (runtime/gqa_executor.cpp:149-249 prepare(); the attention hook of
// patches/llama-b6000-round2.patch:218-244), kept on the GPU.
//
// The reference executor copies the model's current K/V to the host,
// appends it to the store, selects and fetches there, packs a padded
// per-query-head K / V / mask workspace (count slots x 32 heads, ~161 MB at
// N = 32K) and uploads it for ggml's masked attention.  Here the model's
// current K/V tensor is appended to the HBM cache by a kernel, the
// rehearsal query is rounded to F16 by a kernel, and the layer step selects,
// gathers the live slots and attends over them directly -- no mask, no
// padding, no host copy -- writing the attention output in the model's
// layout (F32 [32 query heads][128]).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

// The model's current KV tensor (ggml_concat(k_cur, v_cur, 0) cast to F16):
// [token][KV head][K 128 | V 128].  The cache row of a token: K[8][128] then
// V[8][128] (the payload layout of runtime/gqa_executor.cpp:155).  Blocks
// 0..n-1 move one token each as 256 16-byte words; a non-finite F16 in the
// current KV is an error (runtime/gqa_executor.cpp:153).  With a rehearsal,
// blocks n..n+3 round it to F16 (query_f16, policy/full_gqa_runtime.cpp:
// 61-64: a non-finite input, or an F16 overflow, is an error).  One launch
// per layer.
constexpr int kQueryBlocks = 4;
__global__ void __launch_bounds__(256) executor_prepare_kernel(const uint16_t* __restrict__ current,
                                                               unsigned long long n, uint16_t* __restrict__ cache,
                                                               unsigned long long first,
                                                               const float* __restrict__ rehearsal,
                                                               uint16_t* __restrict__ q16,
                                                               hsb_device_status* status) {
    pdl_wait();
    pdl_trigger();
    const unsigned long long t = blockIdx.x;
    const int i = threadIdx.x;
    if (t >= n) {  // blocks n .. n+3: a quarter of the query each
        constexpr int kPer = kHeads * kDim / kQueryBlocks / 256;  // elements per thread
        const int q0 = (int)(t - n) * (kHeads * kDim / kQueryBlocks);
        float x[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) x[u] = rehearsal[q0 + i + u * 256];  // loads first: one round trip
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int j = q0 + i + u * 256;
            const uint16_t h = half_bits(x[u]);
            q16[j] = h;
            if (!isfinite(x[u])) raise_status(status, HSB_E_EXECUTOR_REHEARSAL, j);
            else if (!is_finite_half(h)) raise_status(status, HSB_E_EXECUTOR_REHEARSAL_F16, j);
        }
        return;
    }
    const int head = i >> 5, part = (i >> 4) & 1, c8 = i & 15;
    const uint4 w = reinterpret_cast<const uint4*>(current + t * 2048 + head * 256 + part * 128)[c8];
    reinterpret_cast<uint4*>(cache + (first + t) * 2048 + part * 1024 + head * 128)[c8] = w;
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    bool finite = true;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        finite &= ((words[k] & 0x7c00u) != 0x7c00u) && ((words[k] & 0x7c000000u) != 0x7c000000u);
    if (!__syncthreads_and(finite) && i == 0) raise_status(status, HSB_E_EXECUTOR_NONFINITE_KV, (int)t);
}

cudaError_t launch_prepare(const uint16_t* current, size_t n, uint16_t* cache, size_t first, const float* rehearsal,
                           uint16_t* q16, hsb_device_status* status, cudaStream_t stream) {
    const unsigned blocks = (unsigned)(n + (rehearsal ? kQueryBlocks : 0));
    return launch_dependent(executor_prepare_kernel, dim3(blocks), dim3(256), 0, stream, false, current,
                            (unsigned long long)n, cache, (unsigned long long)first, rehearsal, q16, status);
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace
}  // namespace hsb

using namespace hsb;

extern "C" {

int hsb_executor_append(const uint16_t* d_current, size_t n_tokens, uint16_t* d_cache, size_t capacity,
                        size_t first_position, hsb_device_status* d_status, void* stream) {
    // runtime/gqa_executor.cpp:151
    if (!d_current || !d_cache || !d_status || !n_tokens || first_position > capacity ||
        n_tokens > capacity - first_position)
        return record_error(HSB_E_EXECUTOR_SHAPE, "GQA current KV ABI mismatch");
    if ((reinterpret_cast<uintptr_t>(d_current) | reinterpret_cast<uintptr_t>(d_cache)) & 15u)
        return record_error(HSB_E_INVALID, "executor tensors must be 16-byte aligned");
    cudaError_t e = launch_prepare(d_current, n_tokens, d_cache, first_position, nullptr, nullptr, d_status,
                                   static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_cuda_error(e, "executor append launch");
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_executor_query(const float* d_rehearsal, uint16_t* d_q16, hsb_device_status* d_status, void* stream) {
    if (!d_rehearsal || !d_q16 || !d_status)
        return record_error(HSB_E_EXECUTOR_SHAPE, "full GQA actual rehearsal must be32x128");
    cudaError_t e = launch_prepare(nullptr, 0, nullptr, 0, d_rehearsal, d_q16, d_status,
                                   static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_cuda_error(e, "executor query launch");
    record_error(HSB_OK, "");
    return HSB_OK;
}

size_t hsb_executor_workspace_bytes(size_t capacity, size_t count) {
    const size_t layer = std::max(hsb_layer_workspace_bytes(capacity, count), hsb_attention_dense_workspace_bytes(capacity));
    return align256(layer) + align256(kHeads * kDim * sizeof(uint16_t));
}

int hsb_executor_decode_layer(const uint16_t* d_current, const float* d_rehearsal, const float* d_q,
                              uint16_t* d_cache, size_t capacity, size_t position, int dense, float alpha,
                              float ratio, size_t count, const hsb_layer_buffers* buffers, float* d_out,
                              hsb_device_status* d_status, void* stream) {
    if (!buffers || !buffers->workspace || !d_out || !d_q)
        return record_error(HSB_E_INVALID, "executor layer arguments");
    if (buffers->workspace_bytes < hsb_executor_workspace_bytes(capacity, count))
        return record_error(HSB_E_WORKSPACE, "workspace missing or too small");
    const size_t layer_bytes = align256(std::max(hsb_layer_workspace_bytes(capacity, count),
                                                 hsb_attention_dense_workspace_bytes(capacity)));
    uint16_t* q16 = reinterpret_cast<uint16_t*>(static_cast<unsigned char*>(buffers->workspace) + layer_bytes);
    if (!d_current || !d_cache || !d_status || position >= capacity || (!dense && !d_rehearsal))
        return record_error(HSB_E_EXECUTOR_SHAPE, "GQA current KV ABI mismatch");
    if ((reinterpret_cast<uintptr_t>(d_current) | reinterpret_cast<uintptr_t>(d_cache)) & 15u)
        return record_error(HSB_E_INVALID, "executor tensors must be 16-byte aligned");
    // the current token's append and (sparse layers) the selection query, one launch
    cudaError_t e = launch_prepare(d_current, 1, d_cache, position, dense ? nullptr : d_rehearsal, q16, d_status,
                                   static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_cuda_error(e, "executor prepare launch");
    const size_t valid = position + 1;
    if (dense) {
        // the two dense layers (runtime/gqa_executor.cpp:174-176): every position
        return hsb_attention_dense(d_q, d_cache, d_cache + 1024, valid, 2048, d_out, buffers->workspace, layer_bytes,
                                   stream);
    }
    hsb_layer_buffers b = *buffers;
    b.workspace_bytes = layer_bytes;
    return hsb_layer_step(q16, d_q, d_cache, d_cache + 1024, 2048, valid, alpha, ratio, count, &b, d_out, stream);
}

}  // extern "C"
