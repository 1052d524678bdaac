// noalloc.cu -- hsb_attention_packed_noalloc: the packed attention of
// hsb_attention_packed for callers that cannot give the library any device
// memory of their own.
//
// Who needs it: an attention step that runs as an operator inside a host
// framework's compute graph (a ggml-style backend op, or a decode step being
// captured into a CUDA graph in global capture mode). Such an operator is
// handed its input and output tensors and a stream, and nothing else. It has
// no workspace slot to pass. It may not call cudaMalloc either: the
// framework's allocator owns device memory, and global-mode capture refuses
// the call.
//
// What it does instead: the attention's scratch (the per-split partial
// results and the per-head arrival counters of its last-CTA combine) lives
// in one file-scope __device__ array of kScratchBytes. Every GPU that loads
// this library holds that array until the process exits. Calls are limited
// to HSB_NOALLOC_MAX_SLOTS slots; larger counts are rejected with
// HSB_E_WORKSPACE before any GPU work.
//
// Rules for callers:
//  - All calls on a device share the one array, which keeps the last call's
//    contents. The arrival counters are cleared on the stream at the start
//    of every call, and the partials are overwritten before they are read.
//    Calls whose executions overlap on the GPU (different streams, or
//    different host threads without ordering) race on the array and give
//    wrong results. Order them on one stream.
//  - The first call on each device resolves the array's device address with
//    cudaGetSymbolAddress (with that device current). Make that first call
//    before any stream capture begins.
//
// The entry point allocates nothing: it calls no cudaMalloc / cudaFree and
// no allocating library routine. It then runs exactly the kernel of
// hsb_attention_packed.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "internal.h"

namespace hsb {
namespace {

// Scratch for HSB_NOALLOC_MAX_SLOTS slots: 128 B of arrival counters plus
// 32 heads x 26 splits x 130 floats of partials (432,896 B), rounded up to
// 448 KiB.
constexpr size_t kScratchBytes = 448 * 1024;
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_address[64] = {};

// Device address of g_noalloc_scratch on the current device; resolved once
// per device.  Returns HSB_OK or an error already recorded.
int scratch_address(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e, "hsb_attention_packed_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return record_error(HSB_E_NO_DEVICE, "hsb_attention_packed_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_address[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                     "hsb_attention_packed_noalloc: cudaGetSymbolAddress of the static scratch");
        g_scratch_address[dev] = p;
    }
    *out = g_scratch_address[dev];
    return HSB_OK;
}

}  // namespace
}  // namespace hsb

using namespace hsb;

extern "C" int hsb_attention_packed_noalloc(const float* d_q, const uint16_t* d_k, const uint16_t* d_v, size_t count,
                                            const float* d_mask, size_t qpad, const uint32_t* d_sizes,
                                            size_t sizes_stride, float* d_out, void* stream) {
    if (count > HSB_NOALLOC_MAX_SLOTS || attention_workspace_bytes(count) > kScratchBytes) {
        char msg[160];
        std::snprintf(msg, sizeof msg,
                      "hsb_attention_packed_noalloc: count %zu exceeds the %d-slot limit of its static scratch",
                      count, HSB_NOALLOC_MAX_SLOTS);
        return record_error(HSB_E_WORKSPACE, msg);
    }
    void* scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != HSB_OK) return rc;
    return hsb_attention_packed(d_q, d_k, d_v, count, d_mask, qpad, d_sizes, sizes_stride, d_out, scratch,
                                kScratchBytes, stream);
}
