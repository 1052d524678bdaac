// noalloc.cu -- hsb_attention_packed_noalloc: the packed attention of
// hsb_attention_packed for callers that cannot give the library any device
// memory of their own.
//
// Who needs it: an attention step that runs as an operator inside a host
// framework's compute graph (a ggml-style backend op, for instance). Such an
// operator is handed its input and output tensors and a stream, and nothing
// else: it has no workspace slot to pass, and it may not call cudaMalloc,
// because the framework's allocator owns the device memory.
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
//  - The first call in each CUDA context (normally once per device: the
//    device's primary context) resolves the array's device address with
//    cudaGetSymbolAddress, with that context current. Make that first call
//    before any stream capture begins. A context created later on the same
//    device -- after cudaDeviceReset, or a host framework's own driver-API
//    context made current -- is a new set-up: its first call resolves the
//    address again (the cache is keyed by the context's unique ID).
//
// The entry point allocates nothing: it calls no cudaMalloc / cudaFree and
// no allocating library routine. It then runs exactly the kernel of
// hsb_attention_packed.
#include <cuda.h>
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

// The address belongs to the module instance of one CUDA context, so the
// cache is keyed by the context's unique ID (cuCtxGetId; the handle from
// cuCtxGetCurrent where the driver lacks it), not by the device ordinal.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
struct ScratchEntry {
    unsigned long long context = 0;
    void* address = nullptr;
};
constexpr int kScratchEntries = 64;
std::mutex g_scratch_mutex;
ScratchEntry g_scratch_cache[kScratchEntries];
int g_scratch_next = 0;

void* driver_entry(const char* name) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return f;
}

// Unique key of the calling thread's current context; 0 on failure.
unsigned long long current_context_key() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        get_current = reinterpret_cast<CtxGetCurrentFn>(driver_entry("cuCtxGetCurrent"));
        get_id = reinterpret_cast<CtxGetIdFn>(driver_entry("cuCtxGetId"));
    });
    if (!get_current) return 0;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
    unsigned long long id = 0;
    if (get_id && get_id(ctx, &id) == CUDA_SUCCESS) return id + 1;  // never 0
    return reinterpret_cast<unsigned long long>(ctx);
}

// Device address of g_noalloc_scratch in the current context, resolved once
// per context.  Returns HSB_OK or an error already recorded.
int scratch_address(void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    unsigned long long key = current_context_key();
    if (key != 0) {
        for (const ScratchEntry& entry : g_scratch_cache) {
            if (entry.context == key) {
                *out = entry.address;
                return HSB_OK;
            }
        }
    }
    // Resolving the symbol also makes the device's primary context current
    // when the thread had none yet.
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
        return record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                 "hsb_attention_packed_noalloc: cudaGetSymbolAddress of the static scratch");
    if (key == 0) key = current_context_key();
    if (key == 0) return record_error(HSB_E_NO_DEVICE, "hsb_attention_packed_noalloc: no current CUDA context");
    g_scratch_cache[g_scratch_next] = ScratchEntry{key, p};
    g_scratch_next = (g_scratch_next + 1) % kScratchEntries;
    *out = p;
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
