// records.cu -- the cold-tier KV record format of SegmentedKVStore v1
// (storage/segmented_store.{hpp,cpp}) and its FNV-1a integrity check, on
// the GPU: the encoder that turns KV rows in HBM into the file image of
// their records, and the verifier that checks records read back from the
// file (uploaded into device memory as raw windows) and gathers their
// payloads into device rows.
//
// Format.  File header: 4096 bytes, 512 little-endian u64 words
// {magic "HSKVSEG1", version 1, request, layers, positions, record bytes,
// stride, extent, 0 ...} (segmented_store.cpp:30).  Record (layer, position)
// at 4096 + (layer * positions + position) * stride, stride = record bytes +
// 32: a 32-byte header {u64 digest, u64 position, u64 request, u32 layer,
// u32 version = 1} then the payload (segmented_store.cpp:18,21,101-102).
// digest = FNV-1a 64 of the payload bytes (storage/file_store.cpp:12-16).
//
// FNV-1a is one serial chain per record (h = (h ^ byte) * P), so a thread
// owns a record; the GPU's parallelism is across records.  The prime is
// P = 2^40 + 0x1b3, so with h = hi:lo in 32-bit halves
//     h * P mod 2^64:  lo' = low32(lo * 0x1b3),
//                      hi' = hi * 0x1b3 + high32(lo * 0x1b3) + (lo << 8),
// one 32x32->64 multiply, one multiply-add and one shift-add per byte.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr uint64_t kFnvSeed = 14695981039346656037ull;
constexpr int kRecordThreads = 64;  // one record per thread; small blocks spread few records over many SMs

struct Fnv {
    uint32_t lo, hi;
};
__device__ __forceinline__ void fnv_byte(Fnv& h, uint32_t byte) {
    h.lo ^= byte;
    const uint64_t w = (uint64_t)h.lo * 0x1b3u;
    h.hi = h.hi * 0x1b3u + (uint32_t)(w >> 32) + (h.lo << 8);
    h.lo = (uint32_t)w;
}
__device__ __forceinline__ void fnv_word(Fnv& h, uint32_t x) {
    fnv_byte(h, x & 0xffu);
    fnv_byte(h, (x >> 8) & 0xffu);
    fnv_byte(h, (x >> 16) & 0xffu);
    fnv_byte(h, x >> 24);
}
__device__ __forceinline__ uint64_t fnv_value(const Fnv& h) { return ((uint64_t)h.hi << 32) | h.lo; }

// Hashes `bytes` bytes from src and copies them to dst (dst may be null).
// Vector path (src, dst 16-byte aligned, bytes % 16 == 0, chosen by the
// caller through `vec`): the payload moves a 128-byte line (eight 16-byte
// loads) at a time, the next line's loads in flight while the current line
// is hashed, so one record's ~800 cycles of hashing per line cover the
// memory latency of the next; from device memory the two lines after it
// are also prefetched to L2 (not from a pinned host window).
__device__ uint64_t hash_copy(const unsigned char* __restrict__ src, unsigned char* __restrict__ dst, size_t bytes,
                              bool vec, bool prefetch) {
    Fnv h{(uint32_t)kFnvSeed, (uint32_t)(kFnvSeed >> 32)};
    if (vec) {
        constexpr int kLine = 8;  // 16-byte chunks per line
        const uint4* s = reinterpret_cast<const uint4*>(src);
        uint4* d = reinterpret_cast<uint4*>(dst);
        const size_t n = bytes / 16;
        uint4 cur[kLine], nxt[kLine];
#pragma unroll
        for (int c = 0; c < kLine; ++c) cur[c] = (size_t)c < n ? __ldg(s + c) : make_uint4(0, 0, 0, 0);
        for (size_t j = 0; j < n; j += kLine) {
            // lines j+2 and j+3 start moving into L2 now, so that the next
            // iterations' loads find them there
            if (prefetch && j + 2 * kLine < n) asm volatile("prefetch.global.L2 [%0];" ::"l"(s + j + 2 * kLine));
            if (prefetch && j + 3 * kLine < n) asm volatile("prefetch.global.L2 [%0];" ::"l"(s + j + 3 * kLine));
#pragma unroll
            for (int c = 0; c < kLine; ++c)
                nxt[c] = j + kLine + c < n ? __ldg(s + j + kLine + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < kLine; ++c) {
                if (j + c < n) {
                    if (d) d[j + c] = cur[c];
                    fnv_word(h, cur[c].x);
                    fnv_word(h, cur[c].y);
                    fnv_word(h, cur[c].z);
                    fnv_word(h, cur[c].w);
                }
            }
#pragma unroll
            for (int c = 0; c < kLine; ++c) cur[c] = nxt[c];
        }
    } else {
        for (size_t i = 0; i < bytes; ++i) {
            const unsigned char b = src[i];
            if (dst) dst[i] = b;
            fnv_byte(h, b);
        }
    }
    return fnv_value(h);
}

struct alignas(16) RecordHeader {  // moved as two 16-byte words
    uint64_t digest, position, request;
    uint32_t layer, version;
};
static_assert(sizeof(RecordHeader) == 32, "fixed on-disk header");

__global__ void __launch_bounds__(kRecordThreads) records_encode_kernel(
    const unsigned char* __restrict__ payload, unsigned long long payload_stride, unsigned long long count,
    unsigned long long record_bytes, unsigned long long request, uint32_t layer, unsigned long long first,
    unsigned char* __restrict__ records, int vec) {
    pdl_wait();
    pdl_trigger();
    const unsigned long long i = (unsigned long long)blockIdx.x * kRecordThreads + threadIdx.x;
    if (i >= count) return;
    unsigned char* rec = records + i * (record_bytes + 32);
    const uint64_t digest = hash_copy(payload + i * payload_stride, rec + 32, record_bytes, vec != 0, true);
    RecordHeader h{digest, first + i, request, layer, 1u};
    if (vec) {
        const uint4* w = reinterpret_cast<const uint4*>(&h);
        reinterpret_cast<uint4*>(rec)[0] = w[0];
        reinterpret_cast<uint4*>(rec)[1] = w[1];
    } else {
        const unsigned char* b = reinterpret_cast<const unsigned char*>(&h);
        for (int j = 0; j < 32; ++j) rec[j] = b[j];
    }
}

// First error in the reference's validation order: by validation group
// (groups[i], or i itself), then identity before checksum, then index.
__device__ __forceinline__ unsigned long long record_rank(const uint32_t* groups, int code, uint32_t index) {
    const unsigned long long g = groups ? groups[index] : index;
    const unsigned long long kind = code == HSB_E_RECORD_IDENTITY ? 1ull : code == HSB_E_RECORD_CHECKSUM ? 2ull : 0ull;
    return (g << 34) | (kind << 32) | index;
}
__device__ void raise_record(hsb_device_status* st, const uint32_t* groups, int code, uint32_t index) {
    unsigned long long* word = reinterpret_cast<unsigned long long*>(st);
    const unsigned long long mine = ((unsigned long long)index << 32) | (unsigned)code;
    const unsigned long long my_rank = record_rank(groups, code, index);
    unsigned long long seen = *reinterpret_cast<volatile unsigned long long*>(word);
    while (true) {
        const int old_code = (int)(seen & 0xffffffffull);
        const uint32_t old_index = (uint32_t)(seen >> 32);
        if (old_code != 0 && record_rank(groups, old_code, old_index) <= my_rank) return;
        const unsigned long long prev = atomicCAS(word, seen, mine);
        if (prev == seen) return;
        seen = prev;
    }
}

struct VerifyParams {
    const unsigned char* window;
    unsigned long long window_bytes;
    const unsigned long long* offsets;
    const unsigned long long* positions;
    const uint32_t* groups;
    unsigned long long count;
    unsigned long long request;
    uint32_t layer;
    unsigned long long record_bytes;
    unsigned char* out;
    unsigned long long out_stride;
    const uint32_t* out_rows;
    unsigned long long out_capacity;
    hsb_device_status* status;
    int vec;
    int host_window;  // the window is pinned host memory read in place
};

__global__ void __launch_bounds__(kRecordThreads) records_verify_kernel(const __grid_constant__ VerifyParams p) {
    pdl_wait();
    pdl_trigger();
    const unsigned long long i = (unsigned long long)blockIdx.x * kRecordThreads + threadIdx.x;
    if (i >= p.count) return;
    const unsigned long long off = p.offsets[i];
    const unsigned long long row = p.out_rows ? p.out_rows[i] : i;
    if (off > p.window_bytes || p.window_bytes - off < p.record_bytes + 32 || row >= p.out_capacity) {
        raise_record(p.status, p.groups, HSB_E_RECORD_BOUNDS, (uint32_t)i);
        return;
    }
    const unsigned char* rec = p.window + off;
    const bool vec = p.vec && (off & 15u) == 0;  // 16-byte loads only from 16-byte aligned records
    RecordHeader h;
    if (vec) {
        const uint4 a = reinterpret_cast<const uint4*>(rec)[0], b = reinterpret_cast<const uint4*>(rec)[1];
        reinterpret_cast<uint4*>(&h)[0] = a;
        reinterpret_cast<uint4*>(&h)[1] = b;
    } else {
        unsigned char* d = reinterpret_cast<unsigned char*>(&h);
        for (int j = 0; j < 32; ++j) d[j] = rec[j];
    }
    const uint64_t digest = hash_copy(rec + 32, p.out + row * p.out_stride, p.record_bytes, vec, !p.host_window);
    // The reference checks the record's identity before its digest
    // (policy/full_gqa_runtime.cpp:397-408, segmented_store.cpp:116-119).
    if (h.position != p.positions[i] || h.request != p.request || h.layer != p.layer || h.version != 1u)
        raise_record(p.status, p.groups, HSB_E_RECORD_IDENTITY, (uint32_t)i);
    else if (digest != h.digest)
        raise_record(p.status, p.groups, HSB_E_RECORD_CHECKSUM, (uint32_t)i);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t launch_records_encode(const void* payload, size_t payload_stride, size_t count, size_t record_bytes,
                                  uint64_t request, uint32_t layer, uint64_t first, void* records,
                                  cudaStream_t stream) {
    const int vec = aligned16(payload) && aligned16(records) && payload_stride % 16 == 0 && record_bytes % 16 == 0;
    const size_t blocks = (count + kRecordThreads - 1) / kRecordThreads;
    return launch_dependent(records_encode_kernel, dim3((unsigned)blocks), dim3(kRecordThreads), 0, stream, false,
                            static_cast<const unsigned char*>(payload), (unsigned long long)payload_stride,
                            (unsigned long long)count, (unsigned long long)record_bytes, (unsigned long long)request,
                            layer, (unsigned long long)first, static_cast<unsigned char*>(records), vec);
}

cudaError_t launch_records_verify(const void* window, size_t window_bytes, const uint64_t* offsets,
                                  const uint64_t* positions, const uint32_t* groups, size_t count, uint64_t request,
                                  uint32_t layer, size_t record_bytes, void* out, size_t out_stride,
                                  const uint32_t* out_rows, size_t out_capacity, int host_window,
                                  hsb_device_status* status, cudaStream_t stream) {
    VerifyParams p{};
    p.window = static_cast<const unsigned char*>(window);
    p.window_bytes = window_bytes;
    p.offsets = reinterpret_cast<const unsigned long long*>(offsets);
    p.positions = reinterpret_cast<const unsigned long long*>(positions);
    p.groups = groups;
    p.count = count;
    p.request = request;
    p.layer = layer;
    p.record_bytes = record_bytes;
    p.out = static_cast<unsigned char*>(out);
    p.out_stride = out_stride;
    p.out_rows = out_rows;
    p.out_capacity = out_capacity;
    p.status = status;
    p.host_window = host_window;
    p.vec = aligned16(window) && aligned16(out) && out_stride % 16 == 0 && record_bytes % 16 == 0;
    const size_t blocks = (count + kRecordThreads - 1) / kRecordThreads;
    return launch_dependent(records_verify_kernel, dim3((unsigned)blocks), dim3(kRecordThreads), 0, stream, false, p);
}

}  // namespace hsb
