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
// owns a record; the GPU's parallelism is across records, and a warp moves
// its 32 records' bytes with coalesced loads (records_kernel).  The prime is
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

// Scalar form: one thread hashes `bytes` bytes from src, copying them to
// dst (may be null).  Used for records that are not 16-byte aligned.
__device__ uint64_t hash_copy_bytes(const unsigned char* __restrict__ src, unsigned char* __restrict__ dst,
                                    size_t bytes) {
    Fnv h{(uint32_t)kFnvSeed, (uint32_t)(kFnvSeed >> 32)};
    for (size_t i = 0; i < bytes; ++i) {
        const unsigned char b = src[i];
        if (dst) dst[i] = b;
        fnv_byte(h, b);
    }
    return fnv_value(h);
}

struct alignas(16) RecordHeader {  // moved as two 16-byte words
    uint64_t digest, position, request;
    uint32_t layer, version;
};
static_assert(sizeof(RecordHeader) == 32, "fixed on-disk header");

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

// Both directions share one kernel.  Encode: record i's payload comes from
// src + i * src_stride and goes, after its header, to records + i * (B+32).
// Verify: record i sits at window + offsets[i]; its payload goes to
// out + row * dst_stride.
struct RecordParams {
    const unsigned char* src;  // encode: payload rows
    unsigned long long src_stride;
    const unsigned char* window;  // verify
    unsigned long long window_bytes;
    const unsigned long long* offsets;
    const unsigned long long* positions;
    const uint32_t* groups;
    const uint32_t* out_rows;
    unsigned long long out_capacity;
    unsigned char* dst;  // encode: the record image; verify: the output rows
    unsigned long long dst_stride;
    unsigned long long count, record_bytes, request, first;
    uint32_t layer;
    int vec;  // 16-byte path allowed (bases, strides and B multiples of 16)
    hsb_device_status* status;
};

constexpr int kPitch = 144;  // staged line pitch: 128 bytes + 16 (conflict-free 16-byte reads)
constexpr int kWarpsMax = 4;

// A warp owns 32 records, lane l hashing record l.  The payloads move a
// 128-byte line of each record at a time: the warp loads line j of its 32
// records with coalesced 16-byte loads (eight lanes per line), writes them
// out (the copy) and into a shared-memory row per record, and each lane
// hashes its own row while the warp's loads of line j+1 are in flight.
template <bool kVerify>
__global__ void __launch_bounds__(kWarpsMax * 32) records_kernel(const __grid_constant__ RecordParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) unsigned char stage[kWarpsMax][32 * kPitch];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned long long r0 = ((unsigned long long)blockIdx.x * (blockDim.x >> 5) + warp) * 32;
    if (r0 >= p.count) return;  // the whole warp leaves together
    const unsigned long long i = r0 + lane;
    const bool live = i < p.count;
    const unsigned long long B = p.record_bytes;

    // This lane's record.
    const unsigned char* src = nullptr;
    unsigned char* dst = nullptr;
    RecordHeader head{};
    bool bounds_ok = true;
    if (live) {
        if (kVerify) {
            const unsigned long long off = p.offsets[i];
            const unsigned long long row = p.out_rows ? p.out_rows[i] : i;
            bounds_ok = off <= p.window_bytes && p.window_bytes - off >= B + 32 && row < p.out_capacity;
            if (bounds_ok) {
                src = p.window + off + 32;
                dst = p.dst + row * p.dst_stride;
                if (p.vec && (off & 15u) == 0) {
                    reinterpret_cast<uint4*>(&head)[0] = reinterpret_cast<const uint4*>(p.window + off)[0];
                    reinterpret_cast<uint4*>(&head)[1] = reinterpret_cast<const uint4*>(p.window + off)[1];
                } else {
                    unsigned char* d = reinterpret_cast<unsigned char*>(&head);
                    for (int b = 0; b < 32; ++b) d[b] = p.window[off + b];
                }
            }
        } else {
            src = p.src + i * p.src_stride;
            dst = p.dst + i * (B + 32) + 32;
        }
    }
    const bool vec_mine = src != nullptr && p.vec && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    const unsigned vec_mask = __ballot_sync(0xffffffffu, vec_mine);

    // Records whose lines this lane moves: q = 4k + lane/8, chunk lane % 8.
    const unsigned char* lsrc[8];
    unsigned char* ldst[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int q = 4 * k + (lane >> 3);
        const unsigned long long s = __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(src), q);
        const unsigned long long d = __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), q);
        const bool on = (vec_mask >> q) & 1u;
        lsrc[k] = on ? reinterpret_cast<const unsigned char*>(s) + (lane & 7) * 16 : nullptr;
        ldst[k] = on ? reinterpret_cast<unsigned char*>(d) + (lane & 7) * 16 : nullptr;
    }
    Fnv h{(uint32_t)kFnvSeed, (uint32_t)(kFnvSeed >> 32)};
    const unsigned long long chunks = B / 16, lines = (chunks + 7) / 8;
    unsigned char* rows = stage[warp];
    uint4 reg[8];
    auto load_line = [&](unsigned long long j) {
        const unsigned long long c = j * 8 + (lane & 7);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            reg[k] = lsrc[k] && c < chunks ? __ldcg(reinterpret_cast<const uint4*>(lsrc[k] + j * 128))
                                           : make_uint4(0, 0, 0, 0);
    };
    if (vec_mask) {
        load_line(0);
        for (unsigned long long j = 0; j < lines; ++j) {
            const unsigned long long c = j * 8 + (lane & 7);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                if (lsrc[k] && c < chunks) {
                    const int q = 4 * k + (lane >> 3);
                    *reinterpret_cast<uint4*>(rows + q * kPitch + (lane & 7) * 16) = reg[k];
                    *reinterpret_cast<uint4*>(ldst[k] + j * 128) = reg[k];
                }
            }
            __syncwarp();
            if (j + 1 < lines) load_line(j + 1);
            if (vec_mine) {
                const unsigned long long n = chunks - j * 8 < 8 ? chunks - j * 8 : 8;
                const unsigned char* mine = rows + lane * kPitch;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if ((unsigned long long)k < n) {
                        const uint4 w = *reinterpret_cast<const uint4*>(mine + k * 16);
                        fnv_word(h, w.x);
                        fnv_word(h, w.y);
                        fnv_word(h, w.z);
                        fnv_word(h, w.w);
                    }
                }
            }
            __syncwarp();
        }
    }
    if (!live) return;
    uint64_t digest = fnv_value(h);
    if (src && !vec_mine) digest = hash_copy_bytes(src, dst, B);  // a record off the 16-byte grid

    if (kVerify) {
        // The reference checks the record's identity before its digest
        // (policy/full_gqa_runtime.cpp:397-408, segmented_store.cpp:116-119).
        if (!bounds_ok)
            raise_record(p.status, p.groups, HSB_E_RECORD_BOUNDS, (uint32_t)i);
        else if (head.position != p.positions[i] || head.request != p.request || head.layer != p.layer ||
                 head.version != 1u)
            raise_record(p.status, p.groups, HSB_E_RECORD_IDENTITY, (uint32_t)i);
        else if (digest != head.digest)
            raise_record(p.status, p.groups, HSB_E_RECORD_CHECKSUM, (uint32_t)i);
    } else {
        RecordHeader out{digest, p.first + i, p.request, p.layer, 1u};
        unsigned char* rec = dst - 32;
        if (vec_mine) {
            reinterpret_cast<uint4*>(rec)[0] = reinterpret_cast<const uint4*>(&out)[0];
            reinterpret_cast<uint4*>(rec)[1] = reinterpret_cast<const uint4*>(&out)[1];
        } else {
            const unsigned char* b = reinterpret_cast<const unsigned char*>(&out);
            for (int j = 0; j < 32; ++j) rec[j] = b[j];
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Warps per block: one for small sets, so that few records still spread
// over many SMs; four otherwise.
unsigned records_block(size_t count) {
    return count >= (size_t)device_info().sms * 4 * 32 ? kWarpsMax * 32 : 32;
}

cudaError_t launch_records_encode(const void* payload, size_t payload_stride, size_t count, size_t record_bytes,
                                  uint64_t request, uint32_t layer, uint64_t first, void* records,
                                  cudaStream_t stream) {
    RecordParams p{};
    p.src = static_cast<const unsigned char*>(payload);
    p.src_stride = payload_stride;
    p.dst = static_cast<unsigned char*>(records);
    p.count = count;
    p.record_bytes = record_bytes;
    p.request = request;
    p.first = first;
    p.layer = layer;
    p.vec = aligned16(payload) && aligned16(records) && payload_stride % 16 == 0 && record_bytes % 16 == 0;
    const unsigned block = records_block(count);
    const size_t grid = (count + block - 1) / block;
    return launch_dependent(records_kernel<false>, dim3((unsigned)grid), dim3(block), 0, stream, false, p);
}

cudaError_t launch_records_verify(const void* window, size_t window_bytes, const uint64_t* offsets,
                                  const uint64_t* positions, const uint32_t* groups, size_t count, uint64_t request,
                                  uint32_t layer, size_t record_bytes, void* out, size_t out_stride,
                                  const uint32_t* out_rows, size_t out_capacity, int host_window,
                                  hsb_device_status* status, cudaStream_t stream) {
    (void)host_window;  // no prefetch hints are issued, so a pinned host window needs nothing different
    RecordParams p{};
    p.window = static_cast<const unsigned char*>(window);
    p.window_bytes = window_bytes;
    p.offsets = reinterpret_cast<const unsigned long long*>(offsets);
    p.positions = reinterpret_cast<const unsigned long long*>(positions);
    p.groups = groups;
    p.out_rows = out_rows;
    p.out_capacity = out_capacity;
    p.dst = static_cast<unsigned char*>(out);
    p.dst_stride = out_stride;
    p.count = count;
    p.record_bytes = record_bytes;
    p.request = request;
    p.layer = layer;
    p.status = status;
    p.vec = aligned16(window) && aligned16(out) && out_stride % 16 == 0 && record_bytes % 16 == 0;
    const unsigned block = records_block(count);
    const size_t grid = (count + block - 1) / block;
    return launch_dependent(records_kernel<true>, dim3((unsigned)grid), dim3(block), 0, stream, false, p);
}

}  // namespace hsb
