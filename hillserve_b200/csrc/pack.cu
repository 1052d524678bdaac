// pack.cu -- stage 3: physical union and the packing / gathering of selected
// K/V rows into the delivery layout of runtime/gqa_pack.hpp:24-58:
//   K    [slot][query head][128]          (head-expanded, slot-major)
//   V    [query head][128][slot]          (transposed)
//   mask [query head][qpad][slot]  F32    (0 visible, -inf otherwise)
// Query head h reads physical KV head h/4 of each selected row.
//
// Every gather is index-driven and tiled: a CTA owns (query head, 32 slots);
// K slices (256 B per slot) are copied with 16-byte loads/stores, V slices go
// through a shared-memory tile so that the transposed stores of 32 slots are
// contiguous.  The grid is (slot-tile stride, query head): each CTA reads its
// head's list size once and walks only live tiles, so slot counts known only
// on the device (the selected k) cost no empty work.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kSlotTile = 32;
constexpr int kThreads = 256;
constexpr int kVPitch = kDim + 2;  // halfs per slot row of the V tile (bank spread)

__device__ __forceinline__ uint32_t head_size(const uint32_t* sizes, size_t sizes_stride, int h) {
    return sizes[(size_t)h * sizes_stride];
}

// Where the K and V slices of one slot come from; null means a zero slot.
struct SlotSource {
    const uint16_t* k;  // 128 halfs
    const uint16_t* v;  // 128 halfs
};

// Writes one (head, 32-slot) tile of the packed K and V from per-slot sources
// held in shared memory.  `live` slots of the tile have sources; the rest are
// zero when zero_rest is set, untouched otherwise.
__device__ void write_tile(const SlotSource* src, int live, bool zero_rest, int h, size_t s0,
                           size_t count, uint16_t* __restrict__ kout, uint16_t* __restrict__ vout,
                           uint16_t (*vt)[kVPitch]) {
    const int tid = threadIdx.x;
    const int limit = zero_rest ? kSlotTile : live;
    // K: 32 slots x 256 B; each thread moves 16-byte pieces.
    for (int i = tid; i < limit * 16; i += kThreads) {
        const int s = i >> 4, piece = i & 15;
        if (s0 + s >= count) continue;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (s < live && src[s].k) val = reinterpret_cast<const uint4*>(src[s].k)[piece];
        reinterpret_cast<uint4*>(kout + ((s0 + s) * kHeads + h) * kDim)[piece] = val;
    }
    // V: stage [slot][d] in shared memory, then store d-major.
    for (int i = tid; i < kSlotTile * 16; i += kThreads) {
        const int s = i >> 4, piece = i & 15;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (s < live && src[s].v) val = reinterpret_cast<const uint4*>(src[s].v)[piece];
        const uint32_t w[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            vt[s][piece * 8 + 2 * j] = (uint16_t)(w[j] & 0xffffu);
            vt[s][piece * 8 + 2 * j + 1] = (uint16_t)(w[j] >> 16);
        }
    }
    __syncthreads();
    for (int i = tid; i < kDim * kSlotTile; i += kThreads) {
        const int d = i >> 5, s = i & 31;
        if (s >= limit || s0 + s >= count) continue;
        vout[((size_t)h * kDim + d) * count + s0 + s] = vt[s][d];
    }
    __syncthreads();
}

// ------------------------------------------------------------------ union
__global__ void union_mark_kernel(const uint32_t* __restrict__ ids, size_t kstride,
                                  const uint32_t* __restrict__ sizes, size_t sizes_stride,
                                  size_t visible, uint32_t* __restrict__ seen,
                                  hsb_device_status* status) {
    const int h = blockIdx.y;
    const uint32_t size = head_size(sizes, sizes_stride, h);
    if (size > kstride) {
        raise_status(status, HSB_E_INVALID, h);
        return;
    }
    const uint32_t bit = 1u << h;
    for (size_t s = blockIdx.x * (size_t)blockDim.x + threadIdx.x; s < size; s += (size_t)gridDim.x * blockDim.x) {
        const uint32_t id = ids[h * kstride + s];
        if (id >= visible) {
            raise_status(status, HSB_E_UNION_DUPLICATE, h);
            continue;
        }
        if (atomicOr(&seen[id], bit) & bit) raise_status(status, HSB_E_UNION_DUPLICATE, h);
    }
}

// Single CTA: sorted list of IDs whose membership word is non-zero.  Each
// thread owns a contiguous run of words (a multiple of 4), read 32 words at a
// time with eight 16-byte loads issued together: one L2 round trip per 32
// words rather than one per word.  The workspace is a whole number of
// 256-byte blocks, so a 16-byte load never leaves it; words at or past
// `visible` are masked.
constexpr int kUnionChunk = 32;
__device__ __forceinline__ void union_chunk(const uint32_t* seen, size_t base, size_t end, uint32_t (&w)[kUnionChunk]) {
#pragma unroll
    for (int u = 0; u < kUnionChunk / 4; ++u) {
        const size_t i = base + 4 * u;
        const uint4 v = i < end ? reinterpret_cast<const uint4*>(seen)[i / 4] : make_uint4(0, 0, 0, 0);
        w[4 * u] = v.x;
        w[4 * u + 1] = v.y;
        w[4 * u + 2] = v.z;
        w[4 * u + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < kUnionChunk; ++j)
        if (base + j >= end) w[j] = 0;
}

__global__ void __launch_bounds__(1024) union_compact_kernel(const uint32_t* __restrict__ seen, size_t visible,
                                                             uint32_t* __restrict__ physical,
                                                             uint32_t* __restrict__ count) {
    __shared__ uint32_t warp_tot[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t seg = ((visible + 1023) / 1024 + 3) / 4 * 4;
    const size_t b0 = std::min(visible, tid * seg), b1 = std::min(visible, b0 + seg);
    uint32_t c = 0;
    uint32_t w[kUnionChunk];
    for (size_t base = b0; base < b1; base += kUnionChunk) {
        union_chunk(seen, base, b1, w);
#pragma unroll
        for (int j = 0; j < kUnionChunk; ++j) c += w[j] != 0;
    }
    uint32_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const uint32_t t = warp_tot[lane];
        uint32_t s = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_tot[lane] = s - t;
        if (lane == 31) *count = s;
    }
    __syncthreads();
    if (!c) return;
    uint32_t pos = warp_tot[warp] + x - c;
    for (size_t base = b0; base < b1; base += kUnionChunk) {
        if (seg > kUnionChunk || base != b0) union_chunk(seen, base, b1, w);  // one chunk: still in registers
#pragma unroll
        for (int j = 0; j < kUnionChunk; ++j)
            if (w[j]) physical[pos++] = (uint32_t)(base + j);
    }
}

// The whole union in one CTA when the membership words fit in shared memory
// (visible <= kUnionSmemWords): the words are cleared, marked by one warp
// per head and compacted there, so the step is one launch with no global
// workspace traffic (the three-node path -- clear, mark, compact -- spends
// most of its time between launches).  Same marks, statuses and sorted
// output as the path above.
constexpr size_t kUnionSmemWords = 49152;  // 192 KB
__global__ void __launch_bounds__(1024) union_smem_kernel(const uint32_t* __restrict__ ids, size_t kstride,
                                                          const uint32_t* __restrict__ sizes, size_t sizes_stride,
                                                          size_t visible, uint32_t* __restrict__ physical,
                                                          uint32_t* __restrict__ count, hsb_device_status* status) {
    extern __shared__ __align__(16) uint32_t seen_s[];
    __shared__ uint32_t warp_tot[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t words4 = (visible + 3) / 4;
    for (size_t i = tid; i < words4; i += 1024) reinterpret_cast<uint4*>(seen_s)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    {  // warp h marks head h
        const int h = warp;
        const uint32_t size = head_size(sizes, sizes_stride, h);
        if (size > kstride) {
            if (lane == 0) raise_status(status, HSB_E_INVALID, h);
        } else {
            const uint32_t bit = 1u << h;
            for (uint32_t s = lane; s < size; s += 32) {
                const uint32_t id = ids[h * kstride + s];
                if (id >= visible) {
                    raise_status(status, HSB_E_UNION_DUPLICATE, h);
                    continue;
                }
                if (atomicOr(&seen_s[id], bit) & bit) raise_status(status, HSB_E_UNION_DUPLICATE, h);
            }
        }
    }
    __syncthreads();
    // Compaction: warp w owns a contiguous run of 32-word rows; lane l reads
    // word l of each row (consecutive words: no bank conflicts), and a
    // ballot gives the row's members in ID order.
    const size_t rows = (visible + 31) / 32, rows_w = (rows + 31) / 32;
    const size_t r0 = std::min(rows, warp * rows_w), r1 = std::min(rows, r0 + rows_w);
    uint32_t c = 0;
    for (size_t r = r0; r < r1; ++r) {
        const size_t i = r * 32 + lane;
        c += __popc(__ballot_sync(0xffffffffu, i < visible && seen_s[i] != 0));
    }
    if (lane == 0) warp_tot[warp] = c;
    __syncthreads();
    if (warp == 0) {
        const uint32_t t = warp_tot[lane];
        uint32_t sum = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, sum, o);
            if (lane >= o) sum += y;
        }
        warp_tot[lane] = sum - t;
        if (lane == 31) *count = sum;
    }
    __syncthreads();
    uint32_t pos = warp_tot[warp];
    for (size_t r = r0; c && r < r1; ++r) {
        const size_t i = r * 32 + lane;
        const bool member = i < visible && seen_s[i] != 0;
        const uint32_t bits = __ballot_sync(0xffffffffu, member);
        if (member) physical[pos + __popc(bits & ((1u << lane) - 1u))] = (uint32_t)i;
        pos += __popc(bits);
    }
}

// ------------------------------------------------------------------ pack
__global__ void pack_offsets_kernel(const uint32_t* __restrict__ physical, size_t nphysical,
                                    uint64_t last_position, int32_t* __restrict__ offsets,
                                    hsb_device_status* status) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nphysical; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t id = physical[i];
        if (id > last_position || atomicCAS(&offsets[id], -1, (int32_t)i) != -1)
            raise_status(status, HSB_E_PACK_PHYSICAL, (int)i);
    }
}

struct PackParams {
    const uint32_t* ids;
    size_t kstride;
    const uint32_t* sizes;
    size_t sizes_stride;
    const int32_t* offsets;  // pack: ID -> payload row, -1 absent
    uint64_t last_position;
    const uint8_t* payload;
    const uint16_t* kcache;  // gather_cache
    const uint16_t* vcache;
    size_t stride_words;
    size_t visible;
    size_t count;
    int zero_padding;
    uint16_t* k;
    uint16_t* v;
    hsb_device_status* status;
};

// mode 0: payload rows via offsets (pack_gqa_workspace); mode 1: HBM cache.
template <int Mode>
__global__ void __launch_bounds__(kThreads) gather_tiles_kernel(const __grid_constant__ PackParams p) {
    __shared__ SlotSource src[kSlotTile];
    __shared__ __align__(16) uint16_t vt[kSlotTile][kVPitch];
    // Grid: x strides over the slot tiles of query head blockIdx.y.  The head's
    // list size is read once; tiles past it cost nothing unless the
    // reference's zero padding is requested.
    const int h = blockIdx.y;
    const uint32_t size = head_size(p.sizes, p.sizes_stride, h);
    const size_t limit = p.zero_padding ? p.count : std::min<size_t>(size, p.count);
    for (size_t s0 = (size_t)blockIdx.x * kSlotTile; s0 < limit || (s0 == 0 && blockIdx.x == 0);
         s0 += (size_t)gridDim.x * kSlotTile) {
        if (size > p.kstride || (Mode == 1 && size > p.count)) {
            if (threadIdx.x == 0 && s0 == 0) raise_status(p.status, HSB_E_INVALID, h);
            continue;
        }
        if (Mode == 0 && (size == 0 || size > p.count)) {
            if (threadIdx.x == 0 && s0 == 0) raise_status(p.status, HSB_E_PACK_SLOTS, h);
            continue;
        }
        const int live = (int)std::min<size_t>(kSlotTile, size > s0 ? size - s0 : 0);
        if (live == 0 && !p.zero_padding) continue;
        const int kh = h >> 2;
        if (threadIdx.x < kSlotTile) {
            SlotSource ss{nullptr, nullptr};
            const int s = threadIdx.x;
            if (s < live) {
                const uint32_t id = p.ids[h * p.kstride + s0 + s];
                if (Mode == 0) {
                    const int32_t row = id <= p.last_position ? p.offsets[id] : -1;
                    if (row < 0) {
                        raise_status(p.status, HSB_E_PACK_MISSING, h);
                    } else {
                        const uint16_t* r = reinterpret_cast<const uint16_t*>(p.payload + (size_t)row * kRowBytes);
                        ss.k = r + kh * kDim;
                        ss.v = r + 1024 + kh * kDim;
                    }
                } else {
                    if (id >= p.visible) {
                        raise_status(p.status, HSB_E_PACK_MISSING, h);
                    } else {
                        ss.k = p.kcache + (size_t)id * p.stride_words + kh * kDim;
                        ss.v = p.vcache + (size_t)id * p.stride_words + kh * kDim;
                    }
                }
            }
            src[s] = ss;
        }
        __syncthreads();
        write_tile(src, live, p.zero_padding != 0, h, s0, p.count, p.k, p.v, vt);
    }
}

struct MaskParams {
    const uint32_t* ids;
    size_t kstride;
    const uint32_t* sizes;
    size_t sizes_stride;
    const uint64_t* positions;
    size_t npositions, qpad, count;
    float* mask;
};

__global__ void mask_kernel(const __grid_constant__ MaskParams p) {
    const size_t total = (size_t)kHeads * p.qpad * p.count;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t s = i % p.count, hq = i / p.count, q = hq % p.qpad, h = hq / p.qpad;
        float val = -INFINITY;
        if (q < p.npositions && s < head_size(p.sizes, p.sizes_stride, (int)h) && s < p.kstride &&
            p.ids[h * p.kstride + s] <= p.positions[q])
            val = 0.0f;
        p.mask[i] = val;
    }
}

// ------------------------------------------------------------ prefetch map
// zero_padding false: the map's sources form a prefix of each head's slots
// (the rest -1) and only that prefix is written; a tile without a source
// is skipped.
__global__ void __launch_bounds__(kThreads) gather_map_kernel(const uint16_t* __restrict__ prefetched,
                                                              size_t prows, const uint16_t* __restrict__ misses,
                                                              size_t mrows, const int32_t* __restrict__ map,
                                                              size_t count, uint16_t* __restrict__ k,
                                                              uint16_t* __restrict__ v, hsb_device_status* status,
                                                              int zero_padding, const uint32_t* __restrict__ live_k) {
    __shared__ SlotSource src[kSlotTile];
    __shared__ __align__(16) uint16_t vt[kSlotTile][kVPitch];
    const size_t tiles_per_head = (count + kSlotTile - 1) / kSlotTile;
    // Live slots only, with their number on the device: walk only the tiles
    // that can hold one.
    const size_t live_tiles =
        (!zero_padding && live_k) ? (std::min<size_t>(*live_k, count) + kSlotTile - 1) / kSlotTile : tiles_per_head;
    const size_t total = live_tiles * kHeads;
    for (size_t item = blockIdx.x; item < total; item += gridDim.x) {
        const int h = (int)(item / live_tiles);
        const size_t s0 = (item % live_tiles) * kSlotTile;
        const int live = (int)std::min<size_t>(kSlotTile, count - s0);
        const int kh = h >> 2;
        if (threadIdx.x < kSlotTile) {
            SlotSource ss{nullptr, nullptr};
            const int s = threadIdx.x;
            if (s < live) {
                const long long row = map[h * count + s0 + s];
                const uint16_t* r = nullptr;
                if (row >= 0) {
                    if ((size_t)row < prows) r = prefetched + (size_t)row * 2048;
                    else raise_status(status, HSB_E_MAP_ROW, h);
                } else if (row <= -2) {
                    if ((size_t)(-2 - row) < mrows) r = misses + (size_t)(-2 - row) * 2048;
                    else raise_status(status, HSB_E_MAP_MISS, h);
                }
                if (r) {
                    ss.k = r + kh * kDim;
                    ss.v = r + 1024 + kh * kDim;
                }
            }
            src[s] = ss;
        }
        const int filled = __syncthreads_count(threadIdx.x < kSlotTile && src[threadIdx.x < kSlotTile ? threadIdx.x : 0].k);
        if (zero_padding) write_tile(src, live, true, h, s0, count, k, v, vt);
        else if (filled) write_tile(src, filled, false, h, s0, count, k, v, vt);
        else __syncthreads();  // src is rewritten by the next item
    }
}

// ------------------------------------------------------------ row staging
__global__ void stage_rows_kernel(const uint8_t* __restrict__ rows, const uint32_t* __restrict__ physical,
                                  const uint32_t* __restrict__ count, size_t max_rows,
                                  uint8_t* __restrict__ dst) {
    const size_t n = std::min<size_t>(*count, max_rows);
    // One warp per row: 32 lanes x 16 B x 8 = 4096 B.
    const size_t warps = (size_t)gridDim.x * (blockDim.x / 32);
    const int lane = threadIdx.x & 31;
    for (size_t r = blockIdx.x * (size_t)(blockDim.x / 32) + threadIdx.x / 32; r < n; r += warps) {
        const uint4* s = reinterpret_cast<const uint4*>(rows + (size_t)physical[r] * kRowBytes);
        uint4* d = reinterpret_cast<uint4*>(dst + r * kRowBytes);
        uint4 tmp[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) tmp[j] = s[lane + 32 * j];
#pragma unroll
        for (int j = 0; j < 8; ++j) d[lane + 32 * j] = tmp[j];
    }
}

// (slot-tile stride, query head): up to 16 CTAs per head.
dim3 tile_grid(size_t count) {
    return dim3((unsigned)std::max<size_t>(1, std::min<size_t>((count + kSlotTile - 1) / kSlotTile, 16)), kHeads);
}

int persistent_grid(size_t items, int per_sm) {
    const DeviceInfo& dev = device_info();
    return (int)std::max<size_t>(1, std::min<size_t>(items, (size_t)dev.sms * per_sm));
}

}  // namespace

size_t union_workspace_bytes(size_t visible) { return (visible * 4 + 255) / 256 * 256; }

cudaError_t launch_union(const uint32_t* ids, size_t kstride, const uint32_t* sizes, size_t sizes_stride,
                         size_t visible, uint32_t* physical, uint32_t* physical_count,
                         hsb_device_status* status, void* workspace, cudaStream_t stream) {
    if (visible <= kUnionSmemWords) {
        const size_t smem = (visible + 3) / 4 * 16;
        const DeviceInfo& dev = device_info();
        static thread_local int configured_device = -1;
        if (configured_device != dev.ordinal) {
            cudaError_t e = cudaFuncSetAttribute(union_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)(kUnionSmemWords * 4));
            if (e != cudaSuccess) return e;
            configured_device = dev.ordinal;
        }
        union_smem_kernel<<<1, 1024, smem, stream>>>(ids, kstride, sizes, sizes_stride, visible, physical,
                                                     physical_count, status);
        return cudaGetLastError();
    }
    uint32_t* seen = static_cast<uint32_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(seen, 0, visible * 4, stream);
    if (e != cudaSuccess) return e;
    const unsigned gx = (unsigned)std::max<size_t>(1, std::min<size_t>((kstride + 255) / 256, 64));
    union_mark_kernel<<<dim3(gx, kHeads), 256, 0, stream>>>(ids, kstride, sizes, sizes_stride, visible, seen, status);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    union_compact_kernel<<<1, 1024, 0, stream>>>(seen, visible, physical, physical_count);
    return cudaGetLastError();
}

size_t pack_workspace_bytes(uint64_t last_position) { return ((last_position + 1) * 4 + 255) / 256 * 256; }

cudaError_t launch_pack(const uint32_t* ids, size_t kstride, const uint32_t* sizes, size_t sizes_stride,
                        const uint64_t* positions, size_t npositions, uint64_t last_position,
                        const uint32_t* physical, size_t nphysical, const uint8_t* payload,
                        size_t count, uint16_t* k, uint16_t* v, float* mask,
                        hsb_device_status* status, void* workspace, cudaStream_t stream) {
    int32_t* offsets = static_cast<int32_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(offsets, 0xff, (last_position + 1) * 4, stream);
    if (e != cudaSuccess) return e;
    if (nphysical) {
        pack_offsets_kernel<<<persistent_grid((nphysical + 255) / 256, 4), 256, 0, stream>>>(
            physical, nphysical, last_position, offsets, status);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    PackParams p{};
    p.ids = ids;
    p.kstride = kstride;
    p.sizes = sizes;
    p.sizes_stride = sizes_stride;
    p.offsets = offsets;
    p.last_position = last_position;
    p.payload = payload;
    p.count = count;
    p.zero_padding = 1;
    p.k = k;
    p.v = v;
    p.status = status;
    gather_tiles_kernel<0><<<tile_grid(count), kThreads, 0, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (mask) {
        MaskParams m{ids, kstride, sizes, sizes_stride, positions, npositions, (npositions + 63) / 64 * 64, count, mask};
        const size_t total = (size_t)kHeads * m.qpad * count;
        mask_kernel<<<persistent_grid((total + 255) / 256, 8), 256, 0, stream>>>(m);
        e = cudaGetLastError();
    }
    return e;
}

cudaError_t launch_gather_map(const uint16_t* prefetched, size_t prefetched_rows, const uint16_t* misses,
                              size_t miss_rows, const int32_t* map, size_t count, uint16_t* k, uint16_t* v,
                              hsb_device_status* status, cudaStream_t stream, int zero_padding,
                              const uint32_t* live_k) {
    const size_t items = (count + kSlotTile - 1) / kSlotTile * kHeads;
    gather_map_kernel<<<persistent_grid(items, 8), kThreads, 0, stream>>>(prefetched, prefetched_rows, misses,
                                                                          miss_rows, map, count, k, v, status,
                                                                          zero_padding, live_k);
    return cudaGetLastError();
}

cudaError_t launch_gather_cache(const uint32_t* ids, size_t kstride, const uint32_t* sizes, size_t sizes_stride,
                                const uint16_t* kcache, const uint16_t* vcache, size_t stride_words,
                                size_t visible, size_t count, int zero_padding, uint16_t* k, uint16_t* v,
                                hsb_device_status* status, cudaStream_t stream) {
    PackParams p{};
    p.ids = ids;
    p.kstride = kstride;
    p.sizes = sizes;
    p.sizes_stride = sizes_stride;
    p.kcache = kcache;
    p.vcache = vcache;
    p.stride_words = stride_words;
    p.visible = visible;
    p.count = count;
    p.zero_padding = zero_padding;
    p.k = k;
    p.v = v;
    p.status = status;
    gather_tiles_kernel<1><<<tile_grid(count), kThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_stage_rows(const uint8_t* rows, const uint32_t* physical, const uint32_t* count,
                              size_t max_rows, uint8_t* dst, cudaStream_t stream) {
    const int grid = persistent_grid((max_rows + 7) / 8, 4);
    stage_rows_kernel<<<grid, 256, 0, stream>>>(rows, physical, count, max_rows, dst);
    return cudaGetLastError();
}

}  // namespace hsb
