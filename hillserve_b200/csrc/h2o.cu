// h2o.cu -- H2O residency statistics: per physical KV head and key, the sum
// of the actual F32 softmax probabilities of the four query heads sharing
// that KV head over every valid query of the block
// (runtime/gqa_h2o_stats.cu:41-57, sum_actual_attention).
//
// Numerics.  out[kv][key] = (((+0 + P[key][0][4kv]) + P[key][1][4kv]) + ...)
// in the order query head 4kv .. 4kv+3 (outer), query 0 .. Q-1 (inner), each
// addition rounded to F32 -- the reference kernel's __fadd_rn chain and
// H2OResidency::observe_attention's CPU order (policy/h2o_residency.cpp:66-76).
// F32 addition is not associative, so one thread owns each output and walks
// its whole chain; the parallelism is across the 8 x keys outputs and the
// work is a pure HBM stream (each probability is read once).
//
// Kernels.
//  - h2o_group_sum_tma_kernel: key-contiguous tensors (nb0 == 4, the other
//    strides and the base 16-byte aligned -- ggml's layout).  A 3-D tensor
//    map {key, query, Q head} feeds 16-row boxes of KT keys through a ring of
//    shared-memory stages filled by a producer warp (TMA) and drained by KT
//    consumer threads, thread t owning key t of the tile.  When 4Q <= 16 one
//    box {KT, Q, 4 heads} holds a whole item (decode: Q = 1); otherwise the
//    boxes are {KT, 16 queries, 1 head}, walked head-major.  The grid is
//    persistent (a few CTAs per SM over items = key tiles x 8 KV heads, the
//    same number of items each), so the producer runs ahead across item
//    boundaries.  KT is 256, or 64 when
//    fewer than two wide items per SM exist.
//  - h2o_group_sum_strided_kernel: any other F32 strides (holes between
//    keys, as in the reference's strided test); one thread per (KV head,
//    key) with eight independent loads issued ahead of their additions.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kH2ORows = 16;  // probability rows per TMA box

struct H2OTmaParams {
    CUtensorMap map;  // {key, query, Q head} F32, box {KT, rq, hb}
    float* out;       // [8][keys]
    unsigned long long keys;
    unsigned queries;
    unsigned rq, hb;    // rows of queries and Q heads per box
    unsigned per_head;  // boxes per query head (hb == 1)
    unsigned items;     // key tiles x 8
    hsb_device_status* status;
};

template <int KT, int S>
constexpr size_t h2o_smem_bytes() {
    return (size_t)S * KT * kH2ORows * sizeof(float) + 2 * S * sizeof(uint64_t);
}

template <int KT, int S>
__global__ void __launch_bounds__(KT + 32) h2o_group_sum_tma_kernel(const __grid_constant__ H2OTmaParams p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float* ring = reinterpret_cast<float*>(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)S * KT * kH2ORows * sizeof(float));
    uint64_t* empty = full + S;
    constexpr int kConsumerWarps = KT / 32;
    constexpr unsigned kStage = KT * kH2ORows;  // floats per stage
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned boxes = p.hb == 4 ? 1u : 4u * p.per_head;  // boxes per item
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane != 0) return;
        // ---------------- producer
        const uint32_t bytes = (uint32_t)KT * p.rq * p.hb * sizeof(float);
        uint32_t it = 0;
        bool ok = true;
        for (unsigned item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
            const unsigned kv = item & 7u, tile = item >> 3;
            for (unsigned b = 0; b < boxes; ++b, ++it) {
                const uint32_t s = it % S;
                if (it >= (uint32_t)S && !mbar_wait(&empty[s], ((it / S) - 1) & 1)) {
                    raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                    ok = false;
                    break;
                }
                const int z = (int)(kv * 4 + (p.hb == 4 ? 0u : b / p.per_head));
                const int y = p.hb == 4 ? 0 : (int)((b % p.per_head) * p.rq);
                mbar_arrive_expect_tx(&full[s], bytes);
                tma_load_3d(ring + s * kStage, &p.map, (int)(tile * KT), y, z, &full[s]);
            }
        }
        if (!ok) {  // let copies in flight land before shared memory is released
            const uint32_t first = it > (uint32_t)S ? it - S : 0;
            for (uint32_t j = first; j < it; ++j) (void)mbar_wait(&full[j % S], (j / S) & 1);
        }
        return;
    }

    // ---------------- consumers: thread t sums key t of the tile
    const unsigned t = threadIdx.x;
    uint32_t it = 0;
    for (unsigned item = blockIdx.x; item < p.items; item += gridDim.x) {
        const unsigned kv = item & 7u, tile = item >> 3;
        float sum = 0.0f;
        for (unsigned b = 0; b < boxes; ++b, ++it) {
            const uint32_t s = it % S;
            if (!mbar_wait(&full[s], (it / S) & 1)) {
                raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                return;
            }
            // Rows of the box in chain order: head-major, then query.
            const unsigned rows = p.hb == 4 ? 4 * p.queries : min(p.rq, p.queries - (b % p.per_head) * p.rq);
            const float* col = ring + s * kStage + t;
            float v[kH2ORows];
#pragma unroll
            for (int r = 0; r < kH2ORows; ++r) v[r] = col[r * KT];
#pragma unroll
            for (int r = 0; r < kH2ORows; ++r)
                if ((unsigned)r < rows) sum = __fadd_rn(sum, v[r]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        const unsigned long long key = (unsigned long long)tile * KT + t;
        if (key < p.keys) p.out[kv * p.keys + key] = sum;
    }
}

__global__ void __launch_bounds__(256) h2o_group_sum_strided_kernel(const unsigned char* __restrict__ probs,
                                                                   unsigned long long keys,
                                                                   unsigned long long queries,
                                                                   unsigned long long nb0, unsigned long long nb1,
                                                                   unsigned long long nb2, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const unsigned long long key = (unsigned long long)blockIdx.x * 256 + threadIdx.x;
    const unsigned kv = blockIdx.y;
    if (key >= keys) return;
    float sum = 0.0f;
    for (unsigned lane = 0; lane < 4; ++lane) {
        const unsigned char* row = probs + key * nb0 + (unsigned long long)(kv * 4 + lane) * nb2;
        for (unsigned long long q0 = 0; q0 < queries; q0 += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                v[j] = q0 + j < queries ? __ldcs(reinterpret_cast<const float*>(row + (q0 + j) * nb1)) : 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (q0 + j < queries) sum = __fadd_rn(sum, v[j]);
        }
    }
    out[kv * keys + key] = sum;
}

struct H2OVariant {
    int keys_per_tile;
    size_t smem;
    void (*kernel)(H2OTmaParams);
};
constexpr int kWideStages = 6, kNarrowStages = 8;
const H2OVariant kWide{256, h2o_smem_bytes<256, kWideStages>(), h2o_group_sum_tma_kernel<256, kWideStages>};
const H2OVariant kNarrow{64, h2o_smem_bytes<64, kNarrowStages>(), h2o_group_sum_tma_kernel<64, kNarrowStages>};

// CTAs per SM of each variant on the current device (configured once).
struct H2OOccupancy {
    int ordinal = -1;
    int wide = 0, narrow = 0;
};

cudaError_t h2o_occupancy(int* wide, int* narrow) {
    static thread_local H2OOccupancy occ;
    const DeviceInfo& dev = device_info();
    if (occ.ordinal != dev.ordinal) {
        for (const H2OVariant* v : {&kWide, &kNarrow}) {
            cudaError_t e = cudaFuncSetAttribute(v->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)v->smem);
            if (e != cudaSuccess) return e;
        }
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ.wide, kWide.kernel, 256 + 32, kWide.smem);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ.narrow, kNarrow.kernel, 64 + 32, kNarrow.smem);
        if (e != cudaSuccess) return e;
        occ.ordinal = dev.ordinal;
    }
    *wide = std::max(occ.wide, 1);
    *narrow = std::max(occ.narrow, 1);
    return cudaSuccess;
}

bool encode_probability_map(CUtensorMap* map, const void* probs, size_t keys, size_t queries, size_t nb1,
                            size_t nb2, unsigned kt, unsigned rq, unsigned hb) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)keys, (cuuint64_t)queries, (cuuint64_t)kHeads};
    const cuuint64_t strides[2] = {(cuuint64_t)nb1, (cuuint64_t)nb2};
    const cuuint32_t box[3] = {kt, rq, hb};
    const cuuint32_t estr[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(probs), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_h2o_group_sums(const void* probs, size_t keys, size_t queries, size_t nb0, size_t nb1,
                                  size_t nb2, float* out, hsb_device_status* status, cudaStream_t stream) {
    const DeviceInfo& dev = device_info();
    const uintptr_t base = reinterpret_cast<uintptr_t>(probs);
    const bool tma_shape = nb0 == sizeof(float) && nb1 % 16 == 0 && nb2 % 16 == 0 && base % 16 == 0 &&
                           nb1 < (1ull << 40) && nb2 < (1ull << 40) && keys < (1ull << 32) &&
                           queries < (1ull << 31);
    if (tma_shape) {
        int wide_per_sm = 1, narrow_per_sm = 1;
        cudaError_t e = h2o_occupancy(&wide_per_sm, &narrow_per_sm);
        if (e != cudaSuccess) return e;
        const size_t wide_items = (keys + 255) / 256 * kKvHeads;
        const bool wide = wide_items >= 2 * (size_t)dev.sms;
        const H2OVariant& v = wide ? kWide : kNarrow;
        const size_t items = (keys + v.keys_per_tile - 1) / v.keys_per_tile * kKvHeads;
        H2OTmaParams t{};
        if (4 * queries <= (size_t)kH2ORows) {
            t.rq = (unsigned)queries;
            t.hb = 4;
            t.per_head = 1;
        } else {
            t.rq = (unsigned)std::min<size_t>(queries, kH2ORows);
            t.hb = 1;
            t.per_head = (unsigned)((queries + t.rq - 1) / t.rq);
        }
        // The last encoded map of this thread is reused when the same tensor
        // is reduced again (a reducer is called once per layer on one buffer).
        struct MapCache {
            int device = -1;
            const void* probs = nullptr;
            size_t keys = 0, queries = 0, nb1 = 0, nb2 = 0;
            unsigned kt = 0;
            CUtensorMap map;
        };
        static thread_local MapCache cache;
        bool have = cache.device == dev.ordinal && cache.probs == probs && cache.keys == keys &&
                    cache.queries == queries && cache.nb1 == nb1 && cache.nb2 == nb2 &&
                    cache.kt == (unsigned)v.keys_per_tile;
        if (!have && items < (1ull << 31) &&
            encode_probability_map(&t.map, probs, keys, queries, nb1, nb2, (unsigned)v.keys_per_tile, t.rq, t.hb)) {
            cache.map = t.map;
            cache.device = dev.ordinal;
            cache.probs = probs;
            cache.keys = keys;
            cache.queries = queries;
            cache.nb1 = nb1;
            cache.nb2 = nb2;
            cache.kt = (unsigned)v.keys_per_tile;
            have = true;
        }
        if (have) {
            t.map = cache.map;
            t.out = out;
            t.keys = keys;
            t.queries = (unsigned)queries;
            t.items = (unsigned)items;
            t.status = status;
            // As many CTAs as fit, trimmed so that every CTA owns the same
            // number of items (no CTA runs a last item alone).
            const size_t slots = (size_t)dev.sms * (wide ? wide_per_sm : narrow_per_sm);
            const size_t rounds = (items + slots - 1) / slots;
            const unsigned grid = (unsigned)((items + rounds - 1) / rounds);
            return launch_dependent(v.kernel, dim3(grid), dim3(v.keys_per_tile + 32), v.smem, stream, false, t);
        }
    }
    const size_t blocks = (keys + 255) / 256;
    return launch_dependent(h2o_group_sum_strided_kernel, dim3((unsigned)blocks, kKvHeads), dim3(256), 0, stream,
                            false, static_cast<const unsigned char*>(probs), (unsigned long long)keys,
                            (unsigned long long)queries, (unsigned long long)nb0, (unsigned long long)nb1,
                            (unsigned long long)nb2, out);
}

}  // namespace hsb
