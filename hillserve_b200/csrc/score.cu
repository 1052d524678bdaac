// score.cu -- stage 1: full-GQA F16 key scoring under the
// HS_FULL_GQA_PIPELINE_F16_V3 contract (kernels/full_gqa_pipeline/ABI.json),
// bit-identical to FullGqaCpuScorer (policy/full_gqa_cpu.cpp:23-92).
//
// Numerics.  S[h,t] = F16_RNE( sum_{c=0..127} q[h,c]*k[t,h/4,c] ) with the sum
// taken in FP32, from +0, channel 0 first.  The reference forbids FMA because
// it computes fl(q*k) and then adds.  Here the product of two binary16 values
// has at most 22 significant bits and magnitude in [2^-48, 2^32] (or is zero),
// so it is EXACT in binary32: fl(q*k) == q*k.  Hence
//     fl(acc + fl(q*k)) == fl(acc + q*k) == fma(q, k, acc)
// for every input, signed zeros included (a +0 accumulator plus a -0 product
// is +0 either way).  The kernel therefore issues one FMA per (head, channel)
// and keeps the reference's order, which is what makes the result bit-exact;
// it never reassociates the channel sum.
//
// Memory.  The scorer streams K once (2 KB per token) and is HBM-bound.  The
// production kernel (score_tma_kernel, below) loads 32-token x 64-channel
// tiles with 3-D tensor-map TMA copies and runs two CTAs per SM.  The
// row-copy kernel (score_v3_kernel) is kept for the case where a tensor map
// cannot be encoded: one persistent CTA per SM, a producer warp moving whole
// 2 KB token rows with 1-D bulk copies into rows of 2064-byte pitch (eight
// consecutive lanes' 16-byte reads fall in distinct bank groups), and Q in
// shared memory as FP32 [kv head][channel][4 heads] (one broadcast 16-byte
// load per channel).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kTile = 32;                       // tokens per stage (one per lane)
constexpr int kStages = 3;
constexpr int kPitch = 2048 + 16;               // bytes per token row in smem
constexpr int kStageBytes = kTile * kPitch;     // 66048
constexpr int kQBytes = kKvHeads * kDim * kGroup * 4;  // 16384
constexpr int kConsumerWarps = kKvHeads;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSmemBytes = kQBytes + kStages * kStageBytes + 2 * kStages * 8;

struct ScoreParams {
    const uint16_t* q;
    const uint16_t* data[HSB_MAX_VIEWS];
    unsigned long long first[HSB_MAX_VIEWS + 1];  // token prefix offsets
    unsigned long long stride[HSB_MAX_VIEWS];     // words per token
    int nviews;
    unsigned long long tokens;      // tokens scored by this launch
    uint16_t* out;                  // [32][out_stride]
    uint16_t* keys;                 // optional [32][out_stride] order keys of normalised scores
    unsigned long long out_stride;  // columns of the output matrix
    unsigned long long col0;        // first output column of this launch
    hsb_device_status* status;
    ScoreExtras extras;
};

// CTA 0 clears the extras' buffers and the unused tail of the head-0 partials.
// Threads [0, nthreads) of the CTA take part.
__device__ __forceinline__ void clear_extras(const ScoreExtras& x, unsigned nthreads) {
    if (blockIdx.x != 0) return;
    for (int i = 0; i < 3; ++i)
        for (unsigned w = threadIdx.x; w < x.zero_words[i]; w += nthreads) x.zero[i][w] = 0u;
    if (x.h0)
        for (unsigned w = gridDim.x + threadIdx.x; w < kH0Partials; w += nthreads) x.h0[w] = 0u;
}

// Running head-0 partial of one lane: order key of a normalised score.
__device__ __forceinline__ void track_head0(uint32_t key, uint32_t& mx, uint32_t& bad) {
    bad |= key_nonfinite(key) ? 1u : 0u;
    mx = key_nan(key) ? mx : max(mx, key);
}
__device__ __forceinline__ void write_head0(const ScoreExtras& x, uint32_t mx, uint32_t bad) {
    mx = __reduce_max_sync(0xffffffffu, mx);
    bad = __reduce_or_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0) x.h0[blockIdx.x] = (bad << 16) | mx;
}

__device__ __forceinline__ const uint16_t* token_row(const ScoreParams& p, unsigned long long t) {
    int v = 0;
#pragma unroll 1
    while (v + 1 < p.nviews && t >= p.first[v + 1]) ++v;
    return p.data[v] + (t - p.first[v]) * p.stride[v];
}

__global__ void __launch_bounds__(kThreads, 1) score_v3_kernel(const __grid_constant__ ScoreParams p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char smem[];
    float* qs = reinterpret_cast<float*>(smem);
    unsigned char* tiles = smem + kQBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(tiles + kStages * kStageBytes);
    uint64_t* empty = full + kStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    clear_extras(p.extras, blockDim.x);
    for (int i = threadIdx.x; i < kHeads * kDim; i += blockDim.x) {
        const int h = i >> 7, c = i & 127;
        qs[((h >> 2) * kDim + c) * kGroup + (h & 3)] = half_value(p.q[i]);
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    const unsigned long long ntiles = (p.tokens + kTile - 1) / kTile;
    if (warp == kConsumerWarps) {
        // ---------------- producer: one bulk copy per token row
        uint32_t it = 0;
        bool ok = true;
        for (unsigned long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
            const uint32_t s = it % kStages;
            if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1)) {
                raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                ok = false;
                break;
            }
            const unsigned long long t0 = tile * kTile;
            const uint32_t rows = (uint32_t)min((unsigned long long)kTile, p.tokens - t0);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], rows * 2048u);
            __syncwarp();
            if ((uint32_t)lane < rows)
                bulk_copy_g2s(tiles + s * kStageBytes + lane * kPitch, token_row(p, t0 + lane), 2048u,
                              &full[s]);
        }
        if (!ok && lane == 0) {
            // Let copies already in flight land before the CTA's shared
            // memory is released (each wait is bounded).
            const uint32_t first = it > kStages ? it - kStages : 0;
            for (uint32_t j = first; j < it; ++j) (void)mbar_wait(&full[j % kStages], (j / kStages) & 1);
        }
        return;
    }

    // ---------------- consumers: warp = KV head, lane = token of the tile
    const int kh = warp;
    const float4* qv = reinterpret_cast<const float4*>(qs) + kh * kDim;
    uint32_t it = 0, h0max = 0, h0bad = 0;
    for (unsigned long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const uint32_t s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1)) {
            raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
            return;
        }
        const unsigned long long t = tile * kTile + lane;
        if (t < p.tokens) {
            const unsigned char* row = tiles + s * kStageBytes + lane * kPitch + kh * (kDim * 2);
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
            for (int c8 = 0; c8 < kDim / 8; ++c8) {
                const uint4 w = *reinterpret_cast<const uint4*>(row + c8 * 16);
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint16_t bits = (uint16_t)((j & 1) ? (words[j >> 1] >> 16) : (words[j >> 1] & 0xffffu));
                    const float k = half_value(bits);
                    const float4 q = qv[c8 * 8 + j];
                    // Exact product => FMA equals the reference's mul-then-add.
                    a0 = __fmaf_rn(q.x, k, a0);
                    a1 = __fmaf_rn(q.y, k, a1);
                    a2 = __fmaf_rn(q.z, k, a2);
                    a3 = __fmaf_rn(q.w, k, a3);
                }
            }
            const unsigned long long at = (unsigned long long)(kh * kGroup) * p.out_stride + p.col0 + t;
            const uint16_t s0 = half_bits(a0), s1 = half_bits(a1), s2 = half_bits(a2), s3 = half_bits(a3);
            uint16_t* o = p.out + at;
            o[0] = s0;
            o[p.out_stride] = s1;
            o[2 * p.out_stride] = s2;
            o[3 * p.out_stride] = s3;
            if (p.keys) {
                uint16_t* kk = p.keys + at;
                const uint32_t key0 = order_key(scale_half(s0));
                kk[0] = (uint16_t)key0;
                kk[p.out_stride] = (uint16_t)order_key(scale_half(s1));
                kk[2 * p.out_stride] = (uint16_t)order_key(scale_half(s2));
                kk[3 * p.out_stride] = (uint16_t)order_key(scale_half(s3));
                if (kh == 0) track_head0(key0, h0max, h0bad);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (kh == 0 && p.extras.h0) write_head0(p.extras, h0max, h0bad);
}

// ===================================================================== TMA
// The production scorer.  Per CTA: one producer warp and eight consumer
// warps; two CTAs per SM.  A work tile is 32 tokens x 8 KV heads; it is
// brought in as two 32 KB half-channel stages (channels 0-63, then 64-127) by
// TMA loads of a 3-D tensor map whose dimensions are ordered {channel, token,
// KV head}, so the shared tile is [KV head][token][64 channels] with the
// 128-byte swizzle (16-byte column XOR token % 8), three stages deep.
// Warp = KV head, lane = token: Q reads are whole-warp broadcasts, K reads of
// any eight consecutive lanes hit eight different columns (conflict-free), and
// the four scores of a lane go to four head rows with coalesced stores.  Q is
// kept as F16 [kv][c][4] and the products use the mixed-precision FMA
// (F16 x F16 + F32 -> F32, one rounding), exact for the same reason as above:
// no conversion instructions at all.
constexpr int kTTile = 32;                               // tokens per tile
constexpr int kTHalf = 64;                               // channels per stage
constexpr int kTStageBytes = kTTile * kKvHeads * kTHalf * 2;  // 32768
constexpr int kTStages = 3;
constexpr int kTConsumerWarps = 8;
constexpr int kTThreads = (kTConsumerWarps + 1) * 32;
constexpr int kTQBytes = kDim * kKvHeads * kGroup * 2;   // 8192
constexpr int kTSmemBytes = 1024 + kTStages * kTStageBytes + kTQBytes + 64;
// Key tiles per CTA prefetched into L2 before the grid dependency wait.  In
// the 32-layer decode step at N 32K (three alternating runs each, one box):
// none 0.965 ms, one 0.954 ms, two 0.968 ms per step.  A deeper prefetch
// floods DRAM while the previous selector's epilogue gathers its rows.
constexpr int kTPrefetchTiles = 1;

struct TmaParams {
    CUtensorMap maps[HSB_MAX_VIEWS];
    const uint16_t* q;
    unsigned long long view_tokens[HSB_MAX_VIEWS];
    unsigned long long view_tile0[HSB_MAX_VIEWS + 1];  // tile prefix per view
    unsigned long long view_col[HSB_MAX_VIEWS];        // first output column
    int nviews;
    unsigned long long tiles;
    uint16_t* out;
    uint16_t* keys;
    unsigned long long out_stride;
    hsb_device_status* status;
    ScoreExtras extras;
    // Batch of sequences (blockIdx.y = sequence; 1 outside shard steps): one
    // view of batch * seq_tokens tokens, sequence b at token b * seq_tokens;
    // per sequence, q advances by q_seq, out / keys by out_seq elements and
    // extras.h0 by kH0Partials words.
    unsigned long long seq_tokens, q_seq, out_seq;
    int prefetch_tiles;  // key tiles per CTA pulled into L2 before the grid dependency wait
    unsigned long long batch;  // score_batch_kernel: sequences (tiles is per sequence)
    ThresholdPush push;        // score_batch_kernel on rank 0 of a peer group
};

__device__ __forceinline__ int tile_view(const TmaParams& p, unsigned long long tile) {
    int v = 0;
#pragma unroll 1
    while (v + 1 < p.nviews && tile >= p.view_tile0[v + 1]) ++v;
    return v;
}

// G = KV heads per cache row (8 for a whole cache, fewer for a KV-head shard);
// a tile is T = 256 / G tokens x G KV heads, so every stage stays 32 KB.
// Consumer warp w scores KV head w % G for tokens [32 (w / G), +32) of the
// tile; its four output rows are the query heads 4 (w % G) + g.
template <int G>
__global__ void __launch_bounds__(kTThreads, 2) score_tma_kernel(const __grid_constant__ TmaParams p) {
    constexpr int T = 256 / G;
    const unsigned seq = blockIdx.y;
    const int y0 = (int)(seq * p.seq_tokens);  // first token row of this sequence in the view
    // Before waiting for the preceding grid (under programmatic dependent
    // launch, the previous layer's selector still running): pull this CTA's
    // first key tiles into L2, so the DRAM stream overlaps that kernel's
    // tail.  Only an L2 hint, never a stale read: the shared-memory loads
    // below are all issued after the wait.
    if (threadIdx.x == kTConsumerWarps * 32) {
        unsigned long long tile = blockIdx.x;
        for (int n = 0; n < p.prefetch_tiles && tile < p.tiles; ++n, tile += gridDim.x) {
            const int v = tile_view(p, tile);
            const int t0 = (int)((tile - p.view_tile0[v]) * T);
            tma_prefetch_3d(&p.maps[v], 0, y0 + t0, 0);
            tma_prefetch_3d(&p.maps[v], kTHalf, y0 + t0, 0);
        }
    }
    extern __shared__ unsigned char smem_raw[];
    // The 128-byte swizzle pattern repeats every 1024 bytes of shared address:
    // align by offsetting the shared array itself (keeps the pointers in the
    // shared address space, so accesses stay shared-memory loads).
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    unsigned char* stages = smem;
    // Q as F16 [kv][c][4 heads]: one 16-byte load gives channels c, c+1.
    uint4* qs = reinterpret_cast<uint4*>(smem + kTStages * kTStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTStages * kTStageBytes + kTQBytes);
    uint64_t* empty = full + kTStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint16_t* qg = p.q + seq * p.q_seq;
    uint16_t* out = p.out + seq * p.out_seq;
    uint16_t* okeys = p.keys ? p.keys + seq * p.out_seq : nullptr;
    ScoreExtras extras = p.extras;
    if (extras.h0) extras.h0 += (size_t)seq * kH0Partials;
    __shared__ unsigned int h0_max, h0_bad, h0_done;
    if (threadIdx.x == 0) {
        h0_max = 0;
        h0_bad = 0;
        h0_done = 0;
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kTConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();  // the ring's barriers are initialised (no global access yet)
    pdl_wait();
    pdl_trigger();
    constexpr int kConsumerThreads = kTConsumerWarps * 32;

    // The producer starts the ring at once; the consumers stage Q meanwhile
    // (in the decode step measured 1-2 % faster per step than staging Q
    // first: the first tiles are L2 hits from the prefetch above).
    if (warp == kTConsumerWarps) {
        if (lane != 0) return;
        // ---------------- producer: two half-channel TMA loads per tile
        uint32_t it = 0;
        bool ok = true;
        for (unsigned long long tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            const int v = tile_view(p, tile);
            const int t0 = (int)((tile - p.view_tile0[v]) * T);
            for (int half = 0; half < 2; ++half, ++it) {
                const uint32_t s = it % kTStages;
                if (it >= kTStages && !mbar_wait(&empty[s], ((it / kTStages) - 1) & 1)) {
                    raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], kTStageBytes);
                tma_load_3d(stages + s * kTStageBytes, &p.maps[v], half * kTHalf, y0 + t0, 0, &full[s]);
            }
        }
        if (!ok) {  // let copies in flight land before shared memory is released
            const uint32_t first = it > kTStages ? it - kTStages : 0;
            for (uint32_t j = first; j < it; ++j) (void)mbar_wait(&full[j % kTStages], (j / kTStages) & 1);
        }
        return;
    }

    // ---------------- consumers: clear the extras, stage Q, then consume
    clear_extras(extras, kConsumerThreads);
    {  // every load issued before any store (one round trip)
        constexpr int kPer = G * kGroup * kDim / kConsumerThreads;
        uint16_t qv[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) qv[u] = qg[threadIdx.x + u * kConsumerThreads];  // coherent: the preceding grid may write Q
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = threadIdx.x + u * kConsumerThreads, h = i >> 7, c = i & 127;
            reinterpret_cast<uint16_t*>(qs)[((h >> 2) * kDim + c) * kGroup + (h & 3)] = qv[u];
        }
    }
    named_sync(1, kConsumerThreads);
    const int kh = warp % G, tl = (warp / G) * 32 + lane;  // KV head, token in tile
    const uint4* qv = qs + kh * (kDim / 2);
    uint32_t it = 0, h0max = 0, h0bad = 0;
    for (unsigned long long tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
        const int v = tile_view(p, tile);
        const unsigned long long t0 = (tile - p.view_tile0[v]) * T;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (int half = 0; half < 2; ++half, ++it) {
            const uint32_t s = it % kTStages;
            if (!mbar_wait(&full[s], (it / kTStages) & 1)) {
                raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                return;
            }
            const unsigned char* row = stages + s * kTStageBytes + (kh * T + tl) * 128;
            const uint4* qh = qv + half * (kTHalf / 2);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint4 w = *reinterpret_cast<const uint4*>(row + ((j ^ (tl & 7)) << 4));
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const uint4 qq = qh[j * 4 + (e >> 1)];  // channels c, c+1: 4 heads each
                    const uint32_t k0 = words[e >> 1] & 0xffffu, k1 = words[e >> 1] >> 16;
                    // Exact F16 products => one rounding per step, as the reference.
                    a0 = fma_f16(qq.x & 0xffffu, k0, a0);
                    a1 = fma_f16(qq.x >> 16, k0, a1);
                    a2 = fma_f16(qq.y & 0xffffu, k0, a2);
                    a3 = fma_f16(qq.y >> 16, k0, a3);
                    a0 = fma_f16(qq.z & 0xffffu, k1, a0);
                    a1 = fma_f16(qq.z >> 16, k1, a1);
                    a2 = fma_f16(qq.w & 0xffffu, k1, a2);
                    a3 = fma_f16(qq.w >> 16, k1, a3);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if ((unsigned long long)tl < p.view_tokens[v] - t0) {
            const unsigned long long col = p.view_col[v] + t0 + tl;
            const float acc[4] = {a0, a1, a2, a3};
#pragma unroll
            for (int g = 0; g < kGroup; ++g) {
                const uint16_t sc = half_bits(acc[g]);
                const unsigned long long at = (unsigned long long)(kh * kGroup + g) * p.out_stride + col;
                out[at] = sc;
                if (okeys) {
                    const uint32_t key = order_key(scale_half(sc));
                    okeys[at] = (uint16_t)key;
                    if (kh == 0 && g == 0) track_head0(key, h0max, h0bad);
                }
            }
        }
    }
    if (extras.h0) {
        if (G == kKvHeads) {
            if (kh == 0) write_head0(extras, h0max, h0bad);
        } else if (kh == 0) {  // 8 / G warps hold KV head 0: the last one to finish writes
            const uint32_t m = __reduce_max_sync(0xffffffffu, h0max);
            const uint32_t b = __reduce_or_sync(0xffffffffu, h0bad);
            if (lane == 0) {
                atomicMax(&h0_max, m);
                atomicOr(&h0_bad, b);
                if (atomicAdd(&h0_done, 1u) == (unsigned)(kTConsumerWarps / G) - 1)
                    extras.h0[blockIdx.x] = (atomicOr(&h0_bad, 0u) << 16) | atomicMax(&h0_max, 0u);
            }
        }
    }
}

// ---------------------------------------------------------- batched shards
// The scorer over a batch of sequences of a KV-head shard: one wave of at
// most two CTAs per SM, CTA c taking the contiguous run of global tiles
// [c T / grid, (c + 1) T / grid) of the T = batch x tiles (sequence-major)
// tiles, so every CTA has the same work within one tile and no second wave
// trails the first.  A run crosses sequence boundaries: at each crossing the
// consumers restage Q and close the head-0 partial of the sequence they
// leave.  Head-0 partials: CTA c writes slot c - first(s) of sequence s,
// first(s) being the CTA that holds the sequence's first tile, and first(s)
// also zeroes the slots past the sequence's CTA count.
__device__ __forceinline__ unsigned long long flat_cta_of(unsigned long long t, unsigned long long total,
                                                          unsigned long long grid) {
    // the CTA whose run [floor(c total / grid), floor((c+1) total / grid)) holds tile t
    return ((t + 1) * grid + total - 1) / total - 1;
}

// The threshold push of rank 0's shard scorer, run by the consumer threads
// of the CTA that finishes last (every head-0 partial is written by then):
// thread t folds sequences t, t + threads, ... -- their ncta partials, loads
// issued together -- into {threshold key, status} records stored into every
// rank's mailbox; then one system-scope fence, the counter reset, and the
// threshold flag (the step's epoch) released on every rank.  Done once at
// the end rather than as each sequence closes, the push never stalls a CTA
// that still has tiles to score.
__device__ void push_thresholds(const ThresholdPush& x, unsigned long long batch, unsigned long long tiles,
                                unsigned long long total, unsigned long long grid, const uint32_t* h0_all,
                                int tid, int threads) {
    for (unsigned long long s = tid; s < batch; s += threads) {
        const unsigned long long first = flat_cta_of(s * tiles, total, grid);
        const unsigned long long last = flat_cta_of(s * tiles + tiles - 1, total, grid);
        const unsigned ncta = (unsigned)(last - first + 1);
        const uint32_t* h0 = h0_all + s * kH0Partials;
        uint32_t mx = 0, bad = 0;
        constexpr int kBatchLoads = 8;
        for (unsigned i0 = 0; i0 < ncta; i0 += kBatchLoads) {
            uint32_t v[kBatchLoads];
#pragma unroll
            for (int j = 0; j < kBatchLoads; ++j) v[j] = i0 + j < ncta ? __ldcg(h0 + i0 + j) : 0u;
#pragma unroll
            for (int j = 0; j < kBatchLoads; ++j) {
                mx = max(mx, v[j] & 0xffffu);
                bad |= v[j] >> 16;
            }
        }
        const uint2 rec = threshold_record(mx, bad, x.alpha);
        for (int w = 0; w < x.world; ++w) *reinterpret_cast<uint2*>(x.mb[w] + x.thr_off + 8 * s) = rec;
    }
}

template <int G>
__global__ void __launch_bounds__(kTThreads, 2) score_batch_kernel(const __grid_constant__ TmaParams p) {
    constexpr int T = 256 / G;
    const unsigned long long total = p.tiles * p.batch, grid = gridDim.x;
    const unsigned long long g0 = blockIdx.x * total / grid, g1 = (blockIdx.x + 1) * total / grid;
    if (threadIdx.x == kTConsumerWarps * 32 && g0 < g1) {  // the first tile into L2 before the dependency wait
        const int y = (int)((g0 / p.tiles) * p.seq_tokens + (g0 % p.tiles) * T);
        tma_prefetch_3d(&p.maps[0], 0, y, 0);
        tma_prefetch_3d(&p.maps[0], kTHalf, y, 0);
    }
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    unsigned char* stages = smem;
    uint4* qs = reinterpret_cast<uint4*>(smem + kTStages * kTStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTStages * kTStageBytes + kTQBytes);
    uint64_t* empty = full + kTStages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ unsigned int h0_max, h0_bad;
    if (threadIdx.x == 0) {
        h0_max = 0;
        h0_bad = 0;
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kTConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    constexpr int kConsumerThreads = kTConsumerWarps * 32;

    if (warp == kTConsumerWarps) {
        if (lane != 0) return;
        uint32_t it = 0;
        bool ok = true;
        for (unsigned long long g = g0; g < g1 && ok; ++g) {
            const int y = (int)((g / p.tiles) * p.seq_tokens + (g % p.tiles) * T);
            for (int half = 0; half < 2; ++half, ++it) {
                const uint32_t s = it % kTStages;
                if (it >= kTStages && !mbar_wait(&empty[s], ((it / kTStages) - 1) & 1)) {
                    raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], kTStageBytes);
                tma_load_3d(stages + s * kTStageBytes, &p.maps[0], half * kTHalf, y, 0, &full[s]);
            }
        }
        if (!ok) {
            const uint32_t first = it > kTStages ? it - kTStages : 0;
            for (uint32_t j = first; j < it; ++j) (void)mbar_wait(&full[j % kTStages], (j / kTStages) & 1);
        }
        return;
    }

    const int kh = warp % G, tl = (warp / G) * 32 + lane;
    const uint4* qv = qs + kh * (kDim / 2);
    uint32_t it = 0, h0max = 0, h0bad = 0;
    unsigned long long seq = ~0ull;
    // A consumer warp whose wait gave up stops consuming but still meets the
    // consumers' named barriers, so no warp is left waiting at one.
    bool aborted = false;
    // Closes sequence s on this CTA: its head-0 partial (slot blockIdx.x -
    // first(s)), and the zero slots when this CTA holds s's first tile.
    auto close_seq = [&](unsigned long long s) {
        if (!p.extras.h0) return;
        if (kh == 0) {
            const uint32_t m = __reduce_max_sync(0xffffffffu, h0max);
            const uint32_t b = __reduce_or_sync(0xffffffffu, h0bad);
            if (lane == 0) {
                atomicMax(&h0_max, m);
                atomicOr(&h0_bad, b);
            }
        }
        h0max = 0;
        h0bad = 0;
        named_sync(1, kConsumerThreads);
        uint32_t* h0 = p.extras.h0 + s * kH0Partials;
        const unsigned long long first = flat_cta_of(s * p.tiles, total, grid);
        const unsigned long long last = flat_cta_of(s * p.tiles + p.tiles - 1, total, grid);
        if (threadIdx.x == 0) {
            h0[blockIdx.x - first] = (h0_bad << 16) | h0_max;
            h0_max = 0;
            h0_bad = 0;
        }
        if (blockIdx.x == first)
            for (unsigned w = (unsigned)(last - first + 1) + threadIdx.x; w < kH0Partials; w += kConsumerThreads)
                h0[w] = 0u;
    };
    for (unsigned long long g = g0; g < g1; ++g) {
        const unsigned long long s_now = g / p.tiles, t0 = (g % p.tiles) * T;
        if (s_now != seq) {
            if (seq != ~0ull) close_seq(seq);
            named_sync(1, kConsumerThreads);  // every consumer is done with the previous Q
            constexpr int kPer = G * kGroup * kDim / kConsumerThreads;
            const uint16_t* qg = p.q + s_now * p.q_seq;
            uint16_t qv16[kPer];
#pragma unroll
            for (int u = 0; u < kPer; ++u) qv16[u] = qg[threadIdx.x + u * kConsumerThreads];
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int i = threadIdx.x + u * kConsumerThreads, h = i >> 7, c = i & 127;
                reinterpret_cast<uint16_t*>(qs)[((h >> 2) * kDim + c) * kGroup + (h & 3)] = qv16[u];
            }
            named_sync(1, kConsumerThreads);
            seq = s_now;
        }
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        if (aborted) continue;  // keeps meeting the named barriers at sequence crossings
        for (int half = 0; half < 2; ++half, ++it) {
            const uint32_t s = it % kTStages;
            if (!mbar_wait(&full[s], (it / kTStages) & 1)) {
                raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                aborted = true;
                break;
            }
            const unsigned char* row = stages + s * kTStageBytes + (kh * T + tl) * 128;
            const uint4* qh = qv + half * (kTHalf / 2);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint4 w = *reinterpret_cast<const uint4*>(row + ((j ^ (tl & 7)) << 4));
                const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const uint4 qq = qh[j * 4 + (e >> 1)];
                    const uint32_t k0 = words[e >> 1] & 0xffffu, k1 = words[e >> 1] >> 16;
                    a0 = fma_f16(qq.x & 0xffffu, k0, a0);
                    a1 = fma_f16(qq.x >> 16, k0, a1);
                    a2 = fma_f16(qq.y & 0xffffu, k0, a2);
                    a3 = fma_f16(qq.y >> 16, k0, a3);
                    a0 = fma_f16(qq.z & 0xffffu, k1, a0);
                    a1 = fma_f16(qq.z >> 16, k1, a1);
                    a2 = fma_f16(qq.w & 0xffffu, k1, a2);
                    a3 = fma_f16(qq.w >> 16, k1, a3);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!aborted && (unsigned long long)tl < p.seq_tokens - t0) {
            const unsigned long long col = seq * p.out_seq + t0 + tl;
            const float acc[4] = {a0, a1, a2, a3};
#pragma unroll
            for (int gq = 0; gq < kGroup; ++gq) {
                const uint16_t sc = half_bits(acc[gq]);
                const unsigned long long at = (unsigned long long)(kh * kGroup + gq) * p.out_stride + col;
                p.out[at] = sc;
                const uint32_t key = order_key(scale_half(sc));
                p.keys[at] = (uint16_t)key;
                if (kh == 0 && gq == 0) track_head0(key, h0max, h0bad);
            }
        }
    }
    if (seq != ~0ull) close_seq(seq);
    if (p.push.world) {
        // Rank 0 of a peer group: the CTA that finishes last pushes every
        // sequence's threshold record (its partials are all written now).
        __shared__ int last_cta;
        named_sync(1, kConsumerThreads);
        if (threadIdx.x == 0) {
            __threadfence();
            last_cta = atomicAdd(p.push.cta_done, 1u) + 1 == (unsigned)grid;
        }
        named_sync(1, kConsumerThreads);
        if (!last_cta) return;
        __threadfence();
        push_thresholds(p.push, p.batch, p.tiles, total, grid, p.extras.h0, threadIdx.x, kConsumerThreads);
        __shared__ unsigned long long push_epoch;
        named_sync(1, kConsumerThreads);
        if (threadIdx.x == 0) {
            __threadfence_system();
            *p.push.cta_done = 0;
            push_epoch = __ldcg(p.push.epoch) + 1;
        }
        named_sync(1, kConsumerThreads);
        // One release per rank, from as many threads at once: a single thread
        // looping over the ranks would pay one system-scope fence per rank.
        if (threadIdx.x < (unsigned)p.push.world)
            st_release_sys(reinterpret_cast<unsigned long long*>(p.push.mb[threadIdx.x] + p.push.flag_off),
                           push_epoch);
    }
}

// Token-major keys of one view seen as a 3-D tensor {channel, token, KV head}
// (strides: token = stride_words words, KV head = 128 words), so that a box
// lands in shared memory as [KV head][token][channels].
bool encode_view(CUtensorMap* map, const hsb_key_view& v, int g = kKvHeads) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)v.tokens, (cuuint64_t)g};
    const cuuint64_t strides[2] = {(cuuint64_t)v.stride_words * 2, (cuuint64_t)kDim * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kTHalf, (cuuint32_t)(256 / g), (cuuint32_t)g};
    const cuuint32_t estr[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(v.data), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__global__ void scale_kernel(const uint16_t* __restrict__ raw, unsigned long long count,
                             uint16_t* __restrict__ out) {
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < count;
         i += (unsigned long long)gridDim.x * blockDim.x)
        out[i] = scale_half(raw[i]);
}

}  // namespace

// Resolves cuTensorMapEncodeTiled through the runtime (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

cudaError_t configure_tma_kernels() {
    cudaError_t e = cudaFuncSetAttribute(score_tma_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_tma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_tma_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_tma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_batch_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_batch_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_batch_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(score_batch_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTSmemBytes);
    return e;
}

bool encode_kv_map(CUtensorMap* map, const uint16_t* data, size_t tokens, size_t stride_words) {
    const hsb_key_view v{data, tokens, stride_words};
    return encode_view(map, v);
}

cudaError_t launch_score(const uint16_t* q, const hsb_key_view* views, size_t nviews,
                         uint16_t* out, size_t out_stride, size_t col0, hsb_device_status* status,
                         cudaStream_t stream, uint16_t* keys, const ScoreExtras* extras) {
    const ScoreExtras none{};
    const ScoreExtras& x = extras ? *extras : none;
    const DeviceInfo& dev = device_info();
    static thread_local int configured_device = -1;
    if (configured_device != dev.ordinal) {
        cudaError_t e = cudaFuncSetAttribute(score_v3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBytes);
        if (e == cudaSuccess) e = configure_tma_kernels();
        if (e != cudaSuccess) return e;
        configured_device = dev.ordinal;
    }
    // Tensor-map path (all views encodable); else the row-copy kernel.
    {
        TmaParams t{};
        bool ok = tensor_map_encoder() != nullptr;
        unsigned long long tiles = 0, col = col0;
        for (size_t v = 0; v < nviews && ok; ++v) {
            ok = encode_view(&t.maps[v], views[v]);
            t.view_tokens[v] = views[v].tokens;
            t.view_tile0[v] = tiles;
            t.view_col[v] = col;
            tiles += (views[v].tokens + kTTile - 1) / kTTile;
            col += views[v].tokens;
        }
        if (ok) {
            t.view_tile0[nviews] = tiles;
            t.nviews = (int)nviews;
            t.tiles = tiles;
            t.q = q;
            t.out = out;
            t.keys = keys;
            t.out_stride = out_stride;
            t.status = status;
            t.extras = x;
            t.prefetch_tiles = kTPrefetchTiles;
            // At most two CTAs per SM, every CTA the same number of tiles
            // (1024 tiles at N 32K: 256 CTAs of four rather than 296 of three
            // or four, whose four-tile CTAs finished ~2.5 us after the rest;
            // step 0.8995 -> 0.8962 ms).
            const unsigned long long most = std::min<unsigned long long>(tiles, (unsigned long long)dev.sms * 2);
            const unsigned long long per = (tiles + most - 1) / most;
            const int grid = (int)((tiles + per - 1) / per);
            return launch_dependent(score_tma_kernel<kKvHeads>, dim3(grid), dim3(kTThreads), kTSmemBytes, stream,
                                    false, t);
        }
    }
    ScoreParams p{};
    p.q = q;
    p.nviews = (int)nviews;
    unsigned long long tokens = 0;
    for (size_t v = 0; v < nviews; ++v) {
        p.data[v] = views[v].data;
        p.first[v] = tokens;
        p.stride[v] = views[v].stride_words;
        tokens += views[v].tokens;
    }
    p.first[nviews] = tokens;
    p.tokens = tokens;
    p.out = out;
    p.keys = keys;
    p.out_stride = out_stride;
    p.col0 = col0;
    p.status = status;
    p.extras = x;
    const unsigned long long ntiles = (tokens + kTile - 1) / kTile;
    const int grid = (int)std::min<unsigned long long>(ntiles, (unsigned long long)dev.sms);
    return launch_dependent(score_v3_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, false, p);
}

cudaError_t launch_score_shard(const uint16_t* q, int kv_heads, const uint16_t* keys_cache, size_t tokens,
                               size_t stride_words, uint16_t* out, uint16_t* keys, hsb_device_status* status,
                               const ScoreExtras* extras, cudaStream_t stream, size_t batch,
                               const ThresholdPush* push) {
    const DeviceInfo& dev = device_info();
    static thread_local int configured_device = -1;
    if (configured_device != dev.ordinal) {
        const cudaError_t e = configure_tma_kernels();
        if (e != cudaSuccess) return e;
        configured_device = dev.ordinal;
    }
    TmaParams t{};
    if (batch == 0 || tokens * batch > 0x7fffffffull) return cudaErrorInvalidValue;
    const hsb_key_view view{keys_cache, tokens * batch, stride_words};  // the whole batch as one view
    if (!encode_view(&t.maps[0], view, kv_heads)) return cudaErrorInvalidValue;
    const unsigned long long tile_tokens = 256 / kv_heads;
    t.seq_tokens = tokens;
    t.q_seq = (unsigned long long)kv_heads * kGroup * kDim;
    t.out_seq = (unsigned long long)kv_heads * kGroup * tokens;
    t.view_tokens[0] = tokens;
    t.view_tile0[0] = 0;
    t.view_col[0] = 0;
    t.tiles = (tokens + tile_tokens - 1) / tile_tokens;
    t.view_tile0[1] = t.tiles;
    t.nviews = 1;
    t.q = q;
    t.out = out;
    t.keys = keys;
    t.out_stride = tokens;
    t.status = status;
    if (extras) t.extras = *extras;
    t.prefetch_tiles = kTPrefetchTiles;
    // One wave: at most two CTAs per SM over the batch's tiles, contiguous
    // runs across sequences (score_batch_kernel).
    t.batch = batch;
    if (push) {
        if (!extras || !extras->h0) return cudaErrorInvalidValue;  // the push derives from the head-0 partials
        t.push = *push;
    }
    const unsigned long long total = t.tiles * batch;
    const dim3 grid((unsigned)std::min<unsigned long long>(total, (unsigned long long)dev.sms * 2));
    if (!keys) return cudaErrorInvalidValue;
    switch (kv_heads) {
    case 1: return launch_dependent(score_batch_kernel<1>, grid, dim3(kTThreads), kTSmemBytes, stream, false, t);
    case 2: return launch_dependent(score_batch_kernel<2>, grid, dim3(kTThreads), kTSmemBytes, stream, false, t);
    case 4: return launch_dependent(score_batch_kernel<4>, grid, dim3(kTThreads), kTSmemBytes, stream, false, t);
    case 8: return launch_dependent(score_batch_kernel<8>, grid, dim3(kTThreads), kTSmemBytes, stream, false, t);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_scale(const uint16_t* raw, size_t count, uint16_t* out, cudaStream_t stream) {
    const DeviceInfo& dev = device_info();
    const unsigned long long blocks = std::min<unsigned long long>((count + 255) / 256, (unsigned long long)dev.sms * 8);
    scale_kernel<<<(unsigned)std::max<unsigned long long>(blocks, 1), 256, 0, stream>>>(raw, count, out);
    return cudaGetLastError();
}

}  // namespace hsb
