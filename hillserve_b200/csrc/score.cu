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
// Memory.  The scorer streams K once (2 KB per token) and is HBM-bound.  One
// persistent CTA per SM: a producer warp moves whole 2 KB token rows into
// shared memory with 1-D bulk copies (the TMA engine), three stages deep; the
// eight consumer warps each own one KV head and read their 256-byte slice of
// 32 rows.  Rows are stored at a 2064-byte pitch so that eight consecutive
// lanes' 16-byte reads fall in distinct bank groups.  Q lives in shared memory
// as FP32, laid out [kv head][channel][4 heads] so each channel's four
// query values are one broadcast 16-byte load.
#include <algorithm>
#include <cstdio>

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
};

__device__ __forceinline__ const uint16_t* token_row(const ScoreParams& p, unsigned long long t) {
    int v = 0;
#pragma unroll 1
    while (v + 1 < p.nviews && t >= p.first[v + 1]) ++v;
    return p.data[v] + (t - p.first[v]) * p.stride[v];
}

__global__ void __launch_bounds__(kThreads, 1) score_v3_kernel(const __grid_constant__ ScoreParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    float* qs = reinterpret_cast<float*>(smem);
    unsigned char* tiles = smem + kQBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(tiles + kStages * kStageBytes);
    uint64_t* empty = full + kStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    uint32_t it = 0;
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
                kk[0] = (uint16_t)order_key(scale_half(s0));
                kk[p.out_stride] = (uint16_t)order_key(scale_half(s1));
                kk[2 * p.out_stride] = (uint16_t)order_key(scale_half(s2));
                kk[3 * p.out_stride] = (uint16_t)order_key(scale_half(s3));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

__global__ void scale_kernel(const uint16_t* __restrict__ raw, unsigned long long count,
                             uint16_t* __restrict__ out) {
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < count;
         i += (unsigned long long)gridDim.x * blockDim.x)
        out[i] = scale_half(raw[i]);
}

}  // namespace

cudaError_t launch_score(const uint16_t* q, const hsb_key_view* views, size_t nviews,
                         uint16_t* out, size_t out_stride, size_t col0, hsb_device_status* status,
                         cudaStream_t stream, uint16_t* keys) {
    const DeviceInfo& dev = device_info();
    static thread_local int configured_device = -1;
    if (configured_device != dev.ordinal) {
        cudaError_t e = cudaFuncSetAttribute(score_v3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBytes);
        if (e != cudaSuccess) return e;
        configured_device = dev.ordinal;
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
    const unsigned long long ntiles = (tokens + kTile - 1) / kTile;
    const int grid = (int)std::min<unsigned long long>(ntiles, (unsigned long long)dev.sms);
    score_v3_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_scale(const uint16_t* raw, size_t count, uint16_t* out, cudaStream_t stream) {
    const DeviceInfo& dev = device_info();
    const unsigned long long blocks = std::min<unsigned long long>((count + 255) / 256, (unsigned long long)dev.sms * 8);
    scale_kernel<<<(unsigned)std::max<unsigned long long>(blocks, 1), 256, 0, stream>>>(raw, count, out);
    return cudaGetLastError();
}

}  // namespace hsb
