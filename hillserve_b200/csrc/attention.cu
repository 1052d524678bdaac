// attention.cu -- stage 4: flash-decode attention.
//
// attention_packed_kernel: the ggml graph of runtime/gqa_delivery.cpp:19-20
// (scores = K.q at F32, softmax(scores/sqrt(128) + mask), out = V.p) over the
// packed layout K [slot][32][128], V [32][128][slot].  Split-K: a CTA owns
// (query head, 256 slots), writes (max, sum, partial output) and the last CTA
// of a head folds the partials.  Decode has one query per head and the four
// heads of a KV group select different slots, so there is no dense
// contraction to give the tensor cores; the kernel is a bandwidth-bound
// GEMV pair on the CUDA cores.
//
// attention_dense_tma_kernel: dense decode attention over a token-major
// cache (the two dense layers).  Every query head reads every row, so the
// four heads of a KV group share one contraction per tile: the kernel streams
// K/V through TMA and runs logits and P.V on the tensor cores (below).
//
// attention_dense_kernel: the fallback when no tensor map can be encoded: a
// CTA owns (KV head, 512 tokens) and serves the four query heads of the group
// from one read of each K and V row on the CUDA cores.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kSplit = 256;
constexpr int kPThreads = 128;
constexpr int kPart = kDim + 2;  // floats per partial: max, sum, out[128]

struct PackedParams {
    const float* q;
    const uint16_t* k;
    const uint16_t* v;
    size_t count;
    const float* mask;
    size_t qpad;
    const uint32_t* sizes;
    size_t sizes_stride;
    float* out;
    float* part;        // [32][nsplit][kPart]
    unsigned* arrive;   // [32], zeroed before launch
    int nsplit;
    float scale;
};

__device__ __forceinline__ float block_reduce_max128(float v, float* red) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    const float r = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    return r;
}
__device__ __forceinline__ float block_reduce_sum128(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    const float r = (red[0] + red[1]) + (red[2] + red[3]);
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kPThreads) attention_packed_kernel(const __grid_constant__ PackedParams p) {
    __shared__ float sc[kSplit];
    __shared__ float red[4];
    __shared__ int last;
    const int h = blockIdx.y, j = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    size_t n = p.count;
    int live = p.nsplit;
    if (!p.mask) {
        n = std::min<size_t>(p.sizes[(size_t)h * p.sizes_stride], p.count);
        live = (int)((n + kSplit - 1) / kSplit);
        if (n == 0) {
            if (j == 0) p.out[h * kDim + tid] = 0.0f;
            return;
        }
    }
    if (j >= live) return;
    const size_t s0 = (size_t)j * kSplit, s1 = std::min(n, s0 + kSplit);
    const int m = (int)(s1 - s0);

    const float4 q4 = reinterpret_cast<const float4*>(p.q + h * kDim)[lane];
    // Scores: each warp takes 4 slots per round (loads issued together).
    for (int base = warp; base < m; base += 16) {
        uint2 raw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int s = base + 4 * u;
            raw[u] = s < m ? *reinterpret_cast<const uint2*>(p.k + ((s0 + s) * kHeads + h) * kDim + lane * 4)
                           : make_uint2(0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int s = base + 4 * u;
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw[u].x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw[u].y));
            float dot = a.x * q4.x + a.y * q4.y + b.x * q4.z + b.y * q4.w;
            dot = warp_sum(dot);
            if (lane == 0 && s < m) {
                float x = dot * p.scale;
                if (p.mask) x += p.mask[(size_t)h * p.qpad * p.count + s0 + s];
                sc[s] = x;
            }
        }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int s = tid; s < m; s += kPThreads) mx = fmaxf(mx, sc[s]);
    mx = block_reduce_max128(mx, red);
    float l = 0.0f;
    for (int s = tid; s < m; s += kPThreads) {
        const float e = mx == -INFINITY ? 0.0f : expf(sc[s] - mx);
        sc[s] = e;
        l += e;
    }
    l = block_reduce_sum128(l, red);
    // out[d] partial: thread d walks its V row over the split's slots.
    const uint16_t* vrow = p.v + ((size_t)h * kDim + tid) * p.count + s0;
    float acc = 0.0f;
    int s = 0;
    if ((p.count & 7) == 0) {  // rows 16-byte aligned: 8 slots per load, 4 loads in flight
        for (; s + 32 <= m; s += 32) {
            uint4 w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) w[u] = *reinterpret_cast<const uint4*>(vrow + s + 8 * u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t x[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&x[e]));
                    acc = fmaf(sc[s + 8 * u + 2 * e], f.x, acc);
                    acc = fmaf(sc[s + 8 * u + 2 * e + 1], f.y, acc);
                }
            }
        }
    }
    for (; s < m; ++s) acc = fmaf(sc[s], half_value(vrow[s]), acc);
    if (live == 1) {  // one split: no partials to fold
        p.out[h * kDim + tid] = l > 0.0f ? acc / l : 0.0f;
        return;
    }
    float* part = p.part + ((size_t)h * p.nsplit + j) * kPart;
    if (tid == 0) {
        part[0] = mx;
        part[1] = l;
    }
    part[2 + tid] = acc;
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&p.arrive[h], 1u) == (unsigned)(live - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float* base = p.part + (size_t)h * p.nsplit * kPart;
    float M = -INFINITY;
    for (int i = 0; i < live; ++i) M = fmaxf(M, __ldcg(base + i * kPart));
    float L = 0.0f, o = 0.0f;
    if (M != -INFINITY) {
        for (int i = 0; i < live; ++i) {
            const float mi = __ldcg(base + i * kPart);
            if (mi == -INFINITY) continue;
            const float w = expf(mi - M);
            L = fmaf(__ldcg(base + i * kPart + 1), w, L);
            o = fmaf(__ldcg(base + i * kPart + 2 + tid), w, o);
        }
    }
    p.out[h * kDim + tid] = L > 0.0f ? o / L : 0.0f;
}

// ------------------------------------------------------------------ dense
constexpr int kDTokens = 512;
constexpr int kDThreads = 256;

struct DenseParams {
    const float* q;
    const uint16_t* kc;
    const uint16_t* vc;
    size_t tokens, stride;
    float* out;
    float* part;       // [32][nsplit][kPart]
    unsigned* arrive;  // [8]
    int nsplit;
    float scale;
};

__global__ void __launch_bounds__(kDThreads) attention_dense_kernel(const __grid_constant__ DenseParams p) {
    __shared__ float4 qs[kDim];         // [c] -> 4 heads of the group
    __shared__ float sc[kGroup][kDTokens];
    __shared__ float red[8][kGroup];
    __shared__ float stat[2][kGroup];   // max, sum
    __shared__ float accs[4][kGroup][kDim];
    __shared__ int last;
    const int kh = blockIdx.y, j = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < kDim * kGroup; i += kDThreads) {
        const int c = i >> 2, g = i & 3;
        reinterpret_cast<float*>(qs)[i] = p.q[(kh * kGroup + g) * kDim + c];
    }
    __syncthreads();
    const size_t t0 = (size_t)j * kDTokens;
    const int m = (int)std::min<size_t>(kDTokens, p.tokens - t0);
    // Scores: two tokens per thread, four heads per token.
    for (int t = tid; t < m; t += kDThreads) {
        const uint4* row = reinterpret_cast<const uint4*>(p.kc + (t0 + t) * p.stride + kh * kDim);
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
        for (int c8 = 0; c8 < 16; ++c8) {
            const uint4 w = row[c8];
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const float2 kv = __half22float2(*reinterpret_cast<const __half2*>(&words[jj]));
                const float4 qa = qs[c8 * 8 + 2 * jj], qb = qs[c8 * 8 + 2 * jj + 1];
                a0 = fmaf(qa.x, kv.x, a0); a1 = fmaf(qa.y, kv.x, a1);
                a2 = fmaf(qa.z, kv.x, a2); a3 = fmaf(qa.w, kv.x, a3);
                a0 = fmaf(qb.x, kv.y, a0); a1 = fmaf(qb.y, kv.y, a1);
                a2 = fmaf(qb.z, kv.y, a2); a3 = fmaf(qb.w, kv.y, a3);
            }
        }
        sc[0][t] = a0 * p.scale; sc[1][t] = a1 * p.scale;
        sc[2][t] = a2 * p.scale; sc[3][t] = a3 * p.scale;
    }
    __syncthreads();
    // Max and exp-sum per head.
    float mx[kGroup];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        float v = -INFINITY;
        for (int t = tid; t < m; t += kDThreads) v = fmaxf(v, sc[g][t]);
        mx[g] = warp_max(v);
        if (lane == 0) red[warp][g] = mx[g];
    }
    __syncthreads();
    if (tid < kGroup) {
        float v = -INFINITY;
        for (int w = 0; w < 8; ++w) v = fmaxf(v, red[w][tid]);
        stat[0][tid] = v;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        const float M = stat[0][g];
        float s = 0.f;
        for (int t = tid; t < m; t += kDThreads) {
            const float e = expf(sc[g][t] - M);
            sc[g][t] = e;
            s += e;
        }
        s = warp_sum(s);
        if (lane == 0) red[warp][g] = s;
    }
    __syncthreads();
    if (tid < kGroup) {
        float v = 0.f;
        for (int w = 0; w < 8; ++w) v += red[w][tid];
        stat[1][tid] = v;
    }
    // Partial outputs: thread = (channel pair, quarter of the tokens).
    const int dp = tid & 63, quarter = tid >> 6;
    float o[kGroup][2] = {};
    const int per = (m + 3) / 4;
    const int tb = quarter * per, te = std::min(m, tb + per);
    for (int t = tb; t < te; ++t) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(p.vc + (t0 + t) * p.stride + kh * kDim + 2 * dp);
        const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&w));
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
            const float pg = sc[g][t];
            o[g][0] = fmaf(pg, v2.x, o[g][0]);
            o[g][1] = fmaf(pg, v2.y, o[g][1]);
        }
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        accs[quarter][g][2 * dp] = o[g][0];
        accs[quarter][g][2 * dp + 1] = o[g][1];
    }
    __syncthreads();
    for (int i = tid; i < kGroup * kDim; i += kDThreads) {
        const int g = i >> 7, d = i & 127;
        const float v = (accs[0][g][d] + accs[1][g][d]) + (accs[2][g][d] + accs[3][g][d]);
        float* part = p.part + ((size_t)(kh * kGroup + g) * p.nsplit + j) * kPart;
        part[2 + d] = v;
        if (d == 0) {
            part[0] = stat[0][g];
            part[1] = stat[1][g];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&p.arrive[kh], 1u) == (unsigned)(p.nsplit - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = tid; i < kGroup * kDim; i += kDThreads) {
        const int g = i >> 7, d = i & 127;
        const float* base = p.part + (size_t)(kh * kGroup + g) * p.nsplit * kPart;
        float M = -INFINITY;
        for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, __ldcg(base + s * kPart));
        float L = 0.f, acc = 0.f;
        for (int s = 0; s < p.nsplit; ++s) {
            const float w = expf(__ldcg(base + s * kPart) - M);
            L = fmaf(__ldcg(base + s * kPart + 1), w, L);
            acc = fmaf(__ldcg(base + s * kPart + 2 + d), w, acc);
        }
        p.out[(kh * kGroup + g) * kDim + d] = acc / L;
    }
}

// ------------------------------------------------------------- dense (TMA)
// Dense decode attention streamed like the scorer: a ring of 32 KB TMA boxes
// ({64 channels, 32 tokens, 8 KV heads}, 128-byte swizzle) carries, per
// 32-token tile, K channels 0-63, K 64-127, V 0-63, V 64-127.  Warp w is KV
// head w and runs both contractions of its four query heads on the tensor
// cores with mma.sync.m16n8k16 (F16 operands, F32 accumulate):
//
//   logits  S^T[token][col] = K[token][ch] . Qx^T[ch][col]
//   output  O^T[ch][col]    = V^T[ch][token] . Px^T[token][col]
//
// Decode has four query heads per KV head, so the MMA's eight columns carry
// each head twice: column h holds the F16 rounding of head h's F32 value
// (x_hi = f16(x)) and column h + 4 its remainder (x_lo = f16(x - x_hi)).
// Summing the two columns gives products of the F32 value to ~2^-22
// relative, near FP32, at no extra MMA cost.  Q is first scaled by a power
// of two per KV head (max |q| in [2^14, 2^15)) so that neither half
// overflows or leaves the F16 normal range; the logit scale undoes it
// exactly.  K and V are F16 already and enter unchanged (ldmatrix from the
// swizzled boxes, .trans for V^T).  An online softmax per query head keeps
// (max, sum); the tile's weights go through a per-warp shared array into the
// B fragments of the P.V product.  One CTA per SM walks tiles blockIdx.x,
// +gridDim.x, ... and writes one (max, sum, out[128]) partial per query
// head; dense_combine_kernel folds them.
constexpr int kDTBox = 32 * kKvHeads * 64 * 2;  // bytes per box
constexpr int kDTSlots = 6;
constexpr int kDTConsumers = kKvHeads;
constexpr int kDTThreads = (kDTConsumers + 1) * 32;
constexpr int kDTPStride = 40;  // halves per weight row (32 tokens + pad: conflict-free B-fragment loads)
constexpr int kDTPBytes = kDTConsumers * 8 * kDTPStride * 2;  // per warp: [8 columns][kDTPStride] F16
constexpr int kDTSmem = 1024 + kDTSlots * kDTBox + kDTPBytes + 2 * kDTSlots * 8;
constexpr int kDenseMaxCtas = 256;

struct DenseTmaParams {
    CUtensorMap kmap, vmap;
    const float* q;
    unsigned tokens, tiles;
    float* part;  // [32][gridDim.x][kPart]
    hsb_device_status* status;
    float scale;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// D += A . B, m16n8k16, A row-major F16, B column-major F16, D F32.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// The F16 half of x that column `lo` of a hi/lo pair carries.
__device__ __forceinline__ __half split_half(float x, bool lo) {
    const __half hi = __float2half_rn(x);
    return lo ? __float2half_rn(x - __half2float(hi)) : hi;
}
__device__ __forceinline__ uint32_t pack_halves(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

__global__ void __launch_bounds__(kDTThreads, 1) attention_dense_tma_kernel(const __grid_constant__ DenseTmaParams p) {
    if (threadIdx.x == kDTConsumers * 32) {
        // The ring's first fill (tile blockIdx.x, then the K boxes of the
        // next) into L2 before the dependency wait: the history rows are not
        // the preceding grid's output, and L2 is the point of coherence for
        // any row it does write.
        for (unsigned j = 0, tile = blockIdx.x; j < 2 && tile < p.tiles; ++j, tile += gridDim.x)
            for (int box = 0; box < (j ? 2 : 4); ++box)
                tma_prefetch_3d(box < 2 ? &p.kmap : &p.vmap, (box & 1) * 64, (int)(tile * 32), 0);
    }
    pdl_wait();
    pdl_trigger();
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    unsigned char* slots = smem;
    __half* pw = reinterpret_cast<__half*>(smem + kDTSlots * kDTBox);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDTSlots * kDTBox + kDTPBytes);
    uint64_t* empty = full + kDTSlots;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kDTSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kDTConsumers);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kDTConsumers) {
        if (lane != 0) return;
        // ---------------- producer: four boxes per tile
        uint32_t it = 0;
        bool ok = true;
        for (unsigned tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            for (int box = 0; box < 4; ++box, ++it) {
                const uint32_t s = it % kDTSlots;
                if (it >= kDTSlots && !mbar_wait(&empty[s], ((it / kDTSlots) - 1) & 1)) {
                    raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], kDTBox);
                tma_load_3d(slots + s * kDTBox, box < 2 ? &p.kmap : &p.vmap, (box & 1) * 64, (int)(tile * 32), 0,
                            &full[s]);
            }
        }
        if (!ok) {  // let copies in flight land before shared memory is released
            const uint32_t first = it > kDTSlots ? it - kDTSlots : 0;
            for (uint32_t j = first; j < it; ++j) (void)mbar_wait(&full[j % kDTSlots], (j / kDTSlots) & 1);
        }
        return;
    }

    // ---------------- consumers: warp kh = KV head kh, query heads 4kh .. 4kh+3
    const int kh = warp;
    const int g = lane >> 2, t = lane & 3;  // MMA fragment row group and thread-in-group
    // Q^T B fragments (column g = head g & 3, half g >> 2) for the 8 channel
    // steps, every load issued first (the preceding grid wrote Q: coherent).
    float2 qv[8][2];
    {
        const float* qh = p.q + (size_t)(kh * kGroup + (g & 3)) * kDim + 2 * t;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qv[ks][0] = make_float2(qh[16 * ks], qh[16 * ks + 1]);  // q needs only 4-byte alignment
            qv[ks][1] = make_float2(qh[16 * ks + 8], qh[16 * ks + 9]);
        }
    }
    float qmax = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
        qmax = fmaxf(qmax, fmaxf(fmaxf(fabsf(qv[ks][0].x), fabsf(qv[ks][0].y)),
                                 fmaxf(fabsf(qv[ks][1].x), fabsf(qv[ks][1].y))));
    qmax = warp_max(qmax);
    // 2^e with max |q| 2^e in [2^14, 2^15); e = 0 for a zero, subnormal or non-finite maximum.
    const int qexp = (int)((__float_as_uint(qmax) >> 23) & 0xffu);
    const int e = (qexp == 0 || qexp == 0xff) ? 0 : max(-100, min(100, 141 - qexp));
    const float up = __uint_as_float((uint32_t)(127 + e) << 23);
    const float sw = p.scale * __uint_as_float((uint32_t)(127 - e) << 23);  // the logit scale, 2^e undone
    const bool lo_col = g >= 4;
    uint32_t bq[8][2];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
#pragma unroll
        for (int j = 0; j < 2; ++j)
            bq[ks][j] = pack_halves(split_half(qv[ks][j].x * up, lo_col), split_half(qv[ks][j].y * up, lo_col));

    // Lane state: heads h0 = 2 (t & 1) and h0 + 1 -- the same two heads for
    // the logits it holds and for its output columns (2t, 2t + 1 mod 4).
    float M[2] = {-INFINITY, -INFINITY}, L[2] = {0.0f, 0.0f};
    float o[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.0f;
    __half* pwarp = pw + kh * 8 * kDTPStride;
    const bool lo_half = t >= 2;
    const int h0 = 2 * (t & 1);
    // ldmatrix row addresses: lane i serves matrix i >> 3, row i & 7.
    const int mi = lane >> 3, mr = lane & 7;
    uint32_t it = 0;
    for (unsigned tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
        float acc[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;
        for (int half = 0; half < 2; ++half, ++it) {
            const uint32_t s = it % kDTSlots;
            if (!mbar_wait(&full[s], (it / kDTSlots) & 1)) {
                raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                return;
            }
            const uint32_t base = smem_addr(slots + s * kDTBox + kh * 32 * 128);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    // A = K rows: matrices {tokens +0/+8} x {channels +0/+8}
                    const int tok = mt * 16 + mr + ((mi & 1) << 3);
                    const int chunk = 2 * kk + (mi >> 1);
                    uint32_t a[4];
                    ldsm_x4(base + tok * 128 + ((chunk ^ (tok & 7)) << 4), a);
                    mma_f16(acc[mt], a, bq[half * 4 + kk][0], bq[half * 4 + kk][1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // Logits of heads h0, h0 + 1 for tokens g, g + 8, 16 + g, 24 + g: the
        // hi column plus the lo column (lane t ^ 2), then the scale.
        float sc[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float x = acc[mt][r] + __shfl_xor_sync(0xffffffffu, acc[mt][r], 2);
                const int tok = mt * 16 + g + ((r >> 1) << 3);
                sc[mt][r] = tile * 32 + tok < p.tokens ? x * sw : -INFINITY;
            }
        float fg[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {  // head h0 + j: registers r = j, j + 2
            float mx = fmaxf(fmaxf(sc[0][j], sc[0][j + 2]), fmaxf(sc[1][j], sc[1][j + 2]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(M[j], mx);  // finite: the tile has a valid token
            fg[j] = expf(M[j] - mn);           // 0 on the first tile
            float sum = 0.0f;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int r = j; r < 4; r += 2) {
                    const float pr = expf(sc[mt][r] - mn);  // 0 for a masked token
                    sum += pr;
                    const int tok = mt * 16 + g + ((r >> 1) << 3);
                    pwarp[(h0 + j + (lo_half ? 4 : 0)) * kDTPStride + tok] = split_half(pr, lo_half);
                }
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            L[j] = fmaf(L[j], fg[j], sum);
            M[j] = mn;
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            o[m][0] *= fg[0];
            o[m][1] *= fg[1];
            o[m][2] *= fg[0];
            o[m][3] *= fg[1];
        }
        __syncwarp();
        // P^T B fragments: column g, tokens 16 kt + 2t (+1) and + 8.
        uint32_t bp[2][2];
#pragma unroll
        for (int kt = 0; kt < 2; ++kt) {
            const uint32_t* row = reinterpret_cast<const uint32_t*>(pwarp + g * kDTPStride + kt * 16);
            bp[kt][0] = row[t];
            bp[kt][1] = row[4 + t];
        }
        for (int half = 0; half < 2; ++half, ++it) {
            const uint32_t s = it % kDTSlots;
            if (!mbar_wait(&full[s], (it / kDTSlots) & 1)) {
                raise_status(p.status, HSB_E_TIMEOUT, blockIdx.x);
                return;
            }
            const uint32_t base = smem_addr(slots + s * kDTBox + kh * 32 * 128);
#pragma unroll
            for (int kt = 0; kt < 2; ++kt) {
#pragma unroll
                for (int mc = 0; mc < 4; ++mc) {
                    // A = V^T: matrices {channels +0/+8} x {tokens +0/+8}, transposed on load
                    const int tok = kt * 16 + mr + ((mi >> 1) << 3);
                    const int chunk = 2 * mc + (mi & 1);
                    uint32_t a[4];
                    ldsm_x4_trans(base + tok * 128 + ((chunk ^ (tok & 7)) << 4), a);
                    mma_f16(o[half * 4 + mc], a, bp[kt][0], bp[kt][1]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        __syncwarp();  // the weights are read before the next tile overwrites them
    }
    // O^T: lane holds channels 16m + g (+8) of columns 2t, 2t + 1; hi + lo.
#pragma unroll
    for (int m = 0; m < 8; ++m)
#pragma unroll
        for (int r = 0; r < 4; ++r) o[m][r] += __shfl_xor_sync(0xffffffffu, o[m][r], 2);
    if (t < 2) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float* part = p.part + ((size_t)(kh * kGroup + h0 + j) * gridDim.x + blockIdx.x) * kPart;
            if (g == 0) {
                part[0] = M[j];
                part[1] = L[j];
            }
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                part[2 + 16 * m + g] = o[m][j];
                part[2 + 16 * m + g + 8] = o[m][j + 2];
            }
        }
    }
}

// out[h][d] = sum_c exp(M_c - M) o_c[d] / sum_c exp(M_c - M) L_c over the
// dense kernel's per-CTA partials.  One CTA per query head: the partials'
// weights go to shared memory once, then 4 groups of 128 threads (thread =
// channel) each sum every 4th partial.  Loads are issued in batches of 20
// before any arithmetic (a loop of dependent loads cost ~4 us per dense
// layer).  512 threads at <= 56 registers fit beside a resident dense CTA
// (288 threads, 120 registers, ~200 KB shared memory), so the programmatic
// launch makes the combine's CTAs resident while the dense kernel still runs
// and they start the moment it completes.
constexpr int kCombineGroups = 4;
constexpr int kCombineBatch = 20;
__global__ void __maxnreg__(56) dense_combine_kernel(const float* __restrict__ part, int nparts,
                                                     float* __restrict__ out) {
    constexpr int kPer = kDenseMaxCtas / kCombineGroups;  // partials per thread, at most
    constexpr int kPerLane = kDenseMaxCtas / 32;          // partials per lane of warp 0
    pdl_wait();
    pdl_trigger();
    __shared__ float w[kDenseMaxCtas];
    __shared__ float acc_s[kCombineGroups][kDim];
    __shared__ float red[2];
    const int h = blockIdx.x, tid = threadIdx.x, d = tid & (kDim - 1), grp = tid / kDim;
    const float* base = part + (size_t)h * nparts * kPart;
    // The first batch of this thread's output channel (partials grp, grp + 4,
    // ...) and, for warp 0, the maxima and sums are all in flight at once.
    float ov[kCombineBatch];
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i) {
        const int c = grp + i * kCombineGroups;
        ov[i] = c < nparts ? __ldcg(base + (size_t)c * kPart + 2 + d) : 0.0f;
    }
    if (tid < 32) {
        float mv[kPerLane], lv[kPerLane];
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int c = tid + 32 * i;
            mv[i] = c < nparts ? __ldcg(base + (size_t)c * kPart) : -INFINITY;
            lv[i] = c < nparts ? __ldcg(base + (size_t)c * kPart + 1) : 0.0f;
        }
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) m = fmaxf(m, mv[i]);
        m = warp_max(m);
        float l = 0.0f;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int c = tid + 32 * i;
            if (c < nparts) {
                const float wc = expf(mv[i] - m);
                w[c] = wc;
                l = fmaf(lv[i], wc, l);
            }
        }
        l = warp_sum(l);
        if (tid == 0) red[0] = l;
    }
    __syncthreads();
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i) {
        const int c = grp + i * kCombineGroups;
        if (c < nparts) acc = fmaf(ov[i], w[c], acc);
    }
    for (int b = kCombineBatch; b < kPer && grp + b * kCombineGroups < nparts; b += kCombineBatch) {
#pragma unroll
        for (int i = 0; i < kCombineBatch; ++i) {
            const int c = grp + (b + i) * kCombineGroups;
            ov[i] = c < nparts ? __ldcg(base + (size_t)c * kPart + 2 + d) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kCombineBatch; ++i) {
            const int c = grp + (b + i) * kCombineGroups;
            if (c < nparts) acc = fmaf(ov[i], w[c], acc);
        }
    }
    acc_s[grp][d] = acc;
    __syncthreads();
    if (tid < kDim) {
        float o = 0.0f;
#pragma unroll
        for (int g = 0; g < kCombineGroups; ++g) o += acc_s[g][d];
        out[h * kDim + d] = red[0] > 0.0f ? o / red[0] : 0.0f;
    }
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

size_t attention_workspace_bytes(size_t count) {
    const size_t nsplit = std::max<size_t>(1, (count + kSplit - 1) / kSplit);
    return align256(kHeads * sizeof(unsigned)) + align256(kHeads * nsplit * kPart * sizeof(float));
}

cudaError_t launch_attention_packed(const float* q, const uint16_t* k, const uint16_t* v, size_t count,
                                    const float* mask, size_t qpad, const uint32_t* sizes,
                                    size_t sizes_stride, float* out, void* workspace, cudaStream_t stream) {
    PackedParams p{};
    p.q = q;
    p.k = k;
    p.v = v;
    p.count = count;
    p.mask = mask;
    p.qpad = qpad;
    p.sizes = sizes;
    p.sizes_stride = sizes_stride;
    p.out = out;
    p.nsplit = (int)std::max<size_t>(1, (count + kSplit - 1) / kSplit);
    p.arrive = static_cast<unsigned*>(workspace);
    p.part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + align256(kHeads * sizeof(unsigned)));
    p.scale = 1.0f / sqrtf(128.0f);
    cudaError_t e = cudaMemsetAsync(p.arrive, 0, kHeads * sizeof(unsigned), stream);
    if (e != cudaSuccess) return e;
    attention_packed_kernel<<<dim3(p.nsplit, kHeads), kPThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

size_t attention_dense_workspace_bytes(size_t tokens) {
    const size_t nsplit = std::max<size_t>(1, (tokens + kDTokens - 1) / kDTokens);
    const size_t legacy = align256(kKvHeads * sizeof(unsigned)) + align256(kHeads * nsplit * kPart * sizeof(float));
    const size_t ctas = std::min<size_t>(kDenseMaxCtas, std::max<size_t>(1, (tokens + 31) / 32));
    return std::max(legacy, align256(kHeads * ctas * kPart * sizeof(float)));
}

cudaError_t launch_attention_dense(const float* q, const uint16_t* kcache, const uint16_t* vcache, size_t tokens,
                                   size_t stride_words, float* out, void* workspace, cudaStream_t stream) {
    // TMA path: one CTA per SM streaming K/V tiles, then a combine kernel.
    {
        DenseTmaParams t{};
        if (tokens <= 0x7fffffffull && encode_kv_map(&t.kmap, kcache, tokens, stride_words) &&
            encode_kv_map(&t.vmap, vcache, tokens, stride_words)) {
            const DeviceInfo& dev = device_info();
            static thread_local int configured_device = -1;
            if (configured_device != dev.ordinal) {
                cudaError_t e = cudaFuncSetAttribute(attention_dense_tma_kernel,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kDTSmem);
                if (e != cudaSuccess) return e;
                configured_device = dev.ordinal;
            }
            t.q = q;
            t.tokens = (unsigned)tokens;
            t.tiles = (unsigned)((tokens + 31) / 32);
            t.part = static_cast<float*>(workspace);
            t.status = nullptr;
            t.scale = 1.0f / sqrtf(128.0f);
            const unsigned grid = std::min<unsigned>({t.tiles, (unsigned)dev.sms, (unsigned)kDenseMaxCtas});
            cudaError_t e = launch_dependent(attention_dense_tma_kernel, dim3(grid), dim3(kDTThreads), kDTSmem,
                                             stream, false, t);
            if (e != cudaSuccess) return e;
            return launch_dependent(dense_combine_kernel, dim3(kHeads), dim3(kDim * kCombineGroups), 0, stream,
                                    false, static_cast<const float*>(t.part), (int)grid, out);
        }
    }
    DenseParams p{};
    p.q = q;
    p.kc = kcache;
    p.vc = vcache;
    p.tokens = tokens;
    p.stride = stride_words;
    p.out = out;
    p.nsplit = (int)((tokens + kDTokens - 1) / kDTokens);
    p.arrive = static_cast<unsigned*>(workspace);
    p.part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + align256(kKvHeads * sizeof(unsigned)));
    p.scale = 1.0f / sqrtf(128.0f);
    cudaError_t e = cudaMemsetAsync(p.arrive, 0, kKvHeads * sizeof(unsigned), stream);
    if (e != cudaSuccess) return e;
    attention_dense_kernel<<<dim3(p.nsplit, kKvHeads), kDThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

// ------------------------------------------------------------ gather + attention
// The layer step's last stage in one kernel: for each (query head, 32-slot
// tile) of the selection it reads the selected K/V rows once from the HBM
// cache, writes them to the packed workspace (K [slot][32][128] straight from
// registers, V [32][128][slot] transposed through shared memory; live slots
// only, as hsb_gather_cache with zero_padding 0), and from the same data forms
// the tile's softmax partial (max, sum, P.V).  The last tile of a head to
// finish folds the head's partials.  Work items (tile-major, head-minor) are
// spread over a fixed grid, so a small selection occupies few CTAs.
namespace {
constexpr int kGAThreads = 128;  // thread t: slot t / 4 of the tile, channel quarter t % 4
constexpr int kGAPitch = kDim + 8;  // V tile row pitch in halves (16-byte aligned rows)

struct GatherAttnParams {
    const float* q;         // F32 [32][128]
    const uint32_t* ids;    // [32][kstride], per-head order (key desc, id asc)
    size_t kstride;
    const uint32_t* size;   // the selection's k (same for every head)
    const uint16_t* kcache;
    const uint16_t* vcache;
    size_t stride_words, visible, count;
    uint16_t* kp;           // [count][32][128]
    uint16_t* vp;           // [32][128][count]
    float* out;             // [32][128]
    float* part;            // [32][tiles_cap][kPart]
    unsigned* arrive;       // [32], zero at launch
    unsigned tiles_cap;
    hsb_device_status* status;
    float scale;
};

__global__ void __launch_bounds__(kGAThreads) gather_attention_kernel(const __grid_constant__ GatherAttnParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) uint16_t vt[32][kGAPitch];
    __shared__ float wgt[32];
    __shared__ float red[4];
    __shared__ int last;
    const int tid = threadIdx.x, slot = tid >> 2, qd = tid & 3;
    uint32_t k = *p.size;
    if (k > p.kstride || k > p.count) {  // cannot come from the selector; keep every access in bounds
        if (blockIdx.x == 0 && tid == 0) raise_status(p.status, HSB_E_INVALID, 0);
        k = 0;
    }
    if (k == 0) {  // empty selection: zero output (the reference throws earlier)
        if (blockIdx.x == 0)
            for (int i = tid; i < kHeads * kDim; i += kGAThreads) p.out[i] = 0.0f;
        return;
    }
    const unsigned ntiles = (k + 31) / 32;
    const unsigned items = ntiles * kHeads;
    const bool vec_v = (p.count & 7) == 0;
    for (unsigned item = blockIdx.x; item < items; item += gridDim.x) {
        const int h = (int)(item % kHeads), kh = h >> 2;
        const unsigned tile = item / kHeads, s0 = tile * 32;
        const int live = (int)min(32u, k - s0);
        // ---- rows of this thread's slot (quarter qd: channels 32*qd .. 32*qd+31)
        uint4 kr[4], vr[4];
        bool ok = slot < live;
        if (ok) {
            const uint32_t id = p.ids[(size_t)h * p.kstride + s0 + slot];
            if (id >= p.visible) {
                raise_status(p.status, HSB_E_PACK_MISSING, h);
                ok = false;
            } else {
                const uint4* ks = reinterpret_cast<const uint4*>(p.kcache + (size_t)id * p.stride_words + kh * kDim) + qd * 4;
                const uint4* vs = reinterpret_cast<const uint4*>(p.vcache + (size_t)id * p.stride_words + kh * kDim) + qd * 4;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    kr[u] = __ldcg(ks + u);
                    vr[u] = __ldcg(vs + u);
                }
            }
        }
        if (!ok) {
#pragma unroll
            for (int u = 0; u < 4; ++u) kr[u] = vr[u] = make_uint4(0, 0, 0, 0);
        }
        if (slot < live) {
            uint4* kd = reinterpret_cast<uint4*>(p.kp + ((size_t)(s0 + slot) * kHeads + h) * kDim) + qd * 4;
#pragma unroll
            for (int u = 0; u < 4; ++u) kd[u] = kr[u];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4*>(&vt[slot][qd * 32 + u * 8]) = vr[u];
        // ---- logit of the slot: four quarter dot products, combined by shuffles
        const float4* qv = reinterpret_cast<const float4*>(p.q + h * kDim + qd * 32);
        float dot = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float4 qa = __ldcg(qv + 2 * u), qb = __ldcg(qv + 2 * u + 1);
            const uint32_t w[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&w[0]));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&w[1]));
            const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&w[2]));
            const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&w[3]));
            dot = fmaf(f0.x, qa.x, dot);
            dot = fmaf(f0.y, qa.y, dot);
            dot = fmaf(f1.x, qa.z, dot);
            dot = fmaf(f1.y, qa.w, dot);
            dot = fmaf(f2.x, qb.x, dot);
            dot = fmaf(f2.y, qb.y, dot);
            dot = fmaf(f3.x, qb.z, dot);
            dot = fmaf(f3.y, qb.w, dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        if (qd == 0) wgt[slot] = slot < live ? dot * p.scale : -INFINITY;
        __syncthreads();
        // ---- tile softmax weights (warp 0), then P.V per channel (thread = channel)
        float mx = -INFINITY;
        if (tid < 32) {
            const float x = wgt[tid];
            mx = warp_max(x);
            const float e = tid < live ? expf(x - mx) : 0.0f;
            wgt[tid] = e;
            const float l = warp_sum(e);
            if (tid == 0) {
                red[0] = mx;
                red[1] = l;
            }
        }
        __syncthreads();
        mx = red[0];
        const float l = red[1];
        const int d = tid;
        float acc = 0.0f;
#pragma unroll 8
        for (int s = 0; s < 32; ++s) acc = fmaf(wgt[s], half_value(vt[s][d]), acc);
        // ---- V packed (transposed): row d of head h, slots s0 .. s0+live-1
        uint16_t* vrow = p.vp + ((size_t)h * kDim + d) * p.count + s0;
        if (live == 32 && vec_v) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    w[e] = (uint32_t)vt[8 * u + 2 * e][d] | ((uint32_t)vt[8 * u + 2 * e + 1][d] << 16);
                reinterpret_cast<uint4*>(vrow)[u] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
            for (int s = 0; s < live; ++s) vrow[s] = vt[s][d];
        }
        if (ntiles == 1) {  // one tile: no partials to fold
            p.out[h * kDim + d] = l > 0.0f ? acc / l : 0.0f;
            __syncthreads();  // vt / wgt are rewritten by the next item
            continue;
        }
        float* part = p.part + ((size_t)h * p.tiles_cap + tile) * kPart;
        if (tid == 0) {
            part[0] = mx;
            part[1] = l;
        }
        part[2 + d] = acc;
        __threadfence();
        __syncthreads();
        if (tid == 0) last = atomicAdd(&p.arrive[h], 1u) == ntiles - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            const float* base = p.part + (size_t)h * p.tiles_cap * kPart;
            float M = -INFINITY;
            for (unsigned i = 0; i < ntiles; ++i) M = fmaxf(M, __ldcg(base + i * kPart));
            float L = 0.0f, o = 0.0f;
            for (unsigned i = 0; i < ntiles; ++i) {
                const float w = expf(__ldcg(base + i * kPart) - M);
                L = fmaf(__ldcg(base + i * kPart + 1), w, L);
                o = fmaf(__ldcg(base + i * kPart + 2 + d), w, o);
            }
            p.out[h * kDim + d] = L > 0.0f ? o / L : 0.0f;
        }
        __syncthreads();
    }
}
}  // namespace

size_t gather_attention_workspace_bytes(size_t count) {
    const size_t tiles = std::max<size_t>(1, (count + 31) / 32);
    return align256(kHeads * sizeof(unsigned)) + align256(kHeads * tiles * kPart * sizeof(float));
}

cudaError_t launch_gather_attention(const float* q, const uint32_t* ids, size_t kstride, const uint32_t* size,
                                    const uint16_t* kcache, const uint16_t* vcache, size_t stride_words,
                                    size_t visible, size_t count, uint16_t* kp, uint16_t* vp, float* out,
                                    void* workspace, int reset_arrive, hsb_device_status* status,
                                    cudaStream_t stream) {
    const DeviceInfo& dev = device_info();
    GatherAttnParams p{};
    p.q = q;
    p.ids = ids;
    p.kstride = kstride;
    p.size = size;
    p.kcache = kcache;
    p.vcache = vcache;
    p.stride_words = stride_words;
    p.visible = visible;
    p.count = count;
    p.kp = kp;
    p.vp = vp;
    p.out = out;
    p.arrive = static_cast<unsigned*>(workspace);
    p.part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + align256(kHeads * sizeof(unsigned)));
    p.tiles_cap = (unsigned)std::max<size_t>(1, (count + 31) / 32);
    p.status = status;
    p.scale = 1.0f / sqrtf(128.0f);
    if (reset_arrive) {
        cudaError_t e = cudaMemsetAsync(p.arrive, 0, kHeads * sizeof(unsigned), stream);
        if (e != cudaSuccess) return e;
    }
    const unsigned items = p.tiles_cap * kHeads;
    const unsigned grid = std::min<unsigned>(items, (unsigned)dev.sms * 8);
    return launch_dependent(gather_attention_kernel, dim3(grid), dim3(kGAThreads), 0, stream, false, p);
}

}  // namespace hsb
