// rehearsal.cu -- the rehearsal query producer (patches/llama-b6000-round2.patch
// :303-317, early-rehearsal.patch:19-47): q = RoPE_pos(W x) for the next
// layer, emitted as F32 and as the F16 query the scorer consumes
// (policy/full_gqa_runtime.cpp:61-64 casts with half_bits).
//
// A memory-bound bf16 GEMV (W is 32 MiB): each warp produces one adjacent
// output pair (2i, 2i+1) of a head -- the pair NORM-mode RoPE rotates
// together -- streaming both W rows with 16-byte loads and reducing in FP32.
// The rotation angle position * theta^(-2i/128) and its sine/cosine are
// evaluated in FP64 so that large positions keep full accuracy.
//
// Also: seeded synthetic inputs for benchmarks (counter-based hash +
// Box-Muller), which are not part of the reference path.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kEmbed = 4096;
constexpr int kRThreads = 256;  // 8 warps, 8 output pairs per CTA

__device__ __forceinline__ float bf16_value(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__global__ void __launch_bounds__(kRThreads) rehearsal_kernel(const uint16_t* __restrict__ x,
                                                              const uint16_t* __restrict__ w,
                                                              unsigned long long position, float theta,
                                                              float* __restrict__ q32,
                                                              uint16_t* __restrict__ q16) {
    __shared__ __align__(16) float xs[kEmbed];
    for (int i = threadIdx.x; i < kEmbed; i += kRThreads) xs[i] = bf16_value(x[i]);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = blockIdx.x * 8 + warp;  // 0..2047
    const int r0 = pair * 2;
    const uint4* w0 = reinterpret_cast<const uint4*>(w + (size_t)r0 * kEmbed);
    const uint4* w1 = reinterpret_cast<const uint4*>(w + (size_t)(r0 + 1) * kEmbed);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
    for (int c = 0; c < kEmbed / 256; ++c) {
        const int idx = c * 32 + lane;  // 16-byte piece: elements idx*8 .. idx*8+7
        const uint4 u = w0[idx], v = w1[idx];
        const float4 xa = reinterpret_cast<const float4*>(xs)[idx * 2];
        const float4 xb = reinterpret_cast<const float4*>(xs)[idx * 2 + 1];
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const uint32_t uw[4] = {u.x, u.y, u.z, u.w}, vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            a0 = fmaf(bf16_value(uw[j] & 0xffffu), xv[2 * j], a0);
            a0 = fmaf(bf16_value(uw[j] >> 16), xv[2 * j + 1], a0);
            a1 = fmaf(bf16_value(vw[j] & 0xffffu), xv[2 * j], a1);
            a1 = fmaf(bf16_value(vw[j] >> 16), xv[2 * j + 1], a1);
        }
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    if (lane == 0) {
        const int i = (r0 & (kDim - 1)) >> 1;  // pair index inside the head
        const double angle = (double)position * pow((double)theta, -2.0 * (double)i / (double)kDim);
        double s, c;
        sincos(angle, &s, &c);
        const float cs = (float)c, sn = (float)s;
        const float o0 = a0 * cs - a1 * sn;
        const float o1 = a0 * sn + a1 * cs;
        if (q32) {
            q32[r0] = o0;
            q32[r0 + 1] = o1;
        }
        if (q16) {
            q16[r0] = half_bits(o0);
            q16[r0 + 1] = half_bits(o1);
        }
    }
}

// ---------------------------------------------------------------- synthetic
__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
// One N(0,1) sample per (seed, index): Box-Muller on two 24-bit uniforms.
__device__ __forceinline__ float normal_sample(unsigned long long seed, unsigned long long i) {
    const unsigned long long u = mix64(seed ^ mix64(i));
    const float u1 = ((float)(u >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = ((float)((u >> 16) & 0xffffffull) + 0.5f) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void synth_normal_kernel(uint16_t* out, unsigned long long count, unsigned long long seed,
                                    float stddev, int bf16) {
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < count;
         i += (unsigned long long)gridDim.x * blockDim.x) {
        const float v = normal_sample(seed, i) * stddev;
        out[i] = bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : half_bits(v);
    }
}

// rows: [tokens][1024 words used] at stride_words; one thread per channel pair.
__global__ void synth_keys_kernel(uint16_t* rows, unsigned long long tokens, unsigned long long stride,
                                  unsigned long long seed, float heavy_fraction, float heavy_scale, int rope,
                                  float theta) {
    const unsigned long long pairs = tokens * 512ull;
    const unsigned long long heavy_cut = (unsigned long long)((double)heavy_fraction * 18446744073709551616.0);
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < pairs;
         i += (unsigned long long)gridDim.x * blockDim.x) {
        const unsigned long long t = i / 512, c2 = (i % 512) * 2;  // c2 = kv_head*128 + even channel
        const float scale = (heavy_fraction > 0.f && mix64(seed * 0x2545f4914f6cdd1dull + t) < heavy_cut)
                                ? heavy_scale : 1.0f;
        float a = normal_sample(seed, t * 1024 + c2) * scale;
        float b = normal_sample(seed, t * 1024 + c2 + 1) * scale;
        if (rope) {
            const int ii = (int)((c2 & 127) >> 1);
            const float inv = powf(theta, -2.0f * (float)ii / 128.0f);
            float s, c;
            sincosf((float)t * inv, &s, &c);
            const float ra = a * c - b * s, rb = a * s + b * c;
            a = ra;
            b = rb;
        }
        uint16_t* row = rows + t * stride;
        row[c2] = half_bits(a);
        row[c2 + 1] = half_bits(b);
    }
}

int grid_for(unsigned long long n) {
    const DeviceInfo& dev = device_info();
    return (int)std::max<unsigned long long>(1, std::min<unsigned long long>((n + 255) / 256, (unsigned long long)dev.sms * 16));
}

}  // namespace

cudaError_t launch_rehearsal(const uint16_t* x, const uint16_t* w, uint64_t position, float theta, float* q32,
                             uint16_t* q16, cudaStream_t stream) {
    rehearsal_kernel<<<kHeads * kDim / 16, kRThreads, 0, stream>>>(x, w, position, theta, q32, q16);
    return cudaGetLastError();
}

cudaError_t launch_synth_normal(uint16_t* out, size_t count, uint64_t seed, float stddev, int bf16,
                                cudaStream_t stream) {
    synth_normal_kernel<<<grid_for(count), 256, 0, stream>>>(out, count, seed, stddev, bf16);
    return cudaGetLastError();
}

cudaError_t launch_synth_keys(uint16_t* rows, size_t tokens, size_t stride_words, uint64_t seed,
                              float heavy_fraction, float heavy_scale, int rope, float theta,
                              cudaStream_t stream) {
    synth_keys_kernel<<<grid_for(tokens * 512ull), 256, 0, stream>>>(rows, tokens, stride_words, seed,
                                                                      heavy_fraction, heavy_scale, rope, theta);
    return cudaGetLastError();
}

}  // namespace hsb
