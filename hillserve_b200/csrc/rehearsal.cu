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
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kEmbed = 4096;
constexpr int kRThreads = 128;  // 4 warps, 4 output pairs per CTA: 512 CTAs, ~3.5 per SM

__device__ __forceinline__ float bf16_value(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// A 16-byte load of weights, which nothing writes while the kernel runs.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__global__ void __launch_bounds__(kRThreads) rehearsal_kernel(const uint16_t* __restrict__ x,
                                                              const uint16_t* __restrict__ w,
                                                              unsigned long long position, float theta,
                                                              float* __restrict__ q32,
                                                              uint16_t* __restrict__ q16) {
    __shared__ __align__(16) float xs[kEmbed];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = blockIdx.x * (kRThreads / 32) + warp;  // 0..2047
    const int r0 = pair * 2;
    const uint4* w0 = reinterpret_cast<const uint4*>(w + (size_t)r0 * kEmbed);
    const uint4* w1 = reinterpret_cast<const uint4*>(w + (size_t)(r0 + 1) * kEmbed);
    // The GEMV is a pure 32 MiB stream: each lane issues the 16-byte loads of
    // half its columns of both rows before any arithmetic (16 loads in flight
    // per lane), twice.  The first half is issued before x is staged, so the
    // stream starts at the kernel's first instruction.
    constexpr int kPieces = kEmbed / 256;  // 16-byte pieces per lane per row
    constexpr int kBatch = kPieces / 2;
    uint4 u[kBatch], v[kBatch];
#pragma unroll
    for (int c = 0; c < kBatch; ++c) {  // volatile asm: issued here, in order, before any use
        u[c] = ldg_stream(w0 + c * 32 + lane);
        v[c] = ldg_stream(w1 + c * 32 + lane);
    }
    {  // x in one round trip: every thread's 16-byte loads first, then the stores
        constexpr int kPer = kEmbed / 8 / kRThreads;  // 16-byte pieces per thread
        uint4 xv[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) xv[k] = reinterpret_cast<const uint4*>(x)[threadIdx.x + k * kRThreads];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int e = (threadIdx.x + k * kRThreads) * 8;
            const uint32_t xw[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                xs[e + 2 * j] = bf16_value(xw[j] & 0xffffu);
                xs[e + 2 * j + 1] = bf16_value(xw[j] >> 16);
            }
        }
    }
    // The rotation of this pair depends on no loaded data: lane 0 evaluates
    // it while the loads are in flight.
    float cs = 1.0f, sn = 0.0f;
    if (lane == 0) {
        const int i = (r0 & (kDim - 1)) >> 1;  // pair index inside the head
        const double angle = (double)position * pow((double)theta, -2.0 * (double)i / (double)kDim);
        double sd, cd;
        sincos(angle, &sd, &cd);
        cs = (float)cd;
        sn = (float)sd;
    }
    __syncthreads();
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int c0 = 0; c0 < kPieces; c0 += kBatch) {
        if (c0 > 0) {
#pragma unroll
            for (int c = 0; c < kBatch; ++c) {
                u[c] = ldg_stream(w0 + (c0 + c) * 32 + lane);
                v[c] = ldg_stream(w1 + (c0 + c) * 32 + lane);
            }
        }
        // The arithmetic below reads the loaded words through these (empty,
        // ordered) statements, so it cannot be scheduled between the loads.
#pragma unroll
        for (int c = 0; c < kBatch; ++c)
            asm volatile("" : "+r"(u[c].x), "+r"(u[c].y), "+r"(u[c].z), "+r"(u[c].w), "+r"(v[c].x), "+r"(v[c].y),
                         "+r"(v[c].z), "+r"(v[c].w));
#pragma unroll
        for (int c = 0; c < kBatch; ++c) {
            const int idx = (c0 + c) * 32 + lane;  // 16-byte piece: elements idx*8 .. idx*8+7
            const float4 xa = reinterpret_cast<const float4*>(xs)[idx * 2];
            const float4 xb = reinterpret_cast<const float4*>(xs)[idx * 2 + 1];
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            const uint32_t uw[4] = {u[c].x, u[c].y, u[c].z, u[c].w}, vw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a0 = fmaf(bf16_value(uw[j] & 0xffffu), xv[2 * j], a0);
                a0 = fmaf(bf16_value(uw[j] >> 16), xv[2 * j + 1], a0);
                a1 = fmaf(bf16_value(vw[j] & 0xffffu), xv[2 * j], a1);
                a1 = fmaf(bf16_value(vw[j] >> 16), xv[2 * j + 1], a1);
            }
        }
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    if (lane == 0) {
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

}  // namespace

cudaError_t launch_rehearsal(const uint16_t* x, const uint16_t* w, uint64_t position, float theta, float* q32,
                             uint16_t* q16, cudaStream_t stream) {
    rehearsal_kernel<<<kHeads * kDim / 2 / (kRThreads / 32), kRThreads, 0, stream>>>(x, w, position, theta, q32, q16);
    return cudaGetLastError();
}

}  // namespace hsb
