// common.cuh -- device helpers shared by the sm_100a kernels of the
// selected-KV decode path: binary16 conversions with the reference's exact
// semantics, the F16 order key, mbarrier + bulk-copy (TMA) primitives with
// bounded waits, and the device status word.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "hsb.h"

namespace hsb {

constexpr int kHeads = 32;
constexpr int kKvHeads = 8;
constexpr int kDim = 128;
constexpr int kGroup = 4;
constexpr int kRowBytes = 4096;  // one interleaved KV row (K[8][128] | V[8][128])

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// ---------------------------------------------------------------- binary16
// Exact widening (policy/host_policy.cpp:9-14).
__device__ __forceinline__ float half_value(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
// Round to nearest even with the reference's NaN rule: canonical quiet NaN
// keeping the sign (policy/host_policy.cpp:18).  Finite values and overflow
// to infinity follow IEEE RNE, which __float2half_rn implements.
__device__ __forceinline__ uint16_t half_bits(float f) {
    if (f != f) return (uint16_t)(((__float_as_uint(f) >> 16) & 0x8000u) | 0x7e00u);
    return __half_as_ushort(__float2half_rn(f));
}
// policy/half_order.hpp:7-10: numeric order of finite F16 values, -0 == +0.
__device__ __forceinline__ uint32_t order_key(uint32_t bits) {
    if ((bits & 0x7fffu) == 0) bits = 0;
    return (bits & 0x8000u) ? (~bits & 0xffffu) : (bits ^ 0x8000u);
}
// Order keys of NaNs lie above +inf's (0xfc00) or below -inf's (0x03ff).
__device__ __forceinline__ bool key_nan(uint32_t key) { return key > 0xfc00u || key < 0x03ffu; }
__device__ __forceinline__ bool key_nonfinite(uint32_t key) { return key >= 0xfc00u || key <= 0x03ffu; }
// The runtime's normalisation (policy/full_gqa_runtime.cpp:571):
// F16(F32(raw) / sqrtf(128)), an IEEE division.
__device__ __forceinline__ uint16_t scale_half(uint16_t raw) {
    return half_bits(__fdiv_rn(half_value(raw), __fsqrt_rn(128.0f)));
}
__device__ __forceinline__ bool is_finite_half(uint16_t h) { return (h & 0x7c00u) != 0x7c00u; }
// Mixed-precision FMA: F16 x F16 + F32 -> F32 with one rounding.  The F16
// product is exact in F32, so this equals the reference's rounded multiply
// followed by a rounded add (kernels/full_gqa_pipeline/ABI.json:31-37).
__device__ __forceinline__ float fma_f16(uint32_t a16, uint32_t b16, float c) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"((unsigned short)a16), "h"((unsigned short)b16), "f"(c));
    return d;
}

// ---------------------------------------------------------------- status
// Order in which the reference would have met two errors: a payload-table
// error (checked before any head) first, then by index (query head or row),
// then by code (a head's slot-count check precedes its ID checks).
__device__ __forceinline__ unsigned long long status_rank(int code, int index) {
    const unsigned long long major = code == HSB_E_PACK_PHYSICAL ? 0ull : 1ull;
    return (major << 56) | ((unsigned long long)(unsigned)index << 8) | (unsigned)code;
}
// Records an error; when several are raised concurrently the one the
// reference would have thrown first is kept.  The status word is 8-byte
// aligned (code in the low half, index in the high half).
__device__ __forceinline__ void raise_status(hsb_device_status* st, int code, int index) {
    if (st == nullptr) return;
    unsigned long long* word = reinterpret_cast<unsigned long long*>(st);
    const unsigned long long mine = ((unsigned long long)(unsigned)index << 32) | (unsigned)code;
    unsigned long long seen = *reinterpret_cast<volatile unsigned long long*>(word);
    while (true) {
        const int old_code = (int)(seen & 0xffffffffull);
        const int old_index = (int)(seen >> 32);
        if (old_code != 0 && status_rank(old_code, old_index) <= status_rank(code, index)) return;
        const unsigned long long prev = atomicCAS(word, seen, mine);
        if (prev == seen) return;
        seen = prev;
    }
}

// System-scope acquire load / release store of a 64-bit flag (flags that
// other GPUs write or read through peer memory).
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* a) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* a, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
// The threshold record of a sequence from its head-0 maximum key and
// non-finite flag (policy/gqa_policy.cpp:50-54): {order key of
// F16(max - alpha), status}.
__device__ __forceinline__ uint2 threshold_record(uint32_t maxkey, uint32_t bad0, float alpha) {
    const uint16_t kb = (uint16_t)((maxkey & 0x8000u) ? (maxkey ^ 0x8000u) : (~maxkey & 0xffffu));
    const float threshold = half_value(half_bits(maxkey ? half_value(kb) - alpha : -INFINITY));
    uint32_t status = 0;
    if (bad0) status = HSB_E_SEL_NONFINITE_HEAD0;
    else if (!isfinite(threshold)) status = HSB_E_SEL_THRESHOLD;
    return make_uint2(status ? 0u : order_key(half_bits(threshold)), status);
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity to complete; returns false if the
// wait ran past kWaitLimitNs (the caller records HSB_E_TIMEOUT and unwinds).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - start > kWaitLimitNs) return false;
    }
    return true;
}

// 1-D bulk copy global -> shared (the TMA engine), completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while its predecessor in the stream drains;
// pdl_wait() blocks until the predecessor grid has completed and its memory
// is visible, so it comes before the kernel's first global access.
// pdl_trigger() lets this kernel's own dependents start launching.  Both are
// no-ops for an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 3-D tiled TMA load into this CTA's own shared memory,
// completing on the mbarrier `bar`.  x (innermost) must be a multiple of 8
// 16-bit elements.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Prefetch of one 3-D box into L2 (no shared memory, no barrier, nothing to
// wait for).  A hint only: L2 is where every SM's global writes land, so a
// prefetched line never hides a later write to it, and the box may be read
// before pdl_wait() while the preceding grid still runs.  Same coordinate
// rule as tma_load_3d.
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// Named barrier `id` (1..15; 0 is __syncthreads) over `count` threads, a
// multiple of 32: whole warps take part.
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

}  // namespace hsb
