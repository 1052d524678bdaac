// synth.cu -- seeded synthetic inputs for benchmarks and tests (not part of
// the reference interface).
//
// The generator is defined so that a CPU restatement reproduces it bit for
// bit: every step is an integer hash or an IEEE double operation with one
// rounding (__dadd_rn, __dmul_rn, __ddiv_rn, __dsqrt_rn: never contracted to
// FMA), and the transcendental functions are our own polynomials rather than
// the CUDA math library:
//   - ln x: exponent split, then 2 atanh(s) with s = (m-1)/(m+1), |s| < 0.172,
//     as the odd series 2 s sum_{j<12} s^(2j) / (2j+1);
//   - e^x: Cody-Waite reduction x = k ln2 + r (ln2 in two parts), Taylor
//     series of e^r to r^16 / 16!;
//   - sin / cos of 2 pi x: x reduced to [-1/2, 1/2] turns by rint, folded to
//     [0, 1/8] turn by symmetry, then Taylor series to the 19th / 18th power.
// Sample i of stream `seed`: a = mix64(seed ^ mix64(i)), b = mix64(a),
// u1 = ((a >> 12) + 1/2) 2^-52, u2 = ((b >> 12) + 1/2) 2^-52 (both exact),
// z = sqrt(-2 ln u1) cos(2 pi u2) (Box-Muller), value = z * stddev in double,
// rounded to F32 then to F16 (or BF16) with round-to-nearest-even.
// Key rows: token t is a heavy hitter when mix64(seed * 0x2545f4914f6cdd1d +
// t) < heavy_cut (heavy_cut = heavy_fraction * 2^64, computed on the host),
// its values then multiplied by heavy_scale; with rope, the adjacent channel
// pair (2i, 2i+1) of each KV head is rotated by the angle t * theta^(-i/64),
// i.e. 2 pi * (t * e^(-(i/64) ln theta) / (2 pi)) turns, NORM mode.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dadd_rn(a, -b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }

// ln x for a positive normal double x.
__device__ double det_log(double x) {
    const unsigned long long bits = (unsigned long long)__double_as_longlong(x);
    int e = (int)((bits >> 52) & 0x7ffull) - 1023;
    double m = __longlong_as_double((long long)((bits & 0x000fffffffffffffull) | 0x3ff0000000000000ull));
    if (m > 0x1.6a09e667f3bcdp+0) {  // sqrt(2): fold to (1/sqrt 2, sqrt 2]
        m = dmul(m, 0.5);
        e += 1;
    }
    const double s = __ddiv_rn(dsub(m, 1.0), dadd(m, 1.0));
    const double z = dmul(s, s);
    // 1 / (2j + 1), j = 11 .. 0
    double t = 0x1.642c8590b2164p-5;
    t = dadd(dmul(t, z), 0x1.8618618618618p-5);
    t = dadd(dmul(t, z), 0x1.af286bca1af28p-5);
    t = dadd(dmul(t, z), 0x1.e1e1e1e1e1e1ep-5);
    t = dadd(dmul(t, z), 0x1.1111111111111p-4);
    t = dadd(dmul(t, z), 0x1.3b13b13b13b14p-4);
    t = dadd(dmul(t, z), 0x1.745d1745d1746p-4);
    t = dadd(dmul(t, z), 0x1.c71c71c71c71cp-4);
    t = dadd(dmul(t, z), 0x1.2492492492492p-3);
    t = dadd(dmul(t, z), 0x1.999999999999ap-3);
    t = dadd(dmul(t, z), 0x1.5555555555555p-2);
    t = dadd(dmul(t, z), 1.0);
    const double lnm = dmul(dadd(s, s), t);
    return dadd(dmul((double)e, 0x1.62e42fefa39efp-1), lnm);
}

// e^x for -700 < x <= 0.
__device__ double det_exp(double x) {
    const double k = rint(dmul(x, 0x1.71547652b82fep+0));  // x / ln2
    const double r = dsub(dsub(x, dmul(k, 0x1.62e42feep-1)), dmul(k, 0x1.a39ef35793c76p-33));
    // 1 / n!, n = 16 .. 1
    double p = 0x1.ae7f3e733b81fp-45;
    p = dadd(dmul(p, r), 0x1.ae7f3e733b81fp-41);
    p = dadd(dmul(p, r), 0x1.93974a8c07c9dp-37);
    p = dadd(dmul(p, r), 0x1.6124613a86d09p-33);
    p = dadd(dmul(p, r), 0x1.1eed8eff8d898p-29);
    p = dadd(dmul(p, r), 0x1.ae64567f544e4p-26);
    p = dadd(dmul(p, r), 0x1.27e4fb7789f5cp-22);
    p = dadd(dmul(p, r), 0x1.71de3a556c734p-19);
    p = dadd(dmul(p, r), 0x1.a01a01a01a01ap-16);
    p = dadd(dmul(p, r), 0x1.a01a01a01a01ap-13);
    p = dadd(dmul(p, r), 0x1.6c16c16c16c17p-10);
    p = dadd(dmul(p, r), 0x1.1111111111111p-7);
    p = dadd(dmul(p, r), 0x1.5555555555555p-5);
    p = dadd(dmul(p, r), 0x1.5555555555555p-3);
    p = dadd(dmul(p, r), 0.5);
    p = dadd(dmul(p, r), 1.0);
    p = dadd(dmul(p, r), 1.0);
    const double two_k = __longlong_as_double((long long)((unsigned long long)((int)k + 1023) << 52));
    return dmul(p, two_k);
}

// sin and cos of 2 pi x.
__device__ void det_sincos_turns(double x, double* sn, double* cs) {
    const double y = dsub(x, rint(x));  // [-1/2, 1/2]
    const bool neg = y < 0.0;
    double a = neg ? -y : y;             // sin(2 pi y) odd, cos even
    bool flip_cos = false, swap = false;
    if (a > 0.25) {
        a = dsub(0.5, a);                // sin(pi - t) = sin t, cos(pi - t) = -cos t
        flip_cos = true;
    }
    if (a > 0.125) {
        a = dsub(0.25, a);               // sin(pi/2 - t) = cos t
        swap = true;
    }
    const double t = dmul(a, 0x1.921fb54442d18p+2);  // radians, [0, pi/4]
    const double z = dmul(t, t);
    // sin t = t (1 - z/3! + z^2/5! - ... - z^9/19!)
    double ps = -0x1.2f49b46814157p-57;
    ps = dadd(dmul(ps, z), 0x1.952c77030ad4ap-49);
    ps = dadd(dmul(ps, z), -0x1.ae7f3e733b81fp-41);
    ps = dadd(dmul(ps, z), 0x1.6124613a86d09p-33);
    ps = dadd(dmul(ps, z), -0x1.ae64567f544e4p-26);
    ps = dadd(dmul(ps, z), 0x1.71de3a556c734p-19);
    ps = dadd(dmul(ps, z), -0x1.a01a01a01a01ap-13);
    ps = dadd(dmul(ps, z), 0x1.1111111111111p-7);
    ps = dadd(dmul(ps, z), -0x1.5555555555555p-3);
    ps = dadd(dmul(ps, z), 1.0);
    const double s = dmul(t, ps);
    // cos t = 1 - z/2! + z^2/4! - ... + z^9/18! (alternating, last term negative)
    double pc = -0x1.6827863b97d97p-53;
    pc = dadd(dmul(pc, z), 0x1.ae7f3e733b81fp-45);
    pc = dadd(dmul(pc, z), -0x1.93974a8c07c9dp-37);
    pc = dadd(dmul(pc, z), 0x1.1eed8eff8d898p-29);
    pc = dadd(dmul(pc, z), -0x1.27e4fb7789f5cp-22);
    pc = dadd(dmul(pc, z), 0x1.a01a01a01a01ap-16);
    pc = dadd(dmul(pc, z), -0x1.6c16c16c16c17p-10);
    pc = dadd(dmul(pc, z), 0x1.5555555555555p-5);
    pc = dadd(dmul(pc, z), -0.5);
    pc = dadd(dmul(pc, z), 1.0);
    double s2 = swap ? pc : s, c2 = swap ? s : pc;
    if (flip_cos) c2 = -c2;
    if (neg) s2 = -s2;
    *sn = s2;
    *cs = c2;
}

// One N(0,1) sample per (seed, index).
__device__ __forceinline__ double normal_sample(unsigned long long seed, unsigned long long i) {
    const unsigned long long a = mix64(seed ^ mix64(i));
    const unsigned long long b = mix64(a);
    const double u1 = dmul(dadd((double)(a >> 12), 0.5), 0x1p-52);
    const double u2 = dmul(dadd((double)(b >> 12), 0.5), 0x1p-52);
    double s, c;
    det_sincos_turns(u2, &s, &c);
    return dmul(__dsqrt_rn(dmul(-2.0, det_log(u1))), c);
}

__device__ __forceinline__ uint16_t round16(double v, int bf16) {
    const float f = __double2float_rn(v);
    return bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(f)) : half_bits(f);
}

__global__ void synth_normal_kernel(uint16_t* out, unsigned long long count, unsigned long long seed,
                                    double stddev, int bf16) {
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < count;
         i += (unsigned long long)gridDim.x * blockDim.x)
        out[i] = round16(dmul(normal_sample(seed, i), stddev), bf16);
}

// rows: [tokens][1024 words used] at stride_words; one thread per channel pair.
__global__ void synth_keys_kernel(uint16_t* rows, unsigned long long tokens, unsigned long long stride,
                                  unsigned long long seed, unsigned long long heavy_cut, double heavy_scale,
                                  int rope, double theta) {
    const unsigned long long pairs = tokens * 512ull;
    const double ln_theta = rope ? det_log(theta) : 0.0;
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < pairs;
         i += (unsigned long long)gridDim.x * blockDim.x) {
        const unsigned long long t = i / 512, c2 = (i % 512) * 2;  // c2 = kv_head*128 + even channel
        const double scale = mix64(seed * 0x2545f4914f6cdd1dull + t) < heavy_cut ? heavy_scale : 1.0;
        double a = dmul(normal_sample(seed, t * 1024 + c2), scale);
        double b = dmul(normal_sample(seed, t * 1024 + c2 + 1), scale);
        if (rope) {
            const double pair = (double)((c2 & 127) >> 1);
            const double inv_freq = det_exp(dmul(-dmul(pair, 0x1p-6), ln_theta));
            const double turns = dmul(dmul((double)t, inv_freq), 0x1.45f306dc9c883p-3);  // / (2 pi)
            double s, c;
            det_sincos_turns(turns, &s, &c);
            const double ra = dsub(dmul(a, c), dmul(b, s));
            const double rb = dadd(dmul(a, s), dmul(b, c));
            a = ra;
            b = rb;
        }
        uint16_t* row = rows + t * stride;
        row[c2] = round16(a, 0);
        row[c2 + 1] = round16(b, 0);
    }
}

int grid_for(unsigned long long n) {
    const DeviceInfo& dev = device_info();
    return (int)std::max<unsigned long long>(
        1, std::min<unsigned long long>((n + 255) / 256, (unsigned long long)dev.sms * 16));
}

}  // namespace

uint64_t synth_heavy_cut(float heavy_fraction) {
    if (!(heavy_fraction > 0.0f)) return 0;
    if (heavy_fraction >= 1.0f) return ~0ull;
    return (uint64_t)((double)heavy_fraction * 18446744073709551616.0);
}

cudaError_t launch_synth_normal(uint16_t* out, size_t count, uint64_t seed, float stddev, int bf16,
                                cudaStream_t stream) {
    synth_normal_kernel<<<grid_for(count), 256, 0, stream>>>(out, count, seed, (double)stddev, bf16);
    return cudaGetLastError();
}

cudaError_t launch_synth_keys(uint16_t* rows, size_t tokens, size_t stride_words, uint64_t seed,
                              float heavy_fraction, float heavy_scale, int rope, float theta,
                              cudaStream_t stream) {
    synth_keys_kernel<<<grid_for(tokens * 512ull), 256, 0, stream>>>(
        rows, tokens, stride_words, seed, synth_heavy_cut(heavy_fraction), (double)heavy_scale, rope, (double)theta);
    return cudaGetLastError();
}

}  // namespace hsb
