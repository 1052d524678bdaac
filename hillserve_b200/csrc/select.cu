// select.cu -- stage 2: the gqa_policy selector (policy/gqa_policy.cpp:47-70)
// and the history-only prefetch cover (policy/full_gqa_runtime.cpp:299-344).
//
// One CTA of 1024 threads per query head, launched cooperatively so that all
// heads are resident and can meet at one bounded grid barrier:
//   1. every CTA reduces the head-0 maximum itself (head 0's row is read from
//      L2 by each CTA, which avoids a second barrier) and forms the F16
//      threshold F16(max - alpha);
//   2. each CTA normalises its own row (F16(raw / sqrtf(128)) when the input is
//      raw), stores the 16-bit order keys and counts keys >= threshold;
//   3. grid barrier; every CTA reads the 32 counts, rounds them as the
//      reference does (F16 count, FP32 sum, F16 mean) and derives k -- all
//      CTAs compute the same k and the same first error;
//   4. radix select on the order key (two 8-bit histogram passes) finds the
//      k-th key K*; an ordered compaction keeps keys > K* and the first
//      k - #(> K*) ties of K* in ID order;
//   5. a stable LSD radix sort (two passes, descending digits) of those k
//      elements reproduces the reference order: key descending, ID ascending.
// Histograms and ranks use warp-aggregated counting (__match_any_sync); the
// ordered scatter walks each warp's contiguous segment in order, so ties keep
// ID order without a comparison sort.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr unsigned long long kSmemKeysMax = 65536;  // keys kept in shared memory up to this

// Workspace header (zeroed before each launch).
struct SelectHeader {
    unsigned int arrived;
    unsigned int pad[31];
    unsigned int err[128];     // bit0 non-finite score, bit1 rounded count overflow
    float rounded[128];
};

struct SelectParams {
    const uint16_t* scores;
    int raw, cover, fp32_counts, zero_is_error;
    uint32_t heads;
    unsigned long long stride, valid, kcap, cover_cap;
    float alpha, ratio;
    uint32_t* ids;
    uint32_t* counts;
    hsb_selection* result;
    SelectHeader* header;
    uint16_t* gkeys;             // [heads][valid] when valid > kSmemKeysMax
    unsigned long long* sortbuf;  // [heads][2][kcap]
};

struct SelectShared {
    unsigned int hist[kWarps][256];  // per-warp histograms / scatter offsets
    unsigned int bins[256];
    unsigned int scan[kWarps];
    float fred[kWarps];
    unsigned int ured[kWarps];
    unsigned int b_bin, b_above, b_eqtotal;
    unsigned int status, status_index;
    unsigned long long k;
    unsigned int last_id, next_id;
    int timeout;
};

__device__ __forceinline__ uint16_t load_norm(const SelectParams& p, unsigned long long i) {
    const uint16_t s = p.scores[i];
    return p.raw ? scale_half(s) : s;
}

// Block-wide exclusive scan of one u32 per thread; returns the exclusive
// prefix and writes the block total to *total.
__device__ unsigned int block_exclusive_scan(unsigned int v, unsigned int* scan, unsigned int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) scan[warp] = x;
    __syncthreads();
    if (warp == 0) {
        unsigned int w = scan[lane];
        unsigned int s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        scan[lane] = s - w;  // exclusive warp offsets
        if (lane == 31) *total = s;
    }
    __syncthreads();
    const unsigned int r = scan[warp] + x - v;
    __syncthreads();
    return r;
}

__device__ __forceinline__ void zero_hist(SelectShared& sh) {
    for (int i = threadIdx.x; i < kWarps * 256; i += kThreads) (&sh.hist[0][0])[i] = 0;
}

// Per-warp histogram of digit(key) over keys[0,n) (strided by the block);
// keys outside the filter count nowhere.  Result summed into sh.bins.
template <class DigitFn>
__device__ void key_histogram(SelectShared& sh, const uint16_t* keys, unsigned long long n, DigitFn digit) {
    zero_hist(sh);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (unsigned long long base = (unsigned long long)warp * 32; base < n; base += kThreads) {
        const unsigned long long i = base + lane;
        const unsigned int d = i < n ? digit(keys[i]) : 0x100u;  // 0x100 = not counted
        const unsigned int peers = __match_any_sync(0xffffffffu, d);
        if (d < 0x100u && lane == __ffs(peers) - 1) sh.hist[warp][d] += __popc(peers);
    }
    __syncthreads();
    if (threadIdx.x < 256) {
        unsigned int s = 0;
#pragma unroll 8
        for (int w = 0; w < kWarps; ++w) s += sh.hist[w][threadIdx.x];
        sh.bins[threadIdx.x] = s;
    }
    __syncthreads();
}

// Finds the bin holding the `need`-th largest element: the bin b with
// (#elements in bins > b) < need <= (#elements in bins >= b).
__device__ void find_bin(SelectShared& sh, unsigned int need) {
    // Suffix sums over 256 bins, computed by warp 0 with 8 bins per lane.
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        unsigned int local[8];
        unsigned int s = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // lane owns bins 255-8*lane-j, descending
            local[j] = sh.bins[255 - 8 * lane - j];
            s += local[j];
        }
        unsigned int x = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        unsigned int above = x - s;  // elements in bins above this lane's first bin
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const unsigned int b = 255 - 8 * lane - j;
            if (above < need && above + local[j] >= need) {
                sh.b_bin = b;
                sh.b_above = above;
                sh.b_eqtotal = local[j];
            }
            above += local[j];
        }
    }
    __syncthreads();
}

// Stable LSD pass over m elements: src -> dst by digit 255-((key>>shift)&255),
// i.e. keys descending, earlier elements first among equal digits.
__device__ void sort_pass(SelectShared& sh, const unsigned long long* src, unsigned long long* dst,
                          unsigned int m, int shift) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned int seg = (m + kWarps - 1) / kWarps;
    const unsigned int begin = min(m, warp * seg), end = min(m, begin + seg);
    zero_hist(sh);
    __syncthreads();
    for (unsigned int base = begin; base < end; base += 32) {
        const unsigned int i = base + lane;
        const unsigned int d = i < end ? 255u - (unsigned int)((src[i] >> (32 + shift)) & 0xffu) : 0x100u;
        const unsigned int peers = __match_any_sync(0xffffffffu, d);
        if (d < 0x100u && lane == __ffs(peers) - 1) sh.hist[warp][d] += __popc(peers);
    }
    __syncthreads();
    // Exclusive scan over (digit, warp) in digit-major order: 8192 counters,
    // eight consecutive ones per thread.
    unsigned int vals[8], local = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const unsigned int f = threadIdx.x * 8 + j;  // f = digit*32 + warp
        vals[j] = sh.hist[f & 31][f >> 5];
        local += vals[j];
    }
    unsigned int total;
    unsigned int off = block_exclusive_scan(local, sh.scan, &total);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const unsigned int f = threadIdx.x * 8 + j;
        sh.hist[f & 31][f >> 5] = off;
        off += vals[j];
    }
    __syncthreads();
    for (unsigned int base = begin; base < end; base += 32) {
        const unsigned int i = base + lane;
        const unsigned long long e = i < end ? src[i] : 0ull;
        const unsigned int d = i < end ? 255u - (unsigned int)((e >> (32 + shift)) & 0xffu) : 0x100u;
        const unsigned int peers = __match_any_sync(0xffffffffu, d);
        unsigned int pos = 0;
        if (d < 0x100u) pos = sh.hist[warp][d] + __popc(peers & lanemask_lt());
        __syncwarp();
        if (d < 0x100u) {
            if (pos < m) dst[pos] = e;
            if (lane == __ffs(peers) - 1) sh.hist[warp][d] += __popc(peers);
        }
        __syncwarp();
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) select_kernel(const __grid_constant__ SelectParams p) {
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ SelectShared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t h = blockIdx.x;
    const unsigned long long n = p.valid;
    uint16_t* keys = n <= kSmemKeysMax ? reinterpret_cast<uint16_t*>(dyn) : p.gkeys + (unsigned long long)h * n;

    // ---- 1. head-0 maximum of the normalised scores, threshold
    float mx = -INFINITY;
    unsigned int bad0 = 0;
    for (unsigned long long i = tid; i < n; i += kThreads) {
        const uint16_t x = load_norm(p, i);
        if (!is_finite_half(x)) bad0 = 1;
        const float v = half_value(x);
        mx = fmaxf(mx, v);  // NaN never replaces the running maximum, as std::max
    }
    mx = warp_max(mx);
    bad0 = __any_sync(0xffffffffu, bad0);
    if (lane == 0) {
        sh.fred[warp] = mx;
        sh.ured[warp] = bad0;
    }
    __syncthreads();
    if (tid == 0) {
        float m = -INFINITY;
        unsigned int b = 0;
        for (int w = 0; w < kWarps; ++w) {
            m = fmaxf(m, sh.fred[w]);
            b |= sh.ured[w];
        }
        sh.fred[0] = m;
        sh.ured[0] = b;
    }
    __syncthreads();
    const float threshold = half_value(half_bits(sh.fred[0] - p.alpha));
    const bool head0_bad = !p.cover && sh.ured[0];
    const bool thr_bad = !isfinite(threshold);
    if (head0_bad || thr_bad) {
        if (h == 0 && tid == 0) {
            p.result->k = 0;
            p.result->status.code = head0_bad ? HSB_E_SEL_NONFINITE_HEAD0
                                              : (p.cover ? HSB_E_COVER_THRESHOLD : HSB_E_SEL_THRESHOLD);
            p.result->status.index = 0;
        }
        return;  // every CTA takes this branch; no barrier is pending
    }
    const unsigned int thr_key = order_key(half_bits(threshold));

    // ---- 2. own row: keys, count >= threshold
    unsigned int cnt = 0, bad = 0;
    const uint16_t* row = p.scores + (unsigned long long)h * p.stride;
    for (unsigned long long i = tid; i < n; i += kThreads) {
        const uint16_t s = row[i];
        const uint16_t x = p.raw ? scale_half(s) : s;
        const bool nan = (x & 0x7fffu) > 0x7c00u;
        if (!is_finite_half(x)) bad = 1;
        const unsigned int key = order_key(x);
        keys[i] = (uint16_t)key;
        cnt += (!nan && key >= thr_key) ? 1u : 0u;
    }
    cnt = warp_sum_u32(cnt);
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        sh.ured[warp] = cnt;
        sh.scan[warp] = bad;
    }
    __syncthreads();
    if (tid == 0) {
        unsigned long long c = 0;
        unsigned int b = 0;
        for (int w = 0; w < kWarps; ++w) {
            c += sh.ured[w];
            b |= sh.scan[w];
        }
        if (p.cover) c += 1;  // at most one newly appended current token
        const float rounded = p.fp32_counts ? (float)c : half_value(half_bits((float)c));
        p.header->rounded[h] = rounded;
        p.header->err[h] = ((!p.cover && b) ? 1u : 0u) | (isfinite(rounded) ? 0u : 2u);
        if (p.counts) p.counts[h] = (uint32_t)c;
        // ---- 3. grid barrier (bounded)
        __threadfence();
        atomicAdd(&p.header->arrived, 1u);
        const unsigned long long start = global_ns();
        sh.timeout = 0;
        while (atomicAdd(&p.header->arrived, 0u) < p.heads) {
            if (global_ns() - start > kWaitLimitNs) {
                sh.timeout = 1;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
        // Every CTA derives the same status and k from the shared counts.
        unsigned int status = 0, index = 0;
        float total = 0.0f;
        if (!sh.timeout) {
            for (uint32_t hh = 0; hh < p.heads; ++hh) {
                const unsigned int e = ((volatile unsigned int*)p.header->err)[hh];
                if (e & 1u) { status = HSB_E_SEL_NONFINITE; index = hh; break; }
                if (e & 2u) { status = p.cover ? HSB_E_COVER_COUNT : HSB_E_SEL_COUNT_F16; index = hh; break; }
                total += ((volatile float*)p.header->rounded)[hh];
            }
        }
        unsigned long long k = 0;
        if (!sh.timeout && !status) {
            const float mean = p.fp32_counts ? __fdiv_rn(total, (float)p.heads)
                                             : half_value(half_bits(__fdiv_rn(total, (float)p.heads)));
            if (p.cover) {
                if (!(isfinite(mean) && mean >= 1.0f)) status = HSB_E_COVER_MEAN;
                else k = min(p.cover_cap, (unsigned long long)mean);
            } else {
                if (!isfinite(mean)) status = HSB_E_SEL_MEAN_F16;
                else {
                    k = (unsigned long long)mean;
                    const unsigned long long cap = (unsigned long long)floor((double)n * (double)p.ratio);
                    k = min(k, min(cap, n));
                }
            }
        }
        if (sh.timeout) status = HSB_E_TIMEOUT;
        if (!status && k == 0 && p.zero_is_error) status = HSB_E_ZERO_SELECTION;
        sh.status = status;
        sh.status_index = index;
        sh.k = status ? 0 : k;
        if (h == 0) {
            p.result->k = (uint32_t)sh.k;
            p.result->status.code = (int)status;
            p.result->status.index = (int)index;
        }
    }
    __syncthreads();
    const unsigned long long k = sh.k;
    if (sh.status || k == 0) return;

    // ---- 4. radix select: K* = k-th largest key
    key_histogram(sh, keys, n, [](unsigned int key) { return key >> 8; });
    find_bin(sh, (unsigned int)k);
    const unsigned int hi = sh.b_bin, above_hi = sh.b_above;
    key_histogram(sh, keys, n, [hi](unsigned int key) { return (key >> 8) == hi ? (key & 0xffu) : 0x100u; });
    find_bin(sh, (unsigned int)(k - above_hi));
    const unsigned int kstar = (hi << 8) | sh.b_bin;
    const unsigned int gt = above_hi + sh.b_above;
    const unsigned int need_eq = (unsigned int)k - gt;  // >= 1
    const unsigned int eq_total = sh.b_eqtotal;

    // ---- ordered compaction into sort buffer A (ID order)
    unsigned long long* bufA = p.sortbuf + (unsigned long long)h * 2 * p.kcap;
    unsigned long long* bufB = bufA + p.kcap;
    const unsigned long long seg = (n + kThreads - 1) / kThreads;
    const unsigned long long b0 = min(n, (unsigned long long)tid * seg), b1 = min(n, b0 + seg);
    unsigned int n_gt = 0, n_eq = 0;
    for (unsigned long long i = b0; i < b1; ++i) {
        const unsigned int key = keys[i];
        n_gt += key > kstar;
        n_eq += key == kstar;
    }
    unsigned int tot;
    const unsigned int gt_before = block_exclusive_scan(n_gt, sh.scan, &tot);
    unsigned int eq_rank = block_exclusive_scan(n_eq, sh.scan, &tot);
    unsigned int pos = gt_before + min(eq_rank, need_eq);
    if (tid == 0) {
        sh.last_id = 0xffffffffu;
        sh.next_id = 0xffffffffu;
    }
    __syncthreads();
    for (unsigned long long i = b0; i < b1; ++i) {
        const unsigned int key = keys[i];
        // pos < k holds by construction; the guard keeps any slip in bounds.
        if (key > kstar) {
            if (pos < k) bufA[pos] = ((unsigned long long)key << 32) | (unsigned int)i;
            ++pos;
        } else if (key == kstar) {
            if (eq_rank < need_eq) {
                if (pos < k) bufA[pos] = ((unsigned long long)key << 32) | (unsigned int)i;
                ++pos;
            }
            if (eq_rank + 1 == need_eq) sh.last_id = (unsigned int)i;
            if (eq_rank == need_eq) sh.next_id = (unsigned int)i;
            ++eq_rank;
        }
    }
    __syncthreads();
    // Boundary tie (gqa_policy.cpp:66): the k-th and (k+1)-th ordered IDs carry
    // the same normalised F16 bits.  Only possible among ties of K*.
    if (!p.cover && tid == 0 && k < n && eq_total > need_eq) {
        const uint16_t a = load_norm(p, (unsigned long long)h * p.stride + sh.last_id);
        const uint16_t b = load_norm(p, (unsigned long long)h * p.stride + sh.next_id);
        if (a == b) atomicAdd(&p.result->boundary_tied_heads, 1u);
    }

    // ---- 5. stable sort by key descending (low byte, then high byte)
    __threadfence_block();
    __syncthreads();
    sort_pass(sh, bufA, bufB, (unsigned int)k, 0);
    sort_pass(sh, bufB, bufA, (unsigned int)k, 8);
    uint32_t* out = p.ids + (unsigned long long)h * p.kcap;
    for (unsigned int j = tid; j < k; j += kThreads) out[j] = (uint32_t)(bufA[j] & 0xffffffffu);
}

}  // namespace

size_t select_workspace_bytes(size_t heads, size_t valid, size_t kcap) {
    size_t bytes = sizeof(SelectHeader);
    bytes = (bytes + 255) / 256 * 256;
    if (valid > kSmemKeysMax) bytes += (heads * valid * 2 + 255) / 256 * 256;
    bytes += heads * 2 * kcap * 8;
    return bytes;
}

cudaError_t launch_select(const SelectLaunch& s, cudaStream_t stream) {
    const DeviceInfo& dev = device_info();
    SelectParams p{};
    p.scores = s.scores;
    p.raw = s.raw;
    p.cover = s.cover;
    p.fp32_counts = s.fp32_counts;
    p.zero_is_error = s.zero_is_error;
    p.heads = s.heads;
    p.stride = s.stride;
    p.valid = s.valid;
    p.kcap = s.kcap;
    p.cover_cap = s.cover_cap;
    p.alpha = s.alpha;
    p.ratio = s.ratio;
    p.ids = s.ids;
    p.counts = s.counts;
    p.result = s.result;
    unsigned char* ws = static_cast<unsigned char*>(s.workspace);
    p.header = reinterpret_cast<SelectHeader*>(ws);
    size_t off = (sizeof(SelectHeader) + 255) / 256 * 256;
    if (s.valid > kSmemKeysMax) {
        p.gkeys = reinterpret_cast<uint16_t*>(ws + off);
        off += (s.heads * s.valid * 2 + 255) / 256 * 256;
    }
    p.sortbuf = reinterpret_cast<unsigned long long*>(ws + off);
    cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(SelectHeader), stream);
    if (e != cudaSuccess) return e;
    if (s.reset_result) {
        e = cudaMemsetAsync(s.result, 0, sizeof(hsb_selection), stream);
        if (e != cudaSuccess) return e;
    }
    const size_t smem = s.valid <= kSmemKeysMax ? (size_t)s.valid * 2 : 0;
    static thread_local int configured_device = -1;
    if (configured_device != dev.ordinal) {
        e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kSmemKeysMax * 2));
        if (e != cudaSuccess) return e;
        configured_device = dev.ordinal;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(s.heads);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, select_kernel, p);
}

}  // namespace hsb
