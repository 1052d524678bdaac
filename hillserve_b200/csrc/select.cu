// select.cu -- stage 2: the gqa_policy selector (policy/gqa_policy.cpp:47-70)
// and the history-only prefetch cover (policy/full_gqa_runtime.cpp:299-344).
//
// Two kernels, both launched cooperatively so that all CTAs are resident and
// can meet at one bounded grid barrier (the cross-head count exchange):
//  - select_cluster_kernel (valid <= 65536, the usual case): each head is a
//    cluster of four 512-thread CTAs, each owning a quarter of the head's
//    tokens, sharing histograms through distributed shared memory;
//  - select_kernel (longer rows, or more heads than clusters fit): one CTA
//    of 1024 threads per head.
// The steps below are those of select_kernel; the cluster kernel runs the
// same steps on its chunk and combines per-chunk histograms and counts.
//
// Everything works on 16-bit order keys of the normalised F16 scores (the key
// order is the FP32 comparator order with -0 == +0, policy/half_order.hpp):
//   1. each CTA reads head 0's row and its own row with 16-byte loads, forms
//      the keys (from normalised bits, from raw bits by the exact division,
//      or as given when the scorer already emitted keys), reduces the head-0
//      maximum, derives the F16 threshold F16(max - alpha), and counts keys
//      >= threshold while storing its row's keys in shared memory;
//   2. grid barrier; every CTA reads the per-head counts, rounds them as the
//      reference does (F16 count, FP32 sum, F16 mean) and derives the same k
//      and the same first error;
//   3. radix select: a 1024-bin histogram of key >> 6 (built while loading)
//      and a 64-bin pass over the keys of the chosen bin give the k-th
//      largest key K*;
//   4. ordered compaction (ballots, warp-contiguous segments) keeps keys > K*
//      and the first k - #(> K*) ties of K* in ID order;
//   5. the k survivors are put in reference order -- key descending, ID
//      ascending -- by a rank sort (small k) or a stable LSD radix sort.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstddef>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr unsigned long long kSmemKeysMax = 65536;  // keys kept in shared memory up to this
constexpr unsigned kSmemSortMax = 2048;             // survivors sorted in shared memory up to this
constexpr unsigned kRankSortMax = 256;              // rank sort up to this, radix above

enum InputMode { kInputScaled = 0, kInputRaw = 1, kInputKeys = 2 };

// Workspace header (zeroed before each launch).
struct SelectHeader {
    unsigned int arrived;
    unsigned int pad[31];
    unsigned int err[128];  // bit0 non-finite score, bit1 rounded count overflow
    float rounded[128];
    // Cluster path, one word per head, added to once by each of the head's
    // CTAs: bits 0-7 CTAs arrived, 8-15 CTAs that saw a non-finite key,
    // 16-63 the threshold count.  The word is both the data and the barrier.
    unsigned long long hc[128];
};

struct SelectParams {
    const uint16_t* scores;   // normalised bits, raw bits, or keys (mode)
    const uint16_t* tie_raw;  // keys mode: raw scores, to tell +0 from -0 at a tie
    int mode, cover, fp32_counts, zero_is_error;
    uint32_t heads;
    unsigned long long stride, valid, kcap, cover_cap;
    float alpha, ratio;
    uint32_t* ids;
    uint32_t* counts;
    hsb_selection* result;
    SelectHeader* header;
    uint16_t* gkeys;              // [heads][valid] when valid > kSmemKeysMax
    unsigned long long* sortbuf;  // [heads][2][kcap] when k > kSmemSortMax
    const uint32_t* h0;           // optional: the scorer's head-0 partials [kH0Partials]
    SelectEpilogue ga;            // cluster path: gather + attention of the selection (ga.out != null)
    // KV-head shard (cluster path): the heads [head_base, head_base + heads)
    // of heads_total; the threshold record ext_thr = {key, status} and every
    // head's count record ext[heads_total] (count | non-finite << 31) come
    // from the exchange between shards, replacing the count and the barrier.
    const uint32_t* ext;
    const uint32_t* ext_thr;
    uint32_t head_base, heads_total;
    // Batch of sequences (shard steps; 1 otherwise): blockIdx.x covers
    // batch x heads x the cluster size (kBatchCluster in record mode).  Sequence b's scores / keys start b *
    // seq_scores elements in; every per-head output advances by its own size.
    uint32_t batch;
    unsigned long long seq_scores;
    // Current position scored here (see SelectLaunch): cur_q, cur_k, cur_raw.
    const uint16_t* cur_q;
    const uint16_t* cur_k;
    uint16_t* cur_raw;
};

// Head-0 maximum key and non-finite flag from the scorer's per-CTA partials
// (the fused layer step), instead of a pass over head 0's row.
template <int NT>
__device__ __forceinline__ void head0_from_partials(const uint32_t* h0, unsigned int& mx, unsigned int& bad0) {
    for (unsigned int i = threadIdx.x; i < kH0Partials; i += NT) {
        const uint32_t v = __ldcg(h0 + i);
        mx = max(mx, v & 0xffffu);
        bad0 |= v >> 16;
    }
}

struct SelectShared {
    unsigned int hist[kWarps][256];  // per-warp histograms / scatter offsets
    unsigned int coarse[1024];       // histogram of key >> 6, built while loading
    unsigned int fine[64];           // histogram of key & 63 inside the chosen coarse bin
    unsigned int scan[kWarps];
    unsigned int wa[kWarps], wb[kWarps];
    unsigned int b_bin, b_above, b_eqtotal, total;
    unsigned int status, status_index;
    unsigned int maxkey, bad0, cnt, bad;
    unsigned long long k;
    unsigned int last_id, next_id;
    int timeout;
};

// key -> F16 bits (inverse of order_key; -0 comes back as +0)
__device__ __forceinline__ uint32_t key_bits(uint32_t key) {
    return (key & 0x8000u) ? (key ^ 0x8000u) : (~key & 0xffffu);
}

__device__ __forceinline__ uint32_t to_key(uint32_t v, int mode) {
    if (mode == kInputKeys) return v;
    return order_key(mode == kInputRaw ? scale_half((uint16_t)v) : v);
}

// Block-wide exclusive scan of one u32 per thread (NT threads); the total
// goes to *total.  scan[] holds one word per warp.
template <int NT>
__device__ unsigned int block_exclusive_scan(unsigned int v, unsigned int* scan, unsigned int* total) {
    constexpr int kW = NT / 32;
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
        const unsigned int w = lane < kW ? scan[lane] : 0u;
        unsigned int s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kW) scan[lane] = s - w;
        if (lane == 31) *total = s;
    }
    __syncthreads();
    const unsigned int r = scan[warp] + x - v;
    __syncthreads();
    return r;
}

// Stable LSD pass over m elements (key << 32 | id): src -> dst by digit
// 255 - ((key >> shift) & 255), i.e. keys descending, earlier first on ties.
// hist is [NT / 32][256] per-warp counts / scatter offsets.
template <int NT>
__device__ void sort_pass(unsigned int (*hist)[256], unsigned int* scan, unsigned int* total,
                          const unsigned long long* src, unsigned long long* dst, unsigned int m, int shift) {
    constexpr int kW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned int seg = (m + kW - 1) / kW;
    const unsigned int begin = min(m, warp * seg), end = min(m, begin + seg);
    for (int i = threadIdx.x; i < kW * 256; i += NT) (&hist[0][0])[i] = 0;
    __syncthreads();
    for (unsigned int base = begin; base < end; base += 32) {
        const unsigned int i = base + lane;
        const unsigned int d = i < end ? 255u - (unsigned int)((src[i] >> (32 + shift)) & 0xffu) : 0x100u;
        const unsigned int peers = __match_any_sync(0xffffffffu, d);
        if (d < 0x100u && lane == __ffs(peers) - 1) hist[warp][d] += __popc(peers);
    }
    __syncthreads();
    // Entry f = digit * kW + warp: digit-major, warp-minor -> stable offsets.
    constexpr int kPer = kW * 256 / NT;  // 8
    unsigned int vals[kPer], local = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const unsigned int f = threadIdx.x * kPer + j;
        vals[j] = hist[f % kW][f / kW];
        local += vals[j];
    }
    unsigned int off = block_exclusive_scan<NT>(local, scan, total);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const unsigned int f = threadIdx.x * kPer + j;
        hist[f % kW][f / kW] = off;
        off += vals[j];
    }
    __syncthreads();
    for (unsigned int base = begin; base < end; base += 32) {
        const unsigned int i = base + lane;
        const unsigned long long e = i < end ? src[i] : 0ull;
        const unsigned int d = i < end ? 255u - (unsigned int)((e >> (32 + shift)) & 0xffu) : 0x100u;
        const unsigned int peers = __match_any_sync(0xffffffffu, d);
        unsigned int pos = 0;
        if (d < 0x100u) pos = hist[warp][d] + __popc(peers & lanemask_lt());
        __syncwarp();
        if (d < 0x100u) {
            if (pos < m) dst[pos] = e;  // pos < m by construction; the guard keeps a slip in bounds
            if (lane == __ffs(peers) - 1) hist[warp][d] += __popc(peers);
        }
        __syncwarp();
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) select_kernel(const __grid_constant__ SelectParams p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ SelectShared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t h = blockIdx.x;
    const unsigned long long n = p.valid;
    const bool smem_keys = n <= kSmemKeysMax;
    uint16_t* keys = smem_keys ? reinterpret_cast<uint16_t*>(dyn) : p.gkeys + (unsigned long long)h * n;
    const uint16_t* row0 = p.scores;
    const uint16_t* row = p.scores + (unsigned long long)h * p.stride;
    // Vector path: 16-byte aligned rows; the tail of a row goes element-wise.
    const bool vec = (p.stride % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.scores) & 15) == 0) &&
                     (smem_keys || (reinterpret_cast<uintptr_t>(keys) & 15) == 0);
    const unsigned long long n8 = vec ? n / 8 : 0;

    if (tid == 0) {
        sh.maxkey = 0;
        sh.bad0 = 0;
        sh.cnt = 0;
        sh.bad = 0;
    }
    sh.coarse[tid] = 0;
    if (tid < 64) sh.fine[tid] = 0;
    // ---- 1a. head-0 maximum key (NaN never becomes the maximum, as std::max)
    unsigned int mx = 0, bad0 = 0;
    if (p.h0) head0_from_partials<kThreads>(p.h0, mx, bad0);
#pragma unroll 4
    for (unsigned long long g = tid; g < (p.h0 ? 0 : n8); g += kThreads) {
        const uint4 w = reinterpret_cast<const uint4*>(row0)[g];
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t key = to_key((v[j >> 1] >> (16 * (j & 1))) & 0xffffu, p.mode);
            bad0 |= key_nonfinite(key);
            mx = key_nan(key) ? mx : max(mx, key);
        }
    }
    for (unsigned long long i = n8 * 8 + tid; i < (p.h0 ? 0 : n); i += kThreads) {
        const uint32_t key = to_key(row0[i], p.mode);
        bad0 |= key_nonfinite(key);
        mx = key_nan(key) ? mx : max(mx, key);
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    bad0 = __any_sync(0xffffffffu, bad0);
    __syncthreads();
    if (lane == 0) {
        atomicMax(&sh.maxkey, mx);
        if (bad0) atomicOr(&sh.bad0, 1u);
    }
    __syncthreads();
    const float maximum = half_value((uint16_t)key_bits(sh.maxkey));
    const float threshold = half_value(half_bits(sh.maxkey ? maximum - p.alpha : -INFINITY));
    const bool head0_bad = !p.cover && sh.bad0;
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

    // ---- 1b. own row: keys to shared memory, count >= threshold
    unsigned int cnt = 0, bad = 0;
#pragma unroll 4
    for (unsigned long long g = tid; g < n8; g += kThreads) {
        const uint4 w = reinterpret_cast<const uint4*>(row)[g];
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
        uint32_t k2[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const uint32_t a = to_key(v[j >> 1] & 0xffffu, p.mode), b = to_key(v[j >> 1] >> 16, p.mode);
            bad |= key_nonfinite(a) | key_nonfinite(b);
            cnt += (!key_nan(a) && a >= thr_key) + (!key_nan(b) && b >= thr_key);
            atomicAdd(&sh.coarse[a >> 6], 1u);
            atomicAdd(&sh.coarse[b >> 6], 1u);
            k2[j >> 1] = a | (b << 16);
        }
        reinterpret_cast<uint4*>(keys)[g] = make_uint4(k2[0], k2[1], k2[2], k2[3]);
    }
    for (unsigned long long i = n8 * 8 + tid; i < n; i += kThreads) {
        const uint32_t key = to_key(row[i], p.mode);
        bad |= key_nonfinite(key);
        cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
        atomicAdd(&sh.coarse[key >> 6], 1u);
        keys[i] = (uint16_t)key;
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        atomicAdd(&sh.cnt, cnt);
        if (bad) atomicOr(&sh.bad, 1u);
    }
    __syncthreads();
    if (tid == 0) {
        unsigned long long c = sh.cnt;
        if (p.cover) c += 1;  // at most one newly appended current token
        const float rounded = p.fp32_counts ? (float)c : half_value(half_bits((float)c));
        p.header->rounded[h] = rounded;
        p.header->err[h] = ((!p.cover && sh.bad) ? 1u : 0u) | (isfinite(rounded) ? 0u : 2u);
        if (p.counts) p.counts[h] = (uint32_t)c;
        // ---- 2. grid barrier (bounded)
        __threadfence();
        atomicAdd(&p.header->arrived, 1u);
        const unsigned long long start = global_ns();
        sh.timeout = 0;
        while (atomicAdd(&p.header->arrived, 0u) < p.heads) {
            if (global_ns() - start > kWaitLimitNs) {
                sh.timeout = 1;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
    }
    __syncthreads();
    if (warp == 0) {
        // All heads' flags and rounded counts, read in parallel (4 per lane),
        // then folded in head order -- the first error is the reference's.
        unsigned int e[4] = {0, 0, 0, 0};
        float r[4] = {0.f, 0.f, 0.f, 0.f};
        if (!sh.timeout) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t hh = lane * 4 + j;
                if (hh < p.heads) {
                    e[j] = __ldcg(&p.header->err[hh]);
                    r[j] = __ldcg(&p.header->rounded[hh]);
                }
            }
        }
        unsigned int status = 0, index = 0;
        float total = 0.0f;
        for (int src = 0; src < 32 && !sh.timeout; ++src) {
            unsigned int ej[4];
            float rj[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ej[j] = __shfl_sync(0xffffffffu, e[j], src);
                rj[j] = __shfl_sync(0xffffffffu, r[j], src);
            }
            bool stop = false;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t hh = src * 4 + j;
                if (stop || hh >= p.heads) continue;
                if (ej[j] & 1u) { status = HSB_E_SEL_NONFINITE; index = hh; stop = true; continue; }
                if (ej[j] & 2u) { status = p.cover ? HSB_E_COVER_COUNT : HSB_E_SEL_COUNT_F16; index = hh; stop = true; continue; }
                total += rj[j];  // FP32 sum in head order (gqa_policy.cpp:60)
            }
            if (stop || (uint32_t)(src + 1) * 4 >= p.heads) break;
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
        if (lane == 0) {
            sh.status = status;
            sh.status_index = index;
            sh.k = status ? 0 : k;
            if (h == 0) {
                p.result->k = status ? 0u : (uint32_t)k;
                p.result->status.code = (int)status;
                p.result->status.index = (int)index;
            }
        }
    }
    __syncthreads();
    const unsigned long long k = sh.k;
    if (k == 0) return;

    // ---- 3. radix select: K* = k-th largest key.  Coarse bins (key >> 6) were
    // counted while loading; thread t owns bin 1023 - t, so an exclusive scan
    // gives "elements in higher bins".
    const unsigned long long seg = ((n + kWarps - 1) / kWarps + 31) / 32 * 32;
    const unsigned long long s0 = min(n, (unsigned long long)warp * seg), s1 = min(n, s0 + seg);
    {
        const unsigned int bin = 1023u - tid, c = sh.coarse[bin];
        const unsigned int above = block_exclusive_scan<kThreads>(c, sh.scan, &sh.total);
        if (above < k && above + c >= k) {
            sh.b_bin = bin;
            sh.b_above = above;
        }
    }
    __syncthreads();
    const unsigned int hi = sh.b_bin, above_hi = sh.b_above;
    for (unsigned long long i = tid; i < n; i += kThreads) {
        const unsigned int key = keys[i];
        if ((key >> 6) == hi) atomicAdd(&sh.fine[key & 63u], 1u);
    }
    __syncthreads();
    if (warp == 0) {  // 64 fine bins, two per lane, descending
        const unsigned int c0 = sh.fine[63 - 2 * lane], c1 = sh.fine[62 - 2 * lane];
        unsigned int x = c0 + c1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        const unsigned int need = (unsigned int)k - above_hi;
        unsigned int above = x - c0 - c1;
        if (above < need && above + c0 >= need) {
            sh.b_bin = 63 - 2 * lane;
            sh.b_above = above;
            sh.b_eqtotal = c0;
        }
        above += c0;
        if (above < need && above + c1 >= need) {
            sh.b_bin = 62 - 2 * lane;
            sh.b_above = above;
            sh.b_eqtotal = c1;
        }
    }
    __syncthreads();
    const unsigned int kstar = (hi << 6) | sh.b_bin;
    const unsigned int gt = above_hi + sh.b_above;
    const unsigned int need_eq = (unsigned int)k - gt;  // >= 1
    const unsigned int eq_total = sh.b_eqtotal;

    // ---- 4. ordered compaction (ID order) of keys > K* and the first need_eq ties
    const bool small = k <= kSmemSortMax;
    unsigned long long* bufA =
        small ? reinterpret_cast<unsigned long long*>(dyn + (smem_keys ? ((n * 2 + 15) / 16 * 16) : 0))
              : p.sortbuf + (unsigned long long)h * 2 * p.kcap;
    unsigned long long* bufB = bufA + (small ? kSmemSortMax : p.kcap);
    unsigned int w_gt = 0, w_eq = 0;
    for (unsigned long long base = s0; base < s1; base += 32) {
        const unsigned long long i = base + lane;
        const unsigned int key = i < s1 ? keys[i] : 0u;
        w_gt += __popc(__ballot_sync(0xffffffffu, i < s1 && key > kstar));
        w_eq += __popc(__ballot_sync(0xffffffffu, i < s1 && key == kstar));
    }
    if (lane == 0) {
        sh.wa[warp] = w_gt;
        sh.wb[warp] = w_eq;
    }
    if (tid == 0) {
        sh.last_id = 0xffffffffu;
        sh.next_id = 0xffffffffu;
    }
    __syncthreads();
    unsigned int gt_before = 0, eq_before = 0;
    for (int w = 0; w < warp; ++w) {
        gt_before += sh.wa[w];
        eq_before += sh.wb[w];
    }
    unsigned int pos = gt_before + min(eq_before, need_eq);
    for (unsigned long long base = s0; base < s1; base += 32) {
        const unsigned long long i = base + lane;
        const unsigned int key = i < s1 ? keys[i] : 0u;
        const bool is_gt = i < s1 && key > kstar;
        const bool is_eq = i < s1 && key == kstar;
        const unsigned int meq = __ballot_sync(0xffffffffu, is_eq);
        const unsigned int my_eq = eq_before + __popc(meq & lanemask_lt());
        const bool take = is_gt || (is_eq && my_eq < need_eq);
        const unsigned int mtake = __ballot_sync(0xffffffffu, take);
        if (take) {
            const unsigned int at = pos + __popc(mtake & lanemask_lt());
            if (at < k) bufA[at] = ((unsigned long long)key << 32) | (unsigned int)i;
        }
        if (is_eq && my_eq + 1 == need_eq) sh.last_id = (unsigned int)i;
        if (is_eq && my_eq == need_eq) sh.next_id = (unsigned int)i;
        pos += __popc(mtake);
        eq_before += __popc(meq);
    }
    __syncthreads();
    // Boundary tie (gqa_policy.cpp:66): the k-th and (k+1)-th ordered IDs carry
    // the same normalised F16 bits.  Only ties of K* can, and equal keys have
    // equal bits except +0 / -0, which are told apart from the scores.
    if (!p.cover && tid == 0 && k < n && eq_total > need_eq) {
        bool tied = true;
        if (kstar == 0x8000u) {
            const unsigned long long base = (unsigned long long)h * p.stride;
            uint16_t a, b;
            if (p.mode == kInputKeys) {
                a = p.tie_raw ? scale_half(p.tie_raw[base + sh.last_id]) : 0;
                b = p.tie_raw ? scale_half(p.tie_raw[base + sh.next_id]) : 0;
            } else {
                a = p.scores[base + sh.last_id];
                b = p.scores[base + sh.next_id];
                if (p.mode == kInputRaw) {
                    a = scale_half(a);
                    b = scale_half(b);
                }
            }
            tied = a == b;
        }
        if (tied) atomicAdd(&p.result->boundary_tied_heads, 1u);
    }

    // ---- 5. reference order: key descending, ID ascending
    __syncthreads();
    uint32_t* out = p.ids + (unsigned long long)h * p.kcap;
    if (k <= kRankSortMax) {
        // rank = #(greater key) + #(equal key earlier in ID order)
        if ((unsigned)tid < k) {
            const unsigned long long e = bufA[tid];
            const unsigned int ek = (unsigned int)(e >> 32);
            unsigned int r = 0;
            for (unsigned int j = 0; j < k; ++j) {
                const unsigned int ok = (unsigned int)(bufA[j] >> 32);
                r += (ok > ek) || (ok == ek && j < (unsigned)tid);
            }
            if (r < k) out[r] = (uint32_t)(e & 0xffffffffu);
        }
        return;
    }
    sort_pass<kThreads>(sh.hist, sh.scan, &sh.total, bufA, bufB, (unsigned int)k, 0);
    sort_pass<kThreads>(sh.hist, sh.scan, &sh.total, bufB, bufA, (unsigned int)k, 8);
    for (unsigned int j = tid; j < k; j += kThreads) out[j] = (uint32_t)(bufA[j] & 0xffffffffu);
}


// ------------------------------------------------------------------ cluster path
// The same selector with each head spread over a cluster of kCluster CTAs
// (kCThreads threads each, two CTAs per SM): CTA r of head h owns the
// contiguous token chunk [r*cs, (r+1)*cs), keeps its keys in its own shared
// memory, and the cluster shares histograms through distributed shared
// memory.  Chunks are in ID order, so the cluster prefix of a CTA's
// survivors is its place in ID order.  Synchronisation per call: one bounded
// grid barrier (the cross-head count exchange, with the cluster barrier's
// release/acquire split around it) and two cluster barriers.
namespace cg = cooperative_groups;
constexpr int kCluster = 4;       // CTAs per head in the layer step's selector
constexpr int kBatchCluster = 2;  // CTAs per head in record mode (shard steps), see the batch kernel
constexpr int kCThreads = 512;
constexpr int kCWarps = kCThreads / 32;
constexpr unsigned long long kClusterKeysMax = 65536;           // valid tokens per head on this path
constexpr unsigned long long kCChunkMax = kClusterKeysMax / kCluster;

template <int C>
struct ClusterShared {
    unsigned int hist[kCWarps][256];  // leader: LSD sort offsets
    unsigned int coarse[1024];        // histogram of key >> 6 over this CTA's chunk
    unsigned int fine[64];            // key & 63 inside the chosen coarse bin, this chunk
    unsigned int scan[32];
    unsigned int red[kCWarps][C];
    unsigned int maxkey, bad0, cnt, bad;
    unsigned int b_bin, b_above, b_eqtotal, total;
    unsigned int gt_before, eq_before;  // survivors of the cluster's earlier chunks
    unsigned int c_hi;                  // keys of the whole head in the chosen coarse bin
    unsigned int tie_key0, tie_key1;    // direct path, leader: keys at ranks k - 1 and k
    unsigned int last_id, next_id;      // leader: the need_eq-th and next tie of K*
    unsigned int cand_slots;            // leader: direct-path candidates placed so far
    unsigned int sel_ids[32];           // leader: the first 32 ordered ids (the one-tile epilogue)
    unsigned int status, status_index;
    unsigned long long k;
    int timeout;
    // Current position: [head 0 / this head][query row, key row]
    __align__(16) uint16_t cur_row[2][2][kDim];
};

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// ---- gather + attention epilogue of the cluster kernel (layer step).
// Each CTA runs four 128-thread groups; group g of CTA r takes the head's
// 32-slot tiles 4g + r, +16, ...  Per tile a thread owns slot t/4 and the
// channel quarter t%4 of its K/V rows: K goes to the packed layout from
// registers, V is staged for the transposed packed write and P.V, and the
// group folds the tile into an online softmax (thread = output channel).
constexpr int kEpiGroups = 4;
constexpr int kEpiThreads = 128;
constexpr int kEpiPitch = kDim + 8;  // halves per staged V row (16-byte aligned)
// Every member that is accessed with 16-byte vectors starts on a 16-byte
// boundary: rows of vt (272 B), each group (sizeof a multiple of 16), q.
struct __align__(16) EpiGroupSmem {
    uint16_t vt[32][kEpiPitch];
    float wgt[32];
    float stat[4];
};
static_assert(sizeof(EpiGroupSmem) % 16 == 0 && (kEpiPitch * 2) % 16 == 0, "16-byte aligned V staging");
template <int C>
struct __align__(16) EpiSmem {
    EpiGroupSmem g[kEpiGroups];
    __align__(16) float q[4][36];  // the head's query, channel quarters padded apart (distinct banks)
    float part[C * kEpiGroups][kDim + 2];  // leader: every group's (max, sum, out[128])
};
static_assert(offsetof(EpiSmem<kCluster>, q) % 16 == 0, "16-byte aligned query");
template <int C>
constexpr size_t epi_smem_bytes() {
    return (sizeof(EpiSmem<C>) + 15) / 16 * 16;
}

__device__ __forceinline__ void group_sync(int id) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kEpiThreads) : "memory");
}

// One 32-slot tile of head h into the group's running (M, L, acc).
template <bool kSharedIds>
__device__ __forceinline__ void epilogue_tile(const SelectEpilogue& e, const uint32_t* ids, int h, unsigned s0,
                                              int live, const float* qs, EpiGroupSmem& gs, int gtid, int bar,
                                              float& M, float& L, float& acc) {
    const int slot = gtid >> 2, qd = gtid & 3, kh = h >> 2;
    uint4 kr[4], vr[4];
    if (slot < live) {
        // written by the leader CTA: its own shared copy, or global memory
        const uint32_t id = kSharedIds ? ids[s0 + slot] : __ldcg(ids + s0 + slot);
        const uint4* ks = reinterpret_cast<const uint4*>(e.kcache + (size_t)id * e.stride_words + kh * kDim) + qd * 4;
        const uint4* vs = reinterpret_cast<const uint4*>(e.vcache + (size_t)id * e.stride_words + kh * kDim) + qd * 4;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            kr[u] = __ldg(ks + u);
            vr[u] = __ldg(vs + u);
        }
        uint4* kd = reinterpret_cast<uint4*>(e.kp + ((size_t)(s0 + slot) * e.heads + h) * kDim) + qd * 4;
#pragma unroll
        for (int u = 0; u < 4; ++u) kd[u] = kr[u];
    } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) kr[u] = vr[u] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4*>(&gs.vt[slot][qd * 32 + u * 8]) = vr[u];
    float dot = 0.0f;
    const float4* q4 = reinterpret_cast<const float4*>(qs + qd * 36);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint32_t w[4] = {kr[u].x, kr[u].y, kr[u].z, kr[u].w};
        const float4 qa = q4[2 * u], qb = q4[2 * u + 1];
        const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            dot = fmaf(f.x, qv[2 * j], dot);
            dot = fmaf(f.y, qv[2 * j + 1], dot);
        }
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    if (qd == 0) gs.wgt[slot] = slot < live ? dot * e.scale : -INFINITY;
    group_sync(bar);
    if (gtid < 32) {
        const float x = gs.wgt[gtid];
        const float mt = warp_max(x);
        const float ex = gtid < live ? expf(x - mt) : 0.0f;
        gs.wgt[gtid] = ex;
        const float lt = warp_sum(ex);
        if (gtid == 0) {
            gs.stat[0] = mt;
            gs.stat[1] = lt;
        }
    }
    group_sync(bar);
    const int d = gtid;
    float acc_t = 0.0f;
#pragma unroll 8
    for (int t = 0; t < 32; ++t) acc_t = fmaf(gs.wgt[t], half_value(gs.vt[t][d]), acc_t);
    uint16_t* vrow = e.vp + ((size_t)h * kDim + d) * e.count + s0;
    if (live == 32 && (e.count & 7) == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[j] = (uint32_t)gs.vt[8 * u + 2 * j][d] | ((uint32_t)gs.vt[8 * u + 2 * j + 1][d] << 16);
            reinterpret_cast<uint4*>(vrow)[u] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    } else {
        for (int t = 0; t < live; ++t) vrow[t] = gs.vt[t][d];
    }
    const float mt = gs.stat[0], lt = gs.stat[1];
    const float mn = fmaxf(M, mt);
    const float a = expf(M - mn), b = expf(mt - mn);  // M = -inf on the first tile: a = 0
    acc = fmaf(acc, a, acc_t * b);
    L = fmaf(L, a, lt * b);
    M = mn;
    group_sync(bar);  // vt / wgt / stat are rewritten by the next tile
}

__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The fold of warp 0 of a selector CTA: the per-head counts (4 heads per
// lane; from the grid barrier's words, or from the exchanged records in
// record mode), each rounded to F16 (or kept in F32), the first failing head
// in head order (non-finite before count overflow within a head), and k from
// the F16 mean and the ratio cap.  The rounded counts are integers below
// 2^16 and there are at most 128 of them, so every partial sum is an integer
// below 2^24 and exact in FP32: the tree sum equals the reference's
// sequential FP32 sum (gqa_policy.cpp:60) bit for bit.
struct CountFold {
    unsigned long long k;
    unsigned int status, index;
    uint32_t own;  // this CTA's head's count
};
__device__ __forceinline__ CountFold fold_counts(const SelectParams& p, uint32_t seqb, uint32_t h,
                                                 unsigned long long n, const unsigned long long word[4],
                                                 int timeout) {
    const int lane = threadIdx.x & 31;
    const bool ext = p.ext != nullptr;
    const uint32_t nh = ext ? p.heads_total : p.heads, own_head = ext ? p.head_base + h : h;
    unsigned int e[4] = {0, 0, 0, 0};
    float rr[4] = {0.f, 0.f, 0.f, 0.f};
    unsigned long long own = 0;
    if (!timeout) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t hh = lane * 4 + j;
            if (hh < nh) {
                unsigned long long c;
                uint32_t nonfinite;
                if (ext) {
                    const uint32_t rec = __ldg(p.ext + seqb * p.heads_total + hh);
                    c = rec & 0x7fffffffu;
                    nonfinite = rec >> 31;
                } else {
                    c = word[j] >> 16;
                    nonfinite = ((word[j] >> 8) & 255ull) ? 1u : 0u;
                }
                if (p.cover) c += 1;  // at most one newly appended current token
                const float rounded = p.fp32_counts ? (float)c : half_value(half_bits((float)c));
                e[j] = nonfinite | (isfinite(rounded) ? 0u : 2u);
                rr[j] = rounded;
                if (hh == own_head) own = c;
            }
        }
    }
    CountFold f{};
    f.own = __reduce_max_sync(0xffffffffu, (unsigned int)own);
    unsigned int my_status = 0, my_index = 0;
#pragma unroll
    for (int j = 3; j >= 0; --j) {
        if (e[j]) {
            my_status = (e[j] & 1u) ? HSB_E_SEL_NONFINITE : (p.cover ? HSB_E_COVER_COUNT : HSB_E_SEL_COUNT_F16);
            my_index = lane * 4 + j;
        }
    }
    const unsigned int failing = __ballot_sync(0xffffffffu, my_status != 0);
    if (failing) {
        const int src = __ffs(failing) - 1;
        f.status = __shfl_sync(0xffffffffu, my_status, src);
        f.index = __shfl_sync(0xffffffffu, my_index, src);
    }
    float total = (rr[0] + rr[1]) + (rr[2] + rr[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (!timeout && !f.status) {
        const float mean = p.fp32_counts ? __fdiv_rn(total, (float)nh)
                                         : half_value(half_bits(__fdiv_rn(total, (float)nh)));
        if (p.cover) {
            if (!(isfinite(mean) && mean >= 1.0f)) f.status = HSB_E_COVER_MEAN;
            else f.k = min(p.cover_cap, (unsigned long long)mean);
        } else {
            if (!isfinite(mean)) f.status = HSB_E_SEL_MEAN_F16;
            else {
                const unsigned long long cap = (unsigned long long)floor((double)n * (double)p.ratio);
                f.k = min((unsigned long long)mean, min(cap, n));
            }
        }
    }
    return f;
}

// The cluster selector's body, shared by its two launch shapes below; C is
// the cluster size (CTAs per head).
template <int C>
__device__ __forceinline__ void select_cluster_body(const SelectParams& p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ ClusterShared<C> sh;
    cg::cluster_group cl = cg::this_cluster();
    const unsigned int r = cl.block_rank();
    const uint32_t h = (blockIdx.x / C) % p.heads;
    const uint32_t seqb = blockIdx.x / (C * p.heads);  // sequence of the batch
    const bool seq_first = blockIdx.x % (C * p.heads) == 0;  // first CTA of the sequence
    const uint16_t* scores = p.scores + seqb * p.seq_scores;
    hsb_selection* result = p.result + seqb;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The epilogue's query channel, loaded now: its latency hides behind the
    // selection instead of following it.
    const float q_own = (p.ga.out && tid < kDim) ? p.ga.q[((size_t)seqb * p.heads + h) * kDim + tid] : 0.0f;
    const unsigned long long n = p.valid;
    const unsigned long long cs = ((n + C - 1) / C + 7) / 8 * 8;
    const unsigned long long b0 = min(n, (unsigned long long)r * cs), b1 = min(n, b0 + cs);
    const unsigned int m = (unsigned int)(b1 - b0);
    uint16_t* keys = reinterpret_cast<uint16_t*>(dyn);  // [cs] this chunk's keys
    unsigned long long* bufA = reinterpret_cast<unsigned long long*>(dyn + (cs * 2 + 15) / 16 * 16);
    unsigned long long* bufB = bufA + kSmemSortMax;
    const uint16_t* row0 = scores;
    const uint16_t* row = scores + (unsigned long long)h * p.stride;
    // 16-byte loads when rows are 16-byte aligned (b0 is a multiple of 8).
    const bool vec = (p.stride % 8 == 0) && ((reinterpret_cast<uintptr_t>(scores) & 15) == 0);
    const unsigned long long n8 = vec ? n / 8 : 0;
    const unsigned int m8 = vec ? m / 8 : 0;

    if (tid == 0) {
        sh.maxkey = 0;
        sh.bad0 = 0;
        sh.cnt = 0;
        sh.bad = 0;
        sh.last_id = 0xffffffffu;
        sh.next_id = 0xffffffffu;
        sh.cand_slots = 0;
    }
    for (int i = tid; i < 1024; i += kCThreads) sh.coarse[i] = 0;
    if (tid < 64) sh.fine[tid] = 0;
    // Record mode (shard steps): k follows from the exchanged records alone,
    // so a sequence whose threshold record carries an error, or which
    // selects nothing, is settled before any of its keys is loaded -- with
    // the same outputs as the full path below.
    if (p.ext != nullptr) {
        const int status0 = (int)p.ext_thr[2 * seqb + 1];
        if (warp == 0 && !status0) {
            const unsigned long long none[4] = {0, 0, 0, 0};
            const CountFold f = fold_counts(p, seqb, h, p.valid, none, 0);
            unsigned int status = f.status;
            if (!status && f.k == 0 && p.zero_is_error) status = HSB_E_ZERO_SELECTION;
            if (lane == 0) {
                sh.k = status ? 0 : f.k;
                sh.status = status;
                sh.status_index = f.index;
                sh.cnt = f.own;
            }
        }
        __syncthreads();
        if (status0 || sh.k == 0) {
            if (status0) {
                if (seq_first && tid == 0) {
                    result->k = 0;
                    result->status.code = status0;
                    result->status.index = 0;
                }
            } else if (tid == 0) {
                if (r == 0 && p.counts) p.counts[seqb * p.heads + h] = sh.cnt;
                if (seq_first && sh.status) raise_status(&result->status, (int)sh.status, (int)sh.status_index);
            }
            if (p.ga.out && r == 0)
                for (int d = tid; d < kDim; d += kCThreads) p.ga.out[(seqb * p.heads + h) * kDim + d] = 0.0f;
            return;  // the whole cluster takes this branch (one k per sequence)
        }
        if (tid == 0) sh.cnt = 0;
    }
    __syncthreads();

    // ---- 1. head-0 maximum over the whole row (every CTA, from L2), own
    // chunk's keys to shared memory with the coarse histogram.
    unsigned int mx = 0, bad0 = 0, bad = 0;
    const bool ext = p.ext != nullptr;
    // Phase 1's global loads go out together, one round trip rather than a
    // chain: the chunk's first kPreW 16-byte words of keys per thread and, in
    // the layer step, the two head-0 partials per thread.
    static_assert(kH0Partials == 2 * kCThreads, "two head-0 partials per thread");
    // Words of keys per thread loaded up front: a 32768-key row's whole chunk.
    constexpr int kPreW = 8 / C;
    uint4 kw[kPreW];
#pragma unroll
    for (int u = 0; u < kPreW; ++u) kw[u] = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < kPreW; ++u)
        if (tid + u * kCThreads < m8) kw[u] = reinterpret_cast<const uint4*>(row + b0)[tid + u * kCThreads];
    // Current position (select after a prepared history): two warps stage
    // a query row and the position's key row, and their lane 0 scores it in
    // the scorer's order (channels 0..127, F32 from +0, one F16 rounding) --
    // head 0 for the threshold in every CTA, and this CTA's head in the CTA
    // whose chunk holds the position.  The key loads above are in flight
    // meanwhile.
    const bool cur_mode = p.cur_k != nullptr;
    const unsigned long long cur = n - 1;
    const bool own_cur = cur_mode && cur >= b0 && cur < b1;
    const unsigned int cur_local = own_cur ? (unsigned int)(cur - b0) : 0xffffffffu;
    const int cur_slot = !cur_mode ? -1 : warp == kCWarps - 1 ? 0 : (warp == kCWarps - 2 && own_cur) ? 1 : -1;
    uint32_t cur_key = 0;
    if (cur_slot >= 0) {
        const uint32_t qh = cur_slot == 0 ? 0u : h;
        const uint4 v = lane < 16 ? reinterpret_cast<const uint4*>(p.cur_q + (size_t)qh * kDim)[lane]
                                  : reinterpret_cast<const uint4*>(p.cur_k + (size_t)(qh / kGroup) * kDim)[lane - 16];
        reinterpret_cast<uint4*>(&sh.cur_row[cur_slot][0][0])[lane] = v;
        __syncwarp();
        if (lane == 0) {
            const uint16_t* qs = sh.cur_row[cur_slot][0];
            const uint16_t* ks = sh.cur_row[cur_slot][1];
            float acc = 0.0f;
#pragma unroll 16
            for (int c = 0; c < kDim; ++c) acc = fma_f16(qs[c], ks[c], acc);
            const uint16_t raw = half_bits(acc);
            cur_key = order_key(scale_half(raw));
            if (cur_slot == 1) p.cur_raw[(size_t)h * p.stride + cur] = raw;
        }
    }
    // Shard steps: the threshold record's status (written by the preceding grid).
    const int ext_status = ext ? (int)p.ext_thr[2 * seqb + 1] : 0;
    if (p.h0 && !ext) {
        const uint32_t v0 = __ldcg(p.h0 + tid), v1 = __ldcg(p.h0 + tid + kCThreads);
        mx = max(v0 & 0xffffu, v1 & 0xffffu);
        bad0 = (v0 | v1) >> 16;
    }
#pragma unroll 4
    for (unsigned long long g = tid; g < ((p.h0 || ext) ? 0 : n8); g += kCThreads) {
        const uint4 w = reinterpret_cast<const uint4*>(row0)[g];
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t key = to_key((v[j >> 1] >> (16 * (j & 1))) & 0xffffu, p.mode);
            bad0 |= key_nonfinite(key);
            mx = key_nan(key) ? mx : max(mx, key);
        }
    }
    for (unsigned long long i = n8 * 8 + tid; i < ((p.h0 || ext) ? 0 : n); i += kCThreads) {
        const uint32_t key = to_key(row0[i], p.mode);
        bad0 |= key_nonfinite(key);
        mx = key_nan(key) ? mx : max(mx, key);
    }
    // One 16-byte word of keys: coarse histogram, order keys to shared memory.
    // The current position's slot (not written by the history scorer) is
    // skipped here and filled below.
    auto take = [&](const uint4 w, unsigned int g) {
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
        uint32_t k2[4];
        const unsigned int skip = (g == (cur_local >> 3)) ? (cur_local & 7u) : 8u;
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const uint32_t a = to_key(v[j >> 1] & 0xffffu, p.mode), b = to_key(v[j >> 1] >> 16, p.mode);
            if ((unsigned)j != skip) {
                bad |= key_nonfinite(a);
                atomicAdd(&sh.coarse[a >> 6], 1u);
            }
            if ((unsigned)j + 1 != skip) {
                bad |= key_nonfinite(b);
                atomicAdd(&sh.coarse[b >> 6], 1u);
            }
            k2[j >> 1] = a | (b << 16);
        }
        reinterpret_cast<uint4*>(keys)[g] = make_uint4(k2[0], k2[1], k2[2], k2[3]);
    };
#pragma unroll
    for (int u = 0; u < kPreW; ++u)
        if (tid + u * kCThreads < m8) take(kw[u], tid + u * kCThreads);
    for (unsigned int g = tid + kPreW * kCThreads; g < m8; g += kCThreads)
        take(reinterpret_cast<const uint4*>(row + b0)[g], g);
    for (unsigned int i = m8 * 8 + tid; i < m; i += kCThreads) {
        if (i == cur_local) continue;
        const uint32_t key = to_key(row[b0 + i], p.mode);
        bad |= key_nonfinite(key);
        atomicAdd(&sh.coarse[key >> 6], 1u);
        keys[i] = (uint16_t)key;
    }
    if (cur_slot == 0 && lane == 0) {  // the current position joins head 0's maximum
        bad0 |= key_nonfinite(cur_key);
        mx = key_nan(cur_key) ? mx : max(mx, cur_key);
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    bad0 = __any_sync(0xffffffffu, bad0);
    if (lane == 0) {
        atomicMax(&sh.maxkey, mx);
        if (bad0) atomicOr(&sh.bad0, 1u);
    }
    __syncthreads();
    const float maximum = half_value((uint16_t)key_bits(sh.maxkey));
    const float threshold = half_value(half_bits(sh.maxkey ? maximum - p.alpha : -INFINITY));
    const bool head0_bad = !ext && !p.cover && sh.bad0;
    const bool thr_bad = !ext && !isfinite(threshold);
    if (head0_bad || thr_bad || ext_status) {
        if (seq_first && tid == 0) {
            result->k = 0;
            result->status.code = ext_status ? ext_status
                                  : head0_bad ? HSB_E_SEL_NONFINITE_HEAD0
                                              : (p.cover ? HSB_E_COVER_THRESHOLD : HSB_E_SEL_THRESHOLD);
            result->status.index = 0;
        }
        if (p.ga.out && r == 0)  // the layer's output stays zero
            for (int d = tid; d < kDim; d += kCThreads) p.ga.out[(seqb * p.heads + h) * kDim + d] = 0.0f;
        return;  // every CTA of the grid takes this branch; nothing is pending
    }
    const unsigned int thr_key = order_key(half_bits(threshold));
    if (cur_mode) {  // the current position's key joins this chunk (after every take() store)
        if (cur_slot == 1 && lane == 0) {
            bad |= key_nonfinite(cur_key);
            atomicAdd(&sh.coarse[cur_key >> 6], 1u);
            keys[cur_local] = (uint16_t)cur_key;
        }
        __syncthreads();
    }
    unsigned int cnt = 0;
    for (unsigned int i = tid; i < (ext ? 0u : m); i += kCThreads) {
        const unsigned int key = keys[i];
        cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        if (cnt) atomicAdd(&sh.cnt, cnt);
        if (bad) atomicOr(&sh.bad, 1u);
    }
    __syncthreads();
    // The coarse histograms are complete: release them to the cluster now,
    // acquire after the grid barrier.
    cluster_arrive_release();
    if (warp == 0) {
        // ---- 2. grid barrier (bounded): lane 0 adds this CTA's record to its
        // head's word (one atomic: count, non-finite flag, arrival); lane j
        // polls heads 4j .. 4j + 3 until each has all its CTAs' records, and
        // the words it read are the counts (no second read, no fence: the
        // data is the atomic itself).
        int timeout = 0;
        const uint32_t nh = ext ? p.heads_total : p.heads;
        unsigned long long word[4] = {0, 0, 0, 0};
        if (!ext) {
            if (lane == 0)
                atomicAdd(&p.header->hc[h], ((unsigned long long)sh.cnt << 16) |
                                                ((!p.cover && sh.bad) ? 256ull : 0ull) | 1ull);
            const unsigned long long start = global_ns();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t hh = lane * 4 + j;
                if (hh >= nh || timeout) continue;
                unsigned long long w;
                while (((w = ld_relaxed_u64(&p.header->hc[hh])) & 255ull) < (unsigned long long)C) {
                    if (global_ns() - start > kWaitLimitNs) {
                        timeout = 1;
                        break;
                    }
                }
                word[j] = w;
            }
        }
        timeout = __any_sync(0xffffffffu, timeout);
        if (lane == 0) sh.timeout = timeout;
        const CountFold f = fold_counts(p, seqb, h, n, word, timeout);
        const unsigned long long own = f.own, k = f.k;
        unsigned int status = f.status, index = f.index;
        if (r == 0 && lane == 0 && p.counts && !timeout) p.counts[seqb * p.heads + h] = (uint32_t)own;
        if (timeout) status = HSB_E_TIMEOUT;
        if (!status && k == 0 && p.zero_is_error) status = HSB_E_ZERO_SELECTION;
        if (lane == 0) {
            sh.status = status;
            sh.status_index = index;
            sh.k = status ? 0 : k;
            // *result starts zeroed (the launcher clears it).
            if (seq_first) result->k = status ? 0u : (uint32_t)k;
            if (timeout) raise_status(&result->status, HSB_E_TIMEOUT, (int)blockIdx.x);
            else if (seq_first && status) raise_status(&result->status, (int)status, (int)index);
        }
    }
    __syncthreads();
    cluster_wait_acquire();  // every chunk's coarse histogram is visible (arrived before the barrier)
    const bool fused = p.ga.out != nullptr;
    if (sh.timeout) {
        // Cluster peers that passed the barrier may still read this CTA's
        // shared memory: stay resident through as many cluster barriers as
        // any of their paths takes (extra ones complete once they exit).
        for (int i = 0; i < (fused ? 4 : 2); ++i) cl.sync();
        return;
    }
    const unsigned long long k = sh.k;
    if (k == 0) {  // the same k in every CTA that passed the barrier
        if (fused && r == 0)
            for (int d = tid; d < kDim; d += kCThreads) p.ga.out[(seqb * p.heads + h) * kDim + d] = 0.0f;
        return;
    }

    uint32_t* out = p.ids + ((unsigned long long)seqb * p.heads + h) * p.kcap;
    // ---- 3. radix select over the cluster's histograms.  Thread t owns
    // coarse bins 1023 - 2t and 1022 - 2t (descending).
    const unsigned int bin0 = 1023u - 2u * tid, bin1 = bin0 - 1u;
    unsigned int cq0[C], cq1[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
        const unsigned int* rc = cl.map_shared_rank(&sh.coarse[0], q);
        cq0[q] = rc[bin0];
        cq1[q] = rc[bin1];
    }
    unsigned int c0 = 0, c1 = 0;
#pragma unroll
    for (int q = 0; q < C; ++q) {
        c0 += cq0[q];
        c1 += cq1[q];
    }
    {
        const unsigned int above = block_exclusive_scan<kCThreads>(c0 + c1, sh.scan, &sh.total);
        if (above < k && above + c0 >= k) {
            sh.b_bin = bin0;
            sh.b_above = above;
            sh.c_hi = c0;
        } else if (above + c0 < k && above + c0 + c1 >= k) {
            sh.b_bin = bin1;
            sh.b_above = above + c0;
            sh.c_hi = c1;
        }
    }
    __syncthreads();
    const unsigned int hi = sh.b_bin, above_hi = sh.b_above;
    // Direct path: when the keys of bins >= hi fit the leader's buffer they
    // are all candidates, and the leader orders them (no fine pass).
    const bool direct = above_hi + sh.c_hi <= kSmemSortMax;
    // Per-chunk counts of bins > hi (radix path) or >= hi (direct path):
    // the cluster prefix of each chunk.
#pragma unroll
    for (int q = 0; q < C; ++q) {
        const unsigned int lo_bin = direct ? hi : hi + 1;
        unsigned int v = (bin0 >= lo_bin ? cq0[q] : 0u) + (bin1 >= lo_bin ? cq1[q] : 0u);
        v = __reduce_add_sync(0xffffffffu, v);
        if (lane == 0) sh.red[warp][q] = v;
    }
    if (direct) {
        // ---- 3'. the candidates: every key of bins >= hi
        unsigned long long* dst = cl.map_shared_rank(bufA, 0);
        if (above_hi + sh.c_hi <= kRankSortMax) {  // the same in every CTA of the cluster
            // Few candidates: each takes a slot from the leader's counter, in any
            // order (the leader's rank sort orders by key, then ID).
            unsigned int* slot = cl.map_shared_rank(&sh.cand_slots, 0);
            for (unsigned int j = tid * 8; j < m; j += kCThreads * 8) {
                // keys[] holds a multiple of 8 entries: the 16-byte load stays inside
                const uint4 v = *reinterpret_cast<const uint4*>(keys + j);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t key = (w[e >> 1] >> (16 * (e & 1))) & 0xffffu;
                    if (j + e < m && (key >> 6) >= hi)
                        dst[atomicAdd(slot, 1u)] = ((unsigned long long)key << 32) | (unsigned int)(b0 + j + e);
                }
            }
        } else {
            // In ID order: a block scan places each thread's candidates after
            // those of the cluster's earlier chunks.
            __syncthreads();
            unsigned int before = 0;
            for (unsigned int q = 0; q < r; ++q)
                for (int w = 0; w < kCWarps; ++w) before += sh.red[w][q];
            const unsigned int per = ((m + kCThreads - 1) / kCThreads + 7) / 8 * 8;
            const unsigned int j0 = min(m, tid * per), j1 = min(m, j0 + per);
            unsigned int mine = 0;
            for (unsigned int j = j0; j < j1; j += 8) {  // 16-byte loads: no bank conflicts
                uint32_t w[4];
                if (j + 8 <= j1) {
                    const uint4 v = *reinterpret_cast<const uint4*>(keys + j);
                    w[0] = v.x;
                    w[1] = v.y;
                    w[2] = v.z;
                    w[3] = v.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        w[e] = (j + 2 * e < j1 ? keys[j + 2 * e] : 0u) | ((j + 2 * e + 1 < j1 ? keys[j + 2 * e + 1] : 0u) << 16);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    mine += (j + e < j1 && ((w[e >> 1] >> (16 * (e & 1))) & 0xffffu) >> 6 >= hi) ? 1u : 0u;
            }
            unsigned int pos = before + block_exclusive_scan<kCThreads>(mine, sh.scan, &sh.total);
            if (mine) {
                for (unsigned int j = j0; j < j1; ++j) {
                    const unsigned int key = keys[j];
                    if ((key >> 6) >= hi && pos < kSmemSortMax)
                        dst[pos++] = ((unsigned long long)key << 32) | (unsigned int)(b0 + j);
                }
            }
        }
        cl.sync();  // every chunk's candidates are in the leader
        if (r == 0) {
            // Stable order by key descending (ID ascending on ties) of the
            // cand candidates; the first k are the selection.
            const unsigned int cand = min(above_hi + sh.c_hi, kSmemSortMax);
            unsigned long long* src = bufA;
            if (cand <= kRankSortMax) {
                if ((unsigned)tid < cand) {
                    // rank by key descending, ID ascending (unique IDs)
                    const unsigned long long e = src[tid];
                    const unsigned int ek = (unsigned int)(e >> 32), eid = (unsigned int)e;
                    unsigned int rk = 0;
                    for (unsigned int j = 0; j < cand; ++j) {
                        const unsigned long long o = src[j];
                        const unsigned int ok = (unsigned int)(o >> 32);
                        rk += (ok > ek) || (ok == ek && (unsigned int)o < eid);
                    }
                    if (rk < k) out[rk] = (uint32_t)(e & 0xffffffffu);
                    if (rk < 32) sh.sel_ids[rk] = (uint32_t)(e & 0xffffffffu);
                    if (rk + 1 == k) {
                        sh.last_id = (uint32_t)(e & 0xffffffffu);
                        sh.tie_key0 = ek;
                    }
                    if (rk == k) {
                        sh.next_id = (uint32_t)(e & 0xffffffffu);
                        sh.tie_key1 = ek;
                    }
                }
            } else {
                sort_pass<kCThreads>(sh.hist, sh.scan, &sh.total, src, bufB, cand, 0);
                sort_pass<kCThreads>(sh.hist, sh.scan, &sh.total, bufB, src, cand, 8);
                for (unsigned int j = tid; j < k; j += kCThreads) out[j] = (uint32_t)(src[j] & 0xffffffffu);
                if ((unsigned)tid < min(k, 32ull)) sh.sel_ids[tid] = (uint32_t)(src[tid] & 0xffffffffu);
                if (tid == 0) {
                    sh.last_id = (uint32_t)(src[k - 1] & 0xffffffffu);
                    sh.tie_key0 = (uint32_t)(src[k - 1] >> 32);
                    if (k < cand) {
                        sh.next_id = (uint32_t)(src[k] & 0xffffffffu);
                        sh.tie_key1 = (uint32_t)(src[k] >> 32);
                    }
                }
            }
            __syncthreads();
            // Boundary tie (gqa_policy.cpp:66): only a (k+1)-th candidate with
            // the k-th key can tie (keys of lower bins are smaller); equal
            // keys are equal bits except +0 / -0, told apart from the scores.
            if (!p.cover && tid == 0 && k < n && k < cand && sh.last_id < n && sh.next_id < n &&
                sh.tie_key0 == sh.tie_key1) {
                bool tied = true;
                if (sh.tie_key0 == 0x8000u) {
                    const unsigned long long base = (unsigned long long)h * p.stride;
                    uint16_t a, b;
                    if (p.mode == kInputKeys) {
                        const uint16_t* raw = p.tie_raw ? p.tie_raw + seqb * p.seq_scores : nullptr;
                        a = raw ? scale_half(raw[base + sh.last_id]) : 0;
                        b = raw ? scale_half(raw[base + sh.next_id]) : 0;
                    } else {
                        a = scores[base + sh.last_id];
                        b = scores[base + sh.next_id];
                        if (p.mode == kInputRaw) {
                            a = scale_half(a);
                            b = scale_half(b);
                        }
                    }
                    tied = a == b;
                }
                if (tied) atomicAdd(&result->boundary_tied_heads, 1u);
            }
        }
    } else {
    for (unsigned int i = tid; i < m; i += kCThreads) {
        const unsigned int key = keys[i];
        if ((key >> 6) == hi) atomicAdd(&sh.fine[key & 63u], 1u);
    }
    cl.sync();  // every chunk's fine histogram is complete
    if (warp == 0) {  // 64 fine bins, two per lane, descending
        unsigned int f0[C], f1[C], s0 = 0, s1 = 0;
#pragma unroll
        for (int q = 0; q < C; ++q) {
            const unsigned int* rf = cl.map_shared_rank(&sh.fine[0], q);
            f0[q] = rf[63 - 2 * lane];
            f1[q] = rf[62 - 2 * lane];
            s0 += f0[q];
            s1 += f1[q];
        }
        unsigned int x = s0 + s1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        const unsigned int need = (unsigned int)k - above_hi;
        unsigned int above = x - s0 - s1;
        int found = -1;
        unsigned int f_above = 0, f_eq = 0;
        if (above < need && above + s0 >= need) {
            found = 63 - 2 * lane;
            f_above = above;
            f_eq = s0;
        } else if (above + s0 < need && above + s0 + s1 >= need) {
            found = 62 - 2 * lane;
            f_above = above + s0;
            f_eq = s1;
        }
        const unsigned int who = __ballot_sync(0xffffffffu, found >= 0);
        const int src = __ffs(who) - 1;  // exactly one lane holds the bin
        const int b2 = __shfl_sync(0xffffffffu, found, src);
        f_above = __shfl_sync(0xffffffffu, f_above, src);
        f_eq = __shfl_sync(0xffffffffu, f_eq, src);
        // Per-chunk gt / eq counts of K* = (hi << 6) | b2, then the prefix of
        // the chunks before this CTA.
        unsigned int gt_before = 0, eq_before = 0;
#pragma unroll
        for (int q = 0; q < C; ++q) {
            unsigned int g = ((63 - 2 * lane) > b2 ? f0[q] : 0u) + ((62 - 2 * lane) > b2 ? f1[q] : 0u);
            unsigned int eq = ((63 - 2 * lane) == b2 ? f0[q] : 0u) + ((62 - 2 * lane) == b2 ? f1[q] : 0u);
            g = __reduce_add_sync(0xffffffffu, g);
            eq = __reduce_add_sync(0xffffffffu, eq);
            unsigned int cg_above = 0;
            for (int w = 0; w < kCWarps; ++w) cg_above += sh.red[w][q];
            if ((unsigned int)q < r) {
                gt_before += g + cg_above;
                eq_before += eq;
            }
        }
        if (lane == 0) {
            sh.b_bin = (unsigned int)b2;
            sh.b_above = f_above;
            sh.b_eqtotal = f_eq;
            sh.gt_before = gt_before;
            sh.eq_before = eq_before;
        }
    }
    __syncthreads();
    const unsigned int kstar = (hi << 6) | sh.b_bin;
    const unsigned int gt = above_hi + sh.b_above;
    const unsigned int need_eq = (unsigned int)k - gt;  // >= 1
    const unsigned int eq_total = sh.b_eqtotal;

    // ---- 4. ordered compaction of this chunk into the leader's buffer (or
    // the head's workspace buffer when k exceeds it)
    const bool small = k <= kSmemSortMax;
    unsigned long long* sortbuf = p.sortbuf + ((unsigned long long)seqb * p.heads + h) * 2 * p.kcap;
    unsigned long long* dst = small ? cl.map_shared_rank(bufA, 0) : sortbuf;
    ClusterShared<C>* lead = cl.map_shared_rank(&sh, 0);
    // Thread t owns keys [t*per, t*per + per) of the chunk (ID order follows
    // thread order); one block scan of (gt << 16 | eq) places its survivors.
    const unsigned int per = ((m + kCThreads - 1) / kCThreads + 7) / 8 * 8;
    const unsigned int j0 = min(m, tid * per), j1 = min(m, j0 + per);
    unsigned int n_gt = 0, n_eq = 0;
    for (unsigned int j = j0; j < j1; j += 8) {
        uint32_t w[4];
        if (j + 8 <= j1) {
            const uint4 v = *reinterpret_cast<const uint4*>(keys + j);
            w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t lo = j + 2 * e < j1 ? keys[j + 2 * e] : 0u;
                const uint32_t hi16 = j + 2 * e + 1 < j1 ? keys[j + 2 * e + 1] : 0u;
                w[e] = lo | (hi16 << 16);  // positions past j1 are masked below
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const bool in = j + e < j1;
            const uint32_t key = (w[e >> 1] >> (16 * (e & 1))) & 0xffffu;
            n_gt += (in && key > kstar) ? 1u : 0u;
            n_eq += (in && key == kstar) ? 1u : 0u;
        }
    }
    const unsigned int excl = block_exclusive_scan<kCThreads>((n_gt << 16) | n_eq, sh.scan, &sh.total);
    if (n_gt | n_eq) {
        unsigned int gt_run = sh.gt_before + (excl >> 16), eq_run = sh.eq_before + (excl & 0xffffu);
        for (unsigned int j = j0; j < j1; ++j) {
            const unsigned int key = keys[j];
            const unsigned int id = (unsigned int)(b0 + j);
            if (key > kstar) {
                const unsigned int at = gt_run + min(eq_run, need_eq);
                if (at < k) dst[at] = ((unsigned long long)key << 32) | id;
                ++gt_run;
            } else if (key == kstar) {
                if (eq_run < need_eq) {
                    const unsigned int at = gt_run + eq_run;
                    if (at < k) dst[at] = ((unsigned long long)key << 32) | id;
                }
                if (eq_run + 1 == need_eq) lead->last_id = id;
                if (eq_run == need_eq) lead->next_id = id;
                ++eq_run;
            }
        }
    }
    cl.sync();  // survivors and tie witnesses are in the leader
    if (r == 0) {
        // ---- leader: boundary tie (gqa_policy.cpp:66) and reference order
        unsigned long long* src = small ? bufA : sortbuf;
        unsigned long long* tmp = small ? bufB : src + p.kcap;
        if (!p.cover && tid == 0 && k < n && eq_total > need_eq && sh.last_id < n && sh.next_id < n) {
            bool tied = true;
            if (kstar == 0x8000u) {
                const unsigned long long base = (unsigned long long)h * p.stride;
                uint16_t a, b;
                if (p.mode == kInputKeys) {
                    const uint16_t* raw = p.tie_raw ? p.tie_raw + seqb * p.seq_scores : nullptr;
                    a = raw ? scale_half(raw[base + sh.last_id]) : 0;
                    b = raw ? scale_half(raw[base + sh.next_id]) : 0;
                } else {
                    a = scores[base + sh.last_id];
                    b = scores[base + sh.next_id];
                    if (p.mode == kInputRaw) {
                        a = scale_half(a);
                        b = scale_half(b);
                    }
                }
                tied = a == b;
            }
            if (tied) atomicAdd(&result->boundary_tied_heads, 1u);
        }
        if (k <= kRankSortMax) {
            if ((unsigned)tid < k) {
                const unsigned long long e = src[tid];
                const unsigned int ek = (unsigned int)(e >> 32);
                unsigned int rk = 0;
                for (unsigned int j = 0; j < k; ++j) {
                    const unsigned int ok = (unsigned int)(src[j] >> 32);
                    rk += (ok > ek) || (ok == ek && j < (unsigned)tid);
                }
                if (rk < k) out[rk] = (uint32_t)(e & 0xffffffffu);
                if (rk < 32) sh.sel_ids[rk] = (uint32_t)(e & 0xffffffffu);
            }
        } else {
            sort_pass<kCThreads>(sh.hist, sh.scan, &sh.total, src, tmp, (unsigned int)k, 0);
            sort_pass<kCThreads>(sh.hist, sh.scan, &sh.total, tmp, src, (unsigned int)k, 8);
            for (unsigned int j = tid; j < k; j += kCThreads) out[j] = (uint32_t)(src[j] & 0xffffffffu);
            if ((unsigned)tid < min(k, 32ull)) sh.sel_ids[tid] = (uint32_t)(src[tid] & 0xffffffffu);
        }
    }
    }  // radix path
    if (!fused) return;

    // ---- epilogue: gather the head's selected rows and attend over them
    EpiSmem<C>& es = *reinterpret_cast<EpiSmem<C>*>(dyn);  // keys and sort buffers are no longer needed
    const int grp = tid / kEpiThreads, gtid = tid % kEpiThreads;
    // This sequence's view of the epilogue's buffers.
    SelectEpilogue ga = p.ga;
    ga.q += ((size_t)seqb * p.heads) * kDim;
    ga.out += ((size_t)seqb * p.heads) * kDim;
    ga.kcache += (size_t)seqb * p.valid * ga.stride_words;
    ga.vcache += (size_t)seqb * p.valid * ga.stride_words;
    ga.kp += (size_t)seqb * ga.count * ga.heads * kDim;
    ga.vp += (size_t)seqb * ga.count * ga.heads * kDim;
    if (k <= 32) {
        // One tile: the leader, which has just written the ordered ids,
        // gathers and attends alone; its peers are done.
        if (r != 0) return;
        __syncthreads();  // the sort's reads of the candidate buffers are over
        if (tid < kDim) es.q[tid >> 5][tid & 31] = q_own;
        __syncthreads();  // the ids (sel_ids, written by this CTA) and q are in place
        if (grp == 0) {
            float M = -INFINITY, L = 0.0f, acc = 0.0f;
            epilogue_tile<true>(ga, sh.sel_ids, (int)h, 0u, (int)k, &es.q[0][0], es.g[0], gtid, 1, M, L, acc);
            ga.out[h * kDim + gtid] = L > 0.0f ? acc / L : 0.0f;
        }
        return;
    }
    cl.sync();  // the ordered ids are written (cluster-scope release / acquire)
    if (tid < kDim) es.q[tid >> 5][tid & 31] = q_own;
    __syncthreads();
    float M = -INFINITY, L = 0.0f, acc = 0.0f;
    const unsigned ntiles = (unsigned)((k + 31) / 32);
    // Tile t goes to CTA t % C, group (t / C) % 4: a few tiles spread over SMs first.
    for (unsigned t = grp * C + r; t < ntiles; t += C * kEpiGroups) {
        const unsigned s0 = t * 32;
        epilogue_tile<false>(ga, out, (int)h, s0, (int)min(32ull, k - s0), &es.q[0][0], es.g[grp], gtid, 1 + grp, M,
                             L, acc);
    }
    EpiSmem<C>* lead_es = cl.map_shared_rank(&es, 0);
    float* part = lead_es->part[r * kEpiGroups + grp];
    if (gtid == 0) {
        part[0] = M;
        part[1] = L;
    }
    part[2 + gtid] = acc;
    cl.sync();  // every group's partial is in the leader
    if (r != 0) return;
    if (tid < kDim) {
        float mx = -INFINITY;
        for (int i = 0; i < C * kEpiGroups; ++i) mx = fmaxf(mx, es.part[i][0]);
        float lsum = 0.0f, o = 0.0f;
        for (int i = 0; i < C * kEpiGroups; ++i) {
            const float w = es.part[i][0] == -INFINITY ? 0.0f : expf(es.part[i][0] - mx);
            lsum = fmaf(es.part[i][1], w, lsum);
            o = fmaf(es.part[i][2 + tid], w, o);
        }
        ga.out[h * kDim + tid] = lsum > 0.0f ? o / lsum : 0.0f;
    }
}

// The layer step's selector: one launch of 32 heads (128 CTAs, one per
// SM), so one CTA's latency sets the pace.  80 registers, no spills (a
// two-CTAs-per-SM bound forced 64 and spilled); 512 x 80 registers still
// leave room for one early-resident CTA of the next layer's scorer
// (288 x 72).  Measured 0.7638 -> 0.7543 ms per decode step.
__global__ void __cluster_dims__(kCluster, 1, 1) __maxnreg__(80)
    select_cluster_kernel(const __grid_constant__ SelectParams p) {
    select_cluster_body<kCluster>(p);
}

// Record mode over a batch of sequences (shard steps): no grid barrier and
// many clusters per launch (64 sequences x 32 / W heads x kBatchCluster
// CTAs), so throughput, not one head's latency, sets the pace: two CTAs per
// head instead of four halve the CTAs and cluster barriers per head, and at
// most 64 registers with a 16384-key chunk still give two CTAs per SM.
__global__ void __cluster_dims__(kBatchCluster, 1, 1) __launch_bounds__(kCThreads, 2)
    select_cluster_batch_kernel(const __grid_constant__ SelectParams p) {
    select_cluster_body<kBatchCluster>(p);
}

// ------------------------------------------------------------- shard steps
// The threshold record of a KV-head-sharded step, on the shard that holds
// query head 0: {order key of F16(max - alpha), status}, the status being the
// reference's head-0 / threshold errors (gqa_policy.cpp:50-54).
constexpr int kShardThreads = 256;
__global__ void __launch_bounds__(kShardThreads) shard_threshold_kernel(const uint32_t* h0, float alpha,
                                                                       uint32_t* thr) {
    pdl_wait();
    pdl_trigger();
    h0 += (size_t)blockIdx.x * kH0Partials;  // one CTA per sequence
    thr += 2 * blockIdx.x;
    __shared__ unsigned int smax, sbad;
    if (threadIdx.x == 0) {
        smax = 0;
        sbad = 0;
    }
    __syncthreads();
    unsigned int mx = 0, bad0 = 0;
    head0_from_partials<kShardThreads>(h0, mx, bad0);
    mx = __reduce_max_sync(0xffffffffu, mx);
    bad0 = __reduce_or_sync(0xffffffffu, bad0);
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&smax, mx);
        atomicOr(&sbad, bad0);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float maximum = half_value((uint16_t)key_bits(smax));
        const float threshold = half_value(half_bits(smax ? maximum - alpha : -INFINITY));
        uint32_t status = 0;
        if (sbad) status = HSB_E_SEL_NONFINITE_HEAD0;
        else if (!isfinite(threshold)) status = HSB_E_SEL_THRESHOLD;
        thr[0] = status ? 0u : order_key(half_bits(threshold));
        thr[1] = status;
    }
}

// Count record of one of the shard's heads: #{keys >= threshold key} (NaN
// never counts) | (any non-finite score) << 31.  One CTA per head.
constexpr int kCountThreads = 1024;
__global__ void __launch_bounds__(kCountThreads) shard_count_kernel(const uint16_t* keys, unsigned long long tokens,
                                                                   unsigned heads, const uint32_t* thr,
                                                                   uint32_t* records) {
    pdl_wait();
    pdl_trigger();
    thr += 2 * (blockIdx.x / heads);  // CTA = (sequence, head), keys [batch][heads][tokens]
    __shared__ unsigned int scnt, sbad;
    if (threadIdx.x == 0) {
        scnt = 0;
        sbad = 0;
    }
    __syncthreads();
    const unsigned int thr_key = __ldcg(thr);
    const uint16_t* row = keys + (unsigned long long)blockIdx.x * tokens;
    const bool vec = tokens % 8 == 0 && (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
    const unsigned long long n8 = vec ? tokens / 8 : 0;
    unsigned int cnt = 0, bad = 0;
    for (unsigned long long g = threadIdx.x; g < n8; g += kCountThreads) {
        const uint4 w = reinterpret_cast<const uint4*>(row)[g];
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t key = (v[j >> 1] >> (16 * (j & 1))) & 0xffffu;
            bad |= key_nonfinite(key);
            cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
        }
    }
    for (unsigned long long i = n8 * 8 + threadIdx.x; i < tokens; i += kCountThreads) {
        const uint32_t key = row[i];
        bad |= key_nonfinite(key);
        cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    bad = __any_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0) {
        if (cnt) atomicAdd(&scnt, cnt);
        if (bad) atomicOr(&sbad, 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) records[blockIdx.x] = scnt | (sbad << 31);
}

// Heads (clusters of kCluster CTAs) the cluster path can hold resident at
// once on a device, at its largest shared-memory size; 0 if unavailable.
// Computed once per device (with that device current).
int cluster_capacity(int device) {
    static std::mutex mu;
    static int cap[64];
    static bool known[64] = {};
    if (device < 0 || device >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!known[device]) {
        int c = 0;
        const int smem = (int)(kCChunkMax * 2 + 2 * kSmemSortMax * 8);
        const int smem_batch = (int)(kClusterKeysMax / kBatchCluster * 2 + 2 * kSmemSortMax * 8);
        if (cudaFuncSetAttribute(select_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
                cudaSuccess &&
            cudaFuncSetAttribute(select_cluster_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem_batch) == cudaSuccess) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(kCluster * 32);
            cfg.blockDim = dim3(kCThreads);
            cfg.dynamicSmemBytes = smem;
            if (cudaOccupancyMaxActiveClusters(&c, select_cluster_kernel, &cfg) != cudaSuccess) c = 0;
        }
        (void)cudaGetLastError();
        cap[device] = c;
        known[device] = true;
    }
    return cap[device];
}

}  // namespace

size_t select_header_bytes() { return sizeof(SelectHeader); }

cudaError_t launch_shard_threshold(const uint32_t* h0, size_t batch, float alpha, uint32_t* thr,
                                   cudaStream_t stream) {
    return launch_dependent(shard_threshold_kernel, dim3((unsigned)batch), dim3(kShardThreads), 0, stream, false, h0,
                            alpha, thr);
}

cudaError_t launch_shard_count(const uint16_t* keys, size_t heads, size_t tokens, size_t batch, const uint32_t* thr,
                               uint32_t* records, cudaStream_t stream) {
    return launch_dependent(shard_count_kernel, dim3((unsigned)(heads * batch)), dim3(kCountThreads), 0, stream, false,
                            keys, (unsigned long long)tokens, (unsigned)heads, thr, records);
}

bool select_cluster_available(size_t valid) {
    return valid <= kClusterKeysMax && cluster_capacity(device_info().ordinal) > 0;
}

size_t select_workspace_bytes(size_t heads, size_t valid, size_t kcap) {
    size_t bytes = (sizeof(SelectHeader) + 255) / 256 * 256;
    if (valid > kSmemKeysMax) bytes += (heads * valid * 2 + 255) / 256 * 256;
    bytes += heads * 2 * kcap * 8;
    return bytes;
}

cudaError_t launch_select(const SelectLaunch& s, cudaStream_t stream) {
    const DeviceInfo& dev = device_info();
    SelectParams p{};
    p.scores = s.scores;
    p.tie_raw = s.tie_raw;
    p.mode = s.keys ? kInputKeys : (s.raw ? kInputRaw : kInputScaled);
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
    p.h0 = s.h0;
    p.ga = s.ga;
    p.ext = s.ext;
    p.ext_thr = s.ext_thr;
    p.head_base = s.head_base;
    p.heads_total = s.ext ? s.heads_total : s.heads;
    p.batch = s.batch ? s.batch : 1;
    p.seq_scores = s.seq_scores;
    p.cur_q = s.cur_q;
    p.cur_k = s.cur_k;
    p.cur_raw = s.cur_raw;
    if (s.cur_k && !(s.keys && s.h0 && !s.ext && p.batch == 1 && s.valid >= 2 &&
                     s.valid <= kClusterKeysMax && s.heads <= (uint32_t)cluster_capacity(dev.ordinal)))
        return cudaErrorInvalidValue;  // the current position is scored by the cluster kernel only
    if (s.ga_done) *s.ga_done = 0;
    cudaError_t e = cudaSuccess;
    if (s.reset_header) {
        e = cudaMemsetAsync(ws, 0, sizeof(SelectHeader), stream);
        if (e != cudaSuccess) return e;
    }
    if (s.reset_result) {
        e = cudaMemsetAsync(s.result, 0, sizeof(hsb_selection), stream);
        if (e != cudaSuccess) return e;
    }
    // Cooperative (the grid barrier needs every CTA resident).  Measured
    // slower with programmatic stream serialization on this launch, so the
    // selector starts only once the scorer has completed; it still lets its
    // own dependents start early (pdl_trigger).
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cudaLaunchConfig_t cfg{};
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int capacity = cluster_capacity(dev.ordinal);  // also configures the cluster kernel
    if (s.valid <= kClusterKeysMax && (s.ext || s.heads <= (uint32_t)capacity)) {
        const int csize = s.ext ? kBatchCluster : kCluster;
        const size_t cs = ((size_t)s.valid + csize - 1) / csize;
        cfg.gridDim = dim3(p.batch * s.heads * csize);
        // Shard steps (records from the exchange) have no grid barrier, so a
        // batch of any size needs no co-residency: an ordinary cluster launch.
        if (s.ext || !s.cooperative) cfg.numAttrs = 0;
        cfg.blockDim = dim3(kCThreads);
        cfg.dynamicSmemBytes = ((cs + 7) / 8 * 8 * 2 + 15) / 16 * 16 + 2 * kSmemSortMax * 8;
        if (s.ga.out)
            cfg.dynamicSmemBytes = std::max(cfg.dynamicSmemBytes,
                                            s.ext ? epi_smem_bytes<kBatchCluster>() : epi_smem_bytes<kCluster>());
        const cudaError_t le = s.ext ? cudaLaunchKernelEx(&cfg, select_cluster_batch_kernel, p)
                                     : cudaLaunchKernelEx(&cfg, select_cluster_kernel, p);
        if (le == cudaSuccess && s.ga_done) *s.ga_done = s.ga.out != nullptr;
        return le;
    }
    if (s.ext) return cudaErrorInvalidValue;  // shard steps need the cluster kernel
    p.ga = SelectEpilogue{};  // the one-CTA-per-head kernel has no epilogue
    const size_t keys_bytes = s.valid <= kSmemKeysMax ? ((size_t)s.valid * 2 + 15) / 16 * 16 : 0;
    static thread_local int configured_device = -1;
    if (configured_device != dev.ordinal) {
        e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kSmemKeysMax * 2 + 2 * kSmemSortMax * 8));
        if (e != cudaSuccess) return e;
        configured_device = dev.ordinal;
    }
    cfg.gridDim = dim3(s.heads);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = keys_bytes + 2 * kSmemSortMax * 8;
    return cudaLaunchKernelEx(&cfg, select_kernel, p);
}

}  // namespace hsb
