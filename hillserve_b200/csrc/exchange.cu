// exchange.cu -- the cross-GPU exchanges of a KV-head-sharded selected-KV
// layer over peer memory (NVLink / NVSwitch P2P loads and stores), replacing
// the NCCL broadcast and all-gathers of the collective path.
//
// The reference couples a sequence's heads twice (policy/gqa_policy.cpp:
// 49-63): the threshold comes from query head 0's maximum, and k from the F16
// mean of all 32 heads' F16 counts.  With the heads split over W GPUs, one
// step of a batch of sequences is, on every rank:
//   score (score_batch_kernel) -> [rank 0] threshold + push -> count + push,
//   wait for every rank's records -> select (the cluster selector in record
//   mode, reading the records from this rank's mailbox) -> finish: push this
//   rank's attention outputs, wait for every rank's.
// Every rank owns one mailbox (cudaMalloc'd, exported by CUDA IPC): its
// header holds one epoch flag per producer (rank 0's thresholds, each rank's
// records, each rank's outputs) and the rank's own step counter; its body the
// thresholds, the 32 heads' count records, the 32 heads' outputs and every
// rank's selection results.  Producers store into every rank's mailbox, fence
// at system scope, and the last CTA to finish releases the flag (the step's
// epoch) on every rank; consumers poll their own mailbox's flags with
// system-scope acquire loads.  Flags only grow (one epoch per step), so
// nothing is reset between steps.  Every wait is bounded (the group's limit,
// 2 s by default): a wait that gives up records HSB_E_TIMEOUT in the
// mailbox's status word and the kernel returns.  After a timeout the group's
// epochs disagree: the mailboxes must be recreated.  Every transfer is a
// plain store by a thread into peer memory.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

struct MailboxHeader {
    unsigned long long thr_flag;        // epoch of the thresholds (from rank 0)
    unsigned long long rec_flag[8];     // epoch of rank w's count records
    unsigned long long out_flag[8];     // epoch of rank w's outputs
    unsigned long long epoch;           // this rank: the last step completed
    unsigned int arrive[4];             // this rank: last-CTA counters (threshold, count, finish)
    hsb_device_status status;           // this rank: first error of the exchange
    unsigned int pad[(256 - 8 * 18 - 16 - 8) / 4];
};
static_assert(sizeof(MailboxHeader) == 256, "mailbox header is 256 bytes");

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

struct Layout {
    size_t thr, rec, out, res, ctr, total;
};
Layout layout(size_t batch) {
    Layout l{};
    l.thr = sizeof(MailboxHeader);
    l.rec = l.thr + align256(batch * 2 * 4);
    l.out = l.rec + align256(batch * kHeads * 4);
    l.res = l.out + align256(batch * kHeads * kDim * 4);
    // this rank's counters of the scorer's threshold push: [batch] CTAs per
    // sequence done, then sequences done
    l.ctr = l.res + align256((size_t)HSB_MAX_PEERS * batch * sizeof(hsb_selection));
    l.total = l.ctr + align256((batch + 1) * 4);
    return l;
}

struct PeerParams {
    unsigned char* mb[HSB_MAX_PEERS];  // every rank's mailbox (own: local)
    int world, rank;
    unsigned long long batch;
    unsigned long long limit_ns;
    Layout lay;
};

__device__ __forceinline__ MailboxHeader* header(const PeerParams& p, int w) {
    return reinterpret_cast<MailboxHeader*>(p.mb[w]);
}
// Bounded wait until *flag >= epoch; false when the limit ran out.
__device__ bool wait_flag(const unsigned long long* flag, unsigned long long epoch, unsigned long long limit_ns) {
    if (ld_acquire_sys(flag) >= epoch) return true;
    const unsigned long long start = global_ns();
    while (ld_acquire_sys(flag) < epoch) {
        if (global_ns() - start > limit_ns) return false;
        __nanosleep(32);
    }
    return true;
}
// The step this launch belongs to: one past the last completed one.
__device__ __forceinline__ unsigned long long step_epoch(const PeerParams& p) {
    return __ldcg(&header(p, p.rank)->epoch) + 1;
}
// Last-CTA election over the grid (after this CTA's stores and a system
// fence): true in exactly one CTA, which also resets the counter.
__device__ bool last_cta(unsigned int* counter) {
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
        if (last) {
            *counter = 0;
            __threadfence_system();
        }
    }
    __syncthreads();
    return last;
}
// One thread per rank releases `flag` (by offset in the header) = epoch on
// every rank's mailbox, then the caller waits for its own copies.
__device__ void release_all(const PeerParams& p, size_t flag_offset, unsigned long long epoch) {
    if (threadIdx.x < (unsigned)p.world)
        st_release_sys(reinterpret_cast<unsigned long long*>(p.mb[threadIdx.x] + flag_offset), epoch);
}
// Waits (thread w < world) for every rank's flag at flag_offset + 8 w; the
// first wait that gives up raises HSB_E_TIMEOUT (index = rank waited for).
__device__ void wait_all(const PeerParams& p, size_t flag_offset, unsigned long long epoch) {
    if (threadIdx.x < (unsigned)p.world) {
        const unsigned long long* f =
            reinterpret_cast<const unsigned long long*>(p.mb[p.rank] + flag_offset) + threadIdx.x;
        if (!wait_flag(f, epoch, p.limit_ns)) raise_status(&header(p, p.rank)->status, HSB_E_TIMEOUT, threadIdx.x);
    }
    __syncthreads();
}

constexpr int kThrThreads = 256;
// Rank 0: each sequence's threshold record {order key of F16(max - alpha),
// status} from the history scorer's head-0 partials (gqa_policy.cpp:50-54),
// stored into every rank's mailbox; the last CTA releases thr_flag.
__global__ void __launch_bounds__(kThrThreads) exch_threshold_kernel(const uint32_t* h0, float alpha,
                                                                     const __grid_constant__ PeerParams p) {
    pdl_wait();
    const unsigned long long epoch = step_epoch(p);
    h0 += (size_t)blockIdx.x * kH0Partials;
    __shared__ unsigned int smax, sbad;
    if (threadIdx.x == 0) {
        smax = 0;
        sbad = 0;
    }
    __syncthreads();
    unsigned int mx = 0, bad0 = 0;
    for (unsigned int i = threadIdx.x; i < kH0Partials; i += kThrThreads) {
        const uint32_t v = __ldcg(h0 + i);
        mx = max(mx, v & 0xffffu);
        bad0 |= v >> 16;
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    bad0 = __reduce_or_sync(0xffffffffu, bad0);
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&smax, mx);
        atomicOr(&sbad, bad0);
    }
    __syncthreads();
    if (threadIdx.x < (unsigned)p.world) {
        uint32_t* thr = reinterpret_cast<uint32_t*>(p.mb[threadIdx.x] + p.lay.thr) + 2 * blockIdx.x;
        *reinterpret_cast<uint2*>(thr) = threshold_record(smax, sbad, alpha);
    }
    if (last_cta(&header(p, p.rank)->arrive[0])) release_all(p, offsetof(MailboxHeader, thr_flag), epoch);
}

constexpr int kCntThreads = 1024;
// Every rank: wait for the thresholds, then for each (sequence, local head)
// item count #{keys >= threshold key} | non-finite << 31 and store the record
// into every rank's mailbox (column head_base + head).  A persistent grid (the
// CTAs that fit resident at once) walks the items, so the flag wait and the
// system-scope fence are paid once per CTA, not once per item; the last CTA
// releases this rank's rec_flag and waits for every rank's records.
__global__ void __launch_bounds__(kCntThreads) exch_count_kernel(const uint16_t* keys, unsigned long long tokens,
                                                                 unsigned heads, unsigned head_base,
                                                                 const __grid_constant__ PeerParams p) {
    pdl_wait();
    const unsigned long long epoch = step_epoch(p);
    MailboxHeader* own = header(p, p.rank);
    const bool vec = tokens % 8 == 0 && (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
    const unsigned long long n8 = vec ? tokens / 8 : 0;
    // The first item's keys (up to kPre 16-byte words per thread) are loaded
    // while thread 0 waits for the thresholds: the count then starts from
    // registers the moment they arrive.  Rows longer than kPre words per
    // thread take the plain loop below instead.
    constexpr int kPre = 4;
    uint4 pre[kPre];
    const bool prefetch = n8 <= (unsigned long long)kPre * kCntThreads && blockIdx.x < p.batch * heads;
    if (prefetch) {
        const uint4* row = reinterpret_cast<const uint4*>(keys + (unsigned long long)blockIdx.x * tokens);
#pragma unroll
        for (int u = 0; u < kPre; ++u) {
            const unsigned long long g = threadIdx.x + (unsigned long long)u * kCntThreads;
            pre[u] = g < n8 ? row[g] : make_uint4(0, 0, 0, 0);
        }
    }
    __shared__ int ready;
    __shared__ unsigned int scnt, sbad;
    if (threadIdx.x == 0) ready = wait_flag(&own->thr_flag, epoch, p.limit_ns);
    __syncthreads();
    if (!ready) {
        if (threadIdx.x == 0) raise_status(&own->status, HSB_E_TIMEOUT, 0);
        return;  // the group's epochs now disagree: the mailboxes must be recreated
    }
    const uint32_t* thr = reinterpret_cast<const uint32_t*>(p.mb[p.rank] + p.lay.thr);
    const unsigned long long items = p.batch * heads;
    for (unsigned long long item = blockIdx.x; item < items; item += gridDim.x) {
        const unsigned seq = (unsigned)(item / heads), head = (unsigned)(item % heads);
        const unsigned int thr_key = __ldcg(thr + 2 * seq);
        if (threadIdx.x == 0) {
            scnt = 0;
            sbad = 0;
        }
        __syncthreads();
        const uint16_t* row = keys + item * tokens;
        unsigned int cnt = 0, bad = 0;
        const bool from_regs = prefetch;
        // The next item's keys go out before this item is counted, so each
        // CTA keeps one item's loads in flight while it counts the previous.
        uint4 nxt[kPre];
        const unsigned long long next = item + gridDim.x;
        if (prefetch && next < items) {
            const uint4* nrow = reinterpret_cast<const uint4*>(keys + next * tokens);
#pragma unroll
            for (int u = 0; u < kPre; ++u) {
                const unsigned long long g = threadIdx.x + (unsigned long long)u * kCntThreads;
                nxt[u] = g < n8 ? nrow[g] : make_uint4(0, 0, 0, 0);
            }
        }
        if (from_regs) {
#pragma unroll
            for (int u = 0; u < kPre; ++u) {
                if (threadIdx.x + (unsigned long long)u * kCntThreads >= n8) continue;
                const uint32_t v[4] = {pre[u].x, pre[u].y, pre[u].z, pre[u].w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t key = (v[j >> 1] >> (16 * (j & 1))) & 0xffffu;
                    bad |= key_nonfinite(key);
                    cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
                }
            }
        }
        for (unsigned long long g = threadIdx.x; g < (from_regs ? 0 : n8); g += kCntThreads) {
            const uint4 w = reinterpret_cast<const uint4*>(row)[g];
            const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t key = (v[j >> 1] >> (16 * (j & 1))) & 0xffffu;
                bad |= key_nonfinite(key);
                cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
            }
        }
        for (unsigned long long i = n8 * 8 + threadIdx.x; i < tokens; i += kCntThreads) {
            const uint32_t key = row[i];
            bad |= key_nonfinite(key);
            cnt += (!key_nan(key) && key >= thr_key) ? 1u : 0u;
        }
        if (prefetch && next < items) {
#pragma unroll
            for (int u = 0; u < kPre; ++u) pre[u] = nxt[u];
        }
        cnt = __reduce_add_sync(0xffffffffu, cnt);
        bad = __any_sync(0xffffffffu, bad);
        if ((threadIdx.x & 31) == 0) {
            if (cnt) atomicAdd(&scnt, cnt);
            if (bad) atomicOr(&sbad, 1u);
        }
        __syncthreads();
        if (threadIdx.x < (unsigned)p.world) {
            uint32_t* rec = reinterpret_cast<uint32_t*>(p.mb[threadIdx.x] + p.lay.rec);
            rec[(size_t)seq * kHeads + head_base + head] = scnt | (sbad << 31);
        }
        __syncthreads();  // scnt / sbad are reset for the next item
    }
    if (last_cta(&own->arrive[1])) {
        release_all(p, offsetof(MailboxHeader, rec_flag) + 8 * p.rank, epoch);
        wait_all(p, offsetof(MailboxHeader, rec_flag), epoch);
    }
}

// The same exchange with the items staged in shared memory by the bulk-copy
// engine: up to kCntStages items (64 KB each at 32768 keys) per CTA are in
// flight at once, so the key stream does not stall on one item's round
// trip; the count then reads shared memory.  Chosen by the host when the
// rows are 16-byte aligned and at least two items fit.  Every wait is
// bounded; a CTA that gives up waits (bounded) for its own copies still in
// flight before it returns.
constexpr int kCntStages = 3;
constexpr size_t kCntStageSmem = 200 * 1024;  // dynamic shared memory the stages may take
__global__ void __launch_bounds__(kCntThreads, 1) exch_count_staged_kernel(const uint16_t* keys,
                                                                           unsigned long long tokens, unsigned heads,
                                                                           unsigned head_base, int stages,
                                                                           const __grid_constant__ PeerParams p) {
    pdl_wait();
    extern __shared__ __align__(128) unsigned char stage_buf[];
    __shared__ uint64_t bar[kCntStages];
    __shared__ int ready;
    const unsigned long long epoch = step_epoch(p);
    MailboxHeader* own = header(p, p.rank);
    const unsigned long long items = p.batch * heads;
    const uint32_t item_bytes = (uint32_t)(tokens * 2);
    const unsigned long long mine = blockIdx.x < items ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const unsigned long long issued0 = mine < (unsigned long long)stages ? mine : (unsigned long long)stages;
    auto issue = [&](unsigned long long j) {  // this CTA's j-th item into stage j % stages
        uint64_t* b = &bar[j % stages];
        mbar_arrive_expect_tx(b, item_bytes);
        bulk_copy_g2s(stage_buf + (j % stages) * item_bytes, keys + (blockIdx.x + j * gridDim.x) * tokens, item_bytes,
                      b);
    };
    // Copies issued and not yet consumed [from, to): waited for before any exit.
    auto drain = [&](unsigned long long from, unsigned long long to) {
        for (unsigned long long j = from; j < to; ++j) (void)mbar_wait(&bar[j % stages], (uint32_t)((j / stages) & 1));
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(&bar[s], 1);
        mbar_fence_init();
        for (unsigned long long j = 0; j < issued0; ++j) issue(j);
        ready = wait_flag(&own->thr_flag, epoch, p.limit_ns);
    }
    __syncthreads();
    if (!ready) {
        if (threadIdx.x == 0) {
            raise_status(&own->status, HSB_E_TIMEOUT, 0);
            drain(0, issued0);
        }
        return;  // the group's epochs now disagree: the mailboxes must be recreated
    }
    const uint32_t* thr = reinterpret_cast<const uint32_t*>(p.mb[p.rank] + p.lay.thr);
    const unsigned long long n8 = tokens / 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Per-warp partials of the last two items (double-buffered by item
    // parity): one CTA barrier per item.  Warp 0 reduces item j's partials
    // after barrier j and before it reaches barrier j + 1, so item j + 2
    // (same slot) cannot overwrite them early.
    __shared__ unsigned int wcnt[2][kCntThreads / 32], wbad[2][kCntThreads / 32];
    for (unsigned long long j = 0; j < mine; ++j) {
        const unsigned long long item = blockIdx.x + j * gridDim.x;
        const unsigned seq = (unsigned)(item / heads), head = (unsigned)(item % heads);
        const unsigned int thr_key = __ldcg(thr + 2 * seq);
        // Counted: not NaN and >= threshold, i.e. key in [max(thr, 0x03ff), 0xfc00];
        // non-finite: key <= 0x03ff or key >= 0xfc00 (from the running min / max).
        const uint32_t lo = max(thr_key, 0x03ffu);
        const uint32_t span = lo <= 0xfc00u ? 0xfc00u - lo : 0u;
        const bool none = lo > 0xfc00u;
        bool ok = mbar_wait(&bar[j % stages], (uint32_t)((j / stages) & 1));
        unsigned int cnt = 0;
        uint32_t kmin = 0xffffu, kmax = 0u;
        if (ok) {
            const uint4* row = reinterpret_cast<const uint4*>(stage_buf + (j % stages) * item_bytes);
            for (unsigned long long g = threadIdx.x; g < n8; g += kCntThreads) {
                const uint4 w = row[g];
                const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t k0 = v[e] & 0xffffu, k1 = v[e] >> 16;
                    kmin = min(kmin, min(k0, k1));
                    kmax = max(kmax, max(k0, k1));
                    cnt += (k0 - lo <= span) ? 1u : 0u;
                    cnt += (k1 - lo <= span) ? 1u : 0u;
                }
            }
        }
        if (none) cnt = 0;
        cnt = __reduce_add_sync(0xffffffffu, cnt);
        kmin = __reduce_min_sync(0xffffffffu, kmin);
        kmax = __reduce_max_sync(0xffffffffu, kmax);
        if (lane == 0) {
            wcnt[j & 1][warp] = cnt;
            wbad[j & 1][warp] = (kmin <= 0x03ffu || kmax >= 0xfc00u) ? 1u : 0u;
        }
        if (__syncthreads_or(!ok)) {  // the stage is read by every warp (or a copy never landed)
            if (threadIdx.x == 0) {
                raise_status(&own->status, HSB_E_TIMEOUT, (int)blockIdx.x);
                const unsigned long long issued = j + stages < mine ? j + stages : mine;
                drain(j, issued);  // item j's own copy included
            }
            return;
        }
        if (threadIdx.x == 0 && j + stages < mine) issue(j + stages);
        if (warp == 0) {
            unsigned int c = wcnt[j & 1][lane], bd = wbad[j & 1][lane];
            c = __reduce_add_sync(0xffffffffu, c);
            bd = __reduce_or_sync(0xffffffffu, bd);
            if (lane < p.world) {
                uint32_t* rec = reinterpret_cast<uint32_t*>(p.mb[lane] + p.lay.rec);
                rec[(size_t)seq * kHeads + head_base + head] = c | (bd << 31);
            }
        }
    }
    if (last_cta(&own->arrive[1])) {
        release_all(p, offsetof(MailboxHeader, rec_flag) + 8 * p.rank, epoch);
        wait_all(p, offsetof(MailboxHeader, rec_flag), epoch);
    }
}

constexpr int kFinThreads = 256;
// Every rank: this rank's outputs [batch][heads][128] and selection results
// [batch] into every rank's mailbox (outputs at heads head_base.., results at
// slot rank); the last CTA releases out_flag, waits for every rank's, and
// closes the step (epoch).
__global__ void __launch_bounds__(kFinThreads) exch_finish_kernel(const float* out, const hsb_selection* results,
                                                                  unsigned heads, unsigned head_base,
                                                                  const __grid_constant__ PeerParams p) {
    pdl_wait();
    const unsigned long long epoch = step_epoch(p);
    const unsigned long long n4 = p.batch * heads * (kDim / 4);  // float4 pieces
    for (unsigned long long i = blockIdx.x * (unsigned long long)kFinThreads + threadIdx.x; i < n4;
         i += (unsigned long long)gridDim.x * kFinThreads) {
        const unsigned long long row = i / (kDim / 4), piece = i % (kDim / 4);
        const unsigned long long seq = row / heads, h = row % heads;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(out) + i);
        const unsigned long long at = ((seq * kHeads + head_base + h) * kDim) / 4 + piece;
        for (int w = 0; w < p.world; ++w) reinterpret_cast<float4*>(p.mb[w] + p.lay.out)[at] = v;
    }
    for (unsigned long long i = blockIdx.x * (unsigned long long)kFinThreads + threadIdx.x; i < p.batch;
         i += (unsigned long long)gridDim.x * kFinThreads) {
        const hsb_selection r = results[i];
        for (int w = 0; w < p.world; ++w)
            reinterpret_cast<hsb_selection*>(p.mb[w] + p.lay.res)[(size_t)p.rank * p.batch + i] = r;
    }
    MailboxHeader* own = header(p, p.rank);
    if (last_cta(&own->arrive[2])) {
        release_all(p, offsetof(MailboxHeader, out_flag) + 8 * p.rank, epoch);
        wait_all(p, offsetof(MailboxHeader, out_flag), epoch);
        if (threadIdx.x == 0) own->epoch = epoch;
    }
}

bool peer_params(const hsb_peer_group* g, PeerParams* p) {
    if (!g || g->world < 1 || g->world > HSB_MAX_PEERS || HSB_KV_HEADS % g->world || g->rank < 0 ||
        g->rank >= g->world || g->batch == 0)
        return false;
    for (int w = 0; w < g->world; ++w) {
        if (!g->mailbox[w] || (reinterpret_cast<uintptr_t>(g->mailbox[w]) & 255)) return false;
        p->mb[w] = static_cast<unsigned char*>(g->mailbox[w]);
    }
    p->world = g->world;
    p->rank = g->rank;
    p->batch = g->batch;
    p->limit_ns = g->wait_limit_ns ? g->wait_limit_ns : kWaitLimitNs;
    p->lay = layout(g->batch);
    return true;
}

}  // namespace

bool threshold_push_params(const hsb_peer_group* g, float alpha, ThresholdPush* out) {
    PeerParams p{};
    if (!peer_params(g, &p) || g->rank != 0) return false;
    *out = ThresholdPush{};
    for (int w = 0; w < g->world; ++w) out->mb[w] = p.mb[w];
    out->world = g->world;
    out->thr_off = p.lay.thr;
    out->flag_off = offsetof(MailboxHeader, thr_flag);
    out->epoch = &reinterpret_cast<MailboxHeader*>(p.mb[0])->epoch;
    out->cta_done = reinterpret_cast<unsigned int*>(p.mb[0] + p.lay.ctr);
    out->alpha = alpha;
    return true;
}

size_t mailbox_bytes(size_t batch) { return layout(batch).total; }

void mailbox_offsets(size_t batch, hsb_mailbox_layout* out) {
    const Layout l = layout(batch);
    out->thr = l.thr;
    out->records = l.rec;
    out->outputs = l.out;
    out->results = l.res;
    out->status = offsetof(MailboxHeader, status);
    out->bytes = l.total;
}

cudaError_t launch_exchange_threshold(const uint32_t* h0, float alpha, const hsb_peer_group* g,
                                      cudaStream_t stream) {
    PeerParams p{};
    if (!peer_params(g, &p)) return cudaErrorInvalidValue;
    return launch_dependent(exch_threshold_kernel, dim3((unsigned)g->batch), dim3(kThrThreads), 0, stream, false, h0,
                            alpha, p);
}

cudaError_t launch_exchange_count(const uint16_t* keys, size_t heads, size_t tokens, const hsb_peer_group* g,
                                  cudaStream_t stream) {
    PeerParams p{};
    if (!peer_params(g, &p) || heads * g->world != kHeads) return cudaErrorInvalidValue;
    const DeviceInfo& dev = device_info();
    // The persistent grid is what stays resident (one 1024-thread CTA per SM
    // at this register count): CTAs beyond it would wait for the first ones
    // to exit and run their items as a second, serial wave.
    static thread_local int resident_device = -1, resident = 1;
    if (resident_device != dev.ordinal) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, exch_count_kernel, kCntThreads, 0) != cudaSuccess ||
            n < 1)
            n = 1;
        (void)cudaGetLastError();
        resident = n;
        resident_device = dev.ordinal;
    }
    // Staged path: rows 16-byte aligned and at least two 64 KB-class items
    // in shared memory (one CTA per SM).
    const size_t item_bytes = tokens * 2;
    const int stages = (int)std::min<size_t>(kCntStages, item_bytes ? kCntStageSmem / item_bytes : 0);
    if (tokens % 8 == 0 && (reinterpret_cast<uintptr_t>(keys) & 15) == 0 && stages >= 2 &&
        item_bytes <= 0xffffffffull) {
        static thread_local int staged_device = -1;
        if (staged_device != dev.ordinal) {
            const cudaError_t e = cudaFuncSetAttribute(exch_count_staged_kernel,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCntStageSmem);
            if (e != cudaSuccess) return e;
            staged_device = dev.ordinal;
        }
        const unsigned sgrid = (unsigned)std::min<unsigned long long>(heads * g->batch, (unsigned long long)dev.sms);
        return launch_dependent(exch_count_staged_kernel, dim3(sgrid), dim3(kCntThreads), (size_t)stages * item_bytes,
                                stream, false, keys, (unsigned long long)tokens, (unsigned)heads,
                                (unsigned)(heads * g->rank), stages, p);
    }
    const unsigned grid =
        (unsigned)std::min<unsigned long long>(heads * g->batch, (unsigned long long)dev.sms * resident);
    return launch_dependent(exch_count_kernel, dim3(grid), dim3(kCntThreads), 0, stream, false, keys,
                            (unsigned long long)tokens, (unsigned)heads, (unsigned)(heads * g->rank), p);
}

cudaError_t launch_exchange_finish(const float* out, const hsb_selection* results, size_t heads,
                                   const hsb_peer_group* g, cudaStream_t stream) {
    PeerParams p{};
    if (!peer_params(g, &p) || heads * g->world != kHeads) return cudaErrorInvalidValue;
    const DeviceInfo& dev = device_info();
    const unsigned long long pieces = g->batch * heads * (kDim / 4);
    const unsigned blocks =
        (unsigned)std::max<unsigned long long>(1, std::min<unsigned long long>((pieces + kFinThreads - 1) / kFinThreads,
                                                                               (unsigned long long)dev.sms));
    return launch_dependent(exch_finish_kernel, dim3(blocks), dim3(kFinThreads), 0, stream, false, out, results,
                            (unsigned)heads, (unsigned)(heads * g->rank), p);
}

}  // namespace hsb
