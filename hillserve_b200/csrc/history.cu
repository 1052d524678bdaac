// history.cu -- the decode history of one request on the GPU: hot/cold
// history scoring and the prepare -> select -> fetch protocol of
// FullGqaRuntimePolicy (policy/full_gqa_runtime.cpp:418-471 score_history,
// :493-516 prepare, :549-585 select, :586-690 fetch), with the hot KV in
// HBM instead of host memory.
//
// Memory (per layer).  The reference keeps hot KV rows in host memory and
// reads cold raw K from a file for every decode step's scoring.  Here:
//  - hot pool: K||V rows (2048 F16 words) of the placement's hot positions,
//    in slot order (plan_full_gqa_runtime's hot_slot_by_position), in HBM;
//  - cold K: the raw K rows (1024 words) of the cold prompt positions, in
//    HBM as well -- scoring reads every position's K at every step, and at
//    2 KB per token a whole 32-layer 64K history fits easily beside the
//    hot pool, so only the cold positions' V (their records) stays in the
//    cold tier and is fetched for the positions a selection needs.
// Scoring [0, valid) is then one TMA scorer launch over the position runs
// (a hot run reads the pool, a cold run the cold K), columns = positions:
// the same raw F16 scores as the reference's hot + cold merge.
//
// Protocol.  prepare() scores the history [0, position) -- raw scores and
// the order keys of the normalised ones -- and selects its payload cover
// (the selector in cover mode, on those keys) on the history's own stream,
// like the reference's async job; cover() then lists the cover's cold
// positions.  select() joins the job on the caller's stream, scores the
// current token and selects on the keys; fetch() builds the gather map of
// the selected IDs (hot -> pool slot, cold -> the caller's staged rows) and
// packs K/V with hsb_gather_map's kernel (live slots only, or zero padding
// up to `count`).  The reference's protocol checks are kept, with its
// messages.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace hsb {
namespace {

constexpr size_t kRowWords = 2048;  // K[8][128] then V[8][128]
constexpr size_t kKeyWords = 1024;

struct Run {
    uint64_t first;  // first position
    uint64_t count;
    bool hot;
    uint64_t row;  // first pool slot or cold row
};

// Runs of positions [0, n) whose rows are consecutive in one source.
// row_of_position: >= 0 hot slot, <= -2 cold row -2-r, -1 not resident.
bool build_runs(const int64_t* row_of_position, size_t n, std::vector<Run>* runs, uint64_t* missing) {
    runs->clear();
    for (uint64_t t = 0; t < n; ++t) {
        const int64_t r = row_of_position[t];
        if (r == -1) {
            *missing = t;
            return false;
        }
        const bool hot = r >= 0;
        const uint64_t row = hot ? (uint64_t)r : (uint64_t)(-2 - r);
        if (!runs->empty()) {
            Run& b = runs->back();
            if (b.hot == hot && b.first + b.count == t && b.row + b.count == row) {
                ++b.count;
                continue;
            }
        }
        runs->push_back(Run{t, 1, hot, row});
    }
    return true;
}

// One scorer launch per HSB_MAX_VIEWS runs, columns = positions.
cudaError_t score_runs(const uint16_t* q, const std::vector<Run>& runs, uint64_t valid, const uint16_t* pool,
                       size_t pool_stride, const uint16_t* cold, size_t cold_stride, uint16_t* out, size_t out_stride,
                       uint16_t* keys, cudaStream_t stream) {
    std::vector<hsb_key_view> views;
    uint64_t col0 = 0;
    for (const Run& r : runs) {
        if (r.first >= valid) break;
        const uint64_t n = std::min<uint64_t>(r.count, valid - r.first);
        views.push_back(r.hot ? hsb_key_view{pool + r.row * pool_stride, n, pool_stride}
                              : hsb_key_view{cold + r.row * cold_stride, n, cold_stride});
        if (views.size() == HSB_MAX_VIEWS) {
            cudaError_t e = launch_score(q, views.data(), views.size(), out, out_stride, col0, nullptr, stream, keys);
            if (e != cudaSuccess) return e;
            for (const auto& v : views) col0 += v.tokens;
            views.clear();
        }
    }
    if (!views.empty()) return launch_score(q, views.data(), views.size(), out, out_stride, col0, nullptr, stream, keys);
    return cudaSuccess;
}

// ------------------------------------------------------------- kernels
// Appended K||V rows land in the pool (hot positions) or, K only, in the
// cold K store (cold positions).
__global__ void history_append_kernel(const uint16_t* __restrict__ rows, unsigned long long first,
                                      unsigned long long count, const int32_t* __restrict__ slot,
                                      const int32_t* __restrict__ cold_row, uint16_t* __restrict__ pool,
                                      uint16_t* __restrict__ cold) {
    pdl_wait();
    pdl_trigger();
    const unsigned long long t = blockIdx.x;
    if (t >= count) return;
    const unsigned long long pos = first + t;
    const uint4* src = reinterpret_cast<const uint4*>(rows + t * kRowWords);
    const int32_t s = slot[pos];
    // 128 threads; each thread's loads are issued before its stores.
    if (s >= 0) {
        uint4* dst = reinterpret_cast<uint4*>(pool + (size_t)s * kRowWords);
        constexpr int kPer = (int)(kRowWords / 8) / 128;
        uint4 w[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) w[u] = src[threadIdx.x + u * 128];
#pragma unroll
        for (int u = 0; u < kPer; ++u) dst[threadIdx.x + u * 128] = w[u];
    } else if (cold_row[pos] >= 0) {
        uint4* dst = reinterpret_cast<uint4*>(cold + (size_t)cold_row[pos] * kKeyWords);
        for (int i = threadIdx.x; i < (int)(kKeyWords / 8); i += blockDim.x) dst[i] = src[i];
    }
}

// The cold positions of a prepared cover, ascending: every position some
// head's top-`bound` list names whose K lives in the cold store (the cold
// tier's read list; the cover's hot rows are in the pool already).  One
// block: a bitmap of the history in shared memory, then a block-wide
// compaction in position order.
constexpr unsigned kCoverWords = (66048 + 31) / 32;
__global__ void __launch_bounds__(1024) history_cover_cold_kernel(const uint32_t* __restrict__ cover,
                                                                  unsigned long long cap,
                                                                  const hsb_selection* __restrict__ result,
                                                                  const int32_t* __restrict__ slot,
                                                                  unsigned long long position,
                                                                  uint32_t* __restrict__ out,
                                                                  uint32_t* __restrict__ out_count) {
    __shared__ uint32_t bits[kCoverWords];
    __shared__ uint32_t warp_total[32];
    pdl_wait();
    pdl_trigger();
    const unsigned tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned words = (unsigned)((position + 31) / 32);
    for (unsigned w = tid; w < words; w += blockDim.x) bits[w] = 0;
    __syncthreads();
    const unsigned long long bound = result->status.code ? 0ull : (result->k < cap ? result->k : cap);
    for (unsigned long long i = tid; i < 32ull * bound; i += blockDim.x) {
        const uint32_t id = cover[(i / bound) * cap + i % bound];
        if (id < position && slot[id] < 0) atomicOr(&bits[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
    const unsigned per = (words + blockDim.x - 1) / blockDim.x;
    const unsigned w0 = min(words, tid * per), w1 = min(words, w0 + per);
    unsigned mine = 0;
    for (unsigned w = w0; w < w1; ++w) mine += __popc(bits[w]);
    unsigned scan = mine;  // inclusive scan within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, scan, o);
        if (lane >= (unsigned)o) scan += y;
    }
    if (lane == 31) warp_total[warp] = scan;
    __syncthreads();
    unsigned before = scan - mine;
    for (unsigned w = 0; w < warp; ++w) before += warp_total[w];
    for (unsigned w = w0; w < w1; ++w) {
        uint32_t b = bits[w];
        while (b) {
            out[before++] = w * 32 + (__ffs(b) - 1);
            b &= b - 1;
        }
    }
    if (tid == blockDim.x - 1) *out_count = before;
}

// Gather map of a selection: map[h * count + j] = the pool slot of
// ids[h][j] (hot), -2 - r for the r-th staged cold row, -1 past k.  A
// selected cold ID that was not staged is an error (the cover guarantees
// every final historical ID), as is an ID past the appended positions.
__global__ void history_map_kernel(const uint32_t* __restrict__ ids, unsigned long long kcap,
                                   const hsb_selection* __restrict__ result, const int32_t* __restrict__ slot,
                                   unsigned long long completed, const uint32_t* __restrict__ staged,
                                   unsigned long long nstaged, unsigned long long count, int32_t* __restrict__ map,
                                   hsb_device_status* status) {
    pdl_wait();
    pdl_trigger();
    const unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 32ull * count) return;
    const unsigned h = (unsigned)(i / count);
    const unsigned long long j = i % count;
    const uint32_t k = result->k;
    if (j >= k || j >= kcap) {
        map[i] = -1;
        return;
    }
    const uint32_t id = ids[h * kcap + j];
    if (id >= completed) {
        map[i] = -1;
        raise_status(status, HSB_E_PACK_MISSING, (int)h);
        return;
    }
    const int32_t s = slot[id];
    if (s >= 0) {
        map[i] = s;
        return;
    }
    unsigned long long lo = 0, hi = nstaged;  // first staged >= id
    while (lo < hi) {
        const unsigned long long mid = (lo + hi) / 2;
        if (staged[mid] < id) lo = mid + 1;
        else hi = mid;
    }
    if (lo < nstaged && staged[lo] == id) {
        map[i] = (int32_t)(-2 - (long long)lo);
    } else {
        map[i] = -1;
        raise_status(status, HSB_E_MAP_MISS, (int)h);
    }
}

// select()'s query must be prepare()'s (policy/full_gqa_runtime.cpp:558):
// the reference throws before selecting, so the mismatch replaces whatever
// status the selection left.
__global__ void history_query_check_kernel(const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                                           hsb_selection* result) {
    pdl_wait();
    pdl_trigger();
    // 256 threads: every load issued before any compare (one round trip).
    constexpr int kPer = kHeads * kDim / 256;
    uint16_t x[kPer], y[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        x[u] = a[threadIdx.x + u * 256];
        y[u] = b[threadIdx.x + u * 256];
    }
    bool same = true;
#pragma unroll
    for (int u = 0; u < kPer; ++u) same &= x[u] == y[u];
    if (!__syncthreads_and(same) && threadIdx.x == 0) {
        result->k = 0;
        result->boundary_tied_heads = 0;
        result->status.code = HSB_E_HISTORY_QUERY;
        result->status.index = 0;
    }
}

template <typename T>
T* dev_alloc(size_t n, cudaError_t* e) {
    void* p = nullptr;
    if (*e == cudaSuccess) *e = cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 256));
    return static_cast<T*>(p);
}

}  // namespace
}  // namespace hsb

using namespace hsb;

struct hsb_history {
    hsb_history_config cfg{};
    int device = 0;
    size_t hot_slots = 0, cold_rows = 0, cover_cap = 0, kcap = 0;
    cudaStream_t work = nullptr;
    struct Layer {
        std::vector<int64_t> row_of_position;  // host: >= 0 slot, <= -2 cold row, -1 not resident
        std::vector<Run> runs;
        int32_t* slot = nullptr;      // device [capacity]
        int32_t* cold_row = nullptr;  // device [capacity]
        uint16_t* pool = nullptr;     // [hot_slots][2048]
        uint16_t* cold = nullptr;     // [cold_rows][1024]
        uint64_t completed = 0;
        uint64_t last_selected = std::numeric_limits<uint64_t>::max();
        int job = -1;  // pending prepared history
    };
    std::vector<Layer> layers;
    struct Job {
        bool used = false;
        size_t layer = 0;
        uint64_t position = 0;
        uint16_t* raw = nullptr;   // [32][capacity]
        uint16_t* keys = nullptr;  // [32][capacity] order keys of the normalised scores
        uint16_t* query = nullptr; // [32][128] F16 of prepare()
        uint32_t* cover = nullptr; // [32][cap]
        size_t cap = 0;
        hsb_selection* cover_result = nullptr;
        cudaEvent_t ready = nullptr;
        cudaEvent_t inputs = nullptr;
    } jobs[2];
    uint16_t* raw_direct = nullptr;  // select() without a prepared history
    uint16_t* keys_direct = nullptr;
    void* select_ws = nullptr;
    size_t select_ws_bytes = 0;
    void* cover_ws = nullptr;
    size_t cover_ws_bytes = 0;
    int32_t* map = nullptr;  // [32][count] of the last fetch
    size_t map_capacity = 0;
    std::vector<void*> allocations;

    ~hsb_history() {
        int previous = 0;
        const bool restore = cudaGetDevice(&previous) == cudaSuccess;
        cudaSetDevice(device);
        if (work) cudaStreamSynchronize(work);
        for (auto& j : jobs) {
            if (j.ready) cudaEventDestroy(j.ready);
            if (j.inputs) cudaEventDestroy(j.inputs);
        }
        for (void* p : allocations)
            if (p) cudaFree(p);
        if (work) cudaStreamDestroy(work);
        if (restore) cudaSetDevice(previous);
    }
};

namespace {
int history_fail(int status, const char* message) { return record_error(status, message); }

template <typename T>
T* keep(hsb_history* h, T* p) {
    h->allocations.push_back(p);
    return p;
}
}  // namespace

extern "C" {

int hsb_score_history(const uint16_t* d_q, const uint16_t* d_hot_pool, size_t pool_stride_words,
                      const uint16_t* d_cold_k, size_t cold_stride_words, const int64_t* row_of_position,
                      size_t valid, uint16_t* d_scores, size_t out_stride, uint16_t* d_order_keys, void* stream) {
    if (!d_q || !row_of_position || !d_scores || !valid || out_stride < valid)
        return history_fail(HSB_E_SCORE_SHAPE, "full GQA CPU query/views shape");
    if ((pool_stride_words != 1024 && pool_stride_words != 2048) ||
        (cold_stride_words != 1024 && cold_stride_words != 2048))
        return history_fail(HSB_E_SCORE_SHAPE, "full GQA CPU key view shape/stride/extent");
    std::vector<Run> runs;
    uint64_t missing = 0;
    if (!build_runs(row_of_position, valid, &runs, &missing))
        return history_fail(HSB_E_HISTORY_RESIDENCY, "full GQA hot lookup on cold/unreserved token");
    for (const Run& r : runs)
        if ((r.hot && !d_hot_pool) || (!r.hot && !d_cold_k))
            return history_fail(HSB_E_SCORE_SHAPE, "full GQA CPU key view shape/stride/extent");
    cudaError_t e = score_runs(d_q, runs, valid, d_hot_pool, pool_stride_words, d_cold_k, cold_stride_words, d_scores,
                               out_stride, d_order_keys, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_cuda_error(e, "history score launch");
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_history_plan_slots(size_t prompt_tokens, size_t generated_capacity, size_t capacity, double beta,
                           int allow_partial_prompt, int64_t* hot_slot_by_position, size_t* hot_prompt_tokens) {
    // runtime/full_gqa_contract.hpp:42-56 (hot blocks), :128-134 (hot tokens
    // and the recent pin), :168-184 (placement).
    if (!hot_slot_by_position) return history_fail(HSB_E_INVALID, "history plan arguments");
    if (!(prompt_tokens >= 128 && (allow_partial_prompt || prompt_tokens % 64 == 0) && prompt_tokens <= 65536))
        return history_fail(HSB_E_HISTORY_GEOMETRY,
                            "full GQA prompt must be >=128; partial tail requires explicit hot-tail mode");
    if (std::isnan(beta) || beta < 0)
        return history_fail(HSB_E_HISTORY_GEOMETRY, "full GQA offline beta must be nonnegative");
    if (generated_capacity < 1 || generated_capacity > 512)
        return history_fail(HSB_E_HISTORY_GEOMETRY, "full GQA generated capacity must be 1..512");
    if (capacity < prompt_tokens + generated_capacity || capacity % 64)
        return history_fail(HSB_E_HISTORY_GEOMETRY,
                            "full GQA common store capacity must cover prompt+decode and align64");
    const uint64_t blocks = prompt_tokens / 64;
    uint64_t hot_blocks = blocks;
    if (!std::isinf(beta)) {
        const long double b = beta;
        const auto rounded = (uint64_t)std::floor((long double)blocks * (b / (1 + b)));
        hot_blocks = std::min<uint64_t>(rounded, blocks - 1);
    }
    const uint64_t tail = prompt_tokens % 64;
    const uint64_t hot = hot_blocks * 64 + tail;
    const uint64_t recent = std::min<uint64_t>(16, hot_blocks) * 64 + tail;
    const uint64_t early = hot - recent, recent_begin = prompt_tokens - recent;
    int64_t next = 0;
    for (size_t t = 0; t < capacity; ++t) hot_slot_by_position[t] = -1;
    for (uint64_t t = 0; t < prompt_tokens; ++t)
        if (t < early || t >= recent_begin) hot_slot_by_position[t] = next++;
    for (uint64_t t = 0; t < generated_capacity; ++t) hot_slot_by_position[prompt_tokens + t] = (int64_t)(hot + t);
    if (hot_prompt_tokens) *hot_prompt_tokens = hot;
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_history_create(const hsb_history_config* cfg, const int64_t* hot_slot_by_position, hsb_history** out) {
    if (!cfg || !hot_slot_by_position || !out) return history_fail(HSB_E_INVALID, "history arguments");
    *out = nullptr;
    const hsb_history_config c = *cfg;
    // runtime/full_gqa_contract.hpp:116-122
    if (!c.layers || c.layers > 32 || c.generated_capacity < 1 || c.generated_capacity > 512 ||
        c.capacity < c.prompt_tokens + c.generated_capacity || c.capacity > (c.fp32_counts ? 66048u : 65536u) ||
        c.capacity % 64 || !c.prompt_tokens || !(c.alpha >= 0.0f) || !std::isfinite(c.alpha))
        return history_fail(HSB_E_HISTORY_GEOMETRY, "full GQA common store capacity must cover prompt+decode and align64");
    if (!c.fp32_counts && c.prompt_tokens + c.generated_capacity > 65504)
        return history_fail(HSB_E_HISTORY_GEOMETRY, "full GQA visible count exceeds finite F16 selection contract");
    std::unique_ptr<hsb_history> h(new hsb_history);
    h->cfg = c;
    cudaGetDevice(&h->device);
    // Placement: the plan's slots for hot positions; cold prompt positions get
    // cold rows in position order; every generated position must be hot.
    std::vector<int64_t> map(c.capacity, -1);
    int64_t max_slot = -1;
    size_t cold = 0;
    for (size_t t = 0; t < c.capacity; ++t) {
        const int64_t s = hot_slot_by_position[t];
        if (s >= 0) {
            map[t] = s;
            max_slot = std::max(max_slot, s);
        } else if (t < c.prompt_tokens) {
            map[t] = -2 - (int64_t)cold++;
        } else if (t < c.prompt_tokens + c.generated_capacity) {
            return history_fail(HSB_E_HISTORY_GEOMETRY, "generated positions must have reserved hot slots");
        }
    }
    {
        std::vector<int64_t> seen(max_slot + 1, -1);
        for (size_t t = 0; t < c.capacity; ++t)
            if (map[t] >= 0) {
                if (seen[map[t]] >= 0) return history_fail(HSB_E_HISTORY_GEOMETRY, "hot slot assigned twice");
                seen[map[t]] = (int64_t)t;
            }
    }
    h->hot_slots = (size_t)(max_slot + 1);
    h->cold_rows = cold;
    h->cover_cap = std::max<size_t>(1, (size_t)std::floor(double(c.capacity) * double(0.2f)));
    h->kcap = h->cover_cap;
    std::vector<int32_t> slot32(c.capacity), cold32(c.capacity);
    for (size_t t = 0; t < c.capacity; ++t) {
        slot32[t] = map[t] >= 0 ? (int32_t)map[t] : -1;
        cold32[t] = map[t] <= -2 ? (int32_t)(-2 - map[t]) : -1;
    }
    cudaError_t e = cudaStreamCreateWithFlags(&h->work, cudaStreamNonBlocking);
    h->layers.resize(c.layers);
    for (auto& L : h->layers) {
        L.row_of_position = map;
        uint64_t missing = 0;
        std::vector<int64_t> resident(map.begin(), map.begin() + (c.prompt_tokens + c.generated_capacity));
        build_runs(resident.data(), resident.size(), &L.runs, &missing);
        L.slot = keep(h.get(), dev_alloc<int32_t>(c.capacity, &e));
        L.cold_row = keep(h.get(), dev_alloc<int32_t>(c.capacity, &e));
        L.pool = keep(h.get(), dev_alloc<uint16_t>(h->hot_slots * kRowWords, &e));
        L.cold = keep(h.get(), dev_alloc<uint16_t>(std::max<size_t>(h->cold_rows, 1) * kKeyWords, &e));
        if (e == cudaSuccess) e = cudaMemcpy(L.slot, slot32.data(), c.capacity * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(L.cold_row, cold32.data(), c.capacity * 4, cudaMemcpyHostToDevice);
    }
    h->cover_ws_bytes = select_workspace_bytes(kHeads, c.capacity, h->cover_cap);
    h->select_ws_bytes = select_workspace_bytes(kHeads, c.capacity, h->kcap);
    for (auto& j : h->jobs) {
        j.raw = keep(h.get(), dev_alloc<uint16_t>((size_t)kHeads * c.capacity, &e));
        j.keys = keep(h.get(), dev_alloc<uint16_t>((size_t)kHeads * c.capacity, &e));
        j.query = keep(h.get(), dev_alloc<uint16_t>((size_t)kHeads * kDim, &e));
        j.cover = keep(h.get(), dev_alloc<uint32_t>((size_t)kHeads * h->cover_cap, &e));
        j.cover_result = keep(h.get(), dev_alloc<hsb_selection>(1, &e));
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&j.ready, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&j.inputs, cudaEventDisableTiming);
    }
    h->raw_direct = keep(h.get(), dev_alloc<uint16_t>((size_t)kHeads * c.capacity, &e));
    h->keys_direct = keep(h.get(), dev_alloc<uint16_t>((size_t)kHeads * c.capacity, &e));
    h->select_ws = keep(h.get(), dev_alloc<unsigned char>(h->select_ws_bytes, &e));
    h->cover_ws = keep(h.get(), dev_alloc<unsigned char>(h->cover_ws_bytes, &e));
    if (e != cudaSuccess) return record_cuda_error(e, "history allocation");
    *out = h.release();
    record_error(HSB_OK, "");
    return HSB_OK;
}

void hsb_history_destroy(hsb_history* h) { delete h; }

size_t hsb_history_hot_slots(const hsb_history* h) { return h ? h->hot_slots : 0; }
size_t hsb_history_cold_rows(const hsb_history* h) { return h ? h->cold_rows : 0; }
size_t hsb_history_select_capacity(const hsb_history* h) { return h ? h->kcap : 0; }

int hsb_history_append(hsb_history* h, size_t layer, uint64_t first, size_t count, const uint16_t* d_rows,
                       void* stream) {
    if (!h || layer >= h->layers.size()) return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA layer out of bounds");
    auto& L = h->layers[layer];
    const auto& c = h->cfg;
    // policy/full_gqa_runtime.cpp:472-476
    if (!count || !d_rows) return history_fail(HSB_E_HISTORY_PROTOCOL, "append after drain or empty append");
    if (first != L.completed || count > c.prompt_tokens + c.generated_capacity - L.completed)
        return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA incremental append range");
    if (L.job >= 0 && (count != 1 || first != h->jobs[L.job].position))
        return history_fail(HSB_E_HISTORY_PROTOCOL, "prefetched history permits only its current-token append");
    if ((reinterpret_cast<uintptr_t>(d_rows) & 15u) != 0)
        return history_fail(HSB_E_INVALID, "history rows must be 16-byte aligned");
    cudaError_t e = launch_dependent(history_append_kernel, dim3((unsigned)count), dim3(128), 0,
                                     static_cast<cudaStream_t>(stream), false, d_rows, (unsigned long long)first,
                                     (unsigned long long)count, (const int32_t*)L.slot, (const int32_t*)L.cold_row,
                                     L.pool, L.cold);
    if (e != cudaSuccess) return record_cuda_error(e, "history append launch");
    L.completed += count;
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_history_prepare(hsb_history* h, size_t layer, uint64_t position, const uint16_t* d_q16, void* stream) {
    if (!h || layer >= h->layers.size()) return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA layer out of bounds");
    auto& L = h->layers[layer];
    const auto& c = h->cfg;
    // policy/full_gqa_runtime.cpp:477-483
    if (!(position >= c.prompt_tokens && position < c.prompt_tokens + c.generated_capacity && L.completed == position))
        return history_fail(HSB_E_HISTORY_PROTOCOL, "history prefetch requires exactly completed past positions");
    int pending = 0, free_job = -1;
    for (int j = 0; j < 2; ++j) {
        if (h->jobs[j].used) ++pending;
        else if (free_job < 0) free_job = j;
    }
    if (pending >= 2 || L.job >= 0)
        return history_fail(HSB_E_HISTORY_PROTOCOL,
                            "at most two distinct full GQA history preparations may be outstanding");
    if (!d_q16) return history_fail(HSB_E_SCORE_SHAPE, "full GQA CPU query/views shape");
    auto& J = h->jobs[free_job];
    const auto s = static_cast<cudaStream_t>(stream);
    // The job starts once the caller's stream has the query and the rows.
    cudaError_t e = cudaEventRecord(J.inputs, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(h->work, J.inputs, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(J.query, d_q16, kHeads * kDim * 2, cudaMemcpyDeviceToDevice, h->work);
    if (e == cudaSuccess)
        e = score_runs(J.query, L.runs, position, L.pool, kRowWords, L.cold, kKeyWords, J.raw, c.capacity, J.keys,
                       h->work);
    if (e != cudaSuccess) return record_cuda_error(e, "history prepare launch");
    // The payload cover of the final selection (policy/full_gqa_runtime.cpp:299-344),
    // from the scorer's order keys: hsb_prefetch_cover's selection on its
    // normalised scores, without normalising them again.
    const size_t cap = std::min<size_t>(position, (size_t)std::floor(double(position + 1) * double(0.2f)));
    if (!cap) return history_fail(HSB_E_COVER_RANGE, "payload prefetch historical cap/range mismatch");
    SelectLaunch sl{};
    sl.scores = J.keys;
    sl.keys = 1;
    sl.tie_raw = J.raw;
    sl.cover = 1;
    sl.heads = kHeads;
    sl.stride = c.capacity;
    sl.valid = position;
    sl.alpha = c.alpha;
    sl.ratio = 1.0f;
    sl.fp32_counts = c.fp32_counts != 0;
    sl.ids = J.cover;
    sl.kcap = cap;
    sl.counts = nullptr;
    sl.result = J.cover_result;
    sl.workspace = h->cover_ws;
    sl.workspace_bytes = h->cover_ws_bytes;
    sl.cover_cap = cap;
    e = launch_select(sl, h->work);
    if (e != cudaSuccess) return record_cuda_error(e, "history cover launch");
    J.cap = cap;
    e = cudaEventRecord(J.ready, h->work);
    if (e != cudaSuccess) return record_cuda_error(e, "history prepare event");
    J.used = true;
    J.layer = layer;
    J.position = position;
    L.job = free_job;
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_history_cover(hsb_history* h, size_t layer, uint32_t* d_cold_ids, uint32_t* d_cold_count,
                      hsb_selection* d_cover_result, void* stream) {
    if (!h || layer >= h->layers.size()) return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA layer out of bounds");
    auto& L = h->layers[layer];
    if (L.job < 0) return history_fail(HSB_E_HISTORY_PROTOCOL, "no prepared history for this layer");
    auto& J = h->jobs[L.job];
    const auto s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamWaitEvent(s, J.ready, 0);
    if (e == cudaSuccess && d_cold_ids && d_cold_count)
        e = launch_dependent(history_cover_cold_kernel, dim3(1), dim3(1024), 0, s, false, (const uint32_t*)J.cover,
                             (unsigned long long)J.cap, (const hsb_selection*)J.cover_result, (const int32_t*)L.slot,
                             (unsigned long long)J.position, d_cold_ids, d_cold_count);
    if (e == cudaSuccess && d_cover_result)
        e = cudaMemcpyAsync(d_cover_result, J.cover_result, sizeof(hsb_selection), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return record_cuda_error(e, "history cover launch");
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_history_select(hsb_history* h, size_t layer, uint64_t position, const uint16_t* d_q16, uint32_t* d_ids,
                       size_t kcap, uint32_t* d_counts, hsb_selection* d_result, void* stream) {
    if (!h || layer >= h->layers.size()) return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA layer out of bounds");
    auto& L = h->layers[layer];
    const auto& c = h->cfg;
    // policy/full_gqa_runtime.cpp:550-552
    if (!(position >= c.prompt_tokens && position < c.prompt_tokens + c.generated_capacity &&
          L.completed == position + 1))
        return history_fail(HSB_E_HISTORY_PROTOCOL,
                            "full GQA selection requires current KV append and valid decode range");
    if (L.last_selected != std::numeric_limits<uint64_t>::max() && position <= L.last_selected)
        return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA duplicate/backwards layer selection");
    if (!d_q16 || !d_ids || !d_result) return history_fail(HSB_E_INVALID, "null selector buffer");
    const auto s = static_cast<cudaStream_t>(stream);
    uint16_t* raw = h->raw_direct;
    uint16_t* keys = h->keys_direct;
    cudaError_t e = cudaSuccess;
    if (L.job >= 0) {
        auto& J = h->jobs[L.job];
        if (J.position != position)
            return history_fail(HSB_E_HISTORY_PROTOCOL, "history Q/position differs from current same-query selection");
        raw = J.raw;
        keys = J.keys;
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, J.ready, 0);
        // the current token, an ordinary candidate (full_gqa_runtime.cpp:531-548)
        const Run current{0, 1, true, (uint64_t)L.row_of_position[position]};  // generated: always hot
        if (e == cudaSuccess)
            e = score_runs(d_q16, std::vector<Run>{current}, 1, L.pool, kRowWords, L.cold, kKeyWords, raw + position,
                           c.capacity, keys + position, s);
    } else if (e == cudaSuccess) {
        e = score_runs(d_q16, L.runs, position + 1, L.pool, kRowWords, L.cold, kKeyWords, raw, c.capacity, keys, s);
    }
    if (e != cudaSuccess) return record_cuda_error(e, "history select launch");
    // select_gqa_scores on the scorer's order keys (the raw scores break a
    // boundary tie between +0 and -0, as in the layer step)
    int rc = hsb_select_keys(keys, raw, kHeads, c.capacity, position + 1, c.alpha, 0.2f, c.fp32_counts, d_ids, kcap,
                             d_counts, d_result, h->select_ws, h->select_ws_bytes, stream);
    if (rc) return rc;
    if (L.job >= 0) {
        e = launch_dependent(history_query_check_kernel, dim3(1), dim3(256), 0, s, false,
                             (const uint16_t*)h->jobs[L.job].query, d_q16, d_result);
        if (e != cudaSuccess) return record_cuda_error(e, "history query check launch");
    }
    L.last_selected = position;
    record_error(HSB_OK, "");
    return HSB_OK;
}

int hsb_history_fetch(hsb_history* h, size_t layer, const uint32_t* d_ids, size_t kcap,
                      const hsb_selection* d_result, const uint32_t* d_staged_ids, size_t nstaged,
                      const uint16_t* d_staged_rows, size_t count, int zero_padding, uint16_t* d_k,
                      uint16_t* d_v, hsb_device_status* d_status, void* stream) {
    if (!h || layer >= h->layers.size()) return history_fail(HSB_E_HISTORY_PROTOCOL, "full GQA layer out of bounds");
    auto& L = h->layers[layer];
    if (!d_ids || !d_result || !d_k || !d_v || !d_status || !count || (nstaged && (!d_staged_ids || !d_staged_rows)))
        return history_fail(HSB_E_INVALID, "history fetch arguments");
    const auto s = static_cast<cudaStream_t>(stream);
    if (32 * count > h->map_capacity) {
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, 32 * count * sizeof(int32_t));
        if (e != cudaSuccess) return record_cuda_error(e, "history map allocation");
        if (h->map) {
            cudaStreamSynchronize(s);
            h->allocations.erase(std::find(h->allocations.begin(), h->allocations.end(), (void*)h->map));
            cudaFree(h->map);
        }
        h->map = keep(h, static_cast<int32_t*>(p));
        h->map_capacity = 32 * count;
    }
    const unsigned threads = 256;
    cudaError_t e = launch_dependent(history_map_kernel, dim3((unsigned)((32 * count + threads - 1) / threads)),
                                     dim3(threads), 0, s, false, d_ids, (unsigned long long)kcap, d_result,
                                     (const int32_t*)L.slot, (unsigned long long)L.completed, d_staged_ids,
                                     (unsigned long long)nstaged, (unsigned long long)count, h->map, d_status);
    if (e == cudaSuccess)
        e = launch_gather_map(L.pool, h->hot_slots, d_staged_rows ? d_staged_rows : L.pool, nstaged, h->map, count,
                              d_k, d_v, d_status, s, zero_padding, &d_result->k);
    if (e != cudaSuccess) return record_cuda_error(e, "history fetch launch");
    // The prepared job is consumed (policy/full_gqa_runtime.cpp:620-622).
    if (L.job >= 0) {
        h->jobs[L.job].used = false;
        L.job = -1;
    }
    record_error(HSB_OK, "");
    return HSB_OK;
}

}  // extern "C"
