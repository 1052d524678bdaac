// compat.cpp -- the reference's C++ interfaces for the selected-KV path
// (policy/full_gqa_cpu.hpp, policy/gqa_policy.hpp, runtime/gqa_pack.hpp,
// runtime/gqa_prefetch_cuda.hpp, runtime/gqa_delivery.hpp), implemented over
// the C ABI of include/hsb.h.  Host vectors in, host results out, exceptions
// as in the reference; device work is enqueued on private streams and
// completed before each synchronous call returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cfenv>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <mutex>
#include <stdexcept>
#include <string>

#include "hsb.h"
#include "hsb_compat.h"
#include "policy/full_gqa_cpu.hpp"
#include "policy/gqa_policy.hpp"
#include "policy/host_policy.hpp"
#include "runtime/gqa_delivery.hpp"
#include "runtime/gqa_h2o_stats.hpp"
#include "runtime/gqa_pack.hpp"
#include "runtime/gqa_prefetch_cuda.hpp"

namespace hillserve {
namespace {

using Clock = std::chrono::steady_clock;
std::uint64_t now_ns() {
    return std::chrono::duration_cast<std::chrono::nanoseconds>(Clock::now().time_since_epoch()).count();
}

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Maps an hsb status to the reference's exception type.
[[noreturn]] void throw_status(int status) {
    const std::string msg = hsb_last_error()[0] ? hsb_last_error() : hsb_status_message(status);
    switch (status) {
    case HSB_E_SCORE_SHAPE: case HSB_E_SCORE_ALIAS: case HSB_E_SCORE_V3_TOKENS:
    case HSB_E_UNION_BOUNDS: case HSB_E_UNION_DUPLICATE: case HSB_E_PACK_SHAPE:
    case HSB_E_PACK_PHYSICAL: case HSB_E_PACK_SLOTS: case HSB_E_PACK_MISSING:
        throw std::invalid_argument(msg);
    default:
        throw std::runtime_error(msg);
    }
}
void hsb_check(int status) {
    if (status != HSB_OK) throw_status(status);
}

bool is_device_pointer(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Growable device buffer.
struct DeviceBuffer {
    void* ptr = nullptr;
    std::size_t bytes = 0;
    ~DeviceBuffer() {
        if (ptr) cudaFree(ptr);
    }
    void* reserve(std::size_t n) {
        if (n > bytes) {
            if (ptr) cudaFree(ptr);
            ptr = nullptr;
            bytes = 0;
            cuda_check(cudaMalloc(&ptr, std::max<std::size_t>(n, 256)), "device allocation");
            bytes = std::max<std::size_t>(n, 256);
        }
        return ptr;
    }
    template <class T>
    T* as() const { return static_cast<T*>(ptr); }
};

struct Stream {
    cudaStream_t s = nullptr;
    Stream() { cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream"); }
    ~Stream() {
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    }
};

// Stream and scratch shared by the free functions of one thread.
struct ThreadContext {
    Stream stream;
    DeviceBuffer a, b, c, d, e, f, ws;
};
ThreadContext& tls() {
    static thread_local ThreadContext ctx;
    return ctx;
}

void h2d(void* dst, const void* src, std::size_t n, cudaStream_t s) {
    if (n) cuda_check(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, s), "host to device copy");
}
void d2h(void* dst, const void* src, std::size_t n, cudaStream_t s) {
    if (n) cuda_check(cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, s), "device to host copy");
}
void sync(cudaStream_t s) { cuda_check(cudaStreamSynchronize(s), "stream synchronize"); }

}  // namespace

// ------------------------------------------------------------ host_policy
float half_value(std::uint16_t h) {
    const std::uint32_t sign = std::uint32_t(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    std::uint32_t bits;
    if (e == 0) {
        float mag = std::ldexp(float(m), -24);
        std::memcpy(&bits, &mag, 4);
        bits |= sign;
    } else {
        bits = sign | (e == 31 ? (0x7f800000u | (m << 13)) : (((e + 112u) << 23) | (m << 13)));
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
std::uint16_t half_bits(float f) {
    std::uint32_t x;
    std::memcpy(&x, &f, 4);
    const std::uint16_t sign = std::uint16_t((x >> 16) & 0x8000u);
    const std::uint32_t e = (x >> 23) & 255u, m = x & 0x7fffffu;
    if (e == 255) return std::uint16_t(sign | 0x7c00u | (m ? 0x200u : 0u));
    const int he = int(e) - 112;
    if (he >= 31) return std::uint16_t(sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return sign;
        const std::uint32_t full = m | 0x800000u, sh = std::uint32_t(14 - he);
        std::uint32_t q = full >> sh;
        const std::uint32_t r = full & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        q += (r > half) || (r == half && (q & 1u));
        return std::uint16_t(sign | q);
    }
    std::uint32_t q = (std::uint32_t(he) << 10) | (m >> 13);
    const std::uint32_t r = m & 0x1fffu;
    q += (r > 0x1000u) || (r == 0x1000u && (q & 1u));
    return std::uint16_t(sign | q);
}

// ------------------------------------------------------------ scorer
struct FullGqaCpuScorer::Impl {
    unsigned count;
    std::mutex invocation;
    Stream stream;
    DeviceBuffer q, keys, out;
    std::vector<hsb_key_view> views;
};

FullGqaCpuScorer::FullGqaCpuScorer(unsigned threads, FullGqaCpuImplementation implementation) {
    // policy/full_gqa_cpu.cpp:153-163
    if (std::fegetround() != FE_TONEAREST)
        throw std::invalid_argument("full GQA CPU workers require round-to-nearest FP32 mode");
    if (threads == 0 || threads > 128) throw std::invalid_argument("full GQA CPU threads must be 1..128");
    if (implementation != FullGqaCpuImplementation::automatic && implementation != FullGqaCpuImplementation::scalar &&
        implementation != FullGqaCpuImplementation::avx2_f16c)
        throw std::invalid_argument("unknown full GQA CPU implementation");
    impl_.reset(new Impl{});
    impl_->count = threads;
}
FullGqaCpuScorer::~FullGqaCpuScorer() = default;
unsigned FullGqaCpuScorer::threads() const noexcept { return impl_->count; }
const char* FullGqaCpuScorer::implementation_name() const noexcept { return "sm100a_ordered_fp32"; }
std::size_t FullGqaCpuScorer::workspace_bytes() const noexcept {
    return sizeof(Impl) + impl_->q.bytes + impl_->keys.bytes + impl_->out.bytes;
}
bool FullGqaCpuScorer::avx2_f16c_available() noexcept { return true; }

void FullGqaCpuScorer::score(const std::vector<std::uint16_t>& q, const std::vector<FullGqaKeyView>& views,
                             std::vector<std::uint16_t>& result) {
    std::lock_guard<std::mutex> call(impl_->invocation);
    // policy/full_gqa_cpu.cpp:210-227, same order and messages
    if (std::fegetround() != FE_TONEAREST)
        throw std::invalid_argument("full GQA CPU scoring requires round-to-nearest FP32 mode");
    if (&q == &result) throw std::invalid_argument("full GQA CPU output must not alias the query");
    if (q.size() != 32 * 128 || views.empty()) throw std::invalid_argument("full GQA CPU query/views shape");
    std::size_t tokens = 0, host_tokens = 0;
    for (const auto& v : views) {
        if (!v.data || v.tokens == 0 || (v.token_stride_words != 1024 && v.token_stride_words != 2048) ||
            v.tokens > std::numeric_limits<std::size_t>::max() / v.token_stride_words ||
            v.tokens > std::numeric_limits<std::size_t>::max() / 32 - tokens)
            throw std::invalid_argument("full GQA CPU key view shape/stride/extent");
        tokens += v.tokens;
        if (!is_device_pointer(v.data)) host_tokens += v.tokens;
    }
    cudaStream_t s = impl_->stream.s;
    auto* dq = static_cast<std::uint16_t*>(impl_->q.reserve(4096 * 2));
    h2d(dq, q.data(), 4096 * 2, s);
    // Host views: stage only their K words (1024 per token) into one buffer.
    auto* staged = static_cast<std::uint16_t*>(impl_->keys.reserve(host_tokens * 2048 + 16));
    impl_->views.clear();
    std::size_t cursor = 0;
    for (const auto& v : views) {
        if (is_device_pointer(v.data)) {
            impl_->views.push_back({v.data, v.tokens, v.token_stride_words});
            continue;
        }
        cuda_check(cudaMemcpy2DAsync(staged + cursor * 1024, 2048, v.data, v.token_stride_words * 2, 2048, v.tokens,
                                     cudaMemcpyHostToDevice, s),
                   "key staging");
        impl_->views.push_back({staged + cursor * 1024, v.tokens, 1024});
        cursor += v.tokens;
    }
    auto* dout = impl_->out.reserve(tokens * 32 * 2);
    hsb_check(hsb_score_views(dq, impl_->views.data(), impl_->views.size(), static_cast<std::uint16_t*>(dout), s));
    result.resize(tokens * 32);
    d2h(result.data(), dout, tokens * 32 * 2, s);
    sync(s);
}

std::vector<std::uint16_t> score_full_gqa_legacy_cpu(const std::vector<std::uint16_t>& q, const std::uint16_t* input,
                                                     std::size_t n, std::size_t token_stride, unsigned threads) {
    // policy/full_gqa_cpu.cpp:111-118
    if (!(q.size() == 32 * 128 && input && n > 0 && (token_stride == 1024 || token_stride == 2048) && threads >= 1 &&
          threads <= 32))
        throw std::invalid_argument("raw128 physical GQA CPU shape/stride/thread bound");
    if (n > std::numeric_limits<std::size_t>::max() / 32 || n > std::numeric_limits<std::size_t>::max() / token_stride)
        throw std::invalid_argument("legacy full GQA CPU extent overflow");
    if (std::fegetround() != FE_TONEAREST)
        throw std::invalid_argument("legacy full GQA CPU requires round-to-nearest FP32 mode");
    static thread_local std::unique_ptr<FullGqaCpuScorer> scorer;
    if (!scorer) scorer.reset(new FullGqaCpuScorer(1));
    std::vector<std::uint16_t> out;
    scorer->score(q, {{input, n, token_stride}}, out);
    return out;
}

// ------------------------------------------------------------ selector
namespace policy {
GQASelection select_gqa_scores(const std::vector<std::uint16_t>& score, std::size_t h, std::size_t stride,
                               std::size_t n, float alpha, float ratio, bool fp32_counts) {
    // policy/gqa_policy.cpp:48-49 shape checks (incl. the vector size)
    if (!(h > 0 && h <= 128 && n > 0 && n <= stride && score.size() == h * stride))
        throw std::runtime_error("GQA selector shape");
    if (!(std::isfinite(alpha) && alpha >= 0 && std::isfinite(ratio) && ratio > 0 && ratio <= 1))
        throw std::runtime_error("GQA selector numeric parameters");
    auto& c = tls();
    cudaStream_t s = c.stream.s;
    const std::size_t kcap = std::max<std::size_t>(1, std::min<std::size_t>(std::floor(double(n) * double(ratio)), n));
    auto* dscores = c.a.reserve(score.size() * 2);
    auto* dids = c.b.reserve(h * kcap * 4);
    auto* dcounts = c.c.reserve(h * 4);
    auto* dres = c.d.reserve(sizeof(hsb_selection));
    const std::size_t wsb = hsb_select_workspace_bytes(h, stride, n, kcap);
    auto* ws = c.ws.reserve(wsb);
    h2d(dscores, score.data(), score.size() * 2, s);
    const int rc = hsb_select(static_cast<const std::uint16_t*>(dscores), 0, h, stride, n, alpha, ratio, fp32_counts,
                              static_cast<std::uint32_t*>(dids), kcap, static_cast<std::uint32_t*>(dcounts),
                              static_cast<hsb_selection*>(dres), ws, c.ws.bytes, s);
    if (rc) throw std::runtime_error(hsb_last_error());
    hsb_selection res{};
    const int st = hsb_selection_read(static_cast<hsb_selection*>(dres), &res, s);
    if (st) throw std::runtime_error(hsb_last_error());
    GQASelection r;
    r.k = res.k;
    r.boundary_tied_heads = res.boundary_tied_heads;
    r.counts.resize(h);
    std::vector<std::uint32_t> ids(h * kcap);
    d2h(r.counts.data(), dcounts, h * 4, s);
    d2h(ids.data(), dids, h * kcap * 4, s);
    sync(s);
    r.ids.resize(h);
    for (std::size_t head = 0; head < h; ++head)
        r.ids[head].assign(ids.begin() + head * kcap, ids.begin() + head * kcap + r.k);
    return r;
}
}  // namespace policy

// ------------------------------------------------------------ union / pack
namespace {
// Flattens ragged per-head lists into [32][kstride] u32 + sizes, as the
// device kernels read them.  IDs >= 2^32 cannot be admitted (visible <= 66048).
void flatten_ids(const std::vector<std::vector<std::uint64_t>>& ids, std::vector<std::uint32_t>& flat,
                 std::vector<std::uint32_t>& sizes, std::size_t& kstride, std::uint32_t out_of_range) {
    kstride = 1;
    for (const auto& h : ids) kstride = std::max(kstride, h.size());
    flat.assign(32 * kstride, 0);
    sizes.assign(32, 0);
    for (std::size_t h = 0; h < ids.size() && h < 32; ++h) {
        sizes[h] = std::uint32_t(ids[h].size());
        for (std::size_t s = 0; s < ids[h].size(); ++s)
            flat[h * kstride + s] = ids[h][s] > 0xffffffffull ? out_of_range : std::uint32_t(ids[h][s]);
    }
}
}  // namespace

std::vector<std::uint64_t> gqa_physical_union(const std::vector<std::vector<std::uint64_t>>& ids, std::size_t visible) {
    if (ids.size() != 32 || !visible || visible > 66048) throw std::invalid_argument("GQA union bounds");
    std::vector<std::uint32_t> flat, sizes;
    std::size_t kstride;
    flatten_ids(ids, flat, sizes, kstride, 0xffffffffu);
    auto& c = tls();
    cudaStream_t s = c.stream.s;
    auto* dids = c.a.reserve(flat.size() * 4);
    auto* dsizes = c.b.reserve(32 * 4);
    auto* dphys = c.c.reserve(visible * 4);
    auto* dcount = c.d.reserve(16);
    auto* dstatus = c.e.reserve(sizeof(hsb_device_status));
    auto* ws = c.ws.reserve(hsb_union_workspace_bytes(visible));
    h2d(dids, flat.data(), flat.size() * 4, s);
    h2d(dsizes, sizes.data(), 32 * 4, s);
    cuda_check(cudaMemsetAsync(dstatus, 0, sizeof(hsb_device_status), s), "status reset");
    hsb_check(hsb_union(static_cast<std::uint32_t*>(dids), kstride, static_cast<std::uint32_t*>(dsizes), 1, visible,
                        static_cast<std::uint32_t*>(dphys), static_cast<std::uint32_t*>(dcount),
                        static_cast<hsb_device_status*>(dstatus), ws, c.ws.bytes, s));
    hsb_check(hsb_status_check(static_cast<hsb_device_status*>(dstatus), s));
    std::uint32_t count = 0;
    d2h(&count, dcount, 4, s);
    sync(s);
    std::vector<std::uint32_t> phys(count);
    d2h(phys.data(), dphys, count * 4, s);
    sync(s);
    return std::vector<std::uint64_t>(phys.begin(), phys.end());
}

void pack_gqa_workspace(const std::vector<std::vector<std::uint64_t>>& ids, const std::vector<std::uint64_t>& positions,
                        const std::vector<std::uint64_t>& physical, const std::vector<std::uint8_t>& payload,
                        std::size_t count, std::uint16_t* k, std::uint16_t* v, float* mask) {
    // runtime/gqa_pack.hpp:29-30
    if (ids.size() != 32 || positions.empty() || positions.size() > 256 || positions.back() >= 66048 || !count ||
        count > 66048 || payload.size() != physical.size() * 4096)
        throw std::invalid_argument("GQA packing shape");
    const std::uint64_t last = positions.back();
    std::vector<std::uint32_t> flat, sizes, phys(physical.size());
    std::size_t kstride;
    flatten_ids(ids, flat, sizes, kstride, 0xffffffffu);
    for (std::size_t i = 0; i < physical.size(); ++i)
        phys[i] = physical[i] > 0xffffffffull ? 0xffffffffu : std::uint32_t(physical[i]);
    auto& c = tls();
    cudaStream_t s = c.stream.s;
    const std::size_t qpad = (positions.size() + 63) / 64 * 64;
    auto* dids = c.a.reserve(flat.size() * 4);
    auto* dsizes = c.b.reserve(32 * 4);
    auto* dpos = c.f.reserve(positions.size() * 8);
    auto* dphys = c.c.reserve(phys.size() * 4 + 16);
    auto* dpayload = c.d.reserve(payload.size() + 16);
    auto* dout = static_cast<std::uint8_t*>(c.e.reserve(count * 4096 * 4 + count * qpad * 32 * 4 + 512));
    auto* dk = reinterpret_cast<std::uint16_t*>(dout);
    auto* dv = dk + count * 4096;
    auto* dmask = reinterpret_cast<float*>(dv + count * 4096);
    auto* dstatus = reinterpret_cast<hsb_device_status*>(dmask + count * qpad * 32);
    auto* ws = c.ws.reserve(hsb_pack_workspace_bytes(last));
    h2d(dids, flat.data(), flat.size() * 4, s);
    h2d(dsizes, sizes.data(), 32 * 4, s);
    h2d(dpos, positions.data(), positions.size() * 8, s);
    h2d(dphys, phys.data(), phys.size() * 4, s);
    h2d(dpayload, payload.data(), payload.size(), s);
    cuda_check(cudaMemsetAsync(dstatus, 0, sizeof(hsb_device_status), s), "status reset");
    hsb_check(hsb_pack(static_cast<std::uint32_t*>(dids), kstride, static_cast<std::uint32_t*>(dsizes), 1,
                       reinterpret_cast<const std::uint64_t*>(dpos), positions.size(), last,
                       static_cast<std::uint32_t*>(dphys), phys.size(), static_cast<std::uint8_t*>(dpayload),
                       payload.size(), count, dk, dv, dmask, dstatus, ws, c.ws.bytes, s));
    hsb_check(hsb_status_check(dstatus, s));
    d2h(k, dk, count * 4096 * 2, s);
    d2h(v, dv, count * 4096 * 2, s);
    d2h(mask, dmask, count * qpad * 32 * 4, s);
    sync(s);
}

// ------------------------------------------------------------ prefetch
namespace {
// Makes `device` current for one scope and restores the caller's device.
struct DeviceScope {
    int previous = 0;
    bool restore = false;
    explicit DeviceScope(int device) {
        cuda_check(cudaGetDevice(&previous), "get CUDA device");
        restore = previous != device;
        if (restore) cuda_check(cudaSetDevice(device), "set CUDA device");
    }
    ~DeviceScope() {
        if (restore) cudaSetDevice(previous);
    }
};
// Pinned host memory (page-locked, so copies run asynchronously).
struct PinnedBuffer {
    unsigned char* ptr = nullptr;
    explicit PinnedBuffer(std::size_t bytes) {
        cuda_check(cudaMallocHost(reinterpret_cast<void**>(&ptr), std::max<std::size_t>(bytes, 256)),
                   "pinned host allocation");
    }
    ~PinnedBuffer() {
        if (ptr) cudaFreeHost(ptr);
    }
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
};
struct Event {
    cudaEvent_t e = nullptr;
    explicit Event(unsigned flags = cudaEventDefault) {
        cuda_check(cudaEventCreateWithFlags(&e, flags), "event");
    }
    ~Event() {
        if (e) cudaEventDestroy(e);
    }
    Event(const Event&) = delete;
    Event& operator=(const Event&) = delete;
};
// A borrowed stream that may still run work of ours: drained before the
// buffers that work uses are released.
struct BorrowedStream {
    cudaStream_t stream = nullptr;
    void hold(cudaStream_t s) { stream = s; }
    void release() { stream = nullptr; }
    void drain() noexcept {
        if (stream && cudaStreamSynchronize(stream) == cudaSuccess) stream = nullptr;
    }
};
}  // namespace

// Members are declared so that destruction runs streams and the borrowed
// consumer first (each drains its work) and frees memory last.
struct GQAPrefetchCuda::Impl {
    int device = 0;
    std::size_t rows = 0, slot_bytes = 0;
    // Both slots' rows: one HBM region and one pinned region, slot s at s * slot_bytes.
    DeviceBuffer staged;
    std::unique_ptr<PinnedBuffer> pinned;
    // A delivery's inputs travel in one copy: [status word | map | miss rows]
    // (the pinned arena starts with a zero status word); the status comes
    // back into the last 8 bytes of the pinned arena.
    std::size_t map_off = 256, miss_off = 0, arena_bytes = 0;
    DeviceBuffer arena;
    std::unique_ptr<PinnedBuffer> arena_host;
    std::unique_ptr<Event> delivered;
    struct Queue {
        std::unique_ptr<Stream> stream;
        std::unique_ptr<Event> start, ready;
        std::size_t rows = 0;
    };
    Queue queue[2];
    BorrowedStream consumer;
    ~Impl() {
        try {
            DeviceScope scope(device);
            consumer.drain();
            for (auto& q : queue) q.stream.reset();  // synchronises the slot's upload
        } catch (...) {
        }
    }
};

GQAPrefetchCuda::GQAPrefetchCuda(void* pointer, std::size_t max_rows) : impl_(new Impl) {
    auto& p = *impl_;
    cudaPointerAttributes a{};
    cuda_check(cudaPointerGetAttributes(&a, pointer), "prefetch GPU pointer attributes");
    if (a.type != cudaMemoryTypeDevice) throw std::runtime_error("prefetch target must be CUDA device memory");
    p.device = a.device;
    p.rows = max_rows;
    p.slot_bytes = max_rows * 4096;
    DeviceScope scope(p.device);
    p.staged.reserve(2 * p.slot_bytes);
    p.pinned.reset(new PinnedBuffer(2 * p.slot_bytes));
    p.miss_off = p.map_off + (max_rows * 32 * 4 + 255) / 256 * 256;
    p.arena_bytes = p.miss_off + p.slot_bytes;
    p.arena.reserve(p.arena_bytes);
    p.arena_host.reset(new PinnedBuffer(p.arena_bytes + 8));
    std::memset(p.arena_host->ptr, 0, p.map_off);
    p.delivered.reset(new Event(cudaEventDisableTiming));
    for (auto& q : p.queue) {
        q.stream.reset(new Stream);
        q.start.reset(new Event);
        q.ready.reset(new Event);
    }
}
GQAPrefetchCuda::~GQAPrefetchCuda() = default;
std::size_t GQAPrefetchCuda::gpu_bytes() const { return impl_->slot_bytes * 3 + impl_->rows * 32 * 4; }
std::size_t GQAPrefetchCuda::host_bytes() const { return impl_->slot_bytes * 2; }

GQAPrefetchCuda::Upload GQAPrefetchCuda::stage(unsigned slot, const std::vector<std::uint8_t>& payload) {
    auto& p = *impl_;
    if (slot >= 2 || payload.size() > p.slot_bytes || payload.size() % 4096)
        throw std::runtime_error("prefetch CUDA slot geometry");
    DeviceScope scope(p.device);
    auto& q = p.queue[slot];
    unsigned char* host = p.pinned->ptr + slot * p.slot_bytes;
    unsigned char* dev = p.staged.as<unsigned char>() + slot * p.slot_bytes;
    if (!payload.empty()) std::memcpy(host, payload.data(), payload.size());
    Upload out;
    out.started_ns = now_ns();
    out.bytes = payload.size();
    q.rows = payload.size() / 4096;
    const cudaStream_t s = q.stream->s;
    try {
        cuda_check(cudaEventRecord(q.start->e, s), "prefetch upload start");
        h2d(dev, host, payload.size(), s);
        cuda_check(cudaEventRecord(q.ready->e, s), "prefetch ready record");
        cuda_check(cudaEventSynchronize(q.ready->e), "prefetch upload completion");
    } catch (...) {
        cudaStreamSynchronize(s);  // the pinned rows stay in use until the copy is over
        throw;
    }
    out.ready_observed_ns = now_ns();
    cuda_check(cudaEventElapsedTime(&out.device_ms, q.start->e, q.ready->e), "prefetch upload interval");
    return out;
}

GQAPrefetchCuda::Delivery GQAPrefetchCuda::deliver(unsigned slot, const std::vector<std::int32_t>& rows,
                                                   const std::vector<std::uint8_t>& misses, const float* mask,
                                                   std::size_t mask_elements, std::size_t count, void* k, void* v,
                                                   void* gpu_mask, void* raw_stream) {
    auto& p = *impl_;
    // runtime/gqa_prefetch_cuda.cu:217-218: geometry, then every map entry.
    if (slot >= 2 || !raw_stream || count > p.rows || rows.size() != count * 32 || misses.size() > p.slot_bytes ||
        misses.size() % 4096)
        throw std::runtime_error("prefetch CUDA delivery geometry/stream");
    const std::size_t staged_rows = p.queue[slot].rows, miss_rows = misses.size() / 4096;
    std::size_t live = 0;
    for (const std::int32_t r : rows) {
        if (r >= 0 && static_cast<std::size_t>(r) >= staged_rows)
            throw std::runtime_error("prefetch row outside uploaded payload");
        if (r <= -2 && static_cast<std::size_t>(-2 - static_cast<long long>(r)) >= miss_rows)
            throw std::runtime_error("prefetch miss row outside payload");
        live += r != -1;
    }
    DeviceScope scope(p.device);
    const auto stream = static_cast<cudaStream_t>(raw_stream);
    unsigned char* host = p.arena_host->ptr;
    unsigned char* dev = p.arena.as<unsigned char>();
    std::memcpy(host + p.map_off, rows.data(), rows.size() * 4);
    if (!misses.empty()) std::memcpy(host + p.miss_off, misses.data(), misses.size());
    const std::size_t copy_bytes = misses.empty() ? p.map_off + rows.size() * 4 : p.miss_off + misses.size();
    auto* status = reinterpret_cast<hsb_device_status*>(dev);
    auto* status_back = reinterpret_cast<hsb_device_status*>(host + p.arena_bytes);
    Delivery out;
    out.started_ns = now_ns();
    p.consumer.hold(stream);
    try {
        cuda_check(cudaStreamWaitEvent(stream, p.queue[slot].ready->e, 0), "attention stream waits for prefetched payload");
        h2d(dev, host, copy_bytes, stream);  // zero status, map, miss rows
        if (mask_elements) h2d(gpu_mask, mask, mask_elements * 4, stream);
        hsb_check(hsb_gather_map(p.staged.as<std::uint16_t>() + slot * p.slot_bytes / 2, staged_rows,
                                 reinterpret_cast<const std::uint16_t*>(dev + p.miss_off), miss_rows,
                                 reinterpret_cast<const std::int32_t*>(dev + p.map_off), count,
                                 static_cast<std::uint16_t*>(k), static_cast<std::uint16_t*>(v), status, stream));
        d2h(status_back, status, sizeof(hsb_device_status), stream);
        cuda_check(cudaEventRecord(p.delivered->e, stream), "prefetch delivery completion record");
        const auto wait = Clock::now();
        cuda_check(cudaEventSynchronize(p.delivered->e), "prefetch delivery completion");
        out.wait_ms = std::chrono::duration<double, std::milli>(Clock::now() - wait).count();
    } catch (...) {
        p.consumer.drain();
        throw;
    }
    p.consumer.release();
    if (status_back->code != HSB_OK) throw_status(status_back->code);
    out.ready_observed_ns = now_ns();
    out.h2d_bytes = misses.size() + rows.size() * 4 + mask_elements * 4;
    out.d2d_bytes = live * 128 * 4;
    return out;
}

// ------------------------------------------------------------ delivery
struct GQADeliveryWorkspace::Impl {
    std::size_t count = 0;
    Stream stream;
    DeviceBuffer q, k, v, mask, ids, sizes, pos, phys, payload, status, out, ws;
    std::vector<float> output;
    std::uint64_t packed = 0;
};

GQADeliveryWorkspace::GQADeliveryWorkspace(std::size_t count, const std::vector<float>& actual) : p(new Impl) {
    // runtime/gqa_delivery.cpp:13,21
    if (!(count > 0 && count <= 6592 && count % 32 == 0 && actual.size() == 4096))
        throw std::runtime_error("bounded real GQA delivery shape");
    p->count = count;
    p->q.reserve(4096 * 4);
    p->k.reserve(count * 4096 * 2);
    p->v.reserve(count * 4096 * 2);
    p->mask.reserve(count * 64 * 32 * 4);
    p->out.reserve(4096 * 4);
    p->status.reserve(sizeof(hsb_device_status));
    p->ws.reserve(std::max(hsb_attention_workspace_bytes(count), hsb_pack_workspace_bytes(66047)));
    if (gpu_bytes() > 256ull * 1024 * 1024) throw std::runtime_error("GPU workspace budget");
    h2d(p->q.ptr, actual.data(), 4096 * 4, p->stream.s);
    sync(p->stream.s);
}
GQADeliveryWorkspace::~GQADeliveryWorkspace() = default;
std::uint64_t GQADeliveryWorkspace::gpu_bytes() const {
    return p->k.bytes + p->v.bytes + p->mask.bytes + p->q.bytes + p->out.bytes;
}
const std::vector<float>& GQADeliveryWorkspace::output() const { return p->output; }

GQADeliveryResult GQADeliveryWorkspace::deliver(const std::vector<std::vector<std::uint64_t>>& ids,
                                                std::uint64_t position, const std::vector<std::uint64_t>& physical,
                                                const std::vector<std::uint8_t>& payload) {
    GQADeliveryResult r;
    const auto t0 = Clock::now();
    if (ids.size() != 32 || position >= 66048 || payload.size() != physical.size() * 4096)
        throw std::invalid_argument("GQA packing shape");
    std::vector<std::uint32_t> flat, sizes, phys(physical.size());
    std::size_t kstride;
    flatten_ids(ids, flat, sizes, kstride, 0xffffffffu);
    for (std::size_t i = 0; i < physical.size(); ++i)
        phys[i] = physical[i] > 0xffffffffull ? 0xffffffffu : std::uint32_t(physical[i]);
    cudaStream_t s = p->stream.s;
    auto* dids = p->ids.reserve(flat.size() * 4);
    auto* dsizes = p->sizes.reserve(32 * 4);
    auto* dpos = p->pos.reserve(8);
    auto* dphys = p->phys.reserve(phys.size() * 4 + 16);
    auto* dpayload = p->payload.reserve(payload.size() + 16);
    h2d(dids, flat.data(), flat.size() * 4, s);
    h2d(dsizes, sizes.data(), 32 * 4, s);
    h2d(dpos, &position, 8, s);
    h2d(dphys, phys.data(), phys.size() * 4, s);
    h2d(dpayload, payload.data(), payload.size(), s);
    cuda_check(cudaMemsetAsync(p->status.ptr, 0, sizeof(hsb_device_status), s), "status reset");
    hsb_check(hsb_pack(static_cast<std::uint32_t*>(dids), kstride, static_cast<std::uint32_t*>(dsizes), 1,
                       static_cast<std::uint64_t*>(dpos), 1, position, static_cast<std::uint32_t*>(dphys),
                       phys.size(), static_cast<std::uint8_t*>(dpayload), payload.size(), p->count,
                       p->k.as<std::uint16_t>(), p->v.as<std::uint16_t>(), p->mask.as<float>(),
                       p->status.as<hsb_device_status>(), p->ws.ptr, p->ws.bytes, s));
    hsb_check(hsb_status_check(p->status.as<hsb_device_status>(), s));
    r.pack_ms = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    r.gpu_ready_ns = now_ns();
    r.upload_bytes = flat.size() * 4 + 32 * 4 + 8 + phys.size() * 4 + payload.size();
    r.upload_wall_ms = r.pack_ms;
    p->packed = 1;
    return r;
}

std::string GQADeliveryWorkspace::verify_and_consume() {
    if (!p->packed) throw std::runtime_error("nothing delivered");
    cudaStream_t s = p->stream.s;
    const auto t0 = Clock::now();
    hsb_check(hsb_attention_packed(p->q.as<float>(), p->k.as<std::uint16_t>(), p->v.as<std::uint16_t>(), p->count,
                                   p->mask.as<float>(), 64, nullptr, 0, p->out.as<float>(), p->ws.ptr, p->ws.bytes, s));
    p->output.resize(4096);
    d2h(p->output.data(), p->out.ptr, 4096 * 4, s);
    sync(s);
    const double ms = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    std::uint64_t h = 1469598103934665603ull;  // FNV-1a over the output bytes
    const auto* b = reinterpret_cast<const unsigned char*>(p->output.data());
    for (std::size_t i = 0; i < 4096 * 4; ++i) h = (h ^ b[i]) * 1099511628211ull;
    for (float x : p->output)
        if (!std::isfinite(x)) throw std::runtime_error("actual attention produced nonfinite output");
    char buf[256];
    std::snprintf(buf, sizeof buf,
                  "{\"attention_output_checksum\":\"%llu\",\"attention_after_delivery_ms_excluded\":%.6f,"
                  "\"attention\":\"sm100a split-K flash-decode\"}",
                  static_cast<unsigned long long>(h), ms);
    return buf;
}

// ------------------------------------------------------- H2O statistics
// The interface of runtime/gqa_h2o_stats.hpp over hsb_h2o_group_sums: the
// reduction and the copy of the sums to pinned memory run on the caller's
// attention stream, bracketed by three timing events.
struct GQAH2OStatsCuda::Impl {
    int device = 0;
    std::size_t keys = 0, bytes = 0;
    DeviceBuffer sums;
    std::unique_ptr<PinnedBuffer> host;
    std::unique_ptr<Event> begin, reduced, copied;
    BorrowedStream consumer;
    ~Impl() {
        // Never throws; a reduction that failed before its completion event
        // may still use the buffers on the borrowed stream: drain it first.
        try {
            DeviceScope scope(device);
            consumer.drain();
        } catch (...) {
        }
    }
};

GQAH2OStatsCuda::GQAH2OStatsCuda(const void* reference, std::size_t capacity) : impl_(new Impl) {
    if (!reference || !capacity) throw std::runtime_error("H2O statistics needs CUDA pointer and nonzero capacity");
    auto& p = *impl_;
    if (capacity > std::numeric_limits<std::size_t>::max() / (8 * sizeof(float)))
        throw std::runtime_error("H2O attention statistics size overflow");
    p.keys = capacity;
    p.bytes = capacity * 8 * sizeof(float);
    cudaPointerAttributes a{};
    cuda_check(cudaPointerGetAttributes(&a, reference), "H2O reference pointer attributes");
    if (a.type != cudaMemoryTypeDevice) throw std::runtime_error("H2O attention statistics requires CUDA device memory");
    p.device = a.device;
    DeviceScope scope(p.device);
    p.sums.reserve(p.bytes);
    p.host.reset(new PinnedBuffer(p.bytes));
    p.begin.reset(new Event);
    p.reduced.reset(new Event);
    p.copied.reset(new Event);
}
GQAH2OStatsCuda::~GQAH2OStatsCuda() = default;
std::size_t GQAH2OStatsCuda::gpu_bytes() const noexcept { return impl_->bytes; }
std::size_t GQAH2OStatsCuda::host_bytes() const noexcept { return impl_->bytes; }

GQAH2OStatsCuda::Result GQAH2OStatsCuda::reduce(const void* probabilities, const std::array<std::int64_t, 4>& ne,
                                                const std::array<std::size_t, 4>& nb, std::size_t keys,
                                                std::size_t queries, void* raw_stream) {
    auto& p = *impl_;
    // The C ABI takes a null stream as the default stream; the reference
    // requires the attention backend's own stream.
    if (!raw_stream) throw std::runtime_error("H2O reduction invalid pointer, actual CUDA stream or capacity");
    DeviceScope scope(p.device);
    const auto stream = static_cast<cudaStream_t>(raw_stream);
    Result out;
    out.started_ns = now_ns();
    float* sums = p.sums.as<float>();
    cuda_check(cudaEventRecord(p.begin->e, stream), "H2O reduction start record");
    const int rc = hsb_h2o_group_sums(probabilities, ne.data(), nb.data(), keys, queries, sums, p.keys, nullptr,
                                      stream);
    if (rc != HSB_OK) throw_status(rc);  // rejected before any launch: nothing of ours uses the buffers
    out.elements = keys * 8;
    out.d2h_bytes = out.elements * sizeof(float);
    p.consumer.hold(stream);
    try {
        cuda_check(cudaEventRecord(p.reduced->e, stream), "H2O reduction ready record");
        d2h(p.host->ptr, sums, out.d2h_bytes, stream);
        cuda_check(cudaEventRecord(p.copied->e, stream), "H2O D2H ready record");
        cuda_check(cudaEventSynchronize(p.copied->e), "H2O group sums completion");
    } catch (...) {
        p.consumer.drain();
        throw;
    }
    p.consumer.release();
    out.ready_observed_ns = now_ns();
    float reduction_ms = 0, d2h_ms = 0;
    cuda_check(cudaEventElapsedTime(&reduction_ms, p.begin->e, p.reduced->e), "H2O reduction interval");
    cuda_check(cudaEventElapsedTime(&d2h_ms, p.reduced->e, p.copied->e), "H2O D2H interval");
    out.reduction_ms = reduction_ms;
    out.d2h_ms = d2h_ms;
    out.sums = reinterpret_cast<const float*>(p.host->ptr);
    return out;
}

}  // namespace hillserve

// ------------------------------------------------------- C handles
namespace {
void copy_message(const std::exception& e, char* err, std::size_t errlen) {
    if (err && errlen) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = 0;
    }
}
}  // namespace

extern "C" {
void* hsb_compat_h2o_create(const void* pointer, std::size_t capacity, char* err, std::size_t errlen) {
    try {
        return new hillserve::GQAH2OStatsCuda(pointer, capacity);
    } catch (const std::exception& e) {
        copy_message(e, err, errlen);
        return nullptr;
    }
}
void hsb_compat_h2o_destroy(void* reducer) { delete static_cast<hillserve::GQAH2OStatsCuda*>(reducer); }
int hsb_compat_h2o_reduce(void* reducer, const void* probabilities, const std::int64_t ne[4], const std::size_t nb[4],
                          std::size_t keys, std::size_t queries, void* stream, const float** sums,
                          double* reduction_ms, double* d2h_ms, char* err, std::size_t errlen) {
    try {
        if (!reducer || !ne || !nb) throw std::runtime_error("H2O reduction invalid pointer, actual CUDA stream or capacity");
        const std::array<std::int64_t, 4> n{{ne[0], ne[1], ne[2], ne[3]}};
        const std::array<std::size_t, 4> b{{nb[0], nb[1], nb[2], nb[3]}};
        const auto r = static_cast<hillserve::GQAH2OStatsCuda*>(reducer)->reduce(probabilities, n, b, keys, queries,
                                                                               stream);
        if (sums) *sums = r.sums;
        if (reduction_ms) *reduction_ms = r.reduction_ms;
        if (d2h_ms) *d2h_ms = r.d2h_ms;
        return 0;
    } catch (const std::exception& e) {
        copy_message(e, err, errlen);
        return 1;
    }
}
}
