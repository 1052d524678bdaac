// internal.h -- host-side declarations shared by the kernel files and the
// C-ABI layer (capi.cu).  Not installed; the public interface is hsb.h.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "hsb.h"

namespace hsb {

struct DeviceInfo {
    int ordinal = -1;
    int sms = 0;
    int major = 0, minor = 0;
    size_t smem_optin = 0;
};
// Properties of the current device, cached per device.
const DeviceInfo& device_info();
// cuTensorMapEncodeTiled resolved through the runtime (no libcuda link);
// null when the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Launch with programmatic stream serialization (the kernel calls pdl_wait()
// before touching global memory), optionally cooperative.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             bool cooperative, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Stage 1
// keys (optional): also writes order_key(F16(raw / sqrtf(128))) per score, the
// selector's input in the fused layer step.
// Extra duties of the scorer inside the fused layer step:
//  - h0: per-CTA head-0 partials, h0[b] = (non-finite seen << 16) | max order
//    key of query head 0 over CTA b's tokens (0 when none); entries from the
//    grid size to kH0Partials are written 0.  Needs keys.
//  - zero[i] / zero_words[i]: small buffers (selector header, selection
//    result, attention counters) cleared by CTA 0 before any use downstream.
constexpr unsigned kH0Partials = 1024;
struct ScoreExtras {
    uint32_t* h0 = nullptr;
    uint32_t* zero[3] = {nullptr, nullptr, nullptr};
    unsigned zero_words[3] = {0, 0, 0};
};
cudaError_t launch_score(const uint16_t* q, const hsb_key_view* views, size_t nviews,
                         uint16_t* out, size_t out_stride, size_t col0,
                         hsb_device_status* status, cudaStream_t stream, uint16_t* keys = nullptr,
                         const ScoreExtras* extras = nullptr);
// A KV-head shard: keys_cache rows hold kv_heads (1, 2, 4 or 8) KV heads of
// 128 channels; q holds the shard's 4 * kv_heads query heads; out / keys are
// [4 * kv_heads][tokens].  extras->h0 when the shard holds query head 0.
// batch > 1: that many sequences back to back (keys_cache [batch][tokens],
// q [batch][4 kv_heads][128], out / keys [batch][4 kv_heads][tokens],
// extras->h0 [batch][kH0Partials]).
struct ThresholdPush;
cudaError_t launch_score_shard(const uint16_t* q, int kv_heads, const uint16_t* keys_cache, size_t tokens,
                               size_t stride_words, uint16_t* out, uint16_t* keys, hsb_device_status* status,
                               const ScoreExtras* extras, cudaStream_t stream, size_t batch = 1,
                               const ThresholdPush* push = nullptr);
cudaError_t launch_scale(const uint16_t* raw, size_t count, uint16_t* out, cudaStream_t stream);
// Tensor map of a token-major [tokens][8][128] F16 cache seen as {channel,
// token, KV head} with 64 x 32 x 8 boxes and the 128-byte swizzle (the
// scorer's tiles).  False if it cannot be encoded.
bool encode_kv_map(CUtensorMap* map, const uint16_t* data, size_t tokens, size_t stride_words);

// Stage 2
// Sets the thread-local message read by hsb_last_error() and returns status
// (record_cuda_error: HSB_E_CUDA with the runtime's error string appended).
int record_error(int status, const char* message);
int record_cuda_error(cudaError_t e, const char* what);

// Optional epilogue of the cluster selector (the layer step): gather each
// head's selected K/V rows from the cache into the packed layout and attend
// over them, writing out[32][128].
struct SelectEpilogue {
    const float* q = nullptr;  // F32 [32][128]
    const uint16_t* kcache = nullptr;
    const uint16_t* vcache = nullptr;
    size_t stride_words = 0;
    uint16_t* kp = nullptr;  // [count][32][128]
    uint16_t* vp = nullptr;  // [32][128][count]
    size_t count = 0;
    float* out = nullptr;    // null: no epilogue
    float scale = 0.0f;
    unsigned heads = 32;     // query heads per packed K slot (a shard packs its own)
};
struct SelectLaunch {
    const uint16_t* scores;
    int raw;           // normalise in the kernel
    int keys = 0;      // scores are order keys of normalised scores (from the scorer)
    const uint16_t* tie_raw = nullptr;  // keys mode: raw scores (tells +0 from -0 at a tie)
    int cover;         // prefetch-cover rules instead of select_gqa_scores
    uint32_t heads;
    unsigned long long stride, valid;
    float alpha, ratio;
    int fp32_counts;
    uint32_t* ids;
    unsigned long long kcap;
    uint32_t* counts;  // may be null (cover)
    hsb_selection* result;
    void* workspace;
    size_t workspace_bytes;
    unsigned long long cover_cap;  // cover: min(position, floor((position+1)*0.2f))
    int reset_result = 1;          // zero *result before the kernel
    int zero_is_error = 0;         // k == 0 -> HSB_E_ZERO_SELECTION (layer step)
    int reset_header = 1;          // zero the workspace header before the kernel
    const uint32_t* h0 = nullptr;  // the scorer's head-0 partials (ScoreExtras::h0)
    SelectEpilogue ga;             // run by the cluster kernel only
    int* ga_done = nullptr;        // out: 1 when the epilogue was launched
    // KV-head shard step: records from the exchange replace count + barrier.
    const uint32_t* ext = nullptr;      // [heads_total] count | non-finite << 31
    const uint32_t* ext_thr = nullptr;  // {threshold key, status}
    uint32_t head_base = 0, heads_total = 0;
    // Shard steps over a batch of sequences: scores / keys [batch][heads][stride]
    // (seq_scores = heads * stride), ids [batch][heads][kcap], counts
    // [batch][heads], result [batch], ext [batch][heads_total], ext_thr [batch][2],
    // and the epilogue's buffers per sequence.
    uint32_t batch = 1;
    unsigned long long seq_scores = 0;
    // The layer's select after a prepared history (cluster path, batch 1,
    // keys mode with h0): the scorer covered positions [0, valid - 1), and
    // the kernel scores the current position valid - 1 itself -- cur_q F16
    // [heads][128] against its key row cur_k (8 KV heads x 128, 16-byte
    // aligned) -- writing the raw scores to cur_raw[h * stride + valid - 1].
    const uint16_t* cur_q = nullptr;
    const uint16_t* cur_k = nullptr;
    uint16_t* cur_raw = nullptr;
    int cooperative = 1;  // launch attribute of the grid-barrier kernels
};
// Exchanges over peer memory (exchange.cu); arguments validated there.
// The scorer's threshold push (rank 0 of a peer group): the CTA that closes a
// sequence's last head-0 partial stores its threshold record into every
// rank's mailbox; the one that closes the batch's last sequence resets the
// counters and releases the threshold flag.
struct ThresholdPush {
    unsigned char* mb[HSB_MAX_PEERS] = {};
    int world = 0;  // 0: no push
    unsigned long long thr_off = 0, flag_off = 0;
    const unsigned long long* epoch = nullptr;  // rank 0's step counter
    unsigned int* cta_done = nullptr;           // CTAs finished, zero between steps
    float alpha = 0.0f;
};
bool threshold_push_params(const hsb_peer_group* g, float alpha, ThresholdPush* out);
size_t mailbox_bytes(size_t batch);
void mailbox_offsets(size_t batch, hsb_mailbox_layout* out);
cudaError_t launch_exchange_threshold(const uint32_t* h0, float alpha, const hsb_peer_group* g, cudaStream_t stream);
cudaError_t launch_exchange_count(const uint16_t* keys, size_t heads, size_t tokens, const hsb_peer_group* g,
                                  cudaStream_t stream);
cudaError_t launch_exchange_finish(const float* out, const hsb_selection* results, size_t heads,
                                   const hsb_peer_group* g, cudaStream_t stream);
cudaError_t launch_shard_threshold(const uint32_t* h0, size_t batch, float alpha, uint32_t* thr,
                                   cudaStream_t stream);
cudaError_t launch_shard_count(const uint16_t* keys, size_t heads, size_t tokens, size_t batch, const uint32_t* thr,
                               uint32_t* records, cudaStream_t stream);
bool select_cluster_available(size_t valid);
size_t select_workspace_bytes(size_t heads, size_t valid, size_t kcap);
size_t select_header_bytes();  // leading bytes of the workspace that start at zero
cudaError_t launch_select(const SelectLaunch& s, cudaStream_t stream);

// Stage 3
size_t union_workspace_bytes(size_t visible);
cudaError_t launch_union(const uint32_t* ids, size_t kstride, const uint32_t* sizes,
                         size_t sizes_stride, size_t visible, uint32_t* physical,
                         uint32_t* physical_count, hsb_device_status* status, void* workspace,
                         cudaStream_t stream);
size_t pack_workspace_bytes(uint64_t last_position);
cudaError_t launch_pack(const uint32_t* ids, size_t kstride, const uint32_t* sizes,
                        size_t sizes_stride, const uint64_t* positions, size_t npositions,
                        uint64_t last_position, const uint32_t* physical, size_t nphysical,
                        const uint8_t* payload, size_t count, uint16_t* k, uint16_t* v,
                        float* mask, hsb_device_status* status, void* workspace,
                        cudaStream_t stream);
// zero_padding 0: only each head's leading slots with a source are written
// (the map must put its sources first); the rest of the layout is untouched.
// live_k (device, with zero_padding 0): no head has a source at slot >= *live_k.
cudaError_t launch_gather_map(const uint16_t* prefetched, size_t prefetched_rows,
                              const uint16_t* misses, size_t miss_rows, const int32_t* map,
                              size_t count, uint16_t* k, uint16_t* v, hsb_device_status* status,
                              cudaStream_t stream, int zero_padding = 1, const uint32_t* live_k = nullptr);
cudaError_t launch_gather_cache(const uint32_t* ids, size_t kstride, const uint32_t* sizes,
                                size_t sizes_stride, const uint16_t* kcache,
                                const uint16_t* vcache, size_t stride_words, size_t visible,
                                size_t count, int zero_padding, uint16_t* k, uint16_t* v,
                                hsb_device_status* status, cudaStream_t stream);
cudaError_t launch_stage_rows(const uint8_t* rows, const uint32_t* physical,
                              const uint32_t* count, size_t max_rows, uint8_t* dst,
                              cudaStream_t stream);

// Stage 4
size_t attention_workspace_bytes(size_t count);
cudaError_t launch_attention_packed(const float* q, const uint16_t* k, const uint16_t* v,
                                    size_t count, const float* mask, size_t qpad,
                                    const uint32_t* sizes, size_t sizes_stride, float* out,
                                    void* workspace, cudaStream_t stream);
// The layer step's fused gather + attention (live slots only, sizes = *size
// for every head).  Workspace: [32] arrival counters (zero at launch: cleared
// here when reset_arrive, else by the caller) + [32][ceil(count/32)] partials.
size_t gather_attention_workspace_bytes(size_t count);
cudaError_t launch_gather_attention(const float* q, const uint32_t* ids, size_t kstride, const uint32_t* size,
                                    const uint16_t* kcache, const uint16_t* vcache, size_t stride_words,
                                    size_t visible, size_t count, uint16_t* kp, uint16_t* vp, float* out,
                                    void* workspace, int reset_arrive, hsb_device_status* status,
                                    cudaStream_t stream);
size_t attention_dense_workspace_bytes(size_t tokens);
cudaError_t launch_attention_dense(const float* q, const uint16_t* kcache, const uint16_t* vcache,
                                   size_t tokens, size_t stride_words, float* out,
                                   void* workspace, cudaStream_t stream);

// H2O residency statistics (runtime/gqa_h2o_stats.cu:41-57): out[kv][key]
// over valid keys x queries of F32 probabilities with byte strides nb0 (key),
// nb1 (query), nb2 (Q head); arguments already validated.
cudaError_t launch_h2o_group_sums(const void* probs, size_t keys, size_t queries, size_t nb0, size_t nb1,
                                  size_t nb2, float* out, hsb_device_status* status, cudaStream_t stream);

// Cold-tier KV records (storage/segmented_store.cpp): the file image of
// `count` records from payload rows, and the check + gather of records read
// back into a device window.  Arguments already validated.
cudaError_t launch_records_encode(const void* payload, size_t payload_stride, size_t count, size_t record_bytes,
                                  uint64_t request, uint32_t layer, uint64_t first, void* records,
                                  cudaStream_t stream);
cudaError_t launch_records_verify(const void* window, size_t window_bytes, const uint64_t* offsets,
                                  const uint64_t* positions, const uint32_t* groups, size_t count, uint64_t request,
                                  uint32_t layer, size_t record_bytes, void* out, size_t out_stride,
                                  const uint32_t* out_rows, size_t out_capacity, int host_window,
                                  hsb_device_status* status, cudaStream_t stream);

// Rehearsal query
cudaError_t launch_rehearsal(const uint16_t* x, const uint16_t* w, uint64_t position, float theta,
                             float* q32, uint16_t* q16, cudaStream_t stream);

// Synthetic inputs
cudaError_t launch_synth_normal(uint16_t* out, size_t count, uint64_t seed, float stddev,
                                int bf16, cudaStream_t stream);
cudaError_t launch_synth_keys(uint16_t* rows, size_t tokens, size_t stride_words, uint64_t seed,
                              float heavy_fraction, float heavy_scale, int rope, float theta,
                              cudaStream_t stream);

}  // namespace hsb
