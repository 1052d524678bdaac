/*
 * hsb.h -- C ABI of the B200-native selected-KV decode path.
 *
 * The path has four stages, each a hand-written sm_100a kernel:
 *   1. full-GQA key scoring under the HS_FULL_GQA_PIPELINE_F16_V3 contract
 *      (F16 Q[32,128] . K[N,8,128], query head h -> KV head h/4, channels
 *      0..127 accumulated in order in FP32 from +0, one RNE rounding to F16);
 *   2. the gqa_policy selector (head-0 maximum broadcast, alpha margin,
 *      inclusive count, F16 count/mean, ratio cap, ordered per-head top-k);
 *   3. the physical union and the packing / gather of selected K/V rows;
 *   4. flash-decode attention over the gathered K/V.
 *
 * Conventions
 *  - Every pointer named d_* is CUDA device memory (or host memory the GPU
 *    can address, where a function says so).  Arrays named h_* are host.
 *  - `stream` is a cudaStream_t passed as void*; NULL means the legacy
 *    default stream.  Every call only enqueues work on `stream` unless its
 *    comment says it synchronises.
 *  - Functions return an hsb_status.  A non-zero status leaves a message,
 *    worded like the reference exception it stands for, in a thread-local
 *    buffer read by hsb_last_error().  Errors that only the GPU can see
 *    (non-finite scores, duplicate IDs, ...) are written to a device status
 *    word that the caller reads after the stream completes (hsb_*_check()).
 *  - Workspaces are caller-allocated device memory sized by the matching
 *    *_workspace_bytes() query; the library allocates nothing per call.
 *  - Token IDs are uint32 (the reference uses uint64; every ID it admits is
 *    below 2^32).
 *
 * Reference citations are paths inside the HillServe project.
 */
#ifndef HSB_H
#define HSB_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define HSB_ABI_VERSION 1
#define HSB_QUERY_HEADS 32
#define HSB_KV_HEADS 8
#define HSB_DIM 128
#define HSB_ROW_WORDS 2048 /* one interleaved KV row: K[8,128] then V[8,128] */
#define HSB_MAX_VIEWS 8    /* key views per scoring launch (more are split) */
#define HSB_MAX_PEERS 8    /* GPUs of one KV-head-sharded group */
#define HSB_IPC_HANDLE_BYTES 64

typedef enum hsb_status {
    HSB_OK = 0,
    HSB_E_INVALID = 1,   /* null pointer / bad enum / misaligned argument */
    HSB_E_CUDA = 2,      /* a CUDA runtime call failed */
    HSB_E_WORKSPACE = 3, /* workspace missing or smaller than required */
    HSB_E_TIMEOUT = 4,   /* a bounded device wait gave up */
    HSB_E_NO_DEVICE = 5, /* no sm_100 device / kernel image */
    /* stage 1 -- policy/full_gqa_cpu.cpp:210-227, smartssd/adapter.hpp:97-104 */
    HSB_E_SCORE_SHAPE = 10,
    HSB_E_SCORE_ALIAS = 11,
    HSB_E_SCORE_V3_TOKENS = 12,
    /* stage 2 -- policy/gqa_policy.cpp:48-61 (same order of checks) */
    HSB_E_SEL_SHAPE = 20,
    HSB_E_SEL_PARAMS = 21,
    HSB_E_SEL_NONFINITE_HEAD0 = 22,
    HSB_E_SEL_THRESHOLD = 23,
    HSB_E_SEL_NONFINITE = 24,
    HSB_E_SEL_U32 = 25,
    HSB_E_SEL_COUNT_F16 = 26,
    HSB_E_SEL_MEAN_F16 = 27,
    HSB_E_SEL_CAPACITY = 28,
    /* stage 3 -- runtime/gqa_pack.hpp:14-44, runtime/gqa_prefetch_cuda.cu:217-218 */
    HSB_E_UNION_BOUNDS = 30,
    HSB_E_UNION_DUPLICATE = 31,
    HSB_E_PACK_SHAPE = 40,
    HSB_E_PACK_PHYSICAL = 41,
    HSB_E_PACK_SLOTS = 42,
    HSB_E_PACK_MISSING = 43,
    HSB_E_MAP_GEOMETRY = 50,
    HSB_E_MAP_ROW = 51,
    HSB_E_MAP_MISS = 52,
    /* prefetch cover -- policy/full_gqa_runtime.cpp:316-333 */
    HSB_E_COVER_RANGE = 60,
    HSB_E_COVER_THRESHOLD = 61,
    HSB_E_COVER_COUNT = 62,
    HSB_E_COVER_MEAN = 63,
    /* layer step -- policy/full_gqa_runtime.cpp:573 */
    HSB_E_ZERO_SELECTION = 70,
    /* H2O statistics -- runtime/gqa_h2o_stats.cu:110-133 */
    HSB_E_H2O_ARGS = 80,
    HSB_E_H2O_SHAPE = 81,
    HSB_E_H2O_STRIDE = 82,
    HSB_E_H2O_OVERFLOW = 83,
    HSB_E_H2O_ALIGN = 84,
    HSB_E_H2O_GRID = 85,
    HSB_E_H2O_DEVICE = 86,
    /* cold-tier KV records -- policy/full_gqa_runtime.cpp:395-409,
     * storage/segmented_store.cpp:24-26,98,116-119, storage/kv_read_plan.hpp:22-59 */
    HSB_E_RECORD_IDENTITY = 90,
    HSB_E_RECORD_CHECKSUM = 91,
    HSB_E_RECORD_BOUNDS = 92,
    HSB_E_SEGMENT_GEOMETRY = 93,
    HSB_E_READ_PLAN = 94,
    /* decode history -- policy/full_gqa_runtime.cpp:236,472-483,550-560,
     * runtime/full_gqa_contract.hpp:116-122 */
    HSB_E_HISTORY_RESIDENCY = 100,
    HSB_E_HISTORY_GEOMETRY = 101,
    HSB_E_HISTORY_PROTOCOL = 102,
    HSB_E_HISTORY_QUERY = 103,
    /* layer executor -- runtime/gqa_executor.cpp:151-153,
     * policy/full_gqa_runtime.cpp:61-64 */
    HSB_E_EXECUTOR_SHAPE = 110,
    HSB_E_EXECUTOR_NONFINITE_KV = 111,
    HSB_E_EXECUTOR_REHEARSAL = 112,
    HSB_E_EXECUTOR_REHEARSAL_F16 = 113
} hsb_status;

int hsb_abi_version(void);
/* Message of the last failing call made by this thread ("" if none). */
const char* hsb_last_error(void);
/* Reference-worded message for a status code. */
const char* hsb_status_message(int status);

/* Device status word written by kernels: 0 = ok, else an hsb_status in the
 * low 8 bits and the (query head or row) index that raised it above them. */
typedef struct hsb_device_status {
    int32_t code;
    int32_t index;
} hsb_device_status;
/* Synchronises `stream`, reads *d_status, sets the last-error message and
 * returns the status it holds.  Does not clear it. */
int hsb_status_check(const hsb_device_status* d_status, void* stream);

/* ------------------------------------------------------------------ stage 1
 * Replaces FullGqaCpuScorer::score (policy/full_gqa_cpu.hpp:43-45,
 * .cpp:206-250) and score_full_gqa_legacy_cpu (.cpp:109-138): identical bits.
 * d_q: F16 [32][128]; keys of token t start at view.data + t*stride_words
 * (stride 1024 = token-major K, 2048 = interleaved K|V rows); tokens of the
 * views are concatenated in order; d_scores: F16 [32][sum tokens]. */
typedef struct hsb_key_view {
    const uint16_t* data;
    size_t tokens;
    size_t stride_words;
} hsb_key_view;

int hsb_score_v3(const uint16_t* d_q, const uint16_t* d_keys, size_t tokens,
                 size_t stride_words, uint16_t* d_scores, void* stream);
int hsb_score_views(const uint16_t* d_q, const hsb_key_view* h_views, size_t nviews,
                    uint16_t* d_scores, void* stream);
/* The V3 pipeline contract (kernels/full_gqa_pipeline/ABI.json:20-30,
 * kernel.cpp:237-253): token-major K, 64 <= tokens <= 32768, tokens % 64 == 0;
 * any other count is rejected before touching memory. */
int hsb_score_pipeline_v3(const uint16_t* d_q, const uint16_t* d_keys, uint32_t tokens,
                          uint16_t* d_scores, void* stream);
/* hsb_score_v3 that also writes, per score, the 16-bit order key
 * (policy/half_order.hpp:7-10) of its normalised value F16(raw / sqrtf(128))
 * to d_order_keys [32][tokens] -- the input of hsb_select_keys. */
int hsb_score_with_keys(const uint16_t* d_q, const uint16_t* d_keys, size_t tokens, size_t stride_words,
                        uint16_t* d_scores, uint16_t* d_order_keys, void* stream);
/* The runtime's normalisation (policy/full_gqa_runtime.cpp:571):
 * d_out[i] = F16(F32(d_raw[i]) / sqrtf(128)).  d_out may equal d_raw. */
int hsb_scale_scores(const uint16_t* d_raw, size_t count, uint16_t* d_out, void* stream);

/* ------------------------------------------------------------------ stage 2
 * Replaces select_gqa_scores (policy/gqa_policy.hpp:19-21, .cpp:47-70).
 * d_scores: F16 [heads][stride], tokens [0,valid) are candidates.  With
 * input_is_raw != 0 the scores are raw dot products and are normalised in the
 * kernel exactly as hsb_scale_scores does (the runtime's select path,
 * full_gqa_runtime.cpp:571-572); otherwise they are already normalised.
 * Outputs: d_ids [heads][kcap] (top-k per head, order key descending then ID
 * ascending), d_counts [heads] (inclusive threshold counts), *d_result.
 * kcap must be >= min(floor(valid*ratio), valid). */
typedef struct hsb_selection {
    uint32_t k;
    uint32_t boundary_tied_heads;
    hsb_device_status status;
} hsb_selection;

size_t hsb_select_workspace_bytes(size_t heads, size_t stride, size_t valid, size_t kcap);
int hsb_select(const uint16_t* d_scores, int input_is_raw, size_t heads, size_t stride,
               size_t valid, float alpha, float ratio, int fp32_counts, uint32_t* d_ids,
               size_t kcap, uint32_t* d_counts, hsb_selection* d_result, void* d_workspace,
               size_t workspace_bytes, void* stream);
/* hsb_select on order keys of normalised scores (hsb_score_with_keys); the
 * raw scores d_raw [heads][stride] are read only to tell +0 from -0 when the
 * boundary-tie rule compares F16 bits.  Same outputs, checks and errors. */
int hsb_select_keys(const uint16_t* d_order_keys, const uint16_t* d_raw, size_t heads, size_t stride,
                    size_t valid, float alpha, float ratio, int fp32_counts, uint32_t* d_ids, size_t kcap,
                    uint32_t* d_counts, hsb_selection* d_result, void* d_workspace,
                    size_t workspace_bytes, void* stream);
/* Synchronises, copies *d_result to *h_result and returns its status. */
int hsb_selection_read(const hsb_selection* d_result, hsb_selection* h_result, void* stream);

/* History-only prefetch cover (policy/full_gqa_runtime.cpp:299-344): from raw
 * scores [32][capacity] of tokens [0,position), the per-head top-`bound`
 * lists that cover every final selection once the current token is added.
 * d_per_head is [32][cap], cap = min(position, floor((position+1)*0.2f));
 * d_result->k receives `bound`. */
int hsb_prefetch_cover(const uint16_t* d_raw, size_t capacity, size_t position, float alpha,
                       int fp32_counts, uint32_t* d_per_head, size_t cap,
                       hsb_selection* d_result, void* d_workspace, size_t workspace_bytes,
                       void* stream);

/* ------------------------------------------------------------------ stage 3
 * Per-head list sizes are read from d_sizes[h * sizes_stride]; pass
 * sizes_stride = 0 to give every head d_sizes[0] (e.g. &selection->k). */

/* gqa_physical_union (runtime/gqa_pack.hpp:12-22): sorted unique IDs of the
 * 32 per-head lists; duplicates within a head or IDs >= visible are errors. */
size_t hsb_union_workspace_bytes(size_t visible);
int hsb_union(const uint32_t* d_ids, size_t kstride, const uint32_t* d_sizes,
              size_t sizes_stride, size_t visible, uint32_t* d_physical,
              uint32_t* d_physical_count, hsb_device_status* d_status, void* d_workspace,
              size_t workspace_bytes, void* stream);

/* pack_gqa_workspace (runtime/gqa_pack.hpp:26-58), bit-exact:
 * K [count][32][128], V [32][128][count] and mask F32 [32][qpad][count]
 * (qpad = roundup(npositions, 64)) from payload rows (4096 B each, F16 K[8][128]
 * then V[8][128]) listed in d_physical order.  d_mask may be NULL. */
size_t hsb_pack_workspace_bytes(uint64_t last_position);
int hsb_pack(const uint32_t* d_ids, size_t kstride, const uint32_t* d_sizes,
             size_t sizes_stride, const uint64_t* d_positions, size_t npositions,
             uint64_t last_position, const uint32_t* d_physical, size_t nphysical,
             const uint8_t* d_payload, size_t payload_bytes, size_t count, uint16_t* d_k,
             uint16_t* d_v, float* d_mask, hsb_device_status* d_status, void* d_workspace,
             size_t workspace_bytes, void* stream);

/* gather_gqa (runtime/gqa_prefetch_cuda.cu:12-22) with deliver's row checks
 * (:217-218): d_map[h*count+s] >= 0 selects prefetched row, <= -2 miss row
 * (-2-index), -1 padding (zeros). */
int hsb_gather_map(const uint16_t* d_prefetched, size_t prefetched_rows,
                   const uint16_t* d_misses, size_t miss_rows, const int32_t* d_map,
                   size_t count, uint16_t* d_k, uint16_t* d_v, hsb_device_status* d_status,
                   void* stream);

/* The device-resident gather: selected rows read straight from an HBM KV
 * cache (K at d_kcache + id*stride_words, V at d_vcache + id*stride_words)
 * into the packed layout of hsb_pack.  zero_padding != 0 zero-fills slots
 * [size_h, count) as the reference does; 0 writes live slots only. */
int hsb_gather_cache(const uint32_t* d_ids, size_t kstride, const uint32_t* d_sizes,
                     size_t sizes_stride, const uint16_t* d_kcache, const uint16_t* d_vcache,
                     size_t stride_words, size_t visible, size_t count, int zero_padding,
                     uint16_t* d_k, uint16_t* d_v, hsb_device_status* d_status, void* stream);

/* Copies union rows (4096 B each) from a row store the GPU can address --
 * HBM or mapped pinned host memory (the cold tier) -- into HBM:
 * d_dst[i] = d_rows[d_physical[i]] for i < *d_count (at most max_rows). */
int hsb_stage_rows(const uint8_t* d_rows, const uint32_t* d_physical,
                   const uint32_t* d_count, size_t max_rows, uint8_t* d_dst, void* stream);

/* ------------------------------------------------------------------ stage 4
 * Attention over the packed workspace (the ggml graph of
 * runtime/gqa_delivery.cpp:19-20): per query head,
 * softmax(K.q / sqrt(128) + mask) . V with q F32 [32][128], out F32 [32][128].
 * Slot validity comes from d_mask (query row 0 of [32][qpad][count]) when it
 * is non-NULL, else from the per-head sizes. */
size_t hsb_attention_workspace_bytes(size_t count);
int hsb_attention_packed(const float* d_q, const uint16_t* d_k, const uint16_t* d_v,
                         size_t count, const float* d_mask, size_t qpad,
                         const uint32_t* d_sizes, size_t sizes_stride, float* d_out,
                         void* d_workspace, size_t workspace_bytes, void* stream);
/* hsb_attention_packed without a workspace argument; it has no counterpart in
 * the reference.  It is meant for callers that cannot provide or allocate any
 * device memory beyond their inputs and outputs, such as an operator run
 * inside a host framework's compute graph, whose tensors are handed to it and
 * whose allocator owns the device memory.  The scratch is a static device
 * array of 448 KiB that every GPU loading this library holds until exit;
 * count must be <= HSB_NOALLOC_MAX_SLOTS (the reference delivery workspace's
 * slot limit), else HSB_E_WORKSPACE.  The call allocates nothing.  The first
 * call in each CUDA context (normally once per device) resolves the array's
 * address (cudaGetSymbolAddress) and should come before any stream capture;
 * a new context on the device (after cudaDeviceReset, or another context
 * made current) resolves it again on its first call.  All calls on a device
 * share the array and its last contents: calls that overlap on the GPU race,
 * so order them on one stream. */
#define HSB_NOALLOC_MAX_SLOTS 6592
int hsb_attention_packed_noalloc(const float* d_q, const uint16_t* d_k, const uint16_t* d_v,
                                 size_t count, const float* d_mask, size_t qpad,
                                 const uint32_t* d_sizes, size_t sizes_stride, float* d_out,
                                 void* stream);
/* Dense decode attention over a token-major cache (dense layers,
 * runtime/gqa_executor.cpp:174-176). */
size_t hsb_attention_dense_workspace_bytes(size_t tokens);
int hsb_attention_dense(const float* d_q, const uint16_t* d_kcache, const uint16_t* d_vcache,
                        size_t tokens, size_t stride_words, float* d_out, void* d_workspace,
                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------- rehearsal query
 * The rehearsal query producer (patches/llama-b6000-round2.patch:303-317 and
 * the F16 cast of policy/full_gqa_runtime.cpp:61-64): q = RoPE_position(W x),
 * x bf16 [4096], W bf16 [4096 out][4096 in] (both 16-byte aligned), NORM-mode
 * RoPE with base theta.
 * Writes d_q_f32 [32][128] and/or d_q_f16 (either may be NULL). */
int hsb_rehearsal_query(const uint16_t* d_x, const uint16_t* d_w, uint64_t position,
                        float theta, float* d_q_f32, uint16_t* d_q_f16, void* stream);

/* ------------------------------------------------------------- layer step
 * One selected-KV decode layer, all on `stream` with no host round trip:
 * score (raw, plus order keys) -> select -> gather from the HBM cache into
 * the packed live-slot layout fused with the attention over those rows:
 * three kernels and no memset or host round trip (capturable in a CUDA
 * graph).  count (slot capacity per head) must be >= min(floor(valid*ratio),
 * valid).  The V cache, d_q32 and the packed buffers must be 16-byte
 * aligned.  d_out receives F32 [32][128]; d_ids/d_counts/d_result as
 * hsb_select.  k == 0 leaves d_out zero and sets d_result->status to
 * HSB_E_ZERO_SELECTION (the reference throws there).  Calls sharing one
 * workspace must be ordered on one stream. */
typedef struct hsb_layer_buffers {
    uint16_t* scores;  /* F16 [32][valid] */
    uint32_t* ids;     /* [32][count] */
    uint32_t* counts;  /* [32] */
    hsb_selection* result;
    uint16_t* k_packed; /* [count][32][128] */
    uint16_t* v_packed; /* [32][128][count] */
    void* workspace;
    size_t workspace_bytes;
} hsb_layer_buffers;
size_t hsb_layer_workspace_bytes(size_t valid, size_t count);
int hsb_layer_step(const uint16_t* d_q16, const float* d_q32, const uint16_t* d_kcache,
                   const uint16_t* d_vcache, size_t stride_words, size_t valid, float alpha,
                   float ratio, size_t count, const hsb_layer_buffers* buffers, float* d_out,
                   void* stream);
/* The layer step split where the reference splits it
 * (FullGqaRuntimePolicy::prepare_history, policy/full_gqa_runtime.cpp:493-516,
 * scores the history ahead of the layer; select, :549-585, adds the current
 * token's scores, :531-548, and selects).  hsb_layer_prepare scores positions
 * [0, valid - 1) with the selection query (the early rehearsal,
 * patches/llama-b6000-early-rehearsal.patch:46-52) and needs only the history
 * rows; hsb_layer_select scores the current position valid - 1 -- whose K row
 * must be in the cache by then -- normalises, selects, gathers and attends.
 * Together they give hsb_layer_step's results bit for bit.  valid >= 2; the
 * select needs the cluster selector (valid <= 65536) and 16-byte aligned
 * d_q16 / key rows.  Order: select after its prepare (same buffers), and the
 * next prepare on those buffers after that select; a decode step runs
 * layer l + 1's prepare beside layer l's select on two buffer sets. */
int hsb_layer_prepare(const uint16_t* d_q16, const uint16_t* d_kcache, size_t stride_words, size_t valid,
                      float alpha, float ratio, size_t count, const hsb_layer_buffers* buffers, void* stream);
int hsb_layer_select(const uint16_t* d_q16, const float* d_q32, const uint16_t* d_kcache,
                     const uint16_t* d_vcache, size_t stride_words, size_t valid, float alpha,
                     float ratio, size_t count, const hsb_layer_buffers* buffers, float* d_out,
                     void* stream);

/* ------------------------------------------------------- KV-head shards
 * One selected-KV layer split across GPUs by KV head (each GPU holds
 * kv_heads of the 8 KV heads, i.e. query heads [head_base, head_base +
 * 4*kv_heads), of every sequence).  The reference couples heads through the
 * head-0 threshold and the mean of all heads' counts (policy/gqa_policy.cpp:
 * 49-63); a shard step reproduces that exactly with two tiny exchanges:
 *   1. every shard: hsb_shard_score (the shard holding query head 0 also
 *      writes head-0 partials);
 *   2. that shard: hsb_shard_threshold -> {threshold key, status}, broadcast;
 *   3. every shard: hsb_shard_count -> one record per local head
 *      (count | non-finite << 31), all-gathered in head order;
 *   4. every shard: hsb_shard_select -> the same k as the unsharded
 *      selector, its heads' ordered IDs, packed K/V and attention output.
 * Shard caches are token-major [tokens][kv_heads][128] F16. */
size_t hsb_shard_head0_words(void);  /* head-0 partial words per sequence */
/* A batch of `batch` sequences back to back: d_q [batch][4 kv_heads][128],
 * d_kshard [batch][tokens][kv_heads][128], d_scores / d_order_keys
 * [batch][4 kv_heads][tokens], d_head0 [batch][hsb_shard_head0_words()]
 * (only on the shard holding query head 0, else NULL). */
int hsb_shard_score(const uint16_t* d_q, int kv_heads, const uint16_t* d_kshard, size_t tokens,
                    size_t batch, uint16_t* d_scores, uint16_t* d_order_keys, uint32_t* d_head0,
                    void* stream);
/* d_thr [batch][2]: {threshold order key, status}. */
int hsb_shard_threshold(const uint32_t* d_head0, size_t batch, float alpha, uint32_t* d_thr,
                        void* stream);
/* d_records [batch][heads]: count | non-finite << 31 per local head. */
int hsb_shard_count(const uint16_t* d_order_keys, size_t heads, size_t tokens, size_t batch,
                    const uint32_t* d_thr, uint32_t* d_records, void* stream);
size_t hsb_shard_select_workspace_bytes(int kv_heads, size_t tokens, size_t kcap, size_t batch);
/* d_records: [batch][heads_total] from every shard, in head order.  Outputs
 * per sequence: d_ids [4 kv_heads][kcap], d_counts [4 kv_heads], d_result,
 * d_k_packed [kcap][4 kv_heads][128], d_v_packed [4 kv_heads][128][kcap],
 * d_out [4 kv_heads][128]; d_q32 [batch][4 kv_heads][128], V as K. */
int hsb_shard_select(const uint16_t* d_order_keys, const uint16_t* d_raw, int kv_heads, size_t tokens,
                     size_t batch, const uint32_t* d_thr, const uint32_t* d_records,
                     size_t heads_total, size_t head_base, float alpha, float ratio, uint32_t* d_ids,
                     size_t kcap, uint32_t* d_counts, hsb_selection* d_result, const float* d_q32,
                     const uint16_t* d_kshard, const uint16_t* d_vshard, uint16_t* d_k_packed,
                     uint16_t* d_v_packed, float* d_out, void* d_workspace, size_t workspace_bytes,
                     void* stream);

/* ------------------------------------- KV-head shards over peer memory
 * The same step with the exchanges done by this library's kernels over
 * NVLink peer memory instead of NCCL collectives (the reference has no
 * multi-GPU code; the coupling reproduced is that of policy/gqa_policy.cpp:
 * 49-63).  Every rank owns a mailbox -- device memory exported by CUDA IPC
 * and opened by every other rank of the node -- and one step is, on every
 * rank, in stream order:
 *   hsb_shard_score (head-0 partials on rank 0)
 *   -> rank 0: hsb_exchange_threshold   (stores the thresholds into every
 *      mailbox, releases a flag)
 *   -> hsb_exchange_count               (waits for the thresholds, stores
 *      its heads' count records into every mailbox, waits for every rank's)
 *   -> hsb_shard_select with d_thr / d_records in this rank's mailbox
 *   -> hsb_exchange_finish              (stores its outputs and selection
 *      results into every mailbox, waits for every rank's).
 * Afterwards this rank's mailbox holds all 32 heads' outputs [batch][32][128]
 * F32 and every rank's results [world][batch].  Flags carry a step epoch
 * kept in the mailbox, so no reset is needed between steps (CUDA graphs
 * replay the step as is).  Every wait is bounded by wait_limit_ns (0: 2 s);
 * one that gives up writes HSB_E_TIMEOUT (index = the rank waited for) to the
 * mailbox's status word and the kernel returns -- the mailboxes must then be
 * recreated.  Plain peer stores by threads only. */
typedef struct hsb_mailbox_layout {
    size_t thr;      /* uint32 [batch][2]: threshold order key, status */
    size_t records;  /* uint32 [batch][32]: count | non-finite << 31 */
    size_t outputs;  /* float [batch][32][128] */
    size_t results;  /* hsb_selection [world][batch] */
    size_t status;   /* hsb_device_status of the exchange */
    size_t bytes;
} hsb_mailbox_layout;
typedef struct hsb_peer_group {
    int world;                        /* 1, 2, 4 or 8 */
    int rank;
    void* mailbox[HSB_MAX_PEERS];     /* every rank's mailbox as mapped in this process (own: local) */
    size_t batch;                     /* sequences per step */
    uint64_t wait_limit_ns;           /* bound of every cross-GPU wait; 0 = 2 s */
} hsb_peer_group;
size_t hsb_mailbox_bytes(size_t batch);
void hsb_mailbox_layout_of(size_t batch, hsb_mailbox_layout* out);
/* Set-up (allocates): a zeroed mailbox for `batch` sequences on the current
 * device and, when ipc_handle != NULL, its HSB_IPC_HANDLE_BYTES CUDA IPC
 * handle for the other ranks. */
int hsb_mailbox_create(size_t batch, void** d_mailbox, void* ipc_handle);
int hsb_mailbox_destroy(void* d_mailbox);
/* Maps another process's mailbox (cudaIpcOpenMemHandle, peer access enabled
 * on demand) / unmaps it. */
int hsb_mailbox_open(const void* ipc_handle, void** d_peer);
int hsb_mailbox_close(void* d_peer);
int hsb_exchange_threshold(const uint32_t* d_head0, float alpha, const hsb_peer_group* group, void* stream);
/* hsb_shard_score and hsb_exchange_threshold in one launch, on rank 0: the
 * scorer CTA that finishes last folds every sequence's head-0 partials into
 * its threshold record, stores the records into every mailbox and releases
 * the threshold flag. */
int hsb_shard_score_push(const uint16_t* d_q, int kv_heads, const uint16_t* d_kshard, size_t tokens, size_t batch,
                         uint16_t* d_scores, uint16_t* d_order_keys, uint32_t* d_head0, float alpha,
                         const hsb_peer_group* group, void* stream);
int hsb_exchange_count(const uint16_t* d_order_keys, size_t heads, size_t tokens, const hsb_peer_group* group,
                       void* stream);
int hsb_exchange_finish(const float* d_out, const hsb_selection* d_results, size_t heads,
                        const hsb_peer_group* group, void* stream);

/* ---------------------------------------------- H2O residency statistics
 * The device work of GQAH2OStatsCuda::reduce (runtime/gqa_h2o_stats.cu:
 * 106-173; kernel sum_actual_attention :41-57).  d_probabilities is the
 * actual F32 softmax tensor, ne = {keys, queries, Q heads, streams} with
 * ggml byte strides nb[] (nb[3] unused); only ne[2] == 32, ne[3] == 1.
 * Writes d_sums[kv * valid_keys + key] for the 8 KV heads: the F32 sum over
 * Q heads 4kv..4kv+3 (outer) and queries 0..valid_queries-1 (inner), from
 * +0, each addition rounded -- the reference's order, bit for bit.  Padding
 * keys and queries are never read.  Validation and messages follow reduce()
 * (:110-133); capacity_keys is the d_sums capacity per KV head (the
 * reducer's constructor argument); as there, the probabilities must be
 * device memory of the current device.  A null stream is the default stream.
 * Enqueues on `stream` and never synchronises; d_status (nullable) receives
 * HSB_E_TIMEOUT if a bounded device wait gave up. */
int hsb_h2o_group_sums(const void* d_probabilities, const int64_t ne[4], const size_t nb[4],
                       size_t valid_keys, size_t valid_queries, float* d_sums, size_t capacity_keys,
                       hsb_device_status* d_status, void* stream);

/* ------------------------------------------------- cold-tier KV records
 * SegmentedKVStore v1 (storage/segmented_store.{hpp,cpp}): a 4096-byte file
 * header, then the record of (layer, position) at byte
 *     4096 + (layer * positions + position) * (record_bytes + 32):
 * a 32-byte header {u64 digest, u64 position, u64 request, u32 layer,
 * u32 version = 1} and the payload (for this model one K||V row, 4096
 * bytes).  digest = FNV-1a 64 of the payload (storage/file_store.cpp:12-16).
 * Geometry bounds as the store's constructor: layers 1..128, positions
 * 1..66048, record_bytes 1..65536 (segmented_store.cpp:24-26). */
#define HSB_SEGMENT_HEADER_BYTES 4096
#define HSB_RECORD_HEADER_BYTES 32
/* Page-rounded file extent (segmented_store.cpp:26); 0 for invalid geometry. */
uint64_t hsb_segment_extent_bytes(size_t layers, uint64_t positions, size_t record_bytes);
/* The 4096-byte file header (segmented_store.cpp:30) into host memory. */
int hsb_segment_header(void* header, uint64_t request, size_t layers, uint64_t positions, size_t record_bytes);
/* FNV-1a 64 of n host bytes (storage/file_store.cpp:12-16). */
uint64_t hsb_fnv1a64(const void* data, size_t n);
/* Device: the file image of records (layer, first .. first+count-1), i.e.
 * the bytes SegmentedKVStore::append writes (segmented_store.cpp:95-104),
 * contiguous at d_records (count * (record_bytes + 32) bytes), from payload
 * rows d_payload + i * payload_stride. */
int hsb_kv_records_encode(const void* d_payload, size_t payload_stride, size_t count, size_t record_bytes,
                          uint64_t request, uint32_t layer, uint64_t first, void* d_records, void* stream);
/* Device: checks records read back from the file into d_window (window_bytes
 * of raw file bytes) and copies their payloads to device rows.  Record i
 * starts at d_window + d_offsets[i]; it must carry position d_positions[i],
 * `request`, `layer` and version 1 (else HSB_E_RECORD_IDENTITY) and a digest
 * equal to the FNV-1a of its payload (else HSB_E_RECORD_CHECKSUM), checked
 * in that order as policy/full_gqa_runtime.cpp:395-409 does.  The payload
 * goes to d_out + row * out_stride, row = d_out_rows ? d_out_rows[i] : i
 * (< out_rows_capacity, else HSB_E_RECORD_BOUNDS, as for a record outside
 * the window).  The first failure in the reference's order is written to
 * *d_status: by validation group (d_groups[i], the reference's batches of
 * four per read window -- hsb_kv_read_groups; NULL: one group per record,
 * SegmentedKVStore::fetch's order), identity before checksum, then index.
 * d_window may also be pinned host memory (the read buffers themselves,
 * mapped at the same address): the kernel then reads only the records'
 * bytes across the bus, with no staging copy.  Pageable memory is rejected
 * (HSB_E_INVALID). */
int hsb_kv_records_verify(const void* d_window, size_t window_bytes, const uint64_t* d_offsets,
                          const uint64_t* d_positions, const uint32_t* d_groups, size_t count, uint64_t request,
                          uint32_t layer, size_t record_bytes, void* d_out, size_t out_stride,
                          const uint32_t* d_out_rows, size_t out_rows_capacity, hsb_device_status* d_status,
                          void* stream);
/* Host: the bounded read plan of storage/kv_read_plan.hpp:34-59 over
 * records at ascending file offsets (record_bytes here includes the 32-byte
 * header, as the reference passes it).  Limits as KVReadLimits (defaults
 * 1 MiB window, 16 KiB gap, 1500 permille). */
typedef struct hsb_kv_read_window {
    uint64_t begin, end, required_page_bytes;
    uint64_t first_record, end_record;
} hsb_kv_read_window;
int hsb_kv_read_plan(const uint64_t* offsets, size_t count, uint64_t record_bytes, uint64_t extent,
                     size_t window_bytes, size_t gap_bytes, unsigned max_amplification_permille,
                     hsb_kv_read_window* windows, size_t windows_capacity, size_t* nwindows);
/* Host: the reference's validation groups for hsb_kv_records_verify: records
 * of each window in batches of four from the window's first record
 * (policy/full_gqa_runtime.cpp:394-395); groups[i] for i < count. */
int hsb_kv_read_groups(const hsb_kv_read_window* windows, size_t nwindows, uint32_t* groups, size_t count);

/* ---------------------------------------------------- decode history
 * One request's decode history on the GPU: FullGqaRuntimePolicy's hot/cold
 * history scoring and its prepare -> select -> fetch protocol
 * (policy/full_gqa_runtime.cpp:418-471, 477-499, 549-585, 586-690) with the
 * hot KV rows in HBM.
 *
 * hsb_score_history: raw V3 scores of positions [0, valid) into
 * d_scores[h * out_stride + t] (order keys too when d_order_keys != NULL),
 * each position's K row found through row_of_position (HOST array): >= 0 a
 * row of the hot pool (rows of pool_stride_words, K first), <= -2 the row
 * -2-r of the cold K store (cold_stride_words), -1 not resident (rejected,
 * HSB_E_HISTORY_RESIDENCY).  Runs of positions whose rows are consecutive
 * become key views of the TMA scorer; the scores are those of the
 * reference's hot + cold merge, bit for bit. */
int hsb_score_history(const uint16_t* d_q, const uint16_t* d_hot_pool, size_t pool_stride_words,
                      const uint16_t* d_cold_k, size_t cold_stride_words, const int64_t* row_of_position,
                      size_t valid, uint16_t* d_scores, size_t out_stride, uint16_t* d_order_keys,
                      void* stream);

/* The hot placement of plan_full_gqa_runtime (runtime/full_gqa_contract.hpp:
 * 42-56, 128-134, 168-184): beta's hot 64-token blocks (the earliest ones
 * plus a recent window of up to 16 blocks and the partial tail), generated
 * positions after them; cold prompt positions -1.  Writes [capacity]. */
int hsb_history_plan_slots(size_t prompt_tokens, size_t generated_capacity, size_t capacity, double beta,
                           int allow_partial_prompt, int64_t* hot_slot_by_position, size_t* hot_prompt_tokens);

/* A history is one request's state: drive it from one host thread at a time
 * (its calls check and update host-side protocol state). */
typedef struct hsb_history hsb_history;
typedef struct hsb_history_config {
    size_t layers;              /* <= 32 */
    size_t capacity;            /* positions per layer, multiple of 64 */
    size_t prompt_tokens;
    size_t generated_capacity;  /* 1 .. 512 */
    float alpha;                /* selector alpha, shared by the cover and the final selection */
    int fp32_counts;
} hsb_history_config;
/* hot_slot_by_position (HOST, [capacity]): the placement of
 * runtime/full_gqa_contract.hpp:168-184 (hot pool slot, -1 cold).  Cold
 * prompt positions keep their K rows in an HBM cold K store; their V stays in
 * the caller's cold tier (records).  Every generated position must be hot. */
int hsb_history_create(const hsb_history_config* cfg, const int64_t* hot_slot_by_position, hsb_history** out);
void hsb_history_destroy(hsb_history* h);
size_t hsb_history_hot_slots(const hsb_history* h);
size_t hsb_history_cold_rows(const hsb_history* h);
size_t hsb_history_select_capacity(const hsb_history* h); /* ids per head kcap that always suffices */
/* append (:472-492): `count` token-major K||V rows (2048 words each, device,
 * 16-byte aligned) for positions first .. first+count-1 = the next ones. */
int hsb_history_append(hsb_history* h, size_t layer, uint64_t first, size_t count, const uint16_t* d_rows,
                       void* stream);
/* prepare_history (:493-516): scores the history [0, position) and its
 * payload cover on the history's own stream, once `stream` has the query;
 * at most two prepared histories, none twice for a layer. */
int hsb_history_prepare(hsb_history* h, size_t layer, uint64_t position, const uint16_t* d_q16, void* stream);
/* The cover of a prepared history, ordered on `stream`: its cold positions
 * (ascending: the records to read) and its per-head bound (d_cover_result->k). */
int hsb_history_cover(hsb_history* h, size_t layer, uint32_t* d_cold_ids, uint32_t* d_cold_count,
                      hsb_selection* d_cover_result, void* stream);
/* select (:549-585): joins the prepared history (or scores it now), adds the
 * current token's score, normalises and selects: d_ids [32][kcap], d_counts
 * [32], *d_result (HSB_E_HISTORY_QUERY when the query differs from prepare's). */
int hsb_history_select(hsb_history* h, size_t layer, uint64_t position, const uint16_t* d_q16, uint32_t* d_ids,
                       size_t kcap, uint32_t* d_counts, hsb_selection* d_result, void* stream);
/* fetch (:586-690) into the packed layout: K [count][32][128], V
 * [32][128][count]; hot rows from the pool, cold rows from d_staged_rows
 * (4096-byte K||V rows of the ascending d_staged_ids, e.g. the cover's cold
 * positions read with hsb_kv_records_verify).  A selected cold ID that was not
 * staged sets HSB_E_MAP_MISS.  zero_padding != 0 zeroes slots k..count-1
 * (the reference's packed layout); 0 writes the live slots only, for
 * attention over sizes = k.  Consumes the layer's prepared history. */
int hsb_history_fetch(hsb_history* h, size_t layer, const uint32_t* d_ids, size_t kcap,
                      const hsb_selection* d_result, const uint32_t* d_staged_ids, size_t nstaged,
                      const uint16_t* d_staged_rows, size_t count, int zero_padding, uint16_t* d_k,
                      uint16_t* d_v, hsb_device_status* d_status, void* stream);

/* ------------------------------------------------------ layer executor
 * The model-facing decode step of GQALayerExecutor::prepare
 * (runtime/gqa_executor.cpp:149-249) with the attention hook of
 * patches/llama-b6000-round2.patch:218-244, on the GPU end to end: the
 * model's current K/V is appended to the HBM cache, the rehearsal query is
 * rounded to F16, and attention runs over the selected live slots only -- no
 * padded per-head K/V/mask workspace, no host copy, no upload.
 *
 * d_current: the model's current KV tensor, ggml_concat(k_cur, v_cur, 0) in
 * F16, [n_tokens][8 KV heads][K 128 | V 128].  d_cache: token-major cache
 * rows [capacity][2048 words] (K[8][128] then V[8][128]).  A non-finite F16
 * in the current KV sets HSB_E_EXECUTOR_NONFINITE_KV (index = token). */
int hsb_executor_append(const uint16_t* d_current, size_t n_tokens, uint16_t* d_cache, size_t capacity,
                        size_t first_position, hsb_device_status* d_status, void* stream);
/* query_f16 (policy/full_gqa_runtime.cpp:61-64) of the F32 rehearsal
 * [32][128]: HSB_E_EXECUTOR_REHEARSAL for a non-finite input,
 * HSB_E_EXECUTOR_REHEARSAL_F16 when its F16 overflows. */
int hsb_executor_query(const float* d_rehearsal, uint16_t* d_q16, hsb_device_status* d_status, void* stream);
size_t hsb_executor_workspace_bytes(size_t capacity, size_t count);
/* One decode layer: append the current token at `position`, then either
 * dense attention over [0, position] (dense != 0: layers 0-1) or the
 * selected-KV layer step with the rehearsal as the selection query and d_q
 * (the layer's own F32 query) for attention; d_out F32 [32][128] (the
 * model's kqv_out layout).  buffers->workspace >= hsb_executor_workspace_bytes. */
int hsb_executor_decode_layer(const uint16_t* d_current, const float* d_rehearsal, const float* d_q,
                              uint16_t* d_cache, size_t capacity, size_t position, int dense, float alpha,
                              float ratio, size_t count, const hsb_layer_buffers* buffers, float* d_out,
                              hsb_device_status* d_status, void* stream);

/* ------------------------------------------------------ synthetic inputs
 * Benchmark inputs, not part of the reference interface, defined so that a
 * CPU program reproduces them bit for bit.  Sample i of stream `seed`:
 * a = mix64(seed ^ mix64(i)), b = mix64(a) (mix64 = the splitmix64
 * finaliser), u1 = ((a >> 12) + 0.5) * 2^-52, u2 = ((b >> 12) + 0.5) * 2^-52,
 * value = sqrt(-2 ln u1) * cos(2 pi u2) * stddev in IEEE double, one rounding
 * per operation, with ln, e^x and sin/cos of 2 pi x evaluated by fixed series
 * (the formulas are in csrc/synth.cu), then rounded to F32 and to F16 (or
 * BF16) with round-to-nearest-even.  Key rows (1024 words each, at
 * stride_words): token t is heavy when mix64(seed * 0x2545f4914f6cdd1d + t)
 * < heavy_fraction * 2^64, its values then times heavy_scale; rope != 0
 * rotates channel pair (2i, 2i+1) of every KV head by t * theta^(-i/64)
 * (NORM mode), in double, before the rounding. */
int hsb_synth_normal_f16(uint16_t* d_out, size_t count, uint64_t seed, float stddev,
                         void* stream);
int hsb_synth_normal_bf16(uint16_t* d_out, size_t count, uint64_t seed, float stddev,
                          void* stream);
int hsb_synth_keys(uint16_t* d_rows, size_t tokens, size_t stride_words, uint64_t seed,
                   float heavy_fraction, float heavy_scale, int rope, float theta,
                   void* stream);

#ifdef __cplusplus
}
#endif
#endif
