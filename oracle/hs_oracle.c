/*
 * hs_oracle.c -- CPU ORACLE FOR TESTS ONLY (see hs_oracle.h).
 *
 * Plain-C restatement of the reference selected-KV decode path.  Built with
 * -O2 -ffp-contract=off (no contraction into FMA) so that every float multiply
 * and add rounds on its
 * own, exactly like the reference (ABI.json:31-37).  Not product code.
 */
#include "hs_oracle.h"
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>


enum { H = 32, KH = 8, D = 128, GROUP = 4 };

/* policy/host_policy.cpp:9-14.  Exact widening; subnormals are m*2^-24. */
float orc_half_value(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        const float mag = ldexpf((float)man, -24);
        memcpy(&bits, &mag, 4);
        bits |= sign;
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* policy/host_policy.cpp:15-28.  Round to nearest even, overflow to
 * infinity, NaN to the canonical quiet NaN with the input's sign. */
uint16_t orc_half_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
    if (e == 0xffu) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0u));
    const int he = (int)e - 112;
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return sign;
        const uint32_t full = m | 0x800000u;
        const unsigned sh = (unsigned)(14 - he);
        uint32_t q = full >> sh;
        const uint32_t r = full & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        q += (r > half) || (r == half && (q & 1u));
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)he << 10) | (m >> 13);
    const uint32_t r = m & 0x1fffu;
    q += (r > 0x1000u) || (r == 0x1000u && (q & 1u));
    return (uint16_t)(sign | q);
}

/* policy/half_order.hpp:7-10 */
uint16_t orc_order_key(uint16_t bits) {
    if ((bits & 0x7fffu) == 0) bits = 0;
    return (bits & 0x8000u) ? (uint16_t)~bits : (uint16_t)(bits ^ 0x8000u);
}

/* ---------------------------------------------------------------- scoring */
typedef struct {
    const float* qf;
    const uint16_t* k;
    size_t stride, t0, t1, out_stride, col0;
    uint16_t* out;
} score_job;

/* One (token, physical head) at a time; each of its four query heads keeps a
 * separate accumulator that starts at +0 and adds the rounded products of
 * channels 0..127 in order (full_gqa_cpu.cpp:23-37). */
static void* score_worker(void* arg) {
    const score_job* j = (const score_job*)arg;
    float kf[D];
    for (size_t t = j->t0; t < j->t1; ++t) {
        const uint16_t* row = j->k + t * j->stride;
        for (int kh = 0; kh < KH; ++kh) {
            for (int c = 0; c < D; ++c) kf[c] = orc_half_value(row[kh * D + c]);
            for (int g = 0; g < GROUP; ++g) {
                const int h = kh * GROUP + g;
                float sum = 0.0f;
                for (int c = 0; c < D; ++c) {
                    const float product = j->qf[h * D + c] * kf[c];
                    sum = sum + product;
                }
                j->out[(size_t)h * j->out_stride + j->col0 + t] = orc_half_bits(sum);
            }
        }
    }
    return NULL;
}

int orc_score(const uint16_t* q, const uint16_t* k, size_t n, size_t stride_words,
              uint16_t* out, size_t out_stride, size_t col0, int threads) {
    if (!q || !k || !out || n == 0 || (stride_words != 1024 && stride_words != 2048) ||
        out_stride < col0 + n)
        return ORC_E_SCORE_SHAPE;
    float qf[H * D];
    for (int i = 0; i < H * D; ++i) qf[i] = orc_half_value(q[i]);
    if (threads < 1) threads = 1;
    if ((size_t)threads > n) threads = (int)n;
    if (threads > 64) threads = 64;
    score_job jobs[64];
    pthread_t tid[64];
    for (int i = 0; i < threads; ++i) {
        jobs[i] = (score_job){qf, k, stride_words, n * (size_t)i / (size_t)threads,
                              n * (size_t)(i + 1) / (size_t)threads, out_stride, col0, out};
    }
    int started = 1;
    for (int i = 1; i < threads; ++i)
        if (pthread_create(&tid[i], NULL, score_worker, &jobs[i]) == 0) ++started;
        else { score_worker(&jobs[i]); }
    score_worker(&jobs[0]);
    for (int i = 1; i < threads; ++i) pthread_join(tid[i], NULL);
    (void)started;
    return ORC_OK;
}

/* policy/full_gqa_runtime.cpp:571: half_bits(half_value(x)/std::sqrt(128.f)) */
void orc_scale(const uint16_t* raw, size_t count, uint16_t* scaled) {
    const float root = sqrtf(128.0f);
    for (size_t i = 0; i < count; ++i) scaled[i] = orc_half_bits(orc_half_value(raw[i]) / root);
}

/* Orders ids [0,n) of one score row by (order key descending, id ascending):
 * a counting sort over the 16-bit key, stable in id.  This is the total
 * order the reference's partial_sort comparator defines (gqa_policy.cpp:63-65). */
static void order_row(const uint16_t* row, size_t n, uint32_t* hist, uint64_t* order) {
    memset(hist, 0, 65536u * sizeof(uint32_t));
    for (size_t i = 0; i < n; ++i) hist[orc_order_key(row[i])]++;
    uint32_t acc = 0;
    for (int key = 65535; key >= 0; --key) {
        const uint32_t c = hist[key];
        hist[key] = acc;
        acc += c;
    }
    for (size_t i = 0; i < n; ++i) order[hist[orc_order_key(row[i])]++] = i;
}

/* policy/gqa_policy.cpp:47-70 */
int orc_select(const uint16_t* score, size_t heads, size_t stride, size_t n, float alpha,
               float ratio, int fp32_counts, uint64_t* ids, size_t kcap, uint32_t* counts,
               size_t* k_out, size_t* tied_out) {
    if (!(heads > 0 && heads <= 128 && n > 0 && n <= stride)) return ORC_E_SEL_SHAPE;
    if (!(isfinite(alpha) && alpha >= 0 && isfinite(ratio) && ratio > 0 && ratio <= 1))
        return ORC_E_SEL_PARAMS;
    float maximum = -INFINITY;
    for (size_t i = 0; i < n; ++i) {
        const float x = orc_half_value(score[i]);
        if (!isfinite(x)) return ORC_E_SEL_NONFINITE_HEAD0;
        if (maximum < x) maximum = x; /* std::max(maximum, x) */
    }
    const float threshold = orc_half_value(orc_half_bits(maximum - alpha));
    if (!isfinite(threshold)) return ORC_E_SEL_THRESHOLD;
    float total = 0.0f;
    for (size_t h = 0; h < heads; ++h) {
        uint64_t count = 0;
        for (size_t i = 0; i < n; ++i) {
            const float x = orc_half_value(score[h * stride + i]);
            if (!isfinite(x)) return ORC_E_SEL_NONFINITE;
            count += x >= threshold;
        }
        if (count > 0xffffffffull) return ORC_E_SEL_U32;
        counts[h] = (uint32_t)count;
        const float rounded = fp32_counts ? (float)count : orc_half_value(orc_half_bits((float)count));
        if (!isfinite(rounded)) return ORC_E_SEL_COUNT_F16;
        total += rounded;
    }
    const float mean = fp32_counts ? total / (float)heads
                                   : orc_half_value(orc_half_bits(total / (float)heads));
    if (!isfinite(mean)) return ORC_E_SEL_MEAN_F16;
    size_t k = (size_t)mean;
    const size_t cap = (size_t)floor((double)n * (double)ratio);
    if (cap < k) k = cap;
    if (n < k) k = n;
    if (k > kcap) return ORC_E_SEL_CAPACITY;
    uint32_t* hist = (uint32_t*)malloc(65536u * sizeof(uint32_t));
    uint64_t* order = (uint64_t*)malloc(n * sizeof(uint64_t));
    size_t tied = 0;
    for (size_t h = 0; h < heads; ++h) {
        const uint16_t* row = score + h * stride;
        order_row(row, n, hist, order);
        if (k && k < n && row[order[k - 1]] == row[order[k]]) ++tied;
        for (size_t j = 0; j < k; ++j) ids[h * kcap + j] = order[j];
    }
    free(order);
    free(hist);
    *k_out = k;
    *tied_out = tied;
    return ORC_OK;
}

/* runtime/gqa_pack.hpp:12-22 */
int orc_union(const uint64_t* ids, size_t kstride, const size_t* sizes, size_t visible,
              uint64_t* physical, size_t* physical_count) {
    if (!visible || visible > 66048) return ORC_E_UNION_BOUNDS;
    uint32_t* seen = (uint32_t*)calloc(visible, sizeof(uint32_t));
    for (size_t h = 0; h < H; ++h) {
        const uint32_t bit = 1u << h;
        for (size_t s = 0; s < sizes[h]; ++s) {
            const uint64_t id = ids[h * kstride + s];
            if (id >= visible || (seen[id] & bit)) {
                free(seen);
                return ORC_E_UNION_DUPLICATE;
            }
            seen[id] |= bit;
        }
    }
    size_t m = 0;
    for (size_t i = 0; i < visible; ++i)
        if (seen[i]) physical[m++] = i;
    free(seen);
    *physical_count = m;
    return ORC_OK;
}

/* runtime/gqa_pack.hpp:26-58.  K [slot][qhead][128]; V [qhead][128][slot];
 * mask [qhead][qpad][slot] = 0 where the selected ID is visible to the query
 * position, -inf elsewhere (including padding). */
int orc_pack(const uint64_t* ids, size_t kstride, const size_t* sizes,
             const uint64_t* positions, size_t npos, const uint64_t* physical, size_t nphys,
             const uint8_t* payload, size_t payload_bytes, size_t count, uint16_t* k,
             uint16_t* v, float* mask) {
    if (npos == 0 || npos > 256 || positions[npos - 1] >= 66048 || count == 0 || count > 66048 ||
        payload_bytes != nphys * 4096)
        return ORC_E_PACK_SHAPE;
    const size_t noff = (size_t)positions[npos - 1] + 1;
    int32_t* off = (int32_t*)malloc(noff * sizeof(int32_t));
    for (size_t i = 0; i < noff; ++i) off[i] = -1;
    for (size_t i = 0; i < nphys; ++i) {
        const uint64_t id = physical[i];
        if (id >= noff || off[id] != -1) {
            free(off);
            return ORC_E_PACK_PHYSICAL;
        }
        off[id] = (int32_t)i;
    }
    const size_t qpad = (npos + 63) / 64 * 64;
    memset(k, 0, count * 4096 * sizeof(uint16_t));
    memset(v, 0, count * 4096 * sizeof(uint16_t));
    for (size_t i = 0; i < count * qpad * H; ++i) mask[i] = -INFINITY;
    int rc = ORC_OK;
    for (size_t h = 0; h < H && rc == ORC_OK; ++h) {
        if (sizes[h] == 0 || sizes[h] > count) { rc = ORC_E_PACK_SLOTS; break; }
        const size_t kh = h / 4;
        for (size_t s = 0; s < sizes[h]; ++s) {
            const uint64_t id = ids[h * kstride + s];
            if (id >= noff || off[id] < 0) { rc = ORC_E_PACK_MISSING; break; }
            const uint8_t* src = payload + (size_t)off[id] * 4096;
            memcpy(k + s * 4096 + h * 128, src + kh * 256, 256);
            for (size_t q = 0; q < npos; ++q)
                if (id <= positions[q]) mask[(h * qpad + q) * count + s] = 0.0f;
            for (size_t d = 0; d < 128; ++d)
                memcpy(&v[(h * 128 + d) * count + s], src + 2048 + (kh * 128 + d) * 2, 2);
        }
    }
    free(off);
    return rc;
}

/* runtime/gqa_prefetch_cuda.cu:12-22 (gather_gqa) and the row checks of
 * deliver (:218).  map[h*count+s]: >=0 prefetched row, <=-2 miss row
 * (-2-index), -1 padding (zero). */
int orc_gather_map(const uint16_t* prefetched, size_t prows, const uint16_t* misses,
                   size_t mrows, const int32_t* map, size_t count, uint16_t* k, uint16_t* v) {
    for (size_t i = 0; i < count * H; ++i) {
        const int64_t row = map[i];
        if (row >= 0 && (size_t)row >= prows) return ORC_E_MAP_ROW;
        if (row <= -2 && (size_t)(-2 - row) >= mrows) return ORC_E_MAP_MISS;
    }
    for (size_t s = 0; s < count; ++s)
        for (size_t h = 0; h < H; ++h) {
            const int64_t row = map[h * count + s];
            const uint16_t* src = NULL;
            if (row >= 0) src = prefetched + (size_t)row * 2048;
            else if (row <= -2) src = misses + (size_t)(-2 - row) * 2048;
            for (size_t d = 0; d < 128; ++d) {
                const uint16_t kval = src ? src[(h / 4) * 128 + d] : 0;
                const uint16_t vval = src ? src[1024 + (h / 4) * 128 + d] : 0;
                k[(s * H + h) * 128 + d] = kval;
                v[(h * 128 + d) * count + s] = vval;
            }
        }
    return ORC_OK;
}

/* policy/full_gqa_runtime.cpp:299-344: the history-only upper-bound cover
 * used to prefetch payload rows before the current token exists. */
int orc_prefetch_cover(const uint16_t* raw, size_t capacity, size_t position, float alpha,
                       int fp32_counts, uint64_t* per_head, size_t* bound_out,
                       uint64_t* physical, size_t* physical_count) {
    const size_t by_ratio = (size_t)floor((double)(position + 1) * (double)0.2f);
    const size_t cap = position < by_ratio ? position : by_ratio;
    if (!(position && position < capacity && cap)) return ORC_E_COVER_RANGE;
    uint16_t* scaled = (uint16_t*)malloc(H * position * sizeof(uint16_t));
    const float root = sqrtf(128.0f);
    for (size_t h = 0; h < H; ++h)
        for (size_t t = 0; t < position; ++t)
            scaled[h * position + t] = orc_half_bits(orc_half_value(raw[h * capacity + t]) / root);
    float maximum = -INFINITY;
    for (size_t t = 0; t < position; ++t) {
        const float x = orc_half_value(scaled[t]);
        if (maximum < x) maximum = x;
    }
    const float threshold = orc_half_value(orc_half_bits(maximum - alpha));
    int rc = ORC_OK;
    float count_sum = 0.0f;
    if (!isfinite(threshold)) rc = ORC_E_COVER_THRESHOLD;
    for (size_t h = 0; h < H && rc == ORC_OK; ++h) {
        uint64_t count = 1; /* at most one newly appended current token */
        for (size_t t = 0; t < position; ++t)
            count += orc_half_value(scaled[h * position + t]) >= threshold;
        const float rounded = fp32_counts ? (float)count : orc_half_value(orc_half_bits((float)count));
        if (!isfinite(rounded)) { rc = ORC_E_COVER_COUNT; break; }
        count_sum += rounded;
    }
    float mean = 0.0f;
    if (rc == ORC_OK) {
        mean = fp32_counts ? count_sum / (float)H : orc_half_value(orc_half_bits(count_sum / (float)H));
        if (!(isfinite(mean) && mean >= 1.0f)) rc = ORC_E_COVER_MEAN;
    }
    if (rc != ORC_OK) {
        free(scaled);
        return rc;
    }
    size_t bound = (size_t)mean;
    if (cap < bound) bound = cap;
    uint32_t* hist = (uint32_t*)malloc(65536u * sizeof(uint32_t));
    uint64_t* order = (uint64_t*)malloc(position * sizeof(uint64_t));
    unsigned char* used = (unsigned char*)calloc(position, 1);
    for (size_t h = 0; h < H; ++h) {
        order_row(scaled + h * position, position, hist, order);
        for (size_t j = 0; j < bound; ++j) {
            per_head[h * cap + j] = order[j];
            used[order[j]] = 1;
        }
    }
    size_t m = 0;
    for (size_t t = 0; t < position; ++t)
        if (used[t]) physical[m++] = t;
    free(used);
    free(order);
    free(hist);
    free(scaled);
    *bound_out = bound;
    *physical_count = m;
    return ORC_OK;
}

/* ------------------------------------------------------------- attention */
/* ggml's soft_max_ext scale, 1.f/std::sqrt(128.f) (gqa_delivery.cpp:20), as a float */
static double scale_value(void) { return (double)(1.0f / sqrtf(128.0f)); }

static void softmax_rows(const double* x, size_t n, double* p) {
    double m = -INFINITY;
    for (size_t j = 0; j < n; ++j)
        if (x[j] > m) m = x[j];
    double sum = 0.0;
    for (size_t j = 0; j < n; ++j) {
        p[j] = (m == -INFINITY) ? 0.0 : exp(x[j] - m);
        sum += p[j];
    }
    for (size_t j = 0; j < n; ++j) p[j] = sum > 0.0 ? p[j] / sum : 0.0;
}

/* ggml graph of runtime/gqa_delivery.cpp:19-20: per query head,
 * softmax(K.q * 1/sqrt(128) + mask) . V */
void orc_attention_packed(const uint16_t* k, const uint16_t* v, const float* mask, size_t count,
                          size_t qpad, const float* q, double* out) {
    double* x = (double*)malloc(count * sizeof(double));
    double* p = (double*)malloc(count * sizeof(double));
    for (size_t h = 0; h < H; ++h) {
        for (size_t j = 0; j < count; ++j) {
            double s = 0.0;
            for (size_t d = 0; d < D; ++d)
                s += (double)orc_half_value(k[(j * H + h) * D + d]) * (double)q[h * D + d];
            x[j] = s * scale_value() + (double)mask[(h * qpad) * count + j];
        }
        softmax_rows(x, count, p);
        for (size_t d = 0; d < D; ++d) {
            double o = 0.0;
            for (size_t j = 0; j < count; ++j)
                o += p[j] * (double)orc_half_value(v[(h * D + d) * count + j]);
            out[h * D + d] = o;
        }
    }
    free(p);
    free(x);
}

void orc_attention_compact(const uint16_t* k, const uint16_t* v, size_t count,
                           const uint32_t* lengths, const float* q, double* out) {
    double* x = (double*)malloc((count ? count : 1) * sizeof(double));
    double* p = (double*)malloc((count ? count : 1) * sizeof(double));
    for (size_t h = 0; h < H; ++h) {
        const size_t n = lengths[h];
        for (size_t j = 0; j < n; ++j) {
            double s = 0.0;
            for (size_t d = 0; d < D; ++d)
                s += (double)orc_half_value(k[(j * H + h) * D + d]) * (double)q[h * D + d];
            x[j] = s * scale_value();
        }
        softmax_rows(x, n, p);
        for (size_t d = 0; d < D; ++d) {
            double o = 0.0;
            for (size_t j = 0; j < n; ++j) o += p[j] * (double)orc_half_value(v[(h * D + d) * count + j]);
            out[h * D + d] = o;
        }
    }
    free(p);
    free(x);
}

void orc_attention_dense(const uint16_t* kc, const uint16_t* vc, size_t n, size_t stride,
                         const float* q, double* out) {
    double* x = (double*)malloc(n * sizeof(double));
    double* p = (double*)malloc(n * sizeof(double));
    for (size_t h = 0; h < H; ++h) {
        const size_t kh = h / 4;
        for (size_t t = 0; t < n; ++t) {
            double s = 0.0;
            for (size_t d = 0; d < D; ++d)
                s += (double)orc_half_value(kc[t * stride + kh * D + d]) * (double)q[h * D + d];
            x[t] = s * scale_value();
        }
        softmax_rows(x, n, p);
        for (size_t d = 0; d < D; ++d) {
            double o = 0.0;
            for (size_t t = 0; t < n; ++t) o += p[t] * (double)orc_half_value(vc[t * stride + kh * D + d]);
            out[h * D + d] = o;
        }
    }
    free(p);
    free(x);
}

/* --------------------------------------------------------------- rehearsal */
static double bf16_value(uint16_t b) {
    const uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return (double)f;
}

/* q = W x, then ggml NORM-mode RoPE: adjacent channel pairs (2i, 2i+1) of each
 * 128-wide head rotate by position * theta^(-2i/128). */
void orc_rehearsal(const uint16_t* x_bf16, const uint16_t* w_bf16, uint64_t position,
                   double theta, double* q_out) {
    enum { E = 4096 };
    double* xd = (double*)malloc(E * sizeof(double));
    for (size_t i = 0; i < E; ++i) xd[i] = bf16_value(x_bf16[i]);
    for (size_t o = 0; o < E; ++o) {
        double s = 0.0;
        const uint16_t* row = w_bf16 + o * E;
        for (size_t i = 0; i < E; ++i) s += bf16_value(row[i]) * xd[i];
        q_out[o] = s;
    }
    for (size_t h = 0; h < H; ++h)
        for (size_t i = 0; i < D / 2; ++i) {
            const double angle = (double)position * pow(theta, -2.0 * (double)i / (double)D);
            const double c = cos(angle), s = sin(angle);
            const double a = q_out[h * D + 2 * i], b = q_out[h * D + 2 * i + 1];
            q_out[h * D + 2 * i] = a * c - b * s;
            q_out[h * D + 2 * i + 1] = a * s + b * c;
        }
    free(xd);
}

/* ------------------------------------------------ CPU-baseline attention
 * Stage 4 has no reference CPU implementation (it runs in ggml on the GPU).
 * For the timed CPU baseline only, these float, multithreaded ports of the
 * same graph (one thread per group of query heads) stand in for it. */
static float g_half_table[65536];
static pthread_once_t g_half_once = PTHREAD_ONCE_INIT;
static void fill_half_table(void) {
    for (uint32_t i = 0; i < 65536; ++i) g_half_table[i] = orc_half_value((uint16_t)i);
}

typedef struct {
    const uint16_t *k, *v;
    const float *mask, *q;
    size_t n, stride, count, qpad;
    float* out;
    int h0, h1, dense;
} attn_job;

static void* attn_worker(void* arg) {
    const attn_job* j = (const attn_job*)arg;
    const float scale = 1.0f / sqrtf(128.0f);
    const size_t n = j->dense ? j->n : j->count;
    float* x = (float*)malloc((n ? n : 1) * sizeof(float));
    for (int h = j->h0; h < j->h1; ++h) {
        const float* qh = j->q + h * D;
        float m = -INFINITY;
        for (size_t t = 0; t < n; ++t) {
            const uint16_t* kr = j->dense ? j->k + t * j->stride + (h / 4) * D : j->k + (t * H + h) * D;
            float s = 0.0f;
            for (int d = 0; d < D; ++d) s += g_half_table[kr[d]] * qh[d];
            s *= scale;
            if (!j->dense) s += j->mask[(size_t)h * j->qpad * j->count + t];
            x[t] = s;
            if (s > m) m = s;
        }
        float sum = 0.0f;
        for (size_t t = 0; t < n; ++t) {
            x[t] = (m == -INFINITY) ? 0.0f : expf(x[t] - m);
            sum += x[t];
        }
        float acc[D];
        for (int d = 0; d < D; ++d) acc[d] = 0.0f;
        if (j->dense) {
            for (size_t t = 0; t < n; ++t) {
                const uint16_t* vr = j->v + t * j->stride + (h / 4) * D;
                for (int d = 0; d < D; ++d) acc[d] += x[t] * g_half_table[vr[d]];
            }
        } else {
            for (int d = 0; d < D; ++d) {
                const uint16_t* vr = j->v + ((size_t)h * D + d) * j->count;
                float a = 0.0f;
                for (size_t t = 0; t < n; ++t) a += x[t] * g_half_table[vr[t]];
                acc[d] = a;
            }
        }
        for (int d = 0; d < D; ++d) j->out[h * D + d] = sum > 0.0f ? acc[d] / sum : 0.0f;
    }
    free(x);
    return NULL;
}

static void run_attn(attn_job base, int threads) {
    pthread_once(&g_half_once, fill_half_table);
    if (threads < 1) threads = 1;
    if (threads > H) threads = H;
    attn_job jobs[H];
    pthread_t tid[H];
    for (int i = 0; i < threads; ++i) {
        jobs[i] = base;
        jobs[i].h0 = H * i / threads;
        jobs[i].h1 = H * (i + 1) / threads;
    }
    for (int i = 1; i < threads; ++i)
        if (pthread_create(&tid[i], NULL, attn_worker, &jobs[i]) != 0) { attn_worker(&jobs[i]); tid[i] = 0; }
    attn_worker(&jobs[0]);
    for (int i = 1; i < threads; ++i)
        if (tid[i]) pthread_join(tid[i], NULL);
}

void orc_attention_dense_f32(const uint16_t* kc, const uint16_t* vc, size_t n, size_t stride, const float* q,
                             float* out, int threads) {
    attn_job j = {kc, vc, NULL, q, n, stride, 0, 0, out, 0, 0, 1};
    run_attn(j, threads);
}

void orc_attention_packed_f32(const uint16_t* k, const uint16_t* v, const float* mask, size_t count, size_t qpad,
                              const float* q, float* out, int threads) {
    attn_job j = {k, v, mask, q, 0, 0, count, qpad, out, 0, 0, 0};
    run_attn(j, threads);
}

/* ------------------------------------------------------------------ H2O
 * runtime/gqa_h2o_stats.cu:41-57: one F32 accumulator per (KV head, key),
 * each addition rounded (this file is built with -ffp-contract=off and SSE
 * single precision, so a float add is one IEEE binary32 addition).  The
 * loops run Q head, query, key as H2OResidency::observe_attention does
 * (policy/h2o_residency.cpp:65-76): each accumulator still sees Q heads
 * 4kv..4kv+3 in turn and, within one, queries 0..Q-1 -- the CUDA kernel's
 * per-output order -- while the key loop streams through memory. */
void orc_h2o_group_sums(const void* probabilities, size_t keys, size_t queries, size_t nb0, size_t nb1,
                        size_t nb2, float* out) {
    const unsigned char* base = (const unsigned char*)probabilities;
    for (size_t i = 0; i < 8 * keys; ++i) out[i] = 0.0f;
    for (size_t h = 0; h < 32; ++h) {
        float* acc = out + (h / 4) * keys;
        for (size_t q = 0; q < queries; ++q) {
            const unsigned char* row = base + q * nb1 + h * nb2;
            for (size_t key = 0; key < keys; ++key) {
                float p;
                memcpy(&p, row + key * nb0, sizeof p);
                acc[key] = acc[key] + p;
            }
        }
    }
}

/* ------------------------------------------------------------- records */
uint64_t orc_fnv1a64(const void* data, size_t n) {
    const unsigned char* p = (const unsigned char*)data;
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

typedef struct {
    uint64_t digest, position, request;
    uint32_t layer, version;
} orc_record_header;

void orc_kv_records_encode(const void* payload, size_t payload_stride, size_t count, size_t record_bytes,
                           uint64_t request, uint32_t layer, uint64_t first, void* records) {
    const unsigned char* src = (const unsigned char*)payload;
    unsigned char* dst = (unsigned char*)records;
    for (size_t i = 0; i < count; ++i) {
        const unsigned char* row = src + i * payload_stride;
        unsigned char* rec = dst + i * (record_bytes + 32);
        orc_record_header h = {orc_fnv1a64(row, record_bytes), first + i, request, layer, 1u};
        memcpy(rec, &h, 32);
        memcpy(rec + 32, row, record_bytes);
    }
}

int orc_kv_records_verify(const void* window, size_t window_bytes, const uint64_t* offsets,
                          const uint64_t* positions, const uint32_t* groups, size_t count, uint64_t request,
                          uint32_t layer, size_t record_bytes, void* out, size_t out_stride,
                          const uint32_t* out_rows, size_t out_capacity, uint32_t* error_index) {
    const unsigned char* base = (const unsigned char*)window;
    unsigned char* dst = (unsigned char*)out;
    size_t g0 = 0;
    while (g0 < count) {  /* one validation group: records g0 .. g1-1 */
        size_t g1 = g0 + 1;
        while (groups && g1 < count && groups[g1] == groups[g0]) ++g1;
        /* bounds (our own guard), then identities, then checksums */
        for (size_t i = g0; i < g1; ++i) {
            const size_t row = out_rows ? out_rows[i] : i;
            if (offsets[i] > window_bytes || window_bytes - offsets[i] < record_bytes + 32 || row >= out_capacity) {
                *error_index = (uint32_t)i;
                return 92;
            }
        }
        for (size_t i = g0; i < g1; ++i) {
            orc_record_header h;
            memcpy(&h, base + offsets[i], 32);
            if (h.position != positions[i] || h.request != request || h.layer != layer || h.version != 1) {
                *error_index = (uint32_t)i;
                return 90;
            }
            memcpy(dst + (out_rows ? out_rows[i] : i) * out_stride, base + offsets[i] + 32, record_bytes);
        }
        for (size_t i = g0; i < g1; ++i) {
            orc_record_header h;
            memcpy(&h, base + offsets[i], 32);
            if (orc_fnv1a64(base + offsets[i] + 32, record_bytes) != h.digest) {
                *error_index = (uint32_t)i;
                return 91;
            }
        }
        g0 = g1;
    }
    return 0;
}

/* ---------------------------------------------------------------------
 * Synthetic benchmark inputs: a restatement of the library's generator
 * (hsb_synth_normal_f16 / _bf16 / hsb_synth_keys), so that the inputs the
 * benchmark times can be rebuilt on the CPU and its selections checked
 * against the reference.  Not a reference algorithm.  Every operation is an
 * IEEE double operation with one rounding (built with -ffp-contract=off), and
 * the elementary functions are series in those operations:
 *   ln m = 2 atanh((m-1)/(m+1)) on m in (1/sqrt2, sqrt2], 12 odd terms;
 *   e^r after Cody-Waite reduction by ln2 (split in two), Taylor to r^16;
 *   sin, cos of 2 pi x after folding x to [0, 1/8] turn, Taylor to t^19. */
static uint64_t syn_mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static double syn_log(double x) {
    uint64_t bits;
    memcpy(&bits, &x, 8);
    int e = (int)((bits >> 52) & 0x7ff) - 1023;
    const uint64_t mb = (bits & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
    double m;
    memcpy(&m, &mb, 8);
    if (m > 0x1.6a09e667f3bcdp+0) {
        m = m * 0.5;
        e += 1;
    }
    static const double inv_odd[12] = {
        1.0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
        0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4,
        0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5};
    const double s = (m - 1.0) / (m + 1.0);
    const double z = s * s;
    double t = inv_odd[11];
    for (int j = 10; j >= 0; --j) t = t * z + inv_odd[j];
    return (double)e * 0x1.62e42fefa39efp-1 + (s + s) * t;
}

/* 1 / n!, n = 0 .. 19 */
static const double syn_inv_fact[20] = {
    1.0, 1.0, 0.5, 0x1.5555555555555p-3, 0x1.5555555555555p-5, 0x1.1111111111111p-7,
    0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13, 0x1.a01a01a01a01ap-16, 0x1.71de3a556c734p-19,
    0x1.27e4fb7789f5cp-22, 0x1.ae64567f544e4p-26, 0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33,
    0x1.93974a8c07c9dp-37, 0x1.ae7f3e733b81fp-41, 0x1.ae7f3e733b81fp-45, 0x1.952c77030ad4ap-49,
    0x1.6827863b97d97p-53, 0x1.2f49b46814157p-57};

static double syn_exp(double x) {
    const double k = rint(x * 0x1.71547652b82fep+0);
    const double r = (x - k * 0x1.62e42feep-1) - k * 0x1.a39ef35793c76p-33;
    double p = syn_inv_fact[16];
    for (int n = 15; n >= 0; --n) p = p * r + syn_inv_fact[n];
    const uint64_t tb = (uint64_t)((int)k + 1023) << 52;
    double two_k;
    memcpy(&two_k, &tb, 8);
    return p * two_k;
}

static void syn_sincos_turns(double x, double* sn, double* cs) {
    const double y = x - rint(x);
    const int neg = y < 0.0;
    double a = neg ? -y : y;
    int flip_cos = 0, swap = 0;
    if (a > 0.25) {
        a = 0.5 - a;
        flip_cos = 1;
    }
    if (a > 0.125) {
        a = 0.25 - a;
        swap = 1;
    }
    const double t = a * 0x1.921fb54442d18p+2;
    const double z = t * t;
    /* alternating signs: odd powers for sin, even for cos */
    double ps = -syn_inv_fact[19];
    for (int n = 17, sg = 1; n >= 1; n -= 2, sg = -sg) ps = ps * z + (sg > 0 ? syn_inv_fact[n] : -syn_inv_fact[n]);
    const double s = t * ps;
    double pc = -syn_inv_fact[18];
    for (int n = 16, sg = 1; n >= 0; n -= 2, sg = -sg) pc = pc * z + (sg > 0 ? syn_inv_fact[n] : -syn_inv_fact[n]);
    double s2 = swap ? pc : s, c2 = swap ? s : pc;
    if (flip_cos) c2 = -c2;
    if (neg) s2 = -s2;
    *sn = s2;
    *cs = c2;
}

static double syn_normal(uint64_t seed, uint64_t i) {
    const uint64_t a = syn_mix64(seed ^ syn_mix64(i));
    const uint64_t b = syn_mix64(a);
    const double u1 = ((double)(a >> 12) + 0.5) * 0x1p-52;
    const double u2 = ((double)(b >> 12) + 0.5) * 0x1p-52;
    double s, c;
    syn_sincos_turns(u2, &s, &c);
    return sqrt(-2.0 * syn_log(u1)) * c;
}

static uint16_t syn_round16(double v, int bf16) {
    const float f = (float)v;
    if (!bf16) return orc_half_bits(f);
    uint32_t x;
    memcpy(&x, &f, 4);
    return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16); /* RNE; the inputs are finite */
}

typedef struct {
    uint16_t* out;
    size_t begin, end, stride;
    uint64_t seed, heavy_cut;
    double stddev, heavy_scale, ln_theta;
    int bf16, rope, keys;
} syn_job;

static void* syn_worker(void* arg) {
    const syn_job* j = (const syn_job*)arg;
    if (!j->keys) {
        for (size_t i = j->begin; i < j->end; ++i) j->out[i] = syn_round16(syn_normal(j->seed, i) * j->stddev, j->bf16);
        return NULL;
    }
    for (size_t t = j->begin; t < j->end; ++t) {
        const double scale = syn_mix64(j->seed * 0x2545f4914f6cdd1dull + t) < j->heavy_cut ? j->heavy_scale : 1.0;
        uint16_t* row = j->out + t * j->stride;
        for (size_t c2 = 0; c2 < 1024; c2 += 2) {
            double a = syn_normal(j->seed, t * 1024 + c2) * scale;
            double b = syn_normal(j->seed, t * 1024 + c2 + 1) * scale;
            if (j->rope) {
                const double pair = (double)((c2 & 127) >> 1);
                const double inv_freq = syn_exp(-(pair * 0x1p-6) * j->ln_theta);
                const double turns = ((double)t * inv_freq) * 0x1.45f306dc9c883p-3;
                double s, c;
                syn_sincos_turns(turns, &s, &c);
                const double ra = a * c - b * s;
                const double rb = a * s + b * c;
                a = ra;
                b = rb;
            }
            row[c2] = syn_round16(a, 0);
            row[c2 + 1] = syn_round16(b, 0);
        }
    }
    return NULL;
}

static void syn_run(syn_job base, size_t total, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 128) threads = 128;
    pthread_t tid[128];
    syn_job jobs[128];
    const size_t per = (total + (size_t)threads - 1) / (size_t)threads;
    for (int i = 0; i < threads; ++i) {
        jobs[i] = base;
        jobs[i].begin = (size_t)i * per < total ? (size_t)i * per : total;
        jobs[i].end = jobs[i].begin + per < total ? jobs[i].begin + per : total;
        if (i == 0 || pthread_create(&tid[i], NULL, syn_worker, &jobs[i]) != 0) {
            if (i) syn_worker(&jobs[i]);
            tid[i] = 0;
        }
    }
    syn_worker(&jobs[0]);
    for (int i = 1; i < threads; ++i)
        if (tid[i]) pthread_join(tid[i], NULL);
}

void orc_synth_normal(uint16_t* out, size_t count, uint64_t seed, float stddev, int bf16, int threads) {
    syn_job j;
    memset(&j, 0, sizeof j);
    j.out = out;
    j.seed = seed;
    j.stddev = (double)stddev;
    j.bf16 = bf16;
    syn_run(j, count, threads);
}

void orc_synth_keys(uint16_t* rows, size_t tokens, size_t stride_words, uint64_t seed, float heavy_fraction,
                    float heavy_scale, int rope, float theta, int threads) {
    syn_job j;
    memset(&j, 0, sizeof j);
    j.out = rows;
    j.stride = stride_words;
    j.seed = seed;
    j.heavy_cut = !(heavy_fraction > 0.0f) ? 0
                  : heavy_fraction >= 1.0f ? ~0ull
                                           : (uint64_t)((double)heavy_fraction * 18446744073709551616.0);
    j.heavy_scale = (double)heavy_scale;
    j.rope = rope;
    j.ln_theta = rope ? syn_log((double)theta) : 0.0;
    j.keys = 1;
    syn_run(j, tokens, threads);
}
