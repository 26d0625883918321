/*
 * kvx_oracle.c -- CPU restatement of the reference KV-cache algorithms.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker).  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load this code;
 * the engine never calls it.  Built with -ffp-contract=off so that every
 * float expression rounds exactly like the reference's x86-64 SSE code.
 *
 * Parity of this file against the reference is pinned by the golden vectors
 * in tests/golden/ (made by the reference sources compiled unmodified).
 */
#include "kvx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- compression/kv_compress.cpp:6-25 --------------------------------- */
uint16_t kvo_f32_to_f16_trunc(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x007FFFFFu;
    int32_t e = (int32_t)((x >> 23) & 0xFFu) - 127;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);          /* overflow, Inf, NaN */
    if (e > -15) return (uint16_t)(sign | ((uint32_t)(e + 15) << 10) | (mant >> 13));
    return (uint16_t)sign;                                   /* underflow -> +-0 */
}

/* ---- compression/kv_compress.cpp:27-46 -------------------------------- */
float kvo_f16_trunc_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h & 0x7C00u) >> 10;
    uint32_t mant = (uint32_t)h & 0x03FFu;
    uint32_t x;
    if (e == 0) x = sign;                                     /* zero / subnormal */
    else if (e == 0x1F) x = sign | 0x7F800000u | (mant << 13);
    else x = sign | ((e - 15 + 127) << 23) | (mant << 13);
    float f;
    memcpy(&f, &x, sizeof f);
    return f;
}

/* ---- compression/kv_compress.cpp:48-60 -------------------------------- */
void kvo_encode_f16_trunc(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = kvo_f32_to_f16_trunc(in[i]);
}
void kvo_decode_f16_trunc(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = kvo_f16_trunc_to_f32(in[i]);
}

/* x86-64 cvttss2si: NaN and out-of-range values give INT32_MIN. */
static int32_t cvt_trunc_i32(float r) {
    if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT32_MIN;
    return (int32_t)r;
}

/* ---- native-engine/cpp/KVCompressionEngine.cpp:83-113 ----------------- */
void kvo_compress_int8(const float *in, int8_t *out, size_t count, float stats[4]) {
    float mn = in[0], mx = in[0];
    for (size_t i = 1; i < count; ++i) {
        /* std::min(a,b) == (b < a) ? b : a ; std::max(a,b) == (a < b) ? b : a */
        mn = (in[i] < mn) ? in[i] : mn;
        mx = (mx < in[i]) ? in[i] : mx;
    }
    float scale = (mx - mn) / 255.0f;
    if (scale == 0.0f) scale = 1.0f;
    stats[0] = mn;
    stats[1] = mx;
    stats[2] = scale;
    stats[3] = mn;
    for (size_t i = 0; i < count; ++i) {
        float normalized = (in[i] - mn) / scale;
        int32_t q = cvt_trunc_i32(roundf(normalized));
        if (q < 0) q = 0;
        if (q > 255) q = 255;
        out[i] = (int8_t)(q - 128);
    }
}

/* ---- native-engine/cpp/KVCompressionEngine.cpp:115-122 ---------------- */
void kvo_decompress_int8(const int8_t *in, float *out, size_t count, const float stats[4]) {
    for (size_t i = 0; i < count; ++i) {
        int32_t quantized = (int32_t)in[i] + 128;
        out[i] = stats[3] + (float)quantized * stats[2];
    }
}

float kvo_f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, sizeof v);
    return (float)v;
}

uint16_t kvo_f32_to_f16_rn(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, sizeof h);
    return h;
}

void kvo_compress_int8_blocks_f16(const uint16_t *in, int8_t *codes, float *stats,
                                  size_t num_blocks, size_t block_elems) {
    float *tmp = (float *)malloc(block_elems * sizeof(float));
    for (size_t b = 0; b < num_blocks; ++b) {
        const uint16_t *src = in + b * block_elems;
        for (size_t i = 0; i < block_elems; ++i) tmp[i] = kvo_f16_to_f32(src[i]);
        kvo_compress_int8(tmp, codes + b * block_elems, block_elems, stats + 4 * b);
    }
    free(tmp);
}

void kvo_compress_int8_blocks_f32(const float *in, int8_t *codes, float *stats,
                                  size_t num_blocks, size_t block_elems) {
    for (size_t b = 0; b < num_blocks; ++b)
        kvo_compress_int8(in + b * block_elems, codes + b * block_elems, block_elems,
                          stats + 4 * b);
}

void kvo_decompress_int8_blocks(const int8_t *codes, const float *stats, float *out,
                                size_t num_blocks, size_t block_elems) {
    for (size_t b = 0; b < num_blocks; ++b)
        kvo_decompress_int8(codes + b * block_elems, out + b * block_elems, block_elems,
                            stats + 4 * b);
}

/* ---- paged append: cache/kv_cache.cpp:111-127 with the paged geometry -- */
int kvo_append(void *pool, size_t elem_bytes, int num_pages, int hkv, int head_dim,
               int page_tokens, const int32_t *block_table, int max_pages,
               const int32_t *positions, int batch, const void *new_k, const void *new_v) {
    const size_t row = (size_t)head_dim * elem_bytes;
    for (int s = 0; s < batch; ++s) {
        int t = positions[s];
        if (t < 0 || t / page_tokens >= max_pages) return -1;
        int page = block_table[(size_t)s * max_pages + t / page_tokens];
        if (page < 0 || page >= num_pages) return -1;
        int slot = t % page_tokens;
        for (int h = 0; h < hkv; ++h) {
            for (int kv = 0; kv < 2; ++kv) {
                size_t dst = ((((size_t)page * 2 + kv) * hkv + h) * page_tokens + slot) * row;
                size_t src = ((size_t)s * hkv + h) * row;
                const char *from = (const char *)(kv == 0 ? new_k : new_v) + src;
                memcpy((char *)pool + dst, from, row);
            }
        }
    }
    return 0;
}

/* ---- runtime/tensor_ops.cpp:179-219, one query row --------------------- */
void kvo_attention_row(const float *q, const float *k, const float *v, size_t T,
                       size_t dim, float *out) {
    if (T == 0) {
        for (size_t d = 0; d < dim; ++d) out[d] = 0.0f;
        return;
    }
    float *scores = (float *)malloc(T * sizeof(float));
    const float scale = 1.0f / sqrtf((float)dim);
    for (size_t j = 0; j < T; ++j) {
        float dot = 0.0f;
        const float *kj = k + j * dim;
        for (size_t d = 0; d < dim; ++d) dot += q[d] * kj[d];
        scores[j] = dot * scale;
    }
    float maxv = scores[0];
    for (size_t j = 1; j < T; ++j) maxv = (maxv < scores[j]) ? scores[j] : maxv;
    float ssum = 0.0f;
    for (size_t j = 0; j < T; ++j) {
        scores[j] = expf(scores[j] - maxv);
        ssum += scores[j];
    }
    if (ssum == 0.0f) ssum = 1e-6f;
    for (size_t j = 0; j < T; ++j) scores[j] /= ssum;
    for (size_t d = 0; d < dim; ++d) {
        float acc = 0.0f;
        for (size_t j = 0; j < T; ++j) acc += scores[j] * v[j * dim + d];
        out[d] = acc;
    }
    free(scores);
}

static float load_elem(const void *pool, int kv_dtype, const float *stats, size_t block,
                       size_t idx) {
    switch (kv_dtype) {
    case 0: return ((const float *)pool)[idx];
    case 1: return kvo_f16_to_f32(((const uint16_t *)pool)[idx]);
    default: {
        const float *st = stats + 4 * block;
        int32_t quantized = (int32_t)((const int8_t *)pool)[idx] + 128;
        return st[3] + (float)quantized * st[2];
    }
    }
}

int kvo_paged_decode(const void *pool, int kv_dtype, const float *stats, int num_pages,
                     int hkv, int head_dim, int page_tokens, const int32_t *block_table,
                     int max_pages, const int32_t *seq_lens, int batch, int hq,
                     const float *q, float *out) {
    if (hkv <= 0 || hq % hkv != 0) return -1;
    const int group = hq / hkv;
    int tmax = 0;
    for (int s = 0; s < batch; ++s) tmax = seq_lens[s] > tmax ? seq_lens[s] : tmax;
    float *K = (float *)malloc(((size_t)tmax + 1) * head_dim * sizeof(float));
    float *V = (float *)malloc(((size_t)tmax + 1) * head_dim * sizeof(float));
    int rc = 0;
    for (int s = 0; s < batch && rc == 0; ++s) {
        const int T = seq_lens[s];
        if (T < 0 || (T + page_tokens - 1) / page_tokens > max_pages) { rc = -1; break; }
        for (int kvh = 0; kvh < hkv && rc == 0; ++kvh) {
            for (int t = 0; t < T; ++t) {
                int page = block_table[(size_t)s * max_pages + t / page_tokens];
                if (page < 0 || page >= num_pages) { rc = -1; break; }
                int slot = t % page_tokens;
                for (int kv = 0; kv < 2; ++kv) {
                    size_t block = ((size_t)page * 2 + kv) * hkv + kvh;
                    size_t base = (block * page_tokens + slot) * head_dim;
                    float *dst = (kv == 0 ? K : V) + (size_t)t * head_dim;
                    for (int d = 0; d < head_dim; ++d)
                        dst[d] = load_elem(pool, kv_dtype, stats, block, base + d);
                }
            }
            if (rc) break;
            for (int g = 0; g < group; ++g) {
                int h = kvh * group + g;
                kvo_attention_row(q + ((size_t)s * hq + h) * head_dim, K, V, (size_t)T,
                                  (size_t)head_dim, out + ((size_t)s * hq + h) * head_dim);
            }
        }
    }
    free(K);
    free(V);
    return rc;
}

/* ---- AdvancedEvictionPolicy.cpp:9-23 / KVCacheGPU.cpp:54-66 ------------ */
int kvo_lru_select(const uint64_t *stamps, size_t n) {
    int best = -1;
    uint64_t mn = UINT64_MAX;
    for (size_t i = 0; i < n; ++i) {
        if (stamps[i] < mn) {
            mn = stamps[i];
            best = (int)i;
        }
    }
    return best;
}

/* ---- cache/kv_cache.cpp:91-127: LRU list, front = most recent ---------- */
int kvo_lru_replay(const int32_t *ids, const uint8_t *ops, size_t n, size_t capacity,
                   int32_t *evicted, uint8_t *hit) {
    (void)ops; /* load_page and save_page apply the same LRU update */
    int32_t maxid = 0;
    for (size_t i = 0; i < n; ++i) {
        if (ids[i] < 0) return -1;
        if (ids[i] > maxid) maxid = ids[i];
    }
    size_t m = (size_t)maxid + 1;
    int32_t *prev = (int32_t *)malloc(m * sizeof(int32_t));
    int32_t *next = (int32_t *)malloc(m * sizeof(int32_t));
    uint8_t *in = (uint8_t *)calloc(m, 1);
    int32_t head = -1, tail = -1; /* head = front (most recent), tail = back */
    size_t size = 0;
    for (size_t i = 0; i < n; ++i) {
        int32_t id = ids[i];
        evicted[i] = -1;
        if (in[id]) {
            hit[i] = 1;
            /* unlink and push front */
            if (head != id) {
                if (prev[id] >= 0) next[prev[id]] = next[id];
                if (next[id] >= 0) prev[next[id]] = prev[id];
                if (tail == id) tail = prev[id];
                prev[id] = -1;
                next[id] = head;
                prev[head] = id;
                head = id;
            }
            continue;
        }
        hit[i] = 0;
        if (size >= capacity && tail >= 0) {
            int32_t ev = tail;
            tail = prev[ev];
            if (tail >= 0) next[tail] = -1; else head = -1;
            in[ev] = 0;
            --size;
            evicted[i] = ev;
        }
        prev[id] = -1;
        next[id] = head;
        if (head >= 0) prev[head] = id;
        head = id;
        if (tail < 0) tail = id;
        in[id] = 1;
        ++size;
    }
    free(prev);
    free(next);
    free(in);
    return 0;
}

/* ---- scheduler/scheduler.cpp:15-37 ------------------------------------- */
int kvo_prefetch_depth(const double *lat, size_t n, size_t cache_size,
                       size_t cache_capacity, int max_depth) {
    double avg = 0.0;
    if (n > 0) {
        size_t first = n > 16 ? n - 16 : 0;
        double sum = 0.0;
        for (size_t i = first; i < n; ++i) sum += lat[i];
        avg = sum / (double)(n - first);
    }
    double pressure = 0.0;
    if (cache_capacity > 0) pressure = (double)cache_size / (double)cache_capacity;
    double latency_factor = avg / 50.0;
    if (latency_factor > 2.0) latency_factor = 2.0;
    double raw = (double)max_depth * latency_factor * (1.0 - pressure);
    int r = (int)round(raw);
    int depth = r < max_depth ? r : max_depth;
    return depth > 1 ? depth : 1;
}

/* ---- native-engine/cpp/KVCompressionEngine.cpp:124-163 (compressToNF4) --
 * Uniform 4-bit asymmetric quantisation (15 steps between min and max),
 * two codes per byte, element 2k in the high nibble, 2k+1 in the low one
 * (0 when the count is odd). */
void kvo_compress_nf4(const float *in, uint8_t *out, size_t count, float stats[4]) {
    float mn = in[0], mx = in[0];
    for (size_t i = 1; i < count; ++i) {
        mn = (in[i] < mn) ? in[i] : mn;
        mx = (mx < in[i]) ? in[i] : mx;
    }
    float scale = (mx - mn) / 15.0f;
    if (scale == 0.0f) scale = 1.0f;
    stats[0] = mn;
    stats[1] = mx;
    stats[2] = scale;
    stats[3] = mn;
    for (size_t i = 0; i < count; i += 2) {
        int32_t q1 = cvt_trunc_i32(roundf((in[i] - mn) / scale));
        q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
        int32_t q2 = 0;
        if (i + 1 < count) {
            q2 = cvt_trunc_i32(roundf((in[i + 1] - mn) / scale));
            q2 = q2 < 0 ? 0 : (q2 > 15 ? 15 : q2);
        }
        out[i / 2] = (uint8_t)((q1 << 4) | q2);
    }
}

/* ---- native-engine/cpp/KVCompressionEngine.cpp:165-180 (decompressNF4) */
void kvo_decompress_nf4(const uint8_t *in, float *out, size_t count, const float stats[4]) {
    for (size_t i = 0; i < count; i += 2) {
        uint8_t packed = in[i / 2];
        out[i] = stats[3] + (float)((packed >> 4) & 0xF) * stats[2];
        if (i + 1 < count) out[i + 1] = stats[3] + (float)(packed & 0xF) * stats[2];
    }
}

void kvo_compress_nf4_blocks_f16(const uint16_t *in, uint8_t *codes, float *stats,
                                 size_t num_blocks, size_t block_elems) {
    float *tmp = (float *)malloc(block_elems * sizeof(float));
    const size_t cb = (block_elems + 1) / 2;
    for (size_t b = 0; b < num_blocks; ++b) {
        const uint16_t *src = in + b * block_elems;
        for (size_t i = 0; i < block_elems; ++i) tmp[i] = kvo_f16_to_f32(src[i]);
        kvo_compress_nf4(tmp, codes + b * cb, block_elems, stats + 4 * b);
    }
    free(tmp);
}

void kvo_compress_nf4_blocks_f32(const float *in, uint8_t *codes, float *stats,
                                 size_t num_blocks, size_t block_elems) {
    const size_t cb = (block_elems + 1) / 2;
    for (size_t b = 0; b < num_blocks; ++b)
        kvo_compress_nf4(in + b * block_elems, codes + b * cb, block_elems, stats + 4 * b);
}

void kvo_decompress_nf4_blocks(const uint8_t *codes, const float *stats, float *out,
                               size_t num_blocks, size_t block_elems) {
    const size_t cb = (block_elems + 1) / 2;
    for (size_t b = 0; b < num_blocks; ++b)
        kvo_decompress_nf4(codes + b * cb, out + b * block_elems, block_elems, stats + 4 * b);
}

/* ---- native-engine/cpp/KVCompressionEngine.cpp:36-61 (compressToFP16) --
 * Not IEEE rounding: Inf and NaN become +-Inf, a zero exponent (zero or
 * denormal) becomes +-0, and otherwise the exponent is rebiased modulo 32
 * (it wraps for |x| >= 2^16 or < 2^-14) and the mantissa truncated. */
uint16_t kvo_fp16_wrap_encode(float f) {
    uint32_t bits;
    memcpy(&bits, &f, sizeof bits);
    uint32_t sign = (bits >> 31) & 1u, exponent = (bits >> 23) & 0xFFu, mantissa = bits & 0x7FFFFFu;
    if (exponent == 0xFFu) return (uint16_t)((sign << 15) | 0x7C00u);
    if (exponent == 0u) return (uint16_t)(sign << 15);
    uint32_t e16 = (uint32_t)((int32_t)exponent - 127 + 15) & 0x1Fu;
    return (uint16_t)((sign << 15) | (e16 << 10) | ((mantissa >> 13) & 0x3FFu));
}

/* ---- native-engine/cpp/KVCompressionEngine.cpp:63-80 (decompressFP16) -
 * The exponent is rebiased modulo 256 with no special cases: a zero
 * exponent decodes to +-2^-15 x (1 + m), exponent 31 to 2^16 x (1 + m). */
float kvo_fp16_wrap_decode(uint16_t h) {
    uint32_t sign = ((uint32_t)h >> 15) & 1u, e = ((uint32_t)h >> 10) & 0x1Fu, m = (uint32_t)h & 0x3FFu;
    uint32_t bits = (sign << 31) | (((e + 127u - 15u) & 0xFFu) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

void kvo_fp16_wrap_encode_n(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = kvo_fp16_wrap_encode(in[i]);
}
void kvo_fp16_wrap_decode_n(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = kvo_fp16_wrap_decode(in[i]);
}

/* ---- native-engine/cpp/AdvancedEvictionPolicy.cpp: the policies' scores as
 * selectPageToEvict evaluates them, i.e. with currentToken = 0, so every
 * token age is 0 - lastAccessToken modulo 2^64. */
float kvo_evict_score(int policy, const kvo_evict_metrics *m, float decay, float predicted) {
    const uint64_t age = (uint64_t)0 - m->last_access_token;
    switch (policy) {
    case 0: /* LRU :29-31 */
        return (float)age;
    case 1: /* TokenWeighted :60-64 */
        return 1.0f - powf(decay, (float)age);
    case 2: { /* AttentionBased :95-105 */
        const float recency = logf((float)age + 1.0f);
        return (1.0f - m->average_attention) * recency;
    }
    default: /* Predictive :142-152 */
        if (predicted < 0) return 1000.0f;
        return (float)(uint64_t)0 - predicted;
    }
}

/* selectPageToEvict (:9-23 LRU; :35-50, :69-84, :119-135 the others). */
int kvo_evict_select(int policy, const kvo_evict_metrics *pages, size_t n, float decay,
                     const float *predicted) {
    if (n == 0) return -1;
    int sel = -1;
    if (policy == 0) {
        uint64_t mn = UINT64_MAX;
        for (size_t i = 0; i < n; ++i)
            if (pages[i].last_access_token < mn) {
                mn = pages[i].last_access_token;
                sel = pages[i].page_id;
            }
        return sel;
    }
    float best = -1.0f;
    for (size_t i = 0; i < n; ++i) {
        const float s = kvo_evict_score(policy, &pages[i], decay, predicted ? predicted[i] : -1.0f);
        if (s > best) {
            best = s;
            sel = pages[i].page_id;
        }
    }
    return sel;
}

/* CompositeEvictionManager::selectPageToEvict with several policies
 * (:238-263): scores[i] += weights[p] * calculateScore_p(m, 0), policy
 * order, then the highest score > -1 (first wins).  One policy: that
 * policy's selectPageToEvict. */
int kvo_evict_select_composite(const int *policies, const float *weights, int np,
                               const kvo_evict_metrics *pages, size_t n, float decay,
                               const float *predicted) {
    if (n == 0) return -1;
    if (np == 1) return kvo_evict_select(policies[0], pages, n, decay, predicted);
    int sel = -1;
    float best = -1.0f;
    for (size_t i = 0; i < n; ++i) {
        float s = 0.0f;
        for (int p = 0; p < np; ++p)
            s += weights[p] * kvo_evict_score(policies[p], &pages[i], decay, predicted ? predicted[i] : -1.0f);
        if (s > best) {
            best = s;
            sel = pages[i].page_id;
        }
    }
    return sel;
}

/* PredictiveEvictionPolicy::predictNextAccess (:154-172): the last access
 * plus the mean interval (integer division), as float; -1 with fewer than
 * two accesses. */
float kvo_predict_next_access(const uint64_t *times, size_t count) {
    if (count < 2) return -1.0f;
    uint64_t total = 0;
    for (size_t i = 1; i < count; ++i) total += times[i] - times[i - 1];
    return (float)(times[count - 1] + total / (count - 1));
}

/* ---- KVCacheGPU page policy (native-engine/cpp/KVCacheGPU.cpp) ----------- */

int kvo_kvcache_gpu_replay(const int64_t *ops, size_t n, uint64_t total, uint64_t page_size,
                           int64_t *result, uint64_t *used_out) {
    (void)page_size; /* maxPages is computed but never consulted (KVCacheGPU.cpp:9) */
    int64_t maxid = -1;
    for (size_t i = 0; i < n; ++i) {
        if ((ops[3 * i] == 0) && ops[3 * i + 1] < 0) return -1;
        if ((ops[3 * i] == 0 || ops[3 * i] == 1 || ops[3 * i] == 4) && ops[3 * i + 1] > maxid)
            maxid = ops[3 * i + 1];
    }
    size_t cap = (size_t)(maxid + 1);
    uint8_t *live = (uint8_t *)calloc(cap ? cap : 1, 1);
    uint64_t *size = (uint64_t *)calloc(cap ? cap : 1, sizeof(uint64_t));
    uint64_t *last = (uint64_t *)calloc(cap ? cap : 1, sizeof(uint64_t));
    size_t len = 0; /* pages.size() */
    uint64_t used = 0;
    for (size_t i = 0; i < n; ++i) {
        const int64_t op = ops[3 * i], a = ops[3 * i + 1], b = ops[3 * i + 2];
        int64_t r = 0;
        /* evictLRUPage (:136-152) over findLRUPage (:54-66): the first page
         * with the strictly smallest lastUsedToken */
#define KVO_EVICT(res)                                                        \
        do {                                                                  \
            int64_t lru = -1;                                                 \
            uint64_t mn = UINT64_MAX;                                         \
            for (size_t k = 0; k < len; ++k)                                  \
                if (live[k] && last[k] < mn) {                                \
                    mn = last[k];                                             \
                    lru = (int64_t)k;                                         \
                }                                                             \
            if (lru < 0) {                                                    \
                (res) = 0;                                                    \
            } else {                                                          \
                used -= size[lru];                                            \
                live[lru] = 0;                                                \
                (res) = 1;                                                    \
            }                                                                 \
        } while (0)
        if (op == 0) {
            /* allocateGPUPage (:21-40): over the budget -> null; a 0-byte
             * cudaMalloc succeeds with a null pointer (nothing counted) */
            uint64_t want = (uint64_t)b;
            int got = used + want <= total && want > 0;
            if (got) used += want;
            if (!got) { /* transferToGPU (:68-79): evict once and retry */
                int ev;
                KVO_EVICT(ev);
                if (ev) {
                    got = used + want <= total && want > 0;
                    if (got) used += want;
                }
            }
            if (got) { /* :89-105; a replaced entry's bytes stay counted */
                if ((size_t)a >= len) len = (size_t)a + 1;
                live[a] = 1;
                size[a] = want;
                last[a] = 0;
            }
            r = got;
        } else if (op == 1) {
            if (a >= 0 && (size_t)a < len && live[a]) last[a] = (uint64_t)b;
        } else if (op == 2) {
            KVO_EVICT(r);
        } else if (op == 3) {
            memset(live, 0, cap ? cap : 1);
            len = 0;
            used = 0;
        } else if (op == 4) {
            r = (a >= 0 && (size_t)a < len && live[a]) ? (int64_t)last[a] : -1;
        }
#undef KVO_EVICT
        result[i] = r;
        used_out[i] = used;
    }
    free(live);
    free(size);
    free(last);
    return 0;
}
