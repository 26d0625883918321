// ref_harness.cpp -- extern "C" entry points over the reference's own CPU
// code, compiled together with the reference sources where they lie
// (oracle/Makefile, target `ref`) into oracle/_ref/libkvref.so.
//
// TEST INFRASTRUCTURE ONLY: this is how the golden vectors in tests/golden/
// are produced and how bench.py's reference arm times the reference.  Every
// function below calls the reference function it names, unmodified; the
// only code of ours here is argument marshalling and the thread fan-out of
// the timing helpers.
#include "kv_cache.h"                 // cache/kv_cache.h
#include "kv_compress.h"              // compression/kv_compress.h
#include "KVCompressionEngine.h"      // native-engine/include
#include "AdvancedEvictionPolicy.h"   // native-engine/include
#include "tensor_ops.h"               // runtime/tensor_ops.h
#include "scheduler.h"                // scheduler/scheduler.h
#include "layer_cache.h"              // cache/layer_cache.h

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <set>
#include <string>
#include <thread>
#include <vector>

extern "C" {

// compression/kv_compress.cpp:48-53
void kvref_f32_to_f16(const float *in, uint16_t *out, size_t n) {
    std::vector<float> v(in, in + n);
    auto r = float32_to_float16(v);
    std::memcpy(out, r.data(), n * sizeof(uint16_t));
}

// compression/kv_compress.cpp:55-60
void kvref_f16_to_f32(const uint16_t *in, float *out, size_t n) {
    std::vector<uint16_t> v(in, in + n);
    auto r = float16_to_float32(v);
    std::memcpy(out, r.data(), n * sizeof(float));
}

// native-engine/cpp/KVCompressionEngine.cpp:185-203 (compress, INT8)
void kvref_compress_int8(const float *in, int8_t *out, size_t count, float *stats) {
    static thread_local KVCompressionEngine *eng = nullptr;
    if (!eng) {
        eng = new KVCompressionEngine();
        eng->setCompressionType(CompressionType::INT8);
    }
    QuantizationStats st{};
    eng->compress(in, out, count, st);
    stats[0] = st.minVal;
    stats[1] = st.maxVal;
    stats[2] = st.scale;
    stats[3] = st.zeroPoint;
}

// native-engine/cpp/KVCompressionEngine.cpp:212-233 (decompress, INT8)
void kvref_decompress_int8(const int8_t *in, float *out, size_t count, const float *stats) {
    static thread_local KVCompressionEngine *eng = nullptr;
    if (!eng) eng = new KVCompressionEngine();
    QuantizationStats st{};
    st.minVal = stats[0];
    st.maxVal = stats[1];
    st.scale = stats[2];
    st.zeroPoint = stats[3];
    st.type = CompressionType::INT8;
    eng->decompress(in, out, count, st);
}

// native-engine/cpp/KVCompressionEngine.cpp:124-163 via compress() with NF4
void kvref_compress_nf4(const float *in, uint8_t *out, size_t count, float *stats) {
    static thread_local KVCompressionEngine *eng = nullptr;
    if (!eng) {
        eng = new KVCompressionEngine();
        eng->setCompressionType(CompressionType::NF4);
    }
    QuantizationStats st{};
    eng->compress(in, out, count, st);
    stats[0] = st.minVal;
    stats[1] = st.maxVal;
    stats[2] = st.scale;
    stats[3] = st.zeroPoint;
}

// native-engine/cpp/KVCompressionEngine.cpp:165-180 via decompress() with NF4
void kvref_decompress_nf4(const uint8_t *in, float *out, size_t count, const float *stats) {
    static thread_local KVCompressionEngine *eng = nullptr;
    if (!eng) eng = new KVCompressionEngine();
    QuantizationStats st{};
    st.minVal = stats[0];
    st.maxVal = stats[1];
    st.scale = stats[2];
    st.zeroPoint = stats[3];
    st.type = CompressionType::NF4;
    eng->decompress(in, out, count, st);
}

// native-engine/cpp/KVCompressionEngine.cpp:36-80 via compress()/decompress() with FP16
void kvref_fp16_wrap_encode(const float *in, uint16_t *out, size_t count) {
    static thread_local KVCompressionEngine *eng = nullptr;
    if (!eng) {
        eng = new KVCompressionEngine();
        eng->setCompressionType(CompressionType::FP16);
    }
    QuantizationStats st{};
    eng->compress(in, out, count, st);
}

void kvref_fp16_wrap_decode(const uint16_t *in, float *out, size_t count) {
    static thread_local KVCompressionEngine *eng = nullptr;
    if (!eng) eng = new KVCompressionEngine();
    QuantizationStats st{};
    st.type = CompressionType::FP16;
    eng->decompress(in, out, count, st);
}

// native-engine/cpp/AdvancedEvictionPolicy.cpp: selectPageToEvict of one
// policy and every page's calculateScore(m, 0).  Predictive: hist holds,
// per page, up to 10 access tokens (hist_len[i] of them) replayed through
// recordAccess first.
static std::unique_ptr<EvictionPolicy> make_policy(int policy, float decay) {
    switch (policy) {
    case 0: return std::make_unique<LRUEvictionPolicy>();
    case 1: return std::make_unique<TokenWeightedEvictionPolicy>(decay);
    case 2: return std::make_unique<AttentionBasedEvictionPolicy>();
    default: return std::make_unique<PredictiveEvictionPolicy>();
    }
}

int kvref_evict_select(int policy, const EvictionMetrics *pages, size_t n, float decay,
                       const uint64_t *hist, const int32_t *hist_len, float *scores) {
    auto pol = make_policy(policy, decay);
    if (policy == 3 && hist) {
        auto *pp = static_cast<PredictiveEvictionPolicy *>(pol.get());
        for (size_t i = 0; i < n; ++i)
            for (int k = 0; k < hist_len[i]; ++k) pp->recordAccess(pages[i].pageId, hist[i * 10 + k]);
    }
    std::vector<EvictionMetrics> v(pages, pages + n);
    if (scores)
        for (size_t i = 0; i < n; ++i) scores[i] = pol->calculateScore(v[i], 0);
    return pol->selectPageToEvict(v);
}

// CompositeEvictionManager (:176-263) with the given policies and raw
// weights (normalised by the manager), pages registered in order.
int kvref_evict_composite(const int32_t *policies, const float *weights, int np,
                          const EvictionMetrics *pages, size_t n, float *norm_weights) {
    CompositeEvictionManager mgr;
    mgr.switchPolicy(static_cast<EvictionStrategy>(policies[0]));
    for (int p = 1; p < np; ++p) {
        switch (policies[p]) {
        case 0: mgr.addPolicy(std::make_unique<LRUEvictionPolicy>(), weights[p]); break;
        case 1: mgr.addPolicy(std::make_unique<TokenWeightedEvictionPolicy>(), weights[p]); break;
        case 2: mgr.addPolicy(std::make_unique<AttentionBasedEvictionPolicy>(), weights[p]); break;
        default: mgr.addPolicy(std::make_unique<PredictiveEvictionPolicy>(), weights[p]); break;
        }
    }
    std::vector<float> w(weights, weights + np);
    mgr.setPolicyWeights(w);
    float total = 0.0f;
    for (float x : w) total += x;
    for (int p = 0; p < np; ++p) norm_weights[p] = w[p] / total;
    for (size_t i = 0; i < n; ++i) mgr.updatePageMetrics(pages[i].pageId, pages[i]);
    return mgr.selectPageToEvict();
}

// runtime/tensor_ops.cpp:179-219
int kvref_attention(const float *Q, const float *K, const float *V, size_t seq, size_t dim,
                    float *out) {
    try {
        std::vector<float> q(Q, Q + seq * dim), k(K, K + seq * dim), v(V, V + seq * dim);
        auto r = runtime::TensorOps::attention(q, k, v, seq, dim);
        std::memcpy(out, r.data(), r.size() * sizeof(float));
        return 0;
    } catch (...) {
        return -1;
    }
}

// runtime/tensor_ops.cpp:155-177
int kvref_softmax(const float *logits, size_t rows, size_t cols, float *out) {
    try {
        std::vector<float> l(logits, logits + rows * cols);
        auto r = runtime::TensorOps::softmax(l, rows, cols);
        std::memcpy(out, r.data(), r.size() * sizeof(float));
        return 0;
    } catch (...) {
        return -1;
    }
}

// One decode query against T keys, composed from the reference's own
// TensorOps::matmul (tensor_ops.cpp:42-63) and TensorOps::softmax
// (tensor_ops.cpp:155-177): scores = K.q, scores *= 1/sqrt(dim) (the scale
// step of tensor_ops.cpp:186,193), p = softmax(scores), out = p.V.  The
// accumulation order of each step equals the row loop of
// TensorOps::attention, so the result equals that function's row for a
// query repeated T times, at O(T*dim) instead of O(T^2*dim).
int kvref_attention_row(const float *q, const float *K, const float *V, size_t T, size_t dim,
                        float *out) {
    try {
        if (T == 0) {
            std::memset(out, 0, dim * sizeof(float));
            return 0;
        }
        std::vector<float> k(K, K + T * dim), qv(q, q + dim), v(V, V + T * dim);
        auto scores = runtime::TensorOps::matmul(k, qv, T, dim, 1);
        const float scale = 1.0f / std::sqrt((float)dim);
        for (auto &s : scores) s = s * scale;
        auto p = runtime::TensorOps::softmax(scores, 1, T);
        auto o = runtime::TensorOps::matmul(p, v, 1, T, dim);
        std::memcpy(out, o.data(), dim * sizeof(float));
        return 0;
    } catch (...) {
        return -1;
    }
}

// native-engine/cpp/AdvancedEvictionPolicy.cpp:9-23
int kvref_lru_select(const uint64_t *stamps, size_t n) {
    std::vector<EvictionMetrics> m(n);
    for (size_t i = 0; i < n; ++i) {
        m[i] = EvictionMetrics{};
        m[i].lastAccessToken = stamps[i];
        m[i].pageId = (int)i;
    }
    LRUEvictionPolicy p;
    return p.selectPageToEvict(m);
}

// cache/kv_cache.cpp:91-127: replay a trace through a real KVManager.
// ops[i]: 0 = load_page, 1 = save_page.  Every id of a load must have a page
// file in dir (the caller saves them first with kvref_save_page).  The id
// evicted by each access is found by probing contains() over the ids that
// were resident before it.
int kvref_lru_replay(const int32_t *ids, const uint8_t *ops, size_t n, size_t capacity,
                     const char *dir, int32_t *evicted, uint8_t *hit) {
    try {
        KVManager m(capacity, dir);
        std::set<int> resident;
        for (size_t i = 0; i < n; ++i) {
            int id = ids[i];
            hit[i] = m.contains(id) ? 1 : 0;
            if (ops[i] == 0) {
                (void)m.load_page(id);
            } else {
                KVPage p;
                p.id = id;
                p.key = {(float)id + 0.5f};
                p.value = {(float)id + 0.25f};
                m.save_page(p);
            }
            evicted[i] = -1;
            for (int r : resident) {
                if (r != id && !m.contains(r)) {
                    evicted[i] = r;
                    break;
                }
            }
            if (evicted[i] >= 0) resident.erase(evicted[i]);
            resident.insert(id);
        }
        return 0;
    } catch (...) {
        return -1;
    }
}

// cache/kv_cache.cpp:111-127 (+ persist_to_disk 21-41): write one page.
int kvref_save_page(int id, const float *key, size_t nk, const float *value, size_t nv,
                    const char *dir, size_t capacity) {
    try {
        KVManager m(capacity, dir);
        KVPage p;
        p.id = id;
        p.key.assign(key, key + nk);
        p.value.assign(value, value + nv);
        m.save_page(p);
        return 0;
    } catch (...) {
        return -1;
    }
}

// cache/kv_cache.cpp:91-109 (+ load_from_disk 43-84): read one page back.
// Returns the number of key elements (values in *nv_out), -1 on error.
long kvref_load_page(int id, const char *dir, float *key, size_t kcap, float *value,
                     size_t vcap, size_t *nv_out) {
    try {
        KVManager m(4, dir);
        KVPage p = m.load_page(id);
        std::memcpy(key, p.key.data(), std::min(kcap, p.key.size()) * sizeof(float));
        std::memcpy(value, p.value.data(), std::min(vcap, p.value.size()) * sizeof(float));
        *nv_out = p.value.size();
        return (long)p.key.size();
    } catch (...) {
        return -1;
    }
}

// scheduler/scheduler.cpp:15-37 with a LayerCache holding `size` of `capacity`.
int kvref_prefetch_depth(const double *lat, size_t n, size_t size, size_t capacity,
                         int max_depth) {
    LayerCache cache(capacity);
    for (size_t i = 0; i < size; ++i) cache.insert((int)i, Tensor(std::vector<int>{1}));
    Scheduler s(cache, max_depth);
    for (size_t i = 0; i < n; ++i) s.observeLoadLatency(lat[i]);
    return s.getPrefetchDepth(0);
}

// ---- timing helpers for the CPU baseline (thread fan-out is ours) -------

// Decode attention over `units` independent (sequence, q-head) rows, each
// with T keys of `dim`, fanned over `threads` std::threads; K/V/q per unit
// are read from the given arrays (unit u uses K + (u % kv_units)*T*dim).
// Returns elapsed seconds.
double kvref_time_decode(const float *q, const float *K, const float *V, size_t kv_units,
                         size_t units, size_t T, size_t dim, int threads, float *out) {
    std::atomic<size_t> next{0};
    auto t0 = std::chrono::steady_clock::now();
    auto work = [&]() {
        for (;;) {
            size_t u = next.fetch_add(1);
            if (u >= units) break;
            size_t kv = u % kv_units;
            kvref_attention_row(q + u * dim, K + kv * T * dim, V + kv * T * dim, T, dim,
                                out + u * dim);
        }
    };
    std::vector<std::thread> th;
    for (int i = 0; i < threads; ++i) th.emplace_back(work);
    for (auto &t : th) t.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// KVCompressionEngine INT8 over `blocks` blocks of `block_elems`, fanned over
// `threads`.  Returns elapsed seconds.
double kvref_time_compress(const float *in, int8_t *codes, float *stats, size_t blocks,
                           size_t block_elems, int threads) {
    std::atomic<size_t> next{0};
    auto t0 = std::chrono::steady_clock::now();
    auto work = [&]() {
        for (;;) {
            size_t b = next.fetch_add(1);
            if (b >= blocks) break;
            kvref_compress_int8(in + b * block_elems, codes + b * block_elems, block_elems,
                                stats + 4 * b);
        }
    };
    std::vector<std::thread> th;
    for (int i = 0; i < threads; ++i) th.emplace_back(work);
    for (auto &t : th) t.join();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// KVManager::save_page for `n` appended tokens of one sequence.  A page is
// [heads][page_tokens][head_dim] fp32 for K and for V; token t writes its
// rows ([heads][head_dim], same data for K and V) into slot t%page_tokens of
// logical page t/page_tokens and saves the whole page (the reference
// persists on every save).  Returns elapsed seconds.
double kvref_time_append(const float *rows, size_t n, size_t heads, size_t head_dim,
                         size_t page_tokens, const char *dir) {
    KVManager m(1u << 20, dir);
    const size_t page_elems = heads * page_tokens * head_dim;
    auto t0 = std::chrono::steady_clock::now();
    KVPage p;
    for (size_t t = 0; t < n; ++t) {
        size_t slot = t % page_tokens;
        if (slot == 0) {
            p.id = (int)(t / page_tokens);
            p.key.assign(page_elems, 0.0f);
            p.value.assign(page_elems, 0.0f);
        }
        for (size_t h = 0; h < heads; ++h) {
            const float *src = rows + (t * heads + h) * head_dim;
            size_t dst = (h * page_tokens + slot) * head_dim;
            std::memcpy(&p.key[dst], src, head_dim * sizeof(float));
            std::memcpy(&p.value[dst], src, head_dim * sizeof(float));
        }
        m.save_page(p);
    }
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}


// The reference's page tier (cache/kv_cache.cpp): KVManager with `capacity`
// pages in memory and every page persisted as an fp16 file in `dir`.  Saves
// pages 0..universe-1 (K and V of `page_floats` fp32 each), then times
// load_page over the id stream: a hit is a list move, a miss reads the page
// file back (fp16 -> fp32) and evicts the least recent page.  Returns
// elapsed seconds of the loads; *misses_out counts the file reads.
double kvref_time_tier(const int32_t *ids, size_t n, size_t universe, size_t capacity,
                       size_t page_floats, const char *dir, int64_t *misses_out) {
    try {
        KVManager m(capacity, dir);
        KVPage p;
        p.key.assign(page_floats, 0.5f);
        p.value.assign(page_floats, 0.25f);
        for (size_t i = 0; i < universe; ++i) {
            p.id = (int)i;
            p.key[0] = (float)i;
            m.save_page(p);
        }
        int64_t misses = 0;
        auto t0 = std::chrono::steady_clock::now();
        for (size_t i = 0; i < n; ++i) {
            if (!m.contains(ids[i])) ++misses;
            (void)m.load_page(ids[i]);
        }
        const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        *misses_out = misses;
        return s;
    } catch (...) {
        return -1.0;
    }
}

}  // extern "C"
