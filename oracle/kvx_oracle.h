/*
 * kvx_oracle.h -- CPU restatement of the reference KV-cache algorithms.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA kernels of the engine: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The engine never links it and
 * has no CPU fallback through it.
 *
 * Every function restates one reference function (cited file:line, paths
 * relative to the reference project root).  Parity of this restatement is
 * pinned against the reference itself: tests/golden/ holds vectors produced
 * by the reference sources compiled unmodified (oracle/Makefile, target
 * `ref`), and tests/test_oracle_golden.py checks every function here
 * against them.
 */
#ifndef KVX_ORACLE_H
#define KVX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* compression/kv_compress.cpp:6-25 (float_to_half): truncating fp32->fp16,
 * exp>15 -> +-Inf (NaN -> Inf), exp<=-15 -> +-0. */
uint16_t kvo_f32_to_f16_trunc(float f);
/* compression/kv_compress.cpp:27-46 (half_to_float): subnormals -> +-0. */
float kvo_f16_trunc_to_f32(uint16_t h);
/* compression/kv_compress.cpp:48-60 (vector wrappers). */
void kvo_encode_f16_trunc(const float *in, uint16_t *out, size_t n);
void kvo_decode_f16_trunc(const uint16_t *in, float *out, size_t n);

/* native-engine/cpp/KVCompressionEngine.cpp:83-113 (compressToINT8).
 * stats[4] = {minVal, maxVal, scale, zeroPoint}
 * (native-engine/include/KVCompressionEngine.h:28-34). */
void kvo_compress_int8(const float *in, int8_t *out, size_t count, float stats[4]);
/* native-engine/cpp/KVCompressionEngine.cpp:115-122 (decompressINT8). */
void kvo_decompress_int8(const int8_t *in, float *out, size_t count, const float stats[4]);

/* Block-wise wrappers over a page pool: block b covers elements
 * [b*block_elems, (b+1)*block_elems); one reference compress call per block.
 * Input is IEEE fp16 bits (widened exactly to fp32) or fp32. */
void kvo_compress_int8_blocks_f16(const uint16_t *in, int8_t *codes, float *stats,
                                  size_t num_blocks, size_t block_elems);
void kvo_compress_int8_blocks_f32(const float *in, int8_t *codes, float *stats,
                                  size_t num_blocks, size_t block_elems);
void kvo_decompress_int8_blocks(const int8_t *codes, const float *stats, float *out,
                                size_t num_blocks, size_t block_elems);

/* native-engine/cpp/KVCompressionEngine.cpp:124-180: uniform 4-bit codes,
 * two per byte (high nibble first); blocks of block_elems take
 * (block_elems + 1) / 2 code bytes each. */
void kvo_compress_nf4(const float *in, uint8_t *out, size_t count, float stats[4]);
void kvo_decompress_nf4(const uint8_t *in, float *out, size_t count, const float stats[4]);
void kvo_compress_nf4_blocks_f16(const uint16_t *in, uint8_t *codes, float *stats,
                                 size_t num_blocks, size_t block_elems);
void kvo_compress_nf4_blocks_f32(const float *in, uint8_t *codes, float *stats,
                                 size_t num_blocks, size_t block_elems);
void kvo_decompress_nf4_blocks(const uint8_t *codes, const float *stats, float *out,
                               size_t num_blocks, size_t block_elems);
/* native-engine/cpp/KVCompressionEngine.cpp:36-80: the engine's own fp16
 * conversion (exponent rebiased with wrap-around, mantissa truncated). */
uint16_t kvo_fp16_wrap_encode(float f);
float kvo_fp16_wrap_decode(uint16_t h);
void kvo_fp16_wrap_encode_n(const float *in, uint16_t *out, size_t n);
void kvo_fp16_wrap_decode_n(const uint16_t *in, float *out, size_t n);

/* IEEE fp16 <-> fp32 (round to nearest even), used to share input bits. */
float kvo_f16_to_f32(uint16_t h);
uint16_t kvo_f32_to_f16_rn(float f);

/* Paged append (KVManager::save_page, cache/kv_cache.cpp:111-127, with the
 * page geometry of the engine): for every sequence s, token t = positions[s]
 * is written to physical page block_table[s*max_pages + t/page_tokens],
 * slot t%page_tokens.  Pool layout [page][2 (K,V)][hkv][page_tokens][head_dim]
 * with elem_bytes-wide elements (copied bit-for-bit).  new_k/new_v are
 * [batch][hkv][head_dim].  Returns 0, or -1 on an out-of-range page. */
int kvo_append(void *pool, size_t elem_bytes, int num_pages, int hkv, int head_dim,
               int page_tokens, const int32_t *block_table, int max_pages,
               const int32_t *positions, int batch, const void *new_k, const void *new_v);

/* Single-query attention of runtime/tensor_ops.cpp:179-219 (row loop order,
 * scale 1/sqrt(dim) applied after the dot, ssum==0 -> 1e-6).  q:[dim],
 * k,v:[T][dim] fp32 contiguous. */
void kvo_attention_row(const float *q, const float *k, const float *v, size_t T,
                       size_t dim, float *out);

/* Paged GQA decode: for each sequence s and q-head h, kv-head h/(hq/hkv),
 * attend over tokens [0, seq_lens[s]) gathered through the block table.
 * kv_dtype: 0 fp32, 1 fp16 (IEEE, widened exactly), 2 int8 codes with
 * stats [page][2][hkv][4] (dequantised with decompressINT8 first).
 * q/out: [batch][hq][head_dim] fp32.  Returns 0 or -1. */
int kvo_paged_decode(const void *pool, int kv_dtype, const float *stats, int num_pages,
                     int hkv, int head_dim, int page_tokens, const int32_t *block_table,
                     int max_pages, const int32_t *seq_lens, int batch, int hq,
                     const float *q, float *out);

/* LRUEvictionPolicy::selectPageToEvict
 * (native-engine/cpp/AdvancedEvictionPolicy.cpp:9-23) and
 * KVCacheGPU::findLRUPage (native-engine/cpp/KVCacheGPU.cpp:54-66):
 * index of the strictly smallest stamp, first index wins ties; -1 if n==0. */
int kvo_lru_select(const uint64_t *stamps, size_t n);

/* KVManager LRU semantics (cache/kv_cache.cpp:91-127): replay a trace of
 * accesses (ops[i]==0 load_page, 1 save_page) of ids with a capacity; for
 * every access write the id evicted by it (or -1) to evicted[i] and whether
 * it was a hit to hit[i].  Returns 0. */
/* native-engine/include/AdvancedEvictionPolicy.h:19-27 (same layout). */
typedef struct kvo_evict_metrics {
    uint64_t last_access_token;
    float total_attention;
    float average_attention;
    float access_frequency;
    uint64_t creation_time;
    size_t page_size;
    int page_id;
} kvo_evict_metrics;
/* policy: 0 LRU, 1 TokenWeighted, 2 AttentionBased, 3 Predictive. */
float kvo_evict_score(int policy, const kvo_evict_metrics *m, float decay, float predicted);
int kvo_evict_select(int policy, const kvo_evict_metrics *pages, size_t n, float decay,
                     const float *predicted);
int kvo_evict_select_composite(const int *policies, const float *weights, int np,
                               const kvo_evict_metrics *pages, size_t n, float decay,
                               const float *predicted);
float kvo_predict_next_access(const uint64_t *times, size_t count);
int kvo_lru_replay(const int32_t *ids, const uint8_t *ops, size_t n, size_t capacity,
                   int32_t *evicted, uint8_t *hit);

/* KVCacheGPU (native-engine/cpp/KVCacheGPU.cpp:21-163): replays ops[n][3]
 * = (op, a, b) on a cache of total bytes and page_size:
 *   0 transferToGPU(pageId a, size b) -> 1 / 0    1 markPageUsed(a, token b)
 *   2 evictLRUPage() -> 1 / 0   3 clear()   4 getPage(a) -> lastUsedToken / -1
 * result[i] per op, used[i] = getUsedMemory() after it.  0, or -1 for a
 * negative page id in a transfer (the reference indexes out of bounds). */
int kvo_kvcache_gpu_replay(const int64_t *ops, size_t n, uint64_t total, uint64_t page_size,
                           int64_t *result, uint64_t *used);

/* Scheduler::getPrefetchDepth (scheduler/scheduler.cpp:23-37) after the
 * latencies lat[0..n) were observed (window of 16, scheduler.cpp:15-21). */
int kvo_prefetch_depth(const double *lat, size_t n, size_t cache_size,
                       size_t cache_capacity, int max_depth);

#ifdef __cplusplus
}
#endif
#endif
