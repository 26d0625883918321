/*
 * kvx.h -- C ABI of the B200 (sm_100a) KV-cache kernels.
 *
 * Plain C: device pointers, sizes and a cudaStream_t passed as void*.  Every
 * entry point returns KVX_OK (0) or a negative kvx_status and never throws.
 * All work is enqueued on the given stream (NULL = legacy default stream);
 * nothing here synchronises the host unless its comment says so.
 *
 * Page pool layout (one layer):
 *     pool[num_pages][2 (0=K, 1=V)][num_kv_heads][page_tokens][head_dim]
 * so one (page, K|V, head) block of page_tokens x head_dim elements is
 * contiguous (4 KiB at fp16, 16 x 128).  For int8 pools a parallel array
 *     stats[num_pages][2][num_kv_heads][4] = {minVal, maxVal, scale, zeroPoint}
 * holds the reference's QuantizationStats of each block.
 *
 * Each entry point names the reference interface it replaces (paths
 * relative to the reference project root).
 */
#ifndef KVX_H
#define KVX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define KVX_API __declspec(dllexport)
#else
#define KVX_API __attribute__((visibility("default")))
#endif

enum kvx_status {
    KVX_OK = 0,
    KVX_EINVAL = -1,       /* bad argument, id or geometry (the reference's -1) */
    KVX_EBUSY = -2,        /* object pinned / in use (the reference's -2) */
    KVX_ECUDA = -3,        /* a CUDA runtime call or launch failed */
    KVX_EUNSUPPORTED = -4, /* geometry/dtype this build has no kernel for */
    KVX_ETIMEOUT = -5,     /* a bounded device wait expired (see error_flag) */
    KVX_ENOSPC = -6,       /* workspace / pool too small */
    KVX_ENODEV = -7,       /* no sm_100 device current */
    KVX_ETOOBIG = -8,      /* request exceeds kvx_decode_noalloc's static scratch */
    KVX_EPEER = -9         /* another rank's part of a multi-GPU engine step failed */
};

enum kvx_dtype { KVX_F32 = 0, KVX_F16 = 1, KVX_I8 = 2 };

/* One layer of the paged cache. */
typedef struct kvx_paged {
    void *pool;           /* see layout above */
    const float *stats;   /* KVX_I8 only, else NULL */
    int32_t dtype;        /* enum kvx_dtype */
    int32_t num_pages;
    int32_t num_kv_heads;
    int32_t head_dim;     /* 128 */
    int32_t page_tokens;  /* 16 */
} kvx_paged;

KVX_API const char *kvx_version(void);
KVX_API const char *kvx_status_string(int status);
/* KVX_OK when the current device is compute capability 10.x (the only
 * target this library carries code for), else KVX_ENODEV. */
KVX_API int kvx_device_check(void);

/* Paged append.  Replaces KVManager::save_page (cache/kv_cache.cpp:111-127)
 * as called by InferenceController::appendKVPage (runtime/inference.cpp:50-54):
 * for each sequence s the token at position positions[s] is stored in
 * physical page block_table[s*max_pages + pos/page_tokens], slot
 * pos % page_tokens.  new_k/new_v: [batch][num_kv_heads][head_dim] in the
 * pool's dtype (KVX_F32 or KVX_F16).  Bit-exact copy.  A position or page
 * id out of range skips that row and sets bit 1 of *error_flag (device
 * int32, may be NULL). */
KVX_API int kvx_append(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                       const int32_t *positions, int32_t batch, const void *new_k,
                       const void *new_v, int32_t *error_flag, void *stream);

/* Chunked paged append: sequence s appends n_new consecutive tokens at
 * positions[s] .. positions[s] + n_new - 1, token t going to physical page
 * block_table[s*max_pages + t/16], slot t % 16 (a prefill chunk, or a step
 * that appends several tokens).  Replaces the per-token KVManager::save_page
 * calls (cache/kv_cache.cpp:111-127) of InferenceController::appendKVPage
 * (runtime/inference.cpp:50-54) for a run of tokens.  new_k/new_v:
 * [batch][n_new][num_kv_heads][128] in the pool's dtype (KVX_F16 or
 * KVX_F32), 16-token pages, head_dim 128.  Bit-exact copy.  A negative
 * position, or a page outside the block table or pool, skips those rows
 * and sets bit 1 of *error_flag (may be NULL). */
KVX_API int kvx_append_chunk(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                             const int32_t *positions, int32_t batch, int32_t n_new,
                             const void *new_k, const void *new_v, int32_t *error_flag, void *stream);

/* Bytes of scratch kvx_decode / kvx_append_decode need: split-K partial
 * results plus one arrival counter per (sequence, q-head). */
KVX_API size_t kvx_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t max_pages,
                                          int32_t page_tokens);
/* Zero-fill a decode workspace (cudaMemsetAsync).  Required once before its
 * first use; every decode launch leaves the counters at zero again. */
KVX_API int kvx_decode_workspace_init(void *workspace, size_t workspace_bytes, void *stream);

/* Paged GQA decode attention.  Replaces the naive attention of
 * runtime/gpu/cuda_executor.cu:246-311 and native-engine/cuda/attention.cu:18-157
 * with the semantics of TensorOps::attention (runtime/tensor_ops.cpp:179-219):
 * for sequence s and q-head h (kv-head h / (num_q_heads/num_kv_heads)),
 * out = softmax(q.K^T * sm_scale) V over tokens [0, seq_lens[s]), gathered
 * through the block table.  sm_scale <= 0 means 1/sqrt(head_dim).
 * q/out: [batch][num_q_heads][head_dim] in io_dtype (KVX_F32 or KVX_F16).
 * seq_lens[s] == 0 gives a zero row.  error_flag (device int, may be NULL)
 * gets bit 0 set if a bounded wait for page data expired, bit 1 for a page
 * id outside the pool (that page is skipped) and bit 2 for a context longer
 * than max_pages*page_tokens (clamped).  workspace:
 * kvx_decode_workspace_bytes() bytes of device memory, zero-filled once by
 * kvx_decode_workspace_init; launches that share a workspace must be
 * ordered (same stream), as they share its counters.  After a launch that
 * set bit 0 of error_flag, zero-fill the workspace again before reuse. */
KVX_API int kvx_decode(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                       const int32_t *seq_lens, int32_t batch, int32_t num_q_heads,
                       const void *q, void *out, int32_t io_dtype, float sm_scale,
                       void *workspace, size_t workspace_bytes, int32_t *error_flag,
                       void *stream);

/* Fused append + decode: kvx_append of the token at positions[s] followed by
 * kvx_decode over seq_lens[s] = positions[s] + 1, in one launch.  Replaces
 * the save_page-then-attention sequence of InferenceController::appendKVPage
 * (runtime/inference.cpp:50-54) + TensorOps::attention
 * (runtime/tensor_ops.cpp:179-219).  fp16 / fp32 pools only. */
KVX_API int kvx_append_decode(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                              const int32_t *positions, int32_t batch, const void *new_k,
                              const void *new_v, int32_t num_q_heads, const void *q, void *out,
                              int32_t io_dtype, float sm_scale, void *workspace,
                              size_t workspace_bytes, int32_t *error_flag, void *stream);

/* kvx_append_decode that also tells other streams when it is done: once
 * every CTA of the launch has written its outputs (out, the appended rows,
 * the workspace counters), the last one stores `epoch` to done[1] with
 * release ordering at GPU scope.  done: two device uint32 words, done[0]
 * zero-filled once before first use (the launch counts its CTAs there and
 * leaves it at zero); launches sharing `done` must be ordered on one
 * stream.  A consumer on another stream waits with kvx_stream_wait_geq
 * (done + 1, epoch) instead of an event recorded on this stream: anything
 * enqueued between two dependent decode launches (an event record, a
 * stream wait) ends their overlap.  The all-gather of a KV-head-sharded
 * step waits this way for the last layer of each group (the reference has
 * no multi-GPU path; its attention is TensorOps::attention,
 * runtime/tensor_ops.cpp:179-219, after KVManager::save_page,
 * cache/kv_cache.cpp:111-127). */
KVX_API int kvx_append_decode_signal(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                                     const int32_t *positions, int32_t batch, const void *new_k,
                                     const void *new_v, int32_t num_q_heads, const void *q, void *out,
                                     int32_t io_dtype, float sm_scale, void *workspace,
                                     size_t workspace_bytes, int32_t *error_flag, uint32_t *done,
                                     uint32_t epoch, void *stream);

/* Enqueue on `stream` a wait until the device word *word reaches `value`
 * (compared cyclically: (int32_t)(*word - value) >= 0), as a stream memory
 * operation (cuStreamWaitValue32): no kernel, no host involvement.  Later
 * work on `stream` sees every write released before the word was stored.
 * KVX_EUNSUPPORTED when the driver offers no stream memory operations. */
KVX_API int kvx_stream_wait_geq(const uint32_t *word, uint32_t value, void *stream);

/* kvx_decode without any allocation, for callers that cannot allocate
 * device memory when they decode: a JNI / FFI caller holding only the
 * buffers it was given, an engine whose KV memory is capped at a fixed
 * budget, or code living under another framework's allocator or stream
 * capture.  No counterpart in the reference.  Same arguments and result as
 * kvx_decode minus the workspace: the split-K scratch is a static device
 * array of kvx_decode_noalloc_scratch_bytes() (8 MiB) that each GPU loading
 * this library holds until exit.  The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress), so make it before any
 * stream capture.  The address is kept for the life of the process: after
 * cudaDeviceReset() of a device, do not call this entry point on that
 * device again.  All calls on a device share the array: calls that
 * overlap on the GPU race, so order them on one stream.  A batch whose
 * batch*num_q_heads rows do not fit even at one split per row returns
 * KVX_ETOOBIG.  Calls no cudaMalloc / cudaFree. */
KVX_API size_t kvx_decode_noalloc_scratch_bytes(void);
KVX_API int kvx_decode_noalloc(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                               const int32_t *seq_lens, int32_t batch, int32_t num_q_heads,
                               const void *q, void *out, int32_t io_dtype, float sm_scale,
                               int32_t *error_flag, void *stream);

/* Per-block int8 quantisation.  Replaces KVCompressionEngine::compressToINT8
 * (native-engine/cpp/KVCompressionEngine.cpp:83-113), one reference call per
 * block of block_elems elements: min/max, scale=(max-min)/255 (0 -> 1),
 * zeroPoint=min, code = clamp(round((x-min)/scale), 0, 255) - 128.
 * src: num_blocks*block_elems elements of src_dtype (KVX_F16 widened
 * exactly, or KVX_F32).  stats: [num_blocks][4] = {min, max, scale, zeroPoint}.
 * Bit-exact with the reference. */
KVX_API int kvx_compress_int8(const void *src, int32_t src_dtype, int8_t *codes, float *stats,
                              size_t num_blocks, int32_t block_elems, void *stream);

/* Inverse.  Replaces KVCompressionEngine::decompressINT8
 * (native-engine/cpp/KVCompressionEngine.cpp:115-122): zeroPoint +
 * (code+128)*scale in fp32 (no FMA).  dst_dtype KVX_F32 (bit-exact) or
 * KVX_F16 (that value rounded to nearest). */
KVX_API int kvx_decompress_int8(const int8_t *codes, const float *stats, void *dst,
                                int32_t dst_dtype, size_t num_blocks, int32_t block_elems,
                                void *stream);

/* Per-block 4-bit quantisation.  Replaces KVCompressionEngine::compressToNF4
 * (native-engine/cpp/KVCompressionEngine.cpp:124-163), which despite its
 * name is uniform: min/max, scale=(max-min)/15 (0 -> 1), zeroPoint=min,
 * q = clamp(round((x-min)/scale), 0, 15), two codes per byte with element
 * 2k in the high nibble (a block of odd length leaves the last low nibble
 * 0).  codes: num_blocks * ((block_elems + 1) / 2) bytes; stats as for int8.
 * Bit-exact with the reference. */
KVX_API int kvx_compress_nf4(const void *src, int32_t src_dtype, uint8_t *codes, float *stats,
                             size_t num_blocks, int32_t block_elems, void *stream);

/* Inverse.  Replaces KVCompressionEngine::decompressNF4
 * (native-engine/cpp/KVCompressionEngine.cpp:165-180): zeroPoint + q*scale
 * in fp32 (no FMA).  dst_dtype KVX_F32 (bit-exact) or KVX_F16. */
KVX_API int kvx_decompress_nf4(const uint8_t *codes, const float *stats, void *dst,
                               int32_t dst_dtype, size_t num_blocks, int32_t block_elems,
                               void *stream);

/* The compression engine's own fp32 -> fp16.  Replaces
 * KVCompressionEngine::compressToFP16 (native-engine/cpp/KVCompressionEngine.cpp:36-61):
 * Inf and NaN -> +-Inf, a zero exponent -> +-0, otherwise the exponent is
 * rebiased modulo 32 (it wraps outside [2^-14, 2^16)) and the mantissa
 * truncated.  Bit-exact, including the wrap. */
KVX_API int kvx_fp16_wrap_encode(const float *src, uint16_t *dst, size_t n, void *stream);
/* Inverse.  Replaces KVCompressionEngine::decompressFP16
 * (native-engine/cpp/KVCompressionEngine.cpp:63-80): exponent rebiased
 * modulo 256 with no special cases (+-0 decodes to +-2^-15, Inf to 65536).
 * Bit-exact. */
KVX_API int kvx_fp16_wrap_decode(const uint16_t *src, float *dst, size_t n, void *stream);

/* Truncating fp32 -> fp16 of the disk tier.  Replaces float32_to_float16
 * (compression/kv_compress.cpp:6-25,48-53).  Bit-exact.  Any naturally
 * aligned arrays (4 elements per access when 16 / 8-byte aligned). */
KVX_API int kvx_f32_to_f16_trunc(const float *src, uint16_t *dst, size_t n, void *stream);
/* Inverse, subnormals to zero.  Replaces float16_to_float32
 * (compression/kv_compress.cpp:27-46,55-60).  Bit-exact. */
KVX_API int kvx_f16_trunc_to_f32(const uint16_t *src, float *dst, size_t n, void *stream);

/* Row softmax of a dense [rows][cols] fp32 matrix (device pointers).
 * Replaces the reference's softmax_row_kernel / cuda_softmax
 * (runtime/gpu/cuda_executor.cu:149-184,224-244) with TensorOps::softmax
 * semantics (runtime/tensor_ops.cpp:155-177, sum==0 -> 1e-6). */
KVX_API int kvx_softmax_rows(const float *in, float *out, int64_t rows, int64_t cols, void *stream);

/* Dense attention: out[i] = softmax(Q[i] . K^T * scale) V for seq_q query
 * rows over seq_k keys, fp32 [rows][dim] device arrays, dim <= 1024,
 * scale <= 0 -> 1/sqrt(dim).  Replaces the reference's cuda_attention
 * (runtime/gpu/cuda_executor.cu:246-311) with the semantics of
 * TensorOps::attention (runtime/tensor_ops.cpp:179-219).  dim 128 with all
 * four arrays 16-byte aligned runs on the tensor cores; when it splits the
 * keys over CTAs it takes stream-ordered scratch (at most about
 * 148 x 128 rows x 520 bytes) from a memory pool of the library's own,
 * which keeps its memory between calls, and returns KVX_ENOSPC if that
 * allocation fails. */
KVX_API int kvx_attention_dense(const float *Q, const float *K, const float *V, float *out,
                                int64_t seq_q, int64_t seq_k, int32_t dim, float scale,
                                void *stream);

/* LRU victim.  Replaces LRUEvictionPolicy::selectPageToEvict
 * (native-engine/cpp/AdvancedEvictionPolicy.cpp:9-23) and KVCacheGPU::findLRUPage
 * (native-engine/cpp/KVCacheGPU.cpp:54-66): the index of the smallest stamp,
 * the lowest index on ties, UINT64_MAX stamps never chosen; -1 if none.
 * Writes the index to *victim (device int32).  No workspace. */
KVX_API int kvx_lru_select(const uint64_t *stamps, size_t n, int32_t *victim, void *stream);

/* The reference's EvictionMetrics (native-engine/include/AdvancedEvictionPolicy.h:19-27),
 * same layout (48 bytes on LP64), so a std::vector<EvictionMetrics> can be
 * copied to the device as is. */
typedef struct kvx_evict_metrics {
    uint64_t last_access_token;
    float total_attention;
    float average_attention;
    float access_frequency;
    uint64_t creation_time;
    size_t page_size;
    int32_t page_id;
} kvx_evict_metrics;

enum kvx_evict_policy {  /* EvictionStrategy (AdvancedEvictionPolicy.h:29-34) */
    KVX_EVICT_LRU = 0,
    KVX_EVICT_TOKEN_WEIGHTED = 1,
    KVX_EVICT_ATTENTION_BASED = 2,
    KVX_EVICT_PREDICTIVE = 3
};

/* selectPageToEvict of one policy over n pages (device array), as the
 * reference evaluates it (native-engine/cpp/AdvancedEvictionPolicy.cpp:9-152):
 * scores use currentToken = 0, so token ages wrap modulo 2^64 (kept, not
 * fixed); LRU takes the smallest lastAccessToken below UINT64_MAX, the
 * others the highest score strictly above -1; lowest index on ties.
 * TokenWeighted: 1 - decay^age (reference default decay 0.95).
 * AttentionBased: (1 - averageAttention) * log(age + 1).
 * Predictive: 1000 when predicted[i] < 0 (or predicted == NULL), else
 * 0 - predicted[i]; predicted[i] is PredictiveEvictionPolicy::predictNextAccess
 * of page i (device float array).  Writes the chosen pageId, or -1, to
 * *page_id (device int32). */
KVX_API int kvx_evict_select(int32_t policy, const kvx_evict_metrics *pages, size_t n, float decay,
                             const float *predicted, int32_t *page_id, void *stream);
/* CompositeEvictionManager::selectPageToEvict (:238-263): with one policy
 * that policy's rule, else score = sum over policies (in order) of
 * weights[p] * score_p, highest above -1 wins.  policies / weights: host
 * arrays of num_policies <= 8, weights already normalised as the manager
 * keeps them. */
KVX_API int kvx_evict_select_composite(const int32_t *policies, const float *weights,
                                       int32_t num_policies, const kvx_evict_metrics *pages,
                                       size_t n, float decay, const float *predicted,
                                       int32_t *page_id, void *stream);

/* Decode (as kvx_decode) that also measures the attention each page got:
 * page_mass[batch][max_pages] (device float) receives, per sequence and
 * logical page, the softmax probability mass on the page's tokens averaged
 * over the q-heads (each sequence's masses sum to 1; 0 past the context).
 * This is the per-page attention AttentionBasedEvictionPolicy scores on
 * (native-engine/cpp/AdvancedEvictionPolicy.cpp:95-111, whose
 * setAttentionWeights is a stub there): the decode kernel records each
 * page's softmax sum with its running max (8 bytes per q-head and page)
 * and a small kernel normalises with the final (max, sum).  fp16 and int8
 * pools (tensor-core path); KVX_EUNSUPPORTED otherwise.  Workspace:
 * kvx_decode_attn_workspace_bytes, zero-filled once like the decode's. */
KVX_API size_t kvx_decode_attn_workspace_bytes(int32_t batch, int32_t num_q_heads,
                                               int32_t max_pages, int32_t page_tokens);
KVX_API int kvx_decode_attn(const kvx_paged *kv, const int32_t *block_table, int32_t max_pages,
                            const int32_t *seq_lens, int32_t batch, int32_t num_q_heads,
                            const void *q, void *out, int32_t io_dtype, float sm_scale,
                            void *workspace, size_t workspace_bytes, float *page_mass,
                            int32_t *error_flag, void *stream);
/* AttentionBasedEvictionPolicy::updateMetrics (:88-91) fed with measured
 * attention: for every page the step read (block_table / seq_lens as given
 * to the decode), metrics[physical page]: lastAccessToken = current_token,
 * averageAttention = the page's mass, totalAttention += mass,
 * accessFrequency += 1 (atomic; a page shared by several sequences keeps
 * the last writer's average).  metrics: device array of num_metrics. */
KVX_API int kvx_attn_to_metrics(const float *page_mass, const int32_t *block_table, int32_t max_pages,
                                const int32_t *seq_lens, int32_t batch, kvx_evict_metrics *metrics,
                                int32_t num_metrics, uint64_t current_token, void *stream);

/* Page-frame migration between the device pool and a host frame arena
 * (pinned, mapped with cudaHostAlloc(..., cudaHostAllocMapped) or registered).
 * Replaces KVCacheGPU::transferToHost / transferToGPU
 * (native-engine/cpp/KVCacheGPU.cpp:68-120) and the simulated copies of
 * lw_moveKvToRam / lw_moveKvToGpu (native-engine/llama_wrapper/llama_wrapper.cpp:220-341).
 * Frame i of the transfer moves frame_bytes between
 *   device  dev_base + dev_frames[i]  * frame_bytes
 *   host    host_base + host_frames[i] * frame_bytes
 * direction 0: device -> host (evict), 1: host -> device (fetch).
 * frame_bytes must be a multiple of 16 and both bases 16-byte aligned.
 * dev_frames/host_frames are device-readable int32 arrays; a frame id
 * outside [0, dev_capacity) / [0, host_capacity) skips that frame and sets
 * bit 1 of *error_flag (may be NULL).  `ctas` bounds the SMs the copy
 * occupies (0 = default 16), so it can run on a side stream beside decode. */
KVX_API int kvx_migrate_frames(void *dev_base, int32_t dev_capacity, void *host_base,
                               int32_t host_capacity, const int32_t *dev_frames,
                               const int32_t *host_frames, int32_t num_frames,
                               size_t frame_bytes, int32_t direction, int32_t ctas,
                               int32_t *error_flag, void *stream);

#ifdef __cplusplus
}
#endif
#endif
