/*
 * adaptive_engine.h -- the C ABI the reference's Java/JNI stack binds
 * (dlopen of libadaptive_engine.so, then adaptive_engine_get_api()), backed
 * by the B200 KV-cache engine.
 *
 * NativeEngineApi keeps the exact layout and calling convention of
 * native-engine/llama_wrapper/llama_wrapper.cpp:26-40 (duplicated in
 * src/main/cpp/adaptive_scheduler.cpp:106-120 and
 * native-engine/shim/adaptive_engine_shim.cpp:13-27): 13 function pointers
 * in this order.  As in the reference, a "kvPageId" is a layer index.  The
 * KV operations do real work here:
 *   moveKvToRam(l)  copy layer l's KV pool to pinned host memory, release
 *                   its device slab                      (llama_wrapper.cpp:220-280)
 *   moveKvToGpu(l)  bring layer l back into a device slab (from RAM, the
 *                   int8 form or the file tier), evicting the least recently
 *                   used resident layer when no slab is free (llama_wrapper.cpp:281-341,
 *                   eviction as native-engine/cpp/KVCacheGPU.cpp:68-109)
 *   compressKv(l)   int8-quantise layer l per (page, K|V, head) block with
 *                   the reference's KVCompressionEngine scheme, release the
 *                   fp16 slab                            (llama_wrapper.cpp:342-406)
 *   offloadKv(l)    write layer l to the file tier, release device and host
 *                   memory                               (llama_wrapper.cpp:407-433)
 * Return convention (llama_wrapper.cpp:187-433): the four KV operations
 * return the milliseconds spent, rounded up and at least 1 on success (also
 * when the layer already was in the requested tier, as the reference's
 * always report their latency); prefetchLayer / evictLayer return 0 when
 * the layer already was cached / evicted (llama_wrapper.cpp:176,192); -1
 * means an invalid id, a stopped engine or an allocation failure, -2 that a
 * pinned layer would have to leave the device.
 */
#ifndef ADAPTIVE_ENGINE_H
#define ADAPTIVE_ENGINE_H

#include <stdint.h>

#include "kvx.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define ADAPTIVE_ENGINE_EXPORT __declspec(dllexport)
#else
#define ADAPTIVE_ENGINE_EXPORT __attribute__((visibility("default")))
#endif

typedef struct NativeEngineApi {
    void (*start)();
    void (*stop)();
    long (*prefetchLayer)(int layerId);
    long (*evictLayer)(int layerId);
    long (*keepLayer)(int layerId);
    long (*moveKvToRam)(long kvPageId);
    long (*moveKvToGpu)(long kvPageId);
    long (*compressKv)(long kvPageId);
    long (*offloadKv)(long kvPageId);
    int (*getCurrentLayer)();
    long (*getGpuMemory)();
    int (*getKvPages)();
    int (*getCachedLayers)();
} NativeEngineApi;

/* native-engine/llama_wrapper/llama_wrapper.cpp:742-744 */
ADAPTIVE_ENGINE_EXPORT NativeEngineApi *adaptive_engine_get_api(void);
/* native-engine/llama_wrapper/llama_wrapper.cpp:733-740: drop one pin. */
ADAPTIVE_ENGINE_EXPORT void adaptive_engine_test_release_layer(int layerId);

/* ---- additive engine interface (the reference has no device engine) ---- */

/* Geometry and budgets.  Defaults: Llama-3.2-3B KV (28 layers, 8 KV heads,
 * 24 q-heads, head_dim 128), 16-token pages, 32 sequences, 256 pages per
 * layer, every layer given a device slab, offload files under /tmp.
 * Environment overrides read by start(): ADAPTIVELLM_KV_LAYERS,
 * ADAPTIVELLM_KV_PAGES, ADAPTIVELLM_KV_BATCH, ADAPTIVELLM_KV_GPU_LAYERS,
 * ADAPTIVELLM_KV_OFFLOAD_DIR, ADAPTIVELLM_DEVICE. */
typedef struct adaptive_engine_config {
    int32_t layers;
    int32_t kv_heads;
    int32_t q_heads;
    int32_t head_dim;         /* 128 */
    int32_t page_tokens;      /* 16 */
    int32_t max_batch;        /* sequence slots */
    int32_t pages_per_layer;  /* physical pages of one layer's pool */
    int32_t gpu_layer_slots;  /* device slabs (< layers: layers compete, LRU) */
    int32_t device;
    char offload_dir[256];
    /* Slabs made once by start(), so that no move allocates: pinned host
     * slabs for layers in RAM (at least layers - gpu_layer_slots) and
     * device int8 slabs (codes + QuantizationStats) for compressed layers.
     * Defaults: one of each per layer.  Environment overrides:
     * ADAPTIVELLM_KV_RAM_LAYERS, ADAPTIVELLM_KV_INT8_LAYERS. */
    int32_t ram_layer_slots;
    int32_t int8_layer_slots;
} adaptive_engine_config;

/* Fill *cfg with the defaults (environment applied). */
ADAPTIVE_ENGINE_EXPORT void adaptive_engine_default_config(adaptive_engine_config *cfg);
/* Set the geometry used by the next start().  KVX_EBUSY while started. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_configure(const adaptive_engine_config *cfg);
/* Layer l's device pool as a kvx_paged view (KVX_EINVAL if the layer has
 * no fp16 device slab right now).  The view stays valid until the layer
 * moves. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_layer_view(int layer, kvx_paged *view);
/* Start `batch` sequences with context lengths lens[0..batch) (host array):
 * pages for the contexts plus `reserve_tokens` future tokens are taken from
 * the pool's free list -- in order, or in a seeded random order when
 * seed != 0 (fragmented page tables).  Page contents are left as they are
 * (the caller fills them, e.g. through adaptive_engine_layer_view). */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_set_sequences(int32_t batch, const int32_t *lens,
                                                         int32_t reserve_tokens, uint64_t seed);
/* One decode step through host buffers for every layer: copy q
 * [layers][batch][q_heads][head_dim], new K and V [layers][batch][kv_heads]
 * [head_dim] (fp16 bits) to the device, append the token and run paged GQA
 * decode per layer, copy the attention output [layers][batch][q_heads]
 * [head_dim] back (skipped when out is NULL, e.g. on all but one rank of a
 * multi-GPU job).  Copies overlap the layers' kernels (side stream, one
 * event per layer).  Returns a kvx_status. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_decode_step(const uint16_t *q, const uint16_t *k,
                                                       const uint16_t *v, uint16_t *out);
/* Copy layer l's whole fp16 pool (slab_bytes = pages_per_layer * 2 *
 * kv_heads * 16 * 128 * 2 bytes) from `src` / to `dst`, host or device
 * memory (cudaMemcpyDefault); the layer is brought to the GPU first.  For
 * restoring / checkpointing a layer's KV.  Return a kvx_status. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_load_layer(int layer, const void *src);
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_read_layer(int layer, void *dst);
/* The block table of the current sequences: returns max_pages (the row
 * length) and, when dst != NULL, copies batch * max_pages int32 physical
 * page ids (-1 = unassigned). */
ADAPTIVE_ENGINE_EXPORT int32_t adaptive_engine_block_table(int32_t *dst);
/* Multi-GPU: one process per GPU, each engine holding its KV-head shard
 * (kv_heads / q_heads of the config are the local counts).  Rank 0 makes a
 * 128-byte NCCL unique id, every rank passes it to set_comm after start();
 * from then on adaptive_engine_decode_step all-gathers each layer's
 * attention output over NCCL (NVLink) and `out` receives
 * [layers][world][batch][q_heads][head_dim].  NCCL is loaded at run time
 * (dlopen of libnccl.so.2, binding to the copy the process already has).
 * Return kvx_status (KVX_EUNSUPPORTED if NCCL cannot be loaded). */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_nccl_unique_id(void *id128);
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_set_comm(int rank, int world, const void *id128);
/* Read-back of a multi-GPU decode step.  share = 0 (the default): `out`
 * receives every layer's gathered rows on each rank that passes it.
 * share = 1: rank r copies back only the layers l with l % world == r into
 * their place in `out`, so the ranks together read the step's result once
 * and the copies spread over every GPU's host link instead of one.  No
 * effect without a communicator.  Returns a kvx_status. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_set_readback_share(int share);
/* 1 while a decode step's device work is still running: the step has
 * queued its kernels and copies and waits for them with the engine lock
 * released, so NativeEngineApi moves of layers proceed meanwhile (each
 * waits only for its own layer's last kernel).  0 otherwise.  With pageable
 * (not pinned) host buffers the step's copies hold the calling thread, and
 * so the lock, until its kernels are done: pass pinned buffers to let moves
 * run beside a step. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_step_in_flight(void);
/* Current context length of sequence s (-1 if none). */
ADAPTIVE_ENGINE_EXPORT int32_t adaptive_engine_seq_len(int32_t s);
/* Tier of layer l: 0 GPU, 1 RAM, 2 COMPRESSED (int8 on device),
 * 3 OFFLOADED (file), 4 COMPRESSED_NF4 (4-bit codes on device, the age
 * policy's heavy compression), -1 invalid. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_layer_tier(int layer);
/* The age-based compression policy of the reference's Java
 * KVCompressionEngine (src/main/java/com/adaptivellm/kv/
 * KVCompressionEngine.java:62-98), over the layers: age = now_ms - the
 * layer's last access (its last decode, or a load); age >=
 * compressed_threshold_ms -> COMPRESSED, else age >= int8_threshold_ms ->
 * INT8; only GPU-resident, unpinned layers change.  INT8 is the int8 tier of
 * compressKv (half of fp16), COMPRESSED the NF4 tier (a quarter), the ratios
 * of the reference's estimateSize.  decisions: NULL or int32[layers],
 * receiving 0 (none), 1 (INT8) or 2 (COMPRESSED) per layer.  apply = 0
 * decides only.  now_ms < 0: the engine clock (ms since start()).
 * Thresholds <= 0 are invalid, as in the reference's constructor.  Returns
 * the number of layers compressed, or a negative kvx_status. */
ADAPTIVE_ENGINE_EXPORT int adaptive_engine_compress_aged(int64_t int8_threshold_ms, int64_t compressed_threshold_ms,
                                                        int64_t now_ms, int32_t apply, int32_t *decisions);
/* Layer l's last access on the engine clock (ms since start()), -1 if
 * invalid. */
ADAPTIVE_ENGINE_EXPORT int64_t adaptive_engine_layer_last_access_ms(int layer);
/* Bytes of device memory the engine holds. */
ADAPTIVE_ENGINE_EXPORT long long adaptive_engine_device_bytes(void);

#ifdef __cplusplus
}
#endif
#endif
