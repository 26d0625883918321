/*
 * kvx_gpu_cache.h -- C entry points behind the Java KVCacheGPUManager
 * natives (native-engine/cpp/JNIInterface.cpp:159-224,
 * src/main/java/com/adaptivellm/runtime/services/KVCacheGPUManager.java:87-177),
 * over one process-wide KVCacheGPU (include/KVCacheGPU.h) on the current
 * device.  A JNI binding forwards each native to one call here, one line
 * per native.
 *
 *   nativeTransferToGPU(hostPtr, size, pageId)  kvx_gpu_cache_transfer_to_gpu
 *   nativeTransferFromGPU(handle, hostPtr, size) kvx_gpu_cache_transfer_from_gpu
 *   nativeMarkPageUsed(pageId, token)           kvx_gpu_cache_mark_page_used
 *   nativeGetUsedMemory()                       kvx_gpu_cache_used_memory
 *   nativeEvictLRU()                            kvx_gpu_cache_evict_lru
 *   initializeKVCache() / shutdownKVCache()     kvx_gpu_cache_init / _shutdown
 *
 * Handles are opaque, nonzero, never reused.  Differences from the
 * reference's natives, whose bookkeeping bypasses the cache:
 * transfer_from_gpu releases the page through the cache (the reference frees
 * the memory behind the cache's back, leaving its entry and byte count
 * behind), and fails for a handle whose page was evicted or replaced since;
 * evict_lru evicts the cache's least recently used page (the reference frees
 * whichever allocation its hash map lists first); used_memory is the cache's
 * byte count.
 */
#ifndef KVX_GPU_CACHE_H
#define KVX_GPU_CACHE_H

#include <stdint.h>

#include "kvx.h"

#ifdef __cplusplus
extern "C" {
#endif

/* (Re)create the process-wide cache with a byte budget and slot size; the
 * reference's NativeEngine uses half the device memory and 128 KiB pages
 * (native-engine/cpp/NativeEngine.cpp:93-96), which is what the other calls
 * create on first use when this was not called.  0 or a negative kvx_status. */
KVX_API int kvx_gpu_cache_init(uint64_t gpu_memory_bytes, uint64_t page_size);
/* Free the cache and every page; later calls start a new one. */
KVX_API int kvx_gpu_cache_shutdown(void);

/* Copy a host page to the GPU; a handle, or 0 on failure. */
KVX_API int64_t kvx_gpu_cache_transfer_to_gpu(const void *host_ptr, int64_t size, int32_t page_id);
/* Copy the handle's page back to host_ptr and release it: 1, or 0. */
KVX_API int32_t kvx_gpu_cache_transfer_from_gpu(int64_t handle, void *host_ptr, int64_t size);
KVX_API void kvx_gpu_cache_mark_page_used(int32_t page_id, int64_t token_position);
KVX_API int64_t kvx_gpu_cache_used_memory(void);
/* Evict the least recently used page: 1, or 0 when there is none. */
KVX_API int32_t kvx_gpu_cache_evict_lru(void);

#ifdef __cplusplus
}
#endif

#endif
