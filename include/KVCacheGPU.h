/*
 * KVCacheGPU -- drop-in for the reference's native-engine/include/KVCacheGPU.h
 * (native-engine/cpp/KVCacheGPU.cpp:1-163): KV pages moved between host
 * memory and the GPU under a byte budget, least recently used page evicted
 * when the budget is full.
 *
 * Same class, struct and public methods, same decisions: an allocation fails
 * when used + size > budget; transferToGPU then evicts ONE page (minimum
 * lastUsedToken, strict comparison so the lowest page id wins ties) and
 * retries once; a new page starts with lastUsedToken = 0; re-sending a page
 * id replaces its entry without releasing the old copy, whose bytes stay
 * counted in getUsedMemory() until clear() -- exactly the reference's
 * accounting.
 *
 * On the GPU side it differs: pages of up to pageSize bytes are slots of a
 * pool that grows in large chunks (one cudaMalloc per chunk instead of one
 * per page, and no cudaFree -- a device-wide synchronisation -- per
 * eviction); larger pages get their own allocation.  Copies run as
 * cudaMemcpyAsync on the cache's own stream and each call returns when its
 * copy is complete, as the reference's cudaMemcpy did.  transferToGPUBatch
 * (additive) queues many pages' copies and waits once.
 *
 * Deviations: a negative page id is refused (nullptr) instead of indexing
 * before the page table; calls are serialised by an internal mutex.
 */
#ifndef KV_CACHE_GPU_H
#define KV_CACHE_GPU_H

#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
#include <vector>

#include "kvx_cxx.h"

struct KVCacheGPUPage {
    void *gpuMemPtr;         // GPU memory pointer
    size_t pageSize;         // Size in bytes
    int pageId;              // Logical page ID
    bool isValid;            // Whether data is current
    uint64_t lastUsedToken;  // Track for LRU
};

class KVX_CXX_API KVCacheGPU {
private:
    std::vector<std::unique_ptr<KVCacheGPUPage>> pages;
    size_t totalGPUMemory;
    size_t usedGPUMemory;
    size_t maxPages;

    struct Pool;                  // device slot pool (engine/kv_cache_gpu.cpp)
    std::unique_ptr<Pool> pool_;
    mutable std::mutex mu_;

    void *allocateGPUPage(size_t size);
    void freeGPUPage(void *ptr, size_t size);
    int findLRUPage();
    bool evictLRUPageLocked();
    void *placeLocked(size_t size, int pageId);
    void installLocked(int pageId, void *gpu, size_t size);
    void clearLocked();

public:
    KVCacheGPU(size_t gpuMemoryBytes, size_t pageSize);
    ~KVCacheGPU();
    KVCacheGPU(const KVCacheGPU &) = delete;
    KVCacheGPU &operator=(const KVCacheGPU &) = delete;

    /* Copy size bytes from hostPtr into a GPU page for pageId (evicting the
     * LRU page once if the budget is full); the device pointer, or nullptr. */
    void *transferToGPU(const void *hostPtr, size_t size, int pageId);

    /* Copy size bytes of GPU memory gpuPtr to hostPtr. */
    bool transferToHost(void *gpuPtr, void *hostPtr, size_t size);

    /* Additive: n pages at once, same decisions as n transferToGPU calls in
     * order; gpuPtrs[i] receives each page's pointer (nullptr on failure).
     * Returns how many succeeded. */
    int transferToGPUBatch(const void *const *hostPtrs, const size_t *sizes, const int *pageIds, int n,
                           void **gpuPtrs);

    KVCacheGPUPage *getPage(int pageId);
    void markPageUsed(int pageId, uint64_t token);
    bool evictLRUPage();
    /* Additive: free pageId's GPU copy (as evictLRUPage does for the LRU
     * page); false when it has none. */
    bool releasePage(int pageId);
    size_t getUsedMemory() const { return usedGPUMemory; }
    size_t getAvailableMemory() const { return totalGPUMemory - usedGPUMemory; }
    void clear();
};

#endif
