// kv_cache_gpu.cpp -- the reference's KVCacheGPU (native-engine/cpp/
// KVCacheGPU.cpp:1-163) on a device slot pool, and the C entry points of the
// KVCacheGPUManager natives (native-engine/cpp/JNIInterface.cpp:159-224).
//
// Decisions and byte accounting follow the reference line for line
// (allocateGPUPage's budget test, transferToGPU's single evict-and-retry,
// findLRUPage's strict minimum, the replaced-page bytes that stay counted);
// only where the bytes live differs: slots of pageSize bytes carved from
// chunks of one cudaMalloc each, larger pages allocated on their own, copies
// on the cache's own stream.
#include "KVCacheGPU.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <limits>
#include <unordered_map>
#include <unordered_set>

#include "kvx.h"
#include "kvx_gpu_cache.h"

namespace {
constexpr size_t kChunkBytes = size_t(256) << 20;  // pool growth step
}

struct KVCacheGPU::Pool {
    size_t slot = 0;                        // bytes per slot (the constructor's pageSize)
    std::vector<void *> chunks;             // cudaMalloc'd, each a run of slots
    std::vector<void *> free_slots;
    std::unordered_set<void *> big;         // pages above the slot size
    std::vector<std::pair<void *, size_t>> replaced;  // entries overwritten by a re-sent page id
    cudaStream_t stream = nullptr;

    ~Pool() {
        for (void *p : big) cudaFree(p);
        for (void *c : chunks) cudaFree(c);
        if (stream) cudaStreamDestroy(stream);
    }
    bool ensure_stream() {
        return stream || cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) == cudaSuccess;
    }
    // One more chunk of slots; smaller chunks when the device is short.
    bool grow(size_t max_slots) {
        size_t n = std::max<size_t>(1, std::min(max_slots, kChunkBytes / std::max<size_t>(slot, 1)));
        for (; n >= 1; n /= 2) {
            void *c = nullptr;
            if (cudaMalloc(&c, n * slot) == cudaSuccess) {
                chunks.push_back(c);
                for (size_t i = n; i-- > 0;) free_slots.push_back(static_cast<char *>(c) + i * slot);
                return true;
            }
            cudaGetLastError();
            if (n == 1) break;
        }
        return false;
    }
};

KVCacheGPU::KVCacheGPU(size_t gpuMemoryBytes, size_t pageSize)
    : totalGPUMemory(gpuMemoryBytes), usedGPUMemory(0), maxPages(pageSize ? gpuMemoryBytes / pageSize : 0),
      pool_(new Pool) {
    pool_->slot = pageSize;
}

KVCacheGPU::~KVCacheGPU() { clear(); }

// KVCacheGPU.cpp:21-40: refuse beyond the budget, else allocate and count.
void *KVCacheGPU::allocateGPUPage(size_t size) {
    if (usedGPUMemory + size > totalGPUMemory) return nullptr;
    if (size == 0) return nullptr;  // cudaMalloc of 0 bytes hands back a null pointer
    void *ptr = nullptr;
    if (size <= pool_->slot) {
        if (pool_->free_slots.empty() && !pool_->grow(maxPages ? maxPages : 1)) return nullptr;
        ptr = pool_->free_slots.back();
        pool_->free_slots.pop_back();
    } else {
        if (cudaMalloc(&ptr, size) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        pool_->big.insert(ptr);
    }
    usedGPUMemory += size;
    return ptr;
}

// KVCacheGPU.cpp:42-52
void KVCacheGPU::freeGPUPage(void *ptr, size_t size) {
    if (!ptr) return;
    if (size <= pool_->slot) {
        pool_->free_slots.push_back(ptr);
    } else {
        pool_->big.erase(ptr);
        cudaFree(ptr);
    }
    usedGPUMemory -= size;
}

// KVCacheGPU.cpp:54-66: minimum lastUsedToken, the first (lowest id) on ties.
int KVCacheGPU::findLRUPage() {
    int lru = -1;
    uint64_t min_used = std::numeric_limits<uint64_t>::max();
    for (size_t i = 0; i < pages.size(); i++)
        if (pages[i] && pages[i]->lastUsedToken < min_used) {
            min_used = pages[i]->lastUsedToken;
            lru = (int)i;
        }
    return lru;
}

// KVCacheGPU.cpp:68-79: allocate, else evict one page and retry once.
void *KVCacheGPU::placeLocked(size_t size, int pageId) {
    if (pageId < 0) return nullptr;
    void *gpu = allocateGPUPage(size);
    if (!gpu && evictLRUPageLocked()) gpu = allocateGPUPage(size);
    return gpu;
}

// KVCacheGPU.cpp:89-105: a new entry with lastUsedToken 0 replaces any old
// one, whose memory stays allocated and counted.
void KVCacheGPU::installLocked(int pageId, void *gpu, size_t size) {
    auto page = std::make_unique<KVCacheGPUPage>();
    page->gpuMemPtr = gpu;
    page->pageSize = size;
    page->pageId = pageId;
    page->isValid = true;
    page->lastUsedToken = 0;
    if (pageId >= (int)pages.size()) pages.resize(pageId + 1);
    if (pages[pageId] && pages[pageId]->gpuMemPtr)
        pool_->replaced.emplace_back(pages[pageId]->gpuMemPtr, pages[pageId]->pageSize);
    pages[pageId] = std::move(page);
}

void *KVCacheGPU::transferToGPU(const void *hostPtr, size_t size, int pageId) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!pool_->ensure_stream()) return nullptr;
    void *gpu = placeLocked(size, pageId);
    if (!gpu) return nullptr;
    if (cudaMemcpyAsync(gpu, hostPtr, size, cudaMemcpyHostToDevice, pool_->stream) != cudaSuccess ||
        cudaStreamSynchronize(pool_->stream) != cudaSuccess) {
        cudaGetLastError();  // KVCacheGPU.cpp:82-86: free it, no entry
        freeGPUPage(gpu, size);
        return nullptr;
    }
    installLocked(pageId, gpu, size);
    return gpu;
}

int KVCacheGPU::transferToGPUBatch(const void *const *hostPtrs, const size_t *sizes, const int *pageIds, int n,
                                   void **gpuPtrs) {
    std::lock_guard<std::mutex> lk(mu_);
    if (n <= 0 || !hostPtrs || !sizes || !pageIds || !gpuPtrs || !pool_->ensure_stream()) return 0;
    int ok = 0;
    for (int i = 0; i < n; ++i) {  // each page is in place before the next one's decision
        gpuPtrs[i] = placeLocked(sizes[i], pageIds[i]);
        if (!gpuPtrs[i]) continue;
        if (cudaMemcpyAsync(gpuPtrs[i], hostPtrs[i], sizes[i], cudaMemcpyHostToDevice, pool_->stream) != cudaSuccess) {
            cudaGetLastError();
            freeGPUPage(gpuPtrs[i], sizes[i]);
            gpuPtrs[i] = nullptr;
            continue;
        }
        installLocked(pageIds[i], gpuPtrs[i], sizes[i]);
        ++ok;
    }
    if (cudaStreamSynchronize(pool_->stream) != cudaSuccess) {  // the copies' data cannot be trusted
        cudaGetLastError();
        return 0;
    }
    return ok;
}

// KVCacheGPU.cpp:111-120
bool KVCacheGPU::transferToHost(void *gpuPtr, void *hostPtr, size_t size) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!pool_->ensure_stream()) return false;
    if (cudaMemcpyAsync(hostPtr, gpuPtr, size, cudaMemcpyDeviceToHost, pool_->stream) != cudaSuccess ||
        cudaStreamSynchronize(pool_->stream) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return true;
}

// KVCacheGPU.cpp:122-127
KVCacheGPUPage *KVCacheGPU::getPage(int pageId) {
    std::lock_guard<std::mutex> lk(mu_);
    if (pageId < 0 || pageId >= (int)pages.size()) return nullptr;
    return pages[pageId].get();
}

// KVCacheGPU.cpp:129-134
void KVCacheGPU::markPageUsed(int pageId, uint64_t token) {
    std::lock_guard<std::mutex> lk(mu_);
    if (pageId >= 0 && pageId < (int)pages.size() && pages[pageId]) pages[pageId]->lastUsedToken = token;
}

// KVCacheGPU.cpp:136-152
bool KVCacheGPU::evictLRUPageLocked() {
    const int lru = findLRUPage();
    if (lru < 0) return false;
    KVCacheGPUPage *page = pages[lru].get();
    if (!page || !page->gpuMemPtr) return false;
    freeGPUPage(page->gpuMemPtr, page->pageSize);
    pages[lru] = nullptr;
    return true;
}

bool KVCacheGPU::evictLRUPage() {
    std::lock_guard<std::mutex> lk(mu_);
    return evictLRUPageLocked();
}

bool KVCacheGPU::releasePage(int pageId) {
    std::lock_guard<std::mutex> lk(mu_);
    if (pageId < 0 || pageId >= (int)pages.size() || !pages[pageId] || !pages[pageId]->gpuMemPtr) return false;
    freeGPUPage(pages[pageId]->gpuMemPtr, pages[pageId]->pageSize);
    pages[pageId] = nullptr;
    return true;
}

// KVCacheGPU.cpp:154-163; replaced entries' memory goes back too (the byte
// count, as in the reference, restarts at 0).
void KVCacheGPU::clearLocked() {
    for (auto &page : pages)
        if (page && page->gpuMemPtr) freeGPUPage(page->gpuMemPtr, page->pageSize);
    for (auto &r : pool_->replaced) freeGPUPage(r.first, r.second);
    pool_->replaced.clear();
    pages.clear();
    usedGPUMemory = 0;
}

void KVCacheGPU::clear() {
    std::lock_guard<std::mutex> lk(mu_);
    clearLocked();
}

// ---------------------------------------------------------------------------
// The KVCacheGPUManager natives over one process-wide cache.

namespace {
struct GpuCacheState {
    std::mutex mu;
    std::unique_ptr<KVCacheGPU> cache;
    struct Entry {
        int page;
        void *ptr;
        int64_t size;
    };
    std::unordered_map<int64_t, Entry> handles;
    int64_t next_handle = 1;
};
GpuCacheState &state() {
    static GpuCacheState *s = new GpuCacheState();  // lives until exit
    return *s;
}
// NativeEngine.cpp:93-96: half the device memory, 128 KiB pages
bool ensure_cache(GpuCacheState &s) {
    if (s.cache) return true;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    s.cache.reset(new KVCacheGPU(total_b / 2, 128 * 1024));
    return true;
}
}  // namespace

extern "C" KVX_API int kvx_gpu_cache_init(uint64_t gpu_memory_bytes, uint64_t page_size) {
    if (page_size == 0) return KVX_EINVAL;
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    s.handles.clear();
    s.cache.reset(new KVCacheGPU((size_t)gpu_memory_bytes, (size_t)page_size));
    return KVX_OK;
}

extern "C" KVX_API int kvx_gpu_cache_shutdown(void) {
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    s.handles.clear();
    s.cache.reset();
    return KVX_OK;
}

extern "C" KVX_API int64_t kvx_gpu_cache_transfer_to_gpu(const void *host_ptr, int64_t size, int32_t page_id) {
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    if (!host_ptr || size < 0 || !ensure_cache(s)) return 0;
    void *p = s.cache->transferToGPU(host_ptr, (size_t)size, page_id);
    if (!p) return 0;
    const int64_t h = s.next_handle++;
    s.handles[h] = {page_id, p, size};
    return h;
}

extern "C" KVX_API int32_t kvx_gpu_cache_transfer_from_gpu(int64_t handle, void *host_ptr, int64_t size) {
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    auto it = s.handles.find(handle);
    if (it == s.handles.end() || !s.cache || !host_ptr || size < 0 || size > it->second.size) return 0;
    const GpuCacheState::Entry e = it->second;
    s.handles.erase(it);
    KVCacheGPUPage *page = s.cache->getPage(e.page);
    if (!page || page->gpuMemPtr != e.ptr) return 0;  // evicted or replaced since
    if (!s.cache->transferToHost(e.ptr, host_ptr, (size_t)size)) return 0;
    return s.cache->releasePage(e.page) ? 1 : 0;
}

extern "C" KVX_API void kvx_gpu_cache_mark_page_used(int32_t page_id, int64_t token_position) {
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    if (s.cache) s.cache->markPageUsed(page_id, (uint64_t)token_position);
}

extern "C" KVX_API int64_t kvx_gpu_cache_used_memory(void) {
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    return s.cache ? (int64_t)s.cache->getUsedMemory() : 0;
}

extern "C" KVX_API int32_t kvx_gpu_cache_evict_lru(void) {
    GpuCacheState &s = state();
    std::lock_guard<std::mutex> lk(s.mu);
    return s.cache && s.cache->evictLRUPage() ? 1 : 0;
}
