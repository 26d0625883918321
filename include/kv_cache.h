/* kv_cache.h -- drop-in for the reference's cache/kv_cache.h: the same
 * KVPage / KVManager interface and LRU semantics (cache/kv_cache.cpp:91-190),
 * with every in-memory page held in device memory.
 *
 *  - save_page(p): persist p to <dir>/page_<id>.bin in the reference's
 *    format (u8 flag=1, u64 n_key, n_key x fp16, u64 n_value, n_value x
 *    fp16, truncating fp16 of kv_compress.h; cache/kv_cache.cpp:21-41), then
 *    insert / update it as most recently used, evicting the least recently
 *    used page when the manager holds `capacity` pages.
 *  - load_page(id): a resident page moves to the front and is returned; a
 *    missing one is read from its file (fp16 widened on the GPU,
 *    cache/kv_cache.cpp:43-84), evicting the least recently used page first
 *    when full.  Throws std::runtime_error if the file cannot be opened.
 *  - evict_page / contains / size / capacity / pageExists as the reference.
 * The reference joins "<dir>" and "page_<id>.bin" with a backslash, which
 * on Linux names a file outside <dir>; this manager writes inside <dir>.
 * Thread-safe (one mutex, as the reference). */
#pragma once

#include <cstddef>
#include <list>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "kvx_cxx.h"

struct KVPage {
    int id;
    std::vector<float> key;    // the page's keys, any layout the caller chose
    std::vector<float> value;  // the page's values
};

class KVX_CXX_API KVManager {
public:
    explicit KVManager(size_t capacity = 4, const std::string &pages_dir = "pages");
    ~KVManager();

    KVPage load_page(int id);            // resident copy, or read back from its file
    void save_page(const KVPage &page);  // write the file, keep the page resident
    void evict_page(int id);             // drop the resident copy, keep the file

    bool contains(int id);
    bool pageExists(int id) const;
    size_t size();
    size_t capacity();

    // Additive: device copy of a resident page (nullptr if not resident);
    // valid until the page is evicted or saved again.
    const float *device_key(int id, size_t *count);
    const float *device_value(int id, size_t *count);

private:
    struct DevicePage {
        float *key = nullptr;
        size_t nk = 0;
        float *value = nullptr;
        size_t nv = 0;
    };
    void ensure_dir();
    void persist_to_disk(const KVPage &p);
    KVPage load_from_disk(int id);
    void insert_locked(int id, const float *key, size_t nk, const float *value, size_t nv,
                       bool from_device);
    void drop_locked(int id);
    KVPage to_host_locked(int id);
    std::string page_path(int id) const;

    std::string dir_;
    size_t capacity_;
    std::mutex mu_;
    std::list<int> lru_;  // front = most recently used
    std::unordered_map<int, std::pair<DevicePage, std::list<int>::iterator>> map_;
    void *stream_ = nullptr;
};
