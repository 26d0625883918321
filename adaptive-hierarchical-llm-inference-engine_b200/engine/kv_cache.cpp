// kv_cache.cpp -- KVManager with device-resident pages: the reference's LRU
// page store (cache/kv_cache.cpp:8-190) whose in-memory copies live in HBM
// and whose disk tier encodes / decodes on the GPU.
#include "kv_cache.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <stdexcept>

#include "kvx.h"

namespace {

cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("KVManager: ") + what + ": " + cudaGetErrorString(e));
}

void check_kvx(int rc, const char *what) {
    if (rc != KVX_OK) throw std::runtime_error(std::string("KVManager: ") + what + ": " + kvx_status_string(rc));
}

}  // namespace

KVManager::KVManager(size_t capacity, const std::string &pages_dir) : dir_(pages_dir), capacity_(capacity) {
    ensure_dir();
    if (kvx_device_check() != KVX_OK) throw std::runtime_error("KVManager: no sm_100 device");
    cudaStream_t st = nullptr;
    check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "stream");
    stream_ = st;
}

KVManager::~KVManager() {
    std::lock_guard<std::mutex> lk(mu_);
    for (auto &kv : map_) {
        if (kv.second.first.key) cudaFreeAsync(kv.second.first.key, as_stream(stream_));
        if (kv.second.first.value) cudaFreeAsync(kv.second.first.value, as_stream(stream_));
    }
    map_.clear();
    lru_.clear();
    cudaStreamSynchronize(as_stream(stream_));
    cudaStreamDestroy(as_stream(stream_));
}

void KVManager::ensure_dir() { std::filesystem::create_directory(dir_); }

std::string KVManager::page_path(int id) const {
    return (std::filesystem::path(dir_) / ("page_" + std::to_string(id) + ".bin")).string();
}

bool KVManager::pageExists(int id) const { return std::filesystem::exists(page_path(id)); }

// Upload host floats (or take ownership of device floats) as page `id`,
// evicting the least recently used page first when the manager is full.
void KVManager::insert_locked(int id, const float *key, size_t nk, const float *value, size_t nv,
                              bool from_device) {
    cudaStream_t st = as_stream(stream_);
    DevicePage dp;
    dp.nk = nk;
    dp.nv = nv;
    if (from_device) {
        dp.key = const_cast<float *>(key);
        dp.value = const_cast<float *>(value);
    } else {
        if (nk) check(cudaMallocAsync(&dp.key, nk * sizeof(float), st), "alloc");
        if (nv) check(cudaMallocAsync(&dp.value, nv * sizeof(float), st), "alloc");
        if (nk) check(cudaMemcpyAsync(dp.key, key, nk * sizeof(float), cudaMemcpyHostToDevice, st), "copy");
        if (nv) check(cudaMemcpyAsync(dp.value, value, nv * sizeof(float), cudaMemcpyHostToDevice, st), "copy");
    }
    auto it = map_.find(id);
    if (it != map_.end()) {  // update in place, move to front
        if (it->second.first.key) cudaFreeAsync(it->second.first.key, st);
        if (it->second.first.value) cudaFreeAsync(it->second.first.value, st);
        lru_.erase(it->second.second);
        lru_.push_front(id);
        it->second = {dp, lru_.begin()};
        return;
    }
    if (map_.size() >= capacity_ && !lru_.empty()) drop_locked(lru_.back());
    lru_.push_front(id);
    map_.emplace(id, std::make_pair(dp, lru_.begin()));
}

void KVManager::drop_locked(int id) {
    auto it = map_.find(id);
    if (it == map_.end()) return;
    if (it->second.first.key) cudaFreeAsync(it->second.first.key, as_stream(stream_));
    if (it->second.first.value) cudaFreeAsync(it->second.first.value, as_stream(stream_));
    lru_.erase(it->second.second);
    map_.erase(it);
}

KVPage KVManager::to_host_locked(int id) {
    const DevicePage &dp = map_.at(id).first;
    KVPage p;
    p.id = id;
    p.key.resize(dp.nk);
    p.value.resize(dp.nv);
    cudaStream_t st = as_stream(stream_);
    if (dp.nk) check(cudaMemcpyAsync(p.key.data(), dp.key, dp.nk * sizeof(float), cudaMemcpyDeviceToHost, st), "copy");
    if (dp.nv) check(cudaMemcpyAsync(p.value.data(), dp.value, dp.nv * sizeof(float), cudaMemcpyDeviceToHost, st), "copy");
    check(cudaStreamSynchronize(st), "sync");
    return p;
}

// File format of cache/kv_cache.cpp:21-41: u8 flag (1 = fp16), u64 n_key,
// n_key x u16, u64 n_value, n_value x u16; fp16 by the truncating codec,
// computed on the GPU from the page's device copy.
void KVManager::persist_to_disk(const KVPage &p) {
    const std::string path = page_path(p.id);
    std::ofstream out(path, std::ios::binary);
    if (!out) throw std::runtime_error("KVManager: failed to open file for write: " + path);
    cudaStream_t st = as_stream(stream_);
    const size_t n = p.key.size() + p.value.size();
    std::vector<uint16_t> h16(n);
    if (n) {
        float *d32 = nullptr;
        uint16_t *d16 = nullptr;
        check(cudaMallocAsync(&d32, n * sizeof(float), st), "alloc");
        check(cudaMallocAsync(&d16, n * sizeof(uint16_t), st), "alloc");
        if (!p.key.empty())
            check(cudaMemcpyAsync(d32, p.key.data(), p.key.size() * 4, cudaMemcpyHostToDevice, st), "copy");
        if (!p.value.empty())
            check(cudaMemcpyAsync(d32 + p.key.size(), p.value.data(), p.value.size() * 4, cudaMemcpyHostToDevice, st),
                  "copy");
        check_kvx(kvx_f32_to_f16_trunc(d32, d16, n, st), "fp16 encode");
        check(cudaMemcpyAsync(h16.data(), d16, n * 2, cudaMemcpyDeviceToHost, st), "copy");
        cudaFreeAsync(d32, st);
        cudaFreeAsync(d16, st);
        check(cudaStreamSynchronize(st), "sync");
    }
    const uint8_t flag = 1;
    const uint64_t ksz = p.key.size(), vsz = p.value.size();
    out.write(reinterpret_cast<const char *>(&flag), 1);
    out.write(reinterpret_cast<const char *>(&ksz), 8);
    if (ksz) out.write(reinterpret_cast<const char *>(h16.data()), ksz * 2);
    out.write(reinterpret_cast<const char *>(&vsz), 8);
    if (vsz) out.write(reinterpret_cast<const char *>(h16.data() + ksz), vsz * 2);
}

// cache/kv_cache.cpp:43-84: fp16 pages (flag 1) are widened on the GPU into
// the device page; legacy raw-float pages (flag 0: u64 n_key, u64 n_value,
// floats) are uploaded as they are.  The page is returned through the map.
KVPage KVManager::load_from_disk(int id) {
    const std::string path = page_path(id);
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("KVManager: failed to open page file: " + path);
    uint8_t flag = 0;
    in.read(reinterpret_cast<char *>(&flag), 1);
    KVPage p;
    p.id = id;
    if (flag == 1) {
        uint64_t ksz = 0, vsz = 0;
        std::vector<uint16_t> h16;
        in.read(reinterpret_cast<char *>(&ksz), 8);
        h16.resize(ksz);
        if (ksz) in.read(reinterpret_cast<char *>(h16.data()), ksz * 2);
        in.read(reinterpret_cast<char *>(&vsz), 8);
        h16.resize(ksz + vsz);
        if (vsz) in.read(reinterpret_cast<char *>(h16.data() + ksz), vsz * 2);
        cudaStream_t st = as_stream(stream_);
        const size_t n = ksz + vsz;
        float *dk = nullptr, *dv = nullptr;
        if (n) {
            uint16_t *d16 = nullptr;
            check(cudaMallocAsync(&d16, n * 2, st), "alloc");
            check(cudaMemcpyAsync(d16, h16.data(), n * 2, cudaMemcpyHostToDevice, st), "copy");
            if (ksz) check(cudaMallocAsync(&dk, ksz * 4, st), "alloc");
            if (vsz) check(cudaMallocAsync(&dv, vsz * 4, st), "alloc");
            if (ksz) check_kvx(kvx_f16_trunc_to_f32(d16, dk, ksz, st), "fp16 decode");
            if (vsz) check_kvx(kvx_f16_trunc_to_f32(d16 + ksz, dv, vsz, st), "fp16 decode");
            cudaFreeAsync(d16, st);
        }
        insert_locked(id, dk, ksz, dv, vsz, /*from_device=*/true);
        return to_host_locked(id);
    }
    uint64_t ksz = 0, vsz = 0;
    in.read(reinterpret_cast<char *>(&ksz), 8);
    in.read(reinterpret_cast<char *>(&vsz), 8);
    p.key.resize(ksz);
    p.value.resize(vsz);
    if (ksz) in.read(reinterpret_cast<char *>(p.key.data()), ksz * 4);
    if (vsz) in.read(reinterpret_cast<char *>(p.value.data()), vsz * 4);
    insert_locked(id, p.key.data(), ksz, p.value.data(), vsz, false);
    return p;
}

KVPage KVManager::load_page(int id) {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = map_.find(id);
    if (it != map_.end()) {  // hit: move to front
        lru_.erase(it->second.second);
        lru_.push_front(id);
        it->second.second = lru_.begin();
        return to_host_locked(id);
    }
    return load_from_disk(id);  // inserts as most recent, evicting the LRU page when full
}

void KVManager::save_page(const KVPage &page) {
    std::lock_guard<std::mutex> lk(mu_);
    persist_to_disk(page);
    insert_locked(page.id, page.key.data(), page.key.size(), page.value.data(), page.value.size(), false);
}

void KVManager::evict_page(int id) {
    std::lock_guard<std::mutex> lk(mu_);
    drop_locked(id);
}

bool KVManager::contains(int id) {
    std::lock_guard<std::mutex> lk(mu_);
    return map_.find(id) != map_.end();
}

size_t KVManager::size() {
    std::lock_guard<std::mutex> lk(mu_);
    return map_.size();
}

size_t KVManager::capacity() { return capacity_; }

const float *KVManager::device_key(int id, size_t *count) {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = map_.find(id);
    if (it == map_.end()) return nullptr;
    if (count) *count = it->second.first.nk;
    return it->second.first.key;
}

const float *KVManager::device_value(int id, size_t *count) {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = map_.find(id);
    if (it == map_.end()) return nullptr;
    if (count) *count = it->second.first.nv;
    return it->second.first.value;
}
