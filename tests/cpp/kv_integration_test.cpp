// KV part of the reference's tests/kv_integration_test.cpp: appending four
// pages at capacity 2 keeps two in memory; an evicted page reloads from disk.
#include <cstdio>
#include <filesystem>

#include "kv_cache.h"

int main(int argc, char **argv) {
    const std::string dir = argc > 1 ? argv[1] : "pages";
    std::filesystem::create_directory(dir);
    try {
        KVManager kv(2, dir);
        for (int i = 0; i < 4; ++i) {
            KVPage p;
            p.id = i;
            p.key = {(float)i + 0.1f};
            p.value = {(float)i + 0.2f};
            kv.save_page(p);
            printf("Appended KV page %d\n", i);
        }
        printf("KV in-memory size: %zu (capacity %zu)\n", kv.size(), kv.capacity());
        if (kv.size() != 2) return 2;
        KVPage p0 = kv.load_page(0);
        printf("Loaded evicted page 0 key[0]=%g\n", p0.key[0]);
        if (!(p0.key[0] > 0.0999f && p0.key[0] < 0.1f)) return 3;
        if (kv.contains(2) || !kv.contains(3)) return 4;  // 2 was the LRU page
    } catch (const std::exception &e) {
        printf("Test failed: %s\n", e.what());
        return 1;
    }
    return 0;
}
