// KVManager LRU at capacity 2 with a disk round trip (the reference's
// tests/kv_test.cpp): save pages 0,1,2; a new manager loads 0,1,2 and page 0
// must be evicted.  Prints key[0] of each page after the fp16 disk tier.
#include <cstdio>
#include <filesystem>

#include "kv_cache.h"

int main(int argc, char **argv) {
    const std::string dir = argc > 1 ? argv[1] : "pages";
    std::filesystem::create_directory(dir);
    KVManager m_create(2, dir);
    for (int i = 0; i < 3; ++i) {
        KVPage p;
        p.id = i;
        p.key = {(float)i + 0.1f, (float)i + 0.2f};
        p.value = {(float)i + 0.3f, (float)i + 0.4f};
        m_create.save_page(p);
    }
    try {
        KVManager m(2, dir);
        auto p0 = m.load_page(0);
        printf("Loaded page 0, key[0]=%g\n", p0.key[0]);
        auto p1 = m.load_page(1);
        printf("Loaded page 1, key[0]=%g\n", p1.key[0]);
        printf("In-memory size: %zu\n", m.size());
        auto p2 = m.load_page(2);
        printf("Loaded page 2, key[0]=%g\n", p2.key[0]);
        printf("In-memory size after loading 3rd: %zu\n", m.size());
        if (m.contains(0)) {
            printf("Eviction failed: page 0 still in memory\n");
            return 2;
        }
        if (m.size() != 2 || !m.contains(1) || !m.contains(2)) return 3;
        printf("Eviction succeeded\n");
    } catch (const std::exception &e) {
        printf("Test failed: %s\n", e.what());
        return 1;
    }
    return 0;
}
