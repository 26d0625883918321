// KVPager prefetches a page into a KVManager asynchronously (the reference's
// tests/kv_pager_test.cpp); a Scheduler receives the load latency.
#include <chrono>
#include <cstdio>
#include <filesystem>
#include <thread>

#include "kv_cache.h"
#include "kv_pager.h"
#include "scheduler.h"

int main(int argc, char **argv) {
    const std::string dir = argc > 1 ? argv[1] : "pages";
    std::filesystem::create_directory(dir);
    KVManager m(4, dir);
    for (int i = 0; i < 4; ++i) {
        KVPage p;
        p.id = i;
        p.key = {(float)i + 0.1f};
        p.value = {(float)i + 0.2f};
        m.save_page(p);
    }
    try {
        KVManager kv(2, dir);
        Scheduler sched(kv, 4);
        KVPager pager(kv, &sched);
        pager.start();
        pager.request(3);
        std::this_thread::sleep_for(std::chrono::milliseconds(100));
        if (!kv.contains(3)) {
            printf("KVPager failed to prefetch page 3\n");
            return 2;
        }
        pager.request(0);
        pager.request(99);  // no such page file: logged, not fatal
        pager.drain();
        if (!kv.contains(0) || kv.contains(99)) return 3;
        pager.stop();
        printf("KVPager prefetch succeeded, depth now %d\n", sched.getPrefetchDepth(0));
    } catch (const std::exception &e) {
        printf("Test failed: %s\n", e.what());
        return 1;
    }
    return 0;
}
