// Drives the Prefetcher drop-in (include/prefetcher.h) with a fake mover:
// FIFO order of requests, hits / loads / failures, the Scheduler fed with
// each load's latency, schedule() as InferenceController::schedulePrefetch.
// Prints one "key value..." line per fact for tests/test_cxx_dropins.py.
#include <cstdio>
#include <mutex>
#include <vector>

#include "prefetcher.h"
#include "scheduler.h"

struct FakeCache {
    size_t s, c;
    size_t size() const { return s; }
    size_t capacity() const { return c; }
};
struct FakeLoader {};
struct FakeLayerCache {};

int main() {
    FakeCache cache{1, 8};
    Scheduler sched(cache, 4), twin(cache, 4);
    std::mutex mu;
    std::vector<int> order;
    auto mover = [&](int id) -> double {
        { std::lock_guard<std::mutex> lk(mu); order.push_back(id); }
        if (id % 3 == 0) return 0.0;   // already resident
        if (id == 13) return -1.0;     // failed move
        return 20.0 + id;              // a load of 20 + id ms
    };
    Prefetcher p(mover, &sched);
    p.start();
    for (int id = 0; id < 16; ++id) p.request(id);
    p.drain();
    for (int id = 0; id < 16; ++id)
        if (id % 3 != 0 && id != 13) twin.observeLoadLatency(20.0 + id);
    std::printf("order");
    for (int id : order) std::printf(" %d", id);
    std::printf("\ncounts %ld %ld %ld\n", p.requests(), p.loads(), p.failures());
    std::printf("depth %d %d\n", sched.getPrefetchDepth(0), twin.getPrefetchDepth(0));
    // schedulePrefetch from layer 5 of 8: layers 6 and 7 at most
    const int depth = sched.getPrefetchDepth(5);
    order.clear();
    p.schedule(5, 8);
    p.drain();
    std::printf("schedule %d", depth);
    for (int id : order) std::printf(" %d", id);
    std::printf("\n");
    p.stop();
    // the reference's constructor shape compiles (no engine call made)
    FakeLoader loader;
    FakeLayerCache lcache;
    Prefetcher q(loader, lcache, &sched);
    q.setScheduler(nullptr);
    std::printf("ok\n");
    return 0;
}
