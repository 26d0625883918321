// The Prefetcher drop-in on the engine: with 4 layers and 2 device slabs,
// prefetching layers 2 and 3 (which start in RAM) brings them to the GPU
// tier and evicts the least recently used layers 0 and 1 to RAM; a second
// request of a resident layer is a hit.  Exit code 0 when all holds.
#include <cstdio>
#include <cstring>

#include "adaptive_engine.h"
#include "prefetcher.h"
#include "scheduler.h"

struct FakeCache {
    size_t size() const { return 1; }
    size_t capacity() const { return 4; }
};

#define CHECK(c)                                            \
    do {                                                    \
        if (!(c)) {                                         \
            std::printf("FAILED %s (line %d)\n", #c, __LINE__); \
            return 1;                                       \
        }                                                   \
    } while (0)

int main(int argc, char **argv) {
    adaptive_engine_config cfg;
    adaptive_engine_default_config(&cfg);
    cfg.layers = 4;
    cfg.pages_per_layer = 16;
    cfg.max_batch = 2;
    cfg.gpu_layer_slots = 2;
    if (argc > 1) std::snprintf(cfg.offload_dir, sizeof(cfg.offload_dir), "%s", argv[1]);
    CHECK(adaptive_engine_configure(&cfg) == 0);
    NativeEngineApi *api = adaptive_engine_get_api();
    api->start();
    CHECK(adaptive_engine_layer_tier(2) == 1 && adaptive_engine_layer_tier(3) == 1);
    FakeCache fc;
    Scheduler sched(fc, 4);
    Prefetcher p(&sched);
    p.start();
    p.request(2);
    p.request(3);
    p.drain();
    CHECK(p.loads() == 2 && p.failures() == 0);
    CHECK(adaptive_engine_layer_tier(2) == 0 && adaptive_engine_layer_tier(3) == 0);
    CHECK(adaptive_engine_layer_tier(0) == 1 && adaptive_engine_layer_tier(1) == 1);
    p.request(3);  // resident: a hit
    p.request(7);  // no such layer: a failure
    p.drain();
    CHECK(p.loads() == 2 && p.failures() == 1 && p.requests() == 4);
    p.stop();
    api->stop();
    std::printf("ok\n");
    return 0;
}
