/* Prefetch miss > 0, hit == 0; evict > 0; cached-layer bookkeeping (the
 * reference's llama_wrapper/tests/test_prefetch_evict.c). */
#include "engine_api.h"

int main(void) {
    void *h = open_engine();
    if (!h) return 1;
    NativeEngineApi *(*get_api)(void) = (NativeEngineApi * (*)(void)) dlsym(h, "adaptive_engine_get_api");
    if (!get_api) return 2;
    NativeEngineApi *api = get_api();
    api->start();
    int cached = api->getCachedLayers();
    if (cached != 0) { printf("cached=%d at start\n", cached); return 4; }
    long r = api->prefetchLayer(0);
    if (r <= 0) { printf("prefetch miss returned %ld\n", r); return 5; }
    if (api->getCachedLayers() != 1) return 6;
    r = api->prefetchLayer(0);
    if (r != 0) { printf("prefetch hit returned %ld\n", r); return 7; }
    r = api->evictLayer(0);
    if (r <= 0) { printf("evict returned %ld\n", r); return 8; }
    if (api->getCachedLayers() != 0) return 9;
    if (api->evictLayer(0) != 0) return 10;
    api->stop();
    dlclose(h);
    printf("TEST PASSED\n");
    return 0;
}
