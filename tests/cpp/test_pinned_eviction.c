/* Evicting a pinned layer is refused with -2 until the pin is released
 * (the reference's llama_wrapper/tests/test_pinned_eviction.c). */
#include "engine_api.h"

int main(void) {
    void *h = open_engine();
    if (!h) return 1;
    NativeEngineApi *(*get_api)(void) = (NativeEngineApi * (*)(void)) dlsym(h, "adaptive_engine_get_api");
    release_t release = (release_t)dlsym(h, "adaptive_engine_test_release_layer");
    if (!get_api || !release) return 2;
    NativeEngineApi *api = get_api();
    api->start();
    api->prefetchLayer(0);
    long pin = api->keepLayer(0);
    printf("pin returned %ld\n", pin);
    if (pin != 1) return 3;
    long ev = api->evictLayer(0);
    printf("evict returned %ld (expected -2)\n", ev);
    if (ev != -2) return 4;
    if (api->moveKvToRam(0) != -2 || api->offloadKv(0) != -2) return 5;
    release(0);
    ev = api->evictLayer(0);
    printf("evict after release returned %ld\n", ev);
    if (ev <= 0) return 6;
    api->stop();
    dlclose(h);
    printf("TEST PASSED\n");
    return 0;
}
