/* Two threads pin and release the same layer 100 times each: no crash, a
 * consistent cached count (the reference's
 * llama_wrapper/tests/test_concurrent_pin_unpin.c, pthreads). */
#include <pthread.h>
#include <unistd.h>

#include "engine_api.h"

static NativeEngineApi *api;
static release_t release_hook;

static void *pin_thread(void *arg) {
    int layer = (int)(long)arg;
    for (int i = 0; i < 100; ++i) {
        api->keepLayer(layer);
        usleep(1000);
    }
    return 0;
}

static void *unpin_thread(void *arg) {
    int layer = (int)(long)arg;
    for (int i = 0; i < 100; ++i) {
        release_hook(layer);
        usleep(1000);
    }
    return 0;
}

int main(void) {
    void *h = open_engine();
    if (!h) return 1;
    NativeEngineApi *(*get_api)(void) = (NativeEngineApi * (*)(void)) dlsym(h, "adaptive_engine_get_api");
    release_hook = (release_t)dlsym(h, "adaptive_engine_test_release_layer");
    if (!get_api || !release_hook) return 2;
    api = get_api();
    api->start();
    api->prefetchLayer(0);
    pthread_t a, b;
    pthread_create(&a, 0, pin_thread, (void *)0);
    pthread_create(&b, 0, unpin_thread, (void *)0);
    pthread_join(a, 0);
    pthread_join(b, 0);
    int cached = api->getCachedLayers();
    printf("concurrent test completed, cached=%d\n", cached);
    if (cached != 1) return 3;
    for (int i = 0; i < 200; ++i) release_hook(0);  /* drop whatever pins remain */
    if (api->evictLayer(0) <= 0) return 4;
    api->stop();
    dlclose(h);
    printf("TEST PASSED\n");
    return 0;
}
