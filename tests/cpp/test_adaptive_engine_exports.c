/* The engine library exports adaptive_engine_get_api (the reference's
 * llama_wrapper/tests/test_adaptive_engine_exports.c, Linux dlopen). */
#include "engine_api.h"

int main(void) {
    void *h = open_engine();
    if (!h) return 1;
    void *f = dlsym(h, "adaptive_engine_get_api");
    if (!f) {
        printf("Symbol adaptive_engine_get_api not found\n");
        dlclose(h);
        return 2;
    }
    if (!dlsym(h, "adaptive_engine_test_release_layer")) {
        printf("Symbol adaptive_engine_test_release_layer not found\n");
        return 3;
    }
    NativeEngineApi *api = ((NativeEngineApi * (*)(void)) f)();
    if (!api || !api->start || !api->getCachedLayers) return 4;
    printf("Symbol adaptive_engine_get_api found\n");
    dlclose(h);
    return 0;
}
