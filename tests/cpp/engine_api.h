/* Shared by the C tests: load the engine the way the reference's JNI loader
 * does (dlopen by file name, dlsym adaptive_engine_get_api;
 * src/main/cpp/adaptive_scheduler.cpp:175-189). */
#ifndef TEST_ENGINE_API_H
#define TEST_ENGINE_API_H
#include <dlfcn.h>
#include <stdio.h>

typedef struct NativeEngineApi {
    void (*start)();
    void (*stop)();
    long (*prefetchLayer)(int layerId);
    long (*evictLayer)(int layerId);
    long (*keepLayer)(int layerId);
    long (*moveKvToRam)(long kvPageId);
    long (*moveKvToGpu)(long kvPageId);
    long (*compressKv)(long kvPageId);
    long (*offloadKv)(long kvPageId);
    int (*getCurrentLayer)();
    long (*getGpuMemory)();
    int (*getKvPages)();
    int (*getCachedLayers)();
} NativeEngineApi;

typedef void (*release_t)(int layerId);

static void *open_engine(void) {
    const char *names[] = {"libadaptive_engine.so", "libnative_engine.so", "libadaptive_scheduler_engine.so"};
    for (int i = 0; i < 3; ++i) {
        void *h = dlopen(names[i], RTLD_NOW | RTLD_LOCAL);
        if (h) return h;
    }
    printf("dlopen failed: %s\n", dlerror());
    return 0;
}
#endif
