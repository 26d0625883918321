/* KV operations return latency > 0 for a valid page and < 0 for an
 * invalid one (the reference's llama_wrapper/tests/test_kv_operations.c). */
#include "engine_api.h"

int main(void) {
    void *h = open_engine();
    if (!h) return 1;
    NativeEngineApi *(*get_api)(void) = (NativeEngineApi * (*)(void)) dlsym(h, "adaptive_engine_get_api");
    if (!get_api) return 2;
    NativeEngineApi *api = get_api();
    if (!api) return 3;
    api->start();
    printf("Total KV pages: %d\n", api->getKvPages());
    int passed = 0, failed = 0;
#define EXPECT(cond, what, val)                                         \
    do {                                                                \
        if (cond) { printf("ok   %s = %ld\n", what, (long)(val)); ++passed; } \
        else { printf("FAIL %s = %ld\n", what, (long)(val)); ++failed; }  \
    } while (0)
    long r = api->moveKvToRam(0);
    EXPECT(r > 0, "moveKvToRam(0)", r);
    r = api->moveKvToRam(-1);
    EXPECT(r < 0, "moveKvToRam(-1)", r);
    r = api->moveKvToGpu(1);
    EXPECT(r > 0, "moveKvToGpu(1)", r);
    r = api->compressKv(2);
    EXPECT(r > 0, "compressKv(2)", r);
    r = api->offloadKv(3);
    EXPECT(r > 0, "offloadKv(3)", r);
    long r1 = api->moveKvToRam(4), r2 = api->moveKvToGpu(4), r3 = api->compressKv(4);
    EXPECT(r1 > 0 && r2 > 0 && r3 > 0, "sequential ram/gpu/compress", r1 + r2 + r3);
    r = api->moveKvToGpu(api->getKvPages());
    EXPECT(r == -1, "moveKvToGpu(out of range)", r);
    api->stop();
    r = api->moveKvToRam(0);
    EXPECT(r == -1, "moveKvToRam after stop", r);
    dlclose(h);
    printf("Passed: %d Failed: %d\n", passed, failed);
    return failed ? 5 : 0;
}
