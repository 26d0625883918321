// Replays a KVCacheGPU op trace on the reference's own class
// (native-engine/cpp/KVCacheGPU.cpp, compiled unmodified against
// oracle/host_cuda/cuda_runtime.h).  Test infrastructure: makes the golden
// traces of tests/golden/make_golden.py.
//
// stdin: "<total_bytes> <page_size>" then one op per line "op a b":
//   0 transfer(pageId a, size b)   -> 1 / 0
//   1 markPageUsed(a, token b)     -> 0
//   2 evictLRUPage()               -> 1 / 0
//   3 clear()                      -> 0
//   4 getPage(a)                   -> lastUsedToken, or -1 without a page
// stdout: "<result> <getUsedMemory()>" per op.
#include <cstdio>
#include <vector>

#include "KVCacheGPU.h"

int main() {
    unsigned long long total = 0, page = 0;
    if (scanf("%llu %llu", &total, &page) != 2) return 1;
    KVCacheGPU cache((size_t)total, (size_t)page);
    std::vector<unsigned char> host(1 << 20, 0x5a);
    long long op, a, b;
    while (scanf("%lld %lld %lld", &op, &a, &b) == 3) {
        long long r = 0;
        if (op == 0) {
            if ((size_t)b > host.size()) host.resize((size_t)b, 0x5a);
            r = cache.transferToGPU(host.data(), (size_t)b, (int)a) != nullptr;
        } else if (op == 1) {
            cache.markPageUsed((int)a, (uint64_t)b);
        } else if (op == 2) {
            r = cache.evictLRUPage();
        } else if (op == 3) {
            cache.clear();
        } else if (op == 4) {
            KVCacheGPUPage *p = cache.getPage((int)a);
            r = p ? (long long)p->lastUsedToken : -1;
        }
        printf("%lld %llu\n", r, (unsigned long long)cache.getUsedMemory());
    }
    return 0;
}
