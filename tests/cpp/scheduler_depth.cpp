// Prints Scheduler::getPrefetchDepth over a grid read from stdin:
// lines "size capacity max_depth n lat_1 ... lat_n" -> one depth per line.
#include <cstdio>
#include <vector>

#include "scheduler.h"

struct FakeCache {
    size_t s, c;
    size_t size() { return s; }
    size_t capacity() { return c; }
};

int main() {
    size_t size, cap;
    int md, n;
    while (scanf("%zu %zu %d %d", &size, &cap, &md, &n) == 4) {
        FakeCache cache{size, cap};
        Scheduler s(cache, md);
        for (int i = 0; i < n; ++i) {
            double x;
            if (scanf("%lf", &x) != 1) return 1;
            s.observeLoadLatency(x);
        }
        printf("%d\n", s.getPrefetchDepth(0));
    }
    return 0;
}
