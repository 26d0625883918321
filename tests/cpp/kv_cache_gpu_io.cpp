// Drives KVCacheGPU (include/KVCacheGPU.h) over an op trace on stdin, in the
// format of oracle/kvcachegpu_ref_driver.cpp ("<budget> <page>", then
// "op a b" lines), twice: one call per op, then with runs of transfers
// grouped into transferToGPUBatch calls.  Prints "<result> <used>" per op
// for each pass ("pass 1" / "pass 2" headers).  Every page sent is filled
// with a pattern of its op index; after each pass every page still held is
// read back and checked, so a slot handed out twice or overwritten shows
// up as "corrupt".
#include <cstdio>
#include <cstring>
#include <map>
#include <vector>

#include "KVCacheGPU.h"

struct Op {
    long long op, a, b;
};

static void fill(std::vector<unsigned char> &buf, size_t n, long long idx) {
    buf.resize(n);
    for (size_t i = 0; i < n; ++i) buf[i] = (unsigned char)((idx * 131 + i * 7 + (i >> 8)) & 0xFF);
}

static int check_live(KVCacheGPU &c, const std::map<int, std::pair<long long, size_t>> &sent) {
    int bad = 0;
    std::vector<unsigned char> want, got;
    for (auto &kv : sent) {
        KVCacheGPUPage *p = c.getPage(kv.first);
        if (!p) continue;
        fill(want, kv.second.second, kv.second.first);
        got.assign(kv.second.second, 0);
        if (p->pageSize != kv.second.second || !c.transferToHost(p->gpuMemPtr, got.data(), got.size()) ||
            memcmp(got.data(), want.data(), got.size()) != 0)
            ++bad;
    }
    return bad;
}

int main() {
    unsigned long long budget = 0, page = 0;
    if (scanf("%llu %llu", &budget, &page) != 2) return 1;
    std::vector<Op> ops;
    Op o;
    while (scanf("%lld %lld %lld", &o.op, &o.a, &o.b) == 3) ops.push_back(o);
    int corrupt = 0;
    for (int pass = 1; pass <= 2; ++pass) {
        printf("pass %d\n", pass);
        KVCacheGPU cache((size_t)budget, (size_t)page);
        std::map<int, std::pair<long long, size_t>> sent;  // page id -> (op index, size) of its last copy
        std::vector<unsigned char> buf;
        for (size_t i = 0; i < ops.size();) {
            const Op &x = ops[i];
            if (x.op == 0 && pass == 2) {  // a run of transfers as one batch
                size_t j = i;
                while (j < ops.size() && ops[j].op == 0 && j - i < 8) ++j;
                std::vector<std::vector<unsigned char>> bufs(j - i);
                std::vector<const void *> hp(j - i);
                std::vector<size_t> sz(j - i);
                std::vector<int> id(j - i);
                std::vector<void *> out(j - i);
                for (size_t k = i; k < j; ++k) {
                    fill(bufs[k - i], (size_t)ops[k].b, (long long)k);
                    hp[k - i] = bufs[k - i].data();
                    sz[k - i] = (size_t)ops[k].b;
                    id[k - i] = (int)ops[k].a;
                }
                cache.transferToGPUBatch(hp.data(), sz.data(), id.data(), (int)(j - i), out.data());
                for (size_t k = i; k < j; ++k) {
                    if (out[k - i]) sent[(int)ops[k].a] = {(long long)k, (size_t)ops[k].b};
                    printf("%d -\n", out[k - i] ? 1 : 0);
                }
                printf("used %zu\n", cache.getUsedMemory());
                i = j;
                continue;
            }
            long long r = 0;
            if (x.op == 0) {
                fill(buf, (size_t)x.b, (long long)i);
                void *g = cache.transferToGPU(buf.data(), (size_t)x.b, (int)x.a);
                r = g != nullptr;
                if (g) {
                    sent[(int)x.a] = {(long long)i, (size_t)x.b};
                    std::vector<unsigned char> back((size_t)x.b);
                    if (!cache.transferToHost(g, back.data(), back.size()) || back != buf) ++corrupt;
                }
            } else if (x.op == 1) {
                cache.markPageUsed((int)x.a, (uint64_t)x.b);
            } else if (x.op == 2) {
                r = cache.evictLRUPage();
            } else if (x.op == 3) {
                cache.clear();
            } else if (x.op == 4) {
                KVCacheGPUPage *p = cache.getPage((int)x.a);
                r = p ? (long long)p->lastUsedToken : -1;
            }
            printf("%lld %zu\n", r, cache.getUsedMemory());
            ++i;
        }
        corrupt += check_live(cache, sent);
    }
    printf("corrupt %d\n", corrupt);
    return corrupt ? 3 : 0;
}
