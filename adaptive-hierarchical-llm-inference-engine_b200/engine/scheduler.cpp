// scheduler.cpp -- prefetch depth policy with the semantics of the
// reference's scheduler/scheduler.cpp:15-37 (sliding window of 16 load
// latencies; depth grows with latency, shrinks with cache pressure).
#include "scheduler.h"

#include <algorithm>
#include <cmath>
#include <new>
#include <numeric>

#include "kvx_scheduler.h"

void Scheduler::observeLoadLatency(double ms) {
    std::lock_guard<std::mutex> lk(mu_);
    window_.push_back(ms);
    while (window_.size() > window_size_) window_.pop_front();
    const double total = std::accumulate(window_.begin(), window_.end(), 0.0);
    avg_latency_ms_ = total / (double)window_.size();
}

int Scheduler::getPrefetchDepth(int /*current*/) {
    std::lock_guard<std::mutex> lk(mu_);
    const size_t cap = capacity_();
    const double pressure = cap > 0 ? (double)size_() / (double)cap : 0.0;
    const double lf = avg_latency_ms_ / 50.0;           // latency normalised to 50 ms
    const double latency_factor = lf < 2.0 ? lf : 2.0;  // capped at 2x
    const double raw = (double)max_depth_ * latency_factor * (1.0 - pressure);
    const int r = (int)std::round(raw);
    const int d = r < max_depth_ ? r : max_depth_;
    return d > 1 ? d : 1;
}

// C entry points (include/kvx_scheduler.h): the Scheduler over a cache whose
// size and capacity the caller states with each question.

struct kvx_scheduler {
    struct Counts {
        int64_t n = 0, cap = 0;
        size_t size() const { return (size_t)n; }
        size_t capacity() const { return (size_t)cap; }
    } cache;
    Scheduler sched;
    explicit kvx_scheduler(int max_depth) : sched(cache, max_depth) {}
};

extern "C" KVX_API int kvx_scheduler_create(int32_t max_depth, kvx_scheduler **out) {
    if (!out || max_depth < 1) return KVX_EINVAL;
    *out = new (std::nothrow) kvx_scheduler(max_depth);
    return *out ? KVX_OK : KVX_ENOSPC;
}

extern "C" KVX_API void kvx_scheduler_destroy(kvx_scheduler *s) { delete s; }

extern "C" KVX_API int kvx_scheduler_observe(kvx_scheduler *s, double ms) {
    if (!s || !(ms >= 0.0)) return KVX_EINVAL;
    s->sched.observeLoadLatency(ms);
    return KVX_OK;
}

extern "C" KVX_API int kvx_scheduler_depth(kvx_scheduler *s, int32_t current, int64_t size, int64_t capacity,
                                           int32_t *depth) {
    if (!s || !depth || size < 0 || capacity < 0) return KVX_EINVAL;
    s->cache.n = size;
    s->cache.cap = capacity;
    *depth = s->sched.getPrefetchDepth(current);
    return KVX_OK;
}
