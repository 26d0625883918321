/* scheduler.h -- drop-in for the reference's scheduler/scheduler.h: prefetch
 * depth from observed load latencies and cache pressure
 * (scheduler/scheduler.cpp:15-37):
 *   avg   = mean of the last 16 observed latencies (0 before any)
 *   depth = clamp(round(max_depth * min(2, avg/50ms) * (1 - size/capacity)),
 *                 1, max_depth)
 * The constructor accepts any cache with size() and capacity() (the
 * reference's LayerCache, the KVManager, ...). */
#pragma once

#include <cstddef>
#include <deque>
#include <functional>
#include <mutex>

#include "kvx_cxx.h"

class KVX_CXX_API Scheduler {
public:
    template <class Cache>
    explicit Scheduler(Cache &cache, int max_depth = 4)
        : size_([&cache]() { return (size_t)cache.size(); }),
          capacity_([&cache]() { return (size_t)cache.capacity(); }),
          max_depth_(max_depth) {}

    void observeLoadLatency(double ms);  // one page / layer load took `ms`
    int getPrefetchDepth(int current);   // how many ids after `current` to prefetch

private:
    std::function<size_t()> size_, capacity_;
    int max_depth_;
    std::mutex mu_;
    std::deque<double> window_;
    size_t window_size_ = 16;
    double avg_latency_ms_ = 0.0;
};
