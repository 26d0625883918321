// scheduler.cpp -- prefetch depth policy with the semantics of the
// reference's scheduler/scheduler.cpp:15-37 (sliding window of 16 load
// latencies; depth grows with latency, shrinks with cache pressure).
#include "scheduler.h"

#include <algorithm>
#include <cmath>
#include <numeric>

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
