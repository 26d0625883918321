// kv_pager.cpp -- background page loader with the reference's interface and
// queue semantics (cache/kv_pager.cpp:13-67): requested ids not resident in
// the KVManager are loaded (into device memory) and each load's latency is
// reported to the Scheduler.
#include "kv_pager.h"

#include <chrono>
#include <cstdio>

#include "scheduler.h"

KVPager::KVPager(KVManager &kv, Scheduler *sched) : kv_(kv), scheduler_(sched) {}

KVPager::~KVPager() { stop(); }

void KVPager::start() {
    bool expected = false;
    if (!running_.compare_exchange_strong(expected, true)) return;
    thread_ = std::thread(&KVPager::worker, this);
}

void KVPager::stop() {
    bool expected = true;
    if (running_.compare_exchange_strong(expected, false)) {
        // pass through the mutex: a worker between its predicate check and
        // its wait would otherwise miss this notification and never wake
        { std::lock_guard<std::mutex> lk(mu_); }
        cv_.notify_all();
        idle_cv_.notify_all();
        if (thread_.joinable()) thread_.join();
    }
}

void KVPager::request(int page_id) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        q_.push(page_id);
    }
    cv_.notify_one();
}

void KVPager::drain() {
    std::unique_lock<std::mutex> lk(mu_);
    idle_cv_.wait(lk, [this] { return (q_.empty() && busy_ == 0) || !running_; });
}

void KVPager::worker() {
    using clock = std::chrono::steady_clock;
    long requests = 0, loads = 0, failures = 0;
    for (;;) {
        int id = -1;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [this] { return !q_.empty() || !running_; });
            if (!running_ && q_.empty()) break;
            id = q_.front();
            q_.pop();
            ++busy_;
        }
        if (id >= 0) {
            ++requests;
            try {
                if (!kv_.contains(id)) {
                    const auto t0 = clock::now();
                    (void)kv_.load_page(id);
                    const double ms = std::chrono::duration<double, std::milli>(clock::now() - t0).count();
                    ++loads;
                    if (scheduler_) scheduler_->observeLoadLatency(ms);
                }
            } catch (const std::exception &e) {
                ++failures;
                fprintf(stderr, "[KVPager] failed to load page %d: %s\n", id, e.what());
            }
        }
        {
            std::lock_guard<std::mutex> lk(mu_);
            --busy_;
        }
        idle_cv_.notify_all();
    }
    idle_cv_.notify_all();
    (void)requests;
    (void)loads;
    (void)failures;
}
