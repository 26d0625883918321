/* kv_pager.h -- drop-in for the reference's cache/kv_pager.h: a background
 * thread that loads requested page ids into a KVManager (so into device
 * memory) and reports each load's latency to an optional Scheduler
 * (cache/kv_pager.cpp:13-67).  The reference's 5 ms sleep after a load
 * ("simulate processing", kv_pager.cpp:58) is not reproduced. */
#pragma once

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <queue>
#include <thread>

#include "kv_cache.h"
#include "kvx_cxx.h"

class Scheduler;  // receives load latencies when given

class KVX_CXX_API KVPager {
public:
    explicit KVPager(KVManager &kv, Scheduler *sched = nullptr);
    ~KVPager();

    void start();
    void stop();

    void request(int page_id);  // queue `page_id` for loading

    // Additive: block until every request made so far was handled.
    void drain();

private:
    void worker();

    KVManager &kv_;
    Scheduler *scheduler_ = nullptr;
    std::thread thread_;
    std::mutex mu_;
    std::condition_variable cv_, idle_cv_;
    std::queue<int> q_;
    std::atomic<bool> running_{false};
    int busy_ = 0;
};
