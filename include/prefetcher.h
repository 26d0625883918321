/* prefetcher.h -- drop-in for the reference's prefetch/prefetcher.h
 * (prefetcher.h:14-38, prefetcher.cpp:41-78) on the page-migration path:
 * request(layer) queues a layer whose KV a background thread brings to the
 * device, and every load's latency goes to the Scheduler
 * (Scheduler::observeLoadLatency), as the reference's worker does after
 * LayerLoader::load.  Here the load is the engine's move of the layer's KV
 * pages to the GPU tier (the NativeEngineApi moveKvToGpu path), or any
 * caller-given mover; a layer already on the device is skipped like a
 * LayerCache hit.  The reference's 10 ms "simulate IO" sleep is not
 * reproduced.  schedule() is InferenceController::schedulePrefetch
 * (runtime/inference.cpp:61-84): layers current+1 .. current+depth with the
 * Scheduler's depth (2 without a Scheduler). */
#pragma once

#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <queue>
#include <thread>

#include "kvx_cxx.h"

class Scheduler;

class KVX_CXX_API Prefetcher {
public:
    // Brings layer `id` to the device: the load's latency in ms (> 0), 0 if
    // it was resident already, < 0 on failure.
    using Mover = std::function<double(int id)>;

    // Moves through the process-wide engine (adaptive_engine.h).
    explicit Prefetcher(Scheduler *sched = nullptr);
    Prefetcher(Mover mover, Scheduler *sched = nullptr);
    // Source compatibility with the reference's constructor: the layer-weight
    // loader and cache are not this library's (weights are out of its scope).
    template <class Loader, class Cache>
    Prefetcher(Loader &, Cache &, Scheduler *sched = nullptr) : Prefetcher(sched) {}
    ~Prefetcher();

    void request(int layer_id);  // thread-safe
    void start();
    void stop();
    void setScheduler(Scheduler *s);

    // Additive.
    void schedule(int current, int num_layers);  // request current+1 .. current+depth (< num_layers)
    void drain();                                // block until every request made so far was handled
    long requests() const { return requests_.load(); }
    long loads() const { return loads_.load(); }
    long failures() const { return failures_.load(); }

private:
    void worker();

    Mover mover_;
    std::atomic<Scheduler *> scheduler_{nullptr};
    std::thread thread_;
    std::mutex mu_;
    std::condition_variable cv_, idle_cv_;
    std::queue<int> q_;
    std::atomic<bool> running_{false};
    int busy_ = 0;
    std::atomic<long> requests_{0}, loads_{0}, failures_{0};
};
