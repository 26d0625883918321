// prefetcher.cpp -- the page-migration Prefetcher (include/prefetcher.h).
#include "prefetcher.h"

#include "engine.h"
#include "scheduler.h"

using kvx_engine::Engine;

namespace {

// The engine's move to the GPU tier; a layer already there is a hit.
double engine_mover(int id) {
    Engine &e = Engine::instance();
    if (e.layer_tier(id) == kvx_engine::kGpu) return 0.0;
    const long ms = e.move_to_gpu(id);
    return ms < 0 ? -1.0 : (double)ms;
}

}  // namespace

Prefetcher::Prefetcher(Scheduler *sched) : Prefetcher(Mover(engine_mover), sched) {}

Prefetcher::Prefetcher(Mover mover, Scheduler *sched) : mover_(std::move(mover)), scheduler_(sched) {}

Prefetcher::~Prefetcher() { stop(); }

void Prefetcher::setScheduler(Scheduler *s) { scheduler_.store(s); }

void Prefetcher::start() {
    bool expected = false;
    if (!running_.compare_exchange_strong(expected, true)) return;
    thread_ = std::thread(&Prefetcher::worker, this);
}

// Passing through the queue mutex before notifying: a worker between its
// predicate check and its wait cannot miss the wake-up.
void Prefetcher::stop() {
    bool expected = true;
    if (!running_.compare_exchange_strong(expected, false)) return;
    { std::lock_guard<std::mutex> lk(mu_); }
    cv_.notify_all();
    if (thread_.joinable()) thread_.join();
    std::lock_guard<std::mutex> lk(mu_);
    busy_ = 0;
    idle_cv_.notify_all();
}

void Prefetcher::request(int layer_id) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        q_.push(layer_id);
    }
    cv_.notify_one();
}

void Prefetcher::schedule(int current, int num_layers) {
    Scheduler *s = scheduler_.load();
    const int depth = s ? s->getPrefetchDepth(current) : 2;
    for (int i = 1; i <= depth; ++i)
        if (current + i >= 0 && current + i < num_layers) request(current + i);
}

void Prefetcher::drain() {
    std::unique_lock<std::mutex> lk(mu_);
    idle_cv_.wait(lk, [this] { return (q_.empty() && busy_ == 0) || !running_; });
}

void Prefetcher::worker() {
    for (;;) {
        int id = -1;
        {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [this] { return !q_.empty() || !running_; });
            if (!running_) break;
            id = q_.front();
            q_.pop();
            ++busy_;
        }
        requests_.fetch_add(1);
        const double ms = mover_ ? mover_(id) : -1.0;
        if (ms < 0) {
            failures_.fetch_add(1);
        } else if (ms > 0) {  // a load happened (0: already resident)
            loads_.fetch_add(1);
            if (Scheduler *s = scheduler_.load()) s->observeLoadLatency(ms);
        }
        std::lock_guard<std::mutex> lk(mu_);
        --busy_;
        if (q_.empty() && busy_ == 0) idle_cv_.notify_all();
    }
}
