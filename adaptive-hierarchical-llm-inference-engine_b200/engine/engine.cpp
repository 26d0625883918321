// engine.cpp -- tier moves, LRU slab eviction and the decode step of the
// KV-cache engine (see engine.h).  All device work goes through the kvx C
// ABI (include/kvx.h); this file only does bookkeeping and copies.
#include "engine.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>

#include <nccl.h>

namespace kvx_engine {
namespace {

// Layers of the edge groups of a decode step: inputs are copied and outputs
// read back per group (one event each way), the group's launches run back to
// back.  The first group's input copy and the last group's read-back overlap
// no kernel, so those groups are short.  On one GPU the layers between them
// form one group: every group boundary puts an event record and wait between
// two dependent launches (about 25 us), while a layer's copies (about 6 us
// in, 4 us out at batch 32) hide easily behind the 2-layer groups' kernels.
// With a communicator they form groups of kCommGroup, so each group's
// all-gather and read-back run under the next group's kernels instead of
// all at the end.  KVX_ENGINE_GROUP = n > 0 sets the middle groups' size.
constexpr int kEdgeGroup = 2;
constexpr int kCommGroup = 7;

int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    if (!v || !*v) return dflt;
    char *end = nullptr;
    long x = strtol(v, &end, 10);
    return (end && *end == 0 && x > 0 && x < (1 << 30)) ? (int)x : dflt;
}

double now_ms() {
    using namespace std::chrono;
    return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

uint64_t splitmix(uint64_t &x) {
    uint64_t z = (x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// NCCL through dlopen: binds to the libnccl.so.2 the process already loaded
// (torch's), else the system one; no link-time dependency.
struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    bool ok = false;
};

const Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        n.ok = n.get_unique_id && n.comm_init_rank && n.all_gather && n.comm_destroy;
    });
    return n;
}

// The moves' stream at the device's highest priority: a running decode step
// keeps a grid pending at all times (dependent launches), so a move kernel
// (int8 compress / decompress) on a default-priority stream would get SMs
// only after the whole step; at high priority its CTAs are dispatched as the
// decode's CTAs retire.
bool create_move_stream(cudaStream_t *st) {
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) greatest = 0;
    return cudaStreamCreateWithPriority(st, cudaStreamNonBlocking, greatest) == cudaSuccess;
}

}  // namespace

int nccl_unique_id(void *id128) {
    const Nccl &n = nccl();
    if (!n.ok) return KVX_EUNSUPPORTED;
    ncclUniqueId id;
    if (n.get_unique_id(&id) != ncclSuccess) return KVX_ECUDA;
    memcpy(id128, &id, sizeof(id));
    return KVX_OK;
}

int Engine::set_comm(int rank, int world, const void *id128) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !step_active_; });
    if (!started_ || world < 1 || rank < 0 || rank >= world || !id128) return KVX_EINVAL;
    const Nccl &n = nccl();
    if (!n.ok) return KVX_EUNSUPPORTED;
    if (comm_) return KVX_EBUSY;
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    ncclComm_t c = nullptr;
    if (n.comm_init_rank(&c, world, id, rank) != ncclSuccess) return KVX_ECUDA;
    const size_t gbytes = (size_t)cfg_.layers * world * cfg_.max_batch * cfg_.q_heads * 128 * 2;
    if (cudaStreamCreateWithFlags(&comm_stream_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&d_gather_, gbytes) != cudaSuccess ||
        cudaMalloc(&d_status_, (2 + 2 * world) * sizeof(int32_t)) != cudaSuccess ||
        cudaHostAlloc(&h_status_, (2 + 2 * world) * sizeof(int32_t), cudaHostAllocDefault) != cudaSuccess) {
        n.comm_destroy(c);
        return KVX_ECUDA;
    }
    ev_gath_.assign(cfg_.layers, nullptr);
    for (auto &e : ev_gath_) cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    device_bytes_ += (long long)gbytes;
    comm_ = c;
    world_ = world;
    rank_ = rank;
    return KVX_OK;
}

int Engine::set_readback_share(int share) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !step_active_; });
    if (share != 0 && share != 1) return KVX_EINVAL;
    readback_share_ = share == 1;
    return KVX_OK;
}

Engine &Engine::instance() {
    static Engine *e = new Engine();  // lives until exit; never destroyed mid-call
    return *e;
}

Engine::~Engine() { release_all(); }

void Engine::default_config(adaptive_engine_config *cfg) const {
    memset(cfg, 0, sizeof(*cfg));
    cfg->layers = env_int("ADAPTIVELLM_KV_LAYERS", 28);
    cfg->kv_heads = 8;
    cfg->q_heads = 24;
    cfg->head_dim = 128;
    cfg->page_tokens = 16;
    cfg->max_batch = env_int("ADAPTIVELLM_KV_BATCH", 32);
    cfg->pages_per_layer = env_int("ADAPTIVELLM_KV_PAGES", 256);
    cfg->gpu_layer_slots = std::min(env_int("ADAPTIVELLM_KV_GPU_LAYERS", cfg->layers), cfg->layers);
    const char *dev = getenv("ADAPTIVELLM_DEVICE");
    cfg->device = dev ? atoi(dev) : 0;
    const char *dir = getenv("ADAPTIVELLM_KV_OFFLOAD_DIR");
    snprintf(cfg->offload_dir, sizeof(cfg->offload_dir), "%s", dir && *dir ? dir : "/tmp");
    cfg->ram_layer_slots = env_int("ADAPTIVELLM_KV_RAM_LAYERS", cfg->layers);
    cfg->int8_layer_slots = env_int("ADAPTIVELLM_KV_INT8_LAYERS", cfg->layers);
}

long long Engine::clock_ms() const { return (long long)(now_ms() - t0_ms_); }

long long Engine::layer_last_access_ms(int layer) {
    std::lock_guard<std::mutex> lk(mu_);
    return valid(layer) ? layers_[layer].last_access_ms : -1;
}

// KVCompressionEngine's age policy (src/main/java/com/adaptivellm/kv/
// KVCompressionEngine.java:62-98) over the layers: age = now - last access;
// age >= compressedThreshold -> COMPRESSED, else age >= int8Threshold ->
// INT8, and only GPU-resident layers change (applyCompression's
// GPU_RESIDENT -> COMPRESSED transition).  The reference only relabels the
// page; here INT8 is the int8 tier (compressKv, a half of fp16) and
// COMPRESSED the NF4 tier (a quarter: estimateSize's ratios).  Thresholds
// must be positive (the constructor's IllegalArgumentException).  Pinned
// layers are left as they are, as compressKv leaves them.
int Engine::compress_aged(long long int8_thr, long long comp_thr, long long now, int apply, int32_t *decisions) {
    if (int8_thr <= 0 || comp_thr <= 0) return KVX_EINVAL;
    std::unique_lock<std::mutex> lk(mu_);
    if (!started_) return KVX_EINVAL;
    if (now < 0) now = clock_ms();
    const int n = (int)layers_.size();
    std::vector<int32_t> d(n, 0);
    for (int l = 0; l < n; ++l) {
        const Layer &L = layers_[l];
        const long long age = now - L.last_access_ms;
        const int want = age >= comp_thr ? 2 : (age >= int8_thr ? 1 : 0);
        d[l] = (L.tier == kGpu && L.refcount == 0) ? want : 0;
        if (decisions) decisions[l] = d[l];
    }
    if (!apply) return 0;
    int done = 0;
    for (int l = 0; l < n; ++l) {
        if (!d[l]) continue;
        wait_not_moving(lk, l);
        if (!started_) return KVX_EINVAL;
        if (layers_[l].tier != kGpu || layers_[l].refcount > 0) continue;  // changed meanwhile
        const int rc = gpu_to_int8(lk, l, d[l] == 2);
        if (rc < 0) return rc;
        ++done;
    }
    return done;
}

int Engine::step_in_flight() {
    std::lock_guard<std::mutex> lk(mu_);
    return step_active_ ? 1 : 0;
}

int Engine::configure(const adaptive_engine_config &cfg) {
    std::lock_guard<std::mutex> lk(mu_);
    if (started_) return KVX_EBUSY;
    if (cfg.layers <= 0 || cfg.kv_heads <= 0 || cfg.q_heads <= 0 || cfg.q_heads % cfg.kv_heads ||
        cfg.head_dim != 128 || cfg.page_tokens != 16 || cfg.max_batch <= 0 || cfg.pages_per_layer <= 0 ||
        cfg.gpu_layer_slots <= 0 || cfg.gpu_layer_slots > cfg.layers || cfg.ram_layer_slots < 0 ||
        cfg.int8_layer_slots < 0)
        return KVX_EINVAL;
    cfg_ = cfg;
    cfg_.offload_dir[sizeof(cfg_.offload_dir) - 1] = 0;
    configured_ = true;
    return KVX_OK;
}

bool Engine::started() {
    std::lock_guard<std::mutex> lk(mu_);
    return started_;
}

void Engine::start() {
    std::lock_guard<std::mutex> lk(mu_);
    if (started_) return;
    if (!configured_) default_config(&cfg_);
    if (cudaSetDevice(cfg_.device) != cudaSuccess || kvx_device_check() != KVX_OK) {
        fprintf(stderr, "[adaptive_engine] start(): no sm_100 device %d\n", cfg_.device);
        return;
    }
    slab_bytes_ = (size_t)cfg_.pages_per_layer * 2 * cfg_.kv_heads * 16 * 128 * sizeof(uint16_t);
    blocks_per_slab_ = (size_t)cfg_.pages_per_layer * 2 * cfg_.kv_heads;
    bool ok = cudaMalloc(&arena_, slab_bytes_ * cfg_.gpu_layer_slots) == cudaSuccess &&
              cudaMemset(arena_, 0, slab_bytes_ * cfg_.gpu_layer_slots) == cudaSuccess;
    ok = ok && cudaStreamCreateWithFlags(&compute_, cudaStreamNonBlocking) == cudaSuccess &&
         cudaStreamCreateWithFlags(&copy_, cudaStreamNonBlocking) == cudaSuccess &&
         create_move_stream(&move_);
    // the RAM and int8 tiers' slabs, once: a move takes a slot, never memory.
    // RAM holds at least the layers that start there (beyond the device slabs)
    const int ram_slots = std::max(std::min(cfg_.ram_layer_slots, cfg_.layers), cfg_.layers - cfg_.gpu_layer_slots);
    const int i8_slots = std::min(cfg_.int8_layer_slots, cfg_.layers);
    if (ok && ram_slots > 0 &&
        cudaHostAlloc((void **)&ram_arena_, slab_bytes_ * ram_slots, cudaHostAllocPortable) != cudaSuccess) {
        ram_arena_ = nullptr;
        ok = false;
    }
    if (ok && i8_slots > 0 &&
        (cudaMalloc((void **)&i8_codes_, slab_bytes_ / 2 * i8_slots) != cudaSuccess ||
         cudaMalloc((void **)&i8_stats_, blocks_per_slab_ * 16 * i8_slots) != cudaSuccess))
        ok = false;
    free_host_.clear();
    free_i8_.clear();
    for (int i = ram_slots - 1; i >= 0; --i) free_host_.push_back(i);
    for (int i = i8_slots - 1; i >= 0; --i) free_i8_.push_back(i);
    // Load the move kernels now: a kernel's first launch loads its code,
    // which can wait for every kernel running on the device, so the first
    // compressKv during a decode step would otherwise wait for the whole
    // step.  One zero block of the zero-filled arena, round trip in place.
    if (ok && i8_slots > 0)
        ok = kvx_compress_int8(arena_, KVX_F16, i8_codes_, i8_stats_, 1, 2048, move_) == KVX_OK &&
             kvx_decompress_int8(i8_codes_, i8_stats_, arena_, KVX_F16, 1, 2048, move_) == KVX_OK &&
             cudaStreamSynchronize(move_) == cudaSuccess;
    const size_t qn = (size_t)cfg_.layers * cfg_.max_batch * cfg_.q_heads * 128;
    const size_t kn = (size_t)cfg_.layers * cfg_.max_batch * cfg_.kv_heads * 128;
    // q / out also carry one layer of fp32 rows for decode_layer_f32
    const size_t qbytes = std::max(qn * 2, (size_t)cfg_.max_batch * cfg_.q_heads * 128 * 4);
    ok = ok && cudaMalloc(&d_q_, qbytes) == cudaSuccess && cudaMalloc(&d_out_, qbytes) == cudaSuccess &&
         cudaMalloc(&d_k_, kn * 2) == cudaSuccess && cudaMalloc(&d_v_, kn * 2) == cudaSuccess &&
         cudaMalloc(&d_pos_, cfg_.max_batch * sizeof(int32_t)) == cudaSuccess &&
         cudaMalloc(&d_err_, sizeof(int32_t)) == cudaSuccess && cudaMemset(d_err_, 0, 4) == cudaSuccess &&
         cudaHostAlloc(&h_pos_, cfg_.max_batch * sizeof(int32_t), cudaHostAllocDefault) == cudaSuccess;
    if (ok && ensure_staging() != KVX_OK) cudaGetLastError();  // else made on the first file move
    ev_in_.assign(cfg_.layers, nullptr);
    ev_out_.assign(cfg_.layers, nullptr);
    for (int l = 0; ok && l < cfg_.layers; ++l)
        ok = cudaEventCreateWithFlags(&ev_in_[l], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&ev_out_[l], cudaEventDisableTiming) == cudaSuccess;
    device_bytes_ = (long long)(slab_bytes_ * cfg_.gpu_layer_slots + 2 * qn * 2 + 2 * kn * 2 +
                                (slab_bytes_ / 2 + blocks_per_slab_ * 16) * i8_slots);
    layers_.assign(cfg_.layers, Layer{});
    free_slabs_.clear();
    for (int i = cfg_.gpu_layer_slots - 1; i >= 0; --i) free_slabs_.push_back(i);
    for (int l = 0; ok && l < cfg_.layers; ++l) {
        if (l < cfg_.gpu_layer_slots) {
            layers_[l].tier = kGpu;
            layers_[l].slab = free_slabs_.back();
            free_slabs_.pop_back();
        } else {  // beyond the device budget: starts in RAM, zero-filled
            layers_[l].tier = kRam;
            layers_[l].host_slot = take_host();
            ok = layers_[l].host_slot >= 0;
            if (ok) memset(host_ptr(layers_[l].host_slot), 0, slab_bytes_);
        }
    }
    free_pages_.clear();
    for (int pg = cfg_.pages_per_layer - 1; pg >= 0; --pg) free_pages_.push_back(pg);
    batch_ = 0;
    max_pages_ = 0;
    clock_ = 0;
    current_layer_ = 0;
    t0_ms_ = now_ms();  // every layer's last access: 0 on the engine clock
    if (!ok) {
        fprintf(stderr, "[adaptive_engine] start(): device allocation failed\n");
        release_all();
        return;
    }
    started_ = true;
}

void Engine::release_all() {
    if (compute_) cudaStreamSynchronize(compute_);
    if (copy_) cudaStreamSynchronize(copy_);
    if (comm_stream_) cudaStreamSynchronize(comm_stream_);
    if (comm_) nccl().comm_destroy(static_cast<ncclComm_t>(comm_));
    comm_ = nullptr;
    world_ = 1;
    rank_ = 0;
    readback_share_ = false;
    for (auto &e : ev_gath_) if (e) cudaEventDestroy(e);
    ev_gath_.clear();
    if (d_gather_) cudaFree(d_gather_);
    d_gather_ = nullptr;
    if (d_status_) cudaFree(d_status_);
    d_status_ = nullptr;
    if (h_status_) cudaFreeHost(h_status_);
    h_status_ = nullptr;
    if (comm_stream_) cudaStreamDestroy(comm_stream_);
    comm_stream_ = nullptr;
    if (move_) cudaStreamSynchronize(move_);
    for (size_t l = 0; l < layers_.size(); ++l) {
        Layer &L = layers_[l];
        if (L.tier == kOffloaded) remove(offload_path((int)l).c_str());
        L = Layer{};
    }
    if (ram_arena_) cudaFreeHost(ram_arena_);
    ram_arena_ = nullptr;
    if (i8_codes_) cudaFree(i8_codes_);
    if (i8_stats_) cudaFree(i8_stats_);
    i8_codes_ = nullptr;
    i8_stats_ = nullptr;
    free_host_.clear();
    free_i8_.clear();
    layers_.clear();
    for (auto &e : ev_in_) if (e) cudaEventDestroy(e);
    for (auto &e : ev_out_) if (e) cudaEventDestroy(e);
    ev_in_.clear();
    ev_out_.clear();
    auto free_dev = [](auto *&p) {
        if (p) cudaFree((void *)p);
        p = nullptr;
    };
    free_dev(arena_);
    free_dev(d_q_);
    free_dev(d_k_);
    free_dev(d_v_);
    free_dev(d_out_);
    free_dev(d_table_);
    free_dev(d_pos_);
    free_dev(d_err_);
    if (d_ws_) cudaFree(d_ws_);
    d_ws_ = nullptr;
    if (h_pos_) cudaFreeHost(h_pos_);
    h_pos_ = nullptr;
    for (int b = 0; b < 2; ++b) {
        if (stage_[b]) cudaFreeHost(stage_[b]);
        if (stage_ev_[b]) cudaEventDestroy(stage_ev_[b]);
        stage_[b] = nullptr;
        stage_ev_[b] = nullptr;
    }
    if (compute_) cudaStreamDestroy(compute_);
    if (copy_) cudaStreamDestroy(copy_);
    if (move_) cudaStreamDestroy(move_);
    compute_ = copy_ = move_ = nullptr;
    free_slabs_.clear();
    device_bytes_ = 0;
    batch_ = 0;
}

void Engine::stop() {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !step_active_ && !any_moving(); });
    if (!started_) return;
    release_all();
    started_ = false;
    cv_.notify_all();
}

bool Engine::valid(long layer) const {
    return started_ && layer >= 0 && layer < (long)layers_.size();
}

long Engine::ms_since(double t0) const {
    const double ms = now_ms() - t0;
    return std::max(1l, (long)std::ceil(ms));  // work was done: at least 1 ms, as callers test > 0
}

std::string Engine::offload_path(int l) const {
    return std::string(cfg_.offload_dir) + "/adaptive_kv_layer_" + std::to_string(l) + ".bin";
}

int Engine::take_host() {
    if (free_host_.empty()) return -1;
    const int s = free_host_.back();
    free_host_.pop_back();
    return s;
}

int Engine::take_i8() {
    if (free_i8_.empty()) return -1;
    const int s = free_i8_.back();
    free_i8_.pop_back();
    return s;
}

bool Engine::any_moving() const {
    for (const Layer &L : layers_)
        if (L.moving) return true;
    return false;
}

void Engine::wait_not_moving(std::unique_lock<std::mutex> &lk, int l) {
    cv_.wait(lk, [&] { return !started_ || l >= (int)layers_.size() || !layers_[l].moving; });
}

// A free device slab for layer `for_layer`, evicting the least recently used
// GPU-resident layer to RAM when none is free (KVCacheGPU::transferToGPU's
// evict-then-retry, native-engine/cpp/KVCacheGPU.cpp:68-109).  The victim is
// the smallest last_used stamp, the lowest layer index on ties
// (KVCacheGPU::findLRUPage, KVCacheGPU.cpp:54-66); pinned layers are skipped.
int Engine::alloc_slab(int for_layer) {
    if (!free_slabs_.empty()) {
        const int s = free_slabs_.back();
        free_slabs_.pop_back();
        return s;
    }
    const int victim = pick_victim(for_layer);
    if (victim < 0) return victim;
    if (to_ram_locked(victim) < 0) return -1;
    const int s = free_slabs_.back();
    free_slabs_.pop_back();
    return s;
}

// The least recently used GPU-resident layer other than `for_layer`
// (smallest last_used, lowest index on ties, KVCacheGPU::findLRUPage,
// native-engine/cpp/KVCacheGPU.cpp:54-66), skipping pinned layers and
// layers being moved; -2 when only pinned ones are left.
int Engine::pick_victim(int for_layer) const {
    int victim = -1;
    uint64_t best = UINT64_MAX;
    bool any_pinned = false;
    for (int l = 0; l < (int)layers_.size(); ++l) {
        const Layer &L = layers_[l];
        if (l == for_layer || L.tier != kGpu || L.moving) continue;
        if (L.refcount > 0) {
            any_pinned = true;
            continue;
        }
        if (L.last_used < best) {
            best = L.last_used;
            victim = l;
        }
    }
    return victim >= 0 ? victim : (any_pinned ? -2 : -1);
}

int Engine::ensure_staging() {
    for (int b = 0; b < 2; ++b) {
        if (!stage_[b] && cudaHostAlloc(&stage_[b], kStageBytes, cudaHostAllocDefault) != cudaSuccess) {
            stage_[b] = nullptr;
            return KVX_ENOSPC;
        }
        if (!stage_ev_[b] && cudaEventCreateWithFlags(&stage_ev_[b], cudaEventDisableTiming) != cudaSuccess) {
            stage_ev_[b] = nullptr;
            return KVX_ECUDA;
        }
    }
    return KVX_OK;
}

// A layer's page file straight to device memory: 64 MiB pieces read into
// one pinned buffer while the other one's copy runs.  No host copy of the
// whole layer is pinned for it (pinning 0.6 GB took ~240 ms on its own).
int Engine::file_to_device(int l, uint8_t *dst) {
    if (ensure_staging() != KVX_OK) return KVX_ENOSPC;
    FILE *f = fopen(offload_path(l).c_str(), "rb");
    if (!f) return KVX_EINVAL;
    int rc = KVX_OK;
    bool pending[2] = {false, false};
    size_t off = 0;
    for (int b = 0; off < slab_bytes_; b ^= 1) {
        const size_t n = std::min(kStageBytes, slab_bytes_ - off);
        if (pending[b] && cudaEventSynchronize(stage_ev_[b]) != cudaSuccess) {
            rc = KVX_ECUDA;
            break;
        }
        if (fread(stage_[b], 1, n, f) != n) {
            rc = KVX_EINVAL;
            break;
        }
        if (cudaMemcpyAsync(dst + off, stage_[b], n, cudaMemcpyHostToDevice, copy_) != cudaSuccess ||
            cudaEventRecord(stage_ev_[b], copy_) != cudaSuccess) {
            rc = KVX_ECUDA;
            break;
        }
        pending[b] = true;
        off += n;
    }
    fclose(f);
    if (cudaStreamSynchronize(copy_) != cudaSuccess && rc == KVX_OK) rc = KVX_ECUDA;
    return rc;
}

// Device memory to the layer's page file, the same way round: one piece's
// copy runs while the previous one is written.
int Engine::device_to_file(int l, const uint8_t *src) {
    if (ensure_staging() != KVX_OK) return KVX_ENOSPC;
    FILE *f = fopen(offload_path(l).c_str(), "wb");
    if (!f) return KVX_EINVAL;
    int rc = KVX_OK;
    size_t n_prev = 0, off = 0;
    int b = 0;
    while (rc == KVX_OK && (off < slab_bytes_ || n_prev)) {
        const size_t n = std::min(kStageBytes, slab_bytes_ - off);
        if (n && (cudaMemcpyAsync(stage_[b], src + off, n, cudaMemcpyDeviceToHost, copy_) != cudaSuccess ||
                  cudaEventRecord(stage_ev_[b], copy_) != cudaSuccess))
            rc = KVX_ECUDA;
        if (rc == KVX_OK && n_prev) {  // the previous piece: wait for it, write it
            if (cudaEventSynchronize(stage_ev_[b ^ 1]) != cudaSuccess)
                rc = KVX_ECUDA;
            else if (fwrite(stage_[b ^ 1], 1, n_prev, f) != n_prev)
                rc = KVX_EINVAL;
        }
        n_prev = n;
        off += n;
        b ^= 1;
    }
    if (fclose(f) != 0 && rc == KVX_OK) rc = KVX_EINVAL;
    if (cudaStreamSynchronize(copy_) != cudaSuccess && rc == KVX_OK) rc = KVX_ECUDA;
    return rc;
}

// Locked moves: the decode step's own tiered path (its victims may still be
// read by its kernels, hence the compute-stream sync) and the file paths.
int Engine::to_ram_locked(int l) {
    Layer &L = layers_[l];
    if (L.tier == kRam) return 0;
    if (L.tier == kOffloaded) {
        const int hs = take_host();
        if (hs < 0) return KVX_ENOSPC;
        FILE *f = fopen(offload_path(l).c_str(), "rb");
        const bool ok = f && fread(host_ptr(hs), 1, slab_bytes_, f) == slab_bytes_;
        if (f) fclose(f);
        if (!ok) {
            free_host_.push_back(hs);
            return KVX_EINVAL;
        }
        remove(offload_path(l).c_str());
        L.host_slot = hs;
        L.tier = kRam;
        return 1;
    }
    if (is_compressed(L.tier)) {  // decompress into a slab first
        const int rc = to_gpu_locked(l);
        if (rc < 0) return rc;
    }
    const int hs = take_host();
    if (hs < 0) return KVX_ENOSPC;
    cudaStreamSynchronize(compute_);
    if (cudaMemcpyAsync(host_ptr(hs), slab_ptr(L.slab), slab_bytes_, cudaMemcpyDeviceToHost, copy_) != cudaSuccess ||
        cudaStreamSynchronize(copy_) != cudaSuccess) {
        free_host_.push_back(hs);
        return KVX_ECUDA;
    }
    free_slabs_.push_back(L.slab);
    L.slab = -1;
    L.host_slot = hs;
    L.tier = kRam;
    L.last_use = nullptr;
    return 1;
}

int Engine::to_gpu_locked(int l) {
    Layer &L = layers_[l];
    L.last_used = ++clock_;
    if (L.tier == kGpu) return 0;
    const int s = alloc_slab(l);
    if (s == -2) return KVX_EBUSY;
    if (s < 0) return KVX_ENOSPC;
    uint8_t *dst = slab_ptr(s);
    int rc = KVX_OK;
    if (is_compressed(L.tier)) {
        rc = decompress_into(L, dst, copy_);
    } else if (L.tier == kOffloaded) {
        rc = file_to_device(l, dst);
    } else if (cudaMemcpyAsync(dst, host_ptr(L.host_slot), slab_bytes_, cudaMemcpyHostToDevice, copy_) != cudaSuccess) {
        rc = KVX_ECUDA;
    }
    if (!rc && cudaStreamSynchronize(copy_) != cudaSuccess) rc = KVX_ECUDA;
    if (rc) {
        free_slabs_.push_back(s);
        return rc;
    }
    if (is_compressed(L.tier)) {
        free_i8_.push_back(L.i8_slot);
        L.i8_slot = -1;
    } else if (L.tier == kOffloaded) {
        remove(offload_path(l).c_str());
    } else {
        free_host_.push_back(L.host_slot);
        L.host_slot = -1;
    }
    L.slab = s;
    L.tier = kGpu;
    L.last_use = nullptr;
    return 1;
}

int Engine::offload_locked(int l) {
    Layer &L = layers_[l];
    if (L.tier == kOffloaded) return 0;
    if (is_compressed(L.tier)) {
        const int rc = to_gpu_locked(l);
        if (rc < 0) return rc;
    }
    if (L.tier == kGpu) {  // device -> file, then the slab is free
        if (L.last_use && cudaEventSynchronize(L.last_use) != cudaSuccess) return KVX_ECUDA;
        const int rc = device_to_file(l, slab_ptr(L.slab));
        if (rc != KVX_OK) return rc;
        free_slabs_.push_back(L.slab);
        L.slab = -1;
    } else {
        FILE *f = fopen(offload_path(l).c_str(), "wb");
        const bool ok = f && fwrite(host_ptr(L.host_slot), 1, slab_bytes_, f) == slab_bytes_;
        if (f) fclose(f);
        if (!ok) return KVX_EINVAL;
        free_host_.push_back(L.host_slot);
        L.host_slot = -1;
    }
    L.tier = kOffloaded;
    L.last_use = nullptr;
    return 1;
}

// Moves whose copies run with the mutex released.  Under the mutex the
// layer (and an eviction victim) is marked `moving`, arena slots are taken
// and the copies queued on move_ behind each layer's last decode work (the
// group event of the step that last read it; nothing else touches its
// slab); the mutex is released while move_ drains, then retaken to commit
// the new tiers.  A running decode step keeps going meanwhile, and so do
// moves of other layers.  layers_ is not resized while a layer is moving
// (stop() waits), so indices stay valid across the unlocked part.
int Engine::gpu_to_ram(std::unique_lock<std::mutex> &lk, int l) {
    const int hs = take_host();
    if (hs < 0) return KVX_ENOSPC;
    layers_[l].moving = true;
    int rc = KVX_OK;
    {
        const Layer &L = layers_[l];
        if ((L.last_use && cudaStreamWaitEvent(move_, L.last_use, 0) != cudaSuccess) ||
            cudaMemcpyAsync(host_ptr(hs), slab_ptr(L.slab), slab_bytes_, cudaMemcpyDeviceToHost, move_) != cudaSuccess)
            rc = KVX_ECUDA;
    }
    lk.unlock();
    if (cudaStreamSynchronize(move_) != cudaSuccess && rc == KVX_OK) rc = KVX_ECUDA;
    lk.lock();
    Layer &L = layers_[l];
    L.moving = false;
    if (rc == KVX_OK) {
        free_slabs_.push_back(L.slab);
        L.slab = -1;
        L.host_slot = hs;
        L.tier = kRam;
        L.last_use = nullptr;
    } else {
        free_host_.push_back(hs);
    }
    cv_.notify_all();
    return rc == KVX_OK ? 1 : rc;
}

int Engine::bring_to_gpu(std::unique_lock<std::mutex> &lk, int l) {
    layers_[l].last_used = ++clock_;
    if (layers_[l].tier == kGpu) return 0;
    if (layers_[l].tier == kOffloaded) return to_gpu_locked(l);  // file reads stay under the mutex
    int s = -1, victim = -1, vhs = -1;
    if (!free_slabs_.empty()) {
        s = free_slabs_.back();
        free_slabs_.pop_back();
    } else {  // the least recently used layer goes to RAM first (KVCacheGPU.cpp:68-109)
        victim = pick_victim(l);
        if (victim == -2) return KVX_EBUSY;
        if (victim < 0) return KVX_ENOSPC;
        vhs = take_host();
        if (vhs < 0) return KVX_ENOSPC;
        s = layers_[victim].slab;
        layers_[victim].moving = true;
    }
    layers_[l].moving = true;
    int rc_victim = KVX_OK, rc = KVX_OK;
    if (victim >= 0) {
        const Layer &V = layers_[victim];
        if ((V.last_use && cudaStreamWaitEvent(move_, V.last_use, 0) != cudaSuccess) ||
            cudaMemcpyAsync(host_ptr(vhs), slab_ptr(s), slab_bytes_, cudaMemcpyDeviceToHost, move_) != cudaSuccess)
            rc_victim = rc = KVX_ECUDA;
    }
    if (rc == KVX_OK) {
        const Layer &L = layers_[l];
        if (is_compressed(L.tier))
            rc = decompress_into(L, slab_ptr(s), move_);
        else if (cudaMemcpyAsync(slab_ptr(s), host_ptr(L.host_slot), slab_bytes_, cudaMemcpyHostToDevice, move_) !=
                 cudaSuccess)
            rc = KVX_ECUDA;
    }
    lk.unlock();
    if (cudaStreamSynchronize(move_) != cudaSuccess) {
        if (rc == KVX_OK) rc = KVX_ECUDA;
        rc_victim = rc;
    }
    lk.lock();
    Layer &L = layers_[l];
    L.moving = false;
    if (victim >= 0) {
        Layer &V = layers_[victim];
        V.moving = false;
        if (rc_victim == KVX_OK) {  // its bytes are in RAM: the slab is the target's (or free again)
            V.slab = -1;
            V.host_slot = vhs;
            V.tier = kRam;
            V.last_use = nullptr;
        } else {
            free_host_.push_back(vhs);
            s = -1;  // the victim keeps its slab
        }
    }
    if (rc != KVX_OK) {
        if (s >= 0) free_slabs_.push_back(s);
        cv_.notify_all();
        return rc;
    }
    if (is_compressed(L.tier)) {
        free_i8_.push_back(L.i8_slot);
        L.i8_slot = -1;
    } else {
        free_host_.push_back(L.host_slot);
        L.host_slot = -1;
    }
    L.slab = s;
    L.tier = kGpu;
    L.last_use = nullptr;
    cv_.notify_all();
    return 1;
}

int Engine::decompress_into(const Layer &L, uint8_t *dst, cudaStream_t st) {
    return L.tier == kCompressedNf4
               ? kvx_decompress_nf4(reinterpret_cast<const uint8_t *>(codes_ptr(L.i8_slot)), stats_ptr(L.i8_slot), dst,
                                    KVX_F16, blocks_per_slab_, 2048, st)
               : kvx_decompress_int8(codes_ptr(L.i8_slot), stats_ptr(L.i8_slot), dst, KVX_F16, blocks_per_slab_, 2048,
                                     st);
}

// Compress a GPU layer into a compressed-arena slot: int8 (compressKv) or
// NF4 (4-bit codes, half of the slot; the age policy's heavy compression).
int Engine::gpu_to_int8(std::unique_lock<std::mutex> &lk, int l, bool nf4) {
    const int is = take_i8();
    if (is < 0) return KVX_ENOSPC;
    layers_[l].moving = true;
    int rc = KVX_OK;
    {
        const Layer &L = layers_[l];
        if (L.last_use && cudaStreamWaitEvent(move_, L.last_use, 0) != cudaSuccess) rc = KVX_ECUDA;
        if (rc == KVX_OK)
            rc = nf4 ? kvx_compress_nf4(slab_ptr(L.slab), KVX_F16, reinterpret_cast<uint8_t *>(codes_ptr(is)),
                                        stats_ptr(is), blocks_per_slab_, 2048, move_)
                     : kvx_compress_int8(slab_ptr(L.slab), KVX_F16, codes_ptr(is), stats_ptr(is), blocks_per_slab_,
                                         2048, move_);
    }
    lk.unlock();
    if (cudaStreamSynchronize(move_) != cudaSuccess && rc == KVX_OK) rc = KVX_ECUDA;
    lk.lock();
    Layer &L = layers_[l];
    L.moving = false;
    if (rc == KVX_OK) {
        free_slabs_.push_back(L.slab);
        L.slab = -1;
        L.i8_slot = is;
        L.tier = nf4 ? kCompressedNf4 : kCompressed;
        L.last_use = nullptr;
    } else {
        free_i8_.push_back(is);
    }
    cv_.notify_all();
    return rc == KVX_OK ? 1 : rc;
}

// ---- NativeEngineApi operations ------------------------------------------

long Engine::move_to_ram(long layer) {
    const double t0 = now_ms();
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, (int)layer);
    if (!valid(layer)) return -1;
    if (layers_[layer].refcount > 0 && layers_[layer].tier != kRam) return -2;
    const int rc = layers_[layer].tier == kGpu ? gpu_to_ram(lk, (int)layer) : to_ram_locked((int)layer);
    return rc < 0 ? (rc == KVX_EBUSY ? -2 : -1) : ms_since(t0);
}

long Engine::move_to_gpu(long layer) {
    const double t0 = now_ms();
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, (int)layer);
    if (!valid(layer)) return -1;
    const int rc = bring_to_gpu(lk, (int)layer);
    return rc < 0 ? (rc == KVX_EBUSY ? -2 : -1) : ms_since(t0);
}

long Engine::compress(long layer) {
    const double t0 = now_ms();
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, (int)layer);
    if (!valid(layer)) return -1;
    if (layers_[layer].refcount > 0 && !is_compressed(layers_[layer].tier)) return -2;
    if (is_compressed(layers_[layer].tier)) return 0;
    int rc = KVX_OK;
    if (layers_[layer].tier != kGpu) rc = bring_to_gpu(lk, (int)layer);
    if (rc >= 0) rc = gpu_to_int8(lk, (int)layer);
    return rc < 0 ? (rc == KVX_EBUSY ? -2 : -1) : ms_since(t0);
}

long Engine::offload(long layer) {
    const double t0 = now_ms();
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, (int)layer);
    if (!valid(layer)) return -1;
    if (layers_[layer].refcount > 0 && layers_[layer].tier != kOffloaded) return -2;
    const int rc = offload_locked((int)layer);
    if (rc > 0) layers_[layer].cached = false;
    return rc < 0 ? (rc == KVX_EBUSY ? -2 : -1) : ms_since(t0);
}

// Layer-cache bitmap with pins (llama_wrapper.cpp:171-219), tied to KV
// residency: a cached layer has its KV on the device.
long Engine::prefetch_layer(int layer) {
    const double t0 = now_ms();
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, layer);
    if (!valid(layer)) return -1;
    if (layers_[layer].cached) return 0;
    const int rc = bring_to_gpu(lk, layer);
    if (rc < 0) return rc == KVX_EBUSY ? -2 : -1;
    layers_[layer].cached = true;
    return ms_since(t0);
}

long Engine::evict_layer(int layer) {
    const double t0 = now_ms();
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, layer);
    if (!valid(layer)) return -1;
    if (!layers_[layer].cached) return 0;
    if (layers_[layer].refcount > 0) return -2;
    const int rc = layers_[layer].tier == kGpu ? gpu_to_ram(lk, layer) : to_ram_locked(layer);
    if (rc < 0) return -1;
    layers_[layer].cached = false;
    return ms_since(t0);
}

long Engine::keep_layer(int layer) {
    std::unique_lock<std::mutex> lk(mu_);
    if (!valid(layer)) return -1;
    wait_not_moving(lk, layer);
    if (!valid(layer)) return -1;
    if (!layers_[layer].cached) {
        const int rc = bring_to_gpu(lk, layer);
        if (rc < 0) return rc == KVX_EBUSY ? -2 : -1;
        layers_[layer].cached = true;
    }
    return ++layers_[layer].refcount;
}

void Engine::release_layer(int layer) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!valid(layer)) return;
    if (layers_[layer].refcount > 0) --layers_[layer].refcount;
}

int Engine::current_layer() {
    std::lock_guard<std::mutex> lk(mu_);
    return current_layer_;
}

long Engine::gpu_memory() {
    std::lock_guard<std::mutex> lk(mu_);
    return (long)device_bytes_;
}

int Engine::kv_pages() {
    std::lock_guard<std::mutex> lk(mu_);
    return started_ ? (int)layers_.size() : (configured_ ? cfg_.layers : 0);
}

int Engine::cached_layers() {
    std::lock_guard<std::mutex> lk(mu_);
    int n = 0;
    for (const Layer &L : layers_) n += L.cached ? 1 : 0;
    return n;
}

int Engine::layer_view(int layer, kvx_paged *view) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!view || !valid(layer) || layers_[layer].tier != kGpu) return KVX_EINVAL;
    view->pool = arena_ + (size_t)layers_[layer].slab * slab_bytes_;
    view->stats = nullptr;
    view->dtype = KVX_F16;
    view->num_pages = cfg_.pages_per_layer;
    view->num_kv_heads = cfg_.kv_heads;
    view->head_dim = 128;
    view->page_tokens = 16;
    return KVX_OK;
}

int Engine::layer_tier(int layer) {
    std::lock_guard<std::mutex> lk(mu_);
    return valid(layer) ? (int)layers_[layer].tier : -1;
}

long long Engine::device_bytes() {
    std::lock_guard<std::mutex> lk(mu_);
    return device_bytes_;
}

int32_t Engine::seq_len(int s) {
    std::lock_guard<std::mutex> lk(mu_);
    return (s >= 0 && s < batch_) ? lens_[s] : -1;
}

int Engine::copy_layer(int layer, void *ptr, bool load) {
    std::unique_lock<std::mutex> lk(mu_);
    if (!ptr || !valid(layer)) return KVX_EINVAL;
    cv_.wait(lk, [&] { return !started_ || (!step_active_ && !layers_[layer].moving); });
    if (!valid(layer)) return KVX_EINVAL;
    const int rc = to_gpu_locked(layer);
    if (rc < 0) return rc;
    cudaStreamSynchronize(compute_);
    uint8_t *slab = arena_ + (size_t)layers_[layer].slab * slab_bytes_;
    const cudaError_t e = load ? cudaMemcpy(slab, ptr, slab_bytes_, cudaMemcpyDefault)
                               : cudaMemcpy(ptr, slab, slab_bytes_, cudaMemcpyDefault);
    if (load) layers_[layer].last_access_ms = clock_ms();  // a write is an access
    return e == cudaSuccess ? KVX_OK : KVX_ECUDA;
}

int32_t Engine::block_table(int32_t *dst) {
    std::lock_guard<std::mutex> lk(mu_);
    if (dst) std::copy(table_.begin(), table_.end(), dst);
    return max_pages_;
}

// ---- sequences and the decode step ---------------------------------------

int Engine::set_sequences(int batch, const int32_t *lens, int reserve_tokens, uint64_t seed) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !step_active_; });
    if (!started_ || batch <= 0 || batch > cfg_.max_batch || !lens || reserve_tokens < 0) return KVX_EINVAL;
    cudaStreamSynchronize(compute_);
    // every physical page back into the free list, then hand them out
    std::vector<int32_t> order(cfg_.pages_per_layer);
    for (int i = 0; i < cfg_.pages_per_layer; ++i) order[i] = i;
    if (seed) {  // Fisher-Yates with splitmix64: fragmented page tables
        uint64_t st = seed;
        for (int i = cfg_.pages_per_layer - 1; i > 0; --i) std::swap(order[i], order[splitmix(st) % (uint64_t)(i + 1)]);
    }
    int max_pages = 1;
    long long need = 0;
    for (int s = 0; s < batch; ++s) {
        if (lens[s] < 0) return KVX_EINVAL;
        const int np = (lens[s] + reserve_tokens + 15) / 16;
        max_pages = std::max(max_pages, np);
        need += np;
    }
    if (need > cfg_.pages_per_layer) return KVX_ENOSPC;
    table_.assign((size_t)batch * max_pages, -1);
    size_t next = 0;
    for (int s = 0; s < batch; ++s) {
        const int np = (lens[s] + reserve_tokens + 15) / 16;
        for (int j = 0; j < np; ++j) table_[(size_t)s * max_pages + j] = order[next++];
    }
    free_pages_.assign(order.begin() + next, order.end());
    if (d_table_) cudaFree(d_table_);
    d_table_ = nullptr;
    if (d_ws_) cudaFree(d_ws_);
    d_ws_ = nullptr;
    ws_bytes_ = kvx_decode_workspace_bytes(batch, cfg_.q_heads, max_pages, 16);
    if (cudaMalloc(&d_table_, table_.size() * sizeof(int32_t)) != cudaSuccess ||
        cudaMalloc(&d_ws_, ws_bytes_) != cudaSuccess ||
        cudaMemcpy(d_table_, table_.data(), table_.size() * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess ||
        kvx_decode_workspace_init(d_ws_, ws_bytes_, nullptr) != KVX_OK || cudaDeviceSynchronize() != cudaSuccess) {
        batch_ = 0;
        return KVX_ECUDA;
    }
    lens_.assign(lens, lens + batch);
    batch_ = batch;
    max_pages_ = max_pages;
    return KVX_OK;
}

int Engine::decode_step(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out) {
    std::unique_lock<std::mutex> lk(mu_);
    // one step at a time (they share the step buffers and the workspace),
    // and none while a layer is being moved
    cv_.wait(lk, [&] { return !step_active_ && !any_moving(); });
    if (!started_ || batch_ == 0 || !q || !k || !v) return KVX_EINVAL;
    for (int s = 0; s < batch_; ++s)  // every sequence needs a page for its next token
        if (lens_[s] / 16 >= max_pages_ || table_[(size_t)s * max_pages_ + lens_[s] / 16] < 0)
            return KVX_ENOSPC;
    const int L = cfg_.layers, B = batch_, hq = cfg_.q_heads, hkv = cfg_.kv_heads;
    const size_t qrow = (size_t)B * hq * 128, krow = (size_t)B * hkv * 128;  // elements per layer
    const size_t qstride = (size_t)cfg_.max_batch * hq * 128, kstride = (size_t)cfg_.max_batch * hkv * 128;
    // With a communicator every rank takes the same collective steps in the
    // same order whatever happens locally: a rank whose step fails launches
    // nothing more but still joins every group's all-gathers and the status
    // exchange at the end, so its peers finish the step and return
    // KVX_EPEER instead of waiting in NCCL.
    int rc = KVX_OK;
    memcpy(h_pos_, lens_.data(), B * sizeof(int32_t));
    if (cudaMemcpyAsync(d_pos_, h_pos_, B * sizeof(int32_t), cudaMemcpyHostToDevice, compute_) != cudaSuccess)
        rc = KVX_ECUDA;
    // Layers run in groups: one input copy event and one output event per
    // group, so within a group the decode launches follow each other with
    // nothing in between and each may start while the previous drains
    // (programmatic dependent launch); the groups' copies overlap the other
    // groups' kernels.
    // group starts: kEdgeGroup layers, the middle ones (in groups of
    // KVX_ENGINE_GROUP when set), the last kEdgeGroup alone
    int gstart[64];
    int ngroups = 0;
    gstart[ngroups++] = 0;
    if (L > 3 * kEdgeGroup) {
        const int mid = std::max(0, env_int("KVX_ENGINE_GROUP", comm_ ? kCommGroup : 0));
        int l = kEdgeGroup;
        gstart[ngroups++] = l;
        if (mid > 0)
            while (L - kEdgeGroup - l > mid && ngroups < 62) gstart[ngroups++] = (l += mid);
        gstart[ngroups++] = L - kEdgeGroup;
    }
    gstart[ngroups] = L;
    // with the batch at max_batch the layers are contiguous on both sides:
    // one copy per tensor per group instead of one per layer
    const bool packed = qstride == qrow && kstride == krow;
    for (int gi = 0; gi < ngroups && rc == KVX_OK; ++gi) {
        const int l0 = gstart[gi], l1 = gstart[gi + 1];
        if (packed) {
            const size_t n = (size_t)(l1 - l0);
            if (cudaMemcpyAsync(d_q_ + l0 * qstride, q + l0 * qrow, n * qrow * 2, cudaMemcpyHostToDevice, copy_) ||
                cudaMemcpyAsync(d_k_ + l0 * kstride, k + l0 * krow, n * krow * 2, cudaMemcpyHostToDevice, copy_) ||
                cudaMemcpyAsync(d_v_ + l0 * kstride, v + l0 * krow, n * krow * 2, cudaMemcpyHostToDevice, copy_))
                rc = KVX_ECUDA;
        } else {
            for (int l = l0; l < l1 && rc == KVX_OK; ++l)
                if (cudaMemcpyAsync(d_q_ + l * qstride, q + l * qrow, qrow * 2, cudaMemcpyHostToDevice, copy_) ||
                    cudaMemcpyAsync(d_k_ + l * kstride, k + l * krow, krow * 2, cudaMemcpyHostToDevice, copy_) ||
                    cudaMemcpyAsync(d_v_ + l * kstride, v + l * krow, krow * 2, cudaMemcpyHostToDevice, copy_))
                    rc = KVX_ECUDA;
        }
        if (rc == KVX_OK && cudaEventRecord(ev_in_[gi], copy_)) rc = KVX_ECUDA;
    }
    if (rc && !comm_) return rc;
    for (int gi = 0; gi < ngroups && (rc == KVX_OK || comm_); ++gi) {
        const int l0 = gstart[gi], l1 = gstart[gi + 1];
        if (rc == KVX_OK && cudaStreamWaitEvent(compute_, ev_in_[gi], 0) != cudaSuccess) rc = KVX_ECUDA;
        for (int l = l0; l < l1 && rc == KVX_OK; ++l) {
            if (layers_[l].tier != kGpu) {  // tiered: bring the layer back (may evict the LRU layer)
                const int r = to_gpu_locked(l);
                if (r < 0) {
                    rc = r;
                    break;
                }
            }
            layers_[l].last_used = ++clock_;
            layers_[l].last_access_ms = clock_ms();
            kvx_paged view{arena_ + (size_t)layers_[l].slab * slab_bytes_, nullptr, KVX_F16,
                           cfg_.pages_per_layer, hkv, 128, 16};
            rc = kvx_append_decode(&view, d_table_, max_pages_, d_pos_, B, d_k_ + l * kstride,
                                   d_v_ + l * kstride, hq, d_q_ + l * qstride, d_out_ + l * qstride,
                                   KVX_F16, 0.f, d_ws_, ws_bytes_, d_err_, compute_);
            current_layer_ = l;
        }
        // recorded after a failure too, so the gathers below never read rows
        // that a kernel still writes
        if (cudaEventRecord(ev_out_[gi], compute_) && rc == KVX_OK) rc = KVX_ECUDA;
        if (comm_) {  // all-gather the group's rows over NCCL, then read them back
            if (cudaStreamWaitEvent(comm_stream_, ev_out_[gi], 0) && rc == KVX_OK) rc = KVX_ECUDA;
            // packed: one all-gather per group, the group's block of d_gather_
            // is [world][layers][B][hq][128]; otherwise one per layer,
            // [world][B][hq][128] at the layer's place
            const int n = l1 - l0;
            uint16_t *gbase = d_gather_ + (size_t)l0 * world_ * qrow;
            if (packed) {
                if (nccl().all_gather(d_out_ + l0 * qstride, gbase, (size_t)n * qrow, ncclFloat16,
                                      static_cast<ncclComm_t>(comm_), comm_stream_) != ncclSuccess &&
                    rc == KVX_OK)
                    rc = KVX_ECUDA;
            } else {
                for (int l = l0; l < l1; ++l)
                    if (nccl().all_gather(d_out_ + l * qstride, d_gather_ + (size_t)l * world_ * qrow, qrow,
                                          ncclFloat16, static_cast<ncclComm_t>(comm_), comm_stream_) != ncclSuccess &&
                        rc == KVX_OK)
                        rc = KVX_ECUDA;
            }
            if (rc == KVX_OK && cudaEventRecord(ev_gath_[gi], comm_stream_)) rc = KVX_ECUDA;
            if (rc == KVX_OK && out && cudaStreamWaitEvent(copy_, ev_gath_[gi], 0)) rc = KVX_ECUDA;
            // host layout [layers][world][B][hq][128]; with the read-back
            // shared, rank r copies the layers l % world == r
            const size_t row = qrow * 2;  // bytes of one (layer, rank) block
            if (rc == KVX_OK && out && packed && !readback_share_ && world_ <= n) {
                for (int r = 0; r < world_ && rc == KVX_OK; ++r)  // rank r's block of every layer
                    if (cudaMemcpy2DAsync(out + ((size_t)l0 * world_ + r) * qrow, world_ * row, gbase + (size_t)r * n * qrow,
                                          row, row, n, cudaMemcpyDeviceToHost, copy_))
                        rc = KVX_ECUDA;
            } else if (rc == KVX_OK && out) {
                for (int l = l0; l < l1 && rc == KVX_OK; ++l) {
                    if (readback_share_ && l % world_ != rank_) continue;
                    const cudaError_t e =
                        packed ? cudaMemcpy2DAsync(out + (size_t)l * world_ * qrow, row, gbase + (size_t)(l - l0) * qrow,
                                                   n * row, row, world_, cudaMemcpyDeviceToHost, copy_)
                               : cudaMemcpyAsync(out + (size_t)l * world_ * qrow, d_gather_ + (size_t)l * world_ * qrow,
                                                 world_ * row, cudaMemcpyDeviceToHost, copy_);
                    if (e) rc = KVX_ECUDA;
                }
            }
        } else if (rc == KVX_OK && out) {
            if (cudaStreamWaitEvent(copy_, ev_out_[gi], 0)) rc = KVX_ECUDA;
            if (packed) {
                if (rc == KVX_OK && cudaMemcpyAsync(out + l0 * qrow, d_out_ + l0 * qstride, (size_t)(l1 - l0) * qrow * 2,
                                                    cudaMemcpyDeviceToHost, copy_))
                    rc = KVX_ECUDA;
            } else {
                for (int l = l0; l < l1 && rc == KVX_OK; ++l)
                    if (cudaMemcpyAsync(out + l * qrow, d_out_ + l * qstride, qrow * 2, cudaMemcpyDeviceToHost, copy_))
                        rc = KVX_ECUDA;
            }
        }
    }
    // Status exchange: {host status, device error flag} of every rank,
    // gathered after the last group's kernels, read with the same sync.
    bool peer_failed = false;
    if (comm_) {
        h_status_[0] = rc;
        if ((cudaStreamWaitEvent(comm_stream_, ev_out_[ngroups - 1], 0) ||
             cudaMemcpyAsync(d_status_, h_status_, sizeof(int32_t), cudaMemcpyHostToDevice, comm_stream_) ||
             cudaMemcpyAsync(d_status_ + 1, d_err_, sizeof(int32_t), cudaMemcpyDeviceToDevice, comm_stream_)) &&
            rc == KVX_OK)
            rc = KVX_ECUDA;
        if (nccl().all_gather(d_status_, d_status_ + 2, 2, ncclInt32, static_cast<ncclComm_t>(comm_),
                              comm_stream_) != ncclSuccess &&
            rc == KVX_OK)
            rc = KVX_ECUDA;
        if (cudaMemcpyAsync(h_status_ + 2, d_status_ + 2, 2 * world_ * sizeof(int32_t), cudaMemcpyDeviceToHost,
                            comm_stream_) &&
            rc == KVX_OK)
            rc = KVX_ECUDA;
    }
    // each layer's last decode work is its group's output event: a move of
    // that layer waits for it, not for the whole step
    for (int gi = 0; gi < ngroups; ++gi)
        for (int l = gstart[gi]; l < gstart[gi + 1]; ++l) layers_[l].last_use = ev_out_[gi];
    // wait for the device with the mutex released, so layer moves proceed
    step_active_ = true;
    lk.unlock();
    int32_t err = 0;
    const bool synced = cudaStreamSynchronize(compute_) == cudaSuccess &&
                        cudaStreamSynchronize(copy_) == cudaSuccess &&
                        (!comm_stream_ || cudaStreamSynchronize(comm_stream_) == cudaSuccess) &&
                        cudaMemcpy(&err, d_err_, sizeof(err), cudaMemcpyDeviceToHost) == cudaSuccess;
    lk.lock();
    step_active_ = false;
    cv_.notify_all();
    if (!synced) return KVX_ECUDA;
    if (comm_)
        for (int r = 0; r < world_; ++r)
            if (r != rank_ && (h_status_[2 + 2 * r] != KVX_OK || h_status_[3 + 2 * r] != 0)) peer_failed = true;
    if (err) cudaMemset(d_err_, 0, sizeof(int32_t));
    if (rc) return rc;
    if (err) return (err & 1) ? KVX_ETIMEOUT : KVX_EINVAL;
    if (peer_failed) return KVX_EPEER;
    for (int s = 0; s < B; ++s) ++lens_[s];
    return KVX_OK;
}

int Engine::decode_layer_f32(int layer, const float *q, const float *k, const float *v, float *out) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !step_active_ && !any_moving(); });
    if (!valid(layer) || batch_ == 0 || !q || !k || !v || !out) return KVX_EINVAL;
    for (int s = 0; s < batch_; ++s)
        if (lens_[s] / 16 >= max_pages_ || table_[(size_t)s * max_pages_ + lens_[s] / 16] < 0)
            return KVX_ENOSPC;
    const int B = batch_, hq = cfg_.q_heads, hkv = cfg_.kv_heads;
    const size_t qn = (size_t)B * hq * 128, kn = (size_t)B * hkv * 128;
    std::vector<_Float16> k16(kn), v16(kn);  // round to nearest, as the pool stores it
    for (size_t i = 0; i < kn; ++i) {
        k16[i] = (_Float16)k[i];
        v16[i] = (_Float16)v[i];
    }
    if (layers_[layer].tier != kGpu) {
        const int r = to_gpu_locked(layer);
        if (r < 0) return r;
    }
    layers_[layer].last_used = ++clock_;
    layers_[layer].last_access_ms = clock_ms();
    // fp32 q / out share the step buffers' space (the fp16 step buffers hold
    // twice the elements needed here)
    float *dq = reinterpret_cast<float *>(d_q_), *dout = reinterpret_cast<float *>(d_out_);
    memcpy(h_pos_, lens_.data(), B * sizeof(int32_t));
    int rc = KVX_OK;
    if (cudaMemcpyAsync(d_pos_, h_pos_, B * 4, cudaMemcpyHostToDevice, compute_) ||
        cudaMemcpyAsync(dq, q, qn * 4, cudaMemcpyHostToDevice, compute_) ||
        cudaMemcpyAsync(d_k_, k16.data(), kn * 2, cudaMemcpyHostToDevice, compute_) ||
        cudaMemcpyAsync(d_v_, v16.data(), kn * 2, cudaMemcpyHostToDevice, compute_))
        return KVX_ECUDA;
    kvx_paged view{arena_ + (size_t)layers_[layer].slab * slab_bytes_, nullptr, KVX_F16,
                   cfg_.pages_per_layer, hkv, 128, 16};
    rc = kvx_append_decode(&view, d_table_, max_pages_, d_pos_, B, d_k_, d_v_, hq, dq, dout, KVX_F32, 0.f,
                           d_ws_, ws_bytes_, d_err_, compute_);
    if (rc) return rc;
    int32_t err = 0;
    if (cudaMemcpyAsync(out, dout, qn * 4, cudaMemcpyDeviceToHost, compute_) ||
        cudaMemcpyAsync(&err, d_err_, 4, cudaMemcpyDeviceToHost, compute_) ||
        cudaStreamSynchronize(compute_))
        return KVX_ECUDA;
    if (err) {
        cudaMemset(d_err_, 0, 4);
        return (err & 1) ? KVX_ETIMEOUT : KVX_EINVAL;
    }
    current_layer_ = layer;
    if (layer == cfg_.layers - 1)
        for (int s = 0; s < B; ++s) ++lens_[s];
    return KVX_OK;
}

void Engine::config(adaptive_engine_config *cfg) {
    std::lock_guard<std::mutex> lk(mu_);
    if (started_ || configured_) *cfg = cfg_;
    else default_config(cfg);
}

}  // namespace kvx_engine
