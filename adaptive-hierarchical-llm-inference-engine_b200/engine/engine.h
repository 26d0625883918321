// engine.h -- the process-wide KV-cache engine behind NativeEngineApi.
//
// Owns, per layer, one fp16 page pool ("slab", [pages][2][kv_heads][16][128])
// that lives in one of four tiers:
//   GPU         a device slab from the engine's arena
//   RAM         a pinned host copy (cudaHostAlloc), no device memory
//   COMPRESSED  int8 codes + per-block QuantizationStats on the device
//   OFFLOADED   a file in the offload directory, no device or host memory
// plus the sequence state (block table, context lengths) shared by all
// layers, and the device buffers of a decode step.  All public methods take
// the engine mutex (the reference serialises its C-ABI calls the same way,
// native-engine/llama_wrapper/llama_wrapper.cpp:56,224).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "adaptive_engine.h"

namespace kvx_engine {

enum Tier { kGpu = 0, kRam = 1, kCompressed = 2, kOffloaded = 3 };

struct Layer {
    Tier tier = kGpu;
    int slab = -1;              // device slab index while on the GPU
    void *host = nullptr;       // pinned fp16 copy (kept for reuse once made)
    int8_t *codes = nullptr;    // device int8 codes while compressed
    float *stats = nullptr;     // device QuantizationStats while compressed
    uint64_t last_used = 0;     // LRU stamp (KVCacheGPU lastUsedToken)
    bool cached = false;        // layer-cache bitmap of prefetch/evict/keep
    int refcount = 0;           // pins taken by keepLayer
};

class Engine {
public:
    static Engine &instance();

    void default_config(adaptive_engine_config *cfg) const;
    int configure(const adaptive_engine_config &cfg);
    void start();
    void stop();
    bool started();

    // NativeEngineApi operations (layer = kvPageId); see adaptive_engine.h
    long move_to_ram(long layer);
    long move_to_gpu(long layer);
    long compress(long layer);
    long offload(long layer);
    long prefetch_layer(int layer);
    long evict_layer(int layer);
    long keep_layer(int layer);
    void release_layer(int layer);
    int current_layer();
    long gpu_memory();
    int kv_pages();
    int cached_layers();

    int layer_view(int layer, kvx_paged *view);
    int layer_tier(int layer);
    int set_sequences(int batch, const int32_t *lens, int reserve_tokens, uint64_t seed);
    int decode_step(const uint16_t *q, const uint16_t *k, const uint16_t *v, uint16_t *out);
    // One layer of a step with fp32 host data: q [B][q_heads][128], new
    // K/V [B][kv_heads][128] (rounded to the pool's fp16), out fp32.  The
    // last layer advances the sequences.
    int decode_layer_f32(int layer, const float *q, const float *k, const float *v, float *out);
    void config(adaptive_engine_config *cfg);
    int32_t seq_len(int s);
    int copy_layer(int layer, void *ptr, bool load);
    int set_comm(int rank, int world, const void *id128);
    int set_readback_share(int share);
    int32_t block_table(int32_t *dst);
    long long device_bytes();

private:
    Engine() = default;
    ~Engine();
    bool valid(long layer) const;
    // helpers below expect the mutex held
    int alloc_slab(int for_layer);  // >= 0, -1 failure, -2 every victim pinned
    long ms_since(double t0) const;
    int to_ram_locked(int l);       // kvx_status
    int to_gpu_locked(int l);       // kvx_status (KVX_EBUSY: victims pinned)
    int compress_locked(int l);
    int offload_locked(int l);
    int ensure_host(int l);
    // file <-> device through a pinned staging pair, no whole-layer host slab
    int file_to_device(int l, uint8_t *dst);
    int device_to_file(int l, const uint8_t *src);
    int ensure_staging();
    std::string offload_path(int l) const;
    void release_all();

    std::mutex mu_;
    adaptive_engine_config cfg_{};
    bool configured_ = false;
    bool started_ = false;
    size_t slab_bytes_ = 0;
    size_t blocks_per_slab_ = 0;
    uint8_t *arena_ = nullptr;
    std::vector<int> free_slabs_;
    std::vector<Layer> layers_;
    uint64_t clock_ = 0;
    int current_layer_ = 0;
    cudaStream_t compute_ = nullptr, copy_ = nullptr;
    std::vector<cudaEvent_t> ev_in_, ev_out_;

    // sequences
    int batch_ = 0, max_pages_ = 0;
    std::vector<int32_t> lens_;         // host mirror of context lengths
    std::vector<int32_t> table_;        // host mirror [max_batch][max_pages]
    std::vector<int32_t> free_pages_;   // physical pages not owned by a sequence
    int32_t *d_table_ = nullptr, *d_pos_ = nullptr, *d_err_ = nullptr;
    int32_t *h_pos_ = nullptr;          // pinned positions for the step
    static constexpr size_t kStageBytes = size_t(64) << 20;
    uint8_t *stage_[2] = {nullptr, nullptr};  // pinned staging for file moves
    cudaEvent_t stage_ev_[2] = {nullptr, nullptr};
    int32_t *d_status_ = nullptr;       // {host status, error flag} then every rank's pair
    int32_t *h_status_ = nullptr;       // pinned mirror of d_status_
    void *d_ws_ = nullptr;
    size_t ws_bytes_ = 0;
    uint16_t *d_q_ = nullptr, *d_k_ = nullptr, *d_v_ = nullptr, *d_out_ = nullptr;
    long long device_bytes_ = 0;
    // NCCL all-gather of the attention outputs (multi-GPU)
    void *comm_ = nullptr;  // ncclComm_t
    int world_ = 1, rank_ = 0;
    cudaStream_t comm_stream_ = nullptr;
    uint16_t *d_gather_ = nullptr;
    bool readback_share_ = false;  // each rank reads back layers l % world == rank only
    std::vector<cudaEvent_t> ev_gath_;
};

// NCCL entry points, resolved at run time.
int nccl_unique_id(void *id128);

}  // namespace kvx_engine
