// engine.h -- the process-wide KV-cache engine behind NativeEngineApi.
//
// Owns, per layer, one fp16 page pool ("slab", [pages][2][kv_heads][16][128])
// that lives in one of four tiers:
//   GPU         a device slab from the engine's arena
//   RAM         a slab of the pinned host arena, no device memory
//   COMPRESSED  a slab of the device compressed arena: int8 codes +
//               per-block QuantizationStats (compressKv)
//   COMPRESSED_NF4  the same arena slab holding 4-bit codes (the age
//               policy's heavy compression, compress_aged)
//   OFFLOADED   a file in the offload directory, no device or host memory
// plus the sequence state (block table, context lengths) shared by all
// layers, and the device buffers of a decode step.  Every arena is made by
// start(), so no move allocates.  All public methods take the engine mutex
// for their bookkeeping (the reference serialises its C-ABI calls with one
// mutex, native-engine/llama_wrapper/llama_wrapper.cpp:56,224), but not for
// their device work: a decode step queues its kernels and then waits for
// them with the mutex released, and a layer move queues its copies on the
// move stream behind that layer's last kernel and releases the mutex while
// they run.  A layer being moved is marked `moving`; decode steps and other
// operations on that layer wait for the mark to clear.
#pragma once

#include <cuda_runtime.h>

#include <condition_variable>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "adaptive_engine.h"

namespace kvx_engine {

enum Tier { kGpu = 0, kRam = 1, kCompressed = 2, kOffloaded = 3, kCompressedNf4 = 4 };

inline bool is_compressed(Tier t) { return t == kCompressed || t == kCompressedNf4; }

struct Layer {
    Tier tier = kGpu;
    int slab = -1;              // device slab index while on the GPU
    int host_slot = -1;         // pinned RAM arena slot while in RAM
    int i8_slot = -1;           // int8 arena slot (codes + stats) while compressed
    uint64_t last_used = 0;     // LRU stamp (KVCacheGPU lastUsedToken)
    bool cached = false;        // layer-cache bitmap of prefetch/evict/keep
    int refcount = 0;           // pins taken by keepLayer
    bool moving = false;        // a move is copying it with the engine mutex released
    cudaEvent_t last_use = nullptr;  // recorded after the last decode work on its slab
    long long last_access_ms = 0;    // engine clock of the last decode or load (the age policy)
};

class Engine {
public:
    static Engine &instance();

    void default_config(adaptive_engine_config *cfg) const;
    int step_in_flight();
    // KVCompressionEngine's age policy over the layers (see adaptive_engine.h)
    int compress_aged(long long int8_threshold_ms, long long compressed_threshold_ms, long long now_ms,
                      int apply, int32_t *decisions);
    long long layer_last_access_ms(int layer);
    long long clock_ms() const;
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
    int alloc_slab(int for_layer);  // >= 0, -1 failure, -2 every victim pinned (locked path)
    long ms_since(double t0) const;
    int to_ram_locked(int l);       // kvx_status
    int to_gpu_locked(int l);       // kvx_status (KVX_EBUSY: victims pinned)
    int offload_locked(int l);
    // arena slots
    int take_host();
    int take_i8();
    uint8_t *slab_ptr(int slab) const { return arena_ + (size_t)slab * slab_bytes_; }
    uint8_t *host_ptr(int slot) const { return ram_arena_ + (size_t)slot * slab_bytes_; }
    int8_t *codes_ptr(int slot) const { return i8_codes_ + (size_t)slot * (slab_bytes_ / 2); }
    float *stats_ptr(int slot) const { return i8_stats_ + (size_t)slot * blocks_per_slab_ * 4; }
    // moves with the mutex released during their copies (see the class comment)
    void wait_not_moving(std::unique_lock<std::mutex> &lk, int l);
    bool any_moving() const;
    int pick_victim(int for_layer) const;  // >= 0, -1 none, -2 every victim pinned
    int gpu_to_ram(std::unique_lock<std::mutex> &lk, int l);
    int bring_to_gpu(std::unique_lock<std::mutex> &lk, int l);
    int gpu_to_int8(std::unique_lock<std::mutex> &lk, int l, bool nf4 = false);
    int decompress_into(const Layer &L, uint8_t *dst, cudaStream_t st);
    // file <-> device through a pinned staging pair, no whole-layer host slab
    int file_to_device(int l, uint8_t *dst);
    int device_to_file(int l, const uint8_t *src);
    int ensure_staging();
    std::string offload_path(int l) const;
    void release_all();

    std::mutex mu_;
    std::condition_variable cv_;  // signalled when a move or a step finishes
    bool step_active_ = false;    // a step's device work may still run (mutex released)
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
    cudaStream_t move_ = nullptr;        // the NativeEngineApi moves
    uint8_t *ram_arena_ = nullptr;       // pinned host slabs, made by start()
    int8_t *i8_codes_ = nullptr;         // int8 code slabs, made by start()
    float *i8_stats_ = nullptr;          // their QuantizationStats
    std::vector<int> free_host_, free_i8_;
    double t0_ms_ = 0;  // engine clock origin (start())
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
