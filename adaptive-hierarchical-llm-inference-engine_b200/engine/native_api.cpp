// native_api.cpp -- the C ABI of include/adaptive_engine.h: the reference's
// NativeEngineApi table (native-engine/llama_wrapper/llama_wrapper.cpp:26-40,
// 465-479, 742-744) and the additive engine entry points, all forwarding to
// the process-wide kvx_engine::Engine.  Nothing here throws across the ABI.
#include "adaptive_engine.h"
#include "engine.h"

using kvx_engine::Engine;

namespace {

void api_start() { Engine::instance().start(); }
void api_stop() { Engine::instance().stop(); }
long api_prefetch_layer(int l) { return Engine::instance().prefetch_layer(l); }
long api_evict_layer(int l) { return Engine::instance().evict_layer(l); }
long api_keep_layer(int l) { return Engine::instance().keep_layer(l); }
long api_move_kv_to_ram(long id) { return Engine::instance().move_to_ram(id); }
long api_move_kv_to_gpu(long id) { return Engine::instance().move_to_gpu(id); }
long api_compress_kv(long id) { return Engine::instance().compress(id); }
long api_offload_kv(long id) { return Engine::instance().offload(id); }
int api_current_layer() { return Engine::instance().current_layer(); }
long api_gpu_memory() { return Engine::instance().gpu_memory(); }
int api_kv_pages() { return Engine::instance().kv_pages(); }
int api_cached_layers() { return Engine::instance().cached_layers(); }

NativeEngineApi g_api = {&api_start,           &api_stop,           &api_prefetch_layer,
                         &api_evict_layer,     &api_keep_layer,     &api_move_kv_to_ram,
                         &api_move_kv_to_gpu,  &api_compress_kv,    &api_offload_kv,
                         &api_current_layer,   &api_gpu_memory,     &api_kv_pages,
                         &api_cached_layers};

}  // namespace

extern "C" {

ADAPTIVE_ENGINE_EXPORT NativeEngineApi *adaptive_engine_get_api(void) { return &g_api; }

ADAPTIVE_ENGINE_EXPORT void adaptive_engine_test_release_layer(int layerId) {
    Engine::instance().release_layer(layerId);
}

ADAPTIVE_ENGINE_EXPORT void adaptive_engine_default_config(adaptive_engine_config *cfg) {
    if (cfg) Engine::instance().default_config(cfg);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_configure(const adaptive_engine_config *cfg) {
    return cfg ? Engine::instance().configure(*cfg) : KVX_EINVAL;
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_layer_view(int layer, kvx_paged *view) {
    return Engine::instance().layer_view(layer, view);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_set_sequences(int32_t batch, const int32_t *lens,
                                                         int32_t reserve_tokens, uint64_t seed) {
    return Engine::instance().set_sequences(batch, lens, reserve_tokens, seed);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_decode_step(const uint16_t *q, const uint16_t *k,
                                                       const uint16_t *v, uint16_t *out) {
    return Engine::instance().decode_step(q, k, v, out);
}

ADAPTIVE_ENGINE_EXPORT int32_t adaptive_engine_seq_len(int32_t s) { return Engine::instance().seq_len(s); }

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_load_layer(int layer, const void *src) {
    return Engine::instance().copy_layer(layer, const_cast<void *>(src), true);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_read_layer(int layer, void *dst) {
    return Engine::instance().copy_layer(layer, dst, false);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_nccl_unique_id(void *id128) {
    return id128 ? kvx_engine::nccl_unique_id(id128) : KVX_EINVAL;
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_set_comm(int rank, int world, const void *id128) {
    return Engine::instance().set_comm(rank, world, id128);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_step_in_flight(void) { return Engine::instance().step_in_flight(); }

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_compress_aged(int64_t int8_threshold_ms, int64_t compressed_threshold_ms,
                                                        int64_t now_ms, int32_t apply, int32_t *decisions) {
    return Engine::instance().compress_aged(int8_threshold_ms, compressed_threshold_ms, now_ms, apply, decisions);
}

ADAPTIVE_ENGINE_EXPORT int64_t adaptive_engine_layer_last_access_ms(int layer) {
    return Engine::instance().layer_last_access_ms(layer);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_set_readback_share(int share) {
    return Engine::instance().set_readback_share(share);
}

ADAPTIVE_ENGINE_EXPORT int32_t adaptive_engine_block_table(int32_t *dst) {
    return Engine::instance().block_table(dst);
}

ADAPTIVE_ENGINE_EXPORT int adaptive_engine_layer_tier(int layer) {
    return Engine::instance().layer_tier(layer);
}

ADAPTIVE_ENGINE_EXPORT long long adaptive_engine_device_bytes(void) {
    return Engine::instance().device_bytes();
}

}  // extern "C"
