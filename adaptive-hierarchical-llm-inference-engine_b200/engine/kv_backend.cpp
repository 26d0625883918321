// kv_backend.cpp -- runtime::ModelBackend over the engine's paged-attention
// layers (see include/kv_backend.h).
#include "kv_backend.h"

#include <fstream>
#include <sstream>
#include <vector>

#include "engine.h"

using kvx_engine::Engine;

bool KvAttentionBackend::load(const std::string &path) {
    Engine &e = Engine::instance();
    adaptive_engine_config cfg;
    e.default_config(&cfg);
    int batch = -1, reserve = -1;
    if (!path.empty()) {
        std::ifstream in(path);
        if (!in) return false;
        std::string line;
        while (std::getline(in, line)) {
            std::istringstream ls(line);
            std::string key, eq;
            long val = 0;
            if (!(ls >> key >> eq >> val) || eq != "=") continue;
            if (key == "layers") cfg.layers = (int)val;
            else if (key == "kv_heads") cfg.kv_heads = (int)val;
            else if (key == "q_heads") cfg.q_heads = (int)val;
            else if (key == "pages_per_layer") cfg.pages_per_layer = (int)val;
            else if (key == "max_batch") cfg.max_batch = (int)val;
            else if (key == "gpu_layer_slots") cfg.gpu_layer_slots = (int)val;
            else if (key == "batch") batch = (int)val;
            else if (key == "reserve") reserve = (int)val;
        }
        if (cfg.gpu_layer_slots > cfg.layers) cfg.gpu_layer_slots = cfg.layers;
    }
    e.stop();
    if (e.configure(cfg) != KVX_OK) return false;
    e.start();
    if (!e.started()) return false;
    if (batch <= 0) batch = cfg.max_batch;
    if (reserve < 0) reserve = cfg.pages_per_layer * 16 / batch;
    std::vector<int32_t> lens(batch, 0);
    if (e.set_sequences(batch, lens.data(), reserve, 0) != KVX_OK) return false;
    batch_ = batch;
    q_heads_ = cfg.q_heads;
    kv_heads_ = cfg.kv_heads;
    meta_.name = "kvx-paged-attention";
    meta_.format = "paged-kv";
    meta_.path = path;
    meta_.num_layers = cfg.layers;
    meta_.hidden_size = (int64_t)cfg.q_heads * 128;
    return true;
}

runtime::Tensor KvAttentionBackend::runLayer(int layer_id, const runtime::Tensor &input) {
    runtime::Tensor out;
    const size_t row = (size_t)(q_heads_ + 2 * kv_heads_) * 128;
    if (batch_ <= 0 || input.data.size() != (size_t)batch_ * row) return out;
    std::vector<float> q((size_t)batch_ * q_heads_ * 128), k((size_t)batch_ * kv_heads_ * 128),
        v((size_t)batch_ * kv_heads_ * 128);
    for (int b = 0; b < batch_; ++b) {  // split [q | k | v] per sequence
        const float *x = input.data.data() + b * row;
        std::copy(x, x + q_heads_ * 128, q.begin() + (size_t)b * q_heads_ * 128);
        std::copy(x + q_heads_ * 128, x + (q_heads_ + kv_heads_) * 128, k.begin() + (size_t)b * kv_heads_ * 128);
        std::copy(x + (q_heads_ + kv_heads_) * 128, x + row, v.begin() + (size_t)b * kv_heads_ * 128);
    }
    out.data.resize(q.size());
    if (Engine::instance().decode_layer_f32(layer_id, q.data(), k.data(), v.data(), out.data.data()) != KVX_OK) {
        out.data.clear();
        return out;
    }
    out.shape.dims = {batch_, q_heads_, 128};
    return out;
}

runtime::ModelMetadata KvAttentionBackend::metadata() const { return meta_; }
