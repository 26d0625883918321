/* kv_backend.h -- a runtime::ModelBackend (runtime/runtime_contract.h:27-33)
 * whose layers are the engine's paged-attention layers: the KV-cache half of
 * the reference's GpuBackend (runtime/gpu_backend.h:9-35; its weight
 * loading and GEMV are not part of this engine).
 *
 *  load(path)      start the engine (the process-wide one behind
 *                  NativeEngineApi) with the geometry of a "key = value"
 *                  file (layers, kv_heads, q_heads, pages_per_layer,
 *                  max_batch, gpu_layer_slots) or the defaults when path is
 *                  empty, then open `batch` empty sequences
 *                  (key `batch`, default max_batch; key `reserve`, default
 *                  pages_per_layer*16/batch tokens each).
 *  runLayer(l, x)  x.shape = {B, q_heads + 2*kv_heads, 128}: per sequence the
 *                  layer's query heads, then the new token's K heads, then
 *                  its V heads (fp32).  Appends the token to layer l's cache
 *                  and returns paged GQA decode attention, shape
 *                  {B, q_heads, 128}.  Running the last layer advances every
 *                  sequence by one token.  Empty tensor on error.
 *  metadata()      name "kvx-paged-attention", format "paged-kv",
 *                  num_layers, hidden_size = q_heads * 128. */
#pragma once

#include <string>

#include "kvx_cxx.h"
#include "runtime_contract.h"

class KVX_CXX_API KvAttentionBackend : public runtime::ModelBackend {
public:
    bool load(const std::string &path) override;
    runtime::Tensor runLayer(int layer_id, const runtime::Tensor &input) override;
    runtime::ModelMetadata metadata() const override;

private:
    runtime::ModelMetadata meta_;
    int batch_ = 0, q_heads_ = 0, kv_heads_ = 0;
};
