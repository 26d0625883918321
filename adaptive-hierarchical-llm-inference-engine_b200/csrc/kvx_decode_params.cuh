// kvx_decode_params.cuh -- parameters shared by the paged decode kernels
// (SIMT path in kvx_decode.cu, tensor-core path in kvx_decode_tc.cu).
#pragma once

#include "kvx_common.cuh"

namespace kvx {

struct DecodeParams {
    const uint8_t *pool;
    const float *stats;
    const int32_t *block_table;
    const int32_t *seq_lens;
    const void *q;
    void *out;
    float *part_o;   // [batch][hq][max_splits][128]
    float *part_ml;  // [batch][hq][max_splits][2]
    int32_t *counters;  // [batch][hkv][nhg], zero between launches
    const int32_t *positions;  // fused append: token position per sequence (else null)
    const uint8_t *new_k, *new_v;  // fused append rows [batch][hkv][128]
    int32_t *error_flag;
    // attention mass (tensor-core path only; null = off): per (sequence,
    // q-head, logical page) the running max and the page's sum of
    // exp2(score - max) [batch][hq][max_pages][2]; per (sequence, q-head)
    // the final max and sum [batch][hq][2]
    float *attn_pm, *attn_ml;
    int num_pages, hkv, hq, max_pages, max_splits, chunk, group, nhg;
    float scale_log2;
};

// Tensor-core path for fp16 and int8 pools (kvx_decode_tc.cu).  Returns a
// kvx_status; KVX_EUNSUPPORTED when the geometry has no tensor-core kernel.
int launch_decode_tc(DecodeParams &p, int kv_dtype, int io_dtype, int batch, cudaStream_t st);

}  // namespace kvx
