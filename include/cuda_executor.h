/* cuda_executor.h -- drop-in for the attention / softmax part of the
 * reference's runtime/gpu/cuda_executor.h (namespace runtime::gpu): host
 * arrays in and out, device work on this library's kernels
 * (kvx_softmax_rows, kvx_attention_dense).  cuda_attention applies the
 * 1/sqrt(dim) scale of TensorOps::attention (runtime/tensor_ops.cpp:186);
 * the reference's cuBLAS version omits it (runtime/gpu/cuda_executor.cu:271-278).
 * The dense GEMM / weight-cache functions of that header are not part of
 * the KV hot path and are not provided here. */
#pragma once

#include <cstddef>

#include "kvx_cxx.h"

namespace runtime {
namespace gpu {

KVX_CXX_API bool cuda_available();
KVX_CXX_API bool cuda_init();
// rows x cols row softmax
KVX_CXX_API bool cuda_softmax(const float *logits, float *out, size_t rows, size_t cols);
// Q, K, V, out: seq_len x dim, row-major
KVX_CXX_API bool cuda_attention(const float *Q, const float *K, const float *V, float *out,
                                size_t seq_len, size_t dim);

}  // namespace gpu
}  // namespace runtime
