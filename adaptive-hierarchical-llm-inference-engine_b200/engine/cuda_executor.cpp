// cuda_executor.cpp -- runtime::gpu::cuda_softmax / cuda_attention on this
// library's kernels: host arrays are staged into device buffers on a private
// stream, the kernel runs, the result comes back (the calling convention of
// the reference's runtime/gpu/cuda_executor.cu:224-311).
#include "cuda_executor.h"

#include <cuda_runtime.h>

#include <mutex>

#include "kvx.h"

namespace runtime {
namespace gpu {
namespace {

std::mutex g_mu;
cudaStream_t g_stream = nullptr;

bool stage(size_t bytes, float **dst) {
    return cudaMallocAsync(reinterpret_cast<void **>(dst), bytes, g_stream) == cudaSuccess;
}

}  // namespace

bool cuda_available() { return kvx_device_check() == KVX_OK; }

bool cuda_init() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_stream) return true;
    if (!cuda_available()) return false;
    return cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) == cudaSuccess;
}

bool cuda_softmax(const float *logits, float *out, size_t rows, size_t cols) {
    if (!logits || !out || !cuda_init()) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    const size_t bytes = rows * cols * sizeof(float);
    float *d_in = nullptr, *d_out = nullptr;
    bool ok = stage(bytes, &d_in) && stage(bytes, &d_out) &&
              cudaMemcpyAsync(d_in, logits, bytes, cudaMemcpyHostToDevice, g_stream) == cudaSuccess &&
              kvx_softmax_rows(d_in, d_out, (int64_t)rows, (int64_t)cols, g_stream) == KVX_OK &&
              cudaMemcpyAsync(out, d_out, bytes, cudaMemcpyDeviceToHost, g_stream) == cudaSuccess;
    if (d_in) cudaFreeAsync(d_in, g_stream);
    if (d_out) cudaFreeAsync(d_out, g_stream);
    return cudaStreamSynchronize(g_stream) == cudaSuccess && ok;
}

bool cuda_attention(const float *Q, const float *K, const float *V, float *out, size_t seq_len,
                    size_t dim) {
    if (!Q || !K || !V || !out || !cuda_init()) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    const size_t bytes = seq_len * dim * sizeof(float);
    float *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
    bool ok = stage(bytes, &dq) && stage(bytes, &dk) && stage(bytes, &dv) && stage(bytes, &dout) &&
              cudaMemcpyAsync(dq, Q, bytes, cudaMemcpyHostToDevice, g_stream) == cudaSuccess &&
              cudaMemcpyAsync(dk, K, bytes, cudaMemcpyHostToDevice, g_stream) == cudaSuccess &&
              cudaMemcpyAsync(dv, V, bytes, cudaMemcpyHostToDevice, g_stream) == cudaSuccess &&
              kvx_attention_dense(dq, dk, dv, dout, (int64_t)seq_len, (int64_t)seq_len, (int32_t)dim, 0.f,
                                  g_stream) == KVX_OK &&
              cudaMemcpyAsync(out, dout, bytes, cudaMemcpyDeviceToHost, g_stream) == cudaSuccess;
    for (float *p : {dq, dk, dv, dout})
        if (p) cudaFreeAsync(p, g_stream);
    return cudaStreamSynchronize(g_stream) == cudaSuccess && ok;
}

}  // namespace gpu
}  // namespace runtime
