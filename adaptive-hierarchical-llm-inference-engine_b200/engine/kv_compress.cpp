// kv_compress.cpp -- the disk tier's truncating fp16 codec
// (compression/kv_compress.cpp:6-60) on the GPU, behind the reference's two
// vector functions.
#include "kv_compress.h"

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "kvx.h"

namespace {

template <typename In, typename Out, typename Fn>
std::vector<Out> run_codec(const std::vector<In> &in, Fn kernel, const char *what) {
    std::vector<Out> out(in.size());
    if (in.empty()) return out;
    if (kvx_device_check() != KVX_OK) throw std::runtime_error(std::string(what) + ": no sm_100 device");
    In *d_in = nullptr;
    Out *d_out = nullptr;
    cudaStream_t st = nullptr;
    bool ok = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
              cudaMallocAsync(&d_in, in.size() * sizeof(In), st) == cudaSuccess &&
              cudaMallocAsync(&d_out, in.size() * sizeof(Out), st) == cudaSuccess &&
              cudaMemcpyAsync(d_in, in.data(), in.size() * sizeof(In), cudaMemcpyHostToDevice, st) == cudaSuccess &&
              kernel(d_in, d_out, in.size(), st) == KVX_OK &&
              cudaMemcpyAsync(out.data(), d_out, in.size() * sizeof(Out), cudaMemcpyDeviceToHost, st) == cudaSuccess;
    if (d_in) cudaFreeAsync(d_in, st);
    if (d_out) cudaFreeAsync(d_out, st);
    ok = st && cudaStreamSynchronize(st) == cudaSuccess && ok;
    if (st) cudaStreamDestroy(st);
    if (!ok) throw std::runtime_error(std::string(what) + ": CUDA failure");
    return out;
}

}  // namespace

std::vector<uint16_t> float32_to_float16(const std::vector<float> &in) {
    return run_codec<float, uint16_t>(
        in, [](const float *a, uint16_t *b, size_t n, cudaStream_t s) { return kvx_f32_to_f16_trunc(a, b, n, s); },
        "float32_to_float16");
}

std::vector<float> float16_to_float32(const std::vector<uint16_t> &in) {
    return run_codec<uint16_t, float>(
        in, [](const uint16_t *a, float *b, size_t n, cudaStream_t s) { return kvx_f16_trunc_to_f32(a, b, n, s); },
        "float16_to_float32");
}
