// kv_compression_engine.cpp -- the reference's KVCompressionEngine
// (native-engine/cpp/KVCompressionEngine.cpp) behind its own class, with
// every codec on the GPU (kvx_quant.cu).  Host pointers in and out, as in
// the reference: one device staging area per engine, grown on demand, one
// stream, each call synchronous.
#include "KVCompressionEngine.h"

#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "kvx.h"

struct KVCompressionEngine::Device {
    cudaStream_t stream = nullptr;
    void *in = nullptr, *out = nullptr;
    float *stats = nullptr;
    size_t cap_in = 0, cap_out = 0;

    ~Device() {
        if (in) cudaFree(in);
        if (out) cudaFree(out);
        if (stats) cudaFree(stats);
        if (stream) cudaStreamDestroy(stream);
    }
    static void check(cudaError_t e, const char *what) {
        if (e != cudaSuccess) throw std::runtime_error(std::string("KVCompressionEngine: ") + what + ": " + cudaGetErrorString(e));
    }
    static void check_status(int rc, const char *what) {
        if (rc != KVX_OK) throw std::runtime_error(std::string("KVCompressionEngine: ") + what + ": " + kvx_status_string(rc));
    }
    void ensure(size_t in_bytes, size_t out_bytes) {
        if (!stream) {
            check_status(kvx_device_check(), "device");
            check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
            check(cudaMalloc(&stats, 16), "stats");
        }
        if (in_bytes > cap_in) {
            if (in) cudaFree(in);
            in = nullptr;
            check(cudaMalloc(&in, in_bytes), "staging");
            cap_in = in_bytes;
        }
        if (out_bytes > cap_out) {
            if (out) cudaFree(out);
            out = nullptr;
            check(cudaMalloc(&out, out_bytes), "staging");
            cap_out = out_bytes;
        }
    }
};

KVCompressionEngine::KVCompressionEngine()
    : strategy(CompressionType::FP16), enableAdaptive(false), compressionThreshold(100.0f), dev(new Device) {}

KVCompressionEngine::~KVCompressionEngine() = default;

void KVCompressionEngine::setCompressionType(CompressionType type) { strategy = type; }

void KVCompressionEngine::enableAdaptiveCompression(float tokenAgeThreshold) {
    enableAdaptive = true;
    compressionThreshold = tokenAgeThreshold;
}

float KVCompressionEngine::compress(const float *input, void *output, size_t count, QuantizationStats &stats) {
    stats.type = strategy;
    if (strategy != CompressionType::NONE && strategy != CompressionType::FP16 &&
        strategy != CompressionType::INT8 && strategy != CompressionType::NF4)
        return 1.0f;  // reference: unknown types leave the output untouched
    const size_t out_bytes = getCompressedSize(strategy, count);
    if (strategy == CompressionType::NONE) {
        std::memcpy(output, input, count * sizeof(float));
        return 1.0f;
    }
    if (count == 0) return getCompressionRatio(strategy);
    if (count > (size_t)INT32_MAX) throw std::runtime_error("KVCompressionEngine: block too large");
    Device &d = *dev;
    d.ensure(count * sizeof(float), out_bytes + 16);
    Device::check(cudaMemcpyAsync(d.in, input, count * sizeof(float), cudaMemcpyHostToDevice, d.stream), "copy in");
    int rc = KVX_OK;
    if (strategy == CompressionType::FP16)
        rc = kvx_fp16_wrap_encode(static_cast<float *>(d.in), static_cast<uint16_t *>(d.out), count, d.stream);
    else if (strategy == CompressionType::INT8)
        rc = kvx_compress_int8(d.in, KVX_F32, static_cast<int8_t *>(d.out), d.stats, 1, (int32_t)count, d.stream);
    else
        rc = kvx_compress_nf4(d.in, KVX_F32, static_cast<uint8_t *>(d.out), d.stats, 1, (int32_t)count, d.stream);
    Device::check_status(rc, "compress");
    float st[4] = {0, 0, 0, 0};
    Device::check(cudaMemcpyAsync(output, d.out, out_bytes, cudaMemcpyDeviceToHost, d.stream), "copy out");
    if (strategy != CompressionType::FP16)
        Device::check(cudaMemcpyAsync(st, d.stats, sizeof st, cudaMemcpyDeviceToHost, d.stream), "copy stats");
    Device::check(cudaStreamSynchronize(d.stream), "compress");
    if (strategy != CompressionType::FP16) {
        stats.minVal = st[0];
        stats.maxVal = st[1];
        stats.scale = st[2];
        stats.zeroPoint = st[3];
    }
    return getCompressionRatio(strategy);
}

void KVCompressionEngine::decompress(const void *input, float *output, size_t count, const QuantizationStats &stats) {
    const CompressionType t = stats.type;
    if (t == CompressionType::NONE) {
        std::memcpy(output, input, count * sizeof(float));
        return;
    }
    if (t != CompressionType::FP16 && t != CompressionType::INT8 && t != CompressionType::NF4) return;
    if (count == 0) return;
    if (count > (size_t)INT32_MAX) throw std::runtime_error("KVCompressionEngine: block too large");
    const size_t in_bytes = getCompressedSize(t, count);
    Device &d = *dev;
    d.ensure(in_bytes + 16, count * sizeof(float));
    const float st[4] = {stats.minVal, stats.maxVal, stats.scale, stats.zeroPoint};
    Device::check(cudaMemcpyAsync(d.in, input, in_bytes, cudaMemcpyHostToDevice, d.stream), "copy in");
    Device::check(cudaMemcpyAsync(d.stats, st, sizeof st, cudaMemcpyHostToDevice, d.stream), "copy stats");
    int rc = KVX_OK;
    if (t == CompressionType::FP16)
        rc = kvx_fp16_wrap_decode(static_cast<uint16_t *>(d.in), static_cast<float *>(d.out), count, d.stream);
    else if (t == CompressionType::INT8)
        rc = kvx_decompress_int8(static_cast<int8_t *>(d.in), d.stats, d.out, KVX_F32, 1, (int32_t)count, d.stream);
    else
        rc = kvx_decompress_nf4(static_cast<uint8_t *>(d.in), d.stats, d.out, KVX_F32, 1, (int32_t)count, d.stream);
    Device::check_status(rc, "decompress");
    Device::check(cudaMemcpyAsync(output, d.out, count * sizeof(float), cudaMemcpyDeviceToHost, d.stream), "copy out");
    Device::check(cudaStreamSynchronize(d.stream), "decompress");
}

size_t KVCompressionEngine::getCompressedSize(CompressionType type, size_t elementCount) const {
    switch (type) {
    case CompressionType::NONE: return elementCount * sizeof(float);
    case CompressionType::FP16: return elementCount * sizeof(uint16_t);
    case CompressionType::INT8: return elementCount * sizeof(int8_t);
    case CompressionType::NF4: return (elementCount + 1) / 2;
    default: return elementCount * sizeof(float);
    }
}

float KVCompressionEngine::getCompressionRatio(CompressionType type) const {
    switch (type) {
    case CompressionType::NONE: return 1.0f;
    case CompressionType::FP16: return 0.5f;
    case CompressionType::INT8: return 0.25f;
    case CompressionType::NF4: return 0.125f;
    default: return 1.0f;
    }
}

size_t KVCompressionEngine::estimateSavings(size_t uncompressedBytes, CompressionType type) const {
    const size_t compressedSize = uncompressedBytes * getCompressionRatio(type);
    return uncompressedBytes - compressedSize;
}
