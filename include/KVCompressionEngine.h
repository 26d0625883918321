/* KVCompressionEngine.h -- drop-in for the reference's
 * native-engine/include/KVCompressionEngine.h: the same enum, stats struct
 * and public member functions with the same results, bit for bit, computed
 * on the GPU (kvx_compress_int8 / kvx_compress_nf4 / kvx_fp16_wrap_encode
 * and their inverses).
 *
 * compress() and decompress() take host pointers, as the reference's do,
 * and treat the `count` elements as one block (one min/max / scale /
 * zeroPoint for the whole call), exactly as the reference computes them:
 *   INT8  native-engine/cpp/KVCompressionEngine.cpp:83-122
 *   NF4   native-engine/cpp/KVCompressionEngine.cpp:124-180 (uniform 4-bit,
 *         two codes per byte, high nibble first)
 *   FP16  native-engine/cpp/KVCompressionEngine.cpp:36-80 (exponent-wrapping
 *         conversion, not IEEE rounding)
 *   NONE  memcpy
 * For KV pages already in device memory use the block-wise C ABI in kvx.h.
 * A call without a usable sm_100 device throws std::runtime_error. */
#ifndef KV_COMPRESSION_ENGINE_H
#define KV_COMPRESSION_ENGINE_H

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

#include "kvx_cxx.h"

enum class CompressionType {
    NONE = 0,
    FP16 = 1,
    INT8 = 2,
    NF4 = 3,
};

struct QuantizationStats {
    float minVal;
    float maxVal;
    float scale;
    float zeroPoint;
    CompressionType type;
};

class KVX_CXX_API KVCompressionEngine {
public:
    KVCompressionEngine();
    ~KVCompressionEngine();
    KVCompressionEngine(const KVCompressionEngine &) = delete;
    KVCompressionEngine &operator=(const KVCompressionEngine &) = delete;

    void setCompressionType(CompressionType type);
    /* Stored as in the reference, which never consults it in compress(). */
    void enableAdaptiveCompression(float tokenAgeThreshold);

    /* Returns the compression ratio of the type (1, 0.5, 0.25, 0.125). */
    float compress(const float *input, void *output, size_t count, QuantizationStats &stats);
    void decompress(const void *input, float *output, size_t count, const QuantizationStats &stats);

    size_t getCompressedSize(CompressionType type, size_t elementCount) const;
    size_t getUncompressedSize(size_t elementCount) const { return elementCount * sizeof(float); }
    float getCompressionRatio(CompressionType type) const;
    CompressionType getStrategy() const { return strategy; }
    size_t estimateSavings(size_t uncompressedBytes, CompressionType type) const;

private:
    struct Device;
    CompressionType strategy;
    bool enableAdaptive;
    float compressionThreshold;
    std::unique_ptr<Device> dev;
};

#endif
