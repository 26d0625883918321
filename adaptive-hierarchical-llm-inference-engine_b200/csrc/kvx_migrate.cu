// kvx_migrate.cu -- page-frame moves between the device pool and a pinned,
// mapped host arena (the RAM tier), the data path of moveKvToRam /
// moveKvToGpu and of eviction.
//
// Replaces KVCacheGPU::transferToHost / transferToGPU
// (native-engine/cpp/KVCacheGPU.cpp:68-120), which issued one synchronous
// cudaMemcpy per page.  Here a gather/scatter kernel moves any list of
// frames in one launch on a side stream: each CTA streams whole frames with
// 16-byte vectors (coalesced on both sides), and the grid is capped by the
// caller so the copy occupies a few SMs while decode keeps the rest.
#include "kvx_common.cuh"

namespace kvx {
namespace {

__global__ void __launch_bounds__(512)
migrate_kernel(uint8_t *dev_base, int dev_cap, uint8_t *host_base, int host_cap,
               const int32_t *__restrict__ dev_frames, const int32_t *__restrict__ host_frames,
               int num_frames, size_t frame_vecs, int to_device, int32_t *error_flag,
               const int32_t *__restrict__ num_frames_dev) {
    if (num_frames_dev) num_frames = min(num_frames, *num_frames_dev);  // a count written on the device
    for (int f = blockIdx.x; f < num_frames; f += gridDim.x) {
        const int32_t dfi = dev_frames[f], hfi = host_frames[f];
        if (dfi < 0 || dfi >= dev_cap || hfi < 0 || hfi >= host_cap) {
            if (error_flag && threadIdx.x == 0) atomicOr(error_flag, 2);
            continue;
        }
        const size_t df = (size_t)dfi, hf = (size_t)hfi;
        uint4 *d = reinterpret_cast<uint4 *>(dev_base) + df * frame_vecs;
        uint4 *h = reinterpret_cast<uint4 *>(host_base) + hf * frame_vecs;
        if (to_device) {
            // host reads cross the link: keep 4 loads in flight per thread
            size_t i = threadIdx.x;
            for (; i + 3 * blockDim.x < frame_vecs; i += 4 * blockDim.x) {
                uint4 a = __ldcv(h + i), b = __ldcv(h + i + blockDim.x),
                      c = __ldcv(h + i + 2 * blockDim.x), e = __ldcv(h + i + 3 * blockDim.x);
                d[i] = a;
                d[i + blockDim.x] = b;
                d[i + 2 * blockDim.x] = c;
                d[i + 3 * blockDim.x] = e;
            }
            for (; i < frame_vecs; i += blockDim.x) d[i] = __ldcv(h + i);
        } else {
            for (size_t i = threadIdx.x; i < frame_vecs; i += blockDim.x) __stcs(h + i, __ldcs(d + i));
        }
    }
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API int kvx_migrate_frames(void *dev_base, int32_t dev_capacity, void *host_base,
                                          int32_t host_capacity, const int32_t *dev_frames,
                                          const int32_t *host_frames, int32_t num_frames,
                                          size_t frame_bytes, int32_t direction, int32_t ctas,
                                          int32_t *error_flag, void *stream) {
    if (!dev_base || !host_base || !dev_frames || !host_frames || num_frames < 0) return KVX_EINVAL;
    if (dev_capacity <= 0 || host_capacity <= 0) return KVX_EINVAL;
    if (frame_bytes == 0 || frame_bytes % 16 || (direction != 0 && direction != 1)) return KVX_EINVAL;
    if ((reinterpret_cast<uintptr_t>(dev_base) | reinterpret_cast<uintptr_t>(host_base)) & 15)
        return KVX_EINVAL;
    if (num_frames == 0) return KVX_OK;
    int grid = ctas > 0 ? ctas : 16;
    if (grid > num_frames) grid = num_frames;
    migrate_kernel<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t *>(dev_base), dev_capacity, static_cast<uint8_t *>(host_base),
        host_capacity, dev_frames, host_frames, num_frames, frame_bytes / 16, direction, error_flag, nullptr);
    return launch_status();
}

#include "kvx_tier_policy.h"

int kvx_tier_dev::migrate_counted(void *dev_base, int32_t dev_capacity, void *host_base, int32_t host_capacity,
                                  const int32_t *dev_frames, const int32_t *host_frames, const int32_t *count_dev,
                                  int32_t max_frames, size_t frame_bytes, int32_t direction, int32_t ctas,
                                  int32_t *error_flag, cudaStream_t st) {
    if (!dev_base || !host_base || !dev_frames || !host_frames || !count_dev || max_frames < 0) return KVX_EINVAL;
    if (frame_bytes == 0 || frame_bytes % 16 || (direction != 0 && direction != 1)) return KVX_EINVAL;
    if (max_frames == 0) return KVX_OK;
    int grid = ctas > 0 ? ctas : 16;
    if (grid > max_frames) grid = max_frames;
    migrate_kernel<<<grid, 512, 0, st>>>(static_cast<uint8_t *>(dev_base), dev_capacity,
                                         static_cast<uint8_t *>(host_base), host_capacity, dev_frames, host_frames,
                                         max_frames, frame_bytes / 16, direction, error_flag, count_dev);
    return launch_status();
}
