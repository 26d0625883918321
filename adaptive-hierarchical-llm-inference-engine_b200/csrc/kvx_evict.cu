// kvx_evict.cu -- device-side eviction bookkeeping.
//
//  * kvx_lru_select: arg-min over access stamps.  Replaces
//    LRUEvictionPolicy::selectPageToEvict
//    (native-engine/cpp/AdvancedEvictionPolicy.cpp:9-23) and
//    KVCacheGPU::findLRUPage (native-engine/cpp/KVCacheGPU.cpp:54-66): the
//    strictly smallest stamp wins, the lowest index on ties, and a stamp of
//    UINT64_MAX (the reference's initial minToken) is never chosen.
//    One CTA of 1024 threads reads the stamps with 16-byte loads; each thread
//    keeps its first minimum in index order, then a (stamp, index)
//    lexicographic tree reduction.  No workspace, deterministic.
#include "kvx_common.cuh"

namespace kvx {
namespace {

__device__ __forceinline__ void take(uint64_t &best, long long &bi, uint64_t v, long long i) {
    if (v < best || (v == best && v != UINT64_MAX && i < bi)) {
        best = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(1024)
lru_select_kernel(const uint64_t *__restrict__ stamps, size_t n, int32_t *victim) {
    uint64_t best = UINT64_MAX;
    long long bi = -1;
    const size_t pairs = n / 2;
    for (size_t i = threadIdx.x; i < pairs; i += blockDim.x) {
        const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2 *>(stamps) + i);
        take(best, bi, v.x, (long long)(2 * i));
        take(best, bi, v.y, (long long)(2 * i + 1));
    }
    if ((n & 1) && threadIdx.x == 0) take(best, bi, stamps[n - 1], (long long)(n - 1));
    // warp then block reduction on (stamp, index)
#pragma unroll
    for (int off = 16; off; off >>= 1) {
        const uint64_t ov = __shfl_xor_sync(0xffffffffu, best, off);
        const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi >= 0 && (bi < 0 || ov < best || (ov == best && oi < bi))) {
            best = ov;
            bi = oi;
        }
    }
    __shared__ uint64_t sv[32];
    __shared__ long long si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : UINT64_MAX;
        bi = lane < nw ? si[lane] : -1;
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            const uint64_t ov = __shfl_xor_sync(0xffffffffu, best, off);
            const long long oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi >= 0 && (bi < 0 || ov < best || (ov == best && oi < bi))) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) *victim = (int32_t)bi;
    }
}

}  // namespace
}  // namespace kvx

using namespace kvx;

extern "C" KVX_API int kvx_lru_select(const uint64_t *stamps, size_t n, int32_t *victim,
                                      void *stream) {
    if (!victim || (n && !stamps)) return KVX_EINVAL;
    if (n > 0x7fffffffull) return KVX_EINVAL;
    if (reinterpret_cast<uintptr_t>(stamps) & 15) return KVX_EINVAL;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n == 0) {
        return cudaMemsetAsync(victim, 0xff, sizeof(int32_t), st) == cudaSuccess ? KVX_OK : KVX_ECUDA;
    }
    lru_select_kernel<<<1, 1024, 0, st>>>(stamps, n, victim);
    return launch_status();
}
