// kvx_common.cuh -- shared device helpers of the sm_100a KV-cache kernels:
// status plumbing, bulk-copy (TMA engine) + mbarrier primitives with bounded
// waits, and element conversions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "kvx.h"

namespace kvx {

constexpr int kHeadDim = 128;
constexpr int kPageTokens = 16;

// Upper bound on mbarrier polls before a wait gives up and reports
// KVX_ETIMEOUT through the error flag.  One try_wait suspends for a bounded
// hardware interval, so this is far above any real copy latency.
constexpr uint32_t kWaitPolls = 1u << 22;

inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? KVX_OK : KVX_ECUDA;
}

// Device ordinals with a cached per-device flag; a higher ordinal sets the
// attribute on every launch.
constexpr int kMaxDevices = 64;

// Raise a kernel's dynamic shared-memory limit on the current device.  The
// attribute belongs to the (kernel, device) pair, so a process decoding on
// several GPUs needs it once per device: `done` is the calling launcher's own
// per-device flag array (a static of that kernel instantiation).  Threads
// racing on the first call both set it, which is harmless.
template <typename Kernel>
inline int ensure_smem_attr(std::atomic<bool> (&done)[kMaxDevices], Kernel kern, int smem) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KVX_ECUDA;
    const bool cached = dev >= 0 && dev < kMaxDevices;
    if (cached && done[dev].load(std::memory_order_acquire)) return KVX_OK;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return KVX_ECUDA;
    if (cached) done[dev].store(true, std::memory_order_release);
    return KVX_OK;
}

// SM count of the current device, looked up once per device.
inline int sm_count() {
    static std::atomic<int> cache[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    const bool cached = dev >= 0 && dev < kMaxDevices;
    int n = cached ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        if (cached) cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's generic-proxy shared memory accesses before later
// async-proxy (bulk copy) writes to the same buffers.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// One arrival on `bar` (release: this thread's earlier shared-memory reads
// and writes are ordered before whoever waits on the phase it completes).
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bulk global -> shared copy completing on `bar` (bytes % 16 == 0, both
// addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_addr(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Bulk shared -> global copy (TMA, no tensor map): both addresses 16-byte
// aligned, bytes a multiple of 16.  Completion through bulk groups.
__device__ __forceinline__ void bulk_s2g(void *dst_global, const void *src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_global),
                 "r"(smem_addr(src_smem)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the source shared memory of every committed group may be reused
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every committed group is complete (its global writes done)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and sets bit 0
// of *error_flag when given) if the barrier did not complete in kWaitPolls
// polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  int32_t *error_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (error_flag) atomicOr(error_flag, 1);
    return false;
}

// Arrival ticket with release + acquire semantics at GPU scope: the
// caller's (and, through a preceding warp/CTA barrier, its peers') prior
// writes are visible to whoever later acquires this counter, and the
// caller sees everything released to it before.  Cheaper than a
// sequentially consistent fence (__threadfence).
__device__ __forceinline__ int atomic_add_acq_rel(int *p, int v) {
    int r;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(r) : "l"(p), "r"(v) : "memory");
    return r;
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
}

template <typename T> struct io_traits;
template <> struct io_traits<float> {
    __device__ static float load(const float *p) { return *p; }
    __device__ static void store(float *p, float v) { *p = v; }
};
template <> struct io_traits<__half> {
    __device__ static float load(const __half *p) { return __half2float(*p); }
    __device__ static void store(__half *p, float v) { *p = __float2half_rn(v); }
};

}  // namespace kvx
