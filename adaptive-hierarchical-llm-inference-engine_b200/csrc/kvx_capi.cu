// kvx_capi.cu -- library-level entry points of the C ABI (version, status
// strings, device check, stream memory wait).
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "kvx.h"

extern "C" KVX_API const char *kvx_version(void) { return "kvx 0.1 sm_100a"; }

extern "C" KVX_API const char *kvx_status_string(int status) {
    switch (status) {
    case KVX_OK: return "ok";
    case KVX_EINVAL: return "invalid argument";
    case KVX_EBUSY: return "object pinned";
    case KVX_ECUDA: return "CUDA error";
    case KVX_EUNSUPPORTED: return "unsupported geometry or dtype";
    case KVX_ETIMEOUT: return "bounded device wait expired";
    case KVX_ENOSPC: return "workspace or pool too small";
    case KVX_ENODEV: return "no sm_100 device";
    case KVX_ETOOBIG: return "request exceeds the static scratch of kvx_decode_noalloc";
    case KVX_EPEER: return "another rank's part of the multi-GPU step failed";
    default: return "unknown status";
    }
}

extern "C" KVX_API int kvx_device_check(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KVX_ENODEV;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return KVX_ENODEV;
    return major == 10 ? KVX_OK : KVX_ENODEV;
}

namespace {
// cuStreamWaitValue32 through the runtime's driver entry point (no link
// against libcuda).
using WaitValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

WaitValue32Fn wait_value_fn() {
    static WaitValue32Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<WaitValue32Fn>(f);
    });
    return fn;
}
}  // namespace

extern "C" KVX_API int kvx_stream_wait_geq(const uint32_t *word, uint32_t value, void *stream) {
    if (!word || (reinterpret_cast<uintptr_t>(word) & 3)) return KVX_EINVAL;
    WaitValue32Fn fn = wait_value_fn();
    if (!fn) return KVX_EUNSUPPORTED;
    return fn(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(word), value,
              CU_STREAM_WAIT_VALUE_GEQ) == CUDA_SUCCESS
               ? KVX_OK
               : KVX_ECUDA;
}
